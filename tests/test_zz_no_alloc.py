"""GPU test of vtx_flash_attn_decode_batched_noalloc, the batched-decode entry
point for callers that cannot allocate device memory (a plugin inside a host
application that owns all device allocations, a process under a hard memory
budget or custom allocator, a real-time loop that must not block in
cudaMalloc).  It keeps its split-KV partials in a buffer compiled into the
library instead of a caller workspace.

Called through the C ABI, its output must match the workspace entry point
(vtx_flash_attn_decode_batched) within the parity tolerance, on two calls in a
row with different inputs (the shared buffer keeps the previous call's
contents), for every decode kernel the call can reach: the F16 streaming
kernel (head_dim 64 and 128), the Q8_0 streaming kernel (head_dim 128), and
the generic split-KV kernel (F32 caches, Q8_0 with head_dim 64).  This file
is named so pytest collects it last; test_noalloc_in_fresh_process re-runs it
alone in a new process, where the first call on the device also performs the
one-time address lookup of the built-in buffer.
"""
import ctypes
import os
import subprocess
import sys

import numpy as np
import pytest

import oracle as O
from vtx_cases import ATOL, RTOL

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

CASES = [("f16", 128), ("f16", 64), ("q8_0", 128), ("q8_0", 64), ("f32", 128), ("f32", 64)]


def _lib():
    import vtx_attn
    L = vtx_attn.load()
    L.vtx_flash_attn_decode_batched_noalloc.argtypes = [ctypes.POINTER(vtx_attn.DecodeBatch), ctypes.c_void_p]
    L.vtx_flash_attn_decode_batched_noalloc.restype = ctypes.c_int
    return L


def _cache(rng, n, Hkv, D, kv):
    x = rng.standard_normal((int(n), Hkv, D)).astype(np.float32)
    if kv == "f16":
        return torch.from_numpy(x.astype(np.float16)).cuda()
    if kv == "f32":
        return torch.from_numpy(x).cuda()
    return torch.from_numpy(O.quantize_q8_0(x)).cuda()          # (n, Hkv, D/32*34) bytes


def _batch(seed, kv, D, n_seq=12, Hq=32, Hkv=8, max_len=2500):
    import vtx_attn
    rng = np.random.default_rng(seed)
    lens = rng.integers(1, max_len, n_seq).astype(np.int32)
    ks = [_cache(rng, L, Hkv, D, kv) for L in lens]
    vs = [_cache(rng, L, Hkv, D, kv) for L in lens]
    kvt = {"f16": vtx_attn.F16, "f32": vtx_attn.F32, "q8_0": vtx_attn.Q8_0}[kv]
    row = {"f16": D * 2, "f32": D * 4, "q8_0": D // 32 * 34}[kv]     # one head's K (or V) row in bytes
    plan = vtx_attn.DecodeBatchPlan(ks, vs, torch.from_numpy(lens).cuda(), Hq, Hkv, D, kvt, Hkv * row, row,
                                    int(lens.max()), D ** -0.5)
    q = torch.from_numpy(rng.standard_normal((n_seq, Hq, D)).astype(np.float32)).cuda()
    return plan, q


@pytest.mark.parametrize("kv,D", CASES, ids=[f"{k}-d{d}" for k, d in CASES])
def test_noalloc_matches_workspace_entry_point_twice(kv, D):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import vtx_attn
    L = _lib()
    stream = torch.cuda.current_stream()
    for call, seed in enumerate((101, 202)):
        plan, q = _batch(seed + D, kv, D)
        assert 0 < plan.need <= (32 << 20), "test batch must use split-KV partials within the built-in buffer"
        ref = plan(q)                                    # workspace entry point
        got = torch.full_like(q, float("nan"))
        plan.batch.q = q.data_ptr()
        plan.batch.dst = got.data_ptr()
        rc = L.vtx_flash_attn_decode_batched_noalloc(ctypes.byref(plan.batch), ctypes.c_void_p(stream.cuda_stream))
        assert rc == 0, L.vtx_strerror(rc)
        torch.cuda.synchronize()
        r, o = ref.cpu().numpy(), got.cpu().numpy()
        assert np.all(np.isfinite(o)), f"call {call}: non-finite output"
        assert np.all(np.abs(o - r) <= ATOL + RTOL * np.abs(r)), f"call {call}: max err {np.abs(o - r).max()}"
    assert vtx_attn.read_device_error() == 0


def test_noalloc_rejects_problems_beyond_its_buffer():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import vtx_attn
    L = _lib()
    # 64 streams of up to 200k keys: partials far beyond 32 MiB.  The call is
    # rejected before anything is launched, so small placeholder buffers do.
    n_seq, Hq, Hkv, D = 64, 32, 8, 128
    buf = torch.zeros(1 << 16, dtype=torch.float32, device="cuda")
    ptrs = torch.full((n_seq,), buf.data_ptr(), dtype=torch.int64, device="cuda")
    lens = torch.ones(n_seq, dtype=torch.int32, device="cuda")
    b = vtx_attn.DecodeBatch()
    b.n_seq, b.n_head_q, b.n_head_kv, b.head_dim = n_seq, Hq, Hkv, D
    b.kv_type, b.max_kv_len, b.kv_nb1, b.kv_nb2 = vtx_attn.F16, 200000, Hkv * D * 2, D * 2
    b.q, b.k_ptrs, b.v_ptrs = buf.data_ptr(), ptrs.data_ptr(), ptrs.data_ptr()
    b.kv_len, b.dst, b.scale = lens.data_ptr(), buf.data_ptr(), D ** -0.5
    assert L.vtx_flash_attn_decode_batched_workspace(ctypes.byref(b)) > (32 << 20)
    rc = L.vtx_flash_attn_decode_batched_noalloc(ctypes.byref(b), None)
    assert rc == -9
    assert b"no-alloc" in L.vtx_strerror(rc)


def test_noalloc_in_fresh_process():
    """The tests above, alone in a new process: there the no-alloc call is the
    first use of the built-in buffer on the device."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    if os.environ.get("VTX_NOALLOC_CHILD"):
        pytest.skip("already the fresh process")
    env = dict(os.environ, VTX_NOALLOC_CHILD="1")
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-x", "-m", "gpu", os.path.abspath(__file__)],
                       cwd=os.path.dirname(os.path.dirname(os.path.abspath(__file__))), env=env,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
