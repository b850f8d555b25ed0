"""GPU test of vtx_flash_attn_decode_batched_noalloc, the batched-decode entry
point for callers that cannot allocate device memory (a plugin inside a host
application that owns all device allocations, a process under a hard memory
budget or custom allocator, a real-time loop that must not block in
cudaMalloc).  It keeps its split-KV partials in a buffer compiled into the
library instead of a caller workspace.

Called through the C ABI, its output must match the workspace entry point
(vtx_flash_attn_decode_batched) within the parity tolerance, on two calls in a
row with different inputs (the shared buffer keeps the previous call's
contents).  This file is named so pytest collects it last; it also runs alone
in a fresh process.
"""
import ctypes

import numpy as np
import pytest

from vtx_cases import ATOL, RTOL

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _batch(seed, n_seq=24, Hq=32, Hkv=8, D=128, max_len=2500):
    import vtx_attn
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    rng = np.random.default_rng(seed)
    lens = rng.integers(1, max_len, n_seq).astype(np.int32)
    ks = [torch.randn((int(L), Hkv, D), generator=g, device="cuda").half() for L in lens]
    vs = [torch.randn((int(L), Hkv, D), generator=g, device="cuda").half() for L in lens]
    plan = vtx_attn.DecodeBatchPlan(ks, vs, torch.from_numpy(lens).cuda(), Hq, Hkv, D, vtx_attn.F16,
                                    Hkv * D * 2, D * 2, int(lens.max()), D ** -0.5)
    q = torch.randn((n_seq, Hq, D), generator=g, device="cuda")
    return plan, q


def test_noalloc_matches_workspace_entry_point_twice():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import vtx_attn
    L = vtx_attn.load()
    L.vtx_flash_attn_decode_batched_noalloc.argtypes = [ctypes.POINTER(vtx_attn.DecodeBatch), ctypes.c_void_p]
    L.vtx_flash_attn_decode_batched_noalloc.restype = ctypes.c_int
    stream = torch.cuda.current_stream()
    for call, seed in enumerate((101, 202)):
        plan, q = _batch(seed)
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
    L = vtx_attn.load()
    L.vtx_flash_attn_decode_batched_noalloc.argtypes = [ctypes.POINTER(vtx_attn.DecodeBatch), ctypes.c_void_p]
    L.vtx_flash_attn_decode_batched_noalloc.restype = ctypes.c_int
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
