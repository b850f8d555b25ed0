"""Decoder KV-cache update (vtx_kv_append): RoPE of Q and K (ggml mode 0) and
the K/V cache write into F32 / F16 / Q8_0 cache rows chosen by ring slots.

CPU tests pin the oracle (oracle/vtx_ref.c vtx_ref_kv_append) against an
independent float64 rotation written here with numpy; GPU tests compare the
CUDA kernel with the oracle on the same seeded inputs and run the whole decode
step (append, then attention over the cache) against the oracle pipeline."""
import numpy as np
import pytest

import oracle as O
from vtx_cases import assert_close, f16_ulp_close as _f16_ulp_close, q8_close as _q8_close

BASE = 1e6           # voxtral's dec_rope_theta (include/voxtral.h:41)


def rope_f64(x: np.ndarray, pos: np.ndarray, base: float = BASE) -> np.ndarray:
    """x: (T, H, D); adjacent pairs rotated by pos * base^(-2i/D), float64."""
    T, H, D = x.shape
    i = np.arange(D // 2)
    th = pos.astype(np.float64)[:, None] * base ** (-2.0 * i / D)[None, :]      # (T, D/2)
    c, s = np.cos(th)[:, None, :], np.sin(th)[:, None, :]
    x = x.astype(np.float64)
    y = np.empty_like(x)
    y[..., 0::2] = x[..., 0::2] * c - x[..., 1::2] * s
    y[..., 1::2] = x[..., 0::2] * s + x[..., 1::2] * c
    return y


def make_inputs(seed, T=6, Hq=8, Hkv=2, D=128, max_pos=9000):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((T, Hq, D)).astype(np.float32)
    k = rng.standard_normal((T, Hkv, D)).astype(np.float32)
    v = rng.standard_normal((T, Hkv, D)).astype(np.float32)
    pos = np.concatenate([[0], rng.integers(1, max_pos, T - 1)]).astype(np.int32)
    return q, k, v, pos


def empty_cache(rows, Hkv, D, kv_type):
    return np.zeros((rows, Hkv * O.cache_head_bytes(kv_type, D)), np.uint8)


# ---- oracle on the CPU ---------------------------------------------------------

def test_oracle_fp64_mode_matches_numpy_rotation():
    q, k, v, pos = make_inputs(1)
    slots = np.arange(len(pos))
    kc, vc = empty_cache(len(pos), 2, 128, O.F32), empty_cache(len(pos), 2, 128, O.F32)
    qo = O.kv_append(q, k, v, pos, slots, O.F32, BASE, kc, vc, mode=O.MODE_FP64)
    np.testing.assert_allclose(qo, rope_f64(q, pos), rtol=0, atol=2e-6)
    np.testing.assert_allclose(kc.view(np.float32).reshape(k.shape), rope_f64(k, pos), rtol=0, atol=2e-6)
    assert np.array_equal(vc.view(np.float32).reshape(v.shape), v)       # V is copied, not rotated


def test_oracle_ggml_mode_is_the_float_angle_recurrence():
    """ggml mode rotates by the float recurrence theta *= powf(base, -2/D): equal
    to the exact rotation at position 0 and within the recurrence's drift
    (relative angle error ~ i * 2^-24 per pair) elsewhere."""
    q, k, v, pos = make_inputs(2)
    slots = np.arange(len(pos))
    kc, vc = empty_cache(len(pos), 2, 128, O.F32), empty_cache(len(pos), 2, 128, O.F32)
    qo = O.kv_append(q, k, v, pos, slots, O.F32, BASE, kc, vc)
    assert np.array_equal(qo[0], q[0])                                   # theta = 0 for every pair
    ref = rope_f64(q, pos)
    bound = 64 * 2.0 ** -24 * pos.max() * np.abs(q).max() * 4 + 1e-5
    assert np.abs(qo - ref).max() < bound
    # the recurrence, restated here in float32 with numpy, gives the same angles
    ts = np.float32(np.power(np.float32(BASE), np.float32(-2.0 / 128)))
    th = np.empty((len(pos), 64), np.float32)
    th[:, 0] = pos.astype(np.float32)
    for i in range(1, 64):
        th[:, i] = th[:, i - 1] * ts
    c, s = np.cos(th.astype(np.float64)), np.sin(th.astype(np.float64))
    y = np.empty_like(ref)
    y[..., 0::2] = q[..., 0::2] * c[:, None] - q[..., 1::2] * s[:, None]
    y[..., 1::2] = q[..., 0::2] * s[:, None] + q[..., 1::2] * c[:, None]
    assert np.abs(qo - y).max() < 2e-5


@pytest.mark.parametrize("kv_type", [O.F16, O.Q8_0])
def test_oracle_cache_formats(kv_type):
    q, k, v, pos = make_inputs(3)
    slots = np.array([5, 0, 3, 1, 7, 2])
    kc, vc = empty_cache(8, 2, 128, kv_type), empty_cache(8, 2, 128, kv_type)
    kf, vf = empty_cache(8, 2, 128, O.F32), empty_cache(8, 2, 128, O.F32)
    O.kv_append(None, k, v, pos, slots, kv_type, BASE, kc, vc)
    O.kv_append(None, k, v, pos, slots, O.F32, BASE, kf, vf)
    kr = kf.view(np.float32).reshape(8, 2, 128)[slots]
    vr = vf.view(np.float32).reshape(8, 2, 128)[slots]
    if kv_type == O.F16:
        assert np.array_equal(kc.view(np.float16).reshape(8, 2, 128)[slots], kr.astype(np.float16))
        assert np.array_equal(vc.view(np.float16).reshape(8, 2, 128)[slots], vr.astype(np.float16))
    else:
        import ctypes
        exp = np.empty((len(slots), 2 * 4 * 34), np.uint8)
        O.lib().vtx_ref_quantize_q8_0_rne(np.ascontiguousarray(kr).ctypes.data, exp.ctypes.data, kr.size)
        assert np.array_equal(kc[slots], exp)
    untouched = np.setdiff1d(np.arange(8), slots)
    assert not kc[untouched].any() and not vc[untouched].any()


# ---- CUDA kernel -----------------------------------------------------------------

def _gpu_append(q, k, v, pos, slots, kv_type, rows, **kw):
    import torch
    import vtx_attn
    dev = "cuda"
    T, Hkv, D = k.shape
    kc = torch.zeros((rows, Hkv * O.cache_head_bytes(kv_type, D)), dtype=torch.uint8, device=dev)
    vc = torch.zeros_like(kc)
    qo = vtx_attn.kv_append(torch.from_numpy(k).to(dev), torch.from_numpy(v).to(dev),
                            torch.from_numpy(pos).to(dev), torch.from_numpy(np.asarray(slots, np.int32)).to(dev),
                            kc, vc, kv_type, BASE, q=None if q is None else torch.from_numpy(q).to(dev), **kw)
    torch.cuda.synchronize()
    return (None if qo is None else qo.cpu().numpy()), kc.cpu().numpy(), vc.cpu().numpy()


@pytest.mark.gpu
@pytest.mark.parametrize("kv_type", [O.F32, O.F16, O.Q8_0])
@pytest.mark.parametrize("D", [128, 64])
def test_gpu_kv_append_matches_oracle(kv_type, D):
    q, k, v, pos = make_inputs(10 + D + kv_type, T=37, Hq=32 if D == 128 else 20,
                               Hkv=8 if D == 128 else 20, D=D)
    rows = 64
    slots = np.random.default_rng(5).permutation(rows)[:len(pos)].astype(np.int32)
    qo, kc, vc = _gpu_append(q, k, v, pos, slots, kv_type, rows)
    Hkv = k.shape[1]
    kr, vr = empty_cache(rows, Hkv, D, kv_type), empty_cache(rows, Hkv, D, kv_type)
    qr = O.kv_append(q, k, v, pos, slots, kv_type, BASE, kr, vr)
    assert_close(qo, qr, "roped Q", atol=2e-6, rtol=2e-6)
    if kv_type == O.F32:
        assert_close(kc.view(np.float32), kr.view(np.float32), "roped K (F32 cache)", atol=2e-6, rtol=2e-6)
        assert np.array_equal(vc, vr)                                   # V copy is exact
    elif kv_type == O.F16:
        _f16_ulp_close(kc.view(np.float16), kr.view(np.float16))
        assert np.array_equal(vc, vr)
    else:
        _q8_close(kc, kr)
        assert np.array_equal(vc, vr)                                   # V quantised from identical floats
    untouched = np.setdiff1d(np.arange(rows), slots)
    assert not kc[untouched].any() and not vc[untouched].any()


@pytest.mark.gpu
@pytest.mark.parametrize("kv_type", [O.F16, O.Q8_0])
def test_gpu_kv_append_many_tokens(kv_type):
    """A prefill-sized call (400 tokens, at least two per SM): one CTA per
    token walks all of the token's rows, where a decode step's few tokens
    spread their rows over CTAs of 8."""
    q, k, v, pos = make_inputs(40 + kv_type, T=400, Hq=32, Hkv=8, D=128)
    rows = 512
    slots = np.random.default_rng(6).permutation(rows)[:len(pos)].astype(np.int32)
    qo, kc, vc = _gpu_append(q, k, v, pos, slots, kv_type, rows)
    kr, vr = empty_cache(rows, 8, 128, kv_type), empty_cache(rows, 8, 128, kv_type)
    qr = O.kv_append(q, k, v, pos, slots, kv_type, BASE, kr, vr)
    assert_close(qo, qr, "roped Q", atol=2e-6, rtol=2e-6)
    if kv_type == O.F16:
        _f16_ulp_close(kc.view(np.float16), kr.view(np.float16))
    else:
        _q8_close(kc, kr)
    assert np.array_equal(vc, vr)


@pytest.mark.gpu
def test_gpu_kv_append_per_stream_caches():
    """Batched decode: one token per stream, each into its own cache (k_cache_ptrs)."""
    import torch
    import vtx_attn
    n_seq, Hkv, D, rows = 5, 8, 128, 32
    q, k, v, pos = make_inputs(21, T=n_seq, Hq=32, Hkv=Hkv, D=D)
    slots = np.array([0, 31, 7, 16, 3], np.int32)
    hb = O.cache_head_bytes(O.Q8_0, D)
    kcs = [torch.zeros((rows, Hkv * hb), dtype=torch.uint8, device="cuda") for _ in range(n_seq)]
    vcs = [torch.zeros_like(c) for c in kcs]
    kp = torch.tensor([c.data_ptr() for c in kcs], dtype=torch.int64, device="cuda")
    vp = torch.tensor([c.data_ptr() for c in vcs], dtype=torch.int64, device="cuda")
    qo = vtx_attn.kv_append(torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda(), torch.from_numpy(pos).cuda(),
                            torch.from_numpy(slots).cuda(), None, None, O.Q8_0, BASE, q=torch.from_numpy(q).cuda(),
                            k_cache_ptrs=kp, v_cache_ptrs=vp, cache_nb1=Hkv * hb)
    torch.cuda.synchronize()
    for s in range(n_seq):
        kr, vr = empty_cache(rows, Hkv, D, O.Q8_0), empty_cache(rows, Hkv, D, O.Q8_0)
        qr = O.kv_append(q[s:s + 1], k[s:s + 1], v[s:s + 1], pos[s:s + 1], slots[s:s + 1], O.Q8_0, BASE, kr, vr)
        assert_close(qo[s:s + 1].cpu().numpy(), qr, f"stream {s} Q", atol=2e-6, rtol=2e-6)
        _q8_close(kcs[s].cpu().numpy(), kr)
        assert np.array_equal(vcs[s].cpu().numpy(), vr)


@pytest.mark.gpu
@pytest.mark.parametrize("kv_type", [O.F16, O.Q8_0])
def test_gpu_ring_append_then_decode(kv_type):
    """A full decode step sequence on a ring of 64 rows: 100 tokens appended
    one at a time at slot = token % 64 (positions keep growing), then attention
    of the last token's Q over the 64 cached rows.  The reference keeps the same
    64 most recent rows with its shift-left memmove; attention over them does
    not depend on the row order.  Checked against the oracle pipeline."""
    import torch
    import vtx_attn
    Hq, Hkv, D, W, n_tok = 32, 8, 128, 64, 100
    rng = np.random.default_rng(33)
    q = rng.standard_normal((n_tok, Hq, D)).astype(np.float32)
    k = rng.standard_normal((n_tok, Hkv, D)).astype(np.float32)
    v = rng.standard_normal((n_tok, Hkv, D)).astype(np.float32)
    pos = np.arange(n_tok, dtype=np.int32) + 375
    hb = O.cache_head_bytes(kv_type, D)
    kc = torch.zeros((W, Hkv * hb), dtype=torch.uint8, device="cuda")
    vc = torch.zeros_like(kc)
    kr, vr = empty_cache(W, Hkv, D, kv_type), empty_cache(W, Hkv, D, kv_type)
    for t in range(n_tok):
        sl = np.array([t % W], np.int32)
        qo = vtx_attn.kv_append(torch.from_numpy(k[t:t + 1]).cuda(), torch.from_numpy(v[t:t + 1]).cuda(),
                                torch.from_numpy(pos[t:t + 1]).cuda(), torch.from_numpy(sl).cuda(), kc, vc, kv_type,
                                BASE, q=torch.from_numpy(q[t:t + 1]).cuda())
        qr = O.kv_append(q[t:t + 1], k[t:t + 1], v[t:t + 1], pos[t:t + 1], sl, kv_type, BASE, kr, vr)
    torch.cuda.synchronize()
    # attention of the last token over the ring: GPU reads the GPU-written cache,
    # the oracle reads the oracle-written cache
    row = Hkv * hb
    kt = kc.view(W, Hkv, hb) if kv_type == O.Q8_0 else kc.view(torch.float16).view(W, Hkv, D)
    vt = vc.view(W, Hkv, hb) if kv_type == O.Q8_0 else vc.view(torch.float16).view(W, Hkv, D)
    got = vtx_attn.flash_attn_ext(qo.view(1, 1, Hq, D).permute(0, 2, 1, 3), kt.permute(1, 0, 2).unsqueeze(0),
                                  vt.permute(1, 0, 2).unsqueeze(0), None, D ** -0.5, kv_type=kv_type)
    kn = kr.reshape(W, Hkv, hb) if kv_type == O.Q8_0 else kr.view(np.float16).reshape(W, Hkv, D)
    vn = vr.reshape(W, Hkv, hb) if kv_type == O.Q8_0 else vr.view(np.float16).reshape(W, Hkv, D)
    ref = O.flash_attn_ext(qr.reshape(1, 1, Hq, D).transpose(0, 2, 1, 3), kn.transpose(1, 0, 2)[None],
                           vn.transpose(1, 0, 2)[None], None, D ** -0.5, kv_type=kv_type)
    assert_close(got.cpu().numpy(), ref, f"ring decode step ({'q8_0' if kv_type == O.Q8_0 else 'f16'})")
    assert row == kc.shape[1]
