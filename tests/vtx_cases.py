"""Seeded attention problems laid out exactly as voxtral.cpp hands them to
ggml_flash_attn_ext, as matched numpy (oracle) / torch (device) views.

Geometry followed:
  * Q: contiguous [D, Hq, n_q] F32 buffer permuted to [D, n_q, Hq]
    (src/voxtral.cpp:1589,1601 encoder; :1785-1786 decoder).
  * K/V encoder: same as Q (:1590-1605).
  * K/V decoder: slice [0, n_kv) of a cache [kv_dim = Hkv*D, n_ctx] viewed as
    [D, n_kv, Hkv] (:1126-1136, :1772-1794).
  * masks: F16 [n_kv, n_q] causal (:2103-2111) or window-750 (:2181-2188).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional

import numpy as np

import oracle as O

ATOL, RTOL = 2e-3, 1e-2          # BASELINE north_star tolerance (fp32 accumulate)


@dataclass
class Case:
    q: np.ndarray                 # (B, Hq, n_q, D) view
    k: np.ndarray                 # (B, Hkv, n_kv, D[bytes]) view
    v: np.ndarray
    mask: Optional[np.ndarray]
    scale: float
    kv_type: int
    max_bias: float = 0.0
    softcap: float = 0.0
    causal: int = 0
    window: int = 0
    bufs: dict = field(default_factory=dict)


def _kv_store(x: np.ndarray, kv: str) -> np.ndarray:
    if kv == "f16":
        return x.astype(np.float16)
    if kv == "f32":
        return x.astype(np.float32)
    return O.quantize_q8_0(x)


def make_case(seed: int, *, B=1, Hq=8, Hkv=2, n_q=16, n_kv=16, D=128, kv="f16", q16=False,
              mask=None, causal=0, window=0, max_bias=0.0, softcap=0.0, cache=True,
              n_ctx=None) -> Case:
    """mask: None | 'causal' | 'window' | 'random' (explicit F16 tensor)."""
    rng = np.random.default_rng(seed)
    qbuf = rng.standard_normal((B, n_q, Hq, D)).astype(np.float16 if q16 else np.float32)
    q = qbuf.transpose(0, 2, 1, 3)                                      # (B, Hq, n_q, D)
    kv_t = {"f16": O.F16, "f32": O.F32, "q8_0": O.Q8_0}[kv]
    if cache:
        n_ctx = n_ctx or n_kv + 3
        kf = rng.standard_normal((B, n_ctx, Hkv, D)).astype(np.float32)
        vf = rng.standard_normal((B, n_ctx, Hkv, D)).astype(np.float32)
        kbuf, vbuf = _kv_store(kf, kv), _kv_store(vf, kv)
        k = kbuf[:, :n_kv].transpose(0, 2, 1, 3)
        v = vbuf[:, :n_kv].transpose(0, 2, 1, 3)
    else:
        kf = rng.standard_normal((B, n_kv, Hkv, D)).astype(np.float32)
        vf = rng.standard_normal((B, n_kv, Hkv, D)).astype(np.float32)
        kbuf, vbuf = _kv_store(kf, kv), _kv_store(vf, kv)
        k, v = kbuf.transpose(0, 2, 1, 3), vbuf.transpose(0, 2, 1, 3)
    m = None
    if mask == "causal":
        m = np.zeros((n_q, n_kv), np.float32)
        m[np.arange(n_q)[:, None] + (n_kv - n_q) < np.arange(n_kv)[None, :]] = -np.inf
        m = m.astype(np.float16)
    elif mask == "window":
        assert n_q == n_kv
        m = O.window_mask(n_q, window or 750)
    elif mask == "random":
        m = (rng.standard_normal((n_q, n_kv)) * 2).astype(np.float16)
        m[rng.random((n_q, n_kv)) < 0.2] = -np.inf
    return Case(q=q, k=k, v=v, mask=m, scale=1.0 / np.sqrt(D), kv_type=kv_t, max_bias=max_bias,
                softcap=softcap, causal=causal, window=window if causal else 0,
                bufs={"q": qbuf, "k": kbuf, "v": vbuf})


def oracle_out(c: Case, mode=O.MODE_GGML) -> np.ndarray:
    return O.flash_attn_ext(c.q, c.k, c.v, c.mask, c.scale, c.max_bias, c.softcap, c.causal,
                            c.window, kv_type=c.kv_type, mode=mode)


def to_device(c: Case):
    """torch views on cuda:0 with the same strides as the numpy views."""
    import torch

    def mirror(view: np.ndarray, buf: np.ndarray):
        tb = torch.from_numpy(np.ascontiguousarray(buf)).cuda()
        es = buf.itemsize
        off = (view.__array_interface__["data"][0] - buf.__array_interface__["data"][0]) // es
        return tb.as_strided(view.shape, [s // es for s in view.strides], off)

    q = mirror(c.q, c.bufs["q"])
    k = mirror(c.k, c.bufs["k"])
    v = mirror(c.v, c.bufs["v"])
    m = torch.from_numpy(c.mask).cuda() if c.mask is not None else None
    return q, k, v, m


def assert_close(got: np.ndarray, ref: np.ndarray, what: str, atol=ATOL, rtol=RTOL) -> None:
    err = np.abs(got.astype(np.float64) - ref.astype(np.float64))
    bound = atol + rtol * np.abs(ref)
    bad = err > bound
    if bad.any():
        idx = np.unravel_index(np.argmax(err - bound), err.shape)
        raise AssertionError(f"{what}: {bad.sum()} / {err.size} elements outside atol={atol} rtol={rtol}; "
                             f"worst at {idx}: got {got[idx]} ref {ref[idx]} (max abs err {err.max():.3e})")


def assert_parity(got: np.ndarray, ggml: np.ndarray, fp64: np.ndarray, what: str) -> dict:
    """oracle.parity_verdict as an assertion (the bound for sizes where ggml's
    half-precision V accumulator drifts from exact arithmetic by more than
    ATOL): within tolerance of fp64 truth everywhere, and of ggml up to
    ggml's own per-element drift."""
    v = O.parity_verdict(got, ggml, fp64)
    assert v["ok"], f"{what}: {v}"
    return v


def f16_ulp_close(got: np.ndarray, ref: np.ndarray) -> None:
    """Rotated K rows in half: within one f16 ulp (the device takes cos/sin in
    double rounded to float, ggml's CPU cosf/sinf may differ in the last bit)."""
    g, r = got.astype(np.float32), ref.astype(np.float32)
    ulp = np.spacing(np.abs(ref).astype(np.float16)).astype(np.float32)
    assert np.all(np.abs(g - r) <= ulp), np.abs(g - r).max()


def q8_close(got: np.ndarray, ref: np.ndarray) -> None:
    """Q8_0 rows: scales within one f16 ulp, values within one step (a float
    that lands on a rounding boundary may differ in its last bit)."""
    g = got.reshape(-1, 34)
    r = ref.reshape(-1, 34)
    gd, rd = g[:, :2].copy().view(np.float16).ravel(), r[:, :2].copy().view(np.float16).ravel()
    f16_ulp_close(gd, rd)
    gq, rq = g[:, 2:].view(np.int8).astype(int), r[:, 2:].view(np.int8).astype(int)
    assert np.abs(gq - rq).max() <= 1
    assert (gq != rq).mean() < 0.01
