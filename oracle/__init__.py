"""CPU oracle for the voxtral.cpp attention node — TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
use this package, as the checker.  The product package (voxtral.cpp_b200)
never imports it.

``vtx_ref.c`` restates ggml's CPU ``flash_attn_ext`` numerics
(ggml/src/ggml-cpu/ops.cpp ``ggml_compute_forward_flash_attn_ext_f16`` at
ggml@5cecdad, the revision pinned by reference CMakeLists.txt:33-41) and an
fp64 "truth" mode.  Parity at the op level is UNPINNED against ggml itself
(no ggml source/binary here; the reference's tests only pin end-to-end logits
that need absent weights).  Pinned pieces: Q8_0 bytes vs gguf-py 0.19.0,
fp64 mode vs torch float64 attention (tests/golden/).

Tensors are numpy arrays in ggml geometry read back to front: an array of
shape (B, H, n, D) with arbitrary strides is the ggml view [D, n, H, B] with
nb = strides reversed.  Q8_0 tensors are uint8 arrays whose last axis holds
D/32 blocks of 34 bytes.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libvtx_ref.so")
_lib = None

F32, F16, Q8_0 = 0, 1, 8
QK8_0 = 32
Q8_0_BLOCK = 34
MODE_GGML, MODE_FP64 = 0, 1


class Tensor(ctypes.Structure):
    _fields_ = [("type", ctypes.c_int32), ("reserved", ctypes.c_int32),
                ("ne", ctypes.c_int64 * 4), ("nb", ctypes.c_size_t * 4),
                ("data", ctypes.c_void_p)]


class Params(ctypes.Structure):
    _fields_ = [("scale", ctypes.c_float), ("max_bias", ctypes.c_float),
                ("logit_softcap", ctypes.c_float), ("causal", ctypes.c_int32),
                ("window", ctypes.c_int32), ("reserved", ctypes.c_int32 * 3)]


class DecodeBatch(ctypes.Structure):
    _fields_ = [("n_seq", ctypes.c_int32), ("n_head_q", ctypes.c_int32),
                ("n_head_kv", ctypes.c_int32), ("head_dim", ctypes.c_int32),
                ("kv_type", ctypes.c_int32), ("max_kv_len", ctypes.c_int32),
                ("kv_nb1", ctypes.c_size_t), ("kv_nb2", ctypes.c_size_t),
                ("q", ctypes.c_void_p), ("k_ptrs", ctypes.c_void_p),
                ("v_ptrs", ctypes.c_void_p), ("kv_len", ctypes.c_void_p),
                ("dst", ctypes.c_void_p), ("scale", ctypes.c_float),
                ("reserved", ctypes.c_int32)]


def build(force: bool = False) -> str:
    """Compile vtx_ref.c (make) unless the library is already there."""
    src = os.path.join(_HERE, "vtx_ref.c")
    if force or not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def build_ref() -> str | None:
    """Compile oracle/_ref/enc_tokens_ref from the reference's own sources
    (`src/voxtral.cpp` encoder token-count functions, extracted by the
    Makefile's `ref` target) when the reference tree sits beside this
    repository; None when it does not.  The binary only generates
    tests/golden/enc_chunks.json; nothing at run time needs it."""
    ref_src = os.path.join(_HERE, "..", "..", "reference", "src", "voxtral.cpp")
    if not os.path.exists(ref_src):
        return None
    subprocess.run(["make", "-s", "-C", _HERE, "ref"], check=True)
    return os.path.join(_HERE, "_ref", "enc_tokens_ref")


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(_LIB_PATH)
        vp, i64 = ctypes.c_void_p, ctypes.c_int64
        for name in ("vtx_ref_quantize_q8_0", "vtx_ref_quantize_q8_0_rne",
                     "vtx_ref_dequantize_q8_0", "vtx_ref_f32_to_f16", "vtx_ref_f16_to_f32"):
            getattr(L, name).argtypes = [vp, vp, i64]
            getattr(L, name).restype = None
        L.vtx_ref_flash_attn_ext.argtypes = [ctypes.POINTER(Tensor)] * 4 + [
            ctypes.POINTER(Params), ctypes.POINTER(Tensor), ctypes.c_int, ctypes.c_int]
        L.vtx_ref_flash_attn_ext.restype = ctypes.c_int
        L.vtx_ref_decode_batched.argtypes = [ctypes.POINTER(DecodeBatch), ctypes.c_int, ctypes.c_int]
        L.vtx_ref_decode_batched.restype = ctypes.c_int
        L.vtx_ref_kv_append.argtypes = [ctypes.c_int] * 5 + [ctypes.c_float] + [vp] * 8 + [ctypes.c_size_t,
                                                                                          ctypes.c_int]
        L.vtx_ref_kv_append.restype = ctypes.c_int
        L.vtx_ref_out_proj.argtypes = [vp, i64, vp, i64, vp, vp, i64, vp, i64] + [ctypes.c_int] * 5
        L.vtx_ref_out_proj.restype = ctypes.c_int
        _lib = L
    return _lib


def n_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1


# ---- formats ------------------------------------------------------------

def quantize_q8_0(x: np.ndarray) -> np.ndarray:
    """ggml quantize_row_q8_0_ref over the last axis (multiple of 32).
    Returns uint8 with last axis D/32*34."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    D = x.shape[-1]
    assert D % QK8_0 == 0
    out = np.empty(x.shape[:-1] + (D // QK8_0 * Q8_0_BLOCK,), dtype=np.uint8)
    lib().vtx_ref_quantize_q8_0(x.ctypes.data, out.ctypes.data, x.size)
    return out


def dequantize_q8_0(b: np.ndarray) -> np.ndarray:
    b = np.ascontiguousarray(b, dtype=np.uint8)
    D = b.shape[-1] // Q8_0_BLOCK * QK8_0
    out = np.empty(b.shape[:-1] + (D,), dtype=np.float32)
    lib().vtx_ref_dequantize_q8_0(b.ctypes.data, out.ctypes.data, out.size)
    return out


def to_f16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.float16)
    lib().vtx_ref_f32_to_f16(x.ctypes.data, out.ctypes.data, x.size)
    return out


# ---- tensors --------------------------------------------------------------

def tensor(a: np.ndarray, ttype: int | None = None) -> Tensor:
    """ggml descriptor for a numpy array (shape reversed = ne)."""
    if a.ndim > 4:
        raise ValueError("at most 4 dims")
    shape = (1,) * (4 - a.ndim) + tuple(a.shape)
    strides = (0,) * (4 - a.ndim) + tuple(a.strides)
    if ttype is None:
        ttype = {np.dtype(np.float32): F32, np.dtype(np.float16): F16}[a.dtype]
    t = Tensor()
    t.type = ttype
    ne = list(reversed(shape))
    nb = list(reversed(strides))
    if ttype == Q8_0:
        ne[0] = ne[0] // Q8_0_BLOCK * QK8_0
        nb[0] = Q8_0_BLOCK
    # broadcast dims of size 1 get a consistent stride
    for i in range(1, 4):
        if nb[i] == 0:
            nb[i] = nb[i - 1] * (ne[i - 1] if i > 1 or ttype != Q8_0 else ne[0] // QK8_0)
    for i in range(4):
        t.ne[i] = ne[i]
        t.nb[i] = nb[i]
    t.data = a.ctypes.data
    return t


def params(scale: float, max_bias: float = 0.0, softcap: float = 0.0,
           causal: int = 0, window: int = 0) -> Params:
    p = Params()
    p.scale, p.max_bias, p.logit_softcap = scale, max_bias, softcap
    p.causal, p.window = int(causal), int(window)
    return p


def flash_attn_ext(q: np.ndarray, k: np.ndarray, v: np.ndarray, mask: np.ndarray | None,
                   scale: float, max_bias: float = 0.0, softcap: float = 0.0,
                   causal: int = 0, window: int = 0, kv_type: int | None = None,
                   mode: int = MODE_GGML, threads: int | None = None) -> np.ndarray:
    """Run the oracle.  q: (B, Hq, n_q, D) view; k/v: (B, Hkv, n_kv, D[bytes]);
    mask: (n_q', n_kv) F16 or (B|1, Hq|1, n_q', n_kv) or None.
    Returns dst as float32 (B, n_q, Hq, Dv) — ggml's [Dv, Hq, n_q, B]."""
    tq = tensor(q)
    tk = tensor(k, kv_type)
    tv = tensor(v, kv_type)
    B, Hq, n_q = tq.ne[3], tq.ne[2], tq.ne[1]
    Dv = tv.ne[0]
    dst = np.zeros((B, n_q, Hq, Dv), dtype=np.float32)
    td = tensor(dst)
    tm = tensor(mask, F16) if mask is not None else None
    p = params(scale, max_bias, softcap, causal, window)
    rc = lib().vtx_ref_flash_attn_ext(ctypes.byref(tq), ctypes.byref(tk), ctypes.byref(tv),
                                      ctypes.byref(tm) if tm is not None else None,
                                      ctypes.byref(p), ctypes.byref(td), mode,
                                      threads or n_cores())
    if rc != 0:
        raise ValueError(f"oracle rejected operands: status {rc}")
    return dst


def decode_batched(q: np.ndarray, k_list, v_list, kv_len, scale: float, kv_type: int,
                   n_head_kv: int, kv_nb1: int, kv_nb2: int, mode: int = MODE_GGML,
                   threads: int | None = None) -> np.ndarray:
    """Host version of vtx_flash_attn_decode_batched.  q: (n_seq, Hq, D) f32;
    k_list/v_list: per-stream numpy buffers (any dtype, byte-addressed with
    kv_nb1 per token and kv_nb2 per head)."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    n_seq, Hq, D = q.shape
    dst = np.zeros_like(q)
    kp = (ctypes.c_void_p * n_seq)(*[a.ctypes.data for a in k_list])
    vp = (ctypes.c_void_p * n_seq)(*[a.ctypes.data for a in v_list])
    kl = np.ascontiguousarray(kv_len, dtype=np.int32)
    b = DecodeBatch()
    b.n_seq, b.n_head_q, b.n_head_kv, b.head_dim = n_seq, Hq, n_head_kv, D
    b.kv_type, b.max_kv_len = kv_type, int(kl.max()) if n_seq else 0
    b.kv_nb1, b.kv_nb2 = kv_nb1, kv_nb2
    b.q, b.k_ptrs, b.v_ptrs = q.ctypes.data, ctypes.addressof(kp), ctypes.addressof(vp)
    b.kv_len, b.dst, b.scale = kl.ctypes.data, dst.ctypes.data, scale
    rc = lib().vtx_ref_decode_batched(ctypes.byref(b), mode, threads or n_cores())
    if rc != 0:
        raise ValueError(f"oracle rejected batch: status {rc}")
    return dst


def cache_head_bytes(kv_type: int, D: int) -> int:
    return D * 4 if kv_type == F32 else D * 2 if kv_type == F16 else D // QK8_0 * Q8_0_BLOCK


def kv_append(q: np.ndarray | None, k: np.ndarray, v: np.ndarray, positions, slots, kv_type: int,
              freq_base: float, k_cache: np.ndarray, v_cache: np.ndarray, mode: int = MODE_GGML):
    """Decoder KV update on the host: RoPE of Q and K (ggml mode 0) and the
    K/V cache write at rows ``slots`` (uint8 caches [n_rows, Hkv * head bytes],
    written in place).  q: (T, Hq, D) or None, k/v: (T, Hkv, D) float32.
    Returns the roped Q (or None)."""
    k = np.ascontiguousarray(k, dtype=np.float32)
    v = np.ascontiguousarray(v, dtype=np.float32)
    T, Hkv, D = k.shape
    pos = np.ascontiguousarray(positions, dtype=np.int32)
    sl = np.ascontiguousarray(slots, dtype=np.int32)
    assert k_cache.flags.c_contiguous and v_cache.flags.c_contiguous and k_cache.dtype == np.uint8
    assert k_cache.shape[1] == Hkv * cache_head_bytes(kv_type, D) and v_cache.shape == k_cache.shape
    assert sl.max(initial=-1) < k_cache.shape[0] and sl.min(initial=0) >= 0
    qo = None
    qp = qop = None
    Hq = 0
    if q is not None:
        q = np.ascontiguousarray(q, dtype=np.float32)
        Hq = q.shape[1]
        qo = np.empty_like(q)
        qp, qop = q.ctypes.data, qo.ctypes.data
    rc = lib().vtx_ref_kv_append(T, Hq, Hkv, D, kv_type, freq_base, qp, qop, k.ctypes.data, v.ctypes.data,
                                 pos.ctypes.data, sl.ctypes.data, k_cache.ctypes.data, v_cache.ctypes.data,
                                 k_cache.strides[0], mode)
    if rc != 0:
        raise ValueError(f"oracle rejected kv_append: status {rc}")
    return qo


# ---- reference masks (host-built, exactly as voxtral.cpp fills them) ------

def causal_mask(n: int) -> np.ndarray:
    """src/voxtral.cpp:2103-2111 fill_causal_mask, cast to F16 (:1801)."""
    m = np.zeros((n, n), dtype=np.float32)
    m[np.triu_indices(n, 1)] = -np.inf
    return m.astype(np.float16)


def window_mask(n: int, window: int = 750) -> np.ndarray:
    """src/voxtral.cpp:2181-2188 sliding causal mask (chunk-local), F16 (:1564)."""
    qi = np.arange(n)[:, None]
    kj = np.arange(n)[None, :]
    allow = (kj <= qi) & (kj >= np.maximum(0, qi - (window - 1)))
    return np.where(allow, 0.0, -np.inf).astype(np.float16)


# ---- realtime encoder chunking ---------------------------------------------------
# Restates the chunk geometry of run_encoder_chunked (src/voxtral.cpp:2234-2335):
# 3000 mel frames per chunk, 1500-frame stride, 750 overlapping encoder tokens
# skipped in every chunk but the first (:26-27), token counts through the two
# causal convolutions (compute_causal_conv1d_dims :1280-1297,
# mel_frames_to_enc_tokens :1300-1305, downsample factor 4 from
# include/voxtral.h:51).  Pinned against the reference's own token-count
# functions compiled from their source (tests/golden/enc_chunks.json).

ENC_CHUNK_MEL, ENC_CHUNK_OVERLAP, DOWNSAMPLE = 3000, 750, 4


def causal_conv1d_out_len(in_len: int, kernel: int, stride: int) -> int:
    """Output length of compute_causal_conv1d_dims (:1280-1297); its frame
    count is float32 arithmetic, reproduced with numpy float32."""
    if in_len <= 0 or kernel <= 0 or stride <= 0:
        return 0
    pad_total = kernel - stride
    n_frames = np.float32(in_len - kernel + pad_total) / np.float32(stride) + np.float32(1.0)
    target = (int(np.ceil(n_frames)) - 1) * stride + (kernel - pad_total)
    padded = in_len + pad_total + max(0, target - in_len)
    return (padded - kernel) // stride + 1


def mel_frames_to_enc_tokens(n_frames: int) -> int:
    """:1300-1305: conv0 (k 3, s 1), conv1 (k 3, s 2), truncated to a
    multiple of the downsample factor."""
    n = causal_conv1d_out_len(causal_conv1d_out_len(n_frames, 3, 1), 3, 2)
    return n - n % DOWNSAMPLE


def compute_total_enc_tokens(total_mel: int) -> int:
    """:1308-1325: the stitched token count (the output allocation)."""
    stride_mel = ENC_CHUNK_MEL - 2 * ENC_CHUNK_OVERLAP
    total, off, first = 0, 0, True
    while off < total_mel:
        toks = mel_frames_to_enc_tokens(min(ENC_CHUNK_MEL, total_mel - off))
        s = toks - (0 if first else ENC_CHUNK_OVERLAP)
        if s <= 0:
            break
        total += s
        off += stride_mel
        first = False
    return total


def encoder_chunk_plan(total_mel: int):
    """The chunks run_encoder_chunked processes, in order, as dicts with
    mel_offset, mel_frames, n_tokens, skip, stride, rope_offset and
    write_offset; plus (alloc_total, enc_seq_used)."""
    alloc_total = compute_total_enc_tokens(total_mel)
    chunks = []
    if alloc_total <= 0:
        return chunks, alloc_total, 0
    stride_mel = ENC_CHUNK_MEL - 2 * ENC_CHUNK_OVERLAP
    off, write, idx = 0, 0, 0
    while off < total_mel:
        frames = min(ENC_CHUNK_MEL, total_mel - off)
        skip = ENC_CHUNK_OVERLAP if idx > 0 else 0
        toks = mel_frames_to_enc_tokens(frames)
        if toks - skip <= 0:                       # pre-check (:2265-2272)
            break
        stride = toks - skip
        if stride <= 0:
            break
        if write + stride > alloc_total:           # clamp (:2307-2311)
            stride = alloc_total - write
            if stride <= 0:
                break
        chunks.append(dict(mel_offset=off, mel_frames=frames, n_tokens=toks, skip=skip, stride=stride,
                           rope_offset=write - skip, write_offset=write))
        write += stride
        off += stride_mel
        idx += 1
    return chunks, alloc_total, write // DOWNSAMPLE * DOWNSAMPLE


def encoder_stitch(chunk_out: np.ndarray, chunks, n_rows: int) -> np.ndarray:
    """Host-side stitch as :2318-2328 does it: rows [skip, skip + stride) of
    chunk c's output to rows [write_offset, write_offset + stride).
    chunk_out: (n_chunks, chunk_rows, ...)."""
    out = np.zeros((n_rows,) + chunk_out.shape[2:], dtype=chunk_out.dtype)
    for c, ch in enumerate(chunks):
        out[ch["write_offset"]:ch["write_offset"] + ch["stride"]] = chunk_out[c, ch["skip"]:ch["skip"] + ch["stride"]]
    return out


def out_proj(attn: np.ndarray, w: np.ndarray, bias: np.ndarray | None = None, residual: np.ndarray | None = None,
             mode: int = MODE_GGML, threads: int | None = None) -> np.ndarray:
    """Host version of vtx_attn_out_proj: attn (n, K) F32 (the attention
    output with its heads flattened, ggml's [Dv*Hq, n]), w (N, K) float16,
    bias (N,) F32 or None, residual (n, N) F32 or None -> (n, N) F32."""
    a = np.ascontiguousarray(attn, dtype=np.float32)
    wh = np.ascontiguousarray(w, dtype=np.float16)
    n, K = a.shape
    N = wh.shape[0]
    assert wh.shape[1] == K
    b = np.ascontiguousarray(bias, dtype=np.float32) if bias is not None else None
    r = np.ascontiguousarray(residual, dtype=np.float32) if residual is not None else None
    out = np.empty((n, N), dtype=np.float32)
    rc = lib().vtx_ref_out_proj(a.ctypes.data, K, wh.ctypes.data, K, b.ctypes.data if b is not None else None,
                                r.ctypes.data if r is not None else None, N, out.ctypes.data, N, n, K, N, mode,
                                threads or n_cores())
    if rc != 0:
        raise ValueError(f"oracle rejected operands: status {rc}")
    return out


# ---- the parity criterion ------------------------------------------------------
ATOL, RTOL = 2e-3, 1e-2          # BASELINE north_star tolerance (fp32 accumulate on the GPU)


def parity_verdict(got: np.ndarray, ggml: np.ndarray, fp64: np.ndarray) -> dict:
    """Judges a device result against the oracle run in both modes.

    drift = |ggml - fp64| per element: how far ggml's own CPU arithmetic is
    from exact attention.  It is large in two places: ggml accumulates P.V
    in half precision when V is F16 (VKQ16), which over thousands of keys
    moves the result by up to a few 1e-3; and for a Q8_0 K ggml quantises Q
    to Q8_0 before the dot product, which the device reproduces on purpose.
    The device result must be within ATOL + RTOL |ref| + drift of BOTH:
      * ggml mode (it may differ from ggml by no more than ggml's own
        rounding beyond the tolerance), and
      * fp64 truth (it may be as far from exact as ggml is, no further).
    Where ggml is exact (drift ~ 0) this is the plain tolerance twice.
    Returns the maxima and the verdict."""
    got = got.astype(np.float64)
    g = ggml.astype(np.float64)
    f = fp64.astype(np.float64)
    e_g, e_f, drift = np.abs(got - g), np.abs(got - f), np.abs(g - f)
    ok_f = bool(np.all(e_f <= ATOL + RTOL * np.abs(f) + drift))
    ok_g = bool(np.all(e_g <= ATOL + RTOL * np.abs(g) + drift))
    return {"max_abs_err_vs_ggml": float(e_g.max()) if e_g.size else 0.0,
            "max_abs_err_vs_fp64": float(e_f.max()) if e_f.size else 0.0,
            "ggml_max_drift_from_fp64": float(drift.max()) if drift.size else 0.0,
            "ok_vs_fp64": ok_f, "ok_vs_ggml": ok_g, "ok": ok_f and ok_g}
