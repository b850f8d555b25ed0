"""Host-side mirror of ggml_flash_attn_ext over the libvtx_fa.so C ABI.

This is the Python face of the node voxtral.cpp builds at src/voxtral.cpp:1611
(encoder) and src/voxtral.cpp:1802 (decoder): same operands, same argument
meaning (ggml views [D, n, H, B] -> here torch tensors (B, H, n, D) with any
strides), same result layout (ggml dst [Dv, Hq, n_q, B] -> torch (B, n_q, Hq,
Dv) float32).  Errors from the library raise ``VtxError`` (ggml would abort
with GGML_ASSERT).  torch supplies device memory and streams only; all
arithmetic runs in the library's sm_100a kernels.  There is no CPU fallback:
without the library or an sm_100 device every call raises.
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional, Sequence

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libvtx_fa.so")

F32, F16, Q8_0 = 0, 1, 8
QK8_0, Q8_0_BLOCK = 32, 34

STATUS = {0: "ok", -1: "null pointer", -2: "type", -3: "shape", -4: "stride", -5: "unsupported",
          -6: "workspace", -7: "cuda", -8: "no sm_100 device"}


class VtxError(RuntimeError):
    def __init__(self, status: int, what: str = ""):
        self.status = status
        super().__init__(f"vtx status {status} ({STATUS.get(status, '?')}){': ' + what if what else ''}")


class VtxTensor(ctypes.Structure):
    _fields_ = [("type", ctypes.c_int32), ("reserved", ctypes.c_int32),
                ("ne", ctypes.c_int64 * 4), ("nb", ctypes.c_size_t * 4),
                ("data", ctypes.c_void_p)]


class FaParams(ctypes.Structure):
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
                ("reserved", ctypes.c_int32), ("fresh_row", ctypes.c_void_p)]


class KvAppendArgs(ctypes.Structure):
    """vtx_kv_append_args (include/vtx_fa.h)."""
    _fields_ = [("n_tokens", ctypes.c_int32), ("n_head_q", ctypes.c_int32),
                ("n_head_kv", ctypes.c_int32), ("head_dim", ctypes.c_int32),
                ("kv_type", ctypes.c_int32), ("freq_base", ctypes.c_float),
                ("q", ctypes.c_void_p), ("q_nb1", ctypes.c_size_t),
                ("q_out", ctypes.c_void_p), ("q_out_nb1", ctypes.c_size_t),
                ("k", ctypes.c_void_p), ("k_nb1", ctypes.c_size_t),
                ("v", ctypes.c_void_p), ("v_nb1", ctypes.c_size_t),
                ("positions", ctypes.c_void_p), ("slots", ctypes.c_void_p),
                ("k_cache", ctypes.c_void_p), ("v_cache", ctypes.c_void_p),
                ("k_cache_ptrs", ctypes.c_void_p), ("v_cache_ptrs", ctypes.c_void_p),
                ("cache_nb1", ctypes.c_size_t), ("reserved", ctypes.c_int32 * 4)]


class DecodeLayerArgs(ctypes.Structure):
    """vtx_decode_layer_args (include/vtx_fa.h)."""
    _fields_ = [("n_seq", ctypes.c_int32), ("n_head_q", ctypes.c_int32),
                ("n_head_kv", ctypes.c_int32), ("head_dim", ctypes.c_int32),
                ("kv_type", ctypes.c_int32), ("max_kv_len", ctypes.c_int32),
                ("freq_base", ctypes.c_float), ("scale", ctypes.c_float),
                ("q", ctypes.c_void_p), ("q_nb1", ctypes.c_size_t),
                ("k", ctypes.c_void_p), ("k_nb1", ctypes.c_size_t),
                ("v", ctypes.c_void_p), ("v_nb1", ctypes.c_size_t),
                ("positions", ctypes.c_void_p), ("slots", ctypes.c_void_p), ("kv_len", ctypes.c_void_p),
                ("k_cache_ptrs", ctypes.c_void_p), ("v_cache_ptrs", ctypes.c_void_p),
                ("cache_nb1", ctypes.c_size_t), ("dst", ctypes.c_void_p), ("dst_nb1", ctypes.c_size_t),
                ("early", ctypes.c_int32), ("reserved", ctypes.c_int32 * 3)]


class OutProjArgs(ctypes.Structure):
    """vtx_out_proj_args (include/vtx_fa.h)."""
    _fields_ = [("attn", ctypes.c_void_p), ("head_block", ctypes.c_int32), ("reserved", ctypes.c_int32),
                ("block_nb", ctypes.c_size_t), ("w", ctypes.c_void_p), ("bias", ctypes.c_void_p),
                ("residual", ctypes.c_void_p), ("dst", ctypes.c_void_p)]


class EncChunk(ctypes.Structure):
    """vtx_enc_chunk (include/vtx_fa.h): one chunk of the realtime encoder run."""
    _fields_ = [("mel_offset", ctypes.c_int32), ("mel_frames", ctypes.c_int32), ("n_tokens", ctypes.c_int32),
                ("skip", ctypes.c_int32), ("stride", ctypes.c_int32), ("rope_offset", ctypes.c_int32),
                ("write_offset", ctypes.c_int32), ("reserved", ctypes.c_int32)]

    def as_dict(self) -> dict:
        return {f: getattr(self, f) for f, _ in self._fields_ if f != "reserved"}


_lib = None


def load(path: str = LIB_PATH):
    """Load libvtx_fa.so (built by build.py).  Raises if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise RuntimeError(f"libvtx_fa.so not built ({path}); run voxtral.cpp_b200/build.py")
    L = ctypes.CDLL(path)
    P = ctypes.POINTER
    L.vtx_flash_attn_ext.argtypes = [P(VtxTensor), P(VtxTensor), P(VtxTensor), P(VtxTensor),
                                     P(FaParams), P(VtxTensor), ctypes.c_void_p, ctypes.c_size_t,
                                     ctypes.c_void_p]
    L.vtx_flash_attn_ext.restype = ctypes.c_int
    L.vtx_flash_attn_ext_workspace.argtypes = [P(VtxTensor), P(VtxTensor), P(VtxTensor), P(FaParams)]
    L.vtx_flash_attn_ext_workspace.restype = ctypes.c_size_t
    L.vtx_flash_attn_decode_batched.argtypes = [P(DecodeBatch), ctypes.c_void_p, ctypes.c_size_t,
                                                ctypes.c_void_p]
    L.vtx_flash_attn_decode_batched.restype = ctypes.c_int
    L.vtx_flash_attn_decode_batched_workspace.argtypes = [P(DecodeBatch)]
    L.vtx_flash_attn_decode_batched_workspace.restype = ctypes.c_size_t
    L.vtx_read_device_error.argtypes = [ctypes.c_void_p]
    L.vtx_read_device_error.restype = ctypes.c_int
    L.vtx_strerror.argtypes = [ctypes.c_int]
    L.vtx_strerror.restype = ctypes.c_char_p
    L.vtx_abi_version.argtypes = []
    L.vtx_abi_version.restype = ctypes.c_int
    L.vtx_kv_append.argtypes = [P(KvAppendArgs), ctypes.c_void_p]
    L.vtx_kv_append.restype = ctypes.c_int
    L.vtx_decode_advance.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32,
                                     ctypes.c_int32, ctypes.c_void_p]
    L.vtx_decode_advance.restype = ctypes.c_int
    L.vtx_encoder_chunk_plan.argtypes = [ctypes.c_int32, P(EncChunk), ctypes.c_int32, P(ctypes.c_int32),
                                         P(ctypes.c_int32)]
    L.vtx_encoder_chunk_plan.restype = ctypes.c_int
    L.vtx_encoder_stitch.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_void_p,
                                     ctypes.c_size_t, ctypes.c_size_t, P(EncChunk), ctypes.c_int32,
                                     ctypes.c_void_p]
    L.vtx_encoder_stitch.restype = ctypes.c_int
    L.vtx_attn_out_proj.argtypes = [P(OutProjArgs), ctypes.c_void_p]
    L.vtx_attn_out_proj.restype = ctypes.c_int
    L.vtx_decode_layer.argtypes = [P(DecodeLayerArgs), ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]
    L.vtx_decode_layer.restype = ctypes.c_int
    L.vtx_decode_layer_workspace.argtypes = [P(DecodeLayerArgs)]
    L.vtx_decode_layer_workspace.restype = ctypes.c_size_t
    _lib = L
    return L


def _ggml_type(t: torch.Tensor, kv_type: Optional[int]) -> int:
    if kv_type is not None:
        return kv_type
    if t.dtype == torch.float32:
        return F32
    if t.dtype == torch.float16:
        return F16
    raise VtxError(-2, f"dtype {t.dtype}")


def desc(t: Optional[torch.Tensor], ttype: Optional[int] = None) -> Optional[VtxTensor]:
    """ggml descriptor of a torch view: shape (B, H, n, D) -> ne [D, n, H, B].
    Q8_0 tensors are uint8 with the last axis holding D/32 blocks of 34 bytes."""
    if t is None:
        return None
    if t.dim() > 4:
        raise VtxError(-3, "at most 4 dims")
    ttype = _ggml_type(t, ttype)
    shape = [1] * (4 - t.dim()) + list(t.shape)
    es = t.element_size()
    strides = [0] * (4 - t.dim()) + [s * es for s in t.stride()]
    ne = list(reversed(shape))
    nb = list(reversed(strides))
    if ttype == Q8_0:
        ne[0] = ne[0] // Q8_0_BLOCK * QK8_0
        nb[0] = Q8_0_BLOCK
    row = nb[0] * (ne[0] // QK8_0 if ttype == Q8_0 else ne[0])
    for i in range(1, 4):
        if nb[i] == 0 or ne[i] == 1:
            nb[i] = nb[i] or (row if i == 1 else nb[i - 1] * ne[i - 1])
    d = VtxTensor()
    d.type = ttype
    for i in range(4):
        d.ne[i] = ne[i]
        d.nb[i] = nb[i]
    d.data = t.data_ptr()
    return d


def params(scale: float, max_bias: float = 0.0, logit_softcap: float = 0.0,
           causal: bool = False, window: int = 0) -> FaParams:
    p = FaParams()
    p.scale, p.max_bias, p.logit_softcap = float(scale), float(max_bias), float(logit_softcap)
    p.causal, p.window = int(bool(causal)), int(window)
    return p


def _check(rc: int, what: str = "") -> None:
    if rc != 0:
        raise VtxError(rc, what)


def workspace_bytes(q, k, v, scale, max_bias=0.0, logit_softcap=0.0, causal=False, window=0,
                    kv_type=None) -> int:
    L = load()
    p = params(scale, max_bias, logit_softcap, causal, window)
    n = L.vtx_flash_attn_ext_workspace(ctypes.byref(desc(q)), ctypes.byref(desc(k, kv_type)),
                                       ctypes.byref(desc(v, kv_type)), ctypes.byref(p))
    if n == ctypes.c_size_t(-1).value:
        raise VtxError(-3, "operands rejected")
    return int(n)


def flash_attn_ext(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                   mask: Optional[torch.Tensor] = None, scale: float = 1.0,
                   max_bias: float = 0.0, logit_softcap: float = 0.0, *,
                   causal: bool = False, window: int = 0, kv_type: Optional[int] = None,
                   out: Optional[torch.Tensor] = None, workspace: Optional[torch.Tensor] = None,
                   stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """ggml_flash_attn_ext(ctx, q, k, v, mask, scale, max_bias, logit_softcap).

    q: (B, Hq, n_q, D) F32/F16 view; k, v: (B, Hkv, n_kv, D) F16/F32 or Q8_0
    bytes (kv_type=Q8_0); mask: (n_q', n_kv) / (B|1, Hq|1, n_q', n_kv) F16 or
    None.  Returns (B, n_q, Hq, D) float32 (ggml's permuted dst)."""
    L = load()
    B, Hq, n_q = q.shape[0], q.shape[1], q.shape[2]
    Dv = v.shape[-1] if (kv_type or _ggml_type(v, None)) != Q8_0 else v.shape[-1] // Q8_0_BLOCK * QK8_0
    if out is None:
        out = torch.empty((B, n_q, Hq, Dv), dtype=torch.float32, device=q.device)
    p = params(scale, max_bias, logit_softcap, causal, window)
    dq, dk, dv = desc(q), desc(k, kv_type), desc(v, kv_type)
    need = L.vtx_flash_attn_ext_workspace(ctypes.byref(dq), ctypes.byref(dk), ctypes.byref(dv), ctypes.byref(p))
    if need == ctypes.c_size_t(-1).value:
        raise VtxError(-3, "operands rejected")
    if need and (workspace is None or workspace.numel() * workspace.element_size() < need):
        workspace = torch.empty(need, dtype=torch.uint8, device=q.device)
    ws_ptr = workspace.data_ptr() if (workspace is not None and need) else None
    ws_len = workspace.numel() * workspace.element_size() if (workspace is not None and need) else 0
    dm = desc(mask, F16) if mask is not None else None
    s = stream if stream is not None else torch.cuda.current_stream(q.device)
    rc = L.vtx_flash_attn_ext(ctypes.byref(dq), ctypes.byref(dk), ctypes.byref(dv),
                              ctypes.byref(dm) if dm is not None else None, ctypes.byref(p),
                              ctypes.byref(desc(out)), ws_ptr, ws_len, ctypes.c_void_p(s.cuda_stream))
    _check(rc, "vtx_flash_attn_ext")
    return out


class DecodeBatchPlan:
    """Device-side arrays for vtx_flash_attn_decode_batched over a fixed set of
    per-stream KV buffers (pointer arrays live on the device so one call can be
    captured in a CUDA graph and replayed)."""

    def __init__(self, k_bufs: Sequence[torch.Tensor], v_bufs: Sequence[torch.Tensor],
                 kv_len: torch.Tensor, n_head_q: int, n_head_kv: int, head_dim: int, kv_type: int,
                 kv_nb1: int, kv_nb2: int, max_kv_len: int, scale: float,
                 fresh_row: Optional[torch.Tensor] = None):
        """fresh_row: optional device int32 [n_seq], the row of each stream that
        the kernel launched just before each call writes (vtx_decode_batch)."""
        dev = kv_len.device
        self.k_ptrs = torch.tensor([t.data_ptr() for t in k_bufs], dtype=torch.int64, device=dev)
        self.v_ptrs = torch.tensor([t.data_ptr() for t in v_bufs], dtype=torch.int64, device=dev)
        self.kv_len = kv_len.to(torch.int32)
        self.keep = (list(k_bufs), list(v_bufs))
        b = DecodeBatch()
        b.n_seq, b.n_head_q, b.n_head_kv, b.head_dim = len(k_bufs), n_head_q, n_head_kv, head_dim
        b.kv_type, b.max_kv_len, b.kv_nb1, b.kv_nb2 = kv_type, max_kv_len, kv_nb1, kv_nb2
        b.k_ptrs, b.v_ptrs, b.kv_len = self.k_ptrs.data_ptr(), self.v_ptrs.data_ptr(), self.kv_len.data_ptr()
        b.scale = scale
        self.fresh_row = fresh_row
        b.fresh_row = fresh_row.data_ptr() if fresh_row is not None else None
        self.batch = b
        need = load().vtx_flash_attn_decode_batched_workspace(ctypes.byref(b))
        if need == ctypes.c_size_t(-1).value:
            raise VtxError(-3, "batch rejected")
        self.workspace = torch.empty(max(int(need), 1), dtype=torch.uint8, device=dev)
        self.need = int(need)

    def __call__(self, q: torch.Tensor, out: Optional[torch.Tensor] = None,
                 stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
        if out is None:
            out = torch.empty_like(q, dtype=torch.float32)
        self.batch.q = q.data_ptr()
        self.batch.dst = out.data_ptr()
        s = stream if stream is not None else torch.cuda.current_stream(q.device)
        rc = load().vtx_flash_attn_decode_batched(ctypes.byref(self.batch), self.workspace.data_ptr(),
                                                  self.workspace.numel(), ctypes.c_void_p(s.cuda_stream))
        _check(rc, "vtx_flash_attn_decode_batched")
        return out


def kv_append(k: torch.Tensor, v: torch.Tensor, positions: torch.Tensor, slots: torch.Tensor,
              k_cache: torch.Tensor, v_cache: torch.Tensor, kv_type: int, freq_base: float = 1e6, *,
              q: Optional[torch.Tensor] = None, q_out: Optional[torch.Tensor] = None,
              k_cache_ptrs: Optional[torch.Tensor] = None, v_cache_ptrs: Optional[torch.Tensor] = None,
              cache_nb1: Optional[int] = None, stream: Optional[torch.cuda.Stream] = None) -> Optional[torch.Tensor]:
    """vtx_kv_append: RoPE (ggml mode 0) of q and k, then k/v written into the
    cache rows ``slots`` (F32, F16 or Q8_0 bytes).  k, v: (T, Hkv, D) float32
    (heads contiguous), q: (T, Hq, D) float32 or None.  Caches: rows of
    Hkv * head bytes, ``cache_nb1`` bytes apart (default: the row size).
    Returns q_out (allocated when q is given and q_out is None)."""
    T, Hkv, D = k.shape
    for t in (k, v) + ((q,) if q is not None else ()):
        if t.dtype != torch.float32 or t.stride(2) != 1 or t.stride(1) != D:
            raise VtxError(-4, "q/k/v must be float32 with heads contiguous")
    if q is not None and q_out is None:
        q_out = torch.empty_like(q)
    a = KvAppendArgs()
    a.n_tokens, a.n_head_kv, a.head_dim, a.kv_type, a.freq_base = T, Hkv, D, kv_type, freq_base
    if q is not None:
        a.n_head_q, a.q, a.q_nb1 = q.shape[1], q.data_ptr(), q.stride(0) * 4
        a.q_out, a.q_out_nb1 = q_out.data_ptr(), q_out.stride(0) * 4
    a.k, a.k_nb1, a.v, a.v_nb1 = k.data_ptr(), k.stride(0) * 4, v.data_ptr(), v.stride(0) * 4
    pos = positions.to(torch.int32).contiguous()
    sl = slots.to(torch.int32).contiguous()
    a.positions, a.slots = pos.data_ptr(), sl.data_ptr()
    a.k_cache = k_cache.data_ptr() if k_cache is not None else None
    a.v_cache = v_cache.data_ptr() if v_cache is not None else None
    a.k_cache_ptrs = k_cache_ptrs.data_ptr() if k_cache_ptrs is not None else None
    a.v_cache_ptrs = v_cache_ptrs.data_ptr() if v_cache_ptrs is not None else None
    if cache_nb1 is None:
        cache_nb1 = k_cache.stride(0) * k_cache.element_size()
    a.cache_nb1 = cache_nb1
    s = stream if stream is not None else torch.cuda.current_stream(k.device)
    _check(load().vtx_kv_append(ctypes.byref(a), ctypes.c_void_p(s.cuda_stream)), "vtx_kv_append")
    return q_out


class DecodeLayerPlan:
    """vtx_decode_layer over a fixed set of per-stream caches: RoPE of Q and K,
    the new K/V row into ring slot ``slots[s]`` and decode attention over rows
    [0, kv_len[s]), one launch per call.  The counters (positions, slots,
    kv_len) and the cache pointer arrays live on the device, so a call can be
    captured in a CUDA graph and replayed while the counters advance."""

    def __init__(self, k_bufs: Sequence[torch.Tensor], v_bufs: Sequence[torch.Tensor], positions: torch.Tensor,
                 slots: torch.Tensor, kv_len: torch.Tensor, n_head_q: int, n_head_kv: int, head_dim: int,
                 kv_type: int, cache_nb1: int, max_kv_len: int, scale: float, freq_base: float = 1e6,
                 early: bool = False):
        dev = kv_len.device
        self.k_ptrs = torch.tensor([t.data_ptr() for t in k_bufs], dtype=torch.int64, device=dev)
        self.v_ptrs = torch.tensor([t.data_ptr() for t in v_bufs], dtype=torch.int64, device=dev)
        self.keep = (list(k_bufs), list(v_bufs), positions, slots, kv_len)
        a = DecodeLayerArgs()
        a.n_seq, a.n_head_q, a.n_head_kv, a.head_dim = len(k_bufs), n_head_q, n_head_kv, head_dim
        a.kv_type, a.max_kv_len, a.freq_base, a.scale = kv_type, max_kv_len, freq_base, scale
        a.positions, a.slots, a.kv_len = positions.data_ptr(), slots.data_ptr(), kv_len.data_ptr()
        a.k_cache_ptrs, a.v_cache_ptrs, a.cache_nb1 = self.k_ptrs.data_ptr(), self.v_ptrs.data_ptr(), cache_nb1
        a.early = 1 if early else 0
        self.args = a
        need = load().vtx_decode_layer_workspace(ctypes.byref(a))
        if need == ctypes.c_size_t(-1).value:
            raise VtxError(-3, "decode layer rejected")
        self.need = int(need)
        # zeroed once: the split-arrival counters start at 0 and every call leaves them there
        self.workspace = torch.zeros(max(self.need, 1), dtype=torch.uint8, device=dev)

    def __call__(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out: Optional[torch.Tensor] = None,
                 stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
        """q: (n_seq, Hq, D), k/v: (n_seq, Hkv, D) float32, heads contiguous;
        returns (n_seq, Hq, D) float32."""
        for t in (q, k, v):
            if t.dtype != torch.float32 or t.stride(2) != 1 or t.stride(1) != t.shape[2]:
                raise VtxError(-4, "q/k/v must be float32 with heads contiguous")
        if out is None:
            out = torch.empty_like(q)
        a = self.args
        a.q, a.q_nb1 = q.data_ptr(), q.stride(0) * 4
        a.k, a.k_nb1 = k.data_ptr(), k.stride(0) * 4
        a.v, a.v_nb1 = v.data_ptr(), v.stride(0) * 4
        a.dst, a.dst_nb1 = out.data_ptr(), out.stride(0) * 4
        s = stream if stream is not None else torch.cuda.current_stream(q.device)
        _check(load().vtx_decode_layer(ctypes.byref(a), self.workspace.data_ptr(), self.workspace.numel(),
                                       ctypes.c_void_p(s.cuda_stream)), "vtx_decode_layer")
        return out


# ---- realtime encoder: chunk plan and device-side stitch ---------------------

def encoder_chunk_plan(total_mel_frames: int):
    """The chunks run_encoder_chunked processes for an utterance
    (src/voxtral.cpp:2234-2335), through vtx_encoder_chunk_plan.  Returns
    (chunks as a ctypes array of EncChunk, stitched token count, count
    trimmed to a multiple of 4)."""
    L = load()
    tot, used = ctypes.c_int32(0), ctypes.c_int32(0)
    n = L.vtx_encoder_chunk_plan(int(total_mel_frames), None, 0, ctypes.byref(tot), ctypes.byref(used))
    _check(n if n < 0 else 0, "vtx_encoder_chunk_plan")
    arr = (EncChunk * max(n, 1))()
    n2 = L.vtx_encoder_chunk_plan(int(total_mel_frames), arr, n, ctypes.byref(tot), ctypes.byref(used))
    _check(n2 if n2 < 0 else 0, "vtx_encoder_chunk_plan")
    return (EncChunk * n).from_buffer(arr) if n else (EncChunk * 0)(), tot.value, used.value


def encoder_stitch(chunk_out: torch.Tensor, chunks, dst: torch.Tensor,
                   stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """Copies rows [skip, skip + stride) of each chunk's output into rows
    [write_offset, ...) of dst on the device (vtx_encoder_stitch).
    chunk_out: (n_chunks, rows, ...) with contiguous rows; dst: (rows_total, ...)."""
    if chunk_out.shape[0] < len(chunks):
        raise ValueError("fewer chunk outputs than chunks")
    row_bytes = chunk_out[0, 0].numel() * chunk_out.element_size()
    if dst[0].numel() * dst.element_size() != row_bytes or not chunk_out[0, 0].is_contiguous():
        raise ValueError("row size mismatch or non-contiguous rows")
    s = stream if stream is not None else torch.cuda.current_stream()
    arr = (EncChunk * max(len(chunks), 1))(*chunks) if len(chunks) else (EncChunk * 1)()
    rc = load().vtx_encoder_stitch(ctypes.c_void_p(chunk_out.data_ptr()), chunk_out.stride(0) * chunk_out.element_size(),
                                   chunk_out.stride(1) * chunk_out.element_size(), ctypes.c_void_p(dst.data_ptr()),
                                   dst.stride(0) * dst.element_size(), row_bytes, arr, len(chunks),
                                   ctypes.c_void_p(s.cuda_stream))
    _check(rc, "vtx_encoder_stitch")
    return dst


def read_device_error(stream: Optional[torch.cuda.Stream] = None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return int(load().vtx_read_device_error(ctypes.c_void_p(s.cuda_stream)))


# ---- reference masks and formats (the shapes voxtral.cpp builds) -----------

def causal_mask(n: int, device=None) -> torch.Tensor:
    """src/voxtral.cpp:2103-2111 fill_causal_mask -> F16 (:1801)."""
    m = torch.full((n, n), float("-inf"), device=device).triu(1)
    return m.to(torch.float16)


def window_mask(n: int, window: int = 750, device=None) -> torch.Tensor:
    """src/voxtral.cpp:2181-2188 chunk-local sliding causal mask -> F16."""
    qi = torch.arange(n, device=device)[:, None]
    kj = torch.arange(n, device=device)[None, :]
    allow = (kj <= qi) & (kj >= (qi - (window - 1)).clamp(min=0))
    return torch.where(allow, 0.0, float("-inf")).to(torch.float16)


def quantize_q8_0(x: torch.Tensor) -> torch.Tensor:
    """ggml's reference Q8_0 quantizer (quantize_row_q8_0_ref, the rule the
    reference's converter uses for Q8_0 tensors) over the last axis of a float
    tensor, on x's device: per 32 values d = amax/127 (stored as f16),
    q = round-half-away(x / d).  Returns uint8 with the last axis holding
    D/32 blocks of 34 bytes {f16 d; int8 qs[32]}.  A data-preparation helper
    for caches built outside vtx_kv_append (which quantizes on write)."""
    D = x.shape[-1]
    if D % QK8_0:
        raise VtxError(-3, "last axis must be a multiple of 32")
    xb = x.float().reshape(*x.shape[:-1], D // QK8_0, QK8_0)
    d = xb.abs().amax(dim=-1) / 127.0
    inv = torch.where(d != 0, 1.0 / d, torch.zeros_like(d))
    y = xb * inv.unsqueeze(-1)
    qs = (torch.sign(y) * torch.floor(y.abs() + 0.5)).to(torch.int8)
    out = torch.empty(*x.shape[:-1], D // QK8_0, Q8_0_BLOCK, dtype=torch.uint8, device=x.device)
    out[..., :2] = d.half().unsqueeze(-1).view(torch.uint8).reshape(*d.shape, 2)
    out[..., 2:] = qs.view(torch.uint8)
    return out.reshape(*x.shape[:-1], D // QK8_0 * Q8_0_BLOCK)


def _raw_tensor(ttype: int, ne, nb, ptr: int) -> VtxTensor:
    d = VtxTensor()
    d.type = ttype
    for i in range(4):
        d.ne[i] = ne[i] if i < len(ne) else 1
        d.nb[i] = nb[i] if i < len(nb) else (d.nb[i - 1] * d.ne[i - 1])
    d.data = ptr
    return d


def out_proj(attn: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor] = None,
             residual: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
             stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """vtx_attn_out_proj: out = residual + bias + f16(attn) @ w^T (f32 accumulate),
    the output projection after the attention node (src/voxtral.cpp:1612-1617,
    :1804-1809).  attn: (1, n, Hq, Dv) float32 as flash_attn_ext returns it,
    any strides, read in place, or float16 (flash_attn_ext with a float16
    `out`: the same rounding, done in the attention epilogue); or
    (1, n, R, h, Dv), the rank-major result of shard.head_split_prefill
    (head = r * h + j).  w: (N, Hq * Dv) float16;
    bias: (N,) float32 or None; residual: (n, N) float32 or None (it may be
    `out`).  Returns out (n, N) float32."""
    if attn.dtype not in (torch.float32, torch.float16) or w.dtype != torch.float16:
        raise VtxError(-2, "attn must be float32 or float16 and w float16")
    es = attn.element_size()
    if attn.dim() == 4:
        _, n, Hq, Dv = attn.shape
        head_nb, tok_nb = attn.stride(2) * es, attn.stride(1) * es
        head_block, block_nb = 0, 0
    elif attn.dim() == 5:
        _, n, R, h, Dv = attn.shape
        Hq = R * h
        head_nb, tok_nb = attn.stride(3) * es, attn.stride(1) * es
        head_block, block_nb = h, attn.stride(2) * es
    else:
        raise VtxError(-3, "attn must be (1, n, Hq, Dv) or (1, n, R, h, Dv)")
    if attn.shape[0] != 1 or attn.stride(-1) != 1:
        raise VtxError(-3, "one batch, unit-stride head dim")
    N, K = w.shape
    if out is None:
        out = torch.empty((n, N), dtype=torch.float32, device=attn.device)
    a = _raw_tensor(F32 if es == 4 else F16, [Dv, Hq, n, 1], [es, head_nb, tok_nb, tok_nb * n], attn.data_ptr())
    wd = _raw_tensor(F16, [K, N, 1, 1], [2, w.stride(0) * 2], w.data_ptr())
    yd = _raw_tensor(F32, [N, n, 1, 1], [4, out.stride(0) * 4], out.data_ptr())
    bd = _raw_tensor(F32, [N, 1, 1, 1], [4], bias.data_ptr()) if bias is not None else None
    rd = _raw_tensor(F32, [N, n, 1, 1], [4, residual.stride(0) * 4], residual.data_ptr()) \
        if residual is not None else None
    args = OutProjArgs()
    args.attn = ctypes.addressof(a)
    args.head_block, args.block_nb = head_block, block_nb
    args.w = ctypes.addressof(wd)
    args.bias = ctypes.addressof(bd) if bd is not None else None
    args.residual = ctypes.addressof(rd) if rd is not None else None
    args.dst = ctypes.addressof(yd)
    s = stream if stream is not None else torch.cuda.current_stream(attn.device)
    _check(load().vtx_attn_out_proj(ctypes.byref(args), ctypes.c_void_p(s.cuda_stream)), "vtx_attn_out_proj")
    return out
