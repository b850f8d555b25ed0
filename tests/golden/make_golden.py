"""Generate the committed golden fixtures under tests/golden/.

Run from the repository root (needs the gguf-py package, version 0.19.0 here):
    python tests/golden/make_golden.py

Two kinds of pins, both independent of this repository's oracle and kernels:

* ``q8_0_blocks.npz`` — float32 rows and their Q8_0 bytes produced by
  gguf-py's ``gguf.quants.quantize(..., GGMLQuantizationType.Q8_0)``, the
  Python port of ggml's ``quantize_row_q8_0_ref``.  Q8_0 is the block format
  the KV cache variants use (34-byte blocks: half scale + 32 int8).
* ``attn_cases.npz`` — small attention problems at voxtral.cpp's geometries
  (encoder bidirectional and 750-window style masks, decoder causal GQA
  prefill, single-token decode, Q8_0 KV, ALiBi + softcap) with outputs
  computed by a straightforward float64 numpy softmax-attention.  These pin
  the oracle's fp64 mode exactly and its ggml mode within tolerance.
"""
from __future__ import annotations

import os

import numpy as np
from gguf import GGMLQuantizationType, quants

HERE = os.path.dirname(os.path.abspath(__file__))


def q8_0_fixture(rng: np.random.Generator) -> dict:
    rows = [
        rng.standard_normal((64, 128)).astype(np.float32),
        (rng.standard_normal((16, 128)) * 1e-3).astype(np.float32),
        (rng.standard_normal((16, 128)) * 300.0).astype(np.float32),
        np.zeros((2, 128), np.float32),
    ]
    # rows whose scaled values land on .5 ties (127 * k / 254 patterns)
    ties = np.tile(np.arange(-16, 16, dtype=np.float32) + 0.5, (4, 4)) / 15.5 * 127.0
    rows.append(ties.astype(np.float32))
    x = np.concatenate(rows, axis=0)
    b = quants.quantize(x, GGMLQuantizationType.Q8_0)
    return {"x": x, "blocks": np.asarray(b, dtype=np.uint8)}


def dequant_q8_0(b: np.ndarray) -> np.ndarray:
    blk = b.reshape(b.shape[:-1] + (-1, 34))
    d = blk[..., :2].copy().view(np.float16).astype(np.float64)
    qs = blk[..., 2:].view(np.int8).astype(np.float64)
    return (d * qs).reshape(b.shape[:-1] + (-1,))


def attn_f64(q, k, v, mask, scale, max_bias=0.0, softcap=0.0, causal=0, window=0):
    """q (B,Hq,nq,D) k/v (B,Hkv,nkv,D) float64; mask (nq,nkv) or None.
    Returns (B, nq, Hq, Dv) like ggml's permuted dst."""
    B, Hq, nq, _ = q.shape
    Hkv, nkv = k.shape[1], k.shape[2]
    G = Hq // Hkv
    n_head_log2 = 1 << int(np.floor(np.log2(Hq)))
    m0 = 2.0 ** (-max_bias / n_head_log2)
    m1 = 2.0 ** (-(max_bias / 2.0) / n_head_log2)
    out = np.zeros((B, nq, Hq, v.shape[-1]))
    qi = np.arange(nq)[:, None] + (nkv - nq)
    kj = np.arange(nkv)[None, :]
    struct = np.zeros((nq, nkv))
    if causal:
        struct[kj > qi] = -np.inf
        if window:
            struct[kj < qi - (window - 1)] = -np.inf
    for b in range(B):
        for h in range(Hq):
            slope = 1.0
            if max_bias > 0:
                slope = m0 ** (h + 1) if h < n_head_log2 else m1 ** (2 * (h - n_head_log2) + 1)
            s = q[b, h] @ k[b, h // G].T
            if softcap:
                s = softcap * np.tanh(s * (scale / softcap))
            else:
                s = s * scale
            s = s + struct
            if mask is not None:
                s = s + slope * mask
            mx = s.max(axis=1, keepdims=True)
            w = np.where(np.isneginf(s), 0.0, np.exp(s - np.where(np.isneginf(mx), 0.0, mx)))
            den = w.sum(axis=1, keepdims=True)
            o = (w @ v[b, h // G]) / np.where(den == 0, 1.0, den)
            out[b, :, h, :] = o
    return out


def main() -> None:
    rng = np.random.default_rng(20261201)
    np.savez_compressed(os.path.join(HERE, "q8_0_blocks.npz"), **q8_0_fixture(rng))

    cases = {}

    def add(name, B, Hq, Hkv, nq, nkv, D, kv="f16", mask=None, **kw):
        q = rng.standard_normal((B, Hq, nq, D)).astype(np.float32)
        kf = rng.standard_normal((B, Hkv, nkv, D)).astype(np.float32)
        vf = rng.standard_normal((B, Hkv, nkv, D)).astype(np.float32)
        if kv == "f16":
            k, v = kf.astype(np.float16), vf.astype(np.float16)
            k64, v64 = k.astype(np.float64), v.astype(np.float64)
        elif kv == "f32":
            k, v = kf, vf
            k64, v64 = k.astype(np.float64), v.astype(np.float64)
        else:
            k = np.asarray(quants.quantize(kf, GGMLQuantizationType.Q8_0), dtype=np.uint8)
            v = np.asarray(quants.quantize(vf, GGMLQuantizationType.Q8_0), dtype=np.uint8)
            k64, v64 = dequant_q8_0(k), dequant_q8_0(v)
        m = None
        if mask == "causal":
            m = np.zeros((nq, nkv), np.float32)
            m[np.arange(nq)[:, None] + (nkv - nq) < np.arange(nkv)[None, :]] = -np.inf
            m = m.astype(np.float16)
        elif mask == "random":
            m = (rng.standard_normal((nq, nkv)) * 2).astype(np.float16)
            m[rng.random((nq, nkv)) < 0.2] = -np.inf
        scale = kw.pop("scale", 1.0 / np.sqrt(D))
        o = attn_f64(q.astype(np.float64), k64, v64,
                     None if m is None else m.astype(np.float64), scale, **kw)
        pre = name + "/"
        cases[pre + "q"], cases[pre + "k"], cases[pre + "v"] = q, k, v
        if m is not None:
            cases[pre + "mask"] = m
        cases[pre + "out"] = o
        cases[pre + "meta"] = np.array([
            {"f16": 1, "f32": 0, "q8_0": 8}[kv], scale, kw.get("max_bias", 0.0),
            kw.get("softcap", 0.0), kw.get("causal", 0), kw.get("window", 0)], np.float64)

    add("enc_bidir", 1, 4, 4, 37, 37, 64)
    add("enc_window", 1, 4, 4, 40, 40, 64, causal=1, window=7)
    add("dec_prefill_causal_mask", 1, 4, 1, 33, 33, 128, mask="causal")
    add("dec_prefill_causal_flag", 1, 4, 2, 19, 27, 128, causal=1)
    add("decode_f16", 1, 8, 2, 1, 97, 128)
    add("decode_q8_0", 1, 8, 2, 1, 70, 128, kv="q8_0")
    add("decode_f32", 2, 8, 2, 1, 45, 64, kv="f32")
    add("random_mask", 1, 4, 2, 9, 61, 64, mask="random")
    add("alibi_softcap", 1, 6, 3, 5, 40, 64, kv="f32", max_bias=8.0, softcap=30.0, mask="random")
    np.savez_compressed(os.path.join(HERE, "attn_cases.npz"), **cases)


if __name__ == "__main__":
    main()
