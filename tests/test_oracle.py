"""CPU tests of the oracle (test infrastructure) against the committed golden
fixtures and hand-made known answers.  No GPU needed."""
import os

import numpy as np
import pytest

import oracle as O
from vtx_cases import assert_close, make_case, oracle_out

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def test_q8_0_matches_gguf_py():
    """Q8_0 block bytes == gguf-py 0.19.0 quantize (ggml quantize_row_q8_0_ref)."""
    z = np.load(os.path.join(GOLD, "q8_0_blocks.npz"))
    got = O.quantize_q8_0(z["x"])
    assert got.shape == z["blocks"].shape
    assert np.array_equal(got, z["blocks"])
    back = O.dequantize_q8_0(z["blocks"])
    d = z["blocks"].reshape(len(z["x"]), -1, 34)[..., :2].copy().view(np.float16).astype(np.float32)
    assert np.allclose(back, z["x"], atol=float(d.max()) * 0.5 + 1e-6)


def _golden_cases():
    z = np.load(os.path.join(GOLD, "attn_cases.npz"))
    names = sorted({k.split("/")[0] for k in z.files})
    return z, names


@pytest.mark.parametrize("name", _golden_cases()[1])
def test_oracle_vs_float64_golden(name):
    z, _ = _golden_cases()
    g = lambda s: z[f"{name}/{s}"]
    meta = g("meta")
    kv_type, scale, max_bias, softcap, causal, window = int(meta[0]), *meta[1:4], int(meta[4]), int(meta[5])
    mask = g("mask") if f"{name}/mask" in z.files else None
    out = g("out")
    f64 = O.flash_attn_ext(g("q"), g("k"), g("v"), mask, scale, max_bias, softcap, causal, window,
                           kv_type=kv_type, mode=O.MODE_FP64)
    # fp64 mode restates the same math in double: agreement to float32 output rounding
    np.testing.assert_allclose(f64, out, rtol=2e-6, atol=2e-7)
    gg = O.flash_attn_ext(g("q"), g("k"), g("v"), mask, scale, max_bias, softcap, causal, window,
                          kv_type=kv_type, mode=O.MODE_GGML)
    # ggml mode carries ggml's own roundings (half Q, half V accumulator, Q8_0 Q)
    assert_close(gg, out, f"{name} ggml-mode vs float64", atol=1e-2 if kv_type == O.Q8_0 else 4e-3)


def test_kat_uniform_v():
    """Every V row identical -> output equals that row, whatever the scores."""
    c = make_case(1, Hq=4, Hkv=2, n_q=5, n_kv=37, D=64, kv="f32")
    row = np.random.default_rng(3).standard_normal(64).astype(np.float32)
    c.bufs["v"][:] = row
    for mode in (O.MODE_GGML, O.MODE_FP64):
        out = oracle_out(c, mode)
        assert np.allclose(out, row, atol=1e-5)


def test_kat_one_hot_mask_selects_row():
    c = make_case(2, Hq=2, Hkv=1, n_q=3, n_kv=20, D=64, kv="f32", mask="random")
    c.mask[:] = -np.inf
    c.mask[0, 7] = 0
    c.mask[1, 0] = 0
    c.mask[2, 19] = 0
    out = oracle_out(c)
    v = c.v[0, 0]
    for i, j in enumerate([7, 0, 19]):
        assert np.allclose(out[0, i, :, :], v[j], atol=1e-6)


def test_kat_identical_keys_mean_of_v():
    c = make_case(3, Hq=2, Hkv=1, n_q=4, n_kv=33, D=128, kv="f32")
    c.bufs["k"][:] = c.bufs["k"][:, :1]
    mean_v = c.v[0, 0].astype(np.float64).mean(axis=0)          # Hkv = 1: both heads share it
    for mode in (O.MODE_GGML, O.MODE_FP64):
        out = oracle_out(c, mode)
        assert np.allclose(out[0], np.broadcast_to(mean_v, out[0].shape), atol=1e-5)


def test_fully_masked_row_is_zero():
    c = make_case(4, Hq=2, Hkv=1, n_q=3, n_kv=10, D=64, mask="random")
    c.mask[1, :] = -np.inf
    for mode in (O.MODE_GGML, O.MODE_FP64):
        assert np.all(oracle_out(c, mode)[:, 1] == 0)


@pytest.mark.parametrize("n", [1, 7, 33])
def test_causal_flag_equals_reference_mask(n):
    """params.causal reproduces fill_causal_mask (src/voxtral.cpp:2103-2111)."""
    a = make_case(5, Hq=4, Hkv=2, n_q=n, n_kv=n, D=64, mask="causal")
    b = make_case(5, Hq=4, Hkv=2, n_q=n, n_kv=n, D=64, causal=1)
    assert np.array_equal(oracle_out(a), oracle_out(b))


def test_window_flag_equals_reference_mask():
    """causal + window 750 reproduces the realtime encoder mask
    (src/voxtral.cpp:2181-2188), edges q-749 allowed and q-750 masked."""
    n = 800
    m = O.window_mask(n, 750)
    assert m[760, 760 - 749] == 0 and m[760, 760 - 750] == -np.inf and m[760, 761] == -np.inf
    a = make_case(6, Hq=1, Hkv=1, n_q=n, n_kv=n, D=64, mask="window", window=750, cache=False)
    b = make_case(6, Hq=1, Hkv=1, n_q=n, n_kv=n, D=64, causal=1, window=750, cache=False)
    assert np.array_equal(oracle_out(a), oracle_out(b))


def test_q8_0_k_quantizes_q_like_ggml():
    """With Q8_0 K the ggml path quantizes Q (int8 dot); fp64 does not.  The
    two differ by Q's quantization error but stay close."""
    c = make_case(7, Hq=4, Hkv=1, n_q=2, n_kv=50, D=128, kv="q8_0")
    assert_close(oracle_out(c), oracle_out(c, O.MODE_FP64), "q8_0 ggml vs fp64", atol=2e-2, rtol=5e-2)


def test_decode_batched_matches_single_calls():
    rng = np.random.default_rng(8)
    Hq, Hkv, D = 8, 2, 64
    lens = [5, 1, 40]
    q = rng.standard_normal((3, Hq, D)).astype(np.float32)
    ks = [rng.standard_normal((L, Hkv, D)).astype(np.float16) for L in lens]
    vs = [rng.standard_normal((L, Hkv, D)).astype(np.float16) for L in lens]
    out = O.decode_batched(q, ks, vs, lens, 0.125, O.F16, Hkv, ks[0].strides[0], ks[0].strides[1])
    for s in range(3):
        one = O.flash_attn_ext(q[s][None, :, None, :], ks[s].transpose(1, 0, 2)[None],
                               vs[s].transpose(1, 0, 2)[None], None, 0.125)
        assert np.array_equal(out[s], one[0, 0])


def test_torch_q8_0_quantizer_matches_ggml_rule_on_cpu():
    """vtx_attn.quantize_q8_0 (the bench's Q8_0 data path) equals the oracle's
    quantize_row_q8_0_ref byte for byte, zero blocks and ties included."""
    import torch
    import vtx_attn
    x = np.random.default_rng(11).standard_normal((64, 8, 128)).astype(np.float32)
    x[1, 2, :32] = 0.0
    x[2, 0, :32] = np.arange(32, dtype=np.float32) - 15.5          # exact halves after scaling
    got = vtx_attn.quantize_q8_0(torch.from_numpy(x)).numpy()
    assert np.array_equal(got, O.quantize_q8_0(x))


def test_parity_verdict_admits_ggml_drift_only():
    """The criterion used at the benchmark's sizes: a result at fp64 truth
    passes even where ggml mode itself drifts past ATOL, and so does one that
    follows ggml there (as the device does for a Q8_0 K, whose Q ggml
    quantises); a candidate off both by more than ATOL where ggml is exact
    fails, and so does one beyond ggml's drift plus ATOL."""
    f = np.linspace(-0.3, 0.3, 1000)
    g = f.copy()
    g[10] += 3e-3                                   # ggml's own drift from exact arithmetic
    assert O.parity_verdict(f.copy(), g, f)["ok"]
    assert O.parity_verdict(g.copy(), g, f)["ok"]
    bad = f.copy()
    bad[500] += 3e-3                                # off truth (|f| ~ 0) where ggml is exact
    v = O.parity_verdict(bad, g, f)
    assert not v["ok_vs_fp64"] and not v["ok_vs_ggml"] and not v["ok"]
    far = f.copy()
    far[10] -= 6e-3                                 # the other way from ggml, beyond its drift + ATOL
    assert not O.parity_verdict(far, g, f)["ok"]


def test_oracle_out_proj_fp64_is_exact_matmul():
    """The out-projection restatement: fp64 mode equals a float64 matmul plus
    bias and residual; ggml mode differs only by rounding the activations to
    f16 (ggml's vec_dot type for an F16 weight)."""
    rng = np.random.default_rng(21)
    a = rng.standard_normal((9, 256)).astype(np.float32)
    w = (rng.standard_normal((130, 256)) / 16).astype(np.float16)
    b = rng.standard_normal(130).astype(np.float32)
    r = rng.standard_normal((9, 130)).astype(np.float32)
    ref = a.astype(np.float64) @ w.astype(np.float64).T + b + r
    assert np.abs(O.out_proj(a, w, b, r, mode=O.MODE_FP64) - ref).max() < 1e-5
    a16 = a.astype(np.float16).astype(np.float64)
    ref16 = a16 @ w.astype(np.float64).T + b + r
    assert np.abs(O.out_proj(a, w, b, r) - ref16).max() < 1e-4
