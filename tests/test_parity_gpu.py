"""GPU parity: libvtx_fa.so (called through its C ABI) vs the CPU oracle's
ggml-mode restatement of ggml's CPU flash_attn_ext, on seeded inputs laid out
like voxtral.cpp's call sites (src/voxtral.cpp:1611 encoder, :1802 decoder).

Tolerance: |gpu - ggml| <= 2e-3 + 1e-2 * |ggml|.  Each
case also checks the GPU against the oracle's fp64 truth with the same bound.
"""
import numpy as np
import pytest

import oracle as O
from vtx_cases import assert_close, make_case, oracle_out, to_device

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module", autouse=True)
def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import vtx_attn
    vtx_attn.load()
    yield
    assert vtx_attn.read_device_error() == 0, "a kernel reported a device-side error"


def run_gpu(c):
    import vtx_attn
    q, k, v, m = to_device(c)
    kvt = O.Q8_0 if c.kv_type == O.Q8_0 else None
    out = vtx_attn.flash_attn_ext(q, k, v, m, c.scale, c.max_bias, c.softcap, causal=bool(c.causal),
                                  window=c.window, kv_type=kvt)
    torch.cuda.synchronize()
    return out.cpu().numpy()


def check(c, what):
    got = run_gpu(c)
    ref = oracle_out(c)
    assert_close(got, ref, what + " vs ggml-mode oracle")
    truth = oracle_out(c, O.MODE_FP64)
    if c.kv_type == O.Q8_0:
        # ggml quantizes Q to Q8_0 for a Q8_0 K (and so do the kernels); the
        # distance to fp64 truth is then bounded by ggml's own, not by 2e-3.
        own = float(np.max(np.abs(ref.astype(np.float64) - truth)))
        err = float(np.max(np.abs(got.astype(np.float64) - truth)))
        assert err <= 1.5 * own + 2e-3, f"{what}: gpu-vs-fp64 {err:.3e}, ggml-vs-fp64 {own:.3e}"
    else:
        assert_close(got, truth, what + " vs fp64")


# ---- BASELINE configs at parity-test sizes ---------------------------------

def test_cfg1_decode_f16():
    """decode step, 32/8 heads x 128, n_kv 1024, Q F32, K/V F16."""
    check(make_case(1, Hq=32, Hkv=8, n_q=1, n_kv=1024, D=128, kv="f16", n_ctx=8192), "cfg1 decode")


def test_cfg2_encoder_bidir_full_length():
    """configs[1] geometry (1500 frames, head_dim 64, no mask), 4 of 20 heads."""
    check(make_case(2, B=1, Hq=4, Hkv=4, n_q=1500, n_kv=1500, D=64, cache=False), "cfg2 encoder")


def test_cfg2_encoder_f16_q():
    check(make_case(3, Hq=2, Hkv=2, n_q=700, n_kv=700, D=64, q16=True, cache=False), "cfg2 f16 q")


@pytest.mark.parametrize("how", ["mask", "flags"])
def test_cfg4_encoder_window(how):
    """configs[3] realtime encoder: causal + 750 window over a 1500 chunk."""
    if how == "mask":
        c = make_case(4, Hq=4, Hkv=4, n_q=1500, n_kv=1500, D=64, cache=False, mask="window", window=750)
    else:
        c = make_case(4, Hq=4, Hkv=4, n_q=1500, n_kv=1500, D=64, cache=False, causal=1, window=750)
    check(c, f"cfg4 window ({how})")


@pytest.mark.parametrize("how", ["mask", "flags"])
def test_cfg3_decoder_prefill(how):
    """decoder prefill 391 tokens, GQA 32/8, head_dim 128, causal."""
    kw = {"mask": "causal"} if how == "mask" else {"causal": 1}
    check(make_case(5, Hq=32, Hkv=8, n_q=391, n_kv=391, D=128, n_ctx=8192, **kw), f"cfg3 prefill ({how})")


def test_cfg4_decode_q8_0():
    check(make_case(6, Hq=32, Hkv=8, n_q=1, n_kv=1777, D=128, kv="q8_0"), "cfg4 q8_0 decode")


def test_reference_f32_cache_decode():
    """The reference's own KV cache is F32 (src/voxtral.cpp:1126-1136)."""
    check(make_case(7, Hq=32, Hkv=8, n_q=1, n_kv=400, D=128, kv="f32", n_ctx=8192), "f32 cache decode")


def test_reference_f32_cache_prefill():
    check(make_case(8, Hq=32, Hkv=8, n_q=200, n_kv=200, D=128, kv="f32", mask="causal"), "f32 cache prefill")


def test_q8_0_prefill():
    check(make_case(9, Hq=8, Hkv=2, n_q=150, n_kv=300, D=128, kv="q8_0", causal=1), "q8_0 prefill")


# ---- causal launches of more than one wave (longest-first CTA order) ----------

def test_realtime_encoder_chunk_multi_wave():
    """The realtime encoder's chunk (1500 tokens, 32 heads x 64, causal +
    window 750): 192 CTAs, more than one wave, so the CTAs run longest first."""
    check(make_case(12, Hq=32, Hkv=32, n_q=1500, n_kv=1500, D=64, causal=1, window=750, cache=False),
          "realtime encoder chunk")


def test_encoder_chunk_window_single_wave():
    """The window-750 chunk with 20 heads: 120 CTAs of two Q tiles, one wave,
    so the causal instantiation keeps the head-major grid while each tile of
    a pair runs over its own key tiles."""
    check(make_case(14, Hq=20, Hkv=20, n_q=1500, n_kv=1500, D=64, causal=1, window=750, cache=False),
          "encoder chunk, 20 heads")


def test_decoder_prefill_multi_wave():
    """A longer decoder prefill (1200 tokens, GQA 32/8 x 128, causal): 152 CTAs."""
    check(make_case(13, Hq=32, Hkv=8, n_q=1200, n_kv=1200, D=128, causal=1, n_ctx=8192), "prefill 1200 tokens")


# ---- edge cases --------------------------------------------------------------

@pytest.mark.parametrize("n", [1, 2, 31, 33, 127, 129, 257])
def test_ragged_lengths_prefill(n):
    check(make_case(100 + n, Hq=4, Hkv=1, n_q=n, n_kv=n, D=64, causal=1), f"ragged n={n}")


@pytest.mark.parametrize("n_kv", [1, 63, 64, 65, 1501])
def test_ragged_lengths_decode(n_kv):
    check(make_case(200 + n_kv, Hq=8, Hkv=2, n_q=1, n_kv=n_kv, D=128), f"decode n_kv={n_kv}")


@pytest.mark.parametrize("kv", ["f16", "f32", "q8_0"])
@pytest.mark.parametrize("D", [64, 128])
def test_dtypes_short_chunk(kv, D):
    check(make_case(300 + D, Hq=8, Hkv=2, n_q=5, n_kv=97, D=D, kv=kv), f"{kv} D={D} n_q=5")


def test_gqa_ratio_1_d128():
    check(make_case(10, Hq=4, Hkv=4, n_q=300, n_kv=300, D=128, causal=1), "gqa1 d128")


def test_gqa_ratio_4_d64():
    check(make_case(11, Hq=8, Hkv=2, n_q=300, n_kv=300, D=64, causal=1, window=100), "gqa4 d64 window")


def test_batch_broadcast_and_kv_offset():
    """B=2, n_kv > n_q (prefill appended after a prefix, causal bottom-right)."""
    check(make_case(12, B=2, Hq=8, Hkv=2, n_q=70, n_kv=170, D=128, causal=1), "b2 offset causal")


def test_random_mask_alibi_softcap():
    check(make_case(13, Hq=6, Hkv=3, n_q=9, n_kv=140, D=64, kv="f32", mask="random",
                    max_bias=8.0, softcap=30.0), "alibi+softcap split path")
    check(make_case(14, Hq=8, Hkv=2, n_q=100, n_kv=140, D=64, mask="random", max_bias=8.0,
                    softcap=30.0), "alibi+softcap prefill path")


def test_fully_masked_rows_are_zero():
    c = make_case(15, Hq=4, Hkv=1, n_q=64, n_kv=64, D=64, mask="random")
    c.mask[:5, :] = -np.inf
    got = run_gpu(c)
    assert np.all(got[:, :5] == 0.0)
    assert_close(got, oracle_out(c), "masked rows")


def test_n_kv_zero_gives_zeros():
    import vtx_attn
    q = torch.randn(1, 4, 3, 64, device="cuda")
    k = torch.zeros(1, 1, 0, 64, device="cuda", dtype=torch.float16)
    out = vtx_attn.flash_attn_ext(q, k, k, None, 0.125)
    torch.cuda.synchronize()
    assert torch.all(out == 0)


# ---- ragged batched decode ----------------------------------------------------

@pytest.mark.parametrize("kv,G", [("f16", 4), ("q8_0", 4), ("f32", 4), ("f16", 1), ("f16", 2), ("q8_0", 2)])
def test_decode_batched_ragged(kv, G):
    """Ragged batched decode; G < 4 leaves rows of the combine kernel's row
    space idle, which its launch grid has to cover all the same."""
    import vtx_attn
    rng = np.random.default_rng(21 + G)
    n_seq, Hkv, D = 12, 8, 128
    Hq = G * Hkv
    lens = rng.integers(1, 3000, n_seq).astype(np.int32)
    lens[0] = 1
    qn = rng.standard_normal((n_seq, Hq, D)).astype(np.float32)
    kvt = {"f16": O.F16, "f32": O.F32, "q8_0": O.Q8_0}[kv]
    ks, vs = [], []
    for L in lens:
        kf = rng.standard_normal((int(L), Hkv, D)).astype(np.float32)
        vf = rng.standard_normal((int(L), Hkv, D)).astype(np.float32)
        if kv == "f16":
            ks.append(kf.astype(np.float16)); vs.append(vf.astype(np.float16))
        elif kv == "f32":
            ks.append(kf); vs.append(vf)
        else:
            ks.append(O.quantize_q8_0(kf)); vs.append(O.quantize_q8_0(vf))
    row = ks[0].strides[0]
    nb2 = ks[0].strides[1]
    ref = O.decode_batched(qn, ks, vs, lens, 1 / np.sqrt(D), kvt, Hkv, row, nb2)
    kt = [torch.from_numpy(a).cuda() for a in ks]
    vt = [torch.from_numpy(a).cuda() for a in vs]
    plan = vtx_attn.DecodeBatchPlan(kt, vt, torch.from_numpy(lens).cuda(), Hq, Hkv, D, kvt, row, nb2,
                                    int(lens.max()), float(1 / np.sqrt(D)))
    got = plan(torch.from_numpy(qn).cuda())
    torch.cuda.synchronize()
    assert_close(got.cpu().numpy(), ref, f"batched decode {kv}")


@pytest.mark.parametrize("Hkv,G", [(2, 4), (4, 4), (8, 1), (8, 3), (16, 2)])
def test_decode_batched_q8_0_head_groups(Hkv, G):
    """Q8_0 streaming decode with fewer than 8 KV heads per token row (one CTA
    copies 2 or 4 heads' slices), with 16 (a CTA's 8 heads are half a token
    row, so rows are copied one by one), and with GQA groups smaller than 4
    (unused head columns of the score tile), lengths that need several splits."""
    import vtx_attn
    rng = np.random.default_rng(30 + Hkv + 10 * G)
    n_seq, D = 5, 128
    Hq = G * Hkv
    lens = np.array([1, 17, 1024, 2049, 4500], dtype=np.int32)
    qn = rng.standard_normal((n_seq, Hq, D)).astype(np.float32)
    ks = [O.quantize_q8_0(rng.standard_normal((int(L), Hkv, D)).astype(np.float32)) for L in lens]
    vs = [O.quantize_q8_0(rng.standard_normal((int(L), Hkv, D)).astype(np.float32)) for L in lens]
    row, nb2 = ks[0].strides[0], ks[0].strides[1]
    ref = O.decode_batched(qn, ks, vs, lens, 1 / np.sqrt(D), O.Q8_0, Hkv, row, nb2)
    plan = vtx_attn.DecodeBatchPlan([torch.from_numpy(a).cuda() for a in ks], [torch.from_numpy(a).cuda() for a in vs],
                                    torch.from_numpy(lens).cuda(), Hq, Hkv, D, O.Q8_0, row, nb2, int(lens.max()),
                                    float(1 / np.sqrt(D)))
    got = plan(torch.from_numpy(qn).cuda())
    torch.cuda.synchronize()
    assert vtx_attn.read_device_error() == 0
    assert_close(got.cpu().numpy(), ref, f"batched q8_0 decode Hkv={Hkv} G={G}")


@pytest.mark.parametrize("kv", ["q8_0", "f16"])
def test_decode_batched_one_stream_many_splits(kv):
    """Batch 1 over a long ring (the decode step's shape): the key range is cut
    into more than 32 splits, so the partials go through the 512-thread
    combine kernel; lengths 7300 and a short 40 in a ring planned for 8192."""
    import vtx_attn
    rng = np.random.default_rng(55)
    Hq, Hkv, D, W = 32, 8, 128, 8192
    kvt = O.Q8_0 if kv == "q8_0" else O.F16
    for L in (7300, 40):
        qn = rng.standard_normal((1, Hq, D)).astype(np.float32)
        kf = rng.standard_normal((W, Hkv, D)).astype(np.float32)
        vf = rng.standard_normal((W, Hkv, D)).astype(np.float32)
        if kv == "q8_0":
            kb, vb = O.quantize_q8_0(kf), O.quantize_q8_0(vf)
        else:
            kb, vb = kf.astype(np.float16), vf.astype(np.float16)
        lens = np.array([L], dtype=np.int32)
        row, nb2 = kb.strides[0], kb.strides[1]
        ref = O.decode_batched(qn, [kb[:L]], [vb[:L]], lens, 1 / np.sqrt(D), kvt, Hkv, row, nb2)
        plan = vtx_attn.DecodeBatchPlan([torch.from_numpy(kb).cuda()], [torch.from_numpy(vb).cuda()],
                                        torch.from_numpy(lens).cuda(), Hq, Hkv, D, kvt, row, nb2, W,
                                        float(1 / np.sqrt(D)))
        got = plan(torch.from_numpy(qn).cuda())
        torch.cuda.synchronize()
        assert vtx_attn.read_device_error() == 0
        assert_close(got.cpu().numpy(), ref, f"one-stream {kv} decode, {L} keys in a {W}-row ring")


@pytest.mark.parametrize("kv", ["f16", "q8_0"])
def test_decode_batched_empty_streams(kv):
    """Streams with no keys yet (kv_len 0) among ragged ones: their rows come
    out zero, as ggml's S = 0 gives, and the others are unaffected."""
    import vtx_attn
    rng = np.random.default_rng(77)
    Hq, Hkv, D = 32, 8, 128
    kvt = O.Q8_0 if kv == "q8_0" else O.F16
    lens = np.array([0, 5, 0, 1300, 0], dtype=np.int32)
    qn = rng.standard_normal((len(lens), Hq, D)).astype(np.float32)
    ks, vs = [], []
    for L in lens:
        kf = rng.standard_normal((max(int(L), 1), Hkv, D)).astype(np.float32)
        vf = rng.standard_normal((max(int(L), 1), Hkv, D)).astype(np.float32)
        if kv == "q8_0":
            ks.append(O.quantize_q8_0(kf)); vs.append(O.quantize_q8_0(vf))
        else:
            ks.append(kf.astype(np.float16)); vs.append(vf.astype(np.float16))
    row, nb2 = ks[0].strides[0], ks[0].strides[1]
    ref = O.decode_batched(qn, ks, vs, lens, 1 / np.sqrt(D), kvt, Hkv, row, nb2)
    plan = vtx_attn.DecodeBatchPlan([torch.from_numpy(a).cuda() for a in ks], [torch.from_numpy(a).cuda() for a in vs],
                                    torch.from_numpy(lens).cuda(), Hq, Hkv, D, kvt, row, nb2, int(lens.max()),
                                    float(1 / np.sqrt(D)))
    got = plan(torch.from_numpy(qn).cuda())
    torch.cuda.synchronize()
    assert vtx_attn.read_device_error() == 0
    got = got.cpu().numpy()
    assert not got[lens == 0].any()
    assert_close(got, ref, f"batched {kv} decode with empty streams")


# ---- error paths through the C ABI ---------------------------------------------

def test_errors_are_status_codes():
    import vtx_attn
    q = torch.randn(1, 4, 8, 96, device="cuda")        # head_dim 96 unsupported
    k = torch.randn(1, 1, 8, 96, device="cuda", dtype=torch.float16)
    with pytest.raises(vtx_attn.VtxError) as e:
        vtx_attn.flash_attn_ext(q, k, k, None, 0.1)
    assert e.value.status == -3 or e.value.status == -5
    q = torch.randn(1, 3, 8, 64, device="cuda")         # Hq % Hkv != 0
    k = torch.randn(1, 2, 8, 64, device="cuda", dtype=torch.float16)
    with pytest.raises(vtx_attn.VtxError):
        vtx_attn.flash_attn_ext(q, k, k, None, 0.1)
