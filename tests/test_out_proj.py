"""GPU parity of vtx_attn_out_proj, the output projection that consumes the
attention node's result (src/voxtral.cpp:1612-1617 encoder: ggml_cont +
mul_mat(attn_o_weight) + attn_o_bias + residual; :1804-1809 decoder: the
same without the bias), as one tcgen05 GEMM that reads the attention's F32
output in place.

Compared with the oracle's restatement of ggml's CPU mul_mat for an F16
weight (activations rounded to f16, f32 accumulation) and its fp64 mode,
under oracle.parity_verdict.  Cases: the Whisper-large encoder shape of
configs[1] (1500 tokens, 20 x 64 -> 1280, with bias), the decoder prefill
of configs[2] (391 tokens, 32 x 128 -> 3072, residual updated in place),
ragged small shapes (1 and 7 tokens, 200 outputs), the rank-major layout a
KV-head-split prefill gathers (bit-identical to the contiguous layout), and
attention chained into the projection against the oracle's attention
followed by its matmul.
"""
import numpy as np
import pytest

import oracle as O

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


def _case(seed, n, Hq, Dv, N, bias=True, residual=True):
    rng = np.random.default_rng(seed)
    a = (rng.standard_normal((n, Hq, Dv)) * 0.3).astype(np.float32)
    w = (rng.standard_normal((N, Hq * Dv)) / np.sqrt(Hq * Dv)).astype(np.float16)
    b = rng.standard_normal(N).astype(np.float32) if bias else None
    r = rng.standard_normal((n, N)).astype(np.float32) if residual else None
    return a, w, b, r


def _check(got, a, w, b, r, what):
    flat = a.reshape(a.shape[0], -1)
    v = O.parity_verdict(got, O.out_proj(flat, w, b, r), O.out_proj(flat, w, b, r, mode=O.MODE_FP64))
    assert v["ok"], f"{what}: {v}"


@pytest.mark.parametrize("n,Hq,Dv,N,bias,inplace", [
    (1500, 20, 64, 1280, True, False),     # configs[1] encoder (Whisper-large): attn_o_weight + attn_o_bias
    (391, 32, 128, 3072, False, True),     # configs[2] decoder prefill: x = residual + W_o attn, in place
    (1, 32, 128, 3072, False, False),      # one decode token
    (7, 2, 64, 200, True, False),          # ragged: 7 tokens, 200 outputs (a partial N tile)
    (300, 20, 64, 1280, False, False),     # no bias, no residual
])
def test_out_proj(n, Hq, Dv, N, bias, inplace):
    import vtx_attn
    a, w, b, r = _case(n + N, n, Hq, Dv, N, bias=bias, residual=inplace or bias)
    ta = torch.from_numpy(a).cuda().unsqueeze(0)                        # (1, n, Hq, Dv)
    tw = torch.from_numpy(w).cuda()
    tb = torch.from_numpy(b).cuda() if b is not None else None
    tr = torch.from_numpy(r).cuda() if r is not None else None
    if inplace:
        out = vtx_attn.out_proj(ta, tw, tb, residual=tr, out=tr)
    else:
        out = vtx_attn.out_proj(ta, tw, tb, residual=tr, out=torch.full((n, N), float("nan"), device="cuda"))
    torch.cuda.synchronize()
    _check(out.cpu().numpy(), a, w, b, r, f"out_proj n={n} K={Hq * Dv} N={N}")


def test_out_proj_reads_a_strided_attention_output():
    """The attention output as a permuted view with padded rows: read in
    place, identical to the contiguous copy."""
    import vtx_attn
    a, w, b, r = _case(3, 257, 8, 128, 512)
    base = torch.zeros((257, 8, 136), device="cuda")                    # rows padded to 136 floats
    base[:, :, :128] = torch.from_numpy(a).cuda()
    view = base[:, :, :128].unsqueeze(0)
    tw, tb, tr = (torch.from_numpy(x).cuda() for x in (w, b, r))
    got = vtx_attn.out_proj(view, tw, tb, tr)
    ref = vtx_attn.out_proj(view.contiguous(), tw, tb, tr)
    torch.cuda.synchronize()
    assert torch.equal(got, ref)
    _check(got.cpu().numpy(), a, w, b, r, "strided attention output")


def test_out_proj_rank_major_head_blocks():
    """The all-gathered result of a KV-head-split prefill, (1, n, R, h, Dv)
    with rank blocks at their own stride, projects bit-identically to the
    contiguous (1, n, Hq, Dv) layout."""
    import vtx_attn
    R, h, Dv, n, N = 4, 8, 128, 100, 3072
    a, w, b, r = _case(5, n, R * h, Dv, N, bias=False)
    blocks = torch.from_numpy(a.reshape(n, R, h, Dv).transpose(1, 0, 2, 3).copy()).cuda()   # (R, n, h, Dv)
    rank_major = blocks.unsqueeze(0).permute(0, 2, 1, 3, 4)             # (1, n, R, h, Dv), a view
    tw, tr = torch.from_numpy(w).cuda(), torch.from_numpy(r).cuda()
    got = vtx_attn.out_proj(rank_major, tw, None, tr)
    ref = vtx_attn.out_proj(torch.from_numpy(a).cuda().unsqueeze(0), tw, None, tr)
    torch.cuda.synchronize()
    assert torch.equal(got, ref)


def test_attention_then_out_proj_matches_oracle_chain():
    """Encoder-style attention (f16 Q/K/V, 600 tokens, 20 heads x 64) fed
    straight into the projection, against the oracle's attention followed by
    its matmul on the oracle's own attention output."""
    import vtx_attn
    rng = np.random.default_rng(8)
    n, H, D, N = 600, 20, 64, 1280
    q, k, v = (rng.standard_normal((n, H, D)).astype(np.float16) for _ in range(3))
    w = (rng.standard_normal((N, H * D)) / np.sqrt(H * D)).astype(np.float16)
    bias = rng.standard_normal(N).astype(np.float32)
    res = rng.standard_normal((n, N)).astype(np.float32)
    tv = lambda x: torch.from_numpy(x).cuda().permute(1, 0, 2).unsqueeze(0)
    attn = vtx_attn.flash_attn_ext(tv(q), tv(k), tv(v), None, D ** -0.5)            # (1, n, H, D)
    got = vtx_attn.out_proj(attn, torch.from_numpy(w).cuda(), torch.from_numpy(bias).cuda(),
                            torch.from_numpy(res).cuda())
    torch.cuda.synchronize()
    view = lambda x: x.transpose(1, 0, 2)[None]
    att_g = O.flash_attn_ext(view(q), view(k), view(v), None, D ** -0.5)[0].reshape(n, H * D)
    att_f = O.flash_attn_ext(view(q), view(k), view(v), None, D ** -0.5, mode=O.MODE_FP64)[0].reshape(n, H * D)
    v_ = O.parity_verdict(got.cpu().numpy(), O.out_proj(att_g, w, bias, res),
                          O.out_proj(att_f, w, bias, res, mode=O.MODE_FP64))
    assert v_["ok"], v_


@pytest.mark.parametrize("n,Hq,Dv,N", [(1500, 20, 64, 1280), (391, 32, 128, 3072), (7, 2, 64, 200)])
def test_out_proj_f16_attention_is_bit_identical(n, Hq, Dv, N):
    """An F16 attention output (the rounding ggml applies to the activations,
    done once upstream) projects bit-identically to the F32 output the
    kernel rounds itself, and so meets the same parity bar."""
    import vtx_attn
    a, w, b, r = _case(11 + n, n, Hq, Dv, N)
    ta = torch.from_numpy(a).cuda().unsqueeze(0)
    tw, tb, tr = (torch.from_numpy(x).cuda() for x in (w, b, r))
    ref = vtx_attn.out_proj(ta, tw, tb, tr)
    got = vtx_attn.out_proj(ta.half(), tw, tb, tr)
    torch.cuda.synchronize()
    assert torch.equal(got, ref)
    _check(got.cpu().numpy(), a, w, b, r, f"f16 attention n={n}")


@pytest.mark.parametrize("shape", ["encoder", "decoder_prefill"])
def test_attention_f16_result_is_the_rounded_f32_result(shape):
    """vtx_flash_attn_ext with an F16 dst writes exactly the F32 result
    rounded to nearest even (configs[1] encoder: f16 Q/K/V, 1500 x 20 x 64;
    configs[2] decoder prefill: F32 Q, causal GQA 32/8 x 128, 391 tokens), and
    the projection of it equals the projection of the F32 result bit for
    bit."""
    import vtx_attn
    rng = np.random.default_rng(21)
    if shape == "encoder":
        n, Hq, Hkv, D, causal, qdt, N = 1500, 20, 20, 64, False, np.float16, 1280
    else:
        n, Hq, Hkv, D, causal, qdt, N = 391, 32, 8, 128, True, np.float32, 3072
    q = torch.from_numpy(rng.standard_normal((1, Hq, n, D)).astype(qdt)).cuda()
    k = torch.from_numpy(rng.standard_normal((1, Hkv, n, D)).astype(np.float16)).cuda()
    v = torch.from_numpy(rng.standard_normal((1, Hkv, n, D)).astype(np.float16)).cuda()
    o32 = vtx_attn.flash_attn_ext(q, k, v, None, D ** -0.5, causal=causal)
    o16 = vtx_attn.flash_attn_ext(q, k, v, None, D ** -0.5, causal=causal,
                                  out=torch.empty(o32.shape, dtype=torch.float16, device="cuda"))
    w = torch.from_numpy((rng.standard_normal((N, Hq * D)) / np.sqrt(Hq * D)).astype(np.float16)).cuda()
    p32 = vtx_attn.out_proj(o32, w)
    p16 = vtx_attn.out_proj(o16, w)
    torch.cuda.synchronize()
    assert torch.equal(o16, o32.half())
    assert torch.equal(p16, p32)


def test_attention_f16_result_rejected_off_the_tensor_core_path():
    """A decode call (one query row) has no F16 result: VTX_ERR_TYPE."""
    import vtx_attn
    q = torch.randn((1, 32, 1, 128), device="cuda")
    k = torch.randn((1, 8, 64, 128), device="cuda").half()
    with pytest.raises(vtx_attn.VtxError) as e:
        vtx_attn.flash_attn_ext(q, k, k, None, 128 ** -0.5, out=torch.empty((1, 1, 32, 128), device="cuda").half())
    assert e.value.status == -2
