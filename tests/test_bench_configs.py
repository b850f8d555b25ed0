"""GPU parity of the exact paths bench.py times, at the benchmark's own sizes.

* configs[1] encoder, as benched: 32 layers of f16 Q/K/V (1500 frames x 20
  heads x 64, ggml's permuted views, src/voxtral.cpp:1601-1605), f16 Q loaded
  by the TMA Q path, one vtx_flash_attn_ext call per layer with the bench's
  workspace and stream, captured in a CUDA graph and replayed; layers 0 and 31
  (all 20 heads) are compared with the oracle's flash_attn_ext.
* configs[4] batched decode at full shape: 256 streams with kv_len
  ~ U[512, 16384], GQA 32/8 x 128, f16 and Q8_0 caches built from N(0,1)
  values (Q8_0 by ggml's quantize_row_q8_0_ref rule); one call for all
  streams, a seeded sample of 12 streams checked against the oracle's batched
  decode.

Inputs come from bench.py's own generators, and the checks are bench.py's
own checkers, so what is tested is what is timed.  Criterion
(oracle.parity_verdict): within 2e-3 + 1e-2 |x| of the oracle's fp64 truth
everywhere, and of its ggml mode up to ggml's own per-element drift from
truth.  At these lengths ggml's half-precision V accumulator (F16 V) drifts
from exact arithmetic by up to ~3e-3 on its own, above the 2e-3 tolerance,
while the device (fp32 accumulate) stays within ~1e-4 of truth.
"""
import numpy as np
import pytest

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


def test_cfg1_encoder_as_benched():
    import bench
    import vtx_attn
    dev = torch.device("cuda", 0)
    L, D = bench.ENC["layers"], bench.ENC["D"]
    qkv = bench.make_encoder_inputs(1234, dev)
    out = torch.full((L, 1, bench.ENC["n"], bench.ENC["H"], D), float("nan"), device=dev)
    views = [bench.enc_views(qkv[l]) for l in range(L)]
    scale = 1.0 / D ** 0.5
    stream = torch.cuda.Stream(device=dev)
    ws = torch.empty(max(1, vtx_attn.workspace_bytes(*views[0], scale)), dtype=torch.uint8, device=dev)

    def step():
        for l in range(L):
            q, k, v = views[l]
            vtx_attn.flash_attn_ext(q, k, v, None, scale, out=out[l], workspace=ws, stream=stream)

    with torch.cuda.stream(stream):
        step()
    torch.cuda.synchronize()
    out.fill_(float("nan"))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step()
    graph.replay()
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()
    for l in (0, L - 1):
        r = bench.check_encoder_layer(qkv[l], out[l])
        assert r["ok"], f"layer {l}: {r}"


@pytest.mark.parametrize("kv", ["f16", "q8_0", "f32"])
def test_cfg4_decode_full_shape(kv):
    """configs[4] at its size, f16 and Q8_0 caches, and the reference's own
    F32 cache (src/voxtral.cpp:1126-1136, f32 arithmetic as ggml's CPU kernel)."""
    import bench
    import vtx_attn
    dev = torch.device("cuda", 0)
    q8 = kv == "q8_0"
    Hq, Hkv, D = bench.DEC["Hq"], bench.DEC["Hkv"], bench.DEC["D"]
    row = D // 32 * 34 if q8 else D * (4 if kv == "f32" else 2)
    lens, ks, vs, q = bench.make_decode_inputs(bench.DEC["n_seq"], "f32" if kv == "f32" else q8, 4321, 77, dev)
    assert lens.min() >= 512 and lens.max() <= 16384 and len(lens) == 256
    kvt = {"f16": vtx_attn.F16, "q8_0": vtx_attn.Q8_0, "f32": vtx_attn.F32}[kv]
    plan = vtx_attn.DecodeBatchPlan(ks, vs, torch.from_numpy(lens).to(dev), Hq, Hkv, D, kvt, Hkv * row, row,
                                    int(lens.max()), 1.0 / D ** 0.5)
    out = torch.full_like(q, float("nan"))
    plan(q, out)
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()
    r = bench.check_decode_rows(q, ks, vs, lens, out, kv, n_check=12, seed=3)
    assert r["ok"], f"{kv}: {r}"


def test_q8_0_device_quantizer_matches_ggml_rule():
    """The bench's device-side Q8_0 data (vtx_attn.quantize_q8_0) is byte for
    byte ggml's quantize_row_q8_0_ref (the oracle's restatement)."""
    import oracle as O
    import vtx_attn
    x = np.random.default_rng(9).standard_normal((300, 8, 128)).astype(np.float32)
    x[7, 3, :32] = 0.0
    got = vtx_attn.quantize_q8_0(torch.from_numpy(x).cuda()).cpu().numpy()
    assert np.array_equal(got, O.quantize_q8_0(x))
