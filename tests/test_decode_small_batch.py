"""GPU parity of the batched Q8_0 decode at the split plans of small
batches: the decode node of src/voxtral.cpp:1802 over a Q8_0 cache with 8 KV
heads (voxtral's decoder), the realtime model's decode step.  The Q8_0
streaming kernel splits a stream's keys for about one CTA per SM, and
fa_combine_kernel merges the splits (one load round, splits folded online).

Cases: one stream over the realtime model's 7300-key cache (115 splits of
64 keys), a stream with one key, streams whose keys fit a few splits or one
split, the full 8192-key window, a mixed batch, and a smaller ring with
fewer, longer splits; every output row is compared with the oracle's batched
decode (ggml mode and fp64), and no row is left unwritten (NaN-filled
outputs before the call).
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


def _run(lens, max_len, seed):
    import vtx_attn
    Hq, Hkv, D = 32, 8, 128
    row = D // 32 * 34
    rng = np.random.default_rng(seed)
    ks = [O.quantize_q8_0(rng.standard_normal((int(L), Hkv, D)).astype(np.float32)) for L in lens]
    vs = [O.quantize_q8_0(rng.standard_normal((int(L), Hkv, D)).astype(np.float32)) for L in lens]
    q = rng.standard_normal((len(lens), Hq, D)).astype(np.float32)
    lens = np.asarray(lens, dtype=np.int32)
    plan = vtx_attn.DecodeBatchPlan([torch.from_numpy(x).cuda() for x in ks], [torch.from_numpy(x).cuda() for x in vs],
                                    torch.from_numpy(lens).cuda(), Hq, Hkv, D, vtx_attn.Q8_0, Hkv * row, row, max_len,
                                    D ** -0.5)
    out = torch.full((len(lens), Hq, D), float("nan"), device="cuda")
    plan(torch.from_numpy(q).cuda(), out)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    assert np.all(np.isfinite(got)), "rows left unwritten"
    args = (q, ks, vs, lens, D ** -0.5, O.Q8_0, Hkv, Hkv * row, row)
    v = O.parity_verdict(got, O.decode_batched(*args), O.decode_batched(*args, mode=O.MODE_FP64))
    assert v["ok"], v


@pytest.mark.parametrize("lens,max_len", [
    ([7300], 8192),                     # configs[3]: 115 splits of 64 keys
    ([1], 8192),                        # one key
    ([200], 8192),                      # four splits
    ([64], 8192),                       # one split
    ([8192], 8192),                     # the full window: every split active
    ([5000, 17, 2600, 64, 8191], 8192), # mixed batch
    ([3000, 1000], 3000),               # a smaller ring: fewer, longer splits
])
def test_small_batch_q8_decode(lens, max_len):
    _run(lens, max_len, seed=len(lens) * 7 + lens[0])
