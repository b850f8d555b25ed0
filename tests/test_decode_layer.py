"""vtx_decode_layer: one launch per decoder layer and token that rotates Q and
K, writes the new K/V row into its ring slot and attends over the ring
(src/voxtral.cpp:1744-1770 and :1783-1805 in run_decoder_step :2438-2473).

Checked against the oracle pipeline the reference runs: oracle.kv_append (RoPE
mode 0, the cache write) on host caches, then oracle attention (ggml mode and
fp64) over the ring's valid rows.  The V row the kernel writes must equal the
oracle's bytes, the rotated K row must match as vtx_kv_append's does (one f16
ulp; Q8_0 within one step), no other row may change, and the output must meet
the parity bar.  Cases cover
one split (short caches), many splits merged in the kernel (long caches),
ragged batches, wrapped rings, GQA group sizes 1 / 4 / 8, odd KV head counts
(F16), and the early ring fill."""
import numpy as np
import pytest

import oracle as O
from vtx_cases import assert_parity, f16_ulp_close, q8_close

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _views(host_k, host_v, n, Hkv, D, hb, kv_type):
    if kv_type == O.Q8_0:
        kk, vv = host_k[:n].reshape(n, Hkv, hb), host_v[:n].reshape(n, Hkv, hb)
    else:
        kk = host_k[:n].view(np.float16).reshape(n, Hkv, D)
        vv = host_v[:n].view(np.float16).reshape(n, Hkv, D)
    return kk.transpose(1, 0, 2)[None], vv.transpose(1, 0, 2)[None]


def run_layer(kv_type, lens, Hq=32, Hkv=8, D=128, W=8192, seed=0, early=False, steps=1, bound=None):
    """lens[s]: tokens in stream s once this step's token is appended.  Runs
    `steps` consecutive calls (the counters advanced on the host between
    them) and checks each against the oracle.  bound: the plan's max_kv_len
    (default: the ring's rows)."""
    import vtx_attn
    rng = np.random.default_rng(seed)
    S = len(lens)
    hb = O.cache_head_bytes(kv_type, D)
    row = Hkv * hb
    host_k = [np.zeros((W, row), np.uint8) for _ in range(S)]
    host_v = [np.zeros((W, row), np.uint8) for _ in range(S)]
    for s, n in enumerate(lens):
        m = n - 1                                            # rows before this step's token
        k = rng.standard_normal((m, Hkv, D)).astype(np.float32)
        v = rng.standard_normal((m, Hkv, D)).astype(np.float32)
        pos = np.arange(m, dtype=np.int32)
        if m > W:                                            # the window keeps the most recent rows
            k, v, pos = k[-W:], v[-W:], pos[-W:]
        if m:
            O.kv_append(None, k, v, pos, pos % W, kv_type, 1e6, host_k[s], host_v[s])
    kc = [torch.from_numpy(h.copy()).cuda() for h in host_k]
    vc = [torch.from_numpy(h.copy()).cuda() for h in host_v]
    positions = torch.tensor([n - 1 for n in lens], dtype=torch.int32, device="cuda")
    slots = torch.tensor([(n - 1) % W for n in lens], dtype=torch.int32, device="cuda")
    kv_len = torch.tensor([min(n, W) for n in lens], dtype=torch.int32, device="cuda")
    plan = vtx_attn.DecodeLayerPlan(kc, vc, positions, slots, kv_len, Hq, Hkv, D, kv_type, row,
                                    W if bound is None else bound, D ** -0.5, 1e6, early=early)
    for step in range(steps):
        q = rng.standard_normal((S, Hq, D)).astype(np.float32)
        k = rng.standard_normal((S, Hkv, D)).astype(np.float32)
        v = rng.standard_normal((S, Hkv, D)).astype(np.float32)
        out = torch.full((S, Hq, D), float("nan"), device="cuda")
        plan(torch.from_numpy(q).cuda(), torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda(), out)
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        pos_h, slot_h, len_h = positions.cpu().numpy(), slots.cpu().numpy(), kv_len.cpu().numpy()
        for s in range(S):
            p, sl, n = int(pos_h[s]), int(slot_h[s]), int(len_h[s])
            qr = O.kv_append(q[s][None], k[s][None], v[s][None], [p], [sl], kv_type, 1e6, host_k[s], host_v[s])
            dk, dv = kc[s].cpu().numpy(), vc[s].cpu().numpy()
            others = np.arange(W) != sl
            assert np.array_equal(dk[others], host_k[s][others]), f"step {step} stream {s}: other K rows"
            assert np.array_equal(dv, host_v[s]), f"step {step} stream {s}: V cache bytes"
            # the rotated K row: as vtx_kv_append's against the oracle (cos/sin
            # in double rounded to float on the device, cosf/sinf in ggml)
            if kv_type == O.Q8_0:
                q8_close(dk[sl], host_k[s][sl])
            else:
                f16_ulp_close(dk[sl].view(np.float16), host_k[s][sl].view(np.float16))
            host_k[s][sl] = dk[sl]                           # attend over the row the device holds
            kk, vv = _views(host_k[s], host_v[s], n, Hkv, D, hb, kv_type)
            qv = qr.reshape(1, 1, Hq, D).transpose(0, 2, 1, 3)
            ref = O.flash_attn_ext(qv, kk, vv, None, D ** -0.5, kv_type=kv_type)
            ref64 = O.flash_attn_ext(qv, kk, vv, None, D ** -0.5, kv_type=kv_type, mode=O.MODE_FP64)
            assert_parity(got[s][None, None], ref, ref64, f"step {step} stream {s} (kv_len {n})")
        positions += 1
        slots.copy_((slots + 1) % W)
        kv_len.copy_(torch.clamp(kv_len + 1, max=W))
    assert vtx_attn.read_device_error() == 0
    return plan


@pytest.mark.parametrize("kv", [O.F16, O.Q8_0], ids=["f16", "q8_0"])
@pytest.mark.parametrize("n", [1, 17, 391, 600, 2000, 7300])
def test_batch1_matches_oracle_pipeline(kv, n):
    """configs[2] / configs[3] decode steps (32/8 heads x 128), from a one-row
    cache (one split) to 7300 rows (18 splits merged in the kernel)."""
    run_layer(kv, [n], seed=n + kv)


@pytest.mark.parametrize("kv", [O.F16, O.Q8_0], ids=["f16", "q8_0"])
def test_consecutive_steps_reuse_the_workspace(kv):
    """Three calls in a row on the same workspace: the split-arrival words
    left by one launch never count for the next."""
    run_layer(kv, [3000, 40], seed=7, steps=3)


@pytest.mark.parametrize("kv", [O.F16, O.Q8_0], ids=["f16", "q8_0"])
def test_ragged_batch(kv):
    run_layer(kv, [5, 700, 3000, 16, 129, 1], seed=11 + kv)


@pytest.mark.parametrize("kv", [O.F16, O.Q8_0], ids=["f16", "q8_0"])
def test_wrapped_ring(kv):
    """Rings of 64 rows that have wrapped: the new row overwrites the oldest."""
    run_layer(kv, [100, 64, 65, 200], W=64, seed=21 + kv, steps=2)


@pytest.mark.parametrize("Hq,Hkv,kv", [(8, 8, O.F16), (8, 8, O.Q8_0), (64, 8, O.F16), (64, 8, O.Q8_0),
                                        (12, 3, O.F16)],
                         ids=["g1-f16", "g1-q8_0", "g8-f16", "g8-q8_0", "g4-hkv3-f16"])
def test_group_sizes(Hq, Hkv, kv):
    run_layer(kv, [1500, 33], Hq=Hq, Hkv=Hkv, seed=31 + Hq + kv)


@pytest.mark.parametrize("kv", [O.F16, O.Q8_0], ids=["f16", "q8_0"])
def test_early_ring_fill(kv):
    """early = 1: the ring rows are streamed before the dependency wait; the
    result and the written row are the same."""
    run_layer(kv, [2500, 9], seed=41 + kv, early=True, steps=2)



@pytest.mark.parametrize("kv,n,bound", [(O.F16, 391, 1024), (O.F16, 1000, 1024), (O.Q8_0, 600, 2048),
                                        (O.Q8_0, 2000, 2048), (O.Q8_0, 3000, 1024)],
                         ids=["f16-391", "f16-1000", "q8_0-600", "q8_0-2000", "q8_0-3000-past-bound"])
def test_cluster_merge(kv, n, bound):
    """A tighter key bound plans few splits (at most 12 here) merged through
    distributed shared memory: the splits of each KV head are the CTAs of one
    thread-block cluster.  A cache longer than the bound stays correct (its
    splits are capped, each longer).  Two calls in a row."""
    run_layer(kv, [n], seed=90 + n + kv, steps=2, bound=bound)


@pytest.mark.parametrize("kv", [O.F16, O.Q8_0], ids=["f16", "q8_0"])
def test_cluster_merge_ragged(kv):
    """Two streams under one bound: one with a single split (its cluster's
    other CTAs leave at once), one merged in the cluster."""
    run_layer(kv, [40, 900], seed=95 + kv, steps=2, bound=1024, early=True)
