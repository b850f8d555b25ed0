"""Graph-replayed decode steps (voxtral.cpp_b200/decode_step.py): per layer,
KV append (RoPE + ring write) and batched decode attention, then the device
counters advance, all captured once and replayed token after token.  Every
step's output is compared with the oracle pipeline (oracle KV append on host
caches, then oracle attention over the ring's valid rows)."""
import numpy as np
import pytest

import oracle as O
from vtx_cases import assert_close

pytestmark = pytest.mark.gpu


def _run_steps(kv_type, fused, L, S, Hq, Hkv, D, W, start, steps, seed):
    import torch
    from decode_step import DecodeStepGraph
    rng = np.random.default_rng(seed)
    g = DecodeStepGraph(L, S, Hq, Hkv, D, kv_type, W, start, fused=fused)
    assert g.fused == fused
    hb = O.cache_head_bytes(kv_type, D)
    host_k = np.zeros((L, S, W, Hkv * hb), np.uint8)
    host_v = np.zeros_like(host_k)
    for l in range(L):
        for s in range(S):
            n = start[s]
            k = rng.standard_normal((n, Hkv, D)).astype(np.float32)
            v = rng.standard_normal((n, Hkv, D)).astype(np.float32)
            pos = np.arange(n, dtype=np.int32)
            g.fill(l, s, torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda(), torch.from_numpy(pos))
            O.kv_append(None, k, v, pos, pos % W, kv_type, 1e6, host_k[l, s], host_v[l, s])
    bounds = []
    for t in range(steps):
        q = rng.standard_normal((L, S, Hq, D)).astype(np.float32)
        k = rng.standard_normal((L, S, Hkv, D)).astype(np.float32)
        v = rng.standard_normal((L, S, Hkv, D)).astype(np.float32)
        g.q.copy_(torch.from_numpy(q))
        g.k.copy_(torch.from_numpy(k))
        g.v.copy_(torch.from_numpy(v))
        bounds.append(g.bound())
        g.step()
        out = g.out.cpu().numpy()
        for l in range(L):
            for s in range(S):
                p = start[s] + t
                qr = O.kv_append(q[l, s][None], k[l, s][None], v[l, s][None], [p], [p % W], kv_type, 1e6,
                                 host_k[l, s], host_v[l, s])
                n = min(p + 1, W)
                if kv_type == O.Q8_0:
                    kk, vv = host_k[l, s, :n].reshape(n, Hkv, hb), host_v[l, s, :n].reshape(n, Hkv, hb)
                else:
                    kk = host_k[l, s, :n].view(np.float16).reshape(n, Hkv, D)
                    vv = host_v[l, s, :n].view(np.float16).reshape(n, Hkv, D)
                ref = O.flash_attn_ext(qr.reshape(1, 1, Hq, D).transpose(0, 2, 1, 3), kk.transpose(1, 0, 2)[None],
                                       vv.transpose(1, 0, 2)[None], None, D ** -0.5, kv_type=kv_type)
                assert_close(out[l, s][None, None], ref, f"step {t} layer {l} stream {s}")
    # the device counters advanced with the replays
    assert g.positions.cpu().tolist() == [x + steps for x in start]
    assert g.kv_len.cpu().tolist() == [min(x + steps + 1, W) for x in start]
    return bounds


@pytest.mark.parametrize("fused", [True, False], ids=["fused", "two-calls"])
@pytest.mark.parametrize("kv_type", [O.F16, O.Q8_0])
def test_graph_decode_steps_match_oracle(kv_type, fused):
    # the last stream's ring has already wrapped
    _run_steps(kv_type, fused, 2, 3, 8, 2, 128, 64, [5, 60, 70], 30, 50 + kv_type)


@pytest.mark.parametrize("kv_type,start", [(O.F16, [100, 247]), (O.Q8_0, [300, 1016])], ids=["f16", "q8_0"])
def test_graph_decode_steps_across_key_bounds(kv_type, start):
    """The fused step's plans follow a power-of-two bound on the key counts:
    the steps cross one (256 -> 512 for F16, 1024 -> 2048 for Q8_0), so a
    second set of plans and a second graph take over, with more key splits,
    merged in a thread-block cluster."""
    bounds = _run_steps(kv_type, True, 2, 2, 32, 8, 128, 4096, start, 14, 70 + kv_type)
    assert len(set(bounds)) == 2 and bounds == sorted(bounds)
