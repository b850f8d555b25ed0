"""Multi-rank placement logic on CPU ranks (gloo, world size 2): LPT stream
sharding and head-split prefill with an all-gather, checked against the CPU
oracle run on the whole problem.  No GPU: the attention callable injected into
the sharder is the oracle itself."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as O
import shard
from vtx_cases import make_case


def test_lpt_shard_covers_and_balances():
    rng = np.random.default_rng(0)
    lens = rng.integers(512, 16385, 256).tolist()
    for n in (1, 2, 4, 8):
        bins = shard.lpt_shard(lens, n)
        flat = sorted(i for b in bins for i in b)
        assert flat == list(range(256))
        loads = shard.shard_loads(lens, bins)
        # LPT bound: max load <= average + largest item
        assert max(loads) <= sum(lens) / n + max(lens)
        if n > 1:
            assert (max(loads) - min(loads)) / (sum(lens) / n) < 0.02
    assert shard.lpt_shard([5, 5, 5], 2) == shard.lpt_shard([5, 5, 5], 2)   # deterministic


def test_head_range_rejects_uneven_split():
    assert list(shard.head_range(8, 1, 4)) == [2, 3]
    with pytest.raises(ValueError):
        shard.head_range(8, 0, 3)


def _oracle_attn(q, k, v, mask, scale, **kw):
    """Attention callable over torch CPU views, computed by the oracle."""
    out = O.flash_attn_ext(q.numpy(), k.numpy(), v.numpy(), None if mask is None else mask.numpy(), scale,
                           causal=int(kw.get("causal", False)), window=int(kw.get("window", 0)))
    return torch.from_numpy(out)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q, k, v, mask, scale, kw, result_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        out = shard.as_heads(shard.head_split_prefill(q, k, v, mask, scale, attn=_oracle_attn, **kw))
        torch.save(out, f"{result_path}.{rank}")
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("how", ["mask", "causal"])
def test_head_split_prefill_matches_unsplit(tmp_path, how):
    kw = {"mask": "causal"} if how == "mask" else {"causal": 1}
    c = make_case(31, Hq=8, Hkv=4, n_q=37, n_kv=37, D=64, **kw)
    full = O.flash_attn_ext(c.q, c.k, c.v, c.mask, c.scale, causal=c.causal)
    q, k, v = (torch.from_numpy(np.ascontiguousarray(a)) for a in (c.q, c.k, c.v))
    mask = torch.from_numpy(c.mask) if c.mask is not None else None
    world = 2
    res = str(tmp_path / "out")
    mp.start_processes(_worker, args=(world, _free_port(), q, k, v, mask, c.scale, {"causal": bool(c.causal)}, res),
                       nprocs=world, start_method="spawn", join=True)
    for r in range(world):
        got = torch.load(f"{res}.{r}").numpy()
        assert got.shape == full.shape
        # every rank ends with the same, complete result, heads in ggml order
        assert np.array_equal(got, full), f"rank {r}"


def test_rank_failure_surfaces_on_host(tmp_path):
    """A rank that raises before the collective makes the launcher fail
    instead of hanging the survivors (process-group timeout bounds the wait)."""
    def bad_attn(*a, **k):
        raise RuntimeError("injected host-side failure")
    port = _free_port()
    with pytest.raises(Exception):
        mp.start_processes(_failing_worker, args=(2, port), nprocs=2, start_method="spawn", join=True)


def _failing_worker(rank, world, port):
    import datetime
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    try:
        if rank == 1:
            raise RuntimeError("injected host-side failure on rank 1")
        q = torch.zeros(1, 2, 3, 64)
        k = torch.zeros(1, 2, 3, 64, dtype=torch.float16)
        shard.head_split_prefill(q, k, k, None, 0.125, attn=_oracle_attn)
    finally:
        dist.destroy_process_group()


def test_head_split_prefill_rejects_alibi():
    """ggml's ALiBi slopes depend on the global head index, which a rank's
    call on its head slice does not see: the split refuses max_bias != 0."""
    q = torch.zeros((1, 8, 4, 64))
    k = torch.zeros((1, 4, 4, 64))
    with pytest.raises(ValueError):
        shard.head_split_prefill(q, k, k, None, 0.125, attn=_oracle_attn, max_bias=8.0)
