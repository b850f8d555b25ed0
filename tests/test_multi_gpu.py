"""Head-split prefill on 2 GPUs over NCCL: one process per GPU, each runs the
CUDA attention on its KV heads and the ranks exchange their slices with one
all_gather (voxtral.cpp_b200/shard.py).  The gathered result must match the
CPU oracle on the whole problem and the single-GPU call on the whole problem.
Skipped when fewer than 2 GPUs are visible."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from vtx_cases import assert_close, make_case, oracle_out, to_device

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, case, result_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        import shard
        # the spawned rank receives copies of the case's views (pickling drops the
        # shared buffers), so they go to the device as contiguous tensors
        q, k, v = (torch.from_numpy(np.ascontiguousarray(a)).cuda(rank) for a in (case.q, case.k, case.v))
        out = shard.as_heads(shard.head_split_prefill(q, k, v, None, case.scale, causal=bool(case.causal)))
        torch.cuda.synchronize()
        torch.save(out.cpu(), f"{result_path}.{rank}")
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_head_split_prefill_nccl_2gpu(tmp_path):
    import vtx_attn
    # configs[2] decoder prefill: 391 tokens, GQA 32/8, head_dim 128, causal
    case = make_case(41, Hq=32, Hkv=8, n_q=391, n_kv=391, D=128, causal=1)
    ref = oracle_out(case)
    q, k, v = to_device(case)[:3]
    whole = vtx_attn.flash_attn_ext(q, k, v, None, case.scale, causal=True).cpu().numpy()
    res = str(tmp_path / "out")
    mp.start_processes(_worker, args=(2, _free_port(), case, res), nprocs=2, start_method="spawn", join=True)
    for r in range(2):
        got = torch.load(f"{res}.{r}").numpy()
        assert got.shape == ref.shape
        assert_close(got, ref, f"head-split prefill, rank {r}")
        # per-head arithmetic does not depend on which heads share a call
        assert np.array_equal(got, whole), f"rank {r} differs from the single-GPU call"
