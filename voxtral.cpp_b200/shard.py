"""Multi-GPU placement of the attention node: one process per GPU.

voxtral.cpp itself runs one utterance per context on one device (no DP/TP:
src/voxtral.cpp:2409, :2451 keep static thread_local graph state).  On an
8 x B200 box the node scales two ways:

* Independent streams / clips per GPU (no collective on the data path).
  ``lpt_shard`` assigns ragged decode streams to ranks by longest-processing-
  time bin packing on kv_len, so every rank streams about the same number of
  KV bytes per decode step; encoder clips are simply dealt round robin.
* Long-context prefill split by KV head (``head_split_prefill``): rank r owns
  KV heads [r*Hkv/N, (r+1)*Hkv/N) and the Hq/Hkv query heads of each, runs the
  attention node on its slice straight into its block of the gather buffer,
  and one in-place all-gather assembles ggml's [Dv, Hq, n_q, B] result.  All remote bytes move through the collective into
  local memory; no kernel reads a peer's memory.

The attention callable is injected (default: vtx_attn.flash_attn_ext) so the
placement logic can be exercised on CPU ranks with any reference function.
"""
from __future__ import annotations

from typing import Callable, List, Optional, Sequence

import torch


def lpt_shard(kv_len: Sequence[int], n_ranks: int) -> List[List[int]]:
    """Longest-processing-time bin packing of streams onto ranks by kv_len.
    Deterministic: ties broken by stream index, then by rank index.  Every
    stream appears exactly once; each rank's list is in ascending stream id."""
    if n_ranks <= 0:
        raise ValueError("n_ranks must be positive")
    order = sorted(range(len(kv_len)), key=lambda i: (-int(kv_len[i]), i))
    load = [0] * n_ranks
    bins: List[List[int]] = [[] for _ in range(n_ranks)]
    for i in order:
        r = min(range(n_ranks), key=lambda j: (load[j], j))
        bins[r].append(i)
        load[r] += int(kv_len[i])
    return [sorted(b) for b in bins]


def shard_loads(kv_len: Sequence[int], bins: List[List[int]]) -> List[int]:
    return [sum(int(kv_len[i]) for i in b) for b in bins]


def head_range(n_head_kv: int, rank: int, world: int) -> range:
    if n_head_kv % world:
        raise ValueError(f"{n_head_kv} KV heads do not split over {world} ranks")
    per = n_head_kv // world
    return range(rank * per, (rank + 1) * per)


def head_split_prefill(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, mask: Optional[torch.Tensor],
                       scale: float, *, group=None, attn: Optional[Callable] = None, **kw) -> torch.Tensor:
    """Attention over KV heads split across the ranks of ``group``.

    q: (B, Hq, n_q, D), k/v: (B, Hkv, n_kv, D) — the full views; each rank
    slices out its heads (views, no copy).  Rank r computes query heads
    [r*Hq/N, (r+1)*Hq/N) straight into block r of one buffer
    (N, B, n_q, Hq/N, Dv) -- the attention writes ggml's strides, so there is
    no copy -- and one in-place all_gather_into_tensor fills the other blocks.
    Returns the buffer as a view (B, n_q, N, Hq/N, Dv): ggml's
    [Dv, Hq, n_q, B] result with the head axis split at rank boundaries
    (head = r * Hq/N + j), every rank holding all of it.  A consumer that
    takes strides (vtx_attn_out_proj's A operand) reads it as is;
    ``as_heads`` makes the contiguous (B, n_q, Hq, Dv) copy."""
    import torch.distributed as dist
    if float(kw.get("max_bias", 0.0)) != 0.0:
        # ggml's ALiBi slope depends on the global head index; each rank's
        # call numbers its heads from 0, so slopes would be wrong past rank 0
        raise ValueError("head_split_prefill does not support max_bias != 0 (ALiBi)")
    direct = attn is None
    if attn is None:
        import vtx_attn
        attn = vtx_attn.flash_attn_ext
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    B, Hq, n_q = q.shape[0], q.shape[1], q.shape[2]
    Hkv = k.shape[1]
    G = Hq // Hkv
    hr = head_range(Hkv, rank, world)
    qs = q[:, hr.start * G:hr.stop * G]
    ks, vs = k[:, hr.start:hr.stop], v[:, hr.start:hr.stop]
    ms = mask
    if mask is not None and mask.dim() == 4 and mask.shape[1] == Hq:
        ms = mask[:, hr.start * G:hr.stop * G]
    Dv = v.shape[-1] if v.dtype != torch.uint8 else v.shape[-1] // 34 * 32
    # blocks concatenated along dim 0, the layout every backend's all-gather takes
    buf = torch.empty((world * B, n_q, Hq // world, Dv), dtype=torch.float32, device=q.device)
    mine = buf[rank * B:(rank + 1) * B]
    if direct:
        attn(qs, ks, vs, ms, scale, out=mine, **kw)              # written in place, ggml strides
    else:
        mine.copy_(attn(qs, ks, vs, ms, scale, **kw))
    dist.all_gather_into_tensor(buf, mine, group=group)           # in place: rank r's block is the input
    return buf.view(world, B, n_q, Hq // world, Dv).permute(1, 2, 0, 3, 4)


def as_heads(x: torch.Tensor) -> torch.Tensor:
    """(B, n_q, N, Hq/N, Dv) result of head_split_prefill -> contiguous
    (B, n_q, Hq, Dv) (ggml's dst layout); a copy when N > 1."""
    B, n_q, N, h, Dv = x.shape
    return x.reshape(B, n_q, N * h, Dv)
