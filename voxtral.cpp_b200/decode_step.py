"""Graph-replayed decode step for the attention part of voxtral.cpp's decoder.

voxtral.cpp rebuilds, allocates and schedules a ggml graph for every decoded
token (run_decoder_step, src/voxtral.cpp:2438-2473; graph build and
scheduling :1921-1973, :2086-2101) and keeps the cache window with a host-side
shift-left memmove (:1237-1266, :2444-2447).  This helper captures one step of
the attention path for all layers once, as a CUDA graph:

    for each layer:  vtx_decode_layer       (RoPE of Q/K, K/V into the ring row,
                                             attention over the ring, one launch)
                     -- or, with fused=False (and for F32 caches), the two calls
                     vtx_kv_append + vtx_flash_attn_decode_batched
    then:            vtx_decode_advance     (positions, ring slots, lengths + 1)

and replays it per token with no host work: positions, ring slots and key
counts live on the device and advance inside the graph.  The fused layer
call's split layout follows a bound on the key counts (max_kv_len): the
helper keeps one set of layer plans and one graph per bound, a power of two
from 256 up to the window, and switches to the next as the caches grow (the
host knows every stream's length from its start and the step count), so
short caches run few splits merged inside a thread-block cluster and long
ones many splits merged through global memory.  Each of the n_seq
streams has its own cache per layer (rows = the window); the step's Q/K/V
projections are read from fixed per-layer buffers that the caller (the rest
of the decoder, out of scope here) fills before each replay.
"""
from __future__ import annotations

from typing import List, Optional

import torch

import vtx_attn


def key_bound(longest: int, window: int) -> int:
    """The key bound a decode step's layer plans are made for: the longest
    stream's kv_len rounded up to a power of two of at least 256, at most
    the window."""
    n = min(longest, window)
    b = 256
    while b < n:
        b *= 2
    return min(b, window)


class DecodeStepGraph:
    def __init__(self, n_layers: int, n_seq: int, n_head_q: int, n_head_kv: int, head_dim: int, kv_type: int,
                 window: int, start_len, rope_base: float = 1e6, device: Optional[torch.device] = None,
                 fused: bool = True):
        """start_len: tokens already in each stream's cache (its prefill), one
        int per stream; the next token goes to ring slot start_len % window at
        position start_len.  fused: one vtx_decode_layer launch per layer
        (F16 / Q8_0 caches, head_dim 128) instead of append + attention."""
        dev = device or torch.device("cuda", torch.cuda.current_device())
        self.dev, self.L, self.S, self.Hq, self.Hkv, self.D = dev, n_layers, n_seq, n_head_q, n_head_kv, head_dim
        self.kv_type, self.W, self.base = kv_type, window, rope_base
        hb = head_dim // 32 * 34 if kv_type == vtx_attn.Q8_0 else head_dim * (4 if kv_type == vtx_attn.F32 else 2)
        self.row = n_head_kv * hb
        start = torch.as_tensor(start_len, dtype=torch.int32)
        self.positions = start.clone().to(dev)
        self.slots = (start % window).to(torch.int32).to(dev)
        self.kv_len = torch.clamp(start + 1, max=window).to(torch.int32).to(dev)   # includes the new token
        self._start = (self.positions.clone(), self.slots.clone(), self.kv_len.clone())
        self._start_max = int(start.max()) if start.numel() else 0
        self._steps = 0                         # steps since the start (or the last reset)
        # caches: [layer][stream] of window rows
        self.k_cache = torch.zeros((n_layers, n_seq, window, self.row), dtype=torch.uint8, device=dev)
        self.v_cache = torch.zeros_like(self.k_cache)
        self.k_ptrs = [torch.tensor([self.k_cache[l, s].data_ptr() for s in range(n_seq)], dtype=torch.int64,
                                    device=dev) for l in range(n_layers)]
        self.v_ptrs = [torch.tensor([self.v_cache[l, s].data_ptr() for s in range(n_seq)], dtype=torch.int64,
                                    device=dev) for l in range(n_layers)]
        # per-layer inputs (this step's projections) and outputs
        self.q = torch.zeros((n_layers, n_seq, n_head_q, head_dim), device=dev)
        self.k = torch.zeros((n_layers, n_seq, n_head_kv, head_dim), device=dev)
        self.v = torch.zeros_like(self.k)
        self.q_rot = torch.zeros_like(self.q)
        self.out = torch.zeros_like(self.q)
        self.fused = fused and kv_type in (vtx_attn.F16, vtx_attn.Q8_0) and head_dim == 128
        self.plans: List[vtx_attn.DecodeBatchPlan] = []
        self._layer_plans: dict = {}            # key bound -> one DecodeLayerPlan per layer
        for l in range(0 if self.fused else n_layers):
            p = vtx_attn.DecodeBatchPlan([self.k_cache[l, s] for s in range(n_seq)],
                                         [self.v_cache[l, s] for s in range(n_seq)], self.kv_len, n_head_q,
                                         n_head_kv, head_dim, kv_type, self.row, hb, window, head_dim ** -0.5,
                                         fresh_row=self.slots)      # the append just before writes this row
            self.plans.append(p)
        self.stream = torch.cuda.Stream(device=dev)
        self._graphs: dict = {}                 # key bound -> captured step

    def fill(self, layer: int, seq: int, k: torch.Tensor, v: torch.Tensor, positions: torch.Tensor) -> None:
        """Writes prefill tokens of one stream into one layer's ring (rows
        positions % window; later tokens overwrite earlier ones, as the
        reference's window keeps the most recent).  k, v: (T, Hkv, D) float32."""
        if k.shape[0] > self.W:      # one call must not write a row twice: keep the most recent window
            k, v, positions = k[-self.W:], v[-self.W:], positions[-self.W:]
        pos = positions.to(device=self.dev, dtype=torch.int32)
        vtx_attn.kv_append(k, v, pos, pos % self.W, self.k_cache[layer, seq], self.v_cache[layer, seq],
                           self.kv_type, self.base, cache_nb1=self.row)

    def bound(self) -> int:
        """The key bound of the next step: the longest stream's kv_len after
        it, rounded up to a power of two of at least 256, at most the window
        (the two-call path uses the window)."""
        if not self.fused:
            return self.W
        return key_bound(self._start_max + 1 + self._steps, self.W)

    def layer_plans(self, bound: int) -> List[vtx_attn.DecodeLayerPlan]:
        """The fused layer calls planned for caches of at most `bound` rows."""
        plans = self._layer_plans.get(bound)
        if plans is None:
            # layer 0 follows vtx_decode_advance, which moves the counters: it
            # waits before reading anything; later layers may stream their ring
            # while the previous layer's kernel still runs
            plans = [vtx_attn.DecodeLayerPlan(
                [self.k_cache[l, s] for s in range(self.S)], [self.v_cache[l, s] for s in range(self.S)],
                self.positions, self.slots, self.kv_len, self.Hq, self.Hkv, self.D, self.kv_type, self.row, bound,
                self.D ** -0.5, self.base, early=l > 0) for l in range(self.L)]
            self._layer_plans[bound] = plans
        return plans

    def _step_calls(self, bound: int) -> None:
        for l, lp in enumerate(self.layer_plans(bound) if self.fused else []):
            lp(self.q[l], self.k[l], self.v[l], self.out[l], self.stream)
        for l in range(0 if self.fused else self.L):
            vtx_attn.kv_append(self.k[l], self.v[l], self.positions, self.slots, None, None, self.kv_type, self.base,
                               q=self.q[l], q_out=self.q_rot[l], k_cache_ptrs=self.k_ptrs[l],
                               v_cache_ptrs=self.v_ptrs[l], cache_nb1=self.row, stream=self.stream)
            self.plans[l](self.q_rot[l], self.out[l], self.stream)
        rc = vtx_attn.load().vtx_decode_advance(
            vtx_attn.ctypes.c_void_p(self.positions.data_ptr()), vtx_attn.ctypes.c_void_p(self.slots.data_ptr()),
            vtx_attn.ctypes.c_void_p(self.kv_len.data_ptr()), self.S, self.W,
            vtx_attn.ctypes.c_void_p(self.stream.cuda_stream))
        vtx_attn._check(rc, "vtx_decode_advance")

    def reset(self) -> None:
        """Rewinds every stream to its start_len (its prefill rows stay in the
        rings): the next step writes slot start_len % window again."""
        self.stream.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(self.stream):
            for dst, src in zip((self.positions, self.slots, self.kv_len), self._start):
                dst.copy_(src)
        torch.cuda.current_stream(self.dev).wait_stream(self.stream)
        self._steps = 0

    def step_eager(self) -> None:
        """One step issued call by call from the host (the uncaptured path)."""
        bound = self.bound()
        self.stream.wait_stream(torch.cuda.current_stream(self.dev))
        self._step_calls(bound)
        torch.cuda.current_stream(self.dev).wait_stream(self.stream)
        self._steps += 1

    def capture(self, bound: int) -> None:
        """Records one step with the plans of `bound` (nothing runs)."""
        torch.cuda.synchronize(self.dev)
        graph = torch.cuda.CUDAGraph()
        # the device counters must not move during capture: record only
        with torch.cuda.graph(graph, stream=self.stream):
            self._step_calls(bound)
        torch.cuda.synchronize(self.dev)
        self._graphs[bound] = graph

    def step(self) -> None:
        """One decode step for every stream and layer.  The first step of each
        key bound runs eagerly (it also performs the library's one-time
        per-device set-up, which a capture must not contain) and is then
        captured; every later step of that bound is a graph replay."""
        bound = self.bound()
        graph = self._graphs.get(bound)
        if graph is None:
            self.step_eager()
            self.capture(bound)
            return
        self.stream.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(self.stream):
            graph.replay()
        torch.cuda.current_stream(self.dev).wait_stream(self.stream)
        self._steps += 1


def _main() -> None:
    """Times the replayed step of one stream: python decode_step.py [--layers L]
    [--keys N] [--kv q8_0|f16]; prints microseconds per layer."""
    import argparse

    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--keys", type=int, default=7300, help="tokens already in the ring")
    ap.add_argument("--kv", default="q8_0", choices=["q8_0", "f16"])
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--unfused", action="store_true", help="append + attention as two calls per layer")
    args = ap.parse_args()
    kvt = vtx_attn.Q8_0 if args.kv == "q8_0" else vtx_attn.F16
    L, start = args.layers, args.keys
    g = DecodeStepGraph(L, 1, 32, 8, 128, kvt, 8192, [start], 1e6, fused=not args.unfused)
    gen = torch.Generator(device=g.dev)
    gen.manual_seed(1)
    for l in range(L):
        k = torch.randn((start, 8, 128), generator=gen, device=g.dev)
        g.fill(l, 0, k, torch.randn_like(k), torch.arange(start, dtype=torch.int32))
    g.q.normal_(generator=gen)
    g.k.normal_(generator=gen)
    g.v.normal_(generator=gen)
    for _ in range(3):
        g.step_eager()
    g.step()                                                 # capture
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(g.stream)
    for _ in range(args.steps):
        g.step()
    e1.record(g.stream)
    torch.cuda.synchronize()
    print(f"layers={L} keys={start} kv={args.kv}: {e0.elapsed_time(e1) / args.steps * 1e3 / L:.2f} us/layer (graph)")


if __name__ == "__main__":
    _main()
