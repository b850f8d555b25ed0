"""Benchmark of the voxtral.cpp attention node on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl vtx|reference]
                    [--workload encoder|decode|kv_append|decode_step|realtime|prefill]

Headline workload: the Whisper-large-shaped audio
encoder self-attention of voxtral.cpp (src/voxtral.cpp:1611): one 30 s clip ->
1500 frames, 20 heads x head_dim 64, 32 layers, bidirectional (mask = NULL),
f16 Q/K/V drawn N(0,1) from a seed, fp32 softmax/accumulate.  One step = the
32 attention calls of one clip, each layer with its own Q/K/V (368 MB per step,
larger than the 126 MB L2, so no flush is needed between steps).  Metric:
attention TFLOP/s = 4 * D * H * n_q * n_kv * layers / time.

--workload decode times configs[4] instead: 256 ragged streams (n_kv ~ U[512,
16384]), GQA 32/8 x 128, f16 KV, one decode token per stream; one step = one
layer's attention for all streams (KV GB/s).  kv_append and decode_step time
the decoder's cache update and the graph-replayed batch-1 decode step
(configs[2], configs[3]); realtime times configs[3] end to end on the
attention path: 10 min of audio as chunked windowed encoder attention, the
chunk stitch and 7461 Q8_0 decode steps (audio-sec/sec).

Multi-GPU: one process per GPU (torchrun); each rank attends its own clips /
streams (weak scaling, no collective on the data path); time = max over ranks.
--impl reference times the CPU restatement of ggml's flash_attn_ext (the
oracle; ggml itself is not buildable here) on a bounded sample of the same
workload with every host core, rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "voxtral.cpp_b200"))

ENC = dict(n=1500, H=20, D=64, layers=32)
DEC = dict(n_seq=256, Hq=32, Hkv=8, D=128, lo=512, hi=16384)
METRIC_ENC = "attn TFLOP/s (prefill/encoder)"
ENC_TRAFFIC_BYTES = 11_590_656          # one encoder launch, dram read + write, from the committed ncu capture
DEC_TRAFFIC_RATIO_F16 = (1_058_088_000 + 7_246_080) / 1_057_517_568   # (read + write) / KV bytes, 32 streams
DEC_TRAFFIC_RATIO_Q8 = (562_400_768 + 6_991_872) / 561_806_208     # (read + write) / KV bytes, 32 streams
METRIC_DEC = "KV GB/s (decode)"
CPU_PORT_NOTE = ("The port is scalar C with per-element f16 conversions: it has ggml-cpu's numerics, not its "
                 "F16C/AVX-512 vector kernels, so it is slower than the reference's real --gpu none path and a "
                 "GPU/CPU ratio against it overstates the speed-up.")


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            j = json.load(f)
        return {"hbm_gbs": j["hbm_gbs"], "bf16_tflops": j["bf16_tflops"], "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "src": "fallback"}


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.samples = []
        self._stop = threading.Event()
        self._t = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                                      "--format=csv,noheader,nounits"], capture_output=True, text=True,
                                     timeout=5).stdout.strip()
                if out:
                    self.samples.append([x.strip() for x in out.split(",")])
            except Exception:
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        self._t.join(timeout=10)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = sorted(float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit())
        mx = max((float(s[2]) for s in self.samples if s[2].replace(".", "").isdigit()), default=None)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for s in self.samples:
            for i, n in enumerate(names):
                if len(s) > 5 + i and s[5 + i].lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(self.samples)}


# ------------------------------------------------------------------------------
def dist_setup(n_gpus: int):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return rank, world, local


def barrier_max(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


# ---- encoder workload ------------------------------------------------------------
def enc_flops_per_layer():
    return 4.0 * ENC["D"] * ENC["H"] * ENC["n"] * ENC["n"]


def make_encoder_inputs(seed: int, device):
    """Per layer: contiguous [D, H, n] f16 buffers (ggml order) permuted to the
    [D, n, H] views voxtral.cpp passes (src/voxtral.cpp:1601-1605)."""
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    n, H, D, L = ENC["n"], ENC["H"], ENC["D"], ENC["layers"]
    qkv = torch.randn((L, 3, n, H, D), generator=g, device=device, dtype=torch.float32).to(torch.float16)
    return qkv


def enc_views(buf_l):
    # buf_l: (3, n, H, D) -> q, k, v views (1, H, n, D)
    return [buf_l[i].permute(1, 0, 2).unsqueeze(0) for i in range(3)]


def run_encoder(args, rank, world, local):
    import torch
    import vtx_attn

    dev = torch.device("cuda", local)
    L, n, H, D = ENC["layers"], ENC["n"], ENC["H"], ENC["D"]
    qkv = make_encoder_inputs(1234 + rank, dev)
    out = torch.empty((L, 1, n, H, D), device=dev, dtype=torch.float32)
    scale = 1.0 / D ** 0.5
    views = [enc_views(qkv[l]) for l in range(L)]
    stream = torch.cuda.Stream(device=dev)
    ws = torch.empty(max(1, vtx_attn.workspace_bytes(*views[0], scale)), dtype=torch.uint8, device=dev)

    def step():
        for l in range(L):
            q, k, v = views[l]
            vtx_attn.flash_attn_ext(q, k, v, None, scale, out=out[l], workspace=ws, stream=stream)

    with torch.cuda.stream(stream):
        for _ in range(max(1, args.warmup)):
            step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step()
    torch.cuda.synchronize()
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()

    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        barrier(world)
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(args.steps):
                graph.replay()
            e1.record(stream)
        torch.cuda.synchronize()
        barrier(world)
    ms_local = e0.elapsed_time(e1)
    ms = barrier_max(ms_local, world)
    flop_step = enc_flops_per_layer() * L
    value = flop_step * args.steps * world / (ms * 1e-3) / 1e12
    launch_ms = ms_local / (args.steps * L)
    err = vtx_attn.read_device_error(stream)
    parity = check_encoder_layer(qkv[0], out[0]) if (rank == 0 and not args.no_check) else None

    # ---- end to end through the public call, host buffers ----------------------
    e2e = run_encoder_e2e(args, dev, world, rank)

    peaks = load_peaks()
    achieved = enc_flops_per_layer() / (launch_ms * 1e-3) / 1e12
    res = {
        "metric": METRIC_ENC, "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic N(0,1) f16 Q/K/V, seeded per rank (no dataset; BASELINE configs[1] shapes)",
        "config": {"workload": "configs[1] audio-encoder self-attention, 30 s clip: 1500 frames, 20 heads x 64, "
                               "32 layers, bidirectional, batch 1 per GPU",
                   "per_step": "32 layer calls (one clip), CUDA-graph replay",
                   "l2": "inputs larger than L2 (368 MB of Q/K/V per step), no flush",
                   "parallelism": f"dp{world} (independent clips per GPU)",
                   "audio_sec_per_step_per_gpu": 30},
        "audio_sec_per_sec": round(30.0 * args.steps * world / (ms * 1e-3), 1),
        "roofline": {"bound": "tensor", "achieved": round(achieved, 2), "peak": peaks["bf16_tflops"],
                     "unit": "TFLOP/s", "frac": round(achieved / peaks["bf16_tflops"], 4),
                     # dram__bytes_read + dram__bytes_write of one launch in the committed
                     # ncu --set full capture of the encoder kernel: 11.59 MB read (= Q+K+V),
                     # 0 written (the 7.68 MB output stays in L2 during the launch)
                     "traffic": ENC_TRAFFIC_BYTES, "traffic_unit": "bytes per launch",
                     "peak_src": f"{peaks['src']} bf16 dense (burst)",
                     "per_launch_ms": round(launch_ms, 5),
                     "per_launch_flop": enc_flops_per_layer()},
        "e2e": e2e,
        "gpu_launches": args.steps * L,
        "clocks": clocks.summary(),
        "device_error": err,
        "parity": parity,
    }
    return res


def run_encoder_e2e(args, dev, world, rank):
    """Host Q/K/V (pinned) -> device -> vtx_flash_attn_ext -> host output, per
    layer, copies on their own streams overlapped with the attention calls."""
    import torch
    import vtx_attn

    L, n, H, D = ENC["layers"], ENC["n"], ENC["H"], ENC["D"]
    scale = 1.0 / D ** 0.5
    host_in = make_encoder_inputs(99 + rank, dev).cpu().pin_memory()          # (L, 3, n, H, D)
    host_out = torch.empty((L, 1, n, H, D), dtype=torch.float32).pin_memory()
    nbuf = 3
    dbuf = [torch.empty((3, n, H, D), device=dev, dtype=torch.float16) for _ in range(nbuf)]
    dout = [torch.empty((1, n, H, D), device=dev, dtype=torch.float32) for _ in range(nbuf)]
    s_h2d, s_cmp, s_d2h = (torch.cuda.Stream(device=dev) for _ in range(3))
    ws = torch.empty(max(1, vtx_attn.workspace_bytes(*enc_views(dbuf[0]), scale)), dtype=torch.uint8, device=dev)
    ev_in = [torch.cuda.Event() for _ in range(nbuf)]
    ev_cmp = [torch.cuda.Event() for _ in range(nbuf)]
    ev_out = [torch.cuda.Event() for _ in range(nbuf)]

    def one_clip():
        for l in range(L):
            b = l % nbuf
            if l >= nbuf:
                s_h2d.wait_event(ev_cmp[b])
            with torch.cuda.stream(s_h2d):
                dbuf[b].copy_(host_in[l], non_blocking=True)
                ev_in[b].record(s_h2d)
            s_cmp.wait_event(ev_in[b])
            if l >= nbuf:
                s_cmp.wait_event(ev_out[b])
            q, k, v = enc_views(dbuf[b])
            vtx_attn.flash_attn_ext(q, k, v, None, scale, out=dout[b], workspace=ws, stream=s_cmp)
            ev_cmp[b].record(s_cmp)
            s_d2h.wait_event(ev_cmp[b])
            with torch.cuda.stream(s_d2h):
                host_out[l].copy_(dout[b], non_blocking=True)
                ev_out[b].record(s_d2h)

    for _ in range(max(1, min(args.warmup, 2))):
        one_clip()
    torch.cuda.synchronize()
    steps = max(1, min(args.steps, 10))
    barrier(world)
    t0 = time.perf_counter()
    for _ in range(steps):
        one_clip()
    torch.cuda.synchronize()
    dt = barrier_max(time.perf_counter() - t0, world)
    h2d = host_in[0].numel() * host_in.element_size() * L
    d2h = host_out[0].numel() * host_out.element_size() * L
    # The host link alone: one clip's inputs H2D and its outputs D2H, each
    # direction timed by itself on its stream (CUDA events).  With the three
    # streams overlapped the step cannot beat the slower direction.
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def link_s(copy, stream):
        with torch.cuda.stream(stream):
            e0.record(stream)
            for l in range(L):
                copy(l)
            e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) * 1e-3

    t_h2d = link_s(lambda l: dbuf[l % nbuf].copy_(host_in[l], non_blocking=True), s_h2d)
    t_d2h = link_s(lambda l: host_out[l].copy_(dout[l % nbuf], non_blocking=True), s_d2h)
    bound_s = max(t_h2d, t_d2h)
    value = enc_flops_per_layer() * L * steps * world / dt / 1e12
    bound_tflops = enc_flops_per_layer() * L * world / bound_s / 1e12
    return {"value": round(value, 3), "unit": "TFLOP/s",
            "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h), "steps": steps,
            "host_link": {"h2d_GBps": round(h2d / t_h2d / 1e9, 1), "d2h_GBps": round(d2h / t_d2h / 1e9, 1),
                          "bound_tflops": round(bound_tflops, 3), "frac_of_bound": round(value / bound_tflops, 3),
                          "how": "one clip's pinned copies per direction alone (CUDA events); the bound is the "
                                 "slower direction, since the three streams overlap"},
            "how": "pinned host Q/K/V per layer -> H2D stream, vtx_flash_attn_ext on compute stream, "
                   "D2H stream; host wall clock after synchronize, max over ranks"}


# ---- CPU baseline (oracle = CPU restatement of ggml's flash_attn_ext) -----------
def cpu_baseline_encoder(budget_s: float = 12.0):
    """The oracle (CPU restatement of ggml's flash_attn_ext, ggml mode) on whole
    encoder layers of configs[1], all host cores, until ~budget_s of CPU work
    (at most the 32 layers of one clip)."""
    import numpy as np
    import oracle as O
    n, H, D, L = ENC["n"], ENC["H"], ENC["D"], ENC["layers"]
    rng = np.random.default_rng(5)
    view = lambda a: a.transpose(1, 0, 2)[None]
    cores = O.n_cores()
    layers, spent = 0, 0.0
    while layers < L and spent < budget_s:
        q, k, v = (rng.standard_normal((n, H, D)).astype(np.float16) for _ in range(3))
        t0 = time.perf_counter()
        O.flash_attn_ext(view(q), view(k), view(v), None, D ** -0.5, threads=cores)
        spent += time.perf_counter() - t0
        layers += 1
    flops = 4.0 * D * H * n * n * layers
    return {"value": round(flops / spent / 1e12, 6), "unit": "TFLOP/s", "cores": cores, "kind": "port",
            "sample": f"{layers} of the 32 encoder layers of one configs[1] clip (1500 x 1500 x 20 heads x 64 each), "
                      f"ggml-mode oracle on {cores} threads, {spent:.1f} s. " + CPU_PORT_NOTE}


# ---- decode workload ---------------------------------------------------------------
def make_decode_inputs(S: int, q8, seed_np: int, seed_dev: int, dev):
    """configs[4] inputs: S streams with kv_len ~ U[512, 16384] (numpy seed),
    per stream a K and a V cache of kv_len rows x 8 KV heads x 128 drawn
    N(0,1) on the device (torch seed), stored f16, quantized to Q8_0 by
    ggml's rule (q8 True or "q8_0"), or F32 as the reference keeps it
    (q8 = "f32"); Q (S, 32, 128) F32 N(0,1)."""
    import numpy as np
    import torch
    import vtx_attn
    Hq, Hkv, D = DEC["Hq"], DEC["Hkv"], DEC["D"]
    rng = np.random.default_rng(seed_np)
    lens = rng.integers(DEC["lo"], DEC["hi"] + 1, S).astype(np.int32)
    g = torch.Generator(device=dev)
    g.manual_seed(seed_dev)

    def cache(L):
        x = torch.randn((int(L), Hkv, D), generator=g, device=dev)
        if q8 == "f32":
            return x
        return vtx_attn.quantize_q8_0(x) if q8 else x.to(torch.float16)

    ks = [cache(L) for L in lens]
    vs = [cache(L) for L in lens]
    q = torch.randn((S, Hq, D), generator=g, device=dev)
    return lens, ks, vs, q


def check_decode_rows(q, ks, vs, lens, out, q8, n_check: int = 8, seed: int = 0):
    """Checker (outside every timed region): the oracle's ggml-mode batched
    decode on a seeded sample of n_check streams against the device output
    rows of the same streams, judged by oracle.parity_verdict (fp64 truth
    and ggml mode, ggml's own half-precision drift admitted)."""
    import numpy as np
    import oracle as O
    Hkv, D = DEC["Hkv"], DEC["D"]
    f32 = q8 == "f32"
    q8 = q8 is True or q8 == "q8_0"
    row = D // 32 * 34 if q8 else D * (4 if f32 else 2)
    idx = sorted(np.random.default_rng(seed).choice(len(lens), size=min(n_check, len(lens)), replace=False).tolist())
    kl = [ks[i].cpu().numpy() for i in idx]
    vl = [vs[i].cpu().numpy() for i in idx]
    args = (q[idx].cpu().numpy(), kl, vl, lens[idx], 1.0 / D ** 0.5, O.Q8_0 if q8 else O.F32 if f32 else O.F16, Hkv,
            Hkv * row, row)
    ref = O.decode_batched(*args)
    truth = O.decode_batched(*args, mode=O.MODE_FP64)
    v = O.parity_verdict(out[idx].cpu().numpy(), ref, truth)
    v["sample"] = f"streams {idx} of {len(lens)} (every head), oracle ggml mode and fp64"
    return v


def check_encoder_layer(qkv_l, out_l):
    """Checker (outside every timed region): one timed encoder layer's output
    against the oracle's flash_attn_ext (ggml mode and fp64) on the same f16
    Q/K/V, judged by oracle.parity_verdict."""
    import numpy as np
    import oracle as O
    D = ENC["D"]
    q, k, v = (qkv_l[i].cpu().numpy() for i in range(3))            # (n, H, D) f16 each
    view = lambda a: a.transpose(1, 0, 2)[None]
    ref = O.flash_attn_ext(view(q), view(k), view(v), None, D ** -0.5)
    truth = O.flash_attn_ext(view(q), view(k), view(v), None, D ** -0.5, mode=O.MODE_FP64)
    v = O.parity_verdict(out_l.cpu().numpy(), ref, truth)
    v["sample"] = "layer 0 of the timed graph, all 20 heads x 1500 tokens, oracle ggml mode and fp64"
    return v


def run_decode(args, rank, world, local):
    import numpy as np
    import torch
    import vtx_attn

    dev = torch.device("cuda", local)
    S, Hq, Hkv, D = args.streams, DEC["Hq"], DEC["Hkv"], DEC["D"]
    kvname = getattr(args, "kv", "f16")
    q8 = kvname == "q8_0"
    f32 = kvname == "f32"
    row = D // 32 * 34 if q8 else D * (4 if f32 else 2)   # bytes of one head's K (or V) row
    lens, ks, vs, q = make_decode_inputs(S, "f32" if f32 else q8, 4321 + rank, 77 + rank, dev)
    kvt = vtx_attn.Q8_0 if q8 else vtx_attn.F32 if f32 else vtx_attn.F16
    plan = vtx_attn.DecodeBatchPlan(ks, vs, torch.from_numpy(lens).to(dev), Hq, Hkv, D, kvt, Hkv * row, row,
                                    int(lens.max()), 1.0 / D ** 0.5)
    out = torch.empty_like(q)
    stream = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(stream):
        for _ in range(max(1, args.warmup)):
            plan(q, out, stream)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        barrier(world)
        e0.record(stream)
        for _ in range(args.steps):
            plan(q, out, stream)
        e1.record(stream)
        torch.cuda.synchronize()
        barrier(world)
    ms_local = e0.elapsed_time(e1)
    ms = barrier_max(ms_local, world)
    kv_bytes = float(lens.astype(np.int64).sum()) * Hkv * row * 2
    value = kv_bytes * args.steps * world / (ms * 1e-3) / 1e9
    peaks = load_peaks()
    achieved = kv_bytes / (ms_local / args.steps * 1e-3) / 1e9
    parity = check_decode_rows(q, ks, vs, lens, out, kvname) \
        if (rank == 0 and not getattr(args, "no_check", False)) else None
    return {
        "parity": parity,
        "metric": METRIC_DEC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": kvname,
        "data": ("synthetic N(0,1) KV quantized to Q8_0 by ggml's rule (quantize_row_q8_0_ref)" if q8
                 else f"synthetic N(0,1) {kvname} KV")
                + ", ragged lengths U[512,16384] seeded per rank",
        "config": {"workload": f"configs[4] batched decode: {S} streams, GQA 32/8 x 128, "
                               f"{kvname.upper()} KV, 1 layer per step",
                   "l2": f"inputs larger than L2 ({kv_bytes / 1e9:.1f} GB KV per step)",
                   "parallelism": f"dp{world} (independent streams per GPU)"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / peaks["hbm_gbs"], 4),
                     # DRAM bytes per KV byte from the committed 32-stream ncu captures of the
                     # decode kernels: reads = algorithmic KV bytes, + partials
                     "traffic": round(kv_bytes * (DEC_TRAFFIC_RATIO_Q8 if q8 else DEC_TRAFFIC_RATIO_F16)),
                     "traffic_unit": "bytes per step (scaled from the capture by KV bytes)",
                     "peak_src": f"{peaks['src']} copy bandwidth"},
        "gpu_launches": args.steps * 2,
        "clocks": clocks.summary(),
    }


# ---- KV append (decoder cache update: RoPE + cache write) ---------------------------
def run_kv_append(args, rank, world, local):
    """vtx_kv_append on the decoder shape (GQA 32/8 x 128, RoPE base 1e6):
    (1) bandwidth: 8192 tokens per call (a long prefill chunk) into an F16 or
    Q8_0 cache, GB/s of algorithmic bytes (Q/K/V read, roped Q and cache rows
    written) against the HBM copy peak; (2) latency: the 256-stream decode
    step, one token per stream into its own cache (per-stream bases)."""
    import numpy as np
    import torch
    import vtx_attn

    dev = torch.device("cuda", local)
    q8 = getattr(args, "kv", "f16") == "q8_0"
    kvt = vtx_attn.Q8_0 if q8 else vtx_attn.F16
    Hq, Hkv, D = DEC["Hq"], DEC["Hkv"], DEC["D"]
    hb = D // 32 * 34 if q8 else D * 2
    g = torch.Generator(device=dev)
    g.manual_seed(91 + rank)
    T = 8192
    q = torch.randn((T, Hq, D), generator=g, device=dev)
    k = torch.randn((T, Hkv, D), generator=g, device=dev)
    v = torch.randn((T, Hkv, D), generator=g, device=dev)
    pos = torch.arange(T, dtype=torch.int32, device=dev) + 391
    slots = torch.arange(T, dtype=torch.int32, device=dev)
    kc = torch.empty((T, Hkv * hb), dtype=torch.uint8, device=dev)
    vc = torch.empty_like(kc)
    qo = torch.empty_like(q)
    stream = torch.cuda.Stream(device=dev)

    def call():
        vtx_attn.kv_append(k, v, pos, slots, kc, vc, kvt, 1e6, q=q, q_out=qo, stream=stream)

    with torch.cuda.stream(stream):
        for _ in range(max(3, args.warmup)):
            call()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    R = 10                                        # calls per step: a step is 10 x 8192 tokens (~0.7 ms)
    with ClockSampler(local) as clocks:
        barrier(world)
        e0.record(stream)
        for _ in range(args.steps * R):
            call()
        e1.record(stream)
        torch.cuda.synchronize()
        barrier(world)
    ms_local = e0.elapsed_time(e1) / (args.steps * R)
    ms = barrier_max(ms_local, world)
    nbytes = T * ((Hq + 2 * Hkv) * D * 4 + Hq * D * 4 + 2 * Hkv * hb)
    peaks = load_peaks()
    achieved = nbytes / (ms_local * 1e-3) / 1e9

    # 256-stream decode step: one token per stream, each into its own cache
    S = DEC["n_seq"]
    W = 8192
    caches_k = torch.empty((S, W, Hkv * hb), dtype=torch.uint8, device=dev)
    caches_v = torch.empty_like(caches_k)
    kp = torch.tensor([caches_k[i].data_ptr() for i in range(S)], dtype=torch.int64, device=dev)
    vp = torch.tensor([caches_v[i].data_ptr() for i in range(S)], dtype=torch.int64, device=dev)
    rng = np.random.default_rng(4321 + rank)
    lens = rng.integers(DEC["lo"], DEC["hi"] + 1, S)
    spos = torch.from_numpy(lens.astype(np.int32)).to(dev)
    sslot = torch.from_numpy((lens % W).astype(np.int32)).to(dev)
    sq, sk, sv = q[:S], k[:S], v[:S]
    sqo = torch.empty_like(sq)

    def step():
        vtx_attn.kv_append(sk, sv, spos, sslot, None, None, kvt, 1e6, q=sq, q_out=sqo, k_cache_ptrs=kp,
                           v_cache_ptrs=vp, cache_nb1=Hkv * hb, stream=stream)

    with torch.cuda.stream(stream):
        for _ in range(max(3, args.warmup)):
            step()
    torch.cuda.synchronize()
    # graph-captured so the host's per-call cost does not enter the device time
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for _ in range(10):
            step()
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        graph.replay()
        e0.record(stream)
        for _ in range(args.steps):
            graph.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    step_us = e0.elapsed_time(e1) / (args.steps * 10) * 1e3
    return {
        "metric": "KV append GB/s (decoder cache update)", "value": round(nbytes * world / (ms * 1e-3) / 1e9, 1),
        "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "q8_0" if q8 else "f16", "data": "synthetic N(0,1) f32 Q/K/V, seeded per rank",
        "config": {"workload": f"decoder KV append: {T} tokens x GQA 32/8 x 128, RoPE base 1e6, "
                               f"{'Q8_0' if q8 else 'f16'} cache rows, {R} calls per step (ms_per_step is one "
                               f"call); plus the {S}-stream decode step",
                   "parallelism": f"dp{world}"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / peaks["hbm_gbs"], 4), "traffic": None,
                     "per_call_bytes": int(nbytes)},
        "decode_step_us": round(step_us, 2),
        "gpu_launches": args.steps * (R + 10),
        "clocks": clocks.summary(),
    }


# ---- graph-replayed decode step (configs[2] and configs[3] decoders) --------------
def run_decode_step(args, rank, world, local):
    """The attention part of one decoded token for every layer (KV append +
    decode attention per layer, device counters advanced), replayed from a
    CUDA graph (decode_step.DecodeStepGraph), one stream (batch 1):
      30 layers, f16 cache, 391-token prefix, 200 steps;
      26 layers, Q8_0 cache, 7300-token prefix (window 8192), 200 steps.
    value = us per decoded token (graph); eager = the same calls from the host."""
    import numpy as np
    import torch
    import vtx_attn
    from decode_step import DecodeStepGraph

    dev = torch.device("cuda", local)
    res = {}
    for name, L, kvt, start, fused in (("configs[2]", 30, vtx_attn.F16, 391, True),
                                       ("configs[3]", 26, vtx_attn.Q8_0, 7300, True),
                                       ("configs[2]_two_calls", 30, vtx_attn.F16, 391, False),
                                       ("configs[3]_two_calls", 26, vtx_attn.Q8_0, 7300, False)):
        g = DecodeStepGraph(L, 1, DEC["Hq"], DEC["Hkv"], DEC["D"], kvt, 8192, [start], device=dev, fused=fused)
        gen = torch.Generator(device=dev)
        gen.manual_seed(61 + rank)
        for l in range(L):                                   # prefill rows
            k = torch.randn((start, DEC["Hkv"], DEC["D"]), generator=gen, device=dev)
            g.fill(l, 0, k, torch.randn_like(k), torch.arange(start, dtype=torch.int32))
        g.q.normal_(generator=gen)
        g.k.normal_(generator=gen)
        g.v.normal_(generator=gen)
        n = 200
        # every key bound the timed steps reach gets its plans and graph first
        # (a bound's first step runs eagerly and is captured), then the counters
        # rewind to the start
        for _ in range(n + max(3, args.warmup)):
            g.step()
        g.reset()
        for _ in range(max(3, args.warmup)):
            g.step()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(g.stream)
        for _ in range(n):
            g.step()
        e1.record(g.stream)
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) / n * 1e3
        e0.record(g.stream)
        for _ in range(20):
            g.step_eager()
        e1.record(g.stream)
        torch.cuda.synchronize()
        us_eager = e0.elapsed_time(e1) / 20 * 1e3
        kv = int(g.kv_len.item())
        row = g.row
        step_bytes = L * kv * row * 2
        res[name] = {"layers": L, "kv_type": "q8_0" if kvt == vtx_attn.Q8_0 else "f16", "kv_len_at_end": kv,
                     "launches_per_layer": 1 if fused else 3,
                     "us_per_token_graph": round(us, 1), "us_per_token_eager": round(us_eager, 1),
                     "us_per_layer_graph": round(us / L, 2), "kv_GBps_graph": round(step_bytes / (us * 1e-6) / 1e9, 1)}
        del g
        torch.cuda.empty_cache()
    peaks = load_peaks()
    main = res["configs[2]"]
    return {"metric": "decode step us/token (attention part, graph replay)", "value": main["us_per_token_graph"],
            "unit": "us", "n_gpus": world, "steps": 200, "warmup": args.warmup, "higher_is_better": False,
            "scaling": "weak", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic N(0,1) f32 Q/K/V projections, seeded",
            "config": {"workload": "batch-1 decode step, attention part of every layer: KV append (RoPE, ring "
                                   "write) + decode attention, counters advanced on the device; vtx_decode_layer "
                                   "(one launch per layer), and the two-call path (append, attention + merge) "
                                   "for comparison",
                       "parallelism": f"dp{world}"},
            "detail": res, "peak_hbm_gbs": peaks["hbm_gbs"], "gpu_launches": 200 * (30 * 1 + 1)}


# ---- decoder prefill (D = 128, causal GQA) ----------------------------
def run_prefill(args, rank, world, local):
    """The decoder's prefill attention (src/voxtral.cpp:1802 with n_tokens =
    n_kv and the causal mask of :2103-2111 as the causal flag), laid out as
    the reference lays it out: Q F32 [128, n, 32] (heads contiguous per
    token), K/V rows of the f16 cache (kv_dim 1024 per token, 8 KV heads x
    128).  configs[2]: 391 tokens (375 audio + 16 prompt), 30 layers, each
    layer with its own buffers, graph-replayed.  Also a long-context case
    (8192 tokens, 4 layers) for the same kernel at full occupancy."""
    import torch
    import vtx_attn

    dev = torch.device("cuda", local)
    Hq, Hkv, D = DEC["Hq"], DEC["Hkv"], DEC["D"]
    g = torch.Generator(device=dev)
    g.manual_seed(515 + rank)
    res = {}
    for name, n, L in (("configs[2]", 391, 30), ("long_context", 8192, 4)):
        q = torch.randn((L, n, Hq, D), generator=g, device=dev)
        kv = torch.randn((L, 2, n, Hkv, D), generator=g, device=dev).to(torch.float16)
        out = torch.empty((L, 1, n, Hq, D), device=dev)
        views = [(q[l].permute(1, 0, 2).unsqueeze(0), kv[l, 0].permute(1, 0, 2).unsqueeze(0),
                  kv[l, 1].permute(1, 0, 2).unsqueeze(0)) for l in range(L)]
        stream = torch.cuda.Stream(device=dev)

        def step():
            for l in range(L):
                qq, kk, vv = views[l]
                vtx_attn.flash_attn_ext(qq, kk, vv, None, D ** -0.5, causal=True, out=out[l], stream=stream)

        with torch.cuda.stream(stream):
            step()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            step()
        with torch.cuda.stream(stream):
            for _ in range(max(3, args.warmup)):
                graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(local) as clocks:
            barrier(world)
            e0.record(stream)
            with torch.cuda.stream(stream):
                for _ in range(args.steps):
                    graph.replay()
            e1.record(stream)
            torch.cuda.synchronize()
            barrier(world)
        ms = barrier_max(e0.elapsed_time(e1) / args.steps, world)
        flop = 4.0 * D * Hq * (n * (n + 1) // 2) * L
        res[name] = {"tokens": n, "layers": L, "ms_per_step": round(ms, 4),
                     "tflops": round(flop * world / (ms * 1e-3) / 1e12, 1), "us_per_layer": round(ms * 1e3 / L, 2),
                     "clocks": clocks.summary()}
        del q, kv, out, graph
        torch.cuda.empty_cache()
    peaks = load_peaks()
    main = res["configs[2]"]
    return {"metric": METRIC_ENC, "value": main["tflops"], "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": max(3, args.warmup), "ms_per_step": main["ms_per_step"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic N(0,1) Q (F32) and K/V (f16), seeded per rank",
            "config": {"workload": "configs[2] decoder prefill: 391 tokens causal, GQA 32/8 x 128, 30 layers "
                                   "(one step = the 30 layer calls, graph-replayed)",
                       "l2": "each layer has its own Q/K/V (8 MB per layer, 240 MB per step)",
                       "parallelism": f"dp{world}"},
            "roofline": {"bound": "tensor", "achieved": main["tflops"] / world, "peak": peaks["bf16_tflops"],
                         "unit": "TFLOP/s", "frac": round(main["tflops"] / world / peaks["bf16_tflops"], 4),
                         "traffic": None},
            "detail": res, "gpu_launches": args.steps * 30, "clocks": main["clocks"]}


# ---- realtime long-form streaming, attention path --------------------
def run_realtime(args, rank, world, local):
    """The attention work of 10 minutes of synthetic audio through the realtime
    model, per GPU (one independent utterance per rank):
      encoder: 60000 mel frames -> 39 chunks of <= 1500 tokens
               (vtx_encoder_chunk_plan, src/voxtral.cpp:2234-2335); each of the
               32 layers is ONE vtx_flash_attn_ext call with the chunks on the
               batch axis (32 heads x 64, causal + window 750, f16 Q/K/V per
               layer), then vtx_encoder_stitch gathers the chunks' new rows
               (the last layer's attention rows stand in for the encoder
               output that the reference stitches through host memory);
      decoder: 7500 tokens (one per 80 ms) over 26 layers, GQA 32/8 x 128,
               Q8_0 ring cache growing from 39 tokens: DecodeStepGraph replays
               (one vtx_decode_layer launch per layer: RoPE, ring write,
               decode attention; device counters).
    One step = the whole 10 minutes; value = audio-sec/sec = 600 x ranks /
    (max over ranks of the step time)."""
    import torch
    import vtx_attn
    from decode_step import DecodeStepGraph

    dev = torch.device("cuda", local)
    audio_s, mel = 600.0, 60000
    H, D, W, L_enc = 32, 64, 750, 32
    L_dec, start, n_tok = 26, 39, 7500
    chunks, total, used = vtx_attn.encoder_chunk_plan(mel)
    C = len(chunks)
    n = max(c.n_tokens for c in chunks)                       # 1500: shorter last chunks are padded (causal)
    g = torch.Generator(device=dev)
    g.manual_seed(303 + rank)
    # two alternating Q/K/V sets: one layer's 690 MB is far above L2 already
    qkv = torch.empty((2, 3, C, n, H, D), dtype=torch.float16, device=dev)
    for i in range(2):
        for j in range(3):
            qkv[i, j].copy_(torch.randn((C, n, H, D), generator=g, device=dev))
    out = torch.empty((C, n, H, D), device=dev)
    stitched = torch.empty((total, H * D), device=dev)
    views = [[qkv[l % 2, i].permute(0, 2, 1, 3) for i in range(3)] for l in range(L_enc)]   # (C, H, n, D)
    stream = torch.cuda.Stream(device=dev)

    def encoder():
        for l in range(L_enc):
            q, k, v = views[l]
            vtx_attn.flash_attn_ext(q, k, v, None, D ** -0.5, causal=True, window=W, out=out, stream=stream)
        vtx_attn.encoder_stitch(out.view(C, n, H * D), chunks, stitched, stream=stream)

    dec = DecodeStepGraph(L_dec, 1, DEC["Hq"], DEC["Hkv"], DEC["D"], vtx_attn.Q8_0, 8192, [start], device=dev)
    for l in range(L_dec):
        k = torch.randn((start, DEC["Hkv"], DEC["D"]), generator=g, device=dev)
        dec.fill(l, 0, k, torch.randn_like(k), torch.arange(start, dtype=torch.int32))
    dec.q.normal_(generator=g)
    dec.k.normal_(generator=g)
    dec.v.normal_(generator=g)
    dec.step()                                                # eager first step + graph capture
    torch.cuda.synchronize()
    steps_dec = n_tok - start
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]

    def pipeline(record: bool):
        dec.reset()
        stream.wait_stream(torch.cuda.current_stream(dev))
        if record:
            ev[0].record(stream)
        encoder()
        if record:
            ev[1].record(stream)
        dec.stream.wait_stream(stream)
        for _ in range(steps_dec):
            dec.step()
        stream.wait_stream(dec.stream)
        if record:
            ev[2].record(stream)

    for _ in range(max(3, args.warmup)):
        pipeline(False)
    torch.cuda.synchronize()
    t_enc = t_dec = 0.0
    with ClockSampler(local) as clocks:
        barrier(world)
        for _ in range(args.steps):
            pipeline(True)
            torch.cuda.synchronize()
            t_enc += ev[0].elapsed_time(ev[1])
            t_dec += ev[1].elapsed_time(ev[2])
        barrier(world)
    ms_local = (t_enc + t_dec) / args.steps
    ms = barrier_max(ms_local, world)
    pairs = sum(sum(min(i + 1, W) for i in range(c.n_tokens)) for c in chunks)
    enc_flop = 4.0 * D * H * pairs * L_enc
    kv_row = DEC["Hkv"] * (DEC["D"] // 32 * 34)
    dec_bytes = L_dec * kv_row * 2 * sum(min(t + 1, 8192) for t in range(start, n_tok))
    e_ms, d_ms = t_enc / args.steps, t_dec / args.steps
    return {"metric": "audio-sec/sec (realtime model, attention path)",
            "value": round(audio_s * world / (ms * 1e-3), 1), "unit": "audio-s/s", "n_gpus": world,
            "steps": args.steps, "warmup": max(3, args.warmup), "ms_per_step": round(ms, 2),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16 encoder / q8_0 KV",
            "data": "synthetic N(0,1) Q/K/V, seeded per rank (10 min of audio per rank)",
            "config": {"workload": f"configs[3] realtime: {audio_s:.0f} s audio = {mel} mel frames -> {C} encoder "
                                   f"chunks ({total} tokens, 32 layers, 32 heads x 64, causal + window 750, one "
                                   f"batched call per layer) + chunk stitch; {n_tok - start} decode steps x 26 "
                                   f"layers, GQA 32/8 x 128, Q8_0 ring cache {start} -> {n_tok} keys",
                       "l2": "an encoder layer reads 690 MB of Q/K/V (two alternating sets); the decoder reads "
                             "26 layers' caches (up to 424 MB) per token",
                       "parallelism": f"dp{world} (one utterance per GPU)"},
            "detail": {"encoder_ms": round(e_ms, 2), "encoder_tflops": round(enc_flop / (e_ms * 1e-3) / 1e12, 1),
                       "decoder_ms": round(d_ms, 2), "decoder_us_per_token": round(d_ms * 1e3 / (n_tok - start), 1),
                       "decoder_kv_GBps": round(dec_bytes / (d_ms * 1e-3) / 1e9, 1), "chunks": C,
                       "enc_tokens": total},
            "gpu_launches": args.steps * (L_enc + 1 + (n_tok - start) * (L_dec + 1)),
            "clocks": clocks.summary()}


# ---- one decode call of the decoder node, batch 1 ---------------------
def run_cfg0(args, rank, world, local):
    """the decode node of src/voxtral.cpp:1802 as ggml builds it
    (vtx_flash_attn_ext, n_q = 1): 32/8 heads x 128, 1024 keys, Q F32, K/V
    f16 rows of a [kv_dim = 1024, n_ctx] cache, scale 1/sqrt(128), no mask.
    GB/s over 64 rotating caches (268 MB > L2) replayed from a CUDA graph,
    the single call's device time in that graph, and its host-to-completion
    latency issued eagerly (median of 50)."""
    import numpy as np
    import torch
    import vtx_attn

    dev = torch.device("cuda", local)
    Hq, Hkv, D, n = 32, 8, 128, 1024
    NB = 64
    g = torch.Generator(device=dev)
    g.manual_seed(707 + rank)
    kc = torch.randn((NB, n, Hkv, D), generator=g, device=dev).to(torch.float16)
    vc = torch.randn((NB, n, Hkv, D), generator=g, device=dev).to(torch.float16)
    q = torch.randn((NB, 1, Hq, D), generator=g, device=dev)
    out = torch.empty((NB, 1, 1, Hq, D), device=dev)
    view = lambda t: t.permute(1, 0, 2).unsqueeze(0)             # (n, H, D) -> (1, H, n, D)
    scale = D ** -0.5
    ws = torch.empty(max(1, vtx_attn.workspace_bytes(view(q[0]), view(kc[0]), view(vc[0]), scale)),
                     dtype=torch.uint8, device=dev)
    stream = torch.cuda.Stream(device=dev)

    def call(i):
        vtx_attn.flash_attn_ext(view(q[i]), view(kc[i]), view(vc[i]), None, scale, out=out[i], workspace=ws,
                                stream=stream)

    with torch.cuda.stream(stream):
        for i in range(NB):
            call(i)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(NB):
            call(i)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(20):
            graph.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    us_graph = e0.elapsed_time(e1) / (20 * NB) * 1e3
    lat = []
    for i in range(50):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        call(i % NB)
        stream.synchronize()
        lat.append((time.perf_counter() - t0) * 1e6)
    kv_bytes = 2 * n * Hkv * D * 2
    peaks = load_peaks()
    res = {"workload": "configs[0] decode call: n_q 1, 32/8 heads x 128, 1024 keys, Q F32, K/V f16 cache rows",
           "us_per_call_graph": round(us_graph, 2), "us_per_call_eager_median": round(float(np.median(lat)), 2),
           "kv_GBps_rotating": round(kv_bytes / (us_graph * 1e-6) / 1e9, 1),
           "hbm_frac": round(kv_bytes / (us_graph * 1e-6) / 1e9 / peaks["hbm_gbs"], 4),
           "l2": f"{NB} rotating caches ({NB * kv_bytes / 1e6:.0f} MB > L2)"}
    if rank == 0 and not getattr(args, "no_check", False):
        import oracle as O
        qn, kn, vn = q[0].cpu().numpy(), kc[0].cpu().numpy(), vc[0].cpu().numpy()
        vw = lambda a: a.transpose(1, 0, 2)[None]
        v = O.parity_verdict(out[0].cpu().numpy(), O.flash_attn_ext(vw(qn), vw(kn), vw(vn), None, scale),
                             O.flash_attn_ext(vw(qn), vw(kn), vw(vn), None, scale, mode=O.MODE_FP64))
        res["parity"] = {k: v[k] for k in ("max_abs_err_vs_ggml", "max_abs_err_vs_fp64", "ok")}
    return res


# ---- the output projection after the attention node --------------------------------
def run_out_proj(args, rank, world, local):
    """vtx_attn_out_proj on the two projection shapes that follow the node:
    configs[1] encoder (1500 tokens, 20 x 64 -> 1280, + attn_o_bias +
    residual; 32 layers) and configs[2] decoder prefill (391 tokens, 32 x 128
    -> 3072, + residual; 30 layers), each layer with its own attention output,
    weight and residual (more than L2 per step), graph-replayed.  Two A
    operands: the attention's F32 result (ggml's node output, converted to
    f16 in the kernel) and its F16 result (vtx_flash_attn_ext with an F16
    dst: the same rounding done once in the attention epilogue), key
    "f16_attention".  Roofline: bytes = A + W (f16) + residual + output,
    FLOPs = 2 M N K; the bound is whichever takes longer at the measured
    peaks."""
    import torch
    import vtx_attn

    dev = torch.device("cuda", local)
    peaks = load_peaks()
    res = {}
    for name, (M, Hq, Dv, N, L, has_bias) in {"configs[1]_encoder": (1500, 20, 64, 1280, 32, True),
                                              "configs[2]_decoder_prefill": (391, 32, 128, 3072, 30, False)}.items():
        K = Hq * Dv
        g = torch.Generator(device=dev)
        g.manual_seed(900 + rank)
        A32 = torch.randn((L, 1, M, Hq, Dv), generator=g, device=dev) * 0.3
        W = (torch.randn((L, N, K), generator=g, device=dev) / K ** 0.5).half()
        R = torch.randn((L, M, N), generator=g, device=dev)
        Bv = torch.randn((L, N), generator=g, device=dev) if has_bias else None
        Y = torch.empty((L, M, N), device=dev)
        stream = torch.cuda.Stream(device=dev)

        def measure(A):
            def step():
                for l in range(L):
                    vtx_attn.out_proj(A[l], W[l], Bv[l] if has_bias else None, R[l], out=Y[l], stream=stream)

            with torch.cuda.stream(stream):
                step()
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                step()
            for _ in range(3):
                graph.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            reps = max(3, args.steps)
            with torch.cuda.stream(stream):
                e0.record(stream)
                for _ in range(reps):
                    graph.replay()
                e1.record(stream)
            torch.cuda.synchronize()
            del graph
            us = e0.elapsed_time(e1) / (reps * L) * 1e3
            flop = 2.0 * M * N * K
            nbytes = M * K * A.element_size() + N * K * 2 + 2 * M * N * 4 + (N * 4 if has_bias else 0)
            tflops = flop / (us * 1e-6) / 1e12
            gbps = nbytes / (us * 1e-6) / 1e9
            t_tensor, t_hbm = flop / (peaks["bf16_tflops"] * 1e12), nbytes / (peaks["hbm_gbs"] * 1e9)
            bound = "hbm" if t_hbm > t_tensor else "tensor"
            e = {"us_per_layer": round(us, 2), "tflops": round(tflops, 1), "GBps": round(gbps, 1), "bound": bound,
                 "frac_of_bound": round((t_hbm if bound == "hbm" else t_tensor) / (us * 1e-6), 4),
                 "tensor_frac": round(tflops / peaks["bf16_tflops"], 4),
                 "hbm_frac": round(gbps / peaks["hbm_gbs"], 4)}
            if rank == 0 and not getattr(args, "no_check", False):
                import oracle as O
                a0 = A32[0, 0].reshape(M, K).cpu().numpy()     # the oracle rounds it to f16 itself
                w0, r0 = W[0].cpu().numpy(), R[0].cpu().numpy()
                b0 = Bv[0].cpu().numpy() if has_bias else None
                v = O.parity_verdict(Y[0].cpu().numpy(), O.out_proj(a0, w0, b0, r0),
                                     O.out_proj(a0, w0, b0, r0, mode=O.MODE_FP64))
                e["parity"] = {k: v[k] for k in ("max_abs_err_vs_ggml", "max_abs_err_vs_fp64", "ok")}
            return e

        entry = {"M": M, "K": K, "N": N, "layers": L, "a": "F32 attention result"}
        entry.update(measure(A32))
        A16 = A32.half()
        entry["f16_attention"] = measure(A16)
        res[name] = entry
        del A32, A16, W, R, Y
        torch.cuda.empty_cache()
    return res


# ---- multi-GPU: configs[4] streams sharded by LPT, long prefill split by KV head ------
def run_decode_sharded(args, rank, world, local, kv="f16"):
    """configs[4]'s 256 ragged streams (the same streams at every N) placed on
    the ranks by LPT bin packing on kv_len (shard.lpt_shard); each rank decodes
    its streams (one layer per step), no collective on the data path.  Strong
    scaling: streams/sec = 256 / (max over ranks of the step time)."""
    import numpy as np
    import torch
    import shard
    import vtx_attn

    dev = torch.device("cuda", local)
    S, Hq, Hkv, D = DEC["n_seq"], DEC["Hq"], DEC["Hkv"], DEC["D"]
    q8 = kv == "q8_0"
    row = D // 32 * 34 if q8 else D * 2
    lens = np.random.default_rng(4321).integers(DEC["lo"], DEC["hi"] + 1, S).astype(np.int32)
    mine = shard.lpt_shard(lens.tolist(), world)[rank]
    ks, vs = [], []
    for i in mine:                                      # per-stream seeds: the same data at every N
        g = torch.Generator(device=dev)
        g.manual_seed(10_000 + int(i))
        x = torch.randn((int(lens[i]), Hkv, D), generator=g, device=dev)
        y = torch.randn((int(lens[i]), Hkv, D), generator=g, device=dev)
        ks.append(vtx_attn.quantize_q8_0(x) if q8 else x.half())
        vs.append(vtx_attn.quantize_q8_0(y) if q8 else y.half())
    ml = lens[mine]
    plan = vtx_attn.DecodeBatchPlan(ks, vs, torch.from_numpy(ml).to(dev), Hq, Hkv, D,
                                    vtx_attn.Q8_0 if q8 else vtx_attn.F16, Hkv * row, row, int(lens.max()),
                                    1.0 / D ** 0.5)
    q = torch.randn((len(mine), Hq, D), device=dev)
    out = torch.empty_like(q)
    stream = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(stream):
        for _ in range(3):
            plan(q, out, stream)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    steps = max(3, min(args.steps, 10))
    barrier(world)
    e0.record(stream)
    for _ in range(steps):
        plan(q, out, stream)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    ms = barrier_max(e0.elapsed_time(e1) / steps, world)
    kv_total = float(lens.astype(np.int64).sum()) * Hkv * row * 2
    mine_bytes = barrier_max(float(ml.astype(np.int64).sum()) * Hkv * row * 2, world)
    return {"workload": f"configs[4] 256 streams, {kv} KV, one layer per step, LPT-sharded over {world} GPU(s)",
            "scaling": "strong", "ms_per_step": round(ms, 4), "streams_per_sec": round(S / (ms * 1e-3), 1),
            "kv_GBps_aggregate": round(kv_total / (ms * 1e-3) / 1e9, 1),
            "max_rank_share": round(mine_bytes / kv_total, 4), "streams_on_rank0": len(mine)}


def run_prefill_head_split(args, rank, world, local):
    """Long-context prefill (8192 tokens, causal GQA 32/8 x 128, f16 Q/K/V)
    split by KV head over the ranks (shard.head_split_prefill: each rank's
    heads straight into its block of the gather buffer, one in-place NCCL
    all-gather).  Reports the step time, aggregate TFLOP/s and the share of
    the step the all-gather adds over the rank's attention alone."""
    import torch
    import vtx_attn

    dev = torch.device("cuda", local)
    n, Hq, Hkv, D = 8192, 32, 8, 128
    g = torch.Generator(device=dev)
    g.manual_seed(818)                                  # the same problem on every rank
    qkv = torch.randn((3, n, Hq, D), generator=g, device=dev).to(torch.float16)
    q = qkv[0].permute(1, 0, 2).unsqueeze(0)
    k = qkv[1, :, :Hkv].permute(1, 0, 2).unsqueeze(0)
    v = qkv[2, :, :Hkv].permute(1, 0, 2).unsqueeze(0)
    scale = D ** -0.5
    per = Hkv // world
    G = Hq // Hkv
    qs, ks_, vs_ = q[:, rank * per * G:(rank + 1) * per * G], k[:, rank * per:(rank + 1) * per], \
        v[:, rank * per:(rank + 1) * per]
    out_local = torch.empty((1, n, per * G, D), device=dev)
    stream = torch.cuda.current_stream(dev)

    def attn_only():
        vtx_attn.flash_attn_ext(qs, ks_, vs_, None, scale, causal=True, out=out_local)

    def step():
        if world == 1:
            return vtx_attn.flash_attn_ext(q, k, v, None, scale, causal=True)
        import shard
        return shard.head_split_prefill(q, k, v, None, scale, causal=True)

    def timed(fn, reps):
        for _ in range(2):
            fn()
        torch.cuda.synchronize()
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        barrier(world)
        return barrier_max(e0.elapsed_time(e1) / reps, world)

    reps = max(3, min(args.steps, 10))
    ms_step = timed(step, reps)
    ms_attn = timed(attn_only, reps)
    flop = 4.0 * D * Hq * (n * (n + 1) // 2)
    return {"workload": f"8192-token causal prefill, GQA 32/8 x 128, f16, KV heads split over {world} GPU(s)",
            "scaling": "strong", "ms_per_step": round(ms_step, 4), "tflops_aggregate": round(flop / (ms_step * 1e-3) / 1e12, 1),
            "ms_attention_only": round(ms_attn, 4),
            "allgather_share": round(max(0.0, 1.0 - ms_attn / ms_step), 4) if world > 1 else 0.0}


# ---- reference arm ------------------------------------------------------------------
def run_reference(args):
    """The reference arm: the CPU restatement of ggml's flash_attn_ext (the
    oracle, ggml mode) on the configs[1] encoder layer, every host core, rank
    0 only.  One step = one encoder layer (1500 x 1500 x 20 heads x 64, a
    bounded sample of the 32-layer clip); the same --steps / --warmup as the
    vtx arm."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    import numpy as np
    import oracle as O
    O.build()
    n, H, D = ENC["n"], ENC["H"], ENC["D"]
    rng = np.random.default_rng(5)
    view = lambda a: a.transpose(1, 0, 2)[None]
    cores = O.n_cores()
    layer = [rng.standard_normal((n, H, D)).astype(np.float16) for _ in range(3)]

    def one_layer():
        t0 = time.perf_counter()
        O.flash_attn_ext(view(layer[0]), view(layer[1]), view(layer[2]), None, D ** -0.5, threads=cores)
        return time.perf_counter() - t0

    for _ in range(args.warmup):
        one_layer()
    spent = sum(one_layer() for _ in range(args.steps))
    v = round(4.0 * D * H * n * n * args.steps / spent / 1e12, 6)
    cb = {"value": v, "unit": "TFLOP/s", "cores": cores, "kind": "port",
          "sample": f"{args.steps} configs[1] encoder layers (1500 x 1500 x 20 heads x 64), {spent:.1f} s on "
                    f"{cores} threads. " + CPU_PORT_NOTE}
    return {"impl": "reference", "metric": METRIC_ENC, "value": v, "unit": "TFLOP/s",
            "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(spent / args.steps * 1e3, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic N(0,1) f16 Q/K/V (BASELINE configs[1] shapes)",
            "config": {"workload": "configs[1] audio-encoder self-attention, 30 s clip: 1500 frames, 20 heads x 64, "
                                   "32 layers, bidirectional, batch 1 per GPU",
                       "reference": "CPU restatement of ggml-cpu flash_attn_ext (oracle/vtx_ref.c); ggml@5cecdad "
                                    "is fetched at configure time by the reference and is not present here"},
            "cpu_baseline": cb,
            "e2e": {"value": v, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="vtx", choices=["vtx", "reference"])
    ap.add_argument("--workload", default="encoder",
                    choices=["encoder", "decode", "kv_append", "decode_step", "realtime", "prefill"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-check", action="store_true", help="skip the oracle check of the timed outputs")
    ap.add_argument("--no-extra", action="store_true",
                    help="encoder workload: skip the other configs' sub-measurements")
    ap.add_argument("--no-decode", action="store_true", help="encoder workload: skip the decode sub-measurement")
    ap.add_argument("--streams", type=int, default=DEC["n_seq"], help="decode workload: streams per GPU")
    ap.add_argument("--kv", default="f16", choices=["f16", "q8_0", "f32"], help="decode workload: KV cache type")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)

    if args.impl == "reference":
        res = run_reference(args)
        if res is not None:
            print(json.dumps(res), flush=True)
        return

    import torch
    import vtx_attn
    vtx_attn.load()
    rank, world, local = dist_setup(args.gpus)
    if args.workload == "encoder":
        res = run_encoder(args, rank, world, local)
        if not args.no_decode:
            # the decode half of the metric (KV GB/s, configs[4]), timed after
            # and separately from the encoder steps above
            import copy
            dargs = copy.copy(args)
            dargs.steps, dargs.warmup = 5, 3
            for kv, key in (("f16", "decode"), ("q8_0", "decode_q8_0"), ("f32", "decode_f32")):
                dargs.kv = kv
                d = run_decode(dargs, rank, world, local)
                res[key] = {k: d[k] for k in ("metric", "value", "unit", "ms_per_step", "dtype", "roofline", "config",
                                              "data", "parity")}
                torch.cuda.empty_cache()
        if not args.no_extra:
            # the other BASELINE configs, each timed on its own after the
            # headline (sub-objects; at N > 1 every rank runs its own copy,
            # except the two sharded measurements, which split one problem)
            import copy
            xargs = copy.copy(args)
            xargs.steps, xargs.warmup = 5, 3
            res["cfg0_decode_call"] = run_cfg0(xargs, rank, world, local)
            pre = run_prefill(xargs, rank, world, local)
            res["cfg2_prefill"] = {k: pre[k] for k in ("metric", "value", "unit", "roofline", "detail")}
            ds = run_decode_step(xargs, rank, world, local)
            res["decode_step_batch1"] = {k: ds[k] for k in ("metric", "unit", "detail")}
            xargs.steps, xargs.warmup = 1, 1
            rt = run_realtime(xargs, rank, world, local)
            res["cfg3_realtime"] = {k: rt[k] for k in ("metric", "value", "unit", "ms_per_step", "detail", "config")}
            torch.cuda.empty_cache()
            xargs.steps = 5
            res["cfg4_decode_sharded"] = {kv: run_decode_sharded(xargs, rank, world, local, kv)
                                          for kv in ("f16", "q8_0")}
            torch.cuda.empty_cache()
            res["prefill_head_split"] = run_prefill_head_split(xargs, rank, world, local)
            res["out_proj"] = run_out_proj(xargs, rank, world, local)
        if rank == 0 and world == 1 and not args.no_cpu_baseline:
            res["cpu_baseline"] = cpu_baseline_encoder()
    else:
        res = {"decode": run_decode, "kv_append": run_kv_append, "decode_step": run_decode_step,
               "realtime": run_realtime, "prefill": run_prefill}[args.workload](args, rank, world, local)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
