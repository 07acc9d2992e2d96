"""Benchmark of the B200 dynamic causal depthwise convolution.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--workload prefill|decode|train|greta|all] [--shard requests|channels]

One JSON line on rank 0. The headline (`value`) is the varlen chunked prefill
with cache-slot state: 8 sequences with lengths ~U[32, 256] packed to <= 1024
tokens, C = 4096, K = 4, G = 1, bf16, state [64 slots, 4096, 3] read from 8
distinct random slots and written back. The decode step (256 one-token
requests, 1024 slots, 10% padding slots) and the training forward + backward
(8 x 4096 packed tokens, C = 4096, K = 4) are reported under "workloads", with
the same three paths at Greta's own layer shape (C = 2048, K = 7, G = 128,
norm and gate on) under "greta_layer".

Timing: W untimed warm-up steps, then exactly K steps between CUDA events on
the launching stream, bracketed by a barrier and torch.cuda.synchronize();
the time is the max over ranks. Prefill and decode inputs are smaller than
L2, so each step reads the next of several rotating input sets (> 2x L2 in
total) and the K launches are replayed from one CUDA graph. Training inputs
are larger than L2.

--impl reference times the reference algorithm on the host CPU cores (the
restated oracle in oracle/, all threads) on the same workload; under torchrun
only rank 0 runs it.

Multi-GPU: one process per GPU. --shard requests (default, weak scaling):
every rank serves its own batch of the same shape (no collective on the data
path). --shard channels (strong scaling): the 4096 channels are split across
ranks (column-parallel TP layout; no collective for the conv).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "dyn-conv tokens/s and % of B200 HBM peak (prefill fwd, train bwd, decode) at 1/2/4/8 GPUs"
L2_BYTES = 126 * 2 ** 20
FALLBACK_HBM_GBS = 6650.0


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def dram_traffic(channels=4096, train_seqs=8):
    """Per-launch DRAM bytes of the kernels from a committed ncu summary
    (captured at 4096 channels and 8 x 4096 training tokens), scaled to the
    channels and training tokens of this run (traffic is proportional to both)."""
    p = ROOT / "profiles" / "dram_traffic.json"
    if not p.exists():
        return {}
    d = {k: v for k, v in json.loads(p.read_text()).items() if not k.startswith("_")}
    scale = channels / 4096
    return {k: round(v * scale * (train_seqs / 8 if k.startswith("train") else 1)) for k, v in d.items()}


# ---------------------------------------------------------------------------
# clocks sampled during the timed work
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"greta_clocks_{os.getpid()}.csv"

    def __enter__(self):
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=self.fh, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.fh.close()

    def summary(self):
        if self.proc is None or not self.path.exists():
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        for line in self.path.read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append(dict(sm=float(parts[1]), smax=float(parts[2]), power=float(parts[3]),
                                 hw=parts[5], hwt=parts[6], swt=parts[7], swp=parts[8]))
            except ValueError:
                continue
        self.path.unlink(missing_ok=True)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        load = [r for r in rows if r["power"] > 250.0] or rows
        reasons = sorted({name for r in load for name, key in (("hw_slowdown", "hw"),
                                                                ("hw_thermal_slowdown", "hwt"),
                                                                ("sw_thermal_slowdown", "swt"),
                                                                ("sw_power_cap", "swp"))
                          if r[key].lower() == "active"})
        return {"sm_mhz": statistics.median(r["sm"] for r in load), "sm_max_mhz": max(r["smax"] for r in rows),
                "reasons": reasons, "samples": len(rows), "samples_under_load": len(load)}


# ---------------------------------------------------------------------------
# workloads (synthetic, seeded, reference layouts)
# ---------------------------------------------------------------------------
def prefill_lengths(gen, torch):
    while True:
        lengths = torch.randint(32, 257, (8,), generator=gen).tolist()
        if sum(lengths) <= 1024:
            return lengths


def make_prefill(torch, dev, seed, D=4096, W=4, G=1, n_slots=64, lengths=None):
    """One prefill batch. `lengths` (default: drawn from the seed) fixes the
    request lengths, so that rotating input sets hold the same batch shape
    with different values."""
    g = torch.Generator().manual_seed(seed)
    drawn = prefill_lengths(g, torch)
    lengths = list(lengths) if lengths is not None else drawn
    T = sum(lengths)
    slots = torch.randperm(n_slots, generator=g)[:8].to(torch.int32)
    gd = torch.Generator(device=dev).manual_seed(seed)
    return dict(
        x=torch.randn(T, D, device=dev, generator=gd).bfloat16(),
        w=(torch.randn(T, W, D // G, device=dev, generator=gd) * (1.0 / W) ** 0.5).bfloat16(),
        state=torch.randn(n_slots, D, W - 1, device=dev, generator=gd).bfloat16(),
        starts=torch.tensor([0] + list(_cumsum(lengths)), dtype=torch.int32, device=dev),
        slots=slots.to(dev), init=torch.ones(8, dtype=torch.int8, device=dev),
        y=torch.empty(T, D, device=dev, dtype=torch.bfloat16), T=T, N=8, D=D, W=W, G=G, lengths=lengths)


def make_decode(torch, dev, seed, D=4096, W=4, G=1, n_slots=1024, B=256):
    g = torch.Generator().manual_seed(seed)
    slots = torch.randperm(n_slots, generator=g)[:B]
    pad = torch.randperm(B, generator=g)[: round(0.1 * B)]
    slots[pad] = -1
    gd = torch.Generator(device=dev).manual_seed(seed)
    return dict(
        x=torch.randn(B, D, device=dev, generator=gd).bfloat16(),
        w=(torch.randn(B, W, D // G, device=dev, generator=gd) * (1.0 / W) ** 0.5).bfloat16(),
        state=torch.randn(n_slots, D, W - 1, device=dev, generator=gd).bfloat16(),
        starts=torch.arange(B + 1, dtype=torch.int32, device=dev), slots=slots.to(torch.int32).to(dev),
        init=torch.ones(B, dtype=torch.int8, device=dev), y=torch.empty(B, D, device=dev, dtype=torch.bfloat16),
        T=B, N=B, D=D, W=W, G=G, n_pad=len(pad))


def _cumsum(v):
    s, out = 0, []
    for a in v:
        s += a
        out.append(s)
    return out


def prefill_bytes(b):
    D, W, T, N, G = b["D"], b["W"], b["T"], b["N"], b["G"]
    per_token = 2 * D + 2 * W * D // G + 2 * D  # x, w, y
    return T * per_token + N * 2 * (2 * (W - 1) * D)  # + state read and write


def decode_bytes(b):
    D, W, B, G = b["D"], b["W"], b["T"], b["G"]
    live = B - b["n_pad"]
    per_live = 2 * D + 2 * W * D // G + 2 * D + 2 * 2 * (W - 1) * D
    per_pad = 2 * D + 2 * W * D // G + 2 * D
    return live * per_live + b["n_pad"] * per_pad


def packed_call(vc, b, out=None):
    return vc.packed_dynamic_conv_triton(b["x"], b["w"], None, b["state"], b["starts"], b["slots"], b["init"],
                                         b["G"], norm=False, eps=1e-6, out=b["y"] if out is None else out)


def hold_stream(torch, stream, us=200):
    """Keep `stream` busy on the device for about `us` microseconds, so that
    the host has submitted the work that follows before the start event after
    this fires: the timed window then holds GPU time only, not the host's
    submission latency (about 20 us for a graph replay)."""
    with torch.cuda.stream(stream):
        torch.cuda._sleep(int(us * 2.0e3))  # cycles at up to 2 GHz


LEAD = 2  # untimed launches ahead of the timed ones in a replayed graph


def time_graph(torch, sets, launch, steps, warmup, dist, spread=None):
    """Replay `steps` launches (rotating over `sets`) from one CUDA graph.
    Returns seconds for the K timed steps (max over ranks); `spread`, when
    given, receives the min / median / max over ranks."""
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        for i in range(max(warmup, 3)):
            launch(sets[i % len(sets)])
    torch.cuda.current_stream().wait_stream(stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    # Event nodes around the K timed launches time them on the device. LEAD
    # untimed launches come first in the same graph, so that the first timed
    # step, like every later one, follows a step of the same stream (a kernel
    # launched with programmatic dependent launch overlaps its start-up with
    # the end of the kernel ahead of it): the window holds K steps in steady
    # state, not the start-up of the graph's first kernel.
    first, last = (torch.cuda.Event(enable_timing=True, external=True),
                   torch.cuda.Event(enable_timing=True, external=True))
    with torch.cuda.graph(graph, stream=stream):
        for i in range(LEAD):
            launch(sets[(steps + i) % len(sets)])
        first.record()
        for i in range(steps):
            launch(sets[i % len(sets)])
        last.record()
    # warm replay (untimed), then the timed replay
    graph.replay()
    torch.cuda.synchronize()
    barrier(dist)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    hold_stream(torch, stream)
    start.record(stream)
    with torch.cuda.stream(stream):
        graph.replay()
    end.record(stream)
    end.synchronize()
    torch.cuda.synchronize()
    barrier(dist)
    outer = start.elapsed_time(end) / 1e3 * steps / (steps + LEAD)  # scaled to K steps
    inner = first.elapsed_time(last) / 1e3
    # the in-graph window when it is sane, else the held outer window
    sec = inner if 0 < inner <= outer * (steps + LEAD) / steps else outer
    del graph
    if spread is not None:
        spread.update(rank_spread(torch, dist, sec))
        spread["outer_window"] = rank_spread(torch, dist, outer)["max"]
    return reduce_max(torch, dist, sec)


def rank_spread(torch, dist, v):
    """min / median / max of a per-rank value over the ranks."""
    if dist is None:
        return {"min": v, "median": v, "max": v, "ranks": 1}
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    out = [torch.zeros_like(t) for _ in range(dist.get_world_size())]
    dist.all_gather(out, t)
    vals = sorted(float(o.item()) for o in out)
    return {"min": vals[0], "median": statistics.median(vals), "max": vals[-1], "ranks": len(vals)}


def barrier(dist):
    if dist is not None:
        dist.barrier()


def reduce_max(torch, dist, v):
    if dist is None:
        return v
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def n_sets(set_bytes):
    return max(2, math.ceil(2.5 * L2_BYTES / set_bytes))


def time_isolated(torch, sets, launch, steps, dist):
    """Per-call time of one launch with no programmatic-launch partner: each
    step writes a 2.5 x L2 buffer (an L2 flush standing in for the GEMMs
    around the conv in a model), then the call runs between two events. Plain
    launches, no graph; the device is held while the host submits, so the
    events time the kernel only. Returns the median step (max over ranks)."""
    stream = torch.cuda.current_stream()
    flush = torch.empty(int(2.5 * L2_BYTES) // 4, dtype=torch.float32, device="cuda")
    n = max(5, min(steps, 50))
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]
    for i in range(3):
        launch(sets[i % len(sets)])
    torch.cuda.synchronize()
    barrier(dist)
    for i in range(n):
        hold_stream(torch, stream, 100)
        flush.zero_()
        ev[i][0].record(stream)
        launch(sets[i % len(sets)])
        ev[i][1].record(stream)
    torch.cuda.synchronize()
    barrier(dist)
    med = statistics.median(a.elapsed_time(b) / 1e3 for a, b in ev)
    del flush
    return reduce_max(torch, dist, med)


# ---------------------------------------------------------------------------
# workload runners
# ---------------------------------------------------------------------------
def run_prefill(torch, vc, dev, args, dist, rank, world, peak, traffic):
    base_seed = 1000 + (rank if args.shard == "requests" else 0)
    sets = []
    probe = make_prefill(torch, dev, base_seed, D=args.channels)
    nbytes = prefill_bytes(probe)
    for i in range(n_sets(nbytes + probe["state"].numel() * 2)):
        sets.append(probe if i == 0 else make_prefill(torch, dev, base_seed + 97 * i, D=args.channels,
                                                      lengths=probe["lengths"]))
    steps = args.steps
    spread = {}
    sec = time_graph(torch, sets, lambda b: packed_call(vc, b), steps, args.warmup, dist, spread)
    iso = time_isolated(torch, sets, lambda b: packed_call(vc, b), steps, dist)
    T = probe["T"]
    per_step = sec / steps
    achieved = nbytes / per_step / 1e9
    return dict(tokens_per_step=T, ms_per_step=per_step * 1e3, tokens_per_s=T / per_step, bytes_per_step=nbytes,
                achieved_gbs=achieved, frac=achieved / peak, sets=len(sets), launches=steps + max(5, min(steps, 50)),
                us_per_step_over_ranks={k: (v / steps * 1e6 if k != "ranks" else v) for k, v in spread.items()},
                isolated=dict(us=iso * 1e6, frac=nbytes / iso / 1e9 / peak),
                lengths=probe["lengths"], traffic=traffic.get("prefill"), channels=args.channels)


def run_decode(torch, vc, dev, args, dist, rank, world, peak, traffic):
    base_seed = 2000 + (rank if args.shard == "requests" else 0)
    probe = make_decode(torch, dev, base_seed, D=args.channels)
    nbytes = decode_bytes(probe)
    set_bytes = nbytes + probe["state"].numel() * 2
    sets = [probe] + [make_decode(torch, dev, base_seed + 31 * i, D=args.channels) for i in range(1, n_sets(set_bytes))]
    steps = args.decode_steps
    spread = {}
    sec = time_graph(torch, sets, lambda b: packed_call(vc, b), steps, args.warmup, dist, spread)
    iso = time_isolated(torch, sets, lambda b: packed_call(vc, b), steps, dist)
    per_step = sec / steps
    achieved = nbytes / per_step / 1e9
    return dict(tokens_per_step=probe["T"], ms_per_step=per_step * 1e3, tokens_per_s=probe["T"] / per_step,
                bytes_per_step=nbytes, achieved_gbs=achieved, frac=achieved / peak, sets=len(sets),
                launches=steps + max(5, min(steps, 50)),
                us_per_step_over_ranks={k: (v / steps * 1e6 if k != "ranks" else v) for k, v in spread.items()},
                isolated=dict(us=iso * 1e6, frac=nbytes / iso / 1e9 / peak),
                traffic=traffic.get("decode"), channels=args.channels)


def run_channel_split(torch, vc, dev, args, dist, rank, world, peak):
    """Channel-split multi-GPU mode: the channels of ONE batch split over
    the ranks in contiguous, group-aligned shards (vLLM's column-parallel
    layout, greta_plugin_b200.sharding.channel_shard); every rank runs the
    kernels on its D/N channels of the same tokens, with no collective on the
    data path. Aggregate tokens/s = the batch's tokens / the slowest rank's
    step (strong scaling of the fixed batch); per-GPU fraction = a rank's
    bytes / its step / the copy peak."""
    import copy

    from greta_plugin_b200.sharding import channel_shard

    a = copy.copy(args)
    a.shard = "channels"
    a.channels = channel_shard(4096, 1, world, rank).channels
    out = {"ranks": world, "channels_per_rank": a.channels, "collective": None}
    for name, fn in (("prefill", run_prefill), ("decode", run_decode)):
        r = fn(torch, vc, dev, a, dist, rank, world, peak, {})
        out[name] = dict(tokens_per_step=r["tokens_per_step"], us_per_step=r["ms_per_step"] * 1e3,
                         tokens_per_s=r["tokens_per_s"], per_gpu_frac=r["frac"], per_gpu_gbs=r["achieved_gbs"],
                         isolated_us=r["isolated"]["us"], launches=r["launches"],
                         us_per_step_over_ranks=r["us_per_step_over_ranks"])
    out["launches"] = sum(out[k]["launches"] for k in ("prefill", "decode"))
    return out


def run_train(torch, dev, args, dist, rank, world, peak, traffic):
    """Training forward + backward through the C ABI (bf16, 8 x 4096 packed)."""
    from greta_plugin_b200 import _capi

    D, W, G, S, L = args.channels, 4, 1, args.train_seqs, 4096
    T = S * L
    gd = torch.Generator(device=dev).manual_seed(3000 + rank)
    x = torch.randn(T, D, device=dev, generator=gd).bfloat16()
    w = (torch.randn(T, W, D // G, device=dev, generator=gd) * 0.5).bfloat16()
    dout = torch.randn(T, D, device=dev, generator=gd).bfloat16()
    y, dx, dw = torch.empty_like(x), torch.empty_like(x), torch.empty_like(w)
    cu = torch.arange(0, T + 1, L, dtype=torch.int32, device=dev)
    lib = _capi.lib()
    stream = torch.cuda.current_stream()
    sp = _capi.stream_of(x)
    P = _capi.ptr

    def fwd():
        _capi.check("fwd", lib.greta_dynconv_fwd(_capi.DT_BF16, P(x), P(w), None, P(y), None, P(cu), 0, S, T, D, W, G,
                                                 0, 1e-6, sp))

    def bwd():
        _capi.check("bwd", lib.greta_dynconv_bwd(_capi.DT_BF16, P(x), P(w), None, None, P(dout), P(dx), P(dw), None,
                                                 P(cu), 0, S, T, D, W, G, 0, 1e-6, sp))

    for _ in range(max(args.warmup, 3)):
        fwd()
        bwd()
    torch.cuda.synchronize()
    barrier(dist)
    torch.cuda.synchronize()
    steps = args.train_steps
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3 * steps)]
    hold_stream(torch, stream)
    for i in range(steps):
        ev[3 * i].record(stream)
        fwd()
        ev[3 * i + 1].record(stream)
        bwd()
        ev[3 * i + 2].record(stream)
    torch.cuda.synchronize()
    barrier(dist)
    f_ms = sum(ev[3 * i].elapsed_time(ev[3 * i + 1]) for i in range(steps)) / steps
    b_ms = sum(ev[3 * i + 1].elapsed_time(ev[3 * i + 2]) for i in range(steps)) / steps
    total = ev[0].elapsed_time(ev[-1]) / 1e3
    total = reduce_max(torch, dist, total)
    f_ms = reduce_max(torch, dist, f_ms)
    b_ms = reduce_max(torch, dist, b_ms)
    fb, bb = T * 12 * D, T * 22 * D
    return dict(tokens_per_step=T, ms_per_step=total / steps * 1e3, tokens_per_s=T * steps / total,
                fwd_ms=f_ms, bwd_ms=b_ms, fwd_bytes=fb, bwd_bytes=bb,
                fwd_gbs=fb / f_ms / 1e6, bwd_gbs=bb / b_ms / 1e6,
                fwd_frac=fb / f_ms / 1e6 / peak, bwd_frac=bb / b_ms / 1e6 / peak,
                fwd_tokens_per_s=T / f_ms * 1e3, bwd_tokens_per_s=T / b_ms * 1e3, launches=2 * steps,
                traffic={"fwd": traffic.get("train_fwd"), "bwd": traffic.get("train_bwd")})


def run_greta(torch, vc, dev, args, dist, rank, world, peak):
    """Greta's own layer shape (configuration defaults: hidden 2048, kernel 7,
    128-channel filter groups, RMS norm and SiLU gate on), informational next to
    the headline shapes: vLLM prefill (the headline's 8 request lengths) and
    decode (256 requests) with cache-slot state and the overflow-safe norm, and
    the training forward (saving the pre-norm output) + backward on 8 x 4096
    tokens with the plain norm."""
    from greta_plugin_b200 import _capi

    D, W, G = 2048 // (world if args.shard == "channels" else 1), 7, 128
    wb = 2 * W * (D // G)  # filter bytes per token
    seed = 5000 + (rank if args.shard == "requests" else 0)

    def add_gate(b, s):
        b["gate"] = torch.randn(b["T"], D, device=dev, generator=torch.Generator(device=dev).manual_seed(s)).bfloat16()
        return b

    def call(b):
        return vc.packed_dynamic_conv_triton(b["x"], b["w"], b["gate"], b["state"], b["starts"], b["slots"],
                                             b["init"], G, norm=True, eps=1e-6, out=b["y"])

    out = {"channels": D, "kernel_size": W, "group_size": G, "norm": True, "gate": True}
    # prefill: x, gate, y per token, filters, old + new slot taps per request
    probe = add_gate(make_prefill(torch, dev, seed, D=D, W=W, G=G), seed)
    nb = probe["T"] * (6 * D + wb) + probe["N"] * 4 * (W - 1) * D
    sets = [probe] + [add_gate(make_prefill(torch, dev, seed + 97 * i, D=D, W=W, G=G, lengths=probe["lengths"]),
                               seed + 97 * i) for i in range(1, n_sets(nb + probe["state"].numel() * 2))]
    sec = time_graph(torch, sets, call, args.steps, args.warmup, dist) / args.steps
    out["prefill"] = dict(tokens=probe["T"], us=sec * 1e6, tokens_per_s=probe["T"] / sec, bytes=nb,
                          frac=nb / sec / 1e9 / peak)
    del sets, probe
    # decode: the same bytes per live request; padding rows skip the slot
    probe = add_gate(make_decode(torch, dev, seed + 1, D=D, W=W, G=G), seed + 1)
    live = probe["T"] - probe["n_pad"]
    nb = probe["T"] * (6 * D + wb) + live * 4 * (W - 1) * D
    sets = [probe] + [add_gate(make_decode(torch, dev, seed + 1 + 31 * i, D=D, W=W, G=G), seed + 1 + 31 * i)
                      for i in range(1, n_sets(nb + probe["state"].numel() * 2))]
    sec = time_graph(torch, sets, call, args.decode_steps, args.warmup, dist) / args.decode_steps
    out["decode"] = dict(tokens=probe["T"], us=sec * 1e6, tokens_per_s=probe["T"] / sec, bytes=nb,
                         frac=nb / sec / 1e9 / peak)
    del sets, probe
    # training
    S, L = args.train_seqs, 4096
    T = S * L
    gd = torch.Generator(device=dev).manual_seed(seed + 2)
    x = torch.randn(T, D, device=dev, generator=gd).bfloat16()
    g = torch.randn(T, D, device=dev, generator=gd).bfloat16()
    w = (torch.randn(T, W, D // G, device=dev, generator=gd) * (1.0 / W) ** 0.5).bfloat16()
    dout = torch.randn(T, D, device=dev, generator=gd).bfloat16()
    y, yr, dx, dg, dw = (torch.empty_like(x), torch.empty_like(x), torch.empty_like(x), torch.empty_like(x),
                         torch.empty_like(w))
    cu = torch.arange(0, T + 1, L, dtype=torch.int32, device=dev)
    lib, P, sp, stream = _capi.lib(), _capi.ptr, _capi.stream_of(x), torch.cuda.current_stream()

    def fwd():
        _capi.check("fwd", lib.greta_dynconv_fwd(_capi.DT_BF16, P(x), P(w), P(g), P(y), P(yr), P(cu), 0, S, T, D, W, G,
                                                 _capi.NORM_PLAIN, 1e-6, sp))

    def bwd():
        _capi.check("bwd", lib.greta_dynconv_bwd(_capi.DT_BF16, P(x), P(w), P(g), P(yr), P(dout), P(dx), P(dw), P(dg),
                                                 P(cu), 0, S, T, D, W, G, _capi.NORM_PLAIN, 1e-6, sp))

    for _ in range(max(args.warmup, 3)):
        fwd()
        bwd()
    torch.cuda.synchronize()
    barrier(dist)
    torch.cuda.synchronize()
    steps = args.train_steps
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3 * steps)]
    hold_stream(torch, stream)
    for i in range(steps):
        ev[3 * i].record(stream)
        fwd()
        ev[3 * i + 1].record(stream)
        bwd()
        ev[3 * i + 2].record(stream)
    torch.cuda.synchronize()
    barrier(dist)
    f_s = reduce_max(torch, dist, sum(ev[3 * i].elapsed_time(ev[3 * i + 1]) for i in range(steps)) / steps / 1e3)
    b_s = reduce_max(torch, dist, sum(ev[3 * i + 1].elapsed_time(ev[3 * i + 2]) for i in range(steps)) / steps / 1e3)
    fb = T * (8 * D + wb)  # x, gate read; y, yr written; filters
    bb = T * (12 * D + 2 * wb)  # x, gate, yr, dout read; dx, dg written; filters read, dw written
    out["train"] = dict(tokens=T, fwd_us=f_s * 1e6, bwd_us=b_s * 1e6, fwd_frac=fb / f_s / 1e9 / peak,
                        bwd_frac=bb / b_s / 1e9 / peak, fwd_bytes=fb, bwd_bytes=bb)
    out["launches"] = args.steps + args.decode_steps + 2 * steps
    return out


def run_tp_layer(torch, dev, args, dist, rank, world):
    """The whole GretaConv layer of a vLLM step (greta_vllm/model.py:115-124) at
    Greta's defaults (hidden 2048, W = 7, G = 128, norm + gate), split over the
    N ranks as tensor parallelism (greta_plugin_b200.tp): column-parallel
    in/gate/kernel projections, the B200 conv on D/N channels and the rank's
    state slice, row-parallel out_proj and an NCCL all-reduce of the layer
    output. Two projection forms: three GEMMs (the reference's) and one GEMM
    over the concatenated weights, whose output the conv reads in place.
    Decode (256 requests) and prefill (the headline's 8 request lengths);
    plain launches between events, max over ranks."""
    from greta_plugin_b200.tp import TPGretaConv, shard_layer_weights

    hidden, D, W, G = 2048, 2048, 7, 128
    Fn = D // G
    gw = torch.Generator(device=dev).manual_seed(777)  # the same layer on every rank
    sc = hidden ** -0.5
    full = [torch.randn(D, hidden, device=dev, generator=gw) * sc for _ in range(2)]
    kw = torch.randn(W * Fn, hidden, device=dev, generator=gw) * sc
    kb = torch.randn(W * Fn, device=dev, generator=gw) * 0.1
    ow = torch.randn(hidden, D, device=dev, generator=gw) * D ** -0.5
    wts = shard_layer_weights(full[0].bfloat16(), full[1].bfloat16(), kw.bfloat16(), kb.bfloat16(), ow.bfloat16(),
                              W, G, rank, world)
    del full, kw, kb, ow
    layers = {f: TPGretaConv(wts, W, G, True, 1e-6, world, None, None, fused=f) for f in (False, True)}
    out = {"hidden": hidden, "channels_per_rank": wts.hi - wts.lo, "kernel_size": W, "group_size": G,
           "ranks": world, "collective": "NCCL all-reduce of the out_proj partial sums" if world > 1 else None}
    steps = max(5, min(args.steps, 50))
    launches = 0
    for name in ("decode", "prefill"):
        g = torch.Generator().manual_seed(4000)
        if name == "decode":
            lengths = [1] * 256
            n_slots = 1024
        else:
            lengths = make_prefill(torch, "cpu", 5000, D=8, W=W, G=8)["lengths"]
            n_slots = 64
        T, N = sum(lengths), len(lengths)
        hs = torch.randn(T, hidden, generator=g).bfloat16().to(dev)
        starts = torch.tensor([0] + _cumsum(lengths), dtype=torch.int32, device=dev)
        slots = torch.randperm(n_slots, generator=g)[:N].to(torch.int32).to(dev)
        init = torch.ones(N, dtype=torch.int8, device=dev)
        state = torch.randn(n_slots, wts.hi - wts.lo, W - 1, generator=g).bfloat16().to(dev)
        res = {"tokens": T}
        for fused, layer in layers.items():
            # a serving step replays the layer from a CUDA graph (as vLLM
            # does), so the host's per-call Python and launch work is not
            # timed; the all-reduce is captured with the rest
            call = lambda _b, layer=layer: layer(hs, state, starts, slots, init)
            sec = time_graph(torch, [None], call, steps, args.warmup, dist) / steps
            res["fused_projection" if fused else "three_projections"] = dict(us=sec * 1e6, tokens_per_s=T / sec)
            launches += steps
        out[name] = res
    out["launches"] = launches
    return out


def run_train_layer(torch, dev, args, dist):
    """Greta's conv layer in training (the HF path) at its defaults, hidden
    2048, W = 7, G = 128, norm + gate, on 8 x 4096 packed tokens: forward and
    backward of the three input projections, the conv and out_proj, as the
    reference runs it (three GEMMs and their three backward GEMM pairs around
    dynamic_causal_conv1d) and with the projections fused into one GEMM whose
    output the conv reads in place and whose gradient the conv backward
    writes in place (greta_plugin_b200.fused_layer). Plain launches between
    events, max over ranks."""
    from greta_plugin_b200 import dynamic_causal_conv1d
    from greta_plugin_b200.fused_layer import FusedGretaConv

    hidden, D, W, G = 2048, 2048, 7, 128
    T = args.train_seqs * 4096
    torch.manual_seed(99)

    class Three(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.kernel_proj = torch.nn.Linear(hidden, (D // G) * W, bias=True)
            self.gate_proj = torch.nn.Linear(hidden, D, bias=False)
            self.in_proj = torch.nn.Linear(hidden, D, bias=False)
            self.out_proj = torch.nn.Linear(D, hidden, bias=False)
            self.kernel_size, self.group_size, self.norm, self.norm_eps = W, G, True, 1e-6

        def forward(self, h, cu):
            w = self.kernel_proj(h).view(h.shape[0], W, D // G)
            y = dynamic_causal_conv1d(self.in_proj(h)[None], w, self.gate_proj(h)[None], cu, G, True, 1e-6)
            return self.out_proj(y[0])

    three = Three().to(device=dev, dtype=torch.bfloat16)
    fused = FusedGretaConv.from_module(three)
    gd = torch.Generator(device=dev).manual_seed(98)
    h = (torch.randn(T, hidden, device=dev, generator=gd) * 0.5).bfloat16().requires_grad_()
    dout = torch.randn(T, hidden, device=dev, generator=gd).bfloat16()
    cu = torch.arange(0, T + 1, 4096, dtype=torch.int32, device=dev)
    out = {"hidden": hidden, "channels": D, "kernel_size": W, "group_size": G, "tokens": T}
    steps = max(3, min(args.train_steps, 10))
    stream = torch.cuda.current_stream()
    for name, layer in (("three_projections", three), ("fused_projection", fused)):
        def step():
            layer(h, cu).backward(dout)
        for _ in range(max(args.warmup, 3)):
            step()
        torch.cuda.synchronize()
        barrier(dist)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        hold_stream(torch, stream)
        ev[0].record(stream)
        for _ in range(steps):
            step()
        ev[1].record(stream)
        torch.cuda.synchronize()
        barrier(dist)
        sec = reduce_max(torch, dist, ev[0].elapsed_time(ev[1]) / 1e3 / steps)
        out[name] = dict(ms=sec * 1e3, tokens_per_s=T / sec)
    out["launches"] = 2 * 2 * steps  # conv forward + backward per step, both forms
    return out


def run_reference_triton(torch, dev, args, dist, peak):
    """The reference's own GPU kernels (Triton, from baseline/_ref, stock code
    path) on the same B200, shapes and timing windows as the B200 kernels:
    packed_dynamic_conv_triton (greta_vllm/triton_conv.py:128-173) on the
    headline prefill and decode and at Greta's layer shape; dynconv_fwd /
    dynconv_bwd (greta/dynamic_conv.py:786-864) on the training batch (their
    autotuner runs during the warm-up). Informational: the reference arm of
    the run is the CPU path."""
    ref = import_reference()
    if ref is None:
        return {"unavailable": "baseline/_ref is not installed"}
    if "triton_conv" not in ref:
        return {"unavailable": ref.get("triton_error", "triton_conv did not import")}
    rtc, rdc = ref["triton_conv"], ref["dynamic_conv"]
    out = {"source": "baseline/_ref (unmodified Garbo-AI/greta-plugin), Triton kernels"}
    D = args.channels

    def packed(b, G=1, norm=False):
        return rtc.packed_dynamic_conv_triton(b["x"], b["w"], b.get("gate"), b["state"], b["starts"], b["slots"],
                                              b["init"], G, norm=norm, eps=1e-6, out=b["y"])

    seed = 1000 + (int(os.environ.get("RANK", "0")) if args.shard == "requests" else 0)
    probe = make_prefill(torch, dev, seed, D=D)
    nb = prefill_bytes(probe)
    sets = [probe] + [make_prefill(torch, dev, seed + 97 * i, D=D, lengths=probe["lengths"])
                      for i in range(1, n_sets(nb + probe["state"].numel() * 2))]
    sec = time_graph(torch, sets, packed, args.steps, args.warmup, dist) / args.steps
    out["prefill"] = dict(tokens=probe["T"], us=sec * 1e6, tokens_per_s=probe["T"] / sec, frac=nb / sec / 1e9 / peak)
    del sets, probe
    probe = make_decode(torch, dev, 2000, D=D)
    nb = decode_bytes(probe)
    sets = [probe] + [make_decode(torch, dev, 2000 + 31 * i, D=D) for i in range(1, n_sets(nb + probe["state"].numel() * 2))]
    sec = time_graph(torch, sets, packed, args.decode_steps, args.warmup, dist) / args.decode_steps
    out["decode"] = dict(tokens=probe["T"], us=sec * 1e6, tokens_per_s=probe["T"] / sec, frac=nb / sec / 1e9 / peak)
    del sets, probe

    # Greta's layer shape on the packed path: D = 2048, W = 7, G = 128, norm + gate
    Dg, Wg, Gg = 2048 // (args.world if args.shard == "channels" else 1), 7, 128

    def with_gate(b, sd):
        b["gate"] = torch.randn(b["T"], Dg, device=dev, generator=torch.Generator(device=dev).manual_seed(sd)).bfloat16()
        return b

    gl = {}
    for name, mk, steps in (("prefill", make_prefill, args.steps), ("decode", make_decode, args.decode_steps)):
        probe = with_gate(mk(torch, dev, 5000, D=Dg, W=Wg, G=Gg), 5000)
        same = {"lengths": probe["lengths"]} if name == "prefill" else {}
        sets = [probe] + [with_gate(mk(torch, dev, 5000 + 31 * i, D=Dg, W=Wg, G=Gg, **same), 5000 + 31 * i)
                          for i in range(1, 6)]
        sec = time_graph(torch, sets, lambda b: packed(b, Gg, True), steps, args.warmup, dist) / steps
        gl[name] = dict(tokens=probe["T"], us=sec * 1e6, tokens_per_s=probe["T"] / sec)
        del sets, probe

    # training, both shapes: plain launches between events (the autotuner ran in the warm-up)
    def train(Dt, Wt, Gt, norm, gate_on, seed_t):
        S, L = args.train_seqs, 4096
        T = S * L
        gd = torch.Generator(device=dev).manual_seed(seed_t)
        x = torch.randn(1, T, Dt, device=dev, generator=gd).bfloat16()
        w = (torch.randn(T, Wt, Dt // Gt, device=dev, generator=gd) * (1.0 / Wt) ** 0.5).bfloat16()
        g = torch.randn(1, T, Dt, device=dev, generator=gd).bfloat16() if gate_on else None
        dout = torch.randn(1, T, Dt, device=dev, generator=gd).bfloat16()
        cu_cpu = torch.arange(0, T + 1, L, dtype=torch.int32)
        cu = cu_cpu.to(dev)
        state = {}

        def fwd():
            y, yr, BT, ci = rdc.dynconv_fwd(x, w, g, cu, Gt, norm=norm, eps=1e-6, save_pre=norm, cu_seqlens_cpu=cu_cpu)
            state.update(yr=yr, BT=BT, ci=ci)

        def bwd():
            rdc.dynconv_bwd(x, w, g, state["yr"], dout, cu, Gt, norm, 1e-6, state["BT"], state["ci"])

        stream = torch.cuda.current_stream()
        for _ in range(max(args.warmup, 3)):
            fwd()
            bwd()
        torch.cuda.synchronize()
        barrier(dist)
        steps = args.train_steps
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3 * steps)]
        for i in range(steps):
            hold_stream(torch, stream, 100)
            ev[3 * i].record(stream)
            fwd()
            ev[3 * i + 1].record(stream)
            bwd()
            ev[3 * i + 2].record(stream)
        torch.cuda.synchronize()
        barrier(dist)
        f = reduce_max(torch, dist, statistics.median(ev[3 * i].elapsed_time(ev[3 * i + 1]) for i in range(steps)))
        bk = reduce_max(torch, dist, statistics.median(ev[3 * i + 1].elapsed_time(ev[3 * i + 2]) for i in range(steps)))
        return dict(tokens=T, fwd_us=f * 1e3, bwd_us=bk * 1e3)

    tr = train(D, 4, 1, False, False, 3000)
    tr["fwd_frac"] = tr["tokens"] * 12 * D / (tr["fwd_us"] * 1e-6) / 1e9 / peak
    tr["bwd_frac"] = tr["tokens"] * 22 * D / (tr["bwd_us"] * 1e-6) / 1e9 / peak
    out["train"] = tr
    gl["train"] = train(Dg, Wg, Gg, True, True, 3100)
    out["greta_layer"] = gl
    return out


def run_hf(torch, dev, args, dist, rank, peak):
    """The HF plugin's two inference entry points (greta/dynamic_conv.py):
    single-token decode keyed by batch row with the in-place state shift
    (dynamic_causal_conv1d_decode, 256 rows) and the forward from an explicit
    context (dynamic_causal_conv1d_inference, 8 rows of 112 query tokens), at
    the headline shape (C=4096, K=4, G=1) and at Greta's layer shape (C=2048,
    K=7, G=128, plain norm and gate). Graph-replayed like prefill/decode,
    rotating over input sets of more than 2.5 x L2."""
    from greta_plugin_b200 import dynamic_causal_conv1d_decode, dynamic_causal_conv1d_inference

    out = {}
    seed = 6000 + (rank if args.shard == "requests" else 0)
    for shape, (D, W, G, norm) in (("headline", (args.channels, 4, 1, False)), ("greta_layer", (2048, 7, 128, True))):
        gate_on = norm
        F = D // G
        # decode rows: x, w, (gate), y per row; the row's state read and written
        B = 256
        per_set = B * (2 * D * (2 + gate_on) + 2 * W * F + 4 * (W - 1) * D)

        def dec_set(sd):
            gd = torch.Generator(device=dev).manual_seed(sd)
            return dict(x=torch.randn(B, D, device=dev, generator=gd).bfloat16(),
                        w=(torch.randn(B, W, F, device=dev, generator=gd) * (1.0 / W) ** 0.5).bfloat16(),
                        g=torch.randn(B, D, device=dev, generator=gd).bfloat16() if gate_on else None,
                        s=torch.randn(B, D, W - 1, device=dev, generator=gd).bfloat16())

        sets = [dec_set(seed + i) for i in range(n_sets(per_set))]
        sec = time_graph(torch, sets, lambda b: dynamic_causal_conv1d_decode(b["x"], b["w"], b["s"], b["g"], G, norm),
                         args.decode_steps, args.warmup, dist) / args.decode_steps
        r = {"decode_rows": dict(rows=B, us=sec * 1e6, tokens_per_s=B / sec, bytes=per_set,
                                 frac=per_set / sec / 1e9 / peak)}
        del sets
        # inference from context: context rows (W-1 history + Q), w, (gate), y
        Bq, Q = 8, 112
        per_set = Bq * (2 * (Q + W - 1) * D + Q * (2 * D * (1 + gate_on) + 2 * W * F))

        def inf_set(sd):
            gd = torch.Generator(device=dev).manual_seed(sd)
            return dict(c=torch.randn(Bq, Q + W - 1, D, device=dev, generator=gd).bfloat16(),
                        w=(torch.randn(Bq, Q, W, F, device=dev, generator=gd) * (1.0 / W) ** 0.5).bfloat16(),
                        g=torch.randn(Bq, Q, D, device=dev, generator=gd).bfloat16() if gate_on else None)

        sets = [inf_set(seed + 50 + i) for i in range(n_sets(per_set))]
        sec = time_graph(torch, sets, lambda b: dynamic_causal_conv1d_inference(b["c"], b["w"], b["g"], G, norm),
                         args.steps, args.warmup, dist) / args.steps
        r["inference"] = dict(rows=Bq, query=Q, tokens=Bq * Q, us=sec * 1e6, tokens_per_s=Bq * Q / sec,
                              bytes=per_set, frac=per_set / sec / 1e9 / peak)
        del sets
        r.update(channels=D, kernel_size=W, group_size=G, norm=norm, gate=gate_on)
        out[shape] = r
    out["launches"] = 2 * (args.decode_steps + args.steps)
    return out


def run_e2e_prefill(torch, vc, dev, args, dist):
    """Public API with host buffers: every step copies its inputs from pinned
    host memory (H2D), makes the call and copies the output back (D2H), all
    inside the timed region. Steps are pipelined the way a server would run
    them: the inputs are double-buffered on the device, H2D runs on one copy
    stream and D2H on another, so step i's D2H and kernel overlap step i+1's
    H2D on the full-duplex link; the calls stay in order on the current
    stream (they update the shared conv state in place)."""
    b = make_prefill(torch, dev, 1000 + (int(os.environ.get("RANK", "0")) if args.shard == "requests" else 0),
                     D=args.channels)  # the headline batch (898 tokens on rank 0)
    hx = b["x"].cpu().pin_memory()
    hw = b["w"].cpu().pin_memory()
    hs = b["starts"].cpu().pin_memory()
    hsl = b["slots"].cpu().pin_memory()
    hi = b["init"].cpu().pin_memory()
    hy = torch.empty(b["y"].shape, dtype=b["y"].dtype).pin_memory()
    host_in = (hx, hw, hs, hsl, hi)
    bufs = [tuple(torch.empty_like(t, device=dev) for t in host_in) for _ in range(2)]
    ys = [torch.empty_like(b["y"]) for _ in range(2)]
    state = b["state"]
    comp = torch.cuda.current_stream()
    up, down = torch.cuda.Stream(), torch.cuda.Stream()
    loaded = [torch.cuda.Event() for _ in range(2)]
    computed = [torch.cuda.Event() for _ in range(2)]
    free = [torch.cuda.Event() for _ in range(2)]
    for k in range(2):
        free[k].record(comp)

    def step(i):
        k = i % 2
        up.wait_event(free[k])  # the kernel and D2H of step i-2 are done with buffer k
        with torch.cuda.stream(up):
            for d, h in zip(bufs[k], host_in):
                d.copy_(h, non_blocking=True)
        loaded[k].record(up)
        comp.wait_event(loaded[k])
        dx, dw, ds, dsl, di = bufs[k]
        vc.packed_dynamic_conv_triton(dx, dw, None, state, ds, dsl, di, b["G"], norm=False, out=ys[k])
        computed[k].record(comp)
        down.wait_event(computed[k])
        with torch.cuda.stream(down):
            hy.copy_(ys[k], non_blocking=True)
        free[k].record(down)

    def drain():
        comp.wait_stream(up)
        comp.wait_stream(down)

    for i in range(max(args.warmup, 3)):
        step(i)
    drain()
    torch.cuda.synchronize()
    barrier(dist)
    torch.cuda.synchronize()
    steps = args.e2e_steps
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(comp)
    for k in range(2):  # the timed steps start from idle copy streams
        free[k].record(comp)
    for i in range(steps):
        step(i)
    drain()
    e.record(comp)
    e.synchronize()
    sec = reduce_max(torch, dist, s.elapsed_time(e) / 1e3)
    h2d = sum(t.numel() * t.element_size() for t in host_in)
    d2h = hy.numel() * hy.element_size()
    # the link's own rate for this step's copies: the same H2D copies alone,
    # back to back (pinned host memory -> device)
    torch.cuda.synchronize()
    barrier(dist)
    s.record(up)
    with torch.cuda.stream(up):
        for _ in range(steps):
            for d, h in zip(bufs[0], host_in):
                d.copy_(h, non_blocking=True)
    e.record(up)
    e.synchronize()
    h2d_sec = reduce_max(torch, dist, s.elapsed_time(e) / 1e3)
    return dict(tokens_per_s=b["T"] * steps / sec, h2d=h2d, d2h=d2h, launches=steps, tokens=b["T"],
                h2d_gbs=h2d * steps / sec / 1e9, h2d_copy_only_gbs=h2d * steps / h2d_sec / 1e9)


# ---------------------------------------------------------------------------
# CPU baselines (the oracle: the reference algorithm restated, host cores)
# ---------------------------------------------------------------------------
def cpu_prefill(seconds, threads):
    import numpy as np
    import torch

    from oracle import oracle

    b = make_prefill(torch, "cpu", 1000)
    x, w, st = (b[k].float().numpy() for k in ("x", "w", "state"))
    starts, slots, init = b["starts"].numpy(), b["slots"].numpy(), b["init"].numpy()
    oracle.packed(x[:64], w[:64], None, st, [0, 64], slots[:1], init[:1], 1, 0, threads=threads)  # warm
    n, t0 = 0, time.perf_counter()
    while True:
        oracle.packed(x, w, None, st, starts, slots, init, 1, 0, threads=threads)
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds or n >= 10000:
            break
    del np
    return dict(value=b["T"] * n / el, unit="tokens/s", cores=threads, kind="port",
                sample=f"{n} full prefill steps ({b['T']} tokens, C=4096, K=4, fp32 oracle) in {el:.1f} s",
                tokens=b["T"], lengths=b["lengths"])


def cpu_decode(seconds, threads):
    import torch

    from oracle import oracle

    b = make_decode(torch, "cpu", 2000)
    x, w, st = (b[k].float().numpy() for k in ("x", "w", "state"))
    starts, slots, init = b["starts"].numpy(), b["slots"].numpy(), b["init"].numpy()
    n, t0 = 0, time.perf_counter()
    while True:
        oracle.packed(x, w, None, st, starts, slots, init, 1, 0, threads=threads)
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds or n >= 100000:
            break
    return dict(value=b["T"] * n / el, unit="tokens/s", cores=threads, kind="port",
                sample=f"{n} decode steps (256 rows, 1024 slots) in {el:.1f} s")


def cpu_train(seconds, threads):
    """One 4096-token sequence of the training batch, fwd + bwd (bounded sample)."""
    import numpy as np

    from oracle import oracle

    rng = np.random.default_rng(0)
    L, D, W = 4096, 4096, 4
    x = rng.standard_normal((L, D), dtype=np.float32)
    w = (rng.standard_normal((L, W, D), dtype=np.float32) * 0.5)
    dy = rng.standard_normal((L, D), dtype=np.float32)
    n, t0 = 0, time.perf_counter()
    while True:
        oracle.fwd(x, w, None, None, 1, 0, threads=threads)
        oracle.bwd(x, w, None, dy, None, 1, 0, threads=threads)
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds or n >= 1000:
            break
    return dict(value=L * n / el, unit="tokens/s", cores=threads, kind="port",
                sample=f"{n} fwd+bwd passes over one 4096-token sequence (of 8) in {el:.1f} s")


REF_DIR = ROOT / "baseline" / "_ref"


def import_reference():
    """Import the unmodified reference installed in baseline/_ref (the driver's
    offline install of Garbo-AI/greta-plugin); None when it is not there."""
    if not (REF_DIR / "greta_vllm" / "conv.py").is_file():
        return None
    if str(REF_DIR) not in sys.path:
        sys.path.insert(0, str(REF_DIR))
    import greta.dynamic_conv as rdc
    import greta_vllm.conv as rconv

    out = {"conv": rconv, "dynamic_conv": rdc}
    try:
        import greta_vllm.triton_conv as rtc

        out["triton_conv"] = rtc
    except Exception as exc:  # Triton missing: the CPU path still runs
        out["triton_error"] = f"{type(exc).__name__}: {exc}"
    return out


def cpu_model():
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return None


def cpu_prefill_reference(seconds, threads):
    """The reference's own CPU path on the headline prefill: its pure-torch
    packed_dynamic_conv (greta_vllm/conv.py:10-70) from baseline/_ref, fp32
    inputs, all host threads, a fresh state clone per step (the call updates
    the state in place). None when the reference is not installed."""
    import torch

    ref = import_reference()
    if ref is None:
        return None
    torch.set_num_threads(threads)
    b = make_prefill(torch, "cpu", 1000)
    x, w, st0 = (b[k].float() for k in ("x", "w", "state"))
    starts, slots, init = b["starts"], b["slots"], b["init"]
    fn = ref["conv"].packed_dynamic_conv
    fn(x[:64], w[:64], None, st0.clone(), torch.tensor([0, 64], dtype=torch.int32), slots[:1], init[:1], 1,
       norm=False)  # warm
    n, t0 = 0, time.perf_counter()
    while True:
        fn(x, w, None, st0.clone(), starts, slots, init, 1, norm=False)
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds or n >= 10000:
            break
    return dict(value=b["T"] * n / el, unit="tokens/s", cores=threads, kind="reference", cpu_model=cpu_model(),
                sample=f"{n} full prefill steps ({b['T']} tokens, C=4096, K=4) of greta_vllm.conv.packed_dynamic_conv"
                       f" (fp32, torch {torch.__version__}, {threads} threads) in {el:.1f} s",
                tokens=b["T"], lengths=b["lengths"])


def host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


# ---------------------------------------------------------------------------
def parse():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--workload", choices=["prefill", "decode", "train", "greta", "hf", "tp", "layer", "all"],
                    default="all")
    ap.add_argument("--shard", choices=["requests", "channels"], default="requests")
    ap.add_argument("--decode-steps", type=int, default=None)
    ap.add_argument("--train-steps", type=int, default=None)
    ap.add_argument("--e2e-steps", type=int, default=None)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-reference-triton", action="store_true",
                    help="skip timing the reference's Triton kernels on the GPU (informational leg)")
    ap.add_argument("--ncu", action="store_true",
                    help="profiling mode: plain launches (no CUDA graph), no e2e or CPU arm, no JSON line")
    ap.add_argument("--train-seqs", type=int, default=8,
                    help="4096-token sequences in the training batch (8 = the full configuration)")
    a = ap.parse_args()
    a.channels = 4096
    a.decode_steps = a.decode_steps or a.steps
    a.train_steps = a.train_steps or max(3, min(a.steps, 20))
    a.e2e_steps = a.e2e_steps or max(3, min(a.steps, 200))
    return a


def config_block(args, world, prefill, greta=None):
    par = f"{args.shard} x{world}" if world > 1 else "single GPU"
    if greta is not None:  # --workload greta: the layer-shape prefill leads
        return {"workload": "varlen chunked prefill with cache-slot state, Greta layer shape (vLLM packed path)",
                "seqs": 8, "tokens": greta["prefill"]["tokens"], "channels": greta["channels"],
                "kernel_size": greta["kernel_size"], "group_size": greta["group_size"], "norm": True, "gate": True,
                "state_slots": 64, "l2": "rotating input sets (> 2x L2)", "parallelism": par}
    return {"workload": "varlen chunked prefill with cache-slot state (vLLM packed path)",
            "seqs": 8, "tokens": prefill["tokens_per_step"] if prefill else None,
            "lengths": prefill.get("lengths") if prefill else None,
            "channels": args.channels, "kernel_size": 4, "group_size": 1, "norm": False, "gate": False,
            "state_slots": 64,
            "l2": (f"rotating {prefill['sets']} input sets (> 2x L2)" if prefill and isinstance(prefill.get("sets"), int)
                   else (prefill or {}).get("sets", "?")),
            "parallelism": par}


def profile_launches(args):
    """--ncu: each selected workload's kernels launched `steps` times after
    `warmup` launches, on plain streams, so that ncu sees ordinary launches
    (`greta`: the layer-shape training forward + backward, D=2048, W=7,
    G=128, plain norm and gate)."""
    import torch

    from greta_plugin_b200 import _capi
    from greta_plugin_b200 import vllm_conv as vc

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    n = args.warmup + args.steps
    if args.workload in ("prefill", "all"):
        b = make_prefill(torch, dev, 1000, D=args.channels)
        for _ in range(n):
            packed_call(vc, b)
    if args.workload in ("decode", "all"):
        b = make_decode(torch, dev, 2000, D=args.channels)
        for _ in range(n):
            packed_call(vc, b)
    if args.workload in ("train", "all"):
        D, W, G, L = args.channels, 4, 1, 4096
        T = args.train_seqs * L
        gd = torch.Generator(device=dev).manual_seed(3000)
        x = torch.randn(T, D, device=dev, generator=gd).bfloat16()
        w = (torch.randn(T, W, D, device=dev, generator=gd) * 0.5).bfloat16()
        dout = torch.randn(T, D, device=dev, generator=gd).bfloat16()
        y, dx, dw = torch.empty_like(x), torch.empty_like(x), torch.empty_like(w)
        cu = torch.arange(0, T + 1, L, dtype=torch.int32, device=dev)
        lib, P, sp = _capi.lib(), _capi.ptr, _capi.stream_of(x)
        for _ in range(n):
            _capi.check("fwd", lib.greta_dynconv_fwd(_capi.DT_BF16, P(x), P(w), None, P(y), None, P(cu), 0,
                                                     args.train_seqs, T, D, W, G, 0, 1e-6, sp))
            _capi.check("bwd", lib.greta_dynconv_bwd(_capi.DT_BF16, P(x), P(w), None, None, P(dout), P(dx), P(dw),
                                                     None, P(cu), 0, args.train_seqs, T, D, W, G, 0, 1e-6, sp))
    if args.workload == "greta":  # Greta's layer shape: training forward + backward, plain norm and gate
        D, W, G, L = 2048, 7, 128, 4096
        T = args.train_seqs * L
        gd = torch.Generator(device=dev).manual_seed(3100)
        x = torch.randn(T, D, device=dev, generator=gd).bfloat16()
        g = torch.randn(T, D, device=dev, generator=gd).bfloat16()
        w = (torch.randn(T, W, D // G, device=dev, generator=gd) * (1.0 / W) ** 0.5).bfloat16()
        dout = torch.randn(T, D, device=dev, generator=gd).bfloat16()
        y, yr, dx, dg, dw = (torch.empty_like(x), torch.empty_like(x), torch.empty_like(x), torch.empty_like(x),
                             torch.empty_like(w))
        cu = torch.arange(0, T + 1, L, dtype=torch.int32, device=dev)
        lib, P, sp = _capi.lib(), _capi.ptr, _capi.stream_of(x)
        for _ in range(n):
            _capi.check("fwd", lib.greta_dynconv_fwd(_capi.DT_BF16, P(x), P(w), P(g), P(y), P(yr), P(cu), 0,
                                                     args.train_seqs, T, D, W, G, _capi.NORM_PLAIN, 1e-6, sp))
            _capi.check("bwd", lib.greta_dynconv_bwd(_capi.DT_BF16, P(x), P(w), P(g), P(yr), P(dout), P(dx), P(dw),
                                                     P(dg), P(cu), 0, args.train_seqs, T, D, W, G, _capi.NORM_PLAIN,
                                                     1e-6, sp))
    torch.cuda.synchronize()


def main():
    args = parse()
    if args.ncu:
        profile_launches(args)
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    args.channels = 4096 // world if (args.shard == "channels" and world > 1) else 4096
    args.world = world

    if args.impl == "reference":
        if rank != 0:
            return
        threads = host_threads()
        # the reference's own CPU code (baseline/_ref), else its restatement
        res = cpu_prefill_reference(min(args.cpu_seconds, 30.0), threads) or cpu_prefill(min(args.cpu_seconds, 30.0),
                                                                                          threads)
        line = {"metric": METRIC, "value": res["value"], "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": 1e3 * res["tokens"] / res["value"], "higher_is_better": True,
                "scaling": "weak" if args.shard == "requests" else "strong", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic (seeded N(0,1) inputs in the reference layouts)", "impl": "reference",
                "source": ("greta_vllm.conv.packed_dynamic_conv from baseline/_ref (the reference's own torch CPU path)"
                           if res["kind"] == "reference" else "oracle/ (the reference algorithm restated in C)"),
                "config": config_block(args, 1, {"tokens_per_step": res.pop("tokens"),
                                                 "lengths": res.pop("lengths"),
                                                 "sets": "one input set in host memory (CPU run, no GPU L2)"}),
                "cpu_baseline": res,
                "e2e": {"value": res["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line))
        return

    import torch

    dist = None
    if world > 1:
        import torch.distributed as tdist
        from datetime import timedelta

        torch.cuda.set_device(local)
        tdist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
        dist = tdist
    else:
        torch.cuda.set_device(0)
    dev = torch.device("cuda", torch.cuda.current_device())
    from greta_plugin_b200 import vllm_conv as vc

    peak, peak_kind = peaks()
    traffic = dram_traffic(args.channels, args.train_seqs)
    out = {}
    with ClockSampler(dev.index) as clocks:
        if args.workload in ("prefill", "all"):
            out["prefill"] = run_prefill(torch, vc, dev, args, dist, rank, world, peak, traffic)
        if args.workload in ("decode", "all"):
            out["decode"] = run_decode(torch, vc, dev, args, dist, rank, world, peak, traffic)
        if args.workload in ("train", "all"):
            out["train"] = run_train(torch, dev, args, dist, rank, world, peak, traffic)
        if args.workload in ("greta", "all"):
            out["greta_layer"] = run_greta(torch, vc, dev, args, dist, rank, world, peak)
        if args.workload in ("hf", "all"):
            out["hf"] = run_hf(torch, dev, args, dist, rank, peak)
        if args.workload in ("tp", "all"):
            out["tp_layer"] = run_tp_layer(torch, dev, args, dist, rank, world)
        if args.workload in ("layer", "all"):
            out["train_layer"] = run_train_layer(torch, dev, args, dist)
        if world > 1 and args.shard == "requests" and args.workload in ("prefill", "all"):
            out["channel_split"] = run_channel_split(torch, vc, dev, args, dist, rank, world, peak)
        e2e = run_e2e_prefill(torch, vc, dev, args, dist) if args.workload in ("prefill", "all") else None
    clk = clocks.summary()
    if args.workload == "all" and not args.no_reference_triton and world == 1:
        try:
            out["reference_triton"] = run_reference_triton(torch, dev, args, dist, peak)
        except Exception as exc:  # informational leg: report, do not fail the run
            out["reference_triton"] = {"error": f"{type(exc).__name__}: {exc}"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and args.workload in ("prefill", "all"):
        port = cpu_prefill(args.cpu_seconds, host_threads())
        port.pop("tokens"), port.pop("lengths")
        port["cpu_model"] = cpu_model()
        cpu = cpu_prefill_reference(args.cpu_seconds, host_threads())
        if cpu is None:
            cpu = port
        else:
            cpu.pop("tokens"), cpu.pop("lengths")
            cpu["port"] = port
        if args.workload == "all":
            out.setdefault("decode", {})["cpu_baseline"] = cpu_decode(min(3.0, args.cpu_seconds), host_threads())
            out.setdefault("train", {})["cpu_baseline"] = cpu_train(min(10.0, args.cpu_seconds), host_threads())

    if dist is not None:
        dist.barrier()
    if rank == 0:
        head = out.get("prefill")
        launches = sum(v.get("launches", 0) for v in out.values()) + (e2e["launches"] if e2e else 0)
        if head is None and "greta_layer" in out and len(out) == 1:  # --workload greta: its prefill leads
            gp = out["greta_layer"]["prefill"]
            head = dict(tokens_per_s=gp["tokens_per_s"], ms_per_step=gp["us"] / 1e3,
                        achieved_gbs=gp["bytes"] / gp["us"] / 1e3, frac=gp["frac"])
        if head is None and set(out) == {"hf"}:  # --workload hf: the headline-shape decode rows lead
            hd = out["hf"]["headline"]["decode_rows"]
            head = dict(tokens_per_s=hd["tokens_per_s"], ms_per_step=hd["us"] / 1e3,
                        achieved_gbs=hd["bytes"] / hd["us"] / 1e3, frac=hd["frac"])
        if head is None and set(out) == {"train_layer"}:  # --workload layer: the fused training layer leads
            tl = out["train_layer"]["fused_projection"]
            head = dict(tokens_per_s=tl["tokens_per_s"], ms_per_step=tl["ms"], achieved_gbs=None, frac=None)
        if head is None and set(out) == {"tp_layer"}:  # --workload tp: the fused decode layer leads
            td = out["tp_layer"]["decode"]["fused_projection"]
            head = dict(tokens_per_s=td["tokens_per_s"], ms_per_step=td["us"] / 1e3, achieved_gbs=None, frac=None)
        if head is None:  # a single non-prefill workload was asked for
            key = next(iter(out))
            head = out[key]
            head.setdefault("achieved_gbs", head.get("bwd_gbs"))
            head.setdefault("frac", head.get("bwd_frac"))
        scale = world if args.shard == "requests" else 1
        line = {
            "metric": METRIC,
            "value": head["tokens_per_s"] * scale,
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": head["ms_per_step"],
            "higher_is_better": True,
            "scaling": "weak" if args.shard == "requests" else "strong",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) inputs in the reference layouts)",
            "config": config_block(args, world, out.get("prefill"),
                                   out["greta_layer"] if set(out) == {"greta_layer"} else None),
            "roofline": {"bound": "hbm", "achieved": head["achieved_gbs"], "peak": peak, "unit": "GB/s",
                         "frac": head["frac"], "traffic": head.get("traffic"),
                         "peak_source": f"{peak_kind} copy bandwidth (MEASURED_PEAKS.json hbm_gbs)"
                         if peak_kind == "measured" else "fallback 6.65 TB/s",
                         "frac_of_8tbs_spec": None if head["achieved_gbs"] is None else head["achieved_gbs"] / 8000.0},
            "cpu_baseline": cpu,
            "e2e": None if e2e is None else {"value": e2e["tokens_per_s"] * scale, "unit": "tokens/s",
                                             "h2d_bytes_per_step": e2e["h2d"], "d2h_bytes_per_step": e2e["d2h"],
                                             "tokens_per_step": e2e["tokens"], "h2d_gbs_per_gpu": e2e["h2d_gbs"],
                                             "h2d_copy_only_gbs_per_gpu": e2e["h2d_copy_only_gbs"],
                                             "bound": "host-to-device copies (PCIe)"},
            "gpu_launches": launches,
            "clocks": clk,
            "workloads": out,
        }
        print(json.dumps(line))
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
