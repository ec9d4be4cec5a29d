"""Throughput of the fused Mamba S6 block forward on B200 (tokens/s = B*T / s).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config 0|1|2|3]

Workload (default --config 0): one Mamba S6 block forward in float32,
d_model=768, d_inner=1536, d_state=24, d_conv=4, dt_rank=48, batch 151 x 180
tokens -- the shape the headline target is quoted on.  Synthetic seeded data:
x ~ N(0,1); Kaiming-uniform linear weights; conv ~ U(-0.5, 0.5);
A_log = log(1..S); D = 1; dt_proj.bias = softplus^-1(log-uniform[1e-3, 0.1]).
Other configs are measurement aids: 1 = bf16 B=8 T=8192 (S=16); 2 = stateful
decode B=64 (d_model 1024): metric over forward_step calls; 3 = int8 weights
(--quant int4 / nf4 for the others), d_model 1536, B=32 T=2048; 4 = 24-layer
RMSNorm pre-norm residual stack in
bf16 (d_model 768, S=16), B=1024 x T=2048 split across the ranks (strong
scaling; tokens/s counts tokens through all 24 layers).

Multi-GPU: one process per GPU (torchrun); each rank runs its own batch
(weak scaling, no data-path collective); time = max over ranks of the
CUDA-event time of the K timed steps.  Inputs rotate over >= 4 buffers whose
total exceeds the 126 MB L2, and every step moves > 1 GB through HBM.

--impl reference times the reference's CPU implementation on the host cores,
on the same workload (config 0: all 151 x 180 tokens per step): the block
composition in torch CPU ops (the same ATen calls the reference makes) around
the reference's own compiled C++ scan op from oracle/_ref; without that op the
arm prints an "unavailable" line.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import torch

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "fused Mamba block tokens/s (B·T/s) at 1/2/4/8 B200; % of HBM roofline"
L2_BYTES = 126 * 2 ** 20

CONFIGS = {
    0: dict(workload="mamba_block_fwd_f32_b151_t180", d_model=768, d_state=24, batch=151,
            seqlen=180, dtype="f32", mode="forward"),
    1: dict(workload="mamba_block_fwd_bf16_b8_t8192", d_model=768, d_state=16, batch=8,
            seqlen=8192, dtype="bf16", mode="forward"),
    2: dict(workload="mamba_block_step_f32_b64_dm1024", d_model=1024, d_state=16, batch=64,
            seqlen=512, dtype="f32", mode="step", dt_rank=64),
    3: dict(workload="mamba_block_fwd_int8_b32_t2048_dm1536", d_model=1536, d_state=16,
            batch=32, seqlen=2048, dtype="f32", mode="forward", quant="int8", dt_rank=96),
    4: dict(workload="mamba_stack24_rmsnorm_fwd_bf16_b1024_t2048", d_model=768, d_state=16,
            batch=1024, seqlen=2048, dtype="bf16", mode="stack", n_layers=24),
}


def peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return d["hbm_gbs"], d["bf16_tflops"], d.get("bf16_tflops_sustained", d["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, 1400.0, "fallback"


# ----------------------------------------------------------------- helpers
def dist_env():
    from cpu_mamba_b200 import dist
    return dist.env()


class ClockSampler:
    """nvidia-smi samples (every 25 ms) of the GPU's clocks and throttle
    reasons.  Started before the warm-up so that it is already sampling when
    the timed region begins; summary() keeps the samples whose arrival time
    lies in the timed region (widened by one interval on each side, so that a
    region shorter than the interval still has its nearest samples)."""

    PERIOD_MS = 25
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: torch.device):
        try:
            self.index = "GPU-" + str(torch.cuda.get_device_properties(device).uuid)
        except Exception:
            self.index = str(device.index or 0)
        self.proc = None
        self.lines = []
        self.t0 = self.t1 = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", str(self.PERIOD_MS)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.perf_counter(), line.strip()))

    def begin(self):
        self.t0 = time.perf_counter()

    def end(self):
        self.t1 = time.perf_counter()

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        # samples inside the timed region (give or take one period); a region
        # shorter than nvidia-smi's actual cadence takes the samples nearest it
        for pad_ms in (self.PERIOD_MS, 100, 250):
            r = self._summary(pad_ms / 1e3)
            if r is not None:
                r["window_pad_ms"] = pad_ms
                return r
        return None

    def _summary(self, pad):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for t, ln in list(self.lines):
            if self.t0 is None or self.t1 is None or not (self.t0 - pad <= t <= self.t1 + pad):
                continue
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm), "period_ms": self.PERIOD_MS}


def make_params(cfg, seed):
    """Seeded synthetic block parameters (same recipe as the oracle's generator,
    restated here so the product path does not import the oracle)."""
    g = torch.Generator().manual_seed(seed)
    dm, S = cfg["d_model"], cfg["d_state"]
    di = 2 * dm
    R = cfg.get("dt_rank", math.ceil(dm / 16))

    def lin(o, i):
        if cfg.get("quant"):
            w = torch.randn(o, i, generator=g) * 0.02
            m = torch.rand(o, i, generator=g) < 0.01
            return torch.where(m, torch.where(torch.rand(o, i, generator=g) < 0.5, -0.5, 0.5), w)
        b = 1.0 / math.sqrt(i)
        return (torch.rand(o, i, generator=g) * 2 - 1) * b

    p = {"in_proj.weight": lin(2 * di, dm),
         "conv1d.weight": torch.rand(di, 1, 4, generator=g) - 0.5,
         "conv1d.bias": torch.rand(di, generator=g) - 0.5,
         "x_proj.weight": lin(R + 2 * S, di), "dt_proj.weight": lin(di, R),
         "out_proj.weight": lin(dm, di),
         "A_log": torch.log(torch.arange(1, S + 1, dtype=torch.float32).repeat(di, 1)),
         "D": torch.ones(di)}
    u = torch.rand(di, generator=g)
    dt = torch.exp(u * (math.log(0.1) - math.log(1e-3)) + math.log(1e-3))
    p["dt_proj.bias"] = dt + torch.log(-torch.expm1(-dt))
    return p, R


def make_stack(cfg):
    """The residual stack with every layer's block drawn as make_params draws
    one (seed = layer index) and RMSNorm weights of one (their init)."""
    from cpu_mamba_b200 import MambaStack
    n, dm = cfg["n_layers"], cfg["d_model"]
    sd = {}
    for i in range(n):
        p, R = make_params(cfg, seed=i)
        sd[f"layers.{i}.norm.weight"] = torch.ones(dm)
        sd.update({f"layers.{i}.mixer.{k}": v for k, v in p.items()})
    m = MambaStack(n, dm, d_state=cfg["d_state"], dt_rank=R, eps=1e-5).eval()
    m.load_state_dict(sd, strict=True)
    return m, R


def stack_roofline(cfg, batch, hbm_gbs, src, ms_per_step):
    """Whole-stack HBM fraction: per layer the four-stage block bytes plus the
    norm pass (x read) and the residual (x read in out_proj's epilogue)."""
    c = dict(cfg, batch=batch)
    es = 4 if cfg["dtype"] == "f32" else 2
    per_layer = realistic_block_bytes(c) + 2 * batch * cfg["seqlen"] * cfg["d_model"] * es
    nbytes = per_layer * cfg["n_layers"]
    ach = nbytes / (ms_per_step / 1e3) / 1e9
    return {"kernel": f"stack of {cfg['n_layers']} layers (7 launches each)", "bound": "hbm",
            "achieved": ach, "peak": hbm_gbs, "unit": "GB/s", "frac": ach / hbm_gbs,
            "traffic": None, "bytes_per_step": nbytes, "peak_source": f"{src} HBM copy"}


# ------------------------------------------------------------- our arm
def run_ours(args, cfg):
    from cpu_mamba_b200 import CPUMamba, QuantConfig, StepGraph, quantize_block
    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    from cpu_mamba_b200 import dist
    dist.init("nccl", dev)
    dtype = torch.float32 if cfg["dtype"] == "f32" else torch.bfloat16
    stack_mode = cfg["mode"] == "stack"
    if stack_mode:
        m, R = make_stack(cfg)
        m = m.to(device=dev, dtype=dtype)
        lo, hi = dist.shard(cfg["batch"], ws, rank)
        B = hi - lo                            # strong scaling: the batch is sharded
    else:
        p, R = make_params(cfg, seed=0)
        m = CPUMamba(cfg["d_model"], d_state=cfg["d_state"], dt_rank=R).eval()
        m.load_state_dict(p, strict=True)
        m = m.to(device=dev, dtype=dtype)
        if cfg.get("quant"):
            quantize_block(m, QuantConfig(cfg["quant"]))
        B = cfg["batch"]
    channels = args.shard == "channels" and not stack_mode
    reducer = None
    if channels:
        # every rank runs the whole batch on its d_inner channels (strong scaling)
        from cpu_mamba_b200.shard import ChannelShardedMamba, PeerReducer
        if args.reduce == "peer" and ws > 1:
            reducer = PeerReducer(max_elems=1 << 22)
        m = ChannelShardedMamba(m, reduce=reducer)
    T, dm = cfg["seqlen"], cfg["d_model"]
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    step_mode = cfg["mode"] == "step"
    in_shape = (B, dm) if step_mode else (B, T, dm)
    in_bytes = math.prod(in_shape) * (4 if dtype == torch.float32 else 2)
    nbuf = 8 if step_mode else max(2 if stack_mode else 4, math.ceil(2 * L2_BYTES / in_bytes))
    xs = [torch.randn(in_shape, generator=g, device=dev).to(dtype) for _ in range(nbuf)]
    state = None
    if step_mode:
        with torch.no_grad():
            g_prompt = torch.Generator(device=dev).manual_seed(99)     # same prompt on all ranks
            prompt = torch.randn(B, T, dm, generator=g_prompt if channels else g,
                                 device=dev).to(dtype)
            _, state = m.forward_with_final_state(prompt)
    if channels:          # every rank feeds the same tokens
        g_in = torch.Generator(device=dev).manual_seed(1234)
        xs = [torch.randn(in_shape, generator=g_in, device=dev).to(dtype) for _ in range(nbuf)]

    graph = StepGraph(m, state, xs[0]) if step_mode else None   # decode: one graph per step

    def step(i):
        with torch.no_grad():
            if step_mode:
                return graph(xs[i % nbuf])
            return m(xs[i % nbuf])

    stream = torch.cuda.current_stream(dev)
    clk = ClockSampler(dev).start()          # sampling before the timed region starts
    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize(dev)
    dist.barrier()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clk.begin()
    e0.record(stream)
    for i in range(args.steps):
        step(i)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    clk.end()
    clk.stop()
    dist.barrier()
    ms = dist.max_over_ranks(e0.elapsed_time(e1), dev)      # the slowest rank's time
    tokens_per_step = B * (1 if step_mode else T)
    # whole job: batch shards add up; channel shards all process the same tokens
    tokens_all = tokens_per_step if channels else dist.sum_over_ranks(tokens_per_step, dev)
    value = tokens_all * args.steps / (ms / 1e3)

    # end to end through the public API from pinned host buffers
    host_in = torch.empty(in_shape, dtype=dtype, pin_memory=True)
    host_in.copy_(xs[0].cpu())
    host_out = torch.empty(in_shape, dtype=dtype, pin_memory=True)
    e2e_ms = []
    for i in range(max(3, min(args.steps, 10)) + 1):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        step_e2e(m, host_in, host_out, graph, step_mode, dev, channels)
        b.record(stream)
        torch.cuda.synchronize(dev)
        if i > 0:
            e2e_ms.append(a.elapsed_time(b))
    e2e_t = dist.max_over_ranks(statistics.median(e2e_ms), dev)
    e2e = {"value": tokens_all / (e2e_t / 1e3), "unit": "tokens/s",
           "h2d_bytes_per_step": in_bytes, "d2h_bytes_per_step": in_bytes}

    stages = (profile_stages(m, xs[0], cfg, dtype, args.steps)
              if cfg["mode"] == "forward" and not channels else {})
    launches_per_step, launch_names = count_launches(lambda: step(0), dev)
    result = None
    if rank == 0:
        hbm, bf16, bf16_s, src = peaks()
        if stack_mode:
            roof = stack_roofline(cfg, B, hbm, src, ms / args.steps)
        elif step_mode:
            roof = decode_roofline(cfg, hbm, src, ms / args.steps, ws if channels else 1)
        else:
            roof = roofline(stages, cfg, hbm, bf16, src, ms / args.steps)
        par = f"batch-sharded x{ws}"
        if channels:
            par = (f"d_inner channel-sharded x{ws}, all-reduce: "
                   f"{'peer-memory kernel' if reducer is not None else 'NCCL'}" if ws > 1
                   else "d_inner channel-sharded x1")
        result = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True,
            "scaling": "strong" if stack_mode or channels else "weak",
            "vs_baseline": None,
            "dtype": cfg["dtype"], "data": "synthetic (seeded; shapes of the configuration)",
            "config": dict(workload_config(cfg, B, int(tokens_all) // (1 if step_mode else T),
                                           ws_label=par),
                           l2=f"inputs rotated over {nbuf} buffers "
                              f"({nbuf * in_bytes / 2**20:.0f} MB > L2)"),
            "roofline": roof, "stages_ms": stages, "e2e": e2e,
            "gpu_launches": launches_per_step * args.steps,
            "gpu_launches_per_step": launch_names,
            "clocks": clk.summary(),
        }
    del graph                       # graphs holding collectives go before the group
    if reducer is not None:
        reducer.close()
    dist.shutdown()
    return result


def count_launches(fn, dev):
    """The library's kernel launches in one untimed call of fn (one step),
    counted by CUPTI through torch.profiler: kernels of the mb2 namespaces
    (torch's own kernels, copies and memsets excluded).  Returns the count and
    a per-kernel breakdown {short name: launches}."""
    from torch.profiler import ProfilerActivity, profile
    torch.cuda.synchronize(dev)
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize(dev)
    names = {}
    for e in prof.events():
        if e.device_type != torch.autograd.DeviceType.CUDA:
            continue
        n = e.name
        if "mb2::" not in n:
            continue
        short = n.split("(")[0].replace("void ", "").split("<")[0].split("::")[-1]
        names[short] = names.get(short, 0) + 1
    return sum(names.values()), names


def workload_config(cfg, batch_per_gpu, global_batch, ws_label):
    """The line's ``config``: the workload and its sizes (both arms)."""
    step_mode = cfg["mode"] == "step"
    dm = cfg["d_model"]
    return {"workload": cfg["workload"], "batch_per_gpu": batch_per_gpu,
            "global_batch": global_batch, "seq_len": 1 if step_mode else cfg["seqlen"],
            "d_model": dm, "d_inner": 2 * dm, "d_state": cfg["d_state"],
            "dt_rank": cfg.get("dt_rank", math.ceil(dm / 16)), "quant": cfg.get("quant"),
            "parallelism": ws_label, "layers": cfg.get("n_layers", 1),
            "decode": "forward_step captured as one CUDA graph" if step_mode else None}


def step_e2e(m, host_in, host_out, graph, step_mode, dev, channels=False):
    """One step through the public API from pinned host memory to pinned host
    memory.  A forward streams batch slices with the copies overlapping the
    kernels (CPUMamba.forward_host); a decode step copies the token in,
    replays the captured step (CPUMamba.capture_step) and copies the output
    out."""
    with torch.no_grad():
        if step_mode:
            y = graph(host_in.to(dev, non_blocking=True))
            host_out.copy_(y, non_blocking=True)
        elif channels:
            host_out.copy_(m(host_in.to(dev, non_blocking=True)), non_blocking=True)
        else:
            m.forward_host(host_in, out=host_out)


STAGES = ("in_proj", "conv1d_silu", "x_proj", "dt_proj", "scan", "out_proj")


def profile_stages(m, x, cfg, dtype, steps):
    """Per-stage CUDA-event durations of the block forward's own launches
    (mb2_block_forward_profile: events between its six stages on one
    stream), averaged over up to 20 forwards after one untimed one; quantised
    blocks included (their stages hold the per-call code conversions)."""
    times = {k: [] for k in STAGES}
    n = max(3, min(steps, 20))
    with torch.no_grad():
        for it in range(n + 1):
            st = m.profile_stages(x)
            if it > 0:
                for k in STAGES:
                    times[k].append(st[k])
    return {k: statistics.mean(v) for k, v in times.items()}


# DRAM bytes (read + write) per token of each launch of the fp32 block at
# d_model 768, d_state 24: ncu's dram__bytes_read.sum and dram__bytes_write.sum
# of one launch over batch 64 x 180 tokens (11,520 rows), divided by the rows.
# Every tensor these kernels touch grows with the token count, so a full-size
# launch moves (bytes per token) x N.  (dt_proj's output mostly stays in L2
# at batch 64, so its figure under-counts a full-size launch.)
TRAFFIC_PER_TOKEN = {
    ("f32", 768, 24, "in_proj"): (54.38208e6 + 96.968192e6) / 11520,
    ("f32", 768, 24, "x_proj"): (71.99104e6 + 1.200896e6) / 11520,
    ("f32", 768, 24, "dt_proj"): (4.326656e6 + 15.051264e6) / 11520,
    ("f32", 768, 24, "out_proj"): (80.250624e6 + 14.976e6) / 11520,
    ("f32", 768, 24, "scan"): (215.583232e6 + 42.584064e6) / 11520,
    ("f32", 768, 24, "conv1d_silu"): (71.217152e6 + 26.989824e6) / 11520,
}


def realistic_block_bytes(cfg):
    """HBM bytes of one block forward for a four-stage fused design (in_proj |
    conv + x_proj | dt_proj + scan + gate | out_proj), each stage reading and
    writing its tensors once: es x (2 d_model + 7 d_inner + 2 (R + 2S)) per
    token, plus the weights once (config 0: 49,920 B per token, 1.372 GB)."""
    B, T, dm, S = cfg["batch"], cfg["seqlen"], cfg["d_model"], cfg["d_state"]
    di = 2 * dm
    R = cfg.get("dt_rank", math.ceil(dm / 16))
    es = 4 if cfg["dtype"] == "f32" else 2
    N = B * T
    xd = R + 2 * S
    act = N * es * (2 * dm + 7 * di + 2 * xd)
    w = es * (2 * di * dm + xd * di + di * R + dm * di)
    return act + w


def decode_roofline(cfg, hbm_gbs, src, ms_per_step, shards):
    """A decode step against HBM: every weight read once, h (fp32) and the
    conv state read and written once, per GPU (channel shards each hold
    1/shards of all of them); the token rows in and out are negligible."""
    B, dm, S = cfg["batch"], cfg["d_model"], cfg["d_state"]
    di = 2 * dm
    R = cfg.get("dt_rank", math.ceil(dm / 16))
    es = 4 if cfg["dtype"] == "f32" else 2
    w = es * (2 * di * dm + (R + 2 * S) * di + di * R + dm * di)
    state = 2 * (B * di * S * 4 + B * di * 3 * es)
    nbytes = (w + state) / shards
    ach = nbytes / (ms_per_step / 1e3) / 1e9
    return {"kernel": "decode step (all launches)", "bound": "hbm", "achieved": ach,
            "peak": hbm_gbs, "unit": "GB/s", "frac": ach / hbm_gbs, "traffic": None,
            "bytes_per_step_per_gpu": nbytes, "peak_source": f"{src} HBM copy"}


def roofline(stages, cfg, hbm_gbs, bf16_tflops, src, ms_per_step):
    if not stages:
        return None
    B, T, dm, S = cfg["batch"], cfg["seqlen"], cfg["d_model"], cfg["d_state"]
    di = 2 * dm
    R = cfg.get("dt_rank", math.ceil(dm / 16))
    es = 4 if cfg["dtype"] == "f32" else 2
    N = B * T
    flops = {"in_proj": 2 * N * dm * 2 * di, "x_proj": 2 * N * di * (R + 2 * S),
             "out_proj": 2 * N * di * dm}
    # algorithmic bytes of the HBM-bound stages (each tensor read / written once)
    nbytes = {"conv1d_silu": N * di * es * 2,
              "dt_proj": N * es * (R + di),                # dt_low in, dt out
              "scan": N * es * (4 * di + 2 * S)}           # x, dt, z, B, C in; y out
    top = max(stages, key=stages.get)
    t = stages[top] / 1e3
    tpt = TRAFFIC_PER_TOKEN.get((cfg["dtype"], dm, S, top))
    traffic = tpt * N if tpt else None
    blk_bytes = realistic_block_bytes(cfg)
    blk_gbs = blk_bytes / (ms_per_step / 1e3) / 1e9
    block = {"bytes": blk_bytes, "achieved": blk_gbs, "peak": hbm_gbs, "unit": "GB/s",
             "frac": blk_gbs / hbm_gbs,
             "note": "whole block vs HBM, each stage reading and writing its tensors once"}
    if top in flops:
        ach = flops[top] / t / 1e12
        r = {"kernel": top, "bound": "tensor", "achieved": ach, "peak": bf16_tflops,
             "unit": "TFLOP/s", "frac": ach / bf16_tflops, "traffic": traffic,
             "peak_source": f"{src} bf16 dense"}
        if cfg["dtype"] == "f32":
            # fp32-faithful path (F16X3): three fp16 MMAs per multiply-add, at the
            # tensor core's fp16 rate (= its bf16 rate); two for int8 / int4
            # codes (exact in fp16: no W_lo term)
            mmas = 2 if cfg.get("quant") in ("int8", "int4") else 3
            ex = mmas * flops[top] / t / 1e12
            r["tensor_pipe"] = {"f16_tflops_executed": ex, "f16_peak": bf16_tflops,
                                "frac": ex / bf16_tflops,
                                "peak_source": f"{src} bf16 dense (fp16 rate)"}
        r["block"] = block
        return r
    ach = nbytes[top] / t / 1e9
    r = {"kernel": top, "bound": "hbm", "achieved": ach, "peak": hbm_gbs, "unit": "GB/s",
         "frac": ach / hbm_gbs, "traffic": traffic, "peak_source": f"{src} HBM copy",
         "block": block}
    if top == "scan":
        # the scan's other bound: d_state exponentials per token and channel on
        # the MUFU pipe, 16 ex2 per clock per SM (148 SMs at the 1965 MHz
        # maximum clock: an upper bound on the rate, so frac is a lower bound)
        ex2 = N * di * S / t
        peak = 16 * 148 * 1965e6
        r["mufu"] = {"ex2_per_s": ex2, "peak_per_s": peak, "frac": ex2 / peak,
                     "note": "d_state ex2 per token-channel (softplus and gate not counted)"}
    return r


# ------------------------------------------------------- reference arm / CPU
def cpu_forward_setup(cfg, batch):
    import oracle
    p, R = make_params(cfg, seed=0)
    op = oracle.load_ref_scan_op()
    kind = "reference" if op is not None else "port"
    g = torch.Generator().manual_seed(1234)
    x = torch.randn(batch, cfg["seqlen"], cfg["d_model"], generator=g)
    if cfg["dtype"] == "bf16":
        p = {k: v.to(torch.bfloat16) for k, v in p.items()}
        x = x.to(torch.bfloat16)
    return oracle, p, op, kind, x


def cpu_cores():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def cpu_baseline_stack(cfg, min_seconds=10.0, max_runs=5):
    """The stack composed from the reference's CPU block (its compiled scan op)
    and torch RMSNorm, in float32, on one sequence of the workload."""
    import oracle
    cores = cpu_cores()
    torch.set_num_threads(cores)
    op = oracle.load_ref_scan_op()
    layers = []
    for i in range(cfg["n_layers"]):
        p, _ = make_params(cfg, seed=i)
        layers.append((p, torch.ones(cfg["d_model"])))
    x = torch.randn(1, cfg["seqlen"], cfg["d_model"], generator=torch.Generator().manual_seed(1))
    ts, t_start = [], time.perf_counter()
    while len(ts) < 2 or (time.perf_counter() - t_start < min_seconds and len(ts) < max_runs):
        t0 = time.perf_counter()
        oracle.stack_forward(layers, x, 1e-5, scan_op=op)
        ts.append(time.perf_counter() - t0)
    return {"value": cfg["seqlen"] / statistics.median(ts), "unit": "tokens/s", "cores": cores,
            "kind": "reference" if op is not None else "port",
            "sample": f"1 x {cfg['seqlen']} tokens through {cfg['n_layers']} layers, float32, "
                      f"median of {len(ts)}"}


def cpu_baseline(cfg, min_seconds=10.0, max_runs=10):
    """The reference's CPU block forward on a bounded sample of the workload."""
    if cfg["mode"] == "stack":
        return cpu_baseline_stack(cfg)
    if cfg["mode"] != "forward" or cfg.get("quant"):
        return None
    cores = cpu_cores()
    torch.set_num_threads(cores)
    batch = cfg["batch"] if cfg["batch"] * cfg["seqlen"] <= 30000 else 1
    oracle, p, op, kind, x = cpu_forward_setup(cfg, batch)
    oracle.block_forward(p, x, scan_op=op)            # warm-up
    ts, t_start = [], time.perf_counter()
    while len(ts) < 3 or (time.perf_counter() - t_start < min_seconds and len(ts) < max_runs):
        t0 = time.perf_counter()
        oracle.block_forward(p, x, scan_op=op)
        ts.append(time.perf_counter() - t0)
    tok = batch * cfg["seqlen"]
    res = {"value": tok / statistics.median(ts), "unit": "tokens/s", "cores": cores,
           "kind": kind, "sample": f"{batch} x {cfg['seqlen']} tokens per forward, median of {len(ts)}"}
    # the scan op alone (selective_scan_cpu, or the oracle's C restatement) on
    # the same sample's shapes, timed apart as the reference's bench does
    T, di, S = cfg["seqlen"], 2 * cfg["d_model"], cfg["d_state"]
    g = torch.Generator().manual_seed(7)
    args = (torch.randn(batch, T, di, generator=g), torch.rand(batch, T, di, generator=g) * 0.1,
            -torch.rand(di, S, generator=g), torch.randn(batch, T, S, generator=g),
            torch.randn(batch, T, S, generator=g), torch.ones(di))
    scan = (lambda: op.selective_scan_cpu(*args)) if op is not None else \
        (lambda: oracle.selective_scan(*args))
    scan()
    st = []
    for _ in range(5):
        t0 = time.perf_counter()
        scan()
        st.append(time.perf_counter() - t0)
    res["scan_only"] = {"value": tok / statistics.median(st), "unit": "tokens/s",
                        "ms": statistics.median(st) * 1e3}
    return res


def run_reference(args, cfg):
    """The reference's CPU block forward on the host cores, on the arm's own
    workload: every step is one forward over the configuration's whole batch
    (config 0: 151 x 180 tokens).  The scan is the reference's own compiled op
    (oracle/_ref); the torch CPU ops around it are the oracle's restatement of
    _mamba.py:204-265, which makes the reference's ATen calls (the reference's
    Python tree cannot be imported where this runs).  Without the compiled op
    there is no reference to time, and the arm says so."""
    ws, rank, _ = dist_env()
    if rank != 0:
        return None
    if cfg["mode"] != "forward" or cfg.get("quant"):
        return {"impl": "reference", "unavailable": "the reference arm times the block forward "
                "workloads (configs 0 and 1); this configuration has no CPU reference arm"}
    cores = cpu_cores()
    torch.set_num_threads(cores)
    batch = cfg["batch"]
    oracle, p, op, kind, x = cpu_forward_setup(cfg, batch)
    if op is None:
        return {"impl": "reference", "unavailable": "the reference's compiled scan op "
                "(oracle/_ref/selective_scan_cpu.so) was not built"}
    for _ in range(args.warmup):
        oracle.block_forward(p, x, scan_op=op)
    ts = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        oracle.block_forward(p, x, scan_op=op)
        ts.append(time.perf_counter() - t0)
    dt = sum(ts)
    tok = batch * cfg["seqlen"]
    value = tok * args.steps / dt
    sample = (f"the whole workload, {batch} x {cfg['seqlen']} tokens, per step; "
              f"{cores} host threads")
    return {"metric": METRIC, "value": value, "unit": "tokens/s", "impl": "reference",
            "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": cfg["dtype"],
            "data": "synthetic (seeded; shapes of the configuration)",
            "config": dict(workload_config(cfg, batch, batch, ws_label="batch-sharded x1"),
                           l2="inputs in host memory (CPU arm)"),
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": kind,
                             "sample": sample},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", type=int, default=0, choices=sorted(CONFIGS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--shard", default="batch", choices=["batch", "channels"],
                    help="multi-GPU split: batch rows (no collective) or d_inner channels "
                         "(two all-reduces per block; for batches smaller than the GPU count "
                         "and decode latency)")
    ap.add_argument("--reduce", default="peer", choices=["peer", "nccl"],
                    help="all-reduce of the channel shards: the library's peer-memory kernel "
                         "or NCCL")
    ap.add_argument("--batch", type=int, default=None,
                    help="override the configuration's batch (small cases for profiling)")
    ap.add_argument("--quant", default=None, choices=["int8", "int4", "nf4"],
                    help="config 3's weight scheme (default int8)")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    cfg = dict(CONFIGS[args.config])
    if args.batch:
        cfg["batch"] = args.batch
        cfg["workload"] += f"_batch{args.batch}"
    if args.quant and cfg.get("quant"):
        cfg["workload"] = cfg["workload"].replace(cfg["quant"], args.quant)
        cfg["quant"] = args.quant
    if args.shard == "channels" and cfg["mode"] != "stack":
        cfg["workload"] += "_dinner_sharded"
    # stdout carries the one result line: whatever the libraries write there
    # (NCCL's version banner, for one) goes to stderr until then
    sys.stdout.flush()
    saved_stdout = os.dup(1)
    os.dup2(2, 1)
    try:
        if args.impl == "reference":
            res = run_reference(args, cfg)
        else:
            res = run_ours(args, cfg)
            ws, rank, _ = dist_env()
            if res is not None and ws == 1 and not args.no_cpu_baseline:
                res["cpu_baseline"] = cpu_baseline(cfg)
    finally:
        sys.stdout.flush()
        os.dup2(saved_stdout, 1)
        os.close(saved_stdout)
    if res is not None:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
