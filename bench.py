"""Benchmark: fwd+bwd attention TFLOPS on B200 (BASELINE.json metric).

Workload (the metric's headline config): bf16
Llama-3-8B-style GQA layer, B=4 per GPU, Hq=32, Hkv=8, D=128, S=4096, causal,
scale 1/sqrt(128); q, k, v, grad_out ~ N(0,1) seeded, synthetic.

One step = one forward + one backward of that layer through the library's
C ABI (bfa_fwd, then the backward as two calls on one workspace: Δ and dQ --
the dQ kernel forms Δ itself on the tcgen05 path -- and dK/dV, so each
kernel is timed on its own). FLOPs count only unmasked (i, j) pairs,
element-exact: 4·D per pair forward, 10·D backward.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--workload c3|c2|c4|c4t|c5|c5u|decode|fp32]

N > 1 is launched with torchrun (one process per GPU); each rank runs its own
batch shard (weak scaling, no collective on the data path); the step time is
the max over ranks and `value` is the aggregate over all ranks (`value_is`
says so; `per_gpu_value` is value / N). The c3 line also carries `cp`: config
5 through the context-parallel K/V ring and through Ulysses on the same N
GPUs, beside the same problem run whole on each GPU alone. `--impl reference`
times the reference's math path on the host CPU cores (the CPU restatement in
oracle/; the reference itself is Triton for Ascend NPUs and has no GPU or CPU
build that runs here).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "npu-flex-att_b200"))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

METRIC = "fwd+bwd attention TFLOPS/GPU (unmasked FLOPs) and % of bf16 tensor peak"
CFG = dict(B=4, Hq=32, Hkv=8, S=4096, D=128, causal=True, window=0, soft_cap=0.0)
WORKLOAD = "c3: bf16 GQA B=4/GPU Hq=32 Hkv=8 D=128 S=4096 causal fwd+bwd"
# Config 4 (Gemma2-style): D=256, causal + window 4096 + soft-cap 50; c4t is
# the second run at S=8190, a key length that is not a tile multiple.
CFG_C4 = dict(B=2, Hq=16, Hkv=8, S=8192, D=256, causal=True, window=4096, soft_cap=50.0)
CFG_C4T = dict(CFG_C4, S=8190)
WORKLOADS = {
    "c3": (CFG, WORKLOAD),
    "c4": (CFG_C4, "c4: bf16 Gemma2-style B=2/GPU Hq=16 Hkv=8 D=256 S=8192 causal + window 4096 + "
                   "soft-cap 50 fwd+bwd"),
    "c4t": (CFG_C4T, "c4: bf16 Gemma2-style B=2/GPU Hq=16 Hkv=8 D=256 S=8190 (key tail not a tile "
                     "multiple) causal + window 4096 + soft-cap 50 fwd+bwd"),
}


def causal_pairs(s: int) -> int:
    return s * (s + 1) // 2


def pairs_per_head(cfg) -> int:
    """Element-exact kept (i, j) pairs of one head (causal, optional window)."""
    s, w = cfg["S"], cfg.get("window", 0)
    if not cfg.get("causal", True):
        raise ValueError("bench workloads are causal")
    if w <= 0 or w >= s - 1:
        return causal_pairs(s)
    return causal_pairs(w + 1) - (w + 1) + (s - w) * (w + 1)


def step_flops(cfg=CFG) -> float:
    return 14.0 * cfg["D"] * pairs_per_head(cfg) * cfg["B"] * cfg["Hq"]


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            m = json.load(f)
        return float(m["bf16_tflops"]), float(m["hbm_gbs"]), "measured"
    except Exception:
        return 1590.0, 6650.0, "fallback"


def committed_traffic(phase: str, workload: str = "c3"):
    """DRAM bytes per launch of a kernel from the committed ncu capture, or None."""
    kernel = {"fwd": "fwd_kernel", "dkdv": "dkdv_kernel", "dq": "dq_kernel",
              "dq_delta": "dq_kernel"}.get(phase)
    try:
        with open(os.path.join(ROOT, "profiles", f"{workload}_dram_traffic.json")) as f:
            return json.load(f)["kernels"][kernel]["dram_bytes_per_launch"]
    except Exception:
        return None


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None
        sm = [num(r[1]) for r in rows if num(r[1])]
        smax = max((num(r[2]) or 0) for r in rows)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": reasons, "samples": len(rows)}


def make_inputs(seed, device, cfg=CFG):
    B, Hq, Hkv, S, D = cfg["B"], cfg["Hq"], cfg["Hkv"], cfg["S"], cfg["D"]
    # Generated on the device from a seeded generator (the full tensors are GBs).
    gd = torch.Generator(device=device).manual_seed(seed)
    q = torch.randn(B, Hq, S, D, generator=gd, device=device, dtype=torch.bfloat16)
    k = torch.randn(B, Hkv, S, D, generator=gd, device=device, dtype=torch.bfloat16)
    v = torch.randn(B, Hkv, S, D, generator=gd, device=device, dtype=torch.bfloat16)
    do = torch.randn(B, Hq, S, D, generator=gd, device=device, dtype=torch.bfloat16)
    return q, k, v, do


def cpu_baseline_sample(budget_s: float = 15.0, cfg=CFG):
    """The reference's math path (oracle restatement) on the host cores.

    Times fwd+bwd of single (b, q-head) slices of the workload (fp32, the
    workload's S, D and mask) until ~budget_s seconds of CPU work, and scales
    FLOPs per slice; returns (TFLOPS, threads, slices, seconds)."""
    from oracle.attention_math import attention_backward, attention_forward
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(0)
    S, D = cfg["S"], cfg["D"]
    mask = dict(causal=True, sliding_window=cfg.get("window", 0), soft_cap=cfg.get("soft_cap", 0.0))
    q, k, v, do = (torch.randn(1, 1, S, D, generator=g) for _ in range(4))
    slice_flops = 14.0 * D * pairs_per_head(cfg)
    attention_forward(q[:, :, :256], k[:, :, :256], v[:, :, :256], dtype=torch.float32, **mask)
    t0 = time.perf_counter()
    n = 0
    while True:
        o, lse = attention_forward(q, k, v, dtype=torch.float32, **mask)
        attention_backward(q, k, v, do, out=o, lse=lse, dtype=torch.float32, **mask)
        n += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    return n * slice_flops / dt / 1e12, threads, n, dt


def run_reference(args):
    """The reference's CPU math path on the workload's own config, timed per
    step: a step is a bounded sample of whole (b, q-head) slices (fwd+bwd,
    fp32, all host threads) taking about `--ref-step-s` seconds. `ms_per_step`
    is the wall time each of those steps took; the time a whole step of the
    workload (every slice) would take at the measured rate is reported apart,
    as `extrapolated_full_step_ms`."""
    rank, world, _ = dist_env()
    if rank != 0:
        return
    cfg, workload = WORKLOADS.get(args.workload, (CFG, WORKLOAD))
    threads = os.cpu_count() or 1
    tflops_all, wall_ms, slices = [], [], []
    for i in range(args.warmup + args.steps):
        budget = args.ref_step_s if i >= args.warmup else min(args.ref_step_s, 0.3)
        tf, threads, n, dt = cpu_baseline_sample(budget_s=budget, cfg=cfg)
        if i >= args.warmup:
            tflops_all.append(tf)
            wall_ms.append(dt * 1e3)
            slices.append(n)
    value = statistics.median(tflops_all)
    full_ms = step_flops(cfg) / (value * 1e12) * 1e3
    n_slices = cfg["B"] * cfg["Hq"]
    sample = (f"per step: fwd+bwd of whole (b, q-head) slices of the workload (S={cfg['S']}, "
              f"D={cfg['D']}, causal" + (f", window {cfg['window']}" if cfg.get("window") else "")
              + (f", soft-cap {cfg['soft_cap']:g}" if cfg.get("soft_cap") else "")
              + f", fp32) for ~{args.ref_step_s:g} s (median {statistics.median(slices)} of the "
              f"step's {n_slices} slices); TFLOPS scale per slice")
    out = {
        "impl": "reference", "metric": METRIC, "value": round(value, 6), "unit": "TFLOPS",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(statistics.mean(wall_ms), 3),
        "ms_per_step_is": "wall time of each timed step, i.e. of its bounded sample of slices",
        "extrapolated_full_step_ms": round(full_ms, 3),
        "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,1))",
        "config": {"workload": workload, "global_batch": cfg["B"] * args.gpus, "seq_len": cfg["S"],
                   "parallelism": "host CPU, all cores, rank 0 only"},
        "cpu_baseline": {"value": round(value, 6), "unit": "TFLOPS", "cores": threads,
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 6), "unit": "TFLOPS", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(out), flush=True)


def init_dist(dev, world):
    """NCCL process group over the ranks of this node (no-op for one rank)."""
    if world > 1 and not torch.distributed.is_initialized():
        import datetime
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                             device_id=dev)


def max_over_ranks(x: float, dev, world: int) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], device=dev)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def run_ours(args):
    import bfa_lib
    import npu_flash_attention as nfa

    cfg, workload = WORKLOADS[args.workload]
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    init_dist(dev, world)
    lib = bfa_lib.load()
    q, k, v, do = make_inputs(1234 + rank, dev, cfg)
    B, Hq, Hkv, S, D = cfg["B"], cfg["Hq"], cfg["Hkv"], cfg["S"], cfg["D"]
    grads = (torch.empty_like(q), torch.empty_like(k), torch.empty_like(v))
    kw = dict(causal=True, sliding_window=cfg.get("window", 0), soft_cap=cfg.get("soft_cap", 0.0))
    pr = nfa._problem(q, k, True, kw["sliding_window"], None, 1.0 / math.sqrt(D), kw["soft_cap"])
    ws = torch.empty(lib.bfa_bwd_workspace_bytes(pr), dtype=torch.uint8, device=dev)

    def step(ev=None):
        if ev:
            ev[0].record()
        out, l_ = nfa.npu_flash_attention_forward(q, k, v, return_lse=True, **kw)
        if ev:
            ev[1].record()
        # Δ and dQ in one call: on the tcgen05 path the dQ kernel forms Δ
        # itself and runs first; dK/dV then reads Δ from the workspace.
        nfa.npu_flash_attention_backward(q, k, v, out, l_, do,
                                         _phases=bfa_lib.PHASE_DELTA | bfa_lib.PHASE_DQ,
                                         _workspace=ws, _outputs=grads, **kw)
        if ev:
            ev[2].record()
        nfa.npu_flash_attention_backward(q, k, v, out, l_, do, _phases=bfa_lib.PHASE_DKDV,
                                         _workspace=ws, _outputs=grads, **kw)
        if ev:
            ev[3].record()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    nfa.check_device_status(dev)

    events = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    launches0 = lib.bfa_launch_count()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record()
    for i in range(args.steps):
        step(events[i])
    end.record()
    torch.cuda.synchronize()
    launches = lib.bfa_launch_count() - launches0
    if world > 1:
        torch.distributed.barrier()
    clocks = sampler.stop()
    nfa.check_device_status(dev)
    total_ms = max_over_ranks(start.elapsed_time(end), dev, world)
    phase_ms = [sum(events[i][j].elapsed_time(events[i][j + 1]) for i in range(args.steps)) / args.steps
                for j in range(3)]
    ms_step = total_ms / args.steps
    flops = step_flops(cfg)
    value = world * flops / (ms_step * 1e-3) / 1e12
    del q, k, v, do, grads, ws

    # ---- e2e: public autograd API, host (pinned) buffers, copies inside the timed region
    e2e = None if args.profile else run_e2e(nfa, dev, args, world, cfg)
    # ---- context parallelism (config 5) on the same GPUs
    cp = run_cp(args, dev, rank, world) if (args.workload == "c3" and not (args.profile or args.no_cp)) else None

    peak_tf, _, peak_kind = peaks()
    pairs = pairs_per_head(cfg) * B * Hq
    # "dq_delta": the dQ kernel with Δ formed in its prologue (head dims
    # 64/128/256), or the Δ pass then dQ (other paths); its FLOPs are dQ's.
    kern_flops = {"fwd": 4.0 * D * pairs, "dq_delta": 6.0 * D * pairs, "dkdv": 8.0 * D * pairs}
    names = ["fwd", "dq_delta", "dkdv"]
    dom = max(range(3), key=lambda j: phase_ms[j])
    achieved = kern_flops[names[dom]] / (phase_ms[dom] * 1e-3) / 1e12
    kernel_frac = {n: round(kern_flops[n] / (phase_ms[j] * 1e-3) / 1e12 / peak_tf, 4)
                   for j, n in enumerate(names) if kern_flops[n] > 0}
    roofline = {"bound": "tensor", "kernel": names[dom], "achieved": round(achieved, 2),
                "peak": peak_tf, "unit": "TFLOP/s", "frac": round(achieved / peak_tf, 4),
                "peak_kind": f"bf16 dense burst, {peak_kind}",
                "traffic": committed_traffic(names[dom], args.workload),
                "traffic_unit": f"DRAM bytes per launch (ncu capture, profiles/{args.workload}_dram_traffic.json)",
                "algorithmic_flop_per_launch": kern_flops[names[dom]],
                "phase_ms": {n: round(x, 4) for n, x in zip(names, phase_ms)},
                "kernel_frac_of_peak": kernel_frac}
    cpu = None
    if rank == 0 and world == 1 and not (args.no_cpu_baseline or args.profile):
        tf, threads, n, dt = cpu_baseline_sample(budget_s=args.cpu_budget, cfg=cfg)
        cpu = {"value": round(tf, 6), "unit": "TFLOPS", "cores": threads, "kind": "port",
               "sample": f"{n} whole (b, q-head) slices of the workload (S={S}, D={D}, same mask, "
                         f"fp32 fwd+bwd) in {dt:.1f} s; TFLOPS scale per slice"}
    if rank == 0:
        l2 = ("inputs larger than L2 (q {:.0f} MB, dO {:.0f} MB, k/v {:.0f} MB each)".format(
            B * Hq * S * D * 2 / 1e6, B * Hq * S * D * 2 / 1e6, B * Hkv * S * D * 2 / 1e6))
        out = {
            "metric": METRIC, "value": round(value, 3), "unit": "TFLOPS", "n_gpus": world,
            "value_is": f"aggregate over the {world} GPU(s) (sum of per-GPU TFLOPS)",
            "per_gpu_value": round(value / world, 3),
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1), generated on device)",
            "config": {"workload": workload, "global_batch": B * world, "seq_len": S,
                       "parallelism": f"batch x head shards on {world} GPU(s), no collective",
                       "l2": l2},
            "pct_of_peak": round(100.0 * value / world / peak_tf, 2),
            "gpu_launches": int(launches),
            "roofline": roofline,
            "cpu_baseline": cpu,
            "e2e": e2e,
            "cp": cp,
            "clocks": clocks,
        }
        print(json.dumps(out), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def run_e2e(nfa, dev, args, world, cfg=CFG):
    """Same metric through the public autograd API with host buffers: every
    step copies q, k, v, dO from pinned host memory, runs flex_attention
    forward + backward, and reads dQ, dK, dV back to pinned host memory.

    The steps are pipelined the way a training loop feeds a GPU: step i+1's
    inputs are copied in on one stream (into the second of two device
    buffers) and step i-1's gradients are copied out on another while step i
    computes, so the two PCIe directions overlap each other and the kernels.
    The timed region holds every step's copies, from the first input copy to
    the last gradient read-back, for the same number of steps as the
    device-timed run."""
    B, Hq, Hkv, S, D = cfg["B"], cfg["Hq"], cfg["Hkv"], cfg["S"], cfg["D"]
    mask = dict(causal=True, sliding_window=cfg.get("window", 0), soft_cap=cfg.get("soft_cap", 0.0))
    shapes = [(B, Hq, S, D), (B, Hkv, S, D), (B, Hkv, S, D), (B, Hq, S, D)]
    host_in = [torch.randn(*s, dtype=torch.float32).to(torch.bfloat16).pin_memory() for s in shapes]
    host_out = [torch.empty(*s, dtype=torch.bfloat16).pin_memory() for s in shapes[:3]]
    h2d = sum(t.numel() * t.element_size() for t in host_in)
    d2h = sum(t.numel() * t.element_size() for t in host_out)
    comp = torch.cuda.current_stream(dev)
    s_in = torch.cuda.Stream(dev)
    s_out = torch.cuda.Stream(dev)
    bufs = [[torch.empty(*s, dtype=torch.bfloat16, device=dev) for s in shapes] for _ in range(2)]
    ev_in = [torch.cuda.Event() for _ in range(2)]    # inputs of the buffer landed
    ev_used = [torch.cuda.Event() for _ in range(2)]  # step using the buffer finished

    def copy_in(i):
        b_ = i % 2
        with torch.cuda.stream(s_in):
            if i >= 2:
                s_in.wait_event(ev_used[b_])
            for dst, src in zip(bufs[b_], host_in):
                dst.copy_(src, non_blocking=True)
            ev_in[b_].record(s_in)

    def run(n):
        copy_in(0)
        for i in range(n):
            b_ = i % 2
            if i + 1 < n:
                copy_in(i + 1)
            comp.wait_event(ev_in[b_])
            qd, kd, vd, dod = bufs[b_]
            qd, kd, vd = (t.detach().requires_grad_(True) for t in (qd, kd, vd))
            out = nfa.flex_attention(qd, kd, vd, **mask)
            out.backward(dod)
            ev_used[b_].record(comp)
            grads = (qd.grad, kd.grad, vd.grad)
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev_used[b_])
                for h, g_ in zip(host_out, grads):
                    h.copy_(g_, non_blocking=True)
                    g_.record_stream(s_out)
        done = torch.cuda.Event()
        done.record(s_out)
        return done

    steps = max(2, args.steps)
    run(2)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(s_in)
    done = run(steps)
    s_in.wait_event(done)
    e.record(s_in)
    torch.cuda.synchronize()
    ms = max_over_ranks(s.elapsed_time(e) / steps, dev, world)
    return {"value": round(world * step_flops(cfg) / (ms * 1e-3) / 1e12, 3), "unit": "TFLOPS",
            "value_is": f"aggregate over the {world} GPU(s)",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(ms, 3),
            "steps": steps, "pipelined": "H2D of step i+1 and D2H of step i-1 overlap step i"}


C5 = dict(B=1, Hq=64, Hkv=8, S=65536, D=128)
C5_WORKLOAD = "c5: bf16 B=1 Hq=64 Hkv=8 D=128 S=65536 causal + ALiBi, context-parallel K/V ring"
C5U_WORKLOAD = ("c5: bf16 B=1 Hq=64 Hkv=8 D=128 S=65536 causal + ALiBi, context-parallel Ulysses "
                "(head-sequence all-to-alls)")


def c5_flops():
    return 14.0 * C5["D"] * causal_pairs(C5["S"]) * C5["B"] * C5["Hq"]


def time_c5(mode, dev, rank, world, steps, warmup):
    """ms per fwd+bwd step of config 5, max over ranks. `mode` "ring" and
    "ulysses" shard the sequence over the ranks (each holds its zigzag shard,
    2 chunks of S/(2N) rows); "single" runs the whole problem on every GPU
    alone, at the same time, with no communication."""
    import context_parallel as cp
    import npu_flash_attention as nfa
    B, Hq, Hkv, S, D = C5["B"], C5["Hq"], C5["Hkv"], C5["S"], C5["D"]
    rows = S if mode == "single" else S // world
    gd = torch.Generator(device=dev).manual_seed(4321 + rank)
    q = torch.randn(B, Hq, rows, D, generator=gd, device=dev, dtype=torch.bfloat16).requires_grad_(True)
    k = torch.randn(B, Hkv, rows, D, generator=gd, device=dev, dtype=torch.bfloat16).requires_grad_(True)
    v = torch.randn(B, Hkv, rows, D, generator=gd, device=dev, dtype=torch.bfloat16).requires_grad_(True)
    do = torch.randn(B, Hq, rows, D, generator=gd, device=dev, dtype=torch.bfloat16)
    slopes = torch.tensor([2.0 ** (-8.0 * (i + 1) / Hq) for i in range(Hq)], device=dev)
    attn = {"ring": cp.context_parallel_attention, "ulysses": cp.ulysses_attention,
            "single": nfa.npu_flex_attention}[mode]

    def step():
        q.grad = k.grad = v.grad = None
        o = attn(q, k, v, causal=True, alibi_slope=slopes)
        o.backward(do)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    s_, e_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s_.record()
    for _ in range(steps):
        step()
    e_.record()
    torch.cuda.synchronize()
    ms = max_over_ranks(s_.elapsed_time(e_) / steps, dev, world)
    del q, k, v, do
    torch.cuda.empty_cache()
    return ms


def run_cp(args, dev, rank, world):
    """Config 5 through context parallelism on the bench's N GPUs, for the
    `cp` key of the c3 line: the K/V ring, Ulysses (when the head counts
    divide by N), and the whole problem on each GPU alone as the N=1 base of
    the strong-scaling efficiency single_ms / (N * ms)."""
    steps = max(1, min(args.steps, args.cp_steps))
    warmup = min(args.warmup, 2)
    flops = c5_flops()
    res = {"workload": "c5: bf16 B=1 Hq=64 Hkv=8 D=128 S=65536 causal + ALiBi, fwd+bwd, "
                       "strong scaling over the bench's GPUs",
           "steps": steps, "warmup": warmup}
    single = time_c5("single", dev, rank, world, steps, warmup)
    res["single_gpu"] = {"ms_per_step": round(single, 3), "tflops": round(flops / (single * 1e-3) / 1e12, 1)}
    modes = [] if world == 1 else ["ring"] + (["ulysses"] if C5["Hkv"] % world == 0 else [])
    for mode in modes:
        ms = time_c5(mode, dev, rank, world, steps, warmup)
        res[mode] = {"ms_per_step": round(ms, 3), "tflops": round(flops / (ms * 1e-3) / 1e12, 1),
                     "eff_vs_single_gpu": round(single / (world * ms), 4)}
    return res


def run_c5(args, ulysses=False):
    """Config 5 through context parallelism (one process per GPU): each rank
    holds its zigzag shard (2 chunks of S/(2N) rows) of Q, K, V and runs
    forward + backward with context_parallel_attention (the K/V ring) or, for
    --workload c5u, ulysses_attention. FLOPs count the unmasked pairs of the
    whole causal sequence (14·D per pair per q-head)."""
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    import datetime
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29517")
    torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev,
                                         rank=rank, world_size=world)
    ms = time_c5("ulysses" if ulysses else "ring", dev, rank, world, args.steps, args.warmup)
    peak_tf, _, peak_kind = peaks()
    if rank == 0:
        value = c5_flops() / (ms * 1e-3) / 1e12
        print(json.dumps({
            "metric": METRIC, "value": round(value, 3), "unit": "TFLOPS", "n_gpus": world,
            "value_is": f"aggregate over the {world} GPU(s)",
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1), generated on device)",
            "config": {"workload": C5U_WORKLOAD if ulysses else C5_WORKLOAD, "global_batch": C5["B"],
                       "seq_len": C5["S"],
                       "parallelism": (f"Ulysses all-to-alls over {world} GPU(s), NCCL" if ulysses else
                                       f"context-parallel zigzag K/V ring over {world} GPU(s), NCCL")},
            "pct_of_peak": round(100.0 * value / world / peak_tf, 2),
            "gpu_launches": None, "roofline": None, "cpu_baseline": None, "e2e": None,
            "note": ("auxiliary measurement of " + ("Ulysses" if ulysses else "the P-2 ring") +
                     "; the headline line is the default c3 run")}),
            flush=True)
    torch.distributed.barrier()
    torch.distributed.destroy_process_group()


# Config 2 and the reference's published 910B3 latencies for it (fp16 causal
# B1 H2 D64, no window): RESULT.md:180-184 (forward) and :200-204 (backward).
C2_S = (128, 512, 1024, 2048)
C2_910B3_MS = {128: (0.325, 1.371), 512: (0.979, 3.265), 1024: (1.547, 4.240), 2048: (2.262, 9.269)}


def run_c2(args):
    """Config 2: fp16 B1 H2 D64 causal, S in {128, 512, 1024, 2048}, with and
    without window 64. Latency-bound, so each case is timed per call: forward
    and backward separately, CUDA events around each call, L2 flushed (a
    256 MB write) before every call, median over the reps. The reference's
    published Ascend 910B3 latencies for the unwindowed cases stand beside
    them as context, not as a target."""
    import bfa_lib
    import npu_flash_attention as nfa
    _, _, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    lib = bfa_lib.load()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    reps = max(args.steps, 30)
    cases = []
    launches = 0
    for w in (0, 64):
        for S in C2_S:
            g = torch.Generator(device=dev).manual_seed(S + w)
            q, k, v, do = (torch.randn(1, 2, S, 64, generator=g, device=dev, dtype=torch.float16)
                           for _ in range(4))
            kw = dict(causal=True, sliding_window=w)
            f_ms, b_ms = [], []
            for i in range(args.warmup + reps):
                flush.fill_(i & 255)
                e = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
                n0 = lib.bfa_launch_count()
                e[0].record()
                o, lse = nfa.npu_flash_attention_forward(q, k, v, return_lse=True, **kw)
                e[1].record()
                flush.fill_((i + 1) & 255)
                e[2].record()
                nfa.npu_flash_attention_backward(q, k, v, o, lse, do, **kw)
                e3 = torch.cuda.Event(enable_timing=True)
                e3.record()
                torch.cuda.synchronize()
                if i >= args.warmup:
                    f_ms.append(e[0].elapsed_time(e[1]))
                    b_ms.append(e[2].elapsed_time(e3))
                    launches += lib.bfa_launch_count() - n0
            nfa.check_device_status(dev)
            pairs = pairs_per_head(dict(S=S, window=w, causal=True)) * 2
            fm, bm = statistics.median(f_ms), statistics.median(b_ms)
            case = {"S": S, "window": w, "fwd_ms": round(fm, 4), "bwd_ms": round(bm, 4),
                    "fwd_bwd_tflops": round(14.0 * 64 * pairs / ((fm + bm) * 1e-3) / 1e12, 3)}
            if w == 0:
                case["ascend_910b3_ms"] = {"fwd": C2_910B3_MS[S][0], "bwd": C2_910B3_MS[S][1],
                                           "source": "reference RESULT.md:180-184, 200-204"}
            cases.append(case)
    head = next(c for c in cases if c["S"] == 2048 and c["window"] == 0)
    print(json.dumps({
        "metric": METRIC, "value": head["fwd_bwd_tflops"], "unit": "TFLOPS", "n_gpus": 1,
        "value_is": "fwd+bwd TFLOPS of the S=2048 unwindowed case (sum of its median fwd and bwd latencies)",
        "steps": reps, "warmup": args.warmup, "ms_per_step": round(head["fwd_ms"] + head["bwd_ms"], 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic (seeded N(0,1), generated on device)",
        "config": {"workload": "c2: fp16 B=1 H=2 D=64 causal, S in {128,512,1024,2048}, window 0 and 64",
                   "global_batch": 1, "seq_len": 2048, "parallelism": "1 GPU",
                   "l2": "flushed (256 MB write) before every timed call"},
        "gpu_launches": int(launches), "cases": cases,
        "roofline": None, "cpu_baseline": None, "e2e": None,
        "note": "latency-bound configuration; auxiliary to the c3 headline line"}), flush=True)


FP32_CASES = [  # (B, Hq, Hkv, S, D): c1 itself, then larger fp32 problems
    (1, 2, 2, 128, 64),
    (1, 8, 2, 2048, 64),
    (1, 8, 2, 2048, 128),
]


def run_fp32(args):
    """fp32 inputs (config 1 and larger causal fp32 problems). fp32 runs on the
    CUDA-core kernels (simt_attention.cu): the tcgen05 kernels take 16-bit
    operands only. Timed per call like c2: forward and backward separately,
    CUDA events, L2 flushed before every call, median over the reps."""
    import bfa_lib
    import npu_flash_attention as nfa
    _, _, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    lib = bfa_lib.load()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    reps = max(args.steps, 10)
    cases, launches = [], 0
    for (B, Hq, Hkv, S, D) in FP32_CASES:
        g = torch.Generator(device=dev).manual_seed(S + D)
        q, do = (torch.randn(B, Hq, S, D, generator=g, device=dev) for _ in range(2))
        k, v = (torch.randn(B, Hkv, S, D, generator=g, device=dev) for _ in range(2))
        f_ms, b_ms = [], []
        for i in range(args.warmup + reps):
            flush.fill_(i & 255)
            e = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
            n0 = lib.bfa_launch_count()
            e[0].record()
            o, lse = nfa.npu_flash_attention_forward(q, k, v, causal=True, return_lse=True)
            e[1].record()
            flush.fill_((i + 1) & 255)
            e[2].record()
            nfa.npu_flash_attention_backward(q, k, v, o, lse, do, causal=True)
            e[3].record()
            torch.cuda.synchronize()
            if i >= args.warmup:
                f_ms.append(e[0].elapsed_time(e[1]))
                b_ms.append(e[2].elapsed_time(e[3]))
                launches += lib.bfa_launch_count() - n0
        nfa.check_device_status(dev)
        fm, bm = statistics.median(f_ms), statistics.median(b_ms)
        pairs = pairs_per_head(dict(S=S, causal=True)) * B * Hq
        cases.append({"B": B, "Hq": Hq, "Hkv": Hkv, "S": S, "D": D, "fwd_ms": round(fm, 4),
                      "bwd_ms": round(bm, 4),
                      "fwd_bwd_tflops": round(14.0 * D * pairs / ((fm + bm) * 1e-3) / 1e12, 3)})
    head = cases[-1]
    print(json.dumps({
        "metric": METRIC, "value": head["fwd_bwd_tflops"], "unit": "TFLOPS", "n_gpus": 1,
        "value_is": "fwd+bwd TFLOPS of the largest fp32 case (sum of its median fwd and bwd latencies)",
        "steps": reps, "warmup": args.warmup, "ms_per_step": round(head["fwd_ms"] + head["bwd_ms"], 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,1), generated on device)",
        "config": {"workload": "fp32 causal: config 1 (B=1 H=2 S=128 D=64) and B=1 Hq=8 Hkv=2 S=2048 "
                               "D=64/128 on the CUDA-core kernels",
                   "global_batch": 1, "seq_len": head["S"], "parallelism": "1 GPU",
                   "l2": "flushed (256 MB write) before every timed call"},
        "gpu_launches": int(launches), "cases": cases,
        "roofline": None, "cpu_baseline": None, "e2e": None,
        "note": "auxiliary line: the fp32 path; the c3 line is the headline"}), flush=True)


DEC = dict(B=8, Hq=32, Hkv=8, Sq=1, Sk=32768, D=128)
DEC_WORKLOAD = ("decode: bf16 B=8 Hq=32 Hkv=8 D=128, 1 query per head, 32768 keys, causal with "
                "the query at the end of the keys (split-KV path)")


def run_decode(args):
    """Decoding forward (one query per q-head, long K/V) through the split-KV
    path on one GPU. The metric is the K/V read bandwidth, bounded by HBM:
    K and V (1.07 GB, larger than L2) are read once per step. The regular
    forward (BFA_FWD_DECODE=0) is timed on the same inputs beside it."""
    import bfa_lib
    import npu_flash_attention as nfa
    _, _, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    lib = bfa_lib.load()
    B, Hq, Hkv, Sq, Sk, D = DEC["B"], DEC["Hq"], DEC["Hkv"], DEC["Sq"], DEC["Sk"], DEC["D"]
    g = torch.Generator(device=dev).manual_seed(777)
    q = torch.randn(B, Hq, Sq, D, generator=g, device=dev, dtype=torch.bfloat16)
    k = torch.randn(B, Hkv, Sk, D, generator=g, device=dev, dtype=torch.bfloat16)
    v = torch.randn(B, Hkv, Sk, D, generator=g, device=dev, dtype=torch.bfloat16)
    kv_bytes = 2 * k.numel() * k.element_size()

    def step():
        return nfa.npu_flash_attention_forward(q, k, v, causal=True, q_pos_offset=Sk - Sq, return_lse=True)

    def timed(steps, sample_clocks):
        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize()
        nfa.check_device_status(dev)
        sampler = ClockSampler(local) if sample_clocks else None
        if sampler:
            sampler.start()
            time.sleep(0.3)
        n0 = lib.bfa_launch_count()
        s_, e_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        s_.record()
        for _ in range(steps):
            step()
        e_.record()
        torch.cuda.synchronize()
        clocks = sampler.stop() if sampler else None
        nfa.check_device_status(dev)
        return s_.elapsed_time(e_) / steps, lib.bfa_launch_count() - n0, clocks

    steps = max(args.steps, 20)
    os.environ.pop("BFA_FWD_DECODE", None)
    ms, launches, clocks = timed(steps, True)
    os.environ["BFA_FWD_DECODE"] = "0"
    ms_regular, _, _ = timed(max(3, steps // 4), False)
    os.environ.pop("BFA_FWD_DECODE", None)
    _, hbm, peak_kind = peaks()
    gbs = kv_bytes / (ms * 1e-3) / 1e9
    print(json.dumps({
        "metric": "decode forward K/V read bandwidth", "value": round(gbs, 1), "unit": "GB/s",
        "n_gpus": 1, "steps": steps, "warmup": args.warmup, "ms_per_step": round(ms, 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1), generated on device)",
        "config": {"workload": DEC_WORKLOAD, "global_batch": B, "seq_len": Sk,
                   "parallelism": "1 GPU", "l2": "K/V 1.07 GB, larger than L2"},
        "gpu_launches": launches,
        "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(gbs / hbm, 4), "peak_kind": f"HBM copy, {peak_kind}",
                     "traffic": None, "algorithmic_bytes_per_launch": kv_bytes},
        "regular_path_ms": round(ms_regular, 5),
        "cpu_baseline": None, "e2e": None, "clocks": clocks,
        "note": "auxiliary measurement of the split-KV decoding path; the headline line is the default c3 run"}),
        flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-budget", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", choices=["c3", "c2", "c4", "c4t", "c5", "c5u", "decode", "fp32"], default="c3",
                    help="c3 (default, the headline), c2 (fp16 latencies), c4 / c4t (D=256 window + "
                         "soft-cap at S=8192 / 8190), c5 (context-parallel ring), c5u (context-"
                         "parallel Ulysses), decode (split-KV decoding forward) or fp32 (the fp32 "
                         "path: config 1 and larger fp32 problems)")
    ap.add_argument("--ref-step-s", type=float, default=2.0,
                    help="CPU seconds per step of the reference arm (a bounded sample of slices)")
    ap.add_argument("--no-cp", action="store_true", help="skip the context-parallel key of the c3 line")
    ap.add_argument("--cp-steps", type=int, default=5, help="timed steps of each context-parallel run")
    ap.add_argument("--profile", action="store_true",
                    help="for ncu: only the warm-up and timed steps (no e2e, no CPU baseline)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.workload in ("c5", "c5u"):
        run_c5(args, ulysses=args.workload == "c5u")
    elif args.workload == "c2":
        run_c2(args)
    elif args.workload == "decode":
        run_decode(args)
    elif args.workload == "fp32":
        run_fp32(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
