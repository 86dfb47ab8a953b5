"""Benchmark: fwd+bwd attention TFLOPS on B200 (BASELINE.json metric).

Workload (the metric's headline config): bf16
Llama-3-8B-style GQA layer, B=4 per GPU, Hq=32, Hkv=8, D=128, S=4096, causal,
scale 1/sqrt(128); q, k, v, grad_out ~ N(0,1) seeded, synthetic.

One step = one forward + one backward of that layer through the library's
C ABI (bfa_fwd, then Δ, dK/dV, dQ as three calls on one workspace so each
kernel is timed on its own). FLOPs count only unmasked (i, j) pairs,
element-exact: 4·D per pair forward, 10·D backward.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 is launched with torchrun (one process per GPU); each rank runs its own
batch shard (weak scaling, no collective on the data path); the step time is
the max over ranks. `--impl reference` times the reference's math path on the
host CPU cores (the CPU restatement in oracle/; the reference itself is
Triton for Ascend NPUs and has no GPU or CPU build that runs here).
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
CFG = dict(B=4, Hq=32, Hkv=8, S=4096, D=128, causal=True)
WORKLOAD = "c3: bf16 GQA B=4/GPU Hq=32 Hkv=8 D=128 S=4096 causal fwd+bwd"


def causal_pairs(s: int) -> int:
    return s * (s + 1) // 2


def step_flops(cfg=CFG) -> float:
    pairs = causal_pairs(cfg["S"]) * cfg["B"] * cfg["Hq"]
    return 14.0 * cfg["D"] * pairs


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            m = json.load(f)
        return float(m["bf16_tflops"]), float(m["hbm_gbs"]), "measured"
    except Exception:
        return 1590.0, 6650.0, "fallback"


def committed_traffic(phase: str):
    """DRAM bytes per launch of a kernel from the committed ncu capture, or None."""
    kernel = {"fwd": "fwd_kernel", "dkdv": "dkdv_kernel", "dq": "dq_kernel"}.get(phase)
    try:
        with open(os.path.join(ROOT, "profiles", "c3_dram_traffic.json")) as f:
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
    g = torch.Generator().manual_seed(seed)
    B, Hq, Hkv, S, D = cfg["B"], cfg["Hq"], cfg["Hkv"], cfg["S"], cfg["D"]
    # Generated on the device from a seeded generator (the full tensors are GBs).
    gd = torch.Generator(device=device).manual_seed(seed)
    q = torch.randn(B, Hq, S, D, generator=gd, device=device, dtype=torch.bfloat16)
    k = torch.randn(B, Hkv, S, D, generator=gd, device=device, dtype=torch.bfloat16)
    v = torch.randn(B, Hkv, S, D, generator=gd, device=device, dtype=torch.bfloat16)
    do = torch.randn(B, Hq, S, D, generator=gd, device=device, dtype=torch.bfloat16)
    del g
    return q, k, v, do


def cpu_baseline_sample(budget_s: float = 15.0):
    """The reference's math path (oracle restatement) on the host cores.

    Times fwd+bwd of single (b, q-head) slices of the workload (S=4096,
    D=128, causal, fp32) until ~budget_s seconds of CPU work, and scales FLOPs
    per slice; returns (TFLOPS, threads, slices)."""
    from oracle.attention_math import attention_backward, attention_forward
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(0)
    S, D = CFG["S"], CFG["D"]
    q, k, v, do = (torch.randn(1, 1, S, D, generator=g) for _ in range(4))
    slice_flops = 14.0 * D * causal_pairs(S)
    attention_forward(q[:, :, :256], k[:, :, :256], v[:, :, :256], causal=True, dtype=torch.float32)
    t0 = time.perf_counter()
    n = 0
    while True:
        o, lse = attention_forward(q, k, v, causal=True, dtype=torch.float32)
        attention_backward(q, k, v, do, causal=True, out=o, lse=lse, dtype=torch.float32)
        n += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    return n * slice_flops / dt / 1e12, threads, n


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    per_step = []
    tflops_all = []
    for i in range(args.warmup + args.steps):
        tf, threads, n = cpu_baseline_sample(budget_s=2.0)
        if i >= args.warmup:
            tflops_all.append(tf)
            per_step.append(n)
    value = statistics.median(tflops_all)
    ms = step_flops() / (value * 1e12) * 1e3
    out = {
        "impl": "reference", "metric": METRIC, "value": round(value, 6), "unit": "TFLOPS",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,1))",
        "config": {"workload": WORKLOAD, "global_batch": CFG["B"] * args.gpus, "seq_len": CFG["S"],
                   "parallelism": "host CPU, all cores"},
        "cpu_baseline": {"value": round(value, 6), "unit": "TFLOPS", "cores": threads,
                         "kind": "port",
                         "sample": "per step: fwd+bwd of whole (b, q-head) slices of the workload "
                                   "(S=4096, D=128, causal, fp32) for ~2 s; TFLOPS scale per slice"},
        "e2e": {"value": round(value, 6), "unit": "TFLOPS", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(out), flush=True)


def run_ours(args):
    import bfa_lib
    import npu_flash_attention as nfa

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                             device_id=dev)
    lib = bfa_lib.load()
    q, k, v, do = make_inputs(1234 + rank, dev)
    B, Hq, Hkv, S, D = CFG["B"], CFG["Hq"], CFG["Hkv"], CFG["S"], CFG["D"]
    o = torch.empty_like(q)
    lse = torch.empty(B, Hq, S, device=dev, dtype=torch.float32)
    grads = (torch.empty_like(q), torch.empty_like(k), torch.empty_like(v))
    pr = nfa._problem(q, k, True, 0, None, 1.0 / math.sqrt(D), 0.0)
    ws = torch.empty(lib.bfa_bwd_workspace_bytes(pr), dtype=torch.uint8, device=dev)
    kw = dict(causal=True)

    def step(ev=None):
        if ev:
            ev[0].record()
        out, l_ = nfa.npu_flash_attention_forward(q, k, v, return_lse=True, **kw)
        if ev:
            ev[1].record()
        nfa.npu_flash_attention_backward(q, k, v, out, l_, do, _phases=bfa_lib.PHASE_DELTA,
                                         _workspace=ws, _outputs=grads, **kw)
        if ev:
            ev[2].record()
        nfa.npu_flash_attention_backward(q, k, v, out, l_, do, _phases=bfa_lib.PHASE_DKDV,
                                         _workspace=ws, _outputs=grads, **kw)
        if ev:
            ev[3].record()
        nfa.npu_flash_attention_backward(q, k, v, out, l_, do, _phases=bfa_lib.PHASE_DQ,
                                         _workspace=ws, _outputs=grads, **kw)
        if ev:
            ev[4].record()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    nfa.check_device_status(dev)

    events = [[torch.cuda.Event(enable_timing=True) for _ in range(5)] for _ in range(args.steps)]
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
    total_ms = start.elapsed_time(end)
    phase_ms = [sum(events[i][j].elapsed_time(events[i][j + 1]) for i in range(args.steps)) / args.steps
                for j in range(4)]
    if world > 1:
        t = torch.tensor([total_ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        total_ms = float(t.item())
    ms_step = total_ms / args.steps
    flops = step_flops()
    value = world * flops / (ms_step * 1e-3) / 1e12

    # ---- e2e: public autograd API, host (pinned) buffers, copies inside the timed region
    e2e = None if args.profile else run_e2e(nfa, dev, args, world)

    peak_tf, _, peak_kind = peaks()
    pairs = causal_pairs(S) * B * Hq
    kern_flops = {"fwd": 4.0 * D * pairs, "delta": 0.0, "dkdv": 8.0 * D * pairs, "dq": 6.0 * D * pairs}
    names = ["fwd", "delta", "dkdv", "dq"]
    dom = max(range(4), key=lambda j: phase_ms[j])
    achieved = kern_flops[names[dom]] / (phase_ms[dom] * 1e-3) / 1e12
    roofline = {"bound": "tensor", "kernel": names[dom], "achieved": round(achieved, 2),
                "peak": peak_tf, "unit": "TFLOP/s", "frac": round(achieved / peak_tf, 4),
                "peak_kind": f"bf16 dense burst, {peak_kind}",
                "traffic": committed_traffic(names[dom]),
                "traffic_unit": "DRAM bytes per launch (ncu capture, profiles/c3_dram_traffic.json)",
                "algorithmic_flop_per_launch": kern_flops[names[dom]],
                "phase_ms": {n: round(x, 4) for n, x in zip(names, phase_ms)}}
    cpu = None
    if rank == 0 and world == 1 and not (args.no_cpu_baseline or args.profile):
        tf, threads, n = cpu_baseline_sample(budget_s=args.cpu_budget)
        cpu = {"value": round(tf, 6), "unit": "TFLOPS", "cores": threads, "kind": "port",
               "sample": f"{n} whole (b, q-head) slices of the workload (S=4096, D=128, causal, "
                         f"fp32 fwd+bwd) in ~{args.cpu_budget:.0f} s; TFLOPS scale per slice"}
    if rank == 0:
        out = {
            "metric": METRIC, "value": round(value, 3), "unit": "TFLOPS", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1), generated on device)",
            "config": {"workload": WORKLOAD, "global_batch": B * world, "seq_len": S,
                       "parallelism": f"batch x head shards on {world} GPU(s), no collective",
                       "l2": "inputs larger than L2 (q 268 MB, dO 268 MB, k/v 67 MB each)"},
            "pct_of_peak": round(100.0 * value / world / peak_tf, 2),
            "gpu_launches": int(launches),
            "roofline": roofline,
            "cpu_baseline": cpu,
            "e2e": e2e,
            "clocks": clocks,
        }
        print(json.dumps(out), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def run_e2e(nfa, dev, args, world):
    """Same metric through the public autograd API with host buffers: every
    step copies q, k, v, dO from pinned host memory, runs flex_attention
    forward + backward, and reads dQ, dK, dV back to pinned host memory.

    The steps are pipelined the way a training loop feeds a GPU: step i+1's
    inputs are copied in on one stream (into the second of two device
    buffers) and step i-1's gradients are copied out on another while step i
    computes, so the two PCIe directions overlap each other and the kernels.
    The timed region holds every step's copies, from the first input copy to
    the last gradient read-back."""
    B, Hq, Hkv, S, D = CFG["B"], CFG["Hq"], CFG["Hkv"], CFG["S"], CFG["D"]
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
            out = nfa.flex_attention(qd, kd, vd, causal=True)
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

    steps = max(2, min(args.steps, 5))
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
    ms = s.elapsed_time(e) / steps
    if world > 1:
        t = torch.tensor([ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    return {"value": round(world * step_flops() / (ms * 1e-3) / 1e12, 3), "unit": "TFLOPS",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(ms, 3),
            "steps": steps, "pipelined": "H2D of step i+1 and D2H of step i-1 overlap step i"}


C5 = dict(B=1, Hq=64, Hkv=8, S=65536, D=128)
C5_WORKLOAD = "c5: bf16 B=1 Hq=64 Hkv=8 D=128 S=65536 causal + ALiBi, context-parallel K/V ring"
C5U_WORKLOAD = ("c5: bf16 B=1 Hq=64 Hkv=8 D=128 S=65536 causal + ALiBi, context-parallel Ulysses "
                "(head-sequence all-to-alls)")


def run_c5(args, ulysses=False):
    """Config 5 through context parallelism (one process per GPU): each rank
    holds its zigzag shard (2 chunks of S/(2N) rows) of Q, K, V and runs
    forward + backward with context_parallel_attention (the K/V ring) or, for
    --workload c5u, ulysses_attention. FLOPs count the unmasked pairs of the
    whole causal sequence (14·D per pair per q-head)."""
    import datetime
    import context_parallel as cp
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29517")
    torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev,
                                         rank=rank, world_size=world)
    B, Hq, Hkv, S, D = C5["B"], C5["Hq"], C5["Hkv"], C5["S"], C5["D"]
    rows = S // world
    gd = torch.Generator(device=dev).manual_seed(4321 + rank)
    q = torch.randn(B, Hq, rows, D, generator=gd, device=dev, dtype=torch.bfloat16).requires_grad_(True)
    k = torch.randn(B, Hkv, rows, D, generator=gd, device=dev, dtype=torch.bfloat16).requires_grad_(True)
    v = torch.randn(B, Hkv, rows, D, generator=gd, device=dev, dtype=torch.bfloat16).requires_grad_(True)
    do = torch.randn(B, Hq, rows, D, generator=gd, device=dev, dtype=torch.bfloat16)
    slopes = torch.tensor([2.0 ** (-8.0 * (i + 1) / Hq) for i in range(Hq)], device=dev)

    def step():
        q.grad = k.grad = v.grad = None
        attn = cp.ulysses_attention if ulysses else cp.context_parallel_attention
        o = attn(q, k, v, causal=True, alibi_slope=slopes)
        o.backward(do)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    torch.distributed.barrier()
    s_, e_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s_.record()
    for _ in range(args.steps):
        step()
    e_.record()
    torch.cuda.synchronize()
    t = torch.tensor([s_.elapsed_time(e_) / args.steps], device=dev)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    ms = float(t.item())
    flops = 14.0 * D * causal_pairs(S) * B * Hq
    peak_tf, _, peak_kind = peaks()
    if rank == 0:
        value = flops / (ms * 1e-3) / 1e12
        print(json.dumps({
            "metric": METRIC, "value": round(value, 3), "unit": "TFLOPS", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1), generated on device)",
            "config": {"workload": C5U_WORKLOAD if ulysses else C5_WORKLOAD, "global_batch": B, "seq_len": S,
                       "parallelism": (f"Ulysses all-to-alls over {world} GPU(s), NCCL" if ulysses else
                                       f"context-parallel zigzag K/V ring over {world} GPU(s), NCCL")},
            "pct_of_peak": round(100.0 * value / world / peak_tf, 2),
            "gpu_launches": None, "roofline": None, "cpu_baseline": None, "e2e": None,
            "note": ("auxiliary measurement of " + ("Ulysses" if ulysses else "the P-2 ring") +
                     "; the headline line is the default c3 run")}),
            flush=True)
    torch.distributed.barrier()
    torch.distributed.destroy_process_group()


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
    ap.add_argument("--workload", choices=["c3", "c5", "c5u", "decode"], default="c3",
                    help="c3 (default, the headline), c5 (context-parallel ring), c5u (context-"
                         "parallel Ulysses) or decode (split-KV decoding forward)")
    ap.add_argument("--profile", action="store_true",
                    help="for ncu: only the warm-up and timed steps (no e2e, no CPU baseline)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.workload in ("c5", "c5u"):
        run_c5(args, ulysses=args.workload == "c5u")
    elif args.workload == "decode":
        run_decode(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
