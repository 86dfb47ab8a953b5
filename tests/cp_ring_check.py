"""Context parallelism over NCCL, one process per GPU (run under torchrun).

Each rank takes its zigzag shard of one long sequence, runs forward and
backward through an autograd entry point -- the K/V ring
(context_parallel_attention) by default, Ulysses (ulysses_attention) with the
argument "ulysses" -- and rank 0 compares the gathered O, dQ, dK, dV with the
single-GPU kernels on the whole sequence. Prints "cp ring ok" / "cp ulysses
ok" on success; exits non-zero otherwise.

With the argument "leave" the ring runs under a RingWatchdog: after one full
step (forward and backward, device synchronised) the last rank leaves between
steps, with nothing in flight. Every other rank must raise PeerFailure at its
next transfer -- learned on the host, through the store -- abort its NCCL
communicator and exit; rank 0 then prints "cp leave ok".
"""
import os
import sys
import time
from datetime import timedelta

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "npu-flex-att_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import context_parallel as cp  # noqa: E402
import npu_flash_attention as nfa  # noqa: E402


def leave_check(rank, world, dev):
    B, Hq, Hkv, S, D = 1, 4, 2, 1024, 128
    g = torch.Generator().manual_seed(5)
    q, k, v, go = (torch.randn(B, h, S, D, generator=g).to(torch.bfloat16).to(dev)
                   for h in (Hq, Hkv, Hkv, Hq))
    lay = cp.ZigzagLayout(S, world)
    wd = cp.RingWatchdog.for_group(timeout_s=5.0)

    def step():
        qs, ks, vs = (lay.shard(t, rank).requires_grad_(True) for t in (q, k, v))
        o = cp.context_parallel_attention(qs, ks, vs, causal=True, watchdog=wd)
        o.backward(lay.shard(go, rank))
        torch.cuda.synchronize()

    step()
    if rank == world - 1:
        print(f"rank {rank}: leaving between steps", flush=True)
        os._exit(0)
    t0 = time.monotonic()
    try:
        step()
        print(f"rank {rank}: no failure seen", file=sys.stderr, flush=True)
        os._exit(1)
    except cp.PeerFailure as e:
        dt = time.monotonic() - t0
        print(f"rank {rank}: PeerFailure after {dt:.2f} s: {e}", flush=True)
        if rank == 0:
            print("cp leave ok", flush=True)
        os._exit(0 if dt < 30 else 1)


def main():
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    mode = sys.argv[1] if len(sys.argv) > 1 else "ring"
    if mode == "leave":
        leave_check(rank, world, dev)
    attn = cp.ulysses_attention if mode == "ulysses" else cp.context_parallel_attention
    ok = True
    try:
        B, Hq, Hkv, S, D = 1, 8, 2, 2048, 128
        g = torch.Generator().manual_seed(11)
        q = torch.randn(B, Hq, S, D, generator=g).to(torch.bfloat16).to(dev)
        k = torch.randn(B, Hkv, S, D, generator=g).to(torch.bfloat16).to(dev)
        v = torch.randn(B, Hkv, S, D, generator=g).to(torch.bfloat16).to(dev)
        go = torch.randn(B, Hq, S, D, generator=g).to(torch.bfloat16).to(dev)
        slopes = torch.tensor([2.0 ** -(i + 1) for i in range(Hq)], device=dev)
        mask = dict(causal=True, alibi_slope=slopes)
        lay = cp.ZigzagLayout(S, world)
        qs, ks, vs = (lay.shard(t, rank).requires_grad_(True) for t in (q, k, v))
        o = attn(qs, ks, vs, **mask)
        o.backward(lay.shard(go, rank))
        outs = [o.detach(), qs.grad, ks.grad, vs.grad]
        gathered = []
        for t in outs:
            parts = [torch.empty_like(t) for _ in range(world)]
            dist.all_gather(parts, t.contiguous())
            gathered.append(lay.unshard(parts))
        torch.cuda.synchronize()
        nfa.check_device_status(dev)
        if rank == 0:
            o1, l1 = nfa.npu_flash_attention_forward(q, k, v, return_lse=True, **mask)
            g1 = nfa.npu_flash_attention_backward(q, k, v, o1, l1, go, **mask)
            for name, a, r in zip(("o", "dq", "dk", "dv"), gathered, (o1, *g1)):
                a, r = a.double(), r.double()
                e = ((a - r).abs() / (1 + r.abs())).max().item()
                print(f"{name}: max err vs single GPU {e:.3e}")
                ok = ok and e < 3e-2
    except Exception as e:  # every rank reaches the barrier-free teardown
        print(f"rank {rank}: {e!r}", file=sys.stderr)
        ok = False
    finally:
        dist.destroy_process_group()
    if rank == 0 and ok:
        print(f"cp {mode} ok")
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
