"""Context-parallel ring on the GPU.

Simulated ranks (one GPU, one process) run the ring with the CUDA block ops:
every block is a libbfa forward that merges its result into the running
(O, LSE) in its epilogue and an accumulate-mode backward, with absolute
position offsets. The gathered result is
checked against the oracle over the whole sequence. With two or more GPUs the
same ring runs over NCCL between processes (tests/cp_ring_check.py).
"""
import os
import subprocess
import sys

import pytest
import torch

import context_parallel as cp
from oracle.attention_math import attention_backward, attention_forward

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
TOL = 2e-2  # bf16, allclose form |a - r| / (1 + |r|)


def _err(a, r):
    a, r = a.detach().cpu().double(), r.double()
    return ((a - r).abs() / (1.0 + r.abs())).max().item()


SLOPES = torch.tensor([2.0 ** -(i + 1) for i in range(8)])
CASES = {
    "causal": dict(causal=True),
    "alibi": dict(causal=True, alibi_slope=SLOPES),
    "window": dict(causal=True, sliding_window=200),
    "full_cap": dict(soft_cap=20.0),
}


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("case", list(CASES), ids=list(CASES))
def test_simulated_ring_cuda_matches_oracle(world, case):
    mask = CASES[case]
    g = torch.Generator().manual_seed(world)
    B, Hq, Hkv, S, D = 1, 8, 2, 1024, 128
    q = torch.randn(B, Hq, S, D, generator=g).to(torch.bfloat16)
    k = torch.randn(B, Hkv, S, D, generator=g).to(torch.bfloat16)
    v = torch.randn(B, Hkv, S, D, generator=g).to(torch.bfloat16)
    go = torch.randn(B, Hq, S, D, generator=g).to(torch.bfloat16)
    lay = cp.ZigzagLayout(S, world)
    m_dev = cp.MaskArgs(**{**mask, **({"alibi_slope": mask["alibi_slope"].to(DEV)}
                                      if "alibi_slope" in mask else {})})
    ops = cp.CudaBlockOps()
    sh = [[lay.shard(t, r).to(DEV) for t in (q, k, v, go)] for r in range(world)]
    fw = cp.run_simulated([cp.ring_forward(s[0], s[1], s[2], r, world, m_dev, ops)
                           for r, s in enumerate(sh)])
    bw = cp.run_simulated([cp.ring_backward(s[0], s[1], s[2], fw[r][0], fw[r][1], s[3],
                                            r, world, m_dev, ops) for r, s in enumerate(sh)])
    torch.cuda.synchronize()
    o = lay.unshard([f[0].cpu() for f in fw])
    lse = lay.unshard([f[1].cpu() for f in fw])
    dq, dk, dv = (lay.unshard([b_[i].cpu() for b_ in bw]) for i in range(3))
    o_r, lse_r = attention_forward(q, k, v, **mask)
    assert _err(o, o_r) < TOL
    assert ((lse.double() - lse_r).abs() / lse_r.abs().clamp_min(1)).max().item() < 1e-3
    # The backward as an operator of (q, k, v, out, lse, dout), given the
    # ring's own out and lse; P and dS enter the products in bf16.
    rq, rk, rv = attention_backward(q, k, v, go, out=o, lse=lse.double(),
                                    operand_dtype=torch.bfloat16, **mask)
    for name, a, r in (("dq", dq, rq), ("dk", dk, rk), ("dv", dv, rv)):
        assert _err(a, r) < TOL, (name, _err(a, r))


def test_accumulate_mode_adds_into_fp32():
    """bfa_bwd with accumulate=1 adds to what the fp32 buffers hold."""
    import npu_flash_attention as nfa
    g = torch.Generator().manual_seed(3)
    q, k, v, go = (torch.randn(1, 4, 384, 128, generator=g).to(torch.bfloat16).to(DEV)
                   for _ in range(4))
    k, v = k[:, :2].contiguous(), v[:, :2].contiguous()
    o, lse = nfa.npu_flash_attention_forward(q, k, v, causal=True, return_lse=True)
    dq, dk, dv = nfa.npu_flash_attention_backward(q, k, v, o, lse, go, causal=True)
    base = [torch.full(t.shape, 0.5, device=DEV, dtype=torch.float32) for t in (dq, dk, dv)]
    acc = [b_.clone() for b_ in base]
    nfa.npu_flash_attention_backward(q, k, v, o, lse, go, causal=True,
                                     _outputs=tuple(acc), _accumulate=True)
    torch.cuda.synchronize()
    for a, b_, ref in zip(acc, base, (dq, dk, dv)):
        got = (a - b_).cpu().double()
        assert _err(got, ref.cpu().double()) < 1e-2
    with pytest.raises(ValueError):
        nfa.npu_flash_attention_backward(q, k, v, o, lse, go, causal=True,
                                         _outputs=(dq, dk, dv), _accumulate=True)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ring_over_nccl_two_gpus():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node=2", "--master-addr", "127.0.0.1",
           "--master-port", "29531", os.path.join(ROOT, "tests", "cp_ring_check.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=400)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "cp ring ok" in r.stdout


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ring_rank_that_leaves_is_detected_over_nccl():
    """Two GPUs, NVLS off: after one full step rank 1 leaves between steps
    (device synchronised, nothing in flight); rank 0's RingWatchdog sees it on
    the host before its next transfer, aborts its communicator and exits."""
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node=2", "--master-addr", "127.0.0.1",
           "--master-port", "29533", os.path.join(ROOT, "tests", "cp_ring_check.py"), "leave"]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=400)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "cp leave ok" in r.stdout


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("case", ["causal", "alibi", "full_cap"])
def test_simulated_ulysses_cuda_matches_single_gpu(world, case):
    """Ulysses over simulated ranks with the CUDA ops: each rank runs the
    single-GPU kernels on the whole sequence for its head group, so the
    gathered O and gradients equal the single-GPU run on all heads."""
    import npu_flash_attention as nfa
    mask = CASES[case]
    mask_dev = {**mask, **({"alibi_slope": mask["alibi_slope"].to(DEV)} if "alibi_slope" in mask else {})}
    g = torch.Generator().manual_seed(10 + world)
    B, Hq, Hkv, S, D = 1, 8, 4, 1024, 128
    q, k, v = (torch.randn(B, h, S, D, generator=g).to(torch.bfloat16).to(DEV) for h in (Hq, Hkv, Hkv))
    go = torch.randn(B, Hq, S, D, generator=g).to(torch.bfloat16).to(DEV)
    lay = cp.ZigzagLayout(S, world)
    sh = [[lay.shard(t, r) for r in range(world)] for t in (q, k, v, go)]
    got = cp.ulysses_simulated(*sh, cp.MaskArgs(**mask_dev), cp.CudaAttentionOps())
    o1, l1 = nfa.npu_flash_attention_forward(q, k, v, return_lse=True, **mask_dev)
    ref = (o1, *nfa.npu_flash_attention_backward(q, k, v, o1, l1, go, **mask_dev))
    torch.cuda.synchronize()
    for name, shards, r in zip(("o", "dq", "dk", "dv"), got, ref):
        assert _err(lay.unshard(shards), r.cpu()) < TOL, name


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ulysses_over_nccl_two_gpus():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node=2", "--master-addr", "127.0.0.1",
           "--master-port", "29532", os.path.join(ROOT, "tests", "cp_ring_check.py"), "ulysses"]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=400)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "cp ulysses ok" in r.stdout
