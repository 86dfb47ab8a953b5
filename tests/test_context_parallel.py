"""Context-parallel ring (CPU): the ring algorithm over oracle block ops.

The ring code that runs on GPUs (ring_forward / ring_backward, the zigzag
layout, block skipping, the merge and the dK/dV travel) runs here with each
block computed by the fp64 oracle, on simulated ranks in one process and on
real gloo ranks (world size 2 and 4). The result must equal single-device
attention over the whole sequence.
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

import context_parallel as cp
from oracle.attention_math import attention_backward, attention_forward


class OracleBlockOps:
    """Block ops through the CPU oracle (fp64), same interface as CudaBlockOps."""

    @staticmethod
    def _kw(m, q_off, k_off):
        return dict(causal=m.causal, sliding_window=m.sliding_window,
                    alibi_slope=m.alibi_slope, scale=m.scale, soft_cap=m.soft_cap,
                    q_offset=q_off, k_offset=k_off)

    def fwd(self, q, k, v, q_off, k_off, m):
        return attention_forward(q, k, v, **self._kw(m, q_off, k_off))

    def fwd_merge(self, o_acc, lse_acc, q, k, v, q_off, k_off, m):
        o_p, lse_p = self.fwd(q, k, v, q_off, k_off, m)
        self.merge(o_acc, lse_acc, o_p, lse_p)

    def merge(self, o_acc, lse_acc, o_part, lse_part):
        new = torch.logaddexp(lse_acc, lse_part.to(lse_acc.dtype))
        safe = torch.where(torch.isfinite(new), new, torch.zeros_like(new))
        wa = torch.where(torch.isfinite(new), torch.exp(lse_acc - safe), torch.zeros_like(new))
        wp = torch.where(torch.isfinite(new), torch.exp(lse_part - safe), torch.zeros_like(new))
        o_acc.copy_(o_acc * wa.unsqueeze(-1) + o_part.to(o_acc.dtype) * wp.unsqueeze(-1))
        lse_acc.copy_(new)

    def bwd_rows(self, q, k, o, do, lse, q_off, m):
        return None

    def bwd_into(self, state, q, k, v, o, lse, do, q_off, k_off, m, dq_acc, dk_acc, dv_acc):
        dq, dk, dv = attention_backward(q, k, v, do, out=o, lse=lse, **self._kw(m, q_off, k_off))
        dq_acc += dq.to(dq_acc.dtype)
        dk_acc += dk.to(dk_acc.dtype)
        dv_acc += dv.to(dv_acc.dtype)


def _close(a, ref, tol=1e-5):
    a, ref = a.double(), ref.double()
    return (a - ref).abs().max().item() / (1.0 + ref.abs().max().item()) < tol


MASKS = {
    "causal": dict(causal=True),
    "full": dict(),
    "causal_window": dict(causal=True, sliding_window=11),
    "alibi_cap": dict(causal=True, soft_cap=4.0,
                      alibi_slope=torch.tensor([0.5, 0.25, 0.125, 0.0625], dtype=torch.float64)),
}


def _data(seed, s, b=1, hq=4, hkv=2, d=16):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(b, hq, s, d, generator=g, dtype=torch.float64)
    k = torch.randn(b, hkv, s, d, generator=g, dtype=torch.float64)
    v = torch.randn(b, hkv, s, d, generator=g, dtype=torch.float64)
    go = torch.randn(b, hq, s, d, generator=g, dtype=torch.float64)
    return q, k, v, go


def _reference(q, k, v, go, mask):
    o, lse = attention_forward(q, k, v, **mask)
    dq, dk, dv = attention_backward(q, k, v, go, out=o, lse=lse, **mask)
    return o, lse, dq, dk, dv


def _ring_simulated(q, k, v, go, world, mask):
    lay = cp.ZigzagLayout(q.shape[2], world)
    m = cp.MaskArgs(**mask)
    ops = OracleBlockOps()
    sh = [[lay.shard(t, r) for t in (q, k, v, go)] for r in range(world)]
    fw = cp.run_simulated([cp.ring_forward(s[0], s[1], s[2], r, world, m, ops)
                           for r, s in enumerate(sh)])
    bw = cp.run_simulated([cp.ring_backward(s[0], s[1], s[2], fw[r][0], fw[r][1], s[3],
                                            r, world, m, ops) for r, s in enumerate(sh)])
    o = lay.unshard([f[0] for f in fw])
    lse = lay.unshard([f[1] for f in fw])
    dq, dk, dv = (lay.unshard([b_[i] for b_ in bw]) for i in range(3))
    return o, lse, dq, dk, dv


def test_zigzag_layout_roundtrip():
    x = torch.arange(2 * 3 * 24).view(1, 2, 24, 3).float()
    lay = cp.ZigzagLayout(24, 3)
    assert lay.chunks(0) == (0, 5) and lay.chunks(2) == (2, 3)
    shards = [lay.shard(x, r) for r in range(3)]
    assert all(s.is_contiguous() and s.shape[2] == 8 for s in shards)
    assert torch.equal(lay.unshard(shards), x)
    with pytest.raises(ValueError):
        cp.ZigzagLayout(25, 3)


def test_block_visible():
    m = cp.MaskArgs(causal=True, sliding_window=10)
    assert cp.block_visible(2, 2, 8, m)           # diagonal
    assert not cp.block_visible(1, 2, 8, m)       # above the diagonal
    assert cp.block_visible(3, 2, 8, m)           # i - j from 1
    assert cp.block_visible(4, 2, 8, m)           # i - j from 9 <= W
    assert not cp.block_visible(5, 2, 8, m)       # i - j from 17 > W
    assert cp.block_visible(2, 5, 8, cp.MaskArgs())


@pytest.mark.parametrize("world", [1, 2, 3, 4])
@pytest.mark.parametrize("mask", list(MASKS), ids=list(MASKS))
def test_ring_simulated_matches_single_device(world, mask):
    s = 48 if world == 3 else 64
    q, k, v, go = _data(world, s)
    ref = _reference(q, k, v, go, MASKS[mask])
    got = _ring_simulated(q, k, v, go, world, MASKS[mask])
    for name, a, r in zip(("o", "lse", "dq", "dk", "dv"), got, ref):
        assert _close(a, r), name


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_rank(rank, world, port, mask_name, out_q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        mask = MASKS[mask_name]
        q, k, v, go = _data(7, 64)
        lay = cp.ZigzagLayout(64, world)
        sh = [lay.shard(t, rank) for t in (q, k, v, go)]
        m = cp.MaskArgs(**mask)
        ops = OracleBlockOps()
        o, lse = cp.run_dist(cp.ring_forward(sh[0], sh[1], sh[2], rank, world, m, ops))
        dq, dk, dv = cp.run_dist(cp.ring_backward(sh[0], sh[1], sh[2], o, lse, sh[3],
                                                  rank, world, m, ops))
        ref = _reference(q, k, v, go, mask)
        ok = all(_close(a, lay.shard(r, rank)) for a, r in zip((o, lse, dq, dk, dv), ref))
        out_q.put((rank, ok))
    except Exception as e:  # report, never hang the parent
        out_q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("mask", ["causal", "alibi_cap"])
def test_ring_over_gloo_ranks(world, mask):
    ctx = mp.get_context("spawn")
    out_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gloo_rank, args=(r, world, port, mask, out_q))
             for r in range(world)]
    for p in procs:
        p.start()
    results = dict(out_q.get(timeout=180) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    assert results == {r: True for r in range(world)}, results


def _lonely_rank(port, out_q):
    import torch.distributed as dist
    from datetime import timedelta
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=0, world_size=2, timeout=timedelta(seconds=3))
        out_q.put("joined")
    except Exception as e:
        out_q.put(type(e).__name__)


def test_rank_that_never_joins_times_out():
    """Failure detection on the host: rank 1 never joins; rank 0's rendezvous
    ends with an error after its short timeout instead of waiting forever."""
    ctx = mp.get_context("spawn")
    out_q = ctx.Queue()
    p = ctx.Process(target=_lonely_rank, args=(_free_port(), out_q))
    p.start()
    res = out_q.get(timeout=120)
    p.join(timeout=30)
    assert res != "joined"
