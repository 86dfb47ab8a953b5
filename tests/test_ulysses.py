"""Ulysses context parallelism (context_parallel.ulysses_attention) on CPU.

The head <-> sequence all-to-alls and the head-group bookkeeping (GQA groups,
ALiBi slopes, zigzag / contiguous layouts) are checked with the CPU oracle as
the per-rank attention: in one process over simulated ranks, and through the
autograd entry point over gloo ranks. The result must equal single-device
attention on the whole sequence (fp64, 1e-9 relative).
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

import context_parallel as cp
from oracle.attention_math import attention_backward, attention_forward


class OracleAttentionOps:
    """Whole-sequence attention through the CPU oracle (fp64), the interface
    of context_parallel.CudaAttentionOps."""

    @staticmethod
    def _kw(m):
        return dict(causal=m.causal, sliding_window=m.sliding_window, alibi_slope=m.alibi_slope,
                    scale=m.scale, soft_cap=m.soft_cap)

    def fwd(self, q, k, v, m):
        return attention_forward(q, k, v, **self._kw(m))

    def bwd(self, q, k, v, o, lse, do, m):
        return attention_backward(q, k, v, do, out=o, lse=lse, **self._kw(m))


HQ, HKV, S, D = 8, 4, 64, 16
SLOPES = torch.tensor([2.0 ** -(i + 1) for i in range(HQ)], dtype=torch.float64)
MASKS = {
    "full": dict(),
    "causal": dict(causal=True),
    "causal_window": dict(causal=True, sliding_window=11),
    "alibi_cap": dict(causal=True, soft_cap=4.0, alibi_slope=SLOPES),
}


def _data(seed, b=2):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(b, HQ, S, D, generator=g, dtype=torch.float64)
    k = torch.randn(b, HKV, S, D, generator=g, dtype=torch.float64)
    v = torch.randn(b, HKV, S, D, generator=g, dtype=torch.float64)
    go = torch.randn(b, HQ, S, D, generator=g, dtype=torch.float64)
    return q, k, v, go


def _reference(q, k, v, go, mask):
    o, lse = attention_forward(q, k, v, **mask)
    dq, dk, dv = attention_backward(q, k, v, go, out=o, lse=lse, **mask)
    return o, dq, dk, dv


def _close(a, ref, tol=1e-9):
    a, ref = a.double(), ref.double()
    return (a - ref).abs().max().item() / (1.0 + ref.abs().max().item()) < tol


def test_layouts_roundtrip():
    x = torch.arange(2 * 3 * 24 * 2).view(2, 3, 24, 2).float()
    for name in ("zigzag", "contiguous"):
        lay = cp.make_layout(name, 24, 3)
        assert torch.equal(lay.unshard([lay.shard(x, r) for r in range(3)]), x)
    with pytest.raises(ValueError):
        cp.make_layout("striped", 24, 3)


def test_all_to_all_helpers_invert_each_other():
    world, lay = 4, cp.ZigzagLayout(S, 4)
    x = torch.randn(2, HQ, S, D, dtype=torch.float64)
    shards = [lay.shard(x, r) for r in range(world)]
    sends = [cp._h2s_send(s, world) for s in shards]
    recvs = [torch.stack([sends[i][r] for i in range(world)], 0) for r in range(world)]
    full = [cp._h2s_finish(rv, lay) for rv in recvs]
    hg = HQ // world
    for r in range(world):  # rank r holds every row of head group r
        assert torch.equal(full[r], x[:, r * hg:(r + 1) * hg])
    sends = [cp._s2h_send(f, world, lay) for f in full]
    recvs = [torch.stack([sends[i][r] for i in range(world)], 0) for r in range(world)]
    back = [cp._s2h_finish(rv) for rv in recvs]
    for r in range(world):
        assert torch.equal(back[r], shards[r])


@pytest.mark.parametrize("world", [1, 2, 4])
@pytest.mark.parametrize("layout", ["zigzag", "contiguous"])
@pytest.mark.parametrize("mask", list(MASKS))
def test_ulysses_simulated_matches_single_device(world, layout, mask):
    q, k, v, go = _data(3)
    lay = cp.make_layout(layout, S, world)
    sh = [[lay.shard(t, r) for r in range(world)] for t in (q, k, v, go)]
    got = cp.ulysses_simulated(*sh, cp.MaskArgs(**MASKS[mask]), OracleAttentionOps(), layout)
    for g_shards, ref in zip(got, _reference(q, k, v, go, MASKS[mask])):
        assert _close(lay.unshard(g_shards), ref)


def test_ulysses_rejects_indivisible_heads():
    q, k, v, go = _data(4)
    lay = cp.ZigzagLayout(S, 8)  # HKV = 4 is not divisible by 8
    sh = [[lay.shard(t, r) for r in range(8)] for t in (q, k, v, go)]
    with pytest.raises(ValueError):
        cp.ulysses_simulated(*sh, cp.MaskArgs(), OracleAttentionOps())


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_rank(rank, world, port, mask_name, layout, out_q):
    import torch.distributed as dist
    from datetime import timedelta
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        mask = MASKS[mask_name]
        q, k, v, go = _data(5)
        lay = cp.make_layout(layout, S, world)
        qs, ks, vs = (lay.shard(t, rank).requires_grad_(True) for t in (q, k, v))
        o = cp.ulysses_attention(qs, ks, vs, layout=layout, _ops=OracleAttentionOps(), **mask)
        o.backward(lay.shard(go, rank))
        ref = _reference(q, k, v, go, mask)
        ok = all(_close(a, lay.shard(r, rank))
                 for a, r in zip((o.detach(), qs.grad, ks.grad, vs.grad), ref))
        out_q.put((rank, ok))
    except Exception as e:  # report, never hang the parent
        out_q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,mask,layout", [(2, "causal", "zigzag"), (4, "alibi_cap", "zigzag"),
                                               (2, "causal_window", "contiguous")])
def test_ulysses_over_gloo_ranks(world, mask, layout):
    ctx = mp.get_context("spawn")
    out_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gloo_rank, args=(r, world, port, mask, layout, out_q))
             for r in range(world)]
    for p in procs:
        p.start()
    results = dict(out_q.get(timeout=180) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    assert results == {r: True for r in range(world)}, results
