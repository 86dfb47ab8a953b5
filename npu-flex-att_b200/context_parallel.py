"""Context-parallel attention: a K/V ring over ranks with LSE merging.

The reference runs one sequence on one device. This module shards a long
sequence across ranks (one process per GPU) and keeps each rank's kernels
exactly the single-GPU ones (``bfa_fwd`` / ``bfa_bwd`` with absolute
position offsets), so masks, ALiBi and the soft-cap see true positions.

Layout (zigzag). The sequence of length S is cut into 2N chunks of C = S/(2N)
rows; rank r holds chunks r and 2N-1-r of Q, K and V. Under a causal mask
every rank then owns the same amount of work.

Forward. At step t = 0..N-1 rank r holds the K/V shard of rank (r - t) mod N;
for each of its two query chunks and each visiting key chunk that the mask
does not hide entirely it runs one attention call whose epilogue folds its
result into the fp32 running (O, LSE) of the query chunk
(``bfa_fwd_args.accumulate``; no partial result goes through memory):
    lse' = logaddexp(lse_acc, lse_p),  o' = o_acc e^(lse_acc-lse') + o_p e^(lse_p-lse').
The next K/V shard is in flight (NCCL send/recv) while the current one is used.

Backward. dK/dV accumulators travel with their K/V shard around the ring and
arrive home after N hops; dQ stays local. Each visible block runs the single-
GPU backward against the FINAL O and LSE (which is what makes the blockwise
gradients exact) and adds its gradients into fp32 accumulators in place
(``bfa_bwd_args.accumulate``), so partial gradients are never rounded to
16 bits. Δ = rowsum(O∘dO) is computed once per query chunk.

The ring algorithm is written as per-rank generators that yield their
communication steps, so the same code runs over ``torch.distributed``
(``run_dist``: NCCL on GPUs, gloo in CPU tests) and in one process over a list
of simulated ranks (``run_simulated``).
"""
from __future__ import annotations

import ctypes
import math
import time
from dataclasses import dataclass
from typing import Optional

import torch

import bfa_lib as _bfa
import npu_flash_attention as _nfa


# ---------------------------------------------------------------- layout
class ZigzagLayout:
    """Chunks {r, 2N-1-r} of the sequence on rank r (N = world size)."""

    def __init__(self, seqlen: int, world: int):
        if world < 1 or seqlen % (2 * world) != 0:
            raise ValueError(f"seqlen {seqlen} must be a multiple of 2*world ({2 * world})")
        self.seqlen, self.world = seqlen, world
        self.chunk = seqlen // (2 * world)

    def chunks(self, rank: int) -> tuple[int, int]:
        return rank, 2 * self.world - 1 - rank

    def shard(self, x: torch.Tensor, rank: int, dim: int = 2) -> torch.Tensor:
        """This rank's rows of a full-sequence tensor, contiguous."""
        a, b = self.chunks(rank)
        c = self.chunk
        return torch.cat([x.narrow(dim, a * c, c), x.narrow(dim, b * c, c)], dim=dim).contiguous()

    def unshard(self, shards: list[torch.Tensor], dim: int = 2) -> torch.Tensor:
        """Inverse of ``shard`` over all ranks' shards."""
        c = self.chunk
        parts: list[Optional[torch.Tensor]] = [None] * (2 * self.world)
        for r, s in enumerate(shards):
            a, b = self.chunks(r)
            parts[a] = s.narrow(dim, 0, c)
            parts[b] = s.narrow(dim, c, c)
        return torch.cat(parts, dim=dim)


class ContiguousLayout:
    """Rows [r·S/N, (r+1)·S/N) of the sequence on rank r (N = world size)."""

    def __init__(self, seqlen: int, world: int):
        if world < 1 or seqlen % world != 0:
            raise ValueError(f"seqlen {seqlen} must be a multiple of world ({world})")
        self.seqlen, self.world = seqlen, world
        self.rows = seqlen // world

    def shard(self, x: torch.Tensor, rank: int, dim: int = 2) -> torch.Tensor:
        return x.narrow(dim, rank * self.rows, self.rows).contiguous()

    def unshard(self, shards: list[torch.Tensor], dim: int = 2) -> torch.Tensor:
        return torch.cat(list(shards), dim=dim)


def make_layout(name: str, seqlen: int, world: int):
    if name == "zigzag":
        return ZigzagLayout(seqlen, world)
    if name == "contiguous":
        return ContiguousLayout(seqlen, world)
    raise ValueError(f"unknown layout {name!r} (zigzag or contiguous)")


@dataclass
class MaskArgs:
    causal: bool = False
    sliding_window: int = 0
    alibi_slope: Optional[torch.Tensor] = None
    scale: Optional[float] = None
    soft_cap: float = 0.0


def block_visible(qa: int, kb: int, chunk: int, m: MaskArgs) -> bool:
    """False when the mask hides every (i, j) of query chunk qa x key chunk kb."""
    q_lo, q_hi = qa * chunk, qa * chunk + chunk - 1
    k_lo, k_hi = kb * chunk, kb * chunk + chunk - 1
    if m.causal and k_lo > q_hi:
        return False
    if m.sliding_window > 0 and q_lo - k_hi > m.sliding_window:
        return False
    return True


# ---------------------------------------------------------------- block ops (CUDA)
class CudaBlockOps:
    """One block of the ring on this rank's GPU through libbfa."""

    def fwd(self, q, k, v, q_off, k_off, m: MaskArgs):
        return _nfa.npu_flash_attention_forward(
            q, k, v, causal=m.causal, sliding_window=m.sliding_window,
            alibi_slope=m.alibi_slope, scale=m.scale, soft_cap=m.soft_cap,
            return_lse=True, q_pos_offset=q_off, k_pos_offset=k_off)

    def fwd_merge(self, o_acc, lse_acc, q, k, v, q_off, k_off, m: MaskArgs):
        """One block's forward merged into the fp32 running (o_acc, lse_acc)
        by the forward kernel's epilogue: no partial (O, LSE) is written."""
        _nfa.npu_flash_attention_forward(
            q, k, v, causal=m.causal, sliding_window=m.sliding_window,
            alibi_slope=m.alibi_slope, scale=m.scale, soft_cap=m.soft_cap,
            return_lse=True, q_pos_offset=q_off, k_pos_offset=k_off,
            _merge_into=(o_acc, lse_acc))

    def merge(self, o_acc, lse_acc, o_part, lse_part):
        """In place: (o_acc, lse_acc) <- LSE merge with (o_part, lse_part)."""
        B, H, S, D = o_acc.shape
        lib = _bfa.load()
        lse_p = lse_part.contiguous()
        dev = o_acc.device
        with torch.cuda.device(dev):
            _bfa.check(lib.bfa_merge_partial(
                B, H, S, D, _bfa.tensor(o_acc), _bfa.bfa_dtype(o_acc.dtype),
                ctypes.c_void_p(lse_acc.data_ptr()), _bfa.tensor(o_part),
                _bfa.bfa_dtype(o_part.dtype), ctypes.c_void_p(lse_p.data_ptr()),
                ctypes.c_void_p(_bfa.stream_ptr(dev))))

    def bwd_rows(self, q, k, o, do, lse, q_off, m: MaskArgs):
        """Per-query-chunk state: Δ and the backward's row statistic, computed
        once. The statistic depends on the rows' absolute positions (the
        ALiBi row constant, alibi_ref in the library), so the chunk's
        position offset is passed; it does not depend on the key offset, so
        every key block of the ring can use it."""
        lib = _bfa.load()
        D = q.shape[-1]
        scale = m.scale if m.scale is not None else 1.0 / math.sqrt(D)
        pr = _nfa._problem(q, k, m.causal, m.sliding_window, None, scale, m.soft_cap)
        ws = torch.empty(max(lib.bfa_bwd_workspace_bytes(pr), 1), dtype=torch.uint8,
                         device=q.device)
        # Δ reads only o, dout and lse; the gradient buffers are not touched.
        z = torch.zeros(1, 1, 1, 1, device=q.device, dtype=torch.float32)
        _nfa.npu_flash_attention_backward(
            q, k, k, o, lse, do, causal=m.causal, sliding_window=m.sliding_window,
            alibi_slope=m.alibi_slope, scale=m.scale, soft_cap=m.soft_cap,
            q_pos_offset=q_off, _phases=_bfa.PHASE_DELTA, _workspace=ws, _outputs=(z, z, z))
        return ws

    def bwd_into(self, state, q, k, v, o, lse, do, q_off, k_off, m: MaskArgs,
                 dq_acc, dk_acc, dv_acc):
        """Add this block's dQ, dK, dV to the fp32 accumulators."""
        _nfa.npu_flash_attention_backward(
            q, k, v, o, lse, do, causal=m.causal, sliding_window=m.sliding_window,
            alibi_slope=m.alibi_slope, scale=m.scale, soft_cap=m.soft_cap,
            q_pos_offset=q_off, k_pos_offset=k_off,
            _phases=_bfa.PHASE_DKDV | _bfa.PHASE_DQ, _workspace=state,
            _outputs=(dq_acc, dk_acc, dv_acc), _accumulate=True)


# ---------------------------------------------------------------- ring (per rank)
def ring_forward(q, k, v, rank: int, world: int, m: MaskArgs, ops):
    """Generator for one rank's forward. Yields ("start", kv) to post the send
    of ``kv`` to rank+1 and the receive from rank-1, ("finish",) to complete
    them (sent back: the received K/V). Returns (O, LSE) of this rank's rows.
    """
    S2 = q.shape[2]
    C = S2 // 2
    lay = ZigzagLayout(S2 * world, world)
    my = lay.chunks(rank)
    B, H, _, D = q.shape
    o_acc = [torch.zeros(B, H, C, D, device=q.device, dtype=torch.float32) for _ in range(2)]
    lse_acc = [torch.full((B, H, C), float("-inf"), device=q.device, dtype=torch.float32)
               for _ in range(2)]
    kv = (k, v)
    for t in range(world):
        src = (rank - t) % world
        if t + 1 < world:
            yield ("start", kv)
        kc, vc = kv
        for ia, qa in enumerate(my):
            for ib, kb in enumerate(lay.chunks(src)):
                if not block_visible(qa, kb, C, m):
                    continue
                ops.fwd_merge(o_acc[ia], lse_acc[ia], q.narrow(2, ia * C, C),
                              kc.narrow(2, ib * C, C), vc.narrow(2, ib * C, C), qa * C, kb * C, m)
        if t + 1 < world:
            kv = yield ("finish",)
    return torch.cat(o_acc, dim=2).to(q.dtype), torch.cat(lse_acc, dim=2)


def ring_backward(q, k, v, o, lse, do, rank: int, world: int, m: MaskArgs, ops):
    """Generator for one rank's backward. K/V move as in the forward; the
    fp32 dK/dV accumulators follow with ("swap", (dk, dv)) after every step,
    so after N steps each rank holds the gradients of its own K/V shard.
    Returns (dQ, dK, dV) in the input dtypes.
    """
    S2 = q.shape[2]
    C = S2 // 2
    lay = ZigzagLayout(S2 * world, world)
    my = lay.chunks(rank)
    dq_acc = torch.zeros(q.shape, device=q.device, dtype=torch.float32)
    dkv = (torch.zeros(k.shape, device=k.device, dtype=torch.float32),
           torch.zeros(v.shape, device=v.device, dtype=torch.float32))
    rows = []
    for ia in range(2):
        sl = slice(ia * C, ia * C + C)
        rows.append(ops.bwd_rows(q[:, :, sl], k, o[:, :, sl], do[:, :, sl],
                                 lse[:, :, sl].contiguous(), my[ia] * C, m))
    kv = (k, v)
    for t in range(world):
        src = (rank - t) % world
        if t + 1 < world:
            yield ("start", kv)
        kc, vc = kv
        dk_acc, dv_acc = dkv
        for ia, qa in enumerate(my):
            qs = slice(ia * C, ia * C + C)
            for ib, kb in enumerate(lay.chunks(src)):
                if not block_visible(qa, kb, C, m):
                    continue
                ks = slice(ib * C, ib * C + C)
                ops.bwd_into(rows[ia], q[:, :, qs], kc[:, :, ks], vc[:, :, ks], o[:, :, qs],
                             lse[:, :, qs].contiguous(), do[:, :, qs], qa * C, kb * C, m,
                             dq_acc[:, :, qs], dk_acc[:, :, ks], dv_acc[:, :, ks])
        if t + 1 < world:
            kv = yield ("finish",)
        if world > 1:
            dkv = yield ("swap", dkv)
    dk_acc, dv_acc = dkv
    return dq_acc.to(q.dtype), dk_acc.to(k.dtype), dv_acc.to(v.dtype)


# ---------------------------------------------------------------- failure detection
class PeerFailure(RuntimeError):
    """A rank stopped taking part in the ring or the all-to-alls (it left,
    crashed or hangs in host code) before a communication step."""


class RingWatchdog:
    """Host-side failure detection for the context-parallel drivers; no GPU
    work is involved.

    Before each communication step a rank publishes a heartbeat (its step
    count) in a key-value store the ranks share (the process group's store,
    ``for_group``) and waits, up to ``timeout_s``, until the peers it
    exchanges data with in that step have published the same count. A peer
    that left between steps, crashed or hangs in host code never does. The
    rank that notices writes the reason into the store, so every other rank
    stops at its own next check at once instead of waiting out its timeout;
    it then runs ``abort`` (``for_group``: abort the NCCL communicator, so no
    call of the group stays posted and the process can exit) and raises
    PeerFailure. Nothing is posted after a failed check, so none of this
    rank's transfers is in flight when it raises. A rank that stops on
    purpose calls ``leave()``.

    The ranks must create their watchdogs in the same order (the store keys
    come from a per-process counter) or give them the same ``name``.
    """

    _created = 0

    def __init__(self, store, rank: int, world: int, timeout_s: float = 30.0,
                 poll_s: float = 0.001, name: Optional[str] = None, abort=None):
        if name is None:
            name = str(RingWatchdog._created)
            RingWatchdog._created += 1
        self.store, self.rank, self.world = store, rank, world
        self.prefix = f"bfa_cp_watchdog/{name}"
        self.timeout_s, self.poll_s = float(timeout_s), float(poll_s)
        self.abort = abort
        self.steps = 0
        self.failed: Optional[str] = None

    @classmethod
    def for_group(cls, group=None, timeout_s: float = 30.0, name: Optional[str] = None):
        """A watchdog over the store, ranks and communicator of ``group``."""
        import torch.distributed as dist
        import torch.distributed.distributed_c10d as c10d
        abort = None
        if dist.get_backend(group) == "nccl":
            def abort():
                c10d._abort_process_group(group)  # None: every group of this process
        return cls(c10d._get_default_store(), dist.get_rank(group), dist.get_world_size(group),
                   timeout_s=timeout_s, name=name, abort=abort)

    def _key(self, what: str) -> str:
        return f"{self.prefix}/{what}"

    def _fail(self, reason: str):
        self.failed = reason
        if self.abort is not None:
            try:
                self.abort()
            except Exception:  # the failure below is the one to report
                pass
        raise PeerFailure(reason)

    def _check_failed(self):
        if self.failed is not None:
            raise PeerFailure(self.failed)
        key = self._key("failed")
        if self.store.check([key]):
            self._fail(self.store.get(key).decode())

    def step(self, peers):
        """Publish this rank's next step and wait until every rank in
        ``peers`` (ranks of the group; this rank is ignored) has reached it.
        A store that stops answering (its host process ended) is a failure
        too."""
        import torch.distributed as dist
        try:
            self._step(peers)
        except dist.DistError as e:
            self._fail(f"the ranks' store stopped answering ({e}): the process that holds it ended")

    def _step(self, peers):
        self._check_failed()
        self.steps += 1
        self.store.set(self._key(f"hb/{self.rank}"), str(self.steps))
        waiting = sorted({p % self.world for p in peers} - {self.rank})
        deadline = time.monotonic() + self.timeout_s
        while waiting:
            still = []
            for p in waiting:
                key = self._key(f"hb/{p}")
                if not (self.store.check([key]) and int(self.store.get(key)) >= self.steps):
                    still.append(p)
            waiting = still
            if not waiting:
                break
            self._check_failed()
            if time.monotonic() > deadline:
                reason = (f"rank {waiting[0]} did not reach communication step {self.steps} "
                          f"within {self.timeout_s:g} s (noticed by rank {self.rank})")
                self.store.set(self._key("failed"), reason)
                self._fail(reason)
            time.sleep(self.poll_s)

    def neighbours(self):
        """The ring's peers: the next rank (send) and the previous one (receive)."""
        return (self.rank + 1, self.rank - 1)

    def leave(self, reason: Optional[str] = None):
        """Stop on purpose: the other ranks raise PeerFailure at their next check."""
        reason = reason or f"rank {self.rank} left"
        self.store.set(self._key("failed"), reason)
        self.failed = reason


# ---------------------------------------------------------------- drivers
class DistRing:
    """Ring transfers over torch.distributed point-to-point (NCCL or gloo)."""

    def __init__(self, group=None):
        import torch.distributed as dist
        self.dist, self.group = dist, group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self._pending = None

    def _peer(self, r: int) -> int:
        r %= self.world
        return r if self.group is None else self.dist.get_global_rank(self.group, r)

    def _post(self, payload):
        dist = self.dist
        recv = tuple(torch.empty_like(t) for t in payload)
        ops = []
        for t, rb in zip(payload, recv):
            ops.append(dist.P2POp(dist.isend, t.contiguous(), self._peer(self.rank + 1), self.group))
            ops.append(dist.P2POp(dist.irecv, rb, self._peer(self.rank - 1), self.group))
        reqs = dist.batch_isend_irecv(ops)
        # The send buffers stay referenced until the requests complete.
        return reqs, recv, payload

    def start(self, payload):
        assert self._pending is None, "ring transfer already in flight"
        self._pending = self._post(payload)

    def finish(self):
        reqs, recv, _ = self._pending
        for r in reqs:
            r.wait()
        self._pending = None
        return recv

    def swap(self, payload):
        reqs, recv, _ = self._post(payload)
        for r in reqs:
            r.wait()
        return recv


def run_dist(gen, group=None, watchdog: Optional[RingWatchdog] = None):
    """Drive one rank's ring generator over torch.distributed. With a
    ``watchdog``, each transfer is posted only after both ring neighbours
    have reached the same step (PeerFailure otherwise)."""
    ring = DistRing(group)
    try:
        step = next(gen)
        while True:
            kind = step[0]
            if kind in ("start", "swap") and watchdog is not None:
                watchdog.step(watchdog.neighbours())
            if kind == "start":
                ring.start(step[1])
                step = gen.send(None)
            elif kind == "finish":
                step = gen.send(ring.finish())
            elif kind == "swap":
                step = gen.send(ring.swap(step[1]))
            else:
                raise RuntimeError(f"unknown ring step {kind!r}")
    except StopIteration as stop:
        return stop.value


def run_simulated(gens):
    """Drive all ranks' generators in one process, in lockstep: every rank
    yields the same step kinds in the same order; rank r receives what rank
    r-1 sent."""
    n = len(gens)
    results = [None] * n
    steps = [None] * n
    done = 0
    for r, g in enumerate(gens):
        try:
            steps[r] = next(g)
        except StopIteration as stop:  # a ring of one rank never communicates
            results[r] = stop.value
            done += 1
    if done == n:
        return results
    if done:
        raise RuntimeError("ranks finished at different steps")
    inflight = None
    while True:
        kinds = {s[0] for s in steps}
        if len(kinds) != 1:
            raise RuntimeError(f"ranks out of step: {kinds}")
        kind = kinds.pop()
        if kind == "start":
            inflight = [s[1] for s in steps]
            sends = [None] * n
        elif kind == "finish":
            sends = [inflight[(r - 1) % n] for r in range(n)]
            inflight = None
        elif kind == "swap":
            sends = [steps[(r - 1) % n][1] for r in range(n)]
        else:
            raise RuntimeError(f"unknown ring step {kind!r}")
        done = 0
        for r, g in enumerate(gens):
            try:
                steps[r] = g.send(sends[r])
            except StopIteration as stop:
                results[r] = stop.value
                done += 1
        if done == n:
            return results
        if done:
            raise RuntimeError("ranks finished at different steps")


# ---------------------------------------------------------------- Ulysses
# The alternative to the ring for head-rich configurations: two all-to-alls
# turn sequence shards of every head into the whole sequence of a group of
# heads, the single-GPU operator runs on it unchanged (positions 0..S-1, no
# blockwise merging), and two all-to-alls turn the result back. Rank r takes
# q-heads [r·Hq/N, (r+1)·Hq/N) and kv-heads [r·Hkv/N, (r+1)·Hkv/N): contiguous
# head groups keep every GQA group (hq -> hq / G) on one rank. Needs Hq and
# Hkv divisible by N. Bytes per rank per all-to-all: the rank's shard of the
# tensor, (N-1)/N of it crossing NVLink; forward moves q, k, v and O, backward
# dO, dq, dk, dv.
class CudaAttentionOps:
    """Whole-sequence attention on this rank's GPU through libbfa."""

    def fwd(self, q, k, v, m: MaskArgs):
        return _nfa.npu_flash_attention_forward(
            q, k, v, causal=m.causal, sliding_window=m.sliding_window,
            alibi_slope=m.alibi_slope, scale=m.scale, soft_cap=m.soft_cap, return_lse=True)

    def bwd(self, q, k, v, o, lse, do, m: MaskArgs):
        return _nfa.npu_flash_attention_backward(
            q, k, v, o, lse, do, causal=m.causal, sliding_window=m.sliding_window,
            alibi_slope=m.alibi_slope, scale=m.scale, soft_cap=m.soft_cap)


def _h2s_send(x, world: int):
    """[B, H, S/N, D] (this rank's rows, every head) -> the all-to-all input
    [N, B, H/N, S/N, D]: entry j (head group j) goes to rank j."""
    B, H, Sl, D = x.shape
    return x.reshape(B, world, H // world, Sl, D).transpose(0, 1).contiguous()


def _h2s_finish(recv, layout):
    """All-to-all output (entry i: rank i's rows of this rank's head group)
    -> [B, H/N, S, D], every row in sequence order."""
    return layout.unshard(list(recv.unbind(0)), dim=2).contiguous()


def _s2h_send(x, world: int, layout):
    """[B, H/N, S, D] -> [N, B, H/N, S/N, D]: entry j holds rank j's rows."""
    return torch.stack([layout.shard(x, j, dim=2) for j in range(world)], 0).contiguous()


def _s2h_finish(recv):
    """All-to-all output (entry j: this rank's rows of head group j)
    -> [B, H, S/N, D]."""
    N, B, Hg, Sl, D = recv.shape
    return recv.transpose(0, 1).reshape(B, N * Hg, Sl, D).contiguous()


def heads_to_sequence(x, world: int, layout, a2a):
    """[B, H, S/N, D] (this rank's rows, every head) -> [B, H/N, S, D] (every
    row, this rank's head group). ``a2a`` exchanges dim 0 of an [N, ...]
    tensor: entry j goes to rank j, entry i of the result came from rank i."""
    return _h2s_finish(a2a(_h2s_send(x, world)), layout)


def sequence_to_heads(x, world: int, layout, a2a):
    """Inverse of ``heads_to_sequence``: [B, H/N, S, D] -> [B, H, S/N, D]."""
    return _s2h_finish(a2a(_s2h_send(x, world, layout)))


def _ulysses_check(hq: int, hkv: int, world: int):
    if hq % world or hkv % world:
        raise ValueError(f"Ulysses needs heads_q ({hq}) and heads_kv ({hkv}) divisible by "
                         f"the group size ({world}); use the ring (context_parallel_attention)")


def _local_mask(m: MaskArgs, rank: int, hq: int, world: int) -> MaskArgs:
    """The mask for this rank's q-head group (ALiBi slopes of those heads)."""
    hg = hq // world
    slopes = None if m.alibi_slope is None else m.alibi_slope[rank * hg:(rank + 1) * hg].contiguous()
    return MaskArgs(m.causal, m.sliding_window, slopes, m.scale, m.soft_cap)


def _dist_a2a(group, watchdog: Optional[RingWatchdog] = None):
    import torch.distributed as dist

    def a2a(send):
        if watchdog is not None:
            watchdog.step(range(watchdog.world))
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send, group=group)
        return recv
    return a2a


class UlyssesFlexAttention(torch.autograd.Function):
    """Autograd over Ulysses: inputs and outputs are this rank's sequence shard."""

    @staticmethod
    def forward(ctx, q, k, v, causal, sliding_window, alibi_slope, scale, soft_cap, group, layout, ops,
                watchdog):
        import torch.distributed as dist
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        _ulysses_check(q.shape[1], k.shape[1], world)
        lay = make_layout(layout, q.shape[2] * world, world)
        a2a = _dist_a2a(group, watchdog)
        m = _local_mask(MaskArgs(causal, int(sliding_window), alibi_slope, scale, float(soft_cap)),
                        rank, q.shape[1], world)
        qf, kf, vf = (heads_to_sequence(t.contiguous(), world, lay, a2a) for t in (q, k, v))
        of, lsef = ops.fwd(qf, kf, vf, m)
        ctx.save_for_backward(qf, kf, vf, of, lsef)
        ctx.m, ctx.world, ctx.lay, ctx.a2a, ctx.ops = m, world, lay, a2a, ops
        return sequence_to_heads(of, world, lay, a2a)

    @staticmethod
    def backward(ctx, grad_out):
        qf, kf, vf, of, lsef = ctx.saved_tensors
        world, lay, a2a = ctx.world, ctx.lay, ctx.a2a
        dof = heads_to_sequence(grad_out.to(qf.dtype).contiguous(), world, lay, a2a)
        dqf, dkf, dvf = ctx.ops.bwd(qf, kf, vf, of, lsef, dof, ctx.m)
        grads = [sequence_to_heads(t, world, lay, a2a) for t in (dqf, dkf, dvf)]
        return (*grads, None, None, None, None, None, None, None, None, None)


def ulysses_attention(q, k, v, causal=False, sliding_window=0, alibi_slope=None, scale=None,
                      soft_cap=0.0, group=None, layout="zigzag", _ops=None, watchdog=None):
    """Attention over a sequence sharded across the ranks of ``group`` by
    head-sequence all-to-alls (Ulysses). q [B, Hq, S/N, D], k/v
    [B, Hkv, S/N, D] are this rank's rows in ``layout`` ("zigzag", as for
    context_parallel_attention, or "contiguous"); Hq and Hkv must be divisible
    by N. Returns this rank's rows of O; differentiable. ``alibi_slope`` holds
    all Hq slopes on every rank. With a ``watchdog`` (RingWatchdog) every
    all-to-all waits for all ranks on the host first and raises PeerFailure
    when one has stopped."""
    return UlyssesFlexAttention.apply(q, k, v, causal, sliding_window, alibi_slope, scale, soft_cap,
                                      group, layout, _ops or CudaAttentionOps(), watchdog)


def ulysses_simulated(qs, ks, vs, dos, m: MaskArgs, ops, layout="zigzag"):
    """Ulysses forward and backward for N simulated ranks in one process
    (shards as lists, one entry per rank); the all-to-alls are in-memory.
    Returns (o shards, dq shards, dk shards, dv shards)."""
    world = len(qs)
    _ulysses_check(qs[0].shape[1], ks[0].shape[1], world)
    lay = make_layout(layout, qs[0].shape[2] * world, world)

    def a2a_all(sends):  # recv_r[i] = send_i[r]
        return [torch.stack([sends[i][r] for i in range(world)], 0) for r in range(world)]

    def h2s(xs):
        return [_h2s_finish(rv, lay) for rv in a2a_all([_h2s_send(x, world) for x in xs])]

    def s2h(xs):
        return [_s2h_finish(rv) for rv in a2a_all([_s2h_send(x, world, lay) for x in xs])]

    qf, kf, vf, dof = (h2s(xs) for xs in (qs, ks, vs, dos))
    masks = [_local_mask(m, r, qs[0].shape[1], world) for r in range(world)]
    fw = [ops.fwd(qf[r], kf[r], vf[r], masks[r]) for r in range(world)]
    o = s2h([f[0] for f in fw])
    bw = [ops.bwd(qf[r], kf[r], vf[r], fw[r][0], fw[r][1], dof[r], masks[r]) for r in range(world)]
    dq, dk, dv = (s2h([b[i] for b in bw]) for i in range(3))
    return o, dq, dk, dv


# ---------------------------------------------------------------- public API
class RingFlexAttention(torch.autograd.Function):
    """Autograd over the ring: inputs and outputs are this rank's zigzag shard."""

    @staticmethod
    def forward(ctx, q, k, v, causal, sliding_window, alibi_slope, scale, soft_cap, group, watchdog):
        import torch.distributed as dist
        m = MaskArgs(causal, int(sliding_window), alibi_slope, scale, float(soft_cap))
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        o, lse = run_dist(ring_forward(q, k, v, rank, world, m, CudaBlockOps()), group, watchdog)
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.m, ctx.group, ctx.rank, ctx.world, ctx.watchdog = m, group, rank, world, watchdog
        return o

    @staticmethod
    def backward(ctx, grad_out):
        q, k, v, o, lse = ctx.saved_tensors
        do = grad_out.to(q.dtype).contiguous()
        dq, dk, dv = run_dist(ring_backward(q, k, v, o, lse, do, ctx.rank, ctx.world, ctx.m,
                                            CudaBlockOps()), ctx.group, ctx.watchdog)
        return dq, dk, dv, None, None, None, None, None, None, None


def context_parallel_attention(q, k, v, causal=False, sliding_window=0, alibi_slope=None,
                               scale=None, soft_cap=0.0, group=None, watchdog=None):
    """Attention over a sequence sharded across the ranks of ``group`` in the
    zigzag layout (``ZigzagLayout.shard``): q [B, Hq, 2C, D], k/v [B, Hkv, 2C, D]
    on this rank's GPU. Returns this rank's rows of O; differentiable. With a
    ``watchdog`` (RingWatchdog) each K/V transfer waits for both ring
    neighbours on the host first and raises PeerFailure when one has stopped."""
    return RingFlexAttention.apply(q, k, v, causal, sliding_window, alibi_slope, scale,
                                   soft_cap, group, watchdog)
