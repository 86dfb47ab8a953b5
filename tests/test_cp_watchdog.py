"""Failure detection of the context-parallel drivers (CPU, no GPU involved).

RingWatchdog is a host-side heartbeat in the ranks' shared key-value store:
before each transfer a rank waits, with a short bound, until its peers reached
the same step. A rank that leaves between steps (here: its process ends
without a word, or it calls ``leave()``) makes the others raise PeerFailure
at their next step, well before the process group's own timeout, and with
none of their transfers posted. Threads over an in-memory store test the
protocol; gloo ranks in separate processes test it through the ring and the
all-to-all drivers.
"""
import os
import threading
import time
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import context_parallel as cp
from test_context_parallel import OracleBlockOps, _data, _free_port


def _pair(timeout_s=0.5, name="t"):
    store = dist.HashStore()
    return [cp.RingWatchdog(store, r, 2, timeout_s=timeout_s, name=name) for r in range(2)]


def test_steps_in_lockstep_pass():
    wds = _pair()
    errors = []

    def run(wd):
        try:
            for _ in range(5):
                wd.step(wd.neighbours())
        except Exception as e:  # collected, asserted below
            errors.append(e)

    ts = [threading.Thread(target=run, args=(w,)) for w in wds]
    for t in ts:
        t.start()
    for t in ts:
        t.join(timeout=30)
    assert not errors and all(w.steps == 5 for w in wds)


def test_missing_peer_times_out_and_the_others_stop_at_once():
    wds = _pair(timeout_s=0.3)
    aborted = []
    wds[0].abort = lambda: aborted.append(True)
    t0 = time.monotonic()
    with pytest.raises(cp.PeerFailure, match="rank 1 did not reach communication step 1"):
        wds[0].step(wds[0].neighbours())
    assert 0.25 < time.monotonic() - t0 < 5.0
    assert aborted == [True]
    # Rank 1 arrives late: the failure is already in the store, no wait.
    t0 = time.monotonic()
    with pytest.raises(cp.PeerFailure, match="noticed by rank 0"):
        wds[1].step(wds[1].neighbours())
    assert time.monotonic() - t0 < 0.25
    with pytest.raises(cp.PeerFailure):  # and the failed watchdog stays failed
        wds[0].step(wds[0].neighbours())


def test_leave_is_seen_at_the_next_step():
    wds = _pair(timeout_s=30.0)
    wds[1].leave()
    t0 = time.monotonic()
    with pytest.raises(cp.PeerFailure, match="rank 1 left"):
        wds[0].step(wds[0].neighbours())
    assert time.monotonic() - t0 < 1.0


class _DeadStore:
    """A store whose host has gone: every call fails as TCPStore's do."""

    def set(self, *a):
        raise dist.DistNetworkError("Connection reset by peer")

    check = get = set


def test_unreachable_store_is_a_peer_failure():
    wd = cp.RingWatchdog(_DeadStore(), 0, 2, timeout_s=5.0, name="dead")
    with pytest.raises(cp.PeerFailure, match="store stopped answering"):
        wd.step(wd.neighbours())


def test_separate_watchdogs_do_not_share_steps():
    store = dist.HashStore()
    a = [cp.RingWatchdog(store, r, 2, timeout_s=0.2, name="a") for r in range(2)]
    b0 = cp.RingWatchdog(store, 0, 2, timeout_s=0.2, name="b")
    t = threading.Thread(target=a[1].step, args=([0],))
    t.start()
    a[0].step([1])
    t.join(timeout=30)
    assert a[0].steps == a[1].steps == 1
    with pytest.raises(cp.PeerFailure):  # rank 1 reached step 1 of "a" only
        b0.step([1])


def _rank(rank, world, port, mode, out_q, release):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    wd = cp.RingWatchdog.for_group(timeout_s=2.0)
    s = 48 if world == 3 else 64
    q, k, v, _ = _data(5, s)
    lay = cp.ZigzagLayout(s, world)
    sh = [lay.shard(t, rank) for t in (q, k, v)]
    m = cp.MaskArgs(causal=True)

    def one_step():
        if mode.startswith("ring"):
            cp.run_dist(cp.ring_forward(sh[0], sh[1], sh[2], rank, world, m, OracleBlockOps()),
                        watchdog=wd)
        else:
            cp._dist_a2a(None, wd)(torch.arange(4 * world, dtype=torch.float32).view(world, 4))

    one_step()  # every rank takes part in the first step
    if rank == world - 1:
        if mode.endswith("leave"):
            wd.leave()
        out_q.put((rank, "left"))
        out_q.close()
        out_q.join_thread()
        os._exit(0)  # leaves between steps: nothing in flight, no teardown
    t0 = time.monotonic()
    try:
        one_step()
        res = "no failure"
    except cp.PeerFailure as e:
        res = ("failure", time.monotonic() - t0, str(e))
    except Exception as e:  # reported, never hangs the parent
        res = repr(e)
    out_q.put((rank, res))
    out_q.close()
    out_q.join_thread()
    release.wait(120)  # rank 0 holds the store: it stays until every rank reported
    os._exit(0)


@pytest.mark.parametrize("world,mode", [(3, "ring"), (2, "ring_leave"), (3, "a2a"), (2, "a2a_leave")])
def test_rank_that_leaves_between_steps_stops_the_others(world, mode):
    ctx = mp.get_context("spawn")
    out_q, release = ctx.Queue(), ctx.Event()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, mode, out_q, release))
             for r in range(world)]
    for p in procs:
        p.start()
    try:
        results = dict(out_q.get(timeout=180) for _ in range(world))
    finally:
        release.set()
    for p in procs:
        p.join(timeout=60)
    assert results.pop(world - 1) == "left"
    bound = 1.0 if mode.endswith("leave") else 2.0 + 3.0
    for r, res in results.items():
        assert isinstance(res, tuple) and res[0] == "failure", (r, res)
        assert res[1] < bound, (r, res)  # far below the group's 60 s timeout
