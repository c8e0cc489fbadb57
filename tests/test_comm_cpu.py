"""CPU: failure handling of the sharded step's process group (kernel_optim_b200/comm.py).

Failures are made on the host: a rank that never joins a collective, one that raises between
steps, one that stops beating, one that exits. Ranks are gloo processes on the CPU; each
collective is bounded by the group's timeout, so nothing here can wait for long.
"""

import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from kernel_optim_b200 import _lib
from kernel_optim_b200.comm import CollectiveError, PeerFailure, PeerWatch, init_group
from kernel_optim_b200.shard import gather_heads

TIMEOUT_S = 3.0


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _step(rank, world, watch):
    local = torch.full((2, 8), float(rank))
    out = gather_heads(local, torch.empty(world, 2, 8), watch=watch)
    assert torch.equal(out[:, 8:], torch.ones(2, 8))


def _worker(case, rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    init_group("gloo", timeout_s=TIMEOUT_S, rank=rank, world_size=world)
    watch = PeerWatch(stale_s=2.0, period_s=0.0)
    res = None
    try:
        watch.check()
        _step(rank, world, watch)          # step 1: both ranks
        if case == "no_join":
            if rank == 0:
                t0 = time.monotonic()
                try:
                    _step(rank, world, watch)
                except CollectiveError as e:
                    res = ("CollectiveError", time.monotonic() - t0, str(e), watch.failed())
            else:   # never joins step 2; waits (bounded) for rank 0's record
                t_end = time.monotonic() + 30
                while watch.failed() is None and time.monotonic() < t_end:
                    time.sleep(0.05)
                res = ("record", watch.failed())
        elif case == "raise":
            if rank == 1:
                try:
                    raise ValueError("bad block table")
                except ValueError as e:
                    watch.fail(f"{type(e).__name__}: {e}")
                res = ("failed", None)
            else:
                time.sleep(1.0)            # this rank's step 2 on the GPU, in the real engine
                try:
                    watch.check()
                    res = ("passed", None)
                except PeerFailure as e:
                    res = ("PeerFailure", e.rank, e.reason)
        elif case == "silent":
            if rank == 1:                  # alive, beating no more, never fails
                time.sleep(4.0)
                res = ("slept", None)
            else:
                t0 = time.monotonic()
                try:
                    while time.monotonic() - t0 < 20:
                        watch.check()
                        time.sleep(0.1)
                    res = ("passed", None)
                except PeerFailure as e:
                    res = ("PeerFailure", e.rank, e.reason, time.monotonic() - t0)
        elif case == "exit":
            if rank == 1:
                q.put((rank, ("exiting", None)))
                q.close()
                q.join_thread()            # the message is out before the process ends
                os._exit(0)
            t0 = time.monotonic()
            time.sleep(0.5)
            try:
                _step(rank, world, watch)
                res = ("passed", None)
            except (CollectiveError, PeerFailure) as e:
                res = (type(e).__name__, time.monotonic() - t0)
        q.put((rank, res))
    except BaseException as e:   # surfaced by the parent
        q.put((rank, ("unexpected", repr(e))))


def _run(case, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(case, r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        res = dict(q.get(timeout=120) for _ in range(world))
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
                p.join()
    for r, v in res.items():
        assert v[0] != "unexpected", f"rank {r}: {v[1]}"
    return res


def test_collective_that_a_peer_never_joins_ends_at_the_timeout_and_aborts():
    res = _run("no_join")
    kind, elapsed, msg, rec = res[0]
    assert kind == "CollectiveError"
    assert elapsed < TIMEOUT_S + 10, f"{elapsed:.1f} s"
    assert "all-gather of the head outputs" in msg
    assert rec is not None and rec[0] == 0              # the failing rank recorded itself
    assert res[1][0] == "record" and res[1][1] is not None and res[1][1][0] == 0


def test_failure_recorded_between_steps_is_seen_before_the_next_launch():
    res = _run("raise")
    assert res[1][0] == "failed"
    assert res[0][0] == "PeerFailure", res[0]
    assert res[0][1] == 1 and "bad block table" in res[0][2]


def test_silent_peer_is_taken_as_gone_after_its_heartbeat_goes_stale():
    res = _run("silent")
    assert res[0][0] == "PeerFailure", res[0]
    assert res[0][1] == 1 and "no heartbeat" in res[0][2]
    assert res[0][3] < 10.0


def test_peer_that_exits_ends_the_next_collective_with_an_error():
    res = _run("exit")
    assert res[1][0] == "exiting"
    assert res[0][0] in ("CollectiveError", "PeerFailure"), res[0]
    assert res[0][1] < TIMEOUT_S + 10


# ------------------------------------------------------------- Engine.generate's host checks
class _FakeAttn:
    def __init__(self, bits):
        self.bits = bits

    def read_error(self):
        b, self.bits = self.bits, 0
        return b


def _engine(watch, steps, bits=0, fail_at=None):
    """An Engine with only what generate touches: _generate yields `steps` lists, raising at
    step `fail_at`; the attention's error word holds `bits`."""
    from kernel_optim_b200.engine import Engine
    eng = Engine.__new__(Engine)
    eng.watch, eng.rank, eng.attn = watch, watch.rank, _FakeAttn(bits)

    def gen(ids, n):
        for j in range(n):
            if j == fail_at:
                raise RuntimeError("CUDA error: an example failure")
            watch.check()
            yield [j]
    eng._generate = gen
    return eng


def _watch(rank=0):
    store = dist.HashStore()
    return PeerWatch(store=store, rank=rank, world=2, period_s=0.0), store


def test_engine_generate_records_its_own_failure():
    watch, store = _watch()
    with pytest.raises(RuntimeError, match="an example failure"):
        list(_engine(watch, 4, fail_at=2).generate([[1]], 4))
    rank, why = watch.failed()
    assert rank == 0 and "an example failure" in why


def test_engine_generate_raises_on_a_device_timeout_and_records_it():
    watch, store = _watch()
    with pytest.raises(_lib.KoptError, match="device error bits 4"):
        list(_engine(watch, 3, bits=_lib.DEV_ERR_TIMEOUT).generate([[1]], 3))
    assert watch.failed()[0] == 0


def test_engine_generate_stops_before_its_first_step_on_a_peer_record():
    watch, store = _watch()
    peer = PeerWatch(store=store, rank=1, world=2)
    peer.fail("ValueError: out of pages")
    got = []
    with pytest.raises(PeerFailure, match="out of pages"):
        for ids in _engine(watch, 3).generate([[1]], 3):
            got.append(ids)
    assert got == []
    assert watch.failed() == (1, "ValueError: out of pages")   # the peer's record stands


def test_first_failure_record_stands():
    watch, store = _watch()
    PeerWatch(store=store, rank=1, world=2).fail("first")
    watch.fail("second")
    assert watch.failed() == (1, "first")
