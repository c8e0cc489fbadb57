"""Host-side failure handling of the sharded decode step.

The reference runs on one GPU and handles no faults (engine/engine.py:34; the fallback at
engine.py:494-498 is for speed). Sharded over G ranks, the decode step exchanges each layer's head
outputs either inside the attention kernel over NVLink (gather.py: the kernel's wait for the
peers' flags is bounded and ends with KOPT_DEV_ERR_TIMEOUT in its error word) or by an all-gather
of the process group (shard.gather_heads: NCCL between GPUs, gloo on CPU). This module bounds
what the host waits for:

* ``init_group`` opens the process group with a short timeout on every collective (torch's
  default, ten minutes, would hold a rank that long after a peer has gone);
* ``collective`` runs one collective; on any error it aborts the group's communicators
  (``ProcessGroup.abort``: ``ncclCommAbort`` on each NCCL communicator of the group), records the
  failure for the peers when a ``PeerWatch`` is given, and raises ``CollectiveError``, so that no
  rank waits again on a communicator that has failed;
* ``PeerWatch`` keeps a failure record and one heartbeat per rank in the group's key-value store.
  A rank that fails on the host between steps (an exception, a device error word) records its
  rank and reason with ``fail``; every rank calls ``check`` before its next launch, which raises
  ``PeerFailure`` when a record exists or a peer's heartbeat is older than the limit, instead of
  entering a collective that the peer will never join.

A rank leaves only between steps, with none of its kernels or collectives in flight; the peers
learn of it on the host before their next launch, or the group's timeout ends their next
collective with an error.
"""

from __future__ import annotations

import datetime
import time

import torch
import torch.distributed as dist

DEFAULT_TIMEOUT_S = 30.0       # every collective of the group
DEFAULT_STALE_S = 10.0         # a peer whose heartbeat is older than this is taken as gone
_FAILED = "kopt/failed"
_BEAT = "kopt/beat/"


class CollectiveError(RuntimeError):
    """A collective of the sharded step failed or timed out; the group has been aborted."""


class PeerFailure(RuntimeError):
    """A peer recorded a failure, or stopped beating, before this rank's next launch."""

    def __init__(self, rank: int, reason: str):
        super().__init__(f"rank {rank}: {reason}")
        self.rank = rank
        self.reason = reason


def init_group(backend: str = "nccl", timeout_s: float = DEFAULT_TIMEOUT_S, device=None, **kw):
    """``dist.init_process_group`` with a timeout of ``timeout_s`` seconds on every collective
    (and on the rendezvous). ``device`` binds an NCCL group to this rank's GPU."""
    if device is not None and backend == "nccl":
        kw.setdefault("device_id", torch.device(device))
    dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s), **kw)
    return dist.group.WORLD


def _pg(group):
    return group if group is not None else dist.group.WORLD


def abort_group(group=None) -> None:
    """Abort the group's communicators (NCCL: ``ncclCommAbort``); pending and later collectives
    on it end with an error instead of waiting. The group is unusable afterwards."""
    pg = _pg(group)
    try:
        pg.abort()
    except (RuntimeError, NotImplementedError):
        pass   # a backend without abort (gloo): its collectives still end at the timeout


def collective(fn, *args, group=None, watch: "PeerWatch | None" = None, what: str = "collective",
               **kw):
    """Run ``fn(*args, group=group, **kw)`` (a torch.distributed collective or a function that
    issues one); on an error or timeout abort the group, record the failure in ``watch`` and
    raise ``CollectiveError``."""
    try:
        return fn(*args, group=group, **kw)
    except Exception as e:   # DistBackendError, DistNetworkError, timeouts: all RuntimeError
        reason = f"{what} failed: {type(e).__name__}: {str(e).splitlines()[0] if str(e) else ''}"
        if watch is not None:
            watch.fail(reason)
        abort_group(group)
        raise CollectiveError(reason) from e


class PeerWatch:
    """Failure record and heartbeats of the group's ranks in its key-value store.

    ``beat`` stamps this rank's heartbeat (wall-clock seconds); ``fail`` records this rank's
    failure; ``check`` raises ``PeerFailure`` when any rank recorded one or, at most every
    ``period_s`` seconds, when a peer's heartbeat is older than ``stale_s`` (a peer that stamped
    none yet is not judged; ``stale_s=None`` judges none: for ranks that may legitimately sit
    idle between their checks for longer than any fixed limit). One store round trip per
    ``check`` in between.
    """

    def __init__(self, group=None, stale_s: float | None = DEFAULT_STALE_S, period_s: float = 0.5,
                 store=None, rank: int | None = None, world: int | None = None):
        pg = _pg(group)
        self.store = store if store is not None else pg.get_group_store()
        self.rank = dist.get_rank(group) if rank is None else rank
        self.world = dist.get_world_size(group) if world is None else world
        self.stale_s, self.period_s = stale_s, period_s
        self._next_scan = 0.0
        self.beat()

    def beat(self) -> None:
        self.store.set(_BEAT + str(self.rank), repr(time.time()))

    def fail(self, reason: str) -> None:
        """Record this rank's failure (the first record stands). Store errors are ignored: a
        store that is gone means the peers find out by their own timeouts."""
        try:
            self.store.compare_set(_FAILED, "", f"{self.rank}:{reason}")
        except Exception:
            pass

    def failed(self) -> tuple[int, str] | None:
        """(rank, reason) of the recorded failure, or None."""
        if not self.store.check([_FAILED]):
            return None
        r, _, why = self.store.get(_FAILED).decode().partition(":")
        return int(r), why

    def check(self) -> None:
        """Raise ``PeerFailure`` if a rank recorded a failure or a peer went silent; otherwise
        stamp this rank's heartbeat (when heartbeats are judged). A store that cannot be reached
        counts as a failure of the rank that hosts it (rank 0)."""
        try:
            rec = self.failed()
            if rec is not None:
                raise PeerFailure(*rec)
            now = time.time()
            if self.stale_s is not None and now >= self._next_scan and self.world > 1:
                self._next_scan = now + self.period_s
                peers = [w for w in range(self.world) if w != self.rank]
                keys = [_BEAT + str(w) for w in peers]
                have = [w for w, k in zip(peers, keys) if self.store.check([k])]
                if have:
                    stamps = self.store.multi_get([_BEAT + str(w) for w in have])
                    for w, t in zip(have, stamps):
                        age = now - float(t.decode())
                        if age > self.stale_s:
                            raise PeerFailure(w, f"no heartbeat for {age:.1f} s")
            if self.stale_s is not None:
                self.beat()
        except PeerFailure:
            raise
        except Exception as e:
            raise PeerFailure(0, f"key-value store unreachable: {type(e).__name__}") from e
