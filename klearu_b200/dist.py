"""Process-group helpers for neuron-sharded networks (one process per GPU).

The NCCL communicator of a sharded network is created by the C library
(kl_net_create_sharded) from a unique id that rank 0 generates.  These helpers
carry that id to every rank over an already initialised torch.distributed
group (NCCL on the GPU box, gloo on CPU) and split a global batch into the
per-rank batches that kl_net_train_step expects.
"""

from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib
from .data import HostBatch


def share_unique_id(rank: int, world: int, group=None) -> bytes:
    """Rank 0's kl_dist_get_unique_id bytes, on every rank of the group."""
    import torch.distributed as dist

    lib = _lib.load()
    n = lib.kl_dist_unique_id_size()
    payload = [None]
    if rank == 0:
        buf = C.create_string_buffer(n)
        _lib.check(lib.kl_dist_get_unique_id(buf), None, "kl_dist_get_unique_id")
        payload = [bytes(buf.raw)]
    if world > 1:
        dist.broadcast_object_list(payload, src=0, group=group)
    uid = payload[0]
    if not isinstance(uid, bytes) or len(uid) != n:
        raise RuntimeError("NCCL unique id was not received")
    return uid


def rank_slice(hb: HostBatch, rank: int, world: int) -> HostBatch:
    """Examples [rank*B, (rank+1)*B) of a global batch of world*B examples:
    the batch rank `rank` passes to a sharded network's train step."""
    if hb.batch % world:
        raise ValueError("global batch must split evenly over the ranks")
    B = hb.batch // world
    s0, s1 = rank * B, (rank + 1) * B
    a, b = int(hb.rowptr[s0]), int(hb.rowptr[s1])
    c, d = int(hb.label_ptr[s0]), int(hb.label_ptr[s1])
    return HostBatch((np.asarray(hb.rowptr[s0:s1 + 1]) - a).astype(np.int32), np.asarray(hb.idx[a:b]),
                     np.asarray(hb.val[a:b]), (np.asarray(hb.label_ptr[s0:s1 + 1]) - c).astype(np.int32),
                     np.asarray(hb.labels[c:d]))


class RankFailure(RuntimeError):
    """A rank of a sharded network left or stopped making progress.

    ``ranks`` are the missing ranks and ``reason`` is "left" (the rank
    announced that it left) or "silent" (no heartbeat within the timeout)."""

    def __init__(self, ranks: list[int], reason: str, step: int):
        self.ranks, self.reason, self.step = ranks, reason, step
        super().__init__(f"rank(s) {ranks} {reason} before step {step}")


class Heartbeat:
    """Host-side liveness of the ranks of a sharded network.

    A sharded step's collectives finish only when every rank joins them, so a
    rank that stops between steps must be noticed before the survivors launch
    the next step.  Each rank counts its finished steps in the process group's
    key-value store (``dist.distributed_c10d._get_default_store()``, a
    TCPStore, or any ``torch.distributed.Store``):

    * ``beat()`` after a step's host call returned;
    * ``check(step)`` before launching ``step`` (0-based): every peer must have
      finished ``step`` steps.  It waits up to ``timeout_s`` and raises
      ``RankFailure`` naming the ranks that announced ``leave()`` or stayed
      silent.  A rank that fails the check should call
      ``Network.comm_abort()`` (nothing is in flight then) and stop;
    * ``leave()`` when a rank stops between steps on purpose: call it before
      the ``beat()`` of its last step, so that no peer launches another one.

    Each call is one or two store round trips (plus the waiting), so on
    sub-millisecond steps ``every`` > 1 checks only every ``every``-th step;
    the collectives of the steps between stay bounded by
    ``Network.set_comm_timeout``.
    """

    def __init__(self, store, rank: int, world: int, timeout_s: float = 30.0, prefix: str = "kl_hb",
                 every: int = 1):
        self.store, self.rank, self.world = store, rank, world
        self.timeout_s, self.every = float(timeout_s), max(1, int(every))
        self.p = prefix
        self.done = 0

    def _count(self, key: str) -> int:
        return int(self.store.add(f"{self.p}/{key}", 0))  # reads without blocking (creates at 0)

    def beat(self) -> None:
        self.done += 1
        self.store.add(f"{self.p}/beat/{self.rank}", 1)
        self.store.add(f"{self.p}/total", 1)

    def leave(self) -> None:
        self.store.add(f"{self.p}/left/{self.rank}", 1)
        self.store.add(f"{self.p}/left", 1)

    def _missing(self, step: int) -> tuple[list[int], str]:
        peers = [r for r in range(self.world) if r != self.rank]
        left = [r for r in peers if self._count(f"left/{r}")]
        if left:
            return left, "left"
        return [r for r in peers if self._count(f"beat/{r}") < step], "silent"

    def check(self, step: int) -> None:
        import time

        if self.world <= 1 or step % self.every:
            return
        deadline = time.monotonic() + self.timeout_s
        nap = 1e-4
        while True:
            # total before left: leave() comes before the leaving rank's last
            # beat(), so a total that counts that beat is read with the flag set
            total = self._count("total")
            if self._count("left"):
                ranks, why = self._missing(step)
                raise RankFailure(ranks, why, step)
            if total >= self.world * step:
                return
            if time.monotonic() >= deadline:
                ranks, why = self._missing(step)
                raise RankFailure(ranks, why, step)
            time.sleep(nap)
            nap = min(nap * 2, 0.01)
