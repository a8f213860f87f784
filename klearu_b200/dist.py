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
