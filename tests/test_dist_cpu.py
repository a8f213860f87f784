"""Host side of the neuron-sharded network on CPU: the NCCL unique id reaches
every rank over a gloo process group (world size 2), and a global batch
splits into the per-rank batches of the sharded train step."""

import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from klearu_b200 import synthetic as S


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from klearu_b200.dist import share_unique_id

        out.put((rank, share_unique_id(rank, world)))
    finally:
        dist.destroy_process_group()


def test_unique_id_reaches_every_rank():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    got = dict(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(60)
        assert p.exitcode == 0
    from klearu_b200 import _lib

    n = _lib.load().kl_dist_unique_id_size()
    assert len(got[0]) == n and got[0] == got[1]


def test_rank_slices_concatenate_to_the_global_batch():
    from klearu_b200.dist import rank_slice

    hb = S.XcGenerator(500, 900, seed=5, mean_nnz=9).batch(12)
    parts = [rank_slice(hb, r, 3) for r in range(3)]
    assert all(p.batch == 4 for p in parts)
    idx = np.concatenate([p.idx for p in parts])
    labels = np.concatenate([p.labels for p in parts])
    assert (idx == hb.idx).all() and (labels == hb.labels).all()
    for r, p in enumerate(parts):
        assert p.rowptr[0] == 0 and p.label_ptr[0] == 0
        assert (np.diff(p.rowptr) == np.diff(hb.rowptr)[4 * r:4 * r + 4]).all()
    with pytest.raises(ValueError):
        rank_slice(hb, 0, 5)
