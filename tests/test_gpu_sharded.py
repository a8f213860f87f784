"""Neuron-sharded network on 2 GPUs (one process each) vs the CPU oracle's
2-shard network trained on the same global batch.

Bar: the per-step loss within 1e-4 relative on every rank; the replicated
hidden layer and each rank's slice of the output layer within the network
tests' tolerance (1e-3 relative, 1e-6 absolute; one bf16 ulp for weights).
Needs two GPUs: skipped on a one-GPU box.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-3, 1e-6


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cfg():
    from klearu_b200 import synthetic as S
    from klearu_b200.config import LshConfig

    # output TopK = n_out / 10 = 500 >= num_tables * bucket_capacity = 320: every candidate is selected
    return S.config_xc(d_in=2000, hidden=64, n_out=5000, out_l=10, cap=32,
                       hidden_lsh=LshConfig(num_tables=10, num_hashes=6), rebuild_base=2, rebuild_decay=0.1)


def _cfg_fallback():
    """Output SimHash K=12 over one table: 4096 buckets for 5000 neurons, so
    some examples find their bucket empty on every shard and take the global
    all-neurons fallback while the others select candidates."""
    from klearu_b200 import synthetic as S
    from klearu_b200.config import HashFunctionType, LshConfig

    return S.config_xc(d_in=2000, hidden=64, n_out=5000, out_hash=HashFunctionType.SimHash, out_k=12, out_l=1,
                       cap=32, hidden_lsh=LshConfig(num_tables=10, num_hashes=6), rebuild_base=2,
                       rebuild_decay=0.1)


def _cfg_select(sampling):
    """Output selection below the candidate count: TopK of 40 out of up to
    10 x 32 candidates, or Threshold 3 of 10 tables (with its single-best
    fallback), both decided over all shards."""
    from klearu_b200 import synthetic as S
    from klearu_b200.config import LshConfig, SamplingType

    cfg = S.config_xc(d_in=2000, hidden=64, n_out=5000, out_l=10, cap=32,
                      hidden_lsh=LshConfig(num_tables=10, num_hashes=6), rebuild_base=2, rebuild_decay=0.1,
                      out_topk=40)
    o = cfg.network.layers[1]
    if sampling == "threshold":
        o.sampling = SamplingType.Threshold
        o.sampling_threshold = 3
    return cfg


def _close(a, b, bf16_weights=False):
    if bf16_weights:
        return not (np.abs(a - b) > np.maximum(np.abs(a), np.abs(b)) * 2.0 ** -7 + ATOL).any()
    return not (np.abs(a - b) > RTOL * np.abs(b) + ATOL).any()


def _worker(rank, world, port, dtype, out, variant="all"):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        _run(rank, world, dtype, out, variant)
    except Exception:  # report instead of leaving the parent waiting
        import traceback

        out.put([f"rank {rank}: " + traceback.format_exc()])
        raise
    finally:
        dist.destroy_process_group()


def _run(rank, world, dtype, out, variant="all"):
    import torch.distributed as dist

    from klearu_b200 import synthetic as S
    from klearu_b200.core import Context, Network
    from klearu_b200.dist import rank_slice, share_unique_id

    cfg = {"all": _cfg, "fallback": _cfg_fallback}.get(variant, lambda: _cfg_select(variant))()
    init = S.make_init(cfg, 42)
    uid = share_unique_id(rank, world)
    net = Network(cfg, init, weight_dtype=dtype, max_batch=24, ctx=Context(rank), shard=(uid, rank, world))
    gen = S.XcGenerator(2000, 5000, seed=3, mean_nnz=20)
    batches = [gen.batch(24 * world) for _ in range(4)]
    losses = [net.train_step_host(rank_slice(hb, rank, world), 1e-3) for hb in batches]
    r, n, base, nloc = net.shard_info()
    # predict_top_k of this rank's examples of a fresh batch, over all shards
    phb = gen.batch(24 * world)
    top = net.predict_top_k_batch(_examples(rank_slice(phb, rank, world)), 10)
    res = {"losses": losses, "hidden": net.get_layer(0), "out": net.get_layer(1), "base": base, "n": nloc,
           "step": net.step, "feat": net.owned_features(), "top": top}
    gathered = [None] * world
    dist.all_gather_object(gathered, res)
    if rank == 0:
        import oracle

        o = oracle.Net(cfg, init, weight_dtype=dtype, nshards=world)
        msgs = []
        if variant == "fallback":  # the first batch must mix fallback and selecting examples
            hb = batches[0]
            n_fb = sum(len(o.forward(hb.idx[hb.rowptr[s]:hb.rowptr[s + 1]], hb.val[hb.rowptr[s]:hb.rowptr[s + 1]])[1][0])
                       == cfg.network.layers[1].num_neurons for s in range(hb.batch))
            if not 0 < n_fb < hb.batch:
                msgs.append(f"{n_fb} of {hb.batch} examples take the fallback: the case is not exercised")
        ol = [o.train_step(hb, 1e-3, mode="batched") for hb in batches]
        for rr, g in enumerate(gathered):  # predict_top_k after the steps (net.rs:159-173)
            ids, sc = g["top"]
            for i in range(24):
                s = rr * 24 + i
                a, b = int(phb.rowptr[s]), int(phb.rowptr[s + 1])
                oi, _, oa = o.forward(phb.idx[a:b], phb.val[a:b])[-1]
                dense = np.zeros(cfg.network.layers[1].num_neurons, np.float32)
                dense[oi] = oa
                order = sorted(range(dense.size), key=lambda j: (-dense[j], j))[:10]
                if [int(j) for j in ids[i]] != order or not np.allclose(sc[i], dense[order], rtol=1e-5):
                    msgs.append(f"rank {rr} example {i}: predict_top_k differs")
        oh, oo = o.get_layer(0), o.get_layer(1)
        for rr, g in enumerate(gathered):
            if g["step"] != 4:
                msgs.append(f"rank {rr}: step {g['step']}")
            for i, (a, b) in enumerate(zip(g["losses"], ol)):
                if abs(a - b) > 1e-4 * abs(b) + 1e-6:
                    msgs.append(f"rank {rr} step {i}: loss {a} vs oracle {b}")
            lo, hi = g["base"], g["base"] + g["n"]
            f0, nf = g["feat"]
            for k in ("weights", "bias", "m", "v", "mb", "vb"):
                a, b = g["hidden"][k], oh[k]
                if k in ("m", "v"):  # the Adam moments of this rank's feature rows
                    a, b = a[:, f0:f0 + nf], b[:, f0:f0 + nf]
                if not _close(a, b, dtype == "bf16" and k == "weights"):
                    msgs.append(f"rank {rr}: hidden {k} differs")
                if not _close(g["out"][k], oo[k][lo:hi], dtype == "bf16" and k == "weights"):
                    msgs.append(f"rank {rr}: output {k} [{lo}, {hi}) differs")
        out.put(msgs)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_sharded_two_gpus_match_oracle(dtype):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, dtype, q)) for r in range(2)]
    for p in ps:
        p.start()
    msgs = q.get(timeout=240)
    for p in ps:
        p.join(120)
        assert p.exitcode == 0
    assert not msgs, "\n".join(msgs)


def test_sharded_empty_selection_fallback_matches_oracle():
    """Examples that no shard selects a candidate for take every neuron on
    every shard (the fallback of the unsharded layer, over the global count);
    the step still matches the oracle's 2-shard network."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, "f32", q, "fallback")) for r in range(2)]
    for p in ps:
        p.start()
    msgs = q.get(timeout=240)
    for p in ps:
        p.join(120)
        assert p.exitcode == 0
    assert not msgs, "\n".join(msgs)


@pytest.mark.parametrize("sampling", ["topk", "threshold"])
def test_sharded_global_selection_matches_oracle(sampling):
    """TopK below the candidate count and Threshold select over the candidates
    of all shards, as the unsharded layer does."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, "f32", q, sampling)) for r in range(2)]
    for p in ps:
        p.start()
    msgs = q.get(timeout=240)
    for p in ps:
        p.join(120)
        assert p.exitcode == 0
    assert not msgs, "\n".join(msgs)


def _examples(hb):
    from klearu_b200.data import Example, SparseVector

    out = []
    for s in range(hb.batch):
        a, b = int(hb.rowptr[s]), int(hb.rowptr[s + 1])
        c, d = int(hb.label_ptr[s]), int(hb.label_ptr[s + 1])
        out.append(Example(SparseVector(hb.idx[a:b], hb.val[a:b], 0), list(hb.labels[c:d])))
    return out


def _fault_worker(rank, world, port, out):
    """Rank 1 passes a batch the exchange cannot carry (more nnz than its fixed
    capacity, then one example short).  Every rank must return the fault from
    the same step, none may block, and no weight may move in that step."""
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from klearu_b200 import _lib
        from klearu_b200 import synthetic as S
        from klearu_b200.core import Context, Network
        from klearu_b200.data import HostBatch
        from klearu_b200.dist import rank_slice, share_unique_id

        cfg = _cfg()
        init = S.make_init(cfg, 42)
        uid = share_unique_id(rank, world)
        B = 24
        net = Network(cfg, init, weight_dtype="f32", max_batch=B, ctx=Context(rank), shard=(uid, rank, world))
        gen = S.XcGenerator(2000, 5000, seed=3, mean_nnz=20)
        good = rank_slice(gen.batch(B * world), rank, world)
        rng = np.random.default_rng(rank)
        nz = 600  # > the exchange's 512 nnz per example
        heavy = HostBatch(np.arange(B + 1, dtype=np.int32) * nz,
                          np.concatenate([np.sort(rng.choice(2000, nz, replace=False)) for _ in range(B)]).astype(np.uint32),
                          np.full(B * nz, 0.05, np.float32), np.arange(B + 1, dtype=np.int32),
                          np.zeros(B, np.uint32))
        short = rank_slice(gen.batch(B * world), rank, world)
        short = HostBatch(short.rowptr[:B], short.idx[:short.rowptr[B - 1]], short.val[:short.rowptr[B - 1]],
                          short.label_ptr[:B], short.labels[:short.label_ptr[B - 1]])
        res = []
        net.train_step_host(good, 1e-3)
        for bad, want in ((heavy, 7), (short, 6)):  # KL_ECAPACITY, KL_EBOUNDS
            w0 = net.get_layer(1)["weights"]
            code = 0
            try:
                net.train_step_host(bad if rank == 1 else good, 1e-3)
            except _lib.KlError as e:
                code = e.status
            moved = not np.array_equal(w0, net.get_layer(1)["weights"])
            res.append((code, want, moved))
        net.train_step_host(good, 1e-3)  # the network keeps working afterwards
        res.append((0, 0, False))
        out.put((rank, res))
    except Exception:
        import traceback

        out.put((rank, traceback.format_exc()))
        raise
    finally:
        dist.destroy_process_group()


def test_sharded_fault_is_raised_on_every_rank():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_fault_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    got = dict(q.get(timeout=240) for _ in range(2))
    for p in ps:
        p.join(120)
    for r in range(2):
        assert not isinstance(got[r], str), got[r]
        for code, want, moved in got[r]:
            assert code == want, (r, got[r])
            assert not moved, (r, got[r])


def _leave_worker(rank, world, port, out):
    """Rank 1 leaves between steps (nothing of it in flight), announced through
    the heartbeat.  Rank 0 must learn of it before launching its next step,
    abort its communicator with nothing in flight, and from then on get
    KL_ENCCL from every call that needs the communicator, without blocking."""
    import datetime
    import time

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    import torch.distributed as dist

    store = dist.TCPStore("127.0.0.1", port, world, rank == 0, timeout=datetime.timedelta(seconds=60))
    try:
        from klearu_b200 import _lib
        from klearu_b200 import synthetic as S
        from klearu_b200.core import Context, Network
        from klearu_b200.dist import Heartbeat, RankFailure, rank_slice

        lib = _lib.load()
        if rank == 0:
            buf = __import__("ctypes").create_string_buffer(lib.kl_dist_unique_id_size())
            _lib.check(lib.kl_dist_get_unique_id(buf))
            store.set("uid", bytes(buf.raw))
        uid = store.get("uid")
        cfg = _cfg()
        net = Network(cfg, S.make_init(cfg, 42), weight_dtype="f32", max_batch=24, ctx=Context(rank),
                      shard=(uid, rank, world))
        net.set_comm_timeout(20000)
        hb = Heartbeat(store, rank, world, timeout_s=20.0)
        gen = S.XcGenerator(2000, 5000, seed=3, mean_nnz=20)
        events = []
        for step in range(4):
            hb.check(step)
            hb_batch = rank_slice(gen.batch(24 * world), rank, world)
            net.train_step_host(hb_batch, 1e-3)
            if rank == 1 and step == 1:
                net.sync()
                hb.leave()
                hb.beat()
                t0 = time.monotonic()  # leave once rank 0 has finished step 1 too
                while hb._count("beat/0") < 2 and time.monotonic() - t0 < 60:
                    time.sleep(0.01)
                net.comm_abort()
                events.append("left")
                break
            hb.beat()
            events.append(f"step{step}")
    except RankFailure as e:
        events.append(f"failure {e.ranks} {e.reason} {e.step}")
        net.sync()
        net.comm_abort()
        for call in (lambda: net.train_step_host(hb_batch, 1e-3), lambda: net.forward_batch(_examples(hb_batch))):
            try:
                call()
                events.append("ran")
            except _lib.KlError as k:
                events.append(_lib.STATUS_NAMES[k.status])
        net.sync()  # the drained queue still answers
        events.append("synced")
    except Exception:
        import traceback

        events = traceback.format_exc()
    out.put((rank, events))
    if rank == 0:
        time.sleep(1.0)  # the store's server lives in rank 0


def test_sharded_rank_leaving_between_steps_is_detected():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_leave_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    got = dict(q.get(timeout=240) for _ in range(2))
    for p in ps:
        p.join(120)
        assert p.exitcode == 0
    assert got[1] == ["step0", "left"], got[1]
    assert got[0] == ["step0", "step1", "failure [1] left 2", "KL_ENCCL", "KL_ENCCL", "synced"], got[0]
