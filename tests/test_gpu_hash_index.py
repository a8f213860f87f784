"""GPU parity: hash codes, bucket contents and query results of the CUDA
engine vs the CPU oracle, bit-exact, on identical explicit parameters."""

import numpy as np
import pytest
import torch

from klearu_b200 import _lib
from klearu_b200 import params as P
from klearu_b200.config import BucketType, HashFunctionType as HF
from klearu_b200.core import HashFamily, LshIndex
from klearu_b200.data import SparseVector

pytestmark = pytest.mark.gpu

KINDS = [HF.SimHash, HF.WtaHash, HF.DwtaHash, HF.MinHash, HF.SparseRandomProjection]
NEAR_ZERO = 1e-6  # projections this close to 0 are sign-ambiguous under reordering: excluded and logged


def rng(s):
    return np.random.default_rng(s)


def _csr(X):
    rows = [SparseVector.from_dense(r) for r in X]
    rp = np.cumsum([0] + [len(r.indices) for r in rows]).astype(np.int32)
    ix = np.concatenate([r.indices for r in rows]).astype(np.uint32) if rows else np.zeros(0, np.uint32)
    vv = np.concatenate([r.values for r in rows]).astype(np.float32) if rows else np.zeros(0, np.float32)
    return rp, ix, vv


def _cmp_codes(gpu, ora, mn=None):
    gpu = gpu.cpu().numpy().view(np.uint64)
    bad = gpu != ora
    if mn is not None:
        near = mn < NEAR_ZERO
        if (bad & near).any():
            print(f"near-zero projections excluded: {int((bad & near).sum())}")
        bad &= ~near
    assert not bad.any(), f"{int(bad.sum())} codes differ"


@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("d", [7, 50, 300])
def test_hash_dense_sparse_match_oracle(gpu_ctx, orc, kind, d):
    K, L = (6, 13) if kind != HF.MinHash else (5, 9)
    prm = P.hash_params(kind, rng(d), d, K, L)
    g = HashFamily(kind, d, K, L, 8, params=prm, ctx=gpu_ctx)
    o = orc.Hash(kind, d, K, L, 8, prm)
    X = rng(d + 1).standard_normal((37, d)).astype(np.float32)
    X[:, ::4] = 0.0
    X[3] = 0.0  # zero vector: SimHash all ones (simhash.rs:231-240)
    gc, gm = g.hash_dense_batch(torch.from_numpy(X), with_min_abs=True)
    oc, om = o.dense(X, with_min_abs=True)
    _cmp_codes(gc, oc, om if kind in (HF.SimHash, HF.SparseRandomProjection) else None)
    rp, ix, vv = _csr(X)
    gs = g.hash_sparse_batch(rp, ix, vv)
    os_ = o.sparse(rp, ix, vv)
    _cmp_codes(gs, os_)


def test_simhash_long_input_matches_oracle(gpu_ctx, orc):
    d, K, L = 20011, 6, 50
    prm = P.hash_params(HF.SimHash, rng(5), d, K, L)
    g = HashFamily(HF.SimHash, d, K, L, params=prm, ctx=gpu_ctx)
    o = orc.Hash(HF.SimHash, d, K, L, 8, prm)
    X = (rng(6).standard_normal((9, d)) * 0.01).astype(np.float32)
    gc = g.hash_dense_batch(torch.from_numpy(X))
    _cmp_codes(gc, o.dense(X))


def _rows(n, d, s):
    return rng(s).standard_normal((n, d)).astype(np.float32)


@pytest.mark.parametrize("bt", [BucketType.Fifo, BucketType.Reservoir])
@pytest.mark.parametrize("kind", [HF.SimHash, HF.DwtaHash])
def test_index_build_incremental_remove_match_oracle(gpu_ctx, orc, bt, kind):
    d, K, L, cap = 24, 5, 11, 8
    prm = P.hash_params(kind, rng(7), d, K, L)
    g = LshIndex(HashFamily(kind, d, K, L, params=prm, ctx=gpu_ctx), bt, cap)
    o = orc.Index(orc.Hash(kind, d, K, L, 8, prm), bt, cap)
    A = _rows(3000, d, 8)
    idsA = rng(9).permutation(100000)[:3000].astype(np.uint32)
    g.insert_batch(idsA, torch.from_numpy(A))
    o.insert(idsA, A)
    for a, b in zip(g.export(), o.export()):
        assert (a == b).all()
    # second batch on non-empty buckets (FIFO shifts, reservoir continues its count)
    B = _rows(1500, d, 10)
    idsB = (np.arange(1500) + 200000).astype(np.uint32)
    g.insert_batch(idsB, torch.from_numpy(B))
    o.insert(idsB, B)
    for a, b in zip(g.export(), o.export()):
        assert (a == b).all()
    # removals (sequential swap_remove semantics)
    rm = np.concatenate([idsA[:40], idsB[-25:]])
    g_rm = torch.as_tensor(rm.view(np.int32)).cuda()
    _lib.check(g.lib.kl_index_remove(g.h, g_rm.data_ptr(), len(rm)), g.ctx.h)
    o.remove(rm)
    for a, b in zip(g.export(), o.export()):
        assert (a == b).all()
    for i in range(5):
        g.remove_with_weights(int(idsA[100 + i]), A[100 + i])
    o.remove_with_weights(idsA[100:105], A[100:105])
    for a, b in zip(g.export(), o.export()):
        assert (a == b).all()
    # batched queries: counts and union, sorted by id
    Q = np.concatenate([A[:20] + 0.01 * _rows(20, d, 11), _rows(20, d, 12)])
    offs, ids, cnt = (t.cpu().numpy() for t in g.query_batch(torch.from_numpy(Q)))
    for q in range(len(Q)):
        oi, oc = o.query(Q[q])
        gi = ids[offs[q]:offs[q + 1]].view(np.uint32)
        assert (gi == oi).all() and (cnt[offs[q]:offs[q + 1]] == oc).all()
    offs2, ids2, _ = (t.cpu().numpy() for t in g.query_batch(torch.from_numpy(Q), _lib.QUERY_UNION))
    assert (offs2 == offs).all() and (ids2[:offs2[-1]] == ids[:offs[-1]]).all()


def test_index_sparse_insert_query_match_oracle(gpu_ctx, orc):
    d, K, L, cap = 200, 6, 9, 16
    prm = P.hash_params(HF.SimHash, rng(13), d, K, L)
    g = LshIndex(HashFamily(HF.SimHash, d, K, L, params=prm, ctx=gpu_ctx), BucketType.Fifo, cap)
    o = orc.Index(orc.Hash(HF.SimHash, d, K, L, 8, prm), BucketType.Fifo, cap)
    X = _rows(500, d, 14)
    X[rng(15).random(X.shape) < 0.9] = 0.0
    rp, ix, vv = _csr(X)
    ids = np.arange(500, dtype=np.uint32)
    for i in range(0, 500, 100):  # batched sparse inserts in order
        sl = slice(i, i + 100)
        r2 = (rp[i:i + 101] - rp[i]).astype(np.int32)
        gi = torch.as_tensor(ids[sl].view(np.int32)).cuda()
        grp = torch.as_tensor(r2).cuda()
        gix = torch.as_tensor(ix[rp[i]:rp[i + 100]].view(np.int32)).cuda()
        gvv = torch.as_tensor(vv[rp[i]:rp[i + 100]]).cuda()
        _lib.check(g.lib.kl_index_insert_sparse_batch(g.h, gi.data_ptr(), grp.data_ptr(), gix.data_ptr(),
                                                      gvv.data_ptr(), 100), g.ctx.h)
    o.insert_sparse(ids, rp, ix, vv)
    for a, b in zip(g.export(), o.export()):
        assert (a == b).all()
    offs, gids, gcnt = (t.cpu().numpy() for t in g.query_sparse_batch(rp[:31], ix[:rp[30]], vv[:rp[30]]))
    for q in range(30):
        oi, oc = o.query_sparse(ix[rp[q]:rp[q + 1]], vv[rp[q]:rp[q + 1]])
        assert (gids[offs[q]:offs[q + 1]].view(np.uint32) == oi).all()
        assert (gcnt[offs[q]:offs[q + 1]] == oc).all()


def test_index_reference_kats_on_gpu(gpu_ctx):  # lsh/index.rs:400-526
    d, K, L = 8, 6, 50
    prm = P.hash_params(HF.SimHash, rng(16), d, K, L)
    ix = LshIndex(HashFamily(HF.SimHash, d, K, L, params=prm, ctx=gpu_ctx), BucketType.Fifo, 128)
    w = np.array([1.0, 0.5, -0.3, 0.0, 2.0, -1.0, 0.1, 0.7], np.float32)
    ix.insert(100, w)
    c = {x.neuron_id: x.count for x in ix.query_with_counts(w)}
    assert c[100] == L
    assert 100 in ix.query_union(w)
    ix.remove(100)
    assert 100 not in ix.query_union(w)
    ix.insert(10, w)
    ix.remove_with_weights(10, w)
    assert 10 not in ix.query_union(w)
    ix.insert(11, w)
    ix.clear()
    assert ix.query_union(w) == []
    w1 = np.array([1, 0, 0, 0, 0, 0, 0, 0], np.float32)
    w2 = np.array([0, 1, 0, 0, 0, 0, 0, 0], np.float32)
    ix.insert(1, w1)
    ix.rebuild([(2, w2)])
    assert 1 not in ix.query_union(w1) and 2 in ix.query_union(w2)
    sv = SparseVector.from_dense(w2)
    assert 2 in ix.query_sparse_union(sv)


def test_query_capacity_overflow_reported(gpu_ctx):
    d, K, L = 8, 2, 4
    prm = P.hash_params(HF.SimHash, rng(17), d, K, L)
    ix = LshIndex(HashFamily(HF.SimHash, d, K, L, params=prm, ctx=gpu_ctx), BucketType.Fifo, 32)
    ix.insert_batch(np.arange(64, dtype=np.uint32), torch.from_numpy(_rows(64, d, 18)))
    with pytest.raises(_lib.KlError) as e:
        ix.query_batch(torch.from_numpy(_rows(4, d, 19)), capacity=3)
        gpu_ctx.sync()
    assert e.value.status == _lib.KL_ECAPACITY


def test_bad_arguments_rejected(gpu_ctx):
    with pytest.raises(_lib.KlError) as e:
        HashFamily(HF.DwtaHash, 4, 3, 2, window_size=8, params={"windows": np.zeros((2, 3, 4), np.uint32) + 9},
                   ctx=gpu_ctx)
    assert e.value.status == _lib.KL_EINVAL
    prm = P.hash_params(HF.SimHash, rng(20), 8, 4, 4)
    with pytest.raises(_lib.KlError) as e:
        LshIndex(HashFamily(HF.SimHash, 8, 4, 4, params=prm, ctx=gpu_ctx), BucketType.Fifo, 0)
    assert e.value.status == _lib.KL_EINVAL
