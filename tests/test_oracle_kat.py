"""Pin the CPU oracle against the reference's own unit tests (known answers).

Each test cites the reference test it ports (crates/klearu-core/src/...).
Seeded constructions of the reference (rand 0.8.5 StdRng) cannot be
reproduced, so seeded tests use explicit parameters drawn with the same
distributions; tests whose answer does not depend on the seed keep the
reference's exact expected values.
"""

import math

import numpy as np
import pytest

from klearu_b200 import params as P
from klearu_b200.config import (ActivationType, BucketType, HashFunctionType as HF, LayerConfig, LshConfig,
                                NetworkConfig, OptimizerType, SamplingType, SlideConfig)
from klearu_b200.data import Example, HostBatch, SparseVector

pytestmark = []


def rng(seed=0):
    return np.random.default_rng(seed)


# ---------------------------------------------------------------- hashes ---
def test_simhash_zero_vector_all_bits(orc):  # hash/simhash.rs:231-240
    d, K, L = 16, 6, 8
    h = orc.Hash(HF.SimHash, d, K, L, 8, P.hash_params(HF.SimHash, rng(1), d, K, L))
    codes = h.dense(np.zeros((1, d), np.float32))
    assert (codes == (1 << K) - 1).all()


def test_srp_sparsity_zero_all_ones(orc):  # hash/srp.rs:240-249
    d, K, L = 10, 5, 4
    rp, ix, cf = P.srp_projections(rng(2), L, K, d, sparsity=0.0)
    assert rp[-1] == 0
    h = orc.Hash(HF.SparseRandomProjection, d, K, L, 8, {"srp_rowptr": rp, "srp_idx": ix, "srp_coef": cf})
    x = rng(3).standard_normal((3, d)).astype(np.float32)
    assert (h.dense(x) == (1 << K) - 1).all()


def _minhash_expected(mins, k):
    prime = 0x517CC1B727220A95
    h, pp = 0, 1
    for m in mins:
        h = (h + m * pp) & 0xFFFFFFFFFFFFFFFF
        pp = (pp * prime) & 0xFFFFFFFFFFFFFFFF
    return h & ((1 << k) - 1)


def test_minhash_densify(orc):  # hash/minhash.rs:257-268: [MAX,5,MAX,MAX] -> [5,5,5,5]
    d, k = 8, 4  # bin_size 2; identity permutation
    perms = np.arange(d, dtype=np.uint32)[None]
    h = orc.Hash(HF.MinHash, d, k, 1, 8, {"perms": perms})
    x = np.zeros((1, d), np.float32)
    x[0, 3] = 1.0  # permuted index 3 -> bin 1 holds 3; bins 0,2,3 empty
    assert int(h.dense(x)[0, 0]) == _minhash_expected([3, 3, 3, 3], k)
    # all bins empty -> all zero
    assert int(h.dense(np.zeros((1, d), np.float32))[0, 0]) == _minhash_expected([0, 0, 0, 0], k)


def test_wta_positive_scale_invariance(orc):  # hash/wta.rs:201-215
    d, K, L = 32, 4, 6
    h = orc.Hash(HF.WtaHash, d, K, L, 8, P.hash_params(HF.WtaHash, rng(4), d, K, L))
    x = rng(5).standard_normal((1, d)).astype(np.float32)
    assert (h.dense(x) == h.dense(x * np.float32(3.5))).all()


@pytest.mark.parametrize("kind", [HF.SimHash, HF.WtaHash, HF.MinHash, HF.SparseRandomProjection, HF.DwtaHash])
def test_dense_sparse_agree(orc, kind):  # hash/mod.rs:44-55 assert_dense_sparse_agree; dwta.rs:223-229
    d, K, L = 40, 5, 7
    h = orc.Hash(kind, d, K, L, 8, P.hash_params(kind, rng(6), d, K, L))
    x = rng(7).standard_normal((5, d)).astype(np.float32)
    if kind != HF.DwtaHash:
        x[:, ::3] = 0.0  # sparse rows (DWTA agrees on fully dense input only)
    rows = [SparseVector.from_dense(r) for r in x]
    rp = np.cumsum([0] + [len(r.indices) for r in rows]).astype(np.int32)
    ix = np.concatenate([r.indices for r in rows])
    vv = np.concatenate([r.values for r in rows])
    assert (h.dense(x) == h.sparse(rp, ix, vv)).all()


def test_hash_in_range(orc):  # hash/mod.rs:58-65 assert_hash_in_range
    for kind in (HF.SimHash, HF.SparseRandomProjection, HF.MinHash):
        d, K, L = 24, 6, 5
        h = orc.Hash(kind, d, K, L, 8, P.hash_params(kind, rng(8), d, K, L))
        x = rng(9).standard_normal((10, d)).astype(np.float32)
        assert (h.dense(x) < (1 << K)).all()


def test_dwta_sparse_fallback_in_window(orc):  # dwta.rs:248-257 (deterministic, in range)
    d, K, L, w = 64, 3, 4, 8
    h = orc.Hash(HF.DwtaHash, d, K, L, w, P.hash_params(HF.DwtaHash, rng(10), d, K, L, w))
    c1 = h.sparse([0, 0], [], [])
    c2 = h.sparse([0, 0], [], [])
    assert (c1 == c2).all()
    for t in range(L):
        for kk in range(K):
            pos = (int(c1[0, t]) >> (3 * kk)) & 7
            assert pos == orc.lib().orc_siphash13_usize2(t, kk) % w


# --------------------------------------------------------------- buckets ---
def test_fifo_order_after_evictions(orc):  # bucket/fifo.rs:99-114
    b = orc.Bucket(BucketType.Fifo, 2)
    b.insert(1)
    b.insert(2)
    b.insert(3)
    assert b.contents() == [2, 3]
    b.insert(4)
    assert b.contents() == [3, 4]
    b.insert(5)
    assert b.contents() == [4, 5]


def test_fifo_capacity_and_eviction(orc):  # bucket/fifo.rs:80-96
    b = orc.Bucket(BucketType.Fifo, 3)
    for v in (10, 20, 30):
        b.insert(v)
    assert b.contents() == [10, 20, 30]
    b.insert(40)
    assert 10 not in b.contents() and 40 in b.contents() and len(b.contents()) == 3


def test_fifo_capacity_one_remove_clear(orc):  # bucket/fifo.rs:116-161
    b = orc.Bucket(BucketType.Fifo, 1)
    b.insert(10)
    assert b.contents() == [10]
    b.insert(20)
    assert b.contents() == [20]
    b = orc.Bucket(BucketType.Fifo, 4)
    for v in (1, 2, 3):
        b.insert(v)
    assert b.remove(2) and b.contents() == [1, 3]  # swap_remove
    assert not b.remove(99)
    b.clear()
    assert b.contents() == []


def test_reservoir_within_capacity(orc):  # bucket/reservoir.rs:110-122
    b = orc.Bucket(BucketType.Reservoir, 4)
    for v in (1, 2, 3):
        b.insert(v)
    assert sorted(b.contents()) == [1, 2, 3] and b.total_insertions() == 3


def test_reservoir_capacity_total_deterministic(orc):  # reservoir.rs:124-148
    b = orc.Bucket(BucketType.Reservoir, 3)
    for i in range(100):
        b.insert(i)
    assert len(b.contents()) <= 3 and b.total_insertions() == 100
    b1, b2 = orc.Bucket(BucketType.Reservoir, 4), orc.Bucket(BucketType.Reservoir, 4)
    for i in range(50):
        b1.insert(i)
        b2.insert(i)
    assert b1.contents() == b2.contents()


def test_reservoir_clear_resets_count(orc):  # reservoir.rs:172-181
    b = orc.Bucket(BucketType.Reservoir, 4)
    b.insert(1)
    b.insert(2)
    b.clear()
    assert b.contents() == [] and b.total_insertions() == 0


def test_reservoir_fairness(orc):  # reservoir.rs:195-222
    counts = np.zeros(10)
    for trial in range(10000):
        b = orc.Bucket(BucketType.Reservoir, 5)
        for i in range(10):
            b.insert(i + trial * 1000)
        for v in b.contents():
            counts[v - trial * 1000] += 1
    ratio = counts / 5000.0
    assert ((ratio >= 0.5) & (ratio <= 1.5)).all(), ratio


def _py_reservoir(ids, cap):
    """Independent pure-Python restatement of reservoir.rs:50-67."""
    M = 0xFFFFFFFFFFFFFFFF

    def sm(seed, bound):
        z = (seed + 0x9E3779B97F4A7C15) & M
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M
        return (z ^ (z >> 31)) % bound

    data, count = [], 0
    for i in ids:
        count += 1
        if len(data) < cap:
            data.append(i)
        else:
            seed = (count * 0x517CC1B727220A95 + i) & M
            if sm(seed, count) < cap:
                data[sm((seed + 1) & M, cap)] = i
    return data


def test_reservoir_matches_independent_restatement(orc):
    ids = list(rng(11).integers(0, 1 << 31, 300))
    b = orc.Bucket(BucketType.Reservoir, 7)
    for i in ids:
        b.insert(int(i))
    assert b.contents() == _py_reservoir([int(i) for i in ids], 7)


# ----------------------------------------------------------------- index ---
def _index(orc, kind=HF.SimHash, d=8, K=6, L=50, cap=128, bt=BucketType.Fifo, seed=12):
    h = orc.Hash(kind, d, K, L, 8, P.hash_params(kind, rng(seed), d, K, L))
    return orc.Index(h, bt, cap)


def test_index_self_query_counts_all_tables(orc):  # lsh/index.rs:416-434
    ix = _index(orc)
    w = np.array([1.0, 0.5, -0.3, 0.0, 2.0, -1.0, 0.1, 0.7], np.float32)
    ix.insert([100], w[None])
    ids, cnt = ix.query(w)
    assert 100 in ids and cnt[list(ids).index(100)] == 50


def test_index_remove_clear_rebuild(orc):  # lsh/index.rs:453-526
    ix = _index(orc, d=4)
    w = np.array([1.0, 0.5, -0.3, 0.2], np.float32)
    ix.insert([10], w[None])
    assert 10 in ix.query(w)[0]
    ix.remove_with_weights([10], w[None])
    assert 10 not in ix.query(w)[0]
    ix.insert([10], w[None])
    ix.remove([10])
    assert 10 not in ix.query(w)[0]
    ix.insert([10], w[None])
    ix.clear()
    assert len(ix.query(w)[0]) == 0
    w1 = np.array([1, 0, 0, 0], np.float32)
    w2 = np.array([0, 1, 0, 0], np.float32)
    ix.insert([1], w1[None])
    ix.clear()
    ix.insert([2], w2[None])  # rebuild = clear + insert
    assert 1 not in ix.query(w1)[0] and 2 in ix.query(w2)[0]


# -------------------------------------------------------------- sampling ---
def test_topk_kats(orc):  # sampling/topk.rs:40-116
    S = SamplingType.TopK
    assert orc.sample(S, 2, 0, [0, 1, 2, 3], [3, 5, 1, 4]) == [1, 3]
    assert orc.sample(S, 10, 0, [0, 1], [1, 2]) == [1, 0]
    assert orc.sample(S, 3, 0, [10, 20, 30], [5, 3, 1]) == [10, 20, 30]
    assert orc.sample(S, 5, 0, [], []) == []
    assert orc.sample(S, 0, 0, [0, 1], [5, 3]) == []
    assert orc.sample(S, 2, 0, [5, 2, 8, 1], [3, 3, 3, 3]) == [1, 2]
    assert orc.sample(S, 1, 0, [0, 1, 2], [1, 10, 5]) == [1]


def test_threshold_kats(orc):  # sampling/threshold.rs tests
    S = SamplingType.Threshold
    assert orc.sample(S, 0, 3, [0, 1, 2], [3, 1, 5]) == [0, 2]
    assert orc.sample(S, 0, 10, [4, 2, 7], [3, 3, 1]) == [2]  # fallback top-1, lowest id on ties
    assert orc.sample(S, 0, 2, [], []) == []


def test_vanilla_returns_all(orc):  # sampling/vanilla.rs
    assert orc.sample(SamplingType.Vanilla, 0, 0, [3, 1, 2], [1, 1, 1]) == [3, 1, 2]


# ------------------------------------------------------------- scheduler ---
def test_scheduler_fixed_interval(orc):  # lsh/maintenance.rs:117-131
    s = orc.Scheduler(5, 0.0)
    fired = [t for t in range(1, 31) if s.should_rebuild(t)]
    assert fired == [5, 10, 15, 20, 25, 30]


def test_scheduler_next_and_count(orc):  # lsh/maintenance.rs:108-115, 150-170
    s = orc.Scheduler(10, 0.0)
    assert s.next_rebuild() == 10
    for t in range(1, 10):
        assert not s.should_rebuild(t)
    assert s.should_rebuild(10)
    assert s.next_rebuild() == 20 and s.rebuild_count() == 1


def test_scheduler_growing_intervals(orc):  # lsh/maintenance.rs:133-148
    s = orc.Scheduler(10, 0.5)
    fired = [t for t in range(1, 501) if s.should_rebuild(t)]
    iv = np.diff([0] + fired)
    assert (np.diff(iv) >= 0).all()
    # next interval = floor(base * e^(decay * count))
    assert iv[1] == int(10 * math.exp(0.5 * 1))


# ------------------------------------------------------------ loss / grad ---
def test_loss_kats(orc):  # network/net.rs:403-462
    assert abs(orc.compute_loss([0.1, 0.7, 0.2], [0, 1, 2], [1]) - (-math.log(0.7))) < 1e-4
    exp = (-math.log(0.3) - math.log(0.5)) / 2
    assert abs(orc.compute_loss([0.3, 0.5, 0.2], [0, 1, 2], [0, 1]) - exp) < 1e-4
    assert orc.compute_loss([0.5, 0.5], [0, 1], []) == 0.0
    assert abs(orc.compute_loss([0.5, 0.5, 0.0], [0, 1], [2]) - (-math.log(1e-7))) < 1.0


def test_loss_gradient_kat(orc):  # network/net.rs:478-493
    g = orc.compute_loss_gradient([0.2, 0.5, 0.3], [0, 1, 2], [1], 3)
    assert abs(g[1] + 0.5) < 1e-6 and abs(g[0] - 0.2) < 1e-6 and abs(g[2] - 0.3) < 1e-6


# -------------------------------------------------------------- optimizers ---
def test_sgd_momentum_trajectory(orc):  # optim/sgd.rs:95-116
    w, b, m, v, mb, vb = [1.0, 2.0], 0.5, [0.0, 0.0], [0.0, 0.0], 0.0, 0.0
    w, b, m, v, mb, vb = orc.optimizer_update(OptimizerType.Sgd, w, [1.0, 1.0], b, 1.0, 0.1, 1, m, v, mb, vb)
    assert abs(w[0] - 0.9) < 1e-6 and abs(w[1] - 1.9) < 1e-6 and abs(b - 0.4) < 1e-6
    w, b, m, v, mb, vb = orc.optimizer_update(OptimizerType.Sgd, w, [1.0, 1.0], b, 1.0, 0.1, 2, m, v, mb, vb)
    assert abs(w[0] - 0.71) < 1e-6 and abs(w[1] - 1.71) < 1e-6 and abs(b - 0.21) < 1e-6


def test_sgd_vanilla_kats(orc):  # optim/sgd.rs:118-181 (momentum 0)
    w, b, *_ = orc.optimizer_update(OptimizerType.Sgd, [5.0, 3.0], [0.0, 0.0], 1.0, 0.0, 0.1, 1, [0, 0], [0, 0],
                                    0.0, 0.0, momentum=0.0)
    assert list(w) == [5.0, 3.0] and b == 1.0
    w, b, *_ = orc.optimizer_update(OptimizerType.Sgd, [0.0], [1.0], 0.0, 1.0, 10.0, 1, [0], [0], 0.0, 0.0,
                                    momentum=0.0)
    assert abs(w[0] + 10.0) < 1e-6 and abs(b + 10.0) < 1e-6


def test_adam_zero_gradient_noop(orc):  # optim/adam.rs:176-191
    w, b, *_ = orc.optimizer_update(OptimizerType.Adam, [1.0, 2.0], [0.0, 0.0], 0.5, 0.0, 0.01, 1, [0, 0], [0, 0],
                                    0.0, 0.0)
    assert abs(w[0] - 1.0) < 1e-6 and abs(w[1] - 2.0) < 1e-6 and abs(b - 0.5) < 1e-6


def test_adam_first_step_is_lr_sign(orc):  # optim/adam.rs:131-155 (single step, bias correction)
    w, b, m, v, mb, vb = orc.optimizer_update(OptimizerType.Adam, [1.0], [0.5], 0.5, 0.5, 0.01, 1, [0], [0], 0.0, 0.0)
    assert abs(w[0] - (1.0 - 0.01)) < 1e-5 and abs(b - (0.5 - 0.01)) < 1e-5
    # step 0 is clamped to 1 (adam.rs:39)
    w0, *_ = orc.optimizer_update(OptimizerType.Adam, [1.0], [0.5], 0.5, 0.5, 0.01, 0, [0], [0], 0.0, 0.0)
    assert w0[0] == w[0]


def test_powi_and_bf16(orc):
    L = orc.lib()
    for b in range(0, 40):
        assert L.orc_powi_f32(0.999, b) == pytest.approx(0.999 ** b, rel=1e-5)
    import torch

    x = rng(13).standard_normal(4096).astype(np.float32) * np.float32(10.0)
    ref = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    got = np.array([L.orc_f32_to_bf16(float(v)) for v in x], np.uint16)
    assert (ref == got).all()


# ----------------------------------------------------------------- network ---
def tiny_config(opt=OptimizerType.Sgd):  # network/net.rs:245-286 make_tiny_config
    lsh = LshConfig(num_tables=3, num_hashes=4)
    return SlideConfig(NetworkConfig([
        LayerConfig(4, 8, ActivationType.Relu, lsh, SamplingType.TopK, 1, 8, False),
        LayerConfig(8, 3, ActivationType.Softmax, LshConfig(num_tables=3, num_hashes=4), SamplingType.TopK, 1, 3,
                    True)], opt, 0.01, 4, 1), 42, False)


def tiny_init(cfg, seed=42):
    r = rng(seed)
    out = []
    for lc in cfg.network.layers:
        d = P.hash_params(lc.lsh.hash_function, r, lc.input_dim, lc.lsh.num_hashes, lc.lsh.num_tables)
        d["weights"] = P.init_weights(r, lc.num_neurons, lc.input_dim)
        d["bias"] = np.zeros(lc.num_neurons, np.float32)
        out.append(d)
    return out


def test_network_train_step_kats(orc):  # network/net.rs:339-393
    cfg = tiny_config()
    net = orc.Net(cfg, tiny_init(cfg))
    ex = Example.new([1.0, 0.5, -0.3, 0.2], [1])
    loss = net.train_step(HostBatch.from_examples([ex]), 0.01)
    assert math.isfinite(loss) and loss >= 0.0 and net.step == 1
    net.train_step(HostBatch.from_examples([ex]), 0.01)
    assert net.step == 2
    assert net.train_step(HostBatch.from_examples([]), 0.01) == 0.0


def test_network_softmax_sums_to_one(orc):  # network/layer.rs:376-400
    cfg = tiny_config()
    net = orc.Net(cfg, tiny_init(cfg))
    sv = SparseVector.from_dense([1.0, 0.5, -0.3, 0.2])
    outs = net.forward(sv.indices, sv.values)
    acts = outs[-1][2]
    assert abs(float(acts.sum()) - 1.0) < 1e-5 and ((acts >= 0) & (acts <= 1)).all()


def test_network_deterministic(orc):  # network/net.rs:548-573
    cfg = tiny_config()
    a, b = orc.Net(cfg, tiny_init(cfg)), orc.Net(cfg, tiny_init(cfg))
    sv = SparseVector.from_dense([1.0, 0.5, -0.3, 0.2])
    for (ia, pa, xa), (ib, pb, xb) in zip(a.forward(sv.indices, sv.values), b.forward(sv.indices, sv.values)):
        assert (ia == ib).all() and (xa == xb).all()


def test_network_adam_and_multilabel_finite(orc):  # network/net.rs:495-546
    cfg = tiny_config(OptimizerType.Adam)
    net = orc.Net(cfg, tiny_init(cfg))
    assert math.isfinite(net.train_step(HostBatch.from_examples([Example.new([1.0, 0.5, -0.3, 0.2], [0])]), 0.001))
    cfg = tiny_config()
    net = orc.Net(cfg, tiny_init(cfg))
    l2 = net.train_step(HostBatch.from_examples([Example.new([1.0, 0.5, -0.3, 0.2], [0, 2])]), 0.01)
    assert math.isfinite(l2) and l2 >= 0


def test_network_training_does_not_diverge(orc):  # network/net.rs:355-381
    cfg = tiny_config()
    net = orc.Net(cfg, tiny_init(cfg))
    exs = [Example.new([1, 0, 0, 0], [0]), Example.new([0, 1, 0, 0], [1]), Example.new([0, 0, 1, 0], [2])]
    hb = HostBatch.from_examples(exs)
    first = net.train_step(hb, 0.1)
    last = first
    for _ in range(20):
        last = net.train_step(hb, 0.1)
    assert math.isfinite(last) and last < first * 2.0
