"""BOLT SparseInferenceEngine (crates/klearu-bolt/src/sparse_inference.rs)
on the GPU against a CPU restatement over the oracle's index.

The reference orders candidates by count with a stable sort over HashMap
order; here ties go by id ascending, and the restatement below does the same
over the oracle's id-sorted query.  Activations are sequential f32 sums, so
ids and activations are compared exactly.
"""

import numpy as np
import pytest
import torch

from klearu_b200 import params as P
from klearu_b200.bolt import SparseInferenceEngine, network_bolt_infer
from klearu_b200.config import BucketType, HashFunctionType as HF
from klearu_b200.core import HashFamily, LshIndex

pytestmark = pytest.mark.gpu


def restated_infer(oidx, x, W, b, base_top_k, mult, relu):
    ids, cnt = oidx.query(x)  # sorted by id
    order = sorted(range(len(ids)), key=lambda i: -int(cnt[i]))  # stable: ties keep id order
    v = np.float32(base_top_k) * np.float32(mult)
    k = 0 if not v > 0 else int(v)
    out = []
    for i in order[:k]:
        nid = int(ids[i])
        if nid >= W.shape[0]:
            continue
        acc = np.float32(0.0)
        for a, w in zip(x, W[nid]):
            acc = np.float32(acc + np.float32(np.float32(a) * np.float32(w)))
        a = np.float32(acc + np.float32(b[nid] if b is not None else 0.0))
        out.append((nid, float(max(a, np.float32(0.0)) if relu else a)))
    return out


@pytest.mark.parametrize("mult,base_k,relu", [(1.0, 40, True), (2.5, 30, False), (0.5, 1000, True)])
def test_bolt_matches_restatement(gpu_ctx, orc, mult, base_k, relu):
    d, K, L, N, cap = 48, 5, 12, 3000, 24
    rng = np.random.default_rng(3)
    prm = P.hash_params(HF.SimHash, rng, d, K, L)
    W = rng.standard_normal((N, d)).astype(np.float32) * 0.3
    b = rng.standard_normal(N).astype(np.float32) * 0.1
    ix = LshIndex(HashFamily(HF.SimHash, d, K, L, params=prm, ctx=gpu_ctx), BucketType.Fifo, cap)
    ix.rebuild_rows(torch.from_numpy(W))
    oi = orc.Index(orc.Hash(HF.SimHash, d, K, L, 8, prm), int(BucketType.Fifo), cap)
    oi.insert(np.arange(N, dtype=np.uint32), W)
    X = (W[rng.integers(0, N, 6)] + 0.1 * rng.standard_normal((6, d))).astype(np.float32)
    eng = SparseInferenceEngine(mult)
    ids, act, cnt = eng.infer_batch(X, ix, W, b, base_k, relu)
    for q in range(len(X)):
        want = restated_infer(oi, X[q], W, b, base_k, mult, relu)
        got = list(zip(ids[q, :cnt[q]].tolist(), act[q, :cnt[q]].tolist()))
        assert [i for i, _ in got] == [i for i, _ in want], q
        assert np.array_equal(np.float32([a for _, a in got]), np.float32([a for _, a in want])), q
    # the single-input forms
    one = eng.infer(X[0], ix, W, b, base_k) if relu else eng.infer_linear(X[0], ix, W, b, base_k)
    assert [i for i, _ in one] == ids[0, :cnt[0]].tolist()


def test_bolt_reference_cases(gpu_ctx):  # sparse_inference.rs:150-200
    eng = SparseInferenceEngine(1.0)
    neurons = np.eye(4, dtype=np.float32)
    ix = LshIndex(HashFamily(HF.SimHash, 4, 4, 50, params=P.hash_params(HF.SimHash, np.random.default_rng(42), 4, 4,
                                                                         50), ctx=gpu_ctx), BucketType.Fifo, 128)
    ix.rebuild_rows(torch.from_numpy(neurons))
    assert eng.infer([1, 0, 0, 0], ix, neurons, np.zeros(4, np.float32), 4)  # basic: some result
    neg = np.array([[-1.0, -1.0]], np.float32)
    ix2 = LshIndex(HashFamily(HF.SimHash, 2, 4, 50, params=P.hash_params(HF.SimHash, np.random.default_rng(1), 2, 4,
                                                                          50), ctx=gpu_ctx), BucketType.Fifo, 128)
    ix2.rebuild_rows(torch.from_numpy(neg))
    assert all(a == 0.0 for _, a in eng.infer([1, 1], ix2, neg, np.zeros(1, np.float32), 1))  # relu clamps
    lin = eng.infer_linear([1, 1], ix2, neg, np.zeros(1, np.float32), 1)
    assert all(a == -2.0 for _, a in lin)  # linear keeps the sign
    assert eng.infer([1, 1], ix2, neg, None, 0) == []  # effective_k 0


def test_network_bolt_layer(gpu_ctx):
    from klearu_b200 import synthetic as S
    from klearu_b200.config import LshConfig
    from klearu_b200.core import Network

    cfg = S.config_xc(d_in=2000, hidden=64, n_out=5000, out_l=10, cap=32,
                      hidden_lsh=LshConfig(num_tables=10, num_hashes=6))
    init = S.make_init(cfg, 42)
    net = Network(cfg, init, weight_dtype="bf16", max_batch=16)
    H = np.abs(np.random.default_rng(2).standard_normal((5, 64))).astype(np.float32)
    ids, act, cnt = network_bolt_infer(net, 1, H, 1.0, 100, relu=False)
    # the same through the engine on the layer's own index and stored (bf16) weights
    lw = torch.from_numpy(net.get_layer(1)["weights"]).to(torch.bfloat16)
    i2, a2, c2 = SparseInferenceEngine(1.0).infer_batch(H, net.layer_index(1), lw, net.get_layer(1)["bias"], 100,
                                                        relu=False)
    assert (cnt == c2).all() and (ids == i2).all() and (act == a2).all()
    assert (cnt > 0).all()
