"""The Deja Vu oracle (oracle/dejavu.cpp) against the behaviour the
reference's own tests pin (klearu-dejavu predictor/mlp_predictor.rs tests,
klearu-dejavu mlp.rs tests, klearu-llm sparse/sparse_mlp.rs tests).  The
reference draws its predictor weights from rand's StdRng, which is not
available here, so the checks use explicit weights; seeded construction is
parity-unpinned."""

import numpy as np

import oracle


def _pred(rng, d, hid, out, scale=0.2):
    return (rng.standard_normal((hid, d)).astype(np.float32) * scale, np.zeros(hid, np.float32),
            rng.standard_normal((out, hid)).astype(np.float32) * scale, np.zeros(out, np.float32))


def test_predict_is_sigmoid_of_relu_mlp():  # mlp_predictor.rs:102-123, test_predict_output_range
    rng = np.random.default_rng(1)
    w1, b1, w2, b2 = _pred(rng, 64, 32, 12)
    b1[:] = rng.standard_normal(32).astype(np.float32)
    x = rng.standard_normal((3, 64)).astype(np.float32)
    got = oracle.pred_predict(w1, b1, w2, b2, x)
    assert got.shape == (3, 12) and ((got >= 0) & (got <= 1)).all()
    for t in range(3):
        h = np.zeros(32, np.float32)
        for i in range(32):  # sequential f32 fold, as iter().sum()
            s = np.float32(0)
            for j in range(64):
                s = np.float32(s + np.float32(w1[i, j] * x[t, j]))
            h[i] = max(np.float32(s + b1[i]), np.float32(0))
        for i in range(12):
            s = np.float32(0)
            for j in range(32):
                s = np.float32(s + np.float32(w2[i, j] * h[j]))
            logit = np.float32(s + b2[i])
            assert abs(got[t, i] - np.float32(1) / (np.float32(1) + np.exp(-logit))) <= 1e-7


def test_select_top_k_order_ties_and_clamp():  # mlp_predictor.rs:126-132 and its tests
    scores = np.array([0.3, 0.9, 0.5, 0.9, 0.1, 0.5], np.float32)
    assert oracle.pred_topk(scores, 4).tolist() == [1, 3, 2, 5]  # stable: equal scores keep index order
    assert oracle.pred_topk(scores, 20).tolist() == [1, 3, 2, 5, 0, 4]  # test_select_top_k_more_than_available
    rng = np.random.default_rng(2)
    w1, b1, w2, b2 = _pred(rng, 64, 32, 12)
    sel = oracle.pred_topk(oracle.pred_predict(w1, b1, w2, b2, np.ones(64, np.float32))[0], 5)
    assert len(set(sel.tolist())) == 5  # test_select_top_k_no_duplicates


def _swiglu_dense(gate, up, down, bias, x):
    g = gate @ x
    u = up @ x
    a = (g / (1 + np.exp(-g))) * u
    out = down @ a
    return out if bias is None else out + bias


def test_sparse_mlp_all_neurons_matches_dense():  # sparse_mlp.rs tests / mlp.rs test_sparse_matches_dense_all_neurons
    rng = np.random.default_rng(3)
    hid, inter = 32, 64
    gate, up = (rng.standard_normal((inter, hid)).astype(np.float32) * 0.2 for _ in range(2))
    down = rng.standard_normal((hid, inter)).astype(np.float32) * 0.2
    bias = rng.standard_normal(hid).astype(np.float32)
    x = np.full(hid, 0.3, np.float32)
    for b in (None, bias):
        got = oracle.sparse_mlp(gate, up, down, b, x, np.arange(inter))
        assert np.abs(got - _swiglu_dense(gate, up, down, b, x)).max() < 1e-4


def test_sparse_mlp_known_weights():  # sparse_mlp.rs test_sparse_mlp_all_neurons_matches_dense
    hid, inter = 4, 8
    gate = np.zeros((inter, hid), np.float32)
    for i in range(inter):
        gate[i, i % 4] = 0.1
    down = np.zeros((hid, inter), np.float32)
    for j in range(hid):
        down[j, j] = 0.1
    x = np.ones(hid, np.float32)
    got = oracle.sparse_mlp(gate, gate.copy(), down, None, x, np.arange(inter))
    silu = np.float32(0.1) / (1 + np.exp(np.float32(-0.1)))
    assert np.allclose(got, np.float32(0.1) * silu * np.float32(0.1), atol=1e-7)
    # a subset: only the selected neurons contribute, in the given order
    sub = oracle.sparse_mlp(gate, gate.copy(), down, None, x, np.array([2, 0]))
    assert np.allclose(sub, [0.1 * silu * 0.1, 0, 0.1 * silu * 0.1, 0], atol=1e-7)
