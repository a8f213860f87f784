"""GPU parity of the SLIDE train step (Network) vs the CPU oracle.

Bar (north_star): active sets bit-exact; logits, gradients and updated
weights within 1e-3 relative error in f32 (absolute floor 1e-6 for values
near zero), or one bf16 ulp for bf16 storage.
"""

import math

import numpy as np
import pytest
import torch

from klearu_b200 import synthetic as S
from klearu_b200.config import (ActivationType, BucketType, HashFunctionType as HF, LayerConfig, LshConfig,
                                NetworkConfig, OptimizerType, SamplingType, SlideConfig)
from klearu_b200.core import Network
from klearu_b200.data import Example, HostBatch

pytestmark = pytest.mark.gpu

RTOL = 1e-3
ATOL = 1e-6


def tiny_config(opt=OptimizerType.Sgd):  # network/net.rs:245-286
    return SlideConfig(NetworkConfig([
        LayerConfig(4, 8, ActivationType.Relu, LshConfig(num_tables=3, num_hashes=4), SamplingType.TopK, 1, 8),
        LayerConfig(8, 3, ActivationType.Softmax, LshConfig(num_tables=3, num_hashes=4), SamplingType.TopK, 1, 3,
                    True)], opt, 0.01, 4, 1), 42, False)


def xc_small(bucket=BucketType.Fifo, out_hash=HF.DwtaHash, out_k=8, sampling=SamplingType.TopK, base=100):
    cfg = S.config_xc(d_in=2000, hidden=64, n_out=5000, out_hash=out_hash, out_k=out_k, out_l=10, bucket=bucket,
                      cap=32, hidden_lsh=LshConfig(num_tables=10, num_hashes=6), rebuild_base=base,
                      rebuild_decay=0.1)
    cfg.network.layers[1].sampling = sampling
    cfg.network.layers[1].sampling_threshold = 2
    return cfg


def c0_small():
    h = LayerConfig.hidden(30, 64)
    h.lsh = LshConfig(num_tables=12, num_hashes=5)
    o = LayerConfig.output(64, 10)
    o.lsh = LshConfig(num_tables=12, num_hashes=4)
    return SlideConfig(NetworkConfig([h, o], OptimizerType.Adam, 1e-3, 16, 1), 42, False)


def three_layer():
    a = LayerConfig.hidden(300, 48)
    a.lsh = LshConfig(num_tables=8, num_hashes=5)
    b = LayerConfig(48, 40, ActivationType.Tanh, LshConfig(HF.WtaHash, num_tables=8, num_hashes=4), SamplingType.TopK,
                    2, 20)
    c = LayerConfig(40, 700, ActivationType.Sigmoid, LshConfig(HF.DwtaHash, num_tables=8, num_hashes=6,
                                                              bucket_capacity=16), SamplingType.Vanilla, 2, 0, True)
    return SlideConfig(NetworkConfig([a, b, c], OptimizerType.Adam, 1e-3, 16, 1), 42, False)


def xc_batches(n_batches, B, d_in=2000, n_out=5000, seed=3):
    g = S.XcGenerator(d_in, n_out, seed=seed, mean_nnz=20)
    return [g.batch(B) for _ in range(n_batches)]


def assert_layers_close(gnet, onet, nl, dtype="f32"):
    for l in range(nl):
        gl, ol = gnet.get_layer(l), onet.get_layer(l)
        for k in ("weights", "bias", "m", "v", "mb", "vb"):
            a, b = gl[k], ol[k]
            if dtype == "bf16" and k == "weights":
                # one bf16 ulp of the larger magnitude
                ulp = np.maximum(np.abs(b), np.abs(a)) * 2.0 ** -7
                bad = np.abs(a - b) > ulp + ATOL
            else:
                bad = np.abs(a - b) > RTOL * np.abs(b) + ATOL
            assert not bad.any(), f"layer {l} {k}: {int(bad.sum())} of {bad.size} differ; max " \
                                  f"{np.abs(a - b).max()}"


def forward_sets_match(gnet, onet, hb, exact_values=True, max_mismatch=0.0):
    outs = gnet.forward_batch(_examples(hb))
    mism = 0
    total = 0
    for s in range(hb.batch):
        a, b = int(hb.rowptr[s]), int(hb.rowptr[s + 1])
        ores = onet.forward(hb.idx[a:b], hb.val[a:b])
        for l, (oi, op, oa) in enumerate(ores):
            g = outs[s][l]
            gi = np.asarray(g.active_neurons, np.uint32)
            total += 1
            if not (len(gi) == len(oi) and (gi == oi).all()):
                mism += 1
                continue
            if exact_values:
                assert (g.pre_activations == op).all(), f"example {s} layer {l}: pre-activations differ"
            act = g.activations[gi]
            assert np.allclose(act, oa, rtol=1e-5, atol=1e-7), f"example {s} layer {l}: activations differ"
    assert mism <= max_mismatch * total, f"{mism}/{total} active sets differ"


def _examples(hb):
    from klearu_b200.data import SparseVector

    out = []
    for s in range(hb.batch):
        a, b = int(hb.rowptr[s]), int(hb.rowptr[s + 1])
        c, d = int(hb.label_ptr[s]), int(hb.label_ptr[s + 1])
        out.append(Example(SparseVector(hb.idx[a:b], hb.val[a:b], 0), list(hb.labels[c:d])))
    return out


def pair(cfg, dtype="f32", max_batch=64, seed=42):
    init = S.make_init(cfg, seed)
    import oracle

    return Network(cfg, init, weight_dtype=dtype, max_batch=max_batch), oracle.Net(cfg, init, weight_dtype=dtype)


def test_tiny_network_exact_mode(gpu_ctx):  # the reference's make_tiny_config
    cfg = tiny_config()
    g, o = pair(cfg)
    exs = [Example.new([1, 0, 0, 0], [0]), Example.new([0, 1, 0, 0], [1]), Example.new([0, 0, 1, 0], [2])]
    hb = HostBatch.from_examples(exs)
    forward_sets_match(g, o, hb)
    for _ in range(5):
        lg = g.train_step(exs, 0.1, mode="exact")
        lo = o.train_step(hb, 0.1, mode="exact")
        assert math.isfinite(lg) and abs(lg - lo) <= 1e-4 * abs(lo) + 1e-6
    assert g.step == o.step == 5
    assert_layers_close(g, o, 2)
    assert g.train_step([], 0.1) == 0.0


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("mode", ["exact", "batched"])
def test_xc_small_matches_oracle(gpu_ctx, dtype, mode):
    cfg = xc_small()
    g, o = pair(cfg, dtype)
    batches = xc_batches(3, 6 if mode == "exact" else 48)
    forward_sets_match(g, o, batches[0])
    for hb in batches:
        db = g.device_batch(hb)
        import ctypes as C

        from klearu_b200 import _lib

        out = C.c_float()
        m = _lib.MODE_EXACT_SEQUENTIAL if mode == "exact" else _lib.MODE_BATCHED
        _lib.check(g.lib.kl_net_train_step(g.h, C.byref(db.c), 1e-3, m, None, C.byref(out)), g.ctx.h)
        lo = o.train_step(hb, 1e-3, mode=mode)
        assert abs(out.value - lo) <= 1e-4 * abs(lo) + 1e-6, (out.value, lo)
    assert_layers_close(g, o, 2, dtype)
    forward_sets_match(g, o, batches[0], exact_values=False, max_mismatch=0.02)


@pytest.mark.parametrize("variant", ["reservoir_simhash", "threshold", "vanilla"])
def test_xc_variants_batched(gpu_ctx, variant):
    if variant == "reservoir_simhash":
        cfg = xc_small(BucketType.Reservoir, HF.SimHash, 9)
    elif variant == "threshold":
        cfg = xc_small(sampling=SamplingType.Threshold)
    else:
        cfg = xc_small(sampling=SamplingType.Vanilla)
    g, o = pair(cfg)
    batches = xc_batches(2, 32, seed=9)
    forward_sets_match(g, o, batches[0])
    for hb in batches:
        lg = g.train_step(_examples(hb), 1e-3, mode="batched")
        lo = o.train_step(hb, 1e-3, mode="batched")
        assert abs(lg - lo) <= 1e-4 * abs(lo) + 1e-6
    assert_layers_close(g, o, 2)


def test_softmax_output_top1(gpu_ctx):  # C0 shape: output top_k = num_neurons/10 = 1
    cfg = c0_small()
    g, o = pair(cfg)
    rng = np.random.default_rng(4)
    for _ in range(3):
        hb = S.dense_batch(rng, 8, 30, 10)
        forward_sets_match(g, o, hb, exact_values=False, max_mismatch=0.02)
        lg = g.train_step(_examples(hb), 1e-3, mode="exact")
        lo = o.train_step(hb, 1e-3, mode="exact")
        assert abs(lg - lo) <= 1e-4 * abs(lo) + 1e-6
    assert_layers_close(g, o, 2)


def test_three_layer_network(gpu_ctx):
    cfg = three_layer()
    g, o = pair(cfg)
    gen = S.XcGenerator(300, 700, seed=5, mean_nnz=15)
    for _ in range(2):
        hb = gen.batch(16)
        lg = g.train_step(_examples(hb), 1e-3, mode="batched")
        lo = o.train_step(hb, 1e-3, mode="batched")
        assert abs(lg - lo) <= 1e-4 * abs(lo) + 1e-6
    assert_layers_close(g, o, 3)


def test_rebuild_schedule_and_tables(gpu_ctx):
    cfg = xc_small(base=2)
    g, o = pair(cfg)
    # initial build (Layer::new) is bit-identical
    for l in range(2):
        for a, b in zip(g.layer_index(l).export(), o.export_index(l)):
            assert (a == b).all()
    for hb in xc_batches(5, 8, seed=11):
        g.train_step(_examples(hb), 1e-3, mode="batched")
        o.train_step(hb, 1e-3, mode="batched")
    s, nxt, cnt = g.scheduler_state()
    assert s == o.step == 5 and nxt == o.next_rebuild() and cnt >= 2
    # a rebuild from identical weights gives identical tables
    for l in range(2):
        g.set_layer(l, **o.get_layer(l))
    g.rebuild()
    import oracle

    oracle.lib().orc_net_rebuild(o.h)
    for l in range(2):
        for a, b in zip(g.layer_index(l).export(), o.export_index(l)):
            assert (a == b).all()


def test_predict_top_k(gpu_ctx):
    cfg = xc_small()
    g, o = pair(cfg)
    hb = xc_batches(1, 4, seed=13)[0]
    ids, sc = g.predict_top_k_batch(_examples(hb), 10)
    for s in range(hb.batch):
        a, b = int(hb.rowptr[s]), int(hb.rowptr[s + 1])
        oi, _, oa = o.forward(hb.idx[a:b], hb.val[a:b])[-1]
        order = sorted(zip(oi.tolist(), oa.tolist()), key=lambda t: (-t[1], t[0]))[:10]
        assert [int(i) for i in ids[s]] == [i for i, _ in order]
        assert np.allclose(sc[s], [v for _, v in order], rtol=1e-5)


def test_determinism_two_runs(gpu_ctx):
    cfg = xc_small()
    init = S.make_init(cfg, 7)
    nets = [Network(cfg, init, max_batch=64) for _ in range(2)]
    for hb in xc_batches(3, 64, seed=17):
        for n in nets:
            n.train_step(_examples(hb), 1e-3, mode="batched")
    for l in range(2):
        a, b = nets[0].get_layer(l), nets[1].get_layer(l)
        for k in a:
            assert (a[k] == b[k]).all(), k


def test_device_batch_and_stats(gpu_ctx):
    cfg = xc_small()
    g, _ = pair(cfg)
    hb = xc_batches(1, 32, seed=19)[0]
    db = g.device_batch(hb)
    loss = torch.zeros(1, device="cuda")
    g.train_step_device(db, 1e-3, loss=loss)
    g.ctx.sync()
    assert math.isfinite(float(loss.item()))
    st = g.stats(1, reset=True)
    assert st.examples == 32 and st.steps == 1 and 0 < st.active_sum <= 32 * 320 and st.touched_rows > 0
    st0 = g.stats(0)
    assert st0.input_nnz == hb.rowptr[-1]


@pytest.mark.parametrize("hidden", [24, 200])
def test_hidden_widths(gpu_ctx, hidden):
    # 24 neurons: several feature rows per warp in the streaming update;
    # 200 neurons: one feature row split over two warps
    cfg = S.config_xc(d_in=2000, hidden=hidden, n_out=3000, out_hash=HF.DwtaHash, out_k=8, out_l=10,
                      bucket=BucketType.Fifo, cap=32, hidden_lsh=LshConfig(num_tables=10, num_hashes=6),
                      rebuild_base=100, rebuild_decay=0.1)
    for dtype in ("f32", "bf16"):
        g, o = pair(cfg, dtype)
        for hb in xc_batches(3, 32, n_out=3000, seed=23):
            lg = g.train_step(_examples(hb), 1e-3, mode="batched")
            lo = o.train_step(hb, 1e-3, mode="batched")
            assert abs(lg - lo) <= 1e-4 * abs(lo) + 1e-6
        assert_layers_close(g, o, 2, dtype)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_first_step_output_gradients_bit_exact(gpu_ctx, dtype):
    # Adam's first moment starts at zero, so after one step m = (1 - b1) * g
    # exactly: equal m means the GPU's per-row output-layer gradient sums
    # (weights and biases) are bit-identical to the oracle's ordered sums.
    # An identity output makes the local gradients (post - label weight)
    # exact arithmetic on both sides, so only the summation is under test
    # (softmax and sigmoid go through exp, whose CPU and GPU results may
    # differ in the last place).  The hidden layer's local gradients come from
    # dX, accumulated in another order than the oracle's: tolerance there.
    cfg = xc_small()
    cfg.network.layers[1].activation = ActivationType.Identity
    g, o = pair(cfg, dtype)
    hb = xc_batches(1, 64, seed=29)[0]
    g.train_step(_examples(hb), 1e-3, mode="batched")
    o.train_step(hb, 1e-3, mode="batched")
    gl, ol = g.get_layer(1), o.get_layer(1)
    for k in ("m", "mb"):
        diff = int((gl[k] != ol[k]).sum())
        assert diff == 0, f"output {k}: {diff} of {gl[k].size} differ"
    assert_layers_close(g, o, 2, dtype)


def test_host_batch_train_step_matches_device_batches(gpu_ctx):
    # kl_net_train_step_host (host CSR arrays, pipelined upload, loss read in
    # stream order) against kl_net_train_step on device batches: the same
    # deterministic steps, so identical losses and weights
    cfg = xc_small()
    init = S.make_init(cfg, 31)
    a, b = Network(cfg, init, max_batch=64), Network(cfg, init, max_batch=64)
    batches = xc_batches(6, 40, seed=37) + [xc_batches(1, 64, seed=41)[0]]  # last one grows the staging slots
    la = [a.train_step(_examples(hb), 1e-3, mode="batched") for hb in batches]
    outs = [torch.zeros(1, dtype=torch.float32).pin_memory() for _ in batches]
    for hb, o in zip(batches, outs):
        assert b.train_step_host(hb, 1e-3, loss_out=o) is None  # no wait between calls
    b.ctx.sync()
    assert [float(o[0]) for o in outs] == la
    for l in range(2):
        x, y = a.get_layer(l), b.get_layer(l)
        for k in x:
            assert (x[k] == y[k]).all(), (l, k)
    assert b.train_step_host(HostBatch.from_examples([]), 1e-3) == 0.0


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_c0_readme_mlp_shape(gpu_ctx, dtype):
    # the README MLP at full width (784 -> 1024 ReLU -> 10 softmax): wide hidden
    # rows with ~10 % active neurons take the active-column gather forward
    cfg = S.config_c0()
    g, o = pair(cfg, dtype, max_batch=32)
    rng = np.random.default_rng(8)
    hb = S.dense_batch(rng, 6, 784, 10)
    forward_sets_match(g, o, hb, exact_values=True)
    for _ in range(2):
        hb = S.dense_batch(rng, 32, 784, 10)
        lg = g.train_step(_examples(hb), 1e-3, mode="batched")
        lo = o.train_step(hb, 1e-3, mode="batched")
        assert abs(lg - lo) <= 1e-4 * abs(lo) + 1e-6
    assert_layers_close(g, o, 2, dtype)


def test_large_batch_dense_update(gpu_ctx):
    # a batch of >= 512 examples takes the dense update's 2-warp blocks and the
    # streamed hidden bias gradient (the shape a shard meets over an 8-rank
    # global batch; 1100 examples span two of its 1024-row chunks and a ragged
    # tail); first Adam moments equal the oracle's bit for bit (identity
    # output: exact local gradients)
    cfg = xc_small()
    cfg.network.layers[1].activation = ActivationType.Identity
    g, o = pair(cfg, "f32", max_batch=1100)
    hb = xc_batches(1, 1100, seed=31)[0]
    g.train_step(_examples(hb), 1e-3, mode="batched")
    o.train_step(hb, 1e-3, mode="batched")
    gl, ol = g.get_layer(1), o.get_layer(1)
    for k in ("m", "mb"):
        assert int((gl[k] != ol[k]).sum()) == 0, k
    assert_layers_close(g, o, 2)
