"""GPU parity at the benchmarked configuration, and of the segmented output update.

* C1 at full size (135909 -> 128 ReLU -> 670091 sigmoid, DWTA K8 L50 FIFO 128,
  B=256, bf16 weight storage): the exact path bench.py times, checked against
  the CPU oracle on the same seeded weights and batches.  Before training, the
  active sets of a sample of examples are bit-exact and their pre-activations
  equal; over three batched steps (eager, captured, replayed) the loss is
  within 1e-4 relative; afterwards the hidden layer and the output layer
  (touched rows and all others) are within 1e-3 relative or one bf16 ulp.
* The segmented output update (rm_touch / seg_alloc / rm_scatter /
  rm_update), which a layer takes when its sample-major gradient matrix would
  exceed the dense path's budget (the 3.1M-way configuration does), forced on
  a small network with dense_update_max_bytes=-1.
"""

import ctypes as C

import numpy as np
import pytest

from klearu_b200 import _lib
from klearu_b200 import synthetic as S
from klearu_b200.config import ActivationType, LshConfig
from klearu_b200.core import Network
from klearu_b200.data import HostBatch

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-3, 1e-6


def _bad(a, b, bf16):
    if bf16:
        return np.abs(a - b) > np.maximum(np.abs(a), np.abs(b)) * 2.0 ** -7 + ATOL
    return np.abs(a - b) > RTOL * np.abs(b) + ATOL


def _compare_layers(g, o, nl, dtype):
    for l in range(nl):
        gl, ol = g.get_layer(l), o.get_layer(l)
        for k in ("weights", "bias", "m", "v", "mb", "vb"):
            bad = _bad(gl[k], ol[k], dtype == "bf16" and k == "weights")
            assert not bad.any(), f"layer {l} {k}: {int(bad.sum())} of {bad.size} differ"
        del gl, ol


def _sub(hb, s0, s1):
    a, b = int(hb.rowptr[s0]), int(hb.rowptr[s1])
    c, d = int(hb.label_ptr[s0]), int(hb.label_ptr[s1])
    return HostBatch((hb.rowptr[s0:s1 + 1] - a).astype(np.int32), hb.idx[a:b], hb.val[a:b],
                     (hb.label_ptr[s0:s1 + 1] - c).astype(np.int32), hb.labels[c:d])


def _step(g, hb):
    db = g.device_batch(hb)
    out = C.c_float()
    _lib.check(g.lib.kl_net_train_step(g.h, C.byref(db.c), 1e-3, _lib.MODE_BATCHED, None, C.byref(out)), g.ctx.h)
    return out.value


def test_c1_full_size_matches_oracle(gpu_ctx):
    import oracle

    cfg = S.config_c1()
    init = S.make_init(cfg, 42)
    g = Network(cfg, init, weight_dtype="bf16", max_batch=256)
    o = oracle.Net(cfg, init, weight_dtype="bf16", sparse_input=True)
    del init
    gen = S.XcGenerator(135909, 670091, seed=1234)
    batches = [gen.batch(256) for _ in range(3)]
    # active sets and pre-activations of a sample of examples at the step-start weights
    probe = _sub(batches[0], 0, 24)
    outs = g.forward_batch(probe)
    for s in range(probe.batch):
        a, b = int(probe.rowptr[s]), int(probe.rowptr[s + 1])
        for l, (oi, op, oa) in enumerate(o.forward(probe.idx[a:b], probe.val[a:b])):
            gi = np.asarray(outs[s][l].active_neurons, np.uint32)
            assert len(gi) == len(oi) and (gi == oi).all(), f"example {s} layer {l}: active sets differ"
            assert (outs[s][l].pre_activations == op).all(), f"example {s} layer {l}: pre-activations differ"
    for i, hb in enumerate(batches):
        lg = _step(g, hb)
        lo = o.train_step(hb, 1e-3, mode="batched")
        assert abs(lg - lo) <= 1e-4 * abs(lo) + 1e-6, (i, lg, lo)
    st = g.stats(1)
    assert st.steps == 3 and st.touched_rows > 0
    _compare_layers(g, o, 2, "bf16")


def _small(dtype):
    cfg = S.config_xc(d_in=2000, hidden=64, n_out=5000, out_l=10, cap=32,
                      hidden_lsh=LshConfig(num_tables=10, num_hashes=6))
    init = S.make_init(cfg, 42)
    import oracle

    return cfg, Network(cfg, init, weight_dtype=dtype, max_batch=64, dense_update_max_bytes=-1), \
        oracle.Net(cfg, init, weight_dtype=dtype)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_segmented_output_update_matches_oracle(gpu_ctx, dtype):
    cfg, g, o = _small(dtype)
    gen = S.XcGenerator(2000, 5000, seed=3, mean_nnz=20)
    for hb in [gen.batch(48) for _ in range(3)]:
        lg = _step(g, hb)
        lo = o.train_step(hb, 1e-3, mode="batched")
        assert abs(lg - lo) <= 1e-4 * abs(lo) + 1e-6
    _compare_layers(g, o, 2, dtype)


def test_segmented_output_update_first_moment_bit_exact(gpu_ctx):
    # identity output: the local gradients are exact on both sides, so an
    # equal first moment after one Adam step means equal ordered gradient sums
    cfg = S.config_xc(d_in=2000, hidden=64, n_out=5000, out_l=10, cap=32,
                      hidden_lsh=LshConfig(num_tables=10, num_hashes=6))
    cfg.network.layers[1].activation = ActivationType.Identity
    init = S.make_init(cfg, 42)
    import oracle

    g = Network(cfg, init, max_batch=64, dense_update_max_bytes=-1)
    o = oracle.Net(cfg, init)
    hb = S.XcGenerator(2000, 5000, seed=29, mean_nnz=20).batch(64)
    _step(g, hb)
    o.train_step(hb, 1e-3, mode="batched")
    gl, ol = g.get_layer(1), o.get_layer(1)
    for k in ("m", "mb"):
        assert int((gl[k] != ol[k]).sum()) == 0, k
