"""Checkpoint save / load and the network's adaptive rebuild policy.

* A network restored from a checkpoint continues exactly as the one that
  wrote it: same losses, weights, Adam state and tables, bit for bit.
* A corrupt or mismatched checkpoint is refused with KL_EINVAL.
* Under KL_REBUILD_ADAPTIVE a layer is rebuilt at max_interval when the
  threshold is never reached, at every check when it is 0, and a rebuilt
  layer's tables are the ones a rebuild from its current weights gives (the
  CPU oracle's index over the same rows).
"""

import numpy as np
import pytest

from klearu_b200 import _lib
from klearu_b200 import synthetic as S
from klearu_b200.config import LshConfig
from klearu_b200.core import Network

pytestmark = pytest.mark.gpu


def _cfg():
    return S.config_xc(d_in=2000, hidden=64, n_out=5000, out_l=10, cap=32,
                       hidden_lsh=LshConfig(num_tables=10, num_hashes=6), rebuild_base=3, rebuild_decay=0.1)


def _batches(n, seed=3, B=32):
    g = S.XcGenerator(2000, 5000, seed=seed, mean_nnz=20)
    return [g.batch(B) for _ in range(n)]


def _state(net):
    out = {}
    for l in range(2):
        for k, v in net.get_layer(l).items():
            out[(l, k)] = v
        for i, a in enumerate(net.layer_index(l).export()):
            out[(l, "table", i)] = a
    out["step"] = net.scheduler_state()
    return out


def _same(a, b):
    assert a.keys() == b.keys()
    for k in a:
        if k == "step":
            assert a[k] == b[k]
        else:
            assert np.array_equal(a[k], b[k]), k


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_checkpoint_round_trip_continues_identically(gpu_ctx, tmp_path, dtype):
    cfg = _cfg()
    init = S.make_init(cfg, 42)
    a = Network(cfg, init, weight_dtype=dtype, max_batch=32)
    bs = _batches(8)
    for hb in bs[:4]:  # crosses a scheduled rebuild (base 3)
        a.train_step_host(hb, 1e-3)
    path = tmp_path / "net.ckpt"
    a.save(path)
    other = S.make_init(cfg, 7)
    for l in range(2):  # other weights and biases (all overwritten), the same hash parameters
        other[l] = {**init[l], "weights": other[l]["weights"], "bias": other[l]["bias"] + 0.5}
    b = Network(cfg, other, weight_dtype=dtype, max_batch=32)
    b.load(path)
    _same(_state(a), _state(b))
    la = [a.train_step_host(hb, 1e-3) for hb in bs[4:]]
    lb = [b.train_step_host(hb, 1e-3) for hb in bs[4:]]
    assert la == lb
    _same(_state(a), _state(b))


def test_checkpoint_refuses_corrupt_and_mismatched_files(gpu_ctx, tmp_path):
    cfg = _cfg()
    a = Network(cfg, S.make_init(cfg, 42), max_batch=32)
    path = tmp_path / "net.ckpt"
    a.save(path)
    raw = bytearray(path.read_bytes())
    raw[len(raw) // 2] ^= 0x40
    bad = tmp_path / "bad.ckpt"
    bad.write_bytes(bytes(raw))
    with pytest.raises(_lib.KlError, match="checksum"):
        a.load(bad)
    other = S.config_xc(d_in=2000, hidden=32, n_out=5000, out_l=10, cap=32,
                        hidden_lsh=LshConfig(num_tables=10, num_hashes=6))
    c = Network(other, S.make_init(other, 1), max_batch=32)
    with pytest.raises(_lib.KlError, match="differs"):
        c.load(path)
    h = Network(cfg, S.make_init(cfg, 9), max_batch=32)  # the same shapes, other hash planes / windows
    with pytest.raises(_lib.KlError, match="hash parameters"):
        h.load(path)
    (tmp_path / "junk.ckpt").write_bytes(b"not a checkpoint at all")
    with pytest.raises(_lib.KlError, match="not a klearu_b200"):
        a.load(tmp_path / "junk.ckpt")


def test_adaptive_policy_forced_and_threshold_rebuilds(gpu_ctx, orc):
    cfg = _cfg()
    init = S.make_init(cfg, 42)
    # threshold 1.0 is never reached before max_interval: forced rebuilds every 4 steps
    n = Network(cfg, init, max_batch=32)
    n.set_rebuild_policy(True, min_interval=2, max_interval=4, sample_fraction=0.2, drift_threshold=1.0, seed=5)
    for hb in _batches(9, seed=11):
        n.train_step_host(hb, 1e-2)
    for l in range(2):
        ema, since, rb = n.rebuild_state(l)
        assert rb == 2 and since == 1 and 0.0 <= ema <= 1.0
    # threshold 0: every drift check (every min_interval steps) rebuilds
    m = Network(cfg, init, max_batch=32)
    m.set_rebuild_policy(True, min_interval=3, max_interval=1000, sample_fraction=0.5, drift_threshold=0.0, seed=5)
    for hb in _batches(6, seed=12):  # checks at steps 3 and 6: the last step rebuilds
        m.train_step_host(hb, 1e-2)
    assert [m.rebuild_state(l)[2] for l in range(2)] == [2, 2]
    # the rebuilt output tables are a rebuild of the current weights
    w = m.get_layer(1)["weights"]
    o = orc.Index(orc.Hash(int(cfg.network.layers[1].lsh.hash_function), 64, 8, 10, 8, init[1]), 0, 32)
    o.insert(np.arange(5000, dtype=np.uint32), w)
    gi, gl, _ = m.layer_index(1).export()
    oi, ol, _ = o.export()
    assert np.array_equal(gl, ol)
    valid = np.arange(gi.shape[2])[None, None, :] < gl[:, :, None]  # slots beyond a bucket's length are unused
    assert np.array_equal(np.where(valid, gi, 0), np.where(valid, oi, 0))
    # the scheduler state travels in a checkpoint
    ema0 = [m.rebuild_state(l) for l in range(2)]
    import tempfile, os

    with tempfile.TemporaryDirectory() as d:
        p = os.path.join(d, "a.ckpt")
        m.save(p)
        k = Network(cfg, init, max_batch=32)
        k.load(p)
    assert [k.rebuild_state(l) for l in range(2)] == ema0
