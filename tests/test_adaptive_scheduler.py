"""mongoose AdaptiveScheduler (crates/klearu-mongoose/src/scheduler.rs:44-213).

The reference's own tests (scheduler.rs:220-420) run against the CPU oracle
and, marked gpu, against the CUDA scheduler; a third test checks that the GPU
drift estimate equals the oracle's on the same weights, sample and hash.
The reference draws its weights from StdRng(seed).gen_range(-1, 1) and samples
neurons with a StdRng shuffle; neither stream is available here, so uniform
weights come from numpy and the sampled indices are explicit."""

import numpy as np
import pytest
import torch

import oracle
from klearu_b200 import params as P
from klearu_b200.config import HashFunctionType as HF

DIM, K, L = 32, 8, 4


def neurons(n, seed):
    return np.random.default_rng(seed).uniform(-1.0, 1.0, (n, DIM)).astype(np.float32)


def hash_params():
    return P.hash_params(HF.SimHash, np.random.default_rng(42), DIM, K, L)


def sample(n, frac, seed):
    size = min(n, max(1, int(np.ceil(n * frac)))) if n else 0
    return np.sort(np.random.default_rng(seed).permutation(n)[:size]).astype(np.uint32)


class OracleSched:
    def __init__(self, *a):
        self.s = oracle.AdaptiveScheduler(*a)
        self.frac = a[2]
        self.h = oracle.Hash(HF.SimHash, DIM, K, L, 8, hash_params())

    def record(self, rows, seed):
        self.s.record_baseline(rows, self.h, sample(len(rows), self.frac, seed))

    def step(self, rows):
        return self.s.should_rebuild(rows, self.h)


class GpuSched:
    def __init__(self, *a):
        from klearu_b200.core import AdaptiveScheduler, HashFamily, default_context

        ctx = default_context(0)
        self.s = AdaptiveScheduler(*a, ctx=ctx)
        self.frac = a[2]
        self.h = HashFamily(HF.SimHash, DIM, K, L, params=hash_params(), ctx=ctx)

    def record(self, rows, seed):
        self.s.record_baseline(torch.from_numpy(rows), self.h, sampled=sample(len(rows), self.frac, seed))

    def step(self, rows):
        return self.s.should_rebuild(torch.from_numpy(rows))


def _impls():
    return [pytest.param(OracleSched, id="oracle"), pytest.param(GpuSched, id="gpu", marks=pytest.mark.gpu)]


@pytest.mark.parametrize("impl", _impls())
def test_forced_rebuild_at_max_interval(impl):  # scheduler.rs:244-266
    s = impl(5, 10, 0.5, 0.5)
    rows = neurons(20, 100)
    s.record(rows, 99)
    for _ in range(1, 10):
        assert not s.step(rows)
    assert s.step(rows)


@pytest.mark.parametrize("impl", _impls())
def test_no_rebuild_before_min_interval(impl):  # scheduler.rs:270-287
    s = impl(5, 100, 0.5, 0.0)
    rows = neurons(20, 100)
    s.record(rows, 99)
    for _ in range(1, 5):
        assert not s.step(rows)


@pytest.mark.parametrize("impl", _impls())
def test_high_drift_triggers_rebuild(impl):  # scheduler.rs:291-308
    s = impl(1, 1000, 1.0, 0.3)
    s.record(neurons(50, 100), 99)
    assert s.step(neurons(50, 999))


@pytest.mark.parametrize("impl", _impls())
def test_no_drift_no_early_rebuild(impl):  # scheduler.rs:312-326
    s = impl(1, 1000, 1.0, 0.3)
    rows = neurons(50, 100)
    s.record(rows, 99)
    for _ in range(20):
        assert not s.step(rows)


@pytest.mark.parametrize("impl", _impls())
def test_notify_rebuild_resets_counters(impl):  # scheduler.rs:330-339
    s = impl(5, 10, 0.5, 0.5)
    rows = neurons(20, 100)
    s.record(rows, 99)
    for _ in range(3):
        s.step(rows)
    s.s.notify_rebuild()
    assert s.s.steps_since_rebuild() == 0


@pytest.mark.parametrize("impl", _impls())
def test_gradual_drift_triggers_rebuild_eventually(impl):  # scheduler.rs:382-405
    s = impl(1, 10000, 1.0, 0.3)
    s.record(neurons(30, 100), 42)
    drifted = neurons(30, 500)
    assert any(s.step(drifted) for _ in range(100))


@pytest.mark.parametrize("impl", _impls())
def test_empty_neurons_does_not_fail(impl):  # scheduler.rs:409-418
    s = impl(1, 10, 0.5, 0.5)
    empty = np.zeros((0, DIM), np.float32)
    s.record(empty, 42)
    s.step(empty)


@pytest.mark.gpu
def test_sample_size_follows_fraction():  # scheduler.rs:362-378 (seeded sampling of this library)
    from klearu_b200.core import AdaptiveScheduler, HashFamily, default_context

    ctx = default_context(0)
    h = HashFamily(HF.SimHash, DIM, K, L, params=hash_params(), ctx=ctx)
    rows = torch.from_numpy(neurons(100, 100))
    for frac, n in ((0.1, 10), (0.5, 50)):
        s = AdaptiveScheduler(1, 100, frac, 0.5, ctx=ctx)
        s.record_baseline(rows, h, seed=42)
        assert s.num_sampled() == n


@pytest.mark.gpu
def test_gpu_drift_equals_oracle():
    rng = np.random.default_rng(3)
    base = neurons(400, 7)
    g, o = GpuSched(2, 50, 0.25, 0.9), OracleSched(2, 50, 0.25, 0.9)
    g.record(base, 5)
    o.record(base, 5)
    rows = base.copy()
    for step in range(12):
        rows = rows + rng.normal(0, 0.05, rows.shape).astype(np.float32)
        assert g.step(rows) == o.step(rows), step
        assert g.s.drift_estimate() == o.s.drift_estimate(), step
