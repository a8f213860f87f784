"""Benchmark configurations and seeded synthetic inputs.

No dataset is available offline, so seeded synthetic inputs with the shapes
and value distributions of the named workloads stand in for them:

* C0 -- the README MLP: dense U[0,1)^784 inputs, 784 -> 1024 ReLU -> 10
  softmax, SimHash K=6 L=50, FIFO cap 128, labels uniform over 10 classes.
* C1 -- extreme classification: 135909-dim sparse inputs (nnz ~ Poisson(75)
  clipped to [1, 300], distinct Zipf(1.1) indices over a seeded permutation,
  log-normal values, L2-normalised), hidden 128 ReLU with the reference's
  LayerConfig::hidden defaults (SimHash K=6 L=50, TopK 12), output 670091
  sigmoid with DWTA K=8 L=50 FIFO cap 128, 1..7 Zipfian labels per example.
* C2 -- the same architecture at 3.1M outputs, hidden 256, SimHash K=9 L=50,
  reservoir buckets.
"""

from __future__ import annotations

import numpy as np

from . import params as P
from .config import (ActivationType, BucketType, HashFunctionType, LayerConfig, LshConfig, NetworkConfig,
                     OptimizerType, SlideConfig)
from .data import HostBatch


def config_c0() -> SlideConfig:
    hidden = LayerConfig.hidden(784, 1024)
    out = LayerConfig.output(1024, 10)
    return SlideConfig(NetworkConfig([hidden, out], OptimizerType.Adam, 1e-3, 128, 1), 42, False)


def config_xc(d_in: int = 135909, hidden: int = 128, n_out: int = 670091, out_hash=HashFunctionType.DwtaHash,
              out_k: int = 8, out_l: int = 50, bucket=BucketType.Fifo, cap: int = 128,
              hidden_lsh: LshConfig | None = None, rebuild_base: int = 100, rebuild_decay: float = 0.1,
              hidden_topk: int | None = None, out_topk: int | None = None) -> SlideConfig:
    h = LayerConfig.hidden(d_in, hidden)
    if hidden_lsh is not None:
        h.lsh = hidden_lsh
    h.lsh.rebuild_interval_base = rebuild_base
    h.lsh.rebuild_decay = rebuild_decay
    if hidden_topk is not None:
        h.top_k = hidden_topk
    o = LayerConfig.output(hidden, n_out)
    o.activation = ActivationType.Sigmoid
    o.lsh = LshConfig(out_hash, bucket, out_l, out_k, out_k, cap, rebuild_base, rebuild_decay)
    if out_topk is not None:
        o.top_k = out_topk
    return SlideConfig(NetworkConfig([h, o], OptimizerType.Adam, 1e-3, 256, 1), 42, False)


def config_c1() -> SlideConfig:
    return config_xc()


def config_c2(n_out: int = 3_100_000) -> SlideConfig:
    return config_xc(hidden=256, n_out=n_out, out_hash=HashFunctionType.SimHash, out_k=9, out_l=50,
                     bucket=BucketType.Reservoir)


def make_init(cfg: SlideConfig, seed: int = 42) -> list[dict]:
    """Explicit parameters of every layer (weights, bias, hash arrays)."""
    rng = np.random.default_rng(seed)
    out = []
    for lc in cfg.network.layers:
        d = P.hash_params(lc.lsh.hash_function, rng, lc.input_dim, lc.lsh.num_hashes, lc.lsh.num_tables,
                          min(8, lc.input_dim))
        d["weights"] = P.init_weights(rng, lc.num_neurons, lc.input_dim)
        d["bias"] = np.zeros(lc.num_neurons, np.float32)
        out.append(d)
    return out


class Zipf:
    """Finite Zipf(s) over a seeded permutation of 0..n-1 (inverse CDF)."""

    def __init__(self, n: int, s: float, rng: np.random.Generator):
        w = 1.0 / np.arange(1, n + 1, dtype=np.float64) ** s
        self.cdf = np.cumsum(w)
        self.cdf /= self.cdf[-1]
        self.perm = rng.permutation(n).astype(np.uint32)

    def draw_distinct(self, rng: np.random.Generator, k: int) -> np.ndarray:
        got: list[int] = []
        seen = set()
        while len(got) < k:
            for r in np.searchsorted(self.cdf, rng.random(2 * k + 4), side="right"):
                v = int(self.perm[min(int(r), len(self.perm) - 1)])
                if v not in seen:
                    seen.add(v)
                    got.append(v)
                    if len(got) == k:
                        break
        return np.asarray(got, np.uint32)


class XcGenerator:
    """Seeded C1/C2 example stream."""

    def __init__(self, d_in: int, n_out: int, seed: int = 1234, mean_nnz: float = 75.0, max_labels: int = 7):
        self.rng = np.random.default_rng(seed)
        self.d_in, self.n_out = d_in, n_out
        self.feat = Zipf(d_in, 1.1, self.rng)
        self.lab = Zipf(n_out, 1.1, self.rng)
        self.mean_nnz, self.max_labels = mean_nnz, max_labels

    def batch(self, B: int) -> HostBatch:
        rng = self.rng
        rp, lp = [0], [0]
        idx, val, labs = [], [], []
        for _ in range(B):
            nnz = int(np.clip(rng.poisson(self.mean_nnz), 1, min(300, self.d_in)))
            ix = np.sort(self.feat.draw_distinct(rng, nnz))
            v = rng.lognormal(0.0, 1.0, nnz).astype(np.float32)
            v = (v / np.float32(np.sqrt(np.sum(v.astype(np.float64) ** 2)))).astype(np.float32)
            idx.append(ix)
            val.append(v)
            rp.append(rp[-1] + nnz)
            nl = int(rng.integers(1, self.max_labels + 1))
            labs.append(self.lab.draw_distinct(rng, nl))
            lp.append(lp[-1] + nl)
        return HostBatch(np.asarray(rp, np.int32), np.concatenate(idx), np.concatenate(val),
                         np.asarray(lp, np.int32), np.concatenate(labs))


def dense_batch(rng: np.random.Generator, B: int, d: int, n_classes: int) -> HostBatch:
    """C0: dense U[0,1) inputs (as CSR of the nonzeros), one uniform label."""
    x = rng.random((B, d), dtype=np.float32)
    rp = np.arange(B + 1, dtype=np.int32) * d
    nz = x.reshape(-1)
    keep = nz != 0.0
    if not keep.all():  # SparseVector::from_dense drops exact zeros
        rows = [np.nonzero(r)[0] for r in x]
        rp = np.cumsum([0] + [len(r) for r in rows]).astype(np.int32)
        idx = np.concatenate(rows).astype(np.uint32)
        val = np.concatenate([x[i, r] for i, r in enumerate(rows)])
    else:
        idx = np.tile(np.arange(d, dtype=np.uint32), B)
        val = nz
    labels = rng.integers(0, n_classes, B).astype(np.uint32)
    return HostBatch(rp, idx, val.astype(np.float32), np.arange(B + 1, dtype=np.int32), labels)
