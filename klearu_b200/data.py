"""Examples and CSR batches (crates/klearu-core/src/data/dataset.rs:5-16,
crates/klearu-core/src/tensor/sparse.rs:14-83)."""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass
class SparseVector:
    """Sorted unique indices with values, like klearu's SparseVector."""

    indices: np.ndarray
    values: np.ndarray
    dim: int

    @staticmethod
    def from_dense(dense) -> "SparseVector":  # sparse.rs:60-74: drops exact zeros
        dense = np.asarray(dense, dtype=np.float32)
        nz = np.nonzero(dense != 0.0)[0]
        return SparseVector(nz.astype(np.uint32), dense[nz].astype(np.float32), len(dense))

    @staticmethod
    def from_pairs(dim: int, pairs) -> "SparseVector":  # sparse.rs:36-58: sorted, duplicates summed
        acc: dict[int, float] = {}
        for i, v in pairs:
            acc[int(i)] = np.float32(acc.get(int(i), np.float32(0.0)) + np.float32(v))
        keys = sorted(acc)
        return SparseVector(np.asarray(keys, dtype=np.uint32), np.asarray([acc[k] for k in keys], np.float32), dim)

    def to_dense(self) -> np.ndarray:  # sparse.rs:77-83
        out = np.zeros(self.dim, dtype=np.float32)
        out[self.indices] = self.values
        return out


@dataclass
class Example:
    features: SparseVector
    labels: list

    @staticmethod
    def new(dense_features, labels) -> "Example":  # dataset.rs:11-16
        return Example(SparseVector.from_dense(dense_features), list(labels))


@dataclass
class HostBatch:
    """A CSR batch in host memory (numpy)."""

    rowptr: np.ndarray   # int32 [B+1]
    idx: np.ndarray      # uint32 [nnz]
    val: np.ndarray      # float32 [nnz]
    label_ptr: np.ndarray  # int32 [B+1]
    labels: np.ndarray   # uint32 [nlabels]

    @property
    def batch(self) -> int:
        return len(self.rowptr) - 1

    @staticmethod
    def from_examples(examples) -> "HostBatch":
        rp, lp = [0], [0]
        idx, val, labs = [], [], []
        for ex in examples:
            idx.append(np.asarray(ex.features.indices, np.uint32))
            val.append(np.asarray(ex.features.values, np.float32))
            rp.append(rp[-1] + len(ex.features.indices))
            labs.append(np.asarray(ex.labels, np.uint32))
            lp.append(lp[-1] + len(ex.labels))
        cat = lambda xs, dt: np.concatenate(xs).astype(dt) if xs else np.zeros(0, dt)  # noqa: E731
        return HostBatch(np.asarray(rp, np.int32), cat(idx, np.uint32), cat(val, np.float32),
                         np.asarray(lp, np.int32), cat(labs, np.uint32))

    def slice(self, s0: int, s1: int) -> "HostBatch":
        a, b = int(self.rowptr[s0]), int(self.rowptr[s1])
        c, d = int(self.label_ptr[s0]), int(self.label_ptr[s1])
        return HostBatch((self.rowptr[s0:s1 + 1] - a).astype(np.int32), self.idx[a:b], self.val[a:b],
                         (self.label_ptr[s0:s1 + 1] - c).astype(np.int32), self.labels[c:d])
