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


# ---------------------------------------------------------------------------
# LibSVM / XML datasets and shuffled batches over the native loader
# (klearu_b200/csrc/data.cu, kl_libsvm_* / kl_dataset_* / kl_batch_iter_*).
# ---------------------------------------------------------------------------
class DatasetError(ValueError):
    """A malformed LibSVM line (the message names the 1-based line, as
    KlearuError::Parse does in crates/klearu-core/src/data/libsvm.rs)."""


def _native():
    from . import _lib

    return _lib


class LibSvmDataset:
    """LibSvmDataset (crates/klearu-core/src/data/libsvm.rs:22-124) backed by
    the native multi-threaded parser; implements the Dataset trait
    (data/dataset.rs:19-35): len, get, feature_dim, num_labels."""

    def __init__(self, handle, lib):
        self.h, self.lib = handle, lib
        import ctypes as C

        n, fd, nl, nnz, nlab = (C.c_int64() for _ in range(5))
        lib.kl_dataset_info(handle, C.byref(n), C.byref(fd), C.byref(nl), C.byref(nnz), C.byref(nlab))
        self._len, self._fd, self._nl = n.value, fd.value, nl.value
        ptrs = [C.c_void_p() for _ in range(5)]
        lib.kl_dataset_csr(handle, *(C.byref(p) for p in ptrs))

        def view(p, ct, count, dt):
            if count == 0 or not p.value:
                return np.zeros(0, dt)
            return np.ctypeslib.as_array(C.cast(p, C.POINTER(ct)), shape=(count,)).view(dt)

        self.rowptr = view(ptrs[0], C.c_int64, self._len + 1, np.int64)
        self.idx = view(ptrs[1], C.c_uint32, nnz.value, np.uint32)
        self.val = view(ptrs[2], C.c_float, nnz.value, np.float32)
        self.label_ptr = view(ptrs[3], C.c_int64, self._len + 1, np.int64)
        self.labels = view(ptrs[4], C.c_uint32, nlab.value, np.uint32)

    @staticmethod
    def _check(st, lib):
        L = _native()
        if st != L.KL_OK:
            msg = (lib.kl_last_error(None) or b"").decode()
            raise DatasetError(msg)

    @classmethod
    def load(cls, path, feature_dim: int, num_labels: int, threads: int = 0) -> "LibSvmDataset":  # libsvm.rs:31-36
        import ctypes as C

        L = _native()
        lib = L.load()
        h = C.c_void_p()
        cls._check(lib.kl_libsvm_load(str(path).encode(), feature_dim, num_labels, threads, C.byref(h)), lib)
        return cls(h, lib)

    @classmethod
    def load_from_str(cls, text: str | bytes, feature_dim: int, num_labels: int,
                      threads: int = 0) -> "LibSvmDataset":  # libsvm.rs:39-111 on an in-memory reader
        import ctypes as C

        L = _native()
        lib = L.load()
        data = text.encode() if isinstance(text, str) else bytes(text)
        h = C.c_void_p()
        cls._check(lib.kl_libsvm_parse(data, len(data), feature_dim, num_labels, threads, C.byref(h)), lib)
        return cls(h, lib)

    @classmethod
    def from_examples(cls, examples, feature_dim: int, num_labels: int) -> "LibSvmDataset":  # libsvm.rs:114-124
        import ctypes as C

        L = _native()
        lib = L.load()
        rp = np.cumsum([0] + [len(e.features.indices) for e in examples]).astype(np.int64)
        lp = np.cumsum([0] + [len(e.labels) for e in examples]).astype(np.int64)
        cat = lambda xs, dt: np.ascontiguousarray(np.concatenate(xs), dt) if xs else np.zeros(1, dt)  # noqa: E731
        idx = cat([np.asarray(e.features.indices, np.uint32) for e in examples], np.uint32)
        val = cat([np.asarray(e.features.values, np.float32) for e in examples], np.float32)
        lab = cat([np.asarray(e.labels, np.uint32) for e in examples], np.uint32)
        h = C.c_void_p()
        cls._check(lib.kl_dataset_from_csr(rp.ctypes.data, idx.ctypes.data, val.ctypes.data, lp.ctypes.data,
                                           lab.ctypes.data, len(examples), feature_dim, num_labels, C.byref(h)), lib)
        return cls(h, lib)

    def __del__(self):
        if getattr(self, "h", None):
            self.lib.kl_dataset_destroy(self.h)
            self.h = None

    def __len__(self) -> int:
        return self._len

    def is_empty(self) -> bool:
        return self._len == 0

    def feature_dim(self) -> int:
        return self._fd

    def num_labels(self) -> int:
        return self._nl

    def get(self, i: int) -> Example:
        if not 0 <= i < self._len:
            raise IndexError(i)
        a, b = int(self.rowptr[i]), int(self.rowptr[i + 1])
        c, d = int(self.label_ptr[i]), int(self.label_ptr[i + 1])
        return Example(SparseVector(self.idx[a:b].copy(), self.val[a:b].copy(), self._fd),
                       [int(x) for x in self.labels[c:d]])


class BatchIterator:
    """BatchIterator (crates/klearu-core/src/data/dataset.rs:38-111): the
    reference's seeded SplitMix64 Fisher-Yates order, batches of batch_size
    (the last one short).  Iterating yields kl_batch structs of page-locked
    host CSR arrays (valid until the next batch is drawn), which
    Network.train_step_batch_host passes straight to kl_net_train_step_host;
    ``as_host_batch`` copies one out as a HostBatch."""

    def __init__(self, dataset: LibSvmDataset, batch_size: int, seed: int, prefetch: bool = True):
        import ctypes as C

        self.ds = dataset  # keeps the store alive
        self.lib = dataset.lib
        h = C.c_void_p()
        LibSvmDataset._check(self.lib.kl_batch_iter_create(dataset.h, int(batch_size), int(seed) & (2**64 - 1),
                                                           int(prefetch), C.byref(h)), self.lib)
        self.h = h

    def __del__(self):
        if getattr(self, "h", None):
            self.lib.kl_batch_iter_destroy(self.h)
            self.h = None

    def reset(self, seed: int) -> None:  # dataset.rs:58-68
        LibSvmDataset._check(self.lib.kl_batch_iter_reset(self.h, int(seed) & (2**64 - 1)), self.lib)

    def next_raw(self):
        """The next batch as a _lib.BatchC over the iterator's buffers, or None at the end."""
        import ctypes as C

        L = _native()
        b = L.BatchC()
        LibSvmDataset._check(self.lib.kl_batch_iter_next(self.h, C.byref(b)), self.lib)
        return b if b.batch > 0 else None

    def __iter__(self):
        return self

    def __next__(self):
        b = self.next_raw()
        if b is None:
            raise StopIteration
        return b

    @staticmethod
    def as_host_batch(b) -> HostBatch:
        import ctypes as C

        def arr(p, ct, n, dt):
            if n == 0:
                return np.zeros(0, dt)
            return np.ctypeslib.as_array(C.cast(p, C.POINTER(ct)), shape=(n,)).view(dt).copy()

        return HostBatch(arr(b.rowptr, C.c_int32, b.batch + 1, np.int32), arr(b.idx, C.c_uint32, b.nnz, np.uint32),
                         arr(b.val, C.c_float, b.nnz, np.float32), arr(b.label_ptr, C.c_int32, b.batch + 1, np.int32),
                         arr(b.labels, C.c_uint32, b.nlabels, np.uint32))
