"""Host-side mirror of klearu-core's SLIDE API over the CUDA engine.

Same names, argument meaning and error behaviour as the Rust reference:
``HashFamily`` (crates/klearu-core/src/hash/mod.rs:24-39), ``LshIndex`` /
``create_lsh_index`` (lsh/index.rs:21-67, 339-374) and ``Network``
(network/net.rs:10-173).  Every call goes through the C ABI of
``include/klearu_gpu.h``; PyTorch only provides device memory and the stream.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from ._lib import check
from .config import BucketType, HashFunctionType, LshConfig, SlideConfig
from .data import Example, HostBatch, SparseVector

_DEFAULT_CTX: dict[int, "Context"] = {}


def _ptr(t) -> int | None:
    if t is None:
        return None
    if isinstance(t, torch.Tensor):
        return t.data_ptr() if t.numel() else None
    if isinstance(t, np.ndarray):
        return t.ctypes.data if t.size else None
    raise TypeError(type(t))


class Context:
    """kl_ctx_t: one CUDA device and the stream the engine issues work on."""

    def __init__(self, device: int = 0, stream: torch.cuda.Stream | None = None):
        self.lib = _lib.load()
        if not torch.cuda.is_available():
            raise RuntimeError("klearu_b200 needs a CUDA device (there is no CPU fallback)")
        self.device = device
        self.stream = stream if stream is not None else torch.cuda.current_stream(device)
        h = C.c_void_p()
        check(self.lib.kl_ctx_create(device, C.c_void_p(self.stream.cuda_stream), C.byref(h)), None, "kl_ctx_create")
        self.h = h

    def sync(self) -> None:
        check(self.lib.kl_ctx_sync(self.h), self.h, "kl_ctx_sync")

    def close(self) -> None:
        if getattr(self, "h", None):
            self.lib.kl_ctx_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def default_context(device: int | None = None) -> Context:
    """One shared context per device; `device` None = torch's current device."""
    if device is None:
        device = torch.cuda.current_device() if torch.cuda.is_available() else 0
    if device not in _DEFAULT_CTX:
        _DEFAULT_CTX[device] = Context(device)
    return _DEFAULT_CTX[device]


def hash_params_c(params: dict | None):
    """kl_hash_params from a dict of numpy arrays; returns (struct, keepalive)."""
    hp = _lib.HashParams()
    keep = []
    if params:
        spec = {"planes": np.int8, "windows": np.uint32, "perms": np.uint32, "srp_rowptr": np.uint32,
                "srp_idx": np.uint32, "srp_coef": np.int8}
        for k, dt in spec.items():
            if k in params and params[k] is not None:
                a = np.ascontiguousarray(params[k], dtype=dt)
                keep.append(a)
                setattr(hp, k, a.ctypes.data)
    return hp, keep


# ---------------------------------------------------------------------------
# Hash families
# ---------------------------------------------------------------------------
class HashFamily:
    """trait HashFamily (hash/mod.rs:24-39), batched on the GPU."""

    def __init__(self, kind, input_dim: int, k: int, num_tables: int, window_size: int = 8,
                 params: dict | None = None, seed: int | None = None, srp_sparsity: float = 1.0 / 3.0,
                 ctx: Context | None = None):
        self.ctx = ctx or default_context()
        self.lib = self.ctx.lib
        self.kind = HashFunctionType(kind)
        self._k, self._d, self._L = k, input_dim, num_tables
        self.window_size = min(window_size, input_dim)
        h = C.c_void_p()
        if params is not None:
            hp, keep = hash_params_c(params)
            st = self.lib.kl_hash_create(self.ctx.h, int(self.kind), input_dim, k, num_tables, self.window_size,
                                         C.byref(hp), C.byref(h))
        else:
            st = self.lib.kl_hash_create_seeded(self.ctx.h, int(self.kind), input_dim, k, num_tables,
                                                self.window_size, srp_sparsity, seed or 0, C.byref(h))
        check(st, self.ctx.h, "kl_hash_create")
        self.h = h
        self.params = params

    def __del__(self):
        if getattr(self, "h", None):
            self.lib.kl_hash_destroy(self.h)

    def k(self) -> int:
        return self._k

    def input_dim(self) -> int:
        return self._d

    def num_tables(self) -> int:
        return self._L

    def hash_dense_batch(self, X: torch.Tensor, with_min_abs: bool = False):
        X = X.to(device=f"cuda:{self.ctx.device}", dtype=torch.float32).contiguous()
        n = X.shape[0]
        codes = torch.empty((n, self._L), dtype=torch.int64, device=X.device)
        mn = torch.empty((n, self._L), dtype=torch.float32, device=X.device) if with_min_abs else None
        check(self.lib.kl_hash_dense_batch(self.h, _ptr(X), n, X.shape[1] if n else self._d, _ptr(codes), _ptr(mn)),
              self.ctx.h, "kl_hash_dense_batch")
        return (codes, mn) if with_min_abs else codes

    def hash_rows(self, rows: torch.Tensor, with_min_abs: bool = False):
        """kl_hash_dense_batch_rows: rows kept in their storage type (bf16 or f32)."""
        rows = torch.as_tensor(rows).to(f"cuda:{self.ctx.device}")
        dt = _lib.DTYPE_BF16 if rows.dtype == torch.bfloat16 else _lib.DTYPE_F32
        rows = (rows if dt == _lib.DTYPE_BF16 else rows.float()).contiguous()
        n = rows.shape[0]
        codes = torch.empty((n, self._L), dtype=torch.int64, device=rows.device)
        mn = torch.empty((n, self._L), dtype=torch.float32, device=rows.device) if with_min_abs else None
        check(self.lib.kl_hash_dense_batch_rows(self.h, _ptr(rows), n, rows.shape[1] if n else self._d, dt,
                                                _ptr(codes), _ptr(mn)), self.ctx.h, "kl_hash_dense_batch_rows")
        return (codes, mn) if with_min_abs else codes

    def set_projection(self, mode: int) -> None:
        """_lib.PROJ_AUTO / PROJ_SEQUENTIAL / PROJ_TENSOR (kl_hash_set_projection)."""
        check(self.lib.kl_hash_set_projection(self.h, int(mode)), self.ctx.h, "kl_hash_set_projection")

    def hash_sparse_batch(self, rowptr, idx, val, with_min_abs: bool = False):
        dev = f"cuda:{self.ctx.device}"
        rowptr = torch.as_tensor(rowptr, dtype=torch.int32).to(dev)
        idx = torch.as_tensor(np.asarray(idx, np.uint32).view(np.int32)).to(dev)
        val = torch.as_tensor(val, dtype=torch.float32).to(dev)
        n = rowptr.numel() - 1
        codes = torch.empty((n, self._L), dtype=torch.int64, device=dev)
        mn = torch.empty((n, self._L), dtype=torch.float32, device=dev) if with_min_abs else None
        check(self.lib.kl_hash_sparse_batch(self.h, _ptr(rowptr), _ptr(idx), _ptr(val), n, _ptr(codes), _ptr(mn)),
              self.ctx.h, "kl_hash_sparse_batch")
        return (codes, mn) if with_min_abs else codes

    def hash_dense(self, x, table: int) -> int:  # hash/mod.rs:26
        return int(self.hash_dense_batch(torch.as_tensor(np.asarray(x, np.float32))[None])[0, table].item()) \
            & 0xFFFFFFFFFFFFFFFF

    def hash_sparse(self, v: SparseVector, table: int) -> int:  # hash/mod.rs:29
        c = self.hash_sparse_batch(np.array([0, len(v.indices)], np.int32), v.indices, v.values)
        return int(c[0, table].item()) & 0xFFFFFFFFFFFFFFFF


def SimHash(input_dim, k, num_tables, seed=None, planes=None, ctx=None):  # simhash.rs:37
    return HashFamily(HashFunctionType.SimHash, input_dim, k, num_tables, params=None if planes is None else
                      {"planes": planes}, seed=seed, ctx=ctx)


def DwtaHash(input_dim, k, num_tables, window_size, seed=None, windows=None, ctx=None):  # dwta.rs:39
    return HashFamily(HashFunctionType.DwtaHash, input_dim, k, num_tables, window_size,
                      params=None if windows is None else {"windows": windows}, seed=seed, ctx=ctx)


def WtaHash(input_dim, k, num_tables, window_size, seed=None, windows=None, ctx=None):  # wta.rs:42
    return HashFamily(HashFunctionType.WtaHash, input_dim, k, num_tables, window_size,
                      params=None if windows is None else {"windows": windows}, seed=seed, ctx=ctx)


def MinHash(input_dim, k, num_tables, seed=None, perms=None, ctx=None):  # minhash.rs:38
    return HashFamily(HashFunctionType.MinHash, input_dim, k, num_tables,
                      params=None if perms is None else {"perms": perms}, seed=seed, ctx=ctx)


def SparseRandomProjection(input_dim, k, num_tables, sparsity=1.0 / 3.0, seed=None, projections=None, ctx=None):
    return HashFamily(HashFunctionType.SparseRandomProjection, input_dim, k, num_tables, params=projections,
                      seed=seed, srp_sparsity=sparsity, ctx=ctx)


# ---------------------------------------------------------------------------
# LSH index
# ---------------------------------------------------------------------------
@dataclass
class LshCandidate:  # lsh/mod.rs:10-14
    neuron_id: int
    count: int


class LshIndex:
    """LshIndex<H> behind trait LshIndexTrait (lsh/index.rs:21-316)."""

    def __init__(self, hash_family: HashFamily, bucket_type=BucketType.Fifo, bucket_capacity: int = 128,
                 _handle=None):
        self.hash = hash_family
        self.ctx = hash_family.ctx if hash_family is not None else None
        self.lib = _lib.load()
        self._owned = _handle is None
        if _handle is None:
            h = C.c_void_p()
            check(self.lib.kl_index_create(self.ctx.h, hash_family.h, int(bucket_type), bucket_capacity, C.byref(h)),
                  self.ctx.h, "kl_index_create")
            self.h = h
        else:
            self.h = _handle
        L, nb, cap, bt = C.c_int(), C.c_int(), C.c_int(), C.c_int()
        check(self.lib.kl_index_info(self.h, C.byref(L), C.byref(nb), C.byref(cap), C.byref(bt)))
        self.L, self.nb, self.cap, self.bucket_type = L.value, nb.value, cap.value, bt.value

    def __del__(self):
        if getattr(self, "_owned", False) and getattr(self, "h", None):
            self.lib.kl_index_destroy(self.h)

    @property
    def _dev(self) -> str:
        return f"cuda:{self.ctx.device}"

    def _ids(self, ids) -> torch.Tensor:
        return torch.as_tensor(np.asarray(ids, dtype=np.uint32).view(np.int32)).to(self._dev)

    # -- mutation ---------------------------------------------------------
    def insert_batch(self, ids, rows: torch.Tensor) -> None:
        rows = torch.as_tensor(rows).to(self._dev)
        dt = _lib.DTYPE_BF16 if rows.dtype == torch.bfloat16 else _lib.DTYPE_F32
        if dt == _lib.DTYPE_F32:
            rows = rows.float()
        rows = rows.contiguous()
        ids_t = self._ids(ids)
        check(self.lib.kl_index_insert_batch(self.h, _ptr(ids_t), _ptr(rows), rows.shape[0], rows.shape[1], dt),
              self.ctx.h, "kl_index_insert_batch")

    def insert(self, id: int, dense_weights) -> None:  # index.rs:257-262
        self.insert_batch([id], torch.as_tensor(np.asarray(dense_weights, np.float32))[None])

    def insert_sparse(self, id: int, weights: SparseVector) -> None:  # index.rs:264-269
        rp = torch.tensor([0, len(weights.indices)], dtype=torch.int32, device=self._dev)
        ix = torch.as_tensor(np.asarray(weights.indices, np.uint32).view(np.int32)).to(self._dev)
        vv = torch.as_tensor(np.asarray(weights.values, np.float32)).to(self._dev)
        check(self.lib.kl_index_insert_sparse_batch(self.h, _ptr(self._ids([id])), _ptr(rp), _ptr(ix), _ptr(vv), 1),
              self.ctx.h, "kl_index_insert_sparse_batch")

    def remove_with_weights(self, id: int, dense_weights) -> None:  # index.rs:271-276
        rows = torch.as_tensor(np.asarray(dense_weights, np.float32))[None].to(self._dev)
        check(self.lib.kl_index_remove_with_weights(self.h, _ptr(self._ids([id])), _ptr(rows), 1, rows.shape[1],
                                                    _lib.DTYPE_F32), self.ctx.h, "kl_index_remove_with_weights")

    def remove(self, id: int) -> None:  # index.rs:278-280
        check(self.lib.kl_index_remove(self.h, _ptr(self._ids([id])), 1), self.ctx.h, "kl_index_remove")

    def rebuild(self, neurons) -> None:  # index.rs:302-307: [(id, weights)]
        if len(neurons) == 0:
            check(self.lib.kl_index_clear(self.h), self.ctx.h, "kl_index_clear")
            return
        ids = [i for i, _ in neurons]
        rows = torch.as_tensor(np.stack([np.asarray(w, np.float32) for _, w in neurons])).to(self._dev)
        check(self.lib.kl_index_rebuild(self.h, _ptr(self._ids(ids)), _ptr(rows), rows.shape[0], rows.shape[1],
                                        _lib.DTYPE_F32), self.ctx.h, "kl_index_rebuild")

    def rebuild_rows(self, rows: torch.Tensor) -> None:
        """rebuild with ids 0..n-1 (Layer::rebuild_index, layer.rs:228-233)."""
        rows = torch.as_tensor(rows).to(self._dev)
        dt = _lib.DTYPE_BF16 if rows.dtype == torch.bfloat16 else _lib.DTYPE_F32
        rows = (rows if dt == _lib.DTYPE_BF16 else rows.float()).contiguous()
        check(self.lib.kl_index_rebuild(self.h, None, _ptr(rows), rows.shape[0], rows.shape[1], dt),
              self.ctx.h, "kl_index_rebuild")

    def set_projection(self, mode: int) -> None:
        check(self.lib.kl_index_set_projection(self.h, int(mode)), self.ctx.h, "kl_index_set_projection")

    def clear(self) -> None:  # index.rs:313-315
        check(self.lib.kl_index_clear(self.h), self.ctx.h, "kl_index_clear")

    def num_tables(self) -> int:
        return self.L

    # -- queries ----------------------------------------------------------
    def query_batch(self, X, mode=_lib.QUERY_COUNTS, capacity: int | None = None):
        """Batched query: (offsets[n+1], ids, counts) device tensors, ids sorted per query."""
        X = torch.as_tensor(X).to(self._dev, torch.float32).contiguous()
        n = X.shape[0]
        cap = capacity if capacity is not None else max(1, n * self.L * self.cap)
        ids = torch.empty(cap, dtype=torch.int32, device=self._dev)
        cnt = torch.empty(cap, dtype=torch.int32, device=self._dev)
        offs = torch.empty(n + 1, dtype=torch.int32, device=self._dev)
        ovf = torch.zeros(1, dtype=torch.int32, device=self._dev)
        check(self.lib.kl_index_query_batch(self.h, _ptr(X), n, X.shape[1] if n else 0, mode, _ptr(ids), _ptr(cnt),
                                            _ptr(offs), cap, _ptr(ovf)), self.ctx.h, "kl_index_query_batch")
        return offs, ids, cnt

    def query_sparse_batch(self, rowptr, idx, val, mode=_lib.QUERY_COUNTS, capacity: int | None = None):
        rp = torch.as_tensor(np.asarray(rowptr, np.int32)).to(self._dev)
        ix = torch.as_tensor(np.asarray(idx, np.uint32).view(np.int32)).to(self._dev)
        vv = torch.as_tensor(np.asarray(val, np.float32)).to(self._dev)
        n = rp.numel() - 1
        cap = capacity if capacity is not None else max(1, n * self.L * self.cap)
        ids = torch.empty(cap, dtype=torch.int32, device=self._dev)
        cnt = torch.empty(cap, dtype=torch.int32, device=self._dev)
        offs = torch.empty(n + 1, dtype=torch.int32, device=self._dev)
        ovf = torch.zeros(1, dtype=torch.int32, device=self._dev)
        check(self.lib.kl_index_query_sparse_batch(self.h, _ptr(rp), _ptr(ix), _ptr(vv), n, mode, _ptr(ids),
                                                   _ptr(cnt), _ptr(offs), cap, _ptr(ovf)),
              self.ctx.h, "kl_index_query_sparse_batch")
        return offs, ids, cnt

    def _one(self, res, counts: bool):
        offs, ids, cnt = (t.cpu().numpy() for t in res)
        a, b = int(offs[0]), int(offs[1])
        if counts:
            return [LshCandidate(int(i) & 0xFFFFFFFF, int(c)) for i, c in zip(ids[a:b], cnt[a:b])]
        return [int(i) & 0xFFFFFFFF for i in ids[a:b]]

    def query(self, x):  # index.rs:282-284
        return self._one(self.query_batch(np.asarray(x, np.float32)[None]), True)

    def query_with_counts(self, x):  # index.rs:290-292
        return self.query(x)

    def query_union(self, x):  # index.rs:286-288
        return self._one(self.query_batch(np.asarray(x, np.float32)[None], _lib.QUERY_UNION), False)

    def query_sparse_union(self, v: SparseVector):  # index.rs:294-296
        return self._one(self.query_sparse_batch([0, len(v.indices)], v.indices, v.values, _lib.QUERY_UNION), False)

    def query_sparse_with_counts(self, v: SparseVector):  # index.rs:298-300
        return self._one(self.query_sparse_batch([0, len(v.indices)], v.indices, v.values), True)

    def export(self):
        """(ids[L][nb][cap], lens[L][nb], counts[L][nb]) as numpy."""
        ids = torch.empty(self.L * self.nb * self.cap, dtype=torch.int32, device=self._dev)
        lens = torch.empty(self.L * self.nb, dtype=torch.int32, device=self._dev)
        cnt = torch.empty(self.L * self.nb, dtype=torch.int64, device=self._dev)
        check(self.lib.kl_index_export(self.h, _ptr(ids), _ptr(lens), _ptr(cnt)), self.ctx.h, "kl_index_export")
        self.ctx.sync()
        return (ids.cpu().numpy().view(np.uint32).reshape(self.L, self.nb, self.cap),
                lens.cpu().numpy().view(np.uint32).reshape(self.L, self.nb),
                cnt.cpu().numpy().view(np.uint64).reshape(self.L, self.nb))

    def bucket_contents(self, table: int, bucket: int) -> list[int]:
        ids, lens, _ = self.export()
        return [int(v) for v in ids[table, bucket, :lens[table, bucket]]]


def create_lsh_index(config: LshConfig, input_dim: int, seed: int, ctx: Context | None = None) -> LshIndex:
    """Factory of lsh/index.rs:339-374 (window 8 for WTA/DWTA, SRP density 1/3)."""
    hf = HashFamily(config.hash_function, input_dim, config.num_hashes, config.num_tables,
                    window_size=min(8, input_dim), seed=seed, ctx=ctx)
    return LshIndex(hf, config.bucket_type, config.bucket_capacity)


# ---------------------------------------------------------------------------
# Network
# ---------------------------------------------------------------------------
class AdaptiveScheduler:
    """klearu_mongoose::AdaptiveScheduler (scheduler.rs:44-213): rebuild the
    LSH tables when the hash codes of sampled neurons have drifted.  Rows are
    a device tensor [n][d] (f32 or bf16); the drift check runs on the GPU."""

    def __init__(self, min_interval: int, max_interval: int, sample_fraction: float, drift_threshold: float,
                 ctx: Context | None = None):
        self.ctx = ctx or default_context()
        self.lib = self.ctx.lib
        h = C.c_void_p()
        check(self.lib.kl_adaptive_create(self.ctx.h, int(min_interval), int(max_interval), float(sample_fraction),
                                          float(drift_threshold), C.byref(h)), self.ctx.h, "kl_adaptive_create")
        self.h = h

    def __del__(self):
        if getattr(self, "h", None):
            self.lib.kl_adaptive_destroy(self.h)

    @staticmethod
    def _rows(rows):
        dt = _lib.DTYPE_BF16 if rows.dtype == torch.bfloat16 else _lib.DTYPE_F32
        rows = (rows if dt == _lib.DTYPE_BF16 else rows.float()).contiguous()
        n = rows.shape[0]
        ld = rows.shape[1] if rows.dim() == 2 and n else 0
        return rows, n, ld, dt

    def record_baseline(self, rows: torch.Tensor, hash_fn: HashFamily, seed: int = 0, sampled=None) -> None:
        rows, n, ld, dt = self._rows(torch.as_tensor(rows).to(f"cuda:{self.ctx.device}"))
        idx = None if sampled is None else np.ascontiguousarray(np.asarray(sampled, np.uint32))
        check(self.lib.kl_adaptive_record_baseline(self.h, hash_fn.h, _ptr(rows) if n else None, n, ld, dt,
                                                   None if idx is None else idx.ctypes.data,
                                                   0 if idx is None else len(idx), int(seed)),
              self.ctx.h, "kl_adaptive_record_baseline")

    def should_rebuild(self, rows: torch.Tensor) -> bool:
        rows, n, ld, dt = self._rows(torch.as_tensor(rows).to(f"cuda:{self.ctx.device}"))
        out = C.c_int()
        check(self.lib.kl_adaptive_should_rebuild(self.h, _ptr(rows) if n else None, n, ld, dt, C.byref(out)),
              self.ctx.h, "kl_adaptive_should_rebuild")
        return bool(out.value)

    def notify_rebuild(self) -> None:
        check(self.lib.kl_adaptive_notify_rebuild(self.h))

    def _state(self):
        e, st, ns = C.c_float(), C.c_uint64(), C.c_int()
        check(self.lib.kl_adaptive_state(self.h, C.byref(e), C.byref(st), C.byref(ns)))
        return e.value, st.value, ns.value

    def drift_estimate(self) -> float:
        return self._state()[0]

    def steps_since_rebuild(self) -> int:
        return self._state()[1]

    def num_sampled(self) -> int:
        return self._state()[2]


@dataclass
class LayerOutput:  # network/layer.rs:19-26
    activations: np.ndarray
    active_neurons: list
    pre_activations: np.ndarray


class DeviceBatch:
    """A CSR batch resident on the device, with its kl_batch descriptor."""

    def __init__(self, hb: HostBatch, device: str, pinned: bool = False):
        def up(a, dt):
            t = torch.from_numpy(np.ascontiguousarray(a).view(dt))
            if pinned:
                t = t.pin_memory()
            return t.to(device, non_blocking=pinned)

        self.host = hb
        self.rowptr = up(hb.rowptr, np.int32)
        self.idx = up(hb.idx.astype(np.uint32), np.int32)
        self.val = up(hb.val.astype(np.float32), np.float32)
        self.label_ptr = up(hb.label_ptr, np.int32)
        self.labels = up(hb.labels.astype(np.uint32), np.int32)
        self.c = _lib.BatchC(hb.batch, _ptr(self.rowptr), _ptr(self.idx), _ptr(self.val), _ptr(self.label_ptr),
                             _ptr(self.labels), int(hb.rowptr[-1]), int(hb.label_ptr[-1]))


class Network:
    """klearu_core::network::Network (net.rs:10-173) on one B200.

    ``init``: optional list (one per layer) of dicts with ``weights`` [N][d]
    f32, ``bias`` [N] and hash parameter arrays (see params.hash_params).
    """

    def __init__(self, config: SlideConfig, init=None, weight_dtype: str = "f32", max_batch: int = 256,
                 ctx: Context | None = None, shard: tuple[bytes, int, int] | None = None,
                 dense_update_max_bytes: int = 0):
        """``shard=(unique_id, rank, nranks)`` builds this rank's part of a
        neuron-sharded network (kl_net_create_sharded); ``unique_id`` comes from
        klearu_b200.dist.share_unique_id.  ``dense_update_max_bytes`` bounds the
        output update's gradient matrix (0: 2 GiB; negative: always the
        segmented update)."""
        self.ctx = ctx or default_context()
        self.lib = self.ctx.lib
        self.config = config
        self.max_batch = max_batch
        self.weight_dtype = _lib.DTYPE_BF16 if weight_dtype == "bf16" else _lib.DTYPE_F32
        cfg, keep_cfg = config.to_c(self.weight_dtype, max_batch)
        cfg.dense_update_max_bytes = int(dense_update_max_bytes)
        keep = [keep_cfg]
        init_arr = None
        if init is not None:
            init_arr = (_lib.LayerInitC * len(init))()
            for i, li in enumerate(init):
                w = li.get("weights")
                b = li.get("bias")
                if w is not None:
                    w = np.ascontiguousarray(w, np.float32)
                    keep.append(w)
                    init_arr[i].weights = w.ctypes.data
                if b is not None:
                    b = np.ascontiguousarray(b, np.float32)
                    keep.append(b)
                    init_arr[i].bias = b.ctypes.data
                hp, k2 = hash_params_c(li)
                keep.append(k2)
                init_arr[i].hash = hp
        h = C.c_void_p()
        if shard is None:
            check(self.lib.kl_net_create(self.ctx.h, C.byref(cfg), init_arr, C.byref(h)), self.ctx.h,
                  "kl_net_create")
        else:
            uid, rank, nranks = shard
            idbuf = C.create_string_buffer(bytes(uid), len(uid))
            check(self.lib.kl_net_create_sharded(self.ctx.h, C.byref(cfg), init_arr, idbuf, int(rank), int(nranks),
                                                 C.byref(h)), self.ctx.h, "kl_net_create_sharded")
        self.h = h
        self.num_layers = len(config.network.layers)

    def __del__(self):
        if getattr(self, "h", None):
            self.lib.kl_net_destroy(self.h)

    @property
    def _dev(self) -> str:
        return f"cuda:{self.ctx.device}"

    def owned_features(self) -> tuple[int, int]:
        """(first, count): the hidden layer's feature rows whose Adam moments this rank updates."""
        f, n = C.c_uint32(), C.c_uint32()
        check(self.lib.kl_net_owned_features(self.h, C.byref(f), C.byref(n)))
        return f.value, n.value

    def shard_info(self) -> tuple[int, int, int, int]:
        """(rank, nranks, global id of the first local output neuron, local output neurons)."""
        r, n, nl = C.c_int(), C.c_int(), C.c_int()
        base = C.c_uint32()
        check(self.lib.kl_net_shard_info(self.h, C.byref(r), C.byref(n), C.byref(base), C.byref(nl)))
        return r.value, n.value, base.value, nl.value

    # -- failure detection of a sharded network ----------------------------
    def set_comm_timeout(self, timeout_ms: int) -> None:
        """Bound every wait that depends on other ranks by ``timeout_ms``
        (0: plain blocking waits).  A wait that runs out raises KL_ETIMEOUT, a
        communicator error KL_ENCCL; both abort the communicator."""
        check(self.lib.kl_net_set_comm_timeout(self.h, int(timeout_ms)), self.ctx.h, "kl_net_set_comm_timeout")

    def sync(self) -> None:
        """Wait for this network's queued work and report device faults."""
        check(self.lib.kl_net_sync(self.h), self.ctx.h, "kl_net_sync")

    def comm_abort(self) -> None:
        """Abort the communicator (a peer rank is known to be gone)."""
        check(self.lib.kl_net_comm_abort(self.h), self.ctx.h, "kl_net_comm_abort")

    @property
    def step(self) -> int:
        s, n, c = C.c_uint64(), C.c_uint64(), C.c_uint64()
        check(self.lib.kl_net_get_step(self.h, C.byref(s), C.byref(n), C.byref(c)))
        return s.value

    def scheduler_state(self) -> tuple[int, int, int]:
        s, n, c = C.c_uint64(), C.c_uint64(), C.c_uint64()
        check(self.lib.kl_net_get_step(self.h, C.byref(s), C.byref(n), C.byref(c)))
        return s.value, n.value, c.value

    def device_batch(self, examples_or_batch, pinned: bool = False) -> DeviceBatch:
        hb = examples_or_batch if isinstance(examples_or_batch, HostBatch) else HostBatch.from_examples(
            examples_or_batch)
        return DeviceBatch(hb, self._dev, pinned)

    # -- training ---------------------------------------------------------
    def train_step_device(self, db: DeviceBatch, lr: float, mode=_lib.MODE_BATCHED, loss: torch.Tensor | None = None):
        check(self.lib.kl_net_train_step(self.h, C.byref(db.c), float(lr), mode, _ptr(loss), None),
              self.ctx.h, "kl_net_train_step")

    def train_step(self, examples, lr: float, mode: str = "exact") -> float:  # net.rs:81-119
        if len(examples) == 0:
            return 0.0
        db = self.device_batch(examples)
        out = C.c_float()
        m = _lib.MODE_EXACT_SEQUENTIAL if mode == "exact" else _lib.MODE_BATCHED
        check(self.lib.kl_net_train_step(self.h, C.byref(db.c), float(lr), m, None, C.byref(out)),
              self.ctx.h, "kl_net_train_step")
        return out.value

    def train_step_host(self, hb: HostBatch, lr: float, mode=_lib.MODE_BATCHED, loss_out=None) -> float | None:
        """One train step on a host CSR batch through kl_net_train_step_host.

        With ``loss_out`` None the call waits for the step and returns the mean
        loss.  Otherwise ``loss_out`` is a 1-element pinned float32 CPU tensor
        that receives the loss in stream order (valid after ``sync()``), and
        the call returns None without waiting, so consecutive calls overlap the
        next batch's upload with the current step."""
        arrs = [np.ascontiguousarray(getattr(hb, k)) for k in ("rowptr", "idx", "val", "label_ptr", "labels")]
        rp, idx, val, lp, lab = arrs
        c = _lib.BatchC(hb.batch, rp.ctypes.data, idx.ctypes.data, val.ctypes.data, lp.ctypes.data,
                        lab.ctypes.data, int(rp[-1]) if hb.batch else 0, int(lp[-1]) if hb.batch else 0)
        if loss_out is None:
            out = torch.zeros(1, dtype=torch.float32).pin_memory()
            check(self.lib.kl_net_train_step_host(self.h, C.byref(c), float(lr), mode, out.data_ptr()),
                  self.ctx.h, "kl_net_train_step_host")
            self.sync()
            return float(out[0])
        check(self.lib.kl_net_train_step_host(self.h, C.byref(c), float(lr), mode, loss_out.data_ptr()),
              self.ctx.h, "kl_net_train_step_host")
        return None

    def train_step_batch_host(self, b, lr: float, mode=_lib.MODE_BATCHED, loss_out=None) -> float | None:
        """kl_net_train_step_host on a kl_batch of host arrays (for example one
        drawn from data.BatchIterator); same waiting rules as train_step_host."""
        if loss_out is None:
            out = torch.zeros(1, dtype=torch.float32).pin_memory()
            check(self.lib.kl_net_train_step_host(self.h, C.byref(b), float(lr), mode, out.data_ptr()),
                  self.ctx.h, "kl_net_train_step_host")
            self.sync()
            return float(out[0])
        check(self.lib.kl_net_train_step_host(self.h, C.byref(b), float(lr), mode, loss_out.data_ptr()),
              self.ctx.h, "kl_net_train_step_host")
        return None

    def train_epoch(self, it, lr: float, mode=_lib.MODE_BATCHED) -> list[float]:
        """One pass over a data.BatchIterator: each batch goes to
        kl_net_train_step_host without waiting (the iterator's worker assembles
        the next batch and the library uploads it while this one trains); the
        per-batch losses are read after the last step."""
        n = 0
        outs = []
        for b in it:
            if n == len(outs):
                outs.append(torch.zeros(1, dtype=torch.float32).pin_memory())
            self.train_step_batch_host(b, lr, mode, loss_out=outs[n])
            # the iterator reuses its buffers two draws later; the library copied them at the call
            n += 1
        self.sync()
        return [float(o[0]) for o in outs[:n]]

    # -- inference --------------------------------------------------------
    def forward_batch(self, examples) -> list[list[LayerOutput]]:
        """Network::forward (net.rs:62-78) for every example: [example][layer]."""
        db = self.device_batch(examples)
        check(self.lib.kl_net_forward(self.h, C.byref(db.c)), self.ctx.h, "kl_net_forward")
        per_layer = [self.layer_output(l, db.host.batch) for l in range(self.num_layers)]
        res = []
        for s in range(db.host.batch):
            outs = []
            for l in range(self.num_layers):
                ids, pre, act, N = per_layer[l]
                dense = np.zeros(N, np.float32)
                dense[ids[s]] = act[s]
                outs.append(LayerOutput(dense, list(ids[s]), pre[s]))
            res.append(outs)
        return res

    def layer_output(self, layer: int, nq: int):
        d, N, ma = C.c_int(), C.c_int(), C.c_int()
        check(self.lib.kl_net_layer_info(self.h, layer, C.byref(d), C.byref(N), C.byref(ma)))
        stride = ma.value
        rows = self.max_batch * self.shard_info()[1]  # a sharded net's outputs cover the global batch
        ids = torch.empty(rows * stride, dtype=torch.int32, device=self._dev)
        cnt = torch.empty(rows, dtype=torch.int32, device=self._dev)
        pre = torch.empty(rows * stride, dtype=torch.float32, device=self._dev)
        act = torch.empty(rows * stride, dtype=torch.float32, device=self._dev)
        check(self.lib.kl_net_layer_output(self.h, layer, _ptr(ids), _ptr(cnt), _ptr(pre), _ptr(act)),
              self.ctx.h, "kl_net_layer_output")
        self.sync()
        ids = ids.cpu().numpy().view(np.uint32).reshape(rows, stride)
        pre = pre.cpu().numpy().reshape(rows, stride)
        act = act.cpu().numpy().reshape(rows, stride)
        cnt = cnt.cpu().numpy()
        return ([ids[s, :cnt[s]] for s in range(nq)], [pre[s, :cnt[s]] for s in range(nq)],
                [act[s, :cnt[s]] for s in range(nq)], N.value)

    def forward(self, x) -> list[LayerOutput]:  # net.rs:62-78, one dense input
        return self.forward_batch([Example.new(x, [])])[0]

    def predict(self, x) -> np.ndarray:  # net.rs:151-154
        return self.forward(x)[-1].activations

    def predict_top_k_batch(self, examples, k: int):
        db = self.device_batch(examples)
        N = self.config.network.layers[-1].num_neurons
        k = min(k, N)
        ids = torch.empty((db.host.batch, k), dtype=torch.int32, device=self._dev)
        sc = torch.empty((db.host.batch, k), dtype=torch.float32, device=self._dev)
        check(self.lib.kl_net_predict_topk(self.h, C.byref(db.c), k, _ptr(ids), _ptr(sc)), self.ctx.h,
              "kl_net_predict_topk")
        self.sync()
        return ids.cpu().numpy().view(np.uint32), sc.cpu().numpy()

    def predict_top_k(self, x, k: int):  # net.rs:159-173
        ids, sc = self.predict_top_k_batch([Example.new(x, [])], k)
        return [(int(i), float(s)) for i, s in zip(ids[0], sc[0])]

    # -- state ------------------------------------------------------------
    def get_layer(self, layer: int) -> dict:
        """Parameters and optimizer state of `layer` (a sharded output layer: this rank's slice)."""
        dd, nn, ma = C.c_int(), C.c_int(), C.c_int()
        check(self.lib.kl_net_layer_info(self.h, layer, C.byref(dd), C.byref(nn), C.byref(ma)), self.ctx.h)
        N, d = nn.value, dd.value
        out = {k: np.empty((N, d), np.float32) for k in ("weights", "m", "v")}
        out.update({k: np.empty(N, np.float32) for k in ("bias", "mb", "vb")})
        check(self.lib.kl_net_get_layer(self.h, layer, *(out[k].ctypes.data for k in
                                                         ("weights", "bias", "m", "v", "mb", "vb"))),
              self.ctx.h, "kl_net_get_layer")
        return out

    def set_layer(self, layer: int, **arrays) -> None:
        ptrs = []
        keep = []
        for k in ("weights", "bias", "m", "v", "mb", "vb"):
            a = arrays.get(k)
            if a is None:
                ptrs.append(None)
            else:
                a = np.ascontiguousarray(a, np.float32)
                keep.append(a)
                ptrs.append(a.ctypes.data)
        check(self.lib.kl_net_set_layer(self.h, layer, *ptrs), self.ctx.h, "kl_net_set_layer")

    def layer_index(self, layer: int) -> LshIndex:
        h = C.c_void_p()
        check(self.lib.kl_net_layer_index(self.h, layer, C.byref(h)))
        ix = LshIndex.__new__(LshIndex)
        ix.hash = None
        ix.ctx = self.ctx
        ix.lib = self.lib
        ix._owned = False
        ix.h = h
        L, nb, cap, bt = C.c_int(), C.c_int(), C.c_int(), C.c_int()
        check(self.lib.kl_index_info(h, C.byref(L), C.byref(nb), C.byref(cap), C.byref(bt)))
        ix.L, ix.nb, ix.cap, ix.bucket_type = L.value, nb.value, cap.value, bt.value
        return ix

    def rebuild(self) -> None:
        check(self.lib.kl_net_rebuild(self.h), self.ctx.h, "kl_net_rebuild")

    def set_rebuild_policy(self, adaptive: bool, min_interval: int = 10, max_interval: int = 1000,
                           sample_fraction: float = 0.05, drift_threshold: float = 0.1, seed: int = 0) -> None:
        """The reference's RebuildScheduler (adaptive=False) or one mongoose
        AdaptiveScheduler per layer (crates/klearu-mongoose/src/scheduler.rs)."""
        p = _lib.RebuildPolicyC(_lib.REBUILD_ADAPTIVE if adaptive else _lib.REBUILD_SCHEDULE, int(min_interval),
                                int(max_interval), float(sample_fraction), float(drift_threshold), int(seed))
        check(self.lib.kl_net_set_rebuild_policy(self.h, C.byref(p)), self.ctx.h, "kl_net_set_rebuild_policy")

    def rebuild_state(self, layer: int) -> tuple[float, int, int]:
        """(drift EMA, steps since the layer's last rebuild, its rebuild count)."""
        e, s, r = C.c_float(), C.c_uint64(), C.c_uint64()
        check(self.lib.kl_net_rebuild_state(self.h, layer, C.byref(e), C.byref(s), C.byref(r)), self.ctx.h,
              "kl_net_rebuild_state")
        return e.value, s.value, r.value

    def save(self, path) -> None:
        """Checkpoint every train-step state array (kl_net_save)."""
        check(self.lib.kl_net_save(self.h, str(path).encode()), self.ctx.h, "kl_net_save")

    def load(self, path) -> None:
        """Restore a checkpoint written by save() from a network of the same configuration."""
        check(self.lib.kl_net_load(self.h, str(path).encode()), self.ctx.h, "kl_net_load")

    def profile(self, enable: bool) -> None:
        check(self.lib.kl_net_profile(self.h, int(enable)), self.ctx.h, "kl_net_profile")

    def profile_read(self, layer: int, reset: bool = True) -> dict:
        ms = (C.c_double * len(_lib.PHASES))()
        calls = (C.c_uint64 * len(_lib.PHASES))()
        check(self.lib.kl_net_profile_read(self.h, layer, ms, calls, int(reset)), self.ctx.h, "kl_net_profile_read")
        return {p: (ms[i], calls[i]) for i, p in enumerate(_lib.PHASES)}

    def stats(self, layer: int, reset: bool = False) -> _lib.LayerStatsC:
        s = _lib.LayerStatsC()
        check(self.lib.kl_net_stats(self.h, layer, C.byref(s), int(reset)), self.ctx.h, "kl_net_stats")
        return s
