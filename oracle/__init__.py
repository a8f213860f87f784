"""CPU oracle of klearu-core's SLIDE path -- TEST INFRASTRUCTURE ONLY.

ctypes wrapper over ``oracle/liboracle.so`` (built from ``oracle/oracle.cpp``
by ``oracle/build.py``).  Only ``tests/``, ``__graft_entry__.smoke()`` and the
CPU-baseline leg of ``bench.py`` use it, as the checker; the product path
(``klearu_b200``) never imports it.

Parity pinning: the restatement is checked against the reference's own unit
tests (known-answer values ported in tests/test_oracle_kat.py).  The
reference's seeded parameter streams (rand 0.8.5 ChaCha12) are not available,
so seeded construction is parity-unpinned; parameters are explicit inputs.
"""

from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"
_lib = None

_P = C.c_void_p


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            from .build import build_oracle

            build_oracle()
        L = C.CDLL(str(LIB_PATH))
        protos = {
            "orc_siphash13_usize2": (C.c_uint64, [C.c_uint64, C.c_uint64]),
            "orc_powi_f32": (C.c_float, [C.c_float, C.c_int]),
            "orc_f32_to_bf16": (C.c_uint16, [C.c_float]),
            "orc_splitmix_mod": (C.c_uint64, [C.c_uint64, C.c_uint64]),
            "orc_hash_create": (_P, [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, _P]),
            "orc_hash_destroy": (None, [_P]),
            "orc_hash_dense": (None, [_P, _P, C.c_int, C.c_int, _P, _P]),
            "orc_hash_sparse": (None, [_P, _P, _P, _P, C.c_int, _P, _P]),
            "orc_bucket_create": (_P, [C.c_int, C.c_int]),
            "orc_bucket_destroy": (None, [_P]),
            "orc_bucket_insert": (None, [_P, C.c_uint32]),
            "orc_bucket_remove": (C.c_int, [_P, C.c_uint32]),
            "orc_bucket_clear": (None, [_P]),
            "orc_bucket_contents": (C.c_int, [_P, _P]),
            "orc_bucket_total": (C.c_uint64, [_P]),
            "orc_index_create": (_P, [_P, C.c_int, C.c_int]),
            "orc_index_destroy": (None, [_P]),
            "orc_index_insert": (None, [_P, _P, _P, C.c_int, C.c_int]),
            "orc_index_insert_sparse": (None, [_P, _P, _P, _P, _P, C.c_int]),
            "orc_index_remove": (None, [_P, _P, C.c_int]),
            "orc_index_remove_with_weights": (None, [_P, _P, _P, C.c_int, C.c_int]),
            "orc_index_clear": (None, [_P]),
            "orc_index_query": (C.c_int, [_P, _P, _P, _P, C.c_int]),
            "orc_index_query_sparse": (C.c_int, [_P, _P, _P, C.c_int, _P, _P, C.c_int]),
            "orc_index_export": (None, [_P, _P, _P, _P]),
            "orc_sample": (C.c_int, [C.c_int, C.c_int, C.c_int, _P, _P, C.c_int, _P]),
            "orc_adaptive_create": (_P, [C.c_uint64, C.c_uint64, C.c_float, C.c_float]),
            "orc_pred_predict": (None, [_P, _P, _P, _P, C.c_int, C.c_int, C.c_int, _P, C.c_int, _P]),
            "orc_pred_topk": (C.c_int, [_P, C.c_int, C.c_int, _P]),
            "orc_sparse_mlp": (None, [_P, _P, _P, _P, C.c_int, C.c_int, _P, _P, C.c_int, _P]),
            "orc_adaptive_destroy": (None, [_P]),
            "orc_adaptive_record_baseline": (None, [_P, _P, _P, C.c_int, C.c_int, _P, C.c_int]),
            "orc_adaptive_should_rebuild": (C.c_int, [_P, _P, _P, C.c_int, C.c_int]),
            "orc_adaptive_notify_rebuild": (None, [_P]),
            "orc_adaptive_drift": (C.c_float, [_P]),
            "orc_adaptive_steps": (C.c_uint64, [_P]),
            "orc_sched_create": (_P, [C.c_uint64, C.c_double]),
            "orc_sched_destroy": (None, [_P]),
            "orc_sched_should_rebuild": (C.c_int, [_P, C.c_uint64]),
            "orc_sched_next": (C.c_uint64, [_P]),
            "orc_sched_count": (C.c_uint64, [_P]),
            "orc_compute_loss": (C.c_float, [_P, C.c_int, _P, C.c_int, _P, C.c_int]),
            "orc_compute_loss_gradient": (None, [_P, C.c_int, _P, C.c_int, _P, C.c_int, _P]),
            "orc_optimizer_update": (None, [C.c_int, _P, _P, C.c_int, _P, C.c_float, C.c_double, C.c_uint64,
                                            _P, _P, _P, _P, C.c_float]),
            "orc_net_create": (_P, [_P, _P, C.c_int, C.c_int]),
            "orc_net_destroy": (None, [_P]),
            "orc_net_train_step": (C.c_float, [_P, _P, _P, _P, _P, _P, C.c_int, C.c_double, C.c_int]),
            "orc_net_train_hogwild": (C.c_float, [_P, _P, _P, _P, _P, _P, C.c_int, C.c_double, C.c_int]),
            "orc_net_forward": (None, [_P, _P, _P, C.c_int]),
            "orc_net_output": (C.c_int, [C.c_int, _P, _P, _P, C.c_int]),
            "orc_net_get_layer": (None, [_P, C.c_int, _P, _P, _P, _P, _P, _P]),
            "orc_net_step": (C.c_uint64, [_P]),
            "orc_net_next_rebuild": (C.c_uint64, [_P]),
            "orc_net_rebuild": (None, [_P]),
            "orc_net_export_index": (None, [_P, C.c_int, C.c_int, _P, _P, _P]),
        }
        for name, (res, args) in protos.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def _p(a):
    return None if a is None or a.size == 0 else a.ctypes.data


def _hash_params(params: dict):
    import sys

    sys.path.insert(0, str(HERE.parent))
    from klearu_b200._lib import HashParams

    hp = HashParams()
    keep = []
    spec = {"planes": np.int8, "windows": np.uint32, "perms": np.uint32, "srp_rowptr": np.uint32,
            "srp_idx": np.uint32, "srp_coef": np.int8}
    for k, dt in spec.items():
        if params.get(k) is not None:
            a = np.ascontiguousarray(params[k], dtype=dt)
            keep.append(a)
            setattr(hp, k, a.ctypes.data if a.size else None)
    return hp, keep


class Hash:
    def __init__(self, kind: int, d: int, k: int, L: int, w: int, params: dict):
        self.kind, self.d, self.k, self.L, self.w = int(kind), d, k, L, min(w, d)
        hp, self._keep = _hash_params(params)
        self.h = lib().orc_hash_create(self.kind, d, k, L, self.w, C.byref(hp))

    def __del__(self):
        if getattr(self, "h", None):
            lib().orc_hash_destroy(self.h)

    def dense(self, X: np.ndarray, with_min_abs=False):
        X = np.ascontiguousarray(X, np.float32)
        n = X.shape[0]
        codes = np.zeros((n, self.L), np.uint64)
        mn = np.zeros((n, self.L), np.float32) if with_min_abs else None
        lib().orc_hash_dense(self.h, _p(X), n, X.shape[1], _p(codes), _p(mn))
        return (codes, mn) if with_min_abs else codes

    def sparse(self, rowptr, idx, val, with_min_abs=False):
        rowptr = np.ascontiguousarray(rowptr, np.int32)
        idx = np.ascontiguousarray(idx, np.uint32)
        val = np.ascontiguousarray(val, np.float32)
        n = len(rowptr) - 1
        codes = np.zeros((n, self.L), np.uint64)
        mn = np.zeros((n, self.L), np.float32) if with_min_abs else None
        lib().orc_hash_sparse(self.h, _p(rowptr), _p(idx), _p(val), n, _p(codes), _p(mn))
        return (codes, mn) if with_min_abs else codes


class Bucket:
    def __init__(self, bucket_type: int, cap: int):
        self.cap = cap
        self.h = lib().orc_bucket_create(int(bucket_type), cap)

    def __del__(self):
        if getattr(self, "h", None):
            lib().orc_bucket_destroy(self.h)

    def insert(self, id):
        lib().orc_bucket_insert(self.h, id)

    def remove(self, id) -> bool:
        return bool(lib().orc_bucket_remove(self.h, id))

    def clear(self):
        lib().orc_bucket_clear(self.h)

    def contents(self) -> list[int]:
        out = np.zeros(self.cap, np.uint32)
        n = lib().orc_bucket_contents(self.h, _p(out))
        return [int(v) for v in out[:n]]

    def total_insertions(self) -> int:
        return int(lib().orc_bucket_total(self.h))


class Index:
    def __init__(self, h: Hash, bucket_type: int, cap: int):
        self.hash = h
        self.L, self.nb, self.cap = h.L, 1 << h.k, cap
        self.h = lib().orc_index_create(h.h, int(bucket_type), cap)

    def __del__(self):
        if getattr(self, "h", None):
            lib().orc_index_destroy(self.h)

    def insert(self, ids, rows):
        ids = np.ascontiguousarray(ids, np.uint32)
        rows = np.ascontiguousarray(rows, np.float32)
        lib().orc_index_insert(self.h, _p(ids), _p(rows), len(ids), rows.shape[1] if rows.ndim > 1 else 0)

    def insert_sparse(self, ids, rowptr, idx, val):
        ids = np.ascontiguousarray(ids, np.uint32)
        rowptr, idx, val = (np.ascontiguousarray(a, t) for a, t in ((rowptr, np.int32), (idx, np.uint32),
                                                                       (val, np.float32)))
        lib().orc_index_insert_sparse(self.h, _p(ids), _p(rowptr), _p(idx), _p(val), len(ids))

    def remove(self, ids):
        ids = np.ascontiguousarray(ids, np.uint32)
        lib().orc_index_remove(self.h, _p(ids), len(ids))

    def remove_with_weights(self, ids, rows):
        ids = np.ascontiguousarray(ids, np.uint32)
        rows = np.ascontiguousarray(rows, np.float32)
        lib().orc_index_remove_with_weights(self.h, _p(ids), _p(rows), len(ids), rows.shape[1])

    def clear(self):
        lib().orc_index_clear(self.h)

    def query(self, x):
        x = np.ascontiguousarray(x, np.float32)
        cap = self.L * self.cap
        ids = np.zeros(cap, np.uint32)
        cnt = np.zeros(cap, np.uint32)
        n = lib().orc_index_query(self.h, _p(x), _p(ids), _p(cnt), cap)
        return ids[:n].copy(), cnt[:n].copy()

    def query_sparse(self, idx, val):
        idx = np.ascontiguousarray(idx, np.uint32)
        val = np.ascontiguousarray(val, np.float32)
        cap = self.L * self.cap
        ids = np.zeros(cap, np.uint32)
        cnt = np.zeros(cap, np.uint32)
        n = lib().orc_index_query_sparse(self.h, _p(idx), _p(val), len(idx), _p(ids), _p(cnt), cap)
        return ids[:n].copy(), cnt[:n].copy()

    def export(self):
        ids = np.zeros((self.L, self.nb, self.cap), np.uint32)
        lens = np.zeros((self.L, self.nb), np.uint32)
        cnt = np.zeros((self.L, self.nb), np.uint64)
        lib().orc_index_export(self.h, _p(ids), _p(lens), _p(cnt))
        return ids, lens, cnt


def sample(sampling: int, top_k: int, threshold: int, ids, counts) -> list[int]:
    ids = np.ascontiguousarray(ids, np.uint32)
    counts = np.ascontiguousarray(counts, np.uint32)
    out = np.zeros(max(1, len(ids)), np.uint32)
    n = lib().orc_sample(int(sampling), top_k, threshold, _p(ids), _p(counts), len(ids), _p(out))
    return [int(v) for v in out[:n]]


class Scheduler:
    def __init__(self, base: int, decay: float):
        self.h = lib().orc_sched_create(base, decay)

    def __del__(self):
        if getattr(self, "h", None):
            lib().orc_sched_destroy(self.h)

    def should_rebuild(self, step: int) -> bool:
        return bool(lib().orc_sched_should_rebuild(self.h, step))

    def next_rebuild(self) -> int:
        return int(lib().orc_sched_next(self.h))

    def rebuild_count(self) -> int:
        return int(lib().orc_sched_count(self.h))


class AdaptiveScheduler:
    """mongoose AdaptiveScheduler (scheduler.rs:44-213) with explicit sampled indices."""

    def __init__(self, min_interval: int, max_interval: int, sample_fraction: float, drift_threshold: float):
        self.h = lib().orc_adaptive_create(min_interval, max_interval, sample_fraction, drift_threshold)

    def __del__(self):
        if getattr(self, "h", None):
            lib().orc_adaptive_destroy(self.h)

    def record_baseline(self, rows, hash_fn: Hash, sampled) -> None:
        rows = np.ascontiguousarray(rows, np.float32)
        idx = np.ascontiguousarray(np.sort(np.asarray(sampled, np.uint32)))
        self._keep = idx
        lib().orc_adaptive_record_baseline(self.h, hash_fn.h, _p(rows), rows.shape[0], rows.shape[1], _p(idx), len(idx))

    def should_rebuild(self, rows, hash_fn: Hash) -> bool:
        rows = np.ascontiguousarray(rows, np.float32)
        return bool(lib().orc_adaptive_should_rebuild(self.h, hash_fn.h, _p(rows), rows.shape[0], rows.shape[1]))

    def notify_rebuild(self) -> None:
        lib().orc_adaptive_notify_rebuild(self.h)

    def drift_estimate(self) -> float:
        return float(lib().orc_adaptive_drift(self.h))

    def steps_since_rebuild(self) -> int:
        return int(lib().orc_adaptive_steps(self.h))


def compute_loss(activations, active, labels) -> float:
    a = np.ascontiguousarray(activations, np.float32)
    ac = np.ascontiguousarray(active, np.uint32)
    lb = np.ascontiguousarray(labels, np.uint32)
    return float(lib().orc_compute_loss(_p(a), len(a), _p(ac), len(ac), _p(lb), len(lb)))


def compute_loss_gradient(activations, active, labels, num_output) -> np.ndarray:
    a = np.zeros(num_output, np.float32)
    a[: len(activations)] = activations
    ac = np.ascontiguousarray(active, np.uint32)
    lb = np.ascontiguousarray(labels, np.uint32)
    g = np.zeros(num_output, np.float32)
    lib().orc_compute_loss_gradient(_p(a), num_output, _p(ac), len(ac), _p(lb), len(lb), _p(g))
    return g


def optimizer_update(opt: int, w, g, bias, gb, lr, step, m, v, mb, vb, momentum: float = 0.9):
    """One Optimizer::update on a row; returns the new (w, bias, m, v, mb, vb)."""
    w = np.array(w, np.float32)
    g = np.ascontiguousarray(g, np.float32)
    m = np.array(m, np.float32)
    v = np.array(v, np.float32)
    b = np.array([bias], np.float32)
    mbb = np.array([mb], np.float32)
    vbb = np.array([vb], np.float32)
    lib().orc_optimizer_update(int(opt), _p(w), _p(g), len(w), _p(b), gb, lr, step, _p(m), _p(v), _p(mbb), _p(vbb),
                               momentum)
    return w, float(b[0]), m, v, float(mbb[0]), float(vbb[0])


class Net:
    """The oracle network.  cfg: klearu_b200.config.SlideConfig; init: list of
    per-layer dicts with weights [N][d], bias [N] and hash parameter arrays."""

    def __init__(self, cfg, init, weight_dtype: str = "f32", nshards: int = 1, sparse_input: bool = True):
        import sys

        sys.path.insert(0, str(HERE.parent))
        from klearu_b200._lib import DTYPE_BF16, DTYPE_F32, LayerInitC

        dt = DTYPE_BF16 if weight_dtype == "bf16" else DTYPE_F32
        self.cfg = cfg
        c, keep_cfg = cfg.to_c(dt, 1)
        self._keep = [keep_cfg]
        arr = (LayerInitC * len(init))()
        for i, li in enumerate(init):
            w = np.ascontiguousarray(li["weights"], np.float32)
            b = np.ascontiguousarray(li.get("bias", np.zeros(w.shape[0], np.float32)), np.float32)
            self._keep += [w, b]
            arr[i].weights = w.ctypes.data
            arr[i].bias = b.ctypes.data
            hp, k2 = _hash_params(li)
            self._keep.append(k2)
            arr[i].hash = hp
        self.h = lib().orc_net_create(C.byref(c), arr, nshards, int(sparse_input))
        self.layers = cfg.network.layers

    def __del__(self):
        if getattr(self, "h", None):
            lib().orc_net_destroy(self.h)

    @staticmethod
    def _b(hb):
        return (np.ascontiguousarray(hb.rowptr, np.int32), np.ascontiguousarray(hb.idx, np.uint32),
                np.ascontiguousarray(hb.val, np.float32), np.ascontiguousarray(hb.label_ptr, np.int32),
                np.ascontiguousarray(hb.labels, np.uint32))

    def train_step(self, hb, lr: float, mode: str = "exact") -> float:
        a = self._b(hb)
        return float(lib().orc_net_train_step(self.h, *(_p(x) for x in a), hb.batch, lr, 1 if mode == "batched" else 0))

    def train_hogwild(self, hb, lr: float, threads: int) -> float:
        a = self._b(hb)
        return float(lib().orc_net_train_hogwild(self.h, *(_p(x) for x in a), hb.batch, lr, threads))

    def forward(self, idx, val):
        """Per layer: (ids sorted, pre, act) of one example."""
        idx = np.ascontiguousarray(idx, np.uint32)
        val = np.ascontiguousarray(val, np.float32)
        lib().orc_net_forward(self.h, _p(idx), _p(val), len(idx))
        outs = []
        for l, lc in enumerate(self.layers):
            cap = lc.num_neurons
            ids = np.zeros(cap, np.uint32)
            pre = np.zeros(cap, np.float32)
            act = np.zeros(cap, np.float32)
            n = lib().orc_net_output(l, _p(ids), _p(pre), _p(act), cap)
            outs.append((ids[:n].copy(), pre[:n].copy(), act[:n].copy()))
        return outs

    def get_layer(self, l: int) -> dict:
        lc = self.layers[l]
        N, d = lc.num_neurons, lc.input_dim
        out = {k: np.zeros((N, d), np.float32) for k in ("weights", "m", "v")}
        out.update({k: np.zeros(N, np.float32) for k in ("bias", "mb", "vb")})
        lib().orc_net_get_layer(self.h, l, *(_p(out[k]) for k in ("weights", "bias", "m", "v", "mb", "vb")))
        return out

    @property
    def step(self) -> int:
        return int(lib().orc_net_step(self.h))

    def next_rebuild(self) -> int:
        return int(lib().orc_net_next_rebuild(self.h))

    def export_index(self, l: int, shard: int = 0):
        lc = self.layers[l]
        L, nb, cap = lc.lsh.num_tables, 1 << lc.lsh.num_hashes, lc.lsh.bucket_capacity
        ids = np.zeros((L, nb, cap), np.uint32)
        lens = np.zeros((L, nb), np.uint32)
        cnt = np.zeros((L, nb), np.uint64)
        lib().orc_net_export_index(self.h, l, shard, _p(ids), _p(lens), _p(cnt))
        return ids, lens, cnt


# ---- Deja Vu sparse FFN (oracle/dejavu.cpp) ----------------------------------

def pred_predict(w1, b1, w2, b2, x) -> np.ndarray:
    """SparsityPredictor::predict (mlp_predictor.rs:102-123) for each row of x."""
    w1, b1, w2, b2 = (np.ascontiguousarray(a, np.float32) for a in (w1, b1, w2, b2))
    x = np.ascontiguousarray(np.atleast_2d(x), np.float32)
    hid, d = w1.shape
    out = w2.shape[0]
    scores = np.empty((x.shape[0], out), np.float32)
    lib().orc_pred_predict(_p(w1), _p(b1), _p(w2), _p(b2), d, hid, out, _p(x), x.shape[0], _p(scores))
    return scores


def pred_topk(scores, k: int) -> np.ndarray:
    """select_top_k (mlp_predictor.rs:126-132) on one score vector."""
    scores = np.ascontiguousarray(scores, np.float32)
    idx = np.empty(min(k, scores.size), np.uint32)
    n = lib().orc_pred_topk(_p(scores), scores.size, k, _p(idx))
    return idx[:n]


def sparse_mlp(gate, up, down, bias, x, sel) -> np.ndarray:
    """forward_sparse (sparse_mlp.rs:4-37) for one token; bias may be None."""
    gate, up, down = (np.ascontiguousarray(a, np.float32) for a in (gate, up, down))
    inter, hid = gate.shape
    x = np.ascontiguousarray(x, np.float32)
    sel = np.ascontiguousarray(sel, np.uint32)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    out = np.empty(hid, np.float32)
    lib().orc_sparse_mlp(_p(gate), _p(up), _p(down), None if b is None else _p(b), hid, inter, _p(x), _p(sel),
                         sel.size, _p(out))
    return out
