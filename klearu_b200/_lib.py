"""ctypes binding of ``include/klearu_gpu.h`` (libklearu_gpu.so).

This is the Python twin of the Rust FFI crate a maintainer would write: one
``argtypes``/``restype`` line per exported symbol and ``ctypes.Structure``
mirrors of the ``#[repr(C)]`` structs.  Loading fails loudly if the library is
missing -- there is no fallback implementation.
"""

from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libklearu_gpu.so"

# enums (config.rs:3-38 order)
KL_OK, KL_EINVAL, KL_ENOMEM, KL_ECUDA, KL_ENCCL, KL_ETIMEOUT, KL_EBOUNDS, KL_ECAPACITY, KL_EUNSUPPORTED = range(9)
STATUS_NAMES = ["KL_OK", "KL_EINVAL", "KL_ENOMEM", "KL_ECUDA", "KL_ENCCL", "KL_ETIMEOUT", "KL_EBOUNDS",
                "KL_ECAPACITY", "KL_EUNSUPPORTED"]
HASH_SIMHASH, HASH_WTA, HASH_DWTA, HASH_MINHASH, HASH_SRP = range(5)
BUCKET_FIFO, BUCKET_RESERVOIR = range(2)
SAMPLING_VANILLA, SAMPLING_TOPK, SAMPLING_THRESHOLD = range(3)
ACT_RELU, ACT_SIGMOID, ACT_TANH, ACT_SOFTMAX, ACT_IDENTITY = range(5)
OPT_SGD, OPT_ADAM = range(2)
DTYPE_F32, DTYPE_BF16 = range(2)
QUERY_COUNTS, QUERY_UNION = range(2)
MODE_EXACT_SEQUENTIAL, MODE_BATCHED = range(2)
PROJ_AUTO, PROJ_SEQUENTIAL, PROJ_TENSOR = 0, 1, 2
PHASES = ["hash", "probe", "forward", "backward", "update", "rebuild", "stream"]


class HashParams(C.Structure):
    _fields_ = [("planes", C.c_void_p), ("windows", C.c_void_p), ("perms", C.c_void_p),
                ("srp_rowptr", C.c_void_p), ("srp_idx", C.c_void_p), ("srp_coef", C.c_void_p)]


class LshConfigC(C.Structure):
    _fields_ = [("hash_function", C.c_int32), ("bucket_type", C.c_int32), ("num_tables", C.c_int32),
                ("range_pow", C.c_int32), ("num_hashes", C.c_int32), ("bucket_capacity", C.c_int32),
                ("rebuild_interval_base", C.c_int32), ("rebuild_decay", C.c_double)]


class LayerConfigC(C.Structure):
    _fields_ = [("input_dim", C.c_int32), ("num_neurons", C.c_int32), ("activation", C.c_int32),
                ("lsh", LshConfigC), ("sampling", C.c_int32), ("sampling_threshold", C.c_int32),
                ("top_k", C.c_int32), ("is_output", C.c_int32)]


class NetConfigC(C.Structure):
    _fields_ = [("num_layers", C.c_int32), ("layers", C.POINTER(LayerConfigC)), ("optimizer", C.c_int32),
                ("learning_rate", C.c_double), ("batch_size", C.c_int32), ("num_threads", C.c_int32),
                ("seed", C.c_uint64), ("weight_dtype", C.c_int32), ("max_batch", C.c_int32),
                ("dense_update_max_bytes", C.c_int64)]


class LayerInitC(C.Structure):
    _fields_ = [("weights", C.c_void_p), ("bias", C.c_void_p), ("hash", HashParams)]


class BatchC(C.Structure):
    _fields_ = [("batch", C.c_int32), ("rowptr", C.c_void_p), ("idx", C.c_void_p), ("val", C.c_void_p),
                ("label_ptr", C.c_void_p), ("labels", C.c_void_p), ("nnz", C.c_int32), ("nlabels", C.c_int32)]


class RebuildPolicyC(C.Structure):
    _fields_ = [("kind", C.c_int32), ("min_interval", C.c_uint64), ("max_interval", C.c_uint64),
                ("sample_fraction", C.c_float), ("drift_threshold", C.c_float), ("seed", C.c_uint64)]


REBUILD_SCHEDULE, REBUILD_ADAPTIVE = 0, 1


class LayerStatsC(C.Structure):
    _fields_ = [("active_sum", C.c_uint64), ("touched_rows", C.c_uint64), ("input_nnz", C.c_uint64),
                ("examples", C.c_uint64), ("steps", C.c_uint64), ("rebuilds", C.c_uint64)]


_H = C.c_void_p  # opaque handles
_P = C.c_void_p
_S = C.c_int     # kl_status

_PROTOS = {
    "kl_abi_version": (C.c_int, []),
    "kl_ctx_create": (_S, [C.c_int, _P, C.POINTER(_H)]),
    "kl_ctx_destroy": (_S, [_H]),
    "kl_ctx_set_stream": (_S, [_H, _P]),
    "kl_ctx_sync": (_S, [_H]),
    "kl_ctx_check": (_S, [_H]),
    "kl_last_error": (C.c_char_p, [_H]),
    "kl_hash_create": (_S, [_H, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(HashParams), C.POINTER(_H)]),
    "kl_hash_create_seeded": (_S, [_H, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float, C.c_uint64,
                                   C.POINTER(_H)]),
    "kl_hash_destroy": (_S, [_H]),
    "kl_hash_info": (_S, [_H, C.POINTER(C.c_int), C.POINTER(C.c_int), C.POINTER(C.c_int), C.POINTER(C.c_int)]),
    "kl_hash_set_projection": (_S, [_H, C.c_int]),
    "kl_hash_dense_batch_rows": (_S, [_H, _P, C.c_int, C.c_int, C.c_int, _P, _P]),
    "kl_index_set_projection": (_S, [_H, C.c_int]),
    "kl_hash_dense_batch": (_S, [_H, _P, C.c_int, C.c_int, _P, _P]),
    "kl_hash_sparse_batch": (_S, [_H, _P, _P, _P, C.c_int, _P, _P]),
    "kl_index_create": (_S, [_H, _H, C.c_int, C.c_int, C.POINTER(_H)]),
    "kl_index_destroy": (_S, [_H]),
    "kl_index_info": (_S, [_H, C.POINTER(C.c_int), C.POINTER(C.c_int), C.POINTER(C.c_int), C.POINTER(C.c_int)]),
    "kl_index_insert_batch": (_S, [_H, _P, _P, C.c_int, C.c_int, C.c_int]),
    "kl_index_insert_sparse_batch": (_S, [_H, _P, _P, _P, _P, C.c_int]),
    "kl_index_remove": (_S, [_H, _P, C.c_int]),
    "kl_index_remove_with_weights": (_S, [_H, _P, _P, C.c_int, C.c_int, C.c_int]),
    "kl_index_rebuild": (_S, [_H, _P, _P, C.c_int, C.c_int, C.c_int]),
    "kl_index_clear": (_S, [_H]),
    "kl_index_query_batch": (_S, [_H, _P, C.c_int, C.c_int, C.c_int, _P, _P, _P, C.c_int32, _P]),
    "kl_index_query_batch_noalloc": (_S, [_H, _P, C.c_int, C.c_int, C.c_int, _P, _P, _P, C.c_int32, _P]),
    "kl_index_query_sparse_batch": (_S, [_H, _P, _P, _P, C.c_int, C.c_int, _P, _P, _P, C.c_int32, _P]),
    "kl_bolt_infer_batch": (_S, [_H, _P, C.c_int, C.c_int, _P, C.c_int, _P, C.c_int, C.c_int, C.c_float, C.c_int,
                                 C.c_int, _P, _P, _P, C.c_int]),
    "kl_net_bolt_infer": (_S, [_H, C.c_int, _P, C.c_int, C.c_int, C.c_float, C.c_int, C.c_int, _P, _P, _P, C.c_int]),
    "kl_index_export": (_S, [_H, _P, _P, _P]),
    "kl_index_import": (_S, [_H, _P, _P, _P]),
    "kl_net_create": (_S, [_H, C.POINTER(NetConfigC), _P, C.POINTER(_H)]),
    "kl_net_destroy": (_S, [_H]),
    "kl_net_train_step": (_S, [_H, C.POINTER(BatchC), C.c_double, C.c_int, _P, C.POINTER(C.c_float)]),
    "kl_net_train_step_host": (_S, [_H, C.POINTER(BatchC), C.c_double, C.c_int, _P]),
    "kl_net_forward": (_S, [_H, C.POINTER(BatchC)]),
    "kl_net_layer_output": (_S, [_H, C.c_int, _P, _P, _P, _P]),
    "kl_net_layer_info": (_S, [_H, C.c_int, C.POINTER(C.c_int), C.POINTER(C.c_int), C.POINTER(C.c_int)]),
    "kl_net_predict_topk": (_S, [_H, C.POINTER(BatchC), C.c_int, _P, _P]),
    "kl_net_get_layer": (_S, [_H, C.c_int, _P, _P, _P, _P, _P, _P]),
    "kl_net_set_layer": (_S, [_H, C.c_int, _P, _P, _P, _P, _P, _P]),
    "kl_net_rebuild": (_S, [_H]),
    "kl_net_layer_index": (_S, [_H, C.c_int, C.POINTER(_H)]),
    "kl_net_get_step": (_S, [_H, C.POINTER(C.c_uint64), C.POINTER(C.c_uint64), C.POINTER(C.c_uint64)]),
    "kl_net_set_step": (_S, [_H, C.c_uint64, C.c_uint64, C.c_uint64]),
    "kl_net_set_rebuild_policy": (_S, [_H, C.POINTER(RebuildPolicyC)]),
    "kl_net_rebuild_state": (_S, [_H, C.c_int, C.POINTER(C.c_float), C.POINTER(C.c_uint64), C.POINTER(C.c_uint64)]),
    "kl_net_save": (_S, [_H, C.c_char_p]),
    "kl_net_load": (_S, [_H, C.c_char_p]),
    "kl_net_stats": (_S, [_H, C.c_int, C.POINTER(LayerStatsC), C.c_int]),
    "kl_net_profile": (_S, [_H, C.c_int]),
    "kl_net_profile_read": (_S, [_H, C.c_int, _P, _P, C.c_int]),
    "kl_launch_count": (_S, [C.POINTER(C.c_uint64)]),
    "kl_alloc_count": (_S, [C.POINTER(C.c_uint64)]),
    "kl_dist_unique_id_size": (C.c_int, []),
    "kl_dist_get_unique_id": (_S, [_P]),
    "kl_net_create_sharded": (_S, [_H, C.POINTER(NetConfigC), _P, _P, C.c_int, C.c_int, C.POINTER(_H)]),
    "kl_net_shard_info": (_S, [_H, _P, _P, _P, _P]),
    "kl_net_owned_features": (_S, [_H, _P, _P]),
    "kl_net_set_comm_timeout": (_S, [_H, C.c_int]),
    "kl_net_sync": (_S, [_H]),
    "kl_net_comm_abort": (_S, [_H]),
    "kl_adaptive_create": (_S, [_H, C.c_uint64, C.c_uint64, C.c_float, C.c_float, C.POINTER(_H)]),
    "kl_predictor_create": (_S, [_H, C.c_int, C.c_int, C.c_int, _P, _P, _P, _P, C.POINTER(_H)]),
    "kl_predictor_destroy": (_S, [_H]),
    "kl_predictor_info": (_S, [_H, C.POINTER(C.c_int), C.POINTER(C.c_int), C.POINTER(C.c_int)]),
    "kl_predictor_predict": (_S, [_H, _P, C.c_int, _P]),
    "kl_predictor_select_topk": (_S, [_H, _P, C.c_int, C.c_int, _P, _P]),
    "kl_sparse_mlp_create": (_S, [_H, C.c_int, C.c_int, _P, _P, _P, _P, C.POINTER(_H)]),
    "kl_sparse_mlp_destroy": (_S, [_H]),
    "kl_sparse_mlp_forward": (_S, [_H, _P, C.c_int, _P, C.c_int, _P]),
    "kl_adaptive_destroy": (_S, [_H]),
    "kl_adaptive_record_baseline": (_S, [_H, _H, _P, C.c_int, C.c_int, C.c_int, _P, C.c_int, C.c_uint64]),
    "kl_adaptive_should_rebuild": (_S, [_H, _P, C.c_int, C.c_int, C.c_int, C.POINTER(C.c_int)]),
    "kl_adaptive_notify_rebuild": (_S, [_H]),
    "kl_adaptive_state": (_S, [_H, _P, _P, _P]),
    "kl_ffn_stack_create": (_S, [_H, C.c_int, _P, _P, _P, C.c_float, C.c_int, C.POINTER(_H)]),
    "kl_ffn_stack_destroy": (_S, [_H]),
    "kl_ffn_stack_decode": (_S, [_H, _P, C.c_int, C.c_float]),
    "kl_libsvm_load": (_S, [C.c_char_p, C.c_int64, C.c_int64, C.c_int, C.POINTER(_H)]),
    "kl_libsvm_parse": (_S, [C.c_char_p, C.c_size_t, C.c_int64, C.c_int64, C.c_int, C.POINTER(_H)]),
    "kl_dataset_from_csr": (_S, [_P, _P, _P, _P, _P, C.c_int64, C.c_int64, C.c_int64, C.POINTER(_H)]),
    "kl_dataset_destroy": (_S, [_H]),
    "kl_dataset_info": (_S, [_H, _P, _P, _P, _P, _P]),
    "kl_dataset_csr": (_S, [_H, _P, _P, _P, _P, _P]),
    "kl_batch_iter_create": (_S, [_H, C.c_int, C.c_uint64, C.c_int, C.POINTER(_H)]),
    "kl_batch_iter_reset": (_S, [_H, C.c_uint64]),
    "kl_batch_iter_next": (_S, [_H, C.POINTER(BatchC)]),
    "kl_batch_iter_destroy": (_S, [_H]),
}

_lib = None


def load(path: str | os.PathLike | None = None) -> C.CDLL:
    """Load libklearu_gpu.so and attach prototypes.  Raises if it is absent."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise ImportError(f"{p} is missing: build it with `python -m klearu_b200.build`")
    lib = C.CDLL(str(p))
    for name, (res, args) in _PROTOS.items():
        f = getattr(lib, name)
        f.restype = res
        f.argtypes = args
    if path is None:
        _lib = lib
    return lib


def exported_symbols() -> list[str]:
    return list(_PROTOS)


class KlError(RuntimeError):
    def __init__(self, status: int, msg: str):
        self.status = status
        name = STATUS_NAMES[status] if 0 <= status < len(STATUS_NAMES) else str(status)
        super().__init__(f"{name}: {msg}")


def check(status: int, ctx=None, what: str = "") -> None:
    if status != KL_OK:
        msg = ""
        if ctx is not None:
            raw = load().kl_last_error(ctx)
            msg = raw.decode() if raw else ""
        raise KlError(status, f"{what}: {msg}" if what else msg)
