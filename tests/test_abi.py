"""The C-ABI library loads and exports every entry point include/klearu_gpu.h
declares.  Host-only calls (no device work) check argument validation."""

import ctypes as C
import re
from pathlib import Path

from klearu_b200 import _lib

ROOT = Path(__file__).resolve().parent.parent


def declared_symbols():
    text = (ROOT / "include" / "klearu_gpu.h").read_text()
    return sorted(set(re.findall(r"^KL_API\s+[\w\s\*]+?\b(kl_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert len(syms) >= 40
    assert "kl_net_train_step" in syms and "kl_index_query_batch" in syms


def test_library_exports_every_declared_symbol():
    lib = C.CDLL(str(_lib.LIB_PATH))
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, missing


def test_binding_covers_header():
    assert sorted(_lib.exported_symbols()) == declared_symbols()


def test_abi_version_and_null_handles():
    lib = _lib.load()
    assert lib.kl_abi_version() == 2
    assert lib.kl_ctx_destroy(None) == _lib.KL_EINVAL
    assert lib.kl_hash_destroy(None) == _lib.KL_EINVAL
    assert lib.kl_index_destroy(None) == _lib.KL_EINVAL
    assert lib.kl_net_destroy(None) == _lib.KL_EINVAL
    assert lib.kl_net_train_step(None, None, 0.1, 0, None, None) == _lib.KL_EINVAL
    assert lib.kl_net_set_comm_timeout(None, 1000) == _lib.KL_EINVAL
    assert lib.kl_net_sync(None) == _lib.KL_EINVAL
    assert lib.kl_net_comm_abort(None) == _lib.KL_EINVAL
    assert isinstance(lib.kl_last_error(None), bytes)  # this thread's last error (context-free calls)


def test_library_is_sm100a_only():
    # the engine is compiled for sm_100a only (no multi-arch fallback)
    from klearu_b200.build import NVCC_FLAGS

    assert "arch=compute_100a,code=sm_100a" in NVCC_FLAGS
    assert not any("sm_90" in f or "sm_80" in f for f in NVCC_FLAGS)
