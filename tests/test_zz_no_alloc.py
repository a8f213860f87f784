"""kl_index_query_batch_noalloc: the index query for callers that cannot call
cudaMalloc.

Such callers own all device memory themselves: a host runtime with its own
allocator, or a process whose GPU memory budget is fixed at start-up.  The
entry point takes its scratch from a fixed array compiled into the library
instead of allocating it.  These tests call it through the C ABI and check it
against kl_index_query_batch, which allocates its scratch.  Ids and counts are
integers, so the results must be identical.  They are checked on two calls in a
row, because the second call reuses scratch that the first call left behind.

This file is named to be collected last, so a failure here comes after every
other test has run.
"""

import ctypes as C

import numpy as np
import pytest
import torch

from klearu_b200 import _lib
from klearu_b200 import params as P
from klearu_b200.config import BucketType, HashFunctionType as HF
from klearu_b200.core import HashFamily, LshIndex

pytestmark = pytest.mark.gpu

SCRATCH_BYTES = 16 << 20  # KL_NOALLOC_SCRATCH_BYTES in include/klearu_gpu.h


def _index(ctx, kind, d, K, L, cap, bucket, n_rows, seed):
    rng = np.random.default_rng(seed)
    prm = P.hash_params(kind, rng, d, K, L)
    ix = LshIndex(HashFamily(kind, d, K, L, params=prm, ctx=ctx), bucket, cap)
    rows = rng.standard_normal((n_rows, d)).astype(np.float32)
    ix.rebuild_rows(torch.from_numpy(rows))
    return ix, rows, rng


def _query(ix, entry, X, mode):
    lib = ix.lib
    X = X.contiguous()
    n = X.shape[0]
    cap = max(1, n * ix.L * ix.cap)
    ids = torch.full((cap,), -1, dtype=torch.int32, device=X.device)
    cnt = torch.full((cap,), -1, dtype=torch.int32, device=X.device)
    offs = torch.empty(n + 1, dtype=torch.int32, device=X.device)
    ovf = torch.zeros(1, dtype=torch.int32, device=X.device)
    st = getattr(lib, entry)(ix.h, C.c_void_p(X.data_ptr()), n, X.shape[1], mode, C.c_void_p(ids.data_ptr()),
                             C.c_void_p(cnt.data_ptr()), C.c_void_p(offs.data_ptr()), cap,
                             C.c_void_p(ovf.data_ptr()))
    _lib.check(st, ix.ctx.h, entry)
    ix.ctx.sync()
    tot = int(offs[-1])
    return offs.cpu().numpy(), ids[:tot].cpu().numpy(), cnt[:tot].cpu().numpy(), int(ovf.item())


@pytest.mark.parametrize("kind,bucket", [(HF.DwtaHash, BucketType.Fifo), (HF.SimHash, BucketType.Reservoir)])
def test_noalloc_query_matches_allocating_query(gpu_ctx, kind, bucket):
    ix, rows, rng = _index(gpu_ctx, kind, 96, 6, 20, 32, bucket, 5000, 11)
    dev = f"cuda:{gpu_ctx.device}"
    for call in range(2):  # two calls in a row: the second reuses the first call's scratch
        n = 300 if call == 0 else 117
        near = rows[rng.integers(0, len(rows), n // 2)] + 0.05 * rng.standard_normal((n // 2, 96)).astype(np.float32)
        X = torch.from_numpy(np.concatenate([near, rng.standard_normal((n - n // 2, 96)).astype(np.float32)]))
        X = X.to(dev)
        for mode in (_lib.QUERY_COUNTS, _lib.QUERY_UNION):
            a = _query(ix, "kl_index_query_batch", X, mode)
            b = _query(ix, "kl_index_query_batch_noalloc", X, mode)
            assert (a[0] == b[0]).all(), "offsets differ"
            assert (a[1] == b[1]).all(), "ids differ"
            if mode == _lib.QUERY_COUNTS:
                assert (a[2] == b[2]).all(), "counts differ"
            assert a[3] == b[3] == 0
            assert a[0][-1] > 0


def test_noalloc_query_allocates_no_device_memory(gpu_ctx):
    ix, rows, rng = _index(gpu_ctx, HF.DwtaHash, 64, 8, 10, 64, BucketType.Fifo, 3000, 12)
    X = torch.from_numpy(rows[:200].copy()).to(f"cuda:{gpu_ctx.device}")
    # outputs are allocated by the caller before the calls
    n, cap = X.shape[0], X.shape[0] * ix.L * ix.cap
    ids = torch.empty(cap, dtype=torch.int32, device=X.device)
    cnt = torch.empty(cap, dtype=torch.int32, device=X.device)
    offs = torch.empty(n + 1, dtype=torch.int32, device=X.device)

    def call():
        _lib.check(ix.lib.kl_index_query_batch_noalloc(ix.h, C.c_void_p(X.data_ptr()), n, X.shape[1],
                                                       _lib.QUERY_COUNTS, C.c_void_p(ids.data_ptr()),
                                                       C.c_void_p(cnt.data_ptr()), C.c_void_p(offs.data_ptr()),
                                                       cap, None), ix.ctx.h)
        ix.ctx.sync()

    def allocs():
        n = C.c_uint64()
        _lib.check(ix.lib.kl_alloc_count(C.byref(n)))
        return n.value

    call()  # first call on the device: symbol address lookup and lazy kernel loading
    a0 = allocs()
    free0 = torch.cuda.mem_get_info(gpu_ctx.device)[0]
    call()
    call()
    # the library's own allocation counter is exact; free device memory is a coarser second check
    assert allocs() == a0
    assert torch.cuda.mem_get_info(gpu_ctx.device)[0] == free0
    # self-queries find their own id in every table
    o = offs.cpu().numpy()
    got = ids.cpu().numpy()
    c = cnt.cpu().numpy()
    for q in range(0, n, 37):
        seg = got[o[q]:o[q + 1]]
        assert q in seg and c[o[q] + int(np.searchsorted(seg, q))] == ix.L


def test_noalloc_query_rejects_batches_beyond_scratch(gpu_ctx):
    ix, rows, _ = _index(gpu_ctx, HF.DwtaHash, 32, 8, 50, 128, BucketType.Fifo, 100, 13)
    per_query = 50 * 128 * 8
    n = SCRATCH_BYTES // per_query + 1
    X = torch.zeros((n, 32), dtype=torch.float32, device=f"cuda:{gpu_ctx.device}")
    st = ix.lib.kl_index_query_batch_noalloc(ix.h, C.c_void_p(X.data_ptr()), n, 32, _lib.QUERY_UNION, None, None,
                                             C.c_void_p(X.data_ptr()), 0, None)
    assert st == 7  # KL_ECAPACITY, nothing launched
    assert b"KL_NOALLOC_SCRATCH_BYTES" in ix.lib.kl_last_error(ix.ctx.h)
