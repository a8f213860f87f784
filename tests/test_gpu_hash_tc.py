"""The tensor-core SimHash / SRP projection (hash_tc.cu) against the CPU oracle.

Products of bf16 rows and ternary planes are exact; only the f32 accumulation
order differs from the reference's sequential sums, so a code may differ only
in a table where some projection is within NEAR_ZERO of zero (those are
counted and printed).  Table contents after a rebuild must then be identical
except in the buckets such a row moved between.
"""

import numpy as np
import pytest
import torch

from klearu_b200 import _lib
from klearu_b200 import params as P
from klearu_b200.config import BucketType, HashFunctionType as HF
from klearu_b200.core import HashFamily, LshIndex

pytestmark = pytest.mark.gpu

NEAR_ZERO = 1e-5


def _rows(n, d, seed):
    x = np.random.default_rng(seed).standard_normal((n, d)).astype(np.float32)
    x /= np.linalg.norm(x, axis=1, keepdims=True)
    xb = torch.from_numpy(x).to(torch.bfloat16)
    return xb, xb.float().numpy()


@pytest.mark.parametrize("kind,d,K,L,n", [
    (HF.SimHash, 128, 6, 50, 20000),    # the LSH microbench's SimHash shape
    (HF.SimHash, 256, 9, 50, 9000),     # the 3.1M-way output layer's shape
    (HF.SimHash, 96, 5, 7, 5000),       # one table group, d not a multiple of 64
    (HF.SparseRandomProjection, 200, 8, 40, 6000),
])
def test_tensor_core_codes_match_oracle(gpu_ctx, orc, kind, d, K, L, n):
    prm = P.hash_params(kind, np.random.default_rng(d), d, K, L)
    g = HashFamily(kind, d, K, L, 8, params=prm, ctx=gpu_ctx)
    o = orc.Hash(kind, d, K, L, 8, prm)
    xb, xf = _rows(n, d, d + 1)
    xb[7] = 0.0  # a zero row: every bit set, as the reference's `>= 0` test gives
    xf[7] = 0.0
    g.set_projection(_lib.PROJ_TENSOR)
    gc, gm = g.hash_rows(xb, with_min_abs=True)
    g.set_projection(_lib.PROJ_SEQUENTIAL)
    sc = g.hash_rows(xb).cpu().numpy().view(np.uint64)
    oc, om = o.dense(xf, with_min_abs=True)
    gc = gc.cpu().numpy().view(np.uint64)
    assert (sc == oc).all()  # the sequential path is the reference's bit for bit
    assert (gc[7] == (1 << K) - 1).all()
    bad = gc != oc
    near = om < NEAR_ZERO
    print(f"tensor-core codes differing from the reference: {int(bad.sum())} of {bad.size}, "
          f"all with |projection| < {NEAR_ZERO}: {bool((~near[bad]).sum() == 0)}")
    assert not (bad & ~near).any(), f"{int((bad & ~near).sum())} codes differ away from zero"
    assert np.allclose(gm.cpu().numpy(), om, rtol=1e-3, atol=1e-6)


@pytest.mark.parametrize("bucket", [BucketType.Fifo, BucketType.Reservoir])
def test_tensor_core_rebuild_tables(gpu_ctx, orc, bucket):
    d, K, L, n, cap = 128, 6, 50, 30000, 128
    prm = P.hash_params(HF.SimHash, np.random.default_rng(5), d, K, L)
    g = HashFamily(HF.SimHash, d, K, L, 8, params=prm, ctx=gpu_ctx)
    ix = LshIndex(g, bucket, cap)
    ix.set_projection(_lib.PROJ_AUTO)  # n >= 4096 bf16 rows: the tensor cores
    xb, xf = _rows(n, d, 6)
    ix.rebuild_rows(xb)
    gi, gl, gc = ix.export()
    oh = orc.Hash(HF.SimHash, d, K, L, 8, prm)
    oi = orc.Index(oh, int(bucket), cap)
    oi.insert(np.arange(n, dtype=np.uint32), xf)
    ti, tl, tc = oi.export()
    # buckets a sign-flipped row moved between are excused
    g.set_projection(_lib.PROJ_TENSOR)
    tcc = g.hash_rows(xb).cpu().numpy().view(np.uint64)
    occ = oh.dense(xf)
    mask = (1 << K) - 1
    excused = np.zeros((L, 1 << K), bool)
    for r, t in zip(*np.nonzero(tcc != occ)):
        excused[t, int(tcc[r, t]) & mask] = True
        excused[t, int(occ[r, t]) & mask] = True
    print(f"buckets excused: {int(excused.sum())} of {excused.size}")
    same = (gl == tl) & (gc == tc) & (gi == ti).all(axis=2)
    assert (same | excused).all()
