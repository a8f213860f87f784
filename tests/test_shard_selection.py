"""The neuron-sharded output layer's global selection protocol, on CPU.

`csrc/shard.cu` selects TopK / Threshold over all shards without exchanging
candidate lists: each rank histograms its candidates' table counts per
example (`sel_hist_kernel`), the ranks sum the histograms, every rank derives
the same cut from the sum (`sel_cut_kernel`), and an all-gather of each
rank's number of candidates AT the cut tells a rank how many of them lie on
lower ranks, i.e. at lower ids (`sel_apply_kernel`).  This test restates that
protocol in numpy over random candidate sets split into contiguous id slices
and checks that the union of the ranks' selections is the oracle's
unsharded selection (topk.rs:19-34, threshold.rs:20-43), ties included.  The
kernels themselves are checked on two GPUs by test_gpu_sharded.py.
"""

import numpy as np
import pytest

import oracle
from klearu_b200 import _lib

L = 10  # tables: counts lie in 1..L


def _cut(ghist, sampling, top_k, threshold):
    """(cut, need, selected) from the summed histogram, as sel_cut_kernel."""
    if sampling == _lib.SAMPLING_TOPK:
        total = int(ghist[1:].sum())
        if total <= top_k:
            return 0, 0, total
        acc = 0
        for c in range(L, 0, -1):
            if acc + ghist[c] >= top_k:
                return c, top_k - acc, top_k
            acc += int(ghist[c])
        raise AssertionError("unreachable")
    thr = max(threshold, 1)
    passing = int(ghist[thr:].sum())
    if passing > 0:
        return thr - 1, 0, passing
    nz = np.nonzero(ghist[1:])[0]
    if len(nz) == 0:
        return L + 1, 0, 0
    return int(nz[-1]) + 1, 1, 1


def _sharded_select(ids, counts, P, N, sampling, top_k, threshold):
    lo = [(r * N) // P for r in range(P + 1)]
    shards = []
    for r in range(P):
        m = (ids >= lo[r]) & (ids < lo[r + 1])
        shards.append((ids[m], counts[m]))
    hists = [np.bincount(c, minlength=L + 1)[: L + 1] for _, c in shards]
    cut, need, gsel = _cut(np.sum(hists, axis=0), sampling, top_k, threshold)
    eq = [int((c == cut).sum()) if need > 0 else 0 for _, c in shards]
    out = []
    for r, (si, sc) in enumerate(shards):
        take = max(0, need - sum(eq[:r])) if need > 0 else 0
        for i, c in zip(si, sc):  # ids ascending within the shard
            if c > cut or (c == cut and take > 0):
                out.append(int(i))
                if c == cut:
                    take -= 1
    assert len(out) == gsel
    return out


@pytest.mark.parametrize("P", [2, 3, 8])
@pytest.mark.parametrize("sampling,top_k,threshold",
                         [(_lib.SAMPLING_TOPK, 40, 0), (_lib.SAMPLING_TOPK, 7, 0), (_lib.SAMPLING_TOPK, 500, 0),
                          (_lib.SAMPLING_THRESHOLD, 0, 3), (_lib.SAMPLING_THRESHOLD, 0, 9)])
def test_union_of_shard_selections_is_the_global_selection(P, sampling, top_k, threshold):
    rng = np.random.default_rng(P * 1000 + top_k + threshold)
    N = 5000
    for _ in range(40):
        n = int(rng.integers(0, 300))
        ids = np.sort(rng.choice(N, n, replace=False)).astype(np.uint32)
        # few distinct counts, so that ties at the cut span several shards
        counts = rng.integers(1, 4, n).astype(np.uint32) + (rng.random(n) < 0.1) * rng.integers(0, L - 3, n)
        counts = np.minimum(counts, L).astype(np.uint32)
        want = sorted(oracle.sample(sampling, top_k, threshold, ids, counts)) if n else []
        got = sorted(_sharded_select(ids.astype(np.int64), counts.astype(np.int64), P, N, sampling, top_k,
                                     threshold))
        assert got == want
