"""LSH index microbenchmark (the C4 workload: 1M-row index) on one B200.

    python -m klearu_b200.bench_index [--rows 1000000] [--queries 4096] [--reps 5]

1M rows x 128 bf16 unit-norm Gaussian; SimHash K6 L50 and DWTA K8 L100, each
with FIFO and reservoir buckets of capacity 128.  For each: a full rebuild
(kl_index_rebuild, hash + ordered bucket fill) and query_union over 4096
queries (2048 near-duplicates of indexed rows: row + N(0, 0.05^2) per
dimension, renormalised; 2048 fresh unit Gaussians), both timed with CUDA
events after a warm-up.  Prints one JSON line per configuration.  Synthetic
data; no dataset items.  ``python bench.py --config c4`` runs this and adds
the CPU baseline of the same workload.
"""

from __future__ import annotations

import argparse
import json

import numpy as np
import torch

from . import _lib
from . import params as P
from .config import BucketType, HashFunctionType as HF
from .core import HashFamily, LshIndex, default_context


def _unit(x: torch.Tensor) -> torch.Tensor:
    return x / x.norm(dim=1, keepdim=True).clamp_min(1e-12)


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--rows", type=int, default=1_000_000)
    ap.add_argument("--dim", type=int, default=128)
    ap.add_argument("--queries", type=int, default=4096)
    ap.add_argument("--reps", type=int, default=5)
    ap.add_argument("--cpu-rows", type=int, default=0, help="ignored: bench.py --config c4 times the CPU baseline")
    args = ap.parse_args(argv)
    ctx = default_context(0)
    dev = "cuda:0"
    g = torch.Generator(device=dev).manual_seed(11)
    rows = _unit(torch.randn(args.rows, args.dim, device=dev, generator=g)).to(torch.bfloat16).contiguous()
    nq = args.queries
    pick = torch.randint(0, args.rows, (nq // 2,), device=dev, generator=g)
    near = _unit(rows[pick].float() + 0.05 * torch.randn(nq // 2, args.dim, device=dev, generator=g))
    fresh = _unit(torch.randn(nq - nq // 2, args.dim, device=dev, generator=g))
    Q = torch.cat([near, fresh]).contiguous()
    for kind, K, L in ((HF.SimHash, 6, 50), (HF.DwtaHash, 8, 100)):
        prm = P.hash_params(kind, np.random.default_rng(7), args.dim, K, L)
        for bucket in (BucketType.Fifo, BucketType.Reservoir):
            ix = LshIndex(HashFamily(kind, args.dim, K, L, params=prm, ctx=ctx), bucket, 128)
            ix.rebuild_rows(rows)
            ix.query_batch(Q, mode=_lib.QUERY_UNION)
            torch.cuda.synchronize()
            e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
            t_rb, t_q = [], []
            for _ in range(args.reps):
                e0.record()
                ix.rebuild_rows(rows)
                e1.record()
                offs, ids, _ = ix.query_batch(Q, mode=_lib.QUERY_UNION)
                e2.record()
                torch.cuda.synchronize()
                t_rb.append(e0.elapsed_time(e1))
                t_q.append(e1.elapsed_time(e2))
            union = float(offs[-1].item()) / nq
            near_hit = float(np.mean([int(pick[i]) in set(ids[offs[i]:offs[i + 1]].cpu().numpy().tolist())
                                      for i in range(0, nq // 2, 64)]))
            rb_seq = None
            if kind == HF.SimHash:
                # the same rebuild with the reference's sequential projection sums
                ix.set_projection(_lib.PROJ_SEQUENTIAL)
                ts = []
                for _ in range(2):
                    e0.record()
                    ix.rebuild_rows(rows)
                    e1.record()
                    torch.cuda.synchronize()
                    ts.append(e0.elapsed_time(e1))
                rb_seq = float(np.median(ts))
                ix.set_projection(_lib.PROJ_AUTO)
            rb_ms = float(np.median(t_rb))
            q_ms = float(np.median(t_q))
            print(json.dumps({
                "workload": "C4 LSH index microbench (synthetic)", "hash": f"{HF(kind).name} K{K} L{L}",
                "bucket": BucketType(bucket).name, "rows": args.rows, "dim": args.dim, "queries": nq,
                "rebuild_ms": rb_ms, "rebuild_rows_per_s": args.rows / (rb_ms / 1e3),
                "rebuild_ms_sequential_projection": rb_seq,
                "query_union_ms": q_ms, "queries_per_s": nq / (q_ms / 1e3), "mean_union": union,
                "near_duplicate_self_hit": near_hit,
            }), flush=True)
            del ix


if __name__ == "__main__":
    main()
