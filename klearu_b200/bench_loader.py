"""LibSVM loader and batch iterator throughput on the host (no GPU needed).

    python -m klearu_b200.bench_loader [--examples 100000] [--threads 0] [--batch 256]

Writes the bench's seeded C1 example stream (135909 features, ~75 distinct
Zipf feature ids per example, L2-normalised log-normal values, 1-7 Zipf labels
out of 670091) as LibSVM text, and times:

* ``kl_libsvm_parse`` of the whole text on 1 thread and on all host threads
  (the reference's ``LibSvmDataset::load_from_reader``, libsvm.rs:39-111, is a
  single-threaded line parser; the 1-thread figure is its stand-in here);
* one epoch of ``kl_batch_iter_next`` (the reference's shuffled
  ``BatchIterator``, dataset.rs:38-111) with and without the prefetching
  worker, in examples/s — the rate the iterator can feed
  ``kl_net_train_step_host`` at.

Prints one JSON line.  Synthetic data; no dataset items.
"""

from __future__ import annotations

import argparse
import json
import os
import time


from .data import BatchIterator, LibSvmDataset
from .synthetic import XcGenerator


def synthetic_text(n: int, dim: int = 135909, nlabels: int = 670091, seed: int = 0) -> bytes:
    """n examples of the bench's C1 example stream (synthetic.XcGenerator) as
    LibSVM lines with the stream's 0-based feature ids and 9 significant digits
    (f32 values round-trip exactly)."""
    gen = XcGenerator(dim, nlabels, seed=seed)
    lines = []
    done = 0
    while done < n:
        hb = gen.batch(min(1024, n - done))
        for s in range(hb.batch):
            a, b = int(hb.rowptr[s]), int(hb.rowptr[s + 1])
            c, d = int(hb.label_ptr[s]), int(hb.label_ptr[s + 1])
            feats = " ".join(f"{i}:{v:.9g}" for i, v in zip(hb.idx[a:b].tolist(), hb.val[a:b].tolist()))
            lines.append(",".join(map(str, hb.labels[c:d].tolist())) + " " + feats)
        done += hb.batch
    return ("\n".join(lines) + "\n").encode()


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--examples", type=int, default=100_000)
    ap.add_argument("--threads", type=int, default=0, help="parser threads (0: all host threads)")
    ap.add_argument("--batch", type=int, default=256)
    ap.add_argument("--reps", type=int, default=3)
    args = ap.parse_args(argv)
    t0 = time.perf_counter()
    text = synthetic_text(args.examples)
    gen_s = time.perf_counter() - t0
    threads = args.threads or os.cpu_count() or 1

    def parse(nt):
        ts = []
        for _ in range(args.reps):
            t = time.perf_counter()
            ds = LibSvmDataset.load_from_str(text, 135909, 670091, nt)
            ts.append(time.perf_counter() - t)
        return ds, min(ts)

    ds, t1 = parse(1)
    _, tn = parse(threads)
    nnz = int(ds.rowptr[-1])

    def epoch(prefetch):
        it = BatchIterator(ds, args.batch, 42, prefetch)
        t = time.perf_counter()
        n = 0
        while True:
            b = it.next_raw()
            if b is None:
                break
            n += b.batch
        return n / (time.perf_counter() - t)

    epoch(True)  # first-touch of the batch buffers
    line = {"bench": "libsvm_loader", "data": "synthetic C1-shaped LibSVM text", "examples": len(ds),
            "nnz": nnz, "text_MB": len(text) / 1e6, "generate_s": gen_s,
            "parse_1_thread": {"MB_per_s": len(text) / 1e6 / t1, "examples_per_s": len(ds) / t1},
            f"parse_{threads}_threads": {"MB_per_s": len(text) / 1e6 / tn, "examples_per_s": len(ds) / tn},
            "parse_speedup": t1 / tn,
            "batch_iter_examples_per_s": {"prefetch": epoch(True), "no_prefetch": epoch(False)},
            "batch": args.batch, "host_threads": os.cpu_count()}
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
