"""One rank of a P-way neuron-sharded C1 step, stood in for on one B200.

    python -m klearu_b200.bench_shard [--ranks 8] [--steps 20] [--kernels]

A rank of the sharded network (kl_net_create_sharded) owns 670091 / P output
neurons with buckets of 128 / P ids and trains on the global batch of P x 256
examples.  This benchmark builds an unsharded network of exactly that shape
(the output TopK kept at the unsharded 67009, so every candidate is selected,
as on a shard) and times its batched step over a 256·P-example batch.  It
measures a rank's compute without the collectives (the hidden layer here is
the full replicated one over the global batch, where a real rank updates 1/P
of its feature rows).  Prints one JSON line: the step time, the per-phase
times of a profiled pass, the active and touched rows per step, and with
`--kernels` each kernel's device time (CUPTI through torch.profiler).
Synthetic data; no dataset items.
"""

from __future__ import annotations

import argparse
import collections
import json

import torch

from . import synthetic as S
from .core import Network, default_context


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ranks", type=int, default=8)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--kernels", action="store_true")
    args = ap.parse_args()
    P, K = args.ranks, args.steps
    cfg = S.config_xc(n_out=670091 // P, cap=max(1, 128 // P))
    cfg.network.layers[1].top_k = 67009  # the unsharded layer's TopK: every candidate is selected
    net = Network(cfg, S.make_init(cfg, 42), weight_dtype="bf16", max_batch=256 * P, ctx=default_context(0))
    gen = S.XcGenerator(135909, 670091 // P, seed=1234)
    dbs = [net.device_batch(gen.batch(256 * P)) for _ in range(4)]
    for i in range(5):
        net.train_step_device(dbs[i % 4], 1e-3)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(K):
        net.train_step_device(dbs[i % 4], 1e-3)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / K
    net.stats(1, reset=True)
    net.profile(True)
    for i in range(K):
        net.train_step_device(dbs[i % 4], 1e-3)
    torch.cuda.synchronize()
    net.profile(False)
    phases = {f"{name}.{k}": round(v[0] / K * 1e3, 1) for l, name in enumerate(("hidden", "output"))
              for k, v in net.profile_read(l).items() if v[0] > 0}
    st = net.stats(1)
    line = {"bench": "shard_rank_standin", "ranks": P, "global_batch": 256 * P, "ms_per_step": ms,
            "phase_us_per_step": phases, "active_out_per_step": st.active_sum / max(1, st.steps),
            "touched_out_per_step": st.touched_rows / max(1, st.steps)}
    if args.kernels:
        from torch.profiler import ProfilerActivity, profile

        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            for i in range(K):
                net.train_step_device(dbs[i % 4], 1e-3)
            torch.cuda.synchronize()
        agg = collections.defaultdict(float)
        for e in prof.events():
            if e.device_type == torch.autograd.DeviceType.CUDA:
                agg[e.name.replace("(anonymous namespace)::", "").split("(")[0]] += e.device_time_total
        line["kernel_us_per_step"] = {k: round(v / K, 1) for k, v in sorted(agg.items(), key=lambda kv: -kv[1])}
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
