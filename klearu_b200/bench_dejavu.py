"""Deja Vu sparse FFN microbenchmark (the C3 workload: LLaMA-7B-shaped MLP) on one B200.

    python -m klearu_b200.bench_dejavu [--tokens 1,16,64] [--layers 32] [--distinct 2] [--reps 5]

LLaMA-7B-shaped MLP: hidden 4096, SwiGLU intermediate 11008, bf16 N(0, 0.02)
weights; a rank-1000 predictor (4096 -> 1000 ReLU -> 11008 sigmoid) keeps the
top ceil(0.1 * 11008) = 1101 neurons per token; Gaussian token activations.
One decode step = 32 layers, each: kl_predictor_select_topk, then
kl_sparse_mlp_forward on the selected neurons; the same step is also timed
through kl_ffn_stack_decode (adds RMSNorm and the residual add per layer, one
CUDA graph).  `--distinct` layers of
weights are cycled (2 x 0.6 GB of bf16 > L2), so every layer reads its
weights from HBM.  Timed with CUDA events after a warm-up.  Prints one JSON
line per token count.  Synthetic data.  ``python bench.py --config c3`` runs
this and adds the CPU baseline of one layer for one token.
"""

from __future__ import annotations

import argparse
import json
import math

import numpy as np
import torch

from ._lib import check
from .core import default_context
from .dejavu import FfnStack, SparseMlp, SparsityPredictor

HID, INTER, RANK = 4096, 11008, 1000


def _peak_gbs() -> tuple[float, str]:
    from pathlib import Path

    p = Path(__file__).resolve().parent.parent / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def _stack_kernels(stack, hs, reps: int, layers: int) -> dict:
    """Device time of each kernel inside the FFN stack's replayed graph, µs per
    layer (CUPTI activity records through torch.profiler)."""
    import collections

    from torch.profiler import ProfilerActivity, profile

    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(reps):
            stack.decode(hs, 0.1)
        torch.cuda.synchronize()
    agg = collections.defaultdict(float)
    for e in prof.events():
        if e.device_type == torch.autograd.DeviceType.CUDA:
            name = e.name.replace("(anonymous namespace)::", "").split("(")[0]
            agg[name] += e.device_time_total
    return {k: round(v / reps / layers, 2) for k, v in sorted(agg.items(), key=lambda kv: -kv[1])}


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", default="1,16,64")
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--distinct", type=int, default=2)
    ap.add_argument("--reps", type=int, default=5)
    ap.add_argument("--kernels", action="store_true",
                    help="also print each kernel's device time inside the FFN stack (CUPTI through torch.profiler)")
    ap.add_argument("--no-cpu", action="store_true", help="ignored: bench.py --config c3 times the CPU baseline")
    args = ap.parse_args(argv)
    ctx = default_context(0)
    lib = ctx.lib
    dev = "cuda:0"
    g = torch.Generator(device=dev).manual_seed(5)
    k = math.ceil(0.1 * INTER)

    def w(*shape):
        return (0.02 * torch.randn(*shape, device=dev, generator=g)).cpu().numpy()

    layers = []
    for i in range(args.distinct):
        w1, w2 = w(RANK, HID), w(INTER, RANK)
        b1, b2 = np.zeros(RANK, np.float32), np.zeros(INTER, np.float32)
        gate, up, down = w(INTER, HID), w(INTER, HID), w(HID, INTER)
        layers.append((SparsityPredictor(w1, b1, w2, b2, ctx=ctx), SparseMlp(gate, up, down, None, ctx=ctx)))
        del w1, w2, gate, up, down
    peak, peak_kind = _peak_gbs()
    pred_bytes = (RANK * HID + INTER * 1024) * 2  # bf16 predictor weights (K padded to 64)
    for T in [int(t) for t in args.tokens.split(",")]:
        x = torch.randn(T, HID, device=dev, generator=g).contiguous()
        idx = torch.empty(T, k, dtype=torch.int32, device=dev)
        out = torch.empty(T, HID, device=dev)

        def select(l):
            p = layers[l % args.distinct][0]
            check(lib.kl_predictor_select_topk(p.h, x.data_ptr(), T, k, idx.data_ptr(), None), ctx.h, "select_topk")

        def mlp(l):
            m = layers[l % args.distinct][1]
            check(lib.kl_sparse_mlp_forward(m.h, x.data_ptr(), T, idx.data_ptr(), k, out.data_ptr()), ctx.h,
                  "sparse_mlp_forward")

        def run(fn_list):
            for l in range(args.layers):
                for fn in fn_list:
                    fn(l)

        for fns in ([select], [mlp], [select, mlp]):
            run(fns)
        ctx.sync()  # raises on a recorded device error
        res = {}
        for name, fns in (("predictor_select", [select]), ("sparse_mlp", [mlp]), ("layer", [select, mlp])):
            ts = []
            for _ in range(args.reps):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                run(fns)
                e1.record()
                torch.cuda.synchronize()
                ts.append(e0.elapsed_time(e1) / args.layers * 1e3)  # us per layer
            res[name] = float(np.median(ts))
        # the whole decode step's FFN half as one call (kl_ffn_stack_decode: RMSNorm, select, sparse
        # MLP and residual add per layer, replayed as a CUDA graph)
        stack = FfnStack([layers[l % args.distinct][0] for l in range(args.layers)],
                         [layers[l % args.distinct][1] for l in range(args.layers)],
                         np.ones((args.layers, HID), np.float32), ctx=ctx)
        hs = torch.randn(T, HID, device=dev, generator=g).contiguous()
        for _ in range(3):
            stack.decode(hs, 0.1)
        ctx.sync()
        ts = []
        for _ in range(args.reps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            stack.decode(hs, 0.1)
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1))
        res["stack_step_ms"] = float(np.median(ts))
        if args.kernels:
            print(json.dumps({"bench": "dejavu_ffn_stack_kernels", "tokens": T, "layers": args.layers,
                              "us_per_layer": _stack_kernels(stack, hs, args.reps, args.layers)}), flush=True)
        del stack
        mlp_bytes = T * k * HID * 2 * 3  # gate, up and down rows gathered per token (bf16)
        step_us = res["layer"] * args.layers
        line = {"bench": "dejavu_sparse_ffn", "config": "C3 LLaMA-7B MLP, predictor rank 1000, keep 1101 of 11008",
                "tokens": T, "layers": args.layers, "us_per_layer": res["layer"],
                "predictor_select_us": res["predictor_select"], "sparse_mlp_us": res["sparse_mlp"],
                "decode_step_ms": step_us / 1e3, "tokens_per_s": T / (step_us / 1e6),
                "ffn_stack_step_ms": res["stack_step_ms"],
                "ffn_stack_tokens_per_s": T / (res["stack_step_ms"] / 1e3),
                "predictor_GBs": pred_bytes / (res["predictor_select"] * 1e-6) / 1e9,
                "predictor_TFLOPs_useful": 2 * T * (HID * RANK + RANK * INTER) / (res["predictor_select"] * 1e-6) / 1e12,
                "sparse_mlp_GBs": mlp_bytes / (res["sparse_mlp"] * 1e-6) / 1e9,
                "sparse_mlp_frac_of_hbm": mlp_bytes / (res["sparse_mlp"] * 1e-6) / 1e9 / peak,
                "peak_gbs": peak, "peak_kind": peak_kind}
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
