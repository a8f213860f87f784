"""SLIDE train-step benchmark (BASELINE.json metric: SLIDE train samples/s on
the 670K-way sparse layer, with % of HBM peak).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one batched train step (hash, probe, active-row forward + loss +
input gradient, segmented gradient reduction + lazy Adam on both layers, and
the table rebuild when the RebuildScheduler fires) over one batch of B=256
synthetic C1 examples.  Prints ONE JSON line on rank 0.

* ``value``: samples/s of the whole job with the batches already resident in
  HBM, timed with CUDA events (max over ranks).
* ``e2e``: the same metric through the C-ABI host-batch train step
  (kl_net_train_step_host), each batch uploaded from pinned host memory inside
  the timed region and the loss read back every step.
* ``roofline``: the dominant phase's algorithmic bytes / its event-timed
  duration, against MEASURED_PEAKS.json's HBM copy bandwidth.
* ``cpu_baseline``: the CPU restatement of the reference path (HOGWILD, all
  host threads) on a bounded sample of the same workload.
* ``--impl reference``: that CPU path alone, as the reference arm.

Multi-GPU (torchrun, one rank per GPU): ONE network, neuron-sharded over the
ranks (kl_net_create_sharded): each rank owns 1/N of the 670K output neurons
(rows, Adam state, LSH tables with bucket capacity 128/N) and contributes its
own B=256 examples to a global batch of N*256 (weak scaling).  The hidden layer
is replicated and data parallel; NCCL all-gathers the batches, hidden
activations and hidden gradients, and all-reduces / reduce-scatters the loss
probabilities and the output layer's input gradient.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "SLIDE train samples/s (670K-way sparse layer) @1/2/4/8 B200; % HBM peak"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=100)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--batch", type=int, default=256)
    p.add_argument("--pool", type=int, default=8, help="distinct resident batches cycled through")
    p.add_argument("--cpu-seconds", type=float, default=15.0)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    return p.parse_args()


def workload(cfg, B):
    lo = cfg.network.layers
    return {"workload": "C1 extreme classification (synthetic Amazon-670K shape)",
            "input_dim": lo[0].input_dim, "hidden": lo[0].num_neurons, "output": lo[1].num_neurons,
            "hidden_lsh": "SimHash K6 L50 TopK12 FIFO128", "output_lsh": "DWTA K8 L50 FIFO128 (union<=6400)",
            "per_gpu_batch": B, "weights": "bf16 storage, fp32 Adam state",
            "l2": "working set > L2 (1.03 GB of output weights + Adam state in total)"}


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid: str | None):
        self.uuid = uuid
        self.proc = None
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)

    def start(self):
        cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200"]
        if self.uuid:
            cmd[1:1] = ["-i", self.uuid]
        try:
            self.proc = subprocess.Popen(cmd, stdout=self.file, stderr=subprocess.DEVNULL)
        except FileNotFoundError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        self.proc.wait()
        self.file.flush()
        rows = [r.split(", ") for r in Path(self.file.name).read_text().splitlines() if r.strip()]
        os.unlink(self.file.name)
        sm = [float(r[0]) for r in rows if r[0].replace(".", "").isdigit()]
        mx = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if len(r) > 4 + i and r[4 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def cpu_baseline(cfg, init, gen_seed, seconds, threads, batch=64):
    """The reference CPU path (oracle restatement: per-example train_step,
    dense to_dense input, f32, HOGWILD over `threads`) on a bounded sample."""
    import oracle
    from klearu_b200 import synthetic as S

    t0 = time.time()
    net = oracle.Net(cfg, init, weight_dtype="f32", sparse_input=False)
    build_s = time.time() - t0
    gen = S.XcGenerator(cfg.network.layers[0].input_dim, cfg.network.layers[-1].num_neurons, seed=gen_seed)
    done, t = 0, 0.0
    nb = 0
    while t < seconds or nb == 0:
        hb = gen.batch(batch)
        t1 = time.perf_counter()
        net.train_hogwild(hb, 1e-3, threads)
        t += time.perf_counter() - t1
        done += hb.batch
        nb += 1
    return {"value": done / t, "unit": "samples/s", "cores": threads, "kind": "port",
            "sample": f"{done} C1 examples in {nb} HOGWILD train_parallel calls of {batch} "
                      f"(f32, dense inputs as the reference), {t:.1f} s timed; network build {build_s:.1f} s"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from klearu_b200 import synthetic as S

    cfg = S.config_c1()
    init = S.make_init(cfg, 42)
    threads = os.cpu_count() or 1
    import oracle

    net = oracle.Net(cfg, init, weight_dtype="f32", sparse_input=False)
    gen = S.XcGenerator(135909, 670091, seed=1234)
    per_step = max(threads, 32)  # bounded sample per step
    for _ in range(args.warmup):
        net.train_hogwild(gen.batch(per_step), 1e-3, threads)
    t = 0.0
    for _ in range(args.steps):
        hb = gen.batch(per_step)
        t0 = time.perf_counter()
        net.train_hogwild(hb, 1e-3, threads)
        t += time.perf_counter() - t0
    v = args.steps * per_step / t
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "samples/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * t / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": workload(cfg, per_step),
            "cpu_baseline": {"value": v, "unit": "samples/s", "cores": threads, "kind": "port",
                             "sample": f"{args.steps} steps of {per_step} examples (HOGWILD train_parallel, "
                                       f"f32, dense inputs), CPU restatement of klearu-core (Rust reference "
                                       f"not buildable here)"},
            "e2e": {"value": v, "unit": "samples/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
        return
    import torch
    import torch.distributed as dist

    from klearu_b200 import _lib
    from klearu_b200 import synthetic as S
    from klearu_b200.core import Network, default_context

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    B = args.batch
    cfg = S.config_c1()
    init = S.make_init(cfg, 42)
    shard = None
    if world > 1:
        from klearu_b200.dist import share_unique_id

        shard = (share_unique_id(rank, world), rank, world)
    net = Network(cfg, init, weight_dtype="bf16", max_batch=B, shard=shard, ctx=default_context(local))
    del init
    gen = S.XcGenerator(135909, 670091, seed=1234 + rank)
    pool_host = [gen.batch(B) for _ in range(args.pool)]
    pool = [net.device_batch(hb) for hb in pool_host]
    # size the per-batch buffers for every pooled batch (forward only, no update) so that no
    # allocation happens inside the timed region
    from klearu_b200 import _lib as _L
    import ctypes as _C
    for db in (sorted(pool, key=lambda db: -db.c.nnz)[:1] if world == 1 else []):  # sharded nets pre-size
        _L.check(net.lib.kl_net_forward(net.h, _C.byref(db.c)), net.ctx.h)
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()

    def step(i):
        net.train_step_device(pool[i % len(pool)], 1e-3)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    for l in range(2):
        net.stats(l, reset=True)
    lib = _lib.load()
    import ctypes as C

    lc0 = C.c_uint64()
    lib.kl_launch_count(C.byref(lc0))
    uuid = None
    try:
        uuid = str(torch.cuda.get_device_properties(local).uuid)
        uuid = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
    except Exception:
        pass
    clocks = ClockSampler(uuid)
    clocks.start()
    barrier()
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for i in range(args.steps):
        step(args.warmup + i)
    e1.record(st)
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1)
    lc1 = C.c_uint64()
    lib.kl_launch_count(C.byref(lc1))
    stats = [net.stats(l) for l in range(2)]
    # Phase times come from a separate, untimed pass with the library's event profiler on (the
    # timed loop above replays the captured step graph, which carries no per-phase events).
    KP = min(args.steps, 20)
    for l in range(2):
        net.profile_read(l, reset=True)
    net.profile(True)
    for i in range(KP):
        step(args.warmup + args.steps + i)
    torch.cuda.synchronize()
    net.profile(False)
    prof = [net.profile_read(l) for l in range(2)]
    t = torch.tensor([ms], device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    value = world * B * args.steps / (ms_max / 1e3)

    # ---- roofline (per-step algorithmic bytes from the device counters)
    K = args.steps
    d_in, d_h, d_o = 135909, 128, 670091
    A = stats[1].active_sum / K              # sum of output active set sizes per step
    U_o = stats[1].touched_rows / K          # output rows updated per step
    U_h = stats[0].touched_rows / K          # hidden neurons updated per step
    nnz = stats[0].input_nnz / K
    A_h = stats[0].active_sum / K
    # The roofline kernel: layer 0's streaming Adam pass (fm_adam_kernel), the step's HBM-bound
    # kernel: W (bf16), m, v (f32) of all 135909 feature rows x U_h touched neurons, read and
    # written = 20 B per element.  Timed alone by the library's KL_PHASE_STREAM events.  The
    # output-layer kernels take more time but read rows resident in L2 (issue-bound, see
    # phase_ms_per_step and profiles/).
    bytes_dom = 20.0 * d_in * U_h
    ms_dom = prof[0]["stream"][0] * K / KP  # per-step time of the profiled pass, scaled to K steps
    peak, peak_kind = measured_peaks()
    achieved = bytes_dom / (ms_dom / K / 1e3) / 1e9 if ms_dom > 0 else 0.0  # one launch per step
    step_bytes_formula = (2 * d_h * A) * 2 + 20 * d_h * U_o + 16 * U_o + 4 * 50 * 128 * B + 2 * d_h * nnz + \
        20 * d_in * U_h + nnz * 8
    roofline = {"bound": "hbm", "kernel": "fm_adam_kernel (hidden-layer Adam over all 135909 feature rows)",
                "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak, "peak_kind": peak_kind,
                # dram__bytes_read.sum + dram__bytes_write.sum of one launch, ncu --set full, C1
                # (profiles/slide_step_c1_kernels_ncu.md): part of W/m/v is served from L2
                "traffic": 295.8e6,
                "bytes_per_launch": bytes_dom / 1.0, "ms_per_launch": ms_dom / K,
                "step_bytes_formula": step_bytes_formula,
                "step_frac_of_peak": step_bytes_formula / (ms_max / K / 1e3) / 1e9 / peak,
                "phase_ms_per_step": {f"{l}.{p}": prof[i][p][0] / KP for i, l in enumerate(("hidden", "output"))
                                      for p in _lib.PHASES},
                "per_step": {"active_out": A, "touched_out": U_o, "touched_hidden": U_h, "nnz": nnz,
                             "rebuilds": int(stats[1].rebuilds)}}

    # ---- end to end through the C ABI with host buffers
    e2e = None
    if not args.no_e2e:
        hosts = []
        for hb in pool_host:
            arrs = {k: torch.from_numpy(np.ascontiguousarray(getattr(hb, k)).view(
                np.int32 if k != "val" else np.float32)).pin_memory()
                    for k in ("rowptr", "idx", "val", "label_ptr", "labels")}
            hosts.append((hb, arrs))
        loss_h = torch.zeros(1).pin_memory()
        bi = sum(int(a.numel()) * 4 for a in hosts[0][1].values())

        def e2e_step(i):
            # the public host-batch call: it packs the pinned CSR arrays,
            # uploads them on its copy stream and enqueues the loss readback
            hb, arrs = hosts[i % len(hosts)]
            c = _lib.BatchC(hb.batch, arrs["rowptr"].data_ptr(), arrs["idx"].data_ptr(), arrs["val"].data_ptr(),
                            arrs["label_ptr"].data_ptr(), arrs["labels"].data_ptr(), int(hb.rowptr[-1]),
                            int(hb.label_ptr[-1]))
            _lib.check(lib.kl_net_train_step_host(net.h, C.byref(c), 1e-3, _lib.MODE_BATCHED, loss_h.data_ptr()),
                       net.ctx.h)

        for i in range(3):
            e2e_step(i)
        torch.cuda.synchronize()
        barrier()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(st)
        for i in range(args.steps):
            e2e_step(i)
        f1.record(st)
        torch.cuda.synchronize()
        barrier()
        t2 = torch.tensor([f0.elapsed_time(f1)], device="cuda")
        if world > 1:
            dist.all_reduce(t2, op=dist.ReduceOp.MAX)
        e2e = {"value": world * B * args.steps / (float(t2.item()) / 1e3), "unit": "samples/s",
               "h2d_bytes_per_step": bi, "d2h_bytes_per_step": 4,
               "api": "kl_net_train_step_host (C ABI): per-step upload of the pinned host CSR batch and loss readback"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(cfg, S.make_init(cfg, 42), 4321, args.cpu_seconds, os.cpu_count() or 1)

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "samples/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                "config": {**workload(cfg, B), "global_batch": B * world,
                           "parallelism": f"output neurons sharded over {world} GPUs, hidden layer data parallel"
                           if world > 1 else "single"},
                "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e,
                "gpu_launches": int(lc1.value - lc0.value), "clocks": clk}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
