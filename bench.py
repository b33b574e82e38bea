#!/usr/bin/env python3
"""Benchmark: HalfKP 256x2-32-32-1 training step.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

One "step" = one Ranger train step (forward, sigmoid-WDL loss, backward,
optimizer over every parameter) on a batch of 16384 synthetic positions
(seeded, shapes and distributions of the reference's teacher data; see
bulletou_b200/synthetic.py).  Prints one JSON line (rank 0).

* value      positions/s with the batches already resident in HBM
             (CUDA events on the library's stream, max over ranks);
* e2e        positions/s through the public runner API from pinned host
             memory: per step the H2D copy of the batch and a D2H read of the
             step's mean loss are inside the timed region;
* roofline   the dominant kernel (from the library's stage profiler, events on
             the launching stream during the timed region) against the measured
             HBM peak in MEASURED_PEAKS.json;
* cpu_baseline  the CPU oracle's forward (C restatement of the reference's
             evaluation path), single thread, on a bounded sample.

--impl reference times the reference's own cuda-cpp backend (built from its
sources into oracle/_ref) through the reference runner's call sequence, on the
same GPU, config and metric.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

BATCH = 16384
ACTIVE = 38
SHAPE = (125388, 256, 32, 32)
N_BATCHES = 8
METRIC = "train positions/sec (HalfKP 256x2-32-32-1, batch 16384)"
PHASES = ("inverse_index", "king_sort", "ft_gather", "dense_fwd_loss_bwd", "batch_reduce", "small_param_ranger",
          "ft_row_grad_ranger")
LAUNCHES_PER_STEP = 13  # index 5 + king sort 3 + gather, dense, reduce, finalize, rows


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("b200", "reference"), default="b200")
    ap.add_argument("--batch", type=int, default=BATCH)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


# --------------------------------------------------------------------------- helpers
def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clock/throttle samples during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(prefix="clocks_", suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except FileNotFoundError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if self.proc is None or not self.path or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, smax, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in Path(self.path).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        os.unlink(self.path)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax), "reasons": sorted(reasons),
                "samples": len(sm)}


def make_batches(batch, rank=0):
    from bulletou_b200 import synthetic

    return [synthetic.halfkp_batch(1000 + i, batch, rank) for i in range(N_BATCHES)]


def make_runner(ctx, batch, fused):
    import bulletou_b200 as bo
    from bulletou_b200 import synthetic

    w = synthetic.halfkp_weights(synthetic.rng_for(7))
    return bo.NnueTrainStepRunner(ctx, bo.NnueForwardHostWeights(bo.NnueForwardShape(*SHAPE), **w), batch, ACTIVE,
                                  fused=fused)


def ranger(step):
    import bulletou_b200 as bo

    return bo.RangerUpdateParams(radam=bo.RAdamUpdateParams(step=step, learning_rate=1e-3))


def device_batches(ctx, batches):
    import bulletou_b200 as bo

    return [(bo.I32Buffer.from_host(ctx, b["stm"]), bo.I32Buffer.from_host(ctx, b["nstm"]),
             bo.F32Buffer.from_host(ctx, b["targets"]), bo.F32Buffer.from_host(ctx, b["entry_weights"]))
            for b in batches]


def bind_batch(runner, dev):
    runner.stm_indices, runner.nstm_indices, runner.targets, runner.entry_weights = dev


def cpu_baseline(batch_cap=2048, budget_s=8.0):
    """CPU oracle forward (C restatement of the reference's evaluation path),
    one thread, on a bounded sample."""
    from bulletou_b200 import synthetic
    from oracle import oracle

    w = synthetic.halfkp_weights(synthetic.rng_for(7))
    b = synthetic.halfkp_batch(4242, batch_cap)
    oracle.nnue_forward(SHAPE, b["stm"][:ACTIVE * 16], b["nstm"][:ACTIVE * 16], 16, ACTIVE, w)  # warm
    t0 = time.perf_counter()
    reps = 0
    while True:
        oracle.nnue_forward(SHAPE, b["stm"], b["nstm"], batch_cap, ACTIVE, w)
        reps += 1
        if time.perf_counter() - t0 >= budget_s:
            break
    dt = time.perf_counter() - t0
    return {"value": reps * batch_cap / dt, "unit": "positions/s (forward only)", "cores": 1, "kind": "port",
            "sample": f"oracle HalfKP forward, {reps} x {batch_cap} positions in {dt:.1f} s "
                      f"(the reference cannot train on CPU; its CPU path is evaluation only)"}


# --------------------------------------------------------------------------- distributed
def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world == 1:
        return 0, 1, 0, None
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    rank = int(os.environ["RANK"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    return rank, world, local, dist


def max_over_ranks(dist, value):
    if dist is None:
        return value
    import torch

    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# --------------------------------------------------------------------------- arms
def run_b200(args, rank, world, local, dist):
    import bulletou_b200 as bo

    if world > 1:
        from bulletou_b200.data_parallel import run_data_parallel_bench

        return run_data_parallel_bench(args, rank, world, local, dist)
    ctx = bo.Context(local)
    runner = make_runner(ctx, args.batch, fused=True)
    batches = make_batches(args.batch, rank)
    devb = device_batches(ctx, batches)
    loss_kind = bo.ScalarLossKind.SigmoidPow(2.0)
    inv = 1.0 / 600.0
    step = 0
    for i in range(args.warmup):
        step += 1
        bind_batch(runner, devb[i % N_BATCHES])
        runner.step_device(ctx, ranger(step), loss_kind, inv, finalize_loss=False)
    ctx.synchronize()
    if dist is not None:
        dist.barrier()
    # ---- device-resident timed region (+ stage profile) ----
    lib = ctx.lib
    start, stop = bo.Event(ctx), bo.Event(ctx)
    lib.call("bulletou_b200_profile_begin", ctx.as_ptr(), 8 * args.steps + 8)
    with ClockSampler(local) as clocks:
        start.record(ctx)
        for i in range(args.steps):
            step += 1
            bind_batch(runner, devb[i % N_BATCHES])
            runner.step_device(ctx, ranger(step), loss_kind, inv, finalize_loss=False)
        stop.record(ctx)
        stop.synchronize()
    import ctypes

    ms = (ctypes.c_float * 8)()
    nsteps, nphases = ctypes.c_size_t(), ctypes.c_size_t()
    lib.call("bulletou_b200_profile_end", ctx.as_ptr(), ms, 8, ctypes.byref(nsteps), ctypes.byref(nphases))
    total_ms = stop.elapsed_ms_since(start)
    total_ms = max_over_ranks(dist, total_ms)
    phase_ms = {PHASES[p]: ms[p] / max(1, nsteps.value) for p in range(nphases.value)}
    clk = clocks.summary()
    # ---- end to end through the public API, host (pinned) buffers ----
    # The reference runner's pipelined step (lib.rs:5801): uploads of step i+1
    # on a second stream overlap step i; per step the batch is copied H2D from
    # pinned host memory and the step's mean loss is copied D2H.
    from bulletou_b200.cuda_cpp import NnueTrainStepHostBatch, NnueTrainStepUploadSlot, PinnedF32Buffer

    upload_ctx = bo.Context(local)
    sources = []
    for b in batches:  # the data loader's output: batches already in pinned host memory
        slot = NnueTrainStepUploadSlot(ctx, args.batch, ACTIVE)
        slot.fill(NnueTrainStepHostBatch(b["stm"], b["nstm"], b["targets"], b["entry_weights"], args.batch, ACTIVE))
        sources.append(slot)
    e2e_steps = max(8, args.steps)
    loss_ring = [PinnedF32Buffer(ctx, 1) for _ in range(e2e_steps)]
    for i in range(3):  # warm the pipelined path
        step += 1
        runner.step_pipelined_no_readback_with_loss_finalize(ctx, upload_ctx, ranger(step), loss_kind, inv, None, True,
                                                             sources[i % N_BATCHES], loss_ring[i])
    ctx.synchronize()
    upload_ctx.synchronize()
    h2d = 0
    e0, e1 = bo.Event(ctx), bo.Event(ctx)
    t0 = time.perf_counter()
    e0.record(ctx)
    for i in range(e2e_steps):
        step += 1
        h2d = runner.step_pipelined_no_readback_with_loss_finalize(ctx, upload_ctx, ranger(step), loss_kind, inv, None,
                                                                   True, sources[i % N_BATCHES], loss_ring[i])
    e1.record(ctx)
    e1.synchronize()
    wall_ms = (time.perf_counter() - t0) * 1000.0
    losses = [float(r.host()[0]) for r in loss_ring]
    e2e_ms = max_over_ranks(dist, max(e1.elapsed_ms_since(e0), wall_ms))
    assert all(np.isfinite(losses)), "non-finite loss"
    return {
        "total_ms": total_ms, "phase_ms": phase_ms, "clocks": clk,
        "e2e": {"value": e2e_steps * args.batch * world / (e2e_ms / 1000.0), "unit": "positions/s",
                "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": 4, "steps": e2e_steps,
                "path": "NnueTrainStepRunner.step_pipelined_no_readback_with_loss_finalize (2 upload slots, "
                        "second stream), inputs in pinned host memory, mean loss copied D2H every step"},
        "gpu_launches": LAUNCHES_PER_STEP * args.steps,
        "final_loss": losses[-1],
    }


def run_reference(args, local):
    import bulletou_b200 as bo

    lib = bo.reference_library()
    ctx = bo.Context(local, lib)
    runner = make_runner(ctx, args.batch, fused=False)
    batches = make_batches(args.batch)
    devb = device_batches(ctx, batches)
    loss_kind = bo.ScalarLossKind.SigmoidPow(2.0)
    inv = 1.0 / 600.0
    step = 0
    for i in range(args.warmup):
        step += 1
        bind_batch(runner, devb[i % N_BATCHES])
        runner.step_device(ctx, ranger(step), loss_kind, inv, finalize_loss=False)
    ctx.synchronize()
    start, stop = bo.Event(ctx), bo.Event(ctx)
    with ClockSampler(local) as clocks:
        start.record(ctx)
        for i in range(args.steps):
            step += 1
            bind_batch(runner, devb[i % N_BATCHES])
            runner.step_device(ctx, ranger(step), loss_kind, inv, finalize_loss=False)
        stop.record(ctx)
        stop.synchronize()
    total_ms = stop.elapsed_ms_since(start)
    clk = clocks.summary()
    # end to end through the reference API: the pipelined runner step
    # (lib.rs:5801) with staged pinned uploads on a second stream; the mean
    # loss is read back every step (the reference ABI's download is synchronous)
    from bulletou_b200.cuda_cpp import NnueTrainStepHostBatch

    upload_ctx = bo.Context(local, lib)
    hbs = [NnueTrainStepHostBatch(b["stm"], b["nstm"], b["targets"], b["entry_weights"], args.batch, ACTIVE)
           for b in batches]
    e2e_steps = max(8, args.steps // 2)
    for i in range(2):
        step += 1
        runner.step_pipelined_no_readback_with_loss_finalize(ctx, upload_ctx, ranger(step), loss_kind, inv,
                                                             hbs[i % N_BATCHES], True)
        runner.loss_workspace.mean.download(ctx)
    ctx.synchronize()
    e0, e1 = bo.Event(ctx), bo.Event(ctx)
    t0 = time.perf_counter()
    e0.record(ctx)
    h2d = 0
    for i in range(e2e_steps):
        step += 1
        h2d = runner.step_pipelined_no_readback_with_loss_finalize(ctx, upload_ctx, ranger(step), loss_kind, inv,
                                                                   hbs[i % N_BATCHES], True)
        runner.loss_workspace.mean.download(ctx)
    e1.record(ctx)
    e1.synchronize()
    e2e_ms = max(e1.elapsed_ms_since(e0), (time.perf_counter() - t0) * 1000.0)
    return {"total_ms": total_ms, "clocks": clk,
            "e2e": {"value": e2e_steps * args.batch / (e2e_ms / 1000.0), "unit": "positions/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4, "steps": e2e_steps}}


# --------------------------------------------------------------------------- roofline
def roofline(phase_ms, batch, hbm_peak, peak_kind, lookahead_frac=1.0 / 6.0):
    """Algorithmic bytes per launch of each phase (the formulas are written
    out in DESIGN.md); the dominant phase is reported."""
    rows, width = SHAPE[0], SHAPE[1]
    entries = 2 * batch * ACTIVE
    algo = {
        # per row: w, m, v read + written (24 B/param), slow r+w on lookahead
        # steps (averaged), the batch's pre-activation gradients read once,
        # the inverse index (entries + offsets)
        "ft_row_grad_ranger": rows * width * 4 * (6 + 2 * lookahead_frac) + 2 * batch * width * 4
                              + 4 * (entries + rows + 1),
        # logical bytes of the gathered FT rows (2*A rows of 1 KB per position,
        # L2-served after the king sort) + indices + activations written
        "ft_gather": 2 * batch * ACTIVE * width * 4 + 2 * batch * ACTIVE * 4 + 2 * batch * width * 4,
        # activations read, pre-activation gradients written, small per-position vectors
        "dense_fwd_loss_bwd": 2 * (2 * batch * width * 4) + batch * 4 * (32 * 4 + 4 * 4),
        "batch_reduce": 2 * (2 * batch * width * 4) + batch * 4 * (32 * 4 + 2),
        "inverse_index": 4 * (entries * 3 + rows * 4),
        "king_sort": 4 * (2 * batch * 4),
        "small_param_ranger": 0.0,
    }
    dom = max(phase_ms, key=phase_ms.get)
    t = phase_ms[dom] / 1000.0
    achieved = algo.get(dom, 0.0) / t / 1e9 if t > 0 else 0.0
    return {"bound": "hbm", "kernel": dom, "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
            "frac": round(achieved / hbm_peak, 4), "peak_source": peak_kind, "traffic": None,
            "algorithmic_bytes_per_launch": int(algo.get(dom, 0.0)), "launch_ms": round(phase_ms[dom], 4),
            "phase_ms": {k: round(v, 4) for k, v in phase_ms.items()}}


def main():
    args = parse_args()
    rank, world, local, dist = dist_setup(args)
    if args.warmup < 3:
        args.warmup = 3
    config = {"workload": "configs[1] HalfKP 256x2-32-32-1 train step", "model": "HalfKP 125388x256x2-32-32-1",
              "global_batch": args.batch * world, "per_gpu_batch": args.batch, "seq_len": 1,
              "max_active": ACTIVE, "optimizer": "Ranger (RAdam + Lookahead k=6, lr 1e-3)",
              "loss": "sigmoid-WDL MSE, scale 600, lambda 0.5",
              "parallelism": f"dp{world}" if world > 1 else "single",
              "l2": "no flush: each step streams 0.5 GB of optimizer state (> 126 MB L2)"}
    base = {"metric": METRIC, "unit": "positions/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded; reference teacher-data shapes and distributions)", "config": config}
    if args.impl == "reference":
        if rank != 0:
            return
        try:
            r = run_reference(args, local)
        except (FileNotFoundError, OSError) as e:
            print(json.dumps({"impl": "reference", "unavailable": f"reference backend not built: {e}"}))
            return
        value = args.steps * args.batch / (r["total_ms"] / 1000.0)
        line = dict(base, impl="reference", value=round(value, 1), ms_per_step=round(r["total_ms"] / args.steps, 4),
                    n_gpus=1, clocks=r["clocks"], e2e={k: (round(v, 1) if isinstance(v, float) else v)
                                                        for k, v in r["e2e"].items()},
                    arm="reference cuda-cpp backend built from its own sources (oracle/_ref), driven through its "
                        "C ABI in the reference runner's call order, same GPU/config/metric",
                    cpu_baseline={"value": round(value, 1), "unit": "positions/s", "cores": 0, "kind": "reference",
                                  "sample": f"{args.steps} steps x {args.batch} positions on the GPU (not a CPU run)"})
        print(json.dumps(line))
        return
    r = run_b200(args, rank, world, local, dist)
    value = args.steps * args.batch * world / (r["total_ms"] / 1000.0)
    if rank == 0:
        hbm, kind = measured_peaks()
        line = dict(base, value=round(value, 1), ms_per_step=round(r["total_ms"] / args.steps, 4),
                    e2e={k: (round(v, 1) if isinstance(v, float) else v) for k, v in r["e2e"].items()},
                    roofline=roofline(r["phase_ms"], args.batch, hbm, kind), clocks=r["clocks"],
                    gpu_launches=r["gpu_launches"], final_loss=r["final_loss"])
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline()
        print(json.dumps(line))
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
