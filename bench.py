#!/usr/bin/env python3
"""Benchmark: BulletOu training step on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--workload sfnn|halfkp]

Workloads (one "step" = one Ranger train step: forward, sigmoid-WDL loss,
backward, optimizer over every parameter):

* sfnn (default, BASELINE configs[2], the north-star target): SFNN
  HalfKA_hm2 1536x2 -> LayerStack k3k3 (9 buckets) 1536 -> 15+1 -> 32 -> 1
  with the FT factorizer (+1629 virtual rows) and the shared L1 factor,
  f32, 65536 positions per GPU;
* halfkp: HalfKP 256x2-32-32-1, 16384 positions.

Synthetic seeded batches with the reference teacher data's shapes and
distributions (bulletou_b200/synthetic.py).  Prints one JSON line (rank 0):

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
same GPU, config and metric.  With N > 1 ranks the product arm trains data
parallel (per-rank batch fixed: weak scaling) with NCCL reduce-scatter /
all-reduce / all-gather.
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

SFNN_BATCH = 65536
SFNN_ACTIVE = 40
SFNN_N_BATCHES = 4
SFNN_METRIC = "train positions/sec (SFNN HalfKA_hm2 1536x2 LayerStack k3k3 15+1-32-1, batch 65536 per GPU)"
SFNN_PHASES = ("fold", "sorts_tiles", "inverse_index", "ft_forward", "l1_head", "l1_backward", "small_grads_ranger",
               "ft_rows_ranger")
# fold 1, king sort 3, bucket sort 3, tile table 1, L1 weights 1, index 5 + row sort 1, FT forward 1,
# L1 forward 1, head 1, L1 backward 1, finalize 1, Ranger on 9 small groups, FT rows 45 kings / 3 per launch
SFNN_LAUNCHES_PER_STEP = 1 + 3 + 3 + 1 + 1 + 6 + 1 + 1 + 1 + 1 + 1 + 9 + 15
# QAT modes (the runner's qat_l1 / qat_ft / qat_l2 / qat_l3).  configs[2] trains
# "with QAT fake-quant": the default quantises every layer (FT, L1, L2, L3),
# which selects the dense integer QAT with the engine's integer FT.
SFNN_QAT_MODES = {
    "none": (False, False, False, False),
    "l1": (True, False, False, False),
    "layers": (True, True, True, False),
    "dense": (True, False, True, True),
    "all": (True, True, True, True),
}
SFNN_QAT_LABELS = {
    "none": "none (f32)",
    "l1": "L1 fake-quant (fold then i8 / i32 rounding, identity STE)",
    "layers": "FT + L1 + L2 fake-quant (identity STE, f32 activations)",
    "dense": "L1 + L2 + L3: dense integer QAT on the 1/127 FT lattice, continuous STEs",
    "all": "FT + L1 + L2 + L3: dense integer QAT with the engine's integer FT, continuous STEs",
}


def sfnn_lr_multipliers(mode):
    from bulletou_b200 import sfnn as bs

    l1, ft, l2, l3 = SFNN_QAT_MODES[mode]
    return bs.SfnnLayerLrMultipliers(qat_l1=l1, qat_ft=ft, qat_l2=l2, qat_l3=l3)


def sfnn_launches_per_step(mode):
    """Kernels of one fused step: the QAT extras are the L1 bias fold (L1 QAT),
    the FT bias rounding (FT QAT), and the integer FT (dense + FT QAT; its i16
    table is written by the fold)."""
    l1, ft, l2, l3 = SFNN_QAT_MODES[mode]
    return SFNN_LAUNCHES_PER_STEP + int(l1) + int(ft) + (1 if (ft and l1 and l2 and l3) else 0)


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("b200", "reference"), default="b200")
    ap.add_argument("--workload", choices=("sfnn", "halfkp", "kppt"), default="sfnn")
    ap.add_argument("--batch", type=int, default=None)
    ap.add_argument("--dp-chunk-launches", type=int, default=3,
                    help="N > 1: FT row launches per exchanged chunk (SFNN)")
    ap.add_argument("--qat", choices=tuple(SFNN_QAT_MODES), default="all",
                    help="SFNN quantisation-aware training mode (both arms)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--data", choices=("psv", "uniform"), default="psv",
                    help="SFNN batches: decoded PackedSfenValue records (kings near home, as in teacher data) or "
                         "feature rows uniform over the king blocks")
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


# --------------------------------------------------------------------------- KPPT workload
KPPT_BATCH = 32768
KPPT_METRIC = "train positions/sec (KPPT KPP component table, 81 x 1548^2 entries, 703 pairs, batch 32768)"


def run_kppt(args, local, reference=False):
    """One KPP component-table train step per iteration (the reference trains
    one component table per runner, lib.rs:4857-5066): device-resident
    batches; the e2e leg uploads every step's pair indices, targets and
    weights from pinned host memory."""
    import bulletou_b200 as bo
    from bulletou_b200 import synthetic
    from bulletou_b200.cuda_cpp import PinnedF32Buffer, PinnedI32Buffer

    lib = bo.reference_library() if reference else None
    ctx = bo.Context(local, lib) if lib else bo.Context(local)
    rng = synthetic.rng_for(77)
    n_inputs = synthetic.KPP_INPUTS
    table = rng.normal(0.0, 0.01, n_inputs).astype(np.float32)
    runner = bo.KpptTableTrainStepRunner(ctx, n_inputs, table, 0.0, [1.0, -1.0], 0.0, args.batch,
                                         synthetic.KPP_PAIRS, fused=None if not reference else False)
    batches = []
    for i in range(2):
        r = synthetic.rng_for(300 + i)
        stm, nstm, _, A = synthetic.kppt_indices(r, args.batch, "kpp")
        t, w = synthetic.targets(r, args.batch)
        batches.append((stm, nstm, t, w))
    loss_kind = bo.ScalarLossKind.SigmoidPow(2.0)
    inv = 1.0 / 600.0
    step = 0
    runner.upload_batch(*batches[0], ctx)
    for _ in range(args.warmup):
        step += 1
        runner.step_device(ctx, ranger(step), loss_kind, inv, finalize_loss=False)
    ctx.synchronize()
    start, stop = bo.Event(ctx), bo.Event(ctx)
    with ClockSampler(local) as clocks:
        start.record(ctx)
        for _ in range(args.steps):
            step += 1
            runner.step_device(ctx, ranger(step), loss_kind, inv, finalize_loss=False)
        stop.record(ctx)
        stop.synchronize()
    total_ms = stop.elapsed_ms_since(start)
    e2e_steps = max(4, args.steps // 2)
    # Both batches sit in pinned host memory before the timed region.  This
    # library copies them straight from there (bulletou_b200_*_upload_pinned);
    # the reference library has no such entry and goes through its staged
    # upload (a copy into its pinned staging buffer, then the H2D copy).
    direct = ctx.lib.has("bulletou_b200_i32_upload_pinned")
    pinned = []
    for b in batches:
        bufs = (PinnedI32Buffer(ctx, b[0].size), PinnedI32Buffer(ctx, b[1].size),
                PinnedF32Buffer(ctx, b[2].size), PinnedF32Buffer(ctx, b[3].size))
        if direct:
            for buf, a in zip(bufs, b):
                np.copyto(buf.host(), np.asarray(a).reshape(-1))
        pinned.append(bufs)
    dsts = (runner.stm_indices, runner.nstm_indices, runner.targets, runner.entry_weights)
    e0, e1 = bo.Event(ctx), bo.Event(ctx)
    t0 = time.perf_counter()
    e0.record(ctx)
    for i in range(e2e_steps):
        step += 1
        src = pinned[i % 2]
        if direct:
            for k, (d, p) in enumerate(zip(dsts, src)):
                ctx.lib.call("bulletou_b200_i32_upload_pinned" if k < 2 else "bulletou_b200_f32_upload_pinned",
                             ctx.as_ptr(), d.as_ptr(), p.as_ptr(), p.length)
        else:
            for d, p, a in zip(dsts, src, batches[i % 2]):
                p.upload_to_device(ctx, d, a)
        runner.step_device(ctx, ranger(step), loss_kind, inv, finalize_loss=True)
        runner.read_loss(ctx)
    e1.record(ctx)
    e1.synchronize()
    e2e_ms = max(e1.elapsed_ms_since(e0), (time.perf_counter() - t0) * 1000.0)
    h2d = sum(a.nbytes for a in batches[0])
    return {"total_ms": total_ms, "clocks": clocks.summary(),
            "e2e": {"value": e2e_steps * args.batch / (e2e_ms / 1000.0), "unit": "positions/s",
                    "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": 4 * (3 * args.batch + 2),
                    "steps": e2e_steps}}


# --------------------------------------------------------------------------- roofline
def roofline(phase_ms, batch, hbm_peak, peak_kind, lookahead_frac=1.0 / 6.0):
    """Algorithmic bytes per launch of each phase (formulas below); the
    dominant phase is reported."""
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


# --------------------------------------------------------------------------- SFNN workload
def sfnn_shape():
    from bulletou_b200 import sfnn as bs

    return bs.SFNN_HALFKA_HM2_1536_15_32_K3K3


def make_sfnn_batches(batch, rank=0):
    from bulletou_b200 import synthetic

    return [synthetic.sfnn_batch(2000 + i, batch, rank) for i in range(SFNN_N_BATCHES)]


def sfnn_host_weights():
    from bulletou_b200 import sfnn as bs
    from bulletou_b200 import synthetic

    return bs.SfnnForwardHostWeights(sfnn_shape(), **synthetic.sfnn_weights(synthetic.rng_for(7)))


def sfnn_batches(args, ctx, rank=0, reference=False):
    """(host batches, device batches) of the SFNN workload.  --data psv (the
    default): seeded PackedSfenValue records of full-set positions, decoded to
    HalfKA_hm2 rows, k3k3 buckets and win-rate targets -- on the device by the
    product's producer, by the CPU oracle of the reference's producer on the
    reference arm (the two agree bit for bit on these targets).  --data uniform:
    rows drawn uniformly over the king blocks (synthetic.sfnn_batch)."""
    if args.data == "uniform":
        batches = make_sfnn_batches(args.batch, rank)
        return batches, sfnn_device_batches(ctx, batches)
    from bulletou_b200 import synthetic

    records = [synthetic.psv_records(3000 + i, args.batch, rank) for i in range(SFNN_RECORD_BATCHES)]
    cfg = sfnn_teacher_config()
    if reference:
        from bulletou_b200 import teacher as bt
        from oracle import teacher as ot

        lb = cfg.layerstack_bucket
        ocfg = ot.config("halfka_hm2", cfg.active, lb.hand, lb.king, cfg.lambda_, cfg.scale)
        table = bt.win_rate_model_score_table(cfg.wrm_target)
        host = []
        for r in records:
            o = ot.prepare(r, ocfg, table)
            assert (o["counts"] <= cfg.active).all()
            host.append({"stm": o["stm"].reshape(-1), "nstm": o["nstm"].reshape(-1), "buckets": o["buckets"],
                         "targets": o["targets"], "entry_weights": o["entry_weights"]})
        return host, sfnn_device_batches(ctx, host)
    from bulletou_b200 import teacher as bt

    producer = bt.TeacherBatchProducer(ctx, cfg, args.batch, pinned=False)
    host, dev = [], []
    for r in records:
        tb = producer.new_batch()
        producer.prepare(ctx, r, tb)
        dev.append((tb.stm_indices, tb.nstm_indices, tb.buckets, tb.targets, tb.entry_weights))
        d = tb.download(ctx)
        host.append({"stm": d["stm"].reshape(-1), "nstm": d["nstm"].reshape(-1), "buckets": d["buckets"],
                     "targets": d["targets"], "entry_weights": d["entry_weights"]})
    producer.check(ctx)
    return host, dev


def sfnn_device_batches(ctx, batches):
    import bulletou_b200 as bo

    return [(bo.I32Buffer.from_host(ctx, b["stm"]), bo.I32Buffer.from_host(ctx, b["nstm"]),
             bo.I32Buffer.from_host(ctx, b["buckets"]), bo.F32Buffer.from_host(ctx, b["targets"]),
             bo.F32Buffer.from_host(ctx, b["entry_weights"])) for b in batches]


def bind_sfnn(runner, dev):
    runner.stm_indices, runner.nstm_indices, runner.buckets, runner.targets, runner.entry_weights = dev


SFNN_RECORD_BATCHES = 2


def sfnn_teacher_config():
    """The reference's SFNN trainer defaults (examples/bulletou.rs:5050-5075,
    18846-18866): lambda 1.0, win-rate-model targets (offset 270, scaling 380),
    k3k3 = KingRank9 LayerStack buckets, no score drop."""
    from bulletou_b200 import teacher as bt

    return bt.TeacherBatchConfig(feature_set="halfka_hm2", lambda_=1.0, scale=600.0, win_rate_model=True)


def sfnn_records_e2e(args, ctx, upload_ctx, runner, step, loss_kind, inv):
    """End to end from teacher records: per step the batch's PackedSfenValue
    records (40 bytes a position) go H2D from pinned memory and are decoded on
    the device (HalfKA_hm2 rows, buckets, targets) on the upload stream while
    the previous step trains; the mean loss comes back D2H every step.  Also
    times the decode kernel alone on records resident in HBM."""
    import bulletou_b200 as bo
    from bulletou_b200 import synthetic
    from bulletou_b200 import teacher as bt
    from bulletou_b200.cuda_cpp import PinnedF32Buffer

    producer = bt.TeacherBatchProducer(ctx, sfnn_teacher_config(), args.batch)
    sources = []
    for i in range(SFNN_RECORD_BATCHES):
        slot = bt.TeacherUploadSlot(ctx, producer)
        slot.fill(synthetic.psv_records(3000 + i, args.batch))
        sources.append(slot)
    # decode kernel alone, records resident
    out = producer.new_batch()
    ctx.lib.call("bulletou_b200_i32_upload_pinned", ctx.as_ptr(), producer.records.as_ptr(),
                 sources[0].pinned.as_ptr(), sources[0].pinned.length)
    for _ in range(3):
        producer.decode(ctx, out)
    d0, d1 = bo.Event(ctx), bo.Event(ctx)
    reps = 20
    d0.record(ctx)
    for _ in range(reps):
        producer.decode(ctx, out)
    d1.record(ctx)
    d1.synchronize()
    decode_ms = d1.elapsed_ms_since(d0) / reps
    e2e_steps = max(8, args.steps)
    ring = [PinnedF32Buffer(ctx, 1) for _ in range(e2e_steps)]
    for i in range(3):
        step += 1
        runner.step_pipelined_records(ctx, upload_ctx, producer, ranger(step), loss_kind, inv, None, True,
                                      sources[i % len(sources)], ring[i])
    ctx.synchronize()
    upload_ctx.synchronize()
    e0, e1 = bo.Event(ctx), bo.Event(ctx)
    h2d = 0
    t0 = time.perf_counter()
    e0.record(ctx)
    for i in range(e2e_steps):
        step += 1
        h2d = runner.step_pipelined_records(ctx, upload_ctx, producer, ranger(step), loss_kind, inv, None, True,
                                            sources[i % len(sources)], ring[i])
    e1.record(ctx)
    e1.synchronize()
    wall_ms = (time.perf_counter() - t0) * 1000.0
    e2e_ms = max(e1.elapsed_ms_since(e0), wall_ms)
    producer.check(ctx)
    losses = [float(r.host()[0]) for r in ring]
    assert all(np.isfinite(losses)), "non-finite loss"
    e2e = {"value": e2e_steps * args.batch / (e2e_ms / 1000.0), "unit": "positions/s",
           "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": 4, "steps": e2e_steps,
           "path": "SfnnTrainStepRunner.step_pipelined_records: PackedSfenValue records in pinned host memory -> "
                   "H2D (40 B/position) -> device decode to HalfKA_hm2 rows / k3k3 buckets / win-rate targets "
                   "(bulletou_b200_teacher_prepare_device) on the upload stream -> fused train step; mean loss "
                   "copied D2H every step"}
    producer_line = {"kernel": "teacher_psv_kernel", "ms_per_batch": round(decode_ms, 4),
                     "positions_per_s": round(args.batch / (decode_ms / 1000.0), 1),
                     "record_bytes_per_s": round(40 * args.batch / (decode_ms / 1000.0), 1)}
    return e2e, producer_line, step


def sfnn_cpu_baseline(batch_cap=256, budget_s=8.0):
    """The reference's CPU evaluation path for SFNN -- the engine's integer
    forward over the exported quantised network (examples/bulletou.rs:
    8001-8163, rayon over positions there) -- as the C oracle's restatement,
    one thread, on a bounded sample."""
    from bulletou_b200 import synthetic
    from oracle import oracle

    sh = sfnn_shape()
    w = synthetic.sfnn_weights(synthetic.rng_for(7))
    q = oracle.sfnn_quantize(sh.as_tuple(), w)
    b = synthetic.sfnn_batch(4242, batch_cap)
    args = (sh.as_tuple(), b["stm"], b["nstm"], b["buckets"])
    oracle.sfnn_integer_forward(sh.as_tuple(), b["stm"][:SFNN_ACTIVE * 8], b["nstm"][:SFNN_ACTIVE * 8],
                                b["buckets"][:8], 8, SFNN_ACTIVE, q)  # warm
    t0 = time.perf_counter()
    reps = 0
    while True:
        oracle.sfnn_integer_forward(*args, batch_cap, SFNN_ACTIVE, q)
        reps += 1
        if time.perf_counter() - t0 >= budget_s:
            break
    dt = time.perf_counter() - t0
    return {"value": reps * batch_cap / dt, "unit": "positions/s (integer forward evaluation only)", "cores": 1,
            "kind": "port",
            "sample": f"oracle quantised SFNN 1536 integer forward (the reference's CPU evaluator), {reps} x "
                      f"{batch_cap} positions in {dt:.1f} s; the reference cannot train on CPU"}


def teacher_cpu_baseline(n=16384, budget_s=6.0):
    """The reference's teacher-batch producer for this workload
    (prepare_sfnn_fast_batch_from_board_features, teacher_batch.rs:2869-3010)
    as the C oracle's restatement, one thread, on a bounded sample."""
    from bulletou_b200 import synthetic
    from oracle import teacher as ot

    recs = synthetic.psv_records(4343, n)
    cfg = sfnn_teacher_config()
    lb = cfg.layerstack_bucket
    ocfg = ot.config("halfka_hm2", cfg.active, lb.hand, lb.king, cfg.lambda_, cfg.scale)
    from bulletou_b200 import teacher as bt

    table = bt.win_rate_model_score_table(cfg.wrm_target)
    ot.prepare(recs[:64], ocfg, table)
    t0 = time.perf_counter()
    reps = 0
    while True:
        ot.prepare(recs, ocfg, table)
        reps += 1
        if time.perf_counter() - t0 >= budget_s:
            break
    dt = time.perf_counter() - t0
    return {"value": round(reps * n / dt, 1), "unit": "positions/s", "cores": 1, "kind": "port",
            "sample": f"oracle PackedSfenValue -> HalfKA_hm2 batch producer, {reps} x {n} records in {dt:.1f} s"}


def sfnn_phases(qat):
    """Stage-profiler phases of one fused step (the integer FT of the dense
    QAT with FT QAT is a phase of its own)."""
    l1, ft, l2, l3 = SFNN_QAT_MODES[qat]
    if ft and l1 and l2 and l3:
        return SFNN_PHASES[:4] + ("ft_integer",) + SFNN_PHASES[4:]
    return SFNN_PHASES


def _profile(lib, ctx, names):
    import ctypes

    ms = (ctypes.c_float * 16)()
    nsteps, nphases = ctypes.c_size_t(), ctypes.c_size_t()
    lib.call("bulletou_b200_profile_end", ctx.as_ptr(), ms, 16, ctypes.byref(nsteps), ctypes.byref(nphases))
    return {names[p]: ms[p] / max(1, nsteps.value) for p in range(min(nphases.value, len(names)))}


def run_sfnn_b200(args, rank, world, local, dist):
    import bulletou_b200 as bo
    from bulletou_b200 import sfnn as bs
    from bulletou_b200.cuda_cpp import PinnedF32Buffer

    if world > 1:
        return run_sfnn_data_parallel(args, rank, world, local, dist)
    ctx = bo.Context(local)
    runner = bs.SfnnTrainStepRunner(ctx, sfnn_host_weights(), args.batch, SFNN_ACTIVE, fused=True,
                                    lr_multipliers=sfnn_lr_multipliers(args.qat))
    batches, devb = sfnn_batches(args, ctx, rank)
    loss_kind = bo.ScalarLossKind.SigmoidPow(2.0)
    inv = 1.0 / 600.0
    step = 0
    for i in range(args.warmup):
        step += 1
        bind_sfnn(runner, devb[i % len(devb)])
        runner.step_device(ctx, ranger(step), loss_kind, inv, finalize_loss=False)
    ctx.synchronize()
    lib = ctx.lib
    start, stop = bo.Event(ctx), bo.Event(ctx)
    lib.call("bulletou_b200_profile_begin", ctx.as_ptr(), 10 * args.steps + 10)
    with ClockSampler(local) as clocks:
        start.record(ctx)
        for i in range(args.steps):
            step += 1
            bind_sfnn(runner, devb[i % len(devb)])
            runner.step_device(ctx, ranger(step), loss_kind, inv, finalize_loss=False)
        stop.record(ctx)
        stop.synchronize()
    phase_ms = _profile(lib, ctx, sfnn_phases(args.qat))
    total_ms = stop.elapsed_ms_since(start)
    clk = clocks.summary()
    # ---- end to end through the public runner API (pipelined step, lib.rs:7627) ----
    upload_ctx = bo.Context(local)
    sources = []
    for b in batches:  # the data loader's output: batches already in pinned host memory
        slot = bs.SfnnTrainStepUploadSlot(ctx, args.batch, SFNN_ACTIVE)
        slot.fill(bs.SfnnTrainStepHostBatch(b["stm"], b["nstm"], b["buckets"], b["targets"], b["entry_weights"],
                                            args.batch, SFNN_ACTIVE))
        sources.append(slot)
    e2e_steps = max(8, args.steps)
    loss_ring = [PinnedF32Buffer(ctx, 1) for _ in range(e2e_steps)]
    for i in range(3):
        step += 1
        runner.step_pipelined_no_readback_with_loss_finalize(ctx, upload_ctx, ranger(step), loss_kind, inv, None, True,
                                                             sources[i % len(sources)], loss_ring[i])
    ctx.synchronize()
    upload_ctx.synchronize()
    h2d = 0
    e0, e1 = bo.Event(ctx), bo.Event(ctx)
    t0 = time.perf_counter()
    e0.record(ctx)
    for i in range(e2e_steps):
        step += 1
        h2d = runner.step_pipelined_no_readback_with_loss_finalize(ctx, upload_ctx, ranger(step), loss_kind, inv, None,
                                                                   True, sources[i % len(sources)], loss_ring[i])
    e1.record(ctx)
    e1.synchronize()
    wall_ms = (time.perf_counter() - t0) * 1000.0
    losses = [float(r.host()[0]) for r in loss_ring]
    e2e_ms = max(e1.elapsed_ms_since(e0), wall_ms)
    assert all(np.isfinite(losses)), "non-finite loss"
    e2e_prepared = {"value": e2e_steps * args.batch / (e2e_ms / 1000.0), "unit": "positions/s",
                    "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": 4, "steps": e2e_steps,
                    "path": "SfnnTrainStepRunner.step_pipelined_no_readback_with_loss_finalize (2 upload slots, "
                            "second stream), prepared sparse batches in pinned host memory, mean loss copied D2H "
                            "every step"}
    e2e, producer_line, step = sfnn_records_e2e(args, ctx, upload_ctx, runner, step, loss_kind, inv)
    return {
        "total_ms": total_ms, "phase_ms": phase_ms, "clocks": clk,
        "e2e": e2e, "e2e_prepared_batches": e2e_prepared, "producer": producer_line,
        "gpu_launches": sfnn_launches_per_step(args.qat) * args.steps,
        "final_loss": losses[-1],
    }


def run_sfnn_data_parallel(args, rank, world, local, dist):
    """N > 1: weak scaling, args.batch positions per rank (NCCL exchange)."""
    import torch

    import bulletou_b200 as bo
    from bulletou_b200.cuda_cpp import F32Buffer, I32Buffer, PinnedF32Buffer, PinnedI32Buffer
    from bulletou_b200.data_parallel import B200Backend, SfnnDataParallelTrainer

    backend = B200Backend(local)
    ctx, lib = backend.ctx, backend.lib
    tr = SfnnDataParallelTrainer(backend, dist, sfnn_host_weights(), args.batch, SFNN_ACTIVE,
                                 lr_multipliers=sfnn_lr_multipliers(args.qat),
                                 launches_per_chunk=args.dp_chunk_launches)
    batches, devb = sfnn_batches(args, ctx, rank)
    loss_kind = bo.ScalarLossKind.SigmoidPow(2.0)
    inv = 1.0 / 600.0
    step = 0

    def bind(i):
        tr.stm_indices, tr.nstm_indices, tr.buckets, tr.targets, tr.entry_weights = devb[i % len(devb)]

    for i in range(args.warmup):
        step += 1
        bind(i)
        tr.step_device(ranger(step), loss_kind, inv, finalize_loss=False)
    torch.cuda.synchronize()
    dist.barrier()
    start, stop = bo.Event(ctx), bo.Event(ctx)
    lib.call("bulletou_b200_profile_begin", ctx.as_ptr(), 10 * args.steps + 10)
    with ClockSampler(local) as clocks:
        start.record(ctx)
        for i in range(args.steps):
            step += 1
            bind(i)
            tr.step_device(ranger(step), loss_kind, inv, finalize_loss=False)
        tr.join()  # the last step's exchange runs on the comm stream
        stop.record(ctx)
        stop.synchronize()
    phase_ms = _profile(lib, ctx, sfnn_phases(args.qat))
    torch.cuda.synchronize()
    dist.barrier()
    total_ms = max_over_ranks(dist, stop.elapsed_ms_since(start))
    # end to end: per step H2D from pinned host memory, step, D2H of the mean loss
    pins = []
    for b in batches:
        p = (PinnedI32Buffer(ctx, b["stm"].size), PinnedI32Buffer(ctx, b["nstm"].size),
             PinnedI32Buffer(ctx, args.batch), PinnedF32Buffer(ctx, args.batch), PinnedF32Buffer(ctx, args.batch))
        for dst, src in zip(p, (b["stm"], b["nstm"], b["buckets"], b["targets"], b["entry_weights"])):
            np.copyto(dst.host(), src)
        pins.append(p)
    n = args.batch * SFNN_ACTIVE
    in_bufs = (I32Buffer(ctx, n), I32Buffer(ctx, n), I32Buffer(ctx, args.batch), F32Buffer(ctx, args.batch),
               F32Buffer(ctx, args.batch))
    tr.stm_indices, tr.nstm_indices, tr.buckets, tr.targets, tr.entry_weights = in_bufs
    e2e_steps = max(8, args.steps)
    ring = [PinnedF32Buffer(ctx, 1) for _ in range(e2e_steps)]
    dist.barrier()
    e0, e1 = bo.Event(ctx), bo.Event(ctx)
    t0 = time.perf_counter()
    e0.record(ctx)
    h2d = 0
    for i in range(e2e_steps):
        step += 1
        p = pins[i % len(pins)]
        c = ctx.as_ptr()
        for dst, src in zip(in_bufs, p):
            name = "bulletou_b200_i32_upload_pinned" if isinstance(dst, I32Buffer) else "bulletou_b200_f32_upload_pinned"
            lib.call(name, c, dst.as_ptr(), src.as_ptr(), src.length)
        h2d = 4 * sum(x.length for x in p)
        tr.step_device(ranger(step), loss_kind, inv, finalize_loss=True)
        lib.call("bulletou_b200_f32_download_pinned", c, ring[i].as_ptr(), tr.loss_workspace.mean.as_ptr(), 1)
    tr.join()
    e1.record(ctx)
    e1.synchronize()
    wall_ms = (time.perf_counter() - t0) * 1000.0
    e2e_ms = max_over_ranks(dist, max(e1.elapsed_ms_since(e0), wall_ms))
    losses = [float(r.host()[0]) for r in ring]
    assert all(np.isfinite(losses)), "non-finite loss"
    # the fused row kernel becomes a gradient-write pass; Ranger runs per group on the shard
    return {"total_ms": total_ms, "phase_ms": phase_ms, "clocks": clocks.summary(),
            "e2e": {"value": e2e_steps * args.batch * world / (e2e_ms / 1000.0), "unit": "positions/s",
                    "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": 4, "steps": e2e_steps,
                    "path": "SfnnDataParallelTrainer.step_device per rank (NCCL reduce-scatter / all-reduce / "
                            "all-gather), inputs from pinned host memory, mean loss copied D2H every step"},
            "gpu_launches": (sfnn_launches_per_step(args.qat) + 1) * args.steps,
            "final_loss": losses[-1]}


def run_sfnn_reference(args, local):
    import bulletou_b200 as bo
    from bulletou_b200 import sfnn as bs

    lib = bo.reference_library()
    ctx = bo.Context(local, lib)
    runner = bs.SfnnTrainStepRunner(ctx, sfnn_host_weights(), args.batch, SFNN_ACTIVE, fused=False,
                                    lr_multipliers=sfnn_lr_multipliers(args.qat))
    batches, devb = sfnn_batches(args, ctx, 0, reference=True)
    loss_kind = bo.ScalarLossKind.SigmoidPow(2.0)
    inv = 1.0 / 600.0
    step = 0
    for i in range(args.warmup):
        step += 1
        bind_sfnn(runner, devb[i % len(devb)])
        runner.step_device(ctx, ranger(step), loss_kind, inv, finalize_loss=False)
    ctx.synchronize()
    start, stop = bo.Event(ctx), bo.Event(ctx)
    with ClockSampler(local) as clocks:
        start.record(ctx)
        for i in range(args.steps):
            step += 1
            bind_sfnn(runner, devb[i % len(devb)])
            runner.step_device(ctx, ranger(step), loss_kind, inv, finalize_loss=False)
        stop.record(ctx)
        stop.synchronize()
    total_ms = stop.elapsed_ms_since(start)
    clk = clocks.summary()
    upload_ctx = bo.Context(local, lib)
    hbs = [bs.SfnnTrainStepHostBatch(b["stm"], b["nstm"], b["buckets"], b["targets"], b["entry_weights"], args.batch,
                                     SFNN_ACTIVE) for b in batches]
    e2e_steps = max(4, args.steps // 2)
    for i in range(2):
        step += 1
        runner.step_pipelined_no_readback_with_loss_finalize(ctx, upload_ctx, ranger(step), loss_kind, inv,
                                                             hbs[i % len(hbs)], True)
        runner.loss_workspace.mean.download(ctx)
    ctx.synchronize()
    e0, e1 = bo.Event(ctx), bo.Event(ctx)
    t0 = time.perf_counter()
    e0.record(ctx)
    h2d = 0
    for i in range(e2e_steps):
        step += 1
        h2d = runner.step_pipelined_no_readback_with_loss_finalize(ctx, upload_ctx, ranger(step), loss_kind, inv,
                                                                   hbs[i % len(hbs)], True)
        runner.loss_workspace.mean.download(ctx)
    e1.record(ctx)
    e1.synchronize()
    e2e_ms = max(e1.elapsed_ms_since(e0), (time.perf_counter() - t0) * 1000.0)
    return {"total_ms": total_ms, "clocks": clk,
            "e2e": {"value": e2e_steps * args.batch / (e2e_ms / 1000.0), "unit": "positions/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4, "steps": e2e_steps}}


# DRAM bytes per step of each phase at B = 65536 (dram__bytes_read.sum +
# dram__bytes_write.sum over the phase's launches), from a full-size ncu
# capture of `bench.py --steps 1 --warmup 3 --data uniform`; keyed by the QAT
# modes whose kernels they were measured on.
SFNN_DRAM_BYTES_B65536 = {
    "ft_rows_ranger": (4813480704, ("none", "l1", "layers", "dense", "all")),
    "ft_forward": (1679058432, ("none", "l1", "dense", "all")),
    "ft_integer": (613106176, ("all",)),
    "l1_backward": (2076098304, ("dense", "all")),
    "fold": (1124865536, ("all",)),
}

# The same on the default --data psv batches (decoded PackedSfenValue records;
# capture of `bench.py --steps 1 --warmup 3 --no-cpu-baseline`).
SFNN_DRAM_BYTES_PSV_B65536 = {
    "ft_rows_ranger": (4668284928, ("all",)),
    "ft_forward": (1181817600, ("all",)),
    "ft_integer": (570697728, ("all",)),
    "l1_backward": (2068230656, ("all",)),
    "fold": (1125304832, ("all",)),
}


def sfnn_roofline(phase_ms, batch, hbm_peak, peak_kind, lookahead_frac=1.0 / 6.0, qat="none", data="psv"):
    """Algorithmic bytes per launch of each SFNN phase (the per-position
    formulas of the hot-path table; gathers counted at their logical size, so
    a fraction above 1 means L2 serves the repeated rows)."""
    sh = sfnn_shape()
    W, A = sh.ft_size, SFNN_ACTIVE
    rows = sh.input_size
    base = sh.factorized_base()
    half_positions = 2 * batch
    algo = {
        "fold": base * W * 4 * 2 + 1629 * W * 4,
        # logical rows gathered + indices + ClippedReLU outputs (2 views) and combined written
        "ft_forward": half_positions * A * W * 4 + half_positions * A * 4 + 3 * batch * W * 4,
        # every FT row's optimizer state (w, m, v read + written; slow on lookahead steps)
        # + the pre-activation gradients gathered (logical) + the inverse index
        "ft_rows_ranger": rows * W * 4 * (6 + 2 * lookahead_frac) + half_positions * A * W * 4
                          + 4 * (half_positions * A + base + 1),
        # both views' FT outputs read, pre-activation gradients written, L1 weight partials
        "l1_backward": 2 * batch * W * 4 + 2 * batch * W * 4 + (batch // 128 + 11) * 16 * W * 4,
        "l1_head": batch * W * 4 + batch * 4 * (16 + 30 + 32 + 16 + 4),
        "inverse_index": 4 * (half_positions * A * 3 + base * 4),
        "sorts_tiles": 4 * (half_positions * A + 4 * half_positions + 3 * batch),
        "small_grads_ranger": 0.0,
    }
    l1, ft, l2, l3 = SFNN_QAT_MODES[qat]
    if ft and l1 and l2 and l3:
        # the fold also writes the i16 table; the integer FT gathers it (logical) and rewrites combined
        algo["fold"] += base * W * 2
        algo["ft_integer"] = half_positions * A * W * 2 + half_positions * A * 4 + batch * W * 4
    if l1 and l2 and l3:
        algo["l1_backward"] += batch * W * 4  # the lattice FT output read for dL1w
    dom = max(phase_ms, key=phase_ms.get)
    t = phase_ms[dom] / 1000.0
    achieved = algo.get(dom, 0.0) / t / 1e9 if t > 0 else 0.0
    traffic = None
    measured = (SFNN_DRAM_BYTES_B65536 if data == "uniform" else SFNN_DRAM_BYTES_PSV_B65536).get(dom)
    if measured is not None and batch == SFNN_BATCH and qat in measured[1]:
        traffic = measured[0]
    launches = 15 if dom == "ft_rows_ranger" else 1
    return {"bound": "hbm", "kernel": dom, "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
            "frac": round(achieved / hbm_peak, 4), "peak_source": peak_kind, "traffic": traffic,
            "traffic_note": "DRAM bytes of the phase per step (ncu capture); algorithmic bytes count the "
                            "logical row gathers, which L2 serves, so traffic is far below them",
            "launches_per_step": launches,
            "algorithmic_bytes_per_step": int(algo.get(dom, 0.0)), "kernel_ms_per_step": round(phase_ms[dom], 4),
            "phase_ms": {k: round(v, 4) for k, v in phase_ms.items()}}


def main():
    args = parse_args()
    rank, world, local, dist = dist_setup(args)
    if args.warmup < 3:
        args.warmup = 3
    sfnn = args.workload == "sfnn"
    if args.batch is None:
        args.batch = {"sfnn": SFNN_BATCH, "halfkp": BATCH, "kppt": KPPT_BATCH}[args.workload]
    if args.workload == "kppt":
        if rank == 0:
            r = run_kppt(args, local, reference=args.impl == "reference")
            line = {"metric": KPPT_METRIC, "unit": "positions/s", "n_gpus": 1, "steps": args.steps,
                    "warmup": args.warmup, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                    "dtype": "f32", "data": "synthetic (seeded KPP pairs, reference shapes)",
                    "config": {"workload": "configs[3] KPPT KPP component train step (Ranger, as the reference's "
                                           "KPPT runner; the reference has no AdaGrad)",
                               "global_batch": args.batch, "pairs": 703, "table": 194100624},
                    "value": round(args.steps * args.batch / (r["total_ms"] / 1000.0), 1),
                    "ms_per_step": round(r["total_ms"] / args.steps, 4), "clocks": r["clocks"],
                    "e2e": {k: (round(v, 1) if isinstance(v, float) else v) for k, v in r["e2e"].items()}}
            if args.impl == "reference":
                line["impl"] = "reference"
            print(json.dumps(line))
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()
        return
    common = {"global_batch": args.batch * world, "per_gpu_batch": args.batch, "seq_len": 1,
              "optimizer": "Ranger (RAdam + Lookahead k=6, lr 1e-3)",
              "loss": "sigmoid-pow(2) MSE of the output, scale 600",
              "parallelism": f"dp{world}" if world > 1 else "single"}
    if sfnn:
        metric = SFNN_METRIC
        config = dict({"workload": "configs[2] SFNN HalfKA_hm2 1536x2 LayerStack k3k3 train step",
                       "model": "SFNN_halfkahm2_1536_15_32_k3k3: (73305+1629 virtual) x 1536 FT, pairwise, "
                                "9 x (1536 -> 15+1), shared L1 factor, 30 -> 32 -> 1",
                       "max_active": SFNN_ACTIVE,
                       "targets": ("win-rate-model probability of the teacher score (offset 270, scaling 380), "
                                   "lambda 1" if args.data == "psv" else "0.5 result + 0.5 sigmoid(score / 600)"),
                       "data": ("seeded PackedSfenValue records (full-set positions, kings near their home ranks) "
                                "decoded to HalfKA_hm2 rows / k3k3 buckets / win-rate targets"
                                if args.data == "psv" else "feature rows uniform over the 45 king blocks, "
                                                           "buckets uniform 0..8"),
                       "qat": f"{args.qat}: {SFNN_QAT_LABELS[args.qat]}",
                       "l2": "no flush: each step streams 1.8 GB of FT optimizer state (> 126 MB L2)"}, **common)
    else:
        metric = METRIC
        config = dict({"workload": "configs[1] HalfKP 256x2-32-32-1 train step",
                       "model": "HalfKP 125388x256x2-32-32-1", "max_active": ACTIVE,
                       "l2": "no flush: each step streams 0.5 GB of optimizer state (> 126 MB L2)"}, **common)
    base = {"metric": metric, "unit": "positions/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded; reference teacher-data shapes and distributions)", "config": config}
    if args.impl == "reference":
        if rank != 0:
            return
        try:
            r = run_sfnn_reference(args, local) if sfnn else run_reference(args, local)
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
                                  "sample": f"{args.steps} steps x {args.batch} positions on the GPU: the reference's "
                                            f"implementation of this path is its CUDA backend (not a CPU run)"})
        print(json.dumps(line))
        return
    r = run_sfnn_b200(args, rank, world, local, dist) if sfnn else run_b200(args, rank, world, local, dist)
    value = args.steps * args.batch * world / (r["total_ms"] / 1000.0)
    if rank == 0:
        hbm, kind = measured_peaks()
        rl = (sfnn_roofline(r["phase_ms"], args.batch, hbm, kind, qat=args.qat, data=args.data) if sfnn
              else roofline(r["phase_ms"], args.batch, hbm, kind))
        line = dict(base, value=round(value, 1), ms_per_step=round(r["total_ms"] / args.steps, 4),
                    e2e={k: (round(v, 1) if isinstance(v, float) else v) for k, v in r["e2e"].items()},
                    roofline=rl, clocks=r["clocks"], gpu_launches=r["gpu_launches"], final_loss=r["final_loss"])
        for extra in ("e2e_prepared_batches", "producer"):
            if extra in r:
                line[extra] = {k: (round(v, 1) if isinstance(v, float) else v) for k, v in r[extra].items()}
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = sfnn_cpu_baseline() if sfnn else cpu_baseline()
            if "producer" in line:
                line["producer"]["cpu_baseline"] = teacher_cpu_baseline()
        print(json.dumps(line))
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
