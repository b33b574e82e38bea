#!/usr/bin/env python3
"""Benchmark: BulletOu training hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--workload sfnn|sfnn_k9k9|halfkp|halfkp_fwd|kppt]

Workloads (a train "step" = forward, sigmoid-pow loss,
backward and Ranger over every parameter):

* sfnn (default, configs[2], the north-star target): SFNN HalfKA_hm2 1536x2
  -> LayerStack k3k3 (9 buckets) 1536 -> 15+1 -> 32 -> 1 with the FT
  factorizer (+1629 virtual rows) and the shared L1 factor, all-layer QAT,
  65536 positions per GPU (weak scaling with N);
* sfnn_k9k9: the same net with 81 LayerStack buckets drawn
  Zipf(1.1), global batch 262144 split over the N GPUs (strong scaling);
* halfkp: HalfKP 256x2-32-32-1 train step, 16384 positions;
* halfkp_fwd: HalfKP forward only, f32 through the drop-in
  forward entry and the engine's int16 FT / int8 dense integer forward,
  16384 positions, L2 flushed before every timed forward;
* kppt: KPP component-table train step, 32768 positions.

Seeded synthetic inputs with the reference teacher data's shapes and
distributions (bulletou_b200/synthetic.py; SFNN rows decoded from seeded
PackedSfenValue records).  Prints one JSON line (rank 0):

* value      positions/s with the batches resident in HBM (CUDA events on
             the library's stream, max over ranks);
* e2e        the same metric end to end through the runner API: per step the
             batch goes H2D from page-locked host memory (the drop-in ABI's
             *_upload entries, an upload stream overlapping the previous step)
             and the step's mean loss comes back D2H synchronously -- exactly
             the same calls for this library and the reference arm;
* roofline   the dominant phase against the measured HBM copy peak
             (MEASURED_PEAKS.json) on its compulsory DRAM bytes; the logical
             row-gather bytes go against an L2 read peak measured in-run;
* cpu_baseline  the reference's CPU evaluation path (the C oracle's
             restatement) on every host core, on a bounded sample.

--impl reference times the reference's own cuda-cpp backend (built from its
sources into oracle/_ref; it has no CPU training path) through the reference
runner's call sequence, on the same GPU, config and metric.
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
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

# HalfKP
BATCH = 16384
ACTIVE = 38
SHAPE = (125388, 256, 32, 32)
N_BATCHES = 8
METRIC = "train positions/sec (HalfKP 256x2-32-32-1, batch 16384)"
FWD_METRIC = "forward positions/sec (HalfKP 256x2-32-32-1, f32, batch 16384)"
PHASES = ("inverse_index", "king_sort", "ft_gather", "dense_fwd_loss_bwd", "batch_reduce", "small_param_ranger",
          "ft_row_grad_ranger")
LAUNCHES_PER_STEP = 13  # index 5 + king sort 3 + gather, dense, reduce, finalize, rows
FWD_LAUNCHES = 5        # king sort 3 + FT gather + dense (either forward)

# SFNN
SFNN_BATCH = 65536
SFNN_ACTIVE = 40
K9K9_GLOBAL_BATCH = 262144
SFNN_N_BATCHES = 4
SFNN_METRIC = "train positions/sec (SFNN HalfKA_hm2 1536x2 LayerStack k3k3 15+1-32-1, batch 65536 per GPU)"
K9K9_METRIC = "train positions/sec (SFNN HalfKA_hm2 1536x2 LayerStack k9k9 15+1-32-1, global batch 262144)"
SFNN_PHASES = ("sorts_tiles", "inverse_index", "fold", "ft_forward", "l1_head", "l1_backward", "small_grads_ranger",
               "ft_rows_ranger")
# fold 1, king sort 3, bucket sort 3, king tiles + tile table 2, L1 weights 1, index 5 + row sort 1, FT forward 1,
# L1 forward 1, head 1, L1 backward 1, finalize 1, Ranger on 9 small groups, heavy keys 5 (plan 3, incidence,
# tensor-core sums), FT rows 45 kings / 3
SFNN_LAUNCHES_PER_STEP = 1 + 3 + 3 + 2 + 1 + 6 + 1 + 1 + 1 + 1 + 1 + 9 + 5 + 15
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
SFNN_RECORD_BATCHES = 2


@dataclass(frozen=True)
class SfnnWorkload:
    """One SFNN configuration of BASELINE.json."""

    key: str
    stacks: int
    zipf: float
    metric: str
    label: str
    strong: bool  # global batch fixed (split over the ranks) instead of per-rank batch

    def shape(self):
        from bulletou_b200 import sfnn as bs

        if self.stacks == 9:
            return bs.SFNN_HALFKA_HM2_1536_15_32_K3K3
        return bs.SfnnForwardShape(bs.HALFKA_HM2_DIMENSIONS + bs.PIECE_INPUTS, 1536, 15, True, 32, self.stacks)

    def batches(self, override, world):
        """(per-rank batch, global batch)."""
        if self.strong:
            g = override or K9K9_GLOBAL_BATCH
            if g % world:
                raise SystemExit(f"global batch {g} is not divisible by {world} ranks")
            return g // world, g
        b = override or SFNN_BATCH
        return b, b * world


SFNN_K3K3 = SfnnWorkload("sfnn", 9, 0.0, SFNN_METRIC, "configs[2] SFNN HalfKA_hm2 1536x2 LayerStack k3k3 train step",
                         False)
SFNN_K9K9 = SfnnWorkload("sfnn_k9k9", 81, 1.1, K9K9_METRIC,
                         "configs[4] SFNN HalfKA_hm2 1536x2 LayerStack k9k9 (81 buckets, Zipf(1.1)) train step, "
                         "global batch split over the GPUs", True)
SFNN_WORKLOADS = {w.key: w for w in (SFNN_K3K3, SFNN_K9K9)}


def sfnn_lr_multipliers(mode):
    from bulletou_b200 import sfnn as bs

    l1, ft, l2, l3 = SFNN_QAT_MODES[mode]
    return bs.SfnnLayerLrMultipliers(qat_l1=l1, qat_ft=ft, qat_l2=l2, qat_l3=l3)


def sfnn_launches_per_step(mode):
    """Kernels of one fused step: the QAT extras are the L1 bias fold (L1 QAT)
    and the FT bias rounding (FT QAT); the engine's integer FT of the dense QAT
    with FT QAT comes out of the FT forward's own gather."""
    l1, ft, l2, l3 = SFNN_QAT_MODES[mode]
    return SFNN_LAUNCHES_PER_STEP + int(l1) + int(ft)


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("b200", "reference"), default="b200")
    ap.add_argument("--workload", choices=("sfnn", "sfnn_k9k9", "halfkp", "halfkp_fwd", "kppt"), default="sfnn")
    ap.add_argument("--batch", type=int, default=None,
                    help="per-GPU batch (sfnn, halfkp, kppt) or global batch (sfnn_k9k9)")
    ap.add_argument("--dp-chunk-launches", type=int, default=3,
                    help="N > 1: FT row launches per exchanged chunk (SFNN)")
    ap.add_argument("--dp-exchange", choices=("p2p", "collectives"), default="p2p",
                    help="N > 1 (SFNN): FT rows exchanged over peer memory by the row kernels, or through NCCL "
                         "reduce-scatter / all-gather")
    ap.add_argument("--dp-last-chunk-launches", type=int, default=1,
                    help="N > 1: FT row launches of the last exchanged chunk (SFNN; 0: no separate last chunk)")
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


def ranger(step):
    import bulletou_b200 as bo

    return bo.RangerUpdateParams(radam=bo.RAdamUpdateParams(step=step, learning_rate=1e-3))


def rounded(d):
    return {k: (round(v, 1) if isinstance(v, float) else v) for k, v in d.items()}


class PinnedHostBatch:
    """A batch in page-locked host memory (torch pin_memory), as the data
    loader hands it over; `.pinned` is what the runners' upload slots copy from
    with the drop-in ABI's *_upload entries."""

    def __init__(self, arrays):
        import torch

        self._keep = []
        views = []
        for a in arrays:
            a = np.ascontiguousarray(a).reshape(-1)
            t = torch.empty(a.size, dtype=torch.int32 if a.dtype == np.int32 else torch.float32, pin_memory=True)
            v = t.numpy()
            np.copyto(v, a)
            self._keep.append(t)
            views.append(v)
        self.pinned = tuple(views)

    @property
    def nbytes(self):
        return sum(v.nbytes for v in self.pinned)


def pipelined_e2e(runner, ctx, upload_ctx, sources, steps, step, loss_kind, inv):
    """Page-locked host batches through the runner's upload slots: step i runs
    on its slot while the batch of step i + 1 is uploaded on a second stream
    (issued right after step i is enqueued), then the step's mean loss is read
    back synchronously (the drop-in ABI's download).  Every step's batch is
    copied H2D and every step's loss read D2H inside the timed region.
    Identical calls for every backend library."""
    import bulletou_b200 as bo

    n = len(sources)
    runner.upload_next(upload_ctx, None, sources[0])
    for i in range(3):
        step += 1
        runner.step_uploaded_no_readback_with_loss_finalize(ctx, ranger(step), loss_kind, inv, True)
        runner.upload_next(upload_ctx, None, sources[(i + 1) % n])
        runner.loss_workspace.mean.download(ctx)
    step += 1  # the warm-up's last upload is consumed here, outside the timed region
    runner.step_uploaded_no_readback_with_loss_finalize(ctx, ranger(step), loss_kind, inv, True)
    runner.loss_workspace.mean.download(ctx)
    ctx.synchronize()
    upload_ctx.synchronize()
    e0, e1 = bo.Event(ctx), bo.Event(ctx)
    losses = []
    h2d = 0
    t0 = time.perf_counter()
    e0.record(ctx)
    h2d = runner.upload_next(upload_ctx, None, sources[0])
    for i in range(steps):
        step += 1
        runner.step_uploaded_no_readback_with_loss_finalize(ctx, ranger(step), loss_kind, inv, True)
        if i + 1 < steps:
            runner.upload_next(upload_ctx, None, sources[(i + 1) % n])
        losses.append(float(runner.loss_workspace.mean.download(ctx)[0]))
    e1.record(ctx)
    e1.synchronize()
    ms = max(e1.elapsed_ms_since(e0), (time.perf_counter() - t0) * 1000.0)
    assert all(np.isfinite(losses)), "non-finite loss"
    return {"ms": ms, "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": 4, "steps": steps,
            "final_loss": losses[-1]}, step


def measure_l2_peak(ctx, megabytes=64, passes=8, reps=6):
    """L2 read peak: this library's probe kernel reads a 64 MB buffer (inside
    the 126 MB L2) `passes` times per launch; best of `reps` launches."""
    import bulletou_b200 as bo

    n = megabytes * (1 << 20) // 4
    buf = bo.F32Buffer(ctx, n)
    buf.fill(1.0, ctx)
    sink = bo.F32Buffer(ctx, 512 * 4 * 256)
    lib = ctx.lib
    for _ in range(2):
        lib.call("bulletou_b200_l2_read_probe", ctx.as_ptr(), buf.as_ptr(), n, passes, sink.as_ptr())
    best = float("inf")
    for _ in range(reps):
        e0, e1 = bo.Event(ctx), bo.Event(ctx)
        e0.record(ctx)
        lib.call("bulletou_b200_l2_read_probe", ctx.as_ptr(), buf.as_ptr(), n, passes, sink.as_ptr())
        e1.record(ctx)
        e1.synchronize()
        best = min(best, e1.elapsed_ms_since(e0))
    gbs = passes * n * 4 / (best / 1000.0) / 1e9
    return {"value": round(gbs, 1), "unit": "GB/s", "how": f"bulletou_b200_l2_read_probe: {megabytes} MB buffer, "
            f"{passes} passes of 16-byte ld.global.cg per launch, best of {reps} launches (CUDA events)"}


def flush_l2(ctx, scratch):
    """Writes a buffer larger than L2 (126 MB) on the context stream."""
    scratch.fill(0.0, ctx)


# --------------------------------------------------------------------------- CPU baselines
def host_cpu():
    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    model = "unknown"
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                model = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    return cores, model


def threaded_rate(run, batch, budget_s=8.0, min_rounds=20):
    """Positions/s of `run(begin, end)` over `batch` positions split across
    every host core (one thread each; the C oracle runs without the GIL),
    repeated for at least `min_rounds` rounds and `budget_s` seconds."""
    cores, model = host_cpu()
    bounds = np.linspace(0, batch, cores + 1).astype(int)
    chunks = [(int(a), int(b)) for a, b in zip(bounds[:-1], bounds[1:]) if b > a]
    run(0, min(4, batch))  # warm
    rounds = 0
    with ThreadPoolExecutor(len(chunks)) as ex:
        t0 = time.perf_counter()
        while True:
            list(ex.map(lambda ab: run(*ab), chunks))
            rounds += 1
            if rounds >= min_rounds and time.perf_counter() - t0 >= budget_s:
                break
        dt = time.perf_counter() - t0
    return rounds * batch / dt, rounds, dt, len(chunks), model


def sfnn_cpu_baseline(shape, budget_s=8.0):
    """The reference's CPU evaluation path for SFNN -- the engine's integer
    forward over the exported quantised network (examples/bulletou.rs:
    8001-8163; rayon over positions there) -- as the C oracle's restatement,
    on every host core."""
    from bulletou_b200 import synthetic
    from oracle import oracle

    cores, _ = host_cpu()
    batch = 64 * cores
    w = synthetic.sfnn_weights(synthetic.rng_for(7), stacks=shape.num_stacks)
    q = oracle.sfnn_quantize(shape.as_tuple(), w)
    b = synthetic.sfnn_batch(4242, batch, stacks=shape.num_stacks)
    A = SFNN_ACTIVE

    def run(lo, hi):
        oracle.sfnn_integer_forward(shape.as_tuple(), b["stm"][lo * A:hi * A], b["nstm"][lo * A:hi * A],
                                    b["buckets"][lo:hi], hi - lo, A, q)

    rate, rounds, dt, threads, model = threaded_rate(run, batch, budget_s)
    return {"value": round(rate, 1), "unit": "positions/s (integer forward evaluation only)", "cores": threads,
            "kind": "port", "cpu": model,
            "sample": f"oracle quantised SFNN 1536 ({shape.num_stacks} buckets) integer forward (the reference's CPU "
                      f"evaluator), {rounds} rounds x {batch} positions over {threads} threads in {dt:.1f} s; the "
                      f"reference cannot train on CPU"}


def halfkp_cpu_baseline(budget_s=6.0):
    """The reference's CPU HalfKP evaluation (fast_nnue.rs:209-271, f32) and
    the engine's integer forward of the written nn.bin, as the C oracle's
    restatements, on every host core."""
    from bulletou_b200 import synthetic
    from oracle import oracle

    cores, _ = host_cpu()
    batch = 128 * cores
    w = synthetic.halfkp_weights(synthetic.rng_for(7))
    b = synthetic.halfkp_batch(4242, batch)
    q = oracle.nnue_quantize(SHAPE, w)

    def f32(lo, hi):
        oracle.nnue_forward(SHAPE, b["stm"][lo * ACTIVE:hi * ACTIVE], b["nstm"][lo * ACTIVE:hi * ACTIVE], hi - lo,
                            ACTIVE, w)

    def i16(lo, hi):
        oracle.nnue_integer_forward(SHAPE, b["stm"][lo * ACTIVE:hi * ACTIVE], b["nstm"][lo * ACTIVE:hi * ACTIVE],
                                    hi - lo, ACTIVE, q)

    r32, n32, t32, threads, model = threaded_rate(f32, batch, budget_s)
    r16, n16, t16, _, _ = threaded_rate(i16, batch, budget_s / 2)
    return {"value": round(r32, 1), "unit": "positions/s (f32 forward evaluation)", "cores": threads, "kind": "port",
            "cpu": model, "integer_forward": round(r16, 1),
            "sample": f"oracle HalfKP 256x2-32-32 f32 forward, {n32} rounds x {batch} positions over {threads} "
                      f"threads in {t32:.1f} s (integer forward: {n16} rounds in {t16:.1f} s)"}


def teacher_cpu_baseline(n=16384, budget_s=6.0):
    """The reference's teacher-batch producer for this workload
    (prepare_sfnn_fast_batch_from_board_features, teacher_batch.rs:2869-3010)
    as the C oracle's restatement, on every host core."""
    from bulletou_b200 import synthetic
    from bulletou_b200 import teacher as bt
    from oracle import teacher as ot

    recs = synthetic.psv_records(4343, n)
    cfg = sfnn_teacher_config()
    lb = cfg.layerstack_bucket
    ocfg = ot.config("halfka_hm2", cfg.active, lb.hand, lb.king, cfg.lambda_, cfg.scale)
    table = bt.win_rate_model_score_table(cfg.wrm_target)

    def run(lo, hi):
        ot.prepare(recs[lo:hi], ocfg, table)

    rate, rounds, dt, threads, model = threaded_rate(run, n, budget_s, min_rounds=3)
    return {"value": round(rate, 1), "unit": "positions/s", "cores": threads, "kind": "port", "cpu": model,
            "sample": f"oracle PackedSfenValue -> HalfKA_hm2 batch producer, {rounds} x {n} records over {threads} "
                      f"threads in {dt:.1f} s"}


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


# --------------------------------------------------------------------------- HalfKP train
def make_batches(batch, rank=0):
    from bulletou_b200 import synthetic

    return [synthetic.halfkp_batch(1000 + i, batch, rank) for i in range(N_BATCHES)]


def make_runner(ctx, batch, fused):
    import bulletou_b200 as bo
    from bulletou_b200 import synthetic

    w = synthetic.halfkp_weights(synthetic.rng_for(7))
    return bo.NnueTrainStepRunner(ctx, bo.NnueForwardHostWeights(bo.NnueForwardShape(*SHAPE), **w), batch, ACTIVE,
                                  fused=fused)


def device_batches(ctx, batches):
    import bulletou_b200 as bo

    return [(bo.I32Buffer.from_host(ctx, b["stm"]), bo.I32Buffer.from_host(ctx, b["nstm"]),
             bo.F32Buffer.from_host(ctx, b["targets"]), bo.F32Buffer.from_host(ctx, b["entry_weights"]))
            for b in batches]


def bind_batch(runner, dev):
    runner.stm_indices, runner.nstm_indices, runner.targets, runner.entry_weights = dev


def run_halfkp(args, rank, world, local, dist, reference=False):
    import ctypes

    import bulletou_b200 as bo

    if world > 1 and not reference:
        from bulletou_b200.data_parallel import run_data_parallel_bench

        return run_data_parallel_bench(args, rank, world, local, dist)
    lib = bo.reference_library() if reference else None
    ctx = bo.Context(local, lib) if lib else bo.Context(local)
    runner = make_runner(ctx, args.batch, fused=not reference)
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
    start, stop = bo.Event(ctx), bo.Event(ctx)
    profiled = not reference
    if profiled:
        ctx.lib.call("bulletou_b200_profile_begin", ctx.as_ptr(), 8 * args.steps + 8)
    with ClockSampler(local) as clocks:
        start.record(ctx)
        for i in range(args.steps):
            step += 1
            bind_batch(runner, devb[i % N_BATCHES])
            runner.step_device(ctx, ranger(step), loss_kind, inv, finalize_loss=False)
        stop.record(ctx)
        stop.synchronize()
    phase_ms = {}
    if profiled:
        ms = (ctypes.c_float * 8)()
        nsteps, nphases = ctypes.c_size_t(), ctypes.c_size_t()
        ctx.lib.call("bulletou_b200_profile_end", ctx.as_ptr(), ms, 8, ctypes.byref(nsteps), ctypes.byref(nphases))
        phase_ms = {PHASES[p]: ms[p] / max(1, nsteps.value) for p in range(nphases.value)}
    total_ms = max_over_ranks(dist, stop.elapsed_ms_since(start))
    clk = clocks.summary()
    upload_ctx = bo.Context(local, lib) if lib else bo.Context(local)
    sources = [PinnedHostBatch((b["stm"], b["nstm"], b["targets"], b["entry_weights"])) for b in batches]
    e2e, step = pipelined_e2e(runner, ctx, upload_ctx, sources, args.steps, step, loss_kind, inv)
    return {"total_ms": total_ms, "phase_ms": phase_ms, "clocks": clk,
            "e2e": {"value": e2e["steps"] * args.batch * world / (e2e["ms"] / 1000.0), "unit": "positions/s",
                    "h2d_bytes_per_step": e2e["h2d_bytes_per_step"], "d2h_bytes_per_step": 4, "steps": e2e["steps"],
                    "path": "NnueTrainStepRunner.upload_next + step_uploaded_no_readback_with_loss_finalize (2 "
                            "upload slots; step i+1's batch uploaded on a second stream while step i runs) from "
                            "page-locked host batches via the ABI's *_upload entries; mean "
                            "loss read back synchronously every step (same calls on both arms)"},
            "gpu_launches": LAUNCHES_PER_STEP * args.steps, "final_loss": e2e["final_loss"]}


def roofline(phase_ms, batch, hbm_peak, peak_kind, l2_peak=None, lookahead_frac=1.0 / 6.0):
    """HalfKP step phases: compulsory DRAM bytes per step of each phase; the
    FT gather's repeated rows come from L2 and are counted separately."""
    rows, width = SHAPE[0], SHAPE[1]
    entries = 2 * batch * ACTIVE
    comp = {
        # every FT row's optimizer state (w, m, v read + written; slow on lookahead steps),
        # the pre-activation gradients read once, the inverse index
        "ft_row_grad_ranger": rows * width * 4 * (6 + 2 * lookahead_frac) + 2 * batch * width * 4
                              + 4 * (entries + rows + 1),
        # the table once + indices + both perspectives' activations written
        "ft_gather": rows * width * 4 + entries * 4 + 2 * batch * width * 4,
        "dense_fwd_loss_bwd": 2 * (2 * batch * width * 4) + batch * 4 * (32 * 4 + 4 * 4),
        "batch_reduce": 2 * (2 * batch * width * 4) + batch * 4 * (32 * 4 + 2),
        "inverse_index": 4 * (entries * 3 + rows * 4),
        "king_sort": 4 * (2 * batch * 4),
        "small_param_ranger": 0.0,
    }
    logical = {"ft_gather": entries * width * 4, "ft_row_grad_ranger": entries * width * 4}
    return phase_roofline(phase_ms, comp, logical, hbm_peak, peak_kind, l2_peak, {}, 1)


def phase_roofline(phase_ms, comp, logical, hbm_peak, peak_kind, l2_peak, traffic, launches, kernels=None):
    dom = max(phase_ms, key=phase_ms.get)
    phases = {}
    for k, ms in phase_ms.items():
        t = ms / 1000.0
        p = {"ms": round(ms, 4), "compulsory_bytes": int(comp.get(k, 0.0)),
             "hbm_frac": round(comp.get(k, 0.0) / t / 1e9 / hbm_peak, 4) if t > 0 else 0.0}
        if k in logical and t > 0:
            p["l2_logical_bytes"] = int(logical[k])
            if l2_peak:
                p["l2_frac"] = round(logical[k] / t / 1e9 / l2_peak, 4)
        phases[k] = p
    t = phase_ms[dom] / 1000.0
    achieved = comp.get(dom, 0.0) / t / 1e9 if t > 0 else 0.0
    out = {"bound": "hbm", "kernel": (kernels or {}).get(dom, dom), "phase": dom, "achieved": round(achieved, 1),
           "peak": hbm_peak, "unit": "GB/s", "frac": round(achieved / hbm_peak, 4), "peak_source": peak_kind,
           "traffic": traffic.get(dom), "launches_per_step": launches,
           "algorithmic_bytes": "compulsory DRAM bytes of the phase per step (each byte the phase must move once)",
           "algorithmic_bytes_per_step": int(comp.get(dom, 0.0)), "kernel_ms_per_step": round(phase_ms[dom], 4),
           "phases": phases}
    if dom in logical and t > 0:
        out["l2_logical_bytes_per_step"] = int(logical[dom])
        out["l2_achieved"] = round(logical[dom] / t / 1e9, 1)
        if l2_peak:
            out["l2_peak"] = l2_peak
            out["l2_frac"] = round(logical[dom] / t / 1e9 / l2_peak, 4)
    return out


# --------------------------------------------------------------------------- HalfKP forward
def run_halfkp_forward(args, local, reference=False):
    """the drop-in f32 forward entry (bulletou_cuda_cpp_nnue_forward_device)
    and, on this library, the engine's integer forward (int16 FT / int8 dense),
    16384 positions; L2 flushed (256 MB write) before each timed forward, which
    is timed alone with events on the library stream."""
    import bulletou_b200 as bo
    from bulletou_b200 import synthetic
    from bulletou_b200.cuda_cpp import NnueForwardShape, NnueForwardWorkspace, nnue_forward_device

    lib = bo.reference_library() if reference else None
    ctx = bo.Context(local, lib) if lib else bo.Context(local)
    shape = NnueForwardShape(*SHAPE)
    w = synthetic.halfkp_weights(synthetic.rng_for(7))
    names = ("l0w", "l0b", "l1w", "l1b", "l2w", "l2b", "outw", "outb")
    dw = [bo.F32Buffer.from_host(ctx, w[n]) for n in names]
    batches = make_batches(args.batch)
    devb = [(bo.I32Buffer.from_host(ctx, b["stm"]), bo.I32Buffer.from_host(ctx, b["nstm"])) for b in batches]
    ws = NnueForwardWorkspace(ctx, shape, args.batch)
    flush = bo.F32Buffer(ctx, 64 << 20)  # 256 MB > L2

    def forward(i):
        s, n = devb[i % len(devb)]
        nnue_forward_device(ctx, shape, args.batch, ACTIVE, s, n, dw, ws)

    def timed(fn, steps):
        total = 0.0
        for i in range(steps):
            flush_l2(ctx, flush)
            e0, e1 = bo.Event(ctx), bo.Event(ctx)
            e0.record(ctx)
            fn(i)
            e1.record(ctx)
            e1.synchronize()
            total += e1.elapsed_ms_since(e0)
        return total

    for i in range(args.warmup):
        forward(i)
    ctx.synchronize()
    with ClockSampler(local) as clocks:
        total_ms = timed(forward, args.steps)
    out = {"total_ms": total_ms, "clocks": clocks.summary()}
    if not reference:
        from bulletou_b200.nnue_quant import (NnueIntegerForwardWorkspace, QuantizedNnueDeviceWeights,
                                              nnue_integer_forward_device, nnue_quantize_device)

        q = QuantizedNnueDeviceWeights(ctx, *SHAPE)
        nnue_quantize_device(ctx, dict(zip(names, dw)), q)
        iws = NnueIntegerForwardWorkspace(ctx, args.batch)

        def int_forward(i):
            s, n = devb[i % len(devb)]
            nnue_integer_forward_device(ctx, q, args.batch, ACTIVE, s, n, iws)

        for i in range(args.warmup):
            int_forward(i)
        ctx.synchronize()
        int_ms = timed(int_forward, args.steps)
        out["integer_forward"] = {"value": round(args.steps * args.batch / (int_ms / 1000.0), 1),
                                  "unit": "positions/s", "ms_per_batch": round(int_ms / args.steps, 4),
                                  "dtype": "i16 FT / i8 dense / i32 (the engine's integer network)",
                                  "algorithmic_bytes_per_position": 39220}
    # end to end: the batch's indices H2D from page-locked memory, the forward,
    # the outputs D2H -- synchronous per batch, same calls on both arms
    src = [PinnedHostBatch((b["stm"], b["nstm"])) for b in batches]
    s_dev, n_dev = bo.I32Buffer(ctx, args.batch * ACTIVE), bo.I32Buffer(ctx, args.batch * ACTIVE)
    from bulletou_b200.cuda_cpp import upload_from_pinned

    def e2e_step(i):
        p = src[i % len(src)]
        upload_from_pinned(ctx, s_dev, p.pinned[0])
        upload_from_pinned(ctx, n_dev, p.pinned[1])
        nnue_forward_device(ctx, shape, args.batch, ACTIVE, s_dev, n_dev, dw, ws)
        return ws.output.download(ctx)

    for i in range(3):
        e2e_step(i)
    t0 = time.perf_counter()
    for i in range(args.steps):
        res = e2e_step(i)
    wall = (time.perf_counter() - t0) * 1000.0
    assert np.all(np.isfinite(res))
    out["e2e"] = {"value": args.steps * args.batch / (wall / 1000.0), "unit": "positions/s",
                  "h2d_bytes_per_step": int(src[0].nbytes), "d2h_bytes_per_step": 4 * args.batch,
                  "steps": args.steps,
                  "path": "page-locked stm/nstm indices -> *_upload -> bulletou_cuda_cpp_nnue_forward_device -> "
                          "f32_download of the outputs, synchronous per batch"}
    return out


def halfkp_forward_roofline(ms_per_batch, batch, hbm_peak, peak_kind, l2_peak):
    """FT gather of the f32 forward: logical 2*A*W*4 + 2*A*4 + 4 = 78,132 B per
    position (the hot-path table's figure), L2-served after the king sort;
    compulsory DRAM: the 128 MB table once (L2 flushed before each forward),
    the indices and the activations written."""
    rows, width = SHAPE[0], SHAPE[1]
    logical = batch * (2 * ACTIVE * width * 4 + 2 * ACTIVE * 4 + 4)
    comp = rows * width * 4 + 2 * batch * ACTIVE * 4 + batch * 4 * (4 * width + 32 + 32 + 1)
    t = ms_per_batch / 1000.0
    return {"bound": "hbm", "kernel": "forward call (king sort 3 + ft_gather_kernel + halfkp_dense_kernel)",
            "achieved": round(comp / t / 1e9, 1), "peak": hbm_peak, "unit": "GB/s",
            "frac": round(comp / t / 1e9 / hbm_peak, 4), "peak_source": peak_kind, "traffic": None,
            "algorithmic_bytes": "compulsory DRAM bytes per forward (table once, indices, activations)",
            "algorithmic_bytes_per_step": int(comp), "kernel_ms_per_step": round(ms_per_batch, 4),
            "l2_logical_bytes_per_step": int(logical), "l2_logical_bytes_per_position": 78132,
            "l2_achieved": round(logical / t / 1e9, 1), "l2_peak": l2_peak,
            "l2_frac": round(logical / t / 1e9 / l2_peak, 4) if l2_peak else None}


# --------------------------------------------------------------------------- KPPT workload
KPPT_BATCH = 32768
KPPT_METRIC = "train positions/sec (KPPT KPP component table, 81 x 1548^2 entries, 703 pairs, batch 32768)"


def run_kppt(args, local, reference=False):
    """One KPP component-table train step per iteration (the reference trains
    one component table per runner, lib.rs:4857-5066): device-resident
    batches; the e2e leg uploads every step's pair indices, targets and
    weights from page-locked host memory through the ABI's *_upload entries
    (same calls on both arms) and reads the mean loss back every step."""
    import bulletou_b200 as bo
    from bulletou_b200 import synthetic
    from bulletou_b200.cuda_cpp import upload_from_pinned

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
    pinned = [PinnedHostBatch(b) for b in batches]
    # two device input sets: step i's batch in set i % 2, step i + 1's uploaded
    # on a second stream while step i runs
    sets = [(runner.stm_indices, runner.nstm_indices, runner.targets, runner.entry_weights)]
    sets.append(tuple(type(b)(ctx, b.length) for b in sets[0]))
    upload_ctx = bo.Context(local, lib) if lib else bo.Context(local)
    ready = [bo.Event(ctx), bo.Event(ctx)]
    done = [bo.Event(ctx), bo.Event(ctx)]
    used = [False, False]

    def upload(k, i):
        if used[k]:
            done[k].wait(upload_ctx)  # the step that read set k has finished
        for d, p in zip(sets[k], pinned[i % 2].pinned):
            upload_from_pinned(upload_ctx, d, p)
        ready[k].record(upload_ctx)
        used[k] = True

    def step_on(k, s):
        ready[k].wait(ctx)
        runner.stm_indices, runner.nstm_indices, runner.targets, runner.entry_weights = sets[k]
        runner.step_device(ctx, ranger(s), loss_kind, inv, finalize_loss=True)
        done[k].record(ctx)

    ctx.synchronize()
    e0, e1 = bo.Event(ctx), bo.Event(ctx)
    t0 = time.perf_counter()
    e0.record(ctx)
    upload(0, 0)
    for i in range(args.steps):
        step += 1
        step_on(i % 2, step)
        if i + 1 < args.steps:
            upload((i + 1) % 2, i + 1)
        runner.loss_workspace.mean.download(ctx)
    e1.record(ctx)
    e1.synchronize()
    e2e_ms = max(e1.elapsed_ms_since(e0), (time.perf_counter() - t0) * 1000.0)
    upload_ctx.synchronize()
    return {"total_ms": total_ms, "clocks": clocks.summary(),
            "e2e": {"value": args.steps * args.batch / (e2e_ms / 1000.0), "unit": "positions/s",
                    "h2d_bytes_per_step": int(pinned[0].nbytes), "d2h_bytes_per_step": 4, "steps": args.steps,
                    "path": "page-locked pair indices / targets / weights -> *_upload on a second stream (step "
                            "i+1's batch while step i runs, two device input sets) -> train step -> mean loss "
                            "download, every step (same calls on both arms)"}}


def kppt_roofline(ms_per_step, batch, hbm_peak, peak_kind, lookahead_frac=1.0 / 6.0):
    """KPP step: the dense Ranger over the 194.1M-entry table (gradient read and
    cleared, w / m / v read and written, slow on lookahead steps) dominates;
    the forward gather and backward scatter touch 2 * 703 entries a position."""
    from bulletou_b200 import synthetic

    n = synthetic.KPP_INPUTS
    ranger_bytes = n * 4 * (8 + 2 * lookahead_frac)
    sparse = 2 * batch * synthetic.KPP_PAIRS * 4 * 3  # gather + scatter read-modify-write
    comp = ranger_bytes + sparse
    t = ms_per_step / 1000.0
    return {"bound": "hbm", "kernel": ("KPPT step (king sort + kppt_view_kernel + kppt_kernel<3> + "
                                       "kppt_scatter_kernel + kppt_small_kernel + ranger_vec4_kernel)"),
            "achieved": round(comp / t / 1e9, 1), "peak": hbm_peak, "unit": "GB/s",
            "frac": round(comp / t / 1e9 / hbm_peak, 4), "peak_source": peak_kind, "traffic": None,
            "algorithmic_bytes": "dense Ranger over the table + the sparse gather / scatter, per step",
            "algorithmic_bytes_per_step": int(comp), "ranger_bytes_per_step": int(ranger_bytes),
            "kernel_ms_per_step": round(ms_per_step, 4)}


# --------------------------------------------------------------------------- SFNN workloads (configs[2], [4])
def sfnn_shape():
    return SFNN_K3K3.shape()


def make_sfnn_batches(batch, rank=0, stacks=9, zipf=0.0):
    from bulletou_b200 import synthetic

    return [synthetic.sfnn_batch(2000 + i, batch, rank, stacks=stacks, zipf=zipf) for i in range(SFNN_N_BATCHES)]


def sfnn_host_weights(stacks=9):
    from bulletou_b200 import sfnn as bs
    from bulletou_b200 import synthetic

    shape = SFNN_K3K3.shape() if stacks == 9 else SFNN_K9K9.shape()
    return bs.SfnnForwardHostWeights(shape, **synthetic.sfnn_weights(synthetic.rng_for(7), stacks=stacks))


def zipf_buckets(i, batch, rank, stacks, zipf):
    from bulletou_b200 import synthetic

    return synthetic.layerstack_buckets(synthetic.rng_for(4400 + i, rank), batch, stacks, zipf)


def sfnn_batches(args, ctx, rank=0, reference=False, workload=None):
    """(host batches, device batches) of an SFNN workload.  --data psv (the
    default): seeded PackedSfenValue records of full-set positions, decoded to
    HalfKA_hm2 rows, k3k3 buckets and win-rate targets -- on the device by the
    product's producer, by the CPU oracle of the reference's producer on the
    reference arm (the two agree bit for bit); configs[4] replaces the buckets
    by Zipf(1.1) draws over its 81 (the same on both arms).  --data uniform:
    rows drawn uniformly over the king blocks (synthetic.sfnn_batch)."""
    wl = workload or SFNN_K3K3
    if args.data == "uniform":
        batches = make_sfnn_batches(args.batch, rank, wl.stacks, wl.zipf)
        return batches, sfnn_device_batches(ctx, batches)
    from bulletou_b200 import synthetic
    from bulletou_b200 import teacher as bt

    records = [synthetic.psv_records(3000 + i, args.batch, rank) for i in range(SFNN_RECORD_BATCHES)]
    cfg = sfnn_teacher_config()
    if reference:
        from oracle import teacher as ot

        lb = cfg.layerstack_bucket
        ocfg = ot.config("halfka_hm2", cfg.active, lb.hand, lb.king, cfg.lambda_, cfg.scale)
        table = bt.win_rate_model_score_table(cfg.wrm_target)
        host = []
        for i, r in enumerate(records):
            o = oracle_prepare_parallel(r, ocfg, table)
            assert (o["counts"] <= cfg.active).all()
            buckets = zipf_buckets(i, args.batch, rank, wl.stacks, wl.zipf) if wl.zipf else o["buckets"]
            host.append({"stm": o["stm"].reshape(-1), "nstm": o["nstm"].reshape(-1), "buckets": buckets,
                         "targets": o["targets"], "entry_weights": o["entry_weights"]})
        return host, sfnn_device_batches(ctx, host)
    producer = bt.TeacherBatchProducer(ctx, cfg, args.batch, pinned=False)
    host, dev = [], []
    for i, r in enumerate(records):
        tb = producer.new_batch()
        producer.prepare(ctx, r, tb)
        if wl.zipf:
            tb.buckets.upload(zipf_buckets(i, args.batch, rank, wl.stacks, wl.zipf), ctx)
        dev.append((tb.stm_indices, tb.nstm_indices, tb.buckets, tb.targets, tb.entry_weights))
        d = tb.download(ctx)
        host.append({"stm": d["stm"].reshape(-1), "nstm": d["nstm"].reshape(-1), "buckets": d["buckets"],
                     "targets": d["targets"], "entry_weights": d["entry_weights"]})
    producer.check(ctx)
    return host, dev


def oracle_prepare_parallel(records, ocfg, table):
    """The oracle producer over every host core (records split into chunks;
    per-record results do not depend on the split)."""
    from oracle import teacher as ot

    cores, _ = host_cpu()
    recs = np.asarray(records)
    parts = np.array_split(np.arange(len(recs)), max(1, min(cores, len(recs) // 1024 or 1)))
    with ThreadPoolExecutor(len(parts)) as ex:
        outs = list(ex.map(lambda ix: ot.prepare(recs[ix[0]:ix[-1] + 1], ocfg, table), parts))
    return {k: np.concatenate([o[k] for o in outs]) for k in outs[0]}


def sfnn_device_batches(ctx, batches):
    import bulletou_b200 as bo

    return [(bo.I32Buffer.from_host(ctx, b["stm"]), bo.I32Buffer.from_host(ctx, b["nstm"]),
             bo.I32Buffer.from_host(ctx, b["buckets"]), bo.F32Buffer.from_host(ctx, b["targets"]),
             bo.F32Buffer.from_host(ctx, b["entry_weights"])) for b in batches]


def bind_sfnn(runner, dev):
    runner.stm_indices, runner.nstm_indices, runner.buckets, runner.targets, runner.entry_weights = dev


def sfnn_sources(host):
    return [PinnedHostBatch((b["stm"], b["nstm"], b["buckets"], b["targets"], b["entry_weights"])) for b in host]


def sfnn_teacher_config():
    """The reference's SFNN trainer defaults (examples/bulletou.rs:5050-5075,
    18846-18866): lambda 1.0, win-rate-model targets (offset 270, scaling 380),
    k3k3 = KingRank9 LayerStack buckets, no score drop."""
    from bulletou_b200 import teacher as bt

    return bt.TeacherBatchConfig(feature_set="halfka_hm2", lambda_=1.0, scale=600.0, win_rate_model=True)


def sfnn_records_e2e(args, ctx, upload_ctx, runner, step, loss_kind, inv):
    """This library only: end to end from teacher records -- per step the
    batch's PackedSfenValue records (40 bytes a position) go H2D from pinned
    memory and are decoded on the device on the upload stream while the
    previous step trains; the mean loss comes back every step.  Also times the
    decode kernel alone on records resident in HBM."""
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
    steps = args.steps
    ring = [PinnedF32Buffer(ctx, 1) for _ in range(max(steps, 3))]
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
    for i in range(steps):
        step += 1
        h2d = runner.step_pipelined_records(ctx, upload_ctx, producer, ranger(step), loss_kind, inv, None, True,
                                            sources[i % len(sources)], ring[i])
    e1.record(ctx)
    e1.synchronize()
    e2e_ms = max(e1.elapsed_ms_since(e0), (time.perf_counter() - t0) * 1000.0)
    producer.check(ctx)
    losses = [float(r.host()[0]) for r in ring]
    assert all(np.isfinite(losses)), "non-finite loss"
    e2e = {"value": steps * args.batch / (e2e_ms / 1000.0), "unit": "positions/s",
           "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": 4, "steps": steps,
           "path": "SfnnTrainStepRunner.step_pipelined_records: PackedSfenValue records in pinned host memory -> "
                   "H2D (40 B/position) -> device decode (bulletou_b200_teacher_prepare_device) on the upload "
                   "stream -> fused train step; mean loss copied D2H asynchronously every step"}
    producer_line = {"kernel": "teacher_psv_kernel", "ms_per_batch": round(decode_ms, 4),
                     "positions_per_s": round(args.batch / (decode_ms / 1000.0), 1),
                     "record_bytes_per_s": round(40 * args.batch / (decode_ms / 1000.0), 1)}
    return e2e, producer_line, step


def sfnn_phases(qat):
    """Stage-profiler phases of one fused step (every QAT mode)."""
    return SFNN_PHASES


def _profile(lib, ctx, names):
    import ctypes

    ms = (ctypes.c_float * 16)()
    nsteps, nphases = ctypes.c_size_t(), ctypes.c_size_t()
    lib.call("bulletou_b200_profile_end", ctx.as_ptr(), ms, 16, ctypes.byref(nsteps), ctypes.byref(nphases))
    return {names[p]: ms[p] / max(1, nsteps.value) for p in range(min(nphases.value, len(names)))}


def run_sfnn_b200(args, wl, rank, world, local, dist):
    import bulletou_b200 as bo
    from bulletou_b200 import sfnn as bs
    from bulletou_b200.cuda_cpp import PinnedF32Buffer

    if world > 1:
        return run_sfnn_data_parallel(args, wl, rank, world, local, dist)
    ctx = bo.Context(local)
    runner = bs.SfnnTrainStepRunner(ctx, sfnn_host_weights(wl.stacks), args.batch, SFNN_ACTIVE, fused=True,
                                    lr_multipliers=sfnn_lr_multipliers(args.qat))
    host, devb = sfnn_batches(args, ctx, rank, workload=wl)
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
    lib.call("bulletou_b200_profile_begin", ctx.as_ptr(), 11 * args.steps + 11)
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
    upload_ctx = bo.Context(local)
    e2e, step = pipelined_e2e(runner, ctx, upload_ctx, sfnn_sources(host), args.steps, step, loss_kind, inv)
    # the same pipelined step with the loss read back asynchronously into a pinned ring
    sources = sfnn_sources(host)
    ring = [PinnedF32Buffer(ctx, 1) for _ in range(args.steps)]
    e0, e1 = bo.Event(ctx), bo.Event(ctx)
    t0 = time.perf_counter()
    e0.record(ctx)
    for i in range(args.steps):
        step += 1
        runner.step_pipelined_no_readback_with_loss_finalize(ctx, upload_ctx, ranger(step), loss_kind, inv, None,
                                                             True, sources[i % len(sources)], ring[i])
    e1.record(ctx)
    e1.synchronize()
    async_ms = max(e1.elapsed_ms_since(e0), (time.perf_counter() - t0) * 1000.0)
    out = {"total_ms": total_ms, "phase_ms": phase_ms, "clocks": clk,
           "e2e": {"value": e2e["steps"] * args.batch / (e2e["ms"] / 1000.0), "unit": "positions/s",
                   "h2d_bytes_per_step": e2e["h2d_bytes_per_step"], "d2h_bytes_per_step": 4, "steps": e2e["steps"],
                   "path": "SfnnTrainStepRunner.upload_next + step_uploaded_no_readback_with_loss_finalize (2 "
                           "upload slots; step i+1's batch uploaded on a second stream while step i runs) from "
                           "page-locked host batches via the ABI's *_upload entries; mean loss read back "
                           "synchronously every step (same calls on both arms)"},
           "e2e_async_loss": {"value": args.steps * args.batch / (async_ms / 1000.0), "unit": "positions/s",
                              "path": "as e2e, the mean loss copied D2H asynchronously into a pinned ring"},
           "gpu_launches": sfnn_launches_per_step(args.qat) * args.steps, "final_loss": e2e["final_loss"]}
    if args.data == "psv" and not wl.zipf:
        rec, producer_line, step = sfnn_records_e2e(args, ctx, upload_ctx, runner, step, loss_kind, inv)
        out["e2e_records"] = rec
        out["producer"] = producer_line
    out["l2_peak"] = measure_l2_peak(ctx)
    return out


def run_sfnn_data_parallel(args, wl, rank, world, local, dist):
    """N > 1: args.batch positions per rank (NCCL exchange)."""
    import torch

    import bulletou_b200 as bo
    from bulletou_b200.data_parallel import B200Backend, SfnnDataParallelTrainer

    backend = B200Backend(local)
    ctx, lib = backend.ctx, backend.lib
    tr = SfnnDataParallelTrainer(backend, dist, sfnn_host_weights(wl.stacks), args.batch, SFNN_ACTIVE,
                                 lr_multipliers=sfnn_lr_multipliers(args.qat),
                                 launches_per_chunk=args.dp_chunk_launches,
                                 last_chunk_launches=args.dp_last_chunk_launches or None,
                                 exchange=args.dp_exchange)
    host, devb = sfnn_batches(args, ctx, rank, workload=wl)
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
    lib.call("bulletou_b200_profile_begin", ctx.as_ptr(), 11 * args.steps + 11)
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
    # end to end: per step the batch H2D from page-locked host memory through
    # the ABI's *_upload entries, the step, a synchronous read of the mean loss
    from bulletou_b200.cuda_cpp import F32Buffer, I32Buffer, upload_from_pinned

    sources = sfnn_sources(host)
    n = args.batch * SFNN_ACTIVE
    in_bufs = (I32Buffer(ctx, n), I32Buffer(ctx, n), I32Buffer(ctx, args.batch), F32Buffer(ctx, args.batch),
               F32Buffer(ctx, args.batch))
    tr.stm_indices, tr.nstm_indices, tr.buckets, tr.targets, tr.entry_weights = in_bufs
    dist.barrier()
    e0, e1 = bo.Event(ctx), bo.Event(ctx)
    losses = []
    t0 = time.perf_counter()
    e0.record(ctx)
    for i in range(args.steps):
        step += 1
        for dst, src in zip(in_bufs, sources[i % len(sources)].pinned):
            upload_from_pinned(ctx, dst, src)
        tr.step_device(ranger(step), loss_kind, inv, finalize_loss=True)
        losses.append(float(tr.loss_workspace.mean.download(ctx)[0]))
    tr.join()
    e1.record(ctx)
    e1.synchronize()
    wall_ms = (time.perf_counter() - t0) * 1000.0
    e2e_ms = max_over_ranks(dist, max(e1.elapsed_ms_since(e0), wall_ms))
    assert all(np.isfinite(losses)), "non-finite loss"
    # after the timed regions: a few steps with events around each collective
    # on the comm stream (the exchange breakdown; not part of any timed number)
    tr.timing = True
    for i in range(min(args.steps, 8)):
        step += 1
        bind(i)
        tr.step_device(ranger(step), loss_kind, inv, finalize_loss=False)
    tr.timing = False
    tr.check()  # raises if a peer-exchange wait timed out in any step above
    exchange = backend.exchange_timing(tr)
    exchange["mode"] = tr.exchange
    exchange["exchange_tail_after_rows_ms_max_over_ranks"] = max_over_ranks(
        dist, exchange.get("exchange_tail_after_rows_ms", 0.0))
    torch.cuda.synchronize()
    tr.close()
    dist.barrier()
    how = ("FT rows stored into their owners' slots by the row kernels, shards updated and stored into every "
           "rank's table over NVLink, the small groups' gradient summed from every rank's slot" if tr.exchange == "p2p" else
           "NCCL reduce-scatter / all-reduce / all-gather")
    return {"total_ms": total_ms, "phase_ms": phase_ms, "clocks": clocks.summary(),
            "e2e": {"value": args.steps * args.batch * world / (e2e_ms / 1000.0), "unit": "positions/s",
                    "h2d_bytes_per_step": int(sources[0].nbytes), "d2h_bytes_per_step": 4, "steps": args.steps,
                    "path": f"SfnnDataParallelTrainer.step_device per rank ({how}), inputs from page-locked host "
                            "memory, mean loss read back every step"},
            # the fused step's kernels; exchange: p2p adds per chunk a signal after its last row launch and the
            # owner's wait / shard Ranger / signal, plus the step's wait before the fold; collectives adds
            # the shard Ranger per chunk (NCCL's own kernels are not counted)
            "gpu_launches": (sfnn_launches_per_step(args.qat) +
                             (4 * len(tr.chunks) + 1 if tr.exchange == "p2p" else len(tr.chunks))) * args.steps,
            "final_loss": losses[-1],
            "exchange": exchange}


def run_sfnn_reference(args, wl, local):
    import bulletou_b200 as bo
    from bulletou_b200 import sfnn as bs

    lib = bo.reference_library()
    ctx = bo.Context(local, lib)
    runner = bs.SfnnTrainStepRunner(ctx, sfnn_host_weights(wl.stacks), args.batch, SFNN_ACTIVE, fused=False,
                                    lr_multipliers=sfnn_lr_multipliers(args.qat))
    host, devb = sfnn_batches(args, ctx, 0, reference=True, workload=wl)
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
    e2e, step = pipelined_e2e(runner, ctx, upload_ctx, sfnn_sources(host), args.steps, step, loss_kind, inv)
    return {"total_ms": total_ms, "clocks": clk,
            "e2e": {"value": e2e["steps"] * args.batch / (e2e["ms"] / 1000.0), "unit": "positions/s",
                    "h2d_bytes_per_step": e2e["h2d_bytes_per_step"], "d2h_bytes_per_step": 4, "steps": e2e["steps"],
                    "path": "the reference runner's pipelined step from page-locked host batches via the ABI's "
                            "*_upload entries; mean loss read back synchronously every step (same calls as the "
                            "product arm)"}}


# DRAM bytes per step of each phase at B = 65536 (dram__bytes_read.sum +
# dram__bytes_write.sum over the phase's launches, ncu), keyed by the QAT modes
# whose kernels they were measured on; profiles/ holds the captures.
SFNN_DRAM_BYTES_B65536 = {
    "ft_forward": (1679058432, ("none", "l1", "dense")),
    "l1_backward": (2076098304, ("dense", "all")),
}
SFNN_DRAM_BYTES_PSV_B65536 = {
    "ft_rows_ranger": (5416400000, ("all",)),
    "ft_forward": (1556600000, ("all",)),
    "l1_backward": (2860700000, ("all",)),
    "fold": (892700000, ("all",)),
}
SFNN_PHASE_KERNELS = {
    "ft_rows_ranger": ("heavy-key plan (3 kernels) + heavy_incidence_kernel + heavy_key_mma_kernel (tcgen05) + 15 "
                       "piece_row_kernel launches (FT gradient rows + fused Ranger)"),
    "ft_forward": "ft_forward_kernel<12> (ft_forward_int_kernel<12, 2> with all-layer QAT)",
    "l1_backward": "l1_backward_kernel<16>",
    "fold": "fold_rows_kernel<true> (FT QAT fold)",
}


def sfnn_roofline(phase_ms, batch, hbm_peak, peak_kind, l2_peak=None, lookahead_frac=1.0 / 6.0, qat="none",
                  data="psv", shape=None):
    """Compulsory DRAM bytes per step of each SFNN phase (what the phase must
    move at least once) against the measured HBM peak; the FT row gathers
    (2 * B * A rows of W floats, repeated rows served by L2) are reported as
    L2 logical bytes against the L2 peak measured in the same run."""
    sh = shape or sfnn_shape()
    W, A = sh.ft_size, SFNN_ACTIVE
    rows = sh.input_size
    base = sh.factorized_base()
    H = 2 * batch
    l1, ft, l2, l3 = SFNN_QAT_MODES[qat]
    dense = l1 and l2 and l3
    keys = (45 + H // 4096 + 1) * 1629
    comp = {
        # the table (+ virtual rows) read, the folded table written
        "fold": rows * W * 4 + base * W * 4,
        "sorts_tiles": 4 * (H * A + 4 * H + 3 * batch),
        "inverse_index": 4 * (H * A * 3 + keys * 4),
        # the folded table once + indices + the FT outputs written (both views' ClippedReLU, combined)
        "ft_forward": base * W * 4 + H * A * 4 + 3 * batch * W * 4,
        "l1_head": batch * W * 4 + batch * 4 * (16 + 30 + 32 + 16 + 4),
        # both views' FT outputs (+ the lattice input) read, king-ordered pre-activation gradients written
        "l1_backward": 2 * batch * W * 4 + (batch * W * 4 if dense else 0) + H * W * 4
                       + (batch // 128 + sh.num_stacks + 2) * 16 * W * 4,
        "small_grads_ranger": 0.0,
        # every FT row's optimizer state (w, m, v read + written; slow on lookahead
        # steps) + the pre-activation gradients read once + the row index
        "ft_rows_ranger": rows * W * 4 * (6 + 2 * lookahead_frac) + H * W * 4 + 4 * (H * A + keys + 1),
    }
    logical = {"ft_forward": H * A * W * 4, "ft_rows_ranger": H * A * W * 4}
    traffic = {}
    table = SFNN_DRAM_BYTES_B65536 if data == "uniform" else SFNN_DRAM_BYTES_PSV_B65536
    if batch == SFNN_BATCH and sh.num_stacks == 9:
        for k, (b, modes) in table.items():
            if qat in modes:
                traffic[k] = b
    out = phase_roofline(phase_ms, comp, logical, hbm_peak, peak_kind, l2_peak, traffic, None, SFNN_PHASE_KERNELS)
    out["launches_per_step"] = 20 if out["phase"] == "ft_rows_ranger" else 1
    out["traffic_note"] = ("DRAM bytes of the phase per step from an ncu capture at B = 65536 (profiles/); "
                           "null where none was taken for this configuration")
    return out


# --------------------------------------------------------------------------- main
def main():
    args = parse_args()
    if args.impl == "reference":
        # the reference backend is single-GPU: under torchrun rank 0 alone runs it
        rank, world, local, dist = int(os.environ.get("RANK", "0")), 1, int(os.environ.get("LOCAL_RANK", "0")), None
        if rank != 0:
            return
    else:
        rank, world, local, dist = dist_setup(args)
    if args.warmup < 3:
        args.warmup = 3
    hbm, kind = measured_peaks()
    common = {"seq_len": 1, "optimizer": "Ranger (RAdam + Lookahead k=6, lr 1e-3)",
              "loss": "sigmoid-pow(2) MSE of the output, scale 600"}

    def emit(line):
        if rank == 0:
            print(json.dumps(line))

    def finish():
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()

    ref = args.impl == "reference"
    reference_run = {"kind": "reference", "where": "GPU (the reference's implementation of this path is its CUDA "
                     "backend; it has no CPU training path)",
                     "library": "oracle/_ref/libref_cudacpp.so built from the reference sources by "
                                "oracle/build_ref.sh, driven through its C ABI in the reference runner's call order"}
    try:
        if args.workload in ("kppt", "halfkp_fwd"):
            args.batch = args.batch or (KPPT_BATCH if args.workload == "kppt" else BATCH)
            if rank == 0:
                if args.workload == "kppt":
                    r = run_kppt(args, local, reference=ref)
                    ms = r["total_ms"] / args.steps
                    line = {"metric": KPPT_METRIC, "unit": "positions/s", "n_gpus": 1, "steps": args.steps,
                            "warmup": args.warmup, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                            "dtype": "f32", "data": "synthetic (seeded KPP pairs, reference shapes)",
                            "config": {"workload": "configs[3] KPPT KPP component train step (Ranger, as the "
                                                   "reference's KPPT runner; the reference has no AdaGrad)",
                                       "global_batch": args.batch, "pairs": 703, "table": 194100624,
                                       "l2": "no flush: each step streams 6.5 GB of table state (> 126 MB L2)"},
                            "value": round(args.steps * args.batch / (r["total_ms"] / 1000.0), 1),
                            "ms_per_step": round(ms, 4), "clocks": r["clocks"], "e2e": rounded(r["e2e"])}
                    if not ref:
                        line["roofline"] = kppt_roofline(ms, args.batch, hbm, kind)
                        # king sort 3, view sums, outputs / loss, gradient scatter, small groups, table Ranger
                        line["gpu_launches"] = 8 * args.steps
                else:
                    r = run_halfkp_forward(args, local, reference=ref)
                    ms = r["total_ms"] / args.steps
                    line = {"metric": FWD_METRIC, "unit": "positions/s", "n_gpus": 1, "steps": args.steps,
                            "warmup": args.warmup, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                            "dtype": "f32", "data": "synthetic (seeded HalfKP rows, reference shapes)",
                            "config": {"workload": "configs[0] HalfKP 256x2-32-32-1 forward (the drop-in f32 "
                                                   "forward entry; integer forward alongside)",
                                       "model": "HalfKP 125388x256x2-32-32-1", "global_batch": args.batch,
                                       "max_active": ACTIVE,
                                       "l2": "flushed (256 MB write) before every timed forward"},
                            "value": round(args.steps * args.batch / (r["total_ms"] / 1000.0), 1),
                            "ms_per_step": round(ms, 4), "clocks": r["clocks"], "e2e": rounded(r["e2e"])}
                    if not ref:
                        ctx_l2 = None
                        import bulletou_b200 as bo

                        c = bo.Context(local)
                        ctx_l2 = measure_l2_peak(c)
                        line["l2_peak"] = ctx_l2
                        line["roofline"] = halfkp_forward_roofline(ms, args.batch, hbm, kind, ctx_l2["value"])
                        line["integer_forward"] = r["integer_forward"]
                        line["gpu_launches"] = 2 * FWD_LAUNCHES * args.steps
                        if not args.no_cpu_baseline:
                            line["cpu_baseline"] = halfkp_cpu_baseline()
                    else:
                        line["integer_forward"] = "unavailable: the reference has no integer HalfKP evaluator (it " \
                                                  "writes nn.bin for the engine)"
                if ref:
                    line.update(impl="reference", reference_run=reference_run)
                emit(line)
            return
        if args.workload == "halfkp":
            args.batch = args.batch or BATCH
            r = run_halfkp(args, rank, world, local, dist, reference=ref)
            metric = METRIC
            config = dict({"workload": "configs[1] HalfKP 256x2-32-32-1 train step",
                           "model": "HalfKP 125388x256x2-32-32-1", "max_active": ACTIVE,
                           "global_batch": args.batch * (1 if ref else world), "per_gpu_batch": args.batch,
                           "parallelism": f"dp{world}" if world > 1 and not ref else "single",
                           "l2": "no flush: each step streams 0.5 GB of optimizer state (> 126 MB L2)"}, **common)
            scaling = "weak"
            n = 1 if ref else world
            rl = None if ref else roofline(r["phase_ms"], args.batch, hbm, kind)
        else:
            wl = SFNN_WORKLOADS[args.workload]
            n = 1 if ref else world
            args.batch, global_batch = wl.batches(args.batch, n)
            if ref:
                r = run_sfnn_reference(args, wl, local)
            else:
                r = run_sfnn_b200(args, wl, rank, world, local, dist)
            metric = wl.metric
            scaling = "strong" if wl.strong else "weak"
            config = dict({"workload": wl.label,
                           "model": f"SFNN_halfkahm2_1536_15_32_k{'9k9' if wl.stacks == 81 else '3k3'}: "
                                    f"(73305+1629 virtual) x 1536 FT, pairwise, {wl.stacks} x (1536 -> 15+1), "
                                    f"shared L1 factor, 30 -> 32 -> 1",
                           "max_active": SFNN_ACTIVE, "global_batch": global_batch, "per_gpu_batch": args.batch,
                           "buckets": (f"Zipf({wl.zipf}) over {wl.stacks} (seeded rank permutation)" if wl.zipf
                                       else "k3k3 LayerStack buckets of the decoded records"),
                           "targets": ("win-rate-model probability of the teacher score (offset 270, scaling 380), "
                                       "lambda 1" if args.data == "psv" else "0.5 result + 0.5 sigmoid(score / 600)"),
                           "data": ("seeded PackedSfenValue records (full-set positions, kings near their home "
                                    "ranks) decoded to HalfKA_hm2 rows" if args.data == "psv" else
                                    "feature rows uniform over the 45 king blocks"),
                           "qat": f"{args.qat}: {SFNN_QAT_LABELS[args.qat]}",
                           "parallelism": f"dp{world}" if n > 1 else "single",
                           "l2": "no flush: each step streams 1.8 GB of FT optimizer state (> 126 MB L2)"}, **common)
            rl = None
            if not ref:
                l2p = r.get("l2_peak", {}).get("value")
                rl = sfnn_roofline(r["phase_ms"], args.batch, hbm, kind, l2p, qat=args.qat, data=args.data,
                                   shape=wl.shape())
        total = args.steps * args.batch * n
        line = {"metric": metric, "unit": "positions/s", "n_gpus": n, "steps": args.steps, "warmup": args.warmup,
                "value": round(total / (r["total_ms"] / 1000.0), 1),
                "ms_per_step": round(r["total_ms"] / args.steps, 4), "higher_is_better": True, "scaling": scaling,
                "vs_baseline": None, "dtype": "f32",
                "data": "synthetic (seeded; reference teacher-data shapes and distributions)", "config": config,
                "clocks": r["clocks"], "e2e": rounded(r["e2e"])}
        if ref:
            line.update(impl="reference", reference_run=reference_run)
            emit(line)
            return
        line.update(roofline=rl, gpu_launches=r["gpu_launches"], final_loss=r["final_loss"])
        for extra in ("e2e_async_loss", "e2e_records", "producer", "l2_peak", "exchange"):
            if extra in r:
                line[extra] = r[extra] if extra == "exchange" else rounded(r[extra])
        if rank == 0 and world == 1 and not args.no_cpu_baseline:
            if args.workload == "halfkp":
                line["cpu_baseline"] = halfkp_cpu_baseline()
            else:
                line["cpu_baseline"] = sfnn_cpu_baseline(wl.shape())
                if "producer" in line:
                    line["producer"]["cpu_baseline"] = teacher_cpu_baseline()
        emit(line)
    except (FileNotFoundError, OSError) as e:
        if not ref:
            raise
        emit({"impl": "reference", "unavailable": f"reference backend not built: {e}"})
    finally:
        if not ref:
            finish()


if __name__ == "__main__":
    main()
