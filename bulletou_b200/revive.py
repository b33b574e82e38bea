"""FT unit revival at an epoch boundary: saturated feature-transformer units
get fresh random rows, the L1 columns that read them are reset to +-1/64 with
the change absorbed into the L1 biases, and the optimizer state of everything
touched restarts.

Restates crates/cuda_cpp/src/ft_revive.rs (saturated_units :5-10,
Calibration :12-52, revive_ft / revive_ft_units :57-117,
compensate_ft_revival_mean :118-138) for the configurations this backend
trains: dense L1 with or without the shared L1 factorizer (the shared term of
crates/cuda_cpp/src/revive_common.rs Common::weight / bias, :228-238, with no
bucket-axis terms), no BatchNorm, no residual count gates, no legacy L2/L3
factorizers.  As in the reference the work is a download, a host-side edit
and an upload of the runner's device tensors; the random stream is the
persistent RevivalRng (crates/cuda_cpp/src/revival_rng.rs), kept on the runner
and saved in state.bin.
"""
from __future__ import annotations

from typing import Iterable, List, Sequence

import numpy as np

from ._lib import CudaCppError
from .state_bin import RevivalRng

F32 = np.float32


def saturated_units(hits: Sequence[int], perspectives: int, threshold: float) -> List[int]:
    """Units whose saturation share hits / perspectives reaches the threshold."""
    h = [int(x) for x in hits]
    if perspectives == 0 or not np.isfinite(threshold) or threshold <= 0.0 or threshold > 1.0 or \
            any(x > perspectives for x in h):
        raise CudaCppError("invalid FT saturation counts or threshold")
    return [i for i, x in enumerate(h) if x / perspectives >= threshold]


class FtCalibration:
    """Per-bucket mean of each FT output over the calibration positions whose
    mask weight is non-zero; an unobserved bucket takes the global mean."""

    def __init__(self, width: int, groups: int):
        self.width = int(width)
        self.counts = np.zeros(groups, np.int64)
        self.means = np.zeros(groups * width, np.float64)
        self._sums = np.zeros((groups, width), np.float64)

    def add(self, buckets, x, weights) -> None:
        b = np.asarray(buckets, np.int64).reshape(-1)
        x = np.asarray(x, np.float32)
        w = np.asarray(weights, np.float32).reshape(-1)
        if x.size != b.size * self.width:
            raise CudaCppError(f"FT calibration length mismatch: expected {b.size * self.width}, got {x.size}")
        if w.size != b.size:
            raise CudaCppError(f"FT calibration mask length mismatch: expected {b.size}, got {w.size}")
        if self.width == 0 or self.width % 2 != 0 or not np.all(np.isfinite(x)) or \
                not np.all(np.isfinite(w)) or np.any(w < 0) or np.any(b < 0) or np.any(b >= self.counts.size):
            raise CudaCppError("invalid FT revival calibration")
        keep = w != 0.0
        rows = x.reshape(b.size, self.width)[keep].astype(np.float64)
        kb = b[keep]
        np.add.at(self.counts, kb, 1)
        # sequential f64 sums per bucket in row order
        for bucket in np.unique(kb):
            sel = rows[kb == bucket]
            acc = self._sums[bucket]
            for r in sel:
                acc += r

    def finish_means(self) -> None:
        total = int(self.counts.sum())
        glob = np.zeros(self.width)
        if total:
            for b in range(self.counts.size):
                glob = glob + self._sums[b]
            glob = glob / total
        for b in range(self.counts.size):
            row = self._sums[b] / self.counts[b] if self.counts[b] > 0 else glob
            self.means[b * self.width:(b + 1) * self.width] = row


def _runner_rng(runner) -> RevivalRng:
    rng = getattr(runner, "revival_rng", None)
    if rng is None:
        rng = RevivalRng()
        runner.revival_rng = rng
    return rng


def begin_revival_epoch(runner) -> None:
    """l2_revive.rs begin_revival_epoch: clears the per-epoch revival flags
    (the random stream continues)."""
    runner.l1_revival_flags = 0
    runner.l2_revival_flags = 0


def _check(runner) -> None:
    if runner.present.get("l2fw") or runner.present.get("l3fw"):
        raise CudaCppError("FT revival requires calibrated non-BN SFNN, L1 none/shared/axis/pair, no residual count "
                           "gates or pending gradients")


def _shared_terms(ctx, runner):
    """Common::weight / bias of the shared factorizer: alpha * l1fw[col][u]
    (fast and slow copies), zero without it; the empty axis sum adds 0.0f."""
    sh = runner.shape
    n, ft = sh.l1_out, sh.ft_size
    if runner.present.get("l1fw"):
        a = F32(runner.alpha.shared)
        w = runner.weights["l1fw"].download(ctx).reshape(ft, n)
        sw = runner.optimizer_states["l1fw"].slow_params.download(ctx).reshape(ft, n)
        return (a * w).T + F32(0.0), (a * sw).T + F32(0.0)     # [u][col]
    z = np.zeros((n, ft), F32)
    return z, z


def _upload_state(ctx, st, state: dict) -> None:
    st.momentum.upload(state["momentum"], ctx)
    st.velocity.upload(state["velocity"], ctx)
    st.slow_params.upload(state["slow_params"], ctx)


def _round_half_away(x: np.ndarray) -> np.ndarray:
    d = x.astype(np.float64)
    return (np.sign(d) * np.floor(np.abs(d) + 0.5)).astype(F32)


def revive_ft(ctx, runner, c: FtCalibration, ids: Iterable[int], base_inputs: int) -> None:
    """Revive FT pairs: unit i and its partner i + ft/2 for each pair id."""
    pairs = runner.shape.ft_size // 2
    ids = [int(i) for i in ids]
    if any(i >= pairs or i < 0 for i in ids):
        raise CudaCppError("invalid FT pair")
    revive_ft_units(ctx, runner, c, [u for i in ids for u in (i, i + pairs)], base_inputs)


def revive_ft_units(ctx, runner, c: FtCalibration, units: Sequence[int], base_inputs: int) -> None:
    sh = runner.shape
    ft, pairs, n, S = sh.ft_size, sh.ft_size // 2, sh.l1_out, sh.num_stacks
    units = [int(u) for u in units]
    _check(runner)
    if c.width != ft or c.counts.size != S or base_inputs == 0 or base_inputs > sh.input_size or \
            any(u >= ft or u < 0 for u in units) or int(c.counts.sum()) == 0:
        raise CudaCppError("FT revival requires calibrated non-BN SFNN, L1 none/shared/axis/pair, no residual count "
                           "gates or pending gradients")
    if not units:
        return
    ids = sorted({u % pairs for u in units})
    cw, cws = _shared_terms(ctx, runner)
    # FT rows: real feature rows re-initialised, virtual factorizer rows zeroed
    w = runner.weights["l0w"].download(ctx).reshape(sh.input_size, ft)
    st = runner.optimizer_states["l0w"].download(ctx)
    mom, vel, slow = (st[k].reshape(sh.input_size, ft) for k in ("momentum", "velocity", "slow_params"))
    bound = max(F32(np.sqrt(F32(6.0) / F32(base_inputs + ft))), F32(1.0 / 127.0))
    rng = _runner_rng(runner)
    for col in units:
        draw = rng.signed_uniform_array(base_inputs)
        v = _round_half_away(draw * bound * F32(127.0)) / F32(127.0)
        w[:base_inputs, col] = v
        w[base_inputs:, col] = 0.0
        mom[:, col] = 0.0
        vel[:, col] = 0.0
        slow[:, col] = w[:, col]
    runner.weights["l0w"].upload(w, ctx)
    _upload_state(ctx, runner.optimizer_states["l0w"], {"momentum": mom, "velocity": vel, "slow_params": slow})
    del w, mom, vel, slow, st
    b0 = runner.weights["l0b"].download(ctx)
    s0 = runner.optimizer_states["l0b"].download(ctx)
    for col in units:
        b0[col] = 0.5
        s0["momentum"][col] = 0.0
        s0["velocity"][col] = 0.0
        s0["slow_params"][col] = 0.5
    runner.weights["l0b"].upload(b0, ctx)
    _upload_state(ctx, runner.optimizer_states["l0b"], s0)
    # L1: absorb the old contribution at the calibration mean into the bias,
    # then point the effective weight at +-1/64.
    w1 = runner.weights["l1w"].download(ctx).reshape(S, n, ft)
    b1 = runner.weights["l1b"].download(ctx).reshape(S, n)
    s1 = runner.optimizer_states["l1w"].download(ctx)
    sb = runner.optimizer_states["l1b"].download(ctx)
    m1, v1, sl1 = (s1[k].reshape(S, n, ft) for k in ("momentum", "velocity", "slow_params"))
    sbm, sbv, sbs = (sb[k].reshape(S, n) for k in ("momentum", "velocity", "slow_params"))
    means = c.means.astype(F32).reshape(S, ft)
    for i in ids:
        for col in (i, i + pairs):
            old = w1[:, :, col] + cw[None, :, col]
            old_slow = sl1[:, :, col] + cws[None, :, col]
            mean = means[:, col][:, None]
            b1 += old * mean
            sbs += old_slow * mean
            v = np.where(old < 0.0, F32(-1.0 / 64.0), F32(1.0 / 64.0)).astype(F32)
            w1[:, :, col] = v - cw[None, :, col]
            m1[:, :, col] = 0.0
            v1[:, :, col] = 0.0
            sl1[:, :, col] = v - cws[None, :, col]
    sbm[:] = 0.0
    sbv[:] = 0.0
    runner.weights["l1w"].upload(w1, ctx)
    _upload_state(ctx, runner.optimizer_states["l1w"], {"momentum": m1, "velocity": v1, "slow_params": sl1})
    runner.weights["l1b"].upload(b1, ctx)
    _upload_state(ctx, runner.optimizer_states["l1b"], {"momentum": sbm, "velocity": sbv, "slow_params": sbs})
    _invalidate_qat(runner)


def compensate_ft_revival_mean(ctx, runner, ids: Iterable[int], c: FtCalibration) -> None:
    """After a recalibration: move the revived columns' mean contribution out of
    the L1 biases (fast and slow copies)."""
    sh = runner.shape
    ft, n, S = sh.ft_size, sh.l1_out, sh.num_stacks
    ids = [int(i) for i in ids]
    if c.width != ft or c.counts.size != S or int(c.counts.sum()) == 0 or any(i >= ft // 2 or i < 0 for i in ids) \
            or not np.all(np.isfinite(c.means)):
        raise CudaCppError("invalid FT mean compensation")
    w1 = runner.weights["l1w"].download(ctx).reshape(S, n, ft)
    sw1 = runner.optimizer_states["l1w"].slow_params.download(ctx).reshape(S, n, ft)
    cw, cws = _shared_terms(ctx, runner)
    b1 = runner.weights["l1b"].download(ctx).reshape(S, n)
    sb1 = runner.optimizer_states["l1b"].slow_params.download(ctx).reshape(S, n)
    means = c.means.astype(F32).reshape(S, ft)
    for i in ids:
        for col in (i, i + ft // 2):
            m = means[:, col][:, None]
            b1 -= (w1[:, :, col] + cw[None, :, col]) * m
            sb1 -= (sw1[:, :, col] + cws[None, :, col]) * m
    runner.weights["l1b"].upload(b1, ctx)
    runner.optimizer_states["l1b"].slow_params.upload(sb1, ctx)
    _invalidate_qat(runner)


def _invalidate_qat(runner) -> None:
    # The fake-quantised L1 and layer-QAT copies are rebuilt from the masters.
    from .sfnn import SfnnLayerQatCopies

    runner.qat_l1 = None
    runner.layer_qat = SfnnLayerQatCopies()
