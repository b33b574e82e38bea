"""Unit revival at an epoch boundary: saturated feature-transformer units
get fresh random rows, the L1 columns that read them are reset to +-1/64 with
the change absorbed into the L1 biases, and the optimizer state of everything
touched restarts; dead or saturated L1 units get fresh rows the same way, with
the L2 weights that read them reset (crates/cuda_cpp/src/l1_revive.rs), and so
do L2 units, with the output weight reset (crates/cuda_cpp/src/l2_revive.rs,
the path without BatchNorm).

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


def _shared_bias(ctx, runner):
    """Common::bias of the shared factorizer: alpha * l1fb[u] (fast, slow)."""
    n = runner.shape.l1_out
    if runner.present.get("l1fb"):
        a = F32(runner.alpha.shared)
        b = runner.weights["l1fb"].download(ctx)
        sb = runner.optimizer_states["l1fb"].slow_params.download(ctx)
        return a * b + F32(0.0), a * sb + F32(0.0)
    z = np.zeros(n, F32)
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


# ------------------------------------------------------------------ L1 revival
class Contribution:
    """Exact mean-absolute-deviation utility of each unit's branches times the
    magnitude of its outgoing weights (crates/cuda_cpp/src/l1_revive.rs
    Contribution, :5-58); units whose utility relative to the bucket's best
    is below the threshold are selected."""

    def __init__(self, width: int, groups: int):
        self.width = int(width)
        self.values = [[] for _ in range(groups)]
        self.means = np.zeros(groups * width, np.float64)
        self.utility = np.zeros(0)
        self.relative = np.zeros(0)
        self.threshold = 0.01

    def add(self, bucket: int, y) -> None:
        self.values[bucket].append(np.asarray(y, np.float32).reshape(-1, self.width))

    def finish(self, w, out: int, branches: int, threshold: float) -> None:
        if not np.isfinite(threshold) or threshold <= 0.0 or threshold > 1.0:
            raise CudaCppError("revive contribution threshold must be finite and in (0, 1]")
        w = np.asarray(w, np.float32).reshape(-1)
        if w.size != len(self.values) * out * self.width:
            raise CudaCppError(f"revive outgoing weights length mismatch: expected "
                               f"{len(self.values) * out * self.width}, got {w.size}")
        if not np.all(np.isfinite(w)) or branches == 0 or self.width % branches != 0:
            raise CudaCppError("invalid contribution weights or branch layout")
        units = self.width // branches
        G = len(self.values)
        self.utility = np.zeros(G * units)
        self.relative = np.zeros(G * units)
        self.threshold = threshold
        wb = np.abs(w.reshape(G, out, self.width).astype(np.float64))
        for b, chunks in enumerate(self.values):
            ys = np.concatenate(chunks).astype(np.float64) if chunks else np.zeros((0, self.width))
            n = ys.shape[0]
            if n == 0:
                continue
            mean = np.zeros(self.width)
            for row in ys:
                mean += row
            mean /= n
            self.means[b * self.width:(b + 1) * self.width] = mean
            dev = np.zeros(self.width)
            for row in ys:
                dev += np.abs(row - mean)
            mad = dev / n
            norm = np.zeros(self.width)
            for j in range(out):
                norm += wb[b, j]
            for col in range(self.width):
                self.utility[b * units + col % units] += mad[col] * norm[col]
            mx = max(0.0, float(self.utility[b * units:(b + 1) * units].max()))
            if mx > 0.0:
                self.relative[b * units:(b + 1) * units] = self.utility[b * units:(b + 1) * units] / mx
        if not (np.all(np.isfinite(self.utility)) and np.all(np.isfinite(self.relative))):
            raise CudaCppError("non-finite revival contribution")
        self.values = [[] for _ in range(G)]

    def selected(self, counts, units: int) -> List[int]:
        return [i for i in range(self.relative.size) if counts[i // units] >= 1024 and self.relative[i] < self.threshold]


class L1Calibration:
    """Per-bucket statistics of the L1 branches over calibration positions
    (l1_revive.rs Calibration, :60-146): input sums, branch sums, the upper /
    zero saturation counts and the contribution samples."""

    def __init__(self, input_size: int, width: int, groups: int):
        self.input, self.width = int(input_size), int(width)
        self.counts = np.zeros(groups, np.int64)
        self.upper = np.zeros(groups * width, np.int64)
        self.lower = np.zeros(groups * width, np.int64)
        self.upper_threshold = 0.99
        self.zero_threshold = 0.99
        self.sums = np.zeros(groups * input_size, np.float64)
        self.branch_sums = np.zeros(groups * 2 * width, np.float64)
        self.contribution = Contribution(2 * width, groups)

    def set_thresholds(self, upper: float, zero: float) -> None:
        if any(not np.isfinite(v) or v <= 0.0 or v > 1.0 for v in (upper, zero)):
            raise CudaCppError("revival thresholds must be finite and in (0, 1]")
        self.upper_threshold, self.zero_threshold = upper, zero

    def is_upper(self, i: int, enabled: bool) -> bool:
        n = self.counts[i // self.width]
        return bool(enabled and n >= 1024 and self.upper[i] / n >= self.upper_threshold)

    def is_zero(self, i: int, enabled: bool) -> bool:
        n = self.counts[i // self.width]
        return bool(enabled and n >= 1024 and self.lower[i] / n >= self.zero_threshold)

    def add(self, buckets, x, y, weights=None) -> None:
        """x: combined FT input [n][input]; y: [n][square branches, normal branches]."""
        b = np.asarray(buckets, np.int64).reshape(-1)
        x = np.asarray(x, np.float32).reshape(-1)
        y = np.asarray(y, np.float32).reshape(-1)
        if x.size != b.size * self.input:
            raise CudaCppError(f"L1 revival inputs length mismatch: expected {b.size * self.input}, got {x.size}")
        if y.size != b.size * 2 * self.width:
            raise CudaCppError(f"L1 revival branches length mismatch: expected {b.size * 2 * self.width}, got {y.size}")
        if weights is not None:
            weights = np.asarray(weights, np.float32).reshape(-1)
            if weights.size != b.size:
                raise CudaCppError(f"L1 revival sample weights length mismatch: expected {b.size}, got {weights.size}")
            if not np.all(np.isfinite(weights)) or np.any(weights < 0):
                raise CudaCppError("invalid L1 revival sample weight")
        if not (np.all(np.isfinite(x)) and np.all(np.isfinite(y))) or np.any(b < 0) or np.any(b >= self.counts.size):
            raise CudaCppError("invalid L1 revival calibration")
        X = x.reshape(b.size, self.input)
        Y = y.reshape(b.size, 2 * self.width)
        W, I = self.width, self.input
        for row in range(b.size):
            if weights is not None and weights[row] == 0.0:
                continue
            k = int(b[row])
            self.counts[k] += 1
            self.contribution.add(k, Y[row])
            self.sums[k * I:(k + 1) * I] += X[row].astype(np.float64)
            sq, nm = Y[row, :W], Y[row, W:]
            self.branch_sums[2 * k * W:(2 * k + 1) * W] += sq.astype(np.float64)
            self.branch_sums[(2 * k + 1) * W:(2 * k + 2) * W] += nm.astype(np.float64)
            self.upper[k * W:(k + 1) * W] += ((sq >= 1.0) & (nm >= 1.0))
            self.lower[k * W:(k + 1) * W] += ((sq <= 0.0) & (nm <= 0.0))

    def candidates_for(self, upper: bool, zero: bool) -> List[int]:
        if self.contribution.relative.size:
            return self.contribution.selected(self.counts, self.width) if (upper or zero) else []
        return [i for i in range(self.upper.size) if self.is_upper(i, upper) or self.is_zero(i, zero)]


def _flags(runner, name: str) -> int:
    return int(getattr(runner, name, 0))


def revive_l1_selected(ctx, runner, c: L1Calibration, upper: bool, zero: bool) -> List[int]:
    """Reinitialise the selected L1 units (bucket * l1_hidden + unit) from the
    revival stream with the bias that puts their calibration mean at 0.5, and
    point the L2 weights reading their two branches at +-1/64 with the old
    branch constants absorbed into the L2 biases (revive_l1_selected,
    l1_revive.rs:150-225).  Once per revival epoch for each kind."""
    flags = _flags(runner, "l1_revival_flags")
    upper = upper and not (flags & 1)
    zero = zero and not (flags & 2)
    if not upper and not zero:
        return []
    if runner.present.get("l2fw") or runner.present.get("l3fw"):
        raise CudaCppError("L1 revival requires non-BN L1 (none/shared/axis/pair), no residual count gates or legacy "
                           "L2/L3 factorizers, and no pending gradients")
    sh = runner.shape
    H, n, ft, S, L2 = sh.l1_hidden, sh.l1_out, sh.ft_size, sh.num_stacks, sh.l2_size
    l2_in = sh.l2_in
    if c.input != ft or c.width != H or c.counts.size != S or int(c.counts.sum()) == 0:
        raise CudaCppError("empty or incompatible L1 calibration")
    ids = c.candidates_for(upper, zero)
    w1 = runner.weights["l1w"].download(ctx).reshape(S * n, ft)
    b1 = runner.weights["l1b"].download(ctx)
    w2 = runner.weights["l2w"].download(ctx).reshape(S * L2, l2_in)
    b2 = runner.weights["l2b"].download(ctx)
    ws = runner.optimizer_states["l1w"].download(ctx)
    bs_ = runner.optimizer_states["l1b"].download(ctx)
    os_ = runner.optimizer_states["l2w"].download(ctx)
    obs = runner.optimizer_states["l2b"].download(ctx)
    wsm, wsv, wss = (ws[k].reshape(S * n, ft) for k in ("momentum", "velocity", "slow_params"))
    osm, osv, oss = (os_[k].reshape(S * L2, l2_in) for k in ("momentum", "velocity", "slow_params"))
    cw, cws = _shared_terms(ctx, runner)
    cb, cbs = _shared_bias(ctx, runner)
    rng = _runner_rng(runner)
    bound = F32(np.sqrt(F32(6.0) / F32(ft + H)))
    for i in ids:
        bucket, u = divmod(i, H)
        out = bucket * n + u
        value = rng.signed_uniform_array(ft) * bound
        mean = 0.0
        sums = c.sums[bucket * ft:(bucket + 1) * ft]
        cnt = float(c.counts[bucket])
        terms = value.astype(np.float64) * sums / cnt
        for t in terms:
            mean += t
        w1[out] = value - cw[u]
        wsm[out] = 0.0
        wsv[out] = 0.0
        wss[out] = value - cws[u]
        bias = F32(0.5) - F32(mean)
        b1[out] = bias - cb[u]
        bs_["momentum"][out] = 0.0
        bs_["velocity"][out] = 0.0
        bs_["slow_params"][out] = bias - cbs[u]
        for j in range(L2):
            row = bucket * L2 + j
            for col in (u, H + u):
                constant = F32(c.branch_sums[bucket * 2 * H + col] / cnt)
                b2[row] += constant * w2[row, col]
                obs["slow_params"][row] += constant * oss[row, col]
                v = F32(-1.0 / 64.0) if w2[row, col] < 0.0 else F32(1.0 / 64.0)
                w2[row, col] = v
                osm[row, col] = 0.0
                osv[row, col] = 0.0
                oss[row, col] = v
            obs["momentum"][row] = 0.0
            obs["velocity"][row] = 0.0
    if not all(np.all(np.isfinite(a)) for a in (w1, b1, w2, b2, wss, bs_["slow_params"], obs["slow_params"])):
        raise CudaCppError("non-finite L1 revival result")
    runner.weights["l1w"].upload(w1, ctx)
    _upload_state(ctx, runner.optimizer_states["l1w"], {"momentum": wsm, "velocity": wsv, "slow_params": wss})
    runner.weights["l1b"].upload(b1, ctx)
    _upload_state(ctx, runner.optimizer_states["l1b"], bs_)
    runner.weights["l2w"].upload(w2, ctx)
    _upload_state(ctx, runner.optimizer_states["l2w"], {"momentum": osm, "velocity": osv, "slow_params": oss})
    runner.weights["l2b"].upload(b2, ctx)
    _upload_state(ctx, runner.optimizer_states["l2b"], obs)
    _invalidate_qat(runner)
    runner.l1_revival_flags = flags | int(upper) | (int(zero) << 1)
    return ids


def compensate_l1_revival_mean(ctx, runner, ids: Sequence[int], c: L1Calibration) -> None:
    """Subtract the revived branches' measured means at each L2 preactivation
    (compensate_l1_revival_mean, l1_revive.rs:227-258)."""
    if not ids:
        return
    sh = runner.shape
    H, S, L2, l2_in = sh.l1_hidden, sh.num_stacks, sh.l2_size, sh.l2_in
    if c.width != H or c.counts.size != S or any(i >= S * H or c.counts[i // H] == 0 for i in ids):
        raise CudaCppError("invalid L1 revival mean calibration")
    w = runner.weights["l2w"].download(ctx).reshape(S * L2, l2_in)
    sw = runner.optimizer_states["l2w"].slow_params.download(ctx).reshape(S * L2, l2_in)
    b = runner.weights["l2b"].download(ctx)
    sb_ = runner.optimizer_states["l2b"].slow_params.download(ctx)
    for i in ids:
        bucket, u = divmod(int(i), H)
        for col in (u, H + u):
            mean = F32(c.branch_sums[bucket * 2 * H + col] / float(c.counts[bucket]))
            rows = slice(bucket * L2, (bucket + 1) * L2)
            b[rows] -= w[rows, col] * mean
            sb_[rows] -= sw[rows, col] * mean
    if not (np.all(np.isfinite(b)) and np.all(np.isfinite(sb_))):
        raise CudaCppError("non-finite L1 revival mean compensation")
    runner.weights["l2b"].upload(b, ctx)
    runner.optimizer_states["l2b"].slow_params.upload(sb_, ctx)
    from .sfnn import SfnnLayerQatCopies

    runner.layer_qat = SfnnLayerQatCopies()


# ------------------------------------------------------------------ L2 revival
class L2Calibration:
    """Per-bucket L2 statistics (crates/cuda_cpp/src/l2_revive.rs Calibration,
    :4-74): the L2 inputs of every calibration position, activation sums,
    upper / zero saturation counts and the contribution samples."""

    def __init__(self, input_size: int, width: int, groups: int):
        self.input, self.width = int(input_size), int(width)
        self.counts = np.zeros(groups, np.int64)
        self.upper = np.zeros(groups * width, np.int64)
        self.lower = np.zeros(groups * width, np.int64)
        self.upper_threshold = 0.99
        self.zero_threshold = 0.99
        self.inputs = [[] for _ in range(groups)]
        self.contribution = Contribution(width, groups)
        self.sums = np.zeros(groups * width, np.float64)

    set_thresholds = L1Calibration.set_thresholds
    is_upper = L1Calibration.is_upper
    is_zero = L1Calibration.is_zero

    def add(self, buckets, x, y, weights=None) -> None:
        b = np.asarray(buckets, np.int64).reshape(-1)
        x = np.asarray(x, np.float32).reshape(-1)
        y = np.asarray(y, np.float32).reshape(-1)
        if x.size != b.size * self.input:
            raise CudaCppError(f"revive inputs length mismatch: expected {b.size * self.input}, got {x.size}")
        if y.size != b.size * self.width:
            raise CudaCppError(f"revive outputs length mismatch: expected {b.size * self.width}, got {y.size}")
        if weights is not None:
            weights = np.asarray(weights, np.float32).reshape(-1)
            if weights.size != b.size:
                raise CudaCppError(f"L2 revival sample weights length mismatch: expected {b.size}, got {weights.size}")
            if not np.all(np.isfinite(weights)) or np.any(weights < 0):
                raise CudaCppError("invalid L2 revival sample weight")
        if not (np.all(np.isfinite(x)) and np.all(np.isfinite(y))) or np.any(b < 0) or np.any(b >= self.counts.size):
            raise CudaCppError("invalid L2 revival calibration")
        X = x.reshape(b.size, self.input)
        Y = y.reshape(b.size, self.width)
        W = self.width
        for row in range(b.size):
            if weights is not None and weights[row] == 0.0:
                continue
            k = int(b[row])
            self.counts[k] += 1
            self.contribution.add(k, Y[row])
            self.inputs[k].append(X[row].copy())
            self.sums[k * W:(k + 1) * W] += Y[row].astype(np.float64)
            self.upper[k * W:(k + 1) * W] += Y[row] >= 1.0
            self.lower[k * W:(k + 1) * W] += Y[row] <= 0.0

    def candidates(self) -> List[int]:
        return self.candidates_for(True, False)

    candidates_for = L1Calibration.candidates_for


def _seq_sum(values) -> float:
    acc = 0.0
    for v in values:
        acc += float(v)
    return acc


def revive_l2_selected(ctx, runner, c: L2Calibration, upper: bool, zero: bool) -> List[int]:
    """Reinitialise the selected L2 units from the revival stream with the bias
    that centres their calibration pre-activation at 0.5, point their output
    weight at +-1/64 and move the old mean contribution (and the new unit's
    quantised mean) into the output bias (revive_l2_selected,
    l2_revive.rs:96-175, the path without BatchNorm)."""
    flags = _flags(runner, "l2_revival_flags")
    upper = upper and not (flags & 1)
    zero = zero and not (flags & 2)
    if not upper and not zero:
        return []
    if runner.present.get("l2fw") or runner.present.get("l3fw"):
        raise CudaCppError("L2 revival requires SFNN L1 (none/shared/axis/pair), no legacy L2/L3 factorizer or "
                           "residual gates, and no pending gradients")
    sh = runner.shape
    I, L2, S = sh.l2_in, sh.l2_size, sh.num_stacks
    if c.input != I or c.width != L2 or c.counts.size != S or int(c.counts.sum()) == 0:
        raise CudaCppError("empty or incompatible L2 calibration")
    ids = c.candidates_for(upper, zero)
    w = runner.weights["l2w"].download(ctx).reshape(S * L2, I)
    b = runner.weights["l2b"].download(ctx)
    out = runner.weights["l3w"].download(ctx)
    ob = runner.weights["l3b"].download(ctx)
    ws = runner.optimizer_states["l2w"].download(ctx)
    bs_ = runner.optimizer_states["l2b"].download(ctx)
    os_ = runner.optimizer_states["l3w"].download(ctx)
    obs = runner.optimizer_states["l3b"].download(ctx)
    wsm, wsv, wss = (ws[k].reshape(S * L2, I) for k in ("momentum", "velocity", "slow_params"))
    rng = _runner_rng(runner)
    bound = F32(np.sqrt(F32(6.0) / F32(I + L2)))
    for i in ids:
        g = i // L2
        w[i] = rng.signed_uniform_array(I) * bound
        wsm[i] = 0.0
        wsv[i] = 0.0
        wss[i] = w[i]
        rows = np.array(c.inputs[g], np.float64).reshape(-1, I)
        count = float(c.counts[g])
        wq = (_round_half_away(w[i] * F32(64.0)) / F32(64.0)).astype(np.float64)
        wd = w[i].astype(np.float64)
        dot = np.zeros(rows.shape[0])
        dq = np.zeros(rows.shape[0])
        for k in range(I):
            dot += rows[:, k] * wd[k]
            dq += rows[:, k] * wq[k]
        mean_dot = _seq_sum(dot) / count
        beta = F32(0.5) - F32(mean_dot)
        bq = float(_round_half_away(np.array([beta * F32(8128.0)], F32))[0] / F32(8128.0))
        mean_y = _seq_sum(np.clip(dq + bq, 0.0, 1.0)) / count
        v = F32(-1.0 / 64.0) if out[i] < 0.0 else F32(1.0 / 64.0)
        old_activation = F32(c.sums[i] / count)
        my = F32(mean_y)
        ob[g] += old_activation * out[i] - v * my
        obs["slow_params"][g] += old_activation * os_["slow_params"][i] - v * my
        out[i] = v
        os_["slow_params"][i] = v
        os_["momentum"][i] = 0.0
        os_["velocity"][i] = 0.0
        b[i] = beta
        bs_["slow_params"][i] = beta
        bs_["momentum"][i] = 0.0
        bs_["velocity"][i] = 0.0
    if not all(np.all(np.isfinite(a)) for a in (w, b, out, ob)):
        raise CudaCppError("non-finite L2 revival result")
    runner.weights["l2w"].upload(w, ctx)
    runner.weights["l2b"].upload(b, ctx)
    runner.weights["l3w"].upload(out, ctx)
    runner.weights["l3b"].upload(ob, ctx)
    _upload_state(ctx, runner.optimizer_states["l2w"], {"momentum": wsm, "velocity": wsv, "slow_params": wss})
    _upload_state(ctx, runner.optimizer_states["l2b"], bs_)
    _upload_state(ctx, runner.optimizer_states["l3w"], os_)
    _upload_state(ctx, runner.optimizer_states["l3b"], obs)
    runner.l2_revival_flags = flags | int(upper) | (int(zero) << 1)
    from .sfnn import SfnnLayerQatCopies

    runner.layer_qat = SfnnLayerQatCopies()
    return ids


def revive_l2(ctx, runner, c: L2Calibration) -> List[int]:
    return revive_l2_selected(ctx, runner, c, True, False)
