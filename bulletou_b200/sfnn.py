"""SFNN LayerStack part of the cuda-cpp crate mirror (crates/cuda_cpp/src/lib.rs).

``SfnnForwardShape`` (lib.rs:928-1056), ``SfnnFactorizerAlpha`` (lib.rs:1280),
``SfnnForwardHostWeights`` (lib.rs:1405), ``SfnnTrainStepHostBatch``
(lib.rs:6027), the forward / backward entry points (lib.rs:2014-2253,
3462-4090) and ``SfnnTrainStepRunner`` (lib.rs:6187-7960) with default layer
multipliers and the FT / shared-L1 factorizers.

Bound to the product library the runner issues one fused call per step
(bulletou_b200_sfnn_train_step_device); bound to the reference backend it
issues the reference runner's call sequence: forward with the gradient
buffer as fold scratch (then cleared, lib.rs:2078-2084), loss, training
backward, and Ranger over every group in update order (lib.rs:8425-8730).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, replace
from typing import Optional

import numpy as np

from ._lib import CudaCppError, QuantRounding, SfnnQat, SfnnShape
from .cuda_cpp import (FLT_MAX, Context, Event, F32Buffer, I32Buffer, PinnedF32Buffer, PinnedI32Buffer,
                       RangerDeviceState, RangerParamState, RangerUpdateParams, ScalarLossKind, ScalarLossReadback,
                       ScalarLossWorkspace, ranger_update_device, scalar_loss_device, upload_from_pinned)

HALFKA_HM2_DIMENSIONS = 73305
HALFKA2_DIMENSIONS = 131949
PIECE_INPUTS = 1629
SFNN_WEIGHT_NAMES = ("l0w", "l0b", "l1w", "l1b", "l1fw", "l1fb", "l2w", "l2b", "l2fw", "l2fb", "l3w", "l3b", "l3fw",
                     "l3fb")
SHARED_NAMES = ("l1fw", "l1fb", "l2fw", "l2fb", "l3fw", "l3fb")


@dataclass(frozen=True)
class SfnnForwardShape:
    """Dense-L1 SFNN shape (lib.rs:928-1056); grouped / common+shard L1 and the
    bucket-axis factorizers are not supported by this backend."""

    input_size: int
    ft_size: int
    l1_hidden: int
    l1_skip: bool
    l2_size: int
    num_stacks: int

    @property
    def l1_out(self) -> int:
        return self.l1_hidden + int(self.l1_skip)

    @property
    def l2_in(self) -> int:
        return 2 * self.l1_hidden

    @property
    def pairwise_size(self) -> int:
        return self.ft_size // 2

    def factorized_base(self) -> int:
        """cu:1180-1184: input_size = base + 1629 virtual piece rows."""
        return {HALFKA_HM2_DIMENSIONS + PIECE_INPUTS: HALFKA_HM2_DIMENSIONS,
                HALFKA2_DIMENSIONS + PIECE_INPUTS: HALFKA2_DIMENSIONS}.get(self.input_size, 0)

    def weight_lengths(self) -> dict:
        W, O, L2, I2, S = self.ft_size, self.l1_out, self.l2_size, self.l2_in, self.num_stacks
        return {"l0w": self.input_size * W, "l0b": W, "l1w": S * O * W, "l1b": S * O, "l1fw": W * O, "l1fb": O,
                "l2w": S * L2 * I2, "l2b": S * L2, "l2fw": L2 * I2, "l2fb": L2, "l3w": S * L2, "l3b": S,
                "l3fw": L2, "l3fb": 1}

    def as_tuple(self) -> tuple:
        return (self.input_size, self.ft_size, self.l1_hidden, int(self.l1_skip), self.l2_size, self.num_stacks)

    def validate(self) -> None:
        if min(self.input_size, self.ft_size, self.l1_hidden, self.l2_size, self.num_stacks) <= 0:
            raise CudaCppError("invalid SFNN shape: every dimension must be > 0")
        if self.ft_size % 2 != 0:
            raise CudaCppError(f"invalid SFNN shape: ft_size must be even, got {self.ft_size}")


# SFNN_halfkahm2_1536_15_32_k3k3 with the FT factorizer (docs/en/shogi/sfnn-1536.md:27-57)
SFNN_HALFKA_HM2_1536_15_32_K3K3 = SfnnForwardShape(HALFKA_HM2_DIMENSIONS + PIECE_INPUTS, 1536, 15, True, 32, 9)


@dataclass(frozen=True)
class SfnnFactorizerAlpha:
    """lib.rs:1280-1312 (ft and shared coefficients; axis terms unsupported)."""

    ft: float = 1.0
    shared: float = 1.0

    def validate(self) -> None:
        if not (np.isfinite(self.ft) and 0.0 <= self.ft <= 100.0):
            raise CudaCppError("SFNN FT factorizer alpha must be in [0, 100]")
        if not (np.isfinite(self.shared) and 0.0 <= self.shared <= 10.0):
            raise CudaCppError("SFNN shared factorizer alpha must be in [0, 10]")


@dataclass
class SfnnForwardHostWeights:
    shape: SfnnForwardShape
    l0w: np.ndarray
    l0b: np.ndarray
    l1w: np.ndarray
    l1b: np.ndarray
    l2w: np.ndarray
    l2b: np.ndarray
    l3w: np.ndarray
    l3b: np.ndarray
    l1fw: Optional[np.ndarray] = None
    l1fb: Optional[np.ndarray] = None
    l2fw: Optional[np.ndarray] = None
    l2fb: Optional[np.ndarray] = None
    l3fw: Optional[np.ndarray] = None
    l3fb: Optional[np.ndarray] = None

    def arrays(self) -> dict:
        return {n: (None if getattr(self, n) is None else np.ascontiguousarray(getattr(self, n), np.float32).reshape(-1))
                for n in SFNN_WEIGHT_NAMES}

    def validate(self) -> None:
        self.shape.validate()
        lens = self.shape.weight_lengths()
        for a, b in (("l1fw", "l1fb"), ("l2fw", "l2fb"), ("l3fw", "l3fb")):
            if (getattr(self, a) is None) != (getattr(self, b) is None):
                raise CudaCppError(f"SFNN factorized state is partial: {a}/{b}")
        for n, a in self.arrays().items():
            if a is not None and a.size != lens[n]:
                raise CudaCppError(f"weight length mismatch for {n}: expected {lens[n]}, got {a.size}")


@dataclass
class SfnnTrainStepHostBatch:
    stm_indices: np.ndarray
    nstm_indices: np.ndarray
    buckets: np.ndarray
    targets: np.ndarray
    entry_weights: np.ndarray
    batch_size: int
    max_active: int

    def validate(self) -> None:
        n = self.batch_size * self.max_active
        if np.asarray(self.stm_indices).size != n or np.asarray(self.nstm_indices).size != n:
            raise CudaCppError("SFNN batch: sparse index length mismatch")
        for name in ("buckets", "targets", "entry_weights"):
            if np.asarray(getattr(self, name)).size != self.batch_size:
                raise CudaCppError(f"SFNN batch: {name} length mismatch")


class SfnnForwardWorkspace:
    """lib.rs:1936-2012."""

    def __init__(self, ctx: Context, shape: SfnnForwardShape, batch_size: int):
        W = shape.ft_size
        self.layout = (shape, batch_size)
        self.stm_l0 = F32Buffer(ctx, batch_size * W)
        self.nstm_l0 = F32Buffer(ctx, batch_size * W)
        self.combined = F32Buffer(ctx, batch_size * W)
        self.l1 = F32Buffer(ctx, batch_size * shape.l1_out)
        self.l2_input = F32Buffer(ctx, batch_size * shape.l2_in)
        self.l2 = F32Buffer(ctx, batch_size * shape.l2_size)
        self.output = F32Buffer(ctx, batch_size)

    def download(self, ctx: Optional[Context] = None) -> dict:
        return {k: getattr(self, k).download(ctx) for k in ("stm_l0", "nstm_l0", "combined", "l1", "l2_input", "l2",
                                                              "output")}


class SfnnBackwardWorkspace:
    """Activation gradients plus one gradient buffer per present parameter group."""

    INTERMEDIATE = ("l2_gradients", "l1_gradients", "l2_input_gradients", "combined_gradients", "stm_l0_gradients",
                    "nstm_l0_gradients", "stm_l0_pre_gradients", "nstm_l0_pre_gradients")

    def __init__(self, ctx: Context, shape: SfnnForwardShape, batch_size: int, present: dict):
        W = shape.ft_size
        sizes = {"l2_gradients": batch_size * shape.l2_size, "l1_gradients": batch_size * shape.l1_out,
                 "l2_input_gradients": batch_size * shape.l2_in}
        for k in self.INTERMEDIATE:
            setattr(self, k, F32Buffer(ctx, sizes.get(k, batch_size * W)))
        # Every gradient buffer exists, as in the reference workspace
        # (lib.rs:3260-3300): shared-factor gradients at full size even when
        # the factor is absent, bucket-axis gradients with length 0.
        lens = shape.weight_lengths()
        self.present = dict(present)
        self.params = {}
        for n in SFNN_WEIGHT_NAMES:
            b = F32Buffer(ctx, lens[n])
            b.fill(0.0)
            self.params[n] = b
        self.axis = {n: F32Buffer(ctx, 0) for n in ("l1axw", "l1axb", "l2axw", "l2axb", "l3axw", "l3axb")}

    def zero_parameter_gradients(self, ctx: Optional[Context] = None) -> None:
        for b in self.params.values():
            b.fill(0.0, ctx)

    def download(self, ctx: Optional[Context] = None) -> dict:
        out = {k: getattr(self, k).download(ctx) for k in self.INTERMEDIATE}
        out.update({f"{n}_gradients": b.download(ctx) for n, b in self.params.items() if self.present[n]})
        return out


def _p(b: Optional[F32Buffer]):
    return None if b is None else b.as_ptr()


def sfnn_forward_device(ctx: Context, shape: SfnnForwardShape, batch_size: int, max_active: int, stm: I32Buffer,
                        nstm: I32Buffer, buckets: I32Buffer, weights: dict, ws: SfnnForwardWorkspace,
                        alpha: SfnnFactorizerAlpha = SfnnFactorizerAlpha(),
                        folded_l0w: Optional[F32Buffer] = None, qat_l1: Optional["SfnnL1Qat"] = None,
                        refresh_qat_l1: int = 1) -> None:
    """bulletou_cuda_cpp_sfnn_forward_device (lib.rs:2033-2253 argument order).
    qat_l1: the L1 QAT scratch (weights, bias); refresh_qat_l1 as in the
    reference (1 rebuild quantised, 0 reuse)."""
    w = weights
    has = [int(w[n] is not None) for n in ("l1fw", "l2fw", "l3fw")]
    ctx.lib.call(
        "bulletou_cuda_cpp_sfnn_forward_device", ctx.as_ptr(), shape.input_size, shape.ft_size, shape.l1_hidden,
        int(shape.l1_skip), shape.l2_size, shape.num_stacks, 1, 0, 0, 0, 0, batch_size, max_active, stm.as_ptr(),
        nstm.as_ptr(), buckets.as_ptr(), _p(w["l0w"]), _p(folded_l0w), _p(w["l0b"]), _p(w["l1w"]), _p(w["l1b"]),
        _p(w["l1fw"]), _p(w["l1fb"]), has[0], None, None, 0, _p(w["l2w"]), _p(w["l2b"]), _p(w["l2fw"]),
        _p(w["l2fb"]), has[1], None, None, 0, _p(w["l3w"]), _p(w["l3b"]), _p(w["l3fw"]), _p(w["l3fb"]), has[2], None,
        None, 0, 0, 0, 0, 0, 0, 0, alpha.ft, alpha.shared, 1.0, 1.0, 1.0, 1.0, None, None, ws.stm_l0.as_ptr(),
        ws.nstm_l0.as_ptr(), ws.combined.as_ptr(), ws.l1.as_ptr(), ws.l2_input.as_ptr(), ws.l2.as_ptr(),
        ws.output.as_ptr(), None if qat_l1 is None else qat_l1.weights.as_ptr(),
        None if qat_l1 is None else qat_l1.bias.as_ptr(), 0 if qat_l1 is None else int(refresh_qat_l1))


def _backward_args(ctx, shape, batch_size, max_active, stm, nstm, buckets, weights, fws, mean_output_gradients, bws,
                   alpha, qat_l1_weights):
    w, g, ax = weights, bws.params, bws.axis
    has = [int(w[n] is not None) for n in ("l1fw", "l2fw", "l3fw")]
    return [
        ctx.as_ptr(), shape.input_size, shape.ft_size,
        shape.l1_hidden, int(shape.l1_skip), shape.l2_size, shape.num_stacks, 1, 0, 0, 0, 0, batch_size, max_active,
        stm.as_ptr(), nstm.as_ptr(), buckets.as_ptr(), fws.stm_l0.as_ptr(), fws.nstm_l0.as_ptr(),
        fws.combined.as_ptr(), fws.l1.as_ptr(), fws.l2_input.as_ptr(), fws.l2.as_ptr(), _p(w["l1w"]),
        _p(qat_l1_weights),
        _p(w["l1fw"]), has[0], None, 0, _p(w["l2w"]), _p(w["l2fw"]), has[1], None, 0, _p(w["l3w"]), _p(w["l3fw"]),
        has[2], None, 0, 0, 0, 0, 0, 0, 0, alpha.ft, alpha.shared, 1.0, 1.0, 1.0, 1.0, None, None,
        mean_output_gradients.as_ptr(), *[getattr(bws, k).as_ptr() for k in bws.INTERMEDIATE], _p(g["l0w"]),
        _p(g["l0b"]), _p(g["l1w"]), _p(g["l1b"]), _p(g["l1fw"]), _p(g["l1fb"]), _p(ax["l1axw"]), _p(ax["l1axb"]),
        _p(g["l2w"]), _p(g["l2b"]), _p(g["l2fw"]), _p(g["l2fb"]), _p(ax["l2axw"]), _p(ax["l2axb"]), _p(g["l3w"]),
        _p(g["l3b"]), _p(g["l3fw"]), _p(g["l3fb"]), _p(ax["l3axw"]), _p(ax["l3axb"])]


def sfnn_backward_train_device(ctx: Context, shape: SfnnForwardShape, batch_size: int, max_active: int,
                               stm: I32Buffer, nstm: I32Buffer, buckets: I32Buffer, weights: dict,
                               fws: SfnnForwardWorkspace, mean_output_gradients: F32Buffer,
                               bws: SfnnBackwardWorkspace, alpha: SfnnFactorizerAlpha = SfnnFactorizerAlpha(),
                               zero_parameter_gradients: bool = False,
                               entry_weights: Optional[F32Buffer] = None,
                               qat_l1_weights: Optional[F32Buffer] = None) -> None:
    """bulletou_cuda_cpp_sfnn_backward_train_device (lib.rs:3529-4090 argument order);
    qat_l1_weights: the forward's L1 QAT weights (input gradients use them)."""
    args = _backward_args(ctx, shape, batch_size, max_active, stm, nstm, buckets, weights, fws,
                          mean_output_gradients, bws, alpha, qat_l1_weights)
    ctx.lib.call("bulletou_cuda_cpp_sfnn_backward_train_device", *args, int(zero_parameter_gradients),
                 _p(entry_weights))


def sfnn_backward_device(ctx: Context, shape: SfnnForwardShape, batch_size: int, max_active: int, stm: I32Buffer,
                         nstm: I32Buffer, buckets: I32Buffer, weights: dict, fws: SfnnForwardWorkspace,
                         mean_output_gradients: F32Buffer, bws: SfnnBackwardWorkspace,
                         alpha: SfnnFactorizerAlpha = SfnnFactorizerAlpha(),
                         qat_l1_weights: Optional[F32Buffer] = None) -> None:
    """bulletou_cuda_cpp_sfnn_backward_device (lib.rs:4002): the backward with
    every parameter gradient cleared first."""
    ctx.lib.call("bulletou_cuda_cpp_sfnn_backward_device",
                 *_backward_args(ctx, shape, batch_size, max_active, stm, nstm, buckets, weights, fws,
                                 mean_output_gradients, bws, alpha, qat_l1_weights))


SFNN_BACKWARD_PROFILE_STAGES = ("zero", "l3", "l2", "l2_input", "l1", "l0", "total")


def sfnn_backward_train_profile_device(ctx: Context, shape: SfnnForwardShape, batch_size: int, max_active: int,
                                       stm: I32Buffer, nstm: I32Buffer, buckets: I32Buffer, weights: dict,
                                       fws: SfnnForwardWorkspace, mean_output_gradients: F32Buffer,
                                       bws: SfnnBackwardWorkspace,
                                       alpha: SfnnFactorizerAlpha = SfnnFactorizerAlpha(),
                                       zero_parameter_gradients: bool = False,
                                       qat_l1_weights: Optional[F32Buffer] = None) -> dict:
    """bulletou_cuda_cpp_sfnn_backward_train_profile_device (lib.rs:3719): the
    training backward and its stage times in ms (SFNN_BACKWARD_PROFILE_STAGES;
    blocks until the backward is done)."""
    import ctypes

    ms = (ctypes.c_float * 7)()
    ctx.lib.call("bulletou_cuda_cpp_sfnn_backward_train_profile_device",
                 *_backward_args(ctx, shape, batch_size, max_active, stm, nstm, buckets, weights, fws,
                                 mean_output_gradients, bws, alpha, qat_l1_weights),
                 int(zero_parameter_gradients), ms, 7)
    return dict(zip(SFNN_BACKWARD_PROFILE_STAGES, list(ms)))


def sfnn_build_quantized_proxy_device(ctx: Context, shape: SfnnForwardShape, weights: dict, dst: dict,
                                      alpha: SfnnFactorizerAlpha = SfnnFactorizerAlpha(),
                                      skip_ft_weights: bool = False) -> None:
    """bulletou_cuda_cpp_sfnn_build_quantized_proxy_device (lib.rs:2378, 6520):
    the engine-lattice proxy of the f32 masters `weights` into `dst` (keys
    l0w l0b l1w l1b l2w l2b l3w l3b; dst l0w has the base rows only when the
    FT is factorized)."""
    w = weights
    base = shape.factorized_base()
    vr = shape.input_size - base if base else 0
    dst_rows = base if base else shape.input_size
    has = [int(w[n] is not None) for n in ("l1fw", "l2fw", "l3fw")]
    ctx.lib.call(
        "bulletou_cuda_cpp_sfnn_build_quantized_proxy_device", ctx.as_ptr(), shape.input_size, dst_rows, vr,
        shape.ft_size, shape.l1_hidden, int(shape.l1_skip), shape.l2_size, shape.num_stacks, 1, 0, 0, 0, 0,
        _p(w["l0w"]), _p(w["l0b"]), _p(w["l1w"]), _p(w["l1b"]), _p(w["l1fw"]), _p(w["l1fb"]), has[0], None, None, 0,
        _p(w["l2w"]), _p(w["l2b"]), _p(w["l2fw"]), _p(w["l2fb"]), has[1], None, None, 0,
        _p(w["l3w"]), _p(w["l3b"]), _p(w["l3fw"]), _p(w["l3fb"]), has[2], None, None, 0,
        0, 0, 0, 0, 0, 0, alpha.ft, alpha.shared, 1.0, 1.0, 1.0, 1.0, None, None,
        *[_p(dst[k]) for k in ("l0w", "l0b", "l1w", "l1b", "l2w", "l2b", "l3w", "l3b")], int(skip_ft_weights))


@dataclass(frozen=True)
class SfnnLayerLrMultipliers:
    """The QAT switches of the runner's layer multipliers (lib.rs:6320-6370);
    the learning-rate multipliers themselves stay at their defaults here."""

    qat_l1: bool = False
    qat_ft: bool = False
    qat_l2: bool = False
    qat_l3: bool = False

    @property
    def layer_qat(self) -> bool:
        return self.qat_ft or self.qat_l2 or self.qat_l3

    @property
    def dense_qat(self) -> bool:
        return self.qat_l1 and self.qat_l2 and self.qat_l3

    def as_struct(self) -> SfnnQat:
        return SfnnQat(int(self.qat_l1), int(self.qat_ft), int(self.qat_l2), int(self.qat_l3))


class SfnnL1Qat:
    """Training-only fake-quantised L1 scratch (SfnnL1Qat, lib.rs:1946-1995)."""

    def __init__(self, ctx: Context, shape: SfnnForwardShape):
        self.weights = F32Buffer(ctx, shape.num_stacks * shape.l1_out * shape.ft_size)
        self.bias = F32Buffer(ctx, shape.num_stacks * shape.l1_out)


class SfnnLayerQatCopies:
    """Fake-quantised copies of the FT / L2 / L3 tensors a layer-QAT step swaps
    in for its forward and backward (layer_qat.rs:5-11, 832-923)."""

    def __init__(self):
        self.copies = {}
        self.checked_ft = False

    def prepare(self, ctx: Context, runner: "SfnnTrainStepRunner", lr: SfnnLayerLrMultipliers) -> dict:
        lib = ctx.lib
        base = runner.shape.factorized_base()
        vr = PIECE_INPUTS if base else 0
        swaps = {}
        for on, w_name, b_name, ft in ((lr.qat_ft, "l0w", "l0b", True), (lr.qat_l2, "l2w", "l2b", False),
                                       (lr.qat_l3, "l3w", "l3b", False)):
            if not on:
                continue
            for name, is_bias in ((w_name, False), (b_name, True)):
                src = runner.weights[name]
                dst = self.copies.get(name)
                if dst is None or dst.length != src.length:
                    dst = F32Buffer(ctx, src.length)
                    self.copies[name] = dst
                scale = 127.0 if ft else (8128.0 if is_bias else 64.0)
                lo, hi = ((-32768.0, 32767.0) if ft else ((-2147483648.0, 2147483647.0) if is_bias else (-128.0, 127.0)))
                rows = vr if (ft and not is_bias) else 0
                lib.call("bulletou_layer_qat", ctx.as_ptr(), src.as_ptr(), dst.as_ptr(), scale, lo, hi,
                         base if rows else 0, rows, runner.shape.ft_size if rows else 0, runner.alpha.ft)
                swaps[name] = dst
        if lr.qat_ft and not self.checked_ft:
            # One readback when FT QAT switches on (layer_qat.rs:968-972).
            flag = F32Buffer.from_host(ctx, np.zeros(1, np.float32))
            lib.call("bulletou_layer_qat_nonzero", ctx.as_ptr(), swaps["l0w"].as_ptr(), swaps["l0b"].as_ptr(),
                     flag.as_ptr())
            if flag.download(ctx)[0] == 0.0:
                raise CudaCppError("FT QAT rounded every effective FT weight and bias to zero (scale=127); "
                                   "pairwise FT gradients vanish")
            self.checked_ft = True
        return swaps


def factor_contribution_clip(params: RangerUpdateParams, alpha: float) -> RangerUpdateParams:
    """lib.rs:8772-8788: bounds of a shared factor refer to alpha * w."""
    r = params.radam
    if alpha == 0.0:
        return replace(params, radam=replace(r, min_weight=-FLT_MAX, max_weight=FLT_MAX))

    def scale(bound: float) -> float:
        if bound in (-FLT_MAX, FLT_MAX):
            return bound
        return float(np.float32(min(FLT_MAX, max(-FLT_MAX, float(bound) / float(alpha)))))

    return replace(params, radam=replace(r, min_weight=scale(r.min_weight), max_weight=scale(r.max_weight)))


class SfnnTrainStepUploadSlot:
    """SfnnTrainStepUploadSlot (lib.rs:6087-6186): device batch, pinned staging,
    upload-ready and compute-done events."""

    def __init__(self, ctx: Context, batch_size: int, max_active: int):
        n = batch_size * max_active
        self.stm_indices, self.nstm_indices = I32Buffer(ctx, n), I32Buffer(ctx, n)
        self.buckets = I32Buffer(ctx, batch_size)
        self.targets, self.entry_weights = F32Buffer(ctx, batch_size), F32Buffer(ctx, batch_size)
        self.pinned = (PinnedI32Buffer(ctx, n), PinnedI32Buffer(ctx, n), PinnedI32Buffer(ctx, batch_size),
                       PinnedF32Buffer(ctx, batch_size), PinnedF32Buffer(ctx, batch_size))
        self.device = (self.stm_indices, self.nstm_indices, self.buckets, self.targets, self.entry_weights)
        self.upload_ready = Event(ctx)
        self.compute_done = Event(ctx)
        self.in_use = False

    def fill(self, batch: SfnnTrainStepHostBatch) -> None:
        for dst, src in zip(self.pinned, (batch.stm_indices, batch.nstm_indices, batch.buckets, batch.targets,
                                          batch.entry_weights)):
            np.copyto(dst.host(), np.asarray(src).reshape(-1))

    def upload(self, upload_ctx: Context, batch: Optional[SfnnTrainStepHostBatch],
               pinned_source: Optional["SfnnTrainStepUploadSlot"] = None) -> int:
        lib = upload_ctx.lib
        if self.in_use:
            self.upload_ready.synchronize()
            self.compute_done.wait(upload_ctx)
        if pinned_source is None and not lib.has("bulletou_b200_i32_upload_pinned"):
            if batch is None:
                raise CudaCppError("this backend needs host batch arrays for staged uploads")
            srcs = (batch.stm_indices, batch.nstm_indices, batch.buckets, batch.targets, batch.entry_weights)
            for pin, dst, src in zip(self.pinned, self.device, srcs):
                pin.upload_to_device(upload_ctx, dst, src)
            self.upload_ready.record(upload_ctx)
            self.in_use = True
            return 4 * sum(x.length for x in self.pinned)
        src = pinned_source.pinned if pinned_source is not None else self.pinned
        if pinned_source is None:
            self.fill(batch)
        for pin, dst in zip(src, self.device):
            upload_from_pinned(upload_ctx, dst, pin)
        self.upload_ready.record(upload_ctx)
        self.in_use = True
        return sum(int(x.nbytes) if isinstance(x, np.ndarray) else 4 * x.length for x in src)


class SfnnTrainStepRunner:
    """SFNN train-step runner (lib.rs:6187-7960), default layer multipliers."""

    def __init__(self, ctx: Context, initial_weights: SfnnForwardHostWeights, batch_size: int, max_active: int,
                 factorizer_alpha: SfnnFactorizerAlpha = SfnnFactorizerAlpha(), fused: Optional[bool] = None,
                 lr_multipliers: SfnnLayerLrMultipliers = SfnnLayerLrMultipliers()):
        initial_weights.validate()
        factorizer_alpha.validate()
        if batch_size == 0 or max_active == 0:
            raise CudaCppError("SFNN train-step batch_size and max_active must be greater than zero")
        self.ctx = ctx
        self.lib = ctx.lib
        self.shape = initial_weights.shape
        self.alpha = factorizer_alpha
        self.batch_size, self.max_active = batch_size, max_active
        self.fused = self.lib.has("bulletou_b200_sfnn_train_step_device") if fused is None else bool(fused)
        arrays = initial_weights.arrays()
        self.present = {n: arrays[n] is not None for n in SFNN_WEIGHT_NAMES}
        self.weights = {n: (None if a is None else F32Buffer.from_host(ctx, a)) for n, a in arrays.items()}
        self.optimizer_states = {n: (None if a is None else RangerParamState(ctx, a)) for n, a in arrays.items()}
        n = batch_size * max_active
        self.stm_indices, self.nstm_indices = I32Buffer(ctx, n), I32Buffer(ctx, n)
        self.buckets = I32Buffer(ctx, batch_size)
        self.targets, self.entry_weights = F32Buffer(ctx, batch_size), F32Buffer(ctx, batch_size)
        self.loss_workspace = ScalarLossWorkspace(ctx, batch_size)
        self.forward_workspace = None
        self.backward_workspace = None
        self.output = F32Buffer(ctx, batch_size) if self.fused else None
        if not self.fused:
            self._reference_workspaces(ctx)
        self._handles_cache = None
        self._slots = None
        self._next_slot = 0
        self.lr_multipliers = lr_multipliers
        self.qat_l1 = None
        self.layer_qat = SfnnLayerQatCopies()

    def _reference_workspaces(self, ctx: Context) -> None:
        self.forward_workspace = SfnnForwardWorkspace(ctx, self.shape, self.batch_size)
        self.output = self.forward_workspace.output
        self.backward_workspace = SfnnBackwardWorkspace(ctx, self.shape, self.batch_size, self.present)

    # -- batch upload ------------------------------------------------------
    def upload_batch(self, batch: SfnnTrainStepHostBatch, ctx: Optional[Context] = None) -> None:
        batch.validate()
        if batch.batch_size != self.batch_size or batch.max_active != self.max_active:
            raise CudaCppError(
                f"SFNN train-step batch layout mismatch: got batch_size={batch.batch_size} "
                f"max_active={batch.max_active}, expected batch_size={self.batch_size} max_active={self.max_active}")
        c = ctx or self.ctx
        self.stm_indices.upload(batch.stm_indices, c)
        self.nstm_indices.upload(batch.nstm_indices, c)
        self.buckets.upload(batch.buckets, c)
        self.targets.upload(batch.targets, c)
        self.entry_weights.upload(batch.entry_weights, c)

    # -- steps -------------------------------------------------------------
    def step(self, ctx: Context, params: RangerUpdateParams, loss_kind: ScalarLossKind, output_inv_scale: float,
             batch: SfnnTrainStepHostBatch) -> ScalarLossReadback:
        self.step_no_readback(ctx, params, loss_kind, output_inv_scale, batch)
        return self.read_loss(ctx)

    def step_no_readback(self, ctx, params, loss_kind, output_inv_scale, batch) -> None:
        self.step_no_readback_with_loss_finalize(ctx, params, loss_kind, output_inv_scale, batch, True)

    def step_no_readback_with_loss_finalize(self, ctx, params, loss_kind, output_inv_scale, batch,
                                            finalize_loss: bool) -> None:
        self.upload_batch(batch, ctx)
        self.step_device(ctx, params, loss_kind, output_inv_scale, finalize_loss)

    def _handles(self):
        if self._handles_cache is None:
            arr = ctypes.c_void_p * 14

            def pack(get):
                return arr(*[(None if self.weights[n] is None else get(n).as_ptr().value) for n in SFNN_WEIGHT_NAMES])

            self._handles_cache = (pack(lambda n: self.weights[n]),
                                   pack(lambda n: self.optimizer_states[n].momentum),
                                   pack(lambda n: self.optimizer_states[n].velocity),
                                   pack(lambda n: self.optimizer_states[n].slow_params))
        return self._handles_cache

    def step_device(self, ctx: Context, params: RangerUpdateParams, loss_kind: ScalarLossKind,
                    output_inv_scale: float, finalize_loss: bool = True) -> None:
        """One step on the batch already resident in this runner's device buffers."""
        # With default layer multipliers the SFNN update applies no norm loss
        # (clip_params, lib.rs:6416-6420).
        params = replace(params, norm_loss_strength=0.0, norm_loss_before=False)
        lw = self.loss_workspace
        lr = self.lr_multipliers
        if (lr.qat_l2 and self.present["l2fw"]) or (lr.qat_l3 and self.present["l3fw"]):
            raise CudaCppError("Layer QAT does not support legacy L2/L3 factorizer tensors; fold them first")
        if self.fused and params.sgd_momentum is None:
            sh = self.shape
            shape = SfnnShape(sh.input_size, sh.ft_size, sh.l1_hidden, int(sh.l1_skip), sh.l2_size, sh.num_stacks,
                              self.alpha.ft, self.alpha.shared)
            spec = loss_kind.spec(output_inv_scale, finalize_loss)
            step = params.ffi_step()
            qat = lr.as_struct()
            w, m, v, s = self._handles()
            self.lib.call("bulletou_b200_sfnn_train_step_device", ctx.as_ptr(), ctypes.byref(shape), self.batch_size,
                          self.max_active, self.stm_indices.as_ptr(), self.nstm_indices.as_ptr(),
                          self.buckets.as_ptr(), self.targets.as_ptr(), self.entry_weights.as_ptr(),
                          ctypes.byref(spec), ctypes.byref(step), w, m, v, s, self.output.as_ptr(),
                          lw.per_sample.as_ptr(), lw.mean_output_gradients.as_ptr(), lw.weighted_sum.as_ptr(),
                          lw.mean.as_ptr(), ctypes.byref(qat))
            return
        if self.forward_workspace is None:
            self._reference_workspaces(ctx)
        fws, bws = self.forward_workspace, self.backward_workspace
        # L1 QAT scratch (prepare_l1_qat, lib.rs:6525-6550); every step follows
        # an update, so the fake-quantised L1 is rebuilt each step.
        if lr.qat_l1 and self.qat_l1 is None:
            self.qat_l1 = SfnnL1Qat(ctx, self.shape)
        qat_l1 = self.qat_l1 if lr.qat_l1 else None
        # Layer QAT (layer_qat::step, layer_qat.rs:925-1004): fake-quantised
        # copies stand in for the masters through forward and backward.
        swaps = self.layer_qat.prepare(ctx, self, lr) if lr.layer_qat else {}
        used = dict(self.weights)
        used.update(swaps)
        dense = lr.dense_qat
        if dense:
            self.lib.call("bulletou_dense_qat_begin", ctx.as_ptr(), self.weights["l2b"].as_ptr(),
                          self.weights["l3b"].as_ptr(), self.batch_size, self.shape.l1_out, self.shape.l2_size,
                          self.shape.num_stacks, int(lr.qat_ft))
        try:
            fold = bws.params["l0w"] if self.shape.factorized_base() else None
            sfnn_forward_device(ctx, self.shape, self.batch_size, self.max_active, self.stm_indices,
                                self.nstm_indices, self.buckets, used, fws, self.alpha, fold, qat_l1, 1)
            if fold is not None:
                fold.fill(0.0, ctx)  # lib.rs:2078-2084: discard the folded weights before backward adds
            scalar_loss_device(ctx, loss_kind, output_inv_scale, self.batch_size, fws.output, self.targets,
                               self.entry_weights, lw, finalize_loss)
            sfnn_backward_train_device(ctx, self.shape, self.batch_size, self.max_active, self.stm_indices,
                                       self.nstm_indices, self.buckets, used, fws, lw.mean_output_gradients, bws,
                                       self.alpha, False, self.entry_weights,
                                       None if qat_l1 is None else qat_l1.weights)
        finally:
            if dense:
                self.lib.call("bulletou_dense_qat_end", ctx.as_ptr())
        for n in SFNN_WEIGHT_NAMES:
            if self.weights[n] is None:
                continue
            p = factor_contribution_clip(params, self.alpha.shared) if n in ("l1fw", "l1fb") else params
            st = self.optimizer_states[n]
            ranger_update_device(ctx, p, RangerDeviceState(bws.params[n], self.weights[n], st.momentum, st.velocity,
                                                           st.slow_params))

    # -- pipelined steps (lib.rs:7535-7720) -------------------------------
    def upload_slots(self, count: int = 2) -> list:
        if self._slots is None or len(self._slots) != count:
            self._slots = [SfnnTrainStepUploadSlot(self.ctx, self.batch_size, self.max_active) for _ in range(count)]
            self._next_slot = 0
        return self._slots

    def upload_next(self, upload_ctx: Context, batch: Optional[SfnnTrainStepHostBatch] = None,
                    pinned_source: Optional[SfnnTrainStepUploadSlot] = None) -> int:
        """The upload half of step_pipelined_no_readback_with_loss_finalize on
        its own: the next step's batch into the next slot on `upload_ctx`, so
        a trainer can issue it while the current step still runs (for example
        before reading the current step's loss).  The step that consumes it is
        step_uploaded_no_readback_with_loss_finalize.  Returns H2D bytes."""
        slots = self.upload_slots()
        slot = slots[self._next_slot]
        self._next_slot = (self._next_slot + 1) % len(slots)
        nbytes = slot.upload(upload_ctx, batch, pinned_source)
        if not hasattr(self, "_uploaded"):
            self._uploaded = []
        self._uploaded.append(slot)
        return nbytes

    def step_uploaded_no_readback_with_loss_finalize(self, ctx: Context, params: RangerUpdateParams,
                                                     loss_kind: ScalarLossKind, output_inv_scale: float,
                                                     finalize_loss: bool = True) -> None:
        """Runs the step on the oldest batch upload_next issued: waits for its
        upload on `ctx`, steps, and releases the slot for a later upload."""
        if not getattr(self, "_uploaded", None):
            raise CudaCppError("no uploaded batch: call upload_next first")
        slot = self._uploaded.pop(0)
        slot.upload_ready.wait(ctx)
        self.stm_indices, self.nstm_indices, self.buckets = slot.stm_indices, slot.nstm_indices, slot.buckets
        self.targets, self.entry_weights = slot.targets, slot.entry_weights
        self.step_device(ctx, params, loss_kind, output_inv_scale, finalize_loss)
        slot.compute_done.record(ctx)

    def step_pipelined_no_readback_with_loss_finalize(self, ctx: Context, upload_ctx: Context,
                                                      params: RangerUpdateParams, loss_kind: ScalarLossKind,
                                                      output_inv_scale: float,
                                                      batch: Optional[SfnnTrainStepHostBatch],
                                                      finalize_loss: bool = True,
                                                      pinned_source: Optional[SfnnTrainStepUploadSlot] = None,
                                                      loss_out: Optional[PinnedF32Buffer] = None) -> int:
        """Upload on `upload_ctx` into the next slot, hand off with an event, run
        the step on `ctx`, then (optionally) an async D2H of the mean loss into
        `loss_out`.  Returns H2D bytes."""
        slots = self.upload_slots()
        slot = slots[self._next_slot]
        self._next_slot = (self._next_slot + 1) % len(slots)
        nbytes = slot.upload(upload_ctx, batch, pinned_source)
        slot.upload_ready.wait(ctx)
        self.stm_indices, self.nstm_indices, self.buckets = slot.stm_indices, slot.nstm_indices, slot.buckets
        self.targets, self.entry_weights = slot.targets, slot.entry_weights
        self.step_device(ctx, params, loss_kind, output_inv_scale, finalize_loss)
        if loss_out is not None:
            if self.lib.has("bulletou_b200_f32_download_pinned"):
                self.lib.call("bulletou_b200_f32_download_pinned", ctx.as_ptr(), loss_out.as_ptr(),
                              self.loss_workspace.mean.as_ptr(), 1)
            else:
                loss_out.host()[0] = self.loss_workspace.mean.download(ctx)[0]
        slot.compute_done.record(ctx)
        return nbytes

    # -- steps on PackedSfenValue records (device-side batch producer) -----
    def _check_producer(self, producer) -> None:
        cfg = producer.config
        if cfg.feature_set != "halfka_hm2" or cfg.active != self.max_active or producer.batch_size != self.batch_size:
            raise CudaCppError(
                f"teacher producer ({cfg.feature_set}, batch {producer.batch_size}, max_active {cfg.active}) does "
                f"not match the SFNN runner (batch {self.batch_size}, max_active {self.max_active})")
        base = self.shape.factorized_base() or self.shape.input_size
        if base != cfg.num_inputs:
            raise CudaCppError(f"HalfKA_hm2 records feed {cfg.num_inputs} inputs, the runner has {base}")
        if cfg.layerstack_bucket.num_stacks != self.shape.num_stacks:
            raise CudaCppError(f"LayerStack bucket kind gives {cfg.layerstack_bucket.num_stacks} stacks, "
                               f"the runner has {self.shape.num_stacks}")

    def step_from_records(self, ctx: Context, params: RangerUpdateParams, loss_kind: ScalarLossKind,
                          output_inv_scale: float, producer, records, finalize_loss: bool = True) -> None:
        """Decode PackedSfenValue records into this runner's batch on the
        device (bulletou_b200_teacher_prepare_device), then step."""
        from .teacher import TeacherBatch

        self._check_producer(producer)
        view = TeacherBatch.wrap(self.stm_indices, self.nstm_indices, self.buckets, self.targets,
                                 self.entry_weights, self.batch_size, self.max_active)
        producer.prepare(ctx, records, view)
        self.step_device(ctx, params, loss_kind, output_inv_scale, finalize_loss)

    def record_slots(self, producer, count: int = 2) -> list:
        from .teacher import TeacherUploadSlot

        if getattr(self, "_record_slots", None) is None or len(self._record_slots) != count:
            self._check_producer(producer)
            self._record_slots = [TeacherUploadSlot(self.ctx, producer) for _ in range(count)]
            self._next_record_slot = 0
        return self._record_slots

    def step_pipelined_records(self, ctx: Context, upload_ctx: Context, producer, params: RangerUpdateParams,
                               loss_kind: ScalarLossKind, output_inv_scale: float, records=None,
                               finalize_loss: bool = True, pinned_source=None,
                               loss_out: Optional[PinnedF32Buffer] = None) -> int:
        """Pipelined step fed by PackedSfenValue records: the records (40 bytes
        a position) go H2D on `upload_ctx` and are decoded there into the next
        slot's batch while the previous step runs on `ctx`; an event hands the
        batch over.  Optionally copies the mean loss D2H into `loss_out`.
        Returns the H2D bytes."""
        slots = self.record_slots(producer)
        slot = slots[self._next_record_slot]
        self._next_record_slot = (self._next_record_slot + 1) % len(slots)
        nbytes = slot.upload(upload_ctx, producer, records, pinned_source)
        slot.upload_ready.wait(ctx)
        b = slot.batch
        self.stm_indices, self.nstm_indices, self.buckets = b.stm_indices, b.nstm_indices, b.buckets
        self.targets, self.entry_weights = b.targets, b.entry_weights
        self.step_device(ctx, params, loss_kind, output_inv_scale, finalize_loss)
        if loss_out is not None:
            self.lib.call("bulletou_b200_f32_download_pinned", ctx.as_ptr(), loss_out.as_ptr(),
                          self.loss_workspace.mean.as_ptr(), 1)
        slot.compute_done.record(ctx)
        return nbytes

    # -- readback ----------------------------------------------------------
    def read_loss(self, ctx: Optional[Context] = None) -> ScalarLossReadback:
        return self.loss_workspace.download(ctx)

    def read_output(self, ctx: Optional[Context] = None) -> np.ndarray:
        return self.output.download(ctx)

    def read_weights(self, ctx: Optional[Context] = None) -> dict:
        return {n: w.download(ctx) for n, w in self.weights.items() if w is not None}

    def read_optimizer_states(self, ctx: Optional[Context] = None) -> dict:
        return {n: s.download(ctx) for n, s in self.optimizer_states.items() if s is not None}


# ------------------------------------------------------------------ quantised SFNN
SFNN_QUANT_NAMES = ("l0w", "l0b", "l1w", "l1b", "l2w", "l2b", "l3w", "l3b")
_QUANT_DTYPES = {"l0w": np.int16, "l0b": np.int16, "l1w": np.int8, "l1b": np.int32, "l2w": np.int8,
                 "l2b": np.int32, "l3w": np.int8, "l3b": np.int32}


def _pad32(n: int) -> int:
    return (n + 31) // 32 * 32


@dataclass(frozen=True)
class QuantizedRounding:
    """The integer evaluator's rounding switches (examples/bulletou.rs:1254-1340
    defaults: FV_SCALE 24, ft shift 7, every right shift floored)."""

    ft_shift: int = 7
    ft_round: bool = False
    crelu_round: bool = False
    sqr_clipped_relu_round: bool = False
    final_div_round: bool = False
    fv_scale: int = 24

    def as_struct(self) -> QuantRounding:
        return QuantRounding(int(self.ft_shift), int(self.ft_round), int(self.crelu_round),
                             int(self.sqr_clipped_relu_round), int(self.final_div_round), int(self.fv_scale))


class QuantizedSfnnDeviceWeights:
    """Engine-format quantised SFNN weights on the device
    (QuantizedSfnnWeights, examples/bulletou.rs:7355-7377): FT i16 rows with the
    factorizer folded, dense i8 rows padded to 32 inputs, i32 biases.  Each
    tensor lives in an I32 buffer holding the packed narrow integers."""

    def __init__(self, ctx: Context, shape: SfnnForwardShape):
        self.shape = shape
        base = shape.factorized_base()
        self.rows = base if base else shape.input_size
        S, O, L2 = shape.num_stacks, shape.l1_out, shape.l2_size
        self.counts = {"l0w": self.rows * shape.ft_size, "l0b": shape.ft_size,
                       "l1w": S * O * _pad32(shape.ft_size), "l1b": S * O,
                       "l2w": S * L2 * _pad32(shape.l2_in), "l2b": S * L2, "l3w": S * _pad32(L2), "l3b": S}
        self.buffers = {}
        for n in SFNN_QUANT_NAMES:
            nbytes = self.counts[n] * np.dtype(_QUANT_DTYPES[n]).itemsize
            self.buffers[n] = I32Buffer(ctx, (nbytes + 3) // 4)

    def _array(self):
        arr = (ctypes.c_void_p * len(SFNN_QUANT_NAMES))()
        for k, n in enumerate(SFNN_QUANT_NAMES):
            arr[k] = self.buffers[n].as_ptr().value
        return arr

    def download(self, ctx: Optional[Context] = None) -> dict:
        out = {}
        for n in SFNN_QUANT_NAMES:
            words = self.buffers[n].download(ctx)
            out[n] = words.view(_QUANT_DTYPES[n])[: self.counts[n]].copy()
        return out

    def upload(self, arrays: dict, ctx: Optional[Context] = None) -> None:
        for n in SFNN_QUANT_NAMES:
            a = np.ascontiguousarray(arrays[n], dtype=_QUANT_DTYPES[n]).reshape(-1)
            if a.size != self.counts[n]:
                raise ValueError(f"quantised {n}: expected {self.counts[n]} values, got {a.size}")
            raw = np.zeros(self.buffers[n].length * 4, np.uint8)
            raw[: a.nbytes] = a.view(np.uint8)
            self.buffers[n].upload(raw.view(np.int32), ctx)


def _shape_struct(shape: SfnnForwardShape, alpha: SfnnFactorizerAlpha) -> SfnnShape:
    return SfnnShape(shape.input_size, shape.ft_size, shape.l1_hidden, int(shape.l1_skip), shape.l2_size,
                     shape.num_stacks, alpha.ft, alpha.shared)


def sfnn_quantize_device(ctx: Context, shape: SfnnForwardShape, weights: dict, out: QuantizedSfnnDeviceWeights,
                         alpha: SfnnFactorizerAlpha = SfnnFactorizerAlpha()) -> None:
    """Export quantisation on the device (bulletou_b200_sfnn_quantize_device;
    quantized_sfnn_weights_from_cuda_cpp_readback, examples/bulletou.rs:10050-10300)."""
    params = (ctypes.c_void_p * 14)()
    for k, n in enumerate(SFNN_WEIGHT_NAMES):
        params[k] = None if weights.get(n) is None else weights[n].as_ptr().value
    sh = _shape_struct(shape, alpha)
    ctx.lib.call("bulletou_b200_sfnn_quantize_device", ctx.as_ptr(), ctypes.byref(sh), params, out._array())


class SfnnIntegerForwardWorkspace:
    """Outputs of the integer forward: raw i32 evaluation, i32 L1 sums, the
    engine score raw / FV_SCALE and the error counter."""

    def __init__(self, ctx: Context, shape: SfnnForwardShape, batch_size: int):
        self.raw = I32Buffer(ctx, batch_size)
        self.l1 = I32Buffer(ctx, batch_size * shape.l1_out)
        self.score = I32Buffer(ctx, batch_size)
        self.errors = I32Buffer(ctx, 1)

    def download(self, ctx: Optional[Context] = None) -> dict:
        return {"raw": self.raw.download(ctx), "l1": self.l1.download(ctx), "score": self.score.download(ctx),
                "errors": int(self.errors.download(ctx)[0])}


def sfnn_integer_forward_device(ctx: Context, shape: SfnnForwardShape, batch_size: int, max_active: int,
                                stm: I32Buffer, nstm: I32Buffer, buckets: I32Buffer,
                                weights: QuantizedSfnnDeviceWeights, ws: SfnnIntegerForwardWorkspace,
                                rounding: QuantizedRounding = QuantizedRounding()) -> None:
    """Integer forward of a batch (bulletou_b200_sfnn_integer_forward_device;
    quantized_sfnn_forward_sample + quantized_final_division,
    examples/bulletou.rs:8001-8163)."""
    sh = _shape_struct(shape, SfnnFactorizerAlpha())
    r = rounding.as_struct()
    ctx.lib.call("bulletou_b200_sfnn_integer_forward_device", ctx.as_ptr(), ctypes.byref(sh), batch_size,
                 max_active, stm.as_ptr(), nstm.as_ptr(), buckets.as_ptr(), weights._array(), ctypes.byref(r),
                 ws.l1.as_ptr(), ws.raw.as_ptr(), ws.score.as_ptr(), ws.errors.as_ptr())
