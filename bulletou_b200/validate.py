"""Held-out validation on the device: forward over decoded teacher records and
the reference's accuracy / loss report.

Mirrors crates/bulletou_lib/src/validate.rs: ``AccuracyReport`` (:54-100),
``ValidationLossKind`` (:134-145) and compute_sign_accuracy_with_loss_masked
(:381-470), which the reference evaluates on the host over downloaded model
outputs; here ``bulletou_b200_validation_metrics_device`` reduces them next to
the outputs and only the ten-int report comes back.  ``SfnnForwardWorkspace``
statistics (``validation_stats``, lib.rs:1955-1970) use the reference entry
``bulletou_cuda_cpp_sfnn_validation_stats``.
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass, field
from typing import Optional

import numpy as np

from ._lib import CudaCppError, ValidationConfig
from .cuda_cpp import Context, F32Buffer, I32Buffer
from .teacher import WinRateModelTargetParams, win_rate_model_score_table

_KINDS = {"sigmoid_pow": 0, "win_rate_model": 1, "bce_with_logits": 2}


@dataclass(frozen=True)
class ValidationLossKind:
    """ValidationLossKind: SigmoidPow{pow_exp}, WinRateModel{pow_exp,
    nnue2score, in_offset, in_scaling, target}, BceWithLogits{nnue2score,
    in_scaling, target}."""

    kind: str = "sigmoid_pow"
    pow_exp: float = 2.0
    nnue2score: float = 600.0
    in_offset: float = 270.0
    in_scaling: float = 380.0
    target: WinRateModelTargetParams = field(default_factory=WinRateModelTargetParams)

    @staticmethod
    def sigmoid_pow(pow_exp: float = 2.0) -> "ValidationLossKind":
        return ValidationLossKind("sigmoid_pow", pow_exp=pow_exp)

    @staticmethod
    def win_rate_model(pow_exp: float, nnue2score: float, in_offset: float, in_scaling: float,
                       target: WinRateModelTargetParams = WinRateModelTargetParams()) -> "ValidationLossKind":
        return ValidationLossKind("win_rate_model", pow_exp, nnue2score, in_offset, in_scaling, target)

    @staticmethod
    def bce_with_logits(nnue2score: float, in_scaling: float,
                        target: WinRateModelTargetParams = WinRateModelTargetParams()) -> "ValidationLossKind":
        return ValidationLossKind("bce_with_logits", nnue2score=nnue2score, in_scaling=in_scaling, target=target)


@dataclass
class AccuracyReport:
    compared: int = 0
    sign_matches: int = 0
    predicted_nonnegative: int = 0
    predicted_negative: int = 0
    predicted_zero: int = 0
    drawn_games: int = 0
    filtered_by_score_cap: int = 0
    loss_sampled: int = 0
    test_loss: Optional[float] = None

    def accuracy(self) -> float:
        return float("nan") if self.compared == 0 else float(np.float32(self.sign_matches) / np.float32(self.compared))


class ValidationMetrics:
    """Device report buffer and the target table of one loss kind."""

    def __init__(self, ctx: Context, loss_kind: ValidationLossKind = ValidationLossKind()):
        if loss_kind.kind not in _KINDS:
            raise CudaCppError(f"unknown validation loss kind {loss_kind.kind!r}")
        self.ctx = ctx
        self.loss_kind = loss_kind
        self.report = I32Buffer(ctx, 10)
        self.table = (None if loss_kind.kind == "sigmoid_pow"
                      else F32Buffer.from_host(ctx, win_rate_model_score_table(loss_kind.target)))

    def compute(self, ctx: Context, outputs: F32Buffer, records: I32Buffer, n: int, *, lambda_: float = 1.0,
                eval_scale: float = 600.0, model_output_scale: float = 1.0, score_drop_abs: Optional[int] = None,
                have_results: bool = True) -> AccuracyReport:
        if not (math.isfinite(lambda_) and 0.0 <= lambda_ <= 1.0):
            raise CudaCppError(f"lambda must be finite and in [0, 1] (got {lambda_})")
        k = self.loss_kind
        cfg = ValidationConfig(int(have_results), -1 if score_drop_abs is None else int(score_drop_abs),
                               _KINDS[k.kind], float(lambda_), float(eval_scale), float(model_output_scale),
                               float(k.pow_exp), float(k.nnue2score), float(k.in_offset), float(k.in_scaling))
        ctx.lib.call("bulletou_b200_validation_metrics_device", ctx.as_ptr(), ctypes.byref(cfg), outputs.as_ptr(),
                     records.as_ptr(), int(n), None if self.table is None else self.table.as_ptr(),
                     self.report.as_ptr())
        raw = self.report.download(ctx)
        rep = AccuracyReport(*[int(v) for v in raw[:8]])
        loss_sum = float(raw[8:10].view(np.float64)[0])
        if have_results and rep.loss_sampled > 0:
            rep.test_loss = float(np.float32(loss_sum / rep.loss_sampled))
        return rep


def sfnn_validation_stats(ctx: Context, ws, partials: F32Buffer) -> list:
    """SfnnForwardWorkspace::validation_stats (lib.rs:1955-1970): FT / L1 normal
    / L1 square / L2 upper counts and the summed squared output, each the f64
    sum of 256 CTA partials."""
    if partials.length != 1280:
        raise CudaCppError(f"validation stats partials length mismatch: expected 1280, got {partials.length}")
    sh, batch = ws.layout
    ctx.lib.call("bulletou_cuda_cpp_sfnn_validation_stats", ctx.as_ptr(), ws.stm_l0.as_ptr(), ws.nstm_l0.as_ptr(),
                 ws.l2_input.as_ptr(), ws.l2.as_ptr(), ws.output.as_ptr(), partials.as_ptr(), batch,
                 sh.ft_size, sh.l1_hidden, sh.l2_size)
    host = partials.download(ctx).astype(np.float64)
    return [float(host[i * 256:(i + 1) * 256].sum()) for i in range(5)]
