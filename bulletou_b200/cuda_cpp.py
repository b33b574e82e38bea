"""Python mirror of the reference's cuda-cpp crate API (crates/cuda_cpp/src/lib.rs).

Same type names, argument meaning and error behaviour as the Rust wrapper, so
code and tests written against the reference read the same here:
``Context``, ``F32Buffer``, ``I32Buffer``, ``Event``, ``GraphExec``,
``NnueForwardShape``, ``RAdamUpdateParams`` (with ``step_scale``),
``RangerUpdateParams``, ``ScalarLossKind``, ``NnueTrainStepRunner``,
``KpptTableTrainStepRunner``, ``ranger_update_device`` ...

Every call goes through the C ABI of a loaded backend library: the product
(libbulletou_b200.so, default) or, for parity tests and the reference timing
arm, the reference backend built from its sources.  A runner bound to the
product uses the fused single-call train step; bound to the reference it
issues the reference runner's exact call sequence (lib.rs:5748-5799).
"""
from __future__ import annotations

import ctypes
import ctypes.util
from dataclasses import dataclass, field, replace
from typing import Optional, Sequence

import numpy as np

from ._lib import CudaCppError, Library, LossSpec, RangerStep, library

FLT_MAX = float(np.finfo(np.float32).max)
_f32 = np.float32

# f32 powf from the C math library: Rust's f32::powf (used by the reference's
# step-scale math) lowers to it, while numpy's float32 power may use its own
# vectorised approximation and differ in the last bit.
_libm = ctypes.CDLL(ctypes.util.find_library("m") or "libm.so.6")
_libm.powf.argtypes = [ctypes.c_float, ctypes.c_float]
_libm.powf.restype = ctypes.c_float


def _powf(x, y) -> np.float32:
    return _f32(_libm.powf(float(x), float(y)))


def _ptr(a: np.ndarray) -> ctypes.c_void_p:
    return ctypes.c_void_p(a.ctypes.data)


# ---------------------------------------------------------------------------
# handles
# ---------------------------------------------------------------------------
class Context:
    """One device context: a CUDA stream plus context-owned scratch (lib.rs:50-120)."""

    def __init__(self, device: int = 0, lib: Optional[Library] = None, stream: Optional[int] = None):
        self.lib = lib or library()
        self.device = device
        h = ctypes.c_void_p()
        if stream is None:
            self.lib.call("bulletou_cuda_cpp_context_create", device, ctypes.byref(h))
        else:
            self.lib.call("bulletou_b200_context_create_on_stream", device, ctypes.c_void_p(stream), ctypes.byref(h))
        self._h = h

    new = classmethod(lambda cls, device=0, lib=None: cls(device, lib))

    def as_ptr(self):
        return self._h

    def synchronize(self) -> None:
        self.lib.call("bulletou_cuda_cpp_context_synchronize", self._h)

    def close(self) -> None:
        if getattr(self, "_h", None) and self._h.value:
            self.lib.call("bulletou_cuda_cpp_context_destroy", self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


class _DeviceBuffer:
    _kind = "f32"
    _dtype = np.float32

    def __init__(self, ctx: Context, length: int):
        self.ctx = ctx
        self.lib = ctx.lib
        self.length = int(length)
        h = ctypes.c_void_p()
        self.lib.call(f"bulletou_cuda_cpp_{self._kind}_buffer_create", ctx.as_ptr(), self.length, ctypes.byref(h))
        self._h = h

    @classmethod
    def new(cls, ctx: Context, length: int):
        return cls(ctx, length)

    @classmethod
    def from_host(cls, ctx: Context, data):
        a = np.ascontiguousarray(data, dtype=cls._dtype).reshape(-1)
        b = cls(ctx, a.size)
        b.upload(a)
        return b

    def __len__(self):
        return self.length

    def as_ptr(self):
        return self._h

    def upload(self, data, ctx: Optional[Context] = None) -> None:
        a = np.ascontiguousarray(data, dtype=self._dtype).reshape(-1)
        if a.size != self.length:
            raise CudaCppError(f"{self._kind} buffer upload length mismatch: expected {self.length}, got {a.size}")
        c = ctx or self.ctx
        self.lib.call(f"bulletou_cuda_cpp_{self._kind}_upload", c.as_ptr(), self._h, _ptr(a), a.size)
        # pageable uploads are synchronous w.r.t. the host buffer only after the copy; keep a ref until sync
        self._keep = a

    def download(self, ctx: Optional[Context] = None) -> np.ndarray:
        out = np.empty(self.length, dtype=self._dtype)
        c = ctx or self.ctx
        self.lib.call(f"bulletou_cuda_cpp_{self._kind}_download", c.as_ptr(), self._h, _ptr(out), self.length)
        return out

    def device_ptr(self) -> int:
        p = ctypes.c_void_p()
        self.lib.call(f"bulletou_b200_{self._kind}_buffer_ptr", self._h, ctypes.byref(p))
        return p.value or 0

    @property
    def __cuda_array_interface__(self):
        return {"shape": (self.length,), "typestr": "<f4" if self._kind == "f32" else "<i4",
                "data": (self.device_ptr(), False), "version": 3, "strides": None}

    def close(self) -> None:
        if getattr(self, "_h", None) and self._h.value:
            self.lib.call(f"bulletou_cuda_cpp_{self._kind}_buffer_destroy", self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class F32Buffer(_DeviceBuffer):
    """Device float buffer (lib.rs:122-300)."""

    _kind = "f32"
    _dtype = np.float32

    def fill(self, value: float, ctx: Optional[Context] = None) -> None:
        c = ctx or self.ctx
        self.lib.call("bulletou_cuda_cpp_f32_fill", c.as_ptr(), self._h, float(value), self.length)

    def copy_from(self, src: "F32Buffer", ctx: Optional[Context] = None) -> None:
        c = ctx or self.ctx
        self.lib.call("bulletou_cuda_cpp_f32_copy_device", c.as_ptr(), self._h, src._h, self.length)

    def view(self, offset: int, length: int) -> "F32BufferView":
        return F32BufferView(self, offset, length)


class F32BufferView(F32Buffer):
    """Non-owning slice of an F32Buffer (product library only)."""

    def __init__(self, parent: F32Buffer, offset: int, length: int):  # noqa: D401
        self.ctx = parent.ctx
        self.lib = parent.lib
        self.length = int(length)
        self._parent = parent
        h = ctypes.c_void_p()
        self.lib.call("bulletou_b200_f32_buffer_view", parent.as_ptr(), int(offset), self.length, ctypes.byref(h))
        self._h = h


class I32Buffer(_DeviceBuffer):
    """Device int32 buffer (sparse feature ids)."""

    _kind = "i32"
    _dtype = np.int32


class _PinnedBuffer:
    _kind = "f32"
    _dtype = np.float32

    def __init__(self, ctx: Context, length: int):
        self.ctx = ctx
        self.lib = ctx.lib
        self.length = int(length)
        h = ctypes.c_void_p()
        self.lib.call(f"bulletou_cuda_cpp_pinned_{self._kind}_buffer_create", ctx.as_ptr(), self.length, ctypes.byref(h))
        self._h = h
        self._host = None

    def as_ptr(self):
        return self._h

    def host(self) -> np.ndarray:
        """numpy view of the pinned host memory (product library only)."""
        if self._host is None:
            p = ctypes.c_void_p()
            self.lib.call(f"bulletou_b200_pinned_{self._kind}_ptr", self._h, ctypes.byref(p))
            ct = ctypes.c_float if self._kind == "f32" else ctypes.c_int32
            arr = (ct * self.length).from_address(p.value)
            self._host = np.ctypeslib.as_array(arr)
        return self._host

    def close(self) -> None:
        if getattr(self, "_h", None) and self._h.value:
            self._host = None
            self.lib.call(f"bulletou_cuda_cpp_pinned_{self._kind}_buffer_destroy", self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class PinnedF32Buffer(_PinnedBuffer):
    _kind = "f32"
    _dtype = np.float32

    def upload_to_device(self, ctx: Context, dst: F32Buffer, data) -> None:
        a = np.ascontiguousarray(data, dtype=np.float32).reshape(-1)
        self.lib.call("bulletou_cuda_cpp_f32_upload_staged", ctx.as_ptr(), dst.as_ptr(), self._h, _ptr(a), a.size)


class PinnedI32Buffer(_PinnedBuffer):
    _kind = "i32"
    _dtype = np.int32

    def upload_to_device(self, ctx: Context, dst: I32Buffer, data) -> None:
        a = np.ascontiguousarray(data, dtype=np.int32).reshape(-1)
        self.lib.call("bulletou_cuda_cpp_i32_upload_staged", ctx.as_ptr(), dst.as_ptr(), self._h, _ptr(a), a.size)


class Event:
    """CUDA event on a context (lib.rs:300-380)."""

    def __init__(self, ctx: Context):
        self.lib = ctx.lib
        h = ctypes.c_void_p()
        self.lib.call("bulletou_cuda_cpp_event_create", ctx.as_ptr(), ctypes.byref(h))
        self._h = h

    def record(self, ctx: Context) -> None:
        self.lib.call("bulletou_cuda_cpp_event_record", ctx.as_ptr(), self._h)

    def wait(self, ctx: Context) -> None:
        self.lib.call("bulletou_cuda_cpp_event_wait", ctx.as_ptr(), self._h)

    def synchronize(self) -> None:
        self.lib.call("bulletou_cuda_cpp_event_synchronize", self._h)

    def elapsed_ms_since(self, start: "Event") -> float:
        out = ctypes.c_float()
        self.lib.call("bulletou_cuda_cpp_event_elapsed_ms", start._h, self._h, ctypes.byref(out))
        return out.value

    def close(self):
        if getattr(self, "_h", None) and self._h.value:
            self.lib.call("bulletou_cuda_cpp_event_destroy", self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class GraphExec:
    """Captured CUDA graph (lib.rs:380-470): begin_capture / end_capture / launch."""

    def __init__(self, lib: Library, handle):
        self.lib = lib
        self._h = handle

    @staticmethod
    def begin_capture(ctx: Context) -> None:
        ctx.lib.call("bulletou_cuda_cpp_graph_begin_capture", ctx.as_ptr())

    @classmethod
    def end_capture(cls, ctx: Context) -> "GraphExec":
        h = ctypes.c_void_p()
        ctx.lib.call("bulletou_cuda_cpp_graph_end_capture", ctx.as_ptr(), ctypes.byref(h))
        return cls(ctx.lib, h)

    def launch(self, ctx: Context) -> None:
        self.lib.call("bulletou_cuda_cpp_graph_launch", ctx.as_ptr(), self._h)

    def close(self):
        if getattr(self, "_h", None) and self._h.value:
            self.lib.call("bulletou_cuda_cpp_graph_destroy", self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ---------------------------------------------------------------------------
# optimizer parameters (lib.rs:9204-9350)
# ---------------------------------------------------------------------------
@dataclass(frozen=True)
class RAdamStepScale:
    step_size: float
    use_denom: bool


@dataclass(frozen=True)
class RAdamUpdateParams:
    step: int = 1
    gradient_factor: float = 1.0
    learning_rate: float = 0.001
    decay: float = 0.0
    beta1: float = 0.9
    beta2: float = 0.999
    n_sma_threshold: float = 5.0
    epsilon: float = 0.00000001
    min_weight: float = -FLT_MAX
    max_weight: float = FLT_MAX

    def validate(self) -> None:
        if self.step == 0:
            raise CudaCppError("RAdam step must be greater than zero")
        if not np.isfinite(self.gradient_factor):
            raise CudaCppError("RAdam gradient_factor must be finite")
        if not (np.isfinite(self.learning_rate) and self.learning_rate >= 0.0):
            raise CudaCppError("RAdam learning_rate must be finite and non-negative")
        if not np.isfinite(self.decay):
            raise CudaCppError("RAdam decay must be finite")
        if not (np.isfinite(self.beta1) and 0.0 <= self.beta1 < 1.0):
            raise CudaCppError("RAdam beta1 must be finite and in [0, 1)")
        if not (np.isfinite(self.beta2) and 0.0 <= self.beta2 < 1.0):
            raise CudaCppError("RAdam beta2 must be finite and in [0, 1)")
        if not (np.isfinite(self.n_sma_threshold) and self.n_sma_threshold >= 0.0):
            raise CudaCppError("RAdam n_sma_threshold must be finite and non-negative")
        if not (np.isfinite(self.epsilon) and self.epsilon > 0.0):
            raise CudaCppError("RAdam epsilon must be finite and positive")
        if not (np.isfinite(self.min_weight) and np.isfinite(self.max_weight) and self.min_weight <= self.max_weight):
            raise CudaCppError("RAdam clamp range must be finite and ordered")

    def step_scale(self) -> RAdamStepScale:
        """f32 arithmetic exactly as lib.rs:9268-9288."""
        self.validate()
        step = _f32(self.step)
        b1, b2 = _f32(self.beta1), _f32(self.beta2)
        one, two = _f32(1.0), _f32(2.0)
        beta2_t = _powf(b2, step)
        n_sma_max = two / (one - b2) - one
        n_sma = n_sma_max - two * step * beta2_t / (one - beta2_t)
        bc1 = one - _powf(b1, step)
        use_denom = bool(n_sma > _f32(self.n_sma_threshold))
        if use_denom:
            p1 = (n_sma - _f32(4.0)) / (n_sma_max - _f32(4.0))
            p2 = (n_sma - two) / n_sma
            p3 = n_sma_max / (n_sma_max - two)
            step_size = np.sqrt(p1 * p2 * p3) / bc1
        else:
            step_size = one / bc1
        return RAdamStepScale(float(_f32(step_size)), use_denom)


@dataclass(frozen=True)
class RangerUpdateParams:
    sgd_momentum: Optional[float] = None
    norm_loss_strength: float = 0.0
    norm_loss_before: bool = False
    radam: RAdamUpdateParams = field(default_factory=RAdamUpdateParams)
    lookahead_alpha: float = 0.5
    lookahead_period: int = 6
    clip_after_lookahead: bool = True

    def norm_loss_rate(self) -> float:
        """lib.rs:9318-9327 (f32 arithmetic)."""
        if self.norm_loss_strength == 0.0:
            return 0.0
        p = self.radam
        if self.norm_loss_before:
            lr = _f32(p.learning_rate)
        else:
            t = _f32(p.step)
            b1, b2 = _f32(p.beta1), _f32(p.beta2)
            lr = _f32(p.learning_rate) * np.sqrt(_f32(1.0) - _powf(b2, t)) / (
                (_f32(1.0) - _powf(b1, t)) * np.sqrt((_f32(1.0) + b2) * (_f32(1.0) + b2) + b2 * b2))
        return float(_f32(2.0) * _f32(self.norm_loss_strength) * _f32(lr))

    def validate(self) -> None:
        if self.sgd_momentum is not None and not (np.isfinite(self.sgd_momentum) and 0.0 <= self.sgd_momentum < 1.0):
            raise CudaCppError("SGD momentum must be finite and in [0, 1)")
        if not np.isfinite(self.norm_loss_strength) or self.norm_loss_strength < 0.0:
            raise CudaCppError("norm loss strength must be finite and non-negative")
        self.radam.validate()
        if not (np.isfinite(self.lookahead_alpha) and 0.0 <= self.lookahead_alpha <= 1.0):
            raise CudaCppError("Ranger lookahead_alpha must be finite and in [0, 1]")
        if self.lookahead_period == 0:
            raise CudaCppError("Ranger lookahead_period must be greater than zero")

    def should_lookahead(self) -> bool:
        self.validate()
        return self.radam.step % self.lookahead_period == 0

    def ffi_step(self, lr_multiplier: float = 1.0) -> RangerStep:
        """The scalars lib.rs:9518-9544 passes to ranger_update_device."""
        p = self.radam if lr_multiplier == 1.0 else replace(self.radam, learning_rate=self.radam.learning_rate * lr_multiplier)
        scale = p.step_scale()
        return RangerStep(self.norm_loss_rate(), int(self.norm_loss_before), p.gradient_factor, p.learning_rate,
                          scale.step_size, int(scale.use_denom), p.decay, p.beta1, p.beta2, p.epsilon, p.min_weight,
                          p.max_weight, int(self.should_lookahead()), self.lookahead_alpha,
                          int(self.clip_after_lookahead))


# ---------------------------------------------------------------------------
# losses (lib.rs:2447-2481)
# ---------------------------------------------------------------------------
@dataclass(frozen=True)
class ScalarLossKind:
    kind: str
    pow_exp: float = 2.0
    in_offset_over_scaling: float = 0.0
    k: float = 0.0

    @staticmethod
    def SigmoidPow(pow_exp: float = 2.0):  # noqa: N802
        return ScalarLossKind("SigmoidPow", pow_exp=pow_exp)

    @staticmethod
    def WinRateModel(pow_exp: float, in_offset_over_scaling: float):  # noqa: N802
        return ScalarLossKind("WinRateModel", pow_exp=pow_exp, in_offset_over_scaling=in_offset_over_scaling)

    @staticmethod
    def BceWithLogits():  # noqa: N802
        return ScalarLossKind("BceWithLogits")

    @staticmethod
    def BceErrorWeighted(k: float):  # noqa: N802
        return ScalarLossKind("BceErrorWeighted", k=k)

    def as_ffi(self) -> int:
        return {"BceWithLogits": 2, "BceErrorWeighted": 2, "SigmoidPow": 0, "WinRateModel": 1}[self.kind]

    def loss_pow_exp(self) -> float:
        return 2.0 if self.kind.startswith("Bce") else self.pow_exp

    def loss_param(self) -> float:
        if self.kind == "BceErrorWeighted":
            return self.k
        if self.kind == "WinRateModel":
            return self.in_offset_over_scaling
        return 0.0

    def spec(self, output_inv_scale: float, finalize: bool = True, normalizer: int = 0) -> LossSpec:
        return LossSpec(self.as_ffi(), output_inv_scale, self.loss_pow_exp(), self.loss_param(), int(finalize),
                        int(normalizer))


@dataclass
class ScalarLossReadback:
    per_sample: np.ndarray
    mean_output_gradients: np.ndarray
    weighted_sum: float
    mean: float


class ScalarLossWorkspace:
    def __init__(self, ctx: Context, batch_size: int):
        self.per_sample = F32Buffer(ctx, batch_size)
        self.mean_output_gradients = F32Buffer(ctx, batch_size)
        self.weighted_sum = F32Buffer(ctx, 1)
        self.mean = F32Buffer(ctx, 1)
        for b in (self.per_sample, self.mean_output_gradients, self.weighted_sum, self.mean):
            b.fill(0.0)

    def download(self, ctx: Optional[Context] = None) -> ScalarLossReadback:
        return ScalarLossReadback(self.per_sample.download(ctx), self.mean_output_gradients.download(ctx),
                                  float(self.weighted_sum.download(ctx)[0]), float(self.mean.download(ctx)[0]))


def scalar_loss_device(ctx: Context, kind: ScalarLossKind, output_inv_scale: float, batch: int,
                       outputs: F32Buffer, targets: F32Buffer, entry_weights: F32Buffer,
                       workspace: ScalarLossWorkspace, finalize_loss: bool = True) -> None:
    ctx.lib.call("bulletou_cuda_cpp_scalar_loss_device_with_finalize", ctx.as_ptr(), kind.as_ffi(), output_inv_scale,
                 kind.loss_pow_exp(), kind.loss_param(), batch, outputs.as_ptr(), targets.as_ptr(),
                 entry_weights.as_ptr(), workspace.per_sample.as_ptr(), workspace.mean_output_gradients.as_ptr(),
                 workspace.weighted_sum.as_ptr(), workspace.mean.as_ptr(), int(finalize_loss))


def scalar_loss_host(device: int, kind: ScalarLossKind, output_inv_scale: float, outputs, targets, entry_weights,
                     lib: Optional[Library] = None) -> ScalarLossReadback:
    lib = lib or library()
    o = np.ascontiguousarray(outputs, np.float32)
    t = np.ascontiguousarray(targets, np.float32)
    w = np.ascontiguousarray(entry_weights, np.float32)
    n = o.size
    ps, mg = np.empty(n, np.float32), np.empty(n, np.float32)
    ws, mean = np.empty(1, np.float32), np.empty(1, np.float32)
    lib.call("bulletou_cuda_cpp_scalar_loss_host", device, kind.as_ffi(), output_inv_scale, kind.loss_pow_exp(),
             kind.loss_param(), n, _ptr(o), _ptr(t), _ptr(w), _ptr(ps), _ptr(mg), _ptr(ws), _ptr(mean))
    return ScalarLossReadback(ps, mg, float(ws[0]), float(mean[0]))


# ---------------------------------------------------------------------------
# optimizer entry points
# ---------------------------------------------------------------------------
@dataclass
class RangerDeviceState:
    gradients: F32Buffer
    weights: F32Buffer
    momentum: F32Buffer
    velocity: F32Buffer
    slow_params: F32Buffer


def ranger_update_device(ctx: Context, params: RangerUpdateParams, state: RangerDeviceState,
                         lr_multiplier: float = 1.0) -> None:
    """lib.rs:9496-9545 (+ SGD branch)."""
    params.validate()
    n = len(state.weights)
    for b in (state.gradients, state.momentum, state.velocity, state.slow_params):
        if len(b) != n:
            raise CudaCppError("ranger state length mismatch")
    if params.sgd_momentum is not None:
        if params.norm_loss_strength != 0.0:
            raise CudaCppError("SGD does not support norm loss")
        p = params.radam
        ctx.lib.call("bulletou_cuda_cpp_sgd_momentum_update_device", ctx.as_ptr(), n, p.gradient_factor,
                     p.learning_rate * lr_multiplier, p.decay, params.sgd_momentum, p.min_weight, p.max_weight,
                     state.gradients.as_ptr(), state.weights.as_ptr(), state.momentum.as_ptr(),
                     state.velocity.as_ptr(), None)
        return
    s = params.ffi_step(lr_multiplier)
    ctx.lib.call("bulletou_cuda_cpp_ranger_update_device", ctx.as_ptr(), s.norm_loss_rate, s.norm_loss_before, n,
                 s.gradient_factor, s.learning_rate, s.step_size, s.use_denom, s.decay, s.beta1, s.beta2, s.epsilon,
                 s.min_weight, s.max_weight, s.do_lookahead, s.lookahead_alpha, s.clip_after_lookahead,
                 state.gradients.as_ptr(), state.weights.as_ptr(), state.momentum.as_ptr(), state.velocity.as_ptr(),
                 state.slow_params.as_ptr(), None)


def ranger_update_stacked_dirty_device(ctx: Context, params: RangerUpdateParams, state: RangerDeviceState,
                                       stride: int, dirty_buckets: I32Buffer, dirty_count: int,
                                       lr_multiplier: float = 1.0) -> None:
    """Ranger on the listed buckets of a [stacks][stride] group
    (update_param_group's dirty-bucket branch, lib.rs:8761-8890)."""
    params.validate()
    n = len(state.weights)
    s = params.ffi_step(lr_multiplier)
    ctx.lib.call("bulletou_cuda_cpp_ranger_update_stacked_dirty_device", ctx.as_ptr(), s.norm_loss_rate,
                 s.norm_loss_before, n, stride, dirty_count, s.gradient_factor, s.learning_rate, s.step_size,
                 s.use_denom, s.decay, s.beta1, s.beta2, s.epsilon, s.min_weight, s.max_weight, s.do_lookahead,
                 s.lookahead_alpha, s.clip_after_lookahead, dirty_buckets.as_ptr(), state.gradients.as_ptr(),
                 state.weights.as_ptr(), state.momentum.as_ptr(), state.velocity.as_ptr(), state.slow_params.as_ptr())


def ranger_update_host(device: int, params: RangerUpdateParams, gradients: np.ndarray, weights: np.ndarray,
                       momentum: np.ndarray, velocity: np.ndarray, slow_params: np.ndarray,
                       lib: Optional[Library] = None) -> None:
    """In-place on float32 numpy arrays (lib.rs RangerStateMut + cu:14087)."""
    lib = lib or library()
    s = params.ffi_step()
    arrs = [gradients, weights, momentum, velocity, slow_params]
    for a in arrs:
        if a.dtype != np.float32 or not a.flags.c_contiguous:
            raise CudaCppError("ranger_update_host needs contiguous float32 arrays")
    lib.call("bulletou_cuda_cpp_ranger_update_host", device, weights.size, s.gradient_factor, s.learning_rate,
             s.step_size, s.use_denom, s.decay, s.beta1, s.beta2, s.epsilon, s.min_weight, s.max_weight,
             s.do_lookahead, s.lookahead_alpha, s.clip_after_lookahead, *[_ptr(a) for a in arrs])


def axpy_host(device: int, a: float, x, y, lib: Optional[Library] = None) -> np.ndarray:
    lib = lib or library()
    xa, ya = np.ascontiguousarray(x, np.float32), np.ascontiguousarray(y, np.float32)
    out = np.empty_like(xa)
    lib.call("bulletou_cuda_cpp_axpy_host", device, xa.size, a, _ptr(xa), _ptr(ya), _ptr(out))
    return out


# ---------------------------------------------------------------------------
# HalfKP NNUE (lib.rs:617-686, 875-1000, 2900-3000, 5430-6024)
# ---------------------------------------------------------------------------
@dataclass(frozen=True)
class NnueForwardShape:
    input_size: int
    l1: int
    l2: int
    l3: int

    def weight_lengths(self) -> list[int]:
        return [self.input_size * self.l1, self.l1, 2 * self.l1 * self.l2, self.l2, self.l2 * self.l3, self.l3,
                self.l3, 1]


NNUE_HALFKP_256X2_32_32 = NnueForwardShape(125388, 256, 32, 32)
NNUE_WEIGHT_NAMES = ("l0w", "l0b", "l1w", "l1b", "l2w", "l2b", "outw", "outb")


@dataclass
class NnueForwardHostWeights:
    shape: NnueForwardShape
    l0w: np.ndarray
    l0b: np.ndarray
    l1w: np.ndarray
    l1b: np.ndarray
    l2w: np.ndarray
    l2b: np.ndarray
    outw: np.ndarray
    outb: np.ndarray

    def arrays(self) -> list[np.ndarray]:
        return [np.ascontiguousarray(getattr(self, n), np.float32).reshape(-1) for n in NNUE_WEIGHT_NAMES]

    def validate(self) -> None:
        for name, arr, n in zip(NNUE_WEIGHT_NAMES, self.arrays(), self.shape.weight_lengths()):
            if arr.size != n:
                raise CudaCppError(f"{name} length mismatch: expected {n}, got {arr.size}")


@dataclass
class NnueTrainStepHostBatch:
    stm_indices: np.ndarray
    nstm_indices: np.ndarray
    targets: np.ndarray
    entry_weights: np.ndarray
    batch_size: int
    max_active: int

    def validate(self) -> None:
        n = self.batch_size * self.max_active
        for name, a, want in (("stm_indices", self.stm_indices, n), ("nstm_indices", self.nstm_indices, n),
                              ("train targets", self.targets, self.batch_size),
                              ("train entry_weights", self.entry_weights, self.batch_size)):
            if np.asarray(a).size != want:
                raise CudaCppError(f"{name} length mismatch: expected {want}, got {np.asarray(a).size}")


def nnue_forward_host(device: int, shape: NnueForwardShape, stm_indices, nstm_indices, batch_size: int,
                      max_active: int, weights: NnueForwardHostWeights, lib: Optional[Library] = None) -> np.ndarray:
    lib = lib or library()
    s = np.ascontiguousarray(stm_indices, np.int32)
    n = np.ascontiguousarray(nstm_indices, np.int32)
    w = weights.arrays()
    out = np.empty(batch_size, np.float32)
    lib.call("bulletou_cuda_cpp_nnue_forward_host", device, shape.input_size, shape.l1, shape.l2, shape.l3,
             batch_size, max_active, _ptr(s), _ptr(n), *[_ptr(a) for a in w], _ptr(out))
    return out


class NnueForwardWorkspace:
    def __init__(self, ctx: Context, shape: NnueForwardShape, batch_size: int):
        b = batch_size
        self.stm_l0 = F32Buffer(ctx, b * shape.l1)
        self.nstm_l0 = F32Buffer(ctx, b * shape.l1)
        self.combined = F32Buffer(ctx, b * shape.l1 * 2)
        self.hidden1 = F32Buffer(ctx, b * shape.l2)
        self.hidden2 = F32Buffer(ctx, b * shape.l3)
        self.output = F32Buffer(ctx, b)


class NnueBackwardWorkspace:
    """All gradient buffers of the reference backward (lib.rs:2860-2880); the
    l0w gradient starts zeroed and is re-zeroed by every Ranger step."""

    NAMES = ("hidden2_gradients", "hidden1_gradients", "combined_gradients", "stm_l0_gradients", "nstm_l0_gradients",
             "l0w_gradients", "l0b_gradients", "l1w_gradients", "l1b_gradients", "l2w_gradients", "l2b_gradients",
             "outw_gradients", "outb_gradients")

    def __init__(self, ctx: Context, shape: NnueForwardShape, batch_size: int):
        b = batch_size
        lens = (b * shape.l3, b * shape.l2, b * shape.l1 * 2, b * shape.l1, b * shape.l1) + tuple(shape.weight_lengths())
        for name, n in zip(self.NAMES, lens):
            buf = F32Buffer(ctx, n)
            buf.fill(0.0)
            setattr(self, name, buf)

    def param_gradients(self) -> list[F32Buffer]:
        return [getattr(self, n) for n in self.NAMES[5:]]

    def download(self, ctx: Optional[Context] = None) -> dict:
        return {n: getattr(self, n).download(ctx) for n in self.NAMES}


def nnue_forward_device(ctx: Context, shape: NnueForwardShape, batch_size: int, max_active: int,
                        stm: I32Buffer, nstm: I32Buffer, weights: Sequence[F32Buffer], ws: NnueForwardWorkspace) -> None:
    ctx.lib.call("bulletou_cuda_cpp_nnue_forward_device", ctx.as_ptr(), shape.input_size, shape.l1, shape.l2,
                 shape.l3, batch_size, max_active, stm.as_ptr(), nstm.as_ptr(), *[w.as_ptr() for w in weights],
                 ws.stm_l0.as_ptr(), ws.nstm_l0.as_ptr(), ws.combined.as_ptr(), ws.hidden1.as_ptr(),
                 ws.hidden2.as_ptr(), ws.output.as_ptr())


def nnue_backward_device(ctx: Context, shape: NnueForwardShape, batch_size: int, max_active: int, stm: I32Buffer,
                         nstm: I32Buffer, weights: Sequence[F32Buffer], fws: NnueForwardWorkspace,
                         mean_output_gradients: F32Buffer, bws: NnueBackwardWorkspace, zero_l0_gradients: bool) -> None:
    ctx.lib.call("bulletou_cuda_cpp_nnue_backward_device", ctx.as_ptr(), shape.input_size, shape.l1, shape.l2,
                 shape.l3, batch_size, max_active, stm.as_ptr(), nstm.as_ptr(), fws.combined.as_ptr(),
                 fws.hidden1.as_ptr(), fws.hidden2.as_ptr(), fws.stm_l0.as_ptr(), fws.nstm_l0.as_ptr(),
                 weights[2].as_ptr(), weights[4].as_ptr(), weights[6].as_ptr(), mean_output_gradients.as_ptr(),
                 *[getattr(bws, n).as_ptr() for n in NnueBackwardWorkspace.NAMES], int(zero_l0_gradients))


class RangerParamState:
    """m = v = 0, slow = initial weights (lib.rs:4123-4130)."""

    def __init__(self, ctx: Context, weights: np.ndarray, momentum=None, velocity=None, slow=None):
        n = weights.size
        self.momentum = F32Buffer.from_host(ctx, momentum) if momentum is not None else F32Buffer(ctx, n)
        self.velocity = F32Buffer.from_host(ctx, velocity) if velocity is not None else F32Buffer(ctx, n)
        if momentum is None:
            self.momentum.fill(0.0)
        if velocity is None:
            self.velocity.fill(0.0)
        self.slow_params = F32Buffer.from_host(ctx, weights if slow is None else slow)

    def download(self, ctx: Optional[Context] = None) -> dict:
        return {"momentum": self.momentum.download(ctx), "velocity": self.velocity.download(ctx),
                "slow_params": self.slow_params.download(ctx)}


def upload_from_pinned(ctx: Context, dst: "_DeviceBuffer", pinned) -> None:
    """Asynchronous H2D copy of a whole page-locked host buffer on ctx's stream,
    with no host copy.  `pinned` is a _PinnedBuffer of this library (its
    *_upload_pinned entries) or a page-locked numpy array (e.g. a view of
    pinned torch memory), which goes through the drop-in ABI's plain *_upload
    entries (cu:10084, 10153: one cudaMemcpyAsync, asynchronous from
    page-locked memory) -- on either backend library."""
    i32 = isinstance(dst, I32Buffer)
    if isinstance(pinned, np.ndarray):
        name = "bulletou_cuda_cpp_i32_upload" if i32 else "bulletou_cuda_cpp_f32_upload"
        ctx.lib.call(name, ctx.as_ptr(), dst.as_ptr(), ctypes.c_void_p(pinned.ctypes.data), pinned.size)
        return
    name = "bulletou_b200_i32_upload_pinned" if i32 else "bulletou_b200_f32_upload_pinned"
    ctx.lib.call(name, ctx.as_ptr(), dst.as_ptr(), pinned.as_ptr(), pinned.length)


def _nbytes(buf) -> int:
    return int(buf.nbytes) if isinstance(buf, np.ndarray) else 4 * buf.length


class NnueTrainStepUploadSlot:
    """Device batch buffers + pinned staging + upload/compute events
    (NnueTrainStepUploadSlot, lib.rs:5509-5600).  Before a slot is refilled,
    the previous upload must have finished (the pinned memory is reused) and
    the compute stream must be done with the device buffers."""

    def __init__(self, ctx: Context, batch_size: int, max_active: int):
        n = batch_size * max_active
        self.stm_indices, self.nstm_indices = I32Buffer(ctx, n), I32Buffer(ctx, n)
        self.targets, self.entry_weights = F32Buffer(ctx, batch_size), F32Buffer(ctx, batch_size)
        self.pinned = (PinnedI32Buffer(ctx, n), PinnedI32Buffer(ctx, n), PinnedF32Buffer(ctx, batch_size),
                       PinnedF32Buffer(ctx, batch_size))
        self.upload_ready = Event(ctx)
        self.compute_done = Event(ctx)
        self.in_use = False

    def fill(self, batch: "NnueTrainStepHostBatch") -> None:
        for dst, src in zip(self.pinned, (batch.stm_indices, batch.nstm_indices, batch.targets, batch.entry_weights)):
            np.copyto(dst.host(), np.asarray(src).reshape(-1))

    def upload(self, upload_ctx: Context, batch, pinned_source=None) -> int:
        lib = upload_ctx.lib
        if self.in_use:
            self.upload_ready.synchronize()
            self.compute_done.wait(upload_ctx)
        dsts = (self.stm_indices, self.nstm_indices, self.targets, self.entry_weights)
        if pinned_source is None and not lib.has("bulletou_b200_i32_upload_pinned"):
            # the reference ABI: staged uploads (host memcpy into the pinned
            # staging buffer, then an async copy), lib.rs:5552-5575
            if batch is None:
                raise CudaCppError("this backend needs host batch arrays for staged uploads")
            srcs = (batch.stm_indices, batch.nstm_indices, batch.targets, batch.entry_weights)
            for pin, dst, a in zip(self.pinned, dsts, srcs):
                pin.upload_to_device(upload_ctx, dst, a)
            self.upload_ready.record(upload_ctx)
            self.in_use = True
            return 4 * sum(x.length for x in self.pinned)
        src = pinned_source.pinned if pinned_source is not None else self.pinned
        if pinned_source is None:
            self.fill(batch)
        for dst, pin in zip(dsts, src):
            upload_from_pinned(upload_ctx, dst, pin)
        self.upload_ready.record(upload_ctx)
        self.in_use = True
        return sum(_nbytes(x) for x in src)


class NnueTrainStepRunner:
    """HalfKP train-step runner (lib.rs:5590-6024).

    ``fused`` (default: whatever the bound library supports) selects the
    product's single-call step (bulletou_b200_nnue_train_step_device); with
    ``fused=False`` the runner issues the reference's call sequence
    forward -> loss -> backward -> 8 x Ranger, on whichever library it is bound to.
    """

    def __init__(self, ctx: Context, initial_weights: NnueForwardHostWeights, batch_size: int, max_active: int,
                 fused: Optional[bool] = None, optimizer_states: Optional[list[dict]] = None):
        initial_weights.validate()
        if batch_size == 0:
            raise CudaCppError("NNUE train-step batch_size must be greater than zero")
        if max_active == 0:
            raise CudaCppError("NNUE train-step max_active must be greater than zero")
        self.ctx = ctx
        self.lib = ctx.lib
        self.shape = initial_weights.shape
        self.batch_size = batch_size
        self.max_active = max_active
        self.fused = self.lib.has("bulletou_b200_nnue_train_step_device") if fused is None else bool(fused)
        arrays = initial_weights.arrays()
        self.weights = [F32Buffer.from_host(ctx, a) for a in arrays]
        states = optimizer_states or [None] * 8
        self.optimizer_states = [
            RangerParamState(ctx, a, **({} if s is None else {"momentum": s["momentum"], "velocity": s["velocity"],
                                                               "slow": s["slow_params"]}))
            for a, s in zip(arrays, states)]
        n = batch_size * max_active
        self.stm_indices = I32Buffer(ctx, n)
        self.nstm_indices = I32Buffer(ctx, n)
        self.targets = F32Buffer(ctx, batch_size)
        self.entry_weights = F32Buffer(ctx, batch_size)
        self.loss_workspace = ScalarLossWorkspace(ctx, batch_size)
        if self.fused:
            self.output = F32Buffer(ctx, batch_size)
            self.forward_workspace = None
            self.backward_workspace = None
        else:
            self.forward_workspace = NnueForwardWorkspace(ctx, self.shape, batch_size)
            self.output = self.forward_workspace.output
            self.backward_workspace = NnueBackwardWorkspace(ctx, self.shape, batch_size)
        self._pinned = None
        self._handle_arrays = None

    # -- batch upload ------------------------------------------------------
    def upload_batch(self, batch: NnueTrainStepHostBatch, ctx: Optional[Context] = None) -> None:
        batch.validate()
        if batch.batch_size != self.batch_size or batch.max_active != self.max_active:
            raise CudaCppError(
                f"NNUE train-step batch layout mismatch: got batch_size={batch.batch_size} "
                f"max_active={batch.max_active}, expected batch_size={self.batch_size} max_active={self.max_active}")
        c = ctx or self.ctx
        self.stm_indices.upload(batch.stm_indices, c)
        self.nstm_indices.upload(batch.nstm_indices, c)
        self.targets.upload(batch.targets, c)
        self.entry_weights.upload(batch.entry_weights, c)

    def pinned_staging(self):
        """Pinned host arrays (stm, nstm, targets, entry_weights) for async uploads."""
        if self._pinned is None:
            n = self.batch_size * self.max_active
            self._pinned = (PinnedI32Buffer(self.ctx, n), PinnedI32Buffer(self.ctx, n),
                            PinnedF32Buffer(self.ctx, self.batch_size), PinnedF32Buffer(self.ctx, self.batch_size))
        return self._pinned

    def upload_pinned(self) -> int:
        """Async H2D of the pinned staging arrays; returns bytes copied."""
        s, n, t, w = self.pinned_staging()
        c = self.ctx.as_ptr()
        self.lib.call("bulletou_b200_i32_upload_pinned", c, self.stm_indices.as_ptr(), s.as_ptr(), s.length)
        self.lib.call("bulletou_b200_i32_upload_pinned", c, self.nstm_indices.as_ptr(), n.as_ptr(), n.length)
        self.lib.call("bulletou_b200_f32_upload_pinned", c, self.targets.as_ptr(), t.as_ptr(), t.length)
        self.lib.call("bulletou_b200_f32_upload_pinned", c, self.entry_weights.as_ptr(), w.as_ptr(), w.length)
        return 4 * (s.length + n.length + t.length + w.length)

    # -- steps -------------------------------------------------------------
    def step(self, ctx: Context, params: RangerUpdateParams, loss_kind: ScalarLossKind, output_inv_scale: float,
             batch: NnueTrainStepHostBatch) -> ScalarLossReadback:
        self.step_no_readback(ctx, params, loss_kind, output_inv_scale, batch)
        return self.read_loss(ctx)

    def step_no_readback(self, ctx, params, loss_kind, output_inv_scale, batch) -> None:
        self.step_no_readback_with_loss_finalize(ctx, params, loss_kind, output_inv_scale, batch, True)

    def step_no_readback_with_loss_finalize(self, ctx, params, loss_kind, output_inv_scale, batch,
                                            finalize_loss: bool) -> None:
        self.upload_batch(batch, ctx)
        self.step_device(ctx, params, loss_kind, output_inv_scale, finalize_loss)

    def step_from_records(self, ctx: Context, params: RangerUpdateParams, loss_kind: ScalarLossKind,
                          output_inv_scale: float, producer, records, finalize_loss: bool = True) -> None:
        """Decode PackedSfenValue records into this runner's batch on the
        device (HalfKP features, prepare_halfkp_direct_fast_batch,
        teacher_batch.rs:1687-1750), then step."""
        from .teacher import TeacherBatch

        cfg = producer.config
        base = self.shape.input_size - (1548 if self.shape.input_size == 125388 + 1548 else 0)
        if (cfg.feature_set != "halfkp" or cfg.active != self.max_active or producer.batch_size != self.batch_size
                or base != cfg.num_inputs):
            raise CudaCppError(
                f"teacher producer ({cfg.feature_set}, batch {producer.batch_size}, max_active {cfg.active}) does "
                f"not match the HalfKP runner (batch {self.batch_size}, max_active {self.max_active}, "
                f"input_size {self.shape.input_size})")
        view = TeacherBatch.wrap(self.stm_indices, self.nstm_indices, None, self.targets, self.entry_weights,
                                 self.batch_size, self.max_active)
        producer.prepare(ctx, records, view)
        self.step_device(ctx, params, loss_kind, output_inv_scale, finalize_loss)

    def _handles(self):
        if self._handle_arrays is None:
            arr = ctypes.c_void_p * 8
            self._handle_arrays = (arr(*[w.as_ptr().value for w in self.weights]),
                                   arr(*[s.momentum.as_ptr().value for s in self.optimizer_states]),
                                   arr(*[s.velocity.as_ptr().value for s in self.optimizer_states]),
                                   arr(*[s.slow_params.as_ptr().value for s in self.optimizer_states]))
        return self._handle_arrays

    def step_device(self, ctx: Context, params: RangerUpdateParams, loss_kind: ScalarLossKind,
                    output_inv_scale: float, finalize_loss: bool = True) -> None:
        """One step on the batch already resident in this runner's device buffers."""
        sh = self.shape
        lw = self.loss_workspace
        if self.fused and params.sgd_momentum is None:
            spec = loss_kind.spec(output_inv_scale, finalize_loss)
            step = params.ffi_step()
            w, m, v, s = self._handles()
            self.lib.call("bulletou_b200_nnue_train_step_device", ctx.as_ptr(), sh.input_size, sh.l1, sh.l2, sh.l3,
                          self.batch_size, self.max_active, self.stm_indices.as_ptr(), self.nstm_indices.as_ptr(),
                          self.targets.as_ptr(), self.entry_weights.as_ptr(), ctypes.byref(spec), ctypes.byref(step),
                          w, m, v, s, self.output.as_ptr(), lw.per_sample.as_ptr(), lw.mean_output_gradients.as_ptr(),
                          lw.weighted_sum.as_ptr(), lw.mean.as_ptr())
            return
        if self.forward_workspace is None:
            self.forward_workspace = NnueForwardWorkspace(ctx, sh, self.batch_size)
            self.output = self.forward_workspace.output
            self.backward_workspace = NnueBackwardWorkspace(ctx, sh, self.batch_size)
        fws, bws = self.forward_workspace, self.backward_workspace
        nnue_forward_device(ctx, sh, self.batch_size, self.max_active, self.stm_indices, self.nstm_indices,
                            self.weights, fws)
        scalar_loss_device(ctx, loss_kind, output_inv_scale, self.batch_size, fws.output, self.targets,
                           self.entry_weights, lw, finalize_loss)
        nnue_backward_device(ctx, sh, self.batch_size, self.max_active, self.stm_indices, self.nstm_indices,
                             self.weights, fws, lw.mean_output_gradients, bws, False)
        for g, w, st in zip(bws.param_gradients(), self.weights, self.optimizer_states):
            ranger_update_device(ctx, params, RangerDeviceState(g, w, st.momentum, st.velocity, st.slow_params))

    # -- pipelined steps (lib.rs:5509-5600, 5801-5856) ----------------------
    def upload_slots(self, count: int = 2) -> list["NnueTrainStepUploadSlot"]:
        if getattr(self, "_slots", None) is None or len(self._slots) != count:
            self._slots = [NnueTrainStepUploadSlot(self.ctx, self.batch_size, self.max_active) for _ in range(count)]
            self._next_slot = 0
        return self._slots

    def upload_next(self, upload_ctx: Context, batch: "NnueTrainStepHostBatch | None" = None,
                    pinned_source: "NnueTrainStepUploadSlot | None" = None) -> int:
        """The upload half of step_pipelined_no_readback_with_loss_finalize on
        its own: the next step's batch into the next slot on `upload_ctx`, so
        a trainer can issue it while the current step still runs.  The step
        that consumes it is step_uploaded_no_readback_with_loss_finalize.
        Returns H2D bytes."""
        slots = self.upload_slots()
        slot = slots[self._next_slot]
        self._next_slot = (self._next_slot + 1) % len(slots)
        nbytes = slot.upload(upload_ctx, batch, pinned_source)
        if getattr(self, "_uploaded", None) is None:
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
        self.stm_indices, self.nstm_indices = slot.stm_indices, slot.nstm_indices
        self.targets, self.entry_weights = slot.targets, slot.entry_weights
        self.step_device(ctx, params, loss_kind, output_inv_scale, finalize_loss)
        slot.compute_done.record(ctx)

    def step_pipelined_no_readback_with_loss_finalize(self, ctx: Context, upload_ctx: Context,
                                                      params: RangerUpdateParams, loss_kind: ScalarLossKind,
                                                      output_inv_scale: float, batch: "NnueTrainStepHostBatch | None",
                                                      finalize_loss: bool = True,
                                                      pinned_source: "NnueTrainStepUploadSlot | None" = None,
                                                      loss_out: "PinnedF32Buffer | None" = None) -> int:
        """Upload on `upload_ctx` into the next slot, hand off with an event,
        run the step on `ctx`, then (optionally) an async D2H of the mean loss
        into `loss_out`.  Returns H2D bytes.  `pinned_source` uploads straight
        from an already-filled pinned slot instead of staging `batch`."""
        slots = self.upload_slots()
        slot = slots[self._next_slot]
        self._next_slot = (self._next_slot + 1) % len(slots)
        nbytes = slot.upload(upload_ctx, batch, pinned_source)
        slot.upload_ready.wait(ctx)
        self.stm_indices, self.nstm_indices = slot.stm_indices, slot.nstm_indices
        self.targets, self.entry_weights = slot.targets, slot.entry_weights
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
        return {n: w.download(ctx) for n, w in zip(NNUE_WEIGHT_NAMES, self.weights)}

    def read_optimizer_states(self, ctx: Optional[Context] = None) -> dict:
        return {n: s.download(ctx) for n, s in zip(NNUE_WEIGHT_NAMES, self.optimizer_states)}


# ---------------------------------------------------------------------------
# KPPT scalar tables (lib.rs:4389-5066)
# ---------------------------------------------------------------------------
KPPT_WEIGHT_NAMES = ("table_w", "table_b", "outw", "outb")


class KpptTableTrainStepRunner:
    """One KPPT component table (KK, KKP or KPP) trained with Ranger."""

    def __init__(self, ctx: Context, input_size: int, table_w: np.ndarray, table_b: float, outw: Sequence[float],
                 outb: float, batch_size: int, max_active: int, fused: Optional[bool] = None):
        self.ctx = ctx
        self.lib = ctx.lib
        self.input_size = int(input_size)
        self.batch_size = batch_size
        self.max_active = max_active
        self.fused = self.lib.has("bulletou_b200_kppt_train_step_device") if fused is None else bool(fused)
        arrays = [np.ascontiguousarray(table_w, np.float32).reshape(-1), np.array([table_b], np.float32),
                  np.asarray(outw, np.float32).reshape(2), np.array([outb], np.float32)]
        if arrays[0].size != self.input_size:
            raise CudaCppError("KPPT table_w length mismatch")
        self.weights = [F32Buffer.from_host(ctx, a) for a in arrays]
        self.optimizer_states = [RangerParamState(ctx, a) for a in arrays]
        n = batch_size * max_active
        self.stm_indices = I32Buffer(ctx, n)
        self.nstm_indices = I32Buffer(ctx, n)
        self.targets = F32Buffer(ctx, batch_size)
        self.entry_weights = F32Buffer(ctx, batch_size)
        self.loss_workspace = ScalarLossWorkspace(ctx, batch_size)
        self.output = F32Buffer(ctx, batch_size)
        self.stm_eval = None
        self._handle_arrays = None

    def upload_batch(self, stm, nstm, targets, entry_weights, ctx: Optional[Context] = None) -> None:
        c = ctx or self.ctx
        self.stm_indices.upload(stm, c)
        self.nstm_indices.upload(nstm, c)
        self.targets.upload(targets, c)
        self.entry_weights.upload(entry_weights, c)

    def _handles(self):
        if self._handle_arrays is None:
            arr = ctypes.c_void_p * 4
            self._handle_arrays = (arr(*[w.as_ptr().value for w in self.weights]),
                                   arr(*[s.momentum.as_ptr().value for s in self.optimizer_states]),
                                   arr(*[s.velocity.as_ptr().value for s in self.optimizer_states]),
                                   arr(*[s.slow_params.as_ptr().value for s in self.optimizer_states]))
        return self._handle_arrays

    def step_device(self, ctx: Context, params: RangerUpdateParams, loss_kind: ScalarLossKind,
                    output_inv_scale: float, finalize_loss: bool = True) -> None:
        lw = self.loss_workspace
        if self.fused:
            spec = loss_kind.spec(output_inv_scale, finalize_loss)
            step = params.ffi_step()
            w, m, v, s = self._handles()
            self.lib.call("bulletou_b200_kppt_train_step_device", ctx.as_ptr(), self.input_size, self.batch_size,
                          self.max_active, self.stm_indices.as_ptr(), self.nstm_indices.as_ptr(), self.targets.as_ptr(),
                          self.entry_weights.as_ptr(), ctypes.byref(spec), ctypes.byref(step), w, m, v, s,
                          self.output.as_ptr(), lw.per_sample.as_ptr(), lw.mean_output_gradients.as_ptr(),
                          lw.weighted_sum.as_ptr(), lw.mean.as_ptr())
            return
        if self.stm_eval is None:
            self.stm_eval = F32Buffer(ctx, self.batch_size)
            self.nstm_eval = F32Buffer(ctx, self.batch_size)
            self.grads = [F32Buffer(ctx, len(w)) for w in self.weights]
            for g in self.grads:
                g.fill(0.0)
        w = self.weights
        ctx.lib.call("bulletou_cuda_cpp_kppt_forward_device", ctx.as_ptr(), self.input_size, self.batch_size,
                     self.max_active, self.stm_indices.as_ptr(), self.nstm_indices.as_ptr(), w[0].as_ptr(),
                     w[1].as_ptr(), w[2].as_ptr(), w[3].as_ptr(), self.stm_eval.as_ptr(), self.nstm_eval.as_ptr(),
                     self.output.as_ptr())
        scalar_loss_device(ctx, loss_kind, output_inv_scale, self.batch_size, self.output, self.targets,
                           self.entry_weights, lw, finalize_loss)
        ctx.lib.call("bulletou_cuda_cpp_kppt_backward_device", ctx.as_ptr(), self.input_size, self.batch_size,
                     self.max_active, self.stm_indices.as_ptr(), self.nstm_indices.as_ptr(), self.stm_eval.as_ptr(),
                     self.nstm_eval.as_ptr(), w[2].as_ptr(), lw.mean_output_gradients.as_ptr(),
                     *[g.as_ptr() for g in self.grads])
        for g, wb, st in zip(self.grads, self.weights, self.optimizer_states):
            ranger_update_device(ctx, params, RangerDeviceState(g, wb, st.momentum, st.velocity, st.slow_params))

    def read_loss(self, ctx: Optional[Context] = None) -> ScalarLossReadback:
        return self.loss_workspace.download(ctx)

    def read_weights(self, ctx: Optional[Context] = None) -> dict:
        return {n: w.download(ctx) for n, w in zip(KPPT_WEIGHT_NAMES, self.weights)}
