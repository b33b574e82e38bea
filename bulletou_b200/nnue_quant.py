"""Quantised HalfKP 256x2-32-32: the reference's nn.bin quantisation of a
trained f32 net (write_cuda_cpp_nnue_nn_bin, examples/bulletou.rs:26303-26413)
and the engine's integer evaluation of it, on the device
(bulletou_b200_nnue_quantize_device / bulletou_b200_nnue_integer_forward_device)."""
from __future__ import annotations

import ctypes
from typing import Optional

import numpy as np

from .cuda_cpp import Context, F32Buffer, I32Buffer

NNUE_QUANT_NAMES = ("l0w", "l0b", "l1w", "l1b", "l2w", "l2b", "outw", "outb")
_DTYPES = {"l0w": np.int16, "l0b": np.int16, "l1w": np.int8, "l1b": np.int32, "l2w": np.int8, "l2b": np.int32,
           "outw": np.int8, "outb": np.int32}
HALFKP_BASE = 125388
HALFKP_PIECES = 1548


def _pad32(n: int) -> int:
    return (n + 31) // 32 * 32


class QuantizedNnueDeviceWeights:
    """The engine's integer tensors on the device: FT i16 (factorizer folded),
    dense i8 output-major padded to 32 inputs, i32 biases."""

    def __init__(self, ctx: Context, input_size: int, l1: int, l2: int, l3: int):
        self.dims = (input_size, l1, l2, l3)
        self.rows = HALFKP_BASE if input_size == HALFKP_BASE + HALFKP_PIECES else input_size
        self.counts = {"l0w": self.rows * l1, "l0b": l1, "l1w": l2 * _pad32(2 * l1), "l1b": l2,
                       "l2w": l3 * _pad32(l2), "l2b": l3, "outw": _pad32(l3), "outb": 1}
        self.buffers = {n: I32Buffer(ctx, (self.counts[n] * np.dtype(_DTYPES[n]).itemsize + 3) // 4)
                        for n in NNUE_QUANT_NAMES}
        self.errors = I32Buffer(ctx, 1)

    def _array(self):
        arr = (ctypes.c_void_p * 8)()
        for k, n in enumerate(NNUE_QUANT_NAMES):
            arr[k] = self.buffers[n].as_ptr().value
        return arr

    def download(self, ctx: Optional[Context] = None) -> dict:
        out = {n: self.buffers[n].download(ctx).view(_DTYPES[n])[: self.counts[n]].copy() for n in NNUE_QUANT_NAMES}
        out["errors"] = int(self.errors.download(ctx)[0])
        return out

    def upload(self, arrays: dict, ctx: Optional[Context] = None) -> None:
        for n in NNUE_QUANT_NAMES:
            a = np.ascontiguousarray(arrays[n], dtype=_DTYPES[n]).reshape(-1)
            if a.size != self.counts[n]:
                raise ValueError(f"quantised {n}: expected {self.counts[n]} values, got {a.size}")
            raw = np.zeros(self.buffers[n].length * 4, np.uint8)
            raw[: a.nbytes] = a.view(np.uint8)
            self.buffers[n].upload(raw.view(np.int32), ctx)


def nnue_quantize_device(ctx: Context, weights: dict, out: QuantizedNnueDeviceWeights) -> None:
    """weights: F32Buffer per name of NNUE_QUANT_NAMES (training layout)."""
    params = (ctypes.c_void_p * 8)(*[weights[n].as_ptr().value for n in NNUE_QUANT_NAMES])
    ctx.lib.call("bulletou_b200_nnue_quantize_device", ctx.as_ptr(), *out.dims, params, out._array(),
                 out.errors.as_ptr())


class NnueIntegerForwardWorkspace:
    def __init__(self, ctx: Context, batch_size: int):
        self.raw = I32Buffer(ctx, batch_size)
        self.score = I32Buffer(ctx, batch_size)
        self.errors = I32Buffer(ctx, 1)

    def download(self, ctx: Optional[Context] = None) -> dict:
        return {"raw": self.raw.download(ctx), "score": self.score.download(ctx),
                "errors": int(self.errors.download(ctx)[0])}


def nnue_integer_forward_device(ctx: Context, q: QuantizedNnueDeviceWeights, batch_size: int, max_active: int,
                                stm: I32Buffer, nstm: I32Buffer, ws: NnueIntegerForwardWorkspace,
                                fv_scale: int = 16) -> None:
    ctx.lib.call("bulletou_b200_nnue_integer_forward_device", ctx.as_ptr(), *q.dims, batch_size, max_active,
                 stm.as_ptr(), nstm.as_ptr(), q._array(), int(fv_scale), ws.raw.as_ptr(), ws.score.as_ptr(),
                 ws.errors.as_ptr())
