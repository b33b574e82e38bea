"""TEST INFRASTRUCTURE ONLY -- numpy/ctypes driver of the C oracle
(oracle/bulletou_oracle.c).  Only tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg import this module, as the checker; the product
(bulletou_b200) never does.

Orchestrates the reference runner's order for one train step
(crates/cuda_cpp/src/lib.rs:5748-5799): forward -> scalar loss -> backward ->
Ranger on each parameter group in the order l0w, l0b, l1w, l1b, l2w, l2b,
outw, outb (lib.rs:5964-6024), with the RAdam step scale of lib.rs:9268-9288
and Lookahead every `lookahead_period` steps (lib.rs:9345-9348).
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "liboracle.so"
FLT_MAX = float(np.finfo(np.float32).max)

_lib = None


def build() -> Path:
    newest = max((HERE / f).stat().st_mtime for f in ("bulletou_oracle.c", "teacher_oracle.c", "Makefile"))
    if not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < newest:
        subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        _lib = ctypes.CDLL(str(LIB_PATH))
        i64, f, i, p = ctypes.c_int64, ctypes.c_float, ctypes.c_int, ctypes.c_void_p
        _lib.oracle_nnue_forward.argtypes = [i64] * 6 + [p] * 16
        _lib.oracle_scalar_loss.argtypes = [i, f, f, f, i64, f] + [p] * 7
        _lib.oracle_nnue_backward.argtypes = [i64] * 6 + [p] * 24
        _lib.oracle_radam_step_scale.argtypes = [ctypes.c_uint64, f, f, f, p, p]
        _lib.oracle_ranger_update.argtypes = [i64, f, f, f, i, f, f, f, f, f, f, i, f, i] + [p] * 5
        _lib.oracle_kppt_forward.argtypes = [i64] * 3 + [p] * 9
        _lib.oracle_kppt_backward.argtypes = [i64] * 3 + [p] * 11
        _lib.oracle_sfnn_forward.argtypes = [p] * 13
        _lib.oracle_sfnn_backward.argtypes = [p] * 17
        _lib.oracle_sfnn_forward_qat.argtypes = [p, p, i] + [p] * 13
        _lib.oracle_sfnn_backward_qat.argtypes = [p, p, i] + [p] * 17
        _lib.oracle_sfnn_quantize.argtypes = [p] * 11
        _lib.oracle_sfnn_integer_forward.argtypes = [p] * 12 + [i] * 4 + [p] * 3
        _lib.oracle_nnue_quantize.argtypes = [p] * 11
        _lib.oracle_nnue_integer_forward.argtypes = [p, i64, i64] + [p] * 10 + [i] + [p] * 3
        for fn in (_lib.oracle_nnue_forward, _lib.oracle_scalar_loss, _lib.oracle_nnue_backward,
                   _lib.oracle_radam_step_scale, _lib.oracle_ranger_update, _lib.oracle_kppt_forward,
                   _lib.oracle_kppt_backward, _lib.oracle_sfnn_forward, _lib.oracle_sfnn_backward,
                   _lib.oracle_sfnn_forward_qat, _lib.oracle_sfnn_backward_qat, _lib.oracle_sfnn_quantize, _lib.oracle_sfnn_integer_forward, _lib.oracle_nnue_quantize,
                   _lib.oracle_nnue_integer_forward):
            fn.restype = None
    return _lib


def _p(a: np.ndarray):
    assert a.flags.c_contiguous
    return ctypes.c_void_p(a.ctypes.data)


def _f(a):
    return np.ascontiguousarray(a, dtype=np.float32).reshape(-1)


def _i(a):
    return np.ascontiguousarray(a, dtype=np.int32).reshape(-1)


NAMES = ("l0w", "l0b", "l1w", "l1b", "l2w", "l2b", "outw", "outb")


def nnue_forward(shape, stm, nstm, batch, max_active, weights: dict) -> dict:
    input_size, l1, l2, l3 = shape
    w = [_f(weights[n]) for n in NAMES]
    out = {k: np.zeros(n, np.float32) for k, n in (("stm_l0", batch * l1), ("nstm_l0", batch * l1),
                                                    ("combined", batch * 2 * l1), ("hidden1", batch * l2),
                                                    ("hidden2", batch * l3), ("output", batch))}
    s, n = _i(stm), _i(nstm)
    lib().oracle_nnue_forward(input_size, l1, l2, l3, batch, max_active, _p(s), _p(n), *[_p(a) for a in w],
                              *[_p(out[k]) for k in ("stm_l0", "nstm_l0", "combined", "hidden1", "hidden2", "output")])
    return out


def scalar_loss(kind: int, inv_scale: float, pow_exp: float, param: float, outputs, targets, entry_weights,
                normalizer: float | None = None) -> dict:
    o, t, w = _f(outputs), _f(targets), _f(entry_weights)
    n = o.size
    ps, mg = np.zeros(n, np.float32), np.zeros(n, np.float32)
    ws, mean = np.zeros(1, np.float32), np.zeros(1, np.float32)
    lib().oracle_scalar_loss(kind, inv_scale, pow_exp, param, n, float(n if normalizer is None else normalizer),
                             _p(o), _p(t), _p(w), _p(ps), _p(mg), _p(ws), _p(mean))
    return {"per_sample": ps, "mean_output_gradients": mg, "weighted_sum": float(ws[0]), "mean": float(mean[0])}


def nnue_backward(shape, stm, nstm, batch, max_active, fwd: dict, weights: dict, mog, l0w_grad=None) -> dict:
    input_size, l1, l2, l3 = shape
    g = {k: np.zeros(n, np.float32) for k, n in (
        ("hidden2_gradients", batch * l3), ("hidden1_gradients", batch * l2), ("combined_gradients", batch * 2 * l1),
        ("stm_l0_gradients", batch * l1), ("nstm_l0_gradients", batch * l1), ("l0w_gradients", input_size * l1),
        ("l0b_gradients", l1), ("l1w_gradients", 2 * l1 * l2), ("l1b_gradients", l2), ("l2w_gradients", l2 * l3),
        ("l2b_gradients", l3), ("outw_gradients", l3), ("outb_gradients", 1))}
    if l0w_grad is not None:
        g["l0w_gradients"][:] = _f(l0w_grad)
    scratch = np.zeros(max(2 * l1 * l2, l2 * l3) + l1 + l2 + l3 + 64, np.float64)
    s, n = _i(stm), _i(nstm)
    mog = _f(mog)
    w1, w2, wo = _f(weights["l1w"]), _f(weights["l2w"]), _f(weights["outw"])
    fw = {k: _f(fwd[k]) for k in ("combined", "hidden1", "hidden2", "stm_l0", "nstm_l0")}
    lib().oracle_nnue_backward(input_size, l1, l2, l3, batch, max_active, _p(s), _p(n), _p(fw["combined"]),
                               _p(fw["hidden1"]), _p(fw["hidden2"]), _p(fw["stm_l0"]), _p(fw["nstm_l0"]),
                               _p(w1), _p(w2), _p(wo), _p(mog),
                               *[_p(g[k]) for k in ("hidden2_gradients", "hidden1_gradients", "combined_gradients",
                                                    "stm_l0_gradients", "nstm_l0_gradients", "l0w_gradients",
                                                    "l0b_gradients", "l1w_gradients", "l1b_gradients",
                                                    "l2w_gradients", "l2b_gradients", "outw_gradients",
                                                    "outb_gradients")], _p(scratch))
    return g


def radam_step_scale(step: int, beta1=0.9, beta2=0.999, n_sma_threshold=5.0):
    ss = ctypes.c_float()
    ud = ctypes.c_int()
    lib().oracle_radam_step_scale(step, beta1, beta2, n_sma_threshold, ctypes.byref(ss), ctypes.byref(ud))
    return ss.value, bool(ud.value)


def ranger_update(grads, weights, momentum, velocity, slow, *, step: int, learning_rate=0.001, beta1=0.9,
                  beta2=0.999, epsilon=1e-8, decay=0.0, gradient_factor=1.0, min_weight=-FLT_MAX,
                  max_weight=FLT_MAX, lookahead_alpha=0.5, lookahead_period=6, clip_after_lookahead=True,
                  n_sma_threshold=5.0) -> None:
    """In place on float32 arrays."""
    ss, ud = radam_step_scale(step, beta1, beta2, n_sma_threshold)
    do_la = int(step % lookahead_period == 0)
    lib().oracle_ranger_update(weights.size, gradient_factor, learning_rate, ss, int(ud), decay, beta1, beta2, epsilon,
                               min_weight, max_weight, do_la, lookahead_alpha, int(clip_after_lookahead),
                               _p(grads), _p(weights), _p(momentum), _p(velocity), _p(slow))


class NnueTrainer:
    """CPU reference runner for HalfKP: weights, Ranger state, one step at a time."""

    def __init__(self, shape, weights: dict):
        self.shape = tuple(shape)
        self.w = {n: _f(weights[n]).copy() for n in NAMES}
        self.m = {n: np.zeros_like(self.w[n]) for n in NAMES}
        self.v = {n: np.zeros_like(self.w[n]) for n in NAMES}
        self.slow = {n: self.w[n].copy() for n in NAMES}
        self.l0w_grad = np.zeros_like(self.w["l0w"])

    def step(self, stm, nstm, batch, max_active, targets, entry_weights, *, loss_kind=0, inv_scale=1.0, pow_exp=2.0,
             loss_param=0.0, **ranger) -> dict:
        fwd = nnue_forward(self.shape, stm, nstm, batch, max_active, self.w)
        loss = scalar_loss(loss_kind, inv_scale, pow_exp, loss_param, fwd["output"], targets, entry_weights)
        g = nnue_backward(self.shape, stm, nstm, batch, max_active, fwd, self.w, loss["mean_output_gradients"],
                          self.l0w_grad)
        for n in NAMES:
            grad = g[f"{n}_gradients"]
            ranger_update(grad, self.w[n], self.m[n], self.v[n], self.slow[n], **ranger)
        self.l0w_grad[:] = 0.0
        return {"forward": fwd, "loss": loss, "gradients": g}


def kppt_forward(input_size, stm, nstm, batch, max_active, table_w, table_b, outw, outb) -> dict:
    out = {k: np.zeros(batch, np.float32) for k in ("stm_eval", "nstm_eval", "output")}
    s, n = _i(stm), _i(nstm)
    tw, tb, ow, ob = _f(table_w), _f(np.atleast_1d(table_b)), _f(outw), _f(np.atleast_1d(outb))
    lib().oracle_kppt_forward(input_size, batch, max_active, _p(s), _p(n), _p(tw), _p(tb), _p(ow), _p(ob),
                              _p(out["stm_eval"]), _p(out["nstm_eval"]), _p(out["output"]))
    return out


def kppt_backward(input_size, stm, nstm, batch, max_active, fwd: dict, outw, mog) -> dict:
    acc = np.zeros(input_size, np.float64)
    g = {"table_w": np.zeros(input_size, np.float32), "table_b": np.zeros(1, np.float32),
         "outw": np.zeros(2, np.float32), "outb": np.zeros(1, np.float32)}
    s, n = _i(stm), _i(nstm)
    ow, mg = _f(outw), _f(mog)
    lib().oracle_kppt_backward(input_size, batch, max_active, _p(s), _p(n), _p(fwd["stm_eval"]), _p(fwd["nstm_eval"]),
                               _p(ow), _p(mg), _p(acc), _p(g["table_w"]), _p(g["table_b"]), _p(g["outw"]),
                               _p(g["outb"]))
    return g


# ---------------------------------------------------------------- SFNN
SFNN_NAMES = ("l0w", "l0b", "l1w", "l1b", "l1fw", "l1fb", "l2w", "l2b", "l2fw", "l2fb", "l3w", "l3b", "l3fw", "l3fb")
SFNN_FACTORIZED_BASES = {73305 + 1629: 73305, 131949 + 1629: 131949}


def _sfnn_shape_arrays(shape, batch, max_active, ft_alpha, shared_alpha):
    input_size, ft_size, l1_hidden, l1_skip, l2_size, num_stacks = shape
    sh = np.array([input_size, ft_size, l1_hidden, int(bool(l1_skip)), l2_size, num_stacks, batch, max_active],
                  np.int64)
    al = np.array([ft_alpha, shared_alpha], np.float32)
    return sh, al


def _ptr_array(arrays):
    arr = (ctypes.c_void_p * len(arrays))()
    for k, a in enumerate(arrays):
        arr[k] = None if a is None else a.ctypes.data
    return arr


QAT_L1, QAT_FT, QAT_L2, QAT_L3 = 1, 2, 4, 8


def qat_mask(l1=False, ft=False, l2=False, l3=False) -> int:
    """SFNN_QAT_* bitmask of the C file (the runner's qat_l1 / qat_ft / qat_l2 / qat_l3)."""
    return (QAT_L1 if l1 else 0) | (QAT_FT if ft else 0) | (QAT_L2 if l2 else 0) | (QAT_L3 if l3 else 0)


def sfnn_forward(shape, stm, nstm, buckets, batch, max_active, weights: dict, ft_alpha=1.0, shared_alpha=1.0,
                 qat: int = 0) -> dict:
    """Forward of the SFNN LayerStack net (oracle_sfnn_forward_qat in the C file).
    shape = (input_size, ft_size, l1_hidden, l1_skip, l2_size, num_stacks);
    qat = qat_mask(...).  Dense QAT also returns the integer l1_raw / l2_raw."""
    _, W, H, skip, L2, _ = shape
    O = H + (1 if skip else 0)
    sh, al = _sfnn_shape_arrays(shape, batch, max_active, ft_alpha, shared_alpha)
    ws = [None if weights.get(n) is None else _f(weights[n]) for n in SFNN_NAMES]
    out = {"stm_l0": np.zeros(batch * W, np.float32), "nstm_l0": np.zeros(batch * W, np.float32),
           "combined": np.zeros(batch * W, np.float32), "l1": np.zeros(batch * O, np.float32),
           "l2_input": np.zeros(batch * 2 * H, np.float32), "l2": np.zeros(batch * L2, np.float32),
           "output": np.zeros(batch, np.float32), "l1_raw": np.zeros(batch * O, np.int32),
           "l2_raw": np.zeros(batch * L2, np.int32)}
    s, n, b = _i(stm), _i(nstm), _i(buckets)
    lib().oracle_sfnn_forward_qat(_p(sh), _p(al), int(qat), _p(s), _p(n), _p(b), _ptr_array(ws), *(_p(out[k]) for k in (
        "stm_l0", "nstm_l0", "combined", "l1", "l2_input", "l2", "output", "l1_raw", "l2_raw")))
    return out


def sfnn_backward(shape, stm, nstm, buckets, batch, max_active, fwd: dict, weights: dict, mog, ft_alpha=1.0,
                  shared_alpha=1.0, qat: int = 0) -> dict:
    """Parameter gradients ("<name>_gradients", FT virtual rows included) plus
    l1_gradients and combined_gradients (oracle_sfnn_backward_qat)."""
    input_size, W, H, skip, L2, S = shape
    O = H + (1 if skip else 0)
    sh, al = _sfnn_shape_arrays(shape, batch, max_active, ft_alpha, shared_alpha)
    ws = [None if weights.get(n) is None else _f(weights[n]) for n in SFNN_NAMES]
    grads = [None if a is None else np.zeros_like(a) for a in ws]
    acc = np.zeros(input_size * W, np.float64)
    l1g = np.zeros(batch * O, np.float32)
    cg = np.zeros(batch * W, np.float32)
    s, n, b = _i(stm), _i(nstm), _i(buckets)
    l1_raw = np.ascontiguousarray(fwd.get("l1_raw", np.zeros(batch * O, np.int32)), np.int32)
    l2_raw = np.ascontiguousarray(fwd.get("l2_raw", np.zeros(batch * L2, np.int32)), np.int32)
    lib().oracle_sfnn_backward_qat(_p(sh), _p(al), int(qat), _p(s), _p(n), _p(b), _ptr_array(ws),
                                   *(_p(_f(fwd[k])) for k in ("stm_l0", "nstm_l0", "combined", "l1", "l2_input",
                                                             "l2")),
                                   _p(l1_raw), _p(l2_raw), _p(_f(mog)), _p(acc), _ptr_array(grads), _p(l1g), _p(cg))
    out = {f"{name}_gradients": g for name, g in zip(SFNN_NAMES, grads) if g is not None}
    out["l1_gradients"] = l1g
    out["combined_gradients"] = cg
    return out


class SfnnTrainer:
    """CPU reference runner for SFNN (SfnnTrainStepRunner with default layer
    multipliers, lib.rs:7448-7533 / 8425-8730): forward -> loss -> backward ->
    Ranger on every present group in the order of SFNN_NAMES."""

    def __init__(self, shape, weights: dict, ft_alpha=1.0, shared_alpha=1.0, qat: int = 0):
        self.shape = tuple(shape)
        self.ft_alpha, self.shared_alpha = ft_alpha, shared_alpha
        self.qat = int(qat)
        self.names = [n for n in SFNN_NAMES if weights.get(n) is not None]
        self.w = {n: _f(weights[n]).copy() for n in self.names}
        self.m = {n: np.zeros_like(self.w[n]) for n in self.names}
        self.v = {n: np.zeros_like(self.w[n]) for n in self.names}
        self.slow = {n: self.w[n].copy() for n in self.names}

    def step(self, stm, nstm, buckets, batch, max_active, targets, entry_weights, *, loss_kind=0, inv_scale=1.0,
             pow_exp=2.0, loss_param=0.0, **ranger) -> dict:
        fwd = sfnn_forward(self.shape, stm, nstm, buckets, batch, max_active, self.w, self.ft_alpha, self.shared_alpha,
                           self.qat)
        loss = scalar_loss(loss_kind, inv_scale, pow_exp, loss_param, fwd["output"], targets, entry_weights)
        g = sfnn_backward(self.shape, stm, nstm, buckets, batch, max_active, fwd, self.w,
                          loss["mean_output_gradients"], self.ft_alpha, self.shared_alpha, self.qat)
        for n in self.names:
            r = dict(ranger)
            if n in ("l1fw", "l1fb"):
                r = shared_factor_clip(r, self.shared_alpha)
            ranger_update(g[f"{n}_gradients"], self.w[n], self.m[n], self.v[n], self.slow[n], **r)
        return {"forward": fwd, "loss": loss, "gradients": g}


def shared_factor_clip(ranger: dict, alpha: float) -> dict:
    """Bounds of a shared factor refer to alpha * w (factor_contribution_clip, lib.rs:8772-8788)."""
    r = dict(ranger)
    lo, hi = r.get("min_weight", -FLT_MAX), r.get("max_weight", FLT_MAX)
    if alpha == 0.0:
        r["min_weight"], r["max_weight"] = -FLT_MAX, FLT_MAX
        return r

    def scale(bound):
        if bound in (-FLT_MAX, FLT_MAX):
            return bound
        return float(np.float32(min(FLT_MAX, max(-FLT_MAX, float(bound) / float(alpha)))))

    r["min_weight"], r["max_weight"] = scale(lo), scale(hi)
    return r


# ------------------------------------------------------------------ quantised SFNN
SFNN_QUANT_NAMES = ("l0w", "l0b", "l1w", "l1b", "l2w", "l2b", "l3w", "l3b")


def pad32(n: int) -> int:
    return (n + 31) // 32 * 32


def sfnn_quant_shapes(shape) -> dict:
    """Element counts and dtypes of the quantised buffers (engine layout,
    dense rows padded to 32 inputs)."""
    input_size, W, H, skip, L2, S = shape
    O = H + (1 if skip else 0)
    base = 131949 if input_size == 131949 + 1629 else (73305 if input_size == 73305 + 1629 else 0)
    rows = base or input_size
    return {"l0w": (rows * W, np.int16), "l0b": (W, np.int16), "l1w": (S * O * pad32(W), np.int8),
            "l1b": (S * O, np.int32), "l2w": (S * L2 * pad32(2 * H), np.int8), "l2b": (S * L2, np.int32),
            "l3w": (S * pad32(L2), np.int8), "l3b": (S, np.int32)}


def sfnn_quantize(shape, weights: dict, ft_alpha=1.0, shared_alpha=1.0) -> dict:
    """Export quantisation (oracle_sfnn_quantize): FT and shared factors folded,
    FT i16 at 127, dense i8 at 64 (rows padded to 32), biases i32 at 8128."""
    sh, al = _sfnn_shape_arrays(shape, 1, 1, ft_alpha, shared_alpha)
    ws = [None if weights.get(n) is None else _f(weights[n]) for n in SFNN_NAMES]
    out = {n: np.zeros(c, dt) for n, (c, dt) in sfnn_quant_shapes(shape).items()}
    lib().oracle_sfnn_quantize(_p(sh), _p(al), _ptr_array(ws), *(_p(out[n]) for n in SFNN_QUANT_NAMES))
    return out


def sfnn_integer_forward(shape, stm, nstm, buckets, batch, max_active, q: dict, *, ft_shift=7, ft_round=0,
                         crelu_round=0, sqr_round=0) -> dict:
    """Engine integer forward (oracle_sfnn_integer_forward): raw i32 output,
    i32 L1 sums, and the first sample with an out-of-range feature or bucket
    (-1 when none)."""
    _, W, H, skip, L2, S = shape
    O = H + (1 if skip else 0)
    sh, al = _sfnn_shape_arrays(shape, batch, max_active, 1.0, 1.0)
    qs = {n: np.ascontiguousarray(q[n], dtype=dt).reshape(-1) for n, (_, dt) in sfnn_quant_shapes(shape).items()}
    l1 = np.zeros(batch * O, np.int32)
    raw = np.zeros(batch, np.int32)
    err = np.zeros(1, np.int64)
    s, n, b = _i(stm), _i(nstm), _i(buckets)
    lib().oracle_sfnn_integer_forward(_p(sh), _p(s), _p(n), _p(b), *(_p(qs[k]) for k in SFNN_QUANT_NAMES),
                                      int(ft_shift), int(ft_round), int(crelu_round), int(sqr_round),
                                      _p(l1), _p(raw), _p(err))
    return {"raw": raw, "l1": l1, "error": int(err[0])}


def final_division(raw, fv_scale: int, nearest: bool) -> np.ndarray:
    """raw / fv_scale truncating toward zero; nearest adds half the scale away
    from zero first (examples/bulletou.rs:8045-8054)."""
    r = np.asarray(raw, np.int64)
    mag = np.abs(r) + (fv_scale // 2 if nearest else 0)
    return (np.sign(r) * (mag // fv_scale)).astype(np.int32)


# ------------------------------------------------------------------ quantised HalfKP
NNUE_QUANT_NAMES = ("l0w", "l0b", "l1w", "l1b", "l2w", "l2b", "outw", "outb")


def nnue_quant_shapes(shape) -> dict:
    input_size, L1, L2, L3 = shape
    rows = 125388 if input_size == 125388 + 1548 else input_size
    return {"l0w": (rows * L1, np.int16), "l0b": (L1, np.int16), "l1w": (L2 * pad32(2 * L1), np.int8),
            "l1b": (L2, np.int32), "l2w": (L3 * pad32(L2), np.int8), "l2b": (L3, np.int32),
            "outw": (pad32(L3), np.int8), "outb": (1, np.int32)}


def nnue_quantize(shape, weights: dict) -> dict:
    """nn.bin quantisation of a HalfKP net (oracle_nnue_quantize); "errors"
    counts values outside their integer range (saturated)."""
    sh = np.asarray(shape, np.int64)
    ws = [_f(weights[n]) for n in NAMES]
    out = {n: np.zeros(c, dt) for n, (c, dt) in nnue_quant_shapes(shape).items()}
    err = np.zeros(1, np.int64)
    lib().oracle_nnue_quantize(_p(sh), _ptr_array(ws), *(_p(out[n]) for n in NNUE_QUANT_NAMES), _p(err))
    out["errors"] = int(err[0])
    return out


def nnue_integer_forward(shape, stm, nstm, batch, max_active, q: dict, fv_scale: int = 16) -> dict:
    """The engine's integer HalfKP evaluation (oracle_nnue_integer_forward)."""
    sh = np.asarray(shape, np.int64)
    qs = {n: np.ascontiguousarray(q[n], dtype=dt).reshape(-1) for n, (_, dt) in nnue_quant_shapes(shape).items()}
    raw = np.zeros(batch, np.int32)
    score = np.zeros(batch, np.int32)
    err = np.zeros(1, np.int64)
    s, n = _i(stm), _i(nstm)
    lib().oracle_nnue_integer_forward(_p(sh), int(batch), int(max_active), _p(s), _p(n),
                                      *(_p(qs[k]) for k in NNUE_QUANT_NAMES), int(fv_scale), _p(raw), _p(score),
                                      _p(err))
    return {"raw": raw, "score": score, "errors": int(err[0])}
