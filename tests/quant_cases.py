"""Hand-built quantised SFNN networks that expose one integer function of the
engine evaluator at the raw output, plus an independent numpy restatement of
the export quantisation and the integer forward (examples/bulletou.rs:
8001-8163, 10050-10300, 26417-26493).  Shared by the CPU oracle tests and the
GPU parity tests."""
from __future__ import annotations

import numpy as np

QUANT_NAMES = ("l0w", "l0b", "l1w", "l1b", "l2w", "l2b", "l3w", "l3b")
DTYPES = {"l0w": np.int16, "l0b": np.int16, "l1w": np.int8, "l1b": np.int32, "l2w": np.int8, "l2b": np.int32,
          "l3w": np.int8, "l3b": np.int32}

# quantized_ft_accumulator_matches_engine_i16_wrapping (bulletou.rs:37876-37882):
# (sum0, sum1, ft_shift, expected pair value), floor rounding.
FT_PAIR_KATS = ((40_000, 254, 7, 0), (-65_500, 254, 7, 17), (254, 254, 7, 126))

# dense_qat_integer_activation_boundaries_match_nn_bin (bulletou.rs:29660-29672).
ACTIVATION_INPUTS = (-2 ** 31, -8193, -8192, -4096, -725, -724, -64, -1, 0, 1, 63, 64, 724, 725, 4096, 8127, 8128,
                     8191, 8192, 2 ** 31 - 1)


def pad32(n: int) -> int:
    return (n + 31) // 32 * 32


def empty_net(shape) -> dict:
    input_size, W, H, skip, L2, S = shape
    O = H + (1 if skip else 0)
    return {"l0w": np.zeros(input_size * W, np.int16), "l0b": np.zeros(W, np.int16),
            "l1w": np.zeros(S * O * pad32(W), np.int8), "l1b": np.zeros(S * O, np.int32),
            "l2w": np.zeros(S * L2 * pad32(2 * H), np.int8), "l2b": np.zeros(S * L2, np.int32),
            "l3w": np.zeros(S * pad32(L2), np.int8), "l3b": np.zeros(S, np.int32)}


def ft_pair_net(sum0: int, sum1: int):
    """W = 2, no features: the stm pair value of (sum0, sum1) reaches the raw
    output through the PSQT skip (l1[1] = ft[0])."""
    shape = (4, 2, 1, 1, 1, 1)
    q = empty_net(shape)
    assert sum0 % 2 == 0 and sum1 % 2 == 0
    q["l0b"][:] = [sum0 // 2, sum1 // 2]
    q["l1w"][1 * 32 + 0] = 1          # stack 0, output 1 (skip), input 0
    return shape, q


def activation_net(inputs):
    """Stack 2k has l1 = inputs[k] and reads SqrCReLU; stack 2k+1 the same l1
    and reads CReLU; each through an L2 weight of 64 (>> 6 restores the value)
    and an L3 weight of 1.  Sample b uses stack b."""
    n = 2 * len(inputs)
    shape = (4, 2, 1, 0, 1, n)
    q = empty_net(shape)
    for k, x in enumerate(inputs):
        for j in range(2):
            s = 2 * k + j
            q["l1b"][s] = x
            q["l2w"][s * 32 + j] = 64
            q["l3w"][s * 32] = 1
    return shape, q


def expected_activation(x: int, kind: int) -> int:
    if kind == 0:
        return min(max((x * x) >> 19, 0), 127)
    return min(max(x >> 6, 0), 127)


def round_half_away(x: np.ndarray) -> np.ndarray:
    return np.sign(x) * np.floor(np.abs(x) + 0.5)


def quantize_numpy(shape, w: dict, ft_alpha: float = 1.0, shared_alpha: float = 1.0) -> dict:
    """Restated export quantisation: f32 folds a + alpha * b (two roundings),
    round half away from zero in f64, saturate."""
    input_size, W, H, skip, L2, S = shape
    O, I2 = H + (1 if skip else 0), 2 * H
    base = 131949 if input_size == 131949 + 1629 else (73305 if input_size == 73305 + 1629 else 0)
    rows = base or input_size
    f32 = np.float32

    def q(v, scale, lo, hi, dt):
        return np.clip(round_half_away(np.asarray(v, np.float64) * scale), lo, hi).astype(dt)

    l0w = np.asarray(w["l0w"], f32).reshape(input_size, W)
    ft = l0w[:rows].copy()
    if base:
        virt = l0w[base + np.arange(rows) % 1629]
        ft = (ft + (f32(ft_alpha) * virt).astype(f32)).astype(f32)
    out = {"l0w": q(ft, 127.0, -32768, 32767, np.int16).reshape(-1),
           "l0b": q(w["l0b"], 127.0, -32768, 32767, np.int16)}
    a = f32(shared_alpha)

    def fold(x, shared):
        x = np.asarray(x, f32)
        if shared is None:
            return x
        return (x + (a * np.asarray(shared, f32)).astype(f32)).astype(f32)

    l1w = np.asarray(w["l1w"], f32).reshape(S, O, W)
    l1fw = None if w.get("l1fw") is None else np.asarray(w["l1fw"], f32).reshape(W, O).T[None]
    l1w = fold(l1w, l1fw)
    l1b = fold(np.asarray(w["l1b"], f32).reshape(S, O), None if w.get("l1fb") is None else w["l1fb"])
    l2w = fold(np.asarray(w["l2w"], f32).reshape(S, L2, I2),
               None if w.get("l2fw") is None else np.asarray(w["l2fw"], f32).reshape(L2, I2)[None])
    l2b = fold(np.asarray(w["l2b"], f32).reshape(S, L2), None if w.get("l2fb") is None else w["l2fb"])
    l3w = fold(np.asarray(w["l3w"], f32).reshape(S, L2), None if w.get("l3fw") is None else w["l3fw"])
    l3b = fold(np.asarray(w["l3b"], f32).reshape(S), None if w.get("l3fb") is None else w["l3fb"][0])

    def padded(x, n_in):
        p = np.zeros(x.shape[:-1] + (pad32(n_in),), np.int8)
        p[..., :n_in] = q(x, 64.0, -128, 127, np.int8)
        return p.reshape(-1)

    out.update({"l1w": padded(l1w, W), "l1b": q(l1b, 8128.0, -2 ** 31, 2 ** 31 - 1, np.int32).reshape(-1),
                "l2w": padded(l2w, I2), "l2b": q(l2b, 8128.0, -2 ** 31, 2 ** 31 - 1, np.int32).reshape(-1),
                "l3w": padded(l3w, L2), "l3b": q(l3b, 8128.0, -2 ** 31, 2 ** 31 - 1, np.int32).reshape(-1)})
    return out


def integer_forward_numpy(shape, stm, nstm, buckets, batch, max_active, q, ft_shift=7, ft_round=0, crelu_round=0,
                          sqr_round=0) -> np.ndarray:
    """Restated engine forward (vectorised over the batch); raw i32 outputs."""
    input_size, W, H, skip, L2, S = shape
    O, I2, half = H + (1 if skip else 0), 2 * H, W // 2
    base = 131949 if input_size == 131949 + 1629 else (73305 if input_size == 73305 + 1629 else 0)
    rows = base or input_size
    l0w = np.asarray(q["l0w"], np.int64).reshape(rows, W)
    l0b = np.asarray(q["l0b"], np.int64)

    def view(idx):
        idx = np.asarray(idx, np.int64).reshape(batch, max_active)
        acc = np.repeat(2 * l0b[None], batch, axis=0)
        for k in range(max_active):
            f = idx[:, k]
            ok = (f >= 0) & (f < rows)
            acc[ok] += 2 * l0w[f[ok]]
        x = ((acc + 32768) % 65536) - 32768        # i16 wrap
        x = np.clip(x, 0, 254)
        p = (x[:, :half] << ft_shift) * x[:, half:]
        p = (p + (1 << 15)) >> 16 if ft_round else p >> 16
        return np.clip(p, 0, 255)

    ft = np.concatenate([view(stm), view(nstm)], axis=1)
    b = np.asarray(buckets, np.int64)
    valid = (b >= 0) & (b < S)
    s = np.where(valid, b, 0)
    l1w = np.asarray(q["l1w"], np.int64).reshape(S, O, pad32(W))[:, :, :W]
    l1 = np.einsum("bi,boi->bo", ft, l1w[s]) + np.asarray(q["l1b"], np.int64).reshape(S, O)[s]
    x = l1[:, :H]
    sq = (x * x + (1 << 18)) >> 19 if sqr_round else (x * x) >> 19
    sq = np.minimum(sq, 127)

    def crelu(v):
        r = np.where(v > 0, (v + 32) >> 6, v >> 6) if crelu_round else v >> 6
        return np.clip(r, 0, 127)

    l2_in = np.concatenate([sq, crelu(x)], axis=1)
    l2w = np.asarray(q["l2w"], np.int64).reshape(S, L2, pad32(I2))[:, :, :I2]
    l2 = crelu(np.einsum("bi,boi->bo", l2_in, l2w[s]) + np.asarray(q["l2b"], np.int64).reshape(S, L2)[s])
    l3w = np.asarray(q["l3w"], np.int64).reshape(S, pad32(L2))[:, :L2]
    out = np.einsum("bi,bi->b", l2, l3w[s]) + np.asarray(q["l3b"], np.int64)[s]
    if skip:
        out = out + l1[:, H]
    out = np.where(valid, out, 0)
    return out.astype(np.int32)


def random_integer_net(rng: np.random.Generator, shape, full_range: bool) -> dict:
    """Random engine-format weights; full_range makes FT sums wrap in i16."""
    q = empty_net(shape)
    input_size, W, H, skip, L2, S = shape
    base = 131949 if input_size == 131949 + 1629 else (73305 if input_size == 73305 + 1629 else 0)
    rows = base or input_size
    lim = 32767 if full_range else 120
    q["l0w"] = rng.integers(-lim, lim + 1, size=rows * W).astype(np.int16)
    q["l0b"] = rng.integers(-60, 200, size=W).astype(np.int16)
    for name, n_in, n_rows in (("l1w", W, S * (H + (1 if skip else 0))), ("l2w", 2 * H, S * L2), ("l3w", L2, S)):
        m = np.zeros((n_rows, pad32(n_in)), np.int8)
        m[:, :n_in] = rng.integers(-128, 128, size=(n_rows, n_in))
        q[name] = m.reshape(-1)
    q["l1b"] = rng.integers(-20000, 20000, size=q["l1b"].size).astype(np.int32)
    q["l2b"] = rng.integers(-3000, 3000, size=q["l2b"].size).astype(np.int32)
    q["l3b"] = rng.integers(-3000, 3000, size=q["l3b"].size).astype(np.int32)
    return q
