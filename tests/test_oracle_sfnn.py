"""CPU: pins the SFNN part of the C oracle to the reference's known answers
(fast_sfnn.rs tiny trace) and to a pure-Python restatement of the reference's
test oracle for the SFNN backward (tiny_sfnn_backward_cpu,
crates/cuda_cpp/src/lib.rs:14516-14710) and Ranger step (lib.rs:14712-14780)."""
import math

import numpy as np
import pytest

from oracle import oracle
from tests.conftest import assert_close

FLT_MAX = float(np.finfo(np.float32).max)
S = 127.0 / 128.0


def _tiny_sfnn_fast(goldens):
    g = goldens["tiny_sfnn_fast"]
    w = {k: np.asarray(v, np.float32) for k, v in g["weights"].items()}
    return g, tuple(g["shape"]), w


def test_tiny_sfnn_trace_matches_fast_sfnn_golden(goldens):
    g, shape, w = _tiny_sfnn_fast(goldens)
    out = oracle.sfnn_forward(shape, g["stm"], g["nstm"], g["buckets"], g["batch"], g["max_active"], w)
    for key, gk in (("stm_l0", "stm_l0"), ("nstm_l0", "nstm_l0"), ("combined", "combined"), ("l1", "l1"),
                    ("l2_input", "l2_input"), ("l2", "l2"), ("output", "outputs")):
        assert_close(out[key], g[gk], 0.0, g["tolerance"], key)


def test_invalid_bucket_gives_zero_head():
    g = {"stm": [0, 1, -1, 3, -1, -1], "nstm": [2, -1, -1, 0, 2, -1]}
    w = {k: np.asarray(v, np.float32) for k, v in {
        "l0w": np.linspace(-0.3, 0.3, 16), "l0b": [0.1] * 4, "l1w": np.linspace(-1, 1, 24), "l1b": [0.0] * 6,
        "l2w": np.linspace(-1, 1, 16), "l2b": [0.1] * 4, "l3w": [1.0, 2.0, 3.0, 4.0], "l3b": [0.5, 0.5]}.items()}
    out = oracle.sfnn_forward((4, 4, 2, 1, 2, 2), g["stm"], g["nstm"], [2, -1], 2, 3, w)
    assert not out["output"].any() and not out["l1"].any() and not out["l2"].any()


# ---------------------------------------------------------------- restatement of lib.rs:14252-14710

def _forward_trace(shape, stm, nstm, buckets, batch, A, w, base):
    _, W, H, skip, L2, _ = shape
    O, I2, half = H + 1, 2 * H, W // 2
    tr = {k: [] for k in ("stm_l0", "nstm_l0", "combined", "l1", "l2_input", "l2", "output")}
    for b in range(batch):
        s = buckets[b]
        views = []
        for idx in (stm, nstm):
            x = [float(v) for v in w["l0b"]]
            for f in idx[b * A:(b + 1) * A]:
                if 0 <= f < (base or shape[0]):
                    for j in range(W):
                        x[j] += float(w["l0w"][f * W + j])
                        if base:
                            x[j] += float(w["l0w"][(base + f % 1629) * W + j])
            views.append([min(max(v, 0.0), 1.0) for v in x])
        c = [views[0][j] * views[0][half + j] * S for j in range(half)] + \
            [views[1][j] * views[1][half + j] * S for j in range(half)]
        l1 = []
        for o in range(O):
            v = float(w["l1b"][s * O + o]) + float(w["l1fb"][o])
            for i in range(W):
                v += c[i] * (float(w["l1w"][(s * O + o) * W + i]) + float(w["l1fw"][i * O + o]))
            l1.append(v)
        l2in = [min(max(abs(l1[i]) ** 2 * S, 0.0), 1.0) for i in range(H)] + [min(max(l1[i], 0.0), 1.0) for i in range(H)]
        l2 = []
        for o in range(L2):
            v = float(w["l2b"][s * L2 + o]) + float(w["l2fb"][o])
            for i in range(I2):
                v += l2in[i] * (float(w["l2w"][(s * L2 + o) * I2 + i]) + float(w["l2fw"][o * I2 + i]))
            l2.append(min(max(v, 0.0), 1.0))
        out = float(w["l3b"][s]) + float(w["l3fb"][0]) + l1[H]
        for o in range(L2):
            out += l2[o] * (float(w["l3w"][s * L2 + o]) + float(w["l3fw"][o]))
        for k, v in (("stm_l0", views[0]), ("nstm_l0", views[1]), ("combined", c), ("l1", l1), ("l2_input", l2in),
                     ("l2", l2), ("output", [out])):
            tr[k].extend(v)
    return tr


def _backward(shape, stm, nstm, buckets, batch, A, w, tr, targets, ew, base):
    input_size, W, H, skip, L2, NS = shape
    O, I2, half = H + 1, 2 * H, W // 2
    cg = lambda a, g: g if 0.0 < a < 1.0 else 0.0  # noqa: E731
    gout = []
    for b in range(batch):
        p = 1.0 / (1.0 + math.exp(-tr["output"][b]))
        gout.append(ew[b] * 2.0 * (p - targets[b]) * p * (1.0 - p) / batch)
    G = {n: np.zeros(np.asarray(w[n]).size) for n in oracle.SFNN_NAMES}
    for b in range(batch):
        s = buckets[b]
        go = gout[b]
        G["l3b"][s] += go
        G["l3fb"][0] += go
        l1g = [0.0] * O
        l1g[H] = go
        g2 = []
        for o in range(L2):
            wt = float(w["l3w"][s * L2 + o]) + float(w["l3fw"][o])
            G["l3fw"][o] += go * tr["l2"][b * L2 + o]
            G["l3w"][s * L2 + o] += go * tr["l2"][b * L2 + o]
            g2.append(cg(tr["l2"][b * L2 + o], go * wt))
        gin = [0.0] * I2
        for o in range(L2):
            G["l2b"][s * L2 + o] += g2[o]
            G["l2fb"][o] += g2[o]
            for i in range(I2):
                x = tr["l2_input"][b * I2 + i]
                wt = float(w["l2w"][(s * L2 + o) * I2 + i]) + float(w["l2fw"][o * I2 + i])
                G["l2fw"][o * I2 + i] += g2[o] * x
                G["l2w"][(s * L2 + o) * I2 + i] += g2[o] * x
                gin[i] += g2[o] * wt
        for i in range(H):
            v = tr["l1"][b * O + i]
            l1g[i] += cg(tr["l2_input"][b * I2 + i], gin[i]) * 2.0 * v * S + cg(tr["l2_input"][b * I2 + H + i], gin[H + i])
        dc = [0.0] * W
        for o in range(O):
            G["l1b"][s * O + o] += l1g[o]
            G["l1fb"][o] += l1g[o]
            for i in range(W):
                x = tr["combined"][b * W + i]
                G["l1w"][(s * O + o) * W + i] += l1g[o] * x
                G["l1fw"][i * O + o] += l1g[o] * x
                dc[i] += l1g[o] * (float(w["l1w"][(s * O + o) * W + i]) + float(w["l1fw"][i * O + o]))
        for v, (idx, key) in enumerate(((stm, "stm_l0"), (nstm, "nstm_l0"))):
            x = tr[key][b * W:(b + 1) * W]
            for col in range(W):
                pair = col % half
                mate = half + pair if col < half else pair
                pre = cg(x[col], dc[v * half + pair] * x[mate] * S)
                G["l0b"][col] += pre
                for f in idx[b * A:(b + 1) * A]:
                    if 0 <= f < (base or input_size):
                        G["l0w"][f * W + col] += pre
                        if base:
                            G["l0w"][(base + f % 1629) * W + col] += pre
    return G, gout


def _runner_case(goldens):
    g = goldens["tiny_sfnn_runner"]
    w = {k: np.asarray(v, np.float32) for k, v in g["weights"].items()}
    return g, tuple(g["shape"]), w


def test_oracle_sfnn_backward_matches_reference_test_oracle(goldens):
    g, shape, w = _runner_case(goldens)
    args = (g["stm"], g["nstm"], g["buckets"], g["batch"], g["max_active"])
    fwd = oracle.sfnn_forward(shape, *args, w)
    tr = _forward_trace(shape, *args, w, 0)
    assert_close(fwd["output"], tr["output"], 1e-6, 1e-7, "output")
    loss = oracle.scalar_loss(0, 1.0, 2.0, 0.0, fwd["output"], g["targets"], g["entry_weights"])
    got = oracle.sfnn_backward(shape, *args, fwd, w, loss["mean_output_gradients"])
    ref, gout = _backward(shape, *args, w, tr, g["targets"], g["entry_weights"], 0)
    assert_close(loss["mean_output_gradients"], gout, 1e-5, 1e-8, "mean output gradients")
    for n in oracle.SFNN_NAMES:
        assert_close(got[f"{n}_gradients"], ref[n], 1e-5, 1e-8, n)


@pytest.mark.parametrize("alpha", [1.0])
def test_oracle_sfnn_factorized_virtual_rows(goldens, alpha):
    """HalfKA_hm2 + 1629 virtual rows: the virtual row of piece p receives the
    sum of the gradients of every king's row for p (add_sfnn_l0w_gradient,
    lib.rs:14782-14804)."""
    g, shape0, w0 = _runner_case(goldens)
    base, W = 73305, 4
    shape = (base + 1629,) + shape0[1:]
    rng = np.random.default_rng(3)
    w = dict(w0)
    w["l0w"] = rng.normal(0, 0.2, (base + 1629) * W).astype(np.float32)
    B, A = 3, 4
    stm = np.array([5, 1629 + 5, 44 * 1629 + 7, -1, 3, 3 + 1629 * 2, 10, -1, 73305 + 3, 8, 9, 11], np.int32)
    nstm = np.array([7, 1629 + 7, 2, -1, 100, 3, 1629 * 3 + 100, 4, 0, 1, 2, 5], np.int32)
    buckets = [0, 1, 1]
    targets, ew = [0.3, 0.6, 0.9], [1.0, 1.0, 0.5]
    fwd = oracle.sfnn_forward(shape, stm, nstm, buckets, B, A, w, alpha, 1.0)
    tr = _forward_trace(shape, list(stm), list(nstm), buckets, B, A, w, base)
    assert_close(fwd["output"], tr["output"], 1e-5, 1e-7, "output")
    loss = oracle.scalar_loss(0, 1.0, 2.0, 0.0, fwd["output"], targets, ew)
    got = oracle.sfnn_backward(shape, stm, nstm, buckets, B, A, fwd, w, loss["mean_output_gradients"], alpha, 1.0)
    ref, _ = _backward(shape, list(stm), list(nstm), buckets, B, A, w, tr, targets, ew, base)
    assert_close(got["l0w_gradients"], ref["l0w"], 1e-5, 1e-9, "l0w")
    assert np.abs(got["l0w_gradients"][base * W:]).max() > 0


def test_oracle_sfnn_train_step_matches_reference_test_oracle(goldens):
    g, shape, w = _runner_case(goldens)
    args = (g["stm"], g["nstm"], g["buckets"], g["batch"], g["max_active"])
    tr = _forward_trace(shape, *args, w, 0)
    grads, _ = _backward(shape, *args, w, tr, g["targets"], g["entry_weights"], 0)
    r = dict(g["ranger"])
    trainer = oracle.SfnnTrainer(shape, w)
    trainer.step(*args, g["targets"], g["entry_weights"], **r)
    for n in oracle.SFNN_NAMES:
        wt = np.asarray(w[n], np.float32).copy()
        gr = grads[n].astype(np.float32)
        m, v, slow = np.zeros_like(wt), np.zeros_like(wt), wt.copy()
        oracle.ranger_update(gr, wt, m, v, slow, **r)
        assert_close(trainer.w[n], wt, 0.0, g["tolerance"], n)


def test_shared_factor_clip_scales_bounds():
    r = oracle.shared_factor_clip({"min_weight": -1.98, "max_weight": 1.98}, 2.0)
    assert r["min_weight"] == pytest.approx(-0.99) and r["max_weight"] == pytest.approx(0.99)
    r0 = oracle.shared_factor_clip({"min_weight": -1.98, "max_weight": 1.98}, 0.0)
    assert r0["min_weight"] == -FLT_MAX and r0["max_weight"] == FLT_MAX
