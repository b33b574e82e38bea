"""CPU: pins the C oracle to the reference's own known-answer values
(tests/golden/reference_goldens.json, transcribed from the reference tests)
and to small pure-Python restatements of the reference CPU loops."""
import numpy as np

from oracle import oracle
from tests.conftest import assert_close

FLT_MAX = float(np.finfo(np.float32).max)


def test_tiny_nnue_trace_matches_fast_nnue_golden(tiny, goldens):
    shape, w = tiny
    g = goldens["tiny_nnue_trace"]
    out = oracle.nnue_forward(shape, g["stm"], g["nstm"], g["batch"], g["max_active"], w)
    for key, gk in (("stm_l0", "stm_l0"), ("nstm_l0", "nstm_l0"), ("combined", "combined"),
                    ("hidden1", "hidden1"), ("hidden2", "hidden2"), ("output", "outputs")):
        assert_close(out[key], g[gk], 0.0, g["tolerance"], key)


def test_tiny_nnue_two_samples(tiny, goldens):
    shape, w = tiny
    g = goldens["tiny_nnue_two_samples"]
    out = oracle.nnue_forward(shape, g["stm"], g["nstm"], g["batch"], g["max_active"], w)
    assert_close(out["output"], g["outputs"], 0.0, g["tolerance"], "outputs")


def test_sigmoid_mse_loss_known_values(goldens):
    g = goldens["sigmoid_mse_loss"]
    r = oracle.scalar_loss(0, g["output_inv_scale"], g["pow_exp"], 0.0, g["outputs"], g["targets"], g["weights"])
    tol = g["tolerance"]
    assert_close(r["per_sample"], g["per_sample"], 0.0, tol, "per_sample")
    assert_close(r["mean_output_gradients"], g["mean_output_gradients"], 0.0, tol, "mean_output_gradients")
    assert abs(r["weighted_sum"] - g["weighted_sum"]) < tol
    assert abs(r["mean"] - g["mean"]) < tol


def test_zero_entry_weight_masks_sample(goldens):
    g = goldens["zero_entry_weight"]
    r = oracle.scalar_loss(0, 1.0, 2.0, 0.0, g["outputs"], g["targets"], g["weights"])
    assert r["per_sample"][0] == g["per_sample0"]
    assert r["per_sample"][1] > g["per_sample1_min"]


def test_pow_exponent_changes_loss():
    # fast_loss.rs:128-143
    o, t, w = [-2.0, 0.0, 2.0], [0.0, 0.25, 1.0], [1.0, 1.0, 1.0]
    mse = oracle.scalar_loss(0, 1.0, 2.0, 0.0, o, t, w)["mean"]
    p15 = oracle.scalar_loss(0, 1.0, 1.5, 0.0, o, t, w)["mean"]
    assert np.isfinite(mse) and np.isfinite(p15) and mse != p15


def test_radam_step_scale_reference_points(goldens):
    g = goldens["radam_step_scale"]
    ss, ud = oracle.radam_step_scale(1)
    assert ud is g["step1"]["use_denom"]
    assert abs(ss - g["step1"]["step_size"]) < g["step1"]["tolerance"]
    ss6, ud6 = oracle.radam_step_scale(6)
    assert np.isfinite(ss6) and ss6 > 0.0 and ud6


def _py_tiny_backward(shape, w, stm, nstm, batch, A, targets, entry_weights):
    """Pure-Python restatement of smoke.rs:594-700 (cpu_tiny_nnue_backward)."""
    input_size, l1, l2, l3 = shape
    f = oracle.nnue_forward(shape, stm, nstm, batch, A, w)
    sig = lambda x: 1.0 / (1.0 + np.exp(-np.float32(x)))  # noqa: E731
    mog = [float(entry_weights[b]) * 2.0 * (sig(f["output"][b]) - targets[b]) * sig(f["output"][b])
           * (1.0 - sig(f["output"][b])) / batch for b in range(batch)]
    h2g = [mog[b] * w["outw"][k] for b in range(batch) for k in range(l3)]
    outw_g = [sum(mog[b] * f["hidden2"][b * l3 + k] for b in range(batch)) for k in range(l3)]

    def dense_bwd(inputs, acts, og, weights, in_dim, out_dim):
        ig = [0.0] * (batch * in_dim)
        wg = [0.0] * (in_dim * out_dim)
        bg = [0.0] * out_dim
        for b in range(batch):
            for o in range(out_dim):
                a = acts[b * out_dim + o]
                gr = og[b * out_dim + o] if 0.0 < a < 1.0 else 0.0
                bg[o] += gr
                for i in range(in_dim):
                    ig[b * in_dim + i] += gr * weights[i * out_dim + o]
                    wg[i * out_dim + o] += gr * inputs[b * in_dim + i]
        return ig, wg, bg

    h1g, l2w_g, l2b_g = dense_bwd(f["hidden1"], f["hidden2"], h2g, w["l2w"], l2, l3)
    cg, l1w_g, l1b_g = dense_bwd(f["combined"], f["hidden1"], h1g, w["l1w"], 2 * l1, l2)
    sg = [cg[b * 2 * l1 + c] if 0.0 < f["stm_l0"][b * l1 + c] < 1.0 else 0.0 for b in range(batch) for c in range(l1)]
    ng = [cg[b * 2 * l1 + l1 + c] if 0.0 < f["nstm_l0"][b * l1 + c] < 1.0 else 0.0
          for b in range(batch) for c in range(l1)]
    l0w_g = [0.0] * (input_size * l1)
    l0b_g = [sum(sg[b * l1 + c] + ng[b * l1 + c] for b in range(batch)) for c in range(l1)]
    for b in range(batch):
        for s in range(A):
            for idx, gg in ((stm[b * A + s], sg), (nstm[b * A + s], ng)):
                if 0 <= idx < input_size:
                    for c in range(l1):
                        l0w_g[idx * l1 + c] += gg[b * l1 + c]
    return f, mog, dict(outw_gradients=outw_g, outb_gradients=[sum(mog)], l2w_gradients=l2w_g,
                        l2b_gradients=l2b_g, l1w_gradients=l1w_g, l1b_gradients=l1b_g, l0w_gradients=l0w_g,
                        l0b_gradients=l0b_g, combined_gradients=cg, stm_l0_gradients=sg, nstm_l0_gradients=ng)


def test_oracle_backward_matches_smoke_cpu_backprop(tiny, goldens):
    shape, w = tiny
    g2 = goldens["tiny_nnue_two_samples"]
    bb = goldens["smoke_backward_batch"]
    f, mog, expect = _py_tiny_backward(shape, w, g2["stm"], g2["nstm"], 2, 3, bb["targets"], bb["entry_weights"])
    loss = oracle.scalar_loss(0, 1.0, 2.0, 0.0, f["output"], bb["targets"], bb["entry_weights"])
    assert_close(loss["mean_output_gradients"], mog, 0.0, 1e-7, "mog")
    got = oracle.nnue_backward(shape, g2["stm"], g2["nstm"], 2, 3, f, w, loss["mean_output_gradients"])
    for k, v in expect.items():
        assert_close(got[k], v, 0.0, bb["tolerance"], k)


def test_oracle_ranger_matches_restatement(goldens):
    g = goldens["smoke_ranger"]
    grads = np.array(g["gradients"], np.float32)
    w = np.array(g["weights"], np.float32)
    m, v, slow = np.zeros(4, np.float32), np.zeros(4, np.float32), w.copy()
    oracle.ranger_update(grads, w, m, v, slow, step=g["step"], learning_rate=g["learning_rate"],
                         min_weight=g["min_weight"], max_weight=g["max_weight"])
    assert np.all(grads == 0.0)
    # step 1: no denominator, step size 1/(1-beta1): w -= lr * 10 * 0.1 g
    expected = np.array(g["weights"], np.float32) - np.float32(0.01) * np.array(g["gradients"], np.float32)
    assert_close(w, expected, 1e-6, 1e-8, "weights")


def test_oracle_lookahead_interpolates_every_period():
    n = 8
    w = np.linspace(-0.5, 0.5, n).astype(np.float32)
    slow = np.zeros(n, np.float32)
    m, v = np.zeros(n, np.float32), np.zeros(n, np.float32)
    grads = np.zeros(n, np.float32)
    before = w.copy()
    oracle.ranger_update(grads, w, m, v, slow, step=6, learning_rate=0.0)
    assert_close(w, 0.5 * before, 1e-7, 0.0, "lookahead")
    assert np.array_equal(w, slow)


def test_oracle_kppt_forward_backward_small():
    rng = np.random.default_rng(3)
    n, batch, A = 50, 6, 5
    tw = rng.normal(0, 0.1, n).astype(np.float32)
    stm = rng.integers(-1, n, size=batch * A).astype(np.int32)
    nstm = rng.integers(-1, n, size=batch * A).astype(np.int32)
    f = oracle.kppt_forward(n, stm, nstm, batch, A, tw, 0.25, [0.7, -0.3], 0.1)
    for b in range(batch):
        s = 0.25 + sum(tw[i] for i in stm[b * A:(b + 1) * A] if i >= 0)
        ns = 0.25 + sum(tw[i] for i in nstm[b * A:(b + 1) * A] if i >= 0)
        assert abs(f["stm_eval"][b] - s) < 1e-6 and abs(f["nstm_eval"][b] - ns) < 1e-6
        assert abs(f["output"][b] - (0.7 * s - 0.3 * ns + 0.1)) < 1e-6
    mog = rng.normal(0, 1, batch).astype(np.float32)
    g = oracle.kppt_backward(n, stm, nstm, batch, A, f, [0.7, -0.3], mog)
    expect = np.zeros(n)
    for b in range(batch):
        for i in stm[b * A:(b + 1) * A]:
            if i >= 0:
                expect[i] += mog[b] * 0.7
        for i in nstm[b * A:(b + 1) * A]:
            if i >= 0:
                expect[i] += mog[b] * -0.3
    assert_close(g["table_w"], expect, 1e-6, 1e-7, "table grad")
    assert abs(g["outb"][0] - mog.sum()) < 1e-5
