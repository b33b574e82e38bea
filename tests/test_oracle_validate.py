"""CPU: the validation-metrics oracle (oracle_validation_metrics, a
restatement of compute_sign_accuracy_with_loss_masked,
crates/bulletou_lib/src/validate.rs:353-470) pinned to the reference's own
validate.rs tests (inline constants, each cited)."""
import math

import numpy as np
import pytest

from bulletou_b200 import teacher as bt
from oracle import teacher as ot

V = "crates/bulletou_lib/src/validate.rs"


def test_accuracy_all_match():  # validate.rs:808-817
    r = ot.validation_metrics([0.5, -0.3, 1.2, -0.01], [200, -150, 800, -10], None, eval_scale=400.0)
    assert (r["compared"], r["sign_matches"], r["test_loss"]) == (4, 4, None)


def test_accuracy_half_mismatch():  # validate.rs:819-828
    r = ot.validation_metrics([0.5, -0.3, 1.2, -0.01], [200, -150, -800, 10], None, eval_scale=400.0)
    assert (r["compared"], r["sign_matches"]) == (4, 2)


def test_accuracy_excludes_draws():  # validate.rs:830-850
    r = ot.validation_metrics([0.5, -0.1, 0.3, -0.2], [200, 100, 0, -50], [1, 0, 0, -1], eval_scale=400.0)
    assert (r["compared"], r["sign_matches"], r["drawn_games"], r["loss_sampled"]) == (2, 2, 2, 4)
    assert r["test_loss"] is not None


def test_decisive_prediction_sign_distribution():  # validate.rs:852-861
    r = ot.validation_metrics([0.0, 0.2, -0.1, -0.3, 0.4], [1, 2, 3, 4, 5], [1, -1, -1, 0, 1], eval_scale=400.0)
    assert (r["compared"], r["predicted_nonnegative"], r["predicted_negative"], r["predicted_zero"]) == (4, 3, 1, 1)


def test_score_sign_fallback_without_results():  # validate.rs:863-876
    r = ot.validation_metrics([0.5, 0.3, 1.2], [200, 0, 0], None, eval_scale=400.0)
    assert (r["compared"], r["sign_matches"], r["drawn_games"], r["loss_sampled"]) == (1, 1, 2, 0)


def test_score_drop_filters_mate_stamps():  # validate.rs:878-887
    r = ot.validation_metrics([0.5, 0.3, 1.2, -0.5], [200, 32000, -32000, -10], None, score_drop_abs=32000,
                              eval_scale=400.0)
    assert (r["compared"], r["sign_matches"], r["filtered_by_score_cap"], r["drawn_games"]) == (2, 2, 2, 0)


def test_empty():  # validate.rs:889-895
    r = ot.validation_metrics([], [], None)
    assert r["compared"] == 0 and r["test_loss"] is None


def test_loss_pure_eval_target():  # validate.rs:897-907
    r = ot.validation_metrics([0.0, 0.0], [400, -400], [1, -1], lambda_=1.0, eval_scale=400.0)
    assert r["compared"] == 2 and abs(r["test_loss"] - 0.0533) < 1e-3


def test_loss_pure_wdl_target():  # validate.rs:909-922
    r = ot.validation_metrics([0.0, 0.0, 0.0], [100, -100, 100], [1, -1, 0], lambda_=0.0, eval_scale=400.0)
    assert abs(r["test_loss"] - 0.1666666) < 1e-3


def test_bce_large_zero_output_mean_is_log_two():  # validate.rs:775-789
    n = 921_060
    table = ot.wrm_table()
    r = ot.validation_metrics(np.zeros(n), np.full(n, 100), np.ones(n), lambda_=1.0, eval_scale=600.0,
                              loss_kind=2, nnue2score=600.0, in_scaling=340.0, wrm_table=table)
    assert r["loss_sampled"] == n and abs(r["test_loss"] - math.log(2.0)) < 1e-7


def test_bce_matches_teacher_transform_and_blend():  # validate.rs:791-806
    target = bt.WinRateModelTargetParams(135.0, 380.0, 0.05)
    table = ot.wrm_table(135.0, 380.0, 0.05)
    outputs, scores, results = [-1.0, 0.0, 1.0], [-300, 100, 500], [-1, 0, 1]
    r = ot.validation_metrics(outputs, scores, results, lambda_=0.7, eval_scale=600.0, loss_kind=2,
                              nnue2score=600.0, in_scaling=340.0, wrm_table=table)
    f32 = np.float32

    def bce(z, t):
        return f32((f32(1) - t) * z if z >= 0 else -t * z) + f32(math.log1p(math.exp(-abs(float(z)))))

    exp_sum = f32(0)
    for i, m in enumerate(outputs):
        t = f32(0.7) * table[scores[i] + 32768] + f32(0.3) * (f32(results[i]) + f32(1)) * f32(0.5)
        exp_sum += bce(f32(m) * f32(600) / f32(340), t)
    assert abs(r["test_loss"] - float(exp_sum / 3)) < 1e-6
    assert (r["sign_matches"], r["loss_sampled"]) == (2, 3)
    assert target.epsilon == 0.05


@pytest.mark.parametrize("kind", [0, 1, 2])
def test_oracle_matches_a_numpy_restatement(kind):
    rng = np.random.default_rng(kind)
    n = 5000
    o = rng.normal(0, 1.5, n).astype(np.float32)
    s = rng.integers(-4000, 4000, n).astype(np.int16)
    s[::50] = 32000
    r = rng.integers(-1, 2, n).astype(np.int8)
    table = ot.wrm_table()
    got = ot.validation_metrics(o, s, r, score_drop_abs=30000, lambda_=0.6, eval_scale=500.0, loss_kind=kind,
                                pow_exp=2.0, wrm_table=table)
    keep = np.abs(s.astype(np.int64)) < 30000
    dec = keep & (r != 0)
    assert got["filtered_by_score_cap"] == (~keep).sum() and got["compared"] == dec.sum()
    assert got["sign_matches"] == ((o >= 0) == (r > 0))[dec].sum()
    f = lambda x: 1 / (1 + np.exp(-x.astype(np.float64)))  # noqa: E731
    t_score = f(s[keep] / 500.0) if kind == 0 else table[s[keep].astype(np.int64) + 32768]
    t = 0.4 * np.where(r[keep] > 0, 1.0, np.where(r[keep] < 0, 0.0, 0.5)) + 0.6 * t_score
    m = o[keep].astype(np.float64)
    if kind == 0:
        loss = (f(m) - t) ** 2
    elif kind == 1:
        sc = m * 600.0
        loss = (0.5 * (1 + f((sc - 270) / 380) - f((-sc - 270) / 380)) - t) ** 2
    else:
        z = m * 600.0 / 380.0
        loss = np.where(z >= 0, (1 - t) * z, -t * z) + np.log1p(np.exp(-np.abs(z)))
    assert got["test_loss"] == pytest.approx(loss.mean(), rel=2e-5)
