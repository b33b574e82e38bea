"""CPU: pins the quantised-SFNN part of the C oracle (oracle_sfnn_quantize,
oracle_sfnn_integer_forward) to the reference's known-answer tests for the
engine evaluator (examples/bulletou.rs:29660-29672, 37876-37882) and to an
independent numpy restatement of the export quantisation and integer forward."""
import numpy as np
import pytest

from bulletou_b200 import synthetic
from oracle import oracle
from tests import quant_cases as qc


@pytest.mark.parametrize("sum0,sum1,shift,expected", qc.FT_PAIR_KATS)
def test_ft_pair_value_wraps_like_engine_i16(sum0, sum1, shift, expected):
    shape, q = qc.ft_pair_net(sum0, sum1)
    out = oracle.sfnn_integer_forward(shape, [-1], [-1], [0], 1, 1, q, ft_shift=shift)
    assert out["error"] == -1
    assert int(out["raw"][0]) == expected


def test_activation_boundaries_match_nn_bin():
    shape, q = qc.activation_net(qc.ACTIVATION_INPUTS)
    n = shape[5]
    out = oracle.sfnn_integer_forward(shape, [-1] * n, [-1] * n, list(range(n)), n, 1, q)
    for k, x in enumerate(qc.ACTIVATION_INPUTS):
        assert int(out["l1"][2 * k]) == x
        assert int(out["raw"][2 * k]) == qc.expected_activation(x, 0), f"square {x}"
        assert int(out["raw"][2 * k + 1]) == qc.expected_activation(x, 1), f"linear {x}"


def test_nearest_rounding_modes():
    # (254 << 7) * 2 / 65536 = 0.992 -> floor 0, nearest 1.
    shape, q = qc.ft_pair_net(254, 2)
    for mode, want in ((0, 0), (1, 1)):
        out = oracle.sfnn_integer_forward(shape, [-1], [-1], [0], 1, 1, q, ft_round=mode)
        assert int(out["raw"][0]) == want
    # CReLU nearest only rounds positive values: 95 >> 6 = 1, (95 + 32) >> 6 = 1; 96 -> 1 / 2; -33 -> 0 both.
    shape, q = qc.activation_net([95, 96, -33, 1000])
    n = shape[5]
    for crelu_round, sqr_round in ((0, 0), (1, 1)):
        out = oracle.sfnn_integer_forward(shape, [-1] * n, [-1] * n, list(range(n)), n, 1, q,
                                          crelu_round=crelu_round, sqr_round=sqr_round)
        for k, x in enumerate([95, 96, -33, 1000]):
            lin = (x + 32) >> 6 if (crelu_round and x > 0) else x >> 6
            sq = (x * x + (1 << 18)) >> 19 if sqr_round else (x * x) >> 19
            assert int(out["raw"][2 * k + 1]) == min(max(lin, 0), 127)
            assert int(out["raw"][2 * k]) == min(sq, 127)


def test_quantize_rounds_half_away_from_zero_and_saturates():
    shape = (4, 2, 1, 0, 1, 1)
    w = {"l0w": np.array([1.0, -1.0, 300.0, -300.0, 0.5 / 127, -0.5 / 127, 0, 0], np.float32),
         "l0b": np.array([0.0, 0.0], np.float32),
         # v * 64 = 0.5, 1.5 ... exactly: half-even would give 0 / 2.
         "l1w": np.array([0.5 / 64, 2.5 / 64], np.float32), "l1b": np.array([1e6], np.float32),
         "l2w": np.array([-0.5 / 64, 3.0], np.float32), "l2b": np.array([-1e6], np.float32),
         "l3w": np.array([-3.0], np.float32), "l3b": np.array([0.25], np.float32)}
    q = oracle.sfnn_quantize(shape, w)
    assert q["l1w"][:2].tolist() == [1, 3]
    assert q["l2w"][:2].tolist() == [-1, 127]
    assert q["l3w"][0] == -128
    assert q["l0w"][:4].tolist() == [127, -127, 32767, -32768]
    assert q["l1b"][0] == 2 ** 31 - 1 and q["l2b"][0] == -2 ** 31 and q["l3b"][0] == 2032
    ref = qc.quantize_numpy(shape, w)
    for n in qc.QUANT_NAMES:
        np.testing.assert_array_equal(q[n], ref[n], err_msg=n)


@pytest.mark.parametrize("case", ["factorized_shared", "plain_all_shared"])
def test_quantize_matches_numpy_restatement(case):
    rng = np.random.default_rng(11)
    if case == "factorized_shared":
        shape = (73305 + 1629, 64, 15, 1, 32, 9)
        w = synthetic.sfnn_weights(rng, input_size=shape[0], ft=64, shared_l1=True, std=0.3)
        alphas = (0.75, 1.25)
    else:
        shape = (500, 96, 7, 0, 16, 3)
        w = synthetic.sfnn_weights(rng, input_size=500, ft=96, l1_hidden=7, l1_skip=False, l2=16, stacks=3,
                                   shared_l1=True, shared_l2_l3=True, std=0.5)
        alphas = (1.0, 0.5)
    q = oracle.sfnn_quantize(shape, w, *alphas)
    ref = qc.quantize_numpy(shape, w, *alphas)
    for n in qc.QUANT_NAMES:
        np.testing.assert_array_equal(q[n], ref[n], err_msg=n)


@pytest.mark.parametrize("full_range", [False, True])
@pytest.mark.parametrize("modes", [(0, 0, 0), (1, 1, 1)])
def test_integer_forward_matches_numpy_restatement(full_range, modes):
    rng = np.random.default_rng(5 + full_range)
    shape = (73305 + 1629, 64, 15, 1, 32, 9)
    batch = 96
    q = qc.random_integer_net(rng, shape, full_range)
    b = synthetic.sfnn_batch(3, batch)
    stm, nstm = b["stm"].copy(), b["nstm"].copy()
    stm[::7] = -1  # padding slots
    out = oracle.sfnn_integer_forward(shape, stm, nstm, b["buckets"], batch, b["max_active"], q,
                                      ft_round=modes[0], crelu_round=modes[1], sqr_round=modes[2])
    ref = qc.integer_forward_numpy(shape, stm, nstm, b["buckets"], batch, b["max_active"], q, 7, *modes)
    assert out["error"] == -1
    np.testing.assert_array_equal(out["raw"], ref)


def test_integer_forward_reports_bad_bucket_and_feature():
    rng = np.random.default_rng(2)
    shape = (100, 8, 3, 1, 4, 2)
    q = qc.random_integer_net(rng, shape, False)
    stm = np.array([1, 2, 3, 4, 5, 6], np.int32)
    nstm = np.array([7, 8, 9, 10, 11, 100], np.int32)   # sample 1 has feature 100 >= rows
    out = oracle.sfnn_integer_forward(shape, stm, nstm, [0, 1], 2, 3, q)
    assert out["error"] == 1
    out = oracle.sfnn_integer_forward(shape, stm[:3], nstm[:3], [5], 1, 3, q)
    assert out["error"] == 0 and out["raw"][0] == 0


def test_final_division_truncates_toward_zero():
    raw = np.array([-49, -48, -36, -35, -12, -11, 0, 11, 12, 35, 36, 48, 49], np.int32)
    np.testing.assert_array_equal(oracle.final_division(raw, 24, False), [-2, -2, -1, -1, 0, 0, 0, 0, 0, 1, 1, 2, 2])
    np.testing.assert_array_equal(oracle.final_division(raw, 24, True), [-2, -2, -2, -1, -1, 0, 0, 0, 1, 1, 2, 2, 2])
