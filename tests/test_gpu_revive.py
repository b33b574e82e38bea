"""FT revival on the device tensors of an SfnnTrainStepRunner, the reference's
GPU tests of crates/cuda_cpp/src/ft_revive.rs:171-258 on this backend."""
import numpy as np
import pytest

import bulletou_b200 as bo
from bulletou_b200 import revive as rv
from bulletou_b200 import sfnn as bs
from bulletou_b200 import state_bin as sb
from bulletou_b200 import synthetic as syn
from bulletou_b200.state_bin import RevivalRng

pytestmark = pytest.mark.gpu

SHAPE = bs.SfnnForwardShape(bs.HALFKA_HM2_DIMENSIONS + bs.PIECE_INPUTS, 12, 3, True, 5, 4)


def _runner(ctx, shared, alpha=bs.SfnnFactorizerAlpha()):
    w = syn.sfnn_weights(syn.rng_for(12), SHAPE.input_size, SHAPE.ft_size, SHAPE.l1_hidden, SHAPE.l1_skip,
                         SHAPE.l2_size, SHAPE.num_stacks, shared, False, 0.1)
    return bs.SfnnTrainStepRunner(ctx, bs.SfnnForwardHostWeights(SHAPE, **w), 1024, 1, alpha)


def _cal(mean=0.25):
    c = rv.FtCalibration(SHAPE.ft_size, SHAPE.num_stacks)
    c.counts[:] = 1024
    c.means[:] = mean
    return c


def test_reset_and_mean_compensation_preserve_other_columns(ctx):
    s = SHAPE
    r = _runner(ctx, False)
    old = r.read_weights(ctx)
    rv.revive_ft(ctx, r, _cal(), [0], s.input_size)
    ch = r.read_weights(ctx)
    ft, half = s.ft_size, s.ft_size // 2
    l0o, l0n = old["l0w"].reshape(-1, ft), ch["l0w"].reshape(-1, ft)
    keep = [j for j in range(ft) if j not in (0, half)]
    np.testing.assert_array_equal(l0n[:, keep], l0o[:, keep])
    assert ch["l0b"][0] == 0.5 and ch["l0b"][half] == 0.5
    # the revived rows are the revival stream, in unit order
    rng = RevivalRng()
    bound = max(np.float32(np.sqrt(np.float32(6.0) / np.float32(s.input_size + ft))), np.float32(1 / 127))
    for col in (0, half):
        want = rv._round_half_away(rng.signed_uniform_array(s.input_size) * bound * np.float32(127.0)) / np.float32(127.0)
        np.testing.assert_array_equal(l0n[:, col], want)
    l1o, l1n = old["l1w"].reshape(-1, ft), ch["l1w"].reshape(-1, ft)
    exp = old["l1b"] + np.float32(0.25) * l1o[:, 0] + np.float32(0.25) * l1o[:, half]
    np.testing.assert_allclose(ch["l1b"], exp, atol=1e-6)
    assert np.all(np.abs(np.abs(l1n[:, [0, half]]) - 1 / 64) < 1e-7)
    rv.compensate_ft_revival_mean(ctx, r, [0], _cal(0.5))
    after = r.read_weights(ctx)
    exp = ch["l1b"] - np.float32(0.5) * (l1n[:, 0] + l1n[:, half])
    np.testing.assert_allclose(after["l1b"], exp, atol=1e-6)
    np.testing.assert_array_equal(old["l2w"], after["l2w"])
    np.testing.assert_array_equal(old["l3w"], after["l3w"])
    st = r.read_optimizer_states(ctx)
    assert np.all(st["l0w"]["momentum"].reshape(-1, ft)[:, [0, half]] == 0.0)
    assert np.all(st["l1b"]["momentum"] == 0.0) and np.all(st["l1b"]["velocity"] == 0.0)
    # no units: the stream does not move; a second revival draws new rows,
    # and restoring the state repeats them exactly
    snap = sb.sfnn_runner_state(ctx, r, 0, 0)
    state_before = r.revival_rng.state
    rv.revive_ft(ctx, r, _cal(), [], s.input_size)
    assert r.revival_rng.state == state_before
    rv.begin_revival_epoch(r)
    rv.revive_ft(ctx, r, _cal(), [0], s.input_size)
    second = r.read_weights(ctx)
    assert not np.array_equal(second["l0w"], after["l0w"])
    sb.restore_sfnn_runner(ctx, r, snap)
    rv.begin_revival_epoch(r)
    rv.revive_ft(ctx, r, _cal(), [0], s.input_size)
    again = r.read_weights(ctx)
    for k in second:
        np.testing.assert_array_equal(again[k], second[k], err_msg=k)


def test_revive_one_saturated_unit_preserves_partner(ctx):
    s = SHAPE
    r = _runner(ctx, False)
    c = _cal()
    c.counts[:] = 0
    c.counts[0] = 1
    old = r.read_weights(ctx)
    rv.revive_ft_units(ctx, r, c, [0], s.input_size)
    new = r.read_weights(ctx)
    np.testing.assert_array_equal(old["l0w"].reshape(-1, s.ft_size)[:, 1:], new["l0w"].reshape(-1, s.ft_size)[:, 1:])
    np.testing.assert_array_equal(old["l0b"][1:], new["l0b"][1:])
    assert new["l0b"][0] == 0.5


def test_shared_and_virtual_columns(ctx):
    s = SHAPE
    r = _runner(ctx, True, bs.SfnnFactorizerAlpha(1.0, 0.7))
    old = r.read_weights(ctx)
    rv.revive_ft(ctx, r, _cal(), [0], s.input_size - 1)
    new = r.read_weights(ctx)
    np.testing.assert_array_equal(old["l1fw"], new["l1fw"])
    np.testing.assert_array_equal(old["l1fb"], new["l1fb"])
    ft, n = s.ft_size, s.l1_out
    l1 = new["l1w"].reshape(s.num_stacks, n, ft)
    fw = new["l1fw"].reshape(ft, n)
    for col in (0, ft // 2):
        assert new["l0w"][(s.input_size - 1) * ft + col] == 0.0
        eff = l1[:, :, col] + np.float32(0.7) * fw[col][None, :]
        assert np.all(np.abs(np.abs(eff) - 1 / 64) < 1e-6)
    st = r.read_optimizer_states(ctx)
    np.testing.assert_array_equal(st["l0w"]["slow_params"].reshape(-1, ft)[:, [0, ft // 2]],
                                  new["l0w"].reshape(-1, ft)[:, [0, ft // 2]])
    assert np.all(st["l0w"]["momentum"].reshape(-1, ft)[:, [0, ft // 2]] == 0.0)
    # the revived net trains on
    b = syn.sfnn_batch(5, 1024, stacks=s.num_stacks)
    k = b["max_active"]
    hb = bs.SfnnTrainStepHostBatch(b["stm"].reshape(-1, k)[:, 0].copy(), b["nstm"].reshape(-1, k)[:, 0].copy(),
                                   b["buckets"], b["targets"], b["entry_weights"], 1024, 1)
    loss = r.step(ctx, bo.RangerUpdateParams(radam=bo.RAdamUpdateParams(step=1)), bo.ScalarLossKind.SigmoidPow(2.0),
                  1 / 600, hb)
    assert np.isfinite(loss.mean)


def test_revival_rejects_legacy_factorizers(ctx):
    s = SHAPE
    w = syn.sfnn_weights(syn.rng_for(13), s.input_size, s.ft_size, s.l1_hidden, s.l1_skip, s.l2_size,
                         s.num_stacks, True, True, 0.1)
    r = bs.SfnnTrainStepRunner(ctx, bs.SfnnForwardHostWeights(s, **w), 1024, 1)
    with pytest.raises(bo.CudaCppError, match="FT revival requires"):
        rv.revive_ft(ctx, r, _cal(), [0], s.input_size)


def test_l1_contribution_mixed_constant_transfers_only_square_mean(ctx):
    """gpu_contribution_mixed_constant_transfers_only_square_mean
    (l1_revive.rs:290-320): unit 0 of bucket 0 has a constant square branch of
    1 and a constant normal branch of 0; reviving it moves exactly the L2
    weight of the square branch into the L2 bias."""
    s = bs.SfnnForwardShape(bs.HALFKA_HM2_DIMENSIONS + bs.PIECE_INPUTS, 12, 2, True, 5, 4)
    w = syn.sfnn_weights(syn.rng_for(14), s.input_size, s.ft_size, s.l1_hidden, s.l1_skip, s.l2_size,
                         s.num_stacks, False, False, 0.1)
    r = bs.SfnnTrainStepRunner(ctx, bs.SfnnForwardHostWeights(s, **w), 1024, 1)
    c = rv.L1Calibration(s.ft_size, s.l1_hidden, s.num_stacks)
    for i in range(1024):
        c.add([0], np.zeros(s.ft_size, np.float32), [1.0, float(i % 2), 0.0, float(i % 2)])
    old = r.read_weights(ctx)
    c.contribution.finish(old["l2w"], s.l2_size, 2, 0.01)
    assert c.candidates_for(True, False) == [0]
    assert rv.revive_l1_selected(ctx, r, c, True, False) == [0]
    new = r.read_weights(ctx)
    l2w = old["l2w"].reshape(-1, s.l2_in)
    for j in range(s.l2_size):
        assert abs(new["l2b"][j] - old["l2b"][j] - l2w[j, 0]) < 1e-6
    np.testing.assert_array_equal(old["l0w"], new["l0w"])
    np.testing.assert_array_equal(old["l3w"], new["l3w"])
    # the revived unit: fresh row from the stream, bias 0.5 at a zero input mean
    rng = RevivalRng()
    bound = np.float32(np.sqrt(np.float32(6.0) / np.float32(s.ft_size + s.l1_hidden)))
    np.testing.assert_array_equal(new["l1w"][:s.ft_size], rng.signed_uniform_array(s.ft_size) * bound)
    assert new["l1b"][0] == np.float32(0.5)
    np.testing.assert_array_equal(new["l1w"][s.ft_size:], old["l1w"][s.ft_size:])
    np.testing.assert_array_equal(new["l1b"][1:], old["l1b"][1:])
    assert set(np.abs(new["l2w"].reshape(-1, s.l2_in)[:s.l2_size, [0, 2]]).ravel().tolist()) == {1 / 64}
    # once per epoch; a no-op leaves the stream alone
    state = r.revival_rng.state
    assert rv.revive_l1_selected(ctx, r, c, True, False) == []
    assert r.revival_rng.state == state
    snap = sb.sfnn_runner_state(ctx, r, 0, 0)
    rv.begin_revival_epoch(r)
    assert r.revival_rng.state == state
    rv.revive_l1_selected(ctx, r, c, True, False)
    second = r.read_weights(ctx)
    assert not np.array_equal(new["l1w"], second["l1w"])
    sb.restore_sfnn_runner(ctx, r, snap)
    rv.begin_revival_epoch(r)
    rv.revive_l1_selected(ctx, r, c, True, False)
    again = r.read_weights(ctx)
    for k in second:
        np.testing.assert_array_equal(again[k], second[k], err_msg=k)
    # mean compensation removes the measured branch means from the L2 biases
    m = rv.L1Calibration(s.ft_size, s.l1_hidden, s.num_stacks)
    for i in range(8):
        m.add([0], np.zeros(s.ft_size, np.float32), [0.5, 0.0, 0.25, 0.0])
    before = r.read_weights(ctx)
    rv.compensate_l1_revival_mean(ctx, r, [0], m)
    after = r.read_weights(ctx)
    w2 = before["l2w"].reshape(-1, s.l2_in)
    for j in range(s.l2_size):
        exp = np.float32(np.float32(before["l2b"][j] - w2[j, 0] * np.float32(0.5)) - w2[j, 2] * np.float32(0.25))
        assert after["l2b"][j] == exp


def test_l2_contribution_preserves_empirical_mean(ctx):
    """gpu_contribution_preserves_empirical_mean_not_upper_or_zero
    (l2_revive.rs:181-202): unit 0 is constant at 0.75; its revival moves
    0.75 * w_old into the output bias and takes out the new unit's mean 0.5
    times its new weight."""
    s = SHAPE
    w = syn.sfnn_weights(syn.rng_for(15), s.input_size, s.ft_size, s.l1_hidden, s.l1_skip, s.l2_size,
                         s.num_stacks, False, False, 0.1)
    r = bs.SfnnTrainStepRunner(ctx, bs.SfnnForwardHostWeights(s, **w), 1024, 1)
    c = rv.L2Calibration(s.l2_in, s.l2_size, s.num_stacks)
    for i in range(1024):
        y = np.full(s.l2_size, float(i % 2), np.float32)
        y[0] = 0.75
        c.add([0], np.zeros(s.l2_in, np.float32), y)
    old = r.read_weights(ctx)
    c.contribution.finish(old["l3w"], 1, 1, 0.01)
    assert c.candidates_for(True, False) == [0]
    assert rv.revive_l2_selected(ctx, r, c, True, False) == [0]
    new = r.read_weights(ctx)
    assert abs(new["l3b"][0] - old["l3b"][0] - 0.75 * old["l3w"][0] + 0.5 * new["l3w"][0]) < 1e-6
    np.testing.assert_array_equal(old["l0w"], new["l0w"])
    np.testing.assert_array_equal(old["l1w"], new["l1w"])
    rng = RevivalRng()
    bound = np.float32(np.sqrt(np.float32(6.0) / np.float32(s.l2_in + s.l2_size)))
    np.testing.assert_array_equal(new["l2w"][:s.l2_in], rng.signed_uniform_array(s.l2_in) * bound)
    assert new["l2b"][0] == np.float32(0.5) and abs(new["l3w"][0]) == np.float32(1 / 64)
    np.testing.assert_array_equal(new["l2w"][s.l2_in:], old["l2w"][s.l2_in:])
    assert rv.revive_l2_selected(ctx, r, c, True, False) == []
