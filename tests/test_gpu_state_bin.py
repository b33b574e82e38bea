"""Resume from state.bin on the GPU: a run checkpointed after three steps and
restored into a fresh runner continues exactly as the uninterrupted run
(the reference's resume-equivalence test, crates/cuda_cpp/src/lib.rs:13857),
and the checkpoint's nn.bin is the device quantisation of the saved weights."""
import numpy as np
import pytest

import bulletou_b200 as bo
from bulletou_b200 import nn_bin as nb
from bulletou_b200 import sfnn as bs
from bulletou_b200 import state_bin as sb
from bulletou_b200 import synthetic as syn
from bulletou_b200 import teacher as bt
from oracle import oracle

pytestmark = pytest.mark.gpu


def _ranger(step):
    return bo.RangerUpdateParams(radam=bo.RAdamUpdateParams(step=step, learning_rate=1e-3))


def test_sfnn_checkpoint_resume_is_exact(ctx, tmp_path):
    shape = bs.SfnnForwardShape(bs.HALFKA_HM2_DIMENSIONS + bs.PIECE_INPUTS, 256, 15, True, 32, 9)
    w = syn.sfnn_weights(syn.rng_for(8), shape.input_size, shape.ft_size, shape.l1_hidden, shape.l1_skip,
                         shape.l2_size, shape.num_stacks, True, True, 0.05)
    other = syn.sfnn_weights(syn.rng_for(9), shape.input_size, shape.ft_size, shape.l1_hidden, shape.l1_skip,
                             shape.l2_size, shape.num_stacks, True, True, 0.05)
    B = 1024
    cfg = bt.TeacherBatchConfig(feature_set="halfka_hm2", lambda_=1.0, scale=600.0, win_rate_model=True)
    prod = bt.TeacherBatchProducer(ctx, cfg, B, pinned=False)
    loss = bo.ScalarLossKind.SigmoidPow(2.0)
    batches = [syn.psv_records(200 + i, B) for i in range(6)]
    full = bs.SfnnTrainStepRunner(ctx, bs.SfnnForwardHostWeights(shape, **w), B, 40, bs.SfnnFactorizerAlpha(0.75, 1.25))
    part = bs.SfnnTrainStepRunner(ctx, bs.SfnnForwardHostWeights(shape, **w), B, 40, bs.SfnnFactorizerAlpha(0.75, 1.25))
    for step, recs in enumerate(batches, 1):
        full.step_from_records(ctx, _ranger(step), loss, 1 / 600, prod, recs)
    for step, recs in enumerate(batches[:3], 1):
        part.step_from_records(ctx, _ranger(step), loss, 1 / 600, prod, recs)
    dq = bs.QuantizedSfnnDeviceWeights(ctx, shape)
    log = sb.CheckpointLog(1, 3, 3, 3 * B, 1e-3, 1e-3, 1.0, dataloader_byte_offset=3 * B * 40)
    d = sb.write_sfnn_checkpoint(tmp_path, ctx, part, log, 3, 3, dq)
    assert sb.latest_complete_checkpoint_dir(tmp_path) == d
    saved = part.read_weights(ctx)
    want = nb.sfnn_nn_bin_bytes(oracle.sfnn_quantize(shape.as_tuple(), saved, 0.75, 1.25), shape.ft_size,
                                shape.l1_out, shape.l2_size, shape.l2_in, shape.num_stacks)
    assert (d / "nn.bin").read_bytes() == want

    resumed = bs.SfnnTrainStepRunner(ctx, bs.SfnnForwardHostWeights(shape, **other), B, 40,
                                     bs.SfnnFactorizerAlpha(0.75, 1.25))
    st = sb.load_sfnn_state(d / "state.bin", sb.sfnn_runner_sizes(resumed))
    assert (st.completed_steps, st.optimizer_steps, st.shared_coefficients) == (3, 3, (0.75, 1.25))
    sb.restore_sfnn_runner(ctx, resumed, st)
    for step, recs in enumerate(batches[3:], st.optimizer_steps + 1):
        resumed.step_from_records(ctx, _ranger(step), loss, 1 / 600, prod, recs)
    assert resumed.read_loss(ctx).mean == full.read_loss(ctx).mean
    wf, wr = full.read_weights(ctx), resumed.read_weights(ctx)
    of, orr = full.read_optimizer_states(ctx), resumed.read_optimizer_states(ctx)
    for k in wf:
        np.testing.assert_array_equal(wr[k], wf[k], err_msg=k)
        for s in ("momentum", "velocity", "slow_params"):
            np.testing.assert_array_equal(orr[k][s], of[k][s], err_msg=f"{k} {s}")


def test_halfkp_state_resume(ctx, tmp_path):
    w = syn.halfkp_weights(syn.rng_for(21))
    w2 = syn.halfkp_weights(syn.rng_for(22))
    B = 512
    mk = lambda ww: bo.NnueTrainStepRunner(ctx, bo.NnueForwardHostWeights(bo.NNUE_HALFKP_256X2_32_32, **ww), B, 38)
    full, part, resumed = mk(w), mk(w), mk(w2)
    loss = bo.ScalarLossKind.SigmoidPow(2.0)
    batches = [syn.halfkp_batch(300 + i, B) for i in range(7)]

    def hb(b):
        return bo.NnueTrainStepHostBatch(b["stm"], b["nstm"], b["targets"], b["entry_weights"], B, 38)

    for step, b in enumerate(batches, 1):
        full.step_no_readback(ctx, _ranger(step), loss, 1 / 600, hb(b))
    for step, b in enumerate(batches[:4], 1):
        part.step_no_readback(ctx, _ranger(step), loss, 1 / 600, hb(b))
    hs = bo.NNUE_HALFKP_256X2_32_32
    shape = (hs.input_size, hs.l1, hs.l2, hs.l3)
    dq = bo.QuantizedNnueDeviceWeights(ctx, *shape)
    log = sb.CheckpointLog(1, 4, 4, 4 * B, 1e-3, 1e-3, 0.5, eval_name="halfkp_256x2-32-32")
    d = sb.write_halfkp_checkpoint(tmp_path, ctx, part, log, 4, dq)
    assert sb.is_complete_checkpoint_dir(d) and sb.latest_complete_checkpoint_dir(tmp_path) == d
    saved = part.read_weights(ctx)
    assert (d / "nn.bin").read_bytes() == nb.nnue_nn_bin_bytes(oracle.nnue_quantize(shape, saved), *shape[1:])
    weights, opt, done = sb.load_halfkp_state(d / "state.bin", sb.halfkp_runner_sizes(resumed))
    assert done == 4
    sb.restore_halfkp_runner(ctx, resumed, weights, opt)
    for step, b in enumerate(batches[4:], done + 1):
        resumed.step_no_readback(ctx, _ranger(step), loss, 1 / 600, hb(b))
    wf, wr = full.read_weights(ctx), resumed.read_weights(ctx)
    for k in wf:
        scale = max(float(np.abs(wf[k]).max()), 1e-30)
        err = float(np.abs(wr[k].astype(np.float64) - wf[k]).max())
        assert err <= 1e-6 * scale, f"{k}: max |diff| {err:.3e} (scale {scale:.3e})"
