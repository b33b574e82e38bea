"""GPU parity of SFNN quantisation-aware training (row a10): the fused step of
the product library with each QAT mode against the CPU oracle, the product's
reference-ABI sequence (bulletou_layer_qat, bulletou_dense_qat_begin/_end and
the L1 QAT scratch of the forward / backward entries) against the reference
backend, and the fused step against the reference backend at the production
shape."""
import numpy as np
import pytest

import bulletou_b200 as bo
from bulletou_b200 import sfnn as bs
from bulletou_b200 import synthetic
from oracle import oracle
from tests.conftest import assert_close_scaled

pytestmark = pytest.mark.gpu

HM2F = bs.HALFKA_HM2_DIMENSIONS + bs.PIECE_INPUTS
PROD = bs.SFNN_HALFKA_HM2_1536_15_32_K3K3
SMALL = bs.SfnnForwardShape(HM2F, 256, 15, True, 32, 9)
MID = bs.SfnnForwardShape(HM2F, 512, 15, True, 32, 9)               # warp integer-FT kernel
GENERIC = bs.SfnnForwardShape(HM2F, 12, 3, True, 5, 4)

MODES = {
    "l1": bs.SfnnLayerLrMultipliers(qat_l1=True),
    "ft": bs.SfnnLayerLrMultipliers(qat_ft=True),
    "l2l3": bs.SfnnLayerLrMultipliers(qat_l2=True, qat_l3=True),
    "ft_l1_l2": bs.SfnnLayerLrMultipliers(qat_ft=True, qat_l1=True, qat_l2=True),
    "dense": bs.SfnnLayerLrMultipliers(qat_l1=True, qat_l2=True, qat_l3=True),
    "dense_ft": bs.SfnnLayerLrMultipliers(qat_l1=True, qat_ft=True, qat_l2=True, qat_l3=True),
}


def _mask(lr):
    return oracle.qat_mask(lr.qat_l1, lr.qat_ft, lr.qat_l2, lr.qat_l3)


def _weights(shape, seed, std=0.05):
    w = synthetic.sfnn_weights(synthetic.rng_for(seed), shape.input_size, shape.ft_size, shape.l1_hidden,
                               shape.l1_skip, shape.l2_size, shape.num_stacks, True, False, std)
    w["l0b"] = (np.abs(w["l0b"]) + 0.25).astype(np.float32)     # FT outputs inside (0, 1)
    w["l1w"] = (w["l1w"] * 8).astype(np.float32)               # L1 sums across the activation ranges
    return w


def _batch(seed, batch, stacks, pad=False):
    b = synthetic.sfnn_batch(seed, batch, stacks=stacks)
    if pad:
        rng = np.random.default_rng(seed)
        for key in ("stm", "nstm"):
            b[key][rng.random(b[key].size) < 0.05] = -1
        b["buckets"][5] = stacks                               # invalid bucket
    return b


def _host_weights(shape, w):
    return bs.SfnnForwardHostWeights(shape, **w)


def _host_batch(b):
    return bs.SfnnTrainStepHostBatch(b["stm"], b["nstm"], b["buckets"], b["targets"], b["entry_weights"], b["batch"],
                                     b["max_active"])


def _params(step, lr=1e-3):
    return bo.RangerUpdateParams(radam=bo.RAdamUpdateParams(step=step, learning_rate=lr))


@pytest.mark.parametrize("mode", list(MODES))
@pytest.mark.parametrize("shape", [SMALL, MID, GENERIC], ids=["small", "mid", "generic"])
def test_fused_qat_steps_vs_oracle(ctx, mode, shape):
    lr = MODES[mode]
    w = _weights(shape, 11)
    B = 256
    runner = bs.SfnnTrainStepRunner(ctx, _host_weights(shape, w), B, 40, lr_multipliers=lr)
    assert runner.fused
    trainer = oracle.SfnnTrainer(shape.as_tuple(), w, qat=_mask(lr))
    for step in range(1, 6):
        b = _batch(40 + step, B, shape.num_stacks, pad=True)
        runner.step_no_readback(ctx, _params(step), bo.ScalarLossKind.SigmoidPow(2.0), 1 / 600, _host_batch(b))
        res = trainer.step(b["stm"], b["nstm"], b["buckets"], B, 40, b["targets"], b["entry_weights"], step=step,
                           learning_rate=1e-3, inv_scale=1 / 600)
        if step == 1:
            out = runner.read_output(ctx)
            if lr.dense_qat:
                # integer L1 / L2 / L3 over bit-identical FT outputs: the same numbers
                np.testing.assert_array_equal(out, res["forward"]["output"])
            else:
                assert_close_scaled(out, res["forward"]["output"], 1e-5, "output")
    got = runner.read_weights(ctx)
    for nm in trainer.names:
        assert_close_scaled(got[nm], trainer.w[nm], 1e-4, nm)


@pytest.mark.parametrize("mode", list(MODES))
def test_reference_abi_qat_sequence_vs_reference_backend(ctx, ref_ctx, mode):
    """The runner's reference call sequence (layer-QAT copies, dense-QAT
    bracket, L1 QAT scratch) bound to this library and to the reference backend."""
    lr = MODES[mode]
    shape = SMALL
    w = _weights(shape, 13)
    B = 512
    ours = bs.SfnnTrainStepRunner(ctx, _host_weights(shape, w), B, 40, fused=False, lr_multipliers=lr)
    ref = bs.SfnnTrainStepRunner(ref_ctx, _host_weights(shape, w), B, 40, lr_multipliers=lr)
    assert not ours.fused and not ref.fused
    for step in range(1, 4):
        hb = _host_batch(_batch(60 + step, B, shape.num_stacks))
        for r, c in ((ours, ctx), (ref, ref_ctx)):
            r.step_no_readback(c, _params(step), bo.ScalarLossKind.SigmoidPow(2.0), 1 / 600, hb)
        if step == 1:
            a, c = ours.read_output(ctx), ref.read_output(ref_ctx)
            if lr.dense_qat:
                np.testing.assert_array_equal(a, c)
            else:
                assert_close_scaled(a, c, 1e-5, "output")
            if lr.qat_l1:
                np.testing.assert_array_equal(ours.qat_l1.weights.download(ctx), ref.qat_l1.weights.download(ref_ctx))
                np.testing.assert_array_equal(ours.qat_l1.bias.download(ctx), ref.qat_l1.bias.download(ref_ctx))
    a, c = ours.read_weights(ctx), ref.read_weights(ref_ctx)
    for nm in a:
        assert_close_scaled(a[nm], c[nm], 1e-5, nm)


def test_layer_qat_entry_vs_reference_backend(ctx, ref_ctx):
    rng = np.random.default_rng(3)
    base, vr, W = 73305, 1629, 16
    src = rng.normal(0, 0.3, (base + vr) * W).astype(np.float32)
    src[:8] = [0.5 / 127, -0.5 / 127, 1.5 / 127, 300.0, -300.0, 2.5 / 64, -2.5 / 64, 0.0]
    for scale, rows in ((127.0, vr), (127.0, 0), (64.0, 0), (8128.0, 0)):
        outs = []
        for c in (ctx, ref_ctx):
            s = bo.F32Buffer.from_host(c, src)
            d = bo.F32Buffer(c, src.size)
            c.lib.call("bulletou_layer_qat", c.as_ptr(), s.as_ptr(), d.as_ptr(), scale, 0.0, 0.0,
                       base if rows else 0, rows, W if rows else 0, 0.75)
            outs.append(d.download(c))
        np.testing.assert_array_equal(outs[0], outs[1], err_msg=f"scale {scale} rows {rows}")


@pytest.mark.parametrize("mode", ["l1", "dense", "dense_ft"])
def test_fused_qat_prod_vs_reference_backend(ctx, ref_ctx, mode):
    """Production shape, 20 steps: weights within 1e-3 of the reference backend."""
    lr = MODES[mode]
    shape = PROD
    w = _weights(shape, 17, std=0.01)
    B = 2048
    ours = bs.SfnnTrainStepRunner(ctx, _host_weights(shape, w), B, 40, lr_multipliers=lr)
    ref = bs.SfnnTrainStepRunner(ref_ctx, _host_weights(shape, w), B, 40, lr_multipliers=lr)
    assert ours.fused and not ref.fused
    batches = [_host_batch(_batch(400 + i, B, shape.num_stacks)) for i in range(5)]
    for step in range(1, 21):
        hb = batches[step % len(batches)]
        for r, c in ((ours, ctx), (ref, ref_ctx)):
            r.step_no_readback(c, _params(step), bo.ScalarLossKind.SigmoidPow(2.0), 1 / 600, hb)
    a, c = ours.read_weights(ctx), ref.read_weights(ref_ctx)
    for nm in a:
        err = float(np.abs(a[nm].astype(np.float64) - c[nm]).max())
        assert err <= 1e-3, f"{nm}: max |diff| {err:.3e} after 20 steps"
    la, lr_ = ours.read_loss(ctx), ref.read_loss(ref_ctx)
    assert abs(la.mean - lr_.mean) <= 1e-4 * max(1.0, abs(lr_.mean))


def test_dense_qat_rejects_l2_shared_factor(ctx):
    shape = SMALL
    w = synthetic.sfnn_weights(synthetic.rng_for(5), shape.input_size, shape.ft_size, shape.l1_hidden,
                               shape.l1_skip, shape.l2_size, shape.num_stacks, True, True, 0.05)
    runner = bs.SfnnTrainStepRunner(ctx, _host_weights(shape, w), 64, 40, lr_multipliers=MODES["dense"])
    b = _batch(1, 64, shape.num_stacks)
    with pytest.raises(bo.CudaCppError, match="L2/L3"):
        runner.step_no_readback(ctx, _params(1), bo.ScalarLossKind.SigmoidPow(2.0), 1 / 600, _host_batch(b))
