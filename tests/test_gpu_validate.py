"""GPU parity of the validation row: the device metrics
(bulletou_b200_validation_metrics_device) against the oracle restatement of
compute_sign_accuracy_with_loss_masked (validate.rs:353-470) on decoded
records -- counts exact, test loss within 2e-6 relative (f32 per-sample
losses summed in double in another order) -- and the reference-ABI statistics
entries (bulletou_cuda_cpp_sfnn_validation_stats / _unit_stats) against the
reference backend."""
import numpy as np
import pytest

import bulletou_b200 as bo
from bulletou_b200 import sfnn as bs
from bulletou_b200 import synthetic as syn
from bulletou_b200 import teacher as bt
from bulletou_b200 import validate as bv
from oracle import teacher as ot

pytestmark = pytest.mark.gpu

KINDS = {"sigmoid_pow": bv.ValidationLossKind.sigmoid_pow(2.0),
         "sigmoid_pow_2.5": bv.ValidationLossKind.sigmoid_pow(2.5),
         "win_rate_model": bv.ValidationLossKind.win_rate_model(2.0, 600.0, 270.0, 380.0),
         "bce": bv.ValidationLossKind.bce_with_logits(600.0, 340.0, bt.WinRateModelTargetParams(135.0, 380.0, 0.05))}
KIND_ID = {"sigmoid_pow": 0, "win_rate_model": 1, "bce_with_logits": 2}


def _records(seed, n):
    recs = syn.psv_records(seed, n)
    rng = np.random.default_rng(seed)
    recs["score"][rng.random(n) < 0.02] = 32000      # mate stamps for the score cap
    return recs.view(np.uint8).reshape(n, 40)


def _scores_results(recs):
    r = np.ascontiguousarray(recs).view(syn.PSV_DTYPE).reshape(-1)
    return r["score"].copy(), r["game_result"].copy()


@pytest.mark.parametrize("name", list(KINDS))
@pytest.mark.parametrize("cap", [None, 30000])
def test_validation_metrics_vs_oracle(ctx, name, cap):
    n = 50000
    recs = _records(7, n)
    outputs = np.random.default_rng(8).normal(0, 1.2, n).astype(np.float32)
    outputs[::97] = 0.0
    kind = KINDS[name]
    vm = bv.ValidationMetrics(ctx, kind)
    rep = vm.compute(ctx, bo.F32Buffer.from_host(ctx, outputs), bo.I32Buffer.from_host(ctx, np.ascontiguousarray(recs).view(np.int32)), n,
                     lambda_=0.7, eval_scale=600.0, score_drop_abs=cap)
    scores, results = _scores_results(recs)
    want = ot.validation_metrics(outputs, scores, results, score_drop_abs=cap, lambda_=0.7, eval_scale=600.0,
                                 loss_kind=KIND_ID[kind.kind], pow_exp=kind.pow_exp, nnue2score=kind.nnue2score,
                                 in_offset=kind.in_offset, in_scaling=kind.in_scaling,
                                 wrm_table=None if kind.kind == "sigmoid_pow" else
                                 bt.win_rate_model_score_table(kind.target))
    for k in ot.VALIDATION_COUNTS:
        assert getattr(rep, k) == want[k], k
    assert rep.test_loss == pytest.approx(want["test_loss"], rel=2e-6)
    if cap is not None:
        assert rep.filtered_by_score_cap > 0


def test_score_sign_path_and_empty(ctx):
    n = 1000
    recs = _records(9, n)
    outputs = np.random.default_rng(10).normal(0, 1, n).astype(np.float32)
    vm = bv.ValidationMetrics(ctx)
    rep = vm.compute(ctx, bo.F32Buffer.from_host(ctx, outputs), bo.I32Buffer.from_host(ctx, np.ascontiguousarray(recs).view(np.int32)), n,
                     have_results=False)
    want = ot.validation_metrics(outputs, _scores_results(recs)[0], None)
    for k in ot.VALIDATION_COUNTS:
        assert getattr(rep, k) == want[k], k
    assert rep.test_loss is None and rep.loss_sampled == 0
    empty = vm.compute(ctx, bo.F32Buffer.from_host(ctx, outputs), bo.I32Buffer.from_host(ctx, np.ascontiguousarray(recs).view(np.int32)), 0)
    assert empty.compared == 0 and np.isnan(empty.accuracy()) and empty.test_loss is None


def _forward(ctx, shape, w, recs, B):
    cfg = bt.TeacherBatchConfig(lambda_=1.0, win_rate_model=True)
    prod = bt.TeacherBatchProducer(ctx, cfg, B, pinned=False)
    tb = prod.new_batch()
    prod.prepare(ctx, recs, tb)
    dev = {k: (None if v is None else bo.F32Buffer.from_host(ctx, v)) for k, v in
           bs.SfnnForwardHostWeights(shape, **w).arrays().items()}
    ws = bs.SfnnForwardWorkspace(ctx, shape, B)
    bs.sfnn_forward_device(ctx, shape, B, 40, tb.stm_indices, tb.nstm_indices, tb.buckets, dev, ws)
    return ws, tb


def test_validation_stats_entries_vs_reference_backend(ctx, ref_ctx):
    """Held-out forward over decoded records, then the two statistics entries
    on both libraries over the same activations."""
    shape = bs.SfnnForwardShape(bs.HALFKA_HM2_DIMENSIONS + bs.PIECE_INPUTS, 256, 15, True, 32, 9)
    w = syn.sfnn_weights(syn.rng_for(12), shape.input_size, shape.ft_size, shape.l1_hidden, shape.l1_skip,
                         shape.l2_size, shape.num_stacks, True, False, 0.3)
    w["l0b"] = (np.abs(w["l0b"]) + 0.6).astype(np.float32)
    B = 4096
    recs = syn.psv_records(13, B)
    ws, tb = _forward(ctx, shape, w, recs, B)
    acts = ws.download(ctx)
    buckets = tb.buckets.download(ctx)
    L = shape.l1_hidden
    stride = 1 + 2 * L + shape.l2_size
    results = []
    for c in (ctx, ref_ctx):
        bufs = {k: bo.F32Buffer.from_host(c, v) for k, v in acts.items()}
        partials = bo.F32Buffer(c, 1280)
        c.lib.call("bulletou_cuda_cpp_sfnn_validation_stats", c.as_ptr(), bufs["stm_l0"].as_ptr(),
                   bufs["nstm_l0"].as_ptr(), bufs["l2_input"].as_ptr(), bufs["l2"].as_ptr(), bufs["output"].as_ptr(),
                   partials.as_ptr(), B, shape.ft_size, L, shape.l2_size)
        counts = bo.I32Buffer(c, shape.ft_size + shape.num_stacks * stride)
        bucket_buf = bo.I32Buffer.from_host(c, buckets)          # kept alive across the call
        c.lib.call("bulletou_cuda_cpp_sfnn_unit_stats", c.as_ptr(), bufs["stm_l0"].as_ptr(), bufs["nstm_l0"].as_ptr(),
                   bufs["l2_input"].as_ptr(), bufs["l2"].as_ptr(), bucket_buf.as_ptr(),
                   counts.as_ptr(), B, shape.ft_size, L, shape.l2_size, shape.num_stacks)
        results.append((partials.download(c), counts.download(c)))
    np.testing.assert_array_equal(results[0][0], results[1][0])
    np.testing.assert_array_equal(results[0][1], results[1][1])
    p = results[0][0].reshape(5, 256).astype(np.float64).sum(axis=1)
    assert p[0] == (acts["stm_l0"] >= 1).sum() + (acts["nstm_l0"] >= 1).sum() and p[0] > 0
    assert p[4] == pytest.approx(float((acts["output"].astype(np.float64) ** 2).sum()), rel=1e-5)
    assert bv.sfnn_validation_stats(ctx, ws, bo.F32Buffer(ctx, 1280)) == pytest.approx(p.tolist())


def test_validation_of_a_trained_net_on_records(ctx):
    """The held-out path end to end: records decoded on the device, forward,
    metrics -- against the oracle's metrics over the same outputs."""
    shape = bs.SfnnForwardShape(bs.HALFKA_HM2_DIMENSIONS + bs.PIECE_INPUTS, 256, 15, True, 32, 9)
    w = syn.sfnn_weights(syn.rng_for(14), shape.input_size, shape.ft_size, shape.l1_hidden, shape.l1_skip,
                         shape.l2_size, shape.num_stacks, True, False, 0.1)
    B = 8192
    recs = syn.psv_records(15, B)
    ws, _ = _forward(ctx, shape, w, recs, B)
    vm = bv.ValidationMetrics(ctx, KINDS["win_rate_model"])
    rec_buf = bo.I32Buffer.from_host(ctx, np.ascontiguousarray(recs).view(np.int32))
    rep = vm.compute(ctx, ws.output, rec_buf, B, lambda_=1.0, eval_scale=600.0, model_output_scale=1.0)
    out = ws.output.download(ctx)
    sc, res = _scores_results(recs)
    want = ot.validation_metrics(out, sc, res,
                                 lambda_=1.0, eval_scale=600.0, loss_kind=1, wrm_table=bt.win_rate_model_score_table(
                                     bt.WinRateModelTargetParams()))
    assert rep.compared == want["compared"] and rep.sign_matches == want["sign_matches"]
    assert rep.test_loss == pytest.approx(want["test_loss"], rel=2e-6)
