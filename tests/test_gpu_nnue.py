"""GPU parity of the HalfKP path: the product library (through the C ABI and
the runner mirror) against the CPU oracle, the reference's golden values, and
the reference backend itself built from its sources (oracle/_ref)."""
import numpy as np
import pytest

import bulletou_b200 as bo
from bulletou_b200 import synthetic
from bulletou_b200.cuda_cpp import (NnueBackwardWorkspace, NnueForwardWorkspace, RangerDeviceState,
                                    ScalarLossWorkspace, nnue_backward_device, nnue_forward_device,
                                    scalar_loss_device)
from oracle import oracle
from tests.conftest import assert_close, assert_close_scaled

pytestmark = pytest.mark.gpu

PROD = (125388, 256, 32, 32)
FACT = (125388 + 1548, 256, 32, 32)


def host_weights(shape, w):
    return bo.NnueForwardHostWeights(bo.NnueForwardShape(*shape), **w)


@pytest.fixture(scope="module")
def prod_weights():
    return synthetic.halfkp_weights(synthetic.rng_for(11))


def _device_forward(ctx, shape, w, stm, nstm, batch, A):
    sh = bo.NnueForwardShape(*shape)
    wb = [bo.F32Buffer.from_host(ctx, a) for a in host_weights(shape, w).arrays()]
    s, n = bo.I32Buffer.from_host(ctx, stm), bo.I32Buffer.from_host(ctx, nstm)
    ws = NnueForwardWorkspace(ctx, sh, batch)
    nnue_forward_device(ctx, sh, batch, A, s, n, wb, ws)
    out = {k: getattr(ws, k).download() for k in ("stm_l0", "nstm_l0", "combined", "hidden1", "hidden2", "output")}
    return out, (sh, wb, s, n, ws)


# ---------------------------------------------------------------- forward
def test_tiny_forward_host_golden(lib, tiny, goldens):
    shape, w = tiny
    g = goldens["tiny_nnue_two_samples"]
    out = bo.nnue_forward_host(0, bo.NnueForwardShape(*shape), g["stm"], g["nstm"], 2, 3, host_weights(shape, w), lib)
    assert_close(out, g["outputs"], 0.0, g["tolerance"], "outputs")


def test_tiny_forward_trace_golden(ctx, tiny, goldens):
    shape, w = tiny
    g = goldens["tiny_nnue_trace"]
    out, _ = _device_forward(ctx, shape, w, g["stm"], g["nstm"], 1, 3)
    for key, gk in (("stm_l0", "stm_l0"), ("nstm_l0", "nstm_l0"), ("combined", "combined"), ("hidden1", "hidden1"),
                    ("hidden2", "hidden2"), ("output", "outputs")):
        assert_close(out[key], g[gk], 0.0, g["tolerance"], key)


@pytest.mark.parametrize("shape", [PROD, FACT], ids=["halfkp", "halfkp_factorized"])
def test_production_forward_bitexact_vs_oracle(ctx, prod_weights, shape):
    batch = 333  # not a multiple of the warp/CTA tiling
    b = synthetic.halfkp_batch(5, batch)
    w = dict(prod_weights)
    if shape == FACT:
        w["l0w"] = synthetic.rng_for(12).normal(0, 0.01, FACT[0] * 256).astype(np.float32)
    out, _ = _device_forward(ctx, shape, w, b["stm"], b["nstm"], batch, 38)
    ref = oracle.nnue_forward(shape, b["stm"], b["nstm"], batch, 38, w)
    for k in ref:
        assert np.array_equal(out[k], ref[k]), f"{k}: max |diff| {np.abs(out[k] - ref[k]).max():.3e}"


def test_forward_handles_padding_and_out_of_range(ctx, prod_weights):
    batch, A = 64, 40
    rng = synthetic.rng_for(21)
    stm = rng.integers(-3, PROD[0] + 50, size=batch * A).astype(np.int32)  # -1 padding and ids >= input_size
    nstm = rng.integers(-3, PROD[0] + 50, size=batch * A).astype(np.int32)
    stm[:A] = -1  # an all-padding position
    out, _ = _device_forward(ctx, PROD, prod_weights, stm, nstm, batch, A)
    ref = oracle.nnue_forward(PROD, stm, nstm, batch, A, prod_weights)
    for k in ref:
        assert np.array_equal(out[k], ref[k]), k


def test_forward_matches_reference_backend(ctx, ref_ctx, prod_weights):
    batch = 1024
    b = synthetic.halfkp_batch(6, batch)
    mine, _ = _device_forward(ctx, PROD, prod_weights, b["stm"], b["nstm"], batch, 38)
    theirs, _ = _device_forward(ref_ctx, PROD, prod_weights, b["stm"], b["nstm"], batch, 38)
    for k in mine:
        assert_close(mine[k], theirs[k], 1e-6, 1e-7, f"vs reference {k}")


# ---------------------------------------------------------------- loss
@pytest.mark.parametrize("kind,param", [(0, 0.0), (1, 0.2), (2, 0.0), (2, 1.5)])
def test_scalar_loss_vs_oracle(ctx, kind, param):
    rng = np.random.default_rng(kind * 10 + int(param))
    n = 5000
    o = rng.normal(0, 600, n).astype(np.float32)
    t = rng.random(n).astype(np.float32)
    w = rng.choice([0.0, 0.5, 1.0], n).astype(np.float32)
    kinds = {0: bo.ScalarLossKind.SigmoidPow(2.0), 1: bo.ScalarLossKind.WinRateModel(2.5, param),
             2: bo.ScalarLossKind.BceErrorWeighted(param) if param else bo.ScalarLossKind.BceWithLogits()}
    lk = kinds[kind]
    got = bo.scalar_loss_host(0, lk, 1 / 600, o, t, w, ctx.lib)
    ref = oracle.scalar_loss(kind, 1 / 600, lk.loss_pow_exp(), 0.0 if kind == 2 else param, o, t, w)
    if kind == 2 and param:
        # detached error weights (cu:2778-2788), restated in numpy double
        z = o.astype(np.float64) / 600
        err = np.abs(1 / (1 + np.exp(-z)) - t)
        mean_err = (err * w)[w > 0].sum() / w[w > 0].sum()
        wt = np.where(w == 0, 1.0, (1 + param * err) / (1 + param * mean_err))
        ref["per_sample"] = ref["per_sample"] * wt
        ref["mean_output_gradients"] = ref["mean_output_gradients"] * wt
        ref["weighted_sum"] = float(ref["per_sample"].sum())
        ref["mean"] = ref["weighted_sum"] / n
    assert_close(got.per_sample, ref["per_sample"], 2e-5, 1e-9, "per_sample")
    assert_close(got.mean_output_gradients, ref["mean_output_gradients"], 2e-5, 1e-12, "mog")
    assert got.mean == pytest.approx(ref["mean"], rel=1e-5)


def test_scalar_loss_goldens(lib, goldens):
    g = goldens["sigmoid_mse_loss"]
    r = bo.scalar_loss_host(0, bo.ScalarLossKind.SigmoidPow(2.0), 1.0, g["outputs"], g["targets"], g["weights"], lib)
    tol = g["tolerance"]
    assert_close(r.per_sample, g["per_sample"], 0.0, tol, "per_sample")
    assert_close(r.mean_output_gradients, g["mean_output_gradients"], 0.0, tol, "mog")
    assert abs(r.weighted_sum - g["weighted_sum"]) <= tol and abs(r.mean - g["mean"]) <= tol


def test_scalar_loss_rejects_bad_parameters(lib):
    with pytest.raises(bo.CudaCppError, match="loss_pow_exp"):
        bo.scalar_loss_host(0, bo.ScalarLossKind.SigmoidPow(0.5), 1.0, [0.0], [0.0], [1.0], lib)
    with pytest.raises(bo.CudaCppError, match="BCE error weight"):
        bo.scalar_loss_host(0, bo.ScalarLossKind.BceErrorWeighted(-1.0), 1.0, [0.0], [0.0], [1.0], lib)
    with pytest.raises(bo.CudaCppError, match="batch size"):
        bo.scalar_loss_host(0, bo.ScalarLossKind.SigmoidPow(2.0), 1.0, [], [], [], lib)


# ---------------------------------------------------------------- backward (drop-in ABI)
def _abi_backward(ctx, shape, w, b, batch, A, targets, entry_weights, zero=True, pre_l0w=None):
    out, (sh, wb, s, n, fws) = _device_forward(ctx, shape, w, b["stm"], b["nstm"], batch, A)
    lw = ScalarLossWorkspace(ctx, batch)
    scalar_loss_device(ctx, bo.ScalarLossKind.SigmoidPow(2.0), 1 / 600, batch, fws.output,
                       bo.F32Buffer.from_host(ctx, targets), bo.F32Buffer.from_host(ctx, entry_weights), lw)
    bws = NnueBackwardWorkspace(ctx, sh, batch)
    if pre_l0w is not None:
        bws.l0w_gradients.upload(pre_l0w)
    nnue_backward_device(ctx, sh, batch, A, s, n, wb, fws, lw.mean_output_gradients, bws, zero)
    return out, lw.download(), bws.download()


@pytest.mark.parametrize("shape", [PROD, FACT], ids=["halfkp", "halfkp_factorized"])
def test_backward_abi_vs_oracle(ctx, prod_weights, shape):
    batch = 257
    b = synthetic.halfkp_batch(8, batch)
    w = dict(prod_weights)
    if shape == FACT:
        w["l0w"] = synthetic.rng_for(13).normal(0, 0.01, FACT[0] * 256).astype(np.float32)
    pre = synthetic.rng_for(14).normal(0, 1e-4, shape[0] * 256).astype(np.float32)
    out, loss, grads = _abi_backward(ctx, shape, w, b, batch, 38, b["targets"], b["entry_weights"], zero=False,
                                     pre_l0w=pre)
    ref = oracle.nnue_backward(shape, b["stm"], b["nstm"], batch, 38, out, w, loss.mean_output_gradients, pre)
    for k in NnueBackwardWorkspace.NAMES:
        assert_close_scaled(grads[k], ref[k], 2e-6 if k in ("l0w_gradients",) else 1e-5, k)


def test_backward_abi_zero_flag_clears_accumulator(ctx, prod_weights):
    batch = 64
    b = synthetic.halfkp_batch(9, batch)
    pre = np.full(PROD[0] * 256, 7.0, np.float32)
    out, loss, grads = _abi_backward(ctx, PROD, prod_weights, b, batch, 38, b["targets"], b["entry_weights"],
                                     zero=True, pre_l0w=pre)
    ref = oracle.nnue_backward(PROD, b["stm"], b["nstm"], batch, 38, out, prod_weights, loss.mean_output_gradients)
    assert_close_scaled(grads["l0w_gradients"], ref["l0w_gradients"], 2e-6, "l0w")


def test_backward_abi_matches_reference_backend(ctx, ref_ctx, prod_weights):
    batch = 2048
    b = synthetic.halfkp_batch(10, batch)
    _, _, mine = _abi_backward(ctx, PROD, prod_weights, b, batch, 38, b["targets"], b["entry_weights"])
    _, _, theirs = _abi_backward(ref_ctx, PROD, prod_weights, b, batch, 38, b["targets"], b["entry_weights"])
    for k in NnueBackwardWorkspace.NAMES:
        # the reference sums the l0w gradient with float atomics and the dense
        # weight gradients with cuBLAS: order differs, 1e-4 / 1e-5 of scale
        assert_close_scaled(mine[k], theirs[k], 1e-4 if k == "l0w_gradients" else 1e-5, k)


# ---------------------------------------------------------------- optimizer
def test_ranger_device_vs_oracle_and_smoke_golden(ctx, goldens):
    g = goldens["smoke_ranger"]
    params = bo.RangerUpdateParams(radam=bo.RAdamUpdateParams(step=1, learning_rate=0.01, min_weight=-1.98,
                                                              max_weight=1.98))
    st = RangerDeviceState(*[bo.F32Buffer.from_host(ctx, a) for a in
                             (g["gradients"], g["weights"], [0.0] * 4, [0.0] * 4, g["weights"])])
    bo.ranger_update_device(ctx, params, st)
    grads, w = st.gradients.download(), st.weights.download()
    assert np.all(grads == 0.0)
    og = np.array(g["gradients"], np.float32)
    ow = np.array(g["weights"], np.float32)
    oracle.ranger_update(og, ow, np.zeros(4, np.float32), np.zeros(4, np.float32), ow.copy(), step=1,
                         learning_rate=0.01, min_weight=-1.98, max_weight=1.98)
    assert_close(w, ow, 1e-6, 0.0, "weights")
    # host entry gives the device result (smoke.rs:218-273)
    hw = np.array(g["weights"], np.float32)
    bo.ranger_update_host(0, params, np.array(g["gradients"], np.float32), hw, np.zeros(4, np.float32),
                          np.zeros(4, np.float32), hw.copy(), ctx.lib)
    assert np.array_equal(hw, w)


@pytest.mark.parametrize("n", [1000, 1 << 14, (1 << 14) + 3])
@pytest.mark.parametrize("step", [1, 5, 6, 7, 12])
def test_ranger_device_vs_oracle_random(ctx, n, step):
    rng = np.random.default_rng(step * 7 + n)
    arrs = [rng.normal(0, s, n).astype(np.float32) for s in (1e-2, 0.05, 1e-3, 1e-5, 0.05)]
    arrs[3] = np.abs(arrs[3])
    params = bo.RangerUpdateParams(radam=bo.RAdamUpdateParams(step=step, learning_rate=1e-3, decay=1e-4,
                                                              min_weight=-0.1, max_weight=0.1))
    st = RangerDeviceState(*[bo.F32Buffer.from_host(ctx, a) for a in arrs])
    bo.ranger_update_device(ctx, params, st)
    oracle.ranger_update(*arrs, step=step, learning_rate=1e-3, decay=1e-4, min_weight=-0.1, max_weight=0.1)
    # EMA updates cancel (m = b1*m + (1-b1)*g); GPU FMA contraction vs the
    # oracle's separate roundings differ by ~1 ulp of the *terms*, so the bound
    # is relative to the tensor's scale.
    for name, buf, ref in zip(("grad", "w", "m", "v", "slow"), (st.gradients, st.weights, st.momentum, st.velocity,
                                                                st.slow_params), arrs):
        assert_close_scaled(buf.download(), ref, 2e-6, name)


def test_zero_radam_skip_bitwise_vs_reference(ctx, ref_ctx, goldens):
    """lib.rs:11112 pattern: quiet coordinates are skipped bit-identically."""
    g = goldens["zero_radam_skip"]
    n = g["n"]
    w = (np.float32(0.1) + np.arange(n, dtype=np.float32) * np.float32(0.002)).astype(np.float32)
    w[4], w[8], w[12] = 2.0, -0.0, np.float32(np.finfo(np.float32).smallest_subnormal)
    gr = np.zeros(n, np.float32)
    gr[16], gr[20] = -0.0, 0.1
    m = np.zeros(n, np.float32)
    m[24] = 0.2
    v = np.zeros(n, np.float32)
    v[28] = 0.3
    for step in g["steps"]:
        res = []
        for c in (ctx, ref_ctx):
            st = RangerDeviceState(*[bo.F32Buffer.from_host(c, a) for a in (gr, w, m, v, w)])
            params = bo.RangerUpdateParams(radam=bo.RAdamUpdateParams(step=step, min_weight=g["min_weight"],
                                                                      max_weight=g["max_weight"]))
            bo.ranger_update_device(c, params, st)
            res.append([x.download().view(np.uint32) for x in (st.weights, st.gradients, st.momentum, st.velocity,
                                                                st.slow_params)])
        for a, b_ in zip(*res):
            assert np.array_equal(a, b_), f"step {step}"


# ---------------------------------------------------------------- train step
def _batch_obj(b):
    return bo.NnueTrainStepHostBatch(b["stm"], b["nstm"], b["targets"], b["entry_weights"], b["batch"],
                                     b["max_active"])


def _ranger(step, **kw):
    return bo.RangerUpdateParams(radam=bo.RAdamUpdateParams(step=step, learning_rate=kw.get("lr", 1e-3),
                                                            min_weight=kw.get("lo", -bo.FLT_MAX),
                                                            max_weight=kw.get("hi", bo.FLT_MAX)))


def test_tiny_train_step_fused_vs_oracle(ctx, tiny, goldens):
    shape, w = tiny
    g = goldens["tiny_nnue_two_samples"]
    bb = goldens["smoke_backward_batch"]
    runner = bo.NnueTrainStepRunner(ctx, host_weights(shape, w), 2, 3)
    assert runner.fused
    tr = oracle.NnueTrainer(shape, w)
    batch = bo.NnueTrainStepHostBatch(g["stm"], g["nstm"], bb["targets"], bb["entry_weights"], 2, 3)
    for step in range(1, 8):
        loss = runner.step(ctx, _ranger(step, lr=0.01, lo=-1.98, hi=1.98), bo.ScalarLossKind.SigmoidPow(2.0), 1.0,
                           batch)
        ref = tr.step(g["stm"], g["nstm"], 2, 3, bb["targets"], bb["entry_weights"], step=step, learning_rate=0.01,
                      min_weight=-1.98, max_weight=1.98)
        assert loss.mean == pytest.approx(ref["loss"]["mean"], rel=1e-5, abs=1e-7)
        got = runner.read_weights(ctx)
        for k in oracle.NAMES:
            assert_close(got[k], tr.w[k], 1e-5, 1e-7, f"step {step} {k}")


@pytest.mark.parametrize("shape", [PROD, FACT], ids=["halfkp", "halfkp_factorized"])
def test_production_train_steps_fused_vs_oracle(ctx, prod_weights, shape):
    batch = 512
    w = dict(prod_weights)
    if shape == FACT:
        w["l0w"] = synthetic.rng_for(15).normal(0, 0.01, FACT[0] * 256).astype(np.float32)
    runner = bo.NnueTrainStepRunner(ctx, host_weights(shape, w), batch, 38)
    tr = oracle.NnueTrainer(shape, w)
    for step in range(1, 7):  # includes the lookahead step 6
        b = synthetic.halfkp_batch(100 + step, batch)
        loss = runner.step(ctx, _ranger(step), bo.ScalarLossKind.SigmoidPow(2.0), 1 / 600, _batch_obj(b))
        ref = tr.step(b["stm"], b["nstm"], batch, 38, b["targets"], b["entry_weights"], step=step, inv_scale=1 / 600)
        assert loss.mean == pytest.approx(ref["loss"]["mean"], rel=1e-5)
        assert_close(runner.read_output(ctx), ref["forward"]["output"], 1e-4, 1e-6, f"step {step} output")
    got = runner.read_weights(ctx)
    states = runner.read_optimizer_states(ctx)
    for k in oracle.NAMES:
        assert_close_scaled(got[k], tr.w[k], 1e-4, f"weights {k}")
        assert_close_scaled(states[k]["momentum"], tr.m[k], 1e-3, f"momentum {k}")
        assert_close_scaled(states[k]["slow_params"], tr.slow[k], 1e-4, f"slow {k}")


def test_unfused_runner_matches_fused(ctx, prod_weights):
    batch = 1024
    fused = bo.NnueTrainStepRunner(ctx, host_weights(PROD, prod_weights), batch, 38, fused=True)
    plain = bo.NnueTrainStepRunner(ctx, host_weights(PROD, prod_weights), batch, 38, fused=False)
    for step in range(1, 4):
        b = synthetic.halfkp_batch(200 + step, batch)
        lf = fused.step(ctx, _ranger(step), bo.ScalarLossKind.SigmoidPow(2.0), 1 / 600, _batch_obj(b))
        lp = plain.step(ctx, _ranger(step), bo.ScalarLossKind.SigmoidPow(2.0), 1 / 600, _batch_obj(b))
        assert lf.mean == pytest.approx(lp.mean, rel=1e-6)
    wf, wp = fused.read_weights(ctx), plain.read_weights(ctx)
    for k in oracle.NAMES:
        assert_close_scaled(wf[k], wp[k], 1e-5, k)


def test_100_step_weights_match_reference_backend(ctx, ref_ctx, prod_weights):
    """BASELINE parity bar: weights after 100 steps within 1e-3 of the
    reference backend's, on identical seeded batches (B=16384)."""
    batch = 16384
    mine = bo.NnueTrainStepRunner(ctx, host_weights(PROD, prod_weights), batch, 38)
    theirs = bo.NnueTrainStepRunner(ref_ctx, host_weights(PROD, prod_weights), batch, 38)
    batches = [synthetic.halfkp_batch(300 + i, batch) for i in range(10)]
    loss_kind = bo.ScalarLossKind.SigmoidPow(2.0)
    for step in range(1, 101):
        hb = _batch_obj(batches[step % len(batches)])
        mine.step_no_readback(ctx, _ranger(step), loss_kind, 1 / 600, hb)
        theirs.step_no_readback(ref_ctx, _ranger(step), loss_kind, 1 / 600, hb)
    lm, lt = mine.read_loss(ctx), theirs.read_loss(ref_ctx)
    assert lm.mean == pytest.approx(lt.mean, rel=1e-3)
    wm, wt = mine.read_weights(ctx), theirs.read_weights(ref_ctx)
    for k in oracle.NAMES:
        diff = np.abs(wm[k].astype(np.float64) - wt[k])
        assert diff.max() <= 1e-3, f"{k}: max |diff| {diff.max():.3e}"
        rel = np.linalg.norm(wm[k] - wt[k]) / max(np.linalg.norm(wt[k]), 1e-30)
        assert rel <= 1e-3, f"{k}: relative L2 diff {rel:.3e}"


def test_train_step_rejects_bad_layout(ctx, tiny):
    shape, w = tiny
    runner = bo.NnueTrainStepRunner(ctx, host_weights(shape, w), 2, 3)
    bad = bo.NnueTrainStepHostBatch([0, 1, 2], [0, 1, 2], [0.5], [1.0], 1, 3)
    with pytest.raises(bo.CudaCppError, match="layout mismatch"):
        runner.step(ctx, _ranger(1), bo.ScalarLossKind.SigmoidPow(2.0), 1.0, bad)


def test_buffer_validation_errors(ctx, lib):
    import ctypes

    small = bo.F32Buffer(ctx, 3)
    other = bo.F32Buffer(ctx, 3)
    out = bo.F32Buffer(ctx, 2)
    with pytest.raises(bo.CudaCppError, match="smaller than requested"):
        lib.call("bulletou_cuda_cpp_axpy_device", ctx.as_ptr(), 3, 1.0, small.as_ptr(), other.as_ptr(), out.as_ptr())
    with pytest.raises(bo.CudaCppError, match="must not be null"):
        lib.call("bulletou_cuda_cpp_axpy_device", ctx.as_ptr(), 3, 1.0, None, other.as_ptr(), small.as_ptr())
    assert bo.cuda_cpp.axpy_host(0, 2.0, [1, 2, 3, 4], [10, 20, 30, 40], lib).tolist() == [12, 24, 36, 48]
    assert ctypes is not None
