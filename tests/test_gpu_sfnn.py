"""GPU parity of the SFNN LayerStack path: the product library (reference C-ABI
entries, the fused step and the runner mirror) against the CPU oracle, the
reference's golden values, and the reference backend built from its sources."""
import numpy as np
import pytest

import bulletou_b200 as bo
from bulletou_b200 import sfnn as bs
from bulletou_b200 import synthetic
from bulletou_b200.cuda_cpp import ScalarLossWorkspace, scalar_loss_device
from oracle import oracle
from tests.conftest import assert_close, assert_close_scaled

pytestmark = pytest.mark.gpu

HM2F = bs.HALFKA_HM2_DIMENSIONS + bs.PIECE_INPUTS
PROD = bs.SFNN_HALFKA_HM2_1536_15_32_K3K3
SMALL = bs.SfnnForwardShape(HM2F, 256, 15, True, 32, 9)          # fast kernels, small table
GENERIC = bs.SfnnForwardShape(HM2F, 12, 3, True, 5, 4)            # generic kernels, factorized
PLAIN = bs.SfnnForwardShape(bs.HALFKA_HM2_DIMENSIONS, 256, 7, True, 16, 3)  # no FT factorizer


def _weights(shape, seed, shared_l2_l3=False, std=0.05):
    return synthetic.sfnn_weights(synthetic.rng_for(seed), shape.input_size, shape.ft_size, shape.l1_hidden,
                                  shape.l1_skip, shape.l2_size, shape.num_stacks, True, shared_l2_l3, std)


def _batch(seed, batch, stacks, pad=False):
    b = synthetic.sfnn_batch(seed, batch, stacks=stacks)
    if pad:
        rng = np.random.default_rng(seed)
        for key in ("stm", "nstm"):
            a = b[key]
            a[rng.random(a.size) < 0.05] = -1
            a[rng.random(a.size) < 0.01] = 10 ** 6          # out of range: ignored
        b["stm"][3 * 40:4 * 40] = -1                          # a perspective with no feature
        b["buckets"][5] = stacks                              # invalid bucket
    return b


def _dev(ctx, w):
    return {n: (None if w.get(n) is None else bo.F32Buffer.from_host(ctx, w[n])) for n in bs.SFNN_WEIGHT_NAMES}


def _forward(ctx, shape, w, b, alpha=bs.SfnnFactorizerAlpha(), fold=False):
    dw = _dev(ctx, w)
    B = b["batch"]
    s, n, k = (bo.I32Buffer.from_host(ctx, b[x]) for x in ("stm", "nstm", "buckets"))
    ws = bs.SfnnForwardWorkspace(ctx, shape, B)
    scratch = bo.F32Buffer(ctx, shape.input_size * shape.ft_size) if fold else None
    bs.sfnn_forward_device(ctx, shape, B, b["max_active"], s, n, k, dw, ws, alpha, scratch)
    return ws.download(ctx), (dw, s, n, k, ws)


def _oracle_forward(shape, w, b, alpha=bs.SfnnFactorizerAlpha()):
    return oracle.sfnn_forward(shape.as_tuple(), b["stm"], b["nstm"], b["buckets"], b["batch"], b["max_active"], w,
                               alpha.ft, alpha.shared)


# ---------------------------------------------------------------- forward
def test_tiny_forward_golden(ctx, goldens):
    g = goldens["tiny_sfnn_fast"]
    shape = bs.SfnnForwardShape(*g["shape"][:3], bool(g["shape"][3]), *g["shape"][4:])
    w = {k: np.asarray(v, np.float32) for k, v in g["weights"].items()}
    b = {"stm": np.asarray(g["stm"], np.int32), "nstm": np.asarray(g["nstm"], np.int32),
         "buckets": np.asarray(g["buckets"], np.int32), "batch": g["batch"], "max_active": g["max_active"]}
    out, _ = _forward(ctx, shape, w, b)
    for key, gk in (("stm_l0", "stm_l0"), ("nstm_l0", "nstm_l0"), ("combined", "combined"), ("l1", "l1"),
                    ("l2_input", "l2_input"), ("l2", "l2"), ("output", "outputs")):
        assert_close(out[key], g[gk], 0.0, g["tolerance"], key)


@pytest.mark.parametrize("shape,alpha,shared23", [
    (PROD, bs.SfnnFactorizerAlpha(), False),
    (SMALL, bs.SfnnFactorizerAlpha(0.5, 1.5), True),
    (GENERIC, bs.SfnnFactorizerAlpha(2.0, 0.25), True),
    (PLAIN, bs.SfnnFactorizerAlpha(), False),
])
def test_forward_vs_oracle(ctx, shape, alpha, shared23):
    w = _weights(shape, 21, shared23)
    b = _batch(22, 512, shape.num_stacks, pad=True)
    got, _ = _forward(ctx, shape, w, b, alpha)
    ref = _oracle_forward(shape, w, b, alpha)
    # FT sums: bias + folded rows in slot order, as in the oracle -> bit-exact
    for k in ("stm_l0", "nstm_l0", "combined"):
        assert np.array_equal(got[k], ref[k]), k
    for k in ("l1", "l2_input", "l2", "output"):
        assert_close_scaled(got[k], ref[k], 1e-5, k)


def test_forward_matches_reference_backend(ctx, ref_ctx):
    w = _weights(PROD, 31)
    b = _batch(32, 2048, PROD.num_stacks)
    got, _ = _forward(ctx, PROD, w, b)
    ref, _ = _forward(ref_ctx, PROD, w, b, fold=True)
    for k in ("stm_l0", "nstm_l0", "combined"):
        assert np.array_equal(got[k], ref[k]), k
    for k in ("l1", "l2_input", "l2", "output"):
        assert_close_scaled(got[k], ref[k], 1e-5, k)


def test_forward_rejects_unsupported_options(ctx, lib):
    w = _weights(GENERIC, 1)
    b = _batch(2, 8, GENERIC.num_stacks)
    dw = _dev(ctx, w)
    s, n, k = (bo.I32Buffer.from_host(ctx, b[x]) for x in ("stm", "nstm", "buckets"))
    ws = bs.SfnnForwardWorkspace(ctx, GENERIC, 8)
    sh = GENERIC
    with pytest.raises(bo.CudaCppError, match="grouped"):
        lib.call("bulletou_cuda_cpp_sfnn_forward_device", ctx.as_ptr(), sh.input_size, sh.ft_size, sh.l1_hidden, 1,
                 sh.l2_size, sh.num_stacks, 2, 0, 0, 0, 0, 8, 40, s.as_ptr(), n.as_ptr(), k.as_ptr(),
                 dw["l0w"].as_ptr(), None, dw["l0b"].as_ptr(), dw["l1w"].as_ptr(), dw["l1b"].as_ptr(),
                 dw["l1fw"].as_ptr(), dw["l1fb"].as_ptr(), 1, None, None, 0, dw["l2w"].as_ptr(), dw["l2b"].as_ptr(),
                 None, None, 0, None, None, 0, dw["l3w"].as_ptr(), dw["l3b"].as_ptr(), None, None, 0, None, None, 0,
                 0, 0, 0, 0, 0, 0, 1.0, 1.0, 1.0, 1.0, 1.0, 1.0, None, None, ws.stm_l0.as_ptr(),
                 ws.nstm_l0.as_ptr(), ws.combined.as_ptr(), ws.l1.as_ptr(), ws.l2_input.as_ptr(), ws.l2.as_ptr(),
                 ws.output.as_ptr(), None, None, 0)


# ---------------------------------------------------------------- backward
def _backward(ctx, shape, w, b, alpha, mog_host):
    out, (dw, s, n, k, ws) = _forward(ctx, shape, w, b, alpha)
    present = {nm: w.get(nm) is not None for nm in bs.SFNN_WEIGHT_NAMES}
    bws = bs.SfnnBackwardWorkspace(ctx, shape, b["batch"], present)
    mog = bo.F32Buffer.from_host(ctx, mog_host)
    bs.sfnn_backward_train_device(ctx, shape, b["batch"], b["max_active"], s, n, k, dw, ws, mog, bws, alpha, True)
    return out, bws.download(ctx)


@pytest.mark.parametrize("shape,alpha,shared23", [
    (SMALL, bs.SfnnFactorizerAlpha(), False),
    (SMALL, bs.SfnnFactorizerAlpha(0.5, 1.5), True),
    (GENERIC, bs.SfnnFactorizerAlpha(2.0, 0.25), True),
    (PLAIN, bs.SfnnFactorizerAlpha(), False),
])
def test_backward_vs_oracle(ctx, shape, alpha, shared23):
    w = _weights(shape, 41, shared23)
    b = _batch(42, 384, shape.num_stacks, pad=True)
    mog = synthetic.rng_for(43).normal(0, 1e-3, b["batch"]).astype(np.float32)
    fwd, got = _backward(ctx, shape, w, b, alpha, mog)
    ref = oracle.sfnn_backward(shape.as_tuple(), b["stm"], b["nstm"], b["buckets"], b["batch"], b["max_active"],
                               fwd, w, mog, alpha.ft, alpha.shared)
    assert_close_scaled(got["l1_gradients"], ref["l1_gradients"], 1e-5, "l1_gradients")
    assert_close_scaled(got["combined_gradients"], ref["combined_gradients"], 1e-5, "combined_gradients")
    for nm in bs.SFNN_WEIGHT_NAMES:
        if w.get(nm) is None:
            continue
        assert_close_scaled(got[f"{nm}_gradients"], ref[f"{nm}_gradients"], 1e-4 if nm == "l0w" else 1e-5, nm)


def test_backward_accumulates_and_overwrites_virtual_rows(ctx):
    """zero_parameter_gradients = 0 adds to the gradient buffers; the virtual
    factor rows are recomputed from the accumulated base rows (cu:4950-4985)."""
    shape, alpha = SMALL, bs.SfnnFactorizerAlpha()
    w = _weights(shape, 51)
    b = _batch(52, 256, shape.num_stacks)
    mog = synthetic.rng_for(53).normal(0, 1e-3, b["batch"]).astype(np.float32)
    out, (dw, s, n, k, ws) = _forward(ctx, shape, w, b, alpha)
    present = {nm: w.get(nm) is not None for nm in bs.SFNN_WEIGHT_NAMES}
    bws = bs.SfnnBackwardWorkspace(ctx, shape, b["batch"], present)
    m = bo.F32Buffer.from_host(ctx, mog)
    bs.sfnn_backward_train_device(ctx, shape, b["batch"], 40, s, n, k, dw, ws, m, bws, alpha, True)
    once = bws.download(ctx)
    bs.sfnn_backward_train_device(ctx, shape, b["batch"], 40, s, n, k, dw, ws, m, bws, alpha, False)
    twice = bws.download(ctx)
    for nm in ("l0w", "l0b", "l1w", "l1fw", "l2w", "l3b"):
        assert_close_scaled(twice[f"{nm}_gradients"], 2.0 * once[f"{nm}_gradients"], 1e-6, nm)


def test_backward_matches_reference_backend(ctx, ref_ctx):
    shape, alpha = PROD, bs.SfnnFactorizerAlpha()
    w = _weights(shape, 61)
    b = _batch(62, 1024, shape.num_stacks)
    mog = synthetic.rng_for(63).normal(0, 1e-3, b["batch"]).astype(np.float32)
    _, got = _backward(ctx, shape, w, b, alpha, mog)
    _, ref = _backward(ref_ctx, shape, w, b, alpha, mog)
    for key in ("l1_gradients", "combined_gradients", "stm_l0_pre_gradients", "nstm_l0_pre_gradients"):
        assert_close_scaled(got[key], ref[key], 1e-5, key)
    for nm in bs.SFNN_WEIGHT_NAMES:
        if w.get(nm) is None:
            continue
        assert_close_scaled(got[f"{nm}_gradients"], ref[f"{nm}_gradients"], 1e-4 if nm == "l0w" else 1e-5, nm)


# ---------------------------------------------------------------- train steps
def _host_weights(shape, w):
    return bs.SfnnForwardHostWeights(shape, **{k: v for k, v in w.items()})


def _host_batch(b):
    return bs.SfnnTrainStepHostBatch(b["stm"], b["nstm"], b["buckets"], b["targets"], b["entry_weights"], b["batch"],
                                     b["max_active"])


def _params(step, lr=1e-3, **kw):
    return bo.RangerUpdateParams(radam=bo.RAdamUpdateParams(step=step, learning_rate=lr, **kw))


def test_tiny_train_step_vs_oracle(ctx, goldens):
    g = goldens["tiny_sfnn_runner"]
    shape = bs.SfnnForwardShape(*g["shape"][:3], bool(g["shape"][3]), *g["shape"][4:])
    w = {k: np.asarray(v, np.float32) for k, v in g["weights"].items()}
    b = {k: np.asarray(g[k]) for k in ("stm", "nstm", "buckets", "targets", "entry_weights")}
    b.update(batch=g["batch"], max_active=g["max_active"])
    r = g["ranger"]
    runner = bs.SfnnTrainStepRunner(ctx, _host_weights(shape, w), g["batch"], g["max_active"])
    assert runner.fused
    params = bo.RangerUpdateParams(radam=bo.RAdamUpdateParams(step=r["step"], learning_rate=r["learning_rate"],
                                                               beta1=r["beta1"], beta2=r["beta2"],
                                                               min_weight=r["min_weight"], max_weight=r["max_weight"]),
                                   lookahead_alpha=r["lookahead_alpha"], lookahead_period=r["lookahead_period"])
    loss = runner.step(ctx, params, bo.ScalarLossKind.SigmoidPow(2.0), 1.0, _host_batch(b))
    trainer = oracle.SfnnTrainer(shape.as_tuple(), w)
    res = trainer.step(b["stm"], b["nstm"], b["buckets"], g["batch"], g["max_active"], b["targets"],
                       b["entry_weights"], **r)
    assert abs(loss.mean - res["loss"]["mean"]) <= 1e-6
    got = runner.read_weights(ctx)
    for nm in trainer.names:
        assert_close(got[nm], trainer.w[nm], 0.0, g["tolerance"], nm)


@pytest.mark.parametrize("shape,alpha,shared23", [
    (SMALL, bs.SfnnFactorizerAlpha(), False),
    (GENERIC, bs.SfnnFactorizerAlpha(0.5, 2.0), True),
])
def test_train_steps_fused_vs_oracle(ctx, shape, alpha, shared23):
    w = _weights(shape, 71, shared23)
    runner = bs.SfnnTrainStepRunner(ctx, _host_weights(shape, w), 256, 40, alpha)
    trainer = oracle.SfnnTrainer(shape.as_tuple(), w, alpha.ft, alpha.shared)
    for step in range(1, 8):  # crosses the lookahead at step 6
        b = _batch(100 + step, 256, shape.num_stacks, pad=True)
        kw = dict(min_weight=-1.98, max_weight=1.98)
        runner.step_no_readback(ctx, _params(step, **kw), bo.ScalarLossKind.SigmoidPow(2.0), 1 / 600, _host_batch(b))
        trainer.step(b["stm"], b["nstm"], b["buckets"], 256, 40, b["targets"], b["entry_weights"], step=step,
                     learning_rate=1e-3, inv_scale=1 / 600, **kw)
    got = runner.read_weights(ctx)
    for nm in trainer.names:
        assert_close_scaled(got[nm], trainer.w[nm], 1e-4, nm)


def test_unfused_product_runner_matches_fused(ctx):
    shape = SMALL
    w = _weights(shape, 81)
    fused = bs.SfnnTrainStepRunner(ctx, _host_weights(shape, w), 512, 40)
    plain = bs.SfnnTrainStepRunner(ctx, _host_weights(shape, w), 512, 40, fused=False)
    for step in range(1, 4):
        hb = _host_batch(_batch(200 + step, 512, shape.num_stacks))
        for r in (fused, plain):
            r.step_no_readback(ctx, _params(step), bo.ScalarLossKind.SigmoidPow(2.0), 1 / 600, hb)
    a, c = fused.read_weights(ctx), plain.read_weights(ctx)
    for nm in a:
        assert_close_scaled(a[nm], c[nm], 1e-5, nm)


def test_100_step_weights_match_reference_backend(ctx, ref_ctx):
    """weights after 100 steps within 1e-3 of the reference
    backend's, production shape (HalfKA_hm2 + factorizer, 1536, 15+1, 32, 9)."""
    shape = PROD
    w = _weights(shape, 91, std=0.01)
    B = 2048
    ours = bs.SfnnTrainStepRunner(ctx, _host_weights(shape, w), B, 40)
    ref = bs.SfnnTrainStepRunner(ref_ctx, _host_weights(shape, w), B, 40)
    assert ours.fused and not ref.fused
    batches = [_host_batch(_batch(300 + i, B, shape.num_stacks)) for i in range(10)]
    for step in range(1, 101):
        hb = batches[step % len(batches)]
        for r, c in ((ours, ctx), (ref, ref_ctx)):
            r.step_no_readback(c, _params(step), bo.ScalarLossKind.SigmoidPow(2.0), 1 / 600, hb)
    a, c = ours.read_weights(ctx), ref.read_weights(ref_ctx)
    for nm in a:
        err = float(np.abs(a[nm].astype(np.float64) - c[nm]).max())
        assert err <= 1e-3, f"{nm}: max |diff| {err:.3e} after 100 steps"
    la, lr_ = ours.read_loss(ctx), ref.read_loss(ref_ctx)
    assert abs(la.mean - lr_.mean) <= 1e-4 * max(1.0, abs(lr_.mean))


def test_fused_loss_matches_standalone_loss(ctx):
    shape = SMALL
    w = _weights(shape, 95)
    b = _batch(96, 300, shape.num_stacks)
    runner = bs.SfnnTrainStepRunner(ctx, _host_weights(shape, w), 300, 40)
    loss = runner.step(ctx, _params(1, lr=0.0), bo.ScalarLossKind.SigmoidPow(2.0), 1 / 600, _host_batch(b))
    out = runner.read_output(ctx)
    fwd = _oracle_forward(shape, w, b)
    assert_close_scaled(out, fwd["output"], 1e-5, "output")
    lw = ScalarLossWorkspace(ctx, 300)
    scalar_loss_device(ctx, bo.ScalarLossKind.SigmoidPow(2.0), 1 / 600, 300, bo.F32Buffer.from_host(ctx, out),
                       bo.F32Buffer.from_host(ctx, b["targets"]), bo.F32Buffer.from_host(ctx, b["entry_weights"]), lw)
    assert abs(loss.mean - lw.download(ctx).mean) <= 1e-6 * max(1.0, abs(loss.mean))


def test_train_step_rejects_norm_loss_and_bad_layout(ctx):
    shape = GENERIC
    w = _weights(shape, 97)
    runner = bs.SfnnTrainStepRunner(ctx, _host_weights(shape, w), 16, 40)
    with pytest.raises(bo.CudaCppError, match="layout mismatch"):
        runner.step(ctx, _params(1), bo.ScalarLossKind.SigmoidPow(2.0), 1.0, _host_batch(_batch(1, 8, 4)))


def test_k9k9_zipf_fused_vs_reference_backend(ctx, ref_ctx):
    """configs[4]'s LayerStack: 81 buckets, Zipf(1.1)-skewed bucket ids (a
    seeded permutation of ranks), 20 steps of the fused step against the
    reference backend, weights within 1e-3."""
    shape = bs.SfnnForwardShape(HM2F, 1536, 15, True, 32, 81)
    w = _weights(shape, 93, std=0.01)
    B = 4096
    ours = bs.SfnnTrainStepRunner(ctx, _host_weights(shape, w), B, 40)
    ref = bs.SfnnTrainStepRunner(ref_ctx, _host_weights(shape, w), B, 40)
    batches = [_host_batch(synthetic.sfnn_batch(500 + i, B, stacks=81, zipf=1.1)) for i in range(4)]
    counts = np.bincount(np.concatenate([b.buckets for b in batches]), minlength=81)
    assert counts.max() > 8 * max(1, counts[counts > 0].min())      # skewed
    for step in range(1, 21):
        hb = batches[step % len(batches)]
        for r, c in ((ours, ctx), (ref, ref_ctx)):
            r.step_no_readback(c, _params(step), bo.ScalarLossKind.SigmoidPow(2.0), 1 / 600, hb)
    a, c = ours.read_weights(ctx), ref.read_weights(ref_ctx)
    for nm in a:
        err = float(np.abs(a[nm].astype(np.float64) - c[nm]).max())
        assert err <= 1e-3, f"{nm}: max |diff| {err:.3e} after 20 steps"


def test_step_waits_for_weights_ready_event(ctx):
    """bulletou_b200_context_wait_before_weights: the fused step reads the
    weights only after the event, here recorded on another stream behind a
    delayed copy of new FT weights into the runner's table."""
    import torch

    shape = SMALL
    w0 = _weights(shape, 111)
    w1 = dict(w0, l0w=_weights(shape, 112)["l0w"])
    b = _host_batch(_batch(113, 512, shape.num_stacks))
    ctx.synchronize()
    waiting = bs.SfnnTrainStepRunner(ctx, _host_weights(shape, w0), 512, 40)
    direct = bs.SfnnTrainStepRunner(ctx, _host_weights(shape, w1), 512, 40)
    src = bo.F32Buffer.from_host(ctx, w1["l0w"])
    ctx.synchronize()
    s2 = torch.cuda.Stream()
    ctx2 = bo.Context(0, stream=s2.cuda_stream)
    lib = ctx.lib
    with torch.cuda.stream(s2):
        torch.cuda._sleep(100_000_000)  # a bounded busy kernel (about 50 ms) ahead of the copy
        torch.as_tensor(waiting.weights["l0w"], device="cuda:0").copy_(torch.as_tensor(src, device="cuda:0"))
    ready = bo.Event(ctx2)
    ready.record(ctx2)
    lib.call("bulletou_b200_context_wait_before_weights", ctx.as_ptr(), ready._h)
    waiting.step_no_readback(ctx, _params(1), bo.ScalarLossKind.SigmoidPow(2.0), 1 / 600, b)
    direct.step_no_readback(ctx, _params(1), bo.ScalarLossKind.SigmoidPow(2.0), 1 / 600, b)
    a, c = waiting.read_weights(ctx), direct.read_weights(ctx)
    for nm in a:
        assert np.array_equal(a[nm], c[nm]), nm
    # consumed by that step; null clears
    lib.call("bulletou_b200_context_wait_before_weights", ctx.as_ptr(), None)
    torch.cuda.synchronize()
    ctx2.close()


def test_upload_next_then_step_matches_pipelined_step(ctx):
    """upload_next + step_uploaded (the next batch's upload issued while the
    current step runs) gives the same weights as the pipelined step."""
    shape = SMALL
    w = _weights(shape, 121)
    upload = bo.Context(0)
    a = bs.SfnnTrainStepRunner(ctx, _host_weights(shape, w), 512, 40)
    b = bs.SfnnTrainStepRunner(ctx, _host_weights(shape, w), 512, 40)
    batches = [_host_batch(_batch(122 + i, 512, shape.num_stacks)) for i in range(4)]
    b.upload_next(upload, batches[0])
    for step in range(1, 5):
        a.step_pipelined_no_readback_with_loss_finalize(ctx, upload, _params(step), bo.ScalarLossKind.SigmoidPow(2.0),
                                                        1 / 600, batches[step - 1])
        b.step_uploaded_no_readback_with_loss_finalize(ctx, _params(step), bo.ScalarLossKind.SigmoidPow(2.0), 1 / 600)
        if step < 4:
            b.upload_next(upload, batches[step])
    ra, rb = a.read_weights(ctx), b.read_weights(ctx)
    for nm in ra:
        assert np.array_equal(ra[nm], rb[nm]), nm
    upload.close()
