"""GPU parity of the KPPT scalar tables (KK / KKP / KPP components): the
reference C-ABI forward / backward and the fused train step of the product
library against the CPU oracle and the reference backend built from its
sources (crates/cuda_cpp/cpp/bulletou_cuda_backend.cu:8970-9140, 11887-11983;
runner lib.rs:4962-5066)."""
import numpy as np
import pytest

import bulletou_b200 as bo
from bulletou_b200 import synthetic
from oracle import oracle
from tests.conftest import assert_close_scaled

pytestmark = pytest.mark.gpu

COMPONENTS = ("kk", "kkp", "kpp")


def _case(comp, seed, batch, pad=False, table=True):
    rng = synthetic.rng_for(seed)
    stm, nstm, n, A = synthetic.kppt_indices(rng, batch, comp)
    if pad:
        for a in (stm, nstm):
            a[rng.random(a.size) < 0.05] = -1
            a[rng.random(a.size) < 0.01] = n + 7       # out of range: ignored
    tw = rng.normal(0.0, 0.02, n).astype(np.float32) if table else None
    t, ew = synthetic.targets(rng, batch)
    return {"stm": stm, "nstm": nstm, "n": n, "A": A, "batch": batch, "table_w": tw, "table_b": 0.125,
            "outw": np.array([0.7, -0.4], np.float32), "outb": 0.05, "targets": t, "entry_weights": ew}


def _abi_forward(ctx, c):
    B = c["batch"]
    bufs = {"stm": bo.I32Buffer.from_host(ctx, c["stm"]), "nstm": bo.I32Buffer.from_host(ctx, c["nstm"]),
            "table_w": bo.F32Buffer.from_host(ctx, c["table_w"]),
            "table_b": bo.F32Buffer.from_host(ctx, np.array([c["table_b"]], np.float32)),
            "outw": bo.F32Buffer.from_host(ctx, c["outw"]),
            "outb": bo.F32Buffer.from_host(ctx, np.array([c["outb"]], np.float32)),
            "stm_eval": bo.F32Buffer(ctx, B), "nstm_eval": bo.F32Buffer(ctx, B), "output": bo.F32Buffer(ctx, B)}
    ctx.lib.call("bulletou_cuda_cpp_kppt_forward_device", ctx.as_ptr(), c["n"], B, c["A"],
                 *[bufs[k].as_ptr() for k in ("stm", "nstm", "table_w", "table_b", "outw", "outb", "stm_eval",
                                              "nstm_eval", "output")])
    return {k: bufs[k].download(ctx) for k in ("stm_eval", "nstm_eval", "output")}, bufs


def _abi_backward(ctx, c, bufs, mog):
    grads = {"table_w": bo.F32Buffer(ctx, c["n"]), "table_b": bo.F32Buffer(ctx, 1), "outw": bo.F32Buffer(ctx, 2),
             "outb": bo.F32Buffer(ctx, 1)}
    for g in grads.values():
        g.fill(123.0)                       # the backward zero-fills what it writes
    m = bo.F32Buffer.from_host(ctx, mog)
    ctx.lib.call("bulletou_cuda_cpp_kppt_backward_device", ctx.as_ptr(), c["n"], c["batch"], c["A"],
                 bufs["stm"].as_ptr(), bufs["nstm"].as_ptr(), bufs["stm_eval"].as_ptr(), bufs["nstm_eval"].as_ptr(),
                 bufs["outw"].as_ptr(), m.as_ptr(), *[grads[k].as_ptr() for k in ("table_w", "table_b", "outw",
                                                                                    "outb")])
    return {k: g.download(ctx) for k, g in grads.items()}


def _oracle_forward(c):
    return oracle.kppt_forward(c["n"], c["stm"], c["nstm"], c["batch"], c["A"], c["table_w"], c["table_b"],
                               c["outw"], c["outb"])


@pytest.mark.parametrize("comp", COMPONENTS)
def test_forward_vs_oracle(ctx, comp):
    c = _case(comp, 1, 4096, pad=True)
    got, _ = _abi_forward(ctx, c)
    want = _oracle_forward(c)
    for k in ("stm_eval", "nstm_eval", "output"):
        assert_close_scaled(got[k], want[k], 1e-5, k)


@pytest.mark.parametrize("comp", COMPONENTS)
def test_forward_vs_reference_backend(ctx, ref_ctx, comp):
    c = _case(comp, 2, 4096, pad=True)
    got, _ = _abi_forward(ctx, c)
    theirs, _ = _abi_forward(ref_ctx, c)
    for k in ("stm_eval", "nstm_eval", "output"):
        assert_close_scaled(got[k], theirs[k], 1e-5, k)


@pytest.mark.parametrize("comp", COMPONENTS)
def test_backward_vs_oracle_and_reference(ctx, ref_ctx, comp):
    c = _case(comp, 3, 4096, pad=True)
    fwd, bufs = _abi_forward(ctx, c)
    mog = synthetic.rng_for(33).normal(0.0, 1e-3, c["batch"]).astype(np.float32)
    got = _abi_backward(ctx, c, bufs, mog)
    want = oracle.kppt_backward(c["n"], c["stm"], c["nstm"], c["batch"], c["A"], fwd, c["outw"], mog)
    for k in ("table_w", "table_b", "outw", "outb"):
        assert_close_scaled(got[k], want[k], 1e-5, f"{k} vs oracle")
    rf, rbufs = _abi_forward(ref_ctx, c)
    theirs = _abi_backward(ref_ctx, c, rbufs, mog)
    for k in ("table_w", "table_b", "outw", "outb"):
        assert_close_scaled(got[k], theirs[k], 1e-5, f"{k} vs reference")


def _runner(ctx, c, fused=None):
    return bo.KpptTableTrainStepRunner(ctx, c["n"], c["table_w"], c["table_b"], c["outw"], c["outb"], c["batch"],
                                       c["A"], fused=fused)


def _ranger(step, lr=1e-3):
    return bo.RangerUpdateParams(radam=bo.RAdamUpdateParams(step=step, learning_rate=lr))


@pytest.mark.parametrize("comp", ("kk", "kkp"))
def test_fused_step_vs_oracle(ctx, comp):
    c = _case(comp, 4, 2048, pad=True)
    runner = _runner(ctx, c)
    assert runner.fused
    w = {"table_w": c["table_w"].copy(), "table_b": np.array([c["table_b"]], np.float32),
         "outw": c["outw"].copy(), "outb": np.array([c["outb"]], np.float32)}
    m = {k: np.zeros_like(v) for k, v in w.items()}
    v2 = {k: np.zeros_like(v) for k, v in w.items()}
    slow = {k: v.copy() for k, v in w.items()}
    loss_kind = bo.ScalarLossKind.SigmoidPow(2.0)
    for step in range(1, 8):
        runner.upload_batch(c["stm"], c["nstm"], c["targets"], c["entry_weights"], ctx)
        runner.step_device(ctx, _ranger(step, 0.01), loss_kind, 1 / 600)
        f = oracle.kppt_forward(c["n"], c["stm"], c["nstm"], c["batch"], c["A"], w["table_w"], w["table_b"],
                                w["outw"], w["outb"])
        loss = oracle.scalar_loss(0, 1 / 600, 2.0, 0.0, f["output"], c["targets"], c["entry_weights"])
        g = oracle.kppt_backward(c["n"], c["stm"], c["nstm"], c["batch"], c["A"], f, w["outw"],
                                 loss["mean_output_gradients"])
        for k in w:
            oracle.ranger_update(g[k], w[k], m[k], v2[k], slow[k], step=step, learning_rate=0.01)
        lm = runner.read_loss(ctx)
        assert lm.mean == pytest.approx(loss["mean"], rel=1e-5)
    got = runner.read_weights(ctx)
    for k in w:
        assert_close_scaled(got[k], w[k], 1e-4, k)


def test_fused_matches_unfused(ctx):
    c = _case("kkp", 5, 4096)
    fused, plain = _runner(ctx, c, True), _runner(ctx, c, False)
    loss_kind = bo.ScalarLossKind.SigmoidPow(2.0)
    for step in range(1, 5):
        for r in (fused, plain):
            r.upload_batch(c["stm"], c["nstm"], c["targets"], c["entry_weights"], ctx)
            r.step_device(ctx, _ranger(step), loss_kind, 1 / 600)
        assert fused.read_loss(ctx).mean == pytest.approx(plain.read_loss(ctx).mean, rel=1e-6)
    wf, wp = fused.read_weights(ctx), plain.read_weights(ctx)
    for k in wf:
        assert_close_scaled(wf[k], wp[k], 1e-5, k)


@pytest.mark.parametrize("comp", ("kkp", "kpp"))
def test_100_step_weights_match_reference_backend(ctx, ref_ctx, comp):
    """Weights after 100 steps within 1e-3 of the reference backend's runner
    sequence on identical seeded batches."""
    cases = [_case(comp, 100 + i, 16384, table=(i == 0)) for i in range(4)]
    c0 = cases[0]
    mine, theirs = _runner(ctx, c0), _runner(ref_ctx, c0)
    assert mine.fused and not theirs.fused
    loss_kind = bo.ScalarLossKind.SigmoidPow(2.0)
    for step in range(1, 101):
        c = cases[step % len(cases)]
        mine.upload_batch(c["stm"], c["nstm"], c["targets"], c["entry_weights"], ctx)
        theirs.upload_batch(c["stm"], c["nstm"], c["targets"], c["entry_weights"], ref_ctx)
        mine.step_device(ctx, _ranger(step), loss_kind, 1 / 600)
        theirs.step_device(ref_ctx, _ranger(step), loss_kind, 1 / 600)
    assert mine.read_loss(ctx).mean == pytest.approx(theirs.read_loss(ref_ctx).mean, rel=1e-3)
    wm, wt = mine.read_weights(ctx), theirs.read_weights(ref_ctx)
    for k in wm:
        diff = np.abs(wm[k].astype(np.float64) - wt[k])
        assert diff.max() <= 1e-3, f"{k}: max |diff| {diff.max():.3e}"
