"""GPU parity of the rest of the reference ABI: the per-bucket ("dirty")
Ranger step, the SFNN backward variants (plain and profiled), the quantised
proxy, the FP16 switches in their off position, and the row / bucket scaling
utilities -- against the reference backend built from its sources and numpy."""
import numpy as np
import pytest

import bulletou_b200 as bo
from bulletou_b200 import sfnn as bs
from bulletou_b200 import synthetic
from bulletou_b200.cuda_cpp import RangerDeviceState
from tests.conftest import assert_close_scaled

pytestmark = pytest.mark.gpu

HM2F = bs.HALFKA_HM2_DIMENSIONS + bs.PIECE_INPUTS
PROD = bs.SFNN_HALFKA_HM2_1536_15_32_K3K3
SMALL = bs.SfnnForwardShape(HM2F, 256, 15, True, 32, 9)


def _state(ctx, host):
    return RangerDeviceState(*[bo.F32Buffer.from_host(ctx, host[k]) for k in ("g", "w", "m", "v", "s")])


def _read(ctx, st):
    return {k: getattr(st, f).download(ctx) for k, f in (("g", "gradients"), ("w", "weights"), ("m", "momentum"),
                                                          ("v", "velocity"), ("s", "slow_params"))}


@pytest.mark.parametrize("stride", [1024, 1001])
@pytest.mark.parametrize("norm", [0.0, 1e-3])
def test_stacked_dirty_ranger_matches_reference(ctx, ref_ctx, stride, norm):
    """Eight steps (a lookahead at step 6) over the dirty buckets of a 9-bucket
    group: untouched buckets keep their gradients and state bit for bit;
    stepped ones match the reference within 2e-6 of scale (FMA contraction of
    the EMA terms differs by an ulp of the terms, as for the dense Ranger)."""
    stacks = 9
    rng = np.random.default_rng(5)
    n = stacks * stride
    host = {"w": rng.normal(0, 0.05, n).astype(np.float32), "m": np.zeros(n, np.float32),
            "v": np.zeros(n, np.float32)}
    host["s"] = host["w"].copy()
    states = {}
    for c in (ctx, ref_ctx):
        h = dict(host, g=np.zeros(n, np.float32))
        states[c] = _state(c, h)
    dirty = np.array([0, 3, 7, -1, 8, 100], np.int32)
    for step in range(1, 9):
        g = rng.normal(0, 1e-2, n).astype(np.float32)
        params = bo.RangerUpdateParams(norm_loss_strength=norm,
                                       radam=bo.RAdamUpdateParams(step=step, min_weight=-1.5, max_weight=1.5))
        for c in (ctx, ref_ctx):
            states[c].gradients.upload(g, c)
            db = bo.I32Buffer.from_host(c, dirty)
            bo.ranger_update_stacked_dirty_device(c, params, states[c], stride, db, dirty.size)
            c.synchronize()
    a, r = _read(ctx, states[ctx]), _read(ref_ctx, states[ref_ctx])
    for k in a:
        assert_close_scaled(a[k], r[k], 2e-6, k)
    untouched = np.ones(stacks, bool)
    untouched[[0, 3, 7, 8]] = False
    rows = a["w"].reshape(stacks, stride)
    if norm == 0.0:
        assert np.array_equal(rows[untouched], host["w"].reshape(stacks, stride)[untouched])
    assert np.all(a["g"].reshape(stacks, stride)[~untouched] == 0.0)


def test_stacked_dirty_zero_learning_rate_only_clears(ctx):
    stride, stacks = 64, 4
    rng = np.random.default_rng(6)
    g = rng.normal(0, 1, stacks * stride).astype(np.float32)
    w = rng.normal(0, 1, stacks * stride).astype(np.float32)
    st = _state(ctx, {"g": g, "w": w, "m": np.zeros_like(w), "v": np.zeros_like(w), "s": w.copy()})
    db = bo.I32Buffer.from_host(ctx, np.array([1, 2], np.int32))
    bo.ranger_update_stacked_dirty_device(ctx, bo.RangerUpdateParams(radam=bo.RAdamUpdateParams(learning_rate=0.0)),
                                          st, stride, db, 2)
    out = _read(ctx, st)
    exp = g.reshape(stacks, stride).copy()
    exp[1:3] = 0.0
    assert np.array_equal(out["g"], exp.reshape(-1))
    assert np.array_equal(out["w"], w)


def _weights(shape, seed, shared_l2_l3=False, std=0.05):
    return synthetic.sfnn_weights(synthetic.rng_for(seed), shape.input_size, shape.ft_size, shape.l1_hidden,
                                  shape.l1_skip, shape.l2_size, shape.num_stacks, True, shared_l2_l3, std)


def _dev(ctx, w):
    return {n: (None if w.get(n) is None else bo.F32Buffer.from_host(ctx, w[n])) for n in bs.SFNN_WEIGHT_NAMES}


def _run_backward(ctx, shape, w, b, mog, which):
    dw = _dev(ctx, w)
    B = b["batch"]
    s, n, k = (bo.I32Buffer.from_host(ctx, b[x]) for x in ("stm", "nstm", "buckets"))
    ws = bs.SfnnForwardWorkspace(ctx, shape, B)
    bs.sfnn_forward_device(ctx, shape, B, b["max_active"], s, n, k, dw, ws)
    present = {nm: w.get(nm) is not None for nm in bs.SFNN_WEIGHT_NAMES}
    bws = bs.SfnnBackwardWorkspace(ctx, shape, B, present)
    for buf in bws.params.values():
        if buf is not None:
            buf.fill(0.25, ctx)  # the plain backward clears these first
    m = bo.F32Buffer.from_host(ctx, mog)
    prof = None
    if which == "plain":
        bs.sfnn_backward_device(ctx, shape, B, b["max_active"], s, n, k, dw, ws, m, bws)
    elif which == "profile":
        prof = bs.sfnn_backward_train_profile_device(ctx, shape, B, b["max_active"], s, n, k, dw, ws, m, bws,
                                                     zero_parameter_gradients=True)
    else:
        bs.sfnn_backward_train_device(ctx, shape, B, b["max_active"], s, n, k, dw, ws, m, bws,
                                      zero_parameter_gradients=True)
    return bws.download(ctx), prof


def test_sfnn_backward_variants_agree(ctx):
    """The plain backward equals the training backward with zeroed gradients,
    and the profiled one computes the same while timing its stages."""
    w = _weights(SMALL, 11, True)
    b = synthetic.sfnn_batch(12, 512, stacks=SMALL.num_stacks)
    mog = synthetic.rng_for(13).normal(0, 1e-3, 512).astype(np.float32)
    train, _ = _run_backward(ctx, SMALL, w, b, mog, "train")
    plain, _ = _run_backward(ctx, SMALL, w, b, mog, "plain")
    prof_out, prof = _run_backward(ctx, SMALL, w, b, mog, "profile")
    for key in train:
        assert np.array_equal(plain[key], train[key]), key
        assert np.array_equal(prof_out[key], train[key]), key
    assert set(prof) == set(bs.SFNN_BACKWARD_PROFILE_STAGES)
    assert all(v >= 0.0 for v in prof.values())
    assert prof["l2"] == 0.0 and prof["l2_input"] == 0.0  # one head kernel: reported under l3
    parts = prof["zero"] + prof["l3"] + prof["l1"] + prof["l0"]
    assert prof["total"] > 0.0 and abs(parts - prof["total"]) <= 0.05 * prof["total"] + 0.05


def test_sfnn_backward_device_matches_reference_backend(ctx, ref_ctx):
    w = _weights(PROD, 14)
    b = synthetic.sfnn_batch(15, 1024, stacks=PROD.num_stacks)
    mog = synthetic.rng_for(16).normal(0, 1e-3, 1024).astype(np.float32)
    got, _ = _run_backward(ctx, PROD, w, b, mog, "plain")
    ref, _ = _run_backward(ref_ctx, PROD, w, b, mog, "plain")
    for key in got:
        if not key.endswith("gradients"):
            continue
        tol = 1e-4 if key == "l0w_gradients" else 1e-5
        assert_close_scaled(got[key], ref[key], tol, key)


def test_profile_rejects_short_output(ctx, lib):
    import ctypes

    w = _weights(SMALL, 17)
    b = synthetic.sfnn_batch(18, 64, stacks=SMALL.num_stacks)
    dw = _dev(ctx, w)
    s, n, k = (bo.I32Buffer.from_host(ctx, b[x]) for x in ("stm", "nstm", "buckets"))
    ws = bs.SfnnForwardWorkspace(ctx, SMALL, 64)
    bs.sfnn_forward_device(ctx, SMALL, 64, 40, s, n, k, dw, ws)
    bws = bs.SfnnBackwardWorkspace(ctx, SMALL, 64, {nm: w.get(nm) is not None for nm in bs.SFNN_WEIGHT_NAMES})
    m = bo.F32Buffer.from_host(ctx, np.zeros(64, np.float32))
    args = bs._backward_args(ctx, SMALL, 64, 40, s, n, k, dw, ws, m, bws, bs.SfnnFactorizerAlpha(), None)
    with pytest.raises(bo.CudaCppError, match="at least 7"):
        lib.call("bulletou_cuda_cpp_sfnn_backward_train_profile_device", *args, 1, (ctypes.c_float * 3)(), 3)


@pytest.mark.parametrize("shape,shared23", [(PROD, False), (SMALL, True)])
def test_quantized_proxy_matches_reference_bitwise(ctx, ref_ctx, shape, shared23):
    w = _weights(shape, 21, shared23, std=0.1)
    base = shape.factorized_base()
    sizes = {"l0w": base * shape.ft_size, "l0b": shape.ft_size,
             "l1w": shape.num_stacks * shape.l1_out * shape.ft_size, "l1b": shape.num_stacks * shape.l1_out,
             "l2w": shape.num_stacks * shape.l2_size * shape.l2_in, "l2b": shape.num_stacks * shape.l2_size,
             "l3w": shape.num_stacks * shape.l2_size, "l3b": shape.num_stacks}
    out = {}
    for c in (ctx, ref_ctx):
        dst = {k: bo.F32Buffer(c, v) for k, v in sizes.items()}
        bs.sfnn_build_quantized_proxy_device(c, shape, _dev(c, w), dst)
        out[c] = {k: v.download(c) for k, v in dst.items()}
    for k in sizes:
        assert np.array_equal(out[ctx][k], out[ref_ctx][k]), k
    # on the engine lattices: FT and dense weights / biases
    for k, scale in (("l0w", 127), ("l1w", 64), ("l2w", 64), ("l1b", 8128)):
        x = out[ctx][k]
        q = np.round(x.astype(np.float64) * scale)
        assert np.array_equal((q.astype(np.float32) / np.float32(scale)).astype(np.float32), x), k
    assert np.abs(np.round(out[ctx]["l1w"].astype(np.float64) * 64)).max() <= 128


def test_quantized_proxy_skip_ft_keeps_destination(ctx):
    shape = SMALL
    w = _weights(shape, 22)
    base = shape.factorized_base()
    dst = {"l0w": bo.F32Buffer.from_host(ctx, np.full(base * shape.ft_size, 3.0, np.float32)),
           "l0b": bo.F32Buffer(ctx, shape.ft_size),
           "l1w": bo.F32Buffer(ctx, shape.num_stacks * shape.l1_out * shape.ft_size),
           "l1b": bo.F32Buffer(ctx, shape.num_stacks * shape.l1_out),
           "l2w": bo.F32Buffer(ctx, shape.num_stacks * shape.l2_size * shape.l2_in),
           "l2b": bo.F32Buffer(ctx, shape.num_stacks * shape.l2_size),
           "l3w": bo.F32Buffer(ctx, shape.num_stacks * shape.l2_size), "l3b": bo.F32Buffer(ctx, shape.num_stacks)}
    bs.sfnn_build_quantized_proxy_device(ctx, shape, _dev(ctx, w), dst, skip_ft_weights=True)
    assert np.all(dst["l0w"].download(ctx) == 3.0)


def test_fp16_switches_off_succeed_on_off_fail(ctx, lib):
    for name in ("set_sfnn_ft_fp16", "set_sfnn_ft_fp16_grad", "set_sfnn_ft_fp16_act"):
        lib.call(f"bulletou_cuda_cpp_context_{name}", ctx.as_ptr(), 0)
        with pytest.raises(bo.CudaCppError, match="unsupported on this backend"):
            lib.call(f"bulletou_cuda_cpp_context_{name}", ctx.as_ptr(), 1)
    lib.call("bulletou_cuda_cpp_context_release_sfnn_ft_fp16_scratch", ctx.as_ptr(), 1, 1, 1)


def test_row_and_bucket_utilities_match_reference(ctx, ref_ctx):
    rng = np.random.default_rng(31)
    stacks, stride = 9, 100
    w = rng.normal(0, 1, stacks * stride).astype(np.float32)
    g = rng.normal(0, 1, stacks * stride).astype(np.float32)
    gates = rng.uniform(0.5, 1.5, stacks).astype(np.float32)
    gates[2] = 1.0
    decay = rng.uniform(0, 1e-2, stacks).astype(np.float32)
    decay[4] = 0.0
    dirty = np.array([1, 2, 4, 8, 50], np.int32)
    res = {}
    for c in (ctx, ref_ctx):
        lib = c.lib
        W, G = bo.F32Buffer.from_host(c, w), bo.F32Buffer.from_host(c, g)
        GA, D, DB = bo.F32Buffer.from_host(c, gates), bo.F32Buffer.from_host(c, decay), bo.I32Buffer.from_host(c, dirty)
        lib.call("bulletou_cuda_cpp_sfnn_add_residual_count_decay_gradients_device", c.as_ptr(), W.as_ptr(),
                 G.as_ptr(), D.as_ptr(), DB.as_ptr(), dirty.size, stride, stacks)
        lib.call("bulletou_cuda_cpp_sfnn_apply_residual_count_gates_to_gradients_device", c.as_ptr(), G.as_ptr(),
                 GA.as_ptr(), None, 0, stride, stacks)
        lib.call("bulletou_cuda_cpp_scale_axis_rows_f32_device", c.as_ptr(), W.as_ptr(), stacks * stride,
                 GA.as_ptr(), stacks, stride)
        X = bo.F32Buffer(c, stacks * stride)
        lib.call("bulletou_center_scale", c.as_ptr(), W.as_ptr(), X.as_ptr(), stacks * stride, 0.5)
        res[c] = (G.download(c), W.download(c), X.download(c))
    for a, r in zip(res[ctx], res[ref_ctx]):
        assert np.array_equal(a, r)
    exp = g.reshape(stacks, stride).copy()
    for s in (1, 2, 4, 8):
        exp[s] += np.float32(2.0) * decay[s] * w.reshape(stacks, stride)[s]
    exp *= gates[:, None]
    assert_close_scaled(res[ctx][0], exp.reshape(-1), 1e-6, "decay + gates")
