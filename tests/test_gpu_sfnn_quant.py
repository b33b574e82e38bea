"""GPU parity of the quantised SFNN path: export quantisation and the engine's
integer forward on the device (bulletou_b200_sfnn_quantize_device,
bulletou_b200_sfnn_integer_forward_device) against the C oracle, bit-exact,
and against the reference's known answers for the evaluator
(examples/bulletou.rs:29660-29672, 37876-37882)."""
import numpy as np
import pytest

import bulletou_b200 as bo
from bulletou_b200 import sfnn as bs
from bulletou_b200 import synthetic
from oracle import oracle
from tests import quant_cases as qc

pytestmark = pytest.mark.gpu

HM2F = bs.HALFKA_HM2_DIMENSIONS + bs.PIECE_INPUTS
PROD = bs.SFNN_HALFKA_HM2_1536_15_32_K3K3
SMALL = bs.SfnnForwardShape(HM2F, 512, 15, True, 32, 9)
GENERIC = bs.SfnnForwardShape(HM2F, 12, 3, True, 5, 4)        # thread-per-pair FT kernel
PLAIN = bs.SfnnForwardShape(bs.HALFKA_HM2_DIMENSIONS, 1024, 7, False, 16, 3)


def _shape(t):
    return bs.SfnnForwardShape(t[0], t[1], t[2], bool(t[3]), t[4], t[5])


def _run(ctx, shape, q, stm, nstm, buckets, batch, max_active, rounding=bs.QuantizedRounding()):
    dq = bs.QuantizedSfnnDeviceWeights(ctx, shape)
    dq.upload(q, ctx)
    s, n, k = (bo.I32Buffer.from_host(ctx, np.asarray(x, np.int32)) for x in (stm, nstm, buckets))
    ws = bs.SfnnIntegerForwardWorkspace(ctx, shape, batch)
    bs.sfnn_integer_forward_device(ctx, shape, batch, max_active, s, n, k, dq, ws, rounding)
    return ws.download(ctx)


@pytest.mark.parametrize("sum0,sum1,shift,expected", qc.FT_PAIR_KATS)
def test_ft_pair_value_known_answers(ctx, sum0, sum1, shift, expected):
    shape, q = qc.ft_pair_net(sum0, sum1)
    out = _run(ctx, _shape(shape), q, [-1], [-1], [0], 1, 1, bs.QuantizedRounding(ft_shift=shift))
    assert int(out["raw"][0]) == expected and out["errors"] == 0


def test_activation_boundaries_known_answers(ctx):
    shape, q = qc.activation_net(qc.ACTIVATION_INPUTS)
    n = shape[5]
    out = _run(ctx, _shape(shape), q, [-1] * n, [-1] * n, list(range(n)), n, 1)
    for k, x in enumerate(qc.ACTIVATION_INPUTS):
        assert int(out["l1"][2 * k]) == x
        assert int(out["raw"][2 * k]) == qc.expected_activation(x, 0), f"square {x}"
        assert int(out["raw"][2 * k + 1]) == qc.expected_activation(x, 1), f"linear {x}"


@pytest.mark.parametrize("shape,alpha,shared23", [
    (PROD, bs.SfnnFactorizerAlpha(), False),
    (SMALL, bs.SfnnFactorizerAlpha(0.75, 1.25), True),
    (GENERIC, bs.SfnnFactorizerAlpha(2.0, 0.5), True),
    (PLAIN, bs.SfnnFactorizerAlpha(), False),
])
def test_quantize_vs_oracle(ctx, shape, alpha, shared23):
    w = synthetic.sfnn_weights(synthetic.rng_for(31), shape.input_size, shape.ft_size, shape.l1_hidden,
                               shape.l1_skip, shape.l2_size, shape.num_stacks, True, shared23, 0.3)
    dw = {n: (None if w.get(n) is None else bo.F32Buffer.from_host(ctx, w[n])) for n in bs.SFNN_WEIGHT_NAMES}
    dq = bs.QuantizedSfnnDeviceWeights(ctx, shape)
    bs.sfnn_quantize_device(ctx, shape, dw, dq, alpha)
    got = dq.download(ctx)
    want = oracle.sfnn_quantize(shape.as_tuple(), w, alpha.ft, alpha.shared)
    for n in qc.QUANT_NAMES:
        np.testing.assert_array_equal(got[n], want[n], err_msg=n)


def _batch(seed, batch, stacks, pad):
    b = synthetic.sfnn_batch(seed, batch, stacks=stacks)
    if pad:
        rng = np.random.default_rng(seed)
        for key in ("stm", "nstm"):
            a = b[key]
            a[rng.random(a.size) < 0.05] = -1
        b["stm"][3 * 40:4 * 40] = -1        # a perspective with no feature
    return b


@pytest.mark.parametrize("shape", [PROD, SMALL, GENERIC, PLAIN], ids=["prod", "small", "generic", "plain"])
@pytest.mark.parametrize("full_range", [False, True], ids=["narrow", "wrapping"])
@pytest.mark.parametrize("modes", [(0, 0, 0, 0), (1, 1, 1, 1)], ids=["floor", "nearest"])
def test_integer_forward_vs_oracle(ctx, shape, full_range, modes):
    rng = np.random.default_rng(7 + full_range)
    q = qc.random_integer_net(rng, shape.as_tuple(), full_range)
    batch = 2048
    b = _batch(13, batch, shape.num_stacks, pad=True)
    if shape is PLAIN:
        b["stm"] = np.where(b["stm"] >= shape.input_size, -1, b["stm"]).astype(np.int32)
        b["nstm"] = np.where(b["nstm"] >= shape.input_size, -1, b["nstm"]).astype(np.int32)
    r = bs.QuantizedRounding(7, *map(bool, modes), 24)
    out = _run(ctx, shape, q, b["stm"], b["nstm"], b["buckets"], batch, b["max_active"], r)
    want = oracle.sfnn_integer_forward(shape.as_tuple(), b["stm"], b["nstm"], b["buckets"], batch, b["max_active"],
                                       q, ft_shift=7, ft_round=modes[0], crelu_round=modes[1], sqr_round=modes[2])
    assert want["error"] == -1 and out["errors"] == 0
    np.testing.assert_array_equal(out["l1"], want["l1"])
    np.testing.assert_array_equal(out["raw"], want["raw"])
    np.testing.assert_array_equal(out["score"], oracle.final_division(want["raw"], 24, bool(modes[3])))


def test_trained_weights_quantize_then_integer_forward(ctx):
    """Production shape end to end on the device: f32 weights -> quantise ->
    integer forward, against the oracle's quantise -> integer forward."""
    shape = PROD
    w = synthetic.sfnn_weights(synthetic.rng_for(41), shape.input_size, shape.ft_size, shape.l1_hidden,
                               shape.l1_skip, shape.l2_size, shape.num_stacks, True, False, 0.08)
    w["l0b"] = (np.abs(w["l0b"]) + 0.3).astype(np.float32)   # open the FT clamp window
    dw = {n: (None if w.get(n) is None else bo.F32Buffer.from_host(ctx, w[n])) for n in bs.SFNN_WEIGHT_NAMES}
    dq = bs.QuantizedSfnnDeviceWeights(ctx, shape)
    bs.sfnn_quantize_device(ctx, shape, dw, dq)
    batch = 4096
    b = _batch(17, batch, shape.num_stacks, pad=False)
    s, n, k = (bo.I32Buffer.from_host(ctx, b[x]) for x in ("stm", "nstm", "buckets"))
    ws = bs.SfnnIntegerForwardWorkspace(ctx, shape, batch)
    bs.sfnn_integer_forward_device(ctx, shape, batch, b["max_active"], s, n, k, dq, ws)
    out = ws.download(ctx)
    q = oracle.sfnn_quantize(shape.as_tuple(), w)
    want = oracle.sfnn_integer_forward(shape.as_tuple(), b["stm"], b["nstm"], b["buckets"], batch, b["max_active"], q)
    np.testing.assert_array_equal(out["raw"], want["raw"])
    assert len(np.unique(out["raw"])) > batch // 4     # not a degenerate network


def test_integer_forward_counts_bad_inputs(ctx):
    shape = SMALL
    q = qc.random_integer_net(np.random.default_rng(3), shape.as_tuple(), False)
    batch = 64
    b = _batch(19, batch, shape.num_stacks, pad=False)
    b["stm"][5 * 40 + 2] = bs.HALFKA_HM2_DIMENSIONS + 10     # a virtual row id: not a table row
    b["nstm"][9 * 40 + 0] = 10 ** 6
    b["buckets"][11] = shape.num_stacks
    out = _run(ctx, shape, q, b["stm"], b["nstm"], b["buckets"], batch, b["max_active"])
    assert out["errors"] == 3
    assert out["raw"][11] == 0 and out["score"][11] == 0
    want = oracle.sfnn_integer_forward(shape.as_tuple(), b["stm"], b["nstm"], b["buckets"], batch, b["max_active"], q)
    np.testing.assert_array_equal(out["raw"], want["raw"])


def test_integer_forward_rejects_bad_rounding(ctx):
    shape, q = qc.ft_pair_net(254, 254)
    with pytest.raises(bo.CudaCppError, match="ft_shift"):
        _run(ctx, _shape(shape), q, [-1], [-1], [0], 1, 1, bs.QuantizedRounding(ft_shift=17))
    with pytest.raises(bo.CudaCppError, match="fv_scale"):
        _run(ctx, _shape(shape), q, [-1], [-1], [0], 1, 1, bs.QuantizedRounding(fv_scale=0))
