"""GPU parity of the quantised HalfKP path (configs[0], int16 FT / int8 dense /
ClippedReLU): device quantisation and integer forward bit-exact against the C
oracle, which tests/test_oracle_nnue_quant.py pins to the reference's writer."""
import numpy as np
import pytest

import bulletou_b200 as bo
from bulletou_b200 import synthetic
from oracle import oracle

pytestmark = pytest.mark.gpu

HALFKP = 125388
PIECES = 1548


def _weights(shape, seed, std=0.01):
    input_size, L1, L2, L3 = shape
    rng = np.random.default_rng(seed)
    n = {"l0w": input_size * L1, "l0b": L1, "l1w": 2 * L1 * L2, "l1b": L2, "l2w": L2 * L3, "l2b": L3,
         "outw": L3, "outb": 1}
    return {k: rng.normal(0, std, v).astype(np.float32) for k, v in n.items()}


def _quantize(ctx, shape, w):
    dq = bo.QuantizedNnueDeviceWeights(ctx, *shape)
    dw = {n: bo.F32Buffer.from_host(ctx, w[n]) for n in oracle.NNUE_QUANT_NAMES}
    bo.nnue_quantize_device(ctx, dw, dq)
    return dq


@pytest.mark.parametrize("shape", [(HALFKP, 256, 32, 32), (HALFKP + PIECES, 256, 32, 32), (1000, 96, 8, 16)],
                         ids=["configs0", "factorized", "generic"])
def test_quantize_vs_oracle(ctx, shape):
    w = _weights(shape, 3, std=0.02)
    w["l1w"][:3] = [0.5 / 64, -0.5 / 64, 5.0]      # ties away from zero, one saturating
    got = _quantize(ctx, shape, w).download(ctx)
    want = oracle.nnue_quantize(shape, w)
    assert got["errors"] == want["errors"] == 1
    for n in oracle.NNUE_QUANT_NAMES:
        np.testing.assert_array_equal(got[n], want[n], err_msg=n)


@pytest.mark.parametrize("shape,std", [((HALFKP, 256, 32, 32), 0.01), ((HALFKP, 256, 32, 32), 0.2),
                                       ((HALFKP + PIECES, 256, 32, 32), 0.2), ((1000, 96, 8, 16), 0.2)],
                         ids=["configs0", "wide", "factorized", "generic"])
def test_integer_forward_vs_oracle(ctx, shape, std):
    """N(0, 0.01) weights quantised by the reference scales, batch
    16384; and wider dense weights, which exercise every integer range."""
    w = _weights(shape, 5, std=0.01)
    if std != 0.01:
        for k in ("l1w", "l2w", "outw"):
            w[k] = (w[k] * (std / 0.01)).astype(np.float32)
        w["l0w"] = (w["l0w"] * 3).astype(np.float32)
    w["l0b"] = (np.abs(w["l0b"]) + 0.1).astype(np.float32)
    dq = _quantize(ctx, shape, w)
    q = oracle.nnue_quantize(shape, w)
    batch = 16384 if shape[0] >= HALFKP else 512
    if shape[0] >= HALFKP:
        b = synthetic.halfkp_batch(9, batch)
        stm, nstm, A = b["stm"], b["nstm"], b["max_active"]
    else:
        rng = np.random.default_rng(9)
        A = 12
        stm = rng.integers(-1, shape[0], batch * A).astype(np.int32)
        nstm = rng.integers(-1, shape[0], batch * A).astype(np.int32)
    s, n = bo.I32Buffer.from_host(ctx, stm), bo.I32Buffer.from_host(ctx, nstm)
    ws = bo.NnueIntegerForwardWorkspace(ctx, batch)
    bo.nnue_integer_forward_device(ctx, dq, batch, A, s, n, ws, 16)
    got = ws.download(ctx)
    want = oracle.nnue_integer_forward(shape, stm, nstm, batch, A, q, 16)
    assert got["errors"] == want["errors"] == 0
    np.testing.assert_array_equal(got["raw"], want["raw"])
    np.testing.assert_array_equal(got["score"], want["score"])
    if std != 0.01:
        assert len(np.unique(got["raw"])) > 16


def test_integer_forward_wraps_and_counts(ctx):
    shape = (HALFKP, 256, 32, 32)
    rng = np.random.default_rng(2)
    q = {"l0w": rng.integers(-32768, 32768, HALFKP * 256).astype(np.int16),
         "l0b": rng.integers(-100, 100, 256).astype(np.int16),
         "l1w": rng.integers(-128, 128, 32 * 512).astype(np.int8), "l1b": rng.integers(-9000, 9000, 32).astype(np.int32),
         "l2w": rng.integers(-128, 128, 32 * 32).astype(np.int8), "l2b": rng.integers(-9000, 9000, 32).astype(np.int32),
         "outw": np.concatenate([rng.integers(-128, 128, 32), np.zeros(0)]).astype(np.int8),
         "outb": np.array([77], np.int32)}
    dq = bo.QuantizedNnueDeviceWeights(ctx, *shape)
    dq.upload(q, ctx)
    batch = 1024
    b = synthetic.halfkp_batch(11, batch)
    stm, nstm = b["stm"].copy(), b["nstm"].copy()
    stm[7] = HALFKP + 3            # out of range: skipped, counted
    s, n = bo.I32Buffer.from_host(ctx, stm), bo.I32Buffer.from_host(ctx, nstm)
    ws = bo.NnueIntegerForwardWorkspace(ctx, batch)
    bo.nnue_integer_forward_device(ctx, dq, batch, b["max_active"], s, n, ws, 16)
    got = ws.download(ctx)
    want = oracle.nnue_integer_forward(shape, stm, nstm, batch, b["max_active"], q, 16)
    assert got["errors"] == want["errors"] == 1
    np.testing.assert_array_equal(got["raw"], want["raw"])
