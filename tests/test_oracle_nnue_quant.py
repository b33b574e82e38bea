"""CPU: the quantised HalfKP path of the C oracle (oracle_nnue_quantize,
oracle_nnue_integer_forward) against an independent numpy restatement of the
reference's nn.bin writer (write_cuda_cpp_nnue_nn_bin, examples/bulletou.rs:
26303-26413; l1_bias_scale / pad_weights_for_simd, crates/bulletou_lib/src/
value/nnue_save.rs:223-252, whose tests pin 127 * 64 and the padding) and of
the engine's halfkp_256x2-32-32 integer evaluation."""
import numpy as np
import pytest

from bulletou_b200 import synthetic
from oracle import oracle

HALFKP = 125388
PIECES = 1548


def _round_away(x):
    return np.sign(x) * np.floor(np.abs(x) + 0.5)


def quantize_numpy(shape, w):
    input_size, L1, L2, L3 = shape
    fact = input_size == HALFKP + PIECES
    l0 = np.asarray(w["l0w"], np.float32).reshape(input_size, L1)
    if fact:
        rows = np.arange(HALFKP)
        table = (l0[PIECES + rows] + l0[rows % PIECES]).astype(np.float32)
    else:
        table = l0

    def q(v, scale, lo, hi, dt):
        return np.clip(_round_away(np.float64(scale) * np.asarray(v, np.float64)), lo, hi).astype(dt)

    def dense(wi, n_in, n_out):   # input-major [n_in][n_out] -> output-major, padded to 32 inputs
        m = np.zeros((n_out, (n_in + 31) // 32 * 32), np.int8)
        m[:, :n_in] = q(np.asarray(wi, np.float32).reshape(n_in, n_out).T, 64, -128, 127, np.int8)
        return m.reshape(-1)

    return {"l0w": q(table, 127, -32768, 32767, np.int16).reshape(-1), "l0b": q(w["l0b"], 127, -32768, 32767, np.int16),
            "l1w": dense(w["l1w"], 2 * L1, L2), "l1b": q(w["l1b"], 8128, -2 ** 31, 2 ** 31 - 1, np.int32),
            "l2w": dense(w["l2w"], L2, L3), "l2b": q(w["l2b"], 8128, -2 ** 31, 2 ** 31 - 1, np.int32),
            "outw": dense(w["outw"], L3, 1), "outb": q(w["outb"], 8128, -2 ** 31, 2 ** 31 - 1, np.int32)}


def forward_numpy(shape, stm, nstm, batch, A, q, fv_scale=16):
    input_size, L1, L2, L3 = shape
    rows = HALFKP if input_size == HALFKP + PIECES else input_size
    l0w = np.asarray(q["l0w"], np.int64).reshape(rows, L1)

    def view(idx):
        idx = np.asarray(idx, np.int64).reshape(batch, A)
        acc = np.repeat(np.asarray(q["l0b"], np.int64)[None], batch, axis=0)
        for k in range(A):
            f = idx[:, k]
            ok = (f >= 0) & (f < rows)
            acc[ok] += l0w[f[ok]]
        acc = ((acc + 32768) % 65536) - 32768
        return np.clip(acc, 0, 127)

    x = np.concatenate([view(stm), view(nstm)], axis=1)

    def affine(inp, wq, bq, n_in, n_out):
        m = np.asarray(wq, np.int64).reshape(n_out, -1)[:, :n_in]
        return inp @ m.T + np.asarray(bq, np.int64)[None]

    h1 = np.clip(affine(x, q["l1w"], q["l1b"], 2 * L1, L2) >> 6, 0, 127)
    h2 = np.clip(affine(h1, q["l2w"], q["l2b"], L2, L3) >> 6, 0, 127)
    raw = affine(h2, q["outw"], q["outb"], L3, 1)[:, 0]
    score = np.sign(raw) * (np.abs(raw) // fv_scale)
    return raw.astype(np.int32), score.astype(np.int32)


def _weights(shape, rng, std=0.01):
    input_size, L1, L2, L3 = shape
    n = {"l0w": input_size * L1, "l0b": L1, "l1w": 2 * L1 * L2, "l1b": L2, "l2w": L2 * L3, "l2b": L3,
         "outw": L3, "outb": 1}
    return {k: rng.normal(0, std, v).astype(np.float32) for k, v in n.items()}


@pytest.mark.parametrize("factorized", [False, True])
def test_quantize_matches_writer_restatement(factorized):
    shape = (HALFKP + PIECES if factorized else HALFKP, 256, 32, 32)
    rng = np.random.default_rng(1)
    w = _weights(shape, rng, 0.05)
    w["l1w"][:4] = [0.5 / 64, -0.5 / 64, 2.5 / 64, 300.0]   # ties away from zero, one out of range
    q = oracle.nnue_quantize(shape, w)
    ref = quantize_numpy(shape, w)
    assert q["errors"] == 1
    for k in oracle.NNUE_QUANT_NAMES:
        np.testing.assert_array_equal(q[k], ref[k], err_msg=k)
    # l1w is output-major: input 0 of output 0 .. output 3 came from l1w[0:4]
    assert q["l1w"][0] == 1 and q["l1w"][512] == -1 and q["l1w"][2 * 512] == 3 and q["l1w"][3 * 512] == 127


def test_bias_scale_and_padding_known_answers():
    """l1_bias_scale(CReLU, false, 127, 64) = 127 * 64 and pad32 rows
    (nnue_save.rs:286-291, 262-283)."""
    shape = (8, 4, 3, 2)
    w = {"l0w": np.zeros(32, np.float32), "l0b": np.zeros(4, np.float32), "l1w": np.zeros(24, np.float32),
         "l1b": np.array([1.0, -1.0, 0.5], np.float32), "l2w": np.zeros(6, np.float32),
         "l2b": np.zeros(2, np.float32), "outw": np.array([1.0, 2.0], np.float32), "outb": np.zeros(1, np.float32)}
    q = oracle.nnue_quantize(shape, w)
    assert q["l1b"].tolist() == [8128, -8128, 4064]
    assert q["l1w"].size == 3 * 32 and q["outw"].size == 32 and q["outw"][:3].tolist() == [64, 127, 0]
    assert q["errors"] == 1   # 2.0 * 64 = 128 is outside i8


@pytest.mark.parametrize("factorized", [False, True])
def test_integer_forward_matches_restatement(factorized):
    shape = (HALFKP + PIECES if factorized else HALFKP, 256, 32, 32)
    rng = np.random.default_rng(2)
    w = _weights(shape, rng, 0.05)
    w["l0b"] = (np.abs(w["l0b"]) + 0.2).astype(np.float32)
    q = oracle.nnue_quantize(shape, w)
    batch = 64
    b = synthetic.halfkp_batch(5, batch)
    stm, nstm = b["stm"].copy(), b["nstm"].copy()
    stm[::9] = -1
    out = oracle.nnue_integer_forward(shape, stm, nstm, batch, b["max_active"], q)
    raw, score = forward_numpy(shape, stm, nstm, batch, b["max_active"], q)
    assert out["errors"] == 0
    np.testing.assert_array_equal(out["raw"], raw)
    np.testing.assert_array_equal(out["score"], score)
    assert len(np.unique(raw)) > batch // 4


def test_integer_forward_wraps_the_i16_accumulator():
    shape = (4, 4, 1, 1)
    q = {"l0w": np.full(16, 20000, np.int16), "l0b": np.zeros(4, np.int16),
         "l1w": np.zeros(32, np.int8), "l1b": np.zeros(1, np.int32), "l2w": np.zeros(32, np.int8),
         "l2b": np.zeros(1, np.int32), "outw": np.zeros(32, np.int8), "outb": np.zeros(1, np.int32)}
    q["l1w"][0] = 1                      # output 0 reads stm column 0
    q["l2w"][0] = 64                     # h2 = h1 after >> 6 twice... h1 = x >> 6
    q["outw"][0] = 1
    # two rows: 40000 wraps to -25536 -> 0; one row: 20000 -> 127
    for feats, x0 in (([0, 1], 0), ([0, -1], 127)):
        out = oracle.nnue_integer_forward(shape, feats, [-1, -1], 1, 2, q)
        assert out["raw"][0] == ((x0 >> 6) * 64 >> 6)
