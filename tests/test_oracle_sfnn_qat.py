"""CPU: pins the SFNN QAT modes of the C oracle (oracle_sfnn_forward_qat /
oracle_sfnn_backward_qat) to the reference's own QAT tests, restated on the CPU:
  - L1 QAT = the f32 net with fold-then-round L1 weights, identity STE
    (sfnn_qat_l1_forward_ste_and_export_parity, crates/cuda_cpp/src/qat_tests.rs:165-330);
  - FT layer QAT = the net with Q(fold(l0w)) and zeroed virtual rows
    (selected_qat_rounding_and_ft_fold, layer_qat.rs:681-705);
  - dense QAT integer FT pair product (dense_qat_ft_forward_uses_integer_pair_product,
    layer_qat.rs:20-36), the integer L1 / L2 / L3 path against an independent
    integer restatement (tests/dense_qat_reference.rs), and gradients against
    finite differences of the lattice loss
    (sgd_dense_qat_output_bias_gradient_matches_lattice_loss_difference,
    sgd_dense_qat_shared_skip_bias_matches_lattice_loss_difference, layer_qat.rs:149-230)."""
import numpy as np
import pytest

from oracle import oracle

PIECES = 1629


def _runner(goldens):
    g = goldens["tiny_sfnn_runner"]
    w = {k: np.asarray(v, np.float32) for k, v in g["weights"].items()}
    return g, tuple(g["shape"]), w


def qdq(x, scale, lo, hi):
    """(x * scale).round().clamp(lo, hi) / scale in f32, ties away from zero
    (qat_tests.rs:161-163)."""
    x = np.asarray(x, np.float32)
    s = (x * np.float32(scale)).astype(np.float32)
    q = np.sign(s) * np.floor(np.abs(s) + np.float32(0.5))
    return (np.clip(q, lo, hi).astype(np.float32) / np.float32(scale)).astype(np.float32)


def _fwd_bwd(shape, w, stm, nstm, buckets, batch, A, targets, qat, alphas=(1.0, 1.0), kind=0):
    f = oracle.sfnn_forward(shape, stm, nstm, buckets, batch, A, w, *alphas, qat=qat)
    loss = oracle.scalar_loss(kind, 1.0, 2.0, 0.0, f["output"], targets, np.ones(batch, np.float32))
    g = oracle.sfnn_backward(shape, stm, nstm, buckets, batch, A, f, w, loss["mean_output_gradients"], *alphas,
                             qat=qat)
    return f, loss, g


def test_l1_qat_is_fold_then_round_with_identity_ste(goldens):
    g, shape, w = _runner(goldens)
    _, W, H, skip, L2, S = shape
    O = H + 1
    w = dict(w)
    w["l1w"] = w["l1w"].copy()
    w["l1w"][:4] = [-0.5 / 64, 0.5 / 64, -8.0, 8.0]          # ties away from zero, both saturation edges
    w["l1fw"] = (0.01 * (np.arange(W * O) - 3.0)).astype(np.float32)
    w["l1fb"] = np.full(O, 0.002, np.float32)
    w.pop("l2fw"), w.pop("l2fb"), w.pop("l3fw"), w.pop("l3fb")
    alpha = 0.7
    fold_w = np.empty(S * O * W, np.float32)
    fold_b = np.empty(S * O, np.float32)
    for s in range(S):
        for o in range(O):
            b = np.float32(w["l1b"][s * O + o]) + np.float32(alpha) * w["l1fb"][o]
            fold_b[s * O + o] = b
            for i in range(W):
                fold_w[(s * O + o) * W + i] = (np.float32(w["l1w"][(s * O + o) * W + i])
                                              + np.float32(alpha) * w["l1fw"][i * O + o])
    fake = dict(w, l1w=qdq(fold_w, 64.0, -128, 127), l1b=qdq(fold_b, 8128.0, -2 ** 31, 2 ** 31 - 1))
    fake.pop("l1fw"), fake.pop("l1fb")
    args = (g["stm"], g["nstm"], g["buckets"], g["batch"], g["max_active"], g["targets"])
    fq, lq, gq = _fwd_bwd(shape, w, *args, qat=oracle.QAT_L1, alphas=(1.0, alpha))
    ff, lf, gf = _fwd_bwd(shape, fake, *args, qat=0, alphas=(1.0, alpha))
    np.testing.assert_allclose(fq["output"], ff["output"], rtol=0, atol=1e-6)
    for k in ("l0w_gradients", "l0b_gradients", "l1w_gradients", "l1b_gradients", "l2w_gradients", "l3w_gradients",
              "combined_gradients"):
        np.testing.assert_allclose(gq[k], gf[k], rtol=0, atol=1e-6, err_msg=k)
    # STE through the fold: the shared factor receives alpha * sum over stacks.
    sg = np.zeros(W * O)
    sb = np.zeros(O)
    for s in range(S):
        for o in range(O):
            sb[o] += alpha * gf["l1b_gradients"][s * O + o]
            for i in range(W):
                sg[i * O + o] += alpha * gf["l1w_gradients"][(s * O + o) * W + i]
    np.testing.assert_allclose(gq["l1fw_gradients"], sg, rtol=0, atol=1e-6)
    np.testing.assert_allclose(gq["l1fb_gradients"], sb, rtol=0, atol=1e-6)


def test_ft_layer_qat_folds_virtual_rows_then_rounds():
    rng = np.random.default_rng(4)
    base = 73305
    shape = (base + PIECES, 8, 3, 1, 4, 2)
    W = shape[1]
    w = {"l0w": rng.normal(0, 0.05, shape[0] * W).astype(np.float32),
         "l0b": rng.uniform(0.1, 0.4, W).astype(np.float32),
         "l1w": rng.normal(0, 0.5, 2 * 4 * W).astype(np.float32), "l1b": rng.normal(0, 0.1, 8).astype(np.float32),
         "l2w": rng.normal(0, 0.5, 2 * 4 * 6).astype(np.float32), "l2b": rng.normal(0, 0.1, 8).astype(np.float32),
         "l3w": rng.normal(0, 0.5, 8).astype(np.float32), "l3b": rng.normal(0, 0.1, 2).astype(np.float32)}
    alpha = np.float32(0.75)
    l0 = w["l0w"].reshape(-1, W)
    fold = (l0[:base] + (alpha * l0[base + np.arange(base) % PIECES]).astype(np.float32)).astype(np.float32)
    ql0 = np.zeros_like(l0)
    ql0[:base] = qdq(fold, 127.0, -32768, 32767)
    fake = dict(w, l0w=ql0.reshape(-1), l0b=qdq(w["l0b"], 127.0, -32768, 32767))
    batch, A = 6, 5
    stm = rng.integers(0, base, batch * A).astype(np.int32)
    nstm = rng.integers(0, base, batch * A).astype(np.int32)
    buckets = np.array([0, 1, 0, 1, 1, 0], np.int32)
    t = rng.uniform(0, 1, batch).astype(np.float32)
    fq, _, gq = _fwd_bwd(shape, w, stm, nstm, buckets, batch, A, t, qat=oracle.QAT_FT, alphas=(float(alpha), 1.0))
    ff, _, gf = _fwd_bwd(shape, fake, stm, nstm, buckets, batch, A, t, qat=0, alphas=(float(alpha), 1.0))
    for k in ("stm_l0", "combined", "output"):
        np.testing.assert_array_equal(fq[k], ff[k], err_msg=k)
    for k in ("l0w_gradients", "l0b_gradients", "l1w_gradients"):
        np.testing.assert_allclose(gq[k], gf[k], rtol=0, atol=1e-7, err_msg=k)


def test_dense_qat_integer_ft_pair_product(goldens):
    """layer_qat.rs:20-36: zero FT weights, FT bias 64/127 -> every combined
    value is ((2 * 64) * (2 * 64)) >> 9 = 32 over 127."""
    g, shape, w = _runner(goldens)
    w = dict(w, l0w=np.zeros_like(w["l0w"]), l0b=np.full(shape[1], 64.0 / 127.0, np.float32))
    for k in ("l2fw", "l2fb", "l3fw", "l3fb"):
        w.pop(k)
    qat = oracle.qat_mask(l1=True, ft=True, l2=True, l3=True)
    f = oracle.sfnn_forward(shape, [0], [0], [0], 1, 1, w, qat=qat)
    np.testing.assert_allclose(f["combined"], np.full(shape[1], 32.0 / 127.0), rtol=0, atol=1e-7)


def _integer_restatement(shape, w, f, buckets, batch, alpha=1.0):
    """tests/dense_qat_reference.rs restated: weight round(64 w), bias
    round(8128 b), input floor(127 x), activations >> 6 and x^2 >> 19."""
    _, W, H, skip, L2, S = shape
    O = H + (1 if skip else 0)

    def wq(v):
        x = np.float64(v) * 64.0
        return int(np.clip(np.sign(x) * np.floor(abs(x) + 0.5), -128, 127))

    def bq(v):
        x = np.float64(v) * 8128.0
        return int(np.clip(np.sign(x) * np.floor(abs(x) + 0.5), -2 ** 31, 2 ** 31 - 1))

    out = np.zeros(batch)
    c = f["combined"].reshape(batch, W)
    for b in range(batch):
        s = buckets[b]
        x = [int(round(float(v) * 127.0)) for v in c[b]]   # the forward's lattice values n / 127
        raw1 = []
        for o in range(O):
            wf = np.float32(w["l1w"][(s * O + o) * W:(s * O + o + 1) * W])
            if "l1fw" in w:
                wf = (wf + np.float32(alpha) * np.asarray(w["l1fw"], np.float32).reshape(W, O)[:, o]).astype(np.float32)
            bb = np.float32(w["l1b"][s * O + o])
            if "l1fb" in w:
                bb = np.float32(bb + np.float32(alpha) * np.float32(w["l1fb"][o]))
            raw1.append(bq(bb) + sum(xi * wq(v) for xi, v in zip(x, wf)))
        inp = [min(127, (r * r) >> 19) for r in raw1[:H]] + [min(127, max(0, r >> 6)) for r in raw1[:H]]
        l2 = []
        for o in range(L2):
            r2 = bq(w["l2b"][s * L2 + o]) + sum(v * wq(w["l2w"][(s * L2 + o) * 2 * H + i]) for i, v in enumerate(inp))
            l2.append(min(127, max(0, r2 >> 6)))
        r3 = bq(w["l3b"][s]) + sum(v * wq(w["l3w"][s * L2 + o]) for o, v in enumerate(l2))
        if skip:
            r3 += raw1[H]
        out[b] = np.float32(r3 / 8128.0)
    return out


def test_dense_qat_integer_path_matches_integer_restatement(goldens):
    g, shape, w = _runner(goldens)
    w = {k: v for k, v in w.items() if k not in ("l2fw", "l2fb", "l3fw", "l3fb")}
    rng = np.random.default_rng(9)
    w["l0w"] = rng.normal(0.1, 0.3, w["l0w"].size).astype(np.float32)
    w["l1w"] = rng.normal(0, 1.0, w["l1w"].size).astype(np.float32)
    w["l2w"] = rng.normal(0, 1.0, w["l2w"].size).astype(np.float32)
    batch, A = 8, 3
    stm = rng.integers(-1, 4, batch * A).astype(np.int32)
    nstm = rng.integers(-1, 4, batch * A).astype(np.int32)
    buckets = rng.integers(0, shape[5], batch).astype(np.int32)
    qat = oracle.qat_mask(l1=True, l2=True, l3=True)
    f = oracle.sfnn_forward(shape, stm, nstm, buckets, batch, A, w, qat=qat)
    c = f["combined"].reshape(batch, -1)
    np.testing.assert_array_equal(np.round(c * 127) / 127, c)       # FT output on the 1/127 lattice
    ref = _integer_restatement(shape, w, f, buckets, batch)
    np.testing.assert_array_equal(f["output"], ref.astype(np.float32))


@pytest.mark.parametrize("which", ["l3b", "l1fb"])
def test_dense_qat_bias_gradient_matches_lattice_loss_difference(goldens, which):
    g, shape, w = _runner(goldens)
    w = {k: v for k, v in w.items() if k not in ("l2fw", "l2fb", "l3fw", "l3fb")}
    w["l3b"] = np.zeros(2, np.float32)
    if which == "l1fb":
        w["l1fb"] = np.zeros(3, np.float32)
    qat = oracle.qat_mask(l1=True, l2=True, l3=True)
    stm, nstm, buckets, t = [0], [2], [0], np.ones(1, np.float32)

    def loss_at(delta):
        ww = dict(w)
        if which == "l3b":
            ww["l3b"] = np.array([delta, 0.0], np.float32)
        else:
            ww["l1fb"] = np.array([0.0, 0.0, delta], np.float32)
        f, loss, gr = _fwd_bwd(shape, ww, stm, nstm, buckets, 1, 1, t, qat=qat, kind=2)
        z = float(f["output"][0])
        return np.log1p(np.exp(-z)), gr

    base, gr = loss_at(0.0)
    grad = gr["l3b_gradients"][0] if which == "l3b" else gr["l1fb_gradients"][2]
    h = 1.0 / 8128.0
    plus, _ = loss_at(h)
    minus, _ = loss_at(-h)
    finite = (plus - minus) / (2 * np.float32(h))
    assert abs(finite - grad) < 1e-3, (base, grad, finite)


def test_dense_qat_zero_lattice_keeps_positive_ste():
    """A raw L1 value of 1 rounds to 0 on both branches but keeps both STE
    derivatives (tests/dense_qat_reference.rs:49-62)."""
    shape = (4, 2, 1, 0, 1, 1)
    w = {"l0w": np.zeros(8, np.float32), "l0b": np.zeros(2, np.float32),
         "l1w": np.zeros(2, np.float32), "l1b": np.array([1.0 / 8128.0], np.float32),
         "l2w": np.array([1.0, 1.0], np.float32), "l2b": np.array([0.5], np.float32),
         "l3w": np.array([1.0], np.float32), "l3b": np.zeros(1, np.float32)}
    qat = oracle.qat_mask(l1=True, l2=True, l3=True)
    f, loss, g = _fwd_bwd(shape, w, [-1], [-1], [0], 1, 1, np.ones(1, np.float32), qat=qat, kind=2)
    assert f["l1_raw"][0] == 1 and f["l2_input"][0] == 0 and f["l2_input"][1] == 0
    assert g["l1_gradients"][0] != 0.0
    assert g["l1b_gradients"][0] == g["l1_gradients"][0]
