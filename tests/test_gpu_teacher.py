"""GPU parity of the device teacher-batch producer
(bulletou_b200_teacher_prepare_device) against the CPU oracle restatement of
the reference's host producer (teacher_batch.rs:1687-1750, 2869-3010 with the
PackedSfenValue decode of packed_sfen.rs and the feature maps of
shogi_halfka_hm2.rs / shogi_halfkp.rs): feature rows, buckets and entry
weights bit-exact, targets bit-exact through the win-rate table and within 2
ulp through the sigmoid; then train steps fed from records against steps fed
from the oracle's batch."""
import numpy as np
import pytest

import bulletou_b200 as bo
from bulletou_b200 import sfnn as bs
from bulletou_b200 import synthetic as syn
from bulletou_b200 import teacher as bt
from oracle import oracle
from oracle import teacher as ot
from tests.conftest import assert_close_scaled

pytestmark = pytest.mark.gpu

BUCKET_KINDS = [("none", "kingrank9"), ("none", "none"), ("hand1024", "kingrank9"), ("hand64z", "k29k29"),
                ("hand256", "k13k13z"), ("hand4", "k9k9z"), ("hand16", "kingrank81"), ("hand64", "k21k21z"),
                ("none", "k21k21")]


def _cfg(fs="halfka_hm2", hand="none", king="kingrank9", lam=0.7, scale=600.0, drop=None, wrm=False):
    return bt.TeacherBatchConfig(feature_set=fs, lambda_=lam, scale=scale, score_drop_abs=drop,
                                 win_rate_model=wrm, layerstack_bucket=bt.LayerStackBucketKind(hand, king))


def _oracle(cfg: bt.TeacherBatchConfig, recs):
    lb = cfg.layerstack_bucket
    o = ot.config(cfg.feature_set, cfg.active, lb.hand, lb.king, cfg.lambda_, cfg.scale, cfg.score_drop_abs)
    table = bt.win_rate_model_score_table(cfg.wrm_target) if cfg.win_rate_model else None
    return ot.prepare(recs, o, table)


def _device(ctx, cfg, recs):
    n = np.asarray(recs).view(np.uint8).size // 40
    prod = bt.TeacherBatchProducer(ctx, cfg, n, pinned=False)
    out = prod.new_batch()
    prod.prepare(ctx, recs, out)
    got = out.download(ctx)
    got["overflow"] = int(prod.overflow.download(ctx)[0])
    return got


def _compare(got, want, cfg, exact_targets=None):
    A = cfg.active
    np.testing.assert_array_equal(got["stm"], want["stm"])
    np.testing.assert_array_equal(got["nstm"], want["nstm"])
    if cfg.feature_set == "halfka_hm2":
        np.testing.assert_array_equal(got["buckets"], want["buckets"])
    np.testing.assert_array_equal(got["entry_weights"], want["entry_weights"])
    assert got["overflow"] == int((want["counts"] > A).sum())
    ulp = np.abs(got["targets"].view(np.int32).astype(np.int64) - want["targets"].view(np.int32).astype(np.int64))
    if exact_targets if exact_targets is not None else cfg.win_rate_model:
        assert ulp.max() == 0
    else:
        # exp in double rounded once vs the C library's expf: 1 ulp of p(score),
        # at most 2 after the blend's product and sum
        assert ulp.max() <= 2 and (ulp == 0).mean() > 0.999


@pytest.mark.parametrize("hand,king", BUCKET_KINDS)
def test_halfka_hm2_full_set_records_vs_oracle(ctx, hand, king):
    recs = syn.psv_records(11, 4096, hand_fraction=0.2, promote_fraction=0.15)
    cfg = _cfg("halfka_hm2", hand, king, drop=900)
    want = _oracle(cfg, recs)
    assert (want["counts"] == 40).all()
    _compare(_device(ctx, cfg, recs), want, cfg)


@pytest.mark.parametrize("lam", [0.0, 0.35, 1.0])
def test_halfkp_full_set_records_vs_oracle(ctx, lam):
    recs = syn.psv_records(12, 4096, hand_fraction=0.2, promote_fraction=0.15)
    cfg = _cfg("halfkp", lam=lam, scale=510.0, drop=1200)
    want = _oracle(cfg, recs)
    assert (want["counts"] == 38).all()
    _compare(_device(ctx, cfg, recs), want, cfg)


@pytest.mark.parametrize("n", [1, 63, 64, 65, 1000])
@pytest.mark.parametrize("fs", ["halfka_hm2", "halfkp"])
def test_ragged_record_counts(ctx, n, fs):
    recs = syn.psv_records(13 + n, n)
    cfg = _cfg(fs, wrm=True)
    _compare(_device(ctx, cfg, recs), _oracle(cfg, recs), cfg)


@pytest.mark.parametrize("fs", ["halfka_hm2", "halfkp"])
def test_random_bytes_and_overflow_count(ctx, fs):
    """Any bit pattern: garbage kings (no features), boards that decode to more
    than max_active features (counted, first max_active kept), reads past bit
    256 (zeros)."""
    rng = np.random.default_rng(17)
    recs = rng.integers(0, 256, (20000, 40), dtype=np.uint8)
    cfg = _cfg(fs, "hand64z" if fs == "halfka_hm2" else "none", "k29k29", drop=0)
    want = _oracle(cfg, recs)
    assert (want["counts"] > cfg.active).sum() > 1000
    _compare(_device(ctx, cfg, recs), want, cfg)


@pytest.mark.parametrize("fs", ["halfka_hm2", "halfkp"])
def test_bit_flipped_records(ctx, fs):
    rng = np.random.default_rng(19)
    recs = syn.psv_records(21, 8192).view(np.uint8).reshape(-1, 40).copy()
    for _ in range(3):
        rows = np.arange(recs.shape[0])
        bit = rng.integers(0, 256, recs.shape[0])
        recs[rows, bit // 8] ^= (1 << (bit % 8)).astype(np.uint8)
    cfg = _cfg(fs, "hand1024" if fs == "halfka_hm2" else "none", "kingrank81", lam=0.5)
    want = _oracle(cfg, recs)
    assert ((want["counts"] > 0) & (want["counts"] < cfg.active)).any()
    _compare(_device(ctx, cfg, recs), want, cfg)


def test_short_material_and_kingless_records(ctx):
    """Handicap-style positions padded with piece-box pieces, and records with
    a king square of 81 or more (no features, bucket from the wrapped square)."""
    rng = syn.rng_for(23)
    p = syn.psv_positions(rng, 3000, hand_fraction=0.3)
    drop = rng.random(p["board"].shape) < 0.3
    p["board"][drop] = 0
    p["hands"] = np.where(rng.random(p["hands"].shape) < 0.5, 0, p["hands"])
    recs = []
    for i in range(3000):
        try:
            recs.append(syn.psv_encode(p["stm"][i], p["black_king"][i], p["white_king"][i], p["board"][i][None],
                                       p["hands"][i][None], int(rng.integers(-3000, 3000)), int(rng.integers(-1, 2))))
        except ValueError:                       # a 1-bit tail cannot be padded
            continue
    recs = np.concatenate(recs)
    kingless = recs.view(np.uint8).reshape(-1, 40)[:400].copy()
    kingless[:, 1] |= 0xFE                                          # black king bits 1..6 set: square >= 81
    allrecs = np.concatenate([recs.view(np.uint8).reshape(-1, 40), kingless])
    for fs, hand, king in (("halfka_hm2", "hand256", "kingrank9"), ("halfka_hm2", "none", "k29k29"),
                           ("halfkp", "none", "none")):
        cfg = _cfg(fs, hand, king, drop=2500)
        want = _oracle(cfg, allrecs)
        assert (want["counts"][-400:] == 0).all()
        _compare(_device(ctx, cfg, allrecs), want, cfg)


def test_production_batch_win_rate_targets(ctx):
    """configs[2]'s batch: 65536 records, HalfKA_hm2, k3k3 buckets, lambda 1,
    win-rate-model targets (the reference's default training target)."""
    recs = syn.psv_records(29, 65536)
    cfg = _cfg("halfka_hm2", "none", "kingrank9", lam=1.0, wrm=True)
    got = _device(ctx, cfg, recs)
    _compare(got, _oracle(cfg, recs), cfg)
    assert got["overflow"] == 0 and (got["stm"] >= 0).all()
    assert set(np.unique(got["buckets"])) <= set(range(9))


def test_overflow_raises_like_the_reference(ctx):
    rng = np.random.default_rng(31)
    recs = rng.integers(0, 256, (256, 40), dtype=np.uint8)
    cfg = _cfg("halfka_hm2")
    prod = bt.TeacherBatchProducer(ctx, cfg, 256, pinned=False)
    out = prod.new_batch()
    prod.prepare(ctx, recs, out)
    with pytest.raises(bo.CudaCppError, match="exceeded max_active 40"):
        prod.check(ctx)
    prod.prepare(ctx, syn.psv_records(1, 256), out)
    prod.check(ctx)                                                 # clean batch: no new overflow


def _ranger(step):
    return bo.RangerUpdateParams(radam=bo.RAdamUpdateParams(step=step, learning_rate=1e-3))


def test_sfnn_steps_from_records_match_oracle_batches(ctx):
    """The fused SFNN step fed by device-decoded records equals the same step
    fed with the oracle's host batch, bit for bit."""
    shape = bs.SfnnForwardShape(bs.HALFKA_HM2_DIMENSIONS + bs.PIECE_INPUTS, 256, 15, True, 32, 9)
    w = syn.sfnn_weights(syn.rng_for(3), shape.input_size, shape.ft_size, shape.l1_hidden, shape.l1_skip,
                         shape.l2_size, shape.num_stacks, True, False, 0.05)
    B = 2048
    cfg = _cfg("halfka_hm2", lam=1.0, wrm=True)
    a = bs.SfnnTrainStepRunner(ctx, bs.SfnnForwardHostWeights(shape, **w), B, 40)
    b = bs.SfnnTrainStepRunner(ctx, bs.SfnnForwardHostWeights(shape, **w), B, 40)
    prod = bt.TeacherBatchProducer(ctx, cfg, B, pinned=False)
    loss = bo.ScalarLossKind.SigmoidPow(2.0)
    for step in range(1, 4):
        recs = syn.psv_records(40 + step, B)
        a.step_from_records(ctx, _ranger(step), loss, 1 / 600, prod, recs)
        o = _oracle(cfg, recs)
        b.step_no_readback(ctx, _ranger(step), loss, 1 / 600,
                           bs.SfnnTrainStepHostBatch(o["stm"].reshape(-1), o["nstm"].reshape(-1), o["buckets"],
                                                     o["targets"], o["entry_weights"], B, 40))
        assert a.read_loss(ctx).mean == b.read_loss(ctx).mean
    wa, wb = a.read_weights(ctx), b.read_weights(ctx)
    for k in wa:
        np.testing.assert_array_equal(wa[k], wb[k], err_msg=k)
    prod.check(ctx)


def test_sfnn_pipelined_record_steps(ctx):
    """step_pipelined_records (two slots, decode on the upload stream) gives
    the same weights as step_from_records on one stream."""
    shape = bs.SfnnForwardShape(bs.HALFKA_HM2_DIMENSIONS + bs.PIECE_INPUTS, 256, 15, True, 32, 9)
    w = syn.sfnn_weights(syn.rng_for(4), shape.input_size, shape.ft_size, shape.l1_hidden, shape.l1_skip,
                         shape.l2_size, shape.num_stacks, True, False, 0.05)
    B = 1024
    cfg = _cfg("halfka_hm2", lam=0.5)
    a = bs.SfnnTrainStepRunner(ctx, bs.SfnnForwardHostWeights(shape, **w), B, 40)
    b = bs.SfnnTrainStepRunner(ctx, bs.SfnnForwardHostWeights(shape, **w), B, 40)
    prod = bt.TeacherBatchProducer(ctx, cfg, B)
    upload = bo.Context(ctx.device)
    loss = bo.ScalarLossKind.SigmoidPow(2.0)
    batches = [syn.psv_records(60 + i, B) for i in range(5)]
    for step, recs in enumerate(batches, 1):
        a.step_pipelined_records(ctx, upload, prod, _ranger(step), loss, 1 / 600, recs)
        b.step_from_records(ctx, _ranger(step), loss, 1 / 600, prod, recs)
    ctx.synchronize()
    wa, wb = a.read_weights(ctx), b.read_weights(ctx)
    for k in wa:
        np.testing.assert_array_equal(wa[k], wb[k], err_msg=k)


def test_halfkp_steps_from_records_match_oracle_batches(ctx):
    shape = bo.NNUE_HALFKP_256X2_32_32
    w = syn.halfkp_weights(syn.rng_for(5), std=0.05)
    B = 2048
    cfg = _cfg("halfkp", lam=0.5, scale=600.0)
    a = bo.NnueTrainStepRunner(ctx, bo.NnueForwardHostWeights(shape, **w), B, 38)
    b = bo.NnueTrainStepRunner(ctx, bo.NnueForwardHostWeights(shape, **w), B, 38)
    prod = bt.TeacherBatchProducer(ctx, cfg, B, pinned=False)
    loss = bo.ScalarLossKind.SigmoidPow(2.0)
    for step in range(1, 4):
        recs = syn.psv_records(80 + step, B)
        o = _oracle(cfg, recs)
        a.step_from_records(ctx, _ranger(step), loss, 1 / 600, prod, recs)
        # the oracle's targets may differ by 1 ulp through expf: feed the device's own targets
        dev = prod.new_batch()
        prod.prepare(ctx, recs, dev)
        t = dev.targets.download(ctx)
        np.testing.assert_allclose(t, o["targets"], rtol=2e-7, atol=0)
        b.step_no_readback(ctx, _ranger(step), loss, 1 / 600,
                           bo.NnueTrainStepHostBatch(o["stm"].reshape(-1), o["nstm"].reshape(-1), t,
                                                     o["entry_weights"], B, 38))
        assert a.read_loss(ctx).mean == b.read_loss(ctx).mean


def oracle_sfnn_trainer(shape, w, qat):
    return oracle.SfnnTrainer(shape.as_tuple(), w, qat=qat)


def _heavy_rows(stm, nstm, threshold=512):
    rows = np.concatenate([stm.reshape(-1), nstm.reshape(-1)])
    counts = np.bincount(rows[rows >= 0])
    return int((counts > threshold).sum()), int(counts.max())


@pytest.mark.parametrize("qat", ["none", "dense_ft"])
def test_fused_steps_on_record_batches_vs_oracle(ctx, qat):
    """Real teacher data concentrates the kings near their home squares, so a
    few FT rows collect thousands of entries (the heavy-row segment path of
    the row kernel); the fused step still matches the oracle trainer."""
    from tests.test_gpu_sfnn_qat import MODES, _mask, _weights

    lr = bs.SfnnLayerLrMultipliers() if qat == "none" else MODES[qat]
    shape = bs.SfnnForwardShape(bs.HALFKA_HM2_DIMENSIONS + bs.PIECE_INPUTS, 256, 15, True, 32, 9)
    w = _weights(shape, 91)
    B = 8192
    cfg = _cfg("halfka_hm2", lam=0.6)
    runner = bs.SfnnTrainStepRunner(ctx, bs.SfnnForwardHostWeights(shape, **w), B, 40, lr_multipliers=lr)
    assert runner.fused
    trainer = oracle_sfnn_trainer(shape, w, _mask(lr))
    prod = bt.TeacherBatchProducer(ctx, cfg, B, pinned=False)
    loss = bo.ScalarLossKind.SigmoidPow(2.0)
    for step in range(1, 4):
        recs = syn.psv_records(100 + step, B)
        o = _oracle(cfg, recs)
        heavy, biggest = _heavy_rows(o["stm"], o["nstm"])
        assert heavy > 0 and biggest > 2 * 512
        runner.step_from_records(ctx, _ranger(step), loss, 1 / 600, prod, recs)
        dev = prod.new_batch()
        prod.prepare(ctx, recs, dev)
        t = dev.targets.download(ctx)
        trainer.step(o["stm"].reshape(-1), o["nstm"].reshape(-1), o["buckets"], B, 40, t, o["entry_weights"],
                     step=step, learning_rate=1e-3, inv_scale=1 / 600)
    got = runner.read_weights(ctx)
    for nm in trainer.names:
        assert_close_scaled(got[nm], trainer.w[nm], 1e-4, nm)


# ------------------------------------------------------------------ HCPE records
def _hcpe_device(ctx, recs):
    n = np.asarray(recs).view(np.uint8).size // 38
    conv = bt.HcpeConverter(ctx, max(n, 1))
    count = conv.convert(ctx, recs)
    psv = conv.psv.download(ctx).view(np.uint8).reshape(-1, 40)[:count]
    return psv, conv.valid.download(ctx)[:n], count


@pytest.mark.parametrize("n", [1, 63, 65, 4096])
def test_hcpe_full_set_records_vs_oracle(ctx, n):
    recs = syn.hcpe_records(50 + n, n, hand_fraction=0.25, promote_fraction=0.2)
    want, wvalid = ot.hcpe_to_psv(recs)
    got, valid, count = _hcpe_device(ctx, recs)
    assert count == n == wvalid.sum()
    np.testing.assert_array_equal(valid, wvalid)
    np.testing.assert_array_equal(got, want)


def test_hcpe_random_and_short_records_vs_oracle(ctx):
    """Random bytes (kings out of range, unknown hand codes: dropped and the
    rest compacted in order) and short-material positions padded with piece-box
    entries."""
    rng = np.random.default_rng(61)
    rand = rng.integers(0, 256, (20000, 38), dtype=np.uint8)
    p = syn.psv_positions(syn.rng_for(62), 2000, hand_fraction=0.3)
    p["board"][syn.rng_for(63).random(p["board"].shape) < 0.3] = 0
    short = []
    for i in range(2000):
        try:
            short.append(syn.hcpe_encode(p["stm"][i], p["black_king"][i], p["white_king"][i], p["board"][i][None],
                                         p["hands"][i][None], 5, 2).view(np.uint8).reshape(-1, 38))
        except ValueError:
            continue
    recs = np.concatenate([rand, np.concatenate(short)])
    want, wvalid = ot.hcpe_to_psv(recs)
    got, valid, count = _hcpe_device(ctx, recs)
    assert count == wvalid.sum() and 0 < count < len(recs)
    np.testing.assert_array_equal(valid, wvalid)
    np.testing.assert_array_equal(got, want)


def test_hcpe_to_training_batch(ctx):
    """HCPE records -> device PackedSfenValue -> device HalfKA_hm2 batch equals
    the oracle's decode_hcpe_record -> prepare chain."""
    recs = syn.hcpe_records(70, 8192)
    cfg = _cfg("halfka_hm2", lam=1.0, wrm=True)
    conv = bt.HcpeConverter(ctx, 8192)
    count = conv.convert(ctx, recs)
    prod = bt.TeacherBatchProducer(ctx, cfg, count, pinned=False)
    out = prod.new_batch()
    bt.teacher_prepare_device(ctx, cfg, conv.psv, count, out.stm_indices, out.nstm_indices, out.buckets,
                              out.targets, out.entry_weights, prod.overflow, prod.wrm_table)
    want_psv, _ = ot.hcpe_to_psv(recs)
    got = out.download(ctx)
    got["overflow"] = int(prod.overflow.download(ctx)[0])
    _compare(got, _oracle(cfg, want_psv), cfg)
