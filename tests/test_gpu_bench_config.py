"""Parity at the configurations bench.py measures, against the reference
backend driven in its runner's call order (lib.rs:7448-7533):

* SFNN HalfKA_hm2 1536 k3k3, 65536 positions, batches decoded on
  the device from seeded PackedSfenValue records (kings near home: heavy FT
  rows and king blocks of many 4096-rank tiles), all-layer QAT -- the exact
  setup of `python bench.py` (its own helpers build runner, weights, batches);
* configs[4] per GPU: k9k9 (81 LayerStack buckets, Zipf(1.1) over a seeded
  permutation), 32768 positions (262144 / 8) of the same record-decoded rows.

Bars (north star): FT activations bit-exact; first-step outputs and
per-sample losses of the integer-lattice forward bit-exact; the mean loss
within 1e-5 relative at every step; FT weights within 1e-4 and the other
groups within 1e-3 after the steps.

The reference's mean loss is a one-thread serial f32 sum over the batch
(loss_finalize_from_per_sample_kernel, cu:2845-2860), whose own rounding at
65536 samples is of order 1e-5 relative, so every mean is compared with the
exact (f64) mean of the reference's per-sample losses.
"""
from types import SimpleNamespace

import numpy as np
import pytest

import bench
import bulletou_b200 as bo
from bulletou_b200 import sfnn as bs
from bulletou_b200 import synthetic

pytestmark = pytest.mark.gpu

STEPS = 5


def _psv_batches(ctx, batch, n):
    """(host, device) batches exactly as bench.py's SFNN workload makes them."""
    args = SimpleNamespace(data="psv", batch=batch)
    host, dev = bench.sfnn_batches(args, ctx)
    assert len(host) >= min(n, bench.SFNN_RECORD_BATCHES)
    return host, dev


def _concentration(b):
    """(largest king block in half-positions, largest FT row's entry count)."""
    f = np.concatenate([b["stm"], b["nstm"]])
    f = f[f >= 0]
    per_row = np.bincount(f)
    halves = np.concatenate([b["stm"].reshape(-1, 40)[:, 0], b["nstm"].reshape(-1, 40)[:, 0]]) // 1629
    return int(np.bincount(halves).max()), int(per_row.max())


def _train_both(ctx, ref_ctx, shape, host_weights, host, ours_dev, ref_dev, lr):
    ours = bs.SfnnTrainStepRunner(ctx, host_weights, host[0]["buckets"].size, 40, fused=True, lr_multipliers=lr)
    ref = bs.SfnnTrainStepRunner(ref_ctx, host_weights, host[0]["buckets"].size, 40, fused=False, lr_multipliers=lr)
    kind = bo.ScalarLossKind.SigmoidPow(2.0)
    first = None
    for step in range(1, STEPS + 1):
        i = (step - 1) % len(ours_dev)
        bench.bind_sfnn(ours, ours_dev[i])
        bench.bind_sfnn(ref, ref_dev[i])
        ours.step_device(ctx, bench.ranger(step), kind, 1 / 600, finalize_loss=True)
        ref.step_device(ref_ctx, bench.ranger(step), kind, 1 / 600, finalize_loss=True)
        got, want = ours.read_loss(ctx), ref.read_loss(ref_ctx)
        exact = float(np.asarray(want.per_sample, np.float64).sum() / want.per_sample.size)
        assert abs(got.mean - exact) <= 1e-5 * abs(exact), f"step {step}: loss {got.mean!r} vs reference {exact!r}"
        if step == 1:
            first = (ours.read_output(ctx), ref.read_output(ref_ctx))
            assert np.array_equal(got.per_sample, want.per_sample), "step 1 per-sample losses differ"
    a, c = ours.read_weights(ctx), ref.read_weights(ref_ctx)
    return first, a, c


def _check_weights(a, c):
    for nm in a:
        err = float(np.abs(a[nm].astype(np.float64) - c[nm]).max())
        bound = 1e-4 if nm == "l0w" else 1e-3
        assert err <= bound, f"{nm}: max |diff| {err:.3e} after {STEPS} steps (bound {bound})"


def test_configs2_bench_setup_matches_reference_backend(ctx, ref_ctx):
    B = bench.SFNN_BATCH
    host, dev = _psv_batches(ctx, B, STEPS)
    king_block, heaviest = _concentration(host[0])
    assert king_block > 3 * 4096, "the bench's record batches put several rank tiles in one king block"
    assert heaviest > 4096, "the bench's record batches have heavy FT rows"
    ref_dev = bench.sfnn_device_batches(ref_ctx, host)
    (out, ref_out), a, c = _train_both(ctx, ref_ctx, bench.sfnn_shape(), bench.sfnn_host_weights(), host, dev,
                                       ref_dev, bench.sfnn_lr_multipliers("all"))
    # all-layer QAT: the first step's forward is the engine's integer network on
    # identical weights -- the outputs agree bit for bit
    assert np.array_equal(out, ref_out), f"{int((out != ref_out).sum())} of {out.size} outputs differ"
    _check_weights(a, c)


def test_configs2_ft_activations_bit_exact_on_record_batches(ctx, ref_ctx):
    """The f32 FT forward (bias + rows in slot order, ClippedReLU, pairwise) of
    the bench's weights on its decoded-record batch equals the reference's."""
    shape = bench.sfnn_shape()
    B = bench.SFNN_BATCH
    host, _ = _psv_batches(ctx, B, 1)
    w = bench.sfnn_host_weights().arrays()
    outs = {}
    for c in (ctx, ref_ctx):
        dw = {n: (None if w.get(n) is None else bo.F32Buffer.from_host(c, w[n])) for n in bs.SFNN_WEIGHT_NAMES}
        s, n, k = (bo.I32Buffer.from_host(c, host[0][x]) for x in ("stm", "nstm", "buckets"))
        ws = bs.SfnnForwardWorkspace(c, shape, B)
        scratch = bo.F32Buffer(c, shape.input_size * shape.ft_size) if c is ref_ctx else None
        bs.sfnn_forward_device(c, shape, B, 40, s, n, k, dw, ws, bs.SfnnFactorizerAlpha(), scratch)
        outs[c] = {key: getattr(ws, key).download(c) for key in ("stm_l0", "nstm_l0", "combined")}
        del ws, scratch
    for key in ("stm_l0", "nstm_l0", "combined"):
        assert np.array_equal(outs[ctx][key], outs[ref_ctx][key]), key


def test_configs4_per_gpu_k9k9_zipf_matches_reference_backend(ctx, ref_ctx):
    """configs[4]'s per-GPU step: 32768 record-decoded positions, 81 buckets
    drawn Zipf(1.1) over a seeded permutation, all-layer QAT."""
    B = 262144 // 8
    shape = bs.SfnnForwardShape(bs.HALFKA_HM2_DIMENSIONS + bs.PIECE_INPUTS, 1536, 15, True, 32, 81)
    host, _ = _psv_batches(ctx, B, STEPS)
    for i, b in enumerate(host):
        b["buckets"] = synthetic.layerstack_buckets(synthetic.rng_for(4400 + i), B, 81, 1.1)
    counts = np.bincount(host[0]["buckets"], minlength=81)
    assert counts.max() > 20 * max(1, np.sort(counts)[40]), "Zipf-skewed buckets"
    ours_dev = bench.sfnn_device_batches(ctx, host)
    ref_dev = bench.sfnn_device_batches(ref_ctx, host)
    weights = bs.SfnnForwardHostWeights(shape, **synthetic.sfnn_weights(synthetic.rng_for(7), stacks=81))
    (out, ref_out), a, c = _train_both(ctx, ref_ctx, shape, weights, host, ours_dev, ref_dev,
                                       bench.sfnn_lr_multipliers("all"))
    assert np.array_equal(out, ref_out), f"{int((out != ref_out).sum())} of {out.size} outputs differ"
    _check_weights(a, c)
