"""CPU (gloo, world size 2): the data-parallel orchestration -- row sharding,
reduce-scatter / all-reduce / all-gather, sharded optimizer state -- with the
arithmetic supplied by the oracle.  Two ranks on half batches must reproduce a
single-process step on the whole batch."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from bulletou_b200.cuda_cpp import NnueForwardHostWeights, NnueForwardShape, RAdamUpdateParams, RangerUpdateParams, \
    ScalarLossKind
from bulletou_b200.data_parallel import NnueDataParallelTrainer, ShardLayout, dense_gradient_layout
from oracle import oracle

SHAPE = NnueForwardShape(51, 8, 4, 3)  # 51 rows: the last shard ends in padding
A = 5
BATCH = 6  # per rank


def test_shard_layout():
    lay = [ShardLayout(125388, 256, 8, r) for r in range(8)]
    assert lay[0].rows_padded == 125392 and lay[0].shard_rows == 15674
    assert sum(l.real_rows for l in lay) == 125388
    assert lay[7].real_rows == 125388 - 7 * 15674
    assert [x[0] for x in dense_gradient_layout(256, 32, 32)] == ["l0b", "l1w", "l1b", "l2w", "l2b", "outw", "outb"]
    assert dense_gradient_layout(256, 32, 32)[-1][1] + 1 == 256 + 512 * 32 + 32 + 1024 + 32 + 32 + 1


def test_sfnn_row_chunks_short_last_chunk():
    from bulletou_b200.data_parallel import sfnn_row_chunks

    ends = [10 * (j + 1) + j for j in range(15)]  # 15 launches of uneven row counts
    for lpc, last, sizes in ((3, None, [3, 3, 3, 3, 3]), (3, 1, [3, 3, 3, 3, 2, 1]), (3, 2, [3, 3, 3, 3, 1, 2]),
                             (1, 1, [1] * 15), (5, 15, [15])):
        chunks = sfnn_row_chunks(ends, 4, lpc, last)
        assert [c.last_launch - c.first_launch + 1 for c in chunks] == sizes
        assert chunks[0].first_launch == 0 and chunks[-1].last_launch == 14
        start = shard = 0
        for c, nxt in zip(chunks, chunks[1:] + [None]):
            assert c.start == start and c.start + c.length == ends[c.last_launch]
            assert c.padded % 4 == 0 and c.padded >= c.length and c.shard_rows == c.padded // 4
            assert c.shard_off == shard
            if nxt is not None:
                assert nxt.first_launch == c.last_launch + 1
                assert nxt.shift == c.shift + c.padded - c.length
            start, shard = c.start + c.length, shard + c.shard_rows


class CpuOracleBackend:
    """Trainer backend on CPU tensors; the math is the oracle's."""

    def zeros(self, n):
        return torch.zeros(n, dtype=torch.float32)

    def from_host(self, a):
        return torch.tensor(np.asarray(a, np.float32).copy())

    def tensor(self, buf):
        return buf

    def view(self, buf, offset, length):
        return buf[offset:offset + length]

    def download(self, buf):
        return buf.numpy().copy()

    def local_gradients(self, tr, spec):
        sh = tr.shape
        w = {n: t.numpy() for n, t in zip(oracle.NAMES, tr.weights)}
        w["l0w"] = w["l0w"][: sh.input_size * sh.l1]
        shape = (sh.input_size, sh.l1, sh.l2, sh.l3)
        fwd = oracle.nnue_forward(shape, tr.stm, tr.nstm, tr.batch_size, tr.max_active, w)
        loss = oracle.scalar_loss(spec.kind, spec.output_inv_scale, spec.loss_pow_exp, spec.loss_param,
                                  fwd["output"], tr.targets, tr.entry_weights, normalizer=spec.normalizer)
        g = oracle.nnue_backward(shape, tr.stm, tr.nstm, tr.batch_size, tr.max_active, fwd, w,
                                 loss["mean_output_gradients"])
        tr.ft_grad.zero_()
        tr.ft_grad[: sh.input_size * sh.l1] = torch.from_numpy(g["l0w_gradients"])
        for (name, off, n) in tr.dense_layout:
            tr.dense_grad[off:off + n] = torch.from_numpy(g[f"{name}_gradients"])

    def sfnn_local_gradients(self, tr, spec):
        sh = tr.shape
        w = {n: (None if b is None else b.numpy()) for n, b in tr.weights.items()}
        w["l0w"] = w["l0w"][: sh.input_size * sh.ft_size]
        args = (sh.as_tuple(), tr.stm, tr.nstm, tr.buckets, tr.batch_size, tr.max_active)
        lr = tr.lr_multipliers
        qat = oracle.qat_mask(lr.qat_l1, lr.qat_ft, lr.qat_l2, lr.qat_l3)
        fwd = oracle.sfnn_forward(*args, w, tr.alpha.ft, tr.alpha.shared, qat=qat)
        loss = oracle.scalar_loss(spec.kind, spec.output_inv_scale, spec.loss_pow_exp, spec.loss_param,
                                  fwd["output"], tr.targets, tr.entry_weights, normalizer=spec.normalizer)
        g = oracle.sfnn_backward(*args, fwd, w, loss["mean_output_gradients"], tr.alpha.ft, tr.alpha.shared,
                                 qat=qat)
        tr.ft_grad.zero_()
        W = sh.ft_size
        for c in tr.chunks:  # the padded chunk layout the row launches write (chunk-wise contiguous)
            tr.ft_grad[(c.start + c.shift) * W:(c.start + c.shift + c.length) * W] = \
                torch.from_numpy(g["l0w_gradients"][c.start * W:(c.start + c.length) * W])
        for (name, off, n) in tr.dense_layout:
            tr.dense_grad[off:off + n] = torch.from_numpy(g[f"{name}_gradients"])

    def sfnn_row_launches(self, sh, alpha):
        base = 73305 if sh.input_size == 73305 + 1629 else (131949 if sh.input_size == 131949 + 1629 else 0)
        kings = base // 1629 if base else 1
        n = -(-kings // 3)
        return [sh.input_size if j == n - 1 else 3 * (j + 1) * 1629 for j in range(n)]

    def ranger(self, params, grad, weights, m, v, slow, ctx=None):
        p = params.radam
        oracle.ranger_update(grad.numpy(), weights.numpy(), m.numpy(), v.numpy(), slow.numpy(), step=p.step,
                             learning_rate=p.learning_rate, beta1=p.beta1, beta2=p.beta2, epsilon=p.epsilon,
                             decay=p.decay, min_weight=p.min_weight, max_weight=p.max_weight,
                             lookahead_alpha=params.lookahead_alpha, lookahead_period=params.lookahead_period,
                             clip_after_lookahead=params.clip_after_lookahead)


def _weights():
    rng = np.random.default_rng(5)
    lens = SHAPE.weight_lengths()
    return {n: rng.normal(0, 0.3, k).astype(np.float32) for n, k in zip(oracle.NAMES, lens)}


def _batches(steps):
    rng = np.random.default_rng(9)
    out = []
    for _ in range(steps):
        n = 2 * BATCH * A
        out.append({"stm": rng.integers(-1, SHAPE.input_size, n).astype(np.int32),
                    "nstm": rng.integers(-1, SHAPE.input_size, n).astype(np.int32),
                    "targets": rng.random(2 * BATCH).astype(np.float32),
                    "entry_weights": np.ones(2 * BATCH, np.float32)})
    return out


def _params(step):
    return RangerUpdateParams(radam=RAdamUpdateParams(step=step, learning_rate=0.01, min_weight=-2.0, max_weight=2.0))


def _rank_main(rank, world, port, steps, out_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w = _weights()
        tr = NnueDataParallelTrainer(CpuOracleBackend(), dist, NnueForwardHostWeights(SHAPE, **w), BATCH, A)
        for step, b in enumerate(_batches(steps), start=1):
            sl = slice(rank * BATCH * A, (rank + 1) * BATCH * A)
            bs = slice(rank * BATCH, (rank + 1) * BATCH)
            tr.stm, tr.nstm = b["stm"][sl], b["nstm"][sl]
            tr.targets, tr.entry_weights = b["targets"][bs], b["entry_weights"][bs]
            tr.step_device(_params(step), ScalarLossKind.SigmoidPow(2.0), 1.0)
        got = tr.read_weights()
        if rank == 0:
            np.savez(out_path, **got)
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.timeout(300)
def test_two_rank_step_equals_single_process_global_batch(tmp_path):
    steps = 7  # crosses a lookahead step
    out = tmp_path / "rank0.npz"
    mp.start_processes(_rank_main, args=(2, _free_port(), steps, str(out)), nprocs=2, start_method="spawn")
    got = np.load(out)
    ref = oracle.NnueTrainer((SHAPE.input_size, SHAPE.l1, SHAPE.l2, SHAPE.l3), _weights())
    for step, b in enumerate(_batches(steps), start=1):
        ref.step(b["stm"], b["nstm"], 2 * BATCH, A, b["targets"], b["entry_weights"], step=step, learning_rate=0.01,
                 min_weight=-2.0, max_weight=2.0)
    for k in oracle.NAMES:
        np.testing.assert_allclose(got[k], ref.w[k], rtol=1e-5, atol=1e-6, err_msg=k)


# ---------------------------------------------------------------- SFNN
from bulletou_b200 import sfnn as bs  # noqa: E402
from bulletou_b200.data_parallel import SfnnDataParallelTrainer  # noqa: E402

SF_SHAPE = bs.SfnnForwardShape(73305 + 1629, 4, 2, True, 3, 3)  # factorized HalfKA_hm2, tiny widths
SF_ALPHA = bs.SfnnFactorizerAlpha(0.5, 2.0)
SF_A = 6


def _sf_weights():
    rng = np.random.default_rng(15)
    lens = SF_SHAPE.weight_lengths()
    return {n: rng.normal(0, 0.3, lens[n]).astype(np.float32) for n in bs.SFNN_WEIGHT_NAMES}


def _sf_batches(steps):
    rng = np.random.default_rng(19)
    out = []
    for _ in range(steps):
        n = 2 * BATCH * SF_A
        kings = rng.integers(0, 45, (2 * BATCH * 2, 1))
        feats = (kings * 1629 + rng.integers(0, 1629, (2 * BATCH * 2, SF_A))).reshape(2, -1).astype(np.int32)
        out.append({"stm": feats[0][:n], "nstm": feats[1][:n],
                    "buckets": rng.integers(0, SF_SHAPE.num_stacks, 2 * BATCH).astype(np.int32),
                    "targets": rng.random(2 * BATCH).astype(np.float32),
                    "entry_weights": np.ones(2 * BATCH, np.float32)})
    return out


def _sf_rank_main(rank, world, port, steps, out_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        tr = SfnnDataParallelTrainer(CpuOracleBackend(), dist, bs.SfnnForwardHostWeights(SF_SHAPE, **_sf_weights()),
                                     BATCH, SF_A, SF_ALPHA)
        for step, b in enumerate(_sf_batches(steps), start=1):
            sl = slice(rank * BATCH * SF_A, (rank + 1) * BATCH * SF_A)
            bsl = slice(rank * BATCH, (rank + 1) * BATCH)
            tr.stm, tr.nstm, tr.buckets = b["stm"][sl], b["nstm"][sl], b["buckets"][bsl]
            tr.targets, tr.entry_weights = b["targets"][bsl], b["entry_weights"][bsl]
            tr.step_device(_params(step), ScalarLossKind.SigmoidPow(2.0), 1.0)
        got = tr.read_weights()
        if rank == 0:
            np.savez(out_path, **got)
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_two_rank_sfnn_step_equals_single_process_global_batch(tmp_path):
    """Factorized FT (virtual rows sharded like any row), shared L1 factor with
    its scaled clip bounds, alpha != 1."""
    steps = 7
    out = tmp_path / "rank0.npz"
    mp.start_processes(_sf_rank_main, args=(2, _free_port(), steps, str(out)), nprocs=2, start_method="spawn")
    got = np.load(out)
    ref = oracle.SfnnTrainer(SF_SHAPE.as_tuple(), _sf_weights(), SF_ALPHA.ft, SF_ALPHA.shared)
    for step, b in enumerate(_sf_batches(steps), start=1):
        ref.step(b["stm"], b["nstm"], b["buckets"], 2 * BATCH, SF_A, b["targets"], b["entry_weights"], step=step,
                 learning_rate=0.01, min_weight=-2.0, max_weight=2.0)
    for k in ref.names:
        np.testing.assert_allclose(got[k], ref.w[k], rtol=1e-5, atol=1e-6, err_msg=k)
