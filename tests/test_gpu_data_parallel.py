"""GPU (>= 2 devices, NCCL): two ranks of data-parallel HalfKP training on half
batches reproduce one single-GPU fused step on the whole batch.  Skipped on a
single GPU."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

BATCH = 2048  # per rank
STEPS = 7


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _batches():
    from bulletou_b200 import synthetic

    return [synthetic.halfkp_batch(700 + i, 2 * BATCH) for i in range(STEPS)]


def _params(step):
    import bulletou_b200 as bo

    return bo.RangerUpdateParams(radam=bo.RAdamUpdateParams(step=step, learning_rate=1e-3))


def _rank_main(rank, world, port, out_path):
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    import bulletou_b200 as bo
    from bulletou_b200 import synthetic
    from bulletou_b200.data_parallel import B200Backend, NnueDataParallelTrainer

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        w = synthetic.halfkp_weights(synthetic.rng_for(17))
        tr = NnueDataParallelTrainer(B200Backend(rank), dist,
                                     bo.NnueForwardHostWeights(bo.NNUE_HALFKP_256X2_32_32, **w), BATCH, 38)
        for step, b in enumerate(_batches(), start=1):
            sl = slice(rank * BATCH * 38, (rank + 1) * BATCH * 38)
            bs = slice(rank * BATCH, (rank + 1) * BATCH)
            tr.upload_batch(b["stm"][sl], b["nstm"][sl], b["targets"][bs], b["entry_weights"][bs])
            tr.step_device(_params(step), bo.ScalarLossKind.SigmoidPow(2.0), 1 / 600)
        torch.cuda.synchronize()
        got = tr.read_weights()
        if rank == 0:
            np.savez(out_path, **got)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(600)
def test_two_gpu_data_parallel_matches_single_gpu_global_batch(tmp_path):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    out = tmp_path / "rank0.npz"
    mp.start_processes(_rank_main, args=(2, _free_port(), str(out)), nprocs=2, start_method="spawn")
    got = np.load(out)

    import bulletou_b200 as bo
    from bulletou_b200 import synthetic

    w = synthetic.halfkp_weights(synthetic.rng_for(17))
    ctx = bo.Context(0)
    runner = bo.NnueTrainStepRunner(ctx, bo.NnueForwardHostWeights(bo.NNUE_HALFKP_256X2_32_32, **w), 2 * BATCH, 38)
    for step, b in enumerate(_batches(), start=1):
        hb = bo.NnueTrainStepHostBatch(b["stm"], b["nstm"], b["targets"], b["entry_weights"], 2 * BATCH, 38)
        runner.step_no_readback(ctx, _params(step), bo.ScalarLossKind.SigmoidPow(2.0), 1 / 600, hb)
    ref = runner.read_weights(ctx)
    for k, v in ref.items():
        scale = max(float(np.abs(v).max()), 1e-30)
        err = float(np.abs(got[k].astype(np.float64) - v).max())
        assert err <= 1e-4 * scale, f"{k}: max |diff| {err:.3e} (scale {scale:.3e})"


# ---------------------------------------------------------------- SFNN
SF_BATCH = 1024  # per rank


def _sf_batches():
    from bulletou_b200 import synthetic

    return [synthetic.sfnn_batch(800 + i, 2 * SF_BATCH) for i in range(STEPS)]


def _sf_qat(mode):
    from bulletou_b200 import sfnn as bs

    return bs.SfnnLayerLrMultipliers() if mode == "none" else bs.SfnnLayerLrMultipliers(
        qat_l1=True, qat_ft=True, qat_l2=True, qat_l3=True)


def _sf_rank_main(rank, world, port, out_path, qat="none", exchange="p2p"):
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    import bulletou_b200 as bo
    from bulletou_b200 import sfnn as bs
    from bulletou_b200 import synthetic
    from bulletou_b200.data_parallel import B200Backend, SfnnDataParallelTrainer

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        w = synthetic.sfnn_weights(synthetic.rng_for(23), ft=256)
        shape = bs.SfnnForwardShape(73305 + 1629, 256, 15, True, 32, 9)
        tr = SfnnDataParallelTrainer(B200Backend(rank), dist, bs.SfnnForwardHostWeights(shape, **w), SF_BATCH, 40,
                                     lr_multipliers=_sf_qat(qat), exchange=exchange)
        assert tr.exchange == exchange
        for step, b in enumerate(_sf_batches(), start=1):
            sl = slice(rank * SF_BATCH * 40, (rank + 1) * SF_BATCH * 40)
            bsl = slice(rank * SF_BATCH, (rank + 1) * SF_BATCH)
            tr.upload_batch(b["stm"][sl], b["nstm"][sl], b["buckets"][bsl], b["targets"][bsl],
                            b["entry_weights"][bsl])
            tr.step_device(_params(step), bo.ScalarLossKind.SigmoidPow(2.0), 1 / 600)
        torch.cuda.synchronize()
        got = tr.read_weights()
        if rank == 0:
            np.savez(out_path, **got)
        tr.close()
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(600)
@pytest.mark.parametrize("qat,exchange", [("none", "collectives"), ("none", "p2p"), ("all", "p2p")])
def test_two_gpu_sfnn_data_parallel_matches_single_gpu_global_batch(tmp_path, qat, exchange):
    """Two ranks on half batches equal one GPU on the whole batch, with the
    exchange through the process group's collectives or over peer memory
    (gradient rows stored into their owners' slots by the row kernels)."""
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    out = tmp_path / "rank0.npz"
    mp.start_processes(_sf_rank_main, args=(2, _free_port(), str(out), qat, exchange), nprocs=2,
                       start_method="spawn")
    got = np.load(out)

    import bulletou_b200 as bo
    from bulletou_b200 import sfnn as bs
    from bulletou_b200 import synthetic

    w = synthetic.sfnn_weights(synthetic.rng_for(23), ft=256)
    shape = bs.SfnnForwardShape(73305 + 1629, 256, 15, True, 32, 9)
    ctx = bo.Context(0)
    runner = bs.SfnnTrainStepRunner(ctx, bs.SfnnForwardHostWeights(shape, **w), 2 * SF_BATCH, 40,
                                    lr_multipliers=_sf_qat(qat))
    for step, b in enumerate(_sf_batches(), start=1):
        hb = bs.SfnnTrainStepHostBatch(b["stm"], b["nstm"], b["buckets"], b["targets"], b["entry_weights"],
                                       2 * SF_BATCH, 40)
        runner.step_no_readback(ctx, _params(step), bo.ScalarLossKind.SigmoidPow(2.0), 1 / 600, hb)
    ref = runner.read_weights(ctx)
    for k, v in ref.items():
        scale = max(float(np.abs(v).max()), 1e-30)
        err = float(np.abs(got[k].astype(np.float64) - v).max())
        assert err <= 1e-4 * scale, f"{k}: max |diff| {err:.3e} (scale {scale:.3e})"


def test_exchange_wait_times_out_with_an_error_code():
    """A bounded exchange wait on a flag nothing sets returns after about 2 s
    with 1 + the flag's index in the error word; the context stays usable."""
    import time

    import bulletou_b200 as bo

    ctx = bo.Context(0)
    flags = bo.I32Buffer.from_host(ctx, np.array([3, 3, 2, 3], np.int32))
    err = bo.I32Buffer.from_host(ctx, np.zeros(1, np.int32))
    lib = ctx.lib
    lib.call("bulletou_b200_exchange_wait_device", ctx.as_ptr(), flags.as_ptr(), 0, 2, 3, err.as_ptr())
    ctx.synchronize()
    assert int(err.download(ctx)[0]) == 0  # both flags already at the epoch
    t0 = time.time()
    lib.call("bulletou_b200_exchange_wait_device", ctx.as_ptr(), flags.as_ptr(), 1, 3, 3, err.as_ptr())
    ctx.synchronize()
    assert 1.0 < time.time() - t0 < 30.0
    assert int(err.download(ctx)[0]) == 1 + 1  # the second flag of the range (value 2) never reaches 3
    x = bo.F32Buffer.from_host(ctx, np.arange(8, dtype=np.float32))
    assert np.array_equal(x.download(ctx), np.arange(8, dtype=np.float32))
    ctx.close()
