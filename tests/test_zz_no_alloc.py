"""GPU: the allocation-free HalfKP forward (bulletou_b200_nnue_forward_device_noalloc).

Callers that cannot allocate device memory while they run get the same
production-shape forward as bulletou_cuda_cpp_nnue_forward_device, with its
scratch in a static device array.  This file is collected last so that a run
stopping at the first failure has already run every other test; it also
passes on its own in a fresh process.
"""
import numpy as np
import pytest

import bulletou_b200 as bo
from bulletou_b200 import synthetic
from bulletou_b200.cuda_cpp import NnueForwardWorkspace

pytestmark = pytest.mark.gpu

SHAPE = bo.NnueForwardShape(125388, 256, 32, 32)


def _outputs(ws):
    return {k: getattr(ws, k).download() for k in ("stm_l0", "nstm_l0", "combined", "hidden1", "hidden2", "output")}


def _call(lib, name, ctx, batch, A, s, n, wb, ws):
    lib.call(name, ctx.as_ptr(), SHAPE.input_size, SHAPE.l1, SHAPE.l2, SHAPE.l3, batch, A, s.as_ptr(), n.as_ptr(),
             *[w.as_ptr() for w in wb], ws.stm_l0.as_ptr(), ws.nstm_l0.as_ptr(), ws.combined.as_ptr(),
             ws.hidden1.as_ptr(), ws.hidden2.as_ptr(), ws.output.as_ptr())


def test_no_alloc_forward_matches_regular_forward_twice():
    lib = bo.library()
    ctx = bo.Context(0, lib)
    w = synthetic.halfkp_weights(synthetic.rng_for(31))
    wb = [bo.F32Buffer.from_host(ctx, a) for a in bo.NnueForwardHostWeights(SHAPE, **w).arrays()]
    # two calls in a row with different batches (and sizes): the shared static
    # scratch keeps the first call's contents, which must not leak into the second
    for call, batch in enumerate((4096, 1500)):
        b = synthetic.halfkp_batch(40 + call, batch)
        s, n = bo.I32Buffer.from_host(ctx, b["stm"]), bo.I32Buffer.from_host(ctx, b["nstm"])
        ws_ref = NnueForwardWorkspace(ctx, SHAPE, batch)
        ws_na = NnueForwardWorkspace(ctx, SHAPE, batch)
        _call(lib, "bulletou_cuda_cpp_nnue_forward_device", ctx, batch, 38, s, n, wb, ws_ref)
        _call(lib, "bulletou_b200_nnue_forward_device_noalloc", ctx, batch, 38, s, n, wb, ws_na)
        ref, got = _outputs(ws_ref), _outputs(ws_na)
        for k in ref:
            # same kernels and summation order: the tolerance is exact equality
            assert np.array_equal(got[k], ref[k]), f"call {call} {k}: max |diff| {np.abs(got[k] - ref[k]).max():.3e}"
    ctx.close()


def _scratch_bytes(lib, ctx):
    import ctypes

    n = ctypes.c_size_t(0)
    lib.call("bulletou_b200_context_scratch_bytes", ctx.as_ptr(), ctypes.byref(n))
    return n.value


def test_no_alloc_forward_allocates_nothing_on_a_fresh_context():
    """On a context no other entry point has used, the allocation-free forward
    leaves the context's scratch empty, while the regular forward then has to
    allocate its king-sort scratch."""
    lib = bo.library()
    ctx = bo.Context(0, lib)
    w = synthetic.halfkp_weights(synthetic.rng_for(33))
    wb = [bo.F32Buffer.from_host(ctx, a) for a in bo.NnueForwardHostWeights(SHAPE, **w).arrays()]
    b = synthetic.halfkp_batch(43, 2048)
    s, n = bo.I32Buffer.from_host(ctx, b["stm"]), bo.I32Buffer.from_host(ctx, b["nstm"])
    ws = NnueForwardWorkspace(ctx, SHAPE, 2048)
    assert _scratch_bytes(lib, ctx) == 0
    for _ in range(2):
        _call(lib, "bulletou_b200_nnue_forward_device_noalloc", ctx, 2048, 38, s, n, wb, ws)
        ctx.synchronize()
        assert _scratch_bytes(lib, ctx) == 0
    first = _outputs(ws)
    _call(lib, "bulletou_cuda_cpp_nnue_forward_device", ctx, 2048, 38, s, n, wb, ws)
    assert _scratch_bytes(lib, ctx) > 0
    again = _outputs(ws)
    for k in first:
        assert np.array_equal(first[k], again[k]), k
    ctx.close()


def test_no_alloc_forward_rejects_oversized_batch():
    lib = bo.library()
    ctx = bo.Context(0, lib)
    batch = 65537
    dummy_i = bo.I32Buffer(ctx, 1)
    dummy_f = bo.F32Buffer(ctx, 1)
    with pytest.raises(bo.CudaCppError, match="static scratch limit"):
        lib.call("bulletou_b200_nnue_forward_device_noalloc", ctx.as_ptr(), SHAPE.input_size, SHAPE.l1, SHAPE.l2,
                 SHAPE.l3, batch, 38, dummy_i.as_ptr(), dummy_i.as_ptr(), *([dummy_f.as_ptr()] * 14))
    ctx.close()
