"""Data-parallel HalfKP and SFNN training over torch.distributed (NCCL on GPUs, gloo on CPU).

The reference trains on one GPU (no collectives, cu:9503-9545); this module is
the additive multi-GPU layer.  Positions are independent, so the only
exchange is the gradient sum:

    local step      forward + loss + backward of the rank's batch, the loss
                    gradient normalised by the *global* batch
                    (bulletou_b200_nnue_local_gradients_device): FT gradient
                    rows [R][L1] and the packed small-parameter gradient
    reduce-scatter  FT gradient by contiguous row shard (in place)
    all-reduce      packed small-parameter gradient
    Ranger          owned FT rows only (optimizer state is sharded: m, v and
                    slow hold just the rank's rows) + all small groups
                    (replicated, identical on every rank)
    all-gather      updated FT rows (in place), so every rank holds the full
                    table for the next forward

The FT table and its gradient are padded to a multiple of the world size in
rows (padding rows are never referenced by a feature).  A step on N ranks of
batch B equals one single-GPU step on the concatenated batch of N*B up to
summation order.

`NnueDataParallelTrainer` / `SfnnDataParallelTrainer` hold the orchestration
(the SFNN one shards the FT table including its virtual factor rows, whose
local gradients are already alpha * the king-row sums, so the reduce-scatter
sums them like any other row); the arithmetic comes from a
backend: `B200Backend` (the CUDA library, zero-copy torch views of its
buffers, collectives ordered on the library's stream) for training, and, in
tests, a CPU backend built on the oracle so the sharding and collective logic
runs on gloo without a GPU.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Optional

import numpy as np

from .cuda_cpp import (NNUE_WEIGHT_NAMES, CudaCppError, F32Buffer, I32Buffer, NnueForwardHostWeights,
                       RangerDeviceState, RangerUpdateParams, ScalarLossKind, ScalarLossWorkspace, ranger_update_device)


@dataclass(frozen=True)
class ShardLayout:
    """Row sharding of the FT table over `world` ranks."""

    rows: int
    width: int
    world: int
    rank: int

    @property
    def rows_padded(self) -> int:
        return -(-self.rows // self.world) * self.world

    @property
    def shard_rows(self) -> int:
        return self.rows_padded // self.world

    @property
    def row_begin(self) -> int:
        return self.rank * self.shard_rows

    @property
    def real_rows(self) -> int:
        """Owned rows that exist (the last shard may end in padding)."""
        return max(0, min(self.rows, self.row_begin + self.shard_rows) - self.row_begin)


def dense_gradient_layout(l1: int, l2: int, l3: int) -> list[tuple[str, int, int]]:
    """(group, offset, length) of the packed small-parameter gradient:
    l0b | l1w | l1b | l2w | l2b | outw | outb."""
    sizes = [("l0b", l1), ("l1w", 2 * l1 * l2), ("l1b", l2), ("l2w", l2 * l3), ("l2b", l3), ("outw", l3), ("outb", 1)]
    out, off = [], 0
    for name, n in sizes:
        out.append((name, off, n))
        off += n
    return out


class B200Backend:
    """libbulletou_b200 on one GPU; the context runs on torch's current stream
    so NCCL collectives issued through torch order with the library's work."""

    def __init__(self, device: int, lib=None):
        import torch

        from . import cuda_cpp as cc

        self.torch = torch
        self.device = device
        stream = torch.cuda.current_stream(device).cuda_stream
        self.ctx = cc.Context(device, lib, stream=stream)
        self.lib = self.ctx.lib

    def zeros(self, n: int) -> F32Buffer:
        b = F32Buffer(self.ctx, n)
        b.fill(0.0)
        return b

    def from_host(self, a) -> F32Buffer:
        return F32Buffer.from_host(self.ctx, a)

    def tensor(self, buf) -> "object":
        return self.torch.as_tensor(buf, device=f"cuda:{self.device}")

    def local_gradients(self, tr: "NnueDataParallelTrainer", loss_spec) -> None:
        sh = tr.shape
        arr = ctypes.c_void_p * 8
        params = arr(*[w.as_ptr().value for w in tr.weights])
        lw = tr.loss_workspace
        self.lib.call("bulletou_b200_nnue_local_gradients_device", self.ctx.as_ptr(), sh.input_size, sh.l1, sh.l2,
                      sh.l3, tr.batch_size, tr.max_active, tr.stm_indices.as_ptr(), tr.nstm_indices.as_ptr(),
                      tr.targets.as_ptr(), tr.entry_weights.as_ptr(), ctypes.byref(loss_spec), params,
                      tr.ft_grad.as_ptr(), tr.dense_grad.as_ptr(), tr.output.as_ptr(), lw.per_sample.as_ptr(),
                      lw.mean_output_gradients.as_ptr(), lw.weighted_sum.as_ptr(), lw.mean.as_ptr())

    @staticmethod
    def _sfnn_shape(sh, alpha):
        from ._lib import SfnnShape

        return SfnnShape(sh.input_size, sh.ft_size, sh.l1_hidden, int(sh.l1_skip), sh.l2_size, sh.num_stacks,
                         alpha.ft, alpha.shared)

    def sfnn_row_launches(self, sh, alpha) -> list:
        shape = self._sfnn_shape(sh, alpha)
        n = ctypes.c_size_t()
        ends = (ctypes.c_size_t * 256)()
        self.lib.call("bulletou_b200_sfnn_row_launches", ctypes.byref(shape), ctypes.byref(n), ends, 256)
        return [int(ends[j]) for j in range(n.value)]

    def sfnn_local_gradients(self, tr: "SfnnDataParallelTrainer", loss_spec, events=None) -> None:
        shape = self._sfnn_shape(tr.shape, tr.alpha)
        arr = ctypes.c_void_p * 14
        params = arr(*[(None if w is None else w.as_ptr().value) for w in tr.weight_list()])
        lw = tr.loss_workspace
        qat = tr.lr_multipliers.as_struct()
        n = len(tr.row_ends)
        shifts = (ctypes.c_size_t * n)(*[tr.chunks[tr.launch_chunk[j]].shift for j in range(n)])
        self.lib.call("bulletou_b200_sfnn_local_gradients_device", self.ctx.as_ptr(), ctypes.byref(shape),
                      tr.batch_size, tr.max_active, tr.stm_indices.as_ptr(), tr.nstm_indices.as_ptr(),
                      tr.buckets.as_ptr(), tr.targets.as_ptr(), tr.entry_weights.as_ptr(), ctypes.byref(loss_spec),
                      params, tr.ft_grad.as_ptr(), tr.dense_grad.as_ptr(), tr.output.as_ptr(),
                      lw.per_sample.as_ptr(), lw.mean_output_gradients.as_ptr(), lw.weighted_sum.as_ptr(),
                      lw.mean.as_ptr(), ctypes.byref(qat), shifts, events, n)

    # -- overlapped exchange (SfnnDataParallelTrainer) --------------------------
    supports_overlap = True

    def prepare_overlap(self, tr: "SfnnDataParallelTrainer") -> None:
        from . import cuda_cpp as cc

        tr._comm = self.torch.cuda.Stream(device=self.device)
        tr._comm_ctx = cc.Context(self.device, self.lib, stream=tr._comm.cuda_stream)
        tr._events = [cc.Event(self.ctx) for _ in tr.row_ends]
        tr._event_handles = (ctypes.c_void_p * len(tr.row_ends))(*[e._h.value for e in tr._events])
        tr._ready = cc.Event(self.ctx)  # recorded on the comm stream after each step's exchange
        tr._ready_pending = False
        tr._timing_steps = []

    def sfnn_step_overlapped(self, tr: "SfnnDataParallelTrainer", loss_spec, params) -> None:
        """Local step on the library's stream; per chunk, on the comm stream:
        wait for the launch that completes it, reduce-scatter, Ranger on the
        owned rows, all-gather.  The small groups' all-reduce and Ranger go
        first (their gradients precede the row launches).  The next step runs
        its batch-only work (sorts, inverse index) at once and waits for this
        exchange only before it reads a weight
        (bulletou_b200_context_wait_before_weights)."""
        torch = self.torch
        compute = torch.cuda.current_stream(self.device)
        if tr._ready_pending:
            # the previous exchange wrote the weights this step reads and read
            # the gradient rows this step writes, both after the batch work
            self.lib.call("bulletou_b200_context_wait_before_weights", self.ctx.as_ptr(), tr._ready._h)
        ev = self._timing_events(tr) if tr.timing else None
        if ev is not None:
            ev["step_start"].record(compute)
        self.sfnn_local_gradients(tr, loss_spec, tr._event_handles)
        if ev is not None:
            ev["rows_end"].record(compute)
        with torch.cuda.stream(tr._comm):
            tr._events[0].wait(tr._comm_ctx)
            if ev is not None:
                ev["small_start"].record(tr._comm)
            tr._small_exchange(params, tr._comm_ctx)
            for j, c in enumerate(tr.chunks):
                tr._events[c.last_launch].wait(tr._comm_ctx)
                tr._chunk_exchange(j, params, tr._comm_ctx, None if ev is None else ev["chunks"][j])
            if ev is not None:
                ev["exchange_end"].record(tr._comm)
        tr._ready.record(tr._comm_ctx)
        tr._ready_pending = True

    def _timing_events(self, tr) -> dict:
        E = lambda: self.torch.cuda.Event(enable_timing=True)  # noqa: E731
        ev = {"step_start": E(), "rows_end": E(), "small_start": E(), "exchange_end": E(),
              "chunks": [{"start": E(), "reduce_scatter": E(), "ranger": E(), "all_gather": E()} for _ in tr.chunks]}
        tr._timing_steps.append(ev)
        return ev

    def exchange_timing(self, tr) -> dict:
        """Mean per step over the steps run with tr.timing on (ms, device
        events): the local step (start to its last row launch's end), the comm
        stream's small-group exchange, reduce-scatters, shard Ranger,
        all-gathers, the exchange's end after the last row launch (the tail
        the next step's weight reads wait for) and per chunk."""
        self.torch.cuda.synchronize(self.device)
        steps = tr._timing_steps
        tr._timing_steps = []
        if not steps:
            return {}
        acc = {"local_step_ms": 0.0, "small_exchange_ms": 0.0, "reduce_scatter_ms": 0.0, "shard_ranger_ms": 0.0,
               "all_gather_ms": 0.0, "exchange_tail_after_rows_ms": 0.0}
        per_chunk = [{"wait_ms": 0.0, "reduce_scatter_ms": 0.0, "shard_ranger_ms": 0.0, "all_gather_ms": 0.0}
                     for _ in tr.chunks]
        for ev in steps:
            acc["local_step_ms"] += ev["step_start"].elapsed_time(ev["rows_end"])
            prev = ev["small_start"]
            for j, c in enumerate(ev["chunks"]):
                if j == 0:
                    acc["small_exchange_ms"] += ev["small_start"].elapsed_time(c["start"])
                else:
                    per_chunk[j]["wait_ms"] += prev.elapsed_time(c["start"])
                rs = c["start"].elapsed_time(c["reduce_scatter"])
                rg = c["reduce_scatter"].elapsed_time(c["ranger"])
                ag = c["ranger"].elapsed_time(c["all_gather"])
                per_chunk[j]["reduce_scatter_ms"] += rs
                per_chunk[j]["shard_ranger_ms"] += rg
                per_chunk[j]["all_gather_ms"] += ag
                acc["reduce_scatter_ms"] += rs
                acc["shard_ranger_ms"] += rg
                acc["all_gather_ms"] += ag
                prev = c["all_gather"]
            acc["exchange_tail_after_rows_ms"] += ev["rows_end"].elapsed_time(ev["exchange_end"])
        n = len(steps)
        out = {k: round(v / n, 4) for k, v in acc.items()}
        out["steps"] = n
        out["chunks"] = [{"launches": [c.first_launch, c.last_launch], "rows": c.length,
                          **{k: round(v / n, 4) for k, v in pc.items()}} for c, pc in zip(tr.chunks, per_chunk)]
        return out

    # -- peer-memory exchange (SfnnDataParallelTrainer, exchange="p2p") ---------
    supports_peer_exchange = True

    def prepare_peer_exchange(self, tr: "SfnnDataParallelTrainer") -> None:
        """Receive slots and flags on this rank, CUDA IPC handles of them and
        of the FT table exchanged over the process group, peers' buffers
        opened: the descriptor of bulletou_b200_sfnn_local_gradients_exchange_
        device and bulletou_b200_sfnn_shard_ranger_exchange_device."""
        from ._lib import RowExchange

        world, rank, W = tr.world, tr.rank, tr.shape.ft_size
        if world > 8:
            raise CudaCppError("the peer exchange supports up to 8 ranks")
        last = tr.chunks[-1]
        slot_rows = last.shard_off + last.shard_rows
        n_chunks = len(tr.chunks)
        small_len = tr.dense_layout[-1][1] + tr.dense_layout[-1][2]
        tr._recv = F32Buffer(self.ctx, world * slot_rows * W)
        tr._small_recv = F32Buffer(self.ctx, world * small_len)
        # flags: scatter [chunk][source], ready [chunk][owner], small [source]
        tr._flags = I32Buffer.from_host(self.ctx, np.zeros(2 * n_chunks * world + world, np.int32))
        tr._xerr = I32Buffer.from_host(self.ctx, np.zeros(1, np.int32))
        own = (tr._recv, tr.weights["l0w"], tr._flags, tr._small_recv)
        mine = []
        for b in own:
            h = (ctypes.c_ubyte * 64)()
            kind = "f32" if isinstance(b, F32Buffer) else "i32"
            self.lib.call(f"bulletou_b200_{kind}_buffer_ipc_handle", b.as_ptr(), h)
            mine.append(bytes(h))
        gathered = [None] * world
        tr.dist.all_gather_object(gathered, mine)
        x = RowExchange()
        x.world, x.rank, x.slot_rows, x.epoch = world, rank, slot_rows, 0
        x.small_len, x.small_flag_base = small_len, 2 * n_chunks * world
        tr._opened = []
        for r in range(world):
            for k, field in enumerate((x.recv, x.table, x.flags, x.small_recv)):
                if r == rank:
                    field[r] = own[k].device_ptr()
                else:
                    addr = ctypes.c_uint64()
                    h = (ctypes.c_ubyte * 64).from_buffer_copy(gathered[r][k])
                    self.lib.call("bulletou_b200_ipc_open", self.ctx.as_ptr(), h, ctypes.byref(addr))
                    field[r] = addr.value
                    tr._opened.append(addr.value)
        tr._x = x
        n = len(tr.row_ends)
        chunk_of = [tr.chunks[tr.launch_chunk[j]] for j in range(n)]
        tr._launch_start = (ctypes.c_size_t * n)(*[c.start for c in chunk_of])
        tr._launch_shard_rows = (ctypes.c_size_t * n)(*[c.shard_rows for c in chunk_of])
        tr._launch_shard_off = (ctypes.c_size_t * n)(*[c.shard_off for c in chunk_of])
        tr._launch_signal = (ctypes.c_longlong * n)(*[tr.launch_chunk[j] if j == chunk_of[j].last_launch else -1
                                                      for j in range(n)])
        tr._epoch = 0

    def sfnn_step_peer_exchange(self, tr: "SfnnDataParallelTrainer", loss_spec, params) -> None:
        """The local step stores its FT gradient rows into their owners'
        receive slots (signalling each chunk) and its small-group gradient into
        every rank's small slots; on the comm stream the small groups' sum +
        Ranger, then per chunk this rank's shard: wait for
        every rank's rows, sum, Ranger, store into every rank's table, signal.
        The next step runs its batch-only work first and waits for every
        owner's signals (and this rank's comm stream) before its first weight
        read."""
        torch, lib, ctx = self.torch, self.lib, self.ctx
        world, rank, W = tr.world, tr.rank, tr.shape.ft_size
        nc = len(tr.chunks)
        if tr._ready_pending:
            lib.call("bulletou_b200_context_wait_before_weights", ctx.as_ptr(), tr._ready._h)
            lib.call("bulletou_b200_context_wait_flags_before_weights", ctx.as_ptr(), tr._flags.as_ptr(), nc * world,
                     nc * world, tr._epoch, tr._xerr.as_ptr())
        tr._epoch += 1
        x = tr._x
        x.epoch = tr._epoch
        compute = torch.cuda.current_stream(self.device)
        ev = self._timing_events(tr) if tr.timing else None
        if ev is not None:
            ev["step_start"].record(compute)
        sh = self._sfnn_shape(tr.shape, tr.alpha)
        arr = ctypes.c_void_p * 14
        prm = arr(*[(None if w is None else w.as_ptr().value) for w in tr.weight_list()])
        lw = tr.loss_workspace
        qat = tr.lr_multipliers.as_struct()
        lib.call("bulletou_b200_sfnn_local_gradients_exchange_device", ctx.as_ptr(), ctypes.byref(sh), tr.batch_size,
                 tr.max_active, tr.stm_indices.as_ptr(), tr.nstm_indices.as_ptr(), tr.buckets.as_ptr(),
                 tr.targets.as_ptr(), tr.entry_weights.as_ptr(), ctypes.byref(loss_spec), prm,
                 tr.dense_grad.as_ptr(), tr.output.as_ptr(), lw.per_sample.as_ptr(),
                 lw.mean_output_gradients.as_ptr(), lw.weighted_sum.as_ptr(), lw.mean.as_ptr(), ctypes.byref(qat),
                 ctypes.byref(x), tr._launch_start, tr._launch_shard_rows, tr._launch_shard_off, tr._launch_signal,
                 tr._event_handles, len(tr.row_ends))
        if ev is not None:
            ev["rows_end"].record(compute)
        step = params.ffi_step()
        m, v, slow = tr.ft_state
        with torch.cuda.stream(tr._comm):
            tr._events[0].wait(tr._comm_ctx)
            if ev is not None:
                ev["small_start"].record(tr._comm)
            tr._small_exchange(params, tr._comm_ctx)
            for j, c in enumerate(tr.chunks):
                tr._events[c.last_launch].wait(tr._comm_ctx)
                ce = None if ev is None else ev["chunks"][j]
                if ce is not None:
                    ce["start"].record()
                    ce["reduce_scatter"].record()
                lib.call("bulletou_b200_sfnn_shard_ranger_exchange_device", tr._comm_ctx.as_ptr(), ctypes.byref(x), W,
                         c.start, c.length, c.shard_rows, c.shard_off, ctypes.byref(step), tr.l0w_compact.as_ptr(),
                         m.as_ptr(), v.as_ptr(), slow.as_ptr(), tr._flags.as_ptr(), j * world,
                         nc * world + j * world + rank, tr._xerr.as_ptr())
                if ce is not None:
                    ce["ranger"].record()
                    ce["all_gather"].record()
            if ev is not None:
                ev["exchange_end"].record(tr._comm)
        tr._ready.record(tr._comm_ctx)
        tr._ready_pending = True

    def check_peer_exchange(self, tr: "SfnnDataParallelTrainer") -> None:
        self.torch.cuda.synchronize(self.device)
        err = int(tr._xerr.download(self.ctx)[0])
        if err:
            raise CudaCppError(f"peer exchange: a wait for flag {err - 1} timed out (a rank stopped or fell behind)")

    def close_peer_exchange(self, tr: "SfnnDataParallelTrainer") -> None:
        for addr in getattr(tr, "_opened", []):
            self.lib.call("bulletou_b200_ipc_close", self.ctx.as_ptr(), addr)
        tr._opened = []

    def join_overlap(self, tr: "SfnnDataParallelTrainer") -> None:
        self.torch.cuda.current_stream(self.device).wait_stream(tr._comm)

    def ranger(self, params: RangerUpdateParams, grad, weights, m, v, slow, ctx=None) -> None:
        ranger_update_device(ctx or self.ctx, params, RangerDeviceState(grad, weights, m, v, slow))

    def view(self, buf: F32Buffer, offset: int, length: int) -> F32Buffer:
        return buf.view(offset, length)

    def download(self, buf: F32Buffer) -> np.ndarray:
        return buf.download()


class NnueDataParallelTrainer:
    """One rank of data-parallel HalfKP training (any backend, any collective group)."""

    def __init__(self, backend, dist, initial_weights: NnueForwardHostWeights, batch_size: int, max_active: int):
        initial_weights.validate()
        self.backend = backend
        self.dist = dist
        self.world = dist.get_world_size()
        self.rank = dist.get_rank()
        self.shape = initial_weights.shape
        self.batch_size = batch_size
        self.max_active = max_active
        sh = self.shape
        self.layout = ShardLayout(sh.input_size, sh.l1, self.world, self.rank)
        lay = self.layout
        arrays = initial_weights.arrays()
        l0w = np.zeros(lay.rows_padded * sh.l1, np.float32)
        l0w[: arrays[0].size] = arrays[0]
        self.weights = [backend.from_host(l0w)] + [backend.from_host(a) for a in arrays[1:]]
        # optimizer state: owned FT rows only; small groups replicated
        own = slice(lay.row_begin * sh.l1, (lay.row_begin + lay.real_rows) * sh.l1)
        n_own = lay.real_rows * sh.l1
        self.ft_state = (backend.zeros(n_own), backend.zeros(n_own), backend.from_host(l0w[own]))
        self.small_state = [(backend.zeros(a.size), backend.zeros(a.size), backend.from_host(a)) for a in arrays[1:]]
        self.ft_grad = backend.zeros(lay.rows_padded * sh.l1)
        self.dense_layout = dense_gradient_layout(sh.l1, sh.l2, sh.l3)
        self.dense_grad = backend.zeros(self.dense_layout[-1][1] + 1)
        ctx = getattr(backend, "ctx", None)
        n = batch_size * max_active
        if ctx is not None:
            self.stm_indices, self.nstm_indices = I32Buffer(ctx, n), I32Buffer(ctx, n)
            self.targets, self.entry_weights = F32Buffer(ctx, batch_size), F32Buffer(ctx, batch_size)
            self.output = F32Buffer(ctx, batch_size)
            self.loss_workspace = ScalarLossWorkspace(ctx, batch_size)
        # views for the update and the collectives
        self.ft_grad_shard = backend.view(self.ft_grad, lay.row_begin * sh.l1, lay.real_rows * sh.l1)
        self.l0w_shard = backend.view(self.weights[0], lay.row_begin * sh.l1, lay.real_rows * sh.l1)
        self.dense_views = [backend.view(self.dense_grad, off, n) for _, off, n in self.dense_layout]
        self._t_ft_grad = backend.tensor(self.ft_grad)
        self._t_l0w = backend.tensor(self.weights[0])
        self._t_dense = backend.tensor(self.dense_grad)

    def upload_batch(self, stm, nstm, targets, entry_weights) -> None:
        self.stm_indices.upload(stm)
        self.nstm_indices.upload(nstm)
        self.targets.upload(targets)
        self.entry_weights.upload(entry_weights)

    def exchange_and_update(self, params: RangerUpdateParams) -> None:
        lay, sh = self.layout, self.shape
        chunk = lay.shard_rows * sh.l1
        shard_t = self._t_ft_grad[self.rank * chunk:(self.rank + 1) * chunk]
        self.dist.reduce_scatter_tensor(shard_t, self._t_ft_grad)
        self.dist.all_reduce(self._t_dense)
        if lay.real_rows > 0:
            m, v, slow = self.ft_state
            self.backend.ranger(params, self.ft_grad_shard, self.l0w_shard, m, v, slow)
        for view, w, (m, v, slow) in zip(self.dense_views, self.weights[1:], self.small_state):
            self.backend.ranger(params, view, w, m, v, slow)
        own_t = self._t_l0w[self.rank * chunk:(self.rank + 1) * chunk]
        self.dist.all_gather_into_tensor(self._t_l0w, own_t)

    def step_device(self, params: RangerUpdateParams, loss_kind: ScalarLossKind, output_inv_scale: float,
                    finalize_loss: bool = True) -> None:
        spec = loss_kind.spec(output_inv_scale, finalize_loss, normalizer=self.batch_size * self.world)
        self.backend.local_gradients(self, spec)
        self.exchange_and_update(params)

    def read_weights(self) -> dict:
        out = {n: self.backend.download(w) for n, w in zip(NNUE_WEIGHT_NAMES, self.weights)}
        out["l0w"] = out["l0w"][: self.shape.input_size * self.shape.l1]
        return out


def sfnn_dense_gradient_layout(shape, present: dict) -> list[tuple[str, int, int]]:
    """(group, offset, length) of the packed SFNN small-parameter gradient:
    the groups after l0w in update order, absent shared factors omitted."""
    from .sfnn import SFNN_WEIGHT_NAMES

    lens = shape.weight_lengths()
    out, off = [], 0
    for name in SFNN_WEIGHT_NAMES[1:]:
        if present[name]:
            out.append((name, off, lens[name]))
            off += lens[name]
    return out


@dataclass(frozen=True)
class RowChunk:
    """One launch's FT rows in the data-parallel layout: table rows
    [start, start + length) sit at gradient rows start + shift ..., padded to
    `padded` rows (a multiple of the world size); each rank owns padded / world
    of them, stored from row `shard_off` of its compact shard."""

    start: int
    length: int
    padded: int
    shift: int
    shard_off: int
    shard_rows: int
    first_launch: int = 0  # row launches [first_launch, last_launch] complete the chunk
    last_launch: int = 0


def sfnn_row_chunks(row_ends: list, world: int, launches_per_chunk: int = 1,
                    last_chunk_launches: Optional[int] = None) -> list:
    """Chunks of `launches_per_chunk` consecutive row launches.  With
    `last_chunk_launches`, the last that many launches form a chunk of their
    own (a short last chunk leaves less exchange after the last launch); the
    chunk before it may then hold fewer."""
    n = len(row_ends)
    lpc = max(1, int(launches_per_chunk))
    tail = n if last_chunk_launches is None else max(1, min(n, int(last_chunk_launches)))
    head = n - tail if last_chunk_launches is not None else n
    bounds = [(i, min(head, i + lpc) - 1) for i in range(0, head, lpc)]
    if last_chunk_launches is not None:
        bounds.append((head, n - 1))
    chunks, shift, off, start = [], 0, 0, 0
    for first, last in bounds:
        end = row_ends[last]
        length = end - start
        padded = -(-length // world) * world
        chunks.append(RowChunk(start, length, padded, shift, off, padded // world, first, last))
        shift += padded - length
        off += padded // world
        start = end
    return chunks


class SfnnDataParallelTrainer:
    """One rank of data-parallel SFNN training (default layer multipliers).

    The FT gradient rows come from a sequence of row-kernel launches, each
    completing a contiguous range of rows (a few king blocks).  Consecutive
    launches form a chunk (`launches_per_chunk` of them, the last
    `last_chunk_launches` a chunk of their own), padded to a multiple of the
    world size: the chunk is reduce-scattered, the owned part updated by
    Ranger and all-gathered back, chunk by chunk.  On the GPU the chunks'
    collectives and updates run on a second stream, each starting when its
    last launch has finished (an event the library records), so the exchange
    overlaps the remaining launches, and its tail overlaps the next step's
    batch-only work."""

    def __init__(self, backend, dist, initial_weights, batch_size: int, max_active: int, alpha=None,
                 lr_multipliers=None, overlap: Optional[bool] = None, launches_per_chunk: int = 3,
                 last_chunk_launches: Optional[int] = 1, exchange: Optional[str] = None):
        from .sfnn import SFNN_WEIGHT_NAMES, SfnnFactorizerAlpha, SfnnLayerLrMultipliers

        initial_weights.validate()
        self.lr_multipliers = lr_multipliers or SfnnLayerLrMultipliers()
        self.backend = backend
        self.dist = dist
        self.world = dist.get_world_size()
        self.rank = dist.get_rank()
        self.shape = initial_weights.shape
        self.alpha = alpha or SfnnFactorizerAlpha()
        self.batch_size, self.max_active = batch_size, max_active
        sh = self.shape
        W = sh.ft_size
        self.row_ends = backend.sfnn_row_launches(sh, self.alpha)
        self.launches_per_chunk = max(1, int(launches_per_chunk))
        self.chunks = sfnn_row_chunks(self.row_ends, self.world, self.launches_per_chunk, last_chunk_launches)
        self.launch_chunk = [j for j, c in enumerate(self.chunks) for _ in range(c.first_launch, c.last_launch + 1)]
        self.timing = False  # GPU: record exchange events per step (exchange_timing)
        last = self.chunks[-1]
        grad_rows = last.start + last.shift + last.padded
        l0w_rows = last.start + last.padded  # a chunk's all-gather writes its padded length
        shard_rows = last.shard_off + last.shard_rows
        arrays = initial_weights.arrays()
        self.present = {n: arrays[n] is not None for n in SFNN_WEIGHT_NAMES}
        l0w = np.zeros(l0w_rows * W, np.float32)
        l0w[: arrays["l0w"].size] = arrays["l0w"]
        compact = np.zeros(shard_rows * W, np.float32)
        for c in self.chunks:
            r0 = c.start + self.rank * c.shard_rows
            n_real = max(0, min(c.shard_rows, c.start + c.length - r0))
            compact[c.shard_off * W:(c.shard_off + n_real) * W] = l0w[r0 * W:(r0 + n_real) * W]
        self.weights = {"l0w": backend.from_host(l0w)}
        for n in SFNN_WEIGHT_NAMES[1:]:
            self.weights[n] = None if arrays[n] is None else backend.from_host(arrays[n])
        self.l0w_compact = backend.from_host(compact)
        self.ft_state = (backend.zeros(shard_rows * W), backend.zeros(shard_rows * W), backend.from_host(compact))
        self.dense_layout = sfnn_dense_gradient_layout(sh, self.present)
        self.small_state = {n: (backend.zeros(arrays[n].size), backend.zeros(arrays[n].size), backend.from_host(arrays[n]))
                            for n, _, _ in self.dense_layout}
        self.ft_grad = backend.zeros(grad_rows * W)
        self.ft_grad_shard = backend.zeros(shard_rows * W)
        total = self.dense_layout[-1][1] + self.dense_layout[-1][2]
        self.dense_grad = backend.zeros(total)
        ctx = getattr(backend, "ctx", None)
        n = batch_size * max_active
        if ctx is not None:
            self.stm_indices, self.nstm_indices = I32Buffer(ctx, n), I32Buffer(ctx, n)
            self.buckets = I32Buffer(ctx, batch_size)
            self.targets, self.entry_weights = F32Buffer(ctx, batch_size), F32Buffer(ctx, batch_size)
            self.output = F32Buffer(ctx, batch_size)
            self.loss_workspace = ScalarLossWorkspace(ctx, batch_size)
        m, v, slow = self.ft_state
        self.chunk_views = [tuple(backend.view(b, c.shard_off * W, c.shard_rows * W)
                                  for b in (self.ft_grad_shard, self.l0w_compact, m, v, slow))
                            for c in self.chunks]
        self.dense_views = {name: backend.view(self.dense_grad, off, k) for name, off, k in self.dense_layout}
        self._t_ft_grad = backend.tensor(self.ft_grad)
        self._t_shard = backend.tensor(self.ft_grad_shard)
        self._t_l0w = backend.tensor(self.weights["l0w"])
        self._t_compact = backend.tensor(self.l0w_compact)
        self._t_dense = backend.tensor(self.dense_grad)
        self.overlap = bool(getattr(backend, "supports_overlap", False)) if overlap is None else bool(overlap)
        # "p2p": gradient rows stored into their owners' slots by the row
        # kernels, shards updated and stored into every table over NVLink;
        # "collectives": reduce-scatter / all-gather through the process group
        peer = bool(getattr(backend, "supports_peer_exchange", False)) and self.overlap
        self.exchange = exchange or ("p2p" if peer else "collectives")
        if self.exchange not in ("p2p", "collectives"):
            raise ValueError(f"exchange must be 'p2p' or 'collectives', got {self.exchange!r}")
        if self.exchange == "p2p" and not peer:
            raise ValueError("the p2p exchange needs a GPU backend with the overlapped step")
        if self.overlap:
            backend.prepare_overlap(self)
        if self.exchange == "p2p":
            backend.prepare_peer_exchange(self)

    def weight_list(self) -> list:
        from .sfnn import SFNN_WEIGHT_NAMES

        return [self.weights[n] for n in SFNN_WEIGHT_NAMES]

    def upload_batch(self, stm, nstm, buckets, targets, entry_weights) -> None:
        self.stm_indices.upload(stm)
        self.nstm_indices.upload(nstm)
        self.buckets.upload(buckets)
        self.targets.upload(targets)
        self.entry_weights.upload(entry_weights)

    def _params(self, params: RangerUpdateParams) -> RangerUpdateParams:
        from dataclasses import replace

        return replace(params, norm_loss_strength=0.0, norm_loss_before=False)  # lib.rs:6416-6420

    def _chunk_exchange(self, j: int, params: RangerUpdateParams, ctx=None, events=None) -> None:
        """Reduce-scatter chunk j, Ranger on the owned part, all-gather it back
        (events: optional timing events recorded on the current stream)."""
        c, W = self.chunks[j], self.shape.ft_size
        g0 = (c.start + c.shift) * W
        s0 = c.shard_off * W
        if events is not None:
            events["start"].record()
        self.dist.reduce_scatter_tensor(self._t_shard[s0:s0 + c.shard_rows * W],
                                        self._t_ft_grad[g0:g0 + c.padded * W])
        if events is not None:
            events["reduce_scatter"].record()
        grad, w, m, v, slow = self.chunk_views[j]
        self.backend.ranger(params, grad, w, m, v, slow, ctx)
        if events is not None:
            events["ranger"].record()
        self.dist.all_gather_into_tensor(self._t_l0w[c.start * W:(c.start + c.padded) * W],
                                         self._t_compact[s0:s0 + c.shard_rows * W])
        if events is not None:
            events["all_gather"].record()

    def _small_exchange(self, params: RangerUpdateParams, ctx=None) -> None:
        from .sfnn import factor_contribution_clip

        if self.exchange == "p2p":
            # every rank's small gradient is in this rank's slots (stored by
            # the local-gradients entry): sum them in rank order
            self.backend.lib.call("bulletou_b200_exchange_reduce_small_device", ctx.as_ptr(), ctypes.byref(self._x),
                                  self.dense_grad.as_ptr(), self._flags.as_ptr(), self._xerr.as_ptr())
        else:
            self.dist.all_reduce(self._t_dense)
        for name, _, _ in self.dense_layout:
            p = factor_contribution_clip(params, self.alpha.shared) if name in ("l1fw", "l1fb") else params
            m, v, slow = self.small_state[name]
            self.backend.ranger(p, self.dense_views[name], self.weights[name], m, v, slow, ctx)

    def exchange_and_update(self, params: RangerUpdateParams) -> None:
        params = self._params(params)
        self._small_exchange(params)
        for j in range(len(self.chunks)):
            self._chunk_exchange(j, params)

    def step_device(self, params: RangerUpdateParams, loss_kind: ScalarLossKind, output_inv_scale: float,
                    finalize_loss: bool = True) -> None:
        spec = loss_kind.spec(output_inv_scale, finalize_loss, normalizer=self.batch_size * self.world)
        if self.exchange == "p2p":
            self.backend.sfnn_step_peer_exchange(self, spec, self._params(params))
            return
        if self.overlap:
            self.backend.sfnn_step_overlapped(self, spec, self._params(params))
            return
        self.backend.sfnn_local_gradients(self, spec)
        self.exchange_and_update(params)

    def join(self) -> None:
        """Makes the library's stream wait for this rank's outstanding exchange."""
        if self.overlap:
            self.backend.join_overlap(self)

    def check(self) -> None:
        """Waits for the device and raises if a peer-exchange wait timed out."""
        self.join()
        if self.exchange == "p2p":
            self.backend.check_peer_exchange(self)

    def close(self) -> None:
        """Unmaps the peers' buffers (peer exchange); call on every rank
        after the last step, before the process group goes."""
        if self.exchange == "p2p":
            self.check()
            self.dist.barrier()
            self.backend.close_peer_exchange(self)

    def read_weights(self) -> dict:
        self.check()
        out = {n: self.backend.download(w) for n, w in self.weights.items() if w is not None}
        out["l0w"] = out["l0w"][: self.shape.input_size * self.shape.ft_size]
        return out


def run_data_parallel_bench(args, rank: int, world: int, local: int, dist):
    """bench.py's N>1 arm: weak scaling, args.batch positions per rank."""
    import time

    import torch

    import bench
    import bulletou_b200 as bo
    from bulletou_b200 import synthetic

    backend = B200Backend(local)
    w = synthetic.halfkp_weights(synthetic.rng_for(7))
    tr = NnueDataParallelTrainer(backend, dist, bo.NnueForwardHostWeights(bo.NnueForwardShape(*bench.SHAPE), **w),
                                 args.batch, bench.ACTIVE)
    batches = bench.make_batches(args.batch, rank)
    dev = bench.device_batches(backend.ctx, batches)
    loss_kind = bo.ScalarLossKind.SigmoidPow(2.0)
    inv = 1.0 / 600.0
    step = 0

    def bind(i):
        tr.stm_indices, tr.nstm_indices, tr.targets, tr.entry_weights = dev[i % len(dev)]

    for i in range(args.warmup):
        step += 1
        bind(i)
        tr.step_device(bench.ranger(step), loss_kind, inv, finalize_loss=False)
    torch.cuda.synchronize()
    dist.barrier()
    lib, ctx = backend.lib, backend.ctx
    start, stop = bo.Event(ctx), bo.Event(ctx)
    lib.call("bulletou_b200_profile_begin", ctx.as_ptr(), 8 * args.steps + 8)
    with bench.ClockSampler(local) as clocks:
        start.record(ctx)
        for i in range(args.steps):
            step += 1
            bind(i)
            tr.step_device(bench.ranger(step), loss_kind, inv, finalize_loss=False)
        stop.record(ctx)
        stop.synchronize()
    ms = (ctypes.c_float * 8)()
    nsteps, nphases = ctypes.c_size_t(), ctypes.c_size_t()
    lib.call("bulletou_b200_profile_end", ctx.as_ptr(), ms, 8, ctypes.byref(nsteps), ctypes.byref(nphases))
    torch.cuda.synchronize()
    dist.barrier()
    total_ms = bench.max_over_ranks(dist, stop.elapsed_ms_since(start))
    phase_ms = {bench.PHASES[p]: ms[p] / max(1, nsteps.value) for p in range(nphases.value)}
    # end to end: per step the batch H2D from page-locked host memory through
    # the ABI's *_upload entries, the step, a synchronous read of the mean loss
    from bulletou_b200.cuda_cpp import upload_from_pinned

    sources = [bench.PinnedHostBatch((b["stm"], b["nstm"], b["targets"], b["entry_weights"])) for b in batches]
    in_bufs = (I32Buffer(ctx, args.batch * bench.ACTIVE), I32Buffer(ctx, args.batch * bench.ACTIVE),
               F32Buffer(ctx, args.batch), F32Buffer(ctx, args.batch))
    tr.stm_indices, tr.nstm_indices, tr.targets, tr.entry_weights = in_bufs
    dist.barrier()
    e0, e1 = bo.Event(ctx), bo.Event(ctx)
    losses = []
    t0 = time.perf_counter()
    e0.record(ctx)
    for i in range(args.steps):
        step += 1
        for dst, src in zip(in_bufs, sources[i % len(sources)].pinned):
            upload_from_pinned(ctx, dst, src)
        tr.step_device(bench.ranger(step), loss_kind, inv, finalize_loss=True)
        losses.append(float(tr.loss_workspace.mean.download(ctx)[0]))
    e1.record(ctx)
    e1.synchronize()
    wall_ms = (time.perf_counter() - t0) * 1000.0
    e2e_ms = bench.max_over_ranks(dist, max(e1.elapsed_ms_since(e0), wall_ms))
    assert all(np.isfinite(losses)), "non-finite loss"
    return {"total_ms": total_ms, "phase_ms": phase_ms, "clocks": clocks.summary(),
            "e2e": {"value": args.steps * args.batch * world / (e2e_ms / 1000.0), "unit": "positions/s",
                    "h2d_bytes_per_step": int(sources[0].nbytes), "d2h_bytes_per_step": 4, "steps": args.steps,
                    "path": "NnueDataParallelTrainer.step_device per rank (NCCL reduce-scatter / all-reduce / "
                            "all-gather), inputs from page-locked host memory, mean loss read back every step"},
            "gpu_launches": (bench.LAUNCHES_PER_STEP + 8) * args.steps,
            "final_loss": losses[-1]}
