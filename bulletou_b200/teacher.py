"""Teacher-batch producer: YaneuraOu PackedSfenValue records -> the sparse
batch a train step consumes, built on the device.

Host-side mirror of the reference's batch preparation for the cuda-cpp
trainers (crates/bulletou_lib/src/value/teacher_batch.rs): the SFNN path
(prepare_sfnn_fast_batch_from_board_features, :2869-3010; HalfKA_hm2 features,
LayerStack bucket, target ``(1 - lambda) * result + lambda' * p(score)``) and
the HalfKP path (prepare_halfkp_direct_fast_batch, :1687-1750).  The decode
itself runs in libbulletou_b200 (``bulletou_b200_teacher_prepare_device``);
only 40 bytes per position cross PCIe instead of the ~330-byte prepared rows.

Configuration names follow SfnnTeacherBatchConfig / HalfkpTeacherBatchConfig
(teacher_batch.rs:60-165): ``lambda_``, ``scale``, ``win_rate_model`` with
``wrm_target`` (WinRateModelTargetParams, value/loader.rs:646-690),
``score_drop_abs`` and the LayerStack bucket kind (game/outputs.rs:1024-1160).
Progress buckets (trainable progress features) are not produced here.
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass, field
from typing import Optional

import numpy as np

from ._lib import CudaCppError, TeacherConfig
from .cuda_cpp import Context, Event, F32Buffer, I32Buffer, PinnedI32Buffer

PSV_RECORD_BYTES = 40
PSV_RECORD_WORDS = PSV_RECORD_BYTES // 4
# PackedSfenValue layout (crates/bulletou_lib/src/shogi/packed_sfen.rs:122-137).
PSV_DTYPE = np.dtype([("sfen", "u1", 32), ("score", "<i2"), ("move16", "<u2"), ("game_ply", "<u2"),
                      ("game_result", "i1"), ("padding", "u1")])
assert PSV_DTYPE.itemsize == PSV_RECORD_BYTES

FEATURE_SETS = {"halfka_hm2": 0, "halfkp": 1}
FEATURE_MAX_ACTIVE = {"halfka_hm2": 40, "halfkp": 38}
FEATURE_INPUTS = {"halfka_hm2": 45 * 1629, "halfkp": 81 * 1548}
# ShogiSfnnHandBucketKind / ShogiSfnnKingBucketKind (game/outputs.rs:826-905) in ABI order.
HAND_BUCKET_KINDS = ("none", "hand4", "hand16", "hand64", "hand64z", "hand256", "hand1024")
KING_BUCKET_KINDS = ("none", "kingrank9", "kingrank81", "k9k9z", "k13k13z", "k21k21", "k21k21z", "k29k29")
_HAND_COUNTS = (1, 4, 16, 64, 64, 256, 1024)
_KING_COUNTS = (1, 9, 81, 81, 169, 441, 441, 841)

DEFAULT_WRM_TARGET_OFFSET = 270.0
DEFAULT_WRM_TARGET_SCALING = 380.0


@dataclass(frozen=True)
class LayerStackBucketKind:
    """ShogiSfnnLayerStackBucketKind without the progress axis; the default is
    KingRank9 like the reference (outputs.rs:1034-1038)."""

    hand: str = "none"
    king: str = "kingrank9"

    def validate(self) -> None:
        if self.hand not in HAND_BUCKET_KINDS:
            raise CudaCppError(f"unknown hand bucket kind {self.hand!r}")
        if self.king not in KING_BUCKET_KINDS:
            raise CudaCppError(f"unknown king bucket kind {self.king!r}")

    @property
    def num_stacks(self) -> int:
        return _HAND_COUNTS[HAND_BUCKET_KINDS.index(self.hand)] * _KING_COUNTS[KING_BUCKET_KINDS.index(self.king)]


@dataclass(frozen=True)
class WinRateModelTargetParams:
    """WinRateModelTargetParams (value/loader.rs:646-673)."""

    offset: float = DEFAULT_WRM_TARGET_OFFSET
    scaling: float = DEFAULT_WRM_TARGET_SCALING
    epsilon: float = 0.0

    def validate(self) -> None:
        ok = (math.isfinite(self.offset) and math.isfinite(self.scaling) and self.scaling > 0.0
              and math.isfinite(self.epsilon) and 0.0 <= self.epsilon < 0.5)
        if not ok:
            raise CudaCppError(f"invalid win-rate-model target params {self}")


def win_rate_model_score_table(params: WinRateModelTargetParams) -> np.ndarray:
    """probability(score) for every i16 score, index score + 32768
    (build_win_rate_model_score_table, value/loader.rs:681-687), in f32 with
    each exp evaluated in double and rounded once."""
    params.validate()
    f32 = np.float32
    score = np.arange(-32768, 32768, dtype=np.float32)
    off, sc, eps = f32(params.offset), f32(params.scaling), f32(params.epsilon)
    p = ((score - off) / sc).astype(np.float32)
    pm = ((-score - off) / sc).astype(np.float32)

    def sigmoid(x):
        with np.errstate(over="ignore"):                   # exp past f32 range is inf, as expf gives
            e = np.exp(-x.astype(np.float64)).astype(np.float32)
        return (f32(1.0) / (f32(1.0) + e)).astype(np.float32)

    prob = (f32(0.5) * ((f32(1.0) + sigmoid(p)) - sigmoid(pm))).astype(np.float32)
    if eps == 0.0:
        return prob
    return (eps + (f32(1.0) - f32(2.0) * eps) * prob).astype(np.float32)


@dataclass(frozen=True)
class TeacherBatchConfig:
    """What the producer needs from SfnnTeacherBatchConfig / HalfkpTeacherBatchConfig."""

    feature_set: str = "halfka_hm2"
    lambda_: float = 1.0
    scale: float = 600.0
    win_rate_model: bool = False
    wrm_target: WinRateModelTargetParams = field(default_factory=WinRateModelTargetParams)
    score_drop_abs: Optional[int] = None
    layerstack_bucket: LayerStackBucketKind = field(default_factory=LayerStackBucketKind)
    max_active: Optional[int] = None

    def validate(self) -> None:
        if self.feature_set not in FEATURE_SETS:
            raise CudaCppError(f"unknown feature set {self.feature_set!r}")
        if not (math.isfinite(self.lambda_) and 0.0 <= self.lambda_ <= 1.0):
            raise CudaCppError(f"lambda must be finite and in [0, 1] (got {self.lambda_})")
        if not (math.isfinite(self.scale) and self.scale > 0.0):
            raise CudaCppError(f"scale must be finite and positive (got {self.scale})")
        if self.score_drop_abs is not None and not 0 <= int(self.score_drop_abs) <= 65535:
            raise CudaCppError(f"score_drop_abs must fit in u16 (got {self.score_drop_abs})")
        self.layerstack_bucket.validate()
        if self.win_rate_model:
            self.wrm_target.validate()
        if self.active < 1 or self.active > 48:
            raise CudaCppError(f"max_active must be in 1..48 (got {self.active})")

    @property
    def active(self) -> int:
        return int(self.max_active if self.max_active is not None else FEATURE_MAX_ACTIVE[self.feature_set])

    @property
    def num_inputs(self) -> int:
        return FEATURE_INPUTS[self.feature_set]

    def blends(self) -> tuple:
        """(result_blend, score_blend) in f32 as each path forms them: the SFNN
        path weighs the score by 1 - (1 - lambda) (teacher_batch.rs:2907,
        2997), the HalfKP path by lambda itself (:1706-1707, 1744)."""
        f32 = np.float32
        result_blend = f32(1.0) - f32(self.lambda_)
        if self.feature_set == "halfka_hm2":
            return float(result_blend), float(f32(1.0) - result_blend)
        return float(result_blend), float(f32(self.lambda_))

    def as_struct(self) -> TeacherConfig:
        rb, sb = self.blends()
        lb = self.layerstack_bucket
        hand = HAND_BUCKET_KINDS.index(lb.hand) if self.feature_set == "halfka_hm2" else 0
        king = KING_BUCKET_KINDS.index(lb.king) if self.feature_set == "halfka_hm2" else 0
        return TeacherConfig(FEATURE_SETS[self.feature_set], self.active, hand, king, rb, sb,
                             float(np.float32(1.0) / np.float32(self.scale)),
                             -1 if self.score_drop_abs is None else int(self.score_drop_abs))


def records_as_words(records) -> np.ndarray:
    """PackedSfenValue records (PSV_DTYPE array, uint8 [n, 40] or raw bytes) as
    int32 words, 10 per record."""
    if isinstance(records, (bytes, bytearray, memoryview)):
        a = np.frombuffer(records, dtype=np.uint8)
    else:
        a = np.asarray(records)
    if a.dtype == PSV_DTYPE:
        a = a.view(np.uint8)
    a = np.ascontiguousarray(a).reshape(-1)
    if a.dtype != np.uint8 and a.dtype != np.int32:
        a = a.view(np.uint8)
    if a.dtype == np.uint8:
        if a.size % PSV_RECORD_BYTES:
            raise CudaCppError(f"teacher records must be {PSV_RECORD_BYTES}-byte PackedSfenValue records "
                               f"(got {a.size} bytes)")
        a = a.view(np.int32)
    return a


def teacher_prepare_device(ctx: Context, config: TeacherBatchConfig, records: I32Buffer, n_records: int,
                           stm: I32Buffer, nstm: I32Buffer, buckets: Optional[I32Buffer], targets: F32Buffer,
                           entry_weights: F32Buffer, overflow: I32Buffer,
                           wrm_table: Optional[F32Buffer] = None) -> None:
    """One launch of the device producer over `n_records` records already in
    `records`; `overflow` accumulates the records with too many features."""
    config.validate()
    if config.win_rate_model and wrm_table is None:
        raise CudaCppError("win_rate_model targets need the device score table")
    s = config.as_struct()
    ctx.lib.call("bulletou_b200_teacher_prepare_device", ctx.as_ptr(), ctypes.byref(s), records.as_ptr(),
                 int(n_records), None if wrm_table is None else wrm_table.as_ptr(), stm.as_ptr(), nstm.as_ptr(),
                 None if buckets is None else buckets.as_ptr(), targets.as_ptr(), entry_weights.as_ptr(),
                 overflow.as_ptr())


class TeacherBatch:
    """Device sparse batch (the layout FastBatchHost carries, value/fast_batch.rs)."""

    def __init__(self, ctx: Optional[Context], batch_size: int, max_active: int, buffers: Optional[tuple] = None):
        self.batch_size, self.max_active = int(batch_size), int(max_active)
        if buffers is not None:
            self.stm_indices, self.nstm_indices, self.buckets, self.targets, self.entry_weights = buffers
            return
        n = self.batch_size * self.max_active
        self.stm_indices, self.nstm_indices = I32Buffer(ctx, n), I32Buffer(ctx, n)
        self.buckets = I32Buffer(ctx, self.batch_size)
        self.targets, self.entry_weights = F32Buffer(ctx, self.batch_size), F32Buffer(ctx, self.batch_size)

    @classmethod
    def wrap(cls, stm, nstm, buckets, targets, entry_weights, batch_size: int, max_active: int) -> "TeacherBatch":
        """A view over existing device buffers (a runner's own batch)."""
        return cls(None, batch_size, max_active, (stm, nstm, buckets, targets, entry_weights))

    def download(self, ctx: Optional[Context] = None) -> dict:
        A = self.max_active
        return {"stm": self.stm_indices.download(ctx).reshape(-1, A),
                "nstm": self.nstm_indices.download(ctx).reshape(-1, A),
                "buckets": self.buckets.download(ctx), "targets": self.targets.download(ctx),
                "entry_weights": self.entry_weights.download(ctx)}


class TeacherBatchProducer:
    """Uploads PackedSfenValue records and decodes them into a TeacherBatch on
    the device.  ``prepare`` is synchronous-safe for pageable arrays; the
    pinned path (``stage`` + ``upload_and_prepare``) is what a pipelined
    trainer uses: the 40-byte records cross PCIe, the decode runs on the
    upload stream, and an event hands the batch to the compute stream."""

    def __init__(self, ctx: Context, config: TeacherBatchConfig, batch_size: int, pinned: bool = True):
        config.validate()
        self.ctx = ctx
        self.config = config
        self.batch_size = int(batch_size)
        if self.batch_size <= 0:
            raise CudaCppError("teacher batch_size must be greater than zero")
        self.records = I32Buffer(ctx, self.batch_size * PSV_RECORD_WORDS)
        self.pinned = PinnedI32Buffer(ctx, self.batch_size * PSV_RECORD_WORDS) if pinned else None
        self.overflow = I32Buffer.from_host(ctx, np.zeros(1, np.int32))
        self._overflow_seen = 0
        self.wrm_table = (F32Buffer.from_host(ctx, win_rate_model_score_table(config.wrm_target))
                          if config.win_rate_model else None)
        self.ready = Event(ctx)

    def new_batch(self) -> TeacherBatch:
        return TeacherBatch(self.ctx, self.batch_size, self.config.active)

    def _words(self, records) -> np.ndarray:
        w = records_as_words(records)
        if w.size != self.batch_size * PSV_RECORD_WORDS:
            raise CudaCppError(f"teacher batch holds {w.size // PSV_RECORD_WORDS} records, "
                               f"expected {self.batch_size}")
        return w

    def decode(self, ctx: Context, out: TeacherBatch) -> None:
        """Decode the records already in ``self.records`` into `out`."""
        teacher_prepare_device(ctx, self.config, self.records, self.batch_size, out.stm_indices, out.nstm_indices,
                               out.buckets if self.config.feature_set == "halfka_hm2" else None, out.targets,
                               out.entry_weights, self.overflow, self.wrm_table)

    def prepare(self, ctx: Context, records, out: TeacherBatch) -> None:
        self.records.upload(self._words(records), ctx)
        self.decode(ctx, out)

    def stage(self, records) -> int:
        """Copy records into the pinned staging buffer; returns the bytes."""
        if self.pinned is None:
            raise CudaCppError("this producer was created without a pinned staging buffer")
        w = self._words(records)
        np.copyto(self.pinned.host(), w)
        return w.size * 4

    def upload_and_prepare(self, upload_ctx: Context, out: TeacherBatch) -> int:
        """Async H2D of the staged records and the decode, both on `upload_ctx`;
        records ``self.ready`` after them.  Returns the H2D bytes."""
        upload_ctx.lib.call("bulletou_b200_i32_upload_pinned", upload_ctx.as_ptr(), self.records.as_ptr(),
                            self.pinned.as_ptr(), self.pinned.length)
        self.decode(upload_ctx, out)
        self.ready.record(upload_ctx)
        return self.pinned.length * 4

    def check(self, ctx: Optional[Context] = None) -> None:
        """Raises like the reference's assert when a decoded record had more
        features than max_active (teacher_batch.rs:2927-2930, 1726-1729)."""
        seen = int(self.overflow.download(ctx)[0])
        if seen != self._overflow_seen:
            bad = seen - self._overflow_seen
            self._overflow_seen = seen
            label = "SFNN/halfkahm2" if self.config.feature_set == "halfka_hm2" else "HalfKP"
            raise CudaCppError(f"{label} active feature count exceeded max_active {self.config.active} "
                               f"({bad} record(s))")


class TeacherUploadSlot:
    """One slot of a pipelined record feed: pinned records, device records, the
    decoded device batch and the hand-off events (the record-level analogue of
    SfnnTrainStepUploadSlot, crates/cuda_cpp/src/lib.rs:6087-6186)."""

    def __init__(self, ctx: Context, producer: TeacherBatchProducer):
        n = producer.batch_size * PSV_RECORD_WORDS
        self.records = I32Buffer(ctx, n)
        self.pinned = PinnedI32Buffer(ctx, n)
        self.batch = producer.new_batch()
        self.upload_ready = Event(ctx)
        self.compute_done = Event(ctx)
        self.in_use = False

    def fill(self, records) -> None:
        np.copyto(self.pinned.host(), records_as_words(records))

    def upload(self, upload_ctx: Context, producer: TeacherBatchProducer, records=None,
               pinned_source: Optional["TeacherUploadSlot"] = None) -> int:
        """H2D of the records and their decode on `upload_ctx` once the step
        that last used this slot has finished; returns the H2D bytes."""
        if self.in_use:
            self.upload_ready.synchronize()          # the pinned copy of the previous upload is done
            self.compute_done.wait(upload_ctx)       # the step that read this batch is done
        src = self.pinned if pinned_source is None else pinned_source.pinned
        if pinned_source is None:
            if records is None:
                raise CudaCppError("an upload needs records or a pinned source")
            self.fill(records)
        upload_ctx.lib.call("bulletou_b200_i32_upload_pinned", upload_ctx.as_ptr(), self.records.as_ptr(),
                            src.as_ptr(), src.length)
        teacher_prepare_device(upload_ctx, producer.config, self.records, producer.batch_size,
                               self.batch.stm_indices, self.batch.nstm_indices,
                               self.batch.buckets if producer.config.feature_set == "halfka_hm2" else None,
                               self.batch.targets, self.batch.entry_weights, producer.overflow, producer.wrm_table)
        self.upload_ready.record(upload_ctx)
        self.in_use = True
        return src.length * 4


# ------------------------------------------------------------------ HCPE records
HCPE_RECORD_BYTES = 38


def hcpe_to_psv_device(ctx: Context, hcpe: I32Buffer, n_records: int, psv: I32Buffer, count: I32Buffer,
                       valid: Optional[I32Buffer] = None) -> None:
    """HCPE records (38 bytes each, back to back in `hcpe`) -> PackedSfenValue
    records, the valid ones compacted in input order into `psv`, their number
    into count[0] (decode_hcpe_record, value/loader/hcpe.rs:65-76)."""
    ctx.lib.call("bulletou_b200_hcpe_to_psv_device", ctx.as_ptr(), hcpe.as_ptr(), int(n_records), psv.as_ptr(),
                 count.as_ptr(), None if valid is None else valid.as_ptr())


class HcpeConverter:
    """Uploads up to `capacity` HCPE records and converts them on the device
    into PackedSfenValue records that TeacherBatchProducer decodes; invalid
    records are dropped like the reference's loader drops them."""

    def __init__(self, ctx: Context, capacity: int):
        self.ctx = ctx
        self.capacity = int(capacity)
        self.hcpe = I32Buffer(ctx, (self.capacity * HCPE_RECORD_BYTES + 3) // 4)
        self.psv = I32Buffer(ctx, self.capacity * PSV_RECORD_WORDS)
        self.count = I32Buffer(ctx, 1)
        self.valid = I32Buffer(ctx, self.capacity)

    def convert(self, ctx: Context, records) -> int:
        """Converts `records` (HCPE_DTYPE array, uint8 [n, 38] or bytes);
        returns how many were valid (a device-to-host read)."""
        if isinstance(records, (bytes, bytearray, memoryview)):
            a = np.frombuffer(records, dtype=np.uint8)
        else:
            a = np.asarray(records)
            if a.dtype.fields is not None:
                a = np.atleast_1d(a).view(np.uint8)
        a = np.ascontiguousarray(a, dtype=np.uint8).reshape(-1)
        if a.size % HCPE_RECORD_BYTES:
            raise CudaCppError(f"HCPE records must be {HCPE_RECORD_BYTES}-byte records (got {a.size} bytes)")
        n = a.size // HCPE_RECORD_BYTES
        if n > self.capacity:
            raise CudaCppError(f"{n} HCPE records exceed the converter capacity {self.capacity}")
        words = np.zeros(self.hcpe.length * 4, np.uint8)
        words[:a.size] = a
        self.hcpe.upload(words.view(np.int32), ctx)
        hcpe_to_psv_device(ctx, self.hcpe, n, self.psv, self.count, self.valid)
        return int(self.count.download(ctx)[0])
