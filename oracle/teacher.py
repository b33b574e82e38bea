"""TEST INFRASTRUCTURE ONLY -- ctypes driver of oracle/teacher_oracle.c, the
CPU restatement of the reference's teacher-batch producer (PackedSfenValue
decode, HalfKA_hm2 / HalfKP features, LayerStack bucket, targets).  Only
tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import it, as
the checker; the product (bulletou_b200) never does."""
from __future__ import annotations

import ctypes

import numpy as np

from . import oracle as _oracle

_ready = False


class TeacherConfig(ctypes.Structure):
    """oracle_teacher_config (same field order as the product's ABI struct)."""

    _fields_ = [("feature_set", ctypes.c_int32), ("max_active", ctypes.c_int32), ("hand_bucket", ctypes.c_int32),
                ("king_bucket", ctypes.c_int32), ("result_blend", ctypes.c_float), ("score_blend", ctypes.c_float),
                ("rscale", ctypes.c_float), ("score_drop_abs", ctypes.c_int32)]


HAND_KINDS = ("none", "hand4", "hand16", "hand64", "hand64z", "hand256", "hand1024")
KING_KINDS = ("none", "kingrank9", "kingrank81", "k9k9z", "k13k13z", "k21k21", "k21k21z", "k29k29")


def lib():
    global _ready
    L = _oracle.lib()
    if not _ready:
        p, i, i64, f = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_float
        L.oracle_teacher_prepare.argtypes = [p, i64, p, p, p, p, p, p, p, p]
        L.oracle_teacher_prepare.restype = None
        L.oracle_psv_decode.argtypes = [p, p, p, p]
        L.oracle_psv_decode.restype = i
        L.oracle_decode_piece.argtypes = [p, i, i, p]
        L.oracle_decode_piece.restype = None
        L.oracle_read_bits.argtypes = [p, i, p, i, p, p]
        L.oracle_read_bits.restype = None
        L.oracle_halfka_hm2_index.argtypes = [i64, i64]
        L.oracle_halfka_hm2_index.restype = i64
        L.oracle_bona_board.argtypes = [i, i, i, i]
        L.oracle_bona_board.restype = i
        L.oracle_bona_hand.argtypes = [i, i, i, i]
        L.oracle_bona_hand.restype = i
        L.oracle_king_single_bucket.argtypes = [i, i]
        L.oracle_king_single_bucket.restype = i
        L.oracle_hand_single_bucket.argtypes = [i, p]
        L.oracle_hand_single_bucket.restype = i
        L.oracle_teacher_bucket_count.argtypes = [i, i]
        L.oracle_teacher_bucket_count.restype = i
        L.oracle_wrm_table.argtypes = [f, f, f, p]
        L.oracle_wrm_table.restype = None
        L.oracle_hcpe_to_psv.argtypes = [p, p]
        L.oracle_hcpe_to_psv.restype = i
        L.oracle_validation_metrics.argtypes = [p, p, p, i64, p, p, p, p]
        L.oracle_validation_metrics.restype = None
        _ready = True
    return L


def _u8(data) -> np.ndarray:
    a = np.asarray(data)
    if a.dtype.fields is not None:
        a = np.atleast_1d(a).view(np.uint8)
    return np.ascontiguousarray(a, dtype=np.uint8).reshape(-1)


def _p(a):
    return ctypes.c_void_p(a.ctypes.data)


def config(feature_set="halfka_hm2", max_active=None, hand="none", king="kingrank9", lambda_=1.0, scale=600.0,
           score_drop_abs=None) -> TeacherConfig:
    """The blends each reference path forms (teacher_batch.rs:1706-1707, 2907)."""
    f32 = np.float32
    rb = f32(1.0) - f32(lambda_)
    sb = f32(1.0) - rb if feature_set == "halfka_hm2" else f32(lambda_)
    fs = 0 if feature_set == "halfka_hm2" else 1
    A = max_active if max_active is not None else (40 if fs == 0 else 38)
    return TeacherConfig(fs, A, HAND_KINDS.index(hand), KING_KINDS.index(king), float(rb), float(sb),
                         float(f32(1.0) / f32(scale)), -1 if score_drop_abs is None else int(score_drop_abs))


def prepare(records, cfg: TeacherConfig, wrm_table=None) -> dict:
    data = _u8(records)
    n = data.size // 40
    A = cfg.max_active
    out = {"stm": np.empty((n, A), np.int32), "nstm": np.empty((n, A), np.int32),
           "buckets": np.empty(n, np.int32), "targets": np.empty(n, np.float32),
           "entry_weights": np.empty(n, np.float32), "counts": np.empty(n, np.int32)}
    table = None if wrm_table is None else np.ascontiguousarray(wrm_table, np.float32)
    lib().oracle_teacher_prepare(_p(data), n, ctypes.byref(cfg), None if table is None else _p(table),
                                 _p(out["stm"]), _p(out["nstm"]), _p(out["buckets"]), _p(out["targets"]),
                                 _p(out["entry_weights"]), _p(out["counts"]))
    return out


def decode(record) -> dict:
    data = _u8(record)
    board = np.empty(81, np.uint8)
    hands = np.empty((2, 7), np.uint8)
    header = np.empty(6, np.int32)
    cursor = lib().oracle_psv_decode(_p(data), _p(board), _p(hands), _p(header))
    return {"board": board, "hands": hands, "stm": int(header[0]), "black_king": int(header[1]),
            "white_king": int(header[2]), "score": int(header[3]), "game_ply": int(header[4]),
            "game_result": int(header[5]), "cursor_after_board": int(cursor)}


def decode_piece(data, hand: bool) -> dict:
    d = _u8(data)
    out = np.empty(4, np.int32)
    lib().oracle_decode_piece(_p(d), d.size, int(hand), _p(out))
    return {"type": int(out[0]), "color": int(out[1]), "piecebox": bool(out[2]), "cursor": int(out[3])}


def read_bits(data, widths) -> tuple:
    d = _u8(data)
    w = np.ascontiguousarray(widths, np.int32)
    vals = np.empty(w.size, np.uint32)
    cur = np.empty(w.size, np.int32)
    lib().oracle_read_bits(_p(d), d.size, _p(w), w.size, _p(vals), _p(cur))
    return vals.tolist(), cur.tolist()


def hm2_index(king: int, bp: int) -> int:
    return int(lib().oracle_halfka_hm2_index(king, bp))


def bona_board(pt: int, color: int, sq: int, perspective: int) -> int:
    return int(lib().oracle_bona_board(pt, color, sq, perspective))


def bona_hand(perspective: int, owner: int, pt: int, count: int) -> int:
    return int(lib().oracle_bona_hand(perspective, owner, pt, count))


def king_single_bucket(kind: str, sq: int) -> int:
    return int(lib().oracle_king_single_bucket(KING_KINDS.index(kind), sq))


def hand_single_bucket(kind: str, hand) -> int:
    h = np.ascontiguousarray(hand, np.uint8)
    return int(lib().oracle_hand_single_bucket(HAND_KINDS.index(kind), _p(h)))


def bucket_count(hand: str, king: str) -> int:
    return int(lib().oracle_teacher_bucket_count(HAND_KINDS.index(hand), KING_KINDS.index(king)))


def wrm_table(offset=270.0, scaling=380.0, epsilon=0.0) -> np.ndarray:
    t = np.empty(65536, np.float32)
    lib().oracle_wrm_table(offset, scaling, epsilon, _p(t))
    return t


class ValidationConfig(ctypes.Structure):
    """oracle_validation_config (same field order as the product's ABI struct)."""

    _fields_ = [("have_results", ctypes.c_int32), ("score_drop_abs", ctypes.c_int32), ("loss_kind", ctypes.c_int32),
                ("lambda_", ctypes.c_float), ("eval_scale", ctypes.c_float), ("model_output_scale", ctypes.c_float),
                ("pow_exp", ctypes.c_float), ("nnue2score", ctypes.c_float), ("in_offset", ctypes.c_float),
                ("in_scaling", ctypes.c_float)]


VALIDATION_COUNTS = ("compared", "sign_matches", "predicted_nonnegative", "predicted_negative", "predicted_zero",
                     "drawn_games", "filtered_by_score_cap", "loss_sampled")


def validation_metrics(outputs, scores, results=None, score_drop_abs=None, lambda_=1.0, eval_scale=400.0,
                       model_output_scale=1.0, loss_kind=0, pow_exp=2.0, nnue2score=600.0, in_offset=270.0,
                       in_scaling=380.0, wrm_table=None) -> dict:
    """compute_sign_accuracy_with_loss_masked; returns the counts, loss_sum and
    test_loss (None without results or samples)."""
    o = np.ascontiguousarray(outputs, np.float32).reshape(-1)
    s = np.ascontiguousarray(scores, np.int16).reshape(-1)
    r = None if results is None or len(results) == 0 else np.ascontiguousarray(results, np.int8).reshape(-1)
    cfg = ValidationConfig(int(r is not None), -1 if score_drop_abs is None else int(score_drop_abs), int(loss_kind),
                           float(lambda_), float(eval_scale), float(model_output_scale), float(pow_exp),
                           float(nnue2score), float(in_offset), float(in_scaling))
    table = None if wrm_table is None else np.ascontiguousarray(wrm_table, np.float32)
    counts = np.zeros(8, np.int64)
    loss = ctypes.c_double()
    lib().oracle_validation_metrics(_p(o), _p(s), None if r is None else _p(r), o.size, ctypes.byref(cfg),
                                    None if table is None else _p(table), _p(counts), ctypes.byref(loss))
    out = dict(zip(VALIDATION_COUNTS, counts.tolist()))
    out["loss_sum"] = loss.value
    out["test_loss"] = float(np.float32(loss.value / out["loss_sampled"])) if out["loss_sampled"] else None
    return out


def hcpe_to_psv(records) -> tuple:
    """(PackedSfenValue records of the valid HCPE records in input order,
    per-record valid flags) -- decode_hcpe_record on each 38-byte record."""
    data = _u8(records)
    n = data.size // 38
    out = np.zeros((n, 40), np.uint8)
    valid = np.zeros(n, np.int32)
    L = lib()
    for i in range(n):
        rec = np.ascontiguousarray(data[38 * i:38 * (i + 1)])
        valid[i] = L.oracle_hcpe_to_psv(_p(rec), _p(out[i]))
    return out[valid == 1].copy(), valid
