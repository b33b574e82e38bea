"""CPU: the teacher-batch producer oracle (oracle/teacher_oracle.c) pinned to
the reference's own known answers (tests/golden/teacher_goldens.json, each
case citing its reference test), the package's PackedSfenValue encoder, and
the producer's host logic (config blends, record views, win-rate table)."""
import json
from pathlib import Path

import numpy as np
import pytest

from bulletou_b200 import CudaCppError
from bulletou_b200 import synthetic as syn
from bulletou_b200 import teacher as bt
from oracle import teacher as ot

G = json.loads((Path(__file__).parent / "golden" / "teacher_goldens.json").read_text())


def _board(d: dict) -> np.ndarray:
    b = np.zeros(81, np.int64)
    for s, (pt, color) in d.items():
        b[int(s)] = pt | (color << 4)
    return b


def _encode(pos: dict, score=0, result=0):
    hands = pos.get("hands", [[0] * 7, [0] * 7])
    return syn.psv_encode(pos["stm"], pos["black_king"], pos["white_king"], _board(pos.get("board", {}))[None],
                          np.asarray(hands)[None], score, result)


def _header_only(pos: dict) -> np.ndarray:
    """psv_with_kings (game/outputs.rs:2236-2244): the 15 header bits, zeros after."""
    bits = [pos["stm"]] + [(pos["black_king"] >> i) & 1 for i in range(7)] + [(pos["white_king"] >> i) & 1
                                                                            for i in range(7)]
    rec = np.zeros(40, np.uint8)
    for i, b in enumerate(bits):
        rec[i // 8] |= b << (i % 8)
    return rec


# ------------------------------------------------------------------ reference known answers
@pytest.mark.parametrize("case", G["bitstream"], ids=lambda c: c["source"].split("(")[1][:-1][:40])
def test_bitstream_known_answers(case):
    values, cursors = ot.read_bits(case["data"], case["widths"])
    assert values == case["values"]
    assert cursors == case["cursors"]


def test_record_accessors_known_answer():
    a = G["accessors"]
    rec = np.zeros(40, np.uint8)
    for k, v in a["bytes"].items():
        rec[int(k)] = v
    d = ot.decode(rec)
    assert (d["score"], d["game_ply"], d["game_result"]) == (a["score"], a["game_ply"], a["game_result"])


@pytest.mark.parametrize("case", G["pieces"], ids=lambda c: c["source"].split("(")[1][:-1])
def test_piece_decode_known_answers(case):
    got = ot.decode_piece(case["data"], case["hand"])
    assert (got["type"], got["color"]) == (case["type"], case["color"])
    if "piecebox" in case:
        assert got["piecebox"] == case["piecebox"]
    if "cursor" in case:
        assert got["cursor"] == case["cursor"]


def test_bona_piece_known_answers():
    b = G["bona"]
    for c in b["board"]:
        assert ot.bona_board(c["piece"][0], c["piece"][1], c["sq"], c["perspective"]) == c["value"]
    for c in b["hand"]:
        assert ot.bona_hand(c["perspective"], c["owner"], c["type"], c["count"]) == c["value"]
    f, e = b["pro_pawn_friend_enemy"]
    assert ot.bona_board(9, 0, 0, 0) == f and ot.bona_board(9, 1, 80, 0) == e + 80


def test_halfka_hm2_index_known_answers():
    h = G["hm2_index"]
    assert h["dimensions"] == h["king_buckets"] * h["piece_inputs"] == bt.FEATURE_INPUTS["halfka_hm2"]
    assert h["max_active"] == bt.FEATURE_MAX_ACTIVE["halfka_hm2"]
    for c in h["cases"]:
        assert ot.hm2_index(c["king"], c["bp"]) == c["index"], c


@pytest.mark.parametrize("case", G["positions"], ids=lambda c: c["name"])
def test_feature_counts_known_answers(case):
    rec = _encode(case)
    hm2 = ot.prepare(rec, ot.config("halfka_hm2"))
    kp = ot.prepare(rec, ot.config("halfkp"))
    assert hm2["counts"][0] == case["halfka_hm2_count"]
    assert kp["counts"][0] == case["halfkp_count"]
    for out, n in ((hm2, bt.FEATURE_INPUTS["halfka_hm2"]), (kp, bt.FEATURE_INPUTS["halfkp"])):
        c = out["counts"][0]
        assert ((out["stm"][0, :c] >= 0) & (out["stm"][0, :c] < n)).all()
        assert (out["stm"][0, c:] == -1).all() and (out["nstm"][0, c:] == -1).all()


def test_mirror_symmetry_known_answer():
    m = G["mirror"]
    sets = []
    for side in ("left", "right"):
        out = ot.prepare(_encode(m[side]), ot.config("halfka_hm2"))
        c = out["counts"][0]
        sets.append(sorted(zip(out["stm"][0, :c].tolist(), out["nstm"][0, :c].tolist())))
    assert sets[0] == sets[1] and len(sets[0]) == 3


@pytest.mark.parametrize("case", G["halfkp_packed"], ids=lambda c: c["name"])
def test_halfkp_packed_position_features(case):
    out = ot.prepare(_encode(case), ot.config("halfkp"))
    want = np.asarray(case["halfkp_features"])
    c = out["counts"][0]
    assert c == len(want)
    np.testing.assert_array_equal(out["stm"][0, :c], want[:, 0])
    np.testing.assert_array_equal(out["nstm"][0, :c], want[:, 1])


@pytest.mark.parametrize("case", G["buckets"]["cases"], ids=lambda c: f"{c['king']}-{c['bucket']}")
def test_layerstack_bucket_known_answers(case):
    out = ot.prepare(_header_only(case["pos"]), ot.config("halfka_hm2", king=case["king"]))
    assert out["buckets"][0] == case["bucket"]


def test_king_and_hand_single_bucket_known_answers():
    for kind, pairs in G["buckets"]["king_single"].items():
        for sq, want in pairs:
            assert ot.king_single_bucket(kind, sq) == want, (kind, sq)
    for kind, hand, want in G["hand_single"]["cases"]:
        assert ot.hand_single_bucket(kind, hand) == want, (kind, hand)


def test_stack_counts_match_reference_and_product():
    sc = G["stack_counts"]
    for h, hc in sc["hand"].items():
        for k, kc in sc["king"].items():
            assert ot.bucket_count(h, k) == hc * kc
            assert bt.LayerStackBucketKind(h, k).num_stacks == hc * kc


def test_header_only_record_decodes_hand_pawns():
    """psv_with_kings leaves zeros after the header: the board decodes empty and
    the tail decodes as 54 black hand pawns (3 bits each), which the hand
    buckets see (packed_sfen.rs:252-270)."""
    d = ot.decode(_header_only({"stm": 0, "black_king": 44, "white_king": 36}))
    assert d["cursor_after_board"] == 15 + 79
    assert d["hands"][0].tolist() == [54, 0, 0, 0, 0, 0, 0] and d["hands"][1].sum() == 0


# ------------------------------------------------------------------ independent restatement of the order
PIECE_BASE = {1: (171, 90), 2: (333, 252), 3: (495, 414), 4: (657, 576), 5: (981, 900), 6: (1305, 1224),
              7: (819, 738), 9: (819, 738), 10: (819, 738), 11: (819, 738), 12: (819, 738), 13: (1143, 1062),
              14: (1467, 1386)}
HAND_BASE = ((20, 1), (44, 39), (54, 49), (64, 59), (74, 69), (82, 79), (88, 85))
BOARD_ORDER = (1, 2, 3, 4, 7, 5, 6, 9, 10, 11, 12, 13, 14)


def _hm2_python(stm, bk, wk, board, hands):
    nstm = 1 - stm
    own = {0: bk, 1: wk}

    def ksq(c):
        return own[c] if c == 0 else 80 - own[c]

    def idx(k, bp):
        if k // 9 >= 5:
            k = (8 - k // 9) * 9 + k % 9
            if bp >= 90:
                off = bp - 90
                s = off % 81
                bp = 90 + (off // 81) * 81 + (8 - s // 9) * 9 + s % 9
        if bp >= 1629:
            bp -= 81
        return k * 1629 + bp

    def persp(s, c):
        return s if c == 0 else 80 - s

    ks, kn = ksq(stm), ksq(nstm)
    out = []
    for pt in BOARD_ORDER:
        for color in (0, 1):
            for s in range(81):
                if s in (bk, wk) or board[s] != (pt | (color << 4)):
                    continue
                out.append((idx(ks, PIECE_BASE[pt][color == stm] + persp(s, stm)),
                            idx(kn, PIECE_BASE[pt][color == nstm] + persp(s, nstm))))
    out.append((idx(ks, 1548 + ks), idx(kn, 1548 + kn)))
    out.append((idx(ks, 1629 + persp(own[nstm], stm)), idx(kn, 1629 + persp(own[stm], nstm))))
    for owner in (0, 1):
        for h in range(7):
            for i in range(hands[owner][h]):
                out.append((idx(ks, HAND_BASE[h][owner == stm] + i), idx(kn, HAND_BASE[h][owner == nstm] + i)))
    return out


def test_oracle_halfka_hm2_order_matches_python_restatement():
    p = syn.psv_positions(syn.rng_for(21), 60, hand_fraction=0.3, promote_fraction=0.3)
    recs = syn.psv_encode(p["stm"], p["black_king"], p["white_king"], p["board"], p["hands"])
    out = ot.prepare(recs, ot.config("halfka_hm2"))
    for i in range(60):
        want = _hm2_python(int(p["stm"][i]), int(p["black_king"][i]), int(p["white_king"][i]), p["board"][i],
                           p["hands"][i])
        assert out["counts"][i] == len(want) == 40
        got = list(zip(out["stm"][i].tolist(), out["nstm"][i].tolist()))
        assert got == want


# ------------------------------------------------------------------ encoder
def test_encoder_round_trips_through_the_oracle_decode():
    rng = syn.rng_for(5)
    p = syn.psv_positions(rng, 300, hand_fraction=0.25, promote_fraction=0.2)
    recs = syn.psv_encode(p["stm"], p["black_king"], p["white_king"], p["board"], p["hands"], 123, -1, 77, 4242)
    for i in range(300):
        d = ot.decode(recs[i])
        board = p["board"][i].copy()
        board[p["black_king"][i]] = 8
        board[p["white_king"][i]] = 8 | 16
        np.testing.assert_array_equal(d["board"], board)
        np.testing.assert_array_equal(d["hands"], p["hands"][i])
        assert (d["stm"], d["black_king"], d["white_king"]) == (p["stm"][i], p["black_king"][i], p["white_king"][i])
        assert (d["score"], d["game_result"], d["game_ply"]) == (123, -1, 77)
    assert recs["move16"][0] == 4242


def test_encoder_pads_short_positions_with_piece_box_pieces():
    # every tail length the padding handles: 0, 2, 3, 4, 5 (mod 3 mixes)
    for extra_pawns in range(0, 6):
        board = np.zeros(81, np.int64)
        for f in range(extra_pawns):
            board[f * 9 + 6] = 1
        rec = syn.psv_encode(0, 44, 36, board[None], np.zeros((1, 2, 7)))
        d = ot.decode(rec[0])
        assert d["hands"].sum() == 0 and (d["board"] == 1).sum() == extra_pawns


def test_encoder_rejects_unpaddable_one_bit_tail():
    # 15 header + 79 empty squares + 161 bits of hand (2 pawns x 3 + 31 silvers x 5) = 255 bits
    hands = np.zeros((1, 2, 7), np.int64)
    hands[0, 0, 0] = 2
    hands[0, 0, 3] = 31
    with pytest.raises(ValueError, match="1-bit tail"):
        syn.psv_encode(0, 44, 36, np.zeros((1, 81)), hands)


# ------------------------------------------------------------------ product host logic
@pytest.mark.parametrize("fs", ["halfka_hm2", "halfkp"])
@pytest.mark.parametrize("lam", [0.0, 0.25, 0.7, 1.0])
def test_product_config_blends_match_the_oracle(fs, lam):
    cfg = bt.TeacherBatchConfig(feature_set=fs, lambda_=lam, scale=510.0, score_drop_abs=3000)
    s = cfg.as_struct()
    o = ot.config(fs, lambda_=lam, scale=510.0, score_drop_abs=3000)
    for f in ("feature_set", "max_active", "result_blend", "score_blend", "rscale", "score_drop_abs"):
        assert getattr(s, f) == getattr(o, f), f


def test_product_config_validation():
    with pytest.raises(CudaCppError, match="lambda"):
        bt.TeacherBatchConfig(lambda_=1.5).validate()
    with pytest.raises(CudaCppError, match="hand bucket"):
        bt.TeacherBatchConfig(layerstack_bucket=bt.LayerStackBucketKind("hand3")).validate()
    with pytest.raises(CudaCppError, match="max_active"):
        bt.TeacherBatchConfig(max_active=64).validate()
    with pytest.raises(CudaCppError, match="u16"):
        bt.TeacherBatchConfig(score_drop_abs=70000).validate()
    with pytest.raises(CudaCppError, match="win-rate"):
        bt.TeacherBatchConfig(win_rate_model=True, wrm_target=bt.WinRateModelTargetParams(scaling=0.0)).validate()


def test_records_as_words_views():
    recs = syn.psv_records(3, 5)
    w = bt.records_as_words(recs)
    assert w.dtype == np.int32 and w.size == 50
    np.testing.assert_array_equal(bt.records_as_words(recs.view(np.uint8).reshape(5, 40)), w)
    np.testing.assert_array_equal(bt.records_as_words(recs.tobytes()), w)
    with pytest.raises(CudaCppError, match="40-byte"):
        bt.records_as_words(np.zeros(41, np.uint8))


@pytest.mark.parametrize("params", [(270.0, 380.0, 0.0), (150.0, 250.0, 0.05)])
def test_product_wrm_table_matches_the_oracle_table(params):
    """The product builds the table with exp in double rounded once; the oracle
    calls the C library's expf like the reference (value/loader.rs:667-687).
    A 1-ulp exp difference near sigmoid 1 shows up as 2 ulp of a small
    probability after 1 + s(p) - s(pm); the default parameters agree exactly."""
    mine = bt.win_rate_model_score_table(bt.WinRateModelTargetParams(*params))
    ref = ot.wrm_table(*params)
    ulp = np.abs(mine.view(np.int32).astype(np.int64) - ref.view(np.int32).astype(np.int64))
    assert ulp.max() <= 2
    assert (ulp == 0).mean() > 0.999
    if params == (270.0, 380.0, 0.0):
        assert ulp.max() == 0


def test_fuzz_records_never_index_out_of_range():
    """Any 40-byte pattern decodes (packed_sfen.rs:441-448): features stay in
    range and the overflowing records are exactly the ones above max_active."""
    rng = np.random.default_rng(7)
    recs = rng.integers(0, 256, (3000, 40), dtype=np.uint8)
    for fs, n in (("halfka_hm2", 73305), ("halfkp", 125388)):
        out = ot.prepare(recs, ot.config(fs, hand="hand64z" if fs == "halfka_hm2" else "none", king="k29k29"))
        A = out["stm"].shape[1]
        valid = out["stm"] >= 0
        assert (out["stm"][valid] < n).all() and (out["nstm"][out["nstm"] >= 0] < n).all()
        np.testing.assert_array_equal(valid.sum(axis=1), np.minimum(out["counts"], A))
        assert (out["counts"] > A).any() and ((out["counts"] > 0) & (out["counts"] <= A)).any()


# ------------------------------------------------------------------ HCPE records
def _hirate_psv_bytes(stm):
    h = G["hcpe"]["hirate_results"]["position"]
    return _encode({"stm": stm, "black_king": h["black_king"], "white_king": h["white_king"], "board": h["board"]})


def test_hcpe_known_answers():
    """decode_converts_game_result_to_stm_perspective (hcpe.rs:581-622): the
    PackedSfen-encoded hirate read as HCP decodes, and the absolute game result
    turns into the side to move's; convert_game_result (shogipack.rs:1356-1363)."""
    g = G["hcpe"]
    assert g["record_bytes"]["value"] == syn.HCPE_DTYPE.itemsize == 38
    for stm, cases in ((0, g["hirate_results"]["stm0"]), (1, g["hirate_results"]["stm1"])):
        sfen = _hirate_psv_bytes(stm).view(np.uint8)[:32]
        for abs_result, want in cases:
            rec = np.zeros(38, np.uint8)
            rec[:32] = sfen
            rec[36] = abs_result
            psv, valid = ot.hcpe_to_psv(rec)
            assert valid[0] == 1
            assert np.int8(psv[0, 38]) == want
            assert psv[0, 36] == 0 and psv[0, 37] == 0                  # game_ply 0
    for abs_result, stm, want in g["convert_game_result"]["cases"]:
        rec = np.zeros(38, np.uint8)
        rec[:32] = _hirate_psv_bytes(stm).view(np.uint8)[:32]
        rec[36] = abs_result
        psv, _ = ot.hcpe_to_psv(rec)
        assert np.int8(psv[0, 38]) == want
    ot.hcpe_to_psv(np.zeros(38, np.uint8))                            # hcpe.rs:625-633: no failure


def test_hcpe_full_set_records_repack_to_the_psv_encoding():
    """A full-set position encoded as HCP repacks to exactly the PackedSfenValue
    bytes of the same position (pack_to_psfen order: board by square, hands by
    colour and type; no padding needed), with eval, bestMove16, game_ply 0 and
    the side to move's result."""
    p = syn.psv_positions(syn.rng_for(44), 400, hand_fraction=0.3, promote_fraction=0.3)
    res = syn.rng_for(45).integers(0, 3, 400)
    h = syn.hcpe_encode(p["stm"], p["black_king"], p["white_king"], p["board"], p["hands"], -321, res, 777)
    psv, valid = ot.hcpe_to_psv(h)
    assert valid.all()
    stm_result = np.where(res == 0, 0, np.where((res == 1) == (p["stm"] == 0), 1, -1))
    want = syn.psv_encode(p["stm"], p["black_king"], p["white_king"], p["board"], p["hands"], -321, stm_result, 0,
                          777)
    np.testing.assert_array_equal(psv, want.view(np.uint8).reshape(-1, 40))


def test_hcpe_invalid_records_are_dropped():
    rng = np.random.default_rng(3)
    recs = rng.integers(0, 256, (3000, 38), dtype=np.uint8)
    psv, valid = ot.hcpe_to_psv(recs)
    kings_ok = []
    for r in recs:
        bits = int.from_bytes(r[:2].tobytes(), "little")
        kings_ok.append(((bits >> 1) & 127) < 81 and ((bits >> 8) & 127) < 81)
    kings_ok = np.array(kings_ok)
    assert not valid[~kings_ok].any()                                  # a king square >= 81: skipped
    assert 0 < valid.sum() < kings_ok.sum()                           # some fail on unknown hand codes
    assert psv.shape == (valid.sum(), 40)
