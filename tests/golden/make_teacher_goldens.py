"""Writes tests/golden/teacher_goldens.json.

Known answers of the teacher-batch producer path, transcribed from the
reference's inline test constants (the reference keeps no golden files), each
with the file:line of the test it comes from.  The positions are given the way
those tests build them (side to move, king squares, pieces by square, hands);
the test encodes them into PackedSfenValue records with the package's
encoder.  The one derived block (the HalfKP packed test position's feature
list) is worked out below from the BonaPiece table and the index formula the
reference documents, independently of the oracle.  Reads nothing at run
time; re-run it only to regenerate the JSON.
"""
import json
from pathlib import Path

PS = "crates/bulletou_lib/src/shogi/packed_sfen.rs"
BP = "crates/bulletou_lib/src/shogi/bona_piece.rs"
HM2 = "crates/bulletou_lib/src/game/inputs/shogi_halfka_hm2.rs"
HKP = "crates/bulletou_lib/src/game/inputs/shogi_halfkp.rs"
OUT = "crates/bulletou_lib/src/game/outputs.rs"

# piece types (types.rs:27-44)
PAWN, LANCE, KNIGHT, SILVER, BISHOP, ROOK, GOLD, KING = 1, 2, 3, 4, 5, 6, 7, 8
PRO_PAWN, PRO_SILVER, DRAGON = 9, 12, 14
F_PAWN, E_PAWN, F_SILVER, F_GOLD, E_GOLD, F_DRAGON, E_DRAGON = 90, 171, 576, 738, 819, 1386, 1467
F_HAND_PAWN, E_HAND_GOLD, E_HAND_ROOK, F_HAND_GOLD, F_HAND_ROOK, E_HAND_PAWN = 1, 74, 88, 69, 85, 20
F_KING, E_KING, FE_END, HM2_PIECES = 1548, 1629, 1548, 1629


def sq(file, rank):
    return file * 9 + rank


def mirror(s):
    return (8 - s // 9) * 9 + s % 9


BITSTREAM = [
    {"source": f"{PS}:482-498 (test_bitstream_read_bits)", "data": [0b10101010, 0b11001100],
     "widths": [4, 4, 4, 4], "values": [0b1010, 0b1010, 0b1100, 0b1100], "cursors": [4, 8, 12, 16]},
    {"source": f"{PS}:500-512 (test_bitstream_cursor)", "data": [0] * 32, "widths": [1, 7, 7],
     "values": [0, 0, 0], "cursors": [1, 8, 15]},
    {"source": f"{PS}:578-594 (test_bitstream_oob_protection): 16 readable bits, then false without panic",
     "data": [0xFF, 0xFF], "widths": [1] * 18, "values": [1] * 16 + [0, 0], "cursors": list(range(1, 17)) + [16, 16]},
    {"source": f"{PS}:657-677 (test_hand_decode_cursor_256_boundary)", "data": [0] * 32, "widths": [1] * 257,
     "values": [0] * 257, "cursors": list(range(1, 257)) + [256]},
]

ACCESSORS = {"source": f"{PS}:514-528 (test_packed_sfen_value_accessors)",
             "bytes": {"32": 0x34, "33": 0x12, "36": 0x56, "37": 0x00, "38": 0xFF},
             "score": 0x1234, "game_ply": 0x56, "game_result": -1}

PIECES = [
    {"source": f"{PS}:531-540 (test_huffman_decode_empty)", "hand": False, "data": [0] * 32,
     "type": 0, "color": 0, "piecebox": False, "cursor": 1},
    {"source": f"{PS}:542-552 (test_huffman_decode_pawn)", "hand": False, "data": [0b00000001, 0, 0, 0],
     "type": PAWN, "color": 0},
    {"source": f"{PS}:554-564 (test_huffman_decode_promoted_pawn)", "hand": False, "data": [0b00001101, 0, 0, 0],
     "type": PRO_PAWN, "color": 1},
    {"source": f"{PS}:566-576 (test_huffman_decode_gold)", "hand": False, "data": [0b00001111, 0, 0, 0],
     "type": GOLD, "color": 0},
    {"source": f"{PS}:596-608 (test_decode_hand_piece_pawn)", "hand": True, "data": [0] * 32,
     "type": PAWN, "color": 0, "piecebox": False},
    {"source": f"{PS}:610-623 (test_decode_hand_piece_gold)", "hand": True, "data": [0b00000111] * 32,
     "type": GOLD, "color": 0, "piecebox": False},
    {"source": f"{PS}:625-639 (test_decode_hand_piece_piecebox_pawn)", "hand": True, "data": [0b00000010] * 32,
     "type": PAWN, "color": 0, "piecebox": True},
    {"source": f"{PS}:641-655 (test_decode_hand_piece_piecebox_rook)", "hand": True, "data": [0b00111111] * 32,
     "type": ROOK, "color": 0, "piecebox": True},
]

BONA = {
    "source": f"{BP}:267-300",
    "board": [{"piece": [PAWN, 0], "sq": sq(6, 6), "perspective": 0, "value": F_PAWN + 60}],
    "hand": [{"perspective": 0, "owner": 0, "type": PAWN, "count": 1, "value": F_HAND_PAWN},
             {"perspective": 0, "owner": 0, "type": PAWN, "count": 2, "value": F_HAND_PAWN + 1},
             {"perspective": 0, "owner": 1, "type": PAWN, "count": 1, "value": E_HAND_PAWN}],
    "pro_pawn_friend_enemy": [F_GOLD, E_GOLD],
}

HM2_INDEX = {
    "source": f"{HM2}:287-357 (dimensions, no-mirror, collapse, mirror, mirror+collapse)",
    "dimensions": 73305, "max_active": 40, "piece_inputs": 1629, "king_buckets": 45,
    "cases": ([{"king": f * 9, "bp": 100, "index": f * 9 * HM2_PIECES + 100} for f in range(5)]
              + [{"king": 0, "bp": E_KING + 40, "index": F_KING + 40},
                 {"king": 0, "bp": F_KING + 40, "index": F_KING + 40},
                 {"king": 5 * 9 + 2, "bp": 10, "index": (3 * 9 + 2) * HM2_PIECES + 10},
                 {"king": 8 * 9 + 5, "bp": 10, "index": (0 * 9 + 5) * HM2_PIECES + 10},
                 {"king": 6 * 9 + 4, "bp": E_KING + 7 * 9 + 3,
                  "index": mirror(6 * 9 + 4) * HM2_PIECES + F_KING + mirror(7 * 9 + 3)}]),
}


def pawns_board():
    board = {}
    for f in range(9):
        board[sq(f, 6)] = [PAWN, 0]
        board[sq(f, 2)] = [PAWN, 1]
    return board


POSITIONS = [
    {"source": f"{HM2}:359-380 (test_map_features_initial_position_count)", "name": "hm2_pawns",
     "stm": 0, "black_king": sq(4, 8), "white_king": sq(4, 0), "board": pawns_board(), "hands": [[0] * 7] * 2,
     "halfka_hm2_count": 20, "halfkp_count": 18},
    {"source": f"{HKP}:579-596 (test_map_features_no_kings)", "name": "kings_only",
     "stm": 0, "black_king": sq(4, 8), "white_king": sq(4, 0), "board": {}, "hands": [[0] * 7] * 2,
     "halfkp_count": 0, "halfka_hm2_count": 2},
    {"source": f"{HKP}:598-614 (test_map_features_sq_nb_guard)", "name": "one_king",
     "stm": 0, "black_king": sq(4, 8), "white_king": 81, "board": {}, "hands": [[0] * 7] * 2,
     "halfkp_count": 0, "halfka_hm2_count": 0},
]

MIRROR = {
    "source": f"{HM2}:407-437 (test_mirror_symmetry): the two positions give the same feature multiset",
    "left": {"stm": 0, "black_king": sq(2, 8), "white_king": sq(2, 0), "board": {sq(1, 6): [PAWN, 0]}},
    "right": {"stm": 0, "black_king": sq(6, 8), "white_king": sq(6, 0), "board": {sq(7, 6): [PAWN, 0]}},
}


def halfkp_packed_test_position(stm):
    """shogi_halfkp.rs:500-529 (packed_halfkp_test_position): kings 5九 / 5一,
    black pawn (0,6), white pawn (8,2), black pro-silver (2,4), white dragon
    (6,4); hands: black 2 pawns, white rook and gold; piece-box padding.
    Features in square order, then hands (Black owner first, HAND_PIECE_TYPES
    order), index = own-king-square * 1548 + BonaPiece, with the board square
    and king square rotated (80 - sq) for the White perspective."""
    bk, wk = sq(4, 8), sq(4, 0)
    pieces = sorted({sq(0, 6): (PAWN, 0), sq(8, 2): (PAWN, 1), sq(2, 4): (PRO_SILVER, 0),
                     sq(6, 4): (DRAGON, 1)}.items())
    base = {PAWN: (E_PAWN, F_PAWN), PRO_SILVER: (E_GOLD, F_GOLD), DRAGON: (E_DRAGON, F_DRAGON)}
    nstm = 1 - stm

    def persp(s, p):
        return s if p == 0 else 80 - s

    ks, kn = persp(bk if stm == 0 else wk, stm), persp(wk if stm == 0 else bk, nstm)
    feats = []
    for s, (pt, color) in pieces:
        a = ks * FE_END + base[pt][color == stm] + persp(s, stm)
        b = kn * FE_END + base[pt][color == nstm] + persp(s, nstm)
        feats.append([a, b])
    hand_base = {PAWN: (E_HAND_PAWN, F_HAND_PAWN), ROOK: (E_HAND_ROOK, F_HAND_ROOK),
                 GOLD: (E_HAND_GOLD, F_HAND_GOLD)}
    # Black owner: pawn x2; White owner: gold before rook in HAND_PIECE_TYPES order
    for owner, pt, count in ((0, PAWN, 2), (1, GOLD, 1), (1, ROOK, 1)):
        for i in range(1, count + 1):
            feats.append([ks * FE_END + hand_base[pt][owner == stm] + i - 1,
                          kn * FE_END + hand_base[pt][owner == nstm] + i - 1])
    return {"source": f"{HKP}:500-552 (packed_halfkp_test_position / test_direct_packed_mapper_matches_board_mapper)",
            "name": f"halfkp_packed_stm{stm}", "stm": stm, "black_king": bk, "white_king": wk,
            "board": {s: [pt, c] for s, (pt, c) in pieces}, "hands": [[2, 0, 0, 0, 0, 0, 0], [0, 0, 0, 0, 1, 0, 1]],
            "halfkp_features": feats}


def psv_with_kings(stm, bk, wk):
    return {"stm": stm, "black_king": bk, "white_king": wk}


BUCKETS = {
    "source": f"{OUT}:2236-2244 (psv_with_kings: header bits only, the rest zero), 2517-2530, 2685-2768",
    "note": "records are the 15 header bits followed by zeros, exactly as psv_with_kings writes them",
    "cases": [
        {"pos": psv_with_kings(0, sq(4, 2), sq(4, 7)), "king": "kingrank81", "bucket": 2 * 9 + 1},
        {"pos": psv_with_kings(0, sq(4, 2), sq(4, 7)), "king": "kingrank9", "bucket": 0},
        {"pos": psv_with_kings(1, sq(4, 2), sq(4, 7)), "king": "kingrank81", "bucket": 1 * 9 + 2},
        {"pos": psv_with_kings(1, sq(4, 2), sq(4, 7)), "king": "kingrank9", "bucket": 0},
        {"pos": psv_with_kings(0, sq(4, 8), sq(4, 0)), "king": "kingrank81", "bucket": 80},
        {"pos": psv_with_kings(0, sq(4, 8), sq(4, 0)), "king": "kingrank9", "bucket": 8},
        {"pos": psv_with_kings(0, sq(4, 8), sq(4, 0)), "king": "k9k9z", "bucket": 7 * 9 + 7},
        {"pos": psv_with_kings(1, sq(4, 8), sq(4, 0)), "king": "k9k9z", "bucket": 7 * 9 + 7},
        {"pos": psv_with_kings(0, sq(4, 8), sq(4, 0)), "king": "k13k13z", "bucket": 11 * 13 + 11},
        {"pos": psv_with_kings(1, sq(4, 8), sq(4, 0)), "king": "k13k13z", "bucket": 11 * 13 + 11},
        {"pos": psv_with_kings(0, sq(4, 8), sq(4, 0)), "king": "k29k29", "bucket": 24 * 29 + 24},
        {"pos": psv_with_kings(1, sq(4, 8), sq(4, 0)), "king": "k29k29", "bucket": 24 * 29 + 24},
        {"pos": psv_with_kings(0, sq(0, 6), sq(8, 2)), "king": "k29k29", "bucket": 2 * 29 + 2},
        {"pos": psv_with_kings(0, sq(4, 8), sq(4, 0)), "king": "k21k21", "bucket": 16 * 21 + 16},
        {"pos": psv_with_kings(1, sq(4, 8), sq(4, 0)), "king": "k21k21", "bucket": 16 * 21 + 16},
        {"pos": psv_with_kings(0, sq(0, 7), sq(8, 1)), "king": "k21k21", "bucket": 3 * 21 + 3},
    ],
    "king_single": {
        "k9k9z": [[sq(0, 0), 0], [sq(8, 2), 0], [sq(0, 3), 1], [sq(8, 5), 1], [sq(0, 6), 2], [sq(0, 7), 3],
                  [sq(8, 7), 5], [sq(0, 8), 6], [sq(8, 8), 8]],
        "k13k13z": [[sq(0, 0), 0], [sq(8, 6), 6], [sq(0, 7), 7], [sq(8, 7), 9], [sq(0, 8), 10], [sq(8, 8), 12]],
        "k29k29": [[sq(0, 0), 0], [sq(8, 2), 0], [sq(0, 3), 1], [sq(8, 5), 1], [sq(0, 6), 2], [sq(8, 6), 10],
                   [sq(0, 7), 11], [sq(8, 8), 28]],
        "k21k21": [[sq(0, 0), 0], [sq(8, 2), 0], [sq(0, 3), 1], [sq(8, 5), 1], [sq(0, 6), 2], [sq(0, 7), 3],
                   [sq(8, 7), 11], [sq(0, 8), 12], [sq(8, 8), 20]],
    },
}

FULL = [18, 4, 4, 4, 4, 2, 2]


def hand(**kw):
    order = ["pawn", "lance", "knight", "silver", "gold", "bishop", "rook"]
    return [kw.get(k, 0) for k in order]


HAND_SINGLE = {
    "source": f"{OUT}:2246-2438 (hand4/16/64/64z/256/1024 single-bucket formulas)",
    "cases": [
        ["hand4", hand(), 0], ["hand16", hand(), 0], ["hand4", hand(pawn=1), 0], ["hand16", hand(pawn=1), 1],
        ["hand4", hand(bishop=1), 1], ["hand16", hand(bishop=1), 2], ["hand16", hand(pawn=1, bishop=1), 3],
        ["hand64", hand(), 0], ["hand64", hand(pawn=1), 1], ["hand64", hand(pawn=5), 1],
        ["hand64", hand(lance=1, knight=1), 1], ["hand64", hand(silver=1, gold=1), 2], ["hand64", hand(bishop=1), 4],
        ["hand64", hand(bishop=1, rook=1), 6], ["hand64", FULL, 7],
        ["hand64z", hand(), 0], ["hand64z", hand(pawn=1), 1], ["hand64z", hand(pawn=5), 2],
        ["hand64z", hand(lance=1, knight=1), 1], ["hand64z", hand(silver=1, gold=1), 2],
        ["hand64z", hand(bishop=1), 2], ["hand64z", hand(bishop=1, rook=1), 3], ["hand64z", FULL, 7],
        ["hand256", hand(), 0], ["hand256", hand(pawn=1), 1], ["hand256", hand(lance=1), 1],
        ["hand256", hand(knight=1), 1], ["hand256", hand(silver=1), 2], ["hand256", hand(gold=1), 2],
        ["hand256", hand(bishop=1), 4], ["hand256", hand(rook=1), 8], ["hand256", FULL, 15],
        ["hand1024", hand(), 0], ["hand1024", hand(pawn=1), 1], ["hand1024", hand(lance=1), 2],
        ["hand1024", hand(knight=1), 2], ["hand1024", hand(silver=1), 4], ["hand1024", hand(gold=1), 4],
        ["hand1024", hand(bishop=1), 8], ["hand1024", hand(rook=1), 16], ["hand1024", FULL, 31],
    ],
}

STACK_COUNTS = {
    "source": f"{OUT}:826-905 (bucket_count of the hand and king axes)",
    "hand": {"none": 1, "hand4": 4, "hand16": 16, "hand64": 64, "hand64z": 64, "hand256": 256, "hand1024": 1024},
    "king": {"none": 1, "kingrank9": 9, "kingrank81": 81, "k9k9z": 81, "k13k13z": 169, "k21k21": 441,
             "k21k21z": 441, "k29k29": 841},
}


HCPE_SRC = "crates/bulletou_lib/src/value/loader"


def hirate():
    """MiniPosition::hirate (shogipack.rs:292-336) in file * 9 + rank squares."""
    back = [LANCE, KNIGHT, SILVER, GOLD, KING, GOLD, SILVER, KNIGHT, LANCE]
    board = {}
    for i, pt in enumerate(back):
        f = 8 - i
        if pt != KING:
            board[sq(f, 0)] = [pt, 1]
            board[sq(f, 8)] = [pt, 0]
    board[sq(7, 1)] = [BISHOP, 1]
    board[sq(1, 1)] = [ROOK, 1]
    board[sq(7, 7)] = [ROOK, 0]
    board[sq(1, 7)] = [BISHOP, 0]
    for f in range(9):
        board[sq(f, 2)] = [PAWN, 1]
        board[sq(f, 6)] = [PAWN, 0]
    return {"black_king": sq(4, 8), "white_king": sq(4, 0), "board": board}


HCPE = {
    "record_bytes": {"source": f"{HCPE_SRC}/hcpe.rs:571-574 (hcpe_record_size_is_38)", "value": 38},
    "convert_game_result": {
        "source": f"{HCPE_SRC}/shogipack.rs:1356-1363 (test_convert_game_result)",
        "cases": [[0, 0, 0], [1, 0, 1], [1, 1, -1], [2, 1, 1], [2, 0, -1]]},
    "hirate_results": {
        "source": f"{HCPE_SRC}/hcpe.rs:581-622 (decode_converts_game_result_to_stm_perspective): the hirate "
                  "position packed in the PackedSfen encoding (pack_to_hcp is pack_to_psfen there), read as HCP",
        "position": hirate(),
        "stm0": [[1, 1], [2, -1], [0, 0]], "stm1": [[1, -1], [2, 1]]},
    "all_zero": {"source": f"{HCPE_SRC}/hcpe.rs:625-633 (decode_invalid_record_returns_none): must not fail"},
}


def main():
    data = {"bitstream": BITSTREAM, "accessors": ACCESSORS, "pieces": PIECES, "bona": BONA,
            "hm2_index": HM2_INDEX, "positions": POSITIONS, "mirror": MIRROR,
            "halfkp_packed": [halfkp_packed_test_position(0), halfkp_packed_test_position(1)],
            "buckets": BUCKETS, "hand_single": HAND_SINGLE, "stack_counts": STACK_COUNTS, "hcpe": HCPE}
    path = Path(__file__).with_name("teacher_goldens.json")
    path.write_text(json.dumps(data, indent=1) + "\n")
    print(f"wrote {path}")


if __name__ == "__main__":
    main()
