"""Seeded synthetic inputs standing in for the reference's private teacher data.

The reference trains on PSV/HCPE teacher files (docs/spec/10-cuda-oxide-tickets.md:503-521)
that are not available; these generators reproduce their shapes, index ranges
and value distributions:

* HalfKP (125388 = 81 kings x 1548 piece-squares): per perspective a king
  k ~ U{0..80} and 38 distinct piece ids p ~ U[0,1548); feature = k*1548 + p
  (crates/bulletou_lib/src/game/inputs/shogi_halfkp.rs:26-40);
* KPPT: 38 distinct BonaPieces per view; KPP = all 703 pairs a<b,
  k*1548^2 + a*1548 + b (shogi_kpp.rs:14); KKP = k*81*1548 + k'*1548 + p;
  KK = k*81 + k';
* HalfKA_hm2 (73305 = 45 mirrored king buckets x 1629): per perspective a
  king bucket k ~ U{0..44} and 40 distinct pieces p ~ U[0,1629); feature =
  k*1629 + p (shogi_halfka_hm2.rs:106-260); LayerStack bucket ~ U{0..8}
  (k3k3) or Zipf(1.1) over 81 buckets through a seeded permutation (k9k9);
* weights ~ N(0, 0.01); targets t = 0.5*r + 0.5*sigmoid(score/600) with
  score = round(N(0,600)) clipped to +-3000 and r in {0, 1/2, 1}
  (teacher_batch.rs:1709-1746 blend with lambda = 0.5); entry weight 1.

numpy's PCG64 generator, one stream per (seed, rank).
"""
from __future__ import annotations

import numpy as np

HALFKP_KINGS = 81
HALFKP_PIECES = 1548
HALFKP_INPUTS = HALFKP_KINGS * HALFKP_PIECES  # 125388
HALFKP_ACTIVE = 38
KPP_INPUTS = HALFKP_KINGS * HALFKP_PIECES * HALFKP_PIECES  # 194100624
KKP_INPUTS = HALFKP_KINGS * HALFKP_KINGS * HALFKP_PIECES  # 10156428
KK_INPUTS = HALFKP_KINGS * HALFKP_KINGS  # 6561
KPP_PAIRS = HALFKP_ACTIVE * (HALFKP_ACTIVE - 1) // 2  # 703


def rng_for(seed: int, rank: int = 0) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64([seed, rank]))


def distinct_pieces(rng: np.random.Generator, rows: int, k: int = HALFKP_ACTIVE, n: int = HALFKP_PIECES,
                    sort: bool = False) -> np.ndarray:
    """rows x k distinct values in [0, n)."""
    out = np.empty((rows, k), np.int32)
    chunk = 2048
    for r0 in range(0, rows, chunk):
        r1 = min(rows, r0 + chunk)
        keys = rng.random((r1 - r0, n), dtype=np.float32)
        pick = np.argpartition(keys, k, axis=1)[:, :k]
        out[r0:r1] = pick
    if sort:
        out.sort(axis=1)
    return out


def halfkp_indices(rng: np.random.Generator, batch: int) -> tuple[np.ndarray, np.ndarray]:
    """(stm, nstm) int32 [batch*38], perspectives drawn independently."""
    views = []
    for _ in range(2):
        kings = rng.integers(0, HALFKP_KINGS, size=(batch, 1), dtype=np.int32)
        pieces = distinct_pieces(rng, batch)
        views.append((kings * HALFKP_PIECES + pieces).astype(np.int32).reshape(-1))
    return views[0], views[1]


def targets(rng: np.random.Generator, batch: int, scale: float = 600.0, lam: float = 0.5) -> tuple[np.ndarray, np.ndarray]:
    """(targets, entry_weights) float32 [batch]."""
    score = np.clip(np.rint(rng.normal(0.0, 600.0, size=batch)), -3000, 3000).astype(np.float32)
    result = rng.integers(-1, 2, size=batch).astype(np.float32)
    r = (result + 1.0) * 0.5
    t = (1.0 - lam) * r + lam * (1.0 / (1.0 + np.exp(-score / scale)))
    return t.astype(np.float32), np.ones(batch, np.float32)


def halfkp_weights(rng: np.random.Generator, input_size: int = HALFKP_INPUTS, l1: int = 256, l2: int = 32,
                   l3: int = 32, std: float = 0.01) -> dict:
    shapes = {"l0w": input_size * l1, "l0b": l1, "l1w": 2 * l1 * l2, "l1b": l2, "l2w": l2 * l3, "l2b": l3,
              "outw": l3, "outb": 1}
    return {k: rng.normal(0.0, std, size=n).astype(np.float32) for k, n in shapes.items()}


def halfkp_batch(seed: int, batch: int, rank: int = 0) -> dict:
    rng = rng_for(seed, rank)
    stm, nstm = halfkp_indices(rng, batch)
    t, w = targets(rng, batch)
    return {"stm": stm, "nstm": nstm, "targets": t, "entry_weights": w, "batch": batch, "max_active": HALFKP_ACTIVE}


def kppt_indices(rng: np.random.Generator, batch: int, component: str) -> tuple[np.ndarray, np.ndarray, int, int]:
    """(stm, nstm, input_size, max_active) for component 'kk' | 'kkp' | 'kpp'."""
    views = []
    if component == "kpp":
        iu, ju = np.triu_indices(HALFKP_ACTIVE, k=1)
        for _ in range(2):
            k = rng.integers(0, HALFKP_KINGS, size=(batch, 1)).astype(np.int64)
            p = distinct_pieces(rng, batch, sort=True).astype(np.int64)
            idx = k * HALFKP_PIECES * HALFKP_PIECES + p[:, iu] * HALFKP_PIECES + p[:, ju]
            views.append(idx.astype(np.int32).reshape(-1))
        return views[0], views[1], KPP_INPUTS, KPP_PAIRS
    if component == "kkp":
        for _ in range(2):
            k0 = rng.integers(0, HALFKP_KINGS, size=(batch, 1)).astype(np.int64)
            k1 = rng.integers(0, HALFKP_KINGS, size=(batch, 1)).astype(np.int64)
            p = distinct_pieces(rng, batch).astype(np.int64)
            views.append((k0 * HALFKP_KINGS * HALFKP_PIECES + k1 * HALFKP_PIECES + p).astype(np.int32).reshape(-1))
        return views[0], views[1], KKP_INPUTS, HALFKP_ACTIVE
    if component == "kk":
        for _ in range(2):
            k0 = rng.integers(0, HALFKP_KINGS, size=batch)
            k1 = rng.integers(0, HALFKP_KINGS, size=batch)
            views.append((k0 * HALFKP_KINGS + k1).astype(np.int32))
        return views[0], views[1], KK_INPUTS, 1
    raise ValueError(f"unknown KPPT component {component!r}")


HM2_KINGS = 45
HM2_PIECES = 1629
HM2_INPUTS = HM2_KINGS * HM2_PIECES  # 73305
HM2_ACTIVE = 40


def hm2_indices(rng: np.random.Generator, batch: int) -> tuple[np.ndarray, np.ndarray]:
    """(stm, nstm) int32 [batch*40] HalfKA_hm2 features, perspectives independent."""
    views = []
    for _ in range(2):
        kings = rng.integers(0, HM2_KINGS, size=(batch, 1), dtype=np.int32)
        pieces = distinct_pieces(rng, batch, HM2_ACTIVE, HM2_PIECES)
        views.append((kings * HM2_PIECES + pieces).astype(np.int32).reshape(-1))
    return views[0], views[1]


def layerstack_buckets(rng: np.random.Generator, batch: int, stacks: int = 9, zipf: float = 0.0) -> np.ndarray:
    """Uniform buckets, or Zipf(s) ranks mapped through a seeded permutation."""
    if zipf <= 0.0:
        return rng.integers(0, stacks, size=batch).astype(np.int32)
    ranks = np.arange(1, stacks + 1, dtype=np.float64)
    p = ranks ** -zipf
    p /= p.sum()
    perm = rng.permutation(stacks)
    return perm[rng.choice(stacks, size=batch, p=p)].astype(np.int32)


def sfnn_batch(seed: int, batch: int, rank: int = 0, stacks: int = 9, zipf: float = 0.0) -> dict:
    rng = rng_for(seed, rank)
    stm, nstm = hm2_indices(rng, batch)
    buckets = layerstack_buckets(rng, batch, stacks, zipf)
    t, w = targets(rng, batch)
    return {"stm": stm, "nstm": nstm, "buckets": buckets, "targets": t, "entry_weights": w, "batch": batch,
            "max_active": HM2_ACTIVE}


def sfnn_weights(rng: np.random.Generator, input_size: int = HM2_INPUTS + HM2_PIECES, ft: int = 1536,
                 l1_hidden: int = 15, l1_skip: bool = True, l2: int = 32, stacks: int = 9, shared_l1: bool = True,
                 shared_l2_l3: bool = False, std: float = 0.01) -> dict:
    """N(0, std) weights of an SFNN LayerStack net (absent shared factors are None)."""
    o = l1_hidden + int(l1_skip)
    i2 = 2 * l1_hidden
    shapes = {"l0w": input_size * ft, "l0b": ft, "l1w": stacks * o * ft, "l1b": stacks * o,
              "l2w": stacks * l2 * i2, "l2b": stacks * l2, "l3w": stacks * l2, "l3b": stacks}
    if shared_l1:
        shapes.update({"l1fw": ft * o, "l1fb": o})
    if shared_l2_l3:
        shapes.update({"l2fw": l2 * i2, "l2fb": l2, "l3fw": l2, "l3fb": 1})
    out = {k: rng.normal(0.0, std, size=n).astype(np.float32) for k, n in shapes.items()}
    for k in ("l1fw", "l1fb", "l2fw", "l2fb", "l3fw", "l3fb"):
        out.setdefault(k, None)
    return out


# ---------------------------------------------------------------- PackedSfenValue records
# Piece types as in crates/bulletou_lib/src/shogi/types.rs:27-44.
PAWN, LANCE, KNIGHT, SILVER, BISHOP, ROOK, GOLD, KING = 1, 2, 3, 4, 5, 6, 7, 8
PRO_PAWN, PRO_LANCE, PRO_KNIGHT, PRO_SILVER, HORSE, DRAGON = 9, 10, 11, 12, 13, 14
HAND_TYPES = (PAWN, LANCE, KNIGHT, SILVER, GOLD, BISHOP, ROOK)          # Hand slot order
# Board Huffman code of each unpromoted type, LSB first (packed_sfen.rs:17-26).
_BOARD_CODE = {PAWN: (0x01, 2), LANCE: (0x03, 4), KNIGHT: (0x0b, 4), SILVER: (0x07, 4), BISHOP: (0x1f, 6),
               ROOK: (0x3f, 6), GOLD: (0x0f, 5)}
_UNPROMOTE = {PRO_PAWN: PAWN, PRO_LANCE: LANCE, PRO_KNIGHT: KNIGHT, PRO_SILVER: SILVER, HORSE: BISHOP, DRAGON: ROOK}
# 38 non-king pieces of a full set.
FULL_SET = (PAWN,) * 18 + (LANCE,) * 4 + (KNIGHT,) * 4 + (SILVER,) * 4 + (GOLD,) * 4 + (BISHOP,) * 2 + (ROOK,) * 2
PSV_DTYPE = np.dtype([("sfen", "u1", 32), ("score", "<i2"), ("move16", "<u2"), ("game_ply", "<u2"),
                      ("game_result", "i1"), ("padding", "u1")])


def _board_token(code: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """(value, length) of the board token for piece codes type | colour << 4."""
    pt = code & 15
    color = (code >> 4) & 1
    value = np.zeros(code.shape, np.int64)
    length = np.ones(code.shape, np.int64)                 # empty square: "0"
    for t in range(1, 15):
        m = pt == t
        if not m.any():
            continue
        base = _UNPROMOTE.get(t, t)
        pattern, n = _BOARD_CODE[base]
        if base == GOLD:
            value[m] = pattern | (color[m] << n)
            length[m] = n + 1
        else:
            promoted = 1 if t in _UNPROMOTE else 0
            value[m] = pattern | (promoted << n) | (color[m] << (n + 1))
            length[m] = n + 2
    return value, length


def _hand_token(pt: int, color: np.ndarray, piecebox: int = 0) -> tuple[np.ndarray, np.ndarray]:
    pattern, n = _BOARD_CODE[pt]
    hp, hn = pattern >> 1, n - 1
    if pt == GOLD:
        return hp | (color << hn), np.full(color.shape, hn + 1, np.int64)
    return hp | (piecebox << hn) | (color << (hn + 1)), np.full(color.shape, hn + 2, np.int64)


def psv_encode(stm, black_king, white_king, board, hands, score=0, result=0, game_ply=0, move16=0) -> np.ndarray:
    """Encode positions into PackedSfenValue records (YaneuraOu's sfen packer
    format, the inverse of ShogiBoard::from_packed_sfen, packed_sfen.rs:228-284).

    stm, black_king, white_king: [n]; board: [n, 81] piece codes type | colour << 4
    (0 empty; king squares are not read); hands: [n, 2, 7] counts in HAND_TYPES
    order.  Positions with fewer than the full 38 pieces are padded to 256 bits
    with piece-box pawns (a lance at a 4/5-bit tail); a position that leaves a
    1-bit tail cannot be padded and raises."""
    stm = np.atleast_1d(np.asarray(stm, np.int64))
    n = stm.size
    bk = np.broadcast_to(np.asarray(black_king, np.int64), (n,))
    wk = np.broadcast_to(np.asarray(white_king, np.int64), (n,))
    board = np.asarray(board, np.int64).reshape(n, 81)
    hands = np.asarray(hands, np.int64).reshape(n, 2, 7)
    bits = np.zeros((n, 256 + 16), np.uint8)
    cursor = np.zeros(n, np.int64)
    rows = np.arange(n)

    def write(value, length, mask=None):
        value = np.broadcast_to(np.asarray(value, np.int64), (n,))
        length = np.broadcast_to(np.asarray(length, np.int64), (n,))
        if mask is not None:
            length = np.where(mask, length, 0)
        for b in range(int(length.max(initial=0))):
            m = b < length
            if (cursor[m] + b >= 256).any():
                raise ValueError("position needs more than 256 bits")
            bits[rows[m], cursor[m] + b] = (value[m] >> b) & 1
        cursor[:] += length

    write(stm, 1)
    write(bk, 7)
    write(wk, 7)
    for sq in range(81):
        v, ln = _board_token(board[:, sq])
        write(v, ln, (sq != bk) & (sq != wk))
    for color in (0, 1):
        for h, pt in enumerate(HAND_TYPES):
            for i in range(int(hands[:, color, h].max(initial=0))):
                v, ln = _hand_token(pt, np.full(n, color, np.int64))
                write(v, ln, hands[:, color, h] > i)
    # piece-box padding up to bit 256
    while True:
        r = 256 - cursor
        if (r == 1).any():
            raise ValueError("a 1-bit tail cannot be padded with piece-box pieces")
        pawn = (r >= 3) & (r != 4) & (r != 5)
        if not pawn.any():
            break
        write(0b010, 3, pawn)                                      # pawn code 0, box 1, black
    r = 256 - cursor
    write(0b10, 2, r == 2)                                         # pawn + box, colour bit past the end
    write(0b1001, 4, r == 4)                                       # lance code + box, colour past the end
    write(0b01001, 5, r == 5)                                      # lance code + box + black
    assert (cursor == 256).all()
    out = np.zeros(n, PSV_DTYPE)
    out["sfen"] = np.packbits(bits[:, :256], axis=1, bitorder="little")
    out["score"] = np.broadcast_to(np.asarray(score, np.int64), (n,)).astype(np.int16)
    out["move16"] = np.broadcast_to(np.asarray(move16, np.int64), (n,)).astype(np.uint16)
    out["game_ply"] = np.broadcast_to(np.asarray(game_ply, np.int64), (n,)).astype(np.uint16)
    out["game_result"] = np.broadcast_to(np.asarray(result, np.int64), (n,)).astype(np.int8)
    return out


def psv_positions(rng: np.random.Generator, n: int, hand_fraction: float = 0.12,
                  promote_fraction: float = 0.06) -> dict:
    """Full-set positions: kings near their home ranks, each of the 38 other
    pieces owned by either side, in hand with probability `hand_fraction`,
    else on a random free square (promoted with probability
    `promote_fraction` unless gold).  A full set packs into exactly 256 bits."""
    def king(home):
        rank = np.where(rng.random(n) < 0.85, home + np.where(home == 0, 1, -1) * rng.integers(0, 2, n),
                        rng.integers(0, 9, n))
        return rng.integers(0, 9, n) * 9 + rank

    bk = king(np.full(n, 8))
    wk = king(np.full(n, 0))
    clash = bk == wk
    wk[clash] = (wk[clash] + 9) % 81
    stm = rng.integers(0, 2, n)
    board = np.zeros((n, 81), np.int64)
    hands = np.zeros((n, 2, 7), np.int64)
    key = rng.random((n, 81))
    key[np.arange(n), bk] = 2.0
    key[np.arange(n), wk] = 2.0
    order = np.argsort(key, axis=1)                                  # free squares first
    slot = np.zeros(n, np.int64)
    rows = np.arange(n)
    for pt in FULL_SET:
        color = rng.integers(0, 2, n)
        in_hand = rng.random(n) < hand_fraction
        h = HAND_TYPES.index(pt)
        np.add.at(hands, (rows[in_hand], color[in_hand], h), 1)
        on = ~in_hand
        sq = order[rows[on], slot[on]]
        code = np.full(on.sum(), pt, np.int64)
        if pt != GOLD:
            promo = rng.random(on.sum()) < promote_fraction
            code[promo] = {PAWN: PRO_PAWN, LANCE: PRO_LANCE, KNIGHT: PRO_KNIGHT, SILVER: PRO_SILVER,
                           BISHOP: HORSE, ROOK: DRAGON}[pt]
        board[rows[on], sq] = code | (color[on] << 4)
        slot[on] += 1
    return {"stm": stm, "black_king": bk, "white_king": wk, "board": board, "hands": hands}


def psv_records(seed: int, n: int, rank: int = 0, **kw) -> np.ndarray:
    """`n` seeded PackedSfenValue records of full-set positions with teacher
    scores round(N(0, 600)) clipped to +-3000, results in {-1, 0, 1}."""
    rng = rng_for(seed, rank)
    p = psv_positions(rng, n, **kw)
    score = np.clip(np.rint(rng.normal(0.0, 600.0, n)), -3000, 3000).astype(np.int64)
    result = rng.integers(-1, 2, n)
    ply = rng.integers(1, 320, n)
    move = rng.integers(0, 1 << 16, n)
    return psv_encode(p["stm"], p["black_king"], p["white_king"], p["board"], p["hands"], score, result, ply, move)


# ---------------------------------------------------------------- HCPE records
# Apery / cshogi HuffmanCodedPos codes (the reference's HCP tables,
# crates/bulletou_lib/src/value/loader/shogipack.rs:60-105): knight and silver
# swapped against the PackedSfen table, the colour bit before the promotion
# bit, hand pieces and piece box in one prefix code.
_HCP_BOARD_CODE = {PAWN: (0x01, 2), LANCE: (0x03, 4), KNIGHT: (0x07, 4), SILVER: (0x0b, 4), BISHOP: (0x1f, 6),
                   ROOK: (0x3f, 6), GOLD: (0x0f, 5)}
_HCP_HAND_CODE = {(PAWN, 0): (0x00, 3), (LANCE, 0): (0x01, 5), (KNIGHT, 0): (0x03, 5), (SILVER, 0): (0x05, 5),
                  (GOLD, 0): (0x07, 5), (BISHOP, 0): (0x1f, 7), (ROOK, 0): (0x3f, 7),
                  (PAWN, 1): (0x04, 3), (LANCE, 1): (0x11, 5), (KNIGHT, 1): (0x13, 5), (SILVER, 1): (0x15, 5),
                  (GOLD, 1): (0x17, 5), (BISHOP, 1): (0x5f, 7), (ROOK, 1): (0x7f, 7)}
HCPE_DTYPE = np.dtype([("hcp", "u1", 32), ("eval", "<i2"), ("best_move16", "<u2"), ("game_result", "u1"),
                       ("dummy", "u1")])


def hcpe_encode(stm, black_king, white_king, board, hands, eval_=0, game_result=0, best_move16=0) -> np.ndarray:
    """Encode positions as HCPE records (38 bytes: HCP, eval, bestMove16,
    gameResult 0 draw / 1 black win / 2 white win, padding) -- the inverse of
    MiniPosition::from_hcp.  Same inputs as psv_encode; short positions are
    padded with piece-box pawns (a piece-box lance at a 4/5-bit tail)."""
    stm = np.atleast_1d(np.asarray(stm, np.int64))
    n = stm.size
    bk = np.broadcast_to(np.asarray(black_king, np.int64), (n,))
    wk = np.broadcast_to(np.asarray(white_king, np.int64), (n,))
    board = np.asarray(board, np.int64).reshape(n, 81)
    hands = np.asarray(hands, np.int64).reshape(n, 2, 7)
    bits = np.zeros((n, 256 + 16), np.uint8)
    cursor = np.zeros(n, np.int64)
    rows = np.arange(n)

    def write(value, length, mask=None):
        value = np.broadcast_to(np.asarray(value, np.int64), (n,))
        length = np.broadcast_to(np.asarray(length, np.int64), (n,))
        if mask is not None:
            length = np.where(mask, length, 0)
        for b in range(int(length.max(initial=0))):
            m = b < length
            if (cursor[m] + b >= 256).any():
                raise ValueError("position needs more than 256 bits")
            bits[rows[m], cursor[m] + b] = (value[m] >> b) & 1
        cursor[:] += length

    write(stm, 1)
    write(bk, 7)
    write(wk, 7)
    for sq in range(81):
        code = board[:, sq]
        pt, color = code & 15, (code >> 4) & 1
        value = np.zeros(n, np.int64)
        length = np.ones(n, np.int64)
        for t in range(1, 15):
            m = pt == t
            if not m.any():
                continue
            base = _UNPROMOTE.get(t, t)
            pattern, k = _HCP_BOARD_CODE[base]
            if base == GOLD:
                value[m] = pattern | (color[m] << k)
                length[m] = k + 1
            else:
                value[m] = pattern | (color[m] << k) | ((1 if t in _UNPROMOTE else 0) << (k + 1))
                length[m] = k + 2
        write(value, length, (sq != bk) & (sq != wk))
    for color in (0, 1):
        for h, pt in enumerate(HAND_TYPES):
            code, k = _HCP_HAND_CODE[(pt, color)]
            for i in range(int(hands[:, color, h].max(initial=0))):
                write(code, k, hands[:, color, h] > i)
    while True:
        r = 256 - cursor
        if (r == 1).any():
            raise ValueError("a 1-bit tail cannot be padded with piece-box pieces")
        pawn = (r >= 3) & (r != 4) & (r != 5)
        if not pawn.any():
            break
        write(0b010, 3, pawn)                                      # piece-box pawn (0x02, 3 bits)
    r = 256 - cursor
    write(0b10, 2, r == 2)                                         # its first two bits; the third reads as 0
    write(0b1001, 4, r == 4)                                       # piece-box lance (0x09, 5 bits), 4 written
    write(0b01001, 5, r == 5)
    assert (cursor == 256).all()
    out = np.zeros(n, HCPE_DTYPE)
    out["hcp"] = np.packbits(bits[:, :256], axis=1, bitorder="little")
    out["eval"] = np.broadcast_to(np.asarray(eval_, np.int64), (n,)).astype(np.int16)
    out["best_move16"] = np.broadcast_to(np.asarray(best_move16, np.int64), (n,)).astype(np.uint16)
    out["game_result"] = np.broadcast_to(np.asarray(game_result, np.int64), (n,)).astype(np.uint8)
    return out


def hcpe_records(seed: int, n: int, rank: int = 0, **kw) -> np.ndarray:
    """`n` seeded HCPE records of full-set positions (as psv_records)."""
    rng = rng_for(seed, rank)
    p = psv_positions(rng, n, **kw)
    ev = np.clip(np.rint(rng.normal(0.0, 600.0, n)), -3000, 3000).astype(np.int64)
    return hcpe_encode(p["stm"], p["black_king"], p["white_king"], p["board"], p["hands"], ev,
                       rng.integers(0, 3, n), rng.integers(0, 1 << 16, n))
