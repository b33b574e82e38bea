/* TEST INFRASTRUCTURE ONLY -- scalar CPU restatement of the reference's
 * teacher-batch producer for the cuda-cpp trainers: PackedSfenValue decode ->
 * sparse feature indices, LayerStack bucket, blended target and entry weight.
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load it,
 * as the checker; the product (bulletou_b200) never does.
 *
 * Follows, step for step:
 *   BitStream / decode_board_piece / decode_hand_piece / ShogiBoard::from_packed_sfen
 *       crates/bulletou_lib/src/shogi/packed_sfen.rs:41-88, 228-284, 329-424
 *   BonaPiece::from_piece_square / from_hand_piece, PIECE_BASE
 *       crates/bulletou_lib/src/shogi/bona_piece.rs:92-124, 162-254
 *   Square::inverse / rank / file, Hand, HAND_PIECE_TYPES, BOARD_PIECE_TYPES
 *       crates/bulletou_lib/src/shogi/types.rs:160-200, 252-300, 380-400
 *   halfka_hm2_index / map_halfka_hm2_features (piece type, colour, square order)
 *       crates/bulletou_lib/src/game/inputs/shogi_halfka_hm2.rs:106-258
 *   map_halfkp_features_from_packed (square order, saturating hand counts)
 *       crates/bulletou_lib/src/game/inputs/shogi_halfkp.rs:161-227
 *   LayerStack bucket (hand axis x king axis; the progress axis is not restated)
 *       crates/bulletou_lib/src/game/outputs.rs:99-133, 200-420, 860-1000, 1177-1231
 *   targets / entry weights of prepare_sfnn_fast_batch_from_board_features and
 *   prepare_halfkp_direct_fast_batch
 *       crates/bulletou_lib/src/value/teacher_batch.rs:1687-1750, 2869-3010
 *   win-rate-model score table lookup  crates/bulletou_lib/src/value/loader.rs:706-709
 *
 * Integer widths follow the reference: squares are u8 (Square::inverse wraps
 * for the king-less sentinel squares 81..127, as a release build does), hand
 * counts are u8.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

enum { PT_NONE = 0, PAWN, LANCE, KNIGHT, SILVER, BISHOP, ROOK, GOLD, KING, PRO_PAWN, PRO_LANCE, PRO_KNIGHT,
       PRO_SILVER, HORSE, DRAGON };
enum { BLACK = 0, WHITE = 1 };

/* ------------------------------------------------------------ bit stream */
typedef struct {
    const uint8_t* data;
    int cursor;
    int limit;
} bitstream;

static int bs_read_bit(bitstream* s) {
    if (s->cursor >= s->limit) return 0;                      /* out of range reads as 0 */
    int bit = (s->data[s->cursor / 8] >> (s->cursor % 8)) & 1;
    s->cursor++;
    return bit;
}

static uint32_t bs_read_bits(bitstream* s, int n) {
    uint32_t r = 0;
    for (int i = 0; i < n; ++i)
        if (bs_read_bit(s)) r |= 1u << i;
    return r;
}

/* ------------------------------------------------------------ Huffman codes */
/* index: 0 = no piece, 1 pawn, 2 lance, 3 knight, 4 silver, 5 bishop, 6 rook, 7 gold */
static const uint32_t HUFF_PATTERN[8] = {0x00, 0x01, 0x03, 0x0b, 0x07, 0x1f, 0x3f, 0x0f};
static const int HUFF_LEN[8] = {1, 2, 4, 4, 4, 6, 6, 5};
static const int HUFF_TYPE[8] = {PT_NONE, PAWN, LANCE, KNIGHT, SILVER, BISHOP, ROOK, GOLD};
#define HUFF_GOLD 7

static int promote(int pt) {
    switch (pt) {
        case PAWN: return PRO_PAWN;
        case LANCE: return PRO_LANCE;
        case KNIGHT: return PRO_KNIGHT;
        case SILVER: return PRO_SILVER;
        case BISHOP: return HORSE;
        case ROOK: return DRAGON;
        default: return pt;
    }
}

typedef struct {
    int pt;
    int color;
} piece;

static piece decode_board_piece(bitstream* s) {
    uint32_t code = 0;
    int bits = 0;
    for (;;) {
        code |= (uint32_t)bs_read_bit(s) << bits;
        bits++;
        for (int idx = 0; idx < 8; ++idx) {
            if (bits == HUFF_LEN[idx] && code == HUFF_PATTERN[idx]) {
                if (idx == 0) return (piece){PT_NONE, BLACK};
                int promoted = idx != HUFF_GOLD ? bs_read_bit(s) : 0;
                int color = bs_read_bit(s) ? WHITE : BLACK;
                int base = HUFF_TYPE[idx];
                return (piece){promoted ? promote(base) : base, color};
            }
        }
        if (bits > 6) return (piece){PT_NONE, BLACK};
    }
}

/* returns the piece; *piecebox = 1 for a piece-box piece */
static piece decode_hand_piece(bitstream* s, int* piecebox) {
    uint32_t code = 0;
    int bits = 0;
    for (;;) {
        code |= (uint32_t)bs_read_bit(s) << bits;
        bits++;
        for (int idx = 1; idx < 8; ++idx) {
            if (bits == HUFF_LEN[idx] - 1 && code == (HUFF_PATTERN[idx] >> 1)) {
                *piecebox = idx != HUFF_GOLD ? bs_read_bit(s) : 0;
                int color = bs_read_bit(s) ? WHITE : BLACK;
                return (piece){HUFF_TYPE[idx], color};
            }
        }
        if (bits > 5) {
            *piecebox = 0;
            return (piece){PT_NONE, BLACK};
        }
    }
}

/* ------------------------------------------------------------ board */
static int hand_index(int pt) {
    switch (pt) {
        case PAWN: return 0;
        case LANCE: return 1;
        case KNIGHT: return 2;
        case SILVER: return 3;
        case GOLD: return 4;
        case BISHOP: return 5;
        case ROOK: return 6;
        default: return -1;
    }
}

typedef struct {
    piece board[81];
    uint8_t hand[2][7];          /* [colour][pawn, lance, knight, silver, gold, bishop, rook] */
    int stm;
    uint8_t king[2];             /* black, white king squares (u8; >= 81 means none) */
    int16_t score;
    int8_t result;
    uint16_t ply;
    int cursor_after_board;
} shogi_board;

static int16_t rd_i16(const uint8_t* p) { return (int16_t)(uint16_t)(p[0] | (p[1] << 8)); }

static void decode_psv(const uint8_t* rec, shogi_board* b) {
    memset(b, 0, sizeof(*b));
    b->score = rd_i16(rec + 32);
    b->ply = (uint16_t)(rec[36] | (rec[37] << 8));
    b->result = (int8_t)rec[38];
    bitstream s = {rec, 0, 256};
    b->stm = bs_read_bit(&s) ? WHITE : BLACK;
    b->king[BLACK] = (uint8_t)bs_read_bits(&s, 7);
    b->king[WHITE] = (uint8_t)bs_read_bits(&s, 7);
    if (b->king[BLACK] < 81) b->board[b->king[BLACK]] = (piece){KING, BLACK};
    if (b->king[WHITE] < 81) b->board[b->king[WHITE]] = (piece){KING, WHITE};
    for (int sq = 0; sq < 81; ++sq) {
        if (sq == b->king[BLACK] || sq == b->king[WHITE]) continue;
        b->board[sq] = decode_board_piece(&s);
    }
    b->cursor_after_board = s.cursor;
    while (s.cursor < 256) {
        int box = 0;
        piece p = decode_hand_piece(&s, &box);
        if (box) continue;
        int h = hand_index(p.pt);
        if (h >= 0) b->hand[p.color][h] = (uint8_t)(b->hand[p.color][h] + 1);
    }
}

/* ------------------------------------------------------------ BonaPiece */
#define FE_HAND_END 90
#define F_KING 1548
#define E_KING 1629
#define FE_END 1548
#define HM2_PIECE_INPUTS 1629

/* [piece type][is_friend] */
static const int PIECE_BASE[15][2] = {
    {0, 0}, {171, 90}, {333, 252}, {495, 414}, {657, 576}, {981, 900}, {1305, 1224}, {819, 738}, {0, 0},
    {819, 738}, {819, 738}, {819, 738}, {819, 738}, {1143, 1062}, {1467, 1386}};
/* hand bases [hand index][is_friend] */
static const int HAND_BASE[7][2] = {{20, 1}, {44, 39}, {54, 49}, {64, 59}, {74, 69}, {82, 79}, {88, 85}};
static const int BOARD_TYPES[13] = {PAWN, LANCE, KNIGHT, SILVER, GOLD, BISHOP, ROOK, PRO_PAWN, PRO_LANCE,
                                    PRO_KNIGHT, PRO_SILVER, HORSE, DRAGON};

static uint8_t sq_inverse(uint8_t sq) { return (uint8_t)(80 - sq); }     /* wraps like a u8 */

static int bona_board(piece p, int sq, int perspective) {
    if (p.pt == PT_NONE || p.pt == KING) return 0;
    int s = perspective == BLACK ? sq : 80 - sq;
    return PIECE_BASE[p.pt][p.color == perspective] + s;
}

static int bona_hand(int perspective, int owner, int h, int count) {
    if (count == 0) return 0;
    return HAND_BASE[h][owner == perspective] + count - 1;
}

static int mirror_file(int sq) { return (8 - sq / 9) * 9 + sq % 9; }

int64_t oracle_halfka_hm2_index(int64_t king, int64_t bp) {
    int64_t k = king;
    int64_t b = bp;
    if (king / 9 >= 5) {
        k = mirror_file((int)king);
        if (bp >= FE_HAND_END) {
            int64_t off = bp - FE_HAND_END;
            b = FE_HAND_END + (off / 81) * 81 + mirror_file((int)(off % 81));
        }
    }
    if (b >= E_KING) b -= 81;
    return k * HM2_PIECE_INPUTS + b;
}

/* ------------------------------------------------------------ features */
typedef struct {
    int32_t* stm;
    int32_t* nstm;
    int cap;
    int count;
} feature_sink;

static void emit(feature_sink* f, int64_t a, int64_t b) {
    if (f->count < f->cap) {
        f->stm[f->count] = (int32_t)a;
        f->nstm[f->count] = (int32_t)b;
    }
    f->count++;
}

static void map_halfka_hm2(const shogi_board* b, feature_sink* f) {
    int stm = b->stm, nstm = 1 - stm;
    uint8_t sk = b->king[stm], nk = b->king[nstm];
    if (sk >= 81 || nk >= 81) return;
    int stm_ksq = stm == BLACK ? sk : 80 - sk;
    int nstm_ksq = nstm == BLACK ? nk : 80 - nk;
    for (int t = 0; t < 13; ++t) {
        int pt = BOARD_TYPES[t];
        for (int color = BLACK; color <= WHITE; ++color) {
            for (int sq = 0; sq < 81; ++sq) {
                if (b->board[sq].pt != pt || b->board[sq].color != color) continue;
                piece p = {pt, color};
                int sbp = bona_board(p, sq, stm);
                if (sbp == 0) continue;
                int nbp = bona_board(p, sq, nstm);
                emit(f, oracle_halfka_hm2_index(stm_ksq, sbp), oracle_halfka_hm2_index(nstm_ksq, nbp));
            }
        }
    }
    {
        int sf = F_KING + (stm == BLACK ? sk : 80 - sk);
        int se = E_KING + (stm == BLACK ? nk : 80 - nk);
        int nf = F_KING + (nstm == BLACK ? nk : 80 - nk);
        int ne = E_KING + (nstm == BLACK ? sk : 80 - sk);
        emit(f, oracle_halfka_hm2_index(stm_ksq, sf), oracle_halfka_hm2_index(nstm_ksq, nf));
        emit(f, oracle_halfka_hm2_index(stm_ksq, se), oracle_halfka_hm2_index(nstm_ksq, ne));
    }
    for (int owner = BLACK; owner <= WHITE; ++owner) {
        for (int h = 0; h < 7; ++h) {
            int count = b->hand[owner][h];
            for (int i = 1; i <= count; ++i) {
                int sbp = bona_hand(stm, owner, h, i);
                if (sbp == 0) continue;
                int nbp = bona_hand(nstm, owner, h, i);
                emit(f, oracle_halfka_hm2_index(stm_ksq, sbp), oracle_halfka_hm2_index(nstm_ksq, nbp));
            }
        }
    }
}

/* map_halfkp_features_from_packed: streams the record itself, board pieces in
 * square order; returns before decoding when a king square is invalid. */
static void map_halfkp_packed(const uint8_t* rec, feature_sink* f) {
    bitstream s = {rec, 0, 256};
    int stm = bs_read_bit(&s) ? WHITE : BLACK, nstm = 1 - stm;
    uint8_t king[2];
    king[BLACK] = (uint8_t)bs_read_bits(&s, 7);
    king[WHITE] = (uint8_t)bs_read_bits(&s, 7);
    uint8_t sk = king[stm], nk = king[nstm];
    if (sk >= 81 || nk >= 81) return;
    int stm_ksq = stm == BLACK ? sk : 80 - sk;
    int nstm_ksq = nstm == BLACK ? nk : 80 - nk;
    for (int sq = 0; sq < 81; ++sq) {
        if (sq == king[BLACK] || sq == king[WHITE]) continue;
        piece p = decode_board_piece(&s);
        if (p.pt == PT_NONE || p.pt == KING) continue;
        int sbp = bona_board(p, sq, stm);
        if (sbp == 0) continue;
        int nbp = bona_board(p, sq, nstm);
        emit(f, (int64_t)stm_ksq * FE_END + sbp, (int64_t)nstm_ksq * FE_END + nbp);
    }
    uint8_t counts[2][7];
    memset(counts, 0, sizeof(counts));
    while (s.cursor < 256) {
        int box = 0;
        piece p = decode_hand_piece(&s, &box);
        if (box || p.pt == PT_NONE) continue;
        int h = hand_index(p.pt);
        if (h >= 0 && counts[p.color][h] < 255) counts[p.color][h]++;         /* saturating_add */
    }
    for (int owner = BLACK; owner <= WHITE; ++owner) {
        for (int h = 0; h < 7; ++h) {
            for (int i = 1; i <= counts[owner][h]; ++i) {
                int sbp = bona_hand(stm, owner, h, i);
                if (sbp == 0) continue;
                int nbp = bona_hand(nstm, owner, h, i);
                emit(f, (int64_t)stm_ksq * FE_END + sbp, (int64_t)nstm_ksq * FE_END + nbp);
            }
        }
    }
}

/* ------------------------------------------------------------ buckets */
static int rank_of(uint8_t sq) { return sq % 9; }
static int file_of(uint8_t sq) { return sq / 9; }
static int imin(int a, int b) { return a < b ? a : b; }

static int king9_zone(uint8_t sq) {
    int r = imin(rank_of(sq), 8);
    if (r < 3) return 0;
    if (r < 6) return 1;
    if (r == 6) return 2;
    return 3 + (r - 7) * 3 + imin(file_of(sq), 8) / 3;
}
static int king13_zone(uint8_t sq) {
    int r = imin(rank_of(sq), 8);
    return r < 7 ? r : 7 + (r - 7) * 3 + imin(file_of(sq), 8) / 3;
}
static int king21(uint8_t sq) {
    int r = imin(rank_of(sq), 8), f = imin(file_of(sq), 8);
    if (r < 3) return 0;
    if (r < 6) return 1;
    if (r < 7) return 2;
    return 3 + (r - 7) * 9 + f;
}
static int king29(uint8_t sq) {
    int r = imin(rank_of(sq), 8), f = imin(file_of(sq), 8);
    if (r < 3) return 0;
    if (r < 6) return 1;
    return 2 + (r - 6) * 9 + f;
}

/* king axis: 0 none, 1 rank9, 2 rank81, 3 k9 zone, 4 k13 zone, 5 k21, 6 k21 zone, 7 k29 */
static const int KING_COUNT[8] = {1, 9, 81, 81, 169, 441, 441, 841};
/* hand axis: 0 none, 1 hand4, 2 hand16, 3 hand64, 4 hand64z, 5 hand256, 6 hand1024 */
static const int HAND_COUNT[7] = {1, 4, 16, 64, 64, 256, 1024};

int oracle_teacher_bucket_count(int hand_kind, int king_kind) {
    if (hand_kind < 0 || hand_kind > 6 || king_kind < 0 || king_kind > 7) return -1;
    return HAND_COUNT[hand_kind] * KING_COUNT[king_kind];
}

static int king_bucket(int kind, uint8_t f_sq, uint8_t e_sq) {
    static const int F_TO[9] = {0, 0, 0, 3, 3, 3, 6, 6, 6};
    static const int E_TO[9] = {0, 0, 0, 1, 1, 1, 2, 2, 2};
    int fr = imin(rank_of(f_sq), 8), er = imin(rank_of(e_sq), 8);
    switch (kind) {
        case 1: return F_TO[fr] + E_TO[er];
        case 2: return fr * 9 + er;
        case 3: return king9_zone(f_sq) * 9 + king9_zone(e_sq);
        case 4: return king13_zone(f_sq) * 13 + king13_zone(e_sq);
        case 5:
        case 6: return king21(f_sq) * 21 + king21(e_sq);
        case 7: return king29(f_sq) * 29 + king29(e_sq);
        default: return 0;
    }
}

/* u8 sums as the reference writes them (no overflow is reachable from 256 bits) */
static int hand_single(int kind, const uint8_t* h) {
    uint8_t pawn = h[0], lance = h[1], knight = h[2], silver = h[3], gold = h[4], bishop = h[5], rook = h[6];
    int b = 0;
    switch (kind) {
        case 1: return bishop > 0;
        case 2: return (pawn > 0 ? 1 : 0) | (bishop > 0 ? 2 : 0);
        case 3:
            if ((uint8_t)(pawn + lance + knight) > 0) b |= 1;
            if ((uint8_t)(gold + silver + rook) > 0) b |= 2;
            if (bishop > 0) b |= 4;
            return b;
        case 4: {
            int score = pawn + (uint8_t)(lance + knight) * 2 + (uint8_t)(silver + gold) * 3 +
                        (uint8_t)(bishop + rook) * 5;
            return imin((score + 3) / 4, 7);
        }
        case 5:
            if ((uint8_t)(pawn + lance + knight) > 0) b |= 1;
            if ((uint8_t)(silver + gold) > 0) b |= 2;
            if (bishop > 0) b |= 4;
            if (rook > 0) b |= 8;
            return b;
        case 6:
            if (pawn > 0) b |= 1;
            if ((uint8_t)(lance + knight) > 0) b |= 2;
            if ((uint8_t)(silver + gold) > 0) b |= 4;
            if (bishop > 0) b |= 8;
            if (rook > 0) b |= 16;
            return b;
        default: return 0;
    }
}

static const int HAND_AXIS[7] = {1, 2, 4, 8, 8, 16, 32};

static int layerstack_bucket(const shogi_board* b, int hand_kind, int king_kind) {
    int stm = b->stm;
    const uint8_t* sh = b->hand[stm];
    const uint8_t* nh = b->hand[1 - stm];
    int hb = hand_kind == 0 ? 0 : hand_single(hand_kind, sh) * HAND_AXIS[hand_kind] + hand_single(hand_kind, nh);
    uint8_t fk = b->king[stm], ek = b->king[1 - stm];
    uint8_t f_sq = stm == BLACK ? fk : sq_inverse(fk);
    uint8_t e_sq = stm == BLACK ? sq_inverse(ek) : ek;
    return hb * KING_COUNT[king_kind] + king_bucket(king_kind, f_sq, e_sq);
}

/* ------------------------------------------------------------ batch */
typedef struct {
    int32_t feature_set;       /* 0 HalfKA_hm2 (SFNN), 1 HalfKP */
    int32_t max_active;
    int32_t hand_bucket;
    int32_t king_bucket;
    float result_blend;
    float score_blend;
    float rscale;
    int32_t score_drop_abs;    /* < 0: none */
} oracle_teacher_config;

static float sigmoid_target(float rscale, int16_t score) {
    float x = -(rscale * (float)score);
    return 1.0f / (1.0f + expf(x));
}

/* One batch: stm/nstm [n][max_active] (-1 padded), buckets [n] (may be NULL),
 * targets [n], weights [n], counts [n] = features enumerated per record (a
 * count above max_active is the reference's "exceeded max_active" abort). */
void oracle_teacher_prepare(const uint8_t* records, int64_t n, const oracle_teacher_config* cfg,
                            const float* wrm_table, int32_t* stm, int32_t* nstm, int32_t* buckets, float* targets,
                            float* weights, int32_t* counts) {
    int A = cfg->max_active;
    for (int64_t i = 0; i < n; ++i) {
        const uint8_t* rec = records + 40 * i;
        feature_sink f = {stm + i * A, nstm + i * A, A, 0};
        for (int k = 0; k < A; ++k) f.stm[k] = f.nstm[k] = -1;
        shogi_board b;
        decode_psv(rec, &b);
        if (cfg->feature_set == 0) {
            map_halfka_hm2(&b, &f);
            if (buckets) buckets[i] = layerstack_bucket(&b, cfg->hand_bucket, cfg->king_bucket);
        } else {
            map_halfkp_packed(rec, &f);
            if (buckets) buckets[i] = 0;
        }
        counts[i] = f.count;
        int16_t score = b.score;
        float w = 1.0f;
        if (cfg->score_drop_abs >= 0) {
            uint32_t mag = score < 0 ? (uint32_t)(-(int32_t)score) : (uint32_t)score;
            if (mag >= (uint32_t)cfg->score_drop_abs) w = 0.0f;
        }
        weights[i] = w;
        float sp = wrm_table ? wrm_table[(int32_t)score + 32768] : sigmoid_target(cfg->rscale, score);
        float result = b.result > 0 ? 1.0f : (b.result < 0 ? 0.0f : 0.5f);
        targets[i] = cfg->result_blend * result + cfg->score_blend * sp;
    }
}

/* ------------------------------------------------------------ pins */
/* Board decode for the known-answer tests: board[sq] = type | colour << 4,
 * hands [2][7], header fields; returns the cursor after the board. */
int oracle_psv_decode(const uint8_t* rec, uint8_t* board, uint8_t* hands, int32_t* header) {
    shogi_board b;
    decode_psv(rec, &b);
    for (int sq = 0; sq < 81; ++sq) board[sq] = (uint8_t)(b.board[sq].pt | (b.board[sq].color << 4));
    memcpy(hands, b.hand, 14);
    header[0] = b.stm;
    header[1] = b.king[BLACK];
    header[2] = b.king[WHITE];
    header[3] = b.score;
    header[4] = b.ply;
    header[5] = b.result;
    return b.cursor_after_board;
}

/* decode one piece from `data` (len bytes) at bit 0: out = {type, colour, piecebox, cursor} */
void oracle_decode_piece(const uint8_t* data, int32_t len, int32_t hand, int32_t* out) {
    bitstream s = {data, 0, 8 * len};
    int box = 0;
    piece p = hand ? decode_hand_piece(&s, &box) : decode_board_piece(&s);
    out[0] = p.pt;
    out[1] = p.color;
    out[2] = box;
    out[3] = s.cursor;
}

void oracle_read_bits(const uint8_t* data, int32_t len, const int32_t* widths, int32_t n, uint32_t* values,
                      int32_t* cursors) {
    bitstream s = {data, 0, 8 * len};
    for (int i = 0; i < n; ++i) {
        values[i] = bs_read_bits(&s, widths[i]);
        cursors[i] = s.cursor;
    }
}

int32_t oracle_bona_board(int32_t pt, int32_t color, int32_t sq, int32_t perspective) {
    return bona_board((piece){pt, color}, sq, perspective);
}

int32_t oracle_bona_hand(int32_t perspective, int32_t owner, int32_t pt, int32_t count) {
    int h = hand_index(pt);
    return h < 0 ? 0 : bona_hand(perspective, owner, h, count);
}

int32_t oracle_king_single_bucket(int32_t kind, int32_t sq) {
    switch (kind) {
        case 3: return king9_zone((uint8_t)sq);
        case 4: return king13_zone((uint8_t)sq);
        case 5: return king21((uint8_t)sq);
        case 7: return king29((uint8_t)sq);
        default: return -1;
    }
}

int32_t oracle_hand_single_bucket(int32_t kind, const uint8_t* hand) { return hand_single(kind, hand); }

/* WinRateModelTargetParams::probability over every i16 score
 * (crates/bulletou_lib/src/value/loader.rs:667-672, 681-687). */
static float sigmoid_f(float x) { return 1.0f / (1.0f + expf(-x)); }

void oracle_wrm_table(float offset, float scaling, float epsilon, float* table) {
    for (int32_t raw = -32768; raw <= 32767; ++raw) {
        float score = (float)raw;
        float p = (score - offset) / scaling;
        float pm = (-score - offset) / scaling;
        float prob = 0.5f * (1.0f + sigmoid_f(p) - sigmoid_f(pm));
        table[raw + 32768] = epsilon == 0.0f ? prob : epsilon + (1.0f - 2.0f * epsilon) * prob;
    }
}

/* ------------------------------------------------------------ HCPE records */
/* decode_hcpe_record (crates/bulletou_lib/src/value/loader/hcpe.rs:65-76):
 * MiniPosition::from_hcp (loader/shogipack.rs:353-408) with the Apery / cshogi
 * tables (shogipack.rs:60-105: knight and silver codes swapped against the
 * PackedSfen table, colour bit before the promotion bit, hands and piece box
 * in one prefix code), then pack_to_psfen (:477-554: board in square order,
 * hands by colour and type, piece-box pawns up to bit 256, writes past bit 256
 * dropped), to_packed_sfen_value (:557-569: game_ply 0) and
 * convert_game_result (:679-697).  Returns 1 and writes the 40-byte record, or
 * 0 for a record the reference skips (a king square >= 81, an unknown hand
 * code). */
static const uint32_t HCP_PATTERN[8] = {0x00, 0x01, 0x03, 0x07, 0x0b, 0x1f, 0x3f, 0x0f};
static const int HCP_LEN[8] = {1, 2, 4, 4, 4, 6, 6, 5};
static const int HCP_TYPE[8] = {PT_NONE, PAWN, LANCE, KNIGHT, SILVER, BISHOP, ROOK, GOLD};
/* {code, bits, piece type, colour (-1: piece box)} in the reference's table order */
static const int HCP_HAND[21][4] = {
    {0x00, 3, PAWN, BLACK},   {0x01, 5, LANCE, BLACK},  {0x03, 5, KNIGHT, BLACK}, {0x05, 5, SILVER, BLACK},
    {0x07, 5, GOLD, BLACK},   {0x1f, 7, BISHOP, BLACK}, {0x3f, 7, ROOK, BLACK},   {0x04, 3, PAWN, WHITE},
    {0x11, 5, LANCE, WHITE},  {0x13, 5, KNIGHT, WHITE}, {0x15, 5, SILVER, WHITE}, {0x17, 5, GOLD, WHITE},
    {0x5f, 7, BISHOP, WHITE}, {0x7f, 7, ROOK, WHITE},   {0x02, 3, PAWN, -1},      {0x09, 5, LANCE, -1},
    {0x0b, 5, KNIGHT, -1},    {0x0d, 5, SILVER, -1},    {0x1d, 5, GOLD, -1},      {0x0f, 7, BISHOP, -1},
    {0x2f, 7, ROOK, -1}};

static int unpromote(int pt) {
    switch (pt) {
        case PRO_PAWN: return PAWN;
        case PRO_LANCE: return LANCE;
        case PRO_KNIGHT: return KNIGHT;
        case PRO_SILVER: return SILVER;
        case HORSE: return BISHOP;
        case DRAGON: return ROOK;
        default: return pt;
    }
}

typedef struct {
    uint8_t data[32];
    int cursor;
} bitwriter;

static void bw_bit(bitwriter* w, int b) {
    if (w->cursor < 256) {
        if (b) w->data[w->cursor / 8] |= (uint8_t)(1u << (w->cursor % 8));
        w->cursor++;
    }
}

static void bw_bits(bitwriter* w, uint32_t v, int n) {
    for (int i = 0; i < n; ++i) bw_bit(w, (v >> i) & 1u);
}

static int psv_index_of(int pt) {       /* piece_type_to_index, shogipack.rs:212-224 */
    switch (unpromote(pt)) {
        case PAWN: return 1;
        case LANCE: return 2;
        case KNIGHT: return 3;
        case SILVER: return 4;
        case BISHOP: return 5;
        case ROOK: return 6;
        case GOLD: return 7;
        default: return 0;
    }
}

static int is_promoted(int pt) { return pt >= PRO_PAWN && pt <= DRAGON; }

int oracle_hcpe_to_psv(const uint8_t* rec, uint8_t* psv) {
    piece board[81];
    uint8_t hands[2][7];
    memset(board, 0, sizeof(board));
    memset(hands, 0, sizeof(hands));
    bitstream s = {rec, 0, 256};
    int stm = bs_read_bit(&s) ? WHITE : BLACK;
    int bk = (int)bs_read_bits(&s, 7);
    if (bk >= 81) return 0;
    board[bk] = (piece){KING, BLACK};
    int wk = (int)bs_read_bits(&s, 7);
    if (wk >= 81) return 0;
    board[wk] = (piece){KING, WHITE};
    for (int sq = 0; sq < 81; ++sq) {
        if (sq == bk || sq == wk) continue;
        uint32_t code = 0;
        int bits = 0, idx = -1;
        for (;;) {
            code |= (uint32_t)bs_read_bit(&s) << bits;
            bits++;
            if (bits > 6) return 0;
            for (int i = 0; i < 8 && idx < 0; ++i)
                if (HCP_PATTERN[i] == code && HCP_LEN[i] == bits) idx = i;
            if (idx >= 0) break;
        }
        if (idx == 0) continue;
        int base = HCP_TYPE[idx];
        int color = bs_read_bit(&s) ? WHITE : BLACK;
        int promoted = base != GOLD ? bs_read_bit(&s) : 0;
        board[sq] = (piece){promoted ? promote(base) : base, color};
    }
    while (s.cursor < 256) {
        uint32_t code = 0;
        int bits = 0, e = -1;
        for (;;) {
            code |= (uint32_t)bs_read_bit(&s) << bits;
            bits++;
            if (bits > 7) return 0;
            for (int i = 0; i < 21 && e < 0; ++i)
                if ((uint32_t)HCP_HAND[i][0] == code && HCP_HAND[i][1] == bits) e = i;
            if (e >= 0) break;
        }
        if (HCP_HAND[e][3] < 0) continue;               /* piece box */
        int h = hand_index(HCP_HAND[e][2]);
        hands[HCP_HAND[e][3]][h] = (uint8_t)(hands[HCP_HAND[e][3]][h] + 1);
    }
    /* pack_to_psfen */
    int kb = 81, kw = 81;
    for (int sq = 80; sq >= 0; --sq) {
        if (board[sq].pt == KING && board[sq].color == BLACK) kb = sq;
        if (board[sq].pt == KING && board[sq].color == WHITE) kw = sq;
    }
    bitwriter w;
    memset(&w, 0, sizeof(w));
    bw_bit(&w, stm == WHITE);
    bw_bits(&w, (uint32_t)kb, 7);
    bw_bits(&w, (uint32_t)kw, 7);
    for (int sq = 0; sq < 81; ++sq) {
        if (sq == kb || sq == kw) continue;
        piece p = board[sq];
        if (p.pt == PT_NONE) {
            bw_bit(&w, 0);
            continue;
        }
        int idx = psv_index_of(p.pt);
        bw_bits(&w, HUFF_PATTERN[idx], HUFF_LEN[idx]);
        if (unpromote(p.pt) != GOLD) bw_bit(&w, is_promoted(p.pt));
        bw_bit(&w, p.color == WHITE);
    }
    static const int HAND_ORDER[7] = {PAWN, LANCE, KNIGHT, SILVER, GOLD, BISHOP, ROOK};
    for (int color = BLACK; color <= WHITE; ++color) {
        for (int t = 0; t < 7; ++t) {
            int pt = HAND_ORDER[t];
            int idx = psv_index_of(pt);
            for (int c = 0; c < hands[color][hand_index(pt)]; ++c) {
                bw_bits(&w, HUFF_PATTERN[idx] >> 1, HUFF_LEN[idx] - 1);
                if (pt != GOLD) bw_bit(&w, 0);
                bw_bit(&w, color == WHITE);
            }
        }
    }
    while (w.cursor < 256) {
        bw_bit(&w, 0);
        bw_bit(&w, 1);
        bw_bit(&w, 0);
    }
    memcpy(psv, w.data, 32);
    psv[32] = rec[32];                                   /* eval (i16 LE) */
    psv[33] = rec[33];
    psv[34] = rec[34];                                   /* bestMove16 */
    psv[35] = rec[35];
    psv[36] = 0;                                         /* game_ply */
    psv[37] = 0;
    int r = rec[36] == 1 ? (stm == BLACK ? 1 : -1) : (rec[36] == 2 ? (stm == WHITE ? 1 : -1) : 0);
    psv[38] = (uint8_t)(int8_t)r;
    psv[39] = 0;
    return 1;
}

/* ------------------------------------------------------------ validation metrics */
/* build_validation_sample_mask + compute_sign_accuracy_with_loss_masked
 * (crates/bulletou_lib/src/validate.rs:353-470), the per-sample loss in f32
 * with the C library's expf / powf / log1pf and the sum in double in index
 * order.  results may be NULL (the score-sign path, no loss).  counts: compared,
 * sign_matches, predicted_nonnegative, predicted_negative, predicted_zero,
 * drawn_games, filtered_by_score_cap, loss_sampled. */
typedef struct {
    int32_t have_results;
    int32_t score_drop_abs;
    int32_t loss_kind;     /* 0 sigmoid-pow, 1 win-rate model, 2 BCE with logits */
    float lambda;
    float eval_scale;
    float model_output_scale;
    float pow_exp;
    float nnue2score;
    float in_offset;
    float in_scaling;
} oracle_validation_config;

static float sig(float x) { return 1.0f / (1.0f + expf(-x)); }

static float bce_logits(float z, float t) {
    float lin = z >= 0.0f ? (1.0f - t) * z : -t * z;
    return lin + log1pf(expf(-fabsf(z)));
}

void oracle_validation_metrics(const float* outputs, const int16_t* scores, const int8_t* results, int64_t n,
                               const oracle_validation_config* c, const float* wrm_table, int64_t* counts,
                               double* loss_sum) {
    for (int k = 0; k < 8; ++k) counts[k] = 0;
    double sum = 0.0;
    int have = results != NULL && c->have_results;
    for (int64_t i = 0; i < n; ++i) {
        int s = scores[i];
        if (c->score_drop_abs >= 0 && (s < 0 ? -s : s) >= c->score_drop_abs) {
            counts[6]++;
            continue;
        }
        int draw = have ? results[i] == 0 : s == 0;
        float m = outputs[i];
        if (draw) {
            counts[5]++;
        } else {
            counts[0]++;
            int pred = m >= 0.0f;
            counts[pred ? 2 : 3]++;
            if (m == 0.0f) counts[4]++;
            int truth = have ? results[i] > 0 : s > 0;
            if (pred == truth) counts[1]++;
        }
        if (!have) continue;
        counts[7]++;
        float blend = 1.0f - c->lambda;
        float inv_scale = c->eval_scale > 0.0f ? 1.0f / c->eval_scale : 0.0025f;
        float model_inv = c->model_output_scale > 0.0f ? 1.0f / c->model_output_scale : 1.0f;
        int r = results[i];
        float result_norm = r > 0 ? 1.0f : (r < 0 ? 0.0f : 0.5f);
        float score_norm = c->loss_kind == 0 ? sig(inv_scale * (float)s) : wrm_table[s + 32768];
        float target = blend * result_norm + (1.0f - blend) * score_norm;
        float l;
        if (c->loss_kind == 2) {
            l = bce_logits(m * c->nnue2score / c->in_scaling, target);
        } else {
            float p;
            if (c->loss_kind == 0) {
                p = sig(m * model_inv);
            } else {
                float sc = m * c->nnue2score;
                float q = (sc - c->in_offset) / c->in_scaling;
                float qm = (-sc - c->in_offset) / c->in_scaling;
                p = 0.5f * (1.0f + sig(q) - sig(qm));
            }
            l = powf(fabsf(p - target), c->pow_exp);
        }
        sum += (double)l;
    }
    *loss_sum = sum;
}
