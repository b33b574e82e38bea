// Teacher-batch producer on the device: YaneuraOu PackedSfenValue records
// (40 bytes) -> the sparse batch the train steps consume (stm / nstm feature
// indices padded with -1, LayerStack bucket, blended target, entry weight).
//
// The reference builds these batches on the host with rayon
// (prepare_sfnn_fast_batch_from_board_features, crates/bulletou_lib/src/value/
// teacher_batch.rs:2869-3010; prepare_halfkp_direct_fast_batch, :1687-1750)
// from ShogiBoard::from_packed_sfen (crates/bulletou_lib/src/shogi/
// packed_sfen.rs:228-284) and the feature maps of shogi_halfka_hm2.rs:106-258 /
// shogi_halfkp.rs:161-227.  Here one thread owns one record:
//   * the block stages its records (coalesced 32-bit loads) in shared memory
//     and each thread reads its own 256-bit Huffman stream through a 64-bit
//     window; one 8-bit peek plus a 256-entry table resolves a board or hand
//     piece code with its promotion / colour bits,
//   * HalfKA_hm2 wants board features grouped by (piece type, colour) in the
//     reference's BOARD_PIECE_TYPES order and by square inside a group, so
//     the decode pass keeps the board in shared memory and counts each group;
//     an exclusive prefix over the 26 groups then gives every piece its slot
//     (a counting sort per record), HalfKP emits in square order directly,
//   * feature rows are assembled in shared memory and written back as one
//     contiguous [records x max_active] block per CTA.
// Bit-exact with the reference for every bit pattern: reads past bit 256 are
// zero (the reference's reader then parks its cursor at 256, this one runs on;
// both end the hand loop there), hand counts and squares keep the reference's
// u8 arithmetic.  A record with more features than max_active is
// counted in `overflow` (the reference aborts on it).
#include <cuda_runtime.h>

#include <climits>
#include <cstdint>

#include "common.cuh"
#include "sparse_rows.cuh"

namespace bou {
namespace {

constexpr int kTeacherThreads = 64;
constexpr int kTeacherMaxActive = 48;
constexpr int kRowStride = kTeacherMaxActive + 1;   // odd: per-thread rows hit distinct banks
constexpr int kRecordWords = 10;
constexpr int kRecordStride = 11;

enum : int { PT_NONE = 0, PAWN, LANCE, KNIGHT, SILVER, BISHOP, ROOK, GOLD, KING, PRO_PAWN, PRO_LANCE, PRO_KNIGHT,
             PRO_SILVER, HORSE, DRAGON };

// Huffman codes, LSB first (packed_sfen.rs:17-26); index 7 is gold (no
// promotion bit).  Board codes use (pattern, len); hand codes drop bit 0.
__constant__ uint8_t kHuffPattern[8] = {0x00, 0x01, 0x03, 0x0b, 0x07, 0x1f, 0x3f, 0x0f};
__constant__ uint8_t kHuffLen[8] = {1, 2, 4, 4, 4, 6, 6, 5};
__constant__ uint8_t kHuffType[8] = {PT_NONE, PAWN, LANCE, KNIGHT, SILVER, BISHOP, ROOK, GOLD};
// BonaPiece bases [piece type][is_friend] (bona_piece.rs:92-124).
__constant__ int16_t kPieceBase[15][2] = {
    {0, 0}, {171, 90}, {333, 252}, {495, 414}, {657, 576}, {981, 900}, {1305, 1224}, {819, 738}, {0, 0},
    {819, 738}, {819, 738}, {819, 738}, {819, 738}, {1143, 1062}, {1467, 1386}};
// Hand bases [pawn..rook in HAND_PIECE_TYPES order][is_friend] (bona_piece.rs:38-57).
__constant__ int16_t kHandBase[7][2] = {{20, 1}, {44, 39}, {54, 49}, {64, 59}, {74, 69}, {82, 79}, {88, 85}};
// Position of a piece type in BOARD_PIECE_TYPES (types.rs:383-397); -1 for none / king.
__constant__ int8_t kBoardOrder[15] = {-1, 0, 1, 2, 3, 5, 6, 4, -1, 7, 8, 9, 10, 11, 12};
// Hand slot of an unpromoted type (Hand::piece_index, types.rs:256-267).
__constant__ int8_t kHandSlot[8] = {-1, 0, 1, 2, 3, 5, 6, 4};
// Unpromoted type of each hand slot (HAND_PIECE_TYPES, types.rs:371-379).
__constant__ int8_t kHandType[7] = {PAWN, LANCE, KNIGHT, SILVER, GOLD, BISHOP, ROOK};
__constant__ int16_t kKingCount[8] = {1, 9, 81, 81, 169, 441, 441, 841};
__constant__ int8_t kHandAxis[7] = {1, 2, 4, 8, 8, 16, 32};

constexpr int kFeHandEnd = 90;
constexpr int kFKing = 1548;
constexpr int kEKing = 1629;
constexpr int kFeEnd = 1548;
constexpr int kHm2PieceInputs = 1629;

struct TeacherArgs {
    const uint32_t* records;
    int64_t n;
    const float* wrm_table;
    int32_t* stm;
    int32_t* nstm;
    int32_t* buckets;
    float* targets;
    float* weights;
    int* overflow;
    int feature_set;
    int max_active;
    int hand_kind;
    int king_kind;
    float result_blend;
    float score_blend;
    float rscale;
    int score_drop_abs;
};

struct TeacherShared {
    uint32_t rec[kTeacherThreads * kRecordStride];
    int32_t out_stm[kTeacherThreads * kRowStride];
    int32_t out_nstm[kTeacherThreads * kRowStride];
    uint8_t board[81][kTeacherThreads];     // type | colour << 4, per thread column
    uint8_t groups[26][kTeacherThreads];    // counts, then running slots
    uint8_t board_code[256];                // idx | len << 4 for the next 8 stream bits
    uint8_t hand_code[256];
};

// LSB-first reader over one record's 8 stream words in shared memory.
struct BitReader {
    const uint32_t* words;
    uint64_t buf;
    int avail;
    int next;
    int cursor;

    __device__ void refill() {
        const uint32_t w = next < 8 ? words[next] : 0u;   // past bit 256 reads as zero
        buf |= static_cast<uint64_t>(w) << avail;
        avail += 32;
        ++next;
    }
    __device__ uint32_t peek8() {
        if (avail < 8) refill();
        return static_cast<uint32_t>(buf & 0xffu);
    }
    __device__ void consume(int k) {
        buf >>= k;
        avail -= k;
        cursor += k;
    }
};

__device__ __forceinline__ int promote_type(int pt) {
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

__device__ __forceinline__ int unpromote_type(int pt) {
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

// Board piece at the reader: returns type | colour << 4 (0 for an empty square).
__device__ __forceinline__ int read_board_piece(BitReader& r, const uint8_t* table) {
    const uint32_t bits = r.peek8();
    const int e = table[bits];
    if (e == 0xff) {        // unreachable: the board code is complete over 8 bits
        r.consume(8);
        return 0;
    }
    const int idx = e & 15, len = e >> 4;
    if (idx == 0) {
        r.consume(len);
        return 0;
    }
    const uint32_t rest = bits >> len;
    int promoted = 0, color;
    if (idx != 7) {
        promoted = rest & 1u;
        color = (rest >> 1) & 1u;
        r.consume(len + 2);
    } else {
        color = rest & 1u;
        r.consume(len + 1);
    }
    const int base = kHuffType[idx];
    return (promoted ? promote_type(base) : base) | (color << 4);
}

// Hand piece at the reader: returns hand slot | colour << 3, or -1 for a piece-box piece.
__device__ __forceinline__ int read_hand_piece(BitReader& r, const uint8_t* table) {
    const uint32_t bits = r.peek8();
    const int e = table[bits];
    if (e == 0xff) {        // unreachable: the hand code is complete over 8 bits
        r.consume(8);
        return -1;
    }
    const int idx = e & 15, len = e >> 4;
    const uint32_t rest = bits >> len;
    int box = 0, color;
    if (idx != 7) {
        box = rest & 1u;
        color = (rest >> 1) & 1u;
        r.consume(len + 2);
    } else {
        color = rest & 1u;
        r.consume(len + 1);
    }
    return box ? -1 : (kHandSlot[idx] | (color << 3));
}

__device__ __forceinline__ int mirror_file(int sq) {
    const int file = sq / 9;
    return (8 - file) * 9 + (sq - file * 9);
}

// halfka_hm2_index (shogi_halfka_hm2.rs:106-133).
__device__ __forceinline__ int32_t hm2_index(int king, int bp) {
    if (king >= 45) {   // file >= 5
        king = mirror_file(king);
        if (bp >= kFeHandEnd) {
            const int off = bp - kFeHandEnd;
            const int piece = off / 81;
            bp = kFeHandEnd + piece * 81 + mirror_file(off - piece * 81);
        }
    }
    if (bp >= kEKing) bp -= 81;
    return king * kHm2PieceInputs + bp;
}

__device__ __forceinline__ int imin(int a, int b) { return a < b ? a : b; }

__device__ int king_single(int kind, int sq) {
    const int rank = imin(sq % 9, 8), file = imin(sq / 9, 8);
    switch (kind) {
        case 3:
            if (rank < 3) return 0;
            if (rank < 6) return 1;
            if (rank == 6) return 2;
            return 3 + (rank - 7) * 3 + file / 3;
        case 4: return rank < 7 ? rank : 7 + (rank - 7) * 3 + file / 3;
        case 5:
        case 6:
            if (rank < 3) return 0;
            if (rank < 6) return 1;
            if (rank < 7) return 2;
            return 3 + (rank - 7) * 9 + file;
        case 7:
            if (rank < 3) return 0;
            if (rank < 6) return 1;
            return 2 + (rank - 6) * 9 + file;
        default: return 0;
    }
}

// ShogiSfnnKingBucketKind::bucket_from_perspective_squares (outputs.rs:955-975).
__device__ int king_bucket(int kind, int f_sq, int e_sq) {
    const int fr = imin(f_sq % 9, 8), er = imin(e_sq % 9, 8);
    switch (kind) {
        case 1: return (fr / 3) * 3 + er / 3;
        case 2: return fr * 9 + er;
        case 3: return king_single(3, f_sq) * 9 + king_single(3, e_sq);
        case 4: return king_single(4, f_sq) * 13 + king_single(4, e_sq);
        case 5:
        case 6: return king_single(5, f_sq) * 21 + king_single(5, e_sq);
        case 7: return king_single(7, f_sq) * 29 + king_single(7, e_sq);
        default: return 0;
    }
}

// shogi_hand*_single_bucket (outputs.rs:318-420); u8 sums as written there.
__device__ int hand_single(int kind, const int* h) {
    const int pawn = h[0], lance = h[1], knight = h[2], silver = h[3], gold = h[4], bishop = h[5], rook = h[6];
    auto u8 = [](int v) { return v & 0xff; };
    int b = 0;
    switch (kind) {
        case 1: return bishop > 0;
        case 2: return (pawn > 0 ? 1 : 0) | (bishop > 0 ? 2 : 0);
        case 3:
            if (u8(pawn + lance + knight) > 0) b |= 1;
            if (u8(gold + silver + rook) > 0) b |= 2;
            if (bishop > 0) b |= 4;
            return b;
        case 4: {
            const int score = pawn + u8(lance + knight) * 2 + u8(silver + gold) * 3 + u8(bishop + rook) * 5;
            return imin((score + 3) / 4, 7);
        }
        case 5:
            if (u8(pawn + lance + knight) > 0) b |= 1;
            if (u8(silver + gold) > 0) b |= 2;
            if (bishop > 0) b |= 4;
            if (rook > 0) b |= 8;
            return b;
        case 6:
            if (pawn > 0) b |= 1;
            if (u8(lance + knight) > 0) b |= 2;
            if (u8(silver + gold) > 0) b |= 4;
            if (bishop > 0) b |= 8;
            if (rook > 0) b |= 16;
            return b;
        default: return 0;
    }
}

__device__ __forceinline__ void put(int32_t* row_s, int32_t* row_n, int& count, int cap, int32_t s, int32_t n) {
    if (count < cap) {
        row_s[count] = s;
        row_n[count] = n;
    }
    ++count;
}

__global__ void __launch_bounds__(kTeacherThreads) teacher_psv_kernel(TeacherArgs a) {
    __shared__ TeacherShared sh;
    const int t = threadIdx.x;
    const int64_t first = static_cast<int64_t>(blockIdx.x) * kTeacherThreads;
    const int here = static_cast<int>(a.n - first < kTeacherThreads ? a.n - first : kTeacherThreads);

    // Decode tables: the first code that the next 8 stream bits start with.
    for (int v = t; v < 256; v += kTeacherThreads) {
        uint8_t board = 0xff, hand = 0xff;
        for (int idx = 0; idx < 8; ++idx) {
            const int len = kHuffLen[idx];
            if ((v & ((1 << len) - 1)) == kHuffPattern[idx]) board = static_cast<uint8_t>(idx | (len << 4));
            if (idx > 0 && (v & ((1 << (len - 1)) - 1)) == (kHuffPattern[idx] >> 1))
                hand = static_cast<uint8_t>(idx | ((len - 1) << 4));
        }
        sh.board_code[v] = board;
        sh.hand_code[v] = hand;
    }
    // Stage the block's records (40 bytes = 10 words each, contiguous).
    const uint32_t* src = a.records + first * kRecordWords;
    for (int w = t; w < here * kRecordWords; w += kTeacherThreads) {
        const int r = w / kRecordWords;
        sh.rec[r * kRecordStride + (w - r * kRecordWords)] = src[w];
    }
    __syncthreads();

    const int A = a.max_active;
    int32_t* row_s = sh.out_stm + t * kRowStride;
    int32_t* row_n = sh.out_nstm + t * kRowStride;
    if (t < here) {
        const uint32_t* rec = sh.rec + t * kRecordStride;
        BitReader r{rec, 0ull, 0, 0, 0};
        const int stm = static_cast<int>(r.peek8() & 1u);
        r.consume(1);
        uint32_t kings = r.peek8();
        r.consume(7);
        const int bk = static_cast<int>(kings & 127u);
        kings = r.peek8();
        r.consume(7);
        const int wk = static_cast<int>(kings & 127u);
        const int sk = stm ? wk : bk, nk = stm ? bk : wk;
        const bool kings_ok = sk < 81 && nk < 81;
        const int stm_ksq = stm ? 80 - sk : sk;        // own king seen from each side
        const int nstm_ksq = stm ? nk : 80 - nk;
        int count = 0;
        int hands[14];
#pragma unroll
        for (int i = 0; i < 14; ++i) hands[i] = 0;

        if (a.feature_set == 0) {
            // HalfKA_hm2: decode the board, count the 26 (type, colour) groups.
#pragma unroll
            for (int g = 0; g < 26; ++g) sh.groups[g][t] = 0;
            for (int sq = 0; sq < 81; ++sq) {
                int code = 0;
                if (sq != bk && sq != wk) code = read_board_piece(r, sh.board_code);
                sh.board[sq][t] = static_cast<uint8_t>(code);
                if (code != 0) {
                    const int g = kBoardOrder[code & 15] * 2 + (code >> 4);
                    sh.groups[g][t] = static_cast<uint8_t>(sh.groups[g][t] + 1);
                }
            }
            while (r.cursor < 256) {
                const int h = read_hand_piece(r, sh.hand_code);
                if (h >= 0) {
                    const int i = (h >> 3) * 7 + (h & 7);
                    hands[i] = (hands[i] + 1) & 0xff;
                }
            }
            if (kings_ok) {
                int total = 0;
                for (int g = 0; g < 26; ++g) {
                    const int c = sh.groups[g][t];
                    sh.groups[g][t] = static_cast<uint8_t>(total);
                    total += c;
                }
                // board pieces never exceed 79, so the slots fit in a byte
                for (int sq = 0; sq < 81; ++sq) {
                    const int code = sh.board[sq][t];
                    if (code == 0) continue;
                    const int pt = code & 15, color = code >> 4;
                    const int g = kBoardOrder[pt] * 2 + color;
                    const int slot = sh.groups[g][t];
                    sh.groups[g][t] = static_cast<uint8_t>(slot + 1);
                    const int s_sq = stm ? 80 - sq : sq;
                    const int sbp = kPieceBase[pt][color == stm] + s_sq;
                    const int nbp = kPieceBase[pt][color != stm] + (80 - s_sq);
                    if (slot < A) {
                        row_s[slot] = hm2_index(stm_ksq, sbp);
                        row_n[slot] = hm2_index(nstm_ksq, nbp);
                    }
                }
                count = total;
                put(row_s, row_n, count, A, hm2_index(stm_ksq, kFKing + stm_ksq),
                    hm2_index(nstm_ksq, kFKing + nstm_ksq));
                put(row_s, row_n, count, A, hm2_index(stm_ksq, kEKing + (stm ? 80 - nk : nk)),
                    hm2_index(nstm_ksq, kEKing + (stm ? sk : 80 - sk)));
                for (int owner = 0; owner < 2; ++owner) {
                    for (int h = 0; h < 7; ++h) {
                        const int c = hands[owner * 7 + h];
                        const int sb = kHandBase[h][owner == stm], nb = kHandBase[h][owner != stm];
                        for (int i = 0; i < c; ++i)
                            put(row_s, row_n, count, A, hm2_index(stm_ksq, sb + i), hm2_index(nstm_ksq, nb + i));
                    }
                }
            }
        } else if (kings_ok) {
            // HalfKP (map_halfkp_features_from_packed): square order, no kings.
            for (int sq = 0; sq < 81; ++sq) {
                if (sq == bk || sq == wk) continue;
                const int code = read_board_piece(r, sh.board_code);
                if (code == 0) continue;
                const int pt = code & 15, color = code >> 4;
                const int s_sq = stm ? 80 - sq : sq;
                put(row_s, row_n, count, A, stm_ksq * kFeEnd + kPieceBase[pt][color == stm] + s_sq,
                    nstm_ksq * kFeEnd + kPieceBase[pt][color != stm] + (80 - s_sq));
            }
            while (r.cursor < 256) {
                const int h = read_hand_piece(r, sh.hand_code);
                if (h >= 0) {
                    const int i = (h >> 3) * 7 + (h & 7);
                    hands[i] = imin(hands[i] + 1, 255);                 // saturating_add
                }
            }
            for (int owner = 0; owner < 2; ++owner) {
                for (int h = 0; h < 7; ++h) {
                    const int c = hands[owner * 7 + h];
                    const int sb = kHandBase[h][owner == stm], nb = kHandBase[h][owner != stm];
                    for (int i = 0; i < c; ++i)
                        put(row_s, row_n, count, A, stm_ksq * kFeEnd + sb + i, nstm_ksq * kFeEnd + nb + i);
                }
            }
        }
        for (int k = count; k < A; ++k) {
            row_s[k] = -1;
            row_n[k] = -1;
        }
        if (count > A) atomicAdd(a.overflow, 1);

        const int64_t i = first + t;
        if (a.buckets != nullptr) {
            int bucket = 0;
            if (a.feature_set == 0) {
                const int* own = hands + stm * 7;
                const int* opp = hands + (1 - stm) * 7;
                const int hb = a.hand_kind == 0
                                   ? 0
                                   : hand_single(a.hand_kind, own) * kHandAxis[a.hand_kind] +
                                         hand_single(a.hand_kind, opp);
                // perspective squares; Square::inverse wraps as a u8 for king-less records
                const int f_sq = stm ? ((80 - sk) & 0xff) : sk;
                const int e_sq = stm ? nk : ((80 - nk) & 0xff);
                bucket = hb * kKingCount[a.king_kind] + king_bucket(a.king_kind, f_sq, e_sq);
            }
            a.buckets[i] = bucket;
        }
        const int score = static_cast<int16_t>(rec[8] & 0xffffu);
        const int result = static_cast<int8_t>((rec[9] >> 16) & 0xffu);
        float w = 1.0f;
        if (a.score_drop_abs >= 0 && (score < 0 ? -score : score) >= a.score_drop_abs) w = 0.0f;
        a.weights[i] = w;
        float sp;
        if (a.wrm_table != nullptr) {
            sp = __ldg(a.wrm_table + (score + 32768));
        } else {
            // 1 / (1 + exp(-(rscale * score))) in f32; exp evaluated in double and
            // rounded once, the f32 operations kept unfused.
            const float x = -__fmul_rn(a.rscale, static_cast<float>(score));
            const float e = static_cast<float>(exp(static_cast<double>(x)));
            sp = __fdiv_rn(1.0f, __fadd_rn(1.0f, e));
        }
        const float res = result > 0 ? 1.0f : (result < 0 ? 0.0f : 0.5f);
        a.targets[i] = __fadd_rn(__fmul_rn(a.result_blend, res), __fmul_rn(a.score_blend, sp));
    }
    __syncthreads();
    // Contiguous write-back of the block's feature rows.
    int32_t* gs = a.stm + first * A;
    int32_t* gn = a.nstm + first * A;
    for (int e = t; e < here * A; e += kTeacherThreads) {
        const int row = e / A, col = e - row * A;
        gs[e] = sh.out_stm[row * kRowStride + col];
        gn[e] = sh.out_nstm[row * kRowStride + col];
    }
}


// ------------------------------------------------------------------ HCPE records
// decode_hcpe_record (crates/bulletou_lib/src/value/loader/hcpe.rs:65-76):
// Apery / cshogi HuffmanCodedPos (MiniPosition::from_hcp, loader/shogipack.rs:
// 353-408: knight / silver codes swapped against the PackedSfen table, colour
// bit before the promotion bit, hands and piece box in one 3/5/7-bit prefix
// code) re-packed as a PackedSfenValue (pack_to_psfen, :477-554; game_ply 0;
// the game result turned to the side to move, convert_game_result :679-697).
// A record with a king square >= 81 or an unknown hand code is invalid: the
// reference's loader skips it, here it is dropped from the compacted output.
constexpr int kHcpeBytes = 38;
constexpr int kHcpeStride = 11;   // words per staged record (44 bytes, odd stride)

__constant__ uint8_t kHcpPattern[8] = {0x00, 0x01, 0x03, 0x07, 0x0b, 0x1f, 0x3f, 0x0f};
// {code, bits, piece type, colour (2: piece box)} (shogipack.rs:81-105)
__constant__ uint8_t kHcpHand[21][4] = {
    {0x00, 3, PAWN, 0},   {0x01, 5, LANCE, 0},  {0x03, 5, KNIGHT, 0}, {0x05, 5, SILVER, 0}, {0x07, 5, GOLD, 0},
    {0x1f, 7, BISHOP, 0}, {0x3f, 7, ROOK, 0},   {0x04, 3, PAWN, 1},   {0x11, 5, LANCE, 1},  {0x13, 5, KNIGHT, 1},
    {0x15, 5, SILVER, 1}, {0x17, 5, GOLD, 1},   {0x5f, 7, BISHOP, 1}, {0x7f, 7, ROOK, 1},   {0x02, 3, PAWN, 2},
    {0x09, 5, LANCE, 2},  {0x0b, 5, KNIGHT, 2}, {0x0d, 5, SILVER, 2}, {0x1d, 5, GOLD, 2},   {0x0f, 7, BISHOP, 2},
    {0x2f, 7, ROOK, 2}};
// PackedSfen table index of an unpromoted type (piece_type_to_index, shogipack.rs:212-224)
__constant__ int8_t kPsvIndex[8] = {0, 1, 2, 3, 4, 5, 6, 7};

struct HcpeShared {
    uint32_t rec[kTeacherThreads * kHcpeStride];
    uint32_t out[kTeacherThreads * kRecordStride];
    uint8_t board[81][kTeacherThreads];
    uint8_t board_code[256];   // idx | len << 4 of the HCP board code the next 8 bits start with
    uint8_t hand_code[256];    // entry of kHcpHand, 0xff: no code within 7 bits
};

// LSB-first writer that drops bits past 256 (BitWriter, shogipack.rs:150-185).
struct BitWriter32 {
    uint32_t* words;
    uint64_t buf;
    int n;
    int cursor;
    __device__ void put(uint32_t v, int k) {
        if (cursor >= 256) return;
        k = min(k, 256 - cursor);
        buf |= static_cast<uint64_t>(v & ((1u << k) - 1u)) << n;
        n += k;
        cursor += k;
        if (n >= 32) {
            words[(cursor - n) >> 5] = static_cast<uint32_t>(buf);
            buf >>= 32;
            n -= 32;
        }
    }
    __device__ void flush() {
        if (n > 0) words[(cursor - n) >> 5] = static_cast<uint32_t>(buf);
    }
};

__global__ void __launch_bounds__(kTeacherThreads) hcpe_psv_kernel(const uint8_t* __restrict__ hcpe, int64_t n,
                                                                   uint32_t* __restrict__ psv, int* __restrict__ valid) {
    __shared__ HcpeShared sh;
    const int t = threadIdx.x;
    const int64_t first = static_cast<int64_t>(blockIdx.x) * kTeacherThreads;
    const int here = static_cast<int>(n - first < kTeacherThreads ? n - first : kTeacherThreads);
    for (int v = t; v < 256; v += kTeacherThreads) {
        uint8_t board = 0xff, hand = 0xff;
        for (int idx = 0; idx < 8; ++idx) {
            const int len = kHuffLen[idx];   // the HCP board lengths equal the PackedSfen ones
            if ((v & ((1 << len) - 1)) == kHcpPattern[idx]) board = static_cast<uint8_t>(idx | (len << 4));
        }
        for (int e = 0; e < 21; ++e) {
            const int len = kHcpHand[e][1];
            if ((v & ((1 << len) - 1)) == kHcpHand[e][0]) hand = static_cast<uint8_t>(e);
        }
        sh.board_code[v] = board;
        sh.hand_code[v] = hand;
    }
    uint8_t* rb = reinterpret_cast<uint8_t*>(sh.rec);
    const uint8_t* src = hcpe + first * kHcpeBytes;
    for (int b = t; b < here * kHcpeBytes; b += kTeacherThreads) {
        const int r = b / kHcpeBytes;
        rb[r * kHcpeStride * 4 + (b - r * kHcpeBytes)] = src[b];
    }
    __syncthreads();
    int ok = 0;
    uint32_t* out = sh.out + t * kRecordStride;
    if (t < here) {
        const uint32_t* rec = sh.rec + t * kHcpeStride;
        BitReader r{rec, 0ull, 0, 0, 0};
        const int stm = static_cast<int>(r.peek8() & 1u);
        r.consume(1);
        const int bk = static_cast<int>(r.peek8() & 127u);
        r.consume(7);
        const int wk = static_cast<int>(r.peek8() & 127u);
        r.consume(7);
        int hands[14];
#pragma unroll
        for (int i = 0; i < 14; ++i) hands[i] = 0;
        ok = bk < 81 && wk < 81;
        if (ok) {
            for (int sq = 0; sq < 81; ++sq) {
                int code = 0;
                if (sq != bk && sq != wk) {
                    const uint32_t bits = r.peek8();
                    const int e = sh.board_code[bits];
                    const int idx = e & 15, len = e >> 4;
                    if (idx == 0) {
                        r.consume(len);
                    } else {
                        const uint32_t rest = bits >> len;
                        const int color = rest & 1u;
                        int promoted = 0;
                        if (idx != 7) {
                            promoted = (rest >> 1) & 1u;
                            r.consume(len + 2);
                        } else {
                            r.consume(len + 1);
                        }
                        const int base = kHuffType[idx];
                        code = (promoted ? promote_type(base) : base) | (color << 4);
                    }
                }
                sh.board[sq][t] = static_cast<uint8_t>(code);
            }
            while (ok && r.cursor < 256) {
                const int e = sh.hand_code[r.peek8()];
                if (e == 0xff) {
                    ok = 0;
                    break;
                }
                r.consume(kHcpHand[e][1]);
                const int owner = kHcpHand[e][3];
                if (owner < 2) {
                    const int i = owner * 7 + kHandSlot[kHcpHand[e][2] == GOLD ? 7 : kHcpHand[e][2]];
                    hands[i] = (hands[i] + 1) & 0xff;
                }
            }
        }
        if (ok) {
            // pack_to_psfen: a king square is the first square holding that king
            const int kb = bk != wk ? bk : 81, kw = wk;
            BitWriter32 w{out, 0ull, 0, 0};
            w.put(static_cast<uint32_t>(stm), 1);
            w.put(static_cast<uint32_t>(kb), 7);
            w.put(static_cast<uint32_t>(kw), 7);
            for (int sq = 0; sq < 81; ++sq) {
                if (sq == kb || sq == kw) continue;
                const int code = sh.board[sq][t];
                if (code == 0) {
                    w.put(0u, 1);
                    continue;
                }
                const int pt = code & 15, color = code >> 4;
                const int raw = unpromote_type(pt);
                const int idx = kPsvIndex[raw == GOLD ? 7 : raw];
                const int len = kHuffLen[idx];
                uint32_t v = kHuffPattern[idx];
                if (raw != GOLD) {
                    v |= static_cast<uint32_t>(pt != raw) << len;
                    v |= static_cast<uint32_t>(color) << (len + 1);
                    w.put(v, len + 2);
                } else {
                    v |= static_cast<uint32_t>(color) << len;
                    w.put(v, len + 1);
                }
            }
            for (int color = 0; color < 2; ++color) {
                for (int h = 0; h < 7; ++h) {
                    const int pt = kHandType[h];
                    const int idx = kPsvIndex[pt];
                    const int len = kHuffLen[idx] - 1;
                    const uint32_t code = kHuffPattern[idx] >> 1;
                    const uint32_t v = pt != GOLD ? (code | (static_cast<uint32_t>(color) << (len + 1)))
                                                  : (code | (static_cast<uint32_t>(color) << len));
                    const int k = pt != GOLD ? len + 2 : len + 1;
                    for (int c = 0; c < hands[color * 7 + h]; ++c) w.put(v, k);
                }
            }
            while (w.cursor < 256) w.put(0b010u, 3);          // piece-box pawns
            w.flush();
            const uint32_t* rw = rec;
            out[8] = rw[8];                                    // eval, bestMove16
            const int res = static_cast<int>((rw[9] >> 0) & 0xffu);   // byte 36: 0 draw, 1 black, 2 white
            const int r8 = res == 1 ? (stm == 0 ? 1 : -1) : (res == 2 ? (stm == 1 ? 1 : -1) : 0);
            out[9] = static_cast<uint32_t>(static_cast<uint8_t>(static_cast<int8_t>(r8))) << 16;  // ply 0
        }
        if (!ok) {
#pragma unroll
            for (int i = 0; i < kRecordWords; ++i) out[i] = 0u;
        }
        valid[first + t] = ok;
    }
    __syncthreads();
    uint32_t* dst = psv + first * kRecordWords;
    for (int e = t; e < here * kRecordWords; e += kTeacherThreads) {
        const int row = e / kRecordWords;
        dst[e] = sh.out[row * kRecordStride + (e - row * kRecordWords)];
    }
}

// Copies the valid records to their compacted positions (offsets: exclusive
// scan of the valid flags, offsets[n] = the count).
__global__ void hcpe_compact_kernel(const uint32_t* __restrict__ psv_all, const int* __restrict__ valid,
                                    const int* __restrict__ offsets, int64_t n, uint32_t* __restrict__ psv,
                                    int* __restrict__ count) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i == 0) *count = offsets[n];
    if (i >= n * kRecordWords) return;
    const int64_t r = i / kRecordWords;
    if (valid[r]) psv[static_cast<int64_t>(offsets[r]) * kRecordWords + (i - r * kRecordWords)] = psv_all[i];
}

}  // namespace
}  // namespace bou

using namespace bou;

extern "C" {

int bulletou_b200_teacher_prepare_device(BulletOuCudaCppContext* ctx, const BulletOuB200TeacherConfig* config,
                                         const BulletOuCudaCppI32Buffer* records, size_t n_records,
                                         const BulletOuCudaCppF32Buffer* wrm_table,
                                         BulletOuCudaCppI32Buffer* stm_indices, BulletOuCudaCppI32Buffer* nstm_indices,
                                         BulletOuCudaCppI32Buffer* buckets, BulletOuCudaCppF32Buffer* targets,
                                         BulletOuCudaCppF32Buffer* entry_weights, BulletOuCudaCppI32Buffer* overflow) {
    if (config == nullptr) return fail_message("teacher config must not be null");
    const BulletOuB200TeacherConfig& c = *config;
    if (c.feature_set != BULLETOU_B200_FEATURES_HALFKA_HM2 && c.feature_set != BULLETOU_B200_FEATURES_HALFKP)
        return fail_messagef("teacher feature_set %d is not supported", c.feature_set);
    if (c.max_active <= 0 || c.max_active > kTeacherMaxActive)
        return fail_messagef("teacher max_active %d must be in 1..%d", c.max_active, kTeacherMaxActive);
    if (c.hand_bucket < 0 || c.hand_bucket > 6 || c.king_bucket < 0 || c.king_bucket > 7)
        return fail_messagef("teacher bucket kind (hand %d, king %d) is not supported", c.hand_bucket, c.king_bucket);
    if (c.score_drop_abs > 65535) return fail_messagef("teacher score_drop_abs %d exceeds u16", c.score_drop_abs);
    const size_t A = static_cast<size_t>(c.max_active);
    if (validate_i32(ctx, records, n_records * kRecordWords, "teacher records") != 0 ||
        validate_i32(ctx, stm_indices, n_records * A, "teacher stm_indices") != 0 ||
        validate_i32(ctx, nstm_indices, n_records * A, "teacher nstm_indices") != 0 ||
        validate_f32(ctx, targets, n_records, "teacher targets") != 0 ||
        validate_f32(ctx, entry_weights, n_records, "teacher entry_weights") != 0 ||
        validate_i32(ctx, overflow, 1, "teacher overflow") != 0)
        return -1;
    if (buckets != nullptr && validate_i32(ctx, buckets, n_records, "teacher buckets") != 0) return -1;
    if (wrm_table != nullptr && validate_f32(ctx, wrm_table, 65536, "teacher wrm_table") != 0) return -1;
    if (set_device(ctx) != 0) return -1;
    if (n_records == 0) return ok();
    int blocks = 0;
    if (grid_1d(n_records, kTeacherThreads, &blocks, "teacher prepare") != 0) return -1;
    TeacherArgs a{};
    a.records = reinterpret_cast<const uint32_t*>(records->ptr);
    a.n = static_cast<int64_t>(n_records);
    a.wrm_table = wrm_table ? wrm_table->ptr : nullptr;
    a.stm = stm_indices->ptr;
    a.nstm = nstm_indices->ptr;
    a.buckets = buckets ? buckets->ptr : nullptr;
    a.targets = targets->ptr;
    a.weights = entry_weights->ptr;
    a.overflow = overflow->ptr;
    a.feature_set = c.feature_set;
    a.max_active = c.max_active;
    a.hand_kind = c.hand_bucket;
    a.king_kind = c.king_bucket;
    a.result_blend = c.result_blend;
    a.score_blend = c.score_blend;
    a.rscale = c.rscale;
    a.score_drop_abs = c.score_drop_abs;
    teacher_psv_kernel<<<blocks, kTeacherThreads, 0, ctx->stream>>>(a);
    if (check_launch("teacher prepare launch") != 0) return -1;
    return ok();
}

}  // extern "C"

extern "C" {

int bulletou_b200_hcpe_to_psv_device(BulletOuCudaCppContext* ctx, const BulletOuCudaCppI32Buffer* hcpe,
                                     size_t n_records, BulletOuCudaCppI32Buffer* psv, BulletOuCudaCppI32Buffer* count,
                                     BulletOuCudaCppI32Buffer* valid) {
    const size_t in_words = (n_records * kHcpeBytes + 3) / 4;
    if (validate_i32(ctx, hcpe, in_words, "hcpe records") != 0 ||
        validate_i32(ctx, psv, n_records * kRecordWords, "hcpe psv output") != 0 ||
        validate_i32(ctx, count, 1, "hcpe count") != 0)
        return -1;
    if (valid != nullptr && validate_i32(ctx, valid, n_records, "hcpe valid flags") != 0) return -1;
    if (n_records >= static_cast<size_t>(INT_MAX) / kRecordWords) return fail_message("hcpe: too many records");
    if (set_device(ctx) != 0) return -1;
    const int n = static_cast<int>(n_records);
    const size_t tiles = static_cast<size_t>(scan_tiles(n)) + 1;
    const size_t ints = n_records * kRecordWords + 2 * n_records + 1 + tiles + (valid == nullptr ? n_records : 0);
    void* sp = nullptr;
    if (scratch_slot(ctx, kScratchHcpe, ints * sizeof(int), &sp, "cudaMalloc HCPE scratch") != 0) return -1;
    uint32_t* psv_all = static_cast<uint32_t*>(sp);
    int* offsets = reinterpret_cast<int*>(psv_all + n_records * kRecordWords);
    int* tile_sums = offsets + n_records + 1;
    int* flags = valid != nullptr ? valid->ptr : tile_sums + tiles;
    if (n_records == 0) {
        cudaError_t st = cudaMemsetAsync(count->ptr, 0, sizeof(int), ctx->stream);
        return st == cudaSuccess ? ok() : fail("cudaMemsetAsync hcpe count", st);
    }
    int blocks = 0;
    if (grid_1d(n_records, kTeacherThreads, &blocks, "hcpe decode") != 0) return -1;
    hcpe_psv_kernel<<<blocks, kTeacherThreads, 0, ctx->stream>>>(reinterpret_cast<const uint8_t*>(hcpe->ptr),
                                                                 static_cast<int64_t>(n_records), psv_all, flags);
    if (check_launch("hcpe decode launch") != 0) return -1;
    if (exclusive_scan_counts(ctx, flags, n, offsets, tile_sums) != 0) return -1;
    if (grid_1d(n_records * kRecordWords, 256, &blocks, "hcpe compact") != 0) return -1;
    hcpe_compact_kernel<<<blocks, 256, 0, ctx->stream>>>(psv_all, flags, offsets, static_cast<int64_t>(n_records),
                                                         reinterpret_cast<uint32_t*>(psv->ptr), count->ptr);
    if (check_launch("hcpe compact launch") != 0) return -1;
    return ok();
}

}  // extern "C"
