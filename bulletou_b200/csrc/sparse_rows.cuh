// Inverse index of a sparse batch ("which (sample, perspective) pairs touched
// feature-transformer row r") and the warp-per-row kernels that consume it.
//
// The reference scatters every (sample, slot, column) gradient with a float
// atomicAdd into a dense gradient table (HalfKP, cu:5301-5354), or builds a
// similar count/scan/scatter index for SFNN (cu:4442-4580) and then gathers.
// Here the index feeds one kernel per row that sums the row's pre-activation
// gradients in ascending (sample, perspective) order -- deterministic up to
// kSortCap occurrences per row -- and either applies the optimizer in the
// same pass (the gradient is never written) or writes/accumulates the
// gradient row.
#pragma once

#include <climits>

#include "common.cuh"
#include "optim.cuh"

namespace bou {

constexpr int kRowWarps = 8;         // warps per CTA in the row kernels
constexpr int kSortCap = 512;        // per-warp SMEM sort capacity (entries)
constexpr int kRowChunk = 64;        // rows per CTA in the row kernels
constexpr int kChunkEntryCap = 4096; // entries of a chunk staged in SMEM (else read from global)

// Row ids touched by one sparse feature id.  HalfKP factorization (input_size
// == 125388 + 1548): feature f < 125388 maps to rows 1548+f and f % 1548,
// cu:1004-1019; every other valid id maps to itself.
struct RowMap {
    int input_size;
    int factorized;  // 1 when input_size == 126936
    __device__ __forceinline__ int rows(int f, int* r0, int* r1) const {
        if (f < 0 || f >= input_size) return 0;
        if (factorized && f < 125388) {
            *r0 = 1548 + f;
            *r1 = f % 1548;
            return 2;
        }
        *r0 = f;
        return 1;
    }
};

inline RowMap make_row_map(size_t input_size) {
    RowMap m;
    m.input_size = static_cast<int>(input_size);
    m.factorized = input_size == 125388 + 1548 ? 1 : 0;
    return m;
}

struct InverseIndex {
    int* offsets = nullptr;   // [n_rows + 1]
    int* entries = nullptr;   // [n_entries] entry id = 2*sample + perspective
    int* counts = nullptr;    // [n_rows + 1] scratch
    int n_rows = 0;
    size_t capacity = 0;
};

// Builds the index for `batch` samples x `max_active` slots x 2 perspectives
// into context scratch.  Enqueued on ctx->stream.  Entry ids are
// h = 2*sample + perspective, or entry_rank[h] when entry_rank is given (the
// position of h in a permuted layout of the gradient rows).
int build_inverse_index(BulletOuCudaCppContext* ctx, const int* stm, const int* nstm, size_t batch,
                        size_t max_active, size_t input_size, size_t n_rows, InverseIndex* out,
                        const int* entry_rank = nullptr);

// Tile-keyed index of a king-ordered layout (SFNN): the entry ids are ranks in
// the king-sorted half-position order, king block k owning the ranks
// [rank_base[k], rank_base[k + 1]).  A king block's ranks are cut into tiles
// of tile_ranks; key = tile * pieces + piece, where tile = tile_base[k] + the
// tile of the entry's rank (clamped into the king's tiles).  A row (k, p) is
// the union of the keys t * pieces + p for t in [tile_base[k], tile_base[k+1]).
struct RowTiles {
    const int* tile_base;  // [kings + 1], device
    const int* rank_base;  // [kings + 1], device
    int pieces;
    int kings;
    int tile_ranks;
    int max_tiles;         // host bound of tile_base[kings]
};

// Builds the tile-keyed index (n_rows = max_tiles * pieces keys); features
// outside [0, kings * pieces) are skipped.  entry_rank must be given.
int build_inverse_index_tiled(BulletOuCudaCppContext* ctx, const int* stm, const int* nstm, size_t batch,
                              size_t max_active, const RowTiles& tiles, InverseIndex* out, const int* entry_rank);

// Deterministic exclusive scan of counts[0, n) into offsets[0, n] (offsets[n]
// = total) on ctx->stream; tile_sums needs scan_tiles(n) + 1 ints.
inline int scan_tiles(int n) { return (n + 4 * 1024 - 1) / (4 * 1024); }
int exclusive_scan_counts(BulletOuCudaCppContext* ctx, const int* counts, int n, int* offsets, int* tile_sums);

// Sorts every row's entry list ascending in place (rows with more than
// kSortCap entries are left in fill order), so that consumers can sum a row in
// a fixed order without sorting it themselves.  Rows with more than
// `skip_above` entries are left unsorted too (their consumer does not read the
// entry list: the tensor-core heavy keys of the SFNN FT rows).
int sort_inverse_index(BulletOuCudaCppContext* ctx, const InverseIndex& index, int skip_above = 0x7fffffff);

// Same, for a plain table: every feature id in [0, n_features) is its own row.
int build_inverse_index_rows(BulletOuCudaCppContext* ctx, const int* stm, const int* nstm, size_t batch,
                             size_t max_active, size_t n_features, InverseIndex* out, const int* entry_rank);

// Parameters of the per-row consumer kernels.
struct RowGradientSource {
    const float* base[2];  // perspective 0 / 1 pre-activation gradients
    size_t sample_stride;  // floats between consecutive samples in base[p]
};

enum RowMode : int {
    kRowRanger = 0,       // sum + Ranger update (gradient never materialised)
    kRowWrite = 1,        // gradient row overwritten with the sum
    kRowAccumulate = 2,   // gradient row += sum
};

struct RowKernelArgs {
    const int* offsets;
    const int* entries;
    int n_rows;
    int row_begin;  // first row handled (for row-sharded updates)
    int width;      // floats per row
    RowGradientSource src;
    float* weights;
    float* momentum;
    float* velocity;
    float* slow;
    float* gradients;  // kRowWrite / kRowAccumulate target, row-major [n_rows][width] relative to row_begin
    RangerArgs ranger;
    int skip_quiet;
};

int launch_row_kernel(BulletOuCudaCppContext* ctx, int mode, const RowKernelArgs& args, int rows_to_process);

}  // namespace bou
