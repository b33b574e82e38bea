// Tensor-core sums of the heavy keys of the SFNN FT gradient (ft_rows_mma.cu).
#pragma once

#include <cuda_bf16.h>

#include "common.cuh"

namespace bou {

// Device plan of the heavy keys, filled by launch_heavy_key_mma.
struct HeavyMmaPlan {
    int* key_local;    // [max_tiles * pieces] heavy rank of the key within its tile, -1: light
    int* key_slot;     // [max_tiles * pieces] global slot (row of partials), -1: light
    int* tile_heavy;   // [max_tiles] heavy keys per tile
    int* tile_slot;    // [max_tiles + 1] first slot of each tile; [max_tiles] = slots used
    int* tile_r0;      // [max_tiles] first rank of the tile
    int* tile_r1;      // [max_tiles] end rank of the tile
    int* tile_mb;      // [max_tiles + 1] first M-block of each tile; [max_tiles] = M-blocks used
    int* work;         // [2 * max_work] tile, (first M-block << 16) | (M-blocks << 8) | column group
    int* n_work;       // device scalar
    int* n_slots;      // device scalar
    int* next_work;    // device scalar: dynamic work counter of the MMA kernel
    int* error;        // sticky: a bounded wait timed out
    float* partials;   // [max_slots][width] sums of the heavy keys
    void* incidence;   // [max_mblocks][64 chunks][16 KB] 0/1 key x rank operand, bf16, MMA layout
    int max_slots;
    int max_mblocks;
    int max_work;
};

struct HeavyMmaArgs {
    HeavyMmaPlan plan;
    // tile-keyed index (key = tile * pieces + piece) and the tiles of each king block
    const int* offsets;    // [max_tiles * pieces + 1]
    const int* tile_base;  // [kings + 1]
    const int* rank_base;  // [kings + 1] first rank of each king block (king sort offsets)
    int rank_base_end;     // end rank when kings == 1
    int kings;
    int pieces;
    int tile_ranks;
    int max_tiles;
    int threshold;         // keys with more entries are heavy
    // the batch: rank -> half-position, its feature rows
    const int* order;
    const int* stm;
    const int* nstm;
    int max_active;
    // the pre-activation gradient rows in king order as bf16 planes, G = hi + lo
    const __nv_bfloat16* hi;
    const __nv_bfloat16* lo;
    int rows;              // ranks (2 * batch)
    int width;
};

constexpr int kHeavyMmaThreshold = 64;  // entries of a key in its 4096-rank tile

bool heavy_mma_supported(int width);
size_t heavy_mma_max_slots(size_t entries, int threshold);
size_t heavy_mma_max_mblocks(int max_tiles, size_t max_slots);
size_t heavy_mma_max_work(int max_tiles, size_t max_slots, int width);
size_t heavy_mma_incidence_bytes(size_t max_mblocks);
// Plans the heavy keys and sums them on the tensor cores into plan.partials.
int launch_heavy_key_mma(BulletOuCudaCppContext* ctx, HeavyMmaArgs a);

}  // namespace bou
