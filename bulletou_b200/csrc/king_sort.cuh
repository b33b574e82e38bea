// Stable counting sort of half-positions by king.
//
// A half-position is h = 2*sample + perspective.  Its key is the king block of
// its first valid feature, feature / piece (HalfKP: 1548 pieces per king,
// HalfKA_hm2 / HalfKA2: 1629), clamped to KEYS-1; a perspective with no valid
// feature gets the last key.  Every feature of a half-position lies in its
// king's block of rows, so processing half-positions in key order keeps the
// feature-transformer rows in use at any moment to a few kings' worth, which
// L2 holds.  The reference sorts SFNN samples the same way for its 2304-wide
// FT path (sfnn_hm2_king_key / sort_count / prefix / scatter, cu:1196-1225),
// with atomics; this sort is deterministic: per-block key histograms,
// per-key bases over blocks, and an ordered scatter (within a key, h ascending).
#pragma once

#include "common.cuh"

namespace bou {

constexpr int kKingSortThreads = 256;
constexpr int kKingSortWarps = kKingSortThreads / 32;

struct KingKey {
    int piece;  // rows per king block
    int limit;  // features in [0, limit) are valid
    int max_active;
};

template <int KEYS>
__device__ __forceinline__ int king_key_of(const int* __restrict__ stm, const int* __restrict__ nstm, int h,
                                           KingKey k) {
    const int* idx = ((h & 1) ? nstm : stm) + static_cast<size_t>(h >> 1) * k.max_active;
    for (int s = 0; s < k.max_active; ++s) {
        const int f = __ldg(idx + s);
        if (f >= 0 && f < k.limit) return min(f / k.piece, KEYS - 1);
    }
    return KEYS - 1;
}

template <int KEYS>
__global__ void __launch_bounds__(kKingSortThreads) king_hist_kernel(const int* __restrict__ stm,
                                                                     const int* __restrict__ nstm, int n_half,
                                                                     KingKey kk, int* __restrict__ keys,
                                                                     int* __restrict__ block_hist) {
    __shared__ int hist[KEYS];
    for (int i = threadIdx.x; i < KEYS; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    const int h = blockIdx.x * kKingSortThreads + threadIdx.x;
    if (h < n_half) {
        const int key = king_key_of<KEYS>(stm, nstm, h, kk);
        keys[h] = key;
        atomicAdd(&hist[key], 1);  // counts only: order-independent
    }
    __syncthreads();
    for (int i = threadIdx.x; i < KEYS; i += blockDim.x) block_hist[blockIdx.x * KEYS + i] = hist[i];
}

// One CTA: key_off[k] = first slot of key k (key_off[KEYS] = n_half); block_hist
// becomes, per (block, key), the first slot of that block's items of that key.
template <int KEYS>
__global__ void __launch_bounds__(128) king_bases_kernel(int* __restrict__ block_hist, int nblocks,
                                                         int* __restrict__ key_off) {
    static_assert(KEYS <= 128, "one thread per key");
    __shared__ int total[KEYS];
    const int k = threadIdx.x;
    if (k < KEYS) {
        int s = 0;
#pragma unroll 8
        for (int b = 0; b < nblocks; ++b) s += block_hist[b * KEYS + k];
        total[k] = s;
    }
    __syncthreads();
    if (k == 0) {
        int run = 0;
        for (int i = 0; i < KEYS; ++i) {
            const int t = total[i];
            total[i] = run;
            run += t;
        }
        key_off[KEYS] = run;
    }
    __syncthreads();
    if (k < KEYS) {
        int run = total[k];
        key_off[k] = run;
#pragma unroll 8
        for (int b = 0; b < nblocks; ++b) {
            const int c = block_hist[b * KEYS + k];
            block_hist[b * KEYS + k] = run;
            run += c;
        }
    }
}

// order[pos] = h; rank (optional) is the inverse permutation, rank[h] = pos.
template <int KEYS>
__global__ void __launch_bounds__(kKingSortThreads) king_scatter_kernel(const int* __restrict__ keys, int n_half,
                                                                        const int* __restrict__ block_base,
                                                                        int* __restrict__ order,
                                                                        int* __restrict__ rank) {
    __shared__ int wcount[kKingSortWarps][KEYS];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int i = threadIdx.x; i < kKingSortWarps * KEYS; i += blockDim.x) (&wcount[0][0])[i] = 0;
    __syncthreads();
    const int h = blockIdx.x * kKingSortThreads + threadIdx.x;
    const bool valid = h < n_half;
    const int key = valid ? keys[h] : -1;
    const unsigned peers = __match_any_sync(0xffffffffu, key);
    const int r = __popc(peers & ((1u << lane) - 1u));
    if (valid && r == 0) wcount[warp][key] = __popc(peers);
    __syncthreads();
    if (valid) {
        int before = 0;
        for (int w = 0; w < warp; ++w) before += wcount[w][key];
        const int pos = block_base[blockIdx.x * KEYS + key] + before + r;
        order[pos] = h;
        if (rank != nullptr) rank[h] = pos;
    }
}

// Ints of scratch the sort needs for n_half items:
// key_off [KEYS+1] | keys [n_half] | order [n_half] | block_hist [nblocks x KEYS]
template <int KEYS>
constexpr size_t king_sort_scratch_ints(size_t n_half) {
    return (KEYS + 1) + 2 * n_half + ((n_half + kKingSortThreads - 1) / kKingSortThreads) * KEYS;
}

struct KingSortOut {
    int* key_off;  // [KEYS + 1]
    int* order;    // [n_half]
};

// Enqueues the three passes on ctx->stream; `scratch` has
// king_sort_scratch_ints<KEYS>(n_half) ints.  rank may be null.
template <int KEYS>
int king_sort(BulletOuCudaCppContext* ctx, const int* stm, const int* nstm, int n_half, KingKey kk, int* scratch,
              int* rank, KingSortOut* out) {
    const int nblocks = (n_half + kKingSortThreads - 1) / kKingSortThreads;
    int* key_off = scratch;
    int* keys = key_off + KEYS + 1;
    int* order = keys + n_half;
    int* block_hist = order + n_half;
    king_hist_kernel<KEYS><<<nblocks, kKingSortThreads, 0, ctx->stream>>>(stm, nstm, n_half, kk, keys, block_hist);
    king_bases_kernel<KEYS><<<1, 128, 0, ctx->stream>>>(block_hist, nblocks, key_off);
    king_scatter_kernel<KEYS><<<nblocks, kKingSortThreads, 0, ctx->stream>>>(keys, n_half, block_hist, order, rank);
    if (check_launch("king sort launch") != 0) return -1;
    out->key_off = key_off;
    out->order = order;
    return 0;
}

}  // namespace bou
