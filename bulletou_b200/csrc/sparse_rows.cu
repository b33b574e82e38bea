// Inverse index build and warp-per-row consumers (see sparse_rows.cuh).
#include <algorithm>

#include "sparse_rows.cuh"

namespace bou {

namespace {

__global__ void count_rows_kernel(const int* __restrict__ stm, const int* __restrict__ nstm, size_t slots,
                                  RowMap map, int* __restrict__ counts) {
    const size_t t = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= 2 * slots) return;
    const int f = t < slots ? stm[t] : nstm[t - slots];
    int r0, r1;
    const int n = map.rows(f, &r0, &r1);
    if (n >= 1) atomicAdd(&counts[r0], 1);
    if (n == 2) atomicAdd(&counts[r1], 1);
}

// Exclusive scan of counts[0, n) into offsets[0, n] in three deterministic
// passes: tile sums (4096 counts per CTA), a scan of the tile sums, and the
// per-tile rescan that adds the tile's offset.
constexpr int kScanThreads = 1024;
constexpr int kScanTile = 4 * kScanThreads;

__device__ __forceinline__ int block_exclusive_scan(int v, int* warp_sums, int* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int incl = v;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const int o = __shfl_up_sync(0xffffffffu, incl, d);
        if (lane >= d) incl += o;
    }
    if (lane == 31) warp_sums[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        int w = warp_sums[lane];
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const int o = __shfl_up_sync(0xffffffffu, w, d);
            if (lane >= d) w += o;
        }
        warp_sums[lane] = w;
    }
    __syncthreads();
    const int excl = (warp > 0 ? warp_sums[warp - 1] : 0) + incl - v;
    *total = warp_sums[31];
    return excl;
}

__global__ void __launch_bounds__(kScanThreads) scan_tile_sums_kernel(const int* __restrict__ counts, int n,
                                                                      int* __restrict__ tile_sums) {
    __shared__ int warp_sums[32];
    const int i0 = blockIdx.x * kScanTile + threadIdx.x * 4;
    int v = 0;
#pragma unroll
    for (int q = 0; q < 4; ++q) v += (i0 + q < n) ? counts[i0 + q] : 0;
    int total = 0;
    block_exclusive_scan(v, warp_sums, &total);
    if (threadIdx.x == 0) tile_sums[blockIdx.x] = total;
}

// One CTA: exclusive scan of the tile sums in place; tile_sums[tiles] = grand total.
__global__ void __launch_bounds__(kScanThreads) scan_tile_offsets_kernel(int* __restrict__ tile_sums, int tiles) {
    __shared__ int warp_sums[32];
    __shared__ int carry_s;
    if (threadIdx.x == 0) carry_s = 0;
    __syncthreads();
    for (int base = 0; base < tiles; base += kScanThreads) {
        const int i = base + threadIdx.x;
        const int v = i < tiles ? tile_sums[i] : 0;
        int total = 0;
        const int excl = block_exclusive_scan(v, warp_sums, &total);
        const int carry = carry_s;
        if (i < tiles) tile_sums[i] = carry + excl;
        __syncthreads();
        if (threadIdx.x == 0) carry_s = carry + total;
        __syncthreads();
    }
    if (threadIdx.x == 0) tile_sums[tiles] = carry_s;
}

__global__ void __launch_bounds__(kScanThreads) scan_apply_kernel(const int* __restrict__ counts, int n,
                                                                  const int* __restrict__ tile_offsets, int tiles,
                                                                  int* __restrict__ offsets) {
    __shared__ int warp_sums[32];
    const int i0 = blockIdx.x * kScanTile + threadIdx.x * 4;
    int v[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) v[q] = (i0 + q < n) ? counts[i0 + q] : 0;
    int total = 0;
    int run = tile_offsets[blockIdx.x] + block_exclusive_scan(v[0] + v[1] + v[2] + v[3], warp_sums, &total);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        if (i0 + q < n) offsets[i0 + q] = run;
        run += v[q];
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) offsets[n] = tile_offsets[tiles];
}

// Scatters entry ids into their rows.  Slots are claimed by decrementing the
// row's count, which leaves every count at zero for the next build (so the
// count array needs no clearing between steps).
__global__ void fill_rows_kernel(const int* __restrict__ stm, const int* __restrict__ nstm, size_t slots,
                                 size_t max_active, RowMap map, const int* __restrict__ offsets,
                                 int* __restrict__ cursor, int* __restrict__ entries,
                                 const int* __restrict__ entry_rank) {
    const size_t t = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= 2 * slots) return;
    const int persp = t < slots ? 0 : 1;
    const size_t s = persp == 0 ? t : t - slots;
    const int f = persp == 0 ? stm[s] : nstm[s];
    const int h = static_cast<int>((s / max_active) * 2 + persp);
    const int entry = entry_rank != nullptr ? entry_rank[h] : h;
    int r0, r1;
    const int n = map.rows(f, &r0, &r1);
    if (n >= 1) entries[offsets[r0] + atomicSub(&cursor[r0], 1) - 1] = entry;
    if (n == 2) entries[offsets[r1] + atomicSub(&cursor[r1], 1) - 1] = entry;
}

__device__ __forceinline__ int warp_sort_ascending(int v, int lane) {
#pragma unroll
    for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll
        for (int j = k >> 1; j > 0; j >>= 1) {
            const int other = __shfl_xor_sync(0xffffffffu, v, j);
            const bool ascending = (lane & k) == 0;
            const bool lower = (lane & j) == 0;
            const int lo = min(v, other), hi = max(v, other);
            v = (lower == ascending) ? lo : hi;
        }
    }
    return v;
}

__device__ void smem_sort_ascending(int* buf, int size, int lane) {
    for (int k = 2; k <= size; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = lane; i < size; i += 32) {
                const int ixj = i ^ j;
                if (ixj > i) {
                    const int a = buf[i], b = buf[ixj];
                    const bool ascending = (i & k) == 0;
                    if ((a > b) == ascending) {
                        buf[i] = b;
                        buf[ixj] = a;
                    }
                }
            }
            __syncwarp();
        }
    }
}

// Warp per row: ascending sort of the row's entry ids in place.
__global__ void __launch_bounds__(kRowWarps * 32) sort_rows_kernel(const int* __restrict__ offsets,
                                                                    int* __restrict__ entries, int n_rows,
                                                                    int skip_above) {
    __shared__ int buf_s[kRowWarps][kSortCap];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int row = blockIdx.x * kRowWarps + warp;
    if (row >= n_rows) return;
    const int beg = offsets[row];
    const int n = offsets[row + 1] - beg;
    int* e = entries + beg;
    if (n <= 1 || n > skip_above) return;
    if (n <= 32) {
        int v = lane < n ? e[lane] : INT_MAX;
        v = warp_sort_ascending(v, lane);
        if (lane < n) e[lane] = v;
    } else if (n <= kSortCap) {
        int size = 64;
        while (size < n) size <<= 1;
        int* buf = buf_s[warp];
        for (int i = lane; i < size; i += 32) buf[i] = i < n ? e[i] : INT_MAX;
        __syncwarp();
        smem_sort_ascending(buf, size, lane);
        for (int i = lane; i < n; i += 32) e[i] = buf[i];
    }
}

template <int VEC>
struct Vec {
    float v[VEC];
};

template <int VEC>
__device__ __forceinline__ void load_vec(const float* p, float* out) {
    if constexpr (VEC == 8) {  // columns [c, c+4) and [c+128, c+132): see lane_col
        const float4 a = *reinterpret_cast<const float4*>(p);
        const float4 b = *reinterpret_cast<const float4*>(p + 128);
        out[0] = a.x; out[1] = a.y; out[2] = a.z; out[3] = a.w;
        out[4] = b.x; out[5] = b.y; out[6] = b.z; out[7] = b.w;
    } else if constexpr (VEC == 4) {
        const float4 a = *reinterpret_cast<const float4*>(p);
        out[0] = a.x; out[1] = a.y; out[2] = a.z; out[3] = a.w;
    } else {
#pragma unroll
        for (int i = 0; i < VEC; ++i) out[i] = p[i];
    }
}

template <int VEC>
__device__ __forceinline__ void store_vec(float* p, const float* in) {
    if constexpr (VEC == 8) {
        *reinterpret_cast<float4*>(p) = make_float4(in[0], in[1], in[2], in[3]);
        *reinterpret_cast<float4*>(p + 128) = make_float4(in[4], in[5], in[6], in[7]);
    } else if constexpr (VEC == 4) {
        *reinterpret_cast<float4*>(p) = make_float4(in[0], in[1], in[2], in[3]);
    } else {
#pragma unroll
        for (int i = 0; i < VEC; ++i) p[i] = in[i];
    }
}

// One CTA per chunk of kRowChunk consecutive rows.  The chunk's offsets and
// its (contiguous) entry range are first copied into shared memory with
// coalesced loads, so the only global reads left per row are the independent
// gradient-row gathers (L2) and the optimizer-state rows (HBM).
template <int VEC, int MODE>
__global__ void __launch_bounds__(kRowWarps * 32, 3) row_kernel(RowKernelArgs a, int rows_to_process) {
    __shared__ int sort_buf[kRowWarps][kSortCap];
    __shared__ int off_s[kRowChunk + 1];
    __shared__ int ent_s[kChunkEntryCap];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int chunk0 = blockIdx.x * kRowChunk;
    const int chunk_rows = min(kRowChunk, rows_to_process - chunk0);
    for (int i = threadIdx.x; i <= chunk_rows; i += blockDim.x) off_s[i] = a.offsets[a.row_begin + chunk0 + i];
    __syncthreads();
    const int e_begin = off_s[0];
    const int e_count = off_s[chunk_rows] - e_begin;
    const bool cached = e_count <= kChunkEntryCap;
    if (cached)
        for (int i = threadIdx.x; i < e_count; i += blockDim.x) ent_s[i] = a.entries[e_begin + i];
    __syncthreads();
    for (int lr = warp; lr < chunk_rows; lr += kRowWarps) {
    const int local = chunk0 + lr;
    const int row = a.row_begin + local;
    const int beg = off_s[lr] - e_begin;
    const int n = off_s[lr + 1] - off_s[lr];
    const int* elist = cached ? ent_s + beg : a.entries + e_begin + beg;

    int mine = INT_MAX;
    int mode = 0;  // 0: register list, 1: sorted SMEM list, 2: unsorted list
    if (n <= 32) {
        mine = lane < n ? elist[lane] : INT_MAX;
        mine = warp_sort_ascending(mine, lane);
    } else if (n <= kSortCap) {
        int size = 64;
        while (size < n) size <<= 1;
        int* buf = sort_buf[warp];
        for (int i = lane; i < size; i += 32) buf[i] = i < n ? elist[i] : INT_MAX;
        __syncwarp();
        smem_sort_ascending(buf, size, lane);
        mode = 1;
    } else {
        mode = 2;
    }
    const int* list = mode == 1 ? sort_buf[warp] : elist;

    const size_t row_off = static_cast<size_t>(row) * a.width;
    const size_t out_off = static_cast<size_t>(local) * a.width;
    for (int col0 = 0; col0 < a.width; col0 += 32 * VEC) {
        // VEC = 8: a lane owns [c, c+4) and [c+128, c+132), so every warp-wide
        // float4 access is 512 contiguous bytes (4 L1 wavefronts, not 8).
        const int c = VEC == 8 ? col0 + lane * 4 : col0 + lane * VEC;
        const bool active = c < a.width;
        // Optimizer state (or the gradient row being accumulated) does not
        // depend on the entry list: issue those loads first so their HBM
        // latency overlaps the gather of the batch's gradient rows.
        float w[VEC], m[VEC], v[VEC];
        if (active) {
            if constexpr (MODE == kRowRanger) {
                load_vec<VEC>(a.weights + row_off + c, w);
                load_vec<VEC>(a.momentum + row_off + c, m);
                load_vec<VEC>(a.velocity + row_off + c, v);
            } else if constexpr (MODE == kRowAccumulate) {
                load_vec<VEC>(a.gradients + out_off + c, w);
            }
        }
        float acc[VEC];
#pragma unroll
        for (int i = 0; i < VEC; ++i) acc[i] = 0.0f;
        int k = 0;
        for (; k + 4 <= n; k += 4) {
            int e[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) e[u] = mode == 0 ? __shfl_sync(0xffffffffu, mine, k + u) : list[k + u];
            if (active) {
                float x[4][VEC];
#pragma unroll
                for (int u = 0; u < 4; ++u)
                    load_vec<VEC>(a.src.base[e[u] & 1] + static_cast<size_t>(e[u] >> 1) * a.src.sample_stride + c, x[u]);
#pragma unroll
                for (int u = 0; u < 4; ++u)
#pragma unroll
                    for (int i = 0; i < VEC; ++i) acc[i] += x[u][i];
            }
        }
        for (; k < n; ++k) {
            const int e = mode == 0 ? __shfl_sync(0xffffffffu, mine, k) : list[k];
            if (active) {
                float x[VEC];
                load_vec<VEC>(a.src.base[e & 1] + static_cast<size_t>(e >> 1) * a.src.sample_stride + c, x);
#pragma unroll
                for (int i = 0; i < VEC; ++i) acc[i] += x[i];
            }
        }
        if (!active) continue;
        if constexpr (MODE == kRowWrite) {
            store_vec<VEC>(a.gradients + out_off + c, acc);
        } else if constexpr (MODE == kRowAccumulate) {
#pragma unroll
            for (int i = 0; i < VEC; ++i) w[i] += acc[i];
            store_vec<VEC>(a.gradients + out_off + c, w);
        } else {
            if (n == 0 && a.skip_quiet && !a.ranger.do_lookahead) {
                bool quiet = true;
#pragma unroll
                for (int i = 0; i < VEC; ++i)
                    quiet = quiet && (__float_as_uint(m[i]) | __float_as_uint(v[i])) == 0u && weight_is_quiet(w[i], a.ranger);
                if (quiet) continue;
            }
            float s[VEC];
            if (a.ranger.do_lookahead) load_vec<VEC>(a.slow + row_off + c, s);
#pragma unroll
            for (int i = 0; i < VEC; ++i) radam_coordinate(a.ranger.gradient_factor * acc[i], a.ranger, w[i], m[i], v[i]);
            if (a.ranger.do_lookahead) {
#pragma unroll
                for (int i = 0; i < VEC; ++i) w[i] = lookahead_coordinate(w[i], s[i], a.ranger);
                store_vec<VEC>(a.slow + row_off + c, w);
            }
            store_vec<VEC>(a.weights + row_off + c, w);
            store_vec<VEC>(a.momentum + row_off + c, m);
            store_vec<VEC>(a.velocity + row_off + c, v);
        }
    }
    __syncwarp();
    }
}

template <int MODE>
int launch_row_mode(BulletOuCudaCppContext* ctx, const RowKernelArgs& a, int rows, int vec) {
    const int blocks = (rows + kRowChunk - 1) / kRowChunk;
    if (vec == 8) row_kernel<8, MODE><<<blocks, kRowWarps * 32, 0, ctx->stream>>>(a, rows);
    else if (vec == 4) row_kernel<4, MODE><<<blocks, kRowWarps * 32, 0, ctx->stream>>>(a, rows);
    else row_kernel<1, MODE><<<blocks, kRowWarps * 32, 0, ctx->stream>>>(a, rows);
    return check_launch("sparse row kernel launch");
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

namespace {

// Tile-keyed map (RowTiles): one key per valid feature.
struct TiledMap {
    RowTiles t;
    const int* entry_rank;
    size_t max_active;
    __device__ __forceinline__ int key(int f, size_t s, int persp, int* entry) const {
        const int h = static_cast<int>((s / max_active) * 2 + persp);
        const int e = entry_rank[h];
        *entry = e;
        if (f < 0 || f >= t.kings * t.pieces) return -1;
        const int k = f / t.pieces;
        const int p = f - k * t.pieces;
        const int t0 = t.tile_base[k], nt = t.tile_base[k + 1] - t0;
        const int off = e - t.rank_base[k];
        const int tile = off <= 0 ? 0 : min(off / t.tile_ranks, nt - 1);
        return (t0 + tile) * t.pieces + p;
    }
};

__global__ void count_tiled_kernel(const int* __restrict__ stm, const int* __restrict__ nstm, size_t slots,
                                   TiledMap map, int* __restrict__ counts) {
    const size_t t = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= 2 * slots) return;
    const int persp = t < slots ? 0 : 1;
    const size_t s = persp == 0 ? t : t - slots;
    int e;
    const int key = map.key(persp == 0 ? stm[s] : nstm[s], s, persp, &e);
    if (key >= 0) atomicAdd(&counts[key], 1);
}

__global__ void fill_tiled_kernel(const int* __restrict__ stm, const int* __restrict__ nstm, size_t slots,
                                  TiledMap map, const int* __restrict__ offsets, int* __restrict__ cursor,
                                  int* __restrict__ entries) {
    const size_t t = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= 2 * slots) return;
    const int persp = t < slots ? 0 : 1;
    const size_t s = persp == 0 ? t : t - slots;
    int e;
    const int key = map.key(persp == 0 ? stm[s] : nstm[s], s, persp, &e);
    if (key >= 0) entries[offsets[key] + atomicSub(&cursor[key], 1) - 1] = e;
}

int build_index_impl(BulletOuCudaCppContext* ctx, const int* stm, const int* nstm, size_t batch, size_t max_active,
                     const RowMap& map, size_t n_rows, InverseIndex* out, const int* entry_rank,
                     const TiledMap* tiled = nullptr) {
    const size_t slots = batch * max_active;
    const size_t max_entries = 2 * slots * (map.factorized ? 2 : 1);
    if (n_rows >= static_cast<size_t>(INT_MAX) - kScanTile || max_entries >= static_cast<size_t>(INT_MAX) ||
        2 * batch >= static_cast<size_t>(INT_MAX))
        return fail_message("sparse index: batch or table too large for 32-bit row indexing");
    const int tiles = static_cast<int>((n_rows + kScanTile - 1) / kScanTile);
    void *counts = nullptr, *offsets = nullptr, *entries = nullptr, *tile_sums = nullptr;
    const bool fresh = ctx->scratch[kScratchCsrCounts].bytes < (n_rows + 1) * sizeof(int);
    if (scratch_slot(ctx, kScratchCsrCounts, (n_rows + 1) * sizeof(int), &counts, "cudaMalloc sparse counts") != 0 ||
        scratch_slot(ctx, kScratchCsrOffsets, (n_rows + 1) * sizeof(int), &offsets, "cudaMalloc sparse offsets") != 0 ||
        scratch_slot(ctx, kScratchCsrCursor, (tiles + 1) * sizeof(int), &tile_sums, "cudaMalloc sparse tiles") != 0 ||
        scratch_slot(ctx, kScratchCsrEntries, max_entries * sizeof(int), &entries, "cudaMalloc sparse entries") != 0)
        return -1;
    if (fresh) {
        // counts are left at zero by every fill; clear them once per allocation
        cudaError_t st = cudaMemsetAsync(counts, 0, ctx->scratch[kScratchCsrCounts].bytes, ctx->stream);
        if (st != cudaSuccess) return fail("cudaMemsetAsync sparse counts", st);
    }
    const int threads = 256;
    int blocks = 0;
    if (grid_1d(2 * slots, threads, &blocks, "sparse count") != 0) return -1;
    int* c = static_cast<int*>(counts);
    int* o = static_cast<int*>(offsets);
    int* t = static_cast<int*>(tile_sums);
    if (blocks > 0) {
        if (tiled != nullptr) count_tiled_kernel<<<blocks, threads, 0, ctx->stream>>>(stm, nstm, slots, *tiled, c);
        else count_rows_kernel<<<blocks, threads, 0, ctx->stream>>>(stm, nstm, slots, map, c);
        if (check_launch("sparse count launch") != 0) return -1;
    }
    const int n = static_cast<int>(n_rows);
    scan_tile_sums_kernel<<<tiles, kScanThreads, 0, ctx->stream>>>(c, n, t);
    scan_tile_offsets_kernel<<<1, kScanThreads, 0, ctx->stream>>>(t, tiles);
    scan_apply_kernel<<<tiles, kScanThreads, 0, ctx->stream>>>(c, n, t, tiles, o);
    if (check_launch("sparse scan launch") != 0) return -1;
    if (blocks > 0) {
        if (tiled != nullptr)
            fill_tiled_kernel<<<blocks, threads, 0, ctx->stream>>>(stm, nstm, slots, *tiled, o, c,
                                                                  static_cast<int*>(entries));
        else
            fill_rows_kernel<<<blocks, threads, 0, ctx->stream>>>(stm, nstm, slots, max_active, map, o, c,
                                                                 static_cast<int*>(entries), entry_rank);
        if (check_launch("sparse fill launch") != 0) return -1;
    }
    out->offsets = o;
    out->entries = static_cast<int*>(entries);
    out->counts = c;
    out->n_rows = n;
    out->capacity = max_entries;
    return 0;
}

}  // namespace

int exclusive_scan_counts(BulletOuCudaCppContext* ctx, const int* counts, int n, int* offsets, int* tile_sums) {
    const int tiles = scan_tiles(n);
    scan_tile_sums_kernel<<<tiles, kScanThreads, 0, ctx->stream>>>(counts, n, tile_sums);
    scan_tile_offsets_kernel<<<1, kScanThreads, 0, ctx->stream>>>(tile_sums, tiles);
    scan_apply_kernel<<<tiles, kScanThreads, 0, ctx->stream>>>(counts, n, tile_sums, tiles, offsets);
    return check_launch("exclusive scan launch");
}

int sort_inverse_index(BulletOuCudaCppContext* ctx, const InverseIndex& index, int skip_above) {
    if (index.n_rows <= 0) return 0;
    const int blocks = (index.n_rows + kRowWarps - 1) / kRowWarps;
    sort_rows_kernel<<<blocks, kRowWarps * 32, 0, ctx->stream>>>(index.offsets, index.entries, index.n_rows,
                                                                  skip_above);
    return check_launch("inverse index row sort launch");
}

int build_inverse_index(BulletOuCudaCppContext* ctx, const int* stm, const int* nstm, size_t batch,
                        size_t max_active, size_t input_size, size_t n_rows, InverseIndex* out,
                        const int* entry_rank) {
    return build_index_impl(ctx, stm, nstm, batch, max_active, make_row_map(input_size), n_rows, out, entry_rank);
}

int build_inverse_index_rows(BulletOuCudaCppContext* ctx, const int* stm, const int* nstm, size_t batch,
                             size_t max_active, size_t n_features, InverseIndex* out, const int* entry_rank) {
    RowMap map;
    map.input_size = static_cast<int>(n_features);
    map.factorized = 0;
    return build_index_impl(ctx, stm, nstm, batch, max_active, map, n_features, out, entry_rank);
}

int build_inverse_index_tiled(BulletOuCudaCppContext* ctx, const int* stm, const int* nstm, size_t batch,
                              size_t max_active, const RowTiles& tiles, InverseIndex* out, const int* entry_rank) {
    if (entry_rank == nullptr) return fail_message("internal: the tiled index needs entry ranks");
    TiledMap tm{tiles, entry_rank, max_active};
    RowMap unused{};
    return build_index_impl(ctx, stm, nstm, batch, max_active, unused,
                            static_cast<size_t>(tiles.max_tiles) * static_cast<size_t>(tiles.pieces), out, entry_rank,
                            &tm);
}

int launch_row_kernel(BulletOuCudaCppContext* ctx, int mode, const RowKernelArgs& args, int rows_to_process) {
    if (rows_to_process <= 0) return 0;
    bool al = aligned16(args.src.base[0]) && aligned16(args.src.base[1]) && args.src.sample_stride % 4 == 0;
    if (mode == kRowRanger)
        al = al && aligned16(args.weights) && aligned16(args.momentum) && aligned16(args.velocity) &&
             aligned16(args.slow);
    else
        al = al && aligned16(args.gradients);
    int vec = 1;
    if (al && args.width % 256 == 0) vec = 8;
    else if (al && args.width % 128 == 0) vec = 4;
    switch (mode) {
        case kRowRanger: return launch_row_mode<kRowRanger>(ctx, args, rows_to_process, vec);
        case kRowWrite: return launch_row_mode<kRowWrite>(ctx, args, rows_to_process, vec);
        default: return launch_row_mode<kRowAccumulate>(ctx, args, rows_to_process, vec);
    }
}

}  // namespace bou
