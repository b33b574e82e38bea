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

// Exclusive scan of counts[0, n) into offsets[0, n], one CTA of 1024 threads,
// 4 consecutive counts per thread per tile.
__global__ void __launch_bounds__(1024) scan_rows_kernel(const int* __restrict__ counts, int* __restrict__ offsets,
                                                         int n) {
    __shared__ int warp_sums[32];
    __shared__ int carry_s;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (threadIdx.x == 0) carry_s = 0;
    __syncthreads();
    for (int base = 0; base < n; base += 4096) {
        const int i0 = base + threadIdx.x * 4;
        int v[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) v[q] = (i0 + q < n) ? counts[i0 + q] : 0;
        const int local = v[0] + v[1] + v[2] + v[3];
        int incl = local;
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
            warp_sums[lane] = w;  // inclusive prefix of warp totals
        }
        __syncthreads();
        const int carry = carry_s;
        int run = carry + (warp > 0 ? warp_sums[warp - 1] : 0) + incl - local;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            if (i0 + q < n) offsets[i0 + q] = run;
            run += v[q];
        }
        __syncthreads();
        if (threadIdx.x == 1023) carry_s = carry + warp_sums[31];
        __syncthreads();
    }
    if (threadIdx.x == 0) offsets[n] = carry_s;
}

__global__ void fill_rows_kernel(const int* __restrict__ stm, const int* __restrict__ nstm, size_t slots,
                                 size_t max_active, RowMap map, const int* __restrict__ offsets,
                                 int* __restrict__ cursor, int* __restrict__ entries) {
    const size_t t = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= 2 * slots) return;
    const int persp = t < slots ? 0 : 1;
    const size_t s = persp == 0 ? t : t - slots;
    const int f = persp == 0 ? stm[s] : nstm[s];
    const int entry = static_cast<int>((s / max_active) * 2 + persp);
    int r0, r1;
    const int n = map.rows(f, &r0, &r1);
    if (n >= 1) entries[offsets[r0] + atomicAdd(&cursor[r0], 1)] = entry;
    if (n == 2) entries[offsets[r1] + atomicAdd(&cursor[r1], 1)] = entry;
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

template <int VEC>
struct Vec {
    float v[VEC];
};

template <int VEC>
__device__ __forceinline__ void load_vec(const float* p, float* out) {
    if constexpr (VEC == 8) {
        const float4 a = *reinterpret_cast<const float4*>(p);
        const float4 b = *reinterpret_cast<const float4*>(p + 4);
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
        *reinterpret_cast<float4*>(p + 4) = make_float4(in[4], in[5], in[6], in[7]);
    } else if constexpr (VEC == 4) {
        *reinterpret_cast<float4*>(p) = make_float4(in[0], in[1], in[2], in[3]);
    } else {
#pragma unroll
        for (int i = 0; i < VEC; ++i) p[i] = in[i];
    }
}

template <int VEC, int MODE>
__global__ void __launch_bounds__(kRowWarps * 32) row_kernel(RowKernelArgs a, int rows_to_process) {
    __shared__ int sort_buf[kRowWarps][kSortCap];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int local = blockIdx.x * kRowWarps + warp;
    if (local >= rows_to_process) return;
    const int row = a.row_begin + local;
    const int beg = a.offsets[row];
    const int n = a.offsets[row + 1] - beg;

    int mine = INT_MAX;
    int mode = 0;  // 0: register list, 1: sorted SMEM list, 2: unsorted global list
    if (n <= 32) {
        mine = lane < n ? a.entries[beg + lane] : INT_MAX;
        mine = warp_sort_ascending(mine, lane);
    } else if (n <= kSortCap) {
        int size = 64;
        while (size < n) size <<= 1;
        int* buf = sort_buf[warp];
        for (int i = lane; i < size; i += 32) buf[i] = i < n ? a.entries[beg + i] : INT_MAX;
        __syncwarp();
        smem_sort_ascending(buf, size, lane);
        mode = 1;
    } else {
        mode = 2;
    }
    const int* list = mode == 1 ? sort_buf[warp] : a.entries + beg;

    const size_t row_off = static_cast<size_t>(row) * a.width;
    const size_t out_off = static_cast<size_t>(local) * a.width;
    for (int col0 = 0; col0 < a.width; col0 += 32 * VEC) {
        const int c = col0 + lane * VEC;
        const bool active = c < a.width;
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
            float g[VEC];
            load_vec<VEC>(a.gradients + out_off + c, g);
#pragma unroll
            for (int i = 0; i < VEC; ++i) g[i] += acc[i];
            store_vec<VEC>(a.gradients + out_off + c, g);
        } else {
            float w[VEC], m[VEC], v[VEC];
            load_vec<VEC>(a.weights + row_off + c, w);
            load_vec<VEC>(a.momentum + row_off + c, m);
            load_vec<VEC>(a.velocity + row_off + c, v);
            if (n == 0 && a.skip_quiet && !a.ranger.do_lookahead) {
                bool quiet = true;
#pragma unroll
                for (int i = 0; i < VEC; ++i)
                    quiet = quiet && (__float_as_uint(m[i]) | __float_as_uint(v[i])) == 0u && weight_is_quiet(w[i], a.ranger);
                if (quiet) continue;
            }
#pragma unroll
            for (int i = 0; i < VEC; ++i) radam_coordinate(a.ranger.gradient_factor * acc[i], a.ranger, w[i], m[i], v[i]);
            if (a.ranger.do_lookahead) {
                float s[VEC];
                load_vec<VEC>(a.slow + row_off + c, s);
#pragma unroll
                for (int i = 0; i < VEC; ++i) w[i] = lookahead_coordinate(w[i], s[i], a.ranger);
                store_vec<VEC>(a.slow + row_off + c, w);
            }
            store_vec<VEC>(a.weights + row_off + c, w);
            store_vec<VEC>(a.momentum + row_off + c, m);
            store_vec<VEC>(a.velocity + row_off + c, v);
        }
    }
}

template <int MODE>
int launch_row_mode(BulletOuCudaCppContext* ctx, const RowKernelArgs& a, int rows, int vec) {
    const int blocks = (rows + kRowWarps - 1) / kRowWarps;
    if (vec == 8) row_kernel<8, MODE><<<blocks, kRowWarps * 32, 0, ctx->stream>>>(a, rows);
    else if (vec == 4) row_kernel<4, MODE><<<blocks, kRowWarps * 32, 0, ctx->stream>>>(a, rows);
    else row_kernel<1, MODE><<<blocks, kRowWarps * 32, 0, ctx->stream>>>(a, rows);
    return check_launch("sparse row kernel launch");
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

int build_inverse_index(BulletOuCudaCppContext* ctx, const int* stm, const int* nstm, size_t batch,
                        size_t max_active, size_t input_size, size_t n_rows, InverseIndex* out) {
    const RowMap map = make_row_map(input_size);
    const size_t slots = batch * max_active;
    const size_t max_entries = 2 * slots * (map.factorized ? 2 : 1);
    if (n_rows >= static_cast<size_t>(INT_MAX) || max_entries >= static_cast<size_t>(INT_MAX) ||
        2 * batch >= static_cast<size_t>(INT_MAX))
        return fail_message("sparse index: batch or table too large for 32-bit row indexing");
    void *counts = nullptr, *offsets = nullptr, *entries = nullptr, *cursor = nullptr;
    if (scratch_slot(ctx, kScratchCsrCounts, (n_rows + 1) * sizeof(int), &counts, "cudaMalloc sparse counts") != 0 ||
        scratch_slot(ctx, kScratchCsrOffsets, (n_rows + 1) * sizeof(int), &offsets, "cudaMalloc sparse offsets") != 0 ||
        scratch_slot(ctx, kScratchCsrCursor, (n_rows + 1) * sizeof(int), &cursor, "cudaMalloc sparse cursor") != 0 ||
        scratch_slot(ctx, kScratchCsrEntries, max_entries * sizeof(int), &entries, "cudaMalloc sparse entries") != 0)
        return -1;
    cudaError_t st = cudaMemsetAsync(counts, 0, (n_rows + 1) * sizeof(int), ctx->stream);
    if (st == cudaSuccess) st = cudaMemsetAsync(cursor, 0, (n_rows + 1) * sizeof(int), ctx->stream);
    if (st != cudaSuccess) return fail("cudaMemsetAsync sparse index", st);
    const int threads = 256;
    int blocks = 0;
    if (grid_1d(2 * slots, threads, &blocks, "sparse count") != 0) return -1;
    if (blocks > 0) {
        count_rows_kernel<<<blocks, threads, 0, ctx->stream>>>(stm, nstm, slots, map, static_cast<int*>(counts));
        if (check_launch("sparse count launch") != 0) return -1;
    }
    scan_rows_kernel<<<1, 1024, 0, ctx->stream>>>(static_cast<int*>(counts), static_cast<int*>(offsets),
                                                   static_cast<int>(n_rows));
    if (check_launch("sparse scan launch") != 0) return -1;
    if (blocks > 0) {
        fill_rows_kernel<<<blocks, threads, 0, ctx->stream>>>(stm, nstm, slots, max_active, map,
                                                             static_cast<int*>(offsets), static_cast<int*>(cursor),
                                                             static_cast<int*>(entries));
        if (check_launch("sparse fill launch") != 0) return -1;
    }
    out->offsets = static_cast<int*>(offsets);
    out->entries = static_cast<int*>(entries);
    out->counts = static_cast<int*>(counts);
    out->n_rows = static_cast<int>(n_rows);
    out->capacity = max_entries;
    return 0;
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
