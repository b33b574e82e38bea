// SFNN LayerStack training and inference path for B200 (see sfnn.cuh for the
// network and the reference lines each stage restates).
//
// One training step, every stage a kernel on the context stream:
//   1. fold        -- factorized FT: folded[f] = l0w[f] + alpha * l0w[base + f % 1629]
//                     (cu:1445-1456), so the gather reads one row per feature.
//   2. sorts       -- the 2B half-positions (sample, perspective) by king
//                     (a king's 1629 rows = 9.4 MB at width 1536, L2-resident while
//                     its half-positions are gathered) and the B samples by
//                     LayerStack bucket, cut into tiles of <= 128 samples of one bucket.
//   3. FT forward  -- one warp per half-position in king order; 128-bit loads,
//                     bias + rows in slot order (the reference's sum), ClippedReLU,
//                     pairwise product * 127/128 (cu:1227-1320).
//   4. L1 forward  -- per bucket tile; the tile's effective L1 weights
//                     (bucket rows + alpha * shared factor, cu:2297-2303) in shared memory.
//   5. head        -- per bucket tile, thread per sample: L2 input (SqrCReLU | CReLU),
//                     L2 + CReLU, L3 + PSQT skip, the loss, and the backward through
//                     L3 / L2 / L2 input to the L1 output gradient; per-tile partial
//                     sums of the L2 / L3 / L1-bias gradients.
//   6. L1 backward -- per (bucket tile, 256 columns): combined gradient, the FT
//                     pre-activation gradients of both pair members, per-tile partial
//                     sums of dL1w and of the FT bias gradient.  The pre-activation
//                     gradients are written in king order.
//   7. finalize    -- partial sums reduced in tile order (deterministic), shared-factor
//                     gradients, loss sum; Ranger on the small groups.
//   8. FT rows     -- one warp per (piece, column group): for the piece's row in every
//                     king block, the row's gradient is summed from the inverse index
//                     (ascending entry order) and Ranger updates the row in the same
//                     pass; the virtual (factor) row of the piece receives
//                     alpha * sum over kings (cu:4950-4985) and is updated last.
//                     The FT gradient table is never written.
#include <algorithm>
#include <cfloat>
#include <climits>
#include <cstring>

#include "ft_rows_mma.cuh"
#include "king_sort.cuh"
#include "sfnn.cuh"
#include "exchange.cuh"
#include "sparse_rows.cuh"

namespace bou {
int launch_ranger(BulletOuCudaCppContext* ctx, size_t len, const RangerArgs& a, float* gradients, float* weights,
                  float* momentum, float* velocity, float* slow);
int loss_args(const BulletOuB200LossSpec* loss, size_t batch, LossArgs* out);
}  // namespace bou

namespace bou {
namespace {

constexpr unsigned kFull = 0xffffffffu;
constexpr float kPairScale = 127.0f / 128.0f;  // SFNN_PAIRWISE_SCALE, cu:1148
constexpr int kBucketKeys = kSfnnMaxStacks + 1;
constexpr int kPieceRowWarps = 8;
constexpr int kKingsPerLaunch = 3;  // FT row kernel: king blocks per launch (L2 working set)
constexpr int kPieceRowCtas = 3;    // FT row kernel: resident CTAs per SM (persistent grid)
constexpr int kTileRanks = 4096;    // half-positions per rank tile of the FT row index (24 MB of gradient rows)
// (Loading a row's Ranger state before its gradient sum, to overlap the two
// latencies, made the FT row phase slower, 2.05 -> 2.33 ms at B = 65536: the
// state stream then competes with the gathers for L2.)

__device__ __forceinline__ float crelu01(float x) { return fminf(fmaxf(x, 0.0f), 1.0f); }
__device__ __forceinline__ float crelu_grad(float a, float g) { return a > 0.0f && a < 1.0f ? g : 0.0f; }

// ------------------------------------------------------------------ QAT arithmetic
// Fake quantisation of the reference's training path (cu:1644-1666): the f32
// product rounded half away from zero, ties and |x| >= 2^22 redone in double,
// clamped, divided back (IEEE division: this file is built with fast math).
__device__ __forceinline__ float qat_round(float v, float scale, float lo, float hi) {
    const float scaled = __fmul_rn(v, scale);
    float q = roundf(scaled);
    if (fabsf(scaled) >= 4194304.0f || fabsf(scaled - truncf(scaled)) == 0.5f)
        q = static_cast<float>(round(static_cast<double>(v) * static_cast<double>(scale)));
    return fminf(fmaxf(q, lo), hi);
}
__device__ __forceinline__ float qat_qd(float v, float scale, float lo, float hi) {
    return __fdiv_rn(qat_round(v, scale, lo, hi), scale);
}
// The IEEE quotient q / 127 of an integer |q| <= 32768 without a division:
// q * rh + RN(q * rl) rounded once (fma), rh = RN(1/127) = 0x1.020408p-7,
// rl = RN(1/127 - rh) = 0x1.020408p-35 -- division by a constant through a
// double-word reciprocal (Brisebarre, Muller and Raina, IEEE Trans. Computers
// 53(8), 2004).  Before the final rounding the error is below 2^-46 |q / 127|,
// and q / 127 lies at least ulp / 254 away from every rounding midpoint (127
// is odd and prime, so q / 127 is an integer or not dyadic), so the result is
// the correctly rounded quotient; checked with exact rationals for every q in
// [-32768, 32767].
__device__ __forceinline__ float div127(float q) { return __fmaf_rn(q, 0x1.020408p-7f, __fmul_rn(q, 0x1.020408p-35f)); }
__device__ __forceinline__ float qat_q64(float v) { return qat_qd(v, 64.0f, -128.0f, 127.0f); }
__device__ __forceinline__ float qat_q8128(float v) { return qat_qd(v, 8128.0f, -2147483648.0f, 2147483647.0f); }
__device__ __forceinline__ float qat_q127(float v) { return div127(qat_round(v, 127.0f, -32768.0f, 32767.0f)); }
// a + alpha * b with two roundings (the QAT folds, cu:1790-1795, 9302-9310).
__device__ __forceinline__ float fold_nf(float a, float alpha, float b) { return __fadd_rn(a, __fmul_rn(alpha, b)); }
// round(v * 8128) in double, saturated to i32 (cu:1986-1988).
__device__ __forceinline__ int qat_bias_int(float v) {
    const double q = fmin(2147483647.0, fmax(-2147483648.0, round(static_cast<double>(v) * 8128.0)));
    return static_cast<int>(q);
}
// floor(clamp(c, 0, 1) * 127), exact: the double product of a float and 127 is exact.
__device__ __forceinline__ int qat_lattice(float c) {
    return static_cast<int>(floor(static_cast<double>(fminf(1.0f, fmaxf(0.0f, c))) * 127.0));
}
__device__ __forceinline__ float qat_on_lattice(int n) { return div127(static_cast<float>(n)); }
// Integer of a value already on a lattice (q / 127 or q / 64): round to nearest.
__device__ __forceinline__ int qat_int127(float v) { return __float2int_rn(__fmul_rn(v, 127.0f)); }
__device__ __forceinline__ int qat_int64(float v) { return __float2int_rn(__fmul_rn(v, 64.0f)); }
__device__ __forceinline__ float qat_raw_to_float(long long raw) {
    return static_cast<float>(static_cast<double>(static_cast<int>(raw)) / 8128.0);
}

// ------------------------------------------------------------------ fold
__global__ void fold_ft1_kernel(const float* __restrict__ l0w, float* __restrict__ folded, size_t total, int width,
                                int base, float alpha) {
    const size_t t = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= total) return;
    const size_t f = t / width;
    const size_t j = t - f * width;
    folded[t] = fmaf(alpha, l0w[(static_cast<size_t>(base) + f % kSfnnPieces) * width + j], l0w[t]);
}

// FT QAT (layer_qat_ft_fold_kernel, cu:9302-9312): base rows folded with their
// virtual row (two roundings), then fake-quantised to i16 at 127.
__global__ void fold_ft_qat_kernel(const float* __restrict__ l0w, float* __restrict__ folded, size_t total, int width,
                                   int base, float alpha) {
    const size_t t = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= total) return;
    float v = l0w[t];
    if (base > 0) {
        const size_t f = t / width;
        const size_t j = t - f * width;
        v = fold_nf(v, alpha, l0w[(static_cast<size_t>(base) + f % kSfnnPieces) * width + j]);
    }
    folded[t] = qat_q127(v);
}

// Both folds row by row: one CTA per table row (the virtual row's index once
// per CTA), each thread up to four float4 columns with every load issued
// before the first store.  QAT: the fake-quantised fold, base == 0 quantises
// the row alone.
constexpr int kFoldThreads = 128;
template <bool QAT>
__global__ void __launch_bounds__(kFoldThreads) fold_rows_kernel(const float4* __restrict__ l0w,
                                                                 float4* __restrict__ folded, int w4, int base,
                                                                 float alpha) {
    const size_t f = blockIdx.x;
    const float4* src = l0w + f * w4;
    const float4* vsrc = l0w + (static_cast<size_t>(base) + f % kSfnnPieces) * w4;
    float4* dst = folded + f * w4;
    for (int j0 = 0; j0 < w4; j0 += 4 * kFoldThreads) {
        float4 a[4], v[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int j = j0 + i * kFoldThreads + static_cast<int>(threadIdx.x);
            if (j < w4) {
                a[i] = src[j];
                if (!QAT || base > 0) v[i] = vsrc[j];
            }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int j = j0 + i * kFoldThreads + static_cast<int>(threadIdx.x);
            if (j >= w4) continue;
            float4 o;
            if (QAT) {
                float4 x = a[i];
                if (base > 0)
                    x = make_float4(fold_nf(x.x, alpha, v[i].x), fold_nf(x.y, alpha, v[i].y),
                                    fold_nf(x.z, alpha, v[i].z), fold_nf(x.w, alpha, v[i].w));
                o = make_float4(qat_q127(x.x), qat_q127(x.y), qat_q127(x.z), qat_q127(x.w));
            } else {
                o = make_float4(fmaf(alpha, v[i].x, a[i].x), fmaf(alpha, v[i].y, a[i].y), fmaf(alpha, v[i].z, a[i].z),
                                fmaf(alpha, v[i].w, a[i].w));
            }
            dst[j] = o;
        }
    }
}

// layer_qat_vector_kernel (cu:9294-9300): element-wise fake quantisation.
__global__ void qat_vector_kernel(const float* __restrict__ src, float* __restrict__ dst, size_t n, int kind) {
    const size_t t = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= n) return;
    const float v = src[t];
    dst[t] = kind == 0 ? qat_q127(v) : (kind == 1 ? qat_q64(v) : qat_q8128(v));
}

// Reference-layout L1 QAT weights [S][O][W] (sfnn_build_quantized_proxy_stacked_
// weights_kernel, cu:1735-1810): bucket rows + alpha * shared (two roundings),
// fake-quantised to i8 at 64 when quantize.
__global__ void qat_l1_fold_kernel(const float* __restrict__ l1w, const float* __restrict__ l1fw, float alpha,
                                   size_t total, int out_dim, int width, int quantize, float* __restrict__ dst) {
    const size_t t = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= total) return;
    float v = l1w[t];
    if (l1fw != nullptr) {
        const size_t i = t % width;
        const size_t o = (t / width) % out_dim;
        v = fold_nf(v, alpha, l1fw[i * out_dim + o]);
    }
    dst[t] = quantize ? qat_q64(v) : v;
}

// L1 QAT biases (sfnn_build_quantized_proxy_stacked_bias_kernel, cu:1921-1991):
// folded master bias, its i32 at 8128 and its fake-quantised value.
__global__ void qat_l1_bias_kernel(const float* __restrict__ l1b, const float* __restrict__ l1fb, float alpha, int n,
                                   int out_dim, int quantize, float* __restrict__ b_eff, int* __restrict__ b_int,
                                   float* __restrict__ b_master) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= n) return;
    float v = l1b[t];
    if (l1fb != nullptr) v = fold_nf(v, alpha, l1fb[t % out_dim]);
    if (b_master != nullptr) b_master[t] = v;
    if (b_int != nullptr) b_int[t] = qat_bias_int(v);
    if (b_eff != nullptr) b_eff[t] = quantize ? qat_q8128(v) : v;
}

// bulletou_layer_qat FT layout (layer_qat_ft_fold_kernel, cu:9302-9312): base
// rows folded with virtual row base + f % vr and fake-quantised; virtual rows 0.
__global__ void layer_qat_ft_kernel(const float* __restrict__ src, float* __restrict__ dst, size_t base, size_t vr,
                                    size_t width, float alpha, size_t total) {
    const size_t t = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= total) return;
    const size_t f = t / width;
    const size_t u = t - f * width;
    if (f >= base) {
        dst[t] = 0.0f;
        return;
    }
    dst[t] = qat_q127(fold_nf(src[t], alpha, src[(base + f % vr) * width + u]));
}

// Quantised-proxy FT rows (sfnn_build_quantized_proxy_l0w_kernel,
// cu:1682-1705): row f < dst_rows folded with virtual row dst_rows + f % vr
// when vr > 0 (two roundings), then rounded to 1/127 in i16 range.
__global__ void proxy_ft_kernel(const float* __restrict__ src, float* __restrict__ dst, size_t dst_rows, size_t vr,
                                size_t width, float alpha) {
    const size_t t = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= dst_rows * width) return;
    float v = src[t];
    if (vr > 0) {
        const size_t f = t / width;
        v = fold_nf(v, alpha, src[(dst_rows + f % vr) * width + (t - f * width)]);
    }
    dst[t] = qat_q127(v);
}

// Quantised-proxy dense tensors laid out [stacks][cells] whose shared factor
// has the same cell order (sfnn_build_quantized_proxy_stacked_weights_kernel /
// _bias_kernel with an output-major factor, cu:1735-1830, 1921-1991): value
// (+ alpha * shared[t % cells], two roundings) rounded to 1/64 in i8 range
// (kind 1) or to 1/8128 in i32 range (kind 2).
__global__ void proxy_stacked_kernel(const float* __restrict__ src, const float* __restrict__ shared, size_t cells,
                                     size_t total, float alpha, int kind, float* __restrict__ dst) {
    const size_t t = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= total) return;
    float v = src[t];
    if (shared != nullptr) v = fold_nf(v, alpha, shared[t % cells]);
    dst[t] = kind == 1 ? qat_q64(v) : qat_q8128(v);
}

__global__ void nonzero_kernel(const float* __restrict__ w, size_t nw, const float* __restrict__ b, size_t nb,
                               float* __restrict__ flag) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const bool nz = i < nw ? w[i] != 0.0f : (i < nw + nb && b[i - nw] != 0.0f);
    if (__syncthreads_or(nz) && threadIdx.x == 0) atomicExch(flag, 1.0f);
}

// ------------------------------------------------------------------ bucket sort + tiles
__global__ void __launch_bounds__(kKingSortThreads) bucket_hist_kernel(const int* __restrict__ buckets, int n,
                                                                       int stacks, int* __restrict__ keys,
                                                                       int* __restrict__ block_hist) {
    __shared__ int hist[kBucketKeys];
    for (int i = threadIdx.x; i < kBucketKeys; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    const int b = blockIdx.x * kKingSortThreads + threadIdx.x;
    if (b < n) {
        const int s = buckets[b];
        const int key = (s >= 0 && s < stacks) ? s : stacks;
        keys[b] = key;
        atomicAdd(&hist[key], 1);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < kBucketKeys; i += blockDim.x) block_hist[blockIdx.x * kBucketKeys + i] = hist[i];
}

// One CTA.  Keys 0..stacks (the last one holds samples with an invalid
// bucket) are cut into tiles of at most kSfnnTile consecutive sorted samples.
// tile_base[k] = first rank tile of king block k, max(1, ceil(N_k / tile_ranks))
// tiles each (one thread; kings <= kSfnnKingKeys).  With a single row block
// (no factorized king blocks) every sorted rank belongs to it.
__global__ void king_tiles_kernel(const int* __restrict__ key_off, int kings, int tile_ranks,
                                  int* __restrict__ tile_base) {
    if (threadIdx.x != 0) return;
    int run = 0;
    for (int k = 0; k < kings; ++k) {
        tile_base[k] = run;
        const int end = kings == 1 ? key_off[kSfnnKingKeys] : key_off[k + 1];
        const int n = end - key_off[k];
        run += max(1, (n + tile_ranks - 1) / tile_ranks);
    }
    tile_base[kings] = run;
}

__global__ void __launch_bounds__(128) tile_table_kernel(const int* __restrict__ key_off, int keys,
                                                         int* __restrict__ n_tiles, int* __restrict__ tile_key,
                                                         int* __restrict__ tile_begin, int* __restrict__ tile_end,
                                                         int* __restrict__ key_first) {
    __shared__ int first[kBucketKeys + 1];
    const int k = threadIdx.x;
    int cnt = 0;
    if (k < keys) cnt = (key_off[k + 1] - key_off[k] + kSfnnTile - 1) / kSfnnTile;
    if (k < keys) first[k + 1] = cnt;
    __syncthreads();
    if (k == 0) {
        first[0] = 0;
        for (int i = 1; i <= keys; ++i) first[i] += first[i - 1];
        *n_tiles = first[keys];
    }
    __syncthreads();
    if (k <= keys) key_first[k] = first[k];
    if (k < keys) {
        const int b0 = key_off[k], b1 = key_off[k + 1];
        for (int i = 0; i < cnt; ++i) {
            const int t = first[k] + i;
            tile_key[t] = k;
            tile_begin[t] = b0 + i * kSfnnTile;
            tile_end[t] = min(b1, b0 + (i + 1) * kSfnnTile);
        }
    }
}

struct Tiles {
    const int* order;      // samples in bucket order
    const int* n_tiles;    // device scalar
    const int* key;        // bucket of each tile (== stacks: invalid-bucket samples)
    const int* begin;
    const int* end;
    const int* key_first;  // first tile of each key, [stacks + 2]
    int max_tiles;
};

// ------------------------------------------------------------------ FT forward
struct FtArgs {
    const int* order;  // king order of half-positions (null: h = position)
    const int* stm;
    const int* nstm;
    const float* table;  // [n_features][width], folded when factorized
    const float* bias;
    float* l0[2];        // ClippedReLU output per perspective, [B][width]
    float* combined;     // [B][width]
    int n_half;
    int max_active;
    int n_features;
    int width;
    int lattice;         // dense QAT: combined floored to the 1/127 lattice (cu:5993-6012)
};

__device__ __forceinline__ float pair_out(float x0, float x1, int lattice) {
    const float c = x0 * x1 * kPairScale;
    return lattice ? qat_on_lattice(qat_lattice(c)) : c;
}

// Widths with a warp FT kernel (NCH = width / 128 float4 chunks per row).
__host__ __device__ inline bool ft_warp_width(int w) {
    return w == 256 || w == 512 || w == 1024 || w == 1536 || w == 2304;
}

// One warp per half-position; lane owns float4 chunks lane + 32 i, so chunk i
// and chunk i + NCH/2 are the two members of a pair (width / 2 apart).
template <int NCH, bool LATTICE>
__global__ void __launch_bounds__(256) ft_forward_kernel(FtArgs a) {
    const int lane = threadIdx.x & 31;
    const int pos = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (pos >= a.n_half) return;
    const int h = a.order != nullptr ? a.order[pos] : pos;
    const int b = h >> 1, v = h & 1;
    const int* idx = (v ? a.nstm : a.stm) + static_cast<size_t>(b) * a.max_active;
    const float4* bias4 = reinterpret_cast<const float4*>(a.bias);
    float4 acc[NCH];
#pragma unroll
    for (int i = 0; i < NCH; ++i) acc[i] = __ldg(bias4 + lane + 32 * i);
    const size_t w4 = static_cast<size_t>(a.width) >> 2;
    for (int s0 = 0; s0 < a.max_active; s0 += 32) {
        const int mine = s0 + lane < a.max_active ? __ldg(idx + s0 + lane) : -1;
        const int n = min(32, a.max_active - s0);
        for (int u = 0; u < n; ++u) {
            const int f = __shfl_sync(kFull, mine, u);
            if (f < 0 || f >= a.n_features) continue;
            const float4* row = reinterpret_cast<const float4*>(a.table) + static_cast<size_t>(f) * w4;
            float4 r[NCH];
#pragma unroll
            for (int i = 0; i < NCH; ++i) r[i] = __ldg(row + lane + 32 * i);
#pragma unroll
            for (int i = 0; i < NCH; ++i) {
                acc[i].x += r[i].x;
                acc[i].y += r[i].y;
                acc[i].z += r[i].z;
                acc[i].w += r[i].w;
            }
        }
    }
    float4* out = reinterpret_cast<float4*>(v ? a.l0[1] : a.l0[0]) + static_cast<size_t>(b) * w4;
#pragma unroll
    for (int i = 0; i < NCH; ++i) {
        acc[i] = make_float4(crelu01(acc[i].x), crelu01(acc[i].y), crelu01(acc[i].z), crelu01(acc[i].w));
        out[lane + 32 * i] = acc[i];
    }
    if (a.combined == nullptr) return;  // the engine's integer FT writes it instead
    float4* comb = reinterpret_cast<float4*>(a.combined) + static_cast<size_t>(b) * w4 + v * (w4 >> 1);
#pragma unroll
    for (int i = 0; i < NCH / 2; ++i) {
        const float4 x0 = acc[i], x1 = acc[i + NCH / 2];
        if (LATTICE) {
            comb[lane + 32 * i] = make_float4(pair_out(x0.x, x1.x, 1), pair_out(x0.y, x1.y, 1),
                                              pair_out(x0.z, x1.z, 1), pair_out(x0.w, x1.w, 1));
        } else {
            comb[lane + 32 * i] = make_float4(x0.x * x1.x * kPairScale, x0.y * x1.y * kPairScale,
                                              x0.z * x1.z * kPairScale, x0.w * x1.w * kPairScale);
        }
    }
}

// Dense QAT with FT QAT in one gather: the f32 sums of the fake-quantised
// folded rows (v = q / 127) give the ClippedReLU outputs the backward reads,
// and the same loaded rows give the engine's integer FT (doubled i16 sums with
// wrap, clamp [0, 254], (s0 s1) >> 9, over 127; dense_qat_exact_ft_kernel,
// cu:6344-6390).  q comes back from v exactly without a conversion:
// fma(v, 127, 1.5 * 2^23) lands in [2^23, 2^24), where the float spacing is 1,
// on 1.5 * 2^23 + q (|v * 127 - q| <= 0.002), so the low 16 bits of its bit
// pattern are q's two's complement.  The engine keeps only the sums modulo
// 2^16: two columns' low halves are packed in one word (byte permute) and
// summed with a per-half-word add (add.u16x2: no carry between the halves).
//
// G warps share a half-position; warp g owns, for every lane, the float4
// chunks g*C .. g*C+C-1 of the first half of the row and their pair partners
// H chunks further (H = NCH / 2, C = H / G).  Each row is loaded in R rounds
// (fewer registers for loads in flight).
constexpr float kQMagic = 12582912.0f;  // 1.5 * 2^23
constexpr int kFtIntWarps = 2;          // width 1536: warps per half-position
constexpr int kFtIntRounds = 1;         // width 1536: load rounds per row

__device__ __forceinline__ unsigned add_u16x2(unsigned a, unsigned b) {
    unsigned d;
    asm("add.u16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ unsigned q_pair(float x, float y) {
    return __byte_perm(__float_as_uint(fmaf(x, 127.0f, kQMagic)), __float_as_uint(fmaf(y, 127.0f, kQMagic)),
                       0x5410);
}
__device__ __forceinline__ unsigned q_pack(int lo, int hi) {
    return (static_cast<unsigned>(lo) & 0xffffu) | (static_cast<unsigned>(hi) << 16);
}

template <int NCH, int G, int R>
__global__ void __launch_bounds__(32 * G * (8 / G)) ft_forward_int_kernel(FtArgs a) {
    constexpr int H = NCH / 2;
    constexpr int C = H / G;
    constexpr int S = 2 * C;   // chunks per warp
    constexpr int SR = S / R;  // chunks per load round
    constexpr int P = 8 / G;   // half-positions per CTA
    static_assert(H % G == 0 && S % R == 0, "chunks must split evenly over warps and rounds");
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int pos = blockIdx.x * P + warp / G;
    const int g = warp - (warp / G) * G;
    if (pos >= a.n_half) return;
    const int h = a.order[pos];
    const int b = h >> 1, v = h & 1;
    const int* idx = (v ? a.nstm : a.stm) + static_cast<size_t>(b) * a.max_active;
    const float4* bias4 = reinterpret_cast<const float4*>(a.bias);
    auto chunk_of = [&](int s) { return (s < C ? 0 : H) + g * C + (s < C ? s : s - C); };
    float4 acc[S];
    uint2 qs[S];
#pragma unroll
    for (int s = 0; s < S; ++s) {
        acc[s] = __ldg(bias4 + lane + 32 * chunk_of(s));
        qs[s] = make_uint2(q_pack(qat_int127(acc[s].x), qat_int127(acc[s].y)),
                           q_pack(qat_int127(acc[s].z), qat_int127(acc[s].w)));
    }
    const size_t w4 = static_cast<size_t>(a.width) >> 2;
    for (int s0 = 0; s0 < a.max_active; s0 += 32) {
        const int mine = s0 + lane < a.max_active ? __ldg(idx + s0 + lane) : -1;
        const int n = min(32, a.max_active - s0);
        for (int u = 0; u < n; ++u) {
            const int f = __shfl_sync(kFull, mine, u);
            if (f < 0 || f >= a.n_features) continue;
            const float4* row = reinterpret_cast<const float4*>(a.table) + static_cast<size_t>(f) * w4;
#pragma unroll
            for (int r = 0; r < R; ++r) {
                float4 t[SR];
#pragma unroll
                for (int k = 0; k < SR; ++k) t[k] = __ldg(row + lane + 32 * chunk_of(r * SR + k));
#pragma unroll
                for (int k = 0; k < SR; ++k) {
                    const int s = r * SR + k;
                    acc[s].x += t[k].x;
                    acc[s].y += t[k].y;
                    acc[s].z += t[k].z;
                    acc[s].w += t[k].w;
                    qs[s].x = add_u16x2(qs[s].x, q_pair(t[k].x, t[k].y));
                    qs[s].y = add_u16x2(qs[s].y, q_pair(t[k].z, t[k].w));
                }
            }
        }
    }
    float4* out = reinterpret_cast<float4*>(v ? a.l0[1] : a.l0[0]) + static_cast<size_t>(b) * w4;
#pragma unroll
    for (int s = 0; s < S; ++s)
        out[lane + 32 * chunk_of(s)] = make_float4(crelu01(acc[s].x), crelu01(acc[s].y), crelu01(acc[s].z),
                                                   crelu01(acc[s].w));
    float4* comb = reinterpret_cast<float4*>(a.combined) + static_cast<size_t>(b) * w4 + v * (w4 >> 1);
    // a 16-bit sum q -> the doubled sum wrapped to i16, clamped to [0, 254]
    auto clip = [](unsigned q) { return min(254, max(0, static_cast<int>(static_cast<short>(q << 1)))); };
    auto pair = [&](unsigned q0, unsigned q1) { return qat_on_lattice((clip(q0) * clip(q1)) >> 9); };
#pragma unroll
    for (int s = 0; s < C; ++s) {
        const uint2 q0 = qs[s], q1 = qs[s + C];
        comb[lane + 32 * (g * C + s)] = make_float4(pair(q0.x & 0xffffu, q1.x & 0xffffu), pair(q0.x >> 16, q1.x >> 16),
                                                    pair(q0.y & 0xffffu, q1.y & 0xffffu), pair(q0.y >> 16, q1.y >> 16));
    }
}

// Any even width: one thread per (half-position, pair).
__global__ void ft_forward_generic_kernel(FtArgs a) {
    const int half = a.width / 2;
    const size_t t = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= static_cast<size_t>(a.n_half) * half) return;
    const int h = static_cast<int>(t / half);
    const int j = static_cast<int>(t - static_cast<size_t>(h) * half);
    const int b = h >> 1, v = h & 1;
    const int* idx = (v ? a.nstm : a.stm) + static_cast<size_t>(b) * a.max_active;
    float s0 = a.bias[j], s1 = a.bias[j + half];
    for (int s = 0; s < a.max_active; ++s) {
        const int f = idx[s];
        if (f < 0 || f >= a.n_features) continue;
        const float* row = a.table + static_cast<size_t>(f) * a.width;
        s0 += row[j];
        s1 += row[j + half];
    }
    const float x0 = crelu01(s0), x1 = crelu01(s1);
    float* out = (v ? a.l0[1] : a.l0[0]) + static_cast<size_t>(b) * a.width;
    out[j] = x0;
    out[j + half] = x1;
    if (a.combined != nullptr) a.combined[static_cast<size_t>(b) * a.width + v * half + j] = pair_out(x0, x1, a.lattice);
}

// Dense QAT with FT QAT: the engine's integer FT from the fake-quantised table
// (q / 127): doubled i16 sums with wrap, clamp [0, 254], (s0 * s1) >> 9, over
// 127 (dense_qat_exact_ft_kernel, cu:6344-6390).  Thread per (half-position, pair).
__global__ void qat_exact_ft_kernel(FtArgs a) {
    const int half = a.width / 2;
    const size_t t = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= static_cast<size_t>(a.n_half) * half) return;
    const int h = static_cast<int>(t / half);
    const int j = static_cast<int>(t - static_cast<size_t>(h) * half);
    const int b = h >> 1, v = h & 1;
    const int* idx = (v ? a.nstm : a.stm) + static_cast<size_t>(b) * a.max_active;
    int s0 = 2 * qat_int127(a.bias[j]), s1 = 2 * qat_int127(a.bias[j + half]);
    for (int s = 0; s < a.max_active; ++s) {
        const int f = idx[s];
        if (f < 0 || f >= a.n_features) continue;
        const float* row = a.table + static_cast<size_t>(f) * a.width;
        s0 += 2 * qat_int127(row[j]);
        s1 += 2 * qat_int127(row[j + half]);
    }
    const int x0 = min(254, max(0, static_cast<int>(static_cast<short>(s0))));
    const int x1 = min(254, max(0, static_cast<int>(static_cast<short>(s1))));
    a.combined[static_cast<size_t>(b) * a.width + v * half + j] = qat_on_lattice((x0 * x1) >> 9);
}

// ------------------------------------------------------------------ L1
// Effective L1 weights, input-major [stacks][width][l1_out]:
// l1w[s][o][i] + alpha * l1fw[i][o]  (cu:2297-2303).
__global__ void l1_eff_kernel(const float* __restrict__ l1w, const float* __restrict__ l1fw, float alpha, int stacks,
                              int out_dim, int width, int quantize, float* __restrict__ w_eff) {
    const size_t t = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const size_t per = static_cast<size_t>(width) * out_dim;
    if (t >= per * stacks) return;
    const size_t s = t / per;
    const size_t r = t - s * per;
    const size_t i = r / out_dim;
    const size_t o = r - i * out_dim;
    float w = l1w[(s * out_dim + o) * width + i];
    if (quantize) {
        // L1 QAT: fold with two roundings, then fake-quantise (cu:11514-11570).
        if (l1fw != nullptr) w = fold_nf(w, alpha, l1fw[i * out_dim + o]);
        w = qat_q64(w);
    } else if (l1fw != nullptr) {
        w = fmaf(alpha, l1fw[i * out_dim + o], w);
    }
    w_eff[t] = w;
}

struct L1Args {
    Tiles tiles;
    const float* combined;
    const float* w_eff;  // [stacks][width][O]
    const float* l1b;
    const float* l1fb;   // null without the shared factor
    float alpha;
    float* l1;           // [B][O]
    int width;
    int out_dim;
    int stacks;
};

// Bias terms are added after the dot product, bucket bias first, as the
// reference does (cu:2318-2322).
__device__ __forceinline__ float l1_bias(const L1Args& a, int s, int o, float dot) {
    float r = dot + a.l1b[s * a.out_dim + o];
    if (a.l1fb != nullptr) r = fmaf(a.alpha, a.l1fb[o], r);
    return r;
}

// O = 16: thread (sample lane, output quad); the tile's effective weights in
// shared memory as [width][16], read as float4 (conflict-free).
__global__ void __launch_bounds__(256) l1_forward16_kernel(L1Args a) {
    extern __shared__ float4 ws4[];
    const int t = blockIdx.x;
    if (t >= *a.tiles.n_tiles) return;
    const int s = a.tiles.key[t];
    const int pb = a.tiles.begin[t], pe = a.tiles.end[t];
    if (s >= a.stacks) {
        for (int i = threadIdx.x; i < (pe - pb) * 16; i += blockDim.x)
            a.l1[static_cast<size_t>(a.tiles.order[pb + i / 16]) * 16 + (i & 15)] = 0.0f;
        return;
    }
    const float4* src = reinterpret_cast<const float4*>(a.w_eff + static_cast<size_t>(s) * a.width * 16);
    for (int i = threadIdx.x; i < a.width * 4; i += blockDim.x) ws4[i] = src[i];
    __syncthreads();
    const int og = threadIdx.x & 3;
    const int w4 = a.width >> 2;
    for (int p = pb + (threadIdx.x >> 2); p < pe; p += 64) {
        const int b = a.tiles.order[p];
        const float4* c4 = reinterpret_cast<const float4*>(a.combined) + static_cast<size_t>(b) * w4;
        float acc0 = 0.0f, acc1 = 0.0f, acc2 = 0.0f, acc3 = 0.0f;
        for (int k4 = 0; k4 < w4; ++k4) {
            const float4 c = __ldg(c4 + k4);
            const float cv[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                const float4 w = ws4[(4 * k4 + kk) * 4 + og];
                acc0 = fmaf(cv[kk], w.x, acc0);
                acc1 = fmaf(cv[kk], w.y, acc1);
                acc2 = fmaf(cv[kk], w.z, acc2);
                acc3 = fmaf(cv[kk], w.w, acc3);
            }
        }
        float* out = a.l1 + static_cast<size_t>(b) * 16 + 4 * og;
        out[0] = l1_bias(a, s, 4 * og + 0, acc0);
        out[1] = l1_bias(a, s, 4 * og + 1, acc1);
        out[2] = l1_bias(a, s, 4 * og + 2, acc2);
        out[3] = l1_bias(a, s, 4 * og + 3, acc3);
    }
}

// Any O / width: one thread per (sample, output) of the tile.
__global__ void __launch_bounds__(256) l1_forward_generic_kernel(L1Args a) {
    const int t = blockIdx.x;
    if (t >= *a.tiles.n_tiles) return;
    const int s = a.tiles.key[t];
    const int pb = a.tiles.begin[t], pe = a.tiles.end[t];
    const int O = a.out_dim;
    for (int i = threadIdx.x; i < (pe - pb) * O; i += blockDim.x) {
        const int b = a.tiles.order[pb + i / O];
        const int o = i % O;
        float* out = a.l1 + static_cast<size_t>(b) * O + o;
        if (s >= a.stacks) {
            *out = 0.0f;
            continue;
        }
        const float* c = a.combined + static_cast<size_t>(b) * a.width;
        const float* w = a.w_eff + static_cast<size_t>(s) * a.width * O + o;
        float acc = 0.0f;
        for (int k = 0; k < a.width; ++k) acc = fmaf(c[k], w[static_cast<size_t>(k) * O], acc);
        *out = l1_bias(a, s, o, acc);
    }
}

// Dense QAT L1 (dense_qat_l1_warp_kernel / _packed, cu:6056-6100, 6223-6280):
// raw = round(b * 8128) + sum_i int(c_i * 127) * int(w_i * 64) over the lattice
// FT output and the fake-quantised weights, exact in integers; l1 = raw / 8128.
struct L1IntArgs {
    Tiles tiles;
    const float* combined;
    const float* w_eff;  // [stacks][width][O] fake-quantised
    const int* b_int;    // [stacks][O]
    float* l1;
    int* raw;
    int width;
    int out_dim;
    int stacks;
};

__device__ __forceinline__ int dp4a_u8s8(unsigned u8x4, int s8x4, int acc) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(u8x4), "r"(s8x4), "r"(acc));
    return d;
}

// O = 16: thread (sample lane, output quad).  The tile's integer weights sit
// in shared memory packed for dp4a: entry (k4, quad) is an int4 whose word j
// holds the four i8 weights of inputs 4 k4 .. 4 k4 + 3 for output 4 quad + j;
// the lattice FT outputs (0..127) are packed four to a word on the fly.
// Warp per sample: lane l takes the float4 groups k4 = l, l + 32, ... of the
// sample's combined row (all its loads independent), quantises them to u8
// and accumulates all 16 outputs with dp4a against the bucket's i8 weights
// in shared memory ([output group og][k4] int4, conflict-free); the 16
// per-lane sums are then reduced across the warp by halving exchanges (lane
// l ends with output (l >> 1) & 15).  Integer sums: any order is exact.
__global__ void __launch_bounds__(256) l1_forward16_int_kernel(L1IntArgs a) {
    extern __shared__ int4 wq4[];
    const int t = blockIdx.x;
    if (t >= *a.tiles.n_tiles) return;
    const int s = a.tiles.key[t];
    const int pb = a.tiles.begin[t], pe = a.tiles.end[t];
    if (s >= a.stacks) {
        for (int i = threadIdx.x; i < (pe - pb) * 16; i += blockDim.x) {
            const size_t k = static_cast<size_t>(a.tiles.order[pb + i / 16]) * 16 + (i & 15);
            a.l1[k] = 0.0f;
            a.raw[k] = 0;
        }
        return;
    }
    const int w4 = a.width >> 2;
    const float* src = a.w_eff + static_cast<size_t>(s) * a.width * 16;  // [width][16]
    for (int i = threadIdx.x; i < w4 * 4; i += blockDim.x) {
        const int og = i / w4, k4 = i - og * w4;
        int word[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            unsigned packed = 0;
#pragma unroll
            for (int e = 0; e < 4; ++e)
                packed |= (static_cast<unsigned>(qat_int64(src[(4 * k4 + e) * 16 + 4 * og + j])) & 0xffu) << (8 * e);
            word[j] = static_cast<int>(packed);
        }
        wq4[og * w4 + k4] = make_int4(word[0], word[1], word[2], word[3]);
    }
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    constexpr int kGroups = 16;  // float4 groups in flight per lane
    for (int p = pb + warp; p < pe; p += 8) {
        const int b = a.tiles.order[p];
        const float4* c4 = reinterpret_cast<const float4*>(a.combined) + static_cast<size_t>(b) * w4;
        int acc[16];
#pragma unroll
        for (int o = 0; o < 16; ++o) acc[o] = 0;
        for (int k0 = 0; k0 < w4; k0 += 32 * kGroups) {
            float4 c[kGroups];
#pragma unroll
            for (int g = 0; g < kGroups; ++g) {
                const int k4 = k0 + g * 32 + lane;
                c[g] = k4 < w4 ? __ldg(c4 + k4) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            }
#pragma unroll
            for (int g = 0; g < kGroups; ++g) {
                const int k4 = k0 + g * 32 + lane;
                if (k4 >= w4) break;
                const unsigned cv = static_cast<unsigned>(qat_int127(c[g].x)) |
                                    (static_cast<unsigned>(qat_int127(c[g].y)) << 8) |
                                    (static_cast<unsigned>(qat_int127(c[g].z)) << 16) |
                                    (static_cast<unsigned>(qat_int127(c[g].w)) << 24);
#pragma unroll
                for (int og = 0; og < 4; ++og) {
                    const int4 w = wq4[og * w4 + k4];
                    acc[4 * og + 0] = dp4a_u8s8(cv, w.x, acc[4 * og + 0]);
                    acc[4 * og + 1] = dp4a_u8s8(cv, w.y, acc[4 * og + 1]);
                    acc[4 * og + 2] = dp4a_u8s8(cv, w.z, acc[4 * og + 2]);
                    acc[4 * og + 3] = dp4a_u8s8(cv, w.w, acc[4 * og + 3]);
                }
            }
        }
        // halving exchanges: 8 + 4 + 2 + 1 + 1 shuffles
#pragma unroll
        for (int d = 16, n = 8; d >= 2; d >>= 1, n >>= 1) {
            const bool upper = (lane & d) != 0;
#pragma unroll
            for (int i = 0; i < n; ++i) {
                const int send = upper ? acc[i] : acc[i + n];
                const int keep = upper ? acc[i + n] : acc[i];
                acc[i] = keep + __shfl_xor_sync(kFull, send, d);
            }
        }
        const int total = acc[0] + __shfl_xor_sync(kFull, acc[0], 1);
        if ((lane & 1) == 0) {
            const int o = (lane >> 1) & 15;
            const long long r = static_cast<long long>(total) + a.b_int[s * 16 + o];
            a.raw[static_cast<size_t>(b) * 16 + o] = static_cast<int>(r);
            a.l1[static_cast<size_t>(b) * 16 + o] = qat_raw_to_float(r);
        }
    }
}

// Any O / width: one thread per (sample, output) of the tile.
__global__ void __launch_bounds__(256) l1_forward_int_generic_kernel(L1IntArgs a) {
    const int t = blockIdx.x;
    if (t >= *a.tiles.n_tiles) return;
    const int s = a.tiles.key[t];
    const int pb = a.tiles.begin[t], pe = a.tiles.end[t];
    const int O = a.out_dim;
    for (int i = threadIdx.x; i < (pe - pb) * O; i += blockDim.x) {
        const int b = a.tiles.order[pb + i / O];
        const int o = i % O;
        const size_t k = static_cast<size_t>(b) * O + o;
        if (s >= a.stacks) {
            a.l1[k] = 0.0f;
            a.raw[k] = 0;
            continue;
        }
        const float* c = a.combined + static_cast<size_t>(b) * a.width;
        const float* w = a.w_eff + static_cast<size_t>(s) * a.width * O + o;
        long long acc = a.b_int[s * O + o];
        for (int j = 0; j < a.width; ++j)
            acc += static_cast<long long>(qat_int127(c[j])) * qat_int64(w[static_cast<size_t>(j) * O]);
        a.raw[k] = static_cast<int>(acc);
        a.l1[k] = qat_raw_to_float(acc);
    }
}

// ------------------------------------------------------------------ head
enum HeadMode : int { kHeadForward = 0, kHeadTrain = 1, kHeadBackward = 2 };

struct HeadArgs {
    Tiles tiles;
    const float* l1;
    const float* l2w;
    const float* l2b;   // null in the backward (biases are forward-only)
    const float* l2fw;
    const float* l2fb;
    const float* l3w;
    const float* l3b;
    const float* l3fw;
    const float* l3fb;
    float alpha;
    float* l2_input;  // [B][I2]   written (forward / train), read (backward)
    float* l2;        // [B][L2]   written (forward / train), read (backward)
    float* output;    // [B]
    const float* targets;
    const float* entry_weights;
    LossArgs loss;
    float* per_sample;
    float* mog;       // written (train), read (backward)
    float* g1;        // [B][O]
    float* l2_gradients;        // optional [B][L2] (reference backward buffers)
    float* l2_input_gradients;  // optional [B][I2]
    float* partials;  // [max_tiles][head_partial_len]
    int l1_hidden;
    int l1_out;
    int l1_skip;
    int l2_size;
    int stacks;
    int mode;
    // QAT
    int qat_l2;               // fake-quantise the staged L2 weights / biases
    int qat_l3;
    const int* l1_raw;        // dense: integer L1 sums [B][O]
    int* l2_raw;              // dense: integer L2 sums [B][L2] (forward-only mode writes, backward mode reads)
    const float* b1_master;   // dense: folded master L1 bias [S][O] and its i32 at 8128
    const int* b1_int;
    const float* l2b_master;  // dense: master L2 / L3 biases (rounded to 8128 for the integer layers)
    const float* l3b_master;
};

__host__ __device__ inline int head_partial_len(int l2, int i2, int o) { return l2 * i2 + 2 * l2 + 1 + o + 1; }

// Thread per sample (blockDim = kSfnnTile).  H / L2: compile-time dims, or 0
// for runtime dims up to the kSfnnMax* bounds.
template <int H, int L2, bool DENSE>
__global__ void __launch_bounds__(kSfnnTile) head_kernel(HeadArgs a) {
    constexpr int kH = H > 0 ? H : (kSfnnMaxL1Out - 1);
    constexpr int kL2 = L2 > 0 ? L2 : kSfnnMaxL2;
    constexpr int kI2 = 2 * kH;
    const int hdim = H > 0 ? H : a.l1_hidden;
    const int l2n = L2 > 0 ? L2 : a.l2_size;
    const int i2n = 2 * hdim;
    const int O = a.l1_out;
    extern __shared__ float sm[];
    float* w2e = sm;                          // [l2n][i2n]
    float* b2e = w2e + l2n * i2n;             // [l2n]
    float* w3e = b2e + l2n;                   // [l2n]
    float* b3e = w3e + l2n;                   // [1]
    float* st_g2 = b3e + 1;                   // [T][l2n] masked L2 gradient
    float* st_in = st_g2 + kSfnnTile * l2n;   // [T][i2n]
    float* st_l2 = st_in + kSfnnTile * i2n;   // [T][l2n]
    float* st_go = st_l2 + kSfnnTile * l2n;   // [T]
    float* st_g1 = st_go + kSfnnTile;         // [T][O]
    float* st_ls = st_g1 + kSfnnTile * O;     // [T]
    int* w2i = reinterpret_cast<int*>(st_ls + kSfnnTile);  // dense: integer weights / biases
    int* b2i = w2i + l2n * i2n;
    int* w3i = b2i + l2n;
    int* b3i = w3i + l2n;

    const int t = blockIdx.x;
    if (t >= *a.tiles.n_tiles) return;
    const int s = a.tiles.key[t];
    const bool valid = s < a.stacks;
    const int pb = a.tiles.begin[t], pe = a.tiles.end[t];
    if (valid) {
        // Effective weights: bucket + alpha * shared (cu:2449-2552).
        // Layer QAT fake-quantises the staged values (layer_qat_vector_kernel, cu:9294).
        for (int i = threadIdx.x; i < l2n * i2n; i += blockDim.x) {
            float w = a.l2w[static_cast<size_t>(s) * l2n * i2n + i];
            if (a.l2fw != nullptr) w = fmaf(a.alpha, a.l2fw[i], w);
            if (a.qat_l2) w = qat_q64(w);
            w2e[i] = w;
            if (DENSE) w2i[i] = qat_int64(w);
        }
        for (int o = threadIdx.x; o < l2n; o += blockDim.x) {
            float b = a.l2b != nullptr ? a.l2b[s * l2n + o] : 0.0f;
            if (a.l2fb != nullptr) b = fmaf(a.alpha, a.l2fb[o], b);
            if (a.qat_l2) b = qat_q8128(b);
            b2e[o] = b;
            float w = a.l3w[s * l2n + o];
            if (a.l3fw != nullptr) w = fmaf(a.alpha, a.l3fw[o], w);
            if (a.qat_l3) w = qat_q64(w);
            w3e[o] = w;
            if (DENSE) {
                w3i[o] = qat_int64(w);
                b2i[o] = qat_bias_int(a.l2b_master[s * l2n + o]);
            }
        }
        if (threadIdx.x == 0) {
            float b = a.l3b != nullptr ? a.l3b[s] : 0.0f;
            if (a.l3fb != nullptr) b = fmaf(a.alpha, a.l3fb[0], b);
            if (a.qat_l3) b = qat_q8128(b);
            b3e[0] = b;
            if (DENSE) b3i[0] = qat_bias_int(a.l3b_master[s]);
        }
    }
    __syncthreads();

    const int lt = threadIdx.x;
    const int p = pb + lt;
    if (p < pe) {
        const int b = a.tiles.order[p];
        float in[kI2], l2v[kL2], hid[kH];
        int r2[DENSE ? kL2 : 1];
        float out = 0.0f;
        const float* l1r = a.l1 + static_cast<size_t>(b) * O;
#pragma unroll
        for (int i = 0; i < kH; ++i) hid[i] = (H > 0 || i < hdim) ? l1r[i] : 0.0f;
        if (DENSE && a.mode != kHeadBackward) {
            // Integer L2 input / L2 / L3 + skip (cu:6282-6320).
            if (valid) {
                const int* r1 = a.l1_raw + static_cast<size_t>(b) * O;
                int ii[kI2];
#pragma unroll
                for (int i = 0; i < kH; ++i) {
                    if (H > 0 || i < hdim) {
                        const long long x = r1[i];
                        const int sq = static_cast<int>(min(127LL, (x * x) >> 19));
                        const int lin = max(0, min(127, r1[i] >> 6));
                        ii[i] = sq;
                        ii[hdim + i] = lin;
                        in[i] = qat_on_lattice(sq);
                        in[hdim + i] = qat_on_lattice(lin);
                    }
                }
                long long outr = b3i[0];
#pragma unroll
                for (int o = 0; o < kL2; ++o) {
                    if (L2 > 0 || o < l2n) {
                        long long sum = b2i[o];
                        const int* wr = w2i + o * i2n;
#pragma unroll
                        for (int i = 0; i < kI2; ++i)
                            if (H > 0 || i < i2n) sum += static_cast<long long>(ii[i]) * wr[i];
                        r2[o] = static_cast<int>(sum);
                        const int v = max(0, min(127, r2[o] >> 6));
                        l2v[o] = qat_on_lattice(v);
                        outr += static_cast<long long>(v) * w3i[o];
                    }
                }
                if (a.l1_skip) outr += r1[hdim];
                out = qat_raw_to_float(outr);
            } else {
#pragma unroll
                for (int i = 0; i < kI2; ++i) in[i] = 0.0f;
#pragma unroll
                for (int o = 0; o < kL2; ++o) {
                    l2v[o] = 0.0f;
                    r2[o] = 0;
                }
            }
            if (a.mode == kHeadForward && a.l2_raw != nullptr) {
#pragma unroll
                for (int o = 0; o < kL2; ++o)
                    if (L2 > 0 || o < l2n) a.l2_raw[static_cast<size_t>(b) * l2n + o] = r2[o];
            }
            float* ir = a.l2_input + static_cast<size_t>(b) * i2n;
            float* lr = a.l2 + static_cast<size_t>(b) * l2n;
#pragma unroll
            for (int i = 0; i < kI2; ++i)
                if (H > 0 || i < i2n) ir[i] = in[i];
#pragma unroll
            for (int o = 0; o < kL2; ++o)
                if (L2 > 0 || o < l2n) lr[o] = l2v[o];
            a.output[b] = out;
        } else if (a.mode != kHeadBackward) {
            if (valid) {
                // L2 input: [SqrCReLU | CReLU] of the hidden L1 outputs (cu:2428-2447).
#pragma unroll
                for (int i = 0; i < kH; ++i) {
                    if (H > 0 || i < hdim) {
                        const float av = fabsf(hid[i]);
                        in[i] = crelu01(av * av * kPairScale);
                        in[hdim + i] = crelu01(hid[i]);
                    }
                }
#pragma unroll
                for (int o = 0; o < kL2; ++o) {
                    if (L2 > 0 || o < l2n) {
                        float sum = b2e[o];
                        const float* wr = w2e + o * i2n;
#pragma unroll
                        for (int i = 0; i < kI2; ++i)
                            if (H > 0 || i < i2n) sum = fmaf(in[i], wr[i], sum);
                        l2v[o] = crelu01(sum);
                    }
                }
                out = b3e[0];
#pragma unroll
                for (int o = 0; o < kL2; ++o)
                    if (L2 > 0 || o < l2n) out = fmaf(l2v[o], w3e[o], out);
                if (a.l1_skip) out += l1r[hdim];
            } else {
#pragma unroll
                for (int i = 0; i < kI2; ++i) in[i] = 0.0f;
#pragma unroll
                for (int o = 0; o < kL2; ++o) l2v[o] = 0.0f;
            }
            float* ir = a.l2_input + static_cast<size_t>(b) * i2n;
            float* lr = a.l2 + static_cast<size_t>(b) * l2n;
#pragma unroll
            for (int i = 0; i < kI2; ++i)
                if (H > 0 || i < i2n) ir[i] = in[i];
#pragma unroll
            for (int o = 0; o < kL2; ++o)
                if (L2 > 0 || o < l2n) lr[o] = l2v[o];
            a.output[b] = out;
        } else {
            const float* ir = a.l2_input + static_cast<size_t>(b) * i2n;
            const float* lr = a.l2 + static_cast<size_t>(b) * l2n;
#pragma unroll
            for (int i = 0; i < kI2; ++i) in[i] = (H > 0 || i < i2n) ? ir[i] : 0.0f;
#pragma unroll
            for (int o = 0; o < kL2; ++o) l2v[o] = (L2 > 0 || o < l2n) ? lr[o] : 0.0f;
            if (DENSE) {
#pragma unroll
                for (int o = 0; o < kL2; ++o)
                    r2[o] = (valid && (L2 > 0 || o < l2n)) ? a.l2_raw[static_cast<size_t>(b) * l2n + o] : 0;
            }
        }
        if (a.mode != kHeadForward) {
            float gout = 0.0f, loss = 0.0f;
            if (a.mode == kHeadTrain) {
                loss = sample_loss(a.loss, out, a.targets[b], a.entry_weights[b], &gout);
                a.per_sample[b] = loss;
                a.mog[b] = gout;
            } else {
                gout = a.mog[b];
            }
            float* g1r = a.g1 + static_cast<size_t>(b) * O;
            float g2m[kL2], gin[kI2];
            if (valid) {
                // L3 backward (cu:3324-3430): unmasked L2 gradient; CReLU mask in L2 backward.
#pragma unroll
                for (int o = 0; o < kL2; ++o) {
                    if (L2 > 0 || o < l2n) {
                        const float g = gout * w3e[o];
                        if (DENSE) {
                            // Continuous STE of the integer CReLU (cu:6322-6342): zero
                            // outside [0, 8128]; at the edges the side of the rounded-off
                            // master-bias fraction decides.
                            const int x = r2[o];
                            float gg = g;
                            if (x < 0 || x > 8128) {
                                gg = 0.0f;
                            } else if (x == 0 || x == 8128) {
                                const double bias = fmin(2147483647.0, fmax(-2147483648.0,
                                    static_cast<double>(a.l2b_master[s * l2n + o]) * 8128.0));
                                const double fraction = bias - round(bias);
                                if ((x == 0 && fraction <= 0.0) || (x == 8128 && fraction >= 0.0)) gg = 0.0f;
                            }
                            g2m[o] = gg;
                            if (a.l2_gradients != nullptr) a.l2_gradients[static_cast<size_t>(b) * l2n + o] = gg;
                        } else {
                            if (a.l2_gradients != nullptr) a.l2_gradients[static_cast<size_t>(b) * l2n + o] = g;
                            g2m[o] = crelu_grad(l2v[o], g);
                        }
                    } else {
                        g2m[o] = 0.0f;
                    }
                }
#pragma unroll
                for (int i = 0; i < kI2; ++i) {
                    if (H > 0 || i < i2n) {
                        float sum = 0.0f;
#pragma unroll
                        for (int o = 0; o < kL2; ++o)
                            if (L2 > 0 || o < l2n) sum = fmaf(g2m[o], w2e[o * i2n + i], sum);
                        gin[i] = sum;
                        if (a.l2_input_gradients != nullptr)
                            a.l2_input_gradients[static_cast<size_t>(b) * i2n + i] = sum;
                    }
                }
                // cu:3709-3770: SqrCReLU branch d/dx (x^2 * 127/128) = 2x * 127/128
                // while x^2 * 127/128 is inside (0, 1); CReLU branch while x is.
#pragma unroll
                for (int i = 0; i < kH; ++i) {
                    if (H > 0 || i < hdim) {
                        float v = hid[i];
                        bool sq_on, lin_on;
                        if (DENSE) {
                            // STE from the pre-rounding L1 value: raw / 8128 plus the
                            // rounded-off part of the master bias (cu:3730-3766).
                            const float master = a.b1_master[s * O + i];
                            const int qi = a.b1_int[s * O + i];
                            float frac;
                            if (qi >= -16777216 && qi <= 16777216) {
                                frac = __fmaf_rn(master, 8128.0f, -static_cast<float>(qi));
                            } else {
                                const double scaled = fmin(2147483647.0, fmax(-2147483648.0,
                                                                              static_cast<double>(master) * 8128.0));
                                frac = static_cast<float>(scaled - static_cast<double>(qi));
                            }
                            v = __fmaf_rn(frac, __fdiv_rn(1.0f, 8128.0f), v);
                            const float cs = fabsf(v) * fabsf(v) * kPairScale;
                            sq_on = cs > 0.0f && cs < 1.0f;
                            lin_on = v > 0.0f && v < 1.0f;
                            const int raw = a.l1_raw[static_cast<size_t>(b) * O + i];
                            if (raw == 0) lin_on = frac > 0.0f;
                            else if (raw == 8128) lin_on = frac < 0.0f;
                            if (raw == 8160 || raw == -8160) {
                                const double xd = static_cast<double>(raw) + static_cast<double>(frac);
                                sq_on = xd * xd * 127.0 < 128.0 * 8128.0 * 8128.0;
                            }
                        } else {
                            const float cs = fabsf(v) * fabsf(v) * kPairScale;
                            sq_on = cs > 0.0f && cs < 1.0f;
                            lin_on = v > 0.0f && v < 1.0f;
                        }
                        const float sg = sq_on ? gin[i] * (2.0f * v * kPairScale) : 0.0f;
                        const float lg = lin_on ? gin[hdim + i] : 0.0f;
                        g1r[i] = sg + lg;
                        st_g1[lt * O + i] = sg + lg;
                    }
                }
            } else {
#pragma unroll
                for (int o = 0; o < kL2; ++o) {
                    g2m[o] = 0.0f;
                    if ((L2 > 0 || o < l2n) && a.l2_gradients != nullptr)
                        a.l2_gradients[static_cast<size_t>(b) * l2n + o] = 0.0f;
                }
#pragma unroll
                for (int i = 0; i < kI2; ++i)
                    if ((H > 0 || i < i2n) && a.l2_input_gradients != nullptr)
                        a.l2_input_gradients[static_cast<size_t>(b) * i2n + i] = 0.0f;
                for (int i = 0; i < hdim; ++i) {
                    g1r[i] = 0.0f;
                    st_g1[lt * O + i] = 0.0f;
                }
            }
            if (a.l1_skip) {
                g1r[hdim] = gout;  // PSQT skip: d out / d l1[hidden] = 1 (cu:3433-3437)
                st_g1[lt * O + hdim] = valid ? gout : 0.0f;
            }
#pragma unroll
            for (int o = 0; o < kL2; ++o)
                if (L2 > 0 || o < l2n) {
                    st_g2[lt * l2n + o] = g2m[o];
                    st_l2[lt * l2n + o] = l2v[o];
                }
#pragma unroll
            for (int i = 0; i < kI2; ++i)
                if (H > 0 || i < i2n) st_in[lt * i2n + i] = in[i];
            st_go[lt] = valid ? gout : 0.0f;
            st_ls[lt] = loss;
        }
    }
    if (a.mode == kHeadForward) return;
    __syncthreads();
    // Per-tile partial sums, samples in tile order.
    const int n = pe - pb;
    const int P = head_partial_len(l2n, i2n, O);
    float* part = a.partials + static_cast<size_t>(t) * P;
    for (int j = threadIdx.x; j < P; j += blockDim.x) {
        float sum = 0.0f;
        int r = j;
        if (r < l2n * i2n) {
            const int o = r / i2n, i = r - o * i2n;
            for (int q = 0; q < n; ++q) sum = fmaf(st_g2[q * l2n + o], st_in[q * i2n + i], sum);
        } else if ((r -= l2n * i2n) < l2n) {
            for (int q = 0; q < n; ++q) sum += st_g2[q * l2n + r];
        } else if ((r -= l2n) < l2n) {
            for (int q = 0; q < n; ++q) sum = fmaf(st_go[q], st_l2[q * l2n + r], sum);
        } else if ((r -= l2n) < 1) {
            for (int q = 0; q < n; ++q) sum += st_go[q];
        } else if ((r -= 1) < O) {
            for (int q = 0; q < n; ++q) sum += st_g1[q * O + r];
        } else {
            for (int q = 0; q < n; ++q) sum += st_ls[q];
        }
        part[j] = sum;
    }
}

// ------------------------------------------------------------------ L1 backward
struct L1BackArgs {
    Tiles tiles;
    const float* g1;     // [B][O]
    const float* w_eff;  // [stacks][width][O]
    const float* l0[2];  // ClippedReLU FT output per perspective
    const float* combined;  // dense QAT: the lattice FT output (dL1w uses it); null: recomputed
    // fused step: pre-activation gradients in king order, row rank[h]
    float* pregrad_sorted;
    __nv_bfloat16* pregrad_hi;  // optional: the same rows as bf16 planes G = hi + lo (tensor-core heavy keys)
    __nv_bfloat16* pregrad_lo;
    const int* rank;
    // reference backward buffers (null in the fused step)
    float* combined_gradients;
    float* l0_gradients[2];
    float* pre_gradients[2];
    float* dw1_partials;  // [max_tiles][O][width]
    float* l0b_partials;  // [max_tiles][2][width]
    int width;
    int out_dim;
    int stacks;
};

// Thread per combined column i of a 256-column chunk; column i belongs to
// perspective v = i / (width/2) and pairs FT outputs j and j + width/2
// (pairwise backward, cu:4376-4440).
template <int O>
__global__ void __launch_bounds__(256) l1_backward_kernel(L1BackArgs a) {
    constexpr int kO = O > 0 ? O : kSfnnMaxL1Out;
    constexpr int kU = 4;  // samples in flight per thread
    __shared__ float g1s[kSfnnTile * kSfnnMaxL1Out];
    __shared__ int bs[kSfnnTile];
    __shared__ int rs[kSfnnTile * 2];
    const int t = blockIdx.x;
    if (t >= *a.tiles.n_tiles) return;
    const int s = a.tiles.key[t];
    const int pb = a.tiles.begin[t], pe = a.tiles.end[t];
    const int n = pe - pb;
    const int od = O > 0 ? O : a.out_dim;
    const int W = a.width, half = W / 2;
    const int i = blockIdx.y * 256 + threadIdx.x;
    const bool valid = s < a.stacks;
    for (int q = threadIdx.x; q < n; q += blockDim.x) {
        const int b = a.tiles.order[pb + q];
        bs[q] = b;
        if (a.rank != nullptr) {
            rs[2 * q] = a.rank[2 * b];
            rs[2 * q + 1] = a.rank[2 * b + 1];
        }
    }
    for (int q = threadIdx.x; q < n * od; q += blockDim.x)
        g1s[q] = valid ? a.g1[static_cast<size_t>(a.tiles.order[pb + q / od]) * od + q % od] : 0.0f;
    __syncthreads();
    if (i >= W) return;
    const int v = i >= half ? 1 : 0;
    const int j = i - v * half;
    float wcol[kO], dw[kO];
#pragma unroll
    for (int o = 0; o < kO; ++o) {
        wcol[o] = (valid && (O > 0 || o < od)) ? a.w_eff[(static_cast<size_t>(s) * W + i) * od + o] : 0.0f;
        dw[o] = 0.0f;
    }
    float p0sum = 0.0f, p1sum = 0.0f;
    const float* x = v ? a.l0[1] : a.l0[0];
    for (int q0 = 0; q0 < n; q0 += kU) {
        // Issue the loads of kU samples before using any of them.
        float xa[kU], xb[kU], cc[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            const int q = q0 + u;
            if (q < n) {
                const size_t row = static_cast<size_t>(bs[q]) * W;
                xa[u] = x[row + j];
                xb[u] = x[row + j + half];
                if (a.combined != nullptr) cc[u] = a.combined[row + i];
            }
        }
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            const int q = q0 + u;
            if (q >= n) break;
            const float x0 = xa[u], x1 = xb[u];
            const float c = a.combined != nullptr ? cc[u] : x0 * x1 * kPairScale;
            float dc = 0.0f;
#pragma unroll
            for (int o = 0; o < kO; ++o) {
                if (O > 0 || o < od) {
                    const float g = g1s[q * od + o];
                    dc = fmaf(g, wcol[o], dc);
                    dw[o] = fmaf(g, c, dw[o]);
                }
            }
            const float pg = dc * kPairScale;
            const float u0 = pg * x1, u1 = pg * x0;
            const float p0 = crelu_grad(x0, u0), p1 = crelu_grad(x1, u1);
            if (a.pregrad_sorted != nullptr) {
                const size_t ro = static_cast<size_t>(rs[2 * q + v]) * W;
                float* pr = a.pregrad_sorted + ro;
                pr[j] = p0;
                pr[j + half] = p1;
                if (a.pregrad_hi != nullptr) {
                    const __nv_bfloat16 h0 = __float2bfloat16_rn(p0), h1 = __float2bfloat16_rn(p1);
                    a.pregrad_hi[ro + j] = h0;
                    a.pregrad_hi[ro + j + half] = h1;
                    a.pregrad_lo[ro + j] = __float2bfloat16_rn(p0 - __bfloat162float(h0));
                    a.pregrad_lo[ro + j + half] = __float2bfloat16_rn(p1 - __bfloat162float(h1));
                }
            }
            if (a.combined_gradients != nullptr) {
                const size_t row = static_cast<size_t>(bs[q]) * W;
                a.combined_gradients[row + i] = dc;
                float* lg = v ? a.l0_gradients[1] : a.l0_gradients[0];
                float* pg = v ? a.pre_gradients[1] : a.pre_gradients[0];
                lg[row + j] = u0;
                lg[row + j + half] = u1;
                pg[row + j] = p0;
                pg[row + j + half] = p1;
            }
            p0sum += p0;
            p1sum += p1;
        }
    }
    float* dwp = a.dw1_partials + static_cast<size_t>(t) * od * W;
#pragma unroll
    for (int o = 0; o < kO; ++o)
        if (O > 0 || o < od) dwp[static_cast<size_t>(o) * W + i] = dw[o];
    float* bp = a.l0b_partials + (static_cast<size_t>(t) * 2 + v) * W;
    bp[j] = p0sum;
    bp[j + half] = p1sum;
}

// ------------------------------------------------------------------ finalize
struct FinalArgs {
    Tiles tiles;
    const float* head_partials;
    const float* dw1_partials;
    const float* l0b_partials;
    float* dst[kSfGroups];  // gradient destinations per small group (null: group absent)
    int accumulate;         // dst += gradient (reference backward) or dst = gradient
    float* weighted_sum;    // optional loss outputs
    float* mean;
    float alpha;
    int width;
    int out_dim;
    int l2_size;
    int l2_in;
    int stacks;
    int batch;
};

__device__ __forceinline__ void put(const FinalArgs& a, int g, size_t i, float v) {
    float* d = a.dst[g];
    if (d == nullptr) return;
    d[i] = a.accumulate ? d[i] + v : v;
}

// Work items (flattened over blockIdx / threadIdx):
//   [0, W)                   l0b[j]
//   [W, W + S*O*W)           l1w[s][o][i]
//   + W*O                    l1fw[i][o]   (alpha * sum over all valid tiles)
//   + S*P                    head groups per bucket (l2w, l2b, l3w, l3b, l1b)
//   + P                      shared head groups (l2fw, l2fb, l3fw, l3fb, l1fb) and the loss
__global__ void finalize_kernel(FinalArgs a) {
    const int W = a.width, O = a.out_dim, L2 = a.l2_size, I2 = a.l2_in, S = a.stacks;
    const int P = head_partial_len(L2, I2, O);
    const size_t n0 = W;
    const size_t n1 = n0 + static_cast<size_t>(S) * O * W;
    const size_t n2 = n1 + static_cast<size_t>(W) * O;
    const size_t n3 = n2 + static_cast<size_t>(S) * P;
    const size_t n4 = n3 + P;
    const size_t t = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= n4) return;
    const int n_tiles = *a.tiles.n_tiles;
    const int valid_tiles = a.tiles.key_first[S];
    if (t < n0) {
        float sum = 0.0f;
        for (int k = 0; k < n_tiles; ++k)
            sum += a.l0b_partials[(static_cast<size_t>(k) * 2) * W + t] +
                   a.l0b_partials[(static_cast<size_t>(k) * 2 + 1) * W + t];
        put(a, kSfL0b, t, sum);
    } else if (t < n1) {
        const size_t r = t - n0;
        const int s = static_cast<int>(r / (static_cast<size_t>(O) * W));
        const size_t oi = r - static_cast<size_t>(s) * O * W;
        float sum = 0.0f;
        for (int k = a.tiles.key_first[s]; k < a.tiles.key_first[s + 1]; ++k)
            sum += a.dw1_partials[static_cast<size_t>(k) * O * W + oi];
        put(a, kSfL1w, r, sum);
    } else if (t < n2) {
        const size_t r = t - n1;  // [i][o]
        const int i = static_cast<int>(r / O), o = static_cast<int>(r % O);
        float sum = 0.0f;
        for (int k = 0; k < valid_tiles; ++k) sum += a.dw1_partials[(static_cast<size_t>(k) * O + o) * W + i];
        put(a, kSfL1fw, r, a.alpha * sum);
    } else if (t < n3) {
        const size_t r = t - n2;
        const int s = static_cast<int>(r / P);
        int j = static_cast<int>(r - static_cast<size_t>(s) * P);
        float sum = 0.0f;
        for (int k = a.tiles.key_first[s]; k < a.tiles.key_first[s + 1]; ++k)
            sum += a.head_partials[static_cast<size_t>(k) * P + j];
        if (j < L2 * I2) put(a, kSfL2w, static_cast<size_t>(s) * L2 * I2 + j, sum);
        else if ((j -= L2 * I2) < L2) put(a, kSfL2b, static_cast<size_t>(s) * L2 + j, sum);
        else if ((j -= L2) < L2) put(a, kSfL3w, static_cast<size_t>(s) * L2 + j, sum);
        else if ((j -= L2) < 1) put(a, kSfL3b, s, sum);
        else if ((j -= 1) < O) put(a, kSfL1b, static_cast<size_t>(s) * O + j, sum);
    } else {
        int j = static_cast<int>(t - n3);
        const bool loss = j == P - 1;
        const int tiles = loss ? n_tiles : valid_tiles;
        float sum = 0.0f;
        for (int k = 0; k < tiles; ++k) sum += a.head_partials[static_cast<size_t>(k) * P + j];
        if (loss) {
            if (a.weighted_sum != nullptr) {
                *a.weighted_sum = sum;
                *a.mean = sum / static_cast<float>(a.batch);
            }
            return;
        }
        sum *= a.alpha;
        if (j < L2 * I2) put(a, kSfL2fw, j, sum);
        else if ((j -= L2 * I2) < L2) put(a, kSfL2fb, j, sum);
        else if ((j -= L2) < L2) put(a, kSfL3fw, j, sum);
        else if ((j -= L2) < 1) put(a, kSfL3fb, 0, sum);
        else if ((j -= 1) < O) put(a, kSfL1fb, j, sum);
    }
}

// ------------------------------------------------------------------ FT rows
struct PieceRowArgs {
    const int* offsets;
    const int* entries;
    const float* src[2];  // gradient row of entry e: src[e & 1] + (e >> 1) * src_stride
    size_t src_stride;
    int pieces;           // P
    int kings;            // rows per piece: row(k, p) = k * P + p
    int virtual_base;     // virtual row of piece p = virtual_base + p; < 0: none
    float alpha;
    int width;
    int col_groups;
    int group_width;
    float* weights;
    float* momentum;
    float* velocity;
    float* slow;
    float* gradients;     // kRowWrite / kRowAccumulate target
    RangerArgs ranger;
    int skip_quiet;
    // The kings are processed in launches of a few king blocks each, so the
    // gradient rows read by one launch (those of its kings' half-positions)
    // stay L2-resident.  The per-piece virtual-row sums carry over between
    // launches in vacc / vany (owned by one warp each: deterministic).
    int king_begin;
    int king_end;
    int first_launch;
    int last_launch;
    float* vacc;          // [pieces][width]
    int* vany;            // [pieces * col_groups]
    // Heavy rows (more than kHeavyRow entries over all their keys, e.g. the
    // piece-squares of the common king squares in real teacher data) are summed
    // beforehand in kHeavySeg-entry segments, each inside one rank tile, by every
    // warp (heavy_segment_kernel); the row kernel then adds the row's segment
    // partials in (tile, segment) order.
    const int* tile_base;        // [kings + 1] rank tiles of each king (tile-keyed index), null: key = row
    int n_keys;                  // keys of the index
    size_t max_entries;          // entries of the index (bounds the segment plan)
    const int* heavy_off;        // [n_keys + 1] exclusive scan of the keys' segment counts
    const float* heavy_partials; // [segments][width]
    int heavy_row;               // rows with more entries are heavy
    int heavy_seg;               // entries per segment
    int heavy_ok;                // the plan fit the scratch (read on the device as well)
    // Heavy keys summed on the tensor cores (ft_rows_mma.cu): slot of each key
    // (-1: light) and the sums [slot][width]; null: the segment plan above.
    const int* key_slot;
    const float* key_partials;
    // Data-parallel peer exchange (kRowWrite): scatter_world > 0 stores row r
    // of the launch's chunk into its owner's receive slot instead of
    // gradients: owner o = (r - chunk_start) / chunk_shard_rows, at row
    // scatter_rank * scatter_slot_rows + chunk_shard_off + (r - chunk_start) -
    // o * chunk_shard_rows of scatter_recv[o].
    float* scatter_recv[kExchangeMaxRanks];
    int scatter_world;
    int scatter_rank;
    size_t scatter_slot_rows;
    size_t chunk_start;
    size_t chunk_shard_rows;
    size_t chunk_shard_off;
};

// Peer-exchange descriptor of the row launches (host side): per launch j its
// chunk and, at a chunk's last launch, the chunk index to signal.
struct RowScatter {
    float* recv[kExchangeMaxRanks];
    int world;
    int rank;
    size_t slot_rows;
    const size_t* chunk_start;
    const size_t* shard_rows;
    const size_t* shard_off;
    const long long* signal;
    PeerFlags flags;
    int epoch;
    PeerBuffers small;       // every rank's small-gradient receive buffer
    size_t small_len;        // 0: the small gradient stays local
    size_t small_flag_base;
};

constexpr int kHeavyRow = 128;  // FT row phase on king-concentrated batches: 512 -> 3.75 ms, 128 -> 3.03 ms
constexpr int kHeavySeg = 128;

// Column layout of a warp's chunk: with VEC = 8 a lane owns columns
// [c, c+4) and [c+128, c+132) for c = 4 * lane, so each warp-wide float4 access
// covers 512 contiguous bytes (4 L1 wavefronts instead of 8).
template <int VEC>
__device__ __forceinline__ int lane_col(int c0, int it, int lane) {
    if constexpr (VEC == 8) return c0 + it * 256 + lane * 4;
    return c0 + (it * 32 + lane) * VEC;
}

template <int VEC>
__device__ __forceinline__ void ldv(const float* p, float* o) {
    if constexpr (VEC == 8) {
        const float4 x = *reinterpret_cast<const float4*>(p);
        const float4 y = *reinterpret_cast<const float4*>(p + 128);
        o[0] = x.x; o[1] = x.y; o[2] = x.z; o[3] = x.w; o[4] = y.x; o[5] = y.y; o[6] = y.z; o[7] = y.w;
    } else if constexpr (VEC == 4) {
        const float4 x = *reinterpret_cast<const float4*>(p);
        o[0] = x.x; o[1] = x.y; o[2] = x.z; o[3] = x.w;
    } else {
        o[0] = *p;
    }
}

template <int VEC>
__device__ __forceinline__ void stv(float* p, const float* v) {
    if constexpr (VEC == 8) {
        *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
        *reinterpret_cast<float4*>(p + 128) = make_float4(v[4], v[5], v[6], v[7]);
    } else if constexpr (VEC == 4) {
        *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
    } else {
        *p = v[0];
    }
}

// The Ranger update of one column chunk from its loaded weights and moments.
template <int VEC>
__device__ __forceinline__ void ranger_row_update(const PieceRowArgs& a, size_t off, const float* g, bool quiet_row,
                                                  float* seen, float* w, float* m, float* v) {
#pragma unroll
    for (int e = 0; e < VEC; ++e) seen[e] = g[e];
    if (quiet_row && a.skip_quiet && !a.ranger.do_lookahead) {
        bool quiet = true;
#pragma unroll
        for (int e = 0; e < VEC; ++e)
            quiet = quiet && (__float_as_uint(m[e]) | __float_as_uint(v[e])) == 0u && weight_is_quiet(w[e], a.ranger);
        if (quiet) return;
    }
#pragma unroll
    for (int e = 0; e < VEC; ++e) radam_coordinate(a.ranger.gradient_factor * g[e], a.ranger, w[e], m[e], v[e]);
    if (a.ranger.do_lookahead) {
        float sl[VEC];
        ldv<VEC>(a.slow + off, sl);
#pragma unroll
        for (int e = 0; e < VEC; ++e) w[e] = lookahead_coordinate(w[e], sl[e], a.ranger);
        stv<VEC>(a.slow + off, w);
    }
    stv<VEC>(a.weights + off, w);
    stv<VEC>(a.momentum + off, m);
    stv<VEC>(a.velocity + off, v);
}

// Where kRowWrite stores the gradient at offset row * width + column: the
// local gradient table, or the row owner's receive slot (peer exchange).
__device__ __forceinline__ float* row_write_target(const PieceRowArgs& a, size_t off) {
    if (a.scatter_world == 0) return a.gradients + off;
    const size_t row = off / static_cast<size_t>(a.width);
    const size_t col = off - row * static_cast<size_t>(a.width);
    const size_t rel = row - a.chunk_start;
    const size_t owner = rel / a.chunk_shard_rows;
    const size_t local = a.chunk_shard_off + (rel - owner * a.chunk_shard_rows);
    return a.scatter_recv[owner] +
           (static_cast<size_t>(a.scatter_rank) * a.scatter_slot_rows + local) * static_cast<size_t>(a.width) + col;
}

// Applies the row update for one column chunk: Ranger / write / accumulate.
// `seen` receives the row's gradient as the virtual row sees it (the
// accumulated value in accumulate mode).
template <int VEC, int MODE>
__device__ __forceinline__ void row_update(const PieceRowArgs& a, size_t off, const float* g, bool quiet_row,
                                           float* seen) {
    if constexpr (MODE == kRowWrite) {
        stv<VEC>(row_write_target(a, off), g);
#pragma unroll
        for (int e = 0; e < VEC; ++e) seen[e] = g[e];
    } else if constexpr (MODE == kRowAccumulate) {
        float x[VEC];
        ldv<VEC>(a.gradients + off, x);
#pragma unroll
        for (int e = 0; e < VEC; ++e) x[e] += g[e];
        stv<VEC>(a.gradients + off, x);
#pragma unroll
        for (int e = 0; e < VEC; ++e) seen[e] = x[e];
    } else {
        float w[VEC], m[VEC], v[VEC];
        ldv<VEC>(a.weights + off, w);
        ldv<VEC>(a.momentum + off, m);
        ldv<VEC>(a.velocity + off, v);
        ranger_row_update<VEC>(a, off, g, quiet_row, seen, w, m, v);
    }
}

// Sum of the gradient rows of entries elist[0, n) over a lane's columns:
// entry ids are broadcast 32 at a time, kGatherDepth rows in flight per lane.
constexpr int kGatherDepth = 4;
template <int VEC, int DEPTH = kGatherDepth>
__device__ __forceinline__ void gather_sum(const PieceRowArgs& a, const int* __restrict__ elist, int n, int c,
                                           bool active, int lane, float* acc) {
    for (int q0 = 0; q0 < n; q0 += 32) {
        const int m = min(32, n - q0);
        const int mine = lane < m ? __ldg(elist + q0 + lane) : 0;
        int q = 0;
        for (; q + DEPTH <= m; q += DEPTH) {
            int en[DEPTH];
#pragma unroll
            for (int u = 0; u < DEPTH; ++u) en[u] = __shfl_sync(kFull, mine, q + u);
            if (active) {
                float x[DEPTH][VEC];
#pragma unroll
                for (int u = 0; u < DEPTH; ++u)
                    ldv<VEC>(a.src[en[u] & 1] + static_cast<size_t>(en[u] >> 1) * a.src_stride + c, x[u]);
#pragma unroll
                for (int u = 0; u < DEPTH; ++u)
#pragma unroll
                    for (int e = 0; e < VEC; ++e) acc[e] += x[u][e];
            }
        }
        for (; q < m; ++q) {
            const int en = __shfl_sync(kFull, mine, q);
            if (active) {
                float x[VEC];
                ldv<VEC>(a.src[en & 1] + static_cast<size_t>(en >> 1) * a.src_stride + c, x);
#pragma unroll
                for (int e = 0; e < VEC; ++e) acc[e] += x[e];
            }
        }
    }
}

// One warp per (piece, column group).  The piece's rows are visited in king
// order; every warp walks the kings at about the same pace, so the gradient
// rows being read at any time belong to a few kings' half-positions (L2).
template <int VEC, int ITERS, int MODE>
__device__ __forceinline__ void piece_rows(const PieceRowArgs& a, int gw, int lane) {
    const int p = gw / a.col_groups;
    const int c0 = (gw - p * a.col_groups) * a.group_width;
    const int c_end = min(a.width, c0 + a.group_width);
    const bool has_virtual = a.virtual_base >= 0;
    float vacc[ITERS][VEC];
    bool any = false;
    float* vsave = a.vacc + static_cast<size_t>(p) * a.width;
#pragma unroll
    for (int it = 0; it < ITERS; ++it) {
        const int c = lane_col<VEC>(c0, it, lane);
        if (has_virtual && !a.first_launch && c < c_end) {
            ldv<VEC>(vsave + c, vacc[it]);
        } else {
#pragma unroll
            for (int e = 0; e < VEC; ++e) vacc[it][e] = 0.0f;
        }
    }
    if (has_virtual && !a.first_launch) any = a.vany[gw] != 0;
    for (int k = a.king_begin; k < a.king_end; ++k) {
        const int row = k * a.pieces + p;
        const size_t row_off = static_cast<size_t>(row) * a.width;
        // the row's keys: one per rank tile of king k (or the row itself)
        const int t0 = a.tile_base != nullptr ? __ldg(a.tile_base + k) : k;
        const int t1 = a.tile_base != nullptr ? __ldg(a.tile_base + k + 1) : k + 1;
        float acc[ITERS][VEC];
#pragma unroll
        for (int it = 0; it < ITERS; ++it)
#pragma unroll
            for (int e = 0; e < VEC; ++e) acc[it][e] = 0.0f;
        int total = 0;
        for (int t = t0; t < t1; ++t) {
            const int key = t * a.pieces + p;
            const int beg = a.offsets[key];
            const int n = a.offsets[key + 1] - beg;
            if (n == 0) continue;
            total += n;
            const int* elist = a.entries + beg;  // ascending up to kSortCap entries (sort_inverse_index)
            const int slot = a.key_slot != nullptr ? __ldg(a.key_slot + key) : -1;
            int hs = -1;
            if (a.heavy_off != nullptr) {
                const int s0 = __ldg(a.heavy_off + key), s1 = __ldg(a.heavy_off + key + 1);
                if (s1 > s0 && __ldg(a.heavy_off + a.n_keys) <= a.heavy_ok) hs = s0;
            }
#pragma unroll
            for (int it = 0; it < ITERS; ++it) {
                const int c = lane_col<VEC>(c0, it, lane);
                const bool active = c < c_end;
                if (slot >= 0) {
                    if (active) {
                        float x[VEC];
                        ldv<VEC>(a.key_partials + static_cast<size_t>(slot) * a.width + c, x);
#pragma unroll
                        for (int e = 0; e < VEC; ++e) acc[it][e] += x[e];
                    }
                } else if (hs >= 0) {
                    const int nseg = (n + a.heavy_seg - 1) / a.heavy_seg;
                    if (active) {
                        for (int sg = 0; sg < nseg; ++sg) {
                            float x[VEC];
                            ldv<VEC>(a.heavy_partials + static_cast<size_t>(hs + sg) * a.width + c, x);
#pragma unroll
                            for (int e = 0; e < VEC; ++e) acc[it][e] += x[e];
                        }
                    }
                } else {
                    gather_sum<VEC>(a, elist, n, c, active, lane, acc[it]);
                }
            }
        }
        any = any || total > 0;
#pragma unroll
        for (int it = 0; it < ITERS; ++it) {
            const int c = lane_col<VEC>(c0, it, lane);
            if (c < c_end) {
                float seen[VEC];
                row_update<VEC, MODE>(a, row_off + c, acc[it], total == 0, seen);
#pragma unroll
                for (int e = 0; e < VEC; ++e) vacc[it][e] += seen[e];
            }
        }
        __syncwarp();
    }
    if (!has_virtual) return;
    if (!a.last_launch) {
#pragma unroll
        for (int it = 0; it < ITERS; ++it) {
            const int c = lane_col<VEC>(c0, it, lane);
            if (c < c_end) stv<VEC>(vsave + c, vacc[it]);
        }
        if (lane == 0) a.vany[gw] = any ? 1 : 0;
        return;
    }
    const size_t vrow = static_cast<size_t>(a.virtual_base + p) * a.width;
#pragma unroll
    for (int it = 0; it < ITERS; ++it) {
        const int c = lane_col<VEC>(c0, it, lane);
        if (c >= c_end) continue;
        float g[VEC], seen[VEC];
#pragma unroll
        for (int e = 0; e < VEC; ++e) g[e] = a.alpha * vacc[it][e];
        if constexpr (MODE == kRowAccumulate) {
            stv<VEC>(a.gradients + vrow + c, g);  // cu:4950-4985 overwrites the factor row's gradient
        } else {
            row_update<VEC, MODE>(a, vrow + c, g, !any, seen);
        }
    }
}

template <int VEC, int ITERS, int MODE>
__global__ void __launch_bounds__(kPieceRowWarps * 32, 3) piece_row_kernel(PieceRowArgs a) {
    const int lane = threadIdx.x & 31;
    const int items = a.pieces * a.col_groups;
    for (int gw = blockIdx.x * kPieceRowWarps + (threadIdx.x >> 5); gw < items; gw += gridDim.x * kPieceRowWarps)
        piece_rows<VEC, ITERS, MODE>(a, gw, lane);
    if (MODE == kRowWrite && a.scatter_world > 0) __threadfence_system();  // peer stores before the chunk's signal
}

// Segments per key: a row (k, p) is heavy when its entries over all its keys
// (the rank tiles of king k) exceed heavy_row; each key of a heavy row is cut
// into ceil(n / heavy_seg) segments, so a segment never crosses a rank tile.
// Keys of unused tiles get 0.  Thread i covers row i and key i.
__global__ void heavy_count_kernel(const int* __restrict__ offsets, const int* __restrict__ tile_base, int kings,
                                   int pieces, int rows, int keys, int heavy_row, int heavy_seg,
                                   int* __restrict__ seg_count) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    const int used_keys = tile_base != nullptr ? tile_base[kings] * pieces : rows;
    if (i < keys && i >= used_keys) seg_count[i] = 0;
    if (i >= rows) return;
    const int k = i / pieces, p = i - k * pieces;
    const int t0 = tile_base != nullptr ? tile_base[k] : i;
    const int t1 = tile_base != nullptr ? tile_base[k + 1] : i + 1;
    const int stride = tile_base != nullptr ? pieces : 1;
    const int base = tile_base != nullptr ? p : 0;
    int total = 0;
    for (int t = t0; t < t1; ++t) total += offsets[t * stride + base + 1] - offsets[t * stride + base];
    const bool heavy = total > heavy_row;
    for (int t = t0; t < t1; ++t) {
        const int key = t * stride + base;
        const int n = offsets[key + 1] - offsets[key];
        seg_count[key] = heavy ? (n + heavy_seg - 1) / heavy_seg : 0;
    }
}

// seg_key[s] = key of segment s (thread per key).
__global__ void heavy_fill_kernel(const int* __restrict__ seg_off, int keys, int max_segments,
                                  int* __restrict__ seg_key) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= keys || seg_off[keys] > max_segments) return;
    for (int s = seg_off[i]; s < seg_off[i + 1]; ++s) seg_key[s] = i;
}

// Partial sums of the heavy rows' segments: warp per (segment, column group),
// persistent over the segment count (segments in key order: tile-major, so the
// warps in flight read the gradient rows of one or two rank tiles).  One CTA
// per SM with 16 rows in flight per lane: the window of segments in flight
// then stays inside L2 and the kernel reads each gradient row from DRAM once
// (0.83 GB a step at B = 65536 instead of 7.4 GB with four CTAs per SM and 4
// rows in flight, at the same L2-throughput-bound duration).  With more segments than the scratch holds no
// row is heavy (heavy_off reads as empty, see piece_rows).
template <int VEC>
__global__ void __launch_bounds__(kPieceRowWarps * 32, 1) heavy_segment_kernel(PieceRowArgs a, int rows,
                                                                               int max_segments,
                                                                               const int* __restrict__ seg_key,
                                                                               float* __restrict__ partials) {
    const int lane = threadIdx.x & 31;
    const int total = a.heavy_off[rows];
    const int items = total <= max_segments ? total * a.col_groups : 0;
    for (int gw = blockIdx.x * kPieceRowWarps + (threadIdx.x >> 5); gw < items; gw += gridDim.x * kPieceRowWarps) {
        const int seg = gw / a.col_groups;
        const int c0 = (gw - seg * a.col_groups) * a.group_width;
        const int c_end = min(a.width, c0 + a.group_width);
        const int row = __ldg(seg_key + seg);
        const int beg = a.offsets[row] + (seg - a.heavy_off[row]) * a.heavy_seg;
        const int n = min(a.heavy_seg, a.offsets[row + 1] - beg);
        const int c = lane_col<VEC>(c0, 0, lane);
        const bool active = c < c_end;
        float acc[VEC];
#pragma unroll
        for (int e = 0; e < VEC; ++e) acc[e] = 0.0f;
        gather_sum<VEC, 16>(a, a.entries + beg, n, c, active, lane, acc);
        if (active) stv<VEC>(partials + static_cast<size_t>(seg) * a.width + c, acc);
    }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

size_t align_floats(size_t n) { return (n + 63) & ~static_cast<size_t>(63); }

// Row ranges each launch of the FT row kernel completes: launch j writes the
// rows of king blocks [3 j, 3 j + 3), the last one also the virtual rows.
// Returns the launch count; row_end[j] = first row after launch j (if given).
int piece_row_launches(const SfnnDims& d, size_t* row_end, size_t cap) {
    const int kings = d.base > 0 ? d.base / kSfnnPieces : 1;
    const int n = (kings + kKingsPerLaunch - 1) / kKingsPerLaunch;
    for (int j = 0; j < n && row_end != nullptr && static_cast<size_t>(j) < cap; ++j)
        row_end[j] = (j == n - 1) ? static_cast<size_t>(d.input_size)
                                  : static_cast<size_t>(kKingsPerLaunch) * (j + 1) * kSfnnPieces;
    return n;
}

template <int MODE>
int launch_piece_rows_mode(BulletOuCudaCppContext* ctx, PieceRowArgs a, int vec, const size_t* row_shift,
                           const cudaEvent_t* events, const RowScatter* scatter) {
    if (scatter != nullptr) {
        for (int r = 0; r < scatter->world; ++r) a.scatter_recv[r] = scatter->recv[r];
        a.scatter_world = scatter->world;
        a.scatter_rank = scatter->rank;
        a.scatter_slot_rows = scatter->slot_rows;
    }
    // Persistent grid: three CTAs per SM, each warp loops over (piece, column
    // group) work items.
    const int warps = a.pieces * a.col_groups;
    const int blocks = std::max(1, std::min((warps + kPieceRowWarps - 1) / kPieceRowWarps, kPieceRowCtas * ctx->sm_count));
    float* const gradients = a.gradients;
    for (int k0 = 0, j = 0; k0 < a.kings; k0 += kKingsPerLaunch, ++j) {
        a.king_begin = k0;
        a.king_end = std::min(a.kings, k0 + kKingsPerLaunch);
        a.first_launch = k0 == 0;
        a.last_launch = a.king_end == a.kings;
        // Data-parallel layout: launch j's rows land row_shift[j] rows further,
        // so each launch's range starts a chunk the collectives can split evenly.
        if (row_shift != nullptr) a.gradients = gradients + row_shift[j] * static_cast<size_t>(a.width);
        if (scatter != nullptr) {
            a.chunk_start = scatter->chunk_start[j];
            a.chunk_shard_rows = scatter->shard_rows[j];
            a.chunk_shard_off = scatter->shard_off[j];
        }
        if (vec == 8) piece_row_kernel<8, 1, MODE><<<blocks, kPieceRowWarps * 32, 0, ctx->stream>>>(a);
        else if (vec == 4) piece_row_kernel<4, 1, MODE><<<blocks, kPieceRowWarps * 32, 0, ctx->stream>>>(a);
        else piece_row_kernel<1, 1, MODE><<<blocks, kPieceRowWarps * 32, 0, ctx->stream>>>(a);
        if (check_launch("SFNN FT row kernel launch") != 0) return -1;
        // peer exchange: the chunk's rows have landed in their owners' slots
        if (scatter != nullptr && scatter->signal[j] >= 0 &&
            launch_exchange_signal(ctx, scatter->flags, scatter->world,
                                   static_cast<size_t>(scatter->signal[j]) * scatter->world + scatter->rank,
                                   scatter->epoch) != 0)
            return -1;
        if (events != nullptr) {
            cudaError_t st = cudaEventRecord(events[j], ctx->stream);
            if (st != cudaSuccess) return fail("cudaEventRecord SFNN row launch", st);
        }
    }
    return 0;
}

// Inputs of the tensor-core heavy-key sums (fused step only): the batch, the
// king sort and the gradient rows as bf16 planes.
struct HeavyMmaInputs {
    const int* rank_base;  // king sort key offsets
    const int* order;      // rank -> half-position
    const int* stm;
    const int* nstm;
    int max_active;
    int max_tiles;
    int rows;
    const __nv_bfloat16* hi;
    const __nv_bfloat16* lo;
};

// The tensor-core plan in its scratch slot; false when it does not apply.
int plan_heavy_mma(BulletOuCudaCppContext* ctx, const PieceRowArgs& a, const HeavyMmaInputs& in, HeavyMmaArgs* m) {
    const size_t keys = static_cast<size_t>(in.max_tiles) * a.pieces;
    const size_t max_slots = heavy_mma_max_slots(a.max_entries, kHeavyMmaThreshold);
    const size_t max_work = heavy_mma_max_work(in.max_tiles, max_slots, a.width);
    const size_t max_mblocks = heavy_mma_max_mblocks(in.max_tiles, max_slots);
    const size_t ints = align_floats(2 * keys + 5 * static_cast<size_t>(in.max_tiles) + 2 + 2 * max_work + 4);
    const size_t part = align_floats(max_slots * static_cast<size_t>(a.width));
    const size_t inc = heavy_mma_incidence_bytes(max_mblocks);
    void* p = nullptr;
    const bool fresh = ctx->scratch[kScratchSfnnHeavyMma].bytes == 0;
    if (scratch_slot(ctx, kScratchSfnnHeavyMma, (ints + part) * sizeof(float) + inc, &p,
                     "cudaMalloc SFNN heavy-key tensor-core plan") != 0)
        return -1;
    int* q = static_cast<int*>(p);
    HeavyMmaPlan& pl = m->plan;
    pl.key_local = q;
    pl.key_slot = q + keys;
    pl.tile_heavy = q + 2 * keys;
    pl.tile_slot = pl.tile_heavy + in.max_tiles;
    pl.tile_r0 = pl.tile_slot + in.max_tiles + 1;
    pl.tile_r1 = pl.tile_r0 + in.max_tiles;
    pl.tile_mb = pl.tile_r1 + in.max_tiles;
    pl.work = pl.tile_mb + in.max_tiles + 1;
    pl.n_work = pl.work + 2 * max_work;
    pl.n_slots = pl.n_work + 1;
    pl.next_work = pl.n_slots + 1;
    pl.error = pl.next_work + 1;
    pl.partials = reinterpret_cast<float*>(q) + ints;
    pl.incidence = reinterpret_cast<float*>(q) + ints + part;
    pl.max_slots = static_cast<int>(std::min<size_t>(max_slots, INT_MAX));
    pl.max_mblocks = static_cast<int>(std::min<size_t>(max_mblocks, INT_MAX));
    pl.max_work = static_cast<int>(std::min<size_t>(max_work, INT_MAX));
    if (fresh) {
        const cudaError_t st = cudaMemsetAsync(pl.error, 0, sizeof(int), ctx->stream);
        if (st != cudaSuccess) return fail("cudaMemsetAsync heavy-key error word", st);
    }
    m->offsets = a.offsets;
    m->tile_base = a.tile_base;
    m->rank_base = in.rank_base;
    m->rank_base_end = 0;
    m->kings = a.kings;
    m->pieces = a.pieces;
    m->tile_ranks = kTileRanks;
    m->max_tiles = in.max_tiles;
    m->threshold = kHeavyMmaThreshold;
    m->order = in.order;
    m->stm = in.stm;
    m->nstm = in.nstm;
    m->max_active = in.max_active;
    m->hi = in.hi;
    m->lo = in.lo;
    m->rows = in.rows;
    m->width = a.width;
    return 0;
}

// Columns per lane of the FT row kernel for these buffers: 8, 4 or 1.
int piece_row_vec(int mode, const PieceRowArgs& a) {
    bool al = aligned16(a.src[0]) && aligned16(a.src[1]) && a.src_stride % 4 == 0;
    if (mode == kRowRanger)
        al = al && aligned16(a.weights) && aligned16(a.momentum) && aligned16(a.velocity) && aligned16(a.slow);
    else
        al = al && aligned16(a.gradients);
    if (al && a.width % 256 == 0) return 8;
    if (al && a.width % 128 == 0) return 4;
    return 1;
}

// Whether launch_piece_rows sums the heavy keys on the tensor cores (then
// their entry lists are not read).
bool piece_rows_use_mma(int mode, const PieceRowArgs& a, const HeavyMmaInputs* mma) {
    return mma != nullptr && piece_row_vec(mode, a) == 8 && a.tile_base != nullptr && a.kings > 1 &&
           heavy_mma_supported(a.width) && a.pieces <= 2048;
}

int launch_piece_rows(BulletOuCudaCppContext* ctx, int mode, PieceRowArgs a, const size_t* row_shift = nullptr,
                      const cudaEvent_t* events = nullptr, const HeavyMmaInputs* mma = nullptr,
                      const RowScatter* scatter = nullptr) {
    const int vec = piece_row_vec(mode, a);
    a.group_width = vec == 8 ? 256 : (vec == 4 ? 128 : 32);
    a.col_groups = (a.width + a.group_width - 1) / a.group_width;
    if (a.virtual_base >= 0 && a.kings > kKingsPerLaunch) {
        const size_t vf = align_floats(static_cast<size_t>(a.pieces) * a.width);
        void* vp = nullptr;
        if (scratch_slot(ctx, kScratchSfnnVirtual, (vf + static_cast<size_t>(a.pieces) * a.col_groups) * sizeof(float),
                         &vp, "cudaMalloc SFNN virtual-row sums") != 0)
            return -1;
        a.vacc = static_cast<float*>(vp);
        a.vany = reinterpret_cast<int*>(a.vacc + vf);
    }
    if (piece_rows_use_mma(mode, a, mma)) {
        // heavy keys on the tensor cores; the row kernel adds their sums
        HeavyMmaArgs m{};
        if (plan_heavy_mma(ctx, a, *mma, &m) != 0 || launch_heavy_key_mma(ctx, m) != 0) return -1;
        a.key_slot = m.plan.key_slot;
        a.key_partials = m.plan.partials;
        a.heavy_off = nullptr;
    } else {
        // Heavy-row segments: counts, their exclusive scan, the segment sums.
        // Segments <= entries / heavy_seg + the keys of heavy rows (each key adds
        // at most one partial segment) <= entries / heavy_seg + n_keys.
        a.heavy_row = kHeavyRow;
        a.heavy_seg = kHeavySeg;
        const int rows = a.n_keys;
        const size_t max_seg = a.max_entries / a.heavy_seg + static_cast<size_t>(a.n_keys) + 1;
        const size_t tiles = static_cast<size_t>(scan_tiles(rows)) + 1;
        const size_t ints = align_floats(2 * static_cast<size_t>(rows) + 1 + tiles + max_seg);
        void* hp = nullptr;
        if (scratch_slot(ctx, kScratchSfnnHeavy, (ints + max_seg * static_cast<size_t>(a.width)) * sizeof(float), &hp,
                         "cudaMalloc SFNN heavy-row segments") != 0)
            return -1;
        int* seg_count = static_cast<int*>(hp);
        int* seg_off = seg_count + rows;
        int* tile_sums = seg_off + rows + 1;
        int* seg_key = tile_sums + tiles;
        float* partials = reinterpret_cast<float*>(hp) + ints;
        const int base_rows = a.kings * a.pieces;
        const int threads = std::max(rows, base_rows);
        heavy_count_kernel<<<(threads + 255) / 256, 256, 0, ctx->stream>>>(
            a.offsets, a.tile_base, a.kings, a.pieces, base_rows, rows, a.heavy_row, a.heavy_seg, seg_count);
        if (check_launch("SFNN heavy-row count launch") != 0) return -1;
        if (exclusive_scan_counts(ctx, seg_count, rows, seg_off, tile_sums) != 0) return -1;
        heavy_fill_kernel<<<(rows + 255) / 256, 256, 0, ctx->stream>>>(seg_off, rows, static_cast<int>(
            std::min<size_t>(max_seg, INT_MAX)), seg_key);
        if (check_launch("SFNN heavy-row segment map launch") != 0) return -1;
        a.heavy_off = seg_off;
        a.heavy_partials = partials;
        a.heavy_ok = static_cast<int>(std::min<size_t>(max_seg, INT_MAX));
        const int blocks = 1 * ctx->sm_count;
        const int ms = a.heavy_ok;
        if (vec == 8)
            heavy_segment_kernel<8><<<blocks, kPieceRowWarps * 32, 0, ctx->stream>>>(a, rows, ms, seg_key, partials);
        else if (vec == 4)
            heavy_segment_kernel<4><<<blocks, kPieceRowWarps * 32, 0, ctx->stream>>>(a, rows, ms, seg_key, partials);
        else
            heavy_segment_kernel<1><<<blocks, kPieceRowWarps * 32, 0, ctx->stream>>>(a, rows, ms, seg_key, partials);
        if (check_launch("SFNN heavy-row segment launch") != 0) return -1;
    }
    switch (mode) {
        case kRowRanger: return launch_piece_rows_mode<kRowRanger>(ctx, a, vec, row_shift, events, nullptr);
        case kRowWrite: return launch_piece_rows_mode<kRowWrite>(ctx, a, vec, row_shift, events, scatter);
        default: return launch_piece_rows_mode<kRowAccumulate>(ctx, a, vec, row_shift, events, nullptr);
    }
}

// ------------------------------------------------------------------ host plan
struct SfnnPlan {
    const float* table;    // what the FT gather reads
    const float* ft_bias;  // FT bias the gather starts from (fake-quantised under FT QAT)
    KingSortOut king;
    int* king_rank;
    int* king_tiles;      // [kings + 1] first rank tile of each king block (tile-keyed FT row index)
    int kings;
    int max_king_tiles;
    Tiles tiles;
    float* w1_eff;
    float* head_partials;
    float* dw1_partials;
    float* l0b_partials;
    float* g1;
    // QAT scratch (l1 or dense)
    float* b1_eff;     // [S][O] fake-quantised folded L1 bias
    int* b1_int;       // [S][O] its i32 at 8128
    float* b1_master;  // [S][O] folded master L1 bias
    int* l1_raw;       // [B][O] integer L1 sums
    int* l2_raw;       // [B][L2] integer L2 sums
};

// QAT scratch: kept in one slot of fixed layout, so the reference forward and
// backward entries see the integer sums of the forward in the backward.
int qat_scratch(BulletOuCudaCppContext* ctx, const SfnnDims& d, SfnnPlan* plan) {
    const size_t so = align_floats(static_cast<size_t>(d.stacks) * d.l1_out);
    const size_t bo = align_floats(static_cast<size_t>(d.batch) * d.l1_out);
    const size_t bl = align_floats(static_cast<size_t>(d.batch) * d.l2_size);
    void* p = nullptr;
    if (scratch_slot(ctx, kScratchSfnnQat, (3 * so + bo + bl) * sizeof(float), &p, "cudaMalloc SFNN QAT") != 0)
        return -1;
    float* f = static_cast<float*>(p);
    plan->b1_eff = f;
    plan->b1_int = reinterpret_cast<int*>(f + so);
    plan->b1_master = f + 2 * so;
    plan->l1_raw = reinterpret_cast<int*>(f + 3 * so);
    plan->l2_raw = reinterpret_cast<int*>(f + 3 * so + bo);
    return 0;
}

// Fold, sorts, tile table and effective L1 weights; every scratch the step needs.
// The weight-dependent preparation: the fold (FT QAT: fake-quantised fold and
// bias), the effective L1 weights and the L1 QAT biases.
int sfnn_prepare_weights(BulletOuCudaCppContext* ctx, const SfnnDims& d, const SfnnWeights& w, float* fold_target,
                         SfnnPlan* plan) {
    const int threads = 256;
    int blocks = 0;
    plan->table = w.l0w;
    plan->ft_bias = w.l0b;
    if (d.qat.ft && w.l0w != nullptr) {
        // FT QAT: Q(row + alpha * virtual row) for the base rows (layer_qat.rs:832-880).
        const size_t n = static_cast<size_t>(d.n_features) * d.width;
        float* folded = fold_target;
        if (folded == nullptr) {
            void* p = nullptr;
            if (scratch_slot(ctx, kScratchSfnnFold, n * sizeof(float), &p, "cudaMalloc SFNN folded FT") != 0) return -1;
            folded = static_cast<float*>(p);
        }
        if (d.width % 4 == 0 && aligned16(w.l0w) && aligned16(folded)) {
            fold_rows_kernel<true><<<d.n_features, kFoldThreads, 0, ctx->stream>>>(
                reinterpret_cast<const float4*>(w.l0w), reinterpret_cast<float4*>(folded), d.width / 4, d.base,
                d.ft_alpha);
        } else {
            if (grid_1d(n, threads, &blocks, "SFNN FT QAT fold") != 0) return -1;
            fold_ft_qat_kernel<<<blocks, threads, 0, ctx->stream>>>(w.l0w, folded, n, d.width, d.base, d.ft_alpha);
        }
        void* bp = nullptr;
        if (scratch_slot(ctx, kScratchSfnnQatFt, static_cast<size_t>(d.width) * sizeof(float), &bp,
                         "cudaMalloc SFNN FT QAT bias") != 0)
            return -1;
        qat_vector_kernel<<<(d.width + threads - 1) / threads, threads, 0, ctx->stream>>>(
            w.l0b, static_cast<float*>(bp), static_cast<size_t>(d.width), 0);
        if (check_launch("SFNN FT QAT launch") != 0) return -1;
        plan->table = folded;
        plan->ft_bias = static_cast<float*>(bp);
    } else if (d.base > 0) {
        float* folded = fold_target;
        const size_t n = static_cast<size_t>(d.base) * d.width;
        if (folded == nullptr) {
            void* p = nullptr;
            if (scratch_slot(ctx, kScratchSfnnFold, n * sizeof(float), &p, "cudaMalloc SFNN folded FT") != 0) return -1;
            folded = static_cast<float*>(p);
        }
        if (d.width % 4 == 0 && aligned16(w.l0w) && aligned16(folded)) {
            fold_rows_kernel<false><<<d.base, kFoldThreads, 0, ctx->stream>>>(
                reinterpret_cast<const float4*>(w.l0w), reinterpret_cast<float4*>(folded), d.width / 4, d.base,
                d.ft_alpha);
        } else {
            if (grid_1d(n, threads, &blocks, "SFNN fold") != 0) return -1;
            fold_ft1_kernel<<<blocks, threads, 0, ctx->stream>>>(w.l0w, folded, n, d.width, d.base, d.ft_alpha);
        }
        if (check_launch("SFNN fold launch") != 0) return -1;
        plan->table = folded;
    }
    const size_t eff = static_cast<size_t>(d.stacks) * d.width * d.l1_out;
    void* ep = nullptr;
    if (scratch_slot(ctx, kScratchSfnnEff, eff * sizeof(float), &ep, "cudaMalloc SFNN L1 weights") != 0) return -1;
    plan->w1_eff = static_cast<float*>(ep);
    if (grid_1d(eff, threads, &blocks, "SFNN L1 weights") != 0) return -1;
    l1_eff_kernel<<<blocks, threads, 0, ctx->stream>>>(w.l1w, d.has_l1f ? w.l1fw : nullptr, d.shared_alpha, d.stacks,
                                                       d.l1_out, d.width, d.qat.l1, plan->w1_eff);
    if (check_launch("SFNN L1 weights launch") != 0) return -1;
    if (d.qat.l1 || d.qat.dense) {
        if (qat_scratch(ctx, d, plan) != 0) return -1;
        if (d.qat.l1 && w.l1b != nullptr) {
            const int n = d.stacks * d.l1_out;
            qat_l1_bias_kernel<<<(n + threads - 1) / threads, threads, 0, ctx->stream>>>(
                w.l1b, d.has_l1f ? w.l1fb : nullptr, d.shared_alpha, n, d.l1_out, 1, plan->b1_eff, plan->b1_int,
                plan->b1_master);
            if (check_launch("SFNN L1 QAT bias launch") != 0) return -1;
        }
    }
    return 0;
}

// The batch-only preparation: king sort of the half-positions, their rank
// tiles, bucket sort of the samples and its tile table, per-tile partial
// buffers.  Reads no weight.
int sfnn_prepare_batch(BulletOuCudaCppContext* ctx, const SfnnDims& d, const int* stm, const int* nstm,
                       const int* buckets, SfnnPlan* plan) {
    const int n_half = 2 * d.batch;
    const int max_tiles = d.batch / kSfnnTile + d.stacks + 2;
    const size_t king_ints = king_sort_scratch_ints<kSfnnKingKeys>(n_half);
    const size_t bucket_ints = king_sort_scratch_ints<kBucketKeys>(d.batch);
    const size_t tile_ints = 1 + 3 * static_cast<size_t>(max_tiles) + (kBucketKeys + 1);
    const size_t sort_ints = king_ints + n_half + bucket_ints + tile_ints + kSfnnKingKeys + 1;
    void* sp = nullptr;
    if (scratch_slot(ctx, kScratchSfnnSort, sort_ints * sizeof(int), &sp, "cudaMalloc SFNN sort") != 0) return -1;
    int* king_scratch = static_cast<int*>(sp);
    int* rank = king_scratch + king_ints;
    int* bucket_scratch = rank + n_half;
    int* tt = bucket_scratch + bucket_ints;
    const int piece = (d.n_features % kSfnnPieces == 0) ? kSfnnPieces : d.n_features;
    if (king_sort<kSfnnKingKeys>(ctx, stm, nstm, n_half, KingKey{piece, d.n_features, d.max_active}, king_scratch, rank,
                                 &plan->king) != 0)
        return -1;
    plan->king_rank = rank;
    {
        // rank tiles of the king blocks (see RowTiles)
        plan->kings = d.base > 0 ? d.base / kSfnnPieces : 1;
        plan->king_tiles = tt + tile_ints;
        plan->max_king_tiles = plan->kings + (n_half + kTileRanks - 1) / kTileRanks;
        king_tiles_kernel<<<1, 32, 0, ctx->stream>>>(plan->king.key_off, plan->kings, kTileRanks, plan->king_tiles);
        if (check_launch("SFNN king tile launch") != 0) return -1;
    }
    {
        const int nblocks = (d.batch + kKingSortThreads - 1) / kKingSortThreads;
        int* key_off = bucket_scratch;
        int* keys = key_off + kBucketKeys + 1;
        int* order = keys + d.batch;
        int* block_hist = order + d.batch;
        bucket_hist_kernel<<<nblocks, kKingSortThreads, 0, ctx->stream>>>(buckets, d.batch, d.stacks, keys, block_hist);
        king_bases_kernel<kBucketKeys><<<1, 128, 0, ctx->stream>>>(block_hist, nblocks, key_off);
        king_scatter_kernel<kBucketKeys><<<nblocks, kKingSortThreads, 0, ctx->stream>>>(keys, d.batch, block_hist, order,
                                                                                         nullptr);
        int* n_tiles = tt;
        int* tile_key = n_tiles + 1;
        int* tile_begin = tile_key + max_tiles;
        int* tile_end = tile_begin + max_tiles;
        int* key_first = tile_end + max_tiles;
        tile_table_kernel<<<1, 128, 0, ctx->stream>>>(key_off, d.stacks + 1, n_tiles, tile_key, tile_begin, tile_end,
                                                      key_first);
        if (check_launch("SFNN bucket sort launch") != 0) return -1;
        plan->tiles = Tiles{order, n_tiles, tile_key, tile_begin, tile_end, key_first, max_tiles};
    }
    // per-tile partial buffers
    const size_t hp = align_floats(static_cast<size_t>(max_tiles) * head_partial_len(d.l2_size, d.l2_in, d.l1_out));
    const size_t dp = align_floats(static_cast<size_t>(max_tiles) * d.l1_out * d.width);
    const size_t bp = align_floats(static_cast<size_t>(max_tiles) * 2 * d.width);
    const size_t gp = align_floats(static_cast<size_t>(d.batch) * d.l1_out);
    void* pp = nullptr;
    if (scratch_slot(ctx, kScratchSfnnPartials, (hp + dp + bp + gp) * sizeof(float), &pp,
                     "cudaMalloc SFNN partials") != 0)
        return -1;
    plan->head_partials = static_cast<float*>(pp);
    plan->dw1_partials = plan->head_partials + hp;
    plan->l0b_partials = plan->dw1_partials + dp;
    plan->g1 = plan->l0b_partials + bp;
    return 0;
}

int sfnn_prepare(BulletOuCudaCppContext* ctx, const SfnnDims& d, const SfnnWeights& w, const int* stm, const int* nstm,
                 const int* buckets, float* fold_target, SfnnPlan* plan) {
    if (sfnn_prepare_weights(ctx, d, w, fold_target, plan) != 0) return -1;
    return sfnn_prepare_batch(ctx, d, stm, nstm, buckets, plan);
}

int launch_ft_forward(BulletOuCudaCppContext* ctx, const SfnnDims& d, const SfnnPlan& plan, const int* stm,
                      const int* nstm, const float* l0b, const SfnnActivations& act) {
    if (d.qat.dense && d.qat.integer_ft) {
        // One gather for both outputs where the width has a warp kernel: the
        // f32 ClippedReLU activations (kept for the backward) and the engine's
        // integer FT into combined (cu:6654-6662).
        const bool fused_al = aligned16(plan.table) && aligned16(l0b) && aligned16(act.stm_l0) &&
                              aligned16(act.nstm_l0) && aligned16(act.combined);
        if (fused_al && ft_warp_width(d.width)) {
            FtArgs fa{};
            fa.order = plan.king.order;
            fa.stm = stm;
            fa.nstm = nstm;
            fa.table = plan.table;
            fa.bias = l0b;
            fa.l0[0] = act.stm_l0;
            fa.l0[1] = act.nstm_l0;
            fa.combined = act.combined;
            fa.n_half = 2 * d.batch;
            fa.max_active = d.max_active;
            fa.n_features = d.n_features;
            fa.width = d.width;
            constexpr int G = kFtIntWarps, P = 8 / kFtIntWarps;
            switch (d.width) {
                case 256: ft_forward_int_kernel<2, 1, 1><<<(fa.n_half + 7) / 8, 256, 0, ctx->stream>>>(fa); break;
                case 512: ft_forward_int_kernel<4, 1, 1><<<(fa.n_half + 7) / 8, 256, 0, ctx->stream>>>(fa); break;
                case 1024: ft_forward_int_kernel<8, 2, 1><<<(fa.n_half + 3) / 4, 256, 0, ctx->stream>>>(fa); break;
                case 1536:
                    ft_forward_int_kernel<12, G, kFtIntRounds><<<(fa.n_half + P - 1) / P, 32 * G * P, 0, ctx->stream>>>(
                        fa);
                    break;
                default: ft_forward_int_kernel<18, 3, 1><<<(fa.n_half + 1) / 2, 192, 0, ctx->stream>>>(fa); break;
            }
            return check_launch("SFNN dense QAT FT launch");
        }
        // Other widths: the f32 pass keeps the activations the backward uses,
        // then combined is overwritten by the engine's integer FT.
        SfnnDims df = d;
        df.qat.integer_ft = 0;
        df.qat.dense = 0;
        if (launch_ft_forward(ctx, df, plan, stm, nstm, l0b, act) != 0) return -1;
        FtArgs ea{};
        ea.stm = stm;
        ea.nstm = nstm;
        ea.table = plan.table;
        ea.bias = l0b;
        ea.combined = act.combined;
        ea.n_half = 2 * d.batch;
        ea.max_active = d.max_active;
        ea.n_features = d.n_features;
        ea.width = d.width;
        ea.order = plan.king.order;
        int gb = 0;
        if (grid_1d(static_cast<size_t>(ea.n_half) * (d.width / 2), 256, &gb, "SFNN exact QAT FT") != 0) return -1;
        qat_exact_ft_kernel<<<gb, 256, 0, ctx->stream>>>(ea);
        return check_launch("SFNN exact QAT FT launch");
    }
    FtArgs fa{};
    fa.lattice = d.qat.dense ? 1 : 0;
    fa.order = plan.king.order;
    fa.stm = stm;
    fa.nstm = nstm;
    fa.table = plan.table;
    fa.bias = l0b;
    fa.l0[0] = act.stm_l0;
    fa.l0[1] = act.nstm_l0;
    fa.combined = act.combined;
    fa.n_half = 2 * d.batch;
    fa.max_active = d.max_active;
    fa.n_features = d.n_features;
    fa.width = d.width;
    const bool al = aligned16(plan.table) && aligned16(l0b) && aligned16(act.stm_l0) && aligned16(act.nstm_l0) &&
                    aligned16(act.combined);
    const int blocks = (fa.n_half + 7) / 8;
    const bool lat = fa.lattice != 0;
#define BOU_FT_FWD(N)                                                              \
    (lat ? ft_forward_kernel<N, true><<<blocks, 256, 0, ctx->stream>>>(fa)        \
         : ft_forward_kernel<N, false><<<blocks, 256, 0, ctx->stream>>>(fa))
    if (al && d.width == 1536) BOU_FT_FWD(12);
    else if (al && d.width == 1024) BOU_FT_FWD(8);
    else if (al && d.width == 2304) BOU_FT_FWD(18);
    else if (al && d.width == 512) BOU_FT_FWD(4);
    else if (al && d.width == 256) BOU_FT_FWD(2);
#undef BOU_FT_FWD
    else {
        fa.order = nullptr;
        int gb = 0;
        if (grid_1d(static_cast<size_t>(fa.n_half) * (d.width / 2), 256, &gb, "SFNN FT forward") != 0) return -1;
        ft_forward_generic_kernel<<<gb, 256, 0, ctx->stream>>>(fa);
    }
    return check_launch("SFNN FT forward launch");
}

int launch_l1_forward(BulletOuCudaCppContext* ctx, const SfnnDims& d, const SfnnWeights& w, const SfnnPlan& plan,
                      const float* combined, float* l1) {
    if (d.qat.dense) {
        L1IntArgs ia{};
        ia.tiles = plan.tiles;
        ia.combined = combined;
        ia.w_eff = plan.w1_eff;
        ia.b_int = plan.b1_int;
        ia.l1 = l1;
        ia.raw = plan.l1_raw;
        ia.width = d.width;
        ia.out_dim = d.l1_out;
        ia.stacks = d.stacks;
        const size_t smem = static_cast<size_t>(d.width) * 4 * sizeof(int);
        if (d.l1_out == 16 && d.width % 4 == 0 && smem <= 200 * 1024 && aligned16(combined)) {
            cudaError_t st = cudaFuncSetAttribute(l1_forward16_int_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                  static_cast<int>(smem));
            if (st != cudaSuccess) return fail("cudaFuncSetAttribute SFNN QAT L1", st);
            l1_forward16_int_kernel<<<plan.tiles.max_tiles, 256, smem, ctx->stream>>>(ia);
        } else {
            l1_forward_int_generic_kernel<<<plan.tiles.max_tiles, 256, 0, ctx->stream>>>(ia);
        }
        return check_launch("SFNN QAT L1 forward launch");
    }
    L1Args la{};
    la.tiles = plan.tiles;
    la.combined = combined;
    la.w_eff = plan.w1_eff;
    // L1 QAT: the fake-quantised folded bias replaces bias + shared factor.
    la.l1b = d.qat.l1 ? plan.b1_eff : w.l1b;
    la.l1fb = (d.has_l1f && !d.qat.l1) ? w.l1fb : nullptr;
    la.alpha = d.shared_alpha;
    la.l1 = l1;
    la.width = d.width;
    la.out_dim = d.l1_out;
    la.stacks = d.stacks;
    const size_t smem = static_cast<size_t>(d.width) * 16 * sizeof(float);
    if (d.l1_out == 16 && d.width % 4 == 0 && smem <= 200 * 1024 && aligned16(combined)) {
        cudaError_t st = cudaFuncSetAttribute(l1_forward16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              static_cast<int>(smem));
        if (st != cudaSuccess) return fail("cudaFuncSetAttribute SFNN L1", st);
        l1_forward16_kernel<<<plan.tiles.max_tiles, 256, smem, ctx->stream>>>(la);
    } else {
        l1_forward_generic_kernel<<<plan.tiles.max_tiles, 256, 0, ctx->stream>>>(la);
    }
    return check_launch("SFNN L1 forward launch");
}

size_t head_smem_bytes(const SfnnDims& d) {
    const size_t l2 = d.l2_size, i2 = d.l2_in, o = d.l1_out;
    const size_t ints = d.qat.dense ? l2 * i2 + 2 * l2 + 1 : 0;
    return (l2 * i2 + 2 * l2 + 1 + kSfnnTile * (2 * l2 + i2 + 1 + o + 1)) * sizeof(float) + ints * sizeof(int);
}

int launch_head(BulletOuCudaCppContext* ctx, const SfnnDims& d, const HeadArgs& h) {
    const size_t smem = head_smem_bytes(d);
    const bool prod = d.l1_hidden == 15 && d.l2_size == 32;
    auto kernel = d.qat.dense ? (prod ? head_kernel<15, 32, true> : head_kernel<0, 0, true>)
                              : (prod ? head_kernel<15, 32, false> : head_kernel<0, 0, false>);
    cudaError_t st = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (st != cudaSuccess) return fail("cudaFuncSetAttribute SFNN head", st);
    kernel<<<h.tiles.max_tiles, kSfnnTile, smem, ctx->stream>>>(h);
    return check_launch("SFNN head launch");
}

HeadArgs head_args(const SfnnDims& d, const SfnnWeights& w, const SfnnPlan& plan, const SfnnActivations& act) {
    HeadArgs h{};
    h.tiles = plan.tiles;
    h.l1 = act.l1;
    h.l2w = w.l2w;
    h.l2b = w.l2b;
    h.l2fw = d.has_l2f ? w.l2fw : nullptr;
    h.l2fb = d.has_l2f ? w.l2fb : nullptr;
    h.l3w = w.l3w;
    h.l3b = w.l3b;
    h.l3fw = d.has_l3f ? w.l3fw : nullptr;
    h.l3fb = d.has_l3f ? w.l3fb : nullptr;
    h.alpha = d.shared_alpha;
    h.l2_input = act.l2_input;
    h.l2 = act.l2;
    h.output = act.output;
    h.g1 = plan.g1;
    h.partials = plan.head_partials;
    h.l1_hidden = d.l1_hidden;
    h.l1_out = d.l1_out;
    h.l1_skip = d.l1_skip;
    h.l2_size = d.l2_size;
    h.stacks = d.stacks;
    h.qat_l2 = d.qat.l2;
    h.qat_l3 = d.qat.l3;
    if (d.qat.dense) {
        h.l1_raw = plan.l1_raw;
        h.l2_raw = plan.l2_raw;
        h.b1_master = plan.b1_master;
        h.b1_int = plan.b1_int;
        h.l2b_master = d.qat.l2b_master;
        h.l3b_master = d.qat.l3b_master;
    }
    return h;
}

int launch_l1_backward(BulletOuCudaCppContext* ctx, const SfnnDims& d, const SfnnPlan& plan, L1BackArgs& b) {
    b.tiles = plan.tiles;
    b.g1 = plan.g1;
    b.w_eff = plan.w1_eff;
    b.dw1_partials = plan.dw1_partials;
    b.l0b_partials = plan.l0b_partials;
    b.width = d.width;
    b.out_dim = d.l1_out;
    b.stacks = d.stacks;
    const dim3 grid(plan.tiles.max_tiles, (d.width + 255) / 256);
    if (d.l1_out == 16) l1_backward_kernel<16><<<grid, 256, 0, ctx->stream>>>(b);
    else l1_backward_kernel<0><<<grid, 256, 0, ctx->stream>>>(b);
    return check_launch("SFNN L1 backward launch");
}

int launch_finalize(BulletOuCudaCppContext* ctx, const SfnnDims& d, const SfnnPlan& plan, FinalArgs& f) {
    f.tiles = plan.tiles;
    f.head_partials = plan.head_partials;
    f.dw1_partials = plan.dw1_partials;
    f.l0b_partials = plan.l0b_partials;
    f.alpha = d.shared_alpha;
    f.width = d.width;
    f.out_dim = d.l1_out;
    f.l2_size = d.l2_size;
    f.l2_in = d.l2_in;
    f.stacks = d.stacks;
    f.batch = d.batch;
    const int P = head_partial_len(d.l2_size, d.l2_in, d.l1_out);
    const size_t n = static_cast<size_t>(d.width) + static_cast<size_t>(d.stacks) * d.l1_out * d.width +
                     static_cast<size_t>(d.width) * d.l1_out + static_cast<size_t>(d.stacks) * P + P;
    int blocks = 0;
    if (grid_1d(n, 256, &blocks, "SFNN finalize") != 0) return -1;
    finalize_kernel<<<blocks, 256, 0, ctx->stream>>>(f);
    return check_launch("SFNN finalize launch");
}

PieceRowArgs piece_row_args(const SfnnDims& d, const InverseIndex& index) {
    PieceRowArgs r{};
    r.offsets = index.offsets;
    r.entries = index.entries;
    r.max_entries = 2 * static_cast<size_t>(d.batch) * static_cast<size_t>(d.max_active);
    r.n_keys = index.n_rows;
    if (d.base > 0) {
        r.pieces = kSfnnPieces;
        r.kings = d.base / kSfnnPieces;
        r.virtual_base = d.base;
    } else {
        r.pieces = d.n_features;
        r.kings = 1;
        r.virtual_base = -1;
    }
    r.alpha = d.ft_alpha;
    r.width = d.width;
    return r;
}

// ------------------------------------------------------------------ validation
}  // namespace

int sfnn_dims(size_t input_size, size_t ft_size, size_t l1_hidden, int l1_skip, size_t l2_size, size_t num_stacks,
              size_t batch, size_t max_active, float ft_alpha, float shared_alpha, SfnnDims* d) {
    if (input_size == 0 || ft_size == 0 || l1_hidden == 0 || l2_size == 0 || num_stacks == 0 || batch == 0 ||
        max_active == 0)
        return fail_message("SFNN shape, batch and max_active must be greater than zero");
    if (ft_size % 2 != 0) return fail_messagef("SFNN ft_size must be even, got %zu", ft_size);
    const size_t l1_out = l1_hidden + (l1_skip ? 1 : 0);
    if (l1_out > static_cast<size_t>(kSfnnMaxL1Out))
        return fail_messagef("SFNN l1_hidden + skip must be at most %d on this backend", kSfnnMaxL1Out);
    if (l2_size > static_cast<size_t>(kSfnnMaxL2))
        return fail_messagef("SFNN l2_size must be at most %d on this backend", kSfnnMaxL2);
    if (num_stacks > static_cast<size_t>(kSfnnMaxStacks))
        return fail_messagef("SFNN num_stacks must be at most %d on this backend", kSfnnMaxStacks);
    if (batch > (1u << 26) || max_active > 4096 || input_size > static_cast<size_t>(INT_MAX) / 2 || ft_size > 8192 ||
        input_size * ft_size > (static_cast<size_t>(1) << 40))
        return fail_message("SFNN batch, max_active or table too large for this backend");
    if (!(ft_alpha >= 0.0f && ft_alpha <= 100.0f) || !(shared_alpha >= 0.0f && shared_alpha <= 10.0f))
        return fail_message("SFNN factorizer alpha out of range");
    d->input_size = static_cast<int>(input_size);
    d->base = sfnn_factorized_base(input_size);
    d->n_features = d->base > 0 ? d->base : static_cast<int>(input_size);
    d->width = static_cast<int>(ft_size);
    d->l1_hidden = static_cast<int>(l1_hidden);
    d->l1_out = static_cast<int>(l1_out);
    d->l1_skip = l1_skip ? 1 : 0;
    d->l2_in = static_cast<int>(2 * l1_hidden);
    d->l2_size = static_cast<int>(l2_size);
    d->stacks = static_cast<int>(num_stacks);
    d->batch = static_cast<int>(batch);
    d->max_active = static_cast<int>(max_active);
    d->ft_alpha = ft_alpha;
    d->shared_alpha = shared_alpha;
    return 0;
}

namespace {

int validate_sfnn_weights(BulletOuCudaCppContext* ctx, const SfnnDims& d, const BulletOuCudaCppF32Buffer* const* p,
                          const char* what) {
    const SfnnGroupLayout g = sfnn_group_layout(d);
    static const char* names[14] = {"l0w", "l0b", "l1w", "l1b", "l1fw", "l1fb", "l2w",
                                    "l2b", "l2fw", "l2fb", "l3w", "l3b", "l3fw", "l3fb"};
    char name[64];
    std::snprintf(name, sizeof(name), "%s l0w", what);
    if (validate_f32(ctx, p[0], static_cast<size_t>(d.input_size) * d.width, name) != 0) return -1;
    for (int k = 0; k < kSfGroups; ++k) {
        std::snprintf(name, sizeof(name), "%s %s", what, names[k + 1]);
        if (g.len[k] == 0) {
            if (p[k + 1] != nullptr) return fail_messagef("%s must be null when its factorizer is inactive", name);
            continue;
        }
        if (validate_f32(ctx, p[k + 1], g.len[k], name) != 0) return -1;
    }
    return 0;
}

SfnnWeights weights_from(const BulletOuCudaCppF32Buffer* const* p) {
    auto ptr = [&](int i) -> const float* { return p[i] != nullptr ? p[i]->ptr : nullptr; };
    return SfnnWeights{ptr(0), ptr(1), ptr(2),  ptr(3),  ptr(4),  ptr(5),  ptr(6),
                       ptr(7), ptr(8), ptr(9), ptr(10), ptr(11), ptr(12), ptr(13)};
}

// Scratch activations of the fused step: stm_l0 | nstm_l0 | combined | l1 |
// l2_input | l2 | pregrad (king order).
struct StepBuffers {
    SfnnActivations act;
    float* pregrad;
    __nv_bfloat16* pregrad_hi;  // null unless the heavy keys go to the tensor cores
    __nv_bfloat16* pregrad_lo;
};

int step_buffers(BulletOuCudaCppContext* ctx, const SfnnDims& d, float* output, StepBuffers* sb) {
    const size_t BW = static_cast<size_t>(d.batch) * d.width;
    const bool planes = heavy_mma_supported(d.width) && d.base > 0;
    const size_t sizes[8] = {align_floats(BW),
                             align_floats(BW),
                             align_floats(BW),
                             align_floats(static_cast<size_t>(d.batch) * d.l1_out),
                             align_floats(static_cast<size_t>(d.batch) * d.l2_in),
                             align_floats(static_cast<size_t>(d.batch) * d.l2_size),
                             align_floats(2 * BW),
                             planes ? align_floats(2 * BW) : 0};  // bf16 hi and lo planes of the pregrad rows
    size_t total = 0;
    for (size_t s : sizes) total += s;
    void* p = nullptr;
    if (scratch_slot(ctx, kScratchSfnnStep, total * sizeof(float), &p, "cudaMalloc SFNN step buffers") != 0) return -1;
    float* f = static_cast<float*>(p);
    float* ptrs[8];
    for (int i = 0; i < 8; ++i) {
        ptrs[i] = f;
        f += sizes[i];
    }
    sb->act = SfnnActivations{ptrs[0], ptrs[1], ptrs[2], ptrs[3], ptrs[4], ptrs[5], output};
    sb->pregrad = ptrs[6];
    sb->pregrad_hi = planes ? reinterpret_cast<__nv_bfloat16*>(ptrs[7]) : nullptr;
    sb->pregrad_lo = planes ? sb->pregrad_hi + 2 * BW : nullptr;
    return 0;
}

// Bounds of the L1 shared factor refer to its contribution alpha * w
// (factor_contribution_clip, lib.rs:8772-8788): divided by alpha, unbounded
// when alpha is 0; infinite bounds stay infinite.
RangerArgs shared_factor_clip(RangerArgs a, float alpha) {
    auto scale = [&](float bound, float lim) -> float {
        if (alpha == 0.0f) return lim;
        if (bound == -FLT_MAX || bound == FLT_MAX) return bound;
        const double x = static_cast<double>(bound) / static_cast<double>(alpha);
        return static_cast<float>(std::min<double>(FLT_MAX, std::max<double>(-FLT_MAX, x)));
    };
    a.min_weight = scale(a.min_weight, -FLT_MAX);
    a.max_weight = scale(a.max_weight, FLT_MAX);
    if (a.lookahead_min != -FLT_MAX || a.lookahead_max != FLT_MAX) {
        a.lookahead_min = a.min_weight;
        a.lookahead_max = a.max_weight;
    }
    return a;
}

// The fused step: forward, loss, backward and Ranger (ranger != null), or the
// local gradients (ranger == null: FT gradient rows written to ft_grad, small
// groups packed into dense_grad in the sfnn_group_layout order).
int sfnn_step(BulletOuCudaCppContext* ctx, const SfnnDims& d, const SfnnWeights& w, const int* stm, const int* nstm,
              const int* buckets, const float* targets, const float* entry_weights, const LossArgs& la, int finalize,
              const BulletOuB200RangerStep* ranger, float* const* wm, float* const* mm, float* const* vm,
              float* const* sm, float* output, float* per_sample, float* mog, float* weighted_sum, float* mean,
              float* ft_grad, float* dense_grad, const size_t* row_shift = nullptr,
              const cudaEvent_t* row_events = nullptr, const RowScatter* scatter = nullptr) {
    // phases: batch sorts and tiles, inverse index, [weights wait] fold and L1
    // weights, FT forward, L1 + head, L1 backward, small groups, FT rows
    ctx->prof_marks_per_step = 9;
    prof_mark(ctx);
    SfnnPlan plan{};
    if (sfnn_prepare_batch(ctx, d, stm, nstm, buckets, &plan) != 0) return -1;
    prof_mark(ctx);
    InverseIndex index;
    const RowTiles row_tiles{plan.king_tiles, plan.king.key_off, d.base > 0 ? kSfnnPieces : d.n_features, plan.kings,
                             kTileRanks, plan.max_king_tiles};
    if (build_inverse_index_tiled(ctx, stm, nstm, d.batch, d.max_active, row_tiles, &index, plan.king_rank) != 0)
        return -1;
    StepBuffers sb{};
    if (step_buffers(ctx, d, output, &sb) != 0) return -1;
    // the FT rows' arguments (their Ranger step is filled in below)
    PieceRowArgs r = piece_row_args(d, index);
    r.tile_base = plan.king_tiles;
    r.src[0] = sb.pregrad;
    r.src[1] = sb.pregrad + d.width;
    r.src_stride = 2 * static_cast<size_t>(d.width);
    const int row_mode = ranger != nullptr ? kRowRanger : kRowWrite;
    if (ranger != nullptr) {
        r.weights = wm[0];
        r.momentum = mm[0];
        r.velocity = vm[0];
        r.slow = sm[0];
    } else {
        r.gradients = ft_grad;
    }
    const HeavyMmaInputs mma{plan.king.key_off, plan.king.order, stm, nstm, d.max_active, plan.max_king_tiles,
                             2 * d.batch, sb.pregrad_hi, sb.pregrad_lo};
    const HeavyMmaInputs* mp = sb.pregrad_hi != nullptr ? &mma : nullptr;
    // the tensor cores sum the heavy keys without their entry lists: only the
    // light keys are sorted
    if (sort_inverse_index(ctx, index, piece_rows_use_mma(row_mode, r, mp) ? kHeavyMmaThreshold : 0x7fffffff) != 0)
        return -1;
    prof_mark(ctx);
    // everything above reads only the batch; from here on the step reads the
    // weights, so it waits for the event a caller set to mark their update
    if (ctx->weights_ready != nullptr) {
        const cudaError_t st = cudaStreamWaitEvent(ctx->stream, ctx->weights_ready, 0);
        ctx->weights_ready = nullptr;
        if (st != cudaSuccess) return fail("cudaStreamWaitEvent weights-ready event", st);
    }
    if (ctx->weights_flags != nullptr) {
        const int* flags = ctx->weights_flags;
        ctx->weights_flags = nullptr;
        if (launch_exchange_wait(ctx, flags, ctx->weights_flag_count, ctx->weights_flag_epoch,
                                 ctx->weights_flag_error) != 0)
            return -1;
    }
    if (sfnn_prepare_weights(ctx, d, w, nullptr, &plan) != 0) return -1;
    prof_mark(ctx);
    if (launch_ft_forward(ctx, d, plan, stm, nstm, plan.ft_bias, sb.act) != 0) return -1;
    prof_mark(ctx);
    if (launch_l1_forward(ctx, d, w, plan, sb.act.combined, sb.act.l1) != 0) return -1;
    HeadArgs h = head_args(d, w, plan, sb.act);
    h.mode = kHeadTrain;
    h.targets = targets;
    h.entry_weights = entry_weights;
    h.loss = la;
    h.per_sample = per_sample;
    h.mog = mog;
    if (launch_head(ctx, d, h) != 0) return -1;
    prof_mark(ctx);
    L1BackArgs lb{};
    lb.l0[0] = sb.act.stm_l0;
    lb.l0[1] = sb.act.nstm_l0;
    lb.pregrad_sorted = sb.pregrad;
    lb.pregrad_hi = sb.pregrad_hi;
    lb.pregrad_lo = sb.pregrad_lo;
    lb.rank = plan.king_rank;
    lb.combined = d.qat.dense ? sb.act.combined : nullptr;
    if (launch_l1_backward(ctx, d, plan, lb) != 0) return -1;
    prof_mark(ctx);
    // small-parameter gradients (packed), loss sum, then Ranger per group
    const SfnnGroupLayout g = sfnn_group_layout(d);
    float* packed = dense_grad;
    if (packed == nullptr) {
        void* gp = nullptr;
        if (scratch_slot(ctx, kScratchSfnnGrads, g.begin[kSfGroups] * sizeof(float), &gp, "cudaMalloc SFNN grads") != 0)
            return -1;
        packed = static_cast<float*>(gp);
    }
    FinalArgs f{};
    for (int k = 0; k < kSfGroups; ++k) f.dst[k] = g.len[k] ? packed + g.begin[k] : nullptr;
    f.accumulate = 0;
    if (finalize) {
        f.weighted_sum = weighted_sum;
        f.mean = mean;
    }
    if (launch_finalize(ctx, d, plan, f) != 0) return -1;
    RangerArgs ra{};
    if (ranger != nullptr) {
        ra = ranger_args_from(*ranger);
        for (int k = 0; k < kSfGroups; ++k) {
            if (!g.len[k]) continue;
            const RangerArgs ga = (k == kSfL1fw || k == kSfL1fb) ? shared_factor_clip(ra, d.shared_alpha) : ra;
            if (launch_ranger(ctx, g.len[k], ga, packed + g.begin[k], wm[k + 1], mm[k + 1], vm[k + 1], sm[k + 1]) != 0)
                return -1;
        }
    }
    // peer exchange: the small groups' gradient into every rank's slot
    if (scatter != nullptr && scatter->small_len > 0) {
        if (launch_exchange_scatter(ctx, packed, scatter->small_len, scatter->small, scatter->world, scatter->rank) !=
                0 ||
            launch_exchange_signal(ctx, scatter->flags, scatter->world, scatter->small_flag_base + scatter->rank,
                                   scatter->epoch) != 0)
            return -1;
    }
    prof_mark(ctx);
    if (ranger != nullptr) {
        r.ranger = ra;
        r.skip_quiet = ranger_zero_step_is_identity(ra) ? 1 : 0;
        if (launch_piece_rows(ctx, kRowRanger, r, nullptr, nullptr, mp) != 0) return -1;
    } else {
        if (launch_piece_rows(ctx, kRowWrite, r, row_shift, row_events, mp, scatter) != 0) return -1;
    }
    prof_mark(ctx);
    return 0;
}

// The fused step's QAT switches (null: none) into d->qat; the f32 masters in
// `w` are what every QAT mode rounds.  Layer QAT of L2 / L3 takes no shared
// factor (layer_qat.rs:937-943).
int apply_qat(const BulletOuB200SfnnQat* q, const SfnnWeights& w, SfnnDims* d) {
    d->qat = SfnnQat{};
    if (q == nullptr) return 0;
    if ((q->l2 && d->has_l2f) || (q->l3 && d->has_l3f))
        return fail_message("SFNN layer QAT does not support L2/L3 shared factors; fold them first");
    d->qat.l1 = q->l1 != 0;
    d->qat.ft = q->ft != 0;
    d->qat.l2 = q->l2 != 0;
    d->qat.l3 = q->l3 != 0;
    d->qat.dense = d->qat.l1 && d->qat.l2 && d->qat.l3;
    d->qat.integer_ft = d->qat.dense && d->qat.ft;
    d->qat.l2b_master = w.l2b;
    d->qat.l3b_master = w.l3b;
    return 0;
}

// Rejects the reference options this backend does not implement: grouped and
// common+shard L1, bucket-axis factorizers, residual count gates.
int reject_unsupported(size_t l1_group_count, size_t l1_common_size, size_t l1_shard_size, int has_l1ax, int has_l2ax,
                       int has_l3ax, int use_king_axis, int use_hand_axis, int use_progress_axis,
                       int use_king_hand_pair, int use_king_progress_pair, int use_hand_progress_pair,
                       const BulletOuCudaCppF32Buffer* residual_count_gates,
                       const BulletOuCudaCppF32Buffer* factorizer_axis_confidences) {
    if (l1_group_count > 1 || l1_common_size != 0 || l1_shard_size != 0)
        return fail_message("unsupported on this backend: grouped / common+shard SFNN L1");
    if (has_l1ax || has_l2ax || has_l3ax || use_king_axis || use_hand_axis || use_progress_axis || use_king_hand_pair ||
        use_king_progress_pair || use_hand_progress_pair)
        return fail_message("unsupported on this backend: SFNN bucket-axis factorizers");
    if (residual_count_gates != nullptr || factorizer_axis_confidences != nullptr)
        return fail_message("unsupported on this backend: SFNN residual count gates / axis confidences");
    return 0;
}

}  // namespace
}  // namespace bou

using namespace bou;

// ------------------------------------------------------------------ C ABI
extern "C" {

int bulletou_cuda_cpp_sfnn_forward_device(
    BulletOuCudaCppContext* ctx, size_t input_size, size_t ft_size, size_t l1_hidden, int l1_skip, size_t l2_size,
    size_t num_stacks, size_t l1_group_count, size_t l1_common_size, size_t l1_shard_size,
    size_t factorizer_king_axis_dim, size_t factorizer_hand_axis_dim, size_t batch, size_t max_active,
    const BulletOuCudaCppI32Buffer* stm_indices, const BulletOuCudaCppI32Buffer* nstm_indices,
    const BulletOuCudaCppI32Buffer* buckets, const BulletOuCudaCppF32Buffer* l0w, BulletOuCudaCppF32Buffer* folded_l0w,
    const BulletOuCudaCppF32Buffer* l0b, const BulletOuCudaCppF32Buffer* l1w, const BulletOuCudaCppF32Buffer* l1b,
    const BulletOuCudaCppF32Buffer* l1fw, const BulletOuCudaCppF32Buffer* l1fb, int has_l1f,
    const BulletOuCudaCppF32Buffer* l1axw, const BulletOuCudaCppF32Buffer* l1axb, int has_l1ax,
    const BulletOuCudaCppF32Buffer* l2w, const BulletOuCudaCppF32Buffer* l2b, const BulletOuCudaCppF32Buffer* l2fw,
    const BulletOuCudaCppF32Buffer* l2fb, int has_l2f, const BulletOuCudaCppF32Buffer* l2axw,
    const BulletOuCudaCppF32Buffer* l2axb, int has_l2ax, const BulletOuCudaCppF32Buffer* l3w,
    const BulletOuCudaCppF32Buffer* l3b, const BulletOuCudaCppF32Buffer* l3fw, const BulletOuCudaCppF32Buffer* l3fb,
    int has_l3f, const BulletOuCudaCppF32Buffer* l3axw, const BulletOuCudaCppF32Buffer* l3axb, int has_l3ax,
    int use_king_axis, int use_hand_axis, int use_progress_axis, int use_king_hand_pair, int use_king_progress_pair,
    int use_hand_progress_pair, float ft_factorizer_alpha, float factorizer_shared_alpha,
    float factorizer_king_axis_alpha, float factorizer_hand_axis_alpha, float factorizer_progress_axis_alpha,
    float factorizer_pair_alpha, const BulletOuCudaCppF32Buffer* residual_count_gates,
    const BulletOuCudaCppF32Buffer* factorizer_axis_confidences, BulletOuCudaCppF32Buffer* stm_l0,
    BulletOuCudaCppF32Buffer* nstm_l0, BulletOuCudaCppF32Buffer* combined, BulletOuCudaCppF32Buffer* l1,
    BulletOuCudaCppF32Buffer* l2_input, BulletOuCudaCppF32Buffer* l2, BulletOuCudaCppF32Buffer* output,
    BulletOuCudaCppF32Buffer* qat_l1w, BulletOuCudaCppF32Buffer* qat_l1b, int refresh_qat_l1) {
    (void)factorizer_king_axis_dim;
    (void)factorizer_hand_axis_dim;
    (void)factorizer_king_axis_alpha;
    (void)factorizer_hand_axis_alpha;
    (void)factorizer_progress_axis_alpha;
    (void)factorizer_pair_alpha;
    (void)l1axw;
    (void)l1axb;
    (void)l2axw;
    (void)l2axb;
    (void)l3axw;
    (void)l3axb;
    if (reject_unsupported(l1_group_count, l1_common_size, l1_shard_size, has_l1ax, has_l2ax, has_l3ax, use_king_axis,
                           use_hand_axis, use_progress_axis, use_king_hand_pair, use_king_progress_pair,
                           use_hand_progress_pair, residual_count_gates, factorizer_axis_confidences) != 0)
        return -1;
    if ((qat_l1w == nullptr) != (qat_l1b == nullptr))
        return fail_message("L1 QAT requires both weight and bias scratch buffers");
    SfnnDims d{};
    if (sfnn_dims(input_size, ft_size, l1_hidden, l1_skip, l2_size, num_stacks, batch, max_active, ft_factorizer_alpha,
                  factorizer_shared_alpha, &d) != 0)
        return -1;
    d.has_l1f = has_l1f ? 1 : 0;
    d.has_l2f = has_l2f ? 1 : 0;
    d.has_l3f = has_l3f ? 1 : 0;
    if ((!has_l1f && (l1fw || l1fb)) || (!has_l2f && (l2fw || l2fb)) || (!has_l3f && (l3fw || l3fb)))
        return fail_message("sfnn shared factor buffers must be null when their has_* flag is false");
    const BulletOuCudaCppF32Buffer* params[14] = {l0w, l0b, l1w, l1b, l1fw, l1fb, l2w,
                                                  l2b, l2fw, l2fb, l3w, l3b, l3fw, l3fb};
    const size_t BW = batch * ft_size;
    if (validate_i32(ctx, stm_indices, batch * max_active, "stm_indices") != 0 ||
        validate_i32(ctx, nstm_indices, batch * max_active, "nstm_indices") != 0 ||
        validate_i32(ctx, buckets, batch, "buckets") != 0 || validate_sfnn_weights(ctx, d, params, "sfnn") != 0 ||
        validate_f32(ctx, stm_l0, BW, "sfnn stm_l0") != 0 || validate_f32(ctx, nstm_l0, BW, "sfnn nstm_l0") != 0 ||
        validate_f32(ctx, combined, BW, "sfnn combined") != 0 ||
        validate_f32(ctx, l1, batch * d.l1_out, "sfnn l1") != 0 ||
        validate_f32(ctx, l2_input, batch * d.l2_in, "sfnn l2_input") != 0 ||
        validate_f32(ctx, l2, batch * l2_size, "sfnn l2") != 0 || validate_f32(ctx, output, batch, "sfnn output") != 0)
        return -1;
    if (folded_l0w != nullptr && validate_f32(ctx, folded_l0w, input_size * ft_size, "sfnn folded_l0w scratch") != 0)
        return -1;
    const size_t l1w_len = static_cast<size_t>(d.stacks) * d.l1_out * d.width;
    if (qat_l1w != nullptr && (validate_f32(ctx, qat_l1w, l1w_len, "QAT L1 weights") != 0 ||
                               validate_f32(ctx, qat_l1b, static_cast<size_t>(d.stacks) * d.l1_out, "QAT L1 bias") != 0))
        return -1;
    // Dense QAT between bulletou_dense_qat_begin / _end (cu:6666-6668).
    d.qat.dense = ctx->dense_qat ? 1 : 0;
    d.qat.integer_ft = ctx->dense_qat && ctx->dense_qat_integer_ft ? 1 : 0;
    d.qat.l2b_master = ctx->dense_qat_l2_bias;
    d.qat.l3b_master = ctx->dense_qat_l3_bias;
    if (d.qat.dense && ((has_l1f && qat_l1w == nullptr) || has_l2f || has_l3f))
        return fail_message("dense QAT requires folded L1 and unfactorized L2/L3 without BN");
    if (d.qat.dense && qat_l1w == nullptr)
        return fail_message("dense QAT on this backend requires the L1 QAT scratch (qat_l1w / qat_l1b)");
    if (set_device(ctx) != 0) return -1;
    SfnnWeights w = weights_from(params);
    SfnnDims dk = d;
    // L1 QAT: fold first, then fake-quantise; the f32 masters stay untouched.
    // refresh_qat_l1: 1 rebuild quantised, 0 reuse quantised, -2 rebuild
    // f32 fold, -1 reuse f32 fold (cu:11514-11590).
    const bool quantize_l1 = refresh_qat_l1 >= 0;
    const bool refresh_l1 = refresh_qat_l1 == 1 || refresh_qat_l1 == -2;
    if (qat_l1w != nullptr) {
        if (refresh_l1) {
            int blocks = 0;
            if (grid_1d(l1w_len, 256, &blocks, "QAT L1 weights") != 0) return -1;
            qat_l1_fold_kernel<<<blocks, 256, 0, ctx->stream>>>(l1w->ptr, has_l1f ? l1fw->ptr : nullptr,
                                                                factorizer_shared_alpha, l1w_len, d.l1_out, d.width,
                                                                quantize_l1 ? 1 : 0, qat_l1w->ptr);
            if (check_launch("QAT L1 weights launch") != 0) return -1;
        }
        w.l1w = qat_l1w->ptr;
        w.l1b = qat_l1b->ptr;
        w.l1fw = nullptr;
        w.l1fb = nullptr;
        dk.has_l1f = 0;
    }
    SfnnPlan plan{};
    if (sfnn_prepare(ctx, dk, w, stm_indices->ptr, nstm_indices->ptr, buckets->ptr,
                     folded_l0w != nullptr ? folded_l0w->ptr : nullptr, &plan) != 0)
        return -1;
    if (qat_l1w != nullptr && (refresh_l1 || d.qat.dense)) {
        const int n = d.stacks * d.l1_out;
        qat_l1_bias_kernel<<<(n + 255) / 256, 256, 0, ctx->stream>>>(
            l1b->ptr, has_l1f ? l1fb->ptr : nullptr, factorizer_shared_alpha, n, d.l1_out, quantize_l1 ? 1 : 0,
            qat_l1b->ptr, d.qat.dense ? plan.b1_int : nullptr, d.qat.dense ? plan.b1_master : nullptr);
        if (check_launch("QAT L1 bias launch") != 0) return -1;
    }
    const SfnnActivations act{stm_l0->ptr, nstm_l0->ptr, combined->ptr, l1->ptr, l2_input->ptr, l2->ptr, output->ptr};
    if (launch_ft_forward(ctx, dk, plan, stm_indices->ptr, nstm_indices->ptr, plan.ft_bias, act) != 0) return -1;
    if (launch_l1_forward(ctx, dk, w, plan, act.combined, act.l1) != 0) return -1;
    HeadArgs h = head_args(dk, w, plan, act);
    h.mode = kHeadForward;
    if (launch_head(ctx, dk, h) != 0) return -1;
    return ok();
}

}  // extern "C"

namespace bou {
namespace {

// Stage events of the reference's backward profile (SfnnBackwardProfileEvents,
// cu:5679-5750): zeroing, L3, L2, L2 input, L1, pairwise + FT, total.  The head
// kernel does the L3 / L2 / L2-input backward at once: its time is reported as
// L3, with L2 and L2 input 0.
struct BackwardProfile {
    float* out = nullptr;
    cudaEvent_t ev[5] = {};
    int n = 0;
    ~BackwardProfile() {
        for (cudaEvent_t e : ev)
            if (e != nullptr) cudaEventDestroy(e);
    }
    int init(BulletOuCudaCppContext* ctx, float* ms, size_t len) {
        if (ms == nullptr) return 0;
        if (len < 7) return fail_message("SFNN backward profile output must have at least 7 floats");
        out = ms;
        for (int i = 0; i < 7; ++i) out[i] = 0.0f;
        for (cudaEvent_t& e : ev) {
            const cudaError_t st = cudaEventCreate(&e);
            if (st != cudaSuccess) return fail("cudaEventCreate SFNN backward profile", st);
        }
        return mark(ctx);
    }
    int mark(BulletOuCudaCppContext* ctx) {
        if (out == nullptr) return 0;
        const cudaError_t st = cudaEventRecord(ev[n++], ctx->stream);
        return st == cudaSuccess ? 0 : fail("cudaEventRecord SFNN backward profile", st);
    }
    int finish() {
        if (out == nullptr) return 0;
        cudaError_t st = cudaEventSynchronize(ev[4]);
        if (st != cudaSuccess) return fail("cudaEventSynchronize SFNN backward profile", st);
        const int from[5] = {0, 1, 2, 3, 0}, to[5] = {1, 2, 3, 4, 4}, slot[5] = {0, 1, 4, 5, 6};
        for (int k = 0; k < 5 && st == cudaSuccess; ++k) st = cudaEventElapsedTime(&out[slot[k]], ev[from[k]], ev[to[k]]);
        return st == cudaSuccess ? 0 : fail("cudaEventElapsedTime SFNN backward profile", st);
    }
};

int sfnn_backward_impl(
    BulletOuCudaCppContext* ctx, size_t input_size, size_t ft_size, size_t l1_hidden, int l1_skip, size_t l2_size,
    size_t num_stacks, size_t l1_group_count, size_t l1_common_size, size_t l1_shard_size,
    size_t factorizer_king_axis_dim, size_t factorizer_hand_axis_dim, size_t batch, size_t max_active,
    const BulletOuCudaCppI32Buffer* stm_indices, const BulletOuCudaCppI32Buffer* nstm_indices,
    const BulletOuCudaCppI32Buffer* buckets, const BulletOuCudaCppF32Buffer* stm_l0,
    const BulletOuCudaCppF32Buffer* nstm_l0, const BulletOuCudaCppF32Buffer* combined,
    const BulletOuCudaCppF32Buffer* l1, const BulletOuCudaCppF32Buffer* l2_input, const BulletOuCudaCppF32Buffer* l2,
    const BulletOuCudaCppF32Buffer* l1w, const BulletOuCudaCppF32Buffer* qat_l1w, const BulletOuCudaCppF32Buffer* l1fw,
    int has_l1f, const BulletOuCudaCppF32Buffer* l1axw, int has_l1ax, const BulletOuCudaCppF32Buffer* l2w,
    const BulletOuCudaCppF32Buffer* l2fw, int has_l2f, const BulletOuCudaCppF32Buffer* l2axw, int has_l2ax,
    const BulletOuCudaCppF32Buffer* l3w, const BulletOuCudaCppF32Buffer* l3fw, int has_l3f,
    const BulletOuCudaCppF32Buffer* l3axw, int has_l3ax, int use_king_axis, int use_hand_axis, int use_progress_axis,
    int use_king_hand_pair, int use_king_progress_pair, int use_hand_progress_pair, float ft_factorizer_alpha,
    float factorizer_shared_alpha, float factorizer_king_axis_alpha, float factorizer_hand_axis_alpha,
    float factorizer_progress_axis_alpha, float factorizer_pair_alpha,
    const BulletOuCudaCppF32Buffer* residual_count_gates, const BulletOuCudaCppF32Buffer* factorizer_axis_confidences,
    const BulletOuCudaCppF32Buffer* mean_output_gradients, BulletOuCudaCppF32Buffer* l2_gradients,
    BulletOuCudaCppF32Buffer* l1_gradients, BulletOuCudaCppF32Buffer* l2_input_gradients,
    BulletOuCudaCppF32Buffer* combined_gradients, BulletOuCudaCppF32Buffer* stm_l0_gradients,
    BulletOuCudaCppF32Buffer* nstm_l0_gradients, BulletOuCudaCppF32Buffer* stm_l0_pre_gradients,
    BulletOuCudaCppF32Buffer* nstm_l0_pre_gradients, BulletOuCudaCppF32Buffer* l0w_gradients,
    BulletOuCudaCppF32Buffer* l0b_gradients, BulletOuCudaCppF32Buffer* l1w_gradients,
    BulletOuCudaCppF32Buffer* l1b_gradients, BulletOuCudaCppF32Buffer* l1fw_gradients,
    BulletOuCudaCppF32Buffer* l1fb_gradients, BulletOuCudaCppF32Buffer* l1axw_gradients,
    BulletOuCudaCppF32Buffer* l1axb_gradients, BulletOuCudaCppF32Buffer* l2w_gradients,
    BulletOuCudaCppF32Buffer* l2b_gradients, BulletOuCudaCppF32Buffer* l2fw_gradients,
    BulletOuCudaCppF32Buffer* l2fb_gradients, BulletOuCudaCppF32Buffer* l2axw_gradients,
    BulletOuCudaCppF32Buffer* l2axb_gradients, BulletOuCudaCppF32Buffer* l3w_gradients,
    BulletOuCudaCppF32Buffer* l3b_gradients, BulletOuCudaCppF32Buffer* l3fw_gradients,
    BulletOuCudaCppF32Buffer* l3fb_gradients, BulletOuCudaCppF32Buffer* l3axw_gradients,
    BulletOuCudaCppF32Buffer* l3axb_gradients, int zero_parameter_gradients, BulletOuCudaCppF32Buffer* entry_weights, float* profile_ms, size_t profile_ms_len) {
    (void)factorizer_king_axis_dim;
    (void)factorizer_hand_axis_dim;
    (void)factorizer_king_axis_alpha;
    (void)factorizer_hand_axis_alpha;
    (void)factorizer_progress_axis_alpha;
    (void)factorizer_pair_alpha;
    (void)l1axw;
    (void)l2axw;
    (void)l3axw;
    (void)l1axw_gradients;
    (void)l1axb_gradients;
    (void)l2axw_gradients;
    (void)l2axb_gradients;
    (void)l3axw_gradients;
    (void)l3axb_gradients;
    if (reject_unsupported(l1_group_count, l1_common_size, l1_shard_size, has_l1ax, has_l2ax, has_l3ax, use_king_axis,
                           use_hand_axis, use_progress_axis, use_king_hand_pair, use_king_progress_pair,
                           use_hand_progress_pair, residual_count_gates, factorizer_axis_confidences) != 0)
        return -1;
    SfnnDims d{};
    if (sfnn_dims(input_size, ft_size, l1_hidden, l1_skip, l2_size, num_stacks, batch, max_active, ft_factorizer_alpha,
                  factorizer_shared_alpha, &d) != 0)
        return -1;
    d.has_l1f = has_l1f ? 1 : 0;
    d.has_l2f = has_l2f ? 1 : 0;
    d.has_l3f = has_l3f ? 1 : 0;
    const SfnnGroupLayout g = sfnn_group_layout(d);
    const size_t BW = batch * ft_size;
    BulletOuCudaCppF32Buffer* grads[kSfGroups] = {l0b_gradients,
                                                  l1w_gradients,
                                                  l1b_gradients,
                                                  has_l1f ? l1fw_gradients : nullptr,
                                                  has_l1f ? l1fb_gradients : nullptr,
                                                  l2w_gradients,
                                                  l2b_gradients,
                                                  has_l2f ? l2fw_gradients : nullptr,
                                                  has_l2f ? l2fb_gradients : nullptr,
                                                  l3w_gradients,
                                                  l3b_gradients,
                                                  has_l3f ? l3fw_gradients : nullptr,
                                                  has_l3f ? l3fb_gradients : nullptr};
    static const char* gnames[kSfGroups] = {"l0b_gradients", "l1w_gradients", "l1b_gradients", "l1fw_gradients",
                                            "l1fb_gradients", "l2w_gradients", "l2b_gradients", "l2fw_gradients",
                                            "l2fb_gradients", "l3w_gradients", "l3b_gradients", "l3fw_gradients",
                                            "l3fb_gradients"};
    for (int k = 0; k < kSfGroups; ++k)
        if (g.len[k] && validate_f32(ctx, grads[k], g.len[k], gnames[k]) != 0) return -1;
    if (validate_i32(ctx, stm_indices, batch * max_active, "stm_indices") != 0 ||
        validate_i32(ctx, nstm_indices, batch * max_active, "nstm_indices") != 0 ||
        validate_i32(ctx, buckets, batch, "buckets") != 0 || validate_f32(ctx, stm_l0, BW, "sfnn stm_l0") != 0 ||
        validate_f32(ctx, nstm_l0, BW, "sfnn nstm_l0") != 0 ||
        validate_f32(ctx, l1, batch * d.l1_out, "sfnn l1") != 0 ||
        validate_f32(ctx, l2_input, batch * d.l2_in, "sfnn l2_input") != 0 ||
        validate_f32(ctx, l2, batch * l2_size, "sfnn l2") != 0 ||
        validate_f32(ctx, l1w, g.len[kSfL1w], "sfnn l1w") != 0 || validate_f32(ctx, l2w, g.len[kSfL2w], "sfnn l2w") != 0 ||
        validate_f32(ctx, l3w, g.len[kSfL3w], "sfnn l3w") != 0 ||
        (has_l1f && validate_f32(ctx, l1fw, g.len[kSfL1fw], "sfnn l1fw") != 0) ||
        (has_l2f && validate_f32(ctx, l2fw, g.len[kSfL2fw], "sfnn l2fw") != 0) ||
        (has_l3f && validate_f32(ctx, l3fw, g.len[kSfL3fw], "sfnn l3fw") != 0) ||
        validate_f32(ctx, mean_output_gradients, batch, "mean_output_gradients") != 0 ||
        validate_f32(ctx, l2_gradients, batch * l2_size, "l2_gradients") != 0 ||
        validate_f32(ctx, l1_gradients, batch * d.l1_out, "l1_gradients") != 0 ||
        validate_f32(ctx, l2_input_gradients, batch * d.l2_in, "l2_input_gradients") != 0 ||
        validate_f32(ctx, combined_gradients, BW, "combined_gradients") != 0 ||
        validate_f32(ctx, stm_l0_gradients, BW, "stm_l0_gradients") != 0 ||
        validate_f32(ctx, nstm_l0_gradients, BW, "nstm_l0_gradients") != 0 ||
        validate_f32(ctx, stm_l0_pre_gradients, BW, "stm_l0_pre_gradients") != 0 ||
        validate_f32(ctx, nstm_l0_pre_gradients, BW, "nstm_l0_pre_gradients") != 0 ||
        validate_f32(ctx, l0w_gradients, input_size * ft_size, "l0w_gradients") != 0)
        return -1;
    if (entry_weights != nullptr && validate_f32(ctx, entry_weights, batch, "backward entry weights") != 0) return -1;
    if (qat_l1w != nullptr && validate_f32(ctx, qat_l1w, g.len[kSfL1w], "QAT L1 weights") != 0) return -1;
    d.qat.dense = ctx->dense_qat ? 1 : 0;
    d.qat.l2b_master = ctx->dense_qat_l2_bias;
    d.qat.l3b_master = ctx->dense_qat_l3_bias;
    if (d.qat.dense && (qat_l1w == nullptr || has_l2f || has_l3f))
        return fail_message("dense QAT requires the L1 QAT weights and unfactorized L2/L3");
    if (d.qat.dense && validate_f32(ctx, combined, BW, "sfnn combined") != 0) return -1;
    if (set_device(ctx) != 0) return -1;
    BackwardProfile prof;
    if (prof.init(ctx, profile_ms, profile_ms_len) != 0) return -1;
    if (zero_parameter_gradients) {
        cudaError_t st = cudaMemsetAsync(l0w_gradients->ptr, 0, l0w_gradients->len * sizeof(float), ctx->stream);
        for (int k = 0; k < kSfGroups && st == cudaSuccess; ++k)
            if (g.len[k]) st = cudaMemsetAsync(grads[k]->ptr, 0, g.len[k] * sizeof(float), ctx->stream);
        if (st != cudaSuccess) return fail("cudaMemsetAsync SFNN gradients", st);
    }
    if (prof.mark(ctx) != 0) return -1;
    // The backward reads only the L1 / L2 / L3 weights (and their shared
    // factors); the FT table is not needed, so nothing is folded.
    // With L1 QAT the input gradient uses the folded, fake-quantised weights
    // (identity STE; the shared factor still receives alpha * sum).
    const SfnnWeights w{nullptr,  nullptr, qat_l1w != nullptr ? qat_l1w->ptr : l1w->ptr, nullptr,
                        (has_l1f && qat_l1w == nullptr) ? l1fw->ptr : nullptr, nullptr,
                        l2w->ptr, nullptr, has_l2f ? l2fw->ptr : nullptr, nullptr,
                        l3w->ptr, nullptr, has_l3f ? l3fw->ptr : nullptr, nullptr};
    SfnnPlan plan{};
    SfnnDims dn = d;
    dn.base = 0;
    if (sfnn_prepare(ctx, dn, w, stm_indices->ptr, nstm_indices->ptr, buckets->ptr, nullptr, &plan) != 0) return -1;
    SfnnActivations act{const_cast<float*>(stm_l0->ptr), const_cast<float*>(nstm_l0->ptr), nullptr,
                        const_cast<float*>(l1->ptr),     const_cast<float*>(l2_input->ptr),
                        const_cast<float*>(l2->ptr),     nullptr};
    HeadArgs h = head_args(d, w, plan, act);
    h.mode = kHeadBackward;
    h.mog = const_cast<float*>(mean_output_gradients->ptr);
    h.g1 = l1_gradients->ptr;
    h.l2_gradients = l2_gradients->ptr;
    h.l2_input_gradients = l2_input_gradients->ptr;
    plan.g1 = l1_gradients->ptr;
    if (launch_head(ctx, d, h) != 0 || prof.mark(ctx) != 0) return -1;
    L1BackArgs lb{};
    lb.l0[0] = stm_l0->ptr;
    lb.l0[1] = nstm_l0->ptr;
    lb.combined_gradients = combined_gradients->ptr;
    lb.l0_gradients[0] = stm_l0_gradients->ptr;
    lb.l0_gradients[1] = nstm_l0_gradients->ptr;
    lb.pre_gradients[0] = stm_l0_pre_gradients->ptr;
    lb.pre_gradients[1] = nstm_l0_pre_gradients->ptr;
    lb.combined = d.qat.dense ? combined->ptr : nullptr;
    if (launch_l1_backward(ctx, d, plan, lb) != 0) return -1;
    FinalArgs f{};
    for (int k = 0; k < kSfGroups; ++k) f.dst[k] = g.len[k] ? grads[k]->ptr : nullptr;
    f.accumulate = 1;
    if (launch_finalize(ctx, d, plan, f) != 0 || prof.mark(ctx) != 0) return -1;
    InverseIndex index;
    if (build_inverse_index_rows(ctx, stm_indices->ptr, nstm_indices->ptr, d.batch, d.max_active, d.n_features, &index,
                                 nullptr) != 0 ||
        sort_inverse_index(ctx, index) != 0)
        return -1;
    PieceRowArgs r = piece_row_args(d, index);
    r.src[0] = stm_l0_pre_gradients->ptr;
    r.src[1] = nstm_l0_pre_gradients->ptr;
    r.src_stride = ft_size;
    r.gradients = l0w_gradients->ptr;
    if (launch_piece_rows(ctx, kRowAccumulate, r) != 0 || prof.mark(ctx) != 0 || prof.finish() != 0) return -1;
    return ok();
}

}  // namespace
}  // namespace bou

extern "C" {

#define BOU_SFNN_BACKWARD_PARAMS                                                                                       \
    BulletOuCudaCppContext *ctx, size_t input_size, size_t ft_size, size_t l1_hidden, int l1_skip, size_t l2_size,     \
        size_t num_stacks, size_t l1_group_count, size_t l1_common_size, size_t l1_shard_size,                         \
        size_t factorizer_king_axis_dim, size_t factorizer_hand_axis_dim, size_t batch, size_t max_active,             \
        const BulletOuCudaCppI32Buffer *stm_indices, const BulletOuCudaCppI32Buffer *nstm_indices,                     \
        const BulletOuCudaCppI32Buffer *buckets, const BulletOuCudaCppF32Buffer *stm_l0,                               \
        const BulletOuCudaCppF32Buffer *nstm_l0, const BulletOuCudaCppF32Buffer *combined,                             \
        const BulletOuCudaCppF32Buffer *l1, const BulletOuCudaCppF32Buffer *l2_input,                                  \
        const BulletOuCudaCppF32Buffer *l2, const BulletOuCudaCppF32Buffer *l1w,                                       \
        const BulletOuCudaCppF32Buffer *qat_l1w, const BulletOuCudaCppF32Buffer *l1fw, int has_l1f,                    \
        const BulletOuCudaCppF32Buffer *l1axw, int has_l1ax, const BulletOuCudaCppF32Buffer *l2w,                      \
        const BulletOuCudaCppF32Buffer *l2fw, int has_l2f, const BulletOuCudaCppF32Buffer *l2axw, int has_l2ax,        \
        const BulletOuCudaCppF32Buffer *l3w, const BulletOuCudaCppF32Buffer *l3fw, int has_l3f,                        \
        const BulletOuCudaCppF32Buffer *l3axw, int has_l3ax, int use_king_axis, int use_hand_axis,                     \
        int use_progress_axis, int use_king_hand_pair, int use_king_progress_pair, int use_hand_progress_pair,         \
        float ft_factorizer_alpha, float factorizer_shared_alpha, float factorizer_king_axis_alpha,                    \
        float factorizer_hand_axis_alpha, float factorizer_progress_axis_alpha, float factorizer_pair_alpha,           \
        const BulletOuCudaCppF32Buffer *residual_count_gates,                                                          \
        const BulletOuCudaCppF32Buffer *factorizer_axis_confidences,                                                   \
        const BulletOuCudaCppF32Buffer *mean_output_gradients, BulletOuCudaCppF32Buffer *l2_gradients,                 \
        BulletOuCudaCppF32Buffer *l1_gradients, BulletOuCudaCppF32Buffer *l2_input_gradients,                          \
        BulletOuCudaCppF32Buffer *combined_gradients, BulletOuCudaCppF32Buffer *stm_l0_gradients,                      \
        BulletOuCudaCppF32Buffer *nstm_l0_gradients, BulletOuCudaCppF32Buffer *stm_l0_pre_gradients,                   \
        BulletOuCudaCppF32Buffer *nstm_l0_pre_gradients, BulletOuCudaCppF32Buffer *l0w_gradients,                      \
        BulletOuCudaCppF32Buffer *l0b_gradients, BulletOuCudaCppF32Buffer *l1w_gradients,                              \
        BulletOuCudaCppF32Buffer *l1b_gradients, BulletOuCudaCppF32Buffer *l1fw_gradients,                             \
        BulletOuCudaCppF32Buffer *l1fb_gradients, BulletOuCudaCppF32Buffer *l1axw_gradients,                           \
        BulletOuCudaCppF32Buffer *l1axb_gradients, BulletOuCudaCppF32Buffer *l2w_gradients,                            \
        BulletOuCudaCppF32Buffer *l2b_gradients, BulletOuCudaCppF32Buffer *l2fw_gradients,                             \
        BulletOuCudaCppF32Buffer *l2fb_gradients, BulletOuCudaCppF32Buffer *l2axw_gradients,                           \
        BulletOuCudaCppF32Buffer *l2axb_gradients, BulletOuCudaCppF32Buffer *l3w_gradients,                            \
        BulletOuCudaCppF32Buffer *l3b_gradients, BulletOuCudaCppF32Buffer *l3fw_gradients,                             \
        BulletOuCudaCppF32Buffer *l3fb_gradients, BulletOuCudaCppF32Buffer *l3axw_gradients,                           \
        BulletOuCudaCppF32Buffer *l3axb_gradients
#define BOU_SFNN_BACKWARD_ARGS                                                                                         \
    ctx, input_size, ft_size, l1_hidden, l1_skip, l2_size, num_stacks, l1_group_count, l1_common_size, l1_shard_size, \
        factorizer_king_axis_dim, factorizer_hand_axis_dim, batch, max_active, stm_indices, nstm_indices, buckets,     \
        stm_l0, nstm_l0, combined, l1, l2_input, l2, l1w, qat_l1w, l1fw, has_l1f, l1axw, has_l1ax, l2w, l2fw, has_l2f, \
        l2axw, has_l2ax, l3w, l3fw, has_l3f, l3axw, has_l3ax, use_king_axis, use_hand_axis, use_progress_axis,         \
        use_king_hand_pair, use_king_progress_pair, use_hand_progress_pair, ft_factorizer_alpha,                       \
        factorizer_shared_alpha, factorizer_king_axis_alpha, factorizer_hand_axis_alpha,                               \
        factorizer_progress_axis_alpha, factorizer_pair_alpha, residual_count_gates, factorizer_axis_confidences,      \
        mean_output_gradients, l2_gradients, l1_gradients, l2_input_gradients, combined_gradients, stm_l0_gradients,   \
        nstm_l0_gradients, stm_l0_pre_gradients, nstm_l0_pre_gradients, l0w_gradients, l0b_gradients, l1w_gradients,  \
        l1b_gradients, l1fw_gradients, l1fb_gradients, l1axw_gradients, l1axb_gradients, l2w_gradients, l2b_gradients, \
        l2fw_gradients, l2fb_gradients, l2axw_gradients, l2axb_gradients, l3w_gradients, l3b_gradients, l3fw_gradients,\
        l3fb_gradients, l3axw_gradients, l3axb_gradients

// cu:12882 -- the training backward.
int bulletou_cuda_cpp_sfnn_backward_train_device(BOU_SFNN_BACKWARD_PARAMS, int zero_parameter_gradients,
                                                 BulletOuCudaCppF32Buffer* entry_weights) {
    return sfnn_backward_impl(BOU_SFNN_BACKWARD_ARGS, zero_parameter_gradients, entry_weights, nullptr, 0);
}

// cu:12274 -- the same with every parameter gradient cleared first.
int bulletou_cuda_cpp_sfnn_backward_device(BOU_SFNN_BACKWARD_PARAMS) {
    return sfnn_backward_impl(BOU_SFNN_BACKWARD_ARGS, 1, nullptr, nullptr, 0);
}

// cu:13080 -- the training backward with the stage times in profile_ms[0..7).
int bulletou_cuda_cpp_sfnn_backward_train_profile_device(BOU_SFNN_BACKWARD_PARAMS, int zero_parameter_gradients,
                                                         float* profile_ms, size_t profile_ms_len) {
    return sfnn_backward_impl(BOU_SFNN_BACKWARD_ARGS, zero_parameter_gradients, nullptr, profile_ms, profile_ms_len);
}
#undef BOU_SFNN_BACKWARD_PARAMS
#undef BOU_SFNN_BACKWARD_ARGS

// cu:10937 -- the engine-lattice proxy of the f32 masters (see the header).
int bulletou_cuda_cpp_sfnn_build_quantized_proxy_device(
    BulletOuCudaCppContext* ctx, size_t src_input_size, size_t dst_input_size, size_t virtual_rows, size_t ft_size,
    size_t l1_hidden, int l1_skip, size_t l2_size, size_t num_stacks, size_t l1_group_count, size_t l1_common_size,
    size_t l1_shard_size, size_t factorizer_king_axis_dim, size_t factorizer_hand_axis_dim,
    const BulletOuCudaCppF32Buffer* src_l0w, const BulletOuCudaCppF32Buffer* src_l0b,
    const BulletOuCudaCppF32Buffer* src_l1w, const BulletOuCudaCppF32Buffer* src_l1b,
    const BulletOuCudaCppF32Buffer* src_l1fw, const BulletOuCudaCppF32Buffer* src_l1fb, int has_l1f,
    const BulletOuCudaCppF32Buffer* src_l1axw, const BulletOuCudaCppF32Buffer* src_l1axb, int has_l1ax,
    const BulletOuCudaCppF32Buffer* src_l2w, const BulletOuCudaCppF32Buffer* src_l2b,
    const BulletOuCudaCppF32Buffer* src_l2fw, const BulletOuCudaCppF32Buffer* src_l2fb, int has_l2f,
    const BulletOuCudaCppF32Buffer* src_l2axw, const BulletOuCudaCppF32Buffer* src_l2axb, int has_l2ax,
    const BulletOuCudaCppF32Buffer* src_l3w, const BulletOuCudaCppF32Buffer* src_l3b,
    const BulletOuCudaCppF32Buffer* src_l3fw, const BulletOuCudaCppF32Buffer* src_l3fb, int has_l3f,
    const BulletOuCudaCppF32Buffer* src_l3axw, const BulletOuCudaCppF32Buffer* src_l3axb, int has_l3ax,
    int use_king_axis, int use_hand_axis, int use_progress_axis, int use_king_hand_pair, int use_king_progress_pair,
    int use_hand_progress_pair, float ft_factorizer_alpha, float factorizer_shared_alpha,
    float factorizer_king_axis_alpha, float factorizer_hand_axis_alpha, float factorizer_progress_axis_alpha,
    float factorizer_pair_alpha, const BulletOuCudaCppF32Buffer* residual_count_gates,
    const BulletOuCudaCppF32Buffer* factorizer_axis_confidences, BulletOuCudaCppF32Buffer* dst_l0w,
    BulletOuCudaCppF32Buffer* dst_l0b, BulletOuCudaCppF32Buffer* dst_l1w, BulletOuCudaCppF32Buffer* dst_l1b,
    BulletOuCudaCppF32Buffer* dst_l2w, BulletOuCudaCppF32Buffer* dst_l2b, BulletOuCudaCppF32Buffer* dst_l3w,
    BulletOuCudaCppF32Buffer* dst_l3b, int skip_ft_weights) {
    (void)factorizer_king_axis_dim;
    (void)factorizer_hand_axis_dim;
    (void)factorizer_king_axis_alpha;
    (void)factorizer_hand_axis_alpha;
    (void)factorizer_progress_axis_alpha;
    (void)factorizer_pair_alpha;
    (void)src_l1axw;
    (void)src_l1axb;
    (void)src_l2axw;
    (void)src_l2axb;
    (void)src_l3axw;
    (void)src_l3axb;
    if (set_device(ctx) != 0) return -1;
    if (src_input_size == 0 || dst_input_size == 0 || ft_size == 0 || l2_size == 0 || num_stacks == 0)
        return fail_message("sfnn quantized GPU proxy dimensions must be non-zero");
    if (!(src_input_size == dst_input_size || (virtual_rows != 0 && src_input_size == dst_input_size + virtual_rows)))
        return fail_message("sfnn quantized GPU proxy input sizes do not match base/factorized layout");
    if (reject_unsupported(l1_group_count, l1_common_size, l1_shard_size, has_l1ax, has_l2ax, has_l3ax, use_king_axis,
                           use_hand_axis, use_progress_axis, use_king_hand_pair, use_king_progress_pair,
                           use_hand_progress_pair, residual_count_gates, factorizer_axis_confidences) != 0)
        return -1;
    SfnnDims d{};
    if (sfnn_dims(src_input_size, ft_size, l1_hidden, l1_skip, l2_size, num_stacks, 1, 1, ft_factorizer_alpha,
                  factorizer_shared_alpha, &d) != 0)
        return -1;
    const size_t O = d.l1_out, I2 = d.l2_in, S = num_stacks;
    const size_t vr = src_input_size == dst_input_size ? 0 : virtual_rows;
    if (validate_f32(ctx, src_l0w, src_input_size * ft_size, "sfnn proxy src l0w") != 0 ||
        validate_f32(ctx, src_l0b, ft_size, "sfnn proxy src l0b") != 0 ||
        validate_f32(ctx, src_l1w, S * O * ft_size, "sfnn proxy src l1w") != 0 ||
        validate_f32(ctx, src_l1b, S * O, "sfnn proxy src l1b") != 0 ||
        validate_f32(ctx, src_l2w, S * l2_size * I2, "sfnn proxy src l2w") != 0 ||
        validate_f32(ctx, src_l2b, S * l2_size, "sfnn proxy src l2b") != 0 ||
        validate_f32(ctx, src_l3w, S * l2_size, "sfnn proxy src l3w") != 0 ||
        validate_f32(ctx, src_l3b, S, "sfnn proxy src l3b") != 0 ||
        validate_f32(ctx, dst_l0w, dst_input_size * ft_size, "sfnn proxy dst l0w") != 0 ||
        validate_f32(ctx, dst_l0b, ft_size, "sfnn proxy dst l0b") != 0 ||
        validate_f32(ctx, dst_l1w, S * O * ft_size, "sfnn proxy dst l1w") != 0 ||
        validate_f32(ctx, dst_l1b, S * O, "sfnn proxy dst l1b") != 0 ||
        validate_f32(ctx, dst_l2w, S * l2_size * I2, "sfnn proxy dst l2w") != 0 ||
        validate_f32(ctx, dst_l2b, S * l2_size, "sfnn proxy dst l2b") != 0 ||
        validate_f32(ctx, dst_l3w, S * l2_size, "sfnn proxy dst l3w") != 0 ||
        validate_f32(ctx, dst_l3b, S, "sfnn proxy dst l3b") != 0)
        return -1;
    if (has_l1f && (validate_f32(ctx, src_l1fw, ft_size * O, "sfnn proxy src l1fw") != 0 ||
                    validate_f32(ctx, src_l1fb, O, "sfnn proxy src l1fb") != 0))
        return -1;
    if (has_l2f && (validate_f32(ctx, src_l2fw, l2_size * I2, "sfnn proxy src l2fw") != 0 ||
                    validate_f32(ctx, src_l2fb, l2_size, "sfnn proxy src l2fb") != 0))
        return -1;
    if (has_l3f && (validate_f32(ctx, src_l3fw, l2_size, "sfnn proxy src l3fw") != 0 ||
                    validate_f32(ctx, src_l3fb, 1, "sfnn proxy src l3fb") != 0))
        return -1;
    const int threads = 256;
    int blocks = 0;
    const float alpha = factorizer_shared_alpha;
    if (!skip_ft_weights) {
        if (grid_1d(dst_input_size * ft_size, threads, &blocks, "sfnn proxy l0w") != 0) return -1;
        proxy_ft_kernel<<<blocks, threads, 0, ctx->stream>>>(src_l0w->ptr, dst_l0w->ptr, dst_input_size, vr, ft_size,
                                                             ft_factorizer_alpha);
    }
    qat_vector_kernel<<<(ft_size + threads - 1) / threads, threads, 0, ctx->stream>>>(src_l0b->ptr, dst_l0b->ptr,
                                                                                      ft_size, 0);
    // L1: input-major shared factor [W][O] (cu:11153 passes shared_weight_input_major = 1)
    if (grid_1d(S * O * ft_size, threads, &blocks, "sfnn proxy l1w") != 0) return -1;
    qat_l1_fold_kernel<<<blocks, threads, 0, ctx->stream>>>(src_l1w->ptr, has_l1f ? src_l1fw->ptr : nullptr, alpha,
                                                            S * O * ft_size, static_cast<int>(O),
                                                            static_cast<int>(ft_size), 1, dst_l1w->ptr);
    qat_l1_bias_kernel<<<(S * O + threads - 1) / threads, threads, 0, ctx->stream>>>(
        src_l1b->ptr, has_l1f ? src_l1fb->ptr : nullptr, alpha, static_cast<int>(S * O), static_cast<int>(O), 1,
        dst_l1b->ptr, nullptr, nullptr);
    struct Part {
        const float* src;
        const float* shared;
        size_t cells;
        size_t total;
        int kind;
        float* dst;
    } parts[4] = {
        {src_l2w->ptr, has_l2f ? src_l2fw->ptr : nullptr, l2_size * I2, S * l2_size * I2, 1, dst_l2w->ptr},
        {src_l2b->ptr, has_l2f ? src_l2fb->ptr : nullptr, l2_size, S * l2_size, 2, dst_l2b->ptr},
        {src_l3w->ptr, has_l3f ? src_l3fw->ptr : nullptr, l2_size, S * l2_size, 1, dst_l3w->ptr},
        {src_l3b->ptr, has_l3f ? src_l3fb->ptr : nullptr, 1, S, 2, dst_l3b->ptr},
    };
    for (const Part& q : parts) {
        if (grid_1d(q.total, threads, &blocks, "sfnn proxy dense") != 0) return -1;
        proxy_stacked_kernel<<<blocks, threads, 0, ctx->stream>>>(q.src, q.shared, q.cells, q.total, alpha, q.kind,
                                                                  q.dst);
    }
    return check_launch("sfnn quantized proxy launch");
}

int bulletou_b200_sfnn_dense_gradient_len(const BulletOuB200SfnnShape* shape, int has_l1f, int has_l2f, int has_l3f,
                                          size_t* out) {
    if (shape == nullptr || out == nullptr) return fail_message("SFNN dense_gradient_len arguments must not be null");
    SfnnDims d{};
    if (sfnn_dims(shape->input_size, shape->ft_size, shape->l1_hidden, shape->l1_skip, shape->l2_size,
                  shape->num_stacks, 1, 1, shape->ft_factorizer_alpha, shape->factorizer_shared_alpha, &d) != 0)
        return -1;
    d.has_l1f = has_l1f != 0;
    d.has_l2f = has_l2f != 0;
    d.has_l3f = has_l3f != 0;
    *out = sfnn_group_layout(d).begin[kSfGroups];
    return ok();
}

int bulletou_b200_sfnn_local_gradients_device(
    BulletOuCudaCppContext* ctx, const BulletOuB200SfnnShape* shape, size_t batch, size_t max_active,
    const BulletOuCudaCppI32Buffer* stm_indices, const BulletOuCudaCppI32Buffer* nstm_indices,
    const BulletOuCudaCppI32Buffer* buckets, const BulletOuCudaCppF32Buffer* targets,
    const BulletOuCudaCppF32Buffer* entry_weights, const BulletOuB200LossSpec* loss,
    BulletOuCudaCppF32Buffer* const* params, BulletOuCudaCppF32Buffer* ft_gradients,
    BulletOuCudaCppF32Buffer* dense_gradients, BulletOuCudaCppF32Buffer* output, BulletOuCudaCppF32Buffer* per_sample,
    BulletOuCudaCppF32Buffer* mean_output_gradients, BulletOuCudaCppF32Buffer* weighted_sum,
    BulletOuCudaCppF32Buffer* mean, const BulletOuB200SfnnQat* qat, const size_t* row_shift,
    BulletOuCudaCppEvent* const* row_events, size_t n_row_launches) {
    if (shape == nullptr || params == nullptr) return fail_message("SFNN shape / parameter array must not be null");
    SfnnDims d{};
    LossArgs la{};
    if (sfnn_dims(shape->input_size, shape->ft_size, shape->l1_hidden, shape->l1_skip, shape->l2_size,
                  shape->num_stacks, batch, max_active, shape->ft_factorizer_alpha, shape->factorizer_shared_alpha,
                  &d) != 0 ||
        loss_args(loss, batch, &la) != 0)
        return -1;
    d.has_l1f = params[4] != nullptr;
    d.has_l2f = params[8] != nullptr;
    d.has_l3f = params[12] != nullptr;
    const SfnnGroupLayout g = sfnn_group_layout(d);
    if (validate_sfnn_weights(ctx, d, params, "params") != 0 ||
        validate_i32(ctx, stm_indices, batch * max_active, "stm_indices") != 0 ||
        validate_i32(ctx, nstm_indices, batch * max_active, "nstm_indices") != 0 ||
        validate_i32(ctx, buckets, batch, "buckets") != 0 || validate_f32(ctx, targets, batch, "targets") != 0 ||
        validate_f32(ctx, entry_weights, batch, "entry_weights") != 0 ||
        validate_f32(ctx, ft_gradients,
                     (static_cast<size_t>(d.input_size) +
                      (row_shift != nullptr ? row_shift[piece_row_launches(d, nullptr, 0) - 1] : 0)) * d.width,
                     "ft_gradients") != 0 ||
        validate_f32(ctx, dense_gradients, g.begin[kSfGroups], "dense_gradients") != 0 ||
        validate_f32(ctx, output, batch, "output") != 0 || validate_f32(ctx, per_sample, batch, "per_sample") != 0 ||
        validate_f32(ctx, mean_output_gradients, batch, "mean_output_gradients") != 0 ||
        validate_f32(ctx, weighted_sum, 1, "weighted_sum") != 0 || validate_f32(ctx, mean, 1, "mean") != 0)
        return -1;
    const int launches = piece_row_launches(d, nullptr, 0);
    if ((row_shift != nullptr || row_events != nullptr) && n_row_launches != static_cast<size_t>(launches))
        return fail_messagef("SFNN local gradients: %d row launches, got %zu shifts / events", launches,
                             n_row_launches);
    cudaEvent_t events[64];
    if (row_events != nullptr) {
        if (launches > 64) return fail_message("SFNN local gradients: too many row launches for events");
        for (int j = 0; j < launches; ++j) {
            if (row_events[j] == nullptr || row_events[j]->device != ctx->device)
                return fail_message("SFNN local gradients: row event missing or on another device");
            events[j] = row_events[j]->event;
        }
    }
    if (set_device(ctx) != 0) return -1;
    const SfnnWeights w = weights_from(params);
    if (apply_qat(qat, w, &d) != 0) return -1;
    if (sfnn_step(ctx, d, w, stm_indices->ptr, nstm_indices->ptr, buckets->ptr, targets->ptr, entry_weights->ptr, la,
                  loss->finalize_loss, nullptr, nullptr, nullptr, nullptr, nullptr, output->ptr, per_sample->ptr,
                  mean_output_gradients->ptr, weighted_sum->ptr, mean->ptr, ft_gradients->ptr, dense_gradients->ptr,
                  row_shift, row_events != nullptr ? events : nullptr) != 0)
        return -1;
    return ok();
}

int bulletou_b200_sfnn_local_gradients_exchange_device(
    BulletOuCudaCppContext* ctx, const BulletOuB200SfnnShape* shape, size_t batch, size_t max_active,
    const BulletOuCudaCppI32Buffer* stm_indices, const BulletOuCudaCppI32Buffer* nstm_indices,
    const BulletOuCudaCppI32Buffer* buckets, const BulletOuCudaCppF32Buffer* targets,
    const BulletOuCudaCppF32Buffer* entry_weights, const BulletOuB200LossSpec* loss,
    BulletOuCudaCppF32Buffer* const* params, BulletOuCudaCppF32Buffer* dense_gradients,
    BulletOuCudaCppF32Buffer* output, BulletOuCudaCppF32Buffer* per_sample,
    BulletOuCudaCppF32Buffer* mean_output_gradients, BulletOuCudaCppF32Buffer* weighted_sum,
    BulletOuCudaCppF32Buffer* mean, const BulletOuB200SfnnQat* qat, const BulletOuB200RowExchange* x,
    const size_t* launch_chunk_start, const size_t* launch_shard_rows, const size_t* launch_shard_off,
    const long long* launch_signal, BulletOuCudaCppEvent* const* row_events, size_t n_row_launches) {
    if (shape == nullptr || params == nullptr) return fail_message("SFNN shape / parameter array must not be null");
    if (x == nullptr || launch_chunk_start == nullptr || launch_shard_rows == nullptr || launch_shard_off == nullptr ||
        launch_signal == nullptr)
        return fail_message("SFNN local gradients exchange: the exchange and per-launch arrays must not be null");
    if (x->world < 1 || x->world > static_cast<size_t>(kExchangeMaxRanks) || x->rank >= x->world)
        return fail_messagef("SFNN local gradients exchange: world %zu / rank %zu outside 1..%d", x->world, x->rank,
                             kExchangeMaxRanks);
    SfnnDims d{};
    LossArgs la{};
    if (sfnn_dims(shape->input_size, shape->ft_size, shape->l1_hidden, shape->l1_skip, shape->l2_size,
                  shape->num_stacks, batch, max_active, shape->ft_factorizer_alpha, shape->factorizer_shared_alpha,
                  &d) != 0 ||
        loss_args(loss, batch, &la) != 0)
        return -1;
    d.has_l1f = params[4] != nullptr;
    d.has_l2f = params[8] != nullptr;
    d.has_l3f = params[12] != nullptr;
    const SfnnGroupLayout g = sfnn_group_layout(d);
    if (validate_sfnn_weights(ctx, d, params, "params") != 0 ||
        validate_i32(ctx, stm_indices, batch * max_active, "stm_indices") != 0 ||
        validate_i32(ctx, nstm_indices, batch * max_active, "nstm_indices") != 0 ||
        validate_i32(ctx, buckets, batch, "buckets") != 0 || validate_f32(ctx, targets, batch, "targets") != 0 ||
        validate_f32(ctx, entry_weights, batch, "entry_weights") != 0 ||
        validate_f32(ctx, dense_gradients, g.begin[kSfGroups], "dense_gradients") != 0 ||
        validate_f32(ctx, output, batch, "output") != 0 || validate_f32(ctx, per_sample, batch, "per_sample") != 0 ||
        validate_f32(ctx, mean_output_gradients, batch, "mean_output_gradients") != 0 ||
        validate_f32(ctx, weighted_sum, 1, "weighted_sum") != 0 || validate_f32(ctx, mean, 1, "mean") != 0)
        return -1;
    const int launches = piece_row_launches(d, nullptr, 0);
    if (n_row_launches != static_cast<size_t>(launches))
        return fail_messagef("SFNN local gradients exchange: %d row launches, got %zu", launches, n_row_launches);
    RowScatter sc{};
    sc.world = static_cast<int>(x->world);
    sc.rank = static_cast<int>(x->rank);
    sc.slot_rows = x->slot_rows;
    sc.chunk_start = launch_chunk_start;
    sc.shard_rows = launch_shard_rows;
    sc.shard_off = launch_shard_off;
    sc.signal = launch_signal;
    sc.epoch = x->epoch;
    size_t ends[64];
    if (launches > 64) return fail_message("SFNN local gradients exchange: too many row launches");
    piece_row_launches(d, ends, 64);
    size_t row0 = 0;
    for (int j = 0; j < launches; ++j) {
        // every row of launch j must fall in its chunk's rows, and the chunk's
        // shard inside a receive slot
        const size_t row_end = ends[j];
        const size_t sr = launch_shard_rows[j];
        if (sr == 0 || launch_chunk_start[j] > row0 || row_end - launch_chunk_start[j] > sr * x->world ||
            launch_shard_off[j] + sr > x->slot_rows || launch_signal[j] >= static_cast<long long>(launches))
            return fail_messagef("SFNN local gradients exchange: launch %d's chunk does not hold its rows", j);
        row0 = row_end;
    }
    for (size_t r = 0; r < x->world; ++r) {
        if (x->recv[r] == 0 || x->flags[r] == 0) return fail_messagef("row exchange: rank %zu's buffers missing", r);
        sc.recv[r] = reinterpret_cast<float*>(static_cast<uintptr_t>(x->recv[r]));
        sc.flags.p[r] = reinterpret_cast<int*>(static_cast<uintptr_t>(x->flags[r]));
    }
    if (x->small_len > 0) {
        if (x->small_len != g.begin[kSfGroups])
            return fail_messagef("SFNN local gradients exchange: small_len %zu, the packed gradient holds %zu",
                                 x->small_len, static_cast<size_t>(g.begin[kSfGroups]));
        for (size_t r = 0; r < x->world; ++r) {
            if (x->small_recv[r] == 0) return fail_messagef("row exchange: rank %zu's small buffer missing", r);
            sc.small.p[r] = reinterpret_cast<float*>(static_cast<uintptr_t>(x->small_recv[r]));
        }
        sc.small_len = x->small_len;
        sc.small_flag_base = x->small_flag_base;
    }
    cudaEvent_t events[64];
    if (row_events != nullptr) {
        for (int j = 0; j < launches; ++j) {
            if (row_events[j] == nullptr || row_events[j]->device != ctx->device)
                return fail_message("SFNN local gradients exchange: row event missing or on another device");
            events[j] = row_events[j]->event;
        }
    }
    if (set_device(ctx) != 0) return -1;
    const SfnnWeights w = weights_from(params);
    if (apply_qat(qat, w, &d) != 0) return -1;
    if (sfnn_step(ctx, d, w, stm_indices->ptr, nstm_indices->ptr, buckets->ptr, targets->ptr, entry_weights->ptr, la,
                  loss->finalize_loss, nullptr, nullptr, nullptr, nullptr, nullptr, output->ptr, per_sample->ptr,
                  mean_output_gradients->ptr, weighted_sum->ptr, mean->ptr, nullptr, dense_gradients->ptr, nullptr,
                  row_events != nullptr ? events : nullptr, &sc) != 0)
        return -1;
    return ok();
}

int bulletou_b200_sfnn_row_launches(const BulletOuB200SfnnShape* shape, size_t* n_launches, size_t* row_end,
                                    size_t cap) {
    if (shape == nullptr || n_launches == nullptr) return fail_message("SFNN row launches: null argument");
    SfnnDims d{};
    if (sfnn_dims(shape->input_size, shape->ft_size, shape->l1_hidden, shape->l1_skip, shape->l2_size,
                  shape->num_stacks, 1, 1, shape->ft_factorizer_alpha, shape->factorizer_shared_alpha, &d) != 0)
        return -1;
    *n_launches = static_cast<size_t>(piece_row_launches(d, row_end, cap));
    return ok();
}

int bulletou_b200_sfnn_train_step_device(
    BulletOuCudaCppContext* ctx, const BulletOuB200SfnnShape* shape, size_t batch, size_t max_active,
    const BulletOuCudaCppI32Buffer* stm_indices, const BulletOuCudaCppI32Buffer* nstm_indices,
    const BulletOuCudaCppI32Buffer* buckets, const BulletOuCudaCppF32Buffer* targets,
    const BulletOuCudaCppF32Buffer* entry_weights, const BulletOuB200LossSpec* loss,
    const BulletOuB200RangerStep* ranger, BulletOuCudaCppF32Buffer* const* params,
    BulletOuCudaCppF32Buffer* const* momentum, BulletOuCudaCppF32Buffer* const* velocity,
    BulletOuCudaCppF32Buffer* const* slow_params, BulletOuCudaCppF32Buffer* output, BulletOuCudaCppF32Buffer* per_sample,
    BulletOuCudaCppF32Buffer* mean_output_gradients, BulletOuCudaCppF32Buffer* weighted_sum,
    BulletOuCudaCppF32Buffer* mean, const BulletOuB200SfnnQat* qat) {
    if (shape == nullptr) return fail_message("SFNN shape must not be null");
    if (ranger == nullptr) return fail_message("ranger step must not be null");
    if (params == nullptr || momentum == nullptr || velocity == nullptr || slow_params == nullptr)
        return fail_message("SFNN parameter / optimizer-state arrays must not be null");
    if (ranger->norm_loss_rate != 0.0f)
        return fail_message("SFNN fused step: the SFNN runner applies no norm loss with default multipliers; pass 0");
    SfnnDims d{};
    LossArgs la{};
    if (sfnn_dims(shape->input_size, shape->ft_size, shape->l1_hidden, shape->l1_skip, shape->l2_size,
                  shape->num_stacks, batch, max_active, shape->ft_factorizer_alpha, shape->factorizer_shared_alpha,
                  &d) != 0 ||
        loss_args(loss, batch, &la) != 0)
        return -1;
    d.has_l1f = params[4] != nullptr;
    d.has_l2f = params[8] != nullptr;
    d.has_l3f = params[12] != nullptr;
    if (validate_sfnn_weights(ctx, d, params, "params") != 0 || validate_sfnn_weights(ctx, d, momentum, "momentum") != 0 ||
        validate_sfnn_weights(ctx, d, velocity, "velocity") != 0 ||
        validate_sfnn_weights(ctx, d, slow_params, "slow_params") != 0 ||
        validate_i32(ctx, stm_indices, batch * max_active, "stm_indices") != 0 ||
        validate_i32(ctx, nstm_indices, batch * max_active, "nstm_indices") != 0 ||
        validate_i32(ctx, buckets, batch, "buckets") != 0 || validate_f32(ctx, targets, batch, "targets") != 0 ||
        validate_f32(ctx, entry_weights, batch, "entry_weights") != 0 ||
        validate_f32(ctx, output, batch, "output") != 0 || validate_f32(ctx, per_sample, batch, "per_sample") != 0 ||
        validate_f32(ctx, mean_output_gradients, batch, "mean_output_gradients") != 0 ||
        validate_f32(ctx, weighted_sum, 1, "weighted_sum") != 0 || validate_f32(ctx, mean, 1, "mean") != 0)
        return -1;
    if (set_device(ctx) != 0) return -1;
    float* wm[14];
    float* mm[14];
    float* vm[14];
    float* smm[14];
    for (int i = 0; i < 14; ++i) {
        wm[i] = params[i] ? params[i]->ptr : nullptr;
        mm[i] = momentum[i] ? momentum[i]->ptr : nullptr;
        vm[i] = velocity[i] ? velocity[i]->ptr : nullptr;
        smm[i] = slow_params[i] ? slow_params[i]->ptr : nullptr;
    }
    const SfnnWeights w = weights_from(params);
    if (apply_qat(qat, w, &d) != 0) return -1;
    if (sfnn_step(ctx, d, w, stm_indices->ptr, nstm_indices->ptr, buckets->ptr, targets->ptr, entry_weights->ptr, la,
                  loss->finalize_loss, ranger, wm, mm, vm, smm, output->ptr, per_sample->ptr,
                  mean_output_gradients->ptr, weighted_sum->ptr, mean->ptr, nullptr, nullptr) != 0)
        return -1;
    return ok();
}

// Fake-quantised copy of one layer's tensor (layer_qat.rs:832-880): scale 127
// (FT, i16; with vr > 0 the virtual rows are folded into the base rows and
// zeroed), 64 (dense weights, i8) or 8128 (dense biases, i32).
int bulletou_layer_qat(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* src, BulletOuCudaCppF32Buffer* dst,
                       float scale, float lo, float hi, size_t base, size_t vr, size_t width, float alpha) {
    (void)lo;
    (void)hi;
    if (ctx == nullptr || src == nullptr || dst == nullptr) return fail_message("layer QAT arguments must not be null");
    if (validate_f32(ctx, src, src->len, "layer QAT input") != 0 ||
        validate_f32(ctx, dst, src->len, "layer QAT output") != 0 || set_device(ctx) != 0)
        return -1;
    if (src->len == 0) return ok();
    int blocks = 0;
    if (grid_1d(src->len, 256, &blocks, "layer QAT") != 0) return -1;
    if (vr != 0) {
        if (width == 0 || src->len != (base + vr) * width) return fail_message("invalid layer QAT FT layout");
        layer_qat_ft_kernel<<<blocks, 256, 0, ctx->stream>>>(src->ptr, dst->ptr, base, vr, width, alpha, src->len);
    } else if (scale == 127.0f) {
        qat_vector_kernel<<<blocks, 256, 0, ctx->stream>>>(src->ptr, dst->ptr, src->len, 0);
    } else if (scale == 64.0f) {
        qat_vector_kernel<<<blocks, 256, 0, ctx->stream>>>(src->ptr, dst->ptr, src->len, 1);
    } else if (scale == 8128.0f) {
        qat_vector_kernel<<<blocks, 256, 0, ctx->stream>>>(src->ptr, dst->ptr, src->len, 2);
    } else {
        return fail_message("unsupported layer QAT scale");
    }
    if (check_launch("layer QAT launch") != 0) return -1;
    return ok();
}

// flag[0] = 1 when any element of w or b is nonzero (the FT QAT zero check).
int bulletou_layer_qat_nonzero(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* w, BulletOuCudaCppF32Buffer* b,
                               BulletOuCudaCppF32Buffer* flag) {
    if (ctx == nullptr || w == nullptr || b == nullptr || flag == nullptr)
        return fail_message("FT QAT zero check arguments must not be null");
    if (validate_f32(ctx, w, w->len, "FT QAT weights") != 0 || validate_f32(ctx, b, b->len, "FT QAT bias") != 0 ||
        validate_f32(ctx, flag, 1, "FT QAT flag") != 0 || set_device(ctx) != 0)
        return -1;
    int blocks = 0;
    if (grid_1d(w->len + b->len, 256, &blocks, "FT QAT zero check") != 0) return -1;
    if (blocks > 0) nonzero_kernel<<<blocks, 256, 0, ctx->stream>>>(w->ptr, w->len, b->ptr, b->len, flag->ptr);
    if (check_launch("FT QAT zero check launch") != 0) return -1;
    return ok();
}

// Enters dense QAT: the SFNN forward / backward entries of this context run the
// integer L1 / L2 / L3 with these master biases until bulletou_dense_qat_end.
int bulletou_dense_qat_begin(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* l2_bias,
                             BulletOuCudaCppF32Buffer* l3_bias, size_t batch, size_t l1_out, size_t l2_size,
                             size_t stacks, int integer_ft) {
    if (ctx == nullptr || batch == 0 || l1_out == 0 || l2_size == 0 || stacks == 0)
        return fail_message("invalid dense QAT dimensions");
    if (validate_f32(ctx, l2_bias, stacks * l2_size, "dense QAT master L2 bias") != 0 ||
        validate_f32(ctx, l3_bias, stacks, "dense QAT master L3 bias") != 0 || set_device(ctx) != 0)
        return -1;
    ctx->dense_qat_l2_bias = l2_bias->ptr;
    ctx->dense_qat_l3_bias = l3_bias->ptr;
    ctx->dense_qat = true;
    ctx->dense_qat_integer_ft = integer_ft != 0;
    return ok();
}

void bulletou_dense_qat_end(BulletOuCudaCppContext* ctx) {
    if (ctx == nullptr) return;
    ctx->dense_qat = false;
    ctx->dense_qat_integer_ft = false;
    ctx->dense_qat_l2_bias = nullptr;
    ctx->dense_qat_l3_bias = nullptr;
}

}  // extern "C"
