// Quantised HalfKP 256x2-32-32 on B200: the reference's nn.bin quantisation
// of a trained f32 net and the engine's integer evaluation of it, bit-exact.
//
// Quantisation (write_cuda_cpp_nnue_nn_bin, examples/bulletou.rs:26303-26413;
// scales in crates/bulletou_lib/src/value/nnue_save.rs:223-252): FT i16 at 127
// (factorized tables: the 1548 leading virtual rows added to every base row),
// dense i8 at 64 transposed to output-major with rows padded to 32 inputs,
// biases i32 at 127 * 64; round half away from zero in double.  The reference
// refuses values outside the integer range; here they saturate and are
// counted in an error word.
//
// Integer forward (the engine's halfkp_256x2-32-32 evaluation): per
// perspective, side to move first, an i16 accumulator (bias + rows, wrapping)
// clamped to [0, 127]; affine layers bias + sum u8 * i8 in i32 then
// clamp(x >> 6, 0, 127); output bias + sum; score = raw / fv_scale.
//
// Kernels:
//   nnue_quantize_kernel -- element-wise, one thread per output integer.
//   nnue_int_ft_kernel   -- warp per half-position; the 64 MB i16 table stays in
//                           L2.  Sums modulo 2^16 kept as packed halves.
//   nnue_int_head_kernel -- warp per sample, lane = output unit, the dense
//                           weights in shared memory; dp4a dot products.
#include <algorithm>
#include <climits>
#include <cstdint>

#include "common.cuh"

namespace bou {
namespace {

constexpr unsigned kFull = 0xffffffffu;
constexpr int kHalfkpBase = 125388;
constexpr int kHalfkpPieces = 1548;

__host__ __device__ inline int pad32i(int n) { return (n + 31) / 32 * 32; }

struct NnueQuantArgs {
    const float* w[8];  // l0w l0b l1w l1b l2w l2b outw outb
    int16_t* l0w;
    int16_t* l0b;
    int8_t* l1w;
    int32_t* l1b;
    int8_t* l2w;
    int32_t* l2b;
    int8_t* outw;
    int32_t* outb;
    int* errors;
    int rows;
    int factorized;
    int l1;
    int l2;
    int l3;
};

__device__ __forceinline__ long long q_round(double v, double lo, double hi, int* bad) {
    double q = round(v);
    if (q < lo) {
        q = lo;
        *bad = 1;
    }
    if (q > hi) {
        q = hi;
        *bad = 1;
    }
    return static_cast<long long>(q);
}

// Work items: FT rows*l1 | l0b l1 | l1w l2*pad32(2 l1) | l1b l2 | l2w l3*pad32(l2) | l2b l3 | outw pad32(l3) | outb 1
__global__ void nnue_quantize_kernel(NnueQuantArgs a) {
    const size_t t = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int L1 = a.l1, L2 = a.l2, L3 = a.l3, I1 = 2 * L1;
    const int p1 = pad32i(I1), p2 = pad32i(L2), p3 = pad32i(L3);
    const size_t n0 = static_cast<size_t>(a.rows) * L1;
    const size_t n1 = n0 + L1;
    const size_t n2 = n1 + static_cast<size_t>(L2) * p1;
    const size_t n3 = n2 + L2;
    const size_t n4 = n3 + static_cast<size_t>(L3) * p2;
    const size_t n5 = n4 + L3;
    const size_t n6 = n5 + p3;
    const size_t n7 = n6 + 1;
    int bad = 0;
    if (t < n0) {
        const size_t r = t / L1, j = t - r * L1;
        // factorized: base row r is stored after the virtual rows; add its piece's virtual row
        const float v = a.factorized ? __fadd_rn(a.w[0][(kHalfkpPieces + r) * L1 + j], a.w[0][(r % kHalfkpPieces) * L1 + j])
                                     : a.w[0][t];
        a.l0w[t] = static_cast<int16_t>(q_round(127.0 * static_cast<double>(v), -32768.0, 32767.0, &bad));
    } else if (t < n1) {
        const size_t j = t - n0;
        a.l0b[j] = static_cast<int16_t>(q_round(127.0 * static_cast<double>(a.w[1][j]), -32768.0, 32767.0, &bad));
    } else if (t < n2) {
        const size_t r = t - n1;
        const int o = static_cast<int>(r / p1), i = static_cast<int>(r % p1);
        a.l1w[r] = i < I1 ? static_cast<int8_t>(q_round(64.0 * static_cast<double>(a.w[2][static_cast<size_t>(i) * L2 + o]),
                                                        -128.0, 127.0, &bad))
                          : 0;
    } else if (t < n3) {
        const size_t o = t - n2;
        a.l1b[o] = static_cast<int32_t>(q_round(8128.0 * static_cast<double>(a.w[3][o]), -2147483648.0, 2147483647.0, &bad));
    } else if (t < n4) {
        const size_t r = t - n3;
        const int o = static_cast<int>(r / p2), i = static_cast<int>(r % p2);
        a.l2w[r] = i < L2 ? static_cast<int8_t>(q_round(64.0 * static_cast<double>(a.w[4][static_cast<size_t>(i) * L3 + o]),
                                                        -128.0, 127.0, &bad))
                          : 0;
    } else if (t < n5) {
        const size_t o = t - n4;
        a.l2b[o] = static_cast<int32_t>(q_round(8128.0 * static_cast<double>(a.w[5][o]), -2147483648.0, 2147483647.0, &bad));
    } else if (t < n6) {
        const int i = static_cast<int>(t - n5);
        a.outw[i] = i < L3 ? static_cast<int8_t>(q_round(64.0 * static_cast<double>(a.w[6][i]), -128.0, 127.0, &bad)) : 0;
    } else if (t < n7) {
        a.outb[0] = static_cast<int32_t>(q_round(8128.0 * static_cast<double>(a.w[7][0]), -2147483648.0, 2147483647.0, &bad));
    }
    const int block_bad = __syncthreads_count(bad);
    if (block_bad != 0 && threadIdx.x == 0 && a.errors != nullptr) atomicAdd(a.errors, block_bad);
}

struct NnueIntArgs {
    const int* stm;
    const int* nstm;
    const int16_t* l0w;
    const int16_t* l0b;
    const int8_t* l1w;
    const int32_t* l1b;
    const int8_t* l2w;
    const int32_t* l2b;
    const int8_t* outw;
    const int32_t* outb;
    uint8_t* x;  // [B][2 l1] transformed features
    int32_t* raw;
    int32_t* score;
    int* errors;
    int n_half;
    int max_active;
    int rows;
    int l1;
    int l2;
    int l3;
    int fv_scale;
};

// Warp per half-position (l1 % 256 == 0): lane owns columns 256 k + 8 lane + e.
// Sums modulo 2^16: each 32-bit word of two i16 columns is added whole into
// `lo` (even column in its low half) and shifted into `hi` (odd column).
template <int NCH>
__global__ void __launch_bounds__(256) nnue_int_ft_kernel(NnueIntArgs a) {
    const int lane = threadIdx.x & 31;
    const int h = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (h >= a.n_half) return;
    const int b = h >> 1, v = h & 1;
    const int* idx = (v ? a.nstm : a.stm) + static_cast<size_t>(b) * a.max_active;
    unsigned lo[NCH][4], hi[NCH][4];
#pragma unroll
    for (int k = 0; k < NCH; ++k) {
        const uint4 bw = __ldg(reinterpret_cast<const uint4*>(a.l0b + 256 * k + 8 * lane));
        const unsigned w4[4] = {bw.x, bw.y, bw.z, bw.w};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            lo[k][c] = w4[c];
            hi[k][c] = w4[c] >> 16;
        }
    }
    int bad = 0;
    for (int s0 = 0; s0 < a.max_active; s0 += 32) {
        const int mine = s0 + lane < a.max_active ? __ldg(idx + s0 + lane) : -1;
        const int n = min(32, a.max_active - s0);
        for (int u = 0; u < n; ++u) {
            const int f = __shfl_sync(kFull, mine, u);
            if (f < 0) continue;
            if (f >= a.rows) {
                ++bad;
                continue;
            }
            const int16_t* row = a.l0w + static_cast<size_t>(f) * a.l1 + 8 * lane;
            uint4 r[NCH];
#pragma unroll
            for (int k = 0; k < NCH; ++k) r[k] = __ldg(reinterpret_cast<const uint4*>(row + 256 * k));
#pragma unroll
            for (int k = 0; k < NCH; ++k) {
                lo[k][0] += r[k].x;
                hi[k][0] += r[k].x >> 16;
                lo[k][1] += r[k].y;
                hi[k][1] += r[k].y >> 16;
                lo[k][2] += r[k].z;
                hi[k][2] += r[k].z >> 16;
                lo[k][3] += r[k].w;
                hi[k][3] += r[k].w >> 16;
            }
        }
    }
    if (bad && lane == 0 && a.errors != nullptr) atomicAdd(a.errors, bad);
    uint8_t* out = a.x + static_cast<size_t>(b) * 2 * a.l1 + v * a.l1 + 8 * lane;
#pragma unroll
    for (int k = 0; k < NCH; ++k) {
        unsigned word[2] = {0u, 0u};
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const unsigned sw = (q & 1) ? hi[k][q >> 1] : lo[k][q >> 1];
            const int s = min(127, max(0, static_cast<int>(static_cast<short>(sw))));
            word[q >> 2] |= static_cast<unsigned>(s) << (8 * (q & 3));
        }
        *reinterpret_cast<uint2*>(out + 256 * k) = make_uint2(word[0], word[1]);
    }
}

// Any l1: thread per (half-position, column).
__global__ void nnue_int_ft_generic_kernel(NnueIntArgs a) {
    const size_t t = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= static_cast<size_t>(a.n_half) * a.l1) return;
    const int h = static_cast<int>(t / a.l1);
    const int j = static_cast<int>(t - static_cast<size_t>(h) * a.l1);
    const int b = h >> 1, v = h & 1;
    const int* idx = (v ? a.nstm : a.stm) + static_cast<size_t>(b) * a.max_active;
    int acc = a.l0b[j];
    int bad = 0;
    for (int k = 0; k < a.max_active; ++k) {
        const int f = idx[k];
        if (f < 0) continue;
        if (f >= a.rows) {
            ++bad;
            continue;
        }
        acc += a.l0w[static_cast<size_t>(f) * a.l1 + j];
    }
    if (bad && j == 0 && a.errors != nullptr) atomicAdd(a.errors, bad);
    a.x[static_cast<size_t>(b) * 2 * a.l1 + v * a.l1 + j] =
        static_cast<uint8_t>(min(127, max(0, static_cast<int>(static_cast<short>(acc)))));
}

__device__ __forceinline__ int dp4a_us(unsigned u8x4, int s8x4, int acc) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(u8x4), "r"(s8x4), "r"(acc));
    return d;
}

// Warp per sample, lane o = output unit (l2, l3 <= 32); block-stride loop over
// samples.  Shared memory: L1 rows with a stride of pad32(2 l1) / 4 + 1 words
// (conflict-free per lane), L2 rows, output weights.
__global__ void __launch_bounds__(256) nnue_int_head_kernel(NnueIntArgs a, int batch) {
    extern __shared__ int smem[];
    const int I1 = 2 * a.l1;
    const int p1w = pad32i(I1) / 4, p2 = pad32i(a.l2), p3 = pad32i(a.l3);
    const int s1 = p1w + 1;
    int* w1 = smem;                                   // [l2][s1] words of 4 i8
    int8_t* w2 = reinterpret_cast<int8_t*>(w1 + a.l2 * s1);  // [l3][p2]
    int8_t* w3 = w2 + a.l3 * p2;                      // [p3]
    for (int i = threadIdx.x; i < a.l2 * p1w; i += blockDim.x) {
        const int o = i / p1w, k = i - o * p1w;
        w1[o * s1 + k] = reinterpret_cast<const int*>(a.l1w)[i];
    }
    for (int i = threadIdx.x; i < a.l3 * p2; i += blockDim.x) w2[i] = a.l2w[i];
    for (int i = threadIdx.x; i < p3; i += blockDim.x) w3[i] = a.outw[i];
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int warps = blockDim.x >> 5;
    for (int b = blockIdx.x * warps + (threadIdx.x >> 5); b < batch; b += gridDim.x * warps) {
        const unsigned* xw = reinterpret_cast<const unsigned*>(a.x + static_cast<size_t>(b) * I1);
        int h1 = 0;
        if (lane < a.l2) {
            int s = a.l1b[lane];
            const int* wr = w1 + lane * s1;
            for (int k = 0; k < I1 / 4; ++k) s = dp4a_us(__ldg(xw + k), wr[k], s);
            h1 = min(127, max(0, s >> 6));
        }
        int s2 = lane < a.l3 ? a.l2b[lane] : 0;
        for (int i = 0; i < a.l2; ++i) {
            const int hv = __shfl_sync(kFull, h1, i);
            if (lane < a.l3) s2 += hv * static_cast<int>(w2[lane * p2 + i]);
        }
        const int h2 = lane < a.l3 ? min(127, max(0, s2 >> 6)) : 0;
        int part = lane < a.l3 ? h2 * static_cast<int>(w3[lane]) : 0;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(kFull, part, o);
        if (lane == 0) {
            const int raw = part + a.outb[0];
            a.raw[b] = raw;
            if (a.score != nullptr) a.score[b] = raw / a.fv_scale;
        }
    }
}

int nnue_quant_dims(size_t input_size, size_t l1, size_t l2, size_t l3, int* rows) {
    if (input_size == 0 || l1 == 0 || l2 == 0 || l3 == 0) return fail_message("NNUE shape must be non-zero");
    if (l1 > 4096 || l1 % 2 != 0 || l2 > 32 || l3 > 32 || input_size > static_cast<size_t>(INT_MAX) / 2)
        return fail_message("quantised NNUE on this backend: even l1 <= 4096, l2 <= 32, l3 <= 32");
    *rows = input_size == static_cast<size_t>(kHalfkpBase + kHalfkpPieces) ? kHalfkpBase : static_cast<int>(input_size);
    return 0;
}

void nnue_quant_lengths(int rows, size_t l1, size_t l2, size_t l3, size_t* n) {
    n[0] = static_cast<size_t>(rows) * l1;
    n[1] = l1;
    n[2] = l2 * pad32i(static_cast<int>(2 * l1));
    n[3] = l2;
    n[4] = l3 * pad32i(static_cast<int>(l2));
    n[5] = l3;
    n[6] = pad32i(static_cast<int>(l3));
    n[7] = 1;
}

int validate_nnue_quant(BulletOuCudaCppContext* ctx, int rows, size_t l1, size_t l2, size_t l3,
                        BulletOuCudaCppI32Buffer* const* q) {
    static const int bytes[8] = {2, 2, 1, 4, 1, 4, 1, 4};
    static const char* names[8] = {"l0w_q", "l0b_q", "l1w_q", "l1b_q", "l2w_q", "l2b_q", "outw_q", "outb_q"};
    if (q == nullptr) return fail_message("quantised NNUE buffer array must not be null");
    size_t n[8];
    nnue_quant_lengths(rows, l1, l2, l3, n);
    for (int i = 0; i < 8; ++i)
        if (validate_i32(ctx, q[i], (n[i] * bytes[i] + 3) / 4, names[i]) != 0) return -1;
    return 0;
}

}  // namespace
}  // namespace bou

using namespace bou;

extern "C" {

int bulletou_b200_nnue_quantize_device(BulletOuCudaCppContext* ctx, size_t input_size, size_t l1, size_t l2,
                                       size_t l3, BulletOuCudaCppF32Buffer* const* params,
                                       BulletOuCudaCppI32Buffer* const* quantized, BulletOuCudaCppI32Buffer* errors) {
    int rows = 0;
    if (nnue_quant_dims(input_size, l1, l2, l3, &rows) != 0) return -1;
    if (params == nullptr) return fail_message("NNUE parameter array must not be null");
    const size_t lens[8] = {input_size * l1, l1, 2 * l1 * l2, l2, l2 * l3, l3, l3, 1};
    static const char* names[8] = {"l0w", "l0b", "l1w", "l1b", "l2w", "l2b", "outw", "outb"};
    for (int i = 0; i < 8; ++i)
        if (validate_f32(ctx, params[i], lens[i], names[i]) != 0) return -1;
    if (validate_nnue_quant(ctx, rows, l1, l2, l3, quantized) != 0) return -1;
    if (errors != nullptr && validate_i32(ctx, errors, 1, "errors") != 0) return -1;
    if (set_device(ctx) != 0) return -1;
    NnueQuantArgs a{};
    for (int i = 0; i < 8; ++i) a.w[i] = params[i]->ptr;
    a.l0w = reinterpret_cast<int16_t*>(quantized[0]->ptr);
    a.l0b = reinterpret_cast<int16_t*>(quantized[1]->ptr);
    a.l1w = reinterpret_cast<int8_t*>(quantized[2]->ptr);
    a.l1b = reinterpret_cast<int32_t*>(quantized[3]->ptr);
    a.l2w = reinterpret_cast<int8_t*>(quantized[4]->ptr);
    a.l2b = reinterpret_cast<int32_t*>(quantized[5]->ptr);
    a.outw = reinterpret_cast<int8_t*>(quantized[6]->ptr);
    a.outb = reinterpret_cast<int32_t*>(quantized[7]->ptr);
    a.errors = errors != nullptr ? errors->ptr : nullptr;
    a.rows = rows;
    a.factorized = rows != static_cast<int>(input_size);
    a.l1 = static_cast<int>(l1);
    a.l2 = static_cast<int>(l2);
    a.l3 = static_cast<int>(l3);
    if (a.errors != nullptr) {
        cudaError_t st = cudaMemsetAsync(a.errors, 0, sizeof(int), ctx->stream);
        if (st != cudaSuccess) return fail("cudaMemsetAsync NNUE quantise errors", st);
    }
    size_t n[8];
    nnue_quant_lengths(rows, l1, l2, l3, n);
    size_t total = 0;
    for (size_t v : n) total += v;
    int blocks = 0;
    if (grid_1d(total, 256, &blocks, "NNUE quantisation") != 0) return -1;
    nnue_quantize_kernel<<<blocks, 256, 0, ctx->stream>>>(a);
    if (check_launch("NNUE quantisation launch") != 0) return -1;
    return ok();
}

int bulletou_b200_nnue_integer_forward_device(BulletOuCudaCppContext* ctx, size_t input_size, size_t l1, size_t l2,
                                              size_t l3, size_t batch, size_t max_active,
                                              const BulletOuCudaCppI32Buffer* stm_indices,
                                              const BulletOuCudaCppI32Buffer* nstm_indices,
                                              BulletOuCudaCppI32Buffer* const* quantized, int fv_scale,
                                              BulletOuCudaCppI32Buffer* raw_output,
                                              BulletOuCudaCppI32Buffer* score_output,
                                              BulletOuCudaCppI32Buffer* errors) {
    int rows = 0;
    if (nnue_quant_dims(input_size, l1, l2, l3, &rows) != 0) return -1;
    if (batch == 0 || max_active == 0 || batch > (1u << 26) || max_active > 4096)
        return fail_message("integer NNUE forward: batch / max_active out of range");
    if (score_output != nullptr && fv_scale <= 0) return fail_message("integer NNUE forward: fv_scale must be > 0");
    if (validate_nnue_quant(ctx, rows, l1, l2, l3, quantized) != 0 ||
        validate_i32(ctx, stm_indices, batch * max_active, "stm_indices") != 0 ||
        validate_i32(ctx, nstm_indices, batch * max_active, "nstm_indices") != 0 ||
        validate_i32(ctx, raw_output, batch, "raw_output") != 0 ||
        (score_output != nullptr && validate_i32(ctx, score_output, batch, "score_output") != 0) ||
        (errors != nullptr && validate_i32(ctx, errors, 1, "errors") != 0))
        return -1;
    if (set_device(ctx) != 0) return -1;
    NnueIntArgs a{};
    a.stm = stm_indices->ptr;
    a.nstm = nstm_indices->ptr;
    a.l0w = reinterpret_cast<const int16_t*>(quantized[0]->ptr);
    a.l0b = reinterpret_cast<const int16_t*>(quantized[1]->ptr);
    a.l1w = reinterpret_cast<const int8_t*>(quantized[2]->ptr);
    a.l1b = reinterpret_cast<const int32_t*>(quantized[3]->ptr);
    a.l2w = reinterpret_cast<const int8_t*>(quantized[4]->ptr);
    a.l2b = reinterpret_cast<const int32_t*>(quantized[5]->ptr);
    a.outw = reinterpret_cast<const int8_t*>(quantized[6]->ptr);
    a.outb = reinterpret_cast<const int32_t*>(quantized[7]->ptr);
    a.raw = raw_output->ptr;
    a.score = score_output != nullptr ? score_output->ptr : nullptr;
    a.errors = errors != nullptr ? errors->ptr : nullptr;
    a.n_half = static_cast<int>(2 * batch);
    a.max_active = static_cast<int>(max_active);
    a.rows = rows;
    a.l1 = static_cast<int>(l1);
    a.l2 = static_cast<int>(l2);
    a.l3 = static_cast<int>(l3);
    a.fv_scale = fv_scale > 0 ? fv_scale : 1;
    void* p = nullptr;
    if (scratch_slot(ctx, kScratchNnueQuant, batch * 2 * l1, &p, "cudaMalloc NNUE integer features") != 0) return -1;
    a.x = static_cast<uint8_t*>(p);
    if (a.errors != nullptr) {
        cudaError_t st = cudaMemsetAsync(a.errors, 0, sizeof(int), ctx->stream);
        if (st != cudaSuccess) return fail("cudaMemsetAsync integer NNUE errors", st);
    }
    if (l1 % 256 == 0 && l1 <= 2048) {
        const int blocks = (a.n_half + 7) / 8;
        switch (l1 / 256) {
            case 1: nnue_int_ft_kernel<1><<<blocks, 256, 0, ctx->stream>>>(a); break;
            case 2: nnue_int_ft_kernel<2><<<blocks, 256, 0, ctx->stream>>>(a); break;
            case 3: nnue_int_ft_kernel<3><<<blocks, 256, 0, ctx->stream>>>(a); break;
            case 4: nnue_int_ft_kernel<4><<<blocks, 256, 0, ctx->stream>>>(a); break;
            default: {
                int gb = 0;
                if (grid_1d(static_cast<size_t>(a.n_half) * l1, 256, &gb, "integer NNUE FT") != 0) return -1;
                nnue_int_ft_generic_kernel<<<gb, 256, 0, ctx->stream>>>(a);
            }
        }
    } else {
        int gb = 0;
        if (grid_1d(static_cast<size_t>(a.n_half) * l1, 256, &gb, "integer NNUE FT") != 0) return -1;
        nnue_int_ft_generic_kernel<<<gb, 256, 0, ctx->stream>>>(a);
    }
    const int p1w = pad32i(static_cast<int>(2 * l1)) / 4;
    const size_t smem = static_cast<size_t>(l2) * (p1w + 1) * 4 + l3 * pad32i(static_cast<int>(l2)) +
                        pad32i(static_cast<int>(l3));
    if (smem > 200 * 1024) return fail_message("integer NNUE forward: dense weights exceed shared memory");
    cudaError_t st = cudaFuncSetAttribute(nnue_int_head_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          static_cast<int>(smem));
    if (st != cudaSuccess) return fail("cudaFuncSetAttribute integer NNUE head", st);
    const int grid = static_cast<int>(std::min<size_t>((batch + 7) / 8, static_cast<size_t>(ctx->sm_count) * 8));
    nnue_int_head_kernel<<<grid, 256, smem, ctx->stream>>>(a, static_cast<int>(batch));
    if (check_launch("integer NNUE forward launch") != 0) return -1;
    return ok();
}

}  // extern "C"
