// Quantised SFNN inference on B200: export quantisation of trained f32
// weights and the engine's integer forward, bit-exact.
//
// Reference: examples/bulletou.rs (the reference's CPU evaluation path)
//   quantisation   10050-10300 (folds 26417-26444, 21339-21520; rounding 26481-26493)
//   integer forward 8001-8163  (quantized_sfnn_ft_pair_value, _clipped_relu,
//                               _sqr_clipped_relu, _forward_sample)
// Engine format: FT i16 at scale 127 (bias and weights doubled and summed with
// i16 wrap-around), dense i8 weights at 64 with rows padded to 32 inputs,
// dense i32 biases at 127 * 64.  Every integer sum here is exact, so the
// result does not depend on the summation order.
//
// Kernels:
//   quantize_ft / quantize_dense -- element-wise folds and rounding (double,
//       half away from zero; f32 folds without fused multiply-add, as the
//       reference's Rust arithmetic).
//   int_ft_kernel   -- warp per half-position in king order: 16-byte i16
//       loads, i32 sums, i16 wrap, [0, 254] clamp, pair product -> u8.
//   int_head_kernel -- warp per sample: L1 as u8 x i8 dp4a dot products,
//       SqrCReLU | CReLU, L2, L3 + PSQT skip -> raw i32 output.
#include <climits>
#include <cstdint>

#include "king_sort.cuh"
#include "sfnn.cuh"

namespace bou {
namespace {

constexpr unsigned kFull = 0xffffffffu;

__device__ __forceinline__ int16_t q16(float v, float s) {
    double q = round(static_cast<double>(v) * static_cast<double>(s));
    q = fmin(fmax(q, -32768.0), 32767.0);
    return static_cast<int16_t>(q);
}
__device__ __forceinline__ int8_t q8(float v, float s) {
    double q = round(static_cast<double>(v) * static_cast<double>(s));
    q = fmin(fmax(q, -128.0), 127.0);
    return static_cast<int8_t>(q);
}
__device__ __forceinline__ int32_t q32(float v, float s) {
    double q = round(static_cast<double>(v) * static_cast<double>(s));
    q = fmin(fmax(q, -2147483648.0), 2147483647.0);
    return static_cast<int32_t>(q);
}
// a + alpha * b with two roundings (no fused multiply-add), as in Rust f32.
__device__ __forceinline__ float fold(float a, float alpha, float b) { return __fadd_rn(a, __fmul_rn(alpha, b)); }

__host__ __device__ inline int pad32(int n) { return (n + 31) / 32 * 32; }

struct QuantArgs {
    const float* w[14];
    int16_t* l0w;
    int16_t* l0b;
    int8_t* l1w;
    int32_t* l1b;
    int8_t* l2w;
    int32_t* l2b;
    int8_t* l3w;
    int32_t* l3b;
    int rows;   // quantised FT rows (the factorizer base, or input_size)
    int base;   // > 0: fold virtual rows base + r % 1629
    int width;
    int out_dim;
    int l2_size;
    int l2_in;
    int stacks;
    float ft_alpha;
    float shared_alpha;
};

__global__ void quantize_ft_kernel(QuantArgs a) {
    const size_t t = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const size_t n = static_cast<size_t>(a.rows) * a.width;
    if (t < n) {
        const size_t r = t / a.width, j = t - r * a.width;
        float v = a.w[0][t];
        if (a.base > 0) v = fold(v, a.ft_alpha, a.w[0][(static_cast<size_t>(a.base) + r % kSfnnPieces) * a.width + j]);
        a.l0w[t] = q16(v, 127.0f);
    }
    if (t < static_cast<size_t>(a.width)) a.l0b[t] = q16(a.w[1][t], 127.0f);
}

// One thread per padded dense weight or bias of every stack.
__global__ void quantize_dense_kernel(QuantArgs a) {
    const int O = a.out_dim, W = a.width, L2 = a.l2_size, I2 = a.l2_in;
    const int p1 = pad32(W), p2 = pad32(I2), p3 = pad32(L2);
    const size_t per = static_cast<size_t>(O) * p1 + O + static_cast<size_t>(L2) * p2 + L2 + p3 + 1;
    const size_t t = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= per * a.stacks) return;
    const int s = static_cast<int>(t / per);
    size_t r = t - static_cast<size_t>(s) * per;
    const float al = a.shared_alpha;
    if (r < static_cast<size_t>(O) * p1) {
        const int o = static_cast<int>(r / p1), i = static_cast<int>(r % p1);
        int8_t q = 0;
        if (i < W) {
            float v = a.w[2][(static_cast<size_t>(s) * O + o) * W + i];
            if (a.w[4] != nullptr) v = fold(v, al, a.w[4][static_cast<size_t>(i) * O + o]);
            q = q8(v, 64.0f);
        }
        a.l1w[(static_cast<size_t>(s) * O + o) * p1 + i] = q;
        return;
    }
    r -= static_cast<size_t>(O) * p1;
    if (r < static_cast<size_t>(O)) {
        float b = a.w[3][s * O + r];
        if (a.w[5] != nullptr) b = fold(b, al, a.w[5][r]);
        a.l1b[s * O + r] = q32(b, 8128.0f);
        return;
    }
    r -= O;
    if (r < static_cast<size_t>(L2) * p2) {
        const int o = static_cast<int>(r / p2), i = static_cast<int>(r % p2);
        int8_t q = 0;
        if (i < I2) {
            float v = a.w[6][(static_cast<size_t>(s) * L2 + o) * I2 + i];
            if (a.w[8] != nullptr) v = fold(v, al, a.w[8][static_cast<size_t>(o) * I2 + i]);
            q = q8(v, 64.0f);
        }
        a.l2w[(static_cast<size_t>(s) * L2 + o) * p2 + i] = q;
        return;
    }
    r -= static_cast<size_t>(L2) * p2;
    if (r < static_cast<size_t>(L2)) {
        float b = a.w[7][s * L2 + r];
        if (a.w[9] != nullptr) b = fold(b, al, a.w[9][r]);
        a.l2b[s * L2 + r] = q32(b, 8128.0f);
        return;
    }
    r -= L2;
    if (r < static_cast<size_t>(p3)) {
        int8_t q = 0;
        if (static_cast<int>(r) < L2) {
            float v = a.w[10][s * L2 + r];
            if (a.w[12] != nullptr) v = fold(v, al, a.w[12][r]);
            q = q8(v, 64.0f);
        }
        a.l3w[static_cast<size_t>(s) * p3 + r] = q;
        return;
    }
    float b = a.w[11][s];
    if (a.w[13] != nullptr) b = fold(b, al, a.w[13][0]);
    a.l3b[s] = q32(b, 8128.0f);
}

// ------------------------------------------------------------------ integer forward
struct IntArgs {
    const int* order;  // king order of half-positions (null in the generic kernel)
    const int* stm;
    const int* nstm;
    const int* buckets;
    const int16_t* l0w;
    const int16_t* l0b;
    const int8_t* l1w;
    const int32_t* l1b;
    const int8_t* l2w;
    const int32_t* l2b;
    const int8_t* l3w;
    const int32_t* l3b;
    uint8_t* ft;       // [B][W] pair values
    int32_t* l1_out;   // optional [B][O]
    int32_t* raw;      // [B]
    int32_t* score;    // optional [B]: raw / fv_scale
    int* errors;       // optional: count of out-of-range features / buckets
    int n_half;
    int batch;
    int max_active;
    int rows;
    int width;
    int hidden;
    int out_dim;
    int skip;
    int l2_size;
    int stacks;
    int ft_shift;
    int ft_round;
    int crelu_round;
    int sqr_round;
    int final_round;
    int fv_scale;
};

__device__ __forceinline__ uint8_t pair_value(int32_t s0, int32_t s1, const IntArgs& a) {
    int32_t x0 = static_cast<int32_t>(static_cast<int16_t>(s0));
    int32_t x1 = static_cast<int32_t>(static_cast<int16_t>(s1));
    x0 = min(max(x0, 0), 254);
    x1 = min(max(x1, 0), 254);
    long long p = (static_cast<long long>(x0) << a.ft_shift) * x1;
    p = a.ft_round ? (p + (1LL << 15)) >> 16 : p >> 16;
    return static_cast<uint8_t>(p > 255 ? 255 : (p < 0 ? 0 : p));
}

// Warp per half-position; W % 512 == 0.  Lane owns columns 256 k + 8 lane + e;
// column chunk k pairs with chunk k + NCH/2 (width / 2 apart).
template <int NCH>
__global__ void __launch_bounds__(256) int_ft_kernel(IntArgs a) {
    const int lane = threadIdx.x & 31;
    const int pos = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (pos >= a.n_half) return;
    const int h = a.order[pos];
    const int b = h >> 1, v = h & 1;
    const int* idx = (v ? a.nstm : a.stm) + static_cast<size_t>(b) * a.max_active;
    int32_t acc[NCH][8];
#pragma unroll
    for (int k = 0; k < NCH; ++k) {
        const int4 raw = __ldg(reinterpret_cast<const int4*>(a.l0b + 256 * k + 8 * lane));
        const int16_t* e = reinterpret_cast<const int16_t*>(&raw);
#pragma unroll
        for (int q = 0; q < 8; ++q) acc[k][q] = 2 * static_cast<int32_t>(e[q]);
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
            const int16_t* row = a.l0w + static_cast<size_t>(f) * a.width + 8 * lane;
            int4 r[NCH];
#pragma unroll
            for (int k = 0; k < NCH; ++k) r[k] = __ldg(reinterpret_cast<const int4*>(row + 256 * k));
#pragma unroll
            for (int k = 0; k < NCH; ++k) {
                const int16_t* e = reinterpret_cast<const int16_t*>(&r[k]);
#pragma unroll
                for (int q = 0; q < 8; ++q) acc[k][q] += 2 * static_cast<int32_t>(e[q]);
            }
        }
    }
    if (bad && lane == 0 && a.errors != nullptr) atomicAdd(a.errors, bad);
    uint8_t* out = a.ft + static_cast<size_t>(b) * a.width + v * (a.width / 2) + 8 * lane;
#pragma unroll
    for (int k = 0; k < NCH / 2; ++k) {
        uint32_t lo = 0, hi = 0;
#pragma unroll
        for (int q = 0; q < 4; ++q) lo |= static_cast<uint32_t>(pair_value(acc[k][q], acc[k + NCH / 2][q], a)) << (8 * q);
#pragma unroll
        for (int q = 0; q < 4; ++q)
            hi |= static_cast<uint32_t>(pair_value(acc[k][q + 4], acc[k + NCH / 2][q + 4], a)) << (8 * q);
        *reinterpret_cast<uint2*>(out + 256 * k) = make_uint2(lo, hi);
    }
}

// Any even width: thread per (half-position, pair).
__global__ void int_ft_generic_kernel(IntArgs a) {
    const int half = a.width / 2;
    const size_t t = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= static_cast<size_t>(a.n_half) * half) return;
    const int h = static_cast<int>(t / half);
    const int j = static_cast<int>(t - static_cast<size_t>(h) * half);
    const int b = h >> 1, v = h & 1;
    const int* idx = (v ? a.nstm : a.stm) + static_cast<size_t>(b) * a.max_active;
    int32_t s0 = 2 * static_cast<int32_t>(a.l0b[j]), s1 = 2 * static_cast<int32_t>(a.l0b[half + j]);
    int bad = 0;
    for (int k = 0; k < a.max_active; ++k) {
        const int f = idx[k];
        if (f < 0) continue;
        if (f >= a.rows) {
            ++bad;
            continue;
        }
        s0 += 2 * static_cast<int32_t>(a.l0w[static_cast<size_t>(f) * a.width + j]);
        s1 += 2 * static_cast<int32_t>(a.l0w[static_cast<size_t>(f) * a.width + half + j]);
    }
    if (bad && j == 0 && a.errors != nullptr) atomicAdd(a.errors, bad);
    a.ft[static_cast<size_t>(b) * a.width + v * half + j] = pair_value(s0, s1, a);
}

__device__ __forceinline__ int dp4a_us(uint32_t u8x4, int32_t s8x4, int acc) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(u8x4), "r"(s8x4), "r"(acc));
    return d;
}

__device__ __forceinline__ int warp_sum(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
    return v;
}

// Warp per sample: L1 (u8 x i8 over the FT pair values), L2 input, L2, L3.
__global__ void __launch_bounds__(256) int_head_kernel(IntArgs a) {
    const int lane = threadIdx.x & 31;
    const int b = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (b >= a.batch) return;
    const int s = a.buckets[b];
    if (s < 0 || s >= a.stacks) {
        if (lane == 0) {
            a.raw[b] = 0;
            if (a.score != nullptr) a.score[b] = 0;
            if (a.errors != nullptr) atomicAdd(a.errors, 1);
        }
        return;
    }
    const int W = a.width, O = a.out_dim, H = a.hidden, L2 = a.l2_size, I2 = 2 * H;
    const int p1 = pad32(W), p2 = pad32(I2), p3 = pad32(L2);
    const uint8_t* ft = a.ft + static_cast<size_t>(b) * W;
    int l1_lane = 0;  // lane o < O ends with l1[o]
    const bool words = (W % 4) == 0;
    for (int o = 0; o < O; ++o) {
        const int8_t* row = a.l1w + (static_cast<size_t>(s) * O + o) * p1;
        int sum = 0;
        if (words) {
            for (int w4 = lane; w4 < W / 4; w4 += 32)
                sum = dp4a_us(reinterpret_cast<const uint32_t*>(ft)[w4], reinterpret_cast<const int32_t*>(row)[w4],
                              sum);
        } else {
            for (int i = lane; i < W; i += 32) sum += static_cast<int>(ft[i]) * static_cast<int>(row[i]);
        }
        sum = warp_sum(sum) + a.l1b[s * O + o];
        if (lane == o) l1_lane = sum;
    }
    if (a.l1_out != nullptr && lane < O) a.l1_out[static_cast<size_t>(b) * O + lane] = l1_lane;
    // L2 input: lane i < H holds SqrCReLU(l1[i]), CReLU(l1[i])
    int sq = 0, cr = 0;
    if (lane < H) {
        const long long x = l1_lane;
        long long v = a.sqr_round ? (x * x + (1LL << 18)) >> 19 : (x * x) >> 19;
        sq = static_cast<int>(v > 127 ? 127 : v);
        int c = (a.crelu_round && l1_lane > 0) ? (l1_lane + 32) >> 6 : l1_lane >> 6;
        cr = min(max(c, 0), 127);
    }
    // L2: output o handled by lane o (and o + 32 ...)
    int out_part = 0;
    for (int o0 = 0; o0 < L2; o0 += 32) {
        const int o = o0 + lane;
        int sum = o < L2 ? a.l2b[s * L2 + o] : 0;
        const int8_t* row = a.l2w + (static_cast<size_t>(s) * L2 + (o < L2 ? o : 0)) * p2;
        for (int i = 0; i < H; ++i) {
            const int xs = __shfl_sync(kFull, sq, i);
            const int xc = __shfl_sync(kFull, cr, i);
            if (o < L2) sum += xs * static_cast<int>(row[i]) + xc * static_cast<int>(row[H + i]);
        }
        if (o < L2) {
            int c = (a.crelu_round && sum > 0) ? (sum + 32) >> 6 : sum >> 6;
            c = min(max(c, 0), 127);
            out_part += c * static_cast<int>(a.l3w[static_cast<size_t>(s) * p3 + o]);
        }
    }
    int out = warp_sum(out_part) + a.l3b[s];
    const int skip = __shfl_sync(kFull, l1_lane, H < 32 ? H : 0);
    if (a.skip) out += skip;
    if (lane == 0) {
        a.raw[b] = out;
        if (a.score != nullptr) {
            // Integer division truncating toward zero; "nearest" adds half the
            // scale away from zero first (bulletou.rs:8045-8054).
            const int half = a.fv_scale / 2;
            a.score[b] = !a.final_round ? out / a.fv_scale
                                        : (out >= 0 ? (out + half) / a.fv_scale : (out - half) / a.fv_scale);
        }
    }
}

}  // namespace
}  // namespace bou

using namespace bou;

namespace {

void quant_lengths(const SfnnDims& d, size_t* lens) {
    const size_t W = d.width, O = d.l1_out, L2 = d.l2_size, S = d.stacks;
    lens[0] = static_cast<size_t>(d.n_features) * W;  // l0w i16
    lens[1] = W;                                      // l0b i16
    lens[2] = S * O * pad32(d.width);                 // l1w i8
    lens[3] = S * O;                                  // l1b i32
    lens[4] = S * L2 * pad32(d.l2_in);                // l2w i8
    lens[5] = S * L2;                                 // l2b i32
    lens[6] = S * pad32(d.l2_size);                   // l3w i8
    lens[7] = S;                                      // l3b i32
}

int validate_quant(BulletOuCudaCppContext* ctx, const SfnnDims& d, BulletOuCudaCppI32Buffer* const* q) {
    size_t lens[8];
    quant_lengths(d, lens);
    static const int bytes[8] = {2, 2, 1, 4, 1, 4, 1, 4};
    static const char* names[8] = {"l0w_q", "l0b_q", "l1w_q", "l1b_q", "l2w_q", "l2b_q", "l3w_q", "l3b_q"};
    if (q == nullptr) return fail_message("quantised SFNN buffer array must not be null");
    for (int i = 0; i < 8; ++i)
        if (validate_i32(ctx, q[i], (lens[i] * bytes[i] + 3) / 4, names[i]) != 0) return -1;
    return 0;
}

int shape_dims(const BulletOuB200SfnnShape* shape, size_t batch, size_t max_active, SfnnDims* d) {
    if (shape == nullptr) return fail_message("SFNN shape must not be null");
    return sfnn_dims(shape->input_size, shape->ft_size, shape->l1_hidden, shape->l1_skip, shape->l2_size,
                     shape->num_stacks, batch, max_active, shape->ft_factorizer_alpha, shape->factorizer_shared_alpha,
                     d);
}

}  // namespace

extern "C" {

int bulletou_b200_sfnn_quantize_device(BulletOuCudaCppContext* ctx, const BulletOuB200SfnnShape* shape,
                                       BulletOuCudaCppF32Buffer* const* params,
                                       BulletOuCudaCppI32Buffer* const* quantized) {
    SfnnDims d{};
    if (shape_dims(shape, 1, 1, &d) != 0) return -1;
    if (params == nullptr) return fail_message("SFNN parameter array must not be null");
    d.has_l1f = params[4] != nullptr;
    d.has_l2f = params[8] != nullptr;
    d.has_l3f = params[12] != nullptr;
    const SfnnGroupLayout g = sfnn_group_layout(d);
    static const char* names[14] = {"l0w", "l0b", "l1w", "l1b", "l1fw", "l1fb", "l2w",
                                    "l2b", "l2fw", "l2fb", "l3w", "l3b", "l3fw", "l3fb"};
    if (validate_f32(ctx, params[0], static_cast<size_t>(d.input_size) * d.width, "l0w") != 0) return -1;
    for (int k = 0; k < kSfGroups; ++k) {
        if (g.len[k] == 0) continue;
        if (validate_f32(ctx, params[k + 1], g.len[k], names[k + 1]) != 0) return -1;
    }
    if (validate_quant(ctx, d, quantized) != 0) return -1;
    if (set_device(ctx) != 0) return -1;
    QuantArgs a{};
    for (int i = 0; i < 14; ++i) a.w[i] = params[i] != nullptr ? params[i]->ptr : nullptr;
    a.l0w = reinterpret_cast<int16_t*>(quantized[0]->ptr);
    a.l0b = reinterpret_cast<int16_t*>(quantized[1]->ptr);
    a.l1w = reinterpret_cast<int8_t*>(quantized[2]->ptr);
    a.l1b = reinterpret_cast<int32_t*>(quantized[3]->ptr);
    a.l2w = reinterpret_cast<int8_t*>(quantized[4]->ptr);
    a.l2b = reinterpret_cast<int32_t*>(quantized[5]->ptr);
    a.l3w = reinterpret_cast<int8_t*>(quantized[6]->ptr);
    a.l3b = reinterpret_cast<int32_t*>(quantized[7]->ptr);
    a.rows = d.n_features;
    a.base = d.base;
    a.width = d.width;
    a.out_dim = d.l1_out;
    a.l2_size = d.l2_size;
    a.l2_in = d.l2_in;
    a.stacks = d.stacks;
    a.ft_alpha = d.ft_alpha;
    a.shared_alpha = d.shared_alpha;
    int blocks = 0;
    if (grid_1d(static_cast<size_t>(d.n_features) * d.width, 256, &blocks, "SFNN FT quantisation") != 0) return -1;
    quantize_ft_kernel<<<blocks, 256, 0, ctx->stream>>>(a);
    const size_t per = static_cast<size_t>(d.l1_out) * pad32(d.width) + d.l1_out +
                       static_cast<size_t>(d.l2_size) * pad32(d.l2_in) + d.l2_size + pad32(d.l2_size) + 1;
    if (grid_1d(per * d.stacks, 256, &blocks, "SFNN dense quantisation") != 0) return -1;
    quantize_dense_kernel<<<blocks, 256, 0, ctx->stream>>>(a);
    if (check_launch("SFNN quantisation launch") != 0) return -1;
    return ok();
}

int bulletou_b200_sfnn_integer_forward_device(BulletOuCudaCppContext* ctx, const BulletOuB200SfnnShape* shape,
                                              size_t batch, size_t max_active,
                                              const BulletOuCudaCppI32Buffer* stm_indices,
                                              const BulletOuCudaCppI32Buffer* nstm_indices,
                                              const BulletOuCudaCppI32Buffer* buckets,
                                              BulletOuCudaCppI32Buffer* const* quantized,
                                              const BulletOuB200QuantRounding* rounding,
                                              BulletOuCudaCppI32Buffer* l1_out, BulletOuCudaCppI32Buffer* raw_output,
                                              BulletOuCudaCppI32Buffer* score_output,
                                              BulletOuCudaCppI32Buffer* errors) {
    SfnnDims d{};
    if (shape_dims(shape, batch, max_active, &d) != 0) return -1;
    if (rounding == nullptr) return fail_message("integer forward: rounding must not be null");
    if (rounding->ft_shift < 0 || rounding->ft_shift > 16)
        return fail_message("integer forward: ft_shift must be in [0, 16]");
    if (score_output != nullptr && rounding->fv_scale <= 0)
        return fail_message("integer forward: fv_scale must be greater than zero");
    if (validate_quant(ctx, d, quantized) != 0 ||
        validate_i32(ctx, stm_indices, batch * max_active, "stm_indices") != 0 ||
        validate_i32(ctx, nstm_indices, batch * max_active, "nstm_indices") != 0 ||
        validate_i32(ctx, buckets, batch, "buckets") != 0 || validate_i32(ctx, raw_output, batch, "raw_output") != 0 ||
        (l1_out != nullptr && validate_i32(ctx, l1_out, batch * d.l1_out, "l1_out") != 0) ||
        (score_output != nullptr && validate_i32(ctx, score_output, batch, "score_output") != 0) ||
        (errors != nullptr && validate_i32(ctx, errors, 1, "errors") != 0))
        return -1;
    if (set_device(ctx) != 0) return -1;
    IntArgs a{};
    a.stm = stm_indices->ptr;
    a.nstm = nstm_indices->ptr;
    a.buckets = buckets->ptr;
    a.l0w = reinterpret_cast<const int16_t*>(quantized[0]->ptr);
    a.l0b = reinterpret_cast<const int16_t*>(quantized[1]->ptr);
    a.l1w = reinterpret_cast<const int8_t*>(quantized[2]->ptr);
    a.l1b = reinterpret_cast<const int32_t*>(quantized[3]->ptr);
    a.l2w = reinterpret_cast<const int8_t*>(quantized[4]->ptr);
    a.l2b = reinterpret_cast<const int32_t*>(quantized[5]->ptr);
    a.l3w = reinterpret_cast<const int8_t*>(quantized[6]->ptr);
    a.l3b = reinterpret_cast<const int32_t*>(quantized[7]->ptr);
    a.l1_out = l1_out != nullptr ? l1_out->ptr : nullptr;
    a.raw = raw_output->ptr;
    a.score = score_output != nullptr ? score_output->ptr : nullptr;
    a.errors = errors != nullptr ? errors->ptr : nullptr;
    a.n_half = 2 * d.batch;
    a.batch = d.batch;
    a.max_active = d.max_active;
    a.rows = d.n_features;
    a.width = d.width;
    a.hidden = d.l1_hidden;
    a.out_dim = d.l1_out;
    a.skip = d.l1_skip;
    a.l2_size = d.l2_size;
    a.stacks = d.stacks;
    a.ft_shift = rounding->ft_shift;
    a.ft_round = rounding->ft_round != 0;
    a.crelu_round = rounding->crelu_round != 0;
    a.sqr_round = rounding->sqr_clipped_relu_round != 0;
    a.final_round = rounding->final_div_round != 0;
    a.fv_scale = rounding->fv_scale;
    // scratch: FT pair values [B][W] u8 | king sort
    const size_t ft_bytes = (static_cast<size_t>(d.batch) * d.width + 255) & ~static_cast<size_t>(255);
    const size_t sort_ints = king_sort_scratch_ints<kSfnnKingKeys>(a.n_half);
    void* p = nullptr;
    if (scratch_slot(ctx, kScratchSfnnQuant, ft_bytes + sort_ints * sizeof(int), &p,
                     "cudaMalloc SFNN integer scratch") != 0)
        return -1;
    a.ft = static_cast<uint8_t*>(p);
    if (a.errors != nullptr) {
        cudaError_t st = cudaMemsetAsync(a.errors, 0, sizeof(int), ctx->stream);
        if (st != cudaSuccess) return fail("cudaMemsetAsync integer forward errors", st);
    }
    if (d.width % 512 == 0 && d.width <= 2560) {
        KingSortOut sorted{};
        const int piece = (d.n_features % kSfnnPieces == 0) ? kSfnnPieces : d.n_features;
        if (king_sort<kSfnnKingKeys>(ctx, a.stm, a.nstm, a.n_half, KingKey{piece, d.n_features, d.max_active},
                                     reinterpret_cast<int*>(static_cast<char*>(p) + ft_bytes), nullptr, &sorted) != 0)
            return -1;
        a.order = sorted.order;
        const int blocks = (a.n_half + 7) / 8;
        switch (d.width / 256) {
            case 2: int_ft_kernel<2><<<blocks, 256, 0, ctx->stream>>>(a); break;
            case 4: int_ft_kernel<4><<<blocks, 256, 0, ctx->stream>>>(a); break;
            case 6: int_ft_kernel<6><<<blocks, 256, 0, ctx->stream>>>(a); break;
            case 8: int_ft_kernel<8><<<blocks, 256, 0, ctx->stream>>>(a); break;
            default: int_ft_kernel<10><<<blocks, 256, 0, ctx->stream>>>(a); break;
        }
    } else {
        int blocks = 0;
        if (grid_1d(static_cast<size_t>(a.n_half) * (d.width / 2), 256, &blocks, "SFNN integer FT") != 0) return -1;
        int_ft_generic_kernel<<<blocks, 256, 0, ctx->stream>>>(a);
    }
    int_head_kernel<<<(d.batch + 7) / 8, 256, 0, ctx->stream>>>(a);
    if (check_launch("SFNN integer forward launch") != 0) return -1;
    return ok();
}

}  // extern "C"
