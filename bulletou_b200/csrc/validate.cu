// Validation on the device: the held-out metrics of the reference's
// compute_sign_accuracy_with_loss_masked (crates/bulletou_lib/src/validate.rs:
// 353-470; sign accuracy over the decisive positions, the loss over every
// position that passes the score cap) computed from the model outputs and the
// teacher records already in HBM, and the reference backend's activation
// statistics entries (bulletou_cuda_cpp_sfnn_validation_stats,
// bulletou_cuda_cpp_sfnn_unit_stats, cu:2659-2730 / 13485-13531).
//
// The metrics reduce per CTA (counts as integers, the loss as a double tree)
// and then over CTAs in a fixed order, so they are deterministic; the loss
// sum is a double like the reference's (its order differs, well below the
// f32 test loss it reports).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "common.cuh"

namespace bou {
namespace {

constexpr int kValThreads = 256;
constexpr int kValCounts = 8;  // compared, sign_matches, predicted_nonnegative, predicted_negative,
                               // predicted_zero, drawn_games, filtered_by_score_cap, loss_sampled

struct ValArgs {
    const float* outputs;
    const uint32_t* records;  // PackedSfenValue, 10 words each
    int n;
    int have_results;
    int score_drop_abs;       // < 0: none
    int loss_kind;            // 0 sigmoid-pow, 1 win-rate model, 2 BCE with logits
    float lambda;
    float eval_scale;
    float model_output_scale;
    float pow_exp;
    float nnue2score;
    float in_offset;
    float in_scaling;
    const float* wrm_table;   // target probability per score (win-rate model / BCE)
    int* block_counts;        // [blocks][kValCounts]
    double* block_loss;       // [blocks]
};

__device__ __forceinline__ float sigmoid_f(float x) {
    const float e = static_cast<float>(exp(static_cast<double>(-x)));
    return __fdiv_rn(1.0f, __fadd_rn(1.0f, e));
}

// |d| ^ p as the C library's powf gives it: d * d for p = 2 (correctly rounded
// there), otherwise pow in double rounded once.
__device__ __forceinline__ float abs_pow(float d, float p) {
    const float a = fabsf(d);
    if (p == 2.0f) return __fmul_rn(a, a);
    return static_cast<float>(pow(static_cast<double>(a), static_cast<double>(p)));
}

__device__ __forceinline__ float wrm_probability(float score, float offset, float scaling) {
    const float q = __fdiv_rn(__fsub_rn(score, offset), scaling);
    const float qm = __fdiv_rn(__fsub_rn(-score, offset), scaling);
    return __fmul_rn(0.5f, __fsub_rn(__fadd_rn(1.0f, sigmoid_f(q)), sigmoid_f(qm)));
}

__device__ __forceinline__ float bce_with_logits(float z, float t) {
    const float lin = z >= 0.0f ? __fmul_rn(__fsub_rn(1.0f, t), z) : __fmul_rn(-t, z);
    const float soft = static_cast<float>(log1p(exp(static_cast<double>(-fabsf(z)))));
    return __fadd_rn(lin, soft);
}

__global__ void __launch_bounds__(kValThreads) validation_block_kernel(ValArgs a) {
    __shared__ int counts[kValCounts];
    __shared__ double loss_s[kValThreads];
    if (threadIdx.x < kValCounts) counts[threadIdx.x] = 0;
    __syncthreads();
    const int i = blockIdx.x * kValThreads + threadIdx.x;
    int c[kValCounts] = {0, 0, 0, 0, 0, 0, 0, 0};
    double loss = 0.0;
    if (i < a.n) {
        const uint32_t w8 = a.records[static_cast<size_t>(i) * 10 + 8];
        const uint32_t w9 = a.records[static_cast<size_t>(i) * 10 + 9];
        const int s = static_cast<int16_t>(w8 & 0xffffu);
        const int r = static_cast<int8_t>((w9 >> 16) & 0xffu);
        const float m = a.outputs[i];
        const bool capped = a.score_drop_abs >= 0 && (s < 0 ? -s : s) >= a.score_drop_abs;
        if (capped) {
            c[6] = 1;
        } else {
            const bool draw = a.have_results ? r == 0 : s == 0;
            if (draw) {
                c[5] = 1;
            } else {
                c[0] = 1;
                const bool pred = m >= 0.0f;
                c[pred ? 2 : 3] = 1;
                c[4] = m == 0.0f;
                const bool truth = a.have_results ? r > 0 : s > 0;
                c[1] = pred == truth;
            }
            if (a.have_results) {
                c[7] = 1;
                const float blend = __fsub_rn(1.0f, a.lambda);
                const float inv_scale = a.eval_scale > 0.0f ? __fdiv_rn(1.0f, a.eval_scale) : 0.0025f;
                const float model_inv = a.model_output_scale > 0.0f ? __fdiv_rn(1.0f, a.model_output_scale) : 1.0f;
                const float result_norm = r > 0 ? 1.0f : (r < 0 ? 0.0f : 0.5f);
                const float sf = static_cast<float>(s);
                const float score_norm = a.loss_kind == 0 ? sigmoid_f(__fmul_rn(inv_scale, sf))
                                                          : __ldg(a.wrm_table + (s + 32768));
                const float target =
                    __fadd_rn(__fmul_rn(blend, result_norm), __fmul_rn(__fsub_rn(1.0f, blend), score_norm));
                float l;
                if (a.loss_kind == 2) {
                    l = bce_with_logits(__fdiv_rn(__fmul_rn(m, a.nnue2score), a.in_scaling), target);
                } else {
                    const float p = a.loss_kind == 0 ? sigmoid_f(__fmul_rn(m, model_inv))
                                                     : wrm_probability(__fmul_rn(m, a.nnue2score), a.in_offset,
                                                                       a.in_scaling);
                    l = abs_pow(__fsub_rn(p, target), a.pow_exp);
                }
                loss = static_cast<double>(l);
            }
        }
    }
#pragma unroll
    for (int k = 0; k < kValCounts; ++k) {
        const int total = __syncthreads_count(c[k] != 0);
        if (threadIdx.x == 0) counts[k] = total;
    }
    loss_s[threadIdx.x] = loss;
    __syncthreads();
    for (int stride = kValThreads / 2; stride > 0; stride >>= 1) {
        if (threadIdx.x < stride) loss_s[threadIdx.x] += loss_s[threadIdx.x + stride];
        __syncthreads();
    }
    if (threadIdx.x < kValCounts) a.block_counts[blockIdx.x * kValCounts + threadIdx.x] = counts[threadIdx.x];
    if (threadIdx.x == 0) a.block_loss[blockIdx.x] = loss_s[0];
}

// One warp: block partials summed in block order; report = 8 counts then the
// loss sum as a double (two ints).
__global__ void validation_final_kernel(const int* __restrict__ block_counts, const double* __restrict__ block_loss,
                                        int blocks, int* __restrict__ report) {
    if (threadIdx.x < kValCounts) {
        int s = 0;
        for (int b = 0; b < blocks; ++b) s += block_counts[b * kValCounts + threadIdx.x];
        report[threadIdx.x] = s;
    }
    if (threadIdx.x == 0) {
        double l = 0.0;
        for (int b = 0; b < blocks; ++b) l += block_loss[b];
        *reinterpret_cast<double*>(report + kValCounts) = l;
    }
}

// The reference's activation statistics, same partial layout: 5 metrics x 256
// CTA partials (FT outputs at 1, L2-input square and normal branches at 1, L2
// at 1, output squared).  Counts are exact in f32 below 2^24 per partial.
__global__ void __launch_bounds__(256) sfnn_validation_stats_kernel(const float* stm, const float* nstm,
                                                                    const float* l2_input, const float* l2,
                                                                    const float* output, float* partials,
                                                                    size_t batch, size_t ft, size_t hidden,
                                                                    size_t l2_size) {
    const int metric = blockIdx.y;
    const size_t n = metric == 0 ? batch * ft
                                 : (metric == 1 || metric == 2) ? batch * hidden : metric == 3 ? batch * l2_size : batch;
    float sum = 0.0f;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        if (metric == 0) {
            sum = __fadd_rn(sum, __fadd_rn(stm[i] >= 1.0f ? 1.0f : 0.0f, nstm[i] >= 1.0f ? 1.0f : 0.0f));
        } else if (metric == 1 || metric == 2) {
            const size_t j = (i / hidden) * (2 * hidden) + i % hidden + (metric == 1 ? hidden : 0);
            sum = __fadd_rn(sum, l2_input[j] >= 1.0f ? 1.0f : 0.0f);
        } else if (metric == 3) {
            sum = __fadd_rn(sum, l2[i] >= 1.0f ? 1.0f : 0.0f);
        } else {
            sum = __fmaf_rn(output[i], output[i], sum);   // the reference build contracts this to an FMA
        }
    }
    __shared__ float red[256];
    red[threadIdx.x] = sum;
    __syncthreads();
    for (int stride = 128; stride > 0; stride >>= 1) {
        if (threadIdx.x < stride) red[threadIdx.x] = __fadd_rn(red[threadIdx.x], red[threadIdx.x + stride]);
        __syncthreads();
    }
    if (threadIdx.x == 0) partials[metric * 256 + blockIdx.x] = red[0];
}

// Per-unit saturation counts: FT units (both views, 256-position tiles, one
// atomic per unit and tile) then per bucket: positions, the hidden units of
// the L2 input's normal and square branches and the L2 units at 1.  Integer
// counts: any order.
__global__ void unit_ft_stats_kernel(const float* stm, const float* nstm, int* counts, size_t batch, size_t ft) {
    const size_t unit = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (unit >= ft) return;
    int count = 0;
    const size_t end = min(batch, (static_cast<size_t>(blockIdx.y) + 1) * 256);
    for (size_t p = static_cast<size_t>(blockIdx.y) * 256; p < end; ++p)
        count += (stm[p * ft + unit] >= 1.0f) + (nstm[p * ft + unit] >= 1.0f);
    if (count) atomicAdd(counts + unit, count);
}

__global__ void unit_dense_stats_kernel(const float* input, const float* l2, const int* buckets, int* counts,
                                        size_t batch, size_t ft, size_t hidden, size_t width, size_t stacks) {
    const size_t p = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (p >= batch) return;
    const int b = buckets[p];
    if (b < 0 || static_cast<size_t>(b) >= stacks) return;
    int* row = counts + ft + static_cast<size_t>(b) * (1 + 2 * hidden + width);
    atomicAdd(row, 1);
    for (size_t u = 0; u < hidden; ++u) {  // normal branch first, then the square branch
        if (input[p * 2 * hidden + hidden + u] >= 1.0f) atomicAdd(row + 1 + u, 1);
        if (input[p * 2 * hidden + u] >= 1.0f) atomicAdd(row + 1 + hidden + u, 1);
    }
    for (size_t u = 0; u < width; ++u)
        if (l2[p * width + u] >= 1.0f) atomicAdd(row + 1 + 2 * hidden + u, 1);
}

}  // namespace
}  // namespace bou

using namespace bou;

extern "C" {

int bulletou_b200_validation_metrics_device(BulletOuCudaCppContext* ctx, const BulletOuB200ValidationConfig* config,
                                            const BulletOuCudaCppF32Buffer* outputs,
                                            const BulletOuCudaCppI32Buffer* records, size_t n,
                                            const BulletOuCudaCppF32Buffer* wrm_table,
                                            BulletOuCudaCppI32Buffer* report) {
    if (config == nullptr) return fail_message("validation config must not be null");
    const BulletOuB200ValidationConfig& c = *config;
    if (c.loss_kind < 0 || c.loss_kind > 2) return fail_messagef("validation loss kind %d is not supported", c.loss_kind);
    if (n > static_cast<size_t>(INT32_MAX) / 16) return fail_message("validation: too many positions");
    if (validate_f32(ctx, outputs, n, "validation outputs") != 0 ||
        validate_i32(ctx, records, n * 10, "validation records") != 0 ||
        validate_i32(ctx, report, kValCounts + 2, "validation report") != 0)
        return -1;
    if (c.loss_kind != 0 && c.have_results &&
        (wrm_table == nullptr || validate_f32(ctx, wrm_table, 65536, "validation target table") != 0))
        return wrm_table == nullptr ? fail_message("win-rate-model / BCE validation needs the target table") : -1;
    if (set_device(ctx) != 0) return -1;
    const int blocks = static_cast<int>(std::max<size_t>(1, (n + kValThreads - 1) / kValThreads));
    void* sp = nullptr;
    const size_t bytes = static_cast<size_t>(blocks) * (kValCounts * sizeof(int) + sizeof(double)) + 16;
    if (scratch_slot(ctx, kScratchValidation, bytes, &sp, "cudaMalloc validation partials") != 0) return -1;
    ValArgs a{};
    a.outputs = outputs->ptr;
    a.records = reinterpret_cast<const uint32_t*>(records->ptr);
    a.n = static_cast<int>(n);
    a.have_results = c.have_results;
    a.score_drop_abs = c.score_drop_abs;
    a.loss_kind = c.loss_kind;
    a.lambda = c.lambda;
    a.eval_scale = c.eval_scale;
    a.model_output_scale = c.model_output_scale;
    a.pow_exp = c.pow_exp;
    a.nnue2score = c.nnue2score;
    a.in_offset = c.in_offset;
    a.in_scaling = c.in_scaling;
    a.wrm_table = wrm_table != nullptr ? wrm_table->ptr : nullptr;
    a.block_loss = static_cast<double*>(sp);
    a.block_counts = reinterpret_cast<int*>(a.block_loss + blocks);
    validation_block_kernel<<<blocks, kValThreads, 0, ctx->stream>>>(a);
    if (check_launch("validation metrics launch") != 0) return -1;
    validation_final_kernel<<<1, 32, 0, ctx->stream>>>(a.block_counts, a.block_loss, blocks, report->ptr);
    if (check_launch("validation metrics final launch") != 0) return -1;
    return ok();
}

int bulletou_cuda_cpp_sfnn_validation_stats(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* stm,
                                            BulletOuCudaCppF32Buffer* nstm, BulletOuCudaCppF32Buffer* l2_input,
                                            BulletOuCudaCppF32Buffer* l2, BulletOuCudaCppF32Buffer* output,
                                            BulletOuCudaCppF32Buffer* partials, size_t batch, size_t ft,
                                            size_t hidden, size_t l2_size) {
    if (set_device(ctx) != 0) return -1;
    if (batch == 0 || ft == 0 || hidden == 0 || l2_size == 0 || ft > SIZE_MAX / batch ||
        hidden > SIZE_MAX / batch / 2 || l2_size > SIZE_MAX / batch)
        return fail_message("invalid SFNN validation stats dimensions");
    if (validate_f32(ctx, stm, batch * ft, "stats stm") != 0 || validate_f32(ctx, nstm, batch * ft, "stats nstm") != 0 ||
        validate_f32(ctx, l2_input, batch * hidden * 2, "stats l2 input") != 0 ||
        validate_f32(ctx, l2, batch * l2_size, "stats l2") != 0 ||
        validate_f32(ctx, output, batch, "stats output") != 0 ||
        validate_f32(ctx, partials, 5 * 256, "stats partials") != 0)
        return -1;
    sfnn_validation_stats_kernel<<<dim3(256, 5), 256, 0, ctx->stream>>>(stm->ptr, nstm->ptr, l2_input->ptr, l2->ptr,
                                                                       output->ptr, partials->ptr, batch, ft, hidden,
                                                                       l2_size);
    return check_launch("SFNN validation stats launch") != 0 ? -1 : ok();
}

int bulletou_cuda_cpp_sfnn_unit_stats(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* stm,
                                      BulletOuCudaCppF32Buffer* nstm, BulletOuCudaCppF32Buffer* input,
                                      BulletOuCudaCppF32Buffer* l2, BulletOuCudaCppI32Buffer* buckets,
                                      BulletOuCudaCppI32Buffer* counts, size_t batch, size_t ft, size_t hidden,
                                      size_t width, size_t stacks) {
    if (set_device(ctx) != 0) return -1;
    if (!batch || batch > 1048576 || !ft || !hidden || !width || !stacks || ft > SIZE_MAX / batch ||
        hidden > SIZE_MAX / batch / 2 || width > SIZE_MAX / batch || hidden > (SIZE_MAX - 1 - width) / 2)
        return fail_message("invalid unit stats dimensions");
    const size_t stride = 1 + 2 * hidden + width;
    if (stacks > (SIZE_MAX / sizeof(int) - ft) / stride) return fail_message("unit stats size overflow");
    const size_t len = ft + stacks * stride;
    if (validate_f32(ctx, stm, batch * ft, "unit stats stm") != 0 ||
        validate_f32(ctx, nstm, batch * ft, "unit stats nstm") != 0 ||
        validate_f32(ctx, input, batch * 2 * hidden, "unit stats input") != 0 ||
        validate_f32(ctx, l2, batch * width, "unit stats l2") != 0 ||
        validate_i32(ctx, buckets, batch, "unit stats buckets") != 0 ||
        validate_i32(ctx, counts, len, "unit stats counts") != 0)
        return -1;
    cudaError_t st = cudaMemsetAsync(counts->ptr, 0, len * sizeof(int), ctx->stream);
    if (st != cudaSuccess) return fail("clear unit stats", st);
    unit_ft_stats_kernel<<<dim3(static_cast<unsigned>((ft + 255) / 256), static_cast<unsigned>((batch + 255) / 256)),
                           256, 0, ctx->stream>>>(stm->ptr, nstm->ptr, counts->ptr, batch, ft);
    if (check_launch("unit FT stats launch") != 0) return -1;
    unit_dense_stats_kernel<<<static_cast<unsigned>((batch + 255) / 256), 256, 0, ctx->stream>>>(
        input->ptr, l2->ptr, buckets->ptr, counts->ptr, batch, ft, hidden, width, stacks);
    return check_launch("unit dense stats launch") != 0 ? -1 : ok();
}

}  // extern "C"
