// The rest of the reference backend's C ABI (crates/cuda_cpp/src/lib.rs
// `mod ffi` and the extern blocks of batch_norm.rs, bn_qat.rs, layer_qat.rs):
// entries a Rust build of crates/cuda_cpp references, so that it links against
// this library unchanged.
//
//   * implemented: the per-bucket ("dirty") Ranger step over a stacked group
//     (cu:10700-10862), the FP16 option switches in their "off" position
//     (cu:9598-9665), row / bucket scaling utilities (cu:10245, 13411-13470,
//     13993);
//   * unsupported on this backend (return -1 with a message naming the entry):
//     FP16 optimizer moments, BatchNorm and its QAT, centering experiments, the
//     FT saturation guard, effective-L1 clipping, bucket-axis factorizer updates,
//     the shared-factor rebase, the saturation penalty, and the reference's
//     single-kernel test hooks.
#include <cfloat>
#include <cstdint>

#include "common.cuh"
#include "optim.cuh"

namespace bou {
int apply_norm_loss(BulletOuCudaCppContext* ctx, float* w, size_t n, float rate);
}  // namespace bou

using namespace bou;

namespace {

constexpr int kThreads = 256;

int unsupported(const char* name) { return fail_messagef("unsupported on this backend: %s", name); }

// One thread per (dirty bucket, column of its stride): RAdam step, gradient
// reset and -- on lookahead steps -- the slow-weight blend, in one pass.
// Arithmetic of radam_update_reset_gradients_stacked_dirty_kernel +
// ranger_lookahead_stacked_dirty_kernel (cu:729-1000).
__global__ void stacked_dirty_ranger_kernel(const int* __restrict__ dirty, size_t dirty_count, size_t stride,
                                            size_t len, float* __restrict__ g, float* __restrict__ w,
                                            float* __restrict__ m, float* __restrict__ v, float* __restrict__ slow,
                                            RangerArgs a, int step, int lookahead) {
    const size_t t = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= dirty_count * stride) return;
    const size_t k = t / stride;
    const int bucket = dirty[k];
    if (bucket < 0) return;
    const size_t i = static_cast<size_t>(bucket) * stride + (t - k * stride);
    if (i >= len) return;
    float wi = w[i];
    if (step) {
        float mi = m[i], vi = v[i];
        radam_coordinate(a.gradient_factor * g[i], a, wi, mi, vi);
        g[i] = 0.0f;
        m[i] = mi;
        v[i] = vi;
    }
    if (lookahead) {
        wi = lookahead_coordinate(wi, slow[i], a);
        slow[i] = wi;
    }
    w[i] = wi;
}

__global__ void clear_dirty_kernel(const int* __restrict__ dirty, size_t dirty_count, size_t stride, size_t len,
                                   float* __restrict__ g) {
    const size_t t = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= dirty_count * stride) return;
    const size_t k = t / stride;
    const int bucket = dirty[k];
    if (bucket < 0) return;
    const size_t i = static_cast<size_t>(bucket) * stride + (t - k * stride);
    if (i < len) g[i] = 0.0f;
}

__global__ void scale_rows_kernel(float* __restrict__ values, size_t len, size_t row_len,
                                  const float* __restrict__ scales) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < len) values[i] *= scales[i / row_len];
}

// mode 0: gradients += 2 * decay[s] * weights (atomic, as repeated buckets add
// twice); mode 1: gradients *= gates[s].  Buckets past num_stacks are skipped.
__global__ void bucket_rows_kernel(const float* __restrict__ weights, float* __restrict__ gradients,
                                   const float* __restrict__ coeff, const int* __restrict__ dirty, size_t dirty_count,
                                   size_t stride, size_t num_stacks, int mode) {
    const size_t n = dirty_count == 0 ? num_stacks : dirty_count;
    const size_t t = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= n * stride) return;
    const size_t k = t / stride;
    const size_t s = dirty_count == 0 ? k : static_cast<size_t>(dirty[k]);
    if (s >= num_stacks) return;
    const float c = coeff[s];
    const size_t i = s * stride + (t - k * stride);
    if (mode == 0) {
        if (c != 0.0f) atomicAdd(gradients + i, 2.0f * c * weights[i]);
    } else if (c != 1.0f) {
        gradients[i] *= c;
    }
}

__global__ void scale_copy_kernel(const float* __restrict__ src, float* __restrict__ dst, size_t n, float scale) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) dst[i] = src[i] * scale;
}

int check_bucket_rows(BulletOuCudaCppContext* ctx, size_t stride, size_t num_stacks, size_t dirty_count,
                      const BulletOuCudaCppI32Buffer* dirty, const char* what) {
    if (stride == 0 || num_stacks == 0) return fail_messagef("%s dimensions must be non-zero", what);
    if (num_stacks > SIZE_MAX / stride) return fail_messagef("%s length overflow", what);
    if (dirty_count != 0 && validate_i32(ctx, dirty, dirty_count, "dirty_buckets") != 0) return -1;
    return 0;
}

}  // namespace

extern "C" {

// ------------------------------------------------------------------ FP16 options
int bulletou_cuda_cpp_context_set_sfnn_ft_fp16(BulletOuCudaCppContext* ctx, int enabled) {
    if (validate_context(ctx) != 0) return -1;
    return enabled ? unsupported("FP16 FT weights (bulletou_cuda_cpp_context_set_sfnn_ft_fp16)") : ok();
}

int bulletou_cuda_cpp_context_set_sfnn_ft_fp16_grad(BulletOuCudaCppContext* ctx, int enabled) {
    if (validate_context(ctx) != 0) return -1;
    return enabled ? unsupported("FP16 FT gradients (bulletou_cuda_cpp_context_set_sfnn_ft_fp16_grad)") : ok();
}

int bulletou_cuda_cpp_context_set_sfnn_ft_fp16_act(BulletOuCudaCppContext* ctx, int enabled) {
    if (validate_context(ctx) != 0) return -1;
    return enabled ? unsupported("FP16 FT activations (bulletou_cuda_cpp_context_set_sfnn_ft_fp16_act)") : ok();
}

int bulletou_cuda_cpp_context_release_sfnn_ft_fp16_scratch(BulletOuCudaCppContext* ctx, int, int, int) {
    if (validate_context(ctx) != 0) return -1;
    return ok();  // no FP16 scratch exists
}

int bulletou_cuda_cpp_context_take_ft_half_grad_clipped(BulletOuCudaCppContext* ctx, unsigned long long* out) {
    if (ctx == nullptr || out == nullptr) return fail_message("null FT FP16 gradient counter argument");
    *out = 0;
    return ok();
}

int bulletou_test_sfnn_ft_fp16_scratch_sizes(BulletOuCudaCppContext* ctx, size_t* weights, size_t* gradients,
                                             size_t* activations) {
    if (ctx == nullptr || weights == nullptr || gradients == nullptr || activations == nullptr) return -1;
    *weights = *gradients = *activations = 0;
    return 0;
}

// ------------------------------------------------------------------ FP16 moments
int bulletou_cuda_cpp_ft_half_moments_create(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer*,
                                             BulletOuCudaCppF32Buffer*, size_t, int,
                                             BulletOuCudaCppHalfMoments** out) {
    if (out != nullptr) *out = nullptr;
    if (validate_context(ctx) != 0) return -1;
    return unsupported("FP16 optimizer moments (bulletou_cuda_cpp_ft_half_moments_create)");
}

int bulletou_cuda_cpp_ft_half_moments_decode(BulletOuCudaCppContext*, BulletOuCudaCppHalfMoments*,
                                             BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*) {
    return unsupported("FP16 optimizer moments (bulletou_cuda_cpp_ft_half_moments_decode)");
}

int bulletou_cuda_cpp_ft_half_moments_take_clipped(BulletOuCudaCppContext*, BulletOuCudaCppHalfMoments*,
                                                   unsigned long long* out) {
    if (out != nullptr) *out = 0;
    return unsupported("FP16 optimizer moments (bulletou_cuda_cpp_ft_half_moments_take_clipped)");
}

int bulletou_cuda_cpp_ft_half_moments_destroy(BulletOuCudaCppHalfMoments* state) {
    return state == nullptr ? 0 : unsupported("FP16 optimizer moments (bulletou_cuda_cpp_ft_half_moments_destroy)");
}

// ------------------------------------------------------------------ stacked dirty Ranger
int bulletou_cuda_cpp_ranger_update_stacked_dirty_device(
    BulletOuCudaCppContext* ctx, float norm_loss_rate, int norm_loss_before, size_t len, size_t stride,
    size_t dirty_count, float gradient_factor, float learning_rate, float step_size, int use_denom, float decay,
    float beta1, float beta2, float epsilon, float min_weight, float max_weight, int do_lookahead,
    float lookahead_alpha, int clip_after_lookahead, const BulletOuCudaCppI32Buffer* dirty_buckets,
    BulletOuCudaCppF32Buffer* gradients, BulletOuCudaCppF32Buffer* weights, BulletOuCudaCppF32Buffer* momentum,
    BulletOuCudaCppF32Buffer* velocity, BulletOuCudaCppF32Buffer* slow_params) {
    if (validate_i32(ctx, dirty_buckets, dirty_count, "dirty_buckets") != 0 ||
        validate_f32(ctx, gradients, len, "gradients") != 0 || validate_f32(ctx, weights, len, "weights") != 0 ||
        validate_f32(ctx, momentum, len, "momentum") != 0 || validate_f32(ctx, velocity, len, "velocity") != 0 ||
        validate_f32(ctx, slow_params, len, "slow_params") != 0)
        return -1;
    if (set_device(ctx) != 0) return -1;
    if (len == 0 || stride == 0 || dirty_count == 0) return ok();
    if (dirty_count > SIZE_MAX / stride) return fail_message("ranger dirty stacked update length overflow");
    int blocks = 0;
    if (grid_1d(dirty_count * stride, kThreads, &blocks, "stacked dirty Ranger") != 0) return -1;
    if (learning_rate == 0.0f) {
        clear_dirty_kernel<<<blocks, kThreads, 0, ctx->stream>>>(dirty_buckets->ptr, dirty_count, stride, len,
                                                                 gradients->ptr);
        return check_launch("stacked dirty gradient clear");
    }
    const BulletOuB200RangerStep s{norm_loss_rate, norm_loss_before, gradient_factor, learning_rate, step_size,
                                   use_denom, decay, beta1, beta2, epsilon, min_weight, max_weight, do_lookahead,
                                   lookahead_alpha, clip_after_lookahead};
    const RangerArgs a = ranger_args_from(s);
    if (norm_loss_before && apply_norm_loss(ctx, weights->ptr, len, norm_loss_rate) != 0) return -1;
    // Norm loss after the step comes before the lookahead (reference order), so
    // the lookahead then runs as its own pass.
    const bool split = !norm_loss_before && norm_loss_rate != 0.0f;
    stacked_dirty_ranger_kernel<<<blocks, kThreads, 0, ctx->stream>>>(
        dirty_buckets->ptr, dirty_count, stride, len, gradients->ptr, weights->ptr, momentum->ptr, velocity->ptr,
        slow_params->ptr, a, 1, do_lookahead && !split ? 1 : 0);
    if (check_launch("stacked dirty Ranger") != 0) return -1;
    if (split) {
        if (apply_norm_loss(ctx, weights->ptr, len, norm_loss_rate) != 0) return -1;
        if (do_lookahead) {
            stacked_dirty_ranger_kernel<<<blocks, kThreads, 0, ctx->stream>>>(
                dirty_buckets->ptr, dirty_count, stride, len, gradients->ptr, weights->ptr, momentum->ptr,
                velocity->ptr, slow_params->ptr, a, 0, 1);
            if (check_launch("stacked dirty lookahead") != 0) return -1;
        }
    }
    return ok();
}

// ------------------------------------------------------------------ row / bucket utilities
int bulletou_cuda_cpp_scale_axis_rows_f32_device(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* values,
                                                 size_t value_len, const BulletOuCudaCppF32Buffer* row_scales,
                                                 size_t row_count, size_t row_len) {
    if (row_len == 0) return fail_message("scale_axis_rows row_len must be greater than zero");
    if (row_count != 0 && row_len > SIZE_MAX / row_count)
        return fail_message("scale_axis_rows row_count * row_len overflow");
    if (value_len != row_count * row_len)
        return fail_message("scale_axis_rows value length does not match row_count * row_len");
    if (validate_f32(ctx, values, value_len, "values") != 0 ||
        validate_f32(ctx, row_scales, row_count, "row_scales") != 0 || set_device(ctx) != 0)
        return -1;
    if (value_len == 0) return ok();
    int blocks = 0;
    if (grid_1d(value_len, kThreads, &blocks, "scale_axis_rows") != 0) return -1;
    scale_rows_kernel<<<blocks, kThreads, 0, ctx->stream>>>(values->ptr, value_len, row_len, row_scales->ptr);
    return check_launch("scale_axis_rows launch");
}

int bulletou_cuda_cpp_sfnn_add_residual_count_decay_gradients_device(
    BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* weights, BulletOuCudaCppF32Buffer* gradients,
    BulletOuCudaCppF32Buffer* decay_by_stack, BulletOuCudaCppI32Buffer* dirty_buckets, size_t dirty_count,
    size_t stride, size_t num_stacks) {
    if (set_device(ctx) != 0 ||
        check_bucket_rows(ctx, stride, num_stacks, dirty_count, dirty_buckets, "sfnn residual count decay") != 0)
        return -1;
    const size_t total = num_stacks * stride;
    if (validate_f32(ctx, weights, total, "sfnn residual count decay weights") != 0 ||
        validate_f32(ctx, gradients, total, "sfnn residual count decay gradients") != 0 ||
        validate_f32(ctx, decay_by_stack, num_stacks, "sfnn residual count decay by-stack coefficients") != 0)
        return -1;
    const size_t n = (dirty_count == 0 ? num_stacks : dirty_count) * stride;
    int blocks = 0;
    if (grid_1d(n, kThreads, &blocks, "sfnn residual count decay") != 0) return -1;
    bucket_rows_kernel<<<blocks, kThreads, 0, ctx->stream>>>(weights->ptr, gradients->ptr, decay_by_stack->ptr,
                                                             dirty_count ? dirty_buckets->ptr : nullptr, dirty_count,
                                                             stride, num_stacks, 0);
    return check_launch("sfnn residual count decay gradients");
}

int bulletou_cuda_cpp_sfnn_apply_residual_count_gates_to_gradients_device(
    BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* gradients, const BulletOuCudaCppF32Buffer* gates,
    const BulletOuCudaCppI32Buffer* dirty_buckets, size_t dirty_count, size_t stride, size_t num_stacks) {
    if (check_bucket_rows(ctx, stride, num_stacks, dirty_count, dirty_buckets, "sfnn residual count gate") != 0 ||
        validate_f32(ctx, gradients, num_stacks * stride, "sfnn residual count gate gradients") != 0 ||
        validate_f32(ctx, gates, num_stacks, "sfnn residual count gates") != 0 || set_device(ctx) != 0)
        return -1;
    const size_t n = (dirty_count == 0 ? num_stacks : dirty_count) * stride;
    int blocks = 0;
    if (grid_1d(n, kThreads, &blocks, "sfnn residual count gates") != 0) return -1;
    bucket_rows_kernel<<<blocks, kThreads, 0, ctx->stream>>>(nullptr, gradients->ptr, gates->ptr,
                                                             dirty_count ? dirty_buckets->ptr : nullptr, dirty_count,
                                                             stride, num_stacks, 1);
    return check_launch("sfnn residual count gates");
}

int bulletou_center_scale(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* src, BulletOuCudaCppF32Buffer* dst,
                          size_t n, float scale) {
    if (n == 0 || !(scale >= -FLT_MAX && scale <= FLT_MAX) || validate_f32(ctx, src, n, "center src") != 0 ||
        validate_f32(ctx, dst, n, "center dst") != 0 || set_device(ctx) != 0)
        return -1;
    int blocks = 0;
    if (grid_1d(n, kThreads, &blocks, "center scale") != 0) return -1;
    scale_copy_kernel<<<blocks, kThreads, 0, ctx->stream>>>(src->ptr, dst->ptr, n, scale);
    return check_launch("center scale/copy");
}

int bulletou_test_stream_delay(BulletOuCudaCppContext* ctx) { return validate_context(ctx) != 0 ? -1 : 0; }

void bulletou_bn_reference_mode(int) {}

// ------------------------------------------------------------------ unsupported research features
int bulletou_bn_bind(BulletOuCudaCppContext*, int, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*,
    BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*,
    size_t, size_t, size_t, size_t, float, float, int) {
    return unsupported("bulletou_bn_bind");  // batch_norm.cuh:365
}
int bulletou_bn_forward(BulletOuCudaCppContext*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*,
    BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppI32Buffer*, BulletOuCudaCppF32Buffer*,
    BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, size_t, size_t, size_t, size_t, float, float, int) {
    return unsupported("bulletou_bn_forward");  // batch_norm.cuh:294
}
int bulletou_bn_backward(BulletOuCudaCppContext*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*,
    BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppI32Buffer*, BulletOuCudaCppF32Buffer*,
    BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, size_t, size_t, size_t, size_t) {
    return unsupported("bulletou_bn_backward");  // batch_norm.cuh:316
}
int bulletou_bn_qat_project_l2(BulletOuCudaCppContext*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*,
    size_t, size_t) {
    return unsupported("bulletou_bn_qat_project_l2");  // bn_qat.cuh:20
}
int bulletou_bn_qat_unfold_training(BulletOuCudaCppContext*, BulletOuCudaCppF32Buffer*,
    BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*,
    BulletOuCudaCppF32Buffer*, size_t, size_t, size_t, int, size_t, float) {
    return unsupported("bulletou_bn_qat_unfold_training");  // bn_qat.cuh:78
}
int bulletou_bn_qat_ft(BulletOuCudaCppContext*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, size_t,
    size_t, size_t, float) {
    return unsupported("bulletou_bn_qat_ft");  // bn_qat.cuh:162
}
int bulletou_bn_qat_ft_training(BulletOuCudaCppContext*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*,
    BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, size_t, size_t, size_t, float) {
    return unsupported("bulletou_bn_qat_ft_training");  // bn_qat.cuh:169
}
int bulletou_bn_qat_pullback(BulletOuCudaCppContext*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*,
    BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*,
    BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, size_t, size_t, size_t, int, size_t, float) {
    return unsupported("bulletou_bn_qat_pullback");  // bn_qat.cuh:178
}
int bulletou_center_l1_groups(BulletOuCudaCppContext*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*,
    BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*,
    BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*,
    BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, size_t, int) {
    return unsupported("bulletou_center_l1_groups");  // cu:13936
}
int bulletou_center_affine_layout(BulletOuCudaCppContext*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*,
    BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*,
    BulletOuCudaCppF32Buffer*, size_t, size_t, int, int) {
    return unsupported("bulletou_center_affine_layout");  // cu:13974
}
int bulletou_center_mean_reference(BulletOuCudaCppContext*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*,
    size_t, size_t) {
    return unsupported("bulletou_center_mean_reference");  // cu:14013
}
int bulletou_experiment_center_affine(BulletOuCudaCppContext*, BulletOuCudaCppF32Buffer*,
    BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*,
    BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, size_t, size_t, int) {
    return unsupported("bulletou_experiment_center_affine");  // cu:13959
}
int bulletou_experiment_column_mean(BulletOuCudaCppContext*, BulletOuCudaCppF32Buffer*,
    BulletOuCudaCppF32Buffer*, size_t, size_t) {
    return unsupported("bulletou_experiment_column_mean");  // cu:14001
}
int bulletou_experiment_bucket_mean(BulletOuCudaCppContext*, BulletOuCudaCppF32Buffer*,
    BulletOuCudaCppI32Buffer*, BulletOuCudaCppF32Buffer*, size_t, size_t, size_t) {
    return unsupported("bulletou_experiment_bucket_mean");  // cu:14043
}
int bulletou_experiment_bucket_centers(BulletOuCudaCppContext*, BulletOuCudaCppF32Buffer*,
    BulletOuCudaCppF32Buffer*, size_t, size_t) {
    return unsupported("bulletou_experiment_bucket_centers");  // cu:14055
}
int bulletou_experiment_center_affine_bucket(BulletOuCudaCppContext*, BulletOuCudaCppF32Buffer*,
    BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*,
    BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, size_t, size_t, size_t, int) {
    return unsupported("bulletou_experiment_center_affine_bucket");  // cu:14062
}
int bulletou_experiment_mean_penalty_test(BulletOuCudaCppContext*, BulletOuCudaCppF32Buffer*,
    BulletOuCudaCppI32Buffer*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, size_t, size_t, size_t,
    size_t, float) {
    return unsupported("bulletou_experiment_mean_penalty_test");  // cu:14075
}
int bulletou_bind_ft_saturation_guard(BulletOuCudaCppContext*, BulletOuCudaCppF32Buffer*,
    BulletOuCudaCppI32Buffer*, BulletOuCudaCppI32Buffer*, size_t, size_t, float, float, int) {
    return unsupported("bulletou_bind_ft_saturation_guard");  // cu:13764
}
int bulletou_ft_saturation_guard(BulletOuCudaCppContext*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*,
    BulletOuCudaCppF32Buffer*, BulletOuCudaCppI32Buffer*, BulletOuCudaCppI32Buffer*, BulletOuCudaCppI32Buffer*,
    BulletOuCudaCppI32Buffer*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, size_t, size_t, size_t,
    size_t, float, float, float, int) {
    return unsupported("bulletou_ft_saturation_guard");  // cu:13780
}
int bulletou_clip_effective_l1(BulletOuCudaCppContext*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*,
    BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, size_t, size_t, float) {
    return unsupported("bulletou_clip_effective_l1");  // cu:13831
}
int bulletou_clip_effective_l1_axis(BulletOuCudaCppContext*, BulletOuCudaCppF32Buffer*,
    BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*,
    BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, size_t, size_t, size_t, size_t, size_t, int, int, int,
    int, int, int, float, float, float, float, float) {
    return unsupported("bulletou_clip_effective_l1_axis");  // cu:13880
}
int bulletou_factor_axis_update_device(BulletOuCudaCppContext*, size_t, size_t, size_t, size_t, size_t, float,
    float, float, float, BulletOuCudaCppF32Buffer*, float, float, float, float, float, float, float, int, int,
    float, float, float, int, int, float, int, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*,
    BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*) {
    return unsupported("bulletou_factor_axis_update_device");  // cu:10522
}
int bulletou_cuda_cpp_rebase_shared_device(BulletOuCudaCppContext*, BulletOuCudaCppF32Buffer*,
    BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*,
    BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*,
    size_t, size_t, size_t, size_t, size_t, float, float) {
    return unsupported("bulletou_cuda_cpp_rebase_shared_device");  // cu:13609
}
int bulletou_cuda_cpp_sfnn_add_saturation_penalty_gradients_device(BulletOuCudaCppContext*,
    BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, int, BulletOuCudaCppF32Buffer*, int,
    BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppI32Buffer*,
    size_t, size_t, size_t, size_t, size_t, size_t, int, int, int, int, int, int, float, float, float, float,
    float, float, const BulletOuCudaCppF32Buffer*, const BulletOuCudaCppF32Buffer*, int, float, float, float) {
    return unsupported("bulletou_cuda_cpp_sfnn_add_saturation_penalty_gradients_device");  // cu:13277
}

// ------------------------------------------------------------------ the reference's kernel test hooks
int bulletou_test_dense_l1_16(BulletOuCudaCppContext*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*,
    BulletOuCudaCppF32Buffer*, BulletOuCudaCppI32Buffer*, BulletOuCudaCppF32Buffer*, size_t, size_t, size_t,
    int) {
    return unsupported("bulletou_test_dense_l1_16");  // cu:4595
}
int bulletou_test_factorized_ft_half_fold(BulletOuCudaCppContext*, BulletOuCudaCppF32Buffer*,
    BulletOuCudaCppF32Buffer*, size_t, size_t, float, int) {
    return unsupported("bulletou_test_factorized_ft_half_fold");  // cu:4620
}
int bulletou_test_sfnn_ft_sort(BulletOuCudaCppContext*, BulletOuCudaCppI32Buffer*, BulletOuCudaCppI32Buffer*,
    BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*,
    BulletOuCudaCppF32Buffer*, BulletOuCudaCppI32Buffer*, BulletOuCudaCppI32Buffer*, size_t, size_t, size_t,
    size_t, int) {
    return unsupported("bulletou_test_sfnn_ft_sort");  // cu:4647
}
int bulletou_test_sfnn_ft_gather(BulletOuCudaCppContext*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppI32Buffer*,
    BulletOuCudaCppI32Buffer*, BulletOuCudaCppF32Buffer*, size_t, size_t, int, int) {
    return unsupported("bulletou_test_sfnn_ft_gather");  // cu:4762
}
int bulletou_test_sfnn_half_grad_gather(BulletOuCudaCppContext*, BulletOuCudaCppF32Buffer*,
    BulletOuCudaCppI32Buffer*, BulletOuCudaCppI32Buffer*, BulletOuCudaCppF32Buffer*, size_t, size_t, size_t,
    size_t, int) {
    return unsupported("bulletou_test_sfnn_half_grad_gather");  // cu:4838
}
int bulletou_test_sfnn_half_grad(BulletOuCudaCppContext*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*,
    BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*,
    size_t, size_t, int) {
    return unsupported("bulletou_test_sfnn_half_grad");  // cu:4866
}
int bulletou_test_l1_bucket_fold(BulletOuCudaCppContext*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*,
    BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*,
    BulletOuCudaCppI32Buffer*, int) {
    return unsupported("bulletou_test_l1_bucket_fold");  // cu:5646
}
int bulletou_test_qat_ft_lattice(BulletOuCudaCppContext*, BulletOuCudaCppF32Buffer*, size_t, int) {
    return unsupported("bulletou_test_qat_ft_lattice");  // cu:6013
}
int bulletou_test_qat_packed_l1(BulletOuCudaCppContext*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*,
    BulletOuCudaCppI32Buffer*, BulletOuCudaCppI32Buffer*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppI32Buffer*,
    size_t, size_t, size_t, size_t, int) {
    return unsupported("bulletou_test_qat_packed_l1");  // cu:6247
}
int bulletou_test_dense_qat_exact_ft(BulletOuCudaCppContext*, BulletOuCudaCppI32Buffer*,
    BulletOuCudaCppI32Buffer*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*,
    BulletOuCudaCppI32Buffer*, size_t, size_t, size_t, size_t) {
    return unsupported("bulletou_test_dense_qat_exact_ft");  // cu:6384
}
int bulletou_test_l1_to_ft_f32_gradient(BulletOuCudaCppContext*, BulletOuCudaCppF32Buffer*,
    BulletOuCudaCppF32Buffer*, BulletOuCudaCppI32Buffer*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*,
    BulletOuCudaCppF32Buffer*, size_t, size_t, size_t, int) {
    return unsupported("bulletou_test_l1_to_ft_f32_gradient");  // cu:7123
}
int bulletou_test_l1_to_ft_half_gradient(BulletOuCudaCppContext*, BulletOuCudaCppF32Buffer*,
    BulletOuCudaCppF32Buffer*, BulletOuCudaCppI32Buffer*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*,
    BulletOuCudaCppF32Buffer*, size_t, size_t, size_t, int) {
    return unsupported("bulletou_test_l1_to_ft_half_gradient");  // cu:7152
}
int bulletou_test_l1_gather2(BulletOuCudaCppContext*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*,
    BulletOuCudaCppI32Buffer*, BulletOuCudaCppI32Buffer*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*,
    BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, size_t, size_t, size_t, size_t, float) {
    return unsupported("bulletou_test_l1_gather2");  // cu:7314
}
int bulletou_test_l1_gather2_king_progress(BulletOuCudaCppContext*, BulletOuCudaCppF32Buffer*,
    BulletOuCudaCppF32Buffer*, BulletOuCudaCppI32Buffer*, BulletOuCudaCppI32Buffer*, BulletOuCudaCppF32Buffer*,
    BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*,
    BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, size_t, size_t, size_t, size_t, size_t, float, float,
    float, float) {
    return unsupported("bulletou_test_l1_gather2_king_progress");  // cu:7338
}
int bulletou_dense_qat_integer_reference(BulletOuCudaCppContext*, BulletOuCudaCppI32Buffer*,
    BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppI32Buffer*, BulletOuCudaCppI32Buffer*,
    size_t, size_t, size_t, size_t) {
    return unsupported("bulletou_dense_qat_integer_reference");  // cu:9336
}
int bulletou_dense_qat_activation_reference(BulletOuCudaCppContext*, BulletOuCudaCppI32Buffer*,
    BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppI32Buffer*, BulletOuCudaCppI32Buffer*,
    BulletOuCudaCppF32Buffer*, size_t) {
    return unsupported("bulletou_dense_qat_activation_reference");  // cu:9403
}
int bulletou_dense_qat_l1_backward_reference(BulletOuCudaCppContext*, BulletOuCudaCppF32Buffer*,
    BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, BulletOuCudaCppF32Buffer*, size_t, size_t, int) {
    return unsupported("bulletou_dense_qat_l1_backward_reference");  // cu:9422
}

}  // extern "C"
