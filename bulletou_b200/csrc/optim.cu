// Standalone optimizer entries of the drop-in ABI:
//   bulletou_cuda_cpp_ranger_update_device  (reference cu:10576)
//   bulletou_cuda_cpp_ranger_update_host    (reference cu:14087)
//   bulletou_cuda_cpp_sgd_momentum_update_device (reference cu:10554)
// One fused kernel per call: the RAdam step, the gradient reset and (on
// lookahead steps) the slow-weight interpolation happen in a single pass over
// the parameter group instead of two.
#include <cmath>
#include <cstring>

#include "common.cuh"
#include "optim.cuh"

using namespace bou;

namespace bou {

namespace {

constexpr int kThreads = 256;

// Vectorised Ranger pass over a contiguous parameter range (len4 float4s).
template <bool kLookahead>
__global__ void ranger_vec4_kernel(float4* __restrict__ gradients, float4* __restrict__ weights,
                                   float4* __restrict__ momentum, float4* __restrict__ velocity,
                                   float4* __restrict__ slow, size_t len4, RangerArgs a, bool skip_quiet) {
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < len4; i += stride) {
        const float4 g4 = gradients[i];
        float4 w4 = weights[i];
        float4 m4 = momentum[i];
        float4 v4 = velocity[i];
        if (skip_quiet && !kLookahead) {
            const unsigned bits = __float_as_uint(g4.x) | __float_as_uint(g4.y) | __float_as_uint(g4.z) |
                                  __float_as_uint(g4.w) | __float_as_uint(m4.x) | __float_as_uint(m4.y) |
                                  __float_as_uint(m4.z) | __float_as_uint(m4.w) | __float_as_uint(v4.x) |
                                  __float_as_uint(v4.y) | __float_as_uint(v4.z) | __float_as_uint(v4.w);
            if (bits == 0 && weight_is_quiet(w4.x, a) && weight_is_quiet(w4.y, a) && weight_is_quiet(w4.z, a) &&
                weight_is_quiet(w4.w, a))
                continue;  // the step would leave every word unchanged
        }
        radam_coordinate(a.gradient_factor * g4.x, a, w4.x, m4.x, v4.x);
        radam_coordinate(a.gradient_factor * g4.y, a, w4.y, m4.y, v4.y);
        radam_coordinate(a.gradient_factor * g4.z, a, w4.z, m4.z, v4.z);
        radam_coordinate(a.gradient_factor * g4.w, a, w4.w, m4.w, v4.w);
        if (kLookahead) {
            const float4 s4 = slow[i];
            w4.x = lookahead_coordinate(w4.x, s4.x, a);
            w4.y = lookahead_coordinate(w4.y, s4.y, a);
            w4.z = lookahead_coordinate(w4.z, s4.z, a);
            w4.w = lookahead_coordinate(w4.w, s4.w, a);
            slow[i] = w4;
        }
        gradients[i] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        weights[i] = w4;
        momentum[i] = m4;
        velocity[i] = v4;
    }
}

__global__ void ranger_scalar_kernel(float* __restrict__ gradients, float* __restrict__ weights,
                                     float* __restrict__ momentum, float* __restrict__ velocity,
                                     float* __restrict__ slow, size_t len, RangerArgs a) {
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < len; i += stride) {
        float w = weights[i], m = momentum[i], v = velocity[i];
        radam_coordinate(a.gradient_factor * gradients[i], a, w, m, v);
        if (a.do_lookahead) {
            w = lookahead_coordinate(w, slow[i], a);
            slow[i] = w;
        }
        gradients[i] = 0.0f;
        weights[i] = w;
        momentum[i] = m;
        velocity[i] = v;
    }
}

__global__ void lookahead_kernel(float* __restrict__ weights, float* __restrict__ slow, size_t len, RangerArgs a) {
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < len; i += stride) {
        const float w = lookahead_coordinate(weights[i], slow[i], a);
        weights[i] = w;
        slow[i] = w;
    }
}

__global__ void sgd_momentum_kernel(float* __restrict__ gradients, float* __restrict__ weights,
                                    float* __restrict__ momentum, float* __restrict__ remainder, size_t len,
                                    float gradient_factor, float learning_rate, float decay, float beta,
                                    float min_weight, float max_weight) {
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < len; i += stride) {
        const float g = gradients[i] * gradient_factor;
        const float m = beta * momentum[i] + g;
        momentum[i] = m;
        float r = remainder[i];
        weights[i] = sgd_compensated(weights[i], r, m, learning_rate, decay, min_weight, max_weight);
        remainder[i] = r;
        gradients[i] = 0.0f;
    }
}

// Norm loss: w *= 1 - rate * (1 - 1/(||w|| + 1e-7)), one norm per tensor
// (reference cu:10308-10364).  Two passes: block sums of squares, then one
// block reduces them in a fixed order and every block rescales.
__global__ void norm_sq_partial_kernel(const float* __restrict__ w, size_t n, float* __restrict__ partials) {
    __shared__ float red[kThreads];
    float s = 0.0f;
    for (size_t i = static_cast<size_t>(blockIdx.x) * kThreads + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * kThreads)
        s += w[i] * w[i];
    red[threadIdx.x] = s;
    __syncthreads();
    for (int d = kThreads / 2; d > 0; d >>= 1) {
        if (threadIdx.x < d) red[threadIdx.x] += red[threadIdx.x + d];
        __syncthreads();
    }
    if (threadIdx.x == 0) partials[blockIdx.x] = red[0];
}

__global__ void norm_scale_kernel(float* __restrict__ w, size_t n, const float* __restrict__ partials, int nparts,
                                  float rate) {
    __shared__ float red[kThreads];
    red[threadIdx.x] = threadIdx.x < nparts ? partials[threadIdx.x] : 0.0f;
    __syncthreads();
    for (int d = kThreads / 2; d > 0; d >>= 1) {
        if (threadIdx.x < d) red[threadIdx.x] += red[threadIdx.x + d];
        __syncthreads();
    }
    const float scale = 1.0f - rate * (1.0f - 1.0f / (sqrtf(red[0]) + 1.0e-7f));
    for (size_t i = static_cast<size_t>(blockIdx.x) * kThreads + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * kThreads)
        w[i] *= scale;
}

int blocks_for(const BulletOuCudaCppContext* ctx, size_t work) {
    size_t b = (work + kThreads - 1) / kThreads;
    size_t cap = static_cast<size_t>(ctx->sm_count) * 8;
    if (b > cap) b = cap;
    if (b == 0) b = 1;
    return static_cast<int>(b);
}

}  // namespace

int apply_norm_loss(BulletOuCudaCppContext* ctx, float* w, size_t n, float rate) {
    if (rate == 0.0f || n == 0) return 0;
    void* scratch = nullptr;
    if (scratch_slot(ctx, kScratchSmallState, kThreads * sizeof(float), &scratch, "norm loss scratch") != 0) return -1;
    float* partials = static_cast<float*>(scratch);
    int nparts = n <= 2048 ? 1 : kThreads;
    norm_sq_partial_kernel<<<nparts, kThreads, 0, ctx->stream>>>(w, n, partials);
    if (check_launch("norm loss partial") != 0) return -1;
    norm_scale_kernel<<<nparts, kThreads, 0, ctx->stream>>>(w, n, partials, nparts, rate);
    return check_launch("norm loss scale");
}

int launch_lookahead(BulletOuCudaCppContext* ctx, size_t len, const RangerArgs& a, float* weights, float* slow) {
    if (len == 0) return 0;
    lookahead_kernel<<<blocks_for(ctx, len), kThreads, 0, ctx->stream>>>(weights, slow, len, a);
    return check_launch("lookahead launch");
}

int launch_ranger(BulletOuCudaCppContext* ctx, size_t len, const RangerArgs& a, float* gradients, float* weights,
                  float* momentum, float* velocity, float* slow) {
    if (len == 0) return 0;
    const bool aligned = (reinterpret_cast<uintptr_t>(gradients) | reinterpret_cast<uintptr_t>(weights) |
                          reinterpret_cast<uintptr_t>(momentum) | reinterpret_cast<uintptr_t>(velocity) |
                          reinterpret_cast<uintptr_t>(slow)) % 16 == 0;
    if (len % 4 == 0 && aligned) {
        const size_t len4 = len / 4;
        const bool skip = !a.do_lookahead && ranger_zero_step_is_identity(a);
        if (a.do_lookahead)
            ranger_vec4_kernel<true><<<blocks_for(ctx, len4), kThreads, 0, ctx->stream>>>(
                reinterpret_cast<float4*>(gradients), reinterpret_cast<float4*>(weights),
                reinterpret_cast<float4*>(momentum), reinterpret_cast<float4*>(velocity),
                reinterpret_cast<float4*>(slow), len4, a, false);
        else
            ranger_vec4_kernel<false><<<blocks_for(ctx, len4), kThreads, 0, ctx->stream>>>(
                reinterpret_cast<float4*>(gradients), reinterpret_cast<float4*>(weights),
                reinterpret_cast<float4*>(momentum), reinterpret_cast<float4*>(velocity),
                reinterpret_cast<float4*>(slow), len4, a, skip);
    } else {
        ranger_scalar_kernel<<<blocks_for(ctx, len), kThreads, 0, ctx->stream>>>(gradients, weights, momentum,
                                                                                  velocity, slow, len, a);
    }
    return check_launch("ranger update launch");
}

}  // namespace bou

extern "C" {

int bulletou_cuda_cpp_ranger_update_device(
    BulletOuCudaCppContext* ctx, float norm_loss_rate, int norm_loss_before, size_t len, float gradient_factor,
    float learning_rate, float step_size, int use_denom, float decay, float beta1, float beta2, float epsilon,
    float min_weight, float max_weight, int do_lookahead, float lookahead_alpha, int clip_after_lookahead,
    BulletOuCudaCppF32Buffer* gradients, BulletOuCudaCppF32Buffer* weights, BulletOuCudaCppF32Buffer* momentum,
    BulletOuCudaCppF32Buffer* velocity, BulletOuCudaCppF32Buffer* slow_params, BulletOuCudaCppHalfMoments* half_moments) {
    if (validate_f32(ctx, gradients, len, "gradients") != 0 || validate_f32(ctx, weights, len, "weights") != 0 ||
        validate_f32(ctx, momentum, len, "momentum") != 0 || validate_f32(ctx, velocity, len, "velocity") != 0 ||
        validate_f32(ctx, slow_params, len, "slow_params") != 0)
        return -1;
    if (set_device(ctx) != 0) return -1;
    if (half_moments != nullptr) return fail_message("FP16 optimizer moments are not supported by this backend");
    if (len == 0) return ok();
    BulletOuB200RangerStep s{norm_loss_rate, norm_loss_before, gradient_factor, learning_rate, step_size, use_denom,
                             decay, beta1, beta2, epsilon, min_weight, max_weight, do_lookahead, lookahead_alpha,
                             clip_after_lookahead};
    const RangerArgs a = ranger_args_from(s);
    if (norm_loss_before && apply_norm_loss(ctx, weights->ptr, len, norm_loss_rate) != 0) return -1;
    if (!norm_loss_before && norm_loss_rate != 0.0f) {
        // Norm loss after the RAdam step but before lookahead (reference order).
        RangerArgs no_la = a;
        no_la.do_lookahead = 0;
        if (launch_ranger(ctx, len, no_la, gradients->ptr, weights->ptr, momentum->ptr, velocity->ptr,
                          slow_params->ptr) != 0)
            return -1;
        if (apply_norm_loss(ctx, weights->ptr, len, norm_loss_rate) != 0) return -1;
        if (a.do_lookahead) {
            lookahead_kernel<<<blocks_for(ctx, len), kThreads, 0, ctx->stream>>>(weights->ptr, slow_params->ptr, len, a);
            if (check_launch("lookahead launch") != 0) return -1;
        }
        return ok();
    }
    if (launch_ranger(ctx, len, a, gradients->ptr, weights->ptr, momentum->ptr, velocity->ptr, slow_params->ptr) != 0)
        return -1;
    return ok();
}

int bulletou_cuda_cpp_ranger_update_host(int device, size_t len, float gradient_factor, float learning_rate,
                                         float step_size, int use_denom, float decay, float beta1, float beta2,
                                         float epsilon, float min_weight, float max_weight, int do_lookahead,
                                         float lookahead_alpha, int clip_after_lookahead, float* gradients,
                                         float* weights, float* momentum, float* velocity, float* slow_params) {
    if (validate_host(gradients, len, "gradients") != 0 || validate_host(weights, len, "weights") != 0 ||
        validate_host(momentum, len, "momentum") != 0 || validate_host(velocity, len, "velocity") != 0 ||
        validate_host(slow_params, len, "slow_params") != 0)
        return -1;
    BulletOuCudaCppContext* ctx = nullptr;
    if (bulletou_cuda_cpp_context_create(device, &ctx) != 0) return -1;
    BulletOuCudaCppF32Buffer* b[5] = {nullptr, nullptr, nullptr, nullptr, nullptr};
    float* host[5] = {gradients, weights, momentum, velocity, slow_params};
    int rc = 0;
    for (int i = 0; i < 5 && rc == 0; ++i) rc = bulletou_cuda_cpp_f32_buffer_create(ctx, len, &b[i]);
    for (int i = 0; i < 5 && rc == 0; ++i) rc = bulletou_cuda_cpp_f32_upload(ctx, b[i], host[i], len);
    if (rc == 0)
        rc = bulletou_cuda_cpp_ranger_update_device(ctx, 0.0f, 0, len, gradient_factor, learning_rate, step_size,
                                                    use_denom, decay, beta1, beta2, epsilon, min_weight, max_weight,
                                                    do_lookahead, lookahead_alpha, clip_after_lookahead, b[0], b[1],
                                                    b[2], b[3], b[4], nullptr);
    for (int i = 0; i < 5 && rc == 0; ++i) rc = bulletou_cuda_cpp_f32_download(ctx, b[i], host[i], len);
    char saved[512] = {0};
    if (rc != 0) bulletou_cuda_cpp_last_error(saved, sizeof(saved));
    for (auto* p : b) bulletou_cuda_cpp_f32_buffer_destroy(p);
    bulletou_cuda_cpp_context_destroy(ctx);
    if (rc != 0) {
        fail_message(saved);
        return rc;
    }
    return ok();
}

int bulletou_cuda_cpp_sgd_momentum_update_device(BulletOuCudaCppContext* ctx, size_t len, float gradient_factor,
                                                 float learning_rate, float decay, float beta, float min_weight,
                                                 float max_weight, BulletOuCudaCppF32Buffer* gradients,
                                                 BulletOuCudaCppF32Buffer* weights, BulletOuCudaCppF32Buffer* momentum,
                                                 BulletOuCudaCppF32Buffer* remainder,
                                                 BulletOuCudaCppHalfMoments* half_moments) {
    if (validate_f32(ctx, gradients, len, "SGD gradients") != 0 || validate_f32(ctx, weights, len, "SGD weights") != 0 ||
        validate_f32(ctx, momentum, len, "SGD momentum") != 0 ||
        validate_f32(ctx, remainder, len, "SGD update remainder") != 0 || set_device(ctx) != 0)
        return -1;
    if (half_moments != nullptr) return fail_message("FP16 optimizer moments are not supported by this backend");
    if (len == 0) return ok();
    sgd_momentum_kernel<<<blocks_for(ctx, len), kThreads, 0, ctx->stream>>>(
        gradients->ptr, weights->ptr, momentum->ptr, remainder->ptr, len, gradient_factor, learning_rate, decay, beta,
        min_weight, max_weight);
    if (check_launch("SGD momentum update") != 0) return -1;
    return ok();
}

}  // extern "C"
