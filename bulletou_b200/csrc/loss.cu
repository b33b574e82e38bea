// Scalar value loss entries of the drop-in ABI (reference cu:8872-8968,
// 11809-11885, 11984-12068).  Per-sample math is shared with the fused train
// step (loss.cuh); the batch sum is a fixed-order tree reduction instead of
// the reference's single-thread serial loop (cu:2845).
#include <cmath>

#include "common.cuh"
#include "loss.cuh"

namespace bou {

namespace {

__global__ void scalar_loss_kernel(LossArgs a, const float* __restrict__ outputs, const float* __restrict__ targets,
                                   const float* __restrict__ entry_weights, float* __restrict__ per_sample,
                                   float* __restrict__ mog, size_t batch) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= batch) return;
    float g = 0.0f;
    per_sample[i] = sample_loss(a, outputs[i], targets[i], entry_weights[i], &g);
    mog[i] = g;
}

// Entry-weighted mean |sigmoid(z) - t| over samples with weight > 0, in
// double (reference cu:2751-2776); stored in *mean_error.
__global__ void bce_mean_error_kernel(const float* __restrict__ outputs, const float* __restrict__ targets,
                                      const float* __restrict__ entry_weights, float scale, size_t batch,
                                      float* __restrict__ mean_error) {
    __shared__ double err[256];
    __shared__ double wsum[256];
    double e = 0.0, w = 0.0;
    for (size_t i = threadIdx.x; i < batch; i += 256) {
        if (entry_weights[i] > 0.0f) {
            e += static_cast<double>(entry_weights[i]) * fabsf(loss_sigmoid(outputs[i] * scale) - targets[i]);
            w += entry_weights[i];
        }
    }
    err[threadIdx.x] = e;
    wsum[threadIdx.x] = w;
    __syncthreads();
    for (int d = 128; d > 0; d >>= 1) {
        if (threadIdx.x < d) {
            err[threadIdx.x] += err[threadIdx.x + d];
            wsum[threadIdx.x] += wsum[threadIdx.x + d];
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) *mean_error = wsum[0] > 0.0 ? static_cast<float>(err[0] / wsum[0]) : 0.0f;
}

// Detached error weight (1 + k|e|) / (1 + k mean|e|) on loss and gradient
// (reference cu:2778-2788).
__global__ void bce_error_weight_kernel(const float* __restrict__ outputs, const float* __restrict__ targets,
                                        const float* __restrict__ entry_weights, float* __restrict__ per_sample,
                                        float* __restrict__ mog, const float* __restrict__ mean_error, float scale,
                                        float k, size_t batch) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= batch || entry_weights[i] == 0.0f) return;
    const float error = fabsf(loss_sigmoid(outputs[i] * scale) - targets[i]);
    const float weight = static_cast<float>((1.0 + static_cast<double>(k) * error) /
                                            (1.0 + static_cast<double>(k) * *mean_error));
    per_sample[i] *= weight;
    mog[i] *= weight;
}

__global__ void __launch_bounds__(1024) loss_finalize_kernel(const float* __restrict__ per_sample, size_t batch,
                                                             float* __restrict__ weighted_sum, float* __restrict__ mean) {
    __shared__ float red[1024];
    float s = 0.0f;
    for (size_t i = threadIdx.x; i < batch; i += 1024) s += per_sample[i];
    red[threadIdx.x] = s;
    __syncthreads();
    for (int d = 512; d > 0; d >>= 1) {
        if (threadIdx.x < d) red[threadIdx.x] += red[threadIdx.x + d];
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        *weighted_sum = red[0];
        *mean = red[0] / static_cast<float>(batch);
    }
}

int validate_scalar_loss(size_t batch, int kind, float pow_exp, float param) {
    if (batch == 0) return fail_message("scalar loss batch size must be greater than zero");
    if (kind != 0 && kind != 1 && kind != 2)
        return fail_message("scalar loss kind must be 0 (sigmoid-pow), 1 (win-rate-model), or 2 (BCE with logits)");
    if (!(std::isfinite(pow_exp) && pow_exp >= 1.0f)) return fail_message("loss_pow_exp must be finite and >= 1");
    if (kind == 1 && !std::isfinite(param)) return fail_message("WRM loss parameter must be finite");
    if (kind == 2 && !(std::isfinite(param) && param >= 0.0f))
        return fail_message("BCE error weight k must be finite and >= 0");
    return 0;
}

}  // namespace

int launch_scalar_loss(BulletOuCudaCppContext* ctx, const LossArgs& la, size_t batch, const float* outputs,
                       const float* targets, const float* entry_weights, float* per_sample, float* mog,
                       float* weighted_sum, float* mean, int finalize) {
    int blocks = 0;
    if (grid_1d(batch, 256, &blocks, "scalar loss") != 0) return -1;
    scalar_loss_kernel<<<blocks, 256, 0, ctx->stream>>>(la, outputs, targets, entry_weights, per_sample, mog, batch);
    if (check_launch("scalar loss launch") != 0) return -1;
    if (la.kind == 2 && la.param > 0.0f) {
        bce_mean_error_kernel<<<1, 256, 0, ctx->stream>>>(outputs, targets, entry_weights, la.output_inv_scale, batch,
                                                          weighted_sum);
        bce_error_weight_kernel<<<blocks, 256, 0, ctx->stream>>>(outputs, targets, entry_weights, per_sample, mog,
                                                                 weighted_sum, la.output_inv_scale, la.param, batch);
        if (check_launch("BCE error weight launch") != 0) return -1;
    }
    if (finalize) {
        loss_finalize_kernel<<<1, 1024, 0, ctx->stream>>>(per_sample, batch, weighted_sum, mean);
        if (check_launch("loss finalize launch") != 0) return -1;
    }
    return 0;
}

// Converts a fused-step loss spec (same validation as the ABI loss entry).
int loss_args(const BulletOuB200LossSpec* loss, size_t batch, LossArgs* out) {
    if (loss == nullptr) return fail_message("loss spec must not be null");
    if (loss->kind < 0 || loss->kind > 2) return fail_message("scalar loss kind must be 0, 1 or 2");
    if (loss->kind == 2 && loss->loss_param != 0.0f)
        return fail_message("BCE error weighting (k > 0) is not supported by the fused train step");
    if (!(std::isfinite(loss->loss_pow_exp) && loss->loss_pow_exp >= 1.0f))
        return fail_message("loss_pow_exp must be finite and >= 1");
    if (loss->kind == 1 && !std::isfinite(loss->loss_param)) return fail_message("WRM loss parameter must be finite");
    out->kind = loss->kind;
    out->output_inv_scale = loss->output_inv_scale;
    out->pow_exp = loss->loss_pow_exp;
    out->param = loss->loss_param;
    out->normalizer = static_cast<float>(loss->normalizer == 0 ? batch : loss->normalizer);
    return 0;
}

}  // namespace bou

using namespace bou;

extern "C" {

int bulletou_cuda_cpp_scalar_loss_device_with_finalize(
    BulletOuCudaCppContext* ctx, int kind, float output_inv_scale, float loss_pow_exp, float loss_param, size_t batch,
    const BulletOuCudaCppF32Buffer* outputs, const BulletOuCudaCppF32Buffer* targets,
    const BulletOuCudaCppF32Buffer* entry_weights, BulletOuCudaCppF32Buffer* per_sample,
    BulletOuCudaCppF32Buffer* mean_output_gradients, BulletOuCudaCppF32Buffer* weighted_sum,
    BulletOuCudaCppF32Buffer* mean, int finalize_loss) {
    if (validate_scalar_loss(batch, kind, loss_pow_exp, loss_param) != 0 ||
        validate_f32(ctx, outputs, batch, "outputs") != 0 || validate_f32(ctx, targets, batch, "targets") != 0 ||
        validate_f32(ctx, entry_weights, batch, "entry_weights") != 0 ||
        validate_f32(ctx, per_sample, batch, "per_sample") != 0 ||
        validate_f32(ctx, mean_output_gradients, batch, "mean_output_gradients") != 0 ||
        validate_f32(ctx, weighted_sum, 1, "weighted_sum") != 0 || validate_f32(ctx, mean, 1, "mean") != 0)
        return -1;
    if (set_device(ctx) != 0) return -1;
    LossArgs la{kind, output_inv_scale, loss_pow_exp, loss_param, static_cast<float>(batch)};
    if (launch_scalar_loss(ctx, la, batch, outputs->ptr, targets->ptr, entry_weights->ptr, per_sample->ptr,
                           mean_output_gradients->ptr, weighted_sum->ptr, mean->ptr, finalize_loss) != 0)
        return -1;
    return ok();
}

int bulletou_cuda_cpp_scalar_loss_device(BulletOuCudaCppContext* ctx, int kind, float output_inv_scale,
                                         float loss_pow_exp, float unused_loss_param, size_t batch,
                                         const BulletOuCudaCppF32Buffer* outputs, const BulletOuCudaCppF32Buffer* targets,
                                         const BulletOuCudaCppF32Buffer* entry_weights,
                                         BulletOuCudaCppF32Buffer* per_sample,
                                         BulletOuCudaCppF32Buffer* mean_output_gradients,
                                         BulletOuCudaCppF32Buffer* weighted_sum, BulletOuCudaCppF32Buffer* mean) {
    return bulletou_cuda_cpp_scalar_loss_device_with_finalize(ctx, kind, output_inv_scale, loss_pow_exp,
                                                              unused_loss_param, batch, outputs, targets,
                                                              entry_weights, per_sample, mean_output_gradients,
                                                              weighted_sum, mean, 1);
}

int bulletou_cuda_cpp_scalar_loss_host(int device, int kind, float output_inv_scale, float loss_pow_exp,
                                       float unused_loss_param, size_t batch, const float* outputs,
                                       const float* targets, const float* entry_weights, float* per_sample,
                                       float* mean_output_gradients, float* weighted_sum, float* mean) {
    if (validate_scalar_loss(batch, kind, loss_pow_exp, unused_loss_param) != 0 ||
        validate_host(outputs, batch, "outputs") != 0 || validate_host(targets, batch, "targets") != 0 ||
        validate_host(entry_weights, batch, "entry_weights") != 0 ||
        validate_host(per_sample, batch, "per_sample") != 0 ||
        validate_host(mean_output_gradients, batch, "mean_output_gradients") != 0 ||
        validate_host(weighted_sum, 1, "weighted_sum") != 0 || validate_host(mean, 1, "mean") != 0)
        return -1;
    BulletOuCudaCppContext* ctx = nullptr;
    if (bulletou_cuda_cpp_context_create(device, &ctx) != 0) return -1;
    BulletOuCudaCppF32Buffer* b[7] = {};
    const size_t lens[7] = {batch, batch, batch, batch, batch, 1, 1};
    int rc = 0;
    for (int i = 0; i < 7 && rc == 0; ++i) rc = bulletou_cuda_cpp_f32_buffer_create(ctx, lens[i], &b[i]);
    if (rc == 0) rc = bulletou_cuda_cpp_f32_upload(ctx, b[0], outputs, batch);
    if (rc == 0) rc = bulletou_cuda_cpp_f32_upload(ctx, b[1], targets, batch);
    if (rc == 0) rc = bulletou_cuda_cpp_f32_upload(ctx, b[2], entry_weights, batch);
    if (rc == 0)
        rc = bulletou_cuda_cpp_scalar_loss_device(ctx, kind, output_inv_scale, loss_pow_exp, unused_loss_param, batch,
                                                  b[0], b[1], b[2], b[3], b[4], b[5], b[6]);
    if (rc == 0) rc = bulletou_cuda_cpp_f32_download(ctx, b[3], per_sample, batch);
    if (rc == 0) rc = bulletou_cuda_cpp_f32_download(ctx, b[4], mean_output_gradients, batch);
    if (rc == 0) rc = bulletou_cuda_cpp_f32_download(ctx, b[5], weighted_sum, 1);
    if (rc == 0) rc = bulletou_cuda_cpp_f32_download(ctx, b[6], mean, 1);
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

}  // extern "C"
