// Per-sample scalar value losses shared by the standalone loss entry and the
// fused train-step kernels.  Same formulas as the reference
// (crates/cuda_cpp/cpp/bulletou_cuda_backend.cu):
//   kind 0  sigmoid-pow   cu:2790-2813  (sigmoid(out*inv_scale) vs target, |err|^p)
//   kind 1  win-rate model cu:2815-2843
//   kind 2  BCE with logits cu:2734-2746 (k = 0 only in the fused kernels)
// Compiled with --use_fast_math like the reference, so expf/powf/division map
// to the same fast-math forms.
#pragma once

namespace bou {

__device__ __forceinline__ float loss_sigmoid(float x) { return 1.0f / (1.0f + expf(-x)); }

__device__ __forceinline__ float signum_or_zero(float x) { return x > 0.0f ? 1.0f : (x < 0.0f ? -1.0f : 0.0f); }

struct LossArgs {
    int kind;
    float output_inv_scale;
    float pow_exp;
    float param;
    float normalizer;  // divisor of the output gradient (the batch, or a global batch)
};

// Returns the weighted per-sample loss and writes the output gradient
// (already multiplied by the entry weight and divided by the normalizer).
__device__ __forceinline__ float sample_loss(const LossArgs& a, float output, float target, float entry_weight,
                                             float* out_gradient) {
    if (a.kind == 2) {
        const float z = output * a.output_inv_scale;
        const float loss = (z >= 0.0f ? (1.0f - target) * z : -target * z) + log1pf(expf(-fabsf(z)));
        *out_gradient = entry_weight * (loss_sigmoid(z) - target) * a.output_inv_scale / a.normalizer;
        return entry_weight * loss;
    }
    if (a.kind == 1) {
        const float score = output * a.output_inv_scale;
        const float q = loss_sigmoid(score - a.param);
        const float qm = loss_sigmoid(-score - a.param);
        const float prediction = (1.0f + q - qm) * 0.5f;
        const float error = prediction - target;
        const float abs_error = fabsf(error);
        const float loss = powf(abs_error, a.pow_exp);
        const float q_prime = q * (1.0f - q);
        const float qm_prime = qm * (1.0f - qm);
        const float prediction_gradient = 0.5f * a.output_inv_scale * (q_prime + qm_prime);
        const float loss_gradient =
            abs_error == 0.0f ? 0.0f : a.pow_exp * signum_or_zero(error) * powf(abs_error, a.pow_exp - 1.0f);
        *out_gradient = entry_weight * loss_gradient * prediction_gradient / a.normalizer;
        return entry_weight * loss;
    }
    const float prediction = loss_sigmoid(output * a.output_inv_scale);
    const float error = prediction - target;
    const float abs_error = fabsf(error);
    const float loss = powf(abs_error, a.pow_exp);
    const float loss_gradient =
        abs_error == 0.0f ? 0.0f : a.pow_exp * signum_or_zero(error) * powf(abs_error, a.pow_exp - 1.0f);
    const float gradient = loss_gradient * prediction * (1.0f - prediction) * a.output_inv_scale;
    *out_gradient = entry_weight * gradient / a.normalizer;
    return entry_weight * loss;
}

}  // namespace bou
