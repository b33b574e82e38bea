// Per-element optimizer arithmetic shared by the standalone optimizer entry
// points and the fused row kernels.
//
// The arithmetic is the reference's, term for term, so that a fused update of
// a parameter is bit-identical to the reference's separate update kernel when
// both are built with --use_fast_math (the reference's build flags,
// crates/cuda_cpp/build.rs:46-49):
//   RAdam step   cu:476-505 (radam_update_one)
//   weight clip  cu:466-473 (disabled when the bounds are -FLT_MAX/FLT_MAX)
//   lookahead    cu:686-728
//   SGD momentum cu:10429-10456 (compensated master weight)
#pragma once

#include <cfloat>

#include "../../include/bulletou_b200.h"

namespace bou {

struct RangerArgs {
    float gradient_factor;
    float learning_rate;
    float step_size;
    int use_denom;
    float decay;
    float beta1;
    float beta2;
    float epsilon;
    float min_weight;
    float max_weight;
    int do_lookahead;
    float lookahead_alpha;
    float lookahead_min;
    float lookahead_max;
};

inline RangerArgs ranger_args_from(const BulletOuB200RangerStep& s) {
    RangerArgs a;
    a.gradient_factor = s.gradient_factor;
    a.learning_rate = s.learning_rate;
    a.step_size = s.step_size;
    a.use_denom = s.use_denom;
    a.decay = s.decay;
    a.beta1 = s.beta1;
    a.beta2 = s.beta2;
    a.epsilon = s.epsilon;
    a.min_weight = s.min_weight;
    a.max_weight = s.max_weight;
    a.do_lookahead = s.do_lookahead;
    a.lookahead_alpha = s.lookahead_alpha;
    a.lookahead_min = s.clip_after_lookahead ? s.min_weight : -FLT_MAX;
    a.lookahead_max = s.clip_after_lookahead ? s.max_weight : FLT_MAX;
    return a;
}

__device__ __forceinline__ float clamp_weight(float w, float lo, float hi) {
    // Both bounds at the float extremes mean "no clipping": the value passes
    // through untouched (NaN and infinities included).
    if (lo == -FLT_MAX && hi == FLT_MAX) return w;
    return fminf(fmaxf(w, lo), hi);
}

// One RAdam step on one coordinate; `grad` already includes gradient_factor.
__device__ __forceinline__ void radam_coordinate(float grad, const RangerArgs& a, float& weight, float& momentum,
                                                 float& velocity) {
    const float rate = a.learning_rate * a.step_size;
    float w = weight * (1.0f - a.decay * rate);
    const float m = a.beta1 * momentum + (1.0f - a.beta1) * grad;
    const float v = a.beta2 * velocity + (1.0f - a.beta2) * grad * grad;
    float step = m;
    if (a.use_denom != 0) step /= sqrtf(v) + a.epsilon;
    w -= rate * step;
    weight = clamp_weight(w, a.min_weight, a.max_weight);
    momentum = m;
    velocity = v;
}

__device__ __forceinline__ float lookahead_coordinate(float weight, float slow, const RangerArgs& a) {
    return clamp_weight(a.lookahead_alpha * weight + (1.0f - a.lookahead_alpha) * slow, a.lookahead_min,
                        a.lookahead_max);
}

// True when a RAdam step with zero gradient and zero moments leaves the
// coordinate bit-for-bit unchanged, so its stores may be skipped.  Mirrors the
// conditions of the reference's skip_unchanged_zero fast path (cu:626-634):
// zero decay, finite positive rates, betas in [0,1], a normal finite weight
// inside the clip range.
__host__ __device__ inline bool ranger_zero_step_is_identity(const RangerArgs& a) {
    const float rate = a.learning_rate * a.step_size;
    return a.decay == 0.0f && a.gradient_factor > 0.0f && a.gradient_factor <= FLT_MAX && a.learning_rate > 0.0f &&
           a.learning_rate <= FLT_MAX && a.step_size > 0.0f && a.step_size <= FLT_MAX && rate <= FLT_MAX &&
           a.beta1 >= 0.0f && a.beta1 <= 1.0f && a.beta2 >= 0.0f && a.beta2 <= 1.0f &&
           (a.use_denom == 0 || (a.epsilon >= FLT_MIN && a.epsilon <= FLT_MAX));
}

__device__ __forceinline__ bool weight_is_quiet(float w, const RangerArgs& a) {
    return isfinite(w) && fabsf(w) >= FLT_MIN && w >= a.min_weight && w <= a.max_weight;
}

// SGD with momentum on a two-float master weight (weight + remainder).
__device__ __forceinline__ float sgd_compensated(float weight, float& remainder, float momentum, float learning_rate,
                                                 float decay, float min_weight, float max_weight) {
    const float decay_rate = learning_rate * decay;
    const float delta =
        __fadd_rn(__fadd_rn(-learning_rate * momentum, -decay_rate * weight), remainder * (1.0f - decay_rate));
    const float updated = __fadd_rn(weight, delta);
    const float clipped = clamp_weight(updated, min_weight, max_weight);
    remainder = clipped == updated ? __fadd_rn(__fsub_rn(weight, updated), delta) : 0.0f;
    if ((clipped >= max_weight && remainder > 0.0f) || (clipped <= min_weight && remainder < 0.0f)) remainder = 0.0f;
    return clipped;
}

}  // namespace bou
