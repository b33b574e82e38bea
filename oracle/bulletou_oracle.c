/*
 * bulletou_oracle.c -- TEST INFRASTRUCTURE ONLY.  Never linked into, loaded
 * by, or called from the product library; only tests/, __graft_entry__.smoke()
 * and bench.py's CPU-baseline leg use it, as the checker.
 *
 * A plain-C, single-threaded restatement of the reference's training-path
 * arithmetic (yaneurao/BulletOu), each function citing what it follows:
 *   "cu"      crates/cuda_cpp/cpp/bulletou_cuda_backend.cu  (the GPU backend
 *             the product replaces; its kernels define the training math)
 *   "lib.rs"  crates/cuda_cpp/src/lib.rs                  (host-side runner)
 *   "smoke"   crates/cuda_cpp/src/bin/smoke.rs             (CPU backprop golden)
 *   fast_nnue / fast_loss: crates/bulletou_lib/src/value/fast_{nnue,loss}.rs (CPU goldens)
 *
 * Deliberate differences from the reference's own CPU loops, for a sharper
 * oracle: batch reductions (weight gradients, loss sums) accumulate in
 * double; dense dots use fmaf in the reference GPU kernels' order, so the
 * forward is bit-comparable with the GPU reference.  Parity pins: the inline
 * goldens of the reference tests (fast_nnue.rs:345-455, fast_loss.rs:98-160,
 * lib.rs:12965, smoke.rs:65-216) are checked against this file in tests/.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#include <float.h>

#define EXPORT __attribute__((visibility("default")))

/* HalfKP factorization: cu:1004-1019. */
static int row_map(int64_t input_size, int f, int64_t* r0, int64_t* r1) {
    if (f < 0 || (int64_t)f >= input_size) return 0;
    if (input_size == 125388 + 1548 && f < 125388) {
        *r0 = 1548 + (int64_t)f;
        *r1 = (int64_t)f % 1548;
        return 2;
    }
    *r0 = f;
    return 1;
}

static float crelu(float x) { return fminf(fmaxf(x, 0.0f), 1.0f); }
static float crelu_grad(float a, float g) { return (a > 0.0f && a < 1.0f) ? g : 0.0f; }

/* Sparse FT forward of one perspective: bias, then slots in order
 * (cu:1021-1052, fast_nnue.rs:284-292). */
static void ft_perspective(int64_t input_size, int64_t l1, int64_t max_active, const int* idx, const float* l0w,
                           const float* l0b, float* out) {
    for (int64_t c = 0; c < l1; ++c) {
        float sum = l0b[c];
        for (int64_t s = 0; s < max_active; ++s) {
            int64_t r0, r1;
            int n = row_map(input_size, idx[s], &r0, &r1);
            if (n == 1) sum += l0w[r0 * l1 + c];
            else if (n == 2) sum += l0w[r0 * l1 + c] + l0w[r1 * l1 + c];
        }
        out[c] = crelu(sum);
    }
}

/* HalfKP forward (cu:5894-5991 launch order; fast_nnue.rs:209-271). */
EXPORT void oracle_nnue_forward(int64_t input_size, int64_t l1, int64_t l2, int64_t l3, int64_t batch,
                                int64_t max_active, const int* stm, const int* nstm, const float* l0w,
                                const float* l0b, const float* l1w, const float* l1b, const float* l2w,
                                const float* l2b, const float* outw, const float* outb, float* stm_l0,
                                float* nstm_l0, float* combined, float* hidden1, float* hidden2, float* output) {
    for (int64_t b = 0; b < batch; ++b) {
        float* s0 = stm_l0 + b * l1;
        float* n0 = nstm_l0 + b * l1;
        ft_perspective(input_size, l1, max_active, stm + b * max_active, l0w, l0b, s0);
        ft_perspective(input_size, l1, max_active, nstm + b * max_active, l0w, l0b, n0);
        float* c = combined + b * 2 * l1;
        memcpy(c, s0, (size_t)l1 * sizeof(float));
        memcpy(c + l1, n0, (size_t)l1 * sizeof(float));
        float* h1 = hidden1 + b * l2;
        for (int64_t o = 0; o < l2; ++o) {
            float sum = l1b[o];
            for (int64_t i = 0; i < 2 * l1; ++i) sum = fmaf(c[i], l1w[i * l2 + o], sum);
            h1[o] = crelu(sum);
        }
        float* h2 = hidden2 + b * l3;
        for (int64_t o = 0; o < l3; ++o) {
            float sum = l2b[o];
            for (int64_t i = 0; i < l2; ++i) sum = fmaf(h1[i], l2w[i * l3 + o], sum);
            h2[o] = crelu(sum);
        }
        float sum = outb[0];
        for (int64_t i = 0; i < l3; ++i) sum = fmaf(h2[i], outw[i], sum);
        output[b] = sum;
    }
}

static float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }
static float signum_(float x) { return x > 0.0f ? 1.0f : (x < 0.0f ? -1.0f : 0.0f); }

/* Scalar losses: kind 0 sigmoid-pow (cu:2790-2813, fast_loss.rs:42-96),
 * kind 1 win-rate model (cu:2815-2843), kind 2 BCE with logits (cu:2734-2746).
 * `normalizer` divides the output gradient (the batch size in the reference). */
EXPORT void oracle_scalar_loss(int kind, float inv_scale, float pow_exp, float param, int64_t batch,
                               float normalizer, const float* outputs, const float* targets,
                               const float* entry_weights, float* per_sample, float* mog, float* weighted_sum,
                               float* mean) {
    double total = 0.0;
    for (int64_t i = 0; i < batch; ++i) {
        float w = entry_weights[i], t = targets[i], loss, grad;
        if (kind == 2) {
            float z = outputs[i] * inv_scale;
            loss = (z >= 0.0f ? (1.0f - t) * z : -t * z) + log1pf(expf(-fabsf(z)));
            grad = w * (sigmoidf_(z) - t) * inv_scale / normalizer;
        } else if (kind == 1) {
            float score = outputs[i] * inv_scale;
            float q = sigmoidf_(score - param), qm = sigmoidf_(-score - param);
            float pred = (1.0f + q - qm) * 0.5f;
            float err = pred - t, ae = fabsf(err);
            loss = powf(ae, pow_exp);
            float pg = 0.5f * inv_scale * (q * (1.0f - q) + qm * (1.0f - qm));
            float lg = ae == 0.0f ? 0.0f : pow_exp * signum_(err) * powf(ae, pow_exp - 1.0f);
            grad = w * lg * pg / normalizer;
        } else {
            float pred = sigmoidf_(outputs[i] * inv_scale);
            float err = pred - t, ae = fabsf(err);
            loss = powf(ae, pow_exp);
            float lg = ae == 0.0f ? 0.0f : pow_exp * signum_(err) * powf(ae, pow_exp - 1.0f);
            grad = w * (lg * pred * (1.0f - pred) * inv_scale) / normalizer;
        }
        per_sample[i] = w * loss;
        mog[i] = grad;
        total += (double)per_sample[i];
    }
    *weighted_sum = (float)total;
    *mean = (float)(total / (double)batch);
}

/* HalfKP backward with the reference ABI's buffer semantics (cu:9142-9290;
 * CPU golden smoke.rs:594-700): hidden2/hidden1 gradients end masked by the
 * ClippedReLU derivative, combined gradient unmasked, l0 gradients masked;
 * l0w_grad ACCUMULATES, every other gradient is overwritten. */
EXPORT void oracle_nnue_backward(int64_t input_size, int64_t l1, int64_t l2, int64_t l3, int64_t batch,
                                 int64_t max_active, const int* stm, const int* nstm, const float* combined,
                                 const float* hidden1, const float* hidden2, const float* stm_l0,
                                 const float* nstm_l0, const float* l1w, const float* l2w, const float* outw,
                                 const float* mog, float* h2g, float* h1g, float* cg, float* stm_g, float* nstm_g,
                                 float* l0w_g, float* l0b_g, float* l1w_g, float* l1b_g, float* l2w_g,
                                 float* l2b_g, float* outw_g, float* outb_g, double* scratch /* >= max(2*l1*l2, l2*l3) + l1 + 64 */) {
    int64_t in = 2 * l1;
    /* output layer (cu:5042-5075) */
    double ob = 0.0;
    for (int64_t k = 0; k < l3; ++k) scratch[k] = 0.0;
    for (int64_t b = 0; b < batch; ++b) {
        ob += mog[b];
        for (int64_t k = 0; k < l3; ++k) {
            h2g[b * l3 + k] = mog[b] * outw[k];
            scratch[k] += (double)mog[b] * hidden2[b * l3 + k];
        }
    }
    for (int64_t k = 0; k < l3; ++k) outw_g[k] = (float)scratch[k];
    outb_g[0] = (float)ob;
    /* L2 (cu:5126-5240): mask in place, dX = W g, dW = sum x g, db = sum g */
    for (int64_t i = 0; i < batch * l3; ++i) h2g[i] = crelu_grad(hidden2[i], h2g[i]);
    for (int64_t b = 0; b < batch; ++b)
        for (int64_t j = 0; j < l2; ++j) {
            float s = 0.0f;
            for (int64_t k = 0; k < l3; ++k) s = fmaf(h2g[b * l3 + k], l2w[j * l3 + k], s);
            h1g[b * l2 + j] = s;
        }
    for (int64_t e = 0; e < l2 * l3 + l3; ++e) scratch[e] = 0.0;
    for (int64_t b = 0; b < batch; ++b)
        for (int64_t j = 0; j < l2; ++j)
            for (int64_t k = 0; k < l3; ++k) scratch[j * l3 + k] += (double)hidden1[b * l2 + j] * h2g[b * l3 + k];
    for (int64_t b = 0; b < batch; ++b)
        for (int64_t k = 0; k < l3; ++k) scratch[l2 * l3 + k] += h2g[b * l3 + k];
    for (int64_t e = 0; e < l2 * l3; ++e) l2w_g[e] = (float)scratch[e];
    for (int64_t k = 0; k < l3; ++k) l2b_g[k] = (float)scratch[l2 * l3 + k];
    /* L1 */
    for (int64_t i = 0; i < batch * l2; ++i) h1g[i] = crelu_grad(hidden1[i], h1g[i]);
    for (int64_t b = 0; b < batch; ++b)
        for (int64_t i = 0; i < in; ++i) {
            float s = 0.0f;
            for (int64_t j = 0; j < l2; ++j) s = fmaf(h1g[b * l2 + j], l1w[i * l2 + j], s);
            cg[b * in + i] = s;
        }
    for (int64_t e = 0; e < in * l2 + l2; ++e) scratch[e] = 0.0;
    for (int64_t b = 0; b < batch; ++b)
        for (int64_t i = 0; i < in; ++i) {
            double x = combined[b * in + i];
            if (x == 0.0) continue;
            for (int64_t j = 0; j < l2; ++j) scratch[i * l2 + j] += x * h1g[b * l2 + j];
        }
    for (int64_t b = 0; b < batch; ++b)
        for (int64_t j = 0; j < l2; ++j) scratch[in * l2 + j] += h1g[b * l2 + j];
    for (int64_t e = 0; e < in * l2; ++e) l1w_g[e] = (float)scratch[e];
    for (int64_t j = 0; j < l2; ++j) l1b_g[j] = (float)scratch[in * l2 + j];
    /* FT (cu:5256-5365) */
    for (int64_t b = 0; b < batch; ++b)
        for (int64_t c = 0; c < l1; ++c) {
            stm_g[b * l1 + c] = crelu_grad(stm_l0[b * l1 + c], cg[b * in + c]);
            nstm_g[b * l1 + c] = crelu_grad(nstm_l0[b * l1 + c], cg[b * in + l1 + c]);
        }
    for (int64_t c = 0; c < l1; ++c) scratch[c] = 0.0;
    for (int64_t b = 0; b < batch; ++b)
        for (int64_t c = 0; c < l1; ++c) scratch[c] += (double)(stm_g[b * l1 + c] + nstm_g[b * l1 + c]);
    for (int64_t c = 0; c < l1; ++c) l0b_g[c] = (float)scratch[c];
    for (int64_t b = 0; b < batch; ++b)
        for (int64_t s = 0; s < max_active; ++s)
            for (int p = 0; p < 2; ++p) {
                int f = (p == 0 ? stm : nstm)[b * max_active + s];
                const float* g = (p == 0 ? stm_g : nstm_g) + b * l1;
                int64_t r0, r1;
                int n = row_map(input_size, f, &r0, &r1);
                for (int k = 0; k < n; ++k) {
                    int64_t r = k == 0 ? r0 : r1;
                    for (int64_t c = 0; c < l1; ++c) l0w_g[r * l1 + c] += g[c];
                }
            }
}

/* RAdam step scale (lib.rs:9268-9288), computed in f32 like the Rust code. */
EXPORT void oracle_radam_step_scale(uint64_t step, float beta1, float beta2, float n_sma_threshold, float* step_size,
                                    int* use_denom) {
    float t = (float)step;
    float beta2_t = powf(beta2, t);
    float n_sma_max = 2.0f / (1.0f - beta2) - 1.0f;
    float n_sma = n_sma_max - 2.0f * t * beta2_t / (1.0f - beta2_t);
    float bc1 = 1.0f - powf(beta1, t);
    *use_denom = n_sma > n_sma_threshold;
    if (*use_denom) {
        float p1 = (n_sma - 4.0f) / (n_sma_max - 4.0f);
        float p2 = (n_sma - 2.0f) / n_sma;
        float p3 = n_sma_max / (n_sma_max - 2.0f);
        *step_size = sqrtf(p1 * p2 * p3) / bc1;
    } else {
        *step_size = 1.0f / bc1;
    }
}

static float clip_w(float w, float lo, float hi) {
    if (lo == -FLT_MAX && hi == FLT_MAX) return w;
    return fminf(fmaxf(w, lo), hi);
}

/* One Ranger step over a parameter group: RAdam (cu:476-505) with gradient
 * reset, then Lookahead every k steps (cu:686-728, lib.rs:9345-9348). */
EXPORT void oracle_ranger_update(int64_t len, float gradient_factor, float learning_rate, float step_size,
                                 int use_denom, float decay, float beta1, float beta2, float epsilon,
                                 float min_weight, float max_weight, int do_lookahead, float lookahead_alpha,
                                 int clip_after_lookahead, float* grads, float* weights, float* momentum,
                                 float* velocity, float* slow) {
    float rate = learning_rate * step_size;
    float la_lo = clip_after_lookahead ? min_weight : -FLT_MAX;
    float la_hi = clip_after_lookahead ? max_weight : FLT_MAX;
    for (int64_t i = 0; i < len; ++i) {
        float g = gradient_factor * grads[i];
        float w = weights[i] * (1.0f - decay * rate);
        float m = beta1 * momentum[i] + (1.0f - beta1) * g;
        float v = beta2 * velocity[i] + (1.0f - beta2) * g * g;
        float u = m;
        if (use_denom) u /= sqrtf(v) + epsilon;
        w -= rate * u;
        w = clip_w(w, min_weight, max_weight);
        if (do_lookahead) {
            w = clip_w(lookahead_alpha * w + (1.0f - lookahead_alpha) * slow[i], la_lo, la_hi);
            slow[i] = w;
        }
        grads[i] = 0.0f;
        weights[i] = w;
        momentum[i] = m;
        velocity[i] = v;
    }
}

/* KPPT scalar-table forward (cu:8970-9004). */
EXPORT void oracle_kppt_forward(int64_t input_size, int64_t batch, int64_t max_active, const int* stm,
                                const int* nstm, const float* table_w, const float* table_b, const float* outw,
                                const float* outb, float* stm_eval, float* nstm_eval, float* output) {
    for (int64_t b = 0; b < batch; ++b) {
        double s = table_b[0], n = table_b[0];
        for (int64_t k = 0; k < max_active; ++k) {
            int fs = stm[b * max_active + k], fn = nstm[b * max_active + k];
            if (fs >= 0 && fs < input_size) s += table_w[fs];
            if (fn >= 0 && fn < input_size) n += table_w[fn];
        }
        stm_eval[b] = (float)s;
        nstm_eval[b] = (float)n;
        output[b] = outw[0] * stm_eval[b] + outw[1] * nstm_eval[b] + outb[0];
    }
}

/* KPPT backward (cu:9006-9050); table gradient is zero-filled first like the
 * reference launcher (cu:9096-9102), accumulated in double per entry by the
 * caller-provided double table. */
EXPORT void oracle_kppt_backward(int64_t input_size, int64_t batch, int64_t max_active, const int* stm,
                                 const int* nstm, const float* stm_eval, const float* nstm_eval, const float* outw,
                                 const float* mog, double* table_grad_acc, float* table_w_g, float* table_b_g,
                                 float* outw_g, float* outb_g) {
    double w0 = 0.0, w1 = 0.0, ob = 0.0, tb = 0.0;
    for (int64_t i = 0; i < input_size; ++i) table_grad_acc[i] = 0.0;
    for (int64_t b = 0; b < batch; ++b) {
        float g = mog[b];
        w0 += (double)g * stm_eval[b];
        w1 += (double)g * nstm_eval[b];
        ob += g;
        float sg = g * outw[0], ng = g * outw[1];
        tb += (double)(sg + ng);
        for (int64_t k = 0; k < max_active; ++k) {
            int fs = stm[b * max_active + k], fn = nstm[b * max_active + k];
            if (fs >= 0 && fs < input_size) table_grad_acc[fs] += sg;
            if (fn >= 0 && fn < input_size) table_grad_acc[fn] += ng;
        }
    }
    for (int64_t i = 0; i < input_size; ++i) table_w_g[i] = (float)table_grad_acc[i];
    table_b_g[0] = (float)tb;
    outw_g[0] = (float)w0;
    outw_g[1] = (float)w1;
    outb_g[0] = (float)ob;
}
