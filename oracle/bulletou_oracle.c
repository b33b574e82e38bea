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
#include <stdlib.h>
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

/* ------------------------------------------------------------------ SFNN
 * SFNN LayerStack network.  Follows the CPU statement
 * crates/bulletou_lib/src/value/fast_sfnn.rs:325-452 (forward, factorized
 * virtual feature) and the reference test oracle tiny_sfnn_forward_cpu /
 * tiny_sfnn_backward_cpu (crates/cuda_cpp/src/lib.rs:14252-14710, shared
 * L1/L2/L3 factors), with the factor coefficients of the GPU kernels
 * (ft alpha: cu:1445-1456 fold; shared alpha: cu:2297-2322, 2449-2600).
 * The FT row sum uses the folded row w[f] + alpha * w[virtual] like the
 * reference's training forward; dense dots and every batch reduction
 * accumulate in double.
 * Weight pointers, in order: l0w l0b l1w l1b l1fw l1fb l2w l2b l2fw l2fb l3w
 * l3b l3fw l3fb (shared factors may be NULL). */
#define SFNN_PIECES 1629

typedef struct {
    int64_t input_size, width, hidden, skip, l2, stacks, batch, max_active;
    float ft_alpha, shared_alpha;
    int64_t base, n_features, l1_out, l2_in;
} sfnn_dims;

static sfnn_dims sfnn_make_dims(const int64_t* shape, const float* alphas) {
    sfnn_dims d;
    d.input_size = shape[0];
    d.width = shape[1];
    d.hidden = shape[2];
    d.skip = shape[3];
    d.l2 = shape[4];
    d.stacks = shape[5];
    d.batch = shape[6];
    d.max_active = shape[7];
    d.ft_alpha = alphas[0];
    d.shared_alpha = alphas[1];
    /* cu:1180-1184: the two HalfKA bases + 1629 virtual piece rows */
    d.base = (d.input_size == 131949 + SFNN_PIECES) ? 131949 : (d.input_size == 73305 + SFNN_PIECES) ? 73305 : 0;
    d.n_features = d.base ? d.base : d.input_size;
    d.l1_out = d.hidden + (d.skip ? 1 : 0);
    d.l2_in = 2 * d.hidden;
    return d;
}

static void sfnn_ft_view(const sfnn_dims* d, const int* idx, const float* l0w, const float* l0b, float* x) {
    for (int64_t j = 0; j < d->width; ++j) x[j] = l0b[j];
    for (int64_t s = 0; s < d->max_active; ++s) {
        int f = idx[s];
        if (f < 0 || (int64_t)f >= d->n_features) continue;
        const float* row = l0w + (int64_t)f * d->width;
        if (d->base) {
            const float* v = l0w + (d->base + (int64_t)f % SFNN_PIECES) * d->width;
            for (int64_t j = 0; j < d->width; ++j) x[j] += fmaf(d->ft_alpha, v[j], row[j]);
        } else {
            for (int64_t j = 0; j < d->width; ++j) x[j] += row[j];
        }
    }
    for (int64_t j = 0; j < d->width; ++j) x[j] = crelu(x[j]);
}

static float sfnn_w1(const sfnn_dims* d, const float* const* w, int64_t s, int64_t o, int64_t i) {
    float v = w[2][(s * d->l1_out + o) * d->width + i];
    if (w[4]) v = fmaf(d->shared_alpha, w[4][i * d->l1_out + o], v);
    return v;
}

static float sfnn_w2(const sfnn_dims* d, const float* const* w, int64_t s, int64_t o, int64_t i) {
    float v = w[6][(s * d->l2 + o) * d->l2_in + i];
    if (w[8]) v = fmaf(d->shared_alpha, w[8][o * d->l2_in + i], v);
    return v;
}

static float sfnn_w3(const sfnn_dims* d, const float* const* w, int64_t s, int64_t o) {
    float v = w[10][s * d->l2 + o];
    if (w[12]) v = fmaf(d->shared_alpha, w[12][o], v);
    return v;
}

/* ------------------------------------------------------------------ SFNN QAT
 * Quantisation-aware training modes of the reference runner (bitmask):
 *   1 L1  fake-quantised folded L1 weights / bias (sfnn_qat_l1; cu:11514-11590,
 *         sfnn_build_quantized_proxy_stacked_{weights,bias}_kernel cu:1735-1990)
 *   2 FT  fake-quantised FT weights / bias, virtual rows folded in and zeroed
 *         (layer QAT, layer_qat.rs:832-880, layer_qat_ft_fold_kernel cu:9302)
 *   4 L2, 8 L3  fake-quantised L2 / L3 weights (scale 64) and biases (8128)
 *         (layer_qat_vector_kernel cu:9294)
 * L1 + L2 + L3 together select the dense integer QAT (layer_qat.rs:977-991):
 * FT output floored to the 1/127 lattice (or the engine's integer FT when FT
 * QAT is on, dense_qat_exact_ft_kernel cu:6344), integer L1 / L2 / L3 with
 * the master L2 / L3 biases rounded to 8128 (cu:6282-6320), and continuous
 * activation STEs in the backward (dense_qat_l2_ste_kernel cu:6322,
 * sfnn_l2_input_backward_kernel cu:3709-3770).  Gradients always reach the
 * f32 masters through an identity STE. */
#define SFNN_QAT_L1 1
#define SFNN_QAT_FT 2
#define SFNN_QAT_L2 4
#define SFNN_QAT_L3 8

/* sfnn_quantize_dequant_clamped, cu:1644-1666 (training form): f32 product
 * rounded half away from zero; ties and |x| >= 2^22 redone in double. */
static float qat_qd(float v, float scale, float lo, float hi) {
    const float scaled = v * scale;
    float q = roundf(scaled);
    if (fabsf(scaled) >= 4194304.0f || fabsf(scaled - truncf(scaled)) == 0.5f)
        q = (float)round((double)v * (double)scale);
    q = fminf(fmaxf(q, lo), hi);
    return q / scale;
}

/* a + alpha * b with two roundings (the QAT folds use __fadd_rn/__fmul_rn). */
static float fold_nf(float a, float alpha, float b) {
    const float t = alpha * b;
    return a + t;
}

static int32_t round_bias_8128(float v) {
    double q = round((double)v * 8128.0);
    q = fmin(2147483647.0, fmax(-2147483648.0, q));
    return (int32_t)q;
}

/* floor(clamp(x, 0, 1) * 127), exact (dense_qat_lattice_integer, cu:5998). */
static int qat_lattice(float x) {
    const float c = fminf(1.0f, fmaxf(0.0f, x));
    return (int)floor((double)c * 127.0);
}

typedef struct {
    int l1, ft, l2, l3, dense;
    float *l0w, *l0b;           /* FT copies (ft): [input_size][W], [W] */
    float *w1, *b1;             /* Q(folded L1) [S][O][W], [S][O] (l1) */
    float *b1_master;           /* folded master L1 bias [S][O] (l1) */
    int32_t* b1_int;            /* round(folded master * 8128) [S][O] (l1) */
    float *w2, *b2, *w3, *b3;   /* Q copies (l2, l3) */
} sfnn_qat;

static void sfnn_qat_prepare(const sfnn_dims* d, int mode, const float* const* w, sfnn_qat* q) {
    memset(q, 0, sizeof(*q));
    q->l1 = (mode & SFNN_QAT_L1) != 0;
    q->ft = (mode & SFNN_QAT_FT) != 0;
    q->l2 = (mode & SFNN_QAT_L2) != 0;
    q->l3 = (mode & SFNN_QAT_L3) != 0;
    q->dense = q->l1 && q->l2 && q->l3;
    const int64_t W = d->width, O = d->l1_out, S = d->stacks, L2 = d->l2, I2 = d->l2_in;
    if (q->ft) {
        q->l0w = (float*)malloc(sizeof(float) * (size_t)(d->input_size * W));
        q->l0b = (float*)malloc(sizeof(float) * (size_t)W);
        for (int64_t f = 0; f < d->input_size; ++f)
            for (int64_t j = 0; j < W; ++j) {
                float v = 0.0f;
                if (!d->base || f < d->base) {
                    v = w[0][f * W + j];
                    if (d->base) v = fold_nf(v, d->ft_alpha, w[0][(d->base + f % SFNN_PIECES) * W + j]);
                    v = qat_qd(v, 127.0f, -32768.0f, 32767.0f);
                }
                q->l0w[f * W + j] = v;
            }
        for (int64_t j = 0; j < W; ++j) q->l0b[j] = qat_qd(w[1][j], 127.0f, -32768.0f, 32767.0f);
    }
    if (q->l1) {
        q->w1 = (float*)malloc(sizeof(float) * (size_t)(S * O * W));
        q->b1 = (float*)malloc(sizeof(float) * (size_t)(S * O));
        q->b1_master = (float*)malloc(sizeof(float) * (size_t)(S * O));
        q->b1_int = (int32_t*)malloc(sizeof(int32_t) * (size_t)(S * O));
        for (int64_t s = 0; s < S; ++s)
            for (int64_t o = 0; o < O; ++o) {
                for (int64_t i = 0; i < W; ++i) {
                    float v = w[2][(s * O + o) * W + i];
                    if (w[4]) v = fold_nf(v, d->shared_alpha, w[4][i * O + o]);
                    q->w1[(s * O + o) * W + i] = qat_qd(v, 64.0f, -128.0f, 127.0f);
                }
                float b = w[3][s * O + o];
                if (w[5]) b = fold_nf(b, d->shared_alpha, w[5][o]);
                q->b1_master[s * O + o] = b;
                q->b1_int[s * O + o] = round_bias_8128(b);
                q->b1[s * O + o] = qat_qd(b, 8128.0f, -2147483648.0f, 2147483647.0f);
            }
    }
    if (q->l2) {
        q->w2 = (float*)malloc(sizeof(float) * (size_t)(S * L2 * I2));
        q->b2 = (float*)malloc(sizeof(float) * (size_t)(S * L2));
        for (int64_t i = 0; i < S * L2 * I2; ++i) q->w2[i] = qat_qd(w[6][i], 64.0f, -128.0f, 127.0f);
        for (int64_t i = 0; i < S * L2; ++i) q->b2[i] = qat_qd(w[7][i], 8128.0f, -2147483648.0f, 2147483647.0f);
    }
    if (q->l3) {
        q->w3 = (float*)malloc(sizeof(float) * (size_t)(S * L2));
        q->b3 = (float*)malloc(sizeof(float) * (size_t)S);
        for (int64_t i = 0; i < S * L2; ++i) q->w3[i] = qat_qd(w[10][i], 64.0f, -128.0f, 127.0f);
        for (int64_t i = 0; i < S; ++i) q->b3[i] = qat_qd(w[11][i], 8128.0f, -2147483648.0f, 2147483647.0f);
    }
}

static void sfnn_qat_free(sfnn_qat* q) {
    free(q->l0w); free(q->l0b); free(q->w1); free(q->b1); free(q->b1_master); free(q->b1_int);
    free(q->w2); free(q->b2); free(q->w3); free(q->b3);
}

/* Weights the forward / backward use under QAT. */
static float qat_w1(const sfnn_dims* d, const sfnn_qat* q, const float* const* w, int64_t s, int64_t o, int64_t i) {
    return q->l1 ? q->w1[(s * d->l1_out + o) * d->width + i] : sfnn_w1(d, w, s, o, i);
}
static float qat_w2(const sfnn_dims* d, const sfnn_qat* q, const float* const* w, int64_t s, int64_t o, int64_t i) {
    return q->l2 ? q->w2[(s * d->l2 + o) * d->l2_in + i] : sfnn_w2(d, w, s, o, i);
}
static float qat_w3(const sfnn_dims* d, const sfnn_qat* q, const float* const* w, int64_t s, int64_t o) {
    return q->l3 ? q->w3[s * d->l2 + o] : sfnn_w3(d, w, s, o);
}

/* Engine integer FT of one view from FT QAT weights (q / 127 values):
 * doubled i16 sums with wrap, clamp [0, 254], (s0 * s1) >> 9 (cu:6344-6390). */
static void qat_exact_ft(const sfnn_dims* d, const sfnn_qat* q, const int* idx, int* pair) {
    const int64_t W = d->width, half = W / 2;
    for (int64_t j = 0; j < half; ++j) {
        int32_t s0 = 2 * (int32_t)rintf(q->l0b[j] * 127.0f), s1 = 2 * (int32_t)rintf(q->l0b[half + j] * 127.0f);
        for (int64_t k = 0; k < d->max_active; ++k) {
            int f = idx[k];
            if (f < 0 || (int64_t)f >= d->n_features) continue;
            s0 += 2 * (int32_t)rintf(q->l0w[(int64_t)f * W + j] * 127.0f);
            s1 += 2 * (int32_t)rintf(q->l0w[(int64_t)f * W + half + j] * 127.0f);
        }
        int32_t x0 = (int32_t)(int16_t)s0, x1 = (int32_t)(int16_t)s1;
        x0 = x0 < 0 ? 0 : (x0 > 254 ? 254 : x0);
        x1 = x1 < 0 ? 0 : (x1 > 254 ? 254 : x1);
        pair[j] = (x0 * x1) >> 9;
    }
}

/* shape: input_size, ft_size, l1_hidden, l1_skip, l2_size, num_stacks, batch, max_active;
 * alphas: ft, shared; qat: SFNN_QAT_* bitmask.  Outputs (row-major per
 * sample): stm_l0, nstm_l0, combined [B][W], l1 [B][l1_out], l2_input [B][2H],
 * l2 [B][L2], output [B]; under dense QAT also l1_raw [B][l1_out] and l2_raw
 * [B][L2] (the integer sums; may be NULL otherwise). */
EXPORT void oracle_sfnn_forward_qat(const int64_t* shape, const float* alphas, int qat, const int* stm,
                                    const int* nstm, const int* buckets, const float* const* w, float* stm_l0,
                                    float* nstm_l0, float* combined, float* l1, float* l2_input, float* l2,
                                    float* output, int32_t* l1_raw, int32_t* l2_raw) {
    sfnn_dims d = sfnn_make_dims(shape, alphas);
    sfnn_qat q;
    sfnn_qat_prepare(&d, qat, w, &q);
    const float* ftw = q.ft ? q.l0w : w[0];
    const float* ftb = q.ft ? q.l0b : w[1];
    const float scale = 127.0f / 128.0f;
    const int64_t W = d.width, half = W / 2, O = d.l1_out;
    int* pair = (int*)malloc(sizeof(int) * (size_t)half);
    int* in_int = (int*)malloc(sizeof(int) * (size_t)d.l2_in);
    for (int64_t b = 0; b < d.batch; ++b) {
        float* xs = stm_l0 + b * W;
        float* xn = nstm_l0 + b * W;
        sfnn_ft_view(&d, stm + b * d.max_active, ftw, ftb, xs);
        sfnn_ft_view(&d, nstm + b * d.max_active, ftw, ftb, xn);
        float* c = combined + b * W;
        for (int64_t j = 0; j < half; ++j) {
            c[j] = xs[j] * xs[j + half] * scale;
            c[half + j] = xn[j] * xn[j + half] * scale;
        }
        if (q.dense) {
            if (q.ft) {
                for (int v = 0; v < 2; ++v) {
                    qat_exact_ft(&d, &q, (v ? nstm : stm) + b * d.max_active, pair);
                    for (int64_t j = 0; j < half; ++j) c[v * half + j] = (float)pair[j] / 127.0f;
                }
            } else {
                for (int64_t j = 0; j < W; ++j) c[j] = (float)qat_lattice(c[j]) / 127.0f;
            }
        }
        float* l1r = l1 + b * O;
        float* in = l2_input + b * d.l2_in;
        float* l2r = l2 + b * d.l2;
        int s = buckets[b];
        if (s < 0 || s >= d.stacks) {  /* cu:2250-2256: invalid bucket -> zeros */
            for (int64_t o = 0; o < O; ++o) l1r[o] = 0.0f;
            for (int64_t i = 0; i < d.l2_in; ++i) in[i] = 0.0f;
            for (int64_t o = 0; o < d.l2; ++o) l2r[o] = 0.0f;
            if (l1_raw) for (int64_t o = 0; o < O; ++o) l1_raw[b * O + o] = 0;
            if (l2_raw) for (int64_t o = 0; o < d.l2; ++o) l2_raw[b * d.l2 + o] = 0;
            output[b] = 0.0f;
            continue;
        }
        if (q.dense) {
            /* integer L1 / L2 / L3 (cu:6223-6320) */
            int32_t raw1[64];
            for (int64_t o = 0; o < O; ++o) {
                int64_t acc = q.b1_int[s * O + o];
                for (int64_t i = 0; i < W; ++i)
                    acc += (int64_t)rintf(c[i] * 127.0f) * (int64_t)rintf(qat_w1(&d, &q, w, s, o, i) * 64.0f);
                raw1[o] = (int32_t)acc;
                l1r[o] = (float)((double)raw1[o] / 8128.0);
                if (l1_raw) l1_raw[b * O + o] = raw1[o];
            }
            for (int64_t i = 0; i < d.hidden; ++i) {
                const int64_t x = raw1[i];
                int64_t sq = (x * x) >> 19;
                if (sq > 127) sq = 127;
                int32_t lin = raw1[i] >> 6;
                lin = lin < 0 ? 0 : (lin > 127 ? 127 : lin);
                in[i] = (float)sq / 127.0f;
                in[d.hidden + i] = (float)lin / 127.0f;
                in_int[i] = (int)sq;
                in_int[d.hidden + i] = lin;
            }
            int64_t out = round_bias_8128(w[11][s]);
            for (int64_t o = 0; o < d.l2; ++o) {
                int64_t acc = round_bias_8128(w[7][s * d.l2 + o]);
                for (int64_t i = 0; i < d.l2_in; ++i)
                    acc += (int64_t)in_int[i] * (int64_t)rintf(qat_w2(&d, &q, w, s, o, i) * 64.0f);
                const int32_t r2 = (int32_t)acc;
                if (l2_raw) l2_raw[b * d.l2 + o] = r2;
                int32_t v = r2 >> 6;
                v = v < 0 ? 0 : (v > 127 ? 127 : v);
                l2r[o] = (float)v / 127.0f;
                out += (int64_t)v * (int64_t)rintf(qat_w3(&d, &q, w, s, o) * 64.0f);
            }
            if (d.skip) out += raw1[d.hidden];
            output[b] = (float)((double)(int32_t)out / 8128.0);
            continue;
        }
        for (int64_t o = 0; o < O; ++o) {
            double acc = 0.0;
            for (int64_t i = 0; i < W; ++i) acc += (double)c[i] * qat_w1(&d, &q, w, s, o, i);
            float r;
            if (q.l1) {
                r = (float)acc + q.b1[s * O + o];
            } else {
                r = (float)acc + w[3][s * O + o];
                if (w[5]) r = fmaf(d.shared_alpha, w[5][o], r);
            }
            l1r[o] = r;
        }
        for (int64_t i = 0; i < d.hidden; ++i) {
            float a = fabsf(l1r[i]);
            in[i] = crelu(a * a * scale);            /* SqrCReLU, cu:2428-2447 */
            in[d.hidden + i] = crelu(l1r[i]);        /* CReLU */
        }
        for (int64_t o = 0; o < d.l2; ++o) {
            float bias;
            if (q.l2) {
                bias = q.b2[s * d.l2 + o];
            } else {
                bias = w[7][s * d.l2 + o];
                if (w[9]) bias = fmaf(d.shared_alpha, w[9][o], bias);
            }
            double acc = bias;
            for (int64_t i = 0; i < d.l2_in; ++i) acc += (double)in[i] * qat_w2(&d, &q, w, s, o, i);
            l2r[o] = crelu((float)acc);
        }
        float b3;
        if (q.l3) {
            b3 = q.b3[s];
        } else {
            b3 = w[11][s];
            if (w[13]) b3 = fmaf(d.shared_alpha, w[13][0], b3);
        }
        double out = b3;
        for (int64_t o = 0; o < d.l2; ++o) out += (double)l2r[o] * qat_w3(&d, &q, w, s, o);
        output[b] = (float)out + (d.skip ? l1r[d.hidden] : 0.0f);
    }
    free(pair);
    free(in_int);
    sfnn_qat_free(&q);
}

EXPORT void oracle_sfnn_forward(const int64_t* shape, const float* alphas, const int* stm, const int* nstm,
                                const int* buckets, const float* const* w, float* stm_l0, float* nstm_l0,
                                float* combined, float* l1, float* l2_input, float* l2, float* output) {
    oracle_sfnn_forward_qat(shape, alphas, 0, stm, nstm, buckets, w, stm_l0, nstm_l0, combined, l1, l2_input, l2,
                            output, 0, 0);
}

/* Backward of oracle_sfnn_forward for output gradients mog (lib.rs:14516-14710
 * with the alphas of the GPU kernels).  grads (same order as w, NULL where w
 * is NULL) are overwritten; l0w's gradient includes the virtual rows
 * (alpha * sum of the base rows' gradients, cu:4950-4985).  l1_gradients
 * [B][l1_out] and combined_gradients [B][W] are written too. */
EXPORT void oracle_sfnn_backward_qat(const int64_t* shape, const float* alphas, int qat, const int* stm,
                                     const int* nstm, const int* buckets, const float* const* w,
                                     const float* stm_l0, const float* nstm_l0, const float* combined,
                                     const float* l1, const float* l2_input, const float* l2, const int32_t* l1_raw,
                                     const int32_t* l2_raw, const float* mog, double* acc_l0w, float* const* grads,
                                     float* l1_gradients, float* combined_gradients) {
    sfnn_dims d = sfnn_make_dims(shape, alphas);
    sfnn_qat q;
    sfnn_qat_prepare(&d, qat, w, &q);
    const float scale = 127.0f / 128.0f;
    const int64_t W = d.width, half = W / 2, O = d.l1_out, L2 = d.l2, I2 = d.l2_in, S = d.stacks;
    const int64_t lens[14] = {d.input_size * W, W, S * O * W, S * O, W * O, O, S * L2 * I2, S * L2, L2 * I2, L2,
                              S * L2, S, L2, 1};
    double* acc[14];
    double* pool = 0;
    int64_t total = 0;
    for (int k = 1; k < 14; ++k) total += lens[k];
    pool = (double*)calloc((size_t)total, sizeof(double));
    int64_t off = 0;
    acc[0] = acc_l0w;
    for (int k = 1; k < 14; ++k) {
        acc[k] = pool + off;
        off += lens[k];
    }
    for (int64_t i = 0; i < lens[0]; ++i) acc_l0w[i] = 0.0;
    float* g2 = (float*)malloc(sizeof(float) * (size_t)L2);
    float* gin = (float*)malloc(sizeof(float) * (size_t)I2);
    float* pre_s = (float*)malloc(sizeof(float) * (size_t)W);
    float* pre_n = (float*)malloc(sizeof(float) * (size_t)W);
    for (int64_t b = 0; b < d.batch; ++b) {
        const float gout = mog[b];
        float* g1 = l1_gradients + b * O;
        float* dc = combined_gradients + b * W;
        for (int64_t o = 0; o < O; ++o) g1[o] = 0.0f;
        for (int64_t i = 0; i < W; ++i) dc[i] = 0.0f;
        if (d.skip) g1[d.hidden] = gout;  /* PSQT skip, cu:3433-3437 */
        int s = buckets[b];
        if (s < 0 || s >= S) continue;
        const float* l2r = l2 + b * L2;
        const float* in = l2_input + b * I2;
        const float* l1r = l1 + b * O;
        /* L3 (cu:3324-3480) */
        acc[11][s] += gout;
        if (w[13]) acc[13][0] += (double)d.shared_alpha * gout;
        for (int64_t o = 0; o < L2; ++o) {
            acc[10][s * L2 + o] += (double)gout * l2r[o];
            if (w[12]) acc[12][o] += (double)d.shared_alpha * gout * l2r[o];
            const float g = gout * qat_w3(&d, &q, w, s, o);
            if (q.dense) {
                /* continuous STE of the integer L2 CReLU (cu:6322-6342) */
                const int32_t x = l2_raw[b * L2 + o];
                float gg = g;
                if (x < 0 || x > 8128) {
                    gg = 0.0f;
                } else if (x == 0 || x == 8128) {
                    const double bias = fmin(2147483647.0, fmax(-2147483648.0, (double)w[7][s * L2 + o] * 8128.0));
                    const double fraction = bias - round(bias);
                    if ((x == 0 && fraction <= 0.0) || (x == 8128 && fraction >= 0.0)) gg = 0.0f;
                }
                g2[o] = gg;
            } else {
                g2[o] = crelu_grad(l2r[o], g);
            }
        }
        /* L2 (cu:3489-3700) */
        for (int64_t i = 0; i < I2; ++i) gin[i] = 0.0f;
        for (int64_t o = 0; o < L2; ++o) {
            acc[7][s * L2 + o] += g2[o];
            if (w[9]) acc[9][o] += (double)d.shared_alpha * g2[o];
            for (int64_t i = 0; i < I2; ++i) {
                acc[6][(s * L2 + o) * I2 + i] += (double)g2[o] * in[i];
                if (w[8]) acc[8][o * I2 + i] += (double)d.shared_alpha * g2[o] * in[i];
                gin[i] += g2[o] * qat_w2(&d, &q, w, s, o, i);
            }
        }
        /* L2 input (cu:3709-3770) */
        for (int64_t i = 0; i < d.hidden; ++i) {
            float v = l1r[i];
            if (q.dense) {
                /* STE from the pre-rounding L1 value: raw / 8128 plus the
                 * rounded-off fraction of the master bias. */
                const float master = q.b1_master[s * O + i];
                const int32_t qi = q.b1_int[s * O + i];
                float frac;
                if (qi >= -16777216 && qi <= 16777216) {
                    frac = fmaf(master, 8128.0f, -(float)qi);
                } else {
                    const double scaled = fmin(2147483647.0, fmax(-2147483648.0, (double)master * 8128.0));
                    frac = (float)(scaled - (double)qi);
                }
                const float ste = fmaf(frac, 1.0f / 8128.0f, v);
                const float cs = fabsf(ste) * fabsf(ste) * scale;
                int sq_on = cs > 0.0f && cs < 1.0f;
                int lin_on = ste > 0.0f && ste < 1.0f;
                const int32_t raw = l1_raw[b * O + i];
                if (raw == 0) lin_on = frac > 0.0f;
                else if (raw == 8128) lin_on = frac < 0.0f;
                if (raw == 8160 || raw == -8160) {
                    const double x = (double)raw + (double)frac;
                    sq_on = x * x * 127.0 < 128.0 * 8128.0 * 8128.0;
                }
                const float sg = sq_on ? gin[i] * (2.0f * ste * scale) : 0.0f;
                const float lg = lin_on ? gin[d.hidden + i] : 0.0f;
                g1[i] = sg + lg;
                continue;
            }
            float sq = crelu_grad(in[i], gin[i] * (2.0f * v * scale));
            float lin = crelu_grad(in[d.hidden + i], gin[d.hidden + i]);
            g1[i] = sq + lin;
        }
        /* L1 (cu:3778-4100) */
        for (int64_t o = 0; o < O; ++o) {
            acc[3][s * O + o] += g1[o];
            if (w[5]) acc[5][o] += (double)d.shared_alpha * g1[o];
            for (int64_t i = 0; i < W; ++i) {
                acc[2][(s * O + o) * W + i] += (double)g1[o] * combined[b * W + i];
                if (w[4]) acc[4][i * O + o] += (double)d.shared_alpha * g1[o] * combined[b * W + i];
            }
        }
        for (int64_t i = 0; i < W; ++i) {
            double t = 0.0;
            for (int64_t o = 0; o < O; ++o) t += (double)g1[o] * qat_w1(&d, &q, w, s, o, i);
            dc[i] = (float)t;
        }
        /* pairwise + ClippedReLU (cu:4376-4440) */
        for (int v = 0; v < 2; ++v) {
            const float* x = (v ? nstm_l0 : stm_l0) + b * W;
            float* pre = v ? pre_n : pre_s;
            for (int64_t j = 0; j < half; ++j) {
                float pg = dc[v * half + j] * scale;
                pre[j] = crelu_grad(x[j], pg * x[j + half]);
                pre[j + half] = crelu_grad(x[j + half], pg * x[j]);
            }
            for (int64_t j = 0; j < W; ++j) acc[1][j] += pre[j];
            const int* idx = (v ? nstm : stm) + b * d.max_active;
            for (int64_t k = 0; k < d.max_active; ++k) {
                int f = idx[k];
                if (f < 0 || (int64_t)f >= d.n_features) continue;
                double* row = acc_l0w + (int64_t)f * W;
                for (int64_t j = 0; j < W; ++j) row[j] += pre[j];
            }
        }
    }
    if (d.base) {
        for (int64_t p = 0; p < SFNN_PIECES; ++p) {
            double* vrow = acc_l0w + (d.base + p) * W;
            for (int64_t j = 0; j < W; ++j) vrow[j] = 0.0;
            for (int64_t f = p; f < d.base; f += SFNN_PIECES)
                for (int64_t j = 0; j < W; ++j) vrow[j] += acc_l0w[f * W + j];
            for (int64_t j = 0; j < W; ++j) vrow[j] *= d.ft_alpha;
        }
    }
    for (int k = 0; k < 14; ++k) {
        if (!grads[k]) continue;
        for (int64_t i = 0; i < lens[k]; ++i) grads[k][i] = (float)acc[k][i];
    }
    sfnn_qat_free(&q);
    free(pool);
    free(g2);
    free(gin);
    free(pre_s);
    free(pre_n);
}

EXPORT void oracle_sfnn_backward(const int64_t* shape, const float* alphas, const int* stm, const int* nstm,
                                 const int* buckets, const float* const* w, const float* stm_l0, const float* nstm_l0,
                                 const float* combined, const float* l1, const float* l2_input, const float* l2,
                                 const float* mog, double* acc_l0w, float* const* grads, float* l1_gradients,
                                 float* combined_gradients) {
    oracle_sfnn_backward_qat(shape, alphas, 0, stm, nstm, buckets, w, stm_l0, nstm_l0, combined, l1, l2_input, l2, 0,
                             0, mog, acc_l0w, grads, l1_gradients, combined_gradients);
}

/* ------------------------------------------------------------------ quantised SFNN
 * Export quantisation of a trained SFNN (examples/bulletou.rs:10050-10300,
 * quantized_sfnn_weights_from_cuda_cpp_readback): fold the FT factorizer
 * (bulletou.rs:26417-26444, f32 `w + alpha * w_virtual`, no fused multiply-add)
 * and the shared L1 / L2 / L3 factors (bulletou.rs:21339-21520,
 * `w += alpha * shared`), then round(x * scale) half away from zero in double
 * and clamp (bulletou.rs:26481-26493): FT i16 at 127, dense i8 at 64, dense
 * biases i32 at 127 * 64.  Dense rows are padded to a multiple of 32 inputs
 * with zeros (nnue_save_sfnn1536.rs layout). */
static int64_t pad32(int64_t n) { return (n + 31) / 32 * 32; }

static int16_t q_i16(float v, float s) {
    double q = round((double)v * (double)s);
    if (q < -32768.0) q = -32768.0;
    if (q > 32767.0) q = 32767.0;
    return (int16_t)q;
}
static int8_t q_i8(float v, float s) {
    double q = round((double)v * (double)s);
    if (q < -128.0) q = -128.0;
    if (q > 127.0) q = 127.0;
    return (int8_t)q;
}
static int32_t q_i32(float v, float s) {
    double q = round((double)v * (double)s);
    if (q < -2147483648.0) q = -2147483648.0;
    if (q > 2147483647.0) q = 2147483647.0;
    return (int32_t)q;
}

EXPORT void oracle_sfnn_quantize(const int64_t* shape, const float* alphas, const float* const* w, int16_t* l0w_q,
                                 int16_t* l0b_q, int8_t* l1w_q, int32_t* l1b_q, int8_t* l2w_q, int32_t* l2b_q,
                                 int8_t* l3w_q, int32_t* l3b_q) {
    sfnn_dims d = sfnn_make_dims(shape, alphas);
    const int64_t W = d.width, O = d.l1_out, L2 = d.l2, I2 = d.l2_in, S = d.stacks;
    const int64_t rows = d.base ? d.base : d.input_size;
    const float a = d.shared_alpha;
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t j = 0; j < W; ++j) {
            float v = w[0][r * W + j];
            if (d.base) {
                float t = d.ft_alpha * w[0][(d.base + r % SFNN_PIECES) * W + j];
                v = v + t;
            }
            l0w_q[r * W + j] = q_i16(v, 127.0f);
        }
    for (int64_t j = 0; j < W; ++j) l0b_q[j] = q_i16(w[1][j], 127.0f);
    const int64_t p1 = pad32(W), p2 = pad32(I2), p3 = pad32(L2);
    for (int64_t s = 0; s < S; ++s) {
        for (int64_t o = 0; o < O; ++o) {
            float b = w[3][s * O + o];
            if (w[5]) { float t = a * w[5][o]; b = b + t; }
            l1b_q[s * O + o] = q_i32(b, 8128.0f);
            for (int64_t i = 0; i < p1; ++i) {
                int8_t q = 0;
                if (i < W) {
                    float v = w[2][(s * O + o) * W + i];
                    if (w[4]) { float t = a * w[4][i * O + o]; v = v + t; }
                    q = q_i8(v, 64.0f);
                }
                l1w_q[(s * O + o) * p1 + i] = q;
            }
        }
        for (int64_t o = 0; o < L2; ++o) {
            float b = w[7][s * L2 + o];
            if (w[9]) { float t = a * w[9][o]; b = b + t; }
            l2b_q[s * L2 + o] = q_i32(b, 8128.0f);
            for (int64_t i = 0; i < p2; ++i) {
                int8_t q = 0;
                if (i < I2) {
                    float v = w[6][(s * L2 + o) * I2 + i];
                    if (w[8]) { float t = a * w[8][o * I2 + i]; v = v + t; }
                    q = q_i8(v, 64.0f);
                }
                l2w_q[(s * L2 + o) * p2 + i] = q;
            }
        }
        float b3 = w[11][s];
        if (w[13]) { float t = a * w[13][0]; b3 = b3 + t; }
        l3b_q[s] = q_i32(b3, 8128.0f);
        for (int64_t i = 0; i < p3; ++i) {
            int8_t q = 0;
            if (i < L2) {
                float v = w[10][s * L2 + i];
                if (w[12]) { float t = a * w[12][i]; v = v + t; }
                q = q_i8(v, 64.0f);
            }
            l3w_q[s * p3 + i] = q;
        }
    }
}

/* Integer SFNN forward of one batch (examples/bulletou.rs:8001-8163,
 * quantized_sfnn_forward_sample): FT sums of doubled i16 weights and bias
 * wrapped to i16, clamped to [0, 254], pair product (s0 << ft_shift) * s1 >> 16
 * (floor or nearest) clamped to 255; L1 = bias + sum u8 * i8; L2 input
 * SqrCReLU min(x^2 >> 19, 127) | CReLU clamp(x >> 6, 0, 127); L2 the same
 * CReLU; raw output = l3 bias + sum + l1 skip.  round: 0 floor, 1 nearest
 * (ft, crelu, sqrcrelu).  Features < 0 are padding; features >= the table's
 * rows and buckets out of range are reported through *error (first sample,
 * or -1 when none) like the reference's errors.  quantised weights as written
 * by oracle_sfnn_quantize; table rows = base (factorized) or input_size. */
static int64_t shr_round(int64_t v, int shift, int nearest) {
    return nearest ? (v + ((int64_t)1 << (shift - 1))) >> shift : v >> shift;
}

EXPORT void oracle_sfnn_integer_forward(const int64_t* shape, const int* stm, const int* nstm, const int* buckets,
                                        const int16_t* l0w_q, const int16_t* l0b_q, const int8_t* l1w_q,
                                        const int32_t* l1b_q, const int8_t* l2w_q, const int32_t* l2b_q,
                                        const int8_t* l3w_q, const int32_t* l3b_q, int ft_shift, int ft_round,
                                        int crelu_round, int sqr_round, int32_t* l1_out, int32_t* raw_out,
                                        int64_t* error) {
    float alphas[2] = {1.0f, 1.0f};
    sfnn_dims d = sfnn_make_dims(shape, alphas);
    const int64_t W = d.width, half = W / 2, O = d.l1_out, L2 = d.l2, I2 = d.l2_in, H = d.hidden;
    const int64_t rows = d.base ? d.base : d.input_size;
    const int64_t p1 = pad32(W), p2 = pad32(I2), p3 = pad32(L2);
    uint8_t* ft = (uint8_t*)malloc((size_t)W);
    int32_t* l1 = (int32_t*)malloc(sizeof(int32_t) * (size_t)O);
    uint8_t* in = (uint8_t*)malloc((size_t)I2 + 1);
    uint8_t* l2 = (uint8_t*)malloc((size_t)L2);
    *error = -1;
    for (int64_t b = 0; b < d.batch; ++b) {
        int s = buckets[b];
        if (s < 0 || s >= d.stacks) {
            if (*error < 0) *error = b;
            raw_out[b] = 0;
            continue;
        }
        for (int v = 0; v < 2; ++v) {
            const int* idx = (v ? nstm : stm) + b * d.max_active;
            for (int64_t j = 0; j < half; ++j) {
                int32_t s0 = (int32_t)l0b_q[j] * 2, s1 = (int32_t)l0b_q[half + j] * 2;
                for (int64_t k = 0; k < d.max_active; ++k) {
                    int f = idx[k];
                    if (f < 0) continue;
                    if ((int64_t)f >= rows) {
                        if (*error < 0) *error = b;
                        continue;
                    }
                    s0 += (int32_t)l0w_q[(int64_t)f * W + j] * 2;
                    s1 += (int32_t)l0w_q[(int64_t)f * W + half + j] * 2;
                }
                int32_t x0 = (int32_t)(int16_t)s0, x1 = (int32_t)(int16_t)s1;
                x0 = x0 < 0 ? 0 : (x0 > 254 ? 254 : x0);
                x1 = x1 < 0 ? 0 : (x1 > 254 ? 254 : x1);
                int64_t p = shr_round(((int64_t)x0 << ft_shift) * x1, 16, ft_round);
                ft[v * half + j] = (uint8_t)(p > 255 ? 255 : (p < 0 ? 0 : p));
            }
        }
        for (int64_t o = 0; o < O; ++o) {
            int32_t sum = l1b_q[s * O + o];
            const int8_t* row = l1w_q + (s * O + o) * p1;
            for (int64_t i = 0; i < W; ++i) sum += (int32_t)ft[i] * (int32_t)row[i];
            l1[o] = sum;
            l1_out[b * O + o] = sum;
        }
        for (int64_t i = 0; i < H; ++i) {
            int64_t sq = shr_round((int64_t)l1[i] * l1[i], 19, sqr_round);
            in[i] = (uint8_t)(sq > 127 ? 127 : sq);
            int32_t c = (crelu_round && l1[i] > 0) ? (l1[i] + 32) >> 6 : l1[i] >> 6;
            in[H + i] = (uint8_t)(c < 0 ? 0 : (c > 127 ? 127 : c));
        }
        for (int64_t o = 0; o < L2; ++o) {
            int32_t sum = l2b_q[s * L2 + o];
            const int8_t* row = l2w_q + (s * L2 + o) * p2;
            for (int64_t i = 0; i < I2; ++i) sum += (int32_t)in[i] * (int32_t)row[i];
            int32_t c = (crelu_round && sum > 0) ? (sum + 32) >> 6 : sum >> 6;
            l2[o] = (uint8_t)(c < 0 ? 0 : (c > 127 ? 127 : c));
        }
        int32_t out = l3b_q[s];
        for (int64_t i = 0; i < L2; ++i) out += (int32_t)l2[i] * (int32_t)l3w_q[s * p3 + i];
        if (d.skip) out += l1[H];
        raw_out[b] = out;
    }
    free(ft);
    free(l1);
    free(in);
    free(l2);
}

/* ------------------------------------------------------------------ quantised HalfKP
 * nn.bin quantisation of the HalfKP 256x2-32-32 net as the reference writes it
 * (write_cuda_cpp_nnue_nn_bin, examples/bulletou.rs:26303-26386; scales
 * qa = 127, qb = 64, L1 bias 127 * 64 = l1_bias_scale(CReLU, false, 127, 64),
 * crates/bulletou_lib/src/value/nnue_save.rs:223-235): the factorized table's
 * virtual rows (first 1548 rows) added to each base row (26390-26413), values
 * round(scale * w) in double, half away from zero; dense weights transposed to
 * output-major and padded to 32 inputs (pad_weights_for_simd, nnue_save.rs:
 * 237-252).  Values outside the integer range are an error there: here they are
 * saturated and counted in *errors.
 * shape: input_size, l1, l2, l3.  Output rows = 125388 when input_size =
 * 125388 + 1548 (factorized), else input_size. */
static int64_t q_round_count(double v, double lo, double hi, int64_t* errors) {
    double q = round(v);
    if (q < lo) { q = lo; ++*errors; }
    if (q > hi) { q = hi; ++*errors; }
    return (int64_t)q;
}

EXPORT void oracle_nnue_quantize(const int64_t* shape, const float* const* w, int16_t* l0w_q, int16_t* l0b_q,
                                 int8_t* l1w_q, int32_t* l1b_q, int8_t* l2w_q, int32_t* l2b_q, int8_t* outw_q,
                                 int32_t* outb_q, int64_t* errors) {
    const int64_t input_size = shape[0], L1 = shape[1], L2 = shape[2], L3 = shape[3];
    const int factorized = input_size == 125388 + 1548;
    const int64_t rows = factorized ? 125388 : input_size;
    *errors = 0;
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t j = 0; j < L1; ++j) {
            float v = factorized ? w[0][(1548 + r) * L1 + j] + w[0][(r % 1548) * L1 + j] : w[0][r * L1 + j];
            l0w_q[r * L1 + j] = (int16_t)q_round_count(127.0 * (double)v, -32768.0, 32767.0, errors);
        }
    for (int64_t j = 0; j < L1; ++j) l0b_q[j] = (int16_t)q_round_count(127.0 * (double)w[1][j], -32768.0, 32767.0, errors);
    const int64_t I1 = 2 * L1, p1 = pad32(I1), p2 = pad32(L2), p3 = pad32(L3);
    for (int64_t o = 0; o < L2; ++o) {
        l1b_q[o] = (int32_t)q_round_count(8128.0 * (double)w[3][o], -2147483648.0, 2147483647.0, errors);
        for (int64_t i = 0; i < p1; ++i)
            l1w_q[o * p1 + i] = i < I1 ? (int8_t)q_round_count(64.0 * (double)w[2][i * L2 + o], -128.0, 127.0, errors) : 0;
    }
    for (int64_t o = 0; o < L3; ++o) {
        l2b_q[o] = (int32_t)q_round_count(8128.0 * (double)w[5][o], -2147483648.0, 2147483647.0, errors);
        for (int64_t i = 0; i < p2; ++i)
            l2w_q[o * p2 + i] = i < L2 ? (int8_t)q_round_count(64.0 * (double)w[4][i * L3 + o], -128.0, 127.0, errors) : 0;
    }
    outb_q[0] = (int32_t)q_round_count(8128.0 * (double)w[7][0], -2147483648.0, 2147483647.0, errors);
    for (int64_t i = 0; i < p3; ++i)
        outw_q[i] = i < L3 ? (int8_t)q_round_count(64.0 * (double)w[6][i], -128.0, 127.0, errors) : 0;
}

/* The engine's integer evaluation of that net (YaneuraOu's halfkp_256x2-32-32
 * NNUE, the engine the reference exports to; not part of the reference tree):
 * per perspective (side to move first) i16 accumulator = bias + sum of rows
 * (i16 wrap), ClippedReLU clamp(acc, 0, 127) -> u8; each affine layer
 * bias + sum u8 * i8 in i32, ClippedReLU clamp(x >> 6, 0, 127); output
 * bias + sum; score = raw / fv_scale (C division, toward zero).  Features
 * outside [0, rows) are skipped and counted in *errors. */
EXPORT void oracle_nnue_integer_forward(const int64_t* shape, int64_t batch, int64_t max_active, const int* stm,
                                        const int* nstm, const int16_t* l0w_q, const int16_t* l0b_q,
                                        const int8_t* l1w_q, const int32_t* l1b_q, const int8_t* l2w_q,
                                        const int32_t* l2b_q, const int8_t* outw_q, const int32_t* outb_q,
                                        int fv_scale, int32_t* raw_out, int32_t* score_out, int64_t* errors) {
    const int64_t input_size = shape[0], L1 = shape[1], L2 = shape[2], L3 = shape[3];
    const int64_t rows = input_size == 125388 + 1548 ? 125388 : input_size;
    const int64_t I1 = 2 * L1, p1 = pad32(I1), p2 = pad32(L2), p3 = pad32(L3);
    uint8_t* x = (uint8_t*)malloc((size_t)I1);
    int32_t* h1 = (int32_t*)malloc(sizeof(int32_t) * (size_t)L2);
    int32_t* h2 = (int32_t*)malloc(sizeof(int32_t) * (size_t)L3);
    *errors = 0;
    for (int64_t b = 0; b < batch; ++b) {
        for (int v = 0; v < 2; ++v) {
            const int* idx = (v ? nstm : stm) + b * max_active;
            for (int64_t j = 0; j < L1; ++j) {
                int32_t acc = l0b_q[j];
                for (int64_t k = 0; k < max_active; ++k) {
                    int f = idx[k];
                    if (f < 0) continue;
                    if ((int64_t)f >= rows) {
                        if (j == 0) ++*errors;
                        continue;
                    }
                    acc += l0w_q[(int64_t)f * L1 + j];
                }
                int32_t a16 = (int32_t)(int16_t)acc;
                x[v * L1 + j] = (uint8_t)(a16 < 0 ? 0 : (a16 > 127 ? 127 : a16));
            }
        }
        for (int64_t o = 0; o < L2; ++o) {
            int32_t s = l1b_q[o];
            for (int64_t i = 0; i < I1; ++i) s += (int32_t)x[i] * (int32_t)l1w_q[o * p1 + i];
            int32_t c = s >> 6;
            h1[o] = c < 0 ? 0 : (c > 127 ? 127 : c);
        }
        for (int64_t o = 0; o < L3; ++o) {
            int32_t s = l2b_q[o];
            for (int64_t i = 0; i < L2; ++i) s += h1[i] * (int32_t)l2w_q[o * p2 + i];
            int32_t c = s >> 6;
            h2[o] = c < 0 ? 0 : (c > 127 ? 127 : c);
        }
        int32_t out = outb_q[0];
        for (int64_t i = 0; i < L3; ++i) out += h2[i] * (int32_t)outw_q[i];
        raw_out[b] = out;
        if (score_out) score_out[b] = out / fv_scale;
        (void)p3;
    }
    free(x);
    free(h1);
    free(h2);
}
