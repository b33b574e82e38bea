// HalfKP / KP NNUE (input -> l1 x 2 perspectives -> l2 -> l3 -> 1) on B200.
//
// Reference semantics: crates/cuda_cpp/cpp/bulletou_cuda_backend.cu
//   forward   cu:1021-1124 (kernels), cu:5894-5991 (launcher), ABI cu:10864
//   backward  cu:5042-5365 (kernels), cu:9142-9290 (launcher), ABI cu:12069
//   runner    crates/cuda_cpp/src/lib.rs:5748-5799 (forward -> loss ->
//             backward -> 8 x Ranger, lib.rs:5964-6024)
//
// Two implementations of the same math:
//   * the production shape (l1 in {256, 512}, l2 = l3 = 32) runs a fused
//     warp-per-position kernel: 128-bit gathers of the active feature rows for
//     both perspectives, ClippedReLU, both dense layers from shared memory,
//     the loss, and the whole dense backward in one pass.  The feature
//     transformer's weight gradient is then summed per row from an inverse
//     index and consumed by the Ranger row kernel directly;
//   * any other shape runs simple one-thread-per-output kernels.
// Forward sums keep the reference's order (bias first, then slots in order;
// dense dots sequential over inputs with FMA), so forward activations match
// the reference bit for bit.
#include <algorithm>
#include <cfloat>
#include <cstring>

#include "common.cuh"
#include "loss.cuh"
#include "optim.cuh"
#include "halfkp_fast.cuh"
#include "sparse_rows.cuh"

namespace bou {
int apply_norm_loss(BulletOuCudaCppContext* ctx, float* w, size_t n, float rate);
int launch_ranger(BulletOuCudaCppContext* ctx, size_t len, const RangerArgs& a, float* gradients, float* weights,
                  float* momentum, float* velocity, float* slow);
int launch_lookahead(BulletOuCudaCppContext* ctx, size_t len, const RangerArgs& a, float* weights, float* slow);
int fill_device(BulletOuCudaCppContext* ctx, float* ptr, size_t len, float value, const char* label);
int launch_scalar_loss(BulletOuCudaCppContext* ctx, const LossArgs& la, size_t batch, const float* outputs,
                       const float* targets, const float* entry_weights, float* per_sample, float* mog,
                       float* weighted_sum, float* mean, int finalize);
int loss_args(const BulletOuB200LossSpec* loss, size_t batch, LossArgs* out);
}  // namespace bou

using namespace bou;

namespace {

__device__ __forceinline__ float crelu01(float x) { return fminf(fmaxf(x, 0.0f), 1.0f); }
__device__ __forceinline__ float crelu_grad(float activation, float g) {
    return activation > 0.0f && activation < 1.0f ? g : 0.0f;
}

// ---------------------------------------------------------------------------
// Generic-shape kernels (any l1/l2/l3).
// ---------------------------------------------------------------------------

__global__ void g_ft_forward_kernel(const int* __restrict__ stm, const int* __restrict__ nstm, const float* __restrict__ l0w,
                                    const float* __restrict__ l0b, float* __restrict__ stm_l0, float* __restrict__ nstm_l0,
                                    float* __restrict__ combined, size_t batch, size_t max_active, size_t l1, RowMap map) {
    const size_t t = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= batch * l1) return;
    const int persp = blockIdx.y;
    const size_t b = t / l1, col = t % l1;
    const int* idx = (persp == 0 ? stm : nstm) + b * max_active;
    float sum = l0b[col];
    for (size_t s = 0; s < max_active; ++s) {
        int r0, r1;
        const int n = map.rows(idx[s], &r0, &r1);
        if (n == 1) sum += l0w[static_cast<size_t>(r0) * l1 + col];
        else if (n == 2) sum += l0w[static_cast<size_t>(r0) * l1 + col] + l0w[static_cast<size_t>(r1) * l1 + col];
    }
    const float x = crelu01(sum);
    (persp == 0 ? stm_l0 : nstm_l0)[t] = x;
    if (combined != nullptr) combined[b * 2 * l1 + persp * l1 + col] = x;
}

__global__ void g_dense_forward_kernel(const float* __restrict__ in, const float* __restrict__ w, const float* __restrict__ bias,
                                       float* __restrict__ out, size_t batch, size_t in_dim, size_t out_dim, int activate) {
    const size_t t = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= batch * out_dim) return;
    const size_t b = t / out_dim, o = t % out_dim;
    float sum = bias[o];
    for (size_t i = 0; i < in_dim; ++i) sum = fmaf(in[b * in_dim + i], w[i * out_dim + o], sum);
    out[t] = activate ? crelu01(sum) : sum;
}

// out[col] = sum_b x[b*ld + col] * (y ? y[b] : 1), one block per column,
// fixed-order tree reduction.
__global__ void g_column_dot_kernel(const float* __restrict__ x, size_t ld, const float* __restrict__ y, size_t batch,
                                    float* __restrict__ out, const float* __restrict__ x2) {
    __shared__ float red[256];
    const size_t col = blockIdx.x;
    float s = 0.0f;
    for (size_t b = threadIdx.x; b < batch; b += 256) {
        float v = x[b * ld + col];
        if (x2 != nullptr) v = v + x2[b * ld + col];
        s = y != nullptr ? fmaf(v, y[b], s) : s + v;
    }
    red[threadIdx.x] = s;
    __syncthreads();
    for (int d = 128; d > 0; d >>= 1) {
        if (threadIdx.x < d) red[threadIdx.x] += red[threadIdx.x + d];
        __syncthreads();
    }
    if (threadIdx.x == 0) out[col] = red[0];
}

__global__ void g_output_backward_kernel(const float* __restrict__ mog, const float* __restrict__ outw,
                                         float* __restrict__ h2g, size_t batch, size_t l3) {
    const size_t t = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= batch * l3) return;
    h2g[t] = mog[t / l3] * outw[t % l3];
}

__global__ void g_mask_kernel(const float* __restrict__ act, float* __restrict__ g, size_t len) {
    const size_t t = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t < len) g[t] = crelu_grad(act[t], g[t]);
}

// in_grad[b][i] = sum_o g[b][o] * w[i][o]
__global__ void g_dense_input_grad_kernel(const float* __restrict__ g, const float* __restrict__ w,
                                          float* __restrict__ in_grad, size_t batch, size_t in_dim, size_t out_dim) {
    const size_t t = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= batch * in_dim) return;
    const size_t b = t / in_dim, i = t % in_dim;
    float s = 0.0f;
    for (size_t o = 0; o < out_dim; ++o) s = fmaf(g[b * out_dim + o], w[i * out_dim + o], s);
    in_grad[t] = s;
}

// w_grad[i][o] = sum_b x[b][i] * g[b][o]; block (32 x 8) per (i, 32 outputs).
__global__ void g_dense_weight_grad_kernel(const float* __restrict__ x, const float* __restrict__ g,
                                           float* __restrict__ w_grad, size_t batch, size_t in_dim, size_t out_dim) {
    __shared__ float red[8][33];
    const size_t i = blockIdx.x;
    const size_t o = static_cast<size_t>(blockIdx.y) * 32 + threadIdx.x;
    float s = 0.0f;
    if (o < out_dim)
        for (size_t b = threadIdx.y; b < batch; b += 8) s = fmaf(x[b * in_dim + i], g[b * out_dim + o], s);
    red[threadIdx.y][threadIdx.x] = s;
    __syncthreads();
    if (threadIdx.y == 0 && o < out_dim) {
        float t = 0.0f;
        for (int y = 0; y < 8; ++y) t += red[y][threadIdx.x];
        w_grad[i * out_dim + o] = t;
    }
}

__global__ void g_l0_mask_kernel(const float* __restrict__ combined_g, const float* __restrict__ stm_l0,
                                 const float* __restrict__ nstm_l0, float* __restrict__ stm_g, float* __restrict__ nstm_g,
                                 size_t batch, size_t l1) {
    const size_t t = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= batch * 2 * l1) return;
    const size_t b = t / (2 * l1), c = t % (2 * l1);
    if (c < l1) stm_g[b * l1 + c] = crelu_grad(stm_l0[b * l1 + c], combined_g[t]);
    else nstm_g[b * l1 + c - l1] = crelu_grad(nstm_l0[b * l1 + c - l1], combined_g[t]);
}

int launch_1d(size_t work, const char* label, int* blocks) { return grid_1d(work, 256, blocks, label); }

struct NnueDims {
    size_t input_size, l1, l2, l3, batch, max_active;
};

int generic_forward(BulletOuCudaCppContext* ctx, const NnueDims& d, const int* stm, const int* nstm, const float* const* w,
                    float* stm_l0, float* nstm_l0, float* combined, float* hidden1, float* hidden2, float* output) {
    int blocks = 0;
    if (launch_1d(d.batch * d.l1, "nnue ft forward", &blocks) != 0) return -1;
    g_ft_forward_kernel<<<dim3(blocks, 2), 256, 0, ctx->stream>>>(stm, nstm, w[0], w[1], stm_l0, nstm_l0, combined,
                                                                  d.batch, d.max_active, d.l1, make_row_map(d.input_size));
    if (check_launch("nnue ft forward launch") != 0) return -1;
    if (launch_1d(d.batch * d.l2, "nnue l1 forward", &blocks) != 0) return -1;
    g_dense_forward_kernel<<<blocks, 256, 0, ctx->stream>>>(combined, w[2], w[3], hidden1, d.batch, 2 * d.l1, d.l2, 1);
    if (launch_1d(d.batch * d.l3, "nnue l2 forward", &blocks) != 0) return -1;
    g_dense_forward_kernel<<<blocks, 256, 0, ctx->stream>>>(hidden1, w[4], w[5], hidden2, d.batch, d.l2, d.l3, 1);
    if (launch_1d(d.batch, "nnue output forward", &blocks) != 0) return -1;
    g_dense_forward_kernel<<<blocks, 256, 0, ctx->stream>>>(hidden2, w[6], w[7], output, d.batch, d.l3, 1, 0);
    return check_launch("nnue dense forward launch");
}

// Dense part of the backward (everything except the l0w gradient), ABI
// buffer semantics of cu:9142-9290: hidden2/hidden1 gradients end up masked
// by the ClippedReLU derivative, combined gradient unmasked, per-perspective
// l0 gradients masked.
int generic_dense_backward(BulletOuCudaCppContext* ctx, const NnueDims& d, const float* combined, const float* hidden1,
                           const float* hidden2, const float* stm_l0, const float* nstm_l0, const float* l1w,
                           const float* l2w, const float* outw, const float* mog, float* h2g, float* h1g, float* cg,
                           float* stm_g, float* nstm_g, float* l0b_g, float* l1w_g, float* l1b_g, float* l2w_g,
                           float* l2b_g, float* outw_g, float* outb_g) {
    int blocks = 0;
    if (launch_1d(d.batch * d.l3, "nnue output backward", &blocks) != 0) return -1;
    g_output_backward_kernel<<<blocks, 256, 0, ctx->stream>>>(mog, outw, h2g, d.batch, d.l3);
    g_column_dot_kernel<<<static_cast<int>(d.l3), 256, 0, ctx->stream>>>(hidden2, d.l3, mog, d.batch, outw_g, nullptr);
    g_column_dot_kernel<<<1, 256, 0, ctx->stream>>>(mog, 1, nullptr, d.batch, outb_g, nullptr);
    // layer 2
    if (launch_1d(d.batch * d.l3, "nnue l2 mask", &blocks) != 0) return -1;
    g_mask_kernel<<<blocks, 256, 0, ctx->stream>>>(hidden2, h2g, d.batch * d.l3);
    if (launch_1d(d.batch * d.l2, "nnue l2 input grad", &blocks) != 0) return -1;
    g_dense_input_grad_kernel<<<blocks, 256, 0, ctx->stream>>>(h2g, l2w, h1g, d.batch, d.l2, d.l3);
    g_dense_weight_grad_kernel<<<dim3(static_cast<unsigned>(d.l2), static_cast<unsigned>((d.l3 + 31) / 32)), dim3(32, 8), 0,
                                 ctx->stream>>>(hidden1, h2g, l2w_g, d.batch, d.l2, d.l3);
    g_column_dot_kernel<<<static_cast<int>(d.l3), 256, 0, ctx->stream>>>(h2g, d.l3, nullptr, d.batch, l2b_g, nullptr);
    // layer 1
    if (launch_1d(d.batch * d.l2, "nnue l1 mask", &blocks) != 0) return -1;
    g_mask_kernel<<<blocks, 256, 0, ctx->stream>>>(hidden1, h1g, d.batch * d.l2);
    if (launch_1d(d.batch * 2 * d.l1, "nnue l1 input grad", &blocks) != 0) return -1;
    g_dense_input_grad_kernel<<<blocks, 256, 0, ctx->stream>>>(h1g, l1w, cg, d.batch, 2 * d.l1, d.l2);
    g_dense_weight_grad_kernel<<<dim3(static_cast<unsigned>(2 * d.l1), static_cast<unsigned>((d.l2 + 31) / 32)),
                                 dim3(32, 8), 0, ctx->stream>>>(combined, h1g, l1w_g, d.batch, 2 * d.l1, d.l2);
    g_column_dot_kernel<<<static_cast<int>(d.l2), 256, 0, ctx->stream>>>(h1g, d.l2, nullptr, d.batch, l1b_g, nullptr);
    // feature transformer activations
    if (launch_1d(d.batch * 2 * d.l1, "nnue l0 mask", &blocks) != 0) return -1;
    g_l0_mask_kernel<<<blocks, 256, 0, ctx->stream>>>(cg, stm_l0, nstm_l0, stm_g, nstm_g, d.batch, d.l1);
    g_column_dot_kernel<<<static_cast<int>(d.l1), 256, 0, ctx->stream>>>(stm_g, d.l1, nullptr, d.batch, l0b_g, nstm_g);
    return check_launch("nnue dense backward launch");
}

bool is_fast_shape(const NnueDims& d) { return halfkp_fast_shape(d.l1, d.l2, d.l3, d.batch, d.max_active); }

HalfkpWeights halfkp_weights(const float* const* w) {
    return HalfkpWeights{w[0], w[1], w[2], w[3], w[4], w[5], w[6], w[7]};
}

HalfkpDims halfkp_dims(const NnueDims& d) {
    return HalfkpDims{static_cast<int>(d.input_size), static_cast<int>(d.l1), static_cast<int>(d.batch),
                      static_cast<int>(d.max_active)};
}

size_t dense_len(size_t l1, size_t l2, size_t l3) { return l1 + 2 * l1 * l2 + l2 + l2 * l3 + l3 + l3 + 1; }

int validate_dims(const NnueDims& d) {
    if (d.input_size == 0 || d.l1 == 0 || d.l2 == 0 || d.l3 == 0)
        return fail_message("NNUE shape dimensions must be greater than zero");
    if (d.batch == 0) return fail_message("NNUE batch size must be greater than zero");
    if (d.max_active == 0) return fail_message("NNUE max_active must be greater than zero");
    return 0;
}

size_t ft_rows(const NnueDims& d) { return d.input_size; }

struct TrainScratch {
    float* combined;
    float* hidden1;
    float* hidden2;
    float* g1;
    float* g2;
    float* pregrad;
    // generic path extras
    float* stm_l0;
    float* nstm_l0;
    float* h2g;
    float* h1g;
    float* cg;
    float* stm_g;
    float* nstm_g;
    float* small_grads;  // packed dense gradient
};

int alloc_train_scratch(BulletOuCudaCppContext* ctx, const NnueDims& d, bool fast, TrainScratch* s) {
    const size_t B = d.batch, in = 2 * d.l1;
    size_t floats = 0;
    auto take = [&](size_t n) {
        size_t off = floats;
        floats += (n + 63) & ~static_cast<size_t>(63);
        return off;
    };
    const size_t o_comb = take(B * in), o_h1 = take(B * d.l2), o_h2 = take(B * d.l3), o_g1 = take(B * d.l2),
                 o_g2 = take(B * d.l3), o_pg = take(B * in), o_small = take(dense_len(d.l1, d.l2, d.l3));
    size_t o_stm = 0, o_nstm = 0, o_h2g = 0, o_h1g = 0, o_cg = 0, o_sg = 0, o_ng = 0;
    if (!fast) {
        o_stm = take(B * d.l1); o_nstm = take(B * d.l1); o_h2g = take(B * d.l3); o_h1g = take(B * d.l2);
        o_cg = take(B * in); o_sg = take(B * d.l1); o_ng = take(B * d.l1);
    }
    void* slab = nullptr;
    if (scratch_slot(ctx, kScratchActivations, floats * sizeof(float), &slab, "cudaMalloc nnue step activations") != 0)
        return -1;
    float* f = static_cast<float*>(slab);
    s->combined = f + o_comb; s->hidden1 = f + o_h1; s->hidden2 = f + o_h2; s->g1 = f + o_g1; s->g2 = f + o_g2;
    s->pregrad = f + o_pg; s->small_grads = f + o_small;
    s->stm_l0 = fast ? nullptr : f + o_stm; s->nstm_l0 = fast ? nullptr : f + o_nstm;
    s->h2g = fast ? nullptr : f + o_h2g; s->h1g = fast ? nullptr : f + o_h1g; s->cg = fast ? nullptr : f + o_cg;
    s->stm_g = fast ? nullptr : f + o_sg; s->nstm_g = fast ? nullptr : f + o_ng;
    return 0;
}

struct StepIO {
    const int* stm;
    const int* nstm;
    const float* targets;
    const float* entry_weights;
    float* const* w;  // 8
    float* const* m;
    float* const* v;
    float* const* s;
    float* output;
    float* per_sample;
    float* mog;
    float* weighted_sum;
    float* mean;
};

SmallGroups small_groups(const NnueDims& d, const StepIO& io) {
    SmallGroups g{};
    for (int i = 0; i < 7; ++i) {
        g.w[i] = io.w ? io.w[i + 1] : nullptr;
        g.m[i] = io.m ? io.m[i + 1] : nullptr;
        g.v[i] = io.v ? io.v[i + 1] : nullptr;
        g.s[i] = io.s ? io.s[i + 1] : nullptr;
    }
    const size_t sizes[7] = {d.l1, 2 * d.l1 * d.l2, d.l2, d.l2 * d.l3, d.l3, d.l3, 1};
    int off = 0;
    for (int i = 0; i < 7; ++i) {
        g.begin[i] = off;
        off += static_cast<int>(sizes[i]);
    }
    g.begin[7] = off;
    return g;
}

// mode 0: full step with Ranger (ranger != null).  mode 1: data-parallel
// local gradients into ft_grad [rows][l1] and dense_grad (packed).
int nnue_step(BulletOuCudaCppContext* ctx, const NnueDims& d, const StepIO& io, const LossArgs& la, int finalize,
              const BulletOuB200RangerStep* ranger_step, float* ft_grad, float* dense_grad) {
    const bool fast = is_fast_shape(d);
    const bool update = ranger_step != nullptr;
    const size_t in = 2 * d.l1;
    const size_t n_rows = ft_rows(d);
    RangerArgs ra{};
    if (update) ra = ranger_args_from(*ranger_step);
    // NormLoss (lib.rs:9318-9327, cu:10652-10696) scales whole tensors, so it
    // runs as separate passes around the fused update: before it, or after it
    // and before lookahead.
    const bool norm_before = update && ranger_step->norm_loss_rate != 0.0f && ranger_step->norm_loss_before;
    const bool norm_after = update && ranger_step->norm_loss_rate != 0.0f && !ranger_step->norm_loss_before;
    const size_t group_lens[8] = {n_rows * d.l1, d.l1, in * d.l2, d.l2, d.l2 * d.l3, d.l3, d.l3, 1};
    ctx->prof_marks_per_step = 8;
    prof_mark(ctx);
    // Inverse index of the batch (depends only on the sparse inputs).
    InverseIndex index;
    if (build_inverse_index(ctx, io.stm, io.nstm, d.batch, d.max_active, d.input_size, n_rows, &index) != 0) return -1;
    prof_mark(ctx);

    TrainScratch s{};
    if (alloc_train_scratch(ctx, d, fast, &s) != 0) return -1;
    float* const* w = io.w;
    const float* wc[8] = {w[0], w[1], w[2], w[3], w[4], w[5], w[6], w[7]};
    const SmallGroups groups = small_groups(d, io);
    float* pregrad_stm = nullptr;
    float* pregrad_nstm = nullptr;
    size_t pregrad_stride = 0;
    RangerArgs fa = ra;
    if (norm_after) fa.do_lookahead = 0;

    if (fast) {
        const HalfkpDims hd = halfkp_dims(d);
        const HalfkpActivations ha{s.combined, s.hidden1, s.hidden2, io.output, s.g1,
                                   s.g2,       s.pregrad, io.per_sample, io.mog};
        if (halfkp_fast_forward_backward(ctx, hd, make_row_map(d.input_size), io.stm, io.nstm, halfkp_weights(wc), ha,
                                         io.targets, io.entry_weights, &la, nullptr, nullptr) != 0)
            return -1;
        prof_mark(ctx);
        if (norm_before)
            for (int g = 0; g < 8; ++g)
                if (apply_norm_loss(ctx, w[g], group_lens[g], ranger_step->norm_loss_rate) != 0) return -1;
        if (halfkp_fast_small_params(ctx, hd, ha, groups, update ? &fa : nullptr, dense_grad, io.weighted_sum,
                                     io.mean, finalize) != 0)
            return -1;
        prof_mark(ctx);
        pregrad_stm = s.pregrad;
        pregrad_nstm = s.pregrad + d.l1;
        pregrad_stride = in;
    } else {
        if (generic_forward(ctx, d, io.stm, io.nstm, wc, s.stm_l0, s.nstm_l0, s.combined, s.hidden1, s.hidden2,
                            io.output) != 0)
            return -1;
        if (launch_scalar_loss(ctx, la, d.batch, io.output, io.targets, io.entry_weights, io.per_sample, io.mog,
                               io.weighted_sum, io.mean, finalize) != 0)
            return -1;
        float* sg = s.small_grads;
        const SmallGroups& g = groups;
        if (generic_dense_backward(ctx, d, s.combined, s.hidden1, s.hidden2, s.stm_l0, s.nstm_l0, wc[2], wc[4], wc[6],
                                   io.mog, s.h2g, s.h1g, s.cg, s.stm_g, s.nstm_g, sg + g.begin[0], sg + g.begin[1],
                                   sg + g.begin[2], sg + g.begin[3], sg + g.begin[4], sg + g.begin[5],
                                   sg + g.begin[6]) != 0)
            return -1;
        if (update) {
            if (norm_before)
                for (int k = 0; k < 8; ++k)
                    if (apply_norm_loss(ctx, w[k], group_lens[k], ranger_step->norm_loss_rate) != 0) return -1;
            for (int k = 0; k < 7; ++k)
                if (launch_ranger(ctx, group_lens[k + 1], fa, sg + g.begin[k], w[k + 1], io.m[k + 1], io.v[k + 1],
                                  io.s[k + 1]) != 0)
                    return -1;
        } else {
            cudaError_t st = cudaMemcpyAsync(dense_grad, sg, static_cast<size_t>(g.begin[7]) * sizeof(float),
                                             cudaMemcpyDeviceToDevice, ctx->stream);
            if (st != cudaSuccess) return fail("cudaMemcpyAsync dense gradients", st);
        }
        pregrad_stm = s.stm_g;
        pregrad_nstm = s.nstm_g;
        pregrad_stride = d.l1;
        for (int k = 0; k < 5; ++k) prof_mark(ctx);
    }

    // Feature-transformer rows: sum each row's gradient from the index, then
    // Ranger (or write the gradient for the data-parallel exchange).
    RowKernelArgs ra_rows{};
    ra_rows.offsets = index.offsets;
    ra_rows.entries = index.entries;
    ra_rows.n_rows = static_cast<int>(n_rows);
    ra_rows.row_begin = 0;
    ra_rows.width = static_cast<int>(d.l1);
    ra_rows.src.base[0] = pregrad_stm;
    ra_rows.src.base[1] = pregrad_nstm;
    ra_rows.src.sample_stride = pregrad_stride;
    if (update) {
        ra_rows.weights = w[0];
        ra_rows.momentum = io.m[0];
        ra_rows.velocity = io.v[0];
        ra_rows.slow = io.s[0];
        ra_rows.ranger = ra;
        if (norm_after) ra_rows.ranger.do_lookahead = 0;
        ra_rows.skip_quiet = ranger_zero_step_is_identity(ra_rows.ranger) ? 1 : 0;
        if (launch_row_kernel(ctx, kRowRanger, ra_rows, static_cast<int>(n_rows)) != 0) return -1;
        if (norm_after) {
            for (int k = 0; k < 8; ++k)
                if (apply_norm_loss(ctx, w[k], group_lens[k], ranger_step->norm_loss_rate) != 0) return -1;
            if (ra.do_lookahead)
                for (int k = 0; k < 8; ++k)
                    if (launch_lookahead(ctx, group_lens[k], ra, w[k], io.s[k]) != 0) return -1;
        }
    } else {
        ra_rows.gradients = ft_grad;
        if (launch_row_kernel(ctx, kRowWrite, ra_rows, static_cast<int>(n_rows)) != 0) return -1;
    }
    prof_mark(ctx);
    return 0;
}

}  // namespace

extern "C" {

int bulletou_cuda_cpp_nnue_forward_device(
    BulletOuCudaCppContext* ctx, size_t input_size, size_t l1, size_t l2, size_t l3, size_t batch, size_t max_active,
    const BulletOuCudaCppI32Buffer* stm_indices, const BulletOuCudaCppI32Buffer* nstm_indices,
    const BulletOuCudaCppF32Buffer* l0w, const BulletOuCudaCppF32Buffer* l0b, const BulletOuCudaCppF32Buffer* l1w,
    const BulletOuCudaCppF32Buffer* l1b, const BulletOuCudaCppF32Buffer* l2w, const BulletOuCudaCppF32Buffer* l2b,
    const BulletOuCudaCppF32Buffer* outw, const BulletOuCudaCppF32Buffer* outb, BulletOuCudaCppF32Buffer* stm_l0,
    BulletOuCudaCppF32Buffer* nstm_l0, BulletOuCudaCppF32Buffer* combined, BulletOuCudaCppF32Buffer* hidden1,
    BulletOuCudaCppF32Buffer* hidden2, BulletOuCudaCppF32Buffer* output) {
    const NnueDims d{input_size, l1, l2, l3, batch, max_active};
    if (validate_i32(ctx, stm_indices, batch * max_active, "stm_indices") != 0 ||
        validate_i32(ctx, nstm_indices, batch * max_active, "nstm_indices") != 0 ||
        validate_f32(ctx, l0w, input_size * l1, "l0w") != 0 || validate_f32(ctx, l0b, l1, "l0b") != 0 ||
        validate_f32(ctx, l1w, l1 * 2 * l2, "l1w") != 0 || validate_f32(ctx, l1b, l2, "l1b") != 0 ||
        validate_f32(ctx, l2w, l2 * l3, "l2w") != 0 || validate_f32(ctx, l2b, l3, "l2b") != 0 ||
        validate_f32(ctx, outw, l3, "outw") != 0 || validate_f32(ctx, outb, 1, "outb") != 0 ||
        validate_f32(ctx, stm_l0, batch * l1, "stm_l0") != 0 || validate_f32(ctx, nstm_l0, batch * l1, "nstm_l0") != 0 ||
        validate_f32(ctx, combined, batch * l1 * 2, "combined") != 0 ||
        validate_f32(ctx, hidden1, batch * l2, "hidden1") != 0 || validate_f32(ctx, hidden2, batch * l3, "hidden2") != 0 ||
        validate_f32(ctx, output, batch, "output") != 0)
        return -1;
    if (validate_dims(d) != 0 || set_device(ctx) != 0) return -1;
    const float* w[8] = {l0w->ptr, l0b->ptr, l1w->ptr, l1b->ptr, l2w->ptr, l2b->ptr, outw->ptr, outb->ptr};
    int rc;
    if (is_fast_shape(d)) {
        const HalfkpActivations ha{combined->ptr, hidden1->ptr, hidden2->ptr, output->ptr, nullptr,
                                   nullptr,       nullptr,      nullptr,      nullptr};
        rc = halfkp_fast_forward_backward(ctx, halfkp_dims(d), make_row_map(input_size), stm_indices->ptr,
                                          nstm_indices->ptr, halfkp_weights(w), ha, nullptr, nullptr, nullptr,
                                          stm_l0->ptr, nstm_l0->ptr);
    } else {
        rc = generic_forward(ctx, d, stm_indices->ptr, nstm_indices->ptr, w, stm_l0->ptr, nstm_l0->ptr, combined->ptr,
                             hidden1->ptr, hidden2->ptr, output->ptr);
    }
    return rc == 0 ? ok() : rc;
}

int bulletou_cuda_cpp_nnue_forward_host(int device, size_t input_size, size_t l1, size_t l2, size_t l3, size_t batch,
                                        size_t max_active, const int* stm_indices, const int* nstm_indices,
                                        const float* l0w, const float* l0b, const float* l1w, const float* l1b,
                                        const float* l2w, const float* l2b, const float* outw, const float* outb,
                                        float* output) {
    const NnueDims d{input_size, l1, l2, l3, batch, max_active};
    if (validate_dims(d) != 0 || validate_host(stm_indices, batch * max_active, "stm_indices") != 0 ||
        validate_host(nstm_indices, batch * max_active, "nstm_indices") != 0 ||
        validate_host(l0w, input_size * l1, "l0w") != 0 || validate_host(l0b, l1, "l0b") != 0 ||
        validate_host(l1w, l1 * 2 * l2, "l1w") != 0 || validate_host(l1b, l2, "l1b") != 0 ||
        validate_host(l2w, l2 * l3, "l2w") != 0 || validate_host(l2b, l3, "l2b") != 0 ||
        validate_host(outw, l3, "outw") != 0 || validate_host(outb, 1, "outb") != 0 ||
        validate_host(output, batch, "output") != 0)
        return -1;
    BulletOuCudaCppContext* ctx = nullptr;
    if (bulletou_cuda_cpp_context_create(device, &ctx) != 0) return -1;
    BulletOuCudaCppI32Buffer *ds = nullptr, *dn = nullptr;
    BulletOuCudaCppF32Buffer* f[14] = {};
    const size_t lens[14] = {input_size * l1, l1, 2 * l1 * l2, l2, l2 * l3, l3, l3, 1,
                             batch * l1, batch * l1, batch * 2 * l1, batch * l2, batch * l3, batch};
    const float* host[8] = {l0w, l0b, l1w, l1b, l2w, l2b, outw, outb};
    int rc = bulletou_cuda_cpp_i32_buffer_create(ctx, batch * max_active, &ds);
    if (rc == 0) rc = bulletou_cuda_cpp_i32_buffer_create(ctx, batch * max_active, &dn);
    for (int i = 0; i < 14 && rc == 0; ++i) rc = bulletou_cuda_cpp_f32_buffer_create(ctx, lens[i], &f[i]);
    if (rc == 0) rc = bulletou_cuda_cpp_i32_upload(ctx, ds, stm_indices, batch * max_active);
    if (rc == 0) rc = bulletou_cuda_cpp_i32_upload(ctx, dn, nstm_indices, batch * max_active);
    for (int i = 0; i < 8 && rc == 0; ++i) rc = bulletou_cuda_cpp_f32_upload(ctx, f[i], host[i], lens[i]);
    if (rc == 0)
        rc = bulletou_cuda_cpp_nnue_forward_device(ctx, input_size, l1, l2, l3, batch, max_active, ds, dn, f[0], f[1],
                                                   f[2], f[3], f[4], f[5], f[6], f[7], f[8], f[9], f[10], f[11], f[12],
                                                   f[13]);
    if (rc == 0) rc = bulletou_cuda_cpp_f32_download(ctx, f[13], output, batch);
    char saved[512] = {0};
    if (rc != 0) bulletou_cuda_cpp_last_error(saved, sizeof(saved));
    bulletou_cuda_cpp_i32_buffer_destroy(ds);
    bulletou_cuda_cpp_i32_buffer_destroy(dn);
    for (auto* p : f) bulletou_cuda_cpp_f32_buffer_destroy(p);
    bulletou_cuda_cpp_context_destroy(ctx);
    if (rc != 0) {
        fail_message(saved);
        return rc;
    }
    return ok();
}

int bulletou_cuda_cpp_nnue_backward_device(
    BulletOuCudaCppContext* ctx, size_t input_size, size_t l1, size_t l2, size_t l3, size_t batch, size_t max_active,
    const BulletOuCudaCppI32Buffer* stm_indices, const BulletOuCudaCppI32Buffer* nstm_indices,
    const BulletOuCudaCppF32Buffer* combined, const BulletOuCudaCppF32Buffer* hidden1,
    const BulletOuCudaCppF32Buffer* hidden2, const BulletOuCudaCppF32Buffer* stm_l0,
    const BulletOuCudaCppF32Buffer* nstm_l0, const BulletOuCudaCppF32Buffer* l1w, const BulletOuCudaCppF32Buffer* l2w,
    const BulletOuCudaCppF32Buffer* outw, const BulletOuCudaCppF32Buffer* mean_output_gradients,
    BulletOuCudaCppF32Buffer* hidden2_gradients, BulletOuCudaCppF32Buffer* hidden1_gradients,
    BulletOuCudaCppF32Buffer* combined_gradients, BulletOuCudaCppF32Buffer* stm_l0_gradients,
    BulletOuCudaCppF32Buffer* nstm_l0_gradients, BulletOuCudaCppF32Buffer* l0w_gradients,
    BulletOuCudaCppF32Buffer* l0b_gradients, BulletOuCudaCppF32Buffer* l1w_gradients,
    BulletOuCudaCppF32Buffer* l1b_gradients, BulletOuCudaCppF32Buffer* l2w_gradients,
    BulletOuCudaCppF32Buffer* l2b_gradients, BulletOuCudaCppF32Buffer* outw_gradients,
    BulletOuCudaCppF32Buffer* outb_gradients, int zero_l0_gradients) {
    const NnueDims d{input_size, l1, l2, l3, batch, max_active};
    if (validate_dims(d) != 0 || validate_i32(ctx, stm_indices, batch * max_active, "stm_indices") != 0 ||
        validate_i32(ctx, nstm_indices, batch * max_active, "nstm_indices") != 0 ||
        validate_f32(ctx, combined, batch * l1 * 2, "combined") != 0 ||
        validate_f32(ctx, hidden1, batch * l2, "hidden1") != 0 || validate_f32(ctx, hidden2, batch * l3, "hidden2") != 0 ||
        validate_f32(ctx, stm_l0, batch * l1, "stm_l0") != 0 || validate_f32(ctx, nstm_l0, batch * l1, "nstm_l0") != 0 ||
        validate_f32(ctx, l1w, l1 * 2 * l2, "l1w") != 0 || validate_f32(ctx, l2w, l2 * l3, "l2w") != 0 ||
        validate_f32(ctx, outw, l3, "outw") != 0 ||
        validate_f32(ctx, mean_output_gradients, batch, "mean_output_gradients") != 0 ||
        validate_f32(ctx, hidden2_gradients, batch * l3, "hidden2_gradients") != 0 ||
        validate_f32(ctx, hidden1_gradients, batch * l2, "hidden1_gradients") != 0 ||
        validate_f32(ctx, combined_gradients, batch * l1 * 2, "combined_gradients") != 0 ||
        validate_f32(ctx, stm_l0_gradients, batch * l1, "stm_l0_gradients") != 0 ||
        validate_f32(ctx, nstm_l0_gradients, batch * l1, "nstm_l0_gradients") != 0 ||
        validate_f32(ctx, l0w_gradients, input_size * l1, "l0w_gradients") != 0 ||
        validate_f32(ctx, l0b_gradients, l1, "l0b_gradients") != 0 ||
        validate_f32(ctx, l1w_gradients, l1 * 2 * l2, "l1w_gradients") != 0 ||
        validate_f32(ctx, l1b_gradients, l2, "l1b_gradients") != 0 ||
        validate_f32(ctx, l2w_gradients, l2 * l3, "l2w_gradients") != 0 ||
        validate_f32(ctx, l2b_gradients, l3, "l2b_gradients") != 0 ||
        validate_f32(ctx, outw_gradients, l3, "outw_gradients") != 0 ||
        validate_f32(ctx, outb_gradients, 1, "outb_gradients") != 0)
        return -1;
    if (set_device(ctx) != 0) return -1;
    if (generic_dense_backward(ctx, d, combined->ptr, hidden1->ptr, hidden2->ptr, stm_l0->ptr, nstm_l0->ptr, l1w->ptr,
                               l2w->ptr, outw->ptr, mean_output_gradients->ptr, hidden2_gradients->ptr,
                               hidden1_gradients->ptr, combined_gradients->ptr, stm_l0_gradients->ptr,
                               nstm_l0_gradients->ptr, l0b_gradients->ptr, l1w_gradients->ptr, l1b_gradients->ptr,
                               l2w_gradients->ptr, l2b_gradients->ptr, outw_gradients->ptr, outb_gradients->ptr) != 0)
        return -1;
    if (zero_l0_gradients != 0 && fill_device(ctx, l0w_gradients->ptr, input_size * l1, 0.0f, "zero l0w gradients") != 0)
        return -1;
    InverseIndex index;
    if (build_inverse_index(ctx, stm_indices->ptr, nstm_indices->ptr, batch, max_active, input_size, input_size, &index) != 0)
        return -1;
    RowKernelArgs ra{};
    ra.offsets = index.offsets;
    ra.entries = index.entries;
    ra.n_rows = static_cast<int>(input_size);
    ra.width = static_cast<int>(l1);
    ra.src.base[0] = stm_l0_gradients->ptr;
    ra.src.base[1] = nstm_l0_gradients->ptr;
    ra.src.sample_stride = l1;
    ra.gradients = l0w_gradients->ptr;
    if (launch_row_kernel(ctx, kRowAccumulate, ra, static_cast<int>(input_size)) != 0) return -1;
    return ok();
}

int bulletou_cuda_cpp_nnue_train_warmup_device(
    BulletOuCudaCppContext* ctx, size_t input_size, size_t l1, size_t l2, size_t l3, size_t batch, size_t max_active,
    const BulletOuCudaCppF32Buffer* combined, const BulletOuCudaCppF32Buffer* hidden1,
    const BulletOuCudaCppF32Buffer* hidden2, const BulletOuCudaCppF32Buffer* l1w, const BulletOuCudaCppF32Buffer* l2w,
    const BulletOuCudaCppF32Buffer* outw, const BulletOuCudaCppF32Buffer* mean_output_gradients,
    BulletOuCudaCppF32Buffer* hidden2_gradients, BulletOuCudaCppF32Buffer* hidden1_gradients,
    BulletOuCudaCppF32Buffer* combined_gradients, BulletOuCudaCppF32Buffer* l1w_gradients,
    BulletOuCudaCppF32Buffer* l1b_gradients, BulletOuCudaCppF32Buffer* l2w_gradients,
    BulletOuCudaCppF32Buffer* l2b_gradients, BulletOuCudaCppF32Buffer* outw_gradients,
    BulletOuCudaCppF32Buffer* outb_gradients) {
    // The reference warms cuBLAS's dense backward before timing (cu:12169).
    // This backend has no library state to warm; validate like the reference
    // and synchronize.
    const NnueDims d{input_size, l1, l2, l3, batch, max_active};
    if (validate_dims(d) != 0 || validate_f32(ctx, combined, batch * l1 * 2, "warmup combined") != 0 ||
        validate_f32(ctx, hidden1, batch * l2, "warmup hidden1") != 0 ||
        validate_f32(ctx, hidden2, batch * l3, "warmup hidden2") != 0 ||
        validate_f32(ctx, l1w, l1 * 2 * l2, "warmup l1w") != 0 || validate_f32(ctx, l2w, l2 * l3, "warmup l2w") != 0 ||
        validate_f32(ctx, outw, l3, "warmup outw") != 0 ||
        validate_f32(ctx, mean_output_gradients, batch, "warmup mean_output_gradients") != 0 ||
        validate_f32(ctx, hidden2_gradients, batch * l3, "warmup hidden2_gradients") != 0 ||
        validate_f32(ctx, hidden1_gradients, batch * l2, "warmup hidden1_gradients") != 0 ||
        validate_f32(ctx, combined_gradients, batch * l1 * 2, "warmup combined_gradients") != 0 ||
        validate_f32(ctx, l1w_gradients, l1 * 2 * l2, "warmup l1w_gradients") != 0 ||
        validate_f32(ctx, l1b_gradients, l2, "warmup l1b_gradients") != 0 ||
        validate_f32(ctx, l2w_gradients, l2 * l3, "warmup l2w_gradients") != 0 ||
        validate_f32(ctx, l2b_gradients, l3, "warmup l2b_gradients") != 0 ||
        validate_f32(ctx, outw_gradients, l3, "warmup outw_gradients") != 0 ||
        validate_f32(ctx, outb_gradients, 1, "warmup outb_gradients") != 0)
        return -1;
    if (set_device(ctx) != 0) return -1;
    cudaError_t st = cudaStreamSynchronize(ctx->stream);
    if (st != cudaSuccess) return fail("cudaStreamSynchronize NNUE train warmup", st);
    return ok();
}

static int validate_step_groups(BulletOuCudaCppContext* ctx, const NnueDims& d, BulletOuCudaCppF32Buffer* const* g,
                                const char* what) {
    if (g == nullptr) return fail_messagef("%s array must not be null", what);
    const size_t lens[8] = {d.input_size * d.l1, d.l1, 2 * d.l1 * d.l2, d.l2, d.l2 * d.l3, d.l3, d.l3, 1};
    static const char* names[8] = {"l0w", "l0b", "l1w", "l1b", "l2w", "l2b", "outw", "outb"};
    for (int i = 0; i < 8; ++i) {
        char name[64];
        std::snprintf(name, sizeof(name), "%s %s", what, names[i]);
        if (validate_f32(ctx, g[i], lens[i], name) != 0) return -1;
    }
    return 0;
}


int bulletou_b200_nnue_train_step_device(
    BulletOuCudaCppContext* ctx, size_t input_size, size_t l1, size_t l2, size_t l3, size_t batch, size_t max_active,
    const BulletOuCudaCppI32Buffer* stm_indices, const BulletOuCudaCppI32Buffer* nstm_indices,
    const BulletOuCudaCppF32Buffer* targets, const BulletOuCudaCppF32Buffer* entry_weights,
    const BulletOuB200LossSpec* loss, const BulletOuB200RangerStep* ranger, BulletOuCudaCppF32Buffer* const* params,
    BulletOuCudaCppF32Buffer* const* momentum, BulletOuCudaCppF32Buffer* const* velocity,
    BulletOuCudaCppF32Buffer* const* slow_params, BulletOuCudaCppF32Buffer* output, BulletOuCudaCppF32Buffer* per_sample,
    BulletOuCudaCppF32Buffer* mean_output_gradients, BulletOuCudaCppF32Buffer* weighted_sum,
    BulletOuCudaCppF32Buffer* mean) {
    const NnueDims d{input_size, l1, l2, l3, batch, max_active};
    LossArgs la{};
    if (validate_dims(d) != 0 || validate_i32(ctx, stm_indices, batch * max_active, "stm_indices") != 0 ||
        validate_i32(ctx, nstm_indices, batch * max_active, "nstm_indices") != 0 ||
        validate_f32(ctx, targets, batch, "targets") != 0 || validate_f32(ctx, entry_weights, batch, "entry_weights") != 0 ||
        validate_step_groups(ctx, d, params, "params") != 0 || validate_step_groups(ctx, d, momentum, "momentum") != 0 ||
        validate_step_groups(ctx, d, velocity, "velocity") != 0 ||
        validate_step_groups(ctx, d, slow_params, "slow_params") != 0 || validate_f32(ctx, output, batch, "output") != 0 ||
        validate_f32(ctx, per_sample, batch, "per_sample") != 0 ||
        validate_f32(ctx, mean_output_gradients, batch, "mean_output_gradients") != 0 ||
        validate_f32(ctx, weighted_sum, 1, "weighted_sum") != 0 || validate_f32(ctx, mean, 1, "mean") != 0 ||
        loss_args(loss, batch, &la) != 0)
        return -1;
    if (ranger == nullptr) return fail_message("ranger step must not be null");
    if (set_device(ctx) != 0) return -1;
    float* w[8];
    float* m[8];
    float* v[8];
    float* s[8];
    for (int i = 0; i < 8; ++i) {
        w[i] = params[i]->ptr;
        m[i] = momentum[i]->ptr;
        v[i] = velocity[i]->ptr;
        s[i] = slow_params[i]->ptr;
    }
    StepIO io{stm_indices->ptr, nstm_indices->ptr, targets->ptr, entry_weights->ptr, w, m, v, s, output->ptr,
              per_sample->ptr, mean_output_gradients->ptr, weighted_sum->ptr, mean->ptr};
    if (nnue_step(ctx, d, io, la, loss->finalize_loss, ranger, nullptr, nullptr) != 0) return -1;
    return ok();
}

int bulletou_b200_nnue_dense_gradient_len(size_t l1, size_t l2, size_t l3, size_t* out) {
    if (out == nullptr) return fail_message("dense_gradient_len output pointer must not be null");
    *out = dense_len(l1, l2, l3);
    return ok();
}

int bulletou_b200_nnue_local_gradients_device(
    BulletOuCudaCppContext* ctx, size_t input_size, size_t l1, size_t l2, size_t l3, size_t batch, size_t max_active,
    const BulletOuCudaCppI32Buffer* stm_indices, const BulletOuCudaCppI32Buffer* nstm_indices,
    const BulletOuCudaCppF32Buffer* targets, const BulletOuCudaCppF32Buffer* entry_weights,
    const BulletOuB200LossSpec* loss, BulletOuCudaCppF32Buffer* const* params, BulletOuCudaCppF32Buffer* ft_gradients,
    BulletOuCudaCppF32Buffer* dense_gradients, BulletOuCudaCppF32Buffer* output, BulletOuCudaCppF32Buffer* per_sample,
    BulletOuCudaCppF32Buffer* mean_output_gradients, BulletOuCudaCppF32Buffer* weighted_sum,
    BulletOuCudaCppF32Buffer* mean) {
    const NnueDims d{input_size, l1, l2, l3, batch, max_active};
    LossArgs la{};
    if (validate_dims(d) != 0 || validate_i32(ctx, stm_indices, batch * max_active, "stm_indices") != 0 ||
        validate_i32(ctx, nstm_indices, batch * max_active, "nstm_indices") != 0 ||
        validate_f32(ctx, targets, batch, "targets") != 0 || validate_f32(ctx, entry_weights, batch, "entry_weights") != 0 ||
        validate_step_groups(ctx, d, params, "params") != 0 ||
        validate_f32(ctx, ft_gradients, input_size * l1, "ft_gradients") != 0 ||
        validate_f32(ctx, dense_gradients, dense_len(l1, l2, l3), "dense_gradients") != 0 ||
        validate_f32(ctx, output, batch, "output") != 0 || validate_f32(ctx, per_sample, batch, "per_sample") != 0 ||
        validate_f32(ctx, mean_output_gradients, batch, "mean_output_gradients") != 0 ||
        validate_f32(ctx, weighted_sum, 1, "weighted_sum") != 0 || validate_f32(ctx, mean, 1, "mean") != 0 ||
        loss_args(loss, batch, &la) != 0)
        return -1;
    if (set_device(ctx) != 0) return -1;
    float* w[8];
    for (int i = 0; i < 8; ++i) w[i] = params[i]->ptr;
    StepIO io{stm_indices->ptr, nstm_indices->ptr, targets->ptr, entry_weights->ptr, w, nullptr, nullptr, nullptr,
              output->ptr, per_sample->ptr, mean_output_gradients->ptr, weighted_sum->ptr, mean->ptr};
    if (nnue_step(ctx, d, io, la, loss->finalize_loss, nullptr, ft_gradients->ptr, dense_gradients->ptr) != 0) return -1;
    return ok();
}

}  // extern "C"
