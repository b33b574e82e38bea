// KPPT scalar tables (KK / KKP / KPP components) on B200.
//
// Reference semantics: crates/cuda_cpp/cpp/bulletou_cuda_backend.cu
//   forward  cu:8970-9004  out = outw0*(b + sum_stm w) + outw1*(b + sum_nstm w) + outb
//   backward cu:9006-9050  zero-fill, then atomicAdd per slot; small grads by atomics
//   ABI      cu:11887-11983; runner lib.rs:4962-5066 (Ranger over table_w,
//            table_b, outw, outb).
//
// B200 layout: one warp per position; lanes stride over the slots (703 KPP
// pairs per view), so the random 4-byte table reads of a position are all in
// flight together; warp-tree sums.  The training step fuses forward, loss and
// the gradient scatter (vector reductions into a persistent, always-zero
// gradient table), and the table's Ranger pass resets that gradient to zero in
// the same sweep, so no separate zero-fill of the table is needed.
#include <cmath>

#include "common.cuh"
#include "king_sort.cuh"
#include "loss.cuh"
#include "optim.cuh"

namespace bou {
int launch_ranger(BulletOuCudaCppContext* ctx, size_t len, const RangerArgs& a, float* gradients, float* weights,
                  float* momentum, float* velocity, float* slow);
int fill_device(BulletOuCudaCppContext* ctx, float* ptr, size_t len, float value, const char* label);
int loss_args(const BulletOuB200LossSpec* loss, size_t batch, LossArgs* out);
}  // namespace bou

using namespace bou;

namespace {

constexpr int kWarps = 8;
constexpr unsigned kFull = 0xffffffffu;
// per-CTA partials: outw0, outw1, outb, table_b, loss
constexpr int kKpptVec = 5;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) v += __shfl_xor_sync(kFull, v, d);
    return v;
}

struct KpptArgs {
    const int* stm;
    const int* nstm;
    int max_active;
    int batch;
    int input_size;
    const float* table_w;
    const float* table_b;
    const float* outw;
    const float* outb;
    float* stm_eval;
    float* nstm_eval;
    float* output;
    // training / backward
    const float* targets;
    const float* entry_weights;
    LossArgs loss;
    const float* mog_in;  // backward-only mode: given output gradients
    float* per_sample;
    float* mog;
    float* table_grad;    // accumulated with vector-free reductions
    float* partials;      // [grid][kKpptVec]
    const float* eval2;   // mode 3: view evaluations, [2 * batch] (h = 2 * sample + view)
};

// mode 0: forward only; 1: forward + loss + backward; 2: backward only
// (stm_eval/nstm_eval/mog given); 3: output + loss from given view
// evaluations (eval2), no table access (the king-ordered train step).
template <int MODE>
__global__ void __launch_bounds__(kWarps * 32) kppt_kernel(KpptArgs a) {
    __shared__ float red[kWarps][kKpptVec];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float acc_w0 = 0.0f, acc_w1 = 0.0f, acc_ob = 0.0f, acc_tb = 0.0f, acc_loss = 0.0f;
    const float w0 = a.outw[0], w1 = a.outw[1];
    for (int b = blockIdx.x * kWarps + warp; b < a.batch; b += gridDim.x * kWarps) {
        const int* si = a.stm + static_cast<size_t>(b) * a.max_active;
        const int* ni = a.nstm + static_cast<size_t>(b) * a.max_active;
        float se, ne, gout;
        if (MODE == 3) {
            se = a.eval2[2 * static_cast<size_t>(b)];
            ne = a.eval2[2 * static_cast<size_t>(b) + 1];
            const float out = w0 * se + w1 * ne + a.outb[0];
            if (lane == 0) a.output[b] = out;
            float g = 0.0f;
            const float ps = sample_loss(a.loss, out, a.targets[b], a.entry_weights[b], &g);
            gout = g;
            if (lane == 0) {
                a.per_sample[b] = ps;
                a.mog[b] = g;
                acc_loss += ps;
            }
        } else if (MODE != 2) {
            float s = 0.0f, n = 0.0f;
            for (int k = lane; k < a.max_active; k += 32) {
                const int fs = __ldg(si + k), fn = __ldg(ni + k);
                if (fs >= 0 && fs < a.input_size) s += __ldg(a.table_w + fs);
                if (fn >= 0 && fn < a.input_size) n += __ldg(a.table_w + fn);
            }
            const float bias = a.table_b[0];
            se = bias + warp_sum(s);
            ne = bias + warp_sum(n);
            const float out = w0 * se + w1 * ne + a.outb[0];
            if (lane == 0) {
                if (a.stm_eval != nullptr) a.stm_eval[b] = se;
                if (a.nstm_eval != nullptr) a.nstm_eval[b] = ne;
                a.output[b] = out;
            }
            if (MODE == 0) continue;
            float g = 0.0f;
            const float ps = sample_loss(a.loss, out, a.targets[b], a.entry_weights[b], &g);
            gout = g;
            if (lane == 0) {
                a.per_sample[b] = ps;
                a.mog[b] = g;
                acc_loss += ps;
            }
        } else {
            se = a.stm_eval[b];
            ne = a.nstm_eval[b];
            gout = a.mog_in[b];
        }
        const float sg = gout * w0, ng = gout * w1;
        if (lane == 0) {
            acc_w0 = fmaf(gout, se, acc_w0);
            acc_w1 = fmaf(gout, ne, acc_w1);
            acc_ob += gout;
            acc_tb += sg + ng;
        }
        if constexpr (MODE != 3) {  // mode 3: the table gradient comes from kppt_scatter_kernel
            for (int k = lane; k < a.max_active; k += 32) {
                const int fs = __ldg(si + k), fn = __ldg(ni + k);
                if (fs >= 0 && fs < a.input_size) atomicAdd(a.table_grad + fs, sg);
                if (fn >= 0 && fn < a.input_size) atomicAdd(a.table_grad + fn, ng);
            }
        }
    }
    if (MODE == 0) return;
    if (lane == 0) {
        red[warp][0] = acc_w0;
        red[warp][1] = acc_w1;
        red[warp][2] = acc_ob;
        red[warp][3] = acc_tb;
        red[warp][4] = acc_loss;
    }
    __syncthreads();
    if (threadIdx.x < kKpptVec) {
        float s = 0.0f;
        for (int w = 0; w < kWarps; ++w) s += red[w][threadIdx.x];
        a.partials[static_cast<size_t>(blockIdx.x) * kKpptVec + threadIdx.x] = s;
    }
}

// King-ordered passes of the train step.  Every feature of a view lies in
// its king's block of the table (input_size / 81 entries), so warps working on
// consecutive half-positions of the king sort gather from (and scatter into)
// a few king blocks at a time, which L2 holds; in batch order every access is
// a DRAM sector of its own.  The view sum keeps the per-lane slot split and
// the warp-tree order of kppt_kernel, so the evaluations are bit-identical.
__global__ void __launch_bounds__(kWarps * 32) kppt_view_kernel(KpptArgs a, const int* __restrict__ order,
                                                                int n_half, float* __restrict__ eval2) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const float bias = a.table_b[0];
    for (int i = blockIdx.x * kWarps + warp; i < n_half; i += gridDim.x * kWarps) {
        const int h = __ldg(order + i);
        const int* idx = ((h & 1) ? a.nstm : a.stm) + static_cast<size_t>(h >> 1) * a.max_active;
        float s = 0.0f;
        for (int k = lane; k < a.max_active; k += 32) {
            const int f = __ldg(idx + k);
            if (f >= 0 && f < a.input_size) s += __ldg(a.table_w + f);
        }
        const float e = bias + warp_sum(s);
        if (lane == 0) eval2[h] = e;
    }
}

__global__ void __launch_bounds__(kWarps * 32) kppt_scatter_kernel(KpptArgs a, const int* __restrict__ order,
                                                                   int n_half) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const float w0 = a.outw[0], w1 = a.outw[1];
    for (int i = blockIdx.x * kWarps + warp; i < n_half; i += gridDim.x * kWarps) {
        const int h = __ldg(order + i);
        const float g = a.mog[h >> 1] * ((h & 1) ? w1 : w0);
        const int* idx = ((h & 1) ? a.nstm : a.stm) + static_cast<size_t>(h >> 1) * a.max_active;
        for (int k = lane; k < a.max_active; k += 32) {
            const int f = __ldg(idx + k);
            if (f >= 0 && f < a.input_size) atomicAdd(a.table_grad + f, g);
        }
    }
}

constexpr int kKpptKings = 81;
constexpr int kKpptKeys = kKpptKings + 1;  // + half-positions without a valid feature

struct KpptSmall {
    float* w[3];  // table_b, outw, outb
    float* m[3];
    float* v[3];
    float* s[3];
    float* grads[3];  // backward-only mode: destination gradients
};

// Reduces the per-CTA partials (fixed order); then either writes the small
// gradients (mode 0) or applies Ranger to them (mode 1).  Also finalizes the
// loss.
__global__ void kppt_small_kernel(const float* __restrict__ partials, int nparts, KpptSmall g, RangerArgs ra, int update,
                                  float* __restrict__ weighted_sum, float* __restrict__ mean, float batch_f,
                                  int finalize) {
    const int t = threadIdx.x;
    if (t >= 5) return;
    float s = 0.0f;
    for (int p = 0; p < nparts; ++p) s += partials[static_cast<size_t>(p) * kKpptVec + t];
    if (t == 4) {
        if (finalize) {
            *weighted_sum = s;
            *mean = s / batch_f;
        }
        return;
    }
    // t: 0 outw0, 1 outw1, 2 outb, 3 table_b
    const int grp = t == 3 ? 0 : (t <= 1 ? 1 : 2);
    const int k = t == 1 ? 1 : 0;
    if (!update) {
        g.grads[grp][k] = s;
        return;
    }
    float w = g.w[grp][k], m = g.m[grp][k], v = g.v[grp][k];
    radam_coordinate(ra.gradient_factor * s, ra, w, m, v);
    if (ra.do_lookahead) {
        w = lookahead_coordinate(w, g.s[grp][k], ra);
        g.s[grp][k] = w;
    }
    g.w[grp][k] = w;
    g.m[grp][k] = m;
    g.v[grp][k] = v;
}

int validate_kppt(size_t input_size, size_t batch, size_t max_active) {
    if (input_size == 0) return fail_message("KPPT table input_size must be greater than zero");
    if (batch == 0) return fail_message("KPPT table batch size must be greater than zero");
    if (max_active == 0) return fail_message("KPPT table max_active must be greater than zero");
    if (input_size > static_cast<size_t>(INT_MAX) || batch > static_cast<size_t>(INT_MAX / 2) ||
        max_active > static_cast<size_t>(INT_MAX))
        return fail_message("KPPT table dimensions exceed 32-bit indexing");
    return 0;
}

int kppt_grid(const BulletOuCudaCppContext* ctx, size_t batch) {
    int grid = ctx->sm_count * 8;
    const int needed = static_cast<int>((batch + kWarps - 1) / kWarps);
    return grid > needed ? needed : grid;
}

// Persistent, always-zero table gradient owned by the context.
int kppt_grad_table(BulletOuCudaCppContext* ctx, size_t len, float** out) {
    Scratch& s = ctx->scratch[kScratchKppt];
    const size_t bytes = len * sizeof(float);
    const bool fresh = s.bytes < bytes;
    void* p = nullptr;
    if (scratch_slot(ctx, kScratchKppt, bytes, &p, "cudaMalloc KPPT gradient table") != 0) return -1;
    if (fresh) {
        cudaError_t st = cudaMemsetAsync(p, 0, s.bytes, ctx->stream);
        if (st != cudaSuccess) return fail("cudaMemsetAsync KPPT gradient table", st);
    }
    *out = static_cast<float*>(p);
    return 0;
}

}  // namespace

extern "C" {

int bulletou_cuda_cpp_kppt_forward_device(BulletOuCudaCppContext* ctx, size_t input_size, size_t batch,
                                          size_t max_active, const BulletOuCudaCppI32Buffer* stm_indices,
                                          const BulletOuCudaCppI32Buffer* nstm_indices,
                                          const BulletOuCudaCppF32Buffer* table_w, const BulletOuCudaCppF32Buffer* table_b,
                                          const BulletOuCudaCppF32Buffer* outw, const BulletOuCudaCppF32Buffer* outb,
                                          BulletOuCudaCppF32Buffer* stm_eval, BulletOuCudaCppF32Buffer* nstm_eval,
                                          BulletOuCudaCppF32Buffer* outputs) {
    const size_t sparse = batch * max_active;
    if (validate_kppt(input_size, batch, max_active) != 0 ||
        validate_i32(ctx, stm_indices, sparse, "kppt stm_indices") != 0 ||
        validate_i32(ctx, nstm_indices, sparse, "kppt nstm_indices") != 0 ||
        validate_f32(ctx, table_w, input_size, "kppt table_w") != 0 ||
        validate_f32(ctx, table_b, 1, "kppt table_b") != 0 || validate_f32(ctx, outw, 2, "kppt outw") != 0 ||
        validate_f32(ctx, outb, 1, "kppt outb") != 0 || validate_f32(ctx, stm_eval, batch, "kppt stm_eval") != 0 ||
        validate_f32(ctx, nstm_eval, batch, "kppt nstm_eval") != 0 ||
        validate_f32(ctx, outputs, batch, "kppt outputs") != 0)
        return -1;
    if (set_device(ctx) != 0) return -1;
    KpptArgs a{};
    a.stm = stm_indices->ptr;
    a.nstm = nstm_indices->ptr;
    a.max_active = static_cast<int>(max_active);
    a.batch = static_cast<int>(batch);
    a.input_size = static_cast<int>(input_size);
    a.table_w = table_w->ptr;
    a.table_b = table_b->ptr;
    a.outw = outw->ptr;
    a.outb = outb->ptr;
    a.stm_eval = stm_eval->ptr;
    a.nstm_eval = nstm_eval->ptr;
    a.output = outputs->ptr;
    kppt_kernel<0><<<kppt_grid(ctx, batch), kWarps * 32, 0, ctx->stream>>>(a);
    if (check_launch("kppt forward launch") != 0) return -1;
    return ok();
}

int bulletou_cuda_cpp_kppt_backward_device(BulletOuCudaCppContext* ctx, size_t input_size, size_t batch,
                                           size_t max_active, const BulletOuCudaCppI32Buffer* stm_indices,
                                           const BulletOuCudaCppI32Buffer* nstm_indices,
                                           const BulletOuCudaCppF32Buffer* stm_eval,
                                           const BulletOuCudaCppF32Buffer* nstm_eval,
                                           const BulletOuCudaCppF32Buffer* outw,
                                           const BulletOuCudaCppF32Buffer* mean_output_gradients,
                                           BulletOuCudaCppF32Buffer* table_w_gradients,
                                           BulletOuCudaCppF32Buffer* table_b_gradients,
                                           BulletOuCudaCppF32Buffer* outw_gradients,
                                           BulletOuCudaCppF32Buffer* outb_gradients) {
    const size_t sparse = batch * max_active;
    if (validate_kppt(input_size, batch, max_active) != 0 ||
        validate_i32(ctx, stm_indices, sparse, "kppt stm_indices") != 0 ||
        validate_i32(ctx, nstm_indices, sparse, "kppt nstm_indices") != 0 ||
        validate_f32(ctx, stm_eval, batch, "kppt stm_eval") != 0 ||
        validate_f32(ctx, nstm_eval, batch, "kppt nstm_eval") != 0 || validate_f32(ctx, outw, 2, "kppt outw") != 0 ||
        validate_f32(ctx, mean_output_gradients, batch, "kppt mean_output_gradients") != 0 ||
        validate_f32(ctx, table_w_gradients, input_size, "kppt table_w_gradients") != 0 ||
        validate_f32(ctx, table_b_gradients, 1, "kppt table_b_gradients") != 0 ||
        validate_f32(ctx, outw_gradients, 2, "kppt outw_gradients") != 0 ||
        validate_f32(ctx, outb_gradients, 1, "kppt outb_gradients") != 0)
        return -1;
    if (set_device(ctx) != 0) return -1;
    if (fill_device(ctx, table_w_gradients->ptr, input_size, 0.0f, "kppt zero table gradients") != 0) return -1;
    const int grid = kppt_grid(ctx, batch);
    void* parts = nullptr;
    if (scratch_slot(ctx, kScratchLossPartials, static_cast<size_t>(grid) * kKpptVec * sizeof(float), &parts,
                     "cudaMalloc kppt partials") != 0)
        return -1;
    KpptArgs a{};
    a.stm = stm_indices->ptr;
    a.nstm = nstm_indices->ptr;
    a.max_active = static_cast<int>(max_active);
    a.batch = static_cast<int>(batch);
    a.input_size = static_cast<int>(input_size);
    a.outw = outw->ptr;
    a.stm_eval = const_cast<float*>(stm_eval->ptr);
    a.nstm_eval = const_cast<float*>(nstm_eval->ptr);
    a.mog_in = mean_output_gradients->ptr;
    a.table_grad = table_w_gradients->ptr;
    a.partials = static_cast<float*>(parts);
    kppt_kernel<2><<<grid, kWarps * 32, 0, ctx->stream>>>(a);
    if (check_launch("kppt backward launch") != 0) return -1;
    KpptSmall g{};
    g.grads[0] = table_b_gradients->ptr;
    g.grads[1] = outw_gradients->ptr;
    g.grads[2] = outb_gradients->ptr;
    kppt_small_kernel<<<1, 32, 0, ctx->stream>>>(static_cast<float*>(parts), grid, g, RangerArgs{}, 0, nullptr,
                                                 nullptr, 1.0f, 0);
    if (check_launch("kppt small gradient launch") != 0) return -1;
    return ok();
}

int bulletou_b200_kppt_train_step_device(
    BulletOuCudaCppContext* ctx, size_t input_size, size_t batch, size_t max_active,
    const BulletOuCudaCppI32Buffer* stm_indices, const BulletOuCudaCppI32Buffer* nstm_indices,
    const BulletOuCudaCppF32Buffer* targets, const BulletOuCudaCppF32Buffer* entry_weights,
    const BulletOuB200LossSpec* loss, const BulletOuB200RangerStep* ranger, BulletOuCudaCppF32Buffer* const* params,
    BulletOuCudaCppF32Buffer* const* momentum, BulletOuCudaCppF32Buffer* const* velocity,
    BulletOuCudaCppF32Buffer* const* slow_params, BulletOuCudaCppF32Buffer* output, BulletOuCudaCppF32Buffer* per_sample,
    BulletOuCudaCppF32Buffer* mean_output_gradients, BulletOuCudaCppF32Buffer* weighted_sum,
    BulletOuCudaCppF32Buffer* mean) {
    const size_t sparse = batch * max_active;
    LossArgs la{};
    if (validate_kppt(input_size, batch, max_active) != 0 ||
        validate_i32(ctx, stm_indices, sparse, "kppt stm_indices") != 0 ||
        validate_i32(ctx, nstm_indices, sparse, "kppt nstm_indices") != 0 ||
        validate_f32(ctx, targets, batch, "kppt targets") != 0 ||
        validate_f32(ctx, entry_weights, batch, "kppt entry_weights") != 0 ||
        validate_f32(ctx, output, batch, "kppt output") != 0 ||
        validate_f32(ctx, per_sample, batch, "kppt per_sample") != 0 ||
        validate_f32(ctx, mean_output_gradients, batch, "kppt mean_output_gradients") != 0 ||
        validate_f32(ctx, weighted_sum, 1, "kppt weighted_sum") != 0 || validate_f32(ctx, mean, 1, "kppt mean") != 0 ||
        loss_args(loss, batch, &la) != 0)
        return -1;
    if (params == nullptr || momentum == nullptr || velocity == nullptr || slow_params == nullptr || ranger == nullptr)
        return fail_message("kppt train step: parameter/state arrays and ranger step must not be null");
    const size_t lens[4] = {input_size, 1, 2, 1};
    static const char* names[4] = {"table_w", "table_b", "outw", "outb"};
    for (int i = 0; i < 4; ++i) {
        char n[64];
        std::snprintf(n, sizeof(n), "kppt %s", names[i]);
        if (validate_f32(ctx, params[i], lens[i], n) != 0 || validate_f32(ctx, momentum[i], lens[i], n) != 0 ||
            validate_f32(ctx, velocity[i], lens[i], n) != 0 || validate_f32(ctx, slow_params[i], lens[i], n) != 0)
            return -1;
    }
    if (ranger->norm_loss_rate != 0.0f) return fail_message("norm loss is not supported by the fused KPPT step");
    if (set_device(ctx) != 0) return -1;
    float* grad = nullptr;
    if (kppt_grad_table(ctx, input_size, &grad) != 0) return -1;
    const int grid = kppt_grid(ctx, batch);
    void* parts = nullptr;
    if (scratch_slot(ctx, kScratchLossPartials, static_cast<size_t>(grid) * kKpptVec * sizeof(float), &parts,
                     "cudaMalloc kppt partials") != 0)
        return -1;
    KpptArgs a{};
    a.stm = stm_indices->ptr;
    a.nstm = nstm_indices->ptr;
    a.max_active = static_cast<int>(max_active);
    a.batch = static_cast<int>(batch);
    a.input_size = static_cast<int>(input_size);
    a.table_w = params[0]->ptr;
    a.table_b = params[1]->ptr;
    a.outw = params[2]->ptr;
    a.outb = params[3]->ptr;
    a.stm_eval = nullptr;  // the fused step keeps no per-view evaluations
    a.nstm_eval = nullptr;
    a.output = output->ptr;
    a.targets = targets->ptr;
    a.entry_weights = entry_weights->ptr;
    a.loss = la;
    a.per_sample = per_sample->ptr;
    a.mog = mean_output_gradients->ptr;
    a.table_grad = grad;
    a.partials = static_cast<float*>(parts);
    if (input_size % kKpptKings == 0 && input_size >= static_cast<size_t>(kKpptKings)) {
        // king order: sort the 2B views by king block, sum the views, then the
        // outputs / loss in sample order, then the gradient scatter
        const int n_half = static_cast<int>(2 * batch);
        const size_t sort_ints = king_sort_scratch_ints<kKpptKeys>(static_cast<size_t>(n_half));
        void* sp = nullptr;
        if (scratch_slot(ctx, kScratchKingSort, (sort_ints + static_cast<size_t>(n_half)) * sizeof(int), &sp,
                         "cudaMalloc kppt king sort") != 0)
            return -1;
        int* sort_scratch = static_cast<int*>(sp);
        float* eval2 = reinterpret_cast<float*>(sort_scratch + sort_ints);
        KingSortOut ks{};
        const KingKey kk{static_cast<int>(input_size / kKpptKings), static_cast<int>(input_size),
                         static_cast<int>(max_active)};
        if (king_sort<kKpptKeys>(ctx, a.stm, a.nstm, n_half, kk, sort_scratch, nullptr, &ks) != 0) return -1;
        // about 4 resident warps' worth of half-positions per SM keeps the
        // king blocks in use to a few (9.6 MB each for the KPP table)
        const int sgrid = std::max(1, std::min((n_half + kWarps - 1) / kWarps, ctx->sm_count * 4));
        a.eval2 = eval2;
        kppt_view_kernel<<<sgrid, kWarps * 32, 0, ctx->stream>>>(a, ks.order, n_half, eval2);
        kppt_kernel<3><<<grid, kWarps * 32, 0, ctx->stream>>>(a);
        kppt_scatter_kernel<<<sgrid, kWarps * 32, 0, ctx->stream>>>(a, ks.order, n_half);
    } else {
        kppt_kernel<1><<<grid, kWarps * 32, 0, ctx->stream>>>(a);
    }
    if (check_launch("kppt train kernel launch") != 0) return -1;
    const RangerArgs ra = ranger_args_from(*ranger);
    KpptSmall g{};
    for (int i = 0; i < 3; ++i) {
        g.w[i] = params[i + 1]->ptr;
        g.m[i] = momentum[i + 1]->ptr;
        g.v[i] = velocity[i + 1]->ptr;
        g.s[i] = slow_params[i + 1]->ptr;
    }
    // small parameters read outw before it is updated: the table pass below
    // does not use them, and the kernel above has already consumed them.
    kppt_small_kernel<<<1, 32, 0, ctx->stream>>>(static_cast<float*>(parts), grid, g, ra, 1, weighted_sum->ptr,
                                                 mean->ptr, static_cast<float>(batch), loss->finalize_loss);
    if (check_launch("kppt small update launch") != 0) return -1;
    if (launch_ranger(ctx, input_size, ra, grad, params[0]->ptr, momentum[0]->ptr, velocity[0]->ptr,
                      slow_params[0]->ptr) != 0)
        return -1;
    return ok();
}

}  // extern "C"
