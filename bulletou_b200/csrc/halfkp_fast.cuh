// Production-shape HalfKP kernels (l1 in {256, 512}, l2 = l3 = 32).
#pragma once

#include "common.cuh"
#include "loss.cuh"
#include "optim.cuh"
#include "sparse_rows.cuh"

namespace bou {

struct HalfkpDims {
    int input_size;
    int l1;
    int batch;
    int max_active;
};

inline bool halfkp_fast_shape(size_t l1, size_t l2, size_t l3, size_t batch, size_t max_active) {
    return (l1 == 256 || l1 == 512) && l2 == 32 && l3 == 32 && batch >= 1 && batch <= (1u << 26) &&
           max_active >= 1 && max_active <= 4096;
}

// Small-parameter groups in packed order l0b | l1w | l1b | l2w | l2b | outw | outb.
struct SmallGroups {
    float* w[7];
    float* m[7];
    float* v[7];
    float* s[7];
    int begin[8];  // packed offsets; begin[7] = total
};

struct HalfkpWeights {
    const float* l0w;
    const float* l0b;
    const float* l1w;
    const float* l1b;
    const float* l2w;
    const float* l2b;
    const float* outw;
    const float* outb;
};

// Per-position buffers of one step (device pointers).
struct HalfkpActivations {
    float* act;       // [B][2*l1]  ClippedReLU(FT) for stm | nstm  (the reference's `combined`)
    float* hidden1;   // [B][32]
    float* hidden2;   // [B][32]
    float* output;    // [B]
    // training only
    float* g1;        // [B][32] masked hidden1 gradient
    float* g2;        // [B][32] masked hidden2 gradient
    float* pregrad;   // [B][2*l1] masked FT pre-activation gradient
    float* per_sample;
    float* mog;
};

// Forward (and, with `loss`, the loss and the whole per-position backward).
// stm_l0/nstm_l0 (optional) receive the per-perspective activations too.
int halfkp_fast_forward_backward(BulletOuCudaCppContext* ctx, const HalfkpDims& d, const RowMap& map, const int* stm,
                                 const int* nstm, const HalfkpWeights& w, const HalfkpActivations& a,
                                 const float* targets, const float* entry_weights, const LossArgs* loss,
                                 float* stm_l0, float* nstm_l0);

// Batch reductions of every small-parameter gradient and the loss sum, then
// Ranger on the small groups (ranger != null) or the packed gradient written
// to dense_out; loss weighted_sum / mean written when finalize != 0.
int halfkp_fast_small_params(BulletOuCudaCppContext* ctx, const HalfkpDims& d, const HalfkpActivations& a,
                             const SmallGroups& groups, const RangerArgs* ranger, float* dense_out,
                             float* weighted_sum, float* mean, int finalize);

}  // namespace bou
