// SFNN LayerStack network (HalfKA_hm2 / HalfKA2 feature transformer, pairwise
// product, bucketed L1 -> dual SqrCReLU/CReLU -> L2 -> L3 + PSQT skip) on B200.
//
// Reference semantics: crates/cuda_cpp/cpp/bulletou_cuda_backend.cu
//   FT fold / gather / pairwise   cu:1180-1320, 1445-1456
//   L1 (stacked + shared factor)  cu:2207-2330
//   L2 input / L2 / L3            cu:2428-2600
//   backward                      cu:3324-3800, 4376-4440, 4950-4985,
//                                 launcher cu:8088-8700, 7983-8087
//   CPU statement of the same math: crates/bulletou_lib/src/value/fast_sfnn.rs:325-545
//   and the test oracle tiny_sfnn_backward_cpu (crates/cuda_cpp/src/lib.rs:14516-14710).
#pragma once

#include "common.cuh"
#include "loss.cuh"
#include "optim.cuh"

namespace bou {

constexpr int kSfnnPieces = 1629;          // piece-square inputs per king block
constexpr int kSfnnHm2Base = 73305;        // HalfKA_hm2: 45 mirrored kings x 1629
constexpr int kSfnnHalfka2Base = 131949;   // HalfKA2: 81 kings x 1629
constexpr int kSfnnKingKeys = 82;          // king sort keys (up to 81 kings + "no valid feature")
constexpr int kSfnnMaxL1Out = 32;
constexpr int kSfnnMaxL2 = 64;
constexpr int kSfnnMaxStacks = 127;        // bucket sort keys (stacks + "invalid bucket")
constexpr int kSfnnTile = 128;             // samples per bucket tile

// Quantisation-aware training (the reference runner's qat_l1 / qat_ft /
// qat_l2 / qat_l3, lib.rs:6332-6336; layer_qat.rs; cu:5993-6400, 9294-9470).
//   l1     L1 weights / bias folded with the shared factor, then fake-quantised
//          (i8 at 64, i32 at 8128); backward input gradients use them.
//   ft     fused step: FT rows folded with their virtual row, then fake-quantised
//          (i16 at 127); FT bias too.
//   l2/l3  fused step: L2 / L3 weights (64) and biases (8128) fake-quantised.
//   dense  l1 && l2 && l3: integer L1 / L2 / L3 on the 1/127 lattice with the
//          master L2 / L3 biases rounded to 8128, continuous activation STEs.
//   integer_ft  dense with FT QAT: combined from the engine's integer FT.
// Every gradient reaches the f32 masters through an identity STE.
struct SfnnQat {
    int l1;
    int ft;
    int l2;
    int l3;
    int dense;
    int integer_ft;
    const float* l2b_master;  // dense: master biases of the integer L2 / L3
    const float* l3b_master;
};

struct SfnnDims {
    int input_size;   // l0w rows (virtual rows included when factorized)
    int base;         // factorized: first virtual row (73305 / 131949); 0 otherwise
    int n_features;   // valid feature ids are [0, n_features)
    int width;        // ft_size
    int l1_hidden;
    int l1_out;
    int l1_skip;
    int l2_in;
    int l2_size;
    int stacks;
    int batch;
    int max_active;
    float ft_alpha;
    float shared_alpha;
    int has_l1f;
    int has_l2f;
    int has_l3f;
    SfnnQat qat;
};

// Factorized FT layout: input_size == base + 1629 for the two HalfKA bases
// (cu:1180-1184); every other size is a plain table.
inline int sfnn_factorized_base(size_t input_size) {
    if (input_size == static_cast<size_t>(kSfnnHalfka2Base + kSfnnPieces)) return kSfnnHalfka2Base;
    if (input_size == static_cast<size_t>(kSfnnHm2Base + kSfnnPieces)) return kSfnnHm2Base;
    return 0;
}

struct SfnnWeights {
    const float* l0w;
    const float* l0b;
    const float* l1w;   // [stacks][l1_out][width]
    const float* l1b;   // [stacks][l1_out]
    const float* l1fw;  // [width][l1_out] shared factor (null when absent)
    const float* l1fb;  // [l1_out]
    const float* l2w;   // [stacks][l2_size][l2_in]
    const float* l2b;   // [stacks][l2_size]
    const float* l2fw;  // [l2_size][l2_in]
    const float* l2fb;  // [l2_size]
    const float* l3w;   // [stacks][l2_size]
    const float* l3b;   // [stacks]
    const float* l3fw;  // [l2_size]
    const float* l3fb;  // [1]
};

// Forward activations, row-major per sample (the reference's buffers).
struct SfnnActivations {
    float* stm_l0;    // [B][width] ClippedReLU FT output, side to move
    float* nstm_l0;   // [B][width]
    float* combined;  // [B][width] pairwise products, stm half | nstm half
    float* l1;        // [B][l1_out]
    float* l2_input;  // [B][l2_in]
    float* l2;        // [B][l2_size]
    float* output;    // [B]
};

// Small-parameter gradient groups, packed in the reference's update order
// (lib.rs:8425-8730): l0b l1w l1b l1fw l1fb l2w l2b l2fw l2fb l3w l3b l3fw l3fb.
enum SfnnSmallGroup : int {
    kSfL0b = 0, kSfL1w, kSfL1b, kSfL1fw, kSfL1fb, kSfL2w, kSfL2b, kSfL2fw, kSfL2fb, kSfL3w, kSfL3b, kSfL3fw, kSfL3fb,
    kSfGroups
};

struct SfnnGroupLayout {
    size_t len[kSfGroups];
    size_t begin[kSfGroups + 1];
};

inline SfnnGroupLayout sfnn_group_layout(const SfnnDims& d) {
    SfnnGroupLayout g{};
    const size_t S = d.stacks, W = d.width, O = d.l1_out, L2 = d.l2_size, I2 = d.l2_in;
    g.len[kSfL0b] = W;
    g.len[kSfL1w] = S * O * W;
    g.len[kSfL1b] = S * O;
    g.len[kSfL1fw] = d.has_l1f ? W * O : 0;
    g.len[kSfL1fb] = d.has_l1f ? O : 0;
    g.len[kSfL2w] = S * L2 * I2;
    g.len[kSfL2b] = S * L2;
    g.len[kSfL2fw] = d.has_l2f ? L2 * I2 : 0;
    g.len[kSfL2fb] = d.has_l2f ? L2 : 0;
    g.len[kSfL3w] = S * L2;
    g.len[kSfL3b] = S;
    g.len[kSfL3fw] = d.has_l3f ? L2 : 0;
    g.len[kSfL3fb] = d.has_l3f ? 1 : 0;
    g.begin[0] = 0;
    for (int i = 0; i < kSfGroups; ++i) g.begin[i + 1] = g.begin[i] + g.len[i];
    return g;
}

// Checks an SFNN shape against this backend's limits and fills `d`
// (has_l*f are left zero).  0 or -1 with the error message set.
int sfnn_dims(size_t input_size, size_t ft_size, size_t l1_hidden, int l1_skip, size_t l2_size, size_t num_stacks,
              size_t batch, size_t max_active, float ft_alpha, float shared_alpha, SfnnDims* d);

}  // namespace bou
