/*
 * bulletou_cuda_cpp.h — drop-in C ABI of the BulletOu cuda-cpp backend,
 * implemented from scratch for NVIDIA B200 (sm_100a) by libbulletou_b200.so.
 *
 * Every entry below has the same name, argument order, argument meaning,
 * ownership rule and error convention as the reference backend's C ABI in
 * yaneurao/BulletOu crates/cuda_cpp/cpp/bulletou_cuda_backend.cu (cited as
 * "cu:LINE"), whose Rust declarations live in crates/cuda_cpp/src/lib.rs
 * `mod ffi` (lib.rs:9605-10640).  A Rust build that links this library
 * instead of the reference's static `bulletou_cuda_cpp_backend` needs no
 * change to lib.rs.
 *
 * Conventions (cu:209-272, cu:5397-5570):
 *   - every call returns 0 on success; on failure it returns -1, or the
 *     cudaError_t code, and stores a message in a thread-local string read by
 *     bulletou_cuda_cpp_last_error();
 *   - handles are opaque and owned by the caller, who destroys them
 *     explicitly; destroy(NULL) is a no-op returning 0;
 *   - buffer arguments are validated (non-null, same device as the context,
 *     length >= the length the call needs) before anything is enqueued;
 *   - all work is enqueued asynchronously on the context's stream; only
 *     *_synchronize, *_download and *_host entries block.
 */
#ifndef BULLETOU_CUDA_CPP_H
#define BULLETOU_CUDA_CPP_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct BulletOuCudaCppContext BulletOuCudaCppContext;             /* cu:99 */
typedef struct BulletOuCudaCppF32Buffer BulletOuCudaCppF32Buffer;         /* cu:173 */
typedef struct BulletOuCudaCppI32Buffer BulletOuCudaCppI32Buffer;         /* cu:189 */
typedef struct BulletOuCudaCppPinnedF32Buffer BulletOuCudaCppPinnedF32Buffer; /* cu:195 */
typedef struct BulletOuCudaCppPinnedI32Buffer BulletOuCudaCppPinnedI32Buffer; /* cu:201 */
typedef struct BulletOuCudaCppEvent BulletOuCudaCppEvent;                 /* cu:207 */
typedef struct BulletOuCudaCppGraphExec BulletOuCudaCppGraphExec;         /* cu:212 */
typedef struct BulletOuCudaCppHalfMoments BulletOuCudaCppHalfMoments;     /* cu:179 (fp16 optimizer moments; not supported: calls that receive one fail) */

/* ---- errors, device, context (cu:9471-9677) ---- */
int bulletou_cuda_cpp_last_error(char* out, size_t out_len);                           /* cu:9471 */
int bulletou_cuda_cpp_device_name(int device, char* out, size_t out_len);              /* cu:9481 */
int bulletou_cuda_cpp_context_create(int device, BulletOuCudaCppContext** out);        /* cu:9503 */
int bulletou_cuda_cpp_context_destroy(BulletOuCudaCppContext* ctx);                    /* cu:9545 */
int bulletou_cuda_cpp_context_synchronize(BulletOuCudaCppContext* ctx);                /* cu:9667 */

/* ---- events and CUDA graphs (cu:9678-9857) ---- */
int bulletou_cuda_cpp_event_create(BulletOuCudaCppContext* ctx, BulletOuCudaCppEvent** out);   /* cu:9678 */
int bulletou_cuda_cpp_event_destroy(BulletOuCudaCppEvent* event);                               /* cu:9699 */
int bulletou_cuda_cpp_event_record(BulletOuCudaCppContext* ctx, BulletOuCudaCppEvent* event);   /* cu:9719 */
int bulletou_cuda_cpp_event_wait(BulletOuCudaCppContext* ctx, BulletOuCudaCppEvent* event);     /* cu:9730 */
int bulletou_cuda_cpp_event_synchronize(BulletOuCudaCppEvent* event);                           /* cu:9741 */
int bulletou_cuda_cpp_event_elapsed_ms(BulletOuCudaCppEvent* start, BulletOuCudaCppEvent* stop, float* out_ms); /* cu:9756 */
int bulletou_cuda_cpp_graph_begin_capture(BulletOuCudaCppContext* ctx);                         /* cu:9777 */
int bulletou_cuda_cpp_graph_end_capture(BulletOuCudaCppContext* ctx, BulletOuCudaCppGraphExec** out); /* cu:9788 */
int bulletou_cuda_cpp_graph_destroy(BulletOuCudaCppGraphExec* graph);                           /* cu:9820 */
int bulletou_cuda_cpp_graph_launch(BulletOuCudaCppContext* ctx, BulletOuCudaCppGraphExec* graph); /* cu:9847 */

/* ---- device and pinned buffers (cu:9858-10033) ---- */
int bulletou_cuda_cpp_f32_buffer_create(BulletOuCudaCppContext* ctx, size_t len, BulletOuCudaCppF32Buffer** out); /* cu:9858 */
int bulletou_cuda_cpp_f32_buffer_destroy(BulletOuCudaCppF32Buffer* buffer);                    /* cu:9882 */
int bulletou_cuda_cpp_i32_buffer_create(BulletOuCudaCppContext* ctx, size_t len, BulletOuCudaCppI32Buffer** out); /* cu:9902 */
int bulletou_cuda_cpp_i32_buffer_destroy(BulletOuCudaCppI32Buffer* buffer);                    /* cu:9926 */
int bulletou_cuda_cpp_pinned_f32_buffer_create(BulletOuCudaCppContext* ctx, size_t len, BulletOuCudaCppPinnedF32Buffer** out); /* cu:9946 */
int bulletou_cuda_cpp_pinned_f32_buffer_destroy(BulletOuCudaCppPinnedF32Buffer* buffer);       /* cu:9970 */
int bulletou_cuda_cpp_pinned_i32_buffer_create(BulletOuCudaCppContext* ctx, size_t len, BulletOuCudaCppPinnedI32Buffer** out); /* cu:9990 */
int bulletou_cuda_cpp_pinned_i32_buffer_destroy(BulletOuCudaCppPinnedI32Buffer* buffer);       /* cu:10014 */

/* ---- transfers and fills (cu:10034-10306) ---- */
int bulletou_cuda_cpp_f32_upload_staged(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* dst,
    BulletOuCudaCppPinnedF32Buffer* staging, const float* src, size_t len);                    /* cu:10034 */
int bulletou_cuda_cpp_i32_upload_staged(BulletOuCudaCppContext* ctx, BulletOuCudaCppI32Buffer* dst,
    BulletOuCudaCppPinnedI32Buffer* staging, const int* src, size_t len);                      /* cu:10059 */
int bulletou_cuda_cpp_i32_upload(BulletOuCudaCppContext* ctx, BulletOuCudaCppI32Buffer* dst, const int* src, size_t len); /* cu:10084 */
int bulletou_cuda_cpp_i32_download(BulletOuCudaCppContext* ctx, const BulletOuCudaCppI32Buffer* src, int* dst, size_t len); /* cu:10105 */
int bulletou_cuda_cpp_i32_copy_device(BulletOuCudaCppContext* ctx, BulletOuCudaCppI32Buffer* dst,
    const BulletOuCudaCppI32Buffer* src, size_t len);                                           /* cu:10131 */
int bulletou_cuda_cpp_f32_upload(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* dst, const float* src, size_t len); /* cu:10153 */
int bulletou_cuda_cpp_f32_download(BulletOuCudaCppContext* ctx, const BulletOuCudaCppF32Buffer* src, float* dst, size_t len); /* cu:10174 */
int bulletou_cuda_cpp_f32_copy_device(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* dst,
    const BulletOuCudaCppF32Buffer* src, size_t len);                                           /* cu:10200 */
int bulletou_cuda_cpp_f32_fill(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* dst, float value, size_t len); /* cu:10222 */
int bulletou_cuda_cpp_axpy_device(BulletOuCudaCppContext* ctx, size_t len, float a,
    const BulletOuCudaCppF32Buffer* x, const BulletOuCudaCppF32Buffer* y, BulletOuCudaCppF32Buffer* out); /* cu:10281 */
int bulletou_cuda_cpp_axpy_host(int device, size_t len, float a, const float* x, const float* y, float* out); /* cu:13536 */

/* ---- optimizers (cu:10554-10699, 14087) ----
 * RAdam + Lookahead ("Ranger") over one parameter group; gradients are reset
 * to zero in the same pass.  step_size/use_denom come from the host-side
 * RAdam step scale (lib.rs:9268-9288).  half_moments must be NULL here. */
int bulletou_cuda_cpp_ranger_update_device(
    BulletOuCudaCppContext* ctx, float norm_loss_rate, int norm_loss_before, size_t len,
    float gradient_factor, float learning_rate, float step_size, int use_denom, float decay,
    float beta1, float beta2, float epsilon, float min_weight, float max_weight,
    int do_lookahead, float lookahead_alpha, int clip_after_lookahead,
    BulletOuCudaCppF32Buffer* gradients, BulletOuCudaCppF32Buffer* weights,
    BulletOuCudaCppF32Buffer* momentum, BulletOuCudaCppF32Buffer* velocity,
    BulletOuCudaCppF32Buffer* slow_params, BulletOuCudaCppHalfMoments* half_moments);     /* cu:10576 */
int bulletou_cuda_cpp_ranger_update_host(
    int device, size_t len,
    float gradient_factor, float learning_rate, float step_size, int use_denom, float decay,
    float beta1, float beta2, float epsilon, float min_weight, float max_weight,
    int do_lookahead, float lookahead_alpha, int clip_after_lookahead,
    float* gradients, float* weights, float* momentum, float* velocity, float* slow_params); /* cu:14087 */
/* SGD with momentum and a compensated (two-float) master weight; `remainder`
 * is the low part of the weight. */
int bulletou_cuda_cpp_sgd_momentum_update_device(
    BulletOuCudaCppContext* ctx, size_t len, float gradient_factor, float learning_rate,
    float decay, float beta, float min_weight, float max_weight,
    BulletOuCudaCppF32Buffer* gradients, BulletOuCudaCppF32Buffer* weights,
    BulletOuCudaCppF32Buffer* momentum, BulletOuCudaCppF32Buffer* remainder,
    BulletOuCudaCppHalfMoments* half_moments);                                                 /* cu:10554 */

/* ---- HalfKP / KP NNUE  (input -> l1 (x2 perspectives) -> l2 -> l3 -> 1) ----
 * Shapes: l0w[input_size][l1] feature-major; l1w[2*l1][l2], l2w[l2][l3] and
 * outw[l3] input-major (cu:1083-1100).  Sparse inputs are [batch][max_active]
 * int32 feature ids; ids < 0 or >= input_size are padding.  When
 * input_size == 125388 + 1548 the table is factorized: rows [0,1548) are
 * virtual piece rows and feature f < 125388 reads rows 1548+f and f%1548
 * (cu:1004-1019). */
int bulletou_cuda_cpp_nnue_forward_device(
    BulletOuCudaCppContext* ctx, size_t input_size, size_t l1, size_t l2, size_t l3,
    size_t batch, size_t max_active,
    const BulletOuCudaCppI32Buffer* stm_indices, const BulletOuCudaCppI32Buffer* nstm_indices,
    const BulletOuCudaCppF32Buffer* l0w, const BulletOuCudaCppF32Buffer* l0b,
    const BulletOuCudaCppF32Buffer* l1w, const BulletOuCudaCppF32Buffer* l1b,
    const BulletOuCudaCppF32Buffer* l2w, const BulletOuCudaCppF32Buffer* l2b,
    const BulletOuCudaCppF32Buffer* outw, const BulletOuCudaCppF32Buffer* outb,
    BulletOuCudaCppF32Buffer* stm_l0, BulletOuCudaCppF32Buffer* nstm_l0,
    BulletOuCudaCppF32Buffer* combined, BulletOuCudaCppF32Buffer* hidden1,
    BulletOuCudaCppF32Buffer* hidden2, BulletOuCudaCppF32Buffer* output);                  /* cu:10864 */
int bulletou_cuda_cpp_nnue_forward_host(
    int device, size_t input_size, size_t l1, size_t l2, size_t l3, size_t batch, size_t max_active,
    const int* stm_indices, const int* nstm_indices,
    const float* l0w, const float* l0b, const float* l1w, const float* l1b,
    const float* l2w, const float* l2b, const float* outw, const float* outb, float* output); /* cu:11670 */
/* Backward of the forward above.  l0w_gradients ACCUMULATES (it is zeroed
 * first only when zero_l0_gradients != 0); every other gradient is
 * overwritten (cu:9142-9290). */
int bulletou_cuda_cpp_nnue_backward_device(
    BulletOuCudaCppContext* ctx, size_t input_size, size_t l1, size_t l2, size_t l3,
    size_t batch, size_t max_active,
    const BulletOuCudaCppI32Buffer* stm_indices, const BulletOuCudaCppI32Buffer* nstm_indices,
    const BulletOuCudaCppF32Buffer* combined, const BulletOuCudaCppF32Buffer* hidden1,
    const BulletOuCudaCppF32Buffer* hidden2, const BulletOuCudaCppF32Buffer* stm_l0,
    const BulletOuCudaCppF32Buffer* nstm_l0, const BulletOuCudaCppF32Buffer* l1w,
    const BulletOuCudaCppF32Buffer* l2w, const BulletOuCudaCppF32Buffer* outw,
    const BulletOuCudaCppF32Buffer* mean_output_gradients,
    BulletOuCudaCppF32Buffer* hidden2_gradients, BulletOuCudaCppF32Buffer* hidden1_gradients,
    BulletOuCudaCppF32Buffer* combined_gradients, BulletOuCudaCppF32Buffer* stm_l0_gradients,
    BulletOuCudaCppF32Buffer* nstm_l0_gradients, BulletOuCudaCppF32Buffer* l0w_gradients,
    BulletOuCudaCppF32Buffer* l0b_gradients, BulletOuCudaCppF32Buffer* l1w_gradients,
    BulletOuCudaCppF32Buffer* l1b_gradients, BulletOuCudaCppF32Buffer* l2w_gradients,
    BulletOuCudaCppF32Buffer* l2b_gradients, BulletOuCudaCppF32Buffer* outw_gradients,
    BulletOuCudaCppF32Buffer* outb_gradients, int zero_l0_gradients);                       /* cu:12069 */
int bulletou_cuda_cpp_nnue_train_warmup_device(
    BulletOuCudaCppContext* ctx, size_t input_size, size_t l1, size_t l2, size_t l3,
    size_t batch, size_t max_active,
    const BulletOuCudaCppF32Buffer* combined, const BulletOuCudaCppF32Buffer* hidden1,
    const BulletOuCudaCppF32Buffer* hidden2, const BulletOuCudaCppF32Buffer* l1w,
    const BulletOuCudaCppF32Buffer* l2w, const BulletOuCudaCppF32Buffer* outw,
    const BulletOuCudaCppF32Buffer* mean_output_gradients,
    BulletOuCudaCppF32Buffer* hidden2_gradients, BulletOuCudaCppF32Buffer* hidden1_gradients,
    BulletOuCudaCppF32Buffer* combined_gradients, BulletOuCudaCppF32Buffer* l1w_gradients,
    BulletOuCudaCppF32Buffer* l1b_gradients, BulletOuCudaCppF32Buffer* l2w_gradients,
    BulletOuCudaCppF32Buffer* l2b_gradients, BulletOuCudaCppF32Buffer* outw_gradients,
    BulletOuCudaCppF32Buffer* outb_gradients);                                                 /* cu:12169 */

/* ---- scalar value loss (cu:2719-2860, 8891-8968, 11809-11885, 11984) ----
 * kind 0 = sigmoid(out*inv_scale) vs target, |err|^pow_exp; kind 1 = win-rate
 * model (loss_param = in_offset/scaling, output_inv_scale = output scale);
 * kind 2 = BCE with logits (loss_param = error-weight k, 0 = plain). */
int bulletou_cuda_cpp_scalar_loss_device_with_finalize(
    BulletOuCudaCppContext* ctx, int kind, float output_inv_scale, float loss_pow_exp, float loss_param,
    size_t batch, const BulletOuCudaCppF32Buffer* outputs, const BulletOuCudaCppF32Buffer* targets,
    const BulletOuCudaCppF32Buffer* entry_weights, BulletOuCudaCppF32Buffer* per_sample,
    BulletOuCudaCppF32Buffer* mean_output_gradients, BulletOuCudaCppF32Buffer* weighted_sum,
    BulletOuCudaCppF32Buffer* mean, int finalize_loss);                                        /* cu:11809 */
int bulletou_cuda_cpp_scalar_loss_device(
    BulletOuCudaCppContext* ctx, int kind, float output_inv_scale, float loss_pow_exp, float unused_loss_param,
    size_t batch, const BulletOuCudaCppF32Buffer* outputs, const BulletOuCudaCppF32Buffer* targets,
    const BulletOuCudaCppF32Buffer* entry_weights, BulletOuCudaCppF32Buffer* per_sample,
    BulletOuCudaCppF32Buffer* mean_output_gradients, BulletOuCudaCppF32Buffer* weighted_sum,
    BulletOuCudaCppF32Buffer* mean);                                                           /* cu:11856 */
int bulletou_cuda_cpp_scalar_loss_host(
    int device, int kind, float output_inv_scale, float loss_pow_exp, float unused_loss_param, size_t batch,
    const float* outputs, const float* targets, const float* entry_weights,
    float* per_sample, float* mean_output_gradients, float* weighted_sum, float* mean);       /* cu:11984 */

/* ---- KPPT scalar tables (cu:8970-9140, 11887-11983) ----
 * out = outw[0]*(b + sum table_w[stm ids]) + outw[1]*(b + sum table_w[nstm ids]) + outb.
 * The backward zero-fills every gradient it writes, then accumulates. */
int bulletou_cuda_cpp_kppt_forward_device(
    BulletOuCudaCppContext* ctx, size_t input_size, size_t batch, size_t max_active,
    const BulletOuCudaCppI32Buffer* stm_indices, const BulletOuCudaCppI32Buffer* nstm_indices,
    const BulletOuCudaCppF32Buffer* table_w, const BulletOuCudaCppF32Buffer* table_b,
    const BulletOuCudaCppF32Buffer* outw, const BulletOuCudaCppF32Buffer* outb,
    BulletOuCudaCppF32Buffer* stm_eval, BulletOuCudaCppF32Buffer* nstm_eval,
    BulletOuCudaCppF32Buffer* outputs);                                                        /* cu:11887 */
int bulletou_cuda_cpp_kppt_backward_device(
    BulletOuCudaCppContext* ctx, size_t input_size, size_t batch, size_t max_active,
    const BulletOuCudaCppI32Buffer* stm_indices, const BulletOuCudaCppI32Buffer* nstm_indices,
    const BulletOuCudaCppF32Buffer* stm_eval, const BulletOuCudaCppF32Buffer* nstm_eval,
    const BulletOuCudaCppF32Buffer* outw, const BulletOuCudaCppF32Buffer* mean_output_gradients,
    BulletOuCudaCppF32Buffer* table_w_gradients, BulletOuCudaCppF32Buffer* table_b_gradients,
    BulletOuCudaCppF32Buffer* outw_gradients, BulletOuCudaCppF32Buffer* outb_gradients);      /* cu:11934 */

/* SFNN LayerStack forward (HalfKA_hm2 / HalfKA2 FT, pairwise product, bucketed
 * L1 -> SqrCReLU|CReLU -> L2 -> L3 + PSQT skip).  Same arguments as the
 * reference (cu:11329).  Supported: dense L1 (l1_group_count <= 1, no
 * common+shard), the shared L1/L2/L3 factors (has_l*f), the FT factorizer
 * (input_size = base + 1629, virtual rows folded with ft_factorizer_alpha);
 * bucket-axis factorizers, residual count gates and the L1 QAT scratch
 * (qat_l1w / qat_l1b) return -1 with "unsupported on this backend".
 * folded_l0w (optional, input_size*ft_size) is used as fold scratch. */
int bulletou_cuda_cpp_sfnn_forward_device(
    BulletOuCudaCppContext* ctx, size_t input_size, size_t ft_size, size_t l1_hidden, int l1_skip,
    size_t l2_size, size_t num_stacks, size_t l1_group_count, size_t l1_common_size,
    size_t l1_shard_size, size_t factorizer_king_axis_dim, size_t factorizer_hand_axis_dim,
    size_t batch, size_t max_active, const BulletOuCudaCppI32Buffer* stm_indices,
    const BulletOuCudaCppI32Buffer* nstm_indices, const BulletOuCudaCppI32Buffer* buckets,
    const BulletOuCudaCppF32Buffer* l0w, BulletOuCudaCppF32Buffer* folded_l0w,
    const BulletOuCudaCppF32Buffer* l0b, const BulletOuCudaCppF32Buffer* l1w,
    const BulletOuCudaCppF32Buffer* l1b, const BulletOuCudaCppF32Buffer* l1fw,
    const BulletOuCudaCppF32Buffer* l1fb, int has_l1f, const BulletOuCudaCppF32Buffer* l1axw,
    const BulletOuCudaCppF32Buffer* l1axb, int has_l1ax, const BulletOuCudaCppF32Buffer* l2w,
    const BulletOuCudaCppF32Buffer* l2b, const BulletOuCudaCppF32Buffer* l2fw,
    const BulletOuCudaCppF32Buffer* l2fb, int has_l2f, const BulletOuCudaCppF32Buffer* l2axw,
    const BulletOuCudaCppF32Buffer* l2axb, int has_l2ax, const BulletOuCudaCppF32Buffer* l3w,
    const BulletOuCudaCppF32Buffer* l3b, const BulletOuCudaCppF32Buffer* l3fw,
    const BulletOuCudaCppF32Buffer* l3fb, int has_l3f, const BulletOuCudaCppF32Buffer* l3axw,
    const BulletOuCudaCppF32Buffer* l3axb, int has_l3ax, int use_king_axis, int use_hand_axis,
    int use_progress_axis, int use_king_hand_pair, int use_king_progress_pair,
    int use_hand_progress_pair, float ft_factorizer_alpha, float factorizer_shared_alpha,
    float factorizer_king_axis_alpha, float factorizer_hand_axis_alpha,
    float factorizer_progress_axis_alpha, float factorizer_pair_alpha,
    const BulletOuCudaCppF32Buffer* residual_count_gates,
    const BulletOuCudaCppF32Buffer* factorizer_axis_confidences, BulletOuCudaCppF32Buffer* stm_l0,
    BulletOuCudaCppF32Buffer* nstm_l0, BulletOuCudaCppF32Buffer* combined, BulletOuCudaCppF32Buffer* l1,
    BulletOuCudaCppF32Buffer* l2_input, BulletOuCudaCppF32Buffer* l2, BulletOuCudaCppF32Buffer* output,
    BulletOuCudaCppF32Buffer* qat_l1w, BulletOuCudaCppF32Buffer* qat_l1b, int refresh_qat_l1); /* cu:11329 */

/* SFNN training backward (cu:12882): parameter gradients are accumulated into
 * the given buffers (cleared first when zero_parameter_gradients != 0); the
 * FT gradient includes the virtual factor rows (alpha * sum over king blocks,
 * overwritten as in cu:4950-4985); intermediate gradient buffers are written.
 * Same support limits as the forward. */
int bulletou_cuda_cpp_sfnn_backward_train_device(
    BulletOuCudaCppContext* ctx, size_t input_size, size_t ft_size, size_t l1_hidden, int l1_skip,
    size_t l2_size, size_t num_stacks, size_t l1_group_count, size_t l1_common_size,
    size_t l1_shard_size, size_t factorizer_king_axis_dim, size_t factorizer_hand_axis_dim,
    size_t batch, size_t max_active, const BulletOuCudaCppI32Buffer* stm_indices,
    const BulletOuCudaCppI32Buffer* nstm_indices, const BulletOuCudaCppI32Buffer* buckets,
    const BulletOuCudaCppF32Buffer* stm_l0, const BulletOuCudaCppF32Buffer* nstm_l0,
    const BulletOuCudaCppF32Buffer* combined, const BulletOuCudaCppF32Buffer* l1,
    const BulletOuCudaCppF32Buffer* l2_input, const BulletOuCudaCppF32Buffer* l2,
    const BulletOuCudaCppF32Buffer* l1w, const BulletOuCudaCppF32Buffer* qat_l1w,
    const BulletOuCudaCppF32Buffer* l1fw, int has_l1f, const BulletOuCudaCppF32Buffer* l1axw,
    int has_l1ax, const BulletOuCudaCppF32Buffer* l2w, const BulletOuCudaCppF32Buffer* l2fw,
    int has_l2f, const BulletOuCudaCppF32Buffer* l2axw, int has_l2ax,
    const BulletOuCudaCppF32Buffer* l3w, const BulletOuCudaCppF32Buffer* l3fw, int has_l3f,
    const BulletOuCudaCppF32Buffer* l3axw, int has_l3ax, int use_king_axis, int use_hand_axis,
    int use_progress_axis, int use_king_hand_pair, int use_king_progress_pair,
    int use_hand_progress_pair, float ft_factorizer_alpha, float factorizer_shared_alpha,
    float factorizer_king_axis_alpha, float factorizer_hand_axis_alpha,
    float factorizer_progress_axis_alpha, float factorizer_pair_alpha,
    const BulletOuCudaCppF32Buffer* residual_count_gates,
    const BulletOuCudaCppF32Buffer* factorizer_axis_confidences,
    const BulletOuCudaCppF32Buffer* mean_output_gradients, BulletOuCudaCppF32Buffer* l2_gradients,
    BulletOuCudaCppF32Buffer* l1_gradients, BulletOuCudaCppF32Buffer* l2_input_gradients,
    BulletOuCudaCppF32Buffer* combined_gradients, BulletOuCudaCppF32Buffer* stm_l0_gradients,
    BulletOuCudaCppF32Buffer* nstm_l0_gradients, BulletOuCudaCppF32Buffer* stm_l0_pre_gradients,
    BulletOuCudaCppF32Buffer* nstm_l0_pre_gradients, BulletOuCudaCppF32Buffer* l0w_gradients,
    BulletOuCudaCppF32Buffer* l0b_gradients, BulletOuCudaCppF32Buffer* l1w_gradients,
    BulletOuCudaCppF32Buffer* l1b_gradients, BulletOuCudaCppF32Buffer* l1fw_gradients,
    BulletOuCudaCppF32Buffer* l1fb_gradients, BulletOuCudaCppF32Buffer* l1axw_gradients,
    BulletOuCudaCppF32Buffer* l1axb_gradients, BulletOuCudaCppF32Buffer* l2w_gradients,
    BulletOuCudaCppF32Buffer* l2b_gradients, BulletOuCudaCppF32Buffer* l2fw_gradients,
    BulletOuCudaCppF32Buffer* l2fb_gradients, BulletOuCudaCppF32Buffer* l2axw_gradients,
    BulletOuCudaCppF32Buffer* l2axb_gradients, BulletOuCudaCppF32Buffer* l3w_gradients,
    BulletOuCudaCppF32Buffer* l3b_gradients, BulletOuCudaCppF32Buffer* l3fw_gradients,
    BulletOuCudaCppF32Buffer* l3fb_gradients, BulletOuCudaCppF32Buffer* l3axw_gradients,
    BulletOuCudaCppF32Buffer* l3axb_gradients, int zero_parameter_gradients,
    BulletOuCudaCppF32Buffer* entry_weights);                                            /* cu:12882 */

/* ---- SFNN quantisation-aware training (cu:9294-9470; driver layer_qat.rs) ----
 * bulletou_layer_qat: dst = fake-quantised src.  scale 127 (FT weights or
 * bias, i16 bounds; with vr > 0 the FT rows are folded with virtual row
 * base + f % vr as src[f] + alpha * src[virtual] and the virtual rows zeroed),
 * 64 (dense weights, i8) or 8128 (dense biases, i32); lo / hi are implied by
 * the scale.  bulletou_layer_qat_nonzero sets flag[0] = 1 when any element of
 * w or b is nonzero.  bulletou_dense_qat_begin / _end bracket a dense-QAT
 * forward + backward: the SFNN entries of the context then run integer
 * L1 / L2 / L3 with the given master L2 / L3 biases (and the engine's integer
 * FT when integer_ft), using the L1 QAT scratch of the forward entry. */
int bulletou_layer_qat(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* src, BulletOuCudaCppF32Buffer* dst,
    float scale, float lo, float hi, size_t base, size_t vr, size_t width, float alpha);             /* cu:9441 */
int bulletou_layer_qat_nonzero(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* w,
    BulletOuCudaCppF32Buffer* b, BulletOuCudaCppF32Buffer* flag);                                     /* cu:9462 */
int bulletou_dense_qat_begin(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* l2_bias,
    BulletOuCudaCppF32Buffer* l3_bias, size_t batch, size_t l1_out, size_t l2_size, size_t stacks,
    int integer_ft);                                                                                  /* cu:9356 */
void bulletou_dense_qat_end(BulletOuCudaCppContext* ctx);                                             /* cu:9375 */

/* cu:13485-13504: activation statistics of a forward workspace, 5 x 256
 * partials (FT outputs at 1, L2-input square / normal branches at 1, L2 at 1,
 * output squared). */
int bulletou_cuda_cpp_sfnn_validation_stats(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* stm,
    BulletOuCudaCppF32Buffer* nstm, BulletOuCudaCppF32Buffer* l2_input, BulletOuCudaCppF32Buffer* l2,
    BulletOuCudaCppF32Buffer* output, BulletOuCudaCppF32Buffer* partials, size_t batch, size_t ft, size_t hidden,
    size_t l2_size);

/* cu:13506-13531: per-unit saturation counts [ft + stacks * (1 + 2 hidden + width)]. */
int bulletou_cuda_cpp_sfnn_unit_stats(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* stm,
    BulletOuCudaCppF32Buffer* nstm, BulletOuCudaCppF32Buffer* input, BulletOuCudaCppF32Buffer* l2,
    BulletOuCudaCppI32Buffer* buckets, BulletOuCudaCppI32Buffer* counts, size_t batch, size_t ft, size_t hidden,
    size_t width, size_t stacks);

/* ---- FP16 feature-transformer options (cu:9598-9665) ----
 * This backend keeps the FT weights, gradients and activations in f32.
 * Turning an option off (enabled = 0) succeeds; turning one on returns -1
 * with "unsupported on this backend".  There is no FP16 scratch, so the
 * release entry only checks its context and the clipped-gradient counter
 * always reads 0. */
int bulletou_cuda_cpp_context_set_sfnn_ft_fp16(BulletOuCudaCppContext* ctx, int enabled);  /* cu:9624 */
int bulletou_cuda_cpp_context_set_sfnn_ft_fp16_grad(BulletOuCudaCppContext* ctx, int enabled);  /* cu:9604 */
int bulletou_cuda_cpp_context_set_sfnn_ft_fp16_act(BulletOuCudaCppContext* ctx, int enabled);  /* cu:9598 */
int bulletou_cuda_cpp_context_release_sfnn_ft_fp16_scratch(BulletOuCudaCppContext* ctx, int release_weights,
    int release_gradients, int release_activations);  /* cu:9633 */
int bulletou_cuda_cpp_context_take_ft_half_grad_clipped(BulletOuCudaCppContext* ctx, unsigned long long* out);  /* cu:9610 */
int bulletou_test_sfnn_ft_fp16_scratch_sizes(BulletOuCudaCppContext* ctx, size_t* weights, size_t* gradients,
    size_t* activations);  /* cu:9658 */

/* ---- FP16 optimizer moments (cu:10366-10420) ----
 * Not supported: create returns -1 with "unsupported on this backend" and
 * leaves *out NULL; decode / take_clipped on a NULL state fail; destroy(NULL)
 * is a no-op returning 0. */
int bulletou_cuda_cpp_ft_half_moments_create(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* momentum,
    BulletOuCudaCppF32Buffer* velocity, size_t len, int sgd, BulletOuCudaCppHalfMoments** out);  /* cu:10366 */
int bulletou_cuda_cpp_ft_half_moments_decode(BulletOuCudaCppContext* ctx, BulletOuCudaCppHalfMoments* state,
    BulletOuCudaCppF32Buffer* momentum, BulletOuCudaCppF32Buffer* velocity);  /* cu:10396 */
int bulletou_cuda_cpp_ft_half_moments_take_clipped(BulletOuCudaCppContext* ctx,
    BulletOuCudaCppHalfMoments* state, unsigned long long* out);  /* cu:10407 */
int bulletou_cuda_cpp_ft_half_moments_destroy(BulletOuCudaCppHalfMoments* state);  /* cu:10420 */

/* ---- per-bucket ("dirty") Ranger over a stacked parameter group (cu:10700) ----
 * The group is [stacks][stride]; only the strides of the buckets listed in
 * dirty_buckets (negative ids and rows past len skipped) are stepped and
 * their gradients reset.  learning_rate == 0 only clears those gradients.
 * Norm loss applies to the whole group, before or after the step as
 * norm_loss_before says; the lookahead follows the step. */
int bulletou_cuda_cpp_ranger_update_stacked_dirty_device(BulletOuCudaCppContext* ctx, float norm_loss_rate,
    int norm_loss_before, size_t len, size_t stride, size_t dirty_count, float gradient_factor,
    float learning_rate, float step_size, int use_denom, float decay, float beta1, float beta2,
    float epsilon, float min_weight, float max_weight, int do_lookahead, float lookahead_alpha,
    int clip_after_lookahead, const BulletOuCudaCppI32Buffer* dirty_buckets,
    BulletOuCudaCppF32Buffer* gradients, BulletOuCudaCppF32Buffer* weights,
    BulletOuCudaCppF32Buffer* momentum, BulletOuCudaCppF32Buffer* velocity,
    BulletOuCudaCppF32Buffer* slow_params);  /* cu:10700 */

/* ---- SFNN backward variants and the quantised proxy ----
 * sfnn_backward_device (cu:12274): the training backward with every parameter
 * gradient cleared first.  sfnn_backward_train_profile_device (cu:13080): the
 * training backward with stage times written to profile_ms[0..7): zeroing,
 * L3, L2, L2 input, L1, pairwise + FT, total (ms).  Here the L3 / L2 / L2-input
 * backward is one kernel, so its time is reported under L3 and the L2 and
 * L2-input entries read 0.  profile_ms may be NULL; otherwise
 * profile_ms_len >= 7.  sfnn_build_quantized_proxy_device (cu:10937): the
 * engine-lattice proxy of the f32 masters (FT rows folded with their virtual
 * row and rounded to 1/127 in i16 range, FT bias likewise, dense weights
 * folded with their shared factor and rounded to 1/64 in i8 range, dense
 * biases to 1/8128 in i32 range); skip_ft_weights leaves dst_l0w untouched.
 * Same support limits as the forward (no axis factorizers, residual gates or
 * grouped L1; no BatchNorm on this backend). */
int bulletou_cuda_cpp_sfnn_backward_device(BulletOuCudaCppContext* ctx, size_t input_size, size_t ft_size,
    size_t l1_hidden, int l1_skip, size_t l2_size, size_t num_stacks, size_t l1_group_count,
    size_t l1_common_size, size_t l1_shard_size, size_t factorizer_king_axis_dim,
    size_t factorizer_hand_axis_dim, size_t batch, size_t max_active,
    const BulletOuCudaCppI32Buffer* stm_indices, const BulletOuCudaCppI32Buffer* nstm_indices,
    const BulletOuCudaCppI32Buffer* buckets, const BulletOuCudaCppF32Buffer* stm_l0,
    const BulletOuCudaCppF32Buffer* nstm_l0, const BulletOuCudaCppF32Buffer* combined,
    const BulletOuCudaCppF32Buffer* l1, const BulletOuCudaCppF32Buffer* l2_input,
    const BulletOuCudaCppF32Buffer* l2, const BulletOuCudaCppF32Buffer* l1w,
    const BulletOuCudaCppF32Buffer* qat_l1w, const BulletOuCudaCppF32Buffer* l1fw, int has_l1f,
    const BulletOuCudaCppF32Buffer* l1axw, int has_l1ax, const BulletOuCudaCppF32Buffer* l2w,
    const BulletOuCudaCppF32Buffer* l2fw, int has_l2f, const BulletOuCudaCppF32Buffer* l2axw, int has_l2ax,
    const BulletOuCudaCppF32Buffer* l3w, const BulletOuCudaCppF32Buffer* l3fw, int has_l3f,
    const BulletOuCudaCppF32Buffer* l3axw, int has_l3ax, int use_king_axis, int use_hand_axis,
    int use_progress_axis, int use_king_hand_pair, int use_king_progress_pair, int use_hand_progress_pair,
    float ft_factorizer_alpha, float factorizer_shared_alpha, float factorizer_king_axis_alpha,
    float factorizer_hand_axis_alpha, float factorizer_progress_axis_alpha, float factorizer_pair_alpha,
    const BulletOuCudaCppF32Buffer* residual_count_gates,
    const BulletOuCudaCppF32Buffer* factorizer_axis_confidences,
    const BulletOuCudaCppF32Buffer* mean_output_gradients, BulletOuCudaCppF32Buffer* l2_gradients,
    BulletOuCudaCppF32Buffer* l1_gradients, BulletOuCudaCppF32Buffer* l2_input_gradients,
    BulletOuCudaCppF32Buffer* combined_gradients, BulletOuCudaCppF32Buffer* stm_l0_gradients,
    BulletOuCudaCppF32Buffer* nstm_l0_gradients, BulletOuCudaCppF32Buffer* stm_l0_pre_gradients,
    BulletOuCudaCppF32Buffer* nstm_l0_pre_gradients, BulletOuCudaCppF32Buffer* l0w_gradients,
    BulletOuCudaCppF32Buffer* l0b_gradients, BulletOuCudaCppF32Buffer* l1w_gradients,
    BulletOuCudaCppF32Buffer* l1b_gradients, BulletOuCudaCppF32Buffer* l1fw_gradients,
    BulletOuCudaCppF32Buffer* l1fb_gradients, BulletOuCudaCppF32Buffer* l1axw_gradients,
    BulletOuCudaCppF32Buffer* l1axb_gradients, BulletOuCudaCppF32Buffer* l2w_gradients,
    BulletOuCudaCppF32Buffer* l2b_gradients, BulletOuCudaCppF32Buffer* l2fw_gradients,
    BulletOuCudaCppF32Buffer* l2fb_gradients, BulletOuCudaCppF32Buffer* l2axw_gradients,
    BulletOuCudaCppF32Buffer* l2axb_gradients, BulletOuCudaCppF32Buffer* l3w_gradients,
    BulletOuCudaCppF32Buffer* l3b_gradients, BulletOuCudaCppF32Buffer* l3fw_gradients,
    BulletOuCudaCppF32Buffer* l3fb_gradients, BulletOuCudaCppF32Buffer* l3axw_gradients,
    BulletOuCudaCppF32Buffer* l3axb_gradients);  /* cu:12274 */
int bulletou_cuda_cpp_sfnn_backward_train_profile_device(BulletOuCudaCppContext* ctx, size_t input_size,
    size_t ft_size, size_t l1_hidden, int l1_skip, size_t l2_size, size_t num_stacks, size_t l1_group_count,
    size_t l1_common_size, size_t l1_shard_size, size_t factorizer_king_axis_dim,
    size_t factorizer_hand_axis_dim, size_t batch, size_t max_active,
    const BulletOuCudaCppI32Buffer* stm_indices, const BulletOuCudaCppI32Buffer* nstm_indices,
    const BulletOuCudaCppI32Buffer* buckets, const BulletOuCudaCppF32Buffer* stm_l0,
    const BulletOuCudaCppF32Buffer* nstm_l0, const BulletOuCudaCppF32Buffer* combined,
    const BulletOuCudaCppF32Buffer* l1, const BulletOuCudaCppF32Buffer* l2_input,
    const BulletOuCudaCppF32Buffer* l2, const BulletOuCudaCppF32Buffer* l1w,
    const BulletOuCudaCppF32Buffer* qat_l1w, const BulletOuCudaCppF32Buffer* l1fw, int has_l1f,
    const BulletOuCudaCppF32Buffer* l1axw, int has_l1ax, const BulletOuCudaCppF32Buffer* l2w,
    const BulletOuCudaCppF32Buffer* l2fw, int has_l2f, const BulletOuCudaCppF32Buffer* l2axw, int has_l2ax,
    const BulletOuCudaCppF32Buffer* l3w, const BulletOuCudaCppF32Buffer* l3fw, int has_l3f,
    const BulletOuCudaCppF32Buffer* l3axw, int has_l3ax, int use_king_axis, int use_hand_axis,
    int use_progress_axis, int use_king_hand_pair, int use_king_progress_pair, int use_hand_progress_pair,
    float ft_factorizer_alpha, float factorizer_shared_alpha, float factorizer_king_axis_alpha,
    float factorizer_hand_axis_alpha, float factorizer_progress_axis_alpha, float factorizer_pair_alpha,
    const BulletOuCudaCppF32Buffer* residual_count_gates,
    const BulletOuCudaCppF32Buffer* factorizer_axis_confidences,
    const BulletOuCudaCppF32Buffer* mean_output_gradients, BulletOuCudaCppF32Buffer* l2_gradients,
    BulletOuCudaCppF32Buffer* l1_gradients, BulletOuCudaCppF32Buffer* l2_input_gradients,
    BulletOuCudaCppF32Buffer* combined_gradients, BulletOuCudaCppF32Buffer* stm_l0_gradients,
    BulletOuCudaCppF32Buffer* nstm_l0_gradients, BulletOuCudaCppF32Buffer* stm_l0_pre_gradients,
    BulletOuCudaCppF32Buffer* nstm_l0_pre_gradients, BulletOuCudaCppF32Buffer* l0w_gradients,
    BulletOuCudaCppF32Buffer* l0b_gradients, BulletOuCudaCppF32Buffer* l1w_gradients,
    BulletOuCudaCppF32Buffer* l1b_gradients, BulletOuCudaCppF32Buffer* l1fw_gradients,
    BulletOuCudaCppF32Buffer* l1fb_gradients, BulletOuCudaCppF32Buffer* l1axw_gradients,
    BulletOuCudaCppF32Buffer* l1axb_gradients, BulletOuCudaCppF32Buffer* l2w_gradients,
    BulletOuCudaCppF32Buffer* l2b_gradients, BulletOuCudaCppF32Buffer* l2fw_gradients,
    BulletOuCudaCppF32Buffer* l2fb_gradients, BulletOuCudaCppF32Buffer* l2axw_gradients,
    BulletOuCudaCppF32Buffer* l2axb_gradients, BulletOuCudaCppF32Buffer* l3w_gradients,
    BulletOuCudaCppF32Buffer* l3b_gradients, BulletOuCudaCppF32Buffer* l3fw_gradients,
    BulletOuCudaCppF32Buffer* l3fb_gradients, BulletOuCudaCppF32Buffer* l3axw_gradients,
    BulletOuCudaCppF32Buffer* l3axb_gradients, int zero_parameter_gradients, float* profile_ms,
    size_t profile_ms_len);  /* cu:13080 */
int bulletou_cuda_cpp_sfnn_build_quantized_proxy_device(BulletOuCudaCppContext* ctx, size_t src_input_size,
    size_t dst_input_size, size_t virtual_rows, size_t ft_size, size_t l1_hidden, int l1_skip,
    size_t l2_size, size_t num_stacks, size_t l1_group_count, size_t l1_common_size, size_t l1_shard_size,
    size_t factorizer_king_axis_dim, size_t factorizer_hand_axis_dim,
    const BulletOuCudaCppF32Buffer* src_l0w, const BulletOuCudaCppF32Buffer* src_l0b,
    const BulletOuCudaCppF32Buffer* src_l1w, const BulletOuCudaCppF32Buffer* src_l1b,
    const BulletOuCudaCppF32Buffer* src_l1fw, const BulletOuCudaCppF32Buffer* src_l1fb, int has_l1f,
    const BulletOuCudaCppF32Buffer* src_l1axw, const BulletOuCudaCppF32Buffer* src_l1axb, int has_l1ax,
    const BulletOuCudaCppF32Buffer* src_l2w, const BulletOuCudaCppF32Buffer* src_l2b,
    const BulletOuCudaCppF32Buffer* src_l2fw, const BulletOuCudaCppF32Buffer* src_l2fb, int has_l2f,
    const BulletOuCudaCppF32Buffer* src_l2axw, const BulletOuCudaCppF32Buffer* src_l2axb, int has_l2ax,
    const BulletOuCudaCppF32Buffer* src_l3w, const BulletOuCudaCppF32Buffer* src_l3b,
    const BulletOuCudaCppF32Buffer* src_l3fw, const BulletOuCudaCppF32Buffer* src_l3fb, int has_l3f,
    const BulletOuCudaCppF32Buffer* src_l3axw, const BulletOuCudaCppF32Buffer* src_l3axb, int has_l3ax,
    int use_king_axis, int use_hand_axis, int use_progress_axis, int use_king_hand_pair,
    int use_king_progress_pair, int use_hand_progress_pair, float ft_factorizer_alpha,
    float factorizer_shared_alpha, float factorizer_king_axis_alpha, float factorizer_hand_axis_alpha,
    float factorizer_progress_axis_alpha, float factorizer_pair_alpha,
    const BulletOuCudaCppF32Buffer* residual_count_gates,
    const BulletOuCudaCppF32Buffer* factorizer_axis_confidences, BulletOuCudaCppF32Buffer* dst_l0w,
    BulletOuCudaCppF32Buffer* dst_l0b, BulletOuCudaCppF32Buffer* dst_l1w, BulletOuCudaCppF32Buffer* dst_l1b,
    BulletOuCudaCppF32Buffer* dst_l2w, BulletOuCudaCppF32Buffer* dst_l2b, BulletOuCudaCppF32Buffer* dst_l3w,
    BulletOuCudaCppF32Buffer* dst_l3b, int skip_ft_weights);  /* cu:10937 */

/* ---- small per-row / per-bucket utilities ----
 * scale_axis_rows (cu:10245): values[r * row_len + j] *= row_scales[r].
 * residual_count_decay (cu:13411): gradients[s][j] += 2 * decay[s] * weights[s][j]
 * over the dirty buckets (all buckets when dirty_count == 0).
 * residual_count_gates (cu:13451): gradients[s][j] *= gates[s] over the same set.
 * center_scale (cu:13993): dst[i] = src[i] * scale. */
int bulletou_cuda_cpp_scale_axis_rows_f32_device(BulletOuCudaCppContext* ctx,
    BulletOuCudaCppF32Buffer* values, size_t value_len, const BulletOuCudaCppF32Buffer* row_scales,
    size_t row_count, size_t row_len);  /* cu:10245 */
int bulletou_cuda_cpp_sfnn_add_residual_count_decay_gradients_device(BulletOuCudaCppContext* ctx,
    BulletOuCudaCppF32Buffer* weights, BulletOuCudaCppF32Buffer* gradients,
    BulletOuCudaCppF32Buffer* decay_by_stack, BulletOuCudaCppI32Buffer* dirty_buckets, size_t dirty_count,
    size_t stride, size_t num_stacks);  /* cu:13411 */
int bulletou_cuda_cpp_sfnn_apply_residual_count_gates_to_gradients_device(BulletOuCudaCppContext* ctx,
    BulletOuCudaCppF32Buffer* gradients, const BulletOuCudaCppF32Buffer* gates,
    const BulletOuCudaCppI32Buffer* dirty_buckets, size_t dirty_count, size_t stride, size_t num_stacks);  /* cu:13451 */
int bulletou_center_scale(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* src,
    BulletOuCudaCppF32Buffer* dst, size_t n, float scale);  /* cu:13993 */

/* ---- research features outside this backend's scope ----
 * Exported so that a Rust build of crates/cuda_cpp links against this
 * library unchanged; each returns -1 with "unsupported on this backend: <name>"
 * after checking nothing else.  BatchNorm (batch_norm.cuh, bn_qat.cuh),
 * FT / L1 centering and its experiments, the FT saturation guard, effective
 * L1 clipping, bucket-axis factorizer updates, the shared-factor rebase and
 * the saturation penalty.  bulletou_bn_reference_mode (void) ignores its
 * argument: there is no BatchNorm to switch. */
int bulletou_bn_bind(BulletOuCudaCppContext* ctx, int layer, BulletOuCudaCppF32Buffer* params,
    BulletOuCudaCppF32Buffer* running, BulletOuCudaCppF32Buffer* stats, BulletOuCudaCppF32Buffer* grads,
    BulletOuCudaCppF32Buffer* xa, BulletOuCudaCppF32Buffer* xb, size_t rows, size_t stride, size_t width,
    size_t groups, float epsilon, float momentum, int training);  /* batch_norm.cuh:365 */
int bulletou_bn_forward(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* a,
    BulletOuCudaCppF32Buffer* b, BulletOuCudaCppF32Buffer* xa, BulletOuCudaCppF32Buffer* xb,
    BulletOuCudaCppI32Buffer* ids, BulletOuCudaCppF32Buffer* params, BulletOuCudaCppF32Buffer* running,
    BulletOuCudaCppF32Buffer* stats, size_t rows, size_t stride, size_t width, size_t groups, float epsilon,
    float momentum, int training);  /* batch_norm.cuh:294 */
int bulletou_bn_backward(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* da,
    BulletOuCudaCppF32Buffer* db, BulletOuCudaCppF32Buffer* xa, BulletOuCudaCppF32Buffer* xb,
    BulletOuCudaCppI32Buffer* ids, BulletOuCudaCppF32Buffer* params, BulletOuCudaCppF32Buffer* stats,
    BulletOuCudaCppF32Buffer* grads, size_t rows, size_t stride, size_t width, size_t groups);  /* batch_norm.cuh:316 */
int bulletou_bn_qat_project_l2(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* w,
    BulletOuCudaCppF32Buffer* slow, size_t input, size_t channels);  /* bn_qat.cuh:20 */
int bulletou_bn_qat_unfold_training(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* w,
    BulletOuCudaCppF32Buffer* b, BulletOuCudaCppF32Buffer* sw, BulletOuCudaCppF32Buffer* sb,
    BulletOuCudaCppF32Buffer* qw, BulletOuCudaCppF32Buffer* qb, size_t input, size_t output, size_t groups,
    int layer, size_t vr, float alpha);  /* bn_qat.cuh:78 */
int bulletou_bn_qat_ft(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* src,
    BulletOuCudaCppF32Buffer* dst, size_t base, size_t vr, size_t width, float alpha);  /* bn_qat.cuh:162 */
int bulletou_bn_qat_ft_training(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* src,
    BulletOuCudaCppF32Buffer* dst, BulletOuCudaCppF32Buffer* bias, BulletOuCudaCppF32Buffer* out_bias,
    size_t base, size_t vr, size_t width, float alpha);  /* bn_qat.cuh:169 */
int bulletou_bn_qat_pullback(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* w,
    BulletOuCudaCppF32Buffer* b, BulletOuCudaCppF32Buffer* sw, BulletOuCudaCppF32Buffer* sb,
    BulletOuCudaCppF32Buffer* gw, BulletOuCudaCppF32Buffer* gb, BulletOuCudaCppF32Buffer* gs,
    BulletOuCudaCppF32Buffer* gsb, size_t input, size_t output, size_t groups, int layer, size_t vr,
    float alpha);  /* bn_qat.cuh:178 */
void bulletou_bn_reference_mode(int enabled);  /* batch_norm.cuh:229 */
int bulletou_center_l1_groups(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* w,
    BulletOuCudaCppF32Buffer* b, BulletOuCudaCppF32Buffer* sw, BulletOuCudaCppF32Buffer* sb,
    BulletOuCudaCppF32Buffer* gw, BulletOuCudaCppF32Buffer* gb, BulletOuCudaCppF32Buffer* fw,
    BulletOuCudaCppF32Buffer* fb, BulletOuCudaCppF32Buffer* fsw, BulletOuCudaCppF32Buffer* fsb,
    BulletOuCudaCppF32Buffer* fgw, BulletOuCudaCppF32Buffer* fgb, BulletOuCudaCppF32Buffer* c, size_t cols,
    int before);  /* cu:13936 */
int bulletou_center_affine_layout(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* w,
    BulletOuCudaCppF32Buffer* b, BulletOuCudaCppF32Buffer* sw, BulletOuCudaCppF32Buffer* sb,
    BulletOuCudaCppF32Buffer* gw, BulletOuCudaCppF32Buffer* gb, BulletOuCudaCppF32Buffer* c, size_t rows,
    size_t cols, int before, int column_major);  /* cu:13974 */
int bulletou_center_mean_reference(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* input,
    BulletOuCudaCppF32Buffer* scratch, size_t rows, size_t cols);  /* cu:14013 */
int bulletou_experiment_center_affine(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* w,
    BulletOuCudaCppF32Buffer* b, BulletOuCudaCppF32Buffer* sw, BulletOuCudaCppF32Buffer* sb,
    BulletOuCudaCppF32Buffer* gw, BulletOuCudaCppF32Buffer* gb, BulletOuCudaCppF32Buffer* c, size_t rows,
    size_t cols, int before);  /* cu:13959 */
int bulletou_experiment_column_mean(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* input,
    BulletOuCudaCppF32Buffer* scratch, size_t rows, size_t cols);  /* cu:14001 */
int bulletou_experiment_bucket_mean(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* input,
    BulletOuCudaCppI32Buffer* buckets, BulletOuCudaCppF32Buffer* scratch, size_t n, size_t d, size_t stacks);  /* cu:14043 */
int bulletou_experiment_bucket_centers(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* sums,
    BulletOuCudaCppF32Buffer* centers, size_t d, size_t stacks);  /* cu:14055 */
int bulletou_experiment_center_affine_bucket(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* w,
    BulletOuCudaCppF32Buffer* b, BulletOuCudaCppF32Buffer* sw, BulletOuCudaCppF32Buffer* sb,
    BulletOuCudaCppF32Buffer* gw, BulletOuCudaCppF32Buffer* gb, BulletOuCudaCppF32Buffer* c, size_t rows,
    size_t cols, size_t group_rows, int before);  /* cu:14062 */
int bulletou_experiment_mean_penalty_test(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* z,
    BulletOuCudaCppI32Buffer* buckets, BulletOuCudaCppF32Buffer* weights, BulletOuCudaCppF32Buffer* grad,
    size_t batch, size_t hidden, size_t stride, size_t stacks, float strength);  /* cu:14075 */
int bulletou_bind_ft_saturation_guard(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* weights,
    BulletOuCudaCppI32Buffer* counts, BulletOuCudaCppI32Buffer* streaks, size_t batch, size_t ft,
    float strength, float rate, int patience);  /* cu:13764 */
int bulletou_ft_saturation_guard(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* a,
    BulletOuCudaCppF32Buffer* b, BulletOuCudaCppF32Buffer* weights, BulletOuCudaCppI32Buffer* ai,
    BulletOuCudaCppI32Buffer* bi, BulletOuCudaCppI32Buffer* counts, BulletOuCudaCppI32Buffer* streaks,
    BulletOuCudaCppF32Buffer* gw, BulletOuCudaCppF32Buffer* gb, size_t batch, size_t ft, size_t active,
    size_t inputs, float ft_alpha, float strength, float rate, int patience);  /* cu:13780 */
int bulletou_clip_effective_l1(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* w,
    BulletOuCudaCppF32Buffer* slow, BulletOuCudaCppF32Buffer* shared, BulletOuCudaCppF32Buffer* shared_slow,
    BulletOuCudaCppF32Buffer* remainder, size_t cols, size_t outputs, float alpha);  /* cu:13831 */
int bulletou_clip_effective_l1_axis(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* w,
    BulletOuCudaCppF32Buffer* slow, BulletOuCudaCppF32Buffer* shared, BulletOuCudaCppF32Buffer* shared_slow,
    BulletOuCudaCppF32Buffer* axis, BulletOuCudaCppF32Buffer* axis_slow, BulletOuCudaCppF32Buffer* remainder,
    size_t cols, size_t outputs, size_t stacks, size_t king_dim, size_t hand_dim, int king, int hand,
    int progress, int kh, int kp, int hp, float shared_alpha, float king_alpha, float hand_alpha,
    float progress_alpha, float pair_alpha);  /* cu:13880 */
int bulletou_factor_axis_update_device(BulletOuCudaCppContext* ctx, size_t len, size_t stride,
    size_t king_end, size_t hand_end, size_t pair_end, float king_alpha, float hand_alpha, float pair_alpha,
    float progress_alpha, BulletOuCudaCppF32Buffer* confidence, float gradient_factor, float lr, float decay,
    float beta1, float beta2, float epsilon, float step_size, int use_denom, int sgd, float min_weight,
    float max_weight, float norm_rate, int norm_before, int do_lookahead, float lookahead_alpha,
    int clip_after, BulletOuCudaCppF32Buffer* gradients, BulletOuCudaCppF32Buffer* weights,
    BulletOuCudaCppF32Buffer* momentum, BulletOuCudaCppF32Buffer* velocity, BulletOuCudaCppF32Buffer* slow);  /* cu:10522 */
int bulletou_cuda_cpp_rebase_shared_device(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* base,
    BulletOuCudaCppF32Buffer* base_slow, BulletOuCudaCppF32Buffer* base_m, BulletOuCudaCppF32Buffer* base_v,
    BulletOuCudaCppF32Buffer* shared, BulletOuCudaCppF32Buffer* shared_slow,
    BulletOuCudaCppF32Buffer* shared_m, BulletOuCudaCppF32Buffer* shared_v, BulletOuCudaCppF32Buffer* gates,
    size_t base_count, size_t shared_count, size_t shared_offset, size_t input_dim, size_t output_dim,
    float old_alpha, float new_alpha);  /* cu:13609 */
int bulletou_cuda_cpp_sfnn_add_saturation_penalty_gradients_device(BulletOuCudaCppContext* ctx,
    BulletOuCudaCppF32Buffer* weights, BulletOuCudaCppF32Buffer* shared_weights, int has_shared,
    BulletOuCudaCppF32Buffer* axis_weights, int has_axis, BulletOuCudaCppF32Buffer* gradients,
    BulletOuCudaCppF32Buffer* shared_gradients, BulletOuCudaCppF32Buffer* axis_gradients,
    BulletOuCudaCppI32Buffer* dirty_buckets, size_t dirty_count, size_t input_dim, size_t output_dim,
    size_t num_stacks, size_t factorizer_king_axis_dim, size_t factorizer_hand_axis_dim, int use_king_axis,
    int use_hand_axis, int use_progress_axis, int use_king_hand_pair, int use_king_progress_pair,
    int use_hand_progress_pair, float ft_factorizer_alpha, float factorizer_shared_alpha,
    float factorizer_king_axis_alpha, float factorizer_hand_axis_alpha, float factorizer_progress_axis_alpha,
    float factorizer_pair_alpha, const BulletOuCudaCppF32Buffer* residual_count_gates,
    const BulletOuCudaCppF32Buffer* factorizer_axis_confidences, int shared_weight_input_major,
    float weight_scale, float threshold, float penalty);  /* cu:13277 */

/* ---- the reference's kernel test hooks (crates/cuda_cpp/src tests) ----
 * Entry points that exist so the reference's own tests can drive single
 * internal kernels of its implementation (its FP16 gather variants, packed
 * L1, sort kernels, the dense-QAT integer references).  They have no
 * counterpart among this backend's kernels: each returns -1 with
 * "unsupported on this backend: <name>".  bulletou_test_stream_delay returns 0
 * (it only delays the stream in the reference). */
int bulletou_test_dense_l1_16(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* input,
    BulletOuCudaCppF32Buffer* weights, BulletOuCudaCppF32Buffer* bias, BulletOuCudaCppI32Buffer* buckets,
    BulletOuCudaCppF32Buffer* output, size_t batch, size_t input_dim, size_t stacks, int optimized);  /* cu:4595 */
int bulletou_test_factorized_ft_half_fold(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* weights,
    BulletOuCudaCppF32Buffer* output, size_t base, size_t ft, float alpha, int fused);  /* cu:4620 */
int bulletou_test_sfnn_ft_sort(BulletOuCudaCppContext* ctx, BulletOuCudaCppI32Buffer* stm,
    BulletOuCudaCppI32Buffer* nstm, BulletOuCudaCppF32Buffer* weights, BulletOuCudaCppF32Buffer* bias,
    BulletOuCudaCppF32Buffer* a, BulletOuCudaCppF32Buffer* b, BulletOuCudaCppF32Buffer* combined,
    BulletOuCudaCppI32Buffer* counts, BulletOuCudaCppI32Buffer* order, size_t batch, size_t active,
    size_t input, size_t ft, int sorted);  /* cu:4647 */
int bulletou_test_sfnn_ft_gather(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* pre,
    BulletOuCudaCppI32Buffer* positions, BulletOuCudaCppI32Buffer* offsets,
    BulletOuCudaCppF32Buffer* gradients, size_t features, size_t ft, int tiled, int add);  /* cu:4762 */
int bulletou_test_sfnn_half_grad_gather(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* pre,
    BulletOuCudaCppI32Buffer* positions, BulletOuCudaCppI32Buffer* offsets, BulletOuCudaCppF32Buffer* out,
    size_t batch, size_t features, size_t ft, size_t occurrences, int vector_width);  /* cu:4838 */
int bulletou_test_sfnn_half_grad(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* stm,
    BulletOuCudaCppF32Buffer* nstm, BulletOuCudaCppF32Buffer* combined, BulletOuCudaCppF32Buffer* out_stm,
    BulletOuCudaCppF32Buffer* out_nstm, BulletOuCudaCppF32Buffer* bias_grad, size_t batch, size_t ft,
    int fused);  /* cu:4866 */
int bulletou_test_stream_delay(BulletOuCudaCppContext* ctx);  /* cu:5639 */
int bulletou_test_l1_bucket_fold(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* w,
    BulletOuCudaCppF32Buffer* shared, BulletOuCudaCppF32Buffer* axis, BulletOuCudaCppF32Buffer* gates,
    BulletOuCudaCppF32Buffer* confidence, BulletOuCudaCppF32Buffer* out, BulletOuCudaCppI32Buffer* packed,
    int fast);  /* cu:5646 */
int bulletou_test_qat_ft_lattice(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* values, size_t n,
    int fast);  /* cu:6013 */
int bulletou_test_qat_packed_l1(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* input,
    BulletOuCudaCppF32Buffer* weights, BulletOuCudaCppI32Buffer* bias, BulletOuCudaCppI32Buffer* buckets,
    BulletOuCudaCppF32Buffer* output, BulletOuCudaCppI32Buffer* raw, size_t batch, size_t inputs,
    size_t outputs, size_t stacks, int packed);  /* cu:6247 */
int bulletou_test_dense_qat_exact_ft(BulletOuCudaCppContext* ctx, BulletOuCudaCppI32Buffer* stm,
    BulletOuCudaCppI32Buffer* nstm, BulletOuCudaCppF32Buffer* w, BulletOuCudaCppF32Buffer* bias,
    BulletOuCudaCppF32Buffer* output, BulletOuCudaCppI32Buffer* packed, size_t batch, size_t active,
    size_t inputs, size_t width);  /* cu:6384 */
int bulletou_test_l1_to_ft_f32_gradient(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* dy,
    BulletOuCudaCppF32Buffer* weights, BulletOuCudaCppI32Buffer* buckets,
    BulletOuCudaCppF32Buffer* activations, BulletOuCudaCppF32Buffer* result, BulletOuCudaCppF32Buffer* bias,
    size_t batch, size_t width, size_t stacks, int fused);  /* cu:7123 */
int bulletou_test_l1_to_ft_half_gradient(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* dy,
    BulletOuCudaCppF32Buffer* weights, BulletOuCudaCppI32Buffer* buckets,
    BulletOuCudaCppF32Buffer* activations, BulletOuCudaCppF32Buffer* result, BulletOuCudaCppF32Buffer* bias,
    size_t batch, size_t width, size_t stacks, int fused);  /* cu:7152 */
int bulletou_test_l1_gather2(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* inputs,
    BulletOuCudaCppF32Buffer* dy, BulletOuCudaCppI32Buffer* offsets, BulletOuCudaCppI32Buffer* positions,
    BulletOuCudaCppF32Buffer* dw, BulletOuCudaCppF32Buffer* db, BulletOuCudaCppF32Buffer* dfw,
    BulletOuCudaCppF32Buffer* dfb, size_t batch, size_t width, size_t outputs, size_t stacks, float alpha);  /* cu:7314 */
int bulletou_test_l1_gather2_king_progress(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* inputs,
    BulletOuCudaCppF32Buffer* dy, BulletOuCudaCppI32Buffer* offsets, BulletOuCudaCppI32Buffer* positions,
    BulletOuCudaCppF32Buffer* dw, BulletOuCudaCppF32Buffer* db, BulletOuCudaCppF32Buffer* dfw,
    BulletOuCudaCppF32Buffer* dfb, BulletOuCudaCppF32Buffer* daw, BulletOuCudaCppF32Buffer* dab,
    BulletOuCudaCppF32Buffer* confidence, size_t batch, size_t width, size_t outputs, size_t stacks,
    size_t king_dim, float shared_alpha, float king_alpha, float progress_alpha, float pair_alpha);  /* cu:7338 */
int bulletou_dense_qat_integer_reference(BulletOuCudaCppContext* ctx, BulletOuCudaCppI32Buffer* input,
    BulletOuCudaCppF32Buffer* weights, BulletOuCudaCppF32Buffer* bias, BulletOuCudaCppI32Buffer* buckets,
    BulletOuCudaCppI32Buffer* output, size_t batch, size_t inputs, size_t outputs, size_t stacks);  /* cu:9336 */
int bulletou_dense_qat_activation_reference(BulletOuCudaCppContext* ctx, BulletOuCudaCppI32Buffer* raw,
    BulletOuCudaCppF32Buffer* square_gradient, BulletOuCudaCppF32Buffer* linear_gradient,
    BulletOuCudaCppI32Buffer* square_output, BulletOuCudaCppI32Buffer* linear_output,
    BulletOuCudaCppF32Buffer* gradient, size_t n);  /* cu:9403 */
int bulletou_dense_qat_l1_backward_reference(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* l1,
    BulletOuCudaCppF32Buffer* l2_input, BulletOuCudaCppF32Buffer* l2_input_gradients,
    BulletOuCudaCppF32Buffer* l1_gradients, size_t batch, size_t hidden, int skip);  /* cu:9422 */

#ifdef __cplusplus
}
#endif

#endif /* BULLETOU_CUDA_CPP_H */
