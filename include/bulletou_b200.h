/*
 * bulletou_b200.h — additive C ABI of libbulletou_b200.so.
 *
 * These entries have no one-to-one counterpart in the reference backend; they
 * are what a train-step runner calls instead of the reference's sequence of
 * forward / loss / backward / per-group optimizer calls.  Each one names the
 * reference sequence it replaces.  Existing bulletou_cuda_cpp_* signatures are
 * unchanged (see bulletou_cuda_cpp.h); handles and error convention are shared.
 */
#ifndef BULLETOU_B200_H
#define BULLETOU_B200_H

#include <stddef.h>

#include "bulletou_cuda_cpp.h"

#ifdef __cplusplus
extern "C" {
#endif

/* One Ranger (RAdam + Lookahead) step, exactly the scalars that
 * crates/cuda_cpp/src/lib.rs:9518-9544 passes to
 * bulletou_cuda_cpp_ranger_update_device for every parameter group. */
typedef struct BulletOuB200RangerStep {
    float norm_loss_rate;
    int norm_loss_before;
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
    int clip_after_lookahead;
} BulletOuB200RangerStep;

/* Scalar loss selection, as bulletou_cuda_cpp_scalar_loss_device_with_finalize
 * (cu:11809).  `normalizer` replaces the batch size as the divisor of the
 * output gradient (0 = batch); a data-parallel rank passes the global batch so
 * that summing rank gradients gives the global-batch mean gradient. */
typedef struct BulletOuB200LossSpec {
    int kind;
    float output_inv_scale;
    float loss_pow_exp;
    float loss_param;
    int finalize_loss;
    size_t normalizer;
} BulletOuB200LossSpec;

/* HalfKP parameter groups, in the update order of NnueTrainStepRunner
 * (lib.rs:5964-6024): l0w, l0b, l1w, l1b, l2w, l2b, outw, outb. */
#define BULLETOU_B200_NNUE_GROUPS 8

/* Library / device queries. */
int bulletou_b200_version(char* out, size_t out_len);
/* Creates a context that enqueues on an existing CUDA stream (not owned), so
 * the library's work orders with a host framework's stream (e.g. the stream a
 * collective library uses). */
int bulletou_b200_context_create_on_stream(int device, void* stream, BulletOuCudaCppContext** out);
int bulletou_b200_context_stream(const BulletOuCudaCppContext* ctx, void** out);
/* Raw device pointer of a buffer (for zero-copy interop with collectives). */
int bulletou_b200_f32_buffer_ptr(const BulletOuCudaCppF32Buffer* buffer, void** out);
int bulletou_b200_i32_buffer_ptr(const BulletOuCudaCppI32Buffer* buffer, void** out);
/* Asynchronous H2D copy straight from a pinned buffer (no staging memcpy),
 * and D2H into one; enqueued on the context stream, non-blocking. */
int bulletou_b200_i32_upload_pinned(BulletOuCudaCppContext* ctx, BulletOuCudaCppI32Buffer* dst,
    const BulletOuCudaCppPinnedI32Buffer* src, size_t len);
int bulletou_b200_f32_upload_pinned(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* dst,
    const BulletOuCudaCppPinnedF32Buffer* src, size_t len);
int bulletou_b200_f32_download_pinned(BulletOuCudaCppContext* ctx, BulletOuCudaCppPinnedF32Buffer* dst,
    const BulletOuCudaCppF32Buffer* src, size_t len);
/* Host pointer of a pinned buffer. */
int bulletou_b200_pinned_f32_ptr(const BulletOuCudaCppPinnedF32Buffer* buffer, void** out);
int bulletou_b200_pinned_i32_ptr(const BulletOuCudaCppPinnedI32Buffer* buffer, void** out);
/* Non-owning view [offset, offset+len) of a buffer; destroy with
 * bulletou_cuda_cpp_f32_buffer_destroy (frees only the handle). */
int bulletou_b200_f32_buffer_view(const BulletOuCudaCppF32Buffer* buffer, size_t offset, size_t len,
    BulletOuCudaCppF32Buffer** out);

/* Stage profiler (the counterpart of the reference's profiled steps,
 * lib.rs:5858-5928): while enabled, the fused train steps record a CUDA event
 * on the context stream at each phase boundary (no host synchronization).
 * profile_begin reserves room for `max_marks` events; profile_end waits for
 * the stream and returns in ms_out[i] the summed time between consecutive
 * marks i and i+1 of every step (phase i), in *steps_out the steps recorded
 * and in *phases_out the phases per step.  HalfKP step phases: inverse index,
 * king sort, FT gather, dense forward/loss/backward, batch reduce,
 * small-group Ranger + loss, FT rows.  SFNN step phases: sorts + tiles,
 * inverse index, fold + L1 weights, FT forward, L1 forward + head, L1
 * backward, small-group Ranger + loss, FT rows. */
int bulletou_b200_profile_begin(BulletOuCudaCppContext* ctx, size_t max_marks);
int bulletou_b200_profile_end(BulletOuCudaCppContext* ctx, float* ms_out, size_t ms_len, size_t* steps_out,
    size_t* phases_out);

/* Device bytes the context currently holds in its grow-only scratch slots
 * (no counterpart in the reference; diagnostics).  The slots are allocated on
 * first use by the entries that need scratch and freed at context destroy. */
int bulletou_b200_context_scratch_bytes(const BulletOuCudaCppContext* ctx, size_t* out);

/* Data-parallel overlap (no counterpart in the reference): the next SFNN
 * fused step on this context (bulletou_b200_sfnn_local_gradients_device or
 * bulletou_b200_sfnn_train_step_device) runs its batch-only work (king and
 * bucket sorts, rank tiles, inverse index) at once and makes the context
 * stream wait for `event` before its first read of a weight (the fold).  A
 * caller whose weight update runs on another stream records `event` after
 * it, so the next step's batch work overlaps the update's tail.  Consumed by
 * that step; null clears it.  The event must stay alive until the step has
 * been enqueued. */
int bulletou_b200_context_wait_before_weights(BulletOuCudaCppContext* ctx, const BulletOuCudaCppEvent* event);

/* L2 read-bandwidth probe (no counterpart in the reference; measurement
 * only): `passes` reads of buffer[0, len) with 16-byte loads cached in L2
 * only, by 4 * SMs CTAs of 512 threads; sink receives one float per thread
 * (len of sink >= 2048 * SMs).  With a buffer well inside L2 (126 MB on B200)
 * every pass after the first is served by L2; time it with events on the
 * context stream to get the L2 peak the row-gather kernels are judged by. */
int bulletou_b200_l2_read_probe(BulletOuCudaCppContext* ctx, const BulletOuCudaCppF32Buffer* buffer, size_t len,
    int passes, BulletOuCudaCppF32Buffer* sink);

/* One complete HalfKP train step on device-resident batch buffers.
 *
 * Replaces NnueTrainStepRunner::step_no_readback_with_loss_finalize
 * (lib.rs:5748-5799): nnue_forward_device (cu:10864) ->
 * scalar_loss_device_with_finalize (cu:11809) ->
 * nnue_backward_device(zero_l0_gradients = 0) (cu:12069) -> 8 x
 * ranger_update_device (cu:10576).  The feature-transformer gradient is never
 * materialised: a per-row inverse index of the batch feeds a row kernel that
 * sums the rows' gradients and applies Ranger in the same pass.
 *
 * params/momentum/velocity/slow_params: 8 handles each (group order above).
 * output [batch] receives the network output; per_sample, mean_output_gradients
 * [batch], weighted_sum and mean [1] follow the scalar-loss contract. */
int bulletou_b200_nnue_train_step_device(
    BulletOuCudaCppContext* ctx, size_t input_size, size_t l1, size_t l2, size_t l3,
    size_t batch, size_t max_active,
    const BulletOuCudaCppI32Buffer* stm_indices, const BulletOuCudaCppI32Buffer* nstm_indices,
    const BulletOuCudaCppF32Buffer* targets, const BulletOuCudaCppF32Buffer* entry_weights,
    const BulletOuB200LossSpec* loss, const BulletOuB200RangerStep* ranger,
    BulletOuCudaCppF32Buffer* const* params, BulletOuCudaCppF32Buffer* const* momentum,
    BulletOuCudaCppF32Buffer* const* velocity, BulletOuCudaCppF32Buffer* const* slow_params,
    BulletOuCudaCppF32Buffer* output, BulletOuCudaCppF32Buffer* per_sample,
    BulletOuCudaCppF32Buffer* mean_output_gradients, BulletOuCudaCppF32Buffer* weighted_sum,
    BulletOuCudaCppF32Buffer* mean);

/* HalfKP forward that allocates no device memory.  No counterpart in the
 * reference backend.  It is for callers that must not call cudaMalloc while
 * they run -- an engine or server that evaluates positions inside its own
 * fixed memory budget, or code running where allocation is forbidden or
 * would stall other work -- and who still want the production-shape kernels.
 * Same arguments and outputs as bulletou_cuda_cpp_nnue_forward_device; only
 * l1 in {256, 512}, l2 = l3 = 32, max_active <= 4096 and batch <= 65536
 * positions are accepted (anything larger is rejected with an error).  Its
 * scratch is one static device array of 1.2 MB that every GPU loading the
 * library holds until exit; the first call on a device looks up that array's
 * device address (make that first call before any stream capture); the
 * address is kept for the life of the process, so it is stale once the
 * device's primary context is destroyed (cudaDeviceReset): do not call this
 * entry after a device reset in the same process.  Nothing in the array needs
 * clearing between calls, but all calls on a device share it: calls whose work
 * overlaps on the GPU (other streams, other threads) race and must be
 * serialized by the caller. */
int bulletou_b200_nnue_forward_device_noalloc(
    BulletOuCudaCppContext* ctx, size_t input_size, size_t l1, size_t l2, size_t l3,
    size_t batch, size_t max_active,
    const BulletOuCudaCppI32Buffer* stm_indices, const BulletOuCudaCppI32Buffer* nstm_indices,
    const BulletOuCudaCppF32Buffer* l0w, const BulletOuCudaCppF32Buffer* l0b,
    const BulletOuCudaCppF32Buffer* l1w, const BulletOuCudaCppF32Buffer* l1b,
    const BulletOuCudaCppF32Buffer* l2w, const BulletOuCudaCppF32Buffer* l2b,
    const BulletOuCudaCppF32Buffer* outw, const BulletOuCudaCppF32Buffer* outb,
    BulletOuCudaCppF32Buffer* stm_l0, BulletOuCudaCppF32Buffer* nstm_l0,
    BulletOuCudaCppF32Buffer* combined, BulletOuCudaCppF32Buffer* hidden1,
    BulletOuCudaCppF32Buffer* hidden2, BulletOuCudaCppF32Buffer* output);

/* Length of the packed small-parameter gradient used by the data-parallel
 * phases: l0b | l1w | l1b | l2w | l2b | outw | outb. */
int bulletou_b200_nnue_dense_gradient_len(size_t l1, size_t l2, size_t l3, size_t* out);

/* Data-parallel phase 1: forward + loss + backward of a rank's local batch.
 * Overwrites ft_gradients [input_size*l1] with this batch's feature-transformer
 * gradient and dense_gradients [dense_gradient_len] with the packed
 * small-parameter gradient.  Between this and the optimizer the caller
 * reduce-scatters ft_gradients by row shard and all-reduces dense_gradients;
 * the update itself is bulletou_cuda_cpp_ranger_update_device on views. */
int bulletou_b200_nnue_local_gradients_device(
    BulletOuCudaCppContext* ctx, size_t input_size, size_t l1, size_t l2, size_t l3,
    size_t batch, size_t max_active,
    const BulletOuCudaCppI32Buffer* stm_indices, const BulletOuCudaCppI32Buffer* nstm_indices,
    const BulletOuCudaCppF32Buffer* targets, const BulletOuCudaCppF32Buffer* entry_weights,
    const BulletOuB200LossSpec* loss, BulletOuCudaCppF32Buffer* const* params,
    BulletOuCudaCppF32Buffer* ft_gradients, BulletOuCudaCppF32Buffer* dense_gradients,
    BulletOuCudaCppF32Buffer* output, BulletOuCudaCppF32Buffer* per_sample,
    BulletOuCudaCppF32Buffer* mean_output_gradients, BulletOuCudaCppF32Buffer* weighted_sum,
    BulletOuCudaCppF32Buffer* mean);

/* One complete KPPT scalar-table train step (one component table).
 * Replaces KpptTableTrainStepRunner::step_no_readback_with_loss_finalize
 * (lib.rs:4962-5036): kppt_forward_device (cu:11887) -> scalar loss ->
 * kppt_backward_device (cu:11934) -> ranger_update_device over table_w,
 * table_b, outw, outb (lib.rs:5037-5066).  The table gradient lives in a
 * context-owned table that is only ever zero between steps: the fused
 * forward/loss kernel scatters into it and the table's Ranger pass resets it
 * in the same sweep, so the reference's whole-table zero fill disappears.
 * params/momentum/velocity/slow_params: 4 handles each
 * (table_w [input_size], table_b [1], outw [2], outb [1]). */
int bulletou_b200_kppt_train_step_device(
    BulletOuCudaCppContext* ctx, size_t input_size, size_t batch, size_t max_active,
    const BulletOuCudaCppI32Buffer* stm_indices, const BulletOuCudaCppI32Buffer* nstm_indices,
    const BulletOuCudaCppF32Buffer* targets, const BulletOuCudaCppF32Buffer* entry_weights,
    const BulletOuB200LossSpec* loss, const BulletOuB200RangerStep* ranger,
    BulletOuCudaCppF32Buffer* const* params, BulletOuCudaCppF32Buffer* const* momentum,
    BulletOuCudaCppF32Buffer* const* velocity, BulletOuCudaCppF32Buffer* const* slow_params,
    BulletOuCudaCppF32Buffer* output, BulletOuCudaCppF32Buffer* per_sample,
    BulletOuCudaCppF32Buffer* mean_output_gradients, BulletOuCudaCppF32Buffer* weighted_sum,
    BulletOuCudaCppF32Buffer* mean);


/* SFNN shape of the fused step (the reference's SfnnForwardShape,
 * lib.rs:928-970, dense L1 only) plus the factorizer coefficients
 * (SfnnFactorizerAlpha::ft / ::shared, lib.rs:1280-1312). */
typedef struct BulletOuB200SfnnShape {
    size_t input_size;  /* 73305 / 131949, or + 1629 with the FT factorizer */
    size_t ft_size;
    size_t l1_hidden;
    int l1_skip;
    size_t l2_size;
    size_t num_stacks;
    float ft_factorizer_alpha;
    float factorizer_shared_alpha;
} BulletOuB200SfnnShape;

/* Quantisation-aware training switches of the SFNN runner
 * (SfnnLayerLrMultipliers::qat_l1 / qat_ft / qat_l2 / qat_l3, lib.rs:6332-6336):
 *   l1  L1 weights folded with the shared factor then fake-quantised to i8 at
 *       64, bias to i32 at 127*64; backward input gradients use them
 *       (cu:11514-11590; the runner's prepare_l1_qat, lib.rs:6525-6550);
 *   ft  FT rows folded with their virtual row then fake-quantised to i16 at
 *       127, FT bias too (layer_qat.rs:832-880);
 *   l2, l3  L2 / L3 weights fake-quantised at 64, biases at 127*64; no L2/L3
 *       shared factors allowed (layer_qat.rs:937-943).
 * l1 && l2 && l3 selects the dense integer QAT (layer_qat.rs:977-991;
 * cu:6654-6712, 6322, 3709-3770): FT output floored to the 1/127 lattice, or
 * the engine's integer FT when ft is set; integer L1 / L2 / L3 with the master
 * L2 / L3 biases rounded to 127*64; continuous activation STEs.  Gradients
 * reach the f32 masters through an identity STE. */
typedef struct BulletOuB200SfnnQat {
    int l1;
    int ft;
    int l2;
    int l3;
} BulletOuB200SfnnQat;

/* One complete SFNN train step.  Replaces
 * SfnnTrainStepRunner::step_no_readback_with_loss_finalize (lib.rs:7448-7533)
 * with default layer multipliers: sfnn_forward_device (cu:11329) -> scalar
 * loss -> sfnn_backward_train_device (cu:12882) -> Ranger on every group
 * (update_weights_with_lr_multipliers_and_dirty_buckets, lib.rs:8425-8730).
 * params / momentum / velocity / slow_params: 14 handles each in the order
 * l0w l0b l1w l1b l1fw l1fb l2w l2b l2fw l2fb l3w l3b l3fw l3fb; the shared
 * factor handles (l1fw/l1fb, l2fw/l2fb, l3fw/l3fb) are null when that factor
 * is absent.  The FT gradient is never materialised: each FT row (and each
 * virtual factor row) is updated by the pass that sums its gradient.
 * ranger->norm_loss_rate must be 0 (with default multipliers the SFNN runner
 * applies no norm loss, lib.rs:6416-6420).  qat: the QAT switches, or null
 * for none. */
int bulletou_b200_sfnn_train_step_device(
    BulletOuCudaCppContext* ctx, const BulletOuB200SfnnShape* shape, size_t batch, size_t max_active,
    const BulletOuCudaCppI32Buffer* stm_indices, const BulletOuCudaCppI32Buffer* nstm_indices,
    const BulletOuCudaCppI32Buffer* buckets, const BulletOuCudaCppF32Buffer* targets,
    const BulletOuCudaCppF32Buffer* entry_weights, const BulletOuB200LossSpec* loss,
    const BulletOuB200RangerStep* ranger, BulletOuCudaCppF32Buffer* const* params,
    BulletOuCudaCppF32Buffer* const* momentum, BulletOuCudaCppF32Buffer* const* velocity,
    BulletOuCudaCppF32Buffer* const* slow_params, BulletOuCudaCppF32Buffer* output,
    BulletOuCudaCppF32Buffer* per_sample, BulletOuCudaCppF32Buffer* mean_output_gradients,
    BulletOuCudaCppF32Buffer* weighted_sum, BulletOuCudaCppF32Buffer* mean, const BulletOuB200SfnnQat* qat);

/* Length of the packed SFNN small-parameter gradient (groups l0b l1w l1b
 * [l1fw l1fb] l2w l2b [l2fw l2fb] l3w l3b [l3fw l3fb], absent shared factors
 * omitted) used by the data-parallel phases. */
int bulletou_b200_sfnn_dense_gradient_len(const BulletOuB200SfnnShape* shape, int has_l1f, int has_l2f, int has_l3f,
    size_t* out);

/* SFNN data-parallel phase 1: forward + loss + backward of a rank's local
 * batch (the loss normalizer in `loss` is the global batch).  Overwrites
 * ft_gradients [input_size*ft_size, virtual factor rows included] with the
 * batch's FT gradient and dense_gradients [sfnn_dense_gradient_len] with the
 * packed small-parameter gradient; params and qat as in
 * sfnn_train_step_device.  The exchange (reduce-scatter / all-reduce) and the
 * update (ranger_update_device on views) are the caller's.
 * The FT gradient rows are written by n_row_launches kernel launches, launch j
 * completing rows [row_end[j-1], row_end[j]) (bulletou_b200_sfnn_row_launches).
 * Optional row_shift[j]: launch j writes its rows row_shift[j] rows further
 * into ft_gradients (so each range can start a padded chunk); optional
 * row_events[j] is recorded on the context stream after launch j, so a
 * collective on another stream can start on that range while later launches
 * run.  Both null: rows at their own index, no events. */
int bulletou_b200_sfnn_local_gradients_device(
    BulletOuCudaCppContext* ctx, const BulletOuB200SfnnShape* shape, size_t batch, size_t max_active,
    const BulletOuCudaCppI32Buffer* stm_indices, const BulletOuCudaCppI32Buffer* nstm_indices,
    const BulletOuCudaCppI32Buffer* buckets, const BulletOuCudaCppF32Buffer* targets,
    const BulletOuCudaCppF32Buffer* entry_weights, const BulletOuB200LossSpec* loss,
    BulletOuCudaCppF32Buffer* const* params, BulletOuCudaCppF32Buffer* ft_gradients,
    BulletOuCudaCppF32Buffer* dense_gradients, BulletOuCudaCppF32Buffer* output,
    BulletOuCudaCppF32Buffer* per_sample, BulletOuCudaCppF32Buffer* mean_output_gradients,
    BulletOuCudaCppF32Buffer* weighted_sum, BulletOuCudaCppF32Buffer* mean, const BulletOuB200SfnnQat* qat,
    const size_t* row_shift, BulletOuCudaCppEvent* const* row_events, size_t n_row_launches);

/* The FT row kernel's launches for a shape: *n_launches, and row_end[j] (up
 * to cap entries) = first row after launch j. */
int bulletou_b200_sfnn_row_launches(const BulletOuB200SfnnShape* shape, size_t* n_launches, size_t* row_end,
    size_t cap);

/* ---------------------------------------------------------------- peer-memory row exchange
 * Data-parallel SFNN without a reduce-scatter / all-gather library call: the
 * FT rows are sharded by chunks of row launches (chunk c = table rows
 * [start_c, start_c + length_c), padded to world * shard_rows_c rows; rank r
 * owns rows start_c + r * shard_rows_c ..., stored from row shard_off_c of
 * its compact shard).  Each rank holds a receive buffer of world slots of
 * slot_rows x width floats (slot s = rank s's gradient rows of the rows this
 * rank owns, at their compact index) and a flag array of 2 * chunks * world
 * ints, zeroed once: scatter flags [chunk][source rank], then ready flags
 * [chunk][owner rank].  Peers' buffers are opened from CUDA IPC handles; all
 * accesses are plain NVLink loads and stores.  `epoch` is the step number
 * (it only grows, so flags are never reset); every wait is bounded (about
 * 2 s), after which the error word holds 1 + the index of the flag waited
 * for and the rows are left unchanged. */
typedef struct BulletOuB200RowExchange {
    size_t world;                /* 1..8 */
    size_t rank;
    unsigned long long recv[8];  /* every rank's receive buffer (device addresses in this process) */
    unsigned long long table[8]; /* every rank's FT table (l0w) */
    unsigned long long flags[8]; /* every rank's flag array */
    size_t slot_rows;
    int epoch;
    /* the small groups' packed gradient (bulletou_b200_sfnn_dense_gradient_len
     * floats): every rank's receive buffer of world slots of small_len floats,
     * and the first of the world small flags in every flag array (0: the
     * small gradient is not exchanged by the local-gradients entry) */
    unsigned long long small_recv[8];
    size_t small_len;
    size_t small_flag_base;
} BulletOuB200RowExchange;

/* CUDA IPC handle (64 bytes) of a buffer's device memory, and its opening /
 * closing in another process (same node, peer GPUs). */
int bulletou_b200_f32_buffer_ipc_handle(const BulletOuCudaCppF32Buffer* buffer, void* handle_out);
int bulletou_b200_i32_buffer_ipc_handle(const BulletOuCudaCppI32Buffer* buffer, void* handle_out);
int bulletou_b200_ipc_open(BulletOuCudaCppContext* ctx, const void* handle, unsigned long long* device_address);
int bulletou_b200_ipc_close(BulletOuCudaCppContext* ctx, unsigned long long device_address);

/* Local gradients as bulletou_b200_sfnn_local_gradients_device, with the FT
 * gradient rows stored into their owners' receive slots instead of a local
 * table.  Per row launch j: the chunk it belongs to (launch_chunk_start,
 * launch_shard_rows, launch_shard_off) and launch_signal[j] = the chunk's
 * index when j is its last launch, else -1; after such a launch the scatter
 * flag [chunk][rank] of every rank is set to x->epoch.  With x->small_len > 0
 * the packed small-group gradient (dense_gradients) is also stored into slot
 * `rank` of every rank's small receive buffer before the row launches and
 * small flag [small_flag_base + rank] of every rank set.  row_events[j]
 * (optional) as in the plain entry. */
int bulletou_b200_sfnn_local_gradients_exchange_device(
    BulletOuCudaCppContext* ctx, const BulletOuB200SfnnShape* shape, size_t batch, size_t max_active,
    const BulletOuCudaCppI32Buffer* stm_indices, const BulletOuCudaCppI32Buffer* nstm_indices,
    const BulletOuCudaCppI32Buffer* buckets, const BulletOuCudaCppF32Buffer* targets,
    const BulletOuCudaCppF32Buffer* entry_weights, const BulletOuB200LossSpec* loss,
    BulletOuCudaCppF32Buffer* const* params, BulletOuCudaCppF32Buffer* dense_gradients,
    BulletOuCudaCppF32Buffer* output, BulletOuCudaCppF32Buffer* per_sample,
    BulletOuCudaCppF32Buffer* mean_output_gradients, BulletOuCudaCppF32Buffer* weighted_sum,
    BulletOuCudaCppF32Buffer* mean, const BulletOuB200SfnnQat* qat, const BulletOuB200RowExchange* x,
    const size_t* launch_chunk_start, const size_t* launch_shard_rows, const size_t* launch_shard_off,
    const long long* launch_signal, BulletOuCudaCppEvent* const* row_events, size_t n_row_launches);

/* The owner's part of chunk `c` (rows [chunk_start, chunk_start +
 * chunk_length), shard_rows / shard_off as above): waits for the chunk's
 * scatter flags [scatter_index, scatter_index + world) of its own flag array,
 * sums the world slots of its rows in rank order, runs Ranger (`step`) on its
 * compact shard state, stores the updated rows into every rank's table and
 * sets ready flag `ready_index` (= ready base + c * world + rank) of every
 * rank to x->epoch. */
int bulletou_b200_sfnn_shard_ranger_exchange_device(
    BulletOuCudaCppContext* ctx, const BulletOuB200RowExchange* x, size_t width, size_t chunk_start,
    size_t chunk_length, size_t shard_rows, size_t shard_off, const BulletOuB200RangerStep* step,
    BulletOuCudaCppF32Buffer* weights, BulletOuCudaCppF32Buffer* momentum, BulletOuCudaCppF32Buffer* velocity,
    BulletOuCudaCppF32Buffer* slow, const BulletOuCudaCppI32Buffer* flags, size_t scatter_index,
    size_t ready_index, BulletOuCudaCppI32Buffer* error);

/* The small groups' all-reduce over peer memory: waits (bounded) for the
 * world small flags of `flags` to reach x->epoch, then dst[i] = the sum over
 * ranks, in rank order, of slot r of this rank's small receive buffer. */
int bulletou_b200_exchange_reduce_small_device(BulletOuCudaCppContext* ctx, const BulletOuB200RowExchange* x,
    BulletOuCudaCppF32Buffer* dst, const BulletOuCudaCppI32Buffer* flags, BulletOuCudaCppI32Buffer* error);

/* Enqueues a bounded wait until flags[offset, offset + count) all reach
 * `epoch` (timeout: *error = 1 + the flag's index). */
int bulletou_b200_exchange_wait_device(BulletOuCudaCppContext* ctx, const BulletOuCudaCppI32Buffer* flags,
    size_t offset, size_t count, int epoch, BulletOuCudaCppI32Buffer* error);

/* As bulletou_b200_context_wait_before_weights, for flags: the next SFNN
 * fused step waits (bounded, as bulletou_b200_exchange_wait_device) until
 * flags[offset, offset + count) reach `epoch` before its first weight read;
 * flags null clears it. */
int bulletou_b200_context_wait_flags_before_weights(BulletOuCudaCppContext* ctx,
    const BulletOuCudaCppI32Buffer* flags, size_t offset, size_t count, int epoch,
    BulletOuCudaCppI32Buffer* error);

/* ---------------------------------------------------------------- quantised HalfKP
 * The reference exports a trained HalfKP 256x2-32-32 net to the engine's
 * nn.bin (write_cuda_cpp_nnue_nn_bin, examples/bulletou.rs:26303-26413); the
 * engine (YaneuraOu's halfkp_256x2-32-32 NNUE, outside the reference tree)
 * evaluates it in integers.  No counterpart in the reference's C ABI.
 * Quantised buffers (I32 handles holding packed narrow integers):
 *   0 l0w  i16 [rows][l1]   rows = 125388 when input_size = 125388 + 1548
 *                           (the 1548 leading virtual rows added to each base
 *                           row), else input_size
 *   1 l0b  i16 [l1]          2 l1w i8 [l2][pad32(2 l1)]   3 l1b i32 [l2]
 *   4 l2w  i8 [l3][pad32(l2)] 5 l2b i32 [l3]   6 outw i8 [pad32(l3)]   7 outb i32 [1]
 * Scales: FT 127, dense weights 64, biases 127 * 64; round half away from zero;
 * values outside their integer range saturate and are counted in errors[0]
 * (the reference's writer refuses them).  params: the 8 f32 handles
 * l0w l0b l1w l1b l2w l2b outw outb in the training layout (dense weights
 * input-major). */
int bulletou_b200_nnue_quantize_device(BulletOuCudaCppContext* ctx, size_t input_size, size_t l1, size_t l2,
    size_t l3, BulletOuCudaCppF32Buffer* const* params, BulletOuCudaCppI32Buffer* const* quantized,
    BulletOuCudaCppI32Buffer* errors);

/* Integer evaluation of a batch: per perspective (side to move first) an i16
 * accumulator (bias + rows, wrapping) clamped to [0, 127]; each affine layer
 * bias + sum u8 * i8 in i32 then clamp(x >> 6, 0, 127); raw_output = output
 * bias + sum; score_output (optional) = raw / fv_scale (toward zero).
 * Features below 0 are padding; features at or above rows are skipped and
 * counted in errors[0] (optional). */
int bulletou_b200_nnue_integer_forward_device(BulletOuCudaCppContext* ctx, size_t input_size, size_t l1, size_t l2,
    size_t l3, size_t batch, size_t max_active, const BulletOuCudaCppI32Buffer* stm_indices,
    const BulletOuCudaCppI32Buffer* nstm_indices, BulletOuCudaCppI32Buffer* const* quantized, int fv_scale,
    BulletOuCudaCppI32Buffer* raw_output, BulletOuCudaCppI32Buffer* score_output, BulletOuCudaCppI32Buffer* errors);

/* ---------------------------------------------------------------- quantised SFNN
 * The reference evaluates a trained SFNN through the engine's integer network
 * on the CPU (examples/bulletou.rs: export quantisation 10050-10300, integer
 * forward quantized_sfnn_forward_sample 8001-8163, final division 8045-8054).
 * These two entries run the same integer arithmetic on the device; they have
 * no counterpart in the reference's C ABI.
 *
 * Quantised buffers (I32 handles holding packed narrow integers, lengths in
 * 32-bit words rounded up), in this order:
 *   0 l0w  i16 [rows][ft_size]     rows = the factorizer base (73305 / 131949)
 *                                  when input_size carries the virtual rows,
 *                                  else input_size; virtual rows folded in
 *   1 l0b  i16 [ft_size]
 *   2 l1w  i8  [stacks][l1_out][pad32(ft_size)]   shared L1 factor folded in
 *   3 l1b  i32 [stacks][l1_out]
 *   4 l2w  i8  [stacks][l2_size][pad32(2*l1_hidden)]
 *   5 l2b  i32 [stacks][l2_size]
 *   6 l3w  i8  [stacks][pad32(l2_size)]
 *   7 l3b  i32 [stacks]
 * Scales: FT 127 (i16), dense weights 64 (i8), dense biases 127*64 (i32);
 * round half away from zero, saturating. */
typedef struct BulletOuB200QuantRounding {
    int ft_shift;               /* sfnn_ft_shift, 0..16 (reference default 7) */
    int ft_round;               /* 0 floor, 1 nearest (quant_ft_round) */
    int crelu_round;            /* quant_crelu_round */
    int sqr_clipped_relu_round; /* quant_sqrcrelu_round */
    int final_div_round;        /* quant_final_div_round */
    int fv_scale;               /* > 0: score = raw / fv_scale */
} BulletOuB200QuantRounding;

/* Quantises f32 SFNN parameters (14 handles as in sfnn_train_step_device;
 * absent shared factors null) into the 8 buffers above.  Replaces
 * quantized_sfnn_weights_from_cuda_cpp_readback (bulletou.rs:10050-10300). */
int bulletou_b200_sfnn_quantize_device(BulletOuCudaCppContext* ctx, const BulletOuB200SfnnShape* shape,
    BulletOuCudaCppF32Buffer* const* params, BulletOuCudaCppI32Buffer* const* quantized);

/* Integer forward of a batch with quantised weights: raw_output[batch] (i32,
 * the engine's raw evaluation), optional l1_out[batch][l1_out] (i32 L1 sums)
 * and score_output[batch] (raw / fv_scale with final_div_round).  Features
 * below 0 are padding; features at or above the table's rows are skipped and
 * buckets out of range give raw 0, each counted in errors[0] when errors is
 * given (the reference stops with an error for either).  shape is the
 * training shape (input_size with or without the virtual rows). */
int bulletou_b200_sfnn_integer_forward_device(BulletOuCudaCppContext* ctx, const BulletOuB200SfnnShape* shape,
    size_t batch, size_t max_active, const BulletOuCudaCppI32Buffer* stm_indices,
    const BulletOuCudaCppI32Buffer* nstm_indices, const BulletOuCudaCppI32Buffer* buckets,
    BulletOuCudaCppI32Buffer* const* quantized, const BulletOuB200QuantRounding* rounding,
    BulletOuCudaCppI32Buffer* l1_out, BulletOuCudaCppI32Buffer* raw_output, BulletOuCudaCppI32Buffer* score_output,
    BulletOuCudaCppI32Buffer* errors);


/* ---- teacher-batch producer (PackedSfenValue records -> sparse batch) ----
 * Replaces the host-side batch preparation of the reference's SFNN and HalfKP
 * trainers: prepare_sfnn_fast_batch_from_board_features
 * (crates/bulletou_lib/src/value/teacher_batch.rs:2869-3010) with the
 * HalfKA_hm2 feature map (game/inputs/shogi_halfka_hm2.rs:195-258) and
 * ShogiSfnnLayerStackBucketKind::bucket_from_board (game/outputs.rs:1227-1231),
 * and prepare_halfkp_direct_fast_batch (teacher_batch.rs:1687-1750) with
 * map_halfkp_features_from_packed (game/inputs/shogi_halfkp.rs:161-227). */
#define BULLETOU_B200_FEATURES_HALFKA_HM2 0
#define BULLETOU_B200_FEATURES_HALFKP 1

typedef struct BulletOuB200TeacherConfig {
    int32_t feature_set;    /* BULLETOU_B200_FEATURES_* */
    int32_t max_active;     /* row stride of stm / nstm (40 HalfKA_hm2, 38 HalfKP); at most 48 */
    int32_t hand_bucket;    /* ShogiSfnnHandBucketKind: 0 none, 1 hand4, 2 hand16, 3 hand64, 4 hand64z,
                               5 hand256, 6 hand1024 */
    int32_t king_bucket;    /* ShogiSfnnKingBucketKind: 0 none, 1 king rank 9, 2 king rank 81, 3 k9k9z,
                               4 k13k13z, 5 k21k21, 6 k21k21z, 7 k29k29 */
    float result_blend;     /* target = result_blend * result + score_blend * p(score) */
    float score_blend;
    float rscale;           /* 1 / scale for p(score) = sigmoid(rscale * score) */
    int32_t score_drop_abs; /* entry weight 0 when |score| >= this; < 0 disables */
} BulletOuB200TeacherConfig;

/* records: n_records PackedSfenValue records (40 bytes = 10 words each) in an
 * i32 buffer.  Writes stm / nstm [n_records][max_active] (-1 padded), buckets
 * [n_records] (optional; 0 for HalfKP), targets and entry_weights [n_records].
 * wrm_table (optional, 65536 floats indexed by score + 32768) replaces the
 * sigmoid with the win-rate-model probability.  overflow[0] is increased by
 * the number of records with more than max_active features (the reference
 * aborts the batch on such a record); the caller zeroes it. */
int bulletou_b200_teacher_prepare_device(BulletOuCudaCppContext* ctx, const BulletOuB200TeacherConfig* config,
    const BulletOuCudaCppI32Buffer* records, size_t n_records, const BulletOuCudaCppF32Buffer* wrm_table,
    BulletOuCudaCppI32Buffer* stm_indices, BulletOuCudaCppI32Buffer* nstm_indices,
    BulletOuCudaCppI32Buffer* buckets, BulletOuCudaCppF32Buffer* targets, BulletOuCudaCppF32Buffer* entry_weights,
    BulletOuCudaCppI32Buffer* overflow);

/* HCPE records (38 bytes each: Apery / cshogi HuffmanCodedPos, eval i16,
 * bestMove16, gameResult 0 draw / 1 black win / 2 white win, padding), packed
 * back to back in an i32 buffer of ceil(38 n / 4) words, converted to
 * PackedSfenValue records as the reference's decode_hcpe_record does
 * (crates/bulletou_lib/src/value/loader/hcpe.rs:65-76: from_hcp, then
 * pack_to_psfen, game_ply 0, the result turned to the side to move).  The
 * records that decode are written compacted, in input order, to psv (n x 10
 * words) and their number to count[0]; a record with a king square >= 81 or
 * an unknown hand code is dropped, as the reference's loader skips it.
 * valid (optional) receives the per-record flags. */
/* ---- validation metrics ----
 * Replaces compute_sign_accuracy_with_loss_masked
 * (crates/bulletou_lib/src/validate.rs:353-470) on the host: model outputs [n]
 * and the positions' PackedSfenValue records [n][10 words] (teacher score and
 * game result read from them) -> report[0..7] = compared, sign_matches,
 * predicted_nonnegative, predicted_negative, predicted_zero, drawn_games,
 * filtered_by_score_cap, loss_sampled; report[8..9] = the loss sum as a
 * double (test loss = sum / loss_sampled).  wrm_table (65536 floats, the
 * target's probability per score) is needed by the win-rate-model and BCE
 * losses. */
typedef struct BulletOuB200ValidationConfig {
    int32_t have_results;       /* 0: the legacy score-sign path, no loss */
    int32_t score_drop_abs;     /* < 0: none */
    int32_t loss_kind;          /* 0 sigmoid-pow, 1 win-rate model, 2 BCE with logits */
    float lambda;
    float eval_scale;           /* <= 0: 1/400 */
    float model_output_scale;   /* <= 0: 1 */
    float pow_exp;
    float nnue2score;
    float in_offset;
    float in_scaling;
} BulletOuB200ValidationConfig;

int bulletou_b200_validation_metrics_device(BulletOuCudaCppContext* ctx, const BulletOuB200ValidationConfig* config,
    const BulletOuCudaCppF32Buffer* outputs, const BulletOuCudaCppI32Buffer* records, size_t n,
    const BulletOuCudaCppF32Buffer* wrm_table, BulletOuCudaCppI32Buffer* report);

int bulletou_b200_hcpe_to_psv_device(BulletOuCudaCppContext* ctx, const BulletOuCudaCppI32Buffer* hcpe,
    size_t n_records, BulletOuCudaCppI32Buffer* psv, BulletOuCudaCppI32Buffer* count, BulletOuCudaCppI32Buffer* valid);

#ifdef __cplusplus
}
#endif

#endif /* BULLETOU_B200_H */
