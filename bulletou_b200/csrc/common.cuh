// Shared runtime pieces of libbulletou_b200: opaque handle layouts, the
// thread-local error string, argument validation and launch helpers.
//
// Error contract follows the reference backend's C ABI
// (crates/cuda_cpp/cpp/bulletou_cuda_backend.cu:209-272): 0 on success, -1 or
// the cudaError_t code on failure, message kept per host thread.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <cstdio>
#include <string>
#include <vector>

#include "../../include/bulletou_cuda_cpp.h"
#include "../../include/bulletou_b200.h"

namespace bou {

// Grow-only device scratch owned by a context.  Never shrinks during a run, so
// buffers handed to an enqueued kernel stay valid until the context dies.
struct Scratch {
    void* ptr = nullptr;
    size_t bytes = 0;
};

}  // namespace bou

struct BulletOuCudaCppContext {
    int device = 0;
    cudaStream_t stream = nullptr;
    bool owns_stream = true;
    int sm_count = 148;
    // Named scratch slots; see scratch_slot in runtime.cu.
    bou::Scratch scratch[32];
    // Dense QAT mode between bulletou_dense_qat_begin / _end (the reference's
    // context flags, cu:9356-9382): integer L1 / L2 / L3 in the SFNN entries.
    bool dense_qat = false;
    bool dense_qat_integer_ft = false;
    const float* dense_qat_l2_bias = nullptr;
    const float* dense_qat_l3_bias = nullptr;
    // Event the next SFNN fused step waits for before reading a weight
    // (bulletou_b200_context_wait_before_weights); cleared by that step.
    cudaEvent_t weights_ready = nullptr;
    // Flags the next SFNN fused step waits for before reading a weight
    // (bulletou_b200_context_wait_flags_before_weights); cleared by that step.
    const int* weights_flags = nullptr;
    int weights_flag_count = 0;
    int weights_flag_epoch = 0;
    int* weights_flag_error = nullptr;
    // Stage profiler (bulletou_b200_profile_*): events recorded on `stream`
    // at phase boundaries of the fused steps, read back after the run.
    bool prof_on = false;
    int prof_marks_per_step = 0;
    std::vector<cudaEvent_t> prof_events;
    size_t prof_used = 0;
};

struct BulletOuCudaCppF32Buffer {
    int device = 0;
    size_t len = 0;
    float* ptr = nullptr;
    bool owned = true;  // false for views (bulletou_b200_f32_buffer_view)
};

struct BulletOuCudaCppI32Buffer {
    int device = 0;
    size_t len = 0;
    int* ptr = nullptr;
};

struct BulletOuCudaCppPinnedF32Buffer {
    int device = 0;
    size_t len = 0;
    float* ptr = nullptr;
};

struct BulletOuCudaCppPinnedI32Buffer {
    int device = 0;
    size_t len = 0;
    int* ptr = nullptr;
};

struct BulletOuCudaCppEvent {
    int device = 0;
    cudaEvent_t event = nullptr;
};

struct BulletOuCudaCppGraphExec {
    int device = 0;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
};

namespace bou {

// Scratch slot ids (one allocation each per context).
enum ScratchSlot : int {
    kScratchCsrCounts = 0,
    kScratchCsrOffsets = 1,
    kScratchCsrCursor = 2,
    kScratchCsrEntries = 3,
    kScratchPregrad = 4,
    kScratchDensePartials = 5,
    kScratchDenseGrads = 6,
    kScratchLossPartials = 7,
    kScratchStepStatus = 8,
    kScratchSmallState = 9,
    kScratchKppt = 10,
    kScratchHost = 11,
    kScratchActivations = 12,
    kScratchKingSort = 13,
    kScratchSfnnFold = 14,      // folded FT table
    kScratchSfnnStep = 15,      // SFNN per-step activations / gradients
    kScratchSfnnSort = 16,      // SFNN king + bucket sort, tile table
    kScratchSfnnPartials = 17,  // SFNN per-tile partial sums
    kScratchSfnnGrads = 18,     // SFNN packed small-parameter gradients
    kScratchSfnnEff = 19,       // SFNN effective (shared-factor folded) dense weights
    kScratchSfnnVirtual = 20,   // SFNN per-piece virtual-row gradient sums between row launches
    kScratchSfnnQuant = 21,     // SFNN integer forward: FT pair values + king sort
    kScratchSfnnQat = 22,       // SFNN QAT: quantised L1 bias, integer biases, raw L1 / L2 sums
    kScratchSfnnQatFt = 23,     // SFNN QAT: fake-quantised FT bias
    kScratchSfnnHeavyMma = 24,  // SFNN FT rows: tensor-core heavy-key plan and sums
    kScratchNnueQuant = 25,     // integer HalfKP forward: transformed features (u8)
    kScratchSfnnHeavy = 26,     // SFNN FT rows: segment plan and partial sums of heavy rows
    kScratchHcpe = 27,          // HCPE -> PackedSfenValue: uncompacted records, valid flags, scan
    kScratchValidation = 28,    // validation metrics: per-CTA partials
};

int ok();
int fail(const char* context, cudaError_t status);
int fail_message(const char* message);
int fail_messagef(const char* fmt, ...);
int check_launch(const char* label);

int validate_context(const BulletOuCudaCppContext* ctx);
int set_device(const BulletOuCudaCppContext* ctx);
int validate_f32(const BulletOuCudaCppContext* ctx, const BulletOuCudaCppF32Buffer* b, size_t len, const char* name);
int validate_i32(const BulletOuCudaCppContext* ctx, const BulletOuCudaCppI32Buffer* b, size_t len, const char* name);
int validate_host(const void* ptr, size_t len, const char* name);

// Returns a device pointer with at least `bytes` bytes (256-byte aligned),
// growing the slot if needed.  Growing synchronizes the context stream first
// so no in-flight kernel still uses the old allocation.
int scratch_slot(BulletOuCudaCppContext* ctx, int slot, size_t bytes, void** out, const char* label);

// Records the next stage-profiler event when profiling is on (no-op otherwise).
void prof_mark(BulletOuCudaCppContext* ctx);

inline int grid_1d(size_t work, int threads, int* blocks, const char* label) {
    size_t b = (work + threads - 1) / threads;
    if (b > 0x7fffffffULL) return fail_messagef("%s: grid too large (%zu blocks)", label, b);
    *blocks = static_cast<int>(b);
    return 0;
}

}  // namespace bou
