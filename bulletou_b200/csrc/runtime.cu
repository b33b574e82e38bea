// Runtime half of the drop-in C ABI: errors, contexts, buffers, events,
// graphs, transfers.  Contract (names, argument meaning, validation, error
// codes) follows crates/cuda_cpp/cpp/bulletou_cuda_backend.cu:9471-10306 of
// the reference; the implementation is this library's own.
#include <cstdarg>
#include <cstring>
#include <cfloat>
#include <algorithm>

#include "common.cuh"

namespace bou {

static thread_local std::string g_last_error;

int ok() {
    g_last_error.clear();
    return 0;
}

int fail(const char* context, cudaError_t status) {
    char buffer[512];
    std::snprintf(buffer, sizeof(buffer), "%s: %s (%d)", context, cudaGetErrorString(status), static_cast<int>(status));
    g_last_error = buffer;
    return status == cudaSuccess ? -1 : static_cast<int>(status);
}

int fail_message(const char* message) {
    g_last_error = message;
    return -1;
}

int fail_messagef(const char* fmt, ...) {
    char buffer[512];
    va_list args;
    va_start(args, fmt);
    std::vsnprintf(buffer, sizeof(buffer), fmt, args);
    va_end(args);
    g_last_error = buffer;
    return -1;
}

int check_launch(const char* label) {
    cudaError_t status = cudaGetLastError();
    if (status != cudaSuccess) return fail(label, status);
    return 0;
}

int validate_context(const BulletOuCudaCppContext* ctx) {
    if (ctx == nullptr) return fail_message("context must not be null");
    if (ctx->stream == nullptr && ctx->owns_stream) return fail_message("context stream must not be null");
    return 0;
}

int set_device(const BulletOuCudaCppContext* ctx) {
    if (validate_context(ctx) != 0) return -1;
    cudaError_t status = cudaSetDevice(ctx->device);
    if (status != cudaSuccess) return fail("cudaSetDevice", status);
    return 0;
}

template <typename B>
static int validate_buffer_common(const BulletOuCudaCppContext* ctx, const B* b, size_t len, const char* name,
                                  const char* kind) {
    if (validate_context(ctx) != 0) return -1;
    if (b == nullptr) return fail_messagef("%s %sbuffer must not be null", name, kind);
    if (b->ptr == nullptr && b->len != 0) return fail_messagef("%s %spointer must not be null", name, kind);
    if (b->device != ctx->device)
        return fail_messagef("%s %sbuffer belongs to device %d, context is device %d", name, kind, b->device, ctx->device);
    if (b->len < len)
        return fail_messagef("%s %sbuffer length %zu is smaller than requested length %zu", name, kind, b->len, len);
    return 0;
}

int validate_f32(const BulletOuCudaCppContext* ctx, const BulletOuCudaCppF32Buffer* b, size_t len, const char* name) {
    return validate_buffer_common(ctx, b, len, name, "");
}

int validate_i32(const BulletOuCudaCppContext* ctx, const BulletOuCudaCppI32Buffer* b, size_t len, const char* name) {
    return validate_buffer_common(ctx, b, len, name, "");
}

int validate_host(const void* ptr, size_t len, const char* name) {
    if (len != 0 && ptr == nullptr) return fail_messagef("%s must not be null when len > 0", name);
    return 0;
}

int scratch_slot(BulletOuCudaCppContext* ctx, int slot, size_t bytes, void** out, const char* label) {
    if (slot < 0 || slot >= static_cast<int>(sizeof(ctx->scratch) / sizeof(ctx->scratch[0])))
        return fail_message("internal: scratch slot out of range");
    Scratch& s = ctx->scratch[slot];
    if (bytes == 0) bytes = 256;
    if (s.bytes < bytes) {
        cudaError_t st;
        if (s.ptr != nullptr) {
            st = cudaStreamSynchronize(ctx->stream);
            if (st != cudaSuccess) return fail(label, st);
            st = cudaFree(s.ptr);
            if (st != cudaSuccess) return fail(label, st);
            s.ptr = nullptr;
            s.bytes = 0;
        }
        size_t rounded = (bytes + 255) & ~static_cast<size_t>(255);
        st = cudaMalloc(&s.ptr, rounded);
        if (st != cudaSuccess) {
            s.ptr = nullptr;
            return fail(label, st);
        }
        s.bytes = rounded;
    }
    *out = s.ptr;
    return 0;
}

void prof_mark(BulletOuCudaCppContext* ctx) {
    if (!ctx->prof_on || ctx->prof_used >= ctx->prof_events.size()) return;
    cudaEventRecord(ctx->prof_events[ctx->prof_used++], ctx->stream);
}

}  // namespace bou

using namespace bou;

namespace {

__global__ void fill_f32_kernel(float* __restrict__ out, size_t len, float value) {
    size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (; i < len; i += stride) out[i] = value;
}

__global__ void axpy_f32_kernel(size_t len, float a, const float* __restrict__ x, const float* __restrict__ y,
                                float* __restrict__ out) {
    size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < len) out[i] = a * x[i] + y[i];
}

int launch_fill(BulletOuCudaCppContext* ctx, float* ptr, size_t len, float value, const char* label) {
    if (len == 0) return 0;
    int blocks = static_cast<int>(std::min<size_t>((len + 255) / 256, static_cast<size_t>(ctx->sm_count) * 16));
    fill_f32_kernel<<<blocks, 256, 0, ctx->stream>>>(ptr, len, value);
    return check_launch(label);
}

int init_context(BulletOuCudaCppContext* ctx, int device) {
    ctx->device = device;
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) == cudaSuccess && sms > 0)
        ctx->sm_count = sms;
    return 0;
}

}  // namespace

namespace bou {
int fill_device(BulletOuCudaCppContext* ctx, float* ptr, size_t len, float value, const char* label) {
    return launch_fill(ctx, ptr, len, value, label);
}
}  // namespace bou

namespace {

static int validate_event(const BulletOuCudaCppContext* ctx, const BulletOuCudaCppEvent* ev, const char* what) {
    if (validate_context(ctx) != 0) return -1;
    if (ev == nullptr || ev->event == nullptr) return fail_messagef("event_%s event must not be null", what);
    if (ev->device != ctx->device)
        return fail_messagef("event_%s event belongs to device %d, context is device %d", what, ev->device, ctx->device);
    return 0;
}

template <typename B, typename T>
static int buffer_create(BulletOuCudaCppContext* ctx, size_t len, B** out, bool pinned, const char* what) {
    if (set_device(ctx) != 0) return -1;
    if (out == nullptr) return fail_messagef("%s_create output pointer must not be null", what);
    *out = nullptr;
    auto* b = new B();
    b->device = ctx->device;
    b->len = len;
    if (len != 0) {
        void* p = nullptr;
        cudaError_t st = pinned ? cudaMallocHost(&p, len * sizeof(T)) : cudaMalloc(&p, len * sizeof(T));
        if (st != cudaSuccess) {
            delete b;
            return fail(pinned ? "cudaMallocHost" : "cudaMalloc", st);
        }
        b->ptr = static_cast<T*>(p);
    }
    *out = b;
    return ok();
}

template <typename B>
static int buffer_destroy(B* b, bool pinned, bool owned) {
    if (b == nullptr) return 0;
    cudaError_t st = cudaSetDevice(b->device);
    if (st != cudaSuccess) {
        delete b;
        return fail("cudaSetDevice", st);
    }
    if (owned && b->ptr != nullptr) {
        st = pinned ? cudaFreeHost(b->ptr) : cudaFree(b->ptr);
        if (st != cudaSuccess) {
            delete b;
            return fail(pinned ? "cudaFreeHost" : "cudaFree", st);
        }
    }
    delete b;
    return ok();
}

template <typename B, typename P, typename T>
static int upload_staged(BulletOuCudaCppContext* ctx, B* dst, P* staging, const T* src, size_t len, const char* what) {
    if (validate_buffer_common(ctx, dst, len, "dst", "") != 0 ||
        validate_buffer_common(ctx, staging, len, "staging", "pinned ") != 0 || validate_host(src, len, "src") != 0)
        return -1;
    if (set_device(ctx) != 0) return -1;
    if (len == 0) return ok();
    std::memcpy(staging->ptr, src, len * sizeof(T));
    cudaError_t st = cudaMemcpyAsync(dst->ptr, staging->ptr, len * sizeof(T), cudaMemcpyHostToDevice, ctx->stream);
    if (st != cudaSuccess) return fail(what, st);
    return ok();
}

template <typename B, typename T>
static int upload(BulletOuCudaCppContext* ctx, B* dst, const T* src, size_t len, const char* what) {
    if (validate_buffer_common(ctx, dst, len, "dst", "") != 0 || validate_host(src, len, "src") != 0) return -1;
    if (set_device(ctx) != 0) return -1;
    if (len == 0) return ok();
    cudaError_t st = cudaMemcpyAsync(dst->ptr, src, len * sizeof(T), cudaMemcpyHostToDevice, ctx->stream);
    if (st != cudaSuccess) return fail(what, st);
    return ok();
}

template <typename B, typename T>
static int download(BulletOuCudaCppContext* ctx, const B* src, T* dst, size_t len, const char* what) {
    if (validate_buffer_common(ctx, src, len, "src", "") != 0 || validate_host(dst, len, "dst") != 0) return -1;
    if (set_device(ctx) != 0) return -1;
    if (len == 0) return ok();
    cudaError_t st = cudaMemcpyAsync(dst, src->ptr, len * sizeof(T), cudaMemcpyDeviceToHost, ctx->stream);
    if (st != cudaSuccess) return fail(what, st);
    st = cudaStreamSynchronize(ctx->stream);
    if (st != cudaSuccess) return fail(what, st);
    return ok();
}

template <typename B, typename T>
static int copy_device(BulletOuCudaCppContext* ctx, B* dst, const B* src, size_t len, const char* what) {
    if (validate_buffer_common(ctx, dst, len, "dst", "") != 0 || validate_buffer_common(ctx, src, len, "src", "") != 0)
        return -1;
    if (set_device(ctx) != 0) return -1;
    if (len == 0) return ok();
    cudaError_t st = cudaMemcpyAsync(dst->ptr, src->ptr, len * sizeof(T), cudaMemcpyDeviceToDevice, ctx->stream);
    if (st != cudaSuccess) return fail(what, st);
    return ok();
}

template <typename B, typename P, typename T>
static int copy_pinned(BulletOuCudaCppContext* ctx, B* dev, P* pinned, size_t len, bool h2d, const char* what) {
    if (validate_buffer_common(ctx, dev, len, "device", "") != 0 ||
        validate_buffer_common(ctx, pinned, len, "pinned", "pinned ") != 0 || set_device(ctx) != 0)
        return -1;
    if (len == 0) return ok();
    cudaError_t st = h2d ? cudaMemcpyAsync(dev->ptr, pinned->ptr, len * sizeof(T), cudaMemcpyHostToDevice, ctx->stream)
                         : cudaMemcpyAsync(pinned->ptr, dev->ptr, len * sizeof(T), cudaMemcpyDeviceToHost, ctx->stream);
    if (st != cudaSuccess) return fail(what, st);
    return ok();
}

}  // namespace

extern "C" {

int bulletou_cuda_cpp_last_error(char* out, size_t out_len) {
    if (out == nullptr || out_len == 0) return fail_message("last_error output buffer is null or empty");
    const std::string& msg = g_last_error;
    size_t n = std::min(out_len - 1, msg.size());
    std::memcpy(out, msg.data(), n);
    out[n] = '\0';
    return 0;
}

int bulletou_cuda_cpp_device_name(int device, char* out, size_t out_len) {
    if (out == nullptr || out_len == 0) return fail_message("device_name output buffer is null or empty");
    cudaError_t st = cudaSetDevice(device);
    if (st != cudaSuccess) return fail("cudaSetDevice", st);
    cudaDeviceProp prop{};
    st = cudaGetDeviceProperties(&prop, device);
    if (st != cudaSuccess) return fail("cudaGetDeviceProperties", st);
    size_t n = std::min(out_len - 1, std::strlen(prop.name));
    std::memcpy(out, prop.name, n);
    out[n] = '\0';
    return ok();
}

int bulletou_b200_version(char* out, size_t out_len) {
    if (out == nullptr || out_len == 0) return fail_message("version output buffer is null or empty");
    const char* v = "bulletou_b200 0.1 (sm_100a)";
    size_t n = std::min(out_len - 1, std::strlen(v));
    std::memcpy(out, v, n);
    out[n] = '\0';
    return ok();
}

int bulletou_cuda_cpp_context_create(int device, BulletOuCudaCppContext** out) {
    if (out == nullptr) return fail_message("context_create output pointer must not be null");
    *out = nullptr;
    cudaError_t st = cudaSetDevice(device);
    if (st != cudaSuccess) return fail("cudaSetDevice", st);
    auto* ctx = new BulletOuCudaCppContext();
    init_context(ctx, device);
    st = cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking);
    if (st != cudaSuccess) {
        delete ctx;
        return fail("cudaStreamCreateWithFlags", st);
    }
    ctx->owns_stream = true;
    *out = ctx;
    return ok();
}

int bulletou_b200_context_create_on_stream(int device, void* stream, BulletOuCudaCppContext** out) {
    if (out == nullptr) return fail_message("context_create_on_stream output pointer must not be null");
    *out = nullptr;
    cudaError_t st = cudaSetDevice(device);
    if (st != cudaSuccess) return fail("cudaSetDevice", st);
    auto* ctx = new BulletOuCudaCppContext();
    init_context(ctx, device);
    ctx->stream = static_cast<cudaStream_t>(stream);
    ctx->owns_stream = false;
    *out = ctx;
    return ok();
}

int bulletou_b200_context_stream(const BulletOuCudaCppContext* ctx, void** out) {
    if (validate_context(ctx) != 0) return -1;
    if (out == nullptr) return fail_message("context_stream output pointer must not be null");
    *out = static_cast<void*>(ctx->stream);
    return ok();
}

int bulletou_cuda_cpp_context_destroy(BulletOuCudaCppContext* ctx) {
    if (ctx == nullptr) return 0;
    cudaError_t st = cudaSetDevice(ctx->device);
    if (st != cudaSuccess) {
        delete ctx;
        return fail("cudaSetDevice", st);
    }
    if (ctx->stream != nullptr) cudaStreamSynchronize(ctx->stream);
    int rc = 0;
    for (auto& s : ctx->scratch) {
        if (s.ptr != nullptr) {
            st = cudaFree(s.ptr);
            if (st != cudaSuccess && rc == 0) rc = fail("cudaFree context scratch", st);
            s.ptr = nullptr;
            s.bytes = 0;
        }
    }
    for (auto e : ctx->prof_events) cudaEventDestroy(e);
    ctx->prof_events.clear();
    if (ctx->owns_stream && ctx->stream != nullptr) {
        st = cudaStreamDestroy(ctx->stream);
        if (st != cudaSuccess && rc == 0) rc = fail("cudaStreamDestroy", st);
    }
    delete ctx;
    return rc == 0 ? ok() : rc;
}

// Read bandwidth of a buffer that stays resident in L2: every pass reads the
// whole buffer as 16-byte loads cached in L2 only (ld.global.cg), so after the
// first pass the bytes come from L2.  One partial per thread keeps the loads
// alive.  Used to measure the L2 peak the gather kernels are compared with.
__global__ void l2_read_probe_kernel(const float4* __restrict__ buf, size_t n4, int passes, float* __restrict__ sink) {
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    const size_t t0 = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    float acc = 0.0f;
    for (int p = 0; p < passes; ++p) {
        // a pass-dependent start keeps each thread's addresses moving across
        // the L2 slices from pass to pass
        const size_t shift = (static_cast<size_t>(p) * 7919u * blockDim.x) % n4;
        for (size_t i = t0; i < n4; i += stride) {
            size_t j = i + shift;
            if (j >= n4) j -= n4;
            const float4 v = __ldcg(buf + j);
            acc += (v.x + v.y) + (v.z + v.w);
        }
    }
    sink[t0] = acc;
}

int bulletou_b200_profile_begin(BulletOuCudaCppContext* ctx, size_t max_marks) {
    if (set_device(ctx) != 0) return -1;
    while (ctx->prof_events.size() < max_marks) {
        cudaEvent_t e = nullptr;
        cudaError_t st = cudaEventCreate(&e);
        if (st != cudaSuccess) return fail("cudaEventCreate profile", st);
        ctx->prof_events.push_back(e);
    }
    ctx->prof_used = 0;
    ctx->prof_marks_per_step = 0;
    ctx->prof_on = true;
    return ok();
}

int bulletou_b200_profile_end(BulletOuCudaCppContext* ctx, float* ms_out, size_t ms_len, size_t* steps_out,
                              size_t* phases_out) {
    if (set_device(ctx) != 0) return -1;
    ctx->prof_on = false;
    cudaError_t st = cudaStreamSynchronize(ctx->stream);
    if (st != cudaSuccess) return fail("cudaStreamSynchronize profile", st);
    const size_t per = static_cast<size_t>(ctx->prof_marks_per_step);
    const size_t steps = per == 0 ? 0 : ctx->prof_used / per;
    const size_t phases = per == 0 ? 0 : per - 1;
    for (size_t i = 0; i < ms_len; ++i) ms_out[i] = 0.0f;
    for (size_t s = 0; s < steps; ++s)
        for (size_t p = 0; p < phases && p < ms_len; ++p) {
            float ms = 0.0f;
            st = cudaEventElapsedTime(&ms, ctx->prof_events[s * per + p], ctx->prof_events[s * per + p + 1]);
            if (st != cudaSuccess) return fail("cudaEventElapsedTime profile", st);
            ms_out[p] += ms;
        }
    if (steps_out) *steps_out = steps;
    if (phases_out) *phases_out = phases;
    ctx->prof_used = 0;
    return ok();
}

int bulletou_b200_context_scratch_bytes(const BulletOuCudaCppContext* ctx, size_t* out) {
    if (validate_context(ctx) != 0) return -1;
    if (out == nullptr) return fail_message("context_scratch_bytes: output must not be null");
    size_t total = 0;
    for (const Scratch& s : ctx->scratch) total += s.bytes;
    *out = total;
    return ok();
}

int bulletou_b200_context_wait_before_weights(BulletOuCudaCppContext* ctx, const BulletOuCudaCppEvent* event) {
    if (validate_context(ctx) != 0) return -1;
    if (event != nullptr && (event->event == nullptr || event->device != ctx->device))
        return fail_message("context_wait_before_weights: event missing or on another device");
    ctx->weights_ready = event != nullptr ? event->event : nullptr;
    return ok();
}

int bulletou_b200_context_wait_flags_before_weights(BulletOuCudaCppContext* ctx,
                                                    const BulletOuCudaCppI32Buffer* flags, size_t offset,
                                                    size_t count, int epoch, BulletOuCudaCppI32Buffer* error) {
    if (validate_context(ctx) != 0) return -1;
    if (flags == nullptr || count == 0) {
        ctx->weights_flags = nullptr;
        return ok();
    }
    if (validate_i32(ctx, flags, offset + count, "weights flags") != 0 ||
        validate_i32(ctx, error, 1, "weights flag error word") != 0)
        return -1;
    if (count > 0x7fffffffULL) return fail_message("context_wait_flags_before_weights: too many flags");
    ctx->weights_flags = flags->ptr + offset;
    ctx->weights_flag_count = static_cast<int>(count);
    ctx->weights_flag_epoch = epoch;
    ctx->weights_flag_error = error->ptr;
    return ok();
}

int bulletou_b200_l2_read_probe(BulletOuCudaCppContext* ctx, const BulletOuCudaCppF32Buffer* buffer, size_t len,
                                int passes, BulletOuCudaCppF32Buffer* sink) {
    if (validate_f32(ctx, buffer, len, "L2 probe buffer") != 0) return -1;
    if (len % 4 != 0 || len == 0 || passes <= 0) return fail_message("L2 probe: len must be a positive multiple of 4");
    if (set_device(ctx) != 0) return -1;
    const int threads = 512;
    const int blocks = 4 * ctx->sm_count;
    if (validate_f32(ctx, sink, static_cast<size_t>(threads) * blocks, "L2 probe sink") != 0) return -1;
    l2_read_probe_kernel<<<blocks, threads, 0, ctx->stream>>>(reinterpret_cast<const float4*>(buffer->ptr), len / 4,
                                                              passes, sink->ptr);
    return check_launch("L2 read probe");
}

int bulletou_cuda_cpp_context_synchronize(BulletOuCudaCppContext* ctx) {
    if (set_device(ctx) != 0) return -1;
    cudaError_t st = cudaStreamSynchronize(ctx->stream);
    if (st != cudaSuccess) return fail("cudaStreamSynchronize", st);
    return ok();
}

// ---- events ----
int bulletou_cuda_cpp_event_create(BulletOuCudaCppContext* ctx, BulletOuCudaCppEvent** out) {
    if (set_device(ctx) != 0) return -1;
    if (out == nullptr) return fail_message("event_create output pointer must not be null");
    *out = nullptr;
    auto* ev = new BulletOuCudaCppEvent();
    ev->device = ctx->device;
    cudaError_t st = cudaEventCreateWithFlags(&ev->event, cudaEventDefault);
    if (st != cudaSuccess) {
        delete ev;
        return fail("cudaEventCreateWithFlags", st);
    }
    *out = ev;
    return ok();
}

int bulletou_cuda_cpp_event_destroy(BulletOuCudaCppEvent* event) {
    if (event == nullptr) return 0;
    cudaError_t st = cudaSetDevice(event->device);
    if (st != cudaSuccess) {
        delete event;
        return fail("cudaSetDevice", st);
    }
    if (event->event != nullptr) {
        st = cudaEventDestroy(event->event);
        if (st != cudaSuccess) {
            delete event;
            return fail("cudaEventDestroy", st);
        }
    }
    delete event;
    return ok();
}


int bulletou_cuda_cpp_event_record(BulletOuCudaCppContext* ctx, BulletOuCudaCppEvent* event) {
    if (validate_event(ctx, event, "record") != 0 || set_device(ctx) != 0) return -1;
    cudaError_t st = cudaEventRecord(event->event, ctx->stream);
    if (st != cudaSuccess) return fail("cudaEventRecord", st);
    return ok();
}

int bulletou_cuda_cpp_event_wait(BulletOuCudaCppContext* ctx, BulletOuCudaCppEvent* event) {
    if (validate_event(ctx, event, "wait") != 0 || set_device(ctx) != 0) return -1;
    cudaError_t st = cudaStreamWaitEvent(ctx->stream, event->event, 0);
    if (st != cudaSuccess) return fail("cudaStreamWaitEvent", st);
    return ok();
}

int bulletou_cuda_cpp_event_synchronize(BulletOuCudaCppEvent* event) {
    if (event == nullptr || event->event == nullptr) return fail_message("event_synchronize event must not be null");
    cudaError_t st = cudaSetDevice(event->device);
    if (st != cudaSuccess) return fail("cudaSetDevice", st);
    st = cudaEventSynchronize(event->event);
    if (st != cudaSuccess) return fail("cudaEventSynchronize", st);
    return ok();
}

int bulletou_cuda_cpp_event_elapsed_ms(BulletOuCudaCppEvent* start, BulletOuCudaCppEvent* stop, float* out_ms) {
    if (start == nullptr || start->event == nullptr || stop == nullptr || stop->event == nullptr || out_ms == nullptr)
        return fail_message("event_elapsed_ms arguments must not be null");
    if (start->device != stop->device) return fail_message("event_elapsed_ms events belong to different devices");
    cudaError_t st = cudaSetDevice(start->device);
    if (st != cudaSuccess) return fail("cudaSetDevice", st);
    st = cudaEventElapsedTime(out_ms, start->event, stop->event);
    if (st != cudaSuccess) return fail("cudaEventElapsedTime", st);
    return ok();
}

// ---- graphs ----
int bulletou_cuda_cpp_graph_begin_capture(BulletOuCudaCppContext* ctx) {
    if (set_device(ctx) != 0) return -1;
    cudaError_t st = cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeGlobal);
    if (st != cudaSuccess) return fail("cudaStreamBeginCapture", st);
    return ok();
}

int bulletou_cuda_cpp_graph_end_capture(BulletOuCudaCppContext* ctx, BulletOuCudaCppGraphExec** out) {
    if (set_device(ctx) != 0) return -1;
    if (out == nullptr) return fail_message("graph_end_capture output pointer must not be null");
    *out = nullptr;
    cudaGraph_t graph = nullptr;
    cudaError_t st = cudaStreamEndCapture(ctx->stream, &graph);
    if (st != cudaSuccess) return fail("cudaStreamEndCapture", st);
    cudaGraphExec_t exec = nullptr;
    st = cudaGraphInstantiate(&exec, graph, 0);
    if (st != cudaSuccess) {
        cudaGraphDestroy(graph);
        return fail("cudaGraphInstantiate", st);
    }
    auto* g = new BulletOuCudaCppGraphExec();
    g->device = ctx->device;
    g->graph = graph;
    g->exec = exec;
    *out = g;
    return ok();
}

int bulletou_cuda_cpp_graph_destroy(BulletOuCudaCppGraphExec* graph) {
    if (graph == nullptr) return 0;
    cudaError_t st = cudaSetDevice(graph->device);
    if (st != cudaSuccess) {
        delete graph;
        return fail("cudaSetDevice", st);
    }
    int rc = 0;
    if (graph->exec != nullptr) {
        st = cudaGraphExecDestroy(graph->exec);
        if (st != cudaSuccess) rc = fail("cudaGraphExecDestroy", st);
    }
    if (graph->graph != nullptr) {
        st = cudaGraphDestroy(graph->graph);
        if (st != cudaSuccess && rc == 0) rc = fail("cudaGraphDestroy", st);
    }
    delete graph;
    return rc == 0 ? ok() : rc;
}

int bulletou_cuda_cpp_graph_launch(BulletOuCudaCppContext* ctx, BulletOuCudaCppGraphExec* graph) {
    if (validate_context(ctx) != 0) return -1;
    if (graph == nullptr || graph->exec == nullptr) return fail_message("graph_launch graph must not be null");
    if (graph->device != ctx->device)
        return fail_messagef("graph_launch graph belongs to device %d, context is device %d", graph->device, ctx->device);
    if (set_device(ctx) != 0) return -1;
    cudaError_t st = cudaGraphLaunch(graph->exec, ctx->stream);
    if (st != cudaSuccess) return fail("cudaGraphLaunch", st);
    return ok();
}

// ---- buffers ----


int bulletou_cuda_cpp_f32_buffer_create(BulletOuCudaCppContext* ctx, size_t len, BulletOuCudaCppF32Buffer** out) {
    return buffer_create<BulletOuCudaCppF32Buffer, float>(ctx, len, out, false, "f32_buffer");
}
int bulletou_cuda_cpp_f32_buffer_destroy(BulletOuCudaCppF32Buffer* buffer) {
    return buffer_destroy(buffer, false, buffer == nullptr ? true : buffer->owned);
}
int bulletou_cuda_cpp_i32_buffer_create(BulletOuCudaCppContext* ctx, size_t len, BulletOuCudaCppI32Buffer** out) {
    return buffer_create<BulletOuCudaCppI32Buffer, int>(ctx, len, out, false, "i32_buffer");
}
int bulletou_cuda_cpp_i32_buffer_destroy(BulletOuCudaCppI32Buffer* buffer) { return buffer_destroy(buffer, false, true); }
int bulletou_cuda_cpp_pinned_f32_buffer_create(BulletOuCudaCppContext* ctx, size_t len, BulletOuCudaCppPinnedF32Buffer** out) {
    return buffer_create<BulletOuCudaCppPinnedF32Buffer, float>(ctx, len, out, true, "pinned_f32_buffer");
}
int bulletou_cuda_cpp_pinned_f32_buffer_destroy(BulletOuCudaCppPinnedF32Buffer* buffer) {
    return buffer_destroy(buffer, true, true);
}
int bulletou_cuda_cpp_pinned_i32_buffer_create(BulletOuCudaCppContext* ctx, size_t len, BulletOuCudaCppPinnedI32Buffer** out) {
    return buffer_create<BulletOuCudaCppPinnedI32Buffer, int>(ctx, len, out, true, "pinned_i32_buffer");
}
int bulletou_cuda_cpp_pinned_i32_buffer_destroy(BulletOuCudaCppPinnedI32Buffer* buffer) {
    return buffer_destroy(buffer, true, true);
}

int bulletou_b200_f32_buffer_ptr(const BulletOuCudaCppF32Buffer* buffer, void** out) {
    if (buffer == nullptr || out == nullptr) return fail_message("f32_buffer_ptr arguments must not be null");
    *out = buffer->ptr;
    return ok();
}
int bulletou_b200_i32_buffer_ptr(const BulletOuCudaCppI32Buffer* buffer, void** out) {
    if (buffer == nullptr || out == nullptr) return fail_message("i32_buffer_ptr arguments must not be null");
    *out = buffer->ptr;
    return ok();
}

int bulletou_b200_f32_buffer_view(const BulletOuCudaCppF32Buffer* buffer, size_t offset, size_t len,
                                  BulletOuCudaCppF32Buffer** out) {
    if (buffer == nullptr || out == nullptr) return fail_message("f32_buffer_view arguments must not be null");
    *out = nullptr;
    if (offset > buffer->len || len > buffer->len - offset)
        return fail_messagef("f32_buffer_view [%zu, %zu) exceeds buffer length %zu", offset, offset + len, buffer->len);
    auto* v = new BulletOuCudaCppF32Buffer();
    v->device = buffer->device;
    v->len = len;
    v->ptr = buffer->ptr == nullptr ? nullptr : buffer->ptr + offset;
    v->owned = false;
    *out = v;
    return ok();
}

// ---- transfers ----

int bulletou_cuda_cpp_f32_upload_staged(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* dst,
                                        BulletOuCudaCppPinnedF32Buffer* staging, const float* src, size_t len) {
    return upload_staged(ctx, dst, staging, src, len, "cudaMemcpyAsync staged f32 upload");
}
int bulletou_cuda_cpp_i32_upload_staged(BulletOuCudaCppContext* ctx, BulletOuCudaCppI32Buffer* dst,
                                        BulletOuCudaCppPinnedI32Buffer* staging, const int* src, size_t len) {
    return upload_staged(ctx, dst, staging, src, len, "cudaMemcpyAsync staged i32 upload");
}





int bulletou_b200_i32_upload_pinned(BulletOuCudaCppContext* ctx, BulletOuCudaCppI32Buffer* dst,
                                    const BulletOuCudaCppPinnedI32Buffer* src, size_t len) {
    return copy_pinned<BulletOuCudaCppI32Buffer, BulletOuCudaCppPinnedI32Buffer, int>(
        ctx, dst, const_cast<BulletOuCudaCppPinnedI32Buffer*>(src), len, true, "cudaMemcpyAsync pinned i32 upload");
}
int bulletou_b200_f32_upload_pinned(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* dst,
                                    const BulletOuCudaCppPinnedF32Buffer* src, size_t len) {
    return copy_pinned<BulletOuCudaCppF32Buffer, BulletOuCudaCppPinnedF32Buffer, float>(
        ctx, dst, const_cast<BulletOuCudaCppPinnedF32Buffer*>(src), len, true, "cudaMemcpyAsync pinned f32 upload");
}
int bulletou_b200_f32_download_pinned(BulletOuCudaCppContext* ctx, BulletOuCudaCppPinnedF32Buffer* dst,
                                      const BulletOuCudaCppF32Buffer* src, size_t len) {
    return copy_pinned<BulletOuCudaCppF32Buffer, BulletOuCudaCppPinnedF32Buffer, float>(
        ctx, const_cast<BulletOuCudaCppF32Buffer*>(src), dst, len, false, "cudaMemcpyAsync pinned f32 download");
}
int bulletou_b200_pinned_f32_ptr(const BulletOuCudaCppPinnedF32Buffer* buffer, void** out) {
    if (buffer == nullptr || out == nullptr) return fail_message("pinned_f32_ptr arguments must not be null");
    *out = buffer->ptr;
    return ok();
}
int bulletou_b200_pinned_i32_ptr(const BulletOuCudaCppPinnedI32Buffer* buffer, void** out) {
    if (buffer == nullptr || out == nullptr) return fail_message("pinned_i32_ptr arguments must not be null");
    *out = buffer->ptr;
    return ok();
}

int bulletou_cuda_cpp_i32_upload(BulletOuCudaCppContext* ctx, BulletOuCudaCppI32Buffer* dst, const int* src, size_t len) {
    return upload(ctx, dst, src, len, "cudaMemcpyAsync i32 upload");
}
int bulletou_cuda_cpp_i32_download(BulletOuCudaCppContext* ctx, const BulletOuCudaCppI32Buffer* src, int* dst, size_t len) {
    return download(ctx, src, dst, len, "cudaMemcpyAsync i32 download");
}
int bulletou_cuda_cpp_i32_copy_device(BulletOuCudaCppContext* ctx, BulletOuCudaCppI32Buffer* dst,
                                      const BulletOuCudaCppI32Buffer* src, size_t len) {
    return copy_device<BulletOuCudaCppI32Buffer, int>(ctx, dst, src, len, "cudaMemcpyAsync i32 device copy");
}
int bulletou_cuda_cpp_f32_upload(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* dst, const float* src, size_t len) {
    return upload(ctx, dst, src, len, "cudaMemcpyAsync f32 upload");
}
int bulletou_cuda_cpp_f32_download(BulletOuCudaCppContext* ctx, const BulletOuCudaCppF32Buffer* src, float* dst, size_t len) {
    return download(ctx, src, dst, len, "cudaMemcpyAsync f32 download");
}
int bulletou_cuda_cpp_f32_copy_device(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* dst,
                                      const BulletOuCudaCppF32Buffer* src, size_t len) {
    return copy_device<BulletOuCudaCppF32Buffer, float>(ctx, dst, src, len, "cudaMemcpyAsync f32 device copy");
}

int bulletou_cuda_cpp_f32_fill(BulletOuCudaCppContext* ctx, BulletOuCudaCppF32Buffer* dst, float value, size_t len) {
    if (validate_f32(ctx, dst, len, "dst") != 0) return -1;
    if (set_device(ctx) != 0) return -1;
    if (launch_fill(ctx, dst->ptr, len, value, "fill_f32_kernel launch") != 0) return -1;
    return ok();
}

int bulletou_cuda_cpp_axpy_device(BulletOuCudaCppContext* ctx, size_t len, float a, const BulletOuCudaCppF32Buffer* x,
                                  const BulletOuCudaCppF32Buffer* y, BulletOuCudaCppF32Buffer* out) {
    if (validate_f32(ctx, x, len, "x") != 0 || validate_f32(ctx, y, len, "y") != 0 ||
        validate_f32(ctx, out, len, "out") != 0)
        return -1;
    if (set_device(ctx) != 0) return -1;
    if (len == 0) return ok();
    int blocks = 0;
    if (grid_1d(len, 256, &blocks, "axpy") != 0) return -1;
    axpy_f32_kernel<<<blocks, 256, 0, ctx->stream>>>(len, a, x->ptr, y->ptr, out->ptr);
    if (check_launch("axpy_kernel launch") != 0) return -1;
    return ok();
}

int bulletou_cuda_cpp_axpy_host(int device, size_t len, float a, const float* x, const float* y, float* out) {
    if (validate_host(x, len, "x") != 0 || validate_host(y, len, "y") != 0 || validate_host(out, len, "out") != 0)
        return -1;
    BulletOuCudaCppContext* ctx = nullptr;
    if (bulletou_cuda_cpp_context_create(device, &ctx) != 0) return -1;
    BulletOuCudaCppF32Buffer *dx = nullptr, *dy = nullptr, *dout = nullptr;
    int rc = bulletou_cuda_cpp_f32_buffer_create(ctx, len, &dx);
    if (rc == 0) rc = bulletou_cuda_cpp_f32_buffer_create(ctx, len, &dy);
    if (rc == 0) rc = bulletou_cuda_cpp_f32_buffer_create(ctx, len, &dout);
    if (rc == 0) rc = bulletou_cuda_cpp_f32_upload(ctx, dx, x, len);
    if (rc == 0) rc = bulletou_cuda_cpp_f32_upload(ctx, dy, y, len);
    if (rc == 0) rc = bulletou_cuda_cpp_axpy_device(ctx, len, a, dx, dy, dout);
    if (rc == 0) rc = bulletou_cuda_cpp_f32_download(ctx, dout, out, len);
    std::string saved = rc == 0 ? std::string() : g_last_error;
    bulletou_cuda_cpp_f32_buffer_destroy(dx);
    bulletou_cuda_cpp_f32_buffer_destroy(dy);
    bulletou_cuda_cpp_f32_buffer_destroy(dout);
    bulletou_cuda_cpp_context_destroy(ctx);
    if (rc != 0) {
        g_last_error = saved;
        return rc;
    }
    return ok();
}

}  // extern "C"
