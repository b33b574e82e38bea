// Data-parallel exchange of the SFNN FT gradient rows over peer memory.
//
// The reference trains on one GPU (no collectives); this file is part of the
// additive multi-GPU layer.  With N ranks (one GPU each, NVLink peers), the
// FT table's rows are sharded by chunks of row launches (the chunk layout of
// bulletou_b200/data_parallel.py).  Instead of writing its gradient rows
// locally for a reduce-scatter, each rank's FT row kernel stores every row
// straight into the receive buffer of the row's owner (slot = its own rank),
// and after a chunk's last launch signals the owners.  Each owner then sums
// the N slots of its rows in rank order, runs Ranger on them and stores the
// updated rows into every rank's FT table (the all-gather), and signals the
// ranks.  The next step waits for those signals before it reads a weight.
//
// Peers' buffers come from CUDA IPC handles (bulletou_b200_*_ipc_handle /
// bulletou_b200_ipc_open); loads and stores to them are plain P2P accesses,
// with no TMA and no multicast.  Flags hold a step counter ("epoch") that
// only grows, so they are never reset; signals are system-scope release
// stores after a system-scope fence, waits are system-scope acquire loads,
// bounded at 2 s (a timeout stores an error code and returns).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>

#include "common.cuh"
#include "exchange.cuh"
#include "optim.cuh"

namespace bou {
namespace {

constexpr unsigned long long kExchangeWaitNs = 2000000000ull;

__device__ __forceinline__ unsigned long long exchange_clock() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ int ld_acquire_sys(const int* p) {
    int v;
    asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release_sys(int* p, int v) {
    asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__global__ void exchange_signal_kernel(PeerFlags flags, int world, size_t index, int epoch) {
    const int r = threadIdx.x;
    if (r >= world) return;
    __threadfence_system();
    st_release_sys(flags.p[r] + index, epoch);
}

__global__ void exchange_wait_kernel(const int* flags, int count, int epoch, int* error) {
    if (threadIdx.x != 0) return;
    const unsigned long long t0 = exchange_clock();
    for (int i = 0; i < count; ++i) {
        while (ld_acquire_sys(flags + i) < epoch) {
            if (exchange_clock() - t0 > kExchangeWaitNs) {
                atomicExch(error, 1 + i);
                return;
            }
            __nanosleep(256);
        }
    }
}

__global__ void exchange_scatter_kernel(const float4* __restrict__ src, size_t len4, PeerBuffers dst, int world,
                                        int rank) {
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < len4; i += stride) {
        const float4 v = src[i];
        for (int r = 0; r < world; ++r) reinterpret_cast<float4*>(dst.p[r])[static_cast<size_t>(rank) * len4 + i] = v;
    }
    __threadfence_system();
}

__global__ void exchange_scatter1_kernel(const float* __restrict__ src, size_t len, PeerBuffers dst, int world,
                                         int rank) {
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < len; i += stride) {
        const float v = src[i];
        for (int r = 0; r < world; ++r) dst.p[r][static_cast<size_t>(rank) * len + i] = v;
    }
    __threadfence_system();
}

// dst[i] = sum over the world slots of len floats, in rank order, after each
// CTA re-reads the small flags with acquire semantics (the wait kernel before
// it has seen them all; on its timeout dst is left unchanged).
__global__ void exchange_reduce_kernel(const float* __restrict__ slots, size_t len, int world, const int* flags,
                                       int epoch, float* __restrict__ dst) {
    __shared__ int ready;
    if (threadIdx.x == 0) {
        int all = 1;
        for (int r = 0; r < world; ++r) all &= ld_acquire_sys(flags + r) >= epoch ? 1 : 0;
        ready = all;
    }
    __syncthreads();
    if (!ready) return;
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < len; i += stride) {
        float g = slots[i];
        for (int r = 1; r < world; ++r) g += slots[static_cast<size_t>(r) * len + i];
        dst[i] = g;
    }
}

struct ShardArgs {
    const float4* recv;  // own receive buffer: world slots of slot4 float4
    size_t slot4;
    size_t recv_off4;    // the chunk's shard within a slot
    float4* tables[kExchangeMaxRanks];  // every rank's FT table
    size_t row0;         // first global row of the shard
    size_t rows;         // real rows of the shard
    int width4;
    int world;
    float4* w;           // compact shard state at the chunk's offset
    float4* m;
    float4* v;
    float4* slow;
    RangerArgs a;
    bool skip_quiet;
    const int* flags;    // the chunk's scatter flags (world of them)
    int epoch;
};

// The owner's part of a chunk: gradient = sum of the world slots in rank
// order, the Ranger step of optim.cuh on the compact state, the updated row
// stored into every rank's table.  Each CTA first re-reads the chunk's
// scatter flags with acquire semantics (the wait kernel before it has seen
// them all; on its timeout the CTAs leave the rows unchanged).
template <bool kLookahead>
__global__ void __launch_bounds__(256) shard_ranger_exchange_kernel(ShardArgs s) {
    __shared__ int ready;
    if (threadIdx.x == 0) {
        int all = 1;
        for (int r = 0; r < s.world; ++r) all &= ld_acquire_sys(s.flags + r) >= s.epoch ? 1 : 0;
        ready = all;
    }
    __syncthreads();
    if (!ready) return;
    const size_t n4 = s.rows * static_cast<size_t>(s.width4);
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4; i += stride) {
        float4 g = s.recv[s.recv_off4 + i];
        for (int r = 1; r < s.world; ++r) {
            const float4 x = s.recv[r * s.slot4 + s.recv_off4 + i];
            g.x += x.x;
            g.y += x.y;
            g.z += x.z;
            g.w += x.w;
        }
        float4 w4 = s.w[i], m4 = s.m[i], v4 = s.v[i];
        if (s.skip_quiet && !kLookahead) {
            const unsigned bits = __float_as_uint(g.x) | __float_as_uint(g.y) | __float_as_uint(g.z) |
                                  __float_as_uint(g.w) | __float_as_uint(m4.x) | __float_as_uint(m4.y) |
                                  __float_as_uint(m4.z) | __float_as_uint(m4.w) | __float_as_uint(v4.x) |
                                  __float_as_uint(v4.y) | __float_as_uint(v4.z) | __float_as_uint(v4.w);
            if (bits == 0 && weight_is_quiet(w4.x, s.a) && weight_is_quiet(w4.y, s.a) &&
                weight_is_quiet(w4.z, s.a) && weight_is_quiet(w4.w, s.a))
                continue;  // the step leaves the row as every rank holds it
        }
        radam_coordinate(s.a.gradient_factor * g.x, s.a, w4.x, m4.x, v4.x);
        radam_coordinate(s.a.gradient_factor * g.y, s.a, w4.y, m4.y, v4.y);
        radam_coordinate(s.a.gradient_factor * g.z, s.a, w4.z, m4.z, v4.z);
        radam_coordinate(s.a.gradient_factor * g.w, s.a, w4.w, m4.w, v4.w);
        if (kLookahead) {
            const float4 s4 = s.slow[i];
            w4.x = lookahead_coordinate(w4.x, s4.x, s.a);
            w4.y = lookahead_coordinate(w4.y, s4.y, s.a);
            w4.z = lookahead_coordinate(w4.z, s4.z, s.a);
            w4.w = lookahead_coordinate(w4.w, s4.w, s.a);
            s.slow[i] = w4;
        }
        s.w[i] = w4;
        s.m[i] = m4;
        s.v[i] = v4;
        const size_t row = i / s.width4;
        const size_t t = (s.row0 + row) * s.width4 + (i - row * s.width4);
        for (int r = 0; r < s.world; ++r) s.tables[r][t] = w4;
    }
    __threadfence_system();
}

int exchange_from(const BulletOuB200RowExchange* x, PeerFlags* flags) {
    if (x == nullptr) return fail_message("row exchange: descriptor must not be null");
    if (x->world < 1 || x->world > static_cast<size_t>(kExchangeMaxRanks) || x->rank >= x->world)
        return fail_messagef("row exchange: world %zu / rank %zu outside 1..%d", x->world, x->rank,
                             kExchangeMaxRanks);
    for (size_t r = 0; r < x->world; ++r) {
        if (x->recv[r] == 0 || x->table[r] == 0 || x->flags[r] == 0)
            return fail_messagef("row exchange: rank %zu's buffers missing", r);
        flags->p[r] = reinterpret_cast<int*>(static_cast<uintptr_t>(x->flags[r]));
    }
    return 0;
}

}  // namespace

int launch_exchange_signal(BulletOuCudaCppContext* ctx, const PeerFlags& flags, int world, size_t index, int epoch) {
    exchange_signal_kernel<<<1, 32, 0, ctx->stream>>>(flags, world, index, epoch);
    return check_launch("exchange signal launch");
}

int launch_exchange_scatter(BulletOuCudaCppContext* ctx, const float* src, size_t len, const PeerBuffers& dst,
                            int world, int rank) {
    const bool vec = len % 4 == 0 && (reinterpret_cast<uintptr_t>(src) & 15u) == 0;
    for (int r = 0; r < world && vec; ++r)
        if ((reinterpret_cast<uintptr_t>(dst.p[r]) & 15u) != 0) return fail_message("exchange scatter: unaligned slot");
    const size_t n = vec ? len / 4 : len;
    const int blocks = static_cast<int>(std::min<size_t>((n + 255) / 256, static_cast<size_t>(ctx->sm_count)));
    if (n == 0) return 0;
    if (vec)
        exchange_scatter_kernel<<<blocks, 256, 0, ctx->stream>>>(reinterpret_cast<const float4*>(src), n, dst, world,
                                                                 rank);
    else
        exchange_scatter1_kernel<<<blocks, 256, 0, ctx->stream>>>(src, n, dst, world, rank);
    return check_launch("exchange scatter launch");
}

int launch_exchange_wait(BulletOuCudaCppContext* ctx, const int* flags, int count, int epoch, int* error) {
    exchange_wait_kernel<<<1, 32, 0, ctx->stream>>>(flags, count, epoch, error);
    return check_launch("exchange wait launch");
}

}  // namespace bou

using namespace bou;

namespace {

int ipc_handle_of(const void* ptr, void* handle_out) {
    if (handle_out == nullptr) return fail_message("ipc handle: output must not be null");
    cudaIpcMemHandle_t h;
    const cudaError_t st = cudaIpcGetMemHandle(&h, const_cast<void*>(ptr));
    if (st != cudaSuccess) return fail("cudaIpcGetMemHandle", st);
    static_assert(sizeof(h) == 64, "CUDA IPC handles are 64 bytes");
    memcpy(handle_out, &h, sizeof(h));
    return ok();
}

}  // namespace

int bulletou_b200_f32_buffer_ipc_handle(const BulletOuCudaCppF32Buffer* buffer, void* handle_out) {
    if (buffer == nullptr || buffer->ptr == nullptr || !buffer->owned)
        return fail_message("f32_buffer_ipc_handle: an owning buffer is required");
    if (cudaSetDevice(buffer->device) != cudaSuccess) return fail_message("f32_buffer_ipc_handle: bad device");
    return ipc_handle_of(buffer->ptr, handle_out);
}

int bulletou_b200_i32_buffer_ipc_handle(const BulletOuCudaCppI32Buffer* buffer, void* handle_out) {
    if (buffer == nullptr || buffer->ptr == nullptr) return fail_message("i32_buffer_ipc_handle: buffer required");
    if (cudaSetDevice(buffer->device) != cudaSuccess) return fail_message("i32_buffer_ipc_handle: bad device");
    return ipc_handle_of(buffer->ptr, handle_out);
}

int bulletou_b200_ipc_open(BulletOuCudaCppContext* ctx, const void* handle, unsigned long long* device_address) {
    if (validate_context(ctx) != 0) return -1;
    if (handle == nullptr || device_address == nullptr) return fail_message("ipc_open: null argument");
    if (set_device(ctx) != 0) return -1;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    void* p = nullptr;
    const cudaError_t st = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (st != cudaSuccess) return fail("cudaIpcOpenMemHandle", st);
    *device_address = static_cast<unsigned long long>(reinterpret_cast<uintptr_t>(p));
    return ok();
}

int bulletou_b200_ipc_close(BulletOuCudaCppContext* ctx, unsigned long long device_address) {
    if (validate_context(ctx) != 0) return -1;
    if (set_device(ctx) != 0) return -1;
    const cudaError_t st = cudaIpcCloseMemHandle(reinterpret_cast<void*>(static_cast<uintptr_t>(device_address)));
    if (st != cudaSuccess) return fail("cudaIpcCloseMemHandle", st);
    return ok();
}

int bulletou_b200_exchange_wait_device(BulletOuCudaCppContext* ctx, const BulletOuCudaCppI32Buffer* flags,
                                       size_t offset, size_t count, int epoch, BulletOuCudaCppI32Buffer* error) {
    if (validate_i32(ctx, flags, offset + count, "exchange flags") != 0 ||
        validate_i32(ctx, error, 1, "exchange error word") != 0)
        return -1;
    if (count > 0x7fffffffULL) return fail_message("exchange wait: too many flags");
    if (set_device(ctx) != 0) return -1;
    if (count == 0) return ok();
    return launch_exchange_wait(ctx, flags->ptr + offset, static_cast<int>(count), epoch, error->ptr) == 0 ? ok()
                                                                                                        : -1;
}

int bulletou_b200_sfnn_shard_ranger_exchange_device(
    BulletOuCudaCppContext* ctx, const BulletOuB200RowExchange* x, size_t width, size_t chunk_start,
    size_t chunk_length, size_t shard_rows, size_t shard_off, const BulletOuB200RangerStep* step,
    BulletOuCudaCppF32Buffer* weights, BulletOuCudaCppF32Buffer* momentum, BulletOuCudaCppF32Buffer* velocity,
    BulletOuCudaCppF32Buffer* slow, const BulletOuCudaCppI32Buffer* flags, size_t scatter_index,
    size_t ready_index, BulletOuCudaCppI32Buffer* error) {
    PeerFlags pf{};
    if (exchange_from(x, &pf) != 0) return -1;
    if (step == nullptr) return fail_message("shard ranger exchange: step must not be null");
    if (width == 0 || width % 4 != 0) return fail_message("shard ranger exchange: width must be a multiple of 4");
    const size_t compact = (shard_off + shard_rows) * width;
    if (validate_f32(ctx, weights, compact, "shard weights") != 0 ||
        validate_f32(ctx, momentum, compact, "shard momentum") != 0 ||
        validate_f32(ctx, velocity, compact, "shard velocity") != 0 ||
        validate_f32(ctx, slow, compact, "shard slow weights") != 0 ||
        validate_i32(ctx, flags, scatter_index + x->world, "exchange flags") != 0 ||
        validate_i32(ctx, flags, ready_index + 1, "exchange flags") != 0 ||
        validate_i32(ctx, error, 1, "exchange error word") != 0)
        return -1;
    if (shard_off + shard_rows > x->slot_rows) return fail_message("shard ranger exchange: shard outside the slot");
    if (set_device(ctx) != 0) return -1;
    // rows of this rank inside the chunk's real rows
    const size_t first = chunk_start + x->rank * shard_rows;
    const size_t end = std::min(chunk_start + chunk_length, first + shard_rows);
    ShardArgs s{};
    s.recv = reinterpret_cast<const float4*>(static_cast<uintptr_t>(x->recv[x->rank]));
    s.width4 = static_cast<int>(width / 4);
    s.slot4 = x->slot_rows * (width / 4);
    s.recv_off4 = shard_off * (width / 4);
    for (size_t r = 0; r < x->world; ++r)
        s.tables[r] = reinterpret_cast<float4*>(static_cast<uintptr_t>(x->table[r]));
    s.row0 = first;
    s.rows = end > first ? end - first : 0;
    s.world = static_cast<int>(x->world);
    s.w = reinterpret_cast<float4*>(weights->ptr) + shard_off * (width / 4);
    s.m = reinterpret_cast<float4*>(momentum->ptr) + shard_off * (width / 4);
    s.v = reinterpret_cast<float4*>(velocity->ptr) + shard_off * (width / 4);
    s.slow = reinterpret_cast<float4*>(slow->ptr) + shard_off * (width / 4);
    s.a = ranger_args_from(*step);
    s.skip_quiet = ranger_zero_step_is_identity(s.a);
    s.flags = flags->ptr + scatter_index;
    s.epoch = x->epoch;
    // every rank's rows of this chunk have landed in this rank's slots
    if (launch_exchange_wait(ctx, s.flags, s.world, x->epoch, error->ptr) != 0) return -1;
    const size_t n4 = s.rows * static_cast<size_t>(s.width4);
    if (n4 > 0) {
        const int blocks = static_cast<int>(std::min<size_t>((n4 + 255) / 256, static_cast<size_t>(ctx->sm_count) * 4));
        if (s.a.do_lookahead) shard_ranger_exchange_kernel<true><<<blocks, 256, 0, ctx->stream>>>(s);
        else shard_ranger_exchange_kernel<false><<<blocks, 256, 0, ctx->stream>>>(s);
        if (check_launch("shard ranger exchange launch") != 0) return -1;
    }
    // the updated rows are in every table
    if (launch_exchange_signal(ctx, pf, s.world, ready_index, x->epoch) != 0) return -1;
    return ok();
}

int bulletou_b200_exchange_reduce_small_device(BulletOuCudaCppContext* ctx, const BulletOuB200RowExchange* x,
                                               BulletOuCudaCppF32Buffer* dst, const BulletOuCudaCppI32Buffer* flags,
                                               BulletOuCudaCppI32Buffer* error) {
    PeerFlags pf{};
    if (exchange_from(x, &pf) != 0) return -1;
    if (x->small_len == 0 || x->small_recv[x->rank] == 0)
        return fail_message("exchange reduce small: no small receive buffer");
    if (validate_f32(ctx, dst, x->small_len, "small gradient") != 0 ||
        validate_i32(ctx, flags, x->small_flag_base + x->world, "exchange flags") != 0 ||
        validate_i32(ctx, error, 1, "exchange error word") != 0)
        return -1;
    if (set_device(ctx) != 0) return -1;
    const int* f = flags->ptr + x->small_flag_base;
    if (launch_exchange_wait(ctx, f, static_cast<int>(x->world), x->epoch, error->ptr) != 0) return -1;
    const int blocks =
        static_cast<int>(std::min<size_t>((x->small_len + 255) / 256, static_cast<size_t>(ctx->sm_count) * 2));
    exchange_reduce_kernel<<<blocks, 256, 0, ctx->stream>>>(
        reinterpret_cast<const float*>(static_cast<uintptr_t>(x->small_recv[x->rank])), x->small_len,
        static_cast<int>(x->world), f, x->epoch, dst->ptr);
    return check_launch("exchange reduce launch") == 0 ? ok() : -1;
}
