// Tensor-core sums of the heavy keys of the SFNN FT gradient (sm_100a).
//
// The FT row phase sums, for every key (rank tile t, piece p) of the
// tile-keyed index, the pre-activation gradient rows of the key's entries:
//   sum[t, p][:] = sum over half-positions r of tile t holding piece p of G[r][:]
// i.e. S_t^T G_t with S_t the 0/1 incidence of the tile's ranks and pieces.
// On teacher data the piece-squares of the common king positions hold hundreds
// to thousands of a tile's 4096 ranks ("heavy" keys, ~80 % of all entries at a
// threshold of 64), so for them the product is a dense contraction: this file
// computes it on the 5th-generation tensor cores (tcgen05.mma, accumulator in
// TMEM), and the row kernel only gathers the light keys' entries.
//
//   * The gradient rows come as two bf16 planes G = hi + lo (hi = bf16(G),
//     lo = bf16(G - hi); relative error <= 2^-17 per element), written by the
//     L1 backward in king order, [ranks][W]; each 64-rank x 64-column box is
//     one TMA load with 128-byte swizzle (an MN-major UMMA operand).
//   * The incidence chunk (128 heavy keys x 64 ranks, bf16 0/1, exact) is built
//     in shared memory from the batch's feature rows (rank -> half-position ->
//     its 40 features -> key -> slot), K-major with the same swizzle.
//   * One M=128 x N=256 x K=16 MMA per 16 ranks and plane accumulates in f32
//     in TMEM (256 columns); the chunk pipeline is two stages deep: TMA and the
//     incidence build of chunk c+1 overlap the MMAs of chunk c.
//   * Epilogue: tcgen05.ld of the accumulator, one key row per thread, into the
//     heavy partial rows [slot][W] the row kernel adds.
// The MMA accumulation order is fixed, so the sums are deterministic.  Every
// wait on an mbarrier is bounded (2 s of globaltimer); on a timeout the CTA
// records an error word, waits (bounded) for its own copies in flight, frees
// its TMEM and returns.  No multicast, no cluster.
#include <cuda.h>
#include <cuda_bf16.h>

#include <climits>
#include <cstdint>

#include "ft_rows_mma.cuh"

namespace bou {
namespace {

constexpr int kM = 128;         // heavy keys per M-block (MMA M)
constexpr int kN = 128;         // columns per work item (MMA N)
constexpr int kMaxMb = 4;       // M-blocks per work item: 4 accumulators x 128 TMEM columns
constexpr int kChunk = 64;      // ranks per pipeline stage (4 MMA K-steps of 16)
constexpr int kMaxChunks = 64;  // 4096-rank tiles
constexpr int kThreads = 128;   // 4 warps: TMEM lanes 0-127
constexpr int kStages = 2;
constexpr uint32_t kABytes = kM * kChunk * 2;         // 16 KB incidence chunk of one M-block
constexpr uint32_t kPlaneBytes = kChunk * kN * 2;     // 16 KB per bf16 plane
constexpr uint32_t kStageBytes = kMaxMb * kABytes + 2 * kPlaneBytes;
constexpr uint32_t kSmemBytes = kStages * kStageBytes + 1024 /* align */ + 64;
constexpr uint32_t kTmemCols = kMaxMb * kN;
constexpr uint64_t kWaitNs = 2000000000ull;  // bounded waits: 2 s

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
// Bounded parity wait; false on timeout.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
    uint64_t t0 = 0;
    for (uint32_t i = 0;; ++i) {
        uint32_t done;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
            : "=r"(done)
            : "r"(bar), "r"(parity)
            : "memory");
        if (done) return true;
        if (i == 0) t0 = global_ns();
        else if ((i & 31) == 0 && global_ns() - t0 > kWaitNs) return false;
    }
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}

// UMMA shared-memory descriptor (sm_100): start >> 4 [0,14), leading byte
// offset >> 4 [16,30), stride byte offset >> 4 [32,46), version 1 [46,48),
// layout SWIZZLE_128B = 2 [61,64).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    return static_cast<uint64_t>((addr >> 4) & 0x3fffu) | (static_cast<uint64_t>((lbo >> 4) & 0x3fffu) << 16) |
           (static_cast<uint64_t>((sbo >> 4) & 0x3fffu) << 32) | (1ull << 46) | (2ull << 61);
}
// Instruction descriptor, kind::f16: D f32 [4,6) = 1, A bf16 [7,10) = 1,
// B bf16 [10,13) = 1, A K-major (bit 15 = 0), B MN-major (bit 16 = 1),
// N >> 3 [17,23), M >> 4 [24,29).
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | (1u << 16) | ((uint32_t(kN) >> 3) << 17) |
                            ((uint32_t(kM) >> 4) << 24);

__device__ __forceinline__ void mma_bf16(uint32_t tmem, uint64_t a, uint64_t b, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(tmem),
        "l"(a), "l"(b), "r"(kIdesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

// 32 columns of the accumulator for this warp's 32 TMEM lanes.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// ------------------------------------------------------------------ planning
// One CTA per tile: its rank range (the tiled index's tile_of rule, same as
// TiledMap::key), the heavy keys (entries > threshold) in piece order with
// their local slots, and their count.
__global__ void __launch_bounds__(256) heavy_plan_tile_kernel(HeavyMmaArgs a) {
    __shared__ int warp_tot[8];
    const int t = blockIdx.x;
    const int n_tiles = a.tile_base[a.kings];
    if (t >= a.max_tiles) return;
    if (t >= n_tiles) {
        for (int p = threadIdx.x; p < a.pieces; p += blockDim.x) a.plan.key_local[t * a.pieces + p] = -1;
        if (threadIdx.x == 0) {
            a.plan.tile_heavy[t] = 0;
            a.plan.tile_r0[t] = a.plan.tile_r1[t] = 0;
        }
        return;
    }
    // king block of tile t
    int k = 0;
    while (k + 1 < a.kings && a.tile_base[k + 1] <= t) ++k;
    const int i = t - a.tile_base[k];
    const int nt = a.tile_base[k + 1] - a.tile_base[k];
    const int rb = a.rank_base[k];
    const int re = a.kings == 1 ? a.rank_base_end : a.rank_base[k + 1];
    const int r0 = rb + i * a.tile_ranks;
    const int r1 = (i == nt - 1) ? re : min(re, r0 + a.tile_ranks);
    // heavy keys in piece order: block-wide scan over the pieces
    int run = 0;
    for (int p0 = 0; p0 < a.pieces; p0 += blockDim.x) {
        const int p = p0 + threadIdx.x;
        int heavy = 0;
        if (p < a.pieces) {
            const int key = t * a.pieces + p;
            heavy = (a.offsets[key + 1] - a.offsets[key]) > a.threshold ? 1 : 0;
        }
        // warp + block exclusive scan of `heavy`
        const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
        int incl = heavy;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, incl, d);
            if (lane >= d) incl += y;
        }
        if (lane == 31) warp_tot[warp] = incl;
        __syncthreads();
        int before = run;
        for (int w = 0; w < warp; ++w) before += warp_tot[w];
        int block_total = 0;
        for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) block_total += warp_tot[w];
        if (p < a.pieces) a.plan.key_local[t * a.pieces + p] = heavy ? before + incl - 1 : -1;
        run += block_total;
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        a.plan.tile_heavy[t] = run;
        a.plan.tile_r0[t] = r0;
        a.plan.tile_r1[t] = r1;
    }
}

// One thread: exclusive scans over the tiles of heavy keys (slot base) and of
// M-blocks (incidence base); the work list: per tile, groups of up to kMaxMb
// M-blocks x column groups of kN.
__global__ void heavy_plan_scan_kernel(HeavyMmaArgs a) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    int slots = 0, mbs = 0, work = 0;
    const int groups = a.width / kN;
    for (int t = 0; t < a.max_tiles; ++t) {
        const int h = a.plan.tile_heavy[t];
        const int mblocks = (h + kM - 1) / kM;
        a.plan.tile_slot[t] = slots;
        a.plan.tile_mb[t] = mbs;
        for (int m0 = 0; m0 < mblocks; m0 += kMaxMb) {
            const int nmb = min(kMaxMb, mblocks - m0);
            for (int g = 0; g < groups && work < a.plan.max_work; ++g) {
                a.plan.work[2 * work] = t;
                a.plan.work[2 * work + 1] = (m0 << 16) | (nmb << 8) | g;
                ++work;
            }
        }
        slots += h;
        mbs += mblocks;
    }
    a.plan.tile_slot[a.max_tiles] = slots;
    a.plan.tile_mb[a.max_tiles] = mbs;
    a.plan.n_work[0] = work;
    a.plan.n_slots[0] = slots;
    a.plan.next_work[0] = 0;
}

// Global slot of every key (-1: light).
__global__ void heavy_plan_slot_kernel(HeavyMmaArgs a) {
    const int key = blockIdx.x * blockDim.x + threadIdx.x;
    if (key >= a.max_tiles * a.pieces) return;
    const int local = a.plan.key_local[key];
    const int t = key / a.pieces;
    const bool fits = a.plan.tile_slot[a.max_tiles] <= a.plan.max_slots &&
                      a.plan.tile_mb[a.max_tiles] <= a.plan.max_mblocks;
    a.plan.key_slot[key] = (local < 0 || !fits) ? -1 : a.plan.tile_slot[t] + local;
}

// ------------------------------------------------------------------ the incidence operand
// One CTA per (tile, 64-rank chunk): the 0/1 incidence of the chunk's ranks
// with every heavy key of the tile, bf16, laid out as the MMA reads it
// (K-major, 128-byte swizzle: key row m of an M-block at (m / 8) * 1024 +
// (m % 8) * 128 bytes, 16-byte unit u of the row at (u ^ (m % 8)) * 16), one
// 16 KB chunk per (M-block, chunk) at incidence[(tile_mb[t] + mb) * 64 + c].
__global__ void __launch_bounds__(kThreads) heavy_incidence_kernel(HeavyMmaArgs a) {
    const int t = blockIdx.x, c = blockIdx.y;
    if (a.plan.tile_slot[a.max_tiles] > a.plan.max_slots || a.plan.tile_mb[a.max_tiles] > a.plan.max_mblocks) return;
    const int heavy = a.plan.tile_heavy[t];
    const int r0 = a.plan.tile_r0[t], r1 = a.plan.tile_r1[t];
    const int rc = r0 + c * kChunk;
    if (heavy == 0 || rc >= r1) return;
    const int nmb = (heavy + kM - 1) / kM;
    uint8_t* const base = reinterpret_cast<uint8_t*>(a.plan.incidence);
    const size_t mb0 = static_cast<size_t>(a.plan.tile_mb[t]);
    for (int mb = 0; mb < nmb; ++mb) {
        uint4* z = reinterpret_cast<uint4*>(base + ((mb0 + mb) * kMaxChunks + c) * kABytes);
        for (int i = threadIdx.x; i < static_cast<int>(kABytes / 16); i += kThreads) z[i] = make_uint4(0, 0, 0, 0);
    }
    __syncthreads();
    // two threads per rank, half of its feature slots each
    const int kk = threadIdx.x >> 1;
    const int r = rc + kk;
    if (r >= r1) return;
    const int h = a.order[r];
    const int* idx = ((h & 1) ? a.nstm : a.stm) + static_cast<size_t>(h >> 1) * a.max_active;
    const int half = (a.max_active + 1) >> 1;
    const int sb = (threadIdx.x & 1) * half, se = min(a.max_active, sb + half);
    const uint32_t unit = static_cast<uint32_t>(kk) >> 3, within = (static_cast<uint32_t>(kk) & 7u) * 2;
    for (int q = sb; q < se; ++q) {
        const int f = __ldg(idx + q);
        if (f < 0 || f >= a.kings * a.pieces) continue;
        const int kf = f / a.pieces, p = f - kf * a.pieces;
        // the tiled index's tile of this entry (TiledMap::key)
        const int t0 = a.tile_base[kf], nt = a.tile_base[kf + 1] - t0;
        const int off = r - a.rank_base[kf];
        const int tile = t0 + (off <= 0 ? 0 : min(off / a.tile_ranks, nt - 1));
        if (tile != t) continue;
        const int l = a.plan.key_local[t * a.pieces + p];
        if (l < 0) continue;
        const uint32_t m = static_cast<uint32_t>(l & (kM - 1));
        const size_t chunk = (mb0 + (l >> 7)) * kMaxChunks + c;
        const uint32_t byte = (m >> 3) * 1024u + (m & 7u) * 128u + ((unit ^ (m & 7u)) << 4) + within;
        *reinterpret_cast<uint16_t*>(base + chunk * kABytes + byte) = 0x3f80u;  // bf16 1.0
    }
}

// ------------------------------------------------------------------ the MMA kernel
// Persistent CTAs over the work list; one thread drives a two-stage pipeline
// (bulk copies of the incidence chunks and TMA loads of the gradient planes
// for chunk c + 1 while the MMAs of chunk c run), every M-block of the item
// accumulating into its own 128 TMEM columns; then all four warps read the
// accumulators (warp w: TMEM lanes 32 w .. 32 w + 31) into the partial rows.
__global__ void __launch_bounds__(kThreads, 1) heavy_key_mma_kernel(const __grid_constant__ CUtensorMap map_hi,
                                                                    const __grid_constant__ CUtensorMap map_lo,
                                                                    HeavyMmaArgs a) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;  // 1024-byte aligned stages (128-byte swizzle atoms)
    uint8_t* const sbase = smem_raw + (base - raw);
    uint64_t* const bars = reinterpret_cast<uint64_t*>(sbase + kStages * kStageBytes);  // full[2], done[2]
    uint32_t* const tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kStages);
    int* const abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const uint32_t full_bar0 = smem_u32(bars), done_bar0 = smem_u32(bars + kStages);

    if (a.plan.tile_slot[a.max_tiles] > a.plan.max_slots || a.plan.tile_mb[a.max_tiles] > a.plan.max_mblocks) return;
    const int n_work = a.plan.n_work[0];
    if (static_cast<int>(blockIdx.x) >= n_work) return;

    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(full_bar0 + 8 * s, 1);
            mbar_init(done_bar0 + 8 * s, 1);
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;

    // pipeline state, thread 0 only
    uint32_t full_phase = 0, done_phase = 0;  // bit s: parity to wait for next on stage s
    int pending = 0;                          // bit s: MMAs committed on stage s not yet waited for
    int loads = 0;                            // bit s: loads issued on stage s not yet waited for
    const uint8_t* const inc = reinterpret_cast<const uint8_t*>(a.plan.incidence);

    int* const next = abort_flag + 1;  // the work item this CTA takes next
    if (tid == 0) *next = atomicAdd(a.plan.next_work, 1);
    __syncthreads();
    for (;;) {
        const int w = *next;
        __syncthreads();  // every thread has read `next` before thread 0 fetches the following item
        if (w >= n_work) break;
        const int t = a.plan.work[2 * w];
        const int packed = a.plan.work[2 * w + 1];
        const int m0 = packed >> 16, nmb = (packed >> 8) & 0xff, grp = packed & 0xff;
        const int r0 = a.plan.tile_r0[t], r1 = a.plan.tile_r1[t];
        const int col0 = grp * kN;
        const int chunks = (r1 - r0 + kChunk - 1) / kChunk;
        const size_t mbase = static_cast<size_t>(a.plan.tile_mb[t]) + m0;
        if (tid == 0 && !*abort_flag) {
            bool ok = true;
            auto issue = [&](int c) {
                const int s = c & 1;
                const uint32_t stage = base + s * kStageBytes;
                mbar_expect_tx(full_bar0 + 8 * s, nmb * kABytes + 2 * kPlaneBytes);
                for (int mb = 0; mb < nmb; ++mb)
                    bulk_load(stage + mb * kABytes, inc + ((mbase + mb) * kMaxChunks + c) * kABytes, kABytes,
                              full_bar0 + 8 * s);
                const uint32_t hi = stage + kMaxMb * kABytes, lo = hi + kPlaneBytes;
                for (int j = 0; j < kN / 64; ++j) {
                    tma_load_2d(hi + j * (kChunk * 128), &map_hi, col0 + 64 * j, r0 + c * kChunk, full_bar0 + 8 * s);
                    tma_load_2d(lo + j * (kChunk * 128), &map_lo, col0 + 64 * j, r0 + c * kChunk, full_bar0 + 8 * s);
                }
                loads |= 1 << s;
            };
            auto retire = [&](int s) {  // the MMAs committed on stage s have completed
                if (!(pending & (1 << s))) return true;
                if (!mbar_wait(done_bar0 + 8 * s, (done_phase >> s) & 1)) return false;
                done_phase ^= 1u << s;
                pending &= ~(1 << s);
                return true;
            };
            ok = retire(0) && retire(1);
            if (ok) issue(0);
            for (int c = 0; c < chunks && ok; ++c) {
                const int s = c & 1;
                if (c + 1 < chunks) {
                    if (!retire((c + 1) & 1)) {
                        ok = false;
                        break;
                    }
                    issue(c + 1);
                }
                if (!mbar_wait(full_bar0 + 8 * s, (full_phase >> s) & 1)) {
                    ok = false;
                    break;
                }
                full_phase ^= 1u << s;
                loads &= ~(1 << s);
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t stage = base + s * kStageBytes;
                const uint32_t hi = stage + kMaxMb * kABytes, lo = hi + kPlaneBytes;
#pragma unroll
                for (int k = 0; k < kChunk / 16; ++k) {
                    const uint64_t bh = smem_desc(hi + 2048u * k, 64u * 128u, 1024u);
                    const uint64_t bl = smem_desc(lo + 2048u * k, 64u * 128u, 1024u);
                    for (int mb = 0; mb < nmb; ++mb) {
                        const uint64_t ad = smem_desc(stage + mb * kABytes + 32u * k, 16u, 1024u);
                        const uint32_t d = tmem + static_cast<uint32_t>(mb * kN);
                        mma_bf16(d, ad, bh, (c > 0 || k > 0) ? 1u : 0u);
                        mma_bf16(d, ad, bl, 1u);
                    }
                }
                mma_commit(done_bar0 + 8 * s);
                pending |= 1 << s;
            }
            ok = ok && retire(0) && retire(1);  // accumulators complete
            if (!ok) *abort_flag = 1;
        }
        if (tid == 0) *next = atomicAdd(a.plan.next_work, 1);  // read after the barrier below
        __syncthreads();
        if (*abort_flag) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        // epilogue: thread = key row of each M-block
        const int heavy = a.plan.tile_heavy[t];
        for (int mb = 0; mb < nmb; ++mb) {
            const int row = (m0 + mb) * kM + warp * 32 + lane;
            float* dst = a.plan.partials + static_cast<size_t>(a.plan.tile_slot[t] + row) * a.width + col0;
            for (int cb = 0; cb < kN / 32; ++cb) {
                float v[32];
                tmem_ld32(tmem + (static_cast<uint32_t>(warp * 32) << 16) + static_cast<uint32_t>(mb * kN + cb * 32), v);
                if (row < heavy) {
                    float4* d4 = reinterpret_cast<float4*>(dst + cb * 32);
#pragma unroll
                    for (int i = 0; i < 8; ++i) d4[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
                }
            }
        }
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncthreads();
    }
    if (tid == 0 && *abort_flag) {
        atomicExch(a.plan.error, 1);
        // copies and MMAs still in flight complete before the memory is released
        for (int s = 0; s < kStages; ++s) {
            if (loads & (1 << s)) mbar_wait(full_bar0 + 8 * s, (full_phase >> s) & 1);
            if (pending & (1 << s)) mbar_wait(done_bar0 + 8 * s, (done_phase >> s) & 1);
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
}

// ------------------------------------------------------------------ host
using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encode_fn() {
    static EncodeTiled fn = nullptr;
    static bool tried = false;
    if (!tried) {
        tried = true;
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiled>(p);
    }
    return fn;
}

int plane_map(CUtensorMap* map, const __nv_bfloat16* plane, int rows, int width) {
    EncodeTiled fn = encode_fn();
    if (fn == nullptr) return fail_message("cuTensorMapEncodeTiled is unavailable");
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(width), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(width) * 2};
    const cuuint32_t box[2] = {64, static_cast<cuuint32_t>(kChunk)};
    const cuuint32_t estride[2] = {1, 1};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<__nv_bfloat16*>(plane), dims, strides,
                          box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail_messagef("cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
    return 0;
}

}  // namespace

bool heavy_mma_supported(int width) { return width >= 256 && width % 256 == 0 && width / kN < 256; }

size_t heavy_mma_max_slots(size_t entries, int threshold) { return entries / static_cast<size_t>(threshold + 1) + 1; }

size_t heavy_mma_max_mblocks(int max_tiles, size_t max_slots) {
    return static_cast<size_t>(max_tiles) + max_slots / kM + 1;
}

size_t heavy_mma_max_work(int max_tiles, size_t max_slots, int width) {
    return (static_cast<size_t>(max_tiles) + heavy_mma_max_mblocks(max_tiles, max_slots) / kMaxMb + 1) *
           static_cast<size_t>(width / kN);
}

size_t heavy_mma_incidence_bytes(size_t max_mblocks) { return max_mblocks * kMaxChunks * kABytes; }

int launch_heavy_key_mma(BulletOuCudaCppContext* ctx, HeavyMmaArgs a) {
    if (!heavy_mma_supported(a.width) || a.max_tiles >= (1 << 15) || a.pieces > 2048)
        return fail_message("internal: heavy-key MMA shape unsupported");
    CUtensorMap map_hi, map_lo;
    if (plane_map(&map_hi, a.hi, a.rows, a.width) != 0 || plane_map(&map_lo, a.lo, a.rows, a.width) != 0) return -1;
    heavy_plan_tile_kernel<<<a.max_tiles, 256, 0, ctx->stream>>>(a);
    heavy_plan_scan_kernel<<<1, 32, 0, ctx->stream>>>(a);
    const int keys = a.max_tiles * a.pieces;
    heavy_plan_slot_kernel<<<(keys + 255) / 256, 256, 0, ctx->stream>>>(a);
    heavy_incidence_kernel<<<dim3(a.max_tiles, kMaxChunks), kThreads, 0, ctx->stream>>>(a);
    if (check_launch("heavy-key plan launch") != 0) return -1;
    const cudaError_t st = cudaFuncSetAttribute(heavy_key_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                static_cast<int>(kSmemBytes));
    if (st != cudaSuccess) return fail("cudaFuncSetAttribute heavy-key MMA", st);
    heavy_key_mma_kernel<<<ctx->sm_count, kThreads, kSmemBytes, ctx->stream>>>(map_hi, map_lo, a);
    return check_launch("heavy-key MMA launch");
}

}  // namespace bou
