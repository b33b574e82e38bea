// Production-shape HalfKP step kernels (l1 in {256, 512}, l2 = l3 = 32) for B200.
//
// Reference semantics: crates/cuda_cpp/cpp/bulletou_cuda_backend.cu
//   FT forward cu:1021-1052, dense forward cu:1083-1124, loss cu:2790-2843,
//   dense backward cu:5042-5240, FT activation backward cu:5256-5283.
//
// Layout of the work:
//   1. king sort  -- the 2*B half-positions (sample, perspective) are
//      counting-sorted by king (feature / 1548).  A HalfKP perspective's 38
//      rows all live in its king's 1548-row block (1.5 MB), so consecutive
//      warps gather from the same block and the 128 MB table is streamed from
//      HBM about once per step instead of re-fetched from random kings.
//   2. gather     -- one warp per half-position, 8 columns per lane, 128-bit
//      loads, four rows in flight; bias + rows in slot order (the reference's
//      summation order), ClippedReLU, written to act[b][persp*l1 + c].
//   3. dense      -- one warp per 8 positions, register-tiled: lane (ps, q)
//      owns outputs 4q..4q+3 of positions ps and ps+4.  Every output keeps the
//      reference's sequential FMA order over its inputs, so activations and
//      outputs are bit-identical to the reference kernels.  Loss and the whole
//      per-position backward (to the FT pre-activation gradient) follow in the
//      same kernel; l1w sits in shared memory with a 36-float row stride so the
//      forward (row-wise) and backward (column-wise) reads are conflict-free.
//   4. reduce     -- every small-parameter gradient (dW1, dW2, biases, output
//      layer, l0 bias) and the loss sum as per-chunk partial sums (fixed order).
//   5. finalize   -- partials summed in chunk order; Ranger on the small groups.
#include <mutex>

#include "halfkp_fast.cuh"
#include "king_sort.cuh"

namespace bou {

namespace {

constexpr unsigned kFull = 0xffffffffu;
constexpr int kKingKeys = 82;  // 81 kings + one bucket for perspectives without a valid feature
constexpr int kHalfkpPieces = 1548;
constexpr int kGatherWarps = 8;
template <int L1>
__host__ __device__ constexpr int dense_warps() { return L1 == 256 ? 16 : 8; }  // l1w in smem: 74 KB (256) / 147 KB (512)
constexpr int kTilePos = 8;     // positions per dense warp tile
constexpr int kWStride = 36;    // smem row stride (floats) of l1w / l2w / l2w^T
constexpr int kReduceTile = 16; // positions per reduce-kernel tile
constexpr int kReduceChunk = 128;

__device__ __forceinline__ float crelu01(float x) { return fminf(fmaxf(x, 0.0f), 1.0f); }
__device__ __forceinline__ float crelu_grad(float a, float g) { return a > 0.0f && a < 1.0f ? g : 0.0f; }

// ------------------------------------------------------------------ gather
// A lane owns columns [4*lane, 4*lane+4) and [128+4*lane, 128+4*lane+4) of
// every 256-column block, so each warp-wide float4 load reads 512 contiguous
// bytes (4 L1 wavefronts).
template <int Q>
__device__ __forceinline__ void add_row(float (&acc)[Q][8], const float* __restrict__ l0w, int row, int lane) {
    const float* p = l0w + static_cast<size_t>(row) * (Q * 256) + lane * 4;
#pragma unroll
    for (int q = 0; q < Q; ++q) {
        const float4 a = __ldg(reinterpret_cast<const float4*>(p + q * 256));
        const float4 b = __ldg(reinterpret_cast<const float4*>(p + q * 256 + 128));
        acc[q][0] += a.x; acc[q][1] += a.y; acc[q][2] += a.z; acc[q][3] += a.w;
        acc[q][4] += b.x; acc[q][5] += b.y; acc[q][6] += b.z; acc[q][7] += b.w;
    }
}

template <int Q>
__device__ __forceinline__ void add_row_pair(float (&acc)[Q][8], const float* __restrict__ l0w, int r0, int r1,
                                             int lane) {
    const float* p0 = l0w + static_cast<size_t>(r0) * (Q * 256) + lane * 4;
    const float* p1 = l0w + static_cast<size_t>(r1) * (Q * 256) + lane * 4;
#pragma unroll
    for (int q = 0; q < Q; ++q) {
        const float4 a0 = __ldg(reinterpret_cast<const float4*>(p0 + q * 256));
        const float4 b0 = __ldg(reinterpret_cast<const float4*>(p0 + q * 256 + 128));
        const float4 a1 = __ldg(reinterpret_cast<const float4*>(p1 + q * 256));
        const float4 b1 = __ldg(reinterpret_cast<const float4*>(p1 + q * 256 + 128));
        acc[q][0] += a0.x + a1.x; acc[q][1] += a0.y + a1.y; acc[q][2] += a0.z + a1.z; acc[q][3] += a0.w + a1.w;
        acc[q][4] += b0.x + b1.x; acc[q][5] += b0.y + b1.y; acc[q][6] += b0.z + b1.z; acc[q][7] += b0.w + b1.w;
    }
}

// acc = bias + the position's valid rows in slot order (cu:1037-1050).
template <int Q>
__device__ __forceinline__ void gather_perspective(float (&acc)[Q][8], const int* __restrict__ idx, int max_active,
                                                   const RowMap& map, const float* __restrict__ l0w,
                                                   const float* __restrict__ l0b, int lane) {
#pragma unroll
    for (int q = 0; q < Q; ++q) {
        const float4 a = __ldg(reinterpret_cast<const float4*>(l0b + q * 256 + lane * 4));
        const float4 b = __ldg(reinterpret_cast<const float4*>(l0b + q * 256 + lane * 4 + 128));
        acc[q][0] = a.x; acc[q][1] = a.y; acc[q][2] = a.z; acc[q][3] = a.w;
        acc[q][4] = b.x; acc[q][5] = b.y; acc[q][6] = b.z; acc[q][7] = b.w;
    }
    for (int c0 = 0; c0 < max_active; c0 += 32) {
        const int mine = c0 + lane < max_active ? __ldg(idx + c0 + lane) : -1;
        const int cnt = min(32, max_active - c0);
        if (map.factorized) {
            for (int s = 0; s < cnt; ++s) {
                const int f = __shfl_sync(kFull, mine, s);
                int r0, r1;
                const int n = map.rows(f, &r0, &r1);
                if (n == 1) add_row<Q>(acc, l0w, r0, lane);
                else if (n == 2) add_row_pair<Q>(acc, l0w, r0, r1, lane);
            }
            continue;
        }
        int s = 0;
        for (; s + 4 <= cnt; s += 4) {
            int f[4];
            bool ok[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                f[u] = __shfl_sync(kFull, mine, s + u);
                ok[u] = f[u] >= 0 && f[u] < map.input_size;
            }
            float4 x[4][Q][2];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const float* p = l0w + static_cast<size_t>(ok[u] ? f[u] : 0) * (Q * 256) + lane * 4;
#pragma unroll
                for (int q = 0; q < Q; ++q) {
                    if (ok[u]) {
                        x[u][q][0] = __ldg(reinterpret_cast<const float4*>(p + q * 256));
                        x[u][q][1] = __ldg(reinterpret_cast<const float4*>(p + q * 256 + 128));
                    }
                }
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                if (!ok[u]) continue;
#pragma unroll
                for (int q = 0; q < Q; ++q) {
                    acc[q][0] += x[u][q][0].x; acc[q][1] += x[u][q][0].y;
                    acc[q][2] += x[u][q][0].z; acc[q][3] += x[u][q][0].w;
                    acc[q][4] += x[u][q][1].x; acc[q][5] += x[u][q][1].y;
                    acc[q][6] += x[u][q][1].z; acc[q][7] += x[u][q][1].w;
                }
            }
        }
        for (; s < cnt; ++s) {
            const int f = __shfl_sync(kFull, mine, s);
            if (f >= 0 && f < map.input_size) add_row<Q>(acc, l0w, f, lane);
        }
    }
}

template <int Q>
__global__ void __launch_bounds__(kGatherWarps * 32) ft_gather_kernel(
    const int* __restrict__ order, int n_half, const int* __restrict__ stm, const int* __restrict__ nstm, int A,
    RowMap map, const float* __restrict__ l0w, const float* __restrict__ l0b, float* __restrict__ act,
    float* __restrict__ stm_l0, float* __restrict__ nstm_l0) {
    constexpr int L1 = Q * 256;
    const int lane = threadIdx.x & 31;
    const int i = blockIdx.x * kGatherWarps + (threadIdx.x >> 5);
    if (i >= n_half) return;
    const int h = order != nullptr ? order[i] : i;
    const int b = h >> 1, persp = h & 1;
    float acc[Q][8];
    gather_perspective<Q>(acc, (persp ? nstm : stm) + static_cast<size_t>(b) * A, A, map, l0w, l0b, lane);
    float* out = act + static_cast<size_t>(b) * (2 * L1) + persp * L1 + lane * 4;
    float* side = persp ? nstm_l0 : stm_l0;
#pragma unroll
    for (int q = 0; q < Q; ++q) {
        const float4 lo = make_float4(crelu01(acc[q][0]), crelu01(acc[q][1]), crelu01(acc[q][2]), crelu01(acc[q][3]));
        const float4 hi = make_float4(crelu01(acc[q][4]), crelu01(acc[q][5]), crelu01(acc[q][6]), crelu01(acc[q][7]));
        *reinterpret_cast<float4*>(out + q * 256) = lo;
        *reinterpret_cast<float4*>(out + q * 256 + 128) = hi;
        if (side != nullptr) {
            float* sp = side + static_cast<size_t>(b) * L1 + q * 256 + lane * 4;
            *reinterpret_cast<float4*>(sp) = lo;
            *reinterpret_cast<float4*>(sp + 128) = hi;
        }
    }
}

// ------------------------------------------------------------------ dense
struct DenseArgs {
    int batch;
    HalfkpWeights w;
    HalfkpActivations a;
    const float* targets;
    const float* entry_weights;
    LossArgs loss;
};

template <int L1>
struct DenseSmem {
    static constexpr int kIn = 2 * L1;
    static constexpr int kW1 = kIn * kWStride;
    static constexpr int kW2 = 32 * kWStride;
    static constexpr int kPerWarp = 4 * kTilePos * kWStride + kTilePos;  // h1, h2, g2, g1 tiles + gout
    static constexpr size_t kBytes = sizeof(float) * (kW1 + 2 * kW2 + 32 + dense_warps<L1>() * kPerWarp);
};

__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }

template <int L1, bool kTrain>
__global__ void __launch_bounds__(dense_warps<L1>() * 32, 1) halfkp_dense_kernel(DenseArgs d) {
    constexpr int kDenseWarps = dense_warps<L1>();
    using S = DenseSmem<L1>;
    constexpr int kIn = S::kIn;
    extern __shared__ float4 smem4[];
    float* w1s = reinterpret_cast<float*>(smem4);  // [kIn][36]  l1w[i][j]
    float* w2s = w1s + S::kW1;                     // [32][36]   l2w[j][k]
    float* w2t = w2s + S::kW2;                     // [32][36]   l2w[j][k] at [k][j]
    float* outw_s = w2t + S::kW2;                  // [32]
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float* wsm = outw_s + 32 + warp * S::kPerWarp;
    float* h1s = wsm;                              // [8][36]
    float* h2s = h1s + kTilePos * kWStride;
    float* g2s = h2s + kTilePos * kWStride;
    float* g1s = g2s + kTilePos * kWStride;
    float* gouts = g1s + kTilePos * kWStride;      // [8]

    for (int e = threadIdx.x; e < kIn * 32; e += blockDim.x) w1s[(e >> 5) * kWStride + (e & 31)] = d.w.l1w[e];
    for (int e = threadIdx.x; e < 32 * 32; e += blockDim.x) {
        const float v = d.w.l2w[e];
        w2s[(e >> 5) * kWStride + (e & 31)] = v;
        w2t[(e & 31) * kWStride + (e >> 5)] = v;
    }
    if (threadIdx.x < 32) outw_s[threadIdx.x] = d.w.outw[threadIdx.x];
    __syncthreads();

    const int ps = lane >> 3, q = lane & 7, jq = q * 4;
    const float4 b1 = ld4(d.w.l1b + jq);
    const float4 b2 = ld4(d.w.l2b + jq);
    const float bout = d.w.outb[0];
    const int tiles = (d.batch + kTilePos - 1) / kTilePos;
    for (int tile = blockIdx.x * kDenseWarps + warp; tile < tiles; tile += gridDim.x * kDenseWarps) {
        const int pa = tile * kTilePos + ps, pb = pa + 4;
        const bool va = pa < d.batch, vb = pb < d.batch;
        const float* acta = d.a.act + static_cast<size_t>(va ? pa : 0) * kIn;
        const float* actb = d.a.act + static_cast<size_t>(vb ? pb : 0) * kIn;
        // ---- L1: h[j] = b[j] + sum_i act[i] * l1w[i][j], i ascending ----
        float ha[4] = {b1.x, b1.y, b1.z, b1.w}, hb[4] = {b1.x, b1.y, b1.z, b1.w};
#pragma unroll 2
        for (int i4 = 0; i4 < kIn / 4; ++i4) {
            const float4 xa = __ldg(reinterpret_cast<const float4*>(acta) + i4);
            const float4 xb = __ldg(reinterpret_cast<const float4*>(actb) + i4);
            const float xav[4] = {xa.x, xa.y, xa.z, xa.w};
            const float xbv[4] = {xb.x, xb.y, xb.z, xb.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float4 w = ld4(w1s + (i4 * 4 + e) * kWStride + jq);
                ha[0] = fmaf(xav[e], w.x, ha[0]); ha[1] = fmaf(xav[e], w.y, ha[1]);
                ha[2] = fmaf(xav[e], w.z, ha[2]); ha[3] = fmaf(xav[e], w.w, ha[3]);
                hb[0] = fmaf(xbv[e], w.x, hb[0]); hb[1] = fmaf(xbv[e], w.y, hb[1]);
                hb[2] = fmaf(xbv[e], w.z, hb[2]); hb[3] = fmaf(xbv[e], w.w, hb[3]);
            }
        }
        float4 h1a = make_float4(crelu01(ha[0]), crelu01(ha[1]), crelu01(ha[2]), crelu01(ha[3]));
        float4 h1b = make_float4(crelu01(hb[0]), crelu01(hb[1]), crelu01(hb[2]), crelu01(hb[3]));
        *reinterpret_cast<float4*>(h1s + ps * kWStride + jq) = h1a;
        *reinterpret_cast<float4*>(h1s + (ps + 4) * kWStride + jq) = h1b;
        if (va) *reinterpret_cast<float4*>(d.a.hidden1 + static_cast<size_t>(pa) * 32 + jq) = h1a;
        if (vb) *reinterpret_cast<float4*>(d.a.hidden1 + static_cast<size_t>(pb) * 32 + jq) = h1b;
        __syncwarp();
        // ---- L2 (j ascending) ----
        float sa[4] = {b2.x, b2.y, b2.z, b2.w}, sb[4] = {b2.x, b2.y, b2.z, b2.w};
#pragma unroll 8
        for (int j = 0; j < 32; ++j) {
            const float4 w = ld4(w2s + j * kWStride + jq);
            const float xa = h1s[ps * kWStride + j], xb = h1s[(ps + 4) * kWStride + j];
            sa[0] = fmaf(xa, w.x, sa[0]); sa[1] = fmaf(xa, w.y, sa[1]); sa[2] = fmaf(xa, w.z, sa[2]);
            sa[3] = fmaf(xa, w.w, sa[3]);
            sb[0] = fmaf(xb, w.x, sb[0]); sb[1] = fmaf(xb, w.y, sb[1]); sb[2] = fmaf(xb, w.z, sb[2]);
            sb[3] = fmaf(xb, w.w, sb[3]);
        }
        const float4 h2a = make_float4(crelu01(sa[0]), crelu01(sa[1]), crelu01(sa[2]), crelu01(sa[3]));
        const float4 h2b = make_float4(crelu01(sb[0]), crelu01(sb[1]), crelu01(sb[2]), crelu01(sb[3]));
        *reinterpret_cast<float4*>(h2s + ps * kWStride + jq) = h2a;
        *reinterpret_cast<float4*>(h2s + (ps + 4) * kWStride + jq) = h2b;
        if (va) *reinterpret_cast<float4*>(d.a.hidden2 + static_cast<size_t>(pa) * 32 + jq) = h2a;
        if (vb) *reinterpret_cast<float4*>(d.a.hidden2 + static_cast<size_t>(pb) * 32 + jq) = h2b;
        __syncwarp();
        // ---- output (k ascending) + loss: lanes q == 0 own positions ps, ps+4 ----
        if (q == 0) {
#pragma unroll
            for (int t = 0; t < 2; ++t) {
                const int p = t == 0 ? pa : pb;
                const int slot = ps + 4 * t;
                float o = bout;
#pragma unroll 8
                for (int k = 0; k < 32; ++k) o = fmaf(h2s[slot * kWStride + k], outw_s[k], o);
                float gout = 0.0f;
                if (p < d.batch) {
                    d.a.output[p] = o;
                    if (kTrain) {
                        const float psl = sample_loss(d.loss, o, d.targets[p], d.entry_weights[p], &gout);
                        d.a.per_sample[p] = psl;
                        d.a.mog[p] = gout;
                    }
                }
                gouts[slot] = gout;
            }
        }
        if (!kTrain) {
            __syncwarp();
            continue;
        }
        __syncwarp();
        // ---- L2 backward: g2 = mask(h2) * (gout * outw) ----
        const float ga_out = gouts[ps], gb_out = gouts[ps + 4];
        const float4 ow = ld4(outw_s + jq);
        const float4 g2a = make_float4(crelu_grad(h2a.x, ga_out * ow.x), crelu_grad(h2a.y, ga_out * ow.y),
                                       crelu_grad(h2a.z, ga_out * ow.z), crelu_grad(h2a.w, ga_out * ow.w));
        const float4 g2b = make_float4(crelu_grad(h2b.x, gb_out * ow.x), crelu_grad(h2b.y, gb_out * ow.y),
                                       crelu_grad(h2b.z, gb_out * ow.z), crelu_grad(h2b.w, gb_out * ow.w));
        *reinterpret_cast<float4*>(g2s + ps * kWStride + jq) = g2a;
        *reinterpret_cast<float4*>(g2s + (ps + 4) * kWStride + jq) = g2b;
        if (va) *reinterpret_cast<float4*>(d.a.g2 + static_cast<size_t>(pa) * 32 + jq) = g2a;
        if (vb) *reinterpret_cast<float4*>(d.a.g2 + static_cast<size_t>(pb) * 32 + jq) = g2b;
        __syncwarp();
        // ---- L1 backward: d1[j] = sum_k g2[k] * l2w[j][k] (k ascending), g1 = mask(h1) * d1 ----
        float da[4] = {0.f, 0.f, 0.f, 0.f}, db[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 8
        for (int k = 0; k < 32; ++k) {
            const float4 w = ld4(w2t + k * kWStride + jq);
            const float xa = g2s[ps * kWStride + k], xb = g2s[(ps + 4) * kWStride + k];
            da[0] = fmaf(xa, w.x, da[0]); da[1] = fmaf(xa, w.y, da[1]); da[2] = fmaf(xa, w.z, da[2]);
            da[3] = fmaf(xa, w.w, da[3]);
            db[0] = fmaf(xb, w.x, db[0]); db[1] = fmaf(xb, w.y, db[1]); db[2] = fmaf(xb, w.z, db[2]);
            db[3] = fmaf(xb, w.w, db[3]);
        }
        const float4 g1a = make_float4(crelu_grad(h1a.x, da[0]), crelu_grad(h1a.y, da[1]), crelu_grad(h1a.z, da[2]),
                                       crelu_grad(h1a.w, da[3]));
        const float4 g1b = make_float4(crelu_grad(h1b.x, db[0]), crelu_grad(h1b.y, db[1]), crelu_grad(h1b.z, db[2]),
                                       crelu_grad(h1b.w, db[3]));
        *reinterpret_cast<float4*>(g1s + ps * kWStride + jq) = g1a;
        *reinterpret_cast<float4*>(g1s + (ps + 4) * kWStride + jq) = g1b;
        if (va) *reinterpret_cast<float4*>(d.a.g1 + static_cast<size_t>(pa) * 32 + jq) = g1a;
        if (vb) *reinterpret_cast<float4*>(d.a.g1 + static_cast<size_t>(pb) * 32 + jq) = g1b;
        __syncwarp();
        // ---- FT pre-activation gradient: dc[i] = sum_j g1[j] * l1w[i][j] (j ascending),
        //      lane q owns rows i = 32*it + q + 8*e (e < 4): conflict-free LDS.128 ----
        float* pga = d.a.pregrad + static_cast<size_t>(va ? pa : 0) * kIn;
        float* pgb = d.a.pregrad + static_cast<size_t>(vb ? pb : 0) * kIn;
        for (int it = 0; it < kIn / 32; ++it) {
            float ca[4] = {0.f, 0.f, 0.f, 0.f}, cb[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int j4 = 0; j4 < 8; ++j4) {
                const float4 xa = ld4(g1s + ps * kWStride + j4 * 4);
                const float4 xb = ld4(g1s + (ps + 4) * kWStride + j4 * 4);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float4 w = ld4(w1s + (it * 32 + q + 8 * e) * kWStride + j4 * 4);
                    ca[e] = fmaf(xa.x, w.x, ca[e]); ca[e] = fmaf(xa.y, w.y, ca[e]);
                    ca[e] = fmaf(xa.z, w.z, ca[e]); ca[e] = fmaf(xa.w, w.w, ca[e]);
                    cb[e] = fmaf(xb.x, w.x, cb[e]); cb[e] = fmaf(xb.y, w.y, cb[e]);
                    cb[e] = fmaf(xb.z, w.z, cb[e]); cb[e] = fmaf(xb.w, w.w, cb[e]);
                }
            }
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int i = it * 32 + q + 8 * e;
                if (va) pga[i] = crelu_grad(__ldg(acta + i), ca[e]);
                if (vb) pgb[i] = crelu_grad(__ldg(actb + i), cb[e]);
            }
        }
        __syncwarp();
    }
}

// ------------------------------------------------------------------ batch reductions
// Per chunk of positions: dW1 = sum act x g1, dW2 = sum h1 x g2, db1 = sum g1,
// db2 = sum g2, dOut = sum mog*h2, dOutb = sum mog, dl0b = sum (pg_stm + pg_nstm),
// loss = sum per_sample.  Partials [chunk][layout below]; fixed summation order.
template <int L1>
struct ReduceLayout {
    static constexpr int kIn = 2 * L1;
    static constexpr int kW1 = 0;
    static constexpr int kW2 = kIn * 32;
    static constexpr int kB1 = kW2 + 1024;
    static constexpr int kB2 = kB1 + 32;
    static constexpr int kOut = kB2 + 32;
    static constexpr int kOutB = kOut + 32;
    static constexpr int kL0b = kOutB + 1;
    static constexpr int kLoss = kL0b + L1;
    static constexpr int kTotal = kLoss + 1;
};

template <int L1>
__global__ void __launch_bounds__(256) halfkp_reduce_kernel(HalfkpActivations a, int batch, int chunk,
                                                            float* __restrict__ partials) {
    using R = ReduceLayout<L1>;
    constexpr int kIn = R::kIn;
    constexpr int kSlice = 512;            // L1-layer inputs per CTA (blockIdx.y selects the slice)
    constexpr int kIPer = kSlice / 8;      // inputs per thread: 8 input groups x 32 outputs
    __shared__ __align__(16) float act_s[kReduceTile][kSlice];
    __shared__ float g1_s[kReduceTile][32];
    __shared__ float h1_s[kReduceTile][32];
    __shared__ float g2_s[kReduceTile][32];
    __shared__ float h2_s[kReduceTile][32];
    __shared__ float mog_s[kReduceTile];
    __shared__ float ps_s[kReduceTile];
    const int t = threadIdx.x;
    const int j = t & 31, ib = t >> 5;
    const int slice = blockIdx.y * kSlice;
    const bool lead = blockIdx.y == 0;     // slice 0 also does every vector reduction
    float acc[kIPer];
#pragma unroll
    for (int i = 0; i < kIPer; ++i) acc[i] = 0.0f;
    float acc2[4] = {0.f, 0.f, 0.f, 0.f};
    float acc_l0b[L1 / 256] = {};
    float acc_vec = 0.0f;  // t < 32: db1[t]; 32..63: db2; 64..95: dOut; 96: dOutb; 97: loss
    const int b0 = blockIdx.x * chunk;
    const int b1 = min(batch, b0 + chunk);
    for (int base = b0; base < b1; base += kReduceTile) {
        const int np = min(kReduceTile, b1 - base);
        for (int e = t; e < kReduceTile * (kSlice / 4); e += 256) {
            const int p = e / (kSlice / 4), c4 = e % (kSlice / 4);
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (p < np)
                v = __ldg(reinterpret_cast<const float4*>(a.act + static_cast<size_t>(base + p) * kIn + slice) + c4);
            *reinterpret_cast<float4*>(&act_s[p][c4 * 4]) = v;
        }
        for (int e = t; e < kReduceTile * 32; e += 256) {
            const int p = e >> 5, c = e & 31;
            const size_t off = static_cast<size_t>(base + p) * 32 + c;
            g1_s[p][c] = p < np ? a.g1[off] : 0.0f;
            h1_s[p][c] = p < np ? a.hidden1[off] : 0.0f;
            g2_s[p][c] = p < np ? a.g2[off] : 0.0f;
        }
        if (lead) {
            // l0 bias: column sums of the pre-activation gradient (stm + nstm)
            float sv[kReduceTile][L1 / 256], nv[kReduceTile][L1 / 256];
#pragma unroll
            for (int p = 0; p < kReduceTile; ++p) {
                const float* pg = a.pregrad + static_cast<size_t>(base + min(p, np - 1)) * kIn;
#pragma unroll
                for (int r = 0; r < L1 / 256; ++r) {
                    sv[p][r] = __ldg(pg + r * 256 + t);
                    nv[p][r] = __ldg(pg + L1 + r * 256 + t);
                }
            }
            for (int p = 0; p < np; ++p)
#pragma unroll
                for (int r = 0; r < L1 / 256; ++r) acc_l0b[r] += sv[p][r] + nv[p][r];
        }
        for (int e = t; e < kReduceTile * 32; e += 256) {
            const int p = e >> 5, c = e & 31;
            h2_s[p][c] = (lead && p < np) ? a.hidden2[static_cast<size_t>(base + p) * 32 + c] : 0.0f;
        }
        if (t < kReduceTile) {
            mog_s[t] = (lead && t < np) ? a.mog[base + t] : 0.0f;
            ps_s[t] = (lead && t < np) ? a.per_sample[base + t] : 0.0f;
        }
        __syncthreads();
        if (lead && t < 98) {
            for (int p = 0; p < np; ++p) {
                if (t < 32) acc_vec += g1_s[p][t];
                else if (t < 64) acc_vec += g2_s[p][t - 32];
                else if (t < 96) acc_vec = fmaf(mog_s[p], h2_s[p][t - 64], acc_vec);
                else if (t == 96) acc_vec += mog_s[p];
                else acc_vec += ps_s[p];
            }
        }
        for (int p = 0; p < np; ++p) {
            const float g = g1_s[p][j];
            const float4* row = reinterpret_cast<const float4*>(&act_s[p][ib * kIPer]);
#pragma unroll
            for (int i4 = 0; i4 < kIPer / 4; ++i4) {
                const float4 x = row[i4];
                acc[i4 * 4 + 0] = fmaf(x.x, g, acc[i4 * 4 + 0]);
                acc[i4 * 4 + 1] = fmaf(x.y, g, acc[i4 * 4 + 1]);
                acc[i4 * 4 + 2] = fmaf(x.z, g, acc[i4 * 4 + 2]);
                acc[i4 * 4 + 3] = fmaf(x.w, g, acc[i4 * 4 + 3]);
            }
            if (lead) {
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int e = t + 256 * u;
                    acc2[u] = fmaf(h1_s[p][e >> 5], g2_s[p][e & 31], acc2[u]);
                }
            }
        }
        __syncthreads();
    }
    float* out = partials + static_cast<size_t>(blockIdx.x) * R::kTotal;
#pragma unroll
    for (int ii = 0; ii < kIPer; ++ii) out[R::kW1 + (slice + ib * kIPer + ii) * 32 + j] = acc[ii];
    if (!lead) return;
#pragma unroll
    for (int u = 0; u < 4; ++u) out[R::kW2 + t + 256 * u] = acc2[u];
#pragma unroll
    for (int r = 0; r < L1 / 256; ++r) out[R::kL0b + r * 256 + t] = acc_l0b[r];
    if (t < 32) out[R::kB1 + t] = acc_vec;
    else if (t < 64) out[R::kB2 + t - 32] = acc_vec;
    else if (t < 96) out[R::kOut + t - 64] = acc_vec;
    else if (t == 96) out[R::kOutB] = acc_vec;
    else if (t == 97) out[R::kLoss] = acc_vec;
}

// Sums the chunk partials in chunk order; Ranger on the small groups, or the
// packed gradient written out.  Packed order l0b | l1w | l1b | l2w | l2b | outw | outb.
template <int L1>
__global__ void __launch_bounds__(256) halfkp_finalize_kernel(const float* __restrict__ partials, int nparts,
                                                              SmallGroups groups, RangerArgs ranger, int write_mode,
                                                              float* __restrict__ dense_out,
                                                              float* __restrict__ weighted_sum, float* __restrict__ mean,
                                                              float batch_f, int finalize) {
    using R = ReduceLayout<L1>;
    const int total = groups.begin[7];
    const int e = blockIdx.x * blockDim.x + threadIdx.x;
    if (e == total && finalize) {
        float s = 0.0f;
        for (int p = 0; p < nparts; ++p) s += partials[static_cast<size_t>(p) * R::kTotal + R::kLoss];
        *weighted_sum = s;
        *mean = s / batch_f;
    }
    if (e >= total) return;
    int g = 0;
    while (e >= groups.begin[g + 1]) ++g;
    const int k = e - groups.begin[g];
    const int src = g == 0 ? R::kL0b + k : g == 1 ? R::kW1 + k : g == 2 ? R::kB1 + k : g == 3 ? R::kW2 + k
                  : g == 4 ? R::kB2 + k : g == 5 ? R::kOut + k : R::kOutB;
    float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
    int p = 0;
    for (; p + 4 <= nparts; p += 4) {
        s0 += partials[static_cast<size_t>(p) * R::kTotal + src];
        s1 += partials[static_cast<size_t>(p + 1) * R::kTotal + src];
        s2 += partials[static_cast<size_t>(p + 2) * R::kTotal + src];
        s3 += partials[static_cast<size_t>(p + 3) * R::kTotal + src];
    }
    for (; p < nparts; ++p) s0 += partials[static_cast<size_t>(p) * R::kTotal + src];
    const float grad = (s0 + s1) + (s2 + s3);
    if (write_mode) {
        dense_out[e] = grad;
        return;
    }
    float w = groups.w[g][k], m = groups.m[g][k], v = groups.v[g][k];
    radam_coordinate(ranger.gradient_factor * grad, ranger, w, m, v);
    if (ranger.do_lookahead) {
        w = lookahead_coordinate(w, groups.s[g][k], ranger);
        groups.s[g][k] = w;
    }
    groups.w[g][k] = w;
    groups.m[g][k] = m;
    groups.v[g][k] = v;
}

template <int Q>
int launch_gather(BulletOuCudaCppContext* ctx, const int* order, int n_half, const int* stm, const int* nstm, int A,
                  const RowMap& map, const float* l0w, const float* l0b, float* act, float* stm_l0, float* nstm_l0) {
    const int blocks = (n_half + kGatherWarps - 1) / kGatherWarps;
    ft_gather_kernel<Q><<<blocks, kGatherWarps * 32, 0, ctx->stream>>>(order, n_half, stm, nstm, A, map, l0w, l0b, act,
                                                                        stm_l0, nstm_l0);
    return check_launch("FT gather launch");
}

template <int L1, bool kTrain>
int launch_dense(BulletOuCudaCppContext* ctx, const DenseArgs& a) {
    auto kernel = halfkp_dense_kernel<L1, kTrain>;
    const size_t smem = DenseSmem<L1>::kBytes;
    cudaError_t st = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (st != cudaSuccess) return fail("cudaFuncSetAttribute HalfKP dense", st);
    constexpr int kDenseWarps = dense_warps<L1>();
    const int tiles = (a.batch + kTilePos - 1) / kTilePos;
    int grid = (tiles + kDenseWarps - 1) / kDenseWarps;
    if (grid > ctx->sm_count) grid = ctx->sm_count;
    kernel<<<grid, kDenseWarps * 32, smem, ctx->stream>>>(a);
    return check_launch("HalfKP dense launch");
}

}  // namespace

int halfkp_fast_forward_backward(BulletOuCudaCppContext* ctx, const HalfkpDims& d, const RowMap& map, const int* stm,
                                 const int* nstm, const HalfkpWeights& w, const HalfkpActivations& a,
                                 const float* targets, const float* entry_weights, const LossArgs* loss,
                                 float* stm_l0, float* nstm_l0) {
    const int n_half = 2 * d.batch;
    void* sort_mem = nullptr;
    const size_t sort_ints = king_sort_scratch_ints<kKingKeys>(n_half);
    if (scratch_slot(ctx, kScratchKingSort, sort_ints * sizeof(int), &sort_mem, "cudaMalloc king sort") != 0) return -1;
    KingSortOut sorted{};
    if (king_sort<kKingKeys>(ctx, stm, nstm, n_half, KingKey{kHalfkpPieces, d.input_size, d.max_active},
                             static_cast<int*>(sort_mem), nullptr, &sorted) != 0)
        return -1;
    const int* order = sorted.order;
    prof_mark(ctx);
    const int rc = d.l1 == 256 ? launch_gather<1>(ctx, order, n_half, stm, nstm, d.max_active, map, w.l0w, w.l0b,
                                                  a.act, stm_l0, nstm_l0)
                               : launch_gather<2>(ctx, order, n_half, stm, nstm, d.max_active, map, w.l0w, w.l0b,
                                                  a.act, stm_l0, nstm_l0);
    if (rc != 0) return -1;
    prof_mark(ctx);
    DenseArgs da{};
    da.batch = d.batch;
    da.w = w;
    da.a = a;
    da.targets = targets;
    da.entry_weights = entry_weights;
    if (loss != nullptr) da.loss = *loss;
    if (loss != nullptr)
        return d.l1 == 256 ? launch_dense<256, true>(ctx, da) : launch_dense<512, true>(ctx, da);
    return d.l1 == 256 ? launch_dense<256, false>(ctx, da) : launch_dense<512, false>(ctx, da);
}

int halfkp_fast_small_params(BulletOuCudaCppContext* ctx, const HalfkpDims& d, const HalfkpActivations& a,
                             const SmallGroups& groups, const RangerArgs* ranger, float* dense_out,
                             float* weighted_sum, float* mean, int finalize) {
    const int chunks = (d.batch + kReduceChunk - 1) / kReduceChunk;
    const size_t per = d.l1 == 256 ? ReduceLayout<256>::kTotal : ReduceLayout<512>::kTotal;
    void* parts = nullptr;
    if (scratch_slot(ctx, kScratchDensePartials, static_cast<size_t>(chunks) * per * sizeof(float), &parts,
                     "cudaMalloc HalfKP partials") != 0)
        return -1;
    float* p = static_cast<float*>(parts);
    if (d.l1 == 256) halfkp_reduce_kernel<256><<<dim3(chunks, 1), 256, 0, ctx->stream>>>(a, d.batch, kReduceChunk, p);
    else halfkp_reduce_kernel<512><<<dim3(chunks, 2), 256, 0, ctx->stream>>>(a, d.batch, kReduceChunk, p);
    if (check_launch("HalfKP reduce launch") != 0) return -1;
    prof_mark(ctx);
    const int total = groups.begin[7];
    const int fblocks = (total + 1 + 255) / 256;
    const RangerArgs ra = ranger != nullptr ? *ranger : RangerArgs{};
    const float batch_f = static_cast<float>(d.batch);
    if (d.l1 == 256)
        halfkp_finalize_kernel<256><<<fblocks, 256, 0, ctx->stream>>>(p, chunks, groups, ra, ranger == nullptr,
                                                                      dense_out, weighted_sum, mean, batch_f, finalize);
    else
        halfkp_finalize_kernel<512><<<fblocks, 256, 0, ctx->stream>>>(p, chunks, groups, ra, ranger == nullptr,
                                                                      dense_out, weighted_sum, mean, batch_f, finalize);
    return check_launch("HalfKP finalize launch");
}

}  // namespace bou

// ---------------------------------------------------------------------------
// Allocation-free HalfKP forward (bulletou_b200_nnue_forward_device_noalloc).
//
// The only scratch the production-shape forward needs is the king sort's
// (bucket offsets, keys, order, per-block histograms).  Here it lives in one
// file-scope device array sized for kNoAllocMaxBatch positions, so the entry
// point never calls cudaMalloc: it is usable by callers that cannot allocate
// device memory at run time.  Every kernel overwrites each scratch word before
// reading it, so nothing needs clearing between calls; the array is shared by
// all calls on a device, so calls whose work overlaps on the GPU race.
namespace bou {
namespace {

constexpr int kNoAllocMaxBatch = 65536;
constexpr int kNoAllocMaxHalf = 2 * kNoAllocMaxBatch;
constexpr size_t kNoAllocInts = king_sort_scratch_ints<kKingKeys>(kNoAllocMaxHalf);
constexpr int kNoAllocMaxDevices = 64;

__device__ __align__(256) int g_noalloc_king_scratch[kNoAllocInts];

std::mutex g_noalloc_mutex;
int* g_noalloc_device_ptr[kNoAllocMaxDevices] = {};

// Device address of the static scratch on `device` (which must be current);
// resolved once per device.
int noalloc_scratch(int device, int** out) {
    if (device < 0 || device >= kNoAllocMaxDevices) return fail_messagef("no-allocation forward: device %d unsupported", device);
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    if (g_noalloc_device_ptr[device] == nullptr) {
        void* p = nullptr;
        cudaError_t st = cudaGetSymbolAddress(&p, g_noalloc_king_scratch);
        if (st != cudaSuccess) return fail("cudaGetSymbolAddress no-allocation scratch", st);
        g_noalloc_device_ptr[device] = static_cast<int*>(p);
    }
    *out = g_noalloc_device_ptr[device];
    return 0;
}

}  // namespace
}  // namespace bou

extern "C" int bulletou_b200_nnue_forward_device_noalloc(
    BulletOuCudaCppContext* ctx, size_t input_size, size_t l1, size_t l2, size_t l3, size_t batch, size_t max_active,
    const BulletOuCudaCppI32Buffer* stm_indices, const BulletOuCudaCppI32Buffer* nstm_indices,
    const BulletOuCudaCppF32Buffer* l0w, const BulletOuCudaCppF32Buffer* l0b, const BulletOuCudaCppF32Buffer* l1w,
    const BulletOuCudaCppF32Buffer* l1b, const BulletOuCudaCppF32Buffer* l2w, const BulletOuCudaCppF32Buffer* l2b,
    const BulletOuCudaCppF32Buffer* outw, const BulletOuCudaCppF32Buffer* outb, BulletOuCudaCppF32Buffer* stm_l0,
    BulletOuCudaCppF32Buffer* nstm_l0, BulletOuCudaCppF32Buffer* combined, BulletOuCudaCppF32Buffer* hidden1,
    BulletOuCudaCppF32Buffer* hidden2, BulletOuCudaCppF32Buffer* output) {
    using namespace bou;
    if (input_size == 0 || l1 == 0 || l2 == 0 || l3 == 0 || batch == 0 || max_active == 0)
        return fail_message("NNUE shape, batch and max_active must be greater than zero");
    if (!halfkp_fast_shape(l1, l2, l3, batch, max_active))
        return fail_message("no-allocation forward supports l1 in {256, 512}, l2 = l3 = 32 and max_active <= 4096; "
                            "use bulletou_cuda_cpp_nnue_forward_device for other shapes");
    if (batch > static_cast<size_t>(kNoAllocMaxBatch))
        return fail_messagef("no-allocation forward: batch %zu exceeds its static scratch limit of %d positions",
                             batch, kNoAllocMaxBatch);
    if (input_size > static_cast<size_t>(INT_MAX / 2))
        return fail_message("no-allocation forward: input_size too large");
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
    if (set_device(ctx) != 0) return -1;
    int* scratch = nullptr;
    if (noalloc_scratch(ctx->device, &scratch) != 0) return -1;
    const HalfkpDims d{static_cast<int>(input_size), static_cast<int>(l1), static_cast<int>(batch),
                       static_cast<int>(max_active)};
    const RowMap map = make_row_map(input_size);
    const int n_half = 2 * d.batch;
    KingSortOut sorted{};
    if (king_sort<kKingKeys>(ctx, stm_indices->ptr, nstm_indices->ptr, n_half,
                             KingKey{kHalfkpPieces, d.input_size, d.max_active}, scratch, nullptr, &sorted) != 0)
        return -1;
    const int* order = sorted.order;
    const int rc = d.l1 == 256 ? launch_gather<1>(ctx, order, n_half, stm_indices->ptr, nstm_indices->ptr,
                                                  d.max_active, map, l0w->ptr, l0b->ptr, combined->ptr, stm_l0->ptr,
                                                  nstm_l0->ptr)
                               : launch_gather<2>(ctx, order, n_half, stm_indices->ptr, nstm_indices->ptr,
                                                  d.max_active, map, l0w->ptr, l0b->ptr, combined->ptr, stm_l0->ptr,
                                                  nstm_l0->ptr);
    if (rc != 0) return -1;
    DenseArgs da{};
    da.batch = d.batch;
    da.w = HalfkpWeights{l0w->ptr, l0b->ptr, l1w->ptr, l1b->ptr, l2w->ptr, l2b->ptr, outw->ptr, outb->ptr};
    da.a = HalfkpActivations{combined->ptr, hidden1->ptr, hidden2->ptr, output->ptr, nullptr,
                             nullptr,       nullptr,      nullptr,      nullptr};
    const int rd = d.l1 == 256 ? launch_dense<256, false>(ctx, da) : launch_dense<512, false>(ctx, da);
    return rd == 0 ? ok() : rd;
}
