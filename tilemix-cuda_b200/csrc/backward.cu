// Backward pass of the unrouted (every tile FP16) TileMix attention on sm_100a
// tensor cores. The reference has no backward; this is the gradient of
//   O = softmax(score_scale * Q K^T [+ causal mask]) V
// given dO, for the fp16 Q, K, V the forward takes. Two kernels, no atomics:
//
//   row kernel (one CTA per 128-row query tile): pass 1 recomputes S = Q K^T
//     block by block for the row log-sum-exp (log2 units), D = rowsum(dO * O)
//     comes from the fp32 O; pass 2 recomputes S and dP = dO V^T, forms
//     dS = P * (dP - D) * score_scale and accumulates dQ += dS K. It writes
//     dQ and the per-row statistics (LSE, D) the column kernel reads.
//   column kernel (one CTA per 128-key tile): for every query block that can
//     see the tile, S^T = K Q^T and dP^T = V dO^T, P^T and dS^T from the row
//     statistics, then dV += P^T dO and dK += dS^T Q.
//
// Both kernels follow the forward's tcgen05 conventions: operand tiles loaded
// by TMA 128-byte swizzled, S-like products as SS MMAs (kind::f16, fp32 in
// TMEM, K-major operands), the P/dS products as TS MMAs with the fp16 tile in
// TMEM (two values per 32-bit column) and an MN-major shared-memory B
// operand, exactly like the forward's PV. Warps 0-3 own TMEM lanes 0-127 (one
// thread per row of the CTA's tile) and do the elementwise work, warp 4 issues
// the TMA loads, warp 5 allocates TMEM and issues every MMA from one elected
// lane (so the in-order tensor pipe orders an MMA that overwrites a TMEM tile
// after the MMAs that read it). Every wait is bounded (1 s); a wait that runs
// out records a status bit (read with tilemix_read_and_clear_status), all
// roles stop, drain their own in-flight copies and MMAs, and return.
#include "kernels.cuh"
#include "sm100.cuh"

#include <cuda.h>

#include <cmath>
#include <cstdint>
#include <cstring>
#include <mutex>

namespace tilemix {

__device__ unsigned int g_backward_status = 0;

namespace {

using namespace sm100;

constexpr int kRows = 128;                    // tile rows of either kernel (tcgen05 M)
constexpr int kBwdThreads = 192;              // warps 0-3 elementwise, 4 producer, 5 MMA
constexpr int kProducer = 4;
constexpr int kMma = 5;
constexpr uint32_t kAtom = 128 * 128;         // one 64-column fp16 atom of a 128-row tile
constexpr uint64_t kLimitNs = 1000000000ull;
constexpr uint32_t kSuspend = 200000;
constexpr float kLog2e = 1.4426950408889634f;

enum : unsigned int { kBwdStatusWait = 1u << 4, kBwdStatusDrain = 1u << 5 };

// Bounded wait by all 32 lanes; warp-uniform result. A wait that runs out
// raises the CTA's abort flag and records the status bit.
__device__ __forceinline__ bool bw_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
    bool ok = mbar_try_wait(bar, parity);
    if (!ok) {
        const uint64_t start = global_timer_ns();
        while (true) {
            if (mbar_try_wait_suspend(bar, parity, kSuspend)) { ok = true; break; }
            if (*abort_flag) break;
            if (global_timer_ns() - start > kLimitNs) {
                *abort_flag = 1;
                atomicOr(&g_backward_status, kBwdStatusWait);
                break;
            }
        }
    }
    return __all_sync(0xffffffffu, ok);
}

// Drain wait for this CTA's own asynchronous work (TMA loads, MMAs): it
// completes on its own, so the abort flag is ignored; bounded by time.
__device__ __forceinline__ void bw_drain(uint32_t bar, uint32_t parity) {
    if (!mbar_try_wait(bar, parity)) {
        const uint64_t start = global_timer_ns();
        while (!mbar_try_wait_suspend(bar, parity, kSuspend)) {
            if (global_timer_ns() - start > kLimitNs) {
                atomicOr(&g_backward_status, kBwdStatusDrain);
                break;
            }
        }
    }
    __syncwarp();
}

struct BwdParams {
    const float* o;            // [heads][M][d] fp32 forward output
    float* dq;                 // [heads][M][d]
    float* dk;                 // [heads][N][d]
    float* dv;                 // [heads][N][d]
    float* lse;                // [heads][M] row log-sum-exp of score_scale * log2(e) * S (log2 units)
    float* dsum;               // [heads][M] rowsum(dO * O)
    int heads, M, N, d;
    int q_tiles, k_tiles;
    float c;                   // score_scale * log2(e)
    float scale;               // score_scale
    int causal;
};

// Shared memory of both kernels: one resident 128-row tile pair (A0, A1) and
// two stages of a streamed pair (B0, B1), each tile kAtoms atoms of 16 KB,
// 1024-byte aligned for the 128-byte swizzle; then barriers and small arrays.
template <int kAtoms>
struct BwdSmem {
    static constexpr uint32_t kTile = kAtoms * kAtom;
    static constexpr uint32_t kA0 = 0;                       // row kernel: Q;  column kernel: K
    static constexpr uint32_t kA1 = kA0 + kTile;             // row kernel: dO; column kernel: V
    static constexpr uint32_t kB0 = kA1 + kTile;             // [2] row kernel: K;  column kernel: Q
    static constexpr uint32_t kB1 = kB0 + 2 * kTile;         // [2] row kernel: V;  column kernel: dO
    static constexpr uint32_t kStats = kB1 + 2 * kTile;      // column kernel: [2][2][128] LSE, D
    static constexpr uint32_t kBars = kStats + 2 * 2 * kRows * 4;
    static constexpr uint32_t kNumBars = 16;
    static constexpr uint32_t kMisc = kBars + kNumBars * 8;  // TMEM base, abort flag
    static constexpr uint32_t kBytes = kMisc + 16 + 1024;    // + alignment slack
    static_assert(kBytes <= 232448, "shared memory");
};

// Barriers (same indices in both kernels):
//   0 A-full (resident pair), 1-2 B-full[stage], 3-4 B-empty[stage],
//   5 S-full (S and dP of the current block in TMEM), 6 P-ready (the
//   elementwise warps have written P / dS), 7-8 S-free[buffer] (row kernel,
//   pass 1: S consumed), 9 done (last accumulation MMA complete), 10 drain
//   (the MMA warp's own drain), 11-12 S-full[buffer] of pass 1.
enum : int { kBarA = 0, kBarBFull = 1, kBarBEmpty = 3, kBarS = 5, kBarP = 6, kBarSFree = 7, kBarDone = 9,
             kBarDrain = 10, kBarS1 = 11 };
constexpr int kElemWarps = 4;               // arrivals on P-ready and S-free

// Common prologue: barriers (one per lane of warp 0), abort flag, TMEM (512
// columns: 1 CTA per SM by shared memory). Returns the TMEM base.
template <int kAtoms>
__device__ __forceinline__ uint32_t bwd_setup(uint8_t* smem, uint32_t sbase) {
    using L = BwdSmem<kAtoms>;
    const int warp = threadIdx.x >> 5;
    const uint32_t lane = threadIdx.x & 31u;
    if (warp == 0) {
        if (lane < L::kNumBars) {
            const bool many = lane == kBarP || lane == kBarSFree || lane == kBarSFree + 1;
            mbar_init(sbase + L::kBars + 8u * lane, many ? kElemWarps : 1);
        }
        if (lane == 0) *reinterpret_cast<volatile int*>(smem + L::kMisc + 4) = 0;
        mbar_init_fence();
        fence_proxy_async_smem();
    }
    if (warp == kMma) {
        tmem_alloc(sbase + L::kMisc, 512);
        tmem_relinquish();
        tc_fence_before();
    }
    __syncthreads();
    tc_fence_after();
    return *reinterpret_cast<volatile uint32_t*>(smem + L::kMisc);
}

// D (128 x 128, fp32 in TMEM) = A B^T over d: A and B 128-row K-major tiles.
__device__ __forceinline__ void mma_abt(uint32_t d_tmem, uint32_t a_lo, uint32_t b_lo, uint32_t dhi, uint32_t idesc,
                                        int ksteps) {
    const uint32_t none[4] = {0u, 0u, 0u, 0u};
    mma_f16_ss_w<0>(d_tmem, a_lo, b_lo, dhi, idesc, none);
    for (int ks = 1; ks < ksteps; ++ks) {
        const uint32_t ko = static_cast<uint32_t>((ks >> 2) * (kAtom >> 4) + (ks & 3) * 2);
        mma_f16_ss_w<1>(d_tmem, a_lo + ko, b_lo + ko, dhi, idesc, none);
    }
}

// D (128 x d) (+)= T B: T a 128 x 128 fp16 tile in TMEM (two values per
// column, 16 rows of B per 8 columns), B a 128-row tile read MN-major.
__device__ __forceinline__ void mma_tb(uint32_t d_tmem, uint32_t t_tmem, uint32_t b_lo, uint32_t dhi,
                                       uint32_t idesc, bool accumulate) {
    for (int t = 0; t < kRows / 16; ++t) {
        mma_f16_ts_w(d_tmem, t_tmem + 8u * static_cast<uint32_t>(t), b_lo + 128u * static_cast<uint32_t>(t), dhi,
                     idesc, (accumulate || t > 0) ? 1u : 0u);
    }
}

// Row kernel: one CTA per (head, 128-row query tile); heaviest tiles first.
template <int kAtoms>
__global__ void __launch_bounds__(kBwdThreads, 1)
backward_rows_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_do,
                     const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                     const BwdParams p) {
    using L = BwdSmem<kAtoms>;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t pad = ((raw + 1023u) & ~1023u) - raw;
    uint8_t* smem = smem_raw + pad;
    const uint32_t sbase = raw + pad;
    auto bar = [&](int i) -> uint32_t { return sbase + L::kBars + 8u * static_cast<uint32_t>(i); };
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kMisc + 4);
    const int warp = threadIdx.x >> 5;
    const uint32_t lane = threadIdx.x & 31u;
    const int bid = static_cast<int>(blockIdx.x);
    const int qt = p.q_tiles - 1 - bid / p.heads;
    const int head = bid % p.heads;
    const int nblk = p.causal ? min(p.k_tiles, qt + 1) : p.k_tiles;
    const uint32_t tmem = bwd_setup<kAtoms>(smem, sbase);

    if (warp == kProducer) {
        // Q and dO once; K (pass 1), then K and V (pass 2) through two stages.
        if (elect_one()) {
            mbar_arrive_expect_tx(bar(kBarA), 2 * L::kTile);
            for (int a = 0; a < kAtoms; ++a) {
                tma_load_3d(sbase + L::kA0 + a * kAtom, &tm_q, bar(kBarA), a * 64, qt * kRows, head);
                tma_load_3d(sbase + L::kA1 + a * kAtom, &tm_do, bar(kBarA), a * 64, qt * kRows, head);
            }
        }
        __syncwarp();
        int issued = 0;
        for (int l = 0; l < 2 * nblk; ++l) {
            const int s = l & 1;
            const bool pass2 = l >= nblk;
            const int j = pass2 ? l - nblk : l;
            if (!bw_wait(bar(kBarBEmpty + s), ((l >> 1) & 1) ^ 1, abort_flag)) break;
            if (elect_one()) {
                mbar_arrive_expect_tx(bar(kBarBFull + s), (pass2 ? 2u : 1u) * L::kTile);
                for (int a = 0; a < kAtoms; ++a) {
                    tma_load_3d(sbase + L::kB0 + s * L::kTile + a * kAtom, &tm_k, bar(kBarBFull + s), a * 64,
                                j * kRows, head);
                    if (pass2) {
                        tma_load_3d(sbase + L::kB1 + s * L::kTile + a * kAtom, &tm_v, bar(kBarBFull + s), a * 64,
                                    j * kRows, head);
                    }
                }
            }
            __syncwarp();
            issued = l + 1;
        }
        bw_drain(bar(kBarA), 0);
        for (int l = max(0, issued - 2); l < issued; ++l) bw_drain(bar(kBarBFull + (l & 1)), (l >> 1) & 1);
    } else if (warp == kMma) {
        const uint32_t dhi = smem_desc_sw128_hi(1024);
        const uint32_t idesc_s = idesc_f16_f32(kRows, kRows, false);
        const uint32_t idesc_o = idesc_f16_f32(kRows, p.d, true);
        const int ksteps = p.d / 16;
        const uint32_t q_lo = smem_desc_sw128_lo(sbase + L::kA0, 16);
        const uint32_t do_lo = smem_desc_sw128_lo(sbase + L::kA1, 16);
        bool ok = bw_wait(bar(kBarA), 0, abort_flag);
        // pass 1: S(j) = Q K(j)^T into TMEM buffer j & 1
        for (int j = 0; ok && j < nblk; ++j) {
            const int s = j & 1;
            ok = bw_wait(bar(kBarBFull + s), (j >> 1) & 1, abort_flag);
            if (ok && j >= 2) ok = bw_wait(bar(kBarSFree + (j & 1)), ((j - 2) >> 1) & 1, abort_flag);
            if (!ok) break;
            tc_fence_after();
            if (elect_one()) {
                mma_abt(tmem + 128u * static_cast<uint32_t>(j & 1), q_lo,
                        smem_desc_sw128_lo(sbase + L::kB0 + s * L::kTile, 16), dhi, idesc_s, ksteps);
                tc_commit(bar(kBarS1 + (j & 1)));
                tc_commit(bar(kBarBEmpty + s));
            }
            __syncwarp();
        }
        // pass 2 reuses both buffers: wait until the last pass-1 blocks are read
        for (int b = 0; ok && b < 2; ++b) {
            const int jb = nblk - 1 - b;
            if (jb >= 0) ok = bw_wait(bar(kBarSFree + (jb & 1)), (jb >> 1) & 1, abort_flag);
        }
        // pass 2: S = Q K^T (columns 0-127), dP = dO V^T (128-255); then, once
        // the elementwise warps have written dS over S, dQ += dS K (256-...)
        for (int j = 0; ok && j < nblk; ++j) {
            const int l = nblk + j, s = l & 1;
            ok = bw_wait(bar(kBarBFull + s), (l >> 1) & 1, abort_flag);
            if (!ok) break;
            tc_fence_after();
            if (elect_one()) {
                mma_abt(tmem, q_lo, smem_desc_sw128_lo(sbase + L::kB0 + s * L::kTile, 16), dhi, idesc_s, ksteps);
                mma_abt(tmem + 128u, do_lo, smem_desc_sw128_lo(sbase + L::kB1 + s * L::kTile, 16), dhi, idesc_s,
                        ksteps);
                tc_commit(bar(kBarS));
            }
            __syncwarp();
            ok = bw_wait(bar(kBarP), j & 1, abort_flag);
            if (!ok) break;
            tc_fence_after();
            if (elect_one()) {
                mma_tb(tmem + 256u, tmem, smem_desc_sw128_lo(sbase + L::kB0 + s * L::kTile, kAtom), dhi, idesc_o,
                       j > 0);
                tc_commit(bar(kBarBEmpty + s));
                if (j == nblk - 1) tc_commit(bar(kBarDone));
            }
            __syncwarp();
        }
        if (lane == 0) tc_commit(bar(kBarDrain));
        __syncwarp();
        bw_drain(bar(kBarDrain), 0);
    } else {
        // elementwise: thread = query row = TMEM lane
        const int r = static_cast<int>(threadIdx.x);
        const int row = qt * kRows + r;
        const bool row_ok = row < p.M;
        const uint32_t lb = static_cast<uint32_t>(warp * 32) << 16;
        bool ok = bw_wait(bar(kBarA), 0, abort_flag);
        // D = rowsum(dO * O): dO from the swizzled tile, O (fp32) from global
        float dsum = 0.0f;
        if (ok && row_ok) {
            const float* orow = p.o + (static_cast<std::size_t>(head) * p.M + row) * p.d;
            for (int c8 = 0; c8 < p.d / 8; ++c8) {
                const int atom = c8 >> 3, c = c8 & 7;
                const uint4 h = *reinterpret_cast<const uint4*>(smem + L::kA1 + atom * kAtom + r * 128 +
                                                                ((c ^ (r & 7)) << 4));
                const __half2* hh = reinterpret_cast<const __half2*>(&h);
                const float4 o0 = *reinterpret_cast<const float4*>(orow + 8 * c8);
                const float4 o1 = *reinterpret_cast<const float4*>(orow + 8 * c8 + 4);
                const float2 f0 = __half22float2(hh[0]), f1 = __half22float2(hh[1]);
                const float2 f2 = __half22float2(hh[2]), f3 = __half22float2(hh[3]);
                dsum = fmaf(f0.x, o0.x, dsum); dsum = fmaf(f0.y, o0.y, dsum);
                dsum = fmaf(f1.x, o0.z, dsum); dsum = fmaf(f1.y, o0.w, dsum);
                dsum = fmaf(f2.x, o1.x, dsum); dsum = fmaf(f2.y, o1.y, dsum);
                dsum = fmaf(f3.x, o1.z, dsum); dsum = fmaf(f3.y, o1.w, dsum);
            }
        }
        // pass 1: running max and sum of 2^(c S) over the row's visible keys
        float m = -INFINITY, l = 0.0f;
        for (int j = 0; ok && j < nblk; ++j) {
            ok = bw_wait(bar(kBarS1 + (j & 1)), (j >> 1) & 1, abort_flag);
            if (!ok) break;
            tc_fence_after();
            const uint32_t sb = tmem + lb + 128u * static_cast<uint32_t>(j & 1);
            #pragma unroll 1
            for (int c = 0; c < 4; ++c) {
                uint32_t x[32];
                tmem_ld32(sb + 32u * c, x);
                tc_wait_ld();
                const int key0 = j * kRows + 32 * c;
                float s2[32];
                float cm = -INFINITY;
                #pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const int key = key0 + i;
                    const bool valid = key < p.N && (!p.causal || key <= row);
                    s2[i] = valid ? __uint_as_float(x[i]) * p.c : -INFINITY;
                    cm = fmaxf(cm, s2[i]);
                }
                const float mn = fmaxf(m, cm);
                if (mn > -INFINITY) {
                    float sum = 0.0f;
                    #pragma unroll
                    for (int i = 0; i < 32; ++i) sum += ex2(s2[i] - mn);
                    l = l * ex2(m - mn) + sum;
                    m = mn;
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(kBarSFree + (j & 1)));
        }
        const float lse = m + log2f(l);
        if (ok && row_ok) {
            p.lse[static_cast<std::size_t>(head) * p.M + row] = lse;
            p.dsum[static_cast<std::size_t>(head) * p.M + row] = dsum;
        }
        // pass 2: dS = P (dP - D) * score_scale, fp16, over S's columns
        for (int j = 0; ok && j < nblk; ++j) {
            ok = bw_wait(bar(kBarS), j & 1, abort_flag);
            if (!ok) break;
            tc_fence_after();
            const uint32_t sb = tmem + lb;
            #pragma unroll 1
            for (int c = 0; c < 4; ++c) {
                uint32_t x[32], y[32];
                tmem_ld32(sb + 32u * c, x);
                tmem_ld32(sb + 128u + 32u * c, y);
                tc_wait_ld();
                const int key0 = j * kRows + 32 * c;
                uint32_t ds[16];
                #pragma unroll
                for (int i = 0; i < 16; ++i) {
                    float v[2];
                    #pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        const int key = key0 + 2 * i + e;
                        const bool valid = key < p.N && (!p.causal || key <= row);
                        const float pr = valid ? ex2(__uint_as_float(x[2 * i + e]) * p.c - lse) : 0.0f;
                        v[e] = pr * (__uint_as_float(y[2 * i + e]) - dsum) * p.scale;
                    }
                    ds[i] = pack_half2(v[0], v[1]);
                }
                // columns [16c, 16c + 16) were read by this or the previous chunk
                tmem_st16(sb + 16u * c, ds);
            }
            tc_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(kBarP));
        }
        // dQ out
        if (ok) ok = bw_wait(bar(kBarDone), 0, abort_flag);
        if (ok) {
            tc_fence_after();
            float* out = p.dq + (static_cast<std::size_t>(head) * p.M + row) * p.d;
            #pragma unroll 1
            for (int c = 0; c < p.d; c += 32) {
                uint32_t x[32];
                tmem_ld32(tmem + lb + 256u + static_cast<uint32_t>(c), x);
                tc_wait_ld();
                if (row_ok) {
                    #pragma unroll
                    for (int i = 0; i < 32; i += 4) {
                        if (c + i < p.d) {
                            *reinterpret_cast<float4*>(out + c + i) =
                                make_float4(__uint_as_float(x[i]), __uint_as_float(x[i + 1]),
                                            __uint_as_float(x[i + 2]), __uint_as_float(x[i + 3]));
                        }
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kMma) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// Column kernel: one CTA per (head, 128-key tile); K and V stay resident, the
// query blocks that see the tile stream through (Q, dO) stages. TMEM: S^T in
// columns 0-127 (P^T written over it), dP^T in 128-255 (dS^T over it), dV in
// 256-383, dK in 384-511.
template <int kAtoms>
__global__ void __launch_bounds__(kBwdThreads, 1)
backward_cols_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_do,
                     const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                     const BwdParams p) {
    using L = BwdSmem<kAtoms>;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t pad = ((raw + 1023u) & ~1023u) - raw;
    uint8_t* smem = smem_raw + pad;
    const uint32_t sbase = raw + pad;
    auto bar = [&](int i) -> uint32_t { return sbase + L::kBars + 8u * static_cast<uint32_t>(i); };
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kMisc + 4);
    const int warp = threadIdx.x >> 5;
    const uint32_t lane = threadIdx.x & 31u;
    const int bid = static_cast<int>(blockIdx.x);
    // causal: the key tiles with the most query blocks first
    const int kt = p.causal ? bid / p.heads : p.k_tiles - 1 - bid / p.heads;
    const int head = bid % p.heads;
    const int i0 = p.causal ? kt : 0;             // first query block that sees the tile
    const int nq = p.q_tiles - i0;                // may be <= 0 (causal, keys past the last query)
    const uint32_t tmem = bwd_setup<kAtoms>(smem, sbase);

    if (warp == kProducer) {
        if (nq > 0) {
            if (elect_one()) {
                mbar_arrive_expect_tx(bar(kBarA), 2 * L::kTile);
                for (int a = 0; a < kAtoms; ++a) {
                    tma_load_3d(sbase + L::kA0 + a * kAtom, &tm_k, bar(kBarA), a * 64, kt * kRows, head);
                    tma_load_3d(sbase + L::kA1 + a * kAtom, &tm_v, bar(kBarA), a * 64, kt * kRows, head);
                }
            }
            __syncwarp();
            int issued = 0;
            for (int b = 0; b < nq; ++b) {
                const int s = b & 1, i = i0 + b;
                if (!bw_wait(bar(kBarBEmpty + s), ((b >> 1) & 1) ^ 1, abort_flag)) break;
                if (elect_one()) {
                    mbar_arrive_expect_tx(bar(kBarBFull + s), 2 * L::kTile);
                    for (int a = 0; a < kAtoms; ++a) {
                        tma_load_3d(sbase + L::kB0 + s * L::kTile + a * kAtom, &tm_q, bar(kBarBFull + s), a * 64,
                                    i * kRows, head);
                        tma_load_3d(sbase + L::kB1 + s * L::kTile + a * kAtom, &tm_do, bar(kBarBFull + s),
                                    a * 64, i * kRows, head);
                    }
                }
                __syncwarp();
                issued = b + 1;
            }
            bw_drain(bar(kBarA), 0);
            for (int b = max(0, issued - 2); b < issued; ++b) bw_drain(bar(kBarBFull + (b & 1)), (b >> 1) & 1);
        }
    } else if (warp == kMma) {
        if (nq > 0) {
            const uint32_t dhi = smem_desc_sw128_hi(1024);
            const uint32_t idesc_s = idesc_f16_f32(kRows, kRows, false);
            const uint32_t idesc_o = idesc_f16_f32(kRows, p.d, true);
            const int ksteps = p.d / 16;
            const uint32_t k_lo = smem_desc_sw128_lo(sbase + L::kA0, 16);
            const uint32_t v_lo = smem_desc_sw128_lo(sbase + L::kA1, 16);
            bool ok = bw_wait(bar(kBarA), 0, abort_flag);
            for (int b = 0; ok && b < nq; ++b) {
                const int s = b & 1;
                ok = bw_wait(bar(kBarBFull + s), (b >> 1) & 1, abort_flag);
                if (!ok) break;
                tc_fence_after();
                if (elect_one()) {
                    // S^T = K Q^T, dP^T = V dO^T (over d)
                    mma_abt(tmem, k_lo, smem_desc_sw128_lo(sbase + L::kB0 + s * L::kTile, 16), dhi, idesc_s, ksteps);
                    mma_abt(tmem + 128u, v_lo, smem_desc_sw128_lo(sbase + L::kB1 + s * L::kTile, 16), dhi, idesc_s,
                            ksteps);
                    tc_commit(bar(kBarS));
                }
                __syncwarp();
                ok = bw_wait(bar(kBarP), b & 1, abort_flag);
                if (!ok) break;
                tc_fence_after();
                if (elect_one()) {
                    // dV += P^T dO, dK += dS^T Q (over the block's queries)
                    mma_tb(tmem + 256u, tmem, smem_desc_sw128_lo(sbase + L::kB1 + s * L::kTile, kAtom), dhi, idesc_o,
                           b > 0);
                    mma_tb(tmem + 384u, tmem + 128u, smem_desc_sw128_lo(sbase + L::kB0 + s * L::kTile, kAtom), dhi,
                           idesc_o, b > 0);
                    tc_commit(bar(kBarBEmpty + s));
                    if (b == nq - 1) tc_commit(bar(kBarDone));
                }
                __syncwarp();
            }
            if (lane == 0) tc_commit(bar(kBarDrain));
            __syncwarp();
            bw_drain(bar(kBarDrain), 0);
        }
    } else {
        // elementwise: thread = key row = TMEM lane
        const int r = static_cast<int>(threadIdx.x);
        const int key = kt * kRows + r;
        const uint32_t lb = static_cast<uint32_t>(warp * 32) << 16;
        float* stats = reinterpret_cast<float*>(smem + L::kStats);
        bool ok = true;
        // Every elementwise warp runs all nq iterations (the named barrier
        // needs all four); after an abort they only pass the barrier.
        for (int b = 0; b < nq; ++b) {
            const int i = i0 + b;
            // the block's row statistics, staged once for all 128 threads
            float* lse_s = stats + (b & 1) * 2 * kRows;
            float* d_s = lse_s + kRows;
            const int q = i * kRows + r;
            lse_s[r] = q < p.M ? p.lse[static_cast<std::size_t>(head) * p.M + q] : 0.0f;
            d_s[r] = q < p.M ? p.dsum[static_cast<std::size_t>(head) * p.M + q] : 0.0f;
            asm volatile("bar.sync 1, 128;" ::: "memory");
            if (ok) ok = bw_wait(bar(kBarS), b & 1, abort_flag);
            if (!ok) continue;
            tc_fence_after();
            const uint32_t sb = tmem + lb;
            #pragma unroll 1
            for (int c = 0; c < 4; ++c) {
                uint32_t x[32], y[32];
                tmem_ld32(sb + 32u * c, x);
                tmem_ld32(sb + 128u + 32u * c, y);
                tc_wait_ld();
                const int q0 = i * kRows + 32 * c;
                uint32_t pt[16], dst[16];
                #pragma unroll
                for (int e = 0; e < 16; ++e) {
                    float pv[2], dv[2];
                    #pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const int col = 32 * c + 2 * e + h;
                        const int qq = q0 + 2 * e + h;
                        const bool valid = qq < p.M && (!p.causal || key <= qq);
                        const float pr = valid ? ex2(__uint_as_float(x[2 * e + h]) * p.c - lse_s[col]) : 0.0f;
                        pv[h] = pr;
                        dv[h] = pr * (__uint_as_float(y[2 * e + h]) - d_s[col]) * p.scale;
                    }
                    pt[e] = pack_half2(pv[0], pv[1]);
                    dst[e] = pack_half2(dv[0], dv[1]);
                }
                tmem_st16(sb + 16u * c, pt);
                tmem_st16(sb + 128u + 16u * c, dst);
            }
            tc_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(kBarP));
        }
        if (ok && key < p.N) {
            float* dv_out = p.dv + (static_cast<std::size_t>(head) * p.N + key) * p.d;
            float* dk_out = p.dk + (static_cast<std::size_t>(head) * p.N + key) * p.d;
            if (nq <= 0) {
                for (int c = 0; c < p.d; c += 4) {
                    *reinterpret_cast<float4*>(dv_out + c) = make_float4(0.f, 0.f, 0.f, 0.f);
                    *reinterpret_cast<float4*>(dk_out + c) = make_float4(0.f, 0.f, 0.f, 0.f);
                }
            }
        }
        if (ok && nq > 0) ok = bw_wait(bar(kBarDone), 0, abort_flag);
        if (ok && nq > 0) {
            tc_fence_after();
            #pragma unroll 1
            for (int part = 0; part < 2; ++part) {
                float* out = (part == 0 ? p.dv : p.dk) + (static_cast<std::size_t>(head) * p.N + key) * p.d;
                #pragma unroll 1
                for (int c = 0; c < p.d; c += 32) {
                    uint32_t x[32];
                    tmem_ld32(tmem + lb + 256u + 128u * part + static_cast<uint32_t>(c), x);
                    tc_wait_ld();
                    if (key < p.N) {
                        #pragma unroll
                        for (int e = 0; e < 32; e += 4) {
                            if (c + e < p.d) {
                                *reinterpret_cast<float4*>(out + c + e) =
                                    make_float4(__uint_as_float(x[e]), __uint_as_float(x[e + 1]),
                                                __uint_as_float(x[e + 2]), __uint_as_float(x[e + 3]));
                            }
                        }
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kMma) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// ------------------------------------------------------------------- host side
using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// fp16 [heads][rows][d] with a {64, 128, 1} box, 128-byte swizzle, zero fill
// past the ends (ragged last tiles, d not a multiple of 64).
bool encode_tile_map(CUtensorMap* map, const __half* base, int heads, int rows, int d) {
    static EncodeFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult status;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &status) == cudaSuccess &&
            status == cudaDriverEntryPointSuccess) {
            fn = reinterpret_cast<EncodeFn>(ptr);
        }
    });
    if (!fn) return false;
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(d), static_cast<cuuint64_t>(rows),
                                static_cast<cuuint64_t>(heads)};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(d) * 2, static_cast<cuuint64_t>(rows) * d * 2};
    const cuuint32_t box[3] = {64u, static_cast<cuuint32_t>(kRows), 1u};
    const cuuint32_t elem_strides[3] = {1u, 1u, 1u};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<__half*>(base), dims, strides, box, elem_strides,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int kAtoms>
cudaError_t launch_backward_atoms(const CUtensorMap* maps, const BwdParams& p, cudaStream_t stream) {
    auto rows = backward_rows_kernel<kAtoms>;
    auto cols = backward_cols_kernel<kAtoms>;
    // at least half the SM's shared memory: one CTA per SM, since each CTA
    // takes all 512 TMEM columns (a second one would only wait in its alloc)
    const int smem = static_cast<int>(BwdSmem<kAtoms>::kBytes > 120u * 1024u ? BwdSmem<kAtoms>::kBytes
                                                                             : 120u * 1024u);
    static int configured[64] = {0};
    int device = 0;
    cudaError_t status = cudaGetDevice(&device);
    if (status != cudaSuccess) return status;
    if (device < 0 || device >= 64) return cudaErrorInvalidDevice;
    if (!configured[device]) {
        status = cudaFuncSetAttribute(rows, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (status == cudaSuccess) status = cudaFuncSetAttribute(cols, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (status != cudaSuccess) return status;
        configured[device] = 1;
    }
    const long long row_grid = static_cast<long long>(p.q_tiles) * p.heads;
    const long long col_grid = static_cast<long long>(p.k_tiles) * p.heads;
    if (row_grid > 0x7fffffffLL || col_grid > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
    rows<<<static_cast<unsigned>(row_grid), kBwdThreads, smem, stream>>>(maps[0], maps[1], maps[2], maps[3], p);
    status = cudaGetLastError();
    if (status != cudaSuccess) return status;
    cols<<<static_cast<unsigned>(col_grid), kBwdThreads, smem, stream>>>(maps[0], maps[1], maps[2], maps[3], p);
    return cudaGetLastError();
}

bool aligned16(const void* ptr) { return (reinterpret_cast<std::uintptr_t>(ptr) & 15u) == 0; }

}  // namespace

cudaError_t launch_attention_backward(const AttentionBackwardProblem& prob, cudaStream_t stream) {
    if (prob.d % 16 != 0 || prob.d > kBackwardMaxHeadDim) return cudaErrorNotSupported;
    if (!aligned16(prob.q) || !aligned16(prob.k) || !aligned16(prob.v) || !aligned16(prob.dout) ||
        !aligned16(prob.o) || !aligned16(prob.dq) || !aligned16(prob.dk) || !aligned16(prob.dv)) {
        return cudaErrorMisalignedAddress;
    }
    BwdParams p{};
    p.o = prob.o;
    p.dq = prob.dq;
    p.dk = prob.dk;
    p.dv = prob.dv;
    p.lse = prob.lse;
    p.dsum = prob.dsum;
    p.heads = prob.heads;
    p.M = prob.M;
    p.N = prob.N;
    p.d = prob.d;
    p.q_tiles = (prob.M - 1) / kRows + 1;
    p.k_tiles = (prob.N - 1) / kRows + 1;
    p.scale = prob.score_scale;
    p.c = prob.score_scale * kLog2e;
    p.causal = prob.causal ? 1 : 0;
    CUtensorMap maps[4];
    std::memset(maps, 0, sizeof(maps));
    if (!encode_tile_map(&maps[0], prob.q, p.heads, p.M, p.d) || !encode_tile_map(&maps[1], prob.dout, p.heads, p.M, p.d) ||
        !encode_tile_map(&maps[2], prob.k, p.heads, p.N, p.d) || !encode_tile_map(&maps[3], prob.v, p.heads, p.N, p.d)) {
        return cudaErrorInvalidValue;
    }
    return p.d <= 64 ? launch_backward_atoms<1>(maps, p, stream) : launch_backward_atoms<2>(maps, p, stream);
}

cudaError_t read_and_clear_backward_status(unsigned int* status) {
    unsigned int zero = 0;
    cudaError_t err = cudaMemcpyFromSymbol(status, g_backward_status, sizeof(unsigned int));
    if (err != cudaSuccess) return err;
    return cudaMemcpyToSymbol(g_backward_status, &zero, sizeof(unsigned int));
}

}  // namespace tilemix
