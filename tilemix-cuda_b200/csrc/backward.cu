// Backward pass of the unrouted (every tile FP16) TileMix attention on sm_100a
// tensor cores. The reference has no backward; this is the gradient of
//   O = softmax(score_scale * Q K^T [+ causal mask]) V
// given dO, for the fp16 Q, K, V the forward takes. Two kernels, no atomics:
//
//   row kernel (one CTA per 128-row query tile): unless the forward's row
//     log-sum-exp is given, pass 1 recomputes S = Q K^T for it (log2 units);
//     D = rowsum(dO * O) comes from the fp32 O; pass 2 recomputes S and
//     dP = dO V^T, forms dS = P * (dP - D) * score_scale and accumulates
//     dQ += dS K. It writes dQ and the per-row statistics (LSE, D) the column
//     kernel reads.
//   column kernel (one CTA per 128-key tile): for every query block that can
//     see the tile, S^T = K Q^T and dP^T = V dO^T, P^T and dS^T from the row
//     statistics, then dV += P^T dO and dK += dS^T Q.
//
// Both kernels work in sub-blocks of 64 columns (keys for the row kernel,
// queries for the column kernel) so that the products of more than one
// sub-block fit in TMEM next to the accumulators: while the elementwise warps
// turn sub-block u into P / dS, the tensor core already computes the S and dP
// of sub-block u + 1 (each TMEM slot is released as soon as its last reader is
// done), and the accumulation products of u follow. The row kernel keeps Q and
// dO in TMEM, so its S and dP products read only K / V from shared memory.
//
// Conventions follow the forward: operand tiles loaded by TMA 128-byte
// swizzled; S-like products as SS MMAs (kind::f16, fp32 in TMEM, K-major
// operands); the P / dS products as TS MMAs with the fp16 tile in TMEM (two
// values per 32-bit column; the 16 values of a K step in 8 consecutive
// columns) and an MN-major shared-memory B operand, exactly like the forward's
// PV. Warps 0-15 do the elementwise work (warp w owns TMEM lanes 32 (w % 4)
// .., one thread per row of the CTA's tile, and the 16-column quarter w / 4
// of every sub-block: four warps per scheduler hide the latency of the TMEM
// loads and the exponentials), warp 16 issues the TMA loads, warp 17
// allocates TMEM and issues the S / dP products, warp 18 the accumulation
// products, each from one
// elected lane. Two issuing warps keep either kind of product from queueing
// behind the other: an accumulation can start as soon as its P / dS is
// written, and the S / dP products that overwrite a TMEM buffer wait (on a
// barrier committed by warp 18) until the accumulation that read it has
// completed. Every wait is
// bounded (1 s); a wait that runs out records a status bit (read with
// tilemix_read_and_clear_status), all roles stop, drain their own in-flight
// copies and MMAs, and return.
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
constexpr int kSub = 64;                      // sub-block columns
constexpr int kSplit = 4;                     // elementwise warps per TMEM lane quadrant
constexpr int kColsPer = kSub / kSplit;       // sub-block columns of one elementwise warp
static_assert(kColsPer == 16, "one elementwise warp produces exactly one K step of the P / dS operands");
constexpr int kElemWarps = 4 * kSplit;
constexpr int kProducer = kElemWarps;
constexpr int kMma = kElemWarps + 1;          // S / dP products; allocates TMEM
constexpr int kMmaAcc = kElemWarps + 2;       // the accumulation products (dQ; dV, dK)
constexpr int kBwdThreads = 32 * (kElemWarps + 3);
constexpr uint32_t kAtom = 128 * 128;         // one 64-column fp16 atom of a 128-row tile
constexpr uint32_t kHalfRows16 = kSub * 128 / 16;   // 64 tile rows, in 16-byte descriptor units
constexpr uint64_t kLimitNs = 1000000000ull;
constexpr uint32_t kSuspend = 200000;
constexpr float kLog2e = 1.4426950408889634f;

enum : unsigned int { kBwdStatusWait = 1u << 4, kBwdStatusDrain = 1u << 5 };

// Bounded wait by all 32 lanes; warp-uniform result. A wait that runs out
// raises the CTA's abort flag and records the status bit.
__device__ __forceinline__ bool bw_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                        uint64_t limit_ns = kLimitNs) {
    bool ok = mbar_try_wait(bar, parity);
    if (!ok) {
        const uint64_t start = global_timer_ns();
        while (true) {
            if (mbar_try_wait_suspend(bar, parity, kSuspend)) { ok = true; break; }
            if (*abort_flag) break;
            if (global_timer_ns() - start > limit_ns) {
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

// Named barrier of the elementwise warps.
__device__ __forceinline__ void elem_sync() { asm volatile("bar.sync 1, %0;" :: "n"(32 * kElemWarps) : "memory"); }

constexpr int kHeadGroup = 8;   // heads scheduled together: their streamed operands stay in L2

// Work item of CTA `bid` over tiles x heads: heads in groups of kHeadGroup;
// inside a group, tile index `order` (0 first) runs for every head of the
// group before order + 1.
__device__ __forceinline__ void work_item(int bid, int heads, int tiles, int& head, int& order) {
    const int per_group = kHeadGroup * tiles;
    const int group0 = (bid / per_group) * kHeadGroup;
    const int group_heads = min(kHeadGroup, heads - group0);
    const int in_group = bid - (bid / per_group) * per_group;
    order = in_group / group_heads;
    head = group0 + in_group % group_heads;
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
    uint64_t limit_ns;         // limit of one pipeline wait (1 s; shorter only in the watchdog self-test)
};

// Shared memory of both kernels: one resident 128-row tile pair (A0, A1) and
// two stages of a streamed pair (B0, B1), each tile kAtoms atoms of 16 KB,
// 1024-byte aligned for the 128-byte swizzle; then row statistics, barriers
// and the TMEM base / abort flag. The row kernel turns A0 / A1 into a third
// K / V stage once Q and dO are in TMEM.
template <int kAtoms>
struct BwdSmem {
    static constexpr uint32_t kTile = kAtoms * kAtom;
    static constexpr uint32_t kA0 = 0;                       // row kernel: Q;  column kernel: K
    static constexpr uint32_t kA1 = kA0 + kTile;             // row kernel: dO; column kernel: V
    static constexpr uint32_t kB0 = kA1 + kTile;             // [2] row kernel: K;  column kernel: Q
    static constexpr uint32_t kB1 = kB0 + 2 * kTile;         // [2] row kernel: V;  column kernel: dO
    static constexpr uint32_t kStats = kB1 + 2 * kTile;      // 2048 floats
    static constexpr uint32_t kBars = kStats + 2048 * 4;
    static constexpr uint32_t kNumBars = 32;
    static constexpr uint32_t kMisc = kBars + kNumBars * 8;  // TMEM base, abort flag
    static constexpr uint32_t kBytes = kMisc + 16 + 1024;    // + alignment slack
    static_assert(kBytes <= 232448, "shared memory");
};

// Barriers (same indices in both kernels):
//   A-full (resident pair); B-full / B-empty [stage]; S-full [slot] (S and dP
//   of a sub-block in TMEM); P-ready [slot] (the elementwise warps have
//   written P / dS); acc-done [slot] (the accumulation products that read it
//   have completed); done (last accumulation complete); drain [issuing warp];
//   dP-free (the elementwise warps have loaded the S / dP slot that the next
//   sub-block's products overwrite); row kernel pass 1: S1-full / S1-free
//   [ring slot], stats (LSE and D of every row known); operands (the row
//   kernel's Q and dO copied into TMEM); A-free (the row kernel's Q / dO
//   shared-memory tiles no longer read: the region becomes a third K / V
//   stage).
enum : int { kBarA = 0, kBarBFull = 1, kBarBEmpty = 4, kBarS = 7, kBarP = 10, kBarAcc = 13, kBarDone = 16,
             kBarDrain = 17, kBarDpFree = 19, kBarS1 = 20, kBarS1Free = 24, kBarStats = 28, kBarOps = 29,
             kBarAFree = 30 };
constexpr int kRing = 4;                      // pass-1 S slots (64 columns each)

// Common prologue: barriers (one per lane of warp 0), abort flag, TMEM (512
// columns: 1 CTA per SM by shared memory). Returns the TMEM base.
template <int kAtoms>
__device__ __forceinline__ uint32_t bwd_setup(uint8_t* smem, uint32_t sbase) {
    using L = BwdSmem<kAtoms>;
    const int warp = threadIdx.x >> 5;
    const uint32_t lane = threadIdx.x & 31u;
    if (warp == 0) {
        if (lane < L::kNumBars) {
            const int i = static_cast<int>(lane);
            const bool many = (i >= kBarP && i < kBarP + 3) || (i >= kBarS1Free && i < kBarS1Free + kRing) ||
                              i == kBarStats || i == kBarOps || i == kBarAFree || i == kBarDpFree;
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

// D (128 x 64, fp32 in TMEM) = A B^T over d: A a 128-row K-major tile, B 64
// rows of one (b_lo already offset to the half). One thread issues every MMA
// back to back, so each instruction on that path adds to the issue time: with
// kSteps > 0 (d = 16 kSteps known at compile time) the loop is unrolled and the
// descriptor offsets are constants; kSteps = 0 takes d / 16 at run time.
template <int kSteps>
__device__ __forceinline__ void mma_sub(uint32_t d_tmem, uint32_t a_lo, uint32_t b_lo, uint32_t dhi, int ksteps) {
    const uint32_t none[4] = {0u, 0u, 0u, 0u};
    constexpr uint32_t idesc = idesc_f16_f32(kRows, kSub, false);
    if constexpr (kSteps > 0) {
        mma_f16_ss_w<0>(d_tmem, a_lo, b_lo, dhi, idesc, none);
        #pragma unroll
        for (int ks = 1; ks < kSteps; ++ks) {
            const uint32_t ko = static_cast<uint32_t>((ks >> 2) * (kAtom >> 4) + (ks & 3) * 2);
            mma_f16_ss_w<1>(d_tmem, a_lo + ko, b_lo + ko, dhi, idesc, none);
        }
    } else {
        mma_f16_ss_w<0>(d_tmem, a_lo, b_lo, dhi, idesc, none);
        for (int ks = 1; ks < ksteps; ++ks) {
            const uint32_t ko = static_cast<uint32_t>((ks >> 2) * (kAtom >> 4) + (ks & 3) * 2);
            mma_f16_ss_w<1>(d_tmem, a_lo + ko, b_lo + ko, dhi, idesc, none);
        }
    }
}

// D (128 x 64) = A B^T over d with A in TMEM (128 lanes, two fp16 per
// column: the 16 values of K step ks in columns 8 ks ..) and B 64 rows of a
// K-major shared-memory tile: only B is read from shared memory.
template <int kSteps>
__device__ __forceinline__ void mma_sub_ts(uint32_t d_tmem, uint32_t a_tmem, uint32_t b_lo, uint32_t dhi,
                                           int ksteps) {
    constexpr uint32_t idesc = idesc_f16_f32(kRows, kSub, false);
    if constexpr (kSteps > 0) {
        #pragma unroll
        for (int ks = 0; ks < kSteps; ++ks) {
            const uint32_t ko = static_cast<uint32_t>((ks >> 2) * (kAtom >> 4) + (ks & 3) * 2);
            mma_f16_ts_w(d_tmem, a_tmem + 8u * ks, b_lo + ko, dhi, idesc, ks > 0 ? 1u : 0u);
        }
    } else {
        for (int ks = 0; ks < ksteps; ++ks) {
            const uint32_t ko = static_cast<uint32_t>((ks >> 2) * (kAtom >> 4) + (ks & 3) * 2);
            mma_f16_ts_w(d_tmem, a_tmem + 8u * static_cast<uint32_t>(ks), b_lo + ko, dhi, idesc, ks > 0 ? 1u : 0u);
        }
    }
}

// Row r of atom `a` (64 columns) of a 128-row, 128-byte-swizzled fp16 tile
// into this thread's TMEM lane at columns [col, col + 32): column c holds
// elements 2c (low half) and 2c + 1, the layout of a TMEM A operand.
__device__ __forceinline__ void atom_row_to_tmem(const uint8_t* tile, int a, int r, uint32_t taddr) {
    uint32_t v[32];
    #pragma unroll
    for (int c = 0; c < 8; ++c) {
        const uint4 h = *reinterpret_cast<const uint4*>(tile + a * kAtom + r * 128 + ((c ^ (r & 7)) << 4));
        v[4 * c] = h.x;
        v[4 * c + 1] = h.y;
        v[4 * c + 2] = h.z;
        v[4 * c + 3] = h.w;
    }
    tmem_st32(taddr, v);
}

// D (128 x d) (+)= T B over a 64-column sub-block: T fp16 in TMEM, the 16
// values of K step t (the columns one elementwise warp produced) in 8 columns
// starting at t_tmem + kStepStride t (16: written over the S columns that warp
// read, row kernel; 8: packed, column kernel); B 64 rows of a tile read
// MN-major (b_lo offset to the half).
template <uint32_t kStepStride>
__device__ __forceinline__ void mma_acc(uint32_t d_tmem, uint32_t t_tmem, uint32_t b_lo, uint32_t dhi,
                                        uint32_t idesc, bool accumulate) {
    #pragma unroll
    for (int t = 0; t < kSub / 16; ++t) {
        mma_f16_ts_w(d_tmem, t_tmem + kStepStride * static_cast<uint32_t>(t), b_lo + 128u * static_cast<uint32_t>(t),
                     dhi, idesc, (accumulate || t > 0) ? 1u : 0u);
    }
}

// Row kernel: one CTA per (head, 128-row query tile); heaviest causal tiles
// first. TMEM: pass 1 S slots at 64 s (s < 4); pass 2 S slots at 0, 64, 128
// (sub-block v in slot v % 3, dS written over it), one dP slot at 192 (free
// again as soon as the elementwise warps have loaded it); dQ at 256; Q at 384
// and dO at 448 (fp16 pairs): the S and dP products take their A operand from
// TMEM, so shared memory only streams the K / V halves.
constexpr uint32_t kColDq = 256, kColQ = 384, kColDo = 448, kColDp = 192;
constexpr int kSSlots = 3;
template <int kAtoms, bool kHaveLse, int kSteps>
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
    int head = 0, order = 0;
    work_item(bid, p.heads, p.q_tiles, head, order);
    const int qt = p.q_tiles - 1 - order;
    const int nblk = p.causal ? min(p.k_tiles, qt + 1) : p.k_tiles;
    const int nsub = 2 * nblk;                    // 64-key sub-blocks
    const int npass1 = kHaveLse ? 0 : nblk;       // K blocks loaded for pass 1
    const uint32_t tmem = bwd_setup<kAtoms>(smem, sbase);

    // K / V stage s: the two B stages, and the A region (Q / dO) as the third
    // once the elementwise warps have copied those into TMEM and read dO
    auto k_at = [&](int st) -> uint32_t { return st < 2 ? L::kB0 + st * L::kTile : L::kA0; };
    auto v_at = [&](int st) -> uint32_t { return st < 2 ? L::kB1 + st * L::kTile : L::kA1; };
    constexpr int kStages = 3;

    if (warp == kProducer) {
        // Q and dO once; K (pass 1, unless the forward's LSE is given), then
        // K and V (pass 2) through the three stages.
        if (elect_one()) {
            mbar_arrive_expect_tx(bar(kBarA), 2 * L::kTile);
            for (int a = 0; a < kAtoms; ++a) {
                tma_load_3d(sbase + L::kA0 + a * kAtom, &tm_q, bar(kBarA), a * 64, qt * kRows, head);
                tma_load_3d(sbase + L::kA1 + a * kAtom, &tm_do, bar(kBarA), a * 64, qt * kRows, head);
            }
        }
        __syncwarp();
        int issued = 0;
        for (int l = 0; l < npass1 + nblk; ++l) {
            const int st = l % kStages, n = l / kStages;
            const bool pass2 = l >= npass1;
            const int j = pass2 ? l - npass1 : l;
            bool free_ok = true;
            if (n > 0) {
                free_ok = bw_wait(bar(kBarBEmpty + st), (n - 1) & 1, abort_flag, p.limit_ns);
            } else if (st == 2) {
                free_ok = bw_wait(bar(kBarAFree), 0, abort_flag, p.limit_ns);
            }
            if (!free_ok) break;
            if (elect_one()) {
                // L2 prefetch of the block kStages loads ahead
                const int la = l + kStages;
                if (la < npass1 + nblk) {
                    const bool p2 = la >= npass1;
                    const int ja = p2 ? la - npass1 : la;
                    for (int a = 0; a < kAtoms; ++a) {
                        tma_prefetch_l2_3d(&tm_k, a * 64, ja * kRows, head);
                        if (p2) tma_prefetch_l2_3d(&tm_v, a * 64, ja * kRows, head);
                    }
                }
                mbar_arrive_expect_tx(bar(kBarBFull + st), (pass2 ? 2u : 1u) * L::kTile);
                for (int a = 0; a < kAtoms; ++a) {
                    tma_load_3d(sbase + k_at(st) + a * kAtom, &tm_k, bar(kBarBFull + st), a * 64, j * kRows, head);
                    if (pass2) {
                        tma_load_3d(sbase + v_at(st) + a * kAtom, &tm_v, bar(kBarBFull + st), a * 64, j * kRows,
                                    head);
                    }
                }
            }
            __syncwarp();
            issued = l + 1;
        }
        bw_drain(bar(kBarA), 0);
        for (int l = max(0, issued - kStages); l < issued; ++l) {
            bw_drain(bar(kBarBFull + l % kStages), (l / kStages) & 1);
        }
    } else if (warp == kMma) {
        // S and dP products (and pass 1's S)
        const uint32_t dhi = smem_desc_sw128_hi(1024);
        const int ksteps = p.d / 16;
        // Q and dO are in TMEM once the elementwise warps have copied them
        bool ok = bw_wait(bar(kBarOps), 0, abort_flag, p.limit_ns);
        // pass 1: S of sub-block v (keys 64 v ..) into ring slot v % kRing
        for (int v = 0; ok && v < 2 * npass1; ++v) {
            const int j = v >> 1, h = v & 1, st = j % kStages;
            if (h == 0) ok = bw_wait(bar(kBarBFull + st), (j / kStages) & 1, abort_flag, p.limit_ns);
            if (ok && v >= kRing) ok = bw_wait(bar(kBarS1Free + v % kRing), ((v - kRing) / kRing) & 1, abort_flag, p.limit_ns);
            if (!ok) break;
            tc_fence_after();
            if (elect_one()) {
                mma_sub_ts<kSteps>(tmem + 64u * static_cast<uint32_t>(v % kRing), tmem + kColQ,
                                   smem_desc_sw128_lo(sbase + k_at(st), 16) + kHalfRows16 * h, dhi, ksteps);
                tc_commit(bar(kBarS1 + v % kRing));
                if (h == 1) tc_commit(bar(kBarBEmpty + st));
            }
            __syncwarp();
        }
        // pass 2 starts once every row's LSE is known (the pass-1 slots have
        // then been read). S(v) and dP(v) go into buffer v & 1 once the dQ
        // product that read sub-block v - 2 from it has completed.
        if (!kHaveLse && ok) ok = bw_wait(bar(kBarStats), 0, abort_flag, p.limit_ns);
        for (int v = 0; ok && v < nsub; ++v) {
            const int l = npass1 + (v >> 1), st = l % kStages, h = v & 1, slot = v % kSSlots;
            if (h == 0) ok = bw_wait(bar(kBarBFull + st), (l / kStages) & 1, abort_flag, p.limit_ns);
            // S(v) once dQ(v - 3) has read the slot
            if (ok && v >= kSSlots) ok = bw_wait(bar(kBarAcc + slot), ((v - kSSlots) / kSSlots) & 1, abort_flag, p.limit_ns);
            if (!ok) break;
            tc_fence_after();
            if (elect_one()) {
                mma_sub_ts<kSteps>(tmem + kSub * static_cast<uint32_t>(slot), tmem + kColQ,
                                   smem_desc_sw128_lo(sbase + k_at(st), 16) + kHalfRows16 * h, dhi, ksteps);
            }
            __syncwarp();
            // dP(v) once the elementwise warps have loaded dP(v - 1)
            if (v >= 1) ok = bw_wait(bar(kBarDpFree), (v - 1) & 1, abort_flag, p.limit_ns);
            if (!ok) break;
            tc_fence_after();
            if (elect_one()) {
                mma_sub_ts<kSteps>(tmem + kColDp, tmem + kColDo,
                                   smem_desc_sw128_lo(sbase + v_at(st), 16) + kHalfRows16 * h, dhi, ksteps);
                tc_commit(bar(kBarS + slot));
            }
            __syncwarp();
        }
        if (lane == 0) tc_commit(bar(kBarDrain));
        __syncwarp();
        bw_drain(bar(kBarDrain), 0);
    } else if (warp == kMmaAcc) {
        // dQ += dS(v) K as soon as the elementwise warps have written dS(v)
        const uint32_t dhi = smem_desc_sw128_hi(1024);
        const uint32_t idesc_o = idesc_f16_f32(kRows, p.d, true);
        bool ok = true;
        for (int v = 0; ok && v < nsub; ++v) {
            const int l = npass1 + (v >> 1), st = l % kStages, h = v & 1, slot = v % kSSlots;
            ok = bw_wait(bar(kBarP + slot), (v / kSSlots) & 1, abort_flag, p.limit_ns);
            if (!ok) break;
            tc_fence_after();
            if (elect_one()) {
                mma_acc<16>(tmem + kColDq, tmem + kSub * static_cast<uint32_t>(slot),
                            smem_desc_sw128_lo(sbase + k_at(st), kAtom) + kHalfRows16 * h, dhi, idesc_o, v > 0);
                tc_commit(bar(kBarAcc + slot));
                if (h == 1) tc_commit(bar(kBarBEmpty + st));
                if (v == nsub - 1) tc_commit(bar(kBarDone));
            }
            __syncwarp();
        }
        if (lane == 0) tc_commit(bar(kBarDrain + 1));
        __syncwarp();
        bw_drain(bar(kBarDrain + 1), 0);
    } else {
        // elementwise: thread = (query row = TMEM lane, column quarter ch)
        const int quad = warp & 3, ch = warp >> 2;
        const int r = quad * 32 + static_cast<int>(lane);
        const int row = qt * kRows + r;
        const bool row_ok = row < p.M;
        const uint32_t lb = static_cast<uint32_t>(quad * 32) << 16;
        float* stats = reinterpret_cast<float*>(smem + L::kStats);   // [ch][max, sum, D][128]
        bool ok = bw_wait(bar(kBarA), 0, abort_flag, p.limit_ns);
        // the MMA operands: warp quarter ch copies this row's atom ch % kAtoms
        // of Q (ch < kAtoms) or of dO (kAtoms <= ch < 2 kAtoms) into TMEM
        if (ok && ch < 2 * kAtoms) {
            const int which = ch / kAtoms, atom = ch % kAtoms;
            atom_row_to_tmem(smem + (which == 0 ? L::kA0 : L::kA1), atom, r,
                             tmem + lb + (which == 0 ? kColQ : kColDo) + 32u * atom);
            tc_wait_st();
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(kBarOps));
        // D = rowsum(dO * O) over this quarter's 8-column chunks: dO from the
        // swizzled tile, O (fp32) from global
        float dsum = 0.0f;
        if (ok && row_ok) {
            const float* orow = p.o + (static_cast<std::size_t>(head) * p.M + row) * p.d;
            for (int c8 = ch; c8 < p.d / 8; c8 += kSplit) {
                const int atom = c8 >> 3, c = c8 & 7;
                const uint4 hv = *reinterpret_cast<const uint4*>(smem + L::kA1 + atom * kAtom + r * 128 +
                                                                 ((c ^ (r & 7)) << 4));
                const __half2* hh = reinterpret_cast<const __half2*>(&hv);
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
        // the Q / dO tiles in shared memory are no longer read: the producer
        // may load K / V there
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(kBarAFree));
        // A sub-block needs no mask when all its keys exist and (causal) lie
        // at or before the tile's first row.
        auto full_sub = [&](int v) {
            const int key_end = (v + 1) * kSub;
            return key_end <= p.N && (!p.causal || key_end - 1 <= qt * kRows);
        };
        float lse = 0.0f;
        if constexpr (!kHaveLse) {
            // pass 1: running max and sum of 2^(c S) over this quarter's
            // visible keys
            float m = -INFINITY, l = 0.0f;
            for (int v = 0; ok && v < nsub; ++v) {
                ok = bw_wait(bar(kBarS1 + v % kRing), (v / kRing) & 1, abort_flag, p.limit_ns);
                if (!ok) break;
                tc_fence_after();
                uint32_t x[kColsPer];
                tmem_ld16(tmem + lb + 64u * static_cast<uint32_t>(v % kRing) + kColsPer * ch, x);
                tc_wait_ld();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(bar(kBarS1Free + v % kRing));
                const int key0 = v * kSub + kColsPer * ch;
                const bool full = full_sub(v);
                float s2[kColsPer];
                float cm = -INFINITY;
                #pragma unroll
                for (int i = 0; i < kColsPer; i += 2) {
                    const float2 t = __fmul2_rn(make_float2(__uint_as_float(x[i]), __uint_as_float(x[i + 1])),
                                                make_float2(p.c, p.c));
                    s2[i] = t.x;
                    s2[i + 1] = t.y;
                }
                if (!full) {
                    #pragma unroll
                    for (int i = 0; i < kColsPer; ++i) {
                        const int key = key0 + i;
                        if (!(key < p.N && (!p.causal || key <= row))) s2[i] = -INFINITY;
                    }
                }
                #pragma unroll
                for (int i = 0; i < kColsPer; i += 4) {
                    cm = fmaxf(cm, max3f(s2[i], s2[i + 1], fmaxf(s2[i + 2], s2[i + 3])));
                }
                const float mn = fmaxf(m, cm);
                if (mn > -INFINITY) {
                    float sum0 = 0.0f, sum1 = 0.0f;
                    #pragma unroll
                    for (int i = 0; i < kColsPer; i += 2) {
                        sum0 += ex2(s2[i] - mn);
                        sum1 += ex2(s2[i + 1] - mn);
                    }
                    l = (m > -INFINITY ? l * ex2(m - mn) : 0.0f) + (sum0 + sum1);
                    m = mn;
                }
            }
            // combine the quarters of each row (in a fixed order, so every
            // warp gets the same values); every elementwise warp reaches this
            // barrier exactly once, aborted or not
            stats[(ch * 3 + 0) * kRows + r] = m;
            stats[(ch * 3 + 1) * kRows + r] = l;
            stats[(ch * 3 + 2) * kRows + r] = dsum;
            elem_sync();
            float mm = -INFINITY;
            #pragma unroll
            for (int k = 0; k < kSplit; ++k) mm = fmaxf(mm, stats[(k * 3 + 0) * kRows + r]);
            float lsum = 0.0f;
            dsum = 0.0f;
            #pragma unroll
            for (int k = 0; k < kSplit; ++k) {
                const float mk = stats[(k * 3 + 0) * kRows + r];
                lsum += mk > -INFINITY ? stats[(k * 3 + 1) * kRows + r] * ex2(mk - mm) : 0.0f;
                dsum += stats[(k * 3 + 2) * kRows + r];
            }
            lse = mm + log2f(lsum);
            if (ok && row_ok && ch == 0) p.lse[static_cast<std::size_t>(head) * p.M + row] = lse;
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(kBarStats));
        } else {
            // the forward's LSE; D's quarters combined in a fixed order
            stats[(ch * 3 + 2) * kRows + r] = dsum;
            elem_sync();
            dsum = 0.0f;
            #pragma unroll
            for (int k = 0; k < kSplit; ++k) dsum += stats[(k * 3 + 2) * kRows + r];
            if (row_ok) lse = p.lse[static_cast<std::size_t>(head) * p.M + row];
        }
        if (ok && row_ok && ch == 0) p.dsum[static_cast<std::size_t>(head) * p.M + row] = dsum;
        // pass 2: dS = P (dP - D) * score_scale, fp16, over this quarter's S
        // columns; P = 2^(c S - LSE)
        const float2 c2 = make_float2(p.c, p.c), nl2 = make_float2(-lse, -lse);
        const float2 sc2 = make_float2(p.scale, p.scale);
        const float2 nd2 = make_float2(-dsum * p.scale, -dsum * p.scale);
        for (int v = 0; ok && v < nsub; ++v) {
            const int slot = v % kSSlots;
            ok = bw_wait(bar(kBarS + slot), (v / kSSlots) & 1, abort_flag, p.limit_ns);
            if (!ok) break;
            tc_fence_after();
            const uint32_t buf = tmem + lb + kSub * static_cast<uint32_t>(slot) + kColsPer * ch;
            uint32_t x[kColsPer], y[kColsPer];
            tmem_ld16(buf, x);
            tmem_ld16(tmem + lb + kColDp + kColsPer * ch, y);
            tc_wait_ld();
            // the dP slot may take the next sub-block's product
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(kBarDpFree));
            const int key0 = v * kSub + kColsPer * ch;
            const bool full = full_sub(v);
            uint32_t ds[kColsPer / 2];
            #pragma unroll
            for (int i = 0; i < kColsPer / 2; ++i) {
                float2 t = __ffma2_rn(make_float2(__uint_as_float(x[2 * i]), __uint_as_float(x[2 * i + 1])), c2, nl2);
                if (!full) {
                    const int key = key0 + 2 * i;
                    if (!(key < p.N && (!p.causal || key <= row))) t.x = -INFINITY;
                    if (!(key + 1 < p.N && (!p.causal || key + 1 <= row))) t.y = -INFINITY;
                }
                const float2 pr = make_float2(ex2(t.x), ex2(t.y));
                const float2 g =
                    __ffma2_rn(make_float2(__uint_as_float(y[2 * i]), __uint_as_float(y[2 * i + 1])), sc2, nd2);
                const float2 dv = __fmul2_rn(pr, g);
                ds[i] = pack_half2(dv.x, dv.y);
            }
            // packed over the first 8 of the S columns this warp read
            tmem_st8(buf, ds);
            tc_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(kBarP + slot));
        }
        // dQ out: 32-column chunks shared round-robin by the quarters
        if (ok) ok = bw_wait(bar(kBarDone), 0, abort_flag, p.limit_ns);
        if (ok) {
            tc_fence_after();
            float* out = p.dq + (static_cast<std::size_t>(head) * p.M + row) * p.d;
            #pragma unroll 1
            for (int c = 32 * ch; c < p.d; c += 32 * kSplit) {
                uint32_t x[32];
                tmem_ld32(tmem + lb + kColDq + static_cast<uint32_t>(c), x);
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
// query blocks that see the tile stream through (Q, dO) stages, each as two
// 64-query sub-blocks. TMEM: S^T at 0 and dP^T at 64 (free again once the
// elementwise warps have loaded them), the operand slot at 128 (P^T packed in
// its first 32 columns, dS^T in the next 32; written once the previous
// sub-block's accumulation products have read it), K at 192 (fp16 pairs: the
// S^T product takes its A operand from TMEM, only dP^T = V dO^T reads both
// operands from shared memory), dV at 256, dK at 384.
constexpr uint32_t kColOp = 128, kColKc = 192;
// kWithhold: watchdog self-test build: elementwise warp 0 withholds its first
// P-ready arrival, so the accumulation warp's wait for it runs out (the
// output is then not valid; the status word is).
template <int kAtoms, int kSteps, bool kWithhold = false>
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
    int head = 0, order = 0;
    work_item(bid, p.heads, p.k_tiles, head, order);
    const int kt = p.causal ? order : p.k_tiles - 1 - order;
    const int i0 = p.causal ? kt : 0;             // first query block that sees the tile
    const int nq = p.q_tiles - i0;                // may be <= 0 (causal, keys past the last query)
    const int nsub = nq > 0 ? 2 * nq : 0;         // 64-query sub-blocks
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
                if (!bw_wait(bar(kBarBEmpty + s), ((b >> 1) & 1) ^ 1, abort_flag, p.limit_ns)) break;
                if (elect_one()) {
                    // L2 prefetch of the block two loads ahead
                    if (b + 2 < nq) {
                        for (int a = 0; a < kAtoms; ++a) {
                            tma_prefetch_l2_3d(&tm_q, a * 64, (i + 2) * kRows, head);
                            tma_prefetch_l2_3d(&tm_do, a * 64, (i + 2) * kRows, head);
                        }
                    }
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
            // S^T and dP^T products
            const uint32_t dhi = smem_desc_sw128_hi(1024);
            const int ksteps = p.d / 16;
            const uint32_t v_lo = smem_desc_sw128_lo(sbase + L::kA1, 16);
            auto q_lo = [&](int s, uint32_t lbo) { return smem_desc_sw128_lo(sbase + L::kB0 + s * L::kTile, lbo); };
            auto do_lo = [&](int s, uint32_t lbo) { return smem_desc_sw128_lo(sbase + L::kB1 + s * L::kTile, lbo); };
            bool ok = bw_wait(bar(kBarA), 0, abort_flag, p.limit_ns);
            // K is in TMEM once the elementwise warps have copied it
            if (ok) ok = bw_wait(bar(kBarOps), 0, abort_flag, p.limit_ns);
            // S^T(u), dP^T(u) once the elementwise warps have loaded u - 1
            for (int u = 0; ok && u < nsub; ++u) {
                const int b = u >> 1, s = b & 1, h = u & 1;
                if (h == 0) ok = bw_wait(bar(kBarBFull + s), (b >> 1) & 1, abort_flag, p.limit_ns);
                if (ok && u >= 1) ok = bw_wait(bar(kBarDpFree), (u - 1) & 1, abort_flag, p.limit_ns);
                if (!ok) break;
                tc_fence_after();
                if (elect_one()) {
                    mma_sub_ts<kSteps>(tmem, tmem + kColKc, q_lo(s, 16) + kHalfRows16 * h, dhi, ksteps);
                    mma_sub<kSteps>(tmem + 64u, v_lo, do_lo(s, 16) + kHalfRows16 * h, dhi, ksteps);
                    tc_commit(bar(kBarS));
                }
                __syncwarp();
            }
            if (lane == 0) tc_commit(bar(kBarDrain));
            __syncwarp();
            bw_drain(bar(kBarDrain), 0);
        }
    } else if (warp == kMmaAcc) {
        if (nq > 0) {
            // dV += P^T(u) dO, dK += dS^T(u) Q as soon as sub-block u's P^T
            // and dS^T are written
            const uint32_t dhi = smem_desc_sw128_hi(1024);
            const uint32_t idesc_o = idesc_f16_f32(kRows, p.d, true);
            bool ok = true;
            for (int u = 0; ok && u < nsub; ++u) {
                const int b = u >> 1, s = b & 1, h = u & 1;
                ok = bw_wait(bar(kBarP + (u & 1)), (u >> 1) & 1, abort_flag, p.limit_ns);
                if (!ok) break;
                tc_fence_after();
                if (elect_one()) {
                    const uint32_t op = tmem + kColOp;
                    mma_acc<8>(tmem + 256u, op,
                                smem_desc_sw128_lo(sbase + L::kB1 + s * L::kTile, kAtom) + kHalfRows16 * h, dhi, idesc_o,
                                u > 0);
                    mma_acc<8>(tmem + 384u, op + 32u,
                                smem_desc_sw128_lo(sbase + L::kB0 + s * L::kTile, kAtom) + kHalfRows16 * h, dhi, idesc_o,
                                u > 0);
                    tc_commit(bar(kBarAcc));
                    if (h == 1) tc_commit(bar(kBarBEmpty + s));
                    if (u == nsub - 1) tc_commit(bar(kBarDone));
                }
                __syncwarp();
            }
            if (lane == 0) tc_commit(bar(kBarDrain + 1));
            __syncwarp();
            bw_drain(bar(kBarDrain + 1), 0);
        }
    } else {
        // elementwise: thread = (key row = TMEM lane, query quarter ch)
        const int quad = warp & 3, ch = warp >> 2;
        const int r = quad * 32 + static_cast<int>(lane);
        const int key = kt * kRows + r;
        const uint32_t lb = static_cast<uint32_t>(quad * 32) << 16;
        float* stats = reinterpret_cast<float*>(smem + L::kStats);   // [block & 1][-LSE, -D scale][128]
        const float2 c2 = make_float2(p.c, p.c), sc2 = make_float2(p.scale, p.scale);
        bool ok = true;
        if (nq > 0) {
            // the S^T product's A operand: warp quarter ch < kAtoms copies
            // this key row's atom ch of K into TMEM
            ok = bw_wait(bar(kBarA), 0, abort_flag, p.limit_ns);
            if (ok && ch < kAtoms) {
                atom_row_to_tmem(smem + L::kA0, ch, r, tmem + lb + kColKc + 32u * ch);
                tc_wait_st();
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(kBarOps));
        }
        // Row statistics of query block i, staged once per block: thread
        // t < 128 holds -LSE of query t, thread 128 + t its -D * scale. Each
        // thread loads its raw value one block ahead and transforms it only
        // when it stores it, so nothing waits on the load in between and the
        // global-load latency overlaps the previous block's work.
        const int t = static_cast<int>(threadIdx.x);
        const bool stager = t < 2 * kRows;
        const float* stat_src = t < kRows ? p.lse : p.dsum;
        const float stat_mul = t < kRows ? -1.0f : -p.scale;
        auto stat_of = [&](int i) -> float {
            const int q = i * kRows + (t & (kRows - 1));
            return stager && q < p.M ? stat_src[static_cast<std::size_t>(head) * p.M + q] : 0.0f;
        };
        float next_stat = nq > 0 ? stat_of(i0) : 0.0f;
        // Every elementwise warp runs all iterations (the named barrier needs
        // all of them); after an abort they only pass the barrier.
        for (int u = 0; u < nsub; ++u) {
            const int b = u >> 1, h = u & 1, i = i0 + b;
            const float* nl_s = stats + (b & 1) * 2 * kRows;
            const float* nd_s = nl_s + kRows;
            if (h == 0) {
                if (stager) stats[(b & 1) * 2 * kRows + t] = next_stat * stat_mul;
                elem_sync();
                if (b + 1 < nq) next_stat = stat_of(i + 1);
            }
            if (ok) ok = bw_wait(bar(kBarS), u & 1, abort_flag, p.limit_ns);
            if (!ok) continue;
            tc_fence_after();
            uint32_t x[kColsPer], y[kColsPer];
            tmem_ld16(tmem + lb + kColsPer * ch, x);
            tmem_ld16(tmem + lb + 64u + kColsPer * ch, y);
            tc_wait_ld();
            // S^T / dP^T may take the next sub-block's products
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(kBarDpFree));
            const int col0 = kSub * h + kColsPer * ch;     // query within the block
            const int q0 = i * kRows + col0;
            // no mask when every query of the sub-block exists and (causal)
            // sees every key of the tile
            const bool full = i * kRows + kSub * (h + 1) <= p.M &&
                              (!p.causal || kt * kRows + kRows - 1 <= i * kRows + kSub * h);
            uint32_t pt[kColsPer / 2], dst[kColsPer / 2];
            #pragma unroll
            for (int e = 0; e < kColsPer / 2; e += 2) {
                const float4 nl = *reinterpret_cast<const float4*>(nl_s + col0 + 2 * e);
                const float4 nd = *reinterpret_cast<const float4*>(nd_s + col0 + 2 * e);
                #pragma unroll
                for (int f = 0; f < 2; ++f) {
                    const int c = 2 * (e + f);
                    float2 t = __ffma2_rn(make_float2(__uint_as_float(x[c]), __uint_as_float(x[c + 1])), c2,
                                          f == 0 ? make_float2(nl.x, nl.y) : make_float2(nl.z, nl.w));
                    if (!full) {
                        if (!(q0 + c < p.M && (!p.causal || key <= q0 + c))) t.x = -INFINITY;
                        if (!(q0 + c + 1 < p.M && (!p.causal || key <= q0 + c + 1))) t.y = -INFINITY;
                    }
                    const float2 pr = make_float2(ex2(t.x), ex2(t.y));
                    const float2 g = __ffma2_rn(make_float2(__uint_as_float(y[c]), __uint_as_float(y[c + 1])), sc2,
                                                f == 0 ? make_float2(nd.x, nd.y) : make_float2(nd.z, nd.w));
                    const float2 dv = __fmul2_rn(pr, g);
                    pt[e + f] = pack_half2(pr.x, pr.y);
                    dst[e + f] = pack_half2(dv.x, dv.y);
                }
            }
            // the operand slot is free once the products of u - 1 have read it
            if (u >= 1) ok = bw_wait(bar(kBarAcc), (u - 1) & 1, abort_flag, p.limit_ns);
            if (!ok) continue;
            tc_fence_after();
            // this quarter's K step, packed: P^T at +8 ch, dS^T at 32 + 8 ch
            const uint32_t op = tmem + lb + kColOp + (kColsPer / 2) * ch;
            tmem_st8(op, pt);
            tmem_st8(op + 32u, dst);
            tc_wait_st();
            tc_fence_before();
            __syncwarp();
            const bool withheld = kWithhold && u == 0 && warp == 0;
            if (lane == 0 && !withheld) mbar_arrive(bar(kBarP + (u & 1)));
        }
        // dV / dK out: 32-column chunks shared round-robin by the quarters
        if (key < p.N && nq <= 0) {
            float* dv_out = p.dv + (static_cast<std::size_t>(head) * p.N + key) * p.d;
            float* dk_out = p.dk + (static_cast<std::size_t>(head) * p.N + key) * p.d;
            for (int c = 32 * ch; c < p.d; c += 32 * kSplit) {
                for (int e = 0; e < 32 && c + e < p.d; e += 4) {
                    *reinterpret_cast<float4*>(dv_out + c + e) = make_float4(0.f, 0.f, 0.f, 0.f);
                    *reinterpret_cast<float4*>(dk_out + c + e) = make_float4(0.f, 0.f, 0.f, 0.f);
                }
            }
        }
        if (ok && nq > 0) ok = bw_wait(bar(kBarDone), 0, abort_flag, p.limit_ns);
        if (ok && nq > 0) {
            tc_fence_after();
            #pragma unroll 1
            for (int part = 0; part < 2; ++part) {
                float* out = (part == 0 ? p.dv : p.dk) + (static_cast<std::size_t>(head) * p.N + key) * p.d;
                #pragma unroll 1
                for (int c = 32 * ch; c < p.d; c += 32 * kSplit) {
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

template <int kAtoms, bool kHaveLse, int kSteps, bool kWithhold = false>
cudaError_t launch_backward_atoms(const CUtensorMap* maps, const BwdParams& p, cudaStream_t stream,
                                  uint64_t cols_limit_ns = kLimitNs) {
    auto rows = backward_rows_kernel<kAtoms, kHaveLse, kSteps>;
    auto cols = backward_cols_kernel<kAtoms, kSteps, kWithhold>;
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
    BwdParams pc = p;
    pc.limit_ns = cols_limit_ns;
    cols<<<static_cast<unsigned>(col_grid), kBwdThreads, smem, stream>>>(maps[0], maps[1], maps[2], maps[3], pc);
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
    p.limit_ns = kLimitNs;
    CUtensorMap maps[4];
    std::memset(maps, 0, sizeof(maps));
    if (!encode_tile_map(&maps[0], prob.q, p.heads, p.M, p.d) || !encode_tile_map(&maps[1], prob.dout, p.heads, p.M, p.d) ||
        !encode_tile_map(&maps[2], prob.k, p.heads, p.N, p.d) || !encode_tile_map(&maps[3], prob.v, p.heads, p.N, p.d)) {
        return cudaErrorInvalidValue;
    }
    if (prob.watchdog_limit_ns != 0) {
        // self-test build (d = 128): the row kernel runs normally, the column
        // kernel withholds one arrival with its waits limited as asked
        if (p.d != 128) return cudaErrorNotSupported;
        return launch_backward_atoms<2, false, 8, true>(maps, p, stream, prob.watchdog_limit_ns);
    }
    // d = 64 and d = 128 take the builds with the K loops unrolled
    if (p.d == 64) {
        return prob.lse_ready ? launch_backward_atoms<1, true, 4>(maps, p, stream)
                              : launch_backward_atoms<1, false, 4>(maps, p, stream);
    }
    if (p.d == 128) {
        return prob.lse_ready ? launch_backward_atoms<2, true, 8>(maps, p, stream)
                              : launch_backward_atoms<2, false, 8>(maps, p, stream);
    }
    if (p.d < 64) {
        return prob.lse_ready ? launch_backward_atoms<1, true, 0>(maps, p, stream)
                              : launch_backward_atoms<1, false, 0>(maps, p, stream);
    }
    return prob.lse_ready ? launch_backward_atoms<2, true, 0>(maps, p, stream)
                          : launch_backward_atoms<2, false, 0>(maps, p, stream);
}

cudaError_t read_and_clear_backward_status(unsigned int* status) {
    unsigned int zero = 0;
    cudaError_t err = cudaMemcpyFromSymbol(status, g_backward_status, sizeof(unsigned int));
    if (err != cudaSuccess) return err;
    return cudaMemcpyToSymbol(g_backward_status, &zero, sizeof(unsigned int));
}

}  // namespace tilemix
