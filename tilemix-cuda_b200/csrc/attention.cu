// Stages 2-5 of TileMix in one sm_100a kernel: routed QK^T on tcgen05 tensor
// cores (kind::i8 with s32 accumulators, or kind::f16 with f32 accumulators),
// online softmax, fp16 PV MMA and output normalisation. The S x S score matrix
// only ever lives in TMEM.
//
// Semantics per head follow the reference kernel (src/tilemix.cu:51-220):
//   * routing bit per (16-row query tile, 32-key tile), decoded exactly as
//     src/tilemix.cu:99-103;
//   * INT8 score = float(dot) * q_scale(row/128) * k_scale(key/64) * score_scale,
//     FP16 score = (q . k in fp32) * score_scale (src/tilemix.cu:151-165);
//   * softmax over all keys < N (plus the causal extension key <= query);
//   * O = (sum_k p_k v_k) / (sum_k p_k) in fp32 (src/tilemix.cu:213-219).
// Differences that stay inside the parity tolerance: exp2 with log2(e) folded
// into the score scale, P carried as two fp16 terms (hi + lo) through two PV
// tensor-core MMAs (~2^-22 relative, vs the reference's fp32 P), and the
// running max only moved when it grows by more than 2^15 (the final result is
// unchanged mathematically; P stays <= 32768, inside fp16's range).
//
// CTA = one 128-row query tile of one head, 512 threads:
//   warps 0-7  softmax: warp w serves TMEM lanes 32*(w%4).. (query rows) and
//              the 64-key half (w/4) of every 128-key block, so each SM
//              sub-partition runs two softmax warps on the same block; each
//              half keeps its own running max, row sum and O accumulator
//   warps 12-15 O rescale: warp w rescales O_0 and O_1 of TMEM lanes
//              32*(w%4).. when a softmax warp of those rows has moved its
//              running max, off the softmax warps' path (they publish the
//              per-row factor and go on to the exponent)
//   warps 8,10 MMA issuers, one per 64-key half h (warp 8 also owns TMEM:
//              S_a | S_b | O_0 | O_1, all 512 columns); S is double-buffered
//              so QK of block j+2 runs while the softmax works on block j+1
//   warp 9     producer: TMA (or, for head dims TMA cannot address, plain
//              loads) of Q/Q8 once, then per 128-key block K/K8 and V (two
//              stages each), 128-byte swizzled; publishes each block's
//              routing summary, per-half MMA plans and K scales in a
//              shared-memory ring
//   warp 11    spare: completes the control warpgroup (warps 8-11), whose
//              registers setmaxnreg lowers so the softmax warps get more
// MMA order, per key half h (one MMA warp each): QK(0), QK(1), then per block
// j: PV(j) of half h as soon as softmax half h has published P(j), then
// QK(j+2) of half h (N = 64) into the S columns that PV(j) just read (same
// issuing thread: the in-order tensor pipe guarantees PV(j) reads P before
// QK(j+2) overwrites it). The halves touch disjoint S and O columns, so their
// P -> PV -> QK -> S chains run in parallel; the K and V stages both halves
// read are released after both MMA warps' commits. P overwrites S in TMEM (per
// 32-key chunk: fp16 hi in the chunk's first 16 columns, lo in the last 16)
// and is the TMEM A operand of the PV MMAs. tcgen05.mma is issued under
// elect.sync (a lane == 0 test made every issue several times slower).
//
// Routing inside the 128-row tile: for each 32-key tile the 8 routing bits of
// the tile's 16-row query tiles select INT8 or FP16 per 16 rows. Per key half,
// a uniform half-block is one MMA (N = 64) of its precision per K step; a mixed
// one is a "base" MMA of one precision for all rows, then "overlay" MMAs of
// the other precision over the key-tile runs that need it, with the TMEM lanes
// of rows that keep the base result disabled (tcgen05.mma disable-output-lane);
// the in-order tensor pipe makes the overlay overwrite the base exactly where
// routed.
//
// Every mbarrier wait is bounded (1 s of %globaltimer). A wait that runs out
// records a code in g_tilemix_status, raises a CTA-wide abort flag and every
// role returns; in-flight TMA loads and MMAs are drained (again bounded)
// before TMEM is freed, so a protocol bug surfaces as an error status instead
// of a hung GPU.
#include "kernels.cuh"
#include "quant_math.cuh"
#include "sm100.cuh"

#include <cuda.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <mutex>

namespace tilemix {

__device__ unsigned int g_tilemix_status = 0;

namespace {

using namespace sm100;

constexpr int kTileRows = 128;               // query rows per CTA (tcgen05 M)
constexpr int kTileKeys = 128;               // keys per block
constexpr int kKStages = 2;
constexpr int kVStages = 2;
constexpr int kRouteSlots = 8;               // the producer runs at most ~3 blocks ahead
constexpr int kSoftmaxWarps = 8;
constexpr int kSoftmaxThreads = 32 * kSoftmaxWarps;
constexpr int kMmaWarp = 8;           // MMA issuer of key half 0, TMEM owner
constexpr int kMmaWarp1 = 10;         // MMA issuer of key half 1
constexpr int kProducerWarp = 9;
constexpr int kCorrWarp0 = 12;        // warps 12-15: O rescale of TMEM lane quarter (warp % 4)
constexpr int kAttnThreads = 512;
// Registers per thread after the role split (setmaxnreg; per warpgroup:
// softmax warps 0-7, control warps 8-11, rescale warps 12-15). The three
// shares add up to the 65536 registers of the SM exactly.
constexpr int kSoftmaxRegs = 160;
constexpr int kCtrlRegs = 80;
constexpr int kCorrRegs = 112;
static_assert(2 * 128 * kSoftmaxRegs + 128 * kCtrlRegs + 128 * kCorrRegs <= 65536, "register split");
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColO = 256;              // S_a at 0, S_b at 128, O_0 at 256, O_1 at 384
constexpr uint32_t kAtomBytes = 128 * 128;   // 128 rows x 128 bytes
constexpr uint64_t kWaitLimitNs = 1000000000ull;   // default watchdog limit of one wait
constexpr uint32_t kSuspendNs = 200000;      // per try_wait suspension (wakes early on completion)
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleLog2 = 15.0f;        // rescale only when the max grows by > 2^15 (P <= 32768)
// Single-term P: rounding p to fp16 changes each p by at most 2^-11 p, so a
// key half-block whose |v| are all <= 3.5 adds at most 2^-11 * 3.5 = 1.7e-3 to
// any output element (O = sum p v / sum p, with the sum over the unrounded p):
// inside the 2e-3 parity bar. Such halves skip the P_lo term (decided from the
// per-64-key-block max |v| the caller passes, v_absmax).
constexpr float kSingleTermVMax = 3.5f;

__device__ __forceinline__ uint32_t col_s(int b) { return static_cast<uint32_t>(b) * 128u; }

// Watchdog codes (bit positions say which wait gave up).
enum : unsigned int {
    kStatusProducer = 1u << 0,
    kStatusMma = 1u << 1,
    kStatusSoftmax = 1u << 2,
    kStatusDrain = 1u << 3,
};

// Per-block routing summary published by the producer in a shared-memory ring
// (global loads issued from the softmax loop proved far costlier than their
// latency; only the producer touches the routing words and K scales):
//   pats   bits [8 kt, 8 kt + 8): INT8 bit of the tile's 8 query tiles for key tile kt
//   scales the block's two 64-key K scales (fp16, 0 when unrouted)
//   plan   the block's QK MMA plan per 64-key half (see make_plan; key
//          tiles counted from the half's first)
//   single bit h set: every |v| of the half's 64 keys is <= kSingleTermVMax, so
//          P of that half is stored as one fp16 term and PV runs once
struct RouteSlot {
    uint32_t pats;
    uint32_t scales;
    std::uint64_t plan[2];
    uint32_t single;    // bit h: key half h of the block takes single-term P (see kSingleTermVMax)
    uint32_t pad;
};

template <int kAtoms>
struct SmemLayout {
    static constexpr uint32_t kTileF16 = kAtoms * kAtomBytes;
    static constexpr uint32_t kQ = 0;
    static constexpr uint32_t kQ8 = kQ + kTileF16;
    static constexpr uint32_t kK = kQ8 + kAtomBytes;                    // [2 stages] fp16
    static constexpr uint32_t kK8 = kK + kKStages * kTileF16;          // [2 stages] int8
    static constexpr uint32_t kV = kK8 + kKStages * kAtomBytes;        // [2 stages]
    static constexpr uint32_t kBiasA = kV + kVStages * kTileF16;       // 8 x 128 B of fp16 2048
    static constexpr uint32_t kBiasB = kBiasA + 1024;                   // 8 x 128 B of fp16 384
    static constexpr uint32_t kAlpha = kBiasB + 1024;                   // [S buffer][half][row] O rescale factors
    static constexpr uint32_t kRoute = kAlpha + 2 * 2 * kTileRows * 4;  // [kRouteSlots]
    static constexpr uint32_t kXchg = kRoute + kRouteSlots * sizeof(RouteSlot);  // [2][256] u64 pair handshake words
    static constexpr uint32_t kBars = kXchg + 2 * kSoftmaxThreads * 8;
    static constexpr uint32_t kNumBars = 23 + kRouteSlots + 16 + 1;
    static constexpr uint32_t kMisc = kBars + kNumBars * 8;            // tmem base, abort flag
    static constexpr uint32_t kQRed = kMisc + 16;                       // [2][8] fused-Q absmax per softmax warp
    static constexpr uint32_t kEnd = kQRed + 64;
    static constexpr uint32_t kBytes = kEnd + 1024;                     // + alignment slack
    static_assert(kBytes <= 232448, "exceeds the 227 KB of shared memory a CTA can opt into");
    static_assert(kBiasA % 1024 == 0, "128-byte-swizzled operands start on 1024-byte boundaries");
};

// S-full, P-full and PV-done are per (S buffer b, key half h) at base + 2 b + h;
// the drain barrier per MMA warp; alpha-ready per (b, h, lane quarter q) at
// base + 4 (2 b + h) + q; Q8-ready (fused Q quantization) takes one arrival per
// softmax warp.
enum Bar : int {
    kBarQFull = 0, kBarKFull = 1, kBarKEmpty = 3, kBarVFull = 5, kBarVEmpty = 7,
    kBarSFull = 9, kBarPFull = 13, kBarPvDone = 17, kBarDrain = 21, kBarRoute = 23,
    kBarAlpha = 23 + kRouteSlots, kBarQ8Ready = 23 + kRouteSlots + 16,
};

// QK plan of the tile for one key block, packed in 64 bits:
//   bit 0 base precision (1 = INT8), bits [1,4) base key tiles (0 = no QK),
//   bits [4,7) overlay count, overlay i at bit 8 + 13 i: key tile (2 bits),
//   key-tile count (3 bits), row-tile set (8 bits). Overlays are of the other
//   precision and run after the base on the listed 16-row tiles only.
// Runs of equal, non-empty row sets over the block's key tiles (byte kt of
// `sets`), packed as the plan's overlay entries; straight-line code for the
// four key tiles of a block.
__device__ __forceinline__ int plan_runs(uint32_t sets, int ktiles, std::uint64_t& packed, int& tiles) {
    int runs = 0, start = 0, len = 0;
    uint32_t cur = 0;
    packed = 0;
    tiles = 0;
    #pragma unroll
    for (int kt = 0; kt <= 4; ++kt) {
        const uint32_t set = kt < ktiles ? (sets >> (8 * kt)) & 0xffu : 0u;
        if (set != cur) {
            if (cur) {
                packed |= static_cast<std::uint64_t>(static_cast<uint32_t>(start) | (static_cast<uint32_t>(len) << 2) |
                                                     (cur << 5)) << (8 + 13 * runs);
                ++runs;
                tiles += len;
            }
            cur = set;
            start = kt;
            len = 0;
        }
        ++len;
    }
    return runs;
}

// A mixed block is one full-width base MMA of one precision, then overlays of
// the other precision. Base chosen by tensor-time estimate per d = 128 (K steps
// x cycles per step; one step of N keys costs about max(N / 2, 32 + N / 4)
// cycles, shared-memory bound below N = 128): INT8 base 256, FP16 base 512,
// FP16 overlay run of L key tiles 256 + 64 L, INT8 overlay run 128 + 32 L.
__device__ __forceinline__ std::uint64_t make_plan(uint32_t i8set, uint32_t f16set, int ktiles) {
    if (ktiles <= 0 || (i8set | f16set) == 0) return 0;
    const std::uint64_t plan = static_cast<std::uint64_t>(ktiles) << 1;
    if (!i8set || !f16set) return plan | (i8set ? 1ull : 0ull);
    std::uint64_t f16_packed, i8_packed;
    int f16_tiles, i8_tiles;
    const int f16_runs = plan_runs(f16set, ktiles, f16_packed, f16_tiles);
    const int i8_runs = plan_runs(i8set, ktiles, i8_packed, i8_tiles);
    const int cost_i8_base = 256 + 256 * f16_runs + 64 * f16_tiles;
    const int cost_f16_base = 512 + 128 * i8_runs + 32 * i8_tiles;
    if (cost_i8_base <= cost_f16_base) return plan | 1ull | (static_cast<std::uint64_t>(f16_runs) << 4) | f16_packed;
    return plan | (static_cast<std::uint64_t>(i8_runs) << 4) | i8_packed;
}

struct Params {
    const __half* q;
    const __half* k;
    const __half* v;
    const std::int8_t* q8;
    const std::int8_t* k8;
    const __half* q_scales;
    const __half* k_scales;
    float* o;
    const std::uint64_t* words;
    std::uint8_t* decoded_bits;
    std::int32_t* score_dots;
    int heads, M, N, d;
    int q_tiles, kv_blocks, q16_tiles, k32_tiles;
    int group;
    int words_per_row;
    long long words_per_head;
    int q_scale_blocks, k_scale_blocks;
    float scale_log2;
    int causal;
    int routed;
    int fuse_q;          // Q quantized inside the CTA (no Q8 / q_scales inputs)
    const __half* v_absmax;   // optional [heads][k_scale_blocks] max |v| per 64-key block
    std::int8_t* q8_out;      // fused Q: optional Q8 output [heads][M][d]
    __half* q_scales_out;     // fused Q: optional scale output [heads][q_scale_blocks]
    float* lse_out;           // optional [heads][M] base-2 log-sum-exp of each row's scores
    int q8_vec;          // q8_out takes 16-byte stores (d % 16 == 0, aligned)
    int f16_ksteps, i8_ksteps, pv_n;
    int o_vec;
    int o_tma;           // fp32 O written by TMA stores from shared memory
    uint64_t wait_limit_ns;  // watchdog limit of one wait
    int head_group;      // heads scheduled together (their K/V stay L2-resident)
    int prefetch_ahead;  // CTA distance of the Q tile prefetched into L2 (the SM count)
    // strided output (kStrided variants)
    void* o_data;
    int o_dtype;         // 0 fp32, 1 fp16, 2 bf16
    int o_hpb;           // heads per batch
    long long o_sb, o_sh, o_sm;
};

// Watchdog state of a CTA: the shared-memory abort flag every role polls and
// the time limit of one wait (1 s; shorter only in the watchdog self-test).
struct Watchdog {
    volatile int* flag;
    uint64_t limit_ns;
};

// Bounded wait, called by all 32 lanes of a warp; returns a warp-uniform
// verdict. On timeout it records `code` and raises the CTA abort flag.
// Slow path of a bounded wait. Kept inline: an out-of-line call from the
// divergent slow path broke the warp convergence that the warp-wide
// (.sync.aligned) tcgen05 instructions after the wait rely on.
__device__ __forceinline__ bool wait_bar_slow(uint32_t bar, uint32_t parity, const Watchdog& wd,
                                           unsigned int code) {
    const uint64_t start = global_timer_ns();
    while (true) {
        if (mbar_try_wait_suspend(bar, parity, kSuspendNs)) return true;
        if (*wd.flag) return false;
        if (global_timer_ns() - start > wd.limit_ns) {
            *wd.flag = 1;
            atomicOr(&g_tilemix_status, code);
            return false;
        }
    }
}

__device__ __forceinline__ bool wait_bar(uint32_t bar, uint32_t parity, const Watchdog& wd,
                                         unsigned int code) {
    bool ok = mbar_try_wait(bar, parity);
    if (!ok) ok = wait_bar_slow(bar, parity, wd, code);
    return __all_sync(0xffffffffu, ok);
}

// Drain wait, for asynchronous work this CTA issued itself (TMA loads into
// its shared memory, MMAs on its TMEM) to finish before that memory is given
// back. That work completes on its own, so this wait ignores the abort flag
// (after an abort it is exactly the wait that matters) and gives up, with
// kStatusDrain recorded, only after the time limit.
__device__ __forceinline__ void drain_wait(uint32_t bar, uint32_t parity, const Watchdog& wd) {
    if (!mbar_try_wait(bar, parity)) {
        const uint64_t start = global_timer_ns();
        while (!mbar_try_wait_suspend(bar, parity, kSuspendNs)) {
            if (global_timer_ns() - start > wd.limit_ns) {
                *wd.flag = 1;
                atomicOr(&g_tilemix_status, kStatusDrain);
                break;
            }
        }
    }
    __syncwarp();
}

// Handshake between the two softmax threads of a query row (threads t and
// t ^ 128: same TMEM lane, other 64-key half). Each publishes (tag, value) as
// one 64-bit shared-memory word, so value and tag are seen together, then
// waits (bounded) for the partner's word with the same tag. Two slot sets
// alternate by tag parity: a thread can only reuse a slot after it has read
// the partner's next word, which the partner writes after reading this one.
__device__ __forceinline__ bool pair_wait_slow(volatile std::uint64_t* slot, uint32_t tag, std::uint64_t& v,
                                            const Watchdog& wd) {
    const uint64_t start = global_timer_ns();
    while (true) {
        v = *slot;
        if (static_cast<uint32_t>(v >> 32) == tag) return true;
        if (*wd.flag) return false;
        if (global_timer_ns() - start > wd.limit_ns) {
            *wd.flag = 1;
            atomicOr(&g_tilemix_status, kStatusSoftmax);
            return false;
        }
    }
}

__device__ __forceinline__ bool pair_exchange(volatile std::uint64_t* slots, int me, uint32_t tag, float mine,
                                              float& theirs, const Watchdog& wd) {
    slots[me] = (static_cast<std::uint64_t>(tag) << 32) | __float_as_uint(mine);
    std::uint64_t v = slots[me ^ 128];
    bool ok = static_cast<uint32_t>(v >> 32) == tag;
    if (!ok) ok = pair_wait_slow(slots + (me ^ 128), tag, v, wd);
    theirs = __uint_as_float(static_cast<uint32_t>(v));
    return __all_sync(0xffffffffu, ok);
}

// Routing of one key block for the tile's 8 query tiles, one routing bit per
// lane: lane = 8 * kt + l reads the word of query tile l for key tile kt of the
// block, so a ballot yields the block's whole pattern (bit 8 kt + l = INT8 for
// query tile l, key tile kt). Words and the block's two K scales are loaded
// one block ahead and decoded in the next iteration: decoding right after the
// load would stall the producer on global-load latency every block.
struct RouteFetch {
    const std::uint64_t* row;   // this lane's query tile's routing words
    uint32_t kt;                // this lane's key tile within a block
    bool q_ok;                  // this lane's query tile exists
    std::uint64_t word;         // prefetched word
    uint32_t bit;               // bit of the prefetched word
    uint32_t scale;             // lanes 0, 1: prefetched K scale (fp16 bits) of the block's 64-key halves
    uint32_t vmax;              // lanes 2, 3: prefetched max |v| (fp16 bits) of the block's 64-key halves

    __device__ __forceinline__ void init(const Params& p, int head, int qt, uint32_t lane) {
        const int q16 = qt * (kTileRows / 16) + static_cast<int>(lane & 7u);
        kt = lane >> 3;
        q_ok = q16 < p.q16_tiles;
        row = p.routed ? p.words + head * p.words_per_head + static_cast<long long>(q16) * p.words_per_row : nullptr;
    }

    __device__ __forceinline__ void fetch(const Params& p, int head, int j, int nblk, uint32_t lane) {
        const uint32_t gkt = 4u * static_cast<uint32_t>(j) + kt;
        const uint32_t group = p.routed ? gkt / static_cast<uint32_t>(p.group) : 0u;
        bit = group & 63u;
        word = p.routed && q_ok && j < nblk && gkt < static_cast<uint32_t>(p.k32_tiles) ? __ldg(row + (group >> 6)) : 0ull;
        const int sb = 2 * j + static_cast<int>(lane);
        scale = p.routed && lane < 2 && j < nblk && sb < p.k_scale_blocks
                    ? __half_as_ushort(p.k_scales[static_cast<std::size_t>(head) * p.k_scale_blocks + sb]) : 0u;
        const int vb = 2 * j + static_cast<int>(lane) - 2;
        vmax = p.v_absmax && (lane == 2 || lane == 3) && j < nblk && vb < p.k_scale_blocks
                   ? __half_as_ushort(p.v_absmax[static_cast<std::size_t>(head) * p.k_scale_blocks + vb]) : 0x7E00u;
    }

    // pats: INT8 bits; valid: bits of existing (query tile, key tile) pairs.
    template <bool kPvHint>
    __device__ __forceinline__ void decode(const Params& p, int j, uint32_t& pats, uint32_t& valid,
                                           uint32_t& scales, uint32_t& single) const {
        const bool ok = q_ok && 4 * j + static_cast<int>(kt) < p.k32_tiles;
        valid = __ballot_sync(0xffffffffu, ok);
        pats = __ballot_sync(0xffffffffu, ok && ((word >> bit) & 1ull) != 0);
        scales = __shfl_sync(0xffffffffu, scale, 0) | (__shfl_sync(0xffffffffu, scale, 1) << 16);
        single = 0u;
        if (kPvHint) {
            // NaN (0x7E00, also "no statistics") compares false
            const bool small = __half2float(__ushort_as_half(static_cast<unsigned short>(vmax))) <= kSingleTermVMax;
            single = (__ballot_sync(0xffffffffu, small) >> 2) & 3u;
        }
    }
};

__device__ __forceinline__ void lane_mask(uint32_t tiles, uint32_t (&m)[4]) {
    #pragma unroll
    for (int w = 0; w < 4; ++w) {
        m[w] = ((tiles >> (2 * w)) & 1u ? 0x0000ffffu : 0u) | ((tiles >> (2 * w + 1)) & 1u ? 0xffff0000u : 0u);
    }
}

// Plain-load fallback for head dims TMA cannot address (d % 16 != 0 or
// unaligned bases): writes the same 128-byte-swizzled K-major layout TMA
// produces, zero-filling rows >= rows_total and columns >= d.
__device__ void manual_tile_f16(uint8_t* dst, const __half* src, int row0, int rows_total, int d,
                                int atoms, uint32_t lane) {
    const uint16_t* s = reinterpret_cast<const uint16_t*>(src);
    for (int c = lane; c < atoms * kTileRows * 8; c += 32) {
        const int atom = c / (kTileRows * 8), rem = c % (kTileRows * 8);
        const int row = rem / 8, chunk = rem % 8;
        const int col0 = atom * 64 + chunk * 8, grow = row0 + row;
        uint32_t w[4];
        #pragma unroll
        for (int e = 0; e < 4; ++e) {
            uint32_t lo = 0, hi = 0;
            const int c0 = col0 + 2 * e;
            if (grow < rows_total) {
                const std::size_t base = static_cast<std::size_t>(grow) * d;
                if (c0 < d) lo = s[base + c0];
                if (c0 + 1 < d) hi = s[base + c0 + 1];
            }
            w[e] = lo | (hi << 16);
        }
        const uint32_t off = atom * kAtomBytes + row * 128 + ((chunk ^ (row & 7)) << 4);
        *reinterpret_cast<uint4*>(dst + off) = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

__device__ void manual_tile_i8(uint8_t* dst, const std::int8_t* src, int row0, int rows_total,
                               int d, uint32_t lane) {
    const uint8_t* s = reinterpret_cast<const uint8_t*>(src);
    for (int c = lane; c < kTileRows * 8; c += 32) {
        const int row = c / 8, chunk = c % 8;
        const int col0 = chunk * 16, grow = row0 + row;
        uint32_t w[4] = {0u, 0u, 0u, 0u};
        if (grow < rows_total) {
            const std::size_t base = static_cast<std::size_t>(grow) * d;
            #pragma unroll
            for (int e = 0; e < 16; ++e) {
                const int col = col0 + e;
                if (col < d) w[e >> 2] |= static_cast<uint32_t>(s[base + col]) << ((e & 3) * 8);
            }
        }
        const uint32_t off = row * 128 + ((chunk ^ (row & 7)) << 4);
        *reinterpret_cast<uint4*>(dst + off) = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

// Strided output: 32 consecutive columns [c, c + 32) of one row, starting at
// element offset row_off, as fp32 / fp16 / bf16 (round to nearest even).
// 16-byte stores when p.o_vec says the base, the strides and d allow them.
__device__ __forceinline__ void store_strided_row(const Params& p, long long row_off, int c,
                                                  const uint32_t (&x)[32]) {
    if (p.o_dtype == 0) {
        float* out = static_cast<float*>(p.o_data) + row_off;
        if (p.o_vec) {
            #pragma unroll
            for (int i = 0; i < 32; i += 4) {
                if (c + i < p.d) {
                    reinterpret_cast<float4*>(out + c + i)[0] = make_float4(
                        __uint_as_float(x[i]), __uint_as_float(x[i + 1]),
                        __uint_as_float(x[i + 2]), __uint_as_float(x[i + 3]));
                }
            }
        } else {
            #pragma unroll
            for (int i = 0; i < 32; ++i) {
                if (c + i < p.d) out[c + i] = __uint_as_float(x[i]);
            }
        }
        return;
    }
    uint32_t h[16];
    #pragma unroll
    for (int i = 0; i < 16; ++i) {
        h[i] = p.o_dtype == 1 ? pack_half2(__uint_as_float(x[2 * i]), __uint_as_float(x[2 * i + 1]))
                              : pack_bf162(__uint_as_float(x[2 * i]), __uint_as_float(x[2 * i + 1]));
    }
    uint16_t* out = static_cast<uint16_t*>(p.o_data) + row_off;
    if (p.o_vec) {
        #pragma unroll
        for (int i = 0; i < 4; ++i) {
            if (c + 8 * i < p.d) {
                reinterpret_cast<uint4*>(out + c + 8 * i)[0] =
                    make_uint4(h[4 * i], h[4 * i + 1], h[4 * i + 2], h[4 * i + 3]);
            }
        }
    } else {
        #pragma unroll
        for (int i = 0; i < 32; ++i) {
            if (c + i < p.d) out[c + i] = static_cast<uint16_t>((i & 1) ? h[i >> 1] >> 16 : h[i >> 1] & 0xffffu);
        }
    }
}

// Absmax of the Q tile over the 256 softmax threads: warp shuffles, then one
// named barrier (id 1) of the eight softmax warps and a read of the eight
// warp maxima in `red`. NaN-propagating when `nan` is set (the fast-path
// verdict), NaN-ignoring otherwise; exact either way (fp16 magnitudes).
__device__ __forceinline__ float block_absmax(float a, float b, float* red, int t, bool nan) {
    auto mx = [nan](float x, float y) { return nan && (x != x || y != y) ? NAN : fmaxf(x, y); };
    float local = mx(a, b);
    #pragma unroll
    for (int offset = 16; offset > 0; offset >>= 1) local = mx(local, __shfl_xor_sync(0xffffffffu, local, offset));
    if ((t & 31) == 0) red[t >> 5] = local;
    asm volatile("bar.sync 1, %0;" :: "r"(kSoftmaxThreads) : "memory");
    float total = 0.0f;
    #pragma unroll
    for (int w = 0; w < kSoftmaxWarps; ++w) total = mx(total, red[w]);
    return total;
}

// Q quantization fused into the attention CTA. The CTA's 128-row query tile
// is exactly one Q quantization block (reference include/attention_fused.h:13),
// so the 256 softmax threads quantize it from the fp16 tile the producer has
// loaded, before their first scores arrive: thread t takes row t / 2 and half
// t % 2 of the row's 16-byte fp16 chunks, the block absmax is reduced through
// warp shuffles and a named barrier of the eight softmax warps, and each
// element is rounded by the standalone quantizer's own functions
// (quant_math.cuh: branch-free for finite tiles, element-wise exact for tiles
// holding NaN or inf), so Q8 and the scale are the same bytes
// quantize_tilemix_qk produces. The INT8 tile goes straight into the
// 128-byte-swizzled Q8 operand in shared memory; the MMA warps wait for the
// Q8-ready barrier. Optionally Q8 and the fp16 scale are also written to
// global memory. Called by all 256 softmax threads; returns false (after the
// named barrier, which every thread reaches) when the Q wait gave up.
template <int kAtoms>
__device__ __forceinline__ bool quantize_q_tile(const Params& p, uint8_t* smem, uint32_t q_full_bar,
                                                uint32_t q8_ready_bar, int head, int qt, const Watchdog& wd,
                                                float& q_scale) {
    using L = SmemLayout<kAtoms>;
    constexpr int kChunks = 4 * kAtoms;                 // fp16 16-byte chunks per thread
    const int t = static_cast<int>(threadIdx.x);        // 0..255
    const int r = t >> 1, part = t & 1;
    const uint32_t lane = threadIdx.x & 31u;
    const bool ok = wait_bar(q_full_bar, 0, wd, kStatusSoftmax);
    uint4 v[kChunks];
    __half2 m2 = __float2half2_rn(0.0f);
    #pragma unroll
    for (int i = 0; i < kChunks; ++i) {
        const int g = part * kChunks + i, atom = g >> 3, c = g & 7;
        v[i] = ok ? *reinterpret_cast<const uint4*>(smem + L::kQ + atom * kAtomBytes + r * 128 + ((c ^ (r & 7)) << 4))
                  : make_uint4(0u, 0u, 0u, 0u);
        const __half2* h = reinterpret_cast<const __half2*>(&v[i]);
        #pragma unroll
        for (int e = 0; e < 4; ++e) m2 = __hmax2_nan(m2, __habs2(h[e]));   // exact; a NaN reaches the verdict
    }
    float* red = reinterpret_cast<float*>(smem + L::kQRed);
    float absmax = block_absmax(__low2float(m2), __high2float(m2), red, t, true);
    uint4 q8[kChunks / 2];
    float scale;
    if (fast_block(absmax)) {
        // every block of finite, not-all-zero inputs: branch-free exact rounding
        scale = __fdiv_rn(absmax, 127.0f);
        const float y = __frcp_rn(scale);
        const float2 neg_s2 = make_float2(-scale, -scale), y2 = make_float2(y, y);
        #pragma unroll
        for (int i = 0; i < kChunks; i += 2) {
            q8[i / 2] = make_uint4(quantize4_fast(v[i].x, v[i].y, neg_s2, y2), quantize4_fast(v[i].z, v[i].w, neg_s2, y2),
                                   quantize4_fast(v[i + 1].x, v[i + 1].y, neg_s2, y2),
                                   quantize4_fast(v[i + 1].z, v[i + 1].w, neg_s2, y2));
        }
    } else {
        // NaN, +-inf or an all-zero tile (uniform over the CTA): absmax without
        // NaN, then the element-wise exact rounding
        m2 = __float2half2_rn(0.0f);
        #pragma unroll
        for (int i = 0; i < kChunks; ++i) {
            const __half2* h = reinterpret_cast<const __half2*>(&v[i]);
            #pragma unroll
            for (int e = 0; e < 4; ++e) m2 = __hmax2(m2, __habs2(h[e]));   // ignores a NaN like fmaxf
        }
        absmax = block_absmax(__low2float(m2), __high2float(m2), red + kSoftmaxWarps, t, false);
        scale = __fdiv_rn(absmax, 127.0f);
        const float recip = scale > 0.0f ? __frcp_rn(scale) : 0.0f;
        const float2 recip2 = make_float2(recip, recip);
        #pragma unroll
        for (int i = 0; i < kChunks; i += 2) {
            uint32_t w[4] = {0u, 0u, 0u, 0u};
            #pragma unroll
            for (int k = 0; k < 2; ++k) {
                const __half2* h = reinterpret_cast<const __half2*>(&v[i + k]);
                #pragma unroll
                for (int e = 0; e < 4; ++e) w[2 * k + (e >> 1)] |= quantize_pair(h[e], scale, recip2) << ((e & 1) * 16);
            }
            q8[i / 2] = make_uint4(w[0], w[1], w[2], w[3]);
        }
    }
    const __half scale_h = __float2half_rn(scale);
    q_scale = __half2float(scale_h);                    // dequantization uses the stored fp16 scale
    #pragma unroll
    for (int i = 0; i < kChunks; i += 2) {
        const int cj = (part * kChunks + i) >> 1;       // int8 16-byte chunk (16 columns)
        *reinterpret_cast<uint4*>(smem + L::kQ8 + r * 128 + ((cj ^ (r & 7)) << 4)) = q8[i / 2];
    }
    fence_proxy_async_smem();                           // generic-proxy writes -> tensor core reads
    __syncwarp();
    if (ok && lane == 0) mbar_arrive(q8_ready_bar);
    if (ok && p.q8_out) {
        const int row = qt * kTileRows + r;
        if (row < p.M) {
            std::int8_t* dst = p.q8_out + (static_cast<std::size_t>(head) * p.M + row) * p.d;
            #pragma unroll
            for (int i = 0; i < kChunks / 2; ++i) {
                const int c0 = (part * kChunks + 2 * i) * 8;
                if (p.q8_vec) {
                    if (c0 < p.d) *reinterpret_cast<uint4*>(dst + c0) = q8[i];
                } else {
                    const uint8_t* b = reinterpret_cast<const uint8_t*>(&q8[i]);
                    for (int e = 0; e < 16 && c0 + e < p.d; ++e) dst[c0 + e] = static_cast<std::int8_t>(b[e]);
                }
            }
        }
    }
    if (ok && p.q_scales_out && t == 0) p.q_scales_out[static_cast<std::size_t>(head) * p.q_scale_blocks + qt] = scale_h;
    return ok;
}

// Work item of CTA `bid`: heads are scheduled in groups (their K/V stay in
// L2 while the group runs); inside a group the heaviest (last) query tiles go
// first.
__device__ __forceinline__ void tile_of(const Params& p, int bid, int& head, int& qt) {
    const int per_group = p.head_group * p.q_tiles;
    const int group0 = (bid / per_group) * p.head_group;
    const int group_heads = min(p.head_group, p.heads - group0);
    const int in_group = bid - (bid / per_group) * per_group;
    qt = p.q_tiles - 1 - in_group / group_heads;
    head = group0 + in_group % group_heads;
}

template <int kAtoms, bool kUseTma, bool kTrace, bool kStrided, bool kWithholdArrive = false, bool kPvHint = false>
__global__ void __launch_bounds__(kAttnThreads, 1)
tilemix_attention_kernel(const __grid_constant__ CUtensorMap tm_q,
                         const __grid_constant__ CUtensorMap tm_k,
                         const __grid_constant__ CUtensorMap tm_v,
                         const __grid_constant__ CUtensorMap tm_q8,
                         const __grid_constant__ CUtensorMap tm_k8,
                         const __grid_constant__ CUtensorMap tm_o,
                         const Params p) {
    using L = SmemLayout<kAtoms>;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_u32 = smem_u32(smem_raw);
    const uint32_t pad = ((raw_u32 + 1023u) & ~1023u) - raw_u32;
    uint8_t* smem = smem_raw + pad;
    const uint32_t sbase = raw_u32 + pad;
    auto bar = [&](int i) -> uint32_t { return sbase + L::kBars + 8u * static_cast<uint32_t>(i); };
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMisc);
    volatile int* abort_ptr = reinterpret_cast<volatile int*>(smem + L::kMisc + 4);
    const Watchdog abort_flag{abort_ptr, p.wait_limit_ns};

    const int warp = threadIdx.x >> 5;
    const uint32_t lane = threadIdx.x & 31u;

    int head, qt;
    tile_of(p, static_cast<int>(blockIdx.x), head, qt);
    const int nblk = p.causal ? min(p.kv_blocks, qt + 1) : p.kv_blocks;
    const int load_i8 = p.routed;
    const int load_q8 = p.routed && !p.fuse_q;    // fused Q: the CTA quantizes Q itself

    if (warp == 0) {
        // One barrier per lane (the set-up barrier waits for the slowest
        // lane, not for ~50 initialisations in a row). Arrival counts: the
        // K and V stages are released by both MMA warps' commits; P-full
        // takes one arrival per softmax warp of the half and per rescale
        // warp; every other barrier one arrival (or one commit).
        for (int i = static_cast<int>(lane); i < static_cast<int>(L::kNumBars); i += 32) {
            const bool stage_empty = (i >= kBarKEmpty && i < kBarKEmpty + kKStages) ||
                                     (i >= kBarVEmpty && i < kBarVEmpty + kVStages);
            const bool p_full = i >= kBarPFull && i < kBarPFull + 4;
            mbar_init(bar(i), p_full ? kSoftmaxWarps / 2 + 4 : stage_empty ? 2 : i == kBarQ8Ready ? kSoftmaxWarps : 1);
        }
        if (lane == 0) *abort_ptr = 0;
        mbar_init_fence();
        fence_proxy_async_smem();
    }
    // The producer's first global loads (routing words, K scales) and the L2
    // prefetch of the Q tile of the CTA one SM-count ahead (likely the next
    // to run on some SM) go out before the set-up barrier, so their latency
    // overlaps the barrier and TMEM set-up.
    RouteFetch route;
    if (warp == kProducerWarp) {
        route.init(p, head, qt, lane);
        route.fetch(p, head, 0, nblk, lane);
        const int ahead = static_cast<int>(blockIdx.x) + p.prefetch_ahead;
        if (kUseTma && lane == 0 && p.prefetch_ahead > 0 && ahead < static_cast<int>(gridDim.x)) {
            int head2, qt2;
            tile_of(p, ahead, head2, qt2);
            for (int a = 0; a < kAtoms; ++a) tma_prefetch_l2_3d(&tm_q, a * 64, qt2 * kTileRows, head2);
            if (load_q8) tma_prefetch_l2_3d(&tm_q8, 0, qt2 * kTileRows, head2);
        }
    }
    for (int i = threadIdx.x; i < 2 * kSoftmaxThreads; i += kAttnThreads) {
        reinterpret_cast<std::uint64_t*>(smem + L::kXchg)[i] = ~0ull;    // no tag matches
    }
    // Constant operands of the INT8 bias MMA: 16 products 2048 * 384 sum to
    // 1.5 * 2^23, exactly, whose fp32 bits are 0x4B400000.
    for (int i = threadIdx.x; i < 512; i += kAttnThreads) {
        reinterpret_cast<uint32_t*>(smem + L::kBiasA)[i] = i < 256 ? 0x68006800u : 0x5E005E00u;
    }
    fence_proxy_async_smem();
    if (warp == kMmaWarp) {
        tmem_alloc(sbase + L::kMisc, kTmemCols);
        tmem_relinquish();
        tc_fence_before();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // Registers follow the roles, one setmaxnreg per warpgroup at the top of
    // its branch: the softmax warpgroups take what the control and rescale
    // warpgroups give up.
    if (warp >= kSoftmaxWarps && warp < kCorrWarp0) {
    // control warpgroup: producer, the two MMA warps and one spare warp
    reg_dealloc<kCtrlRegs>();
    if (warp == kProducerWarp) {
        // ------------------------------------------------------------ producer
        if (kUseTma && lane == 0) {
            tma_prefetch_desc(&tm_q); tma_prefetch_desc(&tm_k); tma_prefetch_desc(&tm_v);
            if (load_q8) tma_prefetch_desc(&tm_q8);
            if (load_i8) tma_prefetch_desc(&tm_k8);
        }
        const std::size_t q_off = static_cast<std::size_t>(head) * p.M * p.d;
        const std::size_t kv_off = static_cast<std::size_t>(head) * p.N * p.d;
        if (kUseTma) {
            if (elect_one()) {
                mbar_arrive_expect_tx(bar(kBarQFull), L::kTileF16 + (load_q8 ? kAtomBytes : 0u));
                for (int a = 0; a < kAtoms; ++a) {
                    tma_load_3d(sbase + L::kQ + a * kAtomBytes, &tm_q, bar(kBarQFull), a * 64, qt * kTileRows, head);
                }
                if (load_q8) tma_load_3d(sbase + L::kQ8, &tm_q8, bar(kBarQFull), 0, qt * kTileRows, head);
            }
        } else {
            manual_tile_f16(smem + L::kQ, p.q + q_off, qt * kTileRows, p.M, p.d, kAtoms, lane);
            if (load_q8) manual_tile_i8(smem + L::kQ8, p.q8 + q_off, qt * kTileRows, p.M, p.d, lane);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(kBarQFull));
        }
        RouteSlot* ring = reinterpret_cast<RouteSlot*>(smem + L::kRoute);
        int k_issued = 0, v_issued = 0;
        // K (and the routing summary) of block i go out one block ahead of V
        // of block i - 1: the K stage frees up when QK(i - 2) completes,
        // earlier than the V stage (PV(i - 3)) on the in-order tensor pipe.
        for (int i = 0; i <= nblk; ++i) {
            if (i < nblk) {
                const int j = i;
                uint32_t pats, valid, scales, single;
                route.decode<kPvHint>(p, j, pats, valid, scales, single);
                route.fetch(p, head, j + 1, nblk, lane);
                const bool need_i8 = pats != 0;
                const bool need_f16 = (valid & ~pats) != 0;
                if (lane == 0) {
                    RouteSlot slot;
                    slot.pats = pats;
                    slot.scales = scales;
                    slot.single = single;
                    const int kt_here = min(4, p.k32_tiles - 4 * j);
                    slot.plan[0] = make_plan(pats & 0xffffu, (valid & ~pats) & 0xffffu, min(2, kt_here));
                    slot.plan[1] = make_plan(pats >> 16, (valid & ~pats) >> 16, min(2, kt_here - 2));
                    ring[j % kRouteSlots] = slot;
                    mbar_arrive(bar(kBarRoute + j % kRouteSlots));   // release: slot visible to its waiters
                }
                __syncwarp();
                const int ks = j % kKStages;
                if (!wait_bar(bar(kBarKEmpty + ks), ((j / kKStages) & 1) ^ 1, abort_flag, kStatusProducer)) break;
                if (kUseTma) {
                    if (elect_one()) {
                        const uint32_t bytes = (need_f16 ? L::kTileF16 : 0u) + (need_i8 ? kAtomBytes : 0u);
                        mbar_arrive_expect_tx(bar(kBarKFull + ks), bytes);
                        if (need_f16) {
                            for (int a = 0; a < kAtoms; ++a) {
                                tma_load_3d(sbase + L::kK + ks * L::kTileF16 + a * kAtomBytes, &tm_k,
                                            bar(kBarKFull + ks), a * 64, j * kTileKeys, head);
                            }
                        }
                        if (need_i8) {
                            tma_load_3d(sbase + L::kK8 + ks * kAtomBytes, &tm_k8, bar(kBarKFull + ks), 0,
                                        j * kTileKeys, head);
                        }
                    }
                } else {
                    if (need_f16) manual_tile_f16(smem + L::kK + ks * L::kTileF16, p.k + kv_off, j * kTileKeys, p.N, p.d, kAtoms, lane);
                    if (need_i8) manual_tile_i8(smem + L::kK8 + ks * kAtomBytes, p.k8 + kv_off, j * kTileKeys, p.N, p.d, lane);
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(bar(kBarKFull + ks));
                }
                k_issued = j + 1;
            }
            if (i >= 1) {
                const int j = i - 1;
                const int vs = j % kVStages;
                if (!wait_bar(bar(kBarVEmpty + vs), ((j / kVStages) & 1) ^ 1, abort_flag, kStatusProducer)) break;
                if (kUseTma) {
                    if (elect_one()) {
                        mbar_arrive_expect_tx(bar(kBarVFull + vs), L::kTileF16);
                        for (int a = 0; a < kAtoms; ++a) {
                            tma_load_3d(sbase + L::kV + vs * L::kTileF16 + a * kAtomBytes, &tm_v, bar(kBarVFull + vs),
                                        a * 64, j * kTileKeys, head);
                        }
                    }
                } else {
                    manual_tile_f16(smem + L::kV + vs * L::kTileF16, p.v + kv_off, j * kTileKeys, p.N, p.d, kAtoms, lane);
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(bar(kBarVFull + vs));
                }
                v_issued = j + 1;
            }
        }
        // Drain: the newest load into each buffer must have landed before the
        // CTA may exit (normally long complete; matters only after an abort).
        if (kUseTma) {
            drain_wait(bar(kBarQFull), 0, abort_flag);
            for (int j = max(0, k_issued - kKStages); j < k_issued; ++j) {
                drain_wait(bar(kBarKFull + j % kKStages), (j / kKStages) & 1, abort_flag);
            }
            for (int j = max(0, v_issued - kVStages); j < v_issued; ++j) {
                drain_wait(bar(kBarVFull + j % kVStages), (j / kVStages) & 1, abort_flag);
            }
        }
    } else if (warp == kMmaWarp || warp == kMmaWarp1) {
        // ----------------------------------------------------------------- MMA
        // Two MMA warps, one per 64-key half mh (on different sub-partitions):
        // each issues its half's PV(j) and QK(j + 2) into S and O columns only
        // that half uses, so the halves' P -> PV -> QK -> S chains run in
        // parallel; the K and V stages both read are released by two commits.
        const int mh = warp == kMmaWarp ? 0 : 1;
        const uint32_t pv_idesc = idesc_f16_f32(kTileRows, p.pv_n, true);
        const RouteSlot* ring = reinterpret_cast<const RouteSlot*>(smem + L::kRoute);
        // Descriptor words: every operand here is 128-byte swizzled with
        // 1024-byte 8-row groups, so the high word is shared; the low word
        // carries the start address (16-byte units) and the leading offset.
        const uint32_t dhi = smem_desc_sw128_hi(1024);
        const uint32_t qf_lo = smem_desc_sw128_lo(sbase + L::kQ, 16);
        const uint32_t qi_lo = smem_desc_sw128_lo(sbase + L::kQ8, 16);
        const uint32_t kf_lo0 = smem_desc_sw128_lo(sbase + L::kK, 16);
        const uint32_t ki_lo0 = smem_desc_sw128_lo(sbase + L::kK8, 16);
        const uint32_t v_lo0 = smem_desc_sw128_lo(sbase + L::kV, kAtomBytes);
        // The bias operands are one 8-row swizzle group each, read for every
        // row group (group stride 0): every element is the same constant.
        const uint32_t bias_a_lo = smem_desc_sw128_lo(sbase + L::kBiasA, 16);
        const uint32_t bias_b_lo = smem_desc_sw128_lo(sbase + L::kBiasB, 16);
        const uint32_t bias_hi = smem_desc_sw128_hi(0);
        const bool f16_full = p.f16_ksteps == 4 * kAtoms;
        const bool i8_full = p.i8_ksteps == 4;
        const uint32_t none[4] = {0u, 0u, 0u, 0u};
        bool ok = wait_bar(bar(kBarQFull), 0, abort_flag, kStatusMma);
        if (ok && p.fuse_q && p.routed) ok = wait_bar(bar(kBarQ8Ready), 0, abort_flag, kStatusMma);
        // One precision over key tiles [kt0, kt0 + nkt) of block j; `off` masks
        // the TMEM lanes (16-row tiles) that keep their previous result.
        // Start addresses advance by byte offset >> 4: 32 B per K step inside
        // a 64-wide (fp16) atom, one atom (kAtomBytes) per 64 of d, 4096 B
        // (32 rows) per key tile.
        auto mma_run = [&](uint32_t d_tmem, int stage, bool int8, int kt0, int nkt, const uint32_t (&off)[4]) {
            const uint32_t d = d_tmem + 32 * kt0;
            const uint32_t kofs = static_cast<uint32_t>(kt0) * 256u;
            if (int8) {
                // The s32 accumulators start at 0x4B400000 (the bits of the
                // float 1.5 * 2^23, written by one f16 MMA of the constant
                // tiles), so they leave the tensor core as the float bits of
                // 1.5 * 2^23 + dot (|dot| < 2^22): the softmax gets the exact
                // float dot with one subtraction.
                mma_f16_ss_w<0>(d, bias_a_lo, bias_b_lo, bias_hi, idesc_f16_f32(kTileRows, 32 * nkt, false), off);
                const uint32_t k_lo = ki_lo0 + static_cast<uint32_t>(stage) * (kAtomBytes >> 4) + kofs;
                const uint32_t idesc = idesc_s8_s32(kTileRows, 32 * nkt);
                if (i8_full) {
                    #pragma unroll
                    for (int ks = 0; ks < 4; ++ks) mma_i8_ss_w<1>(d, qi_lo + 2 * ks, k_lo + 2 * ks, dhi, idesc, off);
                } else {
                    #pragma unroll 1
                    for (int ks = 0; ks < p.i8_ksteps; ++ks) mma_i8_ss_w<1>(d, qi_lo + 2 * ks, k_lo + 2 * ks, dhi, idesc, off);
                }
            } else {
                const uint32_t k_lo = kf_lo0 + static_cast<uint32_t>(stage) * (L::kTileF16 >> 4) + kofs;
                const uint32_t idesc = idesc_f16_f32(kTileRows, 32 * nkt, false);
                if (f16_full) {
                    mma_f16_ss_w<0>(d, qf_lo, k_lo, dhi, idesc, off);
                    #pragma unroll
                    for (int ks = 1; ks < 4 * kAtoms; ++ks) {
                        const uint32_t ko = static_cast<uint32_t>((ks >> 2) * (kAtomBytes >> 4) + (ks & 3) * 2);
                        mma_f16_ss_w<1>(d, qf_lo + ko, k_lo + ko, dhi, idesc, off);
                    }
                } else {
                    mma_f16_ss_w<0>(d, qf_lo, k_lo, dhi, idesc, off);
                    #pragma unroll 1
                    for (int ks = 1; ks < p.f16_ksteps; ++ks) {
                        const uint32_t ko = static_cast<uint32_t>((ks >> 2) * (kAtomBytes >> 4) + (ks & 3) * 2);
                        mma_f16_ss_w<1>(d, qf_lo + ko, k_lo + ko, dhi, idesc, off);
                    }
                }
            }
        };
        // QK^T of block j, key half mh (keys and S columns 64 mh ..), following
        // the producer's plan for that half (the caller has waited for K(j),
        // which also makes block j's routing slot visible).
        auto issue_qk_half = [&](int j) {
            const int ks = j % kKStages;
            const std::uint64_t plan = ring[j % kRouteSlots].plan[mh];
            if (elect_one()) {
                const uint32_t s_tmem = tmem + col_s(j & 1);
                const bool base_i8 = plan & 1ull;
                const int nkt = static_cast<int>((plan >> 1) & 7u);
                if (nkt > 0) mma_run(s_tmem, ks, base_i8, 2 * mh, nkt, none);
                const int overlays = static_cast<int>((plan >> 4) & 7u);
                #pragma unroll 1
                for (int r = 0; r < overlays; ++r) {
                    const uint32_t ov = static_cast<uint32_t>(plan >> (8 + 13 * r)) & 0x1fffu;
                    uint32_t off[4];
                    lane_mask(~(ov >> 5) & 0xffu, off);
                    mma_run(s_tmem, ks, !base_i8, 2 * mh + static_cast<int>(ov & 3u),
                            static_cast<int>((ov >> 2) & 7u), off);
                }
                tc_commit(bar(kBarSFull + 2 * (j & 1) + mh));
                tc_commit(bar(kBarKEmpty + ks));
            }
            __syncwarp();
        };
        // PV of block j, key half mh: O_mh (+)= (P_hi + P_lo) V_j[keys of mh].
        // V tile is MN-major for this MMA: 64-wide d atoms LBO apart, 8-key
        // groups 1024 B apart; each K step covers 16 keys (2048 B). P_hi and
        // P_lo of a 16-key step share the V operand.
        auto issue_pv_half = [&](int j) {
            const int vs = j % kVStages;
            const bool single = kPvHint && ((ring[j % kRouteSlots].single >> mh) & 1u);
            if (elect_one()) {
                const uint32_t v_lo = v_lo0 + static_cast<uint32_t>(vs) * (L::kTileF16 >> 4);
                const uint32_t o_tmem = tmem + kColO + 128u * mh;
                const uint32_t a0 = tmem + col_s(j & 1) + 64u * mh;
                const uint32_t b0 = v_lo + 512u * mh;
                mma_f16_ts_w(o_tmem, a0, b0, dhi, pv_idesc, j > 0 ? 1u : 0u);
                if (single) {
                    #pragma unroll
                    for (int t = 1; t < 4; ++t) {
                        mma_f16_ts_w(o_tmem, a0 + 32 * (t >> 1) + 8 * (t & 1), b0 + 128 * t, dhi, pv_idesc, 1u);
                    }
                } else {
                    mma_f16_ts_w(o_tmem, a0 + 16, b0, dhi, pv_idesc, 1u);
                    #pragma unroll
                    for (int t = 1; t < 4; ++t) {
                        const uint32_t a_hi = a0 + 32 * (t >> 1) + 8 * (t & 1);
                        mma_f16_ts_w(o_tmem, a_hi, b0 + 128 * t, dhi, pv_idesc, 1u);
                        mma_f16_ts_w(o_tmem, a_hi + 16, b0 + 128 * t, dhi, pv_idesc, 1u);
                    }
                }
                tc_commit(bar(kBarPvDone + 2 * (j & 1) + mh));
                tc_commit(bar(kBarVEmpty + vs));
            }
            __syncwarp();
        };
        // QK(0), QK(1), then per block j: PV(j) of this half as soon as the
        // softmax half has published P(j), then QK(j + 2) of this half into
        // the S columns that PV just read (same thread: the in-order tensor
        // pipe makes PV(j) read P before QK(j + 2) overwrites it).
        for (int j = -2; ok && j < nblk; ++j) {
            if (j >= 0) {
                if (!wait_bar(bar(kBarVFull + j % kVStages), (j / kVStages) & 1, abort_flag, kStatusMma) ||
                    !wait_bar(bar(kBarPFull + 2 * (j & 1) + mh), (j >> 1) & 1, abort_flag, kStatusMma)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                issue_pv_half(j);
            }
            const int q = j + 2;
            if (q < nblk) {
                if (!wait_bar(bar(kBarKFull + q % kKStages), (q / kKStages) & 1, abort_flag, kStatusMma)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                issue_qk_half(q);
            }
        }
        // Drain every MMA this thread issued before TMEM can be released
        // (after the final barrier, by warp 8).
        if (lane == 0) tc_commit(bar(kBarDrain + mh));
        __syncwarp();
        drain_wait(bar(kBarDrain + mh), 0, abort_flag);
    }
    } else if (warp < kSoftmaxWarps) {
        reg_alloc<kSoftmaxRegs>();
        // ------------------------------------------------------------- softmax
        // Thread = (query row, 64-key half h). Per block it reads its half's
        // two 32-key chunks from TMEM once, turns INT8 chunks into exact
        // floats, takes the half's max (each half keeps its own running max,
        // sum and O; the two halves of a row meet only in the epilogue), then
        // exponentiates the two chunks from the same registers and writes
        // P (hi, lo) over them. Precision is
        // chosen per 16-row query tile, so a warp (32 rows) can mix INT8 and
        // FP16 chunks: per-lane differences are selects, branches are on
        // warp votes.
        const int half = warp >> 2;                                  // key half of every block
        const int row = (warp & 3) * 32 + static_cast<int>(lane);    // TMEM lane = query row
        const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
        const int q_row = qt * kTileRows + row;
        const bool row_valid = q_row < p.M;
        const int q16 = qt * (kTileRows / 16) + row / 16;
        const bool q16_valid = q16 < p.q16_tiles;
        float q_scale = 0.0f;
        bool ok = true;
        if (p.routed) {
            if (p.fuse_q) {
                ok = quantize_q_tile<kAtoms>(p, smem, bar(kBarQFull), bar(kBarQ8Ready), head, qt, abort_flag, q_scale);
            } else {
                q_scale = __half2float(p.q_scales[head * p.q_scale_blocks + qt]);
            }
        }
        // Scores are kept in "raw" units r with score_log2 = r * c_exp: FP16
        // tiles give r = q.k directly when score_scale > 0 (no multiply); INT8
        // tiles give r = dot * q_scale * k_scale.
        const bool pos_scale = p.scale_log2 > 0.0f;
        const float c_exp = pos_scale ? p.scale_log2 : 1.0f;
        const float a_f16 = pos_scale ? 1.0f : p.scale_log2;
        const float threshold = kRescaleLog2 / c_exp;
        const RouteSlot* ring = reinterpret_cast<const RouteSlot*>(smem + L::kRoute);
        const int qlocal = row / 16;
        float m_run = -INFINITY;    // running max (raw units), possibly stale by < 2^15 in p
        float l_run = 0.0f;         // this half's share of the row sum
        const uint32_t o_addr = tmem + lane_base + kColO + 128u * half;     // O_h
        float* alpha_slots = reinterpret_cast<float*>(smem + L::kAlpha);
        volatile std::uint64_t* xchg = reinterpret_cast<volatile std::uint64_t*>(smem + L::kXchg);
        const int me = static_cast<int>(threadIdx.x);
        uint32_t xa[32], xb[32];
        // Routing of the next block (this half's two INT8 bits and its INT8
        // score ratio) is read and decoded while the current block is being
        // exponentiated, so the loop top only waits for S.
        uint32_t n_types = 0;
        float n_ratio = 0.0f;
        bool n_single = false;
        auto decode = [&](int jb) {
            const RouteSlot sl = ring[jb % kRouteSlots];
            if (kPvHint) n_single = (sl.single >> half) & 1u;
            n_types = q16_valid ? (((sl.pats >> (16 * half + qlocal)) & 1u) |
                                   (((sl.pats >> (16 * half + 8 + qlocal)) & 1u) << 1)) : 0u;
            const uint32_t sc = half ? sl.scales >> 16 : sl.scales & 0xffffu;
            n_ratio = q_scale * __half2float(__ushort_as_half(static_cast<unsigned short>(sc))) * a_f16;
        };
        if (ok && nblk > 0) {
            ok = wait_bar(bar(kBarRoute), 0, abort_flag, kStatusSoftmax);
            if (ok) decode(0);
        }
        bool s_ready = false;
        for (int j = 0; ok && j < nblk; ++j) {
            const int b = j & 1;
            const uint32_t s_row = tmem + lane_base + col_s(b);
            const uint32_t s_own = s_row + 64u * half;
            uint32_t types = n_types;          // bit c: chunk c of this half is INT8
            const float ratio = n_ratio;
            const bool single = kPvHint && n_single;      // this half's P as one fp16 term
            const int key0 = j * kTileKeys;
            const int limit = p.causal ? min(p.N, q_row + 1) : p.N;
            // fast: no key of the block is masked for any row of the warp and
            // score_scale > 0, so FP16 raw units are the accumulator values.
            const bool fast = __all_sync(0xffffffffu, pos_scale && key0 + kTileKeys <= limit);
            if (!s_ready && !wait_bar(bar(kBarSFull + 2 * b + half), (j >> 1) & 1, abort_flag, kStatusSoftmax)) {
                ok = false;
                break;
            }
            tc_fence_after();
            // ---- this half's two 32-key chunks
            tmem_ld32(s_own, xa);
            tmem_ld32(s_own + 32, xb);
            tc_wait_ld();
            if (kTrace && row_valid) {
                // Debug outputs (routing bits, INT32 dots) from the raw accumulators.
                #pragma unroll
                for (int c = 0; c < 2; ++c) {
                    const uint32_t (&x)[32] = c ? xb : xa;
                    const bool is_i8 = (types >> c) & 1u;
                    const int k0 = key0 + 64 * half + 32 * c;
                    if (p.score_dots && is_i8) {
                        for (int i = 0; i < 32; ++i) {
                            if (k0 + i < p.N) {
                                p.score_dots[(static_cast<std::size_t>(head) * p.M + q_row) * p.N + k0 + i] =
                                    static_cast<int32_t>(x[i] - 0x4B400000u);   // accumulators carry the bias
                            }
                        }
                    }
                    const int gkt = 4 * j + 2 * half + c;
                    if (p.decoded_bits && row % 16 == 0 && q16_valid && gkt < p.k32_tiles) {
                        p.decoded_bits[(static_cast<std::size_t>(head) * p.q16_tiles + q16) * p.k32_tiles + gkt] =
                            static_cast<uint8_t>(is_i8);
                    }
                }
            }
            if (!fast) {
                // Rare: edge blocks or score_scale <= 0. Rewrite both chunks as
                // raw-unit floats with masked keys at -inf; they then go through
                // the FP16 (float) path below.
                #pragma unroll
                for (int c = 0; c < 2; ++c) {
                    uint32_t (&x)[32] = c ? xb : xa;
                    const bool is_i8 = (types >> c) & 1u;
                    const float subf = is_i8 ? 12582912.0f : 0.0f;
                    const float mul = is_i8 ? ratio : a_f16;
                    const int k0 = key0 + 64 * half + 32 * c;
                    #pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        const float r = (__uint_as_float(x[i]) - subf) * mul;
                        x[i] = __float_as_uint(k0 + i >= limit ? -INFINITY : r);
                    }
                }
                types = 0;
            }
            // INT8 chunks become exact floats in place: their accumulators
            // hold the float bits of 1.5 * 2^23 + dot (|dot| <= 127^2 * 128 <
            // 2^22), so one subtraction leaves the dot; the max and the
            // exponent below are then one code path for both precisions. FP16
            // lanes of a mixed warp pass through unchanged.
            #pragma unroll
            for (int c = 0; c < 2; ++c) {
                uint32_t (&x)[32] = c ? xb : xa;
                const bool is_i8 = (types >> c) & 1u;
                if (__any_sync(0xffffffffu, is_i8)) {
                    const float subf = is_i8 ? 12582912.0f : 0.0f;
                    const float2 nsub = make_float2(-subf, -subf);
                    #pragma unroll
                    for (int i = 0; i < 32; i += 2) {
                        const float2 t = __fadd2_rn(make_float2(__uint_as_float(x[i]), __uint_as_float(x[i + 1])), nsub);
                        x[i] = __float_as_uint(t.x);
                        x[i + 1] = __float_as_uint(t.y);
                    }
                }
            }
            const float mul0 = ((types & 1u) ? ratio : 1.0f) * c_exp;   // score_log2 = x * mul
            const float mul1 = ((types & 2u) ? ratio : 1.0f) * c_exp;
            // next block's routing: probe now, decode alongside the exponent
            bool r_ready = true;
            if (j + 1 < nblk) {
                r_ready = mbar_test_wait(bar(kBarRoute + (j + 1) % kRouteSlots), ((j + 1) / kRouteSlots) & 1);
                if (r_ready) decode(j + 1);
            }
            // ---- this half's max; the running max moves only when the block
            // exceeds it by more than 2^15 in p. The factor for O_h goes to
            // the rescale warp of these rows, which applies it once the
            // previous block's PV has landed, while this warp exponentiates.
            float rescale = 1.0f;
            {
                float m0 = max3f(__uint_as_float(xa[0]), __uint_as_float(xa[1]), __uint_as_float(xa[2]));
                float m1 = max3f(__uint_as_float(xb[0]), __uint_as_float(xb[1]), __uint_as_float(xb[2]));
                #pragma unroll
                for (int i = 3; i < 31; i += 2) {
                    m0 = max3f(m0, __uint_as_float(xa[i]), __uint_as_float(xa[i + 1]));
                    m1 = max3f(m1, __uint_as_float(xb[i]), __uint_as_float(xb[i + 1]));
                }
                m0 = fmaxf(m0, __uint_as_float(xa[31]));
                m1 = fmaxf(m1, __uint_as_float(xb[31]));
                // raw units: INT8 chunks scale by their (non-negative) ratio
                const float bm = fmaxf((types & 1u) ? m0 * ratio : m0, (types & 2u) ? m1 * ratio : m1);
                float alpha = 1.0f;
                if (bm > m_run + threshold) {            // also true when m_run is -inf
                    alpha = ex2((m_run - bm) * c_exp);   // 0 when m_run is -inf
                    m_run = bm;
                }
                l_run *= alpha;
                rescale = alpha;
            }
            alpha_slots[(2 * b + half) * kTileRows + row] = rescale;
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(kBarAlpha + 4 * (2 * b + half) + (warp & 3)));   // release
            const float neg_m = m_run == -INFINITY ? 0.0f : -m_run * c_exp;
            // ---- P = 2^(score_log2 - m) as P_hi + P_lo, both fp16. P_hi keeps
            // the top 11 significant bits of p (exact in fp16), P_lo = p - P_hi
            // (exact) rounded to fp16; the two PV MMAs make the product
            // accurate to ~2^-22 relative instead of fp16's 2^-11, which the
            // parity tolerance needs once V has large-magnitude (outlier)
            // channels. Chunk c's P_hi goes to its columns [32c, 32c+16), P_lo
            // to [32c+16, 32c+32).
            // Element pairs go through the packed f32x2 FMA/add (one instruction
            // per pair, rounding exactly like the scalar forms).
            float2 s01 = make_float2(0.0f, 0.0f), s23 = make_float2(0.0f, 0.0f);
            const float2 nm2 = make_float2(neg_m, neg_m);
            const float2 minus1 = make_float2(-1.0f, -1.0f);
            if (single) {
                // every |v| of this half is small: P rounded once to fp16
                // (P_hi columns only; PV runs one MMA per K step)
                #pragma unroll
                for (int c = 0; c < 2; ++c) {
                    const uint32_t (&x)[32] = c ? xb : xa;
                    const float mul = c ? mul1 : mul0;
                    const float2 mul2 = make_float2(mul, mul);
                    float2 arg[16];
                    #pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        arg[i] = __ffma2_rn(make_float2(__uint_as_float(x[2 * i]), __uint_as_float(x[2 * i + 1])),
                                            mul2, nm2);
                    }
                    uint32_t hi[16];
                    #pragma unroll
                    for (int i = 0; i < 16; i += 2) {
                        const float2 p01 = make_float2(ex2(arg[i].x), ex2(arg[i].y));
                        const float2 p23 = make_float2(ex2(arg[i + 1].x), ex2(arg[i + 1].y));
                        s01 = __fadd2_rn(s01, p01);
                        s23 = __fadd2_rn(s23, p23);
                        hi[i] = pack_half2(p01.x, p01.y);
                        hi[i + 1] = pack_half2(p23.x, p23.y);
                    }
                    tmem_st16(s_own + 32 * c, hi);
                }
            } else {
                #pragma unroll
                for (int c = 0; c < 2; ++c) {
                    const uint32_t (&x)[32] = c ? xb : xa;
                    const float mul = c ? mul1 : mul0;
                    const float2 mul2 = make_float2(mul, mul);
                    float2 arg[16];
                    #pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        arg[i] = __ffma2_rn(make_float2(__uint_as_float(x[2 * i]), __uint_as_float(x[2 * i + 1])),
                                            mul2, nm2);
                    }
                    uint32_t hi[16], lo[16];
                    #pragma unroll
                    for (int i = 0; i < 16; i += 2) {
                        const float2 p01 = make_float2(ex2(arg[i].x), ex2(arg[i].y));
                        const float2 p23 = make_float2(ex2(arg[i + 1].x), ex2(arg[i + 1].y));
                        s01 = __fadd2_rn(s01, p01);
                        s23 = __fadd2_rn(s23, p23);
                        const float2 h01 = make_float2(__uint_as_float(__float_as_uint(p01.x) & 0xFFFFE000u),
                                                       __uint_as_float(__float_as_uint(p01.y) & 0xFFFFE000u));
                        const float2 h23 = make_float2(__uint_as_float(__float_as_uint(p23.x) & 0xFFFFE000u),
                                                       __uint_as_float(__float_as_uint(p23.y) & 0xFFFFE000u));
                        hi[i] = pack_half2(h01.x, h01.y);
                        hi[i + 1] = pack_half2(h23.x, h23.y);
                        const float2 l01 = __ffma2_rn(h01, minus1, p01);      // p - P_hi, exact
                        const float2 l23 = __ffma2_rn(h23, minus1, p23);
                        lo[i] = pack_half2(l01.x, l01.y);
                        lo[i + 1] = pack_half2(l23.x, l23.y);
                    }
                    tmem_st16(s_own + 32 * c, hi);
                    tmem_st16(s_own + 32 * c + 16, lo);
                }
            }
            l_run += (s01.x + s01.y) + (s23.x + s23.y);
            s_ready = j + 1 < nblk && mbar_test_wait(bar(kBarSFull + 2 * (b ^ 1) + half), ((j + 1) >> 1) & 1);
            tc_wait_st();
            tc_fence_before();
            __syncwarp();
            // Watchdog self-test only: softmax warp 0 withholds its first
            // P-ready arrival, so the MMA warp of key half 0 waits in vain.
            const bool withheld = kWithholdArrive && j == 0 && warp == 0;
            if (lane == 0 && !withheld) mbar_arrive(bar(kBarPFull + 2 * b + half));
            if (!__all_sync(0xffffffffu, r_ready)) {
                if (!wait_bar(bar(kBarRoute + (j + 1) % kRouteSlots), ((j + 1) / kRouteSlots) & 1, abort_flag,
                              kStatusSoftmax)) {
                    ok = false;
                    break;
                }
                decode(j + 1);
            }
            s_ready = __all_sync(0xffffffffu, s_ready);
        }
        // ---- epilogue: combine the two halves of the row; this thread writes
        // output columns [64h, 64h + 64)
        if (ok && nblk > 0) {
            float m_oth = 0.0f, l_oth = 0.0f;
            ok = pair_exchange(xchg + kSoftmaxThreads, me, 1u, m_run, m_oth, abort_flag) &&
                 pair_exchange(xchg, me, 2u, l_run, l_oth, abort_flag);
            // the combine reads both halves' accumulators
            const int bl = (nblk - 1) & 1;
            if (ok && wait_bar(bar(kBarPvDone + 2 * bl), ((nblk - 1) >> 1) & 1, abort_flag, kStatusSoftmax) &&
                wait_bar(bar(kBarPvDone + 2 * bl + 1), ((nblk - 1) >> 1) & 1, abort_flag, kStatusSoftmax)) {
                tc_fence_after();
                const float m = fmaxf(m_run, m_oth);
                const float a_me = m_run == -INFINITY ? 0.0f : ex2((m_run - m) * c_exp);
                const float a_oth = m_oth == -INFINITY ? 0.0f : ex2((m_oth - m) * c_exp);
                const float l_row = l_run * a_me + l_oth * a_oth;
                const float inv_l = 1.0f / l_row;
                // log2 of the row's sum of 2^(score_scale log2(e) q.k): the
                // statistic the backward pass recomputes P from
                if (p.lse_out && half == 0 && row_valid) {
                    p.lse_out[static_cast<std::size_t>(head) * p.M + q_row] = m * c_exp + log2f(l_row);
                }
                const float w_me = a_me * inv_l, w_oth = a_oth * inv_l;
                const uint32_t o_oth = tmem + lane_base + kColO + 128u * (half ^ 1);
                // fp32 O in [heads][M][d], or the strided output's row
                float* out = p.o + (static_cast<std::size_t>(head) * p.M + q_row) * p.d;
                long long row_off = 0;
                if (kStrided) {
                    const int hb = head / p.o_hpb;
                    row_off = hb * p.o_sb + (head - hb * p.o_hpb) * p.o_sh + static_cast<long long>(q_row) * p.o_sm;
                }
                #pragma unroll 1
                for (int c = 64 * half; c < 64 * half + 64 && c < p.pv_n; c += 32) {
                    tmem_ld32(o_addr + c, xa);
                    tmem_ld32(o_oth + c, xb);
                    tc_wait_ld();
                    // explicit roundings, so every output variant stores (a
                    // rounding of) the same fp32 value
                    const float2 w_me2 = make_float2(w_me, w_me), w_oth2 = make_float2(w_oth, w_oth);
                    #pragma unroll
                    for (int i = 0; i < 32; i += 2) {
                        const float2 t = __fmul2_rn(make_float2(__uint_as_float(xb[i]), __uint_as_float(xb[i + 1])),
                                                    w_oth2);
                        const float2 o = __ffma2_rn(make_float2(__uint_as_float(xa[i]), __uint_as_float(xa[i + 1])),
                                                    w_me2, t);
                        xa[i] = __float_as_uint(o.x);
                        xa[i + 1] = __float_as_uint(o.y);
                    }
                    if (kStrided) {
                        if (row_valid) store_strided_row(p, row_off, c, xa);
                    } else if (p.o_tma) {
                        // Coalesced output: the warp stages its 32 rows x 32
                        // columns in shared memory (the K stages: every MMA has
                        // completed), 128-byte swizzled as the TMA store
                        // expects, and one lane stores the box.
                        const uint32_t box_off = L::kK + static_cast<uint32_t>(c >> 5) * 16384u +
                                                 static_cast<uint32_t>(warp & 3) * 4096u;
                        #pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const uint32_t off = box_off + lane * 128u + ((static_cast<uint32_t>(i) ^ (lane & 7u)) << 4);
                            *reinterpret_cast<uint4*>(smem + off) = make_uint4(xa[4 * i], xa[4 * i + 1], xa[4 * i + 2],
                                                                               xa[4 * i + 3]);
                        }
                        fence_proxy_async_smem();
                        __syncwarp();
                        const int y0 = qt * kTileRows + (warp & 3) * 32;
                        if (lane == 0 && y0 < p.M && c < p.d) tma_store_3d(&tm_o, sbase + box_off, c, y0, head);
                    } else if (row_valid) {
                        if (p.o_vec) {
                            #pragma unroll
                            for (int i = 0; i < 32; i += 4) {
                                if (c + i < p.d) {
                                    reinterpret_cast<float4*>(out + c + i)[0] = make_float4(
                                        __uint_as_float(xa[i]), __uint_as_float(xa[i + 1]),
                                        __uint_as_float(xa[i + 2]), __uint_as_float(xa[i + 3]));
                                }
                            }
                        } else {
                            #pragma unroll
                            for (int i = 0; i < 32; ++i) {
                                if (c + i < p.d) out[c + i] = __uint_as_float(xa[i]);
                            }
                        }
                    }
                }
                if (!kStrided && p.o_tma && lane == 0) {
                    // the stores must have read shared memory before the CTA exits
                    bulk_commit_group();
                    bulk_wait_group_read0();
                }
            }
        }
    } else {
        reg_dealloc<kCorrRegs>();
        // ------------------------------------------------------------ rescale
        // Warp w owns TMEM lanes 32*(w%4).. (the rows of softmax warps w%4 and
        // w%4 + 4). Per block and key half: wait for the rows' factors; if any
        // is not 1, wait for the previous block's PV of that half to land,
        // then scale O_h in place. Its arrival on P-full (with the softmax
        // warps') lets the half's PV(j) go ahead.
        const int quarter = warp & 3;
        const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
        const float* alpha_slots = reinterpret_cast<const float*>(smem + L::kAlpha);
        uint32_t xa[32], xb[32];
        bool ok = true;
        for (int j = 0; ok && j < nblk; ++j) {
            const int b = j & 1;
            #pragma unroll 1
            for (int h = 0; h < 2; ++h) {
                if (!wait_bar(bar(kBarAlpha + 4 * (2 * b + h) + quarter), (j >> 1) & 1, abort_flag, kStatusSoftmax)) {
                    ok = false;
                    break;
                }
                const float alpha = alpha_slots[(2 * b + h) * kTileRows + quarter * 32 + static_cast<int>(lane)];
                if (j > 0 && __any_sync(0xffffffffu, alpha != 1.0f)) {
                    if (!wait_bar(bar(kBarPvDone + 2 * ((j - 1) & 1) + h), ((j - 1) >> 1) & 1, abort_flag,
                                  kStatusSoftmax)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t o_addr = tmem + lane_base + kColO + 128u * h;
                    const float2 a2 = make_float2(alpha, alpha);
                    // 64 columns per round trip
                    #pragma unroll 1
                    for (int c = 0; c < p.pv_n; c += 64) {
                        tmem_ld32(o_addr + c, xa);
                        tmem_ld32(o_addr + c + 32, xb);
                        tc_wait_ld();
                        #pragma unroll
                        for (int i = 0; i < 32; i += 2) {
                            const float2 ta = __fmul2_rn(make_float2(__uint_as_float(xa[i]), __uint_as_float(xa[i + 1])), a2);
                            const float2 tb = __fmul2_rn(make_float2(__uint_as_float(xb[i]), __uint_as_float(xb[i + 1])), a2);
                            xa[i] = __float_as_uint(ta.x);
                            xa[i + 1] = __float_as_uint(ta.y);
                            xb[i] = __float_as_uint(tb.x);
                            xb[i + 1] = __float_as_uint(tb.y);
                        }
                        tmem_st32(o_addr + c, xa);
                        tmem_st32(o_addr + c + 32, xb);
                    }
                    tc_wait_st();
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(bar(kBarPFull + 2 * b + h));
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// ------------------------------------------------------------------- host side
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult status;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &status) == cudaSuccess &&
            status == cudaDriverEntryPointSuccess) {
            fn = reinterpret_cast<EncodeTiledFn>(ptr);
        }
    });
    return fn;
}

// 3-D map over [heads][rows][d] with a 128-byte-swizzled {box_x, 128, 1} box.
bool encode_map(CUtensorMap* map, const void* base, CUtensorMapDataType type, int elem_bytes,
                int heads, int rows, int d, int box_x, int box_y = 128) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(d), static_cast<cuuint64_t>(rows),
                                static_cast<cuuint64_t>(heads)};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(d) * elem_bytes,
                                   static_cast<cuuint64_t>(rows) * d * elem_bytes};
    const cuuint32_t box[3] = {static_cast<cuuint32_t>(box_x), static_cast<cuuint32_t>(box_y), 1u};
    const cuuint32_t elem_strides[3] = {1u, 1u, 1u};
    return fn(map, type, 3, const_cast<void*>(base), dims, strides, box, elem_strides,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int kAtoms, bool kUseTma, bool kTrace, bool kStrided = false, bool kWithholdArrive = false,
          bool kPvHint = false>
cudaError_t launch_variant(const CUtensorMap* maps, const Params& p, unsigned grid, cudaStream_t stream) {
    auto kernel = tilemix_attention_kernel<kAtoms, kUseTma, kTrace, kStrided, kWithholdArrive, kPvHint>;
    const int smem = static_cast<int>(SmemLayout<kAtoms>::kBytes);
    // The opt-in attribute is per device; set it the first time a device is seen.
    static int configured[64] = {0};
    int device = 0;
    cudaError_t status = cudaGetDevice(&device);
    if (status != cudaSuccess) return status;
    if (device < 0 || device >= 64) return cudaErrorInvalidDevice;
    if (!configured[device]) {
        status = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (status != cudaSuccess) return status;
        configured[device] = 1;
    }
    kernel<<<grid, kAttnThreads, smem, stream>>>(maps[0], maps[1], maps[2], maps[3], maps[4], maps[5], p);
    return cudaGetLastError();
}

// SM count of the current device, queried once per device.
cudaError_t sm_count(int* out) {
    static int cached[64] = {0};
    int device = 0;
    cudaError_t status = cudaGetDevice(&device);
    if (status != cudaSuccess) return status;
    if (device < 0 || device >= 64) return cudaErrorInvalidDevice;
    if (cached[device] == 0) {
        int n = 0;
        status = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device);
        if (status != cudaSuccess) return status;
        cached[device] = n > 0 ? n : 1;
    }
    *out = cached[device];
    return cudaSuccess;
}

bool aligned16(const void* ptr) {
    return (reinterpret_cast<std::uintptr_t>(ptr) & 15u) == 0;
}

}  // namespace

std::size_t attention_smem_bytes(int d) {
    if (d <= 0 || d > kMaxHeadDim) return 0;
    return d <= 64 ? SmemLayout<1>::kBytes : SmemLayout<2>::kBytes;
}

cudaError_t launch_attention(const AttentionProblem& prob, cudaStream_t stream) {
    Params p{};
    p.q = prob.q; p.k = prob.k; p.v = prob.v;
    p.q8 = prob.q8; p.k8 = prob.k8;
    p.q_scales = prob.q_scales; p.k_scales = prob.k_scales;
    p.o = prob.o;
    p.words = prob.words;
    p.decoded_bits = prob.decoded_bits;
    p.score_dots = prob.score_dots;
    p.heads = prob.heads; p.M = prob.M; p.N = prob.N; p.d = prob.d;
    p.q_tiles = (prob.M - 1) / kTileRows + 1;
    p.kv_blocks = (prob.N - 1) / kTileKeys + 1;
    p.q16_tiles = (prob.M - 1) / 16 + 1;
    p.k32_tiles = (prob.N - 1) / 32 + 1;
    // Group sizes beyond the key-tile count behave like one group per row.
    p.group = std::min(prob.key_tiles_per_group, p.k32_tiles);
    const long long groups = (p.k32_tiles - 1) / prob.key_tiles_per_group + 1;
    p.words_per_row = static_cast<int>((groups - 1) / 64 + 1);
    p.words_per_head = static_cast<long long>(p.q16_tiles) * p.words_per_row;
    p.q_scale_blocks = (prob.M - 1) / kQuantQRows + 1;
    p.k_scale_blocks = (prob.N - 1) / kQuantKRows + 1;
    p.scale_log2 = prob.score_scale * kLog2e;
    p.causal = prob.causal ? 1 : 0;
    p.routed = prob.words != nullptr ? 1 : 0;
    p.fuse_q = prob.fuse_q ? 1 : 0;
    p.v_absmax = prob.v_absmax;
    p.q8_out = prob.q8_out;
    p.q_scales_out = prob.q_scales_out;
    p.lse_out = prob.lse_out;
    p.q8_vec = (prob.d % 16 == 0 && aligned16(prob.q8_out)) ? 1 : 0;
    p.f16_ksteps = (prob.d + 15) / 16;
    p.i8_ksteps = (prob.d + 31) / 32;
    p.pv_n = (prob.d + 15) / 16 * 16;
    p.o_vec = (prob.d % 4 == 0 && aligned16(prob.o)) ? 1 : 0;
    const bool strided = prob.o_data != nullptr;
    if (strided) {
        p.o_data = prob.o_data;
        p.o_dtype = prob.o_dtype;
        p.o_hpb = prob.o_heads_per_batch;
        p.o_sb = prob.o_stride_batch;
        p.o_sh = prob.o_stride_head;
        p.o_sm = prob.o_stride_row;
        // 16-byte stores need the base, every stride and d in 16-byte units
        const long long unit = prob.o_dtype == 0 ? 4 : 8;     // elements per 16 bytes
        p.o_vec = (prob.d % unit == 0 && p.o_sb % unit == 0 && p.o_sh % unit == 0 && p.o_sm % unit == 0 &&
                   aligned16(prob.o_data)) ? 1 : 0;
    }
    p.wait_limit_ns = prob.watchdog_test ? prob.watchdog_limit_ns : kWaitLimitNs;
    p.head_group = std::min(prob.heads, 8);
    const cudaError_t sm_status = sm_count(&p.prefetch_ahead);
    if (sm_status != cudaSuccess) return sm_status;

    const long long grid = static_cast<long long>(p.q_tiles) * p.heads;
    if (grid > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
    const int atoms = prob.d <= 64 ? 1 : 2;
    const bool trace = prob.decoded_bits != nullptr || prob.score_dots != nullptr;

    CUtensorMap maps[6];
    std::memset(maps, 0, sizeof(maps));
    const bool q8_in = p.routed && !p.fuse_q;
    bool tma = prob.d % 16 == 0 && aligned16(prob.q) && aligned16(prob.k) && aligned16(prob.v) &&
               (!p.routed || (aligned16(prob.k8) && (!q8_in || aligned16(prob.q8))));
    if (tma) {
        tma = encode_map(&maps[0], prob.q, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, p.heads, p.M, p.d, 64) &&
              encode_map(&maps[1], prob.k, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, p.heads, p.N, p.d, 64) &&
              encode_map(&maps[2], prob.v, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, p.heads, p.N, p.d, 64);
        if (tma && q8_in) {
            tma = encode_map(&maps[3], prob.q8, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, p.heads, p.M, p.d, 128);
        }
        if (tma && p.routed) {
            tma = encode_map(&maps[4], prob.k8, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, p.heads, p.N, p.d, 128);
        }
    }
    // fp32 O by TMA stores of 32 x 32 boxes (128-byte rows, swizzled)
    p.o_tma = (!strided && prob.d % 32 == 0 && aligned16(prob.o) &&
               encode_map(&maps[5], prob.o, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, p.heads, p.M, p.d, 32, 32)) ? 1 : 0;
    const unsigned g = static_cast<unsigned>(grid);
    if (prob.v_absmax && tma && !strided && !trace && !prob.watchdog_test) {
        // precision hints: the instantiation with per-half single-term P
        return atoms == 1 ? launch_variant<1, true, false, false, false, true>(maps, p, g, stream)
                          : launch_variant<2, true, false, false, false, true>(maps, p, g, stream);
    }
    p.v_absmax = nullptr;   // the other builds keep two-term P everywhere
    if (prob.watchdog_test) {
        // The self-test instantiation exists for d = 65..128 with TMA, fp32
        // output, no routing trace outputs.
        if (atoms != 2 || !tma || strided || trace) return cudaErrorNotSupported;
        return launch_variant<2, true, false, false, true>(maps, p, g, stream);
    }
    if (strided) {
        // strided outputs carry no trace outputs (checked by the API layer)
        if (atoms == 1) return tma ? launch_variant<1, true, false, true>(maps, p, g, stream)
                                   : launch_variant<1, false, false, true>(maps, p, g, stream);
        return tma ? launch_variant<2, true, false, true>(maps, p, g, stream)
                   : launch_variant<2, false, false, true>(maps, p, g, stream);
    }
    if (atoms == 1) {
        if (tma) return trace ? launch_variant<1, true, true>(maps, p, g, stream)
                              : launch_variant<1, true, false>(maps, p, g, stream);
        return trace ? launch_variant<1, false, true>(maps, p, g, stream)
                     : launch_variant<1, false, false>(maps, p, g, stream);
    }
    if (tma) return trace ? launch_variant<2, true, true>(maps, p, g, stream)
                          : launch_variant<2, true, false>(maps, p, g, stream);
    return trace ? launch_variant<2, false, true>(maps, p, g, stream)
                 : launch_variant<2, false, false>(maps, p, g, stream);
}

cudaError_t read_and_clear_status(unsigned int* status) {
    unsigned int zero = 0;
    cudaError_t err = cudaDeviceSynchronize();
    if (err != cudaSuccess) return err;
    err = cudaMemcpyFromSymbol(status, g_tilemix_status, sizeof(unsigned int));
    if (err != cudaSuccess) return err;
    err = cudaMemcpyToSymbol(g_tilemix_status, &zero, sizeof(unsigned int));
    if (err != cudaSuccess) return err;
    unsigned int backward = 0;
    err = read_and_clear_backward_status(&backward);
    *status |= backward;
    return err;
}

}  // namespace tilemix
