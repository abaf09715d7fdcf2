// Thin inline-PTX wrappers for the sm_100a features the TileMix kernels use:
// mbarriers (with bounded waits), TMA tiled loads, tcgen05 TMEM allocation,
// MMA (kind::f16 / kind::i8, SMEM or TMEM A operand, per-lane output masks),
// commit, and TMEM loads/stores. Written against the public PTX ISA.
#pragma once

#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ != 1000)
#error "libtilemix_b200 is built for sm_100a only"
#endif

namespace tilemix {
namespace sm100 {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// One lane of the (converged) warp, chosen by elect.sync.
__device__ __forceinline__ bool elect_one() {
    uint32_t pred = 0;
    asm volatile("{\n\t.reg .pred P1;\n\telect.sync _|P1, 0xffffffff;\n\tselp.b32 %0, 1, 0, P1;\n\t}"
                 : "+r"(pred));
    return pred != 0;
}

__device__ __forceinline__ uint32_t lane_id() {
    uint32_t lane;
    asm volatile("mov.u32 %0, %%laneid;" : "=r"(lane));
    return lane;
}

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ------------------------------------------------------------------ mbarrier
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_init_fence() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("{\n\t.reg .b64 st;\n\t"
                 "mbarrier.arrive.shared::cta.b64 st, [%0];\n\t}"
                 :: "r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\t"
                 "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}"
                 :: "r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(done) : "r"(bar), "r"(parity) : "memory");
    return done != 0;
}

// Non-blocking probe: true if the phase with this parity has completed
// (acquire semantics, like a successful wait).
__device__ __forceinline__ bool mbar_test_wait(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(done) : "r"(bar), "r"(parity) : "memory");
    return done != 0;
}

// As mbar_try_wait, but a thread whose phase is not complete is suspended
// (it does not spin and steal issue slots) until the phase completes or about
// `suspend_ns` nanoseconds pass.
__device__ __forceinline__ bool mbar_try_wait_suspend(uint32_t bar, uint32_t parity, uint32_t suspend_ns) {
    uint32_t done;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(done) : "r"(bar), "r"(parity), "r"(suspend_ns) : "memory");
    return done != 0;
}

// Generic-proxy smem writes -> visible to the async proxy (TMA / tensor core).
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ----------------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const void* tmap, uint32_t bar,
                                            int x, int y, int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5}], [%2];"
        :: "r"(dst), "l"(reinterpret_cast<uint64_t>(tmap)), "r"(bar), "r"(x), "r"(y), "r"(z)
        : "memory");
}

// Tiled TMA store shared -> global (bulk-group completion). Coordinates must
// be non-negative; rows / columns past the tensor's extent are not written.
__device__ __forceinline__ void tma_store_3d(const void* tmap, uint32_t src, int x, int y, int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];"
        :: "l"(reinterpret_cast<uint64_t>(tmap)), "r"(src), "r"(x), "r"(y), "r"(z)
        : "memory");
}

__device__ __forceinline__ void bulk_commit_group() {
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Wait until every committed bulk store of this thread has finished reading
// its shared-memory source.
__device__ __forceinline__ void bulk_wait_group_read0() {
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

// L2 prefetch of one tiled box (no shared-memory destination, no completion).
__device__ __forceinline__ void tma_prefetch_l2_3d(const void* tmap, int x, int y, int z) {
    asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];"
                 :: "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(z) : "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const void* tmap) {
    asm volatile("prefetch.tensormap [%0];" :: "l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

// ------------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 :: "r"(dst_smem), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;"
                 :: "r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tc_wait_st() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Arrives once on `bar` when every tcgen05 op previously issued by this thread
// has completed.
__device__ __forceinline__ void tc_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 :: "r"(bar) : "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]; lanes whose bit is set in
// `disabled` (bit i of word i/32 = TMEM lane i) are not written.
__device__ __forceinline__ void mma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                           uint32_t idesc, const uint32_t (&disabled)[4],
                                           uint32_t accumulate) {
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
                 :: "r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate),
                    "r"(disabled[0]), "r"(disabled[1]), "r"(disabled[2]), "r"(disabled[3])
                 : "memory");
}

__device__ __forceinline__ void mma_i8_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                          uint32_t idesc, const uint32_t (&disabled)[4],
                                          uint32_t accumulate) {
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
                 :: "r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate),
                    "r"(disabled[0]), "r"(disabled[1]), "r"(disabled[2]), "r"(disabled[3])
                 : "memory");
}

// Lean issue forms for hot loops: the 64-bit shared-memory descriptors are
// passed as their two 32-bit words (the low word holds the start address and
// the leading byte offset, so stepping through a tile is one 32-bit add), and
// the accumulate flag is a compile-time constant where the caller knows it.
template <int kAccumulate>
__device__ __forceinline__ void mma_f16_ss_w(uint32_t d_tmem, uint32_t a_lo, uint32_t b_lo, uint32_t desc_hi,
                                             uint32_t idesc, const uint32_t (&disabled)[4]) {
    asm volatile("{\n\t.reg .pred p;\n\t.reg .b64 a, b;\n\t"
                 "setp.ne.b32 p, %5, 0;\n\t"
                 "mov.b64 a, {%1, %3};\n\t"
                 "mov.b64 b, {%2, %3};\n\t"
                 "tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %4, {%6, %7, %8, %9}, p;\n\t}"
                 :: "r"(d_tmem), "r"(a_lo), "r"(b_lo), "r"(desc_hi), "r"(idesc), "n"(kAccumulate),
                    "r"(disabled[0]), "r"(disabled[1]), "r"(disabled[2]), "r"(disabled[3])
                 : "memory");
}

template <int kAccumulate>
__device__ __forceinline__ void mma_i8_ss_w(uint32_t d_tmem, uint32_t a_lo, uint32_t b_lo, uint32_t desc_hi,
                                            uint32_t idesc, const uint32_t (&disabled)[4]) {
    asm volatile("{\n\t.reg .pred p;\n\t.reg .b64 a, b;\n\t"
                 "setp.ne.b32 p, %5, 0;\n\t"
                 "mov.b64 a, {%1, %3};\n\t"
                 "mov.b64 b, {%2, %3};\n\t"
                 "tcgen05.mma.cta_group::1.kind::i8 [%0], a, b, %4, {%6, %7, %8, %9}, p;\n\t}"
                 :: "r"(d_tmem), "r"(a_lo), "r"(b_lo), "r"(desc_hi), "r"(idesc), "n"(kAccumulate),
                    "r"(disabled[0]), "r"(disabled[1]), "r"(disabled[2]), "r"(disabled[3])
                 : "memory");
}

__device__ __forceinline__ void mma_f16_ts_w(uint32_t d_tmem, uint32_t a_tmem, uint32_t b_lo, uint32_t desc_hi,
                                             uint32_t idesc, uint32_t accumulate) {
    asm volatile("{\n\t.reg .pred p;\n\t.reg .b64 b;\n\t"
                 "setp.ne.b32 p, %5, 0;\n\t"
                 "mov.b64 b, {%2, %3};\n\t"
                 "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], b, %4, p;\n\t}"
                 :: "r"(d_tmem), "r"(a_tmem), "r"(b_lo), "r"(desc_hi), "r"(idesc), "r"(accumulate)
                 : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc]  (A is 128 lanes x K fp16, 2 per column).
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                           uint32_t idesc, uint32_t accumulate) {
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
                 :: "r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
                 : "memory");
}

// Instruction descriptor (PTX ISA "Instruction descriptor" table for
// kind::f16 / kind::i8): D format bits [4,6), A format [7,10), B format
// [10,13), A/B major bits 15/16, N>>3 at [17,23), M>>4 at [24,29).
__host__ __device__ constexpr uint32_t idesc_f16_f32(int m, int n, bool b_mn_major) {
    return (1u << 4)                                  // D = f32
         | (0u << 7) | (0u << 10)                     // A = B = f16
         | (static_cast<uint32_t>(b_mn_major) << 16)
         | (static_cast<uint32_t>(n >> 3) << 17)
         | (static_cast<uint32_t>(m >> 4) << 24);
}
__host__ __device__ constexpr uint32_t idesc_s8_s32(int m, int n) {
    return (2u << 4)                                  // D = s32
         | (1u << 7) | (1u << 10)                     // A = B = signed 8-bit
         | (static_cast<uint32_t>(n >> 3) << 17)
         | (static_cast<uint32_t>(m >> 4) << 24);
}

// Shared-memory matrix descriptor, 128-byte swizzle (layout type 2 at bits
// [61,64)), descriptor version 1 (bits [46,48)), base offset 0: the operand
// tile must start on a 1024-byte boundary (modulo the K-step byte offset added
// to the start address).
// Its two 32-bit words, for the lean issue forms above.
__host__ __device__ constexpr uint32_t smem_desc_sw128_lo(uint32_t addr, uint32_t lbo_bytes) {
    return ((addr >> 4) & 0x3FFFu) | (((lbo_bytes >> 4) & 0x3FFFu) << 16);
}
__host__ __device__ constexpr uint32_t smem_desc_sw128_hi(uint32_t sbo_bytes) {
    return ((sbo_bytes >> 4) & 0x3FFFu) | (1u << 14) | (2u << 29);
}

__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr, uint32_t lbo_bytes,
                                                    uint32_t sbo_bytes) {
    return static_cast<uint64_t>((addr >> 4) & 0x3FFFu)
         | (static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16)
         | (static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32)
         | (1ull << 46)
         | (2ull << 61);
}

// -------------------------------------------------------------- TMEM ld / st
// 32x32b shape: thread i of the warp accesses TMEM lane (base lane + i); each
// register is one 32-bit column.
#define TILEMIX_R8(p, o) "=r"(p[o + 0]), "=r"(p[o + 1]), "=r"(p[o + 2]), "=r"(p[o + 3]), \
                         "=r"(p[o + 4]), "=r"(p[o + 5]), "=r"(p[o + 6]), "=r"(p[o + 7])
#define TILEMIX_W8(p, o) "r"(p[o + 0]), "r"(p[o + 1]), "r"(p[o + 2]), "r"(p[o + 3]), \
                         "r"(p[o + 4]), "r"(p[o + 5]), "r"(p[o + 6]), "r"(p[o + 7])

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : TILEMIX_R8(r, 0), TILEMIX_R8(r, 8), TILEMIX_R8(r, 16), TILEMIX_R8(r, 24)
        : "r"(taddr) : "memory");
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
        "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};"
        :: "r"(taddr), TILEMIX_W8(r, 0), TILEMIX_W8(r, 8), TILEMIX_W8(r, 16), TILEMIX_W8(r, 24)
        : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : TILEMIX_R8(r, 0), TILEMIX_R8(r, 8) : "r"(taddr) : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* r) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};"
        :: "r"(taddr), TILEMIX_W8(r, 0), TILEMIX_W8(r, 8) : "memory");
}

__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t* r) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};"
        :: "r"(taddr), TILEMIX_W8(r, 0) : "memory");
}

#undef TILEMIX_R8
#undef TILEMIX_W8

// Warpgroup register reallocation (all 128 threads of the warpgroup execute it).
template <int kRegs>
__device__ __forceinline__ void reg_alloc() {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" :: "n"(kRegs));
}
template <int kRegs>
__device__ __forceinline__ void reg_dealloc() {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" :: "n"(kRegs));
}

// 2^x on the MUFU pipe (PTX ex2.approx.ftz.f32; ex2(-inf) = +0).
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Three-input maximum (PTX max.f32 with three sources, sm_100+); like fmaxf, a
// NaN input is ignored when another input is a number.
__device__ __forceinline__ float max3f(float a, float b, float c) {
    float y;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(y) : "f"(a), "f"(b), "f"(c));
    return y;
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);   // .x (low 16 bits) = lo
    return *reinterpret_cast<const uint32_t*>(&h);
}

__device__ __forceinline__ uint32_t pack_bf162(float lo, float hi) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);   // .x (low 16 bits) = lo
    return *reinterpret_cast<const uint32_t*>(&h);
}

}  // namespace sm100
}  // namespace tilemix
