#pragma once
// TileMix drop-in C++ API for the B200 (sm_100a) implementation.
//
// Same names, signatures, default arguments, constants, mask format and
// cudaError_t contract as the reference's include/attention_fused.h:11-72, so
// existing callers (the reference's src/main.cu and its test suite) compile
// and behave unchanged against libtilemix_b200.so. The batched/causal entry
// point at the end is an addition with no reference counterpart.
//
// Error contract (reference src/tilemix.cu:227-236,242-277):
//   cudaErrorInvalidValue        any null/non-positive/non-finite argument,
//                                partial quantized sets, bad routing masks
//   cudaErrorNotSupported        d > kFusedMaxHeadDim (checked after the
//                                InvalidValue checks), or a device that is not
//                                sm_100 (this library carries sm_100a code only)
//   cudaErrorInvalidConfiguration grid / shared-memory limits exceeded
//   otherwise                    the launch status
// All pointers are caller-owned device pointers; the library allocates nothing,
// never writes its inputs and writes exactly M*d output floats. Every call is
// asynchronous on `stream` and uses the calling thread's current device.

#include "matmul_config.h"

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

inline constexpr int kFusedMaxHeadDim = 128;
inline constexpr int kFusedRowThreads = kThreads / kBlockM;
inline constexpr int kTileMixQQuantRows = 128;   // one Q scale per 128 rows x d
inline constexpr int kTileMixKQuantRows = 64;    // one K scale per 64 rows x d
static_assert(kTileMixQQuantRows % kBlockM == 0 && kTileMixKQuantRows % kBlockN == 0);
static_assert(kFusedRowThreads > 0 && (kFusedRowThreads & (kFusedRowThreads - 1)) == 0);

// Shared-memory footprint formulas of the reference's WMMA kernel
// (reference include/attention_fused.h:21-32). Kept with identical values for
// source compatibility; the B200 kernel's own footprint is
// tilemix_b200_shared_bytes().
inline constexpr std::size_t fused_fp16_shared_bytes(int d) {
    if (d <= 0 || d > kFusedMaxHeadDim) return 0;
    const int padded_d = ((d + kTileK - 1) / kTileK) * kTileK;
    return sizeof(__half) * static_cast<std::size_t>(padded_d) * (kBlockM + 2 * kBlockN)
         + sizeof(float) * kBlockM * kBlockN;
}

inline constexpr std::size_t tilemix_shared_bytes(int d, bool quantized) {
    if (d <= 0 || d > kFusedMaxHeadDim) return 0;
    const int padded_d = ((d + kTileK - 1) / kTileK) * kTileK;
    return fused_fp16_shared_bytes(d) + (quantized ? (kBlockM + kBlockN) * padded_d : 0);
}

// Routing mask format (reference include/attention_fused.h:34-45): one bit per
// (16-row query tile, group of key_tiles_per_group 32-key tiles), packed
// LSB-first into uint64 words, ceil(groups/64) words per query tile, query
// tiles row-major. Bit 1 = INT8 scores, bit 0 = FP16 scores.
inline constexpr std::size_t tilemix_routing_words_per_row(int N, int key_tiles_per_group) {
    if (N <= 0 || key_tiles_per_group <= 0) return 0;
    const std::size_t key_tiles = (static_cast<std::size_t>(N) - 1) / kBlockN + 1;
    const std::size_t groups = (key_tiles - 1) / key_tiles_per_group + 1;
    return (groups - 1) / 64 + 1;
}

inline constexpr std::size_t tilemix_routing_word_count(int M, int N, int key_tiles_per_group) {
    if (M <= 0) return 0;
    return ((static_cast<std::size_t>(M) - 1) / kBlockM + 1)
         * tilemix_routing_words_per_row(N, key_tiles_per_group);
}

struct TileMixRouting {
    const std::uint64_t* words = nullptr;   // null = every tile FP16
    std::size_t word_count = 0;
    int key_tiles_per_group = 1;
    std::uint8_t* decoded_bits = nullptr;   // optional trace: [query_tiles][key_tiles] bytes
};

struct TileMixQuantized {
    const std::int8_t* q = nullptr;         // [M, d] from quantize_tilemix_qk
    const std::int8_t* k = nullptr;         // [N, d]
    const __half* q_scales = nullptr;       // [ceil(M/128)]
    const __half* k_scales = nullptr;       // [ceil(N/64)]
    std::int32_t* score_dots = nullptr;     // optional trace: [M, N] raw INT32 dots of INT8 pairs
};

// Stage 1: per-block symmetric INT8 quantization of Q (128-row blocks) and K
// (64-row blocks); scale = absmax/127 in fp32 (stored fp16), values rounded
// half away from zero and clamped to +-127.
cudaError_t quantize_tilemix_qk(const __half* Q, const __half* K,
                                std::int8_t* Q8, std::int8_t* K8,
                                __half* q_scales, __half* k_scales,
                                int M, int N, int d, cudaStream_t stream = nullptr);

// Stages 2-5: routed QK^T (tcgen05 kind::i8 or kind::f16), online softmax,
// fp16 PV MMA and normalisation in one kernel. O is fp32 [M, d].
cudaError_t launch_fused_fp16_attention(const __half* Q, const __half* K, const __half* V,
                                        float* O, int M, int N, int d, float score_scale,
                                        cudaStream_t stream = nullptr,
                                        const TileMixRouting& routing = {},
                                        const TileMixQuantized& quantized = {});

// ---------------------------------------------------------------- additions
// Shared memory the B200 attention kernel requests for head dim d (0 if d is
// out of range).
std::size_t tilemix_b200_shared_bytes(int d, bool quantized);

// Batched quantizer over `heads` contiguous [M,d] / [N,d] slabs
// ([B*H, S, D] layout). Scales are [heads][ceil(M/128)] and [heads][ceil(N/64)].
cudaError_t quantize_tilemix_qk_batched(const __half* Q, const __half* K,
                                        std::int8_t* Q8, std::int8_t* K8,
                                        __half* q_scales, __half* k_scales,
                                        int heads, int M, int N, int d,
                                        cudaStream_t stream = nullptr);

// Batched / causal attention over `heads` contiguous slabs. Per head the
// semantics are exactly launch_fused_fp16_attention's; routing words, scales
// and trace outputs are concatenated per head (routing.word_count covers all
// heads). causal != 0 masks key > query (top-left aligned) and skips key
// tiles that lie wholly above the diagonal.
cudaError_t tilemix_attention_batched(const __half* Q, const __half* K, const __half* V,
                                      float* O, int heads, int M, int N, int d,
                                      float score_scale, bool causal,
                                      cudaStream_t stream = nullptr,
                                      const TileMixRouting& routing = {},
                                      const TileMixQuantized& quantized = {});

// K alone, quantized in 64-row blocks: the same bytes as the K half of
// quantize_tilemix_qk_batched. The K pre-pass of the fused-Q path below.
cudaError_t quantize_tilemix_k_batched(const __half* K, std::int8_t* K8, __half* k_scales,
                                       int heads, int N, int d, cudaStream_t stream = nullptr);

// Routed attention with the Q quantization fused into the attention kernel
// (no reference counterpart; the reference quantizes Q in a separate kernel,
// src/tilemix.cu:223-236). Each CTA's 128-row query tile is one Q quantization
// block (kTileMixQQuantRows), so the CTA quantizes it itself from the fp16 tile
// it loads anyway: one HBM pass over Q fewer. K8 / k_scales come from
// quantize_tilemix_k_batched; routing words are required. Q8_out and
// q_scales_out, when not null, receive exactly the Q8 bytes and fp16 scales
// quantize_tilemix_qk_batched would produce; O equals, bit for bit, the output
// of tilemix_attention_batched given those quantized operands.
cudaError_t tilemix_attention_batched_qfused(const __half* Q, const __half* K, const __half* V, float* O,
                                             int heads, int M, int N, int d, float score_scale, bool causal,
                                             cudaStream_t stream, const TileMixRouting& routing,
                                             const std::int8_t* K8, const __half* k_scales,
                                             std::int8_t* Q8_out = nullptr, __half* q_scales_out = nullptr);

// Precision hints for PV (no reference counterpart; the reference keeps P in
// fp32, src/tilemix.cu:195-210). quantize_tilemix_qkv_batched quantizes Q and
// K exactly as quantize_tilemix_qk_batched and, in the same launch, records
// max |v| of every 64-row block of V in v_absmax [heads][ceil(N/64)] (fp16,
// exact; NaN when the block holds a NaN).
cudaError_t quantize_tilemix_qkv_batched(const __half* Q, const __half* K, const __half* V,
                                         std::int8_t* Q8, std::int8_t* K8, __half* q_scales,
                                         __half* k_scales, __half* v_absmax, int heads, int M, int N,
                                         int d, cudaStream_t stream = nullptr);

// tilemix_attention_batched using those statistics: the PV product of a
// 64-key half-block whose max |v| is <= 3.5 uses P rounded once to fp16 (one
// MMA per K step) instead of the two-term hi + lo split. fp16 rounding moves
// each p by at most 2^-11 p and O = sum p v / sum p, so such a half adds at
// most 2^-11 * 3.5 = 1.7e-3 to any output element, within the 2e-3 parity
// bar; halves with larger |v| keep the two-term P. v_absmax may be null (every
// half two-term, identical to tilemix_attention_batched); layouts the TMA
// build does not take (d % 16 != 0, unaligned bases) and routing trace
// outputs also run two-term everywhere.
cudaError_t tilemix_attention_batched_hinted(const __half* Q, const __half* K, const __half* V,
                                             float* O, int heads, int M, int N, int d,
                                             float score_scale, bool causal, cudaStream_t stream,
                                             const TileMixRouting& routing,
                                             const TileMixQuantized& quantized,
                                             const __half* v_absmax);

// Device-side routing policy (no reference counterpart: the reference takes
// the mask from the caller, src/main.cu:48). Fills `words` (heads *
// tilemix_routing_word_count(M, N, key_tiles_per_group) words, the reference's
// mask format) from the quantizer's block scales: a (16-row query tile, key
// group) pair is INT8 iff q_scale * (max k_scale over the group's 64-row K
// blocks) <= max_scale_product, as an fp32 product; FP16 otherwise (and for
// NaN scales). Since every quantized element is within s / 2 of its value and
// |x| <= 127 s, the INT8 score then differs from the fp32 one by at most
// |score_scale| * d * 127.25 * q_scale * k_scale: choose max_scale_product =
// tolerance / (|score_scale| * d * 127.25) (tilemix_policy_max_scale_product)
// to bound that error by `tolerance`. Outlier blocks (large absmax, coarse
// INT8 steps) therefore stay FP16.
cudaError_t tilemix_routing_policy(const __half* q_scales, const __half* k_scales, std::uint64_t* words,
                                   int heads, int M, int N, int key_tiles_per_group,
                                   float max_scale_product, cudaStream_t stream = nullptr);

inline float tilemix_policy_max_scale_product(float tolerance, float score_scale, int d) {
    const double denom = (score_scale < 0 ? -static_cast<double>(score_scale) : static_cast<double>(score_scale)) *
                         static_cast<double>(d) * 127.25;
    return denom > 0 ? static_cast<float>(static_cast<double>(tolerance) / denom) : 3.4028234663852886e38f;
}

// Output element types of TileMixOutput.
enum TileMixOutputType : int { kTileMixOutF32 = 0, kTileMixOutF16 = 1, kTileMixOutBF16 = 2 };

// A strided output: head h = b * heads_per_batch + hh (of `heads`), row m,
// column c is written at data + b * stride_batch + hh * stride_head +
// m * stride_row + c (strides in elements), rounded to nearest even for fp16
// and bf16. A [B, S, H, D] (BSHD) tensor is heads_per_batch = H,
// stride_batch = S * H * D, stride_head = D, stride_row = H * D.
struct TileMixOutput {
    void* data = nullptr;
    int dtype = kTileMixOutF32;
    int heads_per_batch = 1;
    long long stride_batch = 0;
    long long stride_head = 0;
    long long stride_row = 0;
};

// tilemix_attention_batched with the output written through `out` (the values
// stored are the roundings of the fp32 outputs tilemix_attention_batched
// produces). Routing trace outputs (decoded_bits, score_dots) are not
// supported here: cudaErrorNotSupported.
cudaError_t tilemix_attention_batched_out(const __half* Q, const __half* K, const __half* V,
                                          const TileMixOutput& out, int heads, int M, int N, int d,
                                          float score_scale, bool causal,
                                          cudaStream_t stream = nullptr,
                                          const TileMixRouting& routing = {},
                                          const TileMixQuantized& quantized = {});

// tilemix_attention_batched (unrouted) that also writes lse [heads, M] fp32:
// log2 of each row's sum of 2^(score_scale * log2(e) * q.k), the statistic
// tilemix_attention_backward recomputes P from (no reference counterpart).
cudaError_t tilemix_attention_batched_lse(const __half* Q, const __half* K, const __half* V, float* O, float* lse,
                                          int heads, int M, int N, int d, float score_scale, bool causal,
                                          cudaStream_t stream = nullptr);

// Backward of the unrouted attention (no reference counterpart: the reference
// is forward only). Given fp16 Q, K, V [heads, M|N, d], the fp32 output O of
// tilemix_attention_batched on them (unrouted, same score_scale and causal)
// and the fp16 output gradient dO [heads, M, d], writes fp32 dQ [heads, M, d],
// dK and dV [heads, N, d] of
//   O = softmax(score_scale * Q K^T [causal: keys <= query]) V.
// lse and dsum are caller-provided [heads, M] fp32 buffers. With
// lse_from_forward, lse holds what tilemix_attention_batched_lse wrote for
// this O and is only read; otherwise the call recomputes each row's
// log-sum-exp (one more Q K^T pass) and writes it there. dsum receives
// rowsum(dO * O). S, dP and the accumulations are fp32 on the tensor cores; P
// and dS enter the second products rounded to fp16. Needs d % 16 == 0,
// d <= 128 and 16-byte aligned pointers (cudaErrorNotSupported /
// cudaErrorMisalignedAddress otherwise); other argument errors as
// tilemix_attention_batched. Two kernel launches, no atomics, deterministic.
cudaError_t tilemix_attention_backward(const __half* Q, const __half* K, const __half* V, const float* O,
                                       const __half* dO, float* dQ, float* dK, float* dV, float* lse,
                                       float* dsum, int heads, int M, int N, int d, float score_scale,
                                       bool causal, bool lse_from_forward = false, cudaStream_t stream = nullptr);
