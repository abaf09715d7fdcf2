// Internal launcher declarations shared by the kernels and the API layer.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace tilemix {

constexpr int kQuantQRows = 128;   // reference include/attention_fused.h:13
constexpr int kQuantKRows = 64;    // reference include/attention_fused.h:14
constexpr int kMaxHeadDim = 128;

// Quantize Q [heads, M, d] (128-row blocks) and K [heads, N, d] (64-row
// blocks) in one launch. Arguments are assumed validated.
cudaError_t launch_quantize(const __half* Q, const __half* K, std::int8_t* Q8, std::int8_t* K8,
                            __half* q_scales, __half* k_scales, int heads, int M, int N, int d,
                            cudaStream_t stream);

struct AttentionProblem {
    const __half* q;
    const __half* k;
    const __half* v;
    const std::int8_t* q8;       // null when not routed
    const std::int8_t* k8;
    const __half* q_scales;
    const __half* k_scales;
    float* o;
    const std::uint64_t* words;  // null = all FP16
    std::uint8_t* decoded_bits;  // optional trace
    std::int32_t* score_dots;    // optional trace
    int heads, M, N, d;
    int key_tiles_per_group;
    float score_scale;
    bool causal;
    // Optional strided output (used instead of `o` when o_data is set):
    // element (row m, column c) of head h = b * o_heads_per_batch + hh sits at
    // o_data + b * o_stride_batch + hh * o_stride_head + m * o_stride_row + c
    // (element units), as fp32 (o_dtype 0), fp16 (1) or bf16 (2).
    void* o_data;
    int o_dtype;
    int o_heads_per_batch;
    long long o_stride_batch, o_stride_head, o_stride_row;
    // Watchdog self-test: launch the instantiation in which one softmax warp
    // withholds its first P-ready arrival, with waits limited to
    // watchdog_limit_ns (the output is not valid; the status word is).
    bool watchdog_test;
    unsigned long long watchdog_limit_ns;
    // Fused Q quantization (routed only): q8 and q_scales are not read; each
    // CTA quantizes its own query tile, and writes the bytes to q8_out /
    // q_scales_out when those are set.
    bool fuse_q;
    std::int8_t* q8_out;
    __half* q_scales_out;
    // Optional max |v| per 64-key block [heads][ceil(N/64)]: key halves whose
    // max is <= 3.5 take single-term P (null: two-term everywhere).
    const __half* v_absmax;
    // Optional [heads][M] fp32 output: log2 of each row's sum of
    // 2^(score_scale * log2(e) * score) (null: not written).
    float* lse_out;
};

// Routing words from the quantizer's block scales (policy.cu): INT8 iff
// q_scale(tile) * max k_scale(group) <= max_scale_product.
cudaError_t launch_routing_policy(const __half* q_scales, const __half* k_scales, std::uint64_t* words, int heads,
                                  int M, int N, int key_tiles_per_group, float max_scale_product,
                                  cudaStream_t stream);

// quantize Q and K as launch_quantize, and record max |V| of every 64-row V
// block (fp16, NaN when the block holds one) in v_absmax [heads][ceil(N/64)],
// all in one launch.
cudaError_t launch_quantize_qkv(const __half* Q, const __half* K, const __half* V, std::int8_t* Q8, std::int8_t* K8,
                                __half* q_scales, __half* k_scales, __half* v_absmax, int heads, int M, int N,
                                int d, cudaStream_t stream);

// Quantize K [heads, N, d] alone (64-row blocks), for the fused-Q path.
cudaError_t launch_quantize_k(const __half* K, std::int8_t* K8, __half* k_scales, int heads, int N, int d,
                              cudaStream_t stream);

// Shared memory the attention kernel requests for head dim d.
std::size_t attention_smem_bytes(int d);

// Launch the fused attention kernel (arguments assumed validated, d <= 128).
cudaError_t launch_attention(const AttentionProblem& problem, cudaStream_t stream);

// Read and clear the device watchdog word of the current device (forward and
// backward kernels' bits together).
cudaError_t read_and_clear_status(unsigned int* status);

// Backward of the unrouted attention (backward.cu): fp16 Q, K, V, dO; fp32 O
// (the forward's output) and fp32 dQ, dK, dV; lse and dsum are [heads][M]
// fp32 row statistics (log2-unit log-sum-exp of score_scale * S, and
// rowsum(dO * O)): the launch writes dsum, and writes lse too unless
// lse_ready (lse then holds the forward's lse_out and is only read).
// d % 16 == 0, d <= 128, every pointer 16-byte aligned; arguments otherwise
// assumed validated.
constexpr int kBackwardMaxHeadDim = 128;
struct AttentionBackwardProblem {
    const __half* q;
    const __half* k;
    const __half* v;
    const float* o;
    const __half* dout;
    float* dq;
    float* dk;
    float* dv;
    float* lse;
    float* dsum;
    int heads, M, N, d;
    float score_scale;
    bool causal;
    bool lse_ready;
    // Watchdog self-test (d = 128 only): nonzero = the column kernel build in
    // which one elementwise warp withholds its first P-ready arrival, its
    // waits limited to this many ns (the gradients are not valid; the status
    // word is).
    unsigned long long watchdog_limit_ns;
};
cudaError_t launch_attention_backward(const AttentionBackwardProblem& problem, cudaStream_t stream);
cudaError_t read_and_clear_backward_status(unsigned int* status);

}  // namespace tilemix
