/*
 * TileMix B200 C-ABI (libtilemix_b200.so).
 *
 * Plain C entry points over the same kernels as the C++ API in
 * attention_fused.h: plain pointers, sizes and POD structs, no C++ references,
 * no default arguments and no torch types, so any FFI (ctypes, cgo, JNI,
 * N-API) can bind them. fp16 tensors are passed as `const void*` holding IEEE
 * binary16 values; streams as `void*` (a cudaStream_t, NULL = legacy default).
 * Return values are cudaError_t codes as int (0 = cudaSuccess,
 * 1 = cudaErrorInvalidValue, 9 = cudaErrorInvalidConfiguration,
 * 801 = cudaErrorNotSupported).
 */
#ifndef TILEMIX_C_API_H
#define TILEMIX_C_API_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TILEMIX_ABI_VERSION 1

/* Layout-compatible with TileMixRouting (reference include/attention_fused.h:47-52). */
typedef struct tilemix_routing {
    const uint64_t* words;
    size_t word_count;
    int key_tiles_per_group;
    uint8_t* decoded_bits;
} tilemix_routing;

/* Layout-compatible with TileMixQuantized (reference include/attention_fused.h:54-60). */
typedef struct tilemix_quantized {
    const int8_t* q;
    const int8_t* k;
    const void* q_scales;   /* fp16 [ceil(M/128)] (per head) */
    const void* k_scales;   /* fp16 [ceil(N/64)]  (per head) */
    int32_t* score_dots;
} tilemix_quantized;

int tilemix_abi_version(void);

/* Replaces quantize_tilemix_qk (reference src/tilemix.cu:223-236). */
int tilemix_quantize_qk(const void* Q, const void* K, int8_t* Q8, int8_t* K8,
                        void* q_scales, void* k_scales, int M, int N, int d, void* stream);

/* Replaces launch_fused_fp16_attention (reference src/tilemix.cu:238-278).
 * routing / quantized may be NULL (same as the reference's `{}` defaults). */
int tilemix_fused_attention(const void* Q, const void* K, const void* V, float* O,
                            int M, int N, int d, float score_scale, void* stream,
                            const tilemix_routing* routing, const tilemix_quantized* quantized);

/* Batched [heads, M|N, d] forms (no reference counterpart: the reference is
 * single-head). Per head identical semantics; causal != 0 masks key > query. */
int tilemix_quantize_qk_batched(const void* Q, const void* K, int8_t* Q8, int8_t* K8,
                                void* q_scales, void* k_scales, int heads, int M, int N,
                                int d, void* stream);
int tilemix_attention_batched(const void* Q, const void* K, const void* V, float* O,
                              int heads, int M, int N, int d, float score_scale, int causal,
                              void* stream, const tilemix_routing* routing,
                              const tilemix_quantized* quantized);

/* K-only quantizer and routed attention with Q quantized inside the kernel
 * (no reference counterpart): C forms of quantize_tilemix_k_batched and
 * tilemix_attention_batched_qfused in attention_fused.h. Routing words, K8 and
 * k_scales are required; Q8_out / q_scales_out may be NULL, else they receive
 * the Q8 bytes and fp16 scales tilemix_quantize_qk_batched would produce. */
int tilemix_quantize_k_batched(const void* K, int8_t* K8, void* k_scales, int heads, int N, int d,
                               void* stream);
int tilemix_attention_batched_qfused(const void* Q, const void* K, const void* V, float* O,
                                     int heads, int M, int N, int d, float score_scale, int causal,
                                     void* stream, const tilemix_routing* routing, const int8_t* K8,
                                     const void* k_scales, int8_t* Q8_out, void* q_scales_out);

/* Strided output of tilemix_attention_batched_out (layout-compatible with
 * TileMixOutput in attention_fused.h): head h = b * heads_per_batch + hh,
 * row m, column c goes to data + b * stride_batch + hh * stride_head +
 * m * stride_row + c (element units), as fp32 (dtype 0), fp16 (1) or bf16 (2),
 * rounded to nearest even. BSHD [B, S, H, D]: heads_per_batch = H,
 * stride_batch = S*H*D, stride_head = D, stride_row = H*D. */
typedef struct tilemix_output {
    void* data;
    int dtype;
    int heads_per_batch;
    long long stride_batch;
    long long stride_head;
    long long stride_row;
} tilemix_output;

/* tilemix_attention_batched writing O through `out` (no reference
 * counterpart: the reference writes fp32 [M, d] only, include/attention_fused.h:68-69).
 * Invalid layouts (null data, bad dtype, heads_per_batch < 1 or not dividing
 * heads, negative strides) return cudaErrorInvalidValue; routing trace
 * outputs together with a strided output return cudaErrorNotSupported. */
int tilemix_attention_batched_out(const void* Q, const void* K, const void* V,
                                  const tilemix_output* out, int heads, int M, int N, int d,
                                  float score_scale, int causal, void* stream,
                                  const tilemix_routing* routing,
                                  const tilemix_quantized* quantized);

/* Caller-owned device buffers of tilemix_attention_from_host, each sized for
 * all `heads` heads: q, k, v fp16 [heads, M|N, d]; q8, k8 int8 of the same
 * shapes; q_scales fp16 [heads, ceil(M/128)]; k_scales fp16 [heads, ceil(N/64)];
 * words [heads * tilemix_routing_word_count_c(M, N, g)]; o fp32 [heads, M, d].
 * q8, k8, q_scales, k_scales and words may be NULL when no routing is given. */
typedef struct tilemix_device_buffers {
    void* q;
    void* k;
    void* v;
    int8_t* q8;
    int8_t* k8;
    void* q_scales;
    void* k_scales;
    uint64_t* words;
    float* o;
} tilemix_device_buffers;

/* The whole path from host memory, as the reference's driver runs it
 * (src/main.cu:44-60: H2D copies, quantize_tilemix_qk,
 * launch_fused_fp16_attention, D2H of O), for [heads, M|N, d] batches and
 * pipelined: heads are processed in chunks of `chunk_heads` (<= 0 picks a
 * size), and the H2D copy of chunk c + 1, the kernels of chunk c and the D2H
 * copy of chunk c - 1 overlap on two library-owned copy streams. hQ, hK, hV
 * (fp16) and hO (fp32) are host buffers in the same layouts as their device
 * counterparts; pinned memory is needed for the copies to overlap. h_words
 * (heads * tilemix_routing_word_count_c(M, N, key_tiles_per_group) words, NULL
 * = every tile FP16) selects the routed path: Q and K are quantized on the
 * device and each tile is scored by its routing bit. Asynchronous: every step
 * is ordered after the work already queued on `stream`, and once `stream`
 * reaches the point of the call's return, hO holds the output. Same error
 * contract as tilemix_attention_batched; nothing is queued when an argument is
 * invalid. If a launch fails after copies were queued, `stream` is made to wait
 * for the copy streams before the error returns: the host buffers must stay
 * valid until `stream` reaches that point (as on success). */
int tilemix_attention_from_host(const void* hQ, const void* hK, const void* hV,
                                const uint64_t* h_words, float* hO,
                                const tilemix_device_buffers* dev, int heads, int M, int N,
                                int d, float score_scale, int causal, int key_tiles_per_group,
                                int chunk_heads, void* stream);

/* Routed attention that allocates nothing (no counterpart in the reference;
 * the reference and tilemix_attention_batched take the INT8 Q/K copies and
 * their scales from the caller). For callers that cannot allocate device
 * memory: an operator or plugin interface handed only its inputs and outputs
 * at launch time, a binding with no access to the process's device allocator,
 * or a framework whose caching allocator owns the device memory. Q, K, V
 * (fp16) and O (fp32) are the caller's device buffers, as in
 * tilemix_attention_batched; the INT8 copies of Q and K and their scales go to
 * a fixed array of TILEMIX_NOALLOC_SCRATCH_BYTES of device memory inside the
 * library, which every GPU that loads the library's code holds until the
 * process exits. The call quantizes Q and K into it and runs the routed
 * attention on the same stream; it calls no cudaMalloc, cudaFree or other
 * allocating routine. With routing NULL or routing->words NULL every tile is
 * FP16 and the scratch is not used.
 *   - Limit: heads*M*d + heads*N*d bytes of INT8 copies, plus the scales, each
 *     part rounded up to 256 bytes, must fit in TILEMIX_NOALLOC_SCRATCH_BYTES
 *     (e.g. 64 heads of S = 4096, d = 128); larger problems return
 *     cudaErrorMemoryAllocation (2) before anything is queued.
 *   - Every call on a device shares the one array: calls whose work overlaps
 *     on the GPU (other streams, other threads) race and corrupt each other's
 *     intermediates. Order them on one stream or with events.
 *   - The array keeps the last call's contents; every byte a call reads is
 *     first written by that call's quantizer, so nothing needs clearing.
 *   - The first call on each device looks up the array's device address (with
 *     that device current); make that first call before any stream capture.
 * Otherwise the error contract of tilemix_attention_batched. */
#define TILEMIX_NOALLOC_SCRATCH_BYTES ((size_t)64 << 20)
int tilemix_attention_routed_noalloc(const void* Q, const void* K, const void* V, float* O,
                                     int heads, int M, int N, int d, float score_scale, int causal,
                                     const tilemix_routing* routing, void* stream);

/* Precision hints for PV (no reference counterpart): C forms of
 * quantize_tilemix_qkv_batched (Q/K quantization plus max |v| per 64-row V
 * block, fp16 [heads][ceil(N/64)]) and tilemix_attention_batched_hinted
 * (key halves with max |v| <= 3.5 take single-term fp16 P: at most 1.7e-3
 * added to any output; v_absmax NULL = tilemix_attention_batched). */
int tilemix_quantize_qkv_batched(const void* Q, const void* K, const void* V, int8_t* Q8, int8_t* K8,
                                 void* q_scales, void* k_scales, void* v_absmax, int heads, int M, int N,
                                 int d, void* stream);
int tilemix_attention_batched_hinted(const void* Q, const void* K, const void* V, float* O, int heads,
                                     int M, int N, int d, float score_scale, int causal, void* stream,
                                     const tilemix_routing* routing, const tilemix_quantized* quantized,
                                     const void* v_absmax);

/* Device-side routing policy (no reference counterpart; the reference takes
 * the mask from the caller, src/main.cu:48): C form of tilemix_routing_policy
 * in attention_fused.h. words: heads * tilemix_routing_word_count_c(M, N, g)
 * words; bit = 1 (INT8) iff q_scale * max k_scale of the key group <=
 * max_scale_product. tilemix_policy_max_scale_product_c(tol, score_scale, d)
 * gives the product that bounds the INT8 score error by tol. */
int tilemix_routing_policy_c(const void* q_scales, const void* k_scales, uint64_t* words, int heads,
                             int M, int N, int key_tiles_per_group, float max_scale_product,
                             void* stream);
float tilemix_policy_max_scale_product_c(float tolerance, float score_scale, int d);

/* Sizing helpers (reference include/attention_fused.h:34-45). */
size_t tilemix_routing_word_count_c(int M, int N, int key_tiles_per_group);
size_t tilemix_routing_words_per_row_c(int N, int key_tiles_per_group);
size_t tilemix_reference_shared_bytes(int d, int quantized);
size_t tilemix_b200_shared_bytes_c(int d, int quantized);

/* Training forward (no reference counterpart): C form of
 * tilemix_attention_batched_lse in attention_fused.h, the unrouted
 * tilemix_attention_batched that also writes lse [heads, M] fp32 (log2 of each
 * row's sum of 2^(score_scale * log2(e) * q.k)). */
int tilemix_attention_batched_lse_c(const void* Q, const void* K, const void* V, float* O, float* lse,
                                    int heads, int M, int N, int d, float score_scale, int causal,
                                    void* stream);

/* Backward of the unrouted attention (no reference counterpart; the reference
 * is forward only): C form of tilemix_attention_backward in attention_fused.h.
 * Q, K, V, dO fp16; O fp32 (the forward's output on the same inputs, unrouted);
 * dQ [heads, M, d], dK and dV [heads, N, d] fp32 outputs; lse and dsum
 * [heads, M] fp32: with lse_from_forward != 0 lse holds what
 * tilemix_attention_batched_lse_c wrote and is read, otherwise it is computed
 * and written; dsum receives rowsum(dO * O). d % 16 == 0, d <= 128, 16-byte
 * aligned pointers. Its waits are bounded like the forward's and report
 * through tilemix_read_and_clear_status (bits 16 and 32). */
int tilemix_attention_backward_c(const void* Q, const void* K, const void* V, const float* O, const void* dO,
                                 float* dQ, float* dK, float* dV, float* lse, float* dsum, int heads, int M,
                                 int N, int d, float score_scale, int causal, int lse_from_forward,
                                 void* stream);

/* Device-side watchdog status of the attention kernel on the current device:
 * every pipeline wait in the kernel is bounded; a wait that runs out records a
 * nonzero code here and the kernel returns early instead of hanging. Reading
 * synchronises the device and clears the word. 0 = no timeout seen. */
int tilemix_read_and_clear_status(unsigned int* status);

/* Watchdog self-test (no counterpart in the reference; for tests only): runs
 * the unrouted attention kernel in a build in which one softmax warp of each
 * CTA withholds its first "P ready" arrival, with every wait limited to
 * wait_limit_us microseconds (1..1000000). The MMA warp's wait for that
 * arrival runs out, the kernel records the MMA-wait bit (2) in the status word
 * that tilemix_read_and_clear_status returns, and every role drains its
 * in-flight copies and MMAs and returns. O is not valid afterwards. Needs
 * 65 <= d <= 128, d % 16 == 0 and 16-byte aligned Q/K/V/O (the TMA build);
 * otherwise cudaErrorNotSupported. */
int tilemix_watchdog_selftest(const void* Q, const void* K, const void* V, float* O, int heads, int M,
                              int N, int d, float score_scale, unsigned int wait_limit_us, void* stream);

/* Backward watchdog self-test (no counterpart in the reference; for tests
 * only): tilemix_attention_backward_c (recomputing the row LSE, not causal)
 * with the column kernel built so that one elementwise warp of each CTA
 * withholds its first "P ready" arrival and every wait of that kernel is
 * limited to wait_limit_us microseconds (1..1000000). The accumulation warp's
 * wait runs out, the kernel records bit 16 in the status word that
 * tilemix_read_and_clear_status returns, every role drains its own copies and
 * MMAs and returns. dQ, dK, dV are not valid afterwards. d must be 128
 * (cudaErrorNotSupported otherwise). */
int tilemix_backward_watchdog_selftest(const void* Q, const void* K, const void* V, const float* O, const void* dO,
                                       float* dQ, float* dK, float* dV, float* lse, float* dsum, int heads,
                                       int M, int N, int d, float score_scale, unsigned int wait_limit_us,
                                       void* stream);

#ifdef __cplusplus
}
#endif

#endif
