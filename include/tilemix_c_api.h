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

/* Sizing helpers (reference include/attention_fused.h:34-45). */
size_t tilemix_routing_word_count_c(int M, int N, int key_tiles_per_group);
size_t tilemix_routing_words_per_row_c(int N, int key_tiles_per_group);
size_t tilemix_reference_shared_bytes(int d, int quantized);
size_t tilemix_b200_shared_bytes_c(int d, int quantized);

/* Device-side watchdog status of the attention kernel on the current device:
 * every pipeline wait in the kernel is bounded; a wait that runs out records a
 * nonzero code here and the kernel returns early instead of hanging. Reading
 * synchronises the device and clears the word. 0 = no timeout seen. */
int tilemix_read_and_clear_status(unsigned int* status);

#ifdef __cplusplus
}
#endif

#endif
