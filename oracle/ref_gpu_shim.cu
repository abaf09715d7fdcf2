// C-ABI shim over the reference's OWN GPU kernels -- BENCHMARK COMPARISON ONLY.
//
// Compiled by oracle/build_ref.sh together with the reference's src/tilemix.cu
// where it lies (nothing from the reference is copied into this repository)
// into oracle/_ref/libtilemix_ref_gpu.so. bench.py times it as the "reference
// GPU" column: the reference's public entry points, quantize_tilemix_qk and
// launch_fused_fp16_attention (include/attention_fused.h:62-72), called once
// per head on the caller's stream, exactly as its own driver (src/main.cu) and
// tests call them. The reference kernel has no causal mask, so this times the
// full (non-causal) attention of each head.
#include "attention_fused.h"

#include <cstddef>
#include <cstdint>

extern "C" {

// One call = the reference's quantizer + fused attention for `heads` heads of
// a [heads][M][d] / [heads][N][d] layout. Routing words are per head,
// `words_per_head` apart (the reference's [ceil(M/16)][words_per_row] layout);
// words == nullptr runs the reference's all-FP16 path without quantization.
// Returns the first non-success cudaError_t, or 0.
int ref_gpu_tilemix_heads(const void* q, const void* k, const void* v, void* q8, void* k8, void* q_scales,
                          void* k_scales, float* o, int heads, int M, int N, int d, float score_scale,
                          const std::uint64_t* words, std::size_t words_per_head, int key_tiles_per_group,
                          void* stream) {
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    const std::size_t q_blocks = (static_cast<std::size_t>(M) - 1) / kTileMixQQuantRows + 1;
    const std::size_t k_blocks = (static_cast<std::size_t>(N) - 1) / kTileMixKQuantRows + 1;
    for (int h = 0; h < heads; ++h) {
        const std::size_t qo = static_cast<std::size_t>(h) * M * d, ko = static_cast<std::size_t>(h) * N * d;
        const __half* qh = static_cast<const __half*>(q) + qo;
        const __half* kh = static_cast<const __half*>(k) + ko;
        const __half* vh = static_cast<const __half*>(v) + ko;
        TileMixRouting routing{};
        TileMixQuantized quantized{};
        if (words) {
            std::int8_t* q8h = static_cast<std::int8_t*>(q8) + qo;
            std::int8_t* k8h = static_cast<std::int8_t*>(k8) + ko;
            __half* qsh = static_cast<__half*>(q_scales) + h * q_blocks;
            __half* ksh = static_cast<__half*>(k_scales) + h * k_blocks;
            cudaError_t e = quantize_tilemix_qk(qh, kh, q8h, k8h, qsh, ksh, M, N, d, s);
            if (e != cudaSuccess) return static_cast<int>(e);
            routing.words = words + h * words_per_head;
            routing.word_count = words_per_head;
            routing.key_tiles_per_group = key_tiles_per_group;
            quantized.q = q8h;
            quantized.k = k8h;
            quantized.q_scales = qsh;
            quantized.k_scales = ksh;
        }
        cudaError_t e = launch_fused_fp16_attention(qh, kh, vh, o + qo, M, N, d, score_scale, s, routing, quantized);
        if (e != cudaSuccess) return static_cast<int>(e);
    }
    return 0;
}

}  // extern "C"
