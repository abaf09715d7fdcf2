// Routed attention for callers that cannot allocate device memory.
//
// The routed path needs INT8 copies of Q and K and their block scales between
// the quantizer and the attention kernel. The regular entry points take those
// buffers from the caller; some callers cannot provide them: an operator or
// plugin interface that is handed only its inputs and outputs at launch time,
// a binding (cgo, JNI, ctypes) with no access to the process's device
// allocator, or a framework whose caching allocator owns the device memory.
// tilemix_attention_routed_noalloc keeps those intermediates in a fixed array
// of device memory that belongs to this file instead, and calls no allocator.
#include "attention_fused.h"
#include "tilemix_c_api.h"

#include <cmath>
#include <cstddef>
#include <cstdint>
#include <mutex>

// The scratch: INT8 Q and K copies and their fp16 scales of one call. Loading
// this file's device code reserves it on every GPU that loads it, until the
// process exits.
static __device__ __align__(256) std::uint8_t g_noalloc_scratch[TILEMIX_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr int kMaxDevices = 64;

std::size_t round256(std::size_t bytes) { return (bytes + 255u) & ~static_cast<std::size_t>(255u); }

// Device address of the scratch on the current device. In host code the
// array's name is a host-side stand-in, not a device address; the runtime
// gives the real address, once per device (the first call on a device does
// this set-up with that device current).
cudaError_t scratch_address(std::uint8_t** out) {
    static std::mutex mu;
    static std::uint8_t* addresses[kMaxDevices] = {};
    int device = 0;
    cudaError_t status = cudaGetDevice(&device);
    if (status != cudaSuccess) return status;
    if (device < 0 || device >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(mu);
    if (!addresses[device]) {
        void* ptr = nullptr;
        status = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
        if (status != cudaSuccess) return status;
        addresses[device] = static_cast<std::uint8_t*>(ptr);
    }
    *out = addresses[device];
    return cudaSuccess;
}

}  // namespace

extern "C" int tilemix_attention_routed_noalloc(const void* Q, const void* K, const void* V, float* O,
                                                int heads, int M, int N, int d, float score_scale,
                                                int causal, const tilemix_routing* routing, void* stream) {
    TileMixRouting r{};
    if (routing) {
        r.words = routing->words;
        r.word_count = routing->word_count;
        r.key_tiles_per_group = routing->key_tiles_per_group;
        r.decoded_bits = routing->decoded_bits;
    }
    const auto* q = static_cast<const __half*>(Q);
    const auto* k = static_cast<const __half*>(K);
    const auto* v = static_cast<const __half*>(V);
    const auto s = static_cast<cudaStream_t>(stream);
    if (!r.words) {
        // No routing: every tile is FP16 and there are no intermediates.
        return static_cast<int>(tilemix_attention_batched(q, k, v, O, heads, M, N, d, score_scale, causal != 0,
                                                          s, r, TileMixQuantized{}));
    }
    // The attention entry point's own checks, made here before anything is
    // queued (the quantizer runs first).
    if (!Q || !K || !V || !O || heads <= 0 || M <= 0 || N <= 0 || d <= 0 || !std::isfinite(score_scale) ||
        r.key_tiles_per_group <= 0) {
        return static_cast<int>(cudaErrorInvalidValue);
    }
    if (d > kFusedMaxHeadDim) return static_cast<int>(cudaErrorNotSupported);
    if (static_cast<long long>(heads) * M > (1ll << 40) / d || static_cast<long long>(heads) * N > (1ll << 40) / d ||
        r.word_count / static_cast<std::size_t>(heads) < tilemix_routing_word_count(M, N, r.key_tiles_per_group)) {
        return static_cast<int>(cudaErrorInvalidValue);
    }
    // Scratch layout, each part on a 256-byte boundary: Q8 [heads, M, d],
    // K8 [heads, N, d], q_scales [heads, ceil(M/128)], k_scales [heads, ceil(N/64)].
    const std::size_t q8_bytes = static_cast<std::size_t>(heads) * M * d;
    const std::size_t k8_bytes = static_cast<std::size_t>(heads) * N * d;
    const std::size_t qs_bytes = sizeof(__half) * heads * ((static_cast<std::size_t>(M) - 1) / kTileMixQQuantRows + 1);
    const std::size_t ks_bytes = sizeof(__half) * heads * ((static_cast<std::size_t>(N) - 1) / kTileMixKQuantRows + 1);
    const std::size_t k8_off = round256(q8_bytes);
    const std::size_t qs_off = k8_off + round256(k8_bytes);
    const std::size_t ks_off = qs_off + round256(qs_bytes);
    if (ks_off + ks_bytes > TILEMIX_NOALLOC_SCRATCH_BYTES) return static_cast<int>(cudaErrorMemoryAllocation);

    std::uint8_t* scratch = nullptr;
    const cudaError_t status = scratch_address(&scratch);
    if (status != cudaSuccess) return static_cast<int>(status);
    auto* q8 = reinterpret_cast<std::int8_t*>(scratch);
    auto* k8 = reinterpret_cast<std::int8_t*>(scratch + k8_off);
    auto* qs = reinterpret_cast<__half*>(scratch + qs_off);
    auto* ks = reinterpret_cast<__half*>(scratch + ks_off);
    // The quantizer writes every byte of these four parts that the attention
    // kernel reads, so nothing left by an earlier call needs clearing.
    cudaError_t err = quantize_tilemix_qk_batched(q, k, q8, k8, qs, ks, heads, M, N, d, s);
    if (err != cudaSuccess) return static_cast<int>(err);
    TileMixQuantized quantized{};
    quantized.q = q8;
    quantized.k = k8;
    quantized.q_scales = qs;
    quantized.k_scales = ks;
    return static_cast<int>(tilemix_attention_batched(q, k, v, O, heads, M, N, d, score_scale, causal != 0, s, r,
                                                      quantized));
}
