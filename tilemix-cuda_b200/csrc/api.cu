// Drop-in API layer: argument validation with the reference's error contract
// (src/tilemix.cu:223-278), device checks, and the extern "C" ABI of
// include/tilemix_c_api.h. Kernels live in quantize.cu, attention.cu, policy.cu
// and backward.cu.
#include "attention_fused.h"
#include "kernels.cuh"
#include "tilemix_c_api.h"

#include <algorithm>
#include <cmath>
#include <cstddef>
#include <cstdint>
#include <mutex>
#include <vector>

namespace {

constexpr int kMaxDevices = 64;

// sm_100 check, cached per device (the reference queries cudaDeviceProp on
// every launch, src/tilemix.cu:254-260; one attribute query per device here).
cudaError_t check_device() {
    static int state[kMaxDevices] = {0};   // 0 unknown, 1 supported, 2 not supported
    int device = 0;
    cudaError_t status = cudaGetDevice(&device);
    if (status != cudaSuccess) return status;
    if (device < 0 || device >= kMaxDevices) return cudaErrorInvalidDevice;
    if (state[device] == 0) {
        int major = 0;
        status = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
        if (status != cudaSuccess) return status;
        state[device] = major == 10 ? 1 : 2;
    }
    return state[device] == 1 ? cudaSuccess : cudaErrorNotSupported;
}

bool fits(long long heads, long long rows, long long d) {
    return heads > 0 && rows > 0 && d > 0 && heads * rows <= (1ll << 40) / d;
}

cudaError_t quantize_impl(const __half* Q, const __half* K, std::int8_t* Q8, std::int8_t* K8,
                          __half* q_scales, __half* k_scales, int heads, int M, int N, int d,
                          cudaStream_t stream) {
    if (!Q || !K || !Q8 || !K8 || !q_scales || !k_scales || heads <= 0 || M <= 0 || N <= 0 || d <= 0) {
        return cudaErrorInvalidValue;
    }
    if (d > kFusedMaxHeadDim) return cudaErrorNotSupported;
    if (!fits(heads, M, d) || !fits(heads, N, d)) return cudaErrorInvalidValue;
    const cudaError_t status = check_device();
    if (status != cudaSuccess) return status;
    return tilemix::launch_quantize(Q, K, Q8, K8, q_scales, k_scales, heads, M, N, d, stream);
}

cudaError_t attention_impl(const __half* Q, const __half* K, const __half* V, float* O, int heads,
                           int M, int N, int d, float score_scale, bool causal, cudaStream_t stream,
                           const TileMixRouting& routing, const TileMixQuantized& quantized,
                           const TileMixOutput* strided = nullptr, unsigned long long watchdog_test_ns = 0,
                           const __half* v_absmax = nullptr, float* lse_out = nullptr) {
    // Same checks, same order as src/tilemix.cu:242-253.
    if (!Q || !K || !V || (!O && !strided) || heads <= 0 || M <= 0 || N <= 0 || d <= 0 ||
        !std::isfinite(score_scale) || routing.key_tiles_per_group <= 0 ||
        (!routing.words && routing.word_count != 0)) {
        return cudaErrorInvalidValue;
    }
    if (d > kFusedMaxHeadDim) return cudaErrorNotSupported;
    const std::size_t per_head = tilemix_routing_word_count(M, N, routing.key_tiles_per_group);
    if (routing.words && routing.word_count / static_cast<std::size_t>(heads) < per_head) {
        return cudaErrorInvalidValue;
    }
    const bool has_quantized = quantized.q && quantized.k && quantized.q_scales && quantized.k_scales;
    const bool any_quantized = quantized.q || quantized.k || quantized.q_scales || quantized.k_scales ||
                               quantized.score_dots;
    if ((any_quantized && !has_quantized) || (routing.words && !has_quantized)) return cudaErrorInvalidValue;
    if (!fits(heads, M, d) || !fits(heads, N, d)) return cudaErrorInvalidValue;
    if (strided) {
        if (!strided->data || strided->dtype < kTileMixOutF32 || strided->dtype > kTileMixOutBF16 ||
            strided->heads_per_batch < 1 || heads % strided->heads_per_batch != 0 || strided->stride_batch < 0 ||
            strided->stride_head < 0 || strided->stride_row < 0) {
            return cudaErrorInvalidValue;
        }
        if (routing.decoded_bits || quantized.score_dots) return cudaErrorNotSupported;
    }
    cudaError_t status = check_device();
    if (status != cudaSuccess) return status;
    if (static_cast<long long>((M - 1) / 128 + 1) * heads > 0x7fffffffLL) return cudaErrorInvalidConfiguration;

    tilemix::AttentionProblem prob{};
    prob.q = Q; prob.k = K; prob.v = V; prob.o = O;
    prob.words = routing.words;
    prob.decoded_bits = routing.decoded_bits;
    prob.key_tiles_per_group = routing.key_tiles_per_group;
    if (has_quantized) {
        prob.q8 = quantized.q; prob.k8 = quantized.k;
        prob.q_scales = quantized.q_scales; prob.k_scales = quantized.k_scales;
        prob.score_dots = quantized.score_dots;
    }
    prob.heads = heads; prob.M = M; prob.N = N; prob.d = d;
    prob.score_scale = score_scale;
    prob.causal = causal;
    if (strided) {
        prob.o_data = strided->data;
        prob.o_dtype = strided->dtype;
        prob.o_heads_per_batch = strided->heads_per_batch;
        prob.o_stride_batch = strided->stride_batch;
        prob.o_stride_head = strided->stride_head;
        prob.o_stride_row = strided->stride_row;
    }
    prob.v_absmax = v_absmax;
    prob.lse_out = lse_out;
    prob.watchdog_test = watchdog_test_ns != 0;
    prob.watchdog_limit_ns = watchdog_test_ns;
    return tilemix::launch_attention(prob, stream);
}

cudaError_t quantize_qkv_impl(const __half* Q, const __half* K, const __half* V, std::int8_t* Q8, std::int8_t* K8,
                              __half* q_scales, __half* k_scales, __half* v_absmax, int heads, int M, int N, int d,
                              cudaStream_t stream) {
    if (!V || !v_absmax) return cudaErrorInvalidValue;
    if (!Q || !K || !Q8 || !K8 || !q_scales || !k_scales || heads <= 0 || M <= 0 || N <= 0 || d <= 0) {
        return cudaErrorInvalidValue;
    }
    if (d > kFusedMaxHeadDim) return cudaErrorNotSupported;
    if (!fits(heads, M, d) || !fits(heads, N, d)) return cudaErrorInvalidValue;
    const cudaError_t status = check_device();
    if (status != cudaSuccess) return status;
    return tilemix::launch_quantize_qkv(Q, K, V, Q8, K8, q_scales, k_scales, v_absmax, heads, M, N, d, stream);
}

cudaError_t quantize_k_impl(const __half* K, std::int8_t* K8, __half* k_scales, int heads, int N, int d,
                            cudaStream_t stream) {
    if (!K || !K8 || !k_scales || heads <= 0 || N <= 0 || d <= 0) return cudaErrorInvalidValue;
    if (d > kFusedMaxHeadDim) return cudaErrorNotSupported;
    if (!fits(heads, N, d)) return cudaErrorInvalidValue;
    const cudaError_t status = check_device();
    if (status != cudaSuccess) return status;
    return tilemix::launch_quantize_k(K, K8, k_scales, heads, N, d, stream);
}

// Routed attention with Q quantized inside the kernel: the checks of
// attention_impl, with the quantized inputs reduced to K8 and the K scales
// (both required, as are the routing words); Q8_out / q_scales_out optional.
cudaError_t attention_qfused_impl(const __half* Q, const __half* K, const __half* V, float* O, int heads, int M,
                                  int N, int d, float score_scale, bool causal, cudaStream_t stream,
                                  const TileMixRouting& routing, const std::int8_t* K8, const __half* k_scales,
                                  std::int8_t* Q8_out, __half* q_scales_out) {
    if (!Q || !K || !V || !O || heads <= 0 || M <= 0 || N <= 0 || d <= 0 || !std::isfinite(score_scale) ||
        routing.key_tiles_per_group <= 0 || !routing.words || !K8 || !k_scales) {
        return cudaErrorInvalidValue;
    }
    if (d > kFusedMaxHeadDim) return cudaErrorNotSupported;
    const std::size_t per_head = tilemix_routing_word_count(M, N, routing.key_tiles_per_group);
    if (routing.word_count / static_cast<std::size_t>(heads) < per_head) return cudaErrorInvalidValue;
    if (!fits(heads, M, d) || !fits(heads, N, d)) return cudaErrorInvalidValue;
    cudaError_t status = check_device();
    if (status != cudaSuccess) return status;
    if (static_cast<long long>((M - 1) / 128 + 1) * heads > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
    tilemix::AttentionProblem prob{};
    prob.q = Q; prob.k = K; prob.v = V; prob.o = O;
    prob.words = routing.words;
    prob.decoded_bits = routing.decoded_bits;
    prob.key_tiles_per_group = routing.key_tiles_per_group;
    prob.k8 = K8;
    prob.k_scales = k_scales;
    prob.heads = heads; prob.M = M; prob.N = N; prob.d = d;
    prob.score_scale = score_scale;
    prob.causal = causal;
    prob.fuse_q = true;
    prob.q8_out = Q8_out;
    prob.q_scales_out = q_scales_out;
    return tilemix::launch_attention(prob, stream);
}

cudaError_t routing_policy_impl(const __half* q_scales, const __half* k_scales, std::uint64_t* words, int heads,
                                int M, int N, int key_tiles_per_group, float max_scale_product, cudaStream_t stream) {
    if (!q_scales || !k_scales || !words || heads <= 0 || M <= 0 || N <= 0 || key_tiles_per_group <= 0 ||
        std::isnan(max_scale_product)) {
        return cudaErrorInvalidValue;
    }
    if (static_cast<long long>(heads) * tilemix_routing_word_count(M, N, key_tiles_per_group) > (1ll << 40)) {
        return cudaErrorInvalidValue;
    }
    const cudaError_t status = check_device();
    if (status != cudaSuccess) return status;
    return tilemix::launch_routing_policy(q_scales, k_scales, words, heads, M, N, key_tiles_per_group,
                                          max_scale_product, stream);
}

TileMixRouting to_cpp(const tilemix_routing* r) {
    TileMixRouting out{};
    if (r) {
        out.words = r->words;
        out.word_count = r->word_count;
        out.key_tiles_per_group = r->key_tiles_per_group;
        out.decoded_bits = r->decoded_bits;
    }
    return out;
}

TileMixQuantized to_cpp(const tilemix_quantized* q) {
    TileMixQuantized out{};
    if (q) {
        out.q = q->q;
        out.k = q->k;
        out.q_scales = static_cast<const __half*>(q->q_scales);
        out.k_scales = static_cast<const __half*>(q->k_scales);
        out.score_dots = q->score_dots;
    }
    return out;
}

// ------------------------------------------------- pipelined host-buffer path
// Per device: two copy streams (host->device, device->host) and a pool of
// events, created on first use and kept for the life of the process. The
// mutex only serialises the enqueueing of calls that share a device.
struct PipelineContext {
    std::mutex mu;
    cudaStream_t h2d = nullptr;
    cudaStream_t d2h = nullptr;
    std::vector<cudaEvent_t> events;
};

PipelineContext g_pipeline[kMaxDevices];

cudaError_t pipeline_context(PipelineContext& ctx, std::size_t events) {
    cudaError_t status = cudaSuccess;
    if (!ctx.h2d) status = cudaStreamCreateWithFlags(&ctx.h2d, cudaStreamNonBlocking);
    if (status == cudaSuccess && !ctx.d2h) status = cudaStreamCreateWithFlags(&ctx.d2h, cudaStreamNonBlocking);
    while (status == cudaSuccess && ctx.events.size() < events) {
        cudaEvent_t e = nullptr;
        status = cudaEventCreateWithFlags(&e, cudaEventDisableTiming);
        if (status == cudaSuccess) ctx.events.push_back(e);
    }
    return status;
}

#define TM_TRY(expr)                                \
    do {                                            \
        const cudaError_t tm_status_ = (expr);      \
        if (tm_status_ != cudaSuccess) return tm_status_; \
    } while (0)

// H2D of chunk c (copy stream 1) -> quantize + attention of chunk c (the
// caller's stream) -> D2H of chunk c (copy stream 2), linked by events, so the
// copies of neighbouring chunks overlap the kernels. A recorded event is only
// re-recorded by a later call, after every wait on it has been enqueued
// (cudaStreamWaitEvent binds to the record current at the time of the wait).
cudaError_t from_host_impl(const __half* hQ, const __half* hK, const __half* hV, const std::uint64_t* h_words,
                           float* hO, const tilemix_device_buffers* dev, int heads, int M, int N, int d,
                           float score_scale, bool causal, int g, int chunk_heads, cudaStream_t stream) {
    if (!hQ || !hK || !hV || !hO || !dev || !dev->q || !dev->k || !dev->v || !dev->o || heads <= 0 ||
        M <= 0 || N <= 0 || d <= 0 || !std::isfinite(score_scale) || g <= 0) {
        return cudaErrorInvalidValue;
    }
    const bool routed = h_words != nullptr;
    if (routed && (!dev->words || !dev->q8 || !dev->k8 || !dev->q_scales || !dev->k_scales)) {
        return cudaErrorInvalidValue;
    }
    if (d > kFusedMaxHeadDim) return cudaErrorNotSupported;
    if (!fits(heads, M, d) || !fits(heads, N, d)) return cudaErrorInvalidValue;
    TM_TRY(check_device());
    int device = 0;
    TM_TRY(cudaGetDevice(&device));

    // Chunk sizes: `chunk_heads` each, or by default ~heads/16 each with the
    // first and last two chunks at a quarter and a half of that, so the
    // pipeline fills (first H2D, nothing to overlap yet) and drains (last
    // kernels and D2H) quickly.
    std::vector<int> sizes;
    if (chunk_heads > 0) {
        const int c = std::min(chunk_heads, heads);
        for (int h0 = 0; h0 < heads; h0 += c) sizes.push_back(std::min(c, heads - h0));
    } else {
        const int c = std::max(1, (heads + 15) / 16);
        const int ramp[2] = {std::max(1, c / 4), std::max(1, c / 2)};
        int left = heads;
        std::vector<int> tail;
        for (int r = 0; r < 2 && left > 0; ++r) {            // ramp up
            sizes.push_back(std::min(ramp[r], left));
            left -= sizes.back();
        }
        for (int r = 0; r < 2 && left > 0; ++r) {            // ramp down (taken from the end)
            tail.push_back(std::min(ramp[r], left));
            left -= tail.back();
        }
        while (left > 0) {
            sizes.push_back(std::min(c, left));
            left -= sizes.back();
        }
        sizes.insert(sizes.end(), tail.rbegin(), tail.rend());
    }
    const int chunks = static_cast<int>(sizes.size());
    const std::size_t q_elems = static_cast<std::size_t>(M) * d;     // per head
    const std::size_t kv_elems = static_cast<std::size_t>(N) * d;
    const std::size_t words_per_head = routed ? tilemix_routing_word_count(M, N, g) : 0;
    const std::size_t q_scale_blocks = (static_cast<std::size_t>(M) - 1) / kTileMixQQuantRows + 1;
    const std::size_t k_scale_blocks = (static_cast<std::size_t>(N) - 1) / kTileMixKQuantRows + 1;
    auto* dq = static_cast<__half*>(dev->q);
    auto* dk = static_cast<__half*>(dev->k);
    auto* dv = static_cast<__half*>(dev->v);
    auto* dqs = static_cast<__half*>(dev->q_scales);
    auto* dks = static_cast<__half*>(dev->k_scales);

    PipelineContext& ctx = g_pipeline[device];
    std::lock_guard<std::mutex> lock(ctx.mu);
    TM_TRY(pipeline_context(ctx, 2 * static_cast<std::size_t>(chunks) + 2));
    cudaEvent_t start = ctx.events[0], done = ctx.events[1];
    TM_TRY(cudaEventRecord(start, stream));
    // From here on copies may be queued on the library's copy streams. If a
    // later step fails, `stream` is made to wait for both copy streams before
    // the error returns, so the caller's host buffers are no longer read or
    // written once `stream` reaches the point of the return.
    auto join_on_error = [&](cudaError_t failure) {
        if (cudaEventRecord(start, ctx.h2d) == cudaSuccess) cudaStreamWaitEvent(stream, start, 0);
        if (cudaEventRecord(done, ctx.d2h) == cudaSuccess) cudaStreamWaitEvent(stream, done, 0);
        return failure;
    };
#define TM_TRY_JOIN(expr)                                          \
    do {                                                           \
        const cudaError_t tm_status_ = (expr);                     \
        if (tm_status_ != cudaSuccess) return join_on_error(tm_status_); \
    } while (0)
    TM_TRY_JOIN(cudaStreamWaitEvent(ctx.h2d, start, 0));
    TM_TRY_JOIN(cudaStreamWaitEvent(ctx.d2h, start, 0));
    int h0 = 0;
    for (int c = 0; c < chunks; h0 += sizes[c], ++c) {
        const int hn = sizes[c];
        const std::size_t qo = h0 * q_elems, kvo = h0 * kv_elems;
        cudaEvent_t in = ctx.events[2 + 2 * c], out = ctx.events[3 + 2 * c];
        TM_TRY_JOIN(cudaMemcpyAsync(dq + qo, hQ + qo, hn * q_elems * sizeof(__half), cudaMemcpyHostToDevice, ctx.h2d));
        TM_TRY_JOIN(cudaMemcpyAsync(dk + kvo, hK + kvo, hn * kv_elems * sizeof(__half), cudaMemcpyHostToDevice, ctx.h2d));
        TM_TRY_JOIN(cudaMemcpyAsync(dv + kvo, hV + kvo, hn * kv_elems * sizeof(__half), cudaMemcpyHostToDevice, ctx.h2d));
        TileMixRouting routing{};
        routing.key_tiles_per_group = g;
        TileMixQuantized quantized{};
        if (routed) {
            const std::size_t wo = h0 * words_per_head;
            TM_TRY_JOIN(cudaMemcpyAsync(dev->words + wo, h_words + wo, hn * words_per_head * sizeof(std::uint64_t),
                                   cudaMemcpyHostToDevice, ctx.h2d));
            routing.words = dev->words + wo;
            routing.word_count = hn * words_per_head;
            quantized.q = dev->q8 + qo;
            quantized.k = dev->k8 + kvo;
            quantized.q_scales = dqs + h0 * q_scale_blocks;
            quantized.k_scales = dks + h0 * k_scale_blocks;
        }
        TM_TRY_JOIN(cudaEventRecord(in, ctx.h2d));
        TM_TRY_JOIN(cudaStreamWaitEvent(stream, in, 0));
        if (routed) {
            TM_TRY_JOIN(quantize_impl(dq + qo, dk + kvo, dev->q8 + qo, dev->k8 + kvo, dqs + h0 * q_scale_blocks,
                                 dks + h0 * k_scale_blocks, hn, M, N, d, stream));
        }
        TM_TRY_JOIN(attention_impl(dq + qo, dk + kvo, dv + kvo, dev->o + qo, hn, M, N, d, score_scale, causal, stream,
                              routing, quantized));
        TM_TRY_JOIN(cudaEventRecord(out, stream));
        TM_TRY_JOIN(cudaStreamWaitEvent(ctx.d2h, out, 0));
        TM_TRY_JOIN(cudaMemcpyAsync(hO + qo, dev->o + qo, hn * q_elems * sizeof(float), cudaMemcpyDeviceToHost, ctx.d2h));
    }
    TM_TRY_JOIN(cudaEventRecord(done, ctx.d2h));
    return cudaStreamWaitEvent(stream, done, 0);
}

#undef TM_TRY_JOIN
#undef TM_TRY

}  // namespace

// ------------------------------------------------------------- C++ drop-in API
cudaError_t quantize_tilemix_qk(const __half* Q, const __half* K, std::int8_t* Q8, std::int8_t* K8,
                                __half* q_scales, __half* k_scales, int M, int N, int d,
                                cudaStream_t stream) {
    return quantize_impl(Q, K, Q8, K8, q_scales, k_scales, 1, M, N, d, stream);
}

cudaError_t launch_fused_fp16_attention(const __half* Q, const __half* K, const __half* V, float* O,
                                        int M, int N, int d, float score_scale, cudaStream_t stream,
                                        const TileMixRouting& routing, const TileMixQuantized& quantized) {
    return attention_impl(Q, K, V, O, 1, M, N, d, score_scale, false, stream, routing, quantized);
}

std::size_t tilemix_b200_shared_bytes(int d, bool quantized) {
    (void)quantized;   // the kernel reserves the INT8 tiles either way
    return tilemix::attention_smem_bytes(d);
}

cudaError_t quantize_tilemix_qk_batched(const __half* Q, const __half* K, std::int8_t* Q8,
                                        std::int8_t* K8, __half* q_scales, __half* k_scales,
                                        int heads, int M, int N, int d, cudaStream_t stream) {
    return quantize_impl(Q, K, Q8, K8, q_scales, k_scales, heads, M, N, d, stream);
}

cudaError_t tilemix_attention_batched(const __half* Q, const __half* K, const __half* V, float* O,
                                      int heads, int M, int N, int d, float score_scale, bool causal,
                                      cudaStream_t stream, const TileMixRouting& routing,
                                      const TileMixQuantized& quantized) {
    return attention_impl(Q, K, V, O, heads, M, N, d, score_scale, causal, stream, routing, quantized);
}

cudaError_t tilemix_attention_batched_out(const __half* Q, const __half* K, const __half* V,
                                          const TileMixOutput& out, int heads, int M, int N, int d,
                                          float score_scale, bool causal, cudaStream_t stream,
                                          const TileMixRouting& routing, const TileMixQuantized& quantized) {
    return attention_impl(Q, K, V, nullptr, heads, M, N, d, score_scale, causal, stream, routing, quantized,
                          &out);
}

cudaError_t quantize_tilemix_k_batched(const __half* K, std::int8_t* K8, __half* k_scales, int heads, int N, int d,
                                       cudaStream_t stream) {
    return quantize_k_impl(K, K8, k_scales, heads, N, d, stream);
}

cudaError_t tilemix_attention_batched_qfused(const __half* Q, const __half* K, const __half* V, float* O, int heads,
                                             int M, int N, int d, float score_scale, bool causal, cudaStream_t stream,
                                             const TileMixRouting& routing, const std::int8_t* K8,
                                             const __half* k_scales, std::int8_t* Q8_out, __half* q_scales_out) {
    return attention_qfused_impl(Q, K, V, O, heads, M, N, d, score_scale, causal, stream, routing, K8, k_scales,
                                 Q8_out, q_scales_out);
}

cudaError_t quantize_tilemix_qkv_batched(const __half* Q, const __half* K, const __half* V, std::int8_t* Q8,
                                         std::int8_t* K8, __half* q_scales, __half* k_scales, __half* v_absmax,
                                         int heads, int M, int N, int d, cudaStream_t stream) {
    return quantize_qkv_impl(Q, K, V, Q8, K8, q_scales, k_scales, v_absmax, heads, M, N, d, stream);
}

cudaError_t tilemix_attention_batched_hinted(const __half* Q, const __half* K, const __half* V, float* O, int heads,
                                             int M, int N, int d, float score_scale, bool causal, cudaStream_t stream,
                                             const TileMixRouting& routing, const TileMixQuantized& quantized,
                                             const __half* v_absmax) {
    return attention_impl(Q, K, V, O, heads, M, N, d, score_scale, causal, stream, routing, quantized, nullptr, 0,
                          v_absmax);
}

cudaError_t tilemix_routing_policy(const __half* q_scales, const __half* k_scales, std::uint64_t* words, int heads,
                                   int M, int N, int key_tiles_per_group, float max_scale_product,
                                   cudaStream_t stream) {
    return routing_policy_impl(q_scales, k_scales, words, heads, M, N, key_tiles_per_group, max_scale_product,
                               stream);
}

cudaError_t tilemix_attention_batched_lse(const __half* Q, const __half* K, const __half* V, float* O, float* lse,
                                          int heads, int M, int N, int d, float score_scale, bool causal,
                                          cudaStream_t stream) {
    if (!lse) return cudaErrorInvalidValue;
    return attention_impl(Q, K, V, O, heads, M, N, d, score_scale, causal, stream, TileMixRouting{},
                          TileMixQuantized{}, nullptr, 0, nullptr, lse);
}

cudaError_t tilemix_attention_backward(const __half* Q, const __half* K, const __half* V, const float* O,
                                       const __half* dO, float* dQ, float* dK, float* dV, float* lse,
                                       float* dsum, int heads, int M, int N, int d, float score_scale,
                                       bool causal, bool lse_from_forward, cudaStream_t stream) {
    if (!Q || !K || !V || !O || !dO || !dQ || !dK || !dV || !lse || !dsum || heads <= 0 || M <= 0 || N <= 0 ||
        d <= 0 || !std::isfinite(score_scale)) {
        return cudaErrorInvalidValue;
    }
    if (d > tilemix::kBackwardMaxHeadDim || d % 16 != 0) return cudaErrorNotSupported;
    if (!fits(heads, M, d) || !fits(heads, N, d)) return cudaErrorInvalidValue;
    const cudaError_t status = check_device();
    if (status != cudaSuccess) return status;
    tilemix::AttentionBackwardProblem prob{};
    prob.q = Q; prob.k = K; prob.v = V; prob.o = O; prob.dout = dO;
    prob.dq = dQ; prob.dk = dK; prob.dv = dV; prob.lse = lse; prob.dsum = dsum;
    prob.heads = heads; prob.M = M; prob.N = N; prob.d = d;
    prob.score_scale = score_scale;
    prob.causal = causal;
    prob.lse_ready = lse_from_forward;
    return tilemix::launch_attention_backward(prob, stream);
}

// ---------------------------------------------------------------------- C-ABI
extern "C" {

int tilemix_abi_version(void) { return TILEMIX_ABI_VERSION; }

int tilemix_quantize_qk(const void* Q, const void* K, int8_t* Q8, int8_t* K8, void* q_scales,
                        void* k_scales, int M, int N, int d, void* stream) {
    return static_cast<int>(quantize_impl(static_cast<const __half*>(Q), static_cast<const __half*>(K),
                                          Q8, K8, static_cast<__half*>(q_scales),
                                          static_cast<__half*>(k_scales), 1, M, N, d,
                                          static_cast<cudaStream_t>(stream)));
}

int tilemix_fused_attention(const void* Q, const void* K, const void* V, float* O, int M, int N,
                            int d, float score_scale, void* stream, const tilemix_routing* routing,
                            const tilemix_quantized* quantized) {
    return static_cast<int>(attention_impl(static_cast<const __half*>(Q), static_cast<const __half*>(K),
                                           static_cast<const __half*>(V), O, 1, M, N, d, score_scale,
                                           false, static_cast<cudaStream_t>(stream), to_cpp(routing),
                                           to_cpp(quantized)));
}

int tilemix_quantize_qk_batched(const void* Q, const void* K, int8_t* Q8, int8_t* K8, void* q_scales,
                                void* k_scales, int heads, int M, int N, int d, void* stream) {
    return static_cast<int>(quantize_impl(static_cast<const __half*>(Q), static_cast<const __half*>(K),
                                          Q8, K8, static_cast<__half*>(q_scales),
                                          static_cast<__half*>(k_scales), heads, M, N, d,
                                          static_cast<cudaStream_t>(stream)));
}

int tilemix_attention_batched(const void* Q, const void* K, const void* V, float* O, int heads,
                              int M, int N, int d, float score_scale, int causal, void* stream,
                              const tilemix_routing* routing, const tilemix_quantized* quantized) {
    return static_cast<int>(attention_impl(static_cast<const __half*>(Q), static_cast<const __half*>(K),
                                           static_cast<const __half*>(V), O, heads, M, N, d,
                                           score_scale, causal != 0, static_cast<cudaStream_t>(stream),
                                           to_cpp(routing), to_cpp(quantized)));
}

int tilemix_attention_batched_out(const void* Q, const void* K, const void* V, const tilemix_output* out,
                                  int heads, int M, int N, int d, float score_scale, int causal, void* stream,
                                  const tilemix_routing* routing, const tilemix_quantized* quantized) {
    if (!out) return static_cast<int>(cudaErrorInvalidValue);
    TileMixOutput o;
    o.data = out->data;
    o.dtype = out->dtype;
    o.heads_per_batch = out->heads_per_batch;
    o.stride_batch = out->stride_batch;
    o.stride_head = out->stride_head;
    o.stride_row = out->stride_row;
    return static_cast<int>(attention_impl(static_cast<const __half*>(Q), static_cast<const __half*>(K),
                                           static_cast<const __half*>(V), nullptr, heads, M, N, d, score_scale,
                                           causal != 0, static_cast<cudaStream_t>(stream), to_cpp(routing),
                                           to_cpp(quantized), &o));
}

int tilemix_attention_from_host(const void* hQ, const void* hK, const void* hV, const uint64_t* h_words,
                                float* hO, const tilemix_device_buffers* dev, int heads, int M, int N, int d,
                                float score_scale, int causal, int key_tiles_per_group, int chunk_heads,
                                void* stream) {
    return static_cast<int>(from_host_impl(static_cast<const __half*>(hQ), static_cast<const __half*>(hK),
                                           static_cast<const __half*>(hV), h_words, hO, dev, heads, M, N, d,
                                           score_scale, causal != 0, key_tiles_per_group, chunk_heads,
                                           static_cast<cudaStream_t>(stream)));
}

int tilemix_quantize_k_batched(const void* K, int8_t* K8, void* k_scales, int heads, int N, int d, void* stream) {
    return static_cast<int>(quantize_k_impl(static_cast<const __half*>(K), K8, static_cast<__half*>(k_scales), heads,
                                            N, d, static_cast<cudaStream_t>(stream)));
}

int tilemix_attention_batched_qfused(const void* Q, const void* K, const void* V, float* O, int heads, int M, int N,
                                     int d, float score_scale, int causal, void* stream,
                                     const tilemix_routing* routing, const int8_t* K8, const void* k_scales,
                                     int8_t* Q8_out, void* q_scales_out) {
    return static_cast<int>(attention_qfused_impl(
        static_cast<const __half*>(Q), static_cast<const __half*>(K), static_cast<const __half*>(V), O, heads, M, N,
        d, score_scale, causal != 0, static_cast<cudaStream_t>(stream), to_cpp(routing), K8,
        static_cast<const __half*>(k_scales), Q8_out, static_cast<__half*>(q_scales_out)));
}

int tilemix_quantize_qkv_batched(const void* Q, const void* K, const void* V, int8_t* Q8, int8_t* K8, void* q_scales,
                                  void* k_scales, void* v_absmax, int heads, int M, int N, int d, void* stream) {
    return static_cast<int>(quantize_qkv_impl(static_cast<const __half*>(Q), static_cast<const __half*>(K),
                                              static_cast<const __half*>(V), Q8, K8, static_cast<__half*>(q_scales),
                                              static_cast<__half*>(k_scales), static_cast<__half*>(v_absmax), heads,
                                              M, N, d, static_cast<cudaStream_t>(stream)));
}

int tilemix_attention_batched_hinted(const void* Q, const void* K, const void* V, float* O, int heads, int M, int N,
                                     int d, float score_scale, int causal, void* stream,
                                     const tilemix_routing* routing, const tilemix_quantized* quantized,
                                     const void* v_absmax) {
    return static_cast<int>(attention_impl(static_cast<const __half*>(Q), static_cast<const __half*>(K),
                                           static_cast<const __half*>(V), O, heads, M, N, d, score_scale,
                                           causal != 0, static_cast<cudaStream_t>(stream), to_cpp(routing),
                                           to_cpp(quantized), nullptr, 0, static_cast<const __half*>(v_absmax)));
}

int tilemix_routing_policy_c(const void* q_scales, const void* k_scales, uint64_t* words, int heads, int M, int N,
                             int key_tiles_per_group, float max_scale_product, void* stream) {
    return static_cast<int>(routing_policy_impl(static_cast<const __half*>(q_scales),
                                                static_cast<const __half*>(k_scales), words, heads, M, N,
                                                key_tiles_per_group, max_scale_product,
                                                static_cast<cudaStream_t>(stream)));
}

float tilemix_policy_max_scale_product_c(float tolerance, float score_scale, int d) {
    return tilemix_policy_max_scale_product(tolerance, score_scale, d);
}

size_t tilemix_routing_word_count_c(int M, int N, int key_tiles_per_group) {
    return tilemix_routing_word_count(M, N, key_tiles_per_group);
}

size_t tilemix_routing_words_per_row_c(int N, int key_tiles_per_group) {
    return tilemix_routing_words_per_row(N, key_tiles_per_group);
}

size_t tilemix_reference_shared_bytes(int d, int quantized) {
    return tilemix_shared_bytes(d, quantized != 0);
}

size_t tilemix_b200_shared_bytes_c(int d, int quantized) {
    return tilemix_b200_shared_bytes(d, quantized != 0);
}

int tilemix_watchdog_selftest(const void* Q, const void* K, const void* V, float* O, int heads, int M, int N,
                              int d, float score_scale, unsigned int wait_limit_us, void* stream) {
    if (wait_limit_us == 0 || wait_limit_us > 1000000u) return static_cast<int>(cudaErrorInvalidValue);
    return static_cast<int>(attention_impl(static_cast<const __half*>(Q), static_cast<const __half*>(K),
                                           static_cast<const __half*>(V), O, heads, M, N, d, score_scale, false,
                                           static_cast<cudaStream_t>(stream), TileMixRouting{}, TileMixQuantized{},
                                           nullptr, 1000ull * wait_limit_us));
}

int tilemix_attention_batched_lse_c(const void* Q, const void* K, const void* V, float* O, float* lse, int heads,
                                    int M, int N, int d, float score_scale, int causal, void* stream) {
    return static_cast<int>(tilemix_attention_batched_lse(static_cast<const __half*>(Q), static_cast<const __half*>(K),
                                                          static_cast<const __half*>(V), O, lse, heads, M, N, d,
                                                          score_scale, causal != 0,
                                                          static_cast<cudaStream_t>(stream)));
}

int tilemix_attention_backward_c(const void* Q, const void* K, const void* V, const float* O, const void* dO,
                                 float* dQ, float* dK, float* dV, float* lse, float* dsum, int heads, int M, int N,
                                 int d, float score_scale, int causal, int lse_from_forward, void* stream) {
    return static_cast<int>(tilemix_attention_backward(
        static_cast<const __half*>(Q), static_cast<const __half*>(K), static_cast<const __half*>(V), O,
        static_cast<const __half*>(dO), dQ, dK, dV, lse, dsum, heads, M, N, d, score_scale, causal != 0,
        lse_from_forward != 0, static_cast<cudaStream_t>(stream)));
}

int tilemix_backward_watchdog_selftest(const void* Q, const void* K, const void* V, const float* O, const void* dO,
                                       float* dQ, float* dK, float* dV, float* lse, float* dsum, int heads, int M,
                                       int N, int d, float score_scale, unsigned int wait_limit_us, void* stream) {
    if (wait_limit_us == 0 || wait_limit_us > 1000000u) return static_cast<int>(cudaErrorInvalidValue);
    if (!Q || !K || !V || !O || !dO || !dQ || !dK || !dV || !lse || !dsum || heads <= 0 || M <= 0 || N <= 0 ||
        d <= 0 || !std::isfinite(score_scale)) {
        return static_cast<int>(cudaErrorInvalidValue);
    }
    if (d != 128) return static_cast<int>(cudaErrorNotSupported);
    if (!fits(heads, M, d) || !fits(heads, N, d)) return static_cast<int>(cudaErrorInvalidValue);
    const cudaError_t status = check_device();
    if (status != cudaSuccess) return static_cast<int>(status);
    tilemix::AttentionBackwardProblem prob{};
    prob.q = static_cast<const __half*>(Q); prob.k = static_cast<const __half*>(K);
    prob.v = static_cast<const __half*>(V); prob.o = O; prob.dout = static_cast<const __half*>(dO);
    prob.dq = dQ; prob.dk = dK; prob.dv = dV; prob.lse = lse; prob.dsum = dsum;
    prob.heads = heads; prob.M = M; prob.N = N; prob.d = d;
    prob.score_scale = score_scale;
    prob.watchdog_limit_ns = 1000ull * wait_limit_us;
    return static_cast<int>(tilemix::launch_attention_backward(prob, static_cast<cudaStream_t>(stream)));
}

int tilemix_read_and_clear_status(unsigned int* status) {
    if (!status) return static_cast<int>(cudaErrorInvalidValue);
    return static_cast<int>(tilemix::read_and_clear_status(status));
}

}  // extern "C"
