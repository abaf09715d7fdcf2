// TileMix demo / benchmark driver against the drop-in C++ API.
//
// Runs the reference driver's problem (src/main.cu:24-63 of the reference:
// M=1000, N=1003, d=128, two 32-key tiles per routing group, every odd group
// INT8 via the 0xaaaa... mask, periodic inputs) through quantize_tilemix_qk and
// launch_fused_fp16_attention and prints output[0] in the same format.
// `tilemix_demo --time [iters]` additionally times the pair with CUDA events.
#include "attention_fused.h"

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <stdexcept>
#include <vector>

namespace {
void ok(cudaError_t e, const char* what) {
    if (e != cudaSuccess) {
        std::fprintf(stderr, "%s: %s\n", what, cudaGetErrorString(e));
        throw std::runtime_error(what);
    }
}

template <class T> struct Device {
    T* ptr = nullptr;
    explicit Device(std::size_t n) { ok(cudaMalloc(&ptr, n * sizeof(T)), "cudaMalloc"); }
    ~Device() { cudaFree(ptr); }
    Device(const Device&) = delete;
    Device& operator=(const Device&) = delete;
};
}  // namespace

int main(int argc, char** argv) {
    try {
        const int M = 1000, N = 1003, d = 128, group = 2;
        const bool timing = argc >= 2 && std::strcmp(argv[1], "--time") == 0;
        const int iters = argc >= 3 ? std::atoi(argv[2]) : 20;
        const std::size_t qn = static_cast<std::size_t>(M) * d, kn = static_cast<std::size_t>(N) * d;
        const std::size_t words = tilemix_routing_word_count(M, N, group);
        const int q_blocks = (M - 1) / kTileMixQQuantRows + 1, k_blocks = (N - 1) / kTileMixKQuantRows + 1;

        std::vector<__half> hq(qn), hk(kn), hv(kn);
        for (std::size_t i = 0; i < qn; ++i) hq[i] = __float2half(0.125f * (static_cast<int>(i % 17) - 8));
        for (std::size_t i = 0; i < kn; ++i) hk[i] = __float2half(0.125f * (static_cast<int>(i % 19) - 9));
        for (std::size_t i = 0; i < kn; ++i) hv[i] = __float2half(0.1f * (static_cast<int>(i % 23) - 11));
        const std::vector<std::uint64_t> mask(words, 0xaaaaaaaaaaaaaaaaull);

        Device<__half> q(qn), k(kn), v(kn), qs(q_blocks), ks(k_blocks);
        Device<std::int8_t> q8(qn), k8(kn);
        Device<float> out(qn);
        Device<std::uint64_t> w(words);
        ok(cudaMemcpy(q.ptr, hq.data(), qn * 2, cudaMemcpyHostToDevice), "copy Q");
        ok(cudaMemcpy(k.ptr, hk.data(), kn * 2, cudaMemcpyHostToDevice), "copy K");
        ok(cudaMemcpy(v.ptr, hv.data(), kn * 2, cudaMemcpyHostToDevice), "copy V");
        ok(cudaMemcpy(w.ptr, mask.data(), words * 8, cudaMemcpyHostToDevice), "copy mask");

        const TileMixRouting routing{w.ptr, words, group};
        const TileMixQuantized quantized{q8.ptr, k8.ptr, qs.ptr, ks.ptr};
        const float scale = 1.0f / std::sqrt(static_cast<float>(d));
        auto run = [&] {
            ok(quantize_tilemix_qk(q.ptr, k.ptr, q8.ptr, k8.ptr, qs.ptr, ks.ptr, M, N, d), "quantize");
            ok(launch_fused_fp16_attention(q.ptr, k.ptr, v.ptr, out.ptr, M, N, d, scale, nullptr,
                                           routing, quantized), "attention");
        };
        run();
        ok(cudaDeviceSynchronize(), "sync");
        std::vector<float> result(qn);
        ok(cudaMemcpy(result.data(), out.ptr, qn * 4, cudaMemcpyDeviceToHost), "copy O");
        std::printf("TileMix attention: M=%d N=%d d=%d output[0]=%.9g\n", M, N, d, result[0]);
        std::printf("Routing: %d key tiles/group, %zu packed words; bit 0=FP16, bit 1=INT8 tcgen05\n",
                    group, words);
        if (timing) {
            cudaEvent_t a, b;
            ok(cudaEventCreate(&a), "event");
            ok(cudaEventCreate(&b), "event");
            for (int i = 0; i < 3; ++i) run();
            ok(cudaEventRecord(a), "record");
            for (int i = 0; i < iters; ++i) run();
            ok(cudaEventRecord(b), "record");
            ok(cudaEventSynchronize(b), "sync");
            float ms = 0.0f;
            ok(cudaEventElapsedTime(&ms, a, b), "elapsed");
            const double flops = 4.0 * M * N * d;
            std::printf("time %.4f ms/iter, %.3f TFLOP/s effective\n", ms / iters,
                        flops / (ms / iters * 1e-3) / 1e12);
        }
        return 0;
    } catch (const std::exception& e) {
        std::fprintf(stderr, "ERROR: %s\n", e.what());
        return 1;
    }
}
