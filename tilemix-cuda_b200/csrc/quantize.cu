// Stage 1: per-block symmetric INT8 quantizer for Q (128-row blocks) and K
// (64-row blocks), one launch for both tensors and all heads.
//
// Semantics follow the reference (src/tilemix.cu:16-49,
// src/tests/reference_tilemix.h:16-41) bit for bit:
//   absmax  = max |x| in fp32 over the block (NaN never replaces the max)
//   scale   = __fdiv_rn(absmax, 127)            (fp32, stored as fp16 RN)
//   q       = clamp(rz(x/scale + copysign(0.5, x/scale)), -127, 127),
//             x/scale by __fdiv_rn, 0 when scale == 0
// i.e. round half AWAY from zero on the fp32 quotient.
//
// B200 design: the block is read from HBM once. Each CTA owns one block
// (<= 128 x 128 fp16 = 32 KB), its 256 threads hold the block in registers
// (up to 8 x 16-byte loads each), reduce the absmax with warp shuffles, then
// quantize from registers with the branch-free exact rounding of
// quant_math.cuh (blocks holding NaN or inf keep the element-wise exact
// path) and write 8-byte stores: 3 bytes of HBM traffic per element, the
// algorithmic minimum. Unaligned pointers or d % 8 != 0 take a
// scalar two-pass path (the second pass hits L2).
#include "kernels.cuh"
#include "quant_math.cuh"

#include <cstdint>

namespace tilemix {
namespace {

constexpr int kQuantThreads = 256;
constexpr int kMaxChunksPerThread = 8;   // 128 rows x 128 d / 8 halves / 256 threads

// NaN-propagating max of two floats (a NaN anywhere in a block must reach
// the block's verdict, unlike fmaxf).
__device__ __forceinline__ float max_nan(float a, float b) { return (a != a || b != b) ? NAN : fmaxf(a, b); }

// Block absmax from per-thread maxima, NaN-propagating (values are exact fp16
// magnitudes, so the float reduction is exact).
__device__ __forceinline__ float block_max_nan(float value, float* scratch) {
    #pragma unroll
    for (int offset = 16; offset > 0; offset >>= 1) {
        value = max_nan(value, __shfl_xor_sync(0xffffffffu, value, offset));
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) scratch[warp] = value;
    __syncthreads();
    float total = 0.0f;
    #pragma unroll
    for (int w = 0; w < kQuantThreads / 32; ++w) total = max_nan(total, scratch[w]);
    return total;
}

__device__ __forceinline__ float block_max(float value, float* scratch) {
    #pragma unroll
    for (int offset = 16; offset > 0; offset >>= 1) {
        value = fmaxf(value, __shfl_xor_sync(0xffffffffu, value, offset));
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) scratch[warp] = value;
    __syncthreads();
    float total = 0.0f;
    #pragma unroll
    for (int w = 0; w < kQuantThreads / 32; ++w) total = fmaxf(total, scratch[w]);
    return total;
}

struct QuantTensor {
    const __half* x;
    std::int8_t* values;
    __half* scales;
    int rows;
    int block_rows;
    int blocks;      // per head
    bool vector_ok;  // 16-byte aligned input, 8-byte aligned output, d % 8 == 0
};

__global__ void __launch_bounds__(kQuantThreads, 4)
quantize_blocks_kernel(QuantTensor qt, QuantTensor kt, QuantTensor vt, int heads, int d) {
    __shared__ float scratch[kQuantThreads / 32];
    // CTAs [0, q) quantize Q blocks, [q, q + k) K blocks, the rest record the
    // absmax of V blocks (vt.values == nullptr: statistics only)
    const int q_ctas = heads * qt.blocks, k_ctas = heads * kt.blocks;
    const int bid = static_cast<int>(blockIdx.x);
    const bool is_q = bid < q_ctas, is_k = !is_q && bid < q_ctas + k_ctas;
    const QuantTensor& t = is_q ? qt : is_k ? kt : vt;
    const int cta = is_q ? bid : is_k ? bid - q_ctas : bid - q_ctas - k_ctas;
    const int head = cta / t.blocks, block = cta % t.blocks;
    const int first_row = block * t.block_rows;
    const int rows_here = min(t.block_rows, t.rows - first_row);
    const std::size_t base = (static_cast<std::size_t>(head) * t.rows + first_row) * d;
    const int count = rows_here * d;
    const __half* src = t.x + base;
    std::int8_t* dst = t.values + base;

    if (t.vector_ok) {
        uint4 chunk[kMaxChunksPerThread];
        const int chunks = count >> 3;
        // absmax on packed halves (|x| and max are exact in fp16), NaN-
        // propagating so that a block holding a NaN takes the exact path
        __half2 m2 = __float2half2_rn(0.0f);
        #pragma unroll
        for (int i = 0; i < kMaxChunksPerThread; ++i) {
            const int c = threadIdx.x + i * kQuantThreads;
            if (c < chunks) {
                chunk[i] = __ldg(reinterpret_cast<const uint4*>(src) + c);
                const __half2* h = reinterpret_cast<const __half2*>(&chunk[i]);
                #pragma unroll
                for (int e = 0; e < 4; ++e) m2 = __hmax2_nan(m2, __habs2(h[e]));
            }
        }
        const float absmax = block_max_nan(max_nan(__low2float(m2), __high2float(m2)), scratch);
        if (!t.values) {   // V statistics: the block's max |v| (exact in fp16; NaN if the block holds one)
            if (threadIdx.x == 0) t.scales[static_cast<std::size_t>(head) * t.blocks + block] = __float2half_rn(absmax);
            return;
        }
        if (fast_block(absmax)) {
            // every block of finite, not-all-zero inputs: branch-free exact rounding
            const float scale = __fdiv_rn(absmax, 127.0f);
            const float y = __frcp_rn(scale);
            const float2 neg_s2 = make_float2(-scale, -scale), y2 = make_float2(y, y);
            if (threadIdx.x == 0) t.scales[static_cast<std::size_t>(head) * t.blocks + block] = __float2half_rn(scale);
            #pragma unroll
            for (int i = 0; i < kMaxChunksPerThread; ++i) {
                const int c = threadIdx.x + i * kQuantThreads;
                if (c < chunks) {
                    reinterpret_cast<uint2*>(dst)[c] = make_uint2(quantize4_fast(chunk[i].x, chunk[i].y, neg_s2, y2),
                                                                  quantize4_fast(chunk[i].z, chunk[i].w, neg_s2, y2));
                }
            }
            return;
        }
        // NaN, +-inf or an all-zero block (uniform over the block): the
        // absmax without NaN, then the element-wise exact rounding
        m2 = __float2half2_rn(0.0f);
        #pragma unroll
        for (int i = 0; i < kMaxChunksPerThread; ++i) {
            const int c = threadIdx.x + i * kQuantThreads;
            if (c < chunks) {
                const __half2* h = reinterpret_cast<const __half2*>(&chunk[i]);
                #pragma unroll
                for (int e = 0; e < 4; ++e) m2 = __hmax2(m2, __habs2(h[e]));   // ignores a NaN like fmaxf
            }
        }
        __syncthreads();   // every thread has read the first reduction's scratch
        const float local = fmaxf(__low2float(m2), __high2float(m2));
        const float scale = __fdiv_rn(block_max(local, scratch), 127.0f);
        const float recip = scale > 0.0f ? __frcp_rn(scale) : 0.0f;
        const float2 recip2 = make_float2(recip, recip);
        if (threadIdx.x == 0) t.scales[static_cast<std::size_t>(head) * t.blocks + block] = __float2half_rn(scale);
        #pragma unroll
        for (int i = 0; i < kMaxChunksPerThread; ++i) {
            const int c = threadIdx.x + i * kQuantThreads;
            if (c < chunks) {
                const __half2* h = reinterpret_cast<const __half2*>(&chunk[i]);
                uint32_t packed[2] = {0u, 0u};
                #pragma unroll
                for (int e = 0; e < 4; ++e) packed[e >> 1] |= quantize_pair(h[e], scale, recip2) << ((e & 1) * 16);
                reinterpret_cast<uint2*>(dst)[c] = make_uint2(packed[0], packed[1]);
            }
        }
    } else {
        if (!t.values) {   // V statistics (NaN-propagating, as on the vector path)
            float vmax = 0.0f;
            for (int i = threadIdx.x; i < count; i += kQuantThreads) vmax = max_nan(vmax, fabsf(__half2float(src[i])));
            const float absmax = block_max_nan(vmax, scratch);
            if (threadIdx.x == 0) t.scales[static_cast<std::size_t>(head) * t.blocks + block] = __float2half_rn(absmax);
            return;
        }
        float local = 0.0f;
        for (int i = threadIdx.x; i < count; i += kQuantThreads) {
            local = fmaxf(local, fabsf(__half2float(src[i])));
        }
        const float scale = __fdiv_rn(block_max(local, scratch), 127.0f);
        if (threadIdx.x == 0) t.scales[static_cast<std::size_t>(head) * t.blocks + block] = __float2half_rn(scale);
        for (int i = threadIdx.x; i < count; i += kQuantThreads) {
            dst[i] = quantize_exact(__half2float(src[i]), scale);
        }
    }
}

bool aligned(const void* p, std::uintptr_t bytes) {
    return (reinterpret_cast<std::uintptr_t>(p) & (bytes - 1)) == 0;
}

}  // namespace

cudaError_t launch_quantize(const __half* Q, const __half* K, std::int8_t* Q8, std::int8_t* K8,
                            __half* q_scales, __half* k_scales, int heads, int M, int N, int d,
                            cudaStream_t stream) {
    QuantTensor qt{Q, Q8, q_scales, M, kQuantQRows, (M - 1) / kQuantQRows + 1,
                   d % 8 == 0 && aligned(Q, 16) && aligned(Q8, 8)};
    QuantTensor kt{K, K8, k_scales, N, kQuantKRows, (N - 1) / kQuantKRows + 1,
                   d % 8 == 0 && aligned(K, 16) && aligned(K8, 8)};
    const long long ctas = static_cast<long long>(heads) * (qt.blocks + kt.blocks);
    if (ctas > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
    const QuantTensor none{nullptr, nullptr, nullptr, 0, kQuantKRows, 0, false};   // no V statistics
    quantize_blocks_kernel<<<static_cast<unsigned>(ctas), kQuantThreads, 0, stream>>>(qt, kt, none, heads, d);
    return cudaGetLastError();
}

cudaError_t launch_quantize_k(const __half* K, std::int8_t* K8, __half* k_scales, int heads, int N, int d,
                              cudaStream_t stream) {
    QuantTensor none{nullptr, nullptr, nullptr, 0, kQuantQRows, 0, false};   // no Q blocks
    QuantTensor kt{K, K8, k_scales, N, kQuantKRows, (N - 1) / kQuantKRows + 1,
                   d % 8 == 0 && aligned(K, 16) && aligned(K8, 8)};
    const long long ctas = static_cast<long long>(heads) * kt.blocks;
    if (ctas > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
    quantize_blocks_kernel<<<static_cast<unsigned>(ctas), kQuantThreads, 0, stream>>>(none, kt, none, heads, d);
    return cudaGetLastError();
}

cudaError_t launch_quantize_qkv(const __half* Q, const __half* K, const __half* V, std::int8_t* Q8, std::int8_t* K8,
                                __half* q_scales, __half* k_scales, __half* v_absmax, int heads, int M, int N,
                                int d, cudaStream_t stream) {
    QuantTensor qt{Q, Q8, q_scales, M, kQuantQRows, (M - 1) / kQuantQRows + 1,
                   d % 8 == 0 && aligned(Q, 16) && aligned(Q8, 8)};
    QuantTensor kt{K, K8, k_scales, N, kQuantKRows, (N - 1) / kQuantKRows + 1,
                   d % 8 == 0 && aligned(K, 16) && aligned(K8, 8)};
    QuantTensor vt{V, nullptr, v_absmax, N, kQuantKRows, (N - 1) / kQuantKRows + 1, d % 8 == 0 && aligned(V, 16)};
    const long long ctas = static_cast<long long>(heads) * (qt.blocks + kt.blocks + vt.blocks);
    if (ctas > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
    quantize_blocks_kernel<<<static_cast<unsigned>(ctas), kQuantThreads, 0, stream>>>(qt, kt, vt, heads, d);
    return cudaGetLastError();
}

}  // namespace tilemix
