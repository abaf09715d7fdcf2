// Device-side routing policy: reference-format routing words chosen from the
// quantizer's block scales (no reference counterpart; the reference only takes
// a mask from the caller, src/main.cu:48).
//
// Policy: with scales s = absmax / 127, the INT8 score of a query row q and a
// key k differs from the fp32 one by at most
//   |score_scale| * d * (127 + 1/4) * s_q * s_k
// (each quantized element is off by at most s / 2 and |x| <= 127 s). A
// (16-row query tile, group of key_tiles_per_group 32-key tiles) pair is
// routed INT8 iff s_q * max s_k <= max_scale_product, with s_q the scale of the
// tile's 128-row Q block and the max over the 64-row K blocks the group's keys
// touch; outlier blocks (large absmax, coarse INT8 steps) stay FP16. Products
// are fp32 of the fp16 scales (exact inputs, one rounding); NaN routes FP16.
// The words follow src/tilemix.cu:99-103: bit (group % 64) of word
// (q16 * words_per_row + group / 64), LSB first, 1 = INT8; bits past the last
// group are 0.
//
// One thread per routing word (64 groups): HBM-trivial (the scales are a few
// KB per head), so the kernel is launch-bound and simple.
#include "kernels.cuh"

#include <cstdint>

namespace tilemix {
namespace {

struct PolicyParams {
    const __half* q_scales;     // [heads][q_blocks]
    const __half* k_scales;     // [heads][k_blocks]
    std::uint64_t* words;       // [heads][q16_tiles][words_per_row]
    long long total_words;
    int q16_tiles, words_per_row, q_blocks, k_blocks, k32_tiles, group, groups, n;
    float max_product;
};

__global__ void __launch_bounds__(256) routing_policy_kernel(const PolicyParams p) {
    const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= p.total_words) return;
    const long long per_head = static_cast<long long>(p.q16_tiles) * p.words_per_row;
    const int head = static_cast<int>(idx / per_head);
    const long long in_head = idx - head * per_head;
    const int q16 = static_cast<int>(in_head / p.words_per_row);
    const int w = static_cast<int>(in_head - static_cast<long long>(q16) * p.words_per_row);
    const float sq = __half2float(p.q_scales[static_cast<long long>(head) * p.q_blocks + q16 / 8]);
    const __half* ks = p.k_scales + static_cast<long long>(head) * p.k_blocks;
    std::uint64_t word = 0;
    for (int b = 0; b < 64; ++b) {
        const int group = w * 64 + b;
        if (group >= p.groups) break;
        // keys of the group: key tiles [group * g, min(group * g + g, k32_tiles))
        const long long kt0 = static_cast<long long>(group) * p.group;
        const long long kt1 = min(kt0 + p.group, static_cast<long long>(p.k32_tiles));
        const int key0 = static_cast<int>(kt0 * 32);
        const int key1 = static_cast<int>(min(kt1 * 32, static_cast<long long>(p.n)));   // exclusive
        float skmax = 0.0f;
        bool nan = false;
        for (int kb = key0 / 64; kb <= (key1 - 1) / 64; ++kb) {
            const float s = __half2float(ks[kb]);
            nan |= s != s;
            skmax = fmaxf(skmax, s);
        }
        const float product = __fmul_rn(sq, skmax);
        if (!nan && product <= p.max_product) word |= 1ull << b;
    }
    p.words[idx] = word;
}

}  // namespace

cudaError_t launch_routing_policy(const __half* q_scales, const __half* k_scales, std::uint64_t* words, int heads,
                                  int M, int N, int key_tiles_per_group, float max_scale_product,
                                  cudaStream_t stream) {
    PolicyParams p{};
    p.q_scales = q_scales;
    p.k_scales = k_scales;
    p.words = words;
    p.q16_tiles = (M - 1) / 16 + 1;
    p.k32_tiles = (N - 1) / 32 + 1;
    const long long groups = (static_cast<long long>(p.k32_tiles) - 1) / key_tiles_per_group + 1;
    p.groups = static_cast<int>(groups);
    p.group = key_tiles_per_group;
    p.words_per_row = static_cast<int>((groups - 1) / 64 + 1);
    p.q_blocks = (M - 1) / kQuantQRows + 1;
    p.k_blocks = (N - 1) / kQuantKRows + 1;
    p.n = N;
    p.max_product = max_scale_product;
    p.total_words = static_cast<long long>(heads) * p.q16_tiles * p.words_per_row;
    const long long blocks = (p.total_words + 255) / 256;
    if (blocks > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
    routing_policy_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace tilemix
