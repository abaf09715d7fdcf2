// C-ABI shim over the reference's OWN CPU oracle headers -- TEST INFRASTRUCTURE.
//
// Compiled by oracle/build_ref.sh directly against the headers where they lie
// in the reference tree (src/tests/reference_tilemix.h and
// src/tests/reference_attention.h); nothing from the reference is copied into
// this repository. The resulting oracle/_ref/libtilemix_ref.so pins the C
// restatement in tilemix_oracle.c (tests compare the two) and serves as the
// timed CPU baseline ("kind": "reference") in bench.py.
#include "reference_attention.h"
#include "reference_tilemix.h"

#include <cstdint>
#include <cstring>
#include <vector>
#ifdef _OPENMP
#include <omp.h>
#endif

namespace {
std::vector<__half> halves(const std::uint16_t* bits, std::size_t count) {
    std::vector<__half> out(count);
    std::memcpy(out.data(), bits, count * sizeof(std::uint16_t));
    return out;
}
}  // namespace

extern "C" {

// reference_quantize (reference_tilemix.h:16-41).
void ref_quantize(const std::uint16_t* x, int rows, int d, int block_rows,
                  std::int8_t* values, std::uint16_t* scales) {
    const auto input = halves(x, static_cast<std::size_t>(rows) * d);
    const ReferenceQuantized result = reference_quantize(input, rows, d, block_rows);
    std::memcpy(values, result.values.data(), result.values.size());
    std::memcpy(scales, result.scales.data(), result.scales.size() * sizeof(std::uint16_t));
}

// reference_int8_dot (reference_tilemix.h:43-51).
std::int32_t ref_int8_dot(const std::int8_t* q8, const std::int8_t* k8, int M, int N,
                          int query, int key, int d) {
    ReferenceQuantized q{std::vector<std::int8_t>(q8, q8 + static_cast<std::size_t>(M) * d), {}};
    ReferenceQuantized k{std::vector<std::int8_t>(k8, k8 + static_cast<std::size_t>(N) * d), {}};
    return reference_int8_dot(q, k, query, key, d);
}

// reference_tilemix (reference_tilemix.h:53-89) for a whole [M,d] x [N,d] head.
// routes: one byte per (16-row query tile, 32-key tile).
void ref_tilemix(const std::uint16_t* q, const std::uint16_t* k, const std::uint16_t* v,
                 const std::int8_t* q8, const std::uint16_t* q_scales,
                 const std::int8_t* k8, const std::uint16_t* k_scales,
                 const std::uint8_t* routes, int M, int N, int d, float score_scale,
                 double* out) {
    const std::size_t qn = static_cast<std::size_t>(M) * d, kn = static_cast<std::size_t>(N) * d;
    const int q_blocks = (M - 1) / 128 + 1, k_blocks = (N - 1) / 64 + 1;
    ReferenceQuantized rq{std::vector<std::int8_t>(q8, q8 + qn), halves(q_scales, q_blocks)};
    ReferenceQuantized rk{std::vector<std::int8_t>(k8, k8 + kn), halves(k_scales, k_blocks)};
    const std::size_t route_count = static_cast<std::size_t>((M + 15) / 16) * ((N + 31) / 32);
    const std::vector<std::uint8_t> r(routes, routes + route_count);
    const auto result = reference_tilemix(halves(q, qn), halves(k, kn), halves(v, kn), rq, rk, r,
                                          M, N, d, 16, 32, score_scale);
    std::memcpy(out, result.data(), result.size() * sizeof(double));
}

// reference_attention (reference_attention.h:12-52).
void ref_attention(const std::uint16_t* q, const std::uint16_t* k, const std::uint16_t* v,
                   int M, int N, int d, double* out) {
    const auto hq = halves(q, static_cast<std::size_t>(M) * d);
    const auto hk = halves(k, static_cast<std::size_t>(N) * d);
    const auto hv = halves(v, static_cast<std::size_t>(N) * d);
    reference_attention(hq.data(), hk.data(), hv.data(), out, M, N, d);
}

// Sampled rows of a [heads, M, d] batch through the reference's own
// reference_tilemix, one query row per call (M=1). For a causal row i the
// call gets N = i + 1, so the reference code only sees keys 0..i; the K/V
// vectors of the head are shared (the reference indexes keys < N only).
// Rows run in parallel with OpenMP. Used as the timed CPU baseline.
void ref_tilemix_sampled(const std::uint16_t* q, const std::uint16_t* k, const std::uint16_t* v,
                         const std::int8_t* q8, const std::uint16_t* q_scales,
                         const std::int8_t* k8, const std::uint16_t* k_scales,
                         const std::uint8_t* routes, int M, int N, int d, float score_scale,
                         int causal, const int* head_ids, int n_heads,
                         const int* row_ids, int n_rows, double* out) {
    const int q_blocks = (M - 1) / 128 + 1, k_blocks = (N - 1) / 64 + 1;
    const int key_tiles = (N + 31) / 32;
    const std::size_t route_count = static_cast<std::size_t>((M + 15) / 16) * key_tiles;
    for (int hi = 0; hi < n_heads; ++hi) {
        const int h = head_ids[hi];
        const std::size_t qo = static_cast<std::size_t>(h) * M * d;
        const std::size_t ko = static_cast<std::size_t>(h) * N * d;
        const auto hk = halves(k + ko, static_cast<std::size_t>(N) * d);
        const auto hv = halves(v + ko, static_cast<std::size_t>(N) * d);
        ReferenceQuantized rk{std::vector<std::int8_t>(k8 + ko, k8 + ko + static_cast<std::size_t>(N) * d),
                              halves(k_scales + static_cast<std::size_t>(h) * k_blocks, k_blocks)};
        #pragma omp parallel for schedule(dynamic, 1)
        for (int ri = 0; ri < n_rows; ++ri) {
            const int row = row_ids[ri];
            const int keys = causal ? (row + 1 < N ? row + 1 : N) : N;
            const auto hq = halves(q + qo + static_cast<std::size_t>(row) * d, d);
            ReferenceQuantized rq{
                std::vector<std::int8_t>(q8 + qo + static_cast<std::size_t>(row) * d,
                                         q8 + qo + static_cast<std::size_t>(row + 1) * d),
                halves(q_scales + static_cast<std::size_t>(h) * q_blocks + row / 128, 1)};
            const std::uint8_t* row_routes = routes + static_cast<std::size_t>(h) * route_count
                                           + static_cast<std::size_t>(row / 16) * key_tiles;
            const std::vector<std::uint8_t> r(row_routes, row_routes + (keys + 31) / 32);
            const auto result = reference_tilemix(hq, hk, hv, rq, rk, r, 1, keys, d, 16, 32,
                                                  score_scale);
            std::memcpy(out + (static_cast<std::size_t>(hi) * n_rows + ri) * d, result.data(),
                        static_cast<std::size_t>(d) * sizeof(double));
        }
    }
}

int ref_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

// Thread count for the calling thread's later OpenMP regions (n > 0); a
// launcher such as torchrun may have set OMP_NUM_THREADS=1 for the process.
void ref_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

}  // extern "C"
