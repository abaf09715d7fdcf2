/*
 * TileMix CPU oracle -- TEST INFRASTRUCTURE ONLY (see tilemix_oracle.h).
 * Never linked into or called by the product library.
 */
#include "tilemix_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static uint32_t f32_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static float bits_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

float orc_half_to_float(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t exponent = (h >> 10) & 0x1fu;
    const uint32_t mantissa = h & 0x3ffu;
    if (exponent == 0) {
        /* zero or subnormal: mantissa * 2^-24 is exact in binary32 */
        const float magnitude = (float)mantissa * 5.9604644775390625e-08f;
        return sign ? -magnitude : magnitude;
    }
    if (exponent == 31) return bits_f32(sign | 0x7f800000u | (mantissa << 13));
    return bits_f32(sign | ((exponent + 112u) << 23) | (mantissa << 13));
}

uint16_t orc_float_to_half(float f) {
    const uint32_t x = f32_bits(f);
    const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    const uint32_t ax = x & 0x7fffffffu;
    if (ax > 0x7f800000u) return (uint16_t)(sign | 0x7fffu);      /* NaN */
    if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);     /* >= 65520 rounds to inf */
    if (ax <= 0x33000000u) return sign;                           /* <= 2^-25 rounds to zero */
    if (ax < 0x38800000u) {                                       /* half subnormal range */
        const uint32_t mantissa = (ax & 0x7fffffu) | 0x800000u;
        const uint32_t shift = 126u - (ax >> 23);                 /* value * 2^24 = m >> shift */
        uint32_t result = mantissa >> shift;
        const uint32_t remainder = mantissa & ((1u << shift) - 1u);
        const uint32_t halfway = 1u << (shift - 1u);
        if (remainder > halfway || (remainder == halfway && (result & 1u))) ++result;
        return (uint16_t)(sign | result);
    }
    uint32_t result = (((ax >> 23) - 112u) << 10) | ((ax >> 13) & 0x3ffu);
    const uint32_t remainder = ax & 0x1fffu;
    if (remainder > 0x1000u || (remainder == 0x1000u && (result & 1u))) ++result;
    return (uint16_t)(sign | result);
}

/* reference_tilemix.h:16-41 with the fp32 operation order of tilemix.cu:37-46. */
void orc_quantize_rows(const uint16_t* x, int rows, int d, int block_rows,
                       int8_t* values, uint16_t* scales) {
    for (int first = 0; first < rows; first += block_rows) {
        const int last = rows < first + block_rows ? rows : first + block_rows;
        float maximum = 0.0f;
        for (size_t i = (size_t)first * d; i < (size_t)last * d; ++i) {
            const float a = fabsf(orc_half_to_float(x[i]));
            if (a > maximum) maximum = a;   /* max(), NaN never replaces the running value */
        }
        const float scale = maximum / 127.0f;
        scales[first / block_rows] = orc_float_to_half(scale);
        for (size_t i = (size_t)first * d; i < (size_t)last * d; ++i) {
            const float normalized = scale > 0.0f ? orc_half_to_float(x[i]) / scale : 0.0f;
            const float shifted = normalized < 0.0f ? normalized - 0.5f : normalized + 0.5f;
            int rounded;
            if (shifted != shifted) rounded = 0;              /* cvt.rzi of NaN is 0 on the GPU */
            else if (shifted >= 127.0f) rounded = 127;
            else if (shifted <= -127.0f) rounded = -127;
            else rounded = (int)shifted;                      /* truncation toward zero */
            values[i] = (int8_t)rounded;
        }
    }
}

void orc_quantize_batched(const uint16_t* x, int heads, int rows, int d, int block_rows,
                          int8_t* values, uint16_t* scales) {
    const int blocks = (rows - 1) / block_rows + 1;
    #pragma omp parallel for schedule(static)
    for (int h = 0; h < heads; ++h) {
        const size_t offset = (size_t)h * rows * d;
        orc_quantize_rows(x + offset, rows, d, block_rows, values + offset,
                          scales + (size_t)h * blocks);
    }
}

int32_t orc_int8_dot(const int8_t* q8, const int8_t* k8, int query, int key, int d) {
    int64_t sum = 0;
    for (int f = 0; f < d; ++f) {
        sum += (int)q8[(size_t)query * d + f] * (int)k8[(size_t)key * d + f];
    }
    return (int32_t)sum;
}

/* tilemix.cu:99-103: group = key_tile / g; word = words[qtile*wpr + group/64];
 * bit = (word >> (group % 64)) & 1. */
int orc_decode_routing(const uint64_t* words, int M, int N, int key_tiles_per_group,
                       uint8_t* bits) {
    if (M <= 0 || N <= 0 || key_tiles_per_group <= 0) return 1;
    const size_t query_tiles = (size_t)(M - 1) / 16 + 1;
    const size_t key_tiles = (size_t)(N - 1) / 32 + 1;
    const size_t groups = (key_tiles - 1) / (size_t)key_tiles_per_group + 1;
    const size_t words_per_row = (groups - 1) / 64 + 1;
    for (size_t qt = 0; qt < query_tiles; ++qt) {
        for (size_t kt = 0; kt < key_tiles; ++kt) {
            const size_t group = kt / (size_t)key_tiles_per_group;
            const uint64_t word = words ? words[qt * words_per_row + group / 64] : 0;
            bits[qt * key_tiles + kt] = (uint8_t)((word >> (group % 64)) & 1u);
        }
    }
    return 0;
}

void orc_pack_block_mask64(const uint8_t* block_mask, int M, int N, uint64_t* words) {
    const size_t query_tiles = (size_t)(M - 1) / 16 + 1;
    const size_t key_tiles = (size_t)(N - 1) / 32 + 1;
    const size_t groups = (key_tiles - 1) / 2 + 1;          /* one group = 64 keys */
    const size_t words_per_row = (groups - 1) / 64 + 1;
    const size_t mask_cols = (size_t)(N - 1) / 64 + 1;
    memset(words, 0, query_tiles * words_per_row * sizeof(uint64_t));
    for (size_t qt = 0; qt < query_tiles; ++qt) {
        const size_t mask_row = qt / 4;                      /* 64 rows = 4 query tiles */
        for (size_t g = 0; g < groups; ++g) {
            if (block_mask[mask_row * mask_cols + g]) {
                words[qt * words_per_row + g / 64] |= (uint64_t)1 << (g % 64);
            }
        }
    }
}

/* reference_tilemix.h:53-89, one query row at a time; causal extension masks
 * key > query. */
static void tilemix_row(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                        const int8_t* q8, const int8_t* k8,
                        const uint16_t* q_scales, const uint16_t* k_scales,
                        const uint8_t* routes, int N, int d, float score_scale,
                        int causal, int query, double* scores, double* out_row) {
    const int key_tiles = (N + 31) / 32;
    const int keys = causal ? (query + 1 < N ? query + 1 : N) : N;
    for (int key = 0; key < keys; ++key) {
        double dot = 0.0;
        if (routes && routes[(size_t)(query / 16) * key_tiles + key / 32]) {
            dot = (double)orc_int8_dot(q8, k8, query, key, d);
            dot *= (double)orc_half_to_float(q_scales[query / 128]);
            dot *= (double)orc_half_to_float(k_scales[key / 64]);
        } else {
            for (int f = 0; f < d; ++f) {
                dot += (double)orc_half_to_float(q[(size_t)query * d + f])
                     * (double)orc_half_to_float(k[(size_t)key * d + f]);
            }
        }
        scores[key] = dot * (double)score_scale;
    }
    double maximum = scores[0];
    for (int key = 1; key < keys; ++key) if (scores[key] > maximum) maximum = scores[key];
    double denominator = 0.0;
    for (int key = 0; key < keys; ++key) {
        scores[key] = exp(scores[key] - maximum);
        denominator += scores[key];
    }
    for (int f = 0; f < d; ++f) out_row[f] = 0.0;
    for (int key = 0; key < keys; ++key) {
        const double probability = scores[key] / denominator;
        for (int f = 0; f < d; ++f) {
            out_row[f] += probability * (double)orc_half_to_float(v[(size_t)key * d + f]);
        }
    }
}

void orc_tilemix_rows(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                      const int8_t* q8, const int8_t* k8,
                      const uint16_t* q_scales, const uint16_t* k_scales,
                      const uint8_t* routes, int M, int N, int d, float score_scale,
                      int causal, int row_begin, int row_end, double* out) {
    (void)M;
    double* scores = (double*)malloc(sizeof(double) * (size_t)N);
    for (int row = row_begin; row < row_end; ++row) {
        tilemix_row(q, k, v, q8, k8, q_scales, k_scales, routes, N, d, score_scale, causal,
                    row, scores, out + (size_t)(row - row_begin) * d);
    }
    free(scores);
}

void orc_tilemix_batched(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                         const int8_t* q8, const int8_t* k8,
                         const uint16_t* q_scales, const uint16_t* k_scales,
                         const uint8_t* routes, int heads, int M, int N, int d,
                         float score_scale, int causal, double* out) {
    const int q_blocks = (M - 1) / 128 + 1, k_blocks = (N - 1) / 64 + 1;
    const size_t route_count = (size_t)((M + 15) / 16) * ((N + 31) / 32);
    const long total = (long)heads * M;
    #pragma omp parallel
    {
        double* scores = (double*)malloc(sizeof(double) * (size_t)N);
        #pragma omp for schedule(dynamic, 16)
        for (long item = 0; item < total; ++item) {
            const int h = (int)(item / M), row = (int)(item % M);
            const size_t qo = (size_t)h * M * d, ko = (size_t)h * N * d;
            tilemix_row(q + qo, k + ko, v + ko, q8 ? q8 + qo : NULL, k8 ? k8 + ko : NULL,
                        q_scales ? q_scales + (size_t)h * q_blocks : NULL,
                        k_scales ? k_scales + (size_t)h * k_blocks : NULL,
                        routes ? routes + (size_t)h * route_count : NULL,
                        N, d, score_scale, causal, row, scores, out + qo + (size_t)row * d);
        }
        free(scores);
    }
}

void orc_tilemix_sampled(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                         const int8_t* q8, const int8_t* k8,
                         const uint16_t* q_scales, const uint16_t* k_scales,
                         const uint8_t* routes, int M, int N, int d,
                         float score_scale, int causal,
                         const int* head_ids, int n_heads, const int* row_ids, int n_rows,
                         double* out) {
    const int q_blocks = (M - 1) / 128 + 1, k_blocks = (N - 1) / 64 + 1;
    const size_t route_count = (size_t)((M + 15) / 16) * ((N + 31) / 32);
    const long total = (long)n_heads * n_rows;
    #pragma omp parallel
    {
        double* scores = (double*)malloc(sizeof(double) * (size_t)N);
        #pragma omp for schedule(dynamic, 1)
        for (long item = 0; item < total; ++item) {
            const int h = head_ids[item / n_rows], row = row_ids[item % n_rows];
            const size_t qo = (size_t)h * M * d, ko = (size_t)h * N * d;
            tilemix_row(q + qo, k + ko, v + ko, q8 ? q8 + qo : NULL, k8 ? k8 + ko : NULL,
                        q_scales ? q_scales + (size_t)h * q_blocks : NULL,
                        k_scales ? k_scales + (size_t)h * k_blocks : NULL,
                        routes ? routes + (size_t)h * route_count : NULL,
                        N, d, score_scale, causal, row, scores, out + (size_t)item * d);
        }
        free(scores);
    }
}

/* reference_attention.h:12-52 (fp64, score scale 1/sqrt(d)). */
void orc_dense_attention(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                         int M, int N, int d, double* out) {
    const double scale = 1.0 / sqrt((double)d);
    double* weights = (double*)malloc(sizeof(double) * (size_t)N);
    for (int query = 0; query < M; ++query) {
        double maximum = -INFINITY;
        for (int key = 0; key < N; ++key) {
            double dot = 0.0;
            for (int f = 0; f < d; ++f) {
                dot += (double)orc_half_to_float(q[(size_t)query * d + f])
                     * (double)orc_half_to_float(k[(size_t)key * d + f]);
            }
            weights[key] = dot * scale;
            if (weights[key] > maximum) maximum = weights[key];
        }
        double denominator = 0.0;
        for (int key = 0; key < N; ++key) {
            weights[key] = exp(weights[key] - maximum);
            denominator += weights[key];
        }
        double* row = out + (size_t)query * d;
        for (int f = 0; f < d; ++f) row[f] = 0.0;
        for (int key = 0; key < N; ++key) {
            const double probability = weights[key] / denominator;
            for (int f = 0; f < d; ++f) {
                row[f] += probability * (double)orc_half_to_float(v[(size_t)key * d + f]);
            }
        }
    }
    free(weights);
}

/* MT19937 (Matsumoto & Nishimura 1998): init_genrand seeding, 624-word state,
 * tempering as published. Matches std::mt19937(seed)() outputs. */
typedef struct { uint32_t state[624]; int index; } mt19937;

static void mt_seed(mt19937* mt, uint32_t seed) {
    mt->state[0] = seed;
    for (int i = 1; i < 624; ++i) {
        mt->state[i] = 1812433253u * (mt->state[i - 1] ^ (mt->state[i - 1] >> 30)) + (uint32_t)i;
    }
    mt->index = 624;
}

static uint32_t mt_next(mt19937* mt) {
    if (mt->index >= 624) {
        for (int i = 0; i < 624; ++i) {
            const uint32_t y = (mt->state[i] & 0x80000000u) | (mt->state[(i + 1) % 624] & 0x7fffffffu);
            mt->state[i] = mt->state[(i + 397) % 624] ^ (y >> 1) ^ ((y & 1u) ? 0x9908b0dfu : 0u);
        }
        mt->index = 0;
    }
    uint32_t y = mt->state[mt->index++];
    y ^= y >> 11;
    y ^= (y << 7) & 0x9d2c5680u;
    y ^= (y << 15) & 0xefc60000u;
    y ^= y >> 18;
    return y;
}

void orc_reference_inputs(int m, int n, int d, uint16_t* q, uint16_t* k, uint16_t* v) {
    mt19937 mt;
    mt_seed(&mt, (uint32_t)(m * 131 + n * 17 + d));
    const size_t qn = (size_t)m * d, kn = (size_t)n * d;
    uint16_t* targets[3] = {q, k, v};
    const size_t counts[3] = {qn, kn, kn};
    for (int t = 0; t < 3; ++t) {
        for (size_t i = 0; i < counts[t]; ++i) {
            const int r = (int)(mt_next(&mt) % 20001u) - 10000;
            targets[t][i] = orc_float_to_half((float)r / 10000.0f);
        }
    }
}

int orc_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void orc_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

/* Routing policy (see tilemix_oracle.h): a plain loop per word and bit. */
void orc_routing_policy(const uint16_t* q_scales, const uint16_t* k_scales, int heads, int M, int N,
                        int key_tiles_per_group, float max_product, uint64_t* words) {
    const int q16_tiles = (M + 15) / 16, k32_tiles = (N + 31) / 32;
    const long long groups = ((long long)k32_tiles + key_tiles_per_group - 1) / key_tiles_per_group;
    const long long wpr = (groups + 63) / 64;
    const int q_blocks = (M + 127) / 128, k_blocks = (N + 63) / 64;
    for (int h = 0; h < heads; ++h) {
        for (int t = 0; t < q16_tiles; ++t) {
            const float sq = orc_half_to_float(q_scales[(size_t)h * q_blocks + t / 8]);
            for (long long w = 0; w < wpr; ++w) {
                uint64_t word = 0;
                for (int b = 0; b < 64; ++b) {
                    const long long g = w * 64 + b;
                    if (g >= groups) break;
                    const long long kt0 = g * key_tiles_per_group;
                    long long kt1 = kt0 + key_tiles_per_group;
                    if (kt1 > k32_tiles) kt1 = k32_tiles;
                    const long long key0 = kt0 * 32;
                    long long key1 = kt1 * 32;
                    if (key1 > N) key1 = N;
                    float skmax = 0.0f;
                    int nan = 0;
                    for (long long kb = key0 / 64; kb <= (key1 - 1) / 64; ++kb) {
                        const float s = orc_half_to_float(k_scales[(size_t)h * k_blocks + kb]);
                        if (s != s) nan = 1;
                        else if (s > skmax) skmax = s;
                    }
                    const float product = sq * skmax;
                    if (!nan && product <= max_product) word |= (uint64_t)1 << b;
                }
                words[((size_t)h * q16_tiles + t) * wpr + w] = word;
            }
        }
    }
}
