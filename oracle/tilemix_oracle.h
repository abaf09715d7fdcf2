/*
 * TileMix CPU oracle -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference's CPU semantics for the TileMix hot
 * path (INT8 block quantizer, routed mixed INT8/FP16 scores, softmax, PV,
 * normalisation). It exists so that tests/, bench.py's CPU baseline leg and
 * __graft_entry__.smoke() can CHECK the CUDA path. The product library never
 * links, loads or calls anything here.
 *
 * Pinned against the reference itself: oracle/build_ref.sh compiles the
 * reference's own CPU oracle (src/tests/reference_tilemix.h,
 * src/tests/reference_attention.h) into oracle/_ref/, and tests compare the
 * two bit-for-bit (quantizer) and to 1e-12 (attention).
 *
 * Reference citations are paths inside the reference project.
 */
#ifndef TILEMIX_ORACLE_H
#define TILEMIX_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* IEEE binary16 <-> binary32 (round to nearest even), written from the IEEE 754
 * definition. Used where the reference calls __half2float / __float2half_rn. */
float orc_half_to_float(uint16_t h);
uint16_t orc_float_to_half(float f);

/* Per-block symmetric INT8 quantizer (reference_tilemix.h:16-41,
 * tilemix.cu:16-49): one fp32 absmax per `block_rows` x d block,
 * scale = absmax / 127 (fp32), stored as fp16 (RN); value =
 * clamp(trunc(x/scale +- 0.5), -127, 127), 0 when scale == 0. */
void orc_quantize_rows(const uint16_t* x, int rows, int d, int block_rows,
                       int8_t* values, uint16_t* scales);

/* Batched form over `heads` contiguous [rows, d] slabs; scales are laid out
 * [heads][ceil(rows/block_rows)]. */
void orc_quantize_batched(const uint16_t* x, int heads, int rows, int d, int block_rows,
                          int8_t* values, uint16_t* scales);

/* Exact INT32 dot of quantized row `query` with quantized row `key`
 * (reference_tilemix.h:43-51). */
int32_t orc_int8_dot(const int8_t* q8, const int8_t* k8, int query, int key, int d);

/* Routing words -> one byte per (16-row query tile, 32-key key tile)
 * (tilemix.cu:99-103, attention_fused.h:34-45). Returns 0 on success. */
int orc_decode_routing(const uint64_t* words, int M, int N, int key_tiles_per_group,
                       uint8_t* bits);

/* Pack a coarse [ceil(M/64)][ceil(N/64)] INT8 block mask (1 = INT8) into the
 * reference's word format with key_tiles_per_group = 2: each 64-row mask row
 * is replicated into its four 16-row query tiles. `words` must hold
 * tilemix_routing_word_count(M, N, 2) words. */
void orc_pack_block_mask64(const uint8_t* block_mask, int M, int N, uint64_t* words);

/* Mixed-precision attention for one head, fp64 (reference_tilemix.h:53-89).
 * routes: one byte per (16-row query tile, 32-key tile), may be NULL (all
 * FP16). q8/k8/q_scales/k_scales may be NULL when routes is NULL.
 * causal != 0 masks key > query before the softmax (an extension; the
 * reference has no causal mode). Rows [row_begin, row_end) are computed and
 * written to out[(row - row_begin) * d + f]. */
void orc_tilemix_rows(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                      const int8_t* q8, const int8_t* k8,
                      const uint16_t* q_scales, const uint16_t* k_scales,
                      const uint8_t* routes, int M, int N, int d, float score_scale,
                      int causal, int row_begin, int row_end, double* out);

/* Whole-batch form over `heads` contiguous slabs (OpenMP over heads x rows).
 * routes: [heads][ceil(M/16)][ceil(N/32)] or NULL. Scales per head as in
 * orc_quantize_batched. out: [heads][M][d]. */
void orc_tilemix_batched(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                         const int8_t* q8, const int8_t* k8,
                         const uint16_t* q_scales, const uint16_t* k_scales,
                         const uint8_t* routes, int heads, int M, int N, int d,
                         float score_scale, int causal, double* out);

/* Sampled form: only rows listed in row_ids (per head) of the heads listed
 * in head_ids; out[(i * n_rows + r) * d + f]. */
void orc_tilemix_sampled(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                         const int8_t* q8, const int8_t* k8,
                         const uint16_t* q_scales, const uint16_t* k_scales,
                         const uint8_t* routes, int M, int N, int d,
                         float score_scale, int causal,
                         const int* head_ids, int n_heads, const int* row_ids, int n_rows,
                         double* out);

/* Dense fp64 attention with score scale 1/sqrt(d) (reference_attention.h:12-52). */
void orc_dense_attention(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                         int M, int N, int d, double* out);

/* std::mt19937 (Matsumoto-Nishimura MT19937, init_genrand seeding) and the
 * reference test's input generator (tilemix_test.cu:48-54): uniform values
 * (r % 20001 - 10000) / 10000 rounded to fp16, drawn for q, then k, then v. */
void orc_reference_inputs(int m, int n, int d, uint16_t* q, uint16_t* k, uint16_t* v);

int orc_max_threads(void);
/* Thread count of the calling thread's later OpenMP regions (n > 0). */
void orc_set_threads(int n);

/* Device routing policy restated (the B200 library's tilemix_routing_policy;
 * the reference has no policy and takes masks from the caller, src/main.cu:48):
 * for each head, 16-row query tile q16 and group of key_tiles_per_group 32-key
 * tiles, bit = 1 (INT8) iff fl32(q_scale[q16 / 8] * max k_scale over the
 * 64-row K blocks the group's keys touch) <= max_product (a NaN scale gives
 * 0). Words in the reference's mask format (src/tilemix.cu:99-103), bits past
 * the last group 0; words has heads * ceil(M/16) * words_per_row entries. */
void orc_routing_policy(const uint16_t* q_scales, const uint16_t* k_scales, int heads, int M, int N,
                        int key_tiles_per_group, float max_product, uint64_t* words);

#ifdef __cplusplus
}
#endif

#endif
