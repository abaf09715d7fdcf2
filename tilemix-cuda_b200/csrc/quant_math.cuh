// Element rounding of the INT8 quantizer, shared by the standalone quantizer
// (quantize.cu) and the Q quantization fused into the attention kernel
// (attention.cu), so both produce the same bytes. Semantics: the reference's
// src/tilemix.cu:37-46 (q = clamp(rz(x/scale + copysign(0.5, x/scale)), +-127),
// x/scale correctly rounded, 0 when scale == 0).
#pragma once

#include <cuda_fp16.h>

#include <cstdint>

namespace tilemix {
namespace {

// Reference rounding: fl(x / scale) by a correctly rounded division, then
// round half away from zero. Exact shortcut: the answer depends on the
// quotient only through trunc(fl(|q| + 0.5)), which changes only where |q| + 0.5
// crosses an integer. With y = fl(|x| * fl(1/scale)), |y - fl(|x| / scale)| <
// 2^-15 for |q| <= 128 (two roundings of 2^-24 relative each, plus the
// quotient's own), and fl(v + 0.5) moves v by at most 2^-17 there; so when
// y + 0.5 is more than 2^-14 away from an integer both give the same integer.
// Anything closer (ties, near-ties), and NaN / inf / zero scales, takes the
// exact division.
__device__ __forceinline__ std::int8_t quantize_exact(float x, float scale) {
    const float normalized = scale > 0.0f ? __fdiv_rn(x, scale) : 0.0f;
    const int rounded = __float2int_rz(__fadd_rn(normalized, copysignf(0.5f, normalized)));
    return static_cast<std::int8_t>(max(-127, min(127, rounded)));
}

__device__ __forceinline__ std::int8_t quantize_one(float x, float scale, float recip) {
    const float t = __fadd_rn(__fmul_rn(fabsf(x), recip), 0.5f);
    const float whole = truncf(t);
    const float frac = t - whole;                         // exact: t and whole share the exponent range
    if (frac > 0x1p-14f && frac < 1.0f - 0x1p-14f) {      // false for NaN
        const int mag = min(127, __float2int_rz(whole));
        return static_cast<std::int8_t>(x < 0.0f ? -mag : mag);
    }
    return quantize_exact(x, scale);
}

// quantize_one for the two elements of a half2, the multiply and the adds on
// packed f32x2 (one instruction per pair, same roundings). Returns the two
// signed bytes in bits [0, 16).
__device__ __forceinline__ uint32_t quantize_pair(__half2 h, float scale, float2 recip2) {
    const float2 x = __half22float2(h);
    const float2 t = __fadd2_rn(__fmul2_rn(make_float2(fabsf(x.x), fabsf(x.y)), recip2), make_float2(0.5f, 0.5f));
    const float2 whole = make_float2(truncf(t.x), truncf(t.y));
    const float2 frac = __ffma2_rn(whole, make_float2(-1.0f, -1.0f), t);   // exact
    uint32_t out = 0u;
    #pragma unroll
    for (int k = 0; k < 2; ++k) {
        const float f = k ? frac.y : frac.x;
        const float xv = k ? x.y : x.x;
        std::int8_t q;
        if (f > 0x1p-14f && f < 1.0f - 0x1p-14f) {        // false for NaN
            const int mag = min(127, __float2int_rz(k ? whole.y : whole.x));
            q = static_cast<std::int8_t>(xv < 0.0f ? -mag : mag);
        } else {
            q = quantize_exact(xv, scale);
        }
        out |= static_cast<uint32_t>(static_cast<uint8_t>(q)) << (8 * k);
    }
    return out;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t selector) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(selector));
    return d;
}

__device__ __forceinline__ float2 half2_bits_to_float2(uint32_t bits) {
    __half2 h;
    *reinterpret_cast<uint32_t*>(&h) = bits;
    return __half22float2(h);
}

// Branch-free exact rounding of four fp16 values (two half2 words) to four
// int8 bytes, for a block whose scale s is finite and > 0 and which holds no
// NaN. With y = fl(1/s) (neg_s2 = -s and y2 = y in both lanes):
//   q0 = fl(|x| y), r = fma(q0, -s, |x|), q1 = fma(r, y, q0)
// is Markstein's correction step: q1 equals the correctly rounded |x| / s, and
// trunc(fl(q1 + 0.5)) the reference's integer, for every fp16 |x| <= absmax
// and every fp16 absmax (checked exhaustively on the CPU by
// tests/native/quant_exhaustive.c: 503,856,639 pairs, no clamp ever needed).
// The integer part is the low byte of fl_rz(u + 2^23) (ulp 1 there). The sign
// is applied per byte: the two's complement of a nonzero magnitude of a
// negative input; -0 and negatives that round to 0 give 0.
__device__ __forceinline__ uint32_t quantize4_fast(uint32_t h01, uint32_t h23, float2 neg_s2, float2 y2) {
    const float2 a01 = half2_bits_to_float2(h01 & 0x7fff7fffu);
    const float2 a23 = half2_bits_to_float2(h23 & 0x7fff7fffu);
    const float2 half = make_float2(0.5f, 0.5f);
    const float2 magic = make_float2(8388608.0f, 8388608.0f);
    float2 q01 = __fmul2_rn(a01, y2);
    float2 q23 = __fmul2_rn(a23, y2);
    const float2 r01 = __ffma2_rn(q01, neg_s2, a01);
    const float2 r23 = __ffma2_rn(q23, neg_s2, a23);
    q01 = __ffma2_rn(r01, y2, q01);
    q23 = __ffma2_rn(r23, y2, q23);
    const float2 w01 = __fadd2_rz(__fadd2_rn(q01, half), magic);
    const float2 w23 = __fadd2_rz(__fadd2_rn(q23, half), magic);
    const uint32_t mag = prmt(prmt(__float_as_uint(w01.x), __float_as_uint(w01.y), 0x0040u),
                              prmt(__float_as_uint(w23.x), __float_as_uint(w23.y), 0x0040u), 0x5410u);
    // prmt selector nibbles with bit 3 set replicate the selected byte's sign
    // bit: 0xff per negative input (sign bits in bytes 1, 3 of each half2
    // word), and 0xff per nonzero magnitude (bit 7 of magnitude + 127).
    const uint32_t negative = prmt(h01, h23, 0xFDB9u);
    const uint32_t nonzero = prmt(mag + 0x7f7f7f7fu, 0u, 0xBA98u);
    const uint32_t flip = negative & nonzero;
    return (mag ^ flip) + (flip & 0x01010101u);     // per byte: 256 - m, no carry since m >= 1
}

// The scale of a block from its absmax, and whether quantize4_fast applies:
// absmax finite and > 0 (a block with NaN reports a NaN absmax here).
__device__ __forceinline__ bool fast_block(float absmax) {
    return absmax > 0.0f && absmax <= 65504.0f;
}

}  // namespace
}  // namespace tilemix
