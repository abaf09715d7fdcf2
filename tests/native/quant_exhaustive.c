/*
 * Exhaustive CPU proof of the quantizer's branch-free element rounding.
 *
 * The reference quantizes x with scale s = fl(absmax / 127) as
 *   q = clamp(trunc(fl(fl(x / s) + copysign(0.5, x))), -127, 127)
 * with fl(x / s) a correctly rounded division (src/tilemix.cu:37-46). The
 * B200 kernels compute the quotient without a division: with y = fl(1 / s),
 *   q0 = fl(|x| * y), r = fma(-q0, s, |x|) (exact), q1 = fma(r, y, q0)
 * (Markstein's correction step: q1 is the correctly rounded |x| / s when y is
 * the correctly rounded reciprocal and q0 is within an ulp of the quotient),
 * then u = fl(q1 + 0.5) and the integer part of u by an add of 2^23 rounded
 * toward zero (u < 2^23). The input domain is finite: x and absmax are fp16
 * values with |x| <= absmax. This program checks every such pair (x >= 0; the
 * sign is applied exactly afterwards): q1 must equal fl(x / s) and the
 * integer must equal the reference's, clamp included. It prints the counts
 * and exits non-zero on any mismatch.
 *
 * Build: gcc -std=c11 -O2 -mfma -ffp-contract=off -fopenmp quant_exhaustive.c -lm
 */
#include <fenv.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>

static float half_to_float(uint16_t h) {
    const int exp = (h >> 10) & 0x1f, man = h & 0x3ff;
    float v;
    if (exp == 0) v = ldexpf((float)man, -24);
    else v = ldexpf((float)(man | 0x400), exp - 25);
    return (h & 0x8000) ? -v : v;
}

int main(void) {
    long long checked = 0, bad_quotient = 0, bad_integer = 0, clamped = 0;
    /* absmax over every positive finite fp16 value; x over 0 .. absmax */
#pragma omp parallel for schedule(dynamic, 64) reduction(+ : checked, bad_quotient, bad_integer, clamped)
    for (int a = 1; a < 0x7c00; ++a) {
        const float amax = half_to_float((uint16_t)a);
        const float s = amax / 127.0f;          /* correctly rounded */
        const float y = 1.0f / s;               /* correctly rounded reciprocal */
        for (int xb = 0; xb <= a; ++xb) {
            const float x = half_to_float((uint16_t)xb);
            /* reference */
            const float q = x / s;
            const float t = q + 0.5f;
            int kr = (int)t;                    /* trunc */
            if (kr > 127) { kr = 127; ++clamped; }
            /* branch-free form */
            const float q0 = x * y;
            const float r = fmaf(-q0, s, x);
            const float q1 = fmaf(r, y, q0);
            const float u = q1 + 0.5f;
            /* fl_rz(u + 2^23) - 2^23 == floor(u) for 0 <= u < 2^23 (ulp 1 there) */
            const int kf = (int)floorf(u);
            checked += 1;
            bad_quotient += q1 != q;
            bad_integer += kf != kr;
        }
    }
    /* the round-toward-zero add itself, on every u the check can meet */
    long long bad_magic = 0;
    fesetround(FE_TOWARDZERO);
    for (float u = 0.5f; u < 129.0f; u = nextafterf(u, 200.0f)) {
        volatile float w = u + 8388608.0f;
        if ((int)(w - 8388608.0f) != (int)floorf(u)) ++bad_magic;
    }
    fesetround(FE_TONEAREST);
    printf("checked %lld pairs: quotient mismatches %lld, integer mismatches %lld, clamped %lld, "
           "magic-add mismatches %lld\n", checked, bad_quotient, bad_integer, clamped, bad_magic);
    return (bad_quotient || bad_integer || bad_magic) ? 1 : 0;
}
