/* Exhaustive check of the quantizers' fast division (test infrastructure, built by test_quant_division.py).
 *
 * For every positive finite bf16 absmax p and every bf16 v with |v| <= p (both signs), the kernels compute the
 * quotient v / s, s = RN(p / 127) (int8) or RN(max(p, 1e-12) / 448) (e4m3), as
 *     s >= 2^-90:  q0 = RN(v * r), r = RN(1 / s);  q = fma(fma(-q0, s, v), r, q0)
 *     otherwise:   q = RN(v / s)
 * This program counts the (p, v) pairs whose int8 code (round half away from zero) or e4m3 byte (nearest even,
 * saturating; zero takes v's sign) differs from the one of the IEEE quotient. It also checks the scales themselves
 * as the kernels form them for bf16 peaks (hn_common.cuh: quot_const): for every positive finite bf16 p,
 *     RN(p / d) == fma(fma(-q0, d, p), RN(1 / d), q0),  q0 = RN(p * RN(1 / d)),  d = 127 and (p floored at 1e-12) 448.
 * Exit status 0 iff nothing differs. */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

uint8_t or_e4m3_from_f32(float x);

static float from_bits(uint32_t b) { float x; memcpy(&x, &b, 4); return x; }
static int code_i8(float y) {
    float r = y >= 0 ? floorf(y + 0.5f) : ceilf(y - 0.5f);
    return (int)fminf(fmaxf(r, -127.f), 127.f);
}
static float fast_quotient(float v, float s, float r) {
    if (!(s >= 0x1p-90f)) return v / s;
    float q0 = v * r;
    return fmaf(fmaf(-q0, s, v), r, q0);
}

static float quot_const(float p, float d) {
    const float rd = 1.0f / d, q0 = p * rd;
    return fmaf(fmaf(-q0, d, p), rd, q0);
}

int main(void) {
    long long bad_scale = 0;
    for (uint32_t pb = 1; pb < 0x7F80; ++pb) {
        const float p = from_bits(pb << 16), pe = fmaxf(p, 1e-12f);
        bad_scale += quot_const(p, 127.0f) != p / 127.0f;
        bad_scale += quot_const(pe, 448.0f) != pe / 448.0f;
    }
    printf("scale mismatches %lld\n", bad_scale);
    long long bad_i8 = 0, bad_e4m3 = 0, pairs = 0;
#pragma omp parallel for schedule(dynamic, 64) reduction(+ : bad_i8, bad_e4m3, pairs)
    for (uint32_t pb = 1; pb < 0x7F80; ++pb) {
        const float p = from_bits(pb << 16);
        const float s8 = p / 127.0f, r8 = 1.0f / s8;
        const float se = fmaxf(p, 1e-12f) / 448.0f, re = 1.0f / se;
        for (uint32_t vb = 0; vb <= pb; ++vb) {
            for (int neg = 0; neg < 2; ++neg) {
                const float v = from_bits((vb << 16) | (neg ? 0x80000000u : 0u));
                ++pairs;
                bad_i8 += code_i8(fast_quotient(v, s8, r8)) != code_i8(v / s8);
                float qe = fast_quotient(v, se, re);
                qe = copysignf(qe, v);
                bad_e4m3 += or_e4m3_from_f32(qe) != or_e4m3_from_f32(v / se);
            }
        }
    }
    printf("pairs %lld: int8 code mismatches %lld, e4m3 byte mismatches %lld\n", pairs, bad_i8, bad_e4m3);
    return (bad_i8 || bad_e4m3 || bad_scale) ? 1 : 0;
}
