// hn_common.cuh - shared device helpers of the B200 quantized DiT linear path (sm_100a only).
//
// Rounding helpers follow the reference's arithmetic (hy_nomas/kernels.py, hy_nomas/fused.py): every
// fp32 operation that the reference rounds separately is written with an explicit _rn intrinsic so the
// compiler cannot contract it into an FMA; where an FMA is intended it is written as __fmaf_rn.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ != 1000)
#error "this library is built for sm_100a (B200) only"
#endif

namespace hn {

// Bits of the device error word (defined in gemm.cu): bounded waits OR them in and return instead of
// hanging.
constexpr int HN_DEVERR_TIMEOUT = 1;

// ---------------------------------------------------------------------------------------------------
// bf16 / code helpers

// hy_nomas/kernels.py:67-71 (_rbf16): fp32 -> nearest-even bf16 value, kept in fp32.
__device__ __forceinline__ float rbf16(float x) {
    uint32_t b = __float_as_uint(x);
    b = (b + (((b >> 16) & 1u) + 0x7FFFu)) & 0xFFFF0000u;
    return __uint_as_float(b);
}
__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
// two bf16-valued floats -> packed bf16x2 (exact: the low halves are zero)
__device__ __forceinline__ uint32_t pack_bf16_exact(float lo, float hi) {
    return (__float_as_uint(lo) >> 16) | (__float_as_uint(hi) & 0xFFFF0000u);
}
// round two floats to bf16 (nearest even) and pack
__device__ __forceinline__ uint32_t pack_bf16_rn(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
}
__device__ __forceinline__ uint32_t pack_f16_rn(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
}

// round half away from zero, clamp +-127 (hy_nomas/kernels.py:35-36, ops.py:50-51)
__device__ __forceinline__ int code_i8(float y) {
    float r = (y >= 0.0f) ? floorf(__fadd_rn(y, 0.5f)) : ceilf(__fsub_rn(y, 0.5f));
    r = fminf(fmaxf(r, -127.0f), 127.0f);
    return (int)r;
}
// round half to even (cvt.rni), clamp +-127: torch.round's convention for per-token int8 codes, an option beside
// the reference's half-away rounding
__device__ __forceinline__ int code_i8_rne(float y) {
    const int r = __float2int_rn(y);
    return r > 127 ? 127 : (r < -127 ? -127 : r);
}
__device__ __forceinline__ uint32_t pack4_i8(int a, int b, int c, int d) {
    return (uint32_t)(a & 0xFF) | ((uint32_t)(b & 0xFF) << 8) | ((uint32_t)(c & 0xFF) << 16) |
           ((uint32_t)(d & 0xFF) << 24);
}
// two floats -> two e4m3 bytes, nearest even, saturating to +-448 (cvt.rn.satfinite.e4m3x2.f32)
__device__ __forceinline__ uint32_t pack2_e4m3(float lo, float hi) {
    return (uint32_t)__nv_cvt_float2_to_fp8x2(make_float2(lo, hi), __NV_SATFINITE, __NV_E4M3);
}

// int8 quantization scale of a 128-group (kernels.py:33): peak > 0 ? peak / 127 : 1
__device__ __forceinline__ float i8_scale(float peak) { return peak > 0.0f ? __fdiv_rn(peak, 127.0f) : 1.0f; }
// e4m3 scale (kernels.py:39): max(peak, 1e-12) / 448
__device__ __forceinline__ float e4m3_scale(float peak) { return __fdiv_rn(fmaxf(peak, 1e-12f), 448.0f); }

// RN(p / d) for a scale divisor d (127, 448) and p a bf16 value (or the 1e-12 floor): q0 = RN(p * RN(1/d)), the
// exact remainder p - q0 * d in one fma, and one more fma corrects q0. tests/division_check.c checks it against
// the IEEE quotient for every positive finite bf16 p. The same scales as i8_scale / e4m3_scale, for peaks that
// are absmaxes of bf16 values.
__device__ __forceinline__ float quot_const(float p, float d, float rd) {
    const float q0 = __fmul_rn(p, rd);
    return __fmaf_rn(__fmaf_rn(-q0, d, p), rd, q0);
}
__device__ __forceinline__ float i8_scale_bf16(float peak) {
    return peak > 0.0f ? quot_const(peak, 127.0f, 1.0f / 127.0f) : 1.0f;
}
__device__ __forceinline__ float e4m3_scale_bf16(float peak) {
    return quot_const(fmaxf(peak, 1e-12f), 448.0f, 1.0f / 448.0f);
}

// 1/sqrt(v) with both steps correctly rounded (the tl.rsqrt of the reference, evaluated as the Triton
// interpreter evaluates it). The correctly rounded reciprocal RN(1/s) is the correctly rounded quotient 1/s.
__device__ __forceinline__ float rsqrt_cr(float v) { return __frcp_rn(__fsqrt_rn(v)); }

// ---------------------------------------------------------------------------------------------------
// exp / GELU (hy_nomas/kernels.py:74-77). exp_cw: Cody & Waite (1980) reduction x = k*ln2 + r with the
// two-part ln2 of fdlibm's expf, Taylor series of e^r to degree 7 (Horner, fused multiply-adds), scaling
// by 2^k in two exact steps. The CPU oracle evaluates the same operations, so GELU outputs compare
// bit-for-bit.
__device__ __forceinline__ float exp_cw(float x) {
    if (x != x) return x;
    if (x > 88.7228394f) return __int_as_float(0x7F800000);
    if (x < -103.972084f) return 0.0f;
    const float log2e = 0x1.715476p+0f, ln2_hi = 0x1.62e4p-1f, ln2_lo = 0x1.7f7d1cp-20f;
    float kf = rintf(__fmul_rn(x, log2e));
    float r = __fmaf_rn(-kf, ln2_hi, x);
    r = __fmaf_rn(-kf, ln2_lo, r);
    float p = 0x1.a01a02p-13f;
    p = __fmaf_rn(p, r, 0x1.6c16c2p-10f);
    p = __fmaf_rn(p, r, 0x1.111112p-7f);
    p = __fmaf_rn(p, r, 0x1.555556p-5f);
    p = __fmaf_rn(p, r, 0x1.555556p-3f);
    p = __fmaf_rn(p, r, 0.5f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    int k = (int)kf;
    int k1 = k / 2, k2 = k - k1;
    p = __fmul_rn(p, __uint_as_float((uint32_t)(k1 + 127) << 23));
    p = __fmul_rn(p, __uint_as_float((uint32_t)(k2 + 127) << 23));
    return p;
}

// 0.5 x (1 + (2 sigmoid(2u) - 1)), u = 0.79788456 (x + 0.044715 x^3), left to right, one rounding per op
__device__ __forceinline__ float gelu_tanh(float x) {
    float x3 = __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, x), x), x);
    float inner = __fmul_rn(0.7978845608028654f, __fadd_rn(x, x3));
    float z = __fmul_rn(2.0f, inner);
    float sig = __frcp_rn(__fadd_rn(1.0f, exp_cw(-z)));   // RN(1 / d): the correctly rounded quotient 1 / d
    return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, __fsub_rn(__fmul_rn(2.0f, sig), 1.0f)));
}

// ---------------------------------------------------------------------------------------------------
// packed pairs of fp32 (sm_100 f32x2 instructions, explicit rounding: never contracted)

__device__ __forceinline__ uint64_t x2(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void x2_split(uint64_t p, float &lo, float &hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(p));
}
__device__ __forceinline__ uint64_t x2_add(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ uint64_t x2_add_rz(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("add.rz.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ uint64_t x2_mul(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ uint64_t x2_fma(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
__device__ __forceinline__ uint64_t x2_splat(float v) { return x2(v, v); }
// (lo, hi) -> bf16x2 word (lo in the low half), each rounded to nearest even: the reference's _rbf16
// (kernels.py:67-71) for finite values, as one conversion instruction
__device__ __forceinline__ uint32_t bf16x2_rn(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

// Quotient v / s for a bf16 value v and a quantization scale s > 0, correctly rounded, given rs = RN(1/s):
// q0 = RN(v * rs) is within an ulp of v / s, the remainder v - q0 * s is exact in one fma, and one more fma
// corrects q0 (Markstein, IBM J. Res. Dev. 34(1), 1990). The remainder underflows for very small s; the
// callers take the IEEE division when s < 2^-90. An exhaustive check over every bf16 absmax p and every bf16
// |v| <= p found the int8 codes (round half away of the quotient) identical to those of RN(v / s), for both
// signs, with s = RN(p / 127); for e4m3 the sign of a zero quotient is restored by the caller.
// Pairs of quotients with the same s: ns = (-s, -s), rs2 = (rs, rs).
__device__ __forceinline__ uint64_t x2_quot(uint64_t v, uint64_t ns, uint64_t rs2) {
    const uint64_t q0 = x2_mul(v, rs2);
    const uint64_t rem = x2_fma(q0, ns, v);
    return x2_fma(rem, rs2, q0);
}

// int8 code bytes of a pair of quotients, round half away from zero (kernels.py:35): the low byte of each
// returned word. w = RN(q + copysign(0.5, q)) is the reference's |q| + 0.5 with q's sign (round to nearest is
// symmetric); the conversion cvt.rzi.s32.f32 truncates it to the integer, whose two's complement low byte is
// the code. |q| <= 127.00001 for the quotients of the quantizers (|v| <= absmax, s = RN(absmax / 127)), so the
// clamp to +-127 of the reference never binds and is not applied.
__device__ __forceinline__ void x2_codes(uint64_t q, uint32_t &c_lo, uint32_t &c_hi) {
    float qlo, qhi;
    x2_split(q, qlo, qhi);
    const uint64_t half = x2(__uint_as_float((__float_as_uint(qlo) & 0x80000000u) | 0x3F000000u),
                             __uint_as_float((__float_as_uint(qhi) & 0x80000000u) | 0x3F000000u));
    float wlo, whi;
    x2_split(x2_add(q, half), wlo, whi);
    c_lo = (uint32_t)__float2int_rz(wlo);
    c_hi = (uint32_t)__float2int_rz(whi);
}
// four code words (low bytes) -> one word, first argument in the low byte
__device__ __forceinline__ uint32_t pack4_lowbytes(uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    return __byte_perm(__byte_perm(a, b, 0x0040), __byte_perm(c, d, 0x0040), 0x5410);
}

// 8 elements of a row -> 8 codes (int8 bytes or e4m3 bytes) for scale `sc`; `fast`: bf16 input with the
// exact fma-corrected quotient of x2_quot, else IEEE division. Shared by the activation quantizers
// (quant.cu) and the decoder fusions (decoder.cu).
template <int KIND, bool RNE>
__device__ __forceinline__ uint2 quant_chunk8(const float (&v)[8], float sc, bool fast, uint64_t ns, uint64_t rs) {
    uint2 out;
    if (fast && KIND == 0 && RNE) {
        int cc[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float q0, q1;
            x2_split(x2_quot(x2(v[2 * i], v[2 * i + 1]), ns, rs), q0, q1);
            cc[2 * i] = code_i8_rne(q0);
            cc[2 * i + 1] = code_i8_rne(q1);
        }
        out.x = pack4_i8(cc[0], cc[1], cc[2], cc[3]);
        out.y = pack4_i8(cc[4], cc[5], cc[6], cc[7]);
    } else if (fast && KIND == 0) {
        uint32_t cc[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) x2_codes(x2_quot(x2(v[2 * i], v[2 * i + 1]), ns, rs), cc[2 * i], cc[2 * i + 1]);
        out.x = pack4_lowbytes(cc[0], cc[1], cc[2], cc[3]);
        out.y = pack4_lowbytes(cc[4], cc[5], cc[6], cc[7]);
    } else if (fast) {
        uint32_t h[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float q0, q1;
            x2_split(x2_quot(x2(v[2 * i], v[2 * i + 1]), ns, rs), q0, q1);
            h[i] = pack2_e4m3(copysignf(q0, v[2 * i]), copysignf(q1, v[2 * i + 1]));
        }
        out.x = h[0] | (h[1] << 16);
        out.y = h[2] | (h[3] << 16);
    } else if (KIND == 0) {
        int cc[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) cc[i] = RNE ? code_i8_rne(__fdiv_rn(v[i], sc)) : code_i8(__fdiv_rn(v[i], sc));
        out.x = pack4_i8(cc[0], cc[1], cc[2], cc[3]);
        out.y = pack4_i8(cc[4], cc[5], cc[6], cc[7]);
    } else {
        uint32_t h[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) h[i] = pack2_e4m3(__fdiv_rn(v[2 * i], sc), __fdiv_rn(v[2 * i + 1], sc));
        out.x = h[0] | (h[1] << 16);
        out.y = h[2] | (h[3] << 16);
    }
    return out;
}

// 2^k for an integer k in [-126, 127], as a float
__device__ __forceinline__ float pow2i(int k) { return __uint_as_float((uint32_t)(k + 127) << 23); }

// exp_cw of a pair, the same operations lane by lane: the products and fused multiply-adds on f32x2 pairs, the
// per-lane steps (rint, the exponent split, the range cases) scalar
__device__ __forceinline__ uint64_t exp_cw_x2(uint64_t v) {
    const float log2e = 0x1.715476p+0f, ln2_hi = 0x1.62e4p-1f, ln2_lo = 0x1.7f7d1cp-20f;
    float v0, v1, t0, t1;
    x2_split(v, v0, v1);
    x2_split(x2_mul(v, x2_splat(log2e)), t0, t1);
    const float k0f = rintf(t0), k1f = rintf(t1);
    const uint64_t nk = x2(-k0f, -k1f);
    uint64_t r = x2_fma(nk, x2_splat(ln2_hi), v);
    r = x2_fma(nk, x2_splat(ln2_lo), r);
    uint64_t p = x2_splat(0x1.a01a02p-13f);
    p = x2_fma(p, r, x2_splat(0x1.6c16c2p-10f));
    p = x2_fma(p, r, x2_splat(0x1.111112p-7f));
    p = x2_fma(p, r, x2_splat(0x1.555556p-5f));
    p = x2_fma(p, r, x2_splat(0x1.555556p-3f));
    p = x2_fma(p, r, x2_splat(0.5f));
    p = x2_fma(p, r, x2_splat(1.0f));
    p = x2_fma(p, r, x2_splat(1.0f));
    const int k0 = (int)k0f, k1 = (int)k1f;
    const int h0 = k0 / 2, h1 = k1 / 2;
    p = x2_mul(p, x2(pow2i(h0), pow2i(h1)));
    p = x2_mul(p, x2(pow2i(k0 - h0), pow2i(k1 - h1)));
    float e0, e1;
    x2_split(p, e0, e1);
    // the range cases of exp_cw, lane by lane (the pair was computed regardless; its value is not used there)
    if (v0 != v0) e0 = v0;
    else if (v0 > 88.7228394f) e0 = __int_as_float(0x7F800000);
    else if (v0 < -103.972084f) e0 = 0.0f;
    if (v1 != v1) e1 = v1;
    else if (v1 > 88.7228394f) e1 = __int_as_float(0x7F800000);
    else if (v1 < -103.972084f) e1 = 0.0f;
    return x2(e0, e1);
}

// rbf16(gelu_tanh(rbf16(v))) of two finite values (kernels.py:126-127): gelu_tanh's operations on an f32x2
// pair - products on packed multiplies, every addition or subtraction whose operand is a product scalar (a
// packed product is never fed to a packed addition) - and the bf16 roundings by one cvt.rn.bf16x2 each
__device__ __forceinline__ void gelu_bf16_pair(float &a, float &b) {
    uint32_t w = bf16x2_rn(a, b);
    const uint64_t x = x2(bf16_lo(w), bf16_hi(w));
    const uint64_t x3 = x2_mul(x2_mul(x2_mul(x2_splat(0.044715f), x), x), x);
    float x0, x1, c0, c1;
    x2_split(x, x0, x1);
    x2_split(x3, c0, c1);
    const uint64_t inner = x2_mul(x2_splat(0.7978845608028654f), x2(__fadd_rn(x0, c0), __fadd_rn(x1, c1)));
    // exp(-z), z = 2 * inner: the product by -2 is exact and equals -RN(2 * inner)
    float e0, e1;
    x2_split(exp_cw_x2(x2_mul(x2_splat(-2.0f), inner)), e0, e1);
    const uint64_t sig2 = x2_mul(x2_splat(2.0f), x2(__frcp_rn(__fadd_rn(1.0f, e0)), __frcp_rn(__fadd_rn(1.0f, e1))));
    float s0, s1;
    x2_split(sig2, s0, s1);
    const uint64_t t = x2(__fadd_rn(1.0f, __fsub_rn(s0, 1.0f)), __fadd_rn(1.0f, __fsub_rn(s1, 1.0f)));
    float g0, g1;
    x2_split(x2_mul(x2_mul(x2_splat(0.5f), x), t), g0, g1);
    w = bf16x2_rn(g0, g1);
    a = bf16_lo(w);
    b = bf16_hi(w);
}

// ---------------------------------------------------------------------------------------------------
// vector loads: 8 bf16 / fp16 or 4 fp32 elements -> fp32

template <typename T> struct Elem;
template <> struct Elem<__nv_bfloat16> {
    static __device__ __forceinline__ void load8(const __nv_bfloat16 *p, float *v) {
        uint4 w = *reinterpret_cast<const uint4 *>(p);
        v[0] = bf16_lo(w.x); v[1] = bf16_hi(w.x); v[2] = bf16_lo(w.y); v[3] = bf16_hi(w.y);
        v[4] = bf16_lo(w.z); v[5] = bf16_hi(w.z); v[6] = bf16_lo(w.w); v[7] = bf16_hi(w.w);
    }
    static __device__ __forceinline__ float load1(const __nv_bfloat16 *p) { return __bfloat162float(*p); }
};
template <> struct Elem<__half> {
    static __device__ __forceinline__ void load8(const __half *p, float *v) {
        uint4 w = *reinterpret_cast<const uint4 *>(p);
        const __half2 *h = reinterpret_cast<const __half2 *>(&w);
        for (int i = 0; i < 4; ++i) { float2 f = __half22float2(h[i]); v[2 * i] = f.x; v[2 * i + 1] = f.y; }
    }
    static __device__ __forceinline__ float load1(const __half *p) { return __half2float(*p); }
};
template <> struct Elem<float> {
    static __device__ __forceinline__ void load8(const float *p, float *v) {
        float4 a = *reinterpret_cast<const float4 *>(p), b = *reinterpret_cast<const float4 *>(p + 4);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    }
    static __device__ __forceinline__ float load1(const float *p) { return *p; }
};

// streaming 16-byte load that does not allocate in L1
__device__ __forceinline__ uint4 ldg_stream(const void *p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}

// max(m, |a|, |b|) in one three-input max (PTX max.abs.f32 with three operands, sm_100); m >= 0. As fmaxf, a NaN
// input is ignored.
__device__ __forceinline__ float absmax3(float m, float a, float b) {
    float r;
    asm("max.abs.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(m), "f"(a), "f"(b));
    return r;
}

// ---------------------------------------------------------------------------------------------------
// warp reductions

__device__ __forceinline__ float warp_max_xor(float v, int width) {
    for (int o = 1; o < width; o <<= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
// butterfly sum over the 32 lanes: every lane ends with the same balanced pairwise tree in lane order
__device__ __forceinline__ float warp_sum_tree(float v) {
    for (int o = 1; o < 32; o <<= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// pairwise tree of 16 values in index order
__device__ __forceinline__ float tree16(const float *v) {
    float a[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) a[i] = __fadd_rn(v[2 * i], v[2 * i + 1]);
#pragma unroll
    for (int i = 0; i < 4; ++i) a[i] = __fadd_rn(a[2 * i], a[2 * i + 1]);
    a[0] = __fadd_rn(a[0], a[1]);
    a[1] = __fadd_rn(a[2], a[3]);
    return __fadd_rn(a[0], a[1]);
}

// ---------------------------------------------------------------------------------------------------
// time

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__host__ __device__ constexpr int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

// a / d for 0 <= a, 0 < d: a shift when d is a power of two, a 32-bit unsigned division when both fit (a few
// instructions instead of the 64-bit division routine), the 64-bit one otherwise
__device__ __forceinline__ int64_t div_nonneg(int64_t a, int64_t d) {
    if ((d & (d - 1)) == 0) return a >> (__ffsll(d) - 1);
    if (((uint64_t)a | (uint64_t)d) <= 0xFFFFFFFFull) return (int64_t)((uint32_t)a / (uint32_t)d);
    return a / d;
}

} // namespace hn
