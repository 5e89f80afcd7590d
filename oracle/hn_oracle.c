/*
 * hn_oracle.c - CPU restatement of the ComfyUI-Hy-Nomas quantized DiT linear path.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the checker that the CUDA kernels are compared against; it is
 * loaded by tests/, by __graft_entry__.smoke() and by bench.py's CPU-baseline leg, and by nothing that
 * ships. It is compiled with -ffp-contract=off so every float operation below is one IEEE-754 binary32
 * operation with round-to-nearest-even, exactly as written.
 *
 * Parity is pinned: tests/test_oracle_golden.py checks these functions against golden vectors produced
 * by running the reference's own code (its Triton kernels under the Triton CPU interpreter, with the
 * interpreter's fp32->bf16 cast corrected to round-to-nearest-even, and its torch functions) - see
 * tests/golden/make_golden.py.
 *
 * Where the reference leaves an arithmetic detail to its compiler (the order of a tl.sum reduction, the
 * lowering of tl.rsqrt / tl.sigmoid / exp, FMA contraction), the reference fixes no bit pattern. This
 * restatement fixes one, and the CUDA kernels follow the same choice:
 *  - sums over a row are a balanced pairwise tree in index order over the row zero-padded to a power of
 *    two (>= 512 elements for the LayerNorm rows, 64 elements per even/odd half for the QK RMSNorm);
 *  - rsqrt(v) is 1 / sqrt(v) with both operations correctly rounded (what the interpreter computes);
 *  - exp is the Cody-Waite reduction + degree-7 Taylor polynomial of hn_expf below;
 *  - products and sums that torch evaluates as separate ops (modulate, RoPE, gated residual) are
 *    separate roundings; the GEMM scale promotion uses one FMA per group (see or_block_gemm).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define GROUP 128

static inline float f32_of(uint32_t b) { float f; memcpy(&f, &b, 4); return f; }
static inline uint32_t bits_of(float f) { uint32_t b; memcpy(&b, &f, 4); return b; }

/* hy_nomas/kernels.py:67-71 and hy_nomas/fused.py:29-34 (_rbf16): nearest-even bf16, kept as fp32. */
static inline float rbf16(float x) {
    uint32_t b = bits_of(x);
    b = (b + (((b >> 16) & 1u) + 0x7FFFu)) & 0xFFFF0000u;
    return f32_of(b);
}

/* round half away from zero, clamp to +-127: kernels.py:33-36, ops.py:47-51, world.py:86-89 */
static inline int8_t code_i8(float y) {
    float r = (y >= 0.0f) ? floorf(y + 0.5f) : ceilf(y - 0.5f);
    if (r < -127.0f) r = -127.0f;
    if (r > 127.0f) r = 127.0f;
    return (int8_t)(int)r;
}

/* round half to even, clamp to +-127: torch.round's convention for per-token codes, offered beside the
 * reference's rounding; nearbyintf rounds to nearest even in the default rounding mode */
static inline int8_t code_i8_rne(float y) {
    float r = nearbyintf(y);
    if (r < -127.0f) r = -127.0f;
    if (r > 127.0f) r = 127.0f;
    return (int8_t)(int)r;
}

/* fp32 -> float8_e4m3fn byte, round to nearest even, saturating to +-448 (the .satfinite conversion the
 * GPU path uses, equal to torch's .to(float8_e4m3fn) for |x| < 464). */
uint8_t or_e4m3_from_f32(float x) {
    uint8_t sign = (uint8_t)((bits_of(x) >> 31) << 7);
    if (isnan(x)) return 0x7F;
    float a = fabsf(x);
    if (a >= 448.0f) return sign | 0x7E;
    if (a == 0.0f) return sign;
    int e;
    frexpf(a, &e);
    int E = e - 1;                   /* a in [2^E, 2^(E+1)) */
    if (E < -6) E = -6;              /* below 2^-6 the quantum is the subnormal step 2^-9 */
    float quantum = ldexpf(1.0f, E - 3);
    float v = rintf(a / quantum) * quantum; /* both exact scalings; rintf rounds half to even */
    if (v > 448.0f) v = 448.0f;
    if (v == 0.0f) return sign;
    frexpf(v, &e);
    E = e - 1;
    if (E < -6) return sign | (uint8_t)(int)(v / ldexpf(1.0f, -9));
    int mant = (int)((v / ldexpf(1.0f, E) - 1.0f) * 8.0f);
    return sign | (uint8_t)(((E + 7) << 3) | mant);
}

float or_f32_from_e4m3(uint8_t b) {
    int s = b >> 7, E = (b >> 3) & 15, m = b & 7;
    float v;
    if (E == 15 && m == 7) return NAN;
    if (E == 0) v = ldexpf((float)m, -9);
    else v = ldexpf(1.0f + m / 8.0f, E - 7);
    return s ? -v : v;
}

/* balanced pairwise sum of v[0..n) zero-padded to the power of two p >= n */
static float pairwise(const float *v, int64_t n, int64_t p) {
    if (p == 1) return n > 0 ? v[0] : 0.0f;
    int64_t h = p / 2;
    float a = pairwise(v, n < h ? n : h, h);
    float b = (n > h) ? pairwise(v + h, n - h, h) : 0.0f;
    return a + b;
}

static int64_t row_pad(int64_t D) {
    /* the LayerNorm kernels give each thread 16 contiguous elements, 32 threads per warp, and a
     * power-of-two number of warp partials: the tree spans 512 * next_pow2(ceil(D / 512)) slots */
    int64_t w = (D + 511) / 512, wp = 1;
    while (wp < w) wp <<= 1;
    return 512 * wp;
}

/* ---------------------------------------------------------------------------------------------------
 * exp, sigmoid and GELU.  hn_expf: Cody & Waite (1980) argument reduction x = k ln2 + r with ln2 split
 * into a 24-bit head and a tail (the split fdlibm's expf uses), then the Taylor series of e^r to degree 7
 * in Horner form with fused multiply-adds, then scaling by 2^k in two exact steps. |r| <= ln2/2, so the
 * truncation error r^8/8! < 1e-8 relative. Accuracy is tested against the C library's expf.
 */
float or_expf(float x) {
    if (isnan(x)) return x;
    if (x > 88.7228394f) return INFINITY;
    if (x < -103.972084f) return 0.0f;
    const float log2e = 0x1.715476p+0f, ln2_hi = 0x1.62e4p-1f, ln2_lo = 0x1.7f7d1cp-20f;
    float kf = rintf(x * log2e);
    float r = fmaf(-kf, ln2_hi, x);
    r = fmaf(-kf, ln2_lo, r);
    float p = 0x1.a01a02p-13f;          /* 1/7! rounded to binary32 */
    p = fmaf(p, r, 0x1.6c16c2p-10f);    /* 1/6! */
    p = fmaf(p, r, 0x1.111112p-7f);     /* 1/5! */
    p = fmaf(p, r, 0x1.555556p-5f);     /* 1/4! */
    p = fmaf(p, r, 0x1.555556p-3f);     /* 1/3! */
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    int k = (int)kf;              /* -150 <= k <= 128 */
    int k1 = k / 2, k2 = k - k1;  /* each half within the normal exponent range */
    p = p * f32_of((uint32_t)(k1 + 127) << 23);
    p = p * f32_of((uint32_t)(k2 + 127) << 23);
    return p;
}

/* hy_nomas/kernels.py:74-77 (_gelu_tanh), evaluated left to right as written, one rounding per op;
 * tl.sigmoid(z) = 1 / (1 + exp(-z)) (triton/language/standard.py). */
float or_gelu_tanh(float x) {
    float x3 = ((0.044715f * x) * x) * x;
    float inner = 0.7978845608028654f * (x + x3);
    float z = 2.0f * inner;
    float sig = 1.0f / (1.0f + or_expf(-z));
    return (0.5f * x) * (1.0f + (2.0f * sig - 1.0f));
}

/* ---------------------------------------------------------------------------------------------------
 * K1 - hy_nomas/kernels.py:22-42 (_quantize_kernel). x fp32 [M, K] (the bf16 input widened exactly);
 * kind 0: int8, 1: e4m3, 2: int8 with codes rounded half to even. group = 128, or K for the per-token
 * variant (one scale per row).
 */
void or_quant_act(const float *x, int64_t M, int64_t K, int kind, int64_t group, uint8_t *q, float *s) {
    int64_t G = K / group;
    for (int64_t m = 0; m < M; ++m)
        for (int64_t g = 0; g < G; ++g) {
            const float *v = x + m * K + g * group;
            float peak = 0.0f;
            for (int64_t i = 0; i < group; ++i) peak = fmaxf(peak, fabsf(v[i]));
            float scale;
            if (kind == 0 || kind == 2) {
                scale = (peak > 0.0f) ? peak / 127.0f : 1.0f;
                for (int64_t i = 0; i < group; ++i)
                    q[m * K + g * group + i] = (uint8_t)(kind == 0 ? code_i8(v[i] / scale) : code_i8_rne(v[i] / scale));
            } else {
                scale = fmaxf(peak, 1e-12f) / 448.0f;
                for (int64_t i = 0; i < group; ++i) q[m * K + g * group + i] = or_e4m3_from_f32(v[i] / scale);
            }
            s[m * G + g] = scale;
        }
}

/* hy_nomas/ops.py:41-52 (quantize_g128) for K % 128 == 0: the same arithmetic as K1's int8 branch
 * ((|x/s| + 0.5).floor() * sign == floor/ceil half-away). */
void or_quantize_g128(const float *w, int64_t N, int64_t K, int8_t *q, float *s) {
    or_quant_act(w, N, K, 0, GROUP, (uint8_t *)q, s);
}

/* hy_nomas/pixelumm.py:77-82 (NomasFP8Block128Layout.quantize): 128x128 blocks, clamp_min(1e-4)/448. */
void or_quantize_fp8_block(const float *w, int64_t N, int64_t K, uint8_t *q, float *s) {
    int64_t NB = N / 128, KB = K / 128;
    for (int64_t bn = 0; bn < NB; ++bn)
        for (int64_t bk = 0; bk < KB; ++bk) {
            float peak = 0.0f;
            for (int64_t i = 0; i < 128; ++i)
                for (int64_t j = 0; j < 128; ++j) peak = fmaxf(peak, fabsf(w[(bn * 128 + i) * K + bk * 128 + j]));
            float sc = fmaxf(peak, 1e-4f) / 448.0f;
            s[bn * KB + bk] = sc;
            for (int64_t i = 0; i < 128; ++i)
                for (int64_t j = 0; j < 128; ++j) {
                    int64_t o = (bn * 128 + i) * K + bk * 128 + j;
                    q[o] = or_e4m3_from_f32(w[o] / sc);
                }
        }
}

/* ---------------------------------------------------------------------------------------------------
 * K2 - hy_nomas/kernels.py:80-137 (_gemm_body).
 * qa [M,K], qw [N,K] codes (int8, or e4m3 bytes when kind == 1). Scale modes as in hynomas_b200.h
 * (0 per row x group, 1 per row, 2 per 128x128 block for sw). bias fp32 [N] or NULL (bf16 values).
 * Promotion per 128-K group g with part = the exact group dot (int32 for int8; for e4m3 the exact dot
 * rounded once to fp32):
 *   sa group, sw group (kernels.py:115):      t = RN(part*sa[m,g]); acc = fma(t, sw[n,g], acc)
 *        (fma == 0: acc = RN(acc + RN(t*sw[n,g])), the interpreter's / torch's separate roundings)
 *   sa row,   sw group: as above with sa[m,g] = sa[m]
 *   sa group, sw row:  acc = fma(part, sa[m,g], acc); at the end acc = RN(acc * sw[n])
 *   sa any,   sw block: acc = fma(part, RN(sa[m,g] * swb[n/128,g]), acc)
 *   sa row,   sw row:  whole-K dot D (int32 exact for int8); acc = RN(RN(RN32(D) * sa[m]) * sw[n])
 * then acc = RN(acc + bias[n]) and the epilogue:
 *   0: out = acc;  1: h = rbf16(gelu(rbf16(acc)));  2: h as in 1, then int8 per row and 128 columns
 *   (kernels.py:126-137) -> codes qh [M,N], scales qs [M,N/128].
 * out receives acc (epilogue 0) or h (1, 2) as fp32.
 */
void or_block_gemm(const uint8_t *qa, const float *sa, int sa_mode, const uint8_t *qw, const float *sw, int sw_mode,
                   const float *bias, int64_t M, int64_t N, int64_t K, int kind, int epilogue, int fma_mode,
                   float *out, int8_t *qh, float *qs) {
    int64_t G = K / GROUP;
    #pragma omp parallel for schedule(static)
    for (int64_t m = 0; m < M; ++m) {
        for (int64_t n = 0; n < N; ++n) {
            float acc = 0.0f;
            const uint8_t *a = qa + m * K, *b = qw + n * K;
            if (sa_mode == 1 && sw_mode == 1) {
                float d;
                if (kind == 0) {
                    int64_t dot = 0;
                    for (int64_t k = 0; k < K; ++k) dot += (int64_t)(int8_t)a[k] * (int64_t)(int8_t)b[k];
                    d = (float)dot; /* RN32 of the exact integer (|dot| < 2^31) */
                } else {
                    double dd = 0.0;
                    for (int64_t k = 0; k < K; ++k) dd += (double)or_f32_from_e4m3(a[k]) * or_f32_from_e4m3(b[k]);
                    d = (float)dd;
                }
                acc = (d * sa[m]) * sw[n];
            } else {
                for (int64_t g = 0; g < G; ++g) {
                    float part;
                    if (kind == 0) {
                        int32_t dot = 0;
                        for (int64_t k = g * GROUP; k < (g + 1) * GROUP; ++k) dot += (int32_t)(int8_t)a[k] * (int32_t)(int8_t)b[k];
                        part = (float)dot; /* exact: |dot| <= 128*127^2 < 2^22 */
                    } else {
                        double dd = 0.0; /* e4m3 products are exact in double and so is their sum */
                        for (int64_t k = g * GROUP; k < (g + 1) * GROUP; ++k)
                            dd += (double)or_f32_from_e4m3(a[k]) * or_f32_from_e4m3(b[k]);
                        part = (float)dd;
                    }
                    float sag = (sa_mode == 0) ? sa[m * G + g] : sa[m];
                    if (sw_mode == 2) {
                        float s = sag * sw[(n / 128) * G + g];
                        acc = fmaf(part, s, acc);
                    } else if (sw_mode == 1) {
                        acc = fmaf(part, sag, acc);
                    } else {
                        float t = part * sag;
                        float swg = sw[n * G + g];
                        if (fma_mode) acc = fmaf(t, swg, acc);
                        else acc = acc + t * swg;
                    }
                }
                if (sw_mode == 1) acc = acc * sw[n];
            }
            if (bias) acc = acc + bias[n];
            if (epilogue == 0) out[m * N + n] = acc;
            else out[m * N + n] = rbf16(or_gelu_tanh(rbf16(acc)));
        }
        if (epilogue == 2) {
            for (int64_t c = 0; c < N / 128; ++c) {
                float peak = 0.0f;
                for (int64_t j = 0; j < 128; ++j) peak = fmaxf(peak, fabsf(out[m * N + c * 128 + j]));
                float scale = (peak > 0.0f) ? peak / 127.0f : 1.0f;
                for (int64_t j = 0; j < 128; ++j) qh[m * N + c * 128 + j] = code_i8(out[m * N + c * 128 + j] / scale);
                qs[m * (N / 128) + c] = scale;
            }
        }
    }
}

/* ---------------------------------------------------------------------------------------------------
 * LayerNorm rows (K3 / K4 / K6+K3).  hy_nomas/kernels.py:181-188, hy_nomas/fused.py:43-51:
 *   mean = sum(x)/D; xc = x - mean; var = sum(xc*xc)/D; n = xc * rsqrt(var + eps)
 *   y = n * rbf16(1 + scale) + shift   (torch's modulate: separate roundings, model.py:109-111)
 */
static void ln_modulate_row(const float *x, const float *shift, const float *scale, int64_t D, float eps,
                            float *y, float *tmp) {
    int64_t P = row_pad(D);
    float sum = pairwise(x, D, P);
    float mean = sum / (float)D;
    for (int64_t i = 0; i < D; ++i) { float c = x[i] - mean; tmp[i] = c * c; }
    float var = pairwise(tmp, D, P) / (float)D;
    float rstd = 1.0f / sqrtf(var + eps);
    for (int64_t i = 0; i < D; ++i) {
        float n = (x[i] - mean) * rstd;
        float r = rbf16(1.0f + scale[i]);
        y[i] = n * r + shift[i];
    }
}

/* K4 - hy_nomas/fused.py:37-52. y receives fp32 values; the caller rounds to bf16 (one rounding, as
 * the kernel's final store). */
void or_adaln(const float *x, const float *shift, const float *scale, int64_t B, int64_t L, int64_t D, float eps,
              float *y) {
    float *tmp = (float *)malloc(sizeof(float) * D);
    for (int64_t r = 0; r < B * L; ++r) {
        int64_t b = r / L;
        ln_modulate_row(x + r * D, shift + b * D, scale + b * D, D, eps, y + r * D, tmp);
    }
    free(tmp);
}

static void quant_row_i8(const float *y, int64_t D, int8_t *q, float *s) {
    for (int64_t g = 0; g < D / GROUP; ++g) {
        float peak = 0.0f;
        for (int64_t i = 0; i < GROUP; ++i) peak = fmaxf(peak, fabsf(y[g * GROUP + i]));
        float sc = (peak > 0.0f) ? peak / 127.0f : 1.0f;
        for (int64_t i = 0; i < GROUP; ++i) q[g * GROUP + i] = code_i8(y[g * GROUP + i] / sc);
        s[g] = sc;
    }
}

/* K3 - hy_nomas/kernels.py:173-195: rbf16(modulated LN) then int8 per 128 channels. */
void or_adaln_quant(const float *x, const float *shift, const float *scale, int64_t B, int64_t L, int64_t D,
                    float eps, int8_t *q, float *s) {
    float *y = (float *)malloc(sizeof(float) * D), *tmp = (float *)malloc(sizeof(float) * D);
    for (int64_t r = 0; r < B * L; ++r) {
        int64_t b = r / L;
        ln_modulate_row(x + r * D, shift + b * D, scale + b * D, D, eps, y, tmp);
        for (int64_t i = 0; i < D; ++i) y[i] = rbf16(y[i]);
        quant_row_i8(y, D, q + r * D, s + r * (D / GROUP));
    }
    free(y);
    free(tmp);
}

/* K6 - hy_nomas/fused.py:108-118: out = x + rbf16(y * gate[b]) (fp32; the caller rounds to bf16). */
void or_gated_residual(const float *x, const float *y, const float *gate, int64_t B, int64_t L, int64_t D,
                       float *out) {
    for (int64_t r = 0; r < B * L; ++r) {
        int64_t b = r / L;
        for (int64_t i = 0; i < D; ++i) out[r * D + i] = x[r * D + i] + rbf16(y[r * D + i] * gate[b * D + i]);
    }
}

/* K6+K3 - model.py:280-282 fused: xo = bf16(x + rbf16(y*gate)); (q, s) = adaln_quant(xo). xo is returned
 * bf16-valued (already rounded). */
void or_gated_residual_adaln_quant(const float *x, const float *y, const float *gate, const float *shift,
                                   const float *scale, int64_t B, int64_t L, int64_t D, float eps, float *xo,
                                   int8_t *q, float *s) {
    or_gated_residual(x, y, gate, B, L, D, xo);
    for (int64_t i = 0; i < B * L * D; ++i) xo[i] = rbf16(xo[i]);
    or_adaln_quant(xo, shift, scale, B, L, D, eps, q, s);
}

/* ---------------------------------------------------------------------------------------------------
 * K5 - hy_nomas/fused.py:65-91 for one tensor. x fp32 [B*L, H*D] gathered contiguous (D == 128);
 * cos/sin [L, D] or NULL. y fp32 (bf16-valued) [B*L, H, D].
 *   r = rsqrt((sum(xe^2) + sum(xo^2)) / D + eps); n = rbf16(rbf16(x*r) * w)
 *   RoPE (model.py:131-138): oe = ne*ce - no*se, oo = no*co + ne*so, rounded once to bf16.
 * Each half-sum is a pairwise tree over the 64 even (odd) squares in index order.
 */
void or_qk_norm_rope(const float *x, const float *w, const float *cos, const float *sin, int64_t B, int64_t L,
                     int64_t H, int64_t D, float eps, float *y) {
    float se[64], so[64];
    int64_t half = D / 2;
    for (int64_t t = 0; t < B * L; ++t) {
        int64_t l = t % L;
        for (int64_t h = 0; h < H; ++h) {
            const float *v = x + (t * H + h) * D;
            float *o = y + (t * H + h) * D;
            for (int64_t i = 0; i < half; ++i) { se[i] = v[2 * i] * v[2 * i]; so[i] = v[2 * i + 1] * v[2 * i + 1]; }
            float ss = pairwise(se, half, half) + pairwise(so, half, half);
            float r = 1.0f / sqrtf(ss / (float)D + eps);
            for (int64_t i = 0; i < half; ++i) {
                float ne = rbf16(rbf16(v[2 * i] * r) * w[2 * i]);
                float no = rbf16(rbf16(v[2 * i + 1] * r) * w[2 * i + 1]);
                if (cos) {
                    const float *c = cos + l * D, *s = sin + l * D;
                    o[2 * i] = rbf16(ne * c[2 * i] - no * s[2 * i]);
                    o[2 * i + 1] = rbf16(no * c[2 * i + 1] + ne * s[2 * i + 1]);
                } else {
                    o[2 * i] = ne;
                    o[2 * i + 1] = no;
                }
            }
        }
    }
}

/* ---------------------------------------------------------------------------------------------------
 * K7 - hy_nomas/fused.py:131-175 (_pixelumm_qk_kernel), D == 128. x fp32 [N*H, D]; wt/whw [D/2];
 * cos/sin [N, D]. y fp32 (bf16-valued).
 *   T half:  rt  = rsqrt((sum(t0^2) + sum(t1^2)) / (D/2) + eps)
 *   HW half: rhw = rsqrt((((sum(h0^2) + sum(h1^2)) + sum(w0^2)) + sum(w1^2)) / (D/2) + eps)
 * each sum a pairwise tree in index order; x * r * w evaluated left to right.
 */
void or_pixelumm_qk(const float *x, const float *wt, const float *whw, const float *cos, const float *sin,
                    int64_t N, int64_t H, int64_t D, float eps, float *y) {
    const int64_t half = D / 2, quarter = D / 4, eighth = D / 8;
    float sq[128];
    for (int64_t row = 0; row < N * H; ++row) {
        int64_t tok = row / H;
        const float *v = x + row * D;
        float *o = y + row * D;
        for (int64_t i = 0; i < D; ++i) sq[i] = v[i] * v[i];
        float st = pairwise(sq, quarter, quarter) + pairwise(sq + quarter, quarter, quarter);
        float shw = ((pairwise(sq + half, eighth, eighth) + pairwise(sq + half + eighth, eighth, eighth)) +
                     pairwise(sq + half + quarter, eighth, eighth)) + pairwise(sq + half + quarter + eighth, eighth, eighth);
        float rt = 1.0f / sqrtf(st / (float)half + eps);
        float rhw = 1.0f / sqrtf(shw / (float)half + eps);
        const float *cb = cos + tok * D, *sb = sin + tok * D;
        for (int64_t i = 0; i < quarter; ++i) {
            float t0 = (v[i] * rt) * wt[i];
            float t1 = (v[quarter + i] * rt) * wt[quarter + i];
            o[i] = rbf16(t0 * cb[i] - t1 * sb[i]);
            o[quarter + i] = rbf16(t1 * cb[quarter + i] + t0 * sb[quarter + i]);
        }
        for (int64_t j = 0; j < eighth; ++j) {
            float h0 = (v[half + j] * rhw) * whw[j];
            float h1 = (v[half + eighth + j] * rhw) * whw[eighth + j];
            float w0 = (v[half + quarter + j] * rhw) * whw[quarter + j];
            float w1 = (v[half + quarter + eighth + j] * rhw) * whw[quarter + eighth + j];
            o[half + j] = rbf16(h0 * cb[half + j] - h1 * sb[half + j]);
            o[half + eighth + j] = rbf16(h1 * cb[half + eighth + j] + h0 * sb[half + eighth + j]);
            o[half + quarter + j] = rbf16(w0 * cb[half + quarter + j] - w1 * sb[half + quarter + j]);
            o[half + quarter + eighth + j] =
                rbf16(w1 * cb[half + quarter + eighth + j] + w0 * sb[half + quarter + eighth + j]);
        }
    }
}

/* hy_nomas/world.py:83-90 (quantize_kv): per row (token, head) absmax/127, half away from zero. */
void or_quantize_kv(const float *x, int64_t rows, int64_t D, int8_t *q, float *s) {
    for (int64_t r = 0; r < rows; ++r) {
        float peak = 0.0f;
        for (int64_t i = 0; i < D; ++i) peak = fmaxf(peak, fabsf(x[r * D + i]));
        float sc = (peak > 0.0f) ? peak / 127.0f : 1.0f;
        for (int64_t i = 0; i < D; ++i) q[r * D + i] = code_i8(x[r * D + i] / sc);
        s[r] = sc;
    }
}

/* hy_nomas/world.py:93-94 (dequantize_kv): bf16(float(q) * s), s per row of D codes; y holds the bf16 values
 * as fp32. */
void or_dequantize_kv(const int8_t *q, const float *s, int64_t rows, int64_t D, float *y) {
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t i = 0; i < D; ++i) y[r * D + i] = rbf16((float)q[r * D + i] * s[r]);
}

/* ---------------------------------------------------------------------------------------------------
 * Helpers the tests use: bf16 rounding of fp32 arrays, and the Markstein-corrected quotient that the
 * quantizers may use in place of a division (checked here against IEEE division on the CPU).
 */
/* ---------------------------------------------------------------------------------------------------
 * PixelUMM decoder fusions (the RMSNorm and SiLU fusions the reference's notes name, README.md:266), each
 * ending in the activation quantizer (kernels.py:22-42) of the linears that read its output: the FP8 decoder
 * linears quantize their input per 1 x 128 through block_linear (pixelumm.py:147-155).
 *
 * or_rmsnorm_quant - pixelumm.py:246-259 (Qwen3 RMSNorm): ss = sum of x^2, a balanced pairwise tree in index
 * order over the row zero-padded to 2048 * next_pow2(ceil(D / 2048)) (the kernel's layout: 8-element chunks,
 * chunk c held by thread c % 256 of a 256-thread CTA); ms = ss / D; r = 1 / sqrt(ms + eps);
 * y = rbf16(w * rbf16(x * r)) (normalize in fp32, cast to bf16, times the bf16 weight); then codes and scales
 * per 128 (kind 0 int8, 1 e4m3).
 */
static int64_t chunk_pad(int64_t D) {
    int64_t n = (D + 2047) / 2048, p = 1;
    while (p < n) p <<= 1;
    return 2048 * p;
}

void or_rmsnorm_quant(const float *x, const float *w, int64_t rows, int64_t D, float eps, int kind, uint8_t *q,
                      float *s) {
    float *sq = (float *)malloc(sizeof(float) * D), *y = (float *)malloc(sizeof(float) * D);
    const int64_t P = chunk_pad(D);
    for (int64_t r = 0; r < rows; ++r) {
        const float *xr = x + r * D;
        for (int64_t i = 0; i < D; ++i) sq[i] = xr[i] * xr[i];
        float ms = pairwise(sq, D, P) / (float)D;
        float rs = 1.0f / sqrtf(ms + eps);
        for (int64_t i = 0; i < D; ++i) y[i] = rbf16(w[i] * rbf16(xr[i] * rs));
        or_quant_act(y, 1, D, kind, GROUP, q + r * D, s + r * (D / GROUP));
    }
    free(sq);
    free(y);
}

/* or_silu_mul_quant - pixelumm.py:322-323 (MLP.forward): h = silu(gate) * up with torch's bf16 roundings,
 * silu(g) = g / (1 + exp(-g)) in fp32 rounded to bf16 (exp: this oracle's, the kernels' own), times u, rounded
 * to bf16; then codes and scales per 128 for down_proj. g, u [rows, I] (bf16 values as fp32). */
void or_silu_mul_quant(const float *g, const float *u, int64_t rows, int64_t I, int kind, uint8_t *q, float *s) {
    float *h = (float *)malloc(sizeof(float) * I);
    for (int64_t r = 0; r < rows; ++r) {
        for (int64_t i = 0; i < I; ++i) {
            float gv = g[r * I + i];
            float sl = rbf16(gv / (1.0f + or_expf(-gv)));
            h[i] = rbf16(sl * u[r * I + i]);
        }
        or_quant_act(h, 1, I, kind, GROUP, q + r * I, s + r * (I / GROUP));
    }
    free(h);
}

void or_round_bf16(const float *x, int64_t n, float *y) {
    for (int64_t i = 0; i < n; ++i) y[i] = rbf16(x[i]);
}

void or_expf_array(const float *x, int64_t n, float *y) {
    for (int64_t i = 0; i < n; ++i) y[i] = or_expf(x[i]);
}

void or_gelu_array(const float *x, int64_t n, float *y) {
    for (int64_t i = 0; i < n; ++i) y[i] = or_gelu_tanh(x[i]);
}
