// norm.cu - the fused DiT elementwise kernels around the GEMMs:
//   K3 adaln_quant       hy_nomas/kernels.py:173-207
//   K4 adaln             hy_nomas/fused.py:37-62
//   K6 gated_residual    hy_nomas/fused.py:108-128
//   K6+K3                hy_nomas/model.py:280-282 (residual, then the next LayerNorm/modulate/quantize)
//   K5 qk_norm_rope      hy_nomas/fused.py:65-105 (one or two tensors per launch)
//   K7 pixelumm_qk       hy_nomas/fused.py:131-186
// All are HBM-bound single passes. Rows of a LayerNorm are handled by one CTA: thread t owns the 16
// contiguous elements [16t, 16t+16), so a 128-channel quantization group is 8 adjacent lanes and the
// row sums are one balanced pairwise tree (in-thread -> butterfly over lanes -> over warps, the warp
// partials zero-padded to a power of two). The CPU oracle evaluates the same tree.
#include "hn_common.cuh"
#include "hn_kernels.h"

namespace hn {

typedef __nv_bfloat16 bf16;


// balanced pairwise tree over WP (power of two) values in index order
template <int WP> __device__ __forceinline__ float tree_smem(const float *red) {
    float t[WP];
#pragma unroll
    for (int i = 0; i < WP; ++i) t[i] = red[i];
#pragma unroll
    for (int n = WP; n > 1; n >>= 1) {
#pragma unroll
        for (int i = 0; i < n / 2; ++i) t[i] = __fadd_rn(t[2 * i], t[2 * i + 1]);
    }
    return t[0];
}

// ---------------------------------------------------------------------------------------------------
// LayerNorm rows (K3, K4, K6+K3), persistent: MODE 0: y = bf16(modulate(LN(x))); MODE 1: int8 codes/scales
// of rbf16(modulate(LN(x))); MODE 2: x' = bf16(x + rbf16(y * gate)), stored, then MODE 1 on x'. Each CTA walks rows blockIdx.x, +gridDim.x, ... and prefetches the next row's inputs before reducing
// the current one; rbf16(1 + scale), shift (and the gate) are formed once per batch item. The thread's 16
// elements are held as packed pairs so the per-element work runs on the f32x2 pipes:
//   P[k] = (e[2k], e[2k+8]), Q[k] = (e[2k+1], e[2k+9]),  k = 0..3   (e = the thread's 16 elements)
// With this pairing the tree of tree16 is vertical pair additions: P[k]+Q[k] = (a[k], a[k+4]) with
// a[i] = e[2i]+e[2i+1]; (a0,a4)+(a1,a5) = (b0,b2); (a2,a6)+(a3,a7) = (b1,b3); (b0,b2)+(b1,b3) = (c0,c1).
// bf16 rounding is the cvt.rn.bf16x2 instruction, the quantizer's division the exact fma-corrected quotient
// of x2_quot, the code the round-half-away of x2_codes. A packed product is never fed straight into a packed
// addition (measured here: that pair can come out with one rounding, as a fused multiply-add); the sums of
// products (the squares of the variance, "+ shift") are scalar __fadd_rn.

struct Row16 {
    uint64_t P[4], Q[4];
};
// 8 bf16x2 words (elements 0..15 in order) -> pairs
__device__ __forceinline__ Row16 row_from_words(const uint32_t *w) {
    Row16 r;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        r.P[k] = x2(bf16_lo(w[k]), bf16_lo(w[k + 4]));
        r.Q[k] = x2(bf16_hi(w[k]), bf16_hi(w[k + 4]));
    }
    return r;
}
// pairs -> 8 bf16x2 words in element order, each value rounded to nearest even
__device__ __forceinline__ void words_from_row(const Row16 &r, uint32_t *w) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        float p0, p1, q0, q1;
        x2_split(r.P[k], p0, p1);
        x2_split(r.Q[k], q0, q1);
        w[k] = bf16x2_rn(p0, q0);
        w[k + 4] = bf16x2_rn(p1, q1);
    }
}
__device__ __forceinline__ float row_tree16(const Row16 &r) {
    const uint64_t a0 = x2_add(r.P[0], r.Q[0]), a1 = x2_add(r.P[1], r.Q[1]);
    const uint64_t a2 = x2_add(r.P[2], r.Q[2]), a3 = x2_add(r.P[3], r.Q[3]);
    const uint64_t c = x2_add(x2_add(a0, a1), x2_add(a2, a3));
    float c0, c1;
    x2_split(c, c0, c1);
    return __fadd_rn(c0, c1);
}
__device__ __forceinline__ void load_words16(const bf16 *p, uint32_t *w) {
    const uint4 a = ldg_stream(p), b = ldg_stream(p + 8);
    w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w; w[4] = b.x; w[5] = b.y; w[6] = b.z; w[7] = b.w;
}
__device__ __forceinline__ void store_words16(bf16 *p, const uint32_t *w) {
    reinterpret_cast<uint4 *>(p)[0] = make_uint4(w[0], w[1], w[2], w[3]);
    reinterpret_cast<uint4 *>(p)[1] = make_uint4(w[4], w[5], w[6], w[7]);
}

// MODE 2 with up to 8 warps keeps the batch item's shift and gate in shared memory (each thread reads back only
// its own 16 values), so that three CTAs fit an SM instead of two.
template <int WP, int MODE> struct LnCfg {
    static constexpr bool MOD_SMEM = MODE == 2 && WP <= 8;
    static constexpr int MIN_CTAS = WP <= 8 ? 3 : 1;
};

template <int WP, int MODE>
__global__ void __launch_bounds__(WP * 32, (LnCfg<WP, MODE>::MIN_CTAS)) k_ln_rows(const bf16 *__restrict__ x, const bf16 *__restrict__ yres,
                                                    const bf16 *__restrict__ gate, const bf16 *__restrict__ shift,
                                                    const bf16 *__restrict__ scale, int64_t rows, int64_t L, int D,
                                                    float eps, bf16 *__restrict__ out, int8_t *__restrict__ q,
                                                    float *__restrict__ s, int64_t s_rs, int64_t s_gs) {
    constexpr bool MOD_SMEM = LnCfg<WP, MODE>::MOD_SMEM;
    __shared__ float red1[WP], red2[WP];
    // [shift, gate][P0..3, Q0..3][thread] (MOD_SMEM)
    __shared__ uint64_t mod_s[MOD_SMEM ? 2 : 1][8][MOD_SMEM ? WP * 32 : 1];
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const bool active = t < (D >> 4);
    const float fd = (float)D;
    // for a power-of-two D, sum / D is the exact product sum * 2^-log2(D)
    const float inv_d = (D & (D - 1)) == 0 ? __fdiv_rn(1.0f, fd) : 0.0f;
    int64_t row = blockIdx.x;
    if (row >= rows) return;
    // the row's inputs, prefetched one row ahead
    uint32_t wx[8], wy[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) { wx[i] = 0u; wy[i] = 0u; }
    if (active) {
        load_words16(x + row * (int64_t)D + 16 * t, wx);
        if (MODE == 2) load_words16(yres + row * (int64_t)D + 16 * t, wy);
    }
    int64_t b_end = 0;   // rows [.., b_end) belong to the current batch item (rows only increase)
    Row16 R, SH, G;   // rbf16(1 + scale), shift, gate of the current batch item
    for (; row < rows; row += gridDim.x) {
        if (row >= b_end) {
            const int64_t b = div_nonneg(row, L);
            b_end = (b + 1) * L;
            uint32_t w[8];
            if (active) load_words16(scale + b * (int64_t)D + 16 * t, w);
            else {
#pragma unroll
                for (int i = 0; i < 8; ++i) w[i] = 0u;
            }
            R = row_from_words(w);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                float p0, p1, q0, q1;
                x2_split(x2_add(R.P[k], x2_splat(1.0f)), p0, p1);
                x2_split(x2_add(R.Q[k], x2_splat(1.0f)), q0, q1);
                const uint32_t lo = bf16x2_rn(p0, q0), hi = bf16x2_rn(p1, q1);
                R.P[k] = x2(bf16_lo(lo), bf16_lo(hi));
                R.Q[k] = x2(bf16_hi(lo), bf16_hi(hi));
            }
            if (active) load_words16(shift + b * (int64_t)D + 16 * t, w);
            SH = row_from_words(w);
            if (MODE == 2) {
                if (active) load_words16(gate + b * (int64_t)D + 16 * t, w);
                G = row_from_words(w);
            }
            if (MOD_SMEM) {
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    mod_s[0][k][t] = SH.P[k];
                    mod_s[0][4 + k][t] = SH.Q[k];
                    mod_s[1][k][t] = G.P[k];
                    mod_s[1][4 + k][t] = G.Q[k];
                }
            }
        }
        const int64_t off = row * (int64_t)D + 16 * t;
        // this row's words; start the next row's loads
        uint32_t cx[8], cy[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) { cx[i] = wx[i]; cy[i] = wy[i]; }
        const int64_t nrow = row + gridDim.x;
        if (active && nrow < rows) {
            load_words16(x + nrow * (int64_t)D + 16 * t, wx);
            if (MODE == 2) load_words16(yres + nrow * (int64_t)D + 16 * t, wy);
        }
        Row16 V = row_from_words(cx);
        if (MODE == 2) {
            // x' = rbf16(x + rbf16(y * gate)), stored, then normalized
            const Row16 Y = row_from_words(cy);
            Row16 YG;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                YG.P[k] = x2_mul(Y.P[k], MOD_SMEM ? mod_s[1][k][t] : G.P[k]);
                YG.Q[k] = x2_mul(Y.Q[k], MOD_SMEM ? mod_s[1][4 + k][t] : G.Q[k]);
            }
            uint32_t w[8];
            words_from_row(YG, w);
            YG = row_from_words(w);
#pragma unroll
            for (int k = 0; k < 4; ++k) { V.P[k] = x2_add(V.P[k], YG.P[k]); V.Q[k] = x2_add(V.Q[k], YG.Q[k]); }
            words_from_row(V, w);
            if (active) store_words16(out + off, w);
            V = row_from_words(w);
        }
        // mean
        float part = warp_sum_tree(row_tree16(V));
        if (lane == 0) red1[warp] = part;
        __syncthreads();
        const float mean = inv_d != 0.0f ? __fmul_rn(tree_smem<WP>(red1), inv_d) : __fdiv_rn(tree_smem<WP>(red1), fd);
        // centred values and variance
        const uint64_t nm = x2_splat(-mean);
        Row16 C;
        float sq[16];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            C.P[k] = x2_add(V.P[k], nm);
            C.Q[k] = x2_add(V.Q[k], nm);
            x2_split(active ? x2_mul(C.P[k], C.P[k]) : 0ull, sq[2 * k], sq[2 * k + 8]);
            x2_split(active ? x2_mul(C.Q[k], C.Q[k]) : 0ull, sq[2 * k + 1], sq[2 * k + 9]);
        }
        part = warp_sum_tree(tree16(sq));
        if (lane == 0) red2[warp] = part;
        __syncthreads();
        const float var = inv_d != 0.0f ? __fmul_rn(tree_smem<WP>(red2), inv_d) : __fdiv_rn(tree_smem<WP>(red2), fd);
        const uint64_t rstd = x2_splat(rsqrt_cr(__fadd_rn(var, eps)));
        // modulate: rbf16(n * rbf16(1 + scale) + shift)
        Row16 Z;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            float a0, a1, h0, h1;
            x2_split(x2_mul(x2_mul(C.P[k], rstd), R.P[k]), a0, a1);
            x2_split(MOD_SMEM ? mod_s[0][k][t] : SH.P[k], h0, h1);
            Z.P[k] = x2(__fadd_rn(a0, h0), __fadd_rn(a1, h1));
            x2_split(x2_mul(x2_mul(C.Q[k], rstd), R.Q[k]), a0, a1);
            x2_split(MOD_SMEM ? mod_s[0][4 + k][t] : SH.Q[k], h0, h1);
            Z.Q[k] = x2(__fadd_rn(a0, h0), __fadd_rn(a1, h1));
        }
        uint32_t zw[8];
        words_from_row(Z, zw);
        if (MODE == 0) {
            if (active) store_words16(out + off, zw);
            continue;
        }
        // int8 per 128-wide group (8 adjacent lanes): absmax, scale, exact quotient, round half away
        Z = row_from_words(zw);
        float peak = 0.0f;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            float a0, a1, b0, b1;
            x2_split(Z.P[k], a0, a1);
            x2_split(Z.Q[k], b0, b1);
            peak = absmax3(absmax3(peak, a0, a1), b0, b1);
        }
        peak = warp_max_xor(peak, 8);
        const float qsc = i8_scale_bf16(peak);   // peak of bf16 values
        uint32_t cP[4][2], cQ[4][2];
        if (qsc >= 0x1p-90f) {
            const uint64_t ns = x2_splat(-qsc), rs = x2_splat(__frcp_rn(qsc));
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                x2_codes(x2_quot(Z.P[k], ns, rs), cP[k][0], cP[k][1]);
                x2_codes(x2_quot(Z.Q[k], ns, rs), cQ[k][0], cQ[k][1]);
            }
        } else {
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                float a0, a1, b0, b1;
                x2_split(Z.P[k], a0, a1);
                x2_split(Z.Q[k], b0, b1);
                x2_codes(x2(__fdiv_rn(a0, qsc), __fdiv_rn(a1, qsc)), cP[k][0], cP[k][1]);
                x2_codes(x2(__fdiv_rn(b0, qsc), __fdiv_rn(b1, qsc)), cQ[k][0], cQ[k][1]);
            }
        }
        if (active) {
            // element 2k -> cP[k][0], 2k+1 -> cQ[k][0], 2k+8 -> cP[k][1], 2k+9 -> cQ[k][1]
            uint4 o;
            o.x = pack4_lowbytes(cP[0][0], cQ[0][0], cP[1][0], cQ[1][0]);
            o.y = pack4_lowbytes(cP[2][0], cQ[2][0], cP[3][0], cQ[3][0]);
            o.z = pack4_lowbytes(cP[0][1], cQ[0][1], cP[1][1], cQ[1][1]);
            o.w = pack4_lowbytes(cP[2][1], cQ[2][1], cP[3][1], cQ[3][1]);
            *reinterpret_cast<uint4 *>(q + off) = o;
            if ((t & 7) == 0) s[row * s_rs + (int64_t)(t >> 3) * s_gs] = qsc;
        }
    }
}

template <int WP, int MODE>
static void launch_ln_rows_t(const void *x, const void *y, const void *gate, const void *shift, const void *scale,
                             int64_t rows, int64_t L, int64_t D, float eps, void *out, int8_t *q, float *s,
                             int64_t s_rs, int64_t s_gs, cudaStream_t st) {
    auto kern = k_ln_rows<WP, MODE>;
    static int per_sm = 0;   // resident CTAs per SM for this instantiation (same on every B200)
    if (per_sm == 0) {
        int n = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, WP * 32, 0) != cudaSuccess || n < 1) n = 1;
        per_sm = n;
    }
    int64_t grid = (int64_t)num_sms() * per_sm;
    if (grid > rows) grid = rows;
    kern<<<(unsigned)grid, WP * 32, 0, st>>>((const bf16 *)x, (const bf16 *)y, (const bf16 *)gate, (const bf16 *)shift,
                                             (const bf16 *)scale, rows, L, (int)D, eps, (bf16 *)out, q, s, s_rs, s_gs);
}

template <int WP>
static void launch_ln_wp(int mode, const void *x, const void *y, const void *gate, const void *shift,
                         const void *scale, int64_t B, int64_t L, int64_t D, float eps, void *out, int8_t *q,
                         float *s, int64_t s_rs, int64_t s_gs, cudaStream_t st) {
    const int64_t rows = B * L;
    if (mode == 0) launch_ln_rows_t<WP, 0>(x, y, gate, shift, scale, rows, L, D, eps, out, q, s, s_rs, s_gs, st);
    else if (mode == 1) launch_ln_rows_t<WP, 1>(x, y, gate, shift, scale, rows, L, D, eps, out, q, s, s_rs, s_gs, st);
    else launch_ln_rows_t<WP, 2>(x, y, gate, shift, scale, rows, L, D, eps, out, q, s, s_rs, s_gs, st);
}

cudaError_t launch_ln_row(int mode, const void *x, const void *y, const void *gate, const void *shift,
                          const void *scale, int64_t B, int64_t L, int64_t D, float eps, void *out, int8_t *q,
                          float *s, int64_t s_rs, int64_t s_gs, cudaStream_t st) {
    const int warps = (int)cdiv(D / 16, 32);
    int wp = 1;
    while (wp < warps) wp <<= 1;
    switch (wp) {
    case 1: launch_ln_wp<1>(mode, x, y, gate, shift, scale, B, L, D, eps, out, q, s, s_rs, s_gs, st); break;
    case 2: launch_ln_wp<2>(mode, x, y, gate, shift, scale, B, L, D, eps, out, q, s, s_rs, s_gs, st); break;
    case 4: launch_ln_wp<4>(mode, x, y, gate, shift, scale, B, L, D, eps, out, q, s, s_rs, s_gs, st); break;
    case 8: launch_ln_wp<8>(mode, x, y, gate, shift, scale, B, L, D, eps, out, q, s, s_rs, s_gs, st); break;
    case 16: launch_ln_wp<16>(mode, x, y, gate, shift, scale, B, L, D, eps, out, q, s, s_rs, s_gs, st); break;
    case 32: launch_ln_wp<32>(mode, x, y, gate, shift, scale, B, L, D, eps, out, q, s, s_rs, s_gs, st); break;
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------------------------------
// K6 gated residual: out = bf16(x + rbf16(y * gate[b])), 8 elements per 16-byte access, grid-stride.
__global__ void __launch_bounds__(256) k_gated_residual(const bf16 *__restrict__ x, const bf16 *__restrict__ y,
                                                        const bf16 *__restrict__ gate, int64_t L, int64_t D,
                                                        int64_t nvec, bf16 *__restrict__ out) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nvec; i += stride) {
        const int64_t e = i * 8;
        const int64_t row = div_nonneg(e, D), col = e - row * D;
        const int64_t b = div_nonneg(row, L);
        uint4 xv = ldg_stream(x + e), yv = ldg_stream(y + e);
        uint4 gv = *reinterpret_cast<const uint4 *>(gate + b * D + col);
        const uint32_t *xw = &xv.x, *yw = &yv.x, *gw = &gv.x;
        uint4 o;
        uint32_t *ow = &o.x;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            float lo = __fadd_rn(bf16_lo(xw[j]), rbf16(__fmul_rn(bf16_lo(yw[j]), bf16_lo(gw[j]))));
            float hi = __fadd_rn(bf16_hi(xw[j]), rbf16(__fmul_rn(bf16_hi(yw[j]), bf16_hi(gw[j]))));
            ow[j] = pack_bf16_rn(lo, hi);
        }
        *reinterpret_cast<uint4 *>(out + e) = o;
    }
}

cudaError_t launch_gated_residual(const void *x, const void *y, const void *gate, int64_t B, int64_t L, int64_t D,
                                  void *out, cudaStream_t st) {
    const int64_t nvec = B * L * D / 8;
    int64_t blocks = cdiv(nvec, 256);
    const int64_t cap = (int64_t)num_sms() * 8;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    k_gated_residual<<<(unsigned)blocks, 256, 0, st>>>((const bf16 *)x, (const bf16 *)y, (const bf16 *)gate, L, D,
                                                       nvec, (bf16 *)out);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------------------------------
// K5 QK-RMSNorm + interleaved RoPE (fused.py:65-91), D = 128. One warp per token, four heads at a time:
// lane l handles head h0 + l/8, elements [16*(l%8), 16*(l%8) + 16) = 8 interleaved (even, odd) pairs, held as
// packed (even, odd) f32x2 values. The even and odd square sums (fused.py:74, sum(xe^2) + sum(xo^2)) are
// pairwise trees over the head's 64 evens / odds in index order: three levels inside the lane (8 pairs), then a
// butterfly over the 8 lanes of the head - both trees at once, as the two halves of a pair. The token's cos/sin
// for the lane's 16 positions are loaded once and reused for every head and both tensors.
//
// Q8: the last tensor's output is also quantized for an int8 KV cache (world.py:83-90 applied to it): per
// (token, head) absmax over the head's 128 bf16 outputs (8 lanes), scale absmax/127 (1 for an all-zero head),
// codes rounded half away from zero; q8 [BL, H, 128] int8, s8 [BL * H] fp32.
//
// The warp walks (tensor, group of four heads) as one sequence, two groups per step: the two groups' loads,
// reductions and rsqrt chains are independent, so they overlap inside the warp.
template <bool ROPE, int NT, bool Q8>
__global__ void __launch_bounds__(256) k_qk_norm_rope(const bf16 *__restrict__ x0, const bf16 *__restrict__ x1,
                                                      int64_t row_stride, const bf16 *__restrict__ w0,
                                                      const bf16 *__restrict__ w1, const float *__restrict__ cosp,
                                                      const float *__restrict__ sinp, int64_t BL, int64_t L, int H,
                                                      float eps, bf16 *__restrict__ y0, bf16 *__restrict__ y1,
                                                      int8_t *__restrict__ q8, float *__restrict__ s8) {
    const int lane = threadIdx.x & 31;
    const int sub = lane & 7, hq = lane >> 3;
    const int64_t tok = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (tok >= BL) return;
    const int64_t l = tok - div_nonneg(tok, L) * L;
    // cos/sin of the lane's 16 positions as (even, odd) pairs
    uint64_t C[8], S[8];
    if (ROPE) {
        const float4 *cv = reinterpret_cast<const float4 *>(cosp + l * 128 + 16 * sub);
        const float4 *sv = reinterpret_cast<const float4 *>(sinp + l * 128 + 16 * sub);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float4 c4 = cv[i], s4 = sv[i];
            C[2 * i] = x2(c4.x, c4.y);
            C[2 * i + 1] = x2(c4.z, c4.w);
            S[2 * i] = x2(s4.x, s4.y);
            S[2 * i + 1] = x2(s4.z, s4.w);
        }
    }
    const float inv_d = 0.0078125f;   // 1/128: ss / 128 is the exact product ss * 2^-7
    const int ng = (H + 3) >> 2;          // groups of four heads per tensor
    const int nit = NT * ng;
    // step `it` = tensor it / ng, heads 4 * (it % ng) + 0..3; this lane's head h, off (h >= H) past the last head
    struct Group {
        int ts, h;
        bool on;
        uint32_t xw[8], ww[8];
    };
    auto load_group = [&](int it, Group &g) {
        g.ts = (NT == 2 && it >= ng) ? 1 : 0;
        g.h = 4 * (it - g.ts * ng) + hq;
        g.on = g.h < H;
        if (g.on) {
            const bf16 *p = (g.ts ? x1 : x0) + tok * row_stride + 16 * sub + g.h * 128;
            const uint4 a = ldg_stream(p), b = ldg_stream(p + 8);
            g.xw[0] = a.x; g.xw[1] = a.y; g.xw[2] = a.z; g.xw[3] = a.w;
            g.xw[4] = b.x; g.xw[5] = b.y; g.xw[6] = b.z; g.xw[7] = b.w;
            const bf16 *ws = (g.ts ? w1 : w0) + 16 * sub;
            const uint4 c = *reinterpret_cast<const uint4 *>(ws), d = *reinterpret_cast<const uint4 *>(ws + 8);
            g.ww[0] = c.x; g.ww[1] = c.y; g.ww[2] = c.z; g.ww[3] = c.w;
            g.ww[4] = d.x; g.ww[5] = d.y; g.ww[6] = d.z; g.ww[7] = d.w;
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) { g.xw[i] = 0u; g.ww[i] = 0u; }
        }
    };
    // rbf16(rbf16(x * r) * w), then the rotation; stores y (and the int8 codes of the last tensor for Q8)
    auto process = [&](const Group &g) {
        uint64_t V[8], SQ[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            V[i] = x2(bf16_lo(g.xw[i]), bf16_hi(g.xw[i]));
            SQ[i] = x2_mul(V[i], V[i]);
        }
        // (sum of even squares, sum of odd squares): tree over the lane's 8 pairs, then over the 8 lanes
        float se, so;
        {
            float a[16];
#pragma unroll
            for (int i = 0; i < 8; ++i) x2_split(SQ[i], a[2 * i], a[2 * i + 1]);
            // scalar first level (a product is not fed straight into a packed addition)
            uint64_t t[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) t[i] = x2(__fadd_rn(a[4 * i], a[4 * i + 2]), __fadd_rn(a[4 * i + 1], a[4 * i + 3]));
            const uint64_t u = x2_add(x2_add(t[0], t[1]), x2_add(t[2], t[3]));
            x2_split(u, se, so);
#pragma unroll
            for (int o = 1; o < 8; o <<= 1) {
                se = __fadd_rn(se, __shfl_xor_sync(0xffffffffu, se, o));
                so = __fadd_rn(so, __shfl_xor_sync(0xffffffffu, so, o));
            }
        }
        const float r = rsqrt_cr(__fadd_rn(__fmul_rn(__fadd_rn(se, so), inv_d), eps));
        const uint64_t r2 = x2_splat(r);
        uint32_t ow[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            float a0, a1;
            x2_split(x2_mul(V[i], r2), a0, a1);
            const uint32_t n1 = bf16x2_rn(a0, a1);
            x2_split(x2_mul(x2(bf16_lo(n1), bf16_hi(n1)), x2(bf16_lo(g.ww[i]), bf16_hi(g.ww[i]))), a0, a1);
            const uint32_t n2 = bf16x2_rn(a0, a1);
            if (ROPE) {
                // (ne*c_e - no*s_e, no*c_o + ne*s_o), the differences and sums rounded separately
                const float ne = bf16_lo(n2), no = bf16_hi(n2);
                float pc0, pc1, ps0, ps1;
                x2_split(x2_mul(x2(ne, no), C[i]), pc0, pc1);
                x2_split(x2_mul(x2(no, ne), S[i]), ps0, ps1);
                ow[i] = bf16x2_rn(__fsub_rn(pc0, ps0), __fadd_rn(pc1, ps1));
            } else {
                ow[i] = n2;
            }
        }
        bf16 *yrow = (g.ts == 0 ? y0 : y1) + tok * (int64_t)H * 128 + 16 * sub + g.h * 128;
        if (g.on) {
            reinterpret_cast<uint4 *>(yrow)[0] = make_uint4(ow[0], ow[1], ow[2], ow[3]);
            reinterpret_cast<uint4 *>(yrow)[1] = make_uint4(ow[4], ow[5], ow[6], ow[7]);
        }
        if (Q8 && g.ts == NT - 1) {
            float peak = 0.0f;
#pragma unroll
            for (int i = 0; i < 8; ++i) peak = absmax3(peak, bf16_lo(ow[i]), bf16_hi(ow[i]));
#pragma unroll
            for (int o = 1; o < 8; o <<= 1) peak = fmaxf(peak, __shfl_xor_sync(0xffffffffu, peak, o));
            const float qsc = i8_scale_bf16(peak);   // peak of bf16 values
            uint32_t c[16];
            if (qsc >= 0x1p-90f) {
                const uint64_t ns = x2_splat(-qsc), rs = x2_splat(__frcp_rn(qsc));
#pragma unroll
                for (int i = 0; i < 8; ++i) x2_codes(x2_quot(x2(bf16_lo(ow[i]), bf16_hi(ow[i])), ns, rs), c[2 * i], c[2 * i + 1]);
            } else {
#pragma unroll
                for (int i = 0; i < 8; ++i)
                    x2_codes(x2(__fdiv_rn(bf16_lo(ow[i]), qsc), __fdiv_rn(bf16_hi(ow[i]), qsc)), c[2 * i], c[2 * i + 1]);
            }
            if (g.on) {
                *reinterpret_cast<uint4 *>(q8 + (tok * H + g.h) * 128 + 16 * sub) =
                    make_uint4(pack4_lowbytes(c[0], c[1], c[2], c[3]), pack4_lowbytes(c[4], c[5], c[6], c[7]),
                               pack4_lowbytes(c[8], c[9], c[10], c[11]), pack4_lowbytes(c[12], c[13], c[14], c[15]));
                if (sub == 0) s8[tok * H + g.h] = qsc;
            }
        }
    };
    for (int it = 0; it < nit; it += 2) {
        // the second group of the last step is off when nit is odd (its heads lie past H)
        Group ga, gb;
        load_group(it, ga);
        load_group(it + 1, gb);
        process(ga);
        process(gb);
    }
}

cudaError_t launch_qk_norm_rope(int ntensors, const void *x0, const void *x1, int64_t row_stride, const void *w0,
                                const void *w1, const float *cos, const float *sin, int64_t B, int64_t L, int64_t H,
                                float eps, void *y0, void *y1, int8_t *q8, float *s8, cudaStream_t st) {
    const int64_t BL = B * L;
    dim3 grid((unsigned)cdiv(BL, 8)), block(256);
    const bf16 *a = (const bf16 *)x0, *b = (const bf16 *)x1, *wa = (const bf16 *)w0, *wb = (const bf16 *)w1;
    bf16 *ya = (bf16 *)y0, *yb = (bf16 *)y1;
    const bool rope = cos != nullptr;
#define HN_QK(R, N, Q) k_qk_norm_rope<R, N, Q><<<grid, block, 0, st>>>(a, b, row_stride, wa, wb, cos, sin, BL, L, (int)H, eps, ya, yb, q8, s8)
    if (q8 != nullptr) {
        if (ntensors == 1) { if (rope) HN_QK(true, 1, true); else HN_QK(false, 1, true); }
        else { if (rope) HN_QK(true, 2, true); else HN_QK(false, 2, true); }
    } else if (ntensors == 1) {
        if (rope) HN_QK(true, 1, false);
        else HN_QK(false, 1, false);
    } else {
        if (rope) HN_QK(true, 2, false);
        else HN_QK(false, 2, false);
    }
#undef HN_QK
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------------------------------
// K7 PixelUMM q/k prep (fused.py:131-175, D == 128): a head is [t0 | t1 | h0 | h1 | w0 | w1] of 32, 32, 16, 16,
// 16, 16 elements; t0/t1, h0/h1 and w0/w1 are rotate-half partners. One warp per token, four heads at a time,
// 8 lanes per head: lane s (0..7) holds t0[4s..4s+4), t1[4s..4s+4) and h0/h1/w0/w1[2s..2s+2), so every
// rotation partner is in the same lane. The sums of squares - pairwise trees in index order over t0 and t1
// (32 each) and over h0, h1, w0, w1 (16 each) - are an in-lane first level (or two) and a butterfly over the
// head's 8 lanes; the norms combine them as (sum t0^2 + sum t1^2) and ((h0 + h1) + w0) + w1 (fused.py:155-160).
__device__ __forceinline__ float sum8_lanes(float v) {
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__global__ void __launch_bounds__(256) k_pixelumm_qk(const bf16 *__restrict__ x, int64_t row_stride,
                                                     const bf16 *__restrict__ wt, const bf16 *__restrict__ whw,
                                                     const float *__restrict__ cosp, const float *__restrict__ sinp,
                                                     int64_t N, int H, float eps, bf16 *__restrict__ y) {
    const int lane = threadIdx.x & 31, sub = lane & 7, hq = lane >> 3;
    const int64_t tok = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (tok >= N) return;
    // this lane's positions inside a head: T at [4s, 4s+4) and 32 + [4s, 4s+4); HW quarters at 64/80/96/112 + [2s, 2s+2)
    const int pt0 = 4 * sub, pt1 = 32 + 4 * sub, ph0 = 64 + 2 * sub, ph1 = 80 + 2 * sub, pw0 = 96 + 2 * sub, pw1 = 112 + 2 * sub;
    // weights (wt over the T half [0, 64), whw over the HW half) and the token's cos/sin at the same positions
    float wgt[16], cs[16], sn[16];
    {
        const uint2 a = *reinterpret_cast<const uint2 *>(wt + pt0), b = *reinterpret_cast<const uint2 *>(wt + pt1);
        wgt[0] = bf16_lo(a.x); wgt[1] = bf16_hi(a.x); wgt[2] = bf16_lo(a.y); wgt[3] = bf16_hi(a.y);
        wgt[4] = bf16_lo(b.x); wgt[5] = bf16_hi(b.x); wgt[6] = bf16_lo(b.y); wgt[7] = bf16_hi(b.y);
        const int ph[4] = {ph0, ph1, pw0, pw1};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const uint32_t w2 = *reinterpret_cast<const uint32_t *>(whw + ph[q] - 64);
            wgt[8 + 2 * q] = bf16_lo(w2);
            wgt[9 + 2 * q] = bf16_hi(w2);
        }
        const float *cb = cosp + tok * 128, *sb = sinp + tok * 128;
        const float4 c0 = *reinterpret_cast<const float4 *>(cb + pt0), c1 = *reinterpret_cast<const float4 *>(cb + pt1);
        const float4 s0 = *reinterpret_cast<const float4 *>(sb + pt0), s1 = *reinterpret_cast<const float4 *>(sb + pt1);
        cs[0] = c0.x; cs[1] = c0.y; cs[2] = c0.z; cs[3] = c0.w; cs[4] = c1.x; cs[5] = c1.y; cs[6] = c1.z; cs[7] = c1.w;
        sn[0] = s0.x; sn[1] = s0.y; sn[2] = s0.z; sn[3] = s0.w; sn[4] = s1.x; sn[5] = s1.y; sn[6] = s1.z; sn[7] = s1.w;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float2 c2 = *reinterpret_cast<const float2 *>(cb + ph[q]);
            const float2 s2 = *reinterpret_cast<const float2 *>(sb + ph[q]);
            cs[8 + 2 * q] = c2.x; cs[9 + 2 * q] = c2.y;
            sn[8 + 2 * q] = s2.x; sn[9 + 2 * q] = s2.y;
        }
    }
    // one group of four heads (this lane: head h0 + hq); the loop below runs two groups per step, whose loads,
    // reductions and rsqrt chains are independent and overlap inside the warp
    auto process = [&](int h0) {
        const int h = h0 + hq;
        const bool on = h < H;
        const bf16 *xr = x + tok * row_stride + (int64_t)h * 128;
        float v[16];
        if (on) {
            const uint2 a = *reinterpret_cast<const uint2 *>(xr + pt0), b = *reinterpret_cast<const uint2 *>(xr + pt1);
            v[0] = bf16_lo(a.x); v[1] = bf16_hi(a.x); v[2] = bf16_lo(a.y); v[3] = bf16_hi(a.y);
            v[4] = bf16_lo(b.x); v[5] = bf16_hi(b.x); v[6] = bf16_lo(b.y); v[7] = bf16_hi(b.y);
            const int ph[4] = {ph0, ph1, pw0, pw1};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const uint32_t w2 = *reinterpret_cast<const uint32_t *>(xr + ph[q]);
                v[8 + 2 * q] = bf16_lo(w2);
                v[9 + 2 * q] = bf16_hi(w2);
            }
        } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = 0.0f;
        }
        // squares; the in-lane levels of each pairwise tree, then the 8-lane butterflies
        float sq[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) sq[i] = __fmul_rn(v[i], v[i]);
        const float t0 = sum8_lanes(__fadd_rn(__fadd_rn(sq[0], sq[1]), __fadd_rn(sq[2], sq[3])));
        const float t1 = sum8_lanes(__fadd_rn(__fadd_rn(sq[4], sq[5]), __fadd_rn(sq[6], sq[7])));
        const float a0 = sum8_lanes(__fadd_rn(sq[8], sq[9]));
        const float a1 = sum8_lanes(__fadd_rn(sq[10], sq[11]));
        const float a2 = sum8_lanes(__fadd_rn(sq[12], sq[13]));
        const float a3 = sum8_lanes(__fadd_rn(sq[14], sq[15]));
        const float st = __fadd_rn(t0, t1);
        const float shw = __fadd_rn(__fadd_rn(__fadd_rn(a0, a1), a2), a3);
        // / 64 (half of D) is the exact product * 2^-6
        const float rt = rsqrt_cr(__fadd_rn(__fmul_rn(st, 0.015625f), eps));
        const float rhw = rsqrt_cr(__fadd_rn(__fmul_rn(shw, 0.015625f), eps));
        float n[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) n[i] = __fmul_rn(__fmul_rn(v[i], i < 8 ? rt : rhw), wgt[i]);
        float o[16];
        // T: (t0*c - t1*s, t1*c + t0*s) for positions i (t0) and 32 + i (t1)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            o[i] = __fsub_rn(__fmul_rn(n[i], cs[i]), __fmul_rn(n[4 + i], sn[i]));
            o[4 + i] = __fadd_rn(__fmul_rn(n[4 + i], cs[4 + i]), __fmul_rn(n[i], sn[4 + i]));
        }
        // HW: h0/h1 (slots 8-9 / 10-11) and w0/w1 (slots 12-13 / 14-15)
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            o[8 + i] = __fsub_rn(__fmul_rn(n[8 + i], cs[8 + i]), __fmul_rn(n[10 + i], sn[8 + i]));
            o[10 + i] = __fadd_rn(__fmul_rn(n[10 + i], cs[10 + i]), __fmul_rn(n[8 + i], sn[10 + i]));
            o[12 + i] = __fsub_rn(__fmul_rn(n[12 + i], cs[12 + i]), __fmul_rn(n[14 + i], sn[12 + i]));
            o[14 + i] = __fadd_rn(__fmul_rn(n[14 + i], cs[14 + i]), __fmul_rn(n[12 + i], sn[14 + i]));
        }
        if (on) {
            bf16 *yr = y + (tok * H + h) * 128;
            *reinterpret_cast<uint2 *>(yr + pt0) = make_uint2(bf16x2_rn(o[0], o[1]), bf16x2_rn(o[2], o[3]));
            *reinterpret_cast<uint2 *>(yr + pt1) = make_uint2(bf16x2_rn(o[4], o[5]), bf16x2_rn(o[6], o[7]));
            *reinterpret_cast<uint32_t *>(yr + ph0) = bf16x2_rn(o[8], o[9]);
            *reinterpret_cast<uint32_t *>(yr + ph1) = bf16x2_rn(o[10], o[11]);
            *reinterpret_cast<uint32_t *>(yr + pw0) = bf16x2_rn(o[12], o[13]);
            *reinterpret_cast<uint32_t *>(yr + pw1) = bf16x2_rn(o[14], o[15]);
        }
    };
    for (int h0 = 0; h0 < H; h0 += 8) {
        process(h0);
        process(h0 + 4);   // heads past H are off
    }
}

cudaError_t launch_pixelumm_qk(const void *x, int64_t row_stride, const void *wt, const void *whw, const float *cos,
                               const float *sin, int64_t N, int64_t H, float eps, void *y, cudaStream_t st) {
    dim3 grid((unsigned)cdiv(N, 8)), block(256);
    k_pixelumm_qk<<<grid, block, 0, st>>>((const bf16 *)x, row_stride, (const bf16 *)wt, (const bf16 *)whw, cos, sin, N,
                                          (int)H, eps, (bf16 *)y);
    return cudaGetLastError();
}

} // namespace hn
