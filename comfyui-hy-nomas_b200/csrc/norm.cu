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

__device__ __forceinline__ void load16_bf16(const bf16 *p, float *v) {
    Elem<bf16>::load8(p, v);
    Elem<bf16>::load8(p + 8, v + 8);
}
__device__ __forceinline__ void store16_bf16_exact(bf16 *p, const float *v) {
    uint4 a, b;
    a.x = pack_bf16_exact(v[0], v[1]); a.y = pack_bf16_exact(v[2], v[3]);
    a.z = pack_bf16_exact(v[4], v[5]); a.w = pack_bf16_exact(v[6], v[7]);
    b.x = pack_bf16_exact(v[8], v[9]); b.y = pack_bf16_exact(v[10], v[11]);
    b.z = pack_bf16_exact(v[12], v[13]); b.w = pack_bf16_exact(v[14], v[15]);
    reinterpret_cast<uint4 *>(p)[0] = a;
    reinterpret_cast<uint4 *>(p)[1] = b;
}

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

// MODE 0: y = bf16(modulate(LN(x)))      (K4)
// MODE 1: codes/scales of rbf16(modulate(LN(x)))   (K3)
// MODE 2: x' = bf16(x + rbf16(y * gate)); store x'; then MODE 1 on x'   (K6+K3)
template <int WP, int MODE>
__global__ void __launch_bounds__(WP * 32) k_ln_row(const bf16 *__restrict__ x, const bf16 *__restrict__ yres,
                                                   const bf16 *__restrict__ gate, const bf16 *__restrict__ shift,
                                                   const bf16 *__restrict__ scale, int64_t L, int D, float eps,
                                                   bf16 *__restrict__ out, int8_t *__restrict__ q,
                                                   float *__restrict__ s, int64_t s_rs, int64_t s_gs) {
    __shared__ float red1[WP], red2[WP];
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int64_t row = blockIdx.x;
    const int64_t b = row / L;
    const int chunks = D >> 4;
    const bool active = t < chunks;
    const int64_t off = row * (int64_t)D + 16 * t;
    const int64_t voff = b * (int64_t)D + 16 * t;
    float v[16];
    if (active) {
        load16_bf16(x + off, v);
        if (MODE == 2) {
            float yv[16], gv[16];
            load16_bf16(yres + off, yv);
            load16_bf16(gate + voff, gv);
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = rbf16(__fadd_rn(v[i], rbf16(__fmul_rn(yv[i], gv[i]))));
            store16_bf16_exact(out + off, v);
        }
    } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = 0.0f;
    }
    if (t < WP) { red1[t] = 0.0f; red2[t] = 0.0f; }
    __syncthreads();
    float part = warp_sum_tree(tree16(v));
    if (lane == 0) red1[warp] = part;
    __syncthreads();
    const float mean = __fdiv_rn(tree_smem<WP>(red1), (float)D);
    float sq[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        v[i] = __fsub_rn(v[i], mean);
        sq[i] = active ? __fmul_rn(v[i], v[i]) : 0.0f;
    }
    part = warp_sum_tree(tree16(sq));
    if (lane == 0) red2[warp] = part;
    __syncthreads();
    const float var = __fdiv_rn(tree_smem<WP>(red2), (float)D);
    const float rstd = rsqrt_cr(__fadd_rn(var, eps));
    float sh[16], sc[16];
    if (active) {
        load16_bf16(shift + voff, sh);
        load16_bf16(scale + voff, sc);
    } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) { sh[i] = 0.0f; sc[i] = 0.0f; }
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        float n = __fmul_rn(v[i], rstd);
        float r = rbf16(__fadd_rn(1.0f, sc[i]));
        v[i] = rbf16(__fadd_rn(__fmul_rn(n, r), sh[i]));
    }
    if (MODE == 0) {
        if (active) store16_bf16_exact(out + off, v);
        return;
    }
    float peak = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; ++i) peak = fmaxf(peak, fabsf(v[i]));
    peak = warp_max_xor(peak, 8);
    const float qsc = i8_scale(peak);
    int c[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) c[i] = code_i8(__fdiv_rn(v[i], qsc));
    if (active) {
        uint4 o;
        o.x = pack4_i8(c[0], c[1], c[2], c[3]);
        o.y = pack4_i8(c[4], c[5], c[6], c[7]);
        o.z = pack4_i8(c[8], c[9], c[10], c[11]);
        o.w = pack4_i8(c[12], c[13], c[14], c[15]);
        *reinterpret_cast<uint4 *>(q + off) = o;
        if ((t & 7) == 0) s[row * s_rs + (int64_t)(t >> 3) * s_gs] = qsc;
    }
}

template <int WP>
static void launch_ln_wp(int mode, const void *x, const void *y, const void *gate, const void *shift,
                         const void *scale, int64_t B, int64_t L, int64_t D, float eps, void *out, int8_t *q,
                         float *s, int64_t s_rs, int64_t s_gs, cudaStream_t st) {
    const int warps = (int)cdiv(D / 16, 32);
    dim3 grid((unsigned)(B * L)), block(warps * 32);
    const bf16 *xp = (const bf16 *)x, *yp = (const bf16 *)y, *gp = (const bf16 *)gate;
    const bf16 *shp = (const bf16 *)shift, *scp = (const bf16 *)scale;
    if (mode == 0) k_ln_row<WP, 0><<<grid, block, 0, st>>>(xp, yp, gp, shp, scp, L, (int)D, eps, (bf16 *)out, q, s, s_rs, s_gs);
    else if (mode == 1) k_ln_row<WP, 1><<<grid, block, 0, st>>>(xp, yp, gp, shp, scp, L, (int)D, eps, (bf16 *)out, q, s, s_rs, s_gs);
    else k_ln_row<WP, 2><<<grid, block, 0, st>>>(xp, yp, gp, shp, scp, L, (int)D, eps, (bf16 *)out, q, s, s_rs, s_gs);
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
        const int64_t row = e / D, col = e - row * D;
        const int64_t b = row / L;
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
// K5 QK-RMSNorm + interleaved RoPE. One warp per token, looping over heads; lane l owns elements
// [4l, 4l+4) of a 128-wide head = the interleaved pairs (4l, 4l+1) and (4l+2, 4l+3). The even and odd
// square sums are separate butterfly trees (fused.py:74: sum(xe^2) + sum(xo^2)). The token's cos/sin
// (16 bytes each per lane) are loaded once and reused for every head and both tensors.
template <bool ROPE, int NT>
__global__ void __launch_bounds__(256) k_qk_norm_rope(const bf16 *__restrict__ x0, const bf16 *__restrict__ x1,
                                                      int64_t row_stride, const bf16 *__restrict__ w0,
                                                      const bf16 *__restrict__ w1, const float *__restrict__ cosp,
                                                      const float *__restrict__ sinp, int64_t BL, int64_t L, int H,
                                                      float eps, bf16 *__restrict__ y0, bf16 *__restrict__ y1) {
    const int lane = threadIdx.x & 31;
    const int64_t tok = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (tok >= BL) return;
    const int64_t l = tok % L;
    float c[4] = {0, 0, 0, 0}, sn[4] = {0, 0, 0, 0};
    if (ROPE) {
        float4 cv = *reinterpret_cast<const float4 *>(cosp + l * 128 + 4 * lane);
        float4 sv = *reinterpret_cast<const float4 *>(sinp + l * 128 + 4 * lane);
        c[0] = cv.x; c[1] = cv.y; c[2] = cv.z; c[3] = cv.w;
        sn[0] = sv.x; sn[1] = sv.y; sn[2] = sv.z; sn[3] = sv.w;
    }
#pragma unroll
    for (int tsel = 0; tsel < NT; ++tsel) {
        const bf16 *xs = tsel == 0 ? x0 : x1;
        const bf16 *ws = tsel == 0 ? w0 : w1;
        bf16 *ys = tsel == 0 ? y0 : y1;
        uint2 wv = *reinterpret_cast<const uint2 *>(ws + 4 * lane);
        const float we0 = bf16_lo(wv.x), wo0 = bf16_hi(wv.x), we1 = bf16_lo(wv.y), wo1 = bf16_hi(wv.y);
        const bf16 *xrow = xs + tok * row_stride + 4 * lane;
        bf16 *yrow = ys + tok * (int64_t)H * 128 + 4 * lane;
        for (int h0 = 0; h0 < H; h0 += 4) {
            uint2 xv[4];
#pragma unroll
            for (int u = 0; u < 4; ++u)
                if (h0 + u < H) xv[u] = *reinterpret_cast<const uint2 *>(xrow + (h0 + u) * 128);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                if (h0 + u >= H) break;
                const float e0 = bf16_lo(xv[u].x), o0 = bf16_hi(xv[u].x), e1 = bf16_lo(xv[u].y), o1 = bf16_hi(xv[u].y);
                float se = __fadd_rn(__fmul_rn(e0, e0), __fmul_rn(e1, e1));
                float so = __fadd_rn(__fmul_rn(o0, o0), __fmul_rn(o1, o1));
                se = warp_sum_tree(se);
                so = warp_sum_tree(so);
                const float r = rsqrt_cr(__fadd_rn(__fdiv_rn(__fadd_rn(se, so), 128.0f), eps));
                const float ne0 = rbf16(__fmul_rn(rbf16(__fmul_rn(e0, r)), we0));
                const float no0 = rbf16(__fmul_rn(rbf16(__fmul_rn(o0, r)), wo0));
                const float ne1 = rbf16(__fmul_rn(rbf16(__fmul_rn(e1, r)), we1));
                const float no1 = rbf16(__fmul_rn(rbf16(__fmul_rn(o1, r)), wo1));
                uint2 ov;
                if (ROPE) {
                    const float oe0 = __fsub_rn(__fmul_rn(ne0, c[0]), __fmul_rn(no0, sn[0]));
                    const float oo0 = __fadd_rn(__fmul_rn(no0, c[1]), __fmul_rn(ne0, sn[1]));
                    const float oe1 = __fsub_rn(__fmul_rn(ne1, c[2]), __fmul_rn(no1, sn[2]));
                    const float oo1 = __fadd_rn(__fmul_rn(no1, c[3]), __fmul_rn(ne1, sn[3]));
                    ov.x = pack_bf16_rn(oe0, oo0);
                    ov.y = pack_bf16_rn(oe1, oo1);
                } else {
                    ov.x = pack_bf16_exact(ne0, no0);
                    ov.y = pack_bf16_exact(ne1, no1);
                }
                *reinterpret_cast<uint2 *>(yrow + (h0 + u) * 128) = ov;
            }
        }
    }
}

cudaError_t launch_qk_norm_rope(int ntensors, const void *x0, const void *x1, int64_t row_stride, const void *w0,
                                const void *w1, const float *cos, const float *sin, int64_t B, int64_t L, int64_t H,
                                float eps, void *y0, void *y1, cudaStream_t st) {
    const int64_t BL = B * L;
    dim3 grid((unsigned)cdiv(BL, 8)), block(256);
    const bf16 *a = (const bf16 *)x0, *b = (const bf16 *)x1, *wa = (const bf16 *)w0, *wb = (const bf16 *)w1;
    bf16 *ya = (bf16 *)y0, *yb = (bf16 *)y1;
    const bool rope = cos != nullptr;
    if (ntensors == 1) {
        if (rope) k_qk_norm_rope<true, 1><<<grid, block, 0, st>>>(a, b, row_stride, wa, wb, cos, sin, BL, L, (int)H, eps, ya, yb);
        else k_qk_norm_rope<false, 1><<<grid, block, 0, st>>>(a, b, row_stride, wa, wb, cos, sin, BL, L, (int)H, eps, ya, yb);
    } else {
        if (rope) k_qk_norm_rope<true, 2><<<grid, block, 0, st>>>(a, b, row_stride, wa, wb, cos, sin, BL, L, (int)H, eps, ya, yb);
        else k_qk_norm_rope<false, 2><<<grid, block, 0, st>>>(a, b, row_stride, wa, wb, cos, sin, BL, L, (int)H, eps, ya, yb);
    }
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------------------------------
// K7 PixelUMM q/k prep (D == 128). Lane l owns elements [4l, 4l+4): lanes 0-15 the T half (t0 = lanes
// 0-7, t1 = lanes 8-15), lanes 16-31 the HW half (h0, h1, w0, w1 in 4-lane quarters). Rotate-half
// partners are lane ^ 8 (T) and lane ^ 4 (HW).
__global__ void __launch_bounds__(256) k_pixelumm_qk(const bf16 *__restrict__ x, int64_t row_stride,
                                                     const bf16 *__restrict__ wt, const bf16 *__restrict__ whw,
                                                     const float *__restrict__ cosp, const float *__restrict__ sinp,
                                                     int64_t N, int H, float eps, bf16 *__restrict__ y) {
    const int lane = threadIdx.x & 31;
    const int64_t tok = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (tok >= N) return;
    const bool tpart = lane < 16;
    const bool first = tpart ? (lane < 8) : ((lane & 4) == 0);
    const int partner = tpart ? (lane ^ 8) : (lane ^ 4);
    uint2 wv = *reinterpret_cast<const uint2 *>(tpart ? (wt + 4 * lane) : (whw + 4 * lane - 64));
    const float w[4] = {bf16_lo(wv.x), bf16_hi(wv.x), bf16_lo(wv.y), bf16_hi(wv.y)};
    float4 cv = *reinterpret_cast<const float4 *>(cosp + tok * 128 + 4 * lane);
    float4 sv = *reinterpret_cast<const float4 *>(sinp + tok * 128 + 4 * lane);
    const float c[4] = {cv.x, cv.y, cv.z, cv.w}, sn[4] = {sv.x, sv.y, sv.z, sv.w};
    for (int h = 0; h < H; ++h) {
        uint2 xv = *reinterpret_cast<const uint2 *>(x + tok * row_stride + (int64_t)h * 128 + 4 * lane);
        const float v[4] = {bf16_lo(xv.x), bf16_hi(xv.x), bf16_lo(xv.y), bf16_hi(xv.y)};
        float s4 = __fadd_rn(__fadd_rn(__fmul_rn(v[0], v[0]), __fmul_rn(v[1], v[1])),
                             __fadd_rn(__fmul_rn(v[2], v[2]), __fmul_rn(v[3], v[3])));
        s4 = __fadd_rn(s4, __shfl_xor_sync(0xffffffffu, s4, 1));
        s4 = __fadd_rn(s4, __shfl_xor_sync(0xffffffffu, s4, 2));   // 16-element sums
        float s8 = __fadd_rn(s4, __shfl_xor_sync(0xffffffffu, s4, 4));   // 32-element sums (T lanes)
        float st = __fadd_rn(s8, __shfl_xor_sync(0xffffffffu, s8, 8));   // sum(t0^2) + sum(t1^2)
        const float sh0 = __shfl_sync(0xffffffffu, s4, 16), sh1 = __shfl_sync(0xffffffffu, s4, 20);
        const float sw0 = __shfl_sync(0xffffffffu, s4, 24), sw1 = __shfl_sync(0xffffffffu, s4, 28);
        const float shw = __fadd_rn(__fadd_rn(__fadd_rn(sh0, sh1), sw0), sw1);
        const float sum = __shfl_sync(0xffffffffu, st, 0);
        const float r = rsqrt_cr(__fadd_rn(__fdiv_rn(tpart ? sum : shw, 64.0f), eps));
        float a[4], p[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) a[i] = __fmul_rn(__fmul_rn(v[i], r), w[i]);
#pragma unroll
        for (int i = 0; i < 4; ++i) p[i] = __shfl_sync(0xffffffffu, a[i], partner);
        float o[4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
            o[i] = first ? __fsub_rn(__fmul_rn(a[i], c[i]), __fmul_rn(p[i], sn[i]))
                         : __fadd_rn(__fmul_rn(a[i], c[i]), __fmul_rn(p[i], sn[i]));
        uint2 ov;
        ov.x = pack_bf16_rn(o[0], o[1]);
        ov.y = pack_bf16_rn(o[2], o[3]);
        *reinterpret_cast<uint2 *>(y + (tok * H + h) * 128 + 4 * lane) = ov;
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
