// decoder.cu - the PixelUMM decoder's norm and MLP-gate fusions, each ending in the activation quantizer of the
// FP8 (or int8) linears that read its output (the "RMSNorm/SiLU fusions" of the reference's notes, README.md:266):
//
//   k_rms_quant       hy_nomas/pixelumm.py:246-259 (Qwen3 RMSNorm: y = w * bf16(x * rsqrt(mean(x^2) + eps)))
//                     then kernels.py:22-42 per 128 columns - the codes and scales q_proj/k_proj/v_proj or
//                     gate_proj/up_proj take, without writing y
//   k_silu_mul_quant  hy_nomas/pixelumm.py:322-323 (silu(gate) * up, torch's bf16 roundings) then the same
//                     quantizer - the codes and scales down_proj takes, without writing the product
//
// Both are single HBM passes. Quantization is per row and 128 columns, with the exact quotient and the code
// rounding of the activation quantizer (quant_chunk8 in hn_common.cuh: e4m3 nearest even saturating, int8 half away).
#include "hn_common.cuh"
#include "hn_kernels.h"

namespace hn {

namespace dec {

// the quantization scale of a 128-group of bf16 values with absmax `peak` (as quant.cu's group_scale for bf16)
template <int KIND> __device__ __forceinline__ float scale_bf16(float peak) {
    return KIND == 0 ? i8_scale_bf16(peak) : e4m3_scale_bf16(peak);
}

// 8 bf16 values (one 16-byte load) -> fp32
__device__ __forceinline__ void load8_bf16(const __nv_bfloat16 *p, float *v) { Elem<__nv_bfloat16>::load8(p, v); }

// RMSNorm + quantize: one CTA of 256 threads per row, the row in registers as NCH chunks of 8 elements per thread
// (chunk c = i * 256 + t at elements [8c, 8c + 8)). The sum of squares is a balanced pairwise tree in index order:
// in-chunk tree, lane butterfly, the 8 warps' partials, then the NCH chunk rows (padded to a power of two).
// A 128-element quantization group is 16 consecutive chunks, i.e. 16 consecutive threads for one i.
template <int KIND, int NCH>
__global__ void __launch_bounds__(256) k_rms_quant(const __nv_bfloat16 *__restrict__ x, int64_t ldx,
                                                   const __nv_bfloat16 *__restrict__ w, int64_t D, float eps,
                                                   uint8_t *__restrict__ q, int64_t ldq, float *__restrict__ s,
                                                   int64_t s_rs, int64_t s_gs) {
    constexpr int NP = NCH <= 1 ? 1 : (NCH <= 2 ? 2 : (NCH <= 4 ? 4 : 8));   // chunk rows padded to a power of 2
    __shared__ float red[NP][8];
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int64_t m = blockIdx.x;
    const int64_t nch = D >> 3;
    float v[NCH][8];
#pragma unroll
    for (int i = 0; i < NCH; ++i) {
        const int64_t c = t + (int64_t)i * 256;
        if (c < nch) load8_bf16(x + m * ldx + 8 * c, v[i]);
        else {
#pragma unroll
            for (int j = 0; j < 8; ++j) v[i][j] = 0.0f;
        }
    }
    // sum of squares
#pragma unroll
    for (int i = 0; i < NP; ++i) {
        float part = 0.0f;
        if (i < NCH) {
            float a[4];
#pragma unroll
            for (int j = 0; j < 4; ++j)
                a[j] = __fadd_rn(__fmul_rn(v[i][2 * j], v[i][2 * j]), __fmul_rn(v[i][2 * j + 1], v[i][2 * j + 1]));
            part = __fadd_rn(__fadd_rn(a[0], a[1]), __fadd_rn(a[2], a[3]));
        }
        part = warp_sum_tree(part);
        if (lane == 0) red[i][warp] = part;
    }
    __syncthreads();
    float rows_sum[NP];
#pragma unroll
    for (int i = 0; i < NP; ++i) {
        float p8[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) p8[k] = red[i][k];
#pragma unroll
        for (int k = 0; k < 4; ++k) p8[k] = __fadd_rn(p8[2 * k], p8[2 * k + 1]);
        p8[0] = __fadd_rn(p8[0], p8[1]);
        p8[1] = __fadd_rn(p8[2], p8[3]);
        rows_sum[i] = __fadd_rn(p8[0], p8[1]);
    }
#pragma unroll
    for (int n = NP; n > 1; n >>= 1) {
#pragma unroll
        for (int i = 0; i < n / 2; ++i) rows_sum[i] = __fadd_rn(rows_sum[2 * i], rows_sum[2 * i + 1]);
    }
    const float fd = (float)D;
    const float ms = (D & (D - 1)) == 0 ? __fmul_rn(rows_sum[0], __fdiv_rn(1.0f, fd)) : __fdiv_rn(rows_sum[0], fd);
    const float r = rsqrt_cr(__fadd_rn(ms, eps));
    // y = rbf16(w * rbf16(x * r)), then the quantizer per 128 columns
#pragma unroll
    for (int i = 0; i < NCH; ++i) {
        const int64_t c = t + (int64_t)i * 256;
        float wv[8];
        if (c < nch) load8_bf16(w + 8 * c, wv);
        else {
#pragma unroll
            for (int j = 0; j < 8; ++j) wv[j] = 0.0f;
        }
        float y[8];
#pragma unroll
        for (int j = 0; j < 8; j += 2) {
            const uint32_t nb = bf16x2_rn(__fmul_rn(v[i][j], r), __fmul_rn(v[i][j + 1], r));
            const uint32_t yb = bf16x2_rn(__fmul_rn(wv[j], bf16_lo(nb)), __fmul_rn(wv[j + 1], bf16_hi(nb)));
            y[j] = bf16_lo(yb);
            y[j + 1] = bf16_hi(yb);
        }
        float gp = 0.0f;
#pragma unroll
        for (int j = 0; j < 8; j += 2) gp = absmax3(gp, y[j], y[j + 1]);
        gp = warp_max_xor(gp, 16);
        const float sc = scale_bf16<KIND>(gp);
        const bool fast = sc >= 0x1p-90f;
        const uint64_t ns = x2_splat(-sc), rs = x2_splat(__frcp_rn(sc));
        if (c < nch) {
            *reinterpret_cast<uint2 *>(q + m * ldq + 8 * c) = quant_chunk8<KIND, false>(y, sc, fast, ns, rs);
            if ((c & 15) == 0) s[m * s_rs + (c >> 4) * s_gs] = sc;
        }
    }
}

// silu(g) * u + quantize: a warp covers two 128-groups of one row (lane l: elements [8l, 8l + 8) of the warp's
// 256), grid-stride over (row, group pair). silu(g) = g / (1 + exp(-g)) in fp32 (exp_cw, IEEE division),
// rounded to bf16, times u, rounded to bf16.
template <int KIND>
__global__ void __launch_bounds__(256) k_silu_mul_quant(const __nv_bfloat16 *__restrict__ g, int64_t ldg,
                                                        const __nv_bfloat16 *__restrict__ u, int64_t ldu,
                                                        int64_t rows, int64_t I, uint8_t *__restrict__ q, int64_t ldq,
                                                        float *__restrict__ s, int64_t s_rs, int64_t s_gs) {
    const int lane = threadIdx.x & 31;
    const int64_t pairs = (I / 128 + 1) / 2;   // group pairs per row
    const int64_t units = rows * pairs;
    const int64_t warp0 = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int64_t wstride = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t unit = warp0; unit < units; unit += wstride) {
        const int64_t m = div_nonneg(unit, pairs);
        const int64_t col = (unit - m * pairs) * 256 + 8 * lane;
        const bool active = col < I;
        float gv[8], uv[8], h[8];
        if (active) {
            load8_bf16(g + m * ldg + col, gv);
            load8_bf16(u + m * ldu + col, uv);
        } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) { gv[j] = 0.0f; uv[j] = 0.0f; }
        }
#pragma unroll
        for (int j = 0; j < 8; j += 2) {
            const float s0 = __fdiv_rn(gv[j], __fadd_rn(1.0f, exp_cw(-gv[j])));
            const float s1 = __fdiv_rn(gv[j + 1], __fadd_rn(1.0f, exp_cw(-gv[j + 1])));
            const uint32_t sb = bf16x2_rn(s0, s1);
            const uint32_t hb = bf16x2_rn(__fmul_rn(bf16_lo(sb), uv[j]), __fmul_rn(bf16_hi(sb), uv[j + 1]));
            h[j] = bf16_lo(hb);
            h[j + 1] = bf16_hi(hb);
        }
        float gp = 0.0f;
#pragma unroll
        for (int j = 0; j < 8; j += 2) gp = absmax3(gp, h[j], h[j + 1]);
        gp = warp_max_xor(gp, 16);
        const float sc = scale_bf16<KIND>(gp);
        const bool fast = sc >= 0x1p-90f;
        const uint64_t ns = x2_splat(-sc), rs = x2_splat(__frcp_rn(sc));
        if (active) {
            *reinterpret_cast<uint2 *>(q + m * ldq + col) = quant_chunk8<KIND, false>(h, sc, fast, ns, rs);
            if ((lane & 15) == 0) s[m * s_rs + (col >> 7) * s_gs] = sc;
        }
    }
}

template <int KIND>
static cudaError_t launch_rms_k(const void *x, int64_t ldx, const void *w, int64_t rows, int64_t D, float eps,
                                void *q, int64_t ldq, float *s, int64_t s_rs, int64_t s_gs, cudaStream_t st) {
    const auto *xp = static_cast<const __nv_bfloat16 *>(x);
    const auto *wp = static_cast<const __nv_bfloat16 *>(w);
    auto *qp = static_cast<uint8_t *>(q);
    const dim3 grid((unsigned)rows), block(256);
    switch (cdiv(D / 8, 256)) {
    case 1: k_rms_quant<KIND, 1><<<grid, block, 0, st>>>(xp, ldx, wp, D, eps, qp, ldq, s, s_rs, s_gs); break;
    case 2: k_rms_quant<KIND, 2><<<grid, block, 0, st>>>(xp, ldx, wp, D, eps, qp, ldq, s, s_rs, s_gs); break;
    case 3: case 4: k_rms_quant<KIND, 4><<<grid, block, 0, st>>>(xp, ldx, wp, D, eps, qp, ldq, s, s_rs, s_gs); break;
    default: k_rms_quant<KIND, 8><<<grid, block, 0, st>>>(xp, ldx, wp, D, eps, qp, ldq, s, s_rs, s_gs); break;
    }
    return cudaGetLastError();
}

} // namespace dec

cudaError_t launch_rmsnorm_quant(const void *x, int64_t ldx, const void *w, int64_t rows, int64_t D, float eps,
                                 int kind, void *q, int64_t ldq, float *s, int64_t s_rs, int64_t s_gs, cudaStream_t st) {
    return kind == 0 ? dec::launch_rms_k<0>(x, ldx, w, rows, D, eps, q, ldq, s, s_rs, s_gs, st)
                     : dec::launch_rms_k<1>(x, ldx, w, rows, D, eps, q, ldq, s, s_rs, s_gs, st);
}

cudaError_t launch_silu_mul_quant(const void *g, int64_t ldg, const void *u, int64_t ldu, int64_t rows, int64_t I,
                                  int kind, void *q, int64_t ldq, float *s, int64_t s_rs, int64_t s_gs, cudaStream_t st) {
    const int64_t units = rows * ((I / 128 + 1) / 2);
    int64_t grid = cdiv(units, 8);
    const int64_t cap = (int64_t)num_sms() * 8;
    if (grid > cap) grid = cap;
    const auto *gp = static_cast<const __nv_bfloat16 *>(g);
    const auto *up = static_cast<const __nv_bfloat16 *>(u);
    auto *qp = static_cast<uint8_t *>(q);
    if (kind == 0) dec::k_silu_mul_quant<0><<<(unsigned)grid, 256, 0, st>>>(gp, ldg, up, ldu, rows, I, qp, ldq, s, s_rs, s_gs);
    else dec::k_silu_mul_quant<1><<<(unsigned)grid, 256, 0, st>>>(gp, ldg, up, ldu, rows, I, qp, ldq, s, s_rs, s_gs);
    return cudaGetLastError();
}

} // namespace hn
