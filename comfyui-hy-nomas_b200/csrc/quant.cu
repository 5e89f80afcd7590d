// quant.cu - K1 activation quantizer (hy_nomas/kernels.py:22-54) and the int8 KV quantizer
// (hy_nomas/world.py:83-90).
//
// Layout: one 128-element group (row m, group g) per 8 consecutive lanes, 16 contiguous elements per lane
// (two 16-byte loads of bf16), 4 groups per warp. The group absmax is a 3-step xor-shuffle max; each lane
// writes its 16 codes as one 16-byte store; the first lane of the group writes the fp32 scale.
// HBM-bound: per element 2 bytes read (bf16) + 1 byte written, plus 4 bytes of scale per 128 elements.
#include <type_traits>

#include "hn_common.cuh"
#include "hn_kernels.h"

namespace hn {

// the quantization scale of a group with absmax `peak`: for bf16 input the peak is a bf16 value and the scale
// comes from the fma-corrected quotient (identical to the IEEE division on that domain), else IEEE division
template <typename TIn, int KIND> __device__ __forceinline__ float group_scale(float peak) {
    constexpr bool BF16_IN = sizeof(TIn) == 2 && !std::is_same<TIn, __half>::value;
    if (BF16_IN) return KIND == 0 ? i8_scale_bf16(peak) : e4m3_scale_bf16(peak);
    return KIND == 0 ? i8_scale(peak) : e4m3_scale(peak);
}

// RNE (int8 only): codes rounded half to even instead of half away from zero.
template <typename TIn, int KIND, bool RNE>
__global__ void __launch_bounds__(256) k_quant_group(const TIn *__restrict__ x, int64_t ldx, int64_t M, int64_t G,
                                                     uint8_t *__restrict__ q, int64_t ldq, float *__restrict__ s,
                                                     int64_t s_rs, int64_t s_gs) {
    const int lane = threadIdx.x & 31, sub = lane & 7;
    const int64_t ngroups = M * G;
    const int64_t warp0 = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int64_t wstride = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t base = warp0 * 4; base < ngroups; base += wstride * 4) {
        const int64_t gi = base + (lane >> 3);
        const bool active = gi < ngroups;
        int64_t m = 0, g = 0;
        float v[16];
        if (active) {
            m = G == 1 ? gi : div_nonneg(gi, G);
            g = gi - m * G;
            const TIn *p = x + m * ldx + g * 128 + sub * 16;
            Elem<TIn>::load8(p, v);
            Elem<TIn>::load8(p + 8, v + 8);
        } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = 0.0f;
        }
        float peak = 0.0f;
#pragma unroll
        for (int i = 0; i < 16; i += 2) peak = absmax3(peak, v[i], v[i + 1]);
        peak = warp_max_xor(peak, 8);
        float sc;
        uint4 out;
        constexpr bool BF16_IN = sizeof(TIn) == 2 && !std::is_same<TIn, __half>::value;
        const float sc_try = group_scale<TIn, KIND>(peak);
        if (BF16_IN && sc_try >= 0x1p-90f) {
            // bf16 input: the exact fma-corrected quotient (x2_quot), checked exhaustively over bf16 inputs
            sc = sc_try;
            const uint64_t ns = x2_splat(-sc), rs = x2_splat(__frcp_rn(sc));
            if (KIND == 0 && RNE) {
                int c[16];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    float q0, q1;
                    x2_split(x2_quot(x2(v[2 * i], v[2 * i + 1]), ns, rs), q0, q1);
                    c[2 * i] = code_i8_rne(q0);
                    c[2 * i + 1] = code_i8_rne(q1);
                }
                out.x = pack4_i8(c[0], c[1], c[2], c[3]);
                out.y = pack4_i8(c[4], c[5], c[6], c[7]);
                out.z = pack4_i8(c[8], c[9], c[10], c[11]);
                out.w = pack4_i8(c[12], c[13], c[14], c[15]);
            } else if (KIND == 0) {
                uint32_t c[16];
#pragma unroll
                for (int i = 0; i < 8; ++i) x2_codes(x2_quot(x2(v[2 * i], v[2 * i + 1]), ns, rs), c[2 * i], c[2 * i + 1]);
                out.x = pack4_lowbytes(c[0], c[1], c[2], c[3]);
                out.y = pack4_lowbytes(c[4], c[5], c[6], c[7]);
                out.z = pack4_lowbytes(c[8], c[9], c[10], c[11]);
                out.w = pack4_lowbytes(c[12], c[13], c[14], c[15]);
            } else {
                uint32_t h[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    float q0, q1;
                    x2_split(x2_quot(x2(v[2 * i], v[2 * i + 1]), ns, rs), q0, q1);
                    // a zero quotient keeps the sign of its input, as the IEEE quotient does
                    h[i] = pack2_e4m3(copysignf(q0, v[2 * i]), copysignf(q1, v[2 * i + 1]));
                }
                out.x = h[0] | (h[1] << 16);
                out.y = h[2] | (h[3] << 16);
                out.z = h[4] | (h[5] << 16);
                out.w = h[6] | (h[7] << 16);
            }
        } else if (KIND == 0) {
            sc = i8_scale(peak);
            int c[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) c[i] = RNE ? code_i8_rne(__fdiv_rn(v[i], sc)) : code_i8(__fdiv_rn(v[i], sc));
            out.x = pack4_i8(c[0], c[1], c[2], c[3]);
            out.y = pack4_i8(c[4], c[5], c[6], c[7]);
            out.z = pack4_i8(c[8], c[9], c[10], c[11]);
            out.w = pack4_i8(c[12], c[13], c[14], c[15]);
        } else {
            sc = e4m3_scale(peak);
            uint32_t h[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) h[i] = pack2_e4m3(__fdiv_rn(v[2 * i], sc), __fdiv_rn(v[2 * i + 1], sc));
            out.x = h[0] | (h[1] << 16);
            out.y = h[2] | (h[3] << 16);
            out.z = h[4] | (h[5] << 16);
            out.w = h[6] | (h[7] << 16);
        }
        if (active) {
            *reinterpret_cast<uint4 *>(q + m * ldq + g * 128 + sub * 16) = out;
            if (sub == 0) s[m * s_rs + g * s_gs] = sc;
        }
    }
}

// Per-row variant: one CTA of 256 threads per row. NCH > 0: the row stays in registers, NCH chunks of 8
// elements per thread (chunk c at elements [8c, 8c + 8), thread t holding chunks t, t + 256, ...: one HBM
// pass, coalesced 16-byte loads); NCH == 0 (rows longer than 16384): two passes, the second from L2.
// GRP: one scale per 128-element group instead of per row - a group is 16 consecutive chunks, i.e. 16
// consecutive threads for one i, so its absmax is a 16-lane shuffle (registers only, NCH > 0).
template <typename TIn, int KIND, bool RNE, int NCH, bool GRP = false>
__global__ void __launch_bounds__(256) k_quant_row(const TIn *__restrict__ x, int64_t ldx, int64_t K,
                                                   uint8_t *__restrict__ q, int64_t ldq, float *__restrict__ s,
                                                   int64_t s_rs, int64_t s_gs = 0) {
    __shared__ float red[8];
    const int64_t m = blockIdx.x;
    const TIn *row = x + m * ldx;
    const int64_t nch = K >> 3;
    float v[NCH > 0 ? NCH : 1][8];
    float peak = 0.0f;
    if (GRP) {
        static_assert(!GRP || NCH > 0, "grouped scales keep the row in registers");
        constexpr bool BF16_IN = sizeof(TIn) == 2 && !std::is_same<TIn, __half>::value;
#pragma unroll
        for (int i = 0; i < (NCH > 0 ? NCH : 1); ++i) {
            const int64_t c = threadIdx.x + (int64_t)i * 256;
            if (c < nch) Elem<TIn>::load8(row + 8 * c, v[i]);
            else {
#pragma unroll
                for (int j = 0; j < 8; ++j) v[i][j] = 0.0f;
            }
        }
#pragma unroll
        for (int i = 0; i < (NCH > 0 ? NCH : 1); ++i) {
            const int64_t c = threadIdx.x + (int64_t)i * 256;
            float gp = 0.0f;
#pragma unroll
            for (int j = 0; j < 8; j += 2) gp = absmax3(gp, v[i][j], v[i][j + 1]);
            gp = warp_max_xor(gp, 16);
            const float sc = group_scale<TIn, KIND>(gp);
            const bool fast = BF16_IN && sc >= 0x1p-90f;
            const uint64_t ns = x2_splat(-sc), rs = x2_splat(__frcp_rn(sc));
            if (c < nch) {
                *reinterpret_cast<uint2 *>(q + m * ldq + 8 * c) = quant_chunk8<KIND, RNE>(v[i], sc, fast, ns, rs);
                if ((c & 15) == 0) s[m * s_rs + (c >> 4) * s_gs] = sc;
            }
        }
        return;
    }
    if (NCH > 0) {
#pragma unroll
        for (int i = 0; i < (NCH > 0 ? NCH : 1); ++i) {
            const int64_t c = threadIdx.x + (int64_t)i * 256;
            if (c < nch) Elem<TIn>::load8(row + 8 * c, v[i]);
            else {
#pragma unroll
                for (int j = 0; j < 8; ++j) v[i][j] = 0.0f;
            }
#pragma unroll
            for (int j = 0; j < 8; j += 2) peak = absmax3(peak, v[i][j], v[i][j + 1]);
        }
    } else {
        for (int64_t c = threadIdx.x; c < nch; c += 256) {
            float w[8];
            Elem<TIn>::load8(row + 8 * c, w);
#pragma unroll
            for (int j = 0; j < 8; j += 2) peak = absmax3(peak, w[j], w[j + 1]);
        }
    }
    peak = warp_max_xor(peak, 32);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = peak;
    __syncthreads();
    peak = 0.0f;
#pragma unroll
    for (int w = 0; w < 8; ++w) peak = fmaxf(peak, red[w]);
    const float sc = group_scale<TIn, KIND>(peak);
    constexpr bool BF16_IN = sizeof(TIn) == 2 && !std::is_same<TIn, __half>::value;
    const bool fast = BF16_IN && sc >= 0x1p-90f;
    const uint64_t ns = x2_splat(-sc), rs = x2_splat(__frcp_rn(sc));
    if (NCH > 0) {
#pragma unroll
        for (int i = 0; i < (NCH > 0 ? NCH : 1); ++i) {
            const int64_t c = threadIdx.x + (int64_t)i * 256;
            if (c < nch) *reinterpret_cast<uint2 *>(q + m * ldq + 8 * c) = quant_chunk8<KIND, RNE>(v[i], sc, fast, ns, rs);
        }
    } else {
        for (int64_t c = threadIdx.x; c < nch; c += 256) {
            float w[8];
            Elem<TIn>::load8(row + 8 * c, w);
            *reinterpret_cast<uint2 *>(q + m * ldq + 8 * c) = quant_chunk8<KIND, RNE>(w, sc, fast, ns, rs);
        }
    }
    if (threadIdx.x == 0) s[m * s_rs] = sc;
}

// grouped scales, rows of up to 16384 elements (NCH <= 8); false when the row is longer
template <typename TIn, int KIND, bool RNE>
static bool launch_quant_group_rows(const TIn *x, int64_t ldx, int64_t M, int64_t K, uint8_t *q, int64_t ldq,
                                    float *s, int64_t s_rs, int64_t s_gs, cudaStream_t st) {
    dim3 grid((unsigned)M), block(256);
    switch (cdiv(K / 8, 256)) {
    case 1: k_quant_row<TIn, KIND, RNE, 1, true><<<grid, block, 0, st>>>(x, ldx, K, q, ldq, s, s_rs, s_gs); return true;
    case 2: k_quant_row<TIn, KIND, RNE, 2, true><<<grid, block, 0, st>>>(x, ldx, K, q, ldq, s, s_rs, s_gs); return true;
    case 3: case 4: k_quant_row<TIn, KIND, RNE, 4, true><<<grid, block, 0, st>>>(x, ldx, K, q, ldq, s, s_rs, s_gs); return true;
    case 5: case 6: case 7: case 8:
        k_quant_row<TIn, KIND, RNE, 8, true><<<grid, block, 0, st>>>(x, ldx, K, q, ldq, s, s_rs, s_gs); return true;
    default: return false;
    }
}

template <typename TIn, int KIND, bool RNE>
static void launch_quant_row(const TIn *x, int64_t ldx, int64_t M, int64_t K, uint8_t *q, int64_t ldq, float *s,
                             int64_t s_rs, cudaStream_t st) {
    dim3 grid((unsigned)M), block(256);
    switch (cdiv(K / 8, 256)) {
    case 1: k_quant_row<TIn, KIND, RNE, 1><<<grid, block, 0, st>>>(x, ldx, K, q, ldq, s, s_rs); break;
    case 2: k_quant_row<TIn, KIND, RNE, 2><<<grid, block, 0, st>>>(x, ldx, K, q, ldq, s, s_rs); break;
    case 3: k_quant_row<TIn, KIND, RNE, 3><<<grid, block, 0, st>>>(x, ldx, K, q, ldq, s, s_rs); break;
    case 4: k_quant_row<TIn, KIND, RNE, 4><<<grid, block, 0, st>>>(x, ldx, K, q, ldq, s, s_rs); break;
    case 5: case 6: k_quant_row<TIn, KIND, RNE, 6><<<grid, block, 0, st>>>(x, ldx, K, q, ldq, s, s_rs); break;
    case 7: case 8: k_quant_row<TIn, KIND, RNE, 8><<<grid, block, 0, st>>>(x, ldx, K, q, ldq, s, s_rs); break;
    default: k_quant_row<TIn, KIND, RNE, 0><<<grid, block, 0, st>>>(x, ldx, K, q, ldq, s, s_rs); break;
    }
}

// flags: bit 0 one scale per row, bit 1 int8 codes rounded half to even
template <typename TIn>
static cudaError_t launch_quant_t(const void *x, int64_t ldx, int64_t M, int64_t K, int kind, int flags, void *q,
                                  int64_t ldq, float *s, int64_t s_rs, int64_t s_gs, cudaStream_t st) {
    const TIn *xp = static_cast<const TIn *>(x);
    uint8_t *qp = static_cast<uint8_t *>(q);
    const bool rne = kind == 0 && (flags & 2);
    if (flags & 1) {
        if (rne) launch_quant_row<TIn, 0, true>(xp, ldx, M, K, qp, ldq, s, s_rs, st);
        else if (kind == 0) launch_quant_row<TIn, 0, false>(xp, ldx, M, K, qp, ldq, s, s_rs, st);
        else launch_quant_row<TIn, 1, false>(xp, ldx, M, K, qp, ldq, s, s_rs, st);
    } else if (M >= 2 * num_sms() && K >= 2048 &&
               (rne ? launch_quant_group_rows<TIn, 0, true>(xp, ldx, M, K, qp, ldq, s, s_rs, s_gs, st)
                    : kind == 0 ? launch_quant_group_rows<TIn, 0, false>(xp, ldx, M, K, qp, ldq, s, s_rs, s_gs, st)
                                : launch_quant_group_rows<TIn, 1, false>(xp, ldx, M, K, qp, ldq, s, s_rs, s_gs, st))) {
        // one CTA per row (enough rows to fill the GPU, and a row that occupies every thread)
    } else {
        const int64_t G = K / 128;
        const int64_t warps = cdiv(M * G, 4);
        int64_t blocks = cdiv(warps, 8);
        const int64_t cap = (int64_t)num_sms() * 16;
        if (blocks > cap) blocks = cap;
        if (rne) k_quant_group<TIn, 0, true><<<(unsigned)blocks, 256, 0, st>>>(xp, ldx, M, G, qp, ldq, s, s_rs, s_gs);
        else if (kind == 0) k_quant_group<TIn, 0, false><<<(unsigned)blocks, 256, 0, st>>>(xp, ldx, M, G, qp, ldq, s, s_rs, s_gs);
        else k_quant_group<TIn, 1, false><<<(unsigned)blocks, 256, 0, st>>>(xp, ldx, M, G, qp, ldq, s, s_rs, s_gs);
    }
    return cudaGetLastError();
}

cudaError_t launch_quant_act(const void *x, int64_t ldx, int x_dtype, int64_t M, int64_t K, int kind, int flags,
                             void *q, int64_t ldq, float *s, int64_t s_rs, int64_t s_gs, cudaStream_t st) {
    switch (x_dtype) {
    case 0: return launch_quant_t<__nv_bfloat16>(x, ldx, M, K, kind, flags, q, ldq, s, s_rs, s_gs, st);
    case 1: return launch_quant_t<__half>(x, ldx, M, K, kind, flags, q, ldq, s, s_rs, s_gs, st);
    default: return launch_quant_t<float>(x, ldx, M, K, kind, flags, q, ldq, s, s_rs, s_gs, st);
    }
}

// ---------------------------------------------------------------------------------------------------
// FP8 weight quantization per 128x128 block (hy_nomas/pixelumm.py:77-82): s = max(absmax, 1e-4) / 448 and
// codes e4m3(w / s). One CTA per block, 8 warps x 16 rows; lane l holds columns [4l, 4l+4) of its rows, so
// the block stays in registers between the absmax and the conversion (one HBM read, coalesced rows).
template <typename TIn>
__global__ void __launch_bounds__(256) k_quant_fp8_block(const TIn *__restrict__ w, int64_t K, uint8_t *__restrict__ q,
                                                         float *__restrict__ s) {
    __shared__ float red[8];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t row0 = (int64_t)blockIdx.y * 128 + warp * 16;
    const int64_t col = (int64_t)blockIdx.x * 128 + lane * 4;
    float v[16][4];
    float peak = 0.0f;
#pragma unroll
    for (int r = 0; r < 16; ++r) {
        const TIn *src = w + (row0 + r) * K + col;
        if constexpr (sizeof(TIn) == 4) {
            const float4 f = *reinterpret_cast<const float4 *>(src);
            v[r][0] = f.x; v[r][1] = f.y; v[r][2] = f.z; v[r][3] = f.w;
        } else {
            const uint2 u = *reinterpret_cast<const uint2 *>(src);
            v[r][0] = bf16_lo(u.x); v[r][1] = bf16_hi(u.x); v[r][2] = bf16_lo(u.y); v[r][3] = bf16_hi(u.y);
        }
#pragma unroll
        for (int j = 0; j < 4; j += 2) peak = absmax3(peak, v[r][j], v[r][j + 1]);
    }
    peak = warp_max_xor(peak, 32);
    if (lane == 0) red[warp] = peak;
    __syncthreads();
    peak = red[0];
#pragma unroll
    for (int i = 1; i < 8; ++i) peak = fmaxf(peak, red[i]);
    const float sc = __fdiv_rn(fmaxf(peak, 1e-4f), 448.0f);
#pragma unroll
    for (int r = 0; r < 16; ++r) {
        const uint32_t lo = pack2_e4m3(__fdiv_rn(v[r][0], sc), __fdiv_rn(v[r][1], sc));
        const uint32_t hi = pack2_e4m3(__fdiv_rn(v[r][2], sc), __fdiv_rn(v[r][3], sc));
        *reinterpret_cast<uint32_t *>(q + (row0 + r) * K + col) = lo | (hi << 16);
    }
    if (threadIdx.x == 0) s[(int64_t)blockIdx.y * gridDim.x + blockIdx.x] = sc;
}

// int8 KV dequantizer (world.py:93-94): y = bf16(float(q) * s) per (token, head) row of D codes. Each thread
// turns 16 codes (one 16-byte load) into 16 bf16 (two 16-byte stores). HBM-bound: 1 byte read + 2 bytes
// written per element, plus 4 bytes of scale per row.
__global__ void __launch_bounds__(256) k_dequant_kv(const int8_t *__restrict__ q, const float *__restrict__ s,
                                                    int64_t rows, int64_t D, __nv_bfloat16 *__restrict__ y) {
    const int64_t per_row = D >> 4;
    const int64_t n = rows * per_row;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t row = i / per_row;
        const uint4 c = ldg_stream(reinterpret_cast<const uint4 *>(q) + i);
        const float sc = __ldg(s + row);
        const uint32_t cw[4] = {c.x, c.y, c.z, c.w};
        uint32_t o[8];
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            float f[4];
#pragma unroll
            for (int b = 0; b < 4; ++b) f[b] = __fmul_rn((float)(int8_t)((cw[w] >> (8 * b)) & 0xFFu), sc);
            o[2 * w] = bf16x2_rn(f[0], f[1]);
            o[2 * w + 1] = bf16x2_rn(f[2], f[3]);
        }
        uint4 *dst = reinterpret_cast<uint4 *>(y) + 2 * i;
        dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
        dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
    }
}

cudaError_t launch_dequant_kv(const int8_t *q, const float *s, int64_t rows, int64_t D, void *y, cudaStream_t st) {
    const int64_t n = rows * (D >> 4);
    int64_t grid = cdiv(n, 256);
    const int64_t cap = (int64_t)num_sms() * 8;
    if (grid > cap) grid = cap;
    k_dequant_kv<<<(unsigned)grid, 256, 0, st>>>(q, s, rows, D, (__nv_bfloat16 *)y);
    return cudaGetLastError();
}

cudaError_t launch_quant_fp8_block(const void *w, int w_dtype, int64_t N, int64_t K, void *q, float *s,
                                   cudaStream_t st) {
    dim3 grid((unsigned)(K / 128), (unsigned)(N / 128));
    if (w_dtype == 2)
        k_quant_fp8_block<float><<<grid, 256, 0, st>>>(static_cast<const float *>(w), K, static_cast<uint8_t *>(q), s);
    else
        k_quant_fp8_block<__nv_bfloat16><<<grid, 256, 0, st>>>(static_cast<const __nv_bfloat16 *>(w), K,
                                                               static_cast<uint8_t *>(q), s);
    return cudaGetLastError();
}

} // namespace hn
