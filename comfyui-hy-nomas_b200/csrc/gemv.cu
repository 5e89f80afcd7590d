// gemv.cu - K2 for a few token rows (M <= GEMV_MAX_M, int8): the block-scaled GEMM as a weight-streaming GEMV.
//
// With one to a few activation rows the 128-row tensor-core tile does 1/128 of useful work and the linear is a
// read of the weight matrix: hy_nomas/model.py:247's Modulate(vec) is one such call per block (M = batch = 1),
// and the DiT step stacks all blocks' modulation weights into one [blocks * 6D, D] linear. Here one warp streams
// one weight row (output column n) with 16-byte non-allocating loads, 512 bytes per warp step: lane l holds bytes
// [16 l, 16 l + 16) of a step, so the 8 lanes of octet j hold K group 4 i + j of step i. The group's
// integer dot for each activation row is dp4a over the lane's 16 bytes and a 3-step butterfly in the octet; the
// four groups of a step are then folded in group order by every lane (4 shuffles), with the same fp32 operations
// as the tile kernel's epilogue (gemm.cu), so both produce identical bits:
//   PMODE 0 (sw per row x group):  t = RN(p * sa_g); acc = fma(t, sw[n,g], acc)
//   PMODE 1 (sw per row):          acc = fma(p, sa_g, acc); y = RN(acc * sw[n])
//   PMODE 2 (both per row):        D = sum over all K (int32); y = RN(RN(RN32(D) * sa[m]) * sw[n])
// then + bias (one rounding), the GELU epilogue if asked, and the store. Lane m writes row m's output.
#include "hn_common.cuh"
#include "hn_kernels.h"

namespace hn {
namespace gemv {

constexpr int WARPS = 8;  // warps per CTA

struct Params {
    const int8_t *qa; int64_t lda;
    const float *sa; int64_t sa_rs, sa_gs; int sa_mode;
    const int8_t *qw; int64_t ldw;
    const float *sw; int64_t sw_rs, sw_gs;
    const void *bias; int bias_dtype;
    void *out; int64_t ldo; int out_dtype;
    int M, N, K, G;
};

__device__ __forceinline__ int dot16(uint4 w, uint4 a) {
    int d = __dp4a((int)w.x, (int)a.x, 0);
    d = __dp4a((int)w.y, (int)a.y, d);
    d = __dp4a((int)w.z, (int)a.z, d);
    return __dp4a((int)w.w, (int)a.w, d);
}

__device__ __forceinline__ float bias_at(const void *bias, int dtype, int64_t n) {
    if (bias == nullptr) return 0.0f;
    if (dtype == 2) return static_cast<const float *>(bias)[n];
    if (dtype == 0) return __bfloat162float(static_cast<const __nv_bfloat16 *>(bias)[n]);
    return __half2float(static_cast<const __half *>(bias)[n]);
}

template <int MM, int PMODE, int EPI>
__global__ void __launch_bounds__(32 * WARPS) k_gemv(const Params p) {
    const int lane = threadIdx.x & 31;
    const int64_t warp0 = (int64_t)blockIdx.x * WARPS + (threadIdx.x >> 5);
    const int64_t nwarps = (int64_t)gridDim.x * WARPS;
    const int steps = (p.K + 511) / 512;
    // one 512-byte step's loads at a time: with the registers of deeper unrolling fewer warps are resident and
    // the kernel was slower (1.13-1.17 ms against 1.07 ms at M = 1 for 983040 x 4096 weights)
    constexpr int U = 1;
    for (int64_t n = warp0; n < p.N; n += nwarps) {
        const int8_t *wrow = p.qw + n * p.ldw;
        float acc[MM];
        int dtot[MM];
#pragma unroll
        for (int m = 0; m < MM; ++m) { acc[m] = 0.0f; dtot[m] = 0; }
        for (int i0 = 0; i0 < steps; i0 += U) {
            uint4 w[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int k0 = (i0 + u) * 512 + lane * 16;
                w[u] = k0 < p.K ? ldg_stream(wrow + k0) : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int i = i0 + u;
                if (i >= steps) break;
                const int k0 = i * 512 + lane * 16;
                const bool in = k0 < p.K;
                int part[MM];
#pragma unroll
                for (int m = 0; m < MM; ++m) {
                    const uint4 a = (in && m < p.M) ? __ldg(reinterpret_cast<const uint4 *>(p.qa + m * p.lda + k0))
                                                    : make_uint4(0, 0, 0, 0);
                    part[m] = dot16(w[u], a);
                }
                if constexpr (PMODE == 2) {
#pragma unroll
                    for (int m = 0; m < MM; ++m) dtot[m] += part[m];
                } else {
                    // the octet's 128 bytes: group 4 i + (lane / 8)
#pragma unroll
                    for (int m = 0; m < MM; ++m) {
                        part[m] += __shfl_xor_sync(0xffffffffu, part[m], 1);
                        part[m] += __shfl_xor_sync(0xffffffffu, part[m], 2);
                        part[m] += __shfl_xor_sync(0xffffffffu, part[m], 4);
                    }
                    // fold the step's four groups in order (every lane, redundantly)
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const int g = 4 * i + j;
                        if (g >= p.G) break;
                        const float swg = (PMODE == 0) ? __ldg(p.sw + n * p.sw_rs + (int64_t)g * p.sw_gs) : 0.0f;
#pragma unroll
                        for (int m = 0; m < MM; ++m) {
                            const int pg = __shfl_sync(0xffffffffu, part[m], 8 * j);
                            const int mr = m < p.M ? m : 0;
                            const float sg = (p.sa_mode == 0) ? __ldg(p.sa + mr * p.sa_rs + (int64_t)g * p.sa_gs)
                                                              : __ldg(p.sa + mr * p.sa_rs);
                            if (PMODE == 0) acc[m] = __fmaf_rn(__fmul_rn((float)pg, sg), swg, acc[m]);
                            else acc[m] = __fmaf_rn((float)pg, sg, acc[m]);
                        }
                    }
                }
            }
        }
        if constexpr (PMODE == 2) {
#pragma unroll
            for (int m = 0; m < MM; ++m) {
                int d = dtot[m];
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
                dtot[m] = d;
            }
        }
        // lane m stores row m
#pragma unroll
        for (int m = 0; m < MM; ++m) {
            if (m >= p.M || lane != m) continue;
            float v;
            if (PMODE == 2) {
                if (p.out_dtype == 3) {
                    reinterpret_cast<int32_t *>(p.out)[m * p.ldo + n] = dtot[m];
                    continue;
                }
                v = __fmul_rn(__fmul_rn(__int2float_rn(dtot[m]), __ldg(p.sa + m * p.sa_rs)), __ldg(p.sw + n * p.sw_rs));
            } else if (PMODE == 1) {
                v = __fmul_rn(acc[m], __ldg(p.sw + n * p.sw_rs));
            } else {
                v = acc[m];
            }
            if (p.bias != nullptr) v = __fadd_rn(v, bias_at(p.bias, p.bias_dtype, n));
            if (EPI == 1) {
                float dummy = 0.0f;
                gelu_bf16_pair(v, dummy);
            }
            const int64_t o = m * p.ldo + n;
            if (p.out_dtype == 0 || EPI == 1) reinterpret_cast<__nv_bfloat16 *>(p.out)[o] = __float2bfloat16_rn(v);
            else if (p.out_dtype == 1) reinterpret_cast<__half *>(p.out)[o] = __float2half_rn(v);
            else reinterpret_cast<float *>(p.out)[o] = v;
        }
    }
}

template <int MM, int PMODE, int EPI>
static cudaError_t launch_e(const Params &p, cudaStream_t st) {
    auto kern = k_gemv<MM, PMODE, EPI>;
    // every CTA resident at once (grid = SMs x resident CTAs per SM), grid-stride over the weight rows: a larger
    // grid would leave the rows of its non-resident CTAs to a second, partial wave
    static int per_sm = 0;
    if (per_sm == 0) {
        int n = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, 32 * WARPS, 0) != cudaSuccess || n < 1) n = 1;
        per_sm = n;
    }
    int64_t grid = (int64_t)num_sms() * per_sm;
    const int64_t need = (p.N + WARPS - 1) / WARPS;
    if (grid > need) grid = need;
    kern<<<(unsigned)grid, 32 * WARPS, 0, st>>>(p);
    return cudaGetLastError();
}

template <int MM, int PMODE>
static cudaError_t launch_m(const Params &p, int epi, cudaStream_t st) {
    return epi == 1 ? launch_e<MM, PMODE, 1>(p, st) : launch_e<MM, PMODE, 0>(p, st);
}

template <int PMODE>
static cudaError_t launch_p(const Params &p, int epi, cudaStream_t st) {
    static_assert(GEMV_MAX_M == 2, "instantiations cover M = 1 and 2");
    if (p.M <= 1) return launch_m<1, PMODE>(p, epi, st);
    return launch_m<2, PMODE>(p, epi, st);
}

} // namespace gemv

bool gemv_applies(const GemmArgs &a) {
    return a.kind == 0 && a.M >= 1 && a.M <= GEMV_MAX_M && a.epilogue != 2 && a.sw_mode != 2;
}

cudaError_t launch_gemv(const GemmArgs &a, cudaStream_t st) {
    gemv::Params p;
    p.qa = static_cast<const int8_t *>(a.qa); p.lda = a.lda;
    p.sa = a.sa; p.sa_rs = a.sa_rs; p.sa_gs = a.sa_gs; p.sa_mode = a.sa_mode;
    p.qw = static_cast<const int8_t *>(a.qw); p.ldw = a.ldw;
    p.sw = a.sw; p.sw_rs = a.sw_rs; p.sw_gs = a.sw_gs;
    p.bias = a.bias; p.bias_dtype = a.bias_dtype;
    p.out = a.out; p.ldo = a.ldo; p.out_dtype = a.out_dtype;
    p.M = (int)a.M; p.N = (int)a.N; p.K = (int)a.K; p.G = (int)(a.K / 128);
    const int pmode = (a.sa_mode == 1 && a.sw_mode == 1) ? 2 : (a.sw_mode == 0 ? 0 : 1);
    if (pmode == 0) return gemv::launch_p<0>(p, a.epilogue, st);
    if (pmode == 1) return gemv::launch_p<1>(p, a.epilogue, st);
    return gemv::launch_p<2>(p, a.epilogue, st);
}

} // namespace hn
