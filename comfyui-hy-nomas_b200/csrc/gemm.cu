// gemm.cu - K2, the block-scaled W8A8 / FP8 GEMM (hy_nomas/kernels.py:80-170) on the sm_100a tensor cores.
//
//   y[m, n] = sum_g sa[m, g] * sw[n, g] * dot_g(qa[m, :], qw[n, :])  (+ bias[n]),  g over 128-wide K groups
//
// Design (one persistent CTA per SM, 384 threads, tile 128 x 256, one K group = 128 bytes per stage):
//   warp 0      producer: cp.async.bulk.tensor 2-D loads of the A tile [128 x 128 B] and the B tile
//               [256 x 128 B] (both 128B-swizzled) into a 4-stage shared-memory ring (48 KB a stage), and
//               (when the weight scale varies per group) the 256 weight scales of each group into a
//               4-slot scale ring.
//   warp 1      MMA issuer: allocates 512 TMEM columns (two 256-column accumulators), and for each K group
//               issues 4 x tcgen05.mma.kind::{i8,f8f6f4} (M=128, N=256, K=32) into one accumulator, then
//               tcgen05.commit to free the smem stage and to signal the epilogue.
//   warps 4-11  epilogue / promotion: warp w reads TMEM lanes 32*(w%4).. (its 32 rows) and the column
//               half (w-4)/4, i.e. each thread owns one output row x 128 columns, held in 64 packed
//               f32x2 registers. Per group: tcgen05.ld of the int32 (or fp32) partial, exact int->float
//               conversion (add 0x4B400000, subtract 1.5*2^23: exact for |p| < 2^22), scale by sa/sw with
//               packed f32x2 multiply / FMA, and release of the accumulator. While the epilogue promotes
//               group g, the tensor core computes group g+1 into the other accumulator.
//   After the last group: scale by the per-row weight scale when it was factored out, + bias, then
//   the epilogue of kernels.py:123-137 (cast / GELU / GELU + int8 requantization per 128 columns).
//
// Promotion arithmetic (the CPU oracle evaluates the same):
//   PMODE 0 (sw per row x group):  t = RN(p * sa[m,g]);  acc = fma(t, sw[n,g], acc)
//   PMODE 1 (sw per row or block):  acc = fma(p, s, acc) with s = sa[m,g] (sw per row, applied at the end)
//                                   or s = RN(sa[m,g] * swb[n/128,g]) (128x128 weight blocks)
//   PMODE 2 (both per row):         one accumulator over all K; y = RN(RN(float(D) * sa[m]) * sw[n])
//
// Every wait on an mbarrier is bounded (globaltimer); on expiry the kernel records HN_DEVERR_TIMEOUT,
// makes the other roles leave their loops, waits briefly for its own copies/MMAs in flight, frees TMEM
// and returns. No TMA multicast is used anywhere (every CTA loads its own tiles).
#include <cuda.h>
#include <cudaTypedefs.h>

#include "hn_common.cuh"
#include "hn_kernels.h"

namespace hn {

// Device error word (0 = ok): bounded waits OR in HN_DEVERR_* bits.
__device__ int g_device_error = 0;

cudaError_t read_and_clear_device_error(int *value) {
    int zero = 0;
    cudaError_t e = cudaMemcpyFromSymbol(value, g_device_error, sizeof(int));
    if (e != cudaSuccess) return e;
    return cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int));
}

namespace gemm {

constexpr int BM = 128, BN = 256, BK = 128;
constexpr int STAGES = 4;
constexpr int A_STAGE = BM * BK;  // bytes
constexpr int B_STAGE = BN * BK;
constexpr int THREADS = 384;   // 3 warpgroups
constexpr int EPI_WARP0 = 4;   // warpgroups 1-2 are the epilogue
// 384 threads at one CTA per SM give every thread 168 registers (registers are allocated per SM
// sub-partition: 3 warps x 32 x 168 <= 16384). The epilogue's 64 packed accumulators fit in that budget,
// so no warpgroup register split (setmaxnreg) is used.
constexpr int SW_SLOTS = 4;
constexpr int TMEM_COLS = 512;
constexpr uint64_t WAIT_NS = 2000000000ull;  // 2 s

// shared-memory map (offsets from a 1024-aligned base)
constexpr int OFF_A = 0;
constexpr int OFF_B = OFF_A + STAGES * A_STAGE;
constexpr int OFF_SW = OFF_B + STAGES * B_STAGE;                  // float[SW_SLOTS][256]
constexpr int OFF_BAR = OFF_SW + SW_SLOTS * 256 * 4;              // full[S] empty[S] tfull[2] tempty[2] sfull[W] sempty[W]
constexpr int OFF_MISC = OFF_BAR + (2 * STAGES + 4 + 2 * SW_SLOTS) * 8;  // tmem base, abort flag
constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;         // + alignment slack

struct Params {
    const float *sa; int64_t ldsa; int sa_mode;
    const float *sw; int64_t ldsw; int sw_mode;
    const void *bias; int bias_dtype;
    void *out; int64_t ldo; int out_dtype;
    float *qs; int64_t ldqs;
    int M, N, K, G;
    int n_blocks, num_tiles;
    int vec_store;
};

// ---------------------------------------------------------------------------------------------------
// PTX wrappers

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok)
                 : "r"(bar), "r"(parity)
                 : "memory");
    return ok != 0;
}
// bounded wait: false when the kernel is aborting (this wait timed out, or another role's did)
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int *abort_flag, uint64_t limit_ns) {
    if (mbar_try(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    while (true) {
#pragma unroll 1
        for (int i = 0; i < 32; ++i)
            if (mbar_try(bar, parity)) return true;
        if (*abort_flag) return false;
        if (globaltimer_ns() - t0 > limit_ns) {
            *abort_flag = 1;
            atomicOr(&g_device_error, HN_DEVERR_TIMEOUT);
            return false;
        }
    }
}

__device__ __forceinline__ void tma_load_2d(const CUtensorMap *map, uint32_t dst, uint32_t bar, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
                 ::"r"(dst), "l"((uint64_t)map), "r"(bar), "r"(x), "r"(y)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// K-major operand tile, 128-byte rows, 128B swizzle: SBO = 1024 B between 8-row core groups,
// LBO unused (16 B), descriptor version 1 (sm_100), layout type 2 (SWIZZLE_128B).
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

template <int KIND>
__device__ __forceinline__ void mma_128x256x32(uint32_t d_tmem, uint64_t ad, uint64_t bd, uint32_t idesc, uint32_t acc) {
    if (KIND == 0)
        asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                     "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}"
                     ::"r"(d_tmem), "l"(ad), "l"(bd), "r"(idesc), "r"(acc) : "memory");
    else
        asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                     "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}"
                     ::"r"(d_tmem), "l"(ad), "l"(bd), "r"(idesc), "r"(acc) : "memory");
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns, completed (wait::ld) inside the same statement so no use of
// the destination registers can be scheduled before the data has arrived.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
}

// ---- packed fp32x2 promotion steps (sm_100 f32x2 instructions, explicit .rn: never contracted) ----
union F2 {
    uint64_t u;
    float f[2];
};
__device__ __forceinline__ uint64_t pk(float lo, float hi) {
    F2 v;
    v.f[0] = lo;
    v.f[1] = hi;
    return v.u;
}

// int8: acc = fma(RN(conv(p) * sa), sw2, acc)     (PMODE 0)
template <int KIND>
__device__ __forceinline__ void promote_gen(uint64_t &acc, uint32_t p0, uint32_t p1, uint64_t sa2, uint64_t sw2) {
    if (KIND == 0)
        asm("{\n\t.reg .b32 a, b;\n\t.reg .b64 f, t;\n\t"
            "add.s32 a, %1, 0x4B400000;\n\tadd.s32 b, %2, 0x4B400000;\n\t"
            "mov.b64 f, {a, b};\n\t"
            "add.rn.f32x2 f, f, %5;\n\t"
            "mul.rn.f32x2 t, f, %3;\n\t"
            "fma.rn.f32x2 %0, t, %4, %0;\n\t}"
            : "+l"(acc)
            : "r"(p0), "r"(p1), "l"(sa2), "l"(sw2), "l"(pk(-12582912.0f, -12582912.0f)));
    else
        asm("{\n\t.reg .b64 f, t;\n\t"
            "mov.b64 f, {%1, %2};\n\t"
            "mul.rn.f32x2 t, f, %3;\n\t"
            "fma.rn.f32x2 %0, t, %4, %0;\n\t}"
            : "+l"(acc)
            : "r"(p0), "r"(p1), "l"(sa2), "l"(sw2));
}
// acc = fma(conv(p), s2, acc)     (PMODE 1)
template <int KIND>
__device__ __forceinline__ void promote_row(uint64_t &acc, uint32_t p0, uint32_t p1, uint64_t s2) {
    if (KIND == 0)
        asm("{\n\t.reg .b32 a, b;\n\t.reg .b64 f;\n\t"
            "add.s32 a, %1, 0x4B400000;\n\tadd.s32 b, %2, 0x4B400000;\n\t"
            "mov.b64 f, {a, b};\n\t"
            "add.rn.f32x2 f, f, %4;\n\t"
            "fma.rn.f32x2 %0, f, %3, %0;\n\t}"
            : "+l"(acc)
            : "r"(p0), "r"(p1), "l"(s2), "l"(pk(-12582912.0f, -12582912.0f)));
    else
        asm("{\n\t.reg .b64 f;\n\t"
            "mov.b64 f, {%1, %2};\n\t"
            "fma.rn.f32x2 %0, f, %3, %0;\n\t}"
            : "+l"(acc)
            : "r"(p0), "r"(p1), "l"(s2));
}

__device__ __forceinline__ float acc_lo(uint64_t a) { F2 v; v.u = a; return v.f[0]; }
__device__ __forceinline__ float acc_hi(uint64_t a) { F2 v; v.u = a; return v.f[1]; }

__device__ __forceinline__ void load_bias8(const void *bias, int dtype, int64_t n, float *b) {
    if (dtype == 2) {
        const float4 *p = reinterpret_cast<const float4 *>(static_cast<const float *>(bias) + n);
        float4 a = p[0], c = p[1];
        b[0] = a.x; b[1] = a.y; b[2] = a.z; b[3] = a.w; b[4] = c.x; b[5] = c.y; b[6] = c.z; b[7] = c.w;
    } else if (dtype == 0) {
        Elem<__nv_bfloat16>::load8(static_cast<const __nv_bfloat16 *>(bias) + n, b);
    } else {
        Elem<__half>::load8(static_cast<const __half *>(bias) + n, b);
    }
}
__device__ __forceinline__ float load_bias1(const void *bias, int dtype, int64_t n) {
    if (dtype == 2) return static_cast<const float *>(bias)[n];
    if (dtype == 0) return __bfloat162float(static_cast<const __nv_bfloat16 *>(bias)[n]);
    return __half2float(static_cast<const __half *>(bias)[n]);
}

// ---------------------------------------------------------------------------------------------------

template <int KIND, int PMODE, int EPI>
__global__ void __launch_bounds__(THREADS, 1)
    k_block_gemm(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bar_full = sbase + OFF_BAR;
    const uint32_t bar_empty = bar_full + STAGES * 8;
    const uint32_t bar_tfull = bar_empty + STAGES * 8;
    const uint32_t bar_tempty = bar_tfull + 2 * 8;
    const uint32_t bar_sfull = bar_tempty + 2 * 8;
    const uint32_t bar_sempty = bar_sfull + SW_SLOTS * 8;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + OFF_MISC);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + OFF_MISC + 4);
    float *sw_s = reinterpret_cast<float *>(smem + OFF_SW);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = p.G;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(bar_full + 8 * s, 1);
            mbar_init(bar_empty + 8 * s, 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(bar_tfull + 8 * b, 1);
            mbar_init(bar_tempty + 8 * b, 8);
        }
        for (int s = 0; s < SW_SLOTS; ++s) {
            mbar_init(bar_sfull + 8 * s, 32);
            mbar_init(bar_sempty + 8 * s, 8);
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 0 && lane == 0) {
        asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmA) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmB) : "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------------------------ producer (TMA + scale ring)
        int stage = 0, slot = 0;
        uint32_t phase = 0, sphase = 0;
        int issued = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
            const int m0 = (tile / p.n_blocks) * BM, n0 = (tile % p.n_blocks) * BN;
            for (int g = 0; g < G; ++g) {
                ok = __all_sync(0xffffffffu, mbar_wait(bar_empty + 8 * stage, phase ^ 1, abort_flag, WAIT_NS));
                if (!ok) break;
                if (lane == 0) {
                    const uint32_t fb = bar_full + 8 * stage;
                    mbar_arrive_tx(fb, A_STAGE + B_STAGE);
                    tma_load_2d(&tmA, sbase + OFF_A + stage * A_STAGE, fb, g * BK, m0);
                    tma_load_2d(&tmB, sbase + OFF_B + stage * B_STAGE, fb, g * BK, n0);
                }
                ++issued;
                if (++stage == STAGES) { stage = 0; phase ^= 1; }
                if (PMODE == 0) {
                    // weight scales of this group for the tile's 256 columns
                    ok = __all_sync(0xffffffffu, mbar_wait(bar_sempty + 8 * slot, sphase ^ 1, abort_flag, WAIT_NS));
                    if (!ok) break;
                    float *dst = sw_s + slot * 256;
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const int c = lane + 32 * i;
                        const int n = n0 + c;
                        dst[c] = (n < p.N) ? p.sw[(int64_t)n * p.ldsw + g] : 0.0f;
                    }
                    mbar_arrive(bar_sfull + 8 * slot);
                    if (++slot == SW_SLOTS) { slot = 0; sphase ^= 1; }
                }
            }
        }
        // drain: wait (briefly) until the last copies issued have landed before the CTA can exit
        int st = stage;
        uint32_t ph = phase;
        for (int i = 0; i < STAGES && i < issued; ++i) {
            if (--st < 0) { st = STAGES - 1; ph ^= 1; }
            volatile int never = 0;
            mbar_wait(bar_full + 8 * st, ph, &never, 100000000ull);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------------ MMA issuer
        const uint32_t idesc = KIND == 0
                                   ? ((2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24))
                                   : ((1u << 4) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24));
        int stage = 0;
        uint32_t phase = 0;
        int tb = 0;
        uint32_t tphase = 0;
        bool ok = true;
        int last_stage = -1;
        uint32_t last_phase = 0;
        for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
            if (PMODE == 2) {
                ok = __all_sync(0xffffffffu, mbar_wait(bar_tempty + 8 * tb, tphase ^ 1, abort_flag, WAIT_NS));
                if (!ok) break;
                tc_fence_after();
            }
            for (int g = 0; g < G; ++g) {
                if (PMODE != 2) {
                    ok = __all_sync(0xffffffffu, mbar_wait(bar_tempty + 8 * tb, tphase ^ 1, abort_flag, WAIT_NS));
                    if (!ok) break;
                    tc_fence_after();
                }
                ok = __all_sync(0xffffffffu, mbar_wait(bar_full + 8 * stage, phase, abort_flag, WAIT_NS));
                if (!ok) break;
                tc_fence_after();
                if (lane == 0) {
                    const uint32_t d = tmem_base + (uint32_t)(tb * BN);
                    const uint64_t ad = sdesc(sbase + OFF_A + stage * A_STAGE);
                    const uint64_t bd = sdesc(sbase + OFF_B + stage * B_STAGE);
#pragma unroll
                    for (int k = 0; k < BK / 32; ++k)
                        mma_128x256x32<KIND>(d, ad + 2 * k, bd + 2 * k, idesc,
                                             (PMODE == 2) ? (uint32_t)(g > 0 || k > 0) : (uint32_t)(k > 0));
                    mma_commit(bar_empty + 8 * stage);
                    if (PMODE != 2) mma_commit(bar_tfull + 8 * tb);
                }
                __syncwarp();
                last_stage = stage;
                last_phase = phase;
                if (++stage == STAGES) { stage = 0; phase ^= 1; }
                if (PMODE != 2) { tb ^= 1; if (tb == 0) tphase ^= 1; }
            }
            if (PMODE == 2 && ok) {
                if (lane == 0) mma_commit(bar_tfull + 8 * tb);
                __syncwarp();
                tb ^= 1;
                if (tb == 0) tphase ^= 1;
            }
        }
        // drain: the MMAs behind the last commit finish before TMEM is released
        if (last_stage >= 0) {
            volatile int never = 0;
            mbar_wait(bar_empty + 8 * last_stage, last_phase, &never, 100000000ull);
        }
    } else if (warp >= EPI_WARP0) {
        // ------------------------------------------------------------------ epilogue / promotion (warps 4-11)
        const int ew = warp - EPI_WARP0;
        const int q = warp & 3;
        const int hf = ew >> 2;
        const int row = q * 32 + lane;
        const uint32_t lane_addr = tmem_base + ((uint32_t)(q * 32) << 16);
        int tb = 0, slot = 0;
        uint32_t tphase = 0, sphase = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
            const int m0 = (tile / p.n_blocks) * BM, n0 = (tile % p.n_blocks) * BN;
            const int m = m0 + row;
            const int mm = m < p.M ? m : p.M - 1;
            const int ncol0 = n0 + hf * 128;
            uint64_t acc[64];
#pragma unroll
            for (int i = 0; i < 64; ++i) acc[i] = 0ull;
            if (PMODE != 2) {
                float sa_next = (p.sa_mode == 0) ? p.sa[(int64_t)mm * p.ldsa] : p.sa[mm];
                for (int g = 0; g < G; ++g) {
                    const float sa_g = sa_next;
                    if (g + 1 < G && p.sa_mode == 0) sa_next = p.sa[(int64_t)mm * p.ldsa + g + 1];
                    float s = sa_g;
                    if (PMODE == 1 && p.sw_mode == 2) s = __fmul_rn(sa_g, p.sw[(int64_t)(ncol0 >> 7) * p.ldsw + g]);
                    const uint64_t s2 = pk(s, s);
                    if (PMODE == 0) {
                        ok = __all_sync(0xffffffffu, mbar_wait(bar_sfull + 8 * slot, sphase, abort_flag, WAIT_NS));
                        if (!ok) break;
                    }
                    ok = __all_sync(0xffffffffu, mbar_wait(bar_tfull + 8 * tb, tphase, abort_flag, WAIT_NS));
                    if (!ok) break;
                    tc_fence_after();
                    const uint32_t tcol = lane_addr + (uint32_t)(tb * BN + hf * 128);
                    const float *sws = sw_s + slot * 256 + hf * 128;
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        uint32_t r[32];
                        tmem_ld32(tcol + c * 32, r);
#pragma unroll
                        for (int j = 0; j < 32; j += 4) {
                            if (PMODE == 0) {
                                const float4 w4 = *reinterpret_cast<const float4 *>(sws + c * 32 + j);
                                promote_gen<KIND>(acc[c * 16 + j / 2], r[j], r[j + 1], s2, pk(w4.x, w4.y));
                                promote_gen<KIND>(acc[c * 16 + j / 2 + 1], r[j + 2], r[j + 3], s2, pk(w4.z, w4.w));
                            } else {
                                promote_row<KIND>(acc[c * 16 + j / 2], r[j], r[j + 1], s2);
                                promote_row<KIND>(acc[c * 16 + j / 2 + 1], r[j + 2], r[j + 3], s2);
                            }
                        }
                    }
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) {
                        mbar_arrive(bar_tempty + 8 * tb);
                        if (PMODE == 0) mbar_arrive(bar_sempty + 8 * slot);
                    }
                    tb ^= 1;
                    if (tb == 0) tphase ^= 1;
                    if (PMODE == 0) { if (++slot == SW_SLOTS) { slot = 0; sphase ^= 1; } }
                }
                if (!ok) break;
                if (PMODE == 1 && p.sw_mode == 1) {
#pragma unroll
                    for (int j = 0; j < 128; j += 2) {
                        const int n = ncol0 + j;
                        const float w0 = (n < p.N) ? p.sw[n] : 0.0f, w1 = (n + 1 < p.N) ? p.sw[n + 1] : 0.0f;
                        acc[j / 2] = pk(__fmul_rn(acc_lo(acc[j / 2]), w0), __fmul_rn(acc_hi(acc[j / 2]), w1));
                    }
                }
            } else {
                // PMODE 2: one accumulator over all of K
                ok = __all_sync(0xffffffffu, mbar_wait(bar_tfull + 8 * tb, tphase, abort_flag, WAIT_NS));
                if (!ok) break;
                tc_fence_after();
                const uint32_t tcol = lane_addr + (uint32_t)(tb * BN + hf * 128);
                const float sam = p.sa[mm];
                const bool raw = (p.out_dtype == 3);
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    uint32_t r[32];
                    tmem_ld32(tcol + c * 32, r);
#pragma unroll
                    for (int j = 0; j < 32; j += 2) {
                        float a0, a1;
                        if (raw) {
                            a0 = __uint_as_float(r[j]);
                            a1 = __uint_as_float(r[j + 1]);
                        } else {
                            const int n = ncol0 + c * 32 + j;
                            const float w0 = (n < p.N) ? p.sw[n] : 0.0f, w1 = (n + 1 < p.N) ? p.sw[n + 1] : 0.0f;
                            const float d0 = KIND == 0 ? __int2float_rn((int)r[j]) : __uint_as_float(r[j]);
                            const float d1 = KIND == 0 ? __int2float_rn((int)r[j + 1]) : __uint_as_float(r[j + 1]);
                            a0 = __fmul_rn(__fmul_rn(d0, sam), w0);
                            a1 = __fmul_rn(__fmul_rn(d1, sam), w1);
                        }
                        acc[c * 16 + j / 2] = pk(a0, a1);
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(bar_tempty + 8 * tb);
                tb ^= 1;
                if (tb == 0) tphase ^= 1;
            }

            // ---------------------------------------------------------- bias + output epilogue
            const bool row_ok = m < p.M;
            const bool full_cols = ncol0 + 128 <= p.N;
            if (p.bias != nullptr && !(PMODE == 2 && p.out_dtype == 3)) {
#pragma unroll
                for (int j = 0; j < 128; j += 8) {
                    float b[8];
                    if (full_cols) load_bias8(p.bias, p.bias_dtype, ncol0 + j, b);
                    else {
#pragma unroll
                        for (int i = 0; i < 8; ++i)
                            b[i] = (ncol0 + j + i < p.N) ? load_bias1(p.bias, p.bias_dtype, ncol0 + j + i) : 0.0f;
                    }
#pragma unroll
                    for (int i = 0; i < 8; i += 2)
                        acc[(j + i) / 2] = pk(__fadd_rn(acc_lo(acc[(j + i) / 2]), b[i]), __fadd_rn(acc_hi(acc[(j + i) / 2]), b[i + 1]));
                }
            }
            if (EPI != 0) {
#pragma unroll
                for (int i = 0; i < 64; ++i)
                    acc[i] = pk(rbf16(gelu_tanh(rbf16(acc_lo(acc[i])))), rbf16(gelu_tanh(rbf16(acc_hi(acc[i])))));
            }
            if (row_ok) {
                if (EPI == 2) {
                    if (full_cols) {  // N % 128 == 0: a 128-column group is entirely inside or outside
                        float peak = 0.0f;
#pragma unroll
                        for (int i = 0; i < 64; ++i) peak = fmaxf(peak, fmaxf(fabsf(acc_lo(acc[i])), fabsf(acc_hi(acc[i]))));
                        const float sc = i8_scale(peak);
                        int8_t *qrow = static_cast<int8_t *>(p.out) + (int64_t)m * p.ldo + ncol0;
#pragma unroll
                        for (int j = 0; j < 128; j += 16) {
                            uint4 o;
                            uint32_t *ow = &o.x;
#pragma unroll
                            for (int w = 0; w < 4; ++w) {
                                const uint64_t a = acc[(j + 4 * w) / 2], b2 = acc[(j + 4 * w) / 2 + 1];
                                ow[w] = pack4_i8(code_i8(__fdiv_rn(acc_lo(a), sc)), code_i8(__fdiv_rn(acc_hi(a), sc)),
                                                 code_i8(__fdiv_rn(acc_lo(b2), sc)), code_i8(__fdiv_rn(acc_hi(b2), sc)));
                            }
                            *reinterpret_cast<uint4 *>(qrow + j) = o;
                        }
                        p.qs[(int64_t)m * p.ldqs + (ncol0 >> 7)] = sc;
                    }
                } else {
                    const int od = (EPI == 1) ? 0 : p.out_dtype;
                    uint8_t *orow = static_cast<uint8_t *>(p.out);
                    if (full_cols && p.vec_store) {
                        if (od == 0 || od == 1) {
                            uint16_t *o16 = reinterpret_cast<uint16_t *>(orow) + (int64_t)m * p.ldo + ncol0;
#pragma unroll
                            for (int j = 0; j < 128; j += 8) {
                                uint4 o;
                                uint32_t *ow = &o.x;
#pragma unroll
                                for (int w = 0; w < 4; ++w) {
                                    const uint64_t a = acc[(j + 2 * w) / 2];
                                    ow[w] = od == 0 ? pack_bf16_rn(acc_lo(a), acc_hi(a)) : pack_f16_rn(acc_lo(a), acc_hi(a));
                                }
                                *reinterpret_cast<uint4 *>(o16 + j) = o;
                            }
                        } else {
                            uint32_t *o32 = reinterpret_cast<uint32_t *>(orow) + (int64_t)m * p.ldo + ncol0;
#pragma unroll
                            for (int j = 0; j < 128; j += 4) {
                                uint4 o;
                                o.x = __float_as_uint(acc_lo(acc[j / 2]));
                                o.y = __float_as_uint(acc_hi(acc[j / 2]));
                                o.z = __float_as_uint(acc_lo(acc[j / 2 + 1]));
                                o.w = __float_as_uint(acc_hi(acc[j / 2 + 1]));
                                *reinterpret_cast<uint4 *>(o32 + j) = o;
                            }
                        }
                    } else {
#pragma unroll
                        for (int j = 0; j < 128; ++j) {
                            const int n = ncol0 + j;
                            if (n < p.N) {
                                const float v = (j & 1) ? acc_hi(acc[j / 2]) : acc_lo(acc[j / 2]);
                                if (od == 0) reinterpret_cast<__nv_bfloat16 *>(orow)[(int64_t)m * p.ldo + n] = __float2bfloat16_rn(v);
                                else if (od == 1) reinterpret_cast<__half *>(orow)[(int64_t)m * p.ldo + n] = __float2half_rn(v);
                                else reinterpret_cast<uint32_t *>(orow)[(int64_t)m * p.ldo + n] = __float_as_uint(v);
                            }
                        }
                    }
                }
            }
        }
        if (!ok) *abort_flag = 1;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) {
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS) : "memory");
    }
}

// ---------------------------------------------------------------------------------------------------
// host side

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (fn == nullptr) {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    }
    return fn;
}

// 2-D map over a row-major byte matrix [rows, cols] with row pitch ld bytes; box = 128 bytes x box_rows,
// 128B swizzle (matches the UMMA SWIZZLE_128B K-major layout), zero fill outside the matrix.
static bool make_map(CUtensorMap *map, const void *base, uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_rows) {
    PFN_cuTensorMapEncodeTiled_v12000 fn = encode_fn();
    if (fn == nullptr) return false;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {ld};
    cuuint32_t box[2] = {128, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

template <int KIND, int PMODE, int EPI>
static cudaError_t launch_t(const CUtensorMap &ma, const CUtensorMap &mb, const Params &p, int grid, cudaStream_t st) {
    auto kern = k_block_gemm<KIND, PMODE, EPI>;
    static bool configured = false;  // per instantiation; attribute setting is idempotent
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
        if (e != cudaSuccess) return e;
        configured = true;
    }
    kern<<<grid, THREADS, SMEM_BYTES, st>>>(ma, mb, p);
    return cudaGetLastError();
}

template <int KIND, int PMODE>
static cudaError_t launch_epi(int epi, const CUtensorMap &ma, const CUtensorMap &mb, const Params &p, int grid,
                              cudaStream_t st) {
    switch (epi) {
    case 0: return launch_t<KIND, PMODE, 0>(ma, mb, p, grid, st);
    case 1: return launch_t<KIND, PMODE, 1>(ma, mb, p, grid, st);
    default: return launch_t<KIND, PMODE, 2>(ma, mb, p, grid, st);
    }
}

} // namespace gemm

cudaError_t launch_block_gemm(const GemmArgs &a, cudaStream_t st, const char **msg) {
    using namespace gemm;
    CUtensorMap ma, mb;
    if (!make_map(&ma, a.qa, (uint64_t)a.M, (uint64_t)a.K, (uint64_t)a.lda, BM) ||
        !make_map(&mb, a.qw, (uint64_t)a.N, (uint64_t)a.K, (uint64_t)a.ldw, BN)) {
        *msg = "cuTensorMapEncodeTiled failed (pointer/stride alignment or driver entry point)";
        return cudaErrorInvalidValue;
    }
    Params p;
    p.sa = a.sa; p.ldsa = a.ldsa; p.sa_mode = a.sa_mode;
    p.sw = a.sw; p.ldsw = a.ldsw; p.sw_mode = a.sw_mode;
    p.bias = a.bias; p.bias_dtype = a.bias_dtype;
    p.out = a.out; p.ldo = a.ldo; p.out_dtype = a.out_dtype;
    p.qs = a.qs; p.ldqs = a.ldqs;
    p.M = (int)a.M; p.N = (int)a.N; p.K = (int)a.K; p.G = (int)(a.K / 128);
    p.n_blocks = (int)cdiv(a.N, BN);
    p.num_tiles = (int)(cdiv(a.M, BM) * p.n_blocks);
    const int esz = (a.epilogue == 2) ? 1 : (a.out_dtype == 0 || a.out_dtype == 1) ? 2 : 4;
    p.vec_store = ((reinterpret_cast<uintptr_t>(a.out) % 16) == 0 && (a.ldo * esz) % 16 == 0) ? 1 : 0;
    int grid = num_sms();
    if (grid > p.num_tiles) grid = p.num_tiles;
    int pmode;
    if (a.sa_mode == 1 && a.sw_mode == 1) pmode = 2;
    else if (a.sw_mode == 0) pmode = 0;
    else pmode = 1;
    if (a.kind == 0) {
        if (pmode == 0) return launch_epi<0, 0>(a.epilogue, ma, mb, p, grid, st);
        if (pmode == 1) return launch_epi<0, 1>(a.epilogue, ma, mb, p, grid, st);
        return launch_epi<0, 2>(a.epilogue, ma, mb, p, grid, st);
    }
    if (pmode == 0) return launch_epi<1, 0>(a.epilogue, ma, mb, p, grid, st);
    if (pmode == 1) return launch_epi<1, 1>(a.epilogue, ma, mb, p, grid, st);
    return launch_epi<1, 2>(a.epilogue, ma, mb, p, grid, st);
}

// ---------------------------------------------------------------------------------------------------
// Bounded-wait self-test: one CTA waits on an mbarrier that nothing completes, with a short limit.
__global__ void k_wait_selftest(uint64_t limit_ns) {
    __shared__ __align__(8) uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        gemm::mbar_init(gemm::smem_u32(&bar), 1);
        abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    if (threadIdx.x == 0) gemm::mbar_wait(gemm::smem_u32(&bar), 0, &abort_flag, limit_ns);
    __syncthreads();
}

cudaError_t launch_wait_selftest(uint32_t timeout_us, cudaStream_t st) {
    k_wait_selftest<<<1, 32, 0, st>>>((uint64_t)timeout_us * 1000ull);
    return cudaGetLastError();
}

} // namespace hn
