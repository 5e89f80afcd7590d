// gemm.cu - K2, the block-scaled W8A8 / FP8 GEMM (hy_nomas/kernels.py:80-170) on the sm_100a tensor cores.
//
//   y[m, n] = sum_g sa[m, g] * sw[n, g] * dot_g(qa[m, :], qw[n, :])  (+ bias[n]),  g over 128-wide K groups
//
// Design: one persistent CTA per SM, one warpgroup of producers/issuer plus NPART epilogue warpgroups,
// tiles of 128 rows x BN columns, GPS 128-wide K groups per pipeline stage.
//   warps 0, 2  producers: cp.async.bulk.tensor 3-D loads (box {128 B, rows, GPS groups}, 128B swizzle, no
//               multicast) of the A tile (warp 0) and the B tile (warp 2) into a ring of shared-memory
//               stages; one thread's bulk-tensor requests are serviced in order, so two issuing warps and
//               two groups per request raise the operand rate an SM draws from L2.
//   warp 3      scale ring: per pair of K groups, both groups' activation scales for the tile's 128 rows
//               (and the weight scales of its BN columns when they vary per group) into two shared-memory
//               slots that complete on one barrier - bulk copies when the scales are group-major, 4-byte
//               cp.async copies otherwise, several pairs in flight either way.
//   warp 1      MMA issuer: owns 512 TMEM columns = NBUF accumulators of BN columns; per K group it issues
//               4 x tcgen05.mma.kind::{i8,f8f6f4} (M=128, N=BN, K=32) and tcgen05.commit's the stage back
//               to the producers and the accumulator (per-group modes: the pair of accumulators) to the
//               epilogue.
//   epilogue    warp w (w >= 4) owns TMEM lanes 32*(w%4).. (32 output rows) and column part (w-4)/4, i.e.
//               each thread one row x BN/NPART columns.
// Two tile shapes, by how the scales vary along K:
//   * per-group scales (PMODE 0, 1): BN = 128, NBUF = 4, GPS = 2, four epilogue warpgroups (640 threads).
//     The four accumulators form two pairs, one pair per stage (two K groups): every handover - operands
//     in, pair to the epilogue, pair back, scales in, scale slots back - is one barrier per pair, since
//     each barrier round trip drains the tensor pipe's short queue. For every group the epilogue reads
//     the int32 (or fp32) partial from TMEM, hands the pair back after its second read, converts the
//     partial exactly (int32 + 0x4B400000 reinterpreted, minus 1.5 * 2^23: exact for |p| < 2^22) and
//     folds it into 32 fp32 accumulators per thread with packed f32x2 multiply / FMA, while the tensor
//     core fills the other pair.
//   * per-row scales on both sides (PMODE 2): BN = 256, NBUF = 2, GPS = 1, two epilogue warpgroups (384
//     threads); the tensor core accumulates all of K in one accumulator and the epilogue streams it out of
//     TMEM in 32-column chunks, overlapped with the next tile's MMAs.
// After the last group: the per-row weight scale when it was factored out, + bias, then the epilogue of
// kernels.py:123-137 (cast / GELU / GELU + int8 requantization per 128 columns; the column quarters of
// a quantization group exchange their absmax through shared memory).
//
// Promotion arithmetic (the CPU oracle evaluates the same):
//   PMODE 0 (sw per row x group):  t = RN(p * sa[m,g]);  acc = fma(t, sw[n,g], acc)
//   PMODE 1 (sw per row or block):  acc = fma(p, s, acc) with s = sa[m,g] (sw per row, applied at the end)
//                                   or s = RN(sa[m,g] * swb[n/128,g]) (128x128 weight blocks)
//   PMODE 2 (both per row):         one accumulator over all K; y = RN(RN(float(D) * sa[m]) * sw[n])
//
// Every wait on an mbarrier is bounded (globaltimer); on expiry the kernel records HN_DEVERR_TIMEOUT,
// makes the other roles leave their loops, waits briefly for its own copies/MMAs in flight, frees TMEM
// and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "hn_common.cuh"
#include "hn_kernels.h"
#include "hn_tc.cuh"

namespace hn {

// Device error words (0 = ok), one per stream slot (err_slot() in capi.cu): a bounded wait that gives up ORs
// HN_DEVERR_* bits into the word of the stream its kernel was launched on, so a timeout is reported to the
// reader of that stream only. Each device holds its own copy of the array.
__device__ int g_device_error[HN_ERR_SLOTS];

cudaError_t device_error_word(int slot, int **ptr) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= HN_MAX_DEV) return cudaErrorInvalidDevice;
    // the array's device address, looked up once per device with that device current (in host code the
    // symbol name itself is only a host-side stand-in)
    static int *base[HN_MAX_DEV];
    if (base[dev] == nullptr) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_device_error);
        if (e != cudaSuccess) return e;
        base[dev] = static_cast<int *>(p);
    }
    *ptr = base[dev] + slot;
    return cudaSuccess;
}

cudaError_t read_and_clear_device_error(int slot, int *value) {
    int zero = 0;
    cudaError_t e = cudaMemcpyFromSymbol(value, g_device_error, sizeof(int), sizeof(int) * slot);
    if (e != cudaSuccess) return e;
    return cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int), sizeof(int) * slot);
}

namespace gemm {

constexpr int BM = 128, BK = 128;
constexpr int EPI_WARP0 = 4;  // warpgroup 0: producers, MMA issuer, scale ring; epilogue warpgroups follow
constexpr int SW_SLOTS = 8;   // scale-ring depth in groups (SW_SLOTS / 2 pair slots the producer runs ahead)
// K groups per pipeline stage (and per TMA request) for the 128-wide and the 256-wide tile
constexpr int GPS_NARROW = 2, GPS_WIDE = 1;
// epilogue warpgroups (column parts of a tile row): the per-group promotion modes hand every 128-column
// group over from TMEM, so more epilogue warps shorten that handoff; the whole-K mode reads TMEM once per
// tile and keeps two
constexpr int NPART_NARROW = 4, NPART_WIDE = 2;
constexpr int TMEM_COLS = 512;
constexpr uint64_t WAIT_NS = 2000000000ull;  // 2 s

template <int BN_, int GPS_, int NPART_> struct Cfg {
    static constexpr int BN = BN_;
    static constexpr int NPART = NPART_;                              // epilogue warpgroups
    static constexpr int EPI_WARPS = 4 * NPART;
    static constexpr int THREADS = 128 + 32 * EPI_WARPS;
    static constexpr int GPS = GPS_;                                  // K groups per pipeline stage
    static constexpr int A_GROUP = BM * BK;                           // bytes of one group's A tile
    static constexpr int B_GROUP = BN * BK;
    static constexpr int A_STAGE = GPS * A_GROUP;
    static constexpr int B_STAGE = GPS * B_GROUP;
    static constexpr int STAGES = (192 * 1024) / (A_STAGE + B_STAGE);  // 3 (BN 128, 2 groups) / 4 (BN 256, 1)
    static constexpr int NBUF = TMEM_COLS / BN;                       // 4 or 2 accumulators
    static constexpr int CPT = BN / NPART;                            // columns per epilogue thread
    static constexpr int PARTS_PER_GROUP = 128 / CPT;                 // parts sharing one quant group
    static constexpr int OFF_A = 0;
    static constexpr int OFF_B = OFF_A + STAGES * A_STAGE;
    // scale ring slot: activation scales of the tile's 128 rows, weight scales of its BN columns, and the
    // weight block scales of its BN / 128 column blocks (padded to 16 bytes)
    static constexpr int RING_SA = 0, RING_SW = 128, RING_SB = 128 + BN, RING_FLOATS = 128 + BN + 4;
    static constexpr int OFF_SW = OFF_B + STAGES * B_STAGE;           // float[SW_SLOTS][RING_FLOATS]
    static constexpr int OFF_PX = OFF_SW + SW_SLOTS * RING_FLOATS * 4; // float[2][NPART][128] absmax exchange
    static constexpr int OFF_BAR = OFF_PX + 2 * NPART * 128 * 4;
    static constexpr int NBARS = 2 * STAGES + 2 * NBUF + 2 * SW_SLOTS + 2;
    static constexpr int OFF_MISC = OFF_BAR + NBARS * 8;              // tmem base, abort flag
    static constexpr int SMEM = OFF_MISC + 16 + 1024;                 // + alignment slack
    static_assert(SMEM <= 232448, "shared memory budget");
};

struct Params {
    const float *sa; int64_t sa_rs, sa_gs; int sa_mode;
    const float *sw; int64_t sw_rs, sw_gs; int sw_mode;
    const void *bias; int bias_dtype;
    void *out; int64_t ldo; int out_dtype;
    float *qs; int64_t qs_rs, qs_gs;
    int *err;       // this launch's device error word (its stream's slot)
    int M, N, K, G;
    int n_blocks, num_tiles;
    int vec_store;
    int sw_vec;     // per-row weight scales contiguous and 16-byte aligned (vector loads)
    int sa_bulk;    // group activation scales group-major, 16-byte aligned: one bulk copy per group
    int sw_bulk;    // group weight scales group-major, 16-byte aligned
};

// ---------------------------------------------------------------------------------------------------
// PTX wrappers (hn_tc.cuh)
using namespace tc;

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

// int8 codes of CPT bf16-valued GELU outputs v(0..CPT-1) of one row's 128-column quantization group, scale sc = RN(peak /
// 127) (kernels.py:131-135): the quotients v / sc by the exact fma-corrected reciprocal of x2_quot (exact for bf16
// values |v| <= peak, checked exhaustively over the bf16 domain; IEEE division below 2^-90), rounded half away
// from zero, 16 codes per 16-byte store.
template <int CPT, typename V> __device__ __forceinline__ void store_codes(int8_t *qrow, V v, float sc) {
    const bool fast = sc >= 0x1p-90f;
    const uint64_t ns = x2_splat(-sc), rs = x2_splat(fast ? __frcp_rn(sc) : 1.0f);
#pragma unroll
    for (int j = 0; j < CPT; j += 16) {
        uint32_t c[16];
        if (fast) {
#pragma unroll
            for (int i = 0; i < 8; ++i) x2_codes(x2_quot(x2(v(j + 2 * i), v(j + 2 * i + 1)), ns, rs), c[2 * i], c[2 * i + 1]);
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i)
                x2_codes(x2(__fdiv_rn(v(j + 2 * i), sc), __fdiv_rn(v(j + 2 * i + 1), sc)), c[2 * i], c[2 * i + 1]);
        }
        *reinterpret_cast<uint4 *>(qrow + j) =
            make_uint4(pack4_lowbytes(c[0], c[1], c[2], c[3]), pack4_lowbytes(c[4], c[5], c[6], c[7]),
                       pack4_lowbytes(c[8], c[9], c[10], c[11]), pack4_lowbytes(c[12], c[13], c[14], c[15]));
    }
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

// ---------------------------------------------------------------------------------------------------
// epilogue output helpers

// store `n` consecutive results of one row (n a multiple of 8, 16-byte aligned destination)
template <int NV>
__device__ __forceinline__ void store_row_vec(void *out, int od, int64_t off, const float *v) {
    if (od == 0 || od == 1) {
        uint16_t *o16 = reinterpret_cast<uint16_t *>(out) + off;
#pragma unroll
        for (int j = 0; j < NV; j += 8) {
            uint4 o;
            uint32_t *ow = &o.x;
#pragma unroll
            for (int w = 0; w < 4; ++w)
                ow[w] = od == 0 ? pack_bf16_rn(v[j + 2 * w], v[j + 2 * w + 1]) : pack_f16_rn(v[j + 2 * w], v[j + 2 * w + 1]);
            *reinterpret_cast<uint4 *>(o16 + j) = o;
        }
    } else {
        uint32_t *o32 = reinterpret_cast<uint32_t *>(out) + off;
#pragma unroll
        for (int j = 0; j < NV; j += 4) {
            uint4 o = make_uint4(__float_as_uint(v[j]), __float_as_uint(v[j + 1]), __float_as_uint(v[j + 2]),
                                 __float_as_uint(v[j + 3]));
            *reinterpret_cast<uint4 *>(o32 + j) = o;
        }
    }
}
__device__ __forceinline__ void store_one(void *out, int od, int64_t off, float v) {
    if (od == 0) reinterpret_cast<__nv_bfloat16 *>(out)[off] = __float2bfloat16_rn(v);
    else if (od == 1) reinterpret_cast<__half *>(out)[off] = __float2half_rn(v);
    else reinterpret_cast<uint32_t *>(out)[off] = __float_as_uint(v);
}

// ---------------------------------------------------------------------------------------------------

template <int KIND, int PMODE, int EPI, int BN, int GPS, int NP>
__global__ void __launch_bounds__(128 + 128 * NP, 1)
    k_block_gemm(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const Params p) {
    using C = Cfg<BN, GPS, NP>;
    constexpr int STAGES = C::STAGES, NBUF = C::NBUF, CPT = C::CPT, NPART = C::NPART, EPI_WARPS = C::EPI_WARPS;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bar_full = sbase + C::OFF_BAR;
    const uint32_t bar_empty = bar_full + STAGES * 8;
    const uint32_t bar_tfull = bar_empty + STAGES * 8;
    const uint32_t bar_tempty = bar_tfull + NBUF * 8;
    const uint32_t bar_sfull = bar_tempty + NBUF * 8;
    const uint32_t bar_sempty = bar_sfull + SW_SLOTS * 8;
    const uint32_t bar_px = bar_sempty + SW_SLOTS * 8;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + C::OFF_MISC);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + C::OFF_MISC + 4);
    float *sw_s = reinterpret_cast<float *>(smem + C::OFF_SW);
    float *px_s = reinterpret_cast<float *>(smem + C::OFF_PX);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = p.G;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(bar_full + 8 * s, 2);   // the A and the B producer each arm it
            mbar_init(bar_empty + 8 * s, 1);
        }
        for (int b = 0; b < NBUF; ++b) {
            mbar_init(bar_tfull + 8 * b, 1);
            mbar_init(bar_tempty + 8 * b, EPI_WARPS);
        }
        for (int s = 0; s < SW_SLOTS; ++s) {
            mbar_init(bar_sfull + 8 * s, 1);
            mbar_init(bar_sempty + 8 * s, EPI_WARPS);
        }
        mbar_init(bar_px, EPI_WARPS);
        mbar_init(bar_px + 8, EPI_WARPS);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 0 && lane == 0) asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmA) : "memory");
    if (warp == 2 && lane == 0) asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmB) : "memory");
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

    if (warp == 0 || warp == 2) {
        // ------------------------------------------------------------------ producers: A tiles (warp 0), B tiles
        // (warp 2). TMA requests issued by one thread are processed one after another, so the two operands
        // come from two issuing warps; each arms the stage's full barrier with its own byte count.
        const bool is_a = warp == 0;
        int stage = 0;
        uint32_t phase = 0;
        int issued = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
            const int m0 = (tile / p.n_blocks) * BM, n0 = (tile % p.n_blocks) * BN;
            for (int g0 = 0; g0 < G; g0 += GPS) {
                ok = warp_wait(lane, bar_empty + 8 * stage, phase ^ 1, abort_flag, WAIT_NS, p.err);
                if (!ok) break;
                if (lane == 0) {
                    // a box that runs past the last group is zero-filled and still counts its full bytes
                    const uint32_t fb = bar_full + 8 * stage;
                    if (is_a) {
                        mbar_arrive_tx(fb, C::A_STAGE);
                        tma_load_3d(&tmA, sbase + C::OFF_A + stage * C::A_STAGE, fb, m0, g0);
                    } else {
                        mbar_arrive_tx(fb, C::B_STAGE);
                        tma_load_3d(&tmB, sbase + C::OFF_B + stage * C::B_STAGE, fb, n0, g0);
                    }
                }
                ++issued;
                if (++stage == STAGES) { stage = 0; phase ^= 1; }
            }
        }
        // drain: the last copies issued land before the CTA can exit
        int st = stage;
        uint32_t ph = phase;
        for (int i = 0; i < STAGES && i < issued; ++i) {
            if (--st < 0) { st = STAGES - 1; ph ^= 1; }
            volatile int never = 0;
            mbar_wait(bar_full + 8 * st, ph, &never, 100000000ull, p.err);
        }
    } else if (warp == 3) {
        // ------------------------------------------------------------------ scale ring (PMODE 0, 1)
        // Per pair of K groups (one pipeline stage): the activation scales of the tile's rows, the weight
        // scales of its columns (group mode) or of its 128-column blocks (block mode), for both groups, in two
        // consecutive slots that complete on one barrier. Group-major scales arrive by bulk copies; other
        // layouts are gathered with 4-byte cp.async copies.
        if (PMODE != 2) {
            static_assert(PMODE == 2 || GPS == 2, "per-group promotion hands over K groups in pairs (GPS == 2)");
            int ps = 0, issued = 0;
            uint32_t sphase = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
                const int m0 = (tile / p.n_blocks) * BM, n0 = (tile % p.n_blocks) * BN;
                const int rows = min(BM, p.M - m0), cols = min(BN, p.N - n0);
                for (int g0 = 0; g0 < G; g0 += 2) {
                    ok = warp_wait(lane, bar_sempty + 8 * ps, sphase ^ 1, abort_flag, WAIT_NS, p.err);
                    if (!ok) break;
                    const int ng = min(2, G - g0);
                    const bool sa_grp = p.sa_mode == 0, sw_grp = PMODE == 0, sw_blk = PMODE == 1 && p.sw_mode == 2;
                    // bulk copies move whole 16-byte units: a tile whose row (column) count is not a multiple
                    // of 4 - only the last one can be - gathers its scales so nothing past the end is read
                    const bool sa_bulk = p.sa_bulk && (rows & 3) == 0, sw_bulk = p.sw_bulk && (cols & 3) == 0;
                    // gathers are cp.async copies that complete on the pair's barrier, so the warp moves on to
                    // the next pair without waiting for their latency
                    for (int gi = 0; gi < ng; ++gi) {
                        const int g = g0 + gi;
                        const uint32_t rbase = smem_u32(sw_s + (2 * ps + gi) * C::RING_FLOATS);
                        if (sa_grp && !sa_bulk) {
#pragma unroll
                            for (int i = 0; i < BM / 32; ++i) {
                                const int r = lane + 32 * i;
                                const bool v = r < rows;
                                cp_async4(rbase + 4 * (C::RING_SA + r),
                                          v ? p.sa + (int64_t)(m0 + r) * p.sa_rs + (int64_t)g * p.sa_gs : p.sa, v);
                            }
                        }
                        if (sw_grp && !sw_bulk) {
#pragma unroll
                            for (int i = 0; i < BN / 32; ++i) {
                                const int c = lane + 32 * i;
                                const bool v = c < cols;
                                cp_async4(rbase + 4 * (C::RING_SW + c),
                                          v ? p.sw + (int64_t)(n0 + c) * p.sw_rs + (int64_t)g * p.sw_gs : p.sw, v);
                            }
                        }
                        if (sw_blk && lane < BN / 128) {
                            const int nb = n0 / 128 + lane;
                            const bool v = nb * 128 < p.N;
                            cp_async4(rbase + 4 * (C::RING_SB + lane), v ? p.sw + (int64_t)nb * p.sw_rs + (int64_t)g * p.sw_gs : p.sw, v);
                        }
                    }
                    if ((sa_grp && !sa_bulk) || (sw_grp && !sw_bulk) || sw_blk) cp_async_arrive(bar_sfull + 8 * ps);
                    __syncwarp();
                    if (lane == 0) {
                        const uint32_t sa_bytes = (sa_grp && sa_bulk) ? (uint32_t)(rows * 4) : 0u;
                        const uint32_t sw_bytes = (sw_grp && sw_bulk) ? (uint32_t)(cols * 4) : 0u;
                        const uint32_t bytes = (uint32_t)ng * (sa_bytes + sw_bytes);
                        const uint32_t fb = bar_sfull + 8 * ps;
                        if (bytes) mbar_arrive_tx(fb, bytes);
                        else mbar_arrive(fb);
                        for (int gi = 0; gi < ng; ++gi) {
                            const int g = g0 + gi;
                            const uint32_t rbase = smem_u32(sw_s + (2 * ps + gi) * C::RING_FLOATS);
                            if (sa_bytes) bulk_load(rbase + 4 * C::RING_SA, p.sa + (int64_t)g * p.sa_gs + m0, sa_bytes, fb);
                            if (sw_bytes) bulk_load(rbase + 4 * C::RING_SW, p.sw + (int64_t)g * p.sw_gs + n0, sw_bytes, fb);
                        }
                    }
                    ++issued;
                    if (++ps == SW_SLOTS / 2) { ps = 0; sphase ^= 1; }
                }
            }
            // drain: the last bulk copies land before the CTA can exit
            int st = ps;
            uint32_t ph = sphase;
            for (int i = 0; i < SW_SLOTS / 2 && i < issued; ++i) {
                if (--st < 0) { st = SW_SLOTS / 2 - 1; ph ^= 1; }
                volatile int never = 0;
                if (lane == 0) mbar_wait(bar_sfull + 8 * st, ph, &never, 100000000ull, p.err);
            }
            __syncwarp();
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------------ MMA issuer
        const uint32_t idesc = KIND == 0
                                   ? ((2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24))
                                   : ((1u << 4) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24));
        int stage = 0, tb = 0;
        uint32_t phase = 0, tphase = 0;
        bool ok = true;
        int last_stage = -1;
        uint32_t last_phase = 0;
        for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
            if (PMODE == 2) {
                ok = warp_wait(lane, bar_tempty + 8 * tb, tphase ^ 1, abort_flag, WAIT_NS, p.err);
                if (!ok) break;
                tc_fence_after();
            }
            for (int g0 = 0; g0 < G && ok; g0 += GPS) {
                ok = warp_wait(lane, bar_full + 8 * stage, phase, abort_flag, WAIT_NS, p.err);
                if (!ok) break;
                if (PMODE != 2) {
                    // per-group promotion: the stage's two groups go to the two accumulators of TMEM pair tb
                    // (NBUF / 2 pairs), handed over with one barrier each way
                    ok = warp_wait(lane, bar_tempty + 8 * tb, tphase ^ 1, abort_flag, WAIT_NS, p.err);
                    if (!ok) break;
                }
                tc_fence_after();
                if (lane == 0) {
#pragma unroll
                    for (int gi = 0; gi < GPS; ++gi) {
                        const int g = g0 + gi;
                        if (g >= G) break;
                        const uint32_t d = tmem_base + (uint32_t)(((PMODE != 2) ? (2 * tb + gi) : tb) * BN);
                        const uint64_t ad = sdesc(sbase + C::OFF_A + stage * C::A_STAGE + gi * C::A_GROUP);
                        const uint64_t bd = sdesc(sbase + C::OFF_B + stage * C::B_STAGE + gi * C::B_GROUP);
#pragma unroll
                        for (int k = 0; k < BK / 32; ++k)
                            mma_128xNx32<KIND>(d, ad + 2 * k, bd + 2 * k, idesc,
                                               (PMODE == 2) ? (uint32_t)(g > 0 || k > 0) : (uint32_t)(k > 0));
                    }
                    if (PMODE != 2) mma_commit(bar_tfull + 8 * tb);
                }
                __syncwarp();
                if (PMODE != 2) { if (++tb == NBUF / 2) { tb = 0; tphase ^= 1; } }
                if (lane == 0) mma_commit(bar_empty + 8 * stage);
                __syncwarp();
                last_stage = stage;
                last_phase = phase;
                if (++stage == STAGES) { stage = 0; phase ^= 1; }
            }
            if (PMODE == 2 && ok) {
                if (lane == 0) mma_commit(bar_tfull + 8 * tb);
                __syncwarp();
                if (++tb == NBUF) { tb = 0; tphase ^= 1; }
            }
        }
        // drain: the MMAs behind the last commit finish before TMEM is released
        if (last_stage >= 0) {
            volatile int never = 0;
            mbar_wait(bar_empty + 8 * last_stage, last_phase, &never, 100000000ull, p.err);
        }
    } else if (warp >= EPI_WARP0) {
        // ------------------------------------------------------------------ epilogue
        const int ew = warp - EPI_WARP0;
        const int q = warp & 3;
        const int hf = ew >> 2;  // column part 0..NPART-1
        const int row = q * 32 + lane;
        const uint32_t lane_addr = tmem_base + ((uint32_t)(q * 32) << 16);
        int tb = 0, slot = 0, it = 0;
        uint32_t tphase = 0, sphase = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x, ++it) {
            const int m0 = (tile / p.n_blocks) * BM, n0 = (tile % p.n_blocks) * BN;
            const int m = m0 + row;
            const int mm = m < p.M ? m : p.M - 1;
            const int ncol0 = n0 + hf * CPT;
            const bool row_ok = m < p.M;
            const bool full_cols = ncol0 + CPT <= p.N;
            const int od = (EPI == 1) ? 0 : p.out_dtype;
            if (PMODE != 2) {
                // ------------------------------------------------ per-group promotion into registers
                static_assert(PMODE == 2 || CPT == 32 || CPT == 64, "per-group promotion: 32 or 64 columns a thread");
                uint64_t acc[CPT / 2];
#pragma unroll
                for (int i = 0; i < CPT / 2; ++i) acc[i] = 0ull;
                const float sa_row = (p.sa_mode == 1) ? p.sa[(int64_t)mm * p.sa_rs] : 0.0f;
                for (int g0 = 0; g0 < G; g0 += 2) {
                    // one pair of K groups: its scales (pair slot ps) and its two accumulators (TMEM pair tb)
                    const int ng = min(2, G - g0);
                    ok = warp_wait(lane, bar_sfull + 8 * slot, sphase, abort_flag, WAIT_NS, p.err);
                    if (!ok) break;
                    // (row-scale mode) the pair's scales into registers before the accumulators are waited for,
                    // so the shared-memory latency hides behind the wait
                    float s_pair[2] = {0.0f, 0.0f};
#pragma unroll
                    for (int gi = 0; gi < 2 && PMODE == 1; ++gi) {
                        const float *ring = sw_s + (2 * slot + gi) * C::RING_FLOATS;
                        const float sa_g = (p.sa_mode == 0) ? ring[C::RING_SA + row] : sa_row;
                        s_pair[gi] = sa_g;
                        if (p.sw_mode == 2)
                            s_pair[gi] = (ncol0 < p.N) ? __fmul_rn(sa_g, ring[C::RING_SB + (hf * CPT) / 128]) : 0.0f;
                    }
                    ok = warp_wait(lane, bar_tfull + 8 * tb, tphase, abort_flag, WAIT_NS, p.err);
                    if (!ok) break;
                    tc_fence_after();
                    // group by group: the partials out of TMEM (after the pair's last read the pair goes back to the
                    // tensor core), then folded in from registers
#pragma unroll
                    for (int gi = 0; gi < 2; ++gi) {
                        if (gi >= ng) break;
                        uint32_t r[CPT];
#pragma unroll
                        for (int c = 0; c < CPT / 32; ++c)
                            tmem_ld32(lane_addr + (uint32_t)((2 * tb + gi) * BN + hf * CPT + 32 * c),
                                      *reinterpret_cast<uint32_t(*)[32]>(r + 32 * c));
                        if (gi == ng - 1) {
                            tc_fence_before();
                            __syncwarp();
                            if (lane == 0) mbar_arrive(bar_tempty + 8 * tb);
                        }
                        const float *ring = sw_s + (2 * slot + gi) * C::RING_FLOATS;
                        const float s_g = (PMODE == 1) ? s_pair[gi] : ((p.sa_mode == 0) ? ring[C::RING_SA + row] : sa_row);
                        const uint64_t s2 = pk(s_g, s_g);
                        const float *sws = ring + C::RING_SW + hf * CPT;
#pragma unroll
                        for (int j = 0; j < CPT; j += 4) {
                            if (PMODE == 0) {
                                const float4 w4 = *reinterpret_cast<const float4 *>(sws + j);
                                promote_gen<KIND>(acc[j / 2], r[j], r[j + 1], s2, pk(w4.x, w4.y));
                                promote_gen<KIND>(acc[j / 2 + 1], r[j + 2], r[j + 3], s2, pk(w4.z, w4.w));
                            } else {
                                promote_row<KIND>(acc[j / 2], r[j], r[j + 1], s2);
                                promote_row<KIND>(acc[j / 2 + 1], r[j + 2], r[j + 3], s2);
                            }
                        }
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(bar_sempty + 8 * slot);
                    if (++tb == NBUF / 2) { tb = 0; tphase ^= 1; }
                    if (++slot == SW_SLOTS / 2) { slot = 0; sphase ^= 1; }
                }
                if (!ok) break;
                float v[CPT];
#pragma unroll
                for (int i = 0; i < CPT / 2; ++i) { v[2 * i] = acc_lo(acc[i]); v[2 * i + 1] = acc_hi(acc[i]); }
                if (PMODE == 1 && p.sw_mode == 1) {
                    if (full_cols && p.sw_vec) {
#pragma unroll
                        for (int j = 0; j < CPT; j += 4) {
                            const float4 w4 = *reinterpret_cast<const float4 *>(p.sw + ncol0 + j);
                            v[j] = __fmul_rn(v[j], w4.x);
                            v[j + 1] = __fmul_rn(v[j + 1], w4.y);
                            v[j + 2] = __fmul_rn(v[j + 2], w4.z);
                            v[j + 3] = __fmul_rn(v[j + 3], w4.w);
                        }
                    } else {
#pragma unroll
                        for (int j = 0; j < CPT; ++j) v[j] = __fmul_rn(v[j], (ncol0 + j < p.N) ? p.sw[(int64_t)(ncol0 + j) * p.sw_rs] : 0.0f);
                    }
                }
                if (p.bias != nullptr) {
#pragma unroll
                    for (int j = 0; j < CPT; j += 8) {
                        float b[8];
                        if (full_cols) load_bias8(p.bias, p.bias_dtype, ncol0 + j, b);
                        else {
#pragma unroll
                            for (int i = 0; i < 8; ++i)
                                b[i] = (ncol0 + j + i < p.N) ? load_bias1(p.bias, p.bias_dtype, ncol0 + j + i) : 0.0f;
                        }
#pragma unroll
                        for (int i = 0; i < 8; ++i) v[j + i] = __fadd_rn(v[j + i], b[i]);
                    }
                }
                if (EPI != 0) {
#pragma unroll
                    for (int j = 0; j < CPT; j += 2) gelu_bf16_pair(v[j], v[j + 1]);
                }
                if (EPI == 2) {
                    // absmax over the 128-column group: this thread's 64 columns + the other half's
                    float peak = 0.0f;
#pragma unroll
                    for (int j = 0; j < CPT; j += 2) peak = absmax3(peak, v[j], v[j + 1]);
                    const int pb = it & 1;
                    px_s[(pb * NPART + hf) * 128 + row] = peak;
                    __syncwarp();
                    if (lane == 0) mbar_arrive(bar_px + 8 * pb);
                    ok = warp_wait(lane, bar_px + 8 * pb, (it >> 1) & 1, abort_flag, WAIT_NS, p.err);
                    if (!ok) break;
                    const int first = hf - hf % C::PARTS_PER_GROUP;
#pragma unroll
                    for (int o = 0; o < C::PARTS_PER_GROUP; ++o) peak = fmaxf(peak, px_s[(pb * NPART + first + o) * 128 + row]);
                    const float sc = i8_scale_bf16(peak);   // peak of bf16 GELU outputs
                    if (row_ok && full_cols) {
                        int8_t *qrow = static_cast<int8_t *>(p.out) + (int64_t)m * p.ldo + ncol0;
                        store_codes<CPT>(qrow, [&](int j) { return v[j]; }, sc);
                        if (hf % C::PARTS_PER_GROUP == 0) p.qs[(int64_t)m * p.qs_rs + (int64_t)(ncol0 >> 7) * p.qs_gs] = sc;
                    }
                } else if (row_ok) {
                    if (full_cols && p.vec_store) store_row_vec<CPT>(p.out, od, (int64_t)m * p.ldo + ncol0, v);
                    else {
#pragma unroll
                        for (int j = 0; j < CPT; ++j)
                            if (ncol0 + j < p.N) store_one(p.out, od, (int64_t)m * p.ldo + ncol0 + j, v[j]);
                    }
                }
            } else {
                // ------------------------------------------------ whole-K accumulator, streamed from TMEM
                ok = warp_wait(lane, bar_tfull + 8 * tb, tphase, abort_flag, WAIT_NS, p.err);
                if (!ok) break;
                tc_fence_after();
                const uint32_t tcol = lane_addr + (uint32_t)(tb * BN + hf * CPT);
                const float sam = p.sa[(int64_t)mm * p.sa_rs];
                const bool raw = (p.out_dtype == 3);
                uint32_t hpk[EPI == 2 ? CPT / 2 : 1];
                float peak = 0.0f;
#pragma unroll
                for (int c = 0; c < CPT / 32; ++c) {
                    uint32_t r[32];
                    tmem_ld32(tcol + c * 32, r);
                    float v[32];
                    const int nc = ncol0 + c * 32;
                    const bool chunk_full = nc + 32 <= p.N;
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        if (raw) { v[j] = __uint_as_float(r[j]); continue; }
                        const float w = (nc + j < p.N) ? p.sw[(int64_t)(nc + j) * p.sw_rs] : 0.0f;
                        const float d = KIND == 0 ? __int2float_rn((int)r[j]) : __uint_as_float(r[j]);
                        v[j] = __fmul_rn(__fmul_rn(d, sam), w);
                    }
                    if (p.bias != nullptr && !raw) {
#pragma unroll
                        for (int j = 0; j < 32; j += 8) {
                            float b[8];
                            if (chunk_full) load_bias8(p.bias, p.bias_dtype, nc + j, b);
                            else {
#pragma unroll
                                for (int i = 0; i < 8; ++i)
                                    b[i] = (nc + j + i < p.N) ? load_bias1(p.bias, p.bias_dtype, nc + j + i) : 0.0f;
                            }
#pragma unroll
                            for (int i = 0; i < 8; ++i) v[j + i] = __fadd_rn(v[j + i], b[i]);
                        }
                    }
                    if (EPI != 0) {
#pragma unroll
                        for (int j = 0; j < 32; j += 2) gelu_bf16_pair(v[j], v[j + 1]);
                    }
                    if (EPI == 2) {
#pragma unroll
                        for (int j = 0; j < 32; j += 2) {
                            peak = absmax3(peak, v[j], v[j + 1]);
                            hpk[c * 16 + j / 2] = pack_bf16_exact(v[j], v[j + 1]);
                        }
                    } else if (row_ok) {
                        if (chunk_full && p.vec_store) store_row_vec<32>(p.out, od, (int64_t)m * p.ldo + nc, v);
                        else {
#pragma unroll
                            for (int j = 0; j < 32; ++j)
                                if (nc + j < p.N) store_one(p.out, od, (int64_t)m * p.ldo + nc + j, v[j]);
                        }
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(bar_tempty + 8 * tb);
                if (++tb == NBUF) { tb = 0; tphase ^= 1; }
                if (EPI == 2) {
                    // absmax over the 128-column group shared by PARTS_PER_GROUP column parts
                    const int pb = it & 1;
                    px_s[(pb * NPART + hf) * 128 + row] = peak;
                    __syncwarp();
                    if (lane == 0) mbar_arrive(bar_px + 8 * pb);
                    ok = warp_wait(lane, bar_px + 8 * pb, (it >> 1) & 1, abort_flag, WAIT_NS, p.err);
                    if (!ok) break;
                    const int first = hf - hf % C::PARTS_PER_GROUP;
#pragma unroll
                    for (int o = 0; o < C::PARTS_PER_GROUP; ++o) peak = fmaxf(peak, px_s[(pb * NPART + first + o) * 128 + row]);
                }
                if (EPI == 2 && row_ok && full_cols) {
                    const float sc = i8_scale_bf16(peak);   // peak of bf16 GELU outputs
                    int8_t *qrow = static_cast<int8_t *>(p.out) + (int64_t)m * p.ldo + ncol0;
                    store_codes<CPT>(qrow, [&](int j) { return j & 1 ? bf16_hi(hpk[j >> 1]) : bf16_lo(hpk[j >> 1]); }, sc);
                    if (hf % C::PARTS_PER_GROUP == 0) p.qs[(int64_t)m * p.qs_rs + (int64_t)(ncol0 >> 7) * p.qs_gs] = sc;
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
// A row-major byte matrix [rows, cols] (row pitch ld bytes, cols % 128 == 0) seen as 3-D
// {128 bytes within a K group, row, K group}; box = {128, box_rows, box_groups}, 128B swizzle (the UMMA
// SWIZZLE_128B K-major layout, one [box_rows][128 B] tile per group), zero fill outside the matrix.
static bool make_map(CUtensorMap *map, const void *base, uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_rows,
                     uint32_t box_groups) {
    PFN_cuTensorMapEncodeTiled_v12000 fn = encode_fn();
    if (fn == nullptr) return false;
    cuuint64_t dims[3] = {128, rows, cols / 128};
    cuuint64_t strides[2] = {ld, 128};
    cuuint32_t box[3] = {128, box_rows, box_groups};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void *>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

template <int KIND, int PMODE, int EPI, int BN, int GPS, int NP>
static cudaError_t launch_t(const CUtensorMap &ma, const CUtensorMap &mb, const Params &p, int grid, cudaStream_t st) {
    using C = Cfg<BN, GPS, NP>;
    auto kern = k_block_gemm<KIND, PMODE, EPI, BN, GPS, NP>;
    // the shared-memory opt-in is a per-device property of the function: set it once per instantiation and
    // device (setting it twice, e.g. by two threads at once, is harmless)
    static bool configured[HN_MAX_DEV];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= HN_MAX_DEV) return cudaErrorInvalidDevice;
    if (!configured[dev]) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
        if (e != cudaSuccess) return e;
        configured[dev] = true;
    }
    kern<<<grid, C::THREADS, C::SMEM, st>>>(ma, mb, p);
    return cudaGetLastError();
}

template <int KIND, int PMODE, int BN, int GPS, int NP>
static cudaError_t launch_epi(int epi, const CUtensorMap &ma, const CUtensorMap &mb, const Params &p, int grid,
                              cudaStream_t st) {
    switch (epi) {
    case 0: return launch_t<KIND, PMODE, 0, BN, GPS, NP>(ma, mb, p, grid, st);
    case 1: return launch_t<KIND, PMODE, 1, BN, GPS, NP>(ma, mb, p, grid, st);
    default: return launch_t<KIND, PMODE, 2, BN, GPS, NP>(ma, mb, p, grid, st);
    }
}

} // namespace gemm

cudaError_t launch_block_gemm(const GemmArgs &a, cudaStream_t st, const char **msg) {
    using namespace gemm;
    if (gemv_applies(a)) return launch_gemv(a, st);
    int *err = nullptr;
    cudaError_t ee = device_error_word(err_slot(st), &err);
    if (ee != cudaSuccess) return ee;
    int pmode;
    if (a.sa_mode == 1 && a.sw_mode == 1) pmode = 2;
    else if (a.sw_mode == 0) pmode = 0;
    else pmode = 1;
    const int bn = pmode == 2 ? 256 : 128;
    const int gps = pmode == 2 ? GPS_WIDE : GPS_NARROW;
    CUtensorMap ma, mb;
    if (!make_map(&ma, a.qa, (uint64_t)a.M, (uint64_t)a.K, (uint64_t)a.lda, BM, (uint32_t)gps) ||
        !make_map(&mb, a.qw, (uint64_t)a.N, (uint64_t)a.K, (uint64_t)a.ldw, (uint32_t)bn, (uint32_t)gps)) {
        *msg = "cuTensorMapEncodeTiled failed (pointer/stride alignment or driver entry point)";
        return cudaErrorInvalidValue;
    }
    Params p;
    p.sa = a.sa; p.sa_rs = a.sa_rs; p.sa_gs = a.sa_gs; p.sa_mode = a.sa_mode;
    p.sw = a.sw; p.sw_rs = a.sw_rs; p.sw_gs = a.sw_gs; p.sw_mode = a.sw_mode;
    p.bias = a.bias; p.bias_dtype = a.bias_dtype;
    p.out = a.out; p.ldo = a.ldo; p.out_dtype = a.out_dtype;
    p.qs = a.qs; p.qs_rs = a.qs_rs; p.qs_gs = a.qs_gs;
    p.err = err;
    p.M = (int)a.M; p.N = (int)a.N; p.K = (int)a.K; p.G = (int)(a.K / 128);
    p.n_blocks = (int)cdiv(a.N, bn);
    p.num_tiles = (int)(cdiv(a.M, BM) * p.n_blocks);
    const int esz = (a.epilogue == 2) ? 1 : (a.out_dtype == 0 || a.out_dtype == 1) ? 2 : 4;
    p.vec_store = ((reinterpret_cast<uintptr_t>(a.out) % 16) == 0 && (a.ldo * esz) % 16 == 0) ? 1 : 0;
    p.sw_vec = (reinterpret_cast<uintptr_t>(a.sw) % 16) == 0 && a.sw_rs == 1 ? 1 : 0;
    // bulk copies of one group's scales: group-major with 16-byte aligned group rows (a tile with a row
    // count that is not a multiple of 4 gathers instead, in the kernel)
    p.sa_bulk = (a.sa_mode == 0 && a.sa_rs == 1 && a.sa_gs % 4 == 0 &&
                 reinterpret_cast<uintptr_t>(a.sa) % 16 == 0) ? 1 : 0;
    p.sw_bulk = (a.sw_mode == 0 && a.sw_rs == 1 && a.sw_gs % 4 == 0 &&
                 reinterpret_cast<uintptr_t>(a.sw) % 16 == 0) ? 1 : 0;
    int grid = num_sms() - a.sm_reserve;
    if (grid > p.num_tiles) grid = p.num_tiles;
    if (a.kind == 0) {
        if (pmode == 0) return launch_epi<0, 0, 128, GPS_NARROW, NPART_NARROW>(a.epilogue, ma, mb, p, grid, st);
        if (pmode == 1) return launch_epi<0, 1, 128, GPS_NARROW, NPART_NARROW>(a.epilogue, ma, mb, p, grid, st);
        return launch_epi<0, 2, 256, GPS_WIDE, NPART_WIDE>(a.epilogue, ma, mb, p, grid, st);
    }
    if (pmode == 0) return launch_epi<1, 0, 128, GPS_NARROW, NPART_NARROW>(a.epilogue, ma, mb, p, grid, st);
    if (pmode == 1) return launch_epi<1, 1, 128, GPS_NARROW, NPART_NARROW>(a.epilogue, ma, mb, p, grid, st);
    return launch_epi<1, 2, 256, GPS_WIDE, NPART_WIDE>(a.epilogue, ma, mb, p, grid, st);
}

// ---------------------------------------------------------------------------------------------------
// Bounded-wait self-test: one CTA waits on an mbarrier that nothing completes, with a short limit.
__global__ void k_wait_selftest(uint64_t limit_ns, int *err) {
    __shared__ __align__(8) uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        gemm::mbar_init(gemm::smem_u32(&bar), 1);
        abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    if (threadIdx.x == 0) gemm::mbar_wait(gemm::smem_u32(&bar), 0, &abort_flag, limit_ns, err);
    __syncthreads();
}

cudaError_t launch_wait_selftest(uint32_t timeout_us, cudaStream_t st) {
    int *err = nullptr;
    cudaError_t e = device_error_word(err_slot(st), &err);
    if (e != cudaSuccess) return e;
    k_wait_selftest<<<1, 32, 0, st>>>((uint64_t)timeout_us * 1000ull, err);
    return cudaGetLastError();
}

} // namespace hn
