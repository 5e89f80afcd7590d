// attention.cu - the DiT's attention (hy_nomas/model.py:145-151: softmax(q k^T * scale) v per batch item and
// head, no mask, head dim 128, bf16 in and out) on the sm_100a tensor cores, with an optional fused int8
// quantization of the output for the projection linear that follows it (the per-token x 128-channel quantizer
// of kernels.py:22-54 applied to the [tokens, heads * 128] output: one 128-channel group is one head's row).
//
// One CTA computes QT = 2 query tiles of 128 rows of one (batch, head) against all keys, 64 keys per step:
//   warp 0      TMA producer: both Q tiles once, then K and V tiles of 64 keys (5-D maps {64 elements, row,
//               2 halves of the head dim, head, batch}, 128B swizzle, no multicast) into a ring of STAGES.
//   warp 1      MMA issuer (one thread): S_t(j) = Q_t K_j^T into a double-buffered 64-column TMEM tile per query
//               tile, and O_t += P_t(j) V_j into a 128-column TMEM accumulator (P from shared memory, K-major; V
//               read MN-major straight from its TMA tile). S of the next key step is issued before the P V of the
//               current one, so the tensor core works while the softmax warps do.
//   warps 4-11  softmax, one warpgroup per query tile, one thread per query row (its TMEM lane): reads its S row,
//               keeps a running maximum m (base-2 logits) and sum l, writes P = 2^(s * scale * log2 e - m) as bf16
//               into the swizzled P tile, and rescales its O row in TMEM only when the maximum grew by more than
//               2^8 (a stale maximum leaves every P <= 2^8: exact in fp32 and bf16 range). After the last step:
//               O / l -> bf16 rows (and the int8 codes + scale of each row).
// TMEM: S[t][b] at columns (2t + b) * 64, O[t] at 256 + 128 t (512 columns, one CTA per SM).
// Every mbarrier wait is bounded (globaltimer); on expiry the kernel records HN_DEVERR_TIMEOUT, the other roles
// leave their loops, the copies and MMAs in flight are drained (bounded) and TMEM is freed.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "hn_common.cuh"
#include "hn_kernels.h"
#include "hn_tc.cuh"

namespace hn {
namespace attn {
using namespace tc;

constexpr int BQ = 128;                 // query rows per tile (TMEM lanes)
constexpr int BKV = 64;                 // keys per step
constexpr int HD = 128;                 // head dim
constexpr int QT = 2;                   // query tiles per CTA
constexpr int STAGES = 3;               // K/V ring
constexpr int SM_WARP0 = 4;             // first softmax warp
constexpr int THREADS = 32 * (SM_WARP0 + 4 * QT);
constexpr int Q_HALF = BQ * 128;        // [128 rows][128 B]: one half (64 elements) of the head dim
constexpr int Q_TILE = 2 * Q_HALF;
constexpr int KV_HALF = BKV * 128;      // [64 rows][128 B]
constexpr int KV_TILE = 2 * KV_HALF;
constexpr int P_TILE = BQ * BKV * 2;    // [128 rows][64 keys] bf16: one 128 B swizzled row per query
constexpr int OFF_Q = 0;
constexpr int OFF_K = OFF_Q + QT * Q_TILE;
constexpr int OFF_V = OFF_K + STAGES * KV_TILE;
constexpr int OFF_P = OFF_V + STAGES * KV_TILE;
constexpr int OFF_BAR = OFF_P + QT * 2 * P_TILE;
// q_full, k_full[S], v_full[S], kv_empty[S], s_full[QT][2], s_free[QT][2], p_full[QT][2], pv_done[QT][2], drain
constexpr int NBARS = 1 + 3 * STAGES + 8 * QT + 1;
constexpr int OFF_MISC = OFF_BAR + NBARS * 8;
constexpr int SMEM = OFF_MISC + 16 + 1024;
static_assert(SMEM <= 232448, "shared memory budget");
constexpr uint32_t TMEM_COLS = 512;
constexpr int O_COL = 256;
constexpr uint64_t WAIT_NS = 2000000000ull;   // 2 s

struct Params {
    int Lq, Lk, H;
    float sl2;                                  // softmax scale * log2(e)
    __nv_bfloat16 *out; int64_t o_rs, o_hs, o_bs;   // elements; out may be null when only codes are wanted
    int8_t *q8; float *s8;                      // [B*Lq, H*128] codes and [B*Lq, H] scales, or null
    int *err;
};

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// bf16 values of 32 consecutive output columns of this thread's row: rbf16(o * inv)
__device__ __forceinline__ void out_chunk(const uint32_t (&o)[32], float inv, float (&v)[32]) {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = rbf16(__fmul_rn(__uint_as_float(o[i]), inv));
}

__global__ void __launch_bounds__(THREADS, 1)
    k_attention(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                const __grid_constant__ CUtensorMap tmV, const Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bar_q = sbase + OFF_BAR;
    const uint32_t bar_kf = bar_q + 8;
    const uint32_t bar_vf = bar_kf + 8 * STAGES;
    const uint32_t bar_ke = bar_vf + 8 * STAGES;
    const uint32_t bar_sf = bar_ke + 8 * STAGES;
    const uint32_t bar_sr = bar_sf + 8 * 2 * QT;
    const uint32_t bar_pf = bar_sr + 8 * 2 * QT;
    const uint32_t bar_pv = bar_pf + 8 * 2 * QT;
    const uint32_t bar_end = bar_pv + 8 * 2 * QT;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + OFF_MISC);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + OFF_MISC + 4);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q0 = blockIdx.x * (QT * BQ), h = blockIdx.y, b = blockIdx.z;
    const int n = (p.Lk + BKV - 1) / BKV;

    if (threadIdx.x == 0) {
        mbar_init(bar_q, 1);
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(bar_kf + 8 * s, 1);
            mbar_init(bar_vf + 8 * s, 1);
            mbar_init(bar_ke + 8 * s, 1);
        }
        for (int i = 0; i < 2 * QT; ++i) {
            mbar_init(bar_sf + 8 * i, 1);
            mbar_init(bar_sr + 8 * i, 4);     // the four warps of the query tile's softmax warpgroup
            mbar_init(bar_pf + 8 * i, 4);
            mbar_init(bar_pv + 8 * i, 1);
        }
        mbar_init(bar_end, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 0 && lane == 0) {
        asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmQ) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmK) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmV) : "memory");
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
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------------------------ TMA producer
        if (lane == 0) {
            mbar_arrive_tx(bar_q, QT * Q_TILE);      // rows past Lq are zero-filled and still count
            for (int t = 0; t < QT; ++t) tma_load_5d(&tmQ, sbase + OFF_Q + t * Q_TILE, bar_q, 0, q0 + t * BQ, 0, h, b);
        }
        bool ok = true;
        int issued = 0;
        for (int j = 0; j < n && ok; ++j) {
            const int s = j % STAGES;
            ok = warp_wait(lane, bar_ke + 8 * s, ((j / STAGES) & 1) ^ 1, abort_flag, WAIT_NS, p.err);
            if (!ok) break;
            if (lane == 0) {
                mbar_arrive_tx(bar_kf + 8 * s, KV_TILE);
                tma_load_5d(&tmK, sbase + OFF_K + s * KV_TILE, bar_kf + 8 * s, 0, j * BKV, 0, h, b);
                mbar_arrive_tx(bar_vf + 8 * s, KV_TILE);
                tma_load_5d(&tmV, sbase + OFF_V + s * KV_TILE, bar_vf + 8 * s, 0, j * BKV, 0, h, b);
            }
            __syncwarp();
            ++issued;
        }
        // drain: every copy issued has landed before the CTA may exit (immediate on the normal path)
        if (lane == 0) {
            volatile int never = 0;
            mbar_wait(bar_q, 0, &never, 100000000ull, p.err);
            for (int j = issued - 1; j >= 0 && j >= issued - STAGES; --j) {
                mbar_wait(bar_kf + 8 * (j % STAGES), (j / STAGES) & 1, &never, 100000000ull, p.err);
                mbar_wait(bar_vf + 8 * (j % STAGES), (j / STAGES) & 1, &never, 100000000ull, p.err);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ------------------------------------------------------------------ MMA issuer
        // kind::f16: D f32 (bits 4-5 = 1), A and B bf16 (bits 7-9, 10-12 = 1), B MN-major for P V (bit 16),
        // N / 8 at bit 17, M / 16 at bit 24
        const uint32_t idesc_s = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BKV >> 3) << 17) |
                                 ((uint32_t)(BQ >> 4) << 24);
        const uint32_t idesc_o = (1u << 4) | (1u << 7) | (1u << 10) | (1u << 16) | ((uint32_t)(HD >> 3) << 17) |
                                 ((uint32_t)(BQ >> 4) << 24);
        auto issue_s = [&](int t, int j) {
            const uint32_t d = tmem + (uint32_t)((2 * t + (j & 1)) * BKV);
            const uint32_t qa = sbase + OFF_Q + t * Q_TILE, kb = sbase + OFF_K + (j % STAGES) * KV_TILE;
#pragma unroll
            for (int i = 0; i < HD / 16; ++i)
                mma_f16(d, sdesc(qa + (i >> 2) * Q_HALF) + 2 * (i & 3), sdesc(kb + (i >> 2) * KV_HALF) + 2 * (i & 3),
                        idesc_s, (uint32_t)(i > 0));
            mma_commit(bar_sf + 8 * (2 * t + (j & 1)));
        };
        auto issue_pv = [&](int t, int j) {
            const uint32_t d = tmem + (uint32_t)(O_COL + t * HD);
            const uint32_t pa = sbase + OFF_P + (2 * t + (j & 1)) * P_TILE, vb = sbase + OFF_V + (j % STAGES) * KV_TILE;
#pragma unroll
            for (int i = 0; i < BKV / 16; ++i)   // 16 keys = two 8-row groups of the V tile = 2048 B
                mma_f16(d, sdesc(pa) + 2 * i, sdesc_mn(vb, KV_HALF) + (uint64_t)(2048 >> 4) * i, idesc_o,
                        (uint32_t)(j > 0 || i > 0));
            mma_commit(bar_pv + 8 * (2 * t + (j & 1)));
        };
        bool ok = warp_wait(lane, bar_q, 0, abort_flag, WAIT_NS, p.err);
        if (ok) ok = warp_wait(lane, bar_kf, 0, abort_flag, WAIT_NS, p.err);
        if (ok) {
            tc_fence_after();
            if (lane == 0)
                for (int t = 0; t < QT; ++t) issue_s(t, 0);
            __syncwarp();
        }
        for (int j = 0; j < n && ok; ++j) {
            const int jn = j + 1;
            if (jn < n) {
                ok = warp_wait(lane, bar_kf + 8 * (jn % STAGES), (jn / STAGES) & 1, abort_flag, WAIT_NS, p.err);
                for (int t = 0; t < QT && ok; ++t) {
                    // S buffer jn % 2 held S_t(jn - 2): its softmax warps have read it
                    if (jn >= 2) ok = warp_wait(lane, bar_sr + 8 * (2 * t + (jn & 1)), ((jn - 2) >> 1) & 1, abort_flag,
                                                WAIT_NS, p.err);
                    if (!ok) break;
                    tc_fence_after();
                    if (lane == 0) issue_s(t, jn);
                    __syncwarp();
                }
                if (!ok) break;
            }
            ok = warp_wait(lane, bar_vf + 8 * (j % STAGES), (j / STAGES) & 1, abort_flag, WAIT_NS, p.err);
            for (int t = 0; t < QT && ok; ++t) {
                ok = warp_wait(lane, bar_pf + 8 * (2 * t + (j & 1)), (j >> 1) & 1, abort_flag, WAIT_NS, p.err);
                if (!ok) break;
                tc_fence_after();
                if (lane == 0) issue_pv(t, j);
                __syncwarp();
            }
            if (!ok) break;
            if (lane == 0) mma_commit(bar_ke + 8 * (j % STAGES));
            __syncwarp();
        }
        // drain: every MMA issued has completed (and its commits have landed) before TMEM is freed
        if (lane == 0) {
            mma_commit(bar_end);
            volatile int never = 0;
            mbar_wait(bar_end, 0, &never, 100000000ull, p.err);
        }
        __syncwarp();
    } else if (warp >= SM_WARP0) {
        // ------------------------------------------------------------------ softmax + epilogue
        const int t = (warp - SM_WARP0) >> 2, wq = warp & 3;
        const int row = 32 * wq + lane;                             // query row in the tile = TMEM lane
        const uint32_t tl = tmem + ((uint32_t)(32 * wq) << 16);
        const uint32_t o_col = (uint32_t)(O_COL + t * HD);
        const float sl2 = p.sl2;
        float m_run = -INFINITY, l = 0.0f;
        bool ok = true;
        for (int j = 0; j < n && ok; ++j) {
            const int bs = 2 * t + (j & 1);
            ok = warp_wait(lane, bar_sf + 8 * bs, (j >> 1) & 1, abort_flag, WAIT_NS, p.err);
            if (!ok) break;
            tc_fence_after();
            uint32_t r0[32], r1[32];
            tmem_ld32(tl + (uint32_t)(bs * BKV), r0);
            tmem_ld32(tl + (uint32_t)(bs * BKV + 32), r1);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar_sr + 8 * bs);
            float s[BKV];
#pragma unroll
            for (int c = 0; c < 32; ++c) { s[c] = __uint_as_float(r0[c]); s[32 + c] = __uint_as_float(r1[c]); }
            const int kb = j * BKV;
            if (kb + BKV > p.Lk) {
#pragma unroll
                for (int c = 0; c < BKV; ++c)
                    if (kb + c >= p.Lk) s[c] = -INFINITY;
            }
            float mx[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) mx[i] = s[i];
#pragma unroll
            for (int c = 8; c < BKV; c += 8)
#pragma unroll
                for (int i = 0; i < 8; ++i) mx[i] = fmaxf(mx[i], s[c + i]);
            const float tmax = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                                     fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
            const float m_new = fmaxf(m_run, tmax * sl2);
            if (j == 0) {
                m_run = m_new;
            } else {
                const bool need = m_new > m_run + 8.0f;
                if (__any_sync(0xffffffffu, need)) {
                    // O holds P V of steps 0 .. j-1: wait for the last of them, then scale the rows that need it
                    const int jp = j - 1;
                    ok = warp_wait(lane, bar_pv + 8 * (2 * t + (jp & 1)), (jp >> 1) & 1, abort_flag, WAIT_NS, p.err);
                    if (!ok) break;
                    tc_fence_after();
                    const float alpha = need ? ex2(m_run - m_new) : 1.0f;
                    if (need) { l *= alpha; m_run = m_new; }
#pragma unroll 1
                    for (int c = 0; c < HD; c += 32) {
                        uint32_t o[32];
                        tmem_ld32(tl + o_col + (uint32_t)c, o);
#pragma unroll
                        for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                        tmem_st32(tl + o_col + (uint32_t)c, o);
                    }
                }
            }
            const float nm = -m_run;
            uint32_t pk[BKV / 2];
            float ps0 = 0.0f, ps1 = 0.0f;
#pragma unroll
            for (int c = 0; c < BKV; c += 2) {
                const float e0 = ex2(fmaf(s[c], sl2, nm)), e1 = ex2(fmaf(s[c + 1], sl2, nm));
                ps0 += e0;
                ps1 += e1;
                pk[c >> 1] = pack_bf16_rn(e0, e1);
            }
            l += ps0 + ps1;
            // the P buffer was last read by P V of step j - 2
            if (j >= 2) {
                ok = warp_wait(lane, bar_pv + 8 * bs, ((j - 2) >> 1) & 1, abort_flag, WAIT_NS, p.err);
                if (!ok) break;
            }
            // row `row` of the [128][128 B] P tile, 16-byte chunks XOR-swizzled by row % 8 (SWIZZLE_128B)
            const uint32_t prow = sbase + OFF_P + (uint32_t)(bs * P_TILE + row * 128);
#pragma unroll
            for (int ch = 0; ch < 8; ++ch)
                asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};"
                             ::"r"(prow + (uint32_t)((ch ^ (row & 7)) << 4)), "r"(pk[4 * ch]), "r"(pk[4 * ch + 1]),
                               "r"(pk[4 * ch + 2]), "r"(pk[4 * ch + 3])
                             : "memory");
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar_pf + 8 * bs);
        }
        if (ok) {
            const int jl = n - 1;
            ok = warp_wait(lane, bar_pv + 8 * (2 * t + (jl & 1)), (jl >> 1) & 1, abort_flag, WAIT_NS, p.err);
        }
        if (ok) {
            tc_fence_after();
            const float inv = __frcp_rn(l);
            const int qrow = q0 + t * BQ + row;
            const bool valid = qrow < p.Lq;
            float peak = 0.0f;
#pragma unroll 1
            for (int c = 0; c < HD; c += 32) {
                uint32_t o[32];
                tmem_ld32(tl + o_col + (uint32_t)c, o);
                float v[32];
                out_chunk(o, inv, v);
#pragma unroll
                for (int i = 0; i < 32; ++i) peak = fmaxf(peak, fabsf(v[i]));
                if (valid && p.out != nullptr) {
                    uint4 *dst = reinterpret_cast<uint4 *>(p.out + (int64_t)b * p.o_bs + (int64_t)qrow * p.o_rs +
                                                           (int64_t)h * p.o_hs + c);
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                        dst[i] = make_uint4(pack_bf16_rn(v[8 * i], v[8 * i + 1]), pack_bf16_rn(v[8 * i + 2], v[8 * i + 3]),
                                            pack_bf16_rn(v[8 * i + 4], v[8 * i + 5]),
                                            pack_bf16_rn(v[8 * i + 6], v[8 * i + 7]));
                }
            }
            if (p.q8 != nullptr) {
                // int8 per 128 channels = this row of this head: the quantizer's scale, exact quotient, half away
                const float sc = i8_scale_bf16(peak);
                const bool fast = sc >= 0x1p-90f;
                const uint64_t ns = x2_splat(-sc), rs = x2_splat(__frcp_rn(sc));
                const int64_t mrow = (int64_t)b * p.Lq + qrow;
                int8_t *qdst = p.q8 + mrow * (int64_t)p.H * HD + (int64_t)h * HD;
#pragma unroll 1
                for (int c = 0; c < HD; c += 32) {
                    uint32_t o[32];
                    tmem_ld32(tl + o_col + (uint32_t)c, o);
                    float v[32];
                    out_chunk(o, inv, v);
                    if (valid) {
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const float (&v8)[8] = *reinterpret_cast<const float (*)[8]>(&v[8 * i]);
                            *reinterpret_cast<uint2 *>(qdst + c + 8 * i) = quant_chunk8<0, false>(v8, sc, fast, ns, rs);
                        }
                    }
                }
                if (valid) p.s8[mrow * p.H + h] = sc;
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
    }
}

// 5-D map {64 elements, rows, 2 halves of the head dim, heads, batch} over a bf16 tensor whose head dim (128) is
// contiguous; strides in elements. Box {64, box_rows, 2, 1, 1} lands as two [box_rows][128 B] swizzled tiles.
static bool make_map(CUtensorMap *map, const void *base, int64_t rows, int64_t rs, int64_t H, int64_t hs, int64_t B,
                     int64_t bs, uint32_t box_rows) {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (fn == nullptr) {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault, &q) !=
                cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return false;
        fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    }
    // a stride of a dimension of extent 1 is never stepped: give it a valid value
    if (H == 1) hs = 2 * 64;
    if (B == 1) bs = 2 * 64;
    cuuint64_t dims[5] = {64, (cuuint64_t)rows, 2, (cuuint64_t)H, (cuuint64_t)B};
    cuuint64_t strides[4] = {(cuuint64_t)rs * 2, 128, (cuuint64_t)hs * 2, (cuuint64_t)bs * 2};
    cuuint32_t box[5] = {64, box_rows, 2, 1, 1};
    cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 5, const_cast<void *>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

} // namespace attn

cudaError_t launch_attention(const AttnArgs &a, cudaStream_t st, const char **msg) {
    using namespace attn;
    int *err = nullptr;
    cudaError_t e = device_error_word(err_slot(st), &err);
    if (e != cudaSuccess) return e;
    CUtensorMap mq, mk, mv;
    if (!make_map(&mq, a.q, a.Lq, a.q_rs, a.H, a.q_hs, a.B, a.q_bs, BQ) ||
        !make_map(&mk, a.k, a.Lk, a.k_rs, a.H, a.k_hs, a.B, a.k_bs, BKV) ||
        !make_map(&mv, a.v, a.Lk, a.v_rs, a.H, a.v_hs, a.B, a.v_bs, BKV)) {
        *msg = "cuTensorMapEncodeTiled failed (pointer/stride alignment or driver entry point)";
        return cudaErrorInvalidValue;
    }
    Params p;
    p.Lq = (int)a.Lq; p.Lk = (int)a.Lk; p.H = (int)a.H;
    p.sl2 = a.scale * 1.4426950408889634f;
    p.out = static_cast<__nv_bfloat16 *>(a.out); p.o_rs = a.o_rs; p.o_hs = a.o_hs; p.o_bs = a.o_bs;
    p.q8 = a.q8; p.s8 = a.s8;
    p.err = err;
    static bool configured[HN_MAX_DEV];
    int dev = 0;
    e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= HN_MAX_DEV) return cudaErrorInvalidDevice;
    if (!configured[dev]) {
        e = cudaFuncSetAttribute(k_attention, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
        if (e != cudaSuccess) return e;
        configured[dev] = true;
    }
    dim3 grid((unsigned)cdiv(a.Lq, QT * BQ), (unsigned)a.H, (unsigned)a.B);
    k_attention<<<grid, THREADS, SMEM, st>>>(mq, mk, mv, p);
    return cudaGetLastError();
}

} // namespace hn
