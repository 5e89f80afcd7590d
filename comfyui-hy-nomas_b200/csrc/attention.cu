// attention.cu - the DiT's attention (hy_nomas/model.py:145-151: softmax(q k^T * scale) v per batch item and
// head, no mask, head dim 128, bf16 in and out) on the sm_100a tensor cores, with an optional fused int8
// quantization of the output for the projection linear that follows it (the per-token x 128-channel quantizer
// of kernels.py:22-54 applied to the [tokens, heads * 128] output: one 128-channel group is one head's row).
//
// One CTA computes one tile of 128 query rows of one (batch, head) against all keys, 128 keys per step:
//   warp 0      TMA producer: the Q tile once, then K and V tiles of 128 keys (5-D maps {64 elements, row,
//               2 halves of the head dim, head, batch}, 128B swizzle, no multicast) into a ring of STAGES.
//   warp 1      MMA issuer (one thread): S(j) = Q K_j^T into one of two 128-column TMEM buffers, and
//               O += P(j) V_j into a 128-column TMEM accumulator, P read from TMEM (the A operand of the
//               tensor-memory form of the MMA) and V MN-major straight from its TMA tile. S(j+1) is issued
//               before P(j) V_j, so the tensor core computes the next logits while the softmax warps work.
//   warps 4-7   softmax, one thread per query row (its TMEM lane): loads its 128 logits of S(j) at once,
//               takes their maximum with three-input max, keeps a running maximum m (base-2 logits) and sum l
//               (the scaling and the sums in packed f32x2 arithmetic), writes P = 2^(s * scale * log2 e - m) as
//               bf16 pairs into one of two 64-column TMEM buffers, and rescales its O row in TMEM only when the
//               maximum grew by more than 2^8 (a stale maximum leaves every P <= 2^8: exact in fp32 and bf16
//               range). After the last step: O / l -> bf16 rows (and the int8 codes + scale of each row).
// TMEM (512 columns, one CTA per SM): S[b] at 128 b, O at 256, P[b] at 384 + 64 b.
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
constexpr int BKV = 128;                // keys per step
constexpr int HD = 128;                 // head dim
constexpr int STAGES = 3;               // K/V ring
constexpr int SM_WARP0 = 4;             // first softmax warp
constexpr int THREADS = 32 * (SM_WARP0 + 4);
constexpr int Q_HALF = BQ * 128;        // [128 rows][128 B]: one half (64 elements) of the head dim
constexpr int Q_TILE = 2 * Q_HALF;
constexpr int KV_HALF = BKV * 128;      // [128 rows][128 B]
constexpr int KV_TILE = 2 * KV_HALF;
constexpr int OFF_Q = 0;
constexpr int OFF_K = OFF_Q + Q_TILE;
constexpr int OFF_V = OFF_K + STAGES * KV_TILE;
constexpr int OFF_BAR = OFF_V + STAGES * KV_TILE;
// q_full, k_full[S], v_full[S], kv_empty[S], s_full[2], p_full[2], pv_done[2], drain
constexpr int NBARS = 1 + 3 * STAGES + 6 + 1;
constexpr int OFF_MISC = OFF_BAR + NBARS * 8;
constexpr int SMEM = OFF_MISC + 16 + 1024;
static_assert(SMEM <= 232448, "shared memory budget");
constexpr uint32_t TMEM_COLS = 512;
constexpr int S_COL = 0, O_COL = 256, P_COL = 384;
constexpr uint64_t WAIT_NS = 2000000000ull;   // 2 s

struct Params {
    int Lq, Lk, H;
    float sl2;                                  // softmax scale * log2(e)
    __nv_bfloat16 *out; int64_t o_rs, o_hs, o_bs;   // elements; out may be null when only codes are wanted
    int8_t *q8; float *s8;                      // [B*Lq, H*128] codes and [B*Lq, H] scales, or null
    int *err;
};

__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float y;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(y) : "f"(a), "f"(b), "f"(c));
    return y;
}

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// 32 lanes x 32 columns into registers WITHOUT waiting; the values are valid only after ld_wait32 on them
__device__ __forceinline__ void tmem_ld32_async(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
}
// tcgen05.wait::ld with the loaded registers as in-out operands: no use of them can be scheduled before it.
// (The first call waits for every load in flight; the others only order their registers after it.)
__device__ __forceinline__ void ld_wait32(uint32_t (&r)[32], bool wait) {
    if (wait)
        asm volatile("tcgen05.wait::ld.sync.aligned;"
                     : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                       "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                       "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                       "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                       "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
                     :
                     : "memory");
    else
        asm volatile(""
                     : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                       "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                       "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                       "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                       "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
                     :
                     : "memory");
}

// 32 lanes x 16 columns from registers (no wait)
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
                 "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
                 ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
                   "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
                 : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// D (TMEM, fp32) (+)= A (TMEM, 16-bit pairs per column, one row per lane) x B (smem), K = 16
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bd, uint32_t idesc, uint32_t acc) {
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
                 ::"r"(d_tmem), "r"(a_tmem), "l"(bd), "r"(idesc), "r"(acc) : "memory");
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
    const uint32_t bar_pf = bar_sf + 16;
    const uint32_t bar_pv = bar_pf + 16;
    const uint32_t bar_end = bar_pv + 16;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + OFF_MISC);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + OFF_MISC + 4);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q0 = blockIdx.x * BQ, h = blockIdx.y, b = blockIdx.z;
    const int n = (p.Lk + BKV - 1) / BKV;

    if (threadIdx.x == 0) {
        mbar_init(bar_q, 1);
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(bar_kf + 8 * s, 1);
            mbar_init(bar_vf + 8 * s, 1);
            mbar_init(bar_ke + 8 * s, 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(bar_sf + 8 * i, 1);
            mbar_init(bar_pf + 8 * i, 4);     // the four softmax warps
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
            mbar_arrive_tx(bar_q, Q_TILE);      // rows past Lq are zero-filled and still count
            tma_load_5d(&tmQ, sbase + OFF_Q, bar_q, 0, q0, 0, h, b);
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
        auto issue_s = [&](int j) {
            const uint32_t d = tmem + (uint32_t)(S_COL + (j & 1) * BKV);
            const uint32_t kb = sbase + OFF_K + (j % STAGES) * KV_TILE;
#pragma unroll
            for (int i = 0; i < HD / 16; ++i)
                mma_f16(d, sdesc(sbase + OFF_Q + (i >> 2) * Q_HALF) + 2 * (i & 3),
                        sdesc(kb + (i >> 2) * KV_HALF) + 2 * (i & 3), idesc_s, (uint32_t)(i > 0));
            mma_commit(bar_sf + 8 * (j & 1));
        };
        auto issue_pv = [&](int j) {
            const uint32_t a = tmem + (uint32_t)(P_COL + (j & 1) * (BKV / 2));
            const uint32_t vb = sbase + OFF_V + (j % STAGES) * KV_TILE;
#pragma unroll
            for (int i = 0; i < BKV / 16; ++i)   // 16 keys = 8 P columns = two 8-row groups of the V tile
                mma_f16_ts(tmem + O_COL, a + 8 * i, sdesc_mn(vb, KV_HALF) + (uint64_t)(2048 >> 4) * i, idesc_o,
                           (uint32_t)(j > 0 || i > 0));
            mma_commit(bar_pv + 8 * (j & 1));
        };
        bool ok = warp_wait(lane, bar_q, 0, abort_flag, WAIT_NS, p.err);
        if (ok) ok = warp_wait(lane, bar_kf, 0, abort_flag, WAIT_NS, p.err);
        if (ok) {
            tc_fence_after();
            if (lane == 0) issue_s(0);
            __syncwarp();
        }
        for (int j = 0; j < n && ok; ++j) {
            const int jn = j + 1;
            if (jn < n) {
                ok = warp_wait(lane, bar_kf + 8 * (jn % STAGES), (jn / STAGES) & 1, abort_flag, WAIT_NS, p.err);
                // S buffer jn % 2 held S(jn - 2): the softmax has read it once it handed over P(jn - 2)
                if (ok && jn >= 2)
                    ok = warp_wait(lane, bar_pf + 8 * (jn & 1), ((jn - 2) >> 1) & 1, abort_flag, WAIT_NS, p.err);
                if (!ok) break;
                tc_fence_after();
                if (lane == 0) issue_s(jn);
                __syncwarp();
            }
            ok = warp_wait(lane, bar_vf + 8 * (j % STAGES), (j / STAGES) & 1, abort_flag, WAIT_NS, p.err);
            if (ok) ok = warp_wait(lane, bar_pf + 8 * (j & 1), (j >> 1) & 1, abort_flag, WAIT_NS, p.err);
            if (!ok) break;
            tc_fence_after();
            if (lane == 0) {
                issue_pv(j);
                mma_commit(bar_ke + 8 * (j % STAGES));
            }
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
        const int wq = warp & 3;
        const int row = 32 * wq + lane;                             // query row in the tile = TMEM lane
        const uint32_t tl = tmem + ((uint32_t)(32 * wq) << 16);
        const float sl2 = p.sl2;
        float m_run = -INFINITY, l = 0.0f;
        bool ok = true;
        for (int j = 0; j < n && ok; ++j) {
            const int bs = j & 1;
            ok = warp_wait(lane, bar_sf + 8 * bs, (j >> 1) & 1, abort_flag, WAIT_NS, p.err);
            if (!ok) break;
            tc_fence_after();
            uint32_t r0[32], r1[32], r2[32], r3[32];
            const uint32_t sa = tl + (uint32_t)(S_COL + bs * BKV);
            tmem_ld32_async(sa, r0);
            tmem_ld32_async(sa + 32, r1);
            tmem_ld32_async(sa + 64, r2);
            tmem_ld32_async(sa + 96, r3);
            ld_wait32(r0, true);
            ld_wait32(r1, false);
            ld_wait32(r2, false);
            ld_wait32(r3, false);
            const int kb = j * BKV;
            if (kb + BKV > p.Lk) {
#pragma unroll
                for (int c = 0; c < 32; ++c) {
                    if (kb + c >= p.Lk) r0[c] = __float_as_uint(-INFINITY);
                    if (kb + 32 + c >= p.Lk) r1[c] = __float_as_uint(-INFINITY);
                    if (kb + 64 + c >= p.Lk) r2[c] = __float_as_uint(-INFINITY);
                    if (kb + 96 + c >= p.Lk) r3[c] = __float_as_uint(-INFINITY);
                }
            }
            // row maximum: three-input max, two new logits per instruction in eight independent chains
            float mx[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) mx[i] = fmax3(__uint_as_float(r0[i]), __uint_as_float(r1[i]), __uint_as_float(r2[i]));
#pragma unroll
            for (int i = 0; i < 8; ++i) mx[i] = fmax3(mx[i], __uint_as_float(r3[i]), __uint_as_float(r0[8 + i]));
#pragma unroll
            for (int c = 8; c < 32; c += 8)
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    mx[i] = fmax3(mx[i], __uint_as_float(r1[c + i]), __uint_as_float(r2[c + i]));
                    mx[i] = fmax3(mx[i], __uint_as_float(r3[c + i]), c + 8 < 32 ? __uint_as_float(r0[c + 8 + i]) : mx[i]);
                }
            const float tmax = fmax3(fmax3(mx[0], mx[1], mx[2]), fmax3(mx[3], mx[4], mx[5]), fmaxf(mx[6], mx[7]));
            const float m_new = fmaxf(m_run, tmax * sl2);
            if (j == 0) {
                m_run = m_new;
            } else {
                const bool need = m_new > m_run + 8.0f;
                if (__any_sync(0xffffffffu, need)) {
                    // O holds P V of steps 0 .. j-1: wait for the last of them, then scale the rows that need it
                    const int jp = j - 1;
                    ok = warp_wait(lane, bar_pv + 8 * (jp & 1), (jp >> 1) & 1, abort_flag, WAIT_NS, p.err);
                    if (!ok) break;
                    tc_fence_after();
                    const float alpha = need ? ex2(m_run - m_new) : 1.0f;
                    if (need) { l *= alpha; m_run = m_new; }
#pragma unroll 1
                    for (int c = 0; c < HD; c += 32) {
                        uint32_t o[32];
                        tmem_ld32(tl + (uint32_t)(O_COL + c), o);
#pragma unroll
                        for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                        tmem_st32(tl + (uint32_t)(O_COL + c), o);
                    }
                }
            }
            // the P buffer was last read by P V of step j - 2
            if (j >= 2) {
                ok = warp_wait(lane, bar_pv + 8 * bs, ((j - 2) >> 1) & 1, abort_flag, WAIT_NS, p.err);
                if (!ok) break;
            }
            const uint32_t pa = tl + (uint32_t)(P_COL + bs * (BKV / 2));
            const uint64_t nm2 = x2_splat(-m_run), sl22 = x2_splat(sl2);
            uint64_t ps2 = 0ull;                                    // packed partial sums (+0.0f, +0.0f)
            auto emit = [&](const uint32_t (&r)[32], uint32_t col) {
                uint32_t pk[16];
#pragma unroll
                for (int c = 0; c < 32; c += 2) {
                    float a0, a1;
                    x2_split(x2_fma(x2(__uint_as_float(r[c]), __uint_as_float(r[c + 1])), sl22, nm2), a0, a1);
                    const float e0 = ex2(a0), e1 = ex2(a1);
                    ps2 = x2_add(ps2, x2(e0, e1));
                    pk[c >> 1] = pack_bf16_rn(e0, e1);
                }
                tmem_st16(pa + col, pk);
            };
            emit(r0, 0);
            emit(r1, 16);
            emit(r2, 32);
            emit(r3, 48);
            {
                float p0, p1;
                x2_split(ps2, p0, p1);
                l += p0 + p1;
            }
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar_pf + 8 * bs);
        }
        if (ok) {
            const int jl = n - 1;
            ok = warp_wait(lane, bar_pv + 8 * (jl & 1), (jl >> 1) & 1, abort_flag, WAIT_NS, p.err);
        }
        if (ok) {
            tc_fence_after();
            const float inv = __frcp_rn(l);
            const int qrow = q0 + row;
            const bool valid = qrow < p.Lq;
            float peak = 0.0f;
#pragma unroll 1
            for (int c = 0; c < HD; c += 32) {
                uint32_t o[32];
                tmem_ld32(tl + (uint32_t)(O_COL + c), o);
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
                    tmem_ld32(tl + (uint32_t)(O_COL + c), o);
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

// ---------------------------------------------------------------------------------------------------
// Merge of attention computed in key pieces (the sequence-parallel step attends to each rank's keys as they
// arrive): piece i gives o_i = softmax over its keys, and lse_i = log of its sum of exp(logits) (natural log);
// the whole is out = sum_i exp(lse_i - L) o_i with L = log sum_i exp(lse_i). One warp per (batch, query, head):
// 4 of the head's 128 elements per lane. Optionally the result is quantized for the projection linear with the
// activation quantizer's arithmetic (one 128-channel group = one head's row).

constexpr int MERGE_MAX = 16;

struct MergeParams {
    const __nv_bfloat16 *part[MERGE_MAX];
    const float *lse[MERGE_MAX];
    int n, B, Lq, H;
    int64_t o_bs, o_qs, o_hs;       // piece strides (elements), the same for every piece
    int64_t l_bs, l_hs, l_qs;       // log-sum-exp strides
    __nv_bfloat16 *out; int64_t out_bs, out_qs, out_hs;
    int8_t *q8; float *s8;
};

__global__ void __launch_bounds__(256) k_attn_merge(const MergeParams p) {
    const int lane = threadIdx.x & 31;
    const int64_t items = (int64_t)p.B * p.Lq * p.H;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t it = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; it < items; it += nwarps) {
        const int h = (int)(it % p.H);
        const int64_t r = it / p.H;
        const int q = (int)(r % p.Lq), b = (int)(r / p.Lq);
        const int64_t lo = (int64_t)b * p.l_bs + (int64_t)h * p.l_hs + (int64_t)q * p.l_qs;
        float lmax = -INFINITY;
        for (int i = 0; i < p.n; ++i) lmax = fmaxf(lmax, p.lse[i][lo]);
        const int64_t po = (int64_t)b * p.o_bs + (int64_t)q * p.o_qs + (int64_t)h * p.o_hs + 4 * lane;
        float den = 0.0f, a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
        for (int i = 0; i < p.n; ++i) {
            const float w = expf(p.lse[i][lo] - lmax);
            const uint2 u = *reinterpret_cast<const uint2 *>(p.part[i] + po);
            den += w;
            a0 = fmaf(w, bf16_lo(u.x), a0);
            a1 = fmaf(w, bf16_hi(u.x), a1);
            a2 = fmaf(w, bf16_lo(u.y), a2);
            a3 = fmaf(w, bf16_hi(u.y), a3);
        }
        const float inv = __frcp_rn(den);
        const float v0 = rbf16(a0 * inv), v1 = rbf16(a1 * inv), v2 = rbf16(a2 * inv), v3 = rbf16(a3 * inv);
        if (p.out != nullptr) {
            uint2 o;
            o.x = pack_bf16_rn(v0, v1);
            o.y = pack_bf16_rn(v2, v3);
            *reinterpret_cast<uint2 *>(p.out + (int64_t)b * p.out_bs + (int64_t)q * p.out_qs + (int64_t)h * p.out_hs +
                                       4 * lane) = o;
        }
        if (p.q8 != nullptr) {
            const float peak = warp_max_xor(fmaxf(fmaxf(fabsf(v0), fabsf(v1)), fmaxf(fabsf(v2), fabsf(v3))), 32);
            const float sc = i8_scale_bf16(peak);
            uint32_t word;
            if (sc >= 0x1p-90f) {
                const uint64_t ns = x2_splat(-sc), rs = x2_splat(__frcp_rn(sc));
                uint32_t c0, c1, c2, c3;
                x2_codes(x2_quot(x2(v0, v1), ns, rs), c0, c1);
                x2_codes(x2_quot(x2(v2, v3), ns, rs), c2, c3);
                word = pack4_lowbytes(c0, c1, c2, c3);
            } else {
                word = pack4_i8(code_i8(__fdiv_rn(v0, sc)), code_i8(__fdiv_rn(v1, sc)), code_i8(__fdiv_rn(v2, sc)),
                                code_i8(__fdiv_rn(v3, sc)));
            }
            const int64_t row = (int64_t)b * p.Lq + q;
            *reinterpret_cast<uint32_t *>(p.q8 + row * (int64_t)p.H * HD + (int64_t)h * HD + 4 * lane) = word;
            if (lane == 0) p.s8[row * p.H + h] = sc;
        }
    }
}

} // namespace attn

cudaError_t launch_attn_merge(const MergeArgs &a, cudaStream_t st) {
    using namespace attn;
    MergeParams p;
    for (int i = 0; i < MERGE_MAX; ++i) {
        p.part[i] = i < a.n ? static_cast<const __nv_bfloat16 *>(a.parts[i]) : nullptr;
        p.lse[i] = i < a.n ? a.lses[i] : nullptr;
    }
    p.n = (int)a.n; p.B = (int)a.B; p.Lq = (int)a.Lq; p.H = (int)a.H;
    p.o_bs = a.o_bs; p.o_qs = a.o_qs; p.o_hs = a.o_hs;
    p.l_bs = a.l_bs; p.l_hs = a.l_hs; p.l_qs = a.l_qs;
    p.out = static_cast<__nv_bfloat16 *>(a.out); p.out_bs = a.out_bs; p.out_qs = a.out_qs; p.out_hs = a.out_hs;
    p.q8 = a.q8; p.s8 = a.s8;
    const int64_t warps = a.B * a.Lq * a.H;
    int64_t grid = cdiv(warps, 8);
    const int64_t cap = (int64_t)num_sms() * 8;
    if (grid > cap) grid = cap;
    k_attn_merge<<<(unsigned)grid, 256, 0, st>>>(p);
    return cudaGetLastError();
}

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
    dim3 grid((unsigned)cdiv(a.Lq, BQ), (unsigned)a.H, (unsigned)a.B);
    k_attention<<<grid, THREADS, SMEM, st>>>(mq, mk, mv, p);
    return cudaGetLastError();
}

} // namespace hn
