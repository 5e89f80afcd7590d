// hn_kernels.h - internal launcher declarations (host side). The C ABI in capi.cu validates arguments
// and calls these; each returns the launch's cudaError_t.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace hn {

constexpr int HN_MAX_DEV = 64;     // device indices the library keeps per-device state for
constexpr int HN_ERR_SLOTS = 64;   // device error words per device: slot 0 = the NULL stream and overflow

int num_sms();  // SM count of the current device (cached per device)
int gemm_sm_reserve();  // SMs the GEMM leaves free for kernels on other streams (hn_set_gemm_sm_reserve)

// Slot of `st`'s device error word: 0 for the NULL stream, else a slot of its own while fewer than
// HN_ERR_SLOTS - 1 streams have launched a kernel that waits (later streams share slot 0).
int err_slot(cudaStream_t st);
// Device address of slot `slot` of the current device's error-word array.
cudaError_t device_error_word(int slot, int **ptr);

cudaError_t launch_quant_act(const void *x, int64_t ldx, int x_dtype, int64_t M, int64_t K, int kind, int flags,
                             void *q, int64_t ldq, float *s, int64_t s_rs, int64_t s_gs, cudaStream_t st);

cudaError_t launch_quant_fp8_block(const void *w, int w_dtype, int64_t N, int64_t K, void *q, float *s,
                                   cudaStream_t st);

// mode 0: adaln (bf16 y), 1: adaln_quant, 2: gated residual + adaln_quant
cudaError_t launch_ln_row(int mode, const void *x, const void *y, const void *gate, const void *shift,
                          const void *scale, int64_t B, int64_t L, int64_t D, float eps, void *out_bf16, int8_t *q,
                          float *s, int64_t s_rs, int64_t s_gs, cudaStream_t st);

cudaError_t launch_gated_residual(const void *x, const void *y, const void *gate, int64_t B, int64_t L, int64_t D,
                                  void *out, cudaStream_t st);

cudaError_t launch_qk_norm_rope(int ntensors, const void *x0, const void *x1, int64_t row_stride, const void *w0,
                                const void *w1, const float *cos, const float *sin, int64_t B, int64_t L, int64_t H,
                                float eps, void *y0, void *y1, int8_t *q8, float *s8, cudaStream_t st);

cudaError_t launch_dequant_kv(const int8_t *q, const float *s, int64_t rows, int64_t D, void *y, cudaStream_t st);

// decoder.cu: kind 0 int8, 1 e4m3 codes
cudaError_t launch_rmsnorm_quant(const void *x, int64_t ldx, const void *w, int64_t rows, int64_t D, float eps,
                                 int kind, void *q, int64_t ldq, float *s, int64_t s_rs, int64_t s_gs, cudaStream_t st);
cudaError_t launch_silu_mul_quant(const void *g, int64_t ldg, const void *u, int64_t ldu, int64_t rows, int64_t I,
                                  int kind, void *q, int64_t ldq, float *s, int64_t s_rs, int64_t s_gs, cudaStream_t st);

cudaError_t launch_pixelumm_qk(const void *x, int64_t row_stride, const void *wt, const void *whw, const float *cos,
                               const float *sin, int64_t N, int64_t H, float eps, void *y, cudaStream_t st);

struct GemmArgs {
    const void *qa; int64_t lda;
    const float *sa; int64_t sa_rs, sa_gs; int sa_mode;
    const void *qw; int64_t ldw;
    const float *sw; int64_t sw_rs, sw_gs; int sw_mode;
    const void *bias; int bias_dtype;
    void *out; int64_t ldo; int out_dtype;
    float *qs; int64_t qs_rs, qs_gs;
    int64_t M, N, K;
    int kind, epilogue;
    int sm_reserve;   // SMs left without a CTA (the grid is num_sms() - sm_reserve persistent CTAs)
};
// Returns cudaSuccess, or cudaErrorInvalidValue with *msg set when a TMA descriptor cannot be encoded.
cudaError_t launch_block_gemm(const GemmArgs &a, cudaStream_t st, const char **msg);

// int8 calls with at most GEMV_MAX_M activation rows (epilogue none or gelu, weight scales per row or per row x
// group) run as a weight-streaming GEMV (gemv.cu) with the tile kernel's arithmetic. Above 2 rows the GEMV's
// per-row folding makes it slower than the tile kernel (measured: 2.87 ms at 4 rows of 983040 x 4096 weights,
// against ~1.8 ms for the tile kernel at any row count up to 128)
constexpr int GEMV_MAX_M = 2;
bool gemv_applies(const GemmArgs &a);
cudaError_t launch_gemv(const GemmArgs &a, cudaStream_t st);

cudaError_t launch_wait_selftest(uint32_t timeout_us, cudaStream_t st);

// read slot `slot` of the current device's error words into *value and clear it (synchronous)
cudaError_t read_and_clear_device_error(int slot, int *value);
// attention (attention.cu): q [B, Lq, H, 128], k / v [B, Lk, H, 128] bf16 with the head dim contiguous (strides
// in elements); out [B, Lq, H, 128] bf16 (or null) and the int8 codes [B*Lq, H*128] + scales [B*Lq, H] (or null)
struct AttnArgs {
    const void *q, *k, *v;
    int64_t q_rs, q_hs, q_bs, k_rs, k_hs, k_bs, v_rs, v_hs, v_bs;
    int64_t B, Lq, Lk, H;
    float scale;
    void *out; int64_t o_rs, o_hs, o_bs;
    int8_t *q8; float *s8;
};
cudaError_t launch_attention(const AttnArgs &a, cudaStream_t st, const char **msg);
// merge of attention pieces by their log-sum-exp (attention.cu); n <= 16 pieces, head dim 128
struct MergeArgs {
    const void *const *parts; const float *const *lses; int64_t n;
    int64_t o_bs, o_qs, o_hs, l_bs, l_hs, l_qs;
    int64_t B, Lq, H;
    void *out; int64_t out_bs, out_qs, out_hs;
    int8_t *q8; float *s8;
};
cudaError_t launch_attn_merge(const MergeArgs &a, cudaStream_t st);

// one warp waits (bounded) until flags[g * group_stride + i] >= value for every g < groups, i < count, i != skip
cudaError_t launch_wait_flags(const uint32_t *flags, int groups, int count, int group_stride, int skip,
                              uint32_t value, uint32_t timeout_us, cudaStream_t st);

} // namespace hn
