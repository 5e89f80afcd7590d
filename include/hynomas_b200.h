/*
 * hynomas_b200.h - C ABI of the B200 (sm_100a) quantized DiT linear path.
 *
 * Every entry point replaces one Triton kernel (or one torch expression) of ComfyUI-Hy-Nomas. The
 * reference interface each one stands in for is cited beside it as `file:line` inside that project
 * (hy_nomas/kernels.py, hy_nomas/fused.py, hy_nomas/ops.py, hy_nomas/model.py, hy_nomas/pixelumm.py,
 * hy_nomas/world.py).
 *
 * Conventions
 *  - All pointers are DEVICE pointers unless the name ends in `_host`. Nothing here allocates device
 *    memory; outputs are caller-owned buffers of the documented shape. Inputs are never written.
 *  - Matrices are row-major with an explicit leading dimension in ELEMENTS (ld >= number of columns).
 *  - `stream` is a cudaStream_t (NULL = legacy default stream) of the device that owns the pointers.
 *  - Return value: HN_OK (0) or an hn_status code. On error nothing was launched and the message is
 *    available from hn_last_error() (per calling thread). Kernels never trap; device-side waits are
 *    bounded and report HN_ERR_TIMEOUT through hn_device_error().
 *  - bf16/fp16/fp32 inputs are named by the HN_DTYPE_* codes. Quantized codes are int8 or
 *    float8_e4m3fn bytes (HN_KIND_*).
 *  - Quantization scales are fp32 with one value per (row, 128-wide group). A scale tensor is given as a
 *    pointer plus two strides in elements: s[row * s_rs + group * s_gs]. The reference's layout is
 *    row-major [rows, groups] (s_rs = groups, s_gs = 1). The group-major layout (s_rs = 1, s_gs >= rows,
 *    i.e. [groups, rows]) lets the GEMM stream one group's scales for a whole tile with one bulk copy;
 *    the quantizers here produce it and the Python layer hands it back as a [rows, groups] view.
 */
#ifndef HYNOMAS_B200_H
#define HYNOMAS_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* the library is built with hidden visibility; everything declared here is exported */
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

#define HN_ABI_VERSION 1

typedef enum {
    HN_OK = 0,
    HN_ERR_SHAPE = 1,       /* a dimension is zero/negative where not allowed, or not a multiple of 128 */
    HN_ERR_ALIGN = 2,       /* a pointer or leading dimension breaks the 16-byte rule of a vector/TMA path */
    HN_ERR_ARCH = 3,        /* the current device is not compute capability 10.0 (B200 / sm_100a) */
    HN_ERR_CUDA = 4,        /* a CUDA runtime/driver call failed (message holds the CUDA error string) */
    HN_ERR_ARG = 5,         /* null pointer or unknown enum value */
    HN_ERR_TIMEOUT = 6,     /* a device-side wait ran past its limit (read via hn_device_error) */
    HN_ERR_UNSUPPORTED = 7  /* a combination of modes that the kernels do not implement */
} hn_status;

/* input element types */
#define HN_DTYPE_BF16 0
#define HN_DTYPE_FP16 1
#define HN_DTYPE_FP32 2
#define HN_DTYPE_INT32 3 /* output only: the raw integer accumulator */

/* quantized code types */
#define HN_KIND_INT8 0
#define HN_KIND_FP8E4M3 1

/* scale layouts of the block-scaled GEMM (hn_block_gemm) */
#define HN_SCALE_GROUP 0  /* one fp32 per row and 128-wide K group: [rows, K/128] (the reference layout) */
#define HN_SCALE_ROW 1    /* one fp32 per row: per-token activations / per-output-channel weights */
#define HN_SCALE_BLOCK 2  /* weights only: one fp32 per 128x128 block, [N/128, K/128] (FP8 decoder layout) */

/* GEMM epilogues, same numbering as kernels.EPILOGUES (hy_nomas/kernels.py:149) */
#define HN_EPI_NONE 0
#define HN_EPI_GELU 1
#define HN_EPI_GELU_QUANT 2

/* Message of the last failed call on this thread ("" if none). */
const char *hn_last_error(void);

/* ABI version (HN_ABI_VERSION) and the number of SMs the kernels size their grids for (0 if no GPU). */
int hn_abi_version(void);
int hn_num_sms(void);

/*
 * Leave `n` SMs without a GEMM CTA in later hn_block_gemm launches (default 0), so that kernels on other
 * streams - the K/V all-gathers of sequence parallelism - run beside a GEMM instead of after it.
 * 0 <= n <= 64. The value is PROCESS-GLOBAL: it applies to every later hn_block_gemm call of every thread
 * and device until it is set again, so a caller that changes it should put the old value
 * (hn_get_gemm_sm_reserve) back when done. No reference counterpart: the reference runs one GPU.
 */
int hn_set_gemm_sm_reserve(int n);
int hn_get_gemm_sm_reserve(void);

/*
 * Device error word of `stream`, written by bounded waits inside the kernels launched on that stream
 * (0 = none). Synchronizes `stream`, copies its word to *code_host and clears it. Returns HN_ERR_TIMEOUT if
 * a wait timed out. Each stream that launches a waiting kernel gets a word of its own, per device, up to 63
 * streams; the NULL stream and any further streams share one word. Call it with the stream's device
 * current.
 */
int hn_device_error(void *stream, int *code_host);

/*
 * Test hook for the bounded-wait machinery: launches one CTA that waits on an mbarrier that nothing
 * completes, with a limit of `timeout_us` microseconds, then returns. The timeout is recorded in the
 * device error word exactly as a stuck GEMM pipeline would record it. No counterpart in the reference
 * (the reference's Triton kernels have no device-side waits).
 */
int hn_selftest_wait_timeout(uint32_t timeout_us, void *stream);

/*
 * K1 - per (row, 128-group) absmax activation quantizer.
 * Replaces hy_nomas/kernels.py:22-54 (_quantize_kernel / quantize_activations).
 * x [M, K] (dtype x_dtype, leading dim ldx), K % 128 == 0 ->
 *   codes q [M, K] (int8, or e4m3 bytes for HN_KIND_FP8E4M3; leading dim ldq),
 *   scales s: one per (row, group) at s[m * s_rs + g * s_gs].
 * int8: s = peak > 0 ? peak/127 : 1, q = round-half-away(x/s) clamped to +-127.
 * e4m3: s = max(peak, 1e-12)/448, q = e4m3(x/s) round-to-nearest-even, saturating.
 * `flags` (0 = the reference's quantizer):
 *   HN_QUANT_PER_ROW: one group spanning all K (per-token scale s[m * s_rs]) - per-token dynamic activation
 *     quantization, the usual W8A8 convention; no counterpart in the reference.
 *   HN_QUANT_ROUND_HALF_EVEN (int8 only): codes rounded half to even instead of half away from zero
 *     (torch.round's convention); no counterpart in the reference.
 */
#define HN_QUANT_PER_ROW 1
#define HN_QUANT_ROUND_HALF_EVEN 2
int hn_quant_act(const void *x, int64_t ldx, int x_dtype, int64_t M, int64_t K, int kind, int flags,
                 void *q, int64_t ldq, float *s, int64_t s_rs, int64_t s_gs, void *stream);

/*
 * K2 - block-scaled W8A8 / FP8 GEMM on the 5th-generation tensor cores (tcgen05, TMEM accumulators).
 * Replaces hy_nomas/kernels.py:80-170 (_gemm_body / block_gemm).
 *   y[m, n] = sum_g sa[m, g] * sw[n, g] * dot_g(qa[m, :], qw[n, :])  (+ bias[n])
 * qa [M, K] codes (lda), qw [N, K] codes (ldw; K-major, the layout the checkpoints store), both of
 * `kind`. K % 128 == 0, lda and ldw multiples of 16, qa/qw 16-byte aligned.
 * sa: sa_mode HN_SCALE_GROUP -> sa[m * sa_rs + g * sa_gs] | HN_SCALE_ROW -> sa[m * sa_rs].
 * sw: sw_mode HN_SCALE_GROUP -> sw[n * sw_rs + g * sw_gs] | HN_SCALE_ROW -> sw[n * sw_rs] |
 *     HN_SCALE_BLOCK -> sw[(n / 128) * sw_rs + g * sw_gs] (one per 128 x 128 weight block).
 * Group scales with unit row stride (group-major) are streamed by bulk copies; others by plain loads.
 * bias: NULL or [N] of bias_dtype (bf16/fp16/fp32), 16-byte aligned.
 * epilogue HN_EPI_NONE: out [M, N] of out_dtype (bf16/fp16/fp32), ldo.
 *          HN_EPI_GELU: out bf16 = rbf16(gelu_tanh(rbf16(y))).
 *          HN_EPI_GELU_QUANT: out int8 [M, N] codes of the GELU output quantized per row and 128
 *                             columns, scales qs[m * qs_rs + c * qs_gs]. Needs N % 128 == 0.
 * out_dtype HN_DTYPE_INT32 (int8 kind, both scale modes HN_SCALE_ROW, no bias, HN_EPI_NONE): out is the
 * exact int32 accumulator sum_k qa*qw - the raw integer result, no scaling.
 * int8 with HN_SCALE_ROW on both sides accumulates all of K in one int32 (|sum| <= K * 128 * 128), so it
 * needs K <= HN_ROW_MODE_MAX_K; the per-group modes accumulate 128 columns at a time and have no such bound.
 */
#define HN_ROW_MODE_MAX_K 130944
int hn_block_gemm(const void *qa, int64_t lda, const float *sa, int64_t sa_rs, int64_t sa_gs, int sa_mode,
                  const void *qw, int64_t ldw, const float *sw, int64_t sw_rs, int64_t sw_gs, int sw_mode,
                  const void *bias, int bias_dtype,
                  void *out, int64_t ldo, int out_dtype, float *qs, int64_t qs_rs, int64_t qs_gs,
                  int64_t M, int64_t N, int64_t K, int kind, int epilogue, void *stream);

/*
 * K3 - LayerNorm (no affine) + adaLN modulate + int8 quantize per 128 channels.
 * Replaces hy_nomas/kernels.py:173-207 (_adaln_quant_kernel / adaln_quant).
 * x [B*L, D] bf16 contiguous, shift/scale [B, D] bf16 -> q [B*L, D] int8, scales s[r * s_rs + g * s_gs]
 * for token row r and channel group g. D % 128 == 0, D <= 16384.
 */
int hn_adaln_quant(const void *x, const void *shift, const void *scale, int64_t B, int64_t L, int64_t D,
                   float eps, int8_t *q, float *s, int64_t s_rs, int64_t s_gs, void *stream);

/*
 * K4 - LayerNorm + modulate -> bf16. Replaces hy_nomas/fused.py:37-62 (_adaln_kernel / adaln).
 * x [B*L, D] bf16, shift/scale [B, D] bf16 -> y [B*L, D] bf16. D % 16 == 0, D <= 16384.
 */
int hn_adaln(const void *x, const void *shift, const void *scale, int64_t B, int64_t L, int64_t D, float eps,
             void *y, void *stream);

/*
 * K5 - per-head RMSNorm (fp32, rounded to bf16) x weight (bf16), then interleaved-pair RoPE.
 * Replaces hy_nomas/fused.py:65-105 (_qk_norm_rope_kernel / qk_norm_rope).
 * x: B*L token rows of H heads x D (D == 128), heads contiguous, token row stride `row_stride`
 * elements (>= H*D; e.g. 3*H*D inside a fused qkv buffer); rows of batch b start at b*L*row_stride.
 * weight [D] bf16. cos/sin [L, D] fp32 or both NULL (no RoPE). y [B, L, H, D] bf16 contiguous.
 * x, weight and y 16-byte aligned, row_stride a multiple of 8; cos/sin 16-byte aligned.
 */
int hn_qk_norm_rope(const void *x, int64_t row_stride, const void *weight, const float *cos, const float *sin,
                    int64_t B, int64_t L, int64_t H, int64_t D, float eps, void *y, void *stream);

/*
 * K5 x2 - the same for the q and k tensors of one attention in a single launch (the RoPE tables are
 * read once per token for both). Same arguments as hn_qk_norm_rope, per tensor.
 * Replaces the pair of calls at hy_nomas/model.py:266-267.
 */
int hn_qk_norm_rope2(const void *xq, const void *xk, int64_t row_stride, const void *wq, const void *wk,
                     const float *cos, const float *sin, int64_t B, int64_t L, int64_t H, int64_t D, float eps,
                     void *yq, void *yk, void *stream);

/*
 * K6 - gated residual x + rbf16(y * gate[b]) -> bf16.
 * Replaces hy_nomas/fused.py:108-128 (_gated_residual_kernel / gated_residual).
 * x, y [B*L, D] bf16, gate [B, D] bf16 -> out [B*L, D] bf16. D % 8 == 0.
 */
int hn_gated_residual(const void *x, const void *y, const void *gate, int64_t B, int64_t L, int64_t D, void *out,
                      void *stream);

/*
 * K6+K3 - gated residual, then the next LayerNorm/modulate/int8 quantize of its result, in one pass.
 * Replaces the pair fused.gated_residual + kernels.adaln_quant at hy_nomas/model.py:280-282.
 * out = x + rbf16(y * gate) (bf16, written) and (q, s) = adaln_quant(out, shift, scale, eps).
 */
int hn_gated_residual_adaln_quant(const void *x, const void *y, const void *gate, const void *shift,
                                  const void *scale, int64_t B, int64_t L, int64_t D, float eps, void *out,
                                  int8_t *q, float *s, int64_t s_rs, int64_t s_gs, void *stream);

/*
 * K7 - PixelUMM decoder q/k prep: split T / HW RMSNorm (own weights) + rotate-half MRoPE.
 * Replaces hy_nomas/fused.py:131-186 (_pixelumm_qk_kernel / pixelumm_qk).
 * x: N tokens x H heads x D (D == 128), token stride row_stride; weight_t/weight_hw [D/2] bf16;
 * cos/sin [N, D] fp32 -> y [N, H, D] bf16.
 */
int hn_pixelumm_qk(const void *x, int64_t row_stride, const void *weight_t, const void *weight_hw, const float *cos,
                   const float *sin, int64_t N, int64_t H, int64_t D, float eps, void *y, void *stream);

/*
 * int8 KV quantizer per (token, head): absmax/127, round half away from zero.
 * Replaces hy_nomas/world.py:83-90 (quantize_kv). x [L*H, D] bf16 -> q [L*H, D] int8, s [L*H] fp32.
 */
int hn_quantize_kv(const void *x, int64_t rows, int64_t D, int8_t *q, float *s, void *stream);

/*
 * int8 KV dequantizer: y = bf16(float(q) * s) with s per (token, head) row.
 * Replaces hy_nomas/world.py:93-94 (dequantize_kv), as called per layer on history load (world.py:197-204).
 * q [rows, D] int8, s [rows] fp32 -> y [rows, D] bf16; D % 16 == 0; q and y 16-byte aligned.
 */
int hn_dequantize_kv(const int8_t *q, const float *s, int64_t rows, int64_t D, void *y, void *stream);

/*
 * K5 for the cache pass: hn_qk_norm_rope, and the same output quantized for the int8 KV cache in the same
 * launch - hy_nomas/world.py:83-90 (quantize_kv) applied to y, fused so y is not read back.
 * Arguments as hn_qk_norm_rope, plus q [B, L, H, D] int8 (16-byte aligned) and s [B*L*H] fp32.
 */
int hn_qk_norm_rope_kv(const void *x, int64_t row_stride, const void *weight, const float *cos, const float *sin,
                       int64_t B, int64_t L, int64_t H, int64_t D, float eps, void *y, int8_t *q, float *s,
                       void *stream);

/*
 * FP8 weight quantizer per 128 x 128 block (load time of the FP8 decoder linears).
 * Replaces hy_nomas/pixelumm.py:77-82 (NomasFP8Block128Layout.quantize). w [N, K] contiguous fp32 or bf16
 * (w_dtype), N % 128 == 0, K % 128 == 0 -> q [N, K] e4m3 bytes = e4m3(w / s) (nearest even), s [N/128, K/128]
 * fp32 row-major = max(absmax of the block, 1e-4) / 448.
 */
int hn_quantize_fp8_block(const void *w, int w_dtype, int64_t N, int64_t K, void *q, float *s, void *stream);

/*
 * PixelUMM decoder: RMSNorm + the activation quantizer of the FP8 (or int8) linears that read its output, in one
 * pass. Replaces hy_nomas/pixelumm.py:246-259 (RMSNorm.forward, the decoder layer's input_norm and
 * post_attn_norm) followed by the quantizer block_linear runs for the next linears (kernels.py:22-54 via
 * pixelumm.py:147-155); the normalized activations are not written. A fusion of the reference's sequence, named
 * in its notes (README.md:266 "RMSNorm/SiLU fusions").
 * x [rows, D] bf16 (row pitch ldx), weight [D] bf16 -> y = rbf16(w * rbf16(x * 1/sqrt(mean(x^2) + eps))) quantized
 * per row and 128 columns: codes q [rows, D] (int8 or e4m3 by `kind`, pitch ldq), scales s[r * s_rs + g * s_gs].
 * D % 128 == 0, D <= 16384; x, weight, q 16-byte aligned with 16-byte row pitches.
 */
int hn_rmsnorm_quant(const void *x, int64_t ldx, const void *weight, int64_t rows, int64_t D, float eps, int kind,
                     void *q, int64_t ldq, float *s, int64_t s_rs, int64_t s_gs, void *stream);

/*
 * PixelUMM decoder MLP gate: silu(gate) * up (torch's bf16 roundings: silu(g) = g / (1 + exp(-g)) in fp32 rounded
 * to bf16, times up, rounded to bf16) quantized for down_proj in the same pass. Replaces hy_nomas/pixelumm.py:322-323
 * (MLP.forward's F.silu(gate_proj(x)) * up_proj(x)) followed by down_proj's activation quantizer (kernels.py:22-54).
 * g, u [rows, I] bf16 (pitches ldg, ldu; e.g. the two halves of one stacked gate|up GEMM output) -> codes q [rows, I]
 * and scales s[r * s_rs + g * s_gs] per 128 columns. I % 128 == 0; g, u, q 16-byte aligned with 16-byte pitches.
 */
int hn_silu_mul_quant(const void *g, int64_t ldg, const void *u, int64_t ldu, int64_t rows, int64_t I, int kind,
                      void *q, int64_t ldq, float *s, int64_t s_rs, int64_t s_gs, void *stream);

/*
 * Attention: out = softmax(q k^T * scale) v per batch item and head, no mask, head dim 128, bf16 - the SDPA call of
 * the DiT block. Replaces hy_nomas/model.py:145-151 (`attention`, ComfyUI's optimized_attention over
 * q/k/v [B, L, H, D]). q [B, Lq, H, 128], k / v [B, Lk, H, 128], out [B, Lq, H, 128]; each with its own row /
 * head / batch strides in elements (multiples of 8), the head dim contiguous, 16-byte aligned bases.
 * Optionally fused: the output quantized per token x 128 channels (one head's row) exactly as hn_quant_act does
 * for the [B*Lq, H*128] attention output (int8, round half away): q8 [B*Lq, H*128] int8 and s8 [B*Lq, H] fp32,
 * row-major - the input of the projection linear. `out` may be NULL when only the codes are wanted; q8 and s8 are
 * both NULL or both set. The softmax runs in base 2 with fp32 statistics, P is rounded to bf16 for the P V
 * product, the accumulators are fp32 (differences to the reference's SDPA are those of two valid bf16 attention
 * implementations, not bit-level).
 */
int hn_attention(const void *q, int64_t q_rs, int64_t q_hs, int64_t q_bs, const void *k, int64_t k_rs, int64_t k_hs,
                 int64_t k_bs, const void *v, int64_t v_rs, int64_t v_hs, int64_t v_bs, int64_t B, int64_t Lq,
                 int64_t Lk, int64_t H, int64_t D, float scale, void *out, int64_t o_rs, int64_t o_hs, int64_t o_bs,
                 int8_t *q8, float *s8, void *stream);

/*
 * Merge of attention computed in key pieces: piece i (i < n <= 16) holds o_i [B, Lq, H, 128] bf16 (strides o_*, the
 * same for every piece) = softmax(q k_i^T * scale) v_i over its keys and lse_i [B, H, Lq] fp32 (strides l_*) = the
 * natural log of that softmax's sum of exp(logits). Writes out = sum_i exp(lse_i - L) o_i, L = log sum_i exp(lse_i),
 * as bf16 [B, Lq, H, 128] (strides out_*) and/or its int8 codes per token x 128 channels (q8 [B*Lq, H*128], s8
 * [B*Lq, H]; the hn_quant_act arithmetic, as in hn_attention). `parts` and `lses` are host arrays of device
 * pointers. No reference counterpart: the reference attends in one call; this lets the sequence-parallel step
 * attend to each rank's keys as they arrive. Piece strides multiples of 4 elements, 8-byte aligned pieces.
 */
int hn_attn_merge(const void *const *parts, const float *const *lses, int64_t n, int64_t o_bs, int64_t o_qs,
                  int64_t o_hs, int64_t l_bs, int64_t l_hs, int64_t l_qs, int64_t B, int64_t Lq, int64_t H, int64_t D,
                  void *out, int64_t out_bs, int64_t out_qs, int64_t out_hs, int8_t *q8, float *s8, void *stream);

/*
 * Sequence-parallel K/V exchange over NVLink by the copy engines. No reference counterpart: the reference runs
 * one GPU; these replace the NCCL all-gather of the build's own sequence-parallel DiT step, whose SM-based kernel
 * cannot run beside the persistent GEMM. All host-side: no kernel of this library is involved.
 *
 * hn_ipc_export: a CUDA IPC handle (64 bytes at handle_host) for the device allocation that holds `ptr` (current
 *   device), and ptr's byte offset in it.
 * hn_ipc_import: map a peer process's exported allocation into the current device's context (peer access
 *   enabled lazily); *base_host receives its base (add the exporter's offset). hn_ipc_close unmaps it.
 * hn_peer_push: on `stream`, copy `bytes` from src (this device) to dst (a mapped peer address) by DMA, then write
 *   the 32-bit `value` to `flag` (a mapped peer address, or NULL for none) after a memory fence, so the data is
 *   visible before the flag.
 * hn_peer_push2d: hn_peer_push for `height` rows of `width` bytes, row r read at src + r * spitch and written at
 *   dst + r * dpitch (one strided DMA): the head-parallel exchange moves one head group of every token this way.
 * hn_wait_flags: on `stream`, one warp waits until every flags[g * group_stride + i] (g < groups, i < count,
 *   i != skip; groups * count <= 1024) has reached `value` (wrap-safe: (int32_t)(flag - value) >= 0), with system-scope
 *   acquire loads, so that kernels after it on the stream see the data pushed before those flags. Bounded: after
 *   `timeout_us` it records HN_ERR_TIMEOUT in the stream's error word (hn_device_error) and returns.
 */
int hn_ipc_export(const void *ptr, void *handle_host, int64_t *offset_host);
int hn_ipc_import(const void *handle_host, void **base_host);
int hn_ipc_close(void *base);
int hn_peer_push(void *dst, const void *src, int64_t bytes, void *flag, uint32_t value, void *stream);
int hn_peer_push2d(void *dst, int64_t dpitch, const void *src, int64_t spitch, int64_t width, int64_t height,
                   void *flag, uint32_t value, void *stream);
int hn_wait_flags(const int32_t *flags, int64_t groups, int64_t count, int64_t group_stride, int64_t skip,
                  uint32_t value, uint32_t timeout_us, void *stream);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif

#endif /* HYNOMAS_B200_H */
