"""CPU oracle for the quantized DiT linear path - TEST INFRASTRUCTURE ONLY.

This module is the checker the CUDA path is compared against. Only `tests/`, `__graft_entry__.smoke()`
and `bench.py`'s CPU-baseline leg import it; the product package (`comfyui-hy-nomas_b200/hy_nomas_b200`)
never does, and it has no CPU fallback.

It wraps `hn_oracle.c` (a plain-C, one-IEEE-operation-per-line restatement of the reference's kernels,
built here with gcc -ffp-contract=off) behind numpy functions named after the reference's Python API:

  quantize_activations   hy_nomas/kernels.py:22-54
  block_gemm             hy_nomas/kernels.py:80-170
  adaln_quant            hy_nomas/kernels.py:173-207
  adaln                  hy_nomas/fused.py:37-62
  qk_norm_rope           hy_nomas/fused.py:65-105
  gated_residual         hy_nomas/fused.py:108-128
  pixelumm_qk            hy_nomas/fused.py:131-186
  quantize_g128          hy_nomas/ops.py:41-52
  dequantize_g128        hy_nomas/ops.py:55-62
  quantize_fp8_block     hy_nomas/pixelumm.py:77-82
  quantize_kv            hy_nomas/world.py:83-90
  rmsnorm_quant          hy_nomas/pixelumm.py:246-259 + kernels.py:22-42 (decoder norm, then the FP8 quantizer)
  silu_mul_quant         hy_nomas/pixelumm.py:322-323 + kernels.py:22-42 (decoder MLP gate, then the quantizer)

Parity of this oracle with the reference is pinned by tests/test_oracle_golden.py against vectors made
by tests/golden/make_golden.py from the reference's own code.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "hn_oracle.c")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(BUILD, "liboracle.so")
GROUP = 128


def build(force=False):
    """Compile hn_oracle.c with gcc (strict IEEE: no contraction, no fast-math)."""
    os.makedirs(BUILD, exist_ok=True)
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= os.path.getmtime(SRC):
        return LIB
    cmd = ["gcc", "-O2", "-std=c11", "-fPIC", "-shared", "-ffp-contract=off", "-fno-fast-math",
           "-fopenmp", SRC, "-o", LIB + ".tmp", "-lm"]
    subprocess.check_call(cmd)
    os.replace(LIB + ".tmp", LIB)
    return LIB


_lib = None


def lib():
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(build())
        f32, i64, i32 = ctypes.c_float, ctypes.c_int64, ctypes.c_int
        p = ctypes.c_void_p
        sig = {
            "or_quant_act": [p, i64, i64, i32, i64, p, p],
            "or_rmsnorm_quant": [p, p, i64, i64, f32, i32, p, p],
            "or_silu_mul_quant": [p, p, i64, i64, i32, p, p],
            "or_quantize_fp8_block": [p, i64, i64, p, p],
            "or_block_gemm": [p, p, i32, p, p, i32, p, i64, i64, i64, i32, i32, i32, p, p, p],
            "or_adaln": [p, p, p, i64, i64, i64, f32, p],
            "or_adaln_quant": [p, p, p, i64, i64, i64, f32, p, p],
            "or_gated_residual": [p, p, p, i64, i64, i64, p],
            "or_gated_residual_adaln_quant": [p, p, p, p, p, i64, i64, i64, f32, p, p, p],
            "or_qk_norm_rope": [p, p, p, p, i64, i64, i64, i64, f32, p],
            "or_pixelumm_qk": [p, p, p, p, p, i64, i64, i64, f32, p],
            "or_quantize_kv": [p, i64, i64, p, p],
            "or_dequantize_kv": [p, p, i64, i64, p],
            "or_round_bf16": [p, i64, p],
            "or_expf_array": [p, i64, p],
            "or_gelu_array": [p, i64, p],
        }
        for name, args in sig.items():
            fn = getattr(_lib, name)
            fn.argtypes = args
            fn.restype = None
        _lib.or_e4m3_from_f32.argtypes = [f32]
        _lib.or_e4m3_from_f32.restype = ctypes.c_uint8
        _lib.or_expf.argtypes = [f32]
        _lib.or_expf.restype = f32
    return _lib


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


# --------------------------------------------------------------------------------------------------------
# bf16 helpers (bf16 arrays are carried as uint16 bit patterns or as bf16-valued float32)


def round_bf16(x):
    """fp32 -> nearest-even bf16, returned as float32 (hy_nomas/kernels.py:67-71)."""
    x = _f32(x)
    y = np.empty_like(x)
    lib().or_round_bf16(_ptr(x), x.size, _ptr(y))
    return y


def bf16_bits(x):
    """bf16-valued float32 -> uint16 bit patterns."""
    return (_f32(x).view(np.uint32) >> 16).astype(np.uint16)


def from_bf16_bits(b):
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def e4m3_to_f32(b):
    """float8_e4m3fn bytes -> float32 values."""
    b = np.asarray(b, dtype=np.uint8)
    s = (b >> 7).astype(np.int32)
    e = ((b >> 3) & 15).astype(np.int32)
    m = (b & 7).astype(np.float32)
    v = np.where(e == 0, np.ldexp(m, -9), np.ldexp(1.0 + m / 8.0, e - 7)).astype(np.float32)
    v = np.where((e == 15) & (b & 7 == 7), np.float32(np.nan), v)
    return np.where(s == 1, -v, v).astype(np.float32)


def expf(x):
    x = _f32(x)
    y = np.empty_like(x)
    lib().or_expf_array(_ptr(x), x.size, _ptr(y))
    return y


def gelu_tanh(x):
    x = _f32(x)
    y = np.empty_like(x)
    lib().or_gelu_array(_ptr(x), x.size, _ptr(y))
    return y


# --------------------------------------------------------------------------------------------------------
# the path


def quantize_activations(x, kind="int8", per_row=False, round_half_even=False):
    """hy_nomas/kernels.py:45-54. x float32 [M, K] -> (codes uint8 [M, K] (int8 bits or e4m3 bytes),
    scales float32 [M, K/128] or [M, 1] per row). round_half_even: int8 codes rounded half to even (torch.round's
    convention) instead of the reference's half away from zero."""
    x = _f32(x)
    m, k = x.shape
    group = k if per_row else GROUP
    q = np.empty((m, k), dtype=np.uint8)
    s = np.empty((m, k // group), dtype=np.float32)
    code = (2 if round_half_even else 0) if kind == "int8" else 1
    lib().or_quant_act(_ptr(x), m, k, code, group, _ptr(q), _ptr(s))
    return q, s


def quantize_g128(w):
    """hy_nomas/ops.py:41-52 (K % 128 == 0). w float32 [N, K] -> (int8 [N, K], float32 [N, K/128])."""
    q, s = quantize_activations(w, "int8")
    return q.view(np.int8), s


def dequantize_g128(q, s):
    """hy_nomas/ops.py:55-62: fp32 product, one bf16 rounding. Returns bf16-valued float32."""
    n, k = q.shape
    w = (q.astype(np.float32).reshape(n, k // GROUP, GROUP) * s[:, :, None].astype(np.float32)).reshape(n, k)
    return round_bf16(w)


def quantize_fp8_block(w):
    """hy_nomas/pixelumm.py:77-82. w float32 [N, K] -> (e4m3 bytes [N, K], float32 [N/128, K/128])."""
    w = _f32(w)
    n, k = w.shape
    q = np.empty((n, k), dtype=np.uint8)
    s = np.empty((n // 128, k // 128), dtype=np.float32)
    lib().or_quantize_fp8_block(_ptr(w), n, k, _ptr(q), _ptr(s))
    return q, s


def dequantize_fp8_block(q, s):
    """hy_nomas/pixelumm.py:60-63. Returns bf16-valued float32."""
    n, k = q.shape
    w = e4m3_to_f32(q).reshape(n // 128, 128, k // 128, 128) * s[:, None, :, None]
    return round_bf16(w.reshape(n, k))


SCALE_MODES = {"group": 0, "row": 1, "block": 2}
EPILOGUES = {None: 0, "gelu": 1, "gelu_quant": 2}


def block_gemm(qa, sa, qw, sw, bias=None, kind="int8", epilogue=None, sa_mode="group", sw_mode="group", fma=True):
    """hy_nomas/kernels.py:80-137. Returns fp32 [M, N]: the accumulator after bias (epilogue None) or the
    bf16-valued GELU output; with "gelu_quant" returns (h, codes int8 [M, N], scales [M, N/128]).
    `fma=False` gives the interpreter's separate roundings of kernels.py:115."""
    qa = np.ascontiguousarray(qa).view(np.uint8)
    qw = np.ascontiguousarray(qw).view(np.uint8)
    m, k = qa.shape
    n = qw.shape[0]
    sa = _f32(sa)
    sw = _f32(sw)
    b = None if bias is None else _f32(bias)
    out = np.empty((m, n), dtype=np.float32)
    ep = EPILOGUES[epilogue]
    qh = np.zeros((m, n), dtype=np.int8) if ep == 2 else None
    qs = np.zeros((m, max(n // 128, 1)), dtype=np.float32) if ep == 2 else None
    lib().or_block_gemm(_ptr(qa), _ptr(sa), SCALE_MODES[sa_mode], _ptr(qw), _ptr(sw), SCALE_MODES[sw_mode],
                        _ptr(b), m, n, k, 0 if kind == "int8" else 1, ep, 1 if fma else 0, _ptr(out), _ptr(qh),
                        _ptr(qs))
    if ep == 2:
        return out, qh, qs
    return out


def int32_gemm(qa, qw):
    """The exact integer accumulator sum_k qa*qw (numpy int64), for bit-exact int32 checks."""
    return qa.astype(np.int64) @ qw.astype(np.int64).T


def adaln(x, shift, scale, eps=1e-6):
    """hy_nomas/fused.py:37-62. x float32 [B, L, D] (bf16-valued), shift/scale [B, D] -> fp32 (pre-store)."""
    x = _f32(x)
    b, l, d = x.shape
    y = np.empty_like(x)
    lib().or_adaln(_ptr(x), _ptr(_f32(shift)), _ptr(_f32(scale)), b, l, d, eps, _ptr(y))
    return y


def adaln_quant(x, shift, scale, eps=1e-6):
    """hy_nomas/kernels.py:198-207. -> (int8 [B*L, D], float32 [B*L, D/128])."""
    x = _f32(x)
    b, l, d = x.shape
    q = np.empty((b * l, d), dtype=np.int8)
    s = np.empty((b * l, d // GROUP), dtype=np.float32)
    lib().or_adaln_quant(_ptr(x), _ptr(_f32(shift)), _ptr(_f32(scale)), b, l, d, eps, _ptr(q), _ptr(s))
    return q, s


def gated_residual(x, y, gate):
    """hy_nomas/fused.py:121-128 -> fp32 (pre-store; round_bf16 gives the stored value)."""
    x = _f32(x)
    b, l, d = x.shape
    out = np.empty_like(x)
    lib().or_gated_residual(_ptr(x), _ptr(_f32(y)), _ptr(_f32(gate)), b, l, d, _ptr(out))
    return out


def gated_residual_adaln_quant(x, y, gate, shift, scale, eps=1e-6):
    """model.py:280-282 fused -> (x_out bf16-valued fp32, int8 codes, scales)."""
    x = _f32(x)
    b, l, d = x.shape
    xo = np.empty_like(x)
    q = np.empty((b * l, d), dtype=np.int8)
    s = np.empty((b * l, d // GROUP), dtype=np.float32)
    lib().or_gated_residual_adaln_quant(_ptr(x), _ptr(_f32(y)), _ptr(_f32(gate)), _ptr(_f32(shift)),
                                        _ptr(_f32(scale)), b, l, d, eps, _ptr(xo), _ptr(q), _ptr(s))
    return xo, q, s


def qk_norm_rope(x, weight, rope=None, eps=1e-6):
    """hy_nomas/fused.py:94-105. x float32 [B, L, H, D] -> bf16-valued float32 [B, L, H, D]."""
    x = _f32(x)
    b, l, h, d = x.shape
    y = np.empty_like(x)
    cos, sin = (None, None) if rope is None else (_f32(rope[0]), _f32(rope[1]))
    lib().or_qk_norm_rope(_ptr(x), _ptr(_f32(weight)), _ptr(cos), _ptr(sin), b, l, h, d, eps, _ptr(y))
    return y


def pixelumm_qk(x, weight_t, weight_hw, cos, sin, eps=1e-6):
    """hy_nomas/fused.py:178-186. x float32 [1, N, H, D] -> bf16-valued float32."""
    x = _f32(x)
    _, n, h, d = x.shape
    y = np.empty_like(x)
    lib().or_pixelumm_qk(_ptr(x), _ptr(_f32(weight_t)), _ptr(_f32(weight_hw)), _ptr(_f32(cos)), _ptr(_f32(sin)),
                         n, h, d, eps, _ptr(y))
    return y


def rmsnorm_quant(x, weight, eps=1e-6, kind="fp8"):
    """The PixelUMM decoder's RMSNorm (hy_nomas/pixelumm.py:246-259) and the activation quantizer of the linears
    that read it (kernels.py:22-42). x [rows, D] bf16 values as float32, weight [D] -> (codes uint8 [rows, D],
    float32 scales [rows, D / 128])."""
    x = _f32(x)
    rows, d = x.shape
    q = np.empty((rows, d), dtype=np.uint8)
    s = np.empty((rows, d // GROUP), dtype=np.float32)
    lib().or_rmsnorm_quant(_ptr(x), _ptr(_f32(weight)), rows, d, eps, 0 if kind == "int8" else 1, _ptr(q), _ptr(s))
    return q, s


def silu_mul_quant(g, u, kind="fp8"):
    """silu(gate) * up of the decoder MLP (hy_nomas/pixelumm.py:322-323) and down_proj's activation quantizer.
    g, u [rows, I] bf16 values as float32 -> (codes uint8 [rows, I], float32 scales [rows, I / 128])."""
    g, u = _f32(g), _f32(u)
    rows, i = g.shape
    q = np.empty((rows, i), dtype=np.uint8)
    s = np.empty((rows, i // GROUP), dtype=np.float32)
    lib().or_silu_mul_quant(_ptr(g), _ptr(u), rows, i, 0 if kind == "int8" else 1, _ptr(q), _ptr(s))
    return q, s


def quantize_kv(x):
    """hy_nomas/world.py:83-90. x float32 [L, H, D] -> (int8 [L, H, D], float32 [L, H, 1])."""
    x = _f32(x)
    l, h, d = x.shape
    q = np.empty((l, h, d), dtype=np.int8)
    s = np.empty((l, h, 1), dtype=np.float32)
    lib().or_quantize_kv(_ptr(x), l * h, d, _ptr(q), _ptr(s))
    return q, s


def dequantize_kv(q, s):
    """hy_nomas/world.py:93-94. int8 [..., D] and float32 scales [..., 1] -> bf16 values as float32 [..., D]."""
    q = np.ascontiguousarray(q, dtype=np.int8)
    s = np.ascontiguousarray(s, dtype=np.float32)
    d = q.shape[-1]
    y = np.empty(q.shape, dtype=np.float32)
    lib().or_dequantize_kv(_ptr(q), _ptr(s), q.size // d, d, _ptr(y))
    return y
