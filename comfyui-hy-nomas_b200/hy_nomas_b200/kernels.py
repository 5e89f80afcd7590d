"""Block-scaled W8A8 / FP8 linears on the B200 tensor cores - the drop-in for hy_nomas/kernels.py.

Same functions, arguments, shapes and dtypes as the reference module (hy_nomas/kernels.py:19-226):

    y[m, n] = sum_g  a_scale[m, g] * w_scale[n, g] * sum_{k in g} qa[m, k] * qw[n, k]   (+ bias[n])

with one scale per token and 128 channels for the activations (absmax/127, round half away from zero for
int8; absmax/448 for e4m3) and the checkpoint's weight scales. The work runs in libhynomas_b200.so
(tcgen05 tensor-core GEMM with the scale promotion, bias, GELU and requantization fused into its
epilogue); this module only allocates outputs with torch and passes pointers.

Beyond the reference's layouts, `block_gemm` also takes per-row scales (a_scale [M] per token, w_scale [N]
per output channel) and 128x128 weight-block scales [N/128, K/128] (the FP8 decoder's stored layout), and
`quantize_activations(..., per_token=True)` quantizes with one scale per row.
"""
import torch

from . import _lib

GROUP = 128
EPILOGUES = {None: 0, "gelu": 1, "gelu_quant": 2}


def _aligned(t):
    return t.data_ptr() % 16 == 0 and (t.stride(0) * t.element_size()) % 16 == 0 and t.stride(-1) == 1


def quantize_activations(x, kind="int8", per_token=False, round_half_even=False):
    """x [M, K] (K % 128 == 0) -> codes [M, K] and fp32 scales [M, K / 128] (hy_nomas/kernels.py:45-54).
    `per_token=True`: one scale per row, scales [M, 1]. `round_half_even=True` (int8): codes rounded half to
    even instead of the reference's half away from zero (torch.round's convention)."""
    _lib.require_cuda(x)
    m, k = x.shape
    if x.dtype not in (torch.bfloat16, torch.float16, torch.float32):
        x = x.float()
    if not _aligned(x):
        x = _lib.dense(x)
    dtype = torch.int8 if kind == "int8" else torch.float8_e4m3fn
    q = torch.empty((m, k), device=x.device, dtype=dtype)
    if per_token:
        s = torch.empty((m, 1), device=x.device, dtype=torch.float32)
        srs, sgs = 1, 1
    else:
        s, srs, sgs = _lib.group_scales(m, k // GROUP, x.device)
    flags = (1 if per_token else 0) | (2 if round_half_even else 0)
    rc = _lib.lib.hn_quant_act(_lib.ptr(x), x.stride(0), _lib.DTYPE[x.dtype], m, k, _lib.KIND[kind], flags,
                               _lib.ptr(q), q.stride(0), _lib.ptr(s), srs, sgs, _lib.stream_of(x))
    _lib.check(rc, "quantize_activations")
    return q, s


def _scale_mode(s, rows, k, weight):
    """Classify a scale tensor: 'group' [rows, K/128], 'row' [rows] or [rows, 1], 'block' [rows/128, K/128]."""
    g = k // GROUP
    if s.dim() == 1 or (s.dim() == 2 and s.shape[1] == 1 and g != 1):
        if s.shape[0] != rows:
            raise ValueError(f"scale shape {tuple(s.shape)} does not match {rows} rows")
        return "row"
    if s.shape == (rows, g):
        return "group"
    if weight and s.shape == ((rows + 127) // 128, g):
        return "block"
    raise ValueError(f"scale shape {tuple(s.shape)} is none of [{rows}, {g}], [{rows}], [{(rows + 127) // 128}, {g}]")


def block_gemm(qa, sa, qw, sw, bias=None, out_dtype=torch.bfloat16, kind="int8", epilogue=None, out=None):
    """Block-scaled GEMM on quantized activations (hy_nomas/kernels.py:152-170). With epilogue "gelu_quant"
    returns (int8 [M, N], scales [M, N / 128]) ready for the next int8 linear; otherwise [M, N] in
    `out_dtype` (bf16, fp16, fp32; torch.int32 gives the raw int32 accumulator when both scales are per
    row and there is no bias).

    `out` (not in the reference): a caller-owned [M, N] destination with unit column stride (rows may be
    strided, e.g. a slice of a larger buffer), written instead of a fresh tensor; epilogues None and "gelu"."""
    _lib.require_cuda(qa, sa, qw, sw, bias)
    m, k = qa.shape
    n = qw.shape[0]
    mode = EPILOGUES[epilogue]
    sa_mode = _scale_mode(sa, m, k, weight=False)
    sw_mode = _scale_mode(sw, n, k, weight=True)
    if sa.dtype != torch.float32:
        sa = sa.float()
    if sw.dtype != torch.float32:
        sw = sw.float()
    if not _aligned(qa):
        qa = _lib.dense(qa)
    if not _aligned(qw):
        qw = _lib.dense(qw)
    if bias is not None and (bias.stride(0) != 1 or bias.data_ptr() % 16):
        bias = _lib.dense(bias)
    if mode == 2:
        if out is not None:
            raise ValueError("block_gemm: `out` is not supported with epilogue 'gelu_quant'")
        out = torch.empty((m, n), device=qa.device, dtype=torch.int8)
        qs, qrs, qgs = _lib.group_scales(m, n // GROUP, qa.device)
    else:
        want = out_dtype if mode == 0 else torch.bfloat16
        if out is None:
            out = torch.empty((m, n), device=qa.device, dtype=want)
        elif out.shape != (m, n) or out.dtype != want or out.stride(1) != 1 or out.device != qa.device:
            raise ValueError(f"block_gemm: out must be a {want} [{m}, {n}] tensor with unit column stride on "
                             f"{qa.device}")
        qs, qrs, qgs = None, 0, 0
    sa_rs, sa_gs = _lib.scale_strides(sa)
    sw_rs, sw_gs = _lib.scale_strides(sw)
    rc = _lib.lib.hn_block_gemm(
        _lib.ptr(qa), qa.stride(0), _lib.ptr(sa), sa_rs, sa_gs, _lib.SCALE_MODE[sa_mode],
        _lib.ptr(qw), qw.stride(0), _lib.ptr(sw), sw_rs, sw_gs, _lib.SCALE_MODE[sw_mode],
        _lib.ptr(bias), _lib.DTYPE[bias.dtype] if bias is not None else 0,
        _lib.ptr(out), out.stride(0), _lib.DTYPE[out.dtype] if mode != 2 else 0,
        _lib.ptr(qs), qrs, qgs,
        m, n, k, _lib.KIND[kind], mode, _lib.stream_of(qa))
    _lib.check(rc, "block_gemm")
    return (out, qs) if mode == 2 else out


def adaln_quant(x, shift, scale, eps=1e-6):
    """x [B, L, D] bf16, shift/scale [B, D] -> int8 codes [B * L, D] and scales [B * L, D / 128] of the modulated
    LayerNorm, for the q/k/v linears (hy_nomas/kernels.py:198-207)."""
    _lib.require_cuda(x, shift, scale)
    b, l, d = x.shape
    if x.dtype != torch.bfloat16 or shift.dtype != torch.bfloat16 or scale.dtype != torch.bfloat16:
        raise TypeError("adaln_quant: x, shift and scale must be bf16")
    x, shift, scale = _lib.dense(x), _lib.dense(shift), _lib.dense(scale)
    q = torch.empty((b * l, d), device=x.device, dtype=torch.int8)
    s, srs, sgs = _lib.group_scales(b * l, d // GROUP, x.device)
    rc = _lib.lib.hn_adaln_quant(_lib.ptr(x), _lib.ptr(shift), _lib.ptr(scale), b, l, d, eps, _lib.ptr(q),
                                 _lib.ptr(s), srs, sgs, _lib.stream_of(x))
    _lib.check(rc, "adaln_quant")
    return q, s


def block_linear(x, qw, sw, bias=None, kind="int8"):
    """F.linear with block-scaled 8-bit weights: x [..., K] -> [..., N] in x's dtype (hy_nomas/kernels.py:210-222).
    As in the reference, K % 128 != 0 or an empty input takes the dequantized bf16 linear."""
    _lib.require_cuda(x)
    shape = x.shape
    x2 = x.reshape(-1, shape[-1])
    if shape[-1] % GROUP or x2.shape[0] == 0:
        from .ops import dequantize_g128
        return torch.nn.functional.linear(x, dequantize_g128(qw, sw, x.dtype), bias)
    with torch.cuda.device(x.device):
        qa, sa = quantize_activations(x2, kind)
        out = block_gemm(qa, sa, qw, sw.float(), bias, x.dtype, kind)
    return out.reshape(*shape[:-1], qw.shape[0])


def int8_g128_linear(x, qw, sw, bias=None):
    """hy_nomas/kernels.py:225-226."""
    return block_linear(x, qw, sw, bias, kind="int8")
