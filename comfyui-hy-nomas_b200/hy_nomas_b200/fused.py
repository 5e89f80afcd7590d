"""Fused elementwise kernels of the DiT block - the drop-in for hy_nomas/fused.py.

Same functions and arguments as the reference (hy_nomas/fused.py:22-186); each is one HBM pass in
libhynomas_b200.so and rounds where the reference rounds:

* `adaln`: LayerNorm in fp32, `* rbf16(1 + scale)`, `+ shift`, one bf16 rounding;
* `qk_norm_rope`: RMSNorm in fp32 rounded to bf16, times the bf16 weight (rounded), interleaved RoPE in fp32,
  rounded;
* `gated_residual`: `x + y * gate`, the product and the sum each rounded to bf16;
* `pixelumm_qk`: PixelUMM's split T/HW RMSNorm + rotate-half MRoPE.

Two fused variants go further than the reference: `gated_residual_adaln_quant` (the residual and the next
LayerNorm/modulate/int8 quantization in one pass, hy_nomas/model.py:280-282) and `qk_norm_rope2` (q and k
in one launch, reading the RoPE tables once). For the PixelUMM decoder, `rmsnorm_quant` and `silu_mul_quant`
are the RMSNorm and SiLU fusions the reference's notes name (README.md:266): each ends in the activation
quantizer of the FP8 linears that read its output, so neither writes its bf16 result. `HY_NOMAS_FUSED=0` disables `available()`, as in the
reference.
"""
import os

import torch

from . import _lib

ENABLED = os.environ.get("HY_NOMAS_FUSED", "1") != "0"


def available(x):
    return ENABLED and x.is_cuda and x.dtype == torch.bfloat16


def _bf16(*ts):
    for t in ts:
        if t.dtype != torch.bfloat16:
            raise TypeError(f"expected a bf16 tensor, got {t.dtype}")


def adaln(x, shift, scale, eps=1e-6):
    """x [B, L, D] bf16, shift/scale [B, D] bf16 -> modulate(layer_norm(x), shift, scale) in bf16."""
    _lib.require_cuda(x, shift, scale)
    _bf16(x, shift, scale)
    b, l, d = x.shape
    x, shift, scale = _lib.dense(x), _lib.dense(shift), _lib.dense(scale)
    y = torch.empty(x.shape, device=x.device, dtype=x.dtype)
    rc = _lib.lib.hn_adaln(_lib.ptr(x), _lib.ptr(shift), _lib.ptr(scale), b, l, d, eps, _lib.ptr(y),
                           _lib.stream_of(x))
    _lib.check(rc, "adaln")
    return y


def _qk_input(x):
    b, l, h, d = x.shape
    if x.stride(3) != 1 or x.stride(2) != d or x.stride(0) != l * x.stride(1) or x.stride(1) % 8 or \
            x.data_ptr() % 16:
        x = _lib.dense(x)
    return x


def _rope_tables(rope, device):
    if rope is None:
        return None, None
    cos, sin = rope
    cos = _lib.dense(cos.to(device=device, dtype=torch.float32))
    sin = _lib.dense(sin.to(device=device, dtype=torch.float32))
    return cos, sin


def qk_norm_rope(x, weight, rope=None, eps=1e-6, out=None):
    """x [B, L, H, D] bf16 (rows may be strided, heads contiguous), weight [D] -> RMSNorm(x) * weight, then RoPE
    with (cos, sin) [L, D] fp32 when given. Returns a contiguous [B, L, H, D] bf16 tensor (`out`, when given:
    a caller-owned contiguous bf16 tensor of that shape)."""
    _lib.require_cuda(x, weight)
    _bf16(x)
    b, l, h, d = x.shape
    x = _qk_input(x)
    if out is None:
        y = torch.empty((b, l, h, d), device=x.device, dtype=torch.bfloat16)
    else:
        y = out
        if y.shape != (b, l, h, d) or y.dtype != torch.bfloat16 or not y.is_contiguous() or y.device != x.device:
            raise ValueError(f"qk_norm_rope: out must be a contiguous bf16 [{b}, {l}, {h}, {d}] tensor")
    w = _lib.dense(weight.to(torch.bfloat16))
    cos, sin = _rope_tables(rope, x.device)
    rc = _lib.lib.hn_qk_norm_rope(_lib.ptr(x), x.stride(1), _lib.ptr(w), _lib.ptr(cos), _lib.ptr(sin), b, l, h, d,
                                  eps, _lib.ptr(y), _lib.stream_of(x))
    _lib.check(rc, "qk_norm_rope")
    return y


def qk_norm_rope_kv(x, weight, rope=None, eps=1e-6, out=None):
    """`qk_norm_rope` for the cache pass: returns (y, q, s) where y is qk_norm_rope's output and (q, s) is
    world.quantize_kv(y) from the same launch - int8 [B, L, H, D] and fp32 [B, L, H, 1] per (token, head)."""
    _lib.require_cuda(x, weight)
    _bf16(x)
    b, l, h, d = x.shape
    x = _qk_input(x)
    if out is None:
        y = torch.empty((b, l, h, d), device=x.device, dtype=torch.bfloat16)
    else:
        y = out
        if y.shape != (b, l, h, d) or y.dtype != torch.bfloat16 or not y.is_contiguous() or y.device != x.device:
            raise ValueError(f"qk_norm_rope_kv: out must be a contiguous bf16 [{b}, {l}, {h}, {d}] tensor")
    q = torch.empty((b, l, h, d), device=x.device, dtype=torch.int8)
    s = torch.empty((b, l, h, 1), device=x.device, dtype=torch.float32)
    w = _lib.dense(weight.to(torch.bfloat16))
    cos, sin = _rope_tables(rope, x.device)
    rc = _lib.lib.hn_qk_norm_rope_kv(_lib.ptr(x), x.stride(1), _lib.ptr(w), _lib.ptr(cos), _lib.ptr(sin), b, l, h, d,
                                     eps, _lib.ptr(y), _lib.ptr(q), _lib.ptr(s), _lib.stream_of(x))
    _lib.check(rc, "qk_norm_rope_kv")
    return y, q, s


def qk_norm_rope2(q, k, weight_q, weight_k, rope=None, eps=1e-6, out=None):
    """`qk_norm_rope` of q and k (same shape and token stride) in one launch -> (q_out, k_out). `out`: optional
    caller-owned contiguous bf16 [B, L, H, D] pair to write into (e.g. a rank's slice of an all-gather buffer)."""
    _lib.require_cuda(q, k, weight_q, weight_k)
    _bf16(q, k)
    b, l, h, d = q.shape
    q, k = _qk_input(q), _qk_input(k)
    if q.stride(1) != k.stride(1):
        q, k = _lib.dense(q), _lib.dense(k)
    if out is None:
        yq = torch.empty((b, l, h, d), device=q.device, dtype=torch.bfloat16)
        yk = torch.empty_like(yq)
    else:
        yq, yk = out
        for y in (yq, yk):
            if y.shape != (b, l, h, d) or y.dtype != torch.bfloat16 or not y.is_contiguous() or y.device != q.device:
                raise ValueError(f"qk_norm_rope2: out tensors must be contiguous bf16 [{b}, {l}, {h}, {d}]")
    wq = _lib.dense(weight_q.to(torch.bfloat16))
    wk = _lib.dense(weight_k.to(torch.bfloat16))
    cos, sin = _rope_tables(rope, q.device)
    rc = _lib.lib.hn_qk_norm_rope2(_lib.ptr(q), _lib.ptr(k), q.stride(1), _lib.ptr(wq), _lib.ptr(wk), _lib.ptr(cos),
                                   _lib.ptr(sin), b, l, h, d, eps, _lib.ptr(yq), _lib.ptr(yk), _lib.stream_of(q))
    _lib.check(rc, "qk_norm_rope2")
    return yq, yk


def gated_residual(x, y, gate):
    """x + y * gate[:, None] with bf16 rounding of the product and the sum; x, y [B, L, D], gate [B, D]."""
    _lib.require_cuda(x, y, gate)
    _bf16(x, y, gate)
    b, l, d = x.shape
    x, y, gate = _lib.dense(x), _lib.dense(y), _lib.dense(gate)
    out = torch.empty(x.shape, device=x.device, dtype=x.dtype)
    rc = _lib.lib.hn_gated_residual(_lib.ptr(x), _lib.ptr(y), _lib.ptr(gate), b, l, d, _lib.ptr(out),
                                    _lib.stream_of(x))
    _lib.check(rc, "gated_residual")
    return out


def gated_residual_adaln_quant(x, y, gate, shift, scale, eps=1e-6):
    """x' = gated_residual(x, y, gate) and kernels.adaln_quant(x', shift, scale) in one pass -> (x', q, s)."""
    _lib.require_cuda(x, y, gate, shift, scale)
    _bf16(x, y, gate, shift, scale)
    b, l, d = x.shape
    x, y, gate = _lib.dense(x), _lib.dense(y), _lib.dense(gate)
    shift, scale = _lib.dense(shift), _lib.dense(scale)
    out = torch.empty(x.shape, device=x.device, dtype=x.dtype)
    q = torch.empty((b * l, d), device=x.device, dtype=torch.int8)
    s, srs, sgs = _lib.group_scales(b * l, d // 128, x.device)
    rc = _lib.lib.hn_gated_residual_adaln_quant(_lib.ptr(x), _lib.ptr(y), _lib.ptr(gate), _lib.ptr(shift),
                                                _lib.ptr(scale), b, l, d, eps, _lib.ptr(out), _lib.ptr(q),
                                                _lib.ptr(s), srs, sgs, _lib.stream_of(x))
    _lib.check(rc, "gated_residual_adaln_quant")
    return out, q, s


def pixelumm_qk(x, weight_t, weight_hw, cos, sin, eps=1e-6):
    """x [1, N, H, D] (a projection's output, heads contiguous), cos/sin [N, D] fp32 -> bf16 [1, N, H, D]."""
    _lib.require_cuda(x, weight_t, weight_hw, cos, sin)
    _bf16(x)
    b, n, h, d = x.shape
    if b != 1:
        raise ValueError("pixelumm_qk: batch must be 1 (the decoder's layout)")
    if x.stride(3) != 1 or x.stride(2) != d or x.stride(1) % 4 or x.data_ptr() % 8:
        x = _lib.dense(x)
    y = torch.empty((b, n, h, d), device=x.device, dtype=torch.bfloat16)
    wt = _lib.dense(weight_t.to(torch.bfloat16))
    whw = _lib.dense(weight_hw.to(torch.bfloat16))
    cos = _lib.dense(cos.to(torch.float32))
    sin = _lib.dense(sin.to(torch.float32))
    rc = _lib.lib.hn_pixelumm_qk(_lib.ptr(x), x.stride(1), _lib.ptr(wt), _lib.ptr(whw), _lib.ptr(cos), _lib.ptr(sin),
                                 n, h, d, eps, _lib.ptr(y), _lib.stream_of(x))
    _lib.check(rc, "pixelumm_qk")
    return y


_KINDS = {"int8": (0, torch.int8), "fp8": (1, torch.float8_e4m3fn)}


def rmsnorm_quant(x, weight, eps=1e-6, kind="fp8"):
    """The decoder's RMSNorm (hy_nomas/pixelumm.py:246-259: normalize in fp32, cast to bf16, times the bf16
    weight) and the quantizer of the linears that read it (kernels.quantize_activations, as block_linear runs it
    for the FP8 decoder linears, pixelumm.py:147-155) in one pass: x [..., D] bf16 -> (codes [rows, D], fp32
    scales [rows, D / 128]), the normalized activations never written."""
    _lib.require_cuda(x, weight)
    _bf16(x)
    d = x.shape[-1]
    x2 = _lib.dense(x.reshape(-1, d))
    rows = x2.shape[0]
    code, dtype = _KINDS[kind]
    w = _lib.dense(weight.to(torch.bfloat16))
    q = torch.empty((rows, d), device=x.device, dtype=dtype)
    s, srs, sgs = _lib.group_scales(rows, d // 128, x.device)
    rc = _lib.lib.hn_rmsnorm_quant(_lib.ptr(x2), x2.stride(0), _lib.ptr(w), rows, d, eps, code, _lib.ptr(q),
                                   q.stride(0), _lib.ptr(s), srs, sgs, _lib.stream_of(x2))
    _lib.check(rc, "rmsnorm_quant")
    return q, s


def silu_mul_quant(gate, up, kind="fp8"):
    """silu(gate) * up of the decoder MLP (hy_nomas/pixelumm.py:322-323, with torch's bf16 roundings) and down_proj's
    activation quantizer in one pass: gate, up [rows, I] bf16 (rows may be strided, e.g. the two halves of one
    stacked gate|up GEMM output) -> (codes [rows, I], fp32 scales [rows, I / 128])."""
    _lib.require_cuda(gate, up)
    _bf16(gate, up)
    rows, i = gate.shape
    if up.shape != gate.shape:
        raise ValueError(f"silu_mul_quant: gate {tuple(gate.shape)} and up {tuple(up.shape)} differ")

    def rows_ok(t):
        return t.stride(1) == 1 and t.stride(0) % 8 == 0 and t.data_ptr() % 16 == 0
    g = gate if rows_ok(gate) else _lib.dense(gate)
    u = up if rows_ok(up) else _lib.dense(up)
    code, dtype = _KINDS[kind]
    q = torch.empty((rows, i), device=gate.device, dtype=dtype)
    s, srs, sgs = _lib.group_scales(rows, i // 128, gate.device)
    rc = _lib.lib.hn_silu_mul_quant(_lib.ptr(g), g.stride(0), _lib.ptr(u), u.stride(0), rows, i, code, _lib.ptr(q),
                                    q.stride(0), _lib.ptr(s), srs, sgs, _lib.stream_of(g))
    _lib.check(rc, "silu_mul_quant")
    return q, s
