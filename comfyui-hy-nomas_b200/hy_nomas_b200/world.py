"""The int8 KV cache of the world model's segment history (hy_nomas/world.py:80-94), on the B200 kernels.

`quantize_kv` / `dequantize_kv` keep the reference's names, shapes and arithmetic: absmax per (token, head)
over the head dimension, scale absmax/127 (1 for an all-zero head), codes rounded half away from zero and
clamped to +-127; dequantization is bf16(float(q) * scale). `fused.qk_norm_rope_kv` produces the same codes
for the cache pass straight from QK-norm + RoPE.
"""
import torch

from . import _lib


def quantize_kv(x):
    """x [L, H, D] bf16 (D % 128 == 0) -> (int8 [L, H, D], fp32 scale [L, H, 1]) (hy_nomas/world.py:83-90)."""
    _lib.require_cuda(x)
    if x.dtype != torch.bfloat16:
        raise TypeError(f"quantize_kv: bf16 input expected, got {x.dtype}")
    l, h, d = x.shape
    x = _lib.dense(x)
    q = torch.empty((l, h, d), device=x.device, dtype=torch.int8)
    s = torch.empty((l, h, 1), device=x.device, dtype=torch.float32)
    rc = _lib.lib.hn_quantize_kv(_lib.ptr(x), l * h, d, _lib.ptr(q), _lib.ptr(s), _lib.stream_of(x))
    _lib.check(rc, "quantize_kv")
    return q, s


def dequantize_kv(q, scale, dtype=torch.bfloat16, out=None):
    """int8 [..., D] codes and fp32 scales [..., 1] -> bf16(float(q) * scale) (hy_nomas/world.py:93-94).
    `out` (not in the reference): a caller-owned contiguous bf16 tensor with q's number of elements, e.g. the
    history part of a block's K or V buffer, written instead of a fresh tensor."""
    _lib.require_cuda(q, scale)
    if dtype != torch.bfloat16:
        raise TypeError("dequantize_kv: the kernel writes bf16 (the reference's default dtype)")
    d = q.shape[-1]
    rows = q.numel() // d if d else 0
    q = _lib.dense(q)
    s = _lib.dense(scale.to(torch.float32))
    if s.numel() != rows:
        raise ValueError(f"dequantize_kv: {s.numel()} scales for {rows} rows")
    if out is None:
        y = torch.empty(q.shape, device=q.device, dtype=torch.bfloat16)
    elif out.dtype != torch.bfloat16 or not out.is_contiguous() or out.numel() != q.numel() or out.device != q.device \
            or out.data_ptr() % 16:
        raise ValueError("dequantize_kv: out must be a contiguous, 16-byte aligned bf16 tensor of q's size on q's device")
    else:
        y = out
    rc = _lib.lib.hn_dequantize_kv(_lib.ptr(q), _lib.ptr(s), rows, d, _lib.ptr(y), _lib.stream_of(q))
    _lib.check(rc, "dequantize_kv")
    return y
