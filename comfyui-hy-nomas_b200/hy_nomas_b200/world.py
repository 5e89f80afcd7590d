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


def dequantize_kv(q, scale, dtype=torch.bfloat16):
    """int8 [..., D] codes and fp32 scales [..., 1] -> bf16(float(q) * scale) (hy_nomas/world.py:93-94)."""
    _lib.require_cuda(q, scale)
    if dtype != torch.bfloat16:
        raise TypeError("dequantize_kv: the kernel writes bf16 (the reference's default dtype)")
    d = q.shape[-1]
    rows = q.numel() // d if d else 0
    q = _lib.dense(q)
    s = _lib.dense(scale.to(torch.float32))
    if s.numel() != rows:
        raise ValueError(f"dequantize_kv: {s.numel()} scales for {rows} rows")
    y = torch.empty(q.shape, device=q.device, dtype=torch.bfloat16)
    rc = _lib.lib.hn_dequantize_kv(_lib.ptr(q), _lib.ptr(s), rows, d, _lib.ptr(y), _lib.stream_of(q))
    _lib.check(rc, "dequantize_kv")
    return y
