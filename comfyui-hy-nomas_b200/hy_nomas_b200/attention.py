"""The DiT's attention on the B200 kernel (hy_nomas/model.py:145-151): out = softmax(q k^T * scale) v per batch
item and head, no mask, head dim 128, q/k/v and out in the reference's [B, L, H, D] layout.

`attention(q, k, v)` keeps the reference function's name, arguments and layout (`transformer_options` is
accepted and ignored: the B200 build has one backend). `attention_quant` is the fusion the block needs before
its projection linear: the output quantized per token x 128 channels - one head's row of the [B*Lq, H*128]
output - with the arithmetic of `kernels.quantize_activations` (int8, round half away), from the same launch.

`attention_lse` + `merge` attend in key pieces (the sequence-parallel step attends to each rank's keys as they
arrive): each piece is torch's cuDNN attention over a key range with its log-sum-exp, and the library's merge
kernel combines them exactly as one softmax over all keys would (up to rounding), optionally quantizing the result
for the projection linear in the same pass.
"""
import ctypes
import math

import torch

from . import _lib

HEAD_DIM = 128


def _check(q, k, v):
    _lib.require_cuda(q, k, v)
    for name, t in (("q", q), ("k", k), ("v", v)):
        if t.dtype != torch.bfloat16:
            raise TypeError(f"attention: {name} must be bf16, got {t.dtype}")
        if t.dim() != 4:
            raise ValueError(f"attention: {name} must be [B, L, H, D], got {tuple(t.shape)}")
    b, lq, h, d = q.shape
    if d != HEAD_DIM:
        raise ValueError(f"attention: head dim {d} (the kernel takes {HEAD_DIM})")
    if k.shape != v.shape or k.shape[0] != b or k.shape[2] != h or k.shape[3] != d:
        raise ValueError(f"attention: k {tuple(k.shape)} / v {tuple(v.shape)} do not match q {tuple(q.shape)}")


def _strides(t):
    """(row, head, batch) strides in elements; a dimension of extent 1 is never stepped, so it gets its
    contiguous stride whatever torch reports for it."""
    b, l, h, d = t.shape
    canon = (l * h * d, h * d, d)
    return tuple(t.stride(i) if t.shape[i] > 1 else canon[i] for i in range(3))


def _operand(t):
    """t itself when the head dim is contiguous and every stride is a multiple of 8 elements on a 16-byte
    aligned base (the TMA rules), else a dense copy."""
    if t.stride(3) == 1 and t.data_ptr() % 16 == 0 and all(s % 8 == 0 for s in _strides(t)):
        return t
    return _lib.dense(t)


def _launch(q, k, v, scale, out, q8, s8):
    b, lq, h, d = q.shape
    lk = k.shape[1]
    q, k, v = _operand(q), _operand(k), _operand(v)
    (qb, qr, qh), (kb, kr, kh), (vb, vr, vh) = _strides(q), _strides(k), _strides(v)
    ob, orow, oh = _strides(out) if out is not None else (0, 0, 0)
    rc = _lib.lib.hn_attention(
        _lib.ptr(q), qr, qh, qb, _lib.ptr(k), kr, kh, kb, _lib.ptr(v), vr, vh, vb, b, lq, lk, h, d, float(scale),
        _lib.ptr(out), orow, oh, ob, _lib.ptr(q8), _lib.ptr(s8), _lib.stream_of(q))
    _lib.check(rc, "attention")


def attention(q, k, v, transformer_options=None, scale=None, out=None):
    """q [B, Lq, H, 128], k / v [B, Lk, H, 128] bf16 -> [B, Lq, H, 128] bf16 (hy_nomas/model.py:145-151).
    `scale` defaults to 1/sqrt(128) as SDPA's does; `out` (not in the reference) is a caller-owned [B, Lq, H, 128]
    bf16 tensor with its head dim contiguous, written instead of a fresh tensor."""
    _check(q, k, v)
    scale = 1.0 / math.sqrt(q.shape[3]) if scale is None else scale
    if out is None:
        out = torch.empty(q.shape, dtype=torch.bfloat16, device=q.device)
    elif out.shape != q.shape or out.dtype != torch.bfloat16 or out.stride(3) != 1 or out.data_ptr() % 16 \
            or any(s % 8 for s in _strides(out)):
        raise ValueError("attention: out must be bf16 [B, Lq, H, 128], head dim contiguous, 16-byte aligned")
    _launch(q, k, v, scale, out, None, None)
    return out


def attention_quant(q, k, v, scale=None, keep_output=False):
    """Attention with its output quantized for the projection linear: returns (codes int8 [B*Lq, H*128], scales
    fp32 [B*Lq, H]) - bit-identical to `kernels.quantize_activations(attention(q, k, v).reshape(B*Lq, H*128))` -
    and, with `keep_output`, the bf16 output first: (out, (codes, scales))."""
    _check(q, k, v)
    b, lq, h, d = q.shape
    scale = 1.0 / math.sqrt(d) if scale is None else scale
    q8 = torch.empty((b * lq, h * d), dtype=torch.int8, device=q.device)
    s8 = torch.empty((b * lq, h), dtype=torch.float32, device=q.device)
    out = torch.empty(q.shape, dtype=torch.bfloat16, device=q.device) if keep_output else None
    _launch(q, k, v, scale, out, q8, s8)
    return (out, (q8, s8)) if keep_output else (q8, s8)


def attention_lse(q, k, v, scale=None):
    """Attention over these keys with its log-sum-exp: (o [B, Lq, H, 128] bf16, lse [B, H, Lq] fp32, natural log),
    torch's cuDNN kernel (the reference's pytorch backend runs the same through SDPA)."""
    r = torch.ops.aten._scaled_dot_product_cudnn_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                                            None, True, 0.0, False, False, scale=scale)
    o, lse = r[0].transpose(1, 2), r[1]
    if lse.dim() == 4:
        lse = lse[..., 0]
    return o, lse


def merge(pieces, quantize=True, keep_output=False):
    """Combine [(o_i, lse_i)] pieces of one attention (disjoint key ranges, same queries) into the attention over
    all their keys. Returns the projection input (codes int8 [B*Lq, H*128], scales fp32 [B*Lq, H]) when
    `quantize`, the bf16 output [B, Lq, H, 128] otherwise, and (out, (codes, scales)) with both."""
    if not 1 <= len(pieces) <= 16:
        raise ValueError(f"merge: {len(pieces)} pieces (1 to 16)")
    parts = [o for o, _ in pieces]
    lses = [l.float() for _, l in pieces]
    b, lq, h, d = parts[0].shape
    if d != HEAD_DIM:
        raise ValueError(f"merge: head dim {d}")
    st = parts[0].stride()
    if any(o.stride() != st or o.shape != parts[0].shape or o.dtype != torch.bfloat16 for o in parts) \
            or st[3] != 1 or any(x % 4 for x in st[:3]) or any(o.data_ptr() % 8 for o in parts):
        parts = [o.contiguous() for o in parts]
        st = parts[0].stride()
    lst = lses[0].stride()
    if any(l.stride() != lst or l.shape != (b, h, lq) for l in lses):
        lses = [l.reshape(b, h, lq).contiguous() for l in lses]
        lst = lses[0].stride()
    _lib.require_cuda(*parts, *lses)
    want_out = keep_output or not quantize
    out = torch.empty((b, lq, h, d), dtype=torch.bfloat16, device=parts[0].device) if want_out else None
    q8 = torch.empty((b * lq, h * d), dtype=torch.int8, device=parts[0].device) if quantize else None
    s8 = torch.empty((b * lq, h), dtype=torch.float32, device=parts[0].device) if quantize else None
    n = len(parts)
    pp = (ctypes.c_void_p * n)(*[o.data_ptr() for o in parts])
    lp = (ctypes.c_void_p * n)(*[l.data_ptr() for l in lses])
    ost = out.stride() if out is not None else (0, 0, 0)
    rc = _lib.lib.hn_attn_merge(pp, lp, n, st[0], st[1], st[2], lst[0], lst[1], lst[2], b, lq, h, d,
                                _lib.ptr(out), ost[0], ost[1], ost[2], _lib.ptr(q8), _lib.ptr(s8),
                                _lib.stream_of(parts[0]))
    _lib.check(rc, "attn_merge")
    if quantize and keep_output:
        return out, (q8, s8)
    return (q8, s8) if quantize else out
