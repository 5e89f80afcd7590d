"""Tencent's per-row x 128-group int8 weight layout - the drop-in for the arithmetic of hy_nomas/ops.py.

`quantize_g128` runs the activation quantizer kernel of libhynomas_b200.so on the weight (the same
absmax/127, round-half-away arithmetic: hy_nomas/ops.py:41-52) and needs a CUDA tensor. `dequantize_g128`
is the reference's plain tensor expression (hy_nomas/ops.py:55-62), used by block_linear for shapes the
GEMM does not take (K % 128 != 0). The ComfyUI layout registration and the Linear module of the reference
file are ComfyUI wiring, not part of this path.
"""
import torch
import torch.nn.functional as F

from . import _lib

GROUP = 128


def quantize_g128(weight):
    """Symmetric per-row, per-128-column-group int8, half away from zero -> (int8 [N, K], fp32 [N, ceil(K/128)])."""
    _lib.require_cuda(weight)
    n, k = weight.shape
    groups = (k + GROUP - 1) // GROUP
    w = weight.float()
    if k % GROUP:
        w = F.pad(w, (0, groups * GROUP - k))
    w = w.contiguous()
    q = torch.empty((n, groups * GROUP), device=w.device, dtype=torch.int8)
    s, srs, sgs = _lib.group_scales(n, groups, w.device)
    rc = _lib.lib.hn_quant_act(_lib.ptr(w), w.stride(0), _lib.DTYPE[torch.float32], n, groups * GROUP,
                               _lib.KIND["int8"], 0, _lib.ptr(q), q.stride(0), _lib.ptr(s), srs, sgs,
                               _lib.stream_of(w))
    _lib.check(rc, "quantize_g128")
    return q[:, :k].contiguous(), s


def dequantize_g128(qdata, scale, dtype=torch.bfloat16):
    """fp32 product, one cast to `dtype` (hy_nomas/ops.py:55-62)."""
    n, k = qdata.shape
    if k % GROUP == 0:
        weight = (qdata.view(n, k // GROUP, GROUP).float() * scale.unsqueeze(-1)).view(n, k)
    else:
        weight = qdata.float() * scale.repeat_interleave(GROUP, dim=1)[:, :k]
    return weight.to(dtype)
