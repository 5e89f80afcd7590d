"""Weight layouts - the drop-in for the arithmetic of hy_nomas/ops.py (Tencent's per-row x 128-group int8)
and of the FP8 128 x 128 block layout of hy_nomas/pixelumm.py.

`quantize_g128` runs the activation quantizer kernel of libhynomas_b200.so on the weight (the same
absmax/127, round-half-away arithmetic: hy_nomas/ops.py:41-52) and needs a CUDA tensor. `dequantize_g128`
is the reference's plain tensor expression (hy_nomas/ops.py:55-62), used by block_linear for shapes the
GEMM does not take (K % 128 != 0). `quantize_fp8_block` runs the 128 x 128 block e4m3 quantizer
(hy_nomas/pixelumm.py:77-82); `fp8_block_linear` is the FP8 decoder linear's dispatch (pixelumm.py:147-155),
taking the [N/128, K/128] block scales directly instead of expanding them per row on every call. The ComfyUI layout registration and the Linear module of the reference
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
    w = _lib.dense(w)
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


def quantize_fp8_block(weight):
    """fp32/bf16 [N, K] (N, K multiples of 128) -> (float8_e4m3fn [N, K], fp32 block scales [N/128, K/128])."""
    _lib.require_cuda(weight)
    n, k = weight.shape
    w = weight if weight.dtype in (torch.float32, torch.bfloat16) else weight.float()
    w = _lib.dense(w)
    q = torch.empty((n, k), device=w.device, dtype=torch.float8_e4m3fn)
    s = torch.empty((n // 128, k // 128), device=w.device, dtype=torch.float32)
    rc = _lib.lib.hn_quantize_fp8_block(_lib.ptr(w), _lib.DTYPE[w.dtype], n, k, _lib.ptr(q), _lib.ptr(s),
                                        _lib.stream_of(w))
    _lib.check(rc, "quantize_fp8_block")
    return q, s


def dequantize_fp8_block(qdata, scale, dtype=torch.bfloat16):
    """fp32 product per 128 x 128 block, one cast to `dtype` (hy_nomas/pixelumm.py:60-63)."""
    n, k = qdata.shape
    w = qdata.float().view(n // 128, 128, k // 128, 128) * scale[:, None, :, None]
    return w.view(n, k).to(dtype)


def fp8_block_linear(x, qdata, scale, bias=None):
    """The FP8 decoder linear (hy_nomas/pixelumm.py:147-155): e4m3 1 x 128 activations against 128 x 128 block
    weights on the tensor cores, output in x's dtype."""
    from .kernels import block_linear
    return block_linear(x, qdata, scale, bias, kind="fp8")


def stack_fp8_linears(*linears):
    """FP8 block-scaled linears with the same K, stacked along N into one: (codes [sum N, K], block scales
    [sum N / 128, K / 128]). The decoder MLP's gate_proj and up_proj read the same input, so one GEMM does both."""
    return torch.cat([q for q, _ in linears]), torch.cat([s for _, s in linears])


def decoder_mlp(x, norm_weight, gate_up, down, eps=1e-6):
    """The MLP half of the PixelUMM decoder layer, x + mlp(post_attn_norm(x)) (hy_nomas/pixelumm.py:320-337), on the
    fused kernels: RMSNorm + e4m3 quantization (one pass), the stacked gate|up FP8 GEMM (bf16 out), silu(gate) *
    up + e4m3 quantization (one pass), down_proj's FP8 GEMM, the residual. x [..., hidden] bf16; gate_up =
    stack_fp8_linears((gate codes, gate block scales), (up codes, up block scales)); down = (codes, block scales)."""
    from . import fused
    from .kernels import block_gemm
    shape = x.shape
    q, s = fused.rmsnorm_quant(x, norm_weight, eps, kind="fp8")
    gu = block_gemm(q, s, gate_up[0], gate_up[1], kind="fp8")
    inter = gu.shape[1] // 2
    hq, hs = fused.silu_mul_quant(gu[:, :inter], gu[:, inter:], kind="fp8")
    y = block_gemm(hq, hs, down[0], down[1], kind="fp8")
    return x + y.view(shape)
