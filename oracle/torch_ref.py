"""The reference's torch arithmetic for this path, restated - TEST INFRASTRUCTURE ONLY.

These are the torch expressions ComfyUI-Hy-Nomas uses as its own reference and as its CPU path (the
int8 kernels only run when the input is on CUDA, hy_nomas/ops.py:172-176). tests/ compare the CUDA
kernels with them under the reference's own tolerances (its tests/test_fused.py), and bench.py times
them on the host cores as the CPU baseline. Nothing in the product imports this module.

  layer_norm        hy_nomas/model.py:103-106
  modulate          hy_nomas/model.py:109-111
  rms_norm          hy_nomas/model.py:89-100 (RMSNorm.forward)
  rope_freqs        hy_nomas/model.py:114-128
  apply_rope        hy_nomas/model.py:131-138
  quantize_g128     hy_nomas/ops.py:41-52
  dequantize_g128   hy_nomas/ops.py:55-62
  int8_linear_cpu   hy_nomas/ops.py:175-176 (dequantize + F.linear, the non-CUDA branch)
  fp8_block_*       hy_nomas/pixelumm.py:60-63, 77-82, 154-155
  quantize_kv       hy_nomas/world.py:83-90
  dit_block_cpu     hy_nomas/model.py:246-286 (DoubleStreamBlock image stream, the non-fused branch)
  make_block_weights_cpu  seeded random int8 weights of one synthetic block (the benchmark's shapes), built
                    here so that the CPU reference arm loads nothing of the product
"""
import math
from collections import namedtuple

import torch
import torch.nn.functional as F

GROUP = 128


def layer_norm(x, eps=1e-6):
    return F.layer_norm(x.float(), (x.shape[-1],), eps=eps)


def modulate(x, shift, scale):
    return x * (1 + scale.unsqueeze(1)) + shift.unsqueeze(1)


def rms_norm(x, weight, eps=1e-6):
    out = x.float()
    out = (out * torch.rsqrt(out.pow(2).mean(-1, keepdim=True) + eps)).type_as(x)
    return out * weight.to(dtype=out.dtype, device=out.device)


def rope_freqs(rope_dims, theta, t, h, w, t_offset=0, device=None):
    axes = []
    for start, n in ((t_offset, t), (0, h), (0, w)):
        axes.append(torch.linspace(start, start + n, n + 1, dtype=torch.float32, device=device)[:n])
    grid = torch.meshgrid(*axes, indexing="ij")
    cos, sin = [], []
    for dim, pos in zip(rope_dims, grid):
        freqs = 1.0 / (theta ** (torch.arange(0, dim, 2, device=device)[: dim // 2].float() / dim))
        angles = torch.outer(pos.reshape(-1), freqs)
        cos.append(angles.cos().repeat_interleave(2, dim=1))
        sin.append(angles.sin().repeat_interleave(2, dim=1))
    return torch.cat(cos, dim=1), torch.cat(sin, dim=1)


def apply_rope(x, cos, sin):
    xf = x.float()
    real, imag = xf.reshape(*x.shape[:-1], -1, 2).unbind(-1)
    rotated = torch.stack([-imag, real], dim=-1).flatten(3)
    cos = cos[None, :, None, :]
    sin = sin[None, :, None, :]
    return (xf * cos + rotated * sin).type_as(x)


def quantize_g128(weight):
    n, k = weight.shape
    groups = (k + GROUP - 1) // GROUP
    padded = F.pad(weight.float(), (0, groups * GROUP - k))
    rows = padded.reshape(n, groups, GROUP)
    peak = rows.abs().amax(dim=-1)
    scale = torch.where(peak > 0, peak / 127.0, 1.0)
    normalized = rows / scale.unsqueeze(-1)
    rounded = (normalized.abs() + 0.5).floor() * normalized.sign()
    q = rounded.clamp_(-127, 127).to(torch.int8).reshape(n, -1)[:, :k].contiguous()
    return q, scale.contiguous()


def dequantize_g128(qdata, scale, dtype=torch.bfloat16):
    n, k = qdata.shape
    if k % GROUP == 0:
        weight = (qdata.view(n, k // GROUP, GROUP).float() * scale.unsqueeze(-1)).view(n, k)
    else:
        weight = qdata.float() * scale.repeat_interleave(GROUP, dim=1)[:, :k]
    return weight.to(dtype)


def int8_linear_cpu(x, qdata, scale, bias=None):
    """The reference's linear when the input is not on CUDA: dequantize to x's dtype, then F.linear."""
    return F.linear(x, dequantize_g128(qdata, scale, x.dtype), bias)


def fp8_block_quantize(w):
    n, k = w.shape
    blocks = w.float().view(n // 128, 128, k // 128, 128)
    s = blocks.abs().amax(dim=(1, 3)).clamp_min(1e-4) / 448.0
    q = (blocks / s[:, None, :, None]).to(torch.float8_e4m3fn).view(n, k)
    return q, s


def fp8_block_dequantize(qdata, scale, dtype=torch.bfloat16):
    n, k = qdata.shape
    w = qdata.float().view(n // 128, 128, k // 128, 128) * scale[:, None, :, None]
    return w.view(n, k).to(dtype)


def fp8_linear_cpu(x, qdata, scale, bias=None):
    return F.linear(x, fp8_block_dequantize(qdata, scale, x.dtype), bias)


def quantize_kv(x):
    xf = x.float()
    peak = xf.abs().amax(dim=-1, keepdim=True)
    scale = torch.where(peak > 0, peak / 127.0, torch.ones_like(peak))
    scaled = xf / scale
    rounded = torch.where(scaled >= 0, torch.floor(scaled + 0.5), torch.ceil(scaled - 0.5))
    return rounded.clamp_(-127, 127).to(torch.int8), scale


def _linear_per_channel(x, ql):
    """An int8 linear with per-output-channel scales [N], broadcast to the reference's [N, K/128] layout."""
    n, k = ql.q.shape
    return int8_linear_cpu(x, ql.q, ql.s[:, None].expand(n, k // GROUP), ql.bias)


def dit_block_cpu(x, vec, w, rope, heads, timings=None):
    """One block on the reference's CPU path: every linear dequantizes its int8 weight and runs F.linear in
    bf16 (ops.py:175-176), norms/modulation/RoPE are the torch expressions above, attention is SDPA.
    `w` has the fields of hy_nomas_b200.dit.BlockWeights (q|k rows stacked in `qk`). `timings`, when a dict,
    gets the attention's seconds under "attention"."""
    import time
    b, n, d = x.shape
    mods = _linear_per_channel(F.silu(vec), w.mod)
    shift1, scale1, gate1, shift2, scale2, gate2 = mods.chunk(6, dim=-1)
    x_mod = modulate(layer_norm(x), shift1, scale1).to(x.dtype)
    qk = _linear_per_channel(x_mod, w.qk)
    q = qk[..., :d].reshape(b, n, heads, -1)
    k = qk[..., d:].reshape(b, n, heads, -1)
    v = _linear_per_channel(x_mod, w.v).view(b, n, heads, -1)
    q = rms_norm(q, w.q_norm).to(v)
    k = rms_norm(k, w.k_norm).to(v)
    q, k = apply_rope(q, *rope), apply_rope(k, *rope)
    t0 = time.perf_counter()
    attn = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)).transpose(1, 2)
    if timings is not None:
        timings["attention"] = timings.get("attention", 0.0) + time.perf_counter() - t0
    x = x + _linear_per_channel(attn.reshape(b, n, d), w.proj) * gate1.unsqueeze(1)
    h = _linear_per_channel(modulate(layer_norm(x), shift2, scale2).to(x.dtype), w.fc1)
    h = F.gelu(h, approximate="tanh")
    return x + _linear_per_channel(h, w.fc2) * gate2.unsqueeze(1)


QLinearCPU = namedtuple("QLinearCPU", "q s bias")
BlockWeightsCPU = namedtuple("BlockWeightsCPU", "mod qk v proj fc1 fc2 q_norm k_norm")
_CODE_STD = math.sqrt((255.0 ** 2 - 1.0) / 12.0)   # std of an integer uniform on [-127, 127]


def _qlinear_cpu(n, k, gen, gain=1.0):
    """int8 codes uniform in [-127, 127], per-output-channel fp32 scales preserving the activations' variance,
    bf16 bias N(0, 0.02): the distribution the benchmark's synthetic DiT uses."""
    q = torch.randint(-127, 128, (n, k), generator=gen, dtype=torch.int8)
    s = (torch.rand(n, generator=gen) + 0.5) * (gain / (_CODE_STD * math.sqrt(k)))
    bias = (torch.randn(n, generator=gen) * 0.02).to(torch.bfloat16)
    return QLinearCPU(q, s.float().contiguous(), bias)


def make_block_weights_cpu(hidden, mlp, head_dim, gen):
    """One block's linears ([6D, D] modulation, q|k [2D, D], v, proj, fc1 [mlp, D], fc2 [D, mlp]) and RMSNorm
    weights (ones, as RMSNorm.__init__ makes them, hy_nomas/model.py:95), on the CPU."""
    d = hidden
    ones = torch.ones(head_dim, dtype=torch.bfloat16)
    return BlockWeightsCPU(mod=_qlinear_cpu(6 * d, d, gen, gain=0.15), qk=_qlinear_cpu(2 * d, d, gen),
                           v=_qlinear_cpu(d, d, gen), proj=_qlinear_cpu(d, d, gen), fc1=_qlinear_cpu(mlp, d, gen),
                           fc2=_qlinear_cpu(d, mlp, gen), q_norm=ones, k_norm=ones.clone())
