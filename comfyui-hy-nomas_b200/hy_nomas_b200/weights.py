"""Checkpoint boundary of the quantized linear path: the reference's safetensors keys -> the tensors the GEMM reads.

The reference stores every quantized DiT Linear as `<prefix>weight_q` (int8 [N, K]) + `<prefix>weight_scale`
(fp32 [N, ceil(K/128)], one scale per output row and 128-wide K group) + `<prefix>bias`, and builds its layout
object from them when the module loads (hy_nomas/ops.py:129-154); a float checkpoint is quantized to the same
pairs first (hy_nomas/loader.py:34-62). The PixelUMM decoder stores `<prefix>fp8_weight` (e4m3 [N, K]) +
`<prefix>fp8_scale` (fp32 [N/128, K/128], one per 128 x 128 block) (hy_nomas/pixelumm.py:126-145).

Here the same keys load straight into the layout `kernels.block_gemm` streams fastest:
  * int8 codes [N, K] stay K-major as stored (the GEMM's TMA reads them without repacking);
  * the row-major [N, G] weight scales are copied into group-major storage ([G, N padded to 4], handed back as
    an [N, G] view), so the GEMM moves one group's scales for a whole tile with one bulk copy. The values are
    the checkpoint's, so every GEMM output is the one the row-major scales give;
  * FP8 block scales stay [N/128, K/128]: the GEMM takes them as they are (the reference expands them per row on
    every call, pixelumm.py:153).
A block of the DiT (`double_blocks.<i>.img_*`, model.py:230-244) becomes a `dit.BlockWeights` with the q and k
rows stacked into the one q|k linear that `dit.block_forward` runs.

Files are read with the `safetensors` package, the reader the reference's loaders use.
"""
import torch

from . import _lib
from .dit import BlockWeights, QLinear

GROUP = 128
# small modules the reference keeps unquantized when it quantizes a float checkpoint (hy_nomas/loader.py:30)
KEEP_FLOAT = ("action_modules.", "extrinsics_embedding_camctrl", "c2ws_hidden_states_layer", "img_in.")


def read_safetensors(path):
    """(state_dict of CPU tensors, metadata dict) of a .safetensors file."""
    from safetensors import safe_open
    out = {}
    with safe_open(path, framework="pt", device="cpu") as f:
        metadata = f.metadata() or {}
        for key in f.keys():
            out[key] = f.get_tensor(key)
    return out, metadata


def write_safetensors(path, state_dict, metadata=None):
    """Write CPU copies of `state_dict`'s tensors (contiguous) to a .safetensors file."""
    from safetensors.torch import save_file
    save_file({k: v.detach().contiguous().cpu() for k, v in state_dict.items()}, path, metadata=metadata)


def detect(state_dict, metadata):
    """"int8" (Tencent's g128 pairs) or "float" (hy_nomas/loader.py:34-39); ValueError for another file."""
    fmt = (metadata or {}).get("format")
    if fmt == "nomas-int8-bf16-single-v1" or any(k.endswith(".weight_q") for k in state_dict):
        return "int8"
    if "double_blocks.0.img_attn_q.weight" in state_dict:
        return "float"
    raise ValueError("not a Hy-Nomas DiT checkpoint (no double_blocks.0.img_attn_q weights)")


def quantize_state_dict(state_dict):
    """A float checkpoint's Linear weights -> `weight_q` / `weight_scale` pairs (hy_nomas/loader.py:42-53): every
    2-D `.weight` with K % 128 == 0 outside KEEP_FLOAT, quantized per row and 128-group on the GPU quantizer."""
    from .ops import quantize_g128
    out = {}
    for key, value in state_dict.items():
        if (key.endswith(".weight") and value.ndim == 2 and not key.startswith(KEEP_FLOAT)
                and value.shape[1] % GROUP == 0):
            q, s = quantize_g128(value if value.is_cuda else value.cuda())
            out[key[:-len("weight")] + "weight_q"] = q
            out[key[:-len("weight")] + "weight_scale"] = s.contiguous()
        else:
            out[key] = value
    return out


def group_major(scale, device):
    """fp32 [N, G] scales (any layout) -> the same values in group-major storage on `device`: an [N, G] view with
    row stride 1 and group stride N padded to 4."""
    n, g = scale.shape
    view, _, _ = _lib.group_scales(n, g, device)
    view.copy_(scale.to(device=device, dtype=torch.float32))
    return view


def int8_linear(state_dict, prefix, out_features, in_features, device="cuda", bias_dtype=torch.bfloat16):
    """`prefix`weight_q / weight_scale / bias -> QLinear(int8 [N, K], fp32 [N, G] group-major, bias [N] or None).

    Raises ValueError with the reference's messages (hy_nomas/ops.py:137-144) for a missing scale or a weight of
    the wrong shape, and for a scale that is not [N, ceil(K/128)]."""
    q = state_dict.get(prefix + "weight_q")
    scale = state_dict.get(prefix + "weight_scale")
    bias = state_dict.get(prefix + "bias")
    if q is None:
        raise ValueError(f"missing {prefix}weight_q")
    if scale is None:
        raise ValueError(f"{prefix}weight_q without {prefix}weight_scale")
    if tuple(q.shape) != (out_features, in_features):
        raise ValueError(f"{prefix}weight_q has shape {tuple(q.shape)}, expected {(out_features, in_features)}")
    groups = (in_features + GROUP - 1) // GROUP
    if tuple(scale.shape) != (out_features, groups):
        raise ValueError(f"{prefix}weight_scale has shape {tuple(scale.shape)}, expected {(out_features, groups)}")
    if q.dtype != torch.int8:
        raise ValueError(f"{prefix}weight_q has dtype {q.dtype}, expected torch.int8")
    return QLinear(q.to(device).contiguous(), group_major(scale.float(), device),
                   None if bias is None else bias.to(device=device, dtype=bias_dtype))


def fp8_linear(state_dict, prefix, device="cuda", bias_dtype=torch.bfloat16):
    """`prefix`fp8_weight / fp8_scale / bias -> QLinear(e4m3 [N, K], fp32 [N/128, K/128], bias or None), the FP8
    decoder linear's stored layout (hy_nomas/pixelumm.py:126-145), for `ops.fp8_block_linear`."""
    q = state_dict.get(prefix + "fp8_weight")
    scale = state_dict.get(prefix + "fp8_scale")
    bias = state_dict.get(prefix + "bias")
    if q is None or scale is None:
        raise ValueError(f"missing {prefix}fp8_weight or {prefix}fp8_scale")
    n, k = q.shape
    if n % 128 or k % 128 or tuple(scale.shape) != (n // 128, k // 128):
        raise ValueError(f"{prefix}fp8_weight {tuple(q.shape)} / fp8_scale {tuple(scale.shape)}: expected N and K "
                         f"multiples of 128 and scales [N/128, K/128]")
    if q.dtype != torch.float8_e4m3fn:
        raise ValueError(f"{prefix}fp8_weight has dtype {q.dtype}, expected torch.float8_e4m3fn")
    return QLinear(q.to(device).contiguous(), scale.to(device=device, dtype=torch.float32).contiguous(),
                   None if bias is None else bias.to(device=device, dtype=bias_dtype))


def _stack(a, b):
    """Two int8 linears with the same K -> one linear with a's output rows then b's (group-major scales)."""
    bias = None if a.bias is None or b.bias is None else torch.cat([a.bias, b.bias])
    return QLinear(torch.cat([a.q, b.q]), group_major(torch.cat([a.s, b.s]), a.q.device), bias)


def block_weights(state_dict, index, hidden, heads, mlp_ratio=4, side="img", device="cuda"):
    """`double_blocks.<index>.<side>_*` of an int8 checkpoint (model.py:230-244) -> dit.BlockWeights: Modulate's
    linear [6D, D], q|k stacked [2D, D], v, proj, MLP fc1 [mlp, D] and fc2 [D, mlp], the q/k RMSNorm weights."""
    d, mlp = hidden, int(hidden * mlp_ratio)
    p = f"double_blocks.{index}.{side}_"

    def lin(name, n, k):
        return int8_linear(state_dict, p + name + ".", n, k, device)

    def norm(name):
        w = state_dict.get(p + name + ".weight")
        if w is None:
            raise ValueError(f"missing {p}{name}.weight")
        if tuple(w.shape) != (d // heads,):
            raise ValueError(f"{p}{name}.weight has shape {tuple(w.shape)}, expected {(d // heads,)}")
        return w.to(device=device, dtype=torch.bfloat16)

    return BlockWeights(mod=lin("mod.linear", 6 * d, d), qk=_stack(lin("attn_q", d, d), lin("attn_k", d, d)),
                        v=lin("attn_v", d, d), proj=lin("attn_proj", d, d), fc1=lin("mlp.fc1", mlp, d),
                        fc2=lin("mlp.fc2", d, mlp), q_norm=norm("attn_q_norm"), k_norm=norm("attn_k_norm"))
