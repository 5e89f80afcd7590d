"""A small DoubleStreamBlock (hy_nomas/model.py:230-303) for the drop-in trace - test infrastructure.

Shared by tests/golden/make_block_trace.py (which runs the reference's own block with this repository's
kernels/fused modules in place of the reference's, and records every call) and tests/test_gpu_dropin.py (which
replays the recorded calls through the CUDA path). The weights are regenerated here from a seed on the CPU, so
the fixture holds only the activations: every Linear is Tencent's int8 layout made by the reference's
quantizer arithmetic (codes [N, K], scales [N, K/128], oracle/torch_ref.quantize_g128), with a bf16 bias.
"""
import torch

HIDDEN, HEADS, MLP_RATIO = 256, 2, 2.0
GRID = (2, 4, 4)          # image tokens: frames x rows x columns
TEXT_TOKENS = 8
ROPE_DIMS, THETA = (32, 48, 48), 10000.0
SEED = 2024


def linear_shapes():
    """name (the DoubleStreamBlock attribute path) -> (out_features, in_features) of every Linear."""
    d, mlp = HIDDEN, int(HIDDEN * MLP_RATIO)
    shapes = {}
    for side in ("img", "txt"):
        shapes[f"{side}_mod.linear"] = (6 * d, d)
        for name in ("q", "k", "v", "proj"):
            shapes[f"{side}_attn_{name}"] = (d, d)
        shapes[f"{side}_mlp.fc1"] = (mlp, d)
        shapes[f"{side}_mlp.fc2"] = (d, mlp)
    return shapes


def make_weights():
    """{linear name: (int8 codes, fp32 scales [N, K/128], bf16 bias)} and {norm name: bf16 weight}."""
    import sys
    import os
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from oracle import torch_ref
    gen = torch.Generator().manual_seed(SEED)
    linears = {}
    for name, (n, k) in linear_shapes().items():
        w = torch.randn(n, k, generator=gen) * (k ** -0.5)
        q, s = torch_ref.quantize_g128(w)
        bias = (torch.randn(n, generator=gen) * 0.02).to(torch.bfloat16)
        linears[name] = (q, s, bias)
    norms = {}
    for side in ("img", "txt"):
        for which in ("q", "k"):
            norms[f"{side}_attn_{which}_norm.weight"] = (1.0 + 0.1 * torch.randn(HIDDEN // HEADS, generator=gen)
                                                         ).to(torch.bfloat16)
    return linears, norms


def make_inputs():
    gen = torch.Generator().manual_seed(SEED + 1)
    t, h, w = GRID
    img = torch.randn(1, t * h * w, HIDDEN, generator=gen).to(torch.bfloat16)
    txt = torch.randn(1, TEXT_TOKENS, HIDDEN, generator=gen).to(torch.bfloat16)
    vec = torch.randn(1, HIDDEN, generator=gen).to(torch.bfloat16)
    return img, txt, vec
