"""Golden vectors of the PixelUMM decoder's RMSNorm and MLP gate from the REFERENCE's own modules.

Run where a checkout of the reference repository is available, its directory given by HY_NOMAS_REFERENCE:

    HY_NOMAS_REFERENCE=<checkout> python tests/golden/make_decoder_golden.py

It writes tests/golden/decoder.npz: the reference's hy_nomas/pixelumm.py RMSNorm.forward (pixelumm.py:246-259,
the decoder layer's input_norm / post_attn_norm) on seeded bf16 rows, and its MLP.forward's silu(gate) * up
(pixelumm.py:322-323) on seeded gate/up activations - the MLP's three linears replaced by modules that return the
given gate and up outputs and pass the product through, so only the reference's own expression runs. Both on
CPU, with the `comfy` modules stubbed as in make_golden.py. bf16 arrays are stored as uint16 bit patterns.
"""
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import make_golden  # noqa: E402


class _Fixed(torch.nn.Module):
    """A stand-in linear that returns a fixed tensor (or its input, for the output projection)."""

    def __init__(self, out=None):
        super().__init__()
        self.out = out

    def forward(self, x):
        return x if self.out is None else self.out


def main():
    make_golden._stub_comfy()
    sys.path.insert(0, make_golden.reference_dir())
    from hy_nomas import pixelumm  # noqa: E402
    gen = torch.Generator().manual_seed(31)
    rows, d, inter = 24, 4096, 768
    x = (torch.randn(rows, d, generator=gen) * 2.0).to(torch.bfloat16)
    x[3] *= 40.0                                        # a large row
    x[5, ::7] = 0.0
    norm = pixelumm.RMSNorm(d, 1e-6, dtype=torch.bfloat16)
    with torch.no_grad():
        norm.weight.copy_((1.0 + 0.2 * torch.randn(d, generator=gen)).to(torch.bfloat16))
        y = norm(x)
    g = (torch.randn(rows, inter, generator=gen) * 3.0).to(torch.bfloat16)
    g[0, :8] = torch.tensor([0.0, -0.0, 90.0, -90.0, 20.0, -20.0, 1e-3, -1e-3]).to(torch.bfloat16)
    u = torch.randn(rows, inter, generator=gen).to(torch.bfloat16)
    mlp = pixelumm.MLP.__new__(pixelumm.MLP)
    torch.nn.Module.__init__(mlp)
    mlp.gate_proj, mlp.up_proj, mlp.down_proj = _Fixed(g), _Fixed(u), _Fixed()
    with torch.no_grad():
        h = mlp(None)
    bits = make_golden.bits
    np.savez_compressed(os.path.join(HERE, "decoder.npz"), x=bits(x), w=bits(norm.weight.detach()), y=bits(y),
                        g=bits(g), u=bits(u), h=bits(h), eps=np.float32(1e-6))
    print("decoder.npz:", {k: v.shape for k, v in np.load(os.path.join(HERE, "decoder.npz")).items()})


if __name__ == "__main__":
    main()
