"""Checkpoint weights through the kernels: a float block quantized into the reference's `weight_q` / `weight_scale`
pairs (hy_nomas/loader.py:42-53), written to and read from safetensors, loaded into group-major scale storage
(hy_nomas_b200.weights), then run by the W8A8 GEMM. Codes and scales equal the oracle's quantize_g128; every
linear's bf16 output equals the oracle's GEMM with the checkpoint's [N, K/128] scales bit for bit; the block on
the loaded weights equals the block on row-major copies of the same scales (the storage changes, the values do
not)."""
import numpy as np
import pytest
import torch

from hn_testutil import bits16

pytestmark = pytest.mark.gpu

D, HEADS, MLP = 256, 2, 1024


def float_block(gen):
    p = "double_blocks.0.img_"
    sd = {}
    for name, (n, k) in {"mod.linear": (6 * D, D), "attn_q": (D, D), "attn_k": (D, D), "attn_v": (D, D),
                         "attn_proj": (D, D), "mlp.fc1": (MLP, D), "mlp.fc2": (D, MLP)}.items():
        sd[p + name + ".weight"] = torch.randn(n, k, generator=gen) * (1.0 / k ** 0.5)
        sd[p + name + ".bias"] = (torch.randn(n, generator=gen) * 0.02).to(torch.bfloat16)
    sd[p + "attn_q_norm.weight"] = torch.ones(D // HEADS, dtype=torch.bfloat16)
    sd[p + "attn_k_norm.weight"] = torch.ones(D // HEADS, dtype=torch.bfloat16)
    sd["img_in.proj.weight"] = torch.randn(D, 128, generator=gen)   # kept float (KEEP_FLOAT)
    return sd


@pytest.fixture(scope="module")
def loaded(hn, cuda, tmp_path_factory):
    from hy_nomas_b200 import weights as W
    gen = torch.Generator().manual_seed(11)
    sd = float_block(gen)
    qsd = W.quantize_state_dict({k: (v.to(cuda) if v.dim() == 2 else v) for k, v in sd.items()})
    path = str(tmp_path_factory.mktemp("ckpt") / "block_int8.safetensors")
    W.write_safetensors(path, qsd, metadata={"format": "nomas-int8-bf16-single-v1"})
    back, meta = W.read_safetensors(path)
    assert W.detect(back, meta) == "int8"
    bw = W.block_weights(back, 0, hidden=D, heads=HEADS, mlp_ratio=MLP // D, device=cuda)
    return sd, back, bw


def test_quantized_pairs_match_oracle(oracle, loaded):
    sd, back, _ = loaded
    for key, w in sd.items():
        if key.startswith("img_in."):
            assert "img_in.proj.weight" in back and back[key].dtype == torch.float32
            continue
        if not key.endswith(".weight") or w.dim() != 2:
            continue
        q, s = oracle.quantize_g128(w.numpy())
        base = key[:-len("weight")]
        assert np.array_equal(back[base + "weight_q"].numpy(), q), key
        assert np.array_equal(back[base + "weight_scale"].numpy().view(np.uint32), s.view(np.uint32)), key


def test_loaded_linears_bit_exact(hn, oracle, cuda, loaded):
    _, _, bw = loaded
    gen = torch.Generator().manual_seed(12)
    x = torch.randn(300, D, generator=gen).to(torch.bfloat16)
    for lin in (bw.mod, bw.qk, bw.v, bw.proj, bw.fc1):
        assert lin.s.stride(0) == 1          # group-major storage
        y = hn.kernels.block_linear(x.to(cuda), lin.q, lin.s, lin.bias)
        qa, sa = oracle.quantize_activations(x.float().numpy())
        ref = oracle.block_gemm(qa.view(np.int8), sa, lin.q.cpu().numpy(), lin.s.cpu().numpy(),
                                lin.bias.float().cpu().numpy(), sa_mode="group", sw_mode="group")
        assert np.array_equal(bits16(y), oracle.bf16_bits(oracle.round_bf16(ref)))
    rc, code = hn.lib.device_error()
    assert rc == 0 and code == 0


def test_loaded_block_equals_row_major_scales(hn, cuda, loaded):
    from hy_nomas_b200.dit import BlockWeights, DiTConfig, QLinear, block_forward, rope_freqs
    from hy_nomas_b200.sequence_parallel import SequenceParallel
    _, _, bw = loaded
    row_major = lambda l: QLinear(l.q, l.s.contiguous(), l.bias)  # noqa: E731
    bw_rm = BlockWeights(mod=row_major(bw.mod), qk=row_major(bw.qk), v=row_major(bw.v), proj=row_major(bw.proj),
                         fc1=row_major(bw.fc1), fc2=row_major(bw.fc2), q_norm=bw.q_norm, k_norm=bw.k_norm)
    cfg = DiTConfig(hidden=D, heads=HEADS, mlp_ratio=MLP // D, blocks=1, grid=(1, 10, 20))
    rope = rope_freqs(cfg.rope_dims, cfg.theta, *cfg.grid, device=cuda)
    gen = torch.Generator().manual_seed(13)
    x = torch.randn(1, cfg.tokens, D, generator=gen).to(torch.bfloat16).to(cuda)
    vec = torch.randn(1, D, generator=gen).to(torch.bfloat16).to(cuda)
    a = block_forward(cfg, bw, x, vec, rope, SequenceParallel())
    b = block_forward(cfg, bw_rm, x, vec, rope, SequenceParallel())
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))
    assert torch.isfinite(a.float()).all()


def test_fp8_decoder_linear_from_file(hn, oracle, cuda, tmp_path):
    """An FP8 decoder linear (pixelumm.py:126-145) written as `fp8_weight` / `fp8_scale`, read back and run by
    `ops.fp8_block_linear`: the same output as the in-memory tensors bit for bit, and the oracle's block-scaled
    GEMM on the same 1x128 e4m3 activations within the stated FP8 tolerance (rel-L2 <= 1e-2)."""
    from hy_nomas_b200 import weights as W
    from hn_testutil import rel_l2
    gen = torch.Generator().manual_seed(14)
    w = torch.randn(384, 512, generator=gen) * 0.02
    q, s = hn.ops.quantize_fp8_block(w.to(cuda))
    bias = (torch.randn(384, generator=gen) * 0.02).to(torch.bfloat16)
    path = str(tmp_path / "decoder_fp8.safetensors")
    W.write_safetensors(path, {"layers.0.mlp.up_proj.fp8_weight": q, "layers.0.mlp.up_proj.fp8_scale": s,
                               "layers.0.mlp.up_proj.bias": bias})
    sd, _ = W.read_safetensors(path)
    lin = W.fp8_linear(sd, "layers.0.mlp.up_proj.", device=cuda)
    x = torch.randn(200, 512, generator=gen).to(torch.bfloat16).to(cuda)
    y = hn.ops.fp8_block_linear(x, lin.q, lin.s, lin.bias)
    y_mem = hn.ops.fp8_block_linear(x, q, s, bias.to(cuda))
    assert torch.equal(y.view(torch.int16), y_mem.view(torch.int16))
    qa, sa = oracle.quantize_activations(x.float().cpu().numpy(), kind="fp8")
    ref = oracle.block_gemm(qa, sa, q.cpu().view(torch.uint8).numpy(), s.cpu().numpy(), bias.float().numpy(),
                            kind="fp8", sa_mode="group", sw_mode="block")
    assert rel_l2(y.float().cpu().numpy(), oracle.round_bf16(ref)) < 1e-2
