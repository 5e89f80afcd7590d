"""The checkpoint boundary (hy_nomas_b200.weights) on the host: safetensors round trips in the reference's key
layout (hy_nomas/ops.py:129-154, hy_nomas/pixelumm.py:126-145, hy_nomas/model.py:230-244), format detection
(hy_nomas/loader.py:34-39), the reference's error messages, and the group-major scale storage. No GPU: tensors
load to the CPU here; `test_gpu_weights.py` runs loaded weights through the kernels."""
import pytest
import torch

from hy_nomas_b200 import weights as W


def int8_entry(sd, prefix, n, k, gen, bias=True):
    sd[prefix + "weight_q"] = torch.randint(-127, 128, (n, k), generator=gen, dtype=torch.int8)
    sd[prefix + "weight_scale"] = torch.rand(n, (k + 127) // 128, generator=gen) * 4e-3 + 1e-3
    if bias:
        sd[prefix + "bias"] = (torch.randn(n, generator=gen) * 0.02).to(torch.bfloat16)


def block_state_dict(d=256, heads=2, mlp=1024, gen=None):
    gen = gen or torch.Generator().manual_seed(0)
    sd = {}
    p = "double_blocks.0.img_"
    int8_entry(sd, p + "mod.linear.", 6 * d, d, gen)
    for name in ("attn_q", "attn_k", "attn_v", "attn_proj"):
        int8_entry(sd, p + name + ".", d, d, gen)
    int8_entry(sd, p + "mlp.fc1.", mlp, d, gen)
    int8_entry(sd, p + "mlp.fc2.", d, mlp, gen)
    sd[p + "attn_q_norm.weight"] = torch.ones(d // heads, dtype=torch.bfloat16)
    sd[p + "attn_k_norm.weight"] = torch.full((d // heads,), 1.5, dtype=torch.bfloat16)
    return sd


def test_round_trip_every_dtype(tmp_path):
    gen = torch.Generator().manual_seed(1)
    sd = {"a.weight_q": torch.randint(-127, 128, (256, 384), generator=gen, dtype=torch.int8),
          "a.weight_scale": torch.rand(256, 3, generator=gen),
          "a.bias": torch.randn(256, generator=gen).to(torch.bfloat16),
          "b.fp8_weight": (torch.randn(256, 128, generator=gen) * 40).to(torch.float8_e4m3fn),
          "b.fp8_scale": torch.rand(2, 1, generator=gen),
          "c.weight": torch.randn(8, 8, generator=gen).half()}
    path = str(tmp_path / "m.safetensors")
    W.write_safetensors(path, sd, metadata={"format": "nomas-int8-bf16-single-v1"})
    back, meta = W.read_safetensors(path)
    assert meta == {"format": "nomas-int8-bf16-single-v1"}
    assert set(back) == set(sd)
    for k, v in sd.items():
        assert back[k].dtype == v.dtype and back[k].shape == v.shape
        assert torch.equal(back[k].view(torch.uint8), v.contiguous().view(torch.uint8))


def test_detect():
    assert W.detect({"x.weight_q": None}, {}) == "int8"
    assert W.detect({}, {"format": "nomas-int8-bf16-single-v1"}) == "int8"
    assert W.detect({"double_blocks.0.img_attn_q.weight": None}, None) == "float"
    with pytest.raises(ValueError, match="not a Hy-Nomas DiT checkpoint"):
        W.detect({"foo": None}, {})


def test_int8_linear_group_major_scales():
    gen = torch.Generator().manual_seed(2)
    sd = {}
    int8_entry(sd, "l.", 6, 300, gen)   # 6 rows (padded to 8 in storage), K = 300 -> 3 groups
    ql = W.int8_linear(sd, "l.", 6, 300, device="cpu")
    assert torch.equal(ql.q, sd["l.weight_q"])
    assert ql.s.shape == (6, 3) and ql.s.stride() == (1, 8)
    assert torch.equal(ql.s, sd["l.weight_scale"])
    assert ql.bias.dtype == torch.bfloat16 and torch.equal(ql.bias, sd["l.bias"])


def test_int8_linear_errors():
    gen = torch.Generator().manual_seed(3)
    sd = {}
    int8_entry(sd, "l.", 8, 256, gen)
    with pytest.raises(ValueError, match=r"l\.weight_q has shape \(8, 256\), expected \(8, 128\)"):
        W.int8_linear(sd, "l.", 8, 128, device="cpu")
    bad = dict(sd)
    del bad["l.weight_scale"]
    with pytest.raises(ValueError, match=r"l\.weight_q without l\.weight_scale"):
        W.int8_linear(bad, "l.", 8, 256, device="cpu")
    bad = dict(sd, **{"l.weight_scale": torch.rand(8)})
    with pytest.raises(ValueError, match="weight_scale has shape"):
        W.int8_linear(bad, "l.", 8, 256, device="cpu")
    bad = dict(sd, **{"l.weight_q": sd["l.weight_q"].to(torch.int16)})
    with pytest.raises(ValueError, match="dtype"):
        W.int8_linear(bad, "l.", 8, 256, device="cpu")
    with pytest.raises(ValueError, match="missing m.weight_q"):
        W.int8_linear(sd, "m.", 8, 256, device="cpu")


def test_fp8_linear():
    gen = torch.Generator().manual_seed(4)
    q = (torch.randn(256, 384, generator=gen) * 40).to(torch.float8_e4m3fn)
    s = torch.rand(2, 3, generator=gen)
    ql = W.fp8_linear({"d.fp8_weight": q, "d.fp8_scale": s}, "d.", device="cpu")
    assert ql.q.dtype == torch.float8_e4m3fn and torch.equal(ql.q.view(torch.uint8), q.view(torch.uint8))
    assert torch.equal(ql.s, s) and ql.bias is None
    with pytest.raises(ValueError, match="multiples of 128"):
        W.fp8_linear({"d.fp8_weight": q, "d.fp8_scale": torch.rand(2, 2)}, "d.", device="cpu")
    with pytest.raises(ValueError, match="missing"):
        W.fp8_linear({"d.fp8_weight": q}, "d.", device="cpu")


def test_block_weights_layout(tmp_path):
    sd = block_state_dict()
    path = str(tmp_path / "block.safetensors")
    W.write_safetensors(path, sd)
    loaded, _ = W.read_safetensors(path)
    bw = W.block_weights(loaded, 0, hidden=256, heads=2, mlp_ratio=4, device="cpu")
    p = "double_blocks.0.img_"
    # q rows then k rows in the one q|k linear, scales and biases alike
    assert torch.equal(bw.qk.q, torch.cat([sd[p + "attn_q.weight_q"], sd[p + "attn_k.weight_q"]]))
    assert torch.equal(bw.qk.s, torch.cat([sd[p + "attn_q.weight_scale"], sd[p + "attn_k.weight_scale"]]))
    assert bw.qk.s.stride() == (1, 512)
    assert torch.equal(bw.qk.bias, torch.cat([sd[p + "attn_q.bias"], sd[p + "attn_k.bias"]]))
    assert bw.mod.q.shape == (6 * 256, 256) and bw.fc1.q.shape == (1024, 256) and bw.fc2.q.shape == (256, 1024)
    assert bw.fc2.s.shape == (256, 8)
    assert torch.equal(bw.k_norm, sd[p + "attn_k_norm.weight"])
    del loaded[p + "attn_q_norm.weight"]
    with pytest.raises(ValueError, match="attn_q_norm.weight"):
        W.block_weights(loaded, 0, hidden=256, heads=2, device="cpu")
