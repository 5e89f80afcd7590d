"""The fused elementwise kernels (hy_nomas/fused.py, kernels.adaln_quant) on the GPU: bit-exact against the
oracle (same reduction tree, correctly rounded rsqrt), and within the reference's own tolerances
(its tests/test_fused.py) against the torch arithmetic of hy_nomas/model.py."""
import numpy as np
import pytest
import torch

from hn_testutil import bf16_from_bits, bits16, f32, rel_l2, u8

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("b,l,d", [(2, 20, 2048), (1, 12, 4096), (1, 37, 3072), (3, 5, 128)])
def test_adaln_quant_and_adaln_bit_exact(hn, oracle, cuda, b, l, d):
    gen = torch.Generator().manual_seed(b * l + d)
    x = (torch.randn(b, l, d, generator=gen) * 3).bfloat16()
    shift, scale = torch.randn(b, d, generator=gen).bfloat16(), torch.randn(b, d, generator=gen).bfloat16()
    q, s = hn.kernels.adaln_quant(x.to(cuda), shift.to(cuda), scale.to(cuda))
    y = hn.fused.adaln(x.to(cuda), shift.to(cuda), scale.to(cuda))
    qo, so = oracle.adaln_quant(f32(x), f32(shift), f32(scale))
    assert np.array_equal(q.cpu().numpy(), qo) and np.array_equal(f32(s), so)
    yo = oracle.bf16_bits(oracle.round_bf16(oracle.adaln(f32(x), f32(shift), f32(scale))))
    assert np.array_equal(bits16(y), yo)


def test_adaln_golden(hn, golden, cuda):
    d = golden("adaln")
    for tag, b in (("d2048", 2), ("d4096", 1)):
        D = int(tag[1:])
        x = bf16_from_bits(d[f"{tag}_x"], cuda).view(b, -1, D)
        sh, sc = bf16_from_bits(d[f"{tag}_shift"], cuda).view(b, D), bf16_from_bits(d[f"{tag}_scale"], cuda).view(b, D)
        q, s = hn.kernels.adaln_quant(x, sh, sc)
        assert (q.cpu().numpy() != d[f"{tag}_q"]).mean() < 1e-3
        assert np.allclose(f32(s), d[f"{tag}_s"], rtol=1e-3)
        y = hn.fused.adaln(x, sh, sc)
        assert (bits16(y).reshape(-1) != d[f"{tag}_torch_y"].reshape(-1)).mean() < 1e-3


def test_reference_adaln_strided(hn, cuda):
    """tests/test_fused.py:12-21 of the reference: strided input, mismatch < 1e-3, max abs < 0.05."""
    from oracle import torch_ref
    x = (torch.randn(2, 2048, 777) * 3).bfloat16().transpose(1, 2)
    shift, scale = torch.randn(2, 2048).bfloat16(), torch.randn(2, 2048).bfloat16()
    ref = torch_ref.modulate(torch_ref.layer_norm(x), shift, scale).to(torch.bfloat16)
    got = hn.fused.adaln(x.to(cuda), shift.to(cuda), scale.to(cuda)).cpu()
    assert (got != ref).float().mean().item() < 1e-3
    assert (got.float() - ref.float()).abs().max().item() < 0.05


def test_reference_adaln_quant_matches_unfused(hn, cuda):
    """tests/test_fused.py:52-60: K3 against K1(K4); here the codes are identical by construction."""
    x = (torch.randn(1, 2048, 300) * 3).bfloat16().transpose(1, 2).to(cuda)
    shift, scale = torch.randn(1, 2048).bfloat16().to(cuda), torch.randn(1, 2048).bfloat16().to(cuda)
    q, s = hn.kernels.adaln_quant(x, shift, scale)
    q_ref, s_ref = hn.kernels.quantize_activations(hn.fused.adaln(x, shift, scale).view(-1, 2048))
    assert torch.equal(q, q_ref) and torch.equal(s, s_ref)


def test_gated_residual_exact(hn, golden, cuda):
    d = golden("gated_residual")
    x = bf16_from_bits(d["x"], cuda).view(2, 33, 256)
    y = bf16_from_bits(d["y"], cuda).view(2, 33, 256)
    g = bf16_from_bits(d["g"], cuda).view(2, 256)
    out = hn.fused.gated_residual(x, y, g)
    assert np.array_equal(bits16(out).reshape(-1), d["out"].reshape(-1))


def test_reference_gated_residual_strided(hn, cuda):
    """tests/test_fused.py:43-49: exact equality with x + y * g."""
    x = torch.randn(1, 2048, 500).bfloat16().transpose(1, 2).to(cuda)
    y = torch.randn(1, 500, 2048).bfloat16().to(cuda)
    g = torch.randn(1, 2048).bfloat16().to(cuda)
    assert torch.equal(hn.fused.gated_residual(x, y, g), x + y * g.unsqueeze(1))


@pytest.mark.parametrize("b,l,d", [(1, 40, 4096), (2, 9, 2048)])
def test_gated_residual_adaln_quant_bit_exact(hn, oracle, cuda, b, l, d):
    gen = torch.Generator().manual_seed(l)
    x, y = torch.randn(b, l, d, generator=gen).bfloat16(), torch.randn(b, l, d, generator=gen).bfloat16()
    g = (torch.randn(b, d, generator=gen) * 0.1).bfloat16()
    sh, sc = torch.randn(b, d, generator=gen).bfloat16(), torch.randn(b, d, generator=gen).bfloat16()
    xo, q, s = hn.fused.gated_residual_adaln_quant(*(t.to(cuda) for t in (x, y, g, sh, sc)))
    xr, qr, sr = oracle.gated_residual_adaln_quant(f32(x), f32(y), f32(g), f32(sh), f32(sc))
    assert np.array_equal(bits16(xo), oracle.bf16_bits(xr))
    assert np.array_equal(q.cpu().numpy(), qr) and np.array_equal(f32(s), sr)
    # the same as the two unfused calls
    x2 = hn.fused.gated_residual(x.to(cuda), y.to(cuda), g.to(cuda))
    q2, s2 = hn.kernels.adaln_quant(x2, sh.to(cuda), sc.to(cuda))
    assert torch.equal(x2, xo) and torch.equal(q2, q) and torch.equal(s2, s)


def test_qk_norm_rope_golden_and_oracle(hn, oracle, golden, cuda):
    d = golden("qk_norm_rope")
    x = bf16_from_bits(d["x"], cuda)
    w = bf16_from_bits(d["w"], cuda)
    cos, sin = torch.from_numpy(d["cos"]).to(cuda), torch.from_numpy(d["sin"]).to(cuda)
    yr = hn.fused.qk_norm_rope(x, w, (cos, sin))
    yp = hn.fused.qk_norm_rope(x, w, None)
    ro = oracle.bf16_bits(oracle.qk_norm_rope(f32(x), f32(w), (d["cos"], d["sin"])))
    po = oracle.bf16_bits(oracle.qk_norm_rope(f32(x), f32(w), None))
    assert np.array_equal(bits16(yr), ro) and np.array_equal(bits16(yp), po)
    assert (bits16(yr) != d["torch_rope"]).mean() < 1e-2
    assert (bits16(yp) != d["torch_plain"]).mean() < 1e-3


def test_reference_qk_norm_rope(hn, cuda):
    """tests/test_fused.py:24-40 of the reference (b2, l96, h16, d128, rope [16, 56, 56] theta 256)."""
    from oracle import torch_ref
    b, l, h, d = 2, 96, 16, 128
    lin = (torch.randn(b, l, h * d) * 5).bfloat16()
    x = lin.view(b, l, h, d)
    weight = (torch.rand(d) + 0.5).bfloat16()
    cos, sin = torch_ref.rope_freqs([16, 56, 56], 256, 4, 4, 6)
    ref_plain = torch_ref.rms_norm(x, weight)
    ref = torch_ref.apply_rope(ref_plain, cos, sin)
    got = hn.fused.qk_norm_rope(x.to(cuda), weight.to(cuda), (cos.to(cuda), sin.to(cuda))).cpu()
    got_plain = hn.fused.qk_norm_rope(x.to(cuda), weight.to(cuda), None).cpu()
    assert (got_plain != ref_plain).float().mean().item() < 1e-3
    assert (got != ref).float().mean().item() < 1e-2
    assert ((got.float() - ref.float()).norm() / ref.float().norm()).item() < 1e-3


@pytest.mark.parametrize("rope", [True, False])
def test_qk_norm_rope_kv_cache_pass(hn, oracle, cuda, rope):
    """The cache pass: qk_norm_rope's output and world.quantize_kv of it from one launch, against the oracle's
    qk_norm_rope then quantize_kv, on a strided k slice of a fused qkv buffer, with an all-zero head."""
    from oracle import torch_ref
    b, l, h, d = 1, 2 * 3 * 4, 8, 128
    qkv = (torch.randn(b, l, 3 * h * d, generator=torch.Generator().manual_seed(9)) * 3).bfloat16()
    qkv[0, 5, h * d + 2 * d: h * d + 3 * d] = 0            # token 5, head 2 of k: zero -> scale 1
    k = qkv.to(cuda)[..., h * d: 2 * h * d].view(b, l, h, d)
    w = (torch.rand(d) + 0.5).bfloat16().to(cuda)
    cos, sin = torch_ref.rope_freqs([16, 56, 56], 10000, 2, 3, 4)
    tables = (cos.to(cuda), sin.to(cuda)) if rope else None
    y, q8, s8 = hn.fused.qk_norm_rope_kv(k, w, tables)
    assert torch.equal(y, hn.fused.qk_norm_rope(k, w, tables))
    ref = oracle.qk_norm_rope(f32(k.contiguous()), f32(w), (cos.numpy(), sin.numpy()) if rope else None)
    assert np.array_equal(bits16(y), oracle.bf16_bits(ref))
    rq, rs = oracle.quantize_kv(oracle.round_bf16(ref).reshape(b * l, h, d))
    assert np.array_equal(q8.cpu().numpy().reshape(b * l, h, d), rq)
    assert np.array_equal(f32(s8).reshape(b * l, h, 1), rs)
    assert f32(s8).reshape(b * l, h)[5, 2] == 1.0


def test_qk_norm_rope_strided_qkv_and_pair(hn, oracle, cuda):
    """q/k as column slices of a fused [L, 3 * H * D] qkv buffer (token stride 3HD), one and two per launch,
    with the benchmark's 3-D RoPE (t,h,w axes 16/56/56, theta 10000)."""
    from oracle import torch_ref
    b, l, h, d = 1, 2 * 3 * 4, 32, 128
    qkv = (torch.randn(b, l, 3 * h * d, generator=torch.Generator().manual_seed(4)) * 2).bfloat16().to(cuda)
    q = qkv[..., : h * d].view(b, l, h, d)
    k = qkv[..., h * d: 2 * h * d].view(b, l, h, d)
    wq, wk = (torch.rand(d) + 0.5).bfloat16().to(cuda), (torch.rand(d) + 0.5).bfloat16().to(cuda)
    cos, sin = torch_ref.rope_freqs([16, 56, 56], 10000, 2, 3, 4)
    rope = (cos.to(cuda), sin.to(cuda))
    yq = hn.fused.qk_norm_rope(q, wq, rope)
    yq2, yk2 = hn.fused.qk_norm_rope2(q, k, wq, wk, rope)
    assert torch.equal(yq, yq2)
    for got, src, w in ((yq2, q, wq), (yk2, k, wk)):
        ref = oracle.qk_norm_rope(f32(src.contiguous()), f32(w), (cos.numpy(), sin.numpy()))
        assert np.array_equal(bits16(got), oracle.bf16_bits(ref))


def test_pixelumm_qk(hn, oracle, golden, cuda):
    d = golden("pixelumm_qk")
    x = bf16_from_bits(d["x"], cuda)
    wt, whw = bf16_from_bits(d["wt"], cuda), bf16_from_bits(d["whw"], cuda)
    cos, sin = torch.from_numpy(d["cos"]).to(cuda), torch.from_numpy(d["sin"]).to(cuda)
    y = hn.fused.pixelumm_qk(x, wt, whw, cos, sin)
    ref = oracle.pixelumm_qk(f32(x), f32(wt), f32(whw), d["cos"], d["sin"])
    assert np.array_equal(bits16(y), oracle.bf16_bits(ref))
    assert (bits16(y) != d["y"]).mean() < 1e-3


@pytest.mark.parametrize("kind", ["fp8", "int8"])
@pytest.mark.parametrize("rows,d", [(300, 4096), (7, 640), (129, 2048), (33, 12288)])
def test_rmsnorm_quant_bit_exact(hn, oracle, cuda, kind, rows, d):
    """The decoder's RMSNorm + activation quantizer (pixelumm.py:246-259 then kernels.py:22-42) in one pass: codes
    and scales equal the oracle's bit for bit (the oracle is pinned to the reference's RMSNorm by
    test_decoder_fusions_pinned_to_reference)."""
    gen = torch.Generator().manual_seed(rows + d)
    x = (torch.randn(rows, d, generator=gen) * 2.0).bfloat16()
    x[0] *= 50.0
    x[1 % rows] = 0.0
    w = (1.0 + 0.2 * torch.randn(d, generator=gen)).bfloat16()
    q, s = hn.fused.rmsnorm_quant(x.to(cuda), w.to(cuda), 1e-6, kind)
    torch.cuda.synchronize()
    qo, so = oracle.rmsnorm_quant(f32(x), f32(w), 1e-6, kind)
    assert np.array_equal(u8(q), qo) and np.array_equal(f32(s), so)


@pytest.mark.parametrize("kind", ["fp8", "int8"])
@pytest.mark.parametrize("rows,inter", [(300, 12288), (5, 384), (64, 128)])
def test_silu_mul_quant_bit_exact(hn, oracle, cuda, kind, rows, inter):
    """silu(gate) * up + quantizer (pixelumm.py:322-323 then kernels.py:22-42), reading the two halves of one
    stacked gate|up output (strided rows): codes and scales equal the oracle's bit for bit."""
    gen = torch.Generator().manual_seed(rows * 3 + inter)
    gu = (torch.randn(rows, 2 * inter, generator=gen) * 3.0).bfloat16()
    gu[0, :6] = torch.tensor([0.0, -0.0, 95.0, -95.0, 1e-3, -1e-3]).bfloat16()
    dev = gu.to(cuda)
    q, s = hn.fused.silu_mul_quant(dev[:, :inter], dev[:, inter:], kind)
    torch.cuda.synchronize()
    qo, so = oracle.silu_mul_quant(f32(gu[:, :inter]), f32(gu[:, inter:]), kind)
    assert np.array_equal(u8(q), qo) and np.array_equal(f32(s), so)


def test_decoder_mlp_against_reference_arithmetic(hn, oracle, cuda):
    """The decoder layer's MLP half on the fused kernels (ops.decoder_mlp: RMSNorm + e4m3 quantization, one
    stacked gate|up FP8 GEMM, silu * up + e4m3 quantization, down_proj's FP8 GEMM, residual) against the
    reference's FP8-mode arithmetic on the same weights (pixelumm.py:320-337 with DecoderOps.Linear in "fp8"
    mode, pixelumm.py:147-155: every linear quantizes its input to 1 x 128 e4m3 blocks), evaluated by the oracle
    (whose norm and gate fusions equal the reference's modules, test_decoder_fusions_pinned_to_reference): within
    the FP8 tolerance, rel-L2 <= 1e-2. The reference's exact bf16 path (dequantized weights, bf16 activations) is
    farther away by the activations' own e4m3 rounding, ~1e-2, and is printed for the record."""
    import torch.nn.functional as F
    from oracle import torch_ref
    gen = torch.Generator().manual_seed(17)
    m, hidden, inter = 256, 1024, 3072
    x = torch.randn(1, m, hidden, generator=gen).bfloat16()
    w_norm = (1.0 + 0.1 * torch.randn(hidden, generator=gen)).bfloat16()
    wg, wu = torch.randn(inter, hidden, generator=gen) * 0.02, torch.randn(inter, hidden, generator=gen) * 0.02
    wd = torch.randn(hidden, inter, generator=gen) * 0.02
    q8 = [hn.ops.quantize_fp8_block(t.to(cuda)) for t in (wg, wu, wd)]
    gate_up = hn.ops.stack_fp8_linears(q8[0], q8[1])
    y = hn.ops.decoder_mlp(x.to(cuda), w_norm.to(cuda), gate_up, q8[2])
    torch.cuda.synchronize()
    # the reference's FP8 mode on the oracle
    x2 = f32(x).reshape(m, hidden)
    qn, sn = oracle.rmsnorm_quant(x2, f32(w_norm), 1e-6, "fp8")
    gu = oracle.round_bf16(oracle.block_gemm(qn, sn, u8(gate_up[0]), f32(gate_up[1]), kind="fp8", sw_mode="block"))
    qh, sh = oracle.silu_mul_quant(gu[:, :inter], gu[:, inter:], "fp8")
    mlp = oracle.round_bf16(oracle.block_gemm(qh, sh, u8(q8[2][0]), f32(q8[2][1]), kind="fp8", sw_mode="block"))
    ref_fp8 = oracle.round_bf16(x2 + mlp)
    err = rel_l2(f32(y).reshape(m, hidden), ref_fp8)
    assert err <= 1e-2, err
    # the exact bf16 path, for the record
    xf = x.float()
    n = w_norm * (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6)).to(torch.bfloat16)
    deq = [torch_ref.fp8_block_dequantize(q.cpu(), s.cpu()) for q, s in q8]
    exact = x + F.linear(F.silu(F.linear(n, deq[0])) * F.linear(n, deq[1]), deq[2])
    print(f"decoder MLP: rel-L2 {err:.2e} vs the FP8-mode arithmetic, {rel_l2(f32(y), f32(exact)):.2e} vs the "
          "exact bf16 path")
