"""Pin the CPU oracle to the reference: golden vectors made by running the reference's own kernels
(Triton interpreter) and torch functions (tests/golden/make_golden.py). CPU only."""
import numpy as np
import pytest


def bf(b):
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def test_quantize_activations_int8_fp8(oracle, golden):
    d = golden("quant_act")   # kernels.py:22-54, includes a zero row, exact ties and tiny values
    x = bf(d["x"])
    for kind in ("int8", "fp8"):
        q, s = oracle.quantize_activations(x, kind)
        assert np.array_equal(q, d[f"{kind}_q"]), kind
        assert np.array_equal(s.view(np.uint32), d[f"{kind}_s"].view(np.uint32)), kind


def test_quantize_ties_round_half_away(oracle):
    # peak 127 -> scale exactly 1.0, so x/s hits k + 0.5 exactly (kernels.py:35 rounds half away from zero)
    x = np.zeros((1, 128), np.float32)
    x[0, :7] = [127.0, 2.5, -3.5, 0.5, -0.5, 126.5, -126.5]
    q, s = oracle.quantize_activations(x)
    assert s[0, 0] == 1.0
    assert list(q.view(np.int8)[0, :7]) == [127, 3, -4, 1, -1, 127, -127]


def test_quantize_g128_and_dequant(oracle, golden):
    d = golden("quantize_g128")  # ops.py:41-62
    q, s = oracle.quantize_g128(d["w"])
    assert np.array_equal(q, d["q"]) and np.array_equal(s, d["s"])
    assert np.array_equal(oracle.bf16_bits(oracle.dequantize_g128(q, s)), d["deq"])


def test_gemm_accumulator_bit_exact_vs_interpreter(oracle, golden):
    d = golden("block_gemm")  # kernels.py:80-137 under the interpreter: no FMA contraction
    acc = oracle.block_gemm(d["qa"], d["sa"], d["qw"], d["sw"], bf(d["bias"]), fma=False)
    assert np.array_equal(acc.view(np.uint32), d["acc_f32"].view(np.uint32))
    assert np.array_equal(oracle.bf16_bits(oracle.round_bf16(acc)), d["ep0_bf16"])


def test_gemm_fma_promotion_close_to_interpreter(oracle, golden):
    # the kernels' promotion fuses the last multiply with the add (one rounding fewer)
    d = golden("block_gemm")
    acc = oracle.block_gemm(d["qa"], d["sa"], d["qw"], d["sw"], bf(d["bias"]), fma=True)
    ref = d["acc_f32"]
    assert np.abs(acc - ref).max() <= 4 * np.spacing(np.abs(ref).max())
    mism = (oracle.bf16_bits(oracle.round_bf16(acc)) != d["ep0_bf16"]).mean()
    assert mism < 1e-2


def test_gemm_gelu_epilogues(oracle, golden):
    d = golden("block_gemm")
    h = oracle.block_gemm(d["qa"], d["sa"], d["qw"], d["sw"], bf(d["bias"]), epilogue="gelu", fma=False)
    assert (oracle.bf16_bits(h) != d["ep1_bf16"]).mean() < 1e-3
    h, qh, qs = oracle.block_gemm(d["qa"], d["sa"], d["qw"], d["sw"], bf(d["bias"]), epilogue="gelu_quant",
                                  fma=False)
    assert (qh != d["ep2_q"]).mean() < 1e-3
    assert np.allclose(qs, d["ep2_s"], rtol=1e-3)


def test_fp8_weight_and_activation_codes(oracle, golden):
    d = golden("block_gemm")  # pixelumm.py:77-82 weights, kernels.py:39-41 activations
    q8, s8 = oracle.quantize_fp8_block(d["w"])
    assert np.array_equal(q8, d["fp8_qw"]) and np.array_equal(s8, d["fp8_sw_block"])
    qa, sa = oracle.quantize_activations(bf(d["x"]), "fp8")
    assert np.array_equal(qa, d["fp8_qa"]) and np.array_equal(sa, d["fp8_sa"])
    assert np.array_equal(oracle.bf16_bits(oracle.dequantize_fp8_block(q8, s8)), d["fp8_deq_w"])


def test_fp8_gemm_close_to_interpreter(oracle, golden):
    d = golden("block_gemm")
    ref = d["fp8_acc_f32"]
    bias = bf(d["bias"])
    blk = oracle.block_gemm(d["fp8_qa"], d["fp8_sa"], d["fp8_qw"], d["fp8_sw_block"], bias, kind="fp8",
                            sw_mode="block")
    exp = np.repeat(d["fp8_sw_block"], 128, axis=0)
    grp = oracle.block_gemm(d["fp8_qa"], d["fp8_sa"], d["fp8_qw"], exp, bias, kind="fp8", fma=False)
    for got in (blk, grp):
        assert np.linalg.norm(got - ref) / np.linalg.norm(ref) < 1e-6


@pytest.mark.parametrize("tag,b", [("d2048", 2), ("d4096", 1)])
def test_adaln_quant_and_adaln(oracle, golden, tag, b):
    d = golden("adaln")  # kernels.py:173-195, fused.py:37-52, model.py:103-111
    D = int(tag[1:])
    x = bf(d[f"{tag}_x"]).reshape(b, -1, D)
    sh, sc = bf(d[f"{tag}_shift"]).reshape(b, D), bf(d[f"{tag}_scale"]).reshape(b, D)
    q, s = oracle.adaln_quant(x, sh, sc)
    assert (q != d[f"{tag}_q"]).mean() < 1e-3          # the reference's own bound (tests/test_fused.py:59)
    assert np.allclose(s, d[f"{tag}_s"], rtol=1e-3)
    y = oracle.bf16_bits(oracle.round_bf16(oracle.adaln(x, sh, sc))).reshape(-1)
    assert (y != d[f"{tag}_y"].reshape(-1)).mean() < 1e-3
    assert (y != d[f"{tag}_torch_y"].reshape(-1)).mean() < 1e-3   # tests/test_fused.py:20


def test_qk_norm_rope(oracle, golden):
    d = golden("qk_norm_rope")  # fused.py:65-91 vs model.py:89-138
    x, w = bf(d["x"]), bf(d["w"])
    yr = oracle.bf16_bits(oracle.qk_norm_rope(x, w, (d["cos"], d["sin"])))
    yp = oracle.bf16_bits(oracle.qk_norm_rope(x, w, None))
    assert (yp != d["y_plain"]).mean() < 1e-3 and (yp != d["torch_plain"]).mean() < 1e-3
    assert (yr != d["y_rope"]).mean() < 1e-2 and (yr != d["torch_rope"]).mean() < 1e-2
    ref = bf(d["torch_rope"])
    assert np.linalg.norm(bf(yr) - ref) / np.linalg.norm(ref) < 1e-3


def test_gated_residual_exact(oracle, golden):
    d = golden("gated_residual")  # fused.py:108-118 and torch x + y * g (tests/test_fused.py:43-49: exact)
    g = bf(d["g"]).reshape(2, -1)
    out = oracle.bf16_bits(oracle.round_bf16(oracle.gated_residual(bf(d["x"]), bf(d["y"]), g)))
    assert np.array_equal(out, d["out"]) and np.array_equal(out, d["torch_out"])


def test_pixelumm_qk(oracle, golden):
    d = golden("pixelumm_qk")  # fused.py:131-175
    y = oracle.pixelumm_qk(bf(d["x"]), bf(d["wt"]), bf(d["whw"]), d["cos"], d["sin"])
    assert (oracle.bf16_bits(y) != d["y"]).mean() < 1e-3


def test_quantize_kv(oracle, golden):
    d = golden("quantize_kv")  # world.py:83-90
    q, s = oracle.quantize_kv(bf(d["x"]))
    assert np.array_equal(q, d["q"]) and np.array_equal(s, d["s"])


def test_dequantize_kv(oracle, golden):
    d = golden("quantize_kv")  # world.py:93-94, on the reference's own codes and scales
    y = oracle.dequantize_kv(d["q"], d["s"])
    assert np.array_equal(oracle.bf16_bits(y), d["y"])


def test_decoder_fusions_pinned_to_reference(oracle, golden):
    """The decoder fusions' oracle against the reference's own pixelumm.RMSNorm and MLP gate expression
    (tests/golden/make_decoder_golden.py), each followed by the reference's activation quantizer: on these vectors
    the codes and scales equal the quantizer's output for the reference's bf16 result, e4m3 and int8 alike
    (torch's summation order and exp move no bf16 rounding here)."""
    d = golden("decoder")
    b2f = oracle.from_bf16_bits
    x, w, y, g, u, h = (b2f(d[k]) for k in ("x", "w", "y", "g", "u", "h"))
    for kind in ("fp8", "int8"):
        q, s = oracle.rmsnorm_quant(x, w, float(d["eps"]), kind=kind)
        q_ref, s_ref = oracle.quantize_activations(y, kind)
        assert np.array_equal(q, q_ref) and np.array_equal(s, s_ref)
        q, s = oracle.silu_mul_quant(g, u, kind=kind)
        q_ref, s_ref = oracle.quantize_activations(h, kind)
        assert np.array_equal(q, q_ref) and np.array_equal(s, s_ref)
