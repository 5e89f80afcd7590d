"""K1 activation quantizer (hy_nomas/kernels.py:22-54), ops.quantize_g128 (ops.py:41-52) and the int8 KV
quantizer (world.py:83-90) on the GPU against the oracle and the reference's golden vectors: codes and
scales bit-exact."""
import numpy as np
import pytest
import torch

from hn_testutil import bf16_from_bits, f32, u8

pytestmark = pytest.mark.gpu


def test_golden_vectors(hn, golden, cuda):
    d = golden("quant_act")
    x = bf16_from_bits(d["x"], cuda)
    for kind in ("int8", "fp8"):
        q, s = hn.kernels.quantize_activations(x, kind)
        torch.cuda.synchronize()
        assert np.array_equal(u8(q), d[f"{kind}_q"]), kind
        assert np.array_equal(f32(s).view(np.uint32), d[f"{kind}_s"].view(np.uint32)), kind


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("m,k", [(1, 128), (17, 384), (1000, 2048), (300, 4096)])
@pytest.mark.parametrize("kind", ["int8", "fp8"])
def test_random_shapes_bit_exact(hn, oracle, cuda, dtype, m, k, kind):
    gen = torch.Generator().manual_seed(m * 7 + k)
    x = (torch.randn(m, k, generator=gen) * 3).to(dtype)
    x[:, torch.randperm(k, generator=gen)[: max(1, k // 100)]] *= 20
    if m > 3:
        x[2] = 0
    q, s = hn.kernels.quantize_activations(x.to(cuda), kind)
    qo, so = oracle.quantize_activations(f32(x), kind)
    assert np.array_equal(u8(q), qo)
    assert np.array_equal(f32(s), so)


def test_strided_rows(hn, oracle, cuda):
    base = (torch.randn(64, 1024) * 2).bfloat16()
    x = base[:, :512]                       # row pitch 1024, 512 columns
    q, s = hn.kernels.quantize_activations(base.to(cuda)[:, :512], "int8")
    qo, so = oracle.quantize_activations(f32(x), "int8")
    assert np.array_equal(u8(q), qo) and np.array_equal(f32(s), so)


@pytest.mark.parametrize("kind", ["int8", "fp8"])
@pytest.mark.parametrize("k", [128, 384, 3072, 4096, 16384, 20480])
def test_per_token(hn, oracle, cuda, kind, k):
    """Row lengths covering every per-row kernel shape: one to eight register chunks per thread (partial last
    chunk rows at 384 and 3072) and the two-pass form beyond 16384."""
    rows = 100 if k <= 4096 else 12
    x = (torch.randn(rows, k, generator=torch.Generator().manual_seed(3)) * 2).bfloat16()
    q, s = hn.kernels.quantize_activations(x.to(cuda), kind, per_token=True)
    qo, so = oracle.quantize_activations(f32(x), kind, per_row=True)
    assert np.array_equal(u8(q), qo) and np.array_equal(f32(s), so)


def test_ops_quantize_g128(hn, golden, cuda):
    d = golden("quantize_g128")
    q, s = hn.ops.quantize_g128(torch.from_numpy(d["w"]).to(cuda))
    assert np.array_equal(q.cpu().numpy(), d["q"]) and np.array_equal(f32(s), d["s"])
    deq = hn.ops.dequantize_g128(q, s)
    assert np.array_equal(deq.cpu().view(torch.int16).numpy().view(np.uint16), d["deq"])


def test_ops_quantize_g128_ragged_k(hn, cuda):
    from oracle import torch_ref
    w = torch.randn(33, 200, generator=torch.Generator().manual_seed(5)) * 0.05
    q, s = hn.ops.quantize_g128(w.to(cuda))
    qr, sr = torch_ref.quantize_g128(w)
    assert torch.equal(q.cpu(), qr) and torch.equal(s.cpu(), sr)


def test_quantize_kv(hn, golden, cuda):
    d = golden("quantize_kv")
    x = bf16_from_bits(d["x"], cuda)
    l, h, dd = x.shape
    q = torch.empty((l * h, dd), dtype=torch.int8, device=cuda)
    s = torch.empty((l * h,), dtype=torch.float32, device=cuda)
    rc = hn.lib.lib.hn_quantize_kv(hn.lib.ptr(x), l * h, dd, hn.lib.ptr(q), hn.lib.ptr(s), hn.lib.stream_of(x))
    hn.lib.check(rc, "hn_quantize_kv")
    torch.cuda.synchronize()
    assert np.array_equal(q.cpu().numpy().reshape(d["q"].shape), d["q"])
    assert np.array_equal(f32(s).reshape(d["s"].shape), d["s"])


def test_world_kv_golden(hn, golden, cuda):
    """hy_nomas/world.py:83-94 through the package's world module: codes, scales and the dequantized bf16,
    bit-exact with the reference's own outputs."""
    d = golden("quantize_kv")
    x = bf16_from_bits(d["x"], cuda)
    q, s = hn.world.quantize_kv(x)
    assert np.array_equal(q.cpu().numpy(), d["q"]) and np.array_equal(f32(s), d["s"])
    y = hn.world.dequantize_kv(torch.from_numpy(d["q"]).to(cuda), torch.from_numpy(d["s"]).to(cuda))
    assert np.array_equal(y.cpu().view(torch.int16).numpy().view(np.uint16), d["y"])


@pytest.mark.parametrize("rows,d", [(1, 128), (37, 128), (4096 * 4, 128), (300, 256), (3, 16)])
def test_dequantize_kv_random(hn, oracle, cuda, rows, d):
    gen = torch.Generator().manual_seed(rows + d)
    q = torch.randint(-127, 128, (rows, d), generator=gen, dtype=torch.int8)
    q[0, :4] = torch.tensor([-127, 127, 0, -1], dtype=torch.int8)
    s = torch.rand(rows, 1, generator=gen) * 0.05
    s[-1] = 1.0                                        # an all-zero head's scale
    y = hn.world.dequantize_kv(q.to(cuda), s.to(cuda))
    torch.cuda.synchronize()
    ref = oracle.dequantize_kv(q.numpy(), s.numpy())
    assert np.array_equal(y.cpu().view(torch.int16).numpy().view(np.uint16), oracle.bf16_bits(ref))


def test_quantize_fp8_block_golden(hn, golden, cuda):
    """pixelumm.NomasFP8Block128Layout.quantize (pixelumm.py:77-82): e4m3 codes and block scales bit-exact
    with the reference's own output, and the block dequantization (pixelumm.py:60-63)."""
    d = golden("block_gemm")
    q, s = hn.ops.quantize_fp8_block(torch.from_numpy(d["w"]).to(cuda))
    assert np.array_equal(u8(q), d["fp8_qw"]) and np.array_equal(f32(s), d["fp8_sw_block"])
    deq = hn.ops.dequantize_fp8_block(q, s)
    assert np.array_equal(deq.cpu().view(torch.int16).numpy().view(np.uint16), d["fp8_deq_w"])


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_quantize_fp8_block_random(hn, oracle, cuda, dtype):
    gen = torch.Generator().manual_seed(21)
    w = (torch.randn(384, 640, generator=gen) * 0.02)
    w[5, 7] = 3.0           # a block whose absmax is one outlier
    w[256:, 512:] = 0.0     # an all-zero block: scale 1e-4 / 448, codes 0
    w = w.to(dtype)
    q, s = hn.ops.quantize_fp8_block(w.to(cuda))
    qr, sr = oracle.quantize_fp8_block(w.float().numpy())
    assert np.array_equal(u8(q), qr) and np.array_equal(f32(s), sr)


@pytest.mark.parametrize("kind", ["int8", "fp8"])
def test_edge_values_bit_exact(hn, oracle, cuda, kind):
    """Groups that exercise the quantizer's division: all zero, negative zeros, subnormal-range values (the
    scale falls below 2^-90 and the kernel takes the IEEE division), exact .5 ties of the int8 rounding (peak
    127 with half-integer values), mixed signs at the group maximum, and values near the bf16 maximum."""
    g = 128
    rows = []
    rows.append(np.zeros(4 * g, np.float32))
    rows.append(np.full(4 * g, -0.0, np.float32))
    tiny = np.float32(1e-37) * np.linspace(-1, 1, 4 * g, dtype=np.float32)
    rows.append(tiny)
    ties = (np.arange(4 * g, dtype=np.float32) % 255 - 127).astype(np.float32) + 0.5
    ties[::g] = 127.0
    rows.append(ties)
    mixed = np.linspace(-3.0, 3.0, 4 * g, dtype=np.float32)
    mixed[5] = -3.0
    rows.append(mixed)
    rows.append(np.linspace(-3e38, 3e38, 4 * g, dtype=np.float32))
    rows.append((np.random.default_rng(3).standard_normal(4 * g) * 1e-30).astype(np.float32))
    x = torch.from_numpy(np.stack(rows)).bfloat16()
    q, s = hn.kernels.quantize_activations(x.to(cuda), kind)
    qo, so = oracle.quantize_activations(f32(x), kind)
    assert np.array_equal(u8(q), qo)
    assert np.array_equal(f32(s), so)


@pytest.mark.parametrize("kind", ["int8", "fp8"])
def test_per_token_edge_rows(hn, oracle, cuda, kind):
    """Per-token quantization of the edge rows (zeros, negative zeros, subnormal-range values, .5 ties, values
    near the bf16 maximum) over a 1024-wide row: codes and scales bit-exact with the oracle."""
    k = 1024
    rows = [np.zeros(k, np.float32), np.full(k, -0.0, np.float32),
            np.float32(1e-37) * np.linspace(-1, 1, k, dtype=np.float32),
            (np.arange(k, dtype=np.float32) % 255 - 127).astype(np.float32) + 0.5,
            np.linspace(-3e38, 3e38, k, dtype=np.float32)]
    rows[3][0] = 127.0
    x = torch.from_numpy(np.stack(rows)).bfloat16()
    q, s = hn.kernels.quantize_activations(x.to(cuda), kind, per_token=True)
    qo, so = oracle.quantize_activations(f32(x), kind, per_row=True)
    assert np.array_equal(u8(q), qo)
    assert np.array_equal(f32(s).reshape(-1), so.reshape(-1))


@pytest.mark.parametrize("per_token", [False, True])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_round_half_even_option(hn, oracle, cuda, per_token, dtype):
    """int8 codes rounded half to even (the option beside the reference's half-away rounding): exact ties
    at scale 1 and random rows (with a tie row), bf16 (fast quotient) and fp32 (IEEE division) inputs,
    bit-exact with the oracle; the default stays half away from zero."""
    import test_oracle_math
    ties, _ = test_oracle_math.tie_rows()
    gen = torch.Generator().manual_seed(7)
    rnd = (torch.randn(30, 512, generator=gen) * 3).numpy()
    x = np.concatenate([np.pad(ties, ((0, 0), (0, 512 - 128))), rnd]).astype(np.float32)
    xt = torch.from_numpy(x).to(dtype)
    xf = xt.float().numpy()
    for rne in (True, False):
        q, s = hn.kernels.quantize_activations(xt.to(cuda), "int8", per_token=per_token, round_half_even=rne)
        qo, so = oracle.quantize_activations(xf, "int8", per_row=per_token, round_half_even=rne)
        assert np.array_equal(u8(q), qo), rne
        assert np.array_equal(f32(s).reshape(-1), so.reshape(-1)), rne
    codes_even = hn.kernels.quantize_activations(xt.to(cuda), "int8", per_token=per_token, round_half_even=True)[0]
    codes_away = hn.kernels.quantize_activations(xt.to(cuda), "int8", per_token=per_token)[0]
    assert not torch.equal(codes_even, codes_away)          # the tie rows differ between the two modes


@pytest.mark.parametrize("k", [384, 2048, 3072, 4096, 16384, 20480])
@pytest.mark.parametrize("kind,rne", [("int8", False), ("int8", True), ("fp8", False)])
def test_group_scales_one_cta_per_row(hn, oracle, cuda, k, kind, rne):
    """Enough rows for the one-CTA-per-row group quantizer (rows of 2048 to 16384 in registers; shorter and
    longer rows on the grid-stride kernel), strided rows, outlier channels and a zero row: codes and scales
    bit-exact."""
    m = 2 * torch.cuda.get_device_properties(0).multi_processor_count + 3
    gen = torch.Generator().manual_seed(k + (7 if rne else 0))
    base = (torch.randn(m, k + 128, generator=gen) * 3).bfloat16()
    base[:, torch.randperm(k, generator=gen)[: max(1, k // 64)]] *= 20
    base[5] = 0
    x = base[:, :k]
    q, s = hn.kernels.quantize_activations(base.to(cuda)[:, :k], kind, round_half_even=rne)
    qo, so = oracle.quantize_activations(f32(x), kind, round_half_even=rne)
    assert np.array_equal(u8(q), qo)
    assert np.array_equal(f32(s), so)


def test_quantize_kv_many_heads(hn, oracle, cuda):
    """world.quantize_kv at a DiT-like size (32 heads of 128 per token) against the oracle."""
    gen = torch.Generator().manual_seed(17)
    x = (torch.randn(700, 32, 128, generator=gen) * 2).bfloat16()
    x[3, 4] = 0
    q, s = hn.world.quantize_kv(x.to(cuda))
    qo, so = oracle.quantize_kv(f32(x))
    assert np.array_equal(q.cpu().numpy(), qo) and np.array_equal(f32(s), so)
