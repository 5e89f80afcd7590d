"""The sm_100a attention kernel (hy_nomas/model.py:145-151) against a torch fp32 reference of the same op, on
ragged and DiT-sized shapes, with logits sharp enough to exercise the running-maximum rescale, strided inputs,
and the fused int8 output quantizer (bit-identical to quantizing the bf16 output with the activation quantizer).

Tolerance: rel-L2 <= 1e-2 against fp32 (a bf16 attention's error: bf16 inputs are exact in fp32, the kernel
rounds P to bf16 for the P V product and writes bf16; torch's own bf16 SDPA lands in the same range, printed).
"""
import math

import pytest
import torch
import torch.nn.functional as F

from hn_testutil import rel_l2

pytestmark = pytest.mark.gpu

TOL = 1e-2


def ref_fp32(q, k, v, scale=None):
    """softmax(q k^T * scale) v in fp32, [B, L, H, D] layout."""
    scale = 1.0 / math.sqrt(q.shape[-1]) if scale is None else scale
    qf, kf, vf = (t.float().transpose(1, 2) for t in (q, k, v))
    return F.scaled_dot_product_attention(qf, kf, vf, scale=scale).transpose(1, 2)


def rand(shape, gen, device, scale=1.0):
    return (torch.randn(shape, generator=gen, device=device) * scale).to(torch.bfloat16)


@pytest.mark.parametrize("b,lq,lk,h", [(1, 128, 64, 1), (1, 256, 256, 2), (1, 300, 777, 2), (2, 200, 130, 3),
                                       (1, 1, 1, 1), (1, 129, 65, 1), (1, 512, 1000, 4)])
def test_attention_matches_fp32_reference(hn, cuda, b, lq, lk, h):
    from hy_nomas_b200.attention import attention
    gen = torch.Generator(device=cuda).manual_seed(lq * 7 + lk)
    q, k, v = rand((b, lq, h, 128), gen, cuda), rand((b, lk, h, 128), gen, cuda), rand((b, lk, h, 128), gen, cuda)
    out = attention(q, k, v)
    again = attention(q, k, v)
    torch.cuda.synchronize()
    ref = ref_fp32(q, k, v)
    sdpa = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)).transpose(1, 2)
    err = rel_l2(out.float().cpu().numpy(), ref.cpu().numpy())
    print(f"rel-L2 vs fp32: kernel {err:.2e}, torch bf16 SDPA "
          f"{rel_l2(sdpa.float().cpu().numpy(), ref.cpu().numpy()):.2e}")
    assert out.shape == q.shape and out.dtype == torch.bfloat16
    assert torch.isfinite(out).all()
    assert err < TOL
    assert torch.equal(out.view(torch.int16), again.view(torch.int16))    # deterministic
    rc, code = hn.lib.device_error()
    assert rc == 0 and code == 0


def test_sharp_logits_rescale_running_maximum(hn, cuda):
    """Logits with a spread of ~60 (base e) and the largest keys last: the running maximum grows by more than 2^8
    across key steps, so the kernel rescales its O rows in TMEM."""
    from hy_nomas_b200.attention import attention
    gen = torch.Generator(device=cuda).manual_seed(5)
    b, lq, lk, h = 1, 256, 640, 2
    q = rand((b, lq, h, 128), gen, cuda, scale=3.0)
    k = rand((b, lk, h, 128), gen, cuda)
    ramp = torch.linspace(0.2, 2.5, lk, device=cuda).view(1, lk, 1, 1)
    k = (k.float() * ramp).to(torch.bfloat16)
    v = rand((b, lk, h, 128), gen, cuda)
    out = attention(q, k, v)
    ref = ref_fp32(q, k, v)
    err = rel_l2(out.float().cpu().numpy(), ref.cpu().numpy())
    print(f"sharp logits rel-L2 {err:.2e}")
    assert err < TOL


def test_scale_argument(hn, cuda):
    from hy_nomas_b200.attention import attention
    gen = torch.Generator(device=cuda).manual_seed(6)
    q, k, v = rand((1, 128, 2, 128), gen, cuda), rand((1, 192, 2, 128), gen, cuda), rand((1, 192, 2, 128), gen, cuda)
    out = attention(q, k, v, scale=0.3)
    assert rel_l2(out.float().cpu().numpy(), ref_fp32(q, k, v, 0.3).cpu().numpy()) < TOL


def test_quantized_output_matches_activation_quantizer(hn, cuda):
    """The fused output quantizer equals kernels.quantize_activations on the bf16 output, code for code."""
    from hy_nomas_b200.attention import attention_quant
    gen = torch.Generator(device=cuda).manual_seed(7)
    b, lq, lk, h = 2, 300, 500, 4
    q, k, v = rand((b, lq, h, 128), gen, cuda), rand((b, lk, h, 128), gen, cuda), rand((b, lk, h, 128), gen, cuda)
    out, (q8, s8) = attention_quant(q, k, v, keep_output=True)
    q8_only, s8_only = attention_quant(q, k, v)
    rq, rs = hn.kernels.quantize_activations(out.reshape(b * lq, h * 128))
    torch.cuda.synchronize()
    assert torch.equal(q8, rq) and torch.equal(s8.view(torch.int32), rs.view(torch.int32))
    assert torch.equal(q8_only, q8) and torch.equal(s8_only, s8)


def test_strided_inputs_equal_contiguous(hn, cuda):
    """q, k, v as views of one packed [B, L, 3, H, 128] buffer (row stride 3 * H * 128) and out into a strided
    view give the contiguous result bit for bit."""
    from hy_nomas_b200.attention import attention
    gen = torch.Generator(device=cuda).manual_seed(8)
    b, l, h = 1, 384, 2
    qkv = rand((b, l, 3, h, 128), gen, cuda)
    q, k, v = qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2]
    dense = attention(q.contiguous(), k.contiguous(), v.contiguous())
    wide = torch.zeros((b, l, h + 1, 128), dtype=torch.bfloat16, device=cuda)
    strided = attention(q, k, v, out=wide[:, :, :h])
    torch.cuda.synchronize()
    assert torch.equal(strided.view(torch.int16), dense.view(torch.int16))
    assert torch.count_nonzero(wide[:, :, h]) == 0


def test_dit_rank_shape(hn, cuda):
    """One rank of the 8-way sequence-parallel step: 2530 queries x 20240 keys x 32 heads."""
    from hy_nomas_b200.attention import attention
    gen = torch.Generator(device=cuda).manual_seed(9)
    q = rand((1, 2530, 32, 128), gen, cuda)
    k, v = rand((1, 20240, 32, 128), gen, cuda), rand((1, 20240, 32, 128), gen, cuda)
    out = attention(q, k, v)
    ref = ref_fp32(q, k, v)
    err = rel_l2(out.float().cpu().numpy(), ref.cpu().numpy())
    print(f"DiT rank shape rel-L2 {err:.2e}")
    assert err < TOL


def test_log_sum_exp_is_natural_log(hn, cuda):
    from hy_nomas_b200.attention import attention_lse
    gen = torch.Generator(device=cuda).manual_seed(10)
    q, k, v = rand((1, 64, 2, 128), gen, cuda), rand((1, 96, 2, 128), gen, cuda), rand((1, 96, 2, 128), gen, cuda)
    o, lse = attention_lse(q, k, v)
    logits = torch.einsum("bqhd,bkhd->bhqk", q.float(), k.float()) / math.sqrt(128)
    want = torch.logsumexp(logits, dim=-1)
    assert lse.shape == (1, 2, 64)
    assert torch.allclose(lse.float(), want, atol=2e-2, rtol=0), (lse.float() - want).abs().max().item()


def test_merge_of_pieces_equals_whole(hn, cuda):
    """Attention in three key pieces merged by log-sum-exp: the whole attention within the bf16 tolerance; its
    fused quantizer equals the activation quantizer on the merged output; one piece merges to itself exactly."""
    from hy_nomas_b200.attention import attention_lse, merge
    gen = torch.Generator(device=cuda).manual_seed(11)
    b, lq, lk, h = 1, 300, 1000, 4
    q, k, v = rand((b, lq, h, 128), gen, cuda), rand((b, lk, h, 128), gen, cuda), rand((b, lk, h, 128), gen, cuda)
    cuts = [0, 100, 612, lk]
    pieces = [attention_lse(q, k[:, a:c], v[:, a:c]) for a, c in zip(cuts[:-1], cuts[1:])]
    out, (q8, s8) = merge(pieces, quantize=True, keep_output=True)
    err = rel_l2(out.float().cpu().numpy(), ref_fp32(q, k, v).cpu().numpy())
    print(f"merged pieces rel-L2 {err:.2e}")
    assert err < TOL
    rq, rs = hn.kernels.quantize_activations(out.reshape(b * lq, h * 128))
    assert torch.equal(q8, rq) and torch.equal(s8.view(torch.int32), rs.view(torch.int32))
    one = attention_lse(q, k, v)
    assert torch.equal(merge([one], quantize=False).view(torch.int16), one[0].contiguous().view(torch.int16))


def test_rejects_bad_arguments(hn, cuda):
    import ctypes
    from hy_nomas_b200.attention import attention
    L = hn.lib
    q = torch.zeros((1, 128, 1, 64), dtype=torch.bfloat16, device=cuda)
    with pytest.raises(ValueError):
        attention(q, q, q)
    x = torch.zeros((1, 128, 1, 128), dtype=torch.bfloat16, device=cuda)
    p = ctypes.c_void_p(x.data_ptr())
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    args = lambda d, rs, out: (p, rs, 128, 128 * 128, p, 128, 128, 128 * 128, p, 128, 128, 128 * 128, 1, 128, 128, 1,
                               d, 0.1, out, 128, 128, 128 * 128, None, None, st)
    y = torch.empty_like(x)
    o = ctypes.c_void_p(y.data_ptr())
    assert L.lib.hn_attention(*args(64, 128, o)) == 7          # HN_ERR_UNSUPPORTED
    assert L.lib.hn_attention(*args(128, 100, o)) == 2         # HN_ERR_ALIGN (row stride)
    assert L.lib.hn_attention(*args(128, 128, None)) == 5      # HN_ERR_ARG (no output)
    assert L.lib.hn_attention(*args(128, 128, o)) == 0
    torch.cuda.synchronize()
