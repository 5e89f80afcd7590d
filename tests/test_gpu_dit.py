"""The synthetic DiT block (hy_nomas/model.py:246-286 on the fused int8 path) on the B200 kernels.

Stage by stage, every kernel output of one block is bit-exact with the oracle evaluated on the same stage
inputs (taken from the GPU run): modulation linear, LN+modulate+quant, the q|k and v GEMMs, QK-norm+RoPE,
the attention projection, residual+LN+quant, fc1 with GELU+requant, fc2 and the final residual. Attention is
torch SDPA (unchanged from the reference) and is compared with a float64 softmax within rel-L2 1e-2. The whole
block, run end to end on the oracle from the same inputs, is within rel-L2 2e-2 (quantization steps amplify
the attention's rounding differences at a few code boundaries).
"""
import multiprocessing as mp
import os
import socket

import numpy as np
import pytest
import torch

import sp_worker
from dit_oracle_ops import OracleOps
from hn_testutil import rel_l2

pytestmark = pytest.mark.gpu


def small_cfg():
    from hy_nomas_b200.dit import DiTConfig
    # 200 tokens (a ragged last M tile), hidden 512 = 4 heads x 128
    return DiTConfig(hidden=512, heads=4, mlp_ratio=4, blocks=1, grid=(2, 10, 10))


def to_cpu_weights(w):
    from hy_nomas_b200.dit import BlockWeights, QLinear
    ql = lambda l: QLinear(l.q.cpu(), l.s.cpu(), l.bias.cpu())  # noqa: E731
    return BlockWeights(mod=ql(w.mod), qk=ql(w.qk), v=ql(w.v), proj=ql(w.proj), fc1=ql(w.fc1), fc2=ql(w.fc2),
                        q_norm=w.q_norm.cpu(), k_norm=w.k_norm.cpu())


def same(a, b):
    a, b = a.detach().cpu(), b.detach().cpu()
    if a.dtype == torch.bfloat16:
        return torch.equal(a.view(torch.int16), b.to(torch.bfloat16).view(torch.int16))
    return torch.equal(a, b.to(a.dtype))


@pytest.fixture(scope="module")
def block_run(hn, oracle, cuda):
    from hy_nomas_b200.dit import block_forward, make_block_weights, rope_freqs
    from hy_nomas_b200.sequence_parallel import SequenceParallel
    cfg = small_cfg()
    gen = torch.Generator(device=cuda).manual_seed(5)
    w = make_block_weights(cfg, gen, cuda)
    rope = rope_freqs(cfg.rope_dims, cfg.theta, *cfg.grid, device=cuda)
    g = torch.Generator().manual_seed(6)
    x = torch.randn(1, cfg.tokens, cfg.hidden, generator=g).to(torch.bfloat16).to(cuda)
    vec = torch.randn(1, cfg.hidden, generator=g).to(torch.bfloat16).to(cuda)
    trace = {}
    out = block_forward(cfg, w, x, vec, rope, SequenceParallel(), trace=trace)
    torch.cuda.synchronize()
    rc, code = hn.lib.device_error()
    assert rc == 0 and code == 0
    return cfg, to_cpu_weights(w), x.cpu(), vec.cpu(), (rope[0].cpu(), rope[1].cpu()), \
        {k: (v.cpu() if torch.is_tensor(v) else v) for k, v in trace.items()}, out.cpu()


def test_stagewise_bit_exact(block_run):
    cfg, w, x, vec, rope, t, out = block_run
    O = OracleOps
    b, l, d = x.shape
    h, hd = cfg.heads, cfg.head_dim
    assert same(t["mods"], O.linear(t["act"], w.mod))
    shift1, scale1, gate1, shift2, scale2, gate2 = t["mods"].chunk(6, dim=-1)
    qa, sa = O.adaln_quant(x, shift1, scale1)
    assert same(t["qa"], qa) and same(t["sa"], sa)
    assert same(t["qk"], O.gemm(t["qa"], t["sa"], w.qk))
    yq, yk = torch.empty(b, l, h, hd, dtype=torch.bfloat16), torch.empty(b, l, h, hd, dtype=torch.bfloat16)
    O.qk_norm_rope2(t["qk"][:, :d].reshape(b, l, h, hd), t["qk"][:, d:].reshape(b, l, h, hd), w.q_norm, w.k_norm,
                    rope, out=(yq, yk))
    assert same(t["q"], yq) and same(t["k_full"], yk)
    assert same(t["v_full"].reshape(b * l, d), O.gemm(t["qa"], t["sa"], w.v))
    assert same(t["proj"].reshape(b * l, d), O.linear(t["attn"], w.proj))
    x1, qa2, sa2 = O.gated_residual_adaln_quant(x, t["proj"], gate1, shift2, scale2)
    assert same(t["x1"], x1) and same(t["qa2"], qa2) and same(t["sa2"], sa2)
    qh, sh = O.gemm(t["qa2"], t["sa2"], w.fc1, epilogue="gelu_quant")
    assert same(t["qh"], qh) and same(t["sh"], sh)
    assert same(t["y"].reshape(b * l, d), O.gemm(t["qh"], t["sh"], w.fc2))
    assert same(out, O.gated_residual(t["x1"], t["y"], gate2))


def test_attention_within_tolerance(block_run):
    cfg, w, x, vec, rope, t, out = block_run
    b, l, d = x.shape
    ref = OracleOps.attention(t["q"], t["k_full"], t["v_full"]).reshape(b * l, d)
    assert rel_l2(t["attn"].float().numpy(), ref.float().numpy()) < 1e-2


def test_block_end_to_end(block_run):
    from hy_nomas_b200.dit import block_forward
    from hy_nomas_b200.sequence_parallel import SequenceParallel
    cfg, w, x, vec, rope, t, out = block_run
    ref = block_forward(cfg, w, x, vec, rope, SequenceParallel(), ops=OracleOps)
    err = rel_l2(out.float().numpy(), ref.float().numpy())
    assert err < 2e-2, err
    assert np.isfinite(out.float().numpy()).all()


def test_batched_modulations_bit_exact(hn, cuda):
    """SyntheticDiT stacks every block's [6D, D] modulation weights and runs one quantize + GEMM per step for all
    blocks (they share vec, model.py:247): each block's slice equals its own linear bit for bit, and the
    whole multi-block forward (which uses the batched path) equals the block-by-block chain."""
    from hy_nomas_b200.dit import DiTConfig, SyntheticDiT, block_forward
    cfg = DiTConfig(hidden=256, heads=2, mlp_ratio=4, blocks=3, grid=(1, 4, 10))
    model = SyntheticDiT(cfg, device=cuda, seed=3)
    g = torch.Generator().manual_seed(4)
    x = torch.randn(1, cfg.tokens, cfg.hidden, generator=g).to(torch.bfloat16).to(cuda)
    vec = torch.randn(1, cfg.hidden, generator=g).to(torch.bfloat16).to(cuda)
    mods = model.modulations(vec)
    n6 = 6 * cfg.hidden
    assert mods.shape == (1, cfg.blocks * n6)
    y = x
    for i, w in enumerate(model.blocks):
        own = model.ops.linear(model.ops.silu(vec), w.mod)
        assert same(mods[:, i * n6:(i + 1) * n6], own)
        y = block_forward(cfg, w, y, vec, model.rope, model.sp)
    assert same(model(x, vec), y)
    torch.cuda.synchronize()


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def run_two_ranks(tmp_path, head_chunks=1, exchange="ce", history_tokens=0, pieces=True, split="tokens"):
    ctx = mp.get_context("spawn")
    port = free_port()
    out_path = os.path.join(tmp_path, f"sp_{exchange}_{head_chunks}_{history_tokens}_{int(pieces)}_{split}.pt")
    procs = [ctx.Process(target=sp_worker.nccl_rank, args=(r, 2, port, out_path, head_chunks, exchange,
                                                           history_tokens, pieces, split)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert codes == [0, 0], codes
    return torch.load(out_path)


@pytest.mark.parametrize("head_chunks,exchange", [(1, "ce"), (1, "nccl"), (2, "nccl")])
def test_sequence_parallel_two_gpus(hn, cuda, tmp_path, head_chunks, exchange):
    """2 ranks (K/V pushed by the copy engines, or all-gathered over NCCL whole or split by head) against the
    same model on one GPU, over two steps (the second reuses the double-buffered exchange buffers)."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from hy_nomas_b200.dit import CudaOps
    from hy_nomas_b200.sequence_parallel import SequenceParallel
    single = sp_worker.run_model(sp_worker.small_config(), SequenceParallel(), CudaOps, "cuda:0").cpu()
    res = run_two_ranks(tmp_path, head_chunks, exchange)
    assert res["exchange"] == exchange
    assert res["errors"] == [0, 0]
    first, second = res["outs"]
    assert first.shape == single.shape
    assert rel_l2(first.float().numpy(), single.float().numpy()) < 1e-2
    assert torch.equal(first.view(torch.int16), second.view(torch.int16))


def test_copy_engine_exchange_matches_nccl(hn, cuda, tmp_path):
    """The copy-engine exchange moves the same bytes as the all-gather: attending once after every slice arrived,
    the outputs are bit-identical to the NCCL run, with and without a 30-token int8 K/V history (its own
    double-buffered exchange buffers). Attending in pieces as the slices arrive (the default) agrees within the
    bf16 attention tolerance."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    whole = run_two_ranks(tmp_path, 1, "ce", history_tokens=30, pieces=False)
    nc = run_two_ranks(tmp_path, 1, "nccl", history_tokens=30)
    piecewise = run_two_ranks(tmp_path, 1, "ce", history_tokens=30, pieces=True)
    assert whole["exchange"] == "ce" and nc["exchange"] == "nccl" and piecewise["exchange"] == "ce"
    assert whole["errors"] == [0, 0] and nc["errors"] == [0, 0] and piecewise["errors"] == [0, 0]
    for a, b, c in zip(whole["outs"], nc["outs"], piecewise["outs"]):
        assert torch.equal(a.view(torch.int16), b.view(torch.int16))
        assert rel_l2(c.float().numpy(), b.float().numpy()) < 1e-2
    assert not torch.equal(whole["outs"][0], whole["outs"][2])      # the history changed the output


def test_head_split_two_gpus(hn, cuda, tmp_path):
    """Head-parallel attention on 2 GPUs: each rank attends for one head over all tokens, Q/K/V and the output
    exchanged by strided copy-engine pushes or by NCCL all-to-all; two steps, then one over a 30-token int8
    history. Both exchanges move the same rows into the same buffers, so their outputs are bit-identical; against
    the same model on one GPU (both heads in one attention call) within the bf16 attention tolerance."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from hy_nomas_b200.dit import CudaOps
    from hy_nomas_b200.sequence_parallel import SequenceParallel
    cfg = sp_worker.small_config()
    single = sp_worker.run_model(cfg, SequenceParallel(), CudaOps, "cuda:0").cpu()
    single_h = sp_worker.run_model(cfg, SequenceParallel(), CudaOps, "cuda:0", history_tokens=30).cpu()
    ce = run_two_ranks(tmp_path, 1, "ce", history_tokens=30, pieces=False, split="heads")
    nc = run_two_ranks(tmp_path, 1, "nccl", history_tokens=30, pieces=False, split="heads")
    assert ce["exchange"] == "heads-ce" and nc["exchange"] == "heads-collective"
    assert ce["errors"] == [0, 0] and nc["errors"] == [0, 0]
    for a, b in zip(ce["outs"], nc["outs"]):
        assert torch.equal(a.view(torch.int16), b.view(torch.int16))
    first, second, hist = ce["outs"]
    assert torch.equal(first.view(torch.int16), second.view(torch.int16))
    assert rel_l2(first.float().numpy(), single.float().numpy()) < 1e-2
    assert rel_l2(hist.float().numpy(), single_h.float().numpy()) < 1e-2
    assert not torch.equal(first, hist)


@pytest.fixture(scope="module")
def history_run(hn, oracle, cuda):
    """One block over 200 current tokens with a 120-token int8 K/V history (the segment-2 layout: earlier frames
    as int8 cache, hy_nomas/model.py:199-209), on the GPU, with its trace and the cache it captures."""
    from hy_nomas_b200.dit import block_forward, make_block_weights, rope_freqs
    from hy_nomas_b200.sequence_parallel import SequenceParallel
    cfg = small_cfg()
    gen = torch.Generator(device=cuda).manual_seed(9)
    w = make_block_weights(cfg, gen, cuda)
    rope = rope_freqs(cfg.rope_dims, cfg.theta, *cfg.grid, t_offset=3, device=cuda)
    g = torch.Generator().manual_seed(10)
    x = torch.randn(1, cfg.tokens, cfg.hidden, generator=g).to(torch.bfloat16).to(cuda)
    vec = torch.randn(1, cfg.hidden, generator=g).to(torch.bfloat16).to(cuda)
    hist = sp_worker.history(cfg.__class__(**{**cfg.__dict__, "blocks": 1}), 120, cuda)[0]
    trace, cap = {}, []
    out = block_forward(cfg, w, x, vec, rope, SequenceParallel(), trace=trace, history=hist, capture=cap)
    torch.cuda.synchronize()
    rc, code = hn.lib.device_error()
    assert rc == 0 and code == 0
    cpu = lambda t: t.cpu() if torch.is_tensor(t) else t  # noqa: E731
    return (cfg, to_cpu_weights(w), x.cpu(), vec.cpu(), (rope[0].cpu(), rope[1].cpu()),
            tuple(cpu(t) for t in hist), {k: cpu(v) for k, v in trace.items()}, out.cpu(), [tuple(map(cpu, c)) for c in cap])


def test_history_dequantized_into_the_kv_prefix(history_run):
    """The history's K and V, dequantized by the int8-KV kernel straight into the first 120 positions of the K/V
    buffers, equal the oracle's dequantize_kv (world.py:93-94) bit for bit; the current tokens follow."""
    cfg, w, x, vec, rope, hist, t, out, cap = history_run
    hk_q, hk_s, hv_q, hv_s = hist
    lh = hk_q.shape[0]
    assert t["k_full"].shape[1] == lh + cfg.tokens
    ref_k = OracleOps.dequantize_kv(hk_q, hk_s, torch.empty(lh, cfg.heads, cfg.head_dim, dtype=torch.bfloat16))
    ref_v = OracleOps.dequantize_kv(hv_q, hv_s, torch.empty(lh, cfg.heads, cfg.head_dim, dtype=torch.bfloat16))
    assert same(t["k_full"][0, :lh], ref_k) and same(t["v_full"][0, :lh], ref_v)


def test_history_attention_and_block_within_tolerance(history_run):
    from hy_nomas_b200.dit import block_forward
    from hy_nomas_b200.sequence_parallel import SequenceParallel
    cfg, w, x, vec, rope, hist, t, out, cap = history_run
    b, l, d = x.shape
    ref = OracleOps.attention(t["q"], t["k_full"], t["v_full"]).reshape(b * l, d)
    assert rel_l2(t["attn"].float().numpy(), ref.float().numpy()) < 1e-2
    full = block_forward(cfg, w, x, vec, rope, SequenceParallel(), ops=OracleOps, history=hist)
    assert rel_l2(out.float().numpy(), full.float().numpy()) < 2e-2


def test_capture_equals_kv_quantizer_on_gpu(history_run):
    """The cache pass on the GPU: the K codes and scales come out of the QK-norm + RoPE kernel (fused quantizer)
    and V's from the KV quantizer, equal to the oracle's world.quantize_kv of the block's own K and V."""
    cfg, w, x, vec, rope, hist, t, out, cap = history_run
    kq, ks, vq, vs = cap[0]
    lh, l, h, d = hist[0].shape[0], cfg.tokens, cfg.heads, cfg.head_dim
    k_ref = OracleOps.quantize_kv(t["k_full"][0, lh:].reshape(l, h, d))
    v_ref = OracleOps.quantize_kv(t["v_full"][0, lh:].reshape(l, h, d))
    assert torch.equal(kq, k_ref[0]) and torch.equal(ks.reshape(l, h, 1), k_ref[1])
    assert torch.equal(vq, v_ref[0]) and torch.equal(vs.reshape(l, h, 1), v_ref[1])
