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


@pytest.mark.parametrize("head_chunks", [1, 2])
def test_sequence_parallel_two_gpus(hn, cuda, tmp_path, head_chunks):
    """2 ranks over NCCL (K/V all-gathered, whole or split by head) against the same model on one GPU."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from hy_nomas_b200.dit import CudaOps
    from hy_nomas_b200.sequence_parallel import SequenceParallel
    single = sp_worker.run_model(sp_worker.small_config(), SequenceParallel(), CudaOps, "cuda:0").cpu()
    ctx = mp.get_context("spawn")
    port = free_port()
    out_path = os.path.join(tmp_path, "sp.pt")
    procs = [ctx.Process(target=sp_worker.nccl_rank, args=(r, 2, port, out_path, head_chunks)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert codes == [0, 0], codes
    got = torch.load(out_path)
    assert got.shape == single.shape
    assert rel_l2(got.float().numpy(), single.float().numpy()) < 1e-2
