"""Sequence-parallel DiT step on CPU ranks (gloo): the token shards, the in-place K/V all-gathers and the
block orchestration of hy_nomas_b200.dit, run with the oracle's ops, must give exactly the single-rank
result for 2 and 4 ranks."""
import multiprocessing as mp
import os
import socket

import pytest
import torch

import sp_worker
from dit_oracle_ops import OracleOps


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.fixture(scope="module")
def single_rank(hn, oracle):
    from hy_nomas_b200.sequence_parallel import SequenceParallel
    return sp_worker.run_model(sp_worker.small_config(), SequenceParallel(), OracleOps, "cpu")


def test_shard_ranges():
    from hy_nomas_b200.sequence_parallel import SequenceParallel
    sp = SequenceParallel()
    assert sp.shard(20240) == (0, 20240)
    for world in (2, 4, 8):
        sp.world = world
        spans = []
        for r in range(world):
            sp.rank = r
            spans.append(sp.shard(20240))
        assert spans[0][0] == 0 and spans[-1][1] == 20240
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
        assert len({hi - lo for lo, hi in spans}) == 1
    sp.world, sp.rank = 3, 0
    with pytest.raises(ValueError):
        sp.shard(20240)


@pytest.mark.parametrize("world,head_chunks", [(2, 1), (4, 1), (2, 2)])
def test_gloo_matches_single_rank(single_rank, tmp_path, world, head_chunks):
    """2 and 4 gloo ranks, and 2 ranks with the K/V gathers split by head, equal the single-rank model."""
    ctx = mp.get_context("spawn")
    port = free_port()
    out_path = os.path.join(tmp_path, "out.pt")
    procs = [ctx.Process(target=sp_worker.gloo_rank, args=(r, world, port, out_path, head_chunks))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert codes == [0] * world, codes
    got = torch.load(out_path)
    assert got.shape == single_rank.shape
    assert torch.equal(got.view(torch.int16), single_rank.view(torch.int16))


def test_gloo_with_history_matches_single_rank(hn, oracle, tmp_path):
    """With a replicated int8 K/V history (every block's attention runs over the dequantized history followed by
    the gathered current tokens), 2 gloo ranks equal the single-rank model bit for bit."""
    from hy_nomas_b200.sequence_parallel import SequenceParallel
    single = sp_worker.run_model(sp_worker.small_config(), SequenceParallel(), OracleOps, "cpu", history_tokens=12)
    ctx = mp.get_context("spawn")
    port = free_port()
    out_path = os.path.join(tmp_path, "out.pt")
    procs = [ctx.Process(target=sp_worker.gloo_rank, args=(r, 2, port, out_path, 1, 12)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert codes == [0, 0], codes
    got = torch.load(out_path)
    assert torch.equal(got.view(torch.int16), single.view(torch.int16))
    no_hist = sp_worker.run_model(sp_worker.small_config(), SequenceParallel(), OracleOps, "cpu")
    assert not torch.equal(no_hist.view(torch.int16), single.view(torch.int16))   # the history is attended to


def test_capture_is_the_kv_quantizer_of_the_block_kv(hn, oracle):
    """The cache pass: each block's captured (kq, ks, vq, vs) equals world.quantize_kv of the K and V the block
    attended with (K after QK-norm + RoPE)."""
    from hy_nomas_b200.dit import block_forward, make_block_weights, rope_freqs
    from hy_nomas_b200.sequence_parallel import SequenceParallel
    cfg = sp_worker.small_config()
    w = make_block_weights(cfg, torch.Generator().manual_seed(8), "cpu")
    x, vec = sp_worker.inputs(cfg)
    rope = rope_freqs(cfg.rope_dims, cfg.theta, *cfg.grid)
    trace, cap = {}, []
    block_forward(cfg, w, x, vec, rope, SequenceParallel(), ops=OracleOps, trace=trace, capture=cap)
    kq, ks, vq, vs = cap[0]
    l, h, d = cfg.tokens, cfg.heads, cfg.head_dim
    k_ref = OracleOps.quantize_kv(trace["k_full"].reshape(l, h, d))
    v_ref = OracleOps.quantize_kv(trace["v_full"].reshape(l, h, d))
    assert torch.equal(kq, k_ref[0]) and torch.equal(ks, k_ref[1])
    assert torch.equal(vq, v_ref[0]) and torch.equal(vs, v_ref[1])


@pytest.mark.parametrize("failing_rank", [0, 1])
def test_copy_engine_setup_failure_falls_back_on_every_rank(tmp_path, failing_rank):
    """If one rank cannot map its peers' memory, the copy-engine exchange is abandoned on every rank (each gets
    None and a warning) - no rank is left waiting in a collective the others skipped."""
    ctx = mp.get_context("spawn")
    port = free_port()
    out_path = os.path.join(tmp_path, "fallback.pt")
    procs = [ctx.Process(target=sp_worker.fallback_rank, args=(r, 2, port, out_path, failing_rank)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert codes == [0, 0], codes
    got = torch.load(out_path)
    assert got[:, 0].tolist() == [1, 1]        # no exchange on either rank
    assert got[:, 1].tolist() == [1, 1]        # each rank warned once
    # the rank whose set-up succeeded released its mappings locally; the failing rank had none
    assert got[:, 2].tolist() == [0 if r == failing_rank else 1 for r in range(2)]
