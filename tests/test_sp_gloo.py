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


def _run_gloo(tmp_path, world, **kw):
    ctx = mp.get_context("spawn")
    port = free_port()
    out_path = os.path.join(tmp_path, "out.pt")
    args = dict(head_chunks=1, history_tokens=0, split="tokens", heads=2)
    args.update(kw)
    procs = [ctx.Process(target=sp_worker.gloo_rank, args=(r, world, port, out_path, args["head_chunks"],
                                                           args["history_tokens"], args["split"], args["heads"]))
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
    return torch.load(out_path)


@pytest.mark.parametrize("world,heads,history_tokens", [(2, 2, 0), (4, 4, 0), (2, 2, 12), (4, 4, 12)])
def test_gloo_head_split_matches_single_rank(hn, oracle, tmp_path, world, heads, history_tokens):
    """Head-parallel attention (every rank attends for heads / world heads over all tokens; Q, K, V and the output
    exchanged by all-to-all), with and without an int8 history, equals the single-rank model bit for bit."""
    from hy_nomas_b200.sequence_parallel import SequenceParallel
    single = sp_worker.run_model(sp_worker.small_config(heads), SequenceParallel(), OracleOps, "cpu",
                                 history_tokens=history_tokens)
    got = _run_gloo(tmp_path, world, split="heads", heads=heads, history_tokens=history_tokens)
    assert got.shape == single.shape
    assert torch.equal(got.view(torch.int16), single.view(torch.int16))


def test_head_split_selection():
    """"auto" takes the head split from HEADS_MIN_WORLD ranks on; never when the heads do not divide over the
    ranks, or with head chunks."""
    from hy_nomas_b200 import sequence_parallel as S
    sp = S.SequenceParallel(split="auto")
    assert not sp.head_split(32)                  # one rank
    for world in (2, 4, 8):
        sp.world = world
        assert sp.head_split(32) == (world >= S.HEADS_MIN_WORLD)
    sp.world = 8
    assert not sp.head_split(12)                  # 12 heads do not split over 8 ranks
    sp.split = "tokens"
    assert not sp.head_split(32)
    sp.split, sp.world = "heads", 2
    assert sp.head_split(32)
    sp.head_chunks = 2
    assert not sp.head_split(32)
    with pytest.raises(ValueError):
        S.SequenceParallel(split="rows")


def test_head_layout_offsets():
    """The head-parallel buffers: per set K, V (history + all tokens), Q (all tokens) and the output (own tokens,
    all heads), each starting on a 256-byte boundary for bf16, in that order and without overlap."""
    from hy_nomas_b200.sequence_parallel import _HeadLayout
    lay = _HeadLayout(world=8, local=2530, heads=32, head_dim=128, prefix=15840)
    assert lay.hpg == 4 and lay.tokens == 20240
    ends = 0
    for kind in ("k", "v", "q", "o"):
        assert lay.offs[kind] == ends and (lay.offs[kind] * 2) % 256 == 0
        ends += lay.sizes[kind]
    assert ends == lay.numel
    flat = torch.arange(lay.numel, dtype=torch.float32)
    q, k, v, o = lay.views(flat)
    assert q.shape == (1, 20240, 4, 128) and k.shape == v.shape == (1, 15840 + 20240, 4, 128)
    assert o.shape == (1, 2530, 32, 128)
    assert lay.row0("k", 3) == 15840 + 3 * 2530 and lay.row0("q", 3) == 3 * 2530


@pytest.mark.parametrize("world,prefix", [(2, 0), (4, 7), (8, 0), (8, 15)])
def test_head_push_plan_tiles_every_buffer(world, prefix):
    """The head exchange's strided copies, checked byte by byte on the host before any of them runs on a GPU:
    each reads inside its source tensor, writes inside the peer's set of its parity, and on every destination
    rank the copies of all ranks (the rank's own one included, which it makes locally) cover each buffer's token
    part exactly once, leaving the history prefix and the other parity untouched."""
    import numpy as np
    from hy_nomas_b200.sequence_parallel import HEAD_KINDS, _HeadLayout
    local, heads, hd, esz = 3, 2 * world, 4, 2
    lay = _HeadLayout(world, local, heads, hd, prefix)
    src_bytes = {"k": local * heads * hd * esz, "o": lay.tokens * lay.hpg * hd * esz}
    for par in (0, 1):
        for dst in range(world):
            cover = np.zeros(2 * lay.numel * esz, dtype=np.int32)
            for kind in HEAD_KINDS:
                for r in range(world):
                    soff, spitch, doff, dpitch, width, height = lay.push_plan(kind, r, dst, par, esz)
                    assert width <= spitch and width <= dpitch
                    assert soff + (height - 1) * spitch + width <= src_bytes["o" if kind == "o" else "k"]
                    for row in range(height):
                        cover[doff + row * dpitch:doff + row * dpitch + width] += 1
            sets = cover.reshape(2, lay.numel * esz)
            assert (sets[1 - par] == 0).all()
            mine = sets[par]
            for kind in HEAD_KINDS:
                lo, n = lay.offs[kind] * esz, lay.sizes[kind] * esz
                skip = prefix * lay.hpg * hd * esz if kind in ("k", "v") else 0
                assert (mine[lo:lo + skip] == 0).all()              # the history prefix is the rank's own
                assert (mine[lo + skip:lo + n] == 1).all()


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
