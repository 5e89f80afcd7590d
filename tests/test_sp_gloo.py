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
