"""Worker processes for the sequence-parallel tests (importable by spawned children)."""
import os

import torch


def small_config(heads=2):
    from hy_nomas_b200.dit import DiTConfig
    # `heads` x 128 (hidden 256 by default), 2 blocks, a 2 x 3 x 4 grid = 24 tokens (splits over 1, 2, 4 ranks)
    return DiTConfig(hidden=128 * heads, heads=heads, mlp_ratio=4, blocks=2, grid=(2, 3, 4))


def inputs(cfg, device="cpu"):
    gen = torch.Generator().manual_seed(11)
    x = torch.randn(1, cfg.tokens, cfg.hidden, generator=gen).to(torch.bfloat16)
    vec = torch.randn(1, cfg.hidden, generator=gen).to(torch.bfloat16)
    return x.to(device), vec.to(device)


def history(cfg, tokens, device="cpu"):
    """A seeded int8 K/V history of `tokens` earlier tokens for every block: codes in [-127, 127] and scales
    (the same on every rank, as a world's staged history is)."""
    gen = torch.Generator().manual_seed(21)
    h, d = cfg.heads, cfg.head_dim
    caches = []
    for _ in range(cfg.blocks):
        part = []
        for _kv in range(2):
            part.append(torch.randint(-127, 128, (tokens, h, d), generator=gen, dtype=torch.int8).to(device))
            part.append((torch.rand(tokens, h, 1, generator=gen) * 0.04 + 0.01).to(device))
        caches.append(tuple(part))
    return caches


def run_model(cfg, sp, ops, device, history_tokens=0):
    from hy_nomas_b200.dit import SyntheticDiT
    model = SyntheticDiT(cfg, device=device, seed=3, sp=sp, ops=ops)
    x, vec = inputs(cfg, device)
    lo, hi = model.token_range
    hist = history(cfg, history_tokens, device) if history_tokens else None
    return model(x[:, lo:hi].contiguous(), vec, history=hist)


def gloo_rank(rank, world, port, out_path, head_chunks=1, history_tokens=0, split="tokens", heads=2):
    import torch.distributed as dist
    from dit_oracle_ops import OracleOps
    from hy_nomas_b200.sequence_parallel import SequenceParallel
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = small_config(heads)
        sp = SequenceParallel(head_chunks=head_chunks, split=split)
        if sp.split_name(cfg.heads) != ("heads-collective" if split == "heads" else "tokens-nccl"):
            raise AssertionError(f"unexpected attention split {sp.split_name(cfg.heads)}")
        out = run_model(cfg, sp, OracleOps, "cpu", history_tokens)
        parts = [torch.empty_like(out) for _ in range(world)]
        dist.all_gather(parts, out)
        if rank == 0:
            torch.save(torch.cat(parts, dim=1), out_path)
    finally:
        dist.destroy_process_group()


def nccl_rank(rank, world, port, out_path, head_chunks=1, exchange="ce", history_tokens=0, pieces=True,
              split="tokens", heads=2):
    """One rank of a sequence-parallel run on GPU `rank`: two steps (the second reuses the double-buffered K/V
    exchange buffers) and, with `history_tokens`, a third step over an int8 K/V history. Rank 0 saves every
    step's gathered output, the exchange used and the ranks' device error words."""
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    os.environ["HN_SP_EXCHANGE"] = exchange
    os.environ["HN_SP_ATTENTION_PIECES"] = "1" if pieces else "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                            timeout=datetime.timedelta(seconds=60))
    try:
        from hy_nomas_b200 import _lib
        from hy_nomas_b200.dit import CudaOps, SyntheticDiT
        from hy_nomas_b200.sequence_parallel import SequenceParallel
        cfg = small_config(heads)
        device = f"cuda:{rank}"
        sp = SequenceParallel(head_chunks=head_chunks, split=split)
        model = SyntheticDiT(cfg, device=device, seed=3, sp=sp, ops=CudaOps)
        x, vec = inputs(cfg, device)
        lo, hi = model.token_range
        xs = x[:, lo:hi].contiguous()
        outs = [model(xs, vec), model(xs, vec)]
        if history_tokens:
            outs.append(model(xs, vec, history=history(cfg, history_tokens, device)))
        torch.cuda.synchronize()
        err = torch.tensor([_lib.device_error(torch.cuda.current_stream())[1]], device=device)
        errs = [torch.empty_like(err) for _ in range(world)]
        dist.all_gather(errs, err)
        gathered = []
        for out in outs:
            parts = [torch.empty_like(out) for _ in range(world)]
            dist.all_gather(parts, out)
            gathered.append(torch.cat(parts, dim=1).cpu())
        torch.cuda.synchronize()
        kind = sp.split_name(cfg.heads) if split == "heads" else sp.exchange
        sp.close()
        if rank == 0:
            torch.save({"outs": gathered, "exchange": kind, "errors": [int(e.item()) for e in errs]}, out_path)
    finally:
        dist.destroy_process_group()


def fallback_rank(rank, world, port, out_path, failing_rank):
    """A copy-engine exchange whose set-up fails on `failing_rank` only (its mapping raises, as it would for
    memory with no IPC handle): every rank must come out without it (NCCL all-gather instead), none may wait
    for the others in a collective they never enter. Host logic only, on gloo."""
    import torch.distributed as dist
    from hy_nomas_b200 import sequence_parallel as S
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        unmapped = []

        class Failing(S.PeerExchange):
            """The real class with set-up replaced: mapping fails on `failing_rank`; close() stays the real,
            collective one, so a fallback that called it on the other ranks would hang this test."""
            def __init__(self, sp):
                if sp.rank == failing_rank:
                    raise RuntimeError("hn_ipc_export failed (no legacy IPC handle)")

            def _unmap(self):
                unmapped.append(True)

        sp = S.SequenceParallel(local=False)
        import warnings
        with warnings.catch_warnings(record=True) as caught:
            warnings.simplefilter("always")
            exch = Failing.create(sp)
        ok = torch.tensor([1 if exch is None else 0, len(caught), len(unmapped)])
        parts = [torch.zeros_like(ok) for _ in range(world)]
        dist.all_gather(parts, ok)
        if rank == 0:
            torch.save(torch.stack(parts), out_path)
    finally:
        dist.destroy_process_group()
