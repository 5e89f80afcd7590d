"""Sequence parallelism for the DiT step: each rank owns a contiguous token range, weights are replicated, and
the only exchange is an all-gather of every block's K and V (after QK-norm + RoPE) so each rank's queries
attend over the whole sequence.

The reference runs one GPU (`sp_size: 1`, docs/upstream/single_gpu_low_mem_inference.yaml:22-23); this module
is the B200 build's partition of the same block: every per-token op (LayerNorm, quantizers, the linears,
QK-norm, the residuals) runs on the rank's own rows with no communication, and attention reads the gathered
K/V. The gathers are issued asynchronously (NCCL on its own stream, or gloo on CPU for host-side tests), so
K's gather overlaps the V projection.

Rank r owns tokens [r * L / P, (r + 1) * L / P); L must divide evenly (20240 does for P = 1, 2, 4, 8).
The gather buffers are rank-major, so with batch 1 a rank's K/V rows are one contiguous slice that its own
kernels write in place and that the all-gather uses as its input.
"""
import os

import torch
import torch.distributed as dist

# K/V head chunks per block under sequence parallelism (HN_SP_HEAD_CHUNKS overrides)
HEAD_CHUNKS = 1


class SequenceParallel:
    """`head_chunks` > 1 splits each block's K/V gathers and attention by heads, so that a chunk's attention runs
    while the next chunk's K is still being gathered (every head's arithmetic is unchanged). `local=True` is a
    partition of one rank even inside a process group: the whole sequence on this process, no exchange."""

    def __init__(self, group=None, head_chunks=None, local=False):
        self.group = group
        if local:
            self.world, self.rank = 1, 0
        elif dist.is_available() and dist.is_initialized():
            self.world = dist.get_world_size(group)
            self.rank = dist.get_rank(group)
        else:
            self.world, self.rank = 1, 0
        if head_chunks is None:
            head_chunks = int(os.environ.get("HN_SP_HEAD_CHUNKS", str(HEAD_CHUNKS)))
        if head_chunks < 1:
            raise ValueError(f"head_chunks must be >= 1, got {head_chunks}")
        self.head_chunks = head_chunks
        self._bufs = {}

    def shard(self, length):
        """(start, stop) of this rank's tokens in a sequence of `length`."""
        if length % self.world:
            raise ValueError(f"sequence length {length} does not split evenly over {self.world} ranks")
        per = length // self.world
        return self.rank * per, (self.rank + 1) * per

    def kv_buffers(self, batch, local, heads, head_dim, dtype, device, prefix=0):
        """Full-sequence K and V buffers [batch, prefix + local * world, heads, head_dim] and this rank's slice of
        each ([batch, local, heads, head_dim], contiguous, at prefix + rank * local). The first `prefix` tokens
        hold the segment history's keys and values (replicated on every rank). Reused across blocks and steps."""
        if self.world > 1 and batch != 1:
            raise ValueError("sequence parallelism takes batch 1 (the denoise step's layout)")
        key = (batch, local, heads, head_dim, dtype, str(device), prefix)
        if key not in self._bufs:
            self._bufs[key] = self._alloc(batch, local, heads, head_dim, dtype, device, prefix)
        return self._bufs[key]

    def kv_chunk_buffers(self, batch, local, heads, head_dim, chunks, dtype, device):
        """`kv_buffers` per head chunk: a list of `chunks` (k_full, v_full, k_mine, v_mine) tuples, each over
        heads // chunks heads, so that every chunk's gather has contiguous rank slices."""
        if self.world > 1 and batch != 1:
            raise ValueError("sequence parallelism takes batch 1 (the denoise step's layout)")
        key = ("chunks", chunks, batch, local, heads, head_dim, dtype, str(device))
        if key not in self._bufs:
            self._bufs[key] = [self._alloc(batch, local, heads // chunks, head_dim, dtype, device) for _ in range(chunks)]
        return self._bufs[key]

    def _alloc(self, batch, local, heads, head_dim, dtype, device, prefix=0):
        total = prefix + local * self.world
        k_full = torch.empty((batch, total, heads, head_dim), dtype=dtype, device=device)
        v_full = torch.empty_like(k_full)
        lo = prefix + self.rank * local
        return k_full, v_full, k_full[:, lo:lo + local], v_full[:, lo:lo + local]

    def all_gather_async(self, full, mine):
        """Start filling `full`'s ranks' part (everything after its history prefix) with every rank's `mine` (a
        slice of `full`); returns a handle for `wait`."""
        if self.world == 1:
            return None
        prefix = full.shape[1] - mine.shape[1] * self.world
        ranks_part = full[:, prefix:]
        # flat views: the rank-major part is `world` equal chunks of the rank slices (NCCL and gloo agree); with
        # batch 1 it is one contiguous range
        return dist.all_gather_into_tensor(ranks_part.view(-1), mine.view(-1), group=self.group, async_op=True)

    @staticmethod
    def wait(*handles):
        """Make the current stream wait for the gathers (device-side; the host does not block)."""
        for h in handles:
            if h is not None:
                h.wait()
