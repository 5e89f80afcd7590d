"""Sequence parallelism for the DiT step: each rank owns a contiguous token range, weights are replicated, and
the only exchange is an all-gather of every block's K and V (after QK-norm + RoPE) so each rank's queries
attend over the whole sequence.

The reference runs one GPU (`sp_size: 1`, docs/upstream/single_gpu_low_mem_inference.yaml:22-23); this module
is the B200 build's partition of the same block: every per-token op (LayerNorm, quantizers, the linears,
QK-norm, the residuals) runs on the rank's own rows with no communication, and attention reads the gathered
K/V. Two exchanges implement the gather:

- the copy-engine exchange (GPUs, the default): every rank maps its peers' K/V buffers (CUDA IPC) and, as soon as
  its own K (then V) slice exists, the copy engines push it into every peer's buffer over NVLink and write a
  block counter into the peer's flag array. No SM is involved, so the pushes run under the V and Q projections
  at full GEMM speed; a one-warp bounded wait for the peers' counters precedes attention. The buffers are double
  buffered by block parity, and a rank's push into a peer's buffer of parity p is ordered after that peer's
  attention of the previous parity-p block (the push follows this rank's wait for the peer's previous counters,
  which the peer wrote after that attention), so no further handshake is needed.
- an NCCL all-gather (or gloo on CPU for host-side tests), issued asynchronously on the library's stream:
  used for head-chunked exchanges, when HN_SP_EXCHANGE=nccl, or when the IPC mappings cannot be made.

Rank r owns tokens [r * L / P, (r + 1) * L / P); L must divide evenly (20240 does for P = 1, 2, 4, 8).
The gather buffers are rank-major, so with batch 1 a rank's K/V rows are one contiguous slice that its own
kernels write in place and that the all-gather uses as its input.
"""
import ctypes
import os
import warnings

import torch
import torch.distributed as dist

# K/V head chunks per block under sequence parallelism (HN_SP_HEAD_CHUNKS overrides)
HEAD_CHUNKS = 1
# limit of the wait for the peers' K/V (HN_SP_WAIT_TIMEOUT_S overrides); past it the stream's error word reads
# HN_ERR_TIMEOUT and attention runs on what arrived
WAIT_TIMEOUT_S = 120.0
# copy streams per kind (K, V) for the pushes, the pushes to the peers spread over them (HN_SP_PUSH_STREAMS
# overrides; capped at world - 1). One per kind: seven per kind measured the same at 8 GPUs (98.8 against 97.9 ms)
PUSH_STREAMS = 1


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
        self.peer = None
        want = os.environ.get("HN_SP_EXCHANGE", "ce")
        if want not in ("ce", "nccl"):
            raise ValueError(f"HN_SP_EXCHANGE must be 'ce' or 'nccl', got {want!r}")
        if (self.world > 1 and want == "ce" and head_chunks == 1 and torch.cuda.is_available()
                and dist.get_backend(group) == "nccl"):
            self.peer = PeerExchange.create(self)

    @property
    def exchange(self):
        """'ce' (copy-engine pushes), 'nccl' (all-gather) or 'none' (one rank)."""
        if self.world == 1:
            return "none"
        return "ce" if self.peer is not None else "nccl"

    def close(self):
        """Unmap the peers' buffers (collective: every rank calls it, after its last step)."""
        if self.peer is not None:
            self.peer.close()
            self.peer = None

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


def _ranks_agree(ok, group):
    flags = [None] * dist.get_world_size(group)
    dist.all_gather_object(flags, bool(ok), group=group)
    return all(flags)


class PeerExchange:
    """The copy-engine K/V exchange of one `SequenceParallel` (its rank's GPU, the current device at creation).

    Per buffer shape one allocation holds [parity 2][K, V][batch 1][prefix + local * world][heads][head_dim]; the
    flags are int32 [K, V][world]: flags[kind][src] = the last block counter whose `kind` slice `src` pushed here.
    Every rank runs the same blocks in the same order, so the counters (`epoch`, +1 per block) agree."""

    def __init__(self, sp):
        from . import _lib
        self._lib = _lib
        self.sp = sp
        self.world, self.rank, self.group = sp.world, sp.rank, sp.group
        self.device = torch.device("cuda", torch.cuda.current_device())
        self.timeout_us = int(float(os.environ.get("HN_SP_WAIT_TIMEOUT_S", str(WAIT_TIMEOUT_S))) * 1e6)
        self.epoch = 0
        self._maps = {}                     # (peer, handle) -> mapped base address
        self._bufs = {}
        nstreams = max(1, min(self.world - 1, int(os.environ.get("HN_SP_PUSH_STREAMS", str(PUSH_STREAMS)))))
        self.side = [[torch.cuda.Stream(self.device) for _ in range(nstreams)] for _kind in range(2)]
        self.flags = torch.zeros(2 * self.world, dtype=torch.int32, device=self.device)
        # the zeros are written before this rank's contribution to the address exchange, which every peer
        # receives before it can push
        self.peer_flags = self._share(self.flags)

    @classmethod
    def create(cls, sp):
        """A PeerExchange, or None (on every rank alike) when some rank cannot map its peers' memory."""
        exch, err = None, None
        try:
            exch = cls(sp)
        except (RuntimeError, OSError) as e:           # this rank failed; the others learn it below
            err = e
        if not _ranks_agree(err is None, sp.group):
            if exch is not None:
                exch._unmap()                      # local only: the failing rank enters no further collective
            warnings.warn(f"copy-engine K/V exchange unavailable ({err or 'a peer failed'}); using NCCL all-gather")
            return None
        return exch

    def _share(self, t):
        """Every rank's address of its `t` (collective), mapped into this process: a list indexed by rank."""
        lib = self._lib
        handle = (ctypes.c_uint8 * 64)()
        off = ctypes.c_int64()
        err = None
        try:
            lib.check(lib.lib.hn_ipc_export(ctypes.c_void_p(t.data_ptr()), handle, ctypes.byref(off)),
                      "hn_ipc_export", launches=0)
        except RuntimeError as e:
            err = e
        infos = [None] * self.world
        dist.all_gather_object(infos, None if err else (bytes(handle), off.value), group=self.group)
        if any(i is None for i in infos):
            raise RuntimeError(f"a rank could not export its K/V buffers ({err})")
        addrs = []
        for r, (h, o) in enumerate(infos):
            if r == self.rank:
                addrs.append(t.data_ptr())
                continue
            if (r, h) not in self._maps:
                base = ctypes.c_void_p()
                buf = (ctypes.c_uint8 * 64).from_buffer_copy(h)
                lib.check(lib.lib.hn_ipc_import(buf, ctypes.byref(base)), "hn_ipc_import", launches=0)
                self._maps[(r, h)] = base.value
            addrs.append(self._maps[(r, h)] + o)
        return addrs

    def _buffers(self, batch, local, heads, head_dim, dtype, prefix):
        key = (batch, local, heads, head_dim, dtype, prefix)
        ent = self._bufs.get(key)
        if ent is None:
            total = prefix + local * self.world
            mem = torch.empty((2, 2, batch, total, heads, head_dim), dtype=dtype, device=self.device)
            ok = True
            try:
                addrs = self._share(mem)
            except RuntimeError as e:
                ok, addrs = False, str(e)
            if not _ranks_agree(ok, self.group):
                raise RuntimeError(f"K/V buffer mapping failed: {addrs if not ok else 'on a peer'}")
            row = heads * head_dim * mem.element_size()
            ent = dict(mem=mem, addrs=addrs, total=total, prefix=prefix, local=local, row=row,
                       done=[[[], []], [[], []]])
            self._bufs[key] = ent
        return ent

    def begin(self, batch, local, heads, head_dim, dtype, prefix=0):
        """Start a block: (k_full, v_full, k_mine, v_mine) of this block's parity. The current stream waits until
        this rank's pushes of the previous block of that parity have read its slices."""
        if batch != 1:
            raise ValueError("sequence parallelism takes batch 1 (the denoise step's layout)")
        self.epoch = (self.epoch + 1) & 0xFFFFFFFF
        par = self.epoch & 1
        ent = self._buffers(batch, local, heads, head_dim, dtype, prefix)
        cur = torch.cuda.current_stream(self.device)
        for evs in ent["done"][par]:
            for ev in evs:
                cur.wait_event(ev)
        self._cur = (ent, par)
        k_full, v_full = ent["mem"][par, 0], ent["mem"][par, 1]
        lo = prefix + self.rank * local
        return k_full, v_full, k_full[:, lo:lo + local], v_full[:, lo:lo + local]

    def push(self, kind):
        """Push this rank's slice of K (kind 0) or V (kind 1) - complete on the current stream - to every peer,
        each followed by this block's counter in the peer's flags."""
        lib = self._lib.lib
        ent, par = self._cur
        cur = torch.cuda.current_stream(self.device)
        sides = self.side[kind]
        ready = torch.cuda.Event()
        ready.record(cur)
        for side in sides:
            side.wait_event(ready)
        nbytes = ent["local"] * ent["row"]
        region = ((par * 2 + kind) * ent["total"] + ent["prefix"] + self.rank * ent["local"]) * ent["row"]
        src = ctypes.c_void_p(ent["mem"].data_ptr() + region)
        for step in range(1, self.world):
            peer = (self.rank + step) % self.world     # staggered, so the ranks start on different peers
            st = ctypes.c_void_p(sides[(step - 1) % len(sides)].cuda_stream)
            dst = ctypes.c_void_p(ent["addrs"][peer] + region)
            flag = ctypes.c_void_p(self.peer_flags[peer] + 4 * (kind * self.world + self.rank))
            self._lib.check(lib.hn_peer_push(dst, src, nbytes, flag, self.epoch, st), "hn_peer_push", launches=0)
        evs = []
        for side in sides:
            ev = torch.cuda.Event()
            ev.record(side)
            evs.append(ev)
        ent["done"][par][kind] = evs

    def wait(self, peer=None):
        """The current stream waits (bounded) for every peer's K and V of this block, or for `peer`'s only."""
        lib = self._lib
        cur = torch.cuda.current_stream(self.device)
        base = self.flags.data_ptr() + (0 if peer is None else 4 * peer)
        count, skip = (self.world, self.rank) if peer is None else (1, -1)
        lib.check(lib.lib.hn_wait_flags(ctypes.c_void_p(base), 2, count, self.world, skip, self.epoch,
                                        self.timeout_us, ctypes.c_void_p(cur.cuda_stream)),
                  "hn_wait_flags")

    def arrival_order(self):
        """The peers in the order their slices reach this rank: every rank pushes to rank + 1 first, so this rank
        hears from rank - 1 first, then rank - 2, ..."""
        return [(self.rank - s) % self.world for s in range(1, self.world)]

    def _unmap(self):
        """Unmap the peers' memory this rank mapped (no collective; nothing may be pushed through it anymore)."""
        for base in self._maps.values():
            self._lib.lib.hn_ipc_close(ctypes.c_void_p(base))
        self._maps.clear()

    def close(self):
        """Unmap the peers' memory once every rank's pushes are complete (collective)."""
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        self._unmap()
        dist.barrier(group=self.group)
