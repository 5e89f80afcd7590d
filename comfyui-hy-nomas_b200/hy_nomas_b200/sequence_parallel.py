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

Attention can instead be split by heads (`split="heads"`, HN_SP_SPLIT; the default from HEADS_MIN_WORLD ranks
on): rank r attends for heads [r * H / P, (r + 1) * H / P) over all L tokens. Every rank sends each peer that
peer's head group of its own tokens' Q, K and V, and after attention returns to each peer the rows of the
peer's tokens of its own head group's output. A rank then receives 4 (P - 1) / P of its token slice's bytes
(Q, K, V in, the output back) instead of the 2 (P - 1) slices' K and V of the all-gather: 4x less at 8 ranks.
Per head the attention is the single-GPU one (all queries, all keys), so the result is unchanged. Two
exchanges implement it, like the gather: copy-engine pushes of strided rows (`HeadExchange`, GPUs) and
all-to-all collectives (`HeadCollective`, NCCL or gloo).
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
# attention split under sequence parallelism (HN_SP_SPLIT overrides): "tokens" (K/V gathered, every rank's own
# queries), "heads" (Q/K/V exchanged by head group, all queries of a head on one rank), or "auto": heads from
# HEADS_MIN_WORLD ranks on, where it moves less data (at 2 ranks both exchanges move the same bytes)
SPLIT = "auto"
HEADS_MIN_WORLD = 4
# copy streams per kind of the head exchange, the peers spread over them (HN_SP_HEAD_PUSH_STREAMS overrides; capped
# at world - 1): its per-peer copies are small (2.6 MB at 8 ranks) and latency-bound, so they go side by side
HEAD_PUSH_STREAMS = 7


class SequenceParallel:
    """`split` ("auto", "tokens", "heads"; HN_SP_SPLIT): how attention's inputs move (see the module docstring).
    `head_chunks` > 1 splits each block's K/V gathers and attention by heads, so that a chunk's attention runs
    while the next chunk's K is still being gathered (every head's arithmetic is unchanged; token split only).
    `local=True` is a partition of one rank even inside a process group: the whole sequence on this process, no
    exchange."""

    def __init__(self, group=None, head_chunks=None, local=False, split=None):
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
        if split is None:
            split = os.environ.get("HN_SP_SPLIT", SPLIT)
        if split not in ("auto", "tokens", "heads"):
            raise ValueError(f"split must be 'auto', 'tokens' or 'heads', got {split!r}")
        self.split = split
        self._heads = None
        if (self.world > 1 and want == "ce" and head_chunks == 1 and torch.cuda.is_available()
                and dist.get_backend(group) == "nccl"):
            self.peer = PeerExchange.create(self)

    @property
    def exchange(self):
        """'ce' (copy-engine pushes), 'nccl' (all-gather) or 'none' (one rank)."""
        if self.world == 1:
            return "none"
        return "ce" if self.peer is not None else "nccl"

    def head_split(self, heads):
        """Whether a model with `heads` attention heads attends head-parallel on this partition."""
        if self.world == 1 or self.head_chunks != 1 or heads % self.world:
            return False
        if self.split == "auto":
            return self.world >= HEADS_MIN_WORLD
        return self.split == "heads"

    def head_exchange(self):
        """The head-parallel exchange (made on first use; collective, so every rank asks at the same block):
        copy-engine pushes where the K/V exchange uses them, else all-to-all collectives."""
        if self._heads is None:
            ex = HeadExchange.create(self) if self.peer is not None else None
            self._heads = ex if ex is not None else HeadCollective(self)
        return self._heads

    def split_name(self, heads):
        """How a model with `heads` heads attends here: 'none' (one rank), 'tokens-ce' / 'tokens-nccl' (K/V
        gathered by copy engines / NCCL), 'heads-ce' / 'heads-collective' (head groups exchanged)."""
        if self.world == 1:
            return "none"
        if self.head_split(heads):
            ce = isinstance(self._heads, HeadExchange) or (self._heads is None and self.peer is not None)
            return "heads-ce" if ce else "heads-collective"
        return "tokens-" + self.exchange

    def close(self):
        """Unmap the peers' buffers (collective: every rank calls it, after its last step)."""
        if self._heads is not None:
            self._heads.close()
            self._heads = None
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


class _IpcExchange:
    """What the copy-engine exchanges share: this rank's GPU (the current device at creation), its peers' memory
    mapped by CUDA IPC, an int32 flag array per rank that the peers' pushes write block counters into, and the
    bounded wait on those flags. Every rank runs the same blocks in the same order, so the counters (`epoch`, +1
    per block) agree."""

    def _setup(self, sp, nflags):
        from . import _lib
        self._lib = _lib
        self.sp = sp
        self.world, self.rank, self.group = sp.world, sp.rank, sp.group
        self.device = torch.device("cuda", torch.cuda.current_device())
        self.timeout_us = int(float(os.environ.get("HN_SP_WAIT_TIMEOUT_S", str(WAIT_TIMEOUT_S))) * 1e6)
        self.epoch = 0
        self._maps = {}                     # (peer, handle) -> mapped base address
        self._bufs = {}
        self.flags = torch.zeros(nflags, dtype=torch.int32, device=self.device)
        # the zeros are written before this rank's contribution to the address exchange, which every peer
        # receives before it can push
        self.peer_flags = self._share(self.flags)

    @classmethod
    def create(cls, sp):
        """An exchange, or None (on every rank alike) when some rank cannot map its peers' memory."""
        exch, err = None, None
        try:
            exch = cls(sp)
        except (RuntimeError, OSError) as e:           # this rank failed; the others learn it below
            err = e
        if not _ranks_agree(err is None, sp.group):
            if exch is not None:
                exch._unmap()                      # local only: the failing rank enters no further collective
            warnings.warn(f"copy-engine exchange {cls.__name__} unavailable ({err or 'a peer failed'}); "
                          "using NCCL collectives")
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

    def _shared_alloc(self, numel, dtype):
        """One allocation of `numel` elements and every rank's address of its own (collective)."""
        mem = torch.empty(numel, dtype=dtype, device=self.device)
        ok = True
        try:
            addrs = self._share(mem)
        except RuntimeError as e:
            ok, addrs = False, str(e)
        if not _ranks_agree(ok, self.group):
            raise RuntimeError(f"exchange buffer mapping failed: {addrs if not ok else 'on a peer'}")
        return mem, addrs

    def _wait_flags(self, first, groups, count, skip):
        """The current stream waits (bounded) until flags[first + g * world + i] (g < groups, i < count, i != skip)
        reached this block's counter."""
        lib = self._lib
        cur = torch.cuda.current_stream(self.device)
        lib.check(lib.lib.hn_wait_flags(ctypes.c_void_p(self.flags.data_ptr() + 4 * first), groups, count, self.world,
                                        skip, self.epoch, self.timeout_us, ctypes.c_void_p(cur.cuda_stream)),
                  "hn_wait_flags")

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


class PeerExchange(_IpcExchange):
    """The copy-engine K/V exchange of one `SequenceParallel` (the token split).

    Per buffer shape one allocation holds [parity 2][K, V][batch 1][prefix + local * world][heads][head_dim]; the
    flags are int32 [K, V][world]: flags[kind][src] = the last block counter whose `kind` slice `src` pushed here."""

    def __init__(self, sp):
        nstreams = max(1, min(sp.world - 1, int(os.environ.get("HN_SP_PUSH_STREAMS", str(PUSH_STREAMS)))))
        self._setup(sp, 2 * sp.world)
        self.side = [[torch.cuda.Stream(self.device) for _ in range(nstreams)] for _kind in range(2)]

    def _buffers(self, batch, local, heads, head_dim, dtype, prefix):
        key = (batch, local, heads, head_dim, dtype, prefix)
        ent = self._bufs.get(key)
        if ent is None:
            total = prefix + local * self.world
            mem, addrs = self._shared_alloc(2 * 2 * batch * total * heads * head_dim, dtype)
            mem = mem.view(2, 2, batch, total, heads, head_dim)
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
        if peer is None:
            self._wait_flags(0, 2, self.world, self.rank)
        else:
            self._wait_flags(peer, 2, 1, -1)

    def arrival_order(self):
        """The peers in the order their slices reach this rank: every rank pushes to rank + 1 first, so this rank
        hears from rank - 1 first, then rank - 2, ..."""
        return [(self.rank - s) % self.world for s in range(1, self.world)]



# the head-parallel exchange's kinds: each has its flag row and copy stream
HEAD_KINDS = ("k", "v", "q", "o")


class _HeadLayout:
    """Buffers of one head-parallel block shape: for this rank's head group (hpg = heads / world heads) the K and V
    of the history and of all tokens, [prefix + L, hpg, head_dim], and the Q of all tokens, [L, hpg, head_dim]; for
    this rank's own tokens the attention output of all heads, [local, heads, head_dim] (the projection's input).
    All rank-major: rank p's tokens are rows [p * local, (p + 1) * local) of the token part."""

    def __init__(self, world, local, heads, head_dim, prefix):
        self.world, self.local, self.heads, self.head_dim, self.prefix = world, local, heads, head_dim, prefix
        self.hpg = heads // world
        self.tokens = local * world
        kv = (prefix + self.tokens) * self.hpg * head_dim
        q = self.tokens * self.hpg * head_dim
        o = local * heads * head_dim
        self.offs = {"k": 0, "v": kv, "q": 2 * kv, "o": 2 * kv + q}   # elements into one set
        self.sizes = {"k": kv, "v": kv, "q": q, "o": o}
        self.numel = 2 * kv + q + o                                   # elements of one set

    def views(self, flat):
        """(q, k, v, o) over one set of `flat` (1-D, `numel` elements)."""
        hd, hpg = self.head_dim, self.hpg
        part = {n: flat[self.offs[n]:self.offs[n] + self.sizes[n]] for n in HEAD_KINDS}
        return (part["q"].view(1, self.tokens, hpg, hd), part["k"].view(1, self.prefix + self.tokens, hpg, hd),
                part["v"].view(1, self.prefix + self.tokens, hpg, hd), part["o"].view(1, self.local, self.heads, hd))

    def row0(self, kind, rank):
        """First row of `rank`'s tokens in a K, V or Q buffer."""
        return (self.prefix if kind in ("k", "v") else 0) + rank * self.local

    def push_plan(self, kind, rank, peer, par, esz):
        """The strided copy of `kind` from `rank` to `peer`'s set of parity `par`: (source byte offset, source
        pitch, destination byte offset in the peer's allocation, destination pitch, row bytes, rows). The source
        is rank's [local, heads, head_dim] tensor for K, V and Q (peer's head group of every own token), its
        [L, hpg, head_dim] output for O (peer's token rows)."""
        hd, hpg = self.head_dim, self.hpg
        width = hpg * hd * esz
        base = par * self.numel + self.offs[kind]
        if kind == "o":
            return (peer * self.local * width, width, (base + rank * hpg * hd) * esz, self.heads * hd * esz, width,
                    self.local)
        return (peer * width, self.heads * hd * esz, (base + self.row0(kind, rank) * hpg * hd) * esz, width, width,
                self.local)


class HeadExchange(_IpcExchange):
    """The copy-engine exchange of head-parallel attention.

    Per block shape one allocation holds two sets (block parity) of `_HeadLayout` buffers, mapped on every peer;
    the flags are int32 [K, V, Q, O][world]: flags[kind][src] = the last block counter whose `kind` rows `src`
    pushed here. Rank r's K (then V, then Q) push is, for every peer p, one strided DMA of p's head group of r's
    tokens (rows of hpg * head_dim elements out of rows of heads * head_dim) into p's buffer at r's token rows; its
    own head group is a copy on the current stream. The output push returns to every peer p the rows of p's tokens
    of r's head group, into p's output buffer at r's head columns. Ordering: a rank's pushes of block n into a
    peer's set of parity n % 2 follow its waits for that peer's K/V/Q of block n - 1, which the peer pushed after
    its attention and projection of block n - 2 (the last readers of that set); the sources are this block's own
    tensors, kept from reuse until the copy streams have read them (`record_stream`)."""

    def __init__(self, sp):
        nstreams = max(1, min(sp.world - 1, int(os.environ.get("HN_SP_HEAD_PUSH_STREAMS", str(HEAD_PUSH_STREAMS)))))
        self._setup(sp, len(HEAD_KINDS) * sp.world)
        self.side = {k: [torch.cuda.Stream(self.device) for _ in range(nstreams)] for k in HEAD_KINDS}

    def _buffers(self, local, heads, head_dim, dtype, prefix):
        key = (local, heads, head_dim, dtype, prefix)
        ent = self._bufs.get(key)
        if ent is None:
            lay = _HeadLayout(self.world, local, heads, head_dim, prefix)
            mem, addrs = self._shared_alloc(2 * lay.numel, dtype)
            ent = dict(lay=lay, mem=mem, addrs=addrs, esz=mem.element_size())
            self._bufs[key] = ent
        return ent

    def begin(self, local, heads, head_dim, dtype, device=None, prefix=0):
        """Start a block: (q, k, v, o) of this block's parity (see `_HeadLayout`)."""
        self.epoch = (self.epoch + 1) & 0xFFFFFFFF
        par = self.epoch & 1
        ent = self._buffers(local, heads, head_dim, dtype, prefix)
        lay = ent["lay"]
        self._cur = (ent, par)
        return lay.views(ent["mem"][par * lay.numel:(par + 1) * lay.numel])

    def _push_rows(self, kind, src, own):
        """On `kind`'s copy streams, after the current stream's work so far: for every peer (staggered from rank + 1,
        spread over the streams) the strided DMA of `_HeadLayout.push_plan` followed by its flag; then `own()` on
        the current stream."""
        lib = self._lib
        ent, par = self._cur
        cur = torch.cuda.current_stream(self.device)
        sides = self.side[kind]
        ready = torch.cuda.Event()
        ready.record(cur)
        for side in sides:
            side.wait_event(ready)
        k = HEAD_KINDS.index(kind)
        for step in range(1, self.world):
            peer = (self.rank + step) % self.world
            st = ctypes.c_void_p(sides[(step - 1) % len(sides)].cuda_stream)
            flag = ctypes.c_void_p(self.peer_flags[peer] + 4 * (k * self.world + self.rank))
            soff, spitch, doff, dpitch, width, height = ent["lay"].push_plan(kind, self.rank, peer, par, ent["esz"])
            lib.check(lib.lib.hn_peer_push2d(ctypes.c_void_p(ent["addrs"][peer] + doff), dpitch,
                                             ctypes.c_void_p(src.data_ptr() + soff), spitch, width, height,
                                             flag, self.epoch, st), "hn_peer_push2d", launches=0)
        for side in sides:
            src.record_stream(side)
        own()

    def send(self, kind, src, bufs):
        """Send this rank's K, V or Q ([1, local, heads, head_dim], contiguous, complete on the current stream):
        every peer's head group to that peer; `bufs` = this block's (q, k, v, o) from `begin`."""
        ent = self._cur[0]
        lay, esz = ent["lay"], ent["esz"]
        hd, hpg = lay.head_dim, lay.hpg
        if (not src.is_contiguous() or tuple(src.shape) != (1, lay.local, lay.heads, hd)
                or src.element_size() != esz or src.device != self.device):
            raise ValueError(f"send: need a contiguous [1, {lay.local}, {lay.heads}, {hd}] tensor on {self.device}")
        r0 = lay.row0(kind, self.rank)
        mine = bufs["qkv".index(kind)]

        def own():
            mine[0, r0:r0 + lay.local].copy_(src[0, :, self.rank * hpg:(self.rank + 1) * hpg])

        self._push_rows(kind, src, own)

    def send_output(self, out, bufs):
        """Return this rank's head group's attention output ([1, L, hpg, head_dim], contiguous) to the ranks that own
        its tokens, into their output buffers."""
        ent = self._cur[0]
        lay, esz = ent["lay"], ent["esz"]
        hd, hpg = lay.head_dim, lay.hpg
        if (not out.is_contiguous() or tuple(out.shape) != (1, lay.tokens, hpg, hd) or out.element_size() != esz
                or out.device != self.device):
            raise ValueError(f"send_output: need a contiguous [1, {lay.tokens}, {hpg}, {hd}] tensor on {self.device}")
        o_mine = bufs[3]
        lo = self.rank * lay.local

        def own():
            o_mine[0, :, self.rank * hpg:(self.rank + 1) * hpg].copy_(out[0, lo:lo + lay.local])

        self._push_rows("o", out, own)

    def wait(self, kinds):
        """The current stream waits (bounded) until every peer's rows of `kinds` ("kvq" or "o") of this block are
        here."""
        if kinds == "kvq":
            self._wait_flags(0, 3, self.world, self.rank)
        elif kinds == "o":
            self._wait_flags(3 * self.world, 1, self.world, self.rank)
        else:
            raise ValueError(f"wait: kinds must be 'kvq' or 'o', got {kinds!r}")


class HeadCollective:
    """The head-parallel exchange by all-to-all collectives (NCCL on GPUs when the copy engines are not used, gloo
    on CPU): the same buffers and calls as `HeadExchange`. A rank's Q, K or V is reordered head-group-major
    ([world, local, hpg, head_dim]) so that chunk p is peer p's, and the received chunks land rank-major in the
    buffer; the output comes back as [world (head group), local, hpg, head_dim] and is reordered into the
    [local, heads, head_dim] buffer."""

    def __init__(self, sp):
        self.world, self.rank, self.group = sp.world, sp.rank, sp.group
        self._bufs = {}
        self._pending = {}

    def begin(self, local, heads, head_dim, dtype, device=None, prefix=0):
        key = (local, heads, head_dim, dtype, str(device), prefix)
        ent = self._bufs.get(key)
        if ent is None:
            lay = _HeadLayout(self.world, local, heads, head_dim, prefix)
            ent = (lay, torch.empty(lay.numel, dtype=dtype, device=device))
            self._bufs[key] = ent
        self._lay = ent[0]
        return ent[0].views(ent[1])

    def send(self, kind, src, bufs):
        lay = self._lay
        inp = src[0].view(lay.local, self.world, lay.hpg, lay.head_dim).permute(1, 0, 2, 3).contiguous()
        r0 = lay.prefix if kind in ("k", "v") else 0
        dst = bufs["qkv".index(kind)][0, r0:r0 + lay.tokens]
        h = dist.all_to_all_single(dst.reshape(-1), inp.view(-1), group=self.group, async_op=True)
        self._pending[kind] = (h, inp)

    def send_output(self, out, bufs):
        inp = out[0].contiguous()
        recv = torch.empty_like(inp)
        h = dist.all_to_all_single(recv.view(-1), inp.view(-1), group=self.group, async_op=True)
        self._pending["o"] = (h, inp, recv, bufs[3])

    def wait(self, kinds):
        for kind in kinds:
            ent = self._pending.pop(kind)
            ent[0].wait()
            if kind == "o":
                lay, recv, o_mine = self._lay, ent[2], ent[3]
                o_mine[0].view(lay.local, self.world, lay.hpg, lay.head_dim).copy_(
                    recv.view(self.world, lay.local, lay.hpg, lay.head_dim).permute(1, 0, 2, 3))

    def close(self):
        self._pending.clear()
