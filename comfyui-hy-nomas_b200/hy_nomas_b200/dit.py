"""Synthetic Hy-Nomas-style DiT on the B200 kernels: one block and the multi-block denoise step.

The block is the image stream of the reference's `DoubleStreamBlock` on its fused int8 path
(hy_nomas/model.py:246-286, with `MLP.forward_int8` model.py:79-86 and `Modulate` model.py:303-311):

    shift1, scale1, gate1, shift2, scale2, gate2 = Modulate(vec)          int8 linear of silu(vec)
    qa, sa  = adaln_quant(x, shift1, scale1)                              LN + modulate + int8 quant
    q, k, v = block_gemm(qa, sa, W_q / W_k / W_v)                         one GEMM for v, one for q|k
    q, k    = qk_norm_rope(q), qk_norm_rope(k)                            one launch for both (one GPU)
    attn    = scaled_dot_product_attention(q, K, V)                       torch SDPA, unchanged
    x       = gated_residual(x, proj(attn), gate1)                        proj = quantize + GEMM
    qh, sh  = block_gemm(adaln_quant(x, shift2, scale2), W_fc1, "gelu_quant")
    x       = gated_residual(x, block_gemm(qh, sh, W_fc2), gate2)

Two launches are merged where the result is identical: q and k come from one GEMM over the concatenated
weights (every output column is computed independently, so the values do not change), and the first
residual is fused with the second LayerNorm/quantization (`gated_residual_adaln_quant`, bit-identical to the
two kernels in sequence). Under sequence parallelism (`SequenceParallel`) each rank runs the block on its own
tokens and K/V are all-gathered; the k and v kernels write straight into the rank's slice of the gather
buffers.

Weights are random and seeded (there is no checkpoint offline): int8 codes uniform in [-127, 127] with
per-output-channel fp32 scales, scaled so each linear preserves the activations' variance, and bf16 biases
N(0, 0.02). The RMSNorm weights are ones, as `RMSNorm.__init__` creates them (model.py:95).

`ops` is the compute seam: the default `CudaOps` calls libhynomas_b200.so for every op except attention;
host-side tests pass a CPU object with the same methods to check the orchestration (shards, gathers) on gloo.
"""
import math
import os
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from . import attention as attention_mod
from . import fused, kernels, world
from .sequence_parallel import SequenceParallel

# the step's attention (HN_ATTENTION overrides): "sdpa" - torch SDPA, as the reference's pytorch backend - or
# "native" - the library's kernel, whose fused output quantizer feeds the projection linear directly
ATTENTION = "sdpa"
# under the copy-engine exchange, HN_SP_ATTENTION_PIECES=1 attends in key pieces - the local keys first, then each
# peer's slice as it arrives - merged by log-sum-exp. Off by default: at 4 GPUs it was slower than attending once
# (159.5 against 155.5 ms per step) and its rounding, compounded over 40 blocks, left the step 1.2% (rel-L2) from
# the one-GPU result, where attending once after every slice arrived is bit-identical to it.
SP_ATTENTION_PIECES = False
# SMs each GEMM leaves free under sequence parallelism (HN_SP_GEMM_SM_RESERVE overrides)
SP_GEMM_SM_RESERVE = 0


@dataclass(frozen=True)
class DiTConfig:
    hidden: int = 4096
    heads: int = 32
    mlp_ratio: int = 4
    blocks: int = 40
    rope_dims: tuple = (16, 56, 56)
    theta: float = 10000.0
    grid: tuple = (23, 22, 40)   # latent frames x patch rows x patch columns = 20240 tokens
    t_offset: int = 0            # frame index of the first latent frame (RoPE positions; > 0 after history)

    @property
    def head_dim(self):
        return self.hidden // self.heads

    @property
    def tokens(self):
        t, h, w = self.grid
        return t * h * w


@dataclass
class QLinear:
    """An int8 linear: codes [N, K], per-output-channel fp32 scales [N], bf16 bias [N]."""
    q: torch.Tensor
    s: torch.Tensor
    bias: torch.Tensor


@dataclass
class BlockWeights:
    mod: QLinear     # [6D, D]
    qk: QLinear      # [2D, D]: the q rows then the k rows
    v: QLinear       # [D, D]
    proj: QLinear    # [D, D]
    fc1: QLinear     # [mlp, D]
    fc2: QLinear     # [D, mlp]
    q_norm: torch.Tensor   # bf16 [head_dim]
    k_norm: torch.Tensor


_CODE_STD = math.sqrt((255.0 ** 2 - 1.0) / 12.0)   # std of an integer uniform on [-127, 127]


def make_qlinear(n, k, gen, device, gain=1.0):
    q = torch.randint(-127, 128, (n, k), generator=gen, device=device, dtype=torch.int8)
    s = (torch.rand(n, generator=gen, device=device) + 0.5) * (gain / (_CODE_STD * math.sqrt(k)))
    bias = (torch.randn(n, generator=gen, device=device) * 0.02).to(torch.bfloat16)
    return QLinear(q, s.float().contiguous(), bias)


def make_block_weights(cfg, gen, device):
    d, mlp = cfg.hidden, cfg.hidden * cfg.mlp_ratio
    ones = torch.ones(cfg.head_dim, dtype=torch.bfloat16, device=device)
    return BlockWeights(mod=make_qlinear(6 * d, d, gen, device, gain=0.15), qk=make_qlinear(2 * d, d, gen, device),
                        v=make_qlinear(d, d, gen, device), proj=make_qlinear(d, d, gen, device),
                        fc1=make_qlinear(mlp, d, gen, device), fc2=make_qlinear(d, mlp, gen, device),
                        q_norm=ones, k_norm=ones.clone())


def rope_freqs(rope_dims, theta, t, h, w, t_offset=0, device=None):
    """3-D RoPE tables (cos, sin) fp32 [t*h*w, sum(rope_dims)] for the grid [t_offset, t_offset+t) x [0, h) x
    [0, w): per axis fp32 positions from a linspace, fp32 frequencies theta^(-2i/dim), cos/sin repeated per
    interleaved pair (hy_nomas/model.py:114-128). Built once per shape; not on the per-step path."""
    axes = [torch.linspace(s, s + n, n + 1, dtype=torch.float32, device=device)[:n]
            for s, n in ((t_offset, t), (0, h), (0, w))]
    grid = torch.meshgrid(*axes, indexing="ij")
    cos, sin = [], []
    for dim, pos in zip(rope_dims, grid):
        freqs = 1.0 / (theta ** (torch.arange(0, dim, 2, device=device)[: dim // 2].float() / dim))
        angles = torch.outer(pos.reshape(-1), freqs)
        cos.append(angles.cos().repeat_interleave(2, dim=1))
        sin.append(angles.sin().repeat_interleave(2, dim=1))
    return torch.cat(cos, dim=1).contiguous(), torch.cat(sin, dim=1).contiguous()


class CudaOps:
    """The block's ops on libhynomas_b200.so (attention: torch SDPA, as the reference's pytorch backend)."""

    @staticmethod
    def linear(x2, w):
        return kernels.block_linear(x2, w.q, w.s, w.bias)

    @staticmethod
    def adaln_quant(x, shift, scale):
        return kernels.adaln_quant(x, shift, scale)

    @staticmethod
    def gemm(qa, sa, w, epilogue=None, out=None):
        return kernels.block_gemm(qa, sa, w.q, w.s, w.bias, epilogue=epilogue, out=out)

    @staticmethod
    def qk_norm_rope2(q, k, wq, wk, rope, out):
        return fused.qk_norm_rope2(q, k, wq, wk, rope, out=out)

    @staticmethod
    def qk_norm_rope(x, w, rope, out):
        return fused.qk_norm_rope(x, w, rope, out=out)

    @staticmethod
    def gated_residual_adaln_quant(x, y, gate, shift, scale):
        return fused.gated_residual_adaln_quant(x, y, gate, shift, scale)

    @staticmethod
    def qk_norm_rope_kv(x, w, rope, out):
        """QK-norm + RoPE into `out`, and its int8 KV-cache codes and scales from the same launch."""
        _, q, s = fused.qk_norm_rope_kv(x, w, rope, out=out)
        return q, s

    @staticmethod
    def quantize_kv(x):
        return world.quantize_kv(x)

    @staticmethod
    def dequantize_kv(q, s, out):
        return world.dequantize_kv(q, s, out=out)

    @staticmethod
    def attention_lse(q, k, v):
        return attention_mod.attention_lse(q, k, v)

    @staticmethod
    def attention_merge(pieces, keep_output=False):
        """The projection input (codes, scales) from attention pieces, and the bf16 output first with keep_output."""
        return attention_mod.merge(pieces, quantize=True, keep_output=keep_output)

    @staticmethod
    def attention_quant(q, k, v, keep_output=False):
        """The library's attention with the projection linear's input quantizer fused into its epilogue:
        (codes, scales) or, with keep_output, (bf16 output, (codes, scales))."""
        return attention_mod.attention_quant(q, k, v, keep_output=keep_output)

    @staticmethod
    def gated_residual(x, y, gate):
        return fused.gated_residual(x, y, gate)

    @staticmethod
    def silu(v):
        return F.silu(v)

    @staticmethod
    def attention(q, k, v):
        """q [B, Lq, H, D], k/v [B, Lk, H, D] -> [B, Lq, H, D] (hy_nomas/model.py:145-151, pytorch backend)."""
        return F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)).transpose(1, 2)


def block_forward(cfg, w, x, vec, rope, sp, ops=CudaOps, trace=None, mods=None, x_q=None, next_mods=None,
                  history=None, capture=None):
    """One block on this rank's tokens. x bf16 [B, l, D] (l = the rank's tokens), vec bf16 [B, D], rope =
    this rank's rows of the (cos, sin) tables. Returns the block output [B, l, D] bf16. `trace`, when a dict,
    receives the block's intermediates (for parity tests). `mods`: this block's Modulate(vec) output [B, 6D] when
    the caller computed it already (`SyntheticDiT` does it for all blocks in one GEMM); else computed here.

    Chaining blocks: `next_mods` (the next block's modulations) fuses this block's final gated residual with the
    next block's LN + modulate + int8 quantization (one pass, bit-identical to the two kernels) and makes the
    return value (out, (qa, sa)); the next block takes that pair as `x_q` instead of quantizing `out` again.

    The segment history (hy_nomas/model.py:199-209, world.py:197-204): `history` = (hk_q, hk_s, hv_q, hv_s), this
    block's int8 K/V cache of earlier frames, codes [Lh, H, D] and scales [Lh, H, 1] (world.quantize_kv's
    format, the same on every rank). They are dequantized straight into the first Lh positions of the K/V
    buffers, ahead of the current tokens', and the current tokens attend over history + current as the
    reference's torch.cat([hk, k]) does. `capture`, when a list, receives this block's int8 cache of the rank's
    own tokens (kq, ks, vq, vs): K quantized inside the QK-norm + RoPE kernel, V by the KV quantizer - the cache
    pass that writes the history of a finished segment."""
    b, l, d = x.shape
    h, hd = cfg.heads, cfg.head_dim
    act = ops.silu(vec) if (mods is None or trace is not None) else None
    if mods is None:
        mods = ops.linear(act, w.mod)
    shift1, scale1, gate1, shift2, scale2, gate2 = mods.chunk(6, dim=-1)
    qa, sa = x_q if x_q is not None else ops.adaln_quant(x, shift1, scale1)
    chunks = sp.head_chunks if (sp.world > 1 and h % sp.head_chunks == 0) else 1
    if (history is not None or capture is not None) and chunks > 1:
        raise NotImplementedError("history and capture take the unchunked K/V exchange (head_chunks = 1)")
    if chunks > 1:
        attn, k_full, v_full, qk, q_out = _attention_chunked(cfg, w, qa, sa, rope, sp, ops, b, l, chunks,
                                                             keep_kv=trace is not None)
        return _post(cfg, w, x, attn, qa, sa, qk, q_out, k_full, v_full, act, mods, gate1, shift2, scale2, gate2,
                     ops, trace, next_mods)
    lh = 0 if history is None else history[0].shape[0]
    if chunks == 1 and sp.head_split(h):
        attn, k_full, v_full, qk, q_out = _attention_heads(cfg, w, qa, sa, rope, sp, ops, b, l, lh, history, capture,
                                                           x.dtype, trace is not None)
        return _post(cfg, w, x, attn, qa, sa, qk, q_out, k_full, v_full, act, mods, gate1, shift2, scale2, gate2,
                     ops, trace, next_mods)
    if sp.peer is not None:
        attn, k_full, v_full, qk, q_out = _attention_pushed(cfg, w, qa, sa, rope, sp.peer, ops, b, l, lh, history,
                                                            capture, x.dtype, trace is not None)
        return _post(cfg, w, x, attn, qa, sa, qk, q_out, k_full, v_full, act, mods, gate1, shift2, scale2, gate2,
                     ops, trace, next_mods)
    k_full, v_full, k_mine, v_mine = sp.kv_buffers(b, l, h, hd, x.dtype, x.device, prefix=lh)
    if history is not None:
        hk_q, hk_s, hv_q, hv_s = history
        for bi in range(b):
            ops.dequantize_kv(hk_q, hk_s, out=k_full[bi, :lh])
            ops.dequantize_kv(hv_q, hv_s, out=v_full[bi, :lh])
    # v first, so its all-gather runs under the q|k GEMM; k is normalized before q, so its gather runs under
    # q's normalization (with one rank the gathers are no-ops and the order changes nothing)
    ops.gemm(qa, sa, w.v, out=v_mine.view(b * l, d))
    gather_v = sp.all_gather_async(v_full, v_mine)
    qk = ops.gemm(qa, sa, w.qk)                                       # [B*l, 2D]
    q_in = qk[:, :d].view(b, l, h, hd)
    k_in = qk[:, d:].view(b, l, h, hd)
    q_out = torch.empty((b, l, h, hd), dtype=x.dtype, device=x.device)
    if capture is not None:
        kq, ks = ops.qk_norm_rope_kv(k_in, w.k_norm, rope, out=k_mine)
        gather_k = sp.all_gather_async(k_full, k_mine)
        ops.qk_norm_rope(q_in, w.q_norm, rope, out=q_out)
        vq, vs = ops.quantize_kv(v_mine.reshape(b * l, h, hd))
        capture.append((kq.reshape(b * l, h, hd), ks.reshape(b * l, h, 1), vq, vs))
    elif sp.world > 1:
        ops.qk_norm_rope(k_in, w.k_norm, rope, out=k_mine)
        gather_k = sp.all_gather_async(k_full, k_mine)
        ops.qk_norm_rope(q_in, w.q_norm, rope, out=q_out)
    else:
        ops.qk_norm_rope2(q_in, k_in, w.q_norm, w.k_norm, rope, out=(q_out, k_mine))
        gather_k = None
    sp.wait(gather_k, gather_v)
    attn = _attend(ops, q_out, k_full, v_full, trace is not None)
    return _post(cfg, w, x, attn, qa, sa, qk, q_out, k_full, v_full, act, mods, gate1, shift2, scale2, gate2, ops,
                 trace, next_mods)


def _attend(ops, q, k, v, keep):
    """Attention for the projection linear: (attn [B*l, D] bf16 or None, (codes, scales) or None). With the native
    kernel the projection's input quantization comes out of attention's epilogue (and the bf16 output only when
    `keep`, for traces); with SDPA the projection quantizes the bf16 output itself."""
    b, l, h, hd = q.shape
    if os.environ.get("HN_ATTENTION", ATTENTION) == "native" and hasattr(ops, "attention_quant"):
        if keep:
            out, codes = ops.attention_quant(q, k, v, keep_output=True)
            return out.reshape(b * l, h * hd), codes
        return None, ops.attention_quant(q, k, v)
    return ops.attention(q, k, v).reshape(b * l, h * hd), None


def _attention_pushed(cfg, w, qa, sa, rope, peer, ops, b, l, lh, history, capture, dtype, keep_qk):
    """Attention under the copy-engine exchange: K is projected and normalized first and pushed to the peers
    while V is projected, V is pushed while Q is projected and normalized, and attention waits for the peers'
    slices. Each of the q|k linear's halves is its own GEMM (the same output columns, so the same values).
    `keep_qk`: also return the q|k projection [B*l, 2D] (for traces), else None."""
    h, hd = cfg.heads, cfg.head_dim
    d = h * hd
    k_full, v_full, k_mine, v_mine = peer.begin(b, l, h, hd, dtype, prefix=lh)
    if history is not None:
        hk_q, hk_s, hv_q, hv_s = history
        ops.dequantize_kv(hk_q, hk_s, out=k_full[0, :lh])
        ops.dequantize_kv(hv_q, hv_s, out=v_full[0, :lh])
    k_in = ops.gemm(qa, sa, _rows(w.qk, d, 2 * d)).view(b, l, h, hd)
    if capture is not None:
        kq, ks = ops.qk_norm_rope_kv(k_in, w.k_norm, rope, out=k_mine)
    else:
        ops.qk_norm_rope(k_in, w.k_norm, rope, out=k_mine)
    peer.push(0)
    ops.gemm(qa, sa, w.v, out=v_mine.view(b * l, d))
    peer.push(1)
    q_in = ops.gemm(qa, sa, _rows(w.qk, 0, d)).view(b, l, h, hd)
    q_out = torch.empty((b, l, h, hd), dtype=dtype, device=qa.device)
    ops.qk_norm_rope(q_in, w.q_norm, rope, out=q_out)
    if capture is not None:
        vq, vs = ops.quantize_kv(v_mine.reshape(b * l, h, hd))
        capture.append((kq.reshape(b * l, h, hd), ks.reshape(b * l, h, 1), vq, vs))
    pieces = os.environ.get("HN_SP_ATTENTION_PIECES", "1" if SP_ATTENTION_PIECES else "0") != "0"
    if pieces and hasattr(ops, "attention_lse"):
        attn = _attend_pieces(ops, q_out, k_full, v_full, lh, l, peer, keep_qk)
    else:
        peer.wait()
        attn = _attend(ops, q_out, k_full, v_full, keep_qk)
    qk = torch.cat([q_in.reshape(b * l, d), k_in.reshape(b * l, d)], dim=1) if keep_qk else None
    return attn, k_full, v_full, qk, q_out


def _attention_heads(cfg, w, qa, sa, rope, sp, ops, b, l, lh, history, capture, dtype, keep_qk):
    """Head-parallel attention: this rank attends for its head group over all tokens. K is projected, normalized
    and sent (every peer's head group to that peer) while V is projected, V is sent while Q is projected and
    normalized, Q is sent; after the wait for the peers' rows, attention over [history + all tokens] for the
    group, and its output goes back to the ranks owning the tokens, into the projection's input [l, heads * D].
    The history, the same on every rank, is dequantized for this rank's heads only. `keep_qk`: also return the
    q|k projection (for traces); the K/V returned are this head group's."""
    h, hd = cfg.heads, cfg.head_dim
    d = h * hd
    ex = sp.head_exchange()
    hpg = h // sp.world
    mine = slice(sp.rank * hpg, (sp.rank + 1) * hpg)
    bufs = ex.begin(l, h, hd, dtype, qa.device, prefix=lh)
    q_all, k_all, v_all, o_mine = bufs
    if history is not None:
        hk_q, hk_s, hv_q, hv_s = history
        ops.dequantize_kv(hk_q[:, mine], hk_s[:, mine], out=k_all[0, :lh])
        ops.dequantize_kv(hv_q[:, mine], hv_s[:, mine], out=v_all[0, :lh])
    k_in = ops.gemm(qa, sa, _rows(w.qk, d, 2 * d)).view(b, l, h, hd)
    k_mine = torch.empty((b, l, h, hd), dtype=dtype, device=qa.device)
    if capture is not None:
        kq, ks = ops.qk_norm_rope_kv(k_in, w.k_norm, rope, out=k_mine)
    else:
        ops.qk_norm_rope(k_in, w.k_norm, rope, out=k_mine)
    ex.send("k", k_mine, bufs)
    v_mine = ops.gemm(qa, sa, w.v).view(b, l, h, hd)
    ex.send("v", v_mine, bufs)
    q_in = ops.gemm(qa, sa, _rows(w.qk, 0, d)).view(b, l, h, hd)
    q_out = torch.empty((b, l, h, hd), dtype=dtype, device=qa.device)
    ops.qk_norm_rope(q_in, w.q_norm, rope, out=q_out)
    ex.send("q", q_out, bufs)
    if capture is not None:
        vq, vs = ops.quantize_kv(v_mine.reshape(b * l, h, hd))
        capture.append((kq.reshape(b * l, h, hd), ks.reshape(b * l, h, 1), vq, vs))
    ex.wait("kvq")
    out = ops.attention(q_all, k_all, v_all).contiguous()              # [1, L, hpg, D]
    ex.send_output(out, bufs)
    ex.wait("o")
    qk = torch.cat([q_in.reshape(b * l, d), k_in.reshape(b * l, d)], dim=1) if keep_qk else None
    return (o_mine.reshape(b * l, d), None), k_all, v_all, qk, q_out


def _attend_pieces(ops, q, k_full, v_full, lh, l, peer, keep):
    """Attention over the history, this rank's slice and then each peer's slice in arrival order, every piece as
    soon as its keys are here (a bounded wait per peer), merged by log-sum-exp into the projection linear's input;
    returns what `_attend` returns."""
    b, lq, h, hd = q.shape
    mine = lh + peer.rank * l
    ranges = ([(0, lh, None)] if lh else []) + [(mine, mine + l, None)]
    ranges += [(lh + p * l, lh + (p + 1) * l, p) for p in peer.arrival_order()]
    pieces = []
    for lo, hi, p in ranges:
        if p is not None:
            peer.wait(p)
        pieces.append(ops.attention_lse(q, k_full[:, lo:hi], v_full[:, lo:hi]))
    if keep:
        out, codes = ops.attention_merge(pieces, keep_output=True)
        return out.reshape(b * lq, h * hd), codes
    return None, ops.attention_merge(pieces)


def _rows(w, lo, hi):
    """Output rows [lo, hi) of an int8 linear (views)."""
    return QLinear(w.q[lo:hi], w.s[lo:hi], w.bias[lo:hi])


def _attention_chunked(cfg, w, qa, sa, rope, sp, ops, b, l, chunks, keep_kv=False):
    """Attention with the K/V all-gathers split into `chunks` head groups: every chunk's V projection and K
    normalization write the rank's slice of that chunk's gather buffers, the gathers are issued as soon as their
    inputs exist (V's under the q|k GEMM), and chunk c's attention only waits for chunk c's K and V, so the
    gathers of later chunks run under it. Per head the arithmetic is that of the unchunked path. `keep_kv`:
    also return the full K and V (for traces), else None."""
    h, hd = cfg.heads, cfg.head_dim
    d = h * hd
    hc = h // chunks
    bufs = sp.kv_chunk_buffers(b, l, h, hd, chunks, torch.bfloat16, qa.device)
    gathers_v, gathers_k = [], []
    for c, (kf, vf, km, vm) in enumerate(bufs):
        ops.gemm(qa, sa, _rows(w.v, c * hc * hd, (c + 1) * hc * hd), out=vm.view(b * l, hc * hd))
        gathers_v.append(sp.all_gather_async(vf, vm))
    qk = ops.gemm(qa, sa, w.qk)                                       # [B*l, 2D]
    q_in = qk[:, :d].view(b, l, h, hd)
    k_in = qk[:, d:].view(b, l, h, hd)
    for c, (kf, vf, km, vm) in enumerate(bufs):
        ops.qk_norm_rope(k_in[:, :, c * hc:(c + 1) * hc], w.k_norm, rope, out=km)
        gathers_k.append(sp.all_gather_async(kf, km))
    q_out = torch.empty((b, l, h, hd), dtype=torch.bfloat16, device=qa.device)
    ops.qk_norm_rope(q_in, w.q_norm, rope, out=q_out)
    attn = torch.empty((b, l, h, hd), dtype=torch.bfloat16, device=qa.device)
    for c, (kf, vf, km, vm) in enumerate(bufs):
        sp.wait(gathers_k[c], gathers_v[c])
        attn[:, :, c * hc:(c + 1) * hc] = ops.attention(q_out[:, :, c * hc:(c + 1) * hc], kf, vf)
    k_full = torch.cat([kf for kf, _, _, _ in bufs], dim=2) if keep_kv else None
    v_full = torch.cat([vf for _, vf, _, _ in bufs], dim=2) if keep_kv else None
    return (attn.view(b * l, d), None), k_full, v_full, qk, q_out


def _post(cfg, w, x, attn, qa, sa, qk, q_out, k_full, v_full, act, mods, gate1, shift2, scale2, gate2, ops, trace,
          next_mods=None):
    """The block after attention: projection, gated residual + LN + quant, MLP, gated residual (fused with the
    next block's LN + quant when `next_mods` is given: returns (out, (qa, sa)) then)."""
    b, l, d = x.shape
    attn, attn_q = attn
    proj = (ops.gemm(*attn_q, w.proj) if attn_q is not None else ops.linear(attn, w.proj)).view(b, l, d)
    x1, qa2, sa2 = ops.gated_residual_adaln_quant(x, proj, gate1, shift2, scale2)
    qh, sh = ops.gemm(qa2, sa2, w.fc1, epilogue="gelu_quant")
    y = ops.gemm(qh, sh, w.fc2).view(b, l, d)
    nxt = None
    if next_mods is None:
        out = ops.gated_residual(x1, y, gate2)
    else:
        nshift1, nscale1 = next_mods.chunk(6, dim=-1)[:2]
        out, nqa, nsa = ops.gated_residual_adaln_quant(x1, y, gate2, nshift1, nscale1)
        nxt = (nqa, nsa)
    if trace is not None:
        trace.update(act=act, mods=mods, qa=qa, sa=sa, qk=qk, q=q_out, k_full=k_full.clone(), v_full=v_full.clone(),
                     attn=attn, proj=proj, x1=x1, qa2=qa2, sa2=sa2, qh=qh, sh=sh, y=y, out=out)
    return out if nxt is None else (out, nxt)


class SyntheticDiT:
    """`cfg.blocks` random-init blocks over a `cfg.grid` token sequence, sequence-parallel over `sp`'s ranks.

    Every rank builds the same weights (same seed; weights are replicated) and its own rows of the RoPE tables.
    `forward(x, vec)` takes this rank's tokens [B, l, D] and returns them after all blocks."""

    def __init__(self, cfg=DiTConfig(), device="cuda", seed=0, sp=None, ops=CudaOps):
        self.cfg = cfg
        self.device = torch.device(device)
        self.sp = sp or SequenceParallel()
        self.ops = ops
        gen = torch.Generator(device=self.device).manual_seed(seed)
        self.blocks = [make_block_weights(cfg, gen, self.device) for _ in range(cfg.blocks)]
        # Every block's Modulate reads the same vec (model.py:247), so the blocks' [6D, D] modulation weights are
        # stacked into one [blocks * 6D, D] linear and each block keeps a row view of it: one quantization of
        # silu(vec) and one GEMM give all blocks' shift/scale/gate per step. Each output column is computed
        # independently, so every block's values are those of its own linear.
        self.mod_all = QLinear(torch.cat([bw.mod.q for bw in self.blocks]),
                               torch.cat([bw.mod.s for bw in self.blocks]),
                               torch.cat([bw.mod.bias for bw in self.blocks]))
        n6 = 6 * cfg.hidden
        for i, bw in enumerate(self.blocks):
            bw.mod = _rows(self.mod_all, i * n6, (i + 1) * n6)
        cos, sin = rope_freqs(cfg.rope_dims, cfg.theta, *cfg.grid, t_offset=cfg.t_offset, device=self.device)
        lo, hi = self.sp.shard(cfg.tokens)
        self.rope = (cos[lo:hi].contiguous(), sin[lo:hi].contiguous())
        self.token_range = (lo, hi)
        # SMs the GEMMs leave to the K/V all-gathers under sequence parallelism (applied only while forward runs)
        self.sm_reserve = int(os.environ.get("HN_SP_GEMM_SM_RESERVE", str(SP_GEMM_SM_RESERVE))) \
            if (self.sp.world > 1 and self.device.type == "cuda") else 0

    def replica(self, sp=None, grid=None, t_offset=None):
        """The same model (weights shared, not copied) over another partition `sp` of the sequence (e.g. the whole
        sequence on one GPU, to check a sequence-parallel run against) and/or another token grid starting at
        frame `t_offset` (e.g. a later segment, or the frames of its history)."""
        import copy
        import dataclasses
        other = copy.copy(self)
        other.sp = sp = sp or self.sp
        changes = {k: v for k, v in (("grid", grid), ("t_offset", t_offset)) if v is not None}
        other.cfg = dataclasses.replace(self.cfg, **changes)
        other.sm_reserve = self.sm_reserve if sp is self.sp else 0
        cos, sin = rope_freqs(other.cfg.rope_dims, other.cfg.theta, *other.cfg.grid, t_offset=other.cfg.t_offset,
                              device=self.device)
        lo, hi = sp.shard(other.cfg.tokens)
        other.rope = (cos[lo:hi].contiguous(), sin[lo:hi].contiguous())
        other.token_range = (lo, hi)
        return other

    def modulations(self, vec):
        """All blocks' Modulate(vec) in one launch pair (quantize + GEMM): [B, blocks * 6D] bf16."""
        return self.ops.linear(self.ops.silu(vec), self.mod_all)

    def forward(self, x, vec, trace=None, history=None, capture=None):
        """This rank's tokens after all blocks. `history`: one (hk_q, hk_s, hv_q, hv_s) int8 cache per block (see
        block_forward); `capture`, when a list, receives one such cache per block for this rank's tokens."""
        if not self.sm_reserve:
            return self._forward(x, vec, trace, history, capture)
        # the library's SM reserve is process-wide: set it for this step only and put the caller's value back
        from . import _lib
        prev = _lib.lib.hn_get_gemm_sm_reserve()
        _lib.check(_lib.lib.hn_set_gemm_sm_reserve(self.sm_reserve), "hn_set_gemm_sm_reserve")
        try:
            return self._forward(x, vec, trace, history, capture)
        finally:
            _lib.lib.hn_set_gemm_sm_reserve(prev)

    def _forward(self, x, vec, trace=None, history=None, capture=None):
        mods = self.modulations(vec)
        n6 = 6 * self.cfg.hidden
        nb = len(self.blocks)
        x_q = None
        for i, w in enumerate(self.blocks):
            # every block but the last ends with its residual fused into the next block's LN + quantization
            last = i == nb - 1
            r = block_forward(self.cfg, w, x, vec, self.rope, self.sp, self.ops,
                              trace=trace if (trace is not None and last) else None,
                              mods=mods[:, i * n6:(i + 1) * n6], x_q=x_q,
                              next_mods=None if last else mods[:, (i + 1) * n6:(i + 2) * n6],
                              history=None if history is None else history[i], capture=capture)
            x, x_q = (r, None) if last else r
        return x

    __call__ = forward
