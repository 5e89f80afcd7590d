"""The DiT block's ops on the CPU oracle - test infrastructure.

`OracleOps` has the methods of `hy_nomas_b200.dit.CudaOps` and computes each with the oracle (oracle/oracle.py)
on CPU tensors, so `block_forward` / `SyntheticDiT` can run on CPU: the host-side sequence-parallel tests run it
under gloo, and the GPU parity tests use it as the per-stage reference. Attention is computed row by row in
float64 and rounded to bf16 once, so a query's result does not depend on how many queries share the call.
"""
import numpy as np
import torch

from oracle import oracle as O


def _bf16(a):
    """bf16-valued float32 numpy -> bf16 torch (exact)."""
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(torch.bfloat16)


def _np(t):
    return t.detach().float().cpu().numpy()


class OracleOps:
    @staticmethod
    def linear(x2, w):
        """block_linear (hy_nomas/kernels.py:210-222): group quantization, then the GEMM with per-channel scales."""
        q, s = O.quantize_activations(_np(x2))
        out = O.block_gemm(q.view(np.int8), s, w.q.cpu().numpy(), _np(w.s), _np(w.bias), sa_mode="group",
                           sw_mode="row")
        return _bf16(O.round_bf16(out))

    @staticmethod
    def adaln_quant(x, shift, scale):
        q, s = O.adaln_quant(_np(x), _np(shift), _np(scale))
        return torch.from_numpy(q), torch.from_numpy(s)

    @staticmethod
    def gemm(qa, sa, w, epilogue=None, out=None):
        qa_n = qa.cpu().numpy()
        sa_n = _np(sa)
        sa_mode = "row" if sa_n.ndim == 1 or (sa_n.shape[1] == 1 and qa_n.shape[1] != 128) else "group"
        r = O.block_gemm(qa_n, sa_n.reshape(sa_n.shape[0], -1) if sa_mode == "group" else sa_n.reshape(-1),
                         w.q.cpu().numpy(), _np(w.s), _np(w.bias), epilogue=epilogue, sa_mode=sa_mode, sw_mode="row")
        if epilogue == "gelu_quant":
            _, qh, qs = r
            return torch.from_numpy(qh), torch.from_numpy(qs)
        y = _bf16(O.round_bf16(r) if epilogue is None else r)
        if out is not None:
            out.copy_(y)
            return out
        return y

    @staticmethod
    def qk_norm_rope2(q, k, wq, wk, rope, out):
        cos, sin = (None, None) if rope is None else (_np(rope[0]), _np(rope[1]))
        rp = None if rope is None else (cos, sin)
        yq = _bf16(O.qk_norm_rope(_np(q), _np(wq), rp))
        yk = _bf16(O.qk_norm_rope(_np(k), _np(wk), rp))
        out[0].copy_(yq)
        out[1].copy_(yk)
        return out

    @staticmethod
    def qk_norm_rope(x, w, rope, out):
        rp = None if rope is None else (_np(rope[0]), _np(rope[1]))
        out.copy_(_bf16(O.qk_norm_rope(_np(x), _np(w), rp)))
        return out

    @staticmethod
    def gated_residual_adaln_quant(x, y, gate, shift, scale):
        xo, q, s = O.gated_residual_adaln_quant(_np(x), _np(y), _np(gate), _np(shift), _np(scale))
        return _bf16(xo), torch.from_numpy(q), torch.from_numpy(s)

    @staticmethod
    def qk_norm_rope_kv(x, w, rope, out):
        """QK-norm + RoPE into `out`, then the KV quantizer of world.quantize_kv on that output."""
        OracleOps.qk_norm_rope(x, w, rope, out)
        b, l, h, d = out.shape
        return OracleOps.quantize_kv(out.reshape(b * l, h, d))

    @staticmethod
    def quantize_kv(x):
        q, s = O.quantize_kv(_np(x).reshape(-1, x.shape[-2], x.shape[-1]))
        return torch.from_numpy(q).reshape(x.shape), torch.from_numpy(s).reshape(*x.shape[:-1], 1)

    @staticmethod
    def dequantize_kv(q, s, out):
        y = O.dequantize_kv(q.cpu().numpy().reshape(-1, q.shape[-1]), _np(s).reshape(-1))
        out.copy_(_bf16(y).reshape(out.shape))
        return out

    @staticmethod
    def gated_residual(x, y, gate):
        return _bf16(O.round_bf16(O.gated_residual(_np(x), _np(y), _np(gate))))

    @staticmethod
    def silu(v):
        return torch.nn.functional.silu(v.cpu())

    @staticmethod
    def attention(q, k, v):
        """softmax(q k^T / sqrt(D)) v per (batch, head, query) in float64 -> bf16 [B, Lq, H, D]."""
        qf = q.double().permute(0, 2, 1, 3)
        kf = k.double().permute(0, 2, 1, 3)
        vf = v.double().permute(0, 2, 1, 3)
        scores = torch.einsum("bhqd,bhkd->bhqk", qf, kf) / np.sqrt(q.shape[-1])
        p = torch.softmax(scores, dim=-1)
        out = torch.einsum("bhqk,bhkd->bhqd", p, vf)
        return out.permute(0, 2, 1, 3).to(torch.bfloat16)
