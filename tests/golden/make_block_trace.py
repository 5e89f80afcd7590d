"""Record the reference's own DoubleStreamBlock driving THIS repository's kernels/fused modules - the drop-in trace.

Run where a checkout of the reference repository is available, its directory given by HY_NOMAS_REFERENCE:

    HY_NOMAS_REFERENCE=<checkout> python tests/golden/make_block_trace.py

What runs: the reference's hy_nomas/model.py DoubleStreamBlock.forward (model.py:288-303: both streams, joint
attention, `_qkv` / `_post` / `MLP.forward_int8`) over the reference's hy_nomas/ops.py NomasOps.Linear (its
`_load_from_state_dict`, `forward_comfy_cast_weights` int8 dispatch, `fast_int8` and `int8_weights`,
ops.py:129-191), in HY_NOMAS_MATMUL=int8 mode. ComfyUI is absent, so its few entry points are stubbed (a cast
context that hands the weight and bias over, a QuantizedTensor carrying codes and scales, attention = torch
SDPA as ComfyUI's pytorch backend), and the inputs are tensors that report `is_cuda` so that the reference takes
its GPU-only fused path on this CPU-only machine.

In place of the reference's `kernels` and `fused` modules (model.py:34, ops.py:172) sits a recorder with the
interface of hy_nomas_b200.kernels / hy_nomas_b200.fused. Each call is first bound to the signature of the
hy_nomas_b200 function of the same name (a call that the drop-in could not take fails here), then answered by
the CPU oracle (the same arithmetic as the CUDA kernels), and recorded: name, arguments, result. The trace and
the block's final outputs go to tests/golden/double_stream_block.npz (+ .json); tests/test_gpu_dropin.py replays
every recorded call through the CUDA path and compares the results bit for bit. Weights are not stored: both
sides regenerate them from tests/dropin_block.py's seed.
"""
import contextlib
import inspect
import json
import os
import sys
import types

import numpy as np
import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
for p in (ROOT, os.path.join(ROOT, "comfyui-hy-nomas_b200"), os.path.join(ROOT, "tests"), HERE):
    if p not in sys.path:
        sys.path.insert(0, p)

import dropin_block as B  # noqa: E402
import make_golden  # noqa: E402
from oracle import oracle as O  # noqa: E402


class CudaLike(torch.Tensor):
    """A CPU tensor that answers `is_cuda` with True, so the reference's CUDA-only branches run here."""

    @property
    def is_cuda(self):
        return True


def plain(t):
    return t.as_subclass(torch.Tensor) if isinstance(t, torch.Tensor) else t


def cudalike(t):
    return t.as_subclass(CudaLike) if isinstance(t, torch.Tensor) else t


def _stubs():
    make_golden._stub_comfy()
    cops, qo = sys.modules["comfy.ops"], sys.modules["comfy.quant_ops"]

    class ManualCastLinear(torch.nn.Module):
        weight_function = []
        bias_function = []

    cops.manual_cast.Linear = ManualCastLinear

    class CastBiasWeightContext:
        """ComfyUI's cast-on-use context: the weight as stored, the bias in the input's dtype."""

        def __init__(self, module, input, offloadable=False):
            self.module, self.input = module, input

        def __enter__(self):
            b = self.module.bias
            return self.module.weight, (None if b is None else plain(b).to(self.input.dtype))

        def __exit__(self, *exc):
            return False

    cops.CastBiasWeightContext = CastBiasWeightContext

    class QuantizedTensor(torch.Tensor):
        """ComfyUI's quantized weight: the codes as the tensor, the layout's parameters (scales) beside them."""

        def __new__(cls, qdata, layout, params):
            t = torch.Tensor._make_subclass(cls, qdata)
            t._qdata, t._layout_name, t._params = qdata, layout, params
            return t

        def detach(self):
            return QuantizedTensor(self._qdata, self._layout_name, self._params)

        def requires_grad_(self, requires_grad=True):
            return self

    qo.QuantizedTensor = QuantizedTensor

    def optimized_attention(q, k, v, heads, skip_reshape=False, skip_output_reshape=False, transformer_options=None):
        assert skip_reshape and skip_output_reshape
        return cudalike(F.scaled_dot_product_attention(plain(q), plain(k), plain(v)))

    sys.modules["comfy.ldm.modules.attention"].optimized_attention = optimized_attention
    comfy = sys.modules["comfy"]
    comfy.ldm = sys.modules["comfy.ldm"]
    comfy.ldm.modules = sys.modules["comfy.ldm.modules"]
    comfy.ldm.modules.attention = sys.modules["comfy.ldm.modules.attention"]


class Recorder:
    """Stands in for hy_nomas.kernels and hy_nomas.fused; see the module docstring."""

    def __init__(self, weights):
        self.calls = []
        self.arrays = {}
        self.weight_keys = {}   # the regenerated weights are recognised by storage, shape and dtype
        for name, (q, s, bias) in weights.items():
            for part, t in (("q", q), ("s", s), ("bias", bias)):
                self.weight_keys[self._key(t)] = f"w:{name}:{part}"

    @staticmethod
    def _key(t):
        return t.data_ptr(), tuple(t.shape), tuple(t.stride()), t.dtype

    def _arg(self, v, tag):
        if isinstance(v, torch.Tensor):
            v = plain(v)
            key = self.weight_keys.get(self._key(v))
            if key is None:
                key = tag
                if v.dtype == torch.bfloat16:
                    self.arrays[key] = v.contiguous().view(torch.int16).numpy().view(np.uint16)
                else:
                    self.arrays[key] = v.contiguous().numpy()
            return {"tensor": key, "dtype": str(v.dtype).replace("torch.", ""), "shape": list(v.shape),
                    "stride": list(v.stride())}
        if isinstance(v, (tuple, list)):
            return {"seq": [self._arg(x, f"{tag}.{i}") for i, x in enumerate(v)]}
        if isinstance(v, torch.dtype):
            return {"dtype_value": str(v).replace("torch.", "")}
        return {"value": v}

    def record(self, name, args, kwargs, result):
        i = len(self.calls)
        self.calls.append({"name": name, "args": [self._arg(a, f"c{i}.a{j}") for j, a in enumerate(args)],
                           "kwargs": {k: self._arg(v, f"c{i}.k.{k}") for k, v in kwargs.items()},
                           "result": self._arg(result, f"c{i}.r")})
        return result


def _bf16(a):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(torch.bfloat16)


def _np(t):
    return plain(t).detach().float().numpy()


def oracle_modules(rec):
    """Module objects with hy_nomas_b200's kernels / fused interface: every call is bound, as the reference made
    it, to the signature of the hy_nomas_b200 function of that name, answered by the oracle and recorded."""
    from hy_nomas_b200 import fused as hf, kernels as hk
    kmod, fmod = types.ModuleType("hy_nomas.kernels"), types.ModuleType("hy_nomas.fused")
    kmod.GROUP, kmod.EPILOGUES = hk.GROUP, hk.EPILOGUES
    fmod.ENABLED = True

    def recorded(module, api, impl):
        sig = inspect.signature(api)
        name = f"{module}.{api.__name__}"

        def call(*args, **kwargs):
            bound = sig.bind(*args, **kwargs)     # raises TypeError if the drop-in could not take this call
            bound.apply_defaults()
            return rec.record(name, args, kwargs, impl(**bound.arguments))
        return call

    def block_gemm(qa, sa, qw, sw, bias=None, out_dtype=torch.bfloat16, kind="int8", epilogue=None, out=None):
        b = None if bias is None else _np(bias)
        r = O.block_gemm(plain(qa).numpy(), _np(sa), plain(qw).numpy(), _np(sw), b, epilogue=epilogue)
        if epilogue == "gelu_quant":
            _, qh, qs = r
            return cudalike(torch.from_numpy(qh)), cudalike(torch.from_numpy(qs))
        return cudalike(_bf16(O.round_bf16(r) if epilogue is None else r).to(out_dtype))

    def adaln_quant(x, shift, scale, eps=1e-6):
        q, s = O.adaln_quant(_np(x), _np(shift), _np(scale), eps)
        return cudalike(torch.from_numpy(q)), cudalike(torch.from_numpy(s))

    def int8_g128_linear(x, qw, sw, bias=None):
        shape = x.shape
        q, s = O.quantize_activations(_np(x).reshape(-1, shape[-1]))
        r = O.block_gemm(q.view(np.int8), s, plain(qw).numpy(), _np(sw), None if bias is None else _np(bias))
        return cudalike(_bf16(O.round_bf16(r)).to(x.dtype).reshape(*shape[:-1], plain(qw).shape[0]))

    def adaln(x, shift, scale, eps=1e-6):
        return cudalike(_bf16(O.adaln(_np(x), _np(shift), _np(scale), eps)))

    def qk_norm_rope(x, weight, rope=None, eps=1e-6, out=None):
        rp = None if rope is None else (_np(rope[0]), _np(rope[1]))
        return cudalike(_bf16(O.qk_norm_rope(_np(x), _np(weight), rp, eps)))

    def gated_residual(x, y, gate):
        return cudalike(_bf16(O.round_bf16(O.gated_residual(_np(x), _np(y), _np(gate)))))

    kmod.block_gemm = recorded("kernels", hk.block_gemm, block_gemm)
    kmod.adaln_quant = recorded("kernels", hk.adaln_quant, adaln_quant)
    kmod.int8_g128_linear = recorded("kernels", hk.int8_g128_linear, int8_g128_linear)
    fmod.available = lambda x: x.dtype == torch.bfloat16
    fmod.adaln = recorded("fused", hf.adaln, adaln)
    fmod.qk_norm_rope = recorded("fused", hf.qk_norm_rope, qk_norm_rope)
    fmod.gated_residual = recorded("fused", hf.gated_residual, gated_residual)
    return kmod, fmod


def main():
    ref = make_golden.reference_dir()
    _stubs()
    linears, norms = B.make_weights()
    rec = Recorder(linears)
    kmod, fmod = oracle_modules(rec)
    sys.modules["hy_nomas.kernels"], sys.modules["hy_nomas.fused"] = kmod, fmod
    os.environ["HY_NOMAS_MATMUL"] = "int8"
    sys.path.insert(0, ref)
    from hy_nomas import model, ops  # noqa: E402  (the reference's own modules)
    assert model.kernels is kmod and model.fused is fmod

    block = model.DoubleStreamBlock(B.HIDDEN, B.HEADS, B.MLP_RATIO, ops.NomasOps.with_matmul("int8"),
                                    dtype=torch.bfloat16)
    state = {}
    for name, (q, s, bias) in linears.items():
        state[name + ".weight_q"], state[name + ".weight_scale"], state[name + ".bias"] = q, s, bias
    state.update(norms)
    missing, unexpected = block.load_state_dict(state, strict=False)
    assert not unexpected, unexpected
    assert not [k for k in missing if not k.endswith("weight")] and all(
        isinstance(getattr(m, "weight"), ops.QuantizedTensor) for m in ops.quantized_linears(block)), missing
    # the codes the Linear hands to the kernels are the very tensors the recorder knows by name
    for name, (q, s, bias) in linears.items():
        lin = block.get_submodule(name)
        lin.weight._qdata, lin.weight._params = q, type(lin.weight._params)(scale=s, orig_dtype=torch.bfloat16,
                                                                           orig_shape=tuple(q.shape))
        lin.bias = torch.nn.Parameter(bias, requires_grad=False)
    img, txt, vec = (cudalike(t) for t in B.make_inputs())
    t, h, w = B.GRID
    rope = model.rope_freqs(list(B.ROPE_DIMS), B.THETA, t, h, w)
    rope = tuple(cudalike(r.contiguous()) for r in rope)
    plan = model.AttentionPlan(img.shape[1], txt.shape[1])
    with torch.no_grad():
        img_out, txt_out = block(img, txt, vec, rope, None, plan, {})
    names = [c["name"] for c in rec.calls]
    for needed in ("kernels.adaln_quant", "kernels.block_gemm", "fused.qk_norm_rope", "kernels.int8_g128_linear",
                   "fused.gated_residual"):
        assert needed in names, (needed, names)
    rec.arrays["out.img"] = plain(img_out).contiguous().view(torch.int16).numpy().view(np.uint16)
    rec.arrays["out.txt"] = plain(txt_out).contiguous().view(torch.int16).numpy().view(np.uint16)
    np.savez_compressed(os.path.join(HERE, "double_stream_block.npz"), **rec.arrays)
    with open(os.path.join(HERE, "double_stream_block.json"), "w") as f:
        json.dump({"calls": rec.calls, "reference": "hy_nomas/model.py DoubleStreamBlock.forward (288-303), "
                   "hy_nomas/ops.py NomasOps.Linear (129-191), HY_NOMAS_MATMUL=int8"}, f, indent=1)
    print(f"recorded {len(rec.calls)} calls: " + ", ".join(f"{n} x{names.count(n)}" for n in sorted(set(names))))


if __name__ == "__main__":
    main()
