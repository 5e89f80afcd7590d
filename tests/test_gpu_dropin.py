"""The reference's own DoubleStreamBlock, replayed through the CUDA path (the drop-in proof).

tests/golden/make_block_trace.py ran the reference's hy_nomas/model.py DoubleStreamBlock.forward (both streams,
joint attention) over its hy_nomas/ops.py NomasOps.Linear in int8 mode, with this repository's kernels/fused
interface in place of the reference's modules: every call was bound to the hy_nomas_b200 signature and recorded
with its arguments exactly as the reference passed them, and answered by the CPU oracle. Here each recorded call
is made again, with the same positional and keyword arguments, to hy_nomas_b200 on the GPU, and its result must
equal the recorded one bit for bit (codes, scales, bf16 values). So the reference's block, with these modules
in place of its own, takes exactly the computation recorded in the trace, ending in the recorded block outputs.
"""
import json
import os

import numpy as np
import pytest
import torch

import dropin_block as B
from hn_testutil import ROOT

TRACE = os.path.join(ROOT, "tests", "golden", "double_stream_block")
DTYPES = {"bfloat16": torch.bfloat16, "float32": torch.float32, "int8": torch.int8, "float16": torch.float16}


@pytest.fixture(scope="module")
def trace():
    with open(TRACE + ".json") as f:
        meta = json.load(f)
    return meta["calls"], np.load(TRACE + ".npz")


@pytest.fixture(scope="module")
def weights():
    return B.make_weights()[0]


def _tensor(spec, arrays, weights, device):
    key, dtype = spec["tensor"], DTYPES[spec["dtype"]]
    if key.startswith("w:"):
        _, name, part = key.split(":")
        t = weights[name][("q", "s", "bias").index(part)]
    else:
        a = arrays[key]
        t = torch.from_numpy(a.view(np.int16)).view(torch.bfloat16) if dtype == torch.bfloat16 else torch.from_numpy(a)
    t = t.reshape(spec["shape"]).to(device)
    if list(t.stride()) != spec["stride"]:
        # the reference handed over a strided view (e.g. a chunk of the modulation output): rebuild it
        base = torch.zeros(max(1, sum((n - 1) * s for n, s in zip(spec["shape"], spec["stride"])) + 1),
                           dtype=t.dtype, device=device)
        view = base.as_strided(spec["shape"], spec["stride"])
        view.copy_(t)
        t = view
    return t


def _value(spec, arrays, weights, device):
    if "tensor" in spec:
        return _tensor(spec, arrays, weights, device)
    if "seq" in spec:
        return tuple(_value(s, arrays, weights, device) for s in spec["seq"])
    if "dtype_value" in spec:
        return DTYPES[spec["dtype_value"]]
    return spec["value"]


def _same(got, spec, arrays):
    if "seq" in spec:
        return all(_same(g, s, arrays) for g, s in zip(got, spec["seq"]))
    want = arrays[spec["tensor"]]
    got = got.detach().contiguous().cpu()
    if got.dtype == torch.bfloat16:
        return np.array_equal(got.view(torch.int16).numpy().view(np.uint16), want)
    return np.array_equal(got.numpy(), want)


def test_trace_covers_the_block(trace):
    calls, _ = trace
    names = [c["name"] for c in calls]
    # both streams: each runs adaln_quant twice (qkv, MLP), three q/k/v GEMMs, two QK-norms, the modulation and
    # projection linears through NomasOps.Linear, fc1 (gelu_quant) and fc2, and two gated residuals
    assert names.count("kernels.adaln_quant") == 4 and names.count("fused.qk_norm_rope") == 4
    assert names.count("kernels.block_gemm") == 10 and names.count("kernels.int8_g128_linear") == 4
    assert names.count("fused.gated_residual") == 4
    assert any(c["kwargs"].get("epilogue", {}).get("value") == "gelu_quant" for c in calls)


@pytest.mark.gpu
def test_reference_block_calls_replayed_bit_exact(hn, cuda, trace, weights):
    calls, arrays = trace
    modules = {"kernels": hn.kernels, "fused": hn.fused}
    for i, c in enumerate(calls):
        mod, fn = c["name"].split(".")
        args = [_value(a, arrays, weights, cuda) for a in c["args"]]
        kwargs = {k: _value(v, arrays, weights, cuda) for k, v in c["kwargs"].items()}
        got = getattr(modules[mod], fn)(*args, **kwargs)
        torch.cuda.synchronize()
        assert _same(got, c["result"], arrays), (i, c["name"])
    rc, code = hn.lib.device_error()
    assert rc == 0 and code == 0


def test_block_outputs_are_the_last_residuals(trace):
    """The recorded block outputs (img, txt) are the results of each stream's final gated residual (the image
    stream's _post runs first, model.py:300-302), so the replay reproduces the reference block's outputs."""
    calls, arrays = trace
    residuals = [c for c in calls if c["name"] == "fused.gated_residual"]
    outs = [arrays[residuals[1]["result"]["tensor"]], arrays[residuals[3]["result"]["tensor"]]]
    assert np.array_equal(outs[0], arrays["out.img"].reshape(outs[0].shape))
    assert np.array_equal(outs[1], arrays["out.txt"].reshape(outs[1].shape))
