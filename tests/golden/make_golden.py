"""Generate the golden vectors of the quantized DiT linear path from the REFERENCE's own code.

Run where a checkout of the reference repository is available, its directory given by HY_NOMAS_REFERENCE:

    HY_NOMAS_REFERENCE=<checkout> python tests/golden/make_golden.py

It writes tests/golden/*.npz. Nothing at test time reads the reference: the tests only read these files.

How the reference is run on a machine without a GPU or ComfyUI:
  * its Triton kernels (hy_nomas/kernels.py, hy_nomas/fused.py) run under the Triton CPU interpreter
    (TRITON_INTERPRET=1), launched through their @triton.jit bodies with the block sizes of one of the
    reference's own autotune configs (kernels.py:57-64);
  * the interpreter's fp32 -> bf16 cast truncates, where the GPU rounds to nearest even, and its
    fp32 -> float8e4nv cast does not carry mantissa overflow into the exponent. Both casts are replaced
    here by the GPU semantics (nearest-even bf16 on the bits; torch's nearest-even e4m3 with
    saturation at +-448, i.e. cvt.rn.satfinite). Every other interpreter operation is untouched
    (numpy float32 arithmetic: IEEE division, 1/np.sqrt for tl.rsqrt, numpy's exp, numpy's sum order);
  * its torch reference functions (model.layer_norm / modulate / RMSNorm / rope_freqs / apply_rope,
    ops.quantize_g128 / dequantize_g128, pixelumm's FP8 block layout, world.quantize_kv / dequantize_kv) run on CPU with
    the `comfy` and `comfy_kitchen` modules stubbed (they are not on this path's arithmetic).
All inputs are seeded (torch.Generator, seeds below). bf16 arrays are stored as uint16 bit patterns,
e4m3 codes as uint8 bytes.
"""
import dataclasses
import os
import sys
import types

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))


def reference_dir():
    """The reference checkout, from HY_NOMAS_REFERENCE (no default: the scripts never guess a path)."""
    ref = os.environ.get("HY_NOMAS_REFERENCE")
    if not ref or not os.path.isdir(os.path.join(ref, "hy_nomas")):
        raise SystemExit("set HY_NOMAS_REFERENCE to a checkout of the ComfyUI-Hy-Nomas repository")
    return ref


def _stub_comfy():
    comfy = types.ModuleType("comfy")
    mm = types.ModuleType("comfy.model_management")
    mm.cast_to = lambda w, dtype=None, device=None, **kw: w.to(dtype=dtype) if dtype is not None else w
    mm.throw_exception_if_processing_interrupted = lambda: None
    cops = types.ModuleType("comfy.ops")

    class _ManualCast:
        class Linear(torch.nn.Module):
            pass

    cops.manual_cast = _ManualCast
    cops.CastBiasWeightContext = None
    qo = types.ModuleType("comfy.quant_ops")
    qo.QuantizedTensor = type("QuantizedTensor", (), {})
    ldm = types.ModuleType("comfy.ldm")
    ldm_mod = types.ModuleType("comfy.ldm.modules")
    attn = types.ModuleType("comfy.ldm.modules.attention")
    attn.optimized_attention = None
    pe = types.ModuleType("comfy.patcher_extension")
    ck = types.ModuleType("comfy_kitchen")
    ckt = types.ModuleType("comfy_kitchen.tensor")

    @dataclasses.dataclass(frozen=True)
    class BaseLayoutParams:
        scale: object = None
        orig_dtype: object = None
        orig_shape: object = None

    ckt.BaseLayoutParams = BaseLayoutParams
    ckt.QuantizedLayout = type("QuantizedLayout", (), {})
    ckt.register_layout_class = lambda name, cls: None
    for name, mod in {"comfy": comfy, "comfy.model_management": mm, "comfy.ops": cops, "comfy.quant_ops": qo,
                      "comfy.ldm": ldm, "comfy.ldm.modules": ldm_mod, "comfy.ldm.modules.attention": attn,
                      "comfy.patcher_extension": pe, "comfy_kitchen": ck, "comfy_kitchen.tensor": ckt}.items():
        sys.modules[name] = mod
    comfy.model_management, comfy.ops, comfy.quant_ops = mm, cops, qo


def _fix_interpreter_casts():
    import triton.language as tl
    from triton.runtime import interpreter as interp
    original = interp._convert_float

    def convert(data, src, dst, rounding_mode):
        if src == tl.float32 and dst == tl.bfloat16:
            a = np.ascontiguousarray(data, dtype=np.float32)
            b = a.view(np.uint32).astype(np.uint64)
            r = ((b + (((b >> 16) & 1) + 0x7FFF)) >> 16) & 0xFFFF
            return r.astype(np.uint16).reshape(a.shape)
        if src == tl.float32 and dst == tl.float8e4nv:
            a = np.clip(np.ascontiguousarray(data, dtype=np.float32), -448.0, 448.0)
            t = torch.from_numpy(a).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
            return t.reshape(a.shape)
        return original(data, src, dst, rounding_mode)

    interp._convert_float = convert


def bits(t):
    """bf16 tensor -> uint16 numpy bit patterns."""
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def main():
    _stub_comfy()
    _fix_interpreter_casts()
    sys.path.insert(0, reference_dir())
    from hy_nomas import fused, kernels, model, ops, pixelumm, world  # noqa: E402

    gen = torch.Generator().manual_seed(0)

    def randn(*shape, scale=1.0):
        return torch.randn(*shape, generator=gen) * scale

    # ---- K1: quantize_activations (kernels.py:22-54), int8 and e4m3 -------------------------------
    m, k = 37, 384
    x = randn(m, k, scale=3.0)
    x[:, torch.randperm(k, generator=gen)[:4]] *= 20.0           # outlier channels
    x[5] = 0.0                                                   # zero row: scale 1, codes 0
    x[6, :128] = 0.0
    x[6, 0] = 127.0                                              # peak 127 -> scale exactly 1.0
    x[6, 1:9] = torch.tensor([2.5, -3.5, 0.5, -0.5, 126.5, -1.5, 4.5, -126.5])   # exact ties
    x[7, 128:256] = 1e-30                                        # tiny values (subnormal e4m3 / int8 scale)
    xb = x.bfloat16()
    rows = 16
    grid = (triton_cdiv(m, rows), k // 128)
    cases = {}
    for kind in ("int8", "fp8"):
        dtype = torch.int8 if kind == "int8" else torch.float8_e4m3fn
        q = torch.empty((m, k), dtype=dtype)
        s = torch.empty((m, k // 128), dtype=torch.float32)
        kernels._quantize_kernel[grid](xb, q, s, m, k, xb.stride(0), q.stride(0), s.stride(0),
                                       IS_INT8=kind == "int8", ROWS=rows)
        cases[f"{kind}_q"] = q.view(torch.uint8).numpy().copy()
        cases[f"{kind}_s"] = s.numpy().copy()
    np.savez_compressed(os.path.join(OUT, "quant_act.npz"), x=bits(xb), **cases)

    # ---- ops.quantize_g128 / dequantize_g128 (ops.py:41-62) --------------------------------------
    w = randn(64, 384, scale=0.02)
    w[3] = 0.0
    qw, sw = ops.quantize_g128(w)
    np.savez_compressed(os.path.join(OUT, "quantize_g128.npz"), w=w.numpy(), q=qw.numpy(), s=sw.numpy(),
                        deq=bits(ops.dequantize_g128(qw, sw)))

    # ---- K2: block_gemm (kernels.py:80-170) ------------------------------------------------------
    m, n, k = 48, 256, 384
    x = randn(m, k, scale=2.0).bfloat16()
    w = randn(n, k, scale=0.02)
    bias = randn(n, scale=0.1).bfloat16()
    qw, sw = ops.quantize_g128(w)
    qa = torch.empty((m, k), dtype=torch.int8)
    sa = torch.empty((m, k // 128), dtype=torch.float32)
    kernels._quantize_kernel[(triton_cdiv(m, 16), k // 128)](x, qa, sa, m, k, x.stride(0), qa.stride(0),
                                                             sa.stride(0), IS_INT8=True, ROWS=16)
    gemm = dict(qa=qa.numpy(), sa=sa.numpy(), qw=qw.numpy(), sw=sw.numpy(), bias=bits(bias))

    def run_gemm(qa_, sa_, qw_, sw_, out, qs, epilogue, is_int8, block_n=128):
        bm = 64
        grid_ = (triton_cdiv(m, bm) * triton_cdiv(n, block_n),)
        kernels._gemm_body[grid_](qa_, qw_, out, sa_, sw_, bias, qs, m, n, k, 64, qa_.stride(0), qw_.stride(0),
                                  out.stride(0), sa_.stride(0), sw_.stride(0), qs.stride(0), HAS_BIAS=True,
                                  IS_INT8=is_int8, EPILOGUE=epilogue, BLOCK_M=bm, BLOCK_N=block_n, GROUP_M=8)

    acc = torch.empty((m, n), dtype=torch.float32)
    run_gemm(qa, sa, qw, sw, acc, acc, 0, True)
    gemm["acc_f32"] = acc.numpy().copy()
    y0 = torch.empty((m, n), dtype=torch.bfloat16)
    run_gemm(qa, sa, qw, sw, y0, y0, 0, True)
    gemm["ep0_bf16"] = bits(y0)
    y1 = torch.empty((m, n), dtype=torch.bfloat16)
    run_gemm(qa, sa, qw, sw, y1, y1, 1, True)
    gemm["ep1_bf16"] = bits(y1)
    q2 = torch.empty((m, n), dtype=torch.int8)
    s2 = torch.empty((m, n // 128), dtype=torch.float32)
    run_gemm(qa, sa, qw, sw, q2, s2, 2, True, block_n=128)
    gemm["ep2_q"], gemm["ep2_s"] = q2.numpy().copy(), s2.numpy().copy()
    # FP8 (pixelumm.py:77-82 weights, K1 e4m3 activations, sw expanded as pixelumm.py:153 does)
    qf, params = pixelumm.NomasFP8Block128Layout.quantize(w)
    sfb = params.scale
    qa8 = torch.empty((m, k), dtype=torch.float8_e4m3fn)
    sa8 = torch.empty((m, k // 128), dtype=torch.float32)
    kernels._quantize_kernel[(triton_cdiv(m, 16), k // 128)](x, qa8, sa8, m, k, x.stride(0), qa8.stride(0),
                                                             sa8.stride(0), IS_INT8=False, ROWS=16)
    sfe = sfb.repeat_interleave(128, dim=0).contiguous()
    acc8 = torch.empty((m, n), dtype=torch.float32)
    run_gemm(qa8, sa8, qf, sfe, acc8, acc8, 0, False)
    gemm.update(x=bits(x), fp8_qa=qa8.view(torch.uint8).numpy().copy(), fp8_sa=sa8.numpy(),
                fp8_qw=qf.view(torch.uint8).numpy().copy(), fp8_sw_block=sfb.numpy(), fp8_acc_f32=acc8.numpy(),
                fp8_deq_w=bits(pixelumm.dequantize_fp8_block(qf, sfb)), w=w.numpy())
    np.savez_compressed(os.path.join(OUT, "block_gemm.npz"), **gemm)

    # ---- K3 / K4: adaln_quant (kernels.py:173-207), adaln (fused.py:37-62) ------------------------
    ada = {}
    for tag, (b, l, d) in {"d2048": (2, 20, 2048), "d4096": (1, 12, 4096)}.items():
        x = (randn(b, l, d, scale=3.0)).bfloat16()
        shift = randn(b, d).bfloat16()
        scale = randn(b, d).bfloat16()
        q = torch.empty((b * l, d), dtype=torch.int8)
        s = torch.empty((b * l, d // 128), dtype=torch.float32)
        kernels._adaln_quant_kernel[(b * l,)](x, shift, scale, q, s, l, d, 1e-6, GROUPS=d // 128)
        y = torch.empty((b, l, d), dtype=torch.bfloat16)
        fused._adaln_kernel[(b * l,)](x, shift, scale, y, l, d, 1e-6, BLOCK=d)
        ref = model.modulate(model.layer_norm(x), shift, scale).to(torch.bfloat16)
        ada.update({f"{tag}_x": bits(x), f"{tag}_shift": bits(shift), f"{tag}_scale": bits(scale),
                    f"{tag}_q": q.numpy().copy(), f"{tag}_s": s.numpy().copy(), f"{tag}_y": bits(y),
                    f"{tag}_torch_y": bits(ref)})
    np.savez_compressed(os.path.join(OUT, "adaln.npz"), **ada)

    # ---- K5: qk_norm_rope (fused.py:65-105) vs RMSNorm + apply_rope (model.py:89-138) -------------
    b, l, h, d = 2, 24, 4, 128
    lin = randn(b, l, h * d, scale=5.0).bfloat16()
    x = lin.view(b, l, h, d)
    norm = model.RMSNorm(d).bfloat16()
    with torch.no_grad():
        norm.weight.copy_(torch.rand(d, generator=gen) + 0.5)
    cos, sin = model.rope_freqs([16, 56, 56], 256, 2, 3, 4)
    yr = torch.empty((b, l, h, d), dtype=torch.bfloat16)
    yp = torch.empty((b, l, h, d), dtype=torch.bfloat16)
    wq = norm.weight.detach().bfloat16().contiguous()
    fused._qk_norm_rope_kernel[(b * l * h,)](x, wq, cos, sin, yr, h, l, x.stride(1), 1e-6, ROPE=True, HALF=d // 2)
    fused._qk_norm_rope_kernel[(b * l * h,)](x, wq, yp, yp, yp, h, l, x.stride(1), 1e-6, ROPE=False, HALF=d // 2)
    with torch.no_grad():
        t_plain = norm(x).to(torch.bfloat16)
        t_rope = model.apply_rope(t_plain, cos, sin)
    c10, s10 = model.rope_freqs([16, 56, 56], 10000, 2, 2, 3)
    np.savez_compressed(os.path.join(OUT, "qk_norm_rope.npz"), x=bits(x), w=bits(wq), cos=cos.numpy(),
                        sin=sin.numpy(), y_rope=bits(yr), y_plain=bits(yp), torch_rope=bits(t_rope),
                        torch_plain=bits(t_plain), cos_t10000=c10.numpy(), sin_t10000=s10.numpy())

    # ---- K6: gated_residual (fused.py:108-128) vs x + y * gate (model.py:284) ---------------------
    b, l, d = 2, 33, 256
    x = randn(b, l, d).bfloat16()
    y = randn(b, l, d).bfloat16()
    g = randn(b, d).bfloat16()
    out = torch.empty((b, l, d), dtype=torch.bfloat16)
    fused._gated_residual_kernel[(b * l,)](x, y, g, out, l, d, BLOCK=d)
    np.savez_compressed(os.path.join(OUT, "gated_residual.npz"), x=bits(x), y=bits(y), g=bits(g), out=bits(out),
                        torch_out=bits(x + y * g.unsqueeze(1)))

    # ---- K7: pixelumm_qk (fused.py:131-186) ------------------------------------------------------
    n, h, d = 20, 4, 128
    x = randn(1, n, h, d, scale=2.0).bfloat16()
    wt = (torch.rand(d // 2, generator=gen) + 0.5).bfloat16()
    whw = (torch.rand(d // 2, generator=gen) + 0.5).bfloat16()
    ang = torch.rand(n, d, generator=gen) * 6.283
    cos, sin = ang.cos(), ang.sin()
    yk = torch.empty((1, n, h, d), dtype=torch.bfloat16)
    fused._pixelumm_qk_kernel[(n * h,)](x, wt, whw, cos, sin, yk, h, x.stride(1), 1e-6, D=d)
    np.savez_compressed(os.path.join(OUT, "pixelumm_qk.npz"), x=bits(x), wt=bits(wt), whw=bits(whw), cos=cos.numpy(),
                        sin=sin.numpy(), y=bits(yk))

    # ---- world.quantize_kv (world.py:83-90) ------------------------------------------------------
    x = randn(12, 4, 128, scale=2.0).bfloat16()
    x[0, 0] = 0.0
    qk, sk = world.quantize_kv(x)
    yk = world.dequantize_kv(qk, sk)   # world.py:93-94
    np.savez_compressed(os.path.join(OUT, "quantize_kv.npz"), x=bits(x), q=qk.numpy(), s=sk.numpy(), y=bits(yk))
    print("golden vectors written to", OUT)


def triton_cdiv(a, b):
    return (a + b - 1) // b


if __name__ == "__main__":
    main()
