"""hy_nomas_b200 - the quantized DiT linear path of ComfyUI-Hy-Nomas, rebuilt for B200 (sm_100a).

Modules mirror the reference package: `kernels` (hy_nomas/kernels.py), `fused` (hy_nomas/fused.py), `ops`
(hy_nomas/ops.py); `dit` is the synthetic DiT block/step built from them, with sequence parallelism.
All compute runs in libhynomas_b200.so through the C ABI of include/hynomas_b200.h.
"""
__all__ = ["kernels", "fused", "ops"]
