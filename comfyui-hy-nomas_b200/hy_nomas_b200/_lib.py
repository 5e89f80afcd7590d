"""ctypes binding of libhynomas_b200.so (the C ABI declared in include/hynomas_b200.h).

The library is the only compute path: there is no Triton, no torch or CPU fallback. If the shared object
is missing, importing this module raises; if a call fails, the C status becomes a RuntimeError carrying
hn_last_error(). Tensors are passed as raw device pointers; every launch goes on torch's current stream
of the tensor's device (the library makes that stream's device current for the call).
"""
import ctypes
import os

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libhynomas_b200.so")

HN_OK = 0
STATUS = {0: "HN_OK", 1: "HN_ERR_SHAPE", 2: "HN_ERR_ALIGN", 3: "HN_ERR_ARCH", 4: "HN_ERR_CUDA", 5: "HN_ERR_ARG",
          6: "HN_ERR_TIMEOUT", 7: "HN_ERR_UNSUPPORTED"}

DTYPE = {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2, torch.int32: 3}
KIND = {"int8": 0, "fp8": 1}
SCALE_MODE = {"group": 0, "row": 1, "block": 2}

# name -> argtypes (all entry points return int)
_V, _I64, _I32, _F32, _U32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float, ctypes.c_uint32
SIGNATURES = {
    "hn_abi_version": [],
    "hn_num_sms": [],
    "hn_set_gemm_sm_reserve": [ctypes.c_int],
    "hn_get_gemm_sm_reserve": [],
    "hn_device_error": [_V, ctypes.POINTER(ctypes.c_int)],
    "hn_selftest_wait_timeout": [_U32, _V],
    "hn_quant_act": [_V, _I64, _I32, _I64, _I64, _I32, _I32, _V, _I64, _V, _I64, _I64, _V],
    "hn_block_gemm": [_V, _I64, _V, _I64, _I64, _I32, _V, _I64, _V, _I64, _I64, _I32, _V, _I32, _V, _I64, _I32,
                      _V, _I64, _I64, _I64, _I64, _I64, _I32, _I32, _V],
    "hn_adaln_quant": [_V, _V, _V, _I64, _I64, _I64, _F32, _V, _V, _I64, _I64, _V],
    "hn_adaln": [_V, _V, _V, _I64, _I64, _I64, _F32, _V, _V],
    "hn_qk_norm_rope": [_V, _I64, _V, _V, _V, _I64, _I64, _I64, _I64, _F32, _V, _V],
    "hn_qk_norm_rope2": [_V, _V, _I64, _V, _V, _V, _V, _I64, _I64, _I64, _I64, _F32, _V, _V, _V],
    "hn_gated_residual": [_V, _V, _V, _I64, _I64, _I64, _V, _V],
    "hn_gated_residual_adaln_quant": [_V, _V, _V, _V, _V, _I64, _I64, _I64, _F32, _V, _V, _V, _I64, _I64, _V],
    "hn_pixelumm_qk": [_V, _I64, _V, _V, _V, _V, _I64, _I64, _I64, _F32, _V, _V],
    "hn_quantize_kv": [_V, _I64, _I64, _V, _V, _V],
    "hn_dequantize_kv": [_V, _V, _I64, _I64, _V, _V],
    "hn_qk_norm_rope_kv": [_V, _I64, _V, _V, _V, _I64, _I64, _I64, _I64, _F32, _V, _V, _V, _V],
    "hn_quantize_fp8_block": [_V, _I32, _I64, _I64, _V, _V, _V],
    "hn_rmsnorm_quant": [_V, _I64, _V, _I64, _I64, _F32, _I32, _V, _I64, _V, _I64, _I64, _V],
    "hn_silu_mul_quant": [_V, _I64, _V, _I64, _I64, _I64, _I32, _V, _I64, _V, _I64, _I64, _V],
    "hn_attention": [_V, _I64, _I64, _I64, _V, _I64, _I64, _I64, _V, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64,
                     _F32, _V, _I64, _I64, _I64, _V, _V, _V],
    "hn_attn_merge": [_V, _V, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _V, _I64, _I64, _I64,
                      _V, _V, _V],
    "hn_ipc_export": [_V, _V, ctypes.POINTER(ctypes.c_int64)],
    "hn_ipc_import": [_V, ctypes.POINTER(ctypes.c_void_p)],
    "hn_ipc_close": [_V],
    "hn_peer_push": [_V, _V, _I64, _V, _U32, _V],
    "hn_peer_push2d": [_V, _I64, _V, _I64, _I64, _I64, _V, _U32, _V],
    "hn_wait_flags": [_V, _I64, _I64, _I64, _I64, _U32, _U32, _V],
}


class StreamArg(ctypes.c_void_p):
    """A cudaStream_t argument that also carries the device of the tensors the call is for."""
    device = None


class _Library:
    """The loaded library; an entry point whose last argument is a StreamArg runs with that stream's device
    current. The library itself makes a non-NULL stream's device current, but torch's default stream is the
    legacy NULL stream, which stands for the current device whichever it is."""

    def __init__(self, cdll):
        self._cdll = cdll

    def __getattr__(self, name):
        fn = getattr(self._cdll, name)

        def call(*args):
            s = args[-1] if args else None
            if isinstance(s, StreamArg) and s.device is not None and s.device != torch.cuda.current_device():
                with torch.cuda.device(s.device):
                    return fn(*args)
            return fn(*args)
        call.__name__ = name
        setattr(self, name, call)
        return call


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: build it with `python -m hy_nomas_b200.build` "
                          "(this package has no fallback path)")
    lib = ctypes.CDLL(LIB_PATH)
    lib.hn_last_error.restype = ctypes.c_char_p
    lib.hn_last_error.argtypes = []
    for name, args in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = ctypes.c_int
    return _Library(lib)


lib = _load()


def last_error():
    return lib.hn_last_error().decode(errors="replace")


calls = 0   # library calls made by this process (each launches at most one kernel); read by bench.py


def check(rc, what, launches=1):
    """Raise on a failed library call; `launches` = the kernels the call starts (0 for host-only entries)."""
    global calls
    calls += launches
    if rc != HN_OK:
        raise RuntimeError(f"{what} failed with {STATUS.get(rc, rc)}: {last_error()}")


def ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def dense(t):
    """`t` as a contiguous tensor whose data starts on a 16-byte boundary (the vector and TMA paths of the
    library need it). Copies only when needed; a contiguous view at an odd offset is copied too, since
    .contiguous() would hand back the same misaligned pointer."""
    t = t.contiguous()
    return t if t.data_ptr() % 16 == 0 else t.clone()


def stream_of(t):
    """torch's current stream on the tensor's device, as a cudaStream_t value that remembers that device."""
    s = StreamArg(torch.cuda.current_stream(t.device).cuda_stream)
    s.device = t.device.index
    return s


def require_cuda(*tensors):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError("hy_nomas_b200 kernels run on CUDA tensors only (there is no CPU path); "
                               f"got a tensor on {t.device}")


def group_scales(rows, groups, device):
    """Scale storage for [rows, groups] in group-major layout (each group's rows contiguous, rows padded to a
    multiple of 4): returns (the [rows, groups] view handed to callers, row stride, group stride)."""
    padded = (rows + 3) // 4 * 4
    store = torch.empty((groups, padded), device=device, dtype=torch.float32)
    view = store[:, :rows].t()
    return view, 1, padded


def scale_strides(s):
    """(row stride, group stride) of a [rows, groups] or [rows] scale tensor, in elements."""
    if s.dim() == 1:
        return s.stride(0), 0
    return s.stride(0), s.stride(1)


def device_error(stream=None):
    """Synchronize `stream` and return (and clear) the device error word of the bounded waits."""
    code = ctypes.c_int(0)
    stream = stream if stream is not None else torch.cuda.current_stream()
    with torch.cuda.device(stream.device):     # a NULL stream means the current device: make it the stream's
        rc = lib.hn_device_error(ctypes.c_void_p(stream.cuda_stream), ctypes.byref(code))
    return rc, code.value
