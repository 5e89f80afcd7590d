"""The C-ABI library: it loads, exports every entry point include/hynomas_b200.h declares, and rejects bad
arguments on the host before touching a GPU. No kernel is launched here (CPU only)."""
import ctypes
import os
import re

import pytest
import torch

from hn_testutil import ROOT

HEADER = os.path.join(ROOT, "include", "hynomas_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^(?:int|const char \*)\s*(hn_\w+)\(", text, flags=re.M)))


def test_header_declares_the_path():
    syms = declared_symbols()
    for name in ("hn_quant_act", "hn_block_gemm", "hn_adaln_quant", "hn_adaln", "hn_qk_norm_rope",
                 "hn_gated_residual", "hn_gated_residual_adaln_quant", "hn_pixelumm_qk", "hn_last_error"):
        assert name in syms


def test_library_exports_every_declared_symbol(hn):
    lib = ctypes.CDLL(hn.lib.LIB_PATH)
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, missing
    assert set(hn.lib.SIGNATURES) | {"hn_last_error"} == set(declared_symbols())


def test_abi_version_and_no_device(hn):
    assert hn.lib.lib.hn_abi_version() == 1
    n = hn.lib.lib.hn_num_sms()
    assert n == (torch.cuda.get_device_properties(0).multi_processor_count if torch.cuda.is_available() else 0)


def test_gemm_sm_reserve_range(hn):
    L = hn.lib.lib
    assert L.hn_set_gemm_sm_reserve(-1) == 5 and L.hn_set_gemm_sm_reserve(65) == 5
    assert L.hn_set_gemm_sm_reserve(16) == 0 and L.hn_get_gemm_sm_reserve() == 16
    assert L.hn_set_gemm_sm_reserve(0) == 0 and L.hn_get_gemm_sm_reserve() == 0


def test_dense_realigns_misaligned_views(hn):
    """A contiguous view at an odd offset keeps its pointer under .contiguous(); dense() copies it to an aligned
    allocation, so the wrappers never hand the library a misaligned input."""
    base = torch.arange(64, dtype=torch.bfloat16)
    view = base[3:3 + 40]
    assert view.is_contiguous() and view.data_ptr() % 16 != 0
    d = hn.lib.dense(view)
    assert d.data_ptr() % 16 == 0 and torch.equal(d, view)
    aligned = base[8:48]
    assert hn.lib.dense(aligned).data_ptr() == aligned.data_ptr()


FAKE = ctypes.c_void_p(0x10000)   # never dereferenced: every call below fails validation first


def test_validation_errors_before_launch(hn):
    L = hn.lib.lib
    assert L.hn_quant_act(None, 128, 0, 4, 128, 0, 0, FAKE, 128, FAKE, 1, 1, None) == 5      # null x
    assert b"null" in L.hn_last_error()
    assert L.hn_quant_act(FAKE, 100, 0, 4, 100, 0, 0, FAKE, 100, FAKE, 1, 1, None) == 1      # K % 128
    assert L.hn_quant_act(FAKE, 128, 9, 4, 128, 0, 0, FAKE, 128, FAKE, 1, 1, None) == 5      # dtype
    assert L.hn_quant_act(ctypes.c_void_p(0x10008), 128, 0, 4, 128, 0, 0, FAKE, 128, FAKE, 1, 1, None) == 2
    assert L.hn_quant_act(FAKE, 256, 0, 4, 256, 0, 0, FAKE, 256, FAKE, 1, 2, None) == 1      # scale strides alias
    assert L.hn_quant_act(FAKE, 128, 0, 4, 128, 0, 4, FAKE, 128, FAKE, 1, 1, None) == 5      # unknown flag
    assert L.hn_quant_act(FAKE, 128, 0, 4, 128, 1, 2, FAKE, 128, FAKE, 1, 1, None) == 5      # RNE on e4m3
    args = dict(qa=FAKE, lda=256, sa=FAKE, sars=2, sags=1, sam=0, qw=FAKE, ldw=256, sw=FAKE, swrs=2, swgs=1, swm=0,
                bias=None, bd=0, out=FAKE, ldo=256, od=0, qs=None, qsrs=0, qsgs=0, M=64, N=256, K=256, kind=0, epi=0)

    def gemm(**kw):
        a = dict(args, **kw)
        return L.hn_block_gemm(*a.values(), None)
    assert gemm(K=200, lda=200, ldw=200) == 1                      # K % 128
    assert gemm(kind=7) == 5
    assert gemm(sam=2) == 5                                        # activations cannot be block-scaled
    assert gemm(epi=2) == 5                                        # gelu_quant needs qs
    assert gemm(epi=2, qs=FAKE, qsrs=2, qsgs=1, N=200, ldo=256) == 1   # gelu_quant needs N % 128
    assert gemm(sars=1, sags=32) == 1                               # group-major sa needs sags >= M
    assert gemm(od=3) == 7                                         # int32 out needs row scales
    assert gemm(lda=100) == 1                                      # lda < K
    assert gemm(qa=ctypes.c_void_p(0x10004)) == 2                  # TMA base alignment
    # a bias that does not start on a 16-byte boundary is refused for every N (the epilogue reads it with
    # 16-byte loads wherever 8 columns are in range), also when N % 8 != 0
    assert gemm(bias=ctypes.c_void_p(0x10002), N=200, ldo=256) == 2
    assert gemm(bias=ctypes.c_void_p(0x10002), N=256) == 2
    # int8 with per-row scales on both sides sums all of K in one int32: K * 128 * 128 must stay below 2^31
    big_k = 130944 + 128
    assert gemm(sam=1, swm=1, sars=1, swrs=1, K=big_k, lda=big_k, ldw=big_k) == 1
    assert b"K <= 130944" in L.hn_last_error()
    assert L.hn_adaln_quant(FAKE, FAKE, FAKE, 1, 4, 200, 1e-6, FAKE, FAKE, 1, 1, None) == 1   # D % 128
    assert L.hn_qk_norm_rope(FAKE, 4096, FAKE, FAKE, None, 1, 4, 32, 128, 1e-6, FAKE, None) == 5  # cos w/o sin
    assert L.hn_qk_norm_rope(FAKE, 4096, FAKE, None, None, 1, 4, 32, 64, 1e-6, FAKE, None) == 7   # D != 128
    assert L.hn_gated_residual(FAKE, FAKE, FAKE, 1, 4, 12, FAKE, None) == 1                     # D % 8
    assert L.hn_selftest_wait_timeout(0, None) in (3, 4, 5)        # no device here, or bad timeout
    # the strided push: null pointers and a row wider than a pitch are refused before anything is queued
    assert L.hn_peer_push2d(None, 1024, FAKE, 4096, 1024, 10, None, 0, None) == 5
    assert L.hn_peer_push2d(FAKE, 1024, FAKE, 512, 1024, 10, None, 0, None) == 1
    assert b"hn_peer_push2d" in L.hn_last_error()


def test_no_cpu_path(hn):
    x = torch.randn(4, 128, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        hn.kernels.quantize_activations(x)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        hn.fused.gated_residual(x.view(1, 4, 128), x.view(1, 4, 128), x[:1])


def test_scale_mode_classification(hn):
    sm = hn.kernels._scale_mode
    assert sm(torch.empty(64, 4), 64, 512, weight=False) == "group"
    assert sm(torch.empty(64), 64, 512, weight=False) == "row"
    assert sm(torch.empty(64, 1), 64, 512, weight=False) == "row"
    assert sm(torch.empty(4, 4), 512, 512, weight=True) == "block"
    assert sm(torch.empty(512, 4), 512, 512, weight=True) == "group"
    with pytest.raises(ValueError):
        sm(torch.empty(4, 4), 512, 512, weight=False)
