"""Failure detection without a GPU fault: a device-side wait on an mbarrier that nothing completes runs
out its (short) limit, records HN_DEVERR_TIMEOUT in the device error word and returns; the host reads the
status and the context stays usable for the next launch."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_timeout_and_context_survives(hn, cuda):
    L = hn.lib
    rc, code = L.device_error()
    assert rc == 0 and code == 0
    st = torch.cuda.current_stream()
    L.check(L.lib.hn_selftest_wait_timeout(20000, L.stream_of(torch.empty(1, device=cuda))), "selftest")
    rc, code = L.device_error(st)
    assert rc == 6 and code == 1          # HN_ERR_TIMEOUT, HN_DEVERR_TIMEOUT
    assert "limit" in L.last_error()
    rc, code = L.device_error(st)        # the word was cleared
    assert rc == 0 and code == 0
    x = torch.randn(64, 256, device=cuda).bfloat16()
    q, s = hn.kernels.quantize_activations(x)   # the context still works
    torch.cuda.synchronize()
    assert q.shape == (64, 256)


def test_timeout_is_reported_on_its_own_stream_only(hn, cuda):
    """Each stream has its own device error word: a wait that runs out on stream A is read by A's reader, and a
    reader of stream B (which launched a GEMM meanwhile) sees nothing."""
    import ctypes
    L = hn.lib
    a, b = torch.cuda.Stream(cuda), torch.cuda.Stream(cuda)
    qa = torch.randint(-127, 128, (256, 512), dtype=torch.int8, device=cuda)
    ones_m, ones_n = torch.ones(256, device=cuda), torch.ones(256, device=cuda)
    with torch.cuda.stream(b):
        hn.kernels.block_gemm(qa, ones_m, qa, ones_n)       # registers stream b's word
    L.check(L.lib.hn_selftest_wait_timeout(20000, ctypes.c_void_p(a.cuda_stream)), "selftest")
    rc_b, code_b = L.device_error(b)
    assert rc_b == 0 and code_b == 0
    rc_a, code_a = L.device_error(a)
    assert rc_a == 6 and code_a == 1
    assert L.device_error(a) == (0, 0)


def test_call_from_another_current_device_uses_the_stream_device(hn, cuda):
    """The library makes the launching stream's device current for the call, so a tensor on one GPU can be
    processed while another GPU is current (only meaningful with two GPUs)."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    x = torch.randn(300, 1024, device="cuda:1").bfloat16()
    with torch.cuda.device(0):
        q1, s1 = hn.kernels.quantize_activations(x)
    q0, s0 = hn.kernels.quantize_activations(x.to("cuda:0"))
    torch.cuda.synchronize(0)
    torch.cuda.synchronize(1)
    assert torch.equal(q1.cpu(), q0.cpu()) and torch.equal(s1.cpu(), s0.cpu())
    qw = torch.randint(-127, 128, (256, 1024), dtype=torch.int8)
    sw = torch.rand(256) * 1e-3
    with torch.cuda.device(0):
        y1 = hn.kernels.block_gemm(q1, s1, qw.to("cuda:1"), sw.to("cuda:1"))
    y0 = hn.kernels.block_gemm(q0, s0, qw.to("cuda:0"), sw.to("cuda:0"))
    assert torch.equal(y1.cpu(), y0.cpu())
