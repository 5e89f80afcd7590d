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
