"""The copy-engine K/V exchange's device side on one GPU: a push (DMA copy + fenced flag write) into local
memory, the bounded flag wait that gates attention, and the wait's time limit (a flag that nothing sets: the
stream's error word reads HN_ERR_TIMEOUT and the context stays usable)."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def vp(x):
    return ctypes.c_void_p(x)


def test_push_then_wait_sees_data(hn, cuda):
    L = hn.lib
    st = torch.cuda.current_stream()
    src = torch.randn(4096, 384, device=cuda).bfloat16()
    dst = torch.zeros_like(src)
    flags = torch.zeros(2 * 4, dtype=torch.int32, device=cuda)
    # four "sources" x two kinds: rank 1's own flags (index 1 of each kind) are skipped
    for kind in range(2):
        for src_rank in (0, 2, 3):
            L.check(L.lib.hn_peer_push(vp(dst.data_ptr()), vp(src.data_ptr()), src.numel() * 2,
                                       vp(flags.data_ptr() + 4 * (kind * 4 + src_rank)), 7, vp(st.cuda_stream)),
                    "hn_peer_push", launches=0)
    L.check(L.lib.hn_wait_flags(vp(flags.data_ptr()), 2, 4, 4, 1, 7, 2000000, vp(st.cuda_stream)), "hn_wait_flags")
    # one source's two flags (kinds 0 and 1, `count` apart)
    L.check(L.lib.hn_wait_flags(vp(flags.data_ptr() + 4 * 2), 2, 1, 4, -1, 7, 2000000, vp(st.cuda_stream)),
            "hn_wait_flags")
    out = dst.float().sum()
    rc, code = L.device_error(st)
    assert rc == 0 and code == 0
    assert torch.equal(dst, src)
    assert flags.tolist() == [7, 0, 7, 7, 7, 0, 7, 7]
    assert torch.isfinite(out)


def test_strided_push_moves_one_head_group(hn, cuda):
    """hn_peer_push2d as the head-parallel exchange uses it: head group 2 (4 heads of 128) of every token of a
    [tokens, 16 heads, 128] tensor into a contiguous [tokens, 4, 128] buffer, and back into the head columns of a
    [tokens, 16, 128] buffer; then the flag."""
    L = hn.lib
    st = torch.cuda.current_stream()
    tok, heads, hpg, g = 1000, 16, 4, 2
    src = torch.randn(tok, heads, 128, device=cuda).bfloat16()
    grp = torch.zeros(tok, hpg, 128, dtype=torch.bfloat16, device=cuda)
    back = torch.zeros_like(src)
    flag = torch.zeros(1, dtype=torch.int32, device=cuda)
    width, row = hpg * 128 * 2, heads * 128 * 2
    L.check(L.lib.hn_peer_push2d(vp(grp.data_ptr()), width, vp(src.data_ptr() + g * width), row, width, tok, None, 0,
                                 vp(st.cuda_stream)), "hn_peer_push2d", launches=0)
    L.check(L.lib.hn_peer_push2d(vp(back.data_ptr() + g * width), row, vp(grp.data_ptr()), width, width, tok,
                                 vp(flag.data_ptr()), 3, vp(st.cuda_stream)), "hn_peer_push2d", launches=0)
    torch.cuda.synchronize()
    assert torch.equal(grp, src[:, g * hpg:(g + 1) * hpg])
    assert torch.equal(back[:, g * hpg:(g + 1) * hpg], src[:, g * hpg:(g + 1) * hpg])
    assert int(back[:, :g * hpg].abs().sum()) == 0 and int(back[:, (g + 1) * hpg:].abs().sum()) == 0
    assert flag.item() == 3
    # a width beyond a pitch is refused before anything is queued
    rc = L.lib.hn_peer_push2d(vp(grp.data_ptr()), width, vp(src.data_ptr()), width - 16, width, tok, None, 0,
                              vp(st.cuda_stream))
    assert rc == 1 and "hn_peer_push2d" in L.last_error()


def test_wait_compares_wrap_safe(hn, cuda):
    """Counters compare by signed difference: 0x00000002 is 'after' 0xFFFFFFFE."""
    L = hn.lib
    st = torch.cuda.current_stream()
    flags = torch.tensor([2, 2], dtype=torch.int32, device=cuda)
    L.check(L.lib.hn_wait_flags(vp(flags.data_ptr()), 1, 2, 2, -1, 0xFFFFFFFE, 2000000, vp(st.cuda_stream)),
            "hn_wait_flags")
    rc, code = L.device_error(st)
    assert rc == 0 and code == 0


def test_wait_runs_out_and_context_survives(hn, cuda):
    L = hn.lib
    st = torch.cuda.current_stream()
    flags = torch.zeros(4, dtype=torch.int32, device=cuda)
    flags[0] = 5                                                # one of the three waited flags arrived
    L.check(L.lib.hn_wait_flags(vp(flags.data_ptr()), 1, 4, 4, 3, 5, 20000, vp(st.cuda_stream)), "hn_wait_flags")
    rc, code = L.device_error(st)
    assert rc == 6 and code == 1                                # HN_ERR_TIMEOUT, HN_DEVERR_TIMEOUT
    rc, code = L.device_error(st)
    assert rc == 0 and code == 0
    x = torch.randn(64, 256, device=cuda).bfloat16()
    q, s = hn.kernels.quantize_activations(x)
    torch.cuda.synchronize()
    assert q.shape == (64, 256)


def test_wait_rejects_bad_arguments(hn, cuda):
    L = hn.lib
    flags = torch.zeros(8, dtype=torch.int32, device=cuda)
    st = vp(torch.cuda.current_stream().cuda_stream)
    assert L.lib.hn_wait_flags(vp(flags.data_ptr()), 2, 1024, 1024, 0, 1, 1000, st) == 1    # HN_ERR_SHAPE
    assert L.lib.hn_wait_flags(vp(flags.data_ptr() + 2), 1, 2, 2, 0, 1, 1000, st) == 2       # HN_ERR_ALIGN
    assert L.lib.hn_wait_flags(vp(flags.data_ptr()), 1, 2, 2, 0, 1, 0, st) == 5              # HN_ERR_ARG
    assert L.lib.hn_wait_flags(None, 1, 2, 2, 0, 1, 1000, st) == 5
