"""Failure detection on the device: bounded waits that run out, and plans that are refused.

Every wait in the expert-parallel exchange (hk_ep_counts, hk_ep_wait) is a bounded spin on
epoch flags.  These tests make such a wait run out on one GPU, with flags that nothing ever
sets, and check that the kernel returns, that the device error word names the site, that the
step's plan is marked invalid so no row moves, and that the CUDA context stays usable.  The
"peers" are plain buffers on the same GPU: no second device, process or NVLink mapping is
involved, and nothing faults, traps or hangs.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

TIMEOUT_US = 1000  # 1 ms: long enough to be a real wait, short enough to keep the test fast


def _addrs(*tensors):
    """A host array of device addresses.  The caller must keep it referenced until the call
    that reads it has returned (ctypes.addressof of a temporary would dangle)."""
    return (ctypes.c_uint64 * len(tensors))(*[t.data_ptr() for t in tensors])


def _expect_device_error(hk, text):
    rc = hk.lib().hk_check_errors()
    msg = hk.last_error()
    assert rc == hk.HK_EDEVICE, (rc, msg)
    assert text in msg, msg


def _context_still_usable(hk, cuda):
    src = torch.arange(64 * 8, dtype=torch.float32, device=cuda).view(64, 8)
    idx = torch.arange(63, -1, -1, dtype=torch.int32, device=cuda)
    out = hk.gather_rows(src, idx)
    assert torch.equal(out, src.flip(0))
    hk.check_errors()


def test_flag_wait_runs_out_and_reports_its_site(hk, cuda):
    hk.check_errors()
    flags = torch.zeros(3 * 8, dtype=torch.int32, device=cuda)  # no rank ever raises a flag
    for which, detail in [(1, 972), (2, 973)]:
        hk.call("hk_ep_wait", hk.ptr(flags), which, 2, 7, TIMEOUT_US, hk.stream_ptr())
        _expect_device_error(hk, f"wait timeout (site 5, detail {detail})")
    _context_still_usable(hk, cuda)


def test_count_exchange_with_a_silent_peer_invalidates_the_step(hk, cuda):
    """world = 2, rank 0: the second rank's count matrix and flags are local buffers that no
    kernel raises, so the count wait runs out; dispatch and return then move nothing and raise
    no flag."""
    hk.check_errors()
    E, world, hidden, rows = 8, 2, 128, 12
    counts = [torch.zeros(world * E, dtype=torch.int32, device=cuda) for _ in range(world)]
    flags = [torch.zeros(3 * 8, dtype=torch.int32, device=cuda) for _ in range(world)]
    offsets = torch.tensor([0, 2, 3, 5, 6, 8, 9, 11, 12], dtype=torch.int32, device=cuda)
    send_base = torch.full((E,), 99, dtype=torch.int32, device=cuda)
    local_off = torch.full((E // world + 1,), 99, dtype=torch.int32, device=cuda)
    ret_base = torch.zeros(world * (E // world), dtype=torch.int32, device=cuda)
    epoch = 3
    counts_at, flags_at = _addrs(*counts), _addrs(*flags)
    hk.call("hk_ep_counts", hk.ptr(offsets), E, world, 0, ctypes.addressof(counts_at),
            ctypes.addressof(flags_at), epoch, TIMEOUT_US, hk.ptr(send_base), hk.ptr(local_off),
            hk.ptr(ret_base), hk.stream_ptr())
    _expect_device_error(hk, "wait timeout (site 5, detail 970)")
    # rank 0 published its counts and its flag before waiting
    assert counts[1][:E].cpu().tolist() == [2, 1, 2, 1, 2, 1, 2, 1]
    assert flags[1][0].item() == epoch and flags[0][0].item() == epoch
    assert send_base.cpu().tolist() == [-1] * E
    assert local_off.cpu().tolist()[-1] == -1

    xq = torch.ones((4, hidden), dtype=torch.uint8, device=cuda)
    sx = torch.ones((4, hidden // 128), dtype=torch.float32, device=cuda)
    perm_token = torch.tensor([0, 1, 2, 3] * 3, dtype=torch.int32, device=cuda)
    cap = 32
    recv_x = [torch.full((cap, hidden), 7, dtype=torch.uint8, device=cuda) for _ in range(world)]
    recv_s = [torch.full((cap, 1), 7.0, dtype=torch.float32, device=cuda) for _ in range(world)]
    done = torch.zeros(2, dtype=torch.int32, device=cuda)
    recv_x_at, recv_s_at = _addrs(*recv_x), _addrs(*recv_s)
    hk.call("hk_ep_dispatch", hk.ptr(xq), hk.ptr(sx), 4, hk.ptr(perm_token), hk.ptr(offsets), rows, E,
            world, 0, hidden, cap, hk.ptr(send_base), ctypes.addressof(recv_x_at),
            ctypes.addressof(recv_s_at), ctypes.addressof(flags_at), hk.ptr(done[0:1]), epoch,
            hk.stream_ptr())
    _expect_device_error(hk, "moe row")
    assert all(bool((r == 7).all()) for r in recv_x)
    assert all(f[8:16].abs().sum().item() == 0 for f in flags)  # no dispatch flag raised
    assert done[0].item() == 0  # the launch counter is reset for the next step

    y = torch.ones((cap, hidden), dtype=torch.bfloat16, device=cuda)
    back = [torch.zeros((cap, hidden), dtype=torch.bfloat16, device=cuda) for _ in range(world)]
    back_at = _addrs(*back)
    hk.call("hk_ep_return", hk.ptr(y), E, world, 0, hidden, hk.ptr(local_off), hk.ptr(counts[0]),
            hk.ptr(ret_base), cap, cap, ctypes.addressof(back_at), ctypes.addressof(flags_at),
            hk.ptr(done[1:2]), epoch, hk.stream_ptr())
    _expect_device_error(hk, "moe row")
    assert all(b.abs().sum().item() == 0 for b in back)
    assert all(f[16:24].abs().sum().item() == 0 for f in flags)
    _context_still_usable(hk, cuda)


def test_return_refuses_more_rows_than_its_buffer_holds(hk, cuda):
    """A plan whose received total (from counts a peer wrote) exceeds the rows of y moves no
    row and raises no return flag."""
    hk.check_errors()
    E, world, hidden = 2, 1, 128
    local_off = torch.tensor([0, 6, 10], dtype=torch.int32, device=cuda)  # 10 rows received
    counts = torch.tensor([6, 4], dtype=torch.int32, device=cuda)
    ret_base = torch.tensor([0, 6], dtype=torch.int32, device=cuda)
    y = torch.ones((4, hidden), dtype=torch.bfloat16, device=cuda)  # but y holds only 4
    back = torch.zeros((16, hidden), dtype=torch.bfloat16, device=cuda)
    flags = torch.zeros(3 * 8, dtype=torch.int32, device=cuda)
    done = torch.zeros(1, dtype=torch.int32, device=cuda)
    back_at, flags_at = _addrs(back), _addrs(flags)
    hk.call("hk_ep_return", hk.ptr(y), E, world, 0, hidden, hk.ptr(local_off), hk.ptr(counts),
            hk.ptr(ret_base), 16, 4, ctypes.addressof(back_at), ctypes.addressof(flags_at),
            hk.ptr(done), 1, hk.stream_ptr())
    _expect_device_error(hk, "moe row")
    assert back.abs().sum().item() == 0 and flags.abs().sum().item() == 0
    # the same call with a y of 10 rows moves them all and raises the flag
    y10 = torch.ones((10, hidden), dtype=torch.bfloat16, device=cuda)
    hk.call("hk_ep_return", hk.ptr(y10), E, world, 0, hidden, hk.ptr(local_off), hk.ptr(counts),
            hk.ptr(ret_base), 16, 10, ctypes.addressof(back_at), ctypes.addressof(flags_at),
            hk.ptr(done), 1, hk.stream_ptr())
    hk.check_errors()
    assert back[:10].float().sum().item() == 10 * hidden and back[10:].abs().sum().item() == 0
    assert flags[16].item() == 1
