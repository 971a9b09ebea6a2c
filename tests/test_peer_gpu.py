"""The context-parallel merge over peer memory (hk_cp_merge) and the shared-buffer allocation
(hk_sym_alloc), on one GPU.

hk_cp_merge raises this rank's epoch flag on every rank, waits for every rank's flag and merges
every rank's (o, lse) partial.  On one GPU the other "ranks" are plain local buffers whose flag
slots the host sets before the launch, so the kernel never waits on another kernel; the merge
must equal hk_lse_merge over the same partials (which the oracle pins).  A slot that is never set
makes the bounded wait run out.  The two-process test with IPC-mapped buffers is in
test_parallel_gpu.py.
"""
import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _addrs(*tensors):
    """Host array of device addresses; keep it referenced while the call that reads it runs."""
    return (C.c_uint64 * len(tensors))(*[t.data_ptr() for t in tensors])


@pytest.mark.parametrize("world,rank", [(2, 0), (4, 3), (8, 5)])
def test_cp_merge_equals_lse_merge(hk, cuda, world, rank):
    rows, dv, epoch = 640, 512, 9
    g = torch.Generator(device=cuda).manual_seed(world * 10 + rank)
    o = [torch.randn((rows, dv), generator=g, device=cuda) for _ in range(world)]
    lse = [torch.randn((rows,), generator=g, device=cuda) * 3 for _ in range(world)]
    lse[0][:5] = -float("inf")  # rows a rank's shard does not reach
    flags = [torch.zeros(8, dtype=torch.int32, device=cuda) for _ in range(world)]
    for f in flags:  # every other rank has already raised its flag everywhere
        for s in range(world):
            if s != rank:
                f[s] = epoch
    out = torch.empty((rows, dv), dtype=torch.bfloat16, device=cuda)
    lse_out = torch.empty((rows,), dtype=torch.float32, device=cuda)
    o_at, l_at, f_at = _addrs(*o), _addrs(*lse), _addrs(*flags)
    hk.call("hk_cp_merge", C.addressof(o_at), C.addressof(l_at), C.addressof(f_at), world, rank, epoch, 1_000_000,
            rows, dv, hk.ptr(out), hk.ptr(lse_out), hk.stream_ptr())
    want, want_lse = hk.lse_merge(torch.stack(o).contiguous(), torch.stack(lse).contiguous())
    hk.check_errors()
    assert all(int(f[rank]) == epoch for f in flags), "this rank's flag raised on every rank"
    d = (out.float() - want.float()).abs().max().item() / want.float().abs().max().item()
    assert d <= 1e-2
    assert (lse_out - want_lse).abs().max().item() <= 1e-5


def test_cp_merge_wait_runs_out_on_a_silent_rank(hk, cuda):
    rows, dv = 16, 512
    o = [torch.zeros((rows, dv), device=cuda) for _ in range(2)]
    lse = [torch.zeros((rows,), device=cuda) for _ in range(2)]
    flags = [torch.zeros(8, dtype=torch.int32, device=cuda) for _ in range(2)]  # rank 1 never raises
    out = torch.full((rows, dv), 3.0, dtype=torch.bfloat16, device=cuda)
    o_at, l_at, f_at = _addrs(*o), _addrs(*lse), _addrs(*flags)
    hk.call("hk_cp_merge", C.addressof(o_at), C.addressof(l_at), C.addressof(f_at), 2, 0, 4, 1000, rows, dv,
            hk.ptr(out), None, hk.stream_ptr())
    rc = hk.lib().hk_check_errors()
    assert rc == hk.HK_EDEVICE and "wait timeout (site 5, detail 980)" in hk.last_error()
    assert bool((out.float() == 3.0).all()), "no row merged after the wait ran out"


def test_sym_alloc_gives_zeroed_memory_and_a_handle(hk, cuda):
    class Handle(C.Structure):
        _fields_ = [("bytes", C.c_uint8 * 64)]

    p, h = C.c_void_p(), Handle()
    hk.call("hk_sym_alloc", 1 << 20, C.byref(p), C.byref(h))
    try:
        assert p.value and any(h.bytes)
        from cuda.bindings import runtime as rt

        host = np.ones(1 << 18, np.int32)
        (err,) = rt.cudaMemcpy(host.ctypes.data, p.value, 1 << 20, rt.cudaMemcpyKind.cudaMemcpyDeviceToHost)
        assert int(err) == 0 and not host.any()
    finally:
        hk.call("hk_sym_free", p)
