"""Expert and context parallelism on B200s over NCCL (hyperkernel_b200/parallel.py).

The row gather / scatter kernels run on one GPU; the two-rank tests need two GPUs (skipped
otherwise) and run each rank as its own process on its own device.  Expert parallelism must
reproduce, bit for bit, the rows the one-GPU grouped FFN computes for the same tokens (a row's
output does not depend on the other rows of its tile); context parallelism must merge to the
whole-lane attention within the bf16 tolerance.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from hyperkernel_b200 import workload as W

pytestmark = pytest.mark.gpu
TOL = 2e-2


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def test_gather_and_scatter_rows(hk, cuda):
    g = torch.Generator(device=cuda)
    g.manual_seed(5)
    for cols, dtype in [(7168, torch.uint8), (56, torch.float32), (2, torch.float32), (512, torch.bfloat16)]:
        src = torch.randint(0, 255, (300, cols), generator=g, device=cuda).to(dtype)
        idx = torch.randperm(300, generator=g, device=cuda)[:200].to(torch.int32)
        out = hk.gather_rows(src, idx)
        assert torch.equal(out, src[idx.long()])
        back = torch.zeros_like(src)
        hk.scatter_rows(out, idx, back)
        assert torch.equal(back[idx.long()], out)
    hk.check_errors()


def _two_gpus():
    return torch.cuda.is_available() and torch.cuda.device_count() >= 2


def _rank_main(rank, port, what):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    import datetime

    dist.init_process_group("nccl", rank=rank, world_size=2, device_id=dev,
                            timeout=datetime.timedelta(seconds=120))
    try:
        if what == "ep":
            _ep(rank, dev)
        elif what == "ep_peer":
            _ep_peer(rank, dev)
        elif what == "ep_peer_shared":
            _ep_peer_shared(rank, dev)
        elif what == "cp_peer":
            _cp_peer(rank, dev)
        else:
            _cp(rank, dev)
    finally:
        dist.barrier()
        dist.destroy_process_group()


def _ep(rank, dev):
    from hyperkernel_b200 import _lib as hk
    from hyperkernel_b200 import parallel as P

    T, E, H, I, K = 64, 8, 512, 256, 4
    inp = W.moe_inputs(T * 2, E, H, I, top_k=K, seed=90)
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    x = torch.from_numpy(inp["x"][rank * T:(rank + 1) * T].view(np.int16)).to(dev).view(torch.bfloat16)
    ids, w = hk.route(d(inp["logits"][rank * T:(rank + 1) * T]), None, K, 1.0)
    off, tok, pw, inv = hk.permute(ids, w, E)
    xq, sx = hk.quant_fp8(x)
    w13, s13, w2, s2 = d(inp["w13"]), d(inp["s13"]), d(inp["w2"]), d(inp["s2"])
    want = hk.moe_grouped(xq, sx, off, tok, T * K, H, I, w13, s13, w2, s2)[:T * K]
    x_recv, s_recv, loc_off, loc_perm, plan = P.ep_dispatch(xq, sx, off, tok, E)
    e0, e1 = P.expert_range(E, 2, rank)
    rows = x_recv.shape[0]
    y_local = hk.moe_grouped(x_recv, s_recv, loc_off, loc_perm, rows, H, I, w13[e0:e1].contiguous(),
                             s13[e0:e1].contiguous(), w2[e0:e1].contiguous(), s2[e0:e1].contiguous())
    y_back = P.ep_return(y_local, plan, loc_perm)
    torch.cuda.synchronize()
    hk.check_errors()
    assert torch.equal(y_back.view(torch.int16), want.view(torch.int16)), f"rank {rank}: EP rows differ"


def _ep_peer(rank, dev):
    """The same expert-parallel step with dispatch and return as NVLink stores from libhk's
    kernels (EpPeer): every routed row must come back bit-identical to the one-GPU result,
    over several steps (the epoch flags advance)."""
    from hyperkernel_b200 import _lib as hk
    from hyperkernel_b200 import parallel as P

    T, E, H, I, K = 64, 8, 512, 256, 4
    inp = W.moe_inputs(T * 2, E, H, I, top_k=K, seed=93)
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    w13, s13, w2, s2 = d(inp["w13"]), d(inp["s13"]), d(inp["w2"]), d(inp["s2"])
    e0, e1 = P.expert_range(E, 2, rank)
    lw = [t[e0:e1].contiguous() for t in (w13, s13, w2, s2)]
    ep = P.EpPeer(E, T, K, H)
    for step in range(3):
        x = torch.from_numpy(inp["x"][rank * T:(rank + 1) * T].view(np.int16)).to(dev).view(torch.bfloat16)
        logits = d(inp["logits"][rank * T:(rank + 1) * T]) * (1.0 + 0.1 * step)
        ids, w = hk.route(logits, None, K, 1.0)
        off, tok, pw, inv = hk.permute(ids, w, E)
        xq, sx = hk.quant_fp8(x)
        want = hk.moe_grouped(xq, sx, off, tok, T * K, H, I, w13, s13, w2, s2)[:T * K]
        rx, rs, loff, ident = ep.dispatch(xq, sx, off, tok)
        y_local = hk.moe_grouped(rx, rs, loff, ident, ep.rows_cap, H, I, *lw)
        back = ep.give_back(y_local)
        torch.cuda.synchronize()
        hk.check_errors()
        assert torch.equal(back[:T * K].view(torch.int16), want.view(torch.int16)), f"rank {rank} step {step}"
    ep.close()


def _ep_peer_shared(rank, dev):
    """EpPeer with the shared expert in the rank's own grouped-FFN call (dispatch_with_shared:
    the shared expert is expert 0 of [shared, local experts], its rows read the rank's own rows
    kept after the peers' part of the receive buffer): the shared rows and every routed row
    that comes back must equal the one-GPU calls bit for bit, over several steps."""
    from hyperkernel_b200 import _lib as hk
    from hyperkernel_b200 import parallel as P

    T, E, H, I, K = 64, 8, 512, 256, 4
    inp = W.moe_inputs(T * 2, E + 1, H, I, top_k=K, seed=94)  # expert E is the shared one
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    w13, s13, w2, s2 = d(inp["w13"]), d(inp["s13"]), d(inp["w2"]), d(inp["s2"])
    e0, e1 = P.expert_range(E, 2, rank)
    fold = [torch.cat([t[E:], t[e0:e1]]) for t in (w13, s13, w2, s2)]
    every = torch.arange(T, dtype=torch.int32, device=dev)
    sh_off = torch.tensor([0, T], dtype=torch.int32, device=dev)
    ep = P.EpPeer(E, T, K, H, shared_tokens=T)
    for step in range(3):
        x = torch.from_numpy(inp["x"][rank * T:(rank + 1) * T].view(np.int16)).to(dev).view(torch.bfloat16)
        logits = d(inp["logits"][rank * T:(rank + 1) * T, :E]) * (1.0 + 0.1 * step)
        ids, w = hk.route(logits, None, K, 1.0)
        off, tok, pw, inv = hk.permute(ids, w, E)
        xq, sx = hk.quant_fp8(x)
        want = hk.moe_grouped(xq, sx, off, tok, T * K, H, I, w13[:E], s13[:E], w2[:E], s2[:E])[:T * K]
        want_sh = hk.moe_grouped(xq, sx, sh_off, every, T, H, I, w13[E:], s13[E:], w2[E:], s2[E:])
        rx, rs, foff, fperm, frows = ep.dispatch_with_shared(xq, sx, off, tok)
        y_all = hk.moe_grouped(rx, rs, foff, fperm, frows, H, I, *fold)
        back = ep.give_back(y_all[T:])
        torch.cuda.synchronize()
        hk.check_errors()
        assert torch.equal(y_all[:T].view(torch.int16), want_sh.view(torch.int16)), f"shared, rank {rank} step {step}"
        assert torch.equal(back[:T * K].view(torch.int16), want.view(torch.int16)), f"rank {rank} step {step}"
    ep.close()


def _cp(rank, dev):
    from hyperkernel_b200 import _lib as hk
    from hyperkernel_b200 import parallel as P
    import oracle

    heads = 128
    rng = W.Rng(91)
    lay = W.paged_layout(rng, np.array([20000]), np.array([5]), 64)
    inp = W.mla_inputs(lay, heads, seed=92)
    T = lay.num_tokens
    p = oracle.pack(lay.new_rows, lay.context, lay.block_table, 64, lay.num_pages, T)
    c8 = np.zeros((lay.num_slots, 576), np.uint8)
    s8 = np.zeros(lay.num_slots, np.float32)
    oracle.kv_append_fp8(inp["kv_cache"], np.arange(lay.num_slots, dtype=np.int32), c8, s8)
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    q = torch.from_numpy(inp["q"].view(np.int16)).to(dev).view(torch.bfloat16)
    args = (q, d(c8), d(s8), d(lay.block_table), d(p["cu_seqlens"]), d(p["positions"][:T].copy()))
    kv = int(lay.kv_len[0])
    full, full_lse = hk.mla_decode_fp8(*args, 64, kv, inp["scale"])
    b, e = P.cp_ranges(kv, 2)[rank]
    kb, ke = d(np.array([b], np.int32)), d(np.array([e], np.int32))
    f = full.reshape(-1, 512).float().cpu().numpy()
    # the CUDA-core FP8 partial, and the tcgen05 partial over this rank's pages converted to bf16
    o, l = hk.mla_partial_fp8(*args, kb, ke, 64, kv, inp["scale"])
    mine = d(lay.block_table[0, b // 64:(e + 63) // 64].astype(np.int32))
    kv_bf16 = torch.zeros((lay.num_slots, 576), dtype=torch.bfloat16, device=dev)
    hk.kv_dequant_fp8(args[1], args[2], 64, out=kv_bf16, pages=mine)
    o2, l2 = hk.mla_partial(q, kv_bf16, args[3], args[4], args[5], kb, ke, 64, kv, inp["scale"])
    for oo, ll in ((o, l), (o2, l2)):
        out, lse = P.cp_merge(oo.reshape(T * heads, 512), ll.reshape(T * heads))
        torch.cuda.synchronize()
        hk.check_errors()
        a = out.float().cpu().numpy()
        assert np.abs(a - f).max() / np.abs(f).max() <= TOL
        assert (lse.cpu() - full_lse.reshape(-1).cpu()).abs().max().item() <= 1e-3


def _cp_peer(rank, dev):
    """Context parallelism through the C ABI only: each rank's tcgen05 partial over its half of a
    20,000-row lane is written into its own hk_sym_alloc buffer, and hk_cp_merge reads both
    ranks' partials over NVLink and merges them, for three steps (the buffer sets alternate);
    the merged rows match the whole lane on one GPU, and the oracle on sampled heads."""
    from hyperkernel_b200 import _lib as hk
    from hyperkernel_b200 import parallel as P
    import oracle

    heads = 128
    rng = W.Rng(94)
    lay = W.paged_layout(rng, np.array([20000]), np.array([5]), 64)
    inp = W.mla_inputs(lay, heads, seed=95)
    T = lay.num_tokens
    p = oracle.pack(lay.new_rows, lay.context, lay.block_table, 64, lay.num_pages, T)
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    q = torch.from_numpy(inp["q"].view(np.int16)).to(dev).view(torch.bfloat16)
    cache = torch.from_numpy(inp["kv_cache"].view(np.int16)).to(dev).view(torch.bfloat16)
    kv = int(lay.kv_len[0])
    bt, cu, pos = d(lay.block_table), d(p["cu_seqlens"]), d(p["positions"][:T].copy())
    whole, whole_lse = hk.mla_decode(q, cache, bt, cu, pos, 64, kv, inp["scale"], impl=2)
    b, e = P.cp_ranges(kv, 2)[rank]
    kb, ke = d(np.array([b], np.int32)), d(np.array([e], np.int32))
    cp = P.CpPeer(T * heads, 512, T * heads)
    heads_s = np.array([0, 77, 127])
    want, want_lse = oracle.mla_decode(np.ascontiguousarray(inp["q"][:, heads_s]), lay.block_table, p["cu_seqlens"],
                                       p["positions"][:T], 64, inp["scale"], kv_bf16=inp["kv_cache"])
    for step in range(3):
        o_buf, l_buf = cp.next_buffers()
        ws = torch.empty(hk.mla_workspace_size(1, T, heads, kv), dtype=torch.uint8, device=dev)
        hk.call("hk_mla_partial", hk.ptr(q), hk.ptr(cache), hk.ptr(bt), bt.shape[1], hk.ptr(cu), hk.ptr(pos),
                hk.ptr(kb), hk.ptr(ke), 1, T, heads, 64, cache.shape[0], kv, inp["scale"], hk.ptr(o_buf),
                hk.ptr(l_buf), hk.ptr(ws), ws.numel(), hk.stream_ptr())
        out, lse = cp.merge()
        torch.cuda.synchronize()
        hk.check_errors()
        a, f = out.float().cpu().numpy(), whole.reshape(-1, 512).float().cpu().numpy()
        assert np.abs(a - f).max() / np.abs(f).max() <= TOL, f"rank {rank} step {step}"
        assert (lse.cpu() - whole_lse.reshape(-1).cpu()).abs().max().item() <= 1e-3
        got = a.reshape(T, heads, 512)[:, heads_s]
        assert np.abs(got - want).max() / np.abs(want).max() <= TOL
    cp.close()


@pytest.mark.skipif(not _two_gpus(), reason="needs two GPUs")
def test_context_parallel_over_peer_memory_on_two_gpus():
    mp.spawn(_rank_main, args=(_port(), "cp_peer"), nprocs=2, join=True)


@pytest.mark.skipif(not _two_gpus(), reason="needs two GPUs")
def test_expert_parallel_on_two_gpus():
    mp.spawn(_rank_main, args=(_port(), "ep"), nprocs=2, join=True)


@pytest.mark.skipif(not _two_gpus(), reason="needs two GPUs")
def test_context_parallel_on_two_gpus():
    mp.spawn(_rank_main, args=(_port(), "cp"), nprocs=2, join=True)


@pytest.mark.skipif(not _two_gpus(), reason="needs two GPUs")
def test_expert_parallel_over_peer_memory_on_two_gpus():
    mp.spawn(_rank_main, args=(_port(), "ep_peer"), nprocs=2, join=True)


@pytest.mark.skipif(not _two_gpus(), reason="needs two GPUs")
def test_ep_peer_with_the_shared_expert_in_the_same_call_on_two_gpus():
    mp.spawn(_rank_main, args=(_port(), "ep_peer_shared"), nprocs=2, join=True)
