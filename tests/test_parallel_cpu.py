"""The multi-GPU host logic (hyperkernel_b200/parallel.py) on world-size-2 gloo ranks, on CPU.

Each rank runs as its own process with the same collectives the GPUs run over NCCL; the oracle
stands in for the kernels each rank runs locally.  Expert parallelism must give every routed
row exactly the bits the single-process grouped FFN gives it (a row's output depends only on
the row and its expert); context parallelism must merge the per-rank partials of a long lane
to the whole-lane attention within the merge's rounding.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from hyperkernel_b200 import parallel as P
from hyperkernel_b200 import workload as W

WORLD = 2


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _init(rank, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)


def _gather(src, idx):
    return src.index_select(0, idx.long())


def _scatter(src, idx, out):
    return out.index_copy_(0, idx.long(), src)


def _ep_rank(rank, port, T, E, H, I, K):
    import oracle

    _init(rank, port)
    try:
        inp = W.moe_inputs(T * WORLD, E, H, I, top_k=K, seed=70)  # same experts on every rank
        x = inp["x"][rank * T:(rank + 1) * T]
        logits = inp["logits"][rank * T:(rank + 1) * T]
        ids, w = oracle.route(logits, None, K, 1.0)
        off, tok, pw, inv = oracle.permute(ids, w, E)
        xq, sx = oracle.quant_fp8(x)
        want = oracle.moe_grouped(xq, sx, off, tok, H, I, inp["w13"], inp["s13"], inp["w2"], inp["s2"])

        x_recv, s_recv, loc_off, loc_perm, plan = P.ep_dispatch(
            torch.from_numpy(xq), torch.from_numpy(sx), torch.from_numpy(off), torch.from_numpy(tok), E,
            gather=_gather)
        assert int(loc_off[-1]) == sum(plan.recv_counts) == x_recv.shape[0]
        e0, e1 = P.expert_range(E, WORLD, rank)
        y_local = oracle.moe_grouped(x_recv.numpy(), s_recv.numpy(), loc_off.numpy(), loc_perm.numpy(), H, I,
                                     inp["w13"][e0:e1], inp["s13"][e0:e1], inp["w2"][e0:e1], inp["s2"][e0:e1])
        y_back = P.ep_return(torch.from_numpy(y_local), plan, loc_perm, scatter=_scatter)
        assert y_back.shape == want.shape
        assert np.array_equal(y_back.numpy(), want), f"rank {rank}: expert-parallel rows differ"
        # the weighted combine reads them in the sender's permuted order, as on one GPU
        yb = W.f32_to_bf16_bits(y_back.numpy())
        got = oracle.combine(yb, pw, inv, None, T, K)
        ref = oracle.combine(W.f32_to_bf16_bits(want), pw, inv, None, T, K)
        assert np.array_equal(got, ref)
    finally:
        dist.destroy_process_group()


def _cp_rank(rank, port, ctx, rows, heads):
    import oracle

    _init(rank, port)
    try:
        rng = W.Rng(80)
        lay = W.paged_layout(rng, np.array([ctx]), np.array([rows]), 64)
        inp = W.mla_inputs(lay, heads, seed=81)
        T = lay.num_tokens
        p = oracle.pack(lay.new_rows, lay.context, lay.block_table, 64, lay.num_pages, T)
        c8 = np.zeros((lay.num_slots, 576), np.uint8)
        s8 = np.zeros(lay.num_slots, np.float32)
        oracle.kv_append_fp8(inp["kv_cache"], np.arange(lay.num_slots, dtype=np.int32), c8, s8)
        args = (inp["q"], lay.block_table, p["cu_seqlens"], p["positions"][:T], 64, inp["scale"])
        want, want_lse = oracle.mla_decode(*args, kv_fp8=c8, kv_scale=s8)
        kv = int(lay.kv_len[0])
        b, e = P.cp_ranges(kv, WORLD)[rank]
        o, l = oracle.mla_decode(*args, kv_fp8=c8, kv_scale=s8, kv_begin=np.array([b], np.int32),
                                 kv_end=np.array([e], np.int32))

        def merge(o_all, l_all):
            out, lse = oracle.lse_merge(o_all.numpy(), l_all.numpy())
            return torch.from_numpy(out), torch.from_numpy(lse)

        out, lse = P.cp_merge(torch.from_numpy(o.reshape(T * heads, 512)),
                              torch.from_numpy(l.reshape(T * heads)), merge=merge)
        err = np.abs(out.numpy() - want.reshape(-1, 512)).max() / np.abs(want).max()
        assert err <= 1e-5, f"rank {rank}: merged partials off by {err}"
        assert np.abs(lse.numpy() - want_lse.ravel()).max() <= 1e-4
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_cp_plan_balances_kv_rows_across_ranks(world):
    """The long lane's ranges are contiguous, page-aligned and cover it; every short lane has
    one owner; no rank holds more than the average plus a page, unless a single short lane is
    itself above the average (then that rank holds only its short lanes)."""
    rng = np.random.default_rng(world)
    for case in range(20):
        long_kv = int(rng.integers(1, 1 << 21))
        short = [int(v) for v in rng.integers(1, 1 << 16, int(rng.integers(0, 12)))]
        ranges, owner = P.cp_plan(long_kv, short, world)
        assert len(ranges) == world and len(owner) == len(short)
        assert ranges[0][0] == 0 and ranges[-1][1] == long_kv
        for (b0, e0), (b1, e1) in zip(ranges, ranges[1:]):
            assert e0 == b1 and b0 <= e0 and (e0 % 64 == 0 or e0 == long_kv)
        rows = [e - b for b, e in ranges]
        for i, r in enumerate(owner):
            assert 0 <= r < world
            rows[r] += short[i]
        avg = (long_kv + sum(short)) / world
        for r in range(world):
            if ranges[r][1] > ranges[r][0]:  # a rank with part of the long lane
                assert rows[r] <= avg + 64 + 1, (case, rows, avg)


def test_cp_ranges_are_page_aligned_and_cover_the_lane():
    for kv, world in [(1 << 20, 8), (7005, 2), (100, 4), (64, 8)]:
        r = P.cp_ranges(kv, world)
        assert r[0][0] == 0 and r[-1][1] == kv
        for (a0, a1), (b0, b1) in zip(r, r[1:]):
            assert a1 == b0 and a0 % 64 == 0
        sizes = [b - a for a, b in r]
        assert max(sizes) - min(sizes) <= 64


def test_expert_range_partitions_the_experts():
    assert [P.expert_range(256, 8, r) for r in (0, 7)] == [(0, 32), (224, 256)]
    with pytest.raises(ValueError):
        P.expert_range(10, 4, 0)


@pytest.mark.parametrize("T,E,H,I,K", [(24, 4, 256, 256, 2), (32, 8, 384, 256, 4)])
def test_expert_parallel_dispatch_and_return_on_two_ranks(T, E, H, I, K):
    mp.spawn(_ep_rank, args=(_port(), T, E, H, I, K), nprocs=WORLD, join=True)


def test_context_parallel_merge_on_two_ranks():
    mp.spawn(_cp_rank, args=(_port(), 3000, 5, 16), nprocs=WORLD, join=True)
