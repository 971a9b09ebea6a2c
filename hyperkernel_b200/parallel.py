"""Multi-GPU decomposition of the decode step over torch.distributed (NCCL over NVLink on the
B200s; any backend whose all_to_all_single / all_gather the tensors support).

Two shards have a real exchange step:

  * expert parallelism for the MoE layer (config 4): rank r owns experts
    [r E/N, (r+1) E/N).  After routing and the global permutation, the permuted rows of
    destination d are contiguous (rows offsets[d E/N] .. offsets[(d+1) E/N]), so dispatch is
    one exchange of per-(destination, expert) counts and one all-to-allv of the routed e4m3
    rows and their 1x128 scales.  The receiver runs the grouped FFN over what it got, its
    rows ordered expert-major through a local permutation (the grouped FFN gathers through
    perm_token, so no extra copy), and combine is the reverse all-to-allv followed by the
    weighted sum of hk_combine on the sender.

  * context parallelism for a long lane (config 5): the lane's KV positions are split into
    page-aligned contiguous ranges, one per rank; each rank computes (o, lse) partials over
    its range (hk_mla_partial_fp8), the partials are all-gathered and merged by
    log-sum-exp (hk_lse_merge).

The decode attention itself shards by lane with no exchange (each rank runs its own lanes).
The row movement defaults to libhk's kernels (hk_gather_rows / hk_scatter_rows) and the merge
to hk_lse_merge; `gather`, `scatter` and `merge` are parameters only so the host-side plan and
exchange can be exercised with CPU tensors.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np
import torch
import torch.distributed as dist

from . import _lib


# ------------------------------------------------------------------------------------------
# expert parallelism
# ------------------------------------------------------------------------------------------

def expert_range(num_experts: int, world: int, rank: int) -> tuple[int, int]:
    """Experts owned by `rank`: a contiguous block of num_experts / world."""
    if num_experts % world:
        raise ValueError(f"{num_experts} experts do not split over {world} ranks")
    per = num_experts // world
    return rank * per, (rank + 1) * per


@dataclass
class EpPlan:
    """One dispatch: rows sent to / received from every rank and the local expert order."""
    send_counts: list          # rows this rank sends to each rank (its permuted-row blocks)
    recv_counts: list          # rows this rank receives from each rank
    recv_expert_counts: np.ndarray  # [world][local experts] rows received per source and expert
    local_offsets: np.ndarray  # [local experts + 1] exclusive scan of the rows per local expert
    local_perm: np.ndarray     # row j of the expert-major order = received row local_perm[j]


def ep_plan(offsets: np.ndarray, num_experts: int, group=None, device=None) -> EpPlan:
    """Exchanges the per-(destination, expert) row counts; offsets is the host copy of the
    global permutation's expert offsets [num_experts + 1]; the counts travel on `device`
    (the process group's device)."""
    world = dist.get_world_size(group)
    per = num_experts // world
    counts = np.diff(np.asarray(offsets, dtype=np.int64)).reshape(world, per)
    send = torch.from_numpy(np.ascontiguousarray(counts)).to(device or "cpu")
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    recv_np = recv.cpu().numpy()
    send_counts = counts.sum(1).tolist()
    recv_counts = recv_np.sum(1).tolist()
    # received layout: source-major, and expert-major inside each source's block
    src_base = np.concatenate([[0], np.cumsum(recv_counts)[:-1]]).astype(np.int64)
    seg = np.concatenate([np.zeros((world, 1), np.int64), np.cumsum(recv_np, axis=1)[:, :-1]], axis=1)
    perm = []
    for e in range(per):
        for s in range(world):
            start = src_base[s] + seg[s, e]
            perm.append(np.arange(start, start + recv_np[s, e], dtype=np.int64))
    local_perm = np.concatenate(perm).astype(np.int32) if perm else np.zeros(0, np.int32)
    local_offsets = np.concatenate([[0], np.cumsum(recv_np.sum(0))]).astype(np.int32)
    return EpPlan(send_counts, recv_counts, recv_np, local_offsets, local_perm)


def _default_gather(src, idx):
    return _lib.gather_rows(src, idx)


def _default_scatter(src, idx, out):
    return _lib.scatter_rows(src, idx, out)


def ep_dispatch(xq, sx, offsets, perm_token, num_experts: int, group=None, gather=None):
    """Sends every routed row to the rank owning its expert.

    xq [tokens][hidden] e4m3 and sx [tokens][hidden/128] are this rank's quantised tokens;
    offsets / perm_token are the global permutation (hk_permute over all experts).  Returns
    (xq_recv, sx_recv, local_offsets, local_perm, plan): the rows of this rank's experts from
    every rank, the expert offsets and permutation to run the grouped FFN over them."""
    gather = gather or _default_gather
    plan = ep_plan(offsets.cpu().numpy(), num_experts, group, device=xq.device)
    x_send = gather(xq, perm_token)
    s_send = gather(sx, perm_token)
    rows_in = int(sum(plan.recv_counts))
    x_recv = torch.empty((rows_in,) + tuple(xq.shape[1:]), dtype=xq.dtype, device=xq.device)
    s_recv = torch.empty((rows_in,) + tuple(sx.shape[1:]), dtype=sx.dtype, device=sx.device)
    dist.all_to_all_single(x_recv, x_send, plan.recv_counts, plan.send_counts, group=group)
    dist.all_to_all_single(s_recv, s_send, plan.recv_counts, plan.send_counts, group=group)
    dev = xq.device
    local_offsets = torch.from_numpy(plan.local_offsets).to(dev)
    local_perm = torch.from_numpy(plan.local_perm).to(dev)
    return x_recv, s_recv, local_offsets, local_perm, plan


def ep_return(y_local, plan: EpPlan, local_perm, group=None, scatter=None):
    """Sends the expert outputs back: y_local holds the grouped FFN's rows in the local
    expert-major order; the result holds this rank's routed rows in its global permuted order
    (what hk_combine reads through inv)."""
    scatter = scatter or _default_scatter
    rows_in = int(sum(plan.recv_counts))
    y_src = torch.empty((rows_in,) + tuple(y_local.shape[1:]), dtype=y_local.dtype, device=y_local.device)
    scatter(y_local[:rows_in], local_perm, y_src)
    rows_out = int(sum(plan.send_counts))
    y_back = torch.empty((rows_out,) + tuple(y_local.shape[1:]), dtype=y_local.dtype, device=y_local.device)
    dist.all_to_all_single(y_back, y_src, plan.send_counts, plan.recv_counts, group=group)
    return y_back


# ------------------------------------------------------------------------------------------
# context parallelism
# ------------------------------------------------------------------------------------------

def cp_ranges(kv_len: int, world: int, page: int = 64) -> list[tuple[int, int]]:
    """Page-aligned contiguous KV ranges [begin, end) covering [0, kv_len), one per rank,
    balanced to within a page."""
    pages = (kv_len + page - 1) // page
    out = []
    for r in range(world):
        p0 = pages * r // world
        p1 = pages * (r + 1) // world
        out.append((min(p0 * page, kv_len), min(p1 * page, kv_len)))
    return out


def cp_plan(long_kv: int, short_kv, world: int, page: int = 64):
    """Context-parallel plan of one long lane and whole short lanes over `world` ranks with
    equal KV rows per rank: the short lanes go, largest first, to the rank holding the fewest
    rows so far; the long lane is then cut into page-aligned contiguous ranges, in rank order,
    that fill every rank up to a common level (a rank whose short lanes already pass it gets
    none of the long lane).  Returns (ranges [(begin, end)] per rank, owner rank per short
    lane).  The same inputs give the same plan on every rank."""
    short_kv = [int(k) for k in short_kv]
    load = [0] * world
    owner = [0] * len(short_kv)
    for i in sorted(range(len(short_kv)), key=lambda i: (-short_kv[i], i)):
        r = min(range(world), key=lambda r: (load[r], r))
        owner[i] = r
        load[r] += short_kv[i]
    # water level L with sum(max(0, L - load[r])) = long_kv
    order = sorted(load)
    level, filled = float(order[0]), 0
    for n in range(1, world + 1):
        nxt = order[n] if n < world else float("inf")
        if filled + n * (nxt - level) >= long_kv:
            level += (long_kv - filled) / n
            break
        filled += n * (nxt - level)
        level = nxt
    ranges, at, cum = [], 0, 0.0
    pages = (long_kv + page - 1) // page
    for r in range(world):
        cum += max(0.0, level - load[r])
        stop = long_kv if r == world - 1 else min(long_kv, int(round(cum / page)) * page)
        stop = max(stop, at)
        ranges.append((at, stop))
        at = stop
    assert at == long_kv and pages * page >= long_kv
    return ranges, owner


def _default_merge(o_parts, lse_parts):
    return _lib.lse_merge(o_parts, lse_parts)


def cp_merge(o_part, lse_part, group=None, merge=None):
    """All-gathers every rank's (o [rows][dv] fp32, lse [rows]) partial for the same query rows
    and merges them by log-sum-exp; every rank gets the merged (out, lse)."""
    merge = merge or _default_merge
    world = dist.get_world_size(group)
    # flat outputs: every backend takes a 1-D concatenation
    o_all = torch.empty(world * o_part.numel(), dtype=o_part.dtype, device=o_part.device)
    lse_all = torch.empty(world * lse_part.numel(), dtype=lse_part.dtype, device=lse_part.device)
    dist.all_gather_into_tensor(o_all, o_part.contiguous().view(-1), group=group)
    dist.all_gather_into_tensor(lse_all, lse_part.contiguous().view(-1), group=group)
    return merge(o_all.view((world,) + tuple(o_part.shape)), lse_all.view((world,) + tuple(lse_part.shape)))


# ------------------------------------------------------------------------------------------
# buffers shared across the node's GPUs (hk_sym_alloc / hk_sym_import)
# ------------------------------------------------------------------------------------------

class IpcHandle(ctypes.Structure):
    """hk_ipc_handle: the 64 bytes of a CUDA IPC memory handle."""
    _fields_ = [("bytes", ctypes.c_uint8 * 64)]


def all_gather_bytes(data: bytes, group=None) -> list:
    """The default handle exchange: every rank's bytes, in rank order, over the process group
    (any backend; only the host-side handles travel, never device data)."""
    out = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, data, group=group)
    return out


class _Cai:
    """A raw device allocation seen through __cuda_array_interface__, for torch.as_tensor."""

    def __init__(self, ptr, shape, typestr):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 2, "strides": None}


_TYPESTR = {torch.uint8: "|u1", torch.int32: "<i4", torch.float32: "<f4", torch.bfloat16: "<i2"}


class SymBuffer:
    """A buffer every rank allocates with hk_sym_alloc (zeroed device memory plus its IPC handle)
    and maps every other rank's copy of with hk_sym_import, after the ranks swap handles through
    `exchange` (bytes in, every rank's bytes out).  `ptrs` is a host array of the world's
    addresses in this process (rank i's copy at i), the form the hk_ep_* and hk_cp_merge entry
    points take; `tensor` views this rank's own copy.  No torch allocator and no NCCL."""

    def __init__(self, shape, dtype, world, rank, exchange):
        self.shape, self.dtype, self.world, self.rank = tuple(shape), dtype, world, rank
        self.nbytes = int(np.prod(self.shape)) * torch.empty((), dtype=dtype).element_size()
        p, h = ctypes.c_void_p(), IpcHandle()
        _lib.call("hk_sym_alloc", max(self.nbytes, 16), ctypes.byref(p), ctypes.byref(h))
        self.local = p.value
        handles = exchange(bytes(h.bytes))
        addrs = []
        self._imported = []
        for i, hb in enumerate(handles):
            if i == rank:
                addrs.append(self.local)
                continue
            ih, q = IpcHandle.from_buffer_copy(hb), ctypes.c_void_p()
            _lib.call("hk_sym_import", ctypes.byref(ih), ctypes.byref(q))
            self._imported.append(q.value)
            addrs.append(q.value)
        self.ptrs = (ctypes.c_uint64 * world)(*addrs)
        view = torch.as_tensor(_Cai(self.local, self.shape, _TYPESTR[dtype]), device=torch.device("cuda"))
        self.tensor = view.view(dtype) if dtype == torch.bfloat16 else view

    def close(self, barrier):
        """Unmaps the peers' copies, waits for every rank to do the same (`barrier`), then frees
        this rank's copy."""
        for q in self._imported:
            _lib.call("hk_sym_close", q)
        self._imported = []
        barrier()
        if self.local:
            _lib.call("hk_sym_free", self.local)
            self.local = None


# ------------------------------------------------------------------------------------------
# expert parallelism over NVLink peer memory
# ------------------------------------------------------------------------------------------

class EpPeer:
    """Expert-parallel dispatch and return written straight into the other ranks' memory
    (hk_ep_counts / hk_ep_dispatch / hk_ep_return over SymBuffers), so a step needs no host
    synchronisation and no NCCL call: the counts, the routed rows and the expert outputs travel
    as NVLink stores from our kernels, and every rank waits on epoch flags with a bound.

    The receive buffer comes out expert-major, so the grouped FFN runs over it with the
    identity permutation.  Buffers are sized for `tokens` tokens per rank routed top_k ways.
    With `shared_tokens` the receive buffer keeps that many more rows after the peers' part,
    for this rank's own rows of the shared expert (`dispatch_with_shared`).  The process group
    only carries the IPC handles at set-up (`exchange`)."""

    FLAGS_COUNTS, FLAGS_DISPATCH, FLAGS_RETURN = 0, 1, 2

    def __init__(self, num_experts, tokens, top_k, hidden, group=None, timeout_us=2_000_000, exchange=None,
                 shared_tokens=0):
        self.group = group or dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        self.E, self.H = num_experts, hidden
        self.El = num_experts // self.world
        self.back_cap = tokens * top_k
        self.rows_cap = tokens * top_k * self.world
        self.shared = shared_tokens
        self.timeout_us = timeout_us
        dev = torch.device("cuda", torch.cuda.current_device())
        ex = exchange or (lambda b: all_gather_bytes(b, self.group))

        def sym(shape, dtype):
            return SymBuffer(shape, dtype, self.world, self.rank, ex)

        self._bufs = [sym((self.world * num_experts,), torch.int32), sym((3 * 8,), torch.int32),
                      sym((self.rows_cap + shared_tokens, hidden), torch.uint8),
                      sym((self.rows_cap + shared_tokens, hidden // 128), torch.float32),
                      sym((self.back_cap, hidden), torch.bfloat16)]
        c, f, x, sc, b = self._bufs
        self.counts, self.counts_ptrs = c.tensor, c.ptrs
        self.flags, self.flags_ptrs = f.tensor, f.ptrs
        self.recv_x, self.recv_x_ptrs = x.tensor, x.ptrs
        self.recv_s, self.recv_s_ptrs = sc.tensor, sc.ptrs
        self.back_y, self.back_y_ptrs = b.tensor, b.ptrs
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        self.send_base = torch.zeros(num_experts, dtype=torch.int32, device=dev)
        self.local_off = torch.zeros(self.El + 1, dtype=torch.int32, device=dev)
        self.ret_base = torch.zeros(self.world * self.El, dtype=torch.int32, device=dev)
        self.done = torch.zeros(2, dtype=torch.int32, device=dev)
        self.identity = torch.arange(self.rows_cap, dtype=torch.int32, device=dev)
        # with the shared expert first: rows [0, T) read the own rows kept after the peers'
        # part, rows [T, T + received) read the received rows in order
        p = torch.arange(self.rows_cap + shared_tokens, dtype=torch.int32, device=dev)
        self.perm_shared = torch.where(p < shared_tokens, p + self.rows_cap, p - shared_tokens)
        self.zero = torch.zeros(1, dtype=torch.int32, device=dev)
        self.epoch = 0

    def close(self):
        torch.cuda.synchronize()
        for b in self._bufs:
            b.close(lambda: dist.barrier(group=self.group))
        self._bufs = []

    def _wait(self, which, stream):
        _lib.call("hk_ep_wait", _lib.ptr(self.flags), which, self.world, self.epoch, self.timeout_us,
                  _lib.stream_ptr(stream))

    def dispatch(self, xq, sx, offsets, perm_token, stream=None):
        """Sends this rank's routed rows; returns (recv_x, recv_s, local_offsets, identity) for
        the grouped FFN over this rank's experts, ready once the call's stream gets there."""
        self.epoch = (self.epoch + 1) & 0x7FFFFFFF or 1
        s = _lib.stream_ptr(stream)
        _lib.call("hk_ep_counts", _lib.ptr(offsets), self.E, self.world, self.rank, ctypes.addressof(self.counts_ptrs),
                  ctypes.addressof(self.flags_ptrs), self.epoch, self.timeout_us, _lib.ptr(self.send_base),
                  _lib.ptr(self.local_off), _lib.ptr(self.ret_base), s)
        rows = perm_token.shape[0]
        _lib.call("hk_ep_dispatch", _lib.ptr(xq), _lib.ptr(sx), xq.shape[0], _lib.ptr(perm_token), _lib.ptr(offsets),
                  rows, self.E, self.world, self.rank, self.H, self.rows_cap, _lib.ptr(self.send_base),
                  ctypes.addressof(self.recv_x_ptrs), ctypes.addressof(self.recv_s_ptrs), ctypes.addressof(self.flags_ptrs),
                  _lib.ptr(self.done[0:1]), self.epoch, s)
        self._wait(self.FLAGS_DISPATCH, stream)
        return self.recv_x, self.recv_s, self.local_off, self.identity

    def dispatch_with_shared(self, xq, sx, offsets, perm_token, stream=None):
        """dispatch() plus this rank's own `shared_tokens` rows for the shared expert, so one
        grouped-FFN call runs the shared expert (expert 0 of its weights) and this rank's
        routed experts (1 .. E/N): returns (x, scales, offsets [E/N + 2], row map, rows).  Rows
        [0, T) of that call's output are the shared expert's, rows [T, ...) go to give_back."""
        T = self.shared
        if T <= 0 or xq.shape[0] != T:
            raise ValueError("dispatch_with_shared: the peer was built for %d shared rows" % T)
        xr, sr, loff, _ = self.dispatch(xq, sx, offsets, perm_token, stream)
        with torch.cuda.stream(stream if stream is not None else torch.cuda.current_stream()):
            xr[self.rows_cap:].copy_(xq)
            sr[self.rows_cap:].copy_(sx)
            off = torch.cat([self.zero, loff + T])
        return xr, sr, off, self.perm_shared, self.rows_cap + T

    def give_back(self, y_local, stream=None):
        """Returns the expert outputs (rows in the receive buffer's order) to their sources;
        the result is this rank's routed rows in its permuted order (back_y)."""
        s = _lib.stream_ptr(stream)
        _lib.call("hk_ep_return", _lib.ptr(y_local), self.E, self.world, self.rank, self.H, _lib.ptr(self.local_off),
                  _lib.ptr(self.counts), _lib.ptr(self.ret_base), self.back_cap, self.rows_cap,
                  ctypes.addressof(self.back_y_ptrs), ctypes.addressof(self.flags_ptrs), _lib.ptr(self.done[1:2]), self.epoch, s)
        self._wait(self.FLAGS_RETURN, stream)
        return self.back_y


# ------------------------------------------------------------------------------------------
# context parallelism over NVLink peer memory
# ------------------------------------------------------------------------------------------

class CpPeer:
    """The context-parallel exchange of a step's (o, lse) partials fused with their LSE merge
    (hk_cp_merge): each rank's partial attention writes straight into its own shared buffer, and
    the merge kernel reads every rank's over NVLink once every rank's epoch flag is up.  Two sets
    of buffers alternate by step parity, so a rank that runs ahead writes the set no peer is
    reading.  `rows` x `dv` partial rows per rank (the attention's whole output), of which the
    first `merge_rows` are merged."""

    def __init__(self, rows, dv, merge_rows, group=None, timeout_us=2_000_000, exchange=None):
        self.group = group or dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        self.rows, self.dv, self.merge_rows, self.timeout_us = rows, dv, merge_rows, timeout_us
        ex = exchange or (lambda b: all_gather_bytes(b, self.group))
        self._o = [SymBuffer((rows, dv), torch.float32, self.world, self.rank, ex) for _ in range(2)]
        self._lse = [SymBuffer((rows,), torch.float32, self.world, self.rank, ex) for _ in range(2)]
        self._flags = [SymBuffer((8,), torch.int32, self.world, self.rank, ex) for _ in range(2)]
        dev = torch.device("cuda", torch.cuda.current_device())
        self.out = torch.empty((merge_rows, dv), dtype=torch.bfloat16, device=dev)
        self.lse_out = torch.empty((merge_rows,), dtype=torch.float32, device=dev)
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        self.epoch = 0

    def next_buffers(self):
        """Starts a step: the (o, lse) tensors this rank's partial attention writes into."""
        self.epoch = (self.epoch + 1) & 0x7FFFFFFF or 1
        k = self.epoch & 1
        return self._o[k].tensor, self._lse[k].tensor

    def merge(self, stream=None):
        """Merges every rank's partial of this step; returns (out bf16, lse) of merge_rows rows."""
        k = self.epoch & 1
        _lib.call("hk_cp_merge", ctypes.addressof(self._o[k].ptrs), ctypes.addressof(self._lse[k].ptrs),
                  ctypes.addressof(self._flags[k].ptrs), self.world, self.rank, self.epoch, self.timeout_us,
                  self.merge_rows, self.dv, _lib.ptr(self.out), _lib.ptr(self.lse_out), _lib.stream_ptr(stream))
        return self.out, self.lse_out

    def close(self):
        torch.cuda.synchronize()
        for b in self._o + self._lse + self._flags:
            b.close(lambda: dist.barrier(group=self.group))
        self._o = self._lse = self._flags = []
