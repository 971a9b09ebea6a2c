"""The decode step's attention path as one object: pack -> KV append -> paged MLA attention.

`MlaDecodeStep` owns the device-resident state of one attention layer — the paged latent
cache, the lanes' block tables and the kernels' scratch — and runs a step either from
device tensors (`run`) or end to end from pinned host buffers (`step_host`: the H2D copy of
the step's inputs, the kernels and the D2H copy of the output, all on one stream).
`HostPipeline` runs a sequence of such host-buffer steps with the copies overlapped with the
neighbouring steps' kernels.  Every kernel is a libhk.so kernel; there is no CPU path.
"""
from __future__ import annotations

import numpy as np
import torch

from . import _lib as hk


class MlaDecodeStep:
    def __init__(self, block_table: np.ndarray, num_pages: int, page_size: int, heads: int,
                 scale: float, max_tokens: int, max_kv_len: int, device, cache=None,
                 impl: int = 0):
        self.device = torch.device(device)
        self.page_size = page_size
        self.num_pages = num_pages
        self.heads = heads
        self.scale = float(scale)
        self.max_tokens = max_tokens
        self.max_kv_len = max_kv_len
        self.impl = impl
        self.lanes = block_table.shape[0]
        self.block_table = torch.from_numpy(np.ascontiguousarray(block_table, np.int32)).to(self.device)
        slots = num_pages * page_size
        self.cache = cache if cache is not None else torch.zeros(
            (slots, 576), dtype=torch.bfloat16, device=self.device)
        ws = hk.mla_workspace_size(self.lanes, max_tokens, heads, max_kv_len)
        self.workspace = torch.empty(max(ws, 16), dtype=torch.uint8, device=self.device)
        T = max_tokens
        self.out = torch.empty((T, heads, 512), dtype=torch.bfloat16, device=self.device)
        self.lse = torch.empty((T, heads), dtype=torch.float32, device=self.device)
        L = self.lanes
        i32 = dict(dtype=torch.int32, device=self.device)
        self.packed = dict(cu_seqlens=torch.empty(L + 1, **i32), seq_lens=torch.empty(L, **i32),
                           positions=torch.empty(T, **i32), slot_mapping=torch.empty(T, **i32),
                           token_lane=torch.empty(T, **i32), active=torch.empty(L + 1, **i32))
        # device copies of the per-step inputs (filled by step_host)
        self.d_lane_tokens = torch.empty(L, **i32)
        self.d_lane_pos = torch.empty(L, **i32)
        self.d_q = torch.empty((T, heads, 576), dtype=torch.bfloat16, device=self.device)
        self.d_kv_new = torch.empty((T, 576), dtype=torch.bfloat16, device=self.device)

    def run(self, lane_tokens, lane_pos, q, kv_new, num_tokens: int, stream=None, out=None, lse=None):
        """One step from device tensors; returns (out, lse) views of the first num_tokens rows
        (written into `out` / `lse` when given, else into the step's own buffers)."""
        out = self.out if out is None else out
        lse = self.lse if lse is None else lse
        s = hk.stream_ptr(stream)
        p = self.packed
        hk.call("hk_pack", hk.ptr(lane_tokens), hk.ptr(lane_pos), hk.ptr(self.block_table),
                self.block_table.shape[1], self.lanes, self.page_size, self.num_pages,
                self.max_tokens, hk.ptr(p["cu_seqlens"]), hk.ptr(p["seq_lens"]),
                hk.ptr(p["positions"]), hk.ptr(p["slot_mapping"]), hk.ptr(p["token_lane"]),
                hk.ptr(p["active"]), s)
        hk.call("hk_kv_append_bf16", hk.ptr(kv_new), hk.ptr(p["slot_mapping"]), num_tokens, 576,
                self.page_size, hk.ptr(self.cache), self.cache.shape[0], s)
        hk.call("hk_mla_decode", hk.ptr(q), hk.ptr(self.cache), hk.ptr(self.block_table),
                self.block_table.shape[1], hk.ptr(p["cu_seqlens"]), hk.ptr(p["positions"]),
                self.lanes, num_tokens, self.heads, self.page_size, self.cache.shape[0],
                self.max_kv_len, self.scale, hk.ptr(out), hk.ptr(lse),
                hk.ptr(self.workspace), self.workspace.numel(), self.impl, s)
        return out[:num_tokens], lse[:num_tokens]

    def attention_only(self, q, num_tokens: int, stream=None):
        """The attention kernel(s) alone on already packed rows (for per-kernel timing)."""
        s = hk.stream_ptr(stream)
        p = self.packed
        hk.call("hk_mla_decode", hk.ptr(q), hk.ptr(self.cache), hk.ptr(self.block_table),
                self.block_table.shape[1], hk.ptr(p["cu_seqlens"]), hk.ptr(p["positions"]),
                self.lanes, num_tokens, self.heads, self.page_size, self.cache.shape[0],
                self.max_kv_len, self.scale, hk.ptr(self.out), hk.ptr(self.lse),
                hk.ptr(self.workspace), self.workspace.numel(), self.impl, s)

    def step_host(self, lane_tokens_h, lane_pos_h, q_h, kv_new_h, out_h, num_tokens: int,
                  stream=None):
        """End to end: pinned host inputs -> device -> kernels -> pinned host output."""
        st = stream if stream is not None else torch.cuda.current_stream()
        with torch.cuda.stream(st):
            self.d_lane_tokens.copy_(lane_tokens_h, non_blocking=True)
            self.d_lane_pos.copy_(lane_pos_h, non_blocking=True)
            self.d_q[:num_tokens].copy_(q_h[:num_tokens], non_blocking=True)
            self.d_kv_new[:num_tokens].copy_(kv_new_h[:num_tokens], non_blocking=True)
            out, _ = self.run(self.d_lane_tokens, self.d_lane_pos, self.d_q, self.d_kv_new,
                              num_tokens, st)
            out_h[:num_tokens].copy_(out, non_blocking=True)

    @staticmethod
    def h2d_bytes(lanes: int, num_tokens: int, heads: int) -> int:
        return 2 * 4 * lanes + num_tokens * heads * 576 * 2 + num_tokens * 576 * 2

    @staticmethod
    def d2h_bytes(num_tokens: int, heads: int) -> int:
        return num_tokens * heads * 512 * 2


class HostPipeline:
    """End-to-end steps from pinned host buffers with the transfers overlapped.

    Step i's inputs go to the device on one copy stream while step i-1's kernels run, and its
    output comes back on a second copy stream while step i+1's kernels run; two device sets
    of inputs and outputs alternate, and events order every reuse.  The kernels of successive
    steps stay in order on one compute stream (each step appends to the cache the next one
    reads).  Every step still copies its own inputs in and its own output out.

        pipe = HostPipeline(step)
        for i in range(n):
            pipe.submit(lane_tokens_h, lane_pos_h, q_h, kv_new_h, out_h[i % 2], T)
        pipe.finish()      # out_h holds the last two steps' outputs
    """

    def __init__(self, step: MlaDecodeStep, compute_stream=None):
        self.step = step
        dev = step.device
        self.compute = compute_stream if compute_stream is not None else torch.cuda.current_stream(dev)
        self.h2d = torch.cuda.Stream(dev)
        self.d2h = torch.cuda.Stream(dev)
        T, H, L = step.max_tokens, step.heads, step.lanes
        i32 = dict(dtype=torch.int32, device=dev)
        self.sets = [dict(lane_tokens=torch.empty(L, **i32), lane_pos=torch.empty(L, **i32),
                          q=torch.empty((T, H, 576), dtype=torch.bfloat16, device=dev),
                          kv_new=torch.empty((T, 576), dtype=torch.bfloat16, device=dev),
                          out=torch.empty((T, H, 512), dtype=torch.bfloat16, device=dev),
                          lse=torch.empty((T, H), dtype=torch.float32, device=dev),
                          ev_in=torch.cuda.Event(), ev_done=torch.cuda.Event(),
                          ev_out=torch.cuda.Event(), used=False) for _ in range(2)]
        self.i = 0

    def submit(self, lane_tokens_h, lane_pos_h, q_h, kv_new_h, out_h, num_tokens: int):
        b = self.sets[self.i % 2]
        self.i += 1
        with torch.cuda.stream(self.h2d):
            if b["used"]:
                self.h2d.wait_event(b["ev_done"])    # the kernels two steps back read these inputs
            b["lane_tokens"].copy_(lane_tokens_h, non_blocking=True)
            b["lane_pos"].copy_(lane_pos_h, non_blocking=True)
            b["q"][:num_tokens].copy_(q_h[:num_tokens], non_blocking=True)
            b["kv_new"][:num_tokens].copy_(kv_new_h[:num_tokens], non_blocking=True)
            b["ev_in"].record(self.h2d)
        self.compute.wait_event(b["ev_in"])
        if b["used"]:
            self.compute.wait_event(b["ev_out"])     # its output buffer has gone to the host
        out, _ = self.step.run(b["lane_tokens"], b["lane_pos"], b["q"], b["kv_new"], num_tokens,
                               self.compute, out=b["out"], lse=b["lse"])
        b["ev_done"].record(self.compute)
        with torch.cuda.stream(self.d2h):
            self.d2h.wait_event(b["ev_done"])
            out_h[:num_tokens].copy_(out, non_blocking=True)
            b["ev_out"].record(self.d2h)
        b["used"] = True

    def finish(self):
        """Waits until every submitted step's output is in its host buffer."""
        self.d2h.synchronize()
        self.compute.synchronize()
