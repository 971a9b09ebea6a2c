"""ctypes binding of libhk.so (include/hk.h) and thin torch-tensor wrappers.

The library is the product: every call below runs a CUDA kernel of libhk.so on the
caller's stream.  There is no CPU fallback — if libhk.so is missing or the device is not an
sm_100 part, calls raise HKError.  torch is used only for device memory and streams.
"""
from __future__ import annotations

import ctypes as C
import os
import re
from pathlib import Path

import numpy as np
import torch

PKG = Path(__file__).resolve().parent
# HK_LIB_PATH selects another build of the same library (A/B timing of kernel variants).
LIB_PATH = Path(os.environ.get("HK_LIB_PATH", PKG / "libhk.so"))
HEADER = PKG.parent / "include" / "hk.h"

HK_OK, HK_EINVAL, HK_ENODEV, HK_ECUDA, HK_EDEVICE, HK_ESPACE, HK_ESTATE = 0, -1, -2, -3, -4, -5, -6

P, I32, I64, F32, SZ, U64 = C.c_void_p, C.c_int32, C.c_int64, C.c_float, C.c_size_t, C.c_uint64

# Prototypes of every entry point in include/hk.h (kept in header order).
SIGNATURES = {
    "hk_version": (C.c_char_p, []),
    "hk_last_error": (C.c_char_p, []),
    "hk_device_info": (C.c_int, [P, P, P]),
    "hk_kernel_launches": (C.c_uint64, []),
    "hk_check_errors": (C.c_int, []),
    "hk_pack": (C.c_int, [P, P, P, I32, I32, I32, I32, I32, P, P, P, P, P, P, P]),
    "hk_kv_append_bf16": (C.c_int, [P, P, I32, I32, I32, P, I64, P]),
    "hk_kv_append_fp8": (C.c_int, [P, P, I32, I32, P, P, I64, P]),
    "hk_kv_dequant_fp8": (C.c_int, [P, P, I64, I32, I32, P, I64, P, P]),
    "hk_kv_dequant_fp8_rows": (C.c_int, [P, P, I64, I32, I32, P, I64, P, P]),
    "hk_pages_within": (C.c_int, [P, U64, P, P]),
    "hk_plan_pools": (C.c_int, [P, P, P, P, P, P]),
    "hk_kv_append_f32": (C.c_int, [P, P, P, I32, I32, P, P, I64, P]),
    "hk_gqa_decode_f32": (C.c_int, [P, P, P, P, I32, P, P, I32, I32, I32, I32, I32, I32, I64, F32, P, P, P]),
    "hk_mla_workspace_size": (SZ, [I32, I32, I32, I32]),
    "hk_mla_decode": (C.c_int, [P, P, P, I32, P, P, I32, I32, I32, I32, I64, I32, F32, P, P, P, SZ, I32, P]),
    "hk_mla_decode_fp8": (C.c_int, [P, P, P, P, I32, P, P, I32, I32, I32, I32, I64, I32, F32, P, P, P, SZ, P]),
    "hk_mla_partial_fp8": (C.c_int, [P, P, P, P, I32, P, P, P, P, I32, I32, I32, I32, I64, I32, F32, P, P, P, SZ, P]),
    "hk_mla_partial": (C.c_int, [P, P, P, I32, P, P, P, P, I32, I32, I32, I32, I64, I32, F32, P, P, P, SZ, P]),
    "hk_lse_merge": (C.c_int, [P, P, I32, I64, I32, P, P, P]),
    "hk_sample_workspace_size": (SZ, [I32, I32]),
    "hk_sample_verify": (C.c_int, [P, I32, P, I32, I32, I32, P, P, P, I32, P, P, P, SZ, P]),
    "hk_quant_fp8": (C.c_int, [P, I64, I32, P, P, P]),
    "hk_gemm_fp8": (C.c_int, [P, P, P, P, I64, I32, I32, P, P]),
    "hk_route": (C.c_int, [P, P, I32, I32, I32, F32, P, P, P]),
    "hk_permute": (C.c_int, [P, P, I32, I32, I32, P, P, P, P, P]),
    "hk_moe_workspace_size": (SZ, [I64, I32, I32]),
    "hk_moe_grouped": (C.c_int, [P, P, I32, P, P, I64, I32, I32, I32, P, P, P, P, P, P, SZ, P]),
    "hk_moe_grouped_noalloc": (C.c_int, [P, P, I32, P, P, I64, I32, I32, I32, P, P, P, P, P, P]),
    "hk_gather_rows": (C.c_int, [P, I64, P, I64, I32, P, P]),
    "hk_scatter_rows": (C.c_int, [P, I64, P, I64, I32, P, P]),
    "hk_ep_counts": (C.c_int, [P, I32, I32, I32, P, P, C.c_uint32, I32, P, P, P, P]),
    "hk_ep_dispatch": (C.c_int, [P, P, I32, P, P, I32, I32, I32, I32, I32, I32, P, P, P, P, P, C.c_uint32, P]),
    "hk_ep_return": (C.c_int, [P, I32, I32, I32, I32, P, P, P, I32, I32, P, P, P, C.c_uint32, P]),
    "hk_ep_wait": (C.c_int, [P, I32, I32, C.c_uint32, I32, P]),
    "hk_sym_alloc": (C.c_int, [SZ, P, P]),
    "hk_sym_import": (C.c_int, [P, P]),
    "hk_sym_close": (C.c_int, [P]),
    "hk_sym_free": (C.c_int, [P]),
    "hk_cp_merge": (C.c_int, [P, P, P, I32, I32, C.c_uint32, I32, I64, I32, P, P, P]),
    "hk_combine": (C.c_int, [P, I64, P, P, P, I32, I32, I32, P, P]),
    "hk_open": (C.c_int, [P, P]),
    "hk_open_mla": (C.c_int, [P, P, P]),
    "hk_model_tensor": (C.c_int, [P, C.c_uint32, C.c_char_p, P, P]),
    "hk_close": (None, [P]),
    "hk_pools": (C.c_int, [P, P, P]),
    "hk_push": (C.c_int, [P, P]),
    "hk_drain": (C.c_int, [P, P, SZ, P, P, SZ, P]),
    "hk_drain_logprobs": (C.c_int, [P, P, SZ, P, P, SZ, P]),
    "hk_encode_share": (C.c_int, [P, P, P, SZ, P]),
    "hk_kernel_ops_of": (C.c_int, [P, P]),
    "hk_engine_defaults": (None, [P]),
    "hk_engine_create": (C.c_int, [P, P, P]),
    "hk_engine_destroy": (None, [P]),
    "hk_engine_submit": (C.c_int, [P, P, SZ, P, U64, P, SZ, P]),
    "hk_engine_reset": (C.c_int, [P, P]),
    "hk_engine_reset_answer": (C.c_int, [P, U64, I64, P]),
    "hk_engine_close": (C.c_int, [P]),
    "hk_engine_run": (C.c_int, [P]),
    "hk_engine_hangup": (C.c_int, [P, U64]),
    "hk_engine_outputs": (C.c_int, [P, U64, I64, P, SZ, P, P, SZ]),
    "hk_engine_outputs_lp": (C.c_int, [P, U64, I64, P, SZ, P, P, SZ, P, SZ, P]),
    "hk_engine_metrics": (C.c_int, [P, P, P, SZ, P, P, SZ, P]),
    "hk_rope_table": (C.c_int, [I64, I32, F32, I32, F32, F32, F32, P]),
}


class HKError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"hk error {code}: {msg}")
        self.code = code


_lib = None


def lib() -> C.CDLL:
    """Loads libhk.so (raises if it was not built: there is no fallback)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise HKError(HK_ENODEV, f"{LIB_PATH} is not built; run python -m hyperkernel_b200.build")
        L = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def header_functions() -> list[str]:
    """Names of the functions declared in include/hk.h."""
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return re.findall(r"^\s*(?:const\s+)?[a-z_0-9]+\s*\*?\s*(hk_[a-z_0-9]+)\s*\(", text, flags=re.M)


def last_error() -> str:
    return lib().hk_last_error().decode()


def check(rc: int) -> None:
    if rc != HK_OK:
        raise HKError(rc, last_error())


def ptr(t):
    """Device address of a tensor (None -> NULL)."""
    if t is None:
        return None
    if isinstance(t, int):
        return t
    assert t.is_cuda and t.is_contiguous(), "tensors passed to libhk must be contiguous CUDA tensors"
    return t.data_ptr()


def stream_ptr(stream=None):
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args))


def check_errors() -> None:
    """Raises if any kernel recorded bad input on the current device (synchronises)."""
    check(lib().hk_check_errors())


def device_info():
    sm, ma, mi = C.c_int(), C.c_int(), C.c_int()
    check(lib().hk_device_info(C.byref(sm), C.byref(ma), C.byref(mi)))
    return sm.value, ma.value, mi.value


def kernel_launches() -> int:
    """Kernels libhk.so has launched in this process."""
    return lib().hk_kernel_launches()


def version() -> str:
    return lib().hk_version().decode()


def _u16(t):
    """bf16 tensor viewed as its bit pattern (no copy)."""
    return t.view(torch.int16) if t.dtype == torch.bfloat16 else t


# ------------------------------------------------------------------------------------------
# Kernel wrappers (all tensors on the current CUDA device, contiguous)
# ------------------------------------------------------------------------------------------

def pack(lane_tokens, lane_pos, block_table, page_size, num_pages, max_tokens, stream=None):
    dev = lane_tokens.device
    L = lane_tokens.shape[0]
    o = dict(
        cu_seqlens=torch.empty(L + 1, dtype=torch.int32, device=dev),
        seq_lens=torch.empty(L, dtype=torch.int32, device=dev),
        positions=torch.empty(max(max_tokens, 1), dtype=torch.int32, device=dev),
        slot_mapping=torch.empty(max(max_tokens, 1), dtype=torch.int32, device=dev),
        token_lane=torch.empty(max(max_tokens, 1), dtype=torch.int32, device=dev),
        active=torch.empty(L + 1, dtype=torch.int32, device=dev))
    call("hk_pack", ptr(lane_tokens), ptr(lane_pos), ptr(block_table), block_table.shape[1], L,
         page_size, num_pages, max_tokens, ptr(o["cu_seqlens"]), ptr(o["seq_lens"]),
         ptr(o["positions"]), ptr(o["slot_mapping"]), ptr(o["token_lane"]), ptr(o["active"]),
         stream_ptr(stream))
    return o


def kv_append_bf16(kv_new, slot_mapping, kv_cache, num_tokens=None, page_rows=64, stream=None):
    """Appends rows into the page-blocked latent cache (page_rows=0: a row-major cache)."""
    n = kv_new.shape[0] if num_tokens is None else num_tokens
    call("hk_kv_append_bf16", ptr(kv_new), ptr(slot_mapping), n, kv_new.shape[-1], page_rows,
         ptr(kv_cache), kv_cache.shape[0], stream_ptr(stream))


def kv_append_fp8(kv_new, slot_mapping, kv_cache, kv_scale, num_tokens=None, stream=None):
    n = kv_new.shape[0] if num_tokens is None else num_tokens
    call("hk_kv_append_fp8", ptr(kv_new), ptr(slot_mapping), n, kv_new.shape[-1], ptr(kv_cache),
         ptr(kv_scale), kv_cache.shape[0], stream_ptr(stream))


def kv_dequant_fp8_rows(kv_cache, kv_scale, slots, out, page_rows=64, stream=None):
    """Refreshes the rows `slots` (int32 device tensor) of the bf16 mirror `out`."""
    slots_n, row = kv_cache.shape
    call("hk_kv_dequant_fp8_rows", ptr(kv_cache), ptr(kv_scale), slots_n, row, page_rows, ptr(slots),
         slots.shape[0], ptr(_u16(out)), stream_ptr(stream))
    return out


def kv_dequant_fp8(kv_cache, kv_scale, page_rows=64, out=None, pages=None, stream=None):
    """The FP8 cache [slots][576] as the page-blocked bf16 cache of hk_mla_decode (only the
    pages listed in `pages`, an int32 device tensor, when given)."""
    slots, row = kv_cache.shape
    if out is None:
        out = torch.empty((slots, row), dtype=torch.bfloat16, device=kv_cache.device)
    n = 0 if pages is None else pages.shape[0]
    call("hk_kv_dequant_fp8", ptr(kv_cache), ptr(kv_scale), slots, row, page_rows, ptr(pages), n,
         ptr(_u16(out)), stream_ptr(stream))
    return out


def kv_append_f32(k_new, v_new, slot_mapping, k_cache, v_cache, stream=None):
    row = k_new[0].numel() if k_new.shape[0] else 4
    call("hk_kv_append_f32", ptr(k_new), ptr(v_new), ptr(slot_mapping), k_new.shape[0], row,
         ptr(k_cache), ptr(v_cache), k_cache.shape[0], stream_ptr(stream))


def gqa_decode(q, k_cache, v_cache, block_table, cu_seqlens, positions, kv_heads, page_size,
               scale, stream=None):
    T, qh, D = q.shape
    out = torch.empty_like(q)
    lse = torch.empty((T, qh), dtype=torch.float32, device=q.device)
    call("hk_gqa_decode_f32", ptr(q), ptr(k_cache), ptr(v_cache), ptr(block_table),
         block_table.shape[1], ptr(cu_seqlens), ptr(positions), cu_seqlens.shape[0] - 1, T, qh,
         kv_heads, D, page_size, k_cache.shape[0], scale, ptr(out), ptr(lse), stream_ptr(stream))
    return out, lse


def mla_workspace_size(num_lanes, num_tokens, heads, max_kv_len) -> int:
    return lib().hk_mla_workspace_size(num_lanes, num_tokens, heads, max_kv_len)


def mla_decode(q, kv_cache, block_table, cu_seqlens, positions, page_size, max_kv_len, scale,
               out=None, lse=None, workspace=None, impl=0, stream=None):
    T, H, _ = q.shape
    dev = q.device
    if out is None:
        out = torch.empty((T, H, 512), dtype=torch.bfloat16, device=dev)
    if lse is None:
        lse = torch.empty((T, H), dtype=torch.float32, device=dev)
    L = cu_seqlens.shape[0] - 1
    if workspace is None:
        ws = mla_workspace_size(L, T, H, max_kv_len)
        workspace = torch.empty(max(ws, 16), dtype=torch.uint8, device=dev)
    call("hk_mla_decode", ptr(q), ptr(kv_cache), ptr(block_table), block_table.shape[1],
         ptr(cu_seqlens), ptr(positions), L, T, H, page_size, kv_cache.shape[0], max_kv_len, scale,
         ptr(out), ptr(lse), ptr(workspace), workspace.numel(), impl, stream_ptr(stream))
    return out, lse


def mla_decode_fp8(q, kv_cache, kv_scale, block_table, cu_seqlens, positions, page_size,
                   max_kv_len, scale, stream=None):
    T, H, _ = q.shape
    dev = q.device
    out = torch.empty((T, H, 512), dtype=torch.bfloat16, device=dev)
    lse = torch.empty((T, H), dtype=torch.float32, device=dev)
    L = cu_seqlens.shape[0] - 1
    ws = mla_workspace_size(L, T, H, max_kv_len)
    workspace = torch.empty(max(ws, 16), dtype=torch.uint8, device=dev)
    call("hk_mla_decode_fp8", ptr(q), ptr(kv_cache), ptr(kv_scale), ptr(block_table),
         block_table.shape[1], ptr(cu_seqlens), ptr(positions), L, T, H, page_size,
         kv_cache.shape[0], max_kv_len, scale, ptr(out), ptr(lse), ptr(workspace),
         workspace.numel(), stream_ptr(stream))
    return out, lse


def mla_partial_fp8(q, kv_cache, kv_scale, block_table, cu_seqlens, positions, kv_begin, kv_end,
                    page_size, max_kv_len, scale, stream=None):
    T, H, _ = q.shape
    dev = q.device
    o = torch.empty((T, H, 512), dtype=torch.float32, device=dev)
    lse = torch.empty((T, H), dtype=torch.float32, device=dev)
    L = cu_seqlens.shape[0] - 1
    ws = mla_workspace_size(L, T, H, max_kv_len)
    workspace = torch.empty(max(ws, 16), dtype=torch.uint8, device=dev)
    call("hk_mla_partial_fp8", ptr(q), ptr(kv_cache), ptr(kv_scale), ptr(block_table),
         block_table.shape[1], ptr(cu_seqlens), ptr(positions), ptr(kv_begin), ptr(kv_end), L, T,
         H, page_size, kv_cache.shape[0], max_kv_len, scale, ptr(o), ptr(lse), ptr(workspace),
         workspace.numel(), stream_ptr(stream))
    return o, lse


def mla_partial(q, kv_cache, block_table, cu_seqlens, positions, kv_begin, kv_end, page_size, max_kv_len,
                scale, stream=None, out=None, lse=None):
    """Partial attention of KV ranges on the tcgen05 kernel over the page-blocked bf16 cache:
    fp32 o [T, H, 512] normalised within the range, lse [T, H] (-inf where it is empty), into
    `out` / `lse` when given (e.g. a context-parallel exchange buffer)."""
    T, H, _ = q.shape
    dev = q.device
    o = out if out is not None else torch.empty((T, H, 512), dtype=torch.float32, device=dev)
    lse = lse if lse is not None else torch.empty((T, H), dtype=torch.float32, device=dev)
    L = cu_seqlens.shape[0] - 1
    ws = mla_workspace_size(L, T, H, max_kv_len)
    workspace = torch.empty(max(ws, 16), dtype=torch.uint8, device=dev)
    call("hk_mla_partial", ptr(q), ptr(_u16(kv_cache)), ptr(block_table), block_table.shape[1],
         ptr(cu_seqlens), ptr(positions), ptr(kv_begin), ptr(kv_end), L, T, H, page_size,
         kv_cache.shape[0], max_kv_len, scale, ptr(o), ptr(lse), ptr(workspace), workspace.numel(),
         stream_ptr(stream))
    return o, lse


SAMPLING_DTYPE = np.dtype([("temperature", "<f4"), ("top_p", "<f4"), ("top_k", "<u4"),
                           ("logprobs", "<u4"), ("seed", "<u8")])


def sampling_array(samplings, device):
    """hk_sampling[] on the device from dicts with temperature, top_p, top_k (logprobs, seed)."""
    a = np.zeros(len(samplings), SAMPLING_DTYPE)
    for i, sm in enumerate(samplings):
        a[i] = (sm["temperature"], sm["top_p"], sm["top_k"], sm.get("logprobs", 0), sm.get("seed", 0))
    return torch.from_numpy(a.view(np.uint8).copy()).to(device)


def sample_verify(logits, cu_rows, sampling, state, drafts, block, n_logprobs, stream=None):
    """Draws and verifies every lane's rows: returns (ids [lanes, block], lp [lanes, block,
    2n+1]); `state` (uint64 stored as int64, one per lane) advances in place."""
    rows, vocab = logits.shape
    lanes = cu_rows.shape[0] - 1
    dev = logits.device
    ids = torch.empty((lanes, block), dtype=torch.int32, device=dev)
    lp = torch.empty((lanes, block, 2 * n_logprobs + 1), dtype=torch.float32, device=dev)
    ws = lib().hk_sample_workspace_size(rows, vocab)
    workspace = torch.empty(ws, dtype=torch.uint8, device=dev)
    call("hk_sample_verify", ptr(logits), vocab, ptr(cu_rows), lanes, rows, block, ptr(sampling), ptr(state),
         ptr(drafts), n_logprobs, ptr(ids), ptr(lp) if n_logprobs > 0 else None, ptr(workspace),
         workspace.numel(), stream_ptr(stream))
    return ids, lp


def lse_merge(o_parts, lse_parts, stream=None):
    n, rows, dv = o_parts.shape
    out = torch.empty((rows, dv), dtype=torch.bfloat16, device=o_parts.device)
    lse = torch.empty(rows, dtype=torch.float32, device=o_parts.device)
    call("hk_lse_merge", ptr(o_parts), ptr(lse_parts), n, rows, dv, ptr(out), ptr(lse),
         stream_ptr(stream))
    return out, lse


def quant_fp8(x, stream=None):
    rows, k = x.shape
    xq = torch.empty((rows, k), dtype=torch.uint8, device=x.device)
    sx = torch.empty((rows, k // 128), dtype=torch.float32, device=x.device)
    call("hk_quant_fp8", ptr(x), rows, k, ptr(xq), ptr(sx), stream_ptr(stream))
    return xq, sx


def gemm_fp8(xq, sx, wq, sw, out=None, stream=None):
    m, k = xq.shape
    n = wq.shape[0]
    if out is None:
        out = torch.empty((m, n), dtype=torch.bfloat16, device=xq.device)
    call("hk_gemm_fp8", ptr(xq), ptr(sx), ptr(wq), ptr(sw), m, n, k, ptr(out), stream_ptr(stream))
    return out


def route(logits, bias, top_k, route_scale, stream=None):
    T, E = logits.shape
    ids = torch.empty((T, top_k), dtype=torch.int32, device=logits.device)
    w = torch.empty((T, top_k), dtype=torch.float32, device=logits.device)
    call("hk_route", ptr(logits), ptr(bias), T, E, top_k, route_scale, ptr(ids), ptr(w),
         stream_ptr(stream))
    return ids, w


def permute(ids, weights, num_experts, stream=None, offsets=None, perm_token=None):
    """`offsets` / `perm_token` may be given as contiguous views of larger buffers (the first
    num_experts + 1 and T * K entries are written)."""
    T, K = ids.shape
    dev = ids.device
    if offsets is None:
        offsets = torch.empty(num_experts + 1, dtype=torch.int32, device=dev)
    if perm_token is None:
        perm_token = torch.empty(max(T * K, 1), dtype=torch.int32, device=dev)
    if offsets.numel() < num_experts + 1 or perm_token.numel() < T * K:
        raise ValueError("permute: output buffers too small")
    perm_weight = torch.empty(max(T * K, 1), dtype=torch.float32, device=dev)
    inv = torch.empty(max(T * K, 1), dtype=torch.int32, device=dev)
    call("hk_permute", ptr(ids), ptr(weights), T, K, num_experts, ptr(offsets), ptr(perm_token),
         ptr(perm_weight), ptr(inv), stream_ptr(stream))
    return offsets, perm_token, perm_weight, inv


def moe_workspace_size(rows, hidden, inter) -> int:
    return lib().hk_moe_workspace_size(rows, hidden, inter)


def moe_grouped(xq, sx, offsets, perm_token, rows, hidden, inter, w13, s13, w2, s2, out=None,
                workspace=None, stream=None):
    E = offsets.shape[0] - 1
    dev = xq.device
    if out is None:
        out = torch.empty((max(rows, 1), hidden), dtype=torch.bfloat16, device=dev)
    if workspace is None:
        workspace = torch.empty(moe_workspace_size(max(rows, 1), hidden, inter), dtype=torch.uint8, device=dev)
    call("hk_moe_grouped", ptr(xq), ptr(sx), xq.shape[0], ptr(offsets), ptr(perm_token), rows, E,
         hidden, inter, ptr(w13), ptr(s13), ptr(w2), ptr(s2), ptr(out), ptr(workspace),
         workspace.numel(), stream_ptr(stream))
    return out


def moe_grouped_noalloc(xq, sx, offsets, perm_token, rows, hidden, inter, w13, s13, w2, s2,
                        out=None, stream=None):
    """hk_moe_grouped with the library's fixed scratch array (no workspace argument)."""
    E = offsets.shape[0] - 1
    if out is None:
        out = torch.empty((max(rows, 1), hidden), dtype=torch.bfloat16, device=xq.device)
    call("hk_moe_grouped_noalloc", ptr(xq), ptr(sx), xq.shape[0], ptr(offsets), ptr(perm_token),
         rows, E, hidden, inter, ptr(w13), ptr(s13), ptr(w2), ptr(s2), ptr(out),
         stream_ptr(stream))
    return out


def gather_rows(src, idx, out=None, stream=None):
    """out[i] = src[idx[i]] (rows of src as bytes; 16-byte multiples)."""
    rows = idx.shape[0]
    if out is None:
        out = torch.empty((rows,) + tuple(src.shape[1:]), dtype=src.dtype, device=src.device)
    row_bytes = src[0].numel() * src.element_size() if src.shape[0] else out[0].numel() * out.element_size()
    call("hk_gather_rows", ptr(src), src.shape[0], ptr(idx), rows, row_bytes, ptr(out), stream_ptr(stream))
    return out


def scatter_rows(src, idx, out, stream=None):
    """out[idx[i]] = src[i]."""
    rows = idx.shape[0]
    row_bytes = out[0].numel() * out.element_size()
    call("hk_scatter_rows", ptr(src), rows, ptr(idx), out.shape[0], row_bytes, ptr(out), stream_ptr(stream))
    return out


def combine(y, perm_weight, inv, shared, tokens, top_k, out=None, stream=None):
    hidden = y.shape[1]
    if out is None:
        out = torch.empty((tokens, hidden), dtype=torch.bfloat16, device=y.device)
    call("hk_combine", ptr(y), y.shape[0], ptr(perm_weight), ptr(inv), ptr(shared), tokens, top_k,
         hidden, ptr(out), stream_ptr(stream))
    return out


def rope_table(rows, dim, base, original_seq_len, factor, beta_fast, beta_slow):
    """Host-side table (numpy float32 [rows][dim]); needs no GPU."""
    import numpy as np

    t = np.zeros((rows, dim), np.float32)
    check(lib().hk_rope_table(rows, dim, base, original_seq_len, factor, beta_fast, beta_slow,
                              t.ctypes.data_as(C.c_void_p)))
    return t


# ---- pool sizing (host arithmetic; hk_plan_pools reads cudaMemGetInfo when free == 0) ----

UNIT_PAGE, UNIT_WINDOW = 0, 1


class PoolStateC(C.Structure):
    _fields_ = [("home", C.c_uint32), ("unit", C.c_uint32), ("bytes", C.c_uint64)]


class PoolSizingC(C.Structure):
    _fields_ = [("pages", C.c_uint64), ("window_pages", C.c_uint64), ("entries", C.c_uint64),
                ("slots", C.c_uint64), ("states", C.POINTER(PoolStateC)), ("n_states", C.c_size_t)]


class PoolBudgetC(C.Structure):
    _fields_ = [("free", C.c_uint64), ("other", C.c_uint64), ("slack", C.c_uint64),
                ("lanes", C.c_uint32), ("context", C.c_uint32), ("device", C.c_int32),
                ("reserved", C.c_uint32)]


def _pool_c(pages, window_pages, entries, slots, states):
    arr = (PoolStateC * max(len(states), 1))(*[PoolStateC(h, u, b) for h, u, b in states])
    return PoolSizingC(pages, window_pages, entries, slots, arr, len(states)), arr


def pages_within(pages, window_pages, entries, states, nbytes, slots=0):
    """(pages, window_pages) for a pool of `states` [(home, unit, bytes per unit)] within
    `nbytes`, or None when the bytes hold no sequence (src/gpu/load.rs:903-908)."""
    pool, _keep = _pool_c(pages, window_pages, entries, slots, states)
    n, w = C.c_size_t(), C.c_size_t()
    rc = lib().hk_pages_within(C.byref(pool), nbytes, C.byref(n), C.byref(w))
    if rc == HK_ESPACE:
        return None
    check(rc)
    return n.value, w.value


def plan_pools(pages, window_pages, entries, slots, states, *, lanes, context, other=0, slack=0,
               free=0, device=0):
    """(pages, window_pages, slots, used bytes) of the loader's pool plan; free = 0 reads the
    device's free memory.  Raises HKError with the reference's wording."""
    pool, _keep = _pool_c(pages, window_pages, entries, slots, states)
    b = PoolBudgetC(free, other, slack, lanes, context, device, 0)
    n, w, sl, used = C.c_size_t(), C.c_size_t(), C.c_size_t(), C.c_uint64()
    check(lib().hk_plan_pools(C.byref(pool), C.byref(b), C.byref(n), C.byref(w), C.byref(sl),
                              C.byref(used)))
    return n.value, w.value, sl.value, used.value
