"""CPU oracle for the decode step — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg (and its
`--impl reference` arm) may import this package, and only as the checker or the timed CPU
baseline.  The product (hyperkernel_b200) never imports it and has no CPU fallback.

numpy wrappers over oracle/_build/liboracle.so (hk_oracle.c); engine.py holds the
restatement of the reference's scheduler (src/engine/*.rs) used to pin the C++ engine.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from .build import build as _build

_lib = None


def lib():
    global _lib
    if _lib is None:
        path = _build()
        _lib = C.CDLL(str(path))
        _lib.orc_f32_to_e4m3.restype = C.c_uint8
        _lib.orc_f32_to_e4m3.argtypes = [C.c_float]
        _lib.orc_e4m3_to_f32.restype = C.c_float
        _lib.orc_e4m3_to_f32.argtypes = [C.c_uint8]
        _lib.orc_f32_to_bf16.restype = C.c_uint16
        _lib.orc_f32_to_bf16.argtypes = [C.c_float]
        _lib.orc_sigmoid.restype = C.c_float
        _lib.orc_sigmoid.argtypes = [C.c_float]
        _lib.orc_threads.restype = C.c_int
        _lib.orc_set_threads.restype = C.c_int
        _lib.orc_set_threads.argtypes = [C.c_int]
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def threads() -> int:
    return lib().orc_threads()


def use_all_cores() -> int:
    """OpenMP threads = the CPUs this process may run on (torchrun sets OMP_NUM_THREADS=1)."""
    import os

    n = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    return lib().orc_set_threads(n)


def pack(lane_tokens, lane_pos, block_table, page_size, num_pages, max_tokens):
    lane_tokens = _c(lane_tokens, np.int32)
    lane_pos = _c(lane_pos, np.int32)
    bt = _c(block_table, np.int32)
    L = lane_tokens.shape[0]
    out = dict(
        cu_seqlens=np.zeros(L + 1, np.int32), seq_lens=np.zeros(L, np.int32),
        positions=np.zeros(max_tokens, np.int32), slot_mapping=np.zeros(max_tokens, np.int32),
        token_lane=np.zeros(max_tokens, np.int32), active=np.zeros(L + 1, np.int32))
    err = C.c_int(0)
    lib().orc_pack.restype = C.c_int
    T = lib().orc_pack(_p(lane_tokens), _p(lane_pos), _p(bt), C.c_int(bt.shape[1]), C.c_int(L),
                       C.c_int(page_size), C.c_int(num_pages), C.c_int(max_tokens),
                       _p(out["cu_seqlens"]), _p(out["seq_lens"]), _p(out["positions"]),
                       _p(out["slot_mapping"]), _p(out["token_lane"]), _p(out["active"]),
                       C.byref(err))
    out["num_tokens"] = T
    out["err"] = err.value
    return out


def kv_append_bf16(kv_new, slot, cache, page_rows=64):
    """Writes rows into `cache` ([slots][row] array holding the page-blocked layout when
    page_rows > 0, row-major when 0)."""
    kv_new = _c(kv_new, np.uint16)
    slot = _c(slot, np.int32)
    lib().orc_kv_append_u16.restype = C.c_int
    return lib().orc_kv_append_u16(_p(kv_new), _p(slot), C.c_int(slot.shape[0]),
                                   C.c_int(kv_new.shape[1]), C.c_int(page_rows), _p(cache),
                                   C.c_int64(cache.shape[0]))


def kv_append_fp8(kv_new, slot, cache, scales):
    kv_new = _c(kv_new, np.uint16)
    slot = _c(slot, np.int32)
    lib().orc_kv_append_fp8.restype = C.c_int
    return lib().orc_kv_append_fp8(_p(kv_new), _p(slot), C.c_int(slot.shape[0]),
                                   C.c_int(kv_new.shape[1]), _p(cache), _p(scales),
                                   C.c_int64(cache.shape[0]))


def kv_append_f32(k, v, slot, kc, vc):
    k = _c(k, np.float32)
    v = _c(v, np.float32)
    slot = _c(slot, np.int32)
    lib().orc_kv_append_f32.restype = C.c_int
    return lib().orc_kv_append_f32(_p(k), _p(v), _p(slot), C.c_int(slot.shape[0]),
                                   C.c_int(k.shape[1]), _p(kc), _p(vc), C.c_int64(kc.shape[0]))


def gqa_decode(q, kc, vc, bt, cu, positions, q_heads, kv_heads, head_dim, page_size, scale):
    q = _c(q, np.float32)
    bt = _c(bt, np.int32)
    T = positions.shape[0]
    out = np.zeros((T, q_heads, head_dim), np.float32)
    lse = np.zeros((T, q_heads), np.float32)
    lib().orc_gqa_decode_f32(_p(q), _p(_c(kc, np.float32)), _p(_c(vc, np.float32)), _p(bt),
                             C.c_int(bt.shape[1]), _p(_c(cu, np.int32)),
                             _p(_c(positions, np.int32)), C.c_int(cu.shape[0] - 1), C.c_int(T),
                             C.c_int(q_heads), C.c_int(kv_heads), C.c_int(head_dim),
                             C.c_int(page_size), C.c_float(scale), _p(out), _p(lse))
    return out, lse


def mla_decode(q, bt, cu, positions, page_size, scale, kv_bf16=None, kv_fp8=None, kv_scale=None,
               kv_begin=None, kv_end=None):
    """kv_bf16 is in the page-blocked layout (pages of page_size rows); kv_fp8 row-major."""
    q = _c(q, np.uint16)
    bt = _c(bt, np.int32)
    T, H = q.shape[0], q.shape[1]
    out = np.zeros((T, H, 512), np.float32)
    lse = np.zeros((T, H), np.float32)
    lib().orc_mla_decode(
        _p(q), _p(None if kv_bf16 is None else _c(kv_bf16, np.uint16)),
        _p(None if kv_fp8 is None else _c(kv_fp8, np.uint8)),
        _p(None if kv_scale is None else _c(kv_scale, np.float32)), _p(bt), C.c_int(bt.shape[1]),
        _p(_c(cu, np.int32)), _p(_c(positions, np.int32)),
        _p(None if kv_begin is None else _c(kv_begin, np.int32)),
        _p(None if kv_end is None else _c(kv_end, np.int32)), C.c_int(cu.shape[0] - 1),
        C.c_int(T), C.c_int(H), C.c_int(page_size), C.c_float(scale), _p(out), _p(lse))
    return out, lse


def lse_merge(o_parts, lse_parts):
    o_parts = _c(o_parts, np.float32)
    lse_parts = _c(lse_parts, np.float32)
    n, rows, dv = o_parts.shape
    out = np.zeros((rows, dv), np.float32)
    lse = np.zeros(rows, np.float32)
    lib().orc_lse_merge(_p(o_parts), _p(lse_parts), C.c_int(n), C.c_int64(rows), C.c_int(dv),
                        _p(out), _p(lse))
    return out, lse


def quant_fp8(x_bf16):
    x = _c(x_bf16, np.uint16)
    rows, k = x.shape
    xq = np.zeros((rows, k), np.uint8)
    sx = np.zeros((rows, k // 128), np.float32)
    lib().orc_quant_fp8(_p(x), C.c_int64(rows), C.c_int(k), _p(xq), _p(sx))
    return xq, sx


def gemm_fp8(xq, sx, wq, sw):
    xq = _c(xq, np.uint8)
    wq = _c(wq, np.uint8)
    m, k = xq.shape
    n = wq.shape[0]
    y = np.zeros((m, n), np.float32)
    lib().orc_gemm_fp8(_p(xq), _p(_c(sx, np.float32)), _p(wq), _p(_c(sw, np.float32)),
                       C.c_int64(m), C.c_int(n), C.c_int(k), _p(y))
    return y


def route(logits, bias, top_k, route_scale):
    logits = _c(logits, np.float32)
    T, E = logits.shape
    ids = np.zeros((T, top_k), np.int32)
    w = np.zeros((T, top_k), np.float32)
    lib().orc_route(_p(logits), _p(None if bias is None else _c(bias, np.float32)), C.c_int(T),
                    C.c_int(E), C.c_int(top_k), C.c_float(route_scale), _p(ids), _p(w))
    return ids, w


def permute(ids, weights, num_experts):
    ids = _c(ids, np.int32)
    weights = _c(weights, np.float32)
    T, K = ids.shape
    P = T * K
    offsets = np.zeros(num_experts + 1, np.int32)
    perm_token = np.zeros(P, np.int32)
    perm_weight = np.zeros(P, np.float32)
    inv = np.zeros(P, np.int32)
    lib().orc_permute(_p(ids), _p(weights), C.c_int(T), C.c_int(K), C.c_int(num_experts),
                      _p(offsets), _p(perm_token), _p(perm_weight), _p(inv))
    return offsets, perm_token, perm_weight, inv


def moe_grouped(xq, sx, offsets, perm_token, hidden, inter, w13, s13, w2, s2):
    offsets = _c(offsets, np.int32)
    E = offsets.shape[0] - 1
    P = int(offsets[-1])
    y = np.zeros((P, hidden), np.float32)
    lib().orc_moe_grouped(_p(_c(xq, np.uint8)), _p(_c(sx, np.float32)), _p(offsets),
                          _p(_c(perm_token, np.int32)), C.c_int(E), C.c_int(hidden),
                          C.c_int(inter), _p(_c(w13, np.uint8)), _p(_c(s13, np.float32)),
                          _p(_c(w2, np.uint8)), _p(_c(s2, np.float32)), _p(y))
    return y


def combine(y_bf16, perm_weight, inv, shared_bf16, tokens, top_k):
    y = _c(y_bf16, np.uint16)
    hidden = y.shape[1]
    out = np.zeros((tokens, hidden), np.float32)
    lib().orc_combine(_p(y), _p(_c(perm_weight, np.float32)), _p(_c(inv, np.int32)),
                      _p(None if shared_bf16 is None else _c(shared_bf16, np.uint16)),
                      C.c_int(tokens), C.c_int(top_k), C.c_int(hidden), _p(out))
    return out


def rope_table(rows, dim, base, original_seq_len, factor, beta_fast, beta_slow):
    t = np.zeros((rows, dim), np.float32)
    lib().orc_rope_table(C.c_int64(rows), C.c_int(dim), C.c_float(base),
                         C.c_int(original_seq_len), C.c_float(factor), C.c_float(beta_fast),
                         C.c_float(beta_slow), _p(t))
    return t


def e4m3_to_f32(v: int) -> float:
    return lib().orc_e4m3_to_f32(v)


def f32_to_e4m3(x: float) -> int:
    return lib().orc_f32_to_e4m3(x)


def sigmoid(x: float) -> float:
    return lib().orc_sigmoid(x)
