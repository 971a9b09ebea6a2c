"""Test infrastructure only: CPU restatement of the HK_MODEL_MLA decoder (numpy + the C oracle).

Only tests/, __graft_entry__.smoke() and bench.py's CPU baseline may use this module, and only
as the checker.

The reference's LLM step runs inside closed sm_103a code, so nothing in the reference pins this
decoder's numerics: the restatement follows the layer math include/hk.h states for
hk_mla_model, with the same rounding points as the device (bf16 after every GEMM, bf16 residual
stream, e4m3 1x128 activation quantisation before every projection) and fp64 accumulation
inside the GEMMs, the attention and the expert FFNs.  `logits(weights, tokens)` gives the
logits of every position of one sequence (causal), which is what the device computes for the
same tokens whether they arrived as prompt chunks or as verified decode rows.
"""
from __future__ import annotations

import math

import numpy as np

from . import combine, gemm_fp8, moe_grouped, permute, quant_fp8, route

HEADS, LATENT, ROPE, ROW = 128, 512, 64, 576


def bf16(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 (round to nearest even) -> fp32."""
    b = np.ascontiguousarray(x, np.float32).view(np.uint32)
    r = ((b + np.uint32(0x7FFF) + ((b >> np.uint32(16)) & np.uint32(1))) & np.uint32(0xFFFF0000))
    return r.view(np.float32)


def bf16_bits(x: np.ndarray) -> np.ndarray:
    return (bf16(x).view(np.uint32) >> np.uint32(16)).astype(np.uint16)


def from_bf16_bits(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def _e4m3_table() -> np.ndarray:
    """The 127 finite non-negative e4m3 values, ascending (code = index)."""
    vals = []
    for code in range(0x7F):
        e, m = code >> 3, code & 7
        vals.append(m * 2.0 ** -9 if e == 0 else (1 + m / 8.0) * 2.0 ** (e - 7))
    return np.array(vals, np.float64)


_E4M3 = _e4m3_table()


def e4m3(x: np.ndarray) -> np.ndarray:
    """fp32 -> e4m3 bytes, round to nearest (ties to the even code), saturating at 448."""
    x = np.asarray(x, np.float32)
    a = np.minimum(np.abs(x).astype(np.float64), 448.0)
    hi = np.clip(np.searchsorted(_E4M3, a, side="left"), 0, 126)
    lo = np.clip(hi - 1, 0, 126)
    dlo, dhi = a - _E4M3[lo], _E4M3[hi] - a
    pick_hi = (dhi < dlo) | ((dhi == dlo) & (hi % 2 == 0))
    code = np.where(pick_hi, hi, lo).astype(np.uint8)
    return code | (np.signbit(x).astype(np.uint8) << 7)


def rms_quant(v: np.ndarray):
    """rmsnorm (no gain, eps 1e-6) then 1x128 e4m3 blocks: (q [rows][H], s [rows][H/128])."""
    v = np.asarray(v, np.float32)
    rows, H = v.shape
    ms = (v.astype(np.float64) ** 2).mean(axis=1).astype(np.float32)
    inv = np.float32(1.0) / np.sqrt(ms + np.float32(1e-6))
    n = (v * inv[:, None]).astype(np.float32)
    blk = n.reshape(rows, H // 128, 128)
    s = (np.maximum(np.abs(blk).max(axis=2), np.float32(1e-12)) / np.float32(448.0)).astype(np.float32)
    q = e4m3((blk / s[:, :, None]).astype(np.float32)).reshape(rows, H)
    return q, s


def _rot(a: np.ndarray, b: np.ndarray, c: np.ndarray, s: np.ndarray):
    return bf16(a * c - b * s), bf16(a * s + b * c)


def rope(n: int, theta: float):
    """cos, sin [n][32] of position * theta^(-i/32) (angles in double)."""
    f = np.array([math.pow(theta, -i / 32.0) for i in range(32)])
    ang = np.arange(n, dtype=np.float64)[:, None] * f[None, :]
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def attention(q: np.ndarray, kv: np.ndarray) -> np.ndarray:
    """Causal absorbed MLA over one sequence: q [L][128][576], kv [L][576] -> o [L][128][512]
    (fp64 softmax and sums, scale 1/sqrt(576))."""
    L = q.shape[0]
    qd, kd = q.astype(np.float64), kv.astype(np.float64)
    s = np.einsum("ihd,jd->hij", qd, kd) / math.sqrt(ROW)
    s = np.where(np.tril(np.ones((L, L), bool))[None], s, -np.inf)
    s -= s.max(axis=2, keepdims=True)
    p = np.exp(s)
    p /= p.sum(axis=2, keepdims=True)
    return np.einsum("hij,jd->ihd", p, kd[:, :LATENT]).astype(np.float32)


def logits(w: dict, dims: dict, tokens, trace: dict | None = None) -> np.ndarray:
    """The decoder over one sequence: fp32 logits [L][vocab] of every position.  `w` holds the
    device's tensors as numpy arrays (hk_model_tensor names; per layer a list under "layers").
    `trace`, when given, receives each layer's cached latent rows ("kv", a list of [L][576])
    and the residual stream after attention ("x_attn")."""
    tokens = np.asarray(tokens, np.int64)
    L = tokens.shape[0]
    H, E, K, I = dims["hidden"], dims["experts"], dims["top_k"], dims["inter"]
    theta = dims.get("rope_theta") or 10000.0
    route_scale = dims.get("route_scale") or 1.0
    x = from_bf16_bits(w["embed"][tokens])
    cs, sn = rope(L, theta)
    pending = None
    for lw in w["layers"]:
        if pending is not None:
            x = bf16(x + pending)
        aq, as_ = rms_quant(x)
        qa = bf16(gemm_fp8(aq, as_, lw["wqa"], lw["wqa.scale"]))
        kv = bf16(gemm_fp8(aq, as_, lw["wkva"], lw["wkva.scale"]))
        qaq, qas = rms_quant(qa)
        q = bf16(gemm_fp8(qaq, qas, lw["wqb"], lw["wqb.scale"])).reshape(L, HEADS, ROW)
        q[:, :, LATENT:LATENT + 32], q[:, :, LATENT + 32:] = _rot(q[:, :, LATENT:LATENT + 32], q[:, :, LATENT + 32:],
                                                                 cs[:, None, :], sn[:, None, :])
        lat = kv[:, :LATENT]
        ms = (lat.astype(np.float64) ** 2).mean(axis=1).astype(np.float32)
        kv[:, :LATENT] = bf16(lat * (np.float32(1.0) / np.sqrt(ms + np.float32(1e-6)))[:, None])
        kv[:, LATENT:LATENT + 32], kv[:, LATENT + 32:] = _rot(kv[:, LATENT:LATENT + 32], kv[:, LATENT + 32:], cs, sn)
        if trace is not None:
            trace.setdefault("kv", []).append(kv.copy())
            trace.setdefault("q", []).append(q.copy())
        o = bf16(attention(q, kv))
        oq, os_ = quant_fp8(bf16_bits(o.reshape(L, HEADS * LATENT)))
        y = bf16(gemm_fp8(oq, os_, lw["wo"], lw["wo.scale"]))
        x = bf16(x + y)
        hq, hs = rms_quant(x)
        rl = bf16(gemm_fp8(hq, hs, lw["router"], lw["router.scale"]))
        ids, wt = route(rl, None, K, route_scale)
        off, tok, pw, inv = permute(ids, wt, E)
        w13, s13 = lw["w13"], lw["w13.scale"]
        w2, s2 = lw["w2"], lw["w2.scale"]
        yr = moe_grouped(hq, hs, off, tok, H, I, w13[:E], s13[:E], w2[:E], s2[:E])
        ys = moe_grouped(hq, hs, np.array([0, L], np.int32), np.arange(L, dtype=np.int32), H, I, w13[E:], s13[E:],
                         w2[E:], s2[E:])
        pending = bf16(combine(bf16_bits(yr), pw, inv, bf16_bits(ys), L, K))
    v = x + pending if pending is not None else x  # the last residual feeds the final norm unrounded
    fq, fs = rms_quant(v)
    return bf16(gemm_fp8(fq, fs, w["vocab"], w["vocab.scale"]))


def log_softmax(row: np.ndarray) -> np.ndarray:
    x = np.asarray(row, np.float64)
    m = x.max()
    return x - (m + np.log(np.exp(x - m).sum()))
