"""Seeded synthetic workloads for the decode-step configurations.

The reference measures on real checkpoints and traces that are not available here, so
every input is synthetic: a splitmix64 counter stream gives uniforms, Box-Muller turns
them into normals, and Fisher-Yates over the same stream scatters pages.  The shapes and
distributions follow the benchmark configurations:

  1. GQA plumbing: 8 lanes, context U[16,512], page 64, 8 query / 2 KV heads, d 128, fp32.
  2. MLA decode: 64 lanes, context log-uniform [1K,128K], 128 heads, latent 512 + rope 64,
     bf16, page 64, scale 1/sqrt(576), one new row per lane appended before attention.
  3. mixed prefill + decode: 48 decode lanes U[2K,32K] + 2 prompt chunks of 2048 rows.
  4. MoE: 512 tokens, 256 routed + 1 shared expert, top-8 sigmoid, hidden 7168, inter 2048.
  5. long context + spec verify: 1 lane at 1,048,576 + 7 lanes U[4K,64K], 1 + 4 rows each,
     e4m3 latent cache with a per-row scale.

`context` below is the number of rows cached before the step; the step's new rows sit at
positions context, context+1, ...
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

_GOLDEN = 0x9E3779B97F4A7C15
_M64 = (1 << 64) - 1


def _mix(z: np.ndarray) -> np.ndarray:
    z = z.astype(np.uint64)
    with np.errstate(over="ignore"):
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        z = z ^ (z >> np.uint64(31))
    return z


class Rng:
    """splitmix64 counter stream: draw i of stream `seed` is mix(seed + (i + 1) * golden)."""

    def __init__(self, seed: int = 0):
        self.seed = seed & _M64
        self.n = 0

    def bits(self, n: int) -> np.ndarray:
        i = np.arange(self.n + 1, self.n + 1 + n, dtype=np.uint64)
        self.n += n
        with np.errstate(over="ignore"):
            z = np.uint64(self.seed) + i * np.uint64(_GOLDEN)
        return _mix(z)

    def uniform(self, n: int) -> np.ndarray:
        """Doubles in [0, 1) from the top 53 bits."""
        return (self.bits(n) >> np.uint64(11)).astype(np.float64) * (1.0 / (1 << 53))

    def normal(self, n: int) -> np.ndarray:
        """Box-Muller: pairs (u1, u2) -> sqrt(-2 ln u1) (cos 2pi u2, sin 2pi u2)."""
        m = (n + 1) // 2
        u = self.uniform(2 * m)
        u1 = 1.0 - u[0::2]  # (0, 1]
        u2 = u[1::2]
        r = np.sqrt(-2.0 * np.log(u1))
        z = np.empty(2 * m)
        z[0::2] = r * np.cos(2 * np.pi * u2)
        z[1::2] = r * np.sin(2 * np.pi * u2)
        return z[:n]

    def integers(self, lo: int, hi: int, n: int) -> np.ndarray:
        """Uniform integers in [lo, hi] (inclusive)."""
        return lo + np.floor(self.uniform(n) * (hi - lo + 1)).astype(np.int64)

    def permutation(self, n: int) -> np.ndarray:
        """Fisher-Yates over the stream."""
        a = np.arange(n, dtype=np.int64)
        u = self.uniform(max(n - 1, 0))
        for i in range(n - 1, 0, -1):
            j = int(u[n - 1 - i] * (i + 1))
            a[i], a[j] = a[j], a[i]
        return a


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bit patterns (uint16)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return u.astype(np.uint16)


def latent_rows(cache: np.ndarray, slots, page_rows: int = 64) -> np.ndarray:
    """Rows `slots` of a page-blocked latent cache ([slots][row] array), as [len][row]."""
    slots = np.asarray(slots, dtype=np.int64)
    row = cache.shape[1]
    flat = cache.reshape(-1)
    e = np.arange(row, dtype=np.int64)
    off = ((slots // page_rows) * page_rows * row)[:, None] + ((e // 64) * page_rows * 64)[None, :] \
        + ((slots % page_rows) * 64)[:, None] + (e % 64)[None, :]
    return flat[off]


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


@dataclass
class Paged:
    """A paged cache layout: per-lane contexts, new rows, block tables over a page pool."""
    context: np.ndarray          # rows cached before the step, per lane
    new_rows: np.ndarray         # rows added this step, per lane
    page_size: int
    num_pages: int               # pool size including the scratch page 0
    block_table: np.ndarray      # [lanes][stride] int32, 0 past the lane's pages
    extra: dict = field(default_factory=dict)

    @property
    def lanes(self) -> int:
        return len(self.context)

    @property
    def kv_len(self) -> np.ndarray:
        return self.context + self.new_rows

    @property
    def num_tokens(self) -> int:
        return int(self.new_rows.sum())

    @property
    def num_slots(self) -> int:
        return self.num_pages * self.page_size


def paged_layout(rng: Rng, context, new_rows, page_size: int, spare_pages: int = 0,
                 stride: int | None = None) -> Paged:
    """Scatters every lane's pages over a seeded permutation of pages 1..N-1 (0 = scratch)."""
    context = np.asarray(context, dtype=np.int64)
    new_rows = np.asarray(new_rows, dtype=np.int64)
    need = (context + new_rows + page_size - 1) // page_size
    total = int(need.sum()) + spare_pages
    perm = rng.permutation(total) + 1
    stride = stride or int(need.max())
    bt = np.zeros((len(context), stride), dtype=np.int32)
    at = 0
    for b, n in enumerate(need):
        bt[b, :n] = perm[at:at + n]
        at += n
    return Paged(context, new_rows, page_size, total + 1, bt)


# ------------------------------------------------------------------------------------------
# configurations
# ------------------------------------------------------------------------------------------

def config1(seed: int = 0) -> dict:
    """GQA plumbing step: 8 lanes, context U[16,512], 1 new row each."""
    rng = Rng(seed)
    ctx = rng.integers(16, 512, 8)
    lay = paged_layout(rng, ctx, np.ones(8, np.int64), 64)
    qh, kvh, d = 8, 2, 128
    T = lay.num_tokens
    return dict(layout=lay, q_heads=qh, kv_heads=kvh, head_dim=d, scale=1.0 / math.sqrt(d),
                q=rng.normal(T * qh * d).astype(np.float32).reshape(T, qh, d),
                k_new=rng.normal(T * kvh * d).astype(np.float32).reshape(T, kvh * d),
                v_new=rng.normal(T * kvh * d).astype(np.float32).reshape(T, kvh * d),
                k_cache=rng.normal(lay.num_slots * kvh * d).astype(np.float32).reshape(lay.num_slots, kvh * d),
                v_cache=rng.normal(lay.num_slots * kvh * d).astype(np.float32).reshape(lay.num_slots, kvh * d))


def config2_contexts(rng: Rng, lanes: int = 64, lo: int = 1024, hi: int = 131072) -> np.ndarray:
    u = rng.uniform(lanes)
    return np.floor(np.exp(math.log(lo) + u * (math.log(hi) - math.log(lo)))).astype(np.int64)


def config2_layout(seed: int = 0, lanes: int = 64, lo: int = 1024, hi: int = 131072,
                   new_rows: int = 1) -> Paged:
    """MLA decode layout: contexts log-uniform [lo, hi], page 64, scattered pages."""
    rng = Rng(seed)
    ctx = config2_contexts(rng, lanes, lo, hi)
    return paged_layout(rng, ctx, np.full(lanes, new_rows, np.int64), 64)


def config5_layout(seed: int = 0, long_ctx: int = 1 << 20, short_lanes: int = 7,
                   lo: int = 4096, hi: int = 65536, rows: int = 5) -> Paged:
    """Long context + spec verify: one lane at long_ctx and short_lanes U[lo, hi], 1+4 rows."""
    rng = Rng(seed)
    ctx = np.concatenate([[long_ctx], rng.integers(lo, hi, short_lanes)]).astype(np.int64)
    return paged_layout(rng, ctx, np.full(len(ctx), rows, np.int64), 64)


def config3_attn_layout(seed: int = 0, decode_lanes: int = 48, lo: int = 2048, hi: int = 32768,
                       chunk: int = 2048, chunk_ctx=(0, 2048)) -> Paged:
    """Configuration 3's attention batch: decode lanes with contexts U[lo, hi] and one new row,
    then one lane per chunked-prefill segment of `chunk` rows after chunk_ctx cached rows
    (the first chunk of a prompt and its second), page 64, scattered pages."""
    rng = Rng(seed)
    ctx = np.concatenate([rng.integers(lo, hi, decode_lanes), np.asarray(chunk_ctx)]).astype(np.int64)
    rows = np.concatenate([np.ones(decode_lanes, np.int64), np.full(len(chunk_ctx), chunk, np.int64)])
    return paged_layout(rng, ctx, rows, 64)


def mla_inputs(lay: Paged, heads: int, seed: int = 1) -> dict:
    """bf16 bit patterns of N(0,1) queries, new latent rows and the cached rows."""
    rng = Rng(seed)
    T = lay.num_tokens
    q = f32_to_bf16_bits(rng.normal(T * heads * 576).astype(np.float32)).reshape(T, heads, 576)
    kv_new = f32_to_bf16_bits(rng.normal(T * 576).astype(np.float32)).reshape(T, 576)
    cache = f32_to_bf16_bits(rng.normal(lay.num_slots * 576).astype(np.float32)).reshape(lay.num_slots, 576)
    return dict(q=q, kv_new=kv_new, kv_cache=cache, scale=1.0 / math.sqrt(576))


def moe_inputs(tokens: int, experts: int, hidden: int, inter: int, top_k: int = 8,
               seed: int = 3) -> dict:
    """Router logits N(0,1); bf16 activations N(0,1); e4m3 weights of N(0, 0.02) values
    quantised per 128x128 block (scale = amax / 448)."""
    rng = Rng(seed)
    logits = rng.normal(tokens * experts).astype(np.float32).reshape(tokens, experts)
    x = f32_to_bf16_bits(rng.normal(tokens * hidden).astype(np.float32)).reshape(tokens, hidden)

    def qweights(n_out: int, n_in: int, count: int):
        w = (rng.normal(count * n_out * n_in) * 0.02).astype(np.float32).reshape(count, n_out, n_in)
        blk = w.reshape(count, n_out // 128, 128, n_in // 128, 128)
        amax = np.abs(blk).max(axis=(2, 4))
        s = (np.maximum(amax, 1e-12) / 448.0).astype(np.float32)
        scaled = blk / s[:, :, None, :, None]
        q = e4m3_encode(scaled.reshape(count, n_out, n_in))
        return q, s

    w13, s13 = qweights(2 * inter, hidden, experts)
    w2, s2 = qweights(hidden, inter, experts)
    return dict(logits=logits, x=x, w13=w13, s13=s13, w2=w2, s2=s2, top_k=top_k)


def e4m3_encode(x: np.ndarray) -> np.ndarray:
    """Vectorised fp32 -> e4m3 (round to nearest even, saturate to 448)."""
    x = np.asarray(x, dtype=np.float32)
    sign = np.signbit(x).astype(np.uint8) << 7
    a = np.minimum(np.abs(x), 448.0).astype(np.float64)
    out = np.zeros(x.shape, dtype=np.uint8)
    sub = a < 2.0 ** -6
    m_sub = np.rint(a * 2.0 ** 9).astype(np.int64)
    out = np.where(sub, np.where(m_sub >= 8, 0x08, m_sub).astype(np.uint8), out)
    with np.errstate(divide="ignore"):
        e = np.floor(np.log2(np.where(sub, 1.0, a))).astype(np.int64)
    mant = np.where(sub, 0.0, a / np.exp2(e) - 1.0)
    m = np.rint(mant * 8).astype(np.int64)
    e = np.where(m == 8, e + 1, e)
    m = np.where(m == 8, 0, m)
    be = e + 7
    sat = (be > 15) | ((be == 15) & (m == 7))
    normal = np.where(sat, 0x7E, (be << 3) | m).astype(np.uint8)
    out = np.where(sub, out, normal)
    return (out | sign).astype(np.uint8)


def e4m3_decode(v: np.ndarray) -> np.ndarray:
    v = np.asarray(v, dtype=np.uint8).astype(np.int64)
    s = np.where(v >> 7, -1.0, 1.0)
    e = (v >> 3) & 15
    m = v & 7
    r = np.where(e == 0, m * 2.0 ** -9, (1 + m / 8.0) * np.exp2(e - 7))
    r = np.where((e == 15) & (m == 7), np.nan, r)
    return (s * r).astype(np.float32)
