"""Test infrastructure only: CPU restatement of the sampling / spec-verify step (numpy).

Only tests/, __graft_entry__.smoke() and bench.py's CPU baseline may use this module, and
only as the checker.

The reference's LLM sampler runs inside closed device code; the one sampler it ships as
source is `Sampling::draw` (src/evo2/draw.rs:14-49, splitmix at :52-58), restated here
step for step.  It is the semantics hk_sample_verify implements for rows that are sampled:

  * greedy (temperature <= 0 — the LLM `Sampling` samples only at temperature > 0,
    src/engine/request.rs:40-42 — or top_k == 1 as in draw.rs:16-18): the first index of the
    greatest logit, no draw;
  * otherwise: sort the row by value, descending and stable (draw.rs:19-20, `total_cmp`), keep
    the first top_k (:21-23), softmax of value / temperature in f64 (:24-29), zero the tail
    whose inclusive sum from the bottom is <= 1 - top_p when 0 < top_p < 1 (:30-38), draw
    u = splitmix(state) / 2^53 * kept and take the first index whose running sum exceeds u
    (:39-47), else the last index with a non-zero probability (:48).

Sums run left to right as in Rust's `Iterator::sum` (np.cumsum is sequential).  A row with a
non-finite logit yields id -1 (the boundary's "negative id = non-finite logits",
src/gpu/mod.rs:13-40), which the evo2 sampler instead maps to 0.

Verification (src/gpu/feed.rs:163-199): a lane's rows are its 1 + drafts positions; row j
is drawn, and the chain continues to row j + 1 only while the drawn token equals draft j.
Each accepted token has a logprob row of `n` (id, logprob) pairs of the row's log-softmax
(temperature 1), best first with ties to the lower id, ids past the vocabulary as -1, then
the token's own logprob (feed.rs:202-208 reads exactly this layout).
"""
from __future__ import annotations

import numpy as np

MASK64 = (1 << 64) - 1


def splitmix(state: int) -> tuple[int, int]:
    """src/evo2/draw.rs:52-58: returns (new state, 53-bit draw)."""
    state = (state + 0x9E3779B97F4A7C15) & MASK64
    z = state
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & MASK64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & MASK64
    return state, (z ^ (z >> 31)) >> 11


def greedy(sampling) -> bool:
    return not (sampling["temperature"] > 0.0) or sampling["top_k"] == 1


def sorted_desc(row: np.ndarray) -> np.ndarray:
    """Indices of the row by value, descending in the IEEE total order (`f32::total_cmp`, so
    +0 before -0), ties in index order (a stable sort)."""
    b = np.ascontiguousarray(row, np.float32).view(np.uint32)
    asc = np.where(b & np.uint32(0x80000000), ~b, b | np.uint32(0x80000000))
    return np.argsort(~asc, kind="stable")


def draw(row: np.ndarray, sampling, state: int) -> tuple[int, int]:
    """One draw (src/evo2/draw.rs:14-49) of a finite fp32 row; returns (id, new state)."""
    row = np.asarray(row, np.float32)
    if greedy(sampling):
        return int(np.argmax(row)), state        # np.argmax returns the first greatest
    top = sorted_desc(row)
    k = int(sampling["top_k"])
    if k > 0:
        top = top[:min(k, row.shape[0])]
    scaled = row[top].astype(np.float64) / np.float64(np.float32(sampling["temperature"]))
    most = scaled[0]
    probs = np.exp(scaled - most)
    total = np.cumsum(probs)[-1]
    probs = probs / total
    top_p = np.float64(np.float32(sampling["top_p"]))
    if 0.0 < top_p < 1.0:
        below = np.cumsum(probs[::-1])[::-1]     # inclusive sums from the bottom
        probs = np.where(below <= 1.0 - top_p, 0.0, probs)
    kept = np.cumsum(probs)[-1]
    state, bits = splitmix(state)
    u = np.float64(bits) / np.float64(1 << 53) * kept
    seen = np.cumsum(probs)
    hit = np.nonzero(u < seen)[0]
    if hit.size:
        return int(top[hit[0]]), state
    pos = np.nonzero(probs > 0.0)[0]
    return int(top[pos[-1] if pos.size else 0]), state


def logprob_row(row: np.ndarray, token: int, n: int) -> np.ndarray:
    """2n + 1 floats: n best (id, logprob) pairs of log-softmax(row), then the token's."""
    x = np.asarray(row, np.float64)
    m = x.max()
    lse = m + np.log(np.exp(x - m).sum())
    out = np.zeros(2 * n + 1, np.float32)
    top = sorted_desc(np.asarray(row, np.float32))
    for q in range(n):
        if q < x.shape[0]:
            out[2 * q] = float(top[q])
            out[2 * q + 1] = np.float32(x[top[q]] - lse)
        else:
            out[2 * q] = -1.0
    out[2 * n] = np.float32(x[token] - lse)
    return out


def sample_verify(logits, cu_rows, samplings, states, drafts, block: int, n_logprobs: int):
    """The verify step over all lanes: returns (ids [lanes][block], lp [lanes][block][2n+1],
    new states).  logits [rows][vocab] fp32; drafts [lanes][block - 1]."""
    logits = np.asarray(logits, np.float32)
    lanes = len(cu_rows) - 1
    ids = np.full((lanes, block), -2, np.int32)
    lp = np.zeros((lanes, block, 2 * n_logprobs + 1), np.float32)
    out_states = list(states)
    for b in range(lanes):
        st = int(states[b])
        rows = int(cu_rows[b + 1] - cu_rows[b])
        for j in range(rows):
            row = logits[cu_rows[b] + j]
            if not np.isfinite(row).all():
                ids[b, j] = -1
                break
            t, st = draw(row, samplings[b], st)
            ids[b, j] = t
            lp[b, j] = logprob_row(row, t, n_logprobs)
            if j + 1 < rows and t != int(drafts[b][j]):
                break
        out_states[b] = st
    return ids, lp, out_states
