"""The sampling / spec-verify oracle (oracle/sample.py) pinned to the reference's own tests.

`Sampling::draw` ships with three tests (src/evo2/draw.rs:60-101): greedy takes the first
greatest logit and leaves the state alone; top-k draws follow their softmax and repeat by
seed; temperature sharpens and top-p drops the tail.  They are restated here against the
oracle, together with the published SplitMix64 vector (seed 0) for the generator at
draw.rs:52-58, the reply layout `sampled` reads (src/gpu/feed.rs:202-208) and the linear
draft chain.
"""
import numpy as np

from oracle import sample as S

G = dict(temperature=0.0, top_k=0, top_p=1.0)


def test_splitmix_matches_the_published_vector():
    st, out = 0, []
    for _ in range(3):
        st, b = S.splitmix(st)
        out.append(b)
    # SplitMix64 from seed 0: 0xE220A8397B1DCDAF, 0x6E789E6AA1B965F4, 0x06C45D188009454F (top 53 bits)
    assert out == [0xE220A8397B1DCDAF >> 11, 0x6E789E6AA1B965F4 >> 11, 0x06C45D188009454F >> 11]


def test_greedy_is_the_first_greatest_and_draws_nothing():
    assert S.draw(np.array([0.0, 3.0, 3.0, -1.0], np.float32), G, 0) == (1, 0)
    assert S.draw(np.array([0.0, 3.0, 3.0, -1.0], np.float32), dict(temperature=1.0, top_k=1, top_p=1.0), 9) == (1, 9)


def test_top_k_draws_follow_their_softmax_and_repeat_by_seed():
    s = dict(temperature=1.0, top_k=2, top_p=0.0)
    row = np.array([0.0, np.log(2.0), -5.0, -9.0], np.float32)

    def draws(seed):
        st, d = seed, []
        for _ in range(30_000):
            t, st = S.draw(row, s, st)
            d.append(t)
        return np.array(d)

    d = draws(7)
    assert np.array_equal(d, draws(7))
    assert not np.array_equal(d, draws(8))
    assert (d < 2).all()
    assert abs((d == 1).mean() - 2.0 / 3.0) < 0.02


def test_temperature_sharpens_and_top_p_drops_the_tail():
    row = np.array([0.0, 1.0, 2.0, 3.0], np.float32)

    def share(s, t):
        st, n = s["seed"], 0
        for _ in range(20_000):
            x, st = S.draw(row, s, st)
            n += x == t
        return n / 20_000

    base = dict(temperature=1.0, top_k=0, top_p=0.0, seed=3)
    assert share(dict(base, temperature=0.25), 3) > share(base, 3)
    assert share(dict(base, temperature=4.0), 3) < share(base, 3)
    assert share(dict(base, top_p=0.5), 0) == 0.0
    assert share(dict(base, top_p=0.5), 3) > 0.99


def test_sort_is_the_total_order_with_ties_in_index_order():
    row = np.array([-0.0, 0.0, 2.0, -1.0, 2.0], np.float32)
    assert S.sorted_desc(row).tolist() == [2, 4, 1, 0, 3]


def test_logprob_row_layout_is_what_the_reply_reader_expects():
    """feed.rs:202-208: pairs while id >= 0, then the token's own logprob last."""
    row = np.array([1.0, 3.0, 2.0], np.float32)
    out = S.logprob_row(row, 2, 4)
    lse = np.log(np.exp(row.astype(np.float64)).sum())
    pairs = out[:-1].reshape(-1, 2)
    assert pairs[:, 0].tolist() == [1, 2, 0, -1]
    assert np.allclose(pairs[:3, 1], row[[1, 2, 0]] - lse, atol=1e-6)
    assert abs(out[-1] - (row[2] - lse)) < 1e-6


def test_chain_accepts_drafts_until_the_first_mismatch_and_stops_at_non_finite_rows():
    V = 16
    logits = np.full((9, V), -4.0, np.float32)
    want = [3, 5, 7, 1, 9, 2, 2, 11, 4]
    for r, t in enumerate(want):
        logits[r, t] = 4.0
    logits[8, 0] = np.nan
    cu = np.array([0, 3, 6, 9])
    drafts = np.array([[3, 5], [9, 9], [2, 11]])   # lane 0 all accepted, lane 1 stops at row 0,
                                                   # lane 2 reaches its non-finite row
    ids, lp, st = S.sample_verify(logits, cu, [G, G, G], [1, 2, 3], drafts, 3, 2)
    assert ids.tolist() == [[3, 5, 7], [1, -2, -2], [2, 11, -1]]
    assert st == [1, 2, 3]
    assert lp[0, 0, 0] == 3 and lp[1, 1].tolist() == [0.0] * 5


def test_greedy_past_a_nan_or_an_infinity_is_the_non_finite_rule():
    """The reference's greedy test (src/evo2/draw.rs:65-71) draws index 2 from
    [NaN, inf, 2.0]: the evo2 sampler cleans non-finite logits to 0.  At the decode step's
    boundary a negative id means non-finite logits (src/gpu/mod.rs:13-40, the Sampled id the
    engine reads as "the logits were not finite"), so this build answers -1 for that row and
    leaves the generator state alone; the finite half of the same test is kept as it is."""
    row = np.array([np.nan, np.inf, 2.0], np.float32)
    greedy = dict(temperature=1.0, top_k=1, top_p=0.0)
    ids, lp, st = S.sample_verify(row[None, :], np.array([0, 1]), [greedy], [0], np.zeros((1, 0), np.int32), 1, 0)
    assert ids.tolist() == [[-1]] and st == [0]
    ids, _, st = S.sample_verify(np.array([[0.0, 3.0, 3.0, -1.0]], np.float32), np.array([0, 1]), [greedy], [0],
                                 np.zeros((1, 0), np.int32), 1, 0)
    assert ids.tolist() == [[1]] and st == [0]
