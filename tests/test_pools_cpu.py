"""Pool sizing (hk_pages_within / hk_plan_pools) against the oracle, and the oracle against the
reference's own test of pages_within (src/gpu/load.rs:1012-1018).  Host arithmetic only: the
library is loaded, no device is touched (free memory is passed in)."""
import random

import pytest

from oracle import pools as O

_lib = pytest.importorskip("hyperkernel_b200._lib")


def _lib_or_skip():
    try:
        _lib.lib()
    except Exception as e:  # library not built
        pytest.skip(f"libhk.so unavailable: {e}")


def ref_pool(page=100, window=10, **kw):
    """The reference test's pool(page, window) (load.rs:993-1009) with its overrides."""
    p = O.PoolSizing(pages=kw.get("pages", 1000), window_pages=kw.get("window_pages", 10), entries=5,
                     slots=9, states=[O.PoolState(0, O.PAGE, page), O.PoolState(1, O.WINDOW, window)])
    return p


def lib_within(p: O.PoolSizing, nbytes: int):
    return _lib.pages_within(p.pages, p.window_pages, p.entries,
                             [(s.home, s.unit, s.bytes) for s in p.states], nbytes, slots=p.slots)


def test_oracle_matches_the_reference_test_of_pages_within():
    p = ref_pool()
    assert O.pages_within(p, 10 * 10 + 520 * 100 + 99) == (520, 10)
    assert O.pages_within(p, 10 * 10 + 5 * 100) is None          # no more than one sequence's pages
    assert O.pages_within(p, 10 * 10 - 1) is None                # no room for the window pages
    assert O.pages_within(ref_pool(pages=7), 1 << 40) == (7, 10)  # at most the bundle's


def test_library_matches_the_reference_test_of_pages_within():
    _lib_or_skip()
    p = ref_pool()
    assert lib_within(p, 10 * 10 + 520 * 100 + 99) == (520, 10)
    assert lib_within(p, 10 * 10 + 5 * 100) is None
    assert lib_within(p, 10 * 10 - 1) is None
    assert lib_within(ref_pool(pages=7), 1 << 40) == (7, 10)


def test_library_matches_the_oracle_on_random_pools():
    _lib_or_skip()
    rng = random.Random(0)
    for _ in range(2000):
        states = [O.PoolState(rng.randrange(4), rng.choice((O.PAGE, O.WINDOW)), rng.choice((0, 1, 7, 4096, 73728, 1 << 22)))
                  for _ in range(rng.randrange(0, 5))]
        p = O.PoolSizing(pages=rng.choice((0, 1, 6, 100, 1 << 20, (1 << 63) - 1)),
                         window_pages=rng.choice((0, 1, 10, 4096)), entries=rng.choice((0, 5, 2048)),
                         slots=rng.randrange(1, 300), states=states)
        nbytes = rng.choice((0, 99, 1 << 20, 180 * 10**9, rng.randrange(1 << 40)))
        assert lib_within(p, nbytes) == O.pages_within(p, nbytes), (p, nbytes)


def test_plan_errors_carry_the_reference_wording():
    _lib_or_skip()
    p = ref_pool()
    st = [(s.home, s.unit, s.bytes) for s in p.states]
    cases = [
        dict(free=1000, other=900, slack=200, lanes=8, context=320),    # kernel past free memory
        dict(free=10_000, other=0, slack=9_400, lanes=8, context=320),  # pools hold no sequence
        dict(free=10**6, other=0, slack=0, lanes=9, context=320),       # lanes past the slots
    ]
    for c in cases:
        with pytest.raises(ValueError) as want:
            O.plan_pools(p, c["free"], c["other"], c["slack"], c["lanes"], c["context"])
        with pytest.raises(_lib.HKError) as got:
            _lib.plan_pools(p.pages, p.window_pages, p.entries, p.slots, st, lanes=c["lanes"],
                            context=c["context"], other=c["other"], slack=c["slack"], free=c["free"])
        assert str(want.value) in str(got.value)


def test_plan_sizes_an_mla_cache_in_a_b200s_memory():
    """The config-2 bf16 MLA cache of a 61-layer model (64-row pages of 576 bf16 per row and
    layer) plus an FP8 window pool, in 180 GB less 40 GB of weights and 4 GB of slack."""
    _lib_or_skip()
    page = 61 * 64 * 576 * 2
    p = O.PoolSizing(pages=1 << 40, window_pages=4096, entries=2049, slots=65,
                     states=[O.PoolState(0, O.PAGE, page), O.PoolState(1, O.WINDOW, 61 * 64 * 580)])
    args = dict(free=180 * 10**9, other=40 * 10**9, slack=4 * 10**9, lanes=64, context=131072)
    want = O.plan_pools(p, args["free"], args["other"], args["slack"], args["lanes"], args["context"])
    got = _lib.plan_pools(p.pages, p.window_pages, p.entries, p.slots,
                          [(s.home, s.unit, s.bytes) for s in p.states], **args)
    assert got == want
    pages, window_pages, slots, used = got
    assert slots == 65 and window_pages == 4096
    assert used <= 136 * 10**9 < used + page        # the pools fill the budget to within a page
    assert pages * 64 >= 64 * 26_803                # config 2's mean context fits every lane
