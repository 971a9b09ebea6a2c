"""Test infrastructure only: CPU restatement of the loader's pool sizing.

Only tests/ may use this module, and only as the checker.

  * pages_within (src/gpu/load.rs:903-908): the window pages are taken whole; the bytes left
    buy pages at the summed per-page cost of the page states (at least 1 B), at most the
    bundle's `pages`; the result must hold more than one row of `entries` pages, else None.
  * plan, pool part (src/gpu/load.rs:510-533): pools get free - (other + slack) bytes (an
    error if that underflows); slots = lanes + 1 must not pass the bundle's slots; the bytes
    used are the sum over states of bytes x (pages or window pages) (state_bytes, :535-537).

Pinned by the reference's own test (load.rs:1012-1018) in tests/test_pools_cpu.py.
"""
from __future__ import annotations

from dataclasses import dataclass, field

PAGE, WINDOW = 0, 1


@dataclass
class PoolState:
    home: int
    unit: int
    bytes: int


@dataclass
class PoolSizing:
    pages: int
    window_pages: int
    entries: int
    slots: int = 9
    states: list = field(default_factory=list)


def _cost(pool: PoolSizing, unit: int) -> int:
    return sum(s.bytes for s in pool.states if s.unit == unit)


def pages_within(pool: PoolSizing, nbytes: int):
    """(pages, window_pages) or None."""
    rest = nbytes - pool.window_pages * _cost(pool, WINDOW)
    if rest < 0:
        return None
    pages = min(rest // max(_cost(pool, PAGE), 1), pool.pages)
    return (pages, pool.window_pages) if pages > pool.entries else None


def plan_pools(pool: PoolSizing, free: int, other: int, slack: int, lanes: int, context: int):
    """(pages, window_pages, slots, used) or raises ValueError with the reference's wording."""
    nbytes = free - (other + slack)
    if nbytes < 0:
        raise ValueError(f"the kernel's {other} B and {slack} B of slack past the GPU's {free} B free")
    got = pages_within(pool, nbytes)
    if got is None:
        raise ValueError(f"{nbytes} B of pools hold no sequence of {context} positions")
    pages, window_pages = got
    slots = lanes + 1
    if slots > pool.slots:
        raise ValueError(f"{lanes} lanes past the bundle's {pool.slots} slots")
    used = sum(s.bytes * (pages if s.unit == PAGE else window_pages) for s in pool.states)
    return pages, window_pages, slots, used
