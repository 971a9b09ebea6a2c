"""The engine on libhk's device kernel (hk_open / hk_push / hk_drain) against the engine oracle.

Every scenario of the reference's tests/engine.rs runs through libhk's C++ engine and libhk's
device kernel: block-table rows, lane state and the paged token / window pools live on the GPU,
the test model (an FNV fold over the sequence read back through the block table) runs there,
and the share stream, each request's outputs and the metrics must equal the oracle engine's on
the reference's test device.  The device checks on every read and write what the reference's
test device asserts (no scratch-page write, no unwritten read, window pages mirroring pages).
"""
import ctypes as C
import re
import threading

import pytest

import engine_port as P
from hyperkernel_b200 import _lib
from hyperkernel_b200 import engine as H
from oracle import engine as E

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("transport", [0, 1], ids=["launch", "ring"])
@pytest.mark.parametrize("sc", P.scenarios(), ids=repr)
def test_device_matches_oracle_share_by_share(cuda, sc, transport):
    """Both transports: a kernel launch per batch and step, and the resident executor that
    polls a mailbox in mapped host memory."""
    want = P.run_oracle(sc)
    dev = H.Device(P.device_config(sc, transport=transport))
    try:
        got = P.run_hk(sc, P.DevicePort(dev))
    finally:
        dev.close()
    P.assert_same(got, want)


@pytest.mark.parametrize("transport", [0, 1], ids=["launch", "ring"])
@pytest.mark.parametrize("name", ["prefixes_default", "small_pool_budget_keep", "drafts_clips"])
def test_device_through_native_ops(cuda, name, transport):
    """The engine calling the device kernel through hk_kernel_ops_of: no Python in the loop."""
    sc = next(s for s in P.scenarios() if s.name == name)
    want = P.run_oracle(sc)
    dev = H.Device(P.device_config(sc, transport=transport))
    try:
        got = P.run_hk_native(sc, dev)
    finally:
        dev.close()
    P.assert_same(got, want, shares=False)


def test_device_reset_empties_the_prefix_cache(cuda):
    sc = P.Scenario("reset", [])
    dev = H.Device(P.device_config(sc))
    port = P.DevicePort(dev)
    kern = H.CallbackKernel(port)
    eng = H.Engine(P.engine_config(sc), kern.ops(), keep=kern)
    result = {}
    loop = threading.Thread(target=lambda: result.setdefault("rc", eng.run()))
    loop.start()
    a = P.Ask(range(1, 20), 6)
    seen = [0]

    def run_one():
        r = eng.submit(a.prompt, a.limit)
        h = eng.heard(r, timeout_ms=60000)
        while h.end is None:
            more = eng.heard(r, timeout_ms=60000)
            h.tokens += more.tokens
            h.end = more.end
        assert (h.tokens, h.end) == P.expected(a)
        new, seen[0] = port.shares[seen[0]:], len(port.shares)
        return next((c.pos for s in new for c in s.commands if isinstance(c, E.Seat)), None)

    try:
        assert run_one() == 0
        assert run_one() == 16, "the second resumed the first's prefix"
        assert eng.reset_answer(eng.reset(), 60000) == (len(a.prompt) + a.limit - 1) // P.PAGE_ROWS
        assert run_one() == 0, "nothing resumed after the reset"
    finally:
        eng.close()
        loop.join(timeout=120)
        dev.close()
    assert result["rc"] == 0


def _drain(dev):
    evs = (H.Event * 64)()
    ids = (H.I32 * 1024)()
    n, ids_n = H.SZ(), H.SZ()
    rc = dev.drain_raw(evs, 64, C.byref(n), ids, 1024, C.byref(ids_n))
    return rc, [(e.kind, e.step, e.lane, e.token) for e in evs[:n.value]], list(ids[:ids_n.value])


def test_device_refuses_a_share_out_of_step(cuda):
    dev = H.Device(P.device_config(P.Scenario("x", [])))
    try:
        share, keep = H.make_share(1, 3, [])
        assert dev.push_raw(share) == _lib.HK_ESTATE
        assert "a share at 1 past a horizon of -1" in _lib.last_error()
        share, keep = H.make_share(0, 2, [])
        assert dev.push_raw(share) == 0
        rc, evs, _ = _drain(dev)
        assert rc == 0 and evs == []
    finally:
        dev.close()


@pytest.mark.parametrize("transport", [0, 1], ids=["launch", "ring"])
def test_device_reports_a_chunk_without_window_pages(cuda, transport):
    """tests/engine.rs:153-160: a prompt chunk whose window entry is the scratch window page is
    a device-side violation; hk_drain fails with the reference's wording."""
    dev = H.Device(P.device_config(P.Scenario("x", []), transport=transport))
    try:
        samp = H.Sampling(0.0, 1.0, 0, 0, 0)
        share, keep = H.make_share(0, 2, [
            (H.CMD_PAGES, 0, 0, 8, [1, 2], (0, 0, 0), None),  # pages, but no window pages
            (H.CMD_SEAT, 0, 0, 0, [], (7, 7, 7), samp),
            (H.CMD_PROMPT, 0, 0, 0, [5, 6, 7], (0, 0, 0), None),
        ])
        assert dev.push_raw(share) == 0
        rc, _, _ = _drain(dev)
        assert rc == _lib.HK_EDEVICE
        assert re.search(r"lane 0's chunk writes position [012]'s window to the scratch window page",
                         _lib.last_error())
    finally:
        dev.close()


@pytest.mark.parametrize("transport", [0, 1], ids=["launch", "ring"])
def test_device_prompt_and_decode_by_hand(cuda, transport):
    """One lane through the raw boundary: its prompt reply and decode tokens are the model's
    `next` over the sequence, steps stop at the reserved rows, and Idle follows."""
    dev = H.Device(P.device_config(P.Scenario("x", []), transport=transport))
    try:
        samp = H.Sampling(0.0, 1.0, 0, 0, 0)
        prompt = [11, 12, 13, 14, 15]
        row = [1, 2] + [0] * 14 + [1, 2] + [0] * 14  # pages 1, 2 and window pages 1, 2
        share, keep = H.make_share(0, 2, [
            (H.CMD_PAGES, 0, 0, 7, row, (0, 0, 0), None),
            (H.CMD_SEAT, 0, 0, 0, [], (7, 7, 7), samp),
            (H.CMD_PROMPT, 0, 0, 0, prompt, (0, 0, 0), None),
            (H.CMD_START, 0, 0, 0, [], (0, 0, 0), None),
        ])
        assert dev.push_raw(share) == 0
        rc, evs, ids = _drain(dev)
        assert rc == 0, _lib.last_error()
        seq = list(prompt)
        t0 = E.next_token(seq)
        assert evs[0] == (H.EV_PROMPTED, 0, 0, t0)
        steps = [e for e in evs if e[0] == H.EV_STEP]
        assert [s[1] for s in steps] == [0, 1], "positions 5 and 6 are reserved (upto 7)"
        seq.append(t0)
        want = []
        for _ in range(2):
            want.append(E.next_token(seq))
            seq.append(want[-1])
        got = [ids[4 * i] for i in range(2)]  # lane 0's first id of each step (width 4, block 1)
        assert got == want
        assert evs[-1][0] == H.EV_IDLE
    finally:
        dev.close()


def test_ring_executor_is_relaunched_after_going_idle(cuda):
    """The resident executor exits after 50 ms without work; the next drain's first post
    relaunches it and the lane carries on where it stopped."""
    import time

    dev = H.Device(P.device_config(P.Scenario("x", []), transport=1))
    try:
        samp = H.Sampling(0.0, 1.0, 0, 0, 0)
        prompt = [21, 22, 23]
        row = [1, 2] + [0] * 14 + [1, 2] + [0] * 14
        share, keep = H.make_share(0, 0, [
            (H.CMD_PAGES, 0, 0, 3, row, (0, 0, 0), None),
            (H.CMD_SEAT, 0, 0, 0, [], (7, 7, 7), samp),
            (H.CMD_PROMPT, 0, 0, 0, prompt, (0, 0, 0), None),
        ])
        assert dev.push_raw(share) == 0
        rc, evs, _ = _drain(dev)
        assert rc == 0, _lib.last_error()
        seq = list(prompt)
        assert evs[0] == (H.EV_PROMPTED, 0, 0, E.next_token(seq))
        seq.append(E.next_token(seq))
        time.sleep(0.3)  # the executor has gone idle and exited
        share, keep = H.make_share(1, 3, [
            (H.CMD_PAGES, 0, 0, 5, row, (0, 0, 0), None),  # positions 3 and 4 reserved
            (H.CMD_START, 0, 0, 0, [], (0, 0, 0), None),
        ])
        assert dev.push_raw(share) == 0
        rc, evs, ids = _drain(dev)
        assert rc == 0, _lib.last_error()
        steps = [e for e in evs if e[0] == H.EV_STEP]
        assert len(steps) == 2
        want = []
        for _ in range(2):
            want.append(E.next_token(seq))
            seq.append(want[-1])
        assert [ids[4 * i] for i in range(2)] == want
    finally:
        dev.close()
