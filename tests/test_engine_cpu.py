"""libhk's C++ engine (hk_engine_*) against the engine oracle, on the reference's test device.

The engine is host code, so these run without a GPU: libhk's engine drives the reference's
test device (oracle.engine.Fake) through hk_kernel_ops callbacks, and every scenario of the
reference's tests/engine.rs must produce the same share stream (every command of every push),
the same outputs per request (seated offsets, tokens, end kind and message) and the same
metrics as the oracle engine on the same device.  The request-ring encoding (hk_encode_share)
is checked against the restatement of ring::encode.
"""
import threading

import numpy as np
import pytest

import engine_port as P
from hyperkernel_b200 import _lib
from hyperkernel_b200 import engine as H
from oracle import engine as E
from oracle import wire as Wr


@pytest.mark.parametrize("sc", P.scenarios(), ids=repr)
def test_engine_matches_oracle_share_by_share(sc):
    want = P.run_oracle(sc)
    got = P.run_hk(sc, P.FakePort(P.oracle_fake(sc), sc.block))
    P.assert_same(got, want)
    for i, a in enumerate(sc.asks):
        if i not in sc.hangup:
            toks, end = P.expected(a)
            assert (got.heard[i][1], got.heard[i][2]) == (toks, end), f"request {i}"


def test_engine_reset_empties_the_prefix_cache():
    """tests/engine.rs:537-580 on libhk's engine: a second run resumes 16 cached tokens, a
    reset frees the tree's whole pages, and nothing resumes after it."""
    sc = P.Scenario("reset", [])
    port = P.FakePort(P.oracle_fake(sc), 1)
    kern = H.CallbackKernel(port)
    eng = H.Engine(P.engine_config(sc), kern.ops(), keep=kern)
    result = {}
    loop = threading.Thread(target=lambda: result.setdefault("rc", eng.run()))
    loop.start()
    a = P.Ask(range(1, 20), 6)
    seen = [0]

    def run_one():
        r = eng.submit(a.prompt, a.limit)
        h = eng.heard(r, timeout_ms=-1)
        while h.end is None:
            more = eng.heard(r, timeout_ms=-1)
            h.tokens += more.tokens
            h.end = more.end
        assert (h.tokens, h.end) == P.expected(a)
        new, seen[0] = port.shares[seen[0]:], len(port.shares)
        return next((c.pos for s in new for c in s.commands if isinstance(c, E.Seat)), None)

    def reset():
        return eng.reset_answer(eng.reset(), timeout_ms=60000)

    page = P.PAGE_ROWS
    assert run_one() == 0
    assert run_one() == 16, "the second resumed the first's prefix"
    cached = eng.metrics()[0]["cached_tokens"]
    assert cached == 16
    assert reset() == (len(a.prompt) + a.limit - 1) // page, "the tree's whole pages freed"
    assert run_one() == 0, "nothing resumed after the reset"
    assert eng.metrics()[0]["cached_tokens"] == cached
    assert reset() == (len(a.prompt) + a.limit - 1) // page
    assert reset() == 0, "an empty tree frees nothing"
    eng.close()
    loop.join(timeout=60)
    assert result["rc"] == 0


def test_a_kernel_error_refuses_every_request():
    """engine::run (src/engine/mod.rs:55-73): an Err from push or drain ends the loop and every
    held, waiting and queued request hears Refused with the kernel's message."""

    class Broken(P.FakePort):
        def drain(self):
            if len(self.shares) >= 3:
                raise RuntimeError("the device fell over")
            return super().drain()

    sc = P.Scenario("broken", P.conversations())
    port = Broken(P.oracle_fake(sc), 1)
    kern = H.CallbackKernel(port)
    eng = H.Engine(P.engine_config(sc), kern.ops(), keep=kern)
    reqs = [eng.submit(a.prompt, a.limit) for a in sc.asks]
    eng.close()
    assert eng.run() == _lib.HK_ESTATE
    assert "the device fell over" in eng.failure
    for r in reqs:
        h = eng.heard(r)
        assert h.end == "refused" and h.message == "the device fell over"


def test_too_many_drafts_is_refused_at_create():
    cfg = H.engine_config(page_rows=4, entries=16, window=16, context=64, width=4, chunk=8, block=18)
    kern = H.CallbackKernel(P.FakePort(P.oracle_fake(P.Scenario("x", [])), 1))
    with pytest.raises(_lib.HKError, match="17 drafts a step, past the 16 the metrics count"):
        H.Engine(cfg, kern.ops(), keep=kern)


# --- request-ring encoding ----------------------------------------------------------------

def test_wire_restatement_pins_to_the_reference_layout_test():
    """src/gpu/ring.rs:150-183, the reference's own known-answer test of encode/decode."""
    m = Wr.Message("seat", 0x104, 0, 56, [
        Wr.Field("lane", 0, "one", "i32", 0), Wr.Field("back", 4, "array", "i32", 3),
        Wr.Field("temp", 16, "one", "f32", 0), Wr.Field("row", 24, "span", "i32", 0),
        Wr.Field("lps", 40, "span", "f32", 33)])
    b = Wr.encode(m, [("lane", Wr.Int(-1)), ("back", Wr.Ints([1, 2, 3])), ("temp", Wr.Float(0.5)),
                      ("row", Wr.Span(0x1000, 7)), ("lps", Wr.Span(0x2000, 99))])
    assert len(b) == 56
    assert Wr.decode(m, b, "lane") == [-1]
    assert Wr.decode(m, b, "back") == [1, 2, 3]
    assert b[16:20] == np.float32(0.5).tobytes()
    assert b[24:40] == (0x1000).to_bytes(8, "little") + (7).to_bytes(8, "little")
    assert b[40:56] == (0x2000).to_bytes(8, "little") + (33).to_bytes(8, "little"), "the layout's count"


def test_encode_share_matches_the_restated_encoder():
    """hk_encode_share == the oracle's ring::encode over the same message table, on every share
    the conversations scenario pushes (all five commands, rows and prompt tokens)."""
    sc = P.Scenario("prefixes_default", P.conversations())
    want = P.run_oracle(sc)
    cfg = P.device_config(sc)
    kinds = set()
    for at, horizon, cmds in want.shares:
        raw = []
        for c in cmds:
            kinds.add(c[0])
            if c[0] == "end":
                raw.append((H.CMD_END, c[1], 0, 0, [], (0, 0, 0), None))
            elif c[0] == "pages":
                raw.append((H.CMD_PAGES, c[1], c[2], c[3], list(c[4]), (0, 0, 0), None))
            elif c[0] == "seat":
                t, p, k, seed, lp = c[4]
                raw.append((H.CMD_SEAT, c[1], c[2], 0, [], c[3], H.Sampling(t, p, k, lp, seed)))
            elif c[0] == "prompt":
                raw.append((H.CMD_PROMPT, c[1], 0, 0, list(c[2]), (0, 0, 0), None))
            else:
                raw.append((H.CMD_START, c[1], 0, 0, [], (0, 0, 0), None))
        share, keep = H.make_share(at, horizon, raw)
        got = H.encode_share(cfg, share)
        assert got == Wr.encode_share(cfg.chunk, cfg.context, at, raw), (at, cmds)
    assert kinds == {"end", "pages", "seat", "prompt", "start"}


def test_encode_share_refuses_bad_commands():
    cfg = P.device_config(P.Scenario("x", []))
    share, keep = H.make_share(0, 2, [(H.CMD_PROMPT, 0, 0, 0, list(range(9)), (0, 0, 0), None)])
    with pytest.raises(_lib.HKError, match="a prompt of 9 tokens"):
        H.encode_share(cfg, share)
    share, keep = H.make_share(0, 2, [(H.CMD_END, 4, 0, 0, [], (0, 0, 0), None)])
    with pytest.raises(_lib.HKError, match="lane 4 past the width 4"):
        H.encode_share(cfg, share)
    share, keep = H.make_share(0, 2, [(H.CMD_PAGES, 0, 30, 8, [1, 2, 3], (0, 0, 0), None)])
    with pytest.raises(_lib.HKError, match="row entries 30..33 past 32"):
        H.encode_share(cfg, share)


def _row(t):
    """A deterministic reply row for token t: three top pairs, then the token's own."""
    return [((t * 7) % 400 + 10, -0.5), ((t * 13) % 400 + 10, -1.25), ((t * 17) % 400 + 10, -2.0), (t, -0.75)]


class _LogprobFake(E.Fake):
    """The reference's test device, with a logprob list on every sampled value."""

    def drain(self):
        evs, err = super().drain()
        for e in evs:
            if isinstance(e, E.Step):
                e.lanes = [[E.Sampled(s.id, _row(s.id) if s.id >= 0 else []) for s in toks] for toks in e.lanes]
            elif isinstance(e, E.Prompted):
                e.token = E.Sampled(e.token.id, _row(e.token.id) if e.token.id >= 0 else [])
        return evs, err


class _LogprobPort(P.FakePort):
    """FakePort that also hands over the last drain's logprob lists (hk_drain_logprobs's layout:
    block slots per lane per Step, one per Prompted)."""

    def drain(self):
        evs, err = self.fake.drain()
        assert err is None
        self._lists = []
        for e in evs:
            if isinstance(e, E.Step):
                for toks in e.lanes:
                    self._lists += [toks[k].logprobs if k < len(toks) else [] for k in range(self.block)]
            elif isinstance(e, E.Prompted):
                self._lists.append(e.token.logprobs)
        self.fake.drain = lambda: (evs, None)  # FakePort.drain converts the same events
        try:
            return super().drain()
        finally:
            del self.fake.drain

    def logprobs(self):
        return self._lists


def test_tokens_carry_the_logprobs_asked():
    """src/engine/lanes.rs:53-73 through libhk's engine: a token's logprobs are its own pair,
    then the first `logprobs` of the top pairs the kernel returned with it (all of them when
    fewer), none when none were asked; the same lists as the oracle engine's."""
    asks = [P.Ask(range(1, 20), 12, sampling=E.Sampling(0.0, 1.0, 0, 0, 0)),
            P.Ask(range(3, 30), 9, sampling=E.Sampling(0.0, 1.0, 0, 0, 2)),
            P.Ask(range(5, 14), 7, sampling=E.Sampling(0.0, 1.0, 0, 0, 5))]
    sc = P.Scenario("logprobs", asks, pages=80, windows=24, block=3)

    def fake():
        return _LogprobFake(sc.pages, sc.windows, P.PAGE_ROWS, P.ENTRIES, P.WIDTH, P.CONTEXT, P.CHUNK,
                            drafts=sc.block - 1)

    jobs, sinks = E.Channel(), []
    for a in asks:
        sink = E.Sink()
        jobs.send(E.JobRun(E.Request(list(a.prompt), a.sampling, a.limit, list(a.stop), sink)))
        sinks.append(sink)
    jobs.close()
    assert E.run(P.oracle_model(sc), P.oracle_pool(sc), fake(), jobs, E.Metrics(), sc.plan, E.EngineConfig()) is None
    want = [[o.logprobs for o in s.items if isinstance(o, E.OutToken)] for s in sinks]

    port = _LogprobPort(fake(), sc.block)
    kern = H.CallbackKernel(port)
    eng = H.Engine(P.engine_config(sc), kern.ops(), keep=kern)
    reqs = [eng.submit(a.prompt, a.limit, a.stop,
                       H.Sampling(a.sampling.temperature, a.sampling.top_p, a.sampling.top_k, a.sampling.logprobs,
                                  a.sampling.seed)) for a in asks]
    eng.close()
    assert eng.run() == 0, eng.failure
    got = [eng.heard(r).logprobs for r in reqs]
    assert got == want
    assert all(lp == [] for lp in got[0])
    assert all(len(lp) == 3 for lp in got[1]) and all(len(lp) == 4 for lp in got[2])
    own = want[1][0][0]  # the first token's list: its own pair, then the top two
    assert want[1][0] == [own] + _row(own[0])[:2]
