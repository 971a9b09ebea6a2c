"""Test helpers: the reference's engine scenarios, runnable on the oracle engine or on libhk's
engine, with the reference's test device (oracle.engine.Fake) or libhk's device kernel.

Test infrastructure only (imports the oracle)."""
from __future__ import annotations

import numpy as np

from hyperkernel_b200 import engine as H
from oracle import engine as E

PAGE_ROWS, ENTRIES, CONTEXT, WIDTH, CHUNK = 4, 16, 64, 4, 8


class Ask:
    def __init__(self, prompt, limit, stop=(), sampling=None):
        self.prompt, self.limit, self.stop = list(prompt), limit, list(stop)
        self.sampling = sampling or E.Sampling(0.0, 1.0, 0, 0, 0)


def nucleus():
    return E.Sampling(0.7, 0.9, 0, 1, 0)


def expected(a):
    return E.expected(a.prompt, a.limit, a.stop, CONTEXT)


def conversations():
    system = list(range(100, 111))
    asks = []
    for c in range(3):
        prompt = system + [200 + c, 201, 202]
        for turn in range(3):
            a = Ask(prompt, 6)
            reply, _ = expected(a)
            asks.append(a)
            prompt = prompt + reply + [300 + turn, 301]
    return asks


def mixed_conversations():
    asks = conversations()
    for i, a in enumerate(asks):
        if i % 2 == 0:
            a.sampling = nucleus()
    return asks


class Scenario:
    """One engine::run of the reference's tests/engine.rs, with its device's shape."""

    def __init__(self, name, asks, plan=None, pages=80, windows=24, keep=0, block=1, clip=False,
                 hangup=()):
        self.name, self.asks, self.plan = name, asks, plan or E.Plan()
        self.pages, self.windows, self.keep, self.block, self.clip = pages, windows, keep, block, clip
        self.hangup = set(hangup)

    def __repr__(self):
        return self.name


def scenarios():
    prompt = list(range(1, 20))
    tokens, _ = expected(Ask(prompt, 10))
    return [
        Scenario("one_request", [Ask(range(1, 20), 30)], pages=40, windows=20),
        Scenario("stop_limit_context", [Ask(prompt, 10, stop=[tokens[4]]), Ask(range(1, 60), 100),
                                        Ask(prompt, 0), Ask(range(0, CONTEXT), 5),
                                        Ask(range(0, CONTEXT - 1), 5)], pages=80, windows=20),
        Scenario("prefixes_default", conversations()),
        Scenario("prefixes_budget12", conversations(), E.Plan(budget=12)),
        Scenario("prefixes_every3", conversations(), E.Plan(every=3)),
        Scenario("prefixes_budget20_every2", conversations(), E.Plan(budget=20, every=2)),
        Scenario("small_pool", conversations(), pages=16, windows=10),
        Scenario("small_pool_budget_keep", conversations(), E.Plan(budget=16, headroom=4), pages=16,
                 windows=10, keep=1),
        Scenario("listener_gone", [Ask([i + 1] * 9, 20) for i in range(6)], hangup={1, 3, 5}),
        Scenario("cadence_every4", [Ask([i + 1] * 30, 12) for i in range(4)], E.Plan(every=4)),
        Scenario("seat_without_cadence", [Ask([i + 1] * 6, lim) for i, lim in enumerate([4, 20, 20, 20, 3])],
                 E.Plan(every=1000)),
        Scenario("no_limit", [Ask([i + 1] * 9, E.USIZE_MAX) for i in range(4)], E.Plan(headroom=8),
                 pages=31),
        Scenario("drafts_clips", mixed_conversations(), block=3, clip=True),
    ]


def oracle_model(sc):
    return E.Model(context=CONTEXT, width=WIDTH, chunk=CHUNK, block=sc.block, pad=7)


def oracle_pool(sc):
    return E.Pool(page_rows=PAGE_ROWS, entries=ENTRIES, window=ENTRIES, window_keep=sc.keep)


def oracle_fake(sc):
    return E.Fake(sc.pages, sc.windows, PAGE_ROWS, ENTRIES, WIDTH, CONTEXT, CHUNK, drafts=sc.block - 1,
                  clip=sc.clip)


# ------------------------------------------------------------------------------------------
# normal forms, so runs on either engine compare with ==
# ------------------------------------------------------------------------------------------

def _f32(x):
    return float(np.float32(x))


def norm_command(c):
    if isinstance(c, E.End_):
        return ("end", c.lane)
    if isinstance(c, E.Pages):
        return ("pages", c.lane, c.from_, c.upto, tuple(c.row))
    if isinstance(c, E.Seat):
        s = c.sampling
        return ("seat", c.lane, c.pos, tuple(c.back),
                (_f32(s.temperature), _f32(s.top_p), s.top_k, s.seed, s.logprobs))
    if isinstance(c, E.Prompt):
        return ("prompt", c.lane, tuple(c.tokens))
    return ("start", c.lane)


def norm_share(s):
    return (s.at, s.horizon, tuple(norm_command(c) for c in s.commands))


def from_raw(kind, lane, pos, upto, data, back, sampling):
    """An hk_command (engine.read_share tuple) as the oracle's Command."""
    if kind == H.CMD_END:
        return E.End_(lane)
    if kind == H.CMD_PAGES:
        return E.Pages(lane, pos, upto, tuple(data))
    if kind == H.CMD_SEAT:
        t, p, k, lp, seed = sampling
        return E.Seat(lane, pos, tuple(back), E.Sampling(t, p, k, seed, lp))
    if kind == H.CMD_PROMPT:
        return E.Prompt(lane, tuple(data))
    return E.Start(lane)


def to_raw(c):
    if isinstance(c, E.End_):
        return (H.CMD_END, c.lane, 0, 0, [], (0, 0, 0), None)
    if isinstance(c, E.Pages):
        return (H.CMD_PAGES, c.lane, c.from_, c.upto, list(c.row), (0, 0, 0), None)
    if isinstance(c, E.Seat):
        s = c.sampling
        return (H.CMD_SEAT, c.lane, c.pos, 0, [], tuple(c.back),
                H.Sampling(s.temperature, s.top_p, s.top_k, s.logprobs, s.seed))
    if isinstance(c, E.Prompt):
        return (H.CMD_PROMPT, c.lane, 0, 0, list(c.tokens), (0, 0, 0), None)
    return (H.CMD_START, c.lane, 0, 0, [], (0, 0, 0), None)


class FakePort:
    """The reference's test device behind hk_kernel_ops (for CallbackKernel)."""

    def __init__(self, fake, block):
        self.fake, self.block = fake, block
        self.shares = []

    def pools(self):
        return self.fake.pools()

    def push(self, raw):
        at, horizon, cmds = H.read_share(raw)
        share = E.Share(at, horizon, tuple(from_raw(*c) for c in cmds))
        self.shares.append(share)
        self.fake.push(share)

    def drain(self):
        evs, err = self.fake.drain()
        assert err is None
        out, flat = [], []
        for e in evs:
            if isinstance(e, E.Idle):
                out.append((H.EV_IDLE, e.step, 0, 0, 0, 0))
            elif isinstance(e, E.Step):
                off = len(flat)
                for toks in e.lanes:
                    flat += [t.id for t in toks] + [-2] * (self.block - len(toks))
                out.append((H.EV_STEP, e.step, 0, 0, 0, off))
            else:
                out.append((H.EV_PROMPTED, 0, e.lane, e.token.id, int(e.clipped), 0))
        return out, flat


class DevicePort:
    """libhk's device kernel (hk_open) behind hk_kernel_ops, recording the shares pushed."""

    def __init__(self, device: H.Device):
        self.device = device
        self.shares = []

    def pools(self):
        return self.device.pools()

    def push(self, raw):
        at, horizon, cmds = H.read_share(raw)
        self.shares.append(E.Share(at, horizon, tuple(from_raw(*c) for c in cmds)))
        rc = self.device.push_raw(raw)
        if rc:
            raise _Failed(rc)

    def drain(self):
        import ctypes as C
        cap, ids_cap = 64, 1024
        while True:
            evs = (H.Event * cap)()
            ids = (H.I32 * ids_cap)()
            n, ids_n = H.SZ(), H.SZ()
            rc = self.device.drain_raw(evs, cap, C.byref(n), ids, ids_cap, C.byref(ids_n))
            if rc == -5:
                cap, ids_cap = max(cap, n.value), max(ids_cap, ids_n.value)
                continue
            if rc:
                raise _Failed(rc)
            return ([(e.kind, e.step, e.lane, e.token, e.clipped, e.ids) for e in evs[:n.value]],
                    list(ids[:ids_n.value]))


class _Failed(RuntimeError):
    def __init__(self, code):
        from hyperkernel_b200 import _lib
        super().__init__(_lib.last_error())
        self.code = code


# ------------------------------------------------------------------------------------------
# runs
# ------------------------------------------------------------------------------------------

class Result:
    def __init__(self, heard, shares, metrics, accepted, counts, total):
        self.heard, self.shares, self.metrics = heard, shares, metrics
        self.accepted, self.counts, self.total = accepted, counts, total


def run_oracle(sc) -> Result:
    jobs = E.Channel()
    sinks = []
    for i, a in enumerate(sc.asks):
        sink = E.Sink(listening=i not in sc.hangup)
        jobs.send(E.JobRun(E.Request(list(a.prompt), a.sampling, a.limit, list(a.stop), sink)))
        sinks.append(sink)
    jobs.close()
    told = []
    fake = oracle_fake(sc)
    fake.told = told
    metrics = E.Metrics()
    assert E.run(oracle_model(sc), oracle_pool(sc), fake, jobs, metrics, sc.plan, E.EngineConfig()) is None
    heard = []
    for i, s in enumerate(sinks):
        if i in sc.hangup:
            heard.append(None)
            continue
        toks = [o.id for o in s.items if isinstance(o, E.OutToken)]
        end = next(o for o in s.items if isinstance(o, E.OutEnd))
        seated = [o.cached for o in s.items if isinstance(o, E.OutSeated)]
        heard.append((seated, toks, end.kind, end.message))
    m = metrics.total()
    fields = {n: getattr(m, n) for n, _ in H.StepMetrics._fields_}
    return Result(heard, [norm_share(s) for s in told], fields, list(m.accepted_per_pos),
                  list(metrics.iteration_tokens.counts), metrics.iteration_tokens.sum)


def engine_config(sc):
    return H.engine_config(page_rows=PAGE_ROWS, entries=ENTRIES, window=ENTRIES, window_keep=sc.keep,
                           context=CONTEXT, width=WIDTH, chunk=CHUNK, block=sc.block, pad=7,
                           budget=sc.plan.budget, every=sc.plan.every, headroom=sc.plan.headroom)


def device_config(sc, device=0, transport=0):
    """transport 0: a launch per batch and step; 1: the resident ring executor."""
    return H.Config(model=H.MODEL_FNV, page_rows=PAGE_ROWS, entries=ENTRIES, window=ENTRIES, width=WIDTH,
                    context=CONTEXT, chunk=CHUNK, block=sc.block, pages=sc.pages, window_pages=sc.windows,
                    clip=int(sc.clip), device=device, transport=transport)


def run_hk(sc, port) -> Result:
    """libhk's engine over `port` (a FakePort or a DevicePort through CallbackKernel)."""
    kern = H.CallbackKernel(port)
    return _run_engine(sc, kern.ops(), kern, port.shares)


def run_hk_native(sc, device: H.Device) -> Result:
    """libhk's engine over libhk's device kernel with no Python in the loop."""
    return _run_engine(sc, device.ops(), device, None)


def _run_engine(sc, ops, keep, shares) -> Result:
    eng = H.Engine(engine_config(sc), ops, keep=keep)
    reqs = []
    for a in sc.asks:
        s = a.sampling
        reqs.append(eng.submit(a.prompt, a.limit, a.stop,
                               H.Sampling(s.temperature, s.top_p, s.top_k, s.logprobs, s.seed)))
    for i in sc.hangup:
        eng.hangup(reqs[i])
    eng.close()
    rc = eng.run()
    assert rc == 0, eng.failure
    heard = []
    for i, r in enumerate(reqs):
        if i in sc.hangup:
            heard.append(None)
            continue
        h = eng.heard(r)
        heard.append((h.seated, h.tokens, h.end, h.message))
    m, acc, counts, total = eng.metrics()
    return Result(heard, [norm_share(s) for s in shares] if shares is not None else None, m, acc, counts,
                  total)


def assert_same(got: Result, want: Result, shares=True):
    assert got.heard == want.heard
    if shares:
        assert len(got.shares) == len(want.shares)
        for i, (g, w) in enumerate(zip(got.shares, want.shares)):
            assert g == w, f"share {i}"
    assert got.metrics == want.metrics
    assert got.accepted == want.accepted
    assert got.counts == want.counts
    assert got.total == want.total
