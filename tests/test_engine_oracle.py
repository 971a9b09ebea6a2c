"""Pins the engine restatement (oracle/engine.py) to the reference's own assertions.

Each test restates one test of the reference: the 11 scenarios of tests/engine.rs:373-580, the
cache unit tests of src/engine/cache.rs:388-424 and the lane test of src/engine/lanes.rs:170-186,
with the same inputs and the same asserted values.  The product engine is then checked against
this oracle share by share (tests/test_engine_cpu.py, tests/test_engine_gpu.py).
"""
import threading

import pytest

from oracle import engine as E

PAGE_ROWS, ENTRIES, CONTEXT, WIDTH, CHUNK = 4, 16, 64, 4, 8
USIZE_MAX = E.USIZE_MAX


def greedy():
    return E.Sampling(0.0, 1.0, 0, 0, 0)


def nucleus():
    return E.Sampling(0.7, 0.9, 0, 1, 0)


class Ask:
    def __init__(self, prompt, limit, stop=(), sampling=None):
        self.prompt, self.limit, self.stop = list(prompt), limit, list(stop)
        self.sampling = sampling or greedy()


def model(block=1):
    return E.Model(context=CONTEXT, width=WIDTH, chunk=CHUNK, block=block, pad=7)


def pool(keep=0):
    return E.Pool(page_rows=PAGE_ROWS, entries=ENTRIES, window=ENTRIES, window_keep=keep)


def fake(pages, windows, drafts=0, clip=False, told=None):
    return E.Fake(pages, windows, PAGE_ROWS, ENTRIES, WIDTH, CONTEXT, CHUNK, drafts=drafts, clip=clip,
                  told=told)


def expected(a):
    return E.expected(a.prompt, a.limit, a.stop, CONTEXT)


def job(a, listening=True):
    sink = E.Sink(listening)
    return E.JobRun(E.Request(list(a.prompt), a.sampling, a.limit, list(a.stop), sink)), sink


def serve_on(mdl, pl, dev, plan, asks):
    jobs = E.Channel()
    sinks = []
    for a in asks:
        j, s = job(a)
        jobs.send(j)
        sinks.append(s)
    jobs.close()
    told = []
    dev.told = told
    metrics = E.Metrics()
    assert E.run(mdl, pl, dev, jobs, metrics, plan, E.EngineConfig()) is None, "served"
    return [E.heard(s) for s in sinks], told, metrics


def check(plan, pages, windows, keep, asks):
    got, shares, _ = serve_on(model(), pool(keep), fake(pages, windows), plan, asks)
    for i, (a, g) in enumerate(zip(asks, got)):
        assert g == expected(a), f"request {i}"
    return shares


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


def commands(shares):
    return [c for s in shares for c in s.commands]


def resumed(shares):
    return sum(1 for c in commands(shares)
               if isinstance(c, E.Seat) and c.pos > 0 and c.pos % PAGE_ROWS == 0)


# --- tests/engine.rs ----------------------------------------------------------------------

def test_next_is_the_reference_fold():
    # h = fold(1469598103, (h ^ (t + 1000 i)) * 1099511628211 mod 2^64); h % 400 + 10
    h = 1469598103
    for i, t in enumerate([5, 6, 7]):
        h = ((h ^ (t + 1000 * i)) * 1099511628211) % (1 << 64)
    assert E.next_token([5, 6, 7]) == h % 400 + 10
    assert 10 <= E.next_token(list(range(1, 20))) < 410


def test_one_request_hears_the_models_tokens():
    check(E.Plan(), 40, 20, 0, [Ask(range(1, 20), 30)])


def test_a_request_ends_at_its_stop_its_limit_or_the_context():
    prompt = list(range(1, 20))
    tokens, _ = expected(Ask(prompt, 10))
    asks = [Ask(prompt, 10, stop=[tokens[4]]), Ask(range(1, 60), 100), Ask(prompt, 0),
            Ask(range(0, CONTEXT), 5), Ask(range(0, CONTEXT - 1), 5)]
    check(E.Plan(), 80, 20, 0, asks)


@pytest.mark.parametrize("plan", [E.Plan(), E.Plan(budget=12), E.Plan(every=3),
                                  E.Plan(budget=20, every=2)])
def test_more_requests_than_lanes_share_their_prefixes(plan):
    shares = check(plan, 80, 24, 0, conversations())
    assert resumed(shares) > 0, f"{plan}: no prompt resumed a prefix"


def test_a_small_pool_evicts_and_waits():
    asks = conversations()
    check(E.Plan(), 16, 10, 0, asks)
    check(E.Plan(budget=16, headroom=4), 16, 10, 1, asks)


def test_a_listener_gone_ends_its_request_and_the_rest_run():
    jobs = E.Channel()
    asks = [Ask([i + 1] * 9, 20) for i in range(6)]
    sinks = []
    for i, a in enumerate(asks):
        j, s = job(a, listening=(i % 2 == 0))
        jobs.send(j)
        sinks.append(s)
    jobs.close()
    assert E.run(model(), pool(0), fake(80, 24), jobs, E.Metrics(), E.Plan(), E.EngineConfig()) is None
    for a, s in zip(asks, sinks):
        if s.listening:
            assert E.heard(s) == expected(a)


def test_the_cadence_sends_pieces_every_nth_step_while_lanes_decode():
    asks = [Ask([i + 1] * 30, 12) for i in range(4)]
    shares = check(E.Plan(every=4), 80, 24, 0, asks)
    prompts = [s for s in shares if any(isinstance(c, E.Prompt) for c in s.commands)]
    pairs = list(zip(prompts, prompts[1:]))[4:]
    assert any(b.at >= a.at + 3 for a, b in pairs), "the pieces ran back to back"


def test_a_request_seats_as_a_lane_frees_without_waiting_for_the_cadence():
    asks = [Ask([i + 1] * 6, limit) for i, limit in enumerate([4, 20, 20, 20, 3])]
    shares = check(E.Plan(every=1000), 80, 24, 0, asks)
    cmds = commands(shares)
    fifth = next(i for i, c in enumerate(cmds) if isinstance(c, E.Prompt) and c.tokens[0] == 5)
    ends = [i for i, c in enumerate(cmds) if isinstance(c, E.End_)]
    assert fifth < ends[3], f"the fifth prefilled before four requests had ended: {fifth} vs {ends}"


def test_requests_of_no_limit_run_at_once_on_a_pool_short_of_their_extents():
    asks = [Ask([i + 1] * 9, USIZE_MAX) for i in range(4)]
    shares = check(E.Plan(headroom=8), 31, 24, 0, asks)
    cmds = commands(shares)
    first_end = next(i for i, c in enumerate(cmds) if isinstance(c, E.End_))
    starts = sum(1 for c in cmds[:first_end] if isinstance(c, E.Start))
    assert starts == WIDTH, "every lane started before any ended"


def test_the_metrics_count_what_ran():
    asks = conversations()
    got, _, m = serve_on(model(), pool(0), fake(80, 24), E.Plan(), asks)
    m = m.total()
    assert m.prompt_tokens == sum(len(a.prompt) for a in asks)
    assert m.cached_tokens % PAGE_ROWS == 0, "cached by whole pages"
    assert m.generation_tokens == sum(len(t) for t, _ in got)
    assert (m.running, m.waiting, m.held_pages, m.pages, m.preemptions) == (0, 0, 0, 79, 0)
    assert (m.spec_tokens, m.drafts, m.top_p_clipped) == (0, 0, 0), "no drafts, no clips"


def test_drafts_clips_and_rounds_are_counted():
    asks = conversations()
    for i, a in enumerate(asks):
        if i % 2 == 0:
            a.sampling = nucleus()
    got, shares, metrics = serve_on(model(block=3), pool(0), fake(80, 24, drafts=2, clip=True),
                                    E.Plan(), asks)
    for i, (a, g) in enumerate(zip(asks, got)):
        assert g == expected(a), f"request {i}"
    rounds, m = metrics.iteration_tokens, metrics.total()
    drafts, accepted = m.drafts, m.accepted_tokens()
    assert m.spec_tokens == 2
    assert drafts > 0 and accepted > 0
    assert m.draft_tokens() == 2 * drafts
    per_pos = m.accepted_per_pos
    assert per_pos[0] >= per_pos[1] and per_pos[1] > 0 and all(c == 0 for c in per_pos[2:]), per_pos
    assert sum(per_pos) == accepted
    assert len(per_pos) <= E.EngineConfig().max_draft_positions
    assert m.generation_tokens <= accepted + drafts + len(asks)
    cmds = commands(shares)
    prompts = [len(c.tokens) for c in cmds if isinstance(c, E.Prompt)]
    seats = sum(1 for c in cmds if isinstance(c, E.Seat) and c.sampling.nucleated())
    assert m.top_p_clipped == seats, "every nucleus chunk's clip"
    assert 0 < m.top_p_clipped < len(prompts)
    assert int(rounds.sum) == sum(prompts) + m.generation_tokens, "a round's pieces and tokens heard"
    assert sum(rounds.counts) > 0


def test_a_reset_empties_the_prefix_cache():
    jobs = E.Channel()
    told = []
    metrics = E.Metrics()
    result = {}
    loop = threading.Thread(target=lambda: result.setdefault(
        "r", E.run(model(), pool(0), fake(80, 24, told=told), jobs, metrics, E.Plan(),
                   E.EngineConfig())))
    loop.start()
    a = Ask(range(1, 20), 6)
    seen = [0]

    def run_one():
        j, s = job(a)
        jobs.send(j)
        while not any(isinstance(o, E.OutEnd) for o in s.items):
            threading.Event().wait(0.001)
        assert E.heard(s) == expected(a)
        new, seen[0] = told[seen[0]:], len(told)
        return next((c.pos for sh in new for c in sh.commands if isinstance(c, E.Seat)), None)

    def reset():
        answer = []
        jobs.send(E.JobReset(answer))
        while not answer:
            threading.Event().wait(0.001)
        return answer[0]

    assert run_one() == 0
    assert run_one() == 16, "the second resumed the first's prefix"
    cached = metrics.total().cached_tokens
    assert cached == 16, "the metrics tell the prefix cached"
    assert reset() == (len(a.prompt) + a.limit - 1) // PAGE_ROWS, "the tree's whole pages freed"
    assert run_one() == 0, "nothing resumed after the reset"
    assert metrics.total().cached_tokens == cached, "nothing more cached"
    assert reset() == (len(a.prompt) + a.limit - 1) // PAGE_ROWS
    assert reset() == 0, "an empty tree frees nothing"
    jobs.close()
    loop.join(timeout=60)
    assert result["r"] is None, "served"


# --- src/engine/cache.rs unit tests -------------------------------------------------------

def cache_pool(keep):
    return E.Pool(page_rows=4, entries=8, window=8, window_keep=keep)


def served(c, lane, tokens, n):
    cached = c.admit(lane, tokens[:n], len(tokens) + 1)
    c.hold(lane, cached, n)
    c.hold(lane, len(tokens) - 1, len(tokens) + 1)
    c.run_to(lane, len(tokens) + 1)
    c.finish(lane, tokens[:len(tokens) - 1])
    return cached


def test_a_prompt_resumes_from_the_longest_prefix_kept():
    c = E.Cache(cache_pool(0), 40, 20, 2)
    a = list(range(15))
    assert served(c, 0, a, 13) == 0
    assert served(c, 1, a, 13) == 12
    b = a[:9] + [99, 98, 97, 96]
    assert c.admit(0, b, 14) == 0, "page 1 holds no window page: nothing to resume from"


def test_pages_evicted_least_recently_used_and_a_prompt_too_long_never_fits():
    c = E.Cache(cache_pool(0), 7, 20, 2)
    a, b = list(range(15)), list(range(100, 115))
    served(c, 0, a, 13)
    served(c, 0, b, 13)
    assert served(c, 0, b, 13) == 12, "b evicted a, not itself"
    assert served(c, 0, a, 13) == 0
    with pytest.raises(E.WaitNever):
        c.admit(0, list(range(40)), 41)


def test_a_row_goes_as_its_changed_runs():
    c = E.Cache(cache_pool(0), 40, 20, 1)
    c.admit(0, [1] * 6, 8)
    c.hold(0, 0, 6)
    assert len(c.pages_cmds(0, E.EngineConfig().gap)) == 1
    assert c.pages_cmds(0, E.EngineConfig().gap) == [], "nothing changed"
    c.hold(0, 5, 8)
    c.run_to(0, 8)
    p = c.pages_cmds(0, E.EngineConfig().gap)
    assert len(p) == 1 and isinstance(p[0], E.Pages) and p[0].upto == 8, p


# --- src/engine/lanes.rs unit test --------------------------------------------------------

def test_a_token_goes_with_the_logprobs_asked_and_is_taken():
    sink = E.Sink()
    sampling = E.Sampling(0.0, 1.0, 0, 0, 2)
    l = E.Lane(0, 1, E.Request([1], sampling, 5, [], sink), 1, 0)
    row = [(7, -0.1), (8, -2.0), (9, -3.0), (7, -0.1)]
    assert l.hear(E.Sampled(7, row), 64) is None
    t = sink.items[0]
    assert isinstance(t, E.OutToken)
    assert t.logprobs == [(7, -0.1), (7, -0.1), (8, -2.0)], "its own, then the top two"
    assert (l.request.prompt, l.request.limit) == ([1, 7], 4)
