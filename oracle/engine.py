"""Restatement of the reference's continuous-batching engine — TEST INFRASTRUCTURE ONLY.

A Python restatement of the scheduler above the `Kernel` boundary, used to pin the product
engine (hyperkernel_b200/csrc/engine.cpp) share by share.  It follows, file by file:

  src/engine/cache.rs    Units :46-79, Cache :81-359 (admit, hold, pages, finish, reset,
                          find, freeable, lru, evict_page, evict_window, remember)
  src/engine/lanes.rs    Lane :7-74 (next_chunk, chunk, ahead, hear), Lanes :82-159
  src/engine/clock.rs    Clock :3-31
  src/engine/pacing.rs   Plan, Pacing, Allowance :1-61
  src/engine/metrics.rs  StepMetrics :4-50, Metrics :52-75, Hist :77-111
  src/engine/request.rs  Request, Sampling, Out, End :6-64
  src/engine/mod.rs      EngineConfig :25-36, run :38-74, Engine :76-359
  src/gpu/mod.rs         Share, Command, Event, Sampled :13-40

and the reference's test harness tests/engine.rs: next() :56-62 (the FNV "model"), Fake
:64-239, expected() :252-268.  It is pinned by the reference's own assertions
(tests/test_engine_oracle.py restates the 11 scenarios of tests/engine.rs:373-580 and the unit
tests of src/engine/cache.rs:388-424 and src/engine/lanes.rs:170-186).
"""
from __future__ import annotations

import threading
from collections import deque
from dataclasses import dataclass, field
from typing import Optional

USIZE_MAX = (1 << 64) - 1


# ------------------------------------------------------------------------------------------
# boundary types (src/gpu/mod.rs:13-40)
# ------------------------------------------------------------------------------------------

@dataclass(frozen=True)
class Sampling:
    temperature: float = 0.0
    top_p: float = 1.0
    top_k: int = 0
    seed: int = 0
    logprobs: int = 0

    def nucleated(self) -> bool:
        return self.temperature > 0.0 and (self.top_p < 1.0 or self.top_k > 0)


@dataclass(frozen=True)
class End_:
    lane: int


@dataclass(frozen=True)
class Pages:
    lane: int
    from_: int
    upto: int
    row: tuple


@dataclass(frozen=True)
class Seat:
    lane: int
    pos: int
    back: tuple
    sampling: Sampling


@dataclass(frozen=True)
class Prompt:
    lane: int
    tokens: tuple


@dataclass(frozen=True)
class Start:
    lane: int


@dataclass(frozen=True)
class Share:
    at: int
    horizon: int
    commands: tuple


@dataclass
class Sampled:
    id: int
    logprobs: list = field(default_factory=list)


@dataclass
class Idle:
    step: int


@dataclass
class Step:
    step: int
    lanes: list


@dataclass
class Prompted:
    lane: int
    token: Sampled
    clipped: bool


# ------------------------------------------------------------------------------------------
# requests and outputs (src/engine/request.rs)
# ------------------------------------------------------------------------------------------

@dataclass
class OutSeated:
    cached: int


@dataclass
class OutToken:
    id: int
    logprobs: list


@dataclass
class OutEnd:
    kind: str          # "stop" | "length" | "refused"
    message: str = ""


class Sink:
    """The per-request output channel; a dropped listener makes send() fail."""

    def __init__(self, listening: bool = True):
        self.items = []
        self.listening = listening

    def send(self, item) -> bool:
        if not self.listening:
            return False
        self.items.append(item)
        return True


@dataclass
class Request:
    prompt: list
    sampling: Sampling
    limit: int
    stop: list
    out: Sink

    def took(self, tid: int):
        self.prompt.append(tid)
        self.limit -= 1

    def reach(self, headroom: int, context: int, block: int) -> int:
        return min(len(self.prompt) + min(self.limit, headroom), context) + block - 1


class Channel:
    """mpsc::channel<Job>: send / close, try_recv / blocking recv."""

    EMPTY, CLOSED = object(), object()

    def __init__(self):
        self.q = deque()
        self.closed = False
        self.cv = threading.Condition()

    def send(self, job):
        with self.cv:
            self.q.append(job)
            self.cv.notify()

    def close(self):
        with self.cv:
            self.closed = True
            self.cv.notify()

    def try_recv(self):
        with self.cv:
            if self.q:
                return self.q.popleft()
            return Channel.CLOSED if self.closed else Channel.EMPTY

    def recv(self):
        with self.cv:
            while not self.q and not self.closed:
                self.cv.wait()
            return self.q.popleft() if self.q else Channel.CLOSED

    def drain(self):
        with self.cv:
            items = list(self.q)
            self.q.clear()
            return items


@dataclass
class JobRun:
    request: Request


@dataclass
class JobReset:
    answer: list  # the freed page count is appended


# ------------------------------------------------------------------------------------------
# configuration (src/bundle.rs Pool/Model fields the engine reads; src/engine/mod.rs:25-36)
# ------------------------------------------------------------------------------------------

@dataclass
class Pool:
    page_rows: int
    entries: int
    window: int
    window_keep: int = 0


@dataclass
class Model:
    context: int
    width: int          # last of `batches`
    chunk: int          # chunks[0]
    block: int = 1
    pad: int = 7


@dataclass
class EngineConfig:
    gap: int = 16
    lead: int = 2
    ahead: int = 16
    max_draft_positions: int = 16


@dataclass
class Plan:
    budget: Optional[int] = None
    every: int = 1
    headroom: int = 2048


# ------------------------------------------------------------------------------------------
# cache (src/engine/cache.rs)
# ------------------------------------------------------------------------------------------

class Units:
    def __init__(self, n: int):
        self.held = [0] * max(n, 1)
        self.held[0] = 1
        self.free = list(range(n - 1, 0, -1))

    def take(self):
        if not self.free:
            return None
        u = self.free.pop()
        self.held[u] = 1
        return u

    def share(self, u):
        self.held[u] += 1

    def release(self, u):
        self.held[u] -= 1
        if self.held[u] == 0:
            self.free.append(u)

    def once(self, u) -> bool:
        return self.held[u] == 1


class Place:
    def __init__(self, row_len):
        self.pages = []
        self.window = []
        self.promise = 0
        self.upto = 0
        self.sent = [0] * row_len
        self.sent_upto = 0


class Node:
    __slots__ = ("parent", "tokens", "page", "window", "children", "used")

    def __init__(self, parent, tokens, page, window, children, used):
        self.parent, self.tokens, self.page = parent, tokens, page
        self.window, self.children, self.used = window, children, used


class WaitLater(Exception):
    pass


class WaitNever(Exception):
    pass


class HoldError(Exception):
    pass


class Cache:
    def __init__(self, pool: Pool, pages: int, window_pages: int, lanes: int):
        self.rows = pool.page_rows
        self.entries = pool.entries
        self.window = pool.window
        self.keep = pool.window_keep > 0
        self.pages = Units(pages)
        self.windows = Units(window_pages)
        self.lanes = [Place(pool.entries + pool.window) for _ in range(lanes)]
        self.nodes = {}      # id -> Node, ids ascending (BTreeMap order)
        self.edges = {}
        self.ids = 0
        self.clock = 0

    def admit(self, lane, prompt, extent) -> int:
        p = self.rows
        extent = min(extent, self.entries * p)
        if len(prompt) > extent:
            raise WaitNever(f"a prompt of {len(prompt)} tokens past a row's {self.entries} pages of {p}")
        path = self.find(prompt)
        need = -(-extent // p) - len(path)
        if self.spare() + self.freeable(path) < need:
            live = any(l.pages or l.promise > 0 for l in self.lanes)
            if not live or need + len(path) > len(self.pages.held) - 1:
                raise WaitNever(f"{need} pages more than its {len(path)} of a pool of "
                                f"{len(self.pages.held) - 1}")
            raise WaitLater()
        while self.spare() < need:
            assert self.evict_page(path), "admission counted pages the tree does not free"
        now = self.tick()
        for n in path:
            node = self.nodes[n]
            node.used = now
            self.pages.share(node.page)
            self.lanes[lane].pages.append(node.page)
        if path:
            w = self.nodes[path[-1]].window
            assert w is not None, "a resume's window page"
            self.windows.share(w)
            self.lanes[lane].window = [None] * (len(path) - 1) + [w]
        self.lanes[lane].promise = need
        return len(path) * p

    def hold(self, lane, start, end):
        p = self.rows
        last = (end - 1) // p
        if last >= self.entries or last >= self.window:
            raise HoldError(f"position {end - 1} past a row's {min(self.entries, self.window)} pages of {p}")
        while len(self.lanes[lane].pages) <= last:
            place = self.lanes[lane]
            if place.promise > 0:
                place.promise -= 1
                page = self.pages.take()
            elif self.spare() > 0:
                page = self.pages.take()
            elif self.evict_page([]):
                continue
            else:
                raise HoldError("no page free")
            assert page is not None, "a free page"
            self.lanes[lane].pages.append(page)
        frm = max((start + 1) // p - 1, 0)
        place = self.lanes[lane]
        for i in range(min(frm, len(place.window))):
            if place.window[i] is not None:
                self.windows.release(place.window[i])
                place.window[i] = None
        if len(place.window) <= last:
            place.window.extend([None] * (last + 1 - len(place.window)))
        for k in range(frm, last + 1):
            while self.lanes[lane].window[k] is None:
                w = self.windows.take()
                if w is not None:
                    self.lanes[lane].window[k] = w
                elif self.evict_window():
                    pass
                else:
                    raise HoldError("no window page free")

    def run_to(self, lane, upto):
        self.lanes[lane].upto = upto

    def upto(self, lane):
        return self.lanes[lane].upto

    def pages_cmds(self, lane, gap):
        place = self.lanes[lane]
        pages = (list(place.pages) + [0] * self.entries)[: self.entries]
        window = ([0 if w is None else w for w in place.window] + [0] * self.window)[: self.window]
        row = pages + window
        runs = []
        for k in range(len(row)):
            if row[k] != place.sent[k]:
                if runs and k < runs[-1][1] + gap:
                    runs[-1][1] = k + 1
                else:
                    runs.append([k, k + 1])
        if not runs and place.upto == place.sent_upto:
            return []
        if not runs:
            runs.append([0, 0])
        upto = place.upto
        cmds = [Pages(lane, a, upto, tuple(row[a:b])) for a, b in runs]
        place.sent, place.sent_upto = row, place.upto
        return cmds

    def finish(self, lane, tokens):
        self.remember(lane, tokens)
        place = self.lanes[lane]
        for p in place.pages:
            self.pages.release(p)
        place.pages = []
        for w in place.window:
            if w is not None:
                self.windows.release(w)
        place.window = []
        place.promise, place.upto, place.sent_upto = 0, 0, 0

    def pool(self):
        return len(self.pages.held) - 1

    def held(self):
        return sum(len(l.pages) for l in self.lanes)

    def reset(self):
        free = len(self.pages.free)
        nodes, self.nodes = self.nodes, {}
        for node in nodes.values():
            self.pages.release(node.page)
            if node.window is not None:
                self.windows.release(node.window)
        self.edges.clear()
        return len(self.pages.free) - free

    def tick(self):
        self.clock += 1
        return self.clock

    def spare(self):
        return len(self.pages.free) - sum(l.promise for l in self.lanes)

    def find(self, prompt):
        path, best, parent = [], 0, None
        r = self.rows
        for i in range(len(prompt) // r):
            block = tuple(prompt[i * r:(i + 1) * r])
            if (len(path) + 1) * r >= len(prompt):
                break
            n = self.edges.get((parent, block))
            if n is None:
                break
            path.append(n)
            if self.nodes[n].window is not None:
                best = len(path)
            parent = n
        return path[:best]

    def freeable(self, keep):
        return sum(1 for n, node in self.nodes.items() if n not in keep and self.pages.once(node.page))

    def lru(self, keep, pick):
        best = None
        for n, node in self.nodes.items():
            if n in keep or not pick(node):
                continue
            if best is None or node.used < self.nodes[best].used:
                best = n
        return best

    def evict_page(self, keep):
        n = self.lru(keep, lambda node: node.children == 0 and self.pages.once(node.page))
        if n is None:
            return False
        node = self.nodes.pop(n)
        del self.edges[(node.parent, node.tokens)]
        if node.parent is not None:
            self.nodes[node.parent].children -= 1
        self.pages.release(node.page)
        if node.window is not None:
            self.windows.release(node.window)
        return True

    def evict_window(self):
        alone = lambda node: node.window is not None and self.windows.once(node.window)
        interior = self.lru([], lambda node: alone(node) and node.children > 0) if self.keep else None
        n = interior if interior is not None else self.lru([], alone)
        if n is None:
            return False
        w = self.nodes[n].window
        self.nodes[n].window = None
        self.windows.release(w)
        return True

    def remember(self, lane, tokens):
        now = self.tick()
        parent = None
        r = self.rows
        for k in range(len(tokens) // r):
            block = tuple(tokens[k * r:(k + 1) * r])
            key = (parent, block)
            n = self.edges.get(key)
            if n is None:
                if k >= len(self.lanes[lane].pages):
                    return
                page = self.lanes[lane].pages[k]
                self.pages.share(page)
                self.ids += 1
                n = self.ids
                self.nodes[n] = Node(parent, block, page, None, 0, now)
                self.edges[key] = n
                if parent is not None:
                    self.nodes[parent].children += 1
            win = self.lanes[lane].window
            held = win[k] if k < len(win) else None
            node = self.nodes[n]
            node.used = now
            if node.window is None and held is not None:
                node.window = held
                self.windows.share(held)
            parent = n


# ------------------------------------------------------------------------------------------
# lanes (src/engine/lanes.rs)
# ------------------------------------------------------------------------------------------

class Lane:
    def __init__(self, lane, seat, request, sent, frm=None):
        self.lane, self.seat, self.request, self.sent, self.frm = lane, seat, request, sent, frm

    def decoding(self):
        return self.frm is not None

    def decodes_at(self, step):
        return self.frm is not None and step >= self.frm

    def written(self):
        return len(self.request.prompt) - 1 if self.decoding() else self.sent

    def next_chunk(self, rows, tokens):
        n = min(len(self.request.prompt) - self.sent, rows, tokens)
        return (self.sent, self.sent + n)

    def chunk(self, piece, pad):
        s, e = piece
        toks = self.request.prompt
        back = tuple(toks[s + j - 3] if s + j >= 3 else pad for j in range(3))
        out = [Seat(self.lane, s, back, self.request.sampling), Prompt(self.lane, tuple(toks[s:e]))]
        if e == len(toks):
            out.append(Start(self.lane))
        return out

    def ahead(self, upto, context, block, ahead):
        nxt = len(self.request.prompt) - 1
        last = min(len(self.request.prompt) + self.request.limit, context) - 2
        end = min(nxt + ahead, last + 1) + block - 1
        if end > nxt + block - 1 and upto < end and upto < nxt + ahead // 2 + block:
            return (nxt, end)
        return None

    def hear(self, t: Sampled, context):
        if t.id < 0:
            return OutEnd("refused", "the kernel's logits were not finite")
        r = self.request
        ask = r.sampling.logprobs
        if t.logprobs and ask > 0:
            own, top = t.logprobs[-1], t.logprobs[:-1]
            logprobs = [own] + top[:ask]
        else:
            logprobs = []
        if not r.out.send(OutToken(t.id, logprobs)):
            return OutEnd("stop")
        if t.id in r.stop:
            return OutEnd("stop")
        r.took(t.id)
        if r.limit == 0 or len(r.prompt) >= context:
            return OutEnd("length")
        return None


class Lanes:
    FREE, ENDING = "free", "ending"

    def __init__(self, width):
        self.slots = [Lanes.FREE] * width
        self.seats = 0

    def free(self):
        for i, s in enumerate(self.slots):
            if s is Lanes.FREE:
                return i
        return None

    def seat(self, lane, request, cached):
        self.seats += 1
        self.slots[lane] = Lane(lane, self.seats, request, cached)

    def take(self, lane):
        l = self.slots[lane]
        assert isinstance(l, Lane), f"lane {lane} taken unheld"
        self.slots[lane] = Lanes.ENDING
        return l

    def ended(self):
        ending = [i for i, s in enumerate(self.slots) if s is Lanes.ENDING]
        for i in ending:
            self.slots[i] = Lanes.FREE
        return ending

    def get(self, lane):
        s = self.slots[lane]
        return s if isinstance(s, Lane) else None

    def is_empty(self):
        return all(s is Lanes.FREE for s in self.slots)

    def _by_seat(self, pick):
        ls = [s for s in self.slots if isinstance(s, Lane) and pick(s)]
        ls.sort(key=lambda l: l.seat)
        return [l.lane for l in ls]

    def held(self):
        return self._by_seat(lambda l: True)

    def prompting(self):
        return self._by_seat(lambda l: not l.decoding())

    def decoding(self):
        return self._by_seat(lambda l: l.decoding())

    def newest(self):
        h = self.held()
        return h[-1] if h else None


# ------------------------------------------------------------------------------------------
# clock, pacing, metrics
# ------------------------------------------------------------------------------------------

class Clock:
    def __init__(self, lead):
        self.lead, self.seen, self.granted = lead, 0, 0

    def saw(self, step):
        self.seen = step

    def next(self):
        return self.granted

    def grant(self, commands, decoding):
        running_out = self.seen + self.lead >= self.granted
        if not commands and not (decoding and running_out):
            return None
        at = self.granted
        frm = self.seen if not commands else max(self.seen, max(at - 1, 0))
        self.granted = frm + self.lead + 1
        return Share(at, frm + self.lead, tuple(commands))


class Allowance:
    def __init__(self, chunks, tokens):
        self.chunks, self.tokens = chunks, tokens

    def left(self):
        return self.chunks > 0 and self.tokens > 0

    def spend(self, n):
        self.chunks -= 1
        self.tokens -= n


class Pacing:
    def __init__(self, plan: Plan):
        self.plan, self.steps = plan, 0

    def due(self, decoding):
        return decoding == 0 or self.steps + 1 >= self.plan.every

    def allowance(self, decoding, block):
        if self.plan.budget is None:
            return Allowance(1, USIZE_MAX)
        return Allowance(USIZE_MAX, max(self.plan.budget - decoding * block, 0))

    def headroom(self):
        return self.plan.headroom

    def stepped(self):
        self.steps += 1

    def prefilled(self):
        self.steps = 0


@dataclass
class StepMetrics:
    running: int = 0
    waiting: int = 0
    held_pages: int = 0
    pages: int = 0
    spec_tokens: int = 0
    prompt_tokens: int = 0
    cached_tokens: int = 0
    prefill_tokens: int = 0
    generation_tokens: int = 0
    preemptions: int = 0
    top_p_clipped: int = 0
    drafts: int = 0
    accepted_per_pos: list = field(default_factory=list)

    def then(self, nxt: "StepMetrics") -> "StepMetrics":
        n = max(len(self.accepted_per_pos), len(nxt.accepted_per_pos))
        a = self.accepted_per_pos + [0] * (n - len(self.accepted_per_pos))
        b = nxt.accepted_per_pos + [0] * (n - len(nxt.accepted_per_pos))
        return StepMetrics(nxt.running, nxt.waiting, nxt.held_pages, nxt.pages, nxt.spec_tokens,
                           self.prompt_tokens + nxt.prompt_tokens,
                           self.cached_tokens + nxt.cached_tokens,
                           self.prefill_tokens + nxt.prefill_tokens,
                           self.generation_tokens + nxt.generation_tokens,
                           self.preemptions + nxt.preemptions,
                           self.top_p_clipped + nxt.top_p_clipped, self.drafts + nxt.drafts,
                           [x + y for x, y in zip(a, b)])

    def verified(self, accepted):
        self.drafts += 1
        if len(self.accepted_per_pos) < accepted:
            self.accepted_per_pos += [0] * (accepted - len(self.accepted_per_pos))
        for i in range(accepted):
            self.accepted_per_pos[i] += 1

    def tokens(self):
        return self.prefill_tokens + self.generation_tokens

    def draft_tokens(self):
        return self.drafts * self.spec_tokens

    def accepted_tokens(self):
        return sum(self.accepted_per_pos)


class Hist:
    def __init__(self, bounds):
        self.bounds = list(bounds)
        self.counts = [0] * (len(bounds) + 1)
        self.sum = 0.0

    def observe(self, x):
        i = 0
        while i < len(self.bounds) and self.bounds[i] < x:
            i += 1
        self.counts[i] += 1
        self.sum += x


class Metrics:
    def __init__(self, bounds=(1, 8, 16, 32, 64, 128, 256, 512, 1024, 2048, 4096, 8192, 16384)):
        self._total = StepMetrics()
        self.iteration_tokens = Hist(bounds)
        self.lock = threading.Lock()

    def record(self, step: StepMetrics):
        if step.tokens() > 0:
            self.iteration_tokens.observe(float(step.tokens()))
        with self.lock:
            self._total = self._total.then(step)

    def total(self):
        with self.lock:
            return self._total


# ------------------------------------------------------------------------------------------
# the engine (src/engine/mod.rs)
# ------------------------------------------------------------------------------------------

@dataclass
class Asked:
    lane: int
    seat: int
    last: bool
    nucleated: bool


class Engine:
    def __init__(self, model: Model, pool: Pool, pools, plan: Plan, config: EngineConfig):
        self.model, self.config = model, config
        self.waiting = deque()
        self.lanes = Lanes(model.width)
        self.cache = Cache(pool, pools[0], pools[1], model.width)
        self.asked = deque()
        self.clock = Clock(config.lead)
        self.pacing = Pacing(plan)
        self.step = StepMetrics()

    def take(self, jobs: Channel) -> bool:
        while True:
            j = jobs.try_recv()
            if j is Channel.EMPTY:
                break
            if j is Channel.CLOSED:
                return not self.idle()
            self.job(j)
        if self.idle():
            j = jobs.recv()
            if j is Channel.CLOSED:
                return False
            self.job(j)
        return True

    def job(self, j):
        if isinstance(j, JobRun):
            self.waiting.append(j.request)
        else:
            j.answer.append(self.cache.reset())

    def idle(self):
        return self.lanes.is_empty() and not self.waiting and not self.asked

    def schedule(self):
        self.extend_decodes()
        prompts = self.prefill()
        commands = [End_(lane) for lane in self.lanes.ended()]
        for lane in self.lanes.held():
            commands += self.cache.pages_cmds(lane, self.config.gap)
        commands += prompts
        return self.clock.grant(commands, bool(self.lanes.decoding()))

    def extend_decodes(self):
        for lane in self.lanes.decoding():
            l = self.lanes.get(lane)
            if l is None:
                continue
            rows = l.ahead(self.cache.upto(lane), self.model.context, self.model.block, self.config.ahead)
            if rows is None:
                continue
            if self.cover(lane, rows):
                self.cache.run_to(lane, rows[1])

    def prefill(self):
        seated = self.seat_waiting()
        due = self.pacing.due(len(self.lanes.decoding()))
        chunks = self.chunks(self.lanes.prompting() if due else seated)
        if due and chunks:
            self.pacing.prefilled()
        return chunks

    def seat_waiting(self):
        context, seated = self.model.context, []
        while True:
            lane = self.lanes.free()
            if lane is None or not self.waiting:
                return seated
            r = self.waiting[0]
            n = len(r.prompt)
            if n == 0:
                end = OutEnd("refused", "an empty prompt")
            elif n >= context:
                end = OutEnd("refused", f"a prompt of {n} tokens: the context holds {context}, a token past it")
            elif r.limit == 0:
                end = OutEnd("length")
            else:
                try:
                    cached = self.cache.admit(lane, r.prompt, r.reach(self.pacing.headroom(), context, self.model.block))
                    self.seat(lane, cached)
                    seated.append(lane)
                    continue
                except WaitLater:
                    return seated
                except WaitNever as e:
                    end = OutEnd("refused", f"the cache: {e}")
            r = self.waiting.popleft()
            r.out.send(end)

    def chunks(self, lanes):
        at, rows, pad = self.clock.next(), self.model.chunk, self.model.pad
        allowance = self.pacing.allowance(len(self.lanes.decoding()), self.model.block)
        out = []
        for lane in lanes:
            if not allowance.left():
                break
            l = self.lanes.get(lane)
            if l is None:
                continue
            piece = l.next_chunk(rows, allowance.tokens)
            last = piece[1] == len(l.request.prompt)
            ahead = l.ahead(self.cache.upto(lane), self.model.context, self.model.block, self.config.ahead)
            if not last:
                ahead = None
            if not self.cover(lane, piece) or (ahead is not None and not self.cover(lane, (piece[0], ahead[1]))):
                continue
            if ahead is not None:
                self.cache.run_to(lane, ahead[1])
            l = self.lanes.get(lane)
            out += l.chunk(piece, pad)
            l.sent = piece[1]
            if last:
                l.frm = at
            self.asked.append(Asked(lane, l.seat, last, l.request.sampling.nucleated()))
            self.step.prefill_tokens += piece[1] - piece[0]
            allowance.spend(piece[1] - piece[0])
        return out

    def cover(self, lane, rows):
        while True:
            try:
                self.cache.hold(lane, rows[0], rows[1])
                return True
            except HoldError as e:
                newest = self.lanes.newest()
                if len(self.lanes.held()) == 1:
                    self.end(lane, OutEnd("refused", f"the cache: {e}"))
                    return False
                self.preempt(newest)
                if newest == lane:
                    return False

    def hear(self, e):
        if isinstance(e, Idle):
            self.clock.saw(e.step)
        elif isinstance(e, Step):
            self.clock.saw(e.step)
            self.pacing.stepped()
            for lane, tokens in enumerate(e.lanes):
                self.decoded(lane, e.step, tokens)
        else:
            self.prompted(e.lane, e.token, e.clipped)

    def prompted(self, lane, token, clipped):
        asked = self.asked.popleft()
        assert asked.lane == lane, "a prompt chunk's reply for another lane"
        self.step.top_p_clipped += int(clipped and asked.nucleated)
        l = self.lanes.get(lane)
        if asked.last and l is not None and l.seat == asked.seat:
            self.heard(lane, token)

    def decoded(self, lane, step, tokens):
        l = self.lanes.get(lane)
        if l is None or not l.decodes_at(step):
            return
        if self.model.block > 1 and tokens and all(t.id >= 0 for t in tokens):
            self.step.verified(len(tokens) - 1)
        for t in tokens:
            if not self.heard(lane, t):
                return

    def heard(self, lane, t):
        self.step.generation_tokens += 1
        end = self.lanes.get(lane).hear(t, self.model.context)
        if end is not None:
            self.end(lane, end)
        return end is None

    def seat(self, lane, cached):
        r = self.waiting.popleft()
        self.step.prompt_tokens += len(r.prompt)
        self.step.cached_tokens += cached
        r.out.send(OutSeated(cached))
        self.lanes.seat(lane, r, cached)

    def preempt(self, lane):
        self.step.preemptions += 1
        r = self.free(lane)
        self.waiting.appendleft(r)

    def end(self, lane, why):
        self.free(lane).out.send(why)

    def free(self, lane):
        l = self.lanes.take(lane)
        self.cache.finish(lane, l.request.prompt[: l.written()])
        return l.request

    def step_metrics(self):
        s = self.step
        self.step = StepMetrics()
        s.running = len(self.lanes.held())
        s.waiting = len(self.waiting)
        s.held_pages = self.cache.held()
        s.pages = self.cache.pool()
        s.spec_tokens = self.model.block - 1
        return s

    def refuse(self, why, jobs: Channel):
        for lane in self.lanes.held():
            self.end(lane, OutEnd("refused", why))
        queued = [j.request for j in jobs.drain() if isinstance(j, JobRun)]
        for r in list(self.waiting) + queued:
            r.out.send(OutEnd("refused", why))
        self.waiting.clear()


def run(model: Model, pool: Pool, kernel, jobs: Channel, metrics: Metrics, plan: Plan,
        config: EngineConfig):
    """engine::run: returns None when the job channel closes idle, else the kernel's error."""
    drafts = model.block - 1
    if drafts > config.max_draft_positions:
        return f"{drafts} drafts a step, past the {config.max_draft_positions} the metrics count"
    engine = Engine(model, pool, kernel.pools(), plan, config)
    metrics.record(engine.step_metrics())
    failure = None
    while True:
        if not engine.take(jobs):
            return None
        share = engine.schedule()
        if share is not None:
            err = kernel.push(share)
            if err is not None:
                failure = err
                break
        events, err = kernel.drain()
        if err is not None:
            failure = err
            break
        for e in events:
            engine.hear(e)
        metrics.record(engine.step_metrics())
    engine.refuse(failure, jobs)
    metrics.record(engine.step_metrics())
    return failure


# ------------------------------------------------------------------------------------------
# the reference's test device (tests/engine.rs:56-239)
# ------------------------------------------------------------------------------------------

def next_token(seq) -> int:
    """tests/engine.rs:56-62: FNV-style fold of (token + 1000 * index), mod 400, + 10."""
    h = 1469598103
    for i, t in enumerate(seq):
        h = ((h ^ (t + 1000 * i)) * 1099511628211) & USIZE_MAX
    return h % 400 + 10


class FakeLane:
    def __init__(self, row_len):
        self.row = [0] * row_len
        self.upto = 0
        self.pos = 0
        self.live = False
        self.tok = 0


class Fake:
    """The reference's fake device: applies commands at their step, writes tokens into pages
    through the block-table rows (mirrored into window pages), reads sequences back through
    them and "samples" next_token(seq)."""

    def __init__(self, pages, windows, page_rows, entries, width, context, chunk, drafts=0,
                 clip=False, told=None):
        self.page_rows, self.entries, self.width, self.context, self.chunk = page_rows, entries, width, context, chunk
        self.lanes = [FakeLane(2 * entries) for _ in range(width)]
        self.queue = deque()
        self.s = 0
        self.horizon = -1
        self.applied = False
        self.pages = [[None] * page_rows for _ in range(pages)]
        self.windows = [[None] * page_rows for _ in range(windows)]
        self.events = []
        self.drafts = drafts
        self.clip = clip
        self.told = told

    def pools(self):
        return (len(self.pages), len(self.windows))

    def write(self, l, p, t):
        row = self.lanes[l].row
        page, window = row[p // self.page_rows], row[self.entries + p // self.page_rows]
        assert page != 0, f"lane {l} writes position {p} to the scratch page"
        self.pages[page][p % self.page_rows] = t
        if window != 0:
            self.windows[window][p % self.page_rows] = t

    def token(self, l, last):
        row = self.lanes[l].row
        seq = []
        for p in range(last + 1):
            v = self.pages[row[p // self.page_rows]][p % self.page_rows]
            assert v is not None, f"lane {l} reads position {p} unwritten"
            seq.append(v)
        for q in range(max(last + 1 - self.page_rows, 0), last + 1):
            w = row[self.entries + q // self.page_rows]
            assert w != 0, f"lane {l} reads position {q}'s window from the scratch window page"
            assert self.windows[w][q % self.page_rows] == seq[q], f"lane {l}'s window at {q}"
        return next_token(seq)

    def run(self):
        while True:
            while self.queue:
                at, c = self.queue[0]
                delta = not isinstance(c, Prompt)
                if delta and at > self.s:
                    break
                self.queue.popleft()
                self.applied |= delta
                if isinstance(c, End_):
                    self.lanes[c.lane].live, self.lanes[c.lane].upto = False, 0
                elif isinstance(c, Pages):
                    l = self.lanes[c.lane]
                    l.row[c.from_:c.from_ + len(c.row)] = list(c.row)
                    l.upto = c.upto
                elif isinstance(c, Seat):
                    self.lanes[c.lane].pos = c.pos
                elif isinstance(c, Start):
                    self.lanes[c.lane].live = True
                else:
                    l, pos = c.lane, self.lanes[c.lane].pos
                    assert len(c.tokens) <= self.chunk
                    for j, t in enumerate(c.tokens):
                        w = self.lanes[l].row[self.entries + (pos + j) // self.page_rows]
                        assert w != 0, f"lane {l}'s chunk writes position {pos + j}'s window to the scratch window page"
                        self.write(l, pos + j, t)
                    end = pos + len(c.tokens)
                    tok = self.token(l, end - 1)
                    self.lanes[l].pos, self.lanes[l].tok = end, tok
                    self.events.append(Prompted(c.lane, Sampled(tok), self.clip))
            runnable = [l for l in range(self.width) if self.lanes[l].live and self.lanes[l].pos < self.lanes[l].upto]
            if runnable and self.s <= self.horizon:
                lanes = [[] for _ in range(self.width)]
                for l in runnable:
                    for k in range((self.s + l) % (self.drafts + 1) + 1):
                        pos, tok = self.lanes[l].pos, self.lanes[l].tok
                        if k > 0 and (pos >= self.lanes[l].upto or pos >= self.context - 1):
                            break
                        assert pos < self.context - 1, f"lane {l} decodes at the idle position"
                        self.write(l, pos, tok)
                        t = self.token(l, pos)
                        self.lanes[l].pos, self.lanes[l].tok = pos + 1, t
                        lanes[l].append(Sampled(t))
                self.events.append(Step(self.s, lanes))
                self.s += 1
                continue
            if not runnable and self.applied:
                self.events.append(Idle(self.s))
                self.applied = False
            if self.queue:
                at, c = self.queue[0]
                if (not runnable and not isinstance(c, Prompt) and at > self.s and at <= self.horizon + 1):
                    self.s = at
                    continue
            return

    def push(self, share: Share):
        assert share.at == self.horizon + 1, f"a share at {share.at} past a horizon of {self.horizon}"
        assert share.horizon >= share.at
        self.queue.extend((share.at, c) for c in share.commands)
        self.horizon = share.horizon
        if self.told is not None:
            self.told.append(share)
        return None

    def drain(self):
        self.run()
        ev, self.events = self.events, []
        return ev, None


def expected(prompt, limit, stop, context):
    """tests/engine.rs:252-268: the token stream and end reason a request must get."""
    if len(prompt) >= context:
        return [], "refused"
    seq, out = list(prompt), []
    while True:
        if len(out) == limit or len(seq) == context:
            return out, "length"
        t = next_token(seq)
        out.append(t)
        if t in stop:
            return out, "stop"
        seq.append(t)


def heard(sink: Sink):
    """tests/engine.rs:270-281: tokens and the end kind a request's listener saw."""
    tokens = []
    for o in sink.items:
        if isinstance(o, OutToken):
            tokens.append(o.id)
        elif isinstance(o, OutEnd):
            return tokens, o.kind
    raise AssertionError("no end")
