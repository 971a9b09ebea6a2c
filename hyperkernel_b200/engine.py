"""ctypes binding of the Kernel boundary and the engine (include/hk.h, hk_open ... hk_engine_*).

Names follow the reference's interfaces:
  - `Device` is a `Kernel` (src/gpu/mod.rs:42-46): pools() / push(share) / drain(), backed by
    libhk's device kernel (hk_open);
  - `CallbackKernel` turns any Python object with those three methods, working on the raw
    hk_share / hk_event structures, into hk_kernel_ops;
  - `Engine` is engine::run with its job channel (src/engine/mod.rs:38-74): submit() is
    Job::Run, reset() is Job::Reset, close() drops the sender, run() runs the loop.
Everything runs in libhk.so; this module only marshals.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

from . import _lib

U32, U64, I32, I64, SZ, F32 = C.c_uint32, C.c_uint64, C.c_int32, C.c_int64, C.c_size_t, C.c_float

CMD_END, CMD_PAGES, CMD_SEAT, CMD_PROMPT, CMD_START = 0, 1, 2, 3, 4
EV_IDLE, EV_STEP, EV_PROMPTED = 0, 1, 2
OUT_SEATED, OUT_TOKEN, OUT_END = 0, 1, 2
END_STOP, END_LENGTH, END_REFUSED = 0, 1, 2
END_NAMES = {END_STOP: "stop", END_LENGTH: "length", END_REFUSED: "refused"}
MODEL_FNV, MODEL_MLA = 1, 2
UNBOUNDED = (1 << 64) - 1


class Sampling(C.Structure):
    _fields_ = [("temperature", F32), ("top_p", F32), ("top_k", U32), ("logprobs", U32), ("seed", U64)]


class Command(C.Structure):
    _fields_ = [("kind", U32), ("lane", U32), ("pos", U32), ("upto", U32), ("count", U32),
                ("arena", U32), ("back", I32 * 3), ("reserved", U32), ("sampling", Sampling)]


class Share(C.Structure):
    _fields_ = [("at", U32), ("horizon", U32), ("commands", C.POINTER(Command)), ("n_commands", SZ),
                ("arena", C.POINTER(I32)), ("arena_words", SZ)]


class Event(C.Structure):
    _fields_ = [("kind", U32), ("step", U32), ("lane", U32), ("token", I32), ("clipped", I32),
                ("ids", U32)]


class Config(C.Structure):
    """hk_config: the device kernel's pool and model shape."""
    _fields_ = [("model", U32), ("page_rows", U32), ("entries", U32), ("window", U32),
                ("width", U32), ("context", U32), ("chunk", U32), ("block", U32),
                ("pages", U64), ("window_pages", U64), ("clip", I32), ("device", I32),
                ("transport", U32), ("reserved", U32)]


class MlaModel(C.Structure):
    """hk_mla_model: the dimensions and weight seed of the HK_MODEL_MLA decoder."""
    _fields_ = [("hidden", U32), ("q_lora", U32), ("vocab", U32), ("experts", U32), ("top_k", U32),
                ("inter", U32), ("layers", U32), ("logprobs", U32), ("seed", U64), ("rope_theta", F32),
                ("route_scale", F32)]


class EngineConfig(C.Structure):
    """hk_engine_config: Pool + Model fields, Plan and EngineConfig."""
    _fields_ = [("page_rows", U32), ("entries", U32), ("window", U32), ("window_keep", U32),
                ("context", U32), ("width", U32), ("chunk", U32), ("block", U32), ("pad", I32),
                ("lead", U32), ("budget", U64), ("every", U64), ("headroom", U64), ("gap", U64),
                ("ahead", U64), ("max_draft_positions", U64)]


class Out(C.Structure):
    _fields_ = [("kind", U32), ("end", U32), ("value", I64)]


class StepMetrics(C.Structure):
    _fields_ = [(n, U64) for n in ("running", "waiting", "held_pages", "pages", "spec_tokens",
                                   "prompt_tokens", "cached_tokens", "prefill_tokens",
                                   "generation_tokens", "preemptions", "top_p_clipped", "drafts")]


PoolsFn = C.CFUNCTYPE(C.c_int, C.c_void_p, C.POINTER(SZ), C.POINTER(SZ))
PushFn = C.CFUNCTYPE(C.c_int, C.c_void_p, C.POINTER(Share))
DrainFn = C.CFUNCTYPE(C.c_int, C.c_void_p, C.POINTER(Event), SZ, C.POINTER(SZ), C.POINTER(I32), SZ,
                      C.POINTER(SZ))
ErrorFn = C.CFUNCTYPE(C.c_void_p, C.c_void_p)


class Logprob(C.Structure):
    """hk_logprob: one (token id, logprob) pair of a Sampled's logprob list."""
    _fields_ = [("id", U32), ("logprob", F32)]


LogprobsFn = C.CFUNCTYPE(C.c_int, C.c_void_p, C.POINTER(U32), SZ, C.POINTER(SZ), C.POINTER(Logprob), SZ,
                         C.POINTER(SZ))


class KernelOps(C.Structure):
    _fields_ = [("self", C.c_void_p), ("pools", PoolsFn), ("push", PushFn), ("drain", DrainFn),
                ("error", ErrorFn), ("logprobs", LogprobsFn)]


def engine_config(**fields) -> EngineConfig:
    """hk_engine_defaults, then the given fields (budget=None means unbounded)."""
    c = EngineConfig()
    _lib.lib().hk_engine_defaults(C.byref(c))
    for k, v in fields.items():
        if k == "budget" and v is None:
            v = UNBOUNDED
        setattr(c, k, v)
    return c


def make_share(at: int, horizon: int, commands):
    """Builds an hk_share from (kind, lane, pos, upto, data, back, sampling) tuples; returns the
    structure and the arrays it points into (keep them alive while the share is used)."""
    n = len(commands)
    cmds = (Command * max(n, 1))()
    arena = []
    for i, (kind, lane, pos, upto, data, back, sampling) in enumerate(commands):
        c = cmds[i]
        c.kind, c.lane, c.pos, c.upto = kind, lane, pos, upto
        c.count, c.arena = len(data), len(arena)
        arena.extend(int(x) if int(x) < (1 << 31) else int(x) - (1 << 32) for x in data)
        for j in range(3):
            c.back[j] = back[j]
        if sampling is not None:
            c.sampling = sampling
    arr = (I32 * max(len(arena), 1))(*arena)
    share = Share(at, horizon, cmds, n, arr, len(arena))
    return share, (cmds, arr)


def read_share(s: Share):
    """hk_share -> (at, horizon, [(kind, lane, pos, upto, data, back, sampling tuple)])."""
    cmds = []
    for i in range(s.n_commands):
        c = s.commands[i]
        data = [s.arena[c.arena + j] for j in range(c.count)]
        if c.kind == CMD_PROMPT:
            data = [x & 0xFFFFFFFF for x in data]
        sp = c.sampling
        cmds.append((c.kind, c.lane, c.pos, c.upto, data, tuple(c.back),
                     (sp.temperature, sp.top_p, sp.top_k, sp.logprobs, sp.seed)))
    return s.at, s.horizon, cmds


def encode_share(config: Config, share: Share) -> bytes:
    """hk_encode_share: the request-ring bytes hk_push sends for this share."""
    need = SZ()
    L = _lib.lib()
    rc = L.hk_encode_share(C.byref(config), C.byref(share), None, 0, C.byref(need))
    if rc == _lib.HK_OK and need.value == 0:
        return b""
    if rc != _lib.HK_OK and need.value == 0:
        _lib.check(rc)
    buf = (C.c_uint8 * need.value)()
    _lib.check(L.hk_encode_share(C.byref(config), C.byref(share), buf, need.value, C.byref(need)))
    return bytes(buf[:need.value])


class Device:
    """A device kernel (hk_open, or hk_open_mla when `model` is given): the Kernel the engine
    drives on a GPU."""

    def __init__(self, config: Config, model: MlaModel | None = None):
        self.config = config
        self.model = model
        self._h = C.c_void_p()
        if model is None:
            _lib.check(_lib.lib().hk_open(C.byref(config), C.byref(self._h)))
        else:
            _lib.check(_lib.lib().hk_open_mla(C.byref(config), C.byref(model), C.byref(self._h)))

    def tensor(self, name: str, layer: int = 0):
        """(device address, bytes) of one of an HK_MODEL_MLA handle's tensors (hk_model_tensor)."""
        p, n = C.c_void_p(), SZ()
        _lib.check(_lib.lib().hk_model_tensor(self._h, layer, name.encode(), C.byref(p), C.byref(n)))
        return p.value, n.value

    def logprob_lists(self):
        """The logprob lists of the last drain's Sampled values (hk_drain_logprobs)."""
        n, m = SZ(), SZ()
        L = _lib.lib()
        rc = L.hk_drain_logprobs(self._h, None, 0, C.byref(n), None, 0, C.byref(m))
        if rc not in (_lib.HK_OK, _lib.HK_ESPACE):
            _lib.check(rc)
        counts = (U32 * max(n.value, 1))()
        pairs = (Logprob * max(m.value, 1))()
        _lib.check(L.hk_drain_logprobs(self._h, counts, n.value, C.byref(n), pairs, m.value, C.byref(m)))
        out, k = [], 0
        for i in range(n.value):
            out.append([(pairs[k + j].id, pairs[k + j].logprob) for j in range(counts[i])])
            k += counts[i]
        return out

    def close(self):
        if self._h:
            _lib.lib().hk_close(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self):
        return self._h

    def ops(self) -> KernelOps:
        ops = KernelOps()
        _lib.check(_lib.lib().hk_kernel_ops_of(self._h, C.byref(ops)))
        return ops

    def pools(self):
        p, w = SZ(), SZ()
        _lib.check(_lib.lib().hk_pools(self._h, C.byref(p), C.byref(w)))
        return p.value, w.value

    def push_raw(self, share: Share) -> int:
        return _lib.lib().hk_push(self._h, C.byref(share))

    def drain_raw(self, events, cap, n, ids, ids_cap, ids_n) -> int:
        return _lib.lib().hk_drain(self._h, events, cap, n, ids, ids_cap, ids_n)


class CallbackKernel:
    """hk_kernel_ops over a Python object with pools() -> (pages, windows), push(Share) -> None
    and drain() -> (events, ids) where events are (kind, step, lane, token, clipped, ids_offset)
    tuples, and optionally logprobs() -> the last drain's logprob lists, one list of
    (id, logprob) pairs per Sampled slot in event order (hk_drain_logprobs's layout).
    Exceptions become HK_ESTATE with their message."""

    def __init__(self, impl):
        self.impl = impl
        self._msg = C.create_string_buffer(512)
        self._pending = None
        self._pending_lp = None
        lp = LogprobsFn(self._logprobs) if hasattr(impl, "logprobs") else LogprobsFn()
        self._fns = (PoolsFn(self._pools), PushFn(self._push), DrainFn(self._drain),
                     ErrorFn(self._error), lp)

    def ops(self) -> KernelOps:
        return KernelOps(None, *self._fns)

    def _logprobs(self, _self, counts, counts_cap, n_counts, pairs, pairs_cap, n_pairs):
        try:
            if self._pending_lp is None:
                self._pending_lp = self.impl.logprobs()
            lists = self._pending_lp
            total = sum(len(x) for x in lists)
            n_counts[0], n_pairs[0] = len(lists), total
            if len(lists) > counts_cap or total > pairs_cap:
                return _lib.HK_ESPACE
            k = 0
            for i, lst in enumerate(lists):
                counts[i] = len(lst)
                for tid, lp in lst:
                    pairs[k].id, pairs[k].logprob = tid, lp
                    k += 1
            self._pending_lp = None
            return 0
        except Exception as e:  # noqa: BLE001
            self._pending_lp = None
            return self._fail(e)

    def _fail(self, e) -> int:
        self._msg.value = str(e).encode()[:511]
        return getattr(e, "code", _lib.HK_ESTATE)

    def _pools(self, _self, pages, windows):
        try:
            p, w = self.impl.pools()
            pages[0], windows[0] = p, w
            return 0
        except Exception as e:  # noqa: BLE001 - reported through the boundary
            return self._fail(e)

    def _push(self, _self, share):
        try:
            self.impl.push(share.contents)
            return 0
        except Exception as e:  # noqa: BLE001
            return self._fail(e)

    def _drain(self, _self, events, cap, n, ids, ids_cap, ids_n):
        try:
            if self._pending is None:
                self._pending = self.impl.drain()
            evs, flat = self._pending
            n[0], ids_n[0] = len(evs), len(flat)
            if len(evs) > cap or len(flat) > ids_cap:
                return _lib.HK_ESPACE
            for i, (kind, step, lane, token, clipped, off) in enumerate(evs):
                e = events[i]
                e.kind, e.step, e.lane, e.token, e.clipped, e.ids = kind, step, lane, token, clipped, off
            for i, x in enumerate(flat):
                ids[i] = x
            self._pending = None
            return 0
        except Exception as e:  # noqa: BLE001
            self._pending = None
            return self._fail(e)

    def _error(self, _self):
        return C.addressof(self._msg)


@dataclass
class Heard:
    seated: list
    tokens: list
    end: str | None
    message: str
    logprobs: list | None = None  # per token, its (id, logprob) pairs


class Engine:
    """engine::run over a kernel (hk_kernel_ops)."""

    def __init__(self, config: EngineConfig, ops: KernelOps, keep=None):
        self.config = config
        self._ops = ops
        self._keep = keep  # keeps the kernel's callbacks alive
        self._e = C.c_void_p()
        _lib.check(_lib.lib().hk_engine_create(C.byref(config), C.byref(ops), C.byref(self._e)))
        self.failure = None

    def __del__(self):
        if getattr(self, "_e", None):
            _lib.lib().hk_engine_destroy(self._e)
            self._e = C.c_void_p()

    def submit(self, prompt, limit, stop=(), sampling: Sampling | None = None) -> int:
        p = (U32 * max(len(prompt), 1))(*prompt)
        s = (U32 * max(len(stop), 1))(*stop)
        req = U64()
        _lib.check(_lib.lib().hk_engine_submit(self._e, p, len(prompt),
                                               C.byref(sampling or Sampling(0.0, 1.0, 0, 0, 0)),
                                               min(limit, UNBOUNDED), s, len(stop), C.byref(req)))
        return req.value

    def reset(self) -> int:
        t = U64()
        _lib.check(_lib.lib().hk_engine_reset(self._e, C.byref(t)))
        return t.value

    def reset_answer(self, ticket: int, timeout_ms: int = -1) -> int:
        f = U64()
        _lib.check(_lib.lib().hk_engine_reset_answer(self._e, ticket, timeout_ms, C.byref(f)))
        return f.value

    def close(self):
        _lib.check(_lib.lib().hk_engine_close(self._e))

    def run(self) -> int:
        """Runs until the jobs close and every request ended; returns 0 or the kernel's error
        code (message in self.failure)."""
        rc = _lib.lib().hk_engine_run(self._e)
        if rc != _lib.HK_OK:
            self.failure = _lib.last_error()
        return rc

    def hangup(self, request: int):
        _lib.check(_lib.lib().hk_engine_hangup(self._e, request))

    def outputs(self, request: int, timeout_ms: int = 0):
        """[(kind, end, value, message, logprobs)] of the request's outputs so far; a token's
        logprobs are its (id, logprob) pairs (empty unless its Sampling asked for logprobs)."""
        buf = (Out * 256)()
        msg = C.create_string_buffer(512)
        cap = 256 * 66
        pairs = (Logprob * cap)()
        out = []
        while True:
            n, npairs = SZ(), SZ()
            rc = _lib.lib().hk_engine_outputs_lp(self._e, request, timeout_ms, buf, 256, C.byref(n), msg, 512,
                                                 pairs, cap, C.byref(npairs))
            if rc == _lib.HK_ESPACE:  # one token's pairs past the buffer
                cap = npairs.value
                pairs = (Logprob * cap)()
                continue
            _lib.check(rc)
            k = 0
            for i in range(n.value):
                o = buf[i]
                lps = []
                if o.kind == OUT_TOKEN:
                    lps = [(pairs[k + j].id, pairs[k + j].logprob) for j in range(o.end)]
                    k += o.end
                out.append((o.kind, o.end, o.value, msg.value.decode() if o.kind == OUT_END else "", lps))
            if n.value == 0:
                return out
            timeout_ms = 0  # then take what else is queued, without waiting

    def heard(self, request: int, timeout_ms: int = 0) -> Heard:
        """The tokens and the end the request's listener saw (tests/engine.rs:270-281)."""
        h = Heard([], [], None, "", [])
        for kind, end, value, message, lps in self.outputs(request, timeout_ms):
            if kind == OUT_SEATED:
                h.seated.append(value)
            elif kind == OUT_TOKEN:
                h.tokens.append(value)
                h.logprobs.append(lps)
            elif h.end is None:
                h.end, h.message = END_NAMES[end], message
        return h

    def metrics(self):
        """(StepMetrics totals as a dict, accepted_per_pos, iteration_tokens counts, sum)."""
        t = StepMetrics()
        pos = (U64 * 64)()
        npos = SZ()
        counts = (U64 * 14)()
        total = C.c_double()
        _lib.check(_lib.lib().hk_engine_metrics(self._e, C.byref(t), pos, 64, C.byref(npos), counts, 14,
                                                C.byref(total)))
        m = {name: getattr(t, name) for name, _ in StepMetrics._fields_}
        return m, list(pos[:npos.value]), list(counts), total.value
