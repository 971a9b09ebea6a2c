"""Restatement of the reference's request-ring encoding — TEST INFRASTRUCTURE ONLY.

encode / decode follow src/gpu/ring.rs:99-144 (fields written at their offsets by kind: one
int or float, an array of ints of the layout's length, a span {u64 address, u64 elements}
whose element count is the layout's when it has one); slots follow Ring::push
(src/gpu/ring.rs:46-66: u32 id at byte 0, body at byte 16, slot = 16 + widest body rounded up
to 16).  The per-command field values follow Feed::command (src/gpu/feed.rs:40-103).
Pinned by the reference's own known-answer test of the encoder (src/gpu/ring.rs:150-183),
restated in tests/test_engine_cpu.py.

MESSAGES is this build's message table (the reference reads its table from a bundle manifest
that is not in the repository; the byte sizes per message are the manifest's: end 8, pages 32,
seat 52, prompt 40, start 56).  It is the specification hk_encode_share is checked against.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass


@dataclass
class Field:
    name: str
    at: int
    kind: str   # "one" | "array" | "span"
    dtype: str  # "i32" | "u32" | "f32" | "u64"
    n: int


@dataclass
class Message:
    name: str
    id: int
    ring: int
    bytes: int
    fields: list


@dataclass
class Int:
    x: int


@dataclass
class Float:
    x: float


@dataclass
class Ints:
    xs: list


@dataclass
class Span:
    addr: int
    elements: int


_SIZE = {"i32": 4, "u32": 4, "f32": 4, "u64": 8}


def _int(dtype, x):
    if dtype == "i32":
        return struct.pack("<i", ((x + (1 << 31)) % (1 << 32)) - (1 << 31))
    if dtype == "u32":
        return struct.pack("<I", x % (1 << 32))
    if dtype == "u64":
        return struct.pack("<Q", x % (1 << 64))
    raise ValueError(f"{x} written as {dtype}")


def _field(m: Message, name: str) -> Field:
    for f in m.fields:
        if f.name == name:
            return f
    raise KeyError(f"{m.name} has no field {name}")


def encode(layout: Message, fields) -> bytes:
    out = bytearray(layout.bytes)
    for name, v in fields:
        f = _field(layout, name)
        at, e = f.at, _SIZE[f.dtype]
        if f.kind == "one" and isinstance(v, Int):
            out[at:at + e] = _int(f.dtype, v.x)
        elif f.kind == "one" and isinstance(v, Float) and f.dtype == "f32":
            out[at:at + 4] = struct.pack("<f", v.x)
        elif f.kind == "array" and isinstance(v, Ints) and len(v.xs) == f.n:
            for i, x in enumerate(v.xs):
                out[at + i * e:at + (i + 1) * e] = _int(f.dtype, x)
        elif f.kind == "span" and isinstance(v, Span):
            elements = f.n if f.n > 0 else v.elements
            out[at:at + 16] = struct.pack("<QQ", v.addr, elements)
        else:
            raise ValueError(f"{layout.name}.{name} ({f.kind} of {f.n} {f.dtype}) written as {v}")
    return bytes(out)


def decode(layout: Message, data: bytes, name: str):
    f = _field(layout, name)
    n = 1 if f.kind == "one" else f.n
    return list(struct.unpack(f"<{n}i", data[f.at:f.at + 4 * n]))


def _m(name, id_, size, *fields):
    return Message(name, id_, 0, size, [Field(*f) for f in fields])


MESSAGES = {
    "end": _m("end", 0x101, 8, ("at", 0, "one", "u32", 0), ("lane", 4, "one", "u32", 0)),
    "pages": _m("pages", 0x102, 32, ("at", 0, "one", "u32", 0), ("lane", 4, "one", "u32", 0),
                ("from", 8, "one", "u32", 0), ("upto", 12, "one", "u32", 0),
                ("row", 16, "span", "i32", 0)),
    "seat": _m("seat", 0x103, 52, ("at", 0, "one", "u32", 0), ("lane", 4, "one", "u32", 0),
               ("pos", 8, "one", "u32", 0), ("back", 12, "array", "i32", 3),
               ("slot", 24, "one", "u32", 0), ("temp", 28, "one", "f32", 0),
               ("seed_lo", 32, "one", "u32", 0), ("seed_hi", 36, "one", "u32", 0),
               ("top_p", 40, "one", "f32", 0), ("top_k", 44, "one", "u32", 0),
               ("logprobs", 48, "one", "u32", 0)),
    "prompt": _m("prompt", 0x104, 40, ("lane", 0, "one", "u32", 0), ("lens", 4, "one", "u32", 0),
                 ("tokens", 8, "span", "u32", 0), ("lps", 24, "span", "f32", 0)),
    "start": _m("start", 0x105, 56, ("at", 0, "one", "u32", 0), ("lane", 4, "one", "u32", 0),
                ("noise", 8, "one", "u32", 0), ("idle", 12, "one", "u32", 0),
                ("scratch", 16, "one", "u32", 0), ("lps", 24, "span", "f32", 0),
                ("commits", 40, "span", "i32", 0)),
}

BODY_AT = 16
SLOT = (BODY_AT + max(m.bytes for m in MESSAGES.values()) + 15) // 16 * 16


def _r16(x):
    return (x + 15) // 16 * 16


def encode_share(chunk: int, context: int, at: int, commands) -> bytes:
    """The request stream of one share: a slot per command, then the side blocks (Pages rows;
    Prompt tokens padded to `chunk` words) at the byte offsets the spans carry.  `commands`
    are (kind, lane, pos, upto, data, back, sampling) with kind 0..4 = end, pages, seat,
    prompt, start and sampling an object with temperature / top_p / top_k / logprobs / seed."""
    slots = bytearray(SLOT * len(commands))
    side = bytearray()
    base = len(slots)
    for i, (kind, lane, pos, upto, data, back, s) in enumerate(commands):
        if kind == 0:
            m, f = MESSAGES["end"], [("at", Int(at)), ("lane", Int(lane))]
        elif kind == 1:
            m = MESSAGES["pages"]
            f = [("at", Int(at)), ("lane", Int(lane)), ("from", Int(pos)), ("upto", Int(upto)),
                 ("row", Span(base + len(side), len(data)))]
            blk = b"".join(_int("i32", x) for x in data)
            side += blk + bytes(_r16(len(blk)) - len(blk))
        elif kind == 2:
            m = MESSAGES["seat"]
            f = [("at", Int(at)), ("lane", Int(lane)), ("pos", Int(pos)), ("back", Ints(list(back))),
                 ("slot", Int(lane + 1)), ("temp", Float(s.temperature)),
                 ("seed_lo", Int(s.seed & 0xFFFFFFFF)), ("seed_hi", Int(s.seed >> 32)),
                 ("top_p", Float(s.top_p)), ("top_k", Int(s.top_k)), ("logprobs", Int(s.logprobs))]
        elif kind == 3:
            m = MESSAGES["prompt"]
            f = [("lane", Int(lane)), ("lens", Int(len(data))), ("tokens", Span(base + len(side), chunk)),
                 ("lps", Span(0, 0))]
            blk = b"".join(_int("u32", x) for x in data) + bytes(4 * (chunk - len(data)))
            side += blk + bytes(_r16(len(blk)) - len(blk))
        else:
            m = MESSAGES["start"]
            f = [("at", Int(at)), ("lane", Int(lane)), ("noise", Int(0)), ("idle", Int(context - 1)),
                 ("scratch", Int(0)), ("lps", Span(0, 0)), ("commits", Span(0, 0))]
        body = encode(m, f)
        slots[i * SLOT:i * SLOT + 4] = struct.pack("<I", m.id)
        slots[i * SLOT + BODY_AT:i * SLOT + BODY_AT + len(body)] = body
    return bytes(slots + side)
