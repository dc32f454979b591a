"""Reading a printed module of several GB in seconds (test infrastructure).

The pass driver prints large constants as `dense<"0x…">` hex literals.  A
full-size configuration's output holds 0.5-5.4 GB of them, far too much for
the line-by-line reader in golden/mlir_text.py.  `scan` cuts every hex body
out of the text (bytes.find jumps from literal to literal), reads the small
remaining skeleton with that reader, and decodes a literal's bytes only
when a test asks for them.
"""
from __future__ import annotations

import binascii
import hashlib
import re
from dataclasses import dataclass

import numpy as np

from mlir_text import parse_funcs, parse_type

OPEN = b'dense<"0x'
_PLACE = re.compile(r'dense<"@(\d+)">')


@dataclass
class Module:
    text: bytes
    spans: list            # (start, end) of each hex body, in text order
    funcs: dict            # name -> mlir_text.Func of the skeleton

    def literal_index(self, op) -> int | None:
        m = _PLACE.search(op.line)
        return int(m.group(1)) if m else None

    def raw(self, op) -> bytes:
        """The raw bytes of a constant op printed as a hex literal."""
        k = self.literal_index(op)
        assert k is not None, op.line
        a, b = self.spans[k]
        return binascii.unhexlify(self.text[a:b])

    def values(self, op, storage) -> np.ndarray:
        """All element bits of a constant op (hex literal, or a splat
        expanded to the type's element count) as `storage` integers."""
        if self.literal_index(op) is not None:
            return np.frombuffer(self.raw(op), dtype=storage)
        ty = parse_type(op.out_types[0])
        assert op.const is not None and op.const.splat, op.line
        return np.full(ty.count, op.const.bits[0], dtype=storage)

    def returned(self, name: str):
        f = self.funcs[name]
        return [f.defs.get(v) for v in f.ret.operands]


def scan(text) -> Module:
    """Parse a printed module, leaving its hex literal bodies in place."""
    if not isinstance(text, bytes):
        text = bytes(text)
    spans, pieces, pos = [], [], 0
    while True:
        i = text.find(OPEN, pos)
        if i < 0:
            pieces.append(text[pos:])
            break
        a = i + len(OPEN)
        b = text.find(b'"', a)
        assert b > 0, "unterminated hex literal"
        pieces.append(text[pos:i])
        pieces.append(b'dense<"@%d"' % len(spans))
        spans.append((a, b))
        pos = b + 1
    skeleton = b"".join(pieces).decode()
    return Module(text, spans, parse_funcs(skeleton))


def entry_const(hex_upper: bytes) -> str:
    return "const " + hashlib.sha256(hex_upper).hexdigest()


def entry_op(name: str) -> str:
    return "op " + name


def combine(entries) -> str:
    """One digest of a module's returned values: for each function in
    order, for each returned value, `const <sha256 of its hex body>` or
    `op <name>` (a value left unfolded)."""
    h = hashlib.sha256()
    for e in entries:
        h.update(e.encode() + b"\n")
    return h.hexdigest()


def returns_digest(m: Module) -> str:
    entries = []
    for name, f in m.funcs.items():
        for v in f.ret.operands:
            d = f.defs.get(v)
            k = m.literal_index(d) if d is not None else None
            if d is not None and d.name in ("arith.constant", "tosa.const") and k is not None:
                a, b = m.spans[k]
                entries.append(f"{name} " + entry_const(m.text[a:b]))
            else:
                entries.append(f"{name} " + entry_op(d.name if d is not None else "?"))
    return combine(entries)
