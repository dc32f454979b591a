"""Minimal reader for MLIR generic-form text, as the reference's fixtures
print it (tests/fixtures/*.in.mlir / *.generic.mlir in mlirpass).

Test infrastructure: used by make_golden.py to turn fixture functions into
golden vectors, and by the tests to decode those vectors.  It understands
only what the fold fixtures need: one op per line, `dense<...>` literals,
float / int scalar literals, and the builtin integer and IEEE float types.
"""
from __future__ import annotations

import re
from dataclasses import dataclass, field
from fractions import Fraction

# name -> (exponent bits, mantissa bits, storage bytes)
FLOATS = {
    "f16": (5, 10, 2),
    "bf16": (8, 7, 2),
    "f32": (8, 23, 4),
    "f64": (11, 52, 8),
    "f8E5M2": (5, 2, 1),
    "f8E4M3": (4, 3, 1),
    "f8E3M4": (3, 4, 1),
}
INTS = {"i1": 1, "i8": 8, "i16": 16, "i32": 32, "i64": 64, "index": 64}


def elem_bytes(dt: str) -> int:
    if dt in FLOATS:
        return FLOATS[dt][2]
    w = INTS[dt]
    return 1 if w == 1 else w // 8


def round_fraction(q: Fraction, neg_zero: bool, E: int, M: int) -> int:
    """Exact rational -> IEEE-like bits, round to nearest, ties to even."""
    sign = 1 if (q < 0 or (q == 0 and neg_zero)) else 0
    q = abs(q)
    sbit = sign << (E + M)
    if q == 0:
        return sbit
    bias = (1 << (E - 1)) - 1
    emin = 1 - bias
    e = q.numerator.bit_length() - q.denominator.bit_length()
    while Fraction(2) ** e > q:
        e -= 1
    while Fraction(2) ** (e + 1) <= q:
        e += 1
    qe = emin - M if e < emin else e - M
    scaled = q / (Fraction(2) ** qe)
    r = scaled.numerator // scaled.denominator
    rem = scaled - r
    if rem > Fraction(1, 2) or (rem == Fraction(1, 2) and (r & 1)):
        r += 1
    bits = r if e < emin else ((e + bias - 1) << M) + r
    if (bits >> M) >= (1 << E) - 1:
        bits = ((1 << E) - 1) << M
    return sbit | bits


def float_literal_bits(tok: str, dt: str) -> int:
    E, M, _ = FLOATS[dt]
    tok = tok.strip()
    if tok.lower().startswith("0x"):
        return int(tok, 16)
    if tok in ("inf", "+inf"):
        return ((1 << E) - 1) << M
    if tok == "-inf":
        return (1 << (E + M)) | (((1 << E) - 1) << M)
    q = Fraction(tok)
    return round_fraction(q, tok.startswith("-"), E, M)


def int_literal_bits(tok: str, dt: str) -> int:
    w = INTS[dt]
    tok = tok.strip()
    if tok == "true":
        return 1
    if tok == "false":
        return 0
    v = int(tok, 0)
    return v & ((1 << w) - 1)


def literal_bits(tok: str, dt: str) -> int:
    return float_literal_bits(tok, dt) if dt in FLOATS else int_literal_bits(tok, dt)


@dataclass
class Ty:
    elem: str                    # element type name
    shape: list[int] | None      # None for a scalar
    kind: str = "scalar"         # scalar | vector | tensor

    @property
    def count(self) -> int:
        n = 1
        for d in self.shape or []:
            n *= d
        return n


_SHAPED = re.compile(r"^(vector|tensor)<(.*)>$")


def parse_type(s: str) -> Ty | None:
    s = s.strip()
    if s in FLOATS or s in INTS:
        return Ty(s, None)
    m = _SHAPED.match(s)
    if not m:
        return None
    kind, body = m.groups()
    # leading "NxMx..." dims, then the element type (which may contain an
    # "x" itself, as index does)
    dm = re.match(r"^((?:\d+x)*)(.+)$", body)
    elem = dm.group(2)
    if elem not in FLOATS and elem not in INTS:
        return None            # dynamic or scalable dims, or another element type
    dims = [int(p) for p in dm.group(1).split("x") if p]
    return Ty(elem, dims, kind)


def split_top(s: str, sep: str = ",") -> list[str]:
    out, depth, cur = [], 0, []
    for ch in s:
        if ch in "[(<{":
            depth += 1
        elif ch in "])>}":
            depth -= 1
        if ch == sep and depth == 0:
            out.append("".join(cur))
            cur = []
        else:
            cur.append(ch)
    if cur:
        out.append("".join(cur))
    return [x.strip() for x in out if x.strip()]


def flatten_list(s: str) -> list[str]:
    s = s.strip()
    if s.startswith("["):
        inner = s[1:-1]
        out = []
        for part in split_top(inner):
            out.extend(flatten_list(part))
        return out
    return [s]


@dataclass
class ConstVal:
    ty: Ty
    splat: bool
    bits: list[int]              # one entry if splat
    elements: bool               # dense (shaped) vs scalar attribute


def parse_const(lit: str, ty: Ty) -> ConstVal | None:
    lit = lit.strip()
    if lit.startswith("dense<") and lit.endswith(">"):
        if ty.shape is None:
            return None
        body = lit[len("dense<"):-1].strip()
        if body.startswith('"0x'):
            raw = bytes.fromhex(body[3:-1])
            eb = elem_bytes(ty.elem)
            if ty.elem == "i1":
                return None      # bit-packed in MLIR's raw form
            vals = [int.from_bytes(raw[i:i + eb], "little") for i in range(0, len(raw), eb)]
            if len(vals) == 1:
                return ConstVal(ty, True, vals, True)
            if len(vals) != ty.count:
                return None
            return ConstVal(ty, False, vals, True)
        if body.startswith("("):
            return None          # complex
        toks = flatten_list(body)
        try:
            vals = [literal_bits(t, ty.elem) for t in toks]
        except (ValueError, ZeroDivisionError):
            return None
        if not body.startswith("["):
            return ConstVal(ty, True, vals, True)
        if len(vals) != ty.count:
            return None
        return ConstVal(ty, False, vals, True)
    if ty.shape is not None:
        return None
    try:
        return ConstVal(ty, True, [literal_bits(lit, ty.elem)], False)
    except (ValueError, ZeroDivisionError):
        return None


_OP = re.compile(r'^\s*(?:(%[\w.$-]+(?::\d+)?)\s*=\s*)?"([\w.]+)"\((.*?)\)\s*(.*)$')


@dataclass
class Op:
    result: str | None
    name: str
    operands: list[str]
    props: str
    in_types: list[str]
    out_types: list[str]
    line: str
    const: ConstVal | None = None
    prop_map: dict = field(default_factory=dict)
    nres: int = 1                  # results (an op printed as %name:N has N)


def _split_sig(rest: str):
    # rest: [<{props}>] [{attrs}] : (in) -> out
    props = ""
    if rest.startswith("<{"):
        depth, i = 0, 0
        while i < len(rest):
            if rest[i] == "<" and rest[i:i + 2] == "<{":
                depth += 1
                i += 2
                continue
            if rest[i:i + 2] == "}>":
                depth -= 1
                i += 2
                if depth == 0:
                    break
                continue
            i += 1
        props = rest[2:i - 2]
        rest = rest[i:].strip()
    if rest.startswith("{"):
        depth = 0
        for i, ch in enumerate(rest):
            if ch == "{":
                depth += 1
            elif ch == "}":
                depth -= 1
                if depth == 0:
                    rest = rest[i + 1:].strip()
                    break
    if not rest.startswith(":"):
        return props, None, None
    sig = rest[1:].strip()
    if "->" not in sig:
        return props, None, None
    ins, outs = sig.split("->", 1)
    ins = ins.strip()
    if ins.startswith("(") and ins.endswith(")"):
        ins = ins[1:-1]
    outs = outs.strip()
    if outs.startswith("(") and outs.endswith(")"):
        outs = outs[1:-1]
    return props, split_top(ins), split_top(outs)


def parse_props(props: str) -> dict:
    out = {}
    for part in split_top(props):
        if "=" not in part:
            continue
        k, v = part.split("=", 1)
        out[k.strip()] = v.strip()
    return out


def parse_op(line: str) -> Op | None:
    m = _OP.match(line)
    if not m:
        return None
    res, name, operands, rest = m.groups()
    nres = 1
    if res and ":" in res:
        res, k = res.split(":")
        nres = int(k)
    props, ins, outs = _split_sig(rest.strip())
    if ins is None:
        return None
    ops = [o.strip() for o in operands.split(",") if o.strip()]
    op = Op(res, name, ops, props, ins, outs, line, prop_map=parse_props(props), nres=nres)
    if name in ("arith.constant", "tosa.const"):
        key = "value" if name == "arith.constant" else "values"
        v = op.prop_map.get(key)
        if v is not None and len(outs) == 1:
            ty = parse_type(outs[0])
            if ty is not None:
                lit = v.rsplit(" : ", 1)[0] if " : " in v else v
                op.const = parse_const(lit, ty)
    return op


@dataclass
class Func:
    name: str
    ops: list[Op]
    defs: dict                     # value name -> defining op
    ret: Op | None
    index: dict = field(default_factory=dict)   # value name -> result number (for %name#k)


_FUNC = re.compile(r'"func\.func"\(\) <\{.*sym_name = "([^"]+)"')


def parse_funcs(text: str) -> dict[str, Func]:
    """Functions by name; nested regions are read as flat op lists."""
    funcs: dict[str, Func] = {}
    cur = None
    for line in text.splitlines():
        m = _FUNC.search(line)
        if m:
            cur = Func(m.group(1), [], {}, None)
            funcs.setdefault(cur.name, cur)
            continue
        if cur is None:
            continue
        op = parse_op(line)
        if op is None:
            continue
        cur.ops.append(op)
        if op.result and op.nres == 1:
            cur.defs[op.result] = op
        elif op.result:
            for k in range(op.nres):
                cur.defs[f"{op.result}#{k}"] = op
                cur.index[f"{op.result}#{k}"] = k
        if op.name == "func.return":
            cur.ret = op
    return funcs
