"""Drive the reference's golden fold vectors through an engine.

An engine is a module with the host API of mlirpass_b200 (binary, convert,
reciprocal): the product library on a GPU, or the oracle on the CPU.  The
prologue that mlirpass's hooks run before the element loop (poison,
type / elements equality, the dense-cmpf filter, the splat-only tosa folds;
src/patterns/arith/canonicalize.rs:203-217, 457-467 and
src/patterns/tosa/canonicalize.rs:497-511, 596-605) is restated here so each
case reaches the engine exactly when the reference would run its loop.
"""
from __future__ import annotations

import json
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
VECTORS = os.path.join(HERE, "golden", "fold_vectors.json")

STORAGE = {1: np.uint8, 2: np.uint16, 4: np.uint32, 8: np.uint64}
SIZE = {"i1": 1, "i8": 1, "i16": 2, "i32": 4, "i64": 8, "index": 8, "f16": 2, "bf16": 2, "f32": 4, "f64": 8,
        "f8E5M2": 1, "f8E4M3": 1, "f8E3M4": 1}
CANON = {"index": "i64"}
EXTENDED = ("addui_extended", "subui_extended", "mulsi_extended", "mului_extended")
UNARY = ("extf", "truncf", "sitofp", "uitofp", "fptosi", "fptoui", "convertf", "negf", "flush_denormals", "extsi",
         "extui", "trunci", "index_cast", "index_castui",
         # math (same type in and out)
         "absf", "ceil", "floor", "roundeven", "round", "trunc", "sqrt", "rsqrt", "absi", "ctlz", "cttz", "ctpop")
CLASSIFY = ("isfinite", "isinf", "isnan", "isnormal")
FLOAT_BITS = {"f16": (5, 10), "bf16": (8, 7), "f32": (8, 23), "f64": (11, 52), "f8E5M2": (5, 2), "f8E4M3": (4, 3),
              "f8E3M4": (3, 4)}


def load_cases():
    with open(VECTORS) as fh:
        return json.load(fh)["cases"]


def element_cases():
    """Cases whose outcome is decided by the element loop (no shortcut)."""
    return [c for c in load_cases() if c["shortcut"] is None]


def case_id(c) -> str:
    return f'{c["fixture"].split("__")[1]}:{c["func"]}:{c["pos"]}'


def _arr(o):
    dt = CANON.get(o["dtype"], o["dtype"])
    return np.array([int(b, 16) for b in o["bits"]], dtype=STORAGE[SIZE[dt]]), dt


def _int_prop(props, key, default=0):
    v = props.get(key)
    if v is None:
        return default
    return int(v.split(":")[0].strip())


def run_case(c, eng):
    """Returns ("not_folded", None) or ("folded", (splat, bits list))."""
    name = c["op"]
    dialect, op = name.split(".", 1)
    ops = c["operands"]
    res = c["result"]
    rdt = CANON.get(res["dtype"], res["dtype"])
    if dialect == "tosa":
        a, dt = _arr(ops[0])
        if op == "reciprocal":
            if dt not in ("f16", "bf16", "f32", "f64") or not ops[0]["splat"]:
                return "not_folded", None
            f = eng.reciprocal(dt, a, n=1, splat=True)
        else:
            raise ValueError(op)
        return ("folded", (True, [int(x) for x in f.out[:1]])) if f.folded else ("not_folded", None)
    if dialect == "math" and op in CLASSIFY:
        # Folder::classify (src/patterns/math/canonicalize.rs:136-143): a
        # splat float operand only, decided on the host.
        if not ops[0]["splat"]:
            return "not_folded", None
        E, M = FLOAT_BITS[ops[0]["dtype"]]
        b = int(ops[0]["bits"][0], 16)
        e, m, emax = (b >> M) & ((1 << E) - 1), b & ((1 << M) - 1), (1 << E) - 1
        nan, inf = e == emax and m != 0, e == emax and m == 0
        v = {"isfinite": not nan and not inf, "isinf": inf, "isnan": nan, "isnormal": e not in (0, emax)}[op]
        return "folded", (True, [int(v)])
    if op == "bitcast":
        # ApInt::from_bits / ApFloat::from_bits of the same bits
        # (src/patterns/arith/canonicalize.rs:764-789): no element work.
        a, dt = _arr(ops[0])
        return "folded", (ops[0]["splat"], [int(x) for x in a])
    if op in UNARY:
        a, dt = _arr(ops[0])
        n = 1 if ops[0]["splat"] else len(a)
        eop = op
        if op == "convertf":
            eop = "truncf"   # the same float_convert closure (:386)
        elif op in ("index_cast", "index_castui"):
            # sext / zext to the wider width, then trunc (:435-454)
            wi, wo = SIZE[dt], SIZE[rdt]
            eop = "trunci" if wo < wi else ("extsi" if op == "index_cast" else "extui")
        f = eng.convert(eop, dt, rdt, a, n=n, splat=ops[0]["splat"])
        if not f.folded:
            return "not_folded", None
        return "folded", (ops[0]["splat"], [int(x) for x in f.out[:n]])
    if op == "select":
        (cnd, _), (t, dt), (fv, _) = _arr(ops[0]), _arr(ops[1]), _arr(ops[2])
        if not (ops[0]["elements"] and ops[1]["elements"] and ops[2]["elements"]):
            return "not_folded", None
        n = 1
        for d in ops[1]["shape"] or []:
            n *= d
        f = eng.select(cnd, t, fv, n=n, cond_splat=ops[0]["splat"], t_splat=ops[1]["splat"],
                       f_splat=ops[2]["splat"])
        return "folded", (False, [int(x) for x in f.out[:n]])
    if op in EXTENDED:
        # Two results over the same operands (:878-949): result 0 is the
        # wrapped sum / difference / product, result 1 the carry, the borrow
        # (a <u b) or the high product half.
        k = c.get("result_index", 0)
        (a, dt), (b, dt2) = _arr(ops[0]), _arr(ops[1])
        if dt != dt2 or ops[0]["elements"] != ops[1]["elements"]:
            return "not_folded", None
        ls, rs = ops[0]["splat"], ops[1]["splat"]
        n = 1 if (ls and rs) else max(len(a), len(b))
        base = {"addui_extended": "addi", "subui_extended": "subi"}.get(op, "muli")
        second = {"addui_extended": ("addui_carry", 0), "subui_extended": ("cmpi", 6 << 8),
                  "mulsi_extended": ("mulsi_hi", 0), "mului_extended": ("mului_hi", 0)}[op]
        eop, fl = (base, 0) if k == 0 else second
        f = eng.binary(eop, dt, a, b, n=n, lhs_splat=ls, rhs_splat=rs, flags=fl)
        if not f.folded:
            return "not_folded", None
        return "folded", (ls and rs, [int(x) for x in f.out[:n]])
    # binary
    (a, dt), (b, dt2) = _arr(ops[0]), _arr(ops[1])
    if dt != dt2 or ops[0]["elements"] != ops[1]["elements"] or ops[0]["shape"] != ops[1]["shape"]:
        return "not_folded", None
    if op == "cmpf" and ops[0]["elements"]:
        return "not_folded", None
    pred = _int_prop(c["props"], "predicate")
    mode = _int_prop(c["props"], "roundingmode")
    fl = (mode & 7) | ((pred & 15) << 8)
    ls, rs = ops[0]["splat"], ops[1]["splat"]
    n = 1 if (ls and rs) else max(len(a), len(b))
    f = eng.binary(op, dt, a, b, n=n, lhs_splat=ls, rhs_splat=rs, flags=fl)
    if not f.folded:
        return "not_folded", None
    return "folded", (ls and rs, [int(x) for x in f.out[:n]])


def check_case(c, eng):
    status, got = run_case(c, eng)
    exp = c["expected"]
    assert status == exp["status"], f"{case_id(c)}: expected {exp['status']}, got {status}"
    if status == "folded":
        splat, bits = got
        want = [int(x, 16) for x in exp["bits"]]
        if exp["splat"]:
            assert all(x == want[0] for x in bits), f"{case_id(c)}: {bits} != splat {want}"
        else:
            assert bits == want, f"{case_id(c)}: {[hex(x) for x in bits]} != {[hex(x) for x in want]}"
