"""Harvest golden fold vectors from the reference's own fixtures.

Run here (the container that has the reference checkout):

    python tests/golden/make_golden.py /path/to/mlirpass

It reads mlirpass's `tests/fixtures/<stem>.in.mlir` (the input, as
mlir-opt 23.1.5 prints it) and `<stem>.generic.mlir` (mlir-opt's output of
the fixture's canonicalize RUN line), for every fixture whose pipeline is a
plain canonicalize.  For each function, every value returned by `func.return`
or stored by `memref.store` that is produced by a hot-path fold op whose
operands are all constants becomes one case; the expected outcome is read at
the same position of the output function: a constant (folded, with its value
and the exact text mlir-opt printed for it) or the same op (not folded).  Cases the output rewrote into something else are dropped.

Math dialect fixtures (ArithFolder::math, src/patterns/math/canonicalize.rs)
contribute the exact folds.  Each case is also labelled with the shortcut,
if any, that ArithFolder::fold
(src/patterns/arith/canonicalize.rs:270-491) or Tf::fold
(src/patterns/tosa/canonicalize.rs:189-232) takes before the per-element
loop, so element-level tests can select the cases that reach the loop.

Output: tests/golden/fold_vectors.json (committed).  The tests read only
that file, never the reference.
"""
from __future__ import annotations

import json
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
from mlir_text import FLOATS, INTS, parse_funcs, parse_type  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "fold_vectors.json")

BINARY_F = {"addf", "subf", "mulf", "divf", "maximumf", "minimumf", "maxnumf", "minnumf", "remf"}
BINARY_I = {"addi", "subi", "muli", "andi", "ori", "xori", "shli", "shrui", "shrsi",
            "divsi", "divui", "remsi", "remui", "maxsi", "maxui", "minsi", "minui",
            "ceildivui", "ceildivsi", "floordivsi"}
CONVERT = {"extf", "truncf", "sitofp", "uitofp", "fptosi", "fptoui", "convertf", "negf", "flush_denormals",
           "extsi", "extui", "trunci", "index_cast", "index_castui", "bitcast"}
CMP = {"cmpi", "cmpf"}
EXTENDED = {"addui_extended", "subui_extended", "mulsi_extended", "mului_extended"}
ARITH = BINARY_F | BINARY_I | CONVERT | CMP | {"select"} | EXTENDED
TOSA = {"reciprocal", "transpose"}
# math dialect folds with an exact result (the transcendental ones are the
# host C library's values in the reference and have no device restatement)
MATH = {"absf", "ceil", "floor", "roundeven", "round", "trunc", "sqrt", "rsqrt", "absi", "ctlz", "cttz", "ctpop",
        "copysign", "ipowi", "isfinite", "isinf", "isnan", "isnormal"}

ALLOWED_FLAGS = ("-split-input-file", "--split-input-file", "-allow-unregistered-dialect",
                 "--allow-unregistered-dialect")


def plain_canonicalize(args: str) -> bool:
    toks = args.split()
    canon = [t for t in toks if t not in ALLOWED_FLAGS]
    if len(canon) == 0:
        return False
    rest = " ".join(canon)
    if "filter-dialects" in rest or "max-iterations" in rest or "enable-patterns" in rest:
        return False
    if rest.startswith("-canonicalize") or rest.startswith("--canonicalize"):
        return all(t.startswith(("-canonicalize", "--canonicalize", "top-down", "region-simplify"))
                   for t in canon)
    if rest.startswith("-pass-pipeline=") or rest.startswith("--pass-pipeline="):
        pipe = rest.split("=", 1)[1]
        return "canonicalize" in pipe and pipe.count("(") <= 3 and "," not in pipe.replace(
            "canonicalize{test-convergence region-simplify=aggressive}", "")
    return False


def f_is(bits: int, dt: str, what: str) -> bool:
    E, M, _ = FLOATS[dt]
    sign = (bits >> (E + M)) & 1
    mag = bits & ((1 << (E + M)) - 1)
    expf = mag >> M
    mant = mag & ((1 << M) - 1)
    if what == "negzero":
        return sign == 1 and mag == 0
    if what == "poszero":
        return sign == 0 and mag == 0
    if what == "zero":
        return mag == 0
    if what == "one":
        bias = (1 << (E - 1)) - 1
        return sign == 0 and expf == bias and mant == 0
    if what == "neginf":
        return sign == 1 and expf == (1 << E) - 1 and mant == 0
    if what == "posinf":
        return sign == 0 and expf == (1 << E) - 1 and mant == 0
    if what == "nan":
        return expf == (1 << E) - 1 and mant != 0
    raise ValueError(what)


def scalar_of(c):
    """as_int / as_float: Some for a scalar or a one-value (splat) Const."""
    if c.splat:
        return c.bits[0]
    return None


def ambiguous(c) -> bool:
    # A non-splat literal whose values are all equal: whether mlirformat's
    # Const treats it as a splat for as_int/as_float is not knowable here.
    return (not c.splat) and len(set(c.bits)) == 1


def shortcut(op: str, ops, consts, props) -> str | None:
    """The value/attribute shortcut ArithFolder::fold takes, or None."""
    rhs = consts[1] if len(consts) > 1 else None
    same = len(ops) > 1 and ops[0].result == ops[1].result
    dt = consts[0].ty.elem
    r = scalar_of(rhs) if rhs is not None else None
    w = INTS.get(dt)
    fast = props.get("fastmath", "")
    if op == "addf" and r is not None and f_is(r, dt, "negzero"):
        return "value0"
    if op == "subf" and r is not None and f_is(r, dt, "poszero"):
        return "value0"
    if op in ("mulf", "divf") and r is not None and f_is(r, dt, "one"):
        return "value0"
    if op == "mulf" and r is not None and f_is(r, dt, "zero") and (
            "fast" in fast or ("nnan" in fast and "nsz" in fast)):
        return "value1"
    if op in ("maximumf", "minimumf", "maxnumf", "minnumf"):
        if same:
            return "value1"
        if r is not None:
            mx = op.startswith("max")
            if op.endswith("imumf") and f_is(r, dt, "neginf" if mx else "posinf"):
                return "value0"
            if op.endswith("numf") and f_is(r, dt, "nan"):
                return "value0"
    if op in EXTENDED:
        zero = r is not None and r == 0
        if zero:
            return "zero_rhs"
        if op == "mului_extended" and r == 1:
            return "one_rhs"
        if op == "subui_extended" and same:
            return "same"
        return None
    if op == "select":
        t_same = ops[1].result == ops[2].result
        c = scalar_of(consts[0])
        if t_same:
            return "value1"
        if c is not None:
            return "value1" if c != 0 else "value2"
        return None
    if op in BINARY_I or op == "cmpi":
        zero = r is not None and r == 0
        one = r is not None and r == 1
        ones = r is not None and r == (1 << w) - 1
        if op == "addi" and zero:
            return "value0"
        if op == "subi" and same:
            return "zero"
        if op == "subi" and zero:
            return "value0"
        if op == "muli" and zero:
            return "value1"
        if op == "muli" and one:
            return "value0"
        if op in ("divsi", "divui", "ceildivui", "ceildivsi", "floordivsi") and one:
            return "value0"
        if op in ("remsi", "remui") and one:
            return "zero"
        if op == "andi" and zero:
            return "value1"
        if op == "andi" and ones:
            return "value0"
        if op == "ori" and r is not None and (zero or ones):
            return "value0" if zero else "attr1"
        if op == "xori" and zero:
            return "value0"
        if op == "xori" and same:
            return "zero"
        if op in ("shli", "shrui", "shrsi") and zero:
            return "value0"
        if op in ("maxsi", "maxui", "minsi", "minui"):
            if same:
                return "value1"
            if r is not None:
                signed = op.endswith("si")
                lo = (1 << (w - 1)) if signed else 0
                hi = ((1 << (w - 1)) - 1) if signed else (1 << w) - 1
                if r == (hi if op.startswith("max") else lo):
                    return "value1"
                if r == (lo if op.startswith("max") else hi):
                    return "value0"
        if op == "cmpi" and same:
            return "same"
    return None


def sinks(f):
    """The values a function observes, in order: those it stores with
    memref.store, then those it returns."""
    out = [op.operands[0] for op in f.ops if op.name == "memref.store" and op.operands]
    return out + list(f.ret.operands)


def main():
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py <path of the mlirpass checkout>")
    fix = os.path.join(sys.argv[1], "tests", "fixtures")
    cases = []
    stems = sorted(f[:-5] for f in os.listdir(fix) if f.endswith(".args"))
    for stem in stems:
        with open(os.path.join(fix, stem + ".args")) as fh:
            args = fh.read().replace("\n", " ")
        if not plain_canonicalize(args):
            continue
        pin = os.path.join(fix, stem + ".in.mlir")
        pout = os.path.join(fix, stem + ".generic.mlir")
        if not (os.path.exists(pin) and os.path.exists(pout)):
            continue
        a_chunks = open(pin).read().split("// -----")
        b_chunks = open(pout).read().split("// -----")
        if len(a_chunks) != len(b_chunks):
            continue
        for a, b in zip(a_chunks, b_chunks):
            fin, fout = parse_funcs(a), parse_funcs(b)
            for name, f in fin.items():
                g = fout.get(name)
                if g is None or f.ret is None or g.ret is None:
                    continue
                fs, gs = sinks(f), sinks(g)
                if len(fs) != len(gs):
                    continue
                for pos, (v, gv) in enumerate(zip(fs, gs)):
                    op = f.defs.get(v)
                    if op is None or "." not in op.name:
                        continue
                    dialect, short = op.name.split(".", 1)
                    if not ((dialect == "arith" and short in ARITH) or (dialect == "tosa" and short in TOSA)
                            or (dialect == "math" and short in MATH)):
                        continue
                    opnds = [f.defs.get(o) for o in op.operands]
                    if short == "transpose":
                        opnds = opnds[:1]
                    if not opnds or any(c is None or c.const is None for c in opnds):
                        continue
                    consts = [c.const for c in opnds]
                    if any(ambiguous(c) for c in consts):
                        continue
                    k = f.index.get(v, 0)
                    if len(op.out_types) != op.nres or k >= len(op.out_types):
                        continue
                    res_ty = parse_type(op.out_types[k])
                    if res_ty is None:
                        continue
                    gop = g.defs.get(gv)
                    if gop is None:
                        continue
                    if gop.name in ("arith.constant", "tosa.const") and gop.const is not None:
                        key = "value" if gop.name == "arith.constant" else "values"
                        exp = {"status": "folded", "splat": gop.const.splat,
                               "dtype": gop.const.ty.elem,
                               "bits": [format(x, "x") for x in gop.const.bits],
                               "text": gop.prop_map[key]}
                    elif gop.name == op.name:
                        exp = {"status": "not_folded"}
                    else:
                        continue
                    props = {k: v for k, v in op.prop_map.items()}
                    case = {
                        "fixture": stem, "func": name, "pos": pos, "op": op.name,
                        "props": props,
                        "operands": [{
                            "ssa": o.result, "dtype": c.ty.elem, "shape": c.ty.shape,
                            "kind": c.ty.kind, "splat": c.splat, "elements": c.elements,
                            "bits": [format(x, "x") for x in c.bits]} for o, c in zip(opnds, consts)],
                        "result": {"dtype": res_ty.elem, "shape": res_ty.shape, "kind": res_ty.kind},
                        "result_index": k, "result_types": op.out_types,
                        "shortcut": shortcut(short, opnds, consts, props) if dialect == "arith" else None,
                        "expected": exp,
                    }
                    cases.append(case)
    with open(OUT, "w") as fh:
        json.dump({"source": "mlirpass tests/fixtures (mlir-opt 23.1.5 outputs)",
                   "generator": "tests/golden/make_golden.py", "cases": cases}, fh, indent=1)
    by = {}
    for c in cases:
        by[c["op"]] = by.get(c["op"], 0) + 1
    print(len(cases), "cases", json.dumps(by, sort_keys=True))


if __name__ == "__main__":
    main()
