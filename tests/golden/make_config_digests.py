"""Digests of the expected results of the five fold configurations at full
size, from the oracle (test infrastructure: run here, on the CPU).

    python tests/golden/make_config_digests.py [config ...]

For each configuration the expected returned values of every function are
written down as the oracle computes them (a folded constant: the sha256 of
the uppercase hex of its raw bytes, as the printer writes its `dense<"0x…">`
body; a value the reference leaves unfolded: the op's name), and combined
into one digest (tests/full_module.py: combine).  bench.py checks the
printed module of every pass run it times against these digests, and
tests/test_gpu_full_configs.py checks that the driver's output, verified
constant by constant against the oracle, has exactly these digests.

Output: tests/golden/config_digests.json (committed).
"""
from __future__ import annotations

import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [ROOT, HERE, os.path.dirname(HERE)]

import numpy as np  # noqa: E402

import oracle  # noqa: E402
from full_module import combine, entry_const, entry_op  # noqa: E402
from mlirpass_b200 import workloads as W  # noqa: E402

OUT = os.path.join(HERE, "config_digests.json")


def hx(a) -> bytes:
    return W.hex_upper(np.ascontiguousarray(a)).encode()


def config1():
    c = W.config1()
    return combine(["main " + entry_const(hx(oracle.binary("addf", "f32", c["A"], c["B"]).out))])


def config2():
    c = W.config2()
    env = {k: c[k].view(np.uint32) for k in "ABCD"}
    for op, a, b, t in W.CHAIN2:
        env[t] = oracle.binary(op, "f32", env[a], env[b]).out
    return combine(["main " + entry_const(hx(env["t6"]))])


def config3(dt):
    c = W.config3(dt)
    e = []
    for op, a, b in [("addi", "X", "Y"), ("muli", "X", "Y"), ("subi", "X", "Y"), ("andi", "X", "Y"),
                     ("xori", "X", "Y"), ("shli", "X", "S"), ("divsi", "Xd", "Yd"), ("remsi", "Xd", "Yd")]:
        r = oracle.binary(op, dt, c[a], c[b])
        e.append("main " + (entry_const(hx(r.out)) if r.folded else entry_op("arith." + op)))
    return combine(e)


def config4(prerounded):
    c = W.config4(prerounded=prerounded)
    e = []
    for src, to in (("x", "bf16"), ("x_f16" if prerounded else "x", "f16")):
        r = oracle.convert("truncf", "f32", to, c[src])
        e.append("main " + (entry_const(hx(r.out)) if r.folded else entry_op("arith.truncf")))
    for src in ("x", "x_f16" if prerounded else "x"):
        e.append("main " + (entry_const(hx(c[src])) if prerounded else entry_op("arith.extf")))
    e.append("main " + entry_const(hx(oracle.convert("fptosi", "f32", "i32", c["inrange"]).out)))
    e.append("main " + entry_const(hx(oracle.convert("sitofp", "i32", "f32", c["ints"]).out)))
    e += ["main " + entry_op("arith.cmpf")] * 2
    return combine(e)


def config5(funcs=4096, side=256, ws=16384):
    e = []
    for i in range(funcs):
        a, b = W.config5_func(i, side)
        t1 = oracle.binary("addf", "f32", a, b).out
        t2 = oracle.binary("mulf", "f32", t1, a).out
        e.append(f"f{i} " + entry_const(hx(oracle.reciprocal("f32", t2).out)))
    w = W.config5_weight(ws).reshape(ws, ws)
    e.append("weights " + entry_const(hx(np.ascontiguousarray(w.T))))
    return combine(e)


MAKERS = {"config1": config1, "config2": config2, "config3-i8": lambda: config3("i8"),
          "config3-i32": lambda: config3("i32"), "config3-i64": lambda: config3("i64"),
          "config4": lambda: config4(False), "config4b": lambda: config4(True), "config5": config5}


def main():
    names = sys.argv[1:] or list(MAKERS)
    d = json.load(open(OUT)) if os.path.exists(OUT) else {}
    d.setdefault("generator", "tests/golden/make_config_digests.py")
    for n in names:
        d[n] = MAKERS[n]()
        print(n, d[n], flush=True)
    with open(OUT, "w") as fh:
        json.dump(d, fh, indent=1, sort_keys=True)


if __name__ == "__main__":
    main()
