"""The five fold configurations at full size through the pass driver.

Each configuration's MLIR text (0.02-5.4 GB of `dense<"0x…">` literals) runs
through `dcf_opt_run` with the pipeline the configuration names, as
mlirpass's fixture harness runs a whole module and compares the printed
result (tests/passes.rs:60-90).  For every function of the printed module
the test checks the op list (what folded, what was left in place) and
compares every returned constant bit for bit with the oracle (the CPU
restatement of the reference's fold closures).  The outcomes are the
reference's: dense cmpf, inexact truncf and divsi with INT_MIN / -1 are not
folded (src/patterns/arith/canonicalize.rs:457-467, :727-762, :538-555);
remsi folds INT_MIN % -1 to 0 (:319-325).

These sizes are where the driver's full-size code paths run: staging slots
and packed uploads of hundreds of MB, several fold rounds, batches of 1024
small folds through the allocation-free batch entry point, and 2^28-element
transposes.
"""
import json
import os

import numpy as np
import pytest

from full_module import returns_digest, scan
from mlirpass_b200 import mlir_gen, opt
from mlirpass_b200 import workloads as W

pytestmark = pytest.mark.gpu

U32, U64, U16, U8 = np.uint32, np.uint64, np.uint16, np.uint8


def run(module, pipeline):
    text = module.tobytes()
    out, st = opt.run(text, pipeline, as_bytes=True)
    del text
    return scan(out), st


def names(f):
    return [o.name for o in f.ops]


DIGESTS = json.load(open(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "config_digests.json")))


def same_digest(m, config):
    """The committed digest of the configuration's results (which bench.py
    checks every timed run against) is the digest of this output, which the
    test has just compared value by value with the oracle."""
    assert returns_digest(m) == DIGESTS[config], config


def test_config1_full(oracle):
    m, st = run(mlir_gen.config1_module(), "canonicalize")
    c = W.config1()
    (d,) = m.returned("main")
    assert names(m.funcs["main"]) == ["arith.constant", "func.return"]
    want = oracle.binary("addf", "f32", c["A"], c["B"]).out
    assert np.array_equal(m.values(d, U32), want)
    assert st["folds"] == 1
    same_digest(m, "config1")


def test_config2_full(oracle):
    m, st = run(mlir_gen.config2_module(), "canonicalize")
    c = W.config2()
    env = {k: c[k].view(U32) for k in "ABCD"}
    for op, a, b, t in W.CHAIN2:
        env[t] = oracle.binary(op, "f32", env[a], env[b]).out
    assert not np.isnan(env["t6"].view(np.float32)).any()      # no NaN-producing arithmetic in the chain
    (d,) = m.returned("main")
    assert names(m.funcs["main"]) == ["arith.constant", "func.return"]
    assert np.array_equal(m.values(d, U32), env["t6"])
    assert st["folds"] == 6 and st["refused"] == 0
    same_digest(m, "config2")


@pytest.mark.parametrize("dt", ["i8", "i32", "i64"])
def test_config3_full(dt, oracle):
    m, st = run(mlir_gen.config3_module(dt), "canonicalize")
    c = W.config3(dt)
    store = {"i8": U8, "i32": U32, "i64": U64}[dt]
    res = m.returned("main")
    expect = [("addi", "X", "Y"), ("muli", "X", "Y"), ("subi", "X", "Y"), ("andi", "X", "Y"), ("xori", "X", "Y"),
              ("shli", "X", "S"), ("divsi", "Xd", "Yd"), ("remsi", "Xd", "Yd")]
    f = m.funcs["main"]
    for d, (op, a, b) in zip(res, expect):
        want = oracle.binary(op, dt, c[a], c[b])
        if op == "divsi":
            # INT_MIN / -1 is planted: the reference refuses the whole fold.
            assert not want.folded and d.name == "arith.divsi"
            la, lb = (f.defs[v] for v in d.operands)
            assert np.array_equal(m.values(la, store), c["Xd"]) and np.array_equal(m.values(lb, store), c["Yd"])
            continue
        assert want.folded and d.name == "arith.constant", op
        assert np.array_equal(m.values(d, store), want.out), op
    assert sorted(set(names(f))) == ["arith.constant", "arith.divsi", "func.return"]
    assert names(f).count("arith.constant") == 9          # 7 folded results + the divsi's two operands
    assert st["folds"] == 7
    same_digest(m, f"config3-{dt}")


def test_config4_full(oracle):
    n = 16 * 1024 * 1024
    m, st = run(mlir_gen.config4_module(n), "canonicalize")
    c = W.config4(n)
    t1, t2, e1, e2, si, fp, c1, c2 = m.returned("main")
    f = m.funcs["main"]
    # normal(0, 1e3) values are not exact in bf16 / f16: truncf refuses, so
    # extf of it has no constant operand; dense cmpf never folds.
    assert not oracle.convert("truncf", "f32", "bf16", c["x"]).folded
    assert not oracle.convert("truncf", "f32", "f16", c["x"]).folded
    assert [t1.name, t2.name, e1.name, e2.name, c1.name, c2.name] == \
        ["arith.truncf", "arith.truncf", "arith.extf", "arith.extf", "arith.cmpf", "arith.cmpf"]
    assert np.array_equal(m.values(f.defs[t1.operands[0]], U32), c["x"])
    assert np.array_equal(m.values(f.defs[c1.operands[1]], U32), c["inrange"])
    assert np.array_equal(m.values(si, U32), oracle.convert("fptosi", "f32", "i32", c["inrange"]).out)
    assert np.array_equal(m.values(fp, U32), oracle.convert("sitofp", "i32", "f32", c["ints"]).out)
    assert st["folds"] == 2
    same_digest(m, "config4")


def test_config4b_full(oracle):
    n = 16 * 1024 * 1024
    m, st = run(mlir_gen.config4_module(n, prerounded=True), "canonicalize")
    c = W.config4(n, prerounded=True)
    t1, t2, e1, e2, si, fp, c1, c2 = m.returned("main")
    tb = oracle.convert("truncf", "f32", "bf16", c["x"])
    th = oracle.convert("truncf", "f32", "f16", c["x_f16"])
    assert tb.folded and th.folded
    assert np.array_equal(m.values(t1, U16), tb.out) and np.array_equal(m.values(t2, U16), th.out)
    # extf(truncf(x)) gives x back (the def-chain shortcut or the fold)
    assert np.array_equal(m.values(e1, U32), c["x"]) and np.array_equal(m.values(e2, U32), c["x_f16"])
    assert np.array_equal(m.values(si, U32), oracle.convert("fptosi", "f32", "i32", c["inrange"]).out)
    assert np.array_equal(m.values(fp, U32), oracle.convert("sitofp", "i32", "f32", c["ints"]).out)
    assert c1.name == "arith.cmpf" and c2.name == "arith.cmpf"
    same_digest(m, "config4b")


def test_config5_full(oracle):
    funcs, side, ws = 4096, 256, 16384
    m, st = run(mlir_gen.config5_module(funcs, side, ws), mlir_gen.LAYERWISE)
    assert len(m.funcs) == funcs + 1
    for i in range(funcs):
        a, b = W.config5_func(i, side)
        t1 = oracle.binary("addf", "f32", a, b).out
        t2 = oracle.binary("mulf", "f32", t1, a).out
        r = oracle.reciprocal("f32", t2)
        f = m.funcs[f"f{i}"]
        assert names(f) == ["tosa.const", "func.return"], f"f{i}"
        assert r.folded and np.array_equal(m.values(f.defs[f.ret.operands[0]], U32), r.out), f"f{i}"
    f = m.funcs["weights"]
    assert names(f) == ["tosa.const", "func.return"]
    w = W.config5_weight(ws).reshape(ws, ws)
    got = m.values(f.defs[f.ret.operands[0]], U16).reshape(ws, ws)
    assert np.array_equal(got, w.T)
    assert st["folds"] == 3 * funcs + 1 and st["refused"] == 0
    same_digest(m, "config5")
