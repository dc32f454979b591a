"""The five fold configurations at full size, through the C ABI, against the
oracle (bit for bit, and the same fold / no-fold decisions the reference
makes: divsi with INT_MIN / -1 refuses, remsi folds, inexact truncf
refuses, pre-rounded truncf folds)."""
import numpy as np
import pytest

from mlirpass_b200 import workloads as W

pytestmark = pytest.mark.gpu


def same(g, c, n):
    assert g.folded == c.folded and g.first_fail_index == c.first_fail_index
    if c.folded:
        assert np.array_equal(g.out[:n], c.out[:n])
        assert g.is_splat == c.is_splat


def test_config1(dcf, oracle):
    d = W.config1()
    g, c = dcf.binary("addf", "f32", d["A"], d["B"]), oracle.binary("addf", "f32", d["A"], d["B"])
    assert c.folded and not c.is_splat
    same(g, c, len(d["A"]))


def test_config2_chain(dcf, oracle):
    d = W.config2()
    env_g = {k: d[k] for k in "ABCD"}
    env_c = dict(env_g)
    for op, a, b, t in W.CHAIN2:
        g = dcf.binary(op, "f32", env_g[a], env_g[b])
        c = oracle.binary(op, "f32", env_c[a], env_c[b])
        assert c.folded
        same(g, c, len(d["A"]))
        env_g[t], env_c[t] = g.out.view(np.float32), c.out.view(np.float32)
        assert not np.isnan(env_c[t]).any(), t
    assert np.isinf(env_c["t4"]).sum() == len(d["zeros"])


@pytest.mark.parametrize("dt", ["i8", "i32", "i64"])
def test_config3(dt, dcf, oracle):
    d = W.config3(dt)
    n = len(d["X"])
    for op in ("addi", "muli", "subi", "andi", "xori"):
        g, c = dcf.binary(op, dt, d["X"], d["Y"]), oracle.binary(op, dt, d["X"], d["Y"])
        assert c.folded
        same(g, c, n)
    g, c = dcf.binary("shli", dt, d["X"], d["S"]), oracle.binary("shli", dt, d["X"], d["S"])
    assert c.folded
    same(g, c, n)
    g, c = dcf.binary("divsi", dt, d["Xd"], d["Yd"]), oracle.binary("divsi", dt, d["Xd"], d["Yd"])
    assert not c.folded and c.first_fail_index == int(d["pairs"][0])
    same(g, c, n)
    g, c = dcf.binary("remsi", dt, d["Xd"], d["Yd"]), oracle.binary("remsi", dt, d["Xd"], d["Yd"])
    assert c.folded
    same(g, c, n)


def test_config4(dcf, oracle):
    d = W.config4()
    x = d["x"]
    for to in ("bf16", "f16"):
        g, c = dcf.convert("truncf", "f32", to, x), oracle.convert("truncf", "f32", to, x)
        assert not c.folded
        same(g, c, len(x))
    g, c = dcf.convert("fptosi", "f32", "i32", d["inrange"]), oracle.convert("fptosi", "f32", "i32", d["inrange"])
    assert c.folded
    same(g, c, len(x))
    g, c = dcf.convert("sitofp", "i32", "f32", d["ints"]), oracle.convert("sitofp", "i32", "f32", d["ints"])
    assert c.folded
    same(g, c, len(x))
    for pred in (4, 13):   # olt, une: computed for completeness; the reference never folds dense cmpf
        g = dcf.binary("cmpf", "f32", x, d["inrange"], flags=pred << 8)
        c = oracle.binary("cmpf", "f32", x, d["inrange"], flags=pred << 8)
        same(g, c, len(x))


def test_config4b_prerounded(dcf, oracle):
    d = W.config4(prerounded=True)
    g, c = dcf.convert("truncf", "f32", "bf16", d["x"]), oracle.convert("truncf", "f32", "bf16", d["x"])
    assert c.folded
    same(g, c, len(d["x"]))
    back_g = dcf.convert("extf", "bf16", "f32", g.out)
    back_c = oracle.convert("extf", "bf16", "f32", c.out)
    assert back_c.folded and np.array_equal(back_c.out, d["x"])
    same(back_g, back_c, len(d["x"]))
    g, c = dcf.convert("truncf", "f32", "f16", d["x_f16"]), oracle.convert("truncf", "f32", "f16", d["x_f16"])
    assert c.folded
    same(g, c, len(d["x"]))


def test_config5_funcs(dcf, oracle):
    funcs = [W.config5_func(i) for i in range(64)]
    s1 = dcf.batch([{"op": "addf", "dtype": "f32", "lhs": a, "rhs": b} for a, b in funcs])
    s2 = dcf.batch([{"op": "mulf", "dtype": "f32", "lhs": r.out, "rhs": a} for r, (a, _) in zip(s1, funcs)])
    s3 = dcf.batch([{"op": "reciprocal", "dtype": "f32", "lhs": r.out} for r in s2])
    for (a, b), r1, r2, r3 in zip(funcs, s1, s2, s3):
        c1 = oracle.binary("addf", "f32", a, b)
        c2 = oracle.binary("mulf", "f32", c1.out, a)
        c3 = oracle.reciprocal("f32", c2.out)
        same(r1, c1, len(a))
        same(r2, c2, len(a))
        same(r3, c3, len(a))


def test_config5_transpose(dcf):
    side = 16384
    w = W.config5_weight(side)
    f = dcf.transpose(w, (side, side), (1, 0))
    assert f.folded and not f.is_splat
    assert np.array_equal(f.out, w.reshape(side, side).T)
