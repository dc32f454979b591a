"""The pass driver on a B200: whole pipelines on MLIR text.

Every golden case (a fold op over constants from the reference's fixtures)
becomes a function and runs through `canonicalize`; the returned value must
be the fixture's folded constant, or the op left in place.  Then the fold
configurations run end to end through `--canonicalize` and
`builtin.module(func.func(tosa-layerwise-constant-fold,canonicalize))`, and
every resulting constant is compared bit for bit with the oracle.
"""
import numpy as np
import pytest

from golden_cases import CANON, SIZE, STORAGE, case_id, load_cases
from mlir_text import parse_funcs
from mlirpass_b200 import mlir_gen, opt
from mlirpass_b200 import workloads as W

pytestmark = pytest.mark.gpu

CASES = load_cases()


def ty_text(o):
    if o["shape"] is None:
        return o["dtype"]
    return f'{o["kind"]}<{"x".join(str(d) for d in o["shape"])}x{o["dtype"]}>'


def literal(o):
    dt = CANON.get(o["dtype"], o["dtype"])
    bits = [int(b, 16) for b in o["bits"]]
    isf = dt.startswith("f") or dt == "bf16"
    def one(b):
        if isf:
            return "0x%0*X" % (2 * SIZE[dt], b)
        if dt == "i1":
            return "true" if b else "false"
        w = 8 * SIZE[dt]
        return str(b - (1 << w) if b >> (w - 1) else b)
    if o["shape"] is None:
        return one(bits[0]) if dt == "i1" else f"{one(bits[0])} : {ty_text(o)}"
    if o["splat"]:
        return f"dense<{one(bits[0])}> : {ty_text(o)}"
    if dt == "i1":   # i1 constants are written as lists (MLIR's raw i1 form is bit-packed)
        return f"dense<[{', '.join(one(b) for b in bits)}]> : {ty_text(o)}"
    raw = np.array(bits, dtype=STORAGE[SIZE[dt]]).tobytes().hex().upper()
    return f'dense<"0x{raw}"> : {ty_text(o)}'


def render(c):
    lines, names = [], []
    dialect = c["op"].split(".")[0]
    for i, o in enumerate(c["operands"]):
        op, key = ("tosa.const", "values") if dialect == "tosa" else ("arith.constant", "value")
        ty = ty_text(o)
        lines.append(f'    %{i} = "{op}"() <{{{key} = {literal(o)}}}> : () -> {ty}')
        names.append(f"%{i}")
    props = dict(c["props"])
    p = ", ".join(f"{k} = {v}" for k, v in props.items())
    rty = ty_text(c["result"])
    ins = ", ".join(ty_text(o) for o in c["operands"])
    args = ", ".join(names)
    if c["op"] == "tosa.transpose":
        args, ins = names[0], ty_text(c["operands"][0])
    pr = " <{" + p + "}>" if p else ""
    all_ty = c.get("result_types") or [rty]
    if len(all_ty) > 1:   # a two-result op: %r:2 = ..., returning %r#k
        lines.append(f'    %r:{len(all_ty)} = "{c["op"]}"({args}){pr} : ({ins}) -> ({", ".join(all_ty)})')
        ret = f'%r#{c["result_index"]}'
    else:
        lines.append(f'    %r = "{c["op"]}"({args}){pr} : ({ins}) -> {rty}')
        ret = "%r"
    return ('"builtin.module"() ({\n'
            f'  "func.func"() <{{function_type = () -> {rty}, sym_name = "t"}}> ({{\n' + "\n".join(lines) +
            f'\n    "func.return"({ret}) : ({rty}) -> ()\n  }}) : () -> ()\n}}) : () -> ()\n')


def check_golden_output(case, out):
    """The returned value is the fixture's: the op left in place, or a
    constant with the fixture's bits whose attribute text is exactly the
    text mlir-opt printed for it."""
    f = parse_funcs(out)["t"]
    d = f.defs.get(f.ret.operands[0])
    exp = case["expected"]
    if exp["status"] == "not_folded":
        assert d is not None and d.name == case["op"], out
        return
    assert d is not None and d.const is not None, out
    want = [int(x, 16) for x in exp["bits"]]
    got = d.const.bits
    if exp["splat"]:
        assert set(got) == {want[0]}, (got, want)
    else:
        assert got == want, (got, want)
    key = "value" if d.name == "arith.constant" else "values"
    assert d.prop_map[key] == exp["text"], (d.prop_map[key], exp["text"])


@pytest.mark.parametrize("case", CASES, ids=[case_id(c) for c in CASES])
def test_golden_through_canonicalize(case):
    out, _ = opt.run(render(case), "canonicalize")
    check_golden_output(case, out)


def consts_returned(out, name="main"):
    f = parse_funcs(out)[name]
    res = []
    for v in f.ret.operands:
        d = f.defs.get(v)
        res.append(d)
    return res


def full(d, n):
    """Values of a parsed constant, expanded if it was printed as a splat."""
    a = np.array(d.const.bits, dtype=np.uint64)
    return np.full(n, a[0], dtype=np.uint64) if d.const.splat else a


def test_config1_pipeline(oracle):
    out, st = opt.run(mlir_gen.config1_text(), "canonicalize")
    (d,) = consts_returned(out)
    c = W.config1()
    want = oracle.binary("addf", "f32", c["A"], c["B"]).out
    assert d.name == "arith.constant" and np.array_equal(full(d, want.size), want.astype(np.uint64))
    assert st["folds"] == 1 and st["run_ms"] > 0


def test_config2_chain_pipeline(oracle):
    out, st = opt.run(mlir_gen.config2_text(1024), "canonicalize")
    (d,) = consts_returned(out)
    c = W.config2(1024)
    env = {k: c[k] for k in "ABCD"}
    for op, a, b, t in W.CHAIN2:
        env[t] = oracle.binary(op, "f32", env[a], env[b]).out.view(np.float32)
    assert np.array_equal(full(d, 1 << 20), env["t6"].view(np.uint32).astype(np.uint64))
    assert st["folds"] == 6
    f = parse_funcs(out)["main"]
    assert [o.name for o in f.ops] == ["arith.constant", "func.return"]


@pytest.mark.parametrize("dt", ["i8", "i32", "i64"])
def test_config3_pipeline(dt, oracle):
    rows, cols = 1024, 512
    out, st = opt.run(mlir_gen.config3_text(dt, rows, cols), "canonicalize")
    res = consts_returned(out)
    c = W.config3(dt, rows, cols)
    n = rows * cols
    expect = [("addi", "X", "Y"), ("muli", "X", "Y"), ("subi", "X", "Y"), ("andi", "X", "Y"), ("xori", "X", "Y"),
              ("shli", "X", "S"), ("divsi", "Xd", "Yd"), ("remsi", "Xd", "Yd")]
    for d, (op, a, b) in zip(res, expect):
        want = oracle.binary(op, dt, c[a], c[b])
        if want.folded:
            assert d.name == "arith.constant", op
            assert np.array_equal(full(d, n), want.out.astype(np.uint64)), op
        else:
            assert d.name == "arith." + op, op   # divsi refuses on INT_MIN / -1
    assert res[6].name == "arith.divsi" and res[7].name == "arith.constant"


@pytest.mark.parametrize("prerounded", [False, True])
def test_config4_pipeline(prerounded, oracle):
    n = 1 << 20
    out, st = opt.run(mlir_gen.config4_text(n, prerounded), "canonicalize")
    t1, t2, e1, e2, si, fp, c1, c2 = consts_returned(out)
    c = W.config4(n, prerounded)
    assert c1.name == "arith.cmpf" and c2.name == "arith.cmpf"      # dense cmpf never folds
    want_si = oracle.convert("fptosi", "f32", "i32", c["inrange"]).out
    assert np.array_equal(full(si, n), want_si.astype(np.uint64))
    want_fp = oracle.convert("sitofp", "i32", "f32", c["ints"]).out
    assert np.array_equal(full(fp, n), want_fp.astype(np.uint64))
    tb = oracle.convert("truncf", "f32", "bf16", c["x"])
    assert (t1.name == "arith.constant") == tb.folded
    if prerounded:
        assert np.array_equal(full(t1, n), tb.out.astype(np.uint64))
        # extf(truncf(x)) folds back to x
        assert np.array_equal(full(e1, n), c["x"].astype(np.uint64))
    else:
        assert t1.name == "arith.truncf" and e1.name == "arith.extf"


def test_config5_layerwise_pipeline(oracle):
    funcs, side, ws = 24, 64, 512
    out, st = opt.run(mlir_gen.config5_text(funcs, side, ws), mlir_gen.LAYERWISE)
    fs = parse_funcs(out)
    for i in range(funcs):
        a, b = W.config5_func(i, side)
        t1 = oracle.binary("addf", "f32", a, b).out
        t2 = oracle.binary("mulf", "f32", t1, a).out
        r = oracle.reciprocal("f32", t2).out
        f = fs[f"f{i}"]
        d = f.defs.get(f.ret.operands[0])
        assert d.name == "tosa.const", f"f{i}"
        assert np.array_equal(full(d, side * side), r.astype(np.uint64)), f"f{i}"
        assert [o.name for o in f.ops] == ["tosa.const", "func.return"]
    w = W.config5_weight(ws)
    f = fs["weights"]
    d = f.defs.get(f.ret.operands[0])
    assert d.name == "tosa.const"
    assert np.array_equal(full(d, ws * ws), w.reshape(ws, ws).T.reshape(-1).astype(np.uint64))


def test_canonicalize_alone_leaves_non_splat_tosa_folds():
    # The reference's canonicalize folds tosa.reciprocal / transpose only for
    # splat inputs: with non-splat constants the ops stay.
    out, st = opt.run(mlir_gen.config5_text(2, 8, 64), "builtin.module(func.func(canonicalize))")
    fs = parse_funcs(out)
    assert any(o.name == "tosa.reciprocal" for o in fs["f0"].ops)
    assert any(o.name == "tosa.transpose" for o in fs["weights"].ops)


def _gpus():
    import torch
    return torch.cuda.device_count()


@pytest.mark.parametrize("n", [2, 4, 8])
def test_config5_sharded_over_gpus_prints_the_same(n):
    # Functions are placed on the GPUs by constant bytes; the printed module
    # must not depend on how many GPUs folded it.
    if _gpus() < n:
        pytest.skip(f"needs {n} GPUs")
    text = mlir_gen.config5_text(64, 64, 512)
    one, s1 = opt.run(text, mlir_gen.LAYERWISE, n_gpus=1)
    many, sn = opt.run(text, mlir_gen.LAYERWISE, n_gpus=n)
    assert many == one
    assert sn["folds"] == s1["folds"] == 3 * 64 + 1


def _hex(a):
    return a.tobytes().hex().upper()


def test_more_arith_folds_through_canonicalize(oracle):
    # The remaining elementwise folds at a size where every one of them is
    # a device fold, through the whole driver, against the oracle.
    from test_gpu_parity import rbits
    n = 1 << 18
    T32, Ti1, Ti8, Ti64 = f"tensor<{n}xi32>", f"tensor<{n}xi1>", f"tensor<{n}xi8>", f"tensor<{n}xindex>"
    F = f"tensor<{n}xf32>"
    x, y = rbits("i32", n, 1), rbits("i32", n, 2)
    y = np.where(y == 0, np.uint32(5), y)
    y = np.where((x == 0x80000000) | (y == 0x80000000), np.uint32(7), y)  # keep ceildivsi folding
    x = np.where(x == 0x80000000, np.uint32(9), x)
    fa, fb = rbits("f32", n, 3), rbits("f32", n, 4)
    c = rbits("i1", n, 5)
    lines = [
        f'    %x = "arith.constant"() <{{value = dense<"0x{_hex(x)}"> : {T32}}}> : () -> {T32}',
        f'    %y = "arith.constant"() <{{value = dense<"0x{_hex(y)}"> : {T32}}}> : () -> {T32}',
        f'    %fa = "arith.constant"() <{{value = dense<"0x{_hex(fa)}"> : {F}}}> : () -> {F}',
        f'    %fb = "arith.constant"() <{{value = dense<"0x{_hex(fb)}"> : {F}}}> : () -> {F}',
        f'    %c = "arith.constant"() <{{value = dense<[{", ".join("true" if v else "false" for v in c)}]> : {Ti1}}}> '
        f': () -> {Ti1}',
        f'    %0 = "arith.floordivsi"(%x, %y) : ({T32}, {T32}) -> {T32}',
        f'    %1 = "arith.ceildivsi"(%x, %y) : ({T32}, {T32}) -> {T32}',
        f'    %2 = "arith.ceildivui"(%x, %y) : ({T32}, {T32}) -> {T32}',
        f'    %3 = "arith.remf"(%fa, %fb) <{{fastmath = #arith.fastmath<none>}}> : ({F}, {F}) -> {F}',
        f'    %4 = "arith.negf"(%fa) <{{fastmath = #arith.fastmath<none>}}> : ({F}) -> {F}',
        f'    %5 = "arith.flush_denormals"(%fb) <{{fastmath = #arith.fastmath<none>}}> : ({F}) -> {F}',
        f'    %6 = "arith.trunci"(%x) <{{overflowFlags = #arith.overflow<none>}}> : ({T32}) -> {Ti8}',
        f'    %7 = "arith.extsi"(%6) : ({Ti8}) -> {T32}',
        f'    %8 = "arith.index_cast"(%y) : ({T32}) -> {Ti64}',
        f'    %9 = "arith.bitcast"(%fa) : ({F}) -> {T32}',
        f'    %10 = "arith.select"(%c, %x, %y) : ({Ti1}, {T32}, {T32}) -> {T32}',
    ]
    rets = [f"%{i}" for i in range(11)]
    tys = [T32, T32, T32, F, F, F, Ti8, T32, Ti64, T32, T32]
    text = ('"builtin.module"() ({\n'
            f'  "func.func"() <{{function_type = () -> ({", ".join(tys)}), sym_name = "main"}}> ({{\n'
            + "\n".join(lines) + f'\n    "func.return"({", ".join(rets)}) : ({", ".join(tys)}) -> ()\n'
            '  }) : () -> ()\n}) : () -> ()\n')
    out, st = opt.run(text, "canonicalize")
    got = consts_returned(out)
    assert all(d.name == "arith.constant" for d in got), [d.name for d in got]
    t6 = oracle.convert("trunci", "i32", "i8", x).out
    want = [oracle.binary("floordivsi", "i32", x, y).out, oracle.binary("ceildivsi", "i32", x, y).out,
            oracle.binary("ceildivui", "i32", x, y).out, oracle.binary("remf", "f32", fa, fb).out,
            oracle.convert("negf", "f32", "f32", fa).out, oracle.convert("flush_denormals", "f32", "f32", fb).out,
            t6, oracle.convert("extsi", "i8", "i32", t6).out, oracle.convert("extsi", "i32", "i64", y).out,
            fa, oracle.select(c, x, y).out]
    for i, (d, w) in enumerate(zip(got, want)):
        assert np.array_equal(full(d, n), w.astype(np.uint64)), i


def test_pinned_text_gives_the_same_module():
    # From page-locked text the driver copies runs of literals straight
    # into HBM and decodes them at whatever alignment they have; the
    # printed module must equal the one from ordinary memory.
    text = mlir_gen.config5_text(40, 64, 256) + " " * 5     # odd sizes shift every literal's alignment
    a, sa = opt.run(text, mlir_gen.LAYERWISE)
    b, sb = opt.run(opt.pinned_text(text), mlir_gen.LAYERWISE)
    assert a == b and sa["folds"] == sb["folds"] == 3 * 40 + 1
    t2 = mlir_gen.config2_text(512)
    assert opt.run(t2, "canonicalize")[0] == opt.run(opt.pinned_text(t2), "canonicalize")[0]


def test_equal_folded_constants_are_deduplicated(oracle):
    # Two folds with bitwise-equal results (addf is commutative on these
    # NaN-free operands) and a parsed constant with the same bytes become one
    # constant, as the constant folder's Attribute-equality dedup makes them
    # (src/rewrite.rs:689-728).
    n = 1 << 16
    c = W.config2(256)
    a, b = c["A"][:n], c["B"][:n]
    s = oracle.binary("addf", "f32", a, b).out
    T = f"tensor<{n}xf32>"
    h = lambda x: np.ascontiguousarray(x).view(np.uint32).tobytes().hex().upper()
    body = "\n".join([
        f'    %a = "arith.constant"() <{{value = dense<"0x{h(a)}"> : {T}}}> : () -> {T}',
        f'    %b = "arith.constant"() <{{value = dense<"0x{h(b)}"> : {T}}}> : () -> {T}',
        f'    %s = "arith.constant"() <{{value = dense<"0x{h(s)}"> : {T}}}> : () -> {T}',
        f'    %0 = "arith.addf"(%a, %b) <{{fastmath = #arith.fastmath<none>}}> : ({T}, {T}) -> {T}',
        f'    %1 = "arith.addf"(%b, %a) <{{fastmath = #arith.fastmath<none>}}> : ({T}, {T}) -> {T}'])
    text = ('"builtin.module"() ({\n'
            f'  "func.func"() <{{function_type = () -> ({T}, {T}, {T}), sym_name = "main"}}> ({{\n{body}\n'
            f'    "func.return"(%0, %1, %s) : ({T}, {T}, {T}) -> ()\n  }}) : () -> ()\n}}) : () -> ()\n')
    out, st = opt.run(text, "canonicalize")
    f = parse_funcs(out)["main"]
    assert len(set(f.ret.operands)) == 1, out[-300:]
    assert [o.name for o in f.ops] == ["arith.constant", "func.return"]
    d = f.defs[f.ret.operands[0]]
    assert np.array_equal(np.array(d.const.bits, dtype=np.uint64), s.astype(np.uint64))


def test_math_folds_through_canonicalize(oracle):
    # The exact math folds at a size where every one is a device fold,
    # through the whole driver, against the oracle; a transcendental op
    # stays in place.
    from test_gpu_parity import rbits
    n = 1 << 18
    F, I = f"tensor<{n}xf32>", f"tensor<{n}xi32>"
    fa = rbits("f32", n, 11) & np.uint32(0x7FFFFFFF)   # non-negative: sqrt / rsqrt fold
    fb = rbits("f32", n, 12)
    x, y = rbits("i32", n, 13), (np.arange(n) % 37).astype(np.uint32)
    fm = "<{fastmath = #arith.fastmath<none>}>"
    ops = [("absf", "fb"), ("ceil", "fb"), ("floor", "fb"), ("roundeven", "fb"), ("round", "fb"),
           ("trunc", "fb"), ("sqrt", "fa"), ("rsqrt", "fa")]
    lines = [
        f'    %fa = "arith.constant"() <{{value = dense<"0x{_hex(fa)}"> : {F}}}> : () -> {F}',
        f'    %fb = "arith.constant"() <{{value = dense<"0x{_hex(fb)}"> : {F}}}> : () -> {F}',
        f'    %x = "arith.constant"() <{{value = dense<"0x{_hex(x)}"> : {I}}}> : () -> {I}',
        f'    %y = "arith.constant"() <{{value = dense<"0x{_hex(y)}"> : {I}}}> : () -> {I}',
    ]
    for i, (op, v) in enumerate(ops):
        lines.append(f'    %{i} = "math.{op}"(%{v}) {fm} : ({F}) -> {F}')
    k = len(ops)
    lines += [f'    %{k} = "math.copysign"(%fa, %fb) {fm} : ({F}, {F}) -> {F}',
              f'    %{k + 1} = "math.ctlz"(%x) : ({I}) -> {I}',
              f'    %{k + 2} = "math.absi"(%x) : ({I}) -> {I}',
              f'    %{k + 3} = "math.ipowi"(%x, %y) : ({I}, {I}) -> {I}',
              f'    %{k + 4} = "math.exp"(%fa) {fm} : ({F}) -> {F}']
    tys = [F] * (k + 1) + [I] * 3 + [F]
    rets = [f"%{i}" for i in range(k + 5)]
    text = ('"builtin.module"() ({\n'
            f'  "func.func"() <{{function_type = () -> ({", ".join(tys)}), sym_name = "main"}}> ({{\n'
            + "\n".join(lines) + f'\n    "func.return"({", ".join(rets)}) : ({", ".join(tys)}) -> ()\n'
            '  }) : () -> ()\n}) : () -> ()\n')
    out, st = opt.run(text, "canonicalize")
    got = consts_returned(out)
    assert [d.name for d in got] == ["arith.constant"] * (k + 4) + ["math.exp"]
    want = [oracle.convert(op, "f32", "f32", fa if v == "fa" else fb).out for op, v in ops]
    want += [oracle.binary("copysign", "f32", fa, fb).out, oracle.convert("ctlz", "i32", "i32", x).out,
             oracle.convert("absi", "i32", "i32", x).out, oracle.binary("ipowi", "i32", x, y).out]
    for i, (d, w) in enumerate(zip(got, want)):
        assert np.array_equal(full(d, n), w.astype(np.uint64)), i


def _ranges_module():
    # Constants of 2^19 elements: a float whose first half is all 1.0 (so a
    # result range comes back as one element), one of all-equal values
    # written out in full (a result that is a splat as a whole), an all-zero
    # literal (addf gives back the first operand, which deduplicates against
    # it), and two i32 constants for a two-result fold and a refusal.
    rng = np.random.default_rng(7)
    n = 1 << 19
    F, I = f"tensor<{n}xf32>", f"tensor<{n}xi32>"
    a = np.concatenate([np.full(n // 2, 1.0, np.float32), rng.standard_normal(n // 2).astype(np.float32)])
    c = np.full(n, 2.0, np.float32)
    z = np.zeros(n, np.float32)
    x = rng.integers(0, 1 << 32, n, dtype=np.uint64).astype(np.uint32)
    y = rng.integers(1, 1 << 31, n, dtype=np.uint64).astype(np.uint32)
    y0 = y.copy()
    y0[n - 5] = 0                                       # divsi refuses in the last range
    fm = "<{fastmath = #arith.fastmath<none>}>"
    lines = [
        f'    %a = "arith.constant"() <{{value = dense<"0x{_hex(a.view(np.uint32))}"> : {F}}}> : () -> {F}',
        f'    %c = "arith.constant"() <{{value = dense<"0x{_hex(c.view(np.uint32))}"> : {F}}}> : () -> {F}',
        f'    %z = "arith.constant"() <{{value = dense<"0x{_hex(z.view(np.uint32))}"> : {F}}}> : () -> {F}',
        f'    %x = "arith.constant"() <{{value = dense<"0x{_hex(x)}"> : {I}}}> : () -> {I}',
        f'    %y = "arith.constant"() <{{value = dense<"0x{_hex(y)}"> : {I}}}> : () -> {I}',
        f'    %y0 = "arith.constant"() <{{value = dense<"0x{_hex(y0)}"> : {I}}}> : () -> {I}',
        f'    %s = "arith.constant"() <{{value = dense<3.000000e+00> : {F}}}> : () -> {F}',
        f'    %0 = "arith.mulf"(%a, %s) {fm} : ({F}, {F}) -> {F}',
        f'    %1 = "arith.addf"(%c, %c) {fm} : ({F}, {F}) -> {F}',
        f'    %2 = "arith.addf"(%a, %z) {fm} : ({F}, {F}) -> {F}',
        f'    %3:2 = "arith.addui_extended"(%x, %y) : ({I}, {I}) -> ({I}, tensor<{n}xi1>)',
        f'    %4 = "arith.divsi"(%x, %y0) : ({I}, {I}) -> {I}',
        f'    %5 = "arith.subf"(%0, %a) {fm} : ({F}, {F}) -> {F}',
    ]
    tys = [F, F, F, I, f"tensor<{n}xi1>", I, F]
    rets = ["%0", "%1", "%2", "%3#0", "%3#1", "%4", "%5"]
    return ('"builtin.module"() ({\n'
            f'  "func.func"() <{{function_type = () -> ({", ".join(tys)}), sym_name = "main"}}> ({{\n'
            + "\n".join(lines) + f'\n    "func.return"({", ".join(rets)}) : ({", ".join(tys)}) -> ()\n'
            '  }) : () -> ()\n}) : () -> ()\n')


@pytest.mark.parametrize("gpus,ranges", [(1, 2), (1, 3), (2, 1), (4, 1), (8, 1), (2, 3)])
def test_canonicalize_by_element_ranges_prints_the_same(gpus, ranges, monkeypatch):
    # Bare canonicalize over several engines cuts large constants into
    # element ranges; the printed module must not depend on it: the same
    # folds, refusals, splat results and deduplications as one engine.
    if _gpus() < gpus:
        pytest.skip(f"needs {gpus} GPUs")
    texts = [_ranges_module(), mlir_gen.config2_text(1024), mlir_gen.config3_text("i32", 1024, 512),
             mlir_gen.config4_text(1 << 19, prerounded=True)]
    want = [opt.run(t, "canonicalize", n_gpus=1) for t in texts]
    monkeypatch.setenv("DCF_OPT_RANGES_PER_GPU", str(ranges))
    for t, (one, s1) in zip(texts, want):
        many, sn = opt.run(t, "canonicalize", n_gpus=gpus)
        assert many == one
        assert (sn["folds"], sn["refused"]) == (s1["folds"], s1["refused"])
    out = want[0][0]
    f = parse_funcs(out)["main"]
    d = [f.defs.get(v) for v in f.ret.operands]
    assert d[1].const.splat and d[5].name == "arith.divsi"


def test_engines_sharing_a_gpu_batch_small_folds_safely(monkeypatch, oracle):
    # Ten independent addf folds of 2^18-element constants: split into three
    # element ranges on one GPU, each of the three engines has ten small
    # folds of one kind in the same round and sends them through the
    # library's allocation-free batch entry point from its own thread at the
    # same time.  The printed module must equal the one-engine module, and
    # every folded constant the oracle's sum.
    n, k = 1 << 18, 10
    F = f"tensor<{n}xf32>"
    fm = "<{fastmath = #arith.fastmath<none>}>"
    rng = np.random.default_rng(11)
    vals = [rng.standard_normal(n).astype(np.float32) for _ in range(2 * k)]
    lines = [f'    %c{i} = "arith.constant"() <{{value = dense<"0x{_hex(v.view(np.uint32))}"> : {F}}}> : () -> {F}'
             for i, v in enumerate(vals)]
    lines += [f'    %{i} = "arith.addf"(%c{2 * i}, %c{2 * i + 1}) {fm} : ({F}, {F}) -> {F}' for i in range(k)]
    tys = ", ".join([F] * k)
    text = ('"builtin.module"() ({\n'
            f'  "func.func"() <{{function_type = () -> ({tys}), sym_name = "main"}}> ({{\n'
            + "\n".join(lines) + f'\n    "func.return"({", ".join(f"%{i}" for i in range(k))}) : ({tys}) -> ()\n'
            '  }) : () -> ()\n}) : () -> ()\n')
    one, s1 = opt.run(text, "canonicalize", n_gpus=1)
    monkeypatch.setenv("DCF_OPT_RANGES_PER_GPU", "3")
    for _ in range(3):
        many, sn = opt.run(text, "canonicalize", n_gpus=1)
        assert many == one
        assert sn["folds"] == s1["folds"] == k
    for i, d in enumerate(consts_returned(one)):
        want = oracle.binary("addf", "f32", vals[2 * i], vals[2 * i + 1]).out
        assert np.array_equal(full(d, n), want.astype(np.uint64)), i


def _resource_module():
    # Constants whose values are dense_resource blobs, as operands of every
    # kind of fold the two passes run: arith binary and cast folds under
    # canonicalize, tosa.reciprocal and tosa.transpose under the layerwise
    # pass.  The reference reads a resource's bytes only when lowering to
    # SPIR-V (resource_const, src/ir.rs:662-696, called only from
    # src/patterns/arith/to_spirv.rs:215), so its folds see no constant
    # value and nothing folds; the blobs stay as they are.
    F4, B4 = "tensor<4xf32>", "tensor<2x2xbf16>"
    fm = "<{fastmath = #arith.fastmath<none>}>"
    body = ('"builtin.module"() ({\n'
            f'  "func.func"() <{{function_type = () -> ({F4}, tensor<4xbf16>), sym_name = "arith"}}> ({{\n'
            f'    %0 = "arith.constant"() <{{value = dense_resource<blob_a> : {F4}}}> : () -> {F4}\n'
            f'    %1 = "arith.constant"() <{{value = dense<[1.000000e+00, 2.000000e+00, 3.000000e+00, 4.000000e+00]> : {F4}}}> : () -> {F4}\n'
            f'    %2 = "arith.addf"(%0, %1) {fm} : ({F4}, {F4}) -> {F4}\n'
            f'    %3 = "arith.truncf"(%0) : ({F4}) -> tensor<4xbf16>\n'
            f'    "func.return"(%2, %3) : ({F4}, tensor<4xbf16>) -> ()\n'
            '  }) : () -> ()\n'
            f'  "func.func"() <{{function_type = () -> ({B4}, {B4}), sym_name = "tosa"}}> ({{\n'
            f'    %0 = "tosa.const"() <{{values = dense_resource<blob_w> : {B4}}}> : () -> {B4}\n'
            f'    %1 = "tosa.transpose"(%0) <{{perms = array<i32: 1, 0>}}> : ({B4}) -> {B4}\n'
            f'    %2 = "tosa.reciprocal"(%0) : ({B4}) -> {B4}\n'
            f'    "func.return"(%1, %2) : ({B4}, {B4}) -> ()\n'
            '  }) : () -> ()\n'
            '}) : () -> ()\n')
    meta = ('\n{-#\n  dialect_resources: {\n    builtin: {\n'
            '      blob_a: "0x040000000000803F000000400000404000008040",\n'
            '      blob_w: "0x02000000803F0040403F8040"\n'
            '    }\n  }\n#-}\n')
    return body + meta


def check_resource_operands_stay(n_gpus):
    text = _resource_module()
    for pipe in ("canonicalize", mlir_gen.LAYERWISE):
        out, st = opt.run(text, pipe, n_gpus=n_gpus)
        fs = parse_funcs(out)
        assert [o.name for o in fs["arith"].ops] == ["arith.constant", "arith.constant", "arith.addf",
                                                     "arith.truncf", "func.return"], (pipe, out)
        assert [o.name for o in fs["tosa"].ops] == ["tosa.const", "tosa.transpose", "tosa.reciprocal",
                                                    "func.return"], (pipe, out)
        assert st["folds"] == 0
        assert 'blob_a: "0x040000000000803F000000400000404000008040"' in out
        assert 'blob_w: "0x02000000803F0040403F8040"' in out
        assert out.count("dense_resource<blob_a>") == 1 and out.count("dense_resource<blob_w>") == 1


def test_dense_resource_operands_are_not_folded():
    check_resource_operands_stay(1)


@pytest.mark.parametrize("memory", ["pageable", "pinned"])
@pytest.mark.parametrize("n", [1 << 12, 1 << 21])
def test_literals_with_a_bad_hex_digit_are_rejected(memory, n):
    # A literal body with a character that is not a hex digit is an error,
    # whichever decoder reads it: the host threads (pageable text, and small
    # page-locked literals at one GPU) or the device (large page-locked
    # literals); lower-case digits are accepted.
    T = f"tensor<{n}xf32>"
    good = np.arange(n, dtype=np.float32)
    h = _hex(good.view(np.uint32))
    fm = "<{fastmath = #arith.fastmath<none>}>"

    def module(body):
        return ('"builtin.module"() ({\n'
                f'  "func.func"() <{{function_type = () -> {T}, sym_name = "main"}}> ({{\n'
                f'    %a = "arith.constant"() <{{value = dense<"0x{body}"> : {T}}}> : () -> {T}\n'
                f'    %b = "arith.constant"() <{{value = dense<"0x{h}"> : {T}}}> : () -> {T}\n'
                f'    %0 = "arith.addf"(%a, %b) {fm} : ({T}, {T}) -> {T}\n'
                f'    "func.return"(%0) : ({T}) -> ()\n  }}) : () -> ()\n}}) : () -> ()\n')

    src = (lambda t: t) if memory == "pageable" else opt.pinned_text
    out, st = opt.run(src(module(h.lower())), "canonicalize")
    (d,) = consts_returned(out)
    assert st["folds"] == 1 and np.array_equal(full(d, n), (good + good).view(np.uint32).astype(np.uint64))
    for pos in (0, len(h) // 2 + 1, len(h) - 1):
        bad = h[:pos] + "G" + h[pos + 1:]
        with pytest.raises(opt.OptError) as e:
            opt.run(src(module(bad)), "canonicalize")
        assert "hex" in str(e.value)
