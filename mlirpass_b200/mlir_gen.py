"""MLIR text (generic form, as mlir-opt prints it) for the five fold
configurations: dense constants as `dense<"0x…">` hex literals (uppercase,
little-endian raw bytes), one function per unit."""
from __future__ import annotations

import numpy as np

from . import workloads as W

ELEM = {np.dtype(np.float32): "f32", np.dtype(np.uint16): "bf16"}


def hexlit(a: np.ndarray) -> str:
    return '"0x' + np.ascontiguousarray(a).tobytes().hex().upper() + '"'


class Func:
    def __init__(self, name: str):
        self.name = name
        self.lines: list[str] = []
        self.n = 0
        self.types: dict[str, str] = {}

    def const(self, arr: np.ndarray, ty: str, op: str = "arith.constant") -> str:
        v = f"%{self.n}"
        self.n += 1
        key = "values" if op == "tosa.const" else "value"
        self.lines.append(f'    {v} = "{op}"() <{{{key} = dense<{hexlit(arr)}> : {ty}}}> : () -> {ty}')
        self.types[v] = ty
        return v

    def op(self, name: str, args: list[str], out_ty: str, props: str = "") -> str:
        v = f"%{self.n}"
        self.n += 1
        ins = ", ".join(self.types[a] for a in args)
        p = f" <{{{props}}}>" if props else ""
        self.lines.append(f'    {v} = "{name}"({", ".join(args)}){p} : ({ins}) -> {out_ty}')
        self.types[v] = out_ty
        return v

    def text(self, ret: list[str]) -> str:
        rt = ", ".join(self.types[r] for r in ret)
        fty = f"() -> {rt}" if len(ret) == 1 else f"() -> ({rt})"
        body = "\n".join(self.lines)
        return (f'  "func.func"() <{{function_type = {fty}, sym_name = "{self.name}"}}> ({{\n{body}\n'
                f'    "func.return"({", ".join(ret)}) : ({rt}) -> ()\n  }}) : () -> ()')


def module(funcs: list[str]) -> str:
    return '"builtin.module"() ({\n' + "\n".join(funcs) + "\n}) : () -> ()\n"


FM = "fastmath = #arith.fastmath<none>"


def config1_text() -> str:
    d = W.config1()
    ty = "tensor<1024x1024xf32>"
    f = Func("main")
    a, b = f.const(d["A"], ty), f.const(d["B"], ty)
    r = f.op("arith.addf", [a, b], ty, FM)
    return module([f.text([r])])


def config2_text(side: int = 4096) -> str:
    d = W.config2(side)
    ty = f"tensor<{side}x{side}xf32>"
    f = Func("main")
    env = {k: f.const(d[k], ty) for k in "ABCD"}
    for op, a, b, t in W.CHAIN2:
        env[t] = f.op("arith." + op, [env[a], env[b]], ty, FM)
    return module([f.text([env["t6"]])])


def config3_text(dtype: str, rows: int = 8192, cols: int = 2048) -> str:
    d = W.config3(dtype, rows, cols)
    ty = f"tensor<{rows}x{cols}x{dtype}>"
    f = Func("main")
    X, Y, S, Xd, Yd = (f.const(d[k], ty) for k in ("X", "Y", "S", "Xd", "Yd"))
    ov = "overflowFlags = #arith.overflow<none>"
    outs = [f.op("arith." + op, [X, Y], ty, ov if op in ("addi", "muli", "subi") else "")
            for op in ("addi", "muli", "subi", "andi", "xori")]
    outs.append(f.op("arith.shli", [X, S], ty, ov))
    outs.append(f.op("arith.divsi", [Xd, Yd], ty))
    outs.append(f.op("arith.remsi", [Xd, Yd], ty))
    return module([f.text(outs)])


def config4_text(n: int = 16 * 1024 * 1024, prerounded: bool = False) -> str:
    d = W.config4(n, prerounded)
    f32, bf, h = f"tensor<{n}xf32>", f"tensor<{n}xbf16>", f"tensor<{n}xf16>"
    i32, i1 = f"tensor<{n}xi32>", f"tensor<{n}xi1>"
    f = Func("main")
    x = f.const(d["x"], f32)
    xh = f.const(d["x_f16"], f32) if prerounded else x
    t1 = f.op("arith.truncf", [x], bf)
    t2 = f.op("arith.truncf", [xh], h)
    e1 = f.op("arith.extf", [t1], f32, FM)
    e2 = f.op("arith.extf", [t2], f32, FM)
    inr = f.const(d["inrange"], f32)
    si = f.op("arith.fptosi", [inr], i32)
    ints = f.const(d["ints"], i32)
    fp = f.op("arith.sitofp", [ints], f32)
    c1 = f.op("arith.cmpf", [x, inr], i1, "fastmath = #arith.fastmath<none>, predicate = 4 : i64")
    c2 = f.op("arith.cmpf", [x, inr], i1, "fastmath = #arith.fastmath<none>, predicate = 13 : i64")
    return module([f.text([t1, t2, e1, e2, si, fp, c1, c2])])


def config5_text(funcs: int = 4096, side: int = 256, weight_side: int = 16384) -> str:
    ty = f"tensor<{side}x{side}xf32>"
    out = []
    for i in range(funcs):
        a, b = W.config5_func(i, side)
        f = Func(f"f{i}")
        ca, cb = f.const(a, ty), f.const(b, ty)
        t1 = f.op("arith.addf", [ca, cb], ty, FM)
        t2 = f.op("arith.mulf", [t1, ca], ty, FM)
        r = f.op("tosa.reciprocal", [t2], ty)
        out.append(f.text([r]))
    if weight_side:
        w = W.config5_weight(weight_side)
        wt = f"tensor<{weight_side}x{weight_side}xbf16>"
        f = Func("weights")
        c = f.const(w, wt, op="tosa.const")
        r = f.op("tosa.transpose", [c], wt, "perms = array<i32: 1, 0>")
        out.append(f.text([r]))
    return module(out)


LAYERWISE = "builtin.module(func.func(tosa-layerwise-constant-fold,canonicalize))"
