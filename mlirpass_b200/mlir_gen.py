"""MLIR text (generic form, as mlir-opt prints it) for the five fold
configurations: dense constants as `dense<"0x…">` hex literals (uppercase,
little-endian raw bytes), one function per unit.

configN_text returns a str; configN_module returns the same text as a Text
whose tobytes() builds it in one bytearray (the full-size modules are
0.5-5.4 GB, where every extra copy of a str costs seconds)."""
from __future__ import annotations

import numpy as np

from . import workloads as W

ELEM = {np.dtype(np.float32): "f32", np.dtype(np.uint16): "bf16"}


def hexlit(a: np.ndarray) -> str:
    return '"0x' + W.hex_upper(a) + '"'


class Text:
    """Module text as a list of parts: small strings, and arrays whose
    uppercase hex is written straight into the final buffer (one pass over
    the memory for literals of hundreds of MB)."""

    def __init__(self, parts=None):
        self.parts = parts or []

    def __add__(self, other):
        return Text(self.parts + (other.parts if isinstance(other, Text) else [other]))

    def __radd__(self, other):
        return Text([other] + self.parts)

    def tobytes(self) -> bytearray:
        import ctypes
        enc = [p.encode() if isinstance(p, str) else np.ascontiguousarray(p).reshape(-1).view(np.uint8)
               for p in self.parts]
        total = sum(len(e) if isinstance(e, bytes) else 2 * e.size for e in enc)
        buf = bytearray(total)
        if not total:
            return buf
        base = ctypes.addressof((ctypes.c_char * total).from_buffer(buf))
        off = 0
        for e in enc:
            if isinstance(e, bytes):
                buf[off:off + len(e)] = e
                off += len(e)
            else:
                if e.size:
                    W.gen_lib().dcg_hex_upper(e.ctypes.data, e.size, base + off)
                off += 2 * e.size
        return buf

    def __str__(self) -> str:
        return self.tobytes().decode("ascii")


class Func:
    def __init__(self, name: str):
        self.name = name
        self.lines: list = []
        self.n = 0
        self.types: dict[str, str] = {}

    def const(self, arr: np.ndarray, ty: str, op: str = "arith.constant") -> str:
        v = f"%{self.n}"
        self.n += 1
        key = "values" if op == "tosa.const" else "value"
        self.lines.append(Text([f'    {v} = "{op}"() <{{{key} = dense<"0x', arr,
                                f'"> : {ty}}}> : () -> {ty}']))
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

    def text(self, ret: list[str]) -> Text:
        rt = ", ".join(self.types[r] for r in ret)
        fty = f"() -> {rt}" if len(ret) == 1 else f"() -> ({rt})"
        parts = [f'  "func.func"() <{{function_type = {fty}, sym_name = "{self.name}"}}> ({{\n']
        for i, line in enumerate(self.lines):
            if i:
                parts.append("\n")
            parts.extend(line.parts if isinstance(line, Text) else [line])
        parts.append(f'\n    "func.return"({", ".join(ret)}) : ({rt}) -> ()\n  }}) : () -> ()')
        return Text(parts)


def module_text(funcs: list[Text]) -> Text:
    parts = ['"builtin.module"() ({\n']
    for i, f in enumerate(funcs):
        if i:
            parts.append("\n")
        parts.extend(f.parts)
    parts.append("\n}) : () -> ()\n")
    return Text(parts)


def module(funcs: list[Text]) -> str:
    return str(module_text(funcs))


FM = "fastmath = #arith.fastmath<none>"


def config1_text() -> str:
    return str(config1_module())


def config1_module() -> Text:
    d = W.config1()
    ty = "tensor<1024x1024xf32>"
    f = Func("main")
    a, b = f.const(d["A"], ty), f.const(d["B"], ty)
    r = f.op("arith.addf", [a, b], ty, FM)
    return module_text([f.text([r])])


def config2_text(side: int = 4096) -> str:
    return str(config2_module(side))


def config2_module(side: int = 4096) -> Text:
    d = W.config2(side)
    ty = f"tensor<{side}x{side}xf32>"
    f = Func("main")
    env = {k: f.const(d[k], ty) for k in "ABCD"}
    for op, a, b, t in W.CHAIN2:
        env[t] = f.op("arith." + op, [env[a], env[b]], ty, FM)
    return module_text([f.text([env["t6"]])])


def config3_text(dtype: str, rows: int = 8192, cols: int = 2048) -> str:
    return str(config3_module(dtype, rows, cols))


def config3_module(dtype: str, rows: int = 8192, cols: int = 2048) -> Text:
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
    return module_text([f.text(outs)])


def config4_text(n: int = 16 * 1024 * 1024, prerounded: bool = False) -> str:
    return str(config4_module(n, prerounded))


def config4_module(n: int = 16 * 1024 * 1024, prerounded: bool = False) -> Text:
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
    return module_text([f.text([t1, t2, e1, e2, si, fp, c1, c2])])


def config5_text(funcs: int = 4096, side: int = 256, weight_side: int = 16384) -> str:
    return str(config5_module(funcs, side, weight_side))


def config5_module(funcs: int = 4096, side: int = 256, weight_side: int = 16384) -> Text:
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
    return module_text(out)


LAYERWISE = "builtin.module(func.func(tosa-layerwise-constant-fold,canonicalize))"
