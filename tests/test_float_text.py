"""The printed text of float elements (include/dcfold_opt.h:
dcf_opt_print_element), on the CPU.

1. Every float literal of the reference's fixtures (mlir-opt 23.1.5's
   printing, harvested into tests/golden/float_literals.json) is printed
   back from its bits exactly as the fixture spells it.
2. Random bit patterns of every float type against an independent Python
   restatement of the same rule (exact integer arithmetic, and exact
   rational parse-back with round-to-nearest-even): six-digit scientific
   form when it parses back to the same bits, else APFloat's default
   round-trip decimal when it has a '.', else the hex bit pattern.
"""
import ctypes
import json
import os

import numpy as np
import pytest

from mlir_text import FLOATS, float_literal_bits
from mlirpass_b200 import DTYPES, opt

HERE = os.path.dirname(os.path.abspath(__file__))


def printed(dtype, bits):
    L = opt.lib()
    L.dcf_opt_print_element.argtypes = [ctypes.c_int, ctypes.c_ulonglong, ctypes.c_char_p, ctypes.c_size_t]
    buf = ctypes.create_string_buffer(128)
    n = L.dcf_opt_print_element(DTYPES[dtype], bits, buf, 128)
    assert n >= 0
    return buf.value.decode()


def test_fixture_float_literals_print_back_exactly():
    cases = json.load(open(os.path.join(HERE, "golden", "float_literals.json")))["cases"]
    assert len(cases) >= 150
    bad = [(c["dtype"], c["text"], printed(c["dtype"], int(c["bits"], 16))) for c in cases
           if printed(c["dtype"], int(c["bits"], 16)) != c["text"]]
    assert not bad, bad[:10]


# ---- an independent restatement (Python integers) -------------------------

def _to_string(neg, sig, exp, precision, fmt_prec, max_pad, trunc_zero):
    out = "-" if neg else ""
    if sig == 0:
        if not max_pad:
            return out + ("0.0E+0" if trunc_zero else "0.0" + "0" * max(0, fmt_prec - 1) + "e+00")
        return out + "0"
    if not fmt_prec:
        fmt_prec = 2 + precision * 59 // 196
    while sig % 2 == 0:
        sig //= 2
        exp += 1
    if exp > 0:
        sig <<= exp
        exp = 0
    elif exp < 0:
        sig *= 5 ** (-exp)
    need = (fmt_prec * 196 + 58) // 59
    if sig.bit_length() > need:
        tens = (sig.bit_length() - need) * 59 // 196
        if tens:
            exp += tens
            sig //= 10 ** tens
    digits = str(sig)                       # most significant first
    stripped = digits.rstrip("0")
    exp += len(digits) - len(stripped)
    digits = stripped
    if len(digits) > fmt_prec:
        cut = len(digits) - fmt_prec        # digits to drop from the end
        head, tail = digits[:fmt_prec], digits[fmt_prec:]
        exp += cut
        if tail[0] >= "5":
            v = int(head) + 1
            if len(str(v)) > len(head):     # carried through every digit
                head = "1"
                exp += len(str(v)) - 1
            else:
                head = str(v).rjust(len(head), "0")
        s2 = head.rstrip("0")
        exp += len(head) - len(s2)
        digits = s2
    nd = len(digits)
    if not max_pad:
        sci = True
    elif exp >= 0:
        sci = exp > max_pad or nd + exp > fmt_prec
    else:
        msd = exp + nd - 1
        sci = msd < 0 and -msd > max_pad
    if sci:
        e = exp + nd - 1
        frac = digits[1:] if not (nd == 1 and trunc_zero) else "0"
        if not trunc_zero and fmt_prec > nd - 1:
            frac += "0" * (fmt_prec - nd + 1)
        es = str(abs(e))
        if not trunc_zero and len(es) < 2:
            es = "0" + es
        return out + digits[0] + "." + frac + ("E" if trunc_zero else "e") + ("+" if e >= 0 else "-") + es
    if exp >= 0:
        return out + digits + "0" * exp
    whole = exp + nd
    if whole > 0:
        return out + digits[:whole] + "." + digits[whole:]
    return out + "0." + "0" * (-whole) + digits


def reference_text(dtype, bits):
    E, M, _ = FLOATS[dtype]
    neg = (bits >> (E + M)) & 1
    ef, m = (bits >> M) & ((1 << E) - 1), bits & ((1 << M) - 1)
    if ef != (1 << E) - 1:
        bias = (1 << (E - 1)) - 1
        sig = (m | (1 << M)) if ef else m
        exp = (ef if ef else 1) - bias - M
        s = _to_string(neg, sig, exp, M + 1, 6, 0, False)
        if float_literal_bits(s, dtype) == bits:
            return s
        s = _to_string(neg, sig, exp, M + 1, 0, 3, True)
        if "." in s:
            return s
    return "0x%X" % bits


@pytest.mark.parametrize("dtype", ["f32", "f64", "f16", "bf16", "f8E5M2", "f8E4M3", "f8E3M4"])
def test_random_bit_patterns_match_the_restatement(dtype):
    E, M, nbytes = FLOATS[dtype]
    rng = np.random.default_rng(E * 100 + M)
    width = 1 + E + M
    n = 1500 if width > 16 else (1 << width if width <= 8 else 3000)
    if width <= 8:
        pats = range(n)
    else:
        pats = [int(x) for x in rng.integers(0, 1 << min(width, 63), n, dtype=np.uint64)]
        if width == 64:
            pats = [p | (int(rng.integers(0, 2)) << 63) for p in pats]
        # values whose six-digit form does not round-trip, and extremes
        pats += [(1 << (M + 4)) + k for k in range(1, 40)] + [1, 2, (1 << M) - 1, (1 << M), ((1 << E) - 2) << M | ((1 << M) - 1)]
    bad = []
    for b in pats:
        want = reference_text(dtype, b)
        got = printed(dtype, b)
        if got != want:
            bad.append((hex(b), want, got))
    assert not bad, bad[:10]


def test_folded_constants_print_as_the_fixtures():
    # Every folded golden case's expected constant, written in hex form,
    # goes through the printer (host only), which prints constants from
    # their values as the reference does after re-reading them at import:
    # the attribute text must be exactly what mlir-opt printed in the
    # fixture.
    from golden_cases import CANON, SIZE, STORAGE, load_cases
    from mlir_text import parse_funcs

    def ty_text(o):
        if o["shape"] is None:
            return o["dtype"]
        return f'{o["kind"]}<{"x".join(str(d) for d in o["shape"])}x{o["dtype"]}>'

    n = 0
    for c in load_cases():
        exp = c["expected"]
        if exp["status"] != "folded":
            continue
        res = c["result"]
        ty = ty_text(res)
        dt = CANON.get(exp["dtype"], exp["dtype"])
        bits = [int(b, 16) for b in exp["bits"]]
        isf = dt.startswith("f") or dt == "bf16"
        if res["shape"] is None:
            lit = ("true" if bits[0] else "false") if dt == "i1" else \
                (("0x%0*X" % (2 * SIZE[dt], bits[0])) if isf else str(bits[0])) + f" : {ty}"
        elif dt == "i1":
            lit = "dense<" + ("true" if bits[0] else "false") + f"> : {ty}" if exp["splat"] else \
                "dense<[" + ", ".join("true" if b else "false" for b in bits) + f"]> : {ty}"
        else:
            vals = bits[:1] if exp["splat"] else bits
            raw = np.array(vals, dtype=STORAGE[SIZE[dt]]).tobytes().hex().upper()
            lit = f'dense<"0x{raw}"> : {ty}'
        op, key = ("tosa.const", "values") if c["op"].startswith("tosa.") else ("arith.constant", "value")
        text = ('"builtin.module"() ({\n'
                f'  "func.func"() <{{function_type = () -> {ty}, sym_name = "t"}}> ({{\n'
                f'    %0 = "{op}"() <{{{key} = {lit}}}> : () -> {ty}\n'
                f'    "func.return"(%0) : ({ty}) -> ()\n  }}) : () -> ()\n}}) : () -> ()\n')
        out, _ = opt.run(text, "builtin.module(func.func())", n_gpus=0)
        f = parse_funcs(out)["t"]
        d = f.defs[f.ret.operands[0]]
        assert d.prop_map[key] == exp["text"], (c["func"], d.prop_map[key], exp["text"])
        n += 1
    assert n >= 165


def test_print_element_rejects_other_types_and_short_buffers():
    L = opt.lib()
    L.dcf_opt_print_element.argtypes = [ctypes.c_int, ctypes.c_ulonglong, ctypes.c_char_p, ctypes.c_size_t]
    buf = ctypes.create_string_buffer(4)
    assert L.dcf_opt_print_element(99, 0, buf, 4) < 0
    assert L.dcf_opt_print_element(DTYPES["f32"], 0x3F800000, buf, 4) < 0     # "1.000000e+00" needs 13 bytes
    assert L.dcf_opt_print_element(DTYPES["i8"], 0xFF, buf, 4) == 2 and buf.value == b"-1"
    assert printed("i1", 1) == "true" and printed("i64", (1 << 64) - 5) == "-5"
