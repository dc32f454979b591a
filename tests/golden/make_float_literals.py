"""Harvest the printed float literals of the reference's fixtures.

Run here (the container that has the reference checkout):

    python tests/golden/make_float_literals.py /path/to/mlirpass

Every `tests/fixtures/*.mlir` file of mlirpass is mlir-opt 23.1.5's printed
output (or input as mlir-opt printed it).  For every arith.constant /
tosa.const whose element type is a float type, each element literal (a
scalar value, or each element of a `dense<...>` list or splat; hex-body
literals excluded) is one case: the literal's exact text and the element
bits it denotes (read with correct rounding to nearest even).  The printer
must produce exactly that text from those bits.

Output: tests/golden/float_literals.json (committed).  The tests read only
that file, never the reference.
"""
from __future__ import annotations

import json
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
from mlir_text import FLOATS, float_literal_bits, flatten_list, parse_funcs, parse_type  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "float_literals.json")


def literals(text: str):
    for chunk in text.split("// -----"):
        for f in parse_funcs(chunk).values():
            for op in f.ops:
                if op.name not in ("arith.constant", "tosa.const") or len(op.out_types) != 1:
                    continue
                v = op.prop_map.get("value" if op.name == "arith.constant" else "values")
                ty = parse_type(op.out_types[0])
                if v is None or ty is None or ty.elem not in FLOATS:
                    continue
                lit = v.rsplit(" : ", 1)[0] if " : " in v else v
                if lit.startswith("dense<") and lit.endswith(">"):
                    body = lit[len("dense<"):-1].strip()
                    if body.startswith('"') or body.startswith("("):
                        continue
                    toks = flatten_list(body)
                else:
                    toks = [lit]
                for t in toks:
                    yield ty.elem, t.strip()


def main():
    if len(sys.argv) != 2:
        sys.exit("usage: make_float_literals.py <path of the mlirpass checkout>")
    fix = os.path.join(sys.argv[1], "tests", "fixtures")
    seen = {}
    for name in sorted(os.listdir(fix)):
        if not name.endswith(".mlir"):
            continue
        with open(os.path.join(fix, name)) as fh:
            text = fh.read()
        for dt, tok in literals(text):
            if (dt, tok) in seen:
                continue
            try:
                bits = float_literal_bits(tok, dt)
            except (ValueError, ZeroDivisionError):
                continue
            seen[(dt, tok)] = {"dtype": dt, "text": tok, "bits": format(bits, "x"), "fixture": name}
    cases = sorted(seen.values(), key=lambda c: (c["dtype"], c["text"]))
    with open(OUT, "w") as fh:
        json.dump({"source": "mlirpass tests/fixtures (mlir-opt 23.1.5 outputs)",
                   "generator": "tests/golden/make_float_literals.py", "cases": cases}, fh, indent=0)
    by = {}
    for c in cases:
        by[c["dtype"]] = by.get(c["dtype"], 0) + 1
    print(len(cases), "literals", json.dumps(by, sort_keys=True))


if __name__ == "__main__":
    main()
