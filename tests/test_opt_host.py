"""The pass driver's host logic on the CPU (host-only mode, no GPU).

Parsing and printing of generic MLIR, the shortcut folds that ArithFolder /
Tf decide without element work (src/patterns/arith/canonicalize.rs:270-491,
src/patterns/tosa/canonicalize.rs:497-511), constant deduplication and
hoisting (src/rewrite.rs:679-729), dead-op removal, the dense-cmpf filter,
and the refusal to compute anything on the CPU.
"""
import pytest

from mlir_text import parse_funcs
from mlirpass_b200 import opt

FM = "fastmath = #arith.fastmath<none>"


def module(body: str, ret: str, ret_ty: str, name: str = "f") -> str:
    return ('"builtin.module"() ({\n'
            f'  "func.func"() <{{function_type = () -> {ret_ty}, sym_name = "{name}"}}> ({{\n{body}\n'
            f'    "func.return"({ret}) : ({ret_ty}) -> ()\n'
            '  }) : () -> ()\n}) : () -> ()\n')


def const(v, lit, ty, op="arith.constant", key="value"):
    return f'    {v} = "{op}"() <{{{key} = {lit} : {ty}}}> : () -> {ty}'


def returned(out: str, name: str = "f"):
    f = parse_funcs(out)[name]
    return f, f.defs.get(f.ret.operands[0])


def run(text, pipeline="canonicalize"):
    return opt.run(text, pipeline, n_gpus=0)[0]


T = "tensor<4xf32>"
C4 = 'dense<[1.000000e+00, 2.000000e+00, 3.000000e+00, 4.000000e+00]>'


def test_constants_only_round_trip():
    body = const("%0", 'dense<"0x0000803F000000400000404000008040">', T)
    out = run(module(body, "%0", T))
    f, d = returned(out)
    assert d.name == "arith.constant" and d.const.bits == [0x3F800000, 0x40000000, 0x40400000, 0x40800000]


@pytest.mark.parametrize("op,rhs", [("arith.addf", "dense<-0.000000e+00>"), ("arith.subf", "dense<0.000000e+00>"),
                                    ("arith.mulf", "dense<1.000000e+00>"), ("arith.divf", "dense<1.000000e+00>")])
def test_float_identity_shortcuts(op, rhs):
    body = "\n".join([const("%0", C4, T), const("%1", rhs, T),
                      f'    %2 = "{op}"(%0, %1) <{{{FM}}}> : ({T}, {T}) -> {T}'])
    f, d = returned(run(module(body, "%2", T)))
    assert d.name == "arith.constant" and not d.const.splat
    assert d.const.bits == [0x3F800000, 0x40000000, 0x40400000, 0x40800000]
    assert not any(o.name == op for o in f.ops)


def test_minimum_with_plus_inf_returns_lhs():
    body = "\n".join([const("%0", C4, T), const("%1", "dense<0x7F800000>", T),
                      f'    %2 = "arith.minimumf"(%0, %1) <{{{FM}}}> : ({T}, {T}) -> {T}'])
    f, d = returned(run(module(body, "%2", T)))
    assert d.const.bits[0] == 0x3F800000


I = "tensor<3xi32>"


@pytest.mark.parametrize("op,expect", [("arith.subi", [0]), ("arith.xori", [0])])
def test_same_operand_gives_zero(op, expect):
    body = "\n".join([const("%0", "dense<[5, -7, 9]>", I), f'    %1 = "{op}"(%0, %0) : ({I}, {I}) -> {I}'])
    f, d = returned(run(module(body, "%1", I)))
    assert d.const.splat and d.const.bits == expect


def test_remsi_by_one_and_muli_by_zero():
    body = "\n".join([const("%0", "dense<[5, -7, 9]>", I), const("%1", "dense<1>", I), const("%2", "dense<0>", I),
                      f'    %3 = "arith.remsi"(%0, %1) : ({I}, {I}) -> {I}',
                      f'    %4 = "arith.muli"(%0, %2) <{{overflowFlags = #arith.overflow<none>}}> : ({I}, {I}) -> {I}',
                      f'    %5 = "arith.addi"(%3, %4) <{{overflowFlags = #arith.overflow<none>}}> : ({I}, {I}) -> {I}'])
    # remsi x, 1 -> 0 and muli x, 0 -> the zero operand, all on the host; then
    # addi 0, 0 takes the x + 0 -> x shortcut: no element work at all
    f, d = returned(run(module(body, "%5", I)))
    assert d.const.splat and d.const.bits == [0]
    assert [o.name for o in f.ops] == ["arith.constant", "func.return"]


def test_cmpi_same_operand_is_a_bool_splat():
    body = "\n".join([const("%0", "dense<[5, -7, 9]>", I),
                      f'    %1 = "arith.cmpi"(%0, %0) <{{predicate = 3 : i64}}> : ({I}, {I}) -> tensor<3xi1>'])
    f, d = returned(run(module(body, "%1", "tensor<3xi1>")))
    assert d.const.splat and d.const.bits == [1]


def test_dense_cmpf_is_not_folded():
    body = "\n".join([const("%0", C4, T), const("%1", C4, T),
                      f'    %2 = "arith.cmpf"(%0, %1) <{{{FM}, predicate = 4 : i64}}> : ({T}, {T}) -> tensor<4xi1>'])
    f, d = returned(run(module(body, "%2", "tensor<4xi1>")))
    assert d.name == "arith.cmpf"


def test_identity_transpose_and_splat_transpose():
    t = "tensor<2x3xf32>"
    body = "\n".join([const("%0", "dense<[[1.0, 2.0, 3.0], [4.0, 5.0, 6.0]]>", t, "tosa.const", "values"),
                      f'    %1 = "tosa.transpose"(%0) <{{perms = array<i32: 0, 1>}}> : ({t}) -> {t}'])
    f, d = returned(run(module(body, "%1", t)))
    assert d.name == "tosa.const" and len(d.const.bits) == 6
    t2 = "tensor<3x2xf32>"
    body = "\n".join([const("%0", "dense<2.500000e+00>", t, "tosa.const", "values"),
                      f'    %1 = "tosa.transpose"(%0) <{{perms = array<i32: 1, 0>}}> : ({t}) -> {t2}'])
    f, d = returned(run(module(body, "%1", t2), "builtin.module(func.func(canonicalize))"))
    assert d.name == "tosa.const" and d.const.splat and d.const.bits == [0x40200000]
    assert d.const.ty.shape == [3, 2]


def test_constants_are_deduplicated_and_dead_ops_removed():
    body = "\n".join([const("%0", C4, T), const("%1", C4, T), const("%9", "dense<0.0>", T),
                      f'    %2 = "arith.maximumf"(%0, %1) <{{{FM}}}> : ({T}, {T}) -> {T}'])
    f, d = returned(run(module(body, "%2", T)))
    # the two equal constants become one, so maximumf(x, x) -> x; the unused constant goes
    assert d.name == "arith.constant"
    assert [o.name for o in f.ops] == ["arith.constant", "func.return"]


def test_element_work_refuses_without_gpu():
    body = "\n".join([const("%0", C4, T), const("%1", C4, T),
                      f'    %2 = "arith.addf"(%0, %1) <{{{FM}}}> : ({T}, {T}) -> {T}'])
    with pytest.raises(opt.OptError, match="needs a GPU"):
        run(module(body, "%2", T))


def test_unknown_pass_and_pipeline_errors():
    body = const("%0", C4, T)
    with pytest.raises(opt.OptError, match="unknown pass"):
        run(module(body, "%0", T), "builtin.module(func.func(cse))")
    with pytest.raises(opt.OptError, match="unsupported pipeline"):
        run(module(body, "%0", T), "builtin.module(cse)")


def test_split_input_file_and_generated_configs_parse():
    from mlirpass_b200 import mlir_gen
    one = module(const("%0", C4, T), "%0", T)
    out = opt.run(one + "// -----\n" + one, "canonicalize", n_gpus=0, split_input_file=True)[0]
    parts = out.split("// -----\n")
    assert len(parts) == 2 and all(returned(p)[1].name == "arith.constant" for p in parts)
    # the generated configurations parse; their folds need element work
    t = mlir_gen.config5_text(funcs=3, side=4, weight_side=0)
    with pytest.raises(opt.OptError, match="needs a GPU"):
        opt.run(t, mlir_gen.LAYERWISE, n_gpus=0)


def test_bitcast_shares_bytes_without_element_work():
    # bitcast keeps the bits under the new element type
    # (src/patterns/arith/canonicalize.rs:764-789): the host-only engine
    # folds it, with the large literal carried over as is.
    n = 4096
    hexs = b"".join((0x3F800000 + i).to_bytes(4, "little") for i in range(n)).hex().upper()
    body = "\n".join([const("%0", f'dense<"0x{hexs}">', f"tensor<{n}xf32>"),
                      f'    %1 = "arith.bitcast"(%0) : (tensor<{n}xf32>) -> tensor<{n}xi32>'])
    out = run(module(body, "%1", f"tensor<{n}xi32>"))
    f, d = returned(out)
    assert d.name == "arith.constant" and d.const.ty.elem == "i32"
    assert d.const.bits == [0x3F800000 + i for i in range(n)]


def test_select_shortcuts():
    c4 = "tensor<4xi1>"
    body = "\n".join([const("%c", "dense<true>", c4), const("%0", C4, T), const("%1", "dense<0.0>", T),
                      f'    %2 = "arith.select"(%c, %0, %1) : ({c4}, {T}, {T}) -> {T}'])
    f, d = returned(run(module(body, "%2", T)))
    assert d.name == "arith.constant" and d.const.bits == [0x3F800000, 0x40000000, 0x40400000, 0x40800000]
    # select(c, x, x) -> x, with a non-constant condition
    body = "\n".join([const("%0", C4, T),
                      f'    %c = "test.cond"() : () -> {c4}',
                      f'    %2 = "arith.select"(%c, %0, %0) : ({c4}, {T}, {T}) -> {T}'])
    f, d = returned(run(module(body, "%2", T)))
    assert d.name == "arith.constant"


def test_ext_trunc_chains_fold_on_the_host():
    i8, i32 = "tensor<4xi8>", "tensor<4xi32>"
    body = "\n".join([f'    %x = "test.src"() : () -> {i8}',
                      f'    %1 = "arith.extsi"(%x) : ({i8}) -> tensor<4xi16>',
                      f'    %2 = "arith.extsi"(%1) : (tensor<4xi16>) -> {i32}',
                      f'    %3 = "arith.trunci"(%2) : ({i32}) -> {i8}'])
    # trunci(extsi(x)) back to x's type is x itself (:685-706)
    f, d = returned(run(module(body, "%3", i8)))
    assert d.name == "test.src"


def test_new_element_folds_need_a_gpu():
    i32 = "tensor<4xi32>"
    body = "\n".join([const("%0", "dense<[7, -7, 9, 3]>", i32), const("%1", "dense<[2, 2, -4, 3]>", i32),
                      f'    %2 = "arith.floordivsi"(%0, %1) : ({i32}, {i32}) -> {i32}'])
    with pytest.raises(opt.OptError, match="needs a GPU"):
        run(module(body, "%2", i32))


def test_big_list_literals_are_constants():
    # A literal list longer than the parser's in-place threshold (i1
    # constants print as lists at any size) is still a constant.
    n = 3000
    lst = ", ".join(str(i) for i in range(n))
    body = "\n".join([const("%0", f"dense<[{lst}]>", f"tensor<{n}xi32>"),
                      f'    %1 = "arith.bitcast"(%0) : (tensor<{n}xi32>) -> tensor<{n}xf32>'])
    f, d = returned(run(module(body, "%1", f"tensor<{n}xf32>")))
    assert d.name == "arith.constant" and d.const.bits == list(range(n))


def test_output_as_array_without_copy():
    body = const("%0", C4, T)
    text = module(body, "%0", T)
    a, st = opt.run(text, "canonicalize", n_gpus=0, as_array=True)
    view = a[5:]
    del a
    import gc
    gc.collect()
    assert bytes(view) == opt.run(text, "canonicalize", n_gpus=0, as_bytes=True)[0][5:]
    assert st["call_ms"] > 0


def test_math_classify_folds_on_the_host_and_transcendentals_stay():
    F, V = "f32", "vector<4xf32>"
    body = "\n".join([
        const("%a", "2.000000e+00", F),
        const("%b", "dense<0x7FC00000>", V),
        '    %p = "ub.poison"() <{value = #ub.poison}> : () -> f32',
        '    %0 = "math.isnormal"(%a) <{fastmath = #arith.fastmath<none>}> : (f32) -> i1',
        '    %1 = "math.isnan"(%b) <{fastmath = #arith.fastmath<none>}> : (vector<4xf32>) -> vector<4xi1>',
        '    %2 = "math.absf"(%p) <{fastmath = #arith.fastmath<none>}> : (f32) -> f32',
        '    %3 = "math.sin"(%a) <{fastmath = #arith.fastmath<none>}> : (f32) -> f32',
        '    %4 = "math.isinf"(%b) <{fastmath = #arith.fastmath<none>}> : (vector<4xf32>) -> vector<4xi1>',
    ])
    out = run(module(body, "%0, %1, %2, %3, %4", "i1, vector<4xi1>, f32, f32, vector<4xi1>"))
    f = parse_funcs(out)["f"]
    d = [f.defs[v] for v in f.ret.operands]
    assert [x.name for x in d] == ["arith.constant", "arith.constant", "ub.poison", "math.sin", "arith.constant"]
    assert d[0].const.bits == [1] and d[1].const.splat and d[1].const.bits == [1] and d[4].const.bits == [0]


def test_math_element_folds_need_a_gpu():
    body = const("%a", C4, T) + '\n    %0 = "math.ceil"(%a) <{fastmath = #arith.fastmath<none>}> : (tensor<4xf32>) -> tensor<4xf32>'
    with pytest.raises(opt.OptError, match="needs a GPU"):
        run(module(body, "%0", T))


def test_output_buffers_given_back_are_reused_safely():
    # dcf_opt_free keeps the last buffer for a later run whose output fits
    # it; outputs of alternating sizes must come out whole each time.
    from mlirpass_b200 import mlir_gen
    big = mlir_gen.config5_text(funcs=8, side=32, weight_side=0)
    small = module(const("%0", C4, T), "%0", T)
    want = {}
    for text in (big, small, big, small, small, big):
        out, _ = opt.run(text, "builtin.module(func.func())", n_gpus=0, as_array=True)
        got = out.tobytes()
        del out
        want.setdefault(text, got)
        assert got == want[text]
        assert got.endswith(b") : () -> ()\n\n")


def test_dense_resource_operands_are_not_folded_host_only():
    # The same module as the GPU test: no fold sees a resource's value, so
    # the host-only driver (which refuses any element work) prints it back.
    from test_gpu_opt import check_resource_operands_stay
    check_resource_operands_stay(0)
