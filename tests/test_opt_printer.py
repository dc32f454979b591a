"""The pass driver's generic-form printer on the CPU, byte for byte.

Each case is a small module whose printed text follows from the reference's
printing rules:
  * SSA names (Names::of with Namer, src/ir.rs:2470-2650): in the generic
    form one value counter and one entry-argument counter run over the whole
    module and are never reset; regions are named from a stack, so the
    regions nested in a region come after its own blocks, the last first;
    entry-block arguments are %argK, other block arguments and results %N,
    an op with k results %N:k with uses %N#i; block labels are ^bbN by
    position in their region;
  * every non-entry block carries mlir-opt's predecessor comment, and an
    empty entry block prints its header;
  * --split-input-file chunks split at lines reading "// -----"; each
    printed module is followed by a blank line unless printing in local
    scope, and the chunks are joined by the marker line (Invocation::chunks,
    ::print, ::run, src/pass.rs:704-820);
  * locations are printed only with debuginfo, alias lines only when the
    printed module uses them (Invocation::print_op, src/pass.rs:769-793);
  * unused dense_resource blobs are dropped (src/ir.rs:2951-2974).
"""
from mlirpass_b200 import opt

NOP = "builtin.module(func.func())"


def show(text, **kw):
    return opt.run(text, NOP, n_gpus=0, **kw)[0]


NESTED_IN = '''"builtin.module"() ({
  "func.func"() <{function_type = (i32) -> i32, sym_name = "a"}> ({
  ^bb0(%x: i32):
    %c = "arith.constant"() <{value = 1 : i32}> : () -> i32
    "foo.region"() ({
    ^bb0(%y: i32):
      %z = "arith.addi"(%y, %c) <{overflowFlags = #arith.overflow<none>}> : (i32, i32) -> i32
      "foo.yield"(%z) : (i32) -> ()
    }, {
    ^bb0(%w: i32):
      "foo.yield"(%w) : (i32) -> ()
    }) : () -> ()
    "func.return"(%x) : (i32) -> ()
  }) : () -> ()
  "func.func"() <{function_type = (i32) -> i32, sym_name = "b"}> ({
  ^bb0(%v: i32):
    %p:2 = "foo.pair"(%v) : (i32) -> (i32, i32)
    "cf.br"(%p#1)[^next] : (i32) -> ()
  ^next(%q: i32):
    "func.return"(%q) : (i32) -> ()
  }) : () -> ()
}) : () -> ()
'''

# The module's region holds both functions; they are pushed in order and
# popped last first, so "b" is numbered before "a", and in "a" the second
# nested region before the first.
NESTED_OUT = '''"builtin.module"() ({
  "func.func"() <{function_type = (i32) -> i32, sym_name = "a"}> ({
  ^bb0(%arg1: i32):
    %2 = "arith.constant"() <{value = 1 : i32}> : () -> i32
    "foo.region"() ({
    ^bb0(%arg3: i32):
      %3 = "arith.addi"(%arg3, %2) <{overflowFlags = #arith.overflow<none>}> : (i32, i32) -> i32
      "foo.yield"(%3) : (i32) -> ()
    }, {
    ^bb0(%arg2: i32):
      "foo.yield"(%arg2) : (i32) -> ()
    }) : () -> ()
    "func.return"(%arg1) : (i32) -> ()
  }) : () -> ()
  "func.func"() <{function_type = (i32) -> i32, sym_name = "b"}> ({
  ^bb0(%arg0: i32):
    %0:2 = "foo.pair"(%arg0) : (i32) -> (i32, i32)
    "cf.br"(%0#1)[^bb1] : (i32) -> ()
  ^bb1(%1: i32):  // pred: ^bb0
    "func.return"(%1) : (i32) -> ()
  }) : () -> ()
}) : () -> ()

'''


def test_names_follow_the_module_wide_region_stack():
    assert show(NESTED_IN) == NESTED_OUT
    # printing is a fixed point
    assert show(NESTED_OUT) == NESTED_OUT


PREDS_IN = '''"builtin.module"() ({
  "func.func"() <{function_type = (i1) -> (), sym_name = "c"}> ({
  ^entry(%a: i1):
    "cf.cond_br"(%a)[^x, ^x] <{operandSegmentSizes = array<i32: 1, 0, 0>}> : (i1) -> ()
  ^x:
    "func.return"() : () -> ()
  ^dead:
    "cf.br"()[^x] : () -> ()
  }) : () -> ()
}) : () -> ()
'''

PREDS_OUT = '''"builtin.module"() ({
  "func.func"() <{function_type = (i1) -> (), sym_name = "c"}> ({
  ^bb0(%arg0: i1):
    "cf.cond_br"(%arg0)[^bb1, ^bb1] <{operandSegmentSizes = array<i32: 1, 0, 0>}> : (i1) -> ()
  ^bb1:  // 3 preds: ^bb0, ^bb0, ^bb2
    "func.return"() : () -> ()
  ^bb2:  // no predecessors
    "cf.br"()[^bb1] : () -> ()
  }) : () -> ()
}) : () -> ()

'''


def test_block_labels_and_predecessor_comments():
    assert show(PREDS_IN) == PREDS_OUT


EMPTY = '"builtin.module"() ({\n^bb0:\n}) : () -> ()\n'


def test_empty_module_and_empty_chunk():
    assert show(EMPTY) == EMPTY + "\n"
    with_attr = '"builtin.module"() ({\n^bb0:\n}) {llvm.data_layout = ""} : () -> ()\n'
    assert show(with_attr) == with_attr + "\n"
    # a chunk of blank lines and comments is an empty module
    assert show("// nothing here\n\n") == EMPTY + "\n"


def test_split_markers_and_joining():
    one = '"builtin.module"() ({\n  "foo.op"() : () -> ()\n}) : () -> ()\n'
    # only a whole line "// -----" (trailing blanks allowed) splits
    text = one + "// -----   \n" + one + "  // -----\n"
    out = opt.run(text, NOP, n_gpus=0, split_input_file=True)[0]
    assert out == one + "\n" + "// -----\n" + one + "\n"
    assert opt.run(text, NOP, n_gpus=0, split_input_file=True, local_scope=True)[0] == one + "// -----\n" + one


LOC_IN = '''#loc = loc("m.mlir":1:1)
#unused = affine_map<(d0) -> (d0)>
#map = affine_map<(d0) -> (d0 + 1)>
"builtin.module"() ({
  "func.func"() <{function_type = (i32) -> (), sym_name = "f"}> ({
  ^bb0(%a: i32 loc("m.mlir":2:3)):
    "foo.use"(%a) <{m = #map}> : (i32) -> () loc(#loc1)
    "func.return"() : () -> () loc(fused[#loc, "x"])
  }) : () -> () loc(#loc)
}) : () -> () loc(#loc)
#loc1 = loc("m.mlir":3:5)
'''


def test_locations_and_aliases():
    plain = show(LOC_IN)
    assert plain == '''#map = affine_map<(d0) -> (d0 + 1)>
"builtin.module"() ({
  "func.func"() <{function_type = (i32) -> (), sym_name = "f"}> ({
  ^bb0(%arg0: i32):
    "foo.use"(%arg0) <{m = #map}> : (i32) -> ()
    "func.return"() : () -> ()
  }) : () -> ()
}) : () -> ()

'''
    dbg = show(LOC_IN, debuginfo=True)
    assert dbg == LOC_IN.replace("#unused = affine_map<(d0) -> (d0)>\n", "").replace("%a", "%arg0") + "\n"


def test_aliases_used_only_by_other_aliases_are_kept():
    text = ('#inner = #foo.attr<1>\n#outer = #foo.wrap<x = #inner>\n'
            '"builtin.module"() ({\n  "foo.op"() {a = #outer} : () -> ()\n}) : () -> ()\n')
    assert show(text) == text + "\n"


def test_unused_resources_are_dropped():
    body = ('"builtin.module"() ({\n'
            '  %0 = "arith.constant"() <{value = dense_resource<used> : tensor<2xi32>}> : () -> tensor<2xi32>\n'
            '  "foo.use"(%0) : (tensor<2xi32>) -> ()\n'
            '}) : () -> ()\n')
    meta = ('\n{-#\n  dialect_resources: {\n    builtin: {\n'
            '      used: "0x040000000100000002000000",\n'
            '      unused: "0x040000000300000004000000"\n'
            '    }\n  }\n#-}\n')
    out = show(body + meta)
    assert out.startswith(body)
    assert "used: \"0x040000000100000002000000\"" in out and "unused" not in out
