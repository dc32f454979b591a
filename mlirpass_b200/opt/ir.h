// ir.h — the IR of dcfold-opt: a small mutable form of MLIR's generic text
// format, enough to run the dense-constant folds of `canonicalize` and
// `tosa-layerwise-constant-fold` over whole modules.
//
// It mirrors the parts of mlirpass's arena IR (src/ir.rs: Body, OpData,
// values with use lists) that the fold path touches.  Attributes other than
// constant values are kept as their printed text and printed back verbatim.
#pragma once

#include <cstdint>
#include <list>
#include <memory>
#include <mutex>
#include <string>
#include <string_view>
#include <unordered_map>
#include <utility>
#include <vector>

namespace dco {

// ------------------------------------------------------------------ types

struct Type {
  std::string text;              // printed form
  std::string kind;              // "tensor", "vector", "" (scalar), "other"
  std::vector<int64_t> shape;    // static dims of a shaped type
  bool dynamic = false;          // a dim is '?' or scalable
  std::string elem;              // element type text
  int dtype = 0;                 // dcf dtype of the element (index as i64), 0 if none
  bool is_float() const;
  bool is_int() const;
  bool shaped() const { return kind == "tensor" || kind == "vector"; }
  bool static_shape() const { return shaped() && !dynamic; }
  int64_t count() const;          // elements of a static shaped type, 1 for scalars
};
using TypeP = std::shared_ptr<const Type>;

// Interned type for a printed type string.
TypeP type_of(const std::string& text);
// The same shape with another element type ("tensor<4xf32>" + "i1").
TypeP with_element(const TypeP& t, const std::string& elem);
// Element type of t (t itself for scalars).
TypeP element_type(const TypeP& t);

// ------------------------------------------------------- dense constants

class DeviceBuf;  // engine.h

// Host bytes of a constant.  resize() leaves new bytes uninitialised: they
// are always overwritten by a download or a decode, and zero-filling a
// multi-GiB result first would cost as much as the copy itself.
// Large host byte buffers come from a replaceable allocator: the engine
// installs a page-locked caching pool, so that copies between a constant's
// host bytes and the GPU need no staging, and the pages are reused from
// run to run.  free() must accept memory it did not hand out (buffers
// allocated before the pool was installed).
struct HostAllocator {
  void* (*alloc)(size_t bytes) = nullptr;
  void (*free)(void* p, size_t bytes) = nullptr;
};
HostAllocator& host_allocator();
constexpr size_t kHostPoolMin = 64u << 10;

template <class T>
struct NoInit : std::allocator<T> {
  template <class U>
  struct rebind {
    using other = NoInit<U>;
  };
  NoInit() = default;
  template <class U>
  NoInit(const NoInit<U>&) noexcept {}
  T* allocate(size_t n) {
    const HostAllocator& h = host_allocator();
    if (n * sizeof(T) >= kHostPoolMin && h.alloc) return (T*)h.alloc(n * sizeof(T));
    return std::allocator<T>::allocate(n);
  }
  void deallocate(T* p, size_t n) {
    const HostAllocator& h = host_allocator();
    if (n * sizeof(T) >= kHostPoolMin && h.free) return h.free(p, n * sizeof(T));
    std::allocator<T>::deallocate(p, n);
  }
  template <class U>
  void construct(U* p) noexcept {
    ::new ((void*)p) U;
  }
  template <class U, class... A>
  void construct(U* p, A&&... a) {
    ::new ((void*)p) U(std::forward<A>(a)...);
  }
};
using Bytes = std::vector<uint8_t, NoInit<uint8_t>>;

// The value of a constant attribute: the reference's `Const` (values, type,
// `elements` flag), stored as raw element bytes.  The bytes live on the
// host, on a GPU, or (straight after parsing) as the hex text of a
// dense<"0x…"> literal that is decoded on first use.
struct DenseValue {
  TypeP ty;                  // attribute type
  bool elements = false;     // dense<...> (shaped) versus a scalar literal
  bool splat = false;        // one stored element
  bool poison = false;       // ub.poison
  int dtype = 0;
  size_t es = 0;             // element bytes
  uint64_t n = 0;            // stored elements (1 when splat)
  Bytes host;                // host bytes, empty when not on the host
  std::string_view hex;      // "HEX…" digits (no 0x), when parsed from text
  std::shared_ptr<DeviceBuf> dev;  // device bytes
  // Element ranges on several GPUs (a sharded constant, ShardedEngine):
  // contiguous, in order, each a DenseValue of its own (one element when
  // that range is all equal).
  std::vector<std::shared_ptr<DenseValue>> parts;
  int all_equal = -1;        // cached "every value equal" test: -1 unknown
  uint64_t hash = 0;         // dcf_hash_many_async of the bytes, when hashed
  bool hashed = false;

  bool on_host() const { return !host.empty() || n == 0; }
  uint64_t bits0() const;    // first element's bits (host bytes required)
  uint64_t bytes() const { return n * es; }
};
using DenseP = std::shared_ptr<DenseValue>;

// --------------------------------------------------------------------- IR

struct Op;
struct Block;
struct Region;

struct Value {
  TypeP ty;
  Op* def = nullptr;          // defining op, or null for a block argument
  int index = 0;              // result or argument number
  Block* owner = nullptr;     // block of a block argument
  std::vector<Op*> uses;      // one entry per operand slot that reads it
  std::string name;           // text name of a block argument ("%arg0")
  std::string loc;            // a block argument's trailing "loc(...)"
};

struct Op {
  std::string name;
  std::vector<Value*> operands;
  std::vector<Value*> results;
  std::vector<std::pair<std::string, std::string>> props;  // <{...}> entries, text
  // A property value too large to copy (a dense literal of a big constant)
  // is kept as a view into the parsed text; its props entry holds "".
  std::string big_key;
  std::string_view big_value;
  std::string attrs;          // "{...}" discardable attributes, verbatim
  std::string successors;     // "[...]" verbatim
  std::vector<Region*> regions;
  std::string loc;            // trailing location, verbatim
  Block* parent = nullptr;
  std::list<Op*>::iterator pos;
  DenseP cst;                 // value of arith.constant / tosa.const / ub.poison
  bool cst_text = false;      // the value prop's text is the parsed original
  bool erased = false;

  const std::string* prop(const std::string& key) const;
  void set_prop(const std::string& key, const std::string& text);
  std::string dialect() const { return name.substr(0, name.find('.')); }
};

struct Block {
  std::string label;          // "^bb0" or empty for an unlabeled entry block
  std::vector<Value*> args;
  std::list<Op*> ops;
  Region* parent = nullptr;
};

struct Region {
  std::vector<Block*> blocks;
  Op* parent = nullptr;
};

// Owns every IR object of one module.
class Module {
 public:
  Op* top = nullptr;          // the builtin.module op
  // Text around the module op, kept verbatim: alias definitions before and
  // after it (`#map = ...`, `!t = ...`, `#loc = loc(...)` lines) and
  // `{-# ... #-}` metadata blocks (dialect resources) after it (the bodies
  // between the markers).
  std::string_view prologue;
  std::string_view epilogue;  // alias lines after the module op
  std::vector<std::string_view> metadata;

  Op* new_op(const std::string& name);
  Value* new_value(TypeP ty);
  Block* new_block();
  Region* new_region();

  // Insert `op` before `before` (in before's block), or at the end of `b`.
  void insert_before(Op* op, Op* before);
  void append(Op* op, Block* b);
  void detach(Op* op);
  // Remove an op whose results are unused; drops its operand uses.
  void erase(Op* op);
  void set_operand(Op* op, size_t i, Value* v);
  void replace_all_uses(Value* from, Value* to);

 private:
  // Isolated functions are rewritten by one thread per GPU at once: the
  // node arenas are the only state they share.
  std::mutex mu_;
  std::vector<std::unique_ptr<Op>> ops_;
  std::vector<std::unique_ptr<Value>> values_;
  std::vector<std::unique_ptr<Block>> blocks_;
  std::vector<std::unique_ptr<Region>> regions_;
};

// Parse a module in MLIR's generic form.  `text` must outlive the module
// (hex literals are decoded from it lazily).  Throws std::runtime_error.
// reformat: parsed constants print through the element printer, as the
// reference re-reads every float and integer dense attribute at import
// (canonical_floats, src/ir.rs:2149-2164); otherwise they keep their input
// text.  Big hex literals keep their text either way: uppercase hex is
// their printed form.
std::unique_ptr<Module> parse_module(std::string_view text, bool reformat = true);

// Print the module in generic form.  Device-resident constants are fetched
// through `fetch` (which fills DenseValue::host or returns hex digits).
struct PrintHooks {
  // Uppercase hex digits of a constant's bytes (no 0x).  Must be set.
  std::string (*hex_of)(DenseValue& v, void* ctx) = nullptr;
  // Host bytes of a splat's element (fetch from the device if needed).
  uint64_t (*bits0_of)(DenseValue& v, void* ctx) = nullptr;
  void* ctx = nullptr;
  // Print locations (mlir-opt's --mlir-print-debuginfo); without it op and
  // block-argument locations and `#loc` alias lines are left out.
  bool debuginfo = false;
};
// A printed module: the text without its large literal bodies, plus where
// each body goes.  write_to() assembles the text with several host threads
// (the hex encoding of host bytes included).  The module and the parsed
// text must outlive it.
struct PrintedModule {
  struct Fill {
    enum Kind { RAW, UPPER, HEX } kind;
    const void* src;  // characters (RAW, UPPER) or bytes (HEX)
    size_t nchars;    // characters it prints
    size_t at;        // skeleton position it goes before
  };
  std::string skeleton;
  std::vector<Fill> fills;
  size_t size_ = 0;
  size_t size() const { return size_; }
  void write_to(char* dst) const;
  std::string str() const;
};
PrintedModule print_module_parts(Module& m, const PrintHooks& hooks);
std::string print_module(Module& m, const PrintHooks& hooks);

// Float literal helpers (MLIR syntax).
bool parse_float_literal(const std::string& tok, int dtype, uint64_t* bits);
std::string print_float_literal(uint64_t bits, int dtype);
std::string print_int_literal(uint64_t bits, int dtype);
// The text of a float element (E exponent bits, M mantissa bits) as
// mlir-opt prints it; parse_back(text, &bits, ctx) reads a candidate text
// back into the element type.
std::string mlir_float_text(uint64_t bits, int E, int M, bool (*parse_back)(const std::string&, uint64_t*, void*),
                            void* ctx);

}  // namespace dco
