// ir.cpp — types, IR mutation, the generic-form parser and printer, and the
// MLIR float / int literal codecs of dcfold-opt.
#include "ir.h"

#include <algorithm>
#include <atomic>
#include <thread>

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <stdexcept>

#include "../../include/dcfold.h"

namespace dco {

HostAllocator& host_allocator() {
  static HostAllocator a;
  return a;
}

// ================================================================== types

static int dtype_of_elem(const std::string& e) {
  static const std::pair<const char*, int> table[] = {
      {"i1", DCF_I1},     {"i8", DCF_I8},       {"i16", DCF_I16},        {"i32", DCF_I32},
      {"i64", DCF_I64},   {"index", DCF_I64},   {"f16", DCF_F16},        {"bf16", DCF_BF16},
      {"f32", DCF_F32},   {"f64", DCF_F64},     {"f8E5M2", DCF_F8E5M2}, {"f8E4M3", DCF_F8E4M3},
      {"f8E3M4", DCF_F8E3M4}};
  for (auto& [n, d] : table)
    if (e == n) return d;
  return 0;
}

bool Type::is_float() const { return dtype >= DCF_F16 && dtype <= DCF_F8E3M4; }
bool Type::is_int() const { return dtype >= DCF_I1 && dtype <= DCF_I64; }

int64_t Type::count() const {
  if (!shaped()) return 1;
  int64_t n = 1;
  for (int64_t d : shape) n *= d;
  return n;
}

static Type make_type(const std::string& text) {
  Type t;
  t.text = text;
  auto shaped = [&](const char* pre) { return text.rfind(pre, 0) == 0 && text.back() == '>'; };
  if (shaped("tensor<") || shaped("vector<")) {
    t.kind = text[0] == 't' ? "tensor" : "vector";
    std::string body = text.substr(7, text.size() - 8);
    // An encoding or other trailing parameter makes the type opaque here.
    int depth = 0;
    for (char c : body) {
      if (c == '<' || c == '(' || c == '[') depth++;
      if (c == '>' || c == ')' || c == ']') depth--;
      if (c == ',' && depth == 0) {
        t.kind = "other";
        return t;
      }
    }
    size_t p = 0;
    for (;;) {
      size_t x = body.find('x', p);
      if (x == std::string::npos) break;
      std::string dim = body.substr(p, x - p);
      bool digits = !dim.empty();
      for (char c : dim) digits = digits && (c >= '0' && c <= '9');
      if (digits) {
        t.shape.push_back(std::stoll(dim));
      } else if (dim == "?" || (!dim.empty() && dim[0] == '[')) {
        t.dynamic = true;
        t.shape.push_back(-1);
      } else {
        break;
      }
      p = x + 1;
    }
    t.elem = body.substr(p);
  } else {
    t.kind = "";
    t.elem = text;
  }
  t.dtype = dtype_of_elem(t.elem);
  if (t.kind == "" && !t.dtype) t.kind = "other";
  return t;
}

TypeP type_of(const std::string& text) {
  static std::mutex mu;
  static std::unordered_map<std::string, TypeP> interned;
  std::lock_guard<std::mutex> g(mu);
  auto it = interned.find(text);
  if (it != interned.end()) return it->second;
  auto t = std::make_shared<const Type>(make_type(text));
  interned.emplace(text, t);
  return t;
}

TypeP with_element(const TypeP& t, const std::string& elem) {
  if (!t->shaped()) return type_of(elem);
  std::string s = t->kind + "<";
  for (int64_t d : t->shape) s += (d < 0 ? std::string("?") : std::to_string(d)) + "x";
  return type_of(s + elem + ">");
}

TypeP element_type(const TypeP& t) { return t->shaped() ? type_of(t->elem) : t; }

uint64_t DenseValue::bits0() const {
  uint64_t v = 0;
  if (!host.empty()) memcpy(&v, host.data(), es);
  return v;
}

// ================================================================ module

const std::string* Op::prop(const std::string& key) const {
  for (auto& kv : props)
    if (kv.first == key) return &kv.second;
  return nullptr;
}

void Op::set_prop(const std::string& key, const std::string& text) {
  for (auto& kv : props)
    if (kv.first == key) {
      kv.second = text;
      return;
    }
  props.emplace_back(key, text);
}

Op* Module::new_op(const std::string& name) {
  std::lock_guard<std::mutex> g(mu_);
  ops_.push_back(std::make_unique<Op>());
  ops_.back()->name = name;
  return ops_.back().get();
}

Value* Module::new_value(TypeP ty) {
  std::lock_guard<std::mutex> g(mu_);
  values_.push_back(std::make_unique<Value>());
  values_.back()->ty = std::move(ty);
  return values_.back().get();
}

Block* Module::new_block() {
  std::lock_guard<std::mutex> g(mu_);
  blocks_.push_back(std::make_unique<Block>());
  return blocks_.back().get();
}

Region* Module::new_region() {
  std::lock_guard<std::mutex> g(mu_);
  regions_.push_back(std::make_unique<Region>());
  return regions_.back().get();
}

void Module::insert_before(Op* op, Op* before) {
  Block* b = before->parent;
  op->parent = b;
  op->pos = b->ops.insert(before->pos, op);
}

void Module::append(Op* op, Block* b) {
  op->parent = b;
  op->pos = b->ops.insert(b->ops.end(), op);
}

void Module::detach(Op* op) {
  if (!op->parent) return;
  op->parent->ops.erase(op->pos);
  op->parent = nullptr;
}

static void drop_use(Value* v, Op* user) {
  for (size_t i = 0; i < v->uses.size(); i++)
    if (v->uses[i] == user) {
      v->uses.erase(v->uses.begin() + (long)i);
      return;
    }
}

void Module::erase(Op* op) {
  for (Region* r : op->regions)
    for (Block* b : r->blocks)
      while (!b->ops.empty()) {
        Op* inner = b->ops.back();
        for (Value* res : inner->results) res->uses.clear();
        erase(inner);
      }
  for (Value* v : op->operands) drop_use(v, op);
  op->operands.clear();
  detach(op);
  op->erased = true;
}

void Module::set_operand(Op* op, size_t i, Value* v) {
  drop_use(op->operands[i], op);
  op->operands[i] = v;
  v->uses.push_back(op);
}

void Module::replace_all_uses(Value* from, Value* to) {
  if (from == to) return;
  std::vector<Op*> users = from->uses;
  for (Op* u : users)
    for (size_t i = 0; i < u->operands.size(); i++)
      if (u->operands[i] == from) set_operand(u, i, to);
}

// ======================================================= literal codecs

struct Layout {
  int E, M;
};

static bool layout_of(int dtype, Layout* l) {
  switch (dtype) {
    case DCF_F16: *l = {5, 10}; return true;
    case DCF_BF16: *l = {8, 7}; return true;
    case DCF_F32: *l = {8, 23}; return true;
    case DCF_F64: *l = {11, 52}; return true;
    case DCF_F8E5M2: *l = {5, 2}; return true;
    case DCF_F8E4M3: *l = {4, 3}; return true;
    case DCF_F8E3M4: *l = {3, 4}; return true;
    default: return false;
  }
}

static int width_of(int dtype) {
  switch (dtype) {
    case DCF_I1: return 1;
    case DCF_I8: return 8;
    case DCF_I16: return 16;
    case DCF_I32: return 32;
    case DCF_I64: return 64;
    default: return 0;
  }
}

static size_t elem_bytes(int dtype) { return dcf_dtype_size((dcf_dtype)dtype); }

// Nearest-even rounding of a finite double into a narrow IEEE-like layout.
static uint64_t narrow_from_double(double x, Layout L) {
  uint64_t d;
  memcpy(&d, &x, 8);
  const uint64_t sign = (d >> 63) << (L.E + L.M);
  if (x != x) return sign | ((((1ull << L.E) - 1)) << L.M) | (1ull << (L.M - 1));
  if (std::isinf(x)) return sign | (((1ull << L.E) - 1) << L.M);
  if (x == 0) return sign;
  int e2;
  double fr = std::frexp(std::fabs(x), &e2);  // |x| = fr * 2^e2, fr in [0.5, 1)
  uint64_t sig = (uint64_t)std::ldexp(fr, 53);  // exact: 53-bit significand
  int exp = e2 - 53;
  const int bias = (1 << (L.E - 1)) - 1, emin = 1 - bias;
  const int p = 63 - __builtin_clzll(sig);
  const int e = p + exp;
  const int q = (e < emin) ? emin - L.M : e - L.M;
  const int sh = q - exp;
  uint64_t r;
  if (sh <= 0) {
    r = sig << (-sh);
  } else if (sh >= 64) {
    r = 0;
  } else {
    const uint64_t rem = sig & ((1ull << sh) - 1), half = 1ull << (sh - 1);
    r = sig >> sh;
    if (rem > half || (rem == half && (r & 1))) r++;
  }
  uint64_t bits = (e < emin) ? r : (((uint64_t)(e + bias - 1) << L.M) + r);
  if ((bits >> L.M) >= ((1ull << L.E) - 1)) bits = ((1ull << L.E) - 1) << L.M;
  return sign | bits;
}

static double widen_to_double(uint64_t b, Layout L) {
  const bool neg = (b >> (L.E + L.M)) & 1;
  const uint64_t ef = (b >> L.M) & ((1ull << L.E) - 1), m = b & ((1ull << L.M) - 1);
  const int bias = (1 << (L.E - 1)) - 1;
  double v;
  if (ef == ((1ull << L.E) - 1)) v = m ? NAN : INFINITY;
  else if (ef == 0) v = std::ldexp((double)m, 1 - bias - L.M);
  else v = std::ldexp((double)(m | (1ull << L.M)), (int)ef - bias - L.M);
  return neg ? -v : v;
}

bool parse_float_literal(const std::string& tok, int dtype, uint64_t* bits) {
  Layout L;
  if (!layout_of(dtype, &L)) return false;
  if (tok.size() > 2 && tok[0] == '0' && (tok[1] == 'x' || tok[1] == 'X')) {
    *bits = strtoull(tok.c_str(), nullptr, 16);
    return true;
  }
  char* end = nullptr;
  if (dtype == DCF_F32) {
    float f = strtof(tok.c_str(), &end);
    uint32_t u;
    memcpy(&u, &f, 4);
    *bits = u;
  } else {
    double x = strtod(tok.c_str(), &end);
    if (dtype == DCF_F64) memcpy(bits, &x, 8);
    else *bits = narrow_from_double(x, L);
  }
  return end && *end == 0;
}

// A float element as mlir-opt prints it (float_text.cpp): six-digit
// scientific form when that parses back to the same bits, else the
// shortest round-trip decimal form, else the hex bit pattern.
std::string print_float_literal(uint64_t bits, int dtype) {
  Layout L;
  if (!layout_of(dtype, &L)) return "0";
  auto back = [](const std::string& text, uint64_t* out, void* ctx) {
    return parse_float_literal(text, *(const int*)ctx, out);
  };
  return mlir_float_text(bits, L.E, L.M, back, &dtype);
}

std::string print_int_literal(uint64_t bits, int dtype) {
  const int w = width_of(dtype);
  if (w == 1) return (bits & 1) ? "true" : "false";
  if (w < 64) {
    const uint64_t m = 1ull << (w - 1);
    bits &= (1ull << w) - 1;
    return std::to_string((long long)((bits ^ m) - m));
  }
  return std::to_string((long long)bits);
}

static bool parse_int_literal(const std::string& tok, int dtype, uint64_t* bits) {
  const int w = width_of(dtype);
  if (!w) return false;
  if (tok == "true") {
    *bits = 1;
    return true;
  }
  if (tok == "false") {
    *bits = 0;
    return true;
  }
  char* end = nullptr;
  uint64_t v;
  if (!tok.empty() && tok[0] == '-') v = (uint64_t)strtoll(tok.c_str(), &end, 0);
  else v = strtoull(tok.c_str(), &end, 0);
  if (!end || *end) return false;
  *bits = (w == 64) ? v : (v & ((1ull << w) - 1));
  return true;
}

// =================================================================== parse

namespace {

// Property values longer than this are not copied out of the parsed text.
constexpr size_t kBigProp = 4096;

[[noreturn]] void fail(const std::string& msg, size_t at) {
  throw std::runtime_error("parse error at offset " + std::to_string(at) + ": " + msg);
}

std::string trim(const std::string& s) {
  size_t a = 0, b = s.size();
  while (a < b && isspace((unsigned char)s[a])) a++;
  while (b > a && isspace((unsigned char)s[b - 1])) b--;
  return s.substr(a, b - a);
}

// Split at top-level occurrences of `sep`, honouring (), [], {}, <> nesting,
// string literals and the "->" arrow.
std::vector<std::string> split_top(const std::string& s, char sep) {
  std::vector<std::string> out;
  int depth = 0;
  size_t start = 0;
  bool str = false;
  for (size_t i = 0; i < s.size(); i++) {
    const char c = s[i];
    if (str) {
      if (c == '\\') i++;
      else if (c == '"') str = false;
      continue;
    }
    if (c == '"') str = true;
    else if (c == '-' && i + 1 < s.size() && s[i + 1] == '>') i++;
    else if (c == '(' || c == '[' || c == '{' || c == '<') depth++;
    else if (c == ')' || c == ']' || c == '}' || c == '>') depth--;
    else if (c == sep && depth == 0) {
      out.push_back(trim(s.substr(start, i - start)));
      start = i + 1;
    }
  }
  std::string last = trim(s.substr(start));
  if (!last.empty() || !out.empty()) out.push_back(last);
  return out;
}

void flatten_list(const std::string& s, std::vector<std::string>& out) {
  std::string t = trim(s);
  if (!t.empty() && t[0] == '[') {
    for (auto& part : split_top(t.substr(1, t.size() - 2), ',')) flatten_list(part, out);
  } else if (!t.empty()) {
    out.push_back(t);
  }
}

// Position of the first " loc(" in `t` outside brackets and string
// literals (where a trailing location starts), or npos.
size_t top_level_loc(const std::string& t) {
  int depth = 0;
  for (size_t k = 0; k < t.size(); k++) {
    const char c = t[k];
    if (c == '"') {
      while (++k < t.size() && t[k] != '"')
        if (t[k] == '\\') k++;
      continue;
    }
    if (c == '-' && k + 1 < t.size() && t[k + 1] == '>') k++;  // an arrow, not a bracket
    else if (c == '<' || c == '(' || c == '[' || c == '{') depth++;
    else if (c == '>' || c == ')' || c == ']' || c == '}') depth--;
    else if (depth == 0 && t.compare(k, 5, " loc(") == 0) return k;
  }
  return std::string::npos;
}

class Parser {
 public:
  Parser(std::string_view s, Module& m, bool reformat) : s_(s), m_(m), reformat_(reformat) { find_hex_literals(); }

  Op* parse_top() {
    scopes_.emplace_back();
    ws();
    // Alias definitions before the module op, one per line.
    const size_t pro0 = p_;
    while (p_ < s_.size() && (s_[p_] == '#' || s_[p_] == '!')) {
      const size_t nl = s_.find('\n', p_);
      p_ = nl == std::string_view::npos ? s_.size() : nl + 1;
      ws();
    }
    m_.prologue = s_.substr(pro0, p_ - pro0);
    if (p_ == s_.size()) {
      // Nothing but blank lines and comments: an empty module, as a parser
      // that wraps top-level ops in an implicit module makes of it.
      Op* op = m_.new_op("builtin.module");
      Region* r = m_.new_region();
      r->parent = op;
      Block* b = m_.new_block();
      b->parent = r;
      r->blocks.push_back(b);
      op->regions.push_back(r);
      close_scope();
      return op;
    }
    Op* op = parse_op(nullptr);
    ws();
    // After it: location / attribute alias lines and metadata blocks.
    const size_t epi0 = p_;
    for (;;) {
      if (p_ < s_.size() && (s_[p_] == '#' || s_[p_] == '!')) {
        const size_t nl = s_.find('\n', p_);
        p_ = nl == std::string_view::npos ? s_.size() : nl + 1;
        m_.epilogue = s_.substr(epi0, p_ - epi0);
        ws();
        continue;
      }
      if (s_.compare(p_, 3, "{-#") == 0) {
        const size_t a = p_ + 3, e = s_.find("#-}", a);
        if (e == std::string_view::npos) fail("unterminated {-# block", p_);
        m_.metadata.push_back(s_.substr(a, e - a));
        p_ = e + 3;
        ws();
        continue;
      }
      break;
    }
    if (p_ != s_.size()) fail("trailing text", p_);
    close_scope();
    return op;
  }

 private:
  const std::string_view s_;
  std::string sub(size_t a, size_t n = std::string_view::npos) const { return std::string(s_.substr(a, n)); }
  Module& m_;
  // Print parsed constants (other than big hex literals, whose uppercase
  // hex is already their printed form) through the element printer instead
  // of as their input text.
  const bool reformat_;
  size_t p_ = 0;
  struct Scope {
    std::unordered_map<std::string, std::vector<Value*>> names;
    std::unordered_map<std::string, Value*> forward;
  };
  std::vector<Scope> scopes_;

  void ws() {
    for (;;) {
      while (p_ < s_.size() && isspace((unsigned char)s_[p_])) p_++;
      if (p_ + 1 < s_.size() && s_[p_] == '/' && s_[p_ + 1] == '/') {
        while (p_ < s_.size() && s_[p_] != '\n') p_++;
        continue;
      }
      break;
    }
  }
  bool peek(char c) {
    ws();
    return p_ < s_.size() && s_[p_] == c;
  }
  bool peek(const char* t) {
    ws();
    return s_.compare(p_, strlen(t), t) == 0;
  }
  bool eat(char c) {
    if (!peek(c)) return false;
    p_++;
    return true;
  }
  bool eat(const char* t) {
    if (!peek(t)) return false;
    p_ += strlen(t);
    return true;
  }
  void expect(char c) {
    if (!eat(c)) fail(std::string("expected '") + c + "'", p_);
  }

  // A balanced span starting here, ending before a top-level char in `stops`.
  std::string span(const char* stops) {
    const auto r = span_pos(stops);
    return trim(sub(r.first, r.second - r.first));
  }

  // Hex literals ("0x... right after `dense<`): [opening quote, closing
  // quote] positions, found up front by several threads, so that the
  // sequential parse jumps over their bodies instead of scanning them.
  // Inside another string a quote is escaped, so the pattern marks real
  // literals only.
  std::vector<std::pair<size_t, size_t>> lits_;
  size_t lit_i_ = 0;

  void find_hex_literals() {
    constexpr size_t kMinText = 64u << 20;
    if (s_.size() < kMinText) return;
    const unsigned nth = std::max(1u, std::min(16u, std::thread::hardware_concurrency()));
    std::vector<std::vector<std::pair<size_t, size_t>>> part(nth);
    auto scan = [&](unsigned t) {
      const char* base = s_.data();
      const size_t n = s_.size();
      size_t p = n * t / nth;
      const size_t end = n * (t + 1) / nth;
      while (p < end) {
        const char* q = (const char*)memchr(base + p, '"', end - p);
        if (!q) break;
        const size_t at = (size_t)(q - base);
        if (at >= 6 && at + 2 < n && memcmp(q - 6, "dense<", 6) == 0 && q[1] == '0' && q[2] == 'x') {
          const char* e = (const char*)memchr(q + 1, '"', n - at - 1);
          if (!e) break;
          part[t].emplace_back(at, (size_t)(e - base));
          p = (size_t)(e - base) + 1;
        } else {
          p = at + 1;
        }
      }
    };
    std::vector<std::thread> th;
    for (unsigned t = 1; t < nth; t++) th.emplace_back(scan, t);
    scan(0);
    for (auto& x : th) x.join();
    for (auto& v : part) lits_.insert(lits_.end(), v.begin(), v.end());
  }

  // The closing quote of the hex literal opening at `at`, or npos.
  size_t hex_literal_end(size_t at) {
    while (lit_i_ < lits_.size() && lits_[lit_i_].first < at) lit_i_++;
    return (lit_i_ < lits_.size() && lits_[lit_i_].first == at) ? lits_[lit_i_].second : std::string_view::npos;
  }

  // The same, as [start, end) offsets: nothing is copied, and string
  // literals (the hex payload of a dense constant) are skipped with memchr.
  std::pair<size_t, size_t> span_pos(const char* stops) {
    ws();
    const size_t start = p_;
    int depth = 0;
    bool str = false;
    for (; p_ < s_.size(); p_++) {
      const char c = s_[p_];
      if (str) {
        if (c == '\\') {
          p_++;
          continue;
        }
        if (c == '"') {
          str = false;
          continue;
        }
        const void* q = memchr(s_.data() + p_, '"', s_.size() - p_);
        const void* bs = memchr(s_.data() + p_, '\\', q ? (size_t)((const char*)q - (s_.data() + p_)) : s_.size() - p_);
        if (q && !bs) {
          p_ = (size_t)((const char*)q - s_.data()) - 1;  // land on the quote next iteration
        }
        continue;
      }
      if (depth == 0 && strchr(stops, c)) break;
      if (c == '"') {
        const size_t e = lits_.empty() ? std::string_view::npos : hex_literal_end(p_);
        if (e != std::string_view::npos) p_ = e;  // at the closing quote; the string is done
        else str = true;
      }
      else if (c == '-' && p_ + 1 < s_.size() && s_[p_ + 1] == '>') p_++;
      else if (c == '(' || c == '[' || c == '{' || c == '<') depth++;
      else if (c == ')' || c == ']' || c == '}' || c == '>') {
        if (depth == 0) break;
        depth--;
      }
    }
    size_t a = start, b = p_;
    while (a < b && isspace((unsigned char)s_[a])) a++;
    while (b > a && isspace((unsigned char)s_[b - 1])) b--;
    return {a, b};
  }

  std::string ident() {
    ws();
    const size_t start = p_;
    while (p_ < s_.size() && (isalnum((unsigned char)s_[p_]) || strchr("_$.-#%^", s_[p_]))) p_++;
    return sub(start, p_ - start);
  }

  void close_scope() {
    Scope& sc = scopes_.back();
    if (!sc.forward.empty()) fail("use of undefined value " + sc.forward.begin()->first, p_);
    scopes_.pop_back();
  }

  Value* lookup(const std::string& ref, TypeP ty) {
    std::string name = ref;
    size_t idx = 0;
    const size_t hash = ref.find('#');
    if (hash != std::string::npos) {
      name = ref.substr(0, hash);
      idx = std::stoul(ref.substr(hash + 1));
    }
    for (auto it = scopes_.rbegin(); it != scopes_.rend(); ++it) {
      auto f = it->names.find(name);
      if (f != it->names.end()) {
        if (idx >= f->second.size()) fail("result index out of range in " + ref, p_);
        return f->second[idx];
      }
    }
    Scope& sc = scopes_.back();
    auto f = sc.forward.find(ref);
    if (f != sc.forward.end()) return f->second;
    Value* v = m_.new_value(std::move(ty));
    sc.forward.emplace(ref, v);
    return v;
  }

  void define(const std::string& name, const std::vector<Value*>& vals) {
    Scope& sc = scopes_.back();
    for (size_t i = 0; i < vals.size(); i++) {
      const std::string ref = vals.size() == 1 ? name : name + "#" + std::to_string(i);
      for (const std::string& key : {ref, name + "#" + std::to_string(i)}) {
        auto f = sc.forward.find(key);
        if (f != sc.forward.end()) {
          m_.replace_all_uses(f->second, vals[i]);
          sc.forward.erase(f);
        }
      }
    }
    sc.names[name] = vals;
  }

  static std::vector<std::string> type_list(const std::string& t) {
    std::string s = trim(t);
    if (!s.empty() && s[0] == '(' && s.back() == ')') {
      // a parenthesised list, unless it is a function type "(..) -> .."
      int depth = 0;
      size_t close = 0;
      for (size_t i = 0; i < s.size(); i++) {
        if (s[i] == '(') depth++;
        if (s[i] == ')' && --depth == 0) {
          close = i;
          break;
        }
      }
      if (close == s.size() - 1) {
        std::string inner = s.substr(1, s.size() - 2);
        if (trim(inner).empty()) return {};
        return split_top(inner, ',');
      }
    }
    return {s};
  }

  Block* parse_block_label(Region* r) {
    Block* b = m_.new_block();
    b->parent = r;
    b->label = ident();
    if (eat('(')) {
      if (!eat(')')) {
        for (;;) {
          std::string name = ident();
          expect(':');
          std::string ty = span(",)");
          // A trailing location belongs to the argument, not its type.
          std::string loc;
          if (const size_t k = top_level_loc(ty); k != std::string::npos) {
            loc = ty.substr(k + 1);
            ty.resize(k);
          }
          Value* v = m_.new_value(type_of(ty));
          v->loc = loc;
          v->owner = b;
          v->index = (int)b->args.size();
          v->name = name;
          b->args.push_back(v);
          define(name, {v});
          if (eat(')')) break;
          expect(',');
        }
      }
    }
    expect(':');
    return b;
  }

  Region* parse_region(Op* parent) {
    Region* r = m_.new_region();
    r->parent = parent;
    expect('{');
    Block* cur = nullptr;
    while (!peek('}')) {
      if (peek('^')) {
        cur = parse_block_label(r);
        r->blocks.push_back(cur);
        continue;
      }
      if (!cur) {
        cur = m_.new_block();
        cur->parent = r;
        r->blocks.push_back(cur);
      }
      parse_op(cur);
    }
    expect('}');
    return r;
  }

  Op* parse_op(Block* blk) {
    std::vector<std::pair<std::string, int>> res;  // name, count
    ws();
    if (peek('%')) {
      for (;;) {
        std::string name = ident();
        int count = 1;
        if (eat(':')) count = std::stoi(ident());
        res.emplace_back(name, count);
        if (!eat(',')) break;
      }
      expect('=');
    }
    ws();
    if (!eat('"')) fail("expected an op name string", p_);
    const size_t q = s_.find('"', p_);
    if (q == std::string::npos) fail("unterminated op name", p_);
    Op* op = m_.new_op(sub(p_, q - p_));
    p_ = q + 1;
    expect('(');
    std::vector<std::string> operand_refs;
    if (!eat(')')) {
      std::string list = span(")");
      expect(')');
      operand_refs = split_top(list, ',');
    }
    if (peek('[')) {
      const size_t a = p_;
      p_++;
      span("]");
      expect(']');
      op->successors = sub(a, p_ - a);
    }
    if (eat("<{")) {
      while (!peek('}')) {
        const auto r = span_pos(",}");
        const size_t eq = s_.find('=', r.first);
        if (eq == std::string::npos || eq >= r.second) {
          op->props.emplace_back(trim(sub(r.first, r.second - r.first)), "");
        } else {
          std::string key = trim(sub(r.first, eq - r.first));
          size_t va = eq + 1;
          while (va < r.second && isspace((unsigned char)s_[va])) va++;
          if (r.second - va > kBigProp) {
            op->big_key = key;
            op->big_value = std::string_view(s_.data() + va, r.second - va);
            op->props.emplace_back(std::move(key), "");
          } else {
            op->props.emplace_back(std::move(key), sub(va, r.second - va));
          }
        }
        if (!eat(',')) break;
      }
      expect('}');
      expect('>');
    }
    const bool isolated = op->name == "func.func" || op->name == "builtin.module";
    if (peek("({")) {
      expect('(');
      for (;;) {
        if (isolated) scopes_.emplace_back();
        op->regions.push_back(parse_region(op));
        if (isolated) close_scope();
        if (eat(')')) break;
        expect(',');
      }
    }
    if (peek('{')) {
      const size_t a = p_;
      p_++;
      span("}");
      expect('}');
      op->attrs = sub(a, p_ - a);
    }
    expect(':');
    std::string fnty = span("\n");
    // trailing location: the first " loc(" outside brackets and strings
    const size_t locp = top_level_loc(fnty);
    if (locp != std::string::npos) {
      op->loc = fnty.substr(locp + 1);
      fnty = trim(fnty.substr(0, locp));
    }
    const size_t arrow = [&] {
      int depth = 0;
      for (size_t i = 0; i + 1 < fnty.size(); i++) {
        const char c = fnty[i];
        if (c == '-' && fnty[i + 1] == '>') {  // an arrow, nested (a function type) or the top one
          if (depth == 0) return i;
          i++;
          continue;
        }
        if (c == '(' || c == '<' || c == '[' || c == '{') depth++;
        if (c == ')' || c == '>' || c == ']' || c == '}') depth--;
      }
      return std::string::npos;
    }();
    if (arrow == std::string::npos) fail("expected a function type", p_);
    const std::vector<std::string> in_types = type_list(fnty.substr(0, arrow));
    const std::vector<std::string> out_types = type_list(fnty.substr(arrow + 2));
    if (in_types.size() != operand_refs.size()) fail("operand count does not match the function type", p_);
    for (size_t i = 0; i < operand_refs.size(); i++) {
      Value* v = lookup(operand_refs[i], type_of(in_types[i]));
      op->operands.push_back(v);
      v->uses.push_back(op);
    }
    size_t total = 0;
    for (auto& r : res) total += (size_t)r.second;
    if (total != out_types.size()) fail("result count does not match the function type", p_);
    size_t k = 0;
    for (auto& r : res) {
      std::vector<Value*> vals;
      for (int i = 0; i < r.second; i++, k++) {
        Value* v = m_.new_value(type_of(out_types[k]));
        v->def = op;
        v->index = (int)k;
        op->results.push_back(v);
        vals.push_back(v);
      }
      define(r.first, vals);
    }
    if (res.empty())
      for (size_t i = 0; i < out_types.size(); i++) {
        Value* v = m_.new_value(type_of(out_types[i]));
        v->def = op;
        v->index = (int)i;
        op->results.push_back(v);
      }
    if (blk) m_.append(op, blk);
    attach_constant(op);
    return op;
  }

  // Decode the value of a constant-like op into a DenseValue.
  void attach_constant(Op* op) {
    if (op->name == "ub.poison") {
      if (op->results.size() == 1) {
        auto d = std::make_shared<DenseValue>();
        d->ty = op->results[0]->ty;
        d->poison = true;
        op->cst = d;
      }
      return;
    }
    const char* key = op->name == "arith.constant" ? "value" : op->name == "tosa.const" ? "values" : nullptr;
    if (!key || op->results.size() != 1) return;
    const std::string* text = op->prop(key);
    if (!text) return;
    const std::string_view full = (op->big_key == key) ? op->big_value : std::string_view(*text);
    // Big hex literals: only the ends are examined here; the hex body is
    // decoded (on the GPU) when the constant is first used.  Big literal
    // lists (i1 constants, which print as lists) are parsed below.
    const bool big_hex = full.size() > kBigProp && full.substr(0, 9) == "dense<\"0x";
    if (big_hex) {
      const size_t colon = full.rfind(" : ");
      const size_t q0 = full.find("\"0x"), q1 = full.rfind('"');
      if (colon == std::string_view::npos || q0 == std::string_view::npos || q1 <= q0) return;
      TypeP ty = type_of(std::string(full.substr(colon + 3)));
      if (!ty->dtype || !ty->static_shape() || ty->dtype == DCF_I1) return;
      auto d = std::make_shared<DenseValue>();
      d->ty = ty;
      d->dtype = ty->dtype;
      d->es = elem_bytes(ty->dtype);
      d->elements = true;
      d->hex = full.substr(q0 + 3, q1 - q0 - 3);
      const uint64_t bytes = d->hex.size() / 2;
      if (bytes != (uint64_t)ty->count() * d->es) return;
      d->n = (uint64_t)ty->count();
      op->cst = d;
      op->cst_text = true;
      return;
    }
    std::string lit(full), ty_text;
    // split "literal : type" at the last top-level " : "
    {
      auto parts = split_top(lit, ':');
      if (parts.size() >= 2) {
        ty_text = parts.back();
        lit = lit.substr(0, lit.rfind(':'));
        lit = trim(lit);
      }
    }
    TypeP ty = ty_text.empty() ? (lit == "true" || lit == "false" ? type_of("i1") : op->results[0]->ty)
                               : type_of(ty_text);
    if (!ty->dtype) return;
    auto d = std::make_shared<DenseValue>();
    d->ty = ty;
    d->dtype = ty->dtype;
    d->es = elem_bytes(ty->dtype);
    const bool is_float = ty->is_float();
    auto encode = [&](const std::string& tok, uint64_t* bits) {
      return is_float ? parse_float_literal(tok, ty->dtype, bits) : parse_int_literal(tok, ty->dtype, bits);
    };
    if (lit.rfind("dense<", 0) == 0) {
      if (!ty->static_shape()) return;
      d->elements = true;
      std::string body = trim(lit.substr(6, lit.size() - 7));
      if (body.size() > 3 && body[0] == '"' && body[1] == '0' && body[2] == 'x') {
        if (ty->dtype == DCF_I1) return;  // bit-packed in MLIR's raw form
        // Point into the attribute text (op->props, or the input for a big
        // literal).
        const size_t a = full.find("\"0x") + 3, b = full.find('"', a);
        if (a < 3 || b == std::string_view::npos) return;
        d->hex = full.substr(a, b - a);
        const uint64_t bytes = d->hex.size() / 2;
        if (bytes == d->es) {
          d->splat = true;
          d->n = 1;
        } else if (bytes == (uint64_t)ty->count() * d->es) {
          d->n = (uint64_t)ty->count();
        } else {
          return;
        }
      } else if (!body.empty() && body[0] == '(') {
        return;  // complex
      } else {
        std::vector<std::string> toks;
        flatten_list(body, toks);
        const bool list = !body.empty() && body[0] == '[';
        if (!list && toks.size() == 1) {
          d->splat = true;
        } else if ((int64_t)toks.size() != ty->count()) {
          return;
        }
        d->n = toks.size();
        d->host.resize(d->n * d->es);
        for (size_t i = 0; i < toks.size(); i++) {
          uint64_t bits;
          if (!encode(toks[i], &bits)) return;
          memcpy(d->host.data() + i * d->es, &bits, d->es);
        }
      }
    } else {
      if (ty->shaped()) return;
      uint64_t bits;
      if (!encode(lit, &bits)) return;
      d->splat = true;
      d->n = 1;
      d->host.resize(d->es);
      memcpy(d->host.data(), &bits, d->es);
    }
    op->cst = d;
    op->cst_text = !reformat_;
  }
};

}  // namespace

std::unique_ptr<Module> parse_module(std::string_view text, bool reformat) {
  auto m = std::make_unique<Module>();
  Parser p(text, *m, reformat);
  m->top = p.parse_top();
  return m;
}

// =================================================================== print

namespace {

class Printer {
 public:
  Printer(const PrintHooks& h) : h_(h) {}
  std::string out;

  // SSA names as the reference's generic printer spells them (Names::of,
  // src/ir.rs:2636-2650 with Namer, :2470-2635): one value counter and one
  // entry-block-argument counter for the whole module, never reset; regions
  // are named from a stack, so after a region's own blocks come the regions
  // nested in it, the last one first.  Entry-block arguments are %argK,
  // other block arguments and op results %N, an op with several results
  // %N:k with uses %N#i.
  void assign_names(Op* root) {
    uint64_t vnext = 0, anext = 0;
    std::vector<Region*> stack(root->regions.begin(), root->regions.end());
    while (!stack.empty()) {
      Region* r = stack.back();
      stack.pop_back();
      for (size_t bi = 0; bi < r->blocks.size(); bi++) {
        Block* b = r->blocks[bi];
        for (Value* a : b->args)
          names_[a] = bi == 0 ? "%arg" + std::to_string(anext++) : "%" + std::to_string(vnext++);
        for (Op* o : b->ops) {
          if (o->results.empty()) continue;
          const std::string name = "%" + std::to_string(vnext++);
          defs_[o] = name;
          for (size_t i = 0; i < o->results.size(); i++)
            names_[o->results[i]] = o->results.size() == 1 ? name : name + "#" + std::to_string(i);
        }
      }
      for (Block* b : r->blocks)
        for (Op* o : b->ops)
          for (Region* nr : o->regions) stack.push_back(nr);
    }
  }

  void op(Op* o, int indent) {
    out.append(indent, ' ');
    if (!o->results.empty()) {
      out += defs_[o];
      if (o->results.size() > 1) out += ":" + std::to_string(o->results.size());
      out += " = ";
    }
    out += "\"" + o->name + "\"(";
    for (size_t i = 0; i < o->operands.size(); i++) {
      if (i) out += ", ";
      out += name_of(o->operands[i]);
    }
    out += ")";
    if (!o->successors.empty()) out += successors(o);
    if (!o->props.empty() || (o->cst && !o->cst_text && !o->cst->poison)) {
      out += " <{";
      bool first = true;
      const char* key = o->name == "tosa.const" ? "values" : "value";
      bool wrote_value = false;
      for (auto& kv : o->props) {
        if (!first) out += ", ";
        first = false;
        out += kv.first;
        if (o->cst && !o->cst_text && !o->cst->poison && kv.first == key) {
          out += " = ";
          put_value(*o->cst);
          wrote_value = true;
        } else if (kv.first == o->big_key && !o->big_value.empty()) {
          out += " = ";
          defer(Fill::RAW, o->big_value.data(), o->big_value.size());
        } else if (!kv.second.empty()) {
          out += " = " + kv.second;
        }
      }
      if (o->cst && !o->cst_text && !wrote_value && !o->cst->poison) {
        if (!first) out += ", ";
        out += std::string(key) + " = ";
        put_value(*o->cst);
      }
      out += "}>";
    }
    if (!o->regions.empty()) {
      out += " (";
      for (size_t r = 0; r < o->regions.size(); r++) {
        if (r) out += ", ";
        region(o->regions[r], indent);
      }
      out += ")";
    }
    if (!o->attrs.empty()) out += " " + o->attrs;
    out += " : (";
    for (size_t i = 0; i < o->operands.size(); i++) {
      if (i) out += ", ";
      out += o->operands[i]->ty->text;
    }
    out += ") -> ";
    if (o->results.size() == 1 && o->results[0]->ty->text.find("->") == std::string::npos) {
      out += o->results[0]->ty->text;
    } else {
      out += "(";
      for (size_t i = 0; i < o->results.size(); i++) {
        if (i) out += ", ";
        out += o->results[i]->ty->text;
      }
      out += ")";
    }
    if (!o->loc.empty() && h_.debuginfo) out += " " + o->loc;
    out += "\n";
  }

  // A large literal body is not copied into the skeleton: its place is
  // recorded, and the final text is assembled from the skeleton and the
  // bodies by several threads (PrintedModule::write_to).
  using Fill = PrintedModule::Fill;
  std::vector<Fill> fills;
  static constexpr size_t kDeferBytes = 32768;

 private:
  const PrintHooks& h_;
  std::unordered_map<Value*, std::string> names_;

  std::unordered_map<Op*, std::string> defs_;

  void defer(Fill::Kind k, const void* src, size_t nchars) { fills.push_back({k, src, nchars, out.size()}); }

  // The successor list with every block label spelled ^bbN, N the block's
  // position in the region (as the reference prints labels).
  std::string successors(Op* o) {
    const std::string& t = o->successors;
    Region* r = o->parent ? o->parent->parent : nullptr;
    if (!r) return t;
    std::string res;
    for (size_t i = 0; i < t.size();) {
      if (t[i] != '^') {
        res += t[i++];
        continue;
      }
      size_t j = i + 1;
      while (j < t.size() && (isalnum((unsigned char)t[j]) || strchr("_$.-", t[j]))) j++;
      const std::string label = t.substr(i, j - i);
      size_t idx = r->blocks.size();
      for (size_t k = 0; k < r->blocks.size(); k++)
        if (r->blocks[k]->label == label) idx = k;
      res += idx < r->blocks.size() ? "^bb" + std::to_string(idx) : label;
      i = j;
    }
    return res;
  }

  std::string name_of(Value* v) {
    auto it = names_.find(v);
    if (it != names_.end()) return it->second;
    return "%<undefined>";
  }

  // Each block's predecessors, one entry per branch edge, by block index.
  static std::vector<std::vector<size_t>> predecessors(Region* r) {
    std::vector<std::vector<size_t>> preds(r->blocks.size());
    if (r->blocks.size() < 2) return preds;
    std::unordered_map<std::string_view, size_t> index;
    for (size_t k = 0; k < r->blocks.size(); k++) index.emplace(r->blocks[k]->label, k);
    for (size_t k = 0; k < r->blocks.size(); k++)
      for (Op* o : r->blocks[k]->ops)
        for_each_label(o->successors, [&](std::string_view l) {
          auto it = index.find(l);
          if (it != index.end()) preds[it->second].push_back(k);
        });
    return preds;
  }

  template <class F>
  static void for_each_label(const std::string& t, F&& f) {
    for (size_t i = 0; i < t.size(); i++) {
      if (t[i] != '^') continue;
      size_t j = i + 1;
      while (j < t.size() && (isalnum((unsigned char)t[j]) || strchr("_$.-", t[j]))) j++;
      f(std::string_view(t).substr(i, j - i));
      i = j - 1;
    }
  }

  // Blocks as mlir-opt writes them in the generic form: the entry block's
  // header only when it has arguments or no ops, every other block with a
  // comment naming its predecessors (sorted by position, one per edge).
  void region(Region* r, int indent) {
    out += "{\n";
    const auto preds = predecessors(r);
    for (size_t bi = 0; bi < r->blocks.size(); bi++) {
      Block* b = r->blocks[bi];
      if (!b->args.empty() || bi > 0 || b->ops.empty()) {
        out.append(indent, ' ');
        out += "^bb" + std::to_string(bi);
        if (!b->args.empty()) {
          out += "(";
          for (size_t i = 0; i < b->args.size(); i++) {
            if (i) out += ", ";
            out += names_[b->args[i]] + ": " + b->args[i]->ty->text;
            if (!b->args[i]->loc.empty() && h_.debuginfo) out += " " + b->args[i]->loc;
          }
          out += ")";
        }
        out += ":";
        if (bi > 0) {
          std::vector<size_t> p = preds[bi];
          std::sort(p.begin(), p.end());
          if (p.empty()) {
            out += "  // no predecessors";
          } else {
            out += p.size() == 1 ? "  // pred: " : "  // " + std::to_string(p.size()) + " preds: ";
            for (size_t k = 0; k < p.size(); k++) out += (k ? ", ^bb" : "^bb") + std::to_string(p[k]);
          }
        }
        out += "\n";
      }
      for (Op* o : b->ops) op(o, indent + 2);
    }
    out.append(indent, ' ');
    out += "}";
  }

  void put_value(DenseValue& v) {
    const bool large = v.n > 100 && v.dtype != DCF_I1 && !v.splat && v.elements;
    if (large && (!v.host.empty() || !v.hex.empty()) && v.bytes() >= kDeferBytes) {
      out += "dense<\"0x";
      if (!v.host.empty()) defer(Fill::HEX, v.host.data(), 2 * v.bytes());
      else defer(Fill::UPPER, v.hex.data(), v.hex.size());
      out += "\"> : " + v.ty->text;
      return;
    }
    out += value_text(v);
  }

  std::string value_text(DenseValue& v) {
    const bool is_float = v.ty->is_float();
    auto scalar = [&](uint64_t bits) {
      return is_float ? print_float_literal(bits, v.dtype) : print_int_literal(bits, v.dtype);
    };
    if (!v.elements) {
      const uint64_t bits = h_.bits0_of(v, h_.ctx);
      if (v.dtype == DCF_I1) return scalar(bits);
      return scalar(bits) + " : " + v.ty->text;
    }
    if (v.splat) return "dense<" + scalar(h_.bits0_of(v, h_.ctx)) + "> : " + v.ty->text;
    // mlir-opt prints up to 100 elements as a literal list and larger
    // attributes as the hex of their raw bytes.  MLIR's raw i1 data is
    // bit-packed, so i1 is always printed as a list here.
    if (v.n <= 100 || v.dtype == DCF_I1) {
      const std::string hex = h_.hex_of(v, h_.ctx);
      std::string s = "dense<";
      // nested brackets follow the shape
      // block[d]: elements in one list at nesting depth d
      const std::vector<int64_t>& shape = v.ty->shape;
      std::vector<uint64_t> block(shape.size(), 1);
      for (int i = (int)shape.size() - 1; i >= 0; i--)
        block[i] = (uint64_t)shape[i] * (i + 1 < (int)shape.size() ? block[i + 1] : 1);
      for (uint64_t e = 0; e < v.n; e++) {
        for (size_t d = 0; d < shape.size(); d++)
          if (e % block[d] == 0) s += "[";
        uint64_t bits = 0;
        for (size_t b = 0; b < v.es; b++) {
          const auto nib = [&](char c) { return (uint64_t)(c <= '9' ? c - '0' : c - 'A' + 10); };
          bits |= ((nib(hex[2 * (e * v.es + b)]) << 4) | nib(hex[2 * (e * v.es + b) + 1])) << (8 * b);
        }
        s += scalar(bits);
        for (size_t d = shape.size(); d-- > 0;)
          if ((e + 1) % block[d] == 0) s += "]";
        if (e + 1 < v.n) s += ", ";
      }
      return s + "> : " + v.ty->text;
    }
    return "dense<\"0x" + h_.hex_of(v, h_.ctx) + "\"> : " + v.ty->text;
  }
};

}  // namespace

// An upper estimate of the printed size, so the output grows without
// reallocating (and re-copying) the big literals.
static size_t estimate(const Op* o) {
  size_t n = 256 + o->big_value.size() + o->attrs.size();
  for (auto& kv : o->props) n += kv.first.size() + kv.second.size() + 4;
  if (o->cst && !o->cst_text) n += 2 * o->cst->bytes() + 64;
  for (const Region* r : o->regions)
    for (const Block* b : r->blocks)
      for (const Op* in : b->ops) n += estimate(in);
  return n;
}

// Names of the dense_resource blobs the module still refers to.
static void used_resources(const Op* o, std::vector<std::string>& out) {
  auto scan = [&](std::string_view t) {
    for (size_t at = t.find("dense_resource<"); at != std::string_view::npos; at = t.find("dense_resource<", at + 1)) {
      const size_t a = at + 15, b = t.find('>', a);
      if (b != std::string_view::npos) out.emplace_back(t.substr(a, b - a));
    }
  };
  for (auto& kv : o->props) scan(kv.second);
  scan(o->big_value);
  scan(o->attrs);
  for (const Region* r : o->regions)
    for (const Block* b : r->blocks)
      for (const Op* in : b->ops) used_resources(in, out);
}

// A metadata block as the reference prints it back
// (src/ir.rs:2951-2974): in a dialect_resources block only the blobs still
// used stay (the last kept one loses its trailing comma), and a block left
// with none is dropped.
static bool keep_resources(std::string_view body, const std::vector<std::string>& used, std::string& out) {
  if (body.find("dialect_resources") == std::string_view::npos) {
    out.assign(body);
    return true;
  }
  std::vector<std::string_view> lines;
  for (size_t a = 0;;) {
    const size_t b = body.find('\n', a);
    lines.push_back(body.substr(a, b == std::string_view::npos ? std::string_view::npos : b - a));
    if (b == std::string_view::npos) break;
    a = b + 1;
  }
  auto blob = [](std::string_view l) -> std::string_view {
    const size_t c = l.find(": \"0x");
    if (c == std::string_view::npos) return {};
    std::string_view k = l.substr(0, c);
    while (!k.empty() && isspace((unsigned char)k.front())) k.remove_prefix(1);
    while (!k.empty() && isspace((unsigned char)k.back())) k.remove_suffix(1);
    return k;
  };
  std::vector<std::string_view> kept;
  size_t n = 0;
  for (std::string_view l : lines) {
    const std::string_view k = blob(l);
    if (k.empty()) {
      kept.push_back(l);
      continue;
    }
    if (std::find(used.begin(), used.end(), std::string(k)) == used.end()) continue;
    kept.push_back(l);
    n++;
  }
  if (n == 0) return false;
  out.clear();
  size_t seen = 0;
  for (size_t i = 0; i < kept.size(); i++) {
    std::string_view l = kept[i];
    if (!blob(l).empty() && ++seen == n)
      while (!l.empty() && l.back() == ',') l.remove_suffix(1);
    if (i) out += '\n';
    out.append(l);
  }
  return true;
}

// Alias definition lines (`#name = ...`, `!name = ...`) that are printed,
// after Invocation::print_op (src/pass.rs:769-793): location aliases only
// with debuginfo, and of the others those the printed module uses (`#name`
// not followed by another name character), directly or through another
// printed alias.  `head` and `tail` receive the kept lines of the text
// before and after the module op.
struct AliasLine {
  std::string_view line, name;
  bool tail, loc, kept = false;
};

static bool names(std::string_view text, std::string_view name) {
  auto name_char = [](char c) { return isalnum((unsigned char)c) || strchr("_$.-", c); };
  for (size_t at = text.find(name); at != std::string_view::npos; at = text.find(name, at + 1))
    if (at + name.size() >= text.size() || !name_char(text[at + name.size()])) return true;
  return false;
}

static void kept_aliases(std::string_view pro, std::string_view epi, std::string_view rest, bool debuginfo,
                         std::string& head, std::string& tail) {
  auto name_char = [](char c) { return isalnum((unsigned char)c) || strchr("_$.-", c); };
  std::vector<AliasLine> al;
  for (int part = 0; part < 2; part++) {
    const std::string_view lines = part ? epi : pro;
    for (size_t a = 0; a < lines.size();) {
      size_t e = lines.find('\n', a);
      e = e == std::string_view::npos ? lines.size() : e + 1;
      const std::string_view line = lines.substr(a, e - a);
      a = e;
      if (line.empty() || (line[0] != '#' && line[0] != '!')) continue;
      size_t n = 1;
      while (n < line.size() && name_char(line[n])) n++;
      const size_t eq = line.find('=', n);
      if (eq == std::string_view::npos) continue;
      size_t v = eq + 1;
      while (v < line.size() && line[v] == ' ') v++;
      al.push_back({line, line.substr(0, n), part == 1, line[0] == '#' && line.compare(v, 4, "loc(") == 0});
    }
  }
  for (auto& x : al) x.kept = (debuginfo || !x.loc) && names(rest, x.name);
  for (bool grew = true; grew;) {
    grew = false;
    for (auto& x : al) {
      if (x.kept || (x.loc && !debuginfo)) continue;
      for (const auto& y : al)
        if (y.kept && names(y.line.substr(y.name.size()), x.name)) {
          x.kept = grew = true;
          break;
        }
    }
  }
  for (const auto& x : al) {
    if (!x.kept) continue;
    std::string& out = x.tail ? tail : head;
    out.append(x.line);
    if (out.back() != '\n') out += '\n';
  }
}

PrintedModule print_module_parts(Module& m, const PrintHooks& hooks) {
  Printer p(hooks);
  p.out.reserve(estimate(m.top) + m.prologue.size() + m.epilogue.size());
  p.assign_names(m.top);
  p.op(m.top, 0);
  std::string meta;
  if (!m.metadata.empty()) {
    std::vector<std::string> used;
    used_resources(m.top, used);
    for (std::string_view body : m.metadata) {
      std::string kept;
      if (!keep_resources(body, used, kept)) continue;
      meta += "\n{-#";
      meta += kept;
      meta += "#-}\n";
    }
  }
  if (!m.prologue.empty() || !m.epilogue.empty()) {
    const std::string rest = p.out + meta;
    std::string head, tail;
    kept_aliases(m.prologue, m.epilogue, rest, hooks.debuginfo, head, tail);
    p.out += tail;
    if (!head.empty()) {
      p.out.insert(0, head);
      for (auto& f : p.fills) f.at += head.size();
    }
  }
  p.out += meta;
  PrintedModule r;
  r.skeleton = std::move(p.out);
  r.fills = std::move(p.fills);
  r.size_ = r.skeleton.size();
  for (const auto& f : r.fills) r.size_ += f.nchars;
  return r;
}

namespace {

struct HexTable {
  uint16_t pair[256];
  HexTable() {
    static const char d[] = "0123456789ABCDEF";
    for (int b = 0; b < 256; b++) {
      const char c[2] = {d[b >> 4], d[b & 15]};
      memcpy(&pair[b], c, 2);
    }
  }
};

// Characters [c0, c1) of a body, written at dst.
void fill_part(const PrintedModule::Fill& f, size_t c0, size_t c1, char* dst) {
  switch (f.kind) {
    case PrintedModule::Fill::RAW:
      memcpy(dst, (const char*)f.src + c0, c1 - c0);
      break;
    case PrintedModule::Fill::UPPER: {
      const char* s = (const char*)f.src + c0;
      for (size_t i = 0; i < c1 - c0; i++) {
        const char c = s[i];
        dst[i] = (c >= 'a' && c <= 'f') ? (char)(c - 32) : c;
      }
      break;
    }
    case PrintedModule::Fill::HEX: {
      static const HexTable t;
      const uint8_t* b = (const uint8_t*)f.src + c0 / 2;  // c0, c1 even
      const size_t n = (c1 - c0) / 2;
      for (size_t i = 0; i < n; i++) memcpy(dst + 2 * i, &t.pair[b[i]], 2);
      break;
    }
  }
}

}  // namespace

void PrintedModule::write_to(char* dst) const {
  // Tasks: skeleton spans and body chunks of at most kChunk characters,
  // each with its output position; threads take them in order.
  constexpr size_t kChunk = 4u << 20;
  struct Task {
    const Fill* f;  // null: skeleton span
    size_t a, b;    // skeleton or body character range
    size_t out;
  };
  std::vector<Task> tasks;
  size_t pos = 0, sk = 0;
  auto span = [&](size_t a, size_t b) {
    for (size_t x = a; x < b; x += kChunk) {
      const size_t y = std::min(b, x + kChunk);
      tasks.push_back({nullptr, x, y, pos});
      pos += y - x;
    }
  };
  for (const Fill& f : fills) {
    span(sk, f.at);
    sk = f.at;
    for (size_t x = 0; x < f.nchars; x += kChunk) {
      const size_t y = std::min(f.nchars, x + kChunk);
      tasks.push_back({&f, x, y, pos});
      pos += y - x;
    }
  }
  span(sk, skeleton.size());
  std::atomic<size_t> next{0};
  auto work = [&] {
    for (size_t i; (i = next.fetch_add(1)) < tasks.size();) {
      const Task& t = tasks[i];
      if (t.f) fill_part(*t.f, t.a, t.b, dst + t.out);
      else memcpy(dst + t.out, skeleton.data() + t.a, t.b - t.a);
    }
  };
  const size_t hw = std::max(1u, std::thread::hardware_concurrency());
  const size_t nth = std::min<size_t>({hw, 32, (size_ >> 22) + 1});
  std::vector<std::thread> th;
  for (size_t i = 1; i < nth; i++) th.emplace_back(work);
  work();
  for (auto& t : th) t.join();
}

std::string PrintedModule::str() const {
  std::string s(size_, '\0');
  write_to(&s[0]);
  return s;
}

std::string print_module(Module& m, const PrintHooks& hooks) { return print_module_parts(m, hooks).str(); }

}  // namespace dco
