// fold.cpp — fold hooks, the resumable greedy driver and the pass pipeline
// of dcfold-opt.  See fold.h for the reference code each part restates.
#include "fold.h"

#include <algorithm>
#include <cstring>
#include <stdexcept>
#include <thread>
#include <unordered_map>

namespace dco {

namespace {

// ------------------------------------------------------------ IR helpers

bool constant_like(const Op* op) {
  return op->name == "arith.constant" || op->name == "tosa.const" || op->name == "ub.poison" ||
         op->name == "tosa.const_shape";
}

DenseP constant_of(Value* v) { return (v->def && constant_like(v->def)) ? v->def->cst : nullptr; }

bool side_effect_free(const Op* op) {
  if (!op->regions.empty()) return false;
  const std::string d = op->dialect();
  return d == "arith" || d == "tosa" || d == "math" || d == "ub";
}

bool isolated(const Op* op) { return op->name == "func.func" || op->name == "builtin.module"; }

int int_width(int dtype) {
  switch (dtype) {
    case DCF_I1: return 1;
    case DCF_I8: return 8;
    case DCF_I16: return 16;
    case DCF_I32: return 32;
    case DCF_I64: return 64;
    default: return 0;
  }
}

uint64_t wmask(int w) { return w >= 64 ? ~0ull : ((1ull << w) - 1); }

struct FloatBits {
  int E, M;
};

bool float_layout(int dtype, FloatBits* f) {
  switch (dtype) {
    case DCF_F16: *f = {5, 10}; return true;
    case DCF_BF16: *f = {8, 7}; return true;
    case DCF_F32: *f = {8, 23}; return true;
    case DCF_F64: *f = {11, 52}; return true;
    case DCF_F8E5M2: *f = {5, 2}; return true;
    case DCF_F8E4M3: *f = {4, 3}; return true;
    case DCF_F8E3M4: *f = {3, 4}; return true;
    default: return false;
  }
}

bool f_is_zero(uint64_t b, FloatBits f) { return (b & ((1ull << (f.E + f.M)) - 1)) == 0; }
bool f_neg(uint64_t b, FloatBits f) { return (b >> (f.E + f.M)) & 1; }
bool f_is_nan(uint64_t b, FloatBits f) {
  const uint64_t em = ((1ull << f.E) - 1) << f.M;
  return (b & em) == em && (b & ((1ull << f.M) - 1));
}
bool f_is_inf(uint64_t b, FloatBits f) {
  const uint64_t em = ((1ull << f.E) - 1) << f.M;
  return (b & (em | ((1ull << f.M) - 1))) == em;
}
bool f_is_one(uint64_t b, FloatBits f) {
  const uint64_t bias = (1ull << (f.E - 1)) - 1;
  return b == (bias << f.M);
}

int64_t parse_int_prop(const std::string& s, bool* ok) {
  const std::string t = s.substr(0, s.find(':'));
  char* end = nullptr;
  const long long v = strtoll(t.c_str(), &end, 10);
  *ok = end != t.c_str();
  return v;
}

// fastmath_has (canonicalize.rs:79-85)
bool fastmath_has(const std::string* a, std::initializer_list<const char*> flags) {
  if (!a) return false;
  const size_t l = a->find('<'), r = a->rfind('>');
  if (l == std::string::npos || r == std::string::npos) return false;
  std::vector<std::string> set;
  std::string cur;
  for (size_t i = l + 1; i < r; i++) {
    const char c = (*a)[i];
    if (c == ',') {
      set.push_back(cur);
      cur.clear();
    } else if (c != ' ') {
      cur += c;
    }
  }
  set.push_back(cur);
  auto has = [&](const char* f) { return std::find(set.begin(), set.end(), f) != set.end(); };
  if (has("fast")) return true;
  for (const char* f : flags)
    if (!has(f)) return false;
  return true;
}

// overflow flags of a muli (canonicalize.rs:20-24): bit 0 nsw, bit 1 nuw
int overflow_bits(const std::string* a) {
  if (!a) return 0;
  return (a->find("nsw") != std::string::npos ? 1 : 0) | (a->find("nuw") != std::string::npos ? 2 : 0);
}

std::vector<int64_t> parse_array_prop(const std::string* a) {
  std::vector<int64_t> out;
  if (!a) return out;
  const size_t c = a->find(':');
  if (c == std::string::npos) return out;
  std::string body = a->substr(c + 1);
  if (!body.empty() && body.back() == '>') body.pop_back();
  size_t p = 0;
  while (p < body.size()) {
    const size_t q = body.find(',', p);
    const std::string tok = body.substr(p, q == std::string::npos ? std::string::npos : q - p);
    if (tok.find_first_not_of(" ") != std::string::npos) out.push_back(std::stoll(tok));
    if (q == std::string::npos) break;
    p = q + 1;
  }
  return out;
}

DenseP splat_value(TypeP ty, uint64_t bits) {
  auto d = std::make_shared<DenseValue>();
  d->ty = ty;
  d->elements = ty->shaped();
  d->splat = true;
  d->dtype = ty->dtype;
  d->es = dcf_dtype_size((dcf_dtype)ty->dtype);
  d->n = 1;
  d->host.resize(d->es);
  memcpy(d->host.data(), &bits, d->es);
  return d;
}

// ------------------------------------------------------------- fold plans

struct Plan {
  enum K { FAILED, INPLACE, VALUE, ATTR, DEVICE, MULTI } k = FAILED;
  Value* value = nullptr;
  DenseP attr;
  std::unique_ptr<FoldRequest> req;
  // MULTI (Fold::Results): one part per result, a value or an attribute.
  std::vector<std::pair<Value*, DenseP>> parts;
  static Plan multi(std::vector<std::pair<Value*, DenseP>> ps) {
    Plan p;
    for (auto& x : ps)
      if (!x.first && !x.second) return p;
    p.k = MULTI;
    p.parts = std::move(ps);
    return p;
  }
  static Plan failed() { return Plan{}; }
  static Plan inplace() {
    Plan p;
    p.k = INPLACE;
    return p;
  }
  static Plan of_value(Value* v) {
    Plan p;
    p.k = VALUE;
    p.value = v;
    return p;
  }
  static Plan of_attr(DenseP a) {
    Plan p;
    if (!a) return p;
    p.k = ATTR;
    p.attr = std::move(a);
    return p;
  }
  static Plan device(std::unique_ptr<FoldRequest> r) {
    Plan p;
    p.k = DEVICE;
    p.req = std::move(r);
    return p;
  }
};

// zero_attr (canonicalize.rs:245-256): a zero splat of `ty`.
DenseP zero_attr(const TypeP& ty) {
  if (!ty->dtype || ty->kind == "other") return nullptr;
  if (ty->shaped() && ty->dynamic) return nullptr;
  return splat_value(ty, 0);
}

// bool_attr (canonicalize.rs:258-264)
DenseP bool_attr(const TypeP& ty, bool v) {
  if (ty->shaped()) {
    if (ty->dynamic) return nullptr;
    return splat_value(with_element(ty, "i1"), v ? 1 : 0);
  }
  return splat_value(type_of("i1"), v ? 1 : 0);
}

class ArithFolder {
 public:
  ArithFolder(Module& m, Op* op, Engine& e) : m_(m), op_(op), eng_(e) {
    for (Value* v : op->operands) c_.push_back(constant_of(v));
  }

  // ArithFolder::math, src/patterns/math/canonicalize.rs:145-234.  The
  // exact element folds run on the GPU; the classification ops decide on
  // the host from a splat operand (:136-143); the inexact ones (sin, exp,
  // log, pow, ...; the host C library's results in the reference) are not
  // folded.
  Plan math() {
    const std::string& name = op_->name;
    if (name.rfind("math.", 0) != 0 || op_->results.size() != 1) return Plan::failed();
    const std::string o = name.substr(5);
    static const std::pair<const char*, int> float_ops[] = {
        {"absf", DCF_ABSF},   {"ceil", DCF_CEIL},   {"floor", DCF_FLOOR}, {"roundeven", DCF_ROUNDEVEN},
        {"round", DCF_ROUND}, {"trunc", DCF_TRUNC}, {"sqrt", DCF_SQRT},   {"rsqrt", DCF_RSQRT}};
    static const std::pair<const char*, int> int_ops[] = {
        {"absi", DCF_ABSI}, {"ctlz", DCF_CTLZ}, {"cttz", DCF_CTTZ}, {"ctpop", DCF_CTPOP}};
    for (const auto& [n, code] : float_ops)
      if (o == n) return float_unary(code);
    for (const auto& [n, code] : int_ops)
      if (o == n) {
        if (!element_type(ty())->is_int()) return Plan::failed();
        return unary(code, element_type(ty())->dtype);
      }
    if (o == "copysign") return binary(DCF_COPYSIGN, 0, nullptr);
    if (o == "ipowi") return binary(DCF_IPOWI, 0, nullptr);
    if (o == "isfinite" || o == "isinf" || o == "isnan" || o == "isnormal") return classify(o);
    return Plan::failed();
  }

  // ArithFolder::fold, src/patterns/arith/canonicalize.rs:270-491.
  Plan fold() {
    const std::string& name = op_->name;
    if (name.rfind("arith.", 0) != 0) return Plan::failed();
    const std::string o = name.substr(6);
    if (op_->results.size() == 2) {  // the *_extended ops (Fold::Results)
      if (o == "addui_extended") return addui_extended();
      if (o == "subui_extended") return subui_extended();
      if (o == "mulsi_extended" || o == "mului_extended") return mul_extended(o == "mulsi_extended");
      return Plan::failed();
    }
    if (op_->results.size() != 1) return Plan::failed();
    uint64_t x;
    if (o == "addi") return addi();
    if (o == "subi") return subi();
    if (o == "muli") {
      if (zero(1)) return Plan::of_value(v(1));
      if (one(1)) return Plan::of_value(v(0));
      return int_binary(DCF_MULI);
    }
    if (o == "divui" || o == "divsi") return div(o == "divsi");
    if (o == "remui" || o == "remsi") {
      if (one(1)) return Plan::of_attr(zero_attr(ty()));
      return int_binary(o == "remsi" ? DCF_REMSI : DCF_REMUI);
    }
    if (o == "andi") return andi();
    if (o == "ori") return ori();
    if (o == "xori") return xori();
    if (o == "addf") {
      if (float_(1, &x) && f_is_zero(x, fl()) && f_neg(x, fl())) return Plan::of_value(v(0));
      return rounded_binary(DCF_ADDF);
    }
    if (o == "subf") {
      if (float_(1, &x) && f_is_zero(x, fl()) && !f_neg(x, fl())) return Plan::of_value(v(0));
      return rounded_binary(DCF_SUBF);
    }
    if (o == "maximumf" || o == "minimumf" || o == "maxnumf" || o == "minnumf") {
      if (v(0) == v(1)) return Plan::of_value(v(1));
      const bool max = o.rfind("max", 0) == 0;
      const bool nan_wins = o.size() > 5 && o.substr(o.size() - 5) == "imumf";
      if (float_(1, &x)) {
        const bool skip = nan_wins ? (f_is_inf(x, fl()) && f_neg(x, fl()) == max) : f_is_nan(x, fl());
        if (skip) return Plan::of_value(v(0));
      }
      const int dop = o == "maximumf" ? DCF_MAXIMUMF : o == "minimumf" ? DCF_MINIMUMF
                      : o == "maxnumf"   ? DCF_MAXNUMF
                                         : DCF_MINNUMF;
      return binary(dop, 0, nullptr);
    }
    if (o == "maxsi" || o == "maxui" || o == "minsi" || o == "minui") return int_minmax(o);
    if (o == "mulf") {
      if (float_(1, &x) && f_is_one(x, fl())) return Plan::of_value(v(0));
      if (fastmath_has(op_->prop("fastmath"), {"nnan", "nsz"}) && float_(1, &x) && f_is_zero(x, fl()))
        return Plan::of_value(v(1));
      return rounded_binary(DCF_MULF);
    }
    if (o == "divf") {
      if (float_(1, &x) && f_is_one(x, fl())) return Plan::of_value(v(0));
      return rounded_binary(DCF_DIVF);
    }
    if (o == "extf") return extf();
    if (o == "truncf") return truncf();
    if (o == "uitofp" || o == "sitofp") {
      if (!element_type(ty())->is_float()) return Plan::failed();
      return unary(o == "sitofp" ? DCF_SITOFP : DCF_UITOFP, element_type(ty())->dtype);
    }
    if (o == "fptoui" || o == "fptosi") {
      if (!element_type(ty())->is_int()) return Plan::failed();
      return unary(o == "fptosi" ? DCF_FPTOSI : DCF_FPTOUI, element_type(ty())->dtype);
    }
    if (o == "cmpi") return cmpi();
    if (o == "cmpf") return cmpf();
    if (o == "shli" || o == "shrui" || o == "shrsi") {
      if (zero(1)) return Plan::of_value(v(0));
      return int_binary(o == "shli" ? DCF_SHLI : o == "shrui" ? DCF_SHRUI : DCF_SHRSI);
    }
    if (o == "ceildivui" || o == "ceildivsi" || o == "floordivsi") {  // :287-317
      if (one(1)) return Plan::of_value(v(0));
      return int_binary(o == "ceildivui" ? DCF_CEILDIVUI : o == "ceildivsi" ? DCF_CEILDIVSI : DCF_FLOORDIVSI);
    }
    if (o == "remf") return binary(DCF_REMF, 0, nullptr);  // :387
    if (o == "negf") {                                       // :327-333
      if (Op* inner = def(0, "arith.negf")) return Plan::of_value(inner->operands[0]);
      return float_unary(DCF_NEGF);
    }
    if (o == "flush_denormals") {                            // :376-385
      if (Op* inner = def(0, "arith.flush_denormals")) return Plan::of_value(inner->results[0]);
      return float_unary(DCF_FLUSH_DENORMALS);
    }
    if (o == "convertf") return float_convert(DCF_TRUNCF);  // :386
    if (o == "extui" || o == "extsi") {                      // :388-398
      if (Op* inner = def(0, name.c_str())) {
        m_.set_operand(op_, 0, inner->operands[0]);
        return Plan::of_value(res());
      }
      if (!element_type(ty())->is_int()) return Plan::failed();
      return unary(o == "extsi" ? DCF_EXTSI : DCF_EXTUI, element_type(ty())->dtype);
    }
    if (o == "trunci") return trunci();
    if (o == "index_cast" || o == "index_castui") return index_cast(o == "index_cast");
    if (o == "bitcast") return bitcast();
    if (o == "select") return select();
    return Plan::failed();
  }

 private:
  Module& m_;
  Op* op_;
  Engine& eng_;
  std::vector<DenseP> c_;

  Value* v(size_t i) { return op_->operands[i]; }
  Value* res() { return op_->results[0]; }
  TypeP ty() { return res()->ty; }
  FloatBits fl() {
    FloatBits f{8, 23};
    float_layout(element_type(v(1)->ty)->dtype, &f);
    return f;
  }
  DenseP cst(size_t i) { return (i < c_.size() && c_[i] && !c_[i]->poison) ? c_[i] : nullptr; }
  bool poison(size_t i) { return i < c_.size() && c_[i] && c_[i]->poison; }
  // Const::as_int / as_float: a value for a one-element (splat) Const.
  bool int_(size_t i, uint64_t* b) {
    DenseP k = cst(i);
    if (!k || !k->splat || !k->ty->is_int()) return false;
    *b = eng_.bits0_of(*k) & wmask(int_width(k->dtype));
    return true;
  }
  bool float_(size_t i, uint64_t* b) {
    DenseP k = cst(i);
    if (!k || !k->splat || !k->ty->is_float()) return false;
    *b = eng_.bits0_of(*k);
    return true;
  }
  bool zero(size_t i) {
    uint64_t b;
    return int_(i, &b) && b == 0;
  }
  bool one(size_t i) {
    uint64_t b;
    return int_(i, &b) && b == 1;
  }
  bool all_ones(size_t i) {
    uint64_t b;
    return int_(i, &b) && b == wmask(int_width(cst(i)->dtype));
  }
  Op* def(size_t i, const char* name) {
    Op* d = v(i)->def;
    return (d && !d->erased && d->name == name) ? d : nullptr;
  }
  bool const_all_ones(Value* x) {
    DenseP k = constant_of(x);
    if (!k || k->poison || !k->splat || !k->ty->is_int()) return false;
    return (eng_.bits0_of(*k) & wmask(int_width(k->dtype))) == wmask(int_width(k->dtype));
  }

  // Folder::binary, canonicalize.rs:203-217: the element loop becomes a
  // FoldRequest; everything before it is decided here.
  Plan binary(int dop, uint32_t flags, TypeP result_ty) {
    for (size_t i = 0; i < 2; i++)
      if (poison(i)) return Plan::of_attr(c_[i]);
    DenseP l = cst(0), r = cst(1);
    if (!l || !r) return Plan::failed();
    if (l->ty->text != r->ty->text || l->elements != r->elements) return Plan::failed();
    TypeP rty = result_ty ? result_ty : l->ty;
    if (!rty->dtype) return Plan::failed();
    auto q = std::make_unique<FoldRequest>();
    q->kind = FoldRequest::BINARY;
    q->op = dop;
    q->dtype = l->dtype;
    q->out_dtype = rty->dtype;
    q->flags = flags;
    q->lhs = l;
    q->rhs = r;
    q->n = (l->splat && r->splat) ? 1 : std::max(l->n, r->n);
    q->out_ty = rty;
    q->out_elements = l->elements;
    return Plan::device(std::move(q));
  }
  Plan int_binary(int dop) { return binary(dop, 0, nullptr); }

  // rounded_binary, canonicalize.rs:916-926
  Plan rounded_binary(int dop) {
    uint32_t mode = 0;
    if (const std::string* rm = op_->prop("roundingmode")) {
      bool ok;
      const int64_t m = parse_int_prop(*rm, &ok);
      if (!ok || m < 0 || m > 4) return Plan::failed();
      mode = (uint32_t)m;
    }
    return binary(dop, mode, nullptr);
  }

  // Folder::unary, canonicalize.rs:227-235
  Plan unary(int dop, int out_dtype) {
    if (poison(0)) return Plan::of_attr(c_[0]);
    DenseP k = cst(0);
    if (!k) return Plan::failed();
    TypeP target = k->elements ? ty() : element_type(ty());
    auto q = std::make_unique<FoldRequest>();
    q->kind = FoldRequest::CONVERT;
    q->op = dop;
    q->dtype = k->dtype;
    q->out_dtype = out_dtype;
    q->lhs = k;
    q->n = k->n;
    q->out_ty = target;
    q->out_elements = k->elements;
    return Plan::device(std::move(q));
  }

  Plan addi() {  // :493-508
    if (zero(1)) return Plan::of_value(v(0));
    if (Op* sub = def(0, "arith.subi"))
      if (v(1) == sub->operands[1]) return Plan::of_value(sub->operands[0]);
    if (Op* sub = def(1, "arith.subi"))
      if (v(0) == sub->operands[1]) return Plan::of_value(sub->operands[0]);
    return int_binary(DCF_ADDI);
  }

  Plan subi() {  // :510-536
    if (v(0) == v(1) && !(ty()->shaped() && ty()->dynamic)) return Plan::of_attr(zero_attr(ty()));
    if (zero(1)) return Plan::of_value(v(0));
    if (Op* sub = def(1, "arith.subi"))
      if (sub->operands[0] == v(0)) return Plan::of_value(sub->operands[1]);
    if (Op* add = def(0, "arith.addi")) {
      Value *x = add->operands[0], *y = add->operands[1];
      if (v(1) == y) return Plan::of_value(x);
      if (v(1) == x) return Plan::of_value(y);
    }
    return int_binary(DCF_SUBI);
  }

  Plan div(bool is_signed) {  // :538-555
    if (one(1)) return Plan::of_value(v(0));
    if (Op* mul = def(0, "arith.muli")) {
      const int need = is_signed ? 1 : 2;
      if ((overflow_bits(mul->prop("overflowFlags")) & need) == need) {
        Value *x = mul->operands[0], *y = mul->operands[1];
        if (x == v(1)) return Plan::of_value(y);
        if (y == v(1)) return Plan::of_value(x);
      }
    }
    return int_binary(is_signed ? DCF_DIVSI : DCF_DIVUI);
  }

  Plan andi() {  // :597-620
    if (zero(1)) return Plan::of_value(v(1));
    if (all_ones(1)) return Plan::of_value(v(0));
    for (auto [x, other] : {std::pair<size_t, size_t>{0, 1}, {1, 0}})
      if (Op* xr = def(other, "arith.xori"))
        if (xr->operands[0] == v(x) && const_all_ones(xr->operands[1])) return Plan::of_attr(zero_attr(ty()));
    for (auto [prev, other] : {std::pair<size_t, size_t>{0, 1}, {1, 0}})
      if (Op* p = def(prev, "arith.andi"))
        if (std::find(p->operands.begin(), p->operands.end(), v(other)) != p->operands.end())
          return Plan::of_value(p->results[0]);
    return int_binary(DCF_ANDI);
  }

  Plan ori() {  // :622-640
    uint64_t r;
    if (int_(1, &r)) {
      if (r == 0) return Plan::of_value(v(0));
      if (r == wmask(int_width(cst(1)->dtype))) return Plan::of_attr(c_[1]);
    }
    for (auto [x, other] : {std::pair<size_t, size_t>{0, 1}, {1, 0}})
      if (Op* xr = def(other, "arith.xori"))
        if (xr->operands[0] == v(x) && const_all_ones(xr->operands[1])) return Plan::of_value(xr->operands[1]);
    return int_binary(DCF_ORI);
  }

  Plan xori() {  // :642-661
    if (zero(1)) return Plan::of_value(v(0));
    if (v(0) == v(1)) return Plan::of_attr(zero_attr(ty()));
    for (auto [prev, other] : {std::pair<size_t, size_t>{0, 1}, {1, 0}})
      if (Op* p = def(prev, "arith.xori")) {
        Value *pl = p->operands[0], *pr = p->operands[1];
        if (pr == v(other)) return Plan::of_value(pl);
        if (pl == v(other)) return Plan::of_value(pr);
      }
    return int_binary(DCF_XORI);
  }

  Plan int_minmax(const std::string& o) {  // :663-683
    if (v(0) == v(1)) return Plan::of_value(v(1));
    const bool is_signed = o.substr(o.size() - 2) == "si";
    const bool max = o.rfind("max", 0) == 0;
    uint64_t r;
    if (int_(1, &r)) {
      const int w = int_width(cst(1)->dtype);
      const uint64_t lo = is_signed ? (1ull << (w - 1)) : 0, hi = is_signed ? (wmask(w) >> 1) : wmask(w);
      if (r == (max ? hi : lo)) return Plan::of_value(v(1));
      if (r == (max ? lo : hi)) return Plan::of_value(v(0));
    }
    const int dop = o == "maxsi" ? DCF_MAXSI : o == "maxui" ? DCF_MAXUI : o == "minsi" ? DCF_MINSI : DCF_MINUI;
    return int_binary(dop);
  }

  Plan extf() {  // :717-725
    if (Op* t = def(0, "arith.truncf")) {
      Value* src = t->operands[0];
      if (src->ty->text == ty()->text && fastmath_has(t->prop("fastmath"), {"contract"}) &&
          fastmath_has(op_->prop("fastmath"), {"contract"}))
        return Plan::of_value(src);
    }
    return float_convert(DCF_EXTF);
  }

  // representable_by (canonicalize.rs:1057-1073)
  static bool representable_by(int a, int b) {
    auto rank = [](int k, int* e, int* p) {
      switch (k) {
        case DCF_F16: *e = 5, *p = 11; return true;
        case DCF_BF16: *e = 8, *p = 8; return true;
        case DCF_F32: *e = 8, *p = 24; return true;
        case DCF_F64: *e = 11, *p = 53; return true;
        default: return false;
      }
    };
    int ea, pa, eb, pb;
    if (rank(a, &ea, &pa) && rank(b, &eb, &pb)) return ea <= eb && pa <= pb;
    return a == b;
  }

  Plan truncf() {  // :744-762
    if (Op* e = def(0, "arith.extf")) {
      Value* src = e->operands[0];
      const int s = element_type(src->ty)->dtype, mid = element_type(e->results[0]->ty)->dtype,
                r = element_type(ty())->dtype;
      if (s && mid && r && representable_by(s, mid)) {
        const size_t sw = dcf_dtype_size((dcf_dtype)s), rw = dcf_dtype_size((dcf_dtype)r);
        if (sw > rw) {
          m_.set_operand(op_, 0, src);
          return Plan::of_value(res());
        }
        if (s == r) return Plan::of_value(src);
      }
    }
    return float_convert(DCF_TRUNCF);
  }

  // The second result of a two-result fold: a second kernel over the same
  // operands, writing `dtype` elements of type `ty`.
  static Plan with_second(Plan p, int op2, uint32_t flags2, int dtype2, TypeP ty2) {
    if (p.k == Plan::ATTR) return Plan::multi({{nullptr, p.attr}, {nullptr, p.attr}});  // poison in, poison out
    if (p.k != Plan::DEVICE) return Plan::failed();
    p.req->op2 = op2;
    p.req->flags2 = flags2;
    p.req->out2_dtype = dtype2;
    p.req->out2_ty = std::move(ty2);
    return p;
  }

  Plan addui_extended() {  // :878-893
    const TypeP ovt = op_->results[1]->ty;
    if (zero(1)) return Plan::multi({{v(0), nullptr}, {nullptr, zero_attr(ovt)}});
    Plan sum = binary(DCF_ADDI, 0, nullptr);
    if (sum.k != Plan::DEVICE) return with_second(std::move(sum), 0, 0, 0, nullptr);
    TypeP i1 = with_element(sum.req->out_ty, "i1");
    return with_second(std::move(sum), DCF_ADDUI_CARRY, 0, DCF_I1, i1);
  }

  Plan subui_extended() {  // :895-914
    const TypeP bt = op_->results[1]->ty;
    if (zero(1)) return Plan::multi({{v(0), nullptr}, {nullptr, zero_attr(bt)}});
    if (v(0) == v(1)) return Plan::multi({{nullptr, zero_attr(op_->results[0]->ty)}, {nullptr, zero_attr(bt)}});
    Plan diff = binary(DCF_SUBI, 0, nullptr);
    if (diff.k != Plan::DEVICE) return with_second(std::move(diff), 0, 0, 0, nullptr);
    TypeP i1 = with_element(diff.req->out_ty, "i1");
    return with_second(std::move(diff), DCF_CMPI, DCF_FLAG_PRED(6), DCF_I1, i1);  // borrow: a <u b
  }

  Plan mul_extended(bool is_signed) {  // :928-949
    if (zero(1)) return Plan::multi({{nullptr, c_[1]}, {nullptr, c_[1]}});
    if (!is_signed && one(1)) return Plan::multi({{v(0), nullptr}, {nullptr, zero_attr(v(0)->ty)}});
    Plan low = binary(DCF_MULI, 0, nullptr);
    if (low.k != Plan::DEVICE) return with_second(std::move(low), 0, 0, 0, nullptr);
    TypeP t = low.req->out_ty;
    const int dt = low.req->out_dtype;
    return with_second(std::move(low), is_signed ? DCF_MULSI_HI : DCF_MULUI_HI, 0, dt, t);
  }

  Plan float_unary(int dop) {
    if (!element_type(ty())->is_float()) return Plan::failed();
    return unary(dop, element_type(ty())->dtype);
  }

  static int width_or(Value* x, int dflt) {
    const TypeP e = element_type(x->ty);
    return e->is_int() ? int_width(e->dtype) : dflt;
  }

  Plan trunci() {  // :685-706
    const int res_w = width_or(res(), 0);
    for (const char* ext : {"arith.extui", "arith.extsi"})
      if (Op* e = def(0, ext)) {
        Value* src = e->operands[0];
        if (width_or(src, 0) > res_w) {
          m_.set_operand(op_, 0, src);
          return Plan::of_value(res());
        }
        if (element_type(src->ty)->text == element_type(ty())->text) return Plan::of_value(src);
      }
    if (Op* t = def(0, "arith.trunci")) {
      m_.set_operand(op_, 0, t->operands[0]);
      return Plan::of_value(res());
    }
    if (!res_w) return Plan::failed();
    return unary(DCF_TRUNCI, element_type(ty())->dtype);
  }

  // index_cast / index_castui (:435-454); index is a 64-bit integer.
  Plan index_cast(bool is_signed) {
    const int w = width_or(res(), 64);
    if (DenseP k = cst(0)) {
      if (!k->ty->is_int()) return Plan::failed();
      const int wi = int_width(k->dtype);
      const int dop = w < wi ? DCF_TRUNCI : (is_signed ? DCF_EXTSI : DCF_EXTUI);
      return unary(dop, element_type(ty())->dtype);
    }
    if (Op* inner = def(0, op_->name.c_str())) {
      Value* x = inner->operands[0];
      if (x->ty->text == ty()->text && width_or(inner->results[0], 64) >= width_or(x, 64)) return Plan::of_value(x);
    }
    return Plan::failed();
  }

  // bitcast (:764-789): the same bits under the result's element type, so
  // no element work; the new constant shares the operand's bytes.
  // Folder::classify (math/canonicalize.rs:136-143): a splat float operand
  // gives an i1 splat (a scalar for a scalar operand).
  Plan classify(const std::string& o) {
    DenseP k = cst(0);
    FloatBits f;
    if (!k || !k->splat || !k->ty->is_float() || !float_layout(k->dtype, &f)) return Plan::failed();
    const uint64_t b = eng_.bits0_of(*k), emax = (1ull << f.E) - 1;
    const uint64_t e = (b >> f.M) & emax, m = b & ((1ull << f.M) - 1);
    const bool nan = e == emax && m != 0, inf = e == emax && m == 0;
    bool v;
    if (o == "isfinite") v = !nan && !inf;
    else if (o == "isinf") v = inf;
    else if (o == "isnan") v = nan;
    else v = e != 0 && e != emax;  // FloatFolds::is_normal (:94-98)
    TypeP rty = ty();
    if (!element_type(rty)->is_int() || (rty->shaped() && rty->dynamic)) return Plan::failed();
    return Plan::of_attr(splat_value(rty, v ? 1 : 0));
  }

  Plan bitcast() {
    if (!c_.size() || !c_[0]) return Plan::failed();
    DenseP a = c_[0];
    if (a->poison) return ty()->shaped() ? Plan::failed() : Plan::of_attr(a);
    if (!a->elements && ty()->shaped()) return Plan::failed();
    const TypeP target = a->elements ? ty() : element_type(ty());
    if (!target->dtype || dcf_dtype_size((dcf_dtype)target->dtype) != a->es) return Plan::failed();
    auto d = std::make_shared<DenseValue>(*a);
    d->ty = target;
    d->dtype = target->dtype;
    return Plan::of_attr(d);
  }

  Plan select() {  // :841-876
    Value *c = v(0), *t = v(1), *f = v(2);
    if (t == f) return Plan::of_value(t);
    if (one(0)) return Plan::of_value(t);
    if (zero(0)) return Plan::of_value(f);
    if (poison(1)) return Plan::of_value(f);
    if (poison(2)) return Plan::of_value(t);
    if (!ty()->shaped() && ty()->dtype == DCF_I1 && one(1) && zero(2)) return Plan::of_value(c);
    if (Op* cmp = c->def; cmp && !cmp->erased && cmp->name == "arith.cmpi") {
      bool ok = false;
      const std::string* pp = cmp->prop("predicate");
      const int64_t p = pp ? parse_int_prop(*pp, &ok) : -1;
      if (ok && (p == 0 || p == 1)) {
        Value *cl = cmp->operands[0], *cr = cmp->operands[1];
        if ((cl == t && cr == f) || (cr == t && cl == f)) return Plan::of_value(p == 1 ? t : f);
      }
    }
    DenseP kc = cst(0), kl = cst(1), kr = cst(2);
    if (!kc || !kl || !kr) return Plan::failed();
    if (!(kc->elements && kl->elements && kr->elements)) return Plan::failed();
    if (kl->es != kr->es || !kl->ty->dtype) return Plan::failed();
    auto q = std::make_unique<FoldRequest>();
    q->kind = FoldRequest::SELECT;
    q->dtype = kl->dtype;
    q->out_dtype = kl->dtype;
    q->cond = kc;
    q->lhs = kl;
    q->rhs = kr;
    q->n = (uint64_t)std::max<int64_t>(1, kl->ty->count());
    q->out_ty = kl->ty;
    q->out_elements = true;
    return Plan::device(std::move(q));
  }

  Plan float_convert(int dop) {  // :727-742
    if (!element_type(ty())->is_float()) return Plan::failed();
    return unary(dop, element_type(ty())->dtype);
  }

  Plan cmpi() {  // :791-839
    const std::string* pp = op_->prop("predicate");
    if (!pp) return Plan::failed();
    bool ok;
    const int64_t pred = parse_int_prop(*pp, &ok);
    if (!ok) return Plan::failed();
    if (v(0) == v(1)) return Plan::of_attr(bool_attr(ty(), pred == 0 || pred == 3 || pred == 5 || pred == 7 || pred == 9));
    auto width1 = [](Value* x) { return element_type(x->ty)->dtype == DCF_I1; };
    if (zero(1)) {
      for (const char* ext : {"arith.extsi", "arith.extui"})
        if (Op* e = def(0, ext))
          if (width1(e->operands[0]) && pred == 1) return Plan::of_value(e->operands[0]);
      if (width1(v(0)) && pred == 1) return Plan::of_value(v(0));
    }
    if (one(1) && width1(v(0)) && pred == 0) return Plan::of_value(v(0));
    if (c_[0] && !c_[1]) {
      static const int swap[10] = {0, 1, 4, 5, 2, 3, 8, 9, 6, 7};
      const int64_t sp = (pred >= 0 && pred < 10) ? swap[pred] : pred;
      op_->set_prop("predicate", std::to_string(sp) + " : i64");
      Value *l = v(0), *r = v(1);
      m_.set_operand(op_, 0, r);
      m_.set_operand(op_, 1, l);
      return Plan::of_value(res());
    }
    DenseP lhs = cst(0);
    if (!lhs) return Plan::failed();
    return binary(DCF_CMPI, DCF_FLAG_PRED(pred), with_element(lhs->ty, "i1"));
  }

  Plan cmpf() {  // :457-467: scalar operands only
    DenseP l = cst(0), r = cst(1);
    if (l && l->elements) l = nullptr;
    if (r && r->elements) r = nullptr;
    if (l && !l->ty->is_float()) l = nullptr;
    if (r && !r->ty->is_float()) r = nullptr;
    const std::string* pp = op_->prop("predicate");
    if (!l || !r || !pp) return Plan::failed();
    bool ok;
    const int64_t pred = parse_int_prop(*pp, &ok);
    if (!ok) return Plan::failed();
    auto q = std::make_unique<FoldRequest>();
    q->kind = FoldRequest::BINARY;
    q->op = DCF_CMPF;
    q->dtype = l->dtype;
    q->out_dtype = DCF_I1;
    q->flags = DCF_FLAG_PRED(pred);
    q->lhs = l;
    q->rhs = r;
    q->n = 1;
    q->out_ty = type_of("i1");
    q->out_elements = false;
    return Plan::device(std::move(q));
  }
};

// Tf::fold, src/patterns/tosa/canonicalize.rs:189-232 (the folds reached
// by constant operands: transpose and reciprocal of splats).
Plan tosa_fold(Module&, Op* op, Engine& eng) {
  if (op->results.size() != 1) return Plan::failed();
  const TypeP rty = op->results[0]->ty;
  auto dense = [&](size_t i) -> DenseP {
    DenseP k = i < op->operands.size() ? constant_of(op->operands[i]) : nullptr;
    return (k && !k->poison && k->elements) ? k : nullptr;
  };
  if (op->name == "tosa.transpose") {  // :497-511
    DenseP k = dense(0);
    if (k && rty->static_shape() && k->ty->elem == rty->elem && eng.all_equal(*k))
      return Plan::of_attr(splat_value(rty, eng.bits0_of(*k)));
    std::vector<int64_t> perms = parse_array_prop(op->prop("perms"));
    if (perms.empty()) return Plan::failed();
    for (size_t i = 0; i < perms.size(); i++)
      if (perms[i] != (int64_t)i) return Plan::failed();
    if (op->operands[0]->ty->text == rty->text) return Plan::of_value(op->operands[0]);
    return Plan::failed();
  }
  if (op->name == "tosa.reciprocal") {  // :596-605
    if (!rty->static_shape()) return Plan::failed();
    DenseP k = dense(0);
    if (!k || !k->ty->is_float() || !eng.all_equal(*k)) return Plan::failed();
    auto q = std::make_unique<FoldRequest>();
    q->kind = FoldRequest::RECIPROCAL;
    q->dtype = k->dtype;
    q->out_dtype = k->dtype;
    q->lhs = splat_value(k->ty, eng.bits0_of(*k));
    q->n = 1;
    q->out_ty = rty;
    q->out_elements = true;
    return Plan::device(std::move(q));
  }
  return Plan::failed();
}

// The constant folds of tosa-layerwise-constant-fold (upstream MLIR
// TosaFolders: reciprocal and transpose of a constant that is a splat or
// has a single use).
Plan layerwise_pattern(Module&, Op* op, Engine& eng) {
  if (op->results.size() != 1 || op->operands.empty()) return Plan::failed();
  const TypeP rty = op->results[0]->ty;
  Value* in = op->operands[0];
  DenseP k = constant_of(in);
  if (!k || k->poison || !k->elements || !rty->static_shape()) return Plan::failed();
  if (op->name == "tosa.reciprocal") {
    if (!k->ty->is_float()) return Plan::failed();
    if (!(k->splat || in->uses.size() == 1 || eng.all_equal(*k))) return Plan::failed();
    auto q = std::make_unique<FoldRequest>();
    q->kind = FoldRequest::RECIPROCAL;
    q->dtype = k->dtype;
    q->out_dtype = k->dtype;
    q->lhs = k;
    q->n = k->n;
    q->out_ty = rty;
    q->out_elements = true;
    return Plan::device(std::move(q));
  }
  if (op->name == "tosa.transpose") {
    if (in->uses.size() != 1) return Plan::failed();
    if (!rty->dtype || k->ty->dynamic) return Plan::failed();
    std::vector<int64_t> perms = parse_array_prop(op->prop("perms"));
    if (perms.size() != k->ty->shape.size()) return Plan::failed();
    if (k->splat) return Plan::of_attr(splat_value(rty, eng.bits0_of(*k)));
    auto q = std::make_unique<FoldRequest>();
    q->kind = FoldRequest::PERMUTE;
    q->dtype = k->dtype;
    q->out_dtype = k->dtype;
    q->lhs = k;
    q->n = k->n;
    q->shape = k->ty->shape;
    q->perms = perms;
    q->out_ty = rty;
    q->out_elements = true;
    return Plan::device(std::move(q));
  }
  return Plan::failed();
}

bool commutative(const Op* op) {
  static const char* names[] = {"arith.addi", "arith.muli", "arith.andi", "arith.ori", "arith.xori",
                                "arith.addf", "arith.mulf", "arith.maximumf", "arith.minimumf",
                                "arith.maxnumf", "arith.minnumf", "arith.maxsi", "arith.maxui",
                                "arith.minsi", "arith.minui"};
  for (const char* n : names)
    if (op->name == n) return true;
  return false;
}

// materialize: ArithCanon (canonicalize.rs:1845-1859), TosaCanon
// (tosa/canonicalize.rs:1237-1241).  Returns the new constant op, unplaced.
Op* materialize(Module& m, const std::string& dialect, const DenseP& value, const TypeP& ty) {
  if (dialect == "arith" || dialect == "math") {
    if (value->poison) {
      Op* p = m.new_op("ub.poison");
      p->props.emplace_back("value", "#ub.poison");
      p->cst = value;
      p->cst_text = true;
      Value* r = m.new_value(ty);
      r->def = p;
      p->results.push_back(r);
      return p;
    }
    if (value->ty->text != ty->text) return nullptr;
    Op* c = m.new_op("arith.constant");
    c->props.emplace_back("value", "");
    c->cst = value;
    Value* r = m.new_value(ty);
    r->def = c;
    c->results.push_back(r);
    return c;
  }
  if (dialect == "tosa") {
    if (!value->elements || value->poison) return nullptr;
    Op* c = m.new_op("tosa.const");
    c->props.emplace_back("values", "");
    c->cst = value;
    Value* r = m.new_value(ty);
    r->def = c;
    c->results.push_back(r);
    return c;
  }
  return nullptr;
}

// Attribute equality of two constants (the key of the constant folder's
// deduplication, src/rewrite.rs:689-728): same type and form, same bytes.
// Bytes on the host (or both still as literal text) compare directly;
// otherwise the device hashes decide, and equal hashes are confirmed byte
// for byte.
bool value_eq(const DenseP& a, const DenseP& b, Engine& eng) {
  if (a == b) return true;
  if (a->poison || b->poison) return a->poison && b->poison && a->ty->text == b->ty->text;
  if (a->ty->text != b->ty->text || a->elements != b->elements || a->splat != b->splat || a->n != b->n) return false;
  if (!a->host.empty() && !b->host.empty()) return a->host == b->host;
  // Two literals still in their parsed text compare as text (mlir-opt
  // prints hex bodies in one case), without uploading either.
  if (!a->hex.empty() && !b->hex.empty() && !a->hashed && !b->hashed) return a->hex == b->hex;
  if (!a->hex.empty() && !b->hex.empty() && a->hex == b->hex) return true;
  if (a->dev && a->dev == b->dev) return true;
  if (eng.device() < 0) {  // host-only: only bytes the host can read compare
    auto readable = [](const DenseValue& v) { return !v.host.empty() || (!v.hex.empty() && v.hex.size() <= 8192); };
    if (!readable(*a) || !readable(*b)) return false;
    eng.to_host(*a);
    eng.to_host(*b);
    return a->host == b->host;
  }
  if (eng.hash_of(*a) != eng.hash_of(*b)) return false;
  eng.to_host(*a);
  eng.to_host(*b);
  return a->host == b->host;
}

}  // namespace

// ============================================================ the driver

struct Greedy::Impl {
  Module& m;
  Region* region;
  GreedyConfig cfg;
  Engine& eng;
  std::vector<Op*> list;
  std::unordered_map<Op*, size_t> at;
  struct Known {
    Region* region;
    std::string dialect;
    DenseP value;
    std::string ty;
    Op* op;
  };
  std::vector<Known> known;
  int iteration = 0;
  bool changed = false, finished = false, conv = false, started = false;
  Op* pend = nullptr;
  bool pend_pattern = false;
  std::unique_ptr<FoldRequest> pend_req;

  Impl(Module& mm, Region* r, GreedyConfig c, Engine& e) : m(mm), region(r), cfg(c), eng(e) {}

  // --- worklist (src/rewrite.rs:573-619)
  void push(Op* op) {
    if (at.count(op)) return;
    at[op] = list.size();
    list.push_back(op);
  }
  Op* pop() {
    while (!list.empty()) {
      Op* op = list.back();
      list.pop_back();
      if (op) {
        at.erase(op);
        return op;
      }
    }
    return nullptr;
  }
  void remove(Op* op) {
    auto it = at.find(op);
    if (it != at.end()) {
      list[it->second] = nullptr;
      at.erase(it);
    }
  }
  void reverse_list() {
    std::reverse(list.begin(), list.end());
    at.clear();
    for (size_t i = 0; i < list.size(); i++)
      if (list[i]) at[list[i]] = i;
  }

  // --- Tracker (src/rewrite.rs:621-677)
  void add(Op* op) {
    std::vector<Op*> chain;
    Op* cur = op;
    for (;;) {
      chain.push_back(cur);
      if (!cur->parent || !cur->parent->parent) return;
      Region* r = cur->parent->parent;
      if (r == region) {
        for (Op* o : chain) push(o);
        return;
      }
      cur = r->parent;
      if (!cur) return;
    }
  }
  void add_operands(Op* op) {
    for (Value* v : op->operands) {
      Op* d = v->def;
      if (!d) continue;
      Op* other = nullptr;
      bool many = false;
      for (auto it = v->uses.rbegin(); it != v->uses.rend(); ++it) {
        if (*it == op || *it == other) continue;
        if (!other) {
          other = *it;
          continue;
        }
        many = true;
        break;
      }
      if (!many) add(d);
    }
  }
  void erase_op(Op* op) {
    add_operands(op);
    remove(op);
    m.erase(op);
  }
  void replace_op(Op* op, const std::vector<Value*>& vals) {
    for (size_t i = 0; i < op->results.size() && i < vals.size(); i++) m.replace_all_uses(op->results[i], vals[i]);
    erase_op(op);
  }

  // --- constant hoisting and dedup (the driver's Folder, src/rewrite.rs:679-729)
  bool owns(Op* op) {
    for (auto& k : known)
      if (k.op == op) return true;
    return false;
  }
  static Op* prev_op(Op* op) {
    if (!op->parent || op->pos == op->parent->ops.begin()) return nullptr;
    auto it = op->pos;
    --it;
    return *it;
  }
  Region* insertion_region(Block* b) {
    for (;;) {
      Region* r = b->parent;
      Op* parent = r->parent;
      if (!parent || isolated(parent) || !parent->parent) return r;
      b = parent->parent;
    }
  }
  void move_to_front(Op* op, Block* b) {
    m.detach(op);
    if (b->ops.empty()) m.append(op, b);
    else m.insert_before(op, b->ops.front());
  }
  bool insert_constant(Op* op) {
    Block* block = op->parent;
    auto prev_owned = [&] {
      Op* p = prev_op(op);
      return p && owns(p);
    };
    if (owns(op)) {
      if (block->ops.front() != op && !prev_owned()) move_to_front(op, block);
      return true;
    }
    Region* r = insertion_region(block);
    const std::string dialect = op->dialect();
    const std::string ty = op->results[0]->ty->text;
    for (auto& k : known)
      if (k.region == r && k.dialect == dialect && k.ty == ty && value_eq(k.value, op->cst, eng)) {
        replace_op(op, k.op->results);
        return false;
      }
    Block* entry = r->blocks[0];
    if (block != entry) move_to_front(op, entry);
    else if (entry->ops.front() != op && !prev_owned()) move_to_front(op, entry);
    known.push_back({r, dialect, op->cst, ty, op});
    return true;
  }
  bool duplicate_constant(Op* op) {
    if (!cfg.cse_constants || !constant_like(op) || !op->cst) return false;
    return !insert_constant(op);
  }
  void collect(Region* r) {
    for (Block* b : r->blocks) {
      std::vector<Op*> ops(b->ops.begin(), b->ops.end());
      for (Op* op : ops) {
        if (op->erased) continue;
        if (cfg.top_down) {
          if (!duplicate_constant(op)) {
            add(op);
            collect_nested(op);
          }
        } else {
          collect_nested(op);
          if (!duplicate_constant(op)) add(op);
        }
      }
    }
  }
  void collect_nested(Op* op) {
    for (Region* r : op->regions) collect(r);
  }

  // --- folding (src/patterns/canonicalize.rs:328-378)
  Plan fold_commutative(Op* op) {
    std::vector<bool> cst;
    for (Value* v : op->operands) cst.push_back(v->def && constant_like(v->def));
    size_t first = 0;
    while (first < cst.size() && !cst[first]) first++;
    if (op->operands.size() < 2) return Plan::failed();
    std::vector<Value*> moved(op->operands.begin(), op->operands.begin() + (long)first);
    for (size_t i = first; i < cst.size(); i++)
      if (!cst[i]) moved.push_back(op->operands[i]);
    for (size_t i = first; i < cst.size(); i++)
      if (cst[i]) moved.push_back(op->operands[i]);
    if (moved == op->operands) return Plan::failed();
    for (size_t i = 0; i < moved.size(); i++) m.set_operand(op, i, moved[i]);
    return Plan::inplace();
  }
  Plan fold_traits(Op* op) { return commutative(op) ? fold_commutative(op) : Plan::failed(); }
  Plan fold_with(Op* op) {
    Plan own;
    const std::string d = op->dialect();
    if (d == "arith") own = ArithFolder(m, op, eng).fold();
    else if (d == "math") own = ArithFolder(m, op, eng).math();
    else if (d == "tosa") own = tosa_fold(m, op, eng);
    if (own.k == Plan::FAILED) return fold_traits(op);
    const bool to_self = own.k == Plan::VALUE && op->results.size() == 1 && own.value == op->results[0];
    if (to_self) {
      Plan t = fold_traits(op);
      return t.k == Plan::FAILED ? Plan::inplace() : std::move(t);
    }
    return own;
  }

  // replace_folded for several results: each part is a value or an
  // attribute that is materialised as a constant; nothing changes unless
  // every attribute materialises.
  bool replace_with_parts(Op* op, const std::vector<std::pair<Value*, DenseP>>& parts) {
    if (parts.size() != op->results.size()) return false;
    std::vector<Op*> made;
    std::vector<Value*> vals;
    for (size_t i = 0; i < parts.size(); i++) {
      if (parts[i].first) {
        vals.push_back(parts[i].first);
        continue;
      }
      Op* c = materialize(m, op->dialect(), parts[i].second, op->results[i]->ty);
      if (!c) return false;
      c->loc = op->loc;
      made.push_back(c);
      vals.push_back(c->results[0]);
    }
    for (Op* c : made) {
      m.insert_before(c, op);
      add(c);
    }
    replace_op(op, vals);
    return true;
  }

  // replace_folded (src/rewrite.rs:880-906) for one result.
  bool replace_with_attr(Op* op, const DenseP& a, const std::string& dialect) {
    Op* c = materialize(m, dialect, a, op->results[0]->ty);
    if (!c) return false;
    c->loc = op->loc;
    m.insert_before(c, op);
    add(c);
    replace_op(op, c->results);
    return true;
  }

  FoldRequest* try_patterns(Op* op) {
    if (!cfg.layerwise || op->erased) return nullptr;
    Plan p = layerwise_pattern(m, op, eng);
    if (p.k == Plan::ATTR) {
      if (replace_with_attr(op, p.attr, "tosa")) changed = true;
      return nullptr;
    }
    if (p.k != Plan::DEVICE) return nullptr;
    pend = op;
    pend_pattern = true;
    pend_req = std::move(p.req);
    return pend_req.get();
  }

  FoldRequest* step() {
    for (;;) {
      if (finished) return nullptr;
      if (!started) {
        iteration++;
        if (iteration > cfg.max_iterations) {
          finished = true;
          conv = false;
          return nullptr;
        }
        list.clear();
        at.clear();
        known.clear();
        collect(region);
        if (cfg.top_down) reverse_list();
        changed = false;
        started = true;
      }
      if (pend) {
        Op* op = pend;
        pend = nullptr;
        std::unique_ptr<FoldRequest> req = std::move(pend_req);
        if (pend_pattern) {
          if (req->folded && replace_with_attr(op, req->out, "tosa")) changed = true;
          continue;
        }
        if (req->folded && req->op2) {
          if (replace_with_parts(op, {{nullptr, req->out}, {nullptr, req->out2}})) changed = true;
          continue;
        }
        if (req->folded && replace_with_attr(op, req->out, op->dialect())) {
          changed = true;
          continue;
        }
        if (FoldRequest* r = try_patterns(op)) return r;
        continue;
      }
      Op* op = pop();
      if (!op) {
        if (!changed) {
          finished = true;
          conv = true;
          return nullptr;
        }
        started = false;
        continue;
      }
      if (op->erased) continue;
      bool dead = side_effect_free(op);
      for (Value* r : op->results) dead = dead && r->uses.empty();
      if (dead) {
        erase_op(op);
        changed = true;
        continue;
      }
      if (cfg.fold && !constant_like(op)) {
        Plan p = fold_with(op);
        if (p.k == Plan::INPLACE) {
          add(op);
          changed = true;
          continue;
        }
        if (p.k == Plan::VALUE) {
          replace_op(op, {p.value});
          changed = true;
          continue;
        }
        if (p.k == Plan::ATTR && replace_with_attr(op, p.attr, op->dialect())) {
          changed = true;
          continue;
        }
        if (p.k == Plan::MULTI && replace_with_parts(op, p.parts)) {
          changed = true;
          continue;
        }
        if (p.k == Plan::DEVICE) {
          pend = op;
          pend_pattern = false;
          pend_req = std::move(p.req);
          return pend_req.get();
        }
      }
      if (FoldRequest* r = try_patterns(op)) return r;
    }
  }
};

Greedy::Greedy(Module& m, Region* region, GreedyConfig cfg, Engine& eng)
    : impl_(std::make_unique<Impl>(m, region, cfg, eng)) {}
Greedy::~Greedy() = default;
FoldRequest* Greedy::step() { return impl_->step(); }
bool Greedy::done() const { return impl_->finished; }
bool Greedy::converged() const { return impl_->conv; }
Engine& Greedy::engine() { return impl_->eng; }

// ============================================================ pipelines

namespace {

std::string strip(std::string s) {
  while (!s.empty() && (s.front() == ' ' || s.front() == '\'' || s.front() == '"')) s.erase(s.begin());
  while (!s.empty() && (s.back() == ' ' || s.back() == '\'' || s.back() == '"')) s.pop_back();
  return s;
}

GreedyConfig config_for(const std::string& pass) {
  GreedyConfig c;
  if (pass.rfind("canonicalize", 0) == 0) {
    c.top_down = true;  // canonicalize's top-down option defaults to true
    return c;
  }
  if (pass == "tosa-layerwise-constant-fold") {
    c.layerwise = true;  // upstream greedy defaults: bottom-up
    return c;
  }
  throw std::runtime_error("unknown pass `" + pass + "`");
}

// Run the drivers of each GPU round by round: a round steps every driver
// until it needs element work and executes all pending requests as one
// batch.  The GPUs' drivers touch disjoint isolated functions, so each GPU
// runs its rounds in its own host thread, independent of the others.
void drive(std::vector<std::unique_ptr<Greedy>>& drivers, std::vector<Engine*>& engines, PassStats* stats) {
  (void)engines;
  std::vector<Engine*> order;
  std::unordered_map<Engine*, std::vector<Greedy*>> per;
  for (auto& d : drivers) {
    if (!per.count(&d->engine())) order.push_back(&d->engine());
    per[&d->engine()].push_back(d.get());
  }
  std::vector<PassStats> local(order.size());
  auto rounds = [&](size_t k) {
    Engine* e = order[k];
    for (;;) {
      std::vector<FoldRequest*> reqs;
      for (Greedy* d : per[e]) {
        if (d->done()) continue;
        if (FoldRequest* r = d->step()) reqs.push_back(r);
      }
      if (reqs.empty()) return;
      e->execute(reqs);
      for (FoldRequest* r : reqs) {
        if (r->folded) local[k].folds++;
        else local[k].refused++;
      }
    }
  };
  if (order.size() == 1) {
    rounds(0);
  } else {
    std::vector<std::thread> th;
    std::vector<std::string> errs(order.size());
    for (size_t k = 0; k < order.size(); k++)
      th.emplace_back([&, k] {
        try {
          rounds(k);
        } catch (const std::exception& ex) {
          errs[k] = ex.what();
        }
      });
    for (auto& t : th) t.join();
    for (auto& e : errs)
      if (!e.empty()) throw std::runtime_error(e);
  }
  if (stats)
    for (const PassStats& p : local) {
      stats->folds += p.folds;
      stats->refused += p.refused;
    }
}

uint64_t constant_bytes(Op* op) {
  uint64_t b = 0;
  for (Region* r : op->regions)
    for (Block* bl : r->blocks)
      for (Op* o : bl->ops) {
        if (o->cst) b += o->cst->n * o->cst->es;
        b += constant_bytes(o);
      }
  return b;
}

}  // namespace

void run_pipeline(Module& m, const std::string& pipeline_in, std::vector<Engine*>& engines, PassStats* stats) {
  if (engines.empty()) throw std::runtime_error("no GPU engine");
  std::string p = strip(pipeline_in);
  if (p.rfind("--", 0) == 0) p = p.substr(2);
  else if (p.rfind("-", 0) == 0) p = p.substr(1);
  if (p.rfind("canonicalize", 0) == 0) {
    std::vector<std::unique_ptr<Greedy>> drivers;
    for (Region* r : m.top->regions)
      drivers.push_back(std::make_unique<Greedy>(m, r, config_for("canonicalize"), *engines[0]));
    drive(drivers, engines, stats);
    return;
  }
  const std::string head = "builtin.module(func.func(";
  if (p.rfind(head, 0) != 0 || p.size() < head.size() + 2 || p.substr(p.size() - 2) != "))")
    throw std::runtime_error("unsupported pipeline: " + p);
  std::vector<std::string> passes;
  {
    std::string body = p.substr(head.size(), p.size() - head.size() - 2);
    size_t a = 0;
    int depth = 0;
    for (size_t i = 0; i <= body.size(); i++) {
      if (i < body.size() && (body[i] == '{' || body[i] == '(')) depth++;
      if (i < body.size() && (body[i] == '}' || body[i] == ')')) depth--;
      if (i == body.size() || (body[i] == ',' && depth == 0)) {
        std::string pass = strip(body.substr(a, i - a));
        const size_t brace = pass.find('{');
        if (brace != std::string::npos) pass = pass.substr(0, brace);
        if (!pass.empty()) passes.push_back(pass);
        a = i + 1;
      }
    }
  }
  // Functions (the reference's per-function task unit) over the GPUs,
  // balanced by constant bytes.
  std::vector<Op*> funcs;
  for (Region* r : m.top->regions)
    for (Block* b : r->blocks)
      for (Op* o : b->ops)
        if (o->name == "func.func") funcs.push_back(o);
  std::vector<std::pair<uint64_t, Op*>> by_size;
  for (Op* f : funcs) by_size.emplace_back(constant_bytes(f), f);
  std::stable_sort(by_size.begin(), by_size.end(), [](auto& a, auto& b) { return a.first > b.first; });
  std::unordered_map<Op*, Engine*> placed;
  std::vector<uint64_t> load(engines.size(), 0);
  for (auto& [bytes, f] : by_size) {
    size_t best = 0;
    for (size_t i = 1; i < engines.size(); i++)
      if (load[i] < load[best]) best = i;
    placed[f] = engines[best];
    load[best] += bytes + 1;
  }
  for (const std::string& pass : passes) {
    const GreedyConfig cfg = config_for(pass);
    std::vector<std::unique_ptr<Greedy>> drivers;
    for (Op* f : funcs)
      for (Region* r : f->regions) drivers.push_back(std::make_unique<Greedy>(m, r, cfg, *placed[f]));
    drive(drivers, engines, stats);
  }
}

void fetch_results(Module& m, std::vector<Engine*>& engines) {
  // Every device-resident constant comes back to the host: one packed
  // download per GPU, the GPUs in parallel.
  std::unordered_map<Engine*, std::vector<DenseValue*>> per;
  std::vector<Op*> stack{m.top};
  while (!stack.empty()) {
    Op* o = stack.back();
    stack.pop_back();
    if (o->cst && (o->cst->dev || !o->cst->parts.empty()) && o->cst->host.empty() && !o->cst_text) {
      Engine* e = engines[0];
      if (o->cst->dev && engines.size() > 1)
        for (Engine* x : engines)
          if (x->device() == o->cst->dev->device) e = x;
      per[e].push_back(o->cst.get());
    }
    for (Region* r : o->regions)
      for (Block* b : r->blocks)
        for (Op* in : b->ops) stack.push_back(in);
  }
  std::vector<std::thread> th;
  std::vector<std::string> errs(per.size());
  size_t i = 0;
  for (auto& kv : per) {
    th.emplace_back([&, i, e = kv.first, vs = &kv.second] {
      try {
        e->to_host_all(*vs);
      } catch (const std::exception& ex) {
        errs[i] = ex.what();
      }
    });
    i++;
  }
  for (auto& t : th) t.join();
  for (auto& e : errs)
    if (!e.empty()) throw std::runtime_error(e);
}

}  // namespace dco
