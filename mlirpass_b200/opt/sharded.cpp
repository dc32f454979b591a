// sharded.cpp — ShardedEngine: bare `canonicalize` over several GPUs by
// element ranges (see engine.h).
#include <algorithm>
#include <cstring>
#include <stdexcept>
#include <string>
#include <thread>

#include "engine.h"

namespace dco {

namespace {

uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

constexpr uint64_t kPhi = 0x9E3779B97F4A7C15ull;

// The device byte hash (dcf_hash_many_async) of `count` copies of one
// element of `es` bytes (es divides 8), computed on the host: the sum over
// 8-byte words w_i of mix(w_i ^ i * phi), the last word zero-padded, plus
// mix(bytes).
uint64_t splat_hash(uint64_t bits, size_t es, uint64_t count) {
  const uint64_t nbytes = count * es;
  auto byte_at = [&](uint64_t k) { return (uint64_t)(uint8_t)(bits >> (8 * (k % es))); };
  uint64_t word = 0;
  for (uint64_t k = 0; k < 8; k++) word |= byte_at(k) << (8 * k);
  const uint64_t nw = nbytes / 8;
  uint64_t h = 0;
  for (uint64_t i = 0; i < nw; i++) h += mix64(word ^ (i * kPhi));
  if (nbytes % 8) {
    uint64_t w = 0;
    for (uint64_t k = nw * 8; k < nbytes; k++) w |= byte_at(k) << (8 * (k - nw * 8));
    h += mix64(w ^ (nw * kPhi));
  }
  return h + mix64(nbytes);
}

// The hash of a sharded constant from its ranges' hashes, in order.
uint64_t combine(const std::vector<uint64_t>& hs) {
  uint64_t h = mix64(hs.size());
  for (size_t g = 0; g < hs.size(); g++) h += mix64(hs[g] + (g + 1) * kPhi);
  return h;
}

// A splat operand for one GPU's fold: its own copy of the one element, so
// that no device copy of it is shared between GPUs.
DenseP splat_copy(const DenseValue& v) {
  auto c = std::make_shared<DenseValue>();
  c->ty = v.ty;
  c->elements = v.elements;
  c->splat = true;
  c->dtype = v.dtype;
  c->es = v.es;
  c->n = v.n;
  c->poison = v.poison;
  if (!v.host.empty()) c->host = v.host;
  else c->hex = v.hex;
  return c;
}

}  // namespace

ShardedEngine::ShardedEngine(std::vector<Engine*> subs) : Engine(-1), subs_(std::move(subs)) {
  if (subs_.empty()) throw std::runtime_error("a sharded engine needs at least one GPU");
}

template <class F> void ShardedEngine::each(size_t parts, F&& f) {
  if (parts <= 1) {
    if (parts == 1) f(0);
    return;
  }
  std::vector<std::thread> th;
  std::vector<std::string> errs(parts);
  for (size_t g = 0; g < parts; g++)
    th.emplace_back([&, g] {
      try {
        f(g);
      } catch (const std::exception& e) {
        errs[g] = e.what();
      }
    });
  for (auto& t : th) t.join();
  for (auto& e : errs)
    if (!e.empty()) throw std::runtime_error(e);
}

bool ShardedEngine::shardable(const DenseValue& v) const {
  return subs_.size() > 1 && !v.splat && !v.poison && v.n >= kMinElements;
}

uint64_t ShardedEngine::chunk(uint64_t n) const {
  const uint64_t g = subs_.size();
  const uint64_t c = (n + g - 1) / g;
  return (c + kAlign - 1) / kAlign * kAlign;
}

Engine* ShardedEngine::owner(const DenseValue& v) const {
  if (v.dev)
    for (Engine* e : subs_)
      if (e->device() == v.dev->device) return e;
  return subs_[0];
}

// Cut a whole constant into its element ranges: views of its literal text
// when it has one, else copies of its host bytes.
void ShardedEngine::split(DenseValue& v) {
  if (!v.parts.empty() || !shardable(v)) return;
  if (v.hex.empty() && v.host.empty()) owner(v)->to_host(v);
  const uint64_t c = chunk(v.n);
  std::vector<DenseP> parts;
  for (uint64_t off = 0; off < v.n; off += c) {
    const uint64_t cnt = std::min<uint64_t>(c, v.n - off);
    auto p = std::make_shared<DenseValue>();
    p->ty = v.ty;
    p->elements = v.elements;
    p->dtype = v.dtype;
    p->es = v.es;
    p->n = cnt;
    if (!v.hex.empty()) p->hex = v.hex.substr(2 * off * v.es, 2 * cnt * v.es);
    parts.push_back(p);
  }
  if (v.hex.empty())
    each(parts.size(), [&](size_t g) {
      DenseValue& p = *parts[g];
      p.host.resize(p.bytes());
      memcpy(p.host.data(), v.host.data() + g * c * v.es, p.bytes());
    });
  v.parts = std::move(parts);
}

// The hash of range g of a sharded constant; a range that is one element
// hashes as that element repeated over the range.
uint64_t ShardedEngine::part_hash(const DenseValue& whole, size_t g) {
  DenseValue& p = *whole.parts[g];
  if (!p.splat) return subs_[g]->hash_of(p);
  const uint64_t c = chunk(whole.n);
  return splat_hash(p.bits0(), p.es, std::min<uint64_t>(c, whole.n - g * c));
}

void ShardedEngine::to_device(DenseValue& v) { owner(v)->to_device(v); }

void ShardedEngine::to_device_all(const std::vector<DenseValue*>& vs) { subs_[0]->to_device_all(vs); }

void ShardedEngine::to_host(DenseValue& v) { to_host_all({&v}); }

void ShardedEngine::to_host_all(const std::vector<DenseValue*>& vs) {
  std::vector<std::vector<DenseValue*>> whole(subs_.size());
  std::vector<DenseValue*> sharded;
  for (DenseValue* v : vs) {
    if (!v || !v->host.empty() || v->bytes() == 0) continue;
    if (!v->parts.empty() && v->hex.empty()) sharded.push_back(v);
    else whole[std::find(subs_.begin(), subs_.end(), owner(*v)) - subs_.begin()].push_back(v);
  }
  // Whole constants through their own GPU; the ranges of sharded ones each
  // straight from their GPU into place in one host buffer.
  for (DenseValue* v : sharded) v->host.resize(v->bytes());
  each(subs_.size(), [&](size_t g) {
    if (!whole[g].empty()) subs_[g]->to_host_all(whole[g]);
    for (DenseValue* v : sharded) {
      if (g >= v->parts.size()) continue;
      DenseValue& p = *v->parts[g];
      const uint64_t c = chunk(v->n), cnt = std::min<uint64_t>(c, v->n - g * c);
      uint8_t* dst = v->host.data() + g * c * v->es;
      if (p.splat) {
        const uint64_t b = p.bits0();
        for (uint64_t i = 0; i < cnt; i++) memcpy(dst + i * p.es, &b, p.es);
      } else if (!p.host.empty()) {
        memcpy(dst, p.host.data(), p.bytes());
      } else {
        subs_[g]->to_device(p);
        subs_[g]->download(dst, p.dev->ptr, p.bytes());
      }
    }
  });
}

std::string ShardedEngine::hex_of(DenseValue& v) {
  if (!v.parts.empty() && v.hex.empty()) to_host(v);
  return owner(v)->hex_of(v);
}

uint64_t ShardedEngine::bits0_of(DenseValue& v) {
  if (!v.parts.empty() && v.host.empty() && v.hex.empty()) {
    DenseValue& p = *v.parts[0];
    return p.splat ? p.bits0() : subs_[0]->bits0_of(p);
  }
  return owner(v)->bits0_of(v);
}

uint64_t ShardedEngine::hash_of(DenseValue& v) {
  if (v.hashed) return v.hash;
  if (!shardable(v)) return owner(v)->hash_of(v);
  split(v);
  std::vector<uint64_t> hs(v.parts.size());
  each(v.parts.size(), [&](size_t g) { hs[g] = part_hash(v, g); });
  v.hash = combine(hs);
  v.hashed = true;
  return v.hash;
}

bool ShardedEngine::all_equal(DenseValue& v) {
  if (v.all_equal >= 0) return v.all_equal;
  if (!shardable(v) || !v.host.empty()) return owner(v)->all_equal(v);
  split(v);
  std::vector<int> eq(v.parts.size(), 0);
  std::vector<uint64_t> first(v.parts.size(), 0);
  each(v.parts.size(), [&](size_t g) {
    DenseValue& p = *v.parts[g];
    eq[g] = subs_[g]->all_equal(p);
    first[g] = p.splat ? p.bits0() : subs_[g]->bits0_of(p);
  });
  bool all = true;
  for (size_t g = 0; g < eq.size(); g++) all = all && eq[g] && first[g] == first[0];
  return (v.all_equal = all ? 1 : 0);
}

void ShardedEngine::execute(const std::vector<FoldRequest*>& reqs) {
  if (reqs.empty()) return;
  const size_t G = subs_.size();
  // Element-wise folds of sharded sizes run range by range; everything else
  // runs whole on the first GPU, its sharded operands gathered first.
  std::vector<FoldRequest*> whole;
  std::vector<FoldRequest*> split_reqs;
  for (FoldRequest* q : reqs) {
    const bool elementwise = q->kind == FoldRequest::BINARY || q->kind == FoldRequest::CONVERT ||
                             q->kind == FoldRequest::RECIPROCAL || q->kind == FoldRequest::SELECT;
    if (elementwise && G > 1 && q->n >= kMinElements) {
      split_reqs.push_back(q);
      continue;
    }
    for (DenseP* o : {&q->lhs, &q->rhs, &q->cond})
      if (*o && !(*o)->parts.empty() && (*o)->hex.empty()) to_host(**o);
    whole.push_back(q);
  }
  // Per GPU, one sub-request per split request over that GPU's range;
  // at[k][g] is the index of request k's range g in sub[g] (-1: none).
  std::vector<std::vector<FoldRequest>> sub(G);
  for (auto& s : sub) s.reserve(split_reqs.size());
  std::vector<std::vector<long>> at(split_reqs.size(), std::vector<long>(G, -1));
  for (size_t k = 0; k < split_reqs.size(); k++) {
    FoldRequest* q = split_reqs[k];
    for (DenseP* o : {&q->lhs, &q->rhs, &q->cond})
      if (*o && !(*o)->splat) split(**o);
    const uint64_t c = chunk(q->n);
    for (size_t g = 0; g * c < q->n; g++) {
      FoldRequest s;
      s.kind = q->kind;
      s.op = q->op;
      s.dtype = q->dtype;
      s.out_dtype = q->out_dtype;
      s.flags = q->flags;
      s.n = std::min<uint64_t>(c, q->n - g * c);
      s.out_ty = q->out_ty;
      s.out_elements = q->out_elements;
      s.op2 = q->op2;
      s.out2_dtype = q->out2_dtype;
      s.flags2 = q->flags2;
      s.out2_ty = q->out2_ty;
      auto range = [&](const DenseP& o) -> DenseP {
        if (!o) return nullptr;
        if (o->splat) return splat_copy(*o);
        if (o->parts.size() <= g) throw std::runtime_error("a sharded operand has fewer ranges than its fold");
        return o->parts[g];
      };
      s.lhs = range(q->lhs);
      s.rhs = range(q->rhs);
      s.cond = range(q->cond);
      at[k][g] = (long)sub[g].size();
      sub[g].push_back(std::move(s));
    }
  }
  each(G, [&](size_t g) {
    if (g == 0 && !whole.empty()) subs_[0]->execute(whole);
    std::vector<FoldRequest*> mine;
    for (FoldRequest& s : sub[g]) mine.push_back(&s);
    subs_[g]->execute(mine);
  });
  // Merge: folded when every range folded, refused at the lowest refusing
  // element of any range.
  auto merge = [&](FoldRequest& q, size_t k, int dtype, const TypeP& ty, bool second) -> DenseP {
    std::vector<DenseP> parts;
    for (size_t g = 0; g < G; g++)
      if (at[k][g] >= 0) parts.push_back(second ? sub[g][at[k][g]].out2 : sub[g][at[k][g]].out);
    bool one = true;
    for (const DenseP& p : parts) one = one && p->splat && p->bits0() == parts[0]->bits0();
    if (one) return parts[0];  // every range the same single element: a splat
    auto d = std::make_shared<DenseValue>();
    d->ty = ty;
    d->elements = q.out_elements;
    d->dtype = dtype;
    d->es = dcf_dtype_size((dcf_dtype)dtype);
    d->n = q.n;
    d->all_equal = 0;
    d->parts = std::move(parts);
    std::vector<uint64_t> hs(d->parts.size());
    for (size_t g = 0; g < hs.size(); g++) hs[g] = part_hash(*d, g);
    d->hash = combine(hs);
    d->hashed = true;
    return d;
  };
  for (size_t k = 0; k < split_reqs.size(); k++) {
    FoldRequest& q = *split_reqs[k];
    q.first_fail = ~0ull;
    const uint64_t c = chunk(q.n);
    for (size_t g = 0; g < G; g++) {
      if (at[k][g] < 0) continue;
      const FoldRequest& s = sub[g][at[k][g]];
      if (!s.folded && s.first_fail != ~0ull) q.first_fail = std::min<uint64_t>(q.first_fail, g * c + s.first_fail);
    }
    q.folded = q.first_fail == ~0ull;
    if (!q.folded) continue;
    q.out = merge(q, k, q.out_dtype, q.out_ty, false);
    if (q.op2) q.out2 = merge(q, k, q.out2_dtype, q.out2_ty, true);
  }
}

}  // namespace dco
