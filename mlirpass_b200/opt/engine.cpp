// engine.cpp — see engine.h.
#include "engine.h"

#include <chrono>
#include <cstring>
#include <map>
#include <mutex>
#include <stdexcept>
#include <thread>
#include <tuple>

namespace dco {

namespace {

[[noreturn]] void cuda_fail(cudaError_t e, const char* what) {
  throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

void ck(cudaError_t e, const char* what) {
  if (e != cudaSuccess) cuda_fail(e, what);
}

int hexval(char c) {
  if (c >= '0' && c <= '9') return c - '0';
  if (c >= 'A' && c <= 'F') return c - 'A' + 10;
  if (c >= 'a' && c <= 'f') return c - 'a' + 10;
  return -1;
}

// Host decode of a short hex literal (a splat element, a small list): not
// worth a transfer and a launch.
void decode_small(std::string_view hex, std::vector<uint8_t>& out) {
  out.resize(hex.size() / 2);
  for (size_t i = 0; i < out.size(); i++) {
    const int h = hexval(hex[2 * i]), l = hexval(hex[2 * i + 1]);
    if (h < 0 || l < 0) throw std::runtime_error("invalid hex digit in a dense literal");
    out[i] = (uint8_t)(h * 16 + l);
  }
}

constexpr size_t kSmallHex = 8192;

}  // namespace

namespace {

struct Pool {
  std::mutex mu;
  std::multimap<size_t, void*> free[64];
  static size_t size_class(size_t n) {
    if (n <= 256) return 256;
    if (n <= (64u << 10)) {
      size_t c = 512;
      while (c < n) c <<= 1;
      return c;
    }
    return (n + (1u << 20) - 1) & ~(size_t)((1u << 20) - 1);
  }
};

Pool& pool() {
  static Pool* p = new Pool;  // outlives every DeviceBuf
  return *p;
}

// Run fn(0..n-1) on n threads and wait (n small: a copy split in parts).
template <class F>
void parallel(int n, F&& fn) {
  if (n <= 1) {
    fn(0);
    return;
  }
  std::vector<std::thread> th;
  for (int i = 1; i < n; i++) th.emplace_back([&, i] { fn(i); });
  fn(0);
  for (auto& t : th) t.join();
}

void copy_parallel(void* dst, const void* src, size_t bytes) {
  const int parts = bytes >= (8u << 20) ? 4 : 1;
  parallel(parts, [&](int i) {
    const size_t a = bytes * (size_t)i / parts, b = bytes * (size_t)(i + 1) / parts;
    memcpy((char*)dst + a, (const char*)src + a, b - a);
  });
}

}  // namespace

DeviceBuf::DeviceBuf(int dev, size_t n) : bytes(n), device(dev) {
  cap = Pool::size_class(n);
  Pool& p = pool();
  {
    std::lock_guard<std::mutex> g(p.mu);
    auto it = p.free[dev & 63].find(cap);
    if (it != p.free[dev & 63].end()) {
      ptr = it->second;
      p.free[dev & 63].erase(it);
      return;
    }
  }
  ck(cudaSetDevice(dev), "cudaSetDevice");
  cudaError_t e = cudaMalloc(&ptr, cap);
  if (e != cudaSuccess) {
    // Give cached blocks back to the driver and try once more.
    cudaGetLastError();
    std::lock_guard<std::mutex> g(p.mu);
    for (auto& kv : p.free[dev & 63]) cudaFree(kv.second);
    p.free[dev & 63].clear();
    ck(cudaMalloc(&ptr, cap), "cudaMalloc");
  }
}

DeviceBuf::~DeviceBuf() {
  if (!ptr) return;
  Pool& p = pool();
  std::lock_guard<std::mutex> g(p.mu);
  p.free[device & 63].emplace(cap, ptr);
}

Engine::Engine(int device) : dev_(device) {
  if (dev_ < 0) return;  // host-only: no element work
  ck(cudaSetDevice(dev_), "cudaSetDevice");
  ck(cudaStreamCreateWithFlags(&s_, cudaStreamNonBlocking), "cudaStreamCreate");
}

Engine::~Engine() {
  if (dev_ < 0) return;
  cudaSetDevice(dev_);
  if (s_) {
    cudaStreamSynchronize(s_);
    cudaStreamDestroy(s_);
  }
  for (int k = 0; k < kSlots; k++) {
    if (pinned_[k]) cudaFreeHost(pinned_[k]);
    if (slot_ev_[k]) cudaEventDestroy(slot_ev_[k]);
  }
}

void Engine::ensure_pinned() {
  if (pinned_[0]) return;
  for (int k = 0; k < kSlots; k++) {
    ck(cudaHostAlloc(&pinned_[k], kSlotBytes, cudaHostAllocPortable), "cudaHostAlloc");
    ck(cudaEventCreateWithFlags(&slot_ev_[k], cudaEventDisableTiming), "cudaEventCreate");
  }
}

void Engine::upload(void* dst, const void* src, size_t bytes) {
  set_device();
  stats.h2d_bytes += bytes;
  if (bytes < (1u << 20)) {
    ck(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, s_), "H2D");
    sync();
    return;
  }
  ensure_pinned();
  bool used[kSlots] = {false};
  size_t off = 0;
  int k = 0;
  while (off < bytes) {
    const size_t n = std::min(kSlotBytes, bytes - off);
    if (used[k]) ck(cudaEventSynchronize(slot_ev_[k]), "cudaEventSynchronize");
    copy_parallel(pinned_[k], (const char*)src + off, n);
    ck(cudaMemcpyAsync((char*)dst + off, pinned_[k], n, cudaMemcpyHostToDevice, s_), "H2D");
    ck(cudaEventRecord(slot_ev_[k], s_), "cudaEventRecord");
    used[k] = true;
    off += n;
    k = (k + 1) % kSlots;
  }
  sync();
}

void Engine::download(void* dst, const void* src, size_t bytes) {
  set_device();
  stats.d2h_bytes += bytes;
  if (bytes < (1u << 20)) {
    ck(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, s_), "D2H");
    sync();
    return;
  }
  ensure_pinned();
  size_t pend_off[kSlots] = {0}, pend_n[kSlots] = {0};
  size_t off = 0;
  int k = 0;
  auto drain = [&](int j) {
    if (!pend_n[j]) return;
    ck(cudaEventSynchronize(slot_ev_[j]), "cudaEventSynchronize");
    copy_parallel((char*)dst + pend_off[j], pinned_[j], pend_n[j]);
    pend_n[j] = 0;
  };
  while (off < bytes) {
    const size_t n = std::min(kSlotBytes, bytes - off);
    drain(k);
    ck(cudaMemcpyAsync(pinned_[k], (const char*)src + off, n, cudaMemcpyDeviceToHost, s_), "D2H");
    ck(cudaEventRecord(slot_ev_[k], s_), "cudaEventRecord");
    pend_off[k] = off;
    pend_n[k] = n;
    off += n;
    k = (k + 1) % kSlots;
  }
  for (int j = 0; j < kSlots; j++) drain((k + j) % kSlots);
}

void Engine::set_device() {
  if (dev_ < 0) throw std::runtime_error("element work needs a GPU (the host-only engine folds nothing)");
  ck(cudaSetDevice(dev_), "cudaSetDevice");
}

void Engine::check(int rc, const char* what) {
  if (rc < 0) throw std::runtime_error(std::string(what) + ": " + dcf_last_error());
}

void Engine::sync() { ck(cudaStreamSynchronize(s_), "cudaStreamSynchronize"); }

dcf_status* Engine::statuses(size_t n) {
  if (status_cap_ < n) {
    status_ = std::make_unique<DeviceBuf>(dev_, n * sizeof(dcf_status));
    status_cap_ = n;
  }
  return (dcf_status*)status_->ptr;
}

void Engine::to_device(DenseValue& v) {
  if (v.dev && v.dev->device == dev_) return;
  if (v.poison) throw std::runtime_error("a poison value has no bytes");
  set_device();
  const uint64_t bytes = v.bytes();
  auto buf = std::make_shared<DeviceBuf>(dev_, bytes);
  if (!v.host.empty()) {
    upload(buf->ptr, v.host.data(), bytes);
  } else if (!v.hex.empty()) {
    DeviceBuf text(dev_, v.hex.size());
    upload(text.ptr, v.hex.data(), v.hex.size());
    if (!aux_) aux_ = std::make_unique<DeviceBuf>(dev_, sizeof(dcf_status));
    dcf_status* st = (dcf_status*)aux_->ptr;
    check(dcf_status_reset_async(st, s_), "status reset");
    check(dcf_hex_decode_async((const char*)text.ptr, v.hex.size(), buf->ptr, st, s_), "hex decode");
    dcf_status h;
    ck(cudaMemcpyAsync(&h, st, sizeof h, cudaMemcpyDeviceToHost, s_), "D2H status");
    sync();
    if (h.first_fail != ~0ull) throw std::runtime_error("invalid hex digit in a dense literal");
  } else if (v.dev) {
    ck(cudaMemcpyPeerAsync(buf->ptr, dev_, v.dev->ptr, v.dev->device, bytes, s_), "peer copy");
    sync();
  } else if (bytes) {
    throw std::runtime_error("constant has no bytes");
  }
  v.dev = buf;
}

void Engine::to_host(DenseValue& v) {
  if (!v.host.empty() || v.bytes() == 0) return;
  if (v.poison) throw std::runtime_error("a poison value has no bytes");
  if (!v.hex.empty() && v.hex.size() <= kSmallHex) {
    decode_small(v.hex, v.host);
    return;
  }
  if (!v.dev) to_device(v);
  set_device();
  v.host.resize(v.bytes());
  download(v.host.data(), v.dev->ptr, v.bytes());
}

uint64_t Engine::bits0_of(DenseValue& v) {
  if (v.host.empty() && !v.hex.empty()) {
    std::vector<uint8_t> b;
    decode_small(v.hex.substr(0, 2 * v.es), b);
    uint64_t x = 0;
    memcpy(&x, b.data(), v.es);
    return x;
  }
  if (v.host.empty() && v.dev) {
    set_device();
    uint64_t x = 0;
    ck(cudaMemcpyAsync(&x, v.dev->ptr, v.es, cudaMemcpyDeviceToHost, s_), "D2H element");
    sync();
    return x;
  }
  return v.bits0();
}

std::string Engine::hex_of(DenseValue& v) {
  static const char digits[] = "0123456789ABCDEF";
  const uint64_t bytes = v.bytes();
  if (v.host.empty() && !v.hex.empty()) {
    std::string s(v.hex);
    for (char& c : s) c = (char)toupper((unsigned char)c);
    return s;
  }
  if (v.host.empty() && v.dev && bytes > kSmallHex) {
    set_device();
    DeviceBuf text(dev_, 2 * bytes);
    check(dcf_hex_encode_async(v.dev->ptr, bytes, (char*)text.ptr, s_), "hex encode");
    std::string s(2 * bytes, '0');
    download(&s[0], text.ptr, 2 * bytes);
    return s;
  }
  to_host(v);
  std::string s(2 * bytes, '0');
  for (uint64_t i = 0; i < bytes; i++) {
    s[2 * i] = digits[v.host[i] >> 4];
    s[2 * i + 1] = digits[v.host[i] & 15];
  }
  return s;
}

bool Engine::all_equal(DenseValue& v) {
  if (v.all_equal >= 0) return v.all_equal;
  if (v.splat || v.n <= 1) return (v.all_equal = 1);
  if (!v.host.empty()) {
    bool eq = true;
    for (uint64_t i = 1; i < v.n && eq; i++) eq = memcmp(v.host.data(), v.host.data() + i * v.es, v.es) == 0;
    return (v.all_equal = eq);
  }
  FoldRequest r;
  r.kind = FoldRequest::SPLAT_SCAN;
  r.lhs = std::shared_ptr<DenseValue>(&v, [](DenseValue*) {});
  execute({&r});
  return v.all_equal == 1;
}

void Engine::execute(const std::vector<FoldRequest*>& reqs) {
  if (reqs.empty()) return;
  const auto t0 = std::chrono::steady_clock::now();
  set_device();
  const size_t R = reqs.size();
  // Every streamed operand is made resident before the batch's statuses
  // are reset and its kernels are queued.
  for (FoldRequest* q : reqs) {
    if (q->lhs && !q->lhs->splat) to_device(*q->lhs);
    if (q->rhs && !q->rhs->splat) to_device(*q->rhs);
  }
  dcf_status* st = statuses(R);
  ck(cudaMemsetAsync(st, 0xFF, R * sizeof(dcf_status), s_), "status reset");

  // Splat operands: one element each, packed 16-byte aligned and uploaded once.
  std::vector<uint8_t> scal;
  std::vector<std::pair<size_t, size_t>> spos(R, {SIZE_MAX, SIZE_MAX});
  auto place = [&](DenseValue& v) {
    const size_t at = scal.size();
    scal.resize(at + 16, 0);
    const uint64_t b = bits0_of(v);
    memcpy(&scal[at], &b, v.es);
    return at;
  };
  for (size_t i = 0; i < R; i++) {
    FoldRequest& q = *reqs[i];
    if (q.lhs && q.lhs->splat) spos[i].first = place(*q.lhs);
    if (q.rhs && q.rhs->splat) spos[i].second = place(*q.rhs);
  }
  std::unique_ptr<DeviceBuf> sdev;
  if (!scal.empty()) {
    sdev = std::make_unique<DeviceBuf>(dev_, scal.size());
    ck(cudaMemcpyAsync(sdev->ptr, scal.data(), scal.size(), cudaMemcpyHostToDevice, s_), "H2D splats");
  }
  auto operand = [&](DenseValue& v, size_t pos) -> const void* {
    if (pos != SIZE_MAX) return (const char*)sdev->ptr + pos;
    to_device(v);
    return v.dev->ptr;
  };

  std::vector<std::shared_ptr<DeviceBuf>> outs(R);
  std::vector<const void*> ls(R, nullptr), rs(R, nullptr);
  for (size_t i = 0; i < R; i++) {
    FoldRequest& q = *reqs[i];
    ls[i] = q.lhs ? operand(*q.lhs, spos[i].first) : nullptr;
    rs[i] = q.rhs ? operand(*q.rhs, spos[i].second) : nullptr;
    if (q.kind != FoldRequest::SPLAT_SCAN)
      outs[i] = std::make_shared<DeviceBuf>(dev_, q.n * dcf_dtype_size((dcf_dtype)q.out_dtype));
  }
  // Many small folds of one kind (one per isolated function, say) go out as
  // one launch per group through the batched kernel.
  std::vector<bool> batched(R, false);
  std::vector<dcf_status> bst(R);
  {
    std::map<std::tuple<int, int, int, int, uint32_t>, std::vector<size_t>> groups;
    for (size_t i = 0; i < R; i++) {
      const FoldRequest& q = *reqs[i];
      if ((q.kind == FoldRequest::BINARY || q.kind == FoldRequest::CONVERT || q.kind == FoldRequest::RECIPROCAL) &&
          q.n <= (4u << 20))
        groups[{(int)q.kind, q.op, q.dtype, q.out_dtype, q.flags}].push_back(i);
    }
    for (auto& [key, idx] : groups) {
      if (idx.size() < 8) continue;
      for (size_t a = 0; a < idx.size(); a += 1024) {
        const size_t b = std::min(idx.size(), a + 1024);
        std::vector<dcf_job> jobs(b - a);
        for (size_t t = a; t < b; t++) {
          const FoldRequest& q = *reqs[idx[t]];
          dcf_job& j = jobs[t - a];
          memset(&j, 0, sizeof j);
          j.op = q.kind == FoldRequest::RECIPROCAL ? DCF_RECIPROCAL : (uint32_t)q.op;
          j.dtype = (uint32_t)q.dtype;
          j.out_dtype = (uint32_t)q.out_dtype;
          j.flags = q.flags;
          j.lhs = ls[idx[t]];
          j.rhs = q.kind == FoldRequest::BINARY ? rs[idx[t]] : nullptr;
          j.out = outs[idx[t]]->ptr;
          j.n = q.n;
          j.lhs_splat = q.lhs->splat;
          j.rhs_splat = q.kind == FoldRequest::BINARY ? q.rhs->splat : 0;
        }
        check(dcf_batch_noalloc(jobs.data(), jobs.size(), s_), "batched fold");
        for (size_t t = a; t < b; t++) {
          const dcf_result& r = jobs[t - a].result;
          bst[idx[t]].first_fail = r.first_fail_index;
          bst[idx[t]].splat_word = r.is_splat ? 1u : 0u;
          bst[idx[t]].error = 0xFFFFFFFFu;
          batched[idx[t]] = true;
        }
      }
    }
  }
  for (size_t i = 0; i < R; i++) {
    if (batched[i]) continue;
    FoldRequest& q = *reqs[i];
    const void* l = ls[i];
    const void* r = rs[i];
    set_device();
    const size_t oes = dcf_dtype_size((dcf_dtype)q.out_dtype);
    switch (q.kind) {
      case FoldRequest::BINARY:
        check(dcf_binary_async((dcf_op)q.op, (dcf_dtype)q.dtype, l, q.lhs->splat, r, q.rhs->splat, q.n, q.flags,
                               outs[i]->ptr, st + i, s_),
              "binary fold");
        break;
      case FoldRequest::CONVERT:
        check(dcf_convert_async((dcf_op)q.op, (dcf_dtype)q.dtype, (dcf_dtype)q.out_dtype, l, q.lhs->splat, q.n,
                                q.flags, outs[i]->ptr, st + i, s_),
              "convert fold");
        break;
      case FoldRequest::RECIPROCAL:
        check(dcf_reciprocal_async((dcf_dtype)q.dtype, l, q.lhs->splat, q.n, q.flags, outs[i]->ptr, st + i, s_),
              "reciprocal fold");
        break;
      case FoldRequest::PERMUTE:
        check(dcf_permute_async(oes, (int)q.shape.size(), q.shape.data(), q.perms.data(), l, outs[i]->ptr, s_),
              "transpose fold");
        break;
      case FoldRequest::SPLAT_SCAN:
        check(dcf_splat_check_async(l, q.lhs->es, q.lhs->n, st + i, s_), "splat scan");
        break;
    }
  }
  std::vector<dcf_status> hst(R);
  ck(cudaMemcpyAsync(hst.data(), st, R * sizeof(dcf_status), cudaMemcpyDeviceToHost, s_), "D2H status");
  sync();
  for (size_t i = 0; i < R; i++)
    if (batched[i]) hst[i] = bst[i];
  // First element of every all-equal result, fetched together.
  std::vector<uint64_t> first(R, 0);
  bool any = false;
  for (size_t i = 0; i < R; i++) {
    FoldRequest& q = *reqs[i];
    if (hst[i].error != 0xFFFFFFFFu) throw std::runtime_error("a fold kernel gave up waiting for its copies");
    if (q.kind == FoldRequest::SPLAT_SCAN || q.kind == FoldRequest::PERMUTE) continue;
    if (hst[i].first_fail == ~0ull && hst[i].splat_word != 0) {
      const size_t oes = dcf_dtype_size((dcf_dtype)q.out_dtype);
      ck(cudaMemcpyAsync(&first[i], outs[i]->ptr, oes, cudaMemcpyDeviceToHost, s_), "D2H element");
      any = true;
    }
  }
  if (any) sync();
  for (size_t i = 0; i < R; i++) {
    FoldRequest& q = *reqs[i];
    stats.requests++;
    if (q.kind == FoldRequest::SPLAT_SCAN) {
      q.lhs->all_equal = (q.lhs->n <= 1 || hst[i].splat_word != 0) ? 1 : 0;
      continue;
    }
    q.first_fail = q.kind == FoldRequest::PERMUTE ? ~0ull : hst[i].first_fail;
    q.folded = q.first_fail == ~0ull;
    if (!q.folded) continue;
    auto d = std::make_shared<DenseValue>();
    d->ty = q.out_ty;
    d->elements = q.out_elements;
    d->dtype = q.out_dtype;
    d->es = dcf_dtype_size((dcf_dtype)q.out_dtype);
    if (q.kind != FoldRequest::PERMUTE && hst[i].splat_word != 0) {
      d->splat = true;
      d->n = 1;
      d->host.resize(d->es);
      memcpy(d->host.data(), &first[i], d->es);
    } else {
      d->n = q.n;
      d->dev = outs[i];
      // The kernel's splat test already said the values differ.
      if (q.kind != FoldRequest::PERMUTE) d->all_equal = 0;
    }
    if (q.kind == FoldRequest::PERMUTE && q.lhs->all_equal == 1) d->all_equal = 1;
    q.out = d;
  }
  stats.batches++;
  stats.device_ms += std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
}

}  // namespace dco
