// engine.cpp — see engine.h.
#include "engine.h"

#include <atomic>
#include <chrono>
#include <condition_variable>
#include <cstdlib>
#include <cstring>
#include <deque>
#include <functional>
#include <map>
#include <mutex>
#include <stdexcept>
#include <thread>
#include <tuple>
#include <unordered_map>
#include <algorithm>

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
void decode_small(std::string_view hex, Bytes& out) {
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

// A process-wide pool of host threads for the staging copies: one slot's
// memcpy is split over several threads, and several engines (one per GPU)
// submit at once.  Threads are started once, not per slot.
class CopyPool {
 public:
  static CopyPool& get() {
    static CopyPool* p = new CopyPool;  // never destroyed: workers may outlive static destructors
    return *p;
  }
  int width() const { return (int)workers_.size() + 1; }
  // Run fn(0..n-1); the caller takes part, and returns when all are done.
  // fn is called only for parts taken before that, so it may live on the
  // caller's stack; the batch record itself is shared with the workers.
  template <class F>
  void run(int n, F&& fn) {
    if (n <= 1 || workers_.empty()) {
      for (int i = 0; i < n; i++) fn(i);
      return;
    }
    auto b = std::make_shared<Batch>();
    b->fn = [&fn](int i) { fn(i); };
    b->n = n;
    {
      std::lock_guard<std::mutex> g(mu_);
      queue_.push_back(b);
    }
    cv_.notify_all();
    work_on(*b);
    std::unique_lock<std::mutex> g(mu_);
    done_cv_.wait(g, [&] { return b->finished == b->n; });
  }

 private:
  struct Batch {
    std::function<void(int)> fn;
    int n = 0;
    int next = 0;      // guarded by mu_
    int finished = 0;  // guarded by mu_
  };
  std::mutex mu_;
  std::condition_variable cv_, done_cv_;
  std::deque<std::shared_ptr<Batch>> queue_;
  std::vector<std::thread> workers_;

  CopyPool() {
    const unsigned hw = std::max(1u, std::thread::hardware_concurrency());
    const unsigned n = std::min(63u, hw > 1 ? hw - 1 : 0u);
    for (unsigned i = 0; i < n; i++) workers_.emplace_back([this] { loop(); });
    for (auto& t : workers_) t.detach();
  }
  // Take parts of b until none are left.
  void work_on(Batch& b) {
    for (;;) {
      int i;
      {
        std::lock_guard<std::mutex> g(mu_);
        if (b.next >= b.n) return;
        i = b.next++;
      }
      b.fn(i);
      std::lock_guard<std::mutex> g(mu_);
      if (++b.finished == b.n) done_cv_.notify_all();
    }
  }
  void loop() {
    for (;;) {
      std::shared_ptr<Batch> b;
      {
        std::unique_lock<std::mutex> g(mu_);
        cv_.wait(g, [&] {
          while (!queue_.empty() && queue_.front()->next >= queue_.front()->n) queue_.pop_front();
          return !queue_.empty();
        });
        b = queue_.front();
      }
      work_on(*b);
    }
  }
};

// Page-locked host memory for constants' host bytes (installed as the
// HostAllocator of ir.h).  Sizes are rounded to a power of two (64 KiB ...
// 32 MiB, carved from 256 MiB slabs) or to 2 MiB (larger, own allocation);
// freed blocks are kept per size and handed out again, so after the first
// run a pipeline's results land in memory that is already pinned and
// touched.  Allocation failures fall back to ordinary memory.
class PinnedPool {
 public:
  static PinnedPool& get() {
    static PinnedPool* p = new PinnedPool;  // never destroyed: buffers may be freed during exit
    return *p;
  }
  void* alloc(size_t n) {
    const size_t c = cls(n);
    std::lock_guard<std::mutex> g(mu_);
    auto& fl = free_[c];
    if (!fl.empty()) {
      void* p = fl.back();
      fl.pop_back();
      return p;
    }
    void* p = nullptr;
    if (c <= kMaxSlabbed) {
      if (left_ < c) {
        if (cudaHostAlloc((void**)&cur_, kSlab, cudaHostAllocPortable) != cudaSuccess) {
          cudaGetLastError();
          cur_ = nullptr;
          left_ = 0;
          return ::operator new(n);
        }
        ranges_.emplace_back((uintptr_t)cur_, (uintptr_t)cur_ + kSlab);
        left_ = kSlab;
      }
      p = cur_;
      cur_ += c;
      left_ -= c;
      return p;
    }
    if (cudaHostAlloc(&p, c, cudaHostAllocPortable) != cudaSuccess) {
      cudaGetLastError();
      return ::operator new(n);
    }
    ranges_.emplace_back((uintptr_t)p, (uintptr_t)p + c);
    return p;
  }
  void release(void* p, size_t n) {
    std::lock_guard<std::mutex> g(mu_);
    if (owned_locked(p)) free_[cls(n)].push_back(p);
    else ::operator delete(p);
  }
  bool owned(const void* p) {
    std::lock_guard<std::mutex> g(mu_);
    return owned_locked(p);
  }

 private:
  static constexpr size_t kSlab = 256u << 20;
  static constexpr size_t kMaxSlabbed = 32u << 20;
  std::mutex mu_;
  std::unordered_map<size_t, std::vector<void*>> free_;
  std::vector<std::pair<uintptr_t, uintptr_t>> ranges_;
  char* cur_ = nullptr;
  size_t left_ = 0;
  static size_t cls(size_t n) {
    if (n > kMaxSlabbed) return (n + (2u << 20) - 1) & ~(size_t)((2u << 20) - 1);
    size_t c = kHostPoolMin;
    while (c < n) c <<= 1;
    return c;
  }
  bool owned_locked(const void* p) const {
    for (auto& r : ranges_)
      if ((uintptr_t)p >= r.first && (uintptr_t)p < r.second) return true;
    return false;
  }
};

void* pinned_alloc(size_t n) { return PinnedPool::get().alloc(n); }
void pinned_free(void* p, size_t n) { PinnedPool::get().release(p, n); }

// Run fn(0..n-1) over the copy pool and wait.
template <class F>
void parallel(int n, F&& fn) {
  CopyPool::get().run(n, std::forward<F>(fn));
}

// Parts for a copy of `bytes`: about 512 KiB each, at most the pool's
// width (a 16 MiB staging slot goes to every host thread).
int parts_for(size_t bytes) {
  const size_t p = bytes >> 19;
  return (int)std::max<size_t>(1, std::min<size_t>(p, (size_t)CopyPool::get().width()));
}

void copy_parallel(void* dst, const void* src, size_t bytes) {
  const int parts = parts_for(bytes);
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

DeviceBuf::DeviceBuf(std::shared_ptr<DeviceBuf> parent, size_t offset, size_t n)
    : ptr((char*)parent->ptr + offset), bytes(n), device(parent->device), parent_(std::move(parent)) {}

DeviceBuf::~DeviceBuf() {
  if (!ptr || parent_) return;
  Pool& p = pool();
  std::lock_guard<std::mutex> g(p.mu);
  p.free[device & 63].emplace(cap, ptr);
}

Engine::Engine(int device) : dev_(device) {
  if (dev_ < 0) return;  // host-only: no element work
  ck(cudaSetDevice(dev_), "cudaSetDevice");
  static std::once_flag once;
  std::call_once(once, [] {
    host_allocator().alloc = pinned_alloc;
    host_allocator().free = pinned_free;
  });
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
    if (pinned_[k]) PinnedPool::get().release(pinned_[k], kSlotBytes);
    if (slot_ev_[k]) cudaEventDestroy(slot_ev_[k]);
  }
}

void Engine::ensure_pinned() {
  if (pinned_[0]) return;
  for (int k = 0; k < kSlots; k++) {
    // from the process-wide page-locked pool: a later engine (the next
    // run) gets the same slots back instead of pinning new memory
    pinned_[k] = PinnedPool::get().alloc(kSlotBytes);
    ck(cudaEventCreateWithFlags(&slot_ev_[k], cudaEventDisableTiming), "cudaEventCreate");
  }
}

void Engine::download(void* dst, const void* src, size_t bytes) {
  set_device();
  stats.d2h_bytes += bytes;
  struct Timer {
    double& acc;
    std::chrono::steady_clock::time_point t = std::chrono::steady_clock::now();
    ~Timer() { acc += std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t).count(); }
  } timer{stats.download_ms};
  if (bytes < (1u << 20) || PinnedPool::get().owned(dst)) {  // small, or page-locked: straight there
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

namespace {

// Copy bytes [a, b) of a packed image between its pieces and `buf`, which
// holds image byte `a` at offset 0.  Bytes between pieces are padding.  A
// hex piece is decoded on the way in; a bad digit sets *bad.
void copy_span(const std::vector<ImagePiece>& pcs, size_t a, size_t b, char* buf, bool to_buf,
               std::atomic<bool>* bad) {
  auto it = std::upper_bound(pcs.begin(), pcs.end(), a,
                             [](size_t x, const ImagePiece& p) { return x < p.off + p.len; });
  for (; it != pcs.end() && it->off < b; ++it) {
    const size_t lo = std::max(a, it->off), hi = std::min(b, it->off + it->len);
    if (lo >= hi) continue;
    if (it->hex) {
      const char* t = (const char*)it->host + 2 * (lo - it->off);
      if (!decode_hex_host(t, hi - lo, (uint8_t*)buf + (lo - a)) && bad) bad->store(true);
      continue;
    }
    char* h = (char*)it->host + (lo - it->off);
    if (to_buf) memcpy(buf + (lo - a), h, hi - lo);
    else memcpy(h, buf + (lo - a), hi - lo);
  }
}

// Split [a, a+n) of the image over host threads (one for small spans).
void copy_slot(const std::vector<ImagePiece>& pcs, size_t a, size_t n, char* buf, bool to_buf,
               std::atomic<bool>* bad = nullptr) {
  const int parts = parts_for(n);
  parallel(parts, [&](int i) {
    const size_t x = n * (size_t)i / parts, y = n * (size_t)(i + 1) / parts;
    copy_span(pcs, a + x, a + y, buf + x, to_buf, bad);
  });
}

// Literal text is decoded on the host while it is staged (the default), or
// copied as text and decoded on the GPU (DCF_OPT_DECODE=device).
bool decode_on_host() {
  static const bool v = [] {
    const char* e = getenv("DCF_OPT_DECODE");
    return !(e && std::string(e) == "device");
  }();
  return v;
}

size_t align16(size_t n) { return (n + 15) & ~(size_t)15; }

}  // namespace

// Host pieces -> pinned slots -> one contiguous device arena (hex pieces
// decoded on the way).
void Engine::upload_image(const std::vector<ImagePiece>& pcs, size_t total, char* arena) {
  ensure_pinned();
  stats.h2d_bytes += total;
  bool used[kSlots] = {false};
  std::atomic<bool> bad{false};
  int k = 0;
  for (size_t off = 0; off < total; off += kSlotBytes) {
    const size_t n = std::min(kSlotBytes, total - off);
    if (used[k]) ck(cudaEventSynchronize(slot_ev_[k]), "cudaEventSynchronize");
    copy_slot(pcs, off, n, (char*)pinned_[k], true, &bad);
    if (bad.load()) throw std::runtime_error("invalid hex digit in a dense literal");
    ck(cudaMemcpyAsync(arena + off, pinned_[k], n, cudaMemcpyHostToDevice, s_), "H2D");
    ck(cudaEventRecord(slot_ev_[k], s_), "cudaEventRecord");
    used[k] = true;
    k = (k + 1) % kSlots;
  }
}

// Device pieces -> pinned slots -> host pieces.  A slot is filled by one
// copy per piece that overlaps it, then emptied by host threads while the
// copy engine fills the next slots.
void Engine::download_image(const std::vector<ImagePiece>& pcs, size_t total) {
  ensure_pinned();
  stats.d2h_bytes += total;
  size_t pend_off[kSlots] = {0}, pend_n[kSlots] = {0};
  auto drain = [&](int j) {
    if (!pend_n[j]) return;
    ck(cudaEventSynchronize(slot_ev_[j]), "cudaEventSynchronize");
    copy_slot(pcs, pend_off[j], pend_n[j], (char*)pinned_[j], false);
    pend_n[j] = 0;
  };
  size_t first = 0;  // first piece that may overlap the next slot
  int k = 0;
  for (size_t off = 0; off < total; off += kSlotBytes) {
    const size_t n = std::min(kSlotBytes, total - off);
    drain(k);
    while (first < pcs.size() && pcs[first].off + pcs[first].len <= off) first++;
    for (size_t i = first; i < pcs.size() && pcs[i].off < off + n; i++) {
      const size_t lo = std::max(off, pcs[i].off), hi = std::min(off + n, pcs[i].off + pcs[i].len);
      if (lo < hi)
        ck(cudaMemcpyAsync((char*)pinned_[k] + (lo - off), (const char*)pcs[i].dev + (lo - pcs[i].off), hi - lo,
                           cudaMemcpyDeviceToHost, s_),
           "D2H");
    }
    ck(cudaEventRecord(slot_ev_[k], s_), "cudaEventRecord");
    pend_off[k] = off;
    pend_n[k] = n;
    k = (k + 1) % kSlots;
  }
  for (int j = 0; j < kSlots; j++) drain((k + j) % kSlots);
}

void Engine::to_device_all(const std::vector<DenseValue*>& in) {
  const auto t0 = std::chrono::steady_clock::now();
  struct Timer {
    double& acc;
    std::chrono::steady_clock::time_point t;
    ~Timer() { acc += std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t).count(); }
  } timer{stats.upload_ms, t0};
  std::vector<DenseValue*> vs;
  std::unordered_map<DenseValue*, size_t> index;
  for (DenseValue* v : in) {
    if (!v || (v->dev && v->dev->device == dev_) || v->bytes() == 0) continue;
    if (index.emplace(v, vs.size()).second) vs.push_back(v);
  }
  if (vs.empty()) return;
  set_device();
  // Text and host bytes from pageable memory share one packed image that
  // goes through the pinned slots; text inside page-locked input memory is
  // copied straight from there into a second arena.  Peer-resident values
  // are copied GPU to GPU.
  std::vector<ImagePiece> staged, direct;
  struct Loc {
    DenseValue* v;
    bool is_direct;
    size_t off;
  };
  std::vector<Loc> text, raw, viewed;
  size_t total = 0, total_direct = 0;
  const bool host_decode = decode_on_host();
  for (DenseValue* v : vs) {
    if (v->poison) throw std::runtime_error("a poison value has no bytes");
    if (!v->host.empty() && PinnedPool::get().owned(v->host.data())) {
      direct.push_back({(void*)v->host.data(), nullptr, v->bytes(), total_direct});
      raw.push_back({v, true, total_direct});
      total_direct = align16(total_direct + v->bytes());
    } else if (!v->host.empty()) {
      staged.push_back({(void*)v->host.data(), nullptr, v->bytes(), total});
      (host_decode ? viewed : raw).push_back({v, false, total});
      total = align16(total + v->bytes());
    } else if (!v->hex.empty() && host_decode &&
               (!in_pinned(v->hex.data(), v->hex.size()) ||
                (pinned_small_on_host_ && v->hex.size() < kSmallPinnedHex))) {
      // Pageable text (which the host must copy anyway) is decoded into the
      // staging slots: raw bytes cross PCIe, and the constant is a view of
      // the arena (no device-side decode or copy).
      staged.push_back({(void*)v->hex.data(), nullptr, v->bytes(), total, true});
      viewed.push_back({v, false, total});
      total = align16(total + v->bytes());
    } else if (!v->hex.empty() && in_pinned(v->hex.data(), v->hex.size())) {
      text.push_back({v, true, 0});  // placed below, with its neighbours in the input
    } else if (!v->hex.empty()) {
      staged.push_back({(void*)v->hex.data(), nullptr, v->hex.size(), total});
      text.push_back({v, false, total});
      total = align16(total + v->hex.size());
    } else if (!v->dev) {
      throw std::runtime_error("constant has no bytes");
    }
  }
  std::vector<std::shared_ptr<DeviceBuf>> bufs(vs.size());
  {
    std::vector<bool> is_view(vs.size(), false);
    for (const Loc& l : viewed) is_view[index.at(l.v)] = true;
    for (size_t i = 0; i < vs.size(); i++)
      if (!is_view[i]) bufs[i] = std::make_shared<DeviceBuf>(dev_, vs[i]->bytes());
  }
  auto buf_of = [&](DenseValue* v) -> std::shared_ptr<DeviceBuf>& { return bufs[index.at(v)]; };
  // Literals inside the page-locked input are copied as runs: literals whose
  // gaps in the input are short go in one copy with the text between them,
  // 16 bytes of context on each side (the decoder reads whole aligned
  // 16-byte blocks around a literal), placed so that device and host
  // addresses agree modulo 16.
  struct Run {
    const char* a;
    const char* b;
    size_t off;
  };
  std::vector<Run> runs;
  {
    constexpr size_t kGap = 64u << 10, kCtx = 16;
    std::vector<Loc*> order;
    for (Loc& l : text)
      if (l.is_direct) order.push_back(&l);
    std::sort(order.begin(), order.end(), [](const Loc* x, const Loc* y) { return x->v->hex.data() < y->v->hex.data(); });
    total_direct = std::max<size_t>(total_direct, kCtx);
    for (Loc* l : order) {
      const char* a = std::max(l->v->hex.data() - kCtx, pinned_src_);
      const char* b = std::min(l->v->hex.data() + l->v->hex.size() + kCtx, pinned_src_ + pinned_len_);
      if (!runs.empty() && a <= runs.back().b + kGap) {
        runs.back().b = std::max(runs.back().b, b);
      } else {
        const size_t off = align16(total_direct) + ((uintptr_t)a & 15);
        runs.push_back({a, b, off});
      }
      total_direct = runs.back().off + (size_t)(runs.back().b - runs.back().a) + kCtx;
      l->off = runs.back().off + (size_t)(l->v->hex.data() - runs.back().a);
    }
  }
  std::shared_ptr<DeviceBuf> arena;
  std::unique_ptr<DeviceBuf> arena_direct;
  if (!direct.empty() || !runs.empty()) {
    arena_direct = std::make_unique<DeviceBuf>(dev_, total_direct + 32);
    for (const ImagePiece& p : direct)
      ck(cudaMemcpyAsync((char*)arena_direct->ptr + p.off, p.host, p.len, cudaMemcpyHostToDevice, s_), "H2D");
    for (const Run& r : runs) {
      ck(cudaMemcpyAsync((char*)arena_direct->ptr + r.off, r.a, (size_t)(r.b - r.a), cudaMemcpyHostToDevice, s_),
         "H2D");
      stats.h2d_bytes += (size_t)(r.b - r.a);
    }
    for (const ImagePiece& p : direct) stats.h2d_bytes += p.len;
  }
  if (total) {
    arena = std::make_shared<DeviceBuf>(dev_, total);
    upload_image(staged, total, (char*)arena->ptr);
    for (const Loc& l : viewed) buf_of(l.v) = std::make_shared<DeviceBuf>(arena, l.off, l.v->bytes());
  }
  auto at = [&](const Loc& l) {
    return (const char*)(l.is_direct ? arena_direct->ptr : arena->ptr) + l.off;
  };
  if (!aux_) aux_ = std::make_unique<DeviceBuf>(dev_, sizeof(dcf_status));
  dcf_status* st = (dcf_status*)aux_->ptr;
  check(dcf_status_reset_async(st, s_), "status reset");
  // Every literal is decoded by one batched launch; long literals are cut
  // into pieces of at most kPieceChars characters so the grid stays even.
  constexpr uint64_t kPieceChars = 4u << 20;
  std::vector<dcf_hex_piece> pieces;
  for (const Loc& l : text) {
    const uint64_t nchars = l.v->hex.size();
    for (uint64_t c = 0; c < nchars; c += kPieceChars) {
      const uint64_t len = std::min<uint64_t>(kPieceChars, nchars - c);
      pieces.push_back({at(l) + c, (char*)buf_of(l.v)->ptr + c / 2, len});
    }
  }
  std::unique_ptr<DeviceBuf> pdesc;
  if (!pieces.empty()) {
    // pieces of similar length together, one launch per length class
    std::stable_sort(pieces.begin(), pieces.end(),
                     [](const dcf_hex_piece& x, const dcf_hex_piece& y) { return x.nchars < y.nchars; });
    pdesc = std::make_unique<DeviceBuf>(dev_, pieces.size() * sizeof(dcf_hex_piece));
    ck(cudaMemcpyAsync(pdesc->ptr, pieces.data(), pieces.size() * sizeof(dcf_hex_piece), cudaMemcpyHostToDevice, s_),
       "H2D pieces");
    auto cls = [](uint64_t n) { return n ? 64 - __builtin_clzll(n) : 0; };
    for (size_t a = 0; a < pieces.size();) {
      size_t b = a + 1;
      while (b < pieces.size() && cls(pieces[b].nchars) == cls(pieces[a].nchars)) b++;
      check(dcf_hex_decode_many_async((const dcf_hex_piece*)pdesc->ptr + a, b - a, pieces[b - 1].nchars, st, s_),
            "hex decode");
      a = b;
    }
  }
  for (const Loc& l : raw)
    ck(cudaMemcpyAsync(buf_of(l.v)->ptr, at(l), l.v->bytes(), cudaMemcpyDeviceToDevice, s_), "D2D");
  for (DenseValue* v : vs)
    if (v->host.empty() && v->hex.empty())
      ck(cudaMemcpyPeerAsync(buf_of(v)->ptr, dev_, v->dev->ptr, v->dev->device, v->bytes(), s_), "peer copy");
  // Hashes of the new device copies (constant deduplication compares
  // hashes first), read back with the decode status.
  std::vector<uint64_t> hashes(vs.size(), 0);
  std::unique_ptr<DeviceBuf> hdesc, hout;
  hash_async(bufs, vs, hdesc, hout);
  dcf_status h;
  ck(cudaMemcpyAsync(&h, st, sizeof h, cudaMemcpyDeviceToHost, s_), "D2H status");
  if (hout) ck(cudaMemcpyAsync(hashes.data(), hout->ptr, vs.size() * 8, cudaMemcpyDeviceToHost, s_), "D2H hashes");
  sync();
  if (h.first_fail != ~0ull) throw std::runtime_error("invalid hex digit in a dense literal");
  for (size_t i = 0; i < vs.size(); i++) {
    vs[i]->dev = bufs[i];
    if (hout) {
      vs[i]->hash = hashes[i];
      vs[i]->hashed = true;
    }
  }
}

// Queue dcf_hash_many_async over device buffers (sizes from the values).
void Engine::hash_async(const std::vector<std::shared_ptr<DeviceBuf>>& bufs, const std::vector<DenseValue*>& vs,
                        std::unique_ptr<DeviceBuf>& desc, std::unique_ptr<DeviceBuf>& out) {
  std::vector<dcf_hash_piece> pcs(bufs.size());
  for (size_t i = 0; i < bufs.size(); i++) pcs[i] = {bufs[i] ? bufs[i]->ptr : nullptr, bufs[i] ? vs[i]->bytes() : 0};
  if (pcs.empty()) return;
  desc = std::make_unique<DeviceBuf>(dev_, pcs.size() * sizeof(dcf_hash_piece));
  out = std::make_unique<DeviceBuf>(dev_, pcs.size() * sizeof(uint64_t));
  ck(cudaMemcpyAsync(desc->ptr, pcs.data(), pcs.size() * sizeof(dcf_hash_piece), cudaMemcpyHostToDevice, s_),
     "H2D hash pieces");
  // The grid follows the longest piece of a launch: pieces within a factor
  // of two of each other's length go in one launch (runs of the given
  // order), so a few long pieces do not widen the grid of many short ones.
  auto cls = [](uint64_t n) { return n ? 64 - __builtin_clzll(n) : 0; };
  for (size_t a = 0; a < pcs.size();) {
    size_t b = a + 1;
    uint64_t maxb = pcs[a].nbytes;
    while (b < pcs.size() && cls(pcs[b].nbytes) == cls(pcs[a].nbytes)) maxb = std::max(maxb, pcs[b++].nbytes);
    check(dcf_hash_many_async((const dcf_hash_piece*)desc->ptr + a, b - a, maxb, (uint64_t*)out->ptr + a, s_),
          "hash");
    a = b;
  }
}

uint64_t Engine::hash_of(DenseValue& v) {
  if (v.hashed) return v.hash;
  to_device(v);  // hashes it when it uploads
  if (!v.hashed) {
    std::unique_ptr<DeviceBuf> d, o;
    hash_async({v.dev}, {&v}, d, o);
    ck(cudaMemcpyAsync(&v.hash, o->ptr, 8, cudaMemcpyDeviceToHost, s_), "D2H hash");
    sync();
    v.hashed = true;
  }
  return v.hash;
}

void Engine::to_host_all(const std::vector<DenseValue*>& in) {
  const auto t0 = std::chrono::steady_clock::now();
  std::vector<DenseValue*> vs;
  std::unordered_map<DenseValue*, int> seen;
  for (DenseValue* v : in) {
    if (!v || !v->host.empty() || v->bytes() == 0 || !seen.emplace(v, 0).second) continue;
    if (v->poison) throw std::runtime_error("a poison value has no bytes");
    if (!v->hex.empty() && v->hex.size() <= kSmallHex) {
      decode_small(v->hex, v->host);
      continue;
    }
    vs.push_back(v);
  }
  if (vs.empty()) return;
  std::vector<DenseValue*> off_device;
  for (DenseValue* v : vs)
    if (!v->dev || v->dev->device != dev_) off_device.push_back(v);
  to_device_all(off_device);
  set_device();
  // Host bytes in page-locked memory take the copy straight from HBM; the
  // rest go through the staging slots.
  std::vector<ImagePiece> pcs;
  size_t total = 0, direct = 0;
  for (DenseValue* v : vs) {
    if (v->host.data() == nullptr || v->host.size() != v->bytes()) v->host.resize(v->bytes());
    if (PinnedPool::get().owned(v->host.data())) {
      ck(cudaMemcpyAsync(v->host.data(), v->dev->ptr, v->bytes(), cudaMemcpyDeviceToHost, s_), "D2H");
      direct += v->bytes();
      continue;
    }
    pcs.push_back({v->host.data(), v->dev->ptr, v->bytes(), total});
    total = align16(total + v->bytes());
  }
  stats.d2h_bytes += direct;
  if (!pcs.empty()) download_image(pcs, total);
  sync();
  stats.download_ms += std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
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
  if (v.bytes() == 0) {
    v.dev = std::make_shared<DeviceBuf>(dev_, 0);
    return;
  }
  to_device_all({&v});
}

void Engine::to_host(DenseValue& v) { to_host_all({&v}); }

uint64_t Engine::bits0_of(DenseValue& v) {
  if (v.host.empty() && !v.hex.empty()) {
    Bytes b;
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
  set_device();
  const size_t R = reqs.size();
  // Every streamed operand is made resident before the batch's statuses
  // are reset and its kernels are queued.
  {
    std::vector<DenseValue*> ins;
    for (FoldRequest* q : reqs) {
      if (q->lhs && !q->lhs->splat) ins.push_back(q->lhs.get());
      if (q->rhs && !q->rhs->splat) ins.push_back(q->rhs.get());
      if (q->cond && !q->cond->splat) ins.push_back(q->cond.get());
    }
    to_device_all(ins);
  }
  const auto t1 = std::chrono::steady_clock::now();
  // Statuses: one per request, and a second block for the second results
  // of two-result folds.
  dcf_status* st = statuses(2 * R);
  ck(cudaMemsetAsync(st, 0xFF, 2 * R * sizeof(dcf_status), s_), "status reset");

  // Splat operands: one element each, packed 16-byte aligned and uploaded once.
  std::vector<uint8_t> scal;
  std::vector<std::pair<size_t, size_t>> spos(R, {SIZE_MAX, SIZE_MAX});
  std::vector<size_t> cpos(R, SIZE_MAX);
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
    if (q.cond && q.cond->splat) cpos[i] = place(*q.cond);
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

  std::vector<std::shared_ptr<DeviceBuf>> outs(R), outs2(R);
  std::vector<const void*> ls(R, nullptr), rs(R, nullptr), cs(R, nullptr);
  for (size_t i = 0; i < R; i++) {
    FoldRequest& q = *reqs[i];
    ls[i] = q.lhs ? operand(*q.lhs, spos[i].first) : nullptr;
    rs[i] = q.rhs ? operand(*q.rhs, spos[i].second) : nullptr;
    cs[i] = q.cond ? operand(*q.cond, cpos[i]) : nullptr;
    if (q.kind != FoldRequest::SPLAT_SCAN)
      outs[i] = std::make_shared<DeviceBuf>(dev_, q.n * dcf_dtype_size((dcf_dtype)q.out_dtype));
    if (q.op2) outs2[i] = std::make_shared<DeviceBuf>(dev_, q.n * dcf_dtype_size((dcf_dtype)q.out2_dtype));
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
          q.n <= (4u << 20) && !q.op2)
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
        if (q.op2)
          check(dcf_binary_async((dcf_op)q.op2, (dcf_dtype)q.dtype, l, q.lhs->splat, r, q.rhs->splat, q.n, q.flags2,
                                 outs2[i]->ptr, st + R + i, s_),
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
        check(dcf_permute_status_async(oes, (int)q.shape.size(), q.shape.data(), q.perms.data(), l, outs[i]->ptr,
                                       st + i, s_),
              "transpose fold");
        break;
      case FoldRequest::SPLAT_SCAN:
        check(dcf_splat_check_async(l, q.lhs->es, q.lhs->n, st + i, s_), "splat scan");
        break;
      case FoldRequest::SELECT:
        check(dcf_select_async(oes, cs[i], q.cond->splat, l, q.lhs->splat, r, q.rhs->splat, q.n, outs[i]->ptr, st + i,
                               s_),
              "select fold");
        break;
    }
  }
  // Hashes of every result (used by constant deduplication), read back
  // with the statuses.
  std::vector<uint64_t> rh(2 * R, 0);
  std::unique_ptr<DeviceBuf> hdesc, hout;
  {
    std::vector<std::shared_ptr<DeviceBuf>> hb(2 * R);
    std::vector<DenseValue> sizes(2 * R);
    std::vector<DenseValue*> sv(2 * R);
    for (size_t i = 0; i < R; i++) {
      const FoldRequest& q = *reqs[i];
      if (q.kind == FoldRequest::SPLAT_SCAN) continue;
      hb[i] = outs[i];
      sizes[i].n = q.n;
      sizes[i].es = dcf_dtype_size((dcf_dtype)q.out_dtype);
      if (q.op2) {
        hb[R + i] = outs2[i];
        sizes[R + i].n = q.n;
        sizes[R + i].es = dcf_dtype_size((dcf_dtype)q.out2_dtype);
      }
    }
    for (size_t i = 0; i < 2 * R; i++) sv[i] = &sizes[i];
    hash_async(hb, sv, hdesc, hout);
  }
  std::vector<dcf_status> hst(2 * R);
  ck(cudaMemcpyAsync(hst.data(), st, 2 * R * sizeof(dcf_status), cudaMemcpyDeviceToHost, s_), "D2H status");
  if (hout) ck(cudaMemcpyAsync(rh.data(), hout->ptr, 2 * R * 8, cudaMemcpyDeviceToHost, s_), "D2H hashes");
  sync();
  for (size_t i = 0; i < R; i++)
    if (batched[i]) hst[i] = bst[i];
  // First element of every all-equal result, fetched together.
  std::vector<uint64_t> first(2 * R, 0);
  bool any = false;
  for (size_t i = 0; i < R; i++) {
    FoldRequest& q = *reqs[i];
    if (hst[i].error != 0xFFFFFFFFu || (q.op2 && hst[R + i].error != 0xFFFFFFFFu))
      throw std::runtime_error("a fold kernel gave up waiting for its copies");
    if (q.kind == FoldRequest::SPLAT_SCAN || q.kind == FoldRequest::PERMUTE) continue;
    for (size_t k = 0; k < (q.op2 ? 2u : 1u); k++) {
      const dcf_status& h = hst[k * R + i];
      if (h.first_fail == ~0ull && h.splat_word != 0) {
        const size_t oes = dcf_dtype_size((dcf_dtype)(k ? q.out2_dtype : q.out_dtype));
        ck(cudaMemcpyAsync(&first[k * R + i], (k ? outs2 : outs)[i]->ptr, oes, cudaMemcpyDeviceToHost, s_),
           "D2H element");
        any = true;
      }
    }
  }
  if (any) sync();
  // A folded result: one element if the kernel saw all values equal (as
  // MLIR stores a splat), else the device buffer.
  auto result = [&](const FoldRequest& q, const dcf_status& h, const std::shared_ptr<DeviceBuf>& buf, int dtype,
                    const TypeP& ty, uint64_t first_bits) {
    auto d = std::make_shared<DenseValue>();
    d->ty = ty;
    d->elements = q.out_elements;
    d->dtype = dtype;
    d->es = dcf_dtype_size((dcf_dtype)dtype);
    if (q.kind != FoldRequest::PERMUTE && h.splat_word != 0) {
      d->splat = true;
      d->n = 1;
      d->host.resize(d->es);
      memcpy(d->host.data(), &first_bits, d->es);
    } else {
      d->n = q.n;
      d->dev = buf;
      // The kernel's splat test already said the values differ.
      if (q.kind != FoldRequest::PERMUTE) d->all_equal = 0;
    }
    if (q.kind == FoldRequest::PERMUTE && q.lhs->all_equal == 1) d->all_equal = 1;
    return d;
  };
  for (size_t i = 0; i < R; i++) {
    FoldRequest& q = *reqs[i];
    stats.requests++;
    if (q.kind == FoldRequest::SPLAT_SCAN) {
      q.lhs->all_equal = (q.lhs->n <= 1 || hst[i].splat_word != 0) ? 1 : 0;
      continue;
    }
    q.first_fail = q.kind == FoldRequest::PERMUTE ? ~0ull : hst[i].first_fail;
    if (q.op2 && hst[R + i].first_fail < q.first_fail) q.first_fail = hst[R + i].first_fail;
    q.folded = q.first_fail == ~0ull;
    if (!q.folded) continue;
    q.out = result(q, hst[i], outs[i], q.out_dtype, q.out_ty, first[i]);
    if (q.out->dev) {
      q.out->hash = rh[i];
      q.out->hashed = true;
    }
    if (q.op2) {
      q.out2 = result(q, hst[R + i], outs2[i], q.out2_dtype, q.out2_ty, first[R + i]);
      if (q.out2->dev) {
        q.out2->hash = rh[R + i];
        q.out2->hashed = true;
      }
    }
  }
  stats.batches++;
  stats.device_ms += std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t1).count();
}

}  // namespace dco
