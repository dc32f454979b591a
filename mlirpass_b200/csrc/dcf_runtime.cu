// dcf_runtime.cu — host runtime and C ABI of libdcfold.so.
//
// The reference folds on host threads, one task per isolated function
// (src/pass.rs:280-341), with the attribute bytes in a host arena.  Here a
// fold call:
//   1. splits its element range into row blocks, one per GPU chosen by
//      dcf_init, each driven by its own host thread (no collective: the
//      blocks are independent; the host ANDs the per-GPU outcomes);
//   2. streams each block through the GPU in chunks on two CUDA streams:
//      host->device copy, the fused fold kernel, device->host copy, so the
//      copy engines in both directions and the SMs work at the same time;
//      pinned caller buffers are copied directly, pageable ones through the
//      library's pinned double buffers;
//   3. reads back one 16-byte status per GPU: lowest refusing index and
//      the splat flag.
// There is no CPU fallback: without a GPU every compute call fails with
// DCF_ENODEV and says so in dcf_last_error().
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "dcf_launch.h"

using namespace dcf;

namespace {

thread_local std::string g_err;

}  // namespace

int dcf::record_error(int code, const char* msg) {
  g_err = msg;
  return code;
}

namespace {

int set_err(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

#define CK(call)                                                                                   \
  do {                                                                                             \
    cudaError_t e_ = (call);                                                                       \
    if (e_ != cudaSuccess)                                                                         \
      return set_err(DCF_ECUDA, "%s failed: %s (%s:%d)", #call, cudaGetErrorString(e_), __FILE__, \
                     __LINE__);                                                                    \
  } while (0)

constexpr size_t kChunkBytes = 32ull << 20;  // per operand per slot (whole-tensor staging)
constexpr uint64_t kAlignElems = 64;         // row-block / chunk granularity
constexpr int kPipeSlots = 4;                // elementwise pipeline depth
constexpr size_t kPipeChunk = 8ull << 20;    // bytes of the widest operand per pipeline chunk

long timeout_ms() {
  static long t = [] {
    const char* s = getenv("DCF_TIMEOUT_MS");
    return s ? atol(s) : 120000L;
  }();
  return t;
}

// Wait for an event with a bound; the kernels have no device-side waits, so
// this only guards against a wedged device or driver.
int wait_event(cudaEvent_t ev) {
  const auto t0 = std::chrono::steady_clock::now();
  int spins = 0;
  for (;;) {
    cudaError_t e = cudaEventQuery(ev);
    if (e == cudaSuccess) return DCF_OK;
    if (e != cudaErrorNotReady) return set_err(DCF_ECUDA, "cudaEventQuery: %s", cudaGetErrorString(e));
    if (++spins > 64) std::this_thread::sleep_for(std::chrono::microseconds(20));
    const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count();
    if (ms > timeout_ms()) return set_err(DCF_ETIMEOUT, "GPU work did not finish within %ld ms", timeout_ms());
  }
}

struct Dev {
  int id = 0;
  cudaStream_t s[2] = {nullptr, nullptr};
  cudaEvent_t ev[2] = {nullptr, nullptr};
  cudaEvent_t start = nullptr;
  void* d[2][3] = {{nullptr}};  // per slot: lhs, rhs, out chunk buffers
  void* h[2][3] = {{nullptr}};  // per slot: pinned staging
  dcf_status* st = nullptr;
  void* d0 = nullptr;           // 32 bytes: lhs element 0 at +0, rhs element 0 at +16
  void* big[4] = {nullptr};     // whole-tensor buffers (transpose, select, batch)
  size_t big_cap[4] = {0};
  void* hbig = nullptr;         // pinned whole-batch staging
  size_t hbig_cap = 0;
  // Elementwise pipeline: copy-in, compute and copy-out streams, with
  // kPipeSlots rotating chunk buffers (lhs, rhs, out) and one event per
  // slot and stage.
  cudaStream_t sin = nullptr, scomp = nullptr, sout = nullptr;
  cudaEvent_t evin[kPipeSlots] = {nullptr}, evcomp[kPipeSlots] = {nullptr}, evout[kPipeSlots] = {nullptr};
  void* pd[kPipeSlots][3] = {{nullptr}};
  void* ph[kPipeSlots][3] = {{nullptr}};
  std::mutex mu;
};

std::mutex g_mu;
std::vector<std::unique_ptr<Dev>> g_devs;
bool g_ready = false;

int dev_setup(Dev& d) {
  CK(cudaSetDevice(d.id));
  for (int k = 0; k < 2; k++) {
    CK(cudaStreamCreateWithFlags(&d.s[k], cudaStreamNonBlocking));
    CK(cudaEventCreateWithFlags(&d.ev[k], cudaEventDisableTiming));
    for (int j = 0; j < 3; j++) {
      CK(cudaMalloc(&d.d[k][j], kChunkBytes));
      CK(cudaHostAlloc(&d.h[k][j], kChunkBytes, cudaHostAllocPortable));
    }
  }
  CK(cudaEventCreateWithFlags(&d.start, cudaEventDisableTiming));
  CK(cudaStreamCreateWithFlags(&d.sin, cudaStreamNonBlocking));
  CK(cudaStreamCreateWithFlags(&d.scomp, cudaStreamNonBlocking));
  CK(cudaStreamCreateWithFlags(&d.sout, cudaStreamNonBlocking));
  for (int k = 0; k < kPipeSlots; k++) {
    CK(cudaEventCreateWithFlags(&d.evin[k], cudaEventDisableTiming));
    CK(cudaEventCreateWithFlags(&d.evcomp[k], cudaEventDisableTiming));
    CK(cudaEventCreateWithFlags(&d.evout[k], cudaEventDisableTiming));
    for (int j = 0; j < 3; j++) {
      CK(cudaMalloc(&d.pd[k][j], kPipeChunk));
      CK(cudaHostAlloc(&d.ph[k][j], kPipeChunk, cudaHostAllocPortable));
    }
  }
  CK(cudaMalloc((void**)&d.st, sizeof(dcf_status)));
  CK(cudaMalloc(&d.d0, 32));
  return DCF_OK;
}

void dev_free(Dev& d) {
  cudaSetDevice(d.id);
  for (int k = 0; k < 2; k++) {
    if (d.s[k]) cudaStreamSynchronize(d.s[k]);
    for (int j = 0; j < 3; j++) {
      if (d.d[k][j]) cudaFree(d.d[k][j]);
      if (d.h[k][j]) cudaFreeHost(d.h[k][j]);
    }
    if (d.ev[k]) cudaEventDestroy(d.ev[k]);
    if (d.s[k]) cudaStreamDestroy(d.s[k]);
  }
  if (d.start) cudaEventDestroy(d.start);
  for (cudaStream_t x : {d.sin, d.scomp, d.sout})
    if (x) cudaStreamSynchronize(x);
  for (int k = 0; k < kPipeSlots; k++) {
    for (int j = 0; j < 3; j++) {
      if (d.pd[k][j]) cudaFree(d.pd[k][j]);
      if (d.ph[k][j]) cudaFreeHost(d.ph[k][j]);
    }
    for (cudaEvent_t e : {d.evin[k], d.evcomp[k], d.evout[k]})
      if (e) cudaEventDestroy(e);
  }
  for (cudaStream_t x : {d.sin, d.scomp, d.sout})
    if (x) cudaStreamDestroy(x);
  for (int j = 0; j < 4; j++)
    if (d.big[j]) cudaFree(d.big[j]);
  if (d.hbig) cudaFreeHost(d.hbig);
  if (d.st) cudaFree(d.st);
  if (d.d0) cudaFree(d.d0);
}

int init_locked(int n_gpus) {
  int visible = 0;
  cudaError_t e = cudaGetDeviceCount(&visible);
  if (e != cudaSuccess || visible <= 0)
    return set_err(DCF_ENODEV, "no CUDA device available (%s); libdcfold has no CPU fallback",
                   e == cudaSuccess ? "0 devices" : cudaGetErrorString(e));
  std::vector<int> ids;
  if (const char* env = getenv("DCF_DEVICES")) {
    std::string s(env);
    size_t pos = 0;
    while (pos < s.size()) {
      size_t c = s.find(',', pos);
      std::string tok = s.substr(pos, c == std::string::npos ? std::string::npos : c - pos);
      if (!tok.empty()) ids.push_back(atoi(tok.c_str()));
      if (c == std::string::npos) break;
      pos = c + 1;
    }
  } else {
    const int n = (n_gpus <= 0 || n_gpus > visible) ? visible : n_gpus;
    int cur = 0;
    cudaGetDevice(&cur);
    if (n == 1) ids.push_back(cur);
    else
      for (int i = 0; i < n; i++) ids.push_back(i);
  }
  for (int id : ids)
    if (id < 0 || id >= visible) return set_err(DCF_EINVAL, "device %d out of range (%d visible)", id, visible);
  for (auto& d : g_devs) dev_free(*d);
  g_devs.clear();
  int prev = 0;
  cudaGetDevice(&prev);
  for (int id : ids) {
    auto d = std::make_unique<Dev>();
    d->id = id;
    int rc = dev_setup(*d);
    if (rc) {
      cudaSetDevice(prev);
      dev_free(*d);
      return rc;
    }
    g_devs.push_back(std::move(d));
  }
  cudaSetDevice(prev);
  g_ready = true;
  return (int)g_devs.size();
}

int ensure_init() {
  std::lock_guard<std::mutex> g(g_mu);
  if (g_ready) return DCF_OK;
  int rc = init_locked(1);
  return rc < 0 ? rc : DCF_OK;
}

bool is_pinned(const void* p) {
  if (!p) return false;
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return a.type == cudaMemoryTypeHost;
}

// Copy host -> device in full (synchronous for the caller).  Pinned
// sources go straight to the copy engine; pageable ones are staged through
// the device's two pinned chunk buffers so the memcpy into one overlaps
// the DMA out of the other.
int h2d_full(Dev& d, void* dst, const void* src, size_t bytes, cudaStream_t s) {
  if (bytes == 0) return DCF_OK;
  if (is_pinned(src)) {
    CK(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, s));
    return DCF_OK;
  }
  size_t off = 0;
  int k = 0;
  bool used[2] = {false, false};
  while (off < bytes) {
    const size_t n = std::min(kChunkBytes, bytes - off);
    if (used[k]) {
      int rc = wait_event(d.ev[k]);
      if (rc) return rc;
    }
    memcpy(d.h[k][0], (const char*)src + off, n);
    CK(cudaMemcpyAsync((char*)dst + off, d.h[k][0], n, cudaMemcpyHostToDevice, s));
    CK(cudaEventRecord(d.ev[k], s));
    used[k] = true;
    off += n;
    k ^= 1;
  }
  // The staging buffers are free again only when their copies are done: a
  // following h2d_full (another operand) refills them from the start.
  for (int j = 0; j < 2; j++)
    if (used[j]) {
      int rc = wait_event(d.ev[j]);
      if (rc) return rc;
    }
  return DCF_OK;
}

int d2h_full(Dev& d, void* dst, const void* src, size_t bytes, cudaStream_t s) {
  if (bytes == 0) return DCF_OK;
  if (is_pinned(dst)) {
    CK(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, s));
    CK(cudaEventRecord(d.ev[0], s));
    return wait_event(d.ev[0]);
  }
  size_t off = 0, pend_off[2] = {0, 0}, pend_n[2] = {0, 0};
  int k = 0;
  while (off < bytes) {
    const size_t n = std::min(kChunkBytes, bytes - off);
    if (pend_n[k]) {
      int rc = wait_event(d.ev[k]);
      if (rc) return rc;
      memcpy((char*)dst + pend_off[k], d.h[k][2], pend_n[k]);
    }
    CK(cudaMemcpyAsync(d.h[k][2], (const char*)src + off, n, cudaMemcpyDeviceToHost, s));
    CK(cudaEventRecord(d.ev[k], s));
    pend_off[k] = off;
    pend_n[k] = n;
    off += n;
    k ^= 1;
  }
  for (int j = 0; j < 2; j++) {
    k ^= 1;
    if (pend_n[k]) {
      int rc = wait_event(d.ev[k]);
      if (rc) return rc;
      memcpy((char*)dst + pend_off[k], d.h[k][2], pend_n[k]);
      pend_n[k] = 0;
    }
  }
  return DCF_OK;
}

int ensure_big(Dev& d, int j, size_t bytes) {
  if (d.big_cap[j] >= bytes) return DCF_OK;
  if (d.big[j]) cudaFree(d.big[j]);
  d.big[j] = nullptr;
  d.big_cap[j] = 0;
  const size_t cap = std::max(bytes, (size_t)1 << 20);
  CK(cudaMalloc(&d.big[j], cap));
  d.big_cap[j] = cap;
  return DCF_OK;
}

int read_status(Dev& d, cudaStream_t s, dcf_status* out) {
  CK(cudaMemcpyAsync(out, d.st, sizeof(dcf_status), cudaMemcpyDeviceToHost, s));
  CK(cudaEventRecord(d.ev[0], s));
  int rc = wait_event(d.ev[0]);
  if (rc) return rc;
  if (out->error != 0xFFFFFFFFu) return set_err(DCF_ETIMEOUT, "a fold kernel gave up waiting for its own copies");
  return DCF_OK;
}

struct EwJob {
  int op, dtype, out_dtype;
  uint32_t flags;
  const void* l;
  int lsplat;
  const void* r;
  int rsplat;
  bool binary;
  void* out;
  size_t ies, oes;
};

// One GPU's row block [lo, hi) of an elementwise fold.
//
// Chunk k uses slot k % kPipeSlots.  Three streams keep both copy engines
// and the SMs busy at once:
//   copy-in  : waits until compute(k - S) has consumed the slot, then H2D;
//   compute  : waits for copy-in(k) and for copy-out(k - S) to have drained
//              the slot's output, then the fold kernel;
//   copy-out : waits for compute(k), then D2H.
// Pinned caller buffers are copied directly; pageable ones go through the
// slot's pinned staging buffers, which the host fills and empties around
// the same events.
int run_block(Dev& d, const EwJob& j, uint64_t lo, uint64_t hi, dcf_status* st_out) {
  std::lock_guard<std::mutex> g(d.mu);
  CK(cudaSetDevice(d.id));
  constexpr int S = kPipeSlots;
  CK(cudaMemsetAsync(d.st, 0xFF, sizeof(dcf_status), d.scomp));
  CK(cudaMemcpyAsync(d.d0, j.l, j.ies, cudaMemcpyHostToDevice, d.scomp));
  if (j.binary) CK(cudaMemcpyAsync((char*)d.d0 + 16, j.r, j.ies, cudaMemcpyHostToDevice, d.scomp));

  const bool lp = j.lsplat || is_pinned(j.l);
  const bool rp = !j.binary || j.rsplat || is_pinned(j.r);
  const bool op = is_pinned(j.out);
  const size_t es = std::max(j.ies, j.oes);
  const uint64_t chunk = std::max<uint64_t>(kAlignElems, (kPipeChunk / es) / kAlignElems * kAlignElems);
  uint64_t pend_off[S] = {0}, pend_n[S] = {0};  // pageable output waiting in slot staging
  bool used[S] = {false};
  uint64_t k = 0;
  for (uint64_t off = lo; off < hi; off += chunk, k++) {
    const int t = (int)(k % S);
    const uint64_t cnt = std::min<uint64_t>(chunk, hi - off);
    if (used[t]) {
      // The slot's previous chunk: its inputs are consumed once its kernel
      // ran; its pageable output is copied out once its D2H finished.
      CK(cudaStreamWaitEvent(d.sin, d.evcomp[t], 0));
      if (!lp || !rp) {
        int rc = wait_event(d.evin[t]);
        if (rc) return rc;
      }
      if (pend_n[t]) {
        int rc = wait_event(d.evout[t]);
        if (rc) return rc;
        memcpy((char*)j.out + pend_off[t] * j.oes, d.ph[t][2], pend_n[t] * j.oes);
        pend_n[t] = 0;
      }
    }
    const void* ldev = d.d0;
    const void* rdev = (char*)d.d0 + 16;
    if (!j.lsplat) {
      const void* src = (const char*)j.l + off * j.ies;
      if (!lp) {
        memcpy(d.ph[t][0], src, cnt * j.ies);
        src = d.ph[t][0];
      }
      CK(cudaMemcpyAsync(d.pd[t][0], src, cnt * j.ies, cudaMemcpyHostToDevice, d.sin));
      ldev = d.pd[t][0];
    }
    if (j.binary && !j.rsplat) {
      const void* src = (const char*)j.r + off * j.ies;
      if (!rp) {
        memcpy(d.ph[t][1], src, cnt * j.ies);
        src = d.ph[t][1];
      }
      CK(cudaMemcpyAsync(d.pd[t][1], src, cnt * j.ies, cudaMemcpyHostToDevice, d.sin));
      rdev = d.pd[t][1];
    }
    CK(cudaEventRecord(d.evin[t], d.sin));
    CK(cudaStreamWaitEvent(d.scomp, d.evin[t], 0));
    if (used[t]) CK(cudaStreamWaitEvent(d.scomp, d.evout[t], 0));
    EwLaunch a;
    a.op = j.op;
    a.dtype = j.dtype;
    a.out_dtype = j.out_dtype;
    a.flags = j.flags;
    a.l = ldev;
    a.r = j.binary ? rdev : nullptr;
    a.o = d.pd[t][2];
    a.n = cnt;
    a.l0 = d.d0;
    a.r0 = (char*)d.d0 + 16;
    a.lsplat = j.lsplat;
    a.rsplat = j.rsplat;
    a.base = off;
    a.st = d.st;
    a.stream = d.scomp;
    int rc = launch_ew(a);
    if (rc == DCF_EUNSUPPORTED)
      return set_err(rc, "op %d on dtype %d -> %d is not supported", j.op, j.dtype, j.out_dtype);
    if (rc) return set_err(rc, "kernel launch failed: %s", cudaGetErrorString(cudaGetLastError()));
    CK(cudaEventRecord(d.evcomp[t], d.scomp));
    CK(cudaStreamWaitEvent(d.sout, d.evcomp[t], 0));
    if (op) {
      CK(cudaMemcpyAsync((char*)j.out + off * j.oes, d.pd[t][2], cnt * j.oes, cudaMemcpyDeviceToHost, d.sout));
    } else {
      CK(cudaMemcpyAsync(d.ph[t][2], d.pd[t][2], cnt * j.oes, cudaMemcpyDeviceToHost, d.sout));
      pend_off[t] = off;
      pend_n[t] = cnt;
    }
    CK(cudaEventRecord(d.evout[t], d.sout));
    used[t] = true;
  }
  for (int t = 0; t < S; t++) {
    if (!used[t]) continue;
    int rc = wait_event(d.evout[t]);
    if (rc) return rc;
    if (pend_n[t]) {
      memcpy((char*)j.out + pend_off[t] * j.oes, d.ph[t][2], pend_n[t] * j.oes);
      pend_n[t] = 0;
    }
  }
  CK(cudaEventRecord(d.start, d.scomp));
  CK(cudaStreamWaitEvent(d.s[0], d.start, 0));
  return read_status(d, d.s[0], st_out);
}

int run_elementwise(const EwJob& j, uint64_t n, dcf_result* res) {
  if (res) {
    memset(res, 0, sizeof *res);
    res->first_fail_index = UINT64_MAX;
  }
  int rc = ensure_init();
  if (rc) return rc;
  if (n == 0) {
    if (res) res->folded = 1, res->is_splat = 1;
    return DCF_OK;
  }
  const size_t G = g_devs.size();
  // Small folds stay on one GPU; large ones split into row blocks.
  const uint64_t min_block = 1ull << 20;
  size_t use = std::max<size_t>(1, std::min<uint64_t>(G, n / min_block));
  std::vector<uint64_t> cut(use + 1, 0);
  for (size_t g = 0; g <= use; g++) {
    uint64_t c = n * g / use;
    c = (g == use) ? n : c / kAlignElems * kAlignElems;
    cut[g] = c;
  }
  std::vector<dcf_status> st(use);
  std::vector<int> rcs(use, 0);
  std::vector<std::string> errs(use);
  if (use == 1) {
    rcs[0] = run_block(*g_devs[0], j, 0, n, &st[0]);
  } else {
    std::vector<std::thread> th;
    for (size_t g = 0; g < use; g++)
      th.emplace_back([&, g] {
        rcs[g] = run_block(*g_devs[g], j, cut[g], cut[g + 1], &st[g]);
        if (rcs[g]) errs[g] = g_err;
      });
    for (auto& t : th) t.join();
  }
  uint64_t first = UINT64_MAX;
  bool splat = true;
  for (size_t g = 0; g < use; g++) {
    if (rcs[g]) {
      if (use > 1) g_err = errs[g];
      return rcs[g];
    }
    first = std::min<uint64_t>(first, st[g].first_fail);
    splat = splat && st[g].splat_word != 0;
  }
  if (res) {
    res->first_fail_index = first;
    res->folded = first == UINT64_MAX;
    res->is_splat = res->folded && splat;
  }
  return DCF_OK;
}

bool binary_op(int op) { return op_binary(op); }

bool convert_op(int op) { return op_convert(op); }

int check_binary(int op, int dtype) {
  if (!binary_op(op)) return set_err(DCF_EINVAL, "op %d is not a binary fold", op);
  const bool fop = op_float_binary(op);
  if (fop && !is_float(dtype)) return set_err(DCF_EINVAL, "op %d needs a float dtype, got %d", op, dtype);
  if (!fop && !is_int(dtype)) return set_err(DCF_EINVAL, "op %d needs an integer dtype, got %d", op, dtype);
  return DCF_OK;
}

int check_convert(int op, int from, int to) {
  if (!convert_op(op)) return set_err(DCF_EINVAL, "op %d is not a conversion fold", op);
  const bool ok = convert_types_ok(op, is_float(from), is_int(from), is_float(to), is_int(to), from, to);
  if (!ok) return set_err(DCF_EINVAL, "op %d cannot convert dtype %d to %d", op, from, to);
  return DCF_OK;
}

}  // namespace

// ======================================================================
// C ABI
// ======================================================================

extern "C" {

const char* dcf_last_error(void) { return g_err.c_str(); }

const char* dcf_version(void) { return "dcfold 0.1 (sm_100a)"; }

size_t dcf_dtype_size(dcf_dtype dtype) { return dtype_size(dtype); }

uint64_t dcf_kernel_launches(void) { return launches(); }

int dcf_init(int n_gpus) {
  std::lock_guard<std::mutex> g(g_mu);
  return init_locked(n_gpus);
}

int dcf_shutdown(void) {
  std::lock_guard<std::mutex> g(g_mu);
  for (auto& d : g_devs) dev_free(*d);
  g_devs.clear();
  g_ready = false;
  return DCF_OK;
}

int dcf_device_count(void) {
  std::lock_guard<std::mutex> g(g_mu);
  return (int)g_devs.size();
}

int dcf_binary(dcf_op op, dcf_dtype dtype, const void* lhs, int lhs_splat, const void* rhs, int rhs_splat,
               uint64_t n, uint32_t flags, void* out, dcf_result* res) {
  int rc = check_binary(op, dtype);
  if (rc) return rc;
  if (n && (!lhs || !rhs || !out)) return set_err(DCF_EINVAL, "null buffer");
  const size_t es = dtype_size(dtype);
  const bool cmp = op_bool_result(op);
  EwJob j{op, dtype, dtype, flags, lhs, lhs_splat, rhs, rhs_splat, true, out, es, cmp ? 1 : es};
  return run_elementwise(j, n, res);
}

int dcf_convert(dcf_op op, dcf_dtype from, dcf_dtype to, const void* in, int in_splat, uint64_t n,
                uint32_t flags, void* out, dcf_result* res) {
  int rc = check_convert(op, from, to);
  if (rc) return rc;
  if (n && (!in || !out)) return set_err(DCF_EINVAL, "null buffer");
  EwJob j{op, from, to, flags, in, in_splat, nullptr, 0, false, out, dtype_size(from), dtype_size(to)};
  return run_elementwise(j, n, res);
}

int dcf_reciprocal(dcf_dtype dtype, const void* in, int in_splat, uint64_t n, uint32_t flags, void* out,
                   dcf_result* res) {
  if (!is_float(dtype)) return set_err(DCF_EINVAL, "reciprocal needs a float dtype, got %d", dtype);
  if (n && (!in || !out)) return set_err(DCF_EINVAL, "null buffer");
  const size_t es = dtype_size(dtype);
  EwJob j{DCF_RECIPROCAL, dtype, dtype, flags, in, in_splat, nullptr, 0, false, out, es, es};
  return run_elementwise(j, n, res);
}

int dcf_transpose(size_t elem_size, int rank, const int64_t* in_shape, const int64_t* perms, const void* in,
                  void* out, dcf_result* res) {
  if (res) {
    memset(res, 0, sizeof *res);
    res->first_fail_index = UINT64_MAX;
  }
  if (elem_size != 1 && elem_size != 2 && elem_size != 4 && elem_size != 8)
    return set_err(DCF_EINVAL, "element size %zu not supported", elem_size);
  if (rank < 1 || rank > 8 || !in_shape || !perms) return set_err(DCF_EINVAL, "bad rank or shape");
  uint64_t total = 1;
  bool seen[8] = {false};
  for (int i = 0; i < rank; i++) {
    if (in_shape[i] < 0) return set_err(DCF_EINVAL, "negative dim");
    if (perms[i] < 0 || perms[i] >= rank || seen[perms[i]]) return set_err(DCF_EINVAL, "perms is not a permutation");
    seen[perms[i]] = true;
    total *= (uint64_t)in_shape[i];
  }
  int rc = ensure_init();
  if (rc) return rc;
  if (total == 0) {
    if (res) res->folded = 1, res->is_splat = 1;
    return DCF_OK;
  }
  if (!in || !out) return set_err(DCF_EINVAL, "null buffer");
  Dev& d = *g_devs[0];
  std::lock_guard<std::mutex> g(d.mu);
  CK(cudaSetDevice(d.id));
  const size_t bytes = total * elem_size;
  if ((rc = ensure_big(d, 0, bytes)) || (rc = ensure_big(d, 1, bytes))) return rc;
  cudaStream_t s = d.s[0];
  if ((rc = h2d_full(d, d.big[0], in, bytes, s))) return rc;
  // Collapse to the 2-D [1,0] kernel when the permutation is a swap of two
  // contiguous groups of dims (rank-2 transposes included).
  int64_t rows = 1, cols = 1;
  bool swap2 = false;
  for (int split = 1; split < rank && !swap2; split++) {
    bool ok = true;
    for (int i = 0; i < rank; i++) {
      const int64_t want = (i < rank - split) ? split + i : i - (rank - split);
      if (perms[i] != want) ok = false;
    }
    if (ok) {
      swap2 = true;
      rows = 1;
      cols = 1;
      for (int i = 0; i < split; i++) rows *= in_shape[i];
      for (int i = split; i < rank; i++) cols *= in_shape[i];
    }
  }
  bool identity = true;
  for (int i = 0; i < rank; i++) identity = identity && perms[i] == i;
  CK(cudaMemsetAsync(d.st, 0xFF, sizeof(dcf_status), s));
  if (identity) {
    CK(cudaMemcpyAsync(d.big[1], d.big[0], bytes, cudaMemcpyDeviceToDevice, s));
  } else if (swap2) {
    rc = launch_transpose2d(elem_size, (uint64_t)rows, (uint64_t)cols, d.big[0], d.big[1], s, d.st);
  } else {
    rc = launch_permute(elem_size, rank, in_shape, perms, d.big[0], d.big[1], s);
  }
  if (rc) return set_err(rc, "transpose launch failed: %s", cudaGetErrorString(cudaGetLastError()));
  if ((rc = d2h_full(d, out, d.big[1], bytes, s))) return rc;
  CK(cudaStreamSynchronize(s));
  // A permutation keeps the multiset of values: splat in, splat out.  The
  // same status carries the transpose's error word.
  if ((rc = launch_splat_check(d.big[0], elem_size, total, d.st, s))) return rc;
  dcf_status st;
  if ((rc = read_status(d, s, &st))) return rc;
  if (res) {
    res->folded = 1;
    res->is_splat = st.splat_word != 0;
  }
  return DCF_OK;
}

int dcf_select(size_t elem_size, const void* cond, int cond_splat, const void* t, int t_splat, const void* f,
               int f_splat, uint64_t n, void* out, dcf_result* res) {
  if (res) {
    memset(res, 0, sizeof *res);
    res->first_fail_index = UINT64_MAX;
  }
  if (elem_size != 1 && elem_size != 2 && elem_size != 4 && elem_size != 8)
    return set_err(DCF_EINVAL, "element size %zu not supported", elem_size);
  int rc = ensure_init();
  if (rc) return rc;
  if (n == 0) {
    if (res) res->folded = 1, res->is_splat = 1;
    return DCF_OK;
  }
  if (!cond || !t || !f || !out) return set_err(DCF_EINVAL, "null buffer");
  Dev& d = *g_devs[0];
  std::lock_guard<std::mutex> g(d.mu);
  CK(cudaSetDevice(d.id));
  const size_t cb = cond_splat ? 1 : n, tb = (t_splat ? 1 : n) * elem_size, fb = (f_splat ? 1 : n) * elem_size;
  const size_t ob = n * elem_size;
  if ((rc = ensure_big(d, 0, cb)) || (rc = ensure_big(d, 1, tb)) || (rc = ensure_big(d, 2, fb)) ||
      (rc = ensure_big(d, 3, ob)))
    return rc;
  cudaStream_t s = d.s[0];
  if ((rc = h2d_full(d, d.big[0], cond, cb, s)) || (rc = h2d_full(d, d.big[1], t, tb, s)) ||
      (rc = h2d_full(d, d.big[2], f, fb, s)))
    return rc;
  CK(cudaMemsetAsync(d.st, 0xFF, sizeof(dcf_status), s));
  if ((rc = launch_select(elem_size, d.big[0], cond_splat, d.big[1], t_splat, d.big[2], f_splat, n, d.big[3], d.st,
                          s)))
    return set_err(rc, "select launch failed: %s", cudaGetErrorString(cudaGetLastError()));
  if ((rc = d2h_full(d, out, d.big[3], ob, s))) return rc;
  dcf_status st;
  if ((rc = read_status(d, s, &st))) return rc;
  if (res) {
    res->folded = 1;
    res->is_splat = st.splat_word != 0;
  }
  return DCF_OK;
}

int dcf_hex_encode(const void* in, uint64_t nbytes, char* out) {
  int rc = ensure_init();
  if (rc) return rc;
  if (nbytes == 0) return DCF_OK;
  if (!in || !out) return set_err(DCF_EINVAL, "null buffer");
  Dev& d = *g_devs[0];
  std::lock_guard<std::mutex> g(d.mu);
  CK(cudaSetDevice(d.id));
  if ((rc = ensure_big(d, 0, nbytes)) || (rc = ensure_big(d, 1, 2 * nbytes))) return rc;
  cudaStream_t s = d.s[0];
  if ((rc = h2d_full(d, d.big[0], in, nbytes, s))) return rc;
  if ((rc = launch_hex_encode(d.big[0], nbytes, (char*)d.big[1], s))) return set_err(rc, "hex encode launch failed");
  if ((rc = d2h_full(d, out, d.big[1], 2 * nbytes, s))) return rc;
  CK(cudaStreamSynchronize(s));
  return DCF_OK;
}

int dcf_hex_decode(const char* in, uint64_t nchars, void* out) {
  if (nchars & 1) return set_err(DCF_EPARSE, "odd number of hex digits (%llu)", (unsigned long long)nchars);
  int rc = ensure_init();
  if (rc) return rc;
  if (nchars == 0) return DCF_OK;
  if (!in || !out) return set_err(DCF_EINVAL, "null buffer");
  Dev& d = *g_devs[0];
  std::lock_guard<std::mutex> g(d.mu);
  CK(cudaSetDevice(d.id));
  if ((rc = ensure_big(d, 0, nchars)) || (rc = ensure_big(d, 1, nchars / 2))) return rc;
  cudaStream_t s = d.s[0];
  if ((rc = h2d_full(d, d.big[0], in, nchars, s))) return rc;
  CK(cudaMemsetAsync(d.st, 0xFF, sizeof(dcf_status), s));
  if ((rc = launch_hex_decode((const char*)d.big[0], nchars, d.big[1], d.st, s)))
    return set_err(rc, "hex decode launch failed");
  dcf_status st;
  if ((rc = read_status(d, s, &st))) return rc;
  if (st.first_fail != ~0ull)
    return set_err(DCF_EPARSE, "invalid hex digit at offset %llu", (unsigned long long)st.first_fail);
  if ((rc = d2h_full(d, out, d.big[1], nchars / 2, s))) return rc;
  CK(cudaStreamSynchronize(s));
  return DCF_OK;
}

int dcf_splat_check(const void* in, size_t elem_size, uint64_t n, int* is_splat) {
  if (!is_splat) return set_err(DCF_EINVAL, "null result");
  if (elem_size != 1 && elem_size != 2 && elem_size != 4 && elem_size != 8)
    return set_err(DCF_EINVAL, "element size %zu not supported", elem_size);
  int rc = ensure_init();
  if (rc) return rc;
  *is_splat = 1;
  if (n <= 1) return DCF_OK;
  if (!in) return set_err(DCF_EINVAL, "null buffer");
  Dev& d = *g_devs[0];
  std::lock_guard<std::mutex> g(d.mu);
  CK(cudaSetDevice(d.id));
  const size_t bytes = n * elem_size;
  if ((rc = ensure_big(d, 0, bytes))) return rc;
  cudaStream_t s = d.s[0];
  if ((rc = h2d_full(d, d.big[0], in, bytes, s))) return rc;
  CK(cudaMemsetAsync(d.st, 0xFF, sizeof(dcf_status), s));
  if ((rc = launch_splat_check(d.big[0], elem_size, n, d.st, s))) return set_err(rc, "splat launch failed");
  dcf_status st;
  if ((rc = read_status(d, s, &st))) return rc;
  *is_splat = st.splat_word != 0;
  return DCF_OK;
}

int dcf_batch(dcf_job* jobs, size_t n_jobs) {
  if (n_jobs == 0) return DCF_OK;
  if (!jobs) return set_err(DCF_EINVAL, "null job list");
  int rc = ensure_init();
  if (rc) return rc;
  // Validate and group jobs by (op, dtype, out_dtype, flags): one launch
  // per group per GPU.
  for (size_t i = 0; i < n_jobs; i++) {
    dcf_job& j = jobs[i];
    memset(&j.result, 0, sizeof j.result);
    j.result.first_fail_index = UINT64_MAX;
    const bool bin = binary_op(j.op);
    if (j.n == 0) j.result.folded = 1, j.result.is_splat = 1;
    if (bin) rc = check_binary(j.op, j.dtype);
    else if (convert_op(j.op)) rc = check_convert(j.op, j.dtype, j.out_dtype);
    else if (j.op == DCF_RECIPROCAL) rc = is_float(j.dtype) ? 0 : set_err(DCF_EINVAL, "reciprocal dtype");
    else rc = set_err(DCF_EINVAL, "job %zu: unknown op %u", i, j.op);
    if (rc) return rc;
    if (!bin && !convert_op(j.op)) j.out_dtype = j.dtype;
    if (bin) j.out_dtype = op_bool_result(j.op) ? DCF_I1 : j.dtype;
    if (j.n && (!j.lhs || !j.out || (bin && !j.rhs))) return set_err(DCF_EINVAL, "job %zu: null buffer", i);
  }
  std::vector<size_t> order;
  for (size_t i = 0; i < n_jobs; i++)
    if (jobs[i].n) order.push_back(i);
  n_jobs = order.size();
  auto key = [&](size_t i) {
    const dcf_job& j = jobs[i];
    return std::make_tuple(j.op, j.dtype, j.out_dtype, j.flags);
  };
  std::stable_sort(order.begin(), order.end(), [&](size_t a, size_t b) { return key(a) < key(b); });
  size_t gstart = 0;
  while (gstart < n_jobs) {
    size_t gend = gstart + 1;
    while (gend < n_jobs && key(order[gend]) == key(order[gstart])) gend++;
    const dcf_job& j0 = jobs[order[gstart]];
    const bool bin = binary_op(j0.op);
    const size_t ies = dtype_size(j0.dtype), oes = dtype_size(j0.out_dtype);
    // Balance the group's jobs over the GPUs by bytes (greedy, largest first).
    const size_t G = g_devs.size();
    std::vector<std::vector<size_t>> per(G);
    std::vector<uint64_t> load(G, 0);
    std::vector<size_t> gj(order.begin() + gstart, order.begin() + gend);
    std::stable_sort(gj.begin(), gj.end(), [&](size_t a, size_t b) { return jobs[a].n > jobs[b].n; });
    for (size_t i : gj) {
      size_t best = 0;
      for (size_t g = 1; g < G; g++)
        if (load[g] < load[best]) best = g;
      per[best].push_back(i);
      load[best] += jobs[i].n * (ies * (bin ? 2 : 1) + oes);
    }
    std::vector<int> rcs(G, 0);
    std::vector<std::string> errs(G);
    auto work = [&](size_t g) -> int {
      if (per[g].empty()) return DCF_OK;
      Dev& d = *g_devs[g];
      std::lock_guard<std::mutex> lk(d.mu);
      CK(cudaSetDevice(d.id));
      cudaStream_t s = d.s[0];
      // Layout: [lhs | rhs | out] per job, each 256-byte aligned; then
      // the descriptors and statuses.
      auto al = [](uint64_t x) { return (x + 255) / 256 * 256; };
      const size_t nj = per[g].size();
      std::vector<uint64_t> lo(nj), ro(nj), oo(nj);
      uint64_t in_bytes = 0, out_bytes = 0, maxn = 0;
      for (size_t t = 0; t < nj; t++) {
        const dcf_job& j = jobs[per[g][t]];
        lo[t] = in_bytes;
        in_bytes += al((j.lhs_splat ? 1 : j.n) * ies);
        ro[t] = in_bytes;
        if (bin) in_bytes += al((j.rhs_splat ? 1 : j.n) * ies);
        oo[t] = out_bytes;
        out_bytes += al(j.n * oes);
        maxn = std::max<uint64_t>(maxn, j.n);
      }
      const uint64_t desc_bytes = al(nj * sizeof(BatchDesc)), st_bytes = al(nj * sizeof(dcf_status));
      int rc2;
      if ((rc2 = ensure_big(d, 0, in_bytes + desc_bytes))) return rc2;
      if ((rc2 = ensure_big(d, 1, out_bytes + st_bytes))) return rc2;
      const size_t hneed = std::max<size_t>(in_bytes + desc_bytes, out_bytes + st_bytes);
      if (d.hbig_cap < hneed) {
        if (d.hbig) cudaFreeHost(d.hbig);
        d.hbig = nullptr;
        d.hbig_cap = 0;
        CK(cudaHostAlloc(&d.hbig, hneed, cudaHostAllocPortable));
        d.hbig_cap = hneed;
      }
      char* hb = (char*)d.hbig;
      char* dbi = (char*)d.big[0];
      char* dbo = (char*)d.big[1];
      BatchDesc* hdesc = (BatchDesc*)(hb + in_bytes);
      dcf_status* dst = (dcf_status*)(dbo + out_bytes);
      for (size_t t = 0; t < nj; t++) {
        const dcf_job& j = jobs[per[g][t]];
        memcpy(hb + lo[t], j.lhs, (j.lhs_splat ? 1 : j.n) * ies);
        if (bin) memcpy(hb + ro[t], j.rhs, (j.rhs_splat ? 1 : j.n) * ies);
        hdesc[t] = BatchDesc{dbi + lo[t], bin ? dbi + ro[t] : nullptr, dbo + oo[t], j.n,
                             j.lhs_splat, bin ? j.rhs_splat : 0, dst + t};
      }
      CK(cudaMemcpyAsync(dbi, hb, in_bytes + desc_bytes, cudaMemcpyHostToDevice, s));
      CK(cudaMemsetAsync(dst, 0xFF, nj * sizeof(dcf_status), s));
      EwLaunch a;
      a.op = j0.op;
      a.dtype = j0.dtype;
      a.out_dtype = j0.out_dtype;
      a.flags = j0.flags;
      a.n = maxn;
      a.batch = (const BatchDesc*)(dbi + in_bytes);
      a.n_jobs = (int)nj;
      a.stream = s;
      // Alignment of every pointer in the table is 256 bytes; pass aligned
      // placeholders so the vector path is chosen.
      a.l = dbi;
      a.r = bin ? dbi : nullptr;
      a.o = dbo;
      if (nj > 65535) return set_err(DCF_EINVAL, "at most 65535 jobs per group per GPU");
      rc2 = launch_ew(a);
      if (rc2) return set_err(rc2, "batch launch failed: %s", cudaGetErrorString(cudaGetLastError()));
      CK(cudaMemcpyAsync(hb, dbo, out_bytes + st_bytes, cudaMemcpyDeviceToHost, s));
      CK(cudaEventRecord(d.ev[0], s));
      if ((rc2 = wait_event(d.ev[0]))) return rc2;
      const dcf_status* hst = (const dcf_status*)(hb + out_bytes);
      for (size_t t = 0; t < nj; t++) {
        dcf_job& j = jobs[per[g][t]];
        memcpy(j.out, hb + oo[t], j.n * oes);
        j.result.first_fail_index = hst[t].first_fail;
        j.result.folded = hst[t].first_fail == ~0ull;
        j.result.is_splat = j.result.folded && hst[t].splat_word != 0;
      }
      return DCF_OK;
    };
    if (G == 1) {
      rcs[0] = work(0);
    } else {
      std::vector<std::thread> th;
      for (size_t g = 0; g < G; g++)
        th.emplace_back([&, g] {
          rcs[g] = work(g);
          if (rcs[g]) errs[g] = g_err;
        });
      for (auto& t : th) t.join();
    }
    for (size_t g = 0; g < G; g++)
      if (rcs[g]) {
        if (G > 1) g_err = errs[g];
        return rcs[g];
      }
    gstart = gend;
  }
  return DCF_OK;
}

// ---------------------------------------------------- device entry points

// Make the device that owns `p` current, so a kernel on another GPU's
// tensor launches there.
static int select_device(const void* p) {
  cudaPointerAttributes at;
  if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
    cudaGetLastError();
    return set_err(DCF_EINVAL, "pointer %p is not known to CUDA", p);
  }
  if (at.type != cudaMemoryTypeDevice && at.type != cudaMemoryTypeManaged)
    return set_err(DCF_EINVAL, "pointer %p is not device memory", p);
  CK(cudaSetDevice(at.device));
  return DCF_OK;
}


int dcf_status_reset_async(dcf_status* status, void* stream) {
  if (!status) return set_err(DCF_EINVAL, "null status");
  if (int rc = select_device(status)) return rc;
  CK(cudaMemsetAsync(status, 0xFF, sizeof(dcf_status), (cudaStream_t)stream));
  return DCF_OK;
}

static int async_ew(EwLaunch& a) {
  int rc = select_device(a.o);
  if (rc) return rc;
  rc = launch_ew(a);
  if (rc == DCF_EUNSUPPORTED) return set_err(rc, "op %d on dtype %d -> %d is not supported", a.op, a.dtype, a.out_dtype);
  if (rc) return set_err(rc, "kernel launch failed: %s", cudaGetErrorString(cudaGetLastError()));
  return DCF_OK;
}

int dcf_binary_async(dcf_op op, dcf_dtype dtype, const void* lhs, int lhs_splat, const void* rhs, int rhs_splat,
                     uint64_t n, uint32_t flags, void* out, dcf_status* status, void* stream) {
  int rc = check_binary(op, dtype);
  if (rc) return rc;
  if (n == 0) return DCF_OK;
  if (!lhs || !rhs || !out || !status) return set_err(DCF_EINVAL, "null pointer");
  EwLaunch a;
  a.op = op;
  a.dtype = dtype;
  a.out_dtype = op_bool_result(op) ? DCF_I1 : dtype;
  a.flags = flags;
  a.l = lhs;
  a.r = rhs;
  a.o = out;
  a.n = n;
  a.l0 = lhs;
  a.r0 = rhs;
  a.lsplat = lhs_splat;
  a.rsplat = rhs_splat;
  a.st = status;
  a.stream = (cudaStream_t)stream;
  return async_ew(a);
}

int dcf_convert_async(dcf_op op, dcf_dtype from, dcf_dtype to, const void* in, int in_splat, uint64_t n,
                      uint32_t flags, void* out, dcf_status* status, void* stream) {
  int rc = check_convert(op, from, to);
  if (rc) return rc;
  if (n == 0) return DCF_OK;
  if (!in || !out || !status) return set_err(DCF_EINVAL, "null pointer");
  EwLaunch a;
  a.op = op;
  a.dtype = from;
  a.out_dtype = to;
  a.flags = flags;
  a.l = in;
  a.o = out;
  a.n = n;
  a.l0 = in;
  a.r0 = in;
  a.lsplat = in_splat;
  a.st = status;
  a.stream = (cudaStream_t)stream;
  return async_ew(a);
}

int dcf_reciprocal_async(dcf_dtype dtype, const void* in, int in_splat, uint64_t n, uint32_t flags, void* out,
                         dcf_status* status, void* stream) {
  if (!is_float(dtype)) return set_err(DCF_EINVAL, "reciprocal needs a float dtype");
  if (n == 0) return DCF_OK;
  if (!in || !out || !status) return set_err(DCF_EINVAL, "null pointer");
  EwLaunch a;
  a.op = DCF_RECIPROCAL;
  a.dtype = dtype;
  a.out_dtype = dtype;
  a.flags = flags;
  a.l = in;
  a.o = out;
  a.n = n;
  a.l0 = in;
  a.r0 = in;
  a.lsplat = in_splat;
  a.st = status;
  a.stream = (cudaStream_t)stream;
  return async_ew(a);
}

int dcf_select_async(size_t elem_size, const void* cond, int cond_splat, const void* t, int t_splat, const void* f,
                     int f_splat, uint64_t n, void* out, dcf_status* status, void* stream) {
  if (elem_size != 1 && elem_size != 2 && elem_size != 4 && elem_size != 8)
    return set_err(DCF_EINVAL, "element size %zu not supported", elem_size);
  if (n == 0) return DCF_OK;
  if (!cond || !t || !f || !out || !status) return set_err(DCF_EINVAL, "null pointer");
  int rc = select_device(out);
  if (rc) return rc;
  rc = launch_select(elem_size, cond, cond_splat, t, t_splat, f, f_splat, n, out, status, (cudaStream_t)stream);
  if (rc) return set_err(rc, "select launch failed: %s", cudaGetErrorString(cudaGetLastError()));
  return DCF_OK;
}

int dcf_transpose2d_async(size_t elem_size, uint64_t rows, uint64_t cols, const void* in, void* out, void* stream) {
  if (elem_size != 1 && elem_size != 2 && elem_size != 4 && elem_size != 8)
    return set_err(DCF_EINVAL, "element size %zu not supported", elem_size);
  if (rows == 0 || cols == 0) return DCF_OK;
  int rc = select_device(out);
  if (rc) return rc;
  rc = launch_transpose2d(elem_size, rows, cols, in, out, (cudaStream_t)stream);
  if (rc) return set_err(rc, "transpose launch failed: %s", cudaGetErrorString(cudaGetLastError()));
  return DCF_OK;
}

int dcf_permute_async(size_t elem_size, int rank, const int64_t* in_shape, const int64_t* perms, const void* in,
                      void* out, void* stream) {
  if (elem_size != 1 && elem_size != 2 && elem_size != 4 && elem_size != 8)
    return set_err(DCF_EINVAL, "element size %zu not supported", elem_size);
  if (rank < 1 || rank > 8 || !in_shape || !perms) return set_err(DCF_EINVAL, "bad rank or shape");
  uint64_t total = 1;
  bool seen[8] = {false};
  for (int i = 0; i < rank; i++) {
    if (in_shape[i] < 0) return set_err(DCF_EINVAL, "negative dim");
    if (perms[i] < 0 || perms[i] >= rank || seen[perms[i]]) return set_err(DCF_EINVAL, "perms is not a permutation");
    seen[perms[i]] = true;
    total *= (uint64_t)in_shape[i];
  }
  if (total == 0) return DCF_OK;
  int rc = select_device(out);
  if (rc) return rc;
  rc = launch_permute(elem_size, rank, in_shape, perms, in, out, (cudaStream_t)stream);
  if (rc) return set_err(rc, "permute launch failed: %s", cudaGetErrorString(cudaGetLastError()));
  return DCF_OK;
}

int dcf_permute_status_async(size_t elem_size, int rank, const int64_t* in_shape, const int64_t* perms,
                             const void* in, void* out, dcf_status* status, void* stream) {
  if (!status) return set_err(DCF_EINVAL, "null status");
  if (elem_size != 1 && elem_size != 2 && elem_size != 4 && elem_size != 8)
    return set_err(DCF_EINVAL, "element size %zu not supported", elem_size);
  if (rank < 1 || rank > 8 || !in_shape || !perms) return set_err(DCF_EINVAL, "bad rank or shape");
  uint64_t total = 1;
  bool seen[8] = {false};
  for (int i = 0; i < rank; i++) {
    if (in_shape[i] < 0) return set_err(DCF_EINVAL, "negative dim");
    if (perms[i] < 0 || perms[i] >= rank || seen[perms[i]]) return set_err(DCF_EINVAL, "perms is not a permutation");
    seen[perms[i]] = true;
    total *= (uint64_t)in_shape[i];
  }
  if (total == 0) return DCF_OK;
  int rc = select_device(out);
  if (rc) return rc;
  rc = launch_permute(elem_size, rank, in_shape, perms, in, out, (cudaStream_t)stream, status);
  if (rc) return set_err(rc, "permute launch failed: %s", cudaGetErrorString(cudaGetLastError()));
  return DCF_OK;
}

int dcf_splat_check_async(const void* in, size_t elem_size, uint64_t n, dcf_status* status, void* stream) {
  if (elem_size != 1 && elem_size != 2 && elem_size != 4 && elem_size != 8)
    return set_err(DCF_EINVAL, "element size %zu not supported", elem_size);
  if (!status) return set_err(DCF_EINVAL, "null status");
  if (n <= 1) return DCF_OK;
  int rc = select_device(status);
  if (rc) return rc;
  rc = launch_splat_check(in, elem_size, n, status, (cudaStream_t)stream);
  if (rc) return set_err(rc, "splat launch failed");
  return DCF_OK;
}

int dcf_hex_encode_async(const void* in, uint64_t nbytes, char* out, void* stream) {
  if (nbytes == 0) return DCF_OK;
  int rc = select_device(out);
  if (rc) return rc;
  rc = launch_hex_encode(in, nbytes, out, (cudaStream_t)stream);
  if (rc) return set_err(rc, "hex encode launch failed");
  return DCF_OK;
}

int dcf_hex_decode_async(const char* in, uint64_t nchars, void* out, dcf_status* status, void* stream) {
  if (!status) return set_err(DCF_EINVAL, "null status");
  if (nchars == 0) return DCF_OK;
  int rc = select_device(out);
  if (rc) return rc;
  rc = launch_hex_decode(in, nchars, out, status, (cudaStream_t)stream);
  if (rc == DCF_EPARSE) return set_err(rc, "odd number of hex digits");
  if (rc) return set_err(rc, "hex decode launch failed");
  return DCF_OK;
}

int dcf_hex_decode_many_async(const dcf_hex_piece* pieces, size_t n, uint64_t max_nchars, dcf_status* status,
                              void* stream) {
  if (n == 0) return DCF_OK;
  if (!pieces || !status) return set_err(DCF_EINVAL, "null pointer");
  int rc = select_device(pieces);
  if (rc) return rc;
  rc = launch_hex_decode_pieces(pieces, n, max_nchars, status, (cudaStream_t)stream);
  if (rc) return set_err(rc, "hex decode launch failed: %s", cudaGetErrorString(cudaGetLastError()));
  return DCF_OK;
}

int dcf_hash_many_async(const dcf_hash_piece* pieces, size_t n, uint64_t max_bytes, uint64_t* out, void* stream) {
  if (n == 0) return DCF_OK;
  if (!pieces || !out) return set_err(DCF_EINVAL, "null pointer");
  int rc = select_device(out);
  if (rc) return rc;
  rc = launch_hash_pieces(pieces, n, max_bytes, out, (cudaStream_t)stream);
  if (rc) return set_err(rc, "hash launch failed: %s", cudaGetErrorString(cudaGetLastError()));
  return DCF_OK;
}

int dcf_status_read(const dcf_status* status, void* stream, dcf_result* res) {
  if (!status || !res) return set_err(DCF_EINVAL, "null pointer");
  if (int rc = select_device(status)) return rc;
  dcf_status h;
  CK(cudaMemcpyAsync(&h, status, sizeof h, cudaMemcpyDeviceToHost, (cudaStream_t)stream));
  CK(cudaStreamSynchronize((cudaStream_t)stream));
  memset(res, 0, sizeof *res);
  if (h.error != 0xFFFFFFFFu) return set_err(DCF_ETIMEOUT, "a fold kernel gave up waiting for its own copies");
  res->first_fail_index = h.first_fail;
  res->folded = h.first_fail == ~0ull;
  res->is_splat = res->folded && h.splat_word != 0;
  return DCF_OK;
}

}  // extern "C"
