// dcf_noalloc.cu — dcf_batch_noalloc: the batched fold on caller-owned
// device buffers, with every byte of scratch memory in a fixed array that
// the library declares at file scope, so the call allocates nothing.
//
// Who needs it: a caller that cannot, or must not, allocate device memory
// at fold time.  Typical cases are an embedding runtime whose caching
// allocator has already reserved all of HBM (a cudaMalloc then fails or
// fragments its arena), and latency-sensitive code that cannot accept the
// device-wide synchronisation that cudaMalloc / cudaFree may imply.  The
// other entry points allocate their staging and status buffers on first
// use; this one only copies into, and launches over, the static array.
//
// Limits and sharing:
//   - at most kNoAllocMaxJobs jobs per call (the array holds one descriptor
//     and one status per job); larger calls are rejected with DCF_EINVAL;
//   - every call shares the one array per device and leaves its contents
//     behind; each call re-initialises what it uses (descriptors written,
//     statuses filled with 0xFF) before its kernels read them;
//   - calls whose work overlaps on a GPU (two host threads, or two streams,
//     at once) race on the array: serialise them;
//   - the first call on each device looks up the array's device address
//     with cudaGetSymbolAddress, with that device current.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <mutex>

#include "dcf_launch.h"

namespace dcf {

constexpr size_t kNoAllocMaxJobs = 1024;
constexpr size_t kNoAllocDescBytes = kNoAllocMaxJobs * sizeof(BatchDesc);
constexpr size_t kNoAllocBytes = kNoAllocDescBytes + kNoAllocMaxJobs * sizeof(dcf_status);

// The scratch: descriptors [0, kNoAllocDescBytes), then the job statuses.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

namespace {

// Errors go to the same per-thread text that dcf_last_error() returns.
int noalloc_fail(int code, const char* msg) { return record_error(code, msg); }

// Device address of g_noalloc_scratch on each device (host code cannot use
// the symbol's host-side name as a device pointer).
std::mutex g_sym_mu;
void* g_sym_addr[64] = {nullptr};

int scratch_on(int dev, unsigned char** out) {
  if (dev < 0 || dev >= 64) return noalloc_fail(DCF_EINVAL, "device index out of range");
  std::lock_guard<std::mutex> g(g_sym_mu);
  if (!g_sym_addr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) {
      char buf[200];
      snprintf(buf, sizeof buf, "cudaGetSymbolAddress(g_noalloc_scratch) failed: %s", cudaGetErrorString(e));
      return noalloc_fail(DCF_ECUDA, buf);
    }
    g_sym_addr[dev] = p;
  }
  *out = (unsigned char*)g_sym_addr[dev];
  return DCF_OK;
}

bool binary_op(uint32_t op) { return op_binary((int)op); }

bool convert_op(uint32_t op) { return op_convert((int)op); }

}  // namespace

}  // namespace dcf

using namespace dcf;

extern "C" int dcf_batch_noalloc(dcf_job* jobs, size_t n_jobs, void* stream) {
  if (n_jobs == 0) return DCF_OK;
  if (!jobs) return noalloc_fail(DCF_EINVAL, "null job list");
  if (n_jobs > kNoAllocMaxJobs)
    return noalloc_fail(DCF_EINVAL, "dcf_batch_noalloc takes at most 1024 jobs per call; split the list");
  // Validate every job before touching the device.
  int dev = -1;
  for (size_t i = 0; i < n_jobs; i++) {
    dcf_job& j = jobs[i];
    memset(&j.result, 0, sizeof j.result);
    j.result.first_fail_index = UINT64_MAX;
    const bool bin = binary_op(j.op);
    bool ok;
    if (bin) {
      ok = op_float_binary((int)j.op) ? is_float(j.dtype) : is_int(j.dtype);
      j.out_dtype = op_bool_result((int)j.op) ? DCF_I1 : j.dtype;
    } else if (convert_op(j.op)) {
      ok = convert_types_ok((int)j.op, is_float(j.dtype), is_int(j.dtype), is_float(j.out_dtype), is_int(j.out_dtype),
                            (int)j.dtype, (int)j.out_dtype);
    } else if (j.op == DCF_RECIPROCAL) {
      ok = is_float(j.dtype);
      j.out_dtype = j.dtype;
    } else {
      ok = false;
    }
    if (!ok) return noalloc_fail(DCF_EINVAL, "a job has an unsupported op / dtype combination");
    if (j.n == 0) {
      j.result.folded = 1;
      j.result.is_splat = 1;
      continue;
    }
    if (!j.lhs || !j.out || (bin && !j.rhs)) return noalloc_fail(DCF_EINVAL, "a job has a null buffer");
    cudaPointerAttributes at;
    if (cudaPointerGetAttributes(&at, j.out) != cudaSuccess || at.type != cudaMemoryTypeDevice) {
      cudaGetLastError();
      return noalloc_fail(DCF_EINVAL, "dcf_batch_noalloc needs device buffers");
    }
    if (dev < 0) dev = at.device;
    else if (dev != at.device) return noalloc_fail(DCF_EINVAL, "all jobs of one call must be on one device");
  }
  if (dev < 0) return DCF_OK;
  if (cudaSetDevice(dev) != cudaSuccess) return noalloc_fail(DCF_ECUDA, "cudaSetDevice failed");
  unsigned char* scratch = nullptr;
  if (int rc = scratch_on(dev, &scratch)) return rc;
  BatchDesc* ddesc = (BatchDesc*)scratch;
  dcf_status* dst = (dcf_status*)(scratch + kNoAllocDescBytes);
  cudaStream_t s = (cudaStream_t)stream;

  // Descriptors are built on the stack (no heap either) and copied into the
  // scratch array in one transfer; statuses are reset to 0xFF there.
  BatchDesc hdesc[kNoAllocMaxJobs];
  dcf_status hst[kNoAllocMaxJobs];
  size_t order[kNoAllocMaxJobs];
  size_t m = 0;
  for (size_t i = 0; i < n_jobs; i++)
    if (jobs[i].n) order[m++] = i;
  // Group jobs of one (op, dtype, out_dtype, flags) next to each other:
  // insertion sort keeps this allocation-free.
  auto key_less = [&](size_t a, size_t b) {
    const dcf_job &x = jobs[a], &y = jobs[b];
    if (x.op != y.op) return x.op < y.op;
    if (x.dtype != y.dtype) return x.dtype < y.dtype;
    if (x.out_dtype != y.out_dtype) return x.out_dtype < y.out_dtype;
    return x.flags < y.flags;
  };
  for (size_t i = 1; i < m; i++)
    for (size_t k = i; k > 0 && key_less(order[k], order[k - 1]); k--) {
      const size_t t = order[k];
      order[k] = order[k - 1];
      order[k - 1] = t;
    }
  for (size_t t = 0; t < m; t++) {
    const dcf_job& j = jobs[order[t]];
    const bool bin = binary_op(j.op);
    hdesc[t] = BatchDesc{j.lhs, bin ? j.rhs : nullptr, j.out, j.n, j.lhs_splat, bin ? j.rhs_splat : 0, dst + t};
  }
  cudaError_t e = cudaMemcpyAsync(ddesc, hdesc, m * sizeof(BatchDesc), cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) e = cudaMemsetAsync(dst, 0xFF, m * sizeof(dcf_status), s);
  if (e != cudaSuccess) return noalloc_fail(DCF_ECUDA, cudaGetErrorString(e));
  size_t g0 = 0;
  while (g0 < m) {
    size_t g1 = g0 + 1;
    while (g1 < m && !key_less(order[g0], order[g1]) && !key_less(order[g1], order[g0])) g1++;
    const dcf_job& j0 = jobs[order[g0]];
    uint64_t maxn = 0;
    for (size_t t = g0; t < g1; t++) maxn = jobs[order[t]].n > maxn ? jobs[order[t]].n : maxn;
    bool aligned = true;
    for (size_t t = g0; t < g1; t++)
      aligned = aligned && (((uintptr_t)hdesc[t].l | (uintptr_t)hdesc[t].r | (uintptr_t)hdesc[t].o) & 15) == 0;
    EwLaunch a;
    a.op = (int)j0.op;
    a.dtype = (int)j0.dtype;
    a.out_dtype = (int)j0.out_dtype;
    a.flags = j0.flags;
    a.n = maxn;
    a.batch = ddesc + g0;
    a.n_jobs = (int)(g1 - g0);
    a.stream = s;
    // The launcher picks the vector kernel from these pointers' alignment.
    a.l = aligned ? (const void*)scratch : (const void*)(scratch + 1);
    a.r = binary_op(j0.op) ? a.l : nullptr;
    a.o = (void*)a.l;
    if (launch_ew(a) != DCF_OK) return noalloc_fail(DCF_ECUDA, cudaGetErrorString(cudaGetLastError()));
    g0 = g1;
  }
  e = cudaMemcpyAsync(hst, dst, m * sizeof(dcf_status), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return noalloc_fail(DCF_ECUDA, cudaGetErrorString(e));
  for (size_t t = 0; t < m; t++) {
    dcf_job& j = jobs[order[t]];
    j.result.first_fail_index = hst[t].first_fail;
    j.result.folded = hst[t].first_fail == ~0ull;
    j.result.is_splat = j.result.folded && hst[t].splat_word != 0;
  }
  return DCF_OK;
}
