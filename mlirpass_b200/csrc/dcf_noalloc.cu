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
//   - work that overlaps on a GPU and uses the array races on it.  The
//     library therefore holds a per-device lock from the first copy into the
//     array to the synchronisation that ends the call, so calls made from
//     several host threads at once (the pass driver's engines that share a
//     GPU, say) take turns instead of overwriting each other's descriptors;
//   - the first call on each device looks up the array's device address
//     with cudaGetSymbolAddress, with that device current.  Make that first
//     call before any stream capture on that device;
//   - the host-side copies of the descriptors and statuses live in static
//     per-device arrays (guarded by the same lock), not on the caller's
//     stack, so the call needs only a few hundred bytes of stack;
//   - every operand and result pointer must be device memory of one device,
//     and the bytes a job touches must lie inside that pointer's allocation
//     (one cuPointerGetAttributes per allocation and call: ranges inside an
//     allocation already checked in the call need none); anything else is
//     rejected with DCF_EINVAL before any copy or launch;
//   - the caller's current device is the same on return as on entry.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <mutex>

#include "dcf_launch.h"

namespace dcf {

constexpr size_t kNoAllocMaxJobs = 1024;
constexpr size_t kNoAllocDescBytes = kNoAllocMaxJobs * sizeof(BatchDesc);
constexpr size_t kNoAllocBytes = kNoAllocDescBytes + kNoAllocMaxJobs * sizeof(dcf_status);
constexpr int kNoAllocMaxDevices = 64;

// The scratch: descriptors [0, kNoAllocDescBytes), then the job statuses.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

namespace {

// Errors go to the same per-thread text that dcf_last_error() returns.
int noalloc_fail(int code, const char* msg) { return record_error(code, msg); }

// Per device: the lock that serialises calls, the array's device address
// (host code cannot use the symbol's host-side name as a device pointer),
// and the host-side images of the descriptors and statuses.
struct DeviceSlot {
  std::mutex mu;
  unsigned char* scratch = nullptr;
  BatchDesc desc[kNoAllocMaxJobs];
  dcf_status status[kNoAllocMaxJobs];
  uint32_t order[kNoAllocMaxJobs];
};
DeviceSlot g_slots[kNoAllocMaxDevices];

// Called with the slot's lock held and its device current.
int scratch_on(DeviceSlot& slot) {
  if (!slot.scratch) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) {
      char buf[200];
      snprintf(buf, sizeof buf, "cudaGetSymbolAddress(g_noalloc_scratch) failed: %s", cudaGetErrorString(e));
      return noalloc_fail(DCF_ECUDA, buf);
    }
    slot.scratch = (unsigned char*)p;
  }
  return DCF_OK;
}

// cuPointerGetAttributes through the runtime's driver entry point (no link
// against libcuda): memory type, device and allocation range of a pointer
// in one driver call.  Null when the driver does not offer it.
using PointerAttrsFn = CUresult (*)(unsigned, CUpointer_attribute*, void**, CUdeviceptr);
PointerAttrsFn pointer_attrs_fn() {
  static PointerAttrsFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuPointerGetAttributes", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return (PointerAttrsFn)p;
    return (PointerAttrsFn) nullptr;
  }();
  return fn;
}

// Allocations already checked within one call: jobs often point into the
// same allocation (a caching allocator's segment, an upload arena), and a
// range inside one of these needs no driver call.
struct RangeCache {
  static constexpr int kSlots = 8;
  uintptr_t start[kSlots] = {0};
  uint64_t size[kSlots] = {0};
  int dev[kSlots] = {0};
  int next = 0;
  bool find(const void* p, uint64_t bytes, int* d) const {
    const uintptr_t a = (uintptr_t)p;
    for (int k = 0; k < kSlots; k++)
      if (size[k] && a >= start[k] && a - start[k] <= size[k] && bytes <= size[k] - (a - start[k])) {
        *d = dev[k];
        return true;
      }
    return false;
  }
  void add(uintptr_t s, uint64_t n, int d) {
    start[next] = s;
    size[next] = n;
    dev[next] = d;
    next = (next + 1) % kSlots;
  }
};

// Whether [p, p + bytes) is device memory of one device, inside the
// allocation that holds p; that device goes to *dev.
bool device_range(const void* p, uint64_t bytes, int* dev, RangeCache& cache) {
  if (cache.find(p, bytes, dev)) return true;
  if (PointerAttrsFn fn = pointer_attrs_fn()) {
    unsigned mem_type = 0;
    int ordinal = -1;
    CUdeviceptr start = 0;
    size_t size = 0;
    CUpointer_attribute attrs[4] = {CU_POINTER_ATTRIBUTE_MEMORY_TYPE, CU_POINTER_ATTRIBUTE_DEVICE_ORDINAL,
                                    CU_POINTER_ATTRIBUTE_RANGE_START_ADDR, CU_POINTER_ATTRIBUTE_RANGE_SIZE};
    void* data[4] = {&mem_type, &ordinal, &start, &size};
    if (fn(4, attrs, data, (CUdeviceptr)(uintptr_t)p) != CUDA_SUCCESS || mem_type != CU_MEMORYTYPE_DEVICE ||
        ordinal < 0)
      return false;
    *dev = ordinal;
    if (size) {
      const uint64_t off = (uint64_t)((uintptr_t)p - (uintptr_t)start);
      if ((uintptr_t)p < (uintptr_t)start || off > size || bytes > size - off) return false;
      cache.add((uintptr_t)start, size, ordinal);
    }
    return true;
  }
  cudaPointerAttributes at;
  if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  if (at.type != cudaMemoryTypeDevice) return false;
  *dev = at.device;
  return true;
}

// Restores the caller's current device on every return path.
struct DeviceRestore {
  int prev = -1;
  DeviceRestore() {
    if (cudaGetDevice(&prev) != cudaSuccess) {
      cudaGetLastError();
      prev = -1;
    }
  }
  ~DeviceRestore() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

}  // namespace

}  // namespace dcf

using namespace dcf;

extern "C" int dcf_batch_noalloc(dcf_job* jobs, size_t n_jobs, void* stream) {
  if (n_jobs == 0) return DCF_OK;
  if (!jobs) return noalloc_fail(DCF_EINVAL, "null job list");
  if (n_jobs > kNoAllocMaxJobs)
    return noalloc_fail(DCF_EINVAL, "dcf_batch_noalloc takes at most 1024 jobs per call; split the list");
  // The device comes from the first job's result buffer; it is made current
  // before the other checks, so that the driver can report allocation
  // extents.
  int dev = -1;
  for (size_t i = 0; i < n_jobs && dev < 0; i++) {
    if (!jobs[i].n || !jobs[i].out) continue;
    cudaPointerAttributes at;
    if (cudaPointerGetAttributes(&at, jobs[i].out) != cudaSuccess || at.type != cudaMemoryTypeDevice) {
      cudaGetLastError();
      return noalloc_fail(DCF_EINVAL, "dcf_batch_noalloc needs device buffers that hold each job's operands and result");
    }
    dev = at.device;
  }
  if (dev >= kNoAllocMaxDevices) return noalloc_fail(DCF_EINVAL, "device index out of range");
  DeviceRestore restore;
  if (dev >= 0 && cudaSetDevice(dev) != cudaSuccess) return noalloc_fail(DCF_ECUDA, "cudaSetDevice failed");
  // Validate every job before any copy or launch.
  RangeCache checked;
  for (size_t i = 0; i < n_jobs; i++) {
    dcf_job& j = jobs[i];
    memset(&j.result, 0, sizeof j.result);
    j.result.first_fail_index = UINT64_MAX;
    const bool bin = op_binary((int)j.op);
    bool ok;
    if (bin) {
      ok = op_float_binary((int)j.op) ? is_float(j.dtype) : is_int(j.dtype);
      j.out_dtype = op_bool_result((int)j.op) ? DCF_I1 : j.dtype;
    } else if (op_convert((int)j.op)) {
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
    const uint64_t es = dtype_size((int)j.dtype), oes = dtype_size((int)j.out_dtype);
    if (j.n > (UINT64_MAX >> 4)) return noalloc_fail(DCF_EINVAL, "a job's element count is too large");
    int d_out = -1, d_l = -1, d_r = -1;
    if (!device_range(j.out, j.n * oes, &d_out, checked) ||
        !device_range(j.lhs, j.lhs_splat ? es : j.n * es, &d_l, checked) ||
        (bin && !device_range(j.rhs, j.rhs_splat ? es : j.n * es, &d_r, checked)))
      return noalloc_fail(DCF_EINVAL,
                          "dcf_batch_noalloc needs device buffers that hold each job's operands and result");
    if (d_out != dev || d_l != dev || (bin && d_r != dev))
      return noalloc_fail(DCF_EINVAL, "all operands and results of one call must be on one device");
  }
  if (dev < 0) return DCF_OK;
  DeviceSlot& slot = g_slots[dev];
  std::lock_guard<std::mutex> lock(slot.mu);
  if (int rc = scratch_on(slot)) return rc;
  unsigned char* scratch = slot.scratch;
  BatchDesc* ddesc = (BatchDesc*)scratch;
  dcf_status* dst = (dcf_status*)(scratch + kNoAllocDescBytes);
  cudaStream_t s = (cudaStream_t)stream;
  BatchDesc* hdesc = slot.desc;
  dcf_status* hst = slot.status;
  uint32_t* order = slot.order;

  // Descriptors are built in the device's static host image and copied into
  // the scratch array in one transfer; statuses are reset to 0xFF there.
  size_t m = 0;
  for (size_t i = 0; i < n_jobs; i++)
    if (jobs[i].n) order[m++] = (uint32_t)i;
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
      const uint32_t t = order[k];
      order[k] = order[k - 1];
      order[k - 1] = t;
    }
  for (size_t t = 0; t < m; t++) {
    const dcf_job& j = jobs[order[t]];
    const bool bin = op_binary((int)j.op);
    hdesc[t] = BatchDesc{j.lhs, bin ? j.rhs : nullptr, j.out, j.n, j.lhs_splat, bin ? j.rhs_splat : 0, dst + t};
  }
  cudaError_t e = cudaMemcpyAsync(ddesc, hdesc, m * sizeof(BatchDesc), cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) e = cudaMemsetAsync(dst, 0xFF, m * sizeof(dcf_status), s);
  if (e != cudaSuccess) return noalloc_fail(DCF_ECUDA, cudaGetErrorString(e));
  size_t g0 = 0;
  int rc = DCF_OK;
  while (g0 < m && rc == DCF_OK) {
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
    a.r = op_binary((int)j0.op) ? a.l : nullptr;
    a.o = (void*)a.l;
    if (launch_ew(a) != DCF_OK) rc = noalloc_fail(DCF_ECUDA, cudaGetErrorString(cudaGetLastError()));
    g0 = g1;
  }
  // Read the statuses back and wait, also after a failed launch, so that no
  // work of this call is still using the array when the lock is released.
  e = cudaMemcpyAsync(hst, dst, m * sizeof(dcf_status), cudaMemcpyDeviceToHost, s);
  const cudaError_t es = cudaStreamSynchronize(s);
  if (e == cudaSuccess) e = es;
  if (rc != DCF_OK) return rc;
  if (e != cudaSuccess) return noalloc_fail(DCF_ECUDA, cudaGetErrorString(e));
  for (size_t t = 0; t < m; t++) {
    dcf_job& j = jobs[order[t]];
    j.result.first_fail_index = hst[t].first_fail;
    j.result.folded = hst[t].first_fail == ~0ull;
    j.result.is_splat = j.result.folded && hst[t].splat_word != 0;
  }
  return DCF_OK;
}
