// dcf_rt.cu — the CUDA runtime calls of the pass driver, made through
// libdcfold.so's own (statically linked) runtime.
//
// libdcfold_opt.so / dcfold-opt link against libdcfold.so and not against a
// CUDA runtime of their own: every runtime call they make goes through the
// wrappers below (mlirpass_b200/opt/cuda_rt.h maps the names), so a process
// running the pass driver has exactly one CUDA runtime instance.  Streams,
// events, device pointers and the per-thread current device and error
// state are therefore all the same runtime's.  Not part of the fold ABI of
// include/dcfold.h.
#include <cuda_runtime.h>

extern "C" {

cudaError_t dcf_rt_cudaEventCreateWithFlags(cudaEvent_t* e, unsigned int flags) {
  return cudaEventCreateWithFlags(e, flags);
}
cudaError_t dcf_rt_cudaEventDestroy(cudaEvent_t e) { return cudaEventDestroy(e); }
cudaError_t dcf_rt_cudaEventRecord(cudaEvent_t e, cudaStream_t s) { return cudaEventRecord(e, s); }
cudaError_t dcf_rt_cudaEventSynchronize(cudaEvent_t e) { return cudaEventSynchronize(e); }
cudaError_t dcf_rt_cudaFree(void* p) { return cudaFree(p); }
cudaError_t dcf_rt_cudaGetDeviceCount(int* n) { return cudaGetDeviceCount(n); }
const char* dcf_rt_cudaGetErrorString(cudaError_t e) { return cudaGetErrorString(e); }
cudaError_t dcf_rt_cudaGetLastError(void) { return cudaGetLastError(); }
cudaError_t dcf_rt_cudaHostAlloc(void** p, size_t n, unsigned int flags) { return cudaHostAlloc(p, n, flags); }
cudaError_t dcf_rt_cudaMalloc(void** p, size_t n) { return cudaMalloc(p, n); }
cudaError_t dcf_rt_cudaMemcpyAsync(void* dst, const void* src, size_t n, cudaMemcpyKind kind, cudaStream_t s) {
  return cudaMemcpyAsync(dst, src, n, kind, s);
}
cudaError_t dcf_rt_cudaMemcpyPeerAsync(void* dst, int dst_dev, const void* src, int src_dev, size_t n,
                                       cudaStream_t s) {
  return cudaMemcpyPeerAsync(dst, dst_dev, src, src_dev, n, s);
}
cudaError_t dcf_rt_cudaMemsetAsync(void* p, int v, size_t n, cudaStream_t s) { return cudaMemsetAsync(p, v, n, s); }
cudaError_t dcf_rt_cudaPointerGetAttributes(cudaPointerAttributes* a, const void* p) {
  return cudaPointerGetAttributes(a, p);
}
cudaError_t dcf_rt_cudaSetDevice(int d) { return cudaSetDevice(d); }
cudaError_t dcf_rt_cudaStreamCreateWithFlags(cudaStream_t* s, unsigned int flags) {
  return cudaStreamCreateWithFlags(s, flags);
}
cudaError_t dcf_rt_cudaStreamDestroy(cudaStream_t s) { return cudaStreamDestroy(s); }
cudaError_t dcf_rt_cudaStreamSynchronize(cudaStream_t s) { return cudaStreamSynchronize(s); }

}  // extern "C"
