// cuda_rt.h — the CUDA runtime as the pass driver sees it: the runtime's
// types from <cuda_runtime.h>, and every call routed to libdcfold.so's
// runtime (csrc/dcf_rt.cu), so that the driver process holds one CUDA
// runtime instance.  Include this instead of <cuda_runtime.h>.
#pragma once

#include <cuda_runtime.h>

extern "C" {
cudaError_t dcf_rt_cudaEventCreateWithFlags(cudaEvent_t* e, unsigned int flags);
cudaError_t dcf_rt_cudaEventDestroy(cudaEvent_t e);
cudaError_t dcf_rt_cudaEventRecord(cudaEvent_t e, cudaStream_t s);
cudaError_t dcf_rt_cudaEventSynchronize(cudaEvent_t e);
cudaError_t dcf_rt_cudaFree(void* p);
cudaError_t dcf_rt_cudaGetDeviceCount(int* n);
const char* dcf_rt_cudaGetErrorString(cudaError_t e);
cudaError_t dcf_rt_cudaGetLastError(void);
cudaError_t dcf_rt_cudaHostAlloc(void** p, size_t n, unsigned int flags);
cudaError_t dcf_rt_cudaMalloc(void** p, size_t n);
cudaError_t dcf_rt_cudaMemcpyAsync(void* dst, const void* src, size_t n, cudaMemcpyKind kind, cudaStream_t s);
cudaError_t dcf_rt_cudaMemcpyPeerAsync(void* dst, int dst_dev, const void* src, int src_dev, size_t n,
                                       cudaStream_t s);
cudaError_t dcf_rt_cudaMemsetAsync(void* p, int v, size_t n, cudaStream_t s);
cudaError_t dcf_rt_cudaPointerGetAttributes(cudaPointerAttributes* a, const void* p);
cudaError_t dcf_rt_cudaSetDevice(int d);
cudaError_t dcf_rt_cudaStreamCreateWithFlags(cudaStream_t* s, unsigned int flags);
cudaError_t dcf_rt_cudaStreamDestroy(cudaStream_t s);
cudaError_t dcf_rt_cudaStreamSynchronize(cudaStream_t s);
}

#define cudaEventCreateWithFlags dcf_rt_cudaEventCreateWithFlags
#define cudaEventDestroy dcf_rt_cudaEventDestroy
#define cudaEventRecord dcf_rt_cudaEventRecord
#define cudaEventSynchronize dcf_rt_cudaEventSynchronize
#define cudaFree dcf_rt_cudaFree
#define cudaGetDeviceCount dcf_rt_cudaGetDeviceCount
#define cudaGetErrorString dcf_rt_cudaGetErrorString
#define cudaGetLastError dcf_rt_cudaGetLastError
#define cudaHostAlloc dcf_rt_cudaHostAlloc
#define cudaMalloc dcf_rt_cudaMalloc
#define cudaMemcpyAsync dcf_rt_cudaMemcpyAsync
#define cudaMemcpyPeerAsync dcf_rt_cudaMemcpyPeerAsync
#define cudaMemsetAsync dcf_rt_cudaMemsetAsync
#define cudaPointerGetAttributes dcf_rt_cudaPointerGetAttributes
#define cudaSetDevice dcf_rt_cudaSetDevice
#define cudaStreamCreateWithFlags dcf_rt_cudaStreamCreateWithFlags
#define cudaStreamDestroy dcf_rt_cudaStreamDestroy
#define cudaStreamSynchronize dcf_rt_cudaStreamSynchronize
