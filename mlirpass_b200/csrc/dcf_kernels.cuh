// dcf_kernels.cuh — elementwise fold kernels (templates) and their launch
// plumbing.  One thread moves 16-byte vectors of each operand; the grid is
// a multiple of the SM count and loops over the range.  Every kernel fuses
// three things the reference does in separate passes over the values:
//   - the element closure,
//   - the all-or-nothing refusal test (`collect::<Option<Vec<_>>>()`,
//     src/patterns/arith/canonicalize.rs:215), reduced to the lowest
//     refusing index with one 64-bit atomicMin per warp that saw one,
//   - the splat test of the result (all elements bitwise equal to element
//     0), which decides the `dense<v>` printed form.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "dcf_elem.cuh"
#include "dcf_launch.h"

namespace dcf {

template <int BYTES> struct VecIO;
template <> struct VecIO<1> {
  __device__ static void st(void* p, const void* s) { *(uint8_t*)p = *(const uint8_t*)s; }
};
template <> struct VecIO<2> {
  __device__ static void st(void* p, const void* s) { *(uint16_t*)p = *(const uint16_t*)s; }
};
template <> struct VecIO<4> {
  __device__ static void st(void* p, const void* s) { *(uint32_t*)p = *(const uint32_t*)s; }
};
template <> struct VecIO<8> {
  __device__ static void st(void* p, const void* s) { *(uint2*)p = *(const uint2*)s; }
};
template <int BYTES> struct VecIO {
  static_assert(BYTES % 16 == 0, "vector store size");
  __device__ static void st(void* p, const void* s) {
#pragma unroll
    for (int i = 0; i < BYTES / 16; i++) ((uint4*)p)[i] = ((const uint4*)s)[i];
  }
};

// Warp-aggregated report of the thread's lowest refusing index and of a
// non-splat element.  All threads of the block must call it.
__device__ __forceinline__ void report(dcf_status* st, uint64_t my_fail, bool nonsplat) {
  const unsigned full = 0xFFFFFFFFu;
  const int lane = threadIdx.x & 31;
  if (__any_sync(full, my_fail != ~0ull)) {
    uint64_t v = my_fail;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const uint64_t w = __shfl_xor_sync(full, v, o);
      v = w < v ? w : v;
    }
    if (lane == 0) atomicMin(&st->first_fail, (unsigned long long)v);
  }
  if (__any_sync(full, nonsplat)) {
    if (lane == 0) st->splat_word = 0u;
  }
}

// Binary functor concept:
//   using In, Out;   static constexpr bool kBinary = true;
//   __device__ static bool apply(In a, In b, uint32_t flags, Out& o);
// Unary functor: kBinary = false, apply(In a, uint32_t flags, Out& o).

struct EwParams {
  const void* l;
  const void* r;
  void* o;
  uint64_t n;      // elements in this launch
  const void* l0;  // device pointer to global element 0 of lhs
  const void* r0;  // device pointer to global element 0 of rhs
  uint64_t base;   // global index of this launch's element 0
  uint32_t flags;
  int lsplat;
  int rsplat;
  dcf_status* st;
};

template <class F>
__device__ __forceinline__ bool apply2(const typename F::In& a, const typename F::In& b, uint32_t flags,
                                       typename F::Out& o) {
  if constexpr (F::kBinary) return F::apply(a, b, flags, o);
  else return F::apply(a, flags, o);
}

constexpr int kThreads = 256;
constexpr int kUnroll = 2;

// VECTOR: operand pointers are 16-byte aligned and VEC = 16 / sizeof(In).
template <class F, bool VECTOR>
__global__ void __launch_bounds__(kThreads) ew_kernel(EwParams p) {
  using In = typename F::In;
  using Out = typename F::Out;
  constexpr int VEC = VECTOR ? int(16 / sizeof(In)) : 1;
  const In* __restrict__ l = (const In*)p.l;
  const In* __restrict__ r = (const In*)p.r;
  Out* __restrict__ o = (Out*)p.o;
  const uint32_t flags = p.flags;

  const In a0 = *(const In*)p.l0;
  const In b0 = F::kBinary ? *(const In*)p.r0 : In(0);
  Out o0;
  apply2<F>(a0, b0, flags, o0);

  uint64_t my_fail = ~0ull;
  bool nonsplat = false;
  const uint64_t nvec = p.n / VEC;
  const uint64_t stride = (uint64_t)gridDim.x * kThreads;
  const uint64_t tid = (uint64_t)blockIdx.x * kThreads + threadIdx.x;

  for (uint64_t c0 = tid; c0 < nvec; c0 += stride * kUnroll) {
    In av[kUnroll][VEC], bv[kUnroll][VEC];
#pragma unroll
    for (int u = 0; u < kUnroll; u++) {
      const uint64_t c = c0 + (uint64_t)u * stride;
      if (c < nvec) {
        if (p.lsplat) {
#pragma unroll
          for (int k = 0; k < VEC; k++) av[u][k] = a0;
        } else if constexpr (VECTOR) {
          *(uint4*)av[u] = __ldg((const uint4*)(l + c * VEC));
        } else {
          av[u][0] = l[c];
        }
        if constexpr (F::kBinary) {
          if (p.rsplat) {
#pragma unroll
            for (int k = 0; k < VEC; k++) bv[u][k] = b0;
          } else if constexpr (VECTOR) {
            *(uint4*)bv[u] = __ldg((const uint4*)(r + c * VEC));
          } else {
            bv[u][0] = r[c];
          }
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; u++) {
      const uint64_t c = c0 + (uint64_t)u * stride;
      if (c < nvec) {
        Out ov[VEC];
#pragma unroll
        for (int k = 0; k < VEC; k++) {
          const bool ok = apply2<F>(av[u][k], F::kBinary ? bv[u][k] : In(0), flags, ov[k]);
          if (!ok) {
            const uint64_t idx = p.base + c * VEC + k;
            my_fail = idx < my_fail ? idx : my_fail;
          }
          nonsplat |= (ov[k] != o0);
        }
        VecIO<int(VEC * sizeof(Out))>::st(o + c * VEC, ov);
      }
    }
  }
  // Tail elements that do not fill a vector.
  const uint64_t tail0 = nvec * VEC;
  if (tid < p.n - tail0) {
    const uint64_t i = tail0 + tid;
    const In a = p.lsplat ? a0 : l[i];
    const In b = F::kBinary ? (p.rsplat ? b0 : r[i]) : In(0);
    Out ov;
    if (!apply2<F>(a, b, flags, ov)) {
      const uint64_t idx = p.base + i;
      my_fail = idx < my_fail ? idx : my_fail;
    }
    nonsplat |= (ov != o0);
    o[i] = ov;
  }
  report(p.st, my_fail, nonsplat);
}

// Batched form: blockIdx.y selects the job, blockIdx.x strides its range.
// One launch folds every function's step of the same op and dtype.
template <class F, bool VECTOR>
__global__ void __launch_bounds__(kThreads) ew_batch_kernel(const BatchDesc* __restrict__ jobs, uint32_t flags) {
  using In = typename F::In;
  using Out = typename F::Out;
  constexpr int VEC = VECTOR ? int(16 / sizeof(In)) : 1;
  const BatchDesc& j = jobs[blockIdx.y];
  const In* __restrict__ l = (const In*)j.l;
  const In* __restrict__ r = (const In*)j.r;
  Out* __restrict__ o = (Out*)j.o;
  const In a0 = l[0];
  const In b0 = F::kBinary ? r[0] : In(0);
  Out o0;
  apply2<F>(a0, b0, flags, o0);
  uint64_t my_fail = ~0ull;
  bool nonsplat = false;
  const uint64_t n = j.n;
  const uint64_t nvec = n / VEC;
  const uint64_t stride = (uint64_t)gridDim.x * kThreads;
  const uint64_t tid = (uint64_t)blockIdx.x * kThreads + threadIdx.x;
  for (uint64_t c0 = tid; c0 < nvec; c0 += stride * kUnroll) {
    In av[kUnroll][VEC], bv[kUnroll][VEC];
#pragma unroll
    for (int u = 0; u < kUnroll; u++) {
      const uint64_t c = c0 + (uint64_t)u * stride;
      if (c < nvec) {
        if (j.lsplat) {
#pragma unroll
          for (int k = 0; k < VEC; k++) av[u][k] = a0;
        } else if constexpr (VECTOR) {
          *(uint4*)av[u] = __ldg((const uint4*)(l + c * VEC));
        } else {
          av[u][0] = l[c];
        }
        if constexpr (F::kBinary) {
          if (j.rsplat) {
#pragma unroll
            for (int k = 0; k < VEC; k++) bv[u][k] = b0;
          } else if constexpr (VECTOR) {
            *(uint4*)bv[u] = __ldg((const uint4*)(r + c * VEC));
          } else {
            bv[u][0] = r[c];
          }
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; u++) {
      const uint64_t c = c0 + (uint64_t)u * stride;
      if (c < nvec) {
        Out ov[VEC];
#pragma unroll
        for (int k = 0; k < VEC; k++) {
          if (!apply2<F>(av[u][k], F::kBinary ? bv[u][k] : In(0), flags, ov[k])) {
            const uint64_t idx = c * VEC + k;
            my_fail = idx < my_fail ? idx : my_fail;
          }
          nonsplat |= (ov[k] != o0);
        }
        VecIO<int(VEC * sizeof(Out))>::st(o + c * VEC, ov);
      }
    }
  }
  const uint64_t tail0 = nvec * VEC;
  if (tid < n - tail0) {
    const uint64_t i = tail0 + tid;
    const In a = j.lsplat ? a0 : l[i];
    const In b = F::kBinary ? (j.rsplat ? b0 : r[i]) : In(0);
    Out ov;
    if (!apply2<F>(a, b, flags, ov)) my_fail = i < my_fail ? i : my_fail;
    nonsplat |= (ov != o0);
    o[i] = ov;
  }
  report(j.st, my_fail, nonsplat);
}

int grid_for(uint64_t work_items, const void* kernel);

template <class F>
int launch_one(const EwLaunch& a) {
  EwParams p{a.l, a.r, a.o, a.n, a.l0, a.r0, a.base, a.flags, a.lsplat, a.rsplat, a.st};
  note_launch();
  const uintptr_t mis = (uintptr_t)a.l | (uintptr_t)(F::kBinary ? a.r : nullptr) | (uintptr_t)a.o;
  const bool vec = (mis & 15) == 0;
  if (a.batch) {
    if (vec) {
      const uint64_t per_job = (a.n / (16 / sizeof(typename F::In))) / kUnroll;
      dim3 grid((unsigned)((per_job + kThreads - 1) / kThreads < 1 ? 1 : (per_job + kThreads - 1) / kThreads),
                (unsigned)a.n_jobs);
      ew_batch_kernel<F, true><<<grid, kThreads, 0, a.stream>>>(a.batch, a.flags);
    } else {
      const uint64_t per_job = a.n / kUnroll;
      dim3 grid((unsigned)((per_job + kThreads - 1) / kThreads < 1 ? 1 : (per_job + kThreads - 1) / kThreads),
                (unsigned)a.n_jobs);
      ew_batch_kernel<F, false><<<grid, kThreads, 0, a.stream>>>(a.batch, a.flags);
    }
  } else if (vec) {
    const uint64_t items = a.n / (16 / sizeof(typename F::In));
    ew_kernel<F, true><<<grid_for(items, (const void*)ew_kernel<F, true>), kThreads, 0, a.stream>>>(p);
  } else {
    ew_kernel<F, false><<<grid_for(a.n, (const void*)ew_kernel<F, false>), kThreads, 0, a.stream>>>(p);
  }
  return cudaPeekAtLastError() == cudaSuccess ? DCF_OK : DCF_ECUDA;
}

}  // namespace dcf
