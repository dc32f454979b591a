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

#include <type_traits>
#include <utility>

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

// Programmatic dependent launch: the fold kernels are launched so that the
// next kernel in the stream may start while this one drains (its CTAs take
// the SM slots this grid's CTAs leave).  Each fold kernel first waits until
// the grid before it has completed and its writes are visible
// (griddepcontrol.wait; a no-op when nothing before it was launched this
// way), then at once allows its own dependents to launch.  Every read of
// an operand, an element 0 or a status comes after the wait, so the
// ordering the stream promises is unchanged; what overlaps is launch
// latency and CTA start-up.
__device__ __forceinline__ void pdl_begin() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
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
constexpr int kUnroll = 4;

template <class F, int VEC>
__device__ __forceinline__ void load_chunk(const typename F::In* __restrict__ l, const typename F::In* __restrict__ r,
                                           uint64_t c, bool lsplat, bool rsplat, typename F::In a0,
                                           typename F::In b0, typename F::In (&av)[VEC], typename F::In (&bv)[VEC]) {
  using In = typename F::In;
  if (lsplat) {
#pragma unroll
    for (int k = 0; k < VEC; k++) av[k] = a0;
  } else if constexpr (VEC * sizeof(In) == 16) {
    *(uint4*)av = __ldg((const uint4*)(l + c * VEC));
  } else {
    av[0] = l[c];
  }
  if constexpr (F::kBinary) {
    if (rsplat) {
#pragma unroll
      for (int k = 0; k < VEC; k++) bv[k] = b0;
    } else if constexpr (VEC * sizeof(In) == 16) {
      *(uint4*)bv = __ldg((const uint4*)(r + c * VEC));
    } else {
      bv[0] = r[c];
    }
  }
}

// Functors whose op never refuses and works lane-wise on 8- or 16-bit
// elements may define `kWord` and `word(a, b)`: the op on four (or two)
// elements packed in one 32-bit word (SIMD-within-a-register), so a
// 16-byte chunk of i8 costs four operations instead of sixteen.
template <class F, class = void> struct HasWord : std::false_type {};
template <class F> struct HasWord<F, std::void_t<decltype(F::kWord)>> : std::bool_constant<F::kWord> {};

// Functors whose op may refuse can define `kWordChecked` and
// `word_checked(a, b, o)`: the op on the packed lanes of one word, returning
// a mask with every bit of each refusing lane set (0: none refuses).  The
// lowest refusing lane gives the element index; no element path is taken,
// so a warp with a refusing lane does not diverge.
template <class F, class = void> struct HasCheckedWord : std::false_type {};
template <class F>
struct HasCheckedWord<F, std::void_t<decltype(F::kWordChecked)>> : std::bool_constant<F::kWordChecked> {};

template <class T> __device__ __forceinline__ uint32_t replicate32(T v) {
  if constexpr (sizeof(T) == 1) return (uint32_t)(uint8_t)v * 0x01010101u;
  else return (uint32_t)(uint16_t)v * 0x00010001u;
}

template <class F, int VEC>
__device__ __forceinline__ void fold_chunk(typename F::Out* __restrict__ o, uint64_t c, uint64_t base,
                                           uint32_t flags, const typename F::In (&av)[VEC],
                                           const typename F::In (&bv)[VEC], typename F::Out o0,
                                           uint64_t& my_fail, bool& nonsplat) {
  using In = typename F::In;
  using Out = typename F::Out;
  if constexpr (HasWord<F>::value && VEC * sizeof(In) == 16 && sizeof(Out) == sizeof(In)) {
    const uint32_t* aw = (const uint32_t*)av;
    const uint32_t* bw = (const uint32_t*)bv;
    const uint32_t o0w = replicate32(o0);
    uint4 r;
    uint32_t* rw = (uint32_t*)&r;
#pragma unroll
    for (int k = 0; k < 4; k++) {
      rw[k] = F::word(aw[k], bw[k]);
      nonsplat |= rw[k] != o0w;
    }
    *(uint4*)(o + c * VEC) = r;
    return;
  }
  if constexpr (HasCheckedWord<F>::value && VEC * sizeof(In) == 16 && sizeof(Out) == sizeof(In)) {
    const uint32_t* aw = (const uint32_t*)av;
    const uint32_t* bw = (const uint32_t*)bv;
    uint4 r;
    uint32_t* rw = (uint32_t*)&r;
    const uint32_t o0w = replicate32(o0);
    constexpr int kLanes = int(4 / sizeof(In));
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const uint32_t m = F::word_checked(aw[k], bw[k], rw[k]);
      if (m) {
        const uint64_t idx = base + c * VEC + k * kLanes + (__ffs((int)m) - 1) / (8 * int(sizeof(In)));
        my_fail = idx < my_fail ? idx : my_fail;
      }
      nonsplat |= rw[k] != o0w;
    }
    *(uint4*)(o + c * VEC) = r;
    return;
  }
  Out ov[VEC];
#pragma unroll
  for (int k = 0; k < VEC; k++) {
    if (!apply2<F>(av[k], F::kBinary ? bv[k] : In(0), flags, ov[k])) {
      const uint64_t idx = base + c * VEC + k;
      my_fail = idx < my_fail ? idx : my_fail;
    }
    nonsplat |= (ov[k] != o0);
  }
  VecIO<int(VEC * sizeof(Out))>::st(o + c * VEC, ov);
}

// VECTOR: operand pointers are 16-byte aligned and VEC = 16 / sizeof(In).
// The main loop issues kUnroll 16-byte loads per operand per thread before
// any arithmetic, with no bounds tests; a final pass handles the ragged end.
template <class F, bool VECTOR>
__global__ void __launch_bounds__(kThreads) ew_kernel(EwParams p) {
  using In = typename F::In;
  using Out = typename F::Out;
  constexpr int VEC = VECTOR ? int(16 / sizeof(In)) : 1;
  pdl_begin();
  const In* __restrict__ l = (const In*)p.l;
  const In* __restrict__ r = (const In*)p.r;
  Out* __restrict__ o = (Out*)p.o;
  const uint32_t flags = p.flags;
  const bool lsplat = p.lsplat != 0, rsplat = p.rsplat != 0;

  const In a0 = *(const In*)p.l0;
  const In b0 = F::kBinary ? *(const In*)p.r0 : In(0);
  Out o0;
  apply2<F>(a0, b0, flags, o0);

  uint64_t my_fail = ~0ull;
  bool nonsplat = false;
  const uint64_t nvec = p.n / VEC;
  const uint64_t stride = (uint64_t)gridDim.x * kThreads;
  const uint64_t tid = (uint64_t)blockIdx.x * kThreads + threadIdx.x;

  uint64_t c0 = tid;
  for (; c0 + (kUnroll - 1) * stride < nvec; c0 += kUnroll * stride) {
    In av[kUnroll][VEC], bv[kUnroll][VEC];
#pragma unroll
    for (int u = 0; u < kUnroll; u++) load_chunk<F, VEC>(l, r, c0 + u * stride, lsplat, rsplat, a0, b0, av[u], bv[u]);
#pragma unroll
    for (int u = 0; u < kUnroll; u++) fold_chunk<F, VEC>(o, c0 + u * stride, p.base, flags, av[u], bv[u], o0, my_fail, nonsplat);
  }
  for (; c0 < nvec; c0 += stride) {
    In av[VEC], bv[VEC];
    load_chunk<F, VEC>(l, r, c0, lsplat, rsplat, a0, b0, av, bv);
    fold_chunk<F, VEC>(o, c0, p.base, flags, av, bv, o0, my_fail, nonsplat);
  }
  // Tail elements that do not fill a vector.
  const uint64_t tail0 = nvec * VEC;
  if (tid < p.n - tail0) {
    const uint64_t i = tail0 + tid;
    const In a = lsplat ? a0 : l[i];
    const In b = F::kBinary ? (rsplat ? b0 : r[i]) : In(0);
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

// ----------------------------------------------------------------------
// Bulk-copy (TMA) pipeline for large aligned folds.  Persistent CTAs; each
// stage holds one 16 KB tile of every streamed operand, filled by one
// cp.async.bulk per operand that completes on the stage's mbarrier.  All
// 256 threads consume the stage from shared memory and store results
// straight from registers; thread 0 refills the stage once every thread has
// read it.  Waits are bounded: a CTA that waits too long records the fact
// in the status's error word, drains its copies (again bounded) and exits.
constexpr int kTileBytes = 16384;
constexpr int kStages = 2;
constexpr int kTmaCtasPerSm = 3;
constexpr long kWaitLimit = 1l << 24;

__device__ __forceinline__ uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, unsigned parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for phase `parity` of `bar`; false when the bound ran out.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, unsigned parity) {
  for (long spins = 0; !mbar_try_wait(bar, parity); spins++)
    if (spins > kWaitLimit) return false;
  return true;
}

__device__ __forceinline__ void bulk_load(void* dst, const void* src, unsigned bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(smem_addr(dst)), "l"(src), "r"(bytes), "r"(smem_addr(bar))
               : "memory");
}

template <class F>
__global__ void __launch_bounds__(kThreads) ew_tma_kernel(EwParams p) {
  using In = typename F::In;
  using Out = typename F::Out;
  pdl_begin();
  constexpr int VEC = int(16 / sizeof(In));
  constexpr int TE = kTileBytes / int(sizeof(In));   // elements per tile
  constexpr int TV = TE / VEC;                       // 16-byte chunks per tile
  extern __shared__ __align__(128) uint8_t smem[];
  const bool lsplat = p.lsplat != 0, rsplat = p.rsplat != 0;
  const bool lcopy = !lsplat, rcopy = F::kBinary && !rsplat;
  In* sl = (In*)smem;
  In* sr = (In*)(smem + (lcopy ? kStages * kTileBytes : 0));
  uint64_t* full = (uint64_t*)(smem + kStages * kTileBytes * ((lcopy ? 1 : 0) + (rcopy ? 1 : 0)));
  const unsigned tx = (lcopy ? kTileBytes : 0) + (rcopy ? kTileBytes : 0);
  const In* __restrict__ l = (const In*)p.l;
  const In* __restrict__ r = (const In*)p.r;
  Out* __restrict__ o = (Out*)p.o;
  const uint32_t flags = p.flags;
  const uint64_t ntiles = p.n / TE;

  const In a0 = *(const In*)p.l0;
  const In b0 = F::kBinary ? *(const In*)p.r0 : In(0);
  Out o0;
  apply2<F>(a0, b0, flags, o0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; s++) mbar_init(&full[s], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    for (int s = 0; s < kStages; s++) {
      const uint64_t t = blockIdx.x + (uint64_t)s * gridDim.x;
      if (t < ntiles) {
        mbar_expect_tx(&full[s], tx);
        if (lcopy) bulk_load(sl + s * TE, l + t * TE, kTileBytes, &full[s]);
        if (rcopy) bulk_load(sr + s * TE, r + t * TE, kTileBytes, &full[s]);
      }
    }
  }
  __syncthreads();

  uint64_t my_fail = ~0ull;
  bool nonsplat = false;
  uint64_t i = 0;
  bool dead = false;
  for (uint64_t t = blockIdx.x; t < ntiles; t += gridDim.x, i++) {
    const int s = (int)(i % kStages);
    const bool ok = mbar_wait_bounded(&full[s], (unsigned)((i / kStages) & 1));
    if (__syncthreads_or(!ok)) {
      dead = true;
      break;
    }
#pragma unroll
    for (int k = threadIdx.x; k < TV; k += kThreads) {
      In av[VEC], bv[VEC];
      if (lsplat) {
#pragma unroll
        for (int e = 0; e < VEC; e++) av[e] = a0;
      } else {
        *(uint4*)av = *(const uint4*)(sl + s * TE + k * VEC);
      }
      if constexpr (F::kBinary) {
        if (rsplat) {
#pragma unroll
          for (int e = 0; e < VEC; e++) bv[e] = b0;
        } else {
          *(uint4*)bv = *(const uint4*)(sr + s * TE + k * VEC);
        }
      }
      fold_chunk<F, VEC>(o, t * TV + k, p.base, flags, av, bv, o0, my_fail, nonsplat);
    }
    __syncthreads();  // every thread has read stage s
    if (threadIdx.x == 0) {
      const uint64_t tn = t + (uint64_t)kStages * gridDim.x;
      if (tn < ntiles) {
        mbar_expect_tx(&full[s], tx);
        if (lcopy) bulk_load(sl + s * TE, l + tn * TE, kTileBytes, &full[s]);
        if (rcopy) bulk_load(sr + s * TE, r + tn * TE, kTileBytes, &full[s]);
      }
    }
  }
  if (dead) {
    // Drain the fills still in flight (bounded) before the CTA exits.
    for (uint64_t j = i; j < i + kStages; j++) {
      if (blockIdx.x + j * gridDim.x >= ntiles) break;
      mbar_wait_bounded(&full[j % kStages], (unsigned)((j / kStages) & 1));
    }
    if (threadIdx.x == 0) atomicExch(&p.st->error, 1u);
    return;
  }
  // Elements past the last whole tile: plain loads, all CTAs.
  const uint64_t stride = (uint64_t)gridDim.x * kThreads;
  for (uint64_t k = ntiles * TE + (uint64_t)blockIdx.x * kThreads + threadIdx.x; k < p.n; k += stride) {
    const In a = lsplat ? a0 : l[k];
    const In b = F::kBinary ? (rsplat ? b0 : r[k]) : In(0);
    Out ov;
    if (!apply2<F>(a, b, flags, ov)) {
      const uint64_t idx = p.base + k;
      my_fail = idx < my_fail ? idx : my_fail;
    }
    nonsplat |= (ov != o0);
    o[k] = ov;
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
  pdl_begin();
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
int sm_count_current();
int tma_min_tiles_per_sm();
bool prepare_smem(const void* kernel, int bytes);
// CTAs of `kernel` (kThreads threads, `smem` bytes of dynamic shared
// memory) that can be resident on one SM at once, capped at `cap`.
int resident_per_sm(const void* kernel, int smem, int cap);
// Whether fold kernels are launched as programmatic dependents (default
// yes; DCF_PDL=0 turns it off).
bool pdl_enabled();

template <typename... Params, typename... Args>
void launch_fold(void (*kernel)(Params...), dim3 grid, int smem, cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

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
      launch_fold(ew_batch_kernel<F, true>, grid, 0, a.stream, a.batch, a.flags);
    } else {
      const uint64_t per_job = a.n / kUnroll;
      dim3 grid((unsigned)((per_job + kThreads - 1) / kThreads < 1 ? 1 : (per_job + kThreads - 1) / kThreads),
                (unsigned)a.n_jobs);
      launch_fold(ew_batch_kernel<F, false>, grid, 0, a.stream, a.batch, a.flags);
    }
    return cudaPeekAtLastError() == cudaSuccess ? DCF_OK : DCF_ECUDA;
  }
  const int streamed = (a.lsplat ? 0 : 1) + (F::kBinary && !a.rsplat ? 1 : 0);
  const uint64_t ntiles = a.n / (kTileBytes / sizeof(typename F::In));
  const int sms = sm_count_current();
  if (vec && streamed > 0 && ntiles >= (uint64_t)sms * tma_min_tiles_per_sm()) {
    const int smem = kStages * kTileBytes * streamed + kStages * 8;
    if (!prepare_smem((const void*)ew_tma_kernel<F>, smem)) return DCF_ECUDA;
    // One wave of persistent CTAs: as many per SM as fit (at most three).
    const int per_sm = resident_per_sm((const void*)ew_tma_kernel<F>, smem, kTmaCtasPerSm);
    const uint64_t cap = (uint64_t)sms * (uint64_t)per_sm;
    const uint64_t g = ntiles < cap ? ntiles : cap;
    launch_fold(ew_tma_kernel<F>, dim3((unsigned)g), smem, a.stream, p);
  } else if (vec) {
    const uint64_t items = a.n / (16 / sizeof(typename F::In));
    launch_fold(ew_kernel<F, true>, dim3(grid_for(items, (const void*)ew_kernel<F, true>)), 0, a.stream, p);
  } else {
    launch_fold(ew_kernel<F, false>, dim3(grid_for(a.n, (const void*)ew_kernel<F, false>)), 0, a.stream, p);
  }
  return cudaPeekAtLastError() == cudaSuccess ? DCF_OK : DCF_ECUDA;
}

}  // namespace dcf
