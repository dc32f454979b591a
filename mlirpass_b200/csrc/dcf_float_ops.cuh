// dcf_float_ops.cuh — functors of the float folds (addf, subf, mulf, divf,
// remf, the four min/max ops, dense cmpf, copysign, tosa reciprocal) and their
// per-layout dispatch.  Each float layout is instantiated in its own
// translation unit (dcf_ew_float_*.cu) so the library builds in parallel.
#pragma once

#include "dcf_kernels.cuh"

namespace dcf {

template <int OP, class L, bool NEAREST> struct FArith {
  using In = typename L::T;
  using Out = typename L::T;
  static constexpr bool kBinary = true;
  __device__ static __forceinline__ bool apply(In a, In b, uint32_t flags, Out& o) {
    if constexpr (NEAREST) {
      o = (Out)arith_rn<OP, L>(a, b, default_nan<L>(flags));
      return true;
    } else {
      uint64_t r = 0;
      const bool ok = rounded<OP, L>(a, b, (int)(flags & DCF_FLAG_ROUND_MASK), default_nan<L>(flags), r);
      o = (Out)r;
      return ok;
    }
  }
};

template <class L, bool MAX, bool NW> struct FMinMax {
  using In = typename L::T;
  using Out = typename L::T;
  static constexpr bool kBinary = true;
  __device__ static __forceinline__ bool apply(In a, In b, uint32_t, Out& o) {
    o = (Out)minmax<L, MAX, NW>(a, b);
    return true;
  }
};

template <class L> struct FCmp {
  using In = typename L::T;
  using Out = uint8_t;
  static constexpr bool kBinary = true;
  __device__ static __forceinline__ bool apply(In a, In b, uint32_t flags, Out& o) {
    o = cmpf<L>((int)((flags & DCF_FLAG_PRED_MASK) >> DCF_FLAG_PRED_SHIFT), a, b);
    return true;
  }
};

template <class L> struct FRem {
  using In = typename L::T;
  using Out = typename L::T;
  static constexpr bool kBinary = true;
  __device__ static __forceinline__ bool apply(In a, In b, uint32_t flags, Out& o) {
    o = (Out)remf<L>(a, b, default_nan<L>(flags));
    return true;
  }
};

// tosa reciprocal: `one.div(f)` at nearest-even.
template <class L> struct FRecip {
  using In = typename L::T;
  using Out = typename L::T;
  static constexpr bool kBinary = false;
  __device__ static __forceinline__ bool apply(In a, uint32_t flags, Out& o) {
    uint64_t one;
    if constexpr (L::B == 8) one = 0x3FF0000000000000ull;
    else one = ((uint64_t)((1 << (L::E - 1)) - 1)) << L::M;
    o = (Out)arith_rn<DCF_DIVF, L>(one, a, default_nan<L>(flags));
    return true;
  }
};

// math.copysign (src/patterns/math/canonicalize.rs:153-156): lhs negated
// when the signs differ, i.e. lhs with rhs's sign bit.
template <class L> struct FCopySign {
  using In = typename L::T;
  using Out = typename L::T;
  static constexpr bool kBinary = true;
  __device__ static __forceinline__ bool apply(In a, In b, uint32_t, Out& o) {
    o = (Out)(((uint64_t)a & ~L::SIGN) | ((uint64_t)b & L::SIGN));
    return true;
  }
};

template <int OP, class L> int arith_for(const EwLaunch& a) {
  if ((a.flags & DCF_FLAG_ROUND_MASK) == 0) return launch_one<FArith<OP, L, true>>(a);
  return launch_one<FArith<OP, L, false>>(a);
}

template <class L> int float_binary_for(const EwLaunch& a) {
  switch (a.op) {
    case DCF_ADDF: return arith_for<DCF_ADDF, L>(a);
    case DCF_SUBF: return arith_for<DCF_SUBF, L>(a);
    case DCF_MULF: return arith_for<DCF_MULF, L>(a);
    case DCF_DIVF: return arith_for<DCF_DIVF, L>(a);
    case DCF_MAXIMUMF: return launch_one<FMinMax<L, true, true>>(a);
    case DCF_MINIMUMF: return launch_one<FMinMax<L, false, true>>(a);
    case DCF_MAXNUMF: return launch_one<FMinMax<L, true, false>>(a);
    case DCF_MINNUMF: return launch_one<FMinMax<L, false, false>>(a);
    case DCF_REMF: return launch_one<FRem<L>>(a);
    case DCF_CMPF: return launch_one<FCmp<L>>(a);
    case DCF_COPYSIGN: return launch_one<FCopySign<L>>(a);
    default: return DCF_EUNSUPPORTED;
  }
}

template <class L> int reciprocal_for(const EwLaunch& a) { return launch_one<FRecip<L>>(a); }

// Defined in dcf_ew_float_{f32,f64,h,f8}.cu.
int float_binary_f16(const EwLaunch& a);
int float_binary_bf16(const EwLaunch& a);
int float_binary_f32(const EwLaunch& a);
int float_binary_f64(const EwLaunch& a);
int float_binary_f8e5m2(const EwLaunch& a);
int float_binary_f8e4m3(const EwLaunch& a);
int float_binary_f8e3m4(const EwLaunch& a);
int reciprocal_f16(const EwLaunch& a);
int reciprocal_bf16(const EwLaunch& a);
int reciprocal_f32(const EwLaunch& a);
int reciprocal_f64(const EwLaunch& a);
int reciprocal_f8e5m2(const EwLaunch& a);
int reciprocal_f8e4m3(const EwLaunch& a);
int reciprocal_f8e3m4(const EwLaunch& a);

}  // namespace dcf
