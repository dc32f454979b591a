// dcf_ew_float.cu — float binary folds (addf, subf, mulf, divf, the four
// min/max ops), dense cmpf and tosa reciprocal.
#include "dcf_kernels.cuh"

namespace dcf {

// NEAREST: the roundingmode property is absent or nearest-even, the only
// mode every fold config uses; the directed modes get their own kernels so
// the common one carries none of their code.
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

template <int OP, class L> static int arith_for(const EwLaunch& a) {
  if ((a.flags & DCF_FLAG_ROUND_MASK) == 0) return launch_one<FArith<OP, L, true>>(a);
  return launch_one<FArith<OP, L, false>>(a);
}

template <class L> static int float_binary_for(const EwLaunch& a) {
  switch (a.op) {
    case DCF_ADDF: return arith_for<DCF_ADDF, L>(a);
    case DCF_SUBF: return arith_for<DCF_SUBF, L>(a);
    case DCF_MULF: return arith_for<DCF_MULF, L>(a);
    case DCF_DIVF: return arith_for<DCF_DIVF, L>(a);
    case DCF_MAXIMUMF: return launch_one<FMinMax<L, true, true>>(a);
    case DCF_MINIMUMF: return launch_one<FMinMax<L, false, true>>(a);
    case DCF_MAXNUMF: return launch_one<FMinMax<L, true, false>>(a);
    case DCF_MINNUMF: return launch_one<FMinMax<L, false, false>>(a);
    case DCF_CMPF: return launch_one<FCmp<L>>(a);
    default: return DCF_EUNSUPPORTED;
  }
}

int launch_float_binary(const EwLaunch& a) {
  switch (a.dtype) {
    case DCF_F16: return float_binary_for<F16L>(a);
    case DCF_BF16: return float_binary_for<BF16L>(a);
    case DCF_F32: return float_binary_for<F32L>(a);
    case DCF_F64: return float_binary_for<F64L>(a);
    case DCF_F8E5M2: return float_binary_for<F8E5M2L>(a);
    case DCF_F8E4M3: return float_binary_for<F8E4M3L>(a);
    case DCF_F8E3M4: return float_binary_for<F8E3M4L>(a);
    default: return DCF_EUNSUPPORTED;
  }
}

int launch_reciprocal(const EwLaunch& a) {
  switch (a.dtype) {
    case DCF_F16: return launch_one<FRecip<F16L>>(a);
    case DCF_BF16: return launch_one<FRecip<BF16L>>(a);
    case DCF_F32: return launch_one<FRecip<F32L>>(a);
    case DCF_F64: return launch_one<FRecip<F64L>>(a);
    case DCF_F8E5M2: return launch_one<FRecip<F8E5M2L>>(a);
    case DCF_F8E4M3: return launch_one<FRecip<F8E4M3L>>(a);
    case DCF_F8E3M4: return launch_one<FRecip<F8E3M4L>>(a);
    default: return DCF_EUNSUPPORTED;
  }
}

}  // namespace dcf
