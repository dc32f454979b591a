// dcf_convert_ops.cuh — functors of the conversion folds: extf / truncf /
// convertf (float_convert with the exactness test), sitofp / uitofp,
// fptosi / fptoui, negf, flush_denormals and extsi / extui / trunci, with
// the layout dispatch helpers.  The float->float, int->float and
// float->int families are instantiated in their own translation units
// (dcf_ew_convert_{ff,if,fi}.cu) so the library builds in parallel.
#pragma once

#include "dcf_kernels.cuh"

namespace dcf {

template <class S, class D> struct CvtFF {
  using In = typename S::T;
  using Out = typename D::T;
  static constexpr bool kBinary = false;
  __device__ static __forceinline__ bool apply(In a, uint32_t, Out& o) {
    uint64_t r = 0;
    const bool ok = float_convert<S, D>(a, r);
    o = (Out)r;
    return ok;
  }
};

template <int W, bool SIGNED, class D> struct CvtIF {
  using In = typename IntW<W>::T;
  using Out = typename D::T;
  static constexpr bool kBinary = false;
  __device__ static __forceinline__ bool apply(In a, uint32_t, Out& o) {
    o = (Out)int_to_float<W, SIGNED, D>(a);
    return true;
  }
};

template <class S, int W, bool SIGNED> struct CvtFI {
  using In = typename S::T;
  using Out = typename IntW<W>::T;
  static constexpr bool kBinary = false;
  __device__ static __forceinline__ bool apply(In a, uint32_t, Out& o) {
    uint64_t r = 0;
    const bool ok = float_to_int<S, W, SIGNED>(a, r);
    o = (Out)r;
    return ok;
  }
};

// negf (a sign flip) and flush_denormals, element type unchanged.
template <class L, bool NEG> struct FSign {
  using In = typename L::T;
  using Out = typename L::T;
  static constexpr bool kBinary = false;
  __device__ static __forceinline__ bool apply(In a, uint32_t, Out& o) {
    if constexpr (NEG) o = (Out)(a ^ (In)L::SIGN);
    else o = (Out)flush_denormal<L>(a);
    return true;
  }
};

// extsi / extui / trunci (ApInt sext / zext / trunc).
template <int WI, int WO, bool SIGNED> struct CvtII {
  using In = typename IntW<WI>::T;
  using Out = typename IntW<WO>::T;
  static constexpr bool kBinary = false;
  __device__ static __forceinline__ bool apply(In a, uint32_t, Out& o) {
    const uint64_t v = SIGNED ? (uint64_t)IntW<WI>::sx(a) : ((uint64_t)a & IntW<WI>::MASK);
    o = (Out)(v & IntW<WO>::MASK);
    return true;
  }
};

template <class F> int with_float(int dtype, F&& f) {
  switch (dtype) {
    case DCF_F16: return f(F16L{});
    case DCF_BF16: return f(BF16L{});
    case DCF_F32: return f(F32L{});
    case DCF_F64: return f(F64L{});
    case DCF_F8E5M2: return f(F8E5M2L{});
    case DCF_F8E4M3: return f(F8E4M3L{});
    case DCF_F8E3M4: return f(F8E3M4L{});
    default: return DCF_EUNSUPPORTED;
  }
}

template <class F> int with_int(int dtype, F&& f) {
  switch (dtype) {
    case DCF_I1: return f(IntW<1>{});
    case DCF_I8: return f(IntW<8>{});
    case DCF_I16: return f(IntW<16>{});
    case DCF_I32: return f(IntW<32>{});
    case DCF_I64: return f(IntW<64>{});
    default: return DCF_EUNSUPPORTED;
  }
}

int launch_convert_ff(const EwLaunch& a);  // extf, truncf
int launch_convert_if(const EwLaunch& a);  // sitofp, uitofp
int launch_convert_fi(const EwLaunch& a);  // fptosi, fptoui

}  // namespace dcf
