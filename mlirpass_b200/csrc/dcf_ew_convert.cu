// dcf_ew_convert.cu — conversion folds: extf / truncf (float_convert with
// the exactness test), sitofp / uitofp, fptosi / fptoui.
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

template <class F> static int with_float(int dtype, F&& f) {
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

template <class F> static int with_int(int dtype, F&& f) {
  switch (dtype) {
    case DCF_I1: return f(IntW<1>{});
    case DCF_I8: return f(IntW<8>{});
    case DCF_I16: return f(IntW<16>{});
    case DCF_I32: return f(IntW<32>{});
    case DCF_I64: return f(IntW<64>{});
    default: return DCF_EUNSUPPORTED;
  }
}

int launch_convert(const EwLaunch& a) {
  switch (a.op) {
    case DCF_EXTF:
    case DCF_TRUNCF:
      return with_float(a.dtype, [&](auto s) {
        return with_float(a.out_dtype, [&](auto d) {
          using S = decltype(s);
          using D = decltype(d);
          return launch_one<CvtFF<S, D>>(a);
        });
      });
    case DCF_SITOFP:
    case DCF_UITOFP: {
      const bool sg = a.op == DCF_SITOFP;
      return with_int(a.dtype, [&](auto i) {
        return with_float(a.out_dtype, [&](auto d) {
          using D = decltype(d);
          constexpr int W = decltype(i)::w;
          return sg ? launch_one<CvtIF<W, true, D>>(a) : launch_one<CvtIF<W, false, D>>(a);
        });
      });
    }
    case DCF_FPTOSI:
    case DCF_FPTOUI: {
      const bool sg = a.op == DCF_FPTOSI;
      return with_float(a.dtype, [&](auto s) {
        return with_int(a.out_dtype, [&](auto i) {
          using S = decltype(s);
          constexpr int W = decltype(i)::w;
          return sg ? launch_one<CvtFI<S, W, true>>(a) : launch_one<CvtFI<S, W, false>>(a);
        });
      });
    }
    default:
      return DCF_EUNSUPPORTED;
  }
}

}  // namespace dcf
