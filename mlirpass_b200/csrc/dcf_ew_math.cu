// dcf_ew_math.cu — the exact math dialect folds that map one element to one
// element of the same type (ArithFolder::math,
// src/patterns/math/canonicalize.rs:145-234): absf, ceil, floor, roundeven,
// round, trunc, sqrt, rsqrt, absi, ctlz, cttz, ctpop.
//
// Every one is exact or correctly rounded, so the device result is the
// reference's bit for bit: the integral roundings are exact in the operand's
// own format, sqrt is IEEE's correctly rounded square root, and rsqrt is
// that root followed by a correctly rounded division, as `1.0 / sqrt(x)` is
// evaluated in the reference.
#include "dcf_convert_ops.cuh"

namespace dcf {

namespace {

// FloatFolds::integral (:87-92): NaN quieted, else round(to_f64) back in
// the same format, which is exact for an integral value.
template <class L, int OP> __device__ __forceinline__ uint64_t integral(uint64_t a) {
  if (is_nan<L>(a)) return a | L::QUIET;
  if constexpr (L::B == 4) {
    const float x = __uint_as_float((uint32_t)a);
    const float r = OP == DCF_CEIL ? ceilf(x) : OP == DCF_FLOOR ? floorf(x) : rintf(x);
    return __float_as_uint(r);
  } else {
    const double x = to_f64<L>(a);
    const double r = OP == DCF_CEIL ? ceil(x) : OP == DCF_FLOOR ? floor(x) : rint(x);
    if constexpr (L::B == 8) return (uint64_t)__double_as_longlong(r);
    else return convert_rn<F64L, L>((uint64_t)__double_as_longlong(r));
  }
}

template <class L, int OP> struct FMath {
  using In = typename L::T;
  using Out = typename L::T;
  static constexpr bool kBinary = false;
  __device__ static __forceinline__ bool apply(In in, uint32_t, Out& o) {
    const uint64_t a = in;
    if constexpr (OP == DCF_ABSF) {
      o = (Out)(a & ~L::SIGN);  // neg() of a negative value: the sign bit cleared
      return true;
    } else if constexpr (OP == DCF_CEIL || OP == DCF_FLOOR || OP == DCF_ROUNDEVEN) {
      o = (Out)integral<L, OP>(a);
      return true;
    } else if constexpr (L::B != 4 && L::B != 8) {
      o = 0;  // round / trunc / sqrt / rsqrt exist for f32 and f64 only
      return false;
    } else {
      if ((OP == DCF_SQRT || OP == DCF_RSQRT) && (a & L::SIGN)) {
        o = 0;  // is_negative(): -0 and NaNs with the sign bit refuse too
        return false;
      }
      if (is_nan<L>(a)) {
        o = (Out)(a | L::QUIET);
        return true;
      }
      if constexpr (L::B == 4) {
        const float x = __uint_as_float((uint32_t)a);
        float r;
        if constexpr (OP == DCF_ROUND) r = roundf(x);
        else if constexpr (OP == DCF_TRUNC) r = truncf(x);
        else if constexpr (OP == DCF_SQRT) r = __fsqrt_rn(x);
        else r = __fdiv_rn(1.0f, __fsqrt_rn(x));
        o = (Out)__float_as_uint(r);
      } else {
        const double x = __longlong_as_double((long long)a);
        double r;
        if constexpr (OP == DCF_ROUND) r = round(x);
        else if constexpr (OP == DCF_TRUNC) r = trunc(x);
        else if constexpr (OP == DCF_SQRT) r = __dsqrt_rn(x);
        else r = __ddiv_rn(1.0, __dsqrt_rn(x));
        o = (Out)(uint64_t)__double_as_longlong(r);
      }
      return true;
    }
  }
};

template <int W, int OP> struct IMath {
  using I = IntW<W>;
  using In = typename I::T;
  using Out = typename I::T;
  static constexpr bool kBinary = false;
  __device__ static __forceinline__ bool apply(In in, uint32_t, Out& o) {
    const uint64_t a = (uint64_t)in & I::MASK;
    uint64_t r;
    if constexpr (OP == DCF_ABSI) r = I::sx(a) < 0 ? (0 - a) & I::MASK : a;
    else if constexpr (OP == DCF_CTLZ) r = a == 0 ? W : (uint64_t)(__clzll((long long)a) - (64 - W));
    else if constexpr (OP == DCF_CTTZ) r = a == 0 ? W : (uint64_t)(__ffsll((long long)a) - 1);
    else r = (uint64_t)__popcll(a);
    o = (Out)r;
    return true;
  }
};

template <class L> int float_math_for(const EwLaunch& a) {
  switch (a.op) {
    case DCF_ABSF: return launch_one<FMath<L, DCF_ABSF>>(a);
    case DCF_CEIL: return launch_one<FMath<L, DCF_CEIL>>(a);
    case DCF_FLOOR: return launch_one<FMath<L, DCF_FLOOR>>(a);
    case DCF_ROUNDEVEN: return launch_one<FMath<L, DCF_ROUNDEVEN>>(a);
    case DCF_ROUND: return launch_one<FMath<L, DCF_ROUND>>(a);
    case DCF_TRUNC: return launch_one<FMath<L, DCF_TRUNC>>(a);
    case DCF_SQRT: return launch_one<FMath<L, DCF_SQRT>>(a);
    case DCF_RSQRT: return launch_one<FMath<L, DCF_RSQRT>>(a);
    default: return DCF_EUNSUPPORTED;
  }
}

template <int W> int int_math_for(const EwLaunch& a) {
  switch (a.op) {
    case DCF_ABSI: return launch_one<IMath<W, DCF_ABSI>>(a);
    case DCF_CTLZ: return launch_one<IMath<W, DCF_CTLZ>>(a);
    case DCF_CTTZ: return launch_one<IMath<W, DCF_CTTZ>>(a);
    case DCF_CTPOP: return launch_one<IMath<W, DCF_CTPOP>>(a);
    default: return DCF_EUNSUPPORTED;
  }
}

}  // namespace

int launch_math_unary(const EwLaunch& a) {
  if (a.dtype != a.out_dtype) return DCF_EUNSUPPORTED;
  if (op_math_float_unary(a.op)) return with_float(a.dtype, [&](auto s) { return float_math_for<decltype(s)>(a); });
  if (op_math_int_unary(a.op))
    return with_int(a.dtype, [&](auto i) { return int_math_for<decltype(i)::w>(a); });
  return DCF_EUNSUPPORTED;
}

}  // namespace dcf
