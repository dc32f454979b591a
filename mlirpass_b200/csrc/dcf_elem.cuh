// dcf_elem.cuh — per-element fold semantics on the device (sm_100a).
//
// Every function here is the device form of one closure of mlirpass's
// constant folder (paths inside the mlirpass repository):
//   float add/sub/mul/div  Rounded::apply   src/patterns/arith/canonicalize.rs:984-1055
//   min/max                minmax           src/patterns/arith/canonicalize.rs:132-150
//   cmpf / cmpi            cmpf, cmpi       src/patterns/arith/canonicalize.rs:94-130
//   integer ops            ArithFolder::fold src/patterns/arith/canonicalize.rs:277-325, 469-683
//   extf / truncf          float_convert + nan_convert :50-67, :727-742
//   sitofp / uitofp        :402-417;  fptosi / fptoui :418-434
//   reciprocal             Tf::reciprocal   src/patterns/tosa/canonicalize.rs:596-605
//
// Floating point uses the explicit round-to-nearest intrinsics (__fadd_rn,
// __fmul_rn, __fdiv_rn, __fmaf_rn, ...) and the library is compiled with
// -fmad=false -ftz=false -prec-div=true, so each operation is one IEEE-754
// rounding with subnormals kept.  The hardware's canonical NaN is never
// emitted: NaN operands propagate quieted (first NaN operand wins) and an
// invalid operation yields the default quiet NaN chosen by the flags.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/dcfold.h"

namespace dcf {

// ------------------------------------------------------------ storage

template <int B> struct Bits;
template <> struct Bits<1> { using T = uint8_t; };
template <> struct Bits<2> { using T = uint16_t; };
template <> struct Bits<4> { using T = uint32_t; };
template <> struct Bits<8> { using T = uint64_t; };

// IEEE-like layout: E exponent bits, M mantissa bits, B storage bytes.
template <int E_, int M_, int B_> struct FL {
  static constexpr int E = E_, M = M_, B = B_;
  using T = typename Bits<B_>::T;
  static constexpr uint64_t SIGN = 1ull << (E_ + M_);
  static constexpr uint64_t EXPM = ((1ull << E_) - 1) << M_;
  static constexpr uint64_t MANT = (1ull << M_) - 1;
  static constexpr uint64_t QUIET = 1ull << (M_ - 1);
};
using F16L = FL<5, 10, 2>;
using BF16L = FL<8, 7, 2>;
using F32L = FL<8, 23, 4>;
using F64L = FL<11, 52, 8>;
using F8E5M2L = FL<5, 2, 1>;
using F8E4M3L = FL<4, 3, 1>;
using F8E3M4L = FL<3, 4, 1>;

template <class L> __device__ __forceinline__ bool is_nan(uint64_t b) {
  return (b & L::EXPM) == L::EXPM && (b & L::MANT) != 0;
}
template <class L> __device__ __forceinline__ bool is_inf(uint64_t b) {
  return (b & (L::EXPM | L::MANT)) == L::EXPM;
}
template <class L> __device__ __forceinline__ bool is_zero(uint64_t b) {
  return (b & (L::EXPM | L::MANT)) == 0;
}
template <class L> __device__ __forceinline__ bool sign_of(uint64_t b) {
  return (b & L::SIGN) != 0;
}
template <class L> __device__ __forceinline__ uint64_t default_nan(uint32_t flags) {
  return ((flags & DCF_FLAG_NEG_DEFAULT_NAN) ? L::SIGN : 0) | L::EXPM | L::QUIET;
}

// Exact widening of a narrow IEEE-like value to float / double.
template <class L> __device__ __forceinline__ float to_f32(uint64_t b);
template <> __device__ __forceinline__ float to_f32<F32L>(uint64_t b) {
  return __uint_as_float((uint32_t)b);
}
template <> __device__ __forceinline__ float to_f32<BF16L>(uint64_t b) {
  return __uint_as_float((uint32_t)b << 16);
}
template <> __device__ __forceinline__ float to_f32<F16L>(uint64_t b) {
  return __half2float(__ushort_as_half((unsigned short)b));
}

// Round a float to the narrow layout, nearest-even (overflow -> inf).
template <class L> __device__ __forceinline__ uint64_t from_f32_rn(float x);
template <> __device__ __forceinline__ uint64_t from_f32_rn<F32L>(float x) {
  return __float_as_uint(x);
}
template <> __device__ __forceinline__ uint64_t from_f32_rn<BF16L>(float x) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(x));
}
template <> __device__ __forceinline__ uint64_t from_f32_rn<F16L>(float x) {
  return __half_as_ushort(__float2half_rn(x));
}

// Generic value -> layout rounding, nearest-even: v = sig * 2^exp, sig != 0
// fits in 64 bits.  Used for the f8 kinds, f16 <-> bf16 and integer ->
// float paths that have no hardware instruction.
template <class L>
__device__ __forceinline__ uint64_t round_pack(bool neg, uint64_t sig, int exp) {
  const uint64_t s = neg ? L::SIGN : 0;
  if (sig == 0) return s;
  const int bias = (1 << (L::E - 1)) - 1;
  const int emin = 1 - bias;
  const int p = 63 - __clzll((long long)sig);
  const int e = p + exp;
  const int q = (e < emin) ? emin - L::M : e - L::M;
  const int sh = q - exp;
  uint64_t r;
  if (sh <= 0) {
    r = sig << (-sh);
  } else if (sh > 64) {
    r = 0;
  } else if (sh == 64) {
    r = (sig > (1ull << 63)) ? 1 : 0;
  } else {
    const uint64_t rem = sig & ((1ull << sh) - 1), half = 1ull << (sh - 1);
    r = sig >> sh;
    r += (rem > half || (rem == half && (r & 1))) ? 1 : 0;
  }
  uint64_t bits = (e < emin) ? r : (((uint64_t)(e + bias - 1) << L::M) + r);
  const uint64_t maxe = (1ull << L::E) - 1;
  if ((bits >> L::M) >= maxe) bits = maxe << L::M;
  return s | bits;
}

// Decode a finite value: v = sig * 2^exp.
template <class L>
__device__ __forceinline__ void decode(uint64_t b, uint64_t& sig, int& exp) {
  const int bias = (1 << (L::E - 1)) - 1;
  const uint64_t ef = (b & L::EXPM) >> L::M, m = b & L::MANT;
  if (ef == 0) {
    sig = m;
    exp = 1 - bias - L::M;
  } else {
    sig = m | (1ull << L::M);
    exp = (int)ef - bias - L::M;
  }
}

// ApFloat::convert between layouts, nearest-even, non-NaN input.
template <class S, class D> __device__ __forceinline__ uint64_t convert_rn(uint64_t b) {
  const bool neg = sign_of<S>(b);
  if (is_inf<S>(b)) return (neg ? D::SIGN : 0) | D::EXPM;
  uint64_t sig;
  int exp;
  decode<S>(b, sig, exp);
  return round_pack<D>(neg, sig, exp);
}

template <class L> __device__ __forceinline__ double to_f64(uint64_t b) {
  if (L::B == 8) return __longlong_as_double((long long)b);
  if (L::B == 4) return (double)__uint_as_float((uint32_t)b);
  if (is_nan<L>(b)) return __longlong_as_double(0x7FF8000000000000ll);
  return __longlong_as_double((long long)convert_rn<L, F64L>(b));
}

// ----------------------------------------------- float binary arithmetic

// NaN result of an operation whose operands were a and b: the first NaN
// operand quieted, else (an invalid operation) the default NaN.
template <class L>
__device__ __forceinline__ uint64_t nan_result(uint64_t a, uint64_t b, uint64_t dnan) {
  if (is_nan<L>(a)) return a | L::QUIET;
  if (is_nan<L>(b)) return b | L::QUIET;
  return dnan;
}

// ApFloat add/sub/mul/div at nearest-even with the NaN rule.  The hardware
// result is used unless it is NaN; only then are the operands examined (a
// non-NaN result implies that neither operand was NaN).
template <int OP, class L>
__device__ __forceinline__ uint64_t arith_rn(uint64_t a, uint64_t b, uint64_t dnan) {
  if constexpr (L::B == 8) {
    const double x = __longlong_as_double((long long)a), y = __longlong_as_double((long long)b);
    double z;
    if constexpr (OP == DCF_ADDF) z = __dadd_rn(x, y);
    else if constexpr (OP == DCF_SUBF) z = __dsub_rn(x, y);
    else if constexpr (OP == DCF_MULF) z = __dmul_rn(x, y);
    else z = __ddiv_rn(x, y);
    if (z != z) return nan_result<L>(a, b, dnan);
    return (uint64_t)__double_as_longlong(z);
  } else if constexpr (L::B == 4 || L::E + L::M == 15) {
    // f32 directly; f16 / bf16 through f32 (precision 24 >= 2p+2, so the
    // two roundings equal one correct rounding to the narrow kind).
    const float x = to_f32<L>(a), y = to_f32<L>(b);
    float z;
    if constexpr (OP == DCF_ADDF) z = __fadd_rn(x, y);
    else if constexpr (OP == DCF_SUBF) z = __fsub_rn(x, y);
    else if constexpr (OP == DCF_MULF) z = __fmul_rn(x, y);
    else z = __fdiv_rn(x, y);
    if (z != z) return nan_result<L>(a, b, dnan);
    return from_f32_rn<L>(z);
  } else {
    // f8 kinds: exact in f32 too; round with the generic packer.
    const float x = __uint_as_float((uint32_t)convert_rn<L, F32L>(a));
    const float y = __uint_as_float((uint32_t)convert_rn<L, F32L>(b));
    float z;
    if constexpr (OP == DCF_ADDF) z = __fadd_rn(x, y);
    else if constexpr (OP == DCF_SUBF) z = __fsub_rn(x, y);
    else if constexpr (OP == DCF_MULF) z = __fmul_rn(x, y);
    else z = __fdiv_rn(x, y);
    if (z != z || is_nan<L>(a) || is_nan<L>(b)) return nan_result<L>(a, b, dnan);
    return convert_rn<F32L, L>(__float_as_uint(z));
  }
}

__device__ __forceinline__ uint32_t f32_next(uint32_t b, bool up) {
  if ((b & 0x7FFFFFFFu) > 0x7F800000u) return b;
  if (up && b == 0x7F800000u) return b;
  if (!up && b == 0xFF800000u) return b;
  const uint32_t abs = b & 0x7FFFFFFFu;
  if (abs == 0) return up ? 1u : 0x80000001u;
  if (b == abs) return up ? b + 1 : b - 1;
  return up ? b - 1 : b + 1;
}

__device__ __forceinline__ uint64_t f64_next(uint64_t b, bool up) {
  if ((b & 0x7FFFFFFFFFFFFFFFull) > 0x7FF0000000000000ull) return b;
  if (up && b == 0x7FF0000000000000ull) return b;
  if (!up && b == 0xFFF0000000000000ull) return b;
  const uint64_t abs = b & 0x7FFFFFFFFFFFFFFFull;
  if (abs == 0) return up ? 1ull : 0x8000000000000001ull;
  if (b == abs) return up ? b + 1 : b - 1;
  return up ? b - 1 : b + 1;
}

// Rounded::apply: nearest-even result, then the directed-rounding step
// from the exact error term (TwoSum for add/sub, FMA for mul/div), the
// way the reference computes it.  Returns false when the element refuses.
template <int OP, class L>
__device__ __forceinline__ bool rounded(uint64_t a, uint64_t b, int mode, uint64_t dnan, uint64_t& out) {
  const uint64_t nearest = arith_rn<OP, L>(a, b, dnan);
  if (mode == 0 || is_nan<L>(nearest)) {
    out = nearest;
    return true;
  }
  double err, r;
  if constexpr (L::B == 8) {
    const double x = __longlong_as_double((long long)a);
    double y = __longlong_as_double((long long)b);
    r = __longlong_as_double((long long)nearest);
    if (isinf(r) && isfinite(x) && isfinite(y)) {
      err = -r;
    } else if constexpr (OP == DCF_ADDF || OP == DCF_SUBF) {
      if (OP == DCF_SUBF) y = -y;
      const double bb = __dsub_rn(r, x);
      err = __dadd_rn(__dsub_rn(x, __dsub_rn(r, bb)), __dsub_rn(y, bb));
    } else if constexpr (OP == DCF_MULF) {
      err = __fma_rn(x, y, -r);
    } else {
      err = __dmul_rn(__fma_rn(-r, y, x), copysign(1.0, y));
    }
  } else if constexpr (L::B == 4) {
    const float x = __uint_as_float((uint32_t)a);
    float y = __uint_as_float((uint32_t)b);
    const float rf = __uint_as_float((uint32_t)nearest);
    float e;
    if (isinf(rf) && isfinite(x) && isfinite(y)) {
      e = -rf;
    } else if constexpr (OP == DCF_ADDF || OP == DCF_SUBF) {
      if (OP == DCF_SUBF) y = -y;
      const float bb = __fsub_rn(rf, x);
      e = __fadd_rn(__fsub_rn(x, __fsub_rn(rf, bb)), __fsub_rn(y, bb));
    } else if constexpr (OP == DCF_MULF) {
      e = __fmaf_rn(x, y, -rf);
    } else {
      e = __fmul_rn(__fmaf_rn(-rf, y, x), copysignf(1.0f, y));
    }
    err = (double)e;
    r = (double)rf;
  } else {
    return false;  // non-nearest modes fold only f32 / f64
  }
  if (err == 0.0) {
    out = nearest;
    return true;
  }
  int step = -1;
  if (mode == 1) step = (err < 0.0) ? 0 : -1;
  else if (mode == 2) step = (err > 0.0) ? 1 : -1;
  else if (mode == 3) step = ((r > 0.0 && err < 0.0) || (r < 0.0 && err > 0.0)) ? (r < 0.0 ? 1 : 0) : -1;
  else if (mode == 4) return false;
  if (step < 0) out = nearest;
  else if constexpr (L::B == 8) out = f64_next(nearest, step == 1);
  else out = f32_next((uint32_t)nearest, step == 1);
  return true;
}

// Partial compare: -2 unordered, else -1 / 0 / 1.
template <class L> __device__ __forceinline__ int fcompare(uint64_t a, uint64_t b) {
  if (is_nan<L>(a) || is_nan<L>(b)) return -2;
  if constexpr (L::B == 8) {
    const double x = __longlong_as_double((long long)a), y = __longlong_as_double((long long)b);
    return x < y ? -1 : (x > y ? 1 : 0);
  } else if constexpr (L::B == 4 || L::E + L::M == 15) {
    const float x = to_f32<L>(a), y = to_f32<L>(b);
    return x < y ? -1 : (x > y ? 1 : 0);
  } else {
    const float x = __uint_as_float((uint32_t)convert_rn<L, F32L>(a));
    const float y = __uint_as_float((uint32_t)convert_rn<L, F32L>(b));
    return x < y ? -1 : (x > y ? 1 : 0);
  }
}

// Total order of the non-NaN values of a sign-magnitude layout as a signed
// integer: -0 just below +0, negatives by magnitude downwards.  It is the
// numeric order with maximumf's -0 < +0 (canonicalize.rs:132-150), so one
// integer compare decides min / max.
template <class L> __device__ __forceinline__ auto order_key(uint64_t x) {
  if constexpr (L::B == 8) {
    const int64_t m = (int64_t)(x & (L::SIGN - 1));
    return (x & L::SIGN) ? -m - 1 : m;
  } else {
    const int32_t m = (int32_t)(x & (L::SIGN - 1));
    return (x & L::SIGN) ? -m - 1 : m;
  }
}

template <class L, bool MAX, bool NANWINS>
__device__ __forceinline__ uint64_t minmax(uint64_t a, uint64_t b) {
  const bool an = is_nan<L>(a), bn = is_nan<L>(b);
  if (an || bn) {
    if (NANWINS) return an ? (a | L::QUIET) : (b | L::QUIET);
    if (an && !(a & L::QUIET)) return a | L::QUIET;
    if (bn && !(b & L::QUIET)) return b | L::QUIET;
    return an ? b : a;
  }
  const auto ka = order_key<L>(a), kb = order_key<L>(b);
  if (MAX) return ka < kb ? b : a;
  return kb < ka ? b : a;
}

template <class L> __device__ __forceinline__ uint8_t cmpf(int pred, uint64_t a, uint64_t b) {
  const int c = fcompare<L>(a, b);
  const bool lt = c == -1, eq = c == 0, gt = c == 1, un = c == -2;
  switch (pred) {
    case 0: return 0;
    case 1: return eq;
    case 2: return gt;
    case 3: return gt || eq;
    case 4: return lt;
    case 5: return lt || eq;
    case 6: return !un && !eq;
    case 7: return !un;
    case 8: return un || eq;
    case 9: return un || gt;
    case 10: return un || gt || eq;
    case 11: return un || lt;
    case 12: return un || lt || eq;
    case 13: return !eq;
    case 14: return un;
    default: return 1;
  }
}

// ------------------------------------------------------------- integers

template <int W> struct IntW {
  static constexpr int w = W;
  using T = typename Bits<(W == 1 ? 1 : W / 8)>::T;
  static constexpr uint64_t MASK = (W == 64) ? ~0ull : ((1ull << W) - 1);
  __device__ static __forceinline__ int64_t sx(uint64_t v) {
    if constexpr (W == 64) return (int64_t)v;
    const uint64_t m = 1ull << (W - 1);
    return (int64_t)(((v & MASK) ^ m) - m);
  }
};

template <int OP, int W>
__device__ __forceinline__ bool int_op(uint64_t a, uint64_t b, uint64_t& out) {
  using I = IntW<W>;
  const uint64_t ua = a & I::MASK, ub = b & I::MASK;
  if constexpr (OP == DCF_ADDI) { out = (ua + ub) & I::MASK; return true; }
  else if constexpr (OP == DCF_SUBI) { out = (ua - ub) & I::MASK; return true; }
  else if constexpr (OP == DCF_MULI) {
    if constexpr (W <= 32) out = (uint64_t)((uint32_t)ua * (uint32_t)ub) & I::MASK;
    else out = ua * ub;
    return true;
  }
  else if constexpr (OP == DCF_ANDI) { out = ua & ub; return true; }
  else if constexpr (OP == DCF_ORI) { out = ua | ub; return true; }
  else if constexpr (OP == DCF_XORI) { out = ua ^ ub; return true; }
  else if constexpr (OP == DCF_SHLI || OP == DCF_SHRUI || OP == DCF_SHRSI) {
    if (ub >= (uint64_t)W) return false;
    if constexpr (OP == DCF_SHLI) out = (ua << ub) & I::MASK;
    else if constexpr (OP == DCF_SHRUI) out = ua >> ub;
    else out = (uint64_t)(I::sx(ua) >> ub) & I::MASK;
    return true;
  }
  else if constexpr (OP == DCF_DIVSI) {
    if (ub == 0) return false;
    const int64_t sa = I::sx(ua), sb = I::sx(ub);
    const int64_t smin = (W == 64) ? (int64_t)0x8000000000000000ull : -(int64_t)(1ull << (W - 1));
    if (sa == smin && sb == -1) return false;
    if constexpr (W <= 32) out = (uint64_t)(int64_t)((int32_t)sa / (int32_t)sb) & I::MASK;
    else out = (uint64_t)(sa / sb);
    return true;
  }
  else if constexpr (OP == DCF_DIVUI) {
    if (ub == 0) return false;
    if constexpr (W <= 32) out = (uint32_t)ua / (uint32_t)ub;
    else out = ua / ub;
    return true;
  }
  else if constexpr (OP == DCF_REMSI) {
    if (ub == 0) return false;
    const int64_t sa = I::sx(ua), sb = I::sx(ub);
    if (sb == -1) { out = 0; return true; }   // INT_MIN % -1 folds to 0
    if constexpr (W <= 32) out = (uint64_t)(int64_t)((int32_t)sa % (int32_t)sb) & I::MASK;
    else out = (uint64_t)(sa % sb);
    return true;
  }
  else if constexpr (OP == DCF_REMUI) {
    if (ub == 0) return false;
    if constexpr (W <= 32) out = (uint32_t)ua % (uint32_t)ub;
    else out = ua % ub;
    return true;
  }
  else if constexpr (OP == DCF_CEILDIVUI) {                  // canonicalize.rs:287-298
    if (ub == 0) return false;
    out = (ua / ub + (ua % ub != 0 ? 1 : 0)) & I::MASK;
    return true;
  }
  else if constexpr (OP == DCF_CEILDIVSI) {                  // ceildivsi, :557-595
    // Every overflow flag of the reference's steps is raised exactly when
    // an operand is the signed minimum (and the dividend is not zero).
    if (ub == 0) return false;
    const int64_t sa = I::sx(ua), sb = I::sx(ub);
    if (sa == 0) { out = 0; return true; }
    const int64_t smin = (W == 64) ? (int64_t)0x8000000000000000ull : -(int64_t)(1ull << (W - 1));
    if (sa == smin || sb == smin) return false;
    int64_t q = sa / sb;
    if (sa % sb != 0 && ((sa > 0) == (sb > 0))) q += 1;
    out = (uint64_t)q & I::MASK;
    return true;
  }
  else if constexpr (OP == DCF_FLOORDIVSI) {                 // :306-317
    if (ub == 0) return false;
    const int64_t sa = I::sx(ua), sb = I::sx(ub);
    const int64_t smin = (W == 64) ? (int64_t)0x8000000000000000ull : -(int64_t)(1ull << (W - 1));
    if (sa == smin && sb == -1) return false;
    int64_t q = sa / sb;
    const int64_t r = sa % sb;
    if (r != 0 && ((r < 0) != (sb < 0))) q -= 1;
    out = (uint64_t)q & I::MASK;
    return true;
  }
  else if constexpr (OP == DCF_MULSI_HI) {                   // mul_extended, :939-944
    if constexpr (W == 64) out = (uint64_t)__mul64hi((long long)ua, (long long)ub);
    else out = (uint64_t)((I::sx(ua) * I::sx(ub)) >> W) & I::MASK;
    return true;
  }
  else if constexpr (OP == DCF_MULUI_HI) {
    if constexpr (W == 64) out = (uint64_t)__umul64hi(ua, ub);
    else out = ((ua * ub) >> W) & I::MASK;
    return true;
  }
  else if constexpr (OP == DCF_MAXSI) { out = I::sx(ua) > I::sx(ub) ? ua : ub; return true; }
  else if constexpr (OP == DCF_MAXUI) { out = ua > ub ? ua : ub; return true; }
  else if constexpr (OP == DCF_MINSI) { out = I::sx(ua) < I::sx(ub) ? ua : ub; return true; }
  else if constexpr (OP == DCF_MINUI) { out = ua < ub ? ua : ub; return true; }
  else { return false; }
}

template <int W> __device__ __forceinline__ uint8_t cmpi(int pred, uint64_t a, uint64_t b) {
  using I = IntW<W>;
  const uint64_t ua = a & I::MASK, ub = b & I::MASK;
  const int64_t sa = I::sx(ua), sb = I::sx(ub);
  switch (pred) {
    case 0: return ua == ub;
    case 1: return ua != ub;
    case 2: return sa < sb;
    case 3: return sa <= sb;
    case 4: return sa > sb;
    case 5: return sa >= sb;
    case 6: return ua < ub;
    case 7: return ua <= ub;
    case 8: return ua > ub;
    default: return ua >= ub;
  }
}

// addui_extended's overflow bit (canonicalize.rs:887-891): sum <u lhs.
template <int W> __device__ __forceinline__ uint8_t add_carry(uint64_t a, uint64_t b) {
  using I = IntW<W>;
  const uint64_t ua = a & I::MASK;
  return ((ua + (b & I::MASK)) & I::MASK) < ua;
}

// remf, `x % y` (canonicalize.rs:387): the remainder of truncating
// division, which is always exact, so computing it in a wider format and
// narrowing back loses nothing.  NaN operands propagate quieted (first one
// wins); inf % y and x % 0 are invalid and give the default NaN.
template <class L> __device__ __forceinline__ uint64_t remf(uint64_t a, uint64_t b, uint64_t dnan) {
  if (is_nan<L>(a) || is_nan<L>(b)) return nan_result<L>(a, b, dnan);
  if (is_inf<L>(a) || is_zero<L>(b)) return dnan;
  if (is_inf<L>(b) || is_zero<L>(a)) return a;
  if constexpr (L::B == 8) {
    return (uint64_t)__double_as_longlong(fmod(__longlong_as_double((long long)a), __longlong_as_double((long long)b)));
  } else if constexpr (L::B == 4 || L::E + L::M == 15) {
    return from_f32_rn<L>(fmodf(to_f32<L>(a), to_f32<L>(b)));
  } else {
    const float x = __uint_as_float((uint32_t)convert_rn<L, F32L>(a));
    const float y = __uint_as_float((uint32_t)convert_rn<L, F32L>(b));
    return convert_rn<F32L, L>(__float_as_uint(fmodf(x, y)));
  }
}

// flush_denormal (canonicalize.rs:69-77): a subnormal becomes the zero of
// its sign; everything else is kept.
template <class L> __device__ __forceinline__ uint64_t flush_denormal(uint64_t b) {
  if ((b & L::EXPM) == 0 && (b & L::MANT) != 0) return b & L::SIGN;
  return b;
}

// --------------------------------------------------------- conversions

// nan_convert (canonicalize.rs:50-67): quiet NaNs only, no payload lost.
template <class S, class D> __device__ __forceinline__ bool nan_convert(uint64_t b, uint64_t& out) {
  uint64_t mant = b & S::MANT;
  if (!(mant & S::QUIET)) return false;
  if constexpr (D::M < S::M) {
    constexpr int lost = S::M - D::M;
    if (mant & ((1ull << lost) - 1)) return false;
    mant >>= lost;
  } else {
    mant <<= (D::M - S::M);
  }
  out = (sign_of<S>(b) ? D::SIGN : 0) | D::EXPM | mant;
  return true;
}

// float_convert closure (canonicalize.rs:730-741): fold only when the value
// survives convert and convert-back bit for bit, infinity-ness kept.
template <class S, class D> __device__ __forceinline__ bool float_convert(uint64_t b, uint64_t& out) {
  if (is_nan<S>(b)) return nan_convert<S, D>(b, out);
  uint64_t to;
  if constexpr (S::B == 4 && D::B == 2 && D::E == 8) {
    // f32 -> bf16: representable iff the low 16 bits are zero.
    if (b & 0xFFFFu) return false;
    out = b >> 16;
    return true;
  } else if constexpr (S::B == 2 && S::E == 8 && D::B == 4) {
    out = b << 16;  // bf16 -> f32, exact
    return true;
  } else if constexpr (S::B == 4 && D::B == 2 && D::E == 5) {
    to = __half_as_ushort(__float2half_rn(__uint_as_float((uint32_t)b)));
    const uint64_t back = __float_as_uint(__half2float(__ushort_as_half((unsigned short)to)));
    if (back != b || is_inf<D>(to) != is_inf<S>(b)) return false;
    out = to;
    return true;
  } else if constexpr (S::B == 2 && S::E == 5 && D::B == 4) {
    out = __float_as_uint(__half2float(__ushort_as_half((unsigned short)b)));
    return true;
  } else if constexpr (S::B == 4 && D::B == 8) {
    out = (uint64_t)__double_as_longlong((double)__uint_as_float((uint32_t)b));
    return true;
  } else if constexpr (S::B == 8 && D::B == 4) {
    to = __float_as_uint(__double2float_rn(__longlong_as_double((long long)b)));
    const uint64_t back = (uint64_t)__double_as_longlong((double)__uint_as_float((uint32_t)to));
    if (back != b || is_inf<D>(to) != is_inf<S>(b)) return false;
    out = to;
    return true;
  } else {
    to = convert_rn<S, D>(b);
    const uint64_t back = convert_rn<D, S>(to);
    if (back != b || is_inf<D>(to) != is_inf<S>(b)) return false;
    out = to;
    return true;
  }
}

// sitofp / uitofp (canonicalize.rs:406-416): f32 results are the one
// rounding of Rust's `as f32`; other kinds round to f64 first (`as f64`)
// and then ApFloat::from_f64.
template <int W, bool SIGNED, class D> __device__ __forceinline__ uint64_t int_to_float(uint64_t v) {
  using I = IntW<W>;
  if constexpr (D::B == 4 && D::E == 8) {
    if constexpr (SIGNED) return __float_as_uint(__ll2float_rn((long long)I::sx(v)));
    else return __float_as_uint(__ull2float_rn((unsigned long long)(v & I::MASK)));
  } else {
    double x;
    if constexpr (SIGNED) x = __ll2double_rn((long long)I::sx(v));
    else x = __ull2double_rn((unsigned long long)(v & I::MASK));
    const uint64_t d = (uint64_t)__double_as_longlong(x);
    if constexpr (D::B == 8) return d;
    else return convert_rn<F64L, D>(d);
  }
}

// fptosi / fptoui (canonicalize.rs:422-433).  Returns false to refuse.
template <class S, int W, bool SIGNED> __device__ __forceinline__ bool float_to_int(uint64_t b, uint64_t& out) {
  if (is_nan<S>(b) || is_inf<S>(b)) return false;
  const double t = trunc(to_f64<S>(b));
  double lo, hi;
  if (SIGNED) {
    lo = -ldexp(1.0, W - 1);
    hi = ldexp(1.0, W - 1);
  } else {
    lo = 0.0;
    hi = ldexp(1.0, W);
  }
  if (t < lo || t >= hi) return false;
  uint64_t v;
  if (t >= 9223372036854775808.0) v = (uint64_t)__double2ull_rz(t);
  else v = (uint64_t)__double2ll_rz(t);
  out = v & IntW<W>::MASK;
  return true;
}

}  // namespace dcf
