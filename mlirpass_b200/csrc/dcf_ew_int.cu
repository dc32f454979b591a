// dcf_ew_int.cu — integer binary folds (wraparound ApInt arithmetic, the
// refusing ops shli/shrui/shrsi, div / rem / ceildiv / floordiv, the high
// half of mul*_extended), dense cmpi and the carry of addui_extended.
#include "dcf_kernels.cuh"

namespace dcf {

// The ops that have a lane-wise form on packed 8- and 16-bit words (none
// of them refuses an element).
template <int OP, int W> constexpr bool word_op() {
  return (W == 8 || W == 16) && (OP == DCF_ADDI || OP == DCF_SUBI || OP == DCF_ANDI || OP == DCF_ORI ||
                                 OP == DCF_XORI || OP == DCF_MAXSI || OP == DCF_MAXUI || OP == DCF_MINSI ||
                                 OP == DCF_MINUI);
}

template <int OP, int W> constexpr bool checked_word_op() {
  return (W == 8 || W == 16) && (OP == DCF_MULI || OP == DCF_SHLI || OP == DCF_SHRUI || OP == DCF_SHRSI ||
                                 OP == DCF_DIVSI || OP == DCF_DIVUI || OP == DCF_REMSI || OP == DCF_REMUI);
}

// 1/d for an integer 1 <= d < 2^16 (as a float), as accurate as a lane
// division of width W needs (below).  The start is the exponent-negation
// seed of the fast inverse methods (e.g. C. Lomont, "Fast Inverse Square
// Root", 2003): r0 = bits(0x7EF311C3 - bits(d)), whose relative error
// e0 = 1 - d r0 is at most 0.0506 over these integers (up to 12.5% only
// for mantissas no integer below 2^16 has).  A Newton-Raphson step
// r <- r + r e (e = 1 - d r) squares the error and costs two FMAs; the
// cubic step r <- r + r (e + e^2) cubes it and costs three.
//   8-bit signed (|x| <= 2^7):     one Newton step, |e| < 2.6e-3
//   8-bit unsigned (x < 2^8):      one cubic step,  |e| < 1.3e-4
//   16-bit signed (|x| <= 2^15):   two Newton steps, |e| < 6.6e-6
//   16-bit unsigned (x < 2^16):    cubic + Newton,  |e| < 2e-7 (f32 rounding)
template <int W, bool kSigned>
__device__ __forceinline__ float lane_recip(float d) {
  float r = __int_as_float(0x7EF311C3 - __float_as_int(d));
  const float e = __fmaf_rn(-d, r, 1.0f);
  if constexpr (kSigned) {
    r = __fmaf_rn(r, e, r);
    if constexpr (W == 16) r = __fmaf_rn(r, __fmaf_rn(-d, r, 1.0f), r);
  } else {
    r = __fmaf_rn(r, __fmaf_rn(e, e, e), r);
    if constexpr (W == 16) r = __fmaf_rn(r, __fmaf_rn(-d, r, 1.0f), r);
  }
  return r;
}

// Quotients and remainders of all 8- or 16-bit lanes of a 32-bit word on
// the FMA pipe, with no division, reciprocal or int<->float conversion
// instruction (those run on the narrow conversion unit) and few integer
// instructions (the integer ALU pipe limited the lane-by-lane form).
//  - Each lane becomes an exact float by the magic-number trick: one byte
//    permutation puts the lane under the exponent of 2^23, so the float is
//    2^23 + v.  Signed lanes are biased by 2^(W-1) first (an xor on the
//    whole word) and unbiased in the same subtraction; unsigned dividends
//    come out as x + 1/2 from it.
//  - floor(|x| / |d|) = floor((|x| + 1/2) r) with r = lane_recip(|d|):
//    (|x| + 1/2) / |d| lies at least 1/(2|d|) away from every integer, and
//    the error (|x| + 1/2) e / |d| stays below that while
//    (|x| + 1/2) |e| < 1/2, which the accuracy of lane_recip gives for each
//    width.  One fma rounded toward zero onto the 2^23 grid takes the floor
//    exactly: no integer correction step.
//  - The remainder |x| - q |d| is exact in f32; truncating signed division
//    gives the quotient the sign of x d and the remainder the sign of x.
//  - Each result v lands in the low mantissa bits of v + 2^23 (+ 2^W for
//    signed lanes, whose v may be negative) and byte permutations pack the
//    lanes back.
// b must hold no zero lane.
template <int OP, int W>
__device__ __forceinline__ uint32_t div_lanes(uint32_t a, uint32_t b) {
  constexpr bool kSigned = OP == DCF_DIVSI || OP == DCF_REMSI;
  constexpr bool kRem = OP == DCF_REMSI || OP == DCF_REMUI;
  constexpr uint32_t kBias = kSigned ? (W == 8 ? 0x80808080u : 0x80008000u) : 0u;
  constexpr float kMagic = 8388608.0f;  // 2^23
  constexpr float kDOff = kMagic + (kSigned ? (float)(1u << (W - 1)) : 0.0f);
  constexpr float kXOff = kSigned ? kDOff : kMagic - 0.5f;
  constexpr float kWrap = kSigned ? kMagic + (float)(1u << W) : kMagic - 0.5f;
  a ^= kBias;
  b ^= kBias;
  uint32_t f[32 / W];
#pragma unroll
  for (int k = 0; k < 32 / W; k++) {
    const uint32_t sel = W == 8 ? (0x7440u | k) : (0x7400u | ((2u * k + 1) << 4) | (2u * k));
    const float x = __int_as_float(__byte_perm(a, 0x4B000000u, sel)) - kXOff;  // unsigned: x + 1/2
    const float d = __int_as_float(__byte_perm(b, 0x4B000000u, sel)) - kDOff;
    const float ad = kSigned ? fabsf(d) : d;
    const float xh = kSigned ? fabsf(x) + 0.5f : x;
    const float qm = __fmaf_rz(xh, lane_recip<W, kSigned>(ad), kMagic);  // 2^23 + floor(|x| / |d|)
    if constexpr (OP == DCF_DIVUI) {
      f[k] = __float_as_uint(qm);
    } else if constexpr (OP == DCF_REMUI) {
      f[k] = __float_as_uint(__fmaf_rn(-(qm - kMagic), ad, xh) + kWrap);
    } else {
      const float q = qm - kMagic;
      const float v = kRem ? copysignf(__fmaf_rn(-q, ad, fabsf(x)), x) : copysignf(q, x * d);
      f[k] = __float_as_uint(v + kWrap);
    }
  }
  if constexpr (W == 8)
    return __byte_perm(__byte_perm(f[0], f[1], 0x0040u), __byte_perm(f[2], f[3], 0x0040u), 0x5410u);
  else
    return __byte_perm(f[0], f[1], 0x5410u);
}

template <int OP, int W> struct IOp {
  using In = typename IntW<W>::T;
  using Out = typename IntW<W>::T;
  static constexpr bool kBinary = true;
  static constexpr bool kWord = word_op<OP, W>();
  static constexpr bool kWordChecked = checked_word_op<OP, W>();
  // Lane by lane in registers, with the refusals of all lanes found at
  // once (the returned mask): a shift amount of the width or more, a zero
  // divisor, and the signed minimum divided by -1; a refusing lane still
  // gets some value, which is never used.  Quotients and remainders come
  // from div_lanes on all lanes at once, a zero divisor lane replaced by 1.
  __device__ static __forceinline__ uint32_t word_checked(uint32_t a, uint32_t b, uint32_t& o) {
    constexpr uint32_t M = (1u << W) - 1;
    if constexpr (OP == DCF_DIVSI || OP == DCF_DIVUI || OP == DCF_REMSI || OP == DCF_REMUI) {
      const uint32_t zero = W == 8 ? __vcmpeq4(b, 0u) : __vcmpeq2(b, 0u);
      uint32_t bad = zero;
      if constexpr (OP == DCF_DIVSI)
        bad |= W == 8 ? (__vcmpeq4(a, 0x80808080u) & __vcmpeq4(b, 0xFFFFFFFFu))
                      : (__vcmpeq2(a, 0x80008000u) & __vcmpeq2(b, 0xFFFFFFFFu));
      o = div_lanes<OP, W>(a, b | (zero & (W == 8 ? 0x01010101u : 0x00010001u)));
      return bad;
    } else {
      uint32_t bad = 0;
      if constexpr (OP == DCF_SHLI || OP == DCF_SHRUI || OP == DCF_SHRSI)
        bad = W == 8 ? __vcmpgeu4(b, 0x08080808u) : __vcmpgeu2(b, 0x00100010u);
      uint32_t r = 0;
#pragma unroll
      for (int k = 0; k < 32 / W; k++) {
        const uint32_t x = (a >> (W * k)) & M;
        uint32_t y = (b >> (W * k)) & M;
        if constexpr (OP == DCF_SHLI || OP == DCF_SHRUI || OP == DCF_SHRSI) y &= W - 1;
        uint32_t z;
        if constexpr (OP == DCF_MULI) z = x * y;
        else if constexpr (OP == DCF_SHLI) z = x << y;
        else if constexpr (OP == DCF_SHRUI) z = x >> y;
        else z = (uint32_t)((int32_t)(x << (32 - W)) >> (32 - W) >> y);
        r |= (z & M) << (W * k);
      }
      o = r;
      return bad;
    }
  }
  __device__ static __forceinline__ uint32_t word(uint32_t a, uint32_t b) {
    if constexpr (OP == DCF_ANDI) return a & b;
    else if constexpr (OP == DCF_ORI) return a | b;
    else if constexpr (OP == DCF_XORI) return a ^ b;
    else if constexpr (W == 8) {
      if constexpr (OP == DCF_ADDI) return __vadd4(a, b);
      else if constexpr (OP == DCF_SUBI) return __vsub4(a, b);
      else if constexpr (OP == DCF_MAXSI) return __vmaxs4(a, b);
      else if constexpr (OP == DCF_MAXUI) return __vmaxu4(a, b);
      else if constexpr (OP == DCF_MINSI) return __vmins4(a, b);
      else return __vminu4(a, b);
    } else {
      if constexpr (OP == DCF_ADDI) return __vadd2(a, b);
      else if constexpr (OP == DCF_SUBI) return __vsub2(a, b);
      else if constexpr (OP == DCF_MAXSI) return __vmaxs2(a, b);
      else if constexpr (OP == DCF_MAXUI) return __vmaxu2(a, b);
      else if constexpr (OP == DCF_MINSI) return __vmins2(a, b);
      else return __vminu2(a, b);
    }
  }
  __device__ static __forceinline__ bool apply(In a, In b, uint32_t, Out& o) {
    uint64_t r = 0;
    const bool ok = int_op<OP, W>(a, b, r);
    o = (Out)r;
    return ok;
  }
};

template <int W> struct ICmp {
  using In = typename IntW<W>::T;
  using Out = uint8_t;
  static constexpr bool kBinary = true;
  __device__ static __forceinline__ bool apply(In a, In b, uint32_t flags, Out& o) {
    o = cmpi<W>((int)((flags & DCF_FLAG_PRED_MASK) >> DCF_FLAG_PRED_SHIFT), a, b);
    return true;
  }
};

template <int W> struct ICarry {
  using In = typename IntW<W>::T;
  using Out = uint8_t;
  static constexpr bool kBinary = true;
  __device__ static __forceinline__ bool apply(In a, In b, uint32_t, Out& o) {
    o = add_carry<W>(a, b);
    return true;
  }
};

// math.ipowi (IntFolds::ipowi, src/patterns/math/canonicalize.rs:95-124):
// the exponent is signed; a negative one gives 1 for base 1, +-1 for base
// -1 by its parity and 0 for any other base except 0, which refuses; a
// non-negative one is a wrapping power by squaring.  An i1 base refuses
// (:163).
template <int W> struct IPow {
  using I = IntW<W>;
  using In = typename I::T;
  using Out = typename I::T;
  static constexpr bool kBinary = true;
  __device__ static __forceinline__ bool apply(In a, In b, uint32_t, Out& o) {
    o = 0;
    if constexpr (W == 1) {
      return false;
    } else {
      const uint64_t base = (uint64_t)a & I::MASK, pw = (uint64_t)b & I::MASK;
      if (pw == 0) {
        o = 1;
        return true;
      }
      if (I::sx(pw) < 0) {
        if (base == 0) return false;
        o = (Out)(base == 1 ? 1 : base != I::MASK ? 0 : (pw & 1) ? I::MASK : 1);
        return true;
      }
      uint64_t r = 1, x = base, p = pw;
      for (;;) {
        if (p & 1) r = (r * x) & I::MASK;
        p >>= 1;
        if (!p) break;
        x = (x * x) & I::MASK;
      }
      o = (Out)r;
      return true;
    }
  }
};

template <int W> static int int_binary_for(const EwLaunch& a) {
  switch (a.op) {
    case DCF_ADDI: return launch_one<IOp<DCF_ADDI, W>>(a);
    case DCF_SUBI: return launch_one<IOp<DCF_SUBI, W>>(a);
    case DCF_MULI: return launch_one<IOp<DCF_MULI, W>>(a);
    case DCF_ANDI: return launch_one<IOp<DCF_ANDI, W>>(a);
    case DCF_ORI: return launch_one<IOp<DCF_ORI, W>>(a);
    case DCF_XORI: return launch_one<IOp<DCF_XORI, W>>(a);
    case DCF_SHLI: return launch_one<IOp<DCF_SHLI, W>>(a);
    case DCF_SHRUI: return launch_one<IOp<DCF_SHRUI, W>>(a);
    case DCF_SHRSI: return launch_one<IOp<DCF_SHRSI, W>>(a);
    case DCF_DIVSI: return launch_one<IOp<DCF_DIVSI, W>>(a);
    case DCF_DIVUI: return launch_one<IOp<DCF_DIVUI, W>>(a);
    case DCF_REMSI: return launch_one<IOp<DCF_REMSI, W>>(a);
    case DCF_REMUI: return launch_one<IOp<DCF_REMUI, W>>(a);
    case DCF_MAXSI: return launch_one<IOp<DCF_MAXSI, W>>(a);
    case DCF_MAXUI: return launch_one<IOp<DCF_MAXUI, W>>(a);
    case DCF_MINSI: return launch_one<IOp<DCF_MINSI, W>>(a);
    case DCF_MINUI: return launch_one<IOp<DCF_MINUI, W>>(a);
    case DCF_CEILDIVUI: return launch_one<IOp<DCF_CEILDIVUI, W>>(a);
    case DCF_CEILDIVSI: return launch_one<IOp<DCF_CEILDIVSI, W>>(a);
    case DCF_FLOORDIVSI: return launch_one<IOp<DCF_FLOORDIVSI, W>>(a);
    case DCF_MULSI_HI: return launch_one<IOp<DCF_MULSI_HI, W>>(a);
    case DCF_MULUI_HI: return launch_one<IOp<DCF_MULUI_HI, W>>(a);
    case DCF_CMPI: return launch_one<ICmp<W>>(a);
    case DCF_ADDUI_CARRY: return launch_one<ICarry<W>>(a);
    case DCF_IPOWI: return launch_one<IPow<W>>(a);
    default: return DCF_EUNSUPPORTED;
  }
}

int launch_int_binary(const EwLaunch& a) {
  switch (a.dtype) {
    case DCF_I1: return int_binary_for<1>(a);
    case DCF_I8: return int_binary_for<8>(a);
    case DCF_I16: return int_binary_for<16>(a);
    case DCF_I32: return int_binary_for<32>(a);
    case DCF_I64: return int_binary_for<64>(a);
    default: return DCF_EUNSUPPORTED;
  }
}

}  // namespace dcf
