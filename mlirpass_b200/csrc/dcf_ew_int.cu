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

// floor(x / d) for 0 <= x < 2^16 and 1 <= d < 2^16 on the FMA and integer
// pipes only: no division, no reciprocal unit and no int<->float conversion
// instruction (those run on the narrow transcendental / conversion unit,
// which limited the lane-wise 8-bit division).  The operands become floats
// exactly by the magic-number trick (2^23 + v has v as its low mantissa
// bits); the reciprocal starts from the exponent-negation seed of the fast
// inverse methods (e.g. C. Lomont, "Fast Inverse Square Root", 2003, whose
// reciprocal form is within 12.5% of 1/d) and takes STEPS Newton-Raphson
// steps r <- r + r (1 - d r), each squaring the relative error (2 steps:
// < 2.5e-4, enough for x < 2^8; 3 steps: < 1e-7 with f32 rounding, enough
// for x < 2^16), so x * r rounded to an integer is floor(x / d) or one more,
// and one integer correction makes it exact.
template <int STEPS>
__device__ __forceinline__ uint32_t udiv_small(uint32_t x, uint32_t d) {
  const float xf = __int_as_float(0x4B000000u | x) - 8388608.0f;
  const float df = __int_as_float(0x4B000000u | d) - 8388608.0f;
  float r = __int_as_float(0x7EF311C3 - __float_as_int(df));
#pragma unroll
  for (int i = 0; i < STEPS; i++) r = __fmaf_rn(r, __fmaf_rn(-df, r, 1.0f), r);
  uint32_t q = (uint32_t)__float_as_int(__fmaf_rn(xf, r, 8388608.0f)) - 0x4B000000u;
  if ((int32_t)(x - q * d) < 0) q--;
  return q;
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
  // gets some value, which is never used.  Quotients of 8- and 16-bit
  // lanes come from udiv_small on the magnitudes (truncating division of
  // signed lanes: the magnitude of the quotient, then its sign).
  __device__ static __forceinline__ uint32_t word_checked(uint32_t a, uint32_t b, uint32_t& o) {
    constexpr uint32_t M = (1u << W) - 1;
    uint32_t bad = 0;
    if constexpr (OP == DCF_SHLI || OP == DCF_SHRUI || OP == DCF_SHRSI)
      bad = W == 8 ? __vcmpgeu4(b, 0x08080808u) : __vcmpgeu2(b, 0x00100010u);
    if constexpr (OP == DCF_DIVSI || OP == DCF_DIVUI || OP == DCF_REMSI || OP == DCF_REMUI)
      bad = W == 8 ? __vcmpeq4(b, 0u) : __vcmpeq2(b, 0u);
    if constexpr (OP == DCF_DIVSI)
      bad |= W == 8 ? (__vcmpeq4(a, 0x80808080u) & __vcmpeq4(b, 0xFFFFFFFFu))
                    : (__vcmpeq2(a, 0x80008000u) & __vcmpeq2(b, 0xFFFFFFFFu));
    uint32_t r = 0;
#pragma unroll
    for (int k = 0; k < 32 / W; k++) {
      const uint32_t x = (a >> (W * k)) & M;
      uint32_t y = (b >> (W * k)) & M;
      if constexpr (OP == DCF_SHLI || OP == DCF_SHRUI || OP == DCF_SHRSI) y &= W - 1;
      if constexpr (OP == DCF_DIVSI || OP == DCF_DIVUI || OP == DCF_REMSI || OP == DCF_REMUI) y = y ? y : 1;
      const int32_t sx = (int32_t)(x << (32 - W)) >> (32 - W), sy = (int32_t)(y << (32 - W)) >> (32 - W);
      uint32_t z;
      if constexpr (OP == DCF_MULI) z = x * y;
      else if constexpr (OP == DCF_SHLI) z = x << y;
      else if constexpr (OP == DCF_SHRUI) z = x >> y;
      else if constexpr (OP == DCF_SHRSI) z = (uint32_t)(sx >> y);
      else if constexpr (OP == DCF_DIVUI || OP == DCF_REMUI) {
        const uint32_t q = udiv_small<W == 8 ? 2 : 3>(x, y);
        z = OP == DCF_DIVUI ? q : x - q * y;
      } else {
        const uint32_t ax = (uint32_t)(sx < 0 ? -sx : sx), ay = (uint32_t)(sy < 0 ? -sy : sy);
        const uint32_t qm = udiv_small<W == 8 ? 2 : 3>(ax, ay);
        const int32_t q = ((sx ^ sy) < 0) ? -(int32_t)qm : (int32_t)qm;
        z = (uint32_t)(OP == DCF_DIVSI ? q : sx - q * sy);
      }
      r |= (z & M) << (W * k);
    }
    o = r;
    return bad;
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
