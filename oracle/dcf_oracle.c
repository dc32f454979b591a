/*
 * dcf_oracle.c — CPU oracle (test infrastructure only; see dcf_oracle.h).
 *
 * A scalar restatement of mlirpass's dense-constant fold closures.  All
 * reference citations are paths inside the mlirpass repository.  Build with
 * -O2 -ffp-contract=off and without -ffast-math, so that `float` and
 * `double` arithmetic is single IEEE-754 round-to-nearest-even operations
 * (SSE on x86-64), as Rust's f32/f64 arithmetic is.
 *
 * Where the reference delegates to the un-vendored mlirformat crate:
 *   - ApFloat add/sub/mul/div: IEEE-754 round-to-nearest-even.  A NaN
 *     operand propagates quieted, the first NaN operand winning; an invalid
 *     operation gives the default quiet NaN (positive, as LLVM APFloat's
 *     makeNaN; negative under DCF_FLAG_NEG_DEFAULT_NAN).  This NaN rule is
 *     the one part not pinned by a reference golden vector.
 *   - ApFloat::convert / from_f64: round-to-nearest-even, overflow to inf.
 *   - Const::at / is_splat: a splat Const holds one value, at(i) returns it.
 */
#include "dcf_oracle.h"

#include <math.h>
#include <string.h>

/* ---------------------------------------------------------------- types */

typedef struct {
  int E, M, bytes;
} fl_t;

static int fl_of(int dtype, fl_t* f) {
  /* float_layout, src/patterns/arith/canonicalize.rs:36-48 */
  switch (dtype) {
    case DCF_F16: *f = (fl_t){5, 10, 2}; return 1;
    case DCF_BF16: *f = (fl_t){8, 7, 2}; return 1;
    case DCF_F32: *f = (fl_t){8, 23, 4}; return 1;
    case DCF_F64: *f = (fl_t){11, 52, 8}; return 1;
    case DCF_F8E5M2: *f = (fl_t){5, 2, 1}; return 1;
    case DCF_F8E4M3: *f = (fl_t){4, 3, 1}; return 1;
    case DCF_F8E3M4: *f = (fl_t){3, 4, 1}; return 1;
    default: return 0;
  }
}

static int int_width(int dtype) {
  switch (dtype) {
    case DCF_I1: return 1;
    case DCF_I8: return 8;
    case DCF_I16: return 16;
    case DCF_I32: return 32;
    case DCF_I64: return 64;
    default: return 0;
  }
}

static int elem_bytes(int dtype) {
  int w = int_width(dtype);
  if (w) return w == 1 ? 1 : w / 8;
  fl_t f;
  return fl_of(dtype, &f) ? f.bytes : 0;
}

static uint64_t load(const void* p, uint64_t i, int bytes) {
  const uint8_t* b = (const uint8_t*)p + i * (uint64_t)bytes;
  uint64_t v = 0;
  memcpy(&v, b, (size_t)bytes); /* little-endian host */
  return v;
}

static void store(void* p, uint64_t i, int bytes, uint64_t v) {
  memcpy((uint8_t*)p + i * (uint64_t)bytes, &v, (size_t)bytes);
}

static uint64_t wmask(int w) { return w >= 64 ? ~0ull : ((1ull << w) - 1); }

static int64_t sext(uint64_t v, int w) {
  if (w >= 64) return (int64_t)v;
  uint64_t m = 1ull << (w - 1);
  v &= wmask(w);
  return (int64_t)((v ^ m) - m);
}

/* ------------------------------------------------------- IEEE helpers */

static uint64_t f_maxexp(fl_t f) { return (1ull << f.E) - 1; }
static uint64_t f_mant(fl_t f, uint64_t b) { return b & ((1ull << f.M) - 1); }
static uint64_t f_expf(fl_t f, uint64_t b) { return (b >> f.M) & f_maxexp(f); }
static int f_sign(fl_t f, uint64_t b) { return (int)((b >> (f.E + f.M)) & 1); }
static int f_isnan(fl_t f, uint64_t b) { return f_expf(f, b) == f_maxexp(f) && f_mant(f, b) != 0; }
static int f_isinf(fl_t f, uint64_t b) { return f_expf(f, b) == f_maxexp(f) && f_mant(f, b) == 0; }
static int f_iszero(fl_t f, uint64_t b) { return (b & ((1ull << (f.E + f.M)) - 1)) == 0; }
static uint64_t f_quiet(fl_t f, uint64_t b) { return b | (1ull << (f.M - 1)); }
static uint64_t f_default_nan(fl_t f, uint32_t flags) {
  uint64_t s = (flags & DCF_FLAG_NEG_DEFAULT_NAN) ? (1ull << (f.E + f.M)) : 0;
  return s | (f_maxexp(f) << f.M) | (1ull << (f.M - 1));
}

/* value = sig * 2^exp, rounded to nearest-even into layout f; overflow
 * gives infinity (IEEE-754 default rounding). */
static uint64_t round_pack(int sign, uint64_t sig, int exp, fl_t f) {
  uint64_t sbit = (uint64_t)(sign & 1) << (f.E + f.M);
  if (sig == 0) return sbit;
  int bias = (1 << (f.E - 1)) - 1;
  int emin = 1 - bias;
  int p = 63 - __builtin_clzll(sig);
  int e = p + exp;
  int q = (e < emin) ? emin - f.M : e - f.M;
  int shift = q - exp;
  uint64_t r;
  if (shift <= 0) {
    r = sig << (-shift);
  } else if (shift > 64) {
    r = 0;
  } else if (shift == 64) {
    uint64_t half = 1ull << 63;
    r = (sig > half) ? 1 : 0;
  } else {
    uint64_t rem = sig & ((1ull << shift) - 1);
    uint64_t half = 1ull << (shift - 1);
    r = sig >> shift;
    if (rem > half || (rem == half && (r & 1))) r++;
  }
  uint64_t bits = (e < emin) ? r : (((uint64_t)(e + bias - 1) << f.M) + r);
  if ((bits >> f.M) >= f_maxexp(f)) bits = f_maxexp(f) << f.M;
  return sbit | bits;
}

/* finite value decode: value = sig * 2^exp (sig may be 0) */
static void f_decode(fl_t f, uint64_t b, uint64_t* sig, int* exp) {
  int bias = (1 << (f.E - 1)) - 1;
  uint64_t ef = f_expf(f, b), m = f_mant(f, b);
  if (ef == 0) {
    *sig = m;
    *exp = 1 - bias - f.M;
  } else {
    *sig = m | (1ull << f.M);
    *exp = (int)ef - bias - f.M;
  }
}

/* ApFloat::convert (mlirformat): round-to-nearest-even between layouts.
 * NaN inputs are handled by the callers (nan_convert). */
static uint64_t f_convert(fl_t from, fl_t to, uint64_t b) {
  int s = f_sign(from, b);
  if (f_isinf(from, b)) return ((uint64_t)s << (to.E + to.M)) | (f_maxexp(to) << to.M);
  uint64_t sig;
  int exp;
  f_decode(from, b, &sig, &exp);
  return round_pack(s, sig, exp, to);
}

static const fl_t F64L = {11, 52, 8};
static const fl_t F32L = {8, 23, 4};

static double f_to_double(fl_t f, uint64_t b) {
  uint64_t d = f_isnan(f, b) ? 0x7FF8000000000000ull : f_convert(f, F64L, b);
  if (f_isnan(f, b)) d |= (uint64_t)f_sign(f, b) << 63;
  double x;
  memcpy(&x, &d, 8);
  return x;
}

static uint64_t double_bits(double x) {
  uint64_t d;
  memcpy(&d, &x, 8);
  return d;
}

static float bits_float(uint32_t b) {
  float x;
  memcpy(&x, &b, 4);
  return x;
}

static uint32_t float_bits(float x) {
  uint32_t b;
  memcpy(&b, &x, 4);
  return b;
}

static double bits_double(uint64_t b) {
  double x;
  memcpy(&x, &b, 8);
  return x;
}

/* Rust f32::next_up / next_down (core::f32), and the f64 versions. */
static uint32_t f32_next(uint32_t b, int up) {
  float x = bits_float(b);
  if (isnan(x)) return b;
  if (up && b == 0x7F800000u) return b;
  if (!up && b == 0xFF800000u) return b;
  uint32_t abs = b & 0x7FFFFFFFu;
  if (abs == 0) return up ? 1u : 0x80000001u;
  if (b == abs) return up ? b + 1 : b - 1;
  return up ? b - 1 : b + 1;
}

static uint64_t f64_next(uint64_t b, int up) {
  double x = bits_double(b);
  if (isnan(x)) return b;
  if (up && b == 0x7FF0000000000000ull) return b;
  if (!up && b == 0xFFF0000000000000ull) return b;
  uint64_t abs = b & 0x7FFFFFFFFFFFFFFFull;
  if (abs == 0) return up ? 1ull : 0x8000000000000001ull;
  if (b == abs) return up ? b + 1 : b - 1;
  return up ? b - 1 : b + 1;
}

/* --------------------------------------------------- float arithmetic */

/* ApFloat::{add,sub,mul,div} at round-to-nearest-even (mlirformat; IEEE-754
 * semantics with the APFloat NaN rule described at the top of the file). */
static uint64_t ap_arith(int op, fl_t f, uint64_t a, uint64_t b, uint32_t flags) {
  if (f_isnan(f, a)) return f_quiet(f, a);
  if (f_isnan(f, b)) return f_quiet(f, b);
  uint64_t r;
  if (f.bytes == 4 && f.E == 8) {
    float x = bits_float((uint32_t)a), y = bits_float((uint32_t)b), z;
    switch (op) {
      case DCF_ADDF: z = x + y; break;
      case DCF_SUBF: z = x - y; break;
      case DCF_MULF: z = x * y; break;
      default: z = x / y; break;
    }
    r = float_bits(z);
  } else if (f.bytes == 8) {
    double x = bits_double(a), y = bits_double(b), z;
    switch (op) {
      case DCF_ADDF: z = x + y; break;
      case DCF_SUBF: z = x - y; break;
      case DCF_MULF: z = x * y; break;
      default: z = x / y; break;
    }
    r = double_bits(z);
  } else {
    /* Narrow kinds: the exact operands widened to f64, one f64 operation,
     * then one rounding to the narrow kind.  f64 has more than 2p+2 bits
     * of precision for every narrow kind, so the double rounding is
     * innocuous and this equals the correctly rounded narrow result. */
    double x = f_to_double(f, a), y = f_to_double(f, b), z;
    switch (op) {
      case DCF_ADDF: z = x + y; break;
      case DCF_SUBF: z = x - y; break;
      case DCF_MULF: z = x * y; break;
      default: z = x / y; break;
    }
    if (isnan(z)) return f_default_nan(f, flags);
    return f_convert(F64L, f, double_bits(z));
  }
  if (f_isnan(f, r)) return f_default_nan(f, flags);
  return r;
}

/* Rounded::apply, src/patterns/arith/canonicalize.rs:984-1055.
 * Returns 0 when the element refuses (None). */
static int rounded_apply(int op, fl_t f, uint64_t a, uint64_t b, int mode, uint32_t flags, uint64_t* out) {
  uint64_t nearest = ap_arith(op, f, a, b, flags);
  if (mode == 0 || f_isnan(f, nearest)) { /* :992-994 */
    *out = nearest;
    return 1;
  }
  double err;
  if (f.bytes == 8) { /* :997-1012 */
    double x = bits_double(a), y = bits_double(b), r = bits_double(nearest);
    if (isinf(r) && isfinite(x) && isfinite(y)) {
      err = -r;
    } else if (op == DCF_ADDF || op == DCF_SUBF) {
      if (op == DCF_SUBF) y = -y;
      double bb = r - x;
      err = (x - (r - bb)) + (y - bb);
    } else if (op == DCF_MULF) {
      err = fma(x, y, -r);
    } else {
      err = fma(-r, y, x) * copysign(1.0, y);
    }
  } else if (f.bytes == 4 && f.E == 8) { /* :1013-1029 */
    float x = bits_float((uint32_t)a), y = bits_float((uint32_t)b), r = bits_float((uint32_t)nearest);
    float e;
    if (isinf(r) && isfinite(x) && isfinite(y)) {
      e = -r;
    } else if (op == DCF_ADDF || op == DCF_SUBF) {
      if (op == DCF_SUBF) y = -y;
      float bb = r - x;
      e = (x - (r - bb)) + (y - bb);
    } else if (op == DCF_MULF) {
      e = fmaf(x, y, -r);
    } else {
      e = fmaf(-r, y, x) * copysignf(1.0f, y);
    }
    err = (double)e;
  } else { /* :1030 */
    return 0;
  }
  if (err == 0.0) { /* :1032-1034 */
    *out = nearest;
    return 1;
  }
  double r = (f.bytes == 8) ? bits_double(nearest) : (double)bits_float((uint32_t)nearest);
  int step = -1; /* -1: keep nearest, 0: down, 1: up */
  switch (mode) { /* :1046-1053 */
    case 1: if (err < 0.0) step = 0; break;
    case 2: if (err > 0.0) step = 1; break;
    case 3: if ((r > 0.0 && err < 0.0) || (r < 0.0 && err > 0.0)) step = (r < 0.0); break;
    case 4: return 0;
    default: break;
  }
  if (step < 0) {
    *out = nearest;
  } else if (f.bytes == 8) {
    *out = f64_next(nearest, step);
  } else {
    *out = f32_next((uint32_t)nearest, step);
  }
  return 1;
}

/* ApFloat::compare: partial order, None (-2) for unordered. */
static int ap_compare(fl_t f, uint64_t a, uint64_t b) {
  if (f_isnan(f, a) || f_isnan(f, b)) return -2;
  double x = f_to_double(f, a), y = f_to_double(f, b);
  return (x < y) ? -1 : (x > y) ? 1 : 0;
}

/* minmax, src/patterns/arith/canonicalize.rs:132-150 */
static uint64_t minmax(fl_t f, uint64_t a, uint64_t b, int max, int nan_wins) {
  int an = f_isnan(f, a), bn = f_isnan(f, b);
  if (an || bn) {
    if (nan_wins) return an ? f_quiet(f, a) : f_quiet(f, b);
    int sa = an && f_quiet(f, a) != a, sb = bn && f_quiet(f, b) != b;
    if (sa) return f_quiet(f, a);
    if (sb) return f_quiet(f, b);
    if (an) return b;
    return a;
  }
  if (f_iszero(f, a) && f_iszero(f, b) && f_sign(f, a) != f_sign(f, b))
    return (f_sign(f, a) == max) ? b : a;
  if (max) return ap_compare(f, a, b) == -1 ? b : a;
  return ap_compare(f, b, a) == -1 ? b : a;
}

/* cmpf, src/patterns/arith/canonicalize.rs:109-130 */
static int cmpf(int pred, fl_t f, uint64_t a, uint64_t b) {
  int c = ap_compare(f, a, b);
  int lt = c == -1, eq = c == 0, gt = c == 1, un = c == -2;
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

/* cmpi, src/patterns/arith/canonicalize.rs:94-107 */
static int cmpi(int pred, int w, uint64_t a, uint64_t b) {
  int64_t sa = sext(a, w), sb = sext(b, w);
  uint64_t ua = a & wmask(w), ub = b & wmask(w);
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

/* ApInt's overflow-reporting signed steps at width w: the wrapped result
 * and whether the exact result left [-2^(w-1), 2^(w-1)). */
static uint64_t s_wrap(__int128 x, int w, int* ov) {
  __int128 lo = -((__int128)1 << (w - 1)), hi = ((__int128)1 << (w - 1)) - 1;
  if (x < lo || x > hi) *ov = 1;
  return (uint64_t)x & wmask(w);
}

/* Folder::ceildivsi, src/patterns/arith/canonicalize.rs:557-595, step by
 * step: ssub_ov / sdiv_ov / sadd_ov, any overflow refuses the element. */
static int ceildivsi(int w, uint64_t ua, uint64_t ub, uint64_t* out) {
  if (ub == 0) return 0;
  if (ua == 0) { *out = 0; return 1; }
  int ov = 0;
  int64_t a = sext(ua, w), b = sext(ub, w);
  /* ceil(a, b) for the two-positive case: (a - 1) / b + 1 */
  #define CEIL_POS(x, y, res) do { \
      int64_t s_ = sext(s_wrap((__int128)(x) - 1, w, &ov), w); \
      int64_t q_; \
      if ((y) == 0) { q_ = s_; ov = 1; } \
      else { q_ = sext(s_wrap((__int128)s_ / (__int128)(y), w, &ov), w); } \
      (res) = sext(s_wrap((__int128)q_ + 1, w, &ov), w); } while (0)
  int64_t r;
  if (a > 0 && b > 0) {
    CEIL_POS(a, b, r);
  } else if (a <= 0 && b <= 0) {
    int64_t pa = sext(s_wrap(-(__int128)a, w, &ov), w);
    int64_t pb = sext(s_wrap(-(__int128)b, w, &ov), w);
    CEIL_POS(pa, pb, r);
  } else if (a <= 0) {
    int64_t pa = sext(s_wrap(-(__int128)a, w, &ov), w);
    int64_t d = sext(s_wrap((__int128)pa / (__int128)b, w, &ov), w);
    r = sext(s_wrap(-(__int128)d, w, &ov), w);
  } else {
    int64_t pb = sext(s_wrap(-(__int128)b, w, &ov), w);
    if (pb == 0) return 0;
    int64_t d = sext(s_wrap((__int128)a / (__int128)pb, w, &ov), w);
    r = sext(s_wrap(-(__int128)d, w, &ov), w);
  }
  #undef CEIL_POS
  if (ov) return 0;
  *out = (uint64_t)r & wmask(w);
  return 1;
}

/* Integer closures of ArithFolder::fold (wraparound ApInt arithmetic).
 * Returns 0 when the element refuses. */
static int int_op(int op, int w, uint64_t a, uint64_t b, uint64_t* out) {
  uint64_t m = wmask(w);
  uint64_t ua = a & m, ub = b & m;
  int64_t sa = sext(a, w), sb = sext(b, w);
  int64_t smin = (w >= 64) ? INT64_MIN : -(int64_t)(1ull << (w - 1));
  switch (op) {
    case DCF_ADDI: *out = (ua + ub) & m; return 1;             /* :507 */
    case DCF_SUBI: *out = (ua - ub) & m; return 1;             /* :535 */
    case DCF_MULI: *out = (ua * ub) & m; return 1;             /* :284 */
    case DCF_ANDI: *out = ua & ub; return 1;                   /* :619 */
    case DCF_ORI: *out = ua | ub; return 1;                    /* :639 */
    case DCF_XORI: *out = ua ^ ub; return 1;                   /* :660 */
    case DCF_SHLI:                                             /* :469-485 */
    case DCF_SHRUI:
    case DCF_SHRSI:
      if (ub >= (uint64_t)w) return 0;
      if (op == DCF_SHLI) *out = (ua << ub) & m;
      else if (op == DCF_SHRUI) *out = ua >> ub;
      else *out = ((uint64_t)(sa >> ub)) & m;
      return 1;
    case DCF_DIVSI:                                            /* :554, sdiv_ov */
      if (ub == 0) return 0;
      if (sa == smin && sb == -1) return 0;
      *out = ((uint64_t)(sa / sb)) & m;
      return 1;
    case DCF_DIVUI:                                            /* :554, udiv */
      if (ub == 0) return 0;
      *out = ua / ub;
      return 1;
    case DCF_REMSI:                                            /* :319-325, srem */
      if (ub == 0) return 0;
      *out = (sb == -1) ? 0 : (((uint64_t)(sa % sb)) & m);
      return 1;
    case DCF_REMUI:
      if (ub == 0) return 0;
      *out = ua % ub;
      return 1;
    case DCF_CEILDIVUI: {                                      /* :287-298 */
      if (ub == 0) return 0;
      uint64_t q = ua / ub;
      if (ua % ub == 0) { *out = q; return 1; }
      if (q == m) return 0;                                    /* uadd_ov */
      *out = q + 1;
      return 1;
    }
    case DCF_CEILDIVSI:                                        /* :557-595 */
      return ceildivsi(w, ua, ub, out);
    case DCF_FLOORDIVSI: {                                     /* :306-317 */
      if (ub == 0) return 0;
      if (sa == smin && sb == -1) return 0;                    /* sdiv_ov */
      int64_t q = sa / sb, r = sa % sb;
      if (r != 0 && ((r < 0) != (sb < 0))) q -= 1;
      *out = (uint64_t)q & m;
      return 1;
    }
    case DCF_MULSI_HI: {                                       /* :939-944 */
      __int128 p = (__int128)sa * (__int128)sb;
      *out = (uint64_t)(p >> w) & m;
      return 1;
    }
    case DCF_MULUI_HI: {
      unsigned __int128 p = (unsigned __int128)ua * (unsigned __int128)ub;
      *out = (uint64_t)(p >> w) & m;
      return 1;
    }
    case DCF_MAXSI: *out = (sa > sb) ? ua : ub; return 1;     /* :679-682 */
    case DCF_MAXUI: *out = (ua > ub) ? ua : ub; return 1;
    case DCF_MINSI: *out = (sa < sb) ? ua : ub; return 1;
    case DCF_MINUI: *out = (ua < ub) ? ua : ub; return 1;
    default: return 0;
  }
}

/* remf: `x % y` through ApFloat::binary (src/patterns/arith/canonicalize.rs:387),
 * Rust's remainder of truncating division.  It is exact, so the double
 * fmod of the exactly widened operands narrows back without rounding.
 * NaN operands and invalid cases follow the same rule as ap_arith. */
static uint64_t remf(fl_t f, uint64_t a, uint64_t b, uint32_t flags) {
  if (f_isnan(f, a)) return f_quiet(f, a);
  if (f_isnan(f, b)) return f_quiet(f, b);
  if (f_isinf(f, a) || f_iszero(f, b)) return f_default_nan(f, flags);
  if (f_isinf(f, b) || f_iszero(f, a)) return a;
  double x = f_to_double(f, a), y = f_to_double(f, b);
  return f_convert(F64L, f, double_bits(fmod(x, y)));
}

/* --------------------------------------------------------- array folds */

static void res_init(dcf_result* res) {
  if (!res) return;
  memset(res, 0, sizeof(*res));
  res->first_fail_index = UINT64_MAX;
}

static void res_finish(dcf_result* res, const void* out, int ob, uint64_t n) {
  if (!res) return;
  res->folded = 1;
  res->is_splat = (uint8_t)dco_splat_check(out, (size_t)ob, n);
}

/* IntFolds::ipowi (src/patterns/math/canonicalize.rs:95-124), with the i1
 * refusal of the math.ipowi closure (:163). */
static int ipowi(int w, uint64_t a, uint64_t b, uint64_t* out) {
  uint64_t m = wmask(w), base = a & m, p = b & m, result = 1;
  if (w == 1) return 0;
  if (p == 0) { *out = 1; return 1; }
  if (sext(p, w) < 0) {
    if (base == 0) return 0;
    if (base == 1) *out = 1;
    else if (base != m) *out = 0;
    else *out = (p & 1) ? m : 1;
    return 1;
  }
  for (;;) {
    if (p & 1) result = (result * base) & m;
    p >>= 1;
    if (p == 0) { *out = result; return 1; }
    base = (base * base) & m;
  }
}

/* Folder::binary loop, src/patterns/arith/canonicalize.rs:214-216:
 * (0..n).map(|i| f(l.at(i), r.at(i))).collect::<Option<Vec<_>>>() */
int dco_binary(int op, int dtype, const void* lhs, int lhs_splat,
               const void* rhs, int rhs_splat, uint64_t n, uint32_t flags,
               void* out, dcf_result* res) {
  res_init(res);
  int ib = elem_bytes(dtype);
  if (!ib) return DCF_EINVAL;
  int is_cmp = (op == DCF_CMPI || op == DCF_CMPF || op == DCF_ADDUI_CARRY);
  int ob = is_cmp ? 1 : ib;
  int w = int_width(dtype);
  fl_t f;
  int isf = fl_of(dtype, &f);
  int pred = (int)((flags & DCF_FLAG_PRED_MASK) >> DCF_FLAG_PRED_SHIFT);
  int mode = (int)(flags & DCF_FLAG_ROUND_MASK);
  int fop = (op >= DCF_ADDF && op <= DCF_REMF) || op == DCF_COPYSIGN;
  if ((fop || op == DCF_CMPF) && !isf) return DCF_EINVAL;
  if (!fop && op != DCF_CMPF && !w) return DCF_EINVAL;
  for (uint64_t i = 0; i < n; i++) {
    uint64_t a = load(lhs, lhs_splat ? 0 : i, ib);
    uint64_t b = load(rhs, rhs_splat ? 0 : i, ib);
    uint64_t r = 0;
    int ok = 1;
    switch (op) {
      case DCF_ADDF: case DCF_SUBF: case DCF_MULF: case DCF_DIVF:
        ok = rounded_apply(op, f, a, b, mode, flags, &r);
        break;
      case DCF_MAXIMUMF: r = minmax(f, a, b, 1, 1); break;
      case DCF_MINIMUMF: r = minmax(f, a, b, 0, 1); break;
      case DCF_MAXNUMF: r = minmax(f, a, b, 1, 0); break;
      case DCF_MINNUMF: r = minmax(f, a, b, 0, 0); break;
      case DCF_CMPF: r = (uint64_t)cmpf(pred, f, a, b); break;
      case DCF_CMPI: r = (uint64_t)cmpi(pred, w, a, b); break;
      case DCF_REMF: r = remf(f, a, b, flags); break;
      /* math.copysign (src/patterns/math/canonicalize.rs:153-156) */
      case DCF_COPYSIGN: {
        uint64_t sign = 1ull << (f.E + f.M);
        r = (f_sign(f, a) != f_sign(f, b)) ? a ^ sign : a;
        break;
      }
      case DCF_IPOWI: ok = ipowi(w, a, b, &r); break;
      case DCF_ADDUI_CARRY:                                    /* :887-891 */
        r = (uint64_t)((((a & wmask(w)) + (b & wmask(w))) & wmask(w)) < (a & wmask(w)));
        break;
      default: ok = int_op(op, w, a, b, &r); break;
    }
    if (!ok) {
      if (res) res->first_fail_index = i;
      return 0;
    }
    if (w == 1 && !is_cmp) r &= 1;
    store(out, i, ob, r);
  }
  res_finish(res, out, ob, n);
  return 0;
}

/* nan_convert, src/patterns/arith/canonicalize.rs:50-67 */
static int nan_convert(fl_t from, fl_t to, uint64_t b, uint64_t* out) {
  int ms = from.M, md = to.M, ed = to.E;
  uint64_t mant = b & ((1ull << ms) - 1);
  if (((mant >> (ms - 1)) & 1) == 0) return 0;
  if (md < ms) {
    int lost = ms - md;
    if (mant & ((1ull << lost) - 1)) return 0;
    mant >>= lost;
  } else {
    mant <<= (md - ms);
  }
  uint64_t sign = (uint64_t)f_sign(from, b) << (ed + md);
  *out = sign | (((1ull << ed) - 1) << md) | mant;
  return 1;
}

/* float_convert closure, src/patterns/arith/canonicalize.rs:730-741 */
static int float_convert(fl_t from, fl_t to, uint64_t b, uint64_t* out) {
  if (f_isnan(from, b)) return nan_convert(from, to, b, out);
  uint64_t t = f_convert(from, to, b);
  uint64_t back = f_convert(to, from, t);
  if (back != b || f_isinf(to, t) != f_isinf(from, b)) return 0;
  *out = t;
  return 1;
}

uint64_t dco_float_convert_bits(int from, int to, uint64_t bits, int* ok) {
  fl_t a, b;
  uint64_t r = 0;
  if (!fl_of(from, &a) || !fl_of(to, &b)) {
    *ok = 0;
    return 0;
  }
  *ok = float_convert(a, b, bits, &r);
  return r;
}

uint64_t dco_round_from_double(int to, double x) {
  fl_t f;
  if (!fl_of(to, &f)) return 0;
  uint64_t d = double_bits(x);
  if (isnan(x)) return f_default_nan(f, 0);
  return f_convert(F64L, f, d);
}

/* int -> float: the sitofp/uitofp closure, :406-416.  F32 results come
 * from Rust's `as f32` on the integer (one rounding); other kinds go through
 * `as f64` and then ApFloat::from_f64 (two roundings). */
static uint64_t int_to_float(int w, uint64_t v, int is_signed, int to_dtype, fl_t to) {
  int sign = 0;
  uint64_t mag;
  if (is_signed) {
    int64_t s = sext(v, w);
    sign = s < 0;
    mag = sign ? (uint64_t)0 - (uint64_t)s : (uint64_t)s;
  } else {
    mag = v & wmask(w);
  }
  if (to_dtype == DCF_F32) return round_pack(sign, mag, 0, F32L);
  uint64_t d = round_pack(sign, mag, 0, F64L);
  if (to_dtype == DCF_F64) return d;
  return f_convert(F64L, to, d);
}

/* float -> int: the fptosi/fptoui closure, :422-433.  Returns 0 to refuse. */
static int float_to_int(fl_t from, uint64_t b, int w, int is_signed, uint64_t* out) {
  if (f_isnan(from, b) || f_isinf(from, b)) return 0;
  double x = f_to_double(from, b);
  double t = trunc(x);
  double lo, hi;
  if (is_signed) {
    lo = -ldexp(1.0, w - 1);
    hi = ldexp(1.0, w - 1);
  } else {
    lo = 0.0;
    hi = ldexp(1.0, w);
  }
  if (t < lo || t >= hi) return 0;
  uint64_t v;
  if (t >= 9223372036854775808.0) v = (uint64_t)t;
  else v = (uint64_t)(int64_t)t;
  *out = v & wmask(w);
  return 1;
}

/* The exact unary math folds, ArithFolder::math
 * (src/patterns/math/canonicalize.rs:145-234). */
static int math_unary(int op, int dtype, fl_t f, int w, uint64_t a, uint64_t* out) {
  uint64_t sign = 1ull << (f.E + f.M);
  switch (op) {
    case DCF_ABSF: *out = f_sign(f, a) ? a ^ sign : a; return 1;   /* :150 */
    case DCF_CEIL: case DCF_FLOOR: case DCF_ROUNDEVEN: {            /* :151-153 */
      /* FloatFolds::integral (:87-92): NaN quieted, else libm
       * ceil / floor / rint of to_f64, back with from_f64 */
      double x, y;
      if (f_isnan(f, a)) { *out = f_quiet(f, a); return 1; }
      x = f_to_double(f, a);
      y = op == DCF_CEIL ? ceil(x) : op == DCF_FLOOR ? floor(x) : nearbyint(x);
      *out = f_convert(F64L, f, double_bits(y));
      return 1;
    }
    case DCF_ROUND: case DCF_TRUNC: case DCF_SQRT: case DCF_RSQRT: {
      /* the exact cmath functions (:47-51, :219-233) and rsqrt (:166-171):
       * f32 / f64 only; sqrt and rsqrt refuse a negative operand; a NaN of
       * the exact functions comes back quieted, and 1 / sqrt(NaN) is the
       * same quieted NaN */
      if (dtype != DCF_F32 && dtype != DCF_F64) return 0;
      if ((op == DCF_SQRT || op == DCF_RSQRT) && f_sign(f, a)) return 0;
      if (f_isnan(f, a)) { *out = f_quiet(f, a); return 1; }
      if (dtype == DCF_F32) {
        float x = bits_float((uint32_t)a), y;
        if (op == DCF_ROUND) y = roundf(x);
        else if (op == DCF_TRUNC) y = truncf(x);
        else if (op == DCF_SQRT) y = sqrtf(x);
        else y = 1.0f / sqrtf(x);
        *out = float_bits(y);
      } else {
        double x = bits_double(a), y;
        if (op == DCF_ROUND) y = round(x);
        else if (op == DCF_TRUNC) y = trunc(x);
        else if (op == DCF_SQRT) y = sqrt(x);
        else y = 1.0 / sqrt(x);
        *out = double_bits(y);
      }
      return 1;
    }
    /* ApInt neg / count_leading_zeros / count_trailing_zeros / popcount
     * (:157-160); the count of a zero is the width */
    case DCF_ABSI: *out = sext(a, w) < 0 ? (0 - a) & wmask(w) : a & wmask(w); return 1;
    case DCF_CTLZ: case DCF_CTTZ: case DCF_CTPOP: {
      uint64_t v = a & wmask(w), n = 0;
      int k;
      if (op == DCF_CTPOP) { for (k = 0; k < w; k++) n += (v >> k) & 1; }
      else if (op == DCF_CTLZ) { for (k = w - 1; k >= 0 && !((v >> k) & 1); k--) n++; }
      else { for (k = 0; k < w && !((v >> k) & 1); k++) n++; }
      *out = n;
      return 1;
    }
    default: return 0;
  }
}

/* Folder::unary -> Const::map with the conversion closures. */
int dco_convert(int op, int from, int to, const void* in, int in_splat,
                uint64_t n, uint32_t flags, void* out, dcf_result* res) {
  (void)flags;
  res_init(res);
  int ib = elem_bytes(from), ob = elem_bytes(to);
  if (!ib || !ob) return DCF_EINVAL;
  fl_t ff, tf;
  int fromf = fl_of(from, &ff), tof = fl_of(to, &tf);
  int wf = int_width(from), wt = int_width(to);
  switch (op) {
    case DCF_EXTF: case DCF_TRUNCF: if (!fromf || !tof) return DCF_EINVAL; break;
    case DCF_SITOFP: case DCF_UITOFP: if (!wf || !tof) return DCF_EINVAL; break;
    case DCF_FPTOSI: case DCF_FPTOUI: if (!fromf || !wt) return DCF_EINVAL; break;
    case DCF_NEGF: case DCF_FLUSH_DENORMALS: if (!fromf || from != to) return DCF_EINVAL; break;
    case DCF_EXTSI: case DCF_EXTUI: case DCF_TRUNCI: if (!wf || !wt) return DCF_EINVAL; break;
    case DCF_ABSF: case DCF_CEIL: case DCF_FLOOR: case DCF_ROUNDEVEN:
    case DCF_ROUND: case DCF_TRUNC: case DCF_SQRT: case DCF_RSQRT:
      if (!fromf || from != to) return DCF_EINVAL;
      break;
    case DCF_ABSI: case DCF_CTLZ: case DCF_CTTZ: case DCF_CTPOP:
      if (!wf || from != to) return DCF_EINVAL;
      break;
    default: return DCF_EINVAL;
  }
  for (uint64_t i = 0; i < n; i++) {
    uint64_t a = load(in, in_splat ? 0 : i, ib), r = 0;
    int ok = 1;
    switch (op) {
      case DCF_EXTF: case DCF_TRUNCF: ok = float_convert(ff, tf, a, &r); break;
      case DCF_SITOFP: r = int_to_float(wf, a, 1, to, tf); break;
      case DCF_UITOFP: r = int_to_float(wf, a, 0, to, tf); break;
      case DCF_FPTOSI: ok = float_to_int(ff, a, wt, 1, &r); break;
      case DCF_FPTOUI: ok = float_to_int(ff, a, wt, 0, &r); break;
      /* negf: ApFloat::neg, the sign flipped (:327-333) */
      case DCF_NEGF: r = a ^ (1ull << (ff.E + ff.M)); break;
      /* flush_denormal (:69-77) */
      case DCF_FLUSH_DENORMALS:
        r = (f_expf(ff, a) == 0 && f_mant(ff, a) != 0) ? ((uint64_t)f_sign(ff, a) << (ff.E + ff.M)) : a;
        break;
      /* ApInt sext / zext / trunc (:388-398, :685-706) */
      case DCF_EXTSI: r = (uint64_t)sext(a, wf) & wmask(wt); break;
      case DCF_EXTUI: case DCF_TRUNCI: r = a & wmask(wf) & wmask(wt); break;
      default: ok = math_unary(op, from, ff, wf, a, &r); break;
    }
    if (!ok) {
      if (res) res->first_fail_index = i;
      return 0;
    }
    store(out, i, ob, r);
  }
  res_finish(res, out, ob, n);
  return 0;
}

/* Folder::select on three dense constants (src/patterns/arith/canonicalize.rs:869-875):
 * out[i] = cond[i] != 0 ? t[i] : f[i]; a splat operand broadcasts. */
int dco_select(size_t elem_size, const uint8_t* cond, int cond_splat, const void* t, int t_splat,
               const void* f, int f_splat, uint64_t n, void* out, dcf_result* res) {
  res_init(res);
  int es = (int)elem_size;
  if (es != 1 && es != 2 && es != 4 && es != 8) return DCF_EINVAL;
  for (uint64_t i = 0; i < n; i++) {
    int c = cond[cond_splat ? 0 : i] != 0;
    uint64_t v = c ? load(t, t_splat ? 0 : i, es) : load(f, f_splat ? 0 : i, es);
    store(out, i, es, v);
  }
  res_finish(res, out, es, n);
  return 0;
}

/* tosa reciprocal: `one.div(f)` (src/patterns/tosa/canonicalize.rs:602) and
 * upstream MLIR's ReciprocalOp::calcOneElement (APFloat divide, nearest-even)
 * for the layerwise fold. */
int dco_reciprocal(int dtype, const void* in, int in_splat, uint64_t n,
                   uint32_t flags, void* out, dcf_result* res) {
  res_init(res);
  fl_t f;
  if (!fl_of(dtype, &f)) return DCF_EINVAL;
  uint64_t one = f_convert(F64L, f, double_bits(1.0));
  for (uint64_t i = 0; i < n; i++) {
    uint64_t a = load(in, in_splat ? 0 : i, f.bytes);
    store(out, i, f.bytes, ap_arith(DCF_DIVF, f, one, a, flags));
  }
  res_finish(res, out, f.bytes, n);
  return 0;
}

/* Dense permutation (upstream TOSA layerwise transpose fold): out has shape
 * in_shape[perms[i]], row-major. */
int dco_transpose(size_t es, int rank, const int64_t* in_shape,
                  const int64_t* perms, const void* in, void* out) {
  if (rank < 1 || rank > 16) return DCF_EINVAL;
  int64_t in_stride[16], out_shape[16], src_stride[16], idx[16];
  int64_t total = 1;
  for (int i = rank - 1; i >= 0; i--) {
    in_stride[i] = total;
    total *= in_shape[i];
  }
  for (int i = 0; i < rank; i++) {
    if (perms[i] < 0 || perms[i] >= rank) return DCF_EINVAL;
    out_shape[i] = in_shape[perms[i]];
    src_stride[i] = in_stride[perms[i]];
    idx[i] = 0;
  }
  if (total == 0) return 0;
  const uint8_t* src = (const uint8_t*)in;
  uint8_t* dst = (uint8_t*)out;
  int64_t off = 0;
  for (int64_t o = 0; o < total; o++) {
    memcpy(dst + (size_t)o * es, src + (size_t)off * es, es);
    for (int d = rank - 1; d >= 0; d--) {
      idx[d]++;
      off += src_stride[d];
      if (idx[d] < out_shape[d]) break;
      off -= src_stride[d] * out_shape[d];
      idx[d] = 0;
    }
  }
  return 0;
}

int dco_hex_encode(const void* in, uint64_t nbytes, char* out) {
  static const char digits[] = "0123456789ABCDEF";
  const uint8_t* b = (const uint8_t*)in;
  for (uint64_t i = 0; i < nbytes; i++) {
    out[2 * i] = digits[b[i] >> 4];
    out[2 * i + 1] = digits[b[i] & 15];
  }
  return 0;
}

static int hexval(char c) {
  if (c >= '0' && c <= '9') return c - '0';
  if (c >= 'A' && c <= 'F') return c - 'A' + 10;
  if (c >= 'a' && c <= 'f') return c - 'a' + 10;
  return -1;
}

int dco_hex_decode(const char* in, uint64_t nchars, void* out) {
  if (nchars & 1) return DCF_EPARSE;
  uint8_t* b = (uint8_t*)out;
  for (uint64_t i = 0; i < nchars / 2; i++) {
    int h = hexval(in[2 * i]), l = hexval(in[2 * i + 1]);
    if (h < 0 || l < 0) return DCF_EPARSE;
    b[i] = (uint8_t)(h * 16 + l);
  }
  return 0;
}

int dco_splat_check(const void* in, size_t es, uint64_t n) {
  const uint8_t* b = (const uint8_t*)in;
  for (uint64_t i = 1; i < n; i++)
    if (memcmp(b, b + i * es, es) != 0) return 0;
  return 1;
}

/* The 64-bit byte hash of dcf_hash_many_async (the documented formula):
 * sum over 8-byte little-endian words w_i (the last zero-padded) of
 * mix(w_i ^ i * 0x9E3779B97F4A7C15) plus mix(nbytes), mix being the
 * SplitMix64 finaliser. */
static uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

uint64_t dco_hash(const void* data, uint64_t nbytes) {
  const uint8_t* b = (const uint8_t*)data;
  uint64_t h = 0, nw = (nbytes + 7) / 8;
  for (uint64_t i = 0; i < nw; i++) {
    uint64_t w = 0;
    for (uint64_t k = 0; k < 8 && 8 * i + k < nbytes; k++) w |= (uint64_t)b[8 * i + k] << (8 * k);
    h += mix64(w ^ (i * 0x9E3779B97F4A7C15ull));
  }
  return h + mix64(nbytes);
}
