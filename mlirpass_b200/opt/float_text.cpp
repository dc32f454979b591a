// float_text.cpp — the decimal text of a float element, as mlir-opt prints
// it (and so as mlirpass's printer must, since its output is compared with
// mlir-opt's byte for byte).
//
// MLIR's printer (AsmPrinter's float printing, llvm-project
// mlir/lib/IR/AsmPrinter.cpp, release 23.x) writes a finite value as:
//   1. APFloat::toString(precision 6, max padding 0, keep zeros): scientific
//      form with six significant digits, "d.dddddde±XX", if parsing that
//      text back into the value's type gives the same bits;
//   2. otherwise APFloat::toString() with its defaults (as many digits as
//      the type needs to round-trip, max padding 3, trailing zeros dropped),
//      if that text contains a '.';
//   3. otherwise, and for infinities and NaNs, the bit pattern as a "0x…"
//      hexadecimal literal.
// APFloat::toString (llvm/lib/Support/APFloat.cpp) is restated below from
// its published algorithm: the exact value N·2^e becomes N'·10^e by
// multiplying by 5^-e, digits beyond the requested precision are first cut
// by a floor division by a power of ten, the digit string is then rounded
// half up to the precision, and the digits are laid out in scientific or
// plain notation.  All steps are integer arithmetic on an arbitrary-size
// integer, so the text is exact for every element type.
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "ir.h"

namespace dco {

namespace {

// Unsigned integer of any size, 32-bit limbs, least significant first.
struct Big {
  std::vector<uint32_t> w;

  explicit Big(uint64_t v) {
    while (v) {
      w.push_back((uint32_t)v);
      v >>= 32;
    }
  }
  bool zero() const { return w.empty(); }
  void trim() {
    while (!w.empty() && w.back() == 0) w.pop_back();
  }
  unsigned bits() const {
    if (w.empty()) return 0;
    return 32 * (unsigned)(w.size() - 1) + (32 - (unsigned)__builtin_clz(w.back()));
  }
  void shl(unsigned k) {
    if (zero() || !k) return;
    const unsigned limbs = k / 32, r = k % 32;
    std::vector<uint32_t> o(w.size() + limbs + 1, 0);
    for (size_t i = 0; i < w.size(); i++) {
      const uint64_t v = (uint64_t)w[i] << r;
      o[i + limbs] |= (uint32_t)v;
      o[i + limbs + 1] |= (uint32_t)(v >> 32);
    }
    w.swap(o);
    trim();
  }
  void mul(uint32_t m) {
    uint64_t carry = 0;
    for (auto& x : w) {
      const uint64_t v = (uint64_t)x * m + carry;
      x = (uint32_t)v;
      carry = v >> 32;
    }
    if (carry) w.push_back((uint32_t)carry);
  }
  // Floor division by d; returns the remainder.
  uint32_t div(uint32_t d) {
    uint64_t rem = 0;
    for (size_t i = w.size(); i-- > 0;) {
      const uint64_t cur = (rem << 32) | w[i];
      w[i] = (uint32_t)(cur / d);
      rem = cur % d;
    }
    trim();
    return (uint32_t)rem;
  }
};

void mul_pow5(Big& b, unsigned k) {
  while (k >= 13) {  // 5^13 < 2^32
    b.mul(1220703125u);
    k -= 13;
  }
  uint32_t m = 1;
  while (k--) m *= 5;
  if (m != 1) b.mul(m);
}

void div_pow10(Big& b, unsigned k) {
  while (k >= 9) {
    b.div(1000000000u);
    k -= 9;
  }
  uint32_t d = 1;
  while (k--) d *= 10;
  if (d != 1) b.div(d);
}

// APFloat::toString of the finite nonzero value (-1)^neg · sig · 2^exp2,
// sig < 2^precision (the type's significand width including the leading
// bit).  format_precision 0 means the type's round-trip digit count.
std::string apfloat_text(bool neg, uint64_t sig, int exp2, unsigned precision, unsigned format_precision,
                         unsigned max_padding, bool truncate_zero) {
  std::string out;
  if (neg) out += '-';
  if (sig == 0) {
    if (!max_padding) {
      if (truncate_zero) out += "0.0E+0";
      else {
        out += "0.0";
        if (format_precision > 1) out.append(format_precision - 1, '0');
        out += "e+00";
      }
    } else {
      out += '0';
    }
    return out;
  }
  int exp = exp2;
  if (!format_precision) format_precision = 2 + precision * 59 / 196;
  // Drop trailing binary zeros.
  const int tz = __builtin_ctzll(sig);
  sig >>= tz;
  exp += tz;
  Big n(sig);
  // From a power of two to a power of ten.
  if (exp > 0) {
    n.shl((unsigned)exp);
    exp = 0;
  } else if (exp < 0) {
    mul_pow5(n, (unsigned)-exp);
  }
  // Cut the digits that lie well below the precision (floor division).
  {
    const unsigned bits = n.bits();
    const unsigned required = (format_precision * 196 + 58) / 59;
    if (bits > required) {
      const unsigned tens = (bits - required) * 59 / 196;
      if (tens) {
        exp += (int)tens;
        div_pow10(n, tens);
      }
    }
  }
  // Digits, least significant first, without trailing zeros.
  std::vector<char> buf;
  bool trailing = true;
  while (!n.zero()) {
    const uint32_t d = n.div(10);
    if (trailing && d == 0) exp++;
    else {
      buf.push_back((char)('0' + d));
      trailing = false;
    }
  }
  // Round half up to the precision (zeros that rounding exposes drop out).
  if (buf.size() > format_precision) {
    size_t first = buf.size() - format_precision;
    if (buf[first - 1] < '5') {
      while (first < buf.size() && buf[first] == '0') first++;
    } else {
      size_t i = first;
      for (; i < buf.size(); i++) {
        if (buf[i] == '9') first++;
        else {
          buf[i]++;
          break;
        }
      }
      if (first == buf.size()) {
        exp += (int)first;
        buf.assign(1, '1');
        first = 0;
        goto laid_out;
      }
    }
    exp += (int)first;
    buf.erase(buf.begin(), buf.begin() + (long)first);
  }
laid_out:
  const unsigned nd = (unsigned)buf.size();
  bool scientific;
  if (!max_padding) {
    scientific = true;
  } else if (exp >= 0) {
    scientific = (unsigned)exp > max_padding || nd + (unsigned)exp > format_precision;
  } else {
    const int msd = exp + (int)(nd - 1);
    scientific = msd < 0 && (unsigned)-msd > max_padding;
  }
  if (scientific) {
    exp += (int)(nd - 1);
    out += buf[nd - 1];
    out += '.';
    if (nd == 1 && truncate_zero) out += '0';
    else
      for (unsigned i = 1; i != nd; i++) out += buf[nd - 1 - i];
    if (!truncate_zero && format_precision > nd - 1) out.append(format_precision - nd + 1, '0');
    out += truncate_zero ? 'E' : 'e';
    out += exp >= 0 ? '+' : '-';
    std::string e = std::to_string(exp < 0 ? -exp : exp);
    if (!truncate_zero && e.size() < 2) e = "0" + e;
    out += e;
    return out;
  }
  if (exp >= 0) {
    for (unsigned i = 0; i != nd; i++) out += buf[nd - 1 - i];
    out.append((size_t)exp, '0');
    return out;
  }
  const int whole = exp + (int)nd;
  unsigned i = 0;
  if (whole > 0) {
    for (; i != (unsigned)whole; i++) out += buf[nd - 1 - i];
    out += '.';
  } else {
    out += "0.";
    out.append((size_t)-whole, '0');
  }
  for (; i != nd; i++) out += buf[nd - 1 - i];
  return out;
}

}  // namespace

std::string mlir_float_text(uint64_t bits, int E, int M, bool (*parse_back)(const std::string&, uint64_t*, void*),
                            void* ctx) {
  const uint64_t emask = (1ull << E) - 1, mmask = (1ull << M) - 1;
  const bool neg = (bits >> (E + M)) & 1;
  const uint64_t ef = (bits >> M) & emask, m = bits & mmask;
  if (ef != emask) {
    const int bias = (1 << (E - 1)) - 1;
    const uint64_t sig = ef ? (m | (1ull << M)) : m;
    const int exp2 = (ef ? (int)ef : 1) - bias - M;
    const unsigned precision = (unsigned)M + 1;
    std::string s = apfloat_text(neg, sig, exp2, precision, 6, 0, false);
    uint64_t back = 0;
    if (parse_back(s, &back, ctx) && back == bits) return s;
    s = apfloat_text(neg, sig, exp2, precision, 0, 3, true);
    if (s.find('.') != std::string::npos) return s;
  }
  // The bit pattern, as APInt prints a C hex literal (no leading zeros).
  char buf[40];
  snprintf(buf, sizeof buf, "0x%llX", (unsigned long long)bits);
  return buf;
}

}  // namespace dco
