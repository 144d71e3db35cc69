// Decimal text -> binary32 for the CSV ingest, host and device.
//
// parse_feature_token() accepts exactly the tokens the reference's CSV feature
// parser accepts (native/decision_programs_csv.hpp:28-34): after trimming
// white space, an empty token or "nan" / "na" / "null" in any case is NaN; one
// leading '+' is dropped; the rest must be a whole decimal number in the
// std::from_chars general format ([-] digits [. digits] [e|E [+|-] digits],
// at least one mantissa digit), whose value rounds to a finite binary32.  As
// std::from_chars does, a non-zero value that rounds to zero or to infinity
// is refused.
//
// Rounding is to nearest, ties to even, for any number of digits:
//  * D < 2^24 and |E| <= 10 (value D x 10^E): one IEEE single-precision
//    multiplication or division of exact operands (Clinger 1990);
//  * otherwise the first 19 significant digits times the correctly rounded
//    binary64 10^E give an approximation within 2^-51 relative; rounding it
//    to binary32 is final unless it lies that close to the midpoint between
//    two binary32 neighbours;
//  * in that case the decimal value (its first 120 significant digits and
//    whether any later digit is non-zero) is compared exactly with the
//    midpoint in fixed-size integer arithmetic.  A binary32 midpoint has at
//    most 112 significant decimal digits, so 120 digits plus the sticky flag
//    decide the comparison exactly.
#pragma once
#include <cstdint>

#include "dp_math.cuh"

namespace dp {
namespace dec {

#ifdef __CUDA_ARCH__
__constant__ unsigned long long kPow10Bits[] = {
#include "pow10_table.inc"
};
#else
static const unsigned long long kPow10Bits[] = {
#include "pow10_table.inc"
};
#endif
constexpr int kPow10Min = -64, kPow10Max = 38;

DP_HD double pow10_bits(int k) {
  union {
    unsigned long long u;
    double d;
  } c;
  c.u = kPow10Bits[k - kPow10Min];
  return c.d;
}

DP_HD std::uint32_t f32_bits(float f) {
  union {
    float f;
    std::uint32_t u;
  } c;
  c.f = f;
  return c.u;
}
DP_HD float bits_f32(std::uint32_t u) {
  union {
    std::uint32_t u;
    float f;
  } c;
  c.u = u;
  return c.f;
}

// Non-negative integer in 32-bit limbs, little endian, fixed capacity.
struct Big {
  static constexpr int kLimbs = 24;
  std::uint32_t w[kLimbs];
  int n;
};

DP_HD void big_zero(Big& b) {
  for (int i = 0; i < Big::kLimbs; ++i) b.w[i] = 0;
  b.n = 0;
}
DP_HD void big_mul_add(Big& b, std::uint32_t m, std::uint32_t a) {
  std::uint64_t carry = a;
  for (int i = 0; i < b.n; ++i) {
    const std::uint64_t t = std::uint64_t(b.w[i]) * m + carry;
    b.w[i] = std::uint32_t(t);
    carry = t >> 32;
  }
  if (carry && b.n < Big::kLimbs) b.w[b.n++] = std::uint32_t(carry);
}
DP_HD void big_mul_pow10(Big& b, int k) {
  while (k >= 9) {
    big_mul_add(b, 1000000000u, 0);
    k -= 9;
  }
  std::uint32_t m = 1;
  while (k-- > 0) m *= 10u;
  if (m != 1) big_mul_add(b, m, 0);
}
DP_HD void big_shl(Big& b, int bits) {
  if (b.n == 0 || bits <= 0) return;
  const int limbs = bits / 32, r = bits % 32;
  int n = b.n + limbs + 1;
  if (n > Big::kLimbs) n = Big::kLimbs;
  for (int i = n - 1; i >= 0; --i) {
    const int s = i - limbs;
    std::uint32_t v = 0;
    if (s >= 0 && s < b.n) v = b.w[s] << r;
    if (r && s - 1 >= 0 && s - 1 < b.n) v |= b.w[s - 1] >> (32 - r);
    b.w[i] = v;
  }
  b.n = n;
  while (b.n > 0 && b.w[b.n - 1] == 0) --b.n;
}
DP_HD int big_cmp(const Big& a, const Big& b) {
  if (a.n != b.n) return a.n < b.n ? -1 : 1;
  for (int i = a.n - 1; i >= 0; --i)
    if (a.w[i] != b.w[i]) return a.w[i] < b.w[i] ? -1 : 1;
  return 0;
}

DP_HD bool is_space(unsigned char c) { return c == ' ' || c == '\t' || c == '\n' || c == '\v' || c == '\f' || c == '\r'; }
DP_HD unsigned char lower(unsigned char c) { return (c >= 'A' && c <= 'Z') ? c + 32 : c; }
DP_HD bool is_digit(unsigned char c) { return c >= '0' && c <= '9'; }

// Exact comparison of the decimal value (digits `dg[0..nd)` after skipping
// leading zeros, value = D x 10^e10, `sticky` when digits beyond nd were
// dropped and non-zero) with the binary32 midpoint mid2 x 2^(k2 - 1) (mid2
// odd).  Returns -1, 0, +1.
DP_HD int cmp_midpoint(const unsigned char* dg, int nd, int e10, bool sticky, std::uint32_t mid2, int k2) {
  Big lhs, rhs;
  big_zero(lhs);
  for (int i = 0; i < nd; ++i) big_mul_add(lhs, 10u, std::uint32_t(dg[i] - '0'));
  big_zero(rhs);
  big_mul_add(rhs, 1u, mid2);  // rhs = mid2 (n becomes 1)
  const int k = k2 - 1;        // midpoint = mid2 x 2^k
  if (e10 >= 0) big_mul_pow10(lhs, e10);
  else big_mul_pow10(rhs, -e10);
  if (k >= 0) big_shl(rhs, k);
  else big_shl(lhs, -k);
  const int c = big_cmp(lhs, rhs);
  if (c == 0 && sticky) return 1;
  return c;
}

// Rounds |value| = D x 10^e10 (D given by its significant digits) to binary32.
// Returns the bits, 0x7f800000 for overflow; 0 for a value that rounds to 0.
DP_HD std::uint32_t round_decimal(const unsigned char* dg, int nd, int e10, bool sticky) {
  // decimal order of magnitude: value in [10^(mag), 10^(mag + 1))
  const int mag = e10 + nd - 1;
  if (mag > 38) return 0x7f800000u;
  if (mag < -46) return 0u;
  // first 19 digits
  std::uint64_t d19 = 0;
  const int n19 = nd < 19 ? nd : 19;
  for (int i = 0; i < n19; ++i) d19 = d19 * 10u + std::uint64_t(dg[i] - '0');
  const int e19 = e10 + (nd - n19);
  if (nd == n19 && !sticky && d19 < (std::uint64_t(1) << 24) && e19 >= -10 && e19 <= 10) {
    // Clinger's exact case in single precision
    const float fd = float(std::uint32_t(d19));
    const float p = float(pow10_bits(e19 < 0 ? -e19 : e19));  // 10^k, k <= 10: exact in binary32
    return f32_bits(e19 < 0 ? fd / p : fd * p);
  }
  const double approx = double(d19) * pow10_bits(e19);
  const float c = float(approx);  // binary32 nearest to the approximation
  const std::uint32_t cb = f32_bits(c);
  const double tol = approx * 0x1p-50;   // above the approximation's error bound
  const double kTopMid = 0x1.ffffffp+127;  // midpoint of FLT_MAX and 2^128
  std::uint32_t base;                      // the nearby midpoint lies between base and base + 1
  if (cb == 0x7f800000u) {
    if (!(approx - kTopMid <= tol)) return cb;
    base = 0x7f7fffffu;
  } else {
    // the midpoints around c, exact in binary64
    const double cv = double(c);
    const double hi_mid = cb == 0x7f7fffffu ? kTopMid : (cv + double(bits_f32(cb + 1))) * 0.5;
    const bool near_hi = hi_mid - approx <= tol;
    bool near_lo = false;
    if (cb != 0) {
      const double lo_mid = (double(bits_f32(cb - 1)) + cv) * 0.5;
      near_lo = approx - lo_mid <= tol;
    }
    if (!near_lo && !near_hi) return cb;
    base = near_hi ? cb : cb - 1;
  }
  std::uint32_t mant, mid2;
  int k2;
  const std::uint32_t ex = base >> 23;
  if (ex == 0) {  // subnormal base (or zero): value = mant x 2^-149
    mant = base & 0x7fffffu;
    k2 = -149;
  } else {
    mant = (base & 0x7fffffu) | 0x800000u;
    k2 = int(ex) - 150;
  }
  mid2 = 2 * mant + 1;  // midpoint = mid2 x 2^(k2 - 1)
  const int c2 = cmp_midpoint(dg, nd, e10, sticky, mid2, k2);
  if (c2 < 0) return base;
  if (c2 > 0) return base + 1;
  return (base & 1u) ? base + 1 : base;  // tie: even
}

// The reference's feature(): see the file comment.  `p[0..n)` is the field's
// content (quotes removed); returns false when the token is refused.
DP_HD bool parse_feature_token(const unsigned char* p, std::uint32_t n, float* out) {
  std::uint32_t b = 0, e = n;
  while (b < e && is_space(p[b])) ++b;
  while (e > b && is_space(p[e - 1])) --e;
  const std::uint32_t len = e - b;
  // NaN tokens
  if (len == 0) {
    *out = bits_f32(0x7fc00000u);
    return true;
  }
  if (len <= 4) {
    unsigned char l[4] = {0, 0, 0, 0};
    for (std::uint32_t i = 0; i < len; ++i) l[i] = lower(p[b + i]);
    const bool nan3 = len == 3 && l[0] == 'n' && l[1] == 'a' && l[2] == 'n';
    const bool na2 = len == 2 && l[0] == 'n' && l[1] == 'a';
    const bool null4 = len == 4 && l[0] == 'n' && l[1] == 'u' && l[2] == 'l' && l[3] == 'l';
    if (nan3 || na2 || null4) {
      *out = bits_f32(0x7fc00000u);
      return true;
    }
  }
  std::uint32_t i = b;
  if (p[i] == '+') ++i;
  if (i >= e) return false;
  bool neg = false;
  if (p[i] == '-') {
    neg = true;
    ++i;
  }
  // mantissa: significant digits (first 120 kept) and the decimal point
  constexpr int kKeep = 120;
  unsigned char dg[kKeep];
  int nd = 0, mant_digits = 0;
  long long e10 = 0;  // value = 0.dg... scaled below
  bool sticky = false, seen_nonzero = false;
  long long dropped = 0;   // significant digits after the kept ones
  long long frac_sig = 0;  // significant digits that came after the point
  bool point = false;
  long long lead_frac_zeros = 0;  // zeros after the point before the first significant digit
  for (; i < e; ++i) {
    const unsigned char c = p[i];
    if (is_digit(c)) {
      ++mant_digits;
      if (!seen_nonzero && c == '0') {
        if (point) ++lead_frac_zeros;
        continue;
      }
      seen_nonzero = true;
      if (point) ++frac_sig;
      if (nd < kKeep) {
        dg[nd++] = c;
      } else {
        ++dropped;
        if (c != '0') sticky = true;
      }
    } else if (c == '.' && !point) {
      point = true;
    } else {
      break;
    }
  }
  if (mant_digits == 0) return false;
  long long ex = 0;
  if (i < e && (p[i] == 'e' || p[i] == 'E')) {
    std::uint32_t j = i + 1;
    bool eneg = false;
    if (j < e && (p[j] == '+' || p[j] == '-')) {
      eneg = p[j] == '-';
      ++j;
    }
    if (j >= e || !is_digit(p[j])) return false;  // "1e", "1e+": the parse stops before 'e'
    for (; j < e && is_digit(p[j]); ++j)
      if (ex < 100000000) ex = ex * 10 + (p[j] - '0');
    if (eneg) ex = -ex;
    i = j;
  }
  if (i != e) return false;
  if (!seen_nonzero) {
    *out = neg ? bits_f32(0x80000000u) : 0.0f;
    return true;
  }
  // drop trailing zeros of the kept digits (exactness is unaffected)
  long long tz = 0;
  while (nd > 1 && dg[nd - 1] == '0') {
    --nd;
    ++tz;
  }
  // value = D x 10^(ex + dropped + tz - frac_sig - lead_frac_zeros) where D = dg
  e10 = ex + dropped + tz - frac_sig - lead_frac_zeros;
  if (e10 > 100000) e10 = 100000;
  if (e10 < -100000) e10 = -100000;
  std::uint32_t bits = round_decimal(dg, nd, int(e10), sticky);
  if (bits == 0u || bits >= 0x7f800000u) return false;  // rounds to zero or infinity
  if (neg) bits |= 0x80000000u;
  *out = bits_f32(bits);
  return true;
}

// The reference's numeric class label: std::from_chars into uint32 over the
// trimmed token, consuming it whole (digits only, no sign).  Returns false
// when the token is not such a number (empty, other characters, > 2^32 - 1).
DP_HD bool parse_label_token(const unsigned char* p, std::uint32_t n, std::uint32_t* out) {
  std::uint32_t b = 0, e = n;
  while (b < e && is_space(p[b])) ++b;
  while (e > b && is_space(p[e - 1])) --e;
  if (b == e) return false;
  std::uint64_t v = 0;
  for (std::uint32_t i = b; i < e; ++i) {
    if (!is_digit(p[i])) return false;
    v = v * 10u + std::uint64_t(p[i] - '0');
    if (v > 0xffffffffull) return false;
  }
  *out = std::uint32_t(v);
  return true;
}

}  // namespace dec
}  // namespace dp
