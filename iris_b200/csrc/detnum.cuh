// Exact Q16.16 / Q32.32 / Q8_0 integer arithmetic for the B200 kernels.
//
// Every function reproduces a det-num rounding or saturation rule bit for bit
// (crates/det-num/src/{ops.rs,q8.rs,mistral.rs}); each cites the rule it
// implements. They are written for the GPU: 64-bit integer operations, 32x32
// and 64x64 multiplies with explicit high halves, divisions only by constants
// or once per row/head, and no 128-bit division. The same source compiles as
// host C++ (IRIS_HD expands to `inline`), which is how the host side of the
// library precomputes tables and how the CPU tests check these functions
// against the oracle without a GPU.
#pragma once
#include <math.h>
#include <stdint.h>

#if defined(__CUDACC__)
#define IRIS_HD __host__ __device__ __forceinline__
#else
#define IRIS_HD inline
#endif

namespace iris {

static constexpr int32_t kOneAct = 1 << 16;
static constexpr int64_t kOneAcc = (int64_t)1 << 32;

IRIS_HD int32_t clamp_i32(int64_t v) {
  return v < (int64_t)INT32_MIN ? INT32_MIN : (v > (int64_t)INT32_MAX ? INT32_MAX : (int32_t)v);
}
IRIS_HD int64_t sat_neg64(int64_t v) { return v == INT64_MIN ? INT64_MAX : -v; }
IRIS_HD int32_t sat_neg32(int32_t v) { return v == INT32_MIN ? INT32_MAX : -v; }

// High 64 bits of a signed / unsigned 64x64 product.
IRIS_HD int64_t mulhi_s64(int64_t a, int64_t b) {
#if defined(__CUDA_ARCH__)
  return __mul64hi(a, b);
#else
  return (int64_t)(((__int128)a * (__int128)b) >> 64);
#endif
}
IRIS_HD uint64_t mulhi_u64(uint64_t a, uint64_t b) {
#if defined(__CUDA_ARCH__)
  return __umul64hi(a, b);
#else
  return (uint64_t)(((unsigned __int128)a * (unsigned __int128)b) >> 64);
#endif
}

// x / 2^s rounded to nearest, ties to even, for 1 <= s <= 62. Matches
// rshift_round_ties_even_bits (ops.rs:773-803) and shift_round_ties_even
// (mistral.rs:23-32): both are round-half-even of the exact quotient.
IRIS_HD int64_t shift_round_even(int64_t x, int s) {
  int64_t f = x >> s;  // floor
  int64_t r = (int64_t)((uint64_t)x & (((uint64_t)1 << s) - 1));
  int64_t half = (int64_t)1 << (s - 1);
  return f + ((r > half) | ((r == half) & (f & 1)));
}

// ops.rs:448-451 requantize: Q32.32 -> Q16.16, ties to even, saturated.
IRIS_HD int32_t requantize(int64_t x) { return clamp_i32(shift_round_even(x, 16)); }
// ops.rs:41-45 mul_sat. |a b| <= 2^62, so x + 2^15 cannot overflow and the
// ties-to-even rounding is one addition: with f = floor(x / 2^16) and
// r = x - 2^16 f, (x + 2^15 - 1 + (f & 1)) >> 16 = f + [r + 2^15 - 1 + (f & 1)
// >= 2^16], i.e. f + 1 exactly when r > 2^15, or r = 2^15 and f is odd.
IRIS_HD int32_t mul_sat(int32_t a, int32_t b) {
  const int64_t x = (int64_t)a * (int64_t)b;
  return clamp_i32((x + 0x7FFF + ((x >> 16) & 1)) >> 16);
}
// ops.rs:36-38 add_sat, ops.rs:431-433 sub_sat (i32 saturating)
IRIS_HD int32_t add_sat(int32_t a, int32_t b) { return clamp_i32((int64_t)a + (int64_t)b); }
IRIS_HD int32_t sub_sat(int32_t a, int32_t b) { return clamp_i32((int64_t)a - (int64_t)b); }
// ops.rs:436-438 acc_add_sat for operands of any sign
IRIS_HD int64_t acc_add_sat(int64_t a, int64_t b) {
  uint64_t s = (uint64_t)a + (uint64_t)b;
  int64_t r = (int64_t)s;
  // overflow iff a and b share a sign that r does not
  if (((a ^ r) & (b ^ r)) < 0) return a < 0 ? INT64_MIN : INT64_MAX;
  return r;
}
// Saturating add of two non-negative accumulators. For non-negative terms the
// saturating sum is min(exact sum, i64::MAX) in any order, so partial sums of
// a row may be combined in any order.
IRIS_HD uint64_t add_sat_nonneg(uint64_t a, uint64_t b) {
  uint64_t s = a + b;
  return s > (uint64_t)INT64_MAX ? (uint64_t)INT64_MAX : s;
}

// Round-half-even quotient n / d for n >= 0, d > 0 (round_ties_even_division,
// ops.rs:691-720, on the non-negative domain).
IRIS_HD uint64_t div_round_even_u64(uint64_t n, uint64_t d) {
  uint64_t q = n / d, r = n - q * d;
  uint64_t other = d - r;  // distance to the next multiple
  if (r > other) return q + 1;
  if (r == other) return q + (q & 1);
  return q;
}
// Round-half-even quotient for signed n and d != 0 (ops.rs:691-720).
IRIS_HD int64_t div_round_even_s64(int64_t n, int64_t d) {
  bool neg = (n < 0) != (d < 0);
  uint64_t un = n < 0 ? (uint64_t)0 - (uint64_t)n : (uint64_t)n;
  uint64_t ud = d < 0 ? (uint64_t)0 - (uint64_t)d : (uint64_t)d;
  uint64_t q = div_round_even_u64(un, ud);
  return neg ? -(int64_t)q : (int64_t)q;
}

// ops.rs:53-64 div_act: (n << 16) / d, ties to even, saturated to i32. The
// magnitudes are below 2^48 and 2^32, exact in double precision, so the
// correctly rounded double quotient is within one of floor(|n 2^16| / |d|);
// one integer correction makes it exact, then the remainder rounds it (ties
// to even) as div_round_even_s64 does.
IRIS_HD int32_t div_act(int32_t n, int32_t d) {
  if (d == 0) return clamp_i32(div_round_even_s64((int64_t)n * 65536, (int64_t)d));
  const int64_t num = (int64_t)n * 65536;
  const bool neg = (num < 0) != (d < 0);
  const uint64_t un = num < 0 ? (uint64_t)0 - (uint64_t)num : (uint64_t)num;
  const uint64_t ud = d < 0 ? (uint64_t)0 - (uint64_t)(int64_t)d : (uint64_t)d;
  uint64_t q = (uint64_t)((double)un / (double)ud);
  int64_t r = (int64_t)(un - q * ud);
  if (r < 0) {
    --q;
    r += (int64_t)ud;
  } else if ((uint64_t)r >= ud) {
    ++q;
    r -= (int64_t)ud;
  }
  const uint64_t other = ud - (uint64_t)r;  // distance to the next multiple
  if ((uint64_t)r > other) ++q;
  else if ((uint64_t)r == other) q += q & 1;
  return clamp_i32(neg ? -(int64_t)q : (int64_t)q);
}

// ops.rs:685-689 acc_mul for non-negative operands whose product is below
// 2^95 (all uses on the hot path: softmax remainders, sine/cosine powers).
IRIS_HD int64_t acc_mul_nonneg(int64_t a, int64_t b) {
  uint64_t lo = (uint64_t)a * (uint64_t)b;
  uint64_t hi = mulhi_u64((uint64_t)a, (uint64_t)b);
  uint64_t f = (lo >> 32) | (hi << 32);
  uint64_t r = lo & 0xFFFFFFFFull;
  f += (r > 0x80000000ull) | ((r == 0x80000000ull) & (f & 1));
  return (int64_t)f;
}
// ops.rs:81-88 div_acc_by_u32 for a non-negative value.
IRIS_HD int64_t div_acc_by_u32_nonneg(int64_t v, uint32_t d) {
  return (int64_t)div_round_even_u64((uint64_t)v, d);
}

// ---- RMSNorm (ops.rs:98-114, 409-428, 722-771) ---------------------------

// inv_sqrt_acc: the u32 c minimising |c^2 * x - 2^64| (ties to even), capped at
// i32::MAX. c^2 * x < 2^125, so the 128-bit product never saturates.
IRIS_HD bool inv_sqrt_le_target(uint32_t c, uint64_t x) {  // c^2 * x <= 2^64
  uint64_t sq = (uint64_t)c * c;
  uint64_t lo = sq * x, hi = mulhi_u64(sq, x);
  return hi == 0 || (hi == 1 && lo == 0);
}
// The tie-break of inv_sqrt_acc between low (the largest c with c^2 x <= 2^64,
// below i32::MAX) and low + 1.
IRIS_HD int32_t inv_sqrt_pick(uint32_t low, uint64_t x) {
  uint32_t lower = low, upper = low + 1;
  // errors |c^2 x - 2^64| as 128-bit (hi, lo) pairs
  uint64_t sq_l = (uint64_t)lower * lower, sq_u = (uint64_t)upper * upper;
  uint64_t l_lo = sq_l * x, l_hi = mulhi_u64(sq_l, x);  // <= 2^64
  uint64_t u_lo = sq_u * x, u_hi = mulhi_u64(sq_u, x);  // > 2^64
  // lower_error = 2^64 - lp  (lp <= 2^64) ; upper_error = up - 2^64
  uint64_t le_hi, le_lo, ue_hi, ue_lo;
  if (l_hi == 1) { le_hi = 0; le_lo = 0; }
  else { le_lo = (uint64_t)0 - l_lo; le_hi = l_lo == 0 ? 1 : 0; }
  ue_lo = u_lo; ue_hi = u_hi - 1;
  bool l_less = (le_hi < ue_hi) || (le_hi == ue_hi && le_lo < ue_lo);
  bool u_less = (ue_hi < le_hi) || (ue_hi == le_hi && ue_lo < le_lo);
  uint32_t r;
  if (l_less) r = lower;
  else if (u_less) r = upper;
  else r = (lower & 1) == 0 ? lower : upper;
  return (int32_t)r;
}
IRIS_HD int32_t inv_sqrt_acc(int64_t xs) {
  if (xs <= 0) return INT32_MAX;  // only 0 reaches here: eps and squares are >= 0
  uint64_t x = (uint64_t)xs;
  const uint32_t max_bits = (uint32_t)INT32_MAX;
  if (inv_sqrt_le_target(max_bits, x)) return INT32_MAX;
  uint32_t low = 0, high = max_bits;
  while (low < high) {
    uint32_t mid = low + ((high - low + 1) >> 1);
    if (inv_sqrt_le_target(mid, x)) low = mid;
    else high = mid - 1;
  }
  return inv_sqrt_pick(low, x);
}
// inv_sqrt_acc from a double-precision estimate of 2^32 / sqrt(x), moved to
// the exact largest c with c^2 x <= 2^64 by exact tests (the estimate is
// within one of it: x < 2^63 and the double's 53-bit rounding), then the
// same tie-break; the binary search of inv_sqrt_acc if the steps ever fail.
IRIS_HD int32_t inv_sqrt_acc_fast(int64_t xs) {
  if (xs <= 0) return INT32_MAX;
  const uint64_t x = (uint64_t)xs;
  if (inv_sqrt_le_target((uint32_t)INT32_MAX, x)) return INT32_MAX;
  const double est = 4294967296.0 / sqrt((double)x);
  uint32_t c = est >= 2147483646.0 ? 2147483646u : (uint32_t)est;
  for (int i = 0; i < 4 && !inv_sqrt_le_target(c, x); ++i) --c;
  for (int i = 0; i < 4 && inv_sqrt_le_target(c + 1, x); ++i) ++c;
  if (!inv_sqrt_le_target(c, x) || inv_sqrt_le_target(c + 1, x)) return inv_sqrt_acc(xs);
  return inv_sqrt_pick(c, x);
}
// n / d rounded half to even for d >= 1, with the power-of-two divisors
// (the models' widths) as a shift.
IRIS_HD uint64_t div_round_even_width(uint64_t n, uint32_t d) {
  if (d >= 2 && (d & (d - 1)) == 0) {
    int s = 0;
    while ((1u << s) != d) ++s;
    uint64_t q = n >> s;
    const uint64_t r = n & (d - 1), half = d >> 1;
    if (r > half || (r == half && (q & 1))) ++q;
    return q;
  }
  return div_round_even_u64(n, d);
}

// ---- Q8_0 (q8.rs) ---------------------------------------------------------

// A half-precision scale as sign * mantissa * 2^exp24 in Q.24 (q8.rs:27-43):
// mantissa <= 2047 and exp24 in [0, 29]. Returns false for Inf/NaN.
IRIS_HD bool q8_scale_parts(uint16_t bits, int32_t* m, int32_t* e) {
  uint32_t ex = (bits >> 10) & 0x1f, man = bits & 0x3ff;
  if (ex == 0x1f) return false;
  int32_t mag = ex == 0 ? (int32_t)man : (int32_t)(man | 0x400);
  *e = ex == 0 ? 0 : (int32_t)ex - 1;
  *m = (bits & 0x8000) ? -mag : mag;
  return true;
}

// q8_scale_parts for bits already known to be finite (checked at upload):
// branch-free.
IRIS_HD void q8_scale_parts_finite(uint16_t bits, int32_t* m, int32_t* e) {
  const uint32_t ex = (bits >> 10) & 0x1f, man = bits & 0x3ff;
  const int32_t mag = (int32_t)(man | (ex ? 0x400u : 0u));
  *e = ex ? (int32_t)ex - 1 : 0;
  *m = (bits & 0x8000) ? -mag : mag;
}

// 128-bit two's-complement accumulator of Q8 partial products.
struct Acc128 {
  uint64_t lo;
  int64_t hi;
};
IRIS_HD void acc128_add(Acc128& a, uint64_t lo, int64_t hi) {
#if defined(__CUDA_ARCH__)
  asm("add.cc.u64 %0, %0, %2;\n\taddc.s64 %1, %1, %3;" : "+l"(a.lo), "+l"(a.hi) : "l"(lo), "l"(hi));
#else
  uint64_t s = a.lo + lo;
  a.hi += hi + (s < lo ? 1 : 0);
  a.lo = s;
#endif
}
// a += p * 2^e for a signed 64-bit p and 0 <= e <= 63.
IRIS_HD void acc128_add_shifted(Acc128& a, int64_t p, int32_t e) {
  uint64_t lo = (uint64_t)p << e;
  int64_t hi = e == 0 ? (p >> 63) : (p >> (64 - e));
  acc128_add(a, lo, hi);
}
// The limbs of an unrounded 128-bit row sum (tensor parallelism's partial
// sums): bits 0-31, 32-63, 64-95 (unsigned) and 96-127 (signed), each in an
// int64, so that the sums of up to 2^31 shards' limbs are exact in int64.
IRIS_HD void limbs_from_acc128(uint64_t lo, int64_t hi, int64_t* l) {
  l[0] = (int64_t)(lo & 0xffffffffull);
  l[1] = (int64_t)(lo >> 32);
  l[2] = (int64_t)((uint64_t)hi & 0xffffffffull);
  l[3] = hi >> 32;
}
// a += the 128-bit total the (summed) limbs l0 + 2^32 l1 + 2^64 l2 + 2^96 l3
// stand for, modulo 2^128: l0, l1, l2 are sums of unsigned 32-bit limbs
// (non-negative, below 2^63), l3 of signed ones.
IRIS_HD void acc128_add_limbs(Acc128& a, int64_t l0, int64_t l1, int64_t l2, int64_t l3) {
  acc128_add(a, (uint64_t)l0, 0);
  acc128_add(a, (uint64_t)l1 << 32, (int64_t)((uint64_t)l1 >> 32));
  acc128_add(a, 0, l2);
  acc128_add(a, 0, (int64_t)((uint64_t)l3 << 32));
}
// round_to_i32(total, 24) (q8.rs:94-104): total / 2^24, ties to even, saturated.
IRIS_HD int32_t acc128_round_q24(Acc128 a) {
  uint64_t flo = (a.lo >> 24) | ((uint64_t)a.hi << 40);
  int64_t fhi = a.hi >> 24;
  uint32_t rem = (uint32_t)(a.lo & 0xFFFFFFull);
  bool up = rem > 0x800000u || (rem == 0x800000u && (flo & 1));
  if (up) {
    flo += 1;
    if (flo == 0) fhi += 1;
  }
  if (fhi > 0 || (fhi == 0 && flo > 0x7FFFFFFFull)) return INT32_MAX;
  if (fhi < -1 || (fhi == -1 && flo < 0xFFFFFFFF80000000ull)) return INT32_MIN;
  return (int32_t)(int64_t)flo;
}
// rms_norm_scale (ops.rs:409-428) from the saturated sum of squares.
IRIS_HD int32_t rms_scale_from_sumsq(uint64_t sumsq_sat, uint32_t n, int64_t eps) {
  int64_t mean = (int64_t)div_round_even_width(sumsq_sat, n);
  return inv_sqrt_acc_fast(acc_add_sat(mean, eps));
}

// acc128_round_q24 of the exact product x m 2^e (|m| < 2^11, 0 <= e <= 29):
// the one-plane GEMM's row value. In 64 bits when |x m| < 2^62 (a rounding
// shift right by 24 - e, or a shift left by e - 24 that saturates), else
// through the 128-bit sum of the two halves of x.
IRIS_HD int32_t round_q24_scaled(int64_t x, int32_t m, int32_t e) {
  const int64_t p = (int64_t)((uint64_t)x * (uint64_t)(int64_t)m);  // the low half
  const int64_t ph = mulhi_s64(x, (int64_t)m);
  if (ph == (p >> 63) && p > -((int64_t)1 << 62) && p < ((int64_t)1 << 62)) {
    if (e < 24) return clamp_i32(shift_round_even(p, 24 - e));
    if (e == 24) return clamp_i32(p);
    const int s = e - 24;
    if (p > ((int64_t)INT32_MAX >> s)) return INT32_MAX;
    if (p < ((int64_t)INT32_MIN >> s)) return INT32_MIN;
    return (int32_t)(p << s);
  }
  Acc128 t{0, 0};
  acc128_add_shifted(t, (int64_t)(x & 0xFFFFFFFFll) * m, e);
  acc128_add_shifted(t, (x >> 32) * m, e + 32);
  return acc128_round_q24(t);
}

// One dequantized weight (dequantize_row, q8.rs:76-91): q * scale / 2^8, ties
// to even, saturated (|q * scale| < 2^47, so it is exact in 64 bits).
IRIS_HD int32_t q8_dequant(int8_t q, int32_t m, int32_t e) {
  int64_t exact = (int64_t)q * (int64_t)m * ((int64_t)1 << e);
  return clamp_i32(shift_round_even(exact, 8));
}

// ---- mistral-dense functions (mistral.rs) ----------------------------------

static constexpr uint64_t kOneQ32 = (uint64_t)1 << 32;
static constexpr uint64_t kLn2Q32 = 2977044472ull;
static constexpr int64_t kHalfPi = 6746518852ll, kPi = 13493037705ll,
                         kThreeHalfPi = 20239556557ll, kTwoPi = 26986075409ll;

IRIS_HD uint32_t mulhi_u32(uint32_t a, uint32_t b) {
#if defined(__CUDA_ARCH__)
  return __umulhi(a, b);
#else
  return (uint32_t)(((uint64_t)a * b) >> 32);
#endif
}
// mistral.rs:43-56 e^-a in Q32 (Horner, products rounded down): acc_15 = 2^32,
// acc_n = 2^32 - floor(floor(r acc_{n+1} / 2^32) / n) for n = 14 .. 1, then
// acc_1 / 2^k. With r < ln 2 in Q32 (below 2^32) and acc <= 2^32 every step
// fits 32-bit halves: floor(r acc / 2^32) is r when acc = 2^32, else the high
// word of the 32 x 32-bit product, and it is below 2^32.
IRIS_HD uint64_t exp_neg_q32(uint64_t a) {
  uint64_t k = a / kLn2Q32;
  if (k >= 32) return 0;
  const uint32_t r = (uint32_t)(a - k * kLn2Q32);
  uint32_t lo = 0;  // acc = 2^32 - d as its low word (0 while acc = 2^32)
  bool top = true;  // acc = 2^32
#pragma unroll
  for (uint32_t n = 14; n >= 1; --n) {
    const uint32_t t = top ? r : mulhi_u32(r, lo);
    const uint32_t d = t / n;
    top = d == 0;
    lo = 0u - d;
  }
  return (top ? kOneQ32 : (uint64_t)lo) >> k;
}
// mistral.rs:59-69. The quotient floor(2^63 / divisor), divisor in
// [2^32, 2^33], is below 2^31 + 1: the double-precision quotient (the
// operands exact, the result correctly rounded with 22 bits below the unit)
// is within one of it, and one integer correction makes it exact.
IRIS_HD uint64_t sigmoid_q32(int32_t x) {
  uint64_t mag = x < 0 ? (uint64_t)0 - (uint64_t)(int64_t)x : (uint64_t)x;
  const uint64_t divisor = kOneQ32 + exp_neg_q32(mag << 16);
  const uint64_t two63 = (uint64_t)1 << 63;
  uint64_t q = (uint64_t)(9223372036854775808.0 / (double)divisor);
  const uint64_t p = q * divisor;  // below 2^64: q is at most one too large
  if (p > two63) --q;
  else if (two63 - p >= divisor) ++q;
  const uint64_t positive = q << 1;
  return x < 0 ? kOneQ32 - positive : positive;
}
// mistral.rs:72-77
IRIS_HD int32_t silu(int32_t x) {
  int64_t product = (int64_t)x * (int64_t)sigmoid_q32(x);
  return clamp_i32(shift_round_even(product, 32));
}
// mistral.rs:84-110, sin and cos of a non-negative Q32.32 angle in Q30.
IRIS_HD void sin_cos_q30(int64_t angle, int64_t* sin_out, int64_t* cos_out) {
  const int64_t one = (int64_t)1 << 30;
  int64_t reduced = angle % kTwoPi;
  if (reduced < 0) reduced += kTwoPi;
  int64_t quarter, ss, cs;
  if (reduced <= kHalfPi) { quarter = reduced; ss = 1; cs = 1; }
  else if (reduced <= kPi) { quarter = kPi - reduced; ss = 1; cs = -1; }
  else if (reduced <= kThreeHalfPi) { quarter = reduced - kPi; ss = -1; cs = -1; }
  else { quarter = kTwoPi - reduced; ss = -1; cs = 1; }
  int64_t t = quarter >> 2;
  int64_t u = (t * t) >> 30;
  int64_t s = one;
  s = one - ((u * s) >> 30) / 210;
  s = one - ((u * s) >> 30) / 156;
  s = one - ((u * s) >> 30) / 110;
  s = one - ((u * s) >> 30) / 72;
  s = one - ((u * s) >> 30) / 42;
  s = one - ((u * s) >> 30) / 20;
  s = one - ((u * s) >> 30) / 6;
  s = (t * s) >> 30;
  int64_t c = one;
  c = one - ((u * c) >> 30) / 240;
  c = one - ((u * c) >> 30) / 182;
  c = one - ((u * c) >> 30) / 132;
  c = one - ((u * c) >> 30) / 90;
  c = one - ((u * c) >> 30) / 56;
  c = one - ((u * c) >> 30) / 30;
  c = one - ((u * c) >> 30) / 12;
  c = one - ((u * c) >> 30) / 2;
  *sin_out = ss * s;
  *cos_out = cs * c;
}
// A pair rotated by an angle of Q2.30 sine s and cosine c (mistral.rs:120-127).
IRIS_HD void rotate_pair_sc(int32_t* a, int32_t* b, int64_t s, int64_t c) {
  int64_t x = *a, y = *b;
  *a = clamp_i32(shift_round_even(x * c - y * s, 30));
  *b = clamp_i32(shift_round_even(x * s + y * c, 30));
}
// One rotated pair (mistral.rs:114-128); position 0 leaves the pair alone.
IRIS_HD void rotate_pair_q30(int32_t* a, int32_t* b, int64_t inverse_frequency, uint32_t position) {
  if (position == 0) return;
  int64_t s, c;
  sin_cos_q30((int64_t)position * inverse_frequency, &s, &c);
  rotate_pair_sc(a, b, s, c);
}
// mistral.rs:130-145 from the wrapping Q32.32 sum.
IRIS_HD int32_t scaled_score_finish(int64_t sum, uint32_t scale_q32) {
  int64_t hi = mulhi_s64(sum, (int64_t)scale_q32);
  uint64_t lo = (uint64_t)sum * (uint64_t)scale_q32;
  int64_t scaled = (int64_t)(((uint64_t)hi << 32) | (lo >> 32));  // floor(sum*scale / 2^32)
  return clamp_i32(shift_round_even(scaled, 16));
}

// ---- softmax (ops.rs:233-276, 508-556) -------------------------------------

// softmax_exp_term(act_to_acc(sub_sat(logit, max))): e^delta in Q32.32.
IRIS_HD int64_t softmax_exp_term_act(int32_t logit, int32_t max_logit) {
  const int64_t ln2 = 2977044472ll;
  int64_t delta = (int64_t)sub_sat(logit, max_logit) * 65536;  // <= 0
  if (delta <= -((int64_t)16 << 32)) return 0;
  int64_t pos = -delta;
  int64_t shift = pos / ln2;
  int64_t r = pos - shift * ln2;
  int64_t r2 = acc_mul_nonneg(r, r), r3 = acc_mul_nonneg(r2, r), r4 = acc_mul_nonneg(r3, r),
          r5 = acc_mul_nonneg(r4, r);
  // 1 - r + r^2/2 - r^3/6 + r^4/24 - r^5/120; no term saturates for r < ln 2.
  int64_t approx = (kOneAcc - r) + (div_acc_by_u32_nonneg(r2, 2) +
                                    (-div_acc_by_u32_nonneg(r3, 6) +
                                     (div_acc_by_u32_nonneg(r4, 24) - div_acc_by_u32_nonneg(r5, 120))));
  if (approx <= 0) return 0;
  if (shift == 0) return approx;
  return shift_round_even(approx, (int)shift);
}
// attention_softmax_raw_weight (ops.rs:269-271): requantize(div_acc(term, sum))
// for 0 <= term <= 2^32 <= sum (the first maximum's term is exactly 2^32).
IRIS_HD int32_t softmax_weight(int64_t term, uint64_t sum) {
  uint64_t q, r;
  if (term < kOneAcc) {
    uint64_t n = (uint64_t)term << 32;
    q = n / sum;
    r = n - q * sum;
  } else {  // term == 2^32: dividend is 2^64
    uint64_t q0 = UINT64_MAX / sum, r0 = UINT64_MAX - q0 * sum;
    if (r0 + 1 == sum) { q = q0 + 1; r = 0; }
    else { q = q0; r = r0 + 1; }
  }
  uint64_t other = sum - r;
  if (r > other) q += 1;
  else if (r == other) q += (q & 1);
  return requantize((int64_t)q);
}

// softmax_weight with the divisor's reciprocal inv = floor((2^64 - 1) / sum)
// computed once for every weight of a head. For n = term * 2^32 < 2^64,
// floor(n * inv / 2^64) is q, q - 1 or q - 2 (q = floor(n / sum)), so two
// exact corrections give the same quotient and remainder as the division;
// sum < 2^62 keeps n - q_est * sum < 3 sum inside 64 bits.
IRIS_HD int32_t softmax_weight_inv(int64_t term, uint64_t sum, uint64_t inv) {
  uint64_t q, r;
  if (term < kOneAcc) {
    const uint64_t n = (uint64_t)term << 32;
    q = mulhi_u64(n, inv);
    r = n - q * sum;
    if (r >= sum) { q += 1; r -= sum; }
    if (r >= sum) { q += 1; r -= sum; }
  } else {  // dividend 2^64 = (2^64 - 1) + 1
    const uint64_t r0 = UINT64_MAX - inv * sum;
    if (r0 + 1 == sum) { q = inv + 1; r = 0; }
    else { q = inv; r = r0 + 1; }
  }
  uint64_t other = sum - r;
  if (r > other) q += 1;
  else if (r == other) q += (q & 1);
  return requantize((int64_t)q);
}

// ---- gemma-dense functions (ops.rs) -----------------------------------------

// ops.rs:357-377 tanh_act
IRIS_HD int32_t tanh_act(int32_t x) {
  const int32_t lin = 27 << 16, quad = 9 << 16, satin = 3 << 16;
  if (x >= satin) return kOneAct;
  if (x <= -satin) return -kOneAct;
  int32_t sq = mul_sat(x, x);
  int32_t num_scale = add_sat(lin, sq);
  int32_t den_scale = add_sat(lin, mul_sat(quad, sq));
  return div_act(mul_sat(x, num_scale), den_scale);
}
// ops.rs:380-388 softcap_act (cap > 0)
IRIS_HD int32_t softcap_act(int32_t x, int32_t cap) { return mul_sat(cap, tanh_act(div_act(x, cap))); }
// ops.rs:391-406 gelu_pytorch_tanh_act
IRIS_HD int32_t gelu_tanh(int32_t x) {
  int32_t sq = mul_sat(x, x);
  int32_t cu = mul_sat(sq, x);
  int32_t inner = add_sat(x, mul_sat(2930, cu));
  int32_t t = tanh_act(mul_sat(52290, inner));
  return mul_sat(mul_sat(1 << 15, x), add_sat(kOneAct, t));
}
// ops.rs:651-683 sine and cosine polynomials, ops.rs:622-649 sin_cos_acc.
IRIS_HD void sin_cos_acc(int64_t angle, int32_t* cos_out, int32_t* sin_out) {
  int64_t reduced = angle % kTwoPi;
  if (reduced < 0) reduced += kTwoPi;
  int64_t x;
  int ss, cs;
  if (reduced <= kHalfPi) { x = reduced; ss = 1; cs = 1; }
  else if (reduced <= kPi) { x = kPi - reduced; ss = 1; cs = -1; }
  else if (reduced <= kThreeHalfPi) { x = reduced - kPi; ss = -1; cs = -1; }
  else { x = kTwoPi - reduced; ss = -1; cs = 1; }
  int64_t x2 = acc_mul_nonneg(x, x), x3 = acc_mul_nonneg(x2, x), x4 = acc_mul_nonneg(x2, x2);
  int64_t x5 = acc_mul_nonneg(x3, x2), x6 = acc_mul_nonneg(x4, x2), x7 = acc_mul_nonneg(x5, x2);
  int64_t sn = (x - div_acc_by_u32_nonneg(x3, 6)) +
               (div_acc_by_u32_nonneg(x5, 120) - div_acc_by_u32_nonneg(x7, 5040));
  int64_t cn = (kOneAcc - div_acc_by_u32_nonneg(x2, 2)) +
               (div_acc_by_u32_nonneg(x4, 24) - div_acc_by_u32_nonneg(x6, 720));
  int32_t s = requantize(sn), c = requantize(cn);
  *sin_out = ss < 0 ? sat_neg32(s) : s;
  *cos_out = cs < 0 ? sat_neg32(c) : c;
}
// One rotate-half pair (ops.rs:186-197) by an angle of cosine c and sine s.
IRIS_HD void rotate_half_pair_cs(int32_t* lhs, int32_t* rhs, int32_t c, int32_t s) {
  int32_t l = *lhs, r = *rhs;
  *lhs = sub_sat(mul_sat(l, c), mul_sat(r, s));
  *rhs = add_sat(mul_sat(r, c), mul_sat(l, s));
}
// One rotate-half pair (ops.rs:186-197) with a precomputed inverse frequency.
IRIS_HD void rotate_half_pair(int32_t* lhs, int32_t* rhs, int64_t inv_frequency, uint32_t position) {
  int64_t angle = (int64_t)position * inv_frequency;  // < 2^63 for positions < 2^31
  int32_t c, s;
  sin_cos_acc(angle, &c, &s);
  rotate_half_pair_cs(lhs, rhs, c, s);
}

}  // namespace iris
