// TEST INFRASTRUCTURE ONLY (CPU oracle). Restates the reference's det-num
// crate function by function; each definition cites the Rust source it
// follows. No floating point except the f32 bit decoding of convert.rs.
#include "det_num.h"

#include <cassert>
#include <cstdlib>
#include <cstring>
#include <limits>

namespace oracle {

static const int ACT_FRAC = 16;  // types.rs:23
static const int ACC_FRAC = 32;  // types.rs:24
static const int REQ_SHIFT = 16; // types.rs:25

static int64_t clamp_i128_to_i64(i128 v) {  // ops.rs:496-498
  if (v < (i128)INT64_MIN) return INT64_MIN;
  if (v > (i128)INT64_MAX) return INT64_MAX;
  return (int64_t)v;
}
static int32_t clamp_i128_to_i32(i128 v) {  // ops.rs:492-494
  if (v < (i128)INT32_MIN) return INT32_MIN;
  if (v > (i128)INT32_MAX) return INT32_MAX;
  return (int32_t)v;
}
static int64_t sat_neg64(int64_t v) { return v == INT64_MIN ? INT64_MAX : -v; }
static int32_t sat_neg32(int32_t v) { return v == INT32_MIN ? INT32_MAX : -v; }
static int64_t one_acc() { return (int64_t)1 << ACC_FRAC; }
static int32_t one_act() { return (int32_t)1 << ACT_FRAC; }

int64_t mac_bits(int64_t acc, int32_t a, int32_t b) {
  // wrapping_add of an exact i64 product
  return (int64_t)((uint64_t)acc + (uint64_t)((int64_t)a * (int64_t)b));
}

int32_t add_sat(int32_t a, int32_t b) {
  int32_t r;
  if (__builtin_add_overflow(a, b, &r)) return a < 0 ? INT32_MIN : INT32_MAX;
  return r;
}
int32_t sub_sat(int32_t a, int32_t b) {
  int32_t r;
  if (__builtin_sub_overflow(a, b, &r)) return b > 0 ? INT32_MIN : INT32_MAX;
  return r;
}
int64_t acc_add_sat(int64_t a, int64_t b) {
  int64_t r;
  if (__builtin_add_overflow(a, b, &r)) return a < 0 ? INT64_MIN : INT64_MAX;
  return r;
}

// ops.rs:773-803
static int64_t rshift_round_ties_even_bits(int64_t x, uint32_t shift) {
  if (shift == 0) return x;
  assert(shift < 64);
  i128 divisor = (i128)1 << shift;
  i128 xx = x;
  i128 q = xx / divisor;
  i128 r = xx % divisor;
  if (r == 0) return (int64_t)q;
  i128 twice = (r < 0 ? -r : r) * 2;
  i128 step = xx < 0 ? -1 : 1;
  i128 rounded;
  if (twice < divisor) rounded = q;
  else if (twice > divisor) rounded = q + step;
  else if ((q & 1) == 0) rounded = q;
  else rounded = q + step;
  return (int64_t)rounded;
}

int64_t rshift_round_ties_even(int64_t x, uint32_t shift) { return rshift_round_ties_even_bits(x, shift); }

int32_t requantize(int64_t x) {  // ops.rs:448-451 + narrow_act_sat ops.rs:487-490
  int64_t r = rshift_round_ties_even_bits(x, REQ_SHIFT);
  if (r < INT32_MIN) return INT32_MIN;
  if (r > INT32_MAX) return INT32_MAX;
  return (int32_t)r;
}

int32_t mul_sat(int32_t a, int32_t b) { return requantize((int64_t)a * (int64_t)b); }

i128 round_ties_even_division(i128 dividend, i128 divisor) {
  assert(divisor != 0);
  i128 q = dividend / divisor;
  i128 r = dividend % divisor;
  if (r == 0) return q;
  i128 twice = (r < 0 ? -r : r) * 2;
  i128 absd = divisor < 0 ? -divisor : divisor;
  i128 step = ((dividend < 0) != (divisor < 0)) ? -1 : 1;
  if (twice < absd) return q;
  if (twice > absd) return q + step;
  if ((q & 1) == 0) return q;
  return q + step;
}

int32_t div_act(int32_t num, int32_t den) {
  assert(den != 0);
  i128 dividend = (i128)num << ACT_FRAC;
  return clamp_i128_to_i32(round_ties_even_division(dividend, (i128)den));
}

int64_t div_acc(int64_t num, int64_t den) {
  assert(den != 0);
  i128 dividend = (i128)num << ACC_FRAC;
  return clamp_i128_to_i64(round_ties_even_division(dividend, (i128)den));
}

int64_t div_acc_by_u32(int64_t value, uint32_t divisor) {
  assert(divisor != 0);
  return clamp_i128_to_i64(round_ties_even_division((i128)value, (i128)divisor));
}

size_t argmax_first(const int32_t* xs, size_t n) {
  assert(n > 0);
  size_t best = 0;
  int32_t bb = xs[0];
  for (size_t i = 1; i < n; ++i)
    if (xs[i] > bb) { best = i; bb = xs[i]; }
  return best;
}

int64_t acc_mul(int64_t a, int64_t b) {
  i128 p = (i128)a * (i128)b;
  return clamp_i128_to_i64(round_ties_even_division(p, (i128)1 << ACC_FRAC));
}

static u128 inv_sqrt_product(uint32_t c, u128 divisor) {  // ops.rs:766-771 (saturating)
  u128 cc = (u128)c;
  u128 sq = cc * cc;
  u128 r;
  if (__builtin_mul_overflow(sq, divisor, &r)) return ~(u128)0;
  return r;
}

int32_t inv_sqrt_acc(int64_t x) {
  assert(x >= 0);
  if (x == 0) return INT32_MAX;
  u128 target = (u128)1 << 64;
  u128 divisor = (u128)(uint64_t)x;
  uint32_t max_bits = (uint32_t)INT32_MAX;
  if (inv_sqrt_product(max_bits, divisor) <= target) return INT32_MAX;
  uint32_t low = 0, high = max_bits;
  while (low < high) {
    uint32_t mid = low + ((high - low + 1) / 2);
    if (inv_sqrt_product(mid, divisor) <= target) low = mid;
    else high = mid - 1;
  }
  uint32_t lower = low;
  uint32_t upper = lower == UINT32_MAX ? lower : lower + 1;
  if (upper > max_bits) upper = max_bits;
  u128 lp = inv_sqrt_product(lower, divisor);
  u128 up = inv_sqrt_product(upper, divisor);
  u128 lerr = target - lp;
  u128 uerr = up > target ? up - target : 0;
  uint32_t r;
  if (upper == lower || lerr < uerr) r = lower;
  else if (uerr < lerr) r = upper;
  else if ((lower & 1) == 0) r = lower;
  else r = upper;
  return (int32_t)r;
}

int32_t rms_norm_scale(const int32_t* v, size_t n, int64_t eps) {
  assert(n > 0 && eps >= 0);
  int64_t sum = 0;
  for (size_t i = 0; i < n; ++i) sum = acc_add_sat(sum, (int64_t)v[i] * (int64_t)v[i]);
  assert(n <= UINT32_MAX);
  int64_t mean = div_acc_by_u32(sum, (uint32_t)n);
  int64_t adjusted = acc_add_sat(mean, eps);
  return inv_sqrt_acc(adjusted);
}

void rms_norm_in_place(int32_t* v, const int32_t* w, size_t n, int64_t eps) {
  int32_t scale = rms_norm_scale(v, n, eps);
  for (size_t i = 0; i < n; ++i) {
    int32_t s = mul_sat(v[i], scale);
    v[i] = mul_sat(s, w[i]);
  }
}

void value_rms_norm_in_place(int32_t* v, size_t n, int64_t eps) {
  int32_t scale = rms_norm_scale(v, n, eps);
  for (size_t i = 0; i < n; ++i) v[i] = mul_sat(v[i], scale);
}

// ops.rs:608-614
static int64_t pow_acc_u32(int64_t base, uint32_t e) {
  int64_t r = one_acc();
  for (uint32_t i = 0; i < e; ++i) r = acc_mul(r, base);
  return r;
}

int64_t nth_root_acc(int64_t value, uint32_t degree) {
  assert(degree > 0 && value > 0);
  if (degree == 1 || value == one_acc()) return value;
  int64_t one = one_acc();
  int64_t low = 0, high = value > one ? value : one;
  while (low < high) {
    int64_t mid = low + ((high - low + 1) / 2);
    if (pow_acc_u32(mid, degree) <= value) low = mid;
    else high = mid - 1;
  }
  int64_t lower = low;
  int64_t upper = lower == INT64_MAX ? lower : lower + 1;
  int64_t lv = pow_acc_u32(lower, degree);
  int64_t uv = pow_acc_u32(upper, degree);
  i128 lerr = (i128)value - (i128)lv; if (lerr < 0) lerr = -lerr;
  i128 uerr = (i128)uv - (i128)value; if (uerr < 0) uerr = -uerr;
  if (uerr < lerr) return upper;
  if (lerr < uerr) return lower;
  if ((lower & 1) == 0) return lower;
  return upper;
}

int64_t rope_frequency_step(int64_t base, size_t freq_base_dim) {
  uint32_t degree = (uint32_t)(freq_base_dim / 2);
  int64_t den = nth_root_acc(base, degree);
  return div_acc(one_acc(), den);
}

// ops.rs:616-620
static int64_t mul_usize_by_acc(size_t m, int64_t value) {
  return clamp_i128_to_i64((i128)m * (i128)value);
}

// ops.rs:651-666
static int64_t sin_polynomial(int64_t x) {
  int64_t x2 = acc_mul(x, x), x3 = acc_mul(x2, x), x5 = acc_mul(x3, x2), x7 = acc_mul(x5, x2);
  return acc_add_sat(acc_add_sat(x, sat_neg64(div_acc_by_u32(x3, 6))),
                     acc_add_sat(div_acc_by_u32(x5, 120), sat_neg64(div_acc_by_u32(x7, 5040))));
}
// ops.rs:668-683
static int64_t cos_polynomial(int64_t x) {
  int64_t x2 = acc_mul(x, x), x4 = acc_mul(x2, x2), x6 = acc_mul(x4, x2);
  return acc_add_sat(acc_add_sat(one_acc(), sat_neg64(div_acc_by_u32(x2, 2))),
                     acc_add_sat(div_acc_by_u32(x4, 24), sat_neg64(div_acc_by_u32(x6, 720))));
}

void sin_cos_acc(int64_t angle, int32_t* cos_out, int32_t* sin_out) {
  const int64_t HALF_PI = 6746518852LL, PI = 13493037705LL, THREE_HALF_PI = 20239556557LL,
                TWO_PI = 26986075409LL;
  int64_t reduced = angle % TWO_PI;
  if (reduced < 0) reduced += TWO_PI;  // rem_euclid
  int64_t qa;
  int ss, cs;
  if (reduced <= HALF_PI) { qa = reduced; ss = 1; cs = 1; }
  else if (reduced <= PI) { qa = PI - reduced; ss = 1; cs = -1; }
  else if (reduced <= THREE_HALF_PI) { qa = reduced - PI; ss = -1; cs = -1; }
  else { qa = TWO_PI - reduced; ss = -1; cs = 1; }
  int32_t s = requantize(sin_polynomial(qa));
  int32_t c = requantize(cos_polynomial(qa));
  if (ss < 0) s = sat_neg32(s);
  if (cs < 0) c = sat_neg32(c);
  *cos_out = c;
  *sin_out = s;
}

void rope_rotate_pairs_in_place(int32_t* v, size_t n, size_t rotary_dim, size_t freq_base_dim,
                                int64_t base, size_t position) {
  if (rotary_dim == 0) return;
  assert(rotary_dim % 2 == 0 && rotary_dim <= n);
  assert(freq_base_dim >= 2 && freq_base_dim % 2 == 0);
  assert(base > 0);
  if (position == 0) return;
  size_t half = rotary_dim / 2;
  int64_t inv = one_acc();
  int64_t step = rope_frequency_step(base, freq_base_dim);
  for (size_t i = 0; i < half; ++i) {
    int64_t angle = mul_usize_by_acc(position, inv);
    int32_t c, s;
    sin_cos_acc(angle, &c, &s);
    int32_t lhs = v[i], rhs = v[i + half];
    v[i] = sub_sat(mul_sat(lhs, c), mul_sat(rhs, s));
    v[i + half] = add_sat(mul_sat(rhs, c), mul_sat(lhs, s));
    inv = acc_mul(inv, step);
  }
}

int64_t softmax_exp_term(int64_t delta) {
  const int64_t LN_2_BITS = 2977044472LL;
  const int64_t MIN_DELTA_BITS = -((int64_t)16 << ACC_FRAC);
  assert(delta <= 0);
  if (delta <= MIN_DELTA_BITS) return 0;
  int64_t pos = sat_neg64(delta);
  int64_t shift = pos / LN_2_BITS;
  int64_t r = pos % LN_2_BITS;
  int64_t r2 = acc_mul(r, r), r3 = acc_mul(r2, r), r4 = acc_mul(r3, r), r5 = acc_mul(r4, r);
  int64_t approx = acc_add_sat(
      acc_add_sat(one_acc(), sat_neg64(r)),
      acc_add_sat(div_acc_by_u32(r2, 2),
                  acc_add_sat(sat_neg64(div_acc_by_u32(r3, 6)),
                              acc_add_sat(div_acc_by_u32(r4, 24), sat_neg64(div_acc_by_u32(r5, 120))))));
  if (approx <= 0) return 0;
  if (shift >= 0 && shift < 64) return rshift_round_ties_even(approx, (uint32_t)shift);
  return 0;
}

int64_t attention_softmax_exp_term(int32_t logit, int32_t max_logit) {
  int32_t d = sub_sat(logit, max_logit);
  return softmax_exp_term((int64_t)d * ((int64_t)1 << REQ_SHIFT));  // act_to_acc ops.rs:500-502
}

void attention_softmax(const int32_t* logits, size_t n, int32_t* weights) {
  assert(n > 0);
  size_t mi = argmax_first(logits, n);
  int32_t mx = logits[mi];
  std::vector<int64_t> terms(n);
  for (size_t i = 0; i < n; ++i) terms[i] = attention_softmax_exp_term(logits[i], mx);
  int64_t sum = 0;
  for (size_t i = 0; i < n; ++i) sum = acc_add_sat(sum, terms[i]);
  for (size_t i = 0; i < n; ++i) weights[i] = requantize(div_acc(terms[i], sum));  // ops.rs:269-271
  int32_t summed = 0;
  for (size_t i = 0; i < n; ++i) summed = add_sat(summed, weights[i]);
  int32_t residual = sub_sat(one_act(), summed);  // ops.rs:274-276
  weights[mi] = add_sat(weights[mi], residual);
}

int32_t tanh_act(int32_t x) {
  const int32_t LIN = 27 << ACT_FRAC, QUAD = 9 << ACT_FRAC, SATIN = 3 << ACT_FRAC;
  if (x >= SATIN) return one_act();
  if (x <= -SATIN) return sat_neg32(one_act());
  int32_t sq = mul_sat(x, x);
  int32_t num_scale = add_sat(LIN, sq);
  int32_t den_scale = add_sat(LIN, mul_sat(QUAD, sq));
  int32_t num = mul_sat(x, num_scale);
  return div_act(num, den_scale);
}

int32_t softcap_act(int32_t x, int32_t cap) {
  assert(cap > 0);
  int32_t normalized = div_act(x, cap);
  return mul_sat(cap, tanh_act(normalized));
}

int32_t gelu_pytorch_tanh_act(int32_t x) {
  const int32_t HALF = 1 << (ACT_FRAC - 1), INNER = 52290, CUBIC = 2930;
  int32_t sq = mul_sat(x, x);
  int32_t cu = mul_sat(sq, x);
  int32_t cubic = mul_sat(CUBIC, cu);
  int32_t inner = add_sat(x, cubic);
  int32_t tin = mul_sat(INNER, inner);
  int32_t t = tanh_act(tin);
  return mul_sat(mul_sat(HALF, x), add_sat(one_act(), t));
}

// ---- q8.rs ----------------------------------------------------------------
bool row_bytes(size_t cols, size_t* out) {
  if (cols > 0 && cols % Q8_BLOCK == 0) { *out = cols / Q8_BLOCK * Q8_BLOCK_BYTES; return true; }
  return false;
}

bool scale_q24(uint16_t bits, int64_t* out) {
  uint32_t exponent = (bits >> 10) & 0x1f;
  int64_t mantissa = bits & 0x3ff;
  int64_t mag;
  if (exponent == 0x1f) return false;
  if (exponent == 0) mag = mantissa;
  else mag = (1024 + mantissa) << (exponent - 1);
  *out = (bits & 0x8000) ? -mag : mag;
  return true;
}

int32_t round_to_i32(i128 value, uint32_t shift) {
  i128 floor = value >> shift;
  i128 rem = value - (floor << shift);
  i128 half = (i128)1 << (shift - 1);
  i128 rounded = (rem > half || (rem == half && (floor & 1) == 1)) ? floor + 1 : floor;
  return clamp_i128_to_i32(rounded);
}

bool dot_row(const int32_t* act, size_t cols, const uint8_t* row, size_t row_len, int32_t* out) {
  size_t rb;
  if (!row_bytes(cols, &rb) || rb != row_len) return false;
  i128 total = 0;
  for (size_t b = 0; b < cols / Q8_BLOCK; ++b) {
    const uint8_t* blk = row + b * Q8_BLOCK_BYTES;
    int64_t scale;
    if (!scale_q24((uint16_t)(blk[0] | (blk[1] << 8)), &scale)) return false;
    int64_t sum = 0;
    for (size_t j = 0; j < Q8_BLOCK; ++j) sum += (int64_t)(int8_t)blk[2 + j] * (int64_t)act[b * Q8_BLOCK + j];
    // wrapping i128 add (never wraps for realistic widths)
    total = (i128)((u128)total + (u128)((i128)sum * (i128)scale));
  }
  *out = round_to_i32(total, 24);
  return true;
}

bool dequantize_row(const uint8_t* row, size_t row_len, int32_t* out, size_t cols) {
  size_t rb;
  if (!row_bytes(cols, &rb) || rb != row_len) return false;
  for (size_t b = 0; b < cols / Q8_BLOCK; ++b) {
    const uint8_t* blk = row + b * Q8_BLOCK_BYTES;
    int64_t scale;
    if (!scale_q24((uint16_t)(blk[0] | (blk[1] << 8)), &scale)) return false;
    for (size_t j = 0; j < Q8_BLOCK; ++j)
      out[b * Q8_BLOCK + j] = round_to_i32((i128)(int8_t)blk[2 + j] * (i128)scale, 24 - 16);
  }
  return true;
}

// ---- mistral.rs -----------------------------------------------------------
static const uint64_t ONE_Q32 = (uint64_t)1 << 32;
static const uint64_t LN_2_Q32 = 2977044472ULL;

static int64_t shift_round_ties_even64(int64_t value, uint32_t shift) {  // mistral.rs:23-32
  int64_t floor = value >> shift;
  int64_t rem = value - (int64_t)((uint64_t)floor << shift);
  int64_t half = (int64_t)1 << (shift - 1);
  if (rem > half || (rem == half && (floor & 1) == 1)) return floor + 1;
  return floor;
}
static int32_t saturate64(int64_t v) {
  if (v < INT32_MIN) return INT32_MIN;
  if (v > INT32_MAX) return INT32_MAX;
  return (int32_t)v;
}

uint64_t exp_neg_q32(uint64_t a) {
  uint64_t k = a / LN_2_Q32;
  if (k >= 32) return 0;
  uint64_t r = a % LN_2_Q32;
  uint64_t acc = ONE_Q32;
  for (uint64_t n = 14; n >= 1; --n) acc = ONE_Q32 - ((r * acc) >> 32) / n;
  return acc >> k;
}

uint64_t sigmoid_q32(int32_t x) {
  uint64_t mag = (uint64_t)(x < 0 ? -(int64_t)x : (int64_t)x);  // unsigned_abs
  uint64_t divisor = ONE_Q32 + exp_neg_q32(mag << 16);
  uint64_t positive = (((uint64_t)1 << 63) / divisor) << 1;
  return x < 0 ? ONE_Q32 - positive : positive;
}

int32_t silu(int32_t x) {
  int64_t product = (int64_t)x * (int64_t)sigmoid_q32(x);
  return saturate64(shift_round_ties_even64(product, 32));
}

void sin_cos_q30(int64_t angle, int64_t* sin_out, int64_t* cos_out) {
  const int64_t ONE_Q30 = (int64_t)1 << 30;
  const int64_t HALF_PI = 6746518852LL, PI = 13493037705LL, THREE_HALF_PI = 20239556557LL,
                TWO_PI = 26986075409LL;
  int64_t reduced = angle % TWO_PI;
  if (reduced < 0) reduced += TWO_PI;
  int64_t quarter, ss, cs;
  if (reduced <= HALF_PI) { quarter = reduced; ss = 1; cs = 1; }
  else if (reduced <= PI) { quarter = PI - reduced; ss = 1; cs = -1; }
  else if (reduced <= THREE_HALF_PI) { quarter = reduced - PI; ss = -1; cs = -1; }
  else { quarter = TWO_PI - reduced; ss = -1; cs = 1; }
  int64_t t = quarter >> 2;
  int64_t u = (t * t) >> 30;
  int64_t s = ONE_Q30;
  const int64_t sd[7] = {210, 156, 110, 72, 42, 20, 6};
  for (int i = 0; i < 7; ++i) s = ONE_Q30 - ((u * s) >> 30) / sd[i];
  s = (t * s) >> 30;
  int64_t c = ONE_Q30;
  const int64_t cd[8] = {240, 182, 132, 90, 56, 30, 12, 2};
  for (int i = 0; i < 8; ++i) c = ONE_Q30 - ((u * c) >> 30) / cd[i];
  *sin_out = ss * s;
  *cos_out = cs * c;
}

void rotate_consecutive_pairs(int32_t* v, size_t n, const int64_t* freqs, size_t n_freqs,
                              uint32_t position) {
  if (position == 0) return;
  size_t pairs = n / 2;
  if (n_freqs < pairs) pairs = n_freqs;  // zip stops at the shorter
  for (size_t j = 0; j < pairs; ++j) {
    int64_t angle = (int64_t)position * freqs[j];
    int64_t s, c;
    sin_cos_q30(angle, &s, &c);
    int64_t a = v[2 * j], b = v[2 * j + 1];
    v[2 * j] = saturate64(shift_round_ties_even64(a * c - b * s, 30));
    v[2 * j + 1] = saturate64(shift_round_ties_even64(a * s + b * c, 30));
  }
}

int32_t scaled_score(const int32_t* q, const int32_t* k, size_t n, uint32_t scale_q32) {
  int64_t sum = 0;
  for (size_t i = 0; i < n; ++i) sum = (int64_t)((uint64_t)sum + (uint64_t)((int64_t)q[i] * (int64_t)k[i]));
  i128 scaled = ((i128)sum * (i128)scale_q32) >> 32;
  i128 half = (i128)1 << 15;
  i128 floor = scaled >> 16;
  i128 rem = scaled - (floor << 16);
  i128 rounded = (rem > half || (rem == half && (floor & 1) == 1)) ? floor + 1 : floor;
  return clamp_i128_to_i32(rounded);
}

uint32_t attention_scale_q32(uint32_t head_dim) {
  u128 target = ((u128)1 << 64) / (u128)(head_dim > 1 ? head_dim : 1);
  u128 low = 0, high = UINT32_MAX;
  while (low < high) {
    u128 mid = (low + high + 1) / 2;
    if (mid * mid <= target) low = mid;
    else high = mid - 1;
  }
  return (uint32_t)low;
}

static u128 integer_sqrt(u128 value) {  // mistral.rs:162-176
  if (value < 2) return value;
  u128 low = 1, high = (u128)1 << 64;
  while (low < high) {
    u128 mid = (low + high + 1) / 2;
    if (mid <= value / mid) low = mid;
    else high = mid - 1;
  }
  return low;
}

bool yarn_inverse_frequencies(uint64_t base, uint32_t pairs, uint32_t factor, uint32_t low,
                              uint32_t high, std::vector<int64_t>* out) {
  bool pow2 = pairs != 0 && (pairs & (pairs - 1)) == 0;
  if (!pow2 || base == 0 || factor == 0 || high <= low) return false;
  u128 root = (u128)base << 32;
  int tz = __builtin_ctz(pairs);
  for (int i = 0; i < tz; ++i) root = integer_sqrt(root << 32);
  u128 step = (((u128)1 << 64) + root / 2) / root;
  u128 span = (u128)(high - low);
  u128 plain = (u128)1 << 32;
  out->clear();
  for (uint32_t pair = 0; pair < pairs; ++pair) {
    u128 kept = (u128)(high > pair ? high - pair : 0);
    if (kept > span) kept = span;
    u128 num = plain * (span + (u128)(factor - 1) * kept);
    u128 den = (u128)factor * span;
    out->push_back((int64_t)((num + den / 2) / den));
    plain = (plain * step + ((u128)1 << 31)) >> 32;
  }
  return true;
}

// ---- convert.rs -------------------------------------------------------------
static u128 round_ties_even_div_pow2(u128 value, uint32_t shift) {  // convert.rs:113-129
  if (shift == 0) return value;
  if (shift >= 128) return 0;
  u128 q = value >> shift;
  u128 mask = ((u128)1 << shift) - 1;
  u128 r = value & mask;
  u128 half = (u128)1 << (shift - 1);
  if (r > half || (r == half && (q & 1) == 1)) return q + 1;
  return q;
}
static u128 saturating_shift_left(u128 value, uint32_t shift, u128 maxm) {  // convert.rs:99-111
  if (value == 0) return 0;
  if (shift >= 128) return maxm;
  u128 threshold = maxm >> shift;
  return value > threshold ? maxm : value << shift;
}
static i128 f32_to_fixed_bits(float x, uint32_t frac, u128 max_pos, u128 max_neg) {  // :52-97
  uint32_t bits;
  std::memcpy(&bits, &x, 4);
  bool neg = (bits >> 31) != 0;
  int32_t eb = (int32_t)((bits >> 23) & 0xff);
  uint32_t fb = bits & 0x7fffff;
  if (eb == 0 && fb == 0) return 0;
  u128 sig;
  int32_t ex;
  if (eb == 0) { sig = fb; ex = -149; }
  else { sig = (u128)((1u << 23) | fb); ex = eb - 127 - 23; }
  int32_t se = ex + (int32_t)frac;
  u128 maxm = neg ? max_neg : max_pos;
  u128 mag;
  if (se >= 0) mag = saturating_shift_left(sig, (uint32_t)se, maxm);
  else { mag = round_ties_even_div_pow2(sig, (uint32_t)(-se)); if (mag > maxm) mag = maxm; }
  if (neg) return mag >= max_neg ? -(i128)max_neg : -(i128)mag;
  return (i128)mag;
}

int32_t f32_to_act(float x) {
  i128 b = f32_to_fixed_bits(x, ACT_FRAC, (u128)INT32_MAX, (u128)1 << 31);
  if (b < 0) return b <= (i128)INT32_MIN ? INT32_MIN : (int32_t)b;
  return b > (i128)INT32_MAX ? INT32_MAX : (int32_t)b;
}

int64_t f32_to_acc(float x) {
  i128 b = f32_to_fixed_bits(x, ACC_FRAC, (u128)INT64_MAX, (u128)1 << 63);
  if (b < 0) return b <= (i128)INT64_MIN ? INT64_MIN : (int64_t)b;
  return b > (i128)INT64_MAX ? INT64_MAX : (int64_t)b;
}

// ---- tensor.rs --------------------------------------------------------------
int32_t dot_bits(const int32_t* a, const int32_t* b, size_t n) {
  int64_t acc = 0;
  for (size_t i = 0; i < n; ++i) acc = mac_bits(acc, a[i], b[i]);
  return requantize(acc);
}
int32_t requantize_acc(int64_t acc) { return requantize(acc); }

}  // namespace oracle
