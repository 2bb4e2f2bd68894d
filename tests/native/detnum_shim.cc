// Test shim: exposes the product's exact-arithmetic header
// (iris_b200/csrc/detnum.cuh, compiled here as host C++) with a C ABI so the
// CPU tests can compare it against the oracle without a GPU.
#include "../../iris_b200/csrc/detnum.cuh"
#include "../../iris_b200/csrc/sha256.cuh"

using namespace iris;

extern "C" {
// SHA-256 of each consecutive `chunk`-byte piece of data (the last one
// shorter), 32 bytes a piece, as the device's record leaves are computed.
void shim_sha256_leaves(const uint32_t* data, uint32_t bytes, uint32_t chunk, uint8_t* out) {
  for (uint32_t off = 0, i = 0; off < bytes; off += chunk, ++i)
    sha256_words(data + off / 4, bytes - off < chunk ? bytes - off : chunk, out + 32 * i);
}
int32_t shim_requantize(int64_t x) { return requantize(x); }
int32_t shim_mul_sat(int32_t a, int32_t b) { return mul_sat(a, b); }
int32_t shim_div_act(int32_t a, int32_t b) { return div_act(a, b); }
int32_t shim_inv_sqrt_acc(int64_t x) { return inv_sqrt_acc(x); }
int32_t shim_inv_sqrt_acc_fast(int64_t x) { return inv_sqrt_acc_fast(x); }
int32_t shim_round_q24_scaled(int64_t x, int32_t m, int32_t e) { return round_q24_scaled(x, m, e); }
// the 128-bit formulation the GEMM's one-plane epilogue used (two halves of x)
int32_t shim_round_q24_scaled_ref(int64_t x, int32_t m, int32_t e) {
  Acc128 t{0, 0};
  acc128_add_shifted(t, (int64_t)(x & 0xFFFFFFFFll) * m, e);
  acc128_add_shifted(t, (x >> 32) * m, e + 32);
  return acc128_round_q24(t);
}
uint64_t shim_div_round_even_width(uint64_t n, uint32_t d) { return div_round_even_width(n, d); }
uint64_t shim_div_round_even_u64(uint64_t n, uint64_t d) { return div_round_even_u64(n, d); }
int32_t shim_rms_scale(const int32_t* v, uint32_t n, int64_t eps) {
  uint64_t s = 0;
  for (uint32_t i = 0; i < n; ++i) s = add_sat_nonneg(s, (uint64_t)((int64_t)v[i] * v[i]));
  return rms_scale_from_sumsq(s, n, eps);
}
int32_t shim_silu(int32_t x) { return silu(x); }
void shim_sin_cos_q30(int64_t a, int64_t* s, int64_t* c) { sin_cos_q30(a, s, c); }
void shim_sin_cos_acc(int64_t a, int32_t* c, int32_t* s) { sin_cos_acc(a, c, s); }
int32_t shim_scaled_score(const int32_t* q, const int32_t* k, uint32_t n, uint32_t scale) {
  int64_t sum = 0;
  for (uint32_t i = 0; i < n; ++i) sum = (int64_t)((uint64_t)sum + (uint64_t)((int64_t)q[i] * k[i]));
  return scaled_score_finish(sum, scale);
}
int64_t shim_exp_term(int32_t logit, int32_t mx) { return softmax_exp_term_act(logit, mx); }
int32_t shim_softmax_weight(int64_t term, uint64_t sum) { return softmax_weight(term, sum); }
int32_t shim_softmax_weight_inv(int64_t term, uint64_t sum) {
  return softmax_weight_inv(term, sum, UINT64_MAX / sum);
}
int32_t shim_tanh(int32_t x) { return tanh_act(x); }
int32_t shim_gelu(int32_t x) { return gelu_tanh(x); }
int32_t shim_softcap(int32_t x, int32_t c) { return softcap_act(x, c); }
// dot_row on a raw Q8_0 row through the device formulation: 4 byte planes,
// per-16-value partial block sums, 128-bit shifted accumulation.
int32_t shim_q8_dot(const int32_t* act, const uint8_t* row, uint32_t cols) {
  Acc128 acc{0, 0};
  for (uint32_t b = 0; b < cols / 32; ++b) {
    const uint8_t* blk = row + b * 34;
    int32_t m, e;
    if (!q8_scale_parts((uint16_t)(blk[0] | (blk[1] << 8)), &m, &e)) return 0x7eadbeef;
    for (int half = 0; half < 2; ++half) {
      int32_t S[4] = {0, 0, 0, 0};
      for (int j = 0; j < 16; ++j) {
        int32_t q = (int8_t)blk[2 + half * 16 + j];
        uint32_t a = (uint32_t)act[b * 32 + half * 16 + j];
        S[0] += q * (int32_t)(a & 0xFF);
        S[1] += q * (int32_t)((a >> 8) & 0xFF);
        S[2] += q * (int32_t)((a >> 16) & 0xFF);
        S[3] += q * (int32_t)(int8_t)(a >> 24);
      }
      int64_t bs = (int64_t)(S[0] + S[1] * 256) + ((int64_t)(S[2] + S[3] * 256) << 16);
      acc128_add_shifted(acc, bs * m, e);
    }
  }
  return acc128_round_q24(acc);
}
int32_t shim_q8_dequant(int8_t q, uint16_t bits) {
  int32_t m, e;
  q8_scale_parts(bits, &m, &e);
  return q8_dequant(q, m, e);
}
void shim_rotate_half(int32_t* l, int32_t* r, int64_t f, uint32_t pos) { rotate_half_pair(l, r, f, pos); }
// Tensor parallelism's partial sum of one row over the blocks [b0, b1) of a
// raw Q8_0 row: the unrounded 128-bit total as the four limbs of
// limbs_from_acc128 (the rank's EPI_PARTIAL output).
void shim_partial_limbs(const int32_t* act, const uint8_t* row, uint32_t b0, uint32_t b1, int64_t* limbs) {
  Acc128 acc{0, 0};
  for (uint32_t b = b0; b < b1; ++b) {
    const uint8_t* blk = row + b * 34;
    int32_t m, e;
    q8_scale_parts_finite((uint16_t)(blk[0] | (blk[1] << 8)), &m, &e);
    int64_t bs = 0;
    for (int j = 0; j < 32; ++j) bs += (int64_t)(int8_t)blk[2 + j] * act[b * 32 + j];
    acc128_add_shifted(acc, (bs & 0xFFFFFFFFll) * m, e);
    acc128_add_shifted(acc, (bs >> 32) * m, e + 32);
  }
  limbs_from_acc128(acc.lo, acc.hi, limbs);
}
// The rounded output from the limbs summed over the ranks (tp_finish).
int32_t shim_round_limb_sums(const int64_t* l) {
  Acc128 acc{0, 0};
  acc128_add_limbs(acc, l[0], l[1], l[2], l[3]);
  return acc128_round_q24(acc);
}
}
