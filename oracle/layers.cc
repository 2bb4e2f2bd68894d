// TEST INFRASTRUCTURE ONLY (CPU oracle). Restates the reference's layer,
// head and decode-loop code on top of det_num.cc. Threads share rows the way
// the reference's rayon code does (at least 64 rows a task,
// crates/inference/kernels/src/tensor.rs:9-10,175-185); every value is
// computed independently, so threading never changes a result.
#include <algorithm>
#include <cstring>
#include <thread>
#include <vector>

#include "det_num.h"
#include "oracle_abi.h"

using namespace oracle;

namespace {

template <class F>
void parallel_for(size_t n, int threads, size_t min_chunk, F f) {
  if (threads <= 1 || n < 2 * min_chunk) {
    for (size_t i = 0; i < n; ++i) f(i);
    return;
  }
  size_t chunk = std::max(min_chunk, (n + threads - 1) / threads);
  std::vector<std::thread> pool;
  for (size_t start = 0; start < n; start += chunk) {
    size_t end = std::min(n, start + chunk);
    pool.emplace_back([=, &f]() {
      for (size_t i = start; i < end; ++i) f(i);
    });
  }
  for (auto& t : pool) t.join();
}

// linear_slab_from_source: out[t][r] = dot_row(in[t], row r) (tensor.rs:437-520).
bool linear(const int32_t* in, size_t tokens, size_t cols, const uint8_t* q8, size_t rows,
            int32_t* out, int threads) {
  size_t rb;
  if (!row_bytes(cols, &rb)) return false;
  std::vector<char> ok(rows, 1);
  parallel_for(rows, threads, 64, [&](size_t r) {
    for (size_t t = 0; t < tokens; ++t)
      if (!dot_row(in + t * cols, cols, q8 + r * rb, rb, &out[t * rows + r])) ok[r] = 0;
  });
  for (char c : ok)
    if (!c) return false;
  return true;
}

void linear_dense(const int32_t* in, size_t tokens, size_t cols, const int32_t* w, size_t rows,
                  int32_t* out, int threads) {
  parallel_for(rows, threads, 64, [&](size_t r) {
    for (size_t t = 0; t < tokens; ++t) out[t * rows + r] = dot_bits(in + t * cols, w + r * cols, cols);
  });
}

// prefill-range/src/input.rs:407-419
void add_row(int32_t* dst, const int32_t* src, size_t n) {
  for (size_t i = 0; i < n; ++i) dst[i] = add_sat(dst[i], src[i]);
}

}  // namespace

extern "C" {

int32_t oracle_requantize(int64_t x) { return requantize(x); }
int64_t oracle_rshift_round_ties_even(int64_t x, uint32_t s) { return rshift_round_ties_even(x, s); }
int64_t oracle_mac_bits(int64_t acc, int32_t a, int32_t b) { return mac_bits(acc, a, b); }
int32_t oracle_add_sat(int32_t a, int32_t b) { return add_sat(a, b); }
int32_t oracle_sub_sat(int32_t a, int32_t b) { return sub_sat(a, b); }
int32_t oracle_mul_sat(int32_t a, int32_t b) { return mul_sat(a, b); }
int32_t oracle_div_act(int32_t a, int32_t b) { return div_act(a, b); }
int64_t oracle_div_acc(int64_t a, int64_t b) { return div_acc(a, b); }
int64_t oracle_acc_mul(int64_t a, int64_t b) { return acc_mul(a, b); }
int32_t oracle_inv_sqrt_acc(int64_t x) { return inv_sqrt_acc(x); }
int32_t oracle_tanh(int32_t x) { return tanh_act(x); }
int32_t oracle_gelu(int32_t x) { return gelu_pytorch_tanh_act(x); }
int32_t oracle_softcap(int32_t x, int32_t cap) { return softcap_act(x, cap); }
int64_t oracle_softmax_exp_term(int64_t d) { return softmax_exp_term(d); }
int32_t oracle_silu(int32_t x) { return silu(x); }
uint64_t oracle_sigmoid_q32(int32_t x) { return sigmoid_q32(x); }
uint64_t oracle_exp_neg_q32(uint64_t a) { return exp_neg_q32(a); }
void oracle_sin_cos_q30(int64_t a, int64_t* s, int64_t* c) { sin_cos_q30(a, s, c); }
void oracle_sin_cos_acc(int64_t a, int32_t* c, int32_t* s) { sin_cos_acc(a, c, s); }
int64_t oracle_rope_frequency_step(int64_t base, uint32_t fbd) { return rope_frequency_step(base, fbd); }
int64_t oracle_nth_root_acc(int64_t v, uint32_t d) { return nth_root_acc(v, d); }
uint32_t oracle_attention_scale_q32(uint32_t d) { return attention_scale_q32(d); }
int oracle_yarn_inverse_frequencies(uint64_t base, uint32_t pairs, uint32_t factor, uint32_t low,
                                    uint32_t high, int64_t* out) {
  std::vector<int64_t> v;
  if (!yarn_inverse_frequencies(base, pairs, factor, low, high, &v)) return -1;
  std::memcpy(out, v.data(), v.size() * sizeof(int64_t));
  return 0;
}
int32_t oracle_scaled_score(const int32_t* q, const int32_t* k, size_t n, uint32_t s) {
  return scaled_score(q, k, n, s);
}
int32_t oracle_dot_bits(const int32_t* a, const int32_t* b, size_t n) { return dot_bits(a, b, n); }
int32_t oracle_f32_to_act(float x) { return f32_to_act(x); }
int64_t oracle_f32_to_acc(float x) { return f32_to_acc(x); }
int oracle_scale_q24(uint16_t bits, int64_t* out) { return scale_q24(bits, out) ? 0 : -1; }
int oracle_dot_row(const int32_t* act, size_t cols, const uint8_t* row, size_t len, int32_t* out) {
  return dot_row(act, cols, row, len, out) ? 0 : -1;
}
int oracle_dequantize_row(const uint8_t* row, size_t len, int32_t* out, size_t cols) {
  return dequantize_row(row, len, out, cols) ? 0 : -1;
}
void oracle_rms_norm(int32_t* v, const int32_t* w, size_t n, int64_t eps) { rms_norm_in_place(v, w, n, eps); }
void oracle_value_rms_norm(int32_t* v, size_t n, int64_t eps) { value_rms_norm_in_place(v, n, eps); }
int32_t oracle_rms_norm_scale(const int32_t* v, size_t n, int64_t eps) { return rms_norm_scale(v, n, eps); }
void oracle_rope_rotate_pairs(int32_t* v, size_t n, size_t rd, size_t fbd, int64_t base, size_t pos) {
  rope_rotate_pairs_in_place(v, n, rd, fbd, base, pos);
}
void oracle_rotate_consecutive_pairs(int32_t* v, size_t n, const int64_t* f, size_t nf, uint32_t pos) {
  rotate_consecutive_pairs(v, n, f, nf, pos);
}
void oracle_attention_softmax(const int32_t* logits, size_t n, int32_t* w) { attention_softmax(logits, n, w); }

int oracle_linear(const int32_t* in, size_t tokens, size_t cols, const uint8_t* q8, size_t rows,
                  int32_t* out, int threads) {
  return linear(in, tokens, cols, q8, rows, out, threads) ? 0 : -1;
}
int oracle_linear_dense(const int32_t* in, size_t tokens, size_t cols, const int32_t* w,
                        size_t rows, int32_t* out, int threads) {
  linear_dense(in, tokens, cols, w, rows, out, threads);
  return 0;
}

// ---------------------------------------------------------------------------
// mistral-dense: crates/inference/kernels/src/mistral/layer.rs
// ---------------------------------------------------------------------------

static bool mistral_params_ok(const OracleMistralLayer* p) {  // layer.rs:53-92
  if (!p->hidden || !p->ffn || !p->heads || !p->kv_heads || !p->head_dim) return false;
  if (p->heads % p->kv_heads) return false;
  if (p->head_dim % 2 || p->n_freqs != p->head_dim / 2) return false;
  for (uint32_t i = 0; i < p->n_freqs; ++i)
    if (p->rope_freqs[i] < 0 || p->rope_freqs[i] > ((int64_t)1 << 32)) return false;
  if (p->norm_eps < 0) return false;
  return true;
}

// attention_context (layer.rs:274-318) for one query row at `position`;
// keys_k/keys_v hold rows 0..=position of kv_dim values.
static void mistral_attention_context(const OracleMistralLayer* p, const int32_t* query,
                                      size_t position, const int32_t* keys_k,
                                      const int32_t* keys_v, int32_t* context) {
  size_t heads = p->heads, kvh = p->kv_heads, d = p->head_dim, group = heads / kvh;
  size_t kvd = kvh * d, visible = position + 1;
  std::vector<int32_t> logits(visible), weights(visible);
  for (size_t h = 0; h < heads; ++h) {
    size_t kv0 = (h / group) * d;
    const int32_t* qh = query + h * d;
    for (size_t t = 0; t < visible; ++t)
      logits[t] = scaled_score(qh, keys_k + t * kvd + kv0, d, p->attention_scale_q32);
    attention_softmax(logits.data(), visible, weights.data());
    for (size_t i = 0; i < d; ++i) {
      int64_t acc = 0;
      for (size_t t = 0; t < visible; ++t) acc = mac_bits(acc, weights[t], keys_v[t * kvd + kv0 + i]);
      context[h * d + i] = requantize_acc(acc);
    }
  }
}

int oracle_mistral_layer(const OracleMistralLayer* p, const int32_t* rows_in, size_t m,
                         uint32_t start, const int32_t* prior_k, const int32_t* prior_v,
                         int32_t* rows_out, int32_t* own_k, int32_t* own_v, int threads) {
  if (!mistral_params_ok(p)) return -1;
  if (m == 0) return 0;
  if ((uint64_t)start + m > p->max_positions) return -2;
  size_t H = p->hidden, F = p->ffn, d = p->head_dim;
  size_t qd = (size_t)p->heads * d, kvd = (size_t)p->kv_heads * d;
  std::vector<int32_t> normed(rows_in, rows_in + m * H);
  parallel_for(m, threads, 1, [&](size_t r) {
    rms_norm_in_place(&normed[r * H], p->norm_attention, H, p->norm_eps);
  });
  std::vector<int32_t> q(m * qd), k(m * kvd), v(m * kvd);
  if (!linear(normed.data(), m, H, p->w_q, qd, q.data(), threads)) return -3;
  if (!linear(normed.data(), m, H, p->w_k, kvd, k.data(), threads)) return -3;
  if (!linear(normed.data(), m, H, p->w_v, kvd, v.data(), threads)) return -3;
  parallel_for(m, threads, 1, [&](size_t r) {  // layer.rs:163-185
    for (size_t h = 0; h < p->heads; ++h)
      rotate_consecutive_pairs(&q[r * qd + h * d], d, p->rope_freqs, p->n_freqs, start + (uint32_t)r);
    for (size_t h = 0; h < p->kv_heads; ++h)
      rotate_consecutive_pairs(&k[r * kvd + h * d], d, p->rope_freqs, p->n_freqs, start + (uint32_t)r);
  });
  // Every key a query of this range may see: the prefix's, then its own.
  std::vector<int32_t> keys_k((start + m) * kvd), keys_v((start + m) * kvd);
  if (start) {
    std::memcpy(keys_k.data(), prior_k, start * kvd * 4);
    std::memcpy(keys_v.data(), prior_v, start * kvd * 4);
  }
  std::memcpy(&keys_k[start * kvd], k.data(), m * kvd * 4);
  std::memcpy(&keys_v[start * kvd], v.data(), m * kvd * 4);
  std::memcpy(own_k, k.data(), m * kvd * 4);
  std::memcpy(own_v, v.data(), m * kvd * 4);

  const size_t CHUNK = 256;  // layer.rs:96
  for (size_t c0 = 0; c0 < m; c0 += CHUNK) {
    size_t n = std::min(CHUNK, m - c0);
    std::vector<int32_t> ctx(n * qd);
    parallel_for(n, threads, 1, [&](size_t i) {
      mistral_attention_context(p, &q[(c0 + i) * qd], start + c0 + i, keys_k.data(), keys_v.data(),
                                &ctx[i * qd]);
    });
    std::vector<int32_t> attended(n * H);
    if (!linear(ctx.data(), n, qd, p->w_o, H, attended.data(), threads)) return -3;
    for (size_t i = 0; i < n; ++i) add_row(&attended[i * H], rows_in + (c0 + i) * H, H);
    std::vector<int32_t> ff_in(attended);
    for (size_t i = 0; i < n; ++i) rms_norm_in_place(&ff_in[i * H], p->norm_feed_forward, H, p->norm_eps);
    std::vector<int32_t> gate(n * F), up(n * F);
    if (!linear(ff_in.data(), n, H, p->w_gate, F, gate.data(), threads)) return -3;
    if (!linear(ff_in.data(), n, H, p->w_up, F, up.data(), threads)) return -3;
    for (size_t i = 0; i < n * F; ++i) gate[i] = mul_sat(silu(gate[i]), up[i]);  // layer.rs:251-258
    std::vector<int32_t> ff(n * H);
    if (!linear(gate.data(), n, F, p->w_down, H, ff.data(), threads)) return -3;
    for (size_t i = 0; i < n; ++i) {
      add_row(&ff[i * H], &attended[i * H], H);
      std::memcpy(rows_out + (c0 + i) * H, &ff[i * H], H * 4);
    }
  }
  return 0;
}

// ---------------------------------------------------------------------------
// gemma-dense: crates/inference/kernels/src/prefill_range.rs
// ---------------------------------------------------------------------------

static uint32_t window_start(uint32_t qpos, uint32_t window) {  // prefill_range.rs:866-874
  if (window == 0) return 0;
  uint64_t a = (uint64_t)qpos + 1;
  return a > window ? (uint32_t)(a - window) : 0;
}
static bool is_visible(uint32_t qpos, uint32_t kpos, uint32_t window) {  // :876-879
  return kpos <= qpos && (window == 0 || qpos - kpos < window);
}

static bool gemma_params_ok(const OracleGemmaLayer* p) {  // prefill_range.rs:403-484
  if (!p->hidden || !p->ffn || !p->heads || !p->kv_heads || !p->head_dim) return false;
  if (p->heads % p->kv_heads) return false;
  if (p->rotary_dim % 2 || p->rotary_dim > p->head_dim) return false;
  if (p->rotary_dim > 0 && (p->rope_freq_base_dim < 2 || p->rope_freq_base_dim % 2)) return false;
  if (p->rotary_dim > 0 && p->rope_base <= 0) return false;
  if (p->norm_eps < 0) return false;
  if (p->donor_a_layer == -1 || p->donor_b_layer == -1) return false;
  if (p->kv_donor_layer >= 0 && p->kv_donor_layer != p->donor_a_layer &&
      p->kv_donor_layer != p->donor_b_layer)
    return false;
  return true;
}

struct KeyRef {
  uint32_t position;
  const int32_t* k;
  const int32_t* v;
};

int oracle_gemma_layer(const OracleGemmaLayer* p, const int32_t* rows_in, size_t m, uint32_t start,
                       OracleKeys prior, OracleKeys donor_a, OracleKeys donor_b,
                       const int32_t* ple_rows, int32_t* rows_out, int32_t* own_k, int32_t* own_v,
                       int threads) {
  if (!gemma_params_ok(p)) return -1;
  if (m == 0) return 0;
  size_t H = p->hidden, F = p->ffn, d = p->head_dim, P = p->ple_width;
  size_t heads = p->heads, kvh = p->kv_heads, qd = heads * d, kvd = kvh * d, group = heads / kvh;
  // project_tokens (prefill_range.rs:497-579)
  std::vector<int32_t> normed(rows_in, rows_in + m * H);
  parallel_for(m, threads, 1, [&](size_t r) { rms_norm_in_place(&normed[r * H], p->norm_input, H, p->norm_eps); });
  std::vector<int32_t> q(m * qd), k(m * kvd), v(m * kvd);
  if (!linear(normed.data(), m, H, p->w_q, qd, q.data(), threads)) return -3;
  if (!linear(normed.data(), m, H, p->w_k, kvd, k.data(), threads)) return -3;
  if (!linear(normed.data(), m, H, p->w_v, kvd, v.data(), threads)) return -3;
  parallel_for(m, threads, 1, [&](size_t r) {  // finish_qkv_row :607-629, apply_rope :631-647
    uint32_t pos = start + (uint32_t)r;
    for (size_t h = 0; h < heads; ++h) {
      int32_t* x = &q[r * qd + h * d];
      rms_norm_in_place(x, p->q_norm, d, p->norm_eps);
      if (p->rotary_dim && pos) rope_rotate_pairs_in_place(x, d, p->rotary_dim, p->rope_freq_base_dim, p->rope_base, pos);
    }
    for (size_t h = 0; h < kvh; ++h) {
      int32_t* x = &k[r * kvd + h * d];
      rms_norm_in_place(x, p->k_norm, d, p->norm_eps);
      if (p->rotary_dim && pos) rope_rotate_pairs_in_place(x, d, p->rotary_dim, p->rope_freq_base_dim, p->rope_base, pos);
    }
    for (size_t h = 0; h < kvh; ++h) value_rms_norm_in_place(&v[r * kvd + h * d], d, p->norm_eps);
  });
  std::memcpy(own_k, k.data(), m * kvd * 4);
  std::memcpy(own_v, v.data(), m * kvd * 4);

  // attend_tokens key sources (:663-684)
  std::vector<KeyRef> keys;
  auto push = [&](OracleKeys ks) {
    for (size_t i = 0; i < ks.n; ++i) keys.push_back({ks.positions[i], ks.k + i * kvd, ks.v + i * kvd});
  };
  if (p->kv_donor_layer == -1) {
    push(prior);
    for (size_t i = 0; i < m; ++i) keys.push_back({start + (uint32_t)i, own_k + i * kvd, own_v + i * kvd});
  } else if (p->kv_donor_layer == p->donor_a_layer) {
    push(donor_a);
  } else if (p->kv_donor_layer == p->donor_b_layer) {
    push(donor_b);
  } else {
    return -1;
  }

  const size_t CHUNK = 256;  // :651
  for (size_t c0 = 0; c0 < m; c0 += CHUNK) {
    size_t n = std::min(CHUNK, m - c0);
    std::vector<int32_t> ctx(n * qd);
    std::vector<char> ok(n, 1);
    parallel_for(n, threads, 1, [&](size_t i) {  // attention_context :755-846
      uint32_t pos = start + (uint32_t)(c0 + i);
      const int32_t* qrow = &q[(c0 + i) * qd];
      uint32_t ws = window_start(pos, p->sliding_window);
      size_t wl = (size_t)(pos - ws) + 1;
      std::vector<int32_t> scores(wl * heads, 0);
      std::vector<const KeyRef*> visible;
      size_t filled = 0;
      for (const KeyRef& key : keys) {
        if (!is_visible(pos, key.position, p->sliding_window)) continue;
        if (key.position < ws) { ok[i] = 0; return; }
        size_t slot = key.position - ws;
        if (slot >= wl) { ok[i] = 0; return; }
        for (size_t h = 0; h < heads; ++h)
          scores[slot * heads + h] = dot_bits(qrow + h * d, key.k + (h / group) * d, d);
        visible.push_back(&key);
        ++filled;
      }
      if (filled != wl) { ok[i] = 0; return; }
      std::vector<int32_t> weights(scores), logits(wl), hw(wl);
      for (size_t h = 0; h < heads; ++h) {
        for (size_t s = 0; s < wl; ++s) logits[s] = scores[s * heads + h];
        attention_softmax(logits.data(), wl, hw.data());
        for (size_t s = 0; s < wl; ++s) weights[s * heads + h] = hw[s];
      }
      std::vector<int64_t> acc(qd, 0);
      for (const KeyRef* key : visible) {
        size_t slot = key->position - ws;
        for (size_t h = 0; h < heads; ++h) {
          int32_t w = weights[slot * heads + h];
          const int32_t* vh = key->v + (h / group) * d;
          for (size_t l = 0; l < d; ++l) acc[h * d + l] = mac_bits(acc[h * d + l], w, vh[l]);
        }
      }
      for (size_t j = 0; j < qd; ++j) ctx[i * qd + j] = requantize_acc(acc[j]);
    });
    for (char c : ok)
      if (!c) return -4;
    // attend_chunk (:692-741)
    std::vector<int32_t> attn(n * H);
    if (!linear(ctx.data(), n, qd, p->w_o, H, attn.data(), threads)) return -3;
    std::vector<int32_t> residual(n * H);
    for (size_t i = 0; i < n; ++i) {  // attn_residual :879-892
      int32_t* a = &attn[i * H];
      rms_norm_in_place(a, p->norm_post_attn, H, p->norm_eps);
      add_row(a, rows_in + (c0 + i) * H, H);
      std::memcpy(&residual[i * H], a, H * 4);
    }
    std::vector<int32_t> ff_in(residual);
    for (size_t i = 0; i < n; ++i) rms_norm_in_place(&ff_in[i * H], p->norm_pre_ffw, H, p->norm_eps);
    std::vector<int32_t> gate(n * F), up(n * F);
    if (!linear(ff_in.data(), n, H, p->w_gate, F, gate.data(), threads)) return -3;
    if (!linear(ff_in.data(), n, H, p->w_up, F, up.data(), threads)) return -3;
    for (size_t i = 0; i < n * F; ++i) gate[i] = mul_sat(gelu_pytorch_tanh_act(gate[i]), up[i]);
    std::vector<int32_t> ff(n * H);
    if (!linear(gate.data(), n, F, p->w_down, H, ff.data(), threads)) return -3;
    for (size_t i = 0; i < n; ++i) {  // finish_mlp :915-929
      rms_norm_in_place(&ff[i * H], p->norm_post_ffw, H, p->norm_eps);
      add_row(&ff[i * H], &residual[i * H], H);
    }
    std::vector<int32_t> pg(n * P);
    linear_dense(ff.data(), n, H, p->ple_input_gate, P, pg.data(), threads);
    for (size_t i = 0; i < n; ++i)  // ple_gate_mul :931-944
      for (size_t j = 0; j < P; ++j)
        pg[i * P + j] = mul_sat(gelu_pytorch_tanh_act(pg[i * P + j]), ple_rows[(c0 + i) * P + j]);
    std::vector<int32_t> proj(n * H);
    linear_dense(pg.data(), n, P, p->ple_layer_projection, H, proj.data(), threads);
    for (size_t i = 0; i < n; ++i) {  // finish_layer :946-957
      int32_t* x = &proj[i * H];
      rms_norm_in_place(x, p->ple_post_norm, H, p->norm_eps);
      add_row(x, &ff[i * H], H);
      if (p->layer_scalar != 0)
        for (size_t j = 0; j < H; ++j) x[j] = mul_sat(x[j], p->layer_scalar);
      std::memcpy(rows_out + (c0 + i) * H, x, H * 4);
    }
  }
  return 0;
}

// ---------------------------------------------------------------------------
// Head, PLE preparation and the decode loop: crates/inference/direct/src
// ---------------------------------------------------------------------------

int oracle_head_logits(const OracleHead* h, const int32_t* row, int32_t* logits, int threads) {
  size_t H = h->hidden;
  std::vector<int32_t> x(row, row + H);
  rms_norm_in_place(x.data(), h->norm, H, h->norm_eps);
  if (!linear(x.data(), 1, H, h->projection, h->vocab, logits, threads)) return -3;
  if (h->softcap > 0)  // sequence-check/src/input.rs:428-433
    for (size_t i = 0; i < h->vocab; ++i) logits[i] = softcap_act(logits[i], h->softcap);
  return 0;
}

int oracle_ple_prepare(const OraclePle* ple, uint32_t layers, uint32_t layer_idx,
                       const int32_t* embedded_row, uint32_t token_id, int32_t* out) {
  size_t P = ple->ple_width, H = ple->hidden;
  size_t start = (size_t)layer_idx * P;
  std::vector<int32_t> projected(P);
  for (size_t j = 0; j < P; ++j) projected[j] = dot_bits(embedded_row, ple->projection + (start + j) * H, H);
  for (size_t j = 0; j < P; ++j) projected[j] = mul_sat(projected[j], ple->projection_scalar);
  rms_norm_in_place(projected.data(), ple->norm, P, ple->norm_eps);
  size_t cols = (size_t)layers * P, rb;
  if (!row_bytes(cols, &rb) || start % Q8_BLOCK || P % Q8_BLOCK) return -1;
  const uint8_t* row = ple->embeddings + (size_t)token_id * rb + start / Q8_BLOCK * Q8_BLOCK_BYTES;
  if (!dequantize_row(row, P / Q8_BLOCK * Q8_BLOCK_BYTES, out, P)) return -3;
  for (size_t j = 0; j < P; ++j) out[j] = mul_sat(out[j], ple->embedding_scale);
  for (size_t j = 0; j < P; ++j) out[j] = add_sat(out[j], projected[j]);
  for (size_t j = 0; j < P; ++j) out[j] = mul_sat(out[j], ple->input_scale);
  return 0;
}

namespace {

struct LayerKv {  // one layer's published K/V list (ActivationSequence.kv)
  std::vector<uint32_t> pos;
  std::vector<int32_t> k, v;
  OracleKeys view() const { return {pos.size(), pos.data(), k.data(), v.data()}; }
};

int embed_rows(const OracleModel* m, const uint32_t* ids, size_t n, std::vector<int32_t>* out) {
  size_t H = m->hidden, rb;
  if (!row_bytes(H, &rb)) return -1;
  out->assign(n * H, 0);
  for (size_t i = 0; i < n; ++i) {  // model.rs:316-330
    if (ids[i] >= m->vocab) return -5;
    if (!dequantize_row(m->embed + (size_t)ids[i] * rb, rb, &(*out)[i * H], H)) return -3;
    if (m->family == 1)
      for (size_t j = 0; j < H; ++j) (*out)[i * H + j] = mul_sat((*out)[i * H + j], m->embedding_scale);
  }
  return 0;
}

// run_layers_and_logits (executor.rs:293-401) for either family. `prior` holds
// the previous pass's per-layer K/V lists (empty on the prompt pass).
int run_pass(const OracleModel* m, const std::vector<uint32_t>& ids, uint32_t start,
             std::vector<LayerKv>* layers_kv, int32_t* logits, int threads) {
  size_t H = m->hidden, n = ids.size();
  std::vector<int32_t> seed;
  int rc = embed_rows(m, ids.data(), n, &seed);
  if (rc) return rc;
  std::vector<int32_t> cur(seed), next(n * H);
  std::vector<LayerKv> outputs(m->layers);
  for (uint32_t l = 0; l < m->layers; ++l) {
    LayerKv& prior = (*layers_kv)[l];
    LayerKv& out = outputs[l];
    if (m->family == 0) {
      const OracleMistralLayer* p = &m->mistral[l];
      size_t kvd = (size_t)p->kv_heads * p->head_dim;
      if (prior.pos.size() != start) return -6;
      std::vector<int32_t> ok(n * kvd), ov(n * kvd);
      rc = oracle_mistral_layer(p, cur.data(), n, start, prior.k.data(), prior.v.data(), next.data(),
                                ok.data(), ov.data(), threads);
      if (rc) return rc;
      out = prior;  // view_kernels.rs:192-199: prior keys, then the range's own
      for (size_t i = 0; i < n; ++i) out.pos.push_back(start + (uint32_t)i);
      out.k.insert(out.k.end(), ok.begin(), ok.end());
      out.v.insert(out.v.end(), ov.begin(), ov.end());
    } else {
      const OracleGemmaLayer* p = &m->gemma[l];
      size_t kvd = (size_t)p->kv_heads * p->head_dim, P = p->ple_width;
      std::vector<int32_t> ple(n * P);
      for (size_t i = 0; i < n; ++i) {
        rc = oracle_ple_prepare(&m->ple, m->layers, l, &seed[i * H], ids[i], &ple[i * P]);
        if (rc) return rc;
      }
      LayerKv empty;
      const LayerKv& da = (p->donor_a_layer >= 0 && (uint32_t)p->donor_a_layer < l) ? outputs[p->donor_a_layer] : empty;
      const LayerKv& db = (p->donor_b_layer >= 0 && (uint32_t)p->donor_b_layer < l) ? outputs[p->donor_b_layer] : empty;
      std::vector<int32_t> ok(n * kvd), ov(n * kvd);
      rc = oracle_gemma_layer(p, cur.data(), n, start, prior.view(), da.view(), db.view(), ple.data(),
                              next.data(), ok.data(), ov.data(), threads);
      if (rc) return rc;
      // output_kv (prefill_range.rs:849-864)
      uint32_t keep_from = window_start(start, p->sliding_window);
      for (size_t i = 0; i < prior.pos.size(); ++i) {
        if (prior.pos[i] < keep_from) continue;
        out.pos.push_back(prior.pos[i]);
        out.k.insert(out.k.end(), prior.k.begin() + i * kvd, prior.k.begin() + (i + 1) * kvd);
        out.v.insert(out.v.end(), prior.v.begin() + i * kvd, prior.v.begin() + (i + 1) * kvd);
      }
      for (size_t i = 0; i < n; ++i) out.pos.push_back(start + (uint32_t)i);
      out.k.insert(out.k.end(), ok.begin(), ok.end());
      out.v.insert(out.v.end(), ov.begin(), ov.end());
    }
    std::swap(cur, next);
  }
  *layers_kv = std::move(outputs);
  return oracle_head_logits(&m->head, &cur[(n - 1) * H], logits, threads);
}

}  // namespace

int oracle_generate(const OracleModel* m, const uint32_t* prompt, size_t n_prompt,
                    uint32_t max_tokens, const uint32_t* eos, size_t n_eos, uint32_t* out_tokens,
                    uint32_t* out_count, int32_t* out_logits, int threads) {
  *out_count = 0;
  if (n_prompt == 0) return -7;
  std::vector<LayerKv> kv(m->layers);
  std::vector<int32_t> logits(m->vocab);
  std::vector<uint32_t> ids(prompt, prompt + n_prompt);
  int rc = run_pass(m, ids, 0, &kv, logits.data(), threads);
  if (rc) return rc;
  uint32_t position = (uint32_t)n_prompt;  // decode_position of the first selection
  size_t pass = 0;
  if (out_logits) std::memcpy(out_logits, logits.data(), m->vocab * 4);
  for (uint32_t t = 0; t < max_tokens; ++t) {
    size_t best = argmax_first(logits.data(), m->vocab);  // generation.rs:25-58: first max wins
    out_tokens[t] = (uint32_t)best;
    *out_count = t + 1;
    bool is_eos = false;
    for (size_t e = 0; e < n_eos; ++e) is_eos |= eos[e] == best;
    if (is_eos || t + 1 == max_tokens) break;
    std::vector<uint32_t> one{(uint32_t)best};
    rc = run_pass(m, one, position, &kv, logits.data(), threads);
    if (rc) return rc;
    ++position;
    ++pass;
    if (out_logits) std::memcpy(out_logits + pass * m->vocab, logits.data(), m->vocab * 4);
  }
  return 0;
}

}  // extern "C"
