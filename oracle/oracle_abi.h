// TEST INFRASTRUCTURE ONLY. C ABI of the CPU oracle, loaded with ctypes by
// tests/, by __graft_entry__.smoke() and by bench.py's CPU baseline leg.
// Nothing in iris_b200/ includes or links this.
//
// Weight matrices are raw Q8_0 rows exactly as GGUF / DETWGT v3 store them
// (34-byte blocks: little-endian fp16 scale bits, then 32 int8 values),
// `rows * cols / 32 * 34` bytes, row after row (crates/det-num/src/q8.rs:1-19).
// Norm weights and dense matrices are Q16.16 int32 values.
#pragma once
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

// mistral-dense layer parameters and matrices
// (crates/inference/kernels/src/mistral/layer.rs:22-50).
typedef struct {
  uint32_t hidden, ffn, heads, kv_heads, head_dim, max_positions;
  int64_t norm_eps;
  uint32_t attention_scale_q32;
  uint32_t n_freqs;
  const int64_t* rope_freqs;
  const int32_t* norm_attention;
  const int32_t* norm_feed_forward;
  const uint8_t *w_q, *w_k, *w_v, *w_o, *w_gate, *w_up, *w_down;
} OracleMistralLayer;

// gemma-dense layer parameters and matrices
// (raster-stages/prefill-range/src/input.rs:106-160 LayerParams, TransformerLayer).
typedef struct {
  uint32_t hidden, ffn, heads, kv_heads, head_dim, sliding_window;
  int32_t attn_scale, layer_scalar;
  int64_t norm_eps, rope_base;
  uint32_t rotary_dim, rope_freq_base_dim;
  int32_t kv_donor_layer, donor_a_layer, donor_b_layer;
  uint32_t ple_width;
  const int32_t *norm_input, *norm_post_attn, *norm_pre_ffw, *norm_post_ffw, *q_norm, *k_norm,
      *ple_post_norm;
  const uint8_t *w_q, *w_k, *w_v, *w_o, *w_gate, *w_up, *w_down;
  const int32_t* ple_input_gate;        // [ple_width][hidden] dense Q16.16
  const int32_t* ple_layer_projection;  // [hidden][ple_width] dense Q16.16
} OracleGemmaLayer;

// The final head (crates/inference/direct/src/view_kernels.rs:203-230).
typedef struct {
  uint32_t hidden, vocab;
  int64_t norm_eps;
  int32_t softcap;  // 0 disables (sequence-check/src/input.rs:428-433)
  const int32_t* norm;
  const uint8_t* projection;  // [vocab][hidden] Q8_0
} OracleHead;

// Gemma per-layer-input preparation (direct/src/view_kernels.rs:59-99).
typedef struct {
  uint32_t hidden, ple_width;
  int32_t embedding_scale, projection_scalar, input_scale;
  int64_t norm_eps;
  const int32_t* norm;          // [ple_width]
  const uint8_t* embeddings;    // [vocab][layers * ple_width] Q8_0
  const int32_t* projection;    // [layers * ple_width][hidden] dense Q16.16
} OraclePle;

typedef struct {
  uint32_t family;  // 0 = mistral-dense, 1 = gemma-dense
  uint32_t layers, hidden, vocab;
  int32_t embedding_scale;  // gemma only (direct/src/model.rs:316-330)
  const uint8_t* embed;     // [vocab][hidden] Q8_0
  const OracleMistralLayer* mistral;  // [layers] when family == 0
  const OracleGemmaLayer* gemma;      // [layers] when family == 1
  OracleHead head;
  OraclePle ple;
} OracleModel;

// Scalar det-num functions (for the known-answer tests).
int32_t oracle_requantize(int64_t x);
int64_t oracle_rshift_round_ties_even(int64_t x, uint32_t shift);
int64_t oracle_mac_bits(int64_t acc, int32_t a, int32_t b);
int32_t oracle_add_sat(int32_t a, int32_t b);
int32_t oracle_sub_sat(int32_t a, int32_t b);
int32_t oracle_mul_sat(int32_t a, int32_t b);
int32_t oracle_div_act(int32_t a, int32_t b);
int64_t oracle_div_acc(int64_t a, int64_t b);
int64_t oracle_acc_mul(int64_t a, int64_t b);
int32_t oracle_inv_sqrt_acc(int64_t x);
int32_t oracle_tanh(int32_t x);
int32_t oracle_gelu(int32_t x);
int32_t oracle_softcap(int32_t x, int32_t cap);
int64_t oracle_softmax_exp_term(int64_t delta);
int32_t oracle_silu(int32_t x);
uint64_t oracle_sigmoid_q32(int32_t x);
uint64_t oracle_exp_neg_q32(uint64_t a);
void oracle_sin_cos_q30(int64_t angle, int64_t* sin_out, int64_t* cos_out);
void oracle_sin_cos_acc(int64_t angle, int32_t* cos_out, int32_t* sin_out);
int64_t oracle_rope_frequency_step(int64_t base, uint32_t freq_base_dim);
int64_t oracle_nth_root_acc(int64_t value, uint32_t degree);
uint32_t oracle_attention_scale_q32(uint32_t head_dim);
int oracle_yarn_inverse_frequencies(uint64_t base, uint32_t pairs, uint32_t factor, uint32_t low,
                                    uint32_t high, int64_t* out);
int32_t oracle_scaled_score(const int32_t* q, const int32_t* k, size_t n, uint32_t scale);
int32_t oracle_dot_bits(const int32_t* a, const int32_t* b, size_t n);
int32_t oracle_f32_to_act(float x);
int64_t oracle_f32_to_acc(float x);
int oracle_scale_q24(uint16_t bits, int64_t* out);
int oracle_dot_row(const int32_t* act, size_t cols, const uint8_t* row, size_t row_len,
                   int32_t* out);
int oracle_dequantize_row(const uint8_t* row, size_t row_len, int32_t* out, size_t cols);

// Row kernels, in place.
void oracle_rms_norm(int32_t* v, const int32_t* w, size_t n, int64_t eps);
void oracle_value_rms_norm(int32_t* v, size_t n, int64_t eps);
int32_t oracle_rms_norm_scale(const int32_t* v, size_t n, int64_t eps);
void oracle_rope_rotate_pairs(int32_t* v, size_t n, size_t rotary_dim, size_t freq_base_dim,
                              int64_t base, size_t position);
void oracle_rotate_consecutive_pairs(int32_t* v, size_t n, const int64_t* freqs, size_t n_freqs,
                                     uint32_t position);
void oracle_attention_softmax(const int32_t* logits, size_t n, int32_t* weights);

// Products: out[t*rows + r] = dot_row(in[t], q8 row r)
// (crates/inference/kernels/src/tensor.rs:437-520). Returns 0, or -1 when a
// row is malformed or a scale is not finite.
int oracle_linear(const int32_t* in, size_t tokens, size_t cols, const uint8_t* q8, size_t rows,
                  int32_t* out, int threads);
// Dense Q16.16 product, dot_bits per value (tensor.rs:522-528).
int oracle_linear_dense(const int32_t* in, size_t tokens, size_t cols, const int32_t* w,
                        size_t rows, int32_t* out, int threads);

// One mistral-dense layer over M rows starting at `start`
// (mistral/layer.rs:107-270). prior_k/prior_v hold `start` rows of
// kv_heads*head_dim values (positions 0..start). Returns 0, or a negative
// code: -1 bad params, -2 position past max_positions, -3 malformed weights.
int oracle_mistral_layer(const OracleMistralLayer* layer, const int32_t* rows_in, size_t m,
                         uint32_t start, const int32_t* prior_k, const int32_t* prior_v,
                         int32_t* rows_out, int32_t* own_k, int32_t* own_v, int threads);

// A list of KeyRows: n rows with their positions, k and v of kv_dim values each.
typedef struct {
  size_t n;
  const uint32_t* positions;
  const int32_t* k;
  const int32_t* v;
} OracleKeys;

// One gemma-dense layer over M rows (prefill_range.rs:307-333). ple_rows is
// [M][ple_width]. Returns 0 or a negative code.
int oracle_gemma_layer(const OracleGemmaLayer* layer, const int32_t* rows_in, size_t m,
                       uint32_t start, OracleKeys prior, OracleKeys donor_a, OracleKeys donor_b,
                       const int32_t* ple_rows, int32_t* rows_out, int32_t* own_k, int32_t* own_v,
                       int threads);

// The head's logits for one final row (view_kernels.rs:203-230).
int oracle_head_logits(const OracleHead* head, const int32_t* row, int32_t* logits, int threads);

// One PLE row for one token at one layer (view_kernels.rs:59-99).
int oracle_ple_prepare(const OraclePle* ple, uint32_t layers, uint32_t layer_idx,
                       const int32_t* embedded_row, uint32_t token_id, int32_t* out);

// The direct decode loop (direct/src/executor.rs:136-186): prefill over the
// prompt, then up to max_tokens greedy selections. Writes the selected ids to
// out_tokens (max_tokens entries), their count to *out_count, and, when
// out_logits is not NULL, each pass's logits ([passes][vocab]; pass p scores
// token p). Returns 0 or a negative code.
int oracle_generate(const OracleModel* model, const uint32_t* prompt, size_t n_prompt,
                    uint32_t max_tokens, const uint32_t* eos, size_t n_eos, uint32_t* out_tokens,
                    uint32_t* out_count, int32_t* out_logits, int threads);

// Seeded synthetic weights of the benchmark configurations (synth.cc): Q8_0
// blocks of a rows x cols tensor, or count dense / norm values (fan_in 0:
// norm weights). `tensor` is the tensor's id in the generator's numbering,
// `layer` -1 for model-level tensors. Returns 0, or -1 on a bad shape.
int oracle_synth_q8(uint64_t seed, uint32_t tensor, int32_t layer, uint32_t rows, uint32_t cols,
                    int per_block_scales, uint8_t* blocks, int threads);
int oracle_synth_values(uint64_t seed, uint32_t tensor, int32_t layer, uint64_t count, uint32_t fan_in,
                        int32_t* values, int threads);

#ifdef __cplusplus
}
#endif
