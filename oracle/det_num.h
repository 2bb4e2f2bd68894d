// TEST INFRASTRUCTURE ONLY. This is the CPU oracle: a line-by-line C++
// restatement of the reference's `det-num` crate, used by tests/, by
// `__graft_entry__.smoke()` and by bench.py's CPU baseline leg as the checker.
// The product (iris_b200/) never links or calls it.
//
// Parity pin: every known-answer test of the reference for this path is
// replayed against these functions in tests/test_oracle_kat.py (literal values
// from crates/det-num/tests/golden_vectors.rs, crates/det-num/src/q8.rs tests,
// crates/det-num/src/mistral.rs tests, crates/det-num/src/convert.rs tests and
// the RoPE answer [35408, 55146] of crates/inference/direct/tests/executor.rs).
//
// Types: Q16.16 activations are int32_t bits, Q32.32 accumulators int64_t
// bits (crates/det-num/src/types.rs:1-25).
#pragma once
#include <cstddef>
#include <cstdint>
#include <vector>

namespace oracle {

typedef __int128 i128;
typedef unsigned __int128 u128;

// ---- crates/det-num/src/ops.rs ------------------------------------------
int64_t mac_bits(int64_t acc, int32_t a, int32_t b);            // ops.rs:17-19
int32_t add_sat(int32_t a, int32_t b);                           // ops.rs:36-38
int32_t sub_sat(int32_t a, int32_t b);                           // ops.rs:431-433
int64_t acc_add_sat(int64_t a, int64_t b);                       // ops.rs:436-438
int32_t mul_sat(int32_t a, int32_t b);                           // ops.rs:41-45
int32_t div_act(int32_t num, int32_t den);                       // ops.rs:53-64
int64_t div_acc(int64_t num, int64_t den);                       // ops.rs:67-78
int64_t div_acc_by_u32(int64_t value, uint32_t divisor);         // ops.rs:81-88
int64_t rshift_round_ties_even(int64_t x, uint32_t shift);       // ops.rs:443-445, 773-803
int32_t requantize(int64_t x);                                   // ops.rs:448-451
size_t argmax_first(const int32_t* xs, size_t n);                // ops.rs:466-481
int64_t acc_mul(int64_t a, int64_t b);                           // ops.rs:685-689
i128 round_ties_even_division(i128 dividend, i128 divisor);      // ops.rs:691-720
int32_t inv_sqrt_acc(int64_t x);                                 // ops.rs:722-771
int32_t rms_norm_scale(const int32_t* v, size_t n, int64_t eps); // ops.rs:409-428
void rms_norm_in_place(int32_t* v, const int32_t* w, size_t n, int64_t eps);  // ops.rs:98-114
void value_rms_norm_in_place(int32_t* v, size_t n, int64_t eps);              // ops.rs:124-134
void rope_rotate_pairs_in_place(int32_t* v, size_t n, size_t rotary_dim, size_t freq_base_dim,
                                int64_t base, size_t position);  // ops.rs:154-199
int64_t rope_frequency_step(int64_t base, size_t freq_base_dim);  // ops.rs:558-562
int64_t nth_root_acc(int64_t value, uint32_t degree);             // ops.rs:564-606
void sin_cos_acc(int64_t angle, int32_t* cos_out, int32_t* sin_out);  // ops.rs:622-649
int64_t softmax_exp_term(int64_t delta);                          // ops.rs:508-556
int64_t attention_softmax_exp_term(int32_t logit, int32_t max_logit);  // ops.rs:264-266
void attention_softmax(const int32_t* logits, size_t n, int32_t* weights);  // ops.rs:233-261
int32_t tanh_act(int32_t x);                                      // ops.rs:357-377
int32_t softcap_act(int32_t x, int32_t cap);                      // ops.rs:380-388
int32_t gelu_pytorch_tanh_act(int32_t x);                         // ops.rs:391-406

// ---- crates/det-num/src/q8.rs ------------------------------------------
const size_t Q8_BLOCK = 32;
const size_t Q8_BLOCK_BYTES = 34;
bool row_bytes(size_t cols, size_t* out);                         // q8.rs:21-23
bool scale_q24(uint16_t bits, int64_t* out);                      // q8.rs:27-43
int32_t round_to_i32(i128 value, uint32_t shift);                 // q8.rs:94-104
// Returns false (the reference's Err) on a width mismatch or a non-finite scale.
bool dot_row(const int32_t* act, size_t cols, const uint8_t* row, size_t row_len,
             int32_t* out);                                       // q8.rs:56-72
bool dequantize_row(const uint8_t* row, size_t row_len, int32_t* out, size_t cols);  // q8.rs:76-91

// ---- crates/det-num/src/mistral.rs -------------------------------------
uint64_t exp_neg_q32(uint64_t a);                                 // mistral.rs:43-56
uint64_t sigmoid_q32(int32_t x);                                  // mistral.rs:59-69
int32_t silu(int32_t x);                                          // mistral.rs:72-77
void sin_cos_q30(int64_t angle, int64_t* sin_out, int64_t* cos_out);  // mistral.rs:84-110
void rotate_consecutive_pairs(int32_t* v, size_t n, const int64_t* freqs, size_t n_freqs,
                              uint32_t position);                 // mistral.rs:114-128
int32_t scaled_score(const int32_t* q, const int32_t* k, size_t n, uint32_t scale_q32);  // :130-145
uint32_t attention_scale_q32(uint32_t head_dim);                  // mistral.rs:148-160
bool yarn_inverse_frequencies(uint64_t base, uint32_t pairs, uint32_t factor, uint32_t low,
                              uint32_t high, std::vector<int64_t>* out);  // mistral.rs:185-214

// ---- crates/det-num/src/convert.rs -------------------------------------
int32_t f32_to_act(float x);                                      // convert.rs:4-7
int64_t f32_to_acc(float x);                                      // convert.rs:10-13

// ---- crates/inference/kernels/src/tensor.rs -----------------------------
int32_t dot_bits(const int32_t* a, const int32_t* b, size_t n);   // tensor.rs:522-528
int32_t requantize_acc(int64_t acc);                              // tensor.rs:534-536

}  // namespace oracle
