// Seeded synthetic weights for the benchmark configurations.
//
// The recipe follows the reference's parity bundles
// (model-bundles/parity-mistral/generate.py:87-160): Q8_0 weights uniform in
// [-127, 127], fp16 block scales near a base value plus a small random offset
// (0..63 in the scale's bit pattern), and Q16.16 norm weights 1.0 +/- 0.125.
// It departs from it in one respect, on purpose: values come from a
// counter-based hash of (seed, tensor, layer, index) instead of one sequential
// xorshift stream, so that the device can generate a 7 GB model in parallel
// and the host can regenerate any single row bit-identically (both compile
// this header). Scales are one value per output row, replicated into every
// block of that row ("per-output-row scales"), or, when per_block is set, one
// random value per block (the parity bundles' choice).
#pragma once
#include <stdint.h>

#include "detnum.cuh"

namespace iris {

IRIS_HD uint64_t synth_mix(uint64_t x) {  // splitmix64 finaliser
  x ^= x >> 30;
  x *= 0xBF58476D1CE4E5B9ull;
  x ^= x >> 27;
  x *= 0x94D049BB133111EBull;
  x ^= x >> 31;
  return x;
}
IRIS_HD uint64_t synth_hash(uint64_t seed, uint32_t tensor, int32_t layer, uint64_t index) {
  uint64_t h = synth_mix(seed ^ 0x9E3779B97F4A7C15ull);
  h = synth_mix(h ^ ((uint64_t)tensor << 40) ^ ((uint64_t)(uint32_t)(layer + 1) << 8));
  return synth_mix(h + index * 0xD1B54A32D192ED03ull);
}

// fp16 bits of a power of two within a factor of sqrt(2) of
// 1 / (73.3 * sqrt(cols)): keeps a product's output RMS near its input RMS for
// uniform [-127,127] weights.
IRIS_HD uint16_t synth_scale_base(uint32_t cols) {
  // 1/(73.3 sqrt(c)) = 2^-(log2(73.3) + log2(c)/2); log2(73.3) ~ 6.196
  uint32_t lg = 0;
  while ((1u << (lg + 1)) <= cols) ++lg;  // floor(log2(cols))
  int32_t exp2 = -(int32_t)(6 + (lg + 1) / 2);
  int32_t biased = exp2 + 15;
  if (biased < 1) biased = 1;
  return (uint16_t)(biased << 10);
}

// Block b (0-based within the row) of row r: its scale bits.
IRIS_HD uint16_t synth_scale_bits(uint64_t seed, uint32_t tensor, int32_t layer, uint32_t row,
                                  uint32_t block, uint32_t cols, int per_block) {
  uint64_t idx = per_block ? ((uint64_t)row * (cols / 32) + block) : (uint64_t)row;
  uint64_t h = synth_hash(seed, tensor | 0x80000000u, layer, idx);
  return (uint16_t)(synth_scale_base(cols) + (uint16_t)(h % 64));
}
// Weight (row, col) as int8 in [-127, 127].
IRIS_HD int8_t synth_q(uint64_t seed, uint32_t tensor, int32_t layer, uint32_t row, uint32_t col,
                       uint32_t cols) {
  uint64_t h = synth_hash(seed, tensor, layer, (uint64_t)row * cols + col);
  return (int8_t)((int32_t)(h % 255) - 127);
}
// Dense Q16.16 value: norm vectors (fan_in == 0) are 1.0 +/- 0.125; matrices
// are uniform with RMS near 1/sqrt(fan_in), never zero (generate.py:98-103).
IRIS_HD int32_t synth_value(uint64_t seed, uint32_t tensor, int32_t layer, uint64_t index,
                            uint32_t fan_in) {
  uint64_t h = synth_hash(seed, tensor, layer, index);
  if (fan_in == 0) return kOneAct + (int32_t)(h % 16384) - 8192;
  uint32_t lg = 0;
  while ((1u << (lg + 1)) <= fan_in) ++lg;
  int32_t amp = (int32_t)(113512u >> ((lg + 1) / 2));  // ~sqrt(3) * 2^16 / sqrt(fan_in)
  if (amp < 2) amp = 2;
  int32_t v = (int32_t)(h % (uint64_t)(2 * amp)) - amp;
  return v ? v : 1;
}

}  // namespace iris
