// TEST INFRASTRUCTURE ONLY: the seeded synthetic weights of the benchmark
// configurations, generated on the host for the CPU legs (bench.py's
// reference arm and CPU baseline, the tests) without loading the product
// library. It is the same counter-based generator the product uses for
// iris_model_synthesize, restated here so that both sides hold the same
// bytes; tests/test_oracle_synth.py checks the two agree byte for byte.
//
// Recipe (after the reference's model-bundles/parity-mistral/generate.py:87-160):
// Q8_0 weights uniform in [-127, 127]; fp16 block scales at a base near
// 1 / (73.3 sqrt(cols)) plus 0..63 in the bit pattern, one value per output
// row replicated into every block of the row (per-output-row scales) or one
// per block; Q16.16 norm weights 1.0 +/- 0.125; dense matrices uniform with
// RMS near 1 / sqrt(fan_in). Each value is a splitmix64 hash of (seed,
// tensor id, layer, index), so any row can be generated independently.
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <thread>
#include <vector>

#include "oracle_abi.h"

namespace {

uint64_t mix(uint64_t x) {
  x ^= x >> 30;
  x *= 0xBF58476D1CE4E5B9ull;
  x ^= x >> 27;
  x *= 0x94D049BB133111EBull;
  x ^= x >> 31;
  return x;
}

// The hash of element `index` of tensor `tensor` in layer `layer` (-1 for
// model-level tensors).
struct Stream {
  uint64_t base;
  Stream(uint64_t seed, uint32_t tensor, int32_t layer) {
    uint64_t h = mix(seed ^ 0x9E3779B97F4A7C15ull);
    base = mix(h ^ ((uint64_t)tensor << 40) ^ ((uint64_t)(uint32_t)(layer + 1) << 8));
  }
  uint64_t at(uint64_t index) const { return mix(base + index * 0xD1B54A32D192ED03ull); }
};

uint32_t floor_log2(uint32_t v) {
  uint32_t lg = 0;
  while ((1u << (lg + 1)) <= v) ++lg;
  return lg;
}

// fp16 bits of the power of two nearest 1 / (73.3 sqrt(cols)) from below
// (2^-(6 + (floor(log2 cols) + 1) / 2)), the exponent field clamped at 1.
uint16_t scale_base(uint32_t cols) {
  int32_t biased = 15 - (int32_t)(6 + (floor_log2(cols) + 1) / 2);
  return (uint16_t)(std::max(biased, 1) << 10);
}

template <class F>
void parallel_rows(uint64_t rows, int threads, F&& body) {
  const uint64_t n = std::max(1, threads);
  if (n == 1 || rows < 64) {
    body(0, rows);
    return;
  }
  std::vector<std::thread> pool;
  for (uint64_t t = 0; t < n; ++t) {
    const uint64_t b = rows * t / n, e = rows * (t + 1) / n;
    if (b < e) pool.emplace_back([&body, b, e] { body(b, e); });
  }
  for (auto& th : pool) th.join();
}

}  // namespace

extern "C" {

int oracle_synth_q8(uint64_t seed, uint32_t tensor, int32_t layer, uint32_t rows, uint32_t cols,
                    int per_block_scales, uint8_t* blocks, int threads) {
  if (cols == 0 || cols % 32 || !blocks) return -1;
  const uint32_t nb = cols / 32;
  const Stream q(seed, tensor, layer), s(seed, tensor | 0x80000000u, layer);
  const uint16_t base = scale_base(cols);
  parallel_rows(rows, threads, [&](uint64_t r0, uint64_t r1) {
    for (uint64_t r = r0; r < r1; ++r) {
      const uint16_t row_bits = (uint16_t)(base + s.at(r) % 64);
      for (uint32_t b = 0; b < nb; ++b) {
        uint8_t* dst = blocks + (r * nb + b) * 34;
        const uint16_t bits = per_block_scales ? (uint16_t)(base + s.at(r * nb + b) % 64) : row_bits;
        dst[0] = (uint8_t)bits;
        dst[1] = (uint8_t)(bits >> 8);
        for (uint32_t j = 0; j < 32; ++j)
          dst[2 + j] = (uint8_t)(int8_t)((int32_t)(q.at(r * cols + b * 32 + j) % 255) - 127);
      }
    }
  });
  return 0;
}

int oracle_synth_values(uint64_t seed, uint32_t tensor, int32_t layer, uint64_t count, uint32_t fan_in,
                        int32_t* values, int threads) {
  if (!values && count) return -1;
  const Stream h(seed, tensor, layer);
  int32_t amp = 0;
  if (fan_in) amp = std::max<int32_t>(2, (int32_t)(113512u >> ((floor_log2(fan_in) + 1) / 2)));
  parallel_rows(count, threads, [&](uint64_t i0, uint64_t i1) {
    for (uint64_t i = i0; i < i1; ++i) {
      const uint64_t x = h.at(i);
      if (!fan_in) {
        values[i] = 65536 + (int32_t)(x % 16384) - 8192;  // 1.0 +/- 0.125
      } else {
        const int32_t v = (int32_t)(x % (uint64_t)(2 * amp)) - amp;
        values[i] = v ? v : 1;
      }
    }
  });
  return 0;
}

}  // extern "C"
