// SHA-256 (FIPS 180-4) of byte strings held as little-endian 32-bit words,
// host and device: the leaf digests of the chain's stage records
// (iris_session_range_layer_leaves) are computed on the device where the
// stage's rows and K/V live, and the same code runs on the host in the
// tests. The constants are the standard's: the first 32 bits of the
// fractional parts of the square roots of the first 8 primes (initial
// hash) and of the cube roots of the first 64 primes (round constants).
#pragma once
#include <stdint.h>

#include "detnum.cuh"

namespace iris {

#define IRIS_SHA256_H0 0x6a09e667u, 0xbb67ae85u, 0x3c6ef372u, 0xa54ff53au, 0x510e527fu, 0x9b05688cu, 0x1f83d9abu, 0x5be0cd19u
#define IRIS_SHA256_K                                                                                            \
  0x428a2f98u, 0x71374491u, 0xb5c0fbcfu, 0xe9b5dba5u, 0x3956c25bu, 0x59f111f1u, 0x923f82a4u, 0xab1c5ed5u,        \
      0xd807aa98u, 0x12835b01u, 0x243185beu, 0x550c7dc3u, 0x72be5d74u, 0x80deb1feu, 0x9bdc06a7u, 0xc19bf174u,    \
      0xe49b69c1u, 0xefbe4786u, 0x0fc19dc6u, 0x240ca1ccu, 0x2de92c6fu, 0x4a7484aau, 0x5cb0a9dcu, 0x76f988dau,    \
      0x983e5152u, 0xa831c66du, 0xb00327c8u, 0xbf597fc7u, 0xc6e00bf3u, 0xd5a79147u, 0x06ca6351u, 0x14292967u,    \
      0x27b70a85u, 0x2e1b2138u, 0x4d2c6dfcu, 0x53380d13u, 0x650a7354u, 0x766a0abbu, 0x81c2c92eu, 0x92722c85u,    \
      0xa2bfe8a1u, 0xa81a664bu, 0xc24b8b70u, 0xc76c51a3u, 0xd192e819u, 0xd6990624u, 0xf40e3585u, 0x106aa070u,    \
      0x19a4c116u, 0x1e376c08u, 0x2748774cu, 0x34b0bcb5u, 0x391c0cb3u, 0x4ed8aa4au, 0x5b9cca4fu, 0x682e6ff3u,    \
      0x748f82eeu, 0x78a5636fu, 0x84c87814u, 0x8cc70208u, 0x90befffau, 0xa4506cebu, 0xbef9a3f7u, 0xc67178f2u

#if defined(__CUDACC__)
static __constant__ uint32_t kSha256KDev[64] = {IRIS_SHA256_K};
#endif
static const uint32_t kSha256KHost[64] = {IRIS_SHA256_K};

IRIS_HD uint32_t sha256_k(int i) {
#if defined(__CUDA_ARCH__)
  return kSha256KDev[i];
#else
  return kSha256KHost[i];
#endif
}

IRIS_HD uint32_t sha256_rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }
IRIS_HD uint32_t sha256_bswap(uint32_t x) {
  return (x >> 24) | ((x >> 8) & 0xFF00u) | ((x << 8) & 0xFF0000u) | (x << 24);
}

// One 64-byte block, w: its sixteen big-endian words (overwritten: the
// message schedule runs in place over a sixteen-word window).
IRIS_HD void sha256_block(uint32_t (&h)[8], uint32_t (&w)[16]) {
  uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], hh = h[7];
#pragma unroll
  for (int i = 0; i < 64; ++i) {
    if (i >= 16) {
      const uint32_t x = w[(i + 1) & 15], y = w[(i + 14) & 15];
      const uint32_t s0 = sha256_rotr(x, 7) ^ sha256_rotr(x, 18) ^ (x >> 3);
      const uint32_t s1 = sha256_rotr(y, 17) ^ sha256_rotr(y, 19) ^ (y >> 10);
      w[i & 15] += s0 + w[(i + 9) & 15] + s1;
    }
    const uint32_t S1 = sha256_rotr(e, 6) ^ sha256_rotr(e, 11) ^ sha256_rotr(e, 25);
    const uint32_t ch = (e & f) ^ (~e & g);
    const uint32_t t1 = hh + S1 + ch + sha256_k(i) + w[i & 15];
    const uint32_t S0 = sha256_rotr(a, 2) ^ sha256_rotr(a, 13) ^ sha256_rotr(a, 22);
    const uint32_t maj = (a & b) ^ (a & c) ^ (b & c);
    hh = g;
    g = f;
    f = e;
    e = d + t1;
    d = c;
    c = b;
    b = a;
    a = t1 + S0 + maj;
  }
  h[0] += a, h[1] += b, h[2] += c, h[3] += d, h[4] += e, h[5] += f, h[6] += g, h[7] += hh;
}

// SHA-256 of `bytes` bytes (a multiple of 4) at p, 16-byte aligned, read as
// 32-bit words in memory order; the digest as 32 bytes at out.
IRIS_HD void sha256_words(const uint32_t* p, uint32_t bytes, uint8_t* out) {
  uint32_t h[8] = {IRIS_SHA256_H0};
  uint32_t w[16];
  const uint32_t full = bytes / 64;
  for (uint32_t blk = 0; blk < full; ++blk) {
    const uint32_t* q = p + blk * 16;
#if defined(__CUDA_ARCH__)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint4 v = ((const uint4*)q)[j];
      w[4 * j] = sha256_bswap(v.x), w[4 * j + 1] = sha256_bswap(v.y);
      w[4 * j + 2] = sha256_bswap(v.z), w[4 * j + 3] = sha256_bswap(v.w);
    }
#else
    for (int j = 0; j < 16; ++j) w[j] = sha256_bswap(q[j]);
#endif
    sha256_block(h, w);
  }
  // the tail: the last rest / 4 words, the 0x80 marker word, zeros and the
  // bit length (one block, or two when the marker lands in words 14-15)
  const uint32_t rest = (bytes % 64) / 4;
  const uint32_t* q = p + full * 16;
#pragma unroll
  for (uint32_t j = 0; j < 16; ++j) w[j] = j < rest ? sha256_bswap(q[j]) : j == rest ? 0x80000000u : 0u;
  const uint64_t bits = (uint64_t)bytes * 8;
  if (rest >= 14) {
    sha256_block(h, w);
#pragma unroll
    for (uint32_t j = 0; j < 16; ++j) w[j] = 0;
  }
  w[14] = (uint32_t)(bits >> 32);
  w[15] = (uint32_t)bits;
  sha256_block(h, w);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    out[4 * j] = (uint8_t)(h[j] >> 24);
    out[4 * j + 1] = (uint8_t)(h[j] >> 16);
    out[4 * j + 2] = (uint8_t)(h[j] >> 8);
    out[4 * j + 3] = (uint8_t)h[j];
  }
}

}  // namespace iris
