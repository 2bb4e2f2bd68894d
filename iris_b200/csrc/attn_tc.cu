// Prefill attention on the tcgen05 tensor cores (kind::i8), exact.
//
// attention_softmax (ops.rs:233-276) over a range of queries with the
// scores (mistral.rs:130-145) and the weighted value sums
// (tensor.rs:530-536) as byte-plane contractions:
//   1. scores: S[h][q][t] = finish_score(sum_d q[d] k[t][d]). q and k are
//      Q16.16 (four byte planes each, planes 0-2 unsigned, 3 signed), so the
//      dot product is sum_{i,j} 2^(8 (i + j)) sum_d k_i[d] q_j[d]: sixteen
//      int8 MMAs (M = 128 keys, N = 64 queries, K = 32 of the 128 dims) into
//      seven int32 diagonals, each exact (|sum| < 2^26 over 128 dims); the
//      epilogue adds them modulo 2^64, as the reference's wrapping sum.
//   2. softmax on CUDA cores, one warp a (query, head): first maximum, exp
//      terms and their sum, weights by one exact reciprocal, the residual
//      1.0 - sum(weights) on the first maximum's weight; the weights
//      (0..65536) are written as three byte planes, zero past the query's
//      position (the causal mask).
//   3. values: ctx[q][h][d] = requantize(sum_t w[q][t] v[t][d]): twelve MMAs
//      (M = 128 dims from the transposed value planes, N = 64 queries, K = the
//      positions) into six diagonals; a diagonal's true sum lies in
//      [L_s, L_s + 2^32) (L_s from the positions and the operand signs), so
//      its wrapped int32 value gives it back exactly up to 22,016 positions.
// The two contractions run the same persistent pipeline as q8_gemm_tc_kernel
// (TMA producer lane, MMA lane, 16 epilogue warps that release the
// accumulators before their arithmetic). Operands are packed per layer range
// into K-major byte planes: queries [h][plane][q][d], keys [g][plane][t][d],
// values transposed [g][plane][d][t], weights [h][plane][q][t].
#include <algorithm>
#include <mutex>

#include "../../include/iris_b200.h"
#include "common.cuh"
#include "detnum.cuh"
#include "layers.cuh"
#include "q8.cuh"
#include "tc.cuh"
#include "tcgen05.cuh"

namespace iris {

namespace {

constexpr uint32_t kAtD = 128;  // head dim these kernels take
constexpr uint32_t kAtEpiWarps = 16;
constexpr uint32_t kAtThreads = 32 * (2 + kAtEpiWarps);
constexpr uint32_t kAtAPlane = kTcTileM * kTcTileK, kAtBPlane = kTcTileN * kTcTileK;
constexpr uint32_t kAtStages = 2;
constexpr uint32_t kAtMaxPositions = 22016;

// Lower bound of one position's contribution to a value-sum diagonal s
// (value planes i: 0-2 unsigned, 3 signed; weight planes j: 0-1 unsigned,
// 2 holds 0 or 1).
__host__ __device__ constexpr int64_t pv_diag_min(uint32_t s) { return s == 3 || s == 4 ? -32640 : s == 5 ? -128 : 0; }

struct ScoreTiles {  // tile = (head, query tile, key tile); one K stage (the 128 dims)
  uint32_t heads, group, qtiles, ktiles;
  __device__ uint32_t count() const { return heads * qtiles * ktiles; }
  __device__ uint32_t nk(uint32_t) const { return 1; }
  __device__ void a_coord(uint32_t t, uint32_t, uint32_t i, int32_t* c) const {  // keys [g][plane][t][d]
    const uint32_t h = t / (qtiles * ktiles), kt = t % ktiles;
    c[0] = 0, c[1] = (int32_t)(kt * kTcTileM), c[2] = (int32_t)((h / group) * 4 + i);
  }
  __device__ void b_coord(uint32_t t, uint32_t, uint32_t j, int32_t* c) const {  // queries [h][plane][q][d]
    const uint32_t h = t / (qtiles * ktiles), qt = (t / ktiles) % qtiles;
    c[0] = 0, c[1] = (int32_t)(qt * kTcTileN), c[2] = (int32_t)(h * 4 + j);
  }
};

struct ValueTiles {  // tile = (head, query tile); K stages over the positions
  uint32_t heads, group, qtiles, kstages;
  __device__ uint32_t count() const { return heads * qtiles; }
  __device__ uint32_t nk(uint32_t) const { return kstages; }
  __device__ void a_coord(uint32_t t, uint32_t kt, uint32_t i, int32_t* c) const {  // values [g][plane][d][t]
    const uint32_t h = t / qtiles;
    c[0] = (int32_t)(kt * kTcTileK), c[1] = 0, c[2] = (int32_t)((h / group) * 4 + i);
  }
  __device__ void b_coord(uint32_t t, uint32_t kt, uint32_t j, int32_t* c) const {  // weights [h][plane][q][t]
    const uint32_t h = t / qtiles, qt = t % qtiles;
    c[0] = (int32_t)(kt * kTcTileK), c[1] = (int32_t)(qt * kTcTileN), c[2] = (int32_t)(h * 3 + j);
  }
};

// The persistent tensor-core pipeline over a problem's tiles: NA planes of A
// (M = 128 rows) against NB planes of B (N = 64 columns), pair (i, j) into
// diagonal i + j. Epi::value turns the diagonals' raw int32 values of one
// (TMEM lane row, column) into the output, Epi::store writes it (after the
// accumulators are released).
template <uint32_t NA, uint32_t NB, class Tiles, class Epi>
__device__ __forceinline__ void at_pipeline(const Tiles& tiles, const Epi& epi, const CUtensorMap* amap,
                                            const CUtensorMap* bmap, unsigned int* fault, uint8_t* ring) {
  constexpr uint32_t ND = NA + NB - 1, kStage = NA * kAtAPlane + NB * kAtBPlane;
  static_assert(ND * kTcTileN <= 512, "TMEM columns");
  __shared__ __align__(8) uint64_t full[kAtStages], empty[kAtStages], done, tfree;
  __shared__ uint32_t tmem_slot;
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t ntiles = tiles.count();
  if (threadIdx.x == 0) {
    for (uint32_t s = 0; s < kAtStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&done, 1);
    mbar_init(&tfree, kAtEpiWarps);
    mbar_fence_init();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&tmem_slot)),
                 "r"(512u)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  pdl_wait();
  pdl_trigger();

  if (warp == 0) {
    if (lane == 0) {  // producer
      uint32_t issued[kAtStages] = {};
      uint32_t G = 0;
      bool ok = true;
      for (uint32_t t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
        const uint32_t nk = tiles.nk(t);
        for (uint32_t kt = 0; kt < nk; ++kt, ++G) {
          const uint32_t s = G % kAtStages, use = G / kAtStages;
          if (use > 0 && !mbar_wait_bounded(&empty[s], (use - 1) & 1, fault)) {
            ok = false;
            break;
          }
          uint8_t* st = ring + s * kStage;
          mbar_arrive_expect_tx(&full[s], kStage);
          int32_t c[3];
#pragma unroll
          for (uint32_t i = 0; i < NA; ++i) {
            tiles.a_coord(t, kt, i, c);
            tma_load_3d(st + i * kAtAPlane, amap, c[0], c[1], c[2], &full[s]);
          }
#pragma unroll
          for (uint32_t j = 0; j < NB; ++j) {
            tiles.b_coord(t, kt, j, c);
            tma_load_3d(st + NA * kAtAPlane + j * kAtBPlane, bmap, c[0], c[1], c[2], &full[s]);
          }
          ++issued[s];
        }
      }
      for (uint32_t s = 0; s < kAtStages; ++s)
        if (issued[s]) mbar_wait_bounded(&full[s], (issued[s] - 1) & 1, fault);
    }
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issuer
      uint32_t G = 0, it = 0;
      bool ok = true;
      for (uint32_t t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ++it) {
        if (it > 0 && !mbar_wait_bounded(&tfree, (it - 1) & 1, fault)) break;
        tc_fence_after();
        uint32_t touched = 0;
        const uint32_t nk = tiles.nk(t);
        for (uint32_t kt = 0; kt < nk; ++kt, ++G) {
          const uint32_t s = G % kAtStages, use = G / kAtStages;
          if (!mbar_wait_bounded(&full[s], use & 1, fault)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t base = smem_addr(ring + s * kStage);
#pragma unroll
          for (uint32_t kk = 0; kk < kTcTileK / 32; ++kk) {
#pragma unroll
            for (uint32_t i = 0; i < NA; ++i) {
              const uint64_t ad = tc_desc(base + i * kAtAPlane + kk * 32);
#pragma unroll
              for (uint32_t j = 0; j < NB; ++j) {
                const uint64_t bd = tc_desc(base + NA * kAtAPlane + j * kAtBPlane + kk * 32);
                const uint32_t d = i + j;
                tc_mma(tmem + d * kTcTileN, ad, bd, tc_idesc(i == 3, Tiles::kBSigned && j == 3), (touched >> d) & 1u);
                touched |= 1u << d;
              }
            }
          }
          tc_commit(&empty[s]);
        }
        tc_commit(&done);
      }
    }
  } else {  // epilogue: warp w reads TMEM lanes 32 (w % 4) .. + 31, 16 of the 64 columns
    const uint32_t quad = warp & 3, cg = (warp - 2) >> 2;
    uint32_t it = 0;
    for (uint32_t t = blockIdx.x; t < ntiles; t += gridDim.x, ++it) {
      if (!mbar_wait_bounded(&done, it & 1, fault)) break;
      tc_fence_after();
      const uint32_t row = 32 * quad + lane;
      int32_t y[16];
#pragma unroll
      for (uint32_t h = 0; h < 2; ++h) {
        uint32_t r[ND][8];
#pragma unroll
        for (uint32_t d = 0; d < ND; ++d) tmem_ld8(tmem + ((32 * quad) << 16) + d * kTcTileN + cg * 16 + h * 8, r[d]);
        tmem_ld_wait();
#pragma unroll
        for (uint32_t c = 0; c < 8; ++c) {
          uint32_t v[ND];
#pragma unroll
          for (uint32_t d = 0; d < ND; ++d) v[d] = r[d][c];
          y[h * 8 + c] = epi.value(v);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tfree);  // the accumulators may be overwritten
#pragma unroll
      for (uint32_t c = 0; c < 16; ++c) epi.store(t, row, cg * 16 + c, y[c]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512u) : "memory");
  }
}

struct ScoreEpi {
  int32_t* s;  // [heads][qcap][pcap]
  uint32_t qtiles, ktiles, qcap, pcap, tokens;
  int mode;
  uint32_t scale;
  __device__ int32_t value(const uint32_t* v) const {  // each diagonal exact in int32; the sum wraps as the reference's
    uint64_t sum = 0;
#pragma unroll
    for (uint32_t d = 0; d < 7; ++d) sum += (uint64_t)(int64_t)(int32_t)v[d] << (8 * d);
    return finish_score((int64_t)sum, mode, scale);
  }
  __device__ void store(uint32_t t, uint32_t row, uint32_t col, int32_t y) const {
    const uint32_t h = t / (qtiles * ktiles), qt = (t / ktiles) % qtiles, kt = t % ktiles;
    const uint32_t q = qt * kTcTileN + col, key = kt * kTcTileM + row;
    if (q < tokens) s[((size_t)h * qcap + q) * pcap + key] = y;
  }
};

struct ValueEpi {
  uint8_t* ctx_planes;  // [tokens][4][heads*d]
  int32_t* ctx;
  uint32_t qtiles, tokens, qd, pcap;
  __device__ int32_t value(const uint32_t* v) const {
    uint64_t acc = 0;
#pragma unroll
    for (uint32_t d = 0; d < 6; ++d) {
      const int64_t lb = pv_diag_min(d) * (int64_t)pcap;
      const int64_t T = lb + (int64_t)(uint32_t)(v[d] - (uint32_t)lb);
      acc += (uint64_t)T << (8 * d);
    }
    return requantize((int64_t)acc);
  }
  __device__ void store(uint32_t t, uint32_t row, uint32_t col, int32_t y) const {
    const uint32_t h = t / qtiles, qt = t % qtiles, q = qt * kTcTileN + col;
    if (q < tokens) {
      put_planes(ctx_planes + (size_t)q * 4 * qd, qd, h * kAtD + row, y);
      if (ctx) ctx[(size_t)q * qd + h * kAtD + row] = y;
    }
  }
};

struct ScoreTilesS : ScoreTiles {
  static constexpr bool kBSigned = true;
};
struct ValueTilesS : ValueTiles {
  static constexpr bool kBSigned = false;  // weight planes are unsigned
};

__global__ void __launch_bounds__(kAtThreads, 1)
    attn_tc_scores_kernel(ScoreTilesS tiles, ScoreEpi epi, const __grid_constant__ CUtensorMap kmap,
                          const __grid_constant__ CUtensorMap qmap, unsigned int* fault) {
  extern __shared__ uint8_t at_raw[];
  uint8_t* ring = (uint8_t*)(((uintptr_t)at_raw + 1023) & ~(uintptr_t)1023);
  at_pipeline<4, 4>(tiles, epi, &kmap, &qmap, fault, ring);
}

__global__ void __launch_bounds__(kAtThreads, 1)
    attn_tc_values_kernel(ValueTilesS tiles, ValueEpi epi, const __grid_constant__ CUtensorMap vmap,
                          const __grid_constant__ CUtensorMap wmap, unsigned int* fault) {
  extern __shared__ uint8_t at_raw[];
  uint8_t* ring = (uint8_t*)(((uintptr_t)at_raw + 1023) & ~(uintptr_t)1023);
  at_pipeline<4, 3>(tiles, epi, &vmap, &wmap, fault, ring);
}

// Byte planes of int32 rows: src row r, group g's 128 values at
// src + r * stride + g * 128 -> dst[g][plane][r][d] (rows_cap rows a plane).
__global__ void at_pack_rows_kernel(const int32_t* __restrict__ src, uint32_t rows, uint32_t stride, uint32_t groups,
                                    uint32_t rows_cap, uint8_t* __restrict__ dst) {
  const uint32_t idx = blockIdx.x * blockDim.x + threadIdx.x;  // (row, group, 4-dim chunk)
  const uint32_t chunk = idx % (kAtD / 4), g = (idx / (kAtD / 4)) % groups, r = idx / (kAtD / 4) / groups;
  if (r >= rows) return;
  const int4 x = *(const int4*)(src + (size_t)r * stride + g * kAtD + 4 * chunk);
  const uint32_t u[4] = {(uint32_t)x.x, (uint32_t)x.y, (uint32_t)x.z, (uint32_t)x.w};
#pragma unroll
  for (uint32_t p = 0; p < 4; ++p) {
    const uint32_t b = ((u[0] >> (8 * p)) & 0xFF) | (((u[1] >> (8 * p)) & 0xFF) << 8) |
                       (((u[2] >> (8 * p)) & 0xFF) << 16) | (((u[3] >> (8 * p)) & 0xFF) << 24);
    *(uint32_t*)(dst + (((size_t)g * 4 + p) * rows_cap + r) * kAtD + 4 * chunk) = b;
  }
}

// Transposed value planes: dst[g][plane][d][t] for t < rows (a 32 x 32 tile a
// block through shared memory).
__global__ void at_pack_values_t_kernel(const int32_t* __restrict__ src, uint32_t rows, uint32_t stride,
                                        uint32_t pcap, uint8_t* __restrict__ dst) {
  __shared__ int32_t tile[32][33];
  const uint32_t t0 = blockIdx.x * 32, d0 = blockIdx.y * 32, g = blockIdx.z;
  const uint32_t tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 256 threads: 8 rows a pass
  for (uint32_t r = ty; r < 32; r += 8) {
    const uint32_t t = t0 + r;
    tile[r][tx] = t < rows ? src[(size_t)t * stride + g * kAtD + d0 + tx] : 0;
  }
  __syncthreads();
  for (uint32_t r = ty; r < 32; r += 8) {  // r: dimension, tx: position
    const uint32_t u = (uint32_t)tile[tx][r], t = t0 + tx;
    if (t < pcap) {
#pragma unroll
      for (uint32_t p = 0; p < 4; ++p) dst[(((size_t)g * 4 + p) * kAtD + d0 + r) * pcap + t] = (uint8_t)(u >> (8 * p));
    }
  }
}

// The exp term of every distance below the maximum: softmax_exp_term_act
// (ops.rs:508-556) depends only on d = sub_sat(score, max), an integer in
// (-2^20, 0] where it is non-zero (d <= -16.0 in Q16.16 gives 0). The table
// holds the term of d = -i at i, filled once per device by the same device
// function; d = 0 gives 2^32, which the 32-bit entry wraps to 0 and
// exp_term_lookup restores. 4 MB, read through L2.
constexpr uint32_t kExpTableSize = kExpTerms;
__device__ uint32_t g_exp_terms[kExpTableSize];

// Entry 0 is never read as a term (distance 0 returns 2^32 before the
// lookup), so it holds a marker: a table without it (a fresh module, or one
// reloaded after cudaDeviceReset) is filled again.
constexpr uint32_t kExpTableMarker = 0x45585054u;

__global__ void exp_table_kernel() {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < kExpTableSize) g_exp_terms[i] = i ? (uint32_t)softmax_exp_term_act(-(int32_t)i, 0) : kExpTableMarker;
}

__device__ __forceinline__ uint64_t exp_term_lookup(int32_t score, int32_t mx) {
  const int32_t d = sub_sat(score, mx);  // <= 0: mx is the maximum
  if (d >= 0) return (uint64_t)1 << 32;
  const uint32_t i = (uint32_t)(-(int64_t)d) < kExpTableSize ? (uint32_t)(-(int64_t)d) : 0;
  return i ? (uint64_t)__ldg(g_exp_terms + i) : 0;
}

// A warp a (query, head), eight a block: the integer softmax of the query's
// scores (positions 0..p) into three weight planes over the pcap positions,
// in three passes over the row with warp shuffles only (no block barrier, no
// shared memory): the first maximum; the exp terms (one table lookup each),
// their sum, each term written over its score; then each stored term into
// its weight (attention_softmax_into, ops.rs:233-261); the residual 1.0 - sum
// of weights goes onto the first maximum (:274-276). Terms are below 2^32
// except at distance 0, where the term is exactly 2^32: stored as
// 0xFFFFFFFF, a value no other distance gives (distance 1 gives 2^32 - 65536).
// Four consecutive positions a lane, two 16-byte loads in flight (rows and
// planes are 16-byte aligned; pcap is a multiple of 128).
constexpr uint32_t kSoftRowsPerBlock = 8;
constexpr uint32_t kTermOne = 0xFFFFFFFFu;
__device__ __forceinline__ uint64_t stored_term(uint32_t v) { return v == kTermOne ? (uint64_t)1 << 32 : v; }

__global__ void __launch_bounds__(32 * kSoftRowsPerBlock) at_softmax_warp_kernel(int32_t* __restrict__ s,
                                                                                 uint8_t* wp, uint32_t qcap,
                                                                                 uint32_t pcap, uint32_t pos0,
                                                                                 uint32_t tokens, uint32_t heads) {
  pdl_wait();
  pdl_trigger();
  const uint32_t lane = threadIdx.x & 31;
  const uint32_t r = blockIdx.x * kSoftRowsPerBlock + (threadIdx.x >> 5);  // row = h * tokens + q
  if (r >= tokens * heads) return;
  const uint32_t h = r / tokens, q = r % tokens;
  const uint32_t n = pos0 + q + 1;
  int32_t* row = s + ((size_t)h * qcap + q) * pcap;
  unsigned long long best = 0;
  auto max4 = [&](int4 v, uint32_t t) {
    const int32_t x[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (uint32_t u = 0; u < 4; ++u) {
      const unsigned long long k = t + u < n ? best_key(x[u], t + u) : 0;
      best = k > best ? k : best;
    }
  };
  for (uint32_t t = 4 * lane; t < n; t += 256) {
    const int4 v0 = *(const int4*)(row + t);
    const int4 v1 = t + 128 < n ? *(const int4*)(row + t + 128) : make_int4(0, 0, 0, 0);
    max4(v0, t);
    if (t + 128 < n) max4(v1, t + 128);
  }
#pragma unroll
  for (uint32_t off = 16; off >= 1; off >>= 1) {
    const unsigned long long o = __shfl_xor_sync(0xffffffffu, best, off);
    best = o > best ? o : best;
  }
  const int32_t mx = best_key_value(best);
  const uint32_t tmax = best_key_token(best);
  uint64_t e = 0;
  auto terms4 = [&](int4 v, uint32_t t) {
    const int32_t x[4] = {v.x, v.y, v.z, v.w};
    uint32_t o[4];
#pragma unroll
    for (uint32_t u = 0; u < 4; ++u) {
      const uint64_t term = t + u < n ? exp_term_lookup(x[u], mx) : 0;
      e += term;
      o[u] = term >> 32 ? kTermOne : (uint32_t)term;
    }
    *(uint4*)(row + t) = make_uint4(o[0], o[1], o[2], o[3]);
  };
  for (uint32_t t = 4 * lane; t < n; t += 256) {
    const int4 v0 = *(const int4*)(row + t);
    const int4 v1 = t + 128 < n ? *(const int4*)(row + t + 128) : make_int4(0, 0, 0, 0);
    terms4(v0, t);
    if (t + 128 < n) terms4(v1, t + 128);
  }
#pragma unroll
  for (uint32_t off = 16; off >= 1; off >>= 1) e += __shfl_xor_sync(0xffffffffu, e, off);
  const uint64_t tot = e, inv = tot ? UINT64_MAX / tot : 0;
  uint8_t* w0 = wp + ((size_t)h * 3 * qcap + q) * pcap;
  uint8_t* w1 = w0 + (size_t)qcap * pcap;
  uint8_t* w2 = w1 + (size_t)qcap * pcap;
  int32_t wsl = 0;
  auto weights4 = [&](uint4 v, uint32_t t) {
    const uint32_t x[4] = {v.x, v.y, v.z, v.w};
    uint32_t b0 = 0, b1 = 0, b2 = 0;
#pragma unroll
    for (uint32_t u = 0; u < 4; ++u) {
      int32_t w = 0;
      if (t + u < n) {
        w = tot ? softmax_weight_inv((int64_t)stored_term(x[u]), tot, inv) : 0;
        wsl += w;
      }
      b0 |= ((uint32_t)w & 0xFFu) << (8 * u);
      b1 |= (((uint32_t)w >> 8) & 0xFFu) << (8 * u);
      b2 |= (((uint32_t)w >> 16) & 0xFFu) << (8 * u);
    }
    *(uint32_t*)(w0 + t) = b0;
    *(uint32_t*)(w1 + t) = b1;
    *(uint32_t*)(w2 + t) = b2;
  };
  for (uint32_t t = 4 * lane; t < pcap; t += 256) {
    const uint4 v0 = t < n ? *(const uint4*)(row + t) : make_uint4(0, 0, 0, 0);
    const uint4 v1 = t + 128 < n ? *(const uint4*)(row + t + 128) : make_uint4(0, 0, 0, 0);
    weights4(v0, t);
    if (t + 128 < pcap) weights4(v1, t + 128);
  }
#pragma unroll
  for (uint32_t off = 16; off >= 1; off >>= 1) wsl += __shfl_xor_sync(0xffffffffu, wsl, off);
  __syncwarp();  // every lane's plane stores come before the first maximum's correction
  if (lane == 0) {
    const int32_t wm = tot ? softmax_weight_inv((int64_t)1 << 32, tot, inv) : 0;  // the first maximum's term
    const int32_t w = wm + sub_sat(kOneAct, wsl);  // no weight saturates
    w0[tmax] = (uint8_t)w;
    w1[tmax] = (uint8_t)(w >> 8);
    w2[tmax] = (uint8_t)(w >> 16);
  }
}


constexpr uint32_t score_smem() { return kAtStages * (4 * kAtAPlane + 4 * kAtBPlane) + 1024; }
constexpr uint32_t value_smem() { return kAtStages * (4 * kAtAPlane + 3 * kAtBPlane) + 1024; }

}  // namespace

size_t attn_tc_scratch_bytes(uint32_t heads, uint32_t kv_heads, uint32_t pcap, uint32_t qcap) {
  return (size_t)heads * qcap * pcap * 4           // scores
         + (size_t)heads * 3 * qcap * pcap          // weight planes
         + 2 * (size_t)kv_heads * 4 * pcap * kAtD   // key planes, transposed value planes
         + (size_t)heads * 4 * qcap * kAtD;         // query planes
}

void attn_tc_scratch_carve(uint8_t* base, uint32_t heads, uint32_t kv_heads, uint32_t pcap, uint32_t qcap,
                           AttnTcScratch* sc) {
  sc->pcap = pcap;
  sc->qcap = qcap;
  sc->s = (int32_t*)base;
  base += (size_t)heads * qcap * pcap * 4;
  sc->wp = base;
  base += (size_t)heads * 3 * qcap * pcap;
  sc->kp = base;
  base += (size_t)kv_heads * 4 * pcap * kAtD;
  sc->vt = base;
  base += (size_t)kv_heads * 4 * pcap * kAtD;
  sc->qp = base;
}

bool attn_tc_usable(const AttnArgs& a, uint32_t tokens, const AttnTcScratch& sc) {
  if (!sc.s || a.d != kAtD || tokens == 0 || tokens > sc.qcap || a.heads % a.kv_heads) return false;
  const uint32_t last = a.pos0 + tokens;  // positions 0..last-1 are seen
  if (a.window != 0 && last > a.window) return false;  // a sliding window cuts the prefix
  const uint32_t pcap = (last + kTcTileM - 1) / kTcTileM * kTcTileM;
  return pcap <= sc.pcap && pcap <= kAtMaxPositions && tensor_map_encoder() != nullptr;
}

cudaError_t launch_attention_prefill_tc(const AttnArgs& a, uint32_t tokens, const AttnTcScratch& sc,
                                        cudaStream_t stream) {
  if (!attn_tc_usable(a, tokens, sc)) return cudaErrorInvalidValue;
  unsigned int* fault = device_fault_word();
  if (!fault) return cudaErrorInvalidValue;
  const uint32_t last = a.pos0 + tokens;
  const uint32_t pcap = (last + kTcTileM - 1) / kTcTileM * kTcTileM;  // positions in this launch's planes
  const uint32_t qcap = (tokens + kTcTileN - 1) / kTcTileN * kTcTileN;
  const uint32_t group = a.heads / a.kv_heads, qd = a.heads * kAtD;
  // operand planes (the scratch is laid out for sc.pcap / sc.qcap; this
  // launch uses the leading pcap / qcap of each)
  cudaError_t e;
  {
    const uint32_t n = tokens * a.heads * (kAtD / 4);
    at_pack_rows_kernel<<<(n + 255) / 256, 256, 0, stream>>>(a.q, tokens, qd, a.heads, qcap, sc.qp);
    const uint32_t m = last * a.kv_heads * (kAtD / 4);
    at_pack_rows_kernel<<<(m + 255) / 256, 256, 0, stream>>>(a.kcache, last, a.kvd, a.kv_heads, pcap, sc.kp);
    at_pack_values_t_kernel<<<dim3(pcap / 32, kAtD / 32, a.kv_heads), 256, 0, stream>>>(a.vcache, last, a.kvd, pcap,
                                                                                        sc.vt);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  CUtensorMap kmap, qmap, vmap, wmap;
  if (!make_map(&kmap, sc.kp, kAtD, pcap, (uint64_t)a.kv_heads * 4, kAtD, (uint64_t)pcap * kAtD, kTcTileM, 1) ||
      !make_map(&qmap, sc.qp, kAtD, qcap, (uint64_t)a.heads * 4, kAtD, (uint64_t)qcap * kAtD, kTcTileN, 1) ||
      !make_map(&vmap, sc.vt, pcap, kAtD, (uint64_t)a.kv_heads * 4, pcap, (uint64_t)kAtD * pcap, kTcTileM, 1) ||
      !make_map(&wmap, sc.wp, pcap, qcap, (uint64_t)a.heads * 3, pcap, (uint64_t)qcap * pcap, kTcTileN, 1))
    return cudaErrorInvalidValue;
  const uint32_t qtiles = qcap / kTcTileN, ktiles = pcap / kTcTileM, sms = (uint32_t)device_sms();
  ScoreTilesS st;
  st.heads = a.heads, st.group = group, st.qtiles = qtiles, st.ktiles = ktiles;
  ScoreEpi se{sc.s, qtiles, ktiles, qcap, pcap, tokens, a.mode, a.scale_q32};
  const uint32_t sc_tiles = a.heads * qtiles * ktiles;
  e = launch_k(attn_tc_scores_kernel, dim3(std::min(sc_tiles, sms)), dim3(kAtThreads), score_smem(), stream, st, se,
               kmap, qmap, fault);
  if (e != cudaSuccess) return e;
  e = launch_k(at_softmax_warp_kernel, dim3((tokens * a.heads + kSoftRowsPerBlock - 1) / kSoftRowsPerBlock),
               dim3(32 * kSoftRowsPerBlock), 0, stream, (int32_t*)sc.s, sc.wp, qcap, pcap, a.pos0, tokens,
               a.heads);
  if (e != cudaSuccess) return e;
  ValueTilesS vt;
  vt.heads = a.heads, vt.group = group, vt.qtiles = qtiles, vt.kstages = pcap / kTcTileK;
  ValueEpi ve{a.ctx_planes, a.ctx, qtiles, tokens, qd, pcap};
  const uint32_t v_tiles = a.heads * qtiles;
  return launch_k(attn_tc_values_kernel, dim3(std::min(v_tiles, sms)), dim3(kAtThreads), value_smem(), stream, vt,
                  ve, vmap, wmap, fault);
}

// Fills the current device's exp-term table unless it holds the marker. The
// marker is read from the device (not a host flag), so a module reloaded
// after cudaDeviceReset is filled again; the mutex keeps two threads creating
// models from filling it at once.
cudaError_t ensure_exp_table() {
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  uint32_t marker = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&marker, g_exp_terms, sizeof(marker));
  if (e != cudaSuccess || marker == kExpTableMarker) return e;
  exp_table_kernel<<<kExpTableSize / 256, 256>>>();
  e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaDeviceSynchronize();  // before any stream reads it
  return e;
}

__global__ void exp_terms_probe_kernel(uint64_t* out, uint32_t first, uint32_t count) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < count) out[i] = exp_term_lookup(-(int32_t)(first + i), 0);
}

cudaError_t exp_term_table(const uint32_t** table) {
  cudaError_t e = ensure_exp_table();
  void* p = nullptr;
  if (e == cudaSuccess) e = cudaGetSymbolAddress(&p, g_exp_terms);
  *table = (const uint32_t*)p;
  return e;
}

cudaError_t prepare_attn_tc_kernels() {
  if (cudaError_t e = ensure_exp_table(); e != cudaSuccess) return e;
  cudaError_t e = cudaFuncSetAttribute(attn_tc_scores_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)score_smem());
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(attn_tc_values_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)value_smem());
  return e;
}

}  // namespace iris

extern "C" int iris_softmax_exp_terms(uint32_t first, uint32_t count, uint64_t* out) {
  using namespace iris;
  if (!out || (uint64_t)first + count > 0x80000000ull) return IRIS_EINVAL;
  if (!count) return 0;
  cudaError_t e = ensure_exp_table();
  uint64_t* d = nullptr;
  if (e == cudaSuccess) e = cudaMalloc((void**)&d, (size_t)count * 8);
  if (e == cudaSuccess) {
    exp_terms_probe_kernel<<<(count + 255) / 256, 256>>>(d, first, count);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) e = cudaMemcpy(out, d, (size_t)count * 8, cudaMemcpyDeviceToHost);
  if (d) cudaFree(d);
  return (int)e;
}
