// Many-token Q8_0 products on the tcgen05 tensor cores (kind::i8).
//
// The exact product (q8.rs:56-72) is sum over 32-value blocks b of
// s_b * sum_{k in b} q_k a_k, s_b = m_b 2^e_b the block's Q.24 scale, rounded
// once (>> 24, ties to even). The tensor-core copy of a matrix turns it into
// one contraction over the whole K, with no per-block read-out, in one of two
// forms:
//
//  - one plane (every row has one scale: the blocks with a non-zero scale
//    share its bits, as in per-output-row quantisation): the row's product is
//    m 2^e sum_k q_k a_k, with q_k zeroed in blocks whose scale is zero. The
//    Q16.16 activations are the four byte planes a0..a2 (unsigned), a3
//    (signed) the other products use, so sum_k q_k a_k = sum_i 2^(8 i)
//    sum_k q_k a_i[k]: four int8 contractions, each into its own int32
//    accumulator, exact without wrapping (|sum| < 128 * 255 * K < 2^31);
//  - three planes (block scales that differ within a row): with e0 the
//    smallest exponent of the row, every weight becomes the integer
//    W'_k = q_k m_b 2^(e_b - e0) and the row's product is 2^e0 sum_k W'_k a_k.
//    When the exponents spread by at most kTcMaxSpread, |W'| < 2^23 and W' is
//    three bytes (w0, w1 unsigned, w2 signed):
//      sum_k W'_k a_k = sum_{i,j} 2^(8 (i + j)) sum_k a_i[k] w_j[k],
//    twelve int8 contractions; the pairs with equal i + j accumulate into one
//    int32 accumulator (six "diagonals"): each diagonal's true sum lies in
//    [L_s, L_s + 2^32) for a lower bound L_s known from K and the operand
//    signs (K <= kTcMaxCols), so its wrapped int32 value gives it back exactly.
//
// The epilogue adds the accumulators in 128 bits, applies the row's scale,
// rounds once and applies the same epilogues as the other products (RoPE and
// cache stores, gating, residual, logits, partial limbs).
//
// A block: 128 weight rows (MMA M, TMEM lane = row) x kTok tokens (MMA N):
// 128 tokens for one plane (4 accumulators x 128 = the 512 TMEM columns),
// 64 for three (6 x 64). Warp 0 lane 0 issues the TMA loads (the weight
// planes, 128 rows x 128 columns each, and the four activation planes,
// kTok tokens x 128 columns each: 80 KB a stage either way, 128-byte swizzle)
// into a two-stage ring; warp 1 lane 0 issues the MMAs and commits each stage
// back to the producer; sixteen epilogue warps wait for a tile's last commit,
// read its accumulators (tcgen05.ld), release them and finish the outputs
// while the next tile accumulates. Every wait is bounded (about one second)
// and records a give-up in the fault word.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "detnum.cuh"
#include "gemv.cuh"
#include "tc.cuh"
#include "tcgen05.cuh"

namespace iris {

namespace {

static_assert(kTcRows == kTcTileM && kTcKChunk == kTcTileK, "tile shape of tcgen05.cuh");
constexpr uint32_t kTcStages = 2;
constexpr uint32_t kTcEpiWarps = 16;  // four a TMEM lane quadrant (8 measured slower: 15.0 against 14.5 ms a 2-layer 2048-token prefill)
constexpr uint32_t kTcTmemCols = 512;
constexpr uint32_t kTcAPlane = kTcRows * kTcKChunk;  // bytes of one weight plane a stage

// The tile shape of each form (P = weight planes).
template <uint32_t P>
struct TcForm {
  static constexpr uint32_t kTok = P == 1 ? 128 : 64;            // tokens a tile (MMA N)
  static constexpr uint32_t kAcc = P == 1 ? 4 : 6;               // int32 accumulators a (row, token)
  static constexpr uint32_t kBPlane = kTok * kTcKChunk;          // bytes of one activation plane a stage
  static constexpr uint32_t kStage = P * kTcAPlane + 4 * kBPlane;
  static constexpr uint32_t kEpiCols = kTok * 4 / kTcEpiWarps;   // token columns an epilogue warp finishes
  static_assert(kAcc * kTok <= kTcTmemCols, "TMEM columns");
  static_assert(kEpiCols % 16 == 0, "epilogue split");
};
static_assert(TcForm<1>::kStage == TcForm<3>::kStage, "one ring size for both forms");
static_assert(TcForm<3>::kTok == kTcTok, "three-plane tile of tc.cuh");
constexpr uint32_t kTcStage = TcForm<1>::kStage;                 // 81,920
constexpr uint32_t kTcSmem = kTcStages * kTcStage + 1024;        // + room to align the ring to 1024 bytes
// warps: 0 TMA producer, 1 MMA issuer, 2-17 epilogue
constexpr uint32_t kTcThreads = 32 * (2 + kTcEpiWarps);

// Three planes: lower bounds of one column's contribution to each diagonal
// (i + j = s): u8 x u8 >= 0, u8 x s8 >= 255 * -128, s8 x s8 >= -128 * 127.
// The largest span of a diagonal, 227,715 a column (s = 2, 3), keeps
// K * span < 2^32 for K <= kTcMaxCols.
__host__ __device__ constexpr int64_t tc_diag_min(uint32_t s) {
  return s == 2 || s == 4 ? -65280 : s == 3 ? -97920 : s == 5 ? -16256 : 0;
}
static_assert((uint64_t)kTcMaxCols * 227715 < (1ull << 32), "diagonal span");
// One plane: |sum_k q_k a_i[k]| <= 128 * 255 * K stays below 2^31.
static_assert((uint64_t)kTcMaxCols * 128 * 255 < (1ull << 31), "one-plane accumulator range");

// The output of one (token, row) from its rounded value (every epilogue but
// EPI_PARTIAL, which writes its limbs while the accumulators are read).
template <int EPI>
__device__ __forceinline__ void tc_finish(const ProductArgs& a, uint32_t tok, uint32_t row, int32_t v,
                                          uint32_t lane) {
  if (EPI == EPI_QKV_ROPE || EPI == EPI_SILU_MUL || EPI == EPI_GELU_MUL) {
    const int32_t partner = __shfl_xor_sync(0xffffffffu, v, 1);  // row ^ 1, same token
    if ((lane & 1) == 0 && tok < a.tokens && row + 1 < a.rows) epi_pair<EPI>(a, tok, row, v, partner);
  } else if (EPI == EPI_LOGITS) {
    if (tok < a.tokens && row < a.rows) {
      if (a.softcap > 0) v = softcap_act(v, a.softcap);
      if (a.out) a.out[(size_t)tok * a.out_stride + row] = v;
      atomicMax(a.best + tok, best_key(v, row + a.row_base));
    }
  } else if (tok < a.tokens && row < a.rows) {
    epi_single<EPI>(a, tok, row, v);
  }
}

// The MMAs of one stage. One plane: the signed weight plane against each
// activation plane i into accumulator i. Three planes: weight plane j
// against activation plane i into diagonal i + j. A tile's first MMA into an
// accumulator overwrites it.
template <uint32_t P>
__device__ __forceinline__ void tc_issue_stage(uint32_t tmem, uint32_t base, uint32_t& touched) {
  using F = TcForm<P>;
#pragma unroll
  for (uint32_t kk = 0; kk < kTcKChunk / 32; ++kk) {
#pragma unroll
    for (uint32_t j = 0; j < P; ++j) {
      const uint64_t ad = tc_desc(base + j * kTcAPlane + kk * 32);
#pragma unroll
      for (uint32_t i = 0; i < 4; ++i) {
        const uint64_t bd = tc_desc(base + P * kTcAPlane + i * F::kBPlane + kk * 32);
        const uint32_t d = i + j;
        tc_mma(tmem + d * F::kTok, ad, bd, tc_idesc_n(P == 1 || j == 2, i == 3, F::kTok), (touched >> d) & 1u);
        touched |= 1u << d;
      }
    }
  }
}

// The 128-bit total of one (row, token) from its accumulators' raw words.
template <uint32_t P>
__device__ __forceinline__ Acc128 tc_total(const uint32_t (&r)[TcForm<P>::kAcc][8], uint32_t c,
                                           const int64_t* lo_bound, int32_t shift, int32_t mant) {
  Acc128 tot{0, 0};
  if constexpr (P == 1) {
    // |x| < 2^31 * 2^24 * 1.01: sum_i 2^(8 i) x_i in one int64, times the
    // 11-bit mantissa in two 32-bit halves, at the row's exponent
    const int64_t x = (int64_t)(int32_t)r[0][c] + (int64_t)(int32_t)r[1][c] * 256 +
                      (int64_t)(int32_t)r[2][c] * 65536 + (int64_t)(int32_t)r[3][c] * 16777216;
    acc128_add_shifted(tot, (int64_t)(x & 0xFFFFFFFFll) * mant, shift);
    acc128_add_shifted(tot, (x >> 32) * mant, shift + 32);
  } else {
    int64_t T[6];
#pragma unroll
    for (uint32_t d = 0; d < 6; ++d) T[d] = lo_bound[d] + (int64_t)(uint32_t)(r[d][c] - (uint32_t)lo_bound[d]);
    // |T| < 2^33: the first four fit one int64 at weights 2^0..2^24,
    // the last two another at 2^32, 2^40
    const int64_t lo = T[0] + T[1] * 256 + T[2] * 65536 + T[3] * 16777216;
    const int64_t hi = T[4] + T[5] * 256;
    acc128_add_shifted(tot, lo, shift);
    acc128_add_shifted(tot, hi, shift + 32);
  }
  return tot;
}

// Persistent: block b takes tiles b, b + gridDim.x, ... (token tiles vary
// fastest, so the blocks sharing a weight tile run at the same time). The
// ring runs on across tiles; the MMA warp starts a tile's accumulation once
// the epilogue warps have read the previous tile's accumulators out of TMEM
// (tfree), so that the epilogue arithmetic (RoPE, the gating's sigmoid,
// residual adds, stores) overlaps the next tile's MMAs.
template <int EPI, uint32_t P>
__global__ void __launch_bounds__(kTcThreads, 1)
    q8_gemm_tc_kernel(ProductArgs a, const __grid_constant__ CUtensorMap wmap,
                      const __grid_constant__ CUtensorMap pmap, unsigned int* fault) {
  using F = TcForm<P>;
  extern __shared__ uint8_t tc_raw[];
  __shared__ __align__(8) uint64_t full[kTcStages], empty[kTcStages], done, tfree;
  __shared__ uint32_t tmem_slot;
  uint8_t* ring = (uint8_t*)(((uintptr_t)tc_raw + 1023) & ~(uintptr_t)1023);
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t nk = (a.cols + kTcKChunk - 1) / kTcKChunk;
  const uint32_t ntt = (a.tokens + F::kTok - 1) / F::kTok, ntiles = ntt * (a.tc_rows / kTcRows);

  if (threadIdx.x == 0) {
    for (uint32_t s = 0; s < kTcStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&done, 1);
    mbar_init(&tfree, kTcEpiWarps);
    mbar_fence_init();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&tmem_slot)),
                 "r"(kTcTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  pdl_wait();  // the activation planes come from the kernel before
  pdl_trigger();

  if (warp == 0) {
    if (lane == 0) {  // producer
      uint32_t issued[kTcStages] = {};
      uint32_t G = 0;  // stages issued so far (all tiles)
      bool ok = true;
      for (uint32_t t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
        const uint32_t m0 = (t % ntt) * F::kTok, n0 = (t / ntt) * kTcRows;
        for (uint32_t kt = 0; kt < nk; ++kt, ++G) {
          const uint32_t s = G % kTcStages, use = G / kTcStages;
          if (use > 0 && !mbar_wait_bounded(&empty[s], (use - 1) & 1, fault)) {
            ok = false;
            break;
          }
          uint8_t* st = ring + s * kTcStage;
          mbar_arrive_expect_tx(&full[s], F::kStage);
#pragma unroll
          for (uint32_t j = 0; j < P; ++j) tma_load_3d(st + j * kTcAPlane, &wmap, kt * kTcKChunk, n0, j, &full[s]);
#pragma unroll
          for (uint32_t i = 0; i < 4; ++i)
            tma_load_3d(st + P * kTcAPlane + i * F::kBPlane, &pmap, kt * kTcKChunk, i, m0, &full[s]);
          ++issued[s];
        }
      }
      // every issued copy has landed before the block may exit
      for (uint32_t s = 0; s < kTcStages; ++s)
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
        for (uint32_t kt = 0; kt < nk; ++kt, ++G) {
          const uint32_t s = G % kTcStages, use = G / kTcStages;
          if (!mbar_wait_bounded(&full[s], use & 1, fault)) {
            ok = false;
            break;
          }
          tc_fence_after();
          tc_issue_stage<P>(tmem, smem_addr(ring + s * kTcStage), touched);
          tc_commit(&empty[s]);
        }
        tc_commit(&done);  // also after a give-up: the epilogue's wait then ends
      }
    }
  } else {  // epilogue: warp w reads TMEM lanes 32 (w % 4) .. + 31, kEpiCols token columns
    constexpr uint32_t EC = F::kEpiCols;
    const uint32_t quad = warp & 3, cg = (warp - 2) >> 2;
    int64_t lo_bound[6];
#pragma unroll
    for (uint32_t d = 0; d < 6; ++d) lo_bound[d] = tc_diag_min(d) * (int64_t)a.cols;
    uint32_t it = 0;
    for (uint32_t t = blockIdx.x; t < ntiles; t += gridDim.x, ++it) {
      const uint32_t m0 = (t % ntt) * F::kTok, n0 = (t / ntt) * kTcRows;
      if (!mbar_wait_bounded(&done, it & 1, fault)) break;
      tc_fence_after();
      const uint32_t row = n0 + 32 * quad + lane;
      const int32_t shift = row < a.tc_rows ? a.tc_shift[row] : 0;
      const int32_t mant = P == 1 && row < a.tc_rows ? a.tc_mant[row] : 1;
      int32_t v[EC];
#pragma unroll
      for (uint32_t h = 0; h < EC / 8; ++h) {
        const uint32_t c0 = cg * EC + h * 8;
        uint32_t r[F::kAcc][8];
#pragma unroll
        for (uint32_t d = 0; d < F::kAcc; ++d) tmem_ld8(tmem + ((32 * quad) << 16) + d * F::kTok + c0, r[d]);
        tmem_ld_wait();
#pragma unroll
        for (uint32_t c = 0; c < 8; ++c) {
          if constexpr (P == 1 && EPI != EPI_PARTIAL) {  // the rounded value in 64 bits where it fits
            const int64_t x = (int64_t)(int32_t)r[0][c] + (int64_t)(int32_t)r[1][c] * 256 +
                              (int64_t)(int32_t)r[2][c] * 65536 + (int64_t)(int32_t)r[3][c] * 16777216;
            v[h * 8 + c] = round_q24_scaled(x, mant, shift);
            continue;
          }
          const Acc128 tot = tc_total<P>(r, c, lo_bound, shift, mant);
          if (EPI == EPI_PARTIAL) {
            const uint32_t tok = m0 + c0 + c;
            if (tok < a.tokens && row < a.rows)
              limbs_from_acc128(tot.lo, tot.hi, a.partial + ((size_t)tok * a.rows + row) * 4);
          } else {
            v[h * 8 + c] = acc128_round_q24(tot);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tfree);  // the accumulators may be overwritten
      if (EPI == EPI_QKV_ROPE || EPI == EPI_SILU_MUL || EPI == EPI_GELU_MUL) {
        // rows 2i, 2i + 1 (lanes 2i, 2i + 1) form a pair: the even lane
        // finishes the pair for the first half of the tokens, the odd lane for the second
        const bool odd = lane & 1;
        const uint32_t rowe = row & ~1u;
#pragma unroll
        for (uint32_t c = 0; c < EC / 2; ++c) {
          const int32_t got = __shfl_xor_sync(0xffffffffu, odd ? v[c] : v[EC / 2 + c], 1);
          const uint32_t tok = m0 + cg * EC + (odd ? EC / 2 + c : c);
          const int32_t v0 = odd ? got : v[c], v1 = odd ? v[EC / 2 + c] : got;
          if (tok < a.tokens && rowe + 1 < a.rows) epi_pair<EPI>(a, tok, rowe, v0, v1);
        }
      } else if (EPI != EPI_PARTIAL) {
#pragma unroll
        for (uint32_t c = 0; c < EC; ++c) tc_finish<EPI>(a, m0 + cg * EC + c, row, v[c], lane);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTcTmemCols) : "memory");
  }
}

// One weight row a block: the row's scale summary. flags bit 0: a row's
// exponents (over blocks with a non-zero scale) spread wider than the three
// planes hold; bit 1: a row whose non-zero scales differ (no one-plane copy).
__global__ void tc_scan_kernel(const uint16_t* __restrict__ s, uint32_t rows, uint32_t cols, uint32_t kc,
                               uint32_t nslices, unsigned int* flags) {
  __shared__ int smin, smax;
  __shared__ unsigned int first, differ;
  const uint32_t row = blockIdx.x, nb = cols / 32;
  if (threadIdx.x == 0) {
    smin = 64;
    smax = -1;
    first = 0xFFFFFFFFu;
    differ = 0;
  }
  __syncthreads();
  int lmin = 64, lmax = -1;
  bool ldiff = false;
  for (uint32_t b = threadIdx.x; b < nb; b += blockDim.x) {
    const uint16_t bits = s[q8_scale_offset(kc, nslices, row, b)];
    int32_t m, e;
    q8_scale_parts_finite(bits, &m, &e);
    if (m != 0) {
      lmin = min(lmin, e);
      lmax = max(lmax, e);
      const unsigned int old = atomicCAS(&first, 0xFFFFFFFFu, (unsigned int)bits);
      ldiff |= old != 0xFFFFFFFFu && old != bits;
    }
  }
  atomicMin(&smin, lmin);
  atomicMax(&smax, lmax);
  if (ldiff) atomicOr(&differ, 1u);
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned int f = differ ? 2u : 0u;
    if (smax >= 0 && smax - smin > kTcMaxSpread) f |= 1u;
    if (f) atomicOr(flags, f);
  }
}

// One-plane copy, one weight row a block: q (zero in blocks whose scale is
// zero) and the row's one scale as (mantissa, exponent); rows past `rows`
// are zero.
__global__ void tc_plane1_kernel(const int8_t* __restrict__ q, const uint16_t* __restrict__ s, uint32_t rows,
                                 uint32_t cols, uint32_t kc, uint32_t nslices, uint8_t* __restrict__ plane,
                                 uint8_t* __restrict__ shift, int16_t* __restrict__ mant) {
  __shared__ unsigned int row_bits;
  const uint32_t row = blockIdx.x, nb = cols / 32;
  if (threadIdx.x == 0) row_bits = 0;
  __syncthreads();
  if (row < rows)
    for (uint32_t b = threadIdx.x; b < nb; b += blockDim.x) {
      const uint16_t bits = s[q8_scale_offset(kc, nslices, row, b)];
      int32_t m, e;
      q8_scale_parts_finite(bits, &m, &e);
      if (m != 0) row_bits = bits;  // every non-zero scale of the row has these bits
    }
  __syncthreads();
  if (threadIdx.x == 0) {
    int32_t m = 0, e = 0;
    if (row_bits) q8_scale_parts_finite((uint16_t)row_bits, &m, &e);
    shift[row] = (uint8_t)(m ? e : 0);
    mant[row] = (int16_t)m;
  }
  uint8_t* p = plane + (size_t)row * cols;
  for (uint32_t k = threadIdx.x * 4; k < cols; k += blockDim.x * 4) {
    uint32_t w = 0;
    if (row < rows) {
      int32_t m, e;
      q8_scale_parts_finite(s[q8_scale_offset(kc, nslices, row, k / 32)], &m, &e);
      if (m != 0) w = *(const uint32_t*)(q + q8_value_offset(kc, nslices, row, k));
    }
    *(uint32_t*)(p + k) = w;
  }
}

// Three-plane copy, one weight row a block: the row's smallest scale
// exponent (over blocks with a non-zero scale), then the three byte planes of
// the pre-scaled weights (the spread was checked by tc_scan_kernel).
__global__ void tc_planes3_kernel(const int8_t* __restrict__ q, const uint16_t* __restrict__ s, uint32_t rows,
                                  uint32_t cols, uint32_t kc, uint32_t nslices, uint32_t tc_rows,
                                  uint8_t* __restrict__ planes, uint8_t* __restrict__ shift) {
  __shared__ int smin, smax;
  const uint32_t row = blockIdx.x, nb = cols / 32;
  if (threadIdx.x == 0) {
    smin = 64;
    smax = -1;
  }
  __syncthreads();
  if (row < rows) {
    int lmin = 64, lmax = -1;
    for (uint32_t b = threadIdx.x; b < nb; b += blockDim.x) {
      int32_t m, e;
      q8_scale_parts_finite(s[q8_scale_offset(kc, nslices, row, b)], &m, &e);
      if (m != 0) {
        lmin = min(lmin, e);
        lmax = max(lmax, e);
      }
    }
    atomicMin(&smin, lmin);
    atomicMax(&smax, lmax);
  }
  __syncthreads();
  const int e0 = smax < 0 ? 0 : smin;
  if (threadIdx.x == 0) shift[row] = (uint8_t)e0;
  uint8_t* p0 = planes + (size_t)row * cols;
  uint8_t* p1 = planes + ((size_t)tc_rows + row) * cols;
  uint8_t* p2 = planes + ((size_t)2 * tc_rows + row) * cols;
  for (uint32_t k = threadIdx.x * 4; k < cols; k += blockDim.x * 4) {
    uint32_t b0 = 0, b1 = 0, b2 = 0;
    if (row < rows) {
      int32_t m, e;
      q8_scale_parts_finite(s[q8_scale_offset(kc, nslices, row, k / 32)], &m, &e);
      const char4 qv = *(const char4*)(q + q8_value_offset(kc, nslices, row, k));
      const int32_t f = m != 0 ? m * (1 << min(e - e0, 8)) : 0;  // spread checked by the scan
      const int32_t w[4] = {qv.x * f, qv.y * f, qv.z * f, qv.w * f};
#pragma unroll
      for (uint32_t u = 0; u < 4; ++u) {
        b0 |= ((uint32_t)w[u] & 0xFFu) << (8 * u);
        b1 |= (((uint32_t)w[u] >> 8) & 0xFFu) << (8 * u);
        b2 |= (((uint32_t)(w[u] >> 16)) & 0xFFu) << (8 * u);
      }
    }
    *(uint32_t*)(p0 + k) = b0;
    *(uint32_t*)(p1 + k) = b1;
    *(uint32_t*)(p2 + k) = b2;
  }
}

template <int EPI, uint32_t P>
cudaError_t launch_tc_form(const ProductArgs& a, cudaStream_t stream) {
  CUtensorMap wmap, pmap;
  if (!make_map(&wmap, a.tc, a.cols, a.tc_rows, P, a.cols, (uint64_t)a.tc_rows * a.cols, kTcRows, 1) ||
      !make_map(&pmap, a.planes, a.cols, 4, a.tokens, a.cols, (uint64_t)4 * a.cols, 1, TcForm<P>::kTok))
    return cudaErrorInvalidValue;
  unsigned int* fault = device_fault_word();
  if (!fault) return cudaErrorInvalidValue;
  // one block a multiprocessor (the shared memory allows no second), persistent over the tiles
  const uint32_t tiles = (a.tokens + TcForm<P>::kTok - 1) / TcForm<P>::kTok * (a.tc_rows / kTcRows);
  const dim3 grid(std::min<uint32_t>(tiles, (uint32_t)device_sms()));
  return launch_k(q8_gemm_tc_kernel<EPI, P>, grid, dim3(kTcThreads), kTcSmem, stream, a, wmap, pmap, fault);
}

template <int EPI>
cudaError_t launch_tc_one(const ProductArgs& a, cudaStream_t stream) {
  return a.tc_planes == 1 ? launch_tc_form<EPI, 1>(a, stream) : launch_tc_form<EPI, 3>(a, stream);
}

template <int EPI>
cudaError_t prepare_tc_one() {
  cudaError_t e =
      cudaFuncSetAttribute(q8_gemm_tc_kernel<EPI, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTcSmem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(q8_gemm_tc_kernel<EPI, 3>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTcSmem);
  return e;
}

}  // namespace

cudaError_t prepare_tc_kernels() {
  cudaError_t e = prepare_tc_one<EPI_STORE>();
  if (e == cudaSuccess) e = prepare_tc_one<EPI_RESID>();
  if (e == cudaSuccess) e = prepare_tc_one<EPI_QKV_ROPE>();
  if (e == cudaSuccess) e = prepare_tc_one<EPI_SILU_MUL>();
  if (e == cudaSuccess) e = prepare_tc_one<EPI_GELU_MUL>();
  if (e == cudaSuccess) e = prepare_tc_one<EPI_LOGITS>();
  if (e == cudaSuccess) e = prepare_tc_one<EPI_PARTIAL>();
  return e;
}

bool tc_usable(const ProductArgs& a) {
  return a.tc && a.tc_shift && (a.tc_planes == 3 || (a.tc_planes == 1 && a.tc_mant)) &&
         a.tc_rows % kTcRows == 0 && a.tc_rows >= a.rows && a.cols % 32 == 0 &&
         a.cols <= kTcMaxCols && a.tokens > 0 && a.planes && ((uintptr_t)a.planes & 15) == 0 &&
         ((uintptr_t)a.tc & 15) == 0 && a.tc_rows / kTcRows <= 65535 && tensor_map_encoder() != nullptr;
}

cudaError_t launch_gemm_tc(const ProductArgs& a, EpiMode epi, cudaStream_t stream) {
  if (!tc_usable(a)) return cudaErrorInvalidValue;
  switch (epi) {
    case EPI_STORE: return launch_tc_one<EPI_STORE>(a, stream);
    case EPI_RESID: return launch_tc_one<EPI_RESID>(a, stream);
    case EPI_QKV_ROPE: return launch_tc_one<EPI_QKV_ROPE>(a, stream);
    case EPI_SILU_MUL: return launch_tc_one<EPI_SILU_MUL>(a, stream);
    case EPI_GELU_MUL: return launch_tc_one<EPI_GELU_MUL>(a, stream);
    case EPI_LOGITS: return launch_tc_one<EPI_LOGITS>(a, stream);
    case EPI_PARTIAL: return launch_tc_one<EPI_PARTIAL>(a, stream);
  }
  return cudaErrorInvalidValue;
}

cudaError_t tc_prepare(Q8GpuMatrix* m, cudaStream_t stream, int planes) {
  if (!tc_state_claim(m)) return cudaSuccess;  // built, unusable, or another thread is building it
  if (m->cols == 0 || m->cols % 32 || m->cols > kTcMaxCols || m->rows == 0) return cudaSuccess;
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &cap) != cudaSuccess || cap != cudaStreamCaptureStatusNone) {
    tc_state_set(m, 0);  // not inside a capture; a later call builds it
    return cudaSuccess;
  }
  const uint32_t tc_rows = (m->rows + kTcRows - 1) / kTcRows * kTcRows;
  // which form: the one-plane copy where every row has one scale, else three
  // planes where the exponents allow them (one host read of the scan's flags)
  unsigned int* flags = nullptr;
  unsigned int h_flags = 0;
  if (cudaMalloc((void**)&flags, 4) != cudaSuccess) {
    cudaGetLastError();  // no room: the mma.sync GEMM serves this matrix
    return cudaSuccess;
  }
  cudaError_t e = cudaMemsetAsync(flags, 0, 4, stream);
  if (e == cudaSuccess) {
    tc_scan_kernel<<<m->rows, 256, 0, stream>>>(m->s, m->rows, m->cols, m->kc, m->nslices, flags);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) e = cudaMemcpyAsync(&h_flags, flags, 4, cudaMemcpyDeviceToHost, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  cudaFree(flags);
  if (e != cudaSuccess) return e;
  uint32_t P = (h_flags & 2u) ? 3 : 1;
  if (planes == 3 && P == 1) P = 3;  // a three-plane copy asked for (measurement)
  if (P == 3 && (h_flags & 1u)) return cudaSuccess;  // exponents too far apart: the mma.sync GEMM
  uint8_t *tc = nullptr, *shift = nullptr;
  int16_t* mant = nullptr;
  if (cudaMalloc((void**)&tc, (size_t)P * tc_rows * m->cols) != cudaSuccess ||
      cudaMalloc((void**)&shift, tc_rows) != cudaSuccess ||
      (P == 1 && cudaMalloc((void**)&mant, (size_t)tc_rows * sizeof(int16_t)) != cudaSuccess)) {
    cudaGetLastError();  // no room: the mma.sync GEMM serves this matrix
    cudaFree(tc);
    cudaFree(shift);
    cudaFree(mant);
    return cudaSuccess;
  }
  if (P == 1)
    tc_plane1_kernel<<<tc_rows, 256, 0, stream>>>(m->q, m->s, m->rows, m->cols, m->kc, m->nslices, tc, shift, mant);
  else
    tc_planes3_kernel<<<tc_rows, 256, 0, stream>>>(m->q, m->s, m->rows, m->cols, m->kc, m->nslices, tc_rows, tc,
                                                   shift);
  e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) {
    cudaFree(tc);
    cudaFree(shift);
    cudaFree(mant);
    return e;
  }
  m->tc = tc;
  m->tc_shift = shift;
  m->tc_mant = mant;
  m->tc_rows = tc_rows;
  m->tc_planes = P;
  tc_state_set(m, 1);
  return cudaSuccess;
}

}  // namespace iris
