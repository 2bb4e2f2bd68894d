// Building blocks of the decode GEMV shared by the one-product kernel
// (q8.cu) and the persistent decode-step kernel (step.cu): the activation
// prologue (byte planes, optionally RMS-normalised), the per-warp tile
// products, the exact split-sum exchange and the fused epilogues.
//
// Values another block of the same launch may have written (activations,
// residuals, split sums) are read through L2 (ld.global.cg), never from a
// possibly stale L1 line.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "q8.cuh"

namespace iris {

// Synchronisation of the threads taking part in a block-wide step: the whole
// block (NT = 0) or the first NT threads through named barrier 1 (the other
// warps of the block keep running).
template <uint32_t NT>
__device__ __forceinline__ uint32_t part_threads() {
  return NT ? NT : blockDim.x;
}
template <uint32_t NT>
__device__ __forceinline__ void part_sync() {
  if constexpr (NT == 0) __syncthreads();
  else asm volatile("bar.sync 1, %0;" ::"n"(NT) : "memory");
}
template <uint32_t NT>
__device__ __forceinline__ bool part_or(bool pred) {
  if constexpr (NT == 0) {
    return __syncthreads_or(pred) != 0;
  } else {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.or.pred q, 1, %2, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)pred), "n"(NT)
        : "memory");
    return r != 0;
  }
}

// ---------------------------------------------------------------------------
// Byte planes
// ---------------------------------------------------------------------------

// Saturating sum of non-negative values over the threads taking part (result
// valid in warp 0).
template <uint32_t NT = 0>
__device__ __forceinline__ uint64_t block_sum_sat(uint64_t v, uint64_t* red) {
  v = warp_sum_sat_nonneg(v);
  int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) red[warp] = v;
  part_sync<NT>();
  uint64_t t = 0;
  if (threadIdx.x < 32) {
    t = threadIdx.x < (part_threads<NT>() >> 5) ? red[threadIdx.x] : 0;
    t = warp_sum_sat_nonneg(t);
  }
  return t;
}

// Builds the byte planes of one K-wide row into `planes` (shared or global),
// RMS-normalising first when norm_w is given (ops.rs:98-114: two mul_sat per
// value, by the inverse-RMS scale and then by the weight).
// The threads taking part are NT (0: the whole block). x may have been
// written by another block of the same launch: it is read through L2.
template <uint32_t NT = 0>
__device__ __forceinline__ bool row_to_planes(const int32_t* x, const int32_t* __restrict__ norm_w, int64_t eps,
                                              uint32_t K, uint8_t* planes, uint64_t* red, int32_t* s_scale) {
  // Rows of up to kHeld values a thread are held in registers, the values and
  // the norm weights loaded together: one pass over global memory.
  constexpr uint32_t kHeld = 2;  // int4 pieces a thread
  const uint32_t step = part_threads<NT>() * 4;
  const bool held = K <= kHeld * step;
  int4 xv[kHeld], wv[kHeld];
  if (held) {
#pragma unroll
    for (uint32_t j = 0; j < kHeld; ++j) {
      const uint32_t i = threadIdx.x * 4 + j * step;
      xv[j] = i < K ? __ldcg((const int4*)(x + i)) : make_int4(0, 0, 0, 0);
      wv[j] = i < K && norm_w ? *(const int4*)(norm_w + i) : make_int4(0, 0, 0, 0);
    }
  }
  int32_t scale = 0;
  if (norm_w) {
    uint64_t ss = 0;
    auto square_sum = [&](int4 v) {
      ss = add_sat_nonneg(ss, (uint64_t)((int64_t)v.x * v.x));
      ss = add_sat_nonneg(ss, (uint64_t)((int64_t)v.y * v.y));
      ss = add_sat_nonneg(ss, (uint64_t)((int64_t)v.z * v.z));
      ss = add_sat_nonneg(ss, (uint64_t)((int64_t)v.w * v.w));
    };
    if (held) {
#pragma unroll
      for (uint32_t j = 0; j < kHeld; ++j) square_sum(xv[j]);
    } else {
      for (uint32_t i = threadIdx.x * 4; i < K; i += step) square_sum(__ldcg((const int4*)(x + i)));
    }
    uint64_t total = block_sum_sat<NT>(ss, red);  // in every lane of warp 0
    if (threadIdx.x < 32) {  // rms_scale_from_sumsq with the warp-parallel inverse square root
      const int32_t sc = inv_sqrt_acc_fast(acc_add_sat((int64_t)div_round_even_width(total, K), eps));
      if (threadIdx.x == 0) *s_scale = sc;
    }
    part_sync<NT>();
    scale = *s_scale;
  }
  int wide = 0;
  auto emit = [&](int4 v, int4 w, uint32_t i) {
    if (norm_w) {
      v.x = mul_sat(mul_sat(v.x, scale), w.x);
      v.y = mul_sat(mul_sat(v.y, scale), w.y);
      v.z = mul_sat(mul_sat(v.z, scale), w.z);
      v.w = mul_sat(mul_sat(v.w, scale), w.w);
    }
    wide |= !fits_three_planes(v.x) | !fits_three_planes(v.y) | !fits_three_planes(v.z) | !fits_three_planes(v.w);
    put_planes4(planes, K, i, v);
  };
  if (held) {
#pragma unroll
    for (uint32_t j = 0; j < kHeld; ++j) {
      const uint32_t i = threadIdx.x * 4 + j * step;
      if (i < K) emit(xv[j], wv[j], i);
    }
  } else {
    for (uint32_t i = threadIdx.x * 4; i < K; i += step)
      emit(__ldcg((const int4*)(x + i)), norm_w ? *(const int4*)(norm_w + i) : make_int4(0, 0, 0, 0), i);
  }
  return part_or<NT>(wide);
}


// ---------------------------------------------------------------------------
// Epilogue helpers shared by both kernels
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t token_position(const ProductArgs& a, uint32_t t) {
  return (a.pos_ptr ? *a.pos_ptr : a.pos0) + t;
}

// A finished (even, odd) row pair of a paired epilogue for token t.
template <int EPI>
__device__ __forceinline__ void epi_pair(const ProductArgs& a, uint32_t t, uint32_t row, int32_t v0,
                                         int32_t v1) {
  if (EPI == EPI_QKV_ROPE) {
    uint32_t pos = token_position(a, t);
    // the rotation of frequency f at this token's position: from the
    // precomputed table when there is one (the same sin_cos_q30 values)
    auto rotate = [&](uint32_t f) {
      if (!a.rope_sc) {
        rotate_pair_q30(&v0, &v1, a.freqs[f], pos);
      } else if (pos) {
        const int64_t* sc = a.rope_sc + ((size_t)t * (a.head_dim / 2) + f) * 2;
        rotate_pair_sc(&v0, &v1, sc[0], sc[1]);
      }
    };
    if (row < a.qd) {
      rotate((row % a.head_dim) >> 1);
      int32_t* o = a.out + (size_t)t * a.out_stride + row;
      o[0] = v0;
      o[1] = v1;
    } else if (row < a.qd + a.kvd) {
      uint32_t c = row - a.qd;
      rotate((c % a.head_dim) >> 1);
      int32_t* o = a.kcache + (size_t)pos * a.kvd + c;
      o[0] = v0;
      o[1] = v1;
    } else {
      uint32_t c = row - a.qd - a.kvd;
      int32_t* o = a.vcache + (size_t)pos * a.kvd + c;
      o[0] = v0;
      o[1] = v1;
    }
  } else {  // gated: v0 = gate_j, v1 = up_j
    int32_t g = EPI == EPI_SILU_MUL ? silu(v0) : gelu_tanh(v0);
    int32_t y = mul_sat(g, v1);
    uint32_t F = a.rows >> 1;
    put_planes(a.out_planes + (size_t)t * 4 * F, F, row >> 1, y);
  }
}

// The one-token RoPE epilogue with the sines and cosines of the token's
// position precomputed (sc[i] = sin, cos of frequency i; none at position 0):
// epi_pair<EPI_QKV_ROPE> for t = 0 with the same rotation.
__device__ __forceinline__ void epi_pair_rope_sc(const ProductArgs& a, uint32_t pos, uint32_t row, int32_t v0,
                                                 int32_t v1, const int64_t (*sc)[2]) {
  if (row < a.qd + a.kvd) {
    const uint32_t c = row < a.qd ? row : row - a.qd;
    if (pos) {
      const uint32_t f = (c % a.head_dim) >> 1;
      rotate_pair_sc(&v0, &v1, sc[f][0], sc[f][1]);
    }
    int32_t* o = row < a.qd ? a.out + row : a.kcache + (size_t)pos * a.kvd + c;
    o[0] = v0;
    o[1] = v1;
  } else {
    int32_t* o = a.vcache + (size_t)pos * a.kvd + (row - a.qd - a.kvd);
    o[0] = v0;
    o[1] = v1;
  }
}
constexpr uint32_t kRopeTablePairs = 128;  // head_dim <= 256

// A finished single-row value for token t; returns the value written.
template <int EPI>
__device__ __forceinline__ int32_t epi_single(const ProductArgs& a, uint32_t t, uint32_t row, int32_t v) {
  size_t o = (size_t)t * a.out_stride + row;
  if (EPI == EPI_RESID) v = add_sat(v, __ldcg(a.resid + o));
  else if (EPI == EPI_LOGITS && a.softcap > 0) v = softcap_act(v, a.softcap);
  if (EPI != EPI_LOGITS || a.out) a.out[o] = v;
  return v;
}


// IN_POST_ATTN (gemma's post-attention step, prefill_range.rs post_attention
// and pre_feedforward norms) fused into the gate|up product's prologue:
// x' = add_sat(rms_norm(o, post_w), x), then the byte planes of
// rms_norm(x', norm_w), each norm as row_to_planes' (two mul_sat a value).
// Every block computes the row itself; block 0 stores x' to post_x. The row
// is held in registers: K <= 2 * 4 * part_threads<NT>() (the host checks).
template <uint32_t NT = 0>
__device__ __forceinline__ bool post_attn_to_planes(const ProductArgs& a, uint32_t K, uint8_t* planes,
                                                    uint64_t* red, int32_t* s_scale) {
  constexpr uint32_t kHeld = 2;
  const uint32_t step = part_threads<NT>() * 4;
  const int4 z = make_int4(0, 0, 0, 0);
  int4 ov[kHeld], xv[kHeld], w1[kHeld], w2[kHeld];
#pragma unroll
  for (uint32_t j = 0; j < kHeld; ++j) {
    const uint32_t i = threadIdx.x * 4 + j * step;
    const bool in = i < K;
    ov[j] = in ? __ldcg((const int4*)(a.post_o + i)) : z;
    xv[j] = in ? __ldcg((const int4*)(a.x + i)) : z;
    w1[j] = in && a.post_w ? *(const int4*)(a.post_w + i) : z;
    w2[j] = in && a.norm_w ? *(const int4*)(a.norm_w + i) : z;
  }
  auto sq4 = [](uint64_t ss, int4 v) {
    ss = add_sat_nonneg(ss, (uint64_t)((int64_t)v.x * v.x));
    ss = add_sat_nonneg(ss, (uint64_t)((int64_t)v.y * v.y));
    ss = add_sat_nonneg(ss, (uint64_t)((int64_t)v.z * v.z));
    return add_sat_nonneg(ss, (uint64_t)((int64_t)v.w * v.w));
  };
  auto row_scale = [&](uint64_t ss) {
    const uint64_t total = block_sum_sat<NT>(ss, red);  // in every lane of warp 0
    if (threadIdx.x < 32) {
      const int32_t sc = inv_sqrt_acc_fast(acc_add_sat((int64_t)div_round_even_width(total, K), a.eps));
      if (threadIdx.x == 0) *s_scale = sc;
    }
    part_sync<NT>();
    return *s_scale;
  };
  auto norm1 = [](int32_t v, int32_t sc, int32_t w, bool weighted) {
    const int32_t y = mul_sat(v, sc);
    return weighted ? mul_sat(y, w) : y;
  };
  uint64_t ss = 0;
#pragma unroll
  for (uint32_t j = 0; j < kHeld; ++j) ss = sq4(ss, ov[j]);
  const int32_t sc1 = row_scale(ss);
  const bool wp = a.post_w != nullptr, wn = a.norm_w != nullptr;
  ss = 0;
#pragma unroll
  for (uint32_t j = 0; j < kHeld; ++j) {
    const uint32_t i = threadIdx.x * 4 + j * step;
    int4 v = xv[j];
    v.x = add_sat(norm1(ov[j].x, sc1, w1[j].x, wp), v.x);
    v.y = add_sat(norm1(ov[j].y, sc1, w1[j].y, wp), v.y);
    v.z = add_sat(norm1(ov[j].z, sc1, w1[j].z, wp), v.z);
    v.w = add_sat(norm1(ov[j].w, sc1, w1[j].w, wp), v.w);
    if (i >= K) v = z;
    xv[j] = v;
    if (blockIdx.x == 0 && i < K) *(int4*)(a.post_x + i) = v;
    ss = sq4(ss, v);
  }
  const int32_t sc2 = row_scale(ss);
  int wide = 0;
#pragma unroll
  for (uint32_t j = 0; j < kHeld; ++j) {
    const uint32_t i = threadIdx.x * 4 + j * step;
    if (i >= K) continue;
    int4 v = xv[j];
    v.x = norm1(v.x, sc2, w2[j].x, wn);
    v.y = norm1(v.y, sc2, w2[j].y, wn);
    v.z = norm1(v.z, sc2, w2[j].z, wn);
    v.w = norm1(v.w, sc2, w2[j].w, wn);
    wide |= !fits_three_planes(v.x) | !fits_three_planes(v.y) | !fits_three_planes(v.z) | !fits_three_planes(v.w);
    put_planes4(planes, K, i, v);
  }
  return part_or<NT>(wide);
}

// ---------------------------------------------------------------------------
// Decode GEMV pieces
// ---------------------------------------------------------------------------

constexpr int kTmaConsumerWarps = 16;
constexpr int kTmaEpilogueWarp = kTmaConsumerWarps + 1;
constexpr int kTmaThreads = (kTmaConsumerWarps + 2) * 32;
constexpr int kTmaRowsPerWarp = 2;
constexpr uint32_t kTmaMaxStages = 8;
constexpr uint32_t kTmaSlots = 4;  // tile groups between the consumers and the epilogue warp
constexpr uint32_t kTmaSmemBudget = 220 * 1024;

struct GemvPlan {
  uint32_t stages;
  uint32_t stage_bytes;      // tile values (16 kc) + tile scales (kc), rounded to 128
  uint32_t planes_bytes;     // 4 K, rounded to 128
  uint32_t items;            // tiles of the matrix: groups * nslices
  uint32_t groups_per_block; // whole-group ranges (split == 0)
  uint32_t split;            // even item ranges through the split scratch
  int32_t e_fast;            // largest scale exponent of the 64-bit accumulator (-1: none)
  uint32_t smem;
  uint32_t grid;
};

__host__ __device__ inline uint32_t round_up(uint32_t v, uint32_t m) { return (v + m - 1) / m * m; }


// One warp's share of a tile: two rows, one 32-value block b of the slice a
// lane (a half slice is at most 32 blocks). The lane first copies its weights
// and scale bits out of the stage into registers, so that the warp can release
// the stage before the products run and the producer refills it at once.
// Lanes 4-7 of every quarter-warp take the two 16-byte chunks in the other
// order, so that each 8-lane phase of a 128-bit shared load touches 8
// different 16-byte bank groups (the block sum does not depend on the order).
struct RowBlocks {
  uint4 wa[kTmaRowsPerWarp], wb[kTmaRowsPerWarp];
  uint16_t sc[kTmaRowsPerWarp];
};

__device__ __forceinline__ void gemv_take_rows(const uint8_t* __restrict__ W, const uint16_t* __restrict__ Sc,
                                               uint32_t kc, uint32_t b, uint32_t lane, RowBlocks& rb) {
  const uint32_t blocks = kc / 32, swap = (lane >> 2) & 1;
  const uint32_t c0 = 2 * b + swap, c1 = 2 * b + (swap ^ 1);
#pragma unroll
  for (int r = 0; r < kTmaRowsPerWarp; ++r) {
    rb.wa[r] = *(const uint4*)(W + r * kc + c0 * 16);
    rb.wb[r] = *(const uint4*)(W + r * kc + c1 * 16);
    rb.sc[r] = Sc[r * blocks + b];
  }
}

// The exact block sums of one lane's block for its two rows, times the
// scales, into the row accumulators. Three planes (|a| < 2^23): one dp4a
// chain a plane over the whole block (|s0|, |s1| < 2^20, |s2| < 2^19), then
// p = (s0 + 256 s1) m + 2^16 (s2 m) with |p| < 2^46.1; a term p 2^e with
// e <= e_fast goes to a 64-bit accumulator (the plan bounds the terms a lane
// adds for a row so that their sum stays below 2^62), any other to the
// 128-bit one. Four planes: the low pair and the high pair of planes are two
// products, lo = (s0 + 256 s1) m and hi = (s2 + 256 s3) m, both below 2^39.1,
// kept in two 64-bit accumulators (fast, fast_hi; a = lo + 2^16 hi) while
// e <= e_fast + 8 (S terms of 2^(39.1 + e) stay below 2^63), else added as
// lo + 2^16 hi (below 2^55) to the 128-bit one.
template <bool kThree>
__device__ __forceinline__ void gemv_rows_product(const RowBlocks& rb, const uint4* __restrict__ P0,
                                                  const uint4* __restrict__ P1, const uint4* __restrict__ P2,
                                                  const uint4* __restrict__ P3, uint32_t cbase, uint32_t b,
                                                  uint32_t lane, int32_t e_fast, Acc128* acc, int64_t* fast,
                                                  int64_t* fast_hi) {
  const uint32_t swap = (lane >> 2) & 1;
  const uint32_t c0 = 2 * b + swap, c1 = 2 * b + (swap ^ 1);
  const uint4 pa0 = P0[cbase + c0], pa1 = P1[cbase + c0], pa2 = P2[cbase + c0];
  const uint4 pb0 = P0[cbase + c1], pb1 = P1[cbase + c1], pb2 = P2[cbase + c1];
  uint4 pa3, pb3;
  if (!kThree) {
    pa3 = P3[cbase + c0];
    pb3 = P3[cbase + c1];
  }
#pragma unroll
  for (int r = 0; r < kTmaRowsPerWarp; ++r) {
    int32_t m, e;
    q8_scale_parts(rb.sc[r], &m, &e);  // finite: checked at upload (padding rows: 0)
    if (kThree) {
      const uint4 wa = rb.wa[r], wb = rb.wb[r];
      int s0 = dp4a_su(wa.x, pa0.x, 0), s1 = dp4a_su(wa.x, pa1.x, 0), s2 = dp4a_ss(wa.x, pa2.x, 0);
      s0 = dp4a_su(wa.y, pa0.y, s0), s1 = dp4a_su(wa.y, pa1.y, s1), s2 = dp4a_ss(wa.y, pa2.y, s2);
      s0 = dp4a_su(wa.z, pa0.z, s0), s1 = dp4a_su(wa.z, pa1.z, s1), s2 = dp4a_ss(wa.z, pa2.z, s2);
      s0 = dp4a_su(wa.w, pa0.w, s0), s1 = dp4a_su(wa.w, pa1.w, s1), s2 = dp4a_ss(wa.w, pa2.w, s2);
      s0 = dp4a_su(wb.x, pb0.x, s0), s1 = dp4a_su(wb.x, pb1.x, s1), s2 = dp4a_ss(wb.x, pb2.x, s2);
      s0 = dp4a_su(wb.y, pb0.y, s0), s1 = dp4a_su(wb.y, pb1.y, s1), s2 = dp4a_ss(wb.y, pb2.y, s2);
      s0 = dp4a_su(wb.z, pb0.z, s0), s1 = dp4a_su(wb.z, pb1.z, s1), s2 = dp4a_ss(wb.z, pb2.z, s2);
      s0 = dp4a_su(wb.w, pb0.w, s0), s1 = dp4a_su(wb.w, pb1.w, s1), s2 = dp4a_ss(wb.w, pb2.w, s2);
      const int64_t p = (int64_t)(s0 + s1 * 256) * m + ((int64_t)(s2 * m) << 16);
      if (e <= e_fast) fast[r] += (int64_t)((uint64_t)p << e);
      else acc128_add_shifted(acc[r], p, e);
    } else {
      const uint4 wa = rb.wa[r], wb = rb.wb[r];
      int s0 = dp4a_su(wa.x, pa0.x, 0), s1 = dp4a_su(wa.x, pa1.x, 0), s2 = dp4a_su(wa.x, pa2.x, 0),
          s3 = dp4a_ss(wa.x, pa3.x, 0);
      s0 = dp4a_su(wa.y, pa0.y, s0), s1 = dp4a_su(wa.y, pa1.y, s1), s2 = dp4a_su(wa.y, pa2.y, s2), s3 = dp4a_ss(wa.y, pa3.y, s3);
      s0 = dp4a_su(wa.z, pa0.z, s0), s1 = dp4a_su(wa.z, pa1.z, s1), s2 = dp4a_su(wa.z, pa2.z, s2), s3 = dp4a_ss(wa.z, pa3.z, s3);
      s0 = dp4a_su(wa.w, pa0.w, s0), s1 = dp4a_su(wa.w, pa1.w, s1), s2 = dp4a_su(wa.w, pa2.w, s2), s3 = dp4a_ss(wa.w, pa3.w, s3);
      s0 = dp4a_su(wb.x, pb0.x, s0), s1 = dp4a_su(wb.x, pb1.x, s1), s2 = dp4a_su(wb.x, pb2.x, s2), s3 = dp4a_ss(wb.x, pb3.x, s3);
      s0 = dp4a_su(wb.y, pb0.y, s0), s1 = dp4a_su(wb.y, pb1.y, s1), s2 = dp4a_su(wb.y, pb2.y, s2), s3 = dp4a_ss(wb.y, pb3.y, s3);
      s0 = dp4a_su(wb.z, pb0.z, s0), s1 = dp4a_su(wb.z, pb1.z, s1), s2 = dp4a_su(wb.z, pb2.z, s2), s3 = dp4a_ss(wb.z, pb3.z, s3);
      s0 = dp4a_su(wb.w, pb0.w, s0), s1 = dp4a_su(wb.w, pb1.w, s1), s2 = dp4a_su(wb.w, pb2.w, s2), s3 = dp4a_ss(wb.w, pb3.w, s3);
      const int64_t lo = (int64_t)(s0 + s1 * 256) * m, hi = (int64_t)(s2 + s3 * 256) * m;
      if (e <= e_fast + 8) {
        fast[r] += (int64_t)((uint64_t)lo << e);
        fast_hi[r] += (int64_t)((uint64_t)hi << e);
      } else {
        acc128_add_shifted(acc[r], lo + (int64_t)((uint64_t)hi << 16), e);
      }
    }
  }
}

// Rows with one scale (every block of the row has the same scale bits): the
// lane's plane sums of its block for its two rows, added into int32 plane
// accumulators that run over the lane's blocks of a whole tile group; the
// scale is applied once a group (gemv_flush_uniform). Over a group a lane
// adds S blocks of 32 products below 128 * 255 in magnitude: below 2^31 for
// S < 2056.
template <bool kThree>
__device__ __forceinline__ void gemv_rows_sums(const RowBlocks& rb, const uint4* __restrict__ P0,
                                               const uint4* __restrict__ P1, const uint4* __restrict__ P2,
                                               const uint4* __restrict__ P3, uint32_t cbase, uint32_t b,
                                               uint32_t lane, int32_t (&ps)[kTmaRowsPerWarp][4]) {
  const uint32_t swap = (lane >> 2) & 1;
  const uint32_t c0 = 2 * b + swap, c1 = 2 * b + (swap ^ 1);
  const uint4 pa0 = P0[cbase + c0], pa1 = P1[cbase + c0], pa2 = P2[cbase + c0];
  const uint4 pb0 = P0[cbase + c1], pb1 = P1[cbase + c1], pb2 = P2[cbase + c1];
  uint4 pa3, pb3;
  if (!kThree) {
    pa3 = P3[cbase + c0];
    pb3 = P3[cbase + c1];
  }
#pragma unroll
  for (int r = 0; r < kTmaRowsPerWarp; ++r) {
    const uint4 wa = rb.wa[r], wb = rb.wb[r];
    int s0 = ps[r][0], s1 = ps[r][1], s2 = ps[r][2];
    if (kThree) {
      s0 = dp4a_su(wa.x, pa0.x, s0), s1 = dp4a_su(wa.x, pa1.x, s1), s2 = dp4a_ss(wa.x, pa2.x, s2);
      s0 = dp4a_su(wa.y, pa0.y, s0), s1 = dp4a_su(wa.y, pa1.y, s1), s2 = dp4a_ss(wa.y, pa2.y, s2);
      s0 = dp4a_su(wa.z, pa0.z, s0), s1 = dp4a_su(wa.z, pa1.z, s1), s2 = dp4a_ss(wa.z, pa2.z, s2);
      s0 = dp4a_su(wa.w, pa0.w, s0), s1 = dp4a_su(wa.w, pa1.w, s1), s2 = dp4a_ss(wa.w, pa2.w, s2);
      s0 = dp4a_su(wb.x, pb0.x, s0), s1 = dp4a_su(wb.x, pb1.x, s1), s2 = dp4a_ss(wb.x, pb2.x, s2);
      s0 = dp4a_su(wb.y, pb0.y, s0), s1 = dp4a_su(wb.y, pb1.y, s1), s2 = dp4a_ss(wb.y, pb2.y, s2);
      s0 = dp4a_su(wb.z, pb0.z, s0), s1 = dp4a_su(wb.z, pb1.z, s1), s2 = dp4a_ss(wb.z, pb2.z, s2);
      s0 = dp4a_su(wb.w, pb0.w, s0), s1 = dp4a_su(wb.w, pb1.w, s1), s2 = dp4a_ss(wb.w, pb2.w, s2);
    } else {
      int s3 = ps[r][3];
      s0 = dp4a_su(wa.x, pa0.x, s0), s1 = dp4a_su(wa.x, pa1.x, s1), s2 = dp4a_su(wa.x, pa2.x, s2), s3 = dp4a_ss(wa.x, pa3.x, s3);
      s0 = dp4a_su(wa.y, pa0.y, s0), s1 = dp4a_su(wa.y, pa1.y, s1), s2 = dp4a_su(wa.y, pa2.y, s2), s3 = dp4a_ss(wa.y, pa3.y, s3);
      s0 = dp4a_su(wa.z, pa0.z, s0), s1 = dp4a_su(wa.z, pa1.z, s1), s2 = dp4a_su(wa.z, pa2.z, s2), s3 = dp4a_ss(wa.z, pa3.z, s3);
      s0 = dp4a_su(wa.w, pa0.w, s0), s1 = dp4a_su(wa.w, pa1.w, s1), s2 = dp4a_su(wa.w, pa2.w, s2), s3 = dp4a_ss(wa.w, pa3.w, s3);
      s0 = dp4a_su(wb.x, pb0.x, s0), s1 = dp4a_su(wb.x, pb1.x, s1), s2 = dp4a_su(wb.x, pb2.x, s2), s3 = dp4a_ss(wb.x, pb3.x, s3);
      s0 = dp4a_su(wb.y, pb0.y, s0), s1 = dp4a_su(wb.y, pb1.y, s1), s2 = dp4a_su(wb.y, pb2.y, s2), s3 = dp4a_ss(wb.y, pb3.y, s3);
      s0 = dp4a_su(wb.z, pb0.z, s0), s1 = dp4a_su(wb.z, pb1.z, s1), s2 = dp4a_su(wb.z, pb2.z, s2), s3 = dp4a_ss(wb.z, pb3.z, s3);
      s0 = dp4a_su(wb.w, pb0.w, s0), s1 = dp4a_su(wb.w, pb1.w, s1), s2 = dp4a_su(wb.w, pb2.w, s2), s3 = dp4a_ss(wb.w, pb3.w, s3);
      ps[r][3] = s3;
    }
    ps[r][0] = s0, ps[r][1] = s1, ps[r][2] = s2;
  }
}

// The end of a tile group for rows with one scale: the warp's exact row sum
// x = sum over its lanes of s0 + 2^8 s1 + 2^16 s2 + 2^24 s3 (the products of
// the row's weights in this half with the whole activations: below
// K 2^37 in magnitude), then x m 2^e (m, e: the row's scale, q8.rs:27-43)
// as a 128-bit value; |x m| < 2^63 for K <= 32768.
__device__ __forceinline__ Acc128 gemv_flush_uniform(const int32_t (&ps)[4], uint16_t scale_bits) {
  int64_t x = (int64_t)ps[0] + (int64_t)ps[1] * 256 + (int64_t)ps[2] * 65536 + (int64_t)ps[3] * 16777216;
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) x += __shfl_xor_sync(0xffffffffu, x, off);
  int32_t m = 0, e = 0;
  q8_scale_parts_finite(scale_bits, &m, &e);
  Acc128 v{0, 0};
  acc128_add_shifted(v, x * m, e);
  return v;
}

// Item range [*ib, *ie) of block b.
__device__ __forceinline__ void gemv_range(const GemvPlan& p, uint32_t S, uint32_t groups, uint32_t b,
                                           uint32_t* ib, uint32_t* ie) {
  if (p.split) {
    *ib = (uint32_t)((uint64_t)b * p.items / p.grid);
    *ie = (uint32_t)((uint64_t)(b + 1) * p.items / p.grid);
  } else {
    const uint32_t g0 = b * p.groups_per_block, g1 = min(groups, g0 + p.groups_per_block);
    *ib = g0 * S;
    *ie = g0 < g1 ? g1 * S : g0 * S;
  }
}

// Exact 128-bit addition into the split scratch (two 64-bit words a row).
__device__ __forceinline__ void atomic_add_acc128(unsigned long long* dst, Acc128 v) {
  const unsigned long long old = atomicAdd(dst, (unsigned long long)v.lo);
  const unsigned long long carry = old + v.lo < old ? 1ull : 0ull;
  atomicAdd(dst + 1, (unsigned long long)v.hi + carry);
}

// Release add of 1 on a global counter (the writes ordered before it first).
__device__ __forceinline__ void gemv_red_add_release(unsigned int* p) {
  asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(p) : "memory");
}

// The epilogue of one finished tile group: lane l < 16 holds the rounded value
// of row g * 16 + l. Single-row epilogues return the value the lane wrote
// (0 for none).
template <int EPI>
__device__ __forceinline__ int32_t gemv_group_epilogue(const ProductArgs& a, uint32_t g, int32_t v, uint32_t lane,
                                                       unsigned long long* best) {
  const uint32_t row0 = g * kQ8TileRows;
  if (EPI == EPI_QKV_ROPE || EPI == EPI_SILU_MUL || EPI == EPI_GELU_MUL) {
    // pairs (2j, 2j + 1): lane j < 8 takes pair j
    const int32_t v0 = __shfl_sync(0xffffffffu, v, (2 * lane) & 31);
    const int32_t v1 = __shfl_sync(0xffffffffu, v, (2 * lane + 1) & 31);
    const uint32_t row = row0 + 2 * lane;
    if (lane < kQ8TileRows / 2 && row + 1 < a.rows) epi_pair<EPI>(a, 0, row, v0, v1);
  } else if (EPI == EPI_LOGITS) {
    const uint32_t row = row0 + lane;
    if (lane < kQ8TileRows && row < a.rows) {
      const int32_t c = a.softcap > 0 ? softcap_act(v, a.softcap) : v;
      if (a.out) a.out[row] = c;
      const unsigned long long key = best_key(c, row + a.row_base);
      *best = key > *best ? key : *best;
    }
  } else {
    const uint32_t row = row0 + lane;
    if (lane < kQ8TileRows && row < a.rows) return epi_single<EPI>(a, 0, row, v);
  }
  return 0;
}

// ---------------------------------------------------------------------------
// The tile ring: producer, consumer and epilogue loops
// ---------------------------------------------------------------------------
//
// A block streams matrix tiles through a ring of shared-memory slots: lane 0
// of the producer warp issues each tile's two bulk copies into the next slot
// once the consumers released it; the sixteen consumer warps take each tile
// into registers, release the slot and run the products; at the end of each
// tile group they hand the group's 128-bit row sums to the epilogue warp
// through a small ring of sum slots. Cursors persist across products, so a
// persistent kernel can run many products through one ring, the producer
// running ahead into the next product's tiles while the consumers wait for
// its input.

// Waits for the phase of `bar` with the given parity (bounded: about one
// second, a give-up recorded in *fault). kWatch: also gives up as soon as any
// thread of the device recorded a fault, so that a stalled persistent kernel
// drains quickly instead of waiting out every later wait.
template <bool kWatch>
__device__ __forceinline__ bool ring_wait(uint64_t* bar, uint32_t parity, unsigned int* fault) {
  if (!kWatch) return mbar_wait_bounded(bar, parity, fault);
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait_suspend(bar, parity)) return true;
    if ((i & 15) == 0) {
      if (*(volatile unsigned int*)fault) return false;
      if (global_ns() - t0 > 1000000000ull) {
        atomicOr(fault, 1u);
        return false;
      }
    }
  }
}

struct TileRing {
  uint8_t* base;             // slots of slot_bytes bytes
  uint32_t slot_bytes, slots;
  uint64_t* full;            // [slots]: the slot's copies landed (count 1 + bytes)
  uint64_t* empty;           // [slots]: released by every consumer warp
};
// A position in the ring: next slot and the parity of the phase to wait for.
// The producer starts at {0, 1, 0} (the first `slots` tiles need no release),
// the consumers at {0, 0, 0}.
struct RingCursor {
  uint32_t slot, parity, count;
};
__device__ __forceinline__ void ring_advance(const TileRing& r, RingCursor& c) {
  ++c.count;
  if (++c.slot == r.slots) {
    c.slot = 0;
    c.parity ^= 1;
  }
}

// Sum slots between the consumer warps and the epilogue warp.
struct SumRing {
  uint64_t* full;   // [kTmaSlots]: written by every consumer warp
  uint64_t* empty;  // [kTmaSlots]: read by the epilogue warp
  Acc128 (*sums)[2][kQ8TileRows];  // [slot][half of the slice][row of the tile]
};

// Producer (one lane): tiles [ib, ie) of the matrix (q, s) with slices of kc
// columns. Returns false after a given-up wait.
template <bool kWatch>
__device__ __forceinline__ bool ring_issue(const TileRing& r, RingCursor& c, const int8_t* q, const uint16_t* s,
                                           uint32_t kc, uint32_t ib, uint32_t ie, uint64_t policy,
                                           unsigned int* fault) {
  for (uint32_t t = ib; t < ie; ++t) {
    if (c.count >= r.slots && !ring_wait<kWatch>(&r.empty[c.slot], c.parity, fault)) return false;
    uint8_t* dst = r.base + c.slot * r.slot_bytes;
    mbar_arrive_expect_tx(&r.full[c.slot], kQ8TileRows * kc + kc);
    bulk_load(dst, q + (size_t)t * kQ8TileRows * kc, kQ8TileRows * kc, &r.full[c.slot], policy);
    bulk_load(dst + kQ8TileRows * kc, (const uint8_t*)s + (size_t)t * kc, kc, &r.full[c.slot], policy);
    ring_advance(r, c);
  }
  return true;
}

// Lets the copies issued last land (bounded) before the block exits.
__device__ __forceinline__ void ring_drain(const TileRing& r, const RingCursor& c, unsigned int* fault) {
  const uint32_t n = c.count, first = n > r.slots ? n - r.slots : 0;
  for (uint32_t t = first; t < n; ++t) mbar_wait_bounded(&r.full[t % r.slots], (t / r.slots) & 1, fault);
}

// Consumer warps: the products of tiles [ib, ie) (slices of kc columns, S a
// row) against the activation planes of K values. Warp w takes rows 2 (w % 8)
// and 2 (w % 8) + 1 of each tile, blocks of the slice's first (w < 8) or
// second half. j counts the sum slots used; after a given-up wait `stalled`
// keeps the warp in step with the others without waiting.

template <bool kWatch, bool kUniform>
__device__ __forceinline__ void ring_consume_impl(const TileRing& r, RingCursor& c, const SumRing& sr, uint32_t& j,
                                                  const uint8_t* planes, bool wide, uint32_t K, uint32_t kc,
                                                  uint32_t S, int32_t e_fast, uint32_t ib, uint32_t ie,
                                                  bool& stalled, unsigned int* fault) {
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint4* P0 = (const uint4*)planes;
  const uint4* P1 = P0 + K / 16;
  const uint4* P2 = P1 + K / 16;
  const uint4* P3 = P2 + K / 16;
  constexpr uint32_t kHalves = kTmaConsumerWarps / 8;
  static_assert(kHalves == 2, "a lane takes one block a row: 2048-value slices need two halves");
  const uint32_t pair = warp % 8, half = warp / 8;
  const uint32_t lr0 = kTmaRowsPerWarp * pair, blocks = kc / 32, mid = (blocks + 1) / 2;
  const uint32_t b0 = half ? mid : 0, b1 = half ? blocks : mid;
  Acc128 acc[kTmaRowsPerWarp];
  int64_t fast[kTmaRowsPerWarp], fast_hi[kTmaRowsPerWarp];
  int32_t ps[kTmaRowsPerWarp][4];  // one scale a row: plane sums of the group so far
#pragma unroll
  for (int i = 0; i < kTmaRowsPerWarp; ++i) {
    acc[i] = Acc128{0, 0};
    fast[i] = 0;
    fast_hi[i] = 0;
    ps[i][0] = ps[i][1] = ps[i][2] = ps[i][3] = 0;
  }
  uint32_t sl = ib % S;  // slice of the current tile, kept without divisions
  for (uint32_t t = ib; t < ie; ++t) {
    if (!stalled && !ring_wait<kWatch>(&r.full[c.slot], c.parity, fault)) stalled = true;
    const uint8_t* st = r.base + c.slot * r.slot_bytes;
    const uint8_t* W = st + lr0 * kc;
    const uint16_t* Sc = (const uint16_t*)(st + kQ8TileRows * kc) + lr0 * blocks;
    const uint32_t cbase = sl * (kc / 16), b = b0 + lane;
    RowBlocks rb;
    if (b < b1) gemv_take_rows(W, Sc, kc, b, lane, rb);
    else
#pragma unroll
      for (int i = 0; i < kTmaRowsPerWarp; ++i) rb.sc[i] = 0;  // a lane without a block adds nothing
    __syncwarp();
    if (lane == 0) mbar_arrive(&r.empty[c.slot]);  // the tile is in registers: refill the slot
    ring_advance(r, c);
    if (b < b1) {
      if (kUniform) {
        if (wide) gemv_rows_sums<false>(rb, P0, P1, P2, P3, cbase, b, lane, ps);
        else gemv_rows_sums<true>(rb, P0, P1, P2, P3, cbase, b, lane, ps);
      } else {
        if (wide) gemv_rows_product<false>(rb, P0, P1, P2, P3, cbase, b, lane, e_fast, acc, fast, fast_hi);
        else gemv_rows_product<true>(rb, P0, P1, P2, P3, cbase, b, lane, e_fast, acc, fast, fast_hi);
      }
    }
    if (++sl == S) sl = 0;
    if (sl == 0 || t + 1 == ie) {  // the end of a tile group in this range
#pragma unroll
      for (int i = 0; i < kTmaRowsPerWarp; ++i) {
        if (kUniform) {
          // lane 0 has a block whenever any lane does; then its scale is the row's
          acc[i] = gemv_flush_uniform(ps[i], __shfl_sync(0xffffffffu, rb.sc[i], 0));
          ps[i][0] = ps[i][1] = ps[i][2] = ps[i][3] = 0;
        } else {
          acc128_add(acc[i], (uint64_t)fast[i], fast[i] >> 63);
          acc128_add(acc[i], (uint64_t)fast_hi[i] << 16, fast_hi[i] >> 48);  // 2^16 fast_hi
          acc[i] = warp_sum_acc128(acc[i]);
          fast[i] = 0;
          fast_hi[i] = 0;
        }
      }
      const uint32_t slot = j % kTmaSlots;
      if (j >= kTmaSlots && !stalled && !ring_wait<kWatch>(&sr.empty[slot], (j / kTmaSlots - 1) & 1, fault))
        stalled = true;
      if (lane == 0) {
        sr.sums[slot][half][lr0] = acc[0];
        sr.sums[slot][half][lr0 + 1] = acc[1];
        mbar_arrive(&sr.full[slot]);
      }
      ++j;
#pragma unroll
      for (int i = 0; i < kTmaRowsPerWarp; ++i) acc[i] = Acc128{0, 0};
    }
  }
}

// The consumer loop for a matrix whose rows each have one scale (uniform:
// scaled once a tile group) or per-block scales.
template <bool kWatch>
__device__ __forceinline__ void ring_consume(const TileRing& r, RingCursor& c, const SumRing& sr, uint32_t& j,
                                             const uint8_t* planes, bool wide, bool uniform, uint32_t K,
                                             uint32_t kc, uint32_t S, int32_t e_fast, uint32_t ib, uint32_t ie,
                                             bool& stalled, unsigned int* fault) {
  if (uniform)
    ring_consume_impl<kWatch, true>(r, c, sr, j, planes, wide, K, kc, S, e_fast, ib, ie, stalled, fault);
  else
    ring_consume_impl<kWatch, false>(r, c, sr, j, planes, wide, K, kc, S, e_fast, ib, ie, stalled, fault);
}

// Epilogue warp: the tile groups overlapping tiles [ib, ie) (S tiles a
// group). A group split between blocks is added into the split scratch with
// exact 128-bit atomics; the block whose share completes the group's slice
// count rounds it once (q8.rs:69-71) and applies the epilogue. Returns false
// after a given-up wait.
//
template <int EPI, bool kWatch>
__device__ __forceinline__ bool ring_epilogue(const ProductArgs& a, const SumRing& sr, uint32_t& j, uint32_t ib,
                                              uint32_t ie, uint32_t S, unsigned int* fault) {
  // Paired epilogues (RoPE, SiLU / GELU gating) cost hundreds of dependent
  // integer operations a pair and take one lane a pair, eight a group: the
  // warp takes up to four finished groups at once (lane 8 q + p: pair p of
  // the q-th), every slot released as soon as it is read.
  constexpr bool kPaired = EPI == EPI_QKV_ROPE || EPI == EPI_SILU_MUL || EPI == EPI_GELU_MUL;
  constexpr uint32_t kBatch = kPaired ? 4 : 1;
  static_assert(kBatch <= kTmaSlots, "a batch fits the sum slots");
  const uint32_t lane = threadIdx.x & 31;
  const uint32_t gfirst = ib / S, ngroups = ie > ib ? (ie - 1) / S - gfirst + 1 : 0;
  // EPI_PARTIAL into a double-buffered peer-exchange slot: the one of the
  // coming exchange (epoch + 1)
  int64_t* part = a.partial;
  if (EPI == EPI_PARTIAL && a.xepoch) part += (size_t)((*a.xepoch + 1) & 1) * a.rows * 4;
  // RoPE: the sine and cosine of every frequency at the token's position,
  // once a call (the warp computes them while the first groups are consumed)
  __shared__ int64_t rope_sc[kRopeTablePairs][2];
  const bool rope_table = EPI == EPI_QKV_ROPE && a.head_dim / 2 <= kRopeTablePairs;
  uint32_t rope_pos = 0;
  if (EPI == EPI_QKV_ROPE && rope_table) {
    rope_pos = token_position(a, 0);
    if (rope_pos)
      for (uint32_t i = lane; i < a.head_dim / 2; i += 32)
        sin_cos_q30((int64_t)rope_pos * a.freqs[i], &rope_sc[i][0], &rope_sc[i][1]);
    __syncwarp();
  }
  unsigned long long best = 0;
  Acc128 squares{0, 0};  // EPI_RESID with a.sumsq: this lane's written values, squared
  bool ok = true;
  for (uint32_t k0 = 0; k0 < ngroups; k0 += kBatch) {
    const uint32_t nbat = min(kBatch, ngroups - k0);
    int32_t r[kBatch];    // lane l < 16: the rounded value of row l of the batch's q-th group
    uint32_t fin = 0;     // bit q: this block completes the q-th group
#pragma unroll
    for (uint32_t q = 0; q < kBatch; ++q) {
      r[q] = 0;
      if (q >= nbat) continue;
      const uint32_t sl = j % kTmaSlots, g = gfirst + k0 + q;
      if (!ring_wait<kWatch>(&sr.full[sl], (j / kTmaSlots) & 1, fault)) {
        ok = false;
        if (!kWatch) return false;
      }
      Acc128 v = Acc128{0, 0};
      if (lane < kQ8TileRows) {
        v = sr.sums[sl][0][lane];
        acc128_add(v, sr.sums[sl][1][lane].lo, sr.sums[sl][1][lane].hi);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sr.empty[sl]);
      ++j;
      const uint32_t lo = max(ib, g * S), hi = min(ie, (g + 1) * S);
      if (hi - lo < S) {  // a share of a group split between blocks
        unsigned long long* acc = a.split_acc + (size_t)g * kQ8TileRows * 2;
        if (lane < kQ8TileRows) atomic_add_acc128(acc + 2 * lane, v);
        __threadfence();
        __syncwarp();
        uint32_t done = 0;
        if (lane == 0) done = atomicAdd(a.split_count + g, hi - lo) + (hi - lo) == S;
        if (!__shfl_sync(0xffffffffu, done, 0)) continue;
        __threadfence();
        if (lane < kQ8TileRows) {
          v.lo = (uint64_t)__ldcg(acc + 2 * lane);
          v.hi = (int64_t)__ldcg(acc + 2 * lane + 1);
          acc[2 * lane] = 0;
          acc[2 * lane + 1] = 0;
        }
        if (lane == 0) a.split_count[g] = 0;
      }
      fin |= 1u << q;
      if (EPI == EPI_PARTIAL) {
        const uint32_t row = g * kQ8TileRows + lane;
        if (lane < kQ8TileRows && row < a.rows) limbs_from_acc128(v.lo, v.hi, part + (size_t)row * 4);
      } else if (kPaired) {
        r[q] = acc128_round_q24(v);
      } else {
        const int32_t y = gemv_group_epilogue<EPI>(a, g, acc128_round_q24(v), lane, &best);
        if (EPI == EPI_RESID && a.sumsq) acc128_add(squares, (uint64_t)((int64_t)y * y), 0);
      }
    }
    if (kPaired) {
      const uint32_t q = lane >> 3, pr = lane & 7;
      int32_t v0 = 0, v1 = 0;
#pragma unroll
      for (uint32_t qq = 0; qq < kBatch; ++qq) {
        const int32_t t0 = __shfl_sync(0xffffffffu, r[qq], 2 * pr), t1 = __shfl_sync(0xffffffffu, r[qq], 2 * pr + 1);
        if (qq == q) v0 = t0, v1 = t1;
      }
      const uint32_t row = (gfirst + k0 + q) * kQ8TileRows + 2 * pr;
      if (q < nbat && ((fin >> q) & 1) && row + 1 < a.rows) {
        if (EPI == EPI_QKV_ROPE && rope_table) epi_pair_rope_sc(a, rope_pos, row, v0, v1, rope_sc);
        else epi_pair<EPI>(a, 0, row, v0, v1);
      }
      if (EPI == EPI_QKV_ROPE && a.gready) {
        // each finished group's rows, stored by this batch's lanes (ordered
        // before the adds by __syncwarp), to the attention groups reading them
        __syncwarp();
        if (lane < nbat && ((fin >> lane) & 1)) {
          const uint32_t r0 = (gfirst + k0 + lane) * kQ8TileRows, G = a.qd / a.kvd;  // query heads a kv head
          const uint32_t hpc = a.gready_hpc, per_kv = G / hpc;  // attention groups a kv head
          if (r0 < a.qd) {
            gemv_red_add_release(a.gready + r0 / a.head_dim / hpc);
          } else {
            const uint32_t kh = ((r0 - a.qd) % a.kvd) / a.head_dim;  // the K or V rows' kv head
            for (uint32_t j = 0; j < per_kv; ++j) gemv_red_add_release(a.gready + kh * per_kv + j);
          }
        }
      }
    }
  }
  if (EPI == EPI_RESID && a.sumsq) {  // the block's share, clamped: the norm's sum saturates there anyway
    squares = warp_sum_acc128(squares);
    if (lane == 0) *a.sumsq = (squares.hi || squares.lo > (uint64_t)INT64_MAX) ? (uint64_t)INT64_MAX : squares.lo;
  }
  if (EPI == EPI_LOGITS) {
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
      const unsigned long long o = __shfl_xor_sync(0xffffffffu, best, off);
      best = o > best ? o : best;
    }
    if (lane == 0 && best) atomicMax(a.best, best);
  }
  return ok;
}

// Plans a decode GEMV over `sms` persistent blocks (q8.cu).
bool plan_gemv(uint32_t rows, uint32_t K, uint32_t kc, int sms, bool split, GemvPlan* p);

}  // namespace iris
