// The persistent decode step for mistral-dense models: one cooperative launch
// of one block per multiprocessor runs the whole pass of one token.
//
// The kernel-per-operation pass (model.cu) pays, at every one of its ~160
// kernel boundaries, the ramp and drain of a weight stream: the next product
// can only prefetch what fits beside the previous kernel's blocks, and the
// HBM pipe idles while the last tiles, the epilogue and the next prologue
// run. Here each block keeps ONE tile ring (gemv.cuh) for the whole pass:
// its producer lane walks the block's share of every matrix of every layer
// in pass order and never waits for data, only for free slots, so while the
// consumers wait for a stage's input (the arrival barrier below), attend, or
// normalise, the ring keeps filling with the next product's weights - about
// 20 MB across the GPU, several microseconds of HBM time.
//
// Stages (StepKind) run in pass order: embedding, then per layer q|k|v with
// RoPE and the cache store, attention, o with the residual, gate|up with
// SiLU gating, down with the residual, then the head and the greedy choice.
// Every block arrives once per stage on the stage's global counter after its
// share of the stage is written (release); a stage's consumers start after
// all blocks arrived at the stage before (acquire). Products split their
// tiles over the blocks in whole tile groups, so each block rounds its groups
// once and applies the fused epilogue itself, exactly as the one-product
// kernel does. The attention of a head group is split over `chunks` blocks
// that meet through global exchange words (first maximum, exp sums, value
// sums) with bounded group barriers, as in the whole-GPU attention kernel
// (layers.cu). The residual epilogues also leave the exact sum of squares of
// the stream they wrote, so a normalised input needs no block-wide reduction.
// The last block to arrive at the head stage selects the next token,
// advances the position and clears the counters for the next launch.
//
// All blocks must be resident at once: the launch is cooperative. Every wait
// is bounded (about one second); after any recorded fault every later wait
// gives up at once, so a stalled pass drains in milliseconds and the host
// reports IRIS_ESTALL.
#include <cuda_runtime.h>

#include <algorithm>

#include "../../include/iris_b200.h"
#include "gemv.cuh"
#include "step.cuh"

namespace iris {

namespace {

constexpr uint32_t kStepConsumers = kTmaConsumerWarps * 32;  // threads of the consumer warps
constexpr int kStepProducerWarp = kTmaConsumerWarps;
constexpr int kStepEpilogueWarp = kTmaEpilogueWarp;

__device__ __forceinline__ bool step_is_product(uint32_t kind) {
  return kind != STEP_EMBED && kind != STEP_ATTN && kind != STEP_XCHG;
}

// Tiles [*ib, *ie) of a product stage for block b of nb: whole tile groups,
// spread evenly (the counts differ by at most one group). Splitting groups
// between blocks would balance exactly but end every stage with an exchange
// of partial sums through L2 (dependent atomics, a fence, a re-read), which
// costs more than one group's stream (measured: 2,580 -> 2,828 us a pass).
__device__ __forceinline__ void step_range(const StepStage& st, uint32_t b, uint32_t nb, uint32_t* ib,
                                           uint32_t* ie) {
  const uint32_t groups = st.items / st.nslices;
  *ib = (uint32_t)((uint64_t)b * groups / nb) * st.nslices;
  *ie = (uint32_t)((uint64_t)(b + 1) * groups / nb) * st.nslices;
}

// Optional timeline stamp (one thread of the block).
__device__ __forceinline__ void step_stamp(const StepArgs& A, uint32_t k, uint32_t ev) {
  if (A.trace) A.trace[((size_t)blockIdx.x * A.nstages + k) * kStepTraceEvents + ev] = global_ns();
}

// Bounded poll of a global arrival counter (one thread).
__device__ __forceinline__ void step_poll(const unsigned int* ctr, unsigned int target, unsigned int* fault) {
  if (ld_acquire_u32(ctr) >= target) return;
  const uint64_t t0 = global_ns();
  for (uint32_t i = 1;; ++i) {
    if (ld_acquire_u32(ctr) >= target) return;
    if ((i & 63) == 0) {
      if (*(volatile unsigned int*)fault) return;
      if (global_ns() - t0 > 1000000000ull) {
        atomicOr(fault, 1u);
        return;
      }
    }
  }
}

// Consumer warps: every block has arrived at stage k - 1. Every stage has
// work for at least one block, and a block with work at a stage has waited
// for the stage before, so this also orders every earlier stage.
__device__ __forceinline__ void step_wait(const StepArgs& A, uint32_t k) {
  if (threadIdx.x == 0) {
    step_poll(A.sync + k - 1, gridDim.x, A.fault);
    step_stamp(A, k, 0);
  }
  part_sync<kStepConsumers>();
}

// Consumer warps: this block's share of stage k is written.
__device__ __forceinline__ void step_consumers_arrive(const StepArgs& A, uint32_t k) {
  part_sync<kStepConsumers>();
  if (threadIdx.x == 0) {
    step_stamp(A, k, 7);
    __threadfence();
    red_add_release(A.sync + k, 1u);
  }
}

// The sum of squares slots of stage k: one a block, each clamped to
// i64::MAX (the norm's saturating sum of non-negative terms clamps there too).
__device__ __forceinline__ unsigned long long* step_sumsq_slot(const StepArgs& A, uint32_t k) {
  return A.sumsq + (size_t)k * gridDim.x + blockIdx.x;
}

// x = dequantize_row(embed[token]) (q8.rs:76-91); blocks take 512 values
// each and leave the sum of the squares of theirs in their slot.
__device__ __forceinline__ void step_embed(const StepArgs& A, Acc128* warp_sq) {
  const uint32_t tok = *A.d_token;
  Acc128 sq{0, 0};
  for (uint32_t i = blockIdx.x * kStepConsumers + threadIdx.x; i < A.H; i += gridDim.x * kStepConsumers) {
    int32_t m, e;
    q8_scale_parts(A.embed_s[q8_scale_offset(A.embed_kc, A.embed_nslices, tok, i >> 5)], &m, &e);
    const int32_t v = q8_dequant(A.embed_q[q8_value_offset(A.embed_kc, A.embed_nslices, tok, i)], m, e);
    A.x[i] = v;
    acc128_add(sq, (uint64_t)((int64_t)v * v), 0);
  }
  sq = warp_sum_acc128(sq);
  if ((threadIdx.x & 31) == 0) warp_sq[threadIdx.x >> 5] = sq;
  part_sync<kStepConsumers>();
  if (threadIdx.x < 32) {
    Acc128 t = threadIdx.x < kStepConsumers / 32 ? warp_sq[threadIdx.x] : Acc128{0, 0};
    t = warp_sum_acc128(t);
    if (threadIdx.x == 0) *step_sumsq_slot(A, 0) = (t.hi || t.lo > (uint64_t)INT64_MAX) ? (uint64_t)INT64_MAX : t.lo;
  }
}

// The byte planes of rms_norm(x) (ops.rs:98-114) for a product whose input is
// the residual stream written by stage k - 1, which also left the 128-bit
// sum of the squares of x: the norm's sum of squares saturates at i64::MAX
// term by term (add_sat_nonneg), which for non-negative terms is the exact
// sum clamped to i64::MAX. wv holds this thread's
// norm weights (loaded before the stage's wait); x is read through L2.
template <uint32_t kHeld>
__device__ __forceinline__ bool step_norm_planes(const StepArgs& A, uint32_t k, uint32_t K, const int4 (&wv)[kHeld],
                                                 const int32_t* norm_w, uint8_t* planes, int32_t* s_scale) {
  constexpr uint32_t step = kStepConsumers * 4;
  const bool held = K <= kHeld * step;
  int4 xv[kHeld];
  if (held) {
#pragma unroll
    for (uint32_t j = 0; j < kHeld; ++j) {
      const uint32_t i = threadIdx.x * 4 + j * step;
      xv[j] = i < K ? __ldcg((const int4*)(A.x + i)) : make_int4(0, 0, 0, 0);
    }
  }
  if (threadIdx.x < 32) {  // the blocks' shares of stage k - 1, summed exactly, then clamped
    const unsigned long long* slots = A.sumsq + (size_t)(k - 1) * gridDim.x;
    Acc128 t{0, 0};
    for (uint32_t b = threadIdx.x; b < gridDim.x; b += 32) acc128_add(t, __ldcg(slots + b), 0);
    t = warp_sum_acc128(t);
    const uint64_t total = (t.hi || t.lo > (uint64_t)INT64_MAX) ? (uint64_t)INT64_MAX : t.lo;
    const int32_t sc = inv_sqrt_acc_fast(acc_add_sat((int64_t)div_round_even_width(total, K), A.eps));
    if (threadIdx.x == 0) *s_scale = sc;
  }
  part_sync<kStepConsumers>();
  if (threadIdx.x == 0) step_stamp(A, k, 3);
  const int32_t scale = *s_scale;
  int wide = 0;
  auto emit = [&](int4 v, int4 w, uint32_t i) {
    v.x = mul_sat(mul_sat(v.x, scale), w.x);
    v.y = mul_sat(mul_sat(v.y, scale), w.y);
    v.z = mul_sat(mul_sat(v.z, scale), w.z);
    v.w = mul_sat(mul_sat(v.w, scale), w.w);
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
      emit(__ldcg((const int4*)(A.x + i)), __ldg((const int4*)(norm_w + i)), i);
  }
  if (threadIdx.x == 0) step_stamp(A, k, 4);
  return part_or<kStepConsumers>(wide);
}

// Activation planes written by an earlier stage -> shared memory; true when
// some value needs the fourth plane.
__device__ __forceinline__ bool step_copy_planes(const uint8_t* src8, uint32_t K, uint8_t* planes) {
  const uint4* src = (const uint4*)src8;
  int w = 0;
  for (uint32_t i = threadIdx.x; i < K / 16; i += kStepConsumers) {
    const uint4 v0 = __ldcg(src + i), v1 = __ldcg(src + K / 16 + i), v2 = __ldcg(src + 2 * (K / 16) + i),
                v3 = __ldcg(src + 3 * (K / 16) + i);
    ((uint4*)planes)[i] = v0;
    ((uint4*)planes)[K / 16 + i] = v1;
    ((uint4*)planes)[2 * (K / 16) + i] = v2;
    ((uint4*)planes)[3 * (K / 16) + i] = v3;
    w |= !planes_sign_extended(v2.x, v3.x) | !planes_sign_extended(v2.y, v3.y) |
         !planes_sign_extended(v2.z, v3.z) | !planes_sign_extended(v2.w, v3.w);
  }
  return part_or<kStepConsumers>(w);
}

// The epilogue arguments of product stage k (xbase: the exchanges finished
// before this pass).
__device__ __forceinline__ ProductArgs step_product_args(const StepArgs& A, const StepStage& st, uint32_t k,
                                                         uint32_t p, uint32_t xbase) {
  ProductArgs a{};
  a.rows = st.rows;
  a.cols = st.cols;
  a.tokens = 1;
  a.kc = st.kc;
  a.nslices = st.nslices;
  a.out_stride = st.rows;
  a.split_acc = A.split_acc;
  a.split_count = A.split_count;
  a.split_groups = 0;
  if (st.kind == STEP_QKV) {
    a.out = A.q;
    a.out_stride = A.qd;
    a.freqs = A.freqs;
    a.head_dim = A.d;
    a.qd = A.qd;
    a.kvd = A.kvd;
    a.kcache = A.kcache + (size_t)st.layer * A.cap * A.kvd;
    a.vcache = A.vcache + (size_t)st.layer * A.cap * A.kvd;
    a.pos0 = p;
    a.gready = A.gready + (size_t)st.layer * (A.heads / A.hpc);
    a.gready_hpc = A.hpc;
  } else if ((st.kind == STEP_O || st.kind == STEP_DOWN) && A.tp_world > 1) {
    // this rank's input columns: unrounded partial sums for exchange xj
    a.partial = A.xpart + (size_t)((xbase + st.xj) & 1) * A.H * 4;
  } else if (st.kind == STEP_O || st.kind == STEP_DOWN) {
    a.out = A.x;
    a.resid = A.x;
    a.sumsq = step_sumsq_slot(A, k);  // for the normalised input of stage k + 1
  } else if (st.kind == STEP_GU) {
    a.out_planes = A.planes2;
  } else {  // STEP_HEAD: this rank's vocabulary rows
    a.out = A.logits;
    a.best = A.best;
    a.row_base = A.tp_rank * st.rows;
  }
  return a;
}

// Tensor parallelism: exchange xj of the pass. Every block of this rank has
// written its partial limbs (the stage before); block 0 publishes the epoch
// into every peer's flags (release, system scope: the blocks' writes are
// ordered before it through the stage counter), every block waits - bounded -
// for every peer's flag of the same epoch, then sums its rows' limbs over the
// ranks (peers' slots read over NVLink), rounds once (q8.rs:69-71), adds the
// residual and leaves the sum of squares of its rows in its slot. Slots
// alternate by epoch parity: a rank rewrites one only after every peer has
// published the next epoch, i.e. finished reading it.
__device__ __forceinline__ void step_exchange(const StepArgs& A, uint32_t k, uint32_t epoch, Acc128* warp_sq) {
  const uint32_t tid = threadIdx.x;
  if (blockIdx.x == 0 && tid < A.tp_world && tid != A.tp_rank) st_release_sys(A.xpeer_flags[tid] + A.tp_rank, epoch);
  if (tid < A.tp_world && tid != A.tp_rank && ld_acquire_sys(A.xflags + tid) < epoch) {
    const uint64_t t0 = global_ns();
    for (uint32_t i = 1;; ++i) {
      if (ld_acquire_sys(A.xflags + tid) >= epoch) break;
      if ((i & 63) == 0) {
        if (*(volatile unsigned int*)A.fault) break;
        if (global_ns() - t0 > 1000000000ull) {
          atomicOr(A.fault, 1u);
          break;
        }
      }
    }
  }
  part_sync<kStepConsumers>();
  const uint32_t r0 = (uint32_t)((uint64_t)blockIdx.x * A.H / gridDim.x);
  const uint32_t r1 = (uint32_t)((uint64_t)(blockIdx.x + 1) * A.H / gridDim.x);
  const size_t slot = (size_t)(epoch & 1) * A.H * 4;
  Acc128 sq{0, 0};
  for (uint32_t row = r0 + tid; row < r1; row += kStepConsumers) {
    Acc128 acc{0, 0};
    for (uint32_t j = 0; j < A.tp_world; ++j) {
      const int64_t* src = A.xpeer_part[j] + slot + (size_t)row * 4;
      const longlong2 a = __ldcg((const longlong2*)src), b = __ldcg((const longlong2*)(src + 2));
      acc128_add(acc, (uint64_t)a.x, 0);
      acc128_add(acc, (uint64_t)a.y << 32, (int64_t)((uint64_t)a.y >> 32));
      acc128_add(acc, 0, b.x);
      acc128_add(acc, 0, (int64_t)((uint64_t)b.y << 32));
    }
    const int32_t y = add_sat(acc128_round_q24(acc), __ldcg(A.x + row));
    A.x[row] = y;
    acc128_add(sq, (uint64_t)((int64_t)y * y), 0);
  }
  sq = warp_sum_acc128(sq);
  if ((tid & 31) == 0) warp_sq[tid >> 5] = sq;
  part_sync<kStepConsumers>();
  if (tid < 32) {
    Acc128 t = tid < kStepConsumers / 32 ? warp_sq[tid] : Acc128{0, 0};
    t = warp_sum_acc128(t);
    if (tid == 0) *step_sumsq_slot(A, k) = (t.hi || t.lo > (uint64_t)INT64_MAX) ? (uint64_t)INT64_MAX : t.lo;
  }
}

// Greedy bookkeeping of the pass (generation.rs:25-58), by the last block.
// With tensor parallelism each rank holds the first maximum of its
// vocabulary shard: it publishes it into every peer's key slot (value, then
// the epoch with release semantics), waits - bounded - for every peer's, and
// all ranks take the same global first maximum.
__device__ __forceinline__ void step_finish(const StepArgs& A, uint32_t p, uint32_t xbase) {
  unsigned long long key = __ldcg(A.best);
  if (A.tp_world > 1) {
    const uint32_t epoch = xbase + A.xchanges;
    for (uint32_t j = 0; j < A.tp_world; ++j) {
      if (j == A.tp_rank) continue;
      unsigned long long* slot = tp_key_slots(A.xpeer_part[j], A.H) + 2 * A.tp_rank;
      st_relaxed_sys(slot, key);
      st_release_sys(slot + 1, (unsigned long long)epoch);
    }
    unsigned long long* mine = tp_key_slots(A.xpart, A.H);
    for (uint32_t j = 0; j < A.tp_world; ++j) {
      if (j == A.tp_rank) continue;
      const uint64_t t0 = global_ns();
      for (uint32_t i = 1; ld_acquire_sys(mine + 2 * j + 1) < epoch; ++i) {
        if ((i & 63) == 0 && ((*(volatile unsigned int*)A.fault) || global_ns() - t0 > 1000000000ull)) {
          atomicOr(A.fault, 1u);
          break;
        }
      }
      const unsigned long long other = __ldcg(mine + 2 * j);
      key = other > key ? other : key;
    }
    *A.xepoch = epoch;
  }
  const uint32_t tok = best_key_token(key);
  *A.d_token = tok;
  *A.best = 0;
  const uint32_t step = *A.d_step;
  if (A.history && step < A.history_cap) A.history[step] = tok;
  *A.d_step = step + 1;
  *A.d_pos = p + 1;
  for (uint32_t k = 0; k < A.nstages; ++k) A.sync[k] = 0;
  for (uint32_t i = 0; i < A.layers * (A.heads / A.hpc); ++i) A.gready[i] = 0;
}

// ---- attention stage --------------------------------------------------------

template <uint32_t HPC>
struct StepAttnShared {
  unsigned long long best[HPC], sum[HPC], gbest[HPC], gtot[HPC], ginv[HPC];
  int32_t wsum[HPC], resid[HPC];
  bool last;
  Acc128 warp_sq[kStepConsumers / 32];  // the embedding stage's per-warp sums of squares
  unsigned long long wbest[kStepConsumers / 32][HPC];  // each warp's first-maximum keys
};

__device__ __forceinline__ void st_relaxed_gpu(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_gpu(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// One exchange of a head group: every block of the group has published HPC
// words (non-zero once written) into its own slots [chunk][HPC]; warp 0
// waits - bounded - until all chunks x HPC are written and combines them per
// head (the maximum, or the sum of the words minus one each), out[h].
// Slots lane, lane + 32, ... all belong to head lane % HPC (32 % HPC == 0).
template <uint32_t HPC, bool kMax>
__device__ __forceinline__ void group_gather(const unsigned long long* slots, uint32_t chunks,
                                             unsigned long long* out, unsigned int* fault) {
  const uint32_t lane = threadIdx.x & 31, n = chunks * HPC;
  const uint64_t t0 = global_ns();
  for (uint32_t it = 1;; ++it) {
    bool ready = true;
    for (uint32_t i = lane; i < n; i += 32) ready &= ld_relaxed_gpu(slots + i) != 0;
    if (__all_sync(0xffffffffu, ready)) break;
    if ((it & 15) == 0) {
      const bool give_up = *(volatile unsigned int*)fault || global_ns() - t0 > 1000000000ull;
      if (__any_sync(0xffffffffu, give_up)) {
        if (lane == 0) atomicOr(fault, 1u);
        break;
      }
    }
  }
  unsigned long long v = 0;
  for (uint32_t i = lane; i < n; i += 32) {
    const unsigned long long w = ld_relaxed_gpu(slots + i);
    v = kMax ? (w > v ? w : v) : v + (w ? w - 1 : 0);
  }
#pragma unroll
  for (uint32_t off = 16; off >= HPC; off >>= 1) {
    const unsigned long long o = __shfl_xor_sync(0xffffffffu, v, off);
    v = kMax ? (o > v ? o : v) : v + o;
  }
  if (lane < HPC) out[lane] = v;
}


// Sums M values a lane over the W-lane groups of a warp (W a power of two,
// M <= W): lane l of a group ends with the group's total of value
// l / (W / M). Halving exchange (offsets W/2, W/4, ...) while a lane holds
// more than one value, then plain sums over the remaining offsets. Wrapping
// 64-bit additions, like the atomics they feed.
template <uint32_t M, uint32_t W>
__device__ __forceinline__ uint64_t reduce_scatter_lanes(uint64_t (&v)[M], uint32_t pos) {
  static_assert(M >= 1 && M <= W && W <= 32 && (M & (M - 1)) == 0 && (W & (W - 1)) == 0, "powers of two");
#pragma unroll
  for (uint32_t n = M, off = W / 2; n > 1; n >>= 1, off >>= 1) {
    const bool upper = (pos & off) != 0;
#pragma unroll
    for (uint32_t i = 0; i < n / 2; ++i) {
      const uint64_t send = upper ? v[i] : v[i + n / 2];
      const uint64_t keep = upper ? v[i + n / 2] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
    }
  }
  uint64_t r = v[0];
#pragma unroll
  for (uint32_t off = W / M / 2; off >= 1; off >>= 1) r += __shfl_xor_sync(0xffffffffu, r, off);
  return r;
}

// Consumer warps of an attention stage: only the rows this block's head
// group reads must be written: the group's q rows (HPC heads) and its kv
// head's K and V rows at position p, (HPC + 2) D / 16 tile groups of the
// q|k|v product, each counted on gready once its rows are stored (a release
// add after the stores; the poll acquires). Earlier stages are ordered
// before through the blocks that wrote those rows (each waited for the
// stage before its own).
template <uint32_t HPC>
__device__ __forceinline__ void step_attn_wait(const StepArgs& A, uint32_t k, uint32_t layer, uint32_t p);

// This block's share of the attention of a decode pass: the head group and
// the chunk [r0, r1) of positions [0, p] (empty when r0 = p + 1); rows
// [r0, rc), rc = max(r0, min(r1, p)) (written by earlier passes) travel
// through the tile ring, row p (written by this pass's q|k|v stage) is read
// from the cache by the consumers.
struct AttnChunk {
  bool active;
  uint32_t grp, rank, h0, g, r0, r1, rc;
  unsigned int* bar;
};
template <uint32_t HPC>
__device__ __forceinline__ AttnChunk attn_chunk(const StepArgs& A, uint32_t p) {
  AttnChunk c{};
  const uint32_t groups = A.heads / HPC, chunks = A.chunks;
  c.active = blockIdx.x < groups * chunks;
  if (!c.active) return c;
  const uint32_t grp = blockIdx.x / chunks, rank = blockIdx.x % chunks;
  c.grp = grp;
  c.rank = rank;
  c.h0 = grp * HPC;
  c.g = c.h0 / (A.heads / A.kv_heads);
  const uint32_t n = p + 1, span = (n + chunks - 1) / chunks;
  c.r0 = min(n, rank * span);
  c.r1 = min(n, c.r0 + span);
  c.rc = max(c.r0, min(c.r1, p));  // an empty chunk (r0 = p + 1) copies nothing
  c.bar = A.gbar + grp;
  return c;
}

// The attention scratch of a block (the planes region during the attention
// stage): scores / weights [span][HPC] int32, exp terms [span][HPC] u64, then
// the group's query rows and row p's keys (HPC + 1 rows, kv_pitch apart).
__host__ __device__ inline uint32_t step_attn_q_offset(uint32_t span_max, uint32_t hpc) {
  return round_up(round_up(span_max * hpc * 4, 16) + span_max * hpc * 8, 16);
}

template <uint32_t HPC>
__device__ __forceinline__ void step_attn_wait(const StepArgs& A, uint32_t k, uint32_t layer, uint32_t p) {
  const AttnChunk c = attn_chunk<HPC>(A, p);
  if (threadIdx.x == 0) {
    if (c.active)
      step_poll(A.gready + (size_t)layer * (A.heads / HPC) + c.grp, (HPC + 2) * A.d / kQ8TileRows, A.fault);
    step_stamp(A, k, 0);
  }
  part_sync<kStepConsumers>();
}

// Key and value rows sit in a ring slot 4 D + 16 bytes apart: lane l of a warp
// reading row t0 + l at a fixed column then starts 4 (t0 + l) banks further
// on, so eight lanes' 16-byte pieces cover all 32 banks (no conflicts).
template <uint32_t D>
__host__ __device__ constexpr uint32_t kv_pitch() {
  return D * 4 + 16;
}

// Producer warp: the chunk's cached key rows, then its value rows, into ring
// slots (slot_bytes / pitch rows a slot, one bulk copy a row, the warp's 32
// lanes issuing a slot's copies together). Lane 0 waits for the slot and arms
// its barrier; every lane keeps the same cursor.
template <uint32_t PER, uint32_t HPC>
__device__ __forceinline__ bool step_issue_kv(const StepArgs& A, const TileRing& ring, RingCursor& pc, uint32_t layer,
                                              uint32_t p, uint64_t policy) {
  constexpr uint32_t D = PER * 8;
  const AttnChunk c = attn_chunk<HPC>(A, p);
  if (!c.active) return true;
  const uint32_t lane = threadIdx.x & 31, per_slot = ring.slot_bytes / kv_pitch<D>();
  const size_t base = (size_t)layer * A.cap * A.kvd + (size_t)c.g * D;
  for (int kv = 0; kv < 2; ++kv) {
    const int32_t* src = (kv ? A.vcache : A.kcache) + base;
    for (uint32_t a = c.r0; a < c.rc; a += per_slot) {
      const uint32_t n = min(per_slot, c.rc - a);
      uint32_t ok = 1;
      if (lane == 0) {
        ok = pc.count < ring.slots || ring_wait<true>(&ring.empty[pc.slot], pc.parity, A.fault);
        if (ok) mbar_arrive_expect_tx(&ring.full[pc.slot], n * D * 4);
      }
      if (!__shfl_sync(0xffffffffu, ok, 0)) return false;
      uint8_t* dst = ring.base + pc.slot * ring.slot_bytes;
      for (uint32_t i = lane; i < n; i += 32)
        bulk_load(dst + i * kv_pitch<D>(), src + (size_t)(a + i) * A.kvd, D * 4, &ring.full[pc.slot], policy);
      ring_advance(ring, pc);
    }
  }
  return true;
}

// attention_softmax (ops.rs:233-261) for the HPC query heads of one group
// over this block's chunk of positions; the same three exchanges as
// attn_decode_grid_kernel (first maximum, exp sums, weighted value sums, each
// through global words of the head group), with the chunk's key and value
// rows taken from ring slots in shared memory (the producer copied them
// ahead, while the q|k|v stage ran) and the scores, exp terms and weights in
// shared `scratch`.
template <uint32_t PER, uint32_t HPC>
__device__ __forceinline__ void step_attention(const StepArgs& A, uint32_t k, uint32_t layer, uint32_t p,
                                               uint8_t* scratch, StepAttnShared<HPC>& sh, const TileRing& ring,
                                               RingCursor& cc, bool& stalled) {
  constexpr uint32_t D = PER * 8, kWarps = kStepConsumers / 32;
  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const AttnChunk c = attn_chunk<HPC>(A, p);
  if (!c.active) return;
  const uint32_t h0 = c.h0, g = c.g, r0 = c.r0, cnt = c.r1 - c.r0, nsm = c.rc - c.r0;
  const bool has_p = cnt > nsm;  // row p is this chunk's last row
  constexpr uint32_t PITCH = kv_pitch<D>() / 4;  // int32 values from one row to the next
  const uint32_t per_slot = ring.slot_bytes / kv_pitch<D>();
  const size_t lay = (size_t)layer * A.cap * A.kvd;
  int32_t* sw = (int32_t*)scratch;                                           // [span][HPC] scores, then weights
  uint64_t* tm = (uint64_t*)(scratch + round_up(A.span_max * HPC * 4, 16));  // [span][HPC] exp terms
  unsigned int* bar = c.bar;

  if (tid < HPC) {
    sh.sum[tid] = 0;
    sh.wsum[tid] = 0;
  }
  // Scores: one lane a (position, head), HPC lanes a position, PPW positions
  // a warp; each lane runs its dot product over all D dimensions, reading
  // the key row (the position's HPC lanes read the same words: a broadcast)
  // and its head's query from shared memory. Query rows and row p's keys are
  // staged behind the exp terms, kv_pitch apart so that the HPC heads'
  // words fall in different banks.
  constexpr uint32_t PPW = 32 / HPC;
  static_assert(32 % HPC == 0, "whole positions a warp");
  const uint32_t my_h = lane % HPC, my_p = lane / HPC;
  int32_t* qs = (int32_t*)(scratch + step_attn_q_offset(A.span_max, HPC));  // [HPC][PITCH]
  int32_t* prow = qs + HPC * PITCH;                                          // row p's keys
  for (uint32_t o = tid * 4; o < HPC * D; o += kStepConsumers * 4)
    *(int4*)(qs + (o / D) * PITCH + o % D) = __ldcg((const int4*)(A.q + (size_t)h0 * D + o));
  if (has_p)
    for (uint32_t o = tid * 4; o < D; o += kStepConsumers * 4)
      *(int4*)(prow + o) = __ldcg((const int4*)(A.kcache + lay + (size_t)p * A.kvd + g * D + o));
  part_sync<kStepConsumers>();

  // ---- 1. scores and each head's first maximum (every lane keeps the key of
  // its head my_h)
  unsigned long long best = 0;
  const int4* q4 = (const int4*)(qs + my_h * PITCH);
  auto score_row = [&](const int32_t* krow, uint32_t t) {  // t: the row's index in the chunk
    const int4* k4 = (const int4*)krow;
    int64_t c0 = 0, c1 = 0;
#pragma unroll 8
    for (uint32_t i = 0; i < D / 4; ++i) {
      const int4 kv = k4[i], qv = q4[i];
      mac_wide(c0, qv.x, kv.x);
      mac_wide(c1, qv.y, kv.y);
      mac_wide(c0, qv.z, kv.z);
      mac_wide(c1, qv.w, kv.w);
    }
    const int32_t sc = finish_score((int64_t)((uint64_t)c0 + (uint64_t)c1), SCORE_MISTRAL, A.scale_q32);
    sw[t * HPC + my_h] = sc;
    const unsigned long long key = best_key(sc, r0 + t);
    best = key > best ? key : best;
  };
  for (uint32_t sb = 0; sb < nsm; sb += per_slot) {
    const uint32_t nrows = min(per_slot, nsm - sb);
    if (!stalled && !ring_wait<true>(&ring.full[cc.slot], cc.parity, A.fault)) stalled = true;
    if (sb == 0 && tid == 0) step_stamp(A, k, 1);
    const int32_t* ks = (const int32_t*)(ring.base + cc.slot * ring.slot_bytes);
    for (uint32_t base = 0; base < nrows; base += kWarps * PPW) {
      const uint32_t t = base + warp * PPW + my_p;
      if (t < nrows) score_row(ks + t * PITCH, sb + t);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&ring.empty[cc.slot]);  // the slot's key rows are used
    ring_advance(ring, cc);
  }
  if (has_p && warp == 0 && my_p == 0) score_row(prow, nsm);
  // the warp's keys a head (lanes my_h, my_h + HPC, ...), then the sixteen
  // warps through shared memory
#pragma unroll
  for (uint32_t off = HPC; off < 32; off <<= 1) {
    const unsigned long long o = __shfl_xor_sync(0xffffffffu, best, off);
    best = o > best ? o : best;
  }
  if (lane < HPC) sh.wbest[warp][lane] = best;
  part_sync<kStepConsumers>();
  if (tid < HPC) {
    unsigned long long b = 0;
    for (uint32_t w = 0; w < kWarps; ++w) b = sh.wbest[w][tid] > b ? sh.wbest[w][tid] : b;
    sh.best[tid] = b;
  }
  part_sync<kStepConsumers>();
  // exchange 1: the group's first maximum (an empty chunk publishes 1, below
  // every key)
  unsigned long long* kslots = A.kslots + (size_t)c.grp * A.chunks * HPC;
  if (tid < HPC) st_relaxed_gpu(kslots + c.rank * HPC + tid, sh.best[tid] ? sh.best[tid] : 1ull);
  if (tid == 0) step_stamp(A, k, 2);
  if (warp == 0) group_gather<HPC, true>(kslots, A.chunks, sh.gbest, A.fault);
  part_sync<kStepConsumers>();
  if (tid == 0) step_stamp(A, k, 3);

  // ---- 2. exp terms against the group's first maximum, their sums.
  // Element e = position * HPC + head: thread tid always meets head tid % HPC
  // (= my_h: 32 % HPC == 0).
  {
    const int32_t mx = best_key_value(sh.gbest[my_h]);
    uint64_t e = 0;
    for (uint32_t el = tid; el < cnt * HPC; el += kStepConsumers) {
      // softmax_exp_term_act(sw[el], mx) from the table (filled by that function)
      const int32_t dist = sub_sat(sw[el], mx);  // <= 0: mx is the maximum
      const uint32_t back = (uint32_t)(-(int64_t)dist);
      const uint64_t term = dist >= 0 ? (uint64_t)1 << 32 : back < kExpTerms ? (uint64_t)__ldg(A.exp_terms + back) : 0;
      tm[el] = term;
      e += term;
    }
    e = head_lane_sum<HPC>(e);
    if (lane < HPC && e) atomicAdd(&sh.sum[lane], (unsigned long long)e);
  }
  part_sync<kStepConsumers>();
  // exchange 2: the sums of exp terms (each published plus one: non-zero)
  unsigned long long* sslots = A.sslots + (size_t)c.grp * A.chunks * HPC;
  if (tid < HPC) st_relaxed_gpu(sslots + c.rank * HPC + tid, sh.sum[tid] + 1);
  if (warp == 0) group_gather<HPC, false>(sslots, A.chunks, sh.gtot, A.fault);
  part_sync<kStepConsumers>();
  if (tid == 0) step_stamp(A, k, 4);
  if (tid < HPC) {
    const unsigned long long tot = sh.gtot[tid];
    sh.ginv[tid] = tot ? UINT64_MAX / tot : 0;  // tot >= 2^32 after a complete exchange
  }
  part_sync<kStepConsumers>();

  // ---- 3. weights and their sums, then the value sums
  {
    const uint64_t tot = sh.gtot[my_h], inv = sh.ginv[my_h];
    int32_t wsum = 0;
    for (uint32_t el = tid; el < cnt * HPC; el += kStepConsumers) {
      const int32_t w = tot ? softmax_weight_inv((int64_t)tm[el], tot, inv) : 0;
      sw[el] = w;
      wsum += w;
    }
    wsum = head_lane_sum<HPC>(wsum);
    if (lane < HPC && wsum) atomicAdd(&sh.wsum[lane], wsum);
  }
  part_sync<kStepConsumers>();
  if (tid < HPC && sh.wsum[tid]) atomicAdd(A.wsum + h0 + tid, sh.wsum[tid]);
  // Value sums: warp w takes dimensions [w DW, (w + 1) DW) of every row. Its
  // HPC DW sums are split into VG groups of at most 16 (lane l takes group
  // l / (32 / VG)) and the rows over the 32 / VG lanes of a group; the lanes'
  // sums then meet in a halving exchange within the group and the lanes
  // holding a total add it into the head group's words.
  constexpr uint32_t DW = D / kWarps, NV_ALL = HPC * DW, VG = NV_ALL > 16 ? NV_ALL / 16 : 1;
  constexpr uint32_t MV = NV_ALL / VG, W = 32 / VG;  // sums a lane, lanes a group
  static_assert(DW >= 1 && MV <= W && NV_ALL % VG == 0, "value sums a lane");
  const uint32_t vg = lane / W, pos = lane % W;
  uint64_t acc[MV];
#pragma unroll
  for (uint32_t i = 0; i < MV; ++i) acc[i] = 0;
  auto add_row = [&](const int32_t* vrow, uint32_t t, bool global) {  // vrow: the row's DW values
    int32_t v[DW];
    if constexpr (DW % 4 == 0) {
#pragma unroll
      for (uint32_t i = 0; i < DW / 4; ++i) {
        const int4 x = global ? __ldcg((const int4*)vrow + i) : *((const int4*)vrow + i);
        v[4 * i] = x.x, v[4 * i + 1] = x.y, v[4 * i + 2] = x.z, v[4 * i + 3] = x.w;
      }
    } else if constexpr (DW == 2) {
      const int2 x = global ? __ldcg((const int2*)vrow) : *(const int2*)vrow;
      v[0] = x.x, v[1 % DW] = x.y;
    } else {
      v[0] = global ? __ldcg(vrow) : *vrow;
    }
#pragma unroll
    for (uint32_t j = 0; j < MV; ++j) {
      const uint32_t val = vg * MV + j, h = val / DW, i = val % DW;
      acc[j] += (uint64_t)((int64_t)sw[t * HPC + h] * (int64_t)v[i]);
    }
  };
  for (uint32_t sb = 0; sb < nsm; sb += per_slot) {
    const uint32_t nrows = min(per_slot, nsm - sb);
    if (!stalled && !ring_wait<true>(&ring.full[cc.slot], cc.parity, A.fault)) stalled = true;
    const int32_t* vs = (const int32_t*)(ring.base + cc.slot * ring.slot_bytes);
    for (uint32_t t = pos; t < nrows; t += W) add_row(vs + t * PITCH + warp * DW, sb + t, false);
    __syncwarp();
    if (lane == 0) mbar_arrive(&ring.empty[cc.slot]);  // the slot's value rows are used
    ring_advance(ring, cc);
  }
  if (has_p && pos == 0) add_row(A.vcache + lay + (size_t)p * A.kvd + g * D + warp * DW, nsm, true);
  const uint64_t tot = reduce_scatter_lanes<MV, W>(acc, pos);
  constexpr uint32_t kLanesPer = W / MV;
  if (pos % kLanesPer == 0 && tot) {
    const uint32_t val = vg * MV + pos / kLanesPer, h = val / DW, i = val % DW;
    atomicAdd((unsigned long long*)(A.acc + (size_t)(h0 + h) * D + warp * DW + i), (unsigned long long)tot);
  }
  if (tid == 0) step_stamp(A, k, 5);

  // ---- 4. the group's last block finishes every output of the group and
  // clears the exchange words for the next layer
  part_sync<kStepConsumers>();
  if (tid == 0) {
    __threadfence();
    sh.last = atom_add_acq_rel(bar, 1u) == A.chunks - 1;
  }
  part_sync<kStepConsumers>();
  if (!sh.last) return;
  if (tid < HPC) sh.resid[tid] = sub_sat(kOneAct, (int32_t)__ldcg((const int*)(A.wsum + h0 + tid)));  // ops.rs:274-276
  part_sync<kStepConsumers>();
  for (uint32_t o = tid; o < HPC * D; o += kStepConsumers) {
    const uint32_t h = o / D, i = o % D, hh = h0 + h;
    unsigned long long* accp = (unsigned long long*)(A.acc + (size_t)hh * D + i);
    uint64_t s = (uint64_t)__ldcg(accp);
    *accp = 0;
    const uint32_t tmax = best_key_token(sh.gbest[h]);
    s += (uint64_t)((int64_t)sh.resid[h] * __ldcg(A.vcache + lay + (size_t)tmax * A.kvd + g * D + i));
    put_planes(A.planes, A.qd, hh * D + i, requantize((int64_t)s));
  }
  if (tid < HPC) A.wsum[h0 + tid] = 0;
  for (uint32_t i = tid; i < A.chunks * HPC; i += kStepConsumers) {  // every block has read them
    kslots[i] = 0;
    sslots[i] = 0;
  }
  if (tid == 0) bar[0] = 0;
}

// ---- the kernel --------------------------------------------------------------

// kUniform: every product stage's matrix has one scale a row (StepStage::
// uniform), so the consumers run only the once-a-group scaling loop; the
// general instantiation runs only the per-block one (one loop a kernel keeps
// the register allocation of each to its own loop).
template <uint32_t PER, uint32_t HPC, bool kUniform>
__global__ void __launch_bounds__(kTmaThreads, 1) decode_step_kernel(const StepArgs A) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t full[kTmaMaxStages];
  __shared__ __align__(8) uint64_t empty[kTmaMaxStages];
  __shared__ __align__(8) uint64_t slot_full[kTmaSlots];
  __shared__ __align__(8) uint64_t slot_empty[kTmaSlots];
  __shared__ int32_t s_scale;
  __shared__ Acc128 slot_sums[kTmaSlots][2][kQ8TileRows];
  __shared__ StepAttnShared<HPC> ash;
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nb = gridDim.x;
  uint8_t* planes = smem;  // activation planes of a product, or the attention scratch
  const TileRing ring{smem + A.planes_bytes, A.slot_bytes, A.ring_slots, full, empty};
  const SumRing sums{slot_full, slot_empty, slot_sums};
  const StepStage* __restrict__ stages = A.stages;

  if (threadIdx.x == 0) {
    for (uint32_t st = 0; st < A.ring_slots; ++st) {
      mbar_init(&full[st], 1);
      mbar_init(&empty[st], kTmaConsumerWarps);
    }
    for (uint32_t sl = 0; sl < kTmaSlots; ++sl) {
      mbar_init(&slot_full[sl], kTmaConsumerWarps);
      mbar_init(&slot_empty[sl], 1);
    }
    mbar_fence_init();
  }
  __syncthreads();
  const uint32_t p = *A.d_pos;  // this token's position (advanced by the previous launch)
  const uint32_t xbase = A.tp_world > 1 ? *A.xepoch : 0;  // exchanges before this pass

  if (warp == kStepProducerWarp) {
    // lane 0 issues the weight tiles; the whole warp issues attention rows
    RingCursor pc{0, 1, 0};
    const uint64_t policy = l2_evict_first_policy();
    bool ok = true;
    for (uint32_t k = 0; k < A.nstages && ok; ++k) {
      const StepStage st = stages[k];
      if (st.kind == STEP_ATTN) {
        ok = step_issue_kv<PER, HPC>(A, ring, pc, st.layer, p, policy);
        if (lane == 0) step_stamp(A, k, 6);
      }
      if (!step_is_product(st.kind)) continue;
      uint32_t ib, ie;
      step_range(st, blockIdx.x, nb, &ib, &ie);
      uint32_t good = 1;
      if (lane == 0) {
        good = ring_issue<true>(ring, pc, st.q, st.s, st.kc, ib, ie, policy, A.fault);
        step_stamp(A, k, 6);
      }
      ok = __shfl_sync(0xffffffffu, good, 0) != 0;
      // the other lanes keep the cursor in step with lane 0's
      if (lane != 0)
        for (uint32_t t = ib; t < ie; ++t) ring_advance(ring, pc);
    }
    if (lane == 0) ring_drain(ring, pc, A.fault);  // no copy may land after the block exits
    return;
  }

  if (warp == kStepEpilogueWarp) {
    uint32_t j = 0;
    for (uint32_t k = 0; k < A.nstages; ++k) {
      const StepStage st = stages[k];
      if (!step_is_product(st.kind)) continue;
      uint32_t ib, ie;
      step_range(st, blockIdx.x, nb, &ib, &ie);
      const ProductArgs a = step_product_args(A, st, k, p, xbase);
      if (st.kind == STEP_QKV) ring_epilogue<EPI_QKV_ROPE, true>(a, sums, j, ib, ie, st.nslices, A.fault);
      else if (st.kind == STEP_GU) ring_epilogue<EPI_SILU_MUL, true>(a, sums, j, ib, ie, st.nslices, A.fault);
      else if (st.kind == STEP_HEAD) ring_epilogue<EPI_LOGITS, true>(a, sums, j, ib, ie, st.nslices, A.fault);
      else if (A.tp_world > 1) ring_epilogue<EPI_PARTIAL, true>(a, sums, j, ib, ie, st.nslices, A.fault);
      else ring_epilogue<EPI_RESID, true>(a, sums, j, ib, ie, st.nslices, A.fault);
      __syncwarp();
      if (lane == 0) {
        step_stamp(A, k, 7);
        __threadfence();
        if (k + 1 < A.nstages) red_add_release(A.sync + k, 1u);
        else if (atom_add_acq_rel(A.sync + k, 1u) == nb - 1) step_finish(A, p, xbase);  // the head stage, last of all
      }
    }
    return;
  }

  // consumer warps
  RingCursor cc{0, 0, 0};
  uint32_t j = 0;
  bool stalled = false;
  for (uint32_t k = 0; k < A.nstages; ++k) {
    const StepStage st = stages[k];
    if (st.kind == STEP_EMBED) {
      step_embed(A, ash.warp_sq);
      step_consumers_arrive(A, k);
      continue;
    }
    if (st.kind == STEP_ATTN) {
      step_attn_wait<HPC>(A, k, st.layer, p);
      step_attention<PER, HPC>(A, k, st.layer, p, planes, ash, ring, cc, stalled);
      step_consumers_arrive(A, k);
      continue;
    }
    if (st.kind == STEP_XCHG) {
      step_wait(A, k);
      step_exchange(A, k, xbase + st.xj, ash.warp_sq);
      step_consumers_arrive(A, k);
      continue;
    }
    uint32_t ib, ie;
    step_range(st, blockIdx.x, nb, &ib, &ie);
    if (ib == ie) continue;
    constexpr uint32_t kHeld = 2;  // int4 pieces of x a thread holds (K up to 4096 values)
    int4 wv[kHeld];
    if (st.norm_w) {  // the norm weights never change: load them before the wait
#pragma unroll
      for (uint32_t jj = 0; jj < kHeld; ++jj) {
        const uint32_t i = threadIdx.x * 4 + jj * kStepConsumers * 4;
        wv[jj] = i < st.cols ? __ldg((const int4*)(st.norm_w + i)) : make_int4(0, 0, 0, 0);
      }
    }
    step_wait(A, k);
    const uint8_t* src = st.kind == STEP_O ? A.planes : A.planes2;
    const bool wide = st.norm_w ? step_norm_planes<kHeld>(A, k, st.cols, wv, st.norm_w, planes, &s_scale)
                                : step_copy_planes(src, st.cols, planes);
    if (threadIdx.x == 0) step_stamp(A, k, 1);
    ring_consume_impl<true, kUniform>(ring, cc, sums, j, planes, wide, st.cols, st.kc, st.nslices, st.e_fast, ib,
                                      ie, stalled, A.fault);
    if (threadIdx.x == 0) step_stamp(A, k, 2);
  }
}

#define IRIS_STEP_SHAPES(X) X(4, 1) X(4, 2) X(4, 4) X(8, 2) X(8, 4) X(16, 1) X(16, 2) X(16, 4)

template <uint32_t PER, uint32_t HPC>
const void* step_kernel_ptr(bool uniform) {
  return uniform ? (const void*)decode_step_kernel<PER, HPC, true> : (const void*)decode_step_kernel<PER, HPC, false>;
}

const void* step_kernel_for(uint32_t per, uint32_t hpc, bool uniform) {
#define IRIS_STEP_PICK(PER, HPC) \
  if (per == PER && hpc == HPC) return step_kernel_ptr<PER, HPC>(uniform);
  IRIS_STEP_SHAPES(IRIS_STEP_PICK)
#undef IRIS_STEP_PICK
  return nullptr;
}

}  // namespace

StepPlan plan_decode_step(uint32_t H, uint32_t F, uint32_t heads, uint32_t kv_heads, uint32_t d, uint32_t V,
                          uint32_t cap, const uint32_t* kcs, uint32_t nkcs) {
  StepPlan p{};
  p.why = 1;
  if (heads == 0 || kv_heads == 0 || heads % kv_heads || d % 8 || cap == 0) return p;
  const uint32_t G = heads / kv_heads;
  uint32_t hpc = 4;
  while (hpc > 1 && (G % hpc || hpc * d > 512)) hpc >>= 1;
  p.why = 2;
  const void* fns[2] = {step_kernel_for(d / 8, hpc, false), step_kernel_for(d / 8, hpc, true)};
  if (!fns[0] || !fns[1]) return p;
  p.why = 3;
  int dev = 0, sms = 0, coop = 0, optin = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess || !coop ||
      sms <= 0) {
    cudaGetLastError();
    return p;
  }
  size_t static_smem = 0;  // the larger of the two instantiations'
  for (const void* fn : fns) {
    cudaFuncAttributes fa{};
    if (cudaFuncGetAttributes(&fa, fn) != cudaSuccess) {
      cudaGetLastError();
      return p;
    }
    static_smem = std::max(static_smem, fa.sharedSizeBytes);
  }
  p.why = 1;
  const uint32_t groups = heads / hpc, chunks = (uint32_t)sms / groups;
  if (chunks == 0) return p;
  p.why = 4;
  const uint32_t span_max = (cap + chunks - 1) / chunks;
  uint32_t slot = 0;
  for (uint32_t i = 0; i < nkcs; ++i) slot = std::max(slot, round_up(kQ8TileRows * kcs[i] + kcs[i], 128));
  // The planes region holds the widest input's byte planes and the attention
  // scratch (scores, then weights, and exp terms); the rest of the shared
  // memory is ring slots.
  const uint32_t widest = std::max(std::max(H, heads * d), F);
  const uint32_t attn = step_attn_q_offset(span_max, hpc) + (hpc + 1) * (d * 4 + 16);
  const uint32_t planes = round_up(std::max(4 * widest, attn), 128);
  if ((size_t)optin <= static_smem) return p;
  const uint32_t dyn = (uint32_t)optin - (uint32_t)static_smem;
  if (planes + 2 * slot > dyn) return p;
  const uint32_t slots = std::min<uint32_t>(kTmaMaxStages, (dyn - planes) / slot);
  const uint32_t smem = planes + slots * slot;
  for (const void* fn : fns) {
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) {
      cudaGetLastError();
      return p;
    }
  }
  p.why = 5;
  for (const void* fn : fns) {
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kTmaThreads, smem) != cudaSuccess || per_sm < 1) {
      cudaGetLastError();
      return p;
    }
  }
  p.blocks = (uint32_t)sms;
  p.ring_slots = slots;
  p.slot_bytes = slot;
  p.planes_bytes = planes;
  p.smem = smem;
  p.chunks = chunks;
  p.span_max = span_max;
  p.hpc = hpc;
  (void)V;
  p.why = 0;
  p.ok = true;
  return p;
}

cudaError_t launch_decode_step(const StepArgs& a, const StepPlan& p, bool uniform, cudaStream_t s) {
  const void* fn = step_kernel_for(a.d / 8, p.hpc, uniform);
  if (!fn || !p.ok) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(p.blocks);
  cfg.blockDim = dim3(kTmaThreads);
  cfg.dynamicSmemBytes = p.smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  void* args[] = {(void*)&a};
  return cudaLaunchKernelExC(&cfg, fn, args);
}

cudaError_t prepare_step_kernels() { return cudaSuccess; }

namespace {

// The two bounded waits the kernels use, alone in one block: thread 0 waits
// for an mbarrier phase (kind 0, as the TMA rings and the tensor-core
// pipelines do) or polls a global arrival counter (kind 1, as the persistent
// step's stage barriers do); thread 32 arrives or adds first unless `release`
// is 0, in which case nothing ever does and the wait runs out after about a
// second, records the give-up in the fault word and the kernel returns.
// Nothing asynchronous is in flight, so the block ends cleanly either way.
__global__ void wait_probe_kernel(int kind, int release, unsigned int* ctr, unsigned int* fault) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    mbar_fence_init();
  }
  __syncthreads();
  if (threadIdx.x == 32 && release) {
    if (kind == 0) mbar_arrive(&bar);
    else red_add_release(ctr, 1u);
  }
  if (threadIdx.x == 0) {
    if (kind == 0) mbar_wait_bounded(&bar, 0, fault);
    else step_poll(ctr, 1u, fault);
  }
  __syncthreads();
}

}  // namespace

}  // namespace iris

extern "C" int iris_wait_probe(int kind, int release) {
  using namespace iris;
  if (kind != 0 && kind != 1) return IRIS_EINVAL;
  uint32_t stale = 0;
  cudaError_t e = take_device_fault(&stale);  // start from a clear fault word
  unsigned int* fault = device_fault_word();
  if (e == cudaSuccess && !fault) e = cudaErrorInvalidDevice;
  unsigned int* ctr = nullptr;
  if (e == cudaSuccess) e = cudaMalloc((void**)&ctr, sizeof(unsigned int));
  if (e == cudaSuccess) e = cudaMemset(ctr, 0, sizeof(unsigned int));
  if (e == cudaSuccess) {
    wait_probe_kernel<<<1, 64>>>(kind, release, ctr, fault);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (ctr) cudaFree(ctr);
  uint32_t gave_up = 0;
  if (e == cudaSuccess) e = take_device_fault(&gave_up);
  if (e != cudaSuccess) return (int)e;
  return gave_up ? IRIS_ESTALL : 0;
}
