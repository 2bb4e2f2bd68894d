// Row-level kernels of the mistral-dense and gemma-dense layers.
//
// Attention reproduces attention_softmax (crates/det-num/src/ops.rs:233-261)
// exactly while splitting the positions over many blocks:
//   1. scores (mistral.rs:130-145 scaled, or tensor.rs:522-528 dot_bits),
//      and each chunk's first maximum (value, then lowest position);
//   2. e^(score - max) terms against the global first maximum and their
//      chunk sums (exact: every term is at most 2^32, so the i64 sum of fewer
//      than 2^31 terms cannot saturate);
//   3. weights requantize((term << 32) / sum) (ties to even), the chunk's
//      weighted value sums and weight sums added atomically into per-head
//      totals (wrapping i64, order-free); the last block adds the residual
//      1.0 - sum(weights) times the first maximum's value row (the same as
//      adding it to that weight first, since no weight saturates) and
//      requantizes.
#include <algorithm>
#include <cooperative_groups.h>
#include <cuda_runtime.h>

#include "layers.cuh"

namespace iris {


__device__ __forceinline__ int64_t ldcg_i64(const int64_t* p) { return (int64_t)__ldcg((const long long*)p); }

// The decode query's position: from device memory inside the captured decode
// pass, else the host-given position (a single-row chain range).
__device__ __forceinline__ uint32_t query_position(const AttnArgs& a) {
  return a.pos_ptr ? *a.pos_ptr : a.pos0;
}

// ---------------------------------------------------------------------------
// Decode attention
// ---------------------------------------------------------------------------
//
// Grid (heads / hpc, position chunks of kAttnChunk), 256 threads. A block
// owns hpc query heads of one kv group and 64 consecutive positions of the
// window [ws, p]. Scores: each warp takes its 8 positions four at a time, 8
// lanes a position, each lane d/8 contiguous dimensions of the key row
// (coalesced), reduced over the 8 lanes with shuffles.

constexpr int kAttnThreads = 256;
constexpr uint32_t kAttnChunk = 64;
constexpr int kMaxHpc = 4;  // query heads a block

template <uint32_t PER, uint32_t HPC>
__device__ __forceinline__ void attn_scores_body(const AttnArgs& a, uint32_t p, uint32_t t0, uint32_t h0, uint32_t g,
                                                 unsigned long long* best_s) {
  const uint32_t d = a.d, warp = threadIdx.x >> 5, lane = threadIdx.x & 31, quad = lane >> 3, ql = lane & 7;
  const uint32_t i0 = ql * PER;  // this lane's dimensions
  int32_t q[HPC][PER];
#pragma unroll
  for (uint32_t h = 0; h < HPC; ++h)
#pragma unroll
    for (uint32_t i = 0; i < PER; i += 4) {
      const int4 v = *(const int4*)(a.q + (size_t)(h0 + h) * d + i0 + i);
      q[h][i] = v.x;
      q[h][i + 1] = v.y;
      q[h][i + 2] = v.z;
      q[h][i + 3] = v.w;
    }
  // both rounds' key segments first: eight positions a warp, four at a time
  int4 k[2][PER / 4];
  uint32_t t[2];
#pragma unroll
  for (uint32_t r = 0; r < 2; ++r) {
    t[r] = t0 + warp * 8 + r * 4 + quad;
    const int32_t* krow = a.kcache + (size_t)(t[r] <= p ? t[r] : t0) * a.kvd + g * d + i0;
#pragma unroll
    for (uint32_t i = 0; i < PER / 4; ++i) k[r][i] = *(const int4*)(krow + 4 * i);
  }
#pragma unroll
  for (uint32_t r = 0; r < 2; ++r) {
#pragma unroll
    for (uint32_t h = 0; h < HPC; ++h) {
      uint64_t sum = 0;
#pragma unroll
      for (uint32_t i = 0; i < PER / 4; ++i) {
        sum += (uint64_t)((int64_t)q[h][4 * i] * k[r][i].x) + (uint64_t)((int64_t)q[h][4 * i + 1] * k[r][i].y) +
               (uint64_t)((int64_t)q[h][4 * i + 2] * k[r][i].z) + (uint64_t)((int64_t)q[h][4 * i + 3] * k[r][i].w);
      }
      sum += __shfl_xor_sync(0xffffffffu, sum, 4);
      sum += __shfl_xor_sync(0xffffffffu, sum, 2);
      sum += __shfl_xor_sync(0xffffffffu, sum, 1);
      if (ql == 0 && t[r] <= p) {
        const int32_t sc = finish_score((int64_t)sum, a.mode, a.scale_q32);
        a.scores[(size_t)(h0 + h) * a.cap + t[r]] = sc;
        atomicMax(&best_s[h], best_key(sc, t[r]));
      }
    }
  }
}

template <uint32_t PER, uint32_t HPC>
__global__ void __launch_bounds__(kAttnThreads) attn_scores_kernel(AttnArgs a) {
  pdl_wait();
  pdl_trigger();
  __shared__ unsigned long long best_s[kMaxHpc];
  const uint32_t p = query_position(a), ws = window_start(p, a.window);
  const uint32_t G = a.heads / a.kv_heads, h0 = blockIdx.x * HPC, g = h0 / G;
  const uint32_t c = blockIdx.y, t0 = ws + c * kAttnChunk;
  if (t0 > p) return;
  if (threadIdx.x < HPC) best_s[threadIdx.x] = 0;
  __syncthreads();
  attn_scores_body<PER, HPC>(a, p, t0, h0, g, best_s);
  __syncthreads();
  if (threadIdx.x < HPC) a.chunk_best[(size_t)(h0 + threadIdx.x) * a.nchunks + c] = best_s[threadIdx.x];
}

cudaError_t launch_attn_scores(const AttnArgs& a, dim3 grid, cudaStream_t s) {
  const uint32_t per = a.d / 8;
#define IRIS_SCORES(PER, HPC)                                               \
  if (per == PER && a.hpc == HPC) {                                         \
    cudaError_t e_ = launch_k(attn_scores_kernel<PER, HPC>, grid, dim3(kAttnThreads), 0, s, a); \
    if (e_ != cudaSuccess) return e_;          \
    return cudaGetLastError();                                              \
  }
  IRIS_SCORES(4, 1) IRIS_SCORES(4, 2) IRIS_SCORES(4, 4)
  IRIS_SCORES(8, 1) IRIS_SCORES(8, 2) IRIS_SCORES(8, 4)
  IRIS_SCORES(16, 1) IRIS_SCORES(16, 2) IRIS_SCORES(16, 4)
  IRIS_SCORES(32, 1) IRIS_SCORES(32, 2)
#undef IRIS_SCORES
  return cudaErrorInvalidValue;
}

// First maximum of each of the block's heads over the active chunks.
__device__ void block_global_best(const AttnArgs& a, uint32_t h0, uint32_t nact, unsigned long long* best_s) {
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp < a.hpc) {
    const unsigned long long* cb = a.chunk_best + (size_t)(h0 + warp) * a.nchunks;
    unsigned long long b = 0;
    for (uint32_t k = lane; k < nact; k += 32) b = cb[k] > b ? cb[k] : b;
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
      unsigned long long o = __shfl_xor_sync(0xffffffffu, b, off);
      b = o > b ? o : b;
    }
    if (lane == 0) best_s[warp] = b;
  }
}

__global__ void __launch_bounds__(kAttnThreads) attn_exp_kernel(AttnArgs a) {
  pdl_wait();
  pdl_trigger();
  __shared__ unsigned long long best_s[kMaxHpc];
  __shared__ unsigned long long sum_s[kMaxHpc];
  const uint32_t p = query_position(a), ws = window_start(p, a.window);
  const uint32_t n = p - ws + 1, nact = (n + kAttnChunk - 1) / kAttnChunk;
  const uint32_t h0 = blockIdx.x * a.hpc, c = blockIdx.y;
  if (c >= nact) return;
  block_global_best(a, h0, nact, best_s);
  if (threadIdx.x < a.hpc) sum_s[threadIdx.x] = 0;
  __syncthreads();
  const uint32_t hl = threadIdx.x / kAttnChunk, t = ws + c * kAttnChunk + threadIdx.x % kAttnChunk;
  uint64_t e = 0;
  if (hl < a.hpc && t <= p) {
    const size_t at = (size_t)(h0 + hl) * a.cap + t;
    e = (uint64_t)softmax_exp_term_act(a.scores[at], best_key_value(best_s[hl]));
    a.terms[at] = (int64_t)e;
  }
  // 64 consecutive threads share a head: two warps, one shuffle sum each
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) e += __shfl_xor_sync(0xffffffffu, e, off);
  if ((threadIdx.x & 31) == 0 && hl < a.hpc) atomicAdd(&sum_s[hl], e);
  __syncthreads();
  if (threadIdx.x < a.hpc) a.chunk_sum[(size_t)(h0 + threadIdx.x) * a.nchunks + c] = sum_s[threadIdx.x];
}

__global__ void __launch_bounds__(kAttnThreads) attn_out_kernel(AttnArgs a) {
  pdl_wait();
  pdl_trigger();
  __shared__ int32_t w_s[kMaxHpc * kAttnChunk];
  __shared__ unsigned long long best_s[kMaxHpc];
  __shared__ unsigned long long total_s[kMaxHpc];
  __shared__ int32_t wsum_s[kMaxHpc];
  __shared__ bool last_s;
  const uint32_t p = query_position(a), ws = window_start(p, a.window);
  const uint32_t n = p - ws + 1, nact = (n + kAttnChunk - 1) / kAttnChunk;
  const uint32_t hpc = a.hpc, G = a.heads / a.kv_heads, h0 = blockIdx.x * hpc, g = h0 / G, d = a.d;
  const uint32_t c = blockIdx.y, t0 = ws + c * kAttnChunk;
  if (c < nact) {
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (warp < hpc) {
      const uint64_t* cs = a.chunk_sum + (size_t)(h0 + warp) * a.nchunks;
      uint64_t tot = 0;
      for (uint32_t k = lane; k < nact; k += 32) tot += cs[k];
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, off);
      if (lane == 0) {
        total_s[warp] = tot;
        wsum_s[warp] = 0;
      }
    }
    __syncthreads();
    const uint32_t hl = threadIdx.x / kAttnChunk, lp = threadIdx.x % kAttnChunk, t = t0 + lp;
    if (hl < hpc) {
      int32_t w = 0;
      if (t <= p) w = softmax_weight(a.terms[(size_t)(h0 + hl) * a.cap + t], total_s[hl]);
      w_s[hl * kAttnChunk + lp] = w;
      int32_t ws_w = w;
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) ws_w += __shfl_xor_sync(0xffffffffu, ws_w, off);
      if (lane == 0) atomicAdd(&wsum_s[hl], ws_w);
    }
    __syncthreads();
    // This chunk's weighted value sums go straight into the head's running
    // total: wrapping 64-bit addition is exact in any order.
    // Thread: one dimension i for every head of the block, over the chunk's
    // positions j = pg, pg + npg, ... (each value row element read once).
    const uint32_t live = min(kAttnChunk, p + 1 - t0);
    const uint32_t npg = blockDim.x / d, pg = threadIdx.x / d, i = threadIdx.x % d;
    if (pg < npg) {
      const int32_t* vcol = a.vcache + (size_t)t0 * a.kvd + g * d + i;
      uint64_t acc[kMaxHpc] = {0, 0, 0, 0};
#pragma unroll 8
      for (uint32_t j = pg; j < live; j += npg) {
        const int64_t v = vcol[(size_t)j * a.kvd];
#pragma unroll
        for (uint32_t h = 0; h < kMaxHpc; ++h)
          if (h < hpc) acc[h] += (uint64_t)((int64_t)w_s[h * kAttnChunk + j] * v);
      }
#pragma unroll
      for (uint32_t h = 0; h < kMaxHpc; ++h)
        if (h < hpc) atomicAdd((unsigned long long*)(a.acc + (size_t)(h0 + h) * d + i), (unsigned long long)acc[h]);
    }
    if (threadIdx.x < hpc) atomicAdd(a.wsum + h0 + threadIdx.x, wsum_s[threadIdx.x]);
  }
  // The last block of this head block finishes the heads and clears the totals.
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) last_s = atomicAdd(&a.counters[blockIdx.x], 1u) == gridDim.y - 1;
  __syncthreads();
  if (!last_s) return;
  __threadfence();
  block_global_best(a, h0, nact, best_s);
  if (threadIdx.x < hpc)  // residual 1.0 - sum of weights (ops.rs:274-276)
    wsum_s[threadIdx.x] = sub_sat(kOneAct, (int32_t)atomicExch((unsigned int*)(a.wsum + h0 + threadIdx.x), 0u));
  __syncthreads();
  const uint32_t qd = a.heads * d;
  for (uint32_t o = threadIdx.x; o < hpc * d; o += blockDim.x) {
    const uint32_t h = o / d, i = o % d, hh = h0 + h;
    int64_t acc = (int64_t)atomicExch((unsigned long long*)(a.acc + (size_t)hh * d + i), 0ull);
    const uint32_t tmax = best_key_token(best_s[h]);
    acc = (int64_t)((uint64_t)acc + (uint64_t)((int64_t)wsum_s[h] * a.vcache[(size_t)tmax * a.kvd + g * d + i]));
    const int32_t v = requantize(acc);
    put_planes(a.ctx_planes, qd, hh * d + i, v);
    if (a.ctx) a.ctx[hh * d + i] = v;
  }
  if (threadIdx.x == 0) a.counters[blockIdx.x] = 0;
}

uint32_t attention_hpc(uint32_t heads, uint32_t kv_heads) {
  uint32_t G = heads / kv_heads, hpc = G < (uint32_t)kMaxHpc ? G : (uint32_t)kMaxHpc;
  while (hpc > 1 && (G % hpc || heads / hpc < 8)) --hpc;
  return hpc;
}

uint32_t attention_chunks(uint32_t cap) { return (cap + kAttnChunk - 1) / kAttnChunk; }

// ---------------------------------------------------------------------------
// Decode attention in one launch: a thread-block cluster a head block
// ---------------------------------------------------------------------------
//
// A cluster of C blocks (16 where the device allows it, else 8) owns HPC
// query heads of one kv group; block rank r takes the r-th of C contiguous
// ranges of the window [ws, p]. The block's key rows and then its value rows
// stream as one sequence of 32-position tiles through a ring of shared-memory
// buffers with cp.async: all of them are in flight from the start when the
// ring holds them, and the HPC query heads share every key and value read.
// The three dependent steps of attention_softmax (ops.rs:233-261) meet
// through distributed shared memory:
//   1. scores of the block's positions and the block's first maximum a head;
//      cluster barrier; every block takes the maximum over the cluster;
//   2. exp terms against it (kept) and their sum a head; cluster barrier;
//      every block takes the total over the cluster;
//   3. weights (one reciprocal a head, softmax_weight_inv), their sum a head,
//      and the wrapping weighted value sums of the block's positions;
//      cluster barrier; block r finishes its share of the head dimensions:
//      the sum over the cluster plus (1.0 - sum of weights) times the first
//      maximum's value row (ops.rs:274-276), requantized into the context
//      planes.
// Every block passes every cluster barrier, also one with no positions.

constexpr uint32_t kCThreads = 512;   // 16 warps
constexpr uint32_t kTileP = 32;       // positions a tile (= 8 warps x 4 positions)
constexpr uint32_t kMaxRing = 12;     // tile buffers at most
constexpr size_t kClusterSmemMax = 200 * 1024;

// Waits until at most n of this thread's committed groups are pending.
__device__ __forceinline__ void cp_async_wait_pending(uint32_t n) {
  switch (n) {
    case 0: asm volatile("cp.async.wait_group 0;" ::: "memory"); break;
    case 1: asm volatile("cp.async.wait_group 1;" ::: "memory"); break;
    case 2: asm volatile("cp.async.wait_group 2;" ::: "memory"); break;
    case 3: asm volatile("cp.async.wait_group 3;" ::: "memory"); break;
    case 4: asm volatile("cp.async.wait_group 4;" ::: "memory"); break;
    case 5: asm volatile("cp.async.wait_group 5;" ::: "memory"); break;
    case 6: asm volatile("cp.async.wait_group 6;" ::: "memory"); break;
    case 7: asm volatile("cp.async.wait_group 7;" ::: "memory"); break;
    case 8: asm volatile("cp.async.wait_group 8;" ::: "memory"); break;
    case 9: asm volatile("cp.async.wait_group 9;" ::: "memory"); break;
    case 10: asm volatile("cp.async.wait_group 10;" ::: "memory"); break;
    default: asm volatile("cp.async.wait_group 11;" ::: "memory"); break;
  }
}

// The 16-byte pieces this thread copies of every [kTileP][D] tile: piece c =
// tid + j kCThreads is row c / (D/4), column piece c % (D/4). Offsets are
// fixed for the kernel; a tile only moves the base position.
template <uint32_t D>
struct TileCopier {
  static constexpr uint32_t kPieces = (kTileP * D / 4 + kCThreads - 1) / kCThreads;
  uint32_t row[kPieces], soff[kPieces];
  size_t goff[kPieces];
  __device__ TileCopier(uint32_t kvd, uint32_t g) {
#pragma unroll
    for (uint32_t j = 0; j < kPieces; ++j) {
      const uint32_t c = threadIdx.x + j * kCThreads, r = c / (D / 4), piece = c % (D / 4);
      row[j] = c < kTileP * D / 4 ? r : kTileP;  // kTileP: no piece
      soff[j] = r * D + 4 * piece;
      goff[j] = (size_t)r * kvd + g * D + 4 * piece;
    }
  }
  // Rows [t0, min(t0 + kTileP, r1)) of the cache into buf.
  __device__ __forceinline__ void load(int32_t* buf, const int32_t* cache, uint32_t kvd, uint32_t t0,
                                       uint32_t r1) const {
    const int32_t* base = cache + (size_t)t0 * kvd;
#pragma unroll
    for (uint32_t j = 0; j < kPieces; ++j)
      if (row[j] < kTileP && t0 + row[j] < r1) cp_async16(buf + soff[j], base + goff[j]);
  }
};


template <uint32_t PER, uint32_t HPC>
__global__ void __launch_bounds__(kCThreads, 1) attn_decode_cluster_kernel(AttnArgs a) {
  pdl_wait();
  pdl_trigger();
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  constexpr uint32_t D = PER * 8, NH = kCThreads / D;
  constexpr uint32_t HG = HPC >= 2 ? 2 : 1, HH = HPC / HG;  // warp groups of the score step, heads each
  constexpr uint32_t tile_ints = kTileP * D;
  const uint32_t ring = a.ring, span_a = a.span;      // span_a even
  extern __shared__ __align__(16) int32_t dsm[];
  int32_t* tiles = dsm;                               // [ring][kTileP][D]
  uint64_t* tm = (uint64_t*)(tiles + ring * tile_ints);  // [span][HPC] exp terms
  int32_t* sw = (int32_t*)(tm + span_a * HPC);        // [span][HPC] scores, then weights
  int64_t* part = (int64_t*)(sw + span_a * HPC);      // [HPC][D]
  __shared__ unsigned long long best_s[HPC], sum_s[HPC], gbest_s[HPC], gtotal_s[HPC], ginv_s[HPC];
  __shared__ int32_t wsum_s[HPC], resid_s[HPC];

  const uint32_t C = cluster.num_blocks(), rank = cluster.block_rank();
  const uint32_t h0 = (blockIdx.x / C) * HPC, G = a.heads / a.kv_heads, g = h0 / G;
  const uint32_t p = query_position(a), ws = window_start(p, a.window), n = p - ws + 1;
  const uint32_t span = (n + C - 1) / C;
  const uint32_t r0 = min(p + 1, ws + rank * span), r1 = min(p + 1, r0 + span);
  const uint32_t cnt = r1 - r0, ntiles = (cnt + kTileP - 1) / kTileP, nitems = 2 * ntiles;
  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, quad = lane >> 3, ql = lane & 7;

  // item i < ntiles: key tile i; item ntiles + i: value tile i. One commit
  // group an item, issued in order; item i uses buffer i % ring.
  const TileCopier<D> copier(a.kvd, g);
  uint32_t issued = 0;
  auto issue_upto = [&](uint32_t limit) {
    limit = min(limit, nitems);
    for (; issued < limit; ++issued) {
      const bool key = issued < ntiles;
      const uint32_t t0 = r0 + (key ? issued : issued - ntiles) * kTileP;
      copier.load(tiles + (issued % ring) * tile_ints, key ? a.kcache : a.vcache, a.kvd, t0, r1);
      cp_async_commit();
    }
  };
  // Before consuming item i: its group has landed for every thread, and
  // every thread is done with item i - 1, whose buffer item i - 1 + ring
  // then takes.
  auto acquire = [&](uint32_t i) {
    cp_async_wait_pending(issued - (i + 1));
    __syncthreads();
    if (i >= 1) issue_upto(i - 1 + ring + 1);
  };
  issue_upto(ring);

  for (uint32_t i = tid; i < HPC * D; i += kCThreads) part[i] = 0;
  if (tid < HPC) {
    best_s[tid] = 0;
    sum_s[tid] = 0;
    wsum_s[tid] = 0;
  }

  // ---- 1. scores: warp group wg (of HG) takes heads [wg HH, wg HH + HH); 8
  // lanes a position, lane ql holding the 16-byte pieces ql, ql + 8, ...
  const uint32_t wg = warp / 8, wl = warp % 8, hb = wg * HH;
  const bool scoring = wg < HG;
  int4 q[HH][PER / 4];
#pragma unroll
  for (uint32_t h = 0; h < HH; ++h)
#pragma unroll
    for (uint32_t i = 0; i < PER / 4; ++i)
      q[h][i] = scoring ? *(const int4*)(a.q + (size_t)(h0 + hb + h) * D + 4 * (ql + 8 * i)) : make_int4(0, 0, 0, 0);
  unsigned long long best[HH];
#pragma unroll
  for (uint32_t h = 0; h < HH; ++h) best[h] = 0;
  for (uint32_t k = 0; k < ntiles; ++k) {
    acquire(k);
    if (!scoring) continue;
    const uint32_t tl = wl * 4 + quad, t = r0 + k * kTileP + tl;
    const int32_t* krow = tiles + (k % ring) * tile_ints + tl * D;
    int4 kv[PER / 4];
#pragma unroll
    for (uint32_t i = 0; i < PER / 4; ++i) kv[i] = *(const int4*)(krow + 4 * (ql + 8 * i));
#pragma unroll
    for (uint32_t h = 0; h < HH; ++h) {
      int64_t c0 = 0, c1 = 0, c2 = 0, c3 = 0;
#pragma unroll
      for (uint32_t i = 0; i < PER / 4; ++i) {
        mac_wide(c0, q[h][i].x, kv[i].x);
        mac_wide(c1, q[h][i].y, kv[i].y);
        mac_wide(c2, q[h][i].z, kv[i].z);
        mac_wide(c3, q[h][i].w, kv[i].w);
      }
      uint64_t sum = (uint64_t)c0 + (uint64_t)c1 + (uint64_t)c2 + (uint64_t)c3;
      sum += __shfl_xor_sync(0xffffffffu, sum, 4);
      sum += __shfl_xor_sync(0xffffffffu, sum, 2);
      sum += __shfl_xor_sync(0xffffffffu, sum, 1);
      if (ql == 0 && t < r1) {
        const int32_t sc = finish_score((int64_t)sum, a.mode, a.scale_q32);
        sw[(t - r0) * HPC + hb + h] = sc;
        const unsigned long long key = best_key(sc, t);
        best[h] = key > best[h] ? key : best[h];
      }
    }
  }
#pragma unroll
  for (uint32_t h = 0; h < HH; ++h)
    if (scoring && ql == 0 && best[h]) atomicMax(&best_s[hb + h], best[h]);
  cluster.sync();
  if (tid < HPC) {
    unsigned long long b = 0;
    for (uint32_t r = 0; r < C; ++r) {
      const unsigned long long v = *cluster.map_shared_rank(&best_s[tid], r);
      b = v > b ? v : b;
    }
    gbest_s[tid] = b;
  }
  __syncthreads();

  // ---- 2. exp terms against the global first maximum (kept), and their sums.
  // Element e = position * HPC + head: thread tid always meets head tid % HPC.
  const uint32_t my_h = tid % HPC;
  {
    const int32_t mx = best_key_value(gbest_s[my_h]);
    uint64_t e = 0;
    for (uint32_t el = tid; el < cnt * HPC; el += kCThreads) {
      const uint64_t term = (uint64_t)softmax_exp_term_act(sw[el], mx);
      tm[el] = term;
      e += term;
    }
    e = head_lane_sum<HPC>(e);
    if (lane < HPC && e) atomicAdd(&sum_s[lane], (unsigned long long)e);
  }
  cluster.sync();
  if (tid < HPC) {
    unsigned long long tot = 0;
    for (uint32_t r = 0; r < C; ++r) tot += *cluster.map_shared_rank(&sum_s[tid], r);
    gtotal_s[tid] = tot;
    ginv_s[tid] = UINT64_MAX / tot;  // tot >= 2^32: the first maximum's term is 2^32
  }
  __syncthreads();

  // ---- 3. weights over the scores and their sums, then the value sums
  {
    const uint64_t tot = gtotal_s[my_h], inv = ginv_s[my_h];
    int32_t wsum = 0;
    for (uint32_t el = tid; el < cnt * HPC; el += kCThreads) {
      const int32_t w = softmax_weight_inv((int64_t)tm[el], tot, inv);
      sw[el] = w;
      wsum += w;
    }
    wsum = head_lane_sum<HPC>(wsum);
    if (lane < HPC && wsum) atomicAdd(&wsum_s[lane], wsum);
  }
  const uint32_t dim = tid % D, hv = tid / D;
  int64_t acc[HPC];
#pragma unroll
  for (uint32_t h = 0; h < HPC; ++h) acc[h] = 0;
  for (uint32_t k = 0; k < ntiles; ++k) {
    acquire(ntiles + k);  // also orders the weights above before their reads
    const int32_t* buf = tiles + ((ntiles + k) % ring) * tile_ints;
    const uint32_t base = k * kTileP, rows = min(kTileP, cnt - base);
#pragma unroll 4
    for (uint32_t r = hv; r < rows; r += NH) {
      const int32_t v = buf[r * D + dim];
      int32_t w[HPC];
      if (HPC == 4) {
        const int4 w4 = *(const int4*)(sw + (base + r) * HPC);
        w[0] = w4.x, w[1] = w4.y, w[2 % HPC] = w4.z, w[3 % HPC] = w4.w;
      } else if (HPC == 2) {
        const int2 w2 = *(const int2*)(sw + (base + r) * HPC);
        w[0] = w2.x, w[1 % HPC] = w2.y;
      } else {
        w[0] = sw[base + r];
      }
#pragma unroll
      for (uint32_t h = 0; h < HPC; ++h) mac_wide(acc[h], w[h], v);
    }
  }
#pragma unroll
  for (uint32_t h = 0; h < HPC; ++h)
    if (acc[h]) atomicAdd((unsigned long long*)&part[h * D + dim], (unsigned long long)acc[h]);
  cluster.sync();

  // ---- 4. block `rank` finishes outputs [rank * share, (rank + 1) * share)
  if (tid < HPC) {
    int32_t total_w = 0;
    for (uint32_t r = 0; r < C; ++r) total_w += *cluster.map_shared_rank(&wsum_s[tid], r);
    resid_s[tid] = sub_sat(kOneAct, total_w);  // residual (ops.rs:274-276)
  }
  __syncthreads();
  const uint32_t share = (HPC * D + C - 1) / C, qd = a.heads * D;
  for (uint32_t o = rank * share + tid; o < min(HPC * D, (rank + 1) * share); o += kCThreads) {
    const uint32_t h = o / D, i = o % D, hh = h0 + h;
    uint64_t s = 0;
    for (uint32_t r = 0; r < C; ++r) s += (uint64_t)*cluster.map_shared_rank(&part[o], r);
    const uint32_t tmax = best_key_token(gbest_s[h]);
    s += (uint64_t)((int64_t)resid_s[h] * a.vcache[(size_t)tmax * a.kvd + g * D + i]);
    const int32_t v = requantize((int64_t)s);
    put_planes(a.ctx_planes, qd, hh * D + i, v);
    if (a.ctx) a.ctx[hh * D + i] = v;
  }
  cluster.sync();  // every block's shared memory stays until all have read it
}

// ---------------------------------------------------------------------------
// Decode attention in one launch over the whole GPU
// ---------------------------------------------------------------------------
//
// A head group (HPC query heads of one kv group) is split over `chunks`
// blocks, about one block a multiprocessor over all groups; block r takes the
// r-th contiguous range of the window [ws, p] and copies all of its key rows
// and value rows into shared memory with cp.async at its start (two commit
// groups), so the whole cache read of the step is in flight at once. The
// three dependent steps of attention_softmax (ops.rs:233-261) meet through
// global memory: first-maximum keys (atomicMax), sums of exp terms and of
// weights, and the wrapping weighted value sums (atomicAdd) of the group,
// with a bounded arrival barrier after the first two steps. The group's last
// block to add its value sums finishes every output of the group and clears
// the exchange words for the next launch. The blocks of a launch must be
// resident together (the plan checks the occupancy); a barrier that waits
// about a second records a fault instead of hanging.

constexpr uint32_t kGThreads = 256;


// Arrival barrier of one head group: returns once *bar reaches target. The
// block's earlier global atomics are published by the release arrival (after
// the block barrier) and seen by the acquire loads of the other blocks.
__device__ __forceinline__ void group_barrier(unsigned int* bar, unsigned int target, unsigned int* fault) {
  __syncthreads();
  if (threadIdx.x == 0) {
    red_add_release(bar, 1u);
    if (ld_acquire_u32(bar) < target) {
      const uint64_t t0 = global_ns();
      for (uint32_t i = 1;; ++i) {
        __nanosleep(32);
        if (ld_acquire_u32(bar) >= target) break;
        if ((i & 255) == 0 && global_ns() - t0 > 1000000000ull) {
          if (fault) atomicOr(fault, 1u);
          break;
        }
      }
    }
  }
  __syncthreads();
}

template <uint32_t PER, uint32_t HPC>
__global__ void __launch_bounds__(kGThreads) attn_decode_grid_kernel(AttnArgs a) {
  constexpr uint32_t D = PER * 8, NH = kGThreads / D, kWarps = kGThreads / 32;
  const uint32_t span_a = a.gspan;                   // even
  extern __shared__ __align__(16) int32_t gsm[];
  int32_t* ks = gsm;                                  // [span][D]
  int32_t* vs = ks + span_a * D;                      // [span][D]
  uint64_t* tm = (uint64_t*)(vs + span_a * D);        // [span][HPC] exp terms
  int32_t* sw = (int32_t*)(tm + span_a * HPC);        // [span][HPC] scores, then weights
  __shared__ unsigned long long best_s[HPC], sum_s[HPC], gbest_s[HPC], gtot_s[HPC], ginv_s[HPC];
  __shared__ int32_t wsum_s[HPC], resid_s[HPC];

  const uint32_t chunks = a.chunks, grp = blockIdx.x / chunks, rank = blockIdx.x % chunks;
  const uint32_t h0 = grp * HPC, G = a.heads / a.kv_heads, g = h0 / G;
  const uint32_t p = query_position(a), ws = window_start(p, a.window), n = p - ws + 1;
  const uint32_t span = (n + chunks - 1) / chunks;
  const uint32_t r0 = min(p + 1, ws + rank * span), r1 = min(p + 1, r0 + span), cnt = r1 - r0;
  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, quad = lane >> 3, ql = lane & 7;
  unsigned int* bar = a.gbar + grp;

  // Every key row, then every value row of the block's range, except the
  // query's own position: those rows were written by earlier passes, so they
  // stream while the q|k|v product that precedes this kernel finishes (the
  // decode position was written two or more kernels earlier).
  const uint32_t held = cnt - (cnt && r1 == p + 1 ? 1u : 0u);  // rows before position p
  for (uint32_t c = tid; c < held * (D / 4); c += kGThreads) {
    const uint32_t r = c / (D / 4), j = c % (D / 4);
    cp_async16(ks + r * D + 4 * j, a.kcache + (size_t)(r0 + r) * a.kvd + g * D + 4 * j);
  }
  cp_async_commit();
  for (uint32_t c = tid; c < held * (D / 4); c += kGThreads) {
    const uint32_t r = c / (D / 4), j = c % (D / 4);
    cp_async16(vs + r * D + 4 * j, a.vcache + (size_t)(r0 + r) * a.kvd + g * D + 4 * j);
  }
  cp_async_commit();
  pdl_wait();
  pdl_trigger();
  if (held < cnt)  // position p: this pass's key and value rows
    for (uint32_t j = tid; j < D / 4; j += kGThreads) {
      *(int4*)(ks + held * D + 4 * j) = *(const int4*)(a.kcache + (size_t)p * a.kvd + g * D + 4 * j);
      *(int4*)(vs + held * D + 4 * j) = *(const int4*)(a.vcache + (size_t)p * a.kvd + g * D + 4 * j);
    }
  if (tid < HPC) {
    best_s[tid] = 0;
    sum_s[tid] = 0;
    wsum_s[tid] = 0;
  }
  int4 q[HPC][PER / 4];
#pragma unroll
  for (uint32_t h = 0; h < HPC; ++h)
#pragma unroll
    for (uint32_t i = 0; i < PER / 4; ++i) q[h][i] = *(const int4*)(a.q + (size_t)(h0 + h) * D + 4 * (ql + 8 * i));
  asm volatile("cp.async.wait_group 1;" ::: "memory");
  __syncthreads();  // every key row has landed

  // ---- 1. scores: 8 lanes a position, four positions a warp at a time
  unsigned long long best[HPC];
#pragma unroll
  for (uint32_t h = 0; h < HPC; ++h) best[h] = 0;
  for (uint32_t base = 0; base < cnt; base += kWarps * 4) {
    const uint32_t tl = base + warp * 4 + quad;
    const bool live = tl < cnt;
    const int32_t* krow = ks + (live ? tl : 0) * D;
    int4 kv[PER / 4];
#pragma unroll
    for (uint32_t i = 0; i < PER / 4; ++i) kv[i] = *(const int4*)(krow + 4 * (ql + 8 * i));
#pragma unroll
    for (uint32_t h = 0; h < HPC; ++h) {
      int64_t c0 = 0, c1 = 0, c2 = 0, c3 = 0;
#pragma unroll
      for (uint32_t i = 0; i < PER / 4; ++i) {
        mac_wide(c0, q[h][i].x, kv[i].x);
        mac_wide(c1, q[h][i].y, kv[i].y);
        mac_wide(c2, q[h][i].z, kv[i].z);
        mac_wide(c3, q[h][i].w, kv[i].w);
      }
      uint64_t sum = (uint64_t)c0 + (uint64_t)c1 + (uint64_t)c2 + (uint64_t)c3;
      sum += __shfl_xor_sync(0xffffffffu, sum, 4);
      sum += __shfl_xor_sync(0xffffffffu, sum, 2);
      sum += __shfl_xor_sync(0xffffffffu, sum, 1);
      if (ql == 0 && live) {
        const int32_t sc = finish_score((int64_t)sum, a.mode, a.scale_q32);
        sw[tl * HPC + h] = sc;
        const unsigned long long key = best_key(sc, r0 + tl);
        best[h] = key > best[h] ? key : best[h];
      }
    }
  }
#pragma unroll
  for (uint32_t h = 0; h < HPC; ++h)
    if (ql == 0 && best[h]) atomicMax(&best_s[h], best[h]);
  __syncthreads();
  if (tid < HPC && best_s[tid]) atomicMax(a.gbest + h0 + tid, best_s[tid]);
  group_barrier(bar, chunks, a.fault);
  if (tid < HPC) gbest_s[tid] = __ldcg(a.gbest + h0 + tid);
  __syncthreads();

  // ---- 2. exp terms against the group's first maximum (kept), their sums.
  // Element e = position * HPC + head: thread tid always meets head tid % HPC.
  const uint32_t my_h = tid % HPC;
  {
    const int32_t mx = best_key_value(gbest_s[my_h]);
    uint64_t e = 0;
    for (uint32_t el = tid; el < cnt * HPC; el += kGThreads) {
      const uint64_t term = (uint64_t)softmax_exp_term_act(sw[el], mx);
      tm[el] = term;
      e += term;
    }
    e = head_lane_sum<HPC>(e);
    if (lane < HPC && e) atomicAdd(&sum_s[lane], (unsigned long long)e);
  }
  __syncthreads();
  if (tid < HPC && sum_s[tid]) atomicAdd(a.gsum + h0 + tid, sum_s[tid]);
  group_barrier(bar, 2 * chunks, a.fault);
  if (tid < HPC) {
    const unsigned long long tot = __ldcg(a.gsum + h0 + tid);
    gtot_s[tid] = tot;
    ginv_s[tid] = tot ? UINT64_MAX / tot : 0;  // tot >= 2^32 after a complete exchange
  }
  __syncthreads();

  // ---- 3. weights over the scores and their sums, then the value sums
  {
    const uint64_t tot = gtot_s[my_h], inv = ginv_s[my_h];
    int32_t wsum = 0;
    for (uint32_t el = tid; el < cnt * HPC; el += kGThreads) {
      const int32_t w = tot ? softmax_weight_inv((int64_t)tm[el], tot, inv) : 0;
      sw[el] = w;
      wsum += w;
    }
    wsum = head_lane_sum<HPC>(wsum);
    if (lane < HPC && wsum) atomicAdd(&wsum_s[lane], wsum);
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncthreads();  // every value row has landed; the weights are written
  if (tid < HPC && wsum_s[tid]) atomicAdd(a.wsum + h0 + tid, wsum_s[tid]);
  {
    const uint32_t dim = tid % D, hv = tid / D;
    int64_t acc[HPC];
#pragma unroll
    for (uint32_t h = 0; h < HPC; ++h) acc[h] = 0;
#pragma unroll 4
    for (uint32_t r = hv; r < cnt; r += NH) {
      const int32_t v = vs[r * D + dim];
      int32_t w[HPC];
      if (HPC == 4) {
        const int4 w4 = *(const int4*)(sw + r * HPC);
        w[0] = w4.x, w[1] = w4.y, w[2 % HPC] = w4.z, w[3 % HPC] = w4.w;
      } else if (HPC == 2) {
        const int2 w2 = *(const int2*)(sw + r * HPC);
        w[0] = w2.x, w[1 % HPC] = w2.y;
      } else {
        w[0] = sw[r];
      }
#pragma unroll
      for (uint32_t h = 0; h < HPC; ++h) mac_wide(acc[h], w[h], v);
    }
#pragma unroll
    for (uint32_t h = 0; h < HPC; ++h)
      if (acc[h]) atomicAdd((unsigned long long*)(a.acc + (size_t)(h0 + h) * D + dim), (unsigned long long)acc[h]);
  }
  // ---- 4. the group's last block to add its sums finishes every output of
  // the group and clears the exchange words for the next launch
  __shared__ bool last_s;
  __syncthreads();
  if (tid == 0) last_s = atom_add_acq_rel(bar, 1u) == 3 * chunks - 1;
  __syncthreads();
  if (!last_s) return;
  if (tid < HPC) resid_s[tid] = sub_sat(kOneAct, (int32_t)__ldcg((const int*)(a.wsum + h0 + tid)));  // ops.rs:274-276
  __syncthreads();
  const uint32_t qd = a.heads * D;
  for (uint32_t o = tid; o < HPC * D; o += kGThreads) {
    const uint32_t h = o / D, i = o % D, hh = h0 + h;
    uint64_t* accp = (uint64_t*)(a.acc + (size_t)hh * D + i);
    uint64_t s = (uint64_t)__ldcg((const unsigned long long*)accp);
    *accp = 0;
    const uint32_t tmax = best_key_token(gbest_s[h]);
    s += (uint64_t)((int64_t)resid_s[h] * a.vcache[(size_t)tmax * a.kvd + g * D + i]);
    const int32_t v = requantize((int64_t)s);
    put_planes(a.ctx_planes, qd, hh * D + i, v);
    if (a.ctx) a.ctx[hh * D + i] = v;
  }
  if (tid < HPC) {
    a.gbest[h0 + tid] = 0;
    a.gsum[h0 + tid] = 0;
    a.wsum[h0 + tid] = 0;
  }
  if (tid == 0) bar[0] = 0;
}

size_t attention_grid_smem(uint32_t d, uint32_t hpc, uint32_t span) {
  return (size_t)span * d * 8 + (size_t)span * hpc * 12;
}

int grid_blocks_per_sm(uint32_t d, uint32_t hpc, size_t smem) {
  int n = 0;
  cudaError_t e = cudaErrorInvalidValue;
  const uint32_t per = d / 8;
#define IRIS_GFITS(PER, HPC) \
  if (per == PER && hpc == HPC) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, attn_decode_grid_kernel<PER, HPC>, kGThreads, smem);
  IRIS_GFITS(4, 1) IRIS_GFITS(4, 2) IRIS_GFITS(4, 4)
  IRIS_GFITS(8, 1) IRIS_GFITS(8, 2) IRIS_GFITS(8, 4)
  IRIS_GFITS(16, 1) IRIS_GFITS(16, 2) IRIS_GFITS(16, 4)
  IRIS_GFITS(32, 1) IRIS_GFITS(32, 2)
#undef IRIS_GFITS
  if (e != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

void attention_grid_plan(uint32_t heads, uint32_t kv_heads, uint32_t d, uint32_t cap, uint32_t* hpc,
                         uint32_t* chunks, uint32_t* span) {
  const uint32_t G = heads / kv_heads;
  uint32_t h = 4;
  while (h > 1 && (G % h || h * d > 512)) h >>= 1;
  *hpc = h;
  *chunks = 0;
  *span = 0;
  if (d % 32 || d > 256 || (d == 256 && h > 2)) return;
  int sms = 0, dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
    return;
  const uint32_t groups = heads / h;
  // two blocks a multiprocessor where they fit (shorter serial work a block),
  // else one; every block of the launch must be resident at once
  for (uint32_t per_sm = 2; per_sm >= 1; --per_sm) {
    const uint32_t c = per_sm * (uint32_t)sms / groups;
    if (c < 2) continue;
    const uint32_t sp = (((cap + c - 1) / c) + 1) & ~1u;
    const size_t smem = attention_grid_smem(d, h, sp);
    if (smem > kClusterSmemMax) continue;
    if ((uint64_t)grid_blocks_per_sm(d, h, smem) * (uint32_t)sms < (uint64_t)groups * c) continue;
    *chunks = c;
    *span = sp;
    return;
  }
}

cudaError_t launch_attention_grid(const AttnArgs& a, cudaStream_t s) {
  const uint32_t per = a.d / 8;
  const dim3 grid(a.chunks * (a.heads / a.ghpc));
  const size_t smem = attention_grid_smem(a.d, a.ghpc, a.gspan);
#define IRIS_GRID(PER, HPC) \
  if (per == PER && a.ghpc == HPC) return launch_k(attn_decode_grid_kernel<PER, HPC>, grid, dim3(kGThreads), smem, s, a);
  IRIS_GRID(4, 1) IRIS_GRID(4, 2) IRIS_GRID(4, 4)
  IRIS_GRID(8, 1) IRIS_GRID(8, 2) IRIS_GRID(8, 4)
  IRIS_GRID(16, 1) IRIS_GRID(16, 2) IRIS_GRID(16, 4)
  IRIS_GRID(32, 1) IRIS_GRID(32, 2)
#undef IRIS_GRID
  return cudaErrorInvalidValue;
}

template <uint32_t PER, uint32_t HPC>
cudaError_t prepare_grid_one() {
  return cudaFuncSetAttribute(attn_decode_grid_kernel<PER, HPC>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              (int)kClusterSmemMax);
}

// Shared memory of one block of the one-launch decode attention.
size_t cluster_smem_bytes(uint32_t d, uint32_t hpc, uint32_t span, uint32_t ring) {
  return (size_t)ring * kTileP * d * 4 + (size_t)span * hpc * 12 + (size_t)hpc * d * 8;
}

// Whether (cluster c, hpc, ring) is a valid one-launch shape for the model
// and cache capacity, with every cluster resident at once; sets *span.
int cluster_fits(uint32_t d, uint32_t hpc, uint32_t c, size_t smem);
bool attention_cluster_shape_ok(uint32_t heads, uint32_t kv_heads, uint32_t d, uint32_t cap, uint32_t c,
                                uint32_t hpc, uint32_t ring, uint32_t* span) {
  const uint32_t G = heads / kv_heads;
  if (d % 32 || d > 256 || hpc == 0 || hpc > 4 || (hpc & (hpc - 1)) || G % hpc || hpc * d > 512) return false;
  if (c != 4 && c != 8 && c != 16) return false;
  if (ring < 2 || ring > kMaxRing) return false;
  const uint32_t sp = (((cap + c - 1) / c) + 1) & ~1u;
  const size_t smem = cluster_smem_bytes(d, hpc, sp, ring);
  if (smem > kClusterSmemMax) return false;
  if (cluster_fits(d, hpc, c, smem) < (int)(heads / hpc)) return false;
  *span = sp;
  return true;
}

// Query heads a block and blocks a cluster of the one-launch decode attention
// (0 blocks: the shape is served by the three-launch path), the positions a
// block at most and the tile buffers of its ring: the first shape of a
// preference list whose clusters are all resident at once. Six buffers a
// block (about 100 KB for d = 128) keep enough reads in flight and let two
// blocks share a multiprocessor.
void attention_cluster_plan(uint32_t heads, uint32_t kv_heads, uint32_t d, uint32_t cap, uint32_t* hpc,
                            uint32_t* cluster, uint32_t* span, uint32_t* ring) {
  const uint32_t G = heads / kv_heads;
  uint32_t hmax = 4;
  while (hmax > 1 && (G % hmax || hmax * d > 512)) hmax >>= 1;
  const uint32_t hhalf = hmax > 1 ? hmax / 2 : 1;
  const uint32_t shapes[4][2] = {{16, hmax}, {16, hhalf}, {8, hhalf}, {8, hmax}};
  *hpc = hmax;
  *cluster = 0;
  *span = 0;
  *ring = 0;
  for (const auto& sh : shapes) {
    const uint32_t sp = (((cap + sh[0] - 1) / sh[0]) + 1) & ~1u;
    uint32_t rg = 2 * ((sp + kTileP - 1) / kTileP);  // every key and value tile of a block
    rg = rg < 6 ? rg : 6;
    rg = rg < 2 ? 2 : rg;
    uint32_t got = 0;
    if (!attention_cluster_shape_ok(heads, kv_heads, d, cap, sh[0], sh[1], rg, &got)) continue;
    *hpc = sh[1];
    *cluster = sh[0];
    *span = got;
    *ring = rg;
    return;
  }
}

size_t attention_cluster_smem(const AttnArgs& a) { return cluster_smem_bytes(a.d, a.chpc, a.span, a.ring); }

cudaError_t launch_attention_cluster(const AttnArgs& a, cudaStream_t s) {
  const uint32_t per = a.d / 8;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.cluster * (a.heads / a.chpc));
  cfg.blockDim = dim3(kCThreads);
  cfg.dynamicSmemBytes = attention_cluster_smem(a);
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = a.cluster;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
#define IRIS_CLUSTER(PER, HPC) \
  if (per == PER && a.chpc == HPC) return cudaLaunchKernelEx(&cfg, attn_decode_cluster_kernel<PER, HPC>, a);
  IRIS_CLUSTER(4, 1) IRIS_CLUSTER(4, 2) IRIS_CLUSTER(4, 4)
  IRIS_CLUSTER(8, 1) IRIS_CLUSTER(8, 2) IRIS_CLUSTER(8, 4)
  IRIS_CLUSTER(16, 1) IRIS_CLUSTER(16, 2) IRIS_CLUSTER(16, 4)
  IRIS_CLUSTER(32, 1) IRIS_CLUSTER(32, 2)
#undef IRIS_CLUSTER
  return cudaErrorInvalidValue;
}

template <uint32_t PER, uint32_t HPC>
cudaError_t prepare_cluster_one() {
  cudaError_t e = cudaFuncSetAttribute(attn_decode_cluster_kernel<PER, HPC>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kClusterSmemMax);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(attn_decode_cluster_kernel<PER, HPC>, cudaFuncAttributeNonPortableClusterSizeAllowed,
                             1);
  return e;
}

// Clusters of c blocks of the (d / 8, hpc) instantiation with `smem` bytes
// of shared memory that the device runs at once (0 when it runs none).
int cluster_fits(uint32_t d, uint32_t hpc, uint32_t c, size_t smem) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(c * 64);
  cfg.blockDim = dim3(kCThreads);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = c;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  cudaError_t e = cudaErrorInvalidValue;
  const uint32_t per = d / 8;
#define IRIS_FITS(PER, HPC) \
  if (per == PER && hpc == HPC) e = cudaOccupancyMaxActiveClusters(&n, attn_decode_cluster_kernel<PER, HPC>, &cfg);
  IRIS_FITS(4, 1) IRIS_FITS(4, 2) IRIS_FITS(4, 4)
  IRIS_FITS(8, 1) IRIS_FITS(8, 2) IRIS_FITS(8, 4)
  IRIS_FITS(16, 1) IRIS_FITS(16, 2) IRIS_FITS(16, 4)
  IRIS_FITS(32, 1) IRIS_FITS(32, 2)
#undef IRIS_FITS
  if (e != cudaSuccess) {
    cudaGetLastError();  // a refused query leaves no error behind
    return 0;
  }
  return n;
}

cudaError_t prepare_attention_cluster_kernels() {
  cudaError_t e = cudaSuccess;
#define IRIS_CLUSTER_ATTR(PER, HPC) \
  if (e == cudaSuccess) e = prepare_cluster_one<PER, HPC>();
  IRIS_CLUSTER_ATTR(4, 1) IRIS_CLUSTER_ATTR(4, 2) IRIS_CLUSTER_ATTR(4, 4)
  IRIS_CLUSTER_ATTR(8, 1) IRIS_CLUSTER_ATTR(8, 2) IRIS_CLUSTER_ATTR(8, 4)
  IRIS_CLUSTER_ATTR(16, 1) IRIS_CLUSTER_ATTR(16, 2) IRIS_CLUSTER_ATTR(16, 4)
  IRIS_CLUSTER_ATTR(32, 1) IRIS_CLUSTER_ATTR(32, 2)
#undef IRIS_CLUSTER_ATTR
#define IRIS_GRID_ATTR(PER, HPC) \
  if (e == cudaSuccess) e = prepare_grid_one<PER, HPC>();
  IRIS_GRID_ATTR(4, 1) IRIS_GRID_ATTR(4, 2) IRIS_GRID_ATTR(4, 4)
  IRIS_GRID_ATTR(8, 1) IRIS_GRID_ATTR(8, 2) IRIS_GRID_ATTR(8, 4)
  IRIS_GRID_ATTR(16, 1) IRIS_GRID_ATTR(16, 2) IRIS_GRID_ATTR(16, 4)
  IRIS_GRID_ATTR(32, 1) IRIS_GRID_ATTR(32, 2)
#undef IRIS_GRID_ATTR
  return e;
}

cudaError_t launch_attention_decode(const AttnArgs& a, cudaStream_t s) {
  const uint32_t G = a.heads / a.kv_heads;
  if (a.d % 32 || a.d > 256 || a.hpc == 0 || a.hpc > (uint32_t)kMaxHpc || G % a.hpc ||
      (a.d == 256 && a.hpc > 2))
    return cudaErrorInvalidValue;
  if (a.chunks) return launch_attention_grid(a, s);
  if (a.cluster) return launch_attention_cluster(a, s);
  dim3 grid(a.heads / a.hpc, a.nchunks);
  cudaError_t e = launch_attn_scores(a, grid, s);
  if (e != cudaSuccess) return e;
  e = launch_k(attn_exp_kernel, grid, dim3(kAttnThreads), 0, s, a);
  if (e != cudaSuccess) return e;
  return launch_k(attn_out_kernel, grid, dim3(kAttnThreads), 0, s, a);
}

// ---------------------------------------------------------------------------
// Prefill attention: one block a (query, head)
// ---------------------------------------------------------------------------

__global__ void __launch_bounds__(kAttnThreads) attn_prefill_kernel(AttnArgs a) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ __align__(16) unsigned char sm[];
  __shared__ unsigned long long best_s, total_s;
  __shared__ int32_t wsum_s;
  const uint32_t tok = blockIdx.x, h = blockIdx.y;
  const uint32_t G = a.heads / a.kv_heads, g = h / G;
  const uint32_t p = a.pos0 + tok, ws = window_start(p, a.window), n = p - ws + 1;
  int32_t* q_s = (int32_t*)sm;                       // [d]
  int64_t* te = (int64_t*)(sm + ((a.d * 4 + 15) & ~15u));  // [n]
  int32_t* sc = (int32_t*)(te + n);                  // [n]
  const uint32_t qd = a.heads * a.d;
  for (uint32_t i = threadIdx.x; i < a.d; i += blockDim.x) q_s[i] = a.q[(size_t)tok * qd + h * a.d + i];
  if (threadIdx.x == 0) { best_s = 0; total_s = 0; wsum_s = 0; }
  __syncthreads();
  unsigned long long best = 0;
  for (uint32_t j = threadIdx.x; j < n; j += blockDim.x) {
    const int32_t* krow = a.kcache + (size_t)(ws + j) * a.kvd + g * a.d;
    int64_t sum = 0;
    for (uint32_t i = 0; i < a.d; i += 4) {
      int4 k4 = *(const int4*)(krow + i);
      int4 q4 = *(const int4*)(q_s + i);
      sum = (int64_t)((uint64_t)sum + (uint64_t)((int64_t)q4.x * k4.x) + (uint64_t)((int64_t)q4.y * k4.y) +
                      (uint64_t)((int64_t)q4.z * k4.z) + (uint64_t)((int64_t)q4.w * k4.w));
    }
    int32_t s = finish_score(sum, a.mode, a.scale_q32);
    sc[j] = s;
    unsigned long long k = best_key(s, j);
    best = k > best ? k : best;
  }
  atomicMax(&best_s, best);
  __syncthreads();
  const int32_t mx = best_key_value(best_s);
  const uint32_t mslot = best_key_token(best_s);
  unsigned long long tot = 0;
  for (uint32_t j = threadIdx.x; j < n; j += blockDim.x) {
    int64_t e = softmax_exp_term_act(sc[j], mx);
    te[j] = e;
    tot += (unsigned long long)e;
  }
  atomicAdd(&total_s, tot);
  __syncthreads();
  int32_t ws_local = 0;
  for (uint32_t j = threadIdx.x; j < n; j += blockDim.x) {
    int32_t w = softmax_weight(te[j], total_s);
    sc[j] = w;
    ws_local += w;
  }
  atomicAdd(&wsum_s, ws_local);
  __syncthreads();
  if (threadIdx.x == 0) sc[mslot] = add_sat(sc[mslot], sub_sat(kOneAct, wsum_s));
  __syncthreads();
  for (uint32_t i = threadIdx.x; i < a.d; i += blockDim.x) {
    const int32_t* vcol = a.vcache + (size_t)ws * a.kvd + g * a.d + i;
    int64_t acc = 0;
    for (uint32_t j = 0; j < n; ++j)
      acc = (int64_t)((uint64_t)acc + (uint64_t)((int64_t)sc[j] * vcol[(size_t)j * a.kvd]));
    int32_t v = requantize(acc);
    put_planes(a.ctx_planes + (size_t)tok * 4 * qd, qd, h * a.d + i, v);
    if (a.ctx) a.ctx[(size_t)tok * qd + h * a.d + i] = v;
  }
}

// Many queries, one block a (query, head group): the group's HPC query heads
// share each key and value row of the cache (one read for all of them).
// attention_softmax (ops.rs:233-261) as in the decode kernels: scores with
// one key row a thread (the group's query heads in shared memory, read as
// broadcasts) and each head's first maximum, exp terms and their sums,
// weights by one exact reciprocal a head, then the weighted value sums:
// warp w takes rows w, w + 8, ..., lane l dimensions [DL l, DL l + DL)
// (DL = D / 32 values), and the eight warps' sums meet in shared memory. The
// residual 1.0 - sum(weights) times the first maximum's value row is added
// before the one rounding (the same as adding it to that weight, since no
// weight saturates). Shared memory holds only the scores (then the weights):
// the exp terms are computed twice, for their sums and for the weights, so
// that the footprint (16 B a position) leaves room for four blocks a
// multiprocessor up to 3,000-odd positions.
constexpr uint32_t kPrefillThreads = 256;

template <uint32_t PER, uint32_t HPC>
__global__ void __launch_bounds__(kPrefillThreads, 4) attn_prefill_group_kernel(AttnArgs a) {
  pdl_wait();
  pdl_trigger();
  constexpr uint32_t D = PER * 8, kWarps = kPrefillThreads / 32, DL = D / 32;
  static_assert(DL >= 1 && HPC * DL <= 16, "shapes");
  extern __shared__ __align__(16) unsigned char sm[];
  __shared__ unsigned long long wkey[kWarps][HPC], wsum[kWarps][HPC], gkey[HPC], ginv[HPC], gtot[HPC];
  __shared__ int32_t wws[kWarps][HPC], resid[HPC];
  __shared__ __align__(16) int32_t qs[HPC * D];
  const uint32_t tok = blockIdx.x, h0 = blockIdx.y * HPC, g = h0 / (a.heads / a.kv_heads);
  const uint32_t p = a.pos0 + tok, ws = window_start(p, a.window), n = p - ws + 1;
  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t qd = a.heads * D;
  int32_t* sw = (int32_t*)sm;  // [n][HPC] scores, then weights; then the warps' value sums
  const int32_t* kbase = a.kcache + (size_t)ws * a.kvd + g * D;
  const int32_t* vbase = a.vcache + (size_t)ws * a.kvd + g * D;
  for (uint32_t i = tid; i < HPC * D / 4; i += kPrefillThreads)
    ((int4*)qs)[i] = *(const int4*)(a.q + (size_t)tok * qd + (size_t)h0 * D + 4 * i);
  __syncthreads();

  // ---- 1. scores: thread tid takes rows tid, tid + 256, ...
  unsigned long long best[HPC];
#pragma unroll
  for (uint32_t h = 0; h < HPC; ++h) best[h] = 0;
  for (uint32_t t = tid; t < n; t += kPrefillThreads) {
    const int4* krow = (const int4*)(kbase + (size_t)t * a.kvd);
    int64_t c0[HPC], c1[HPC];
#pragma unroll
    for (uint32_t h = 0; h < HPC; ++h) c0[h] = c1[h] = 0;
#pragma unroll 4
    for (uint32_t i = 0; i < D / 4; ++i) {
      const int4 k = __ldg(krow + i);
#pragma unroll
      for (uint32_t h = 0; h < HPC; ++h) {
        const int4 q = ((const int4*)qs)[h * (D / 4) + i];
        mac_wide(c0[h], q.x, k.x);
        mac_wide(c1[h], q.y, k.y);
        mac_wide(c0[h], q.z, k.z);
        mac_wide(c1[h], q.w, k.w);
      }
    }
#pragma unroll
    for (uint32_t h = 0; h < HPC; ++h) {
      const int32_t sc = finish_score((int64_t)((uint64_t)c0[h] + (uint64_t)c1[h]), a.mode, a.scale_q32);
      sw[t * HPC + h] = sc;
      const unsigned long long key = best_key(sc, t);
      best[h] = key > best[h] ? key : best[h];
    }
  }
#pragma unroll
  for (uint32_t h = 0; h < HPC; ++h) {
#pragma unroll
    for (uint32_t off = 16; off >= 1; off >>= 1) {
      const unsigned long long o = __shfl_xor_sync(0xffffffffu, best[h], off);
      best[h] = o > best[h] ? o : best[h];
    }
    if (lane == 0) wkey[warp][h] = best[h];
  }
  __syncthreads();
  if (tid < HPC) {
    unsigned long long b = 0;
    for (uint32_t w = 0; w < kWarps; ++w) b = wkey[w][tid] > b ? wkey[w][tid] : b;
    gkey[tid] = b;
  }
  __syncthreads();

  // ---- 2. exp terms against each head's first maximum, their sums.
  // Element e = position * HPC + head: thread tid always meets head tid % HPC.
  const uint32_t my_h = tid % HPC;
  const int32_t my_max = best_key_value(gkey[my_h]);
  {
    uint64_t e = 0;
    for (uint32_t el = tid; el < n * HPC; el += kPrefillThreads) e += (uint64_t)softmax_exp_term_act(sw[el], my_max);
    e = head_lane_sum<HPC>(e);
    if (lane < HPC) wsum[warp][lane] = e;
  }
  __syncthreads();
  if (tid < HPC) {
    unsigned long long t = 0;
    for (uint32_t w = 0; w < kWarps; ++w) t += wsum[w][tid];
    gtot[tid] = t;
    ginv[tid] = t ? UINT64_MAX / t : 0;
  }
  __syncthreads();

  // ---- 3. weights and their sums
  {
    const uint64_t tot = gtot[my_h], inv = ginv[my_h];
    int32_t wsl = 0;
    for (uint32_t el = tid; el < n * HPC; el += kPrefillThreads) {
      const int32_t w = tot ? softmax_weight_inv(softmax_exp_term_act(sw[el], my_max), tot, inv) : 0;
      sw[el] = w;
      wsl += w;
    }
    wsl = head_lane_sum<HPC>(wsl);
    if (lane < HPC) wws[warp][lane] = wsl;
  }
  __syncthreads();
  if (tid < HPC) {
    int32_t t = 0;
    for (uint32_t w = 0; w < kWarps; ++w) t += wws[w][tid];
    resid[tid] = sub_sat(kOneAct, t);  // ops.rs:274-276
  }

  // ---- 4. value sums
  uint64_t acc[HPC][DL];
#pragma unroll
  for (uint32_t h = 0; h < HPC; ++h)
#pragma unroll
    for (uint32_t i = 0; i < DL; ++i) acc[h][i] = 0;
#pragma unroll 2
  for (uint32_t t = warp; t < n; t += kWarps) {
    const int32_t* vrow = vbase + (size_t)t * a.kvd + lane * DL;
    int32_t v[DL];
    if constexpr (DL % 4 == 0) {
#pragma unroll
      for (uint32_t i = 0; i < DL / 4; ++i) {
        const int4 x = __ldg((const int4*)vrow + i);
        v[4 * i] = x.x, v[4 * i + 1] = x.y, v[4 * i + 2] = x.z, v[4 * i + 3] = x.w;
      }
    } else if constexpr (DL == 2) {
      const int2 x = __ldg((const int2*)vrow);
      v[0] = x.x, v[1 % DL] = x.y;
    } else {
      v[0] = __ldg(vrow);
    }
#pragma unroll
    for (uint32_t h = 0; h < HPC; ++h) {
      const int32_t w = sw[t * HPC + h];
#pragma unroll
      for (uint32_t i = 0; i < DL; ++i) acc[h][i] += (uint64_t)((int64_t)w * (int64_t)v[i]);
    }
  }
  __syncthreads();  // every weight is read: their space takes the warps' sums
  uint64_t* tree = (uint64_t*)sm;  // [kWarps / 2][HPC DL][32], over the weights (all read)
  constexpr uint32_t NA = HPC * DL;
  for (uint32_t half = kWarps / 2; half >= 1; half >>= 1) {
    if (warp >= half && warp < 2 * half) {
#pragma unroll
      for (uint32_t v = 0; v < NA; ++v) tree[((warp - half) * NA + v) * 32 + lane] = acc[v / DL][v % DL];
    }
    __syncthreads();
    if (warp < half) {
#pragma unroll
      for (uint32_t v = 0; v < NA; ++v) acc[v / DL][v % DL] += tree[(warp * NA + v) * 32 + lane];
    }
    __syncthreads();
  }
  if (warp == 0) {
#pragma unroll
    for (uint32_t h = 0; h < HPC; ++h) {
      const uint32_t tmax = best_key_token(gkey[h]);
#pragma unroll
      for (uint32_t i = 0; i < DL; ++i) {
        const uint32_t dim = lane * DL + i;
        const uint64_t s = acc[h][i] + (uint64_t)((int64_t)resid[h] * __ldg(vbase + (size_t)tmax * a.kvd + dim));
        const int32_t y = requantize((int64_t)s);
        put_planes(a.ctx_planes + (size_t)tok * 4 * qd, qd, (h0 + h) * D + dim, y);
        if (a.ctx) a.ctx[(size_t)tok * qd + (h0 + h) * D + dim] = y;
      }
    }
  }
}

size_t prefill_group_smem(uint32_t hpc, uint32_t d, uint32_t max_visible) {
  const size_t tree = (size_t)kPrefillThreads / 64 * hpc * (d / 32) * 32 * 8;  // [warps / 2][HPC DL][32] u64
  return std::max((size_t)max_visible * hpc * 4, tree);
}

#define IRIS_PREFILL_SHAPES(X) X(4, 1) X(4, 2) X(4, 4) X(8, 1) X(8, 2) X(8, 4) X(16, 1) X(16, 2) X(16, 4) X(32, 1) X(32, 2)

cudaError_t launch_attention_prefill(const AttnArgs& a, uint32_t tokens, uint32_t max_visible,
                                     cudaStream_t s) {
  if (tokens == 0) return cudaSuccess;
  if (a.d % 4) return cudaErrorInvalidValue;
  // the group kernel: the group's query heads share each cached row
  const uint32_t G = a.heads / a.kv_heads, per = a.d / 8;
  uint32_t hpc = 4;
  while (hpc > 1 && (G % hpc || hpc * a.d > 512)) hpc >>= 1;
  const size_t gsmem = prefill_group_smem(hpc, a.d, max_visible);
  if (a.d % 32 == 0 && gsmem <= 200 * 1024) {
    const dim3 grid(tokens, a.heads / hpc);
#define IRIS_PREFILL_LAUNCH(PER, HPC) \
    if (per == PER && hpc == HPC) return launch_k(attn_prefill_group_kernel<PER, HPC>, grid, dim3(kPrefillThreads), gsmem, s, a);
    IRIS_PREFILL_SHAPES(IRIS_PREFILL_LAUNCH)
#undef IRIS_PREFILL_LAUNCH
  }
  size_t smem = ((a.d * 4 + 15) & ~15u) + (size_t)max_visible * 12;
  if (smem > 200 * 1024) return cudaErrorInvalidValue;
  dim3 grid(tokens, a.heads);
  return launch_k(attn_prefill_kernel, grid, dim3(kAttnThreads), smem, s, a);
}

cudaError_t prepare_layer_kernels() {
  cudaError_t e = cudaFuncSetAttribute(attn_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
#define IRIS_PREFILL_PREPARE(PER, HPC)                                                                          \
  if (e == cudaSuccess)                                                                                        \
    e = cudaFuncSetAttribute(attn_prefill_group_kernel<PER, HPC>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                             200 * 1024);
  IRIS_PREFILL_SHAPES(IRIS_PREFILL_PREPARE)
#undef IRIS_PREFILL_PREPARE
  if (e == cudaSuccess) e = prepare_attention_cluster_kernels();
  return e;
}

// ---------------------------------------------------------------------------
// Embeddings, selection bookkeeping
// ---------------------------------------------------------------------------

__global__ void embed_kernel(const int8_t* __restrict__ q, const uint16_t* __restrict__ s, uint32_t cols,
                             uint32_t kc, uint32_t nslices, const uint32_t* ids, int32_t scale, int has_scale,
                             int32_t* out) {
  pdl_wait();
  pdl_trigger();
  uint32_t t = blockIdx.x, id = ids[t];
  for (uint32_t i = threadIdx.x; i < cols; i += blockDim.x) {
    int32_t m, e;
    q8_scale_parts(s[q8_scale_offset(kc, nslices, id, i >> 5)], &m, &e);
    int32_t v = q8_dequant(q[q8_value_offset(kc, nslices, id, i)], m, e);  // dequantize_row, q8.rs:76-91
    if (has_scale) v = mul_sat(v, scale);   // model.rs:316-330 (gemma)
    out[(size_t)t * cols + i] = v;
  }
}

cudaError_t launch_embed(const Q8GpuMatrix* embed, const uint32_t* d_ids, uint32_t tokens,
                         int has_scale, int32_t scale, int32_t* out, cudaStream_t s) {
  if (tokens == 0) return cudaSuccess;
  return launch_k(embed_kernel, dim3(tokens), dim3(256), 0, s, (const int8_t*)embed->q, (const uint16_t*)embed->s,
                  embed->cols, embed->kc, embed->nslices, d_ids, scale, has_scale, out);
}

__global__ void fill_u64_kernel(unsigned long long* p, uint32_t n) {
  pdl_wait();
  pdl_trigger();
  uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) p[i] = 0;
}
cudaError_t launch_fill_u64(unsigned long long* p, uint32_t n, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  return launch_k(fill_u64_kernel, dim3((n + 255) / 256), dim3(256), 0, s, p, n);
}

__global__ void decode_finish_kernel(unsigned long long* best, uint32_t* d_token, uint32_t* d_pos,
                                     uint32_t* d_step, uint32_t* history, uint32_t cap) {
  pdl_wait();
  pdl_trigger();
  uint32_t tok = best_key_token(*best);  // first maximum (generation.rs:25-58)
  *d_token = tok;
  *best = 0;
  uint32_t step = *d_step;
  if (history && step < cap) history[step] = tok;
  *d_step = step + 1;
  *d_pos = *d_pos + 1;
}
cudaError_t launch_decode_finish(const unsigned long long* best, uint32_t* d_token, uint32_t* d_pos,
                                 uint32_t* d_step, uint32_t* history, uint32_t history_cap,
                                 cudaStream_t s) {
  return launch_k(decode_finish_kernel, dim3(1), dim3(1), 0, s, (unsigned long long*)best, d_token, d_pos, d_step,
                  history, history_cap);
}

// ---------------------------------------------------------------------------
// Gemma rows
// ---------------------------------------------------------------------------

__device__ uint64_t block_sumsq(const int32_t* v, uint32_t n, uint64_t* red) {
  uint64_t ss = 0;
  for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) ss = add_sat_nonneg(ss, (uint64_t)((int64_t)v[i] * v[i]));
  ss = warp_sum_sat_nonneg(ss);
  int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  uint64_t t = 0;
  for (uint32_t w = 0; w < (blockDim.x + 31) / 32; ++w) t = add_sat_nonneg(t, red[w]);
  return t;  // every thread
}

// In-place rms_norm (weighted when w != NULL) of an n-value row in shared memory.
__device__ void block_rms_norm(int32_t* v, uint32_t n, const int32_t* w, int64_t eps, uint64_t* red) {
  int32_t scale = rms_scale_from_sumsq(block_sumsq(v, n, red), n, eps);
  __syncthreads();
  for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
    int32_t y = mul_sat(v[i], scale);
    v[i] = w ? mul_sat(y, w[i]) : y;
  }
  __syncthreads();
}

// Heads of at most kQkvPer * kQkvThreads values; the norm weights (they
// never change), the position (advanced two or more kernels earlier) and the
// rotation's cosines and sines come before the dependent-launch wait, so that
// they overlap the end of the q|k|v product.
constexpr uint32_t kQkvThreads = 128, kQkvPer = 4;
__global__ void __launch_bounds__(kQkvThreads) gemma_qkv_finish_kernel(QkvFinishArgs a) {
  extern __shared__ __align__(16) int32_t hv[];  // [d]
  __shared__ uint64_t red[32];
  const uint32_t tok = blockIdx.x, which = blockIdx.y, d = a.d, nt = blockDim.x;
  const uint32_t qd = a.heads * d, kvd = a.kv_heads * d;
  const bool is_q = which < a.heads, is_k = !is_q && which < a.heads + a.kv_heads;
  const int32_t* w = is_q ? a.q_norm : is_k ? a.k_norm : nullptr;
  const bool regs = d <= kQkvPer * nt && a.rotary_dim / 2 <= kQkvPer * nt;
  const uint32_t pos = (a.pos_ptr ? *a.pos_ptr : a.pos0) + tok;
  const uint32_t half = a.rotary_dim / 2;
  int32_t wv[kQkvPer], cv[kQkvPer], sv[kQkvPer];
  if (regs) {
#pragma unroll
    for (uint32_t j = 0; j < kQkvPer; ++j) {
      const uint32_t i = threadIdx.x + j * nt;
      wv[j] = w && i < d ? w[i] : 0;
      cv[j] = sv[j] = 0;
      if ((is_q || is_k) && pos && i < half) sin_cos_acc((int64_t)pos * a.inv_freq[i], &cv[j], &sv[j]);
    }
  }
  pdl_wait();
  pdl_trigger();
  const int32_t* src = a.qkv + (size_t)tok * (qd + 2 * kvd) + (size_t)which * d;
  for (uint32_t i = threadIdx.x; i < d; i += nt) hv[i] = src[i];
  __syncthreads();
  if (regs) {
    // block_rms_norm with the weights from registers (prefill_range.rs:617-627)
    const int32_t scale = rms_scale_from_sumsq(block_sumsq(hv, d, red), d, a.eps);
#pragma unroll
    for (uint32_t j = 0; j < kQkvPer; ++j) {
      const uint32_t i = threadIdx.x + j * nt;
      if (i >= d) continue;
      const int32_t y = mul_sat(hv[i], scale);
      hv[i] = w ? mul_sat(y, wv[j]) : y;
    }
    __syncthreads();
    if ((is_q || is_k) && half && pos) {  // apply_rope, prefill_range.rs:631-647
#pragma unroll
      for (uint32_t j = 0; j < kQkvPer; ++j) {
        const uint32_t i = threadIdx.x + j * nt;
        if (i >= half) continue;
        int32_t l = hv[i], r = hv[i + half];
        rotate_half_pair_cs(&l, &r, cv[j], sv[j]);
        hv[i] = l;
        hv[i + half] = r;
      }
      __syncthreads();
    }
  } else if (is_q || is_k) {
    block_rms_norm(hv, d, w, a.eps, red);  // prefill_range.rs:617-624
    if (half && pos) {  // apply_rope, prefill_range.rs:631-647
      for (uint32_t i = threadIdx.x; i < half; i += nt) {
        int32_t l = hv[i], r = hv[i + half];
        rotate_half_pair(&l, &r, a.inv_freq[i], pos);
        hv[i] = l;
        hv[i + half] = r;
      }
      __syncthreads();
    }
  } else {
    block_rms_norm(hv, d, nullptr, a.eps, red);  // value_rms_norm, prefill_range.rs:625-627
  }
  int32_t* dst;
  if (is_q) dst = a.q_out + (size_t)tok * qd + (size_t)which * d;
  else if (is_k) dst = a.kcache ? a.kcache + (size_t)pos * kvd + (size_t)(which - a.heads) * d : nullptr;
  else dst = a.vcache ? a.vcache + (size_t)pos * kvd + (size_t)(which - a.heads - a.kv_heads) * d : nullptr;
  if (dst)
    for (uint32_t i = threadIdx.x; i < d; i += nt) dst[i] = hv[i];
}

cudaError_t launch_gemma_qkv_finish(const QkvFinishArgs& a, uint32_t tokens, cudaStream_t s) {
  if (tokens == 0) return cudaSuccess;
  dim3 grid(tokens, a.heads + 2 * a.kv_heads);
  return launch_k(gemma_qkv_finish_kernel, grid, dim3(kQkvThreads), a.d * 4, s, a);
}

// Sum of the squares of kPer register values a thread (saturating, as
// block_sumsq: for non-negative terms the order does not matter), block-wide.
template <uint32_t kPer>
__device__ uint64_t block_sumsq_regs(const int32_t (&v)[kPer], uint64_t* red) {
  uint64_t ss = 0;
#pragma unroll
  for (uint32_t j = 0; j < kPer; ++j) ss = add_sat_nonneg(ss, (uint64_t)((int64_t)v[j] * v[j]));
  ss = warp_sum_sat_nonneg(ss);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  uint64_t t = 0;
  for (uint32_t w = 0; w < (blockDim.x + 31) / 32; ++w) t = add_sat_nonneg(t, red[w]);
  return t;  // every thread
}

// Rows of at most kNormPer * blockDim.x values run from registers: each
// thread's values i = threadIdx.x + j * blockDim.x (zero past H, which adds
// nothing to a sum of squares). Few registers and no dynamic shared memory,
// so that the block fits beside the product kernel still running before it
// and its loads of weights overlap that kernel's end (kNormPer, kNormThreads:
// layers.cuh).
__global__ void __launch_bounds__(kNormThreads) gemma_post_attn_kernel(const int32_t* o, int32_t* x, const int32_t* w_post_attn,
                                       const int32_t* w_pre_ffw, int64_t eps, uint32_t H,
                                       uint8_t* planes) {
  __shared__ uint64_t red[32];
  const uint32_t t = blockIdx.x, nt = blockDim.x;
  if (H <= kNormPer * nt) {
    // The norm weights never change and x was written two or more kernels
    // earlier (the o product is the predecessor): both load before the wait.
    int32_t w1[kNormPer], w2[kNormPer], xv[kNormPer], v[kNormPer];
#pragma unroll
    for (uint32_t j = 0; j < kNormPer; ++j) {
      const uint32_t i = threadIdx.x + j * nt;
      const bool in = i < H;
      w1[j] = in && w_post_attn ? w_post_attn[i] : 0;
      w2[j] = in && w_pre_ffw ? w_pre_ffw[i] : 0;
      xv[j] = in ? x[(size_t)t * H + i] : 0;
    }
    pdl_wait();
    pdl_trigger();
#pragma unroll
    for (uint32_t j = 0; j < kNormPer; ++j) {
      const uint32_t i = threadIdx.x + j * nt;
      v[j] = i < H ? o[(size_t)t * H + i] : 0;
    }
    int32_t sc = rms_scale_from_sumsq(block_sumsq_regs(v, red), H, eps);
#pragma unroll
    for (uint32_t j = 0; j < kNormPer; ++j) {
      const uint32_t i = threadIdx.x + j * nt;
      const int32_t n = mul_sat(v[j], sc);
      const int32_t y = add_sat(w_post_attn ? mul_sat(n, w1[j]) : n, xv[j]);
      v[j] = i < H ? y : 0;
      if (i < H) x[(size_t)t * H + i] = y;
    }
    sc = rms_scale_from_sumsq(block_sumsq_regs(v, red), H, eps);
#pragma unroll
    for (uint32_t j = 0; j < kNormPer; ++j) {
      const uint32_t i = threadIdx.x + j * nt;
      const int32_t n = mul_sat(v[j], sc);
      if (i < H) put_planes(planes + (size_t)t * 4 * H, H, i, w_pre_ffw ? mul_sat(n, w2[j]) : n);
    }
    return;
  }
  pdl_wait();
  pdl_trigger();
  extern __shared__ __align__(16) int32_t row[];  // [H]
  for (uint32_t i = threadIdx.x; i < H; i += blockDim.x) row[i] = o[(size_t)t * H + i];
  __syncthreads();
  block_rms_norm(row, H, w_post_attn, eps, red);
  for (uint32_t i = threadIdx.x; i < H; i += blockDim.x) {
    int32_t v = add_sat(row[i], x[(size_t)t * H + i]);
    row[i] = v;
    x[(size_t)t * H + i] = v;
  }
  __syncthreads();
  block_rms_norm(row, H, w_pre_ffw, eps, red);
  for (uint32_t i = threadIdx.x; i < H; i += blockDim.x) put_planes(planes + (size_t)t * 4 * H, H, i, row[i]);
}

cudaError_t launch_gemma_post_attn(const int32_t* o, int32_t* x, const int32_t* w_post_attn,
                                   const int32_t* w_pre_ffw, int64_t eps, uint32_t tokens,
                                   uint32_t hidden, uint8_t* planes, cudaStream_t s) {
  if (tokens == 0) return cudaSuccess;
  const size_t smem = hidden <= kNormPer * kNormThreads ? 0 : hidden * 4;
  return launch_k(gemma_post_attn_kernel, dim3(tokens), dim3(kNormThreads), smem, s, o, x, w_post_attn, w_pre_ffw,
                  eps, hidden, planes);
}

__global__ void __launch_bounds__(kNormThreads) gemma_norm_add_kernel(const int32_t* v_in, const int32_t* add, const int32_t* w,
                                      int64_t eps, int32_t scalar, uint32_t H, int32_t* out) {
  __shared__ uint64_t red[32];
  const uint32_t t = blockIdx.x, nt = blockDim.x;
  if (H <= kNormPer * nt) {
    // The norm weights never change and `add` was written two or more
    // kernels earlier (x after the FFN, xs after the PLE products): both
    // load before the wait.
    int32_t wv[kNormPer], av[kNormPer], v[kNormPer];
#pragma unroll
    for (uint32_t j = 0; j < kNormPer; ++j) {
      const uint32_t i = threadIdx.x + j * nt;
      const bool in = i < H;
      wv[j] = in && w ? w[i] : 0;
      av[j] = in ? add[(size_t)t * H + i] : 0;
    }
    pdl_wait();
    pdl_trigger();
#pragma unroll
    for (uint32_t j = 0; j < kNormPer; ++j) {
      const uint32_t i = threadIdx.x + j * nt;
      v[j] = i < H ? v_in[(size_t)t * H + i] : 0;
    }
    const int32_t sc = rms_scale_from_sumsq(block_sumsq_regs(v, red), H, eps);
#pragma unroll
    for (uint32_t j = 0; j < kNormPer; ++j) {
      const uint32_t i = threadIdx.x + j * nt;
      if (i >= H) continue;
      const int32_t y = mul_sat(v[j], sc);
      int32_t r = add_sat(w ? mul_sat(y, wv[j]) : y, av[j]);
      if (scalar != 0) r = mul_sat(r, scalar);  // scale_row (finish_layer, :953-955)
      out[(size_t)t * H + i] = r;
    }
    return;
  }
  pdl_wait();
  pdl_trigger();
  extern __shared__ __align__(16) int32_t row[];
  for (uint32_t i = threadIdx.x; i < H; i += blockDim.x) row[i] = v_in[(size_t)t * H + i];
  __syncthreads();
  block_rms_norm(row, H, w, eps, red);
  for (uint32_t i = threadIdx.x; i < H; i += blockDim.x) {
    int32_t v = add_sat(row[i], add[(size_t)t * H + i]);
    if (scalar != 0) v = mul_sat(v, scalar);  // scale_row (finish_layer, :953-955)
    out[(size_t)t * H + i] = v;
  }
}

cudaError_t launch_gemma_post_ffw(const int32_t* ff, const int32_t* x, const int32_t* w_post_ffw,
                                  int64_t eps, uint32_t tokens, uint32_t hidden, int32_t* xs,
                                  cudaStream_t s) {
  if (tokens == 0) return cudaSuccess;
  const size_t smem = hidden <= kNormPer * kNormThreads ? 0 : hidden * 4;
  return launch_k(gemma_norm_add_kernel, dim3(tokens), dim3(kNormThreads), smem, s, ff, x, w_post_ffw, eps,
                  (int32_t)0, hidden, xs);
}

cudaError_t launch_gemma_finish(const int32_t* proj, const int32_t* xs, const int32_t* w_ple_post,
                                int64_t eps, int32_t layer_scalar, uint32_t tokens, uint32_t hidden,
                                int32_t* x_out, cudaStream_t s) {
  if (tokens == 0) return cudaSuccess;
  const size_t smem = hidden <= kNormPer * kNormThreads ? 0 : hidden * 4;
  return launch_k(gemma_norm_add_kernel, dim3(tokens), dim3(kNormThreads), smem, s, proj, xs, w_ple_post, eps,
                  layer_scalar, hidden, x_out);
}

// post_ffw (gemma_norm_add_kernel with no scale) and the PLE gate product
// for one token: each block of kNormThreads threads normalises the whole row
// into shared memory (x and the norm weights load before the wait: x was
// written two or more kernels earlier), block 0 stores xs, then each warp
// takes rows of the gate product (dense_kernel's sum and gating).
__global__ void __launch_bounds__(kNormThreads)
    gemma_post_ffw_ple_gate_kernel(const int32_t* ff, const int32_t* x, const int32_t* w_post_ffw, int64_t eps,
                                   uint32_t H, int32_t* xs_out, const int32_t* __restrict__ w_gate, uint32_t P,
                                   const int32_t* gate_rows, int32_t* pg) {
  __shared__ uint64_t red[32];
  __shared__ __align__(16) int32_t xs[kNormPer * kNormThreads];
  const uint32_t nt = blockDim.x;
  int32_t wv[kNormPer], av[kNormPer], v[kNormPer];
#pragma unroll
  for (uint32_t j = 0; j < kNormPer; ++j) {
    const uint32_t i = threadIdx.x + j * nt;
    wv[j] = i < H && w_post_ffw ? w_post_ffw[i] : 0;
    av[j] = i < H ? x[i] : 0;
  }
  pdl_wait();
  pdl_trigger();
#pragma unroll
  for (uint32_t j = 0; j < kNormPer; ++j) {
    const uint32_t i = threadIdx.x + j * nt;
    v[j] = i < H ? ff[i] : 0;
  }
  const int32_t sc = rms_scale_from_sumsq(block_sumsq_regs(v, red), H, eps);
#pragma unroll
  for (uint32_t j = 0; j < kNormPer; ++j) {
    const uint32_t i = threadIdx.x + j * nt;
    if (i >= H) continue;
    const int32_t y = mul_sat(v[j], sc);
    const int32_t r = add_sat(w_post_ffw ? mul_sat(y, wv[j]) : y, av[j]);
    xs[i] = r;
    if (blockIdx.x == 0) xs_out[i] = r;
  }
  __syncthreads();
  const uint32_t lane = threadIdx.x & 31, warps = nt / 32;
  for (uint32_t r = blockIdx.x * warps + (threadIdx.x >> 5); r < P; r += gridDim.x * warps) {
    const int32_t* wr = w_gate + (size_t)r * H;
    int64_t acc = 0;
    for (uint32_t i = lane; i < H; i += 32) acc = (int64_t)((uint64_t)acc + (uint64_t)((int64_t)xs[i] * wr[i]));
    acc = warp_sum_i64(acc);
    if (lane == 0) pg[r] = mul_sat(gelu_tanh(requantize(acc)), gate_rows[r]);  // ple_gate_mul :931-944
  }
}

cudaError_t launch_gemma_post_ffw_ple_gate(const int32_t* ff, const int32_t* x, const int32_t* w_post_ffw,
                                          int64_t eps, uint32_t hidden, int32_t* xs, const int32_t* w_gate,
                                          uint32_t P, const int32_t* gate_rows, int32_t* pg, cudaStream_t s) {
  if (hidden > kNormPer * kNormThreads || P == 0) return cudaErrorInvalidValue;
  const uint32_t warps = kNormThreads / 32, blocks = (P + warps - 1) / warps;
  return launch_k(gemma_post_ffw_ple_gate_kernel, dim3(blocks), dim3(kNormThreads), 0, s, ff, x, w_post_ffw, eps,
                  hidden, xs, w_gate, P, gate_rows, pg);
}

// The PLE projection's rows (a warp a row, dense_kernel's sum) and, in the
// block that completes the row, gemma_norm_add_kernel's layer finish. The
// completion count is a release/acquire pair on *done (no block waits for
// another), and the finishing block reads the other blocks' rows through L2.
__global__ void __launch_bounds__(kNormThreads)
    gemma_ple_proj_finish_kernel(const int32_t* pg, const int32_t* __restrict__ w_proj, uint32_t P, uint32_t H,
                                 int32_t* proj, const int32_t* xs, const int32_t* w_ple_post, int64_t eps,
                                 int32_t scalar, int32_t* x_out, unsigned int* done) {
  __shared__ uint64_t red[32];
  __shared__ bool last;
  pdl_wait();
  pdl_trigger();
  const uint32_t lane = threadIdx.x & 31, nt = blockDim.x;
  const uint32_t r = blockIdx.x * (nt / 32) + (threadIdx.x >> 5);
  if (r < H) {
    const int32_t* wr = w_proj + (size_t)r * P;
    int64_t acc = 0;
    for (uint32_t i = lane; i < P; i += 32) acc = (int64_t)((uint64_t)acc + (uint64_t)((int64_t)pg[i] * wr[i]));
    acc = warp_sum_i64(acc);
    if (lane == 0) proj[r] = requantize(acc);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    last = atom_add_acq_rel(done, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!last) return;
  int32_t wv[kNormPer], av[kNormPer], v[kNormPer];
#pragma unroll
  for (uint32_t j = 0; j < kNormPer; ++j) {
    const uint32_t i = threadIdx.x + j * nt;
    const bool in = i < H;
    wv[j] = in && w_ple_post ? w_ple_post[i] : 0;
    av[j] = in ? xs[i] : 0;
    v[j] = in ? __ldcg(proj + i) : 0;
  }
  const int32_t sc = rms_scale_from_sumsq(block_sumsq_regs(v, red), H, eps);
#pragma unroll
  for (uint32_t j = 0; j < kNormPer; ++j) {
    const uint32_t i = threadIdx.x + j * nt;
    if (i >= H) continue;
    const int32_t y = mul_sat(v[j], sc);
    int32_t o = add_sat(w_ple_post ? mul_sat(y, wv[j]) : y, av[j]);
    if (scalar != 0) o = mul_sat(o, scalar);  // scale_row (finish_layer, :953-955)
    x_out[i] = o;
  }
  if (threadIdx.x == 0) *done = 0;
}

cudaError_t launch_gemma_ple_proj_finish(const int32_t* pg, const int32_t* w_proj, uint32_t P, uint32_t hidden,
                                         int32_t* proj, const int32_t* xs, const int32_t* w_ple_post, int64_t eps,
                                         int32_t layer_scalar, int32_t* x_out, unsigned int* done,
                                         cudaStream_t s) {
  if (hidden > kNormPer * kNormThreads || P == 0 || hidden == 0) return cudaErrorInvalidValue;
  const uint32_t warps = kNormThreads / 32, blocks = (hidden + warps - 1) / warps;
  return launch_k(gemma_ple_proj_finish_kernel, dim3(blocks), dim3(kNormThreads), 0, s, pg, w_proj, P, hidden, proj,
                  xs, w_ple_post, eps, layer_scalar, x_out, done);
}

__global__ void rope_table_kernel(const int64_t* freqs, uint32_t half, const uint32_t* pos_ptr, uint32_t pos0,
                                  uint32_t tokens, int64_t* out) {
  pdl_wait();
  pdl_trigger();
  const uint32_t j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= tokens * half) return;
  const uint32_t t = j / half, i = j % half;
  const uint32_t pos = (pos_ptr ? *pos_ptr : pos0) + t;
  sin_cos_q30((int64_t)pos * freqs[i], out + 2 * (size_t)j, out + 2 * (size_t)j + 1);
}

cudaError_t launch_rope_table(const int64_t* freqs, uint32_t half, const uint32_t* pos_ptr, uint32_t pos0,
                              uint32_t tokens, int64_t* out, cudaStream_t s) {
  const uint32_t n = tokens * half;
  if (n == 0) return cudaSuccess;
  return launch_k(rope_table_kernel, dim3((n + 255) / 256), dim3(256), 0, s, freqs, half, pos_ptr, pos0, tokens, out);
}

// Warp per (token, row) dense product.
__global__ void dense_kernel(const int32_t* __restrict__ w, uint32_t rows, uint32_t cols,
                             const int32_t* __restrict__ in, uint32_t in_stride, uint32_t tokens,
                             int32_t* out, uint32_t out_stride, const int32_t* gate, uint32_t gate_stride) {
  pdl_wait();
  pdl_trigger();
  const uint32_t warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= rows * tokens) return;
  const uint32_t t = warp / rows, r = warp % rows;
  const int32_t* x = in + (size_t)t * in_stride;
  const int32_t* wr = w + (size_t)r * cols;
  int64_t acc = 0;
  for (uint32_t i = lane; i < cols; i += 32)
    acc = (int64_t)((uint64_t)acc + (uint64_t)((int64_t)x[i] * wr[i]));
  acc = warp_sum_i64(acc);
  if (lane == 0) {
    int32_t v = requantize(acc);
    if (gate) v = mul_sat(gelu_tanh(v), gate[(size_t)t * gate_stride + r]);  // ple_gate_mul :931-944
    out[(size_t)t * out_stride + r] = v;
  }
}

cudaError_t launch_dense(const int32_t* w, uint32_t rows, uint32_t cols, const int32_t* in,
                         uint32_t in_stride, uint32_t tokens, int32_t* out, uint32_t out_stride,
                         const int32_t* gelu_gate, uint32_t gate_stride, cudaStream_t s) {
  uint64_t warps = (uint64_t)rows * tokens;
  if (warps == 0) return cudaSuccess;
  return launch_k(dense_kernel, dim3((unsigned)((warps + 7) / 8)), dim3(256), 0, s, w, rows, cols, in, in_stride, tokens,
                  out, out_stride, gelu_gate, gate_stride);
}

__global__ void ple_prepare_kernel(const int32_t* projected, const int8_t* eq, const uint16_t* es,
                                   uint32_t ekc, uint32_t enslices, const uint32_t* ids, const int32_t* ple_norm,
                                   int64_t eps, int32_t projection_scalar, int32_t embedding_scale,
                                   int32_t input_scale, uint32_t L, uint32_t P, int32_t* out) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ __align__(16) int32_t row[];  // [P]
  __shared__ uint64_t red[32];
  const uint32_t t = blockIdx.x, l = blockIdx.y, id = ids[t];
  for (uint32_t j = threadIdx.x; j < P; j += blockDim.x)
    row[j] = mul_sat(projected[((size_t)t * L + l) * P + j], projection_scalar);
  __syncthreads();
  block_rms_norm(row, P, ple_norm, eps, red);
  for (uint32_t j = threadIdx.x; j < P; j += blockDim.x) {
    uint32_t col = l * P + j;
    int32_t m, e;
    q8_scale_parts(es[q8_scale_offset(ekc, enslices, id, col >> 5)], &m, &e);
    int32_t v = mul_sat(q8_dequant(eq[q8_value_offset(ekc, enslices, id, col)], m, e), embedding_scale);
    v = add_sat(v, row[j]);
    out[((size_t)t * L + l) * P + j] = mul_sat(v, input_scale);
  }
}

cudaError_t launch_ple_prepare(const int32_t* projected, const Q8GpuMatrix* ple_embed,
                               const uint32_t* d_ids, const int32_t* ple_norm, int64_t eps,
                               int32_t projection_scalar, int32_t embedding_scale,
                               int32_t input_scale, uint32_t tokens, uint32_t layers, uint32_t P,
                               int32_t* out, cudaStream_t s) {
  if (tokens == 0) return cudaSuccess;
  dim3 grid(tokens, layers);
  return launch_k(ple_prepare_kernel, grid, dim3(128), P * 4, s, projected, (const int8_t*)ple_embed->q,
                  (const uint16_t*)ple_embed->s, ple_embed->kc, ple_embed->nslices, d_ids, ple_norm, eps,
                  projection_scalar, embedding_scale, input_scale, layers, P, out);
}

}  // namespace iris
