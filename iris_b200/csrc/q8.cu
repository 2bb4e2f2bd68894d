// Exact Q8_0 x Q16.16 products on B200 (sm_100a).
//
// Every output equals det_num::q8::dot_row (crates/det-num/src/q8.rs:56-72):
// exact block sums, each times its Q.24 block scale, summed in 128 bits,
// rounded once to Q16.16 with ties to even and saturated. Here a block sum is
// formed from four byte planes with dp4a (common.cuh), multiplied by the
// scale's 11-bit mantissa (exact in int64) and added, shifted by the scale's
// exponent, into a 128-bit accumulator. Integer addition is associative, so
// the order in which lanes, warps or blocks combine partial sums never
// changes a value.
//
// Kernels:
//  - q8_gemv_tma_kernel: one token (the decode step). A persistent block an SM
//    streams whole weight tiles (q8.cuh) from HBM through a ring of
//    shared-memory stages with bulk copies (TMA) while sixteen consumer warps
//    run the products against activation planes held in shared memory and an
//    epilogue warp rounds and finishes the rows.
//  - q8_gemm_kernel: many tokens (prefill, the chain's ranges), a 64-row x
//    32-token tile per block staged through shared memory.
// Both end in a fused epilogue (residual add, RoPE and K/V store, SiLU/GELU
// gating, logits with a first-maximum key).
#include <cuda_runtime.h>

#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

#include "../../include/iris_b200.h"
#include "gemv.cuh"
#include "tc.cuh"
#include "q8.cuh"
#include "synth.cuh"

namespace iris {

// ---------------------------------------------------------------------------
// Layout: allocation, upload, download, synthesis
// ---------------------------------------------------------------------------

// Natural row-major int8 values and scale bits -> tiled layout.
__global__ void tile_from_natural_kernel(const int8_t* __restrict__ q_nat, const uint16_t* __restrict__ s_nat,
                                         uint32_t rows, uint32_t cols, uint32_t kc, uint32_t nslices, int8_t* q,
                                         uint16_t* s, int* bad) {
  const uint32_t nb = cols / 32;
  const uint64_t b = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= (uint64_t)rows * nb) return;
  const uint32_t r = (uint32_t)(b / nb), blk = (uint32_t)(b % nb);
  const uint16_t bits = s_nat[b];
  if (((bits >> 10) & 0x1f) == 0x1f) atomicExch(bad, 1);
  s[q8_scale_offset(kc, nslices, r, blk)] = bits;
  const uint4* src = (const uint4*)(q_nat + (size_t)r * cols + (size_t)blk * 32);
  uint4* dst = (uint4*)(q + q8_value_offset(kc, nslices, r, blk * 32));
  dst[0] = src[0];
  dst[1] = src[1];
}

// Raw 34-byte Q8_0 blocks -> rows (row_offset + i * row_stride) of the tiles.
__global__ void tile_from_blocks_kernel(const uint8_t* __restrict__ raw, uint32_t rows, uint32_t cols,
                                        uint32_t row_stride, uint32_t row_offset, uint32_t kc, uint32_t nslices,
                                        int8_t* q, uint16_t* s, int* bad) {
  const uint32_t nb = cols / 32;
  const uint64_t b = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= (uint64_t)rows * nb) return;
  const uint32_t r = (uint32_t)(b / nb), blk = (uint32_t)(b % nb);
  const uint8_t* src = raw + b * 34;
  const uint16_t bits = (uint16_t)(src[0] | (src[1] << 8));
  if (((bits >> 10) & 0x1f) == 0x1f) atomicExch(bad, 1);
  const uint32_t dr = r * row_stride + row_offset;
  s[q8_scale_offset(kc, nslices, dr, blk)] = bits;
  uint32_t w[8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
    w[i] = (uint32_t)src[2 + 4 * i] | ((uint32_t)src[3 + 4 * i] << 8) | ((uint32_t)src[4 + 4 * i] << 16) |
           ((uint32_t)src[5 + 4 * i] << 24);
  uint4* dst = (uint4*)(q + q8_value_offset(kc, nslices, dr, blk * 32));
  dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
  dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
}

__global__ void blocks_from_tile_kernel(const int8_t* q, const uint16_t* s, uint32_t kc, uint32_t nslices,
                                        uint32_t rows, uint32_t cols, uint32_t row_stride, uint32_t row_offset,
                                        uint8_t* raw) {
  const uint32_t nb = cols / 32;
  const uint64_t b = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= (uint64_t)rows * nb) return;
  const uint32_t r = (uint32_t)(b / nb), blk = (uint32_t)(b % nb);
  const uint32_t dr = r * row_stride + row_offset;
  const uint16_t bits = s[q8_scale_offset(kc, nslices, dr, blk)];
  uint8_t* dst = raw + b * 34;
  dst[0] = (uint8_t)bits;
  dst[1] = (uint8_t)(bits >> 8);
  const int8_t* src = q + q8_value_offset(kc, nslices, dr, blk * 32);
  for (int i = 0; i < 32; ++i) dst[2 + i] = (uint8_t)src[i];
}

// Rows [row0, row0 + rows) x columns [col0, col0 + cols) of the synthetic
// tensor with full_cols columns, into rows (i * row_stride + row_offset) of
// dst (a shard of a tensor-parallel model is such a block).
__global__ void synth_q8_kernel(int8_t* q, uint16_t* s, uint32_t kc, uint32_t nslices, uint64_t seed,
                                uint32_t tensor, int32_t layer, uint32_t rows, uint32_t cols, uint32_t row0,
                                uint32_t col0, uint32_t full_cols, uint32_t row_stride, uint32_t row_offset,
                                int per_block) {
  pdl_wait();
  pdl_trigger();
  const uint32_t nb = cols / 32;
  const uint64_t b = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= (uint64_t)rows * nb) return;
  const uint32_t r = (uint32_t)(b / nb), blk = (uint32_t)(b % nb);
  const uint32_t dr = r * row_stride + row_offset, sr = row0 + r, sblk = col0 / 32 + blk;
  s[q8_scale_offset(kc, nslices, dr, blk)] = synth_scale_bits(seed, tensor, layer, sr, sblk, full_cols, per_block);
  uint32_t w[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    uint32_t v = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j)
      v |= (uint32_t)(uint8_t)synth_q(seed, tensor, layer, sr, sblk * 32 + i * 4 + j, full_cols) << (8 * j);
    w[i] = v;
  }
  uint4* dst = (uint4*)(q + q8_value_offset(kc, nslices, dr, blk * 32));
  dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
  dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
}

__global__ void synth_values_kernel(int32_t* dst, uint64_t seed, uint32_t tensor, int32_t layer,
                                    uint64_t count, uint32_t fan_in) {
  uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < count) dst[i] = synth_value(seed, tensor, layer, i, fan_in);
}

Q8GpuMatrix* alloc_q8(uint32_t rows, uint32_t cols, cudaError_t* err) {
  Q8GpuMatrix* m = (Q8GpuMatrix*)std::calloc(1, sizeof(Q8GpuMatrix));
  if (!m) {
    *err = cudaErrorMemoryAllocation;
    return nullptr;
  }
  m->rows = rows;
  m->cols = cols;
  m->kc = q8_slice_cols(cols);
  m->nslices = cols / m->kc;
  m->groups = (rows + kQ8TileRows - 1) / kQ8TileRows;
  m->owns = true;
  const size_t padded = (size_t)m->groups * kQ8TileRows;
  *err = cudaMalloc((void**)&m->q, padded * cols);
  if (*err == cudaSuccess) *err = cudaMemset(m->q, 0, padded * cols);
  if (*err == cudaSuccess) *err = cudaMalloc((void**)&m->s, padded * (cols / 32) * 2);
  if (*err == cudaSuccess) *err = cudaMemset(m->s, 0, padded * (cols / 32) * 2);
  if (*err != cudaSuccess) {
    free_q8(m);
    return nullptr;
  }
  return m;
}

void free_q8(Q8GpuMatrix* m) {
  if (!m) return;
  if (m->owns) {
    cudaFree(m->q);
    cudaFree(m->s);
  }
  cudaFree(m->tc);
  cudaFree(m->tc_shift);
  cudaFree(m->tc_mant);
  std::free(m);
}

ProductArgs product_args(const Q8GpuMatrix* w, uint32_t tokens) {
  ProductArgs a{};
  a.q = w->q;
  a.s = w->s;
  a.rows = w->rows;
  a.cols = w->cols;
  a.kc = w->kc;
  a.nslices = w->nslices;
  a.tokens = tokens;
  if (tc_state_get(w) == 1) {
    a.tc = w->tc;
    a.tc_shift = w->tc_shift;
    a.tc_mant = w->tc_mant;
    a.tc_rows = w->tc_rows;
    a.tc_planes = w->tc_planes;
  }
  return a;
}

// Drops the tensor-core copy of a matrix whose weights change.
void tc_invalidate(Q8GpuMatrix* m) {
  cudaFree(m->tc);
  cudaFree(m->tc_shift);
  cudaFree(m->tc_mant);
  m->tc = nullptr;
  m->tc_shift = nullptr;
  m->tc_mant = nullptr;
  m->tc_rows = 0;
  m->tc_planes = 0;
  tc_state_set(m, 0);
  __atomic_add_fetch(&m->version, 1u, __ATOMIC_RELEASE);
}

namespace {
// One row a thread: flags[0] |= 1 when a row's blocks have different scale bits.
__global__ void rows_uniform_kernel(const uint16_t* __restrict__ s, uint32_t rows, uint32_t cols, uint32_t kc,
                                    uint32_t nslices, unsigned int* flags) {
  const uint32_t row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= rows) return;
  const uint16_t first = s[q8_scale_offset(kc, nslices, row, 0)];
  bool differ = false;
  for (uint32_t b = 1; b < cols / 32 && !differ; ++b) differ = s[q8_scale_offset(kc, nslices, row, b)] != first;
  if (differ) atomicOr(flags, 1u);
}
}  // namespace

cudaError_t q8_rows_uniform(const Q8GpuMatrix* m, cudaStream_t stream, bool* uniform) {
  *uniform = false;
  if (m->cols > 32768 || m->cols == 0 || m->rows == 0) return cudaSuccess;
  unsigned int* flags = nullptr;
  cudaError_t e = cudaMallocAsync((void**)&flags, sizeof(unsigned int), stream);
  if (e != cudaSuccess) return e;
  e = cudaMemsetAsync(flags, 0, sizeof(unsigned int), stream);
  if (e == cudaSuccess)
    e = launch_k(rows_uniform_kernel, dim3((m->rows + 255) / 256), dim3(256), 0, stream, m->s, m->rows, m->cols,
                 m->kc, m->nslices, flags);
  unsigned int h = 1;
  if (e == cudaSuccess) e = cudaMemcpyAsync(&h, flags, sizeof(h), cudaMemcpyDeviceToHost, stream);
  cudaError_t f = cudaFreeAsync(flags, stream);
  if (e == cudaSuccess) e = f;
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  if (e == cudaSuccess) *uniform = h == 0;
  return e;
}

bool q8_uniform_cached(Q8GpuMatrix* m, cudaStream_t stream) {
  const uint64_t v = q8_version(m);
  const uint64_t c = __atomic_load_n(&m->uniform_cache, __ATOMIC_ACQUIRE);
  if (c && (c >> 1) == v + 1) return (c & 1) != 0;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) {
    cudaGetLastError();
    return false;
  }
  bool u = false;
  // the weights may have been written on any stream
  if (cudaDeviceSynchronize() != cudaSuccess || q8_rows_uniform(m, stream, &u) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  __atomic_store_n(&m->uniform_cache, ((v + 1) << 1) | (u ? 1u : 0u), __ATOMIC_RELEASE);
  return u;
}

cudaError_t upload_q8_blocks(Q8GpuMatrix* dst, const uint8_t* host_blocks, uint32_t rows,
                             uint32_t cols, uint32_t row_stride, uint32_t row_offset,
                             int* bad_scale) {
  tc_invalidate(dst);
  size_t bytes = (size_t)rows * (cols / 32) * 34;
  uint8_t* staging = nullptr;
  int* bad = nullptr;
  cudaError_t e = cudaMalloc((void**)&staging, bytes);
  if (e == cudaSuccess) e = cudaMalloc((void**)&bad, sizeof(int));
  if (e == cudaSuccess) e = cudaMemset(bad, 0, sizeof(int));
  if (e == cudaSuccess) e = cudaMemcpy(staging, host_blocks, bytes, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) {
    uint64_t nblk = (uint64_t)rows * (cols / 32);
    tile_from_blocks_kernel<<<(unsigned)((nblk + 255) / 256), 256>>>(staging, rows, cols, row_stride, row_offset,
                                                                     dst->kc, dst->nslices, dst->q, dst->s, bad);
    e = cudaGetLastError();
  }
  int h_bad = 0;
  if (e == cudaSuccess) e = cudaMemcpy(&h_bad, bad, sizeof(int), cudaMemcpyDeviceToHost);
  cudaFree(staging);
  cudaFree(bad);
  *bad_scale = h_bad;
  return e;
}

cudaError_t download_q8_blocks(const Q8GpuMatrix* src, uint8_t* host_blocks, uint32_t rows,
                               uint32_t cols, uint32_t row_stride, uint32_t row_offset) {
  size_t bytes = (size_t)rows * (cols / 32) * 34;
  uint8_t* staging = nullptr;
  cudaError_t e = cudaMalloc((void**)&staging, bytes);
  if (e == cudaSuccess) {
    uint64_t nblk = (uint64_t)rows * (cols / 32);
    blocks_from_tile_kernel<<<(unsigned)((nblk + 255) / 256), 256>>>(src->q, src->s, src->kc, src->nslices, rows,
                                                                     cols, row_stride, row_offset, staging);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) e = cudaMemcpy(host_blocks, staging, bytes, cudaMemcpyDeviceToHost);
  cudaFree(staging);
  return e;
}

cudaError_t synth_q8_rows(Q8GpuMatrix* dst, uint64_t seed, uint32_t tensor, int32_t layer,
                          uint32_t rows, uint32_t cols, uint32_t row_stride, uint32_t row_offset,
                          int per_block, cudaStream_t stream) {
  return synth_q8_block(dst, seed, tensor, layer, rows, cols, 0, 0, cols, row_stride, row_offset, per_block, stream);
}

cudaError_t synth_q8_block(Q8GpuMatrix* dst, uint64_t seed, uint32_t tensor, int32_t layer, uint32_t rows,
                           uint32_t cols, uint32_t row0, uint32_t col0, uint32_t full_cols, uint32_t row_stride,
                           uint32_t row_offset, int per_block, cudaStream_t stream) {
  if (cols % 32 || col0 % 32) return cudaErrorInvalidValue;
  tc_invalidate(dst);
  uint64_t nblk = (uint64_t)rows * (cols / 32);
  if (nblk == 0) return cudaSuccess;
  return launch_k(synth_q8_kernel, dim3((unsigned)((nblk + 255) / 256)), dim3(256), 0, stream, dst->q, dst->s,
                  dst->kc, dst->nslices, seed, tensor, layer, rows, cols, row0, col0, full_cols, row_stride,
                  row_offset, per_block);
}

cudaError_t synth_values_dev(int32_t* dst, uint64_t seed, uint32_t tensor, int32_t layer,
                             uint64_t count, uint32_t fan_in, cudaStream_t stream) {
  if (count == 0) return cudaSuccess;
  synth_values_kernel<<<(unsigned)((count + 255) / 256), 256, 0, stream>>>(dst, seed, tensor, layer,
                                                                           count, fan_in);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Byte planes
// ---------------------------------------------------------------------------

__global__ void planes_kernel(const int32_t* __restrict__ x, const int32_t* __restrict__ norm_w,
                              int64_t eps, uint32_t K, uint8_t* planes) {
  pdl_wait();
  pdl_trigger();
  __shared__ uint64_t red[32];
  __shared__ int32_t s_scale;
  uint32_t t = blockIdx.x;
  row_to_planes(x + (size_t)t * K, norm_w, eps, K, planes + (size_t)t * 4 * K, red, &s_scale);
}

cudaError_t launch_planes(const int32_t* x, const int32_t* norm_w, int64_t eps, uint32_t tokens,
                          uint32_t cols, uint8_t* planes, cudaStream_t stream) {
  if (tokens == 0) return cudaSuccess;
  return launch_k(planes_kernel, dim3(tokens), dim3(256), 0, stream, x, norm_w, eps, cols, planes);
}

// ---------------------------------------------------------------------------
// Decode GEMV, bulk-copy pipeline: one persistent block an SM
// ---------------------------------------------------------------------------
//
// The matrix's tiles (16 rows x kc values, tile (g, s) at index g * S + s)
// are the work items. A block owns a contiguous range of items; three warp
// roles run concurrently:
//   - a producer warp streams every tile of the range - two contiguous runs,
//     values and scale bits - from HBM into a ring of shared-memory stages
//     with cp.async.bulk (TMA, evict-first in L2), completing on the stage's
//     "full" mbarrier;
//   - sixteen consumer warps - two rows and half of the slice's blocks each -
//     run the dp4a byte-plane products against the activation planes held in
//     shared memory (three planes when every activation fits in +-2^23, else
//     four), release the stage on its "empty" mbarrier and, at the end of a
//     tile group, leave their exact 128-bit row sums in a slot of a small
//     ring for
//   - an epilogue warp, which adds the two halves of each row, rounds once
//     (q8.rs:69-71) and applies the epilogue, off the consumers' path.
// With split scratch (stream-K), ranges are even item counts and may start
// or end inside a tile group: the blocks sharing a group add their partial
// 128-bit sums into the scratch with 64-bit atomics (wrapping 128-bit
// addition, exact in any order) and the block completing the group's slice
// count rounds it. Without it, ranges are whole tile groups.
// The activation prologue (planes, or the fused RMSNorm) runs once per block
// while the first stages are already in flight. Every wait is bounded (about
// one second): a stalled pipeline records a fault and the kernel returns
// instead of hanging.

__device__ unsigned int g_fault;

bool plan_gemv(uint32_t rows, uint32_t K, uint32_t kc, int sms, bool split, GemvPlan* p) {
  if (K % 32 || rows == 0 || kc == 0) return false;
  p->planes_bytes = round_up(4 * K, 128);
  p->stage_bytes = round_up(kQ8TileRows * kc + kc, 128);
  if (p->planes_bytes + 2 * p->stage_bytes > kTmaSmemBudget) return false;
  uint32_t fit = (kTmaSmemBudget - p->planes_bytes) / p->stage_bytes;
  p->stages = fit < kTmaMaxStages ? fit : kTmaMaxStages;
  p->smem = p->planes_bytes + p->stages * p->stage_bytes;
  const uint32_t groups = (rows + kQ8TileRows - 1) / kQ8TileRows;
  p->items = groups * (K / kc);
  // a lane adds one term a slice to each row: S terms below 2^(46.1 + e)
  // stay below 2^62 for e <= 15 - ceil(log2 S)
  const uint32_t S = K / kc;
  uint32_t lg = 0;
  while ((1u << lg) < S) ++lg;
  p->e_fast = 15 - (int32_t)lg;
  p->split = split ? 1 : 0;
  if (split) {
    p->grid = (uint32_t)sms < p->items ? (uint32_t)sms : p->items;
    p->groups_per_block = 0;
  } else {
    const uint32_t grid = (uint32_t)sms < groups ? (uint32_t)sms : groups;
    p->groups_per_block = (groups + grid - 1) / grid;
    p->grid = (groups + p->groups_per_block - 1) / p->groups_per_block;
  }
  return true;
}

// kUniform: every row of the matrix has one scale (ProductArgs::uniform):
// the consumers add plane sums over a tile group and scale each row once.
template <int IN, int EPI, bool kUniform>
__global__ void __launch_bounds__(kTmaThreads, 1) q8_gemv_tma_kernel(ProductArgs a, GemvPlan p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t full[kTmaMaxStages];
  __shared__ __align__(8) uint64_t empty[kTmaMaxStages];
  __shared__ __align__(8) uint64_t slot_full[kTmaSlots];
  __shared__ __align__(8) uint64_t slot_empty[kTmaSlots];
  __shared__ uint64_t red[32];
  __shared__ int32_t s_scale;
  __shared__ Acc128 slot_sums[kTmaSlots][2][kQ8TileRows];
  const uint32_t K = a.cols, kc = a.kc, S = a.nslices;
  uint8_t* planes = smem;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t groups = (a.rows + kQ8TileRows - 1) / kQ8TileRows;
  uint32_t ib, ie;
  gemv_range(p, S, groups, blockIdx.x, &ib, &ie);
  const TileRing ring{smem + p.planes_bytes, p.stage_bytes, p.stages, full, empty};
  const SumRing sums{slot_full, slot_empty, slot_sums};

  if (threadIdx.x == 0) {
    for (uint32_t st = 0; st < p.stages; ++st) {
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

  // Weights never change: the first tiles stream while the previous kernel
  // of the stream finishes; the activations are read only after pdl_wait().
  RingCursor pc{0, 1, 0};
  const uint64_t policy = l2_evict_first_policy();
  const uint32_t first = min(ie, ib + p.stages);
  if (warp == kTmaConsumerWarps && lane == 0) ring_issue<false>(ring, pc, a.q, a.s, kc, ib, first, policy, &g_fault);
  pdl_wait();
  pdl_trigger();

  // Activation planes; `wide` when some value needs the fourth plane.
  bool wide;
  if (IN == IN_PLANES) {
    const uint4* src = (const uint4*)a.planes;
    int w = 0;
    for (uint32_t i = threadIdx.x; i < K / 16; i += blockDim.x) {
      const uint4 v0 = __ldcg(src + i), v1 = __ldcg(src + K / 16 + i), v2 = __ldcg(src + 2 * (K / 16) + i),
                  v3 = __ldcg(src + 3 * (K / 16) + i);
      ((uint4*)planes)[i] = v0;
      ((uint4*)planes)[K / 16 + i] = v1;
      ((uint4*)planes)[2 * (K / 16) + i] = v2;
      ((uint4*)planes)[3 * (K / 16) + i] = v3;
      w |= !planes_sign_extended(v2.x, v3.x) | !planes_sign_extended(v2.y, v3.y) |
           !planes_sign_extended(v2.z, v3.z) | !planes_sign_extended(v2.w, v3.w);
    }
    wide = __syncthreads_or(w) != 0;
  } else if (IN == IN_POST_ATTN) {
    wide = post_attn_to_planes(a, K, planes, red, &s_scale);
  } else {
    wide = row_to_planes(a.x, IN == IN_NORM ? a.norm_w : nullptr, a.eps, K, planes, red, &s_scale);
  }

  uint32_t j = 0;
  if (warp == kTmaConsumerWarps) {
    if (lane == 0 && !ring_issue<false>(ring, pc, a.q, a.s, kc, first, ie, policy, &g_fault))
      ring_drain(ring, pc, &g_fault);  // let the copies already issued land before the block exits
  } else if (warp == kTmaEpilogueWarp) {
    ring_epilogue<EPI, false>(a, sums, j, ib, ie, S, &g_fault);
  } else {
    RingCursor cc{0, 0, 0};
    bool stalled = false;
    ring_consume_impl<false, kUniform>(ring, cc, sums, j, planes, wide, K, kc, S, p.e_fast, ib, ie, stalled,
                                       &g_fault);
  }
}

unsigned int* device_fault_word() {
  static unsigned int* addr[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  if (!addr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_fault) != cudaSuccess) return nullptr;
    addr[dev] = (unsigned int*)p;
  }
  return addr[dev];
}

cudaError_t take_device_fault(uint32_t* fault) {
  uint32_t zero = 0;
  cudaError_t e = cudaMemcpyFromSymbol(fault, g_fault, sizeof(uint32_t));
  if (e == cudaSuccess && *fault) e = cudaMemcpyToSymbol(g_fault, &zero, sizeof(uint32_t));
  return e;
}

// ---------------------------------------------------------------------------
// Tiled GEMM: 64 rows x 32 tokens a block, 4 rows x 2 tokens a thread
// ---------------------------------------------------------------------------

constexpr int kTileN = 64, kTileM = 32, kWPitch = 48;

template <int EPI>
__global__ void __launch_bounds__(256) q8_gemm_kernel(ProductArgs a) {
  pdl_wait();
  pdl_trigger();
  __shared__ __align__(16) uint8_t sw[kTileN * kWPitch];
  __shared__ uint16_t ssc[kTileN];
  __shared__ __align__(16) uint8_t sp[kTileM * 4 * 32];
  const uint32_t K = a.cols, nblk = K / 32;
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const uint32_t n0 = blockIdx.x * kTileN, m0 = blockIdx.y * kTileM;

  Acc128 acc[4][2];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 2; ++j) acc[i][j] = Acc128{0, 0};

  for (uint32_t kb = 0; kb < nblk; ++kb) {
    if (tid < 128) {
      int r = tid >> 1, h = tid & 1;
      uint32_t row = n0 + r;
      uint4 v = row < a.rows ? ld_stream_v4(a.q + q8_value_offset(a.kc, a.nslices, row, kb * 32) + h * 16)
                             : make_uint4(0, 0, 0, 0);
      *(uint4*)(sw + r * kWPitch + h * 16) = v;
    } else if (tid < 128 + kTileN) {
      int r = tid - 128;
      uint32_t row = n0 + r;
      ssc[r] = row < a.rows ? a.s[q8_scale_offset(a.kc, a.nslices, row, kb)] : (uint16_t)0;
    }
    {
      int t = tid >> 3, p = (tid >> 1) & 3, h = tid & 1;
      uint32_t tok = m0 + t;
      uint4 v = tok < a.tokens
                    ? *(const uint4*)(a.planes + (size_t)tok * 4 * K + (size_t)p * K + kb * 32 + h * 16)
                    : make_uint4(0, 0, 0, 0);
      *(uint4*)(sp + (t * 4 + p) * 32 + h * 16) = v;
    }
    __syncthreads();
    int32_t m[4], e[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (!q8_scale_parts(ssc[tx + 16 * i], &m[i], &e[i])) { m[i] = 0; e[i] = 0; }
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint4 w[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) w[i] = *(const uint4*)(sw + (tx + 16 * i) * kWPitch + h * 16);
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const uint8_t* pb = sp + (ty * 2 + j) * 128 + h * 16;
        uint4 p0 = *(const uint4*)(pb), p1 = *(const uint4*)(pb + 32), p2 = *(const uint4*)(pb + 64),
              p3 = *(const uint4*)(pb + 96);
#pragma unroll
        for (int i = 0; i < 4; ++i) acc128_add_shifted(acc[i][j], q8_partial16(w[i], p0, p1, p2, p3) * m[i], e[i]);
      }
    }
    __syncthreads();
  }

#pragma unroll
  for (int j = 0; j < 2; ++j) {
    uint32_t tok = m0 + ty * 2 + j;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint32_t row = n0 + tx + 16 * i;
      int32_t v = acc128_round_q24(acc[i][j]);
      if (EPI == EPI_PARTIAL) {
        if (tok < a.tokens && row < a.rows)
          limbs_from_acc128(acc[i][j].lo, acc[i][j].hi, a.partial + ((size_t)tok * a.rows + row) * 4);
      } else if (EPI == EPI_QKV_ROPE || EPI == EPI_SILU_MUL || EPI == EPI_GELU_MUL) {
        int32_t partner = __shfl_xor_sync(0xffffffffu, v, 1);
        if ((tx & 1) == 0 && tok < a.tokens && row + 1 < a.rows) epi_pair<EPI>(a, tok, row, v, partner);
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
  }
}

// ---------------------------------------------------------------------------
// Tiled GEMM on the tensor cores (mma.sync, int8): 128 rows x 16 tokens a block
// ---------------------------------------------------------------------------
//
// Eight warps, each 16 rows x 16 tokens (two 8-token tiles). A stage holds
// four 32-value blocks (128 columns) of the block's rows (weights and scale
// bits) and of its tokens' four activation planes, staged through a
// three-stage cp.async ring (16-byte pieces, XOR-swizzled by row so that the
// ldmatrix reads are free of bank conflicts). For every 32-value block and
// 8-token tile a warp runs four m16n8k32 MMAs (s8 weights against the u8
// planes 0-2 and the s8 plane 3), whose exact int32 results are the block's
// plane sums s0..s3 for each (row, token). The block sum is
// (s0 + 256 s1) + 2^16 (s2 + 256 s3); times the block's Q.24 scale m 2^e it
// is accumulated exactly:
//   - e <= 12: m 2^e fits 23 bits, so (s0 + 256 s1) m 2^e and
//     (s2 + 256 s3) m 2^e are 32 x 32 -> 64-bit multiply-adds into two int64
//     accumulators (weights 1 and 2^16) that cannot overflow for up to 2048
//     blocks (|term| < 2^51);
//   - larger exponents: the 64-bit product shifted into a 128-bit
//     accumulator.
// The three are added in 128 bits at the end and rounded once (q8.rs:69-71).

constexpr int kMmaRows = 128, kMmaTok = 16, kMmaKB = 4, kMmaStages = 3, kMmaThreads = 256;
constexpr int kMmaNT = kMmaTok / 8;  // 8-token tiles a warp
constexpr uint32_t kMmaAStage = kMmaRows * kMmaKB * 32;     // weight bytes a stage
constexpr uint32_t kMmaSStage = kMmaRows * kMmaKB * 2;      // scale bytes a stage
constexpr uint32_t kMmaBStage = kMmaTok * 4 * kMmaKB * 32;  // plane bytes a stage
constexpr uint32_t kMmaStageBytes = kMmaAStage + kMmaSStage + kMmaBStage;
constexpr uint32_t kMmaSmem = kMmaStages * kMmaStageBytes + kMmaRows * kMmaTok * sizeof(Acc128);
constexpr int32_t kMmaEFast = 12;

__device__ __forceinline__ void cp_async16_zfill(void* dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(dst)), "l"(src), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async8_zfill(void* dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(smem_addr(dst)), "l"(src), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void ldmatrix_x4(uint32_t* r, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_addr(p)));
}
// D = A (16x32 s8, rows) x B (32x8, columns), zero accumulator; B u8 or s8.
template <bool kSignedB>
__device__ __forceinline__ void mma_i8(int32_t* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  if (kSignedB)
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0));
  else
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0));
}

// The global offsets a thread copies from, split into a part fixed for the
// block (its rows and tokens) and a part that moves with the stage, so that a
// stage costs no divisions. A stage's four blocks lie in one slice.
struct MmaCopier {
  uint32_t a_row[4];  // value offset of piece i's row in slice 0, or ~0u outside the matrix
  uint32_t s_row;     // scale offset of the thread's row (threads < kMmaRows), or ~0u
  uint32_t b_tok[kMmaTok * 32 / kMmaThreads];  // plane offset of piece i's token at column 0, or ~0u
};

__device__ __forceinline__ void mma_copier_init(const ProductArgs& a, uint32_t n0, uint32_t m0, MmaCopier& cp) {
  const uint32_t tid = threadIdx.x, bps = a.kc / 32;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t row = n0 + ((tid + i * kMmaThreads) >> 3);
    cp.a_row[i] = row < a.rows ? (uint32_t)q8_value_offset(a.kc, a.nslices, row, 0) : ~0u;
  }
  cp.s_row = tid < kMmaRows && n0 + tid < a.rows ? (uint32_t)q8_scale_offset(a.kc, a.nslices, n0 + tid, 0) : ~0u;
  (void)bps;
#pragma unroll
  for (int i = 0; i < kMmaTok * 32 / kMmaThreads; ++i) {
    const uint32_t id = tid + i * kMmaThreads, tok = m0 + (id >> 5), pl = (id >> 3) & 3;
    cp.b_tok[i] = tok < a.tokens ? tok * 4 * a.cols + pl * a.cols : ~0u;
  }
}

// One stage: weights, scale bits and planes of blocks [kb0, kb0 + 4) of slice
// sl (block bi = kb0 - sl * kc / 32 within it).
__device__ __forceinline__ void mma_load_stage(const ProductArgs& a, const MmaCopier& cp, uint8_t* st, uint32_t kb0,
                                               uint32_t sl, uint32_t bi) {
  uint8_t* As = st;
  uint8_t* Ss = st + kMmaAStage;
  uint8_t* Bs = st + kMmaAStage + kMmaSStage;
  const uint32_t tid = threadIdx.x, c = tid & 7;
  const uint32_t a_stage = sl * kQ8TileRows * a.kc + bi * 32 + (c >> 1) * 32 + (c & 1) * 16;
#pragma unroll
  for (int i = 0; i < 4; ++i) {  // 128 rows x 8 pieces: row (tid >> 3) + 32 i, piece c
    const uint32_t row = (tid >> 3) + 32 * i;
    const bool ok = cp.a_row[i] != ~0u;
    cp_async16_zfill(As + row * 128 + ((c ^ (row & 7)) << 4), ok ? a.q + cp.a_row[i] + a_stage : a.q, ok ? 16u : 0u);
  }
  if (tid < kMmaRows) {
    const bool ok = cp.s_row != ~0u;
    const uint16_t* src = ok ? a.s + cp.s_row + sl * kQ8TileRows * (a.kc / 32) + bi : a.s;
    cp_async8_zfill(Ss + tid * 8, src, ok ? 8u : 0u);
  }
#pragma unroll
  for (int i = 0; i < kMmaTok * 32 / kMmaThreads; ++i) {  // tokens x 4 planes x 8 pieces
    const uint32_t id = tid + i * kMmaThreads, tok = id >> 5, pl = (id >> 3) & 3;
    const bool ok = cp.b_tok[i] != ~0u;
    cp_async16_zfill(Bs + (tok * 4 + pl) * 128 + ((c ^ (tok & 7)) << 4),
                     ok ? a.planes + cp.b_tok[i] + kb0 * 32 + c * 16 : a.planes, ok ? 16u : 0u);
  }
}

template <int EPI>
__global__ void __launch_bounds__(kMmaThreads, 2) q8_gemm_mma_kernel(ProductArgs a) {
  extern __shared__ __align__(128) uint8_t mma_smem[];
  // token tiles vary fastest, so the blocks sharing a weight tile run together (L2 reuse)
  const uint32_t n0 = blockIdx.y * kMmaRows, m0 = blockIdx.x * kMmaTok, nblk = a.cols / 32;
  const uint32_t nst = (nblk + kMmaKB - 1) / kMmaKB;
  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  pdl_wait();
  pdl_trigger();

  int64_t alo[kMmaNT][4], ahi[kMmaNT][4];  // [8-token tile][d index]: (g, 2t) (g, 2t+1) (g+8, 2t) (g+8, 2t+1)
#pragma unroll
  for (int nt = 0; nt < kMmaNT; ++nt)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      alo[nt][i] = 0;
      ahi[nt][i] = 0;
    }
  // 128-bit accumulators of the rare blocks with a scale exponent above
  // kMmaEFast: [row][token] of the block tile, each owned by one thread
  Acc128* slow_s = (Acc128*)(mma_smem + kMmaStages * kMmaStageBytes);
  for (uint32_t i = tid; i < kMmaRows * kMmaTok; i += kMmaThreads) slow_s[i] = Acc128{0, 0};
  bool any_slow_seen = false;

  MmaCopier cp;
  mma_copier_init(a, n0, m0, cp);
  const uint32_t bps = a.kc / 32;
  uint32_t ld_kb = 0, ld_sl = 0, ld_bi = 0;  // next stage to load: first block, its slice and place there
  auto load_next = [&](uint32_t buf) {
    mma_load_stage(a, cp, mma_smem + buf * kMmaStageBytes, ld_kb, ld_sl, ld_bi);
    ld_kb += kMmaKB;
    ld_bi += kMmaKB;
    if (ld_bi == bps) {
      ld_bi = 0;
      ++ld_sl;
    }
  };
#pragma unroll
  for (int s = 0; s < kMmaStages - 1; ++s) {
    if ((uint32_t)s < nst) load_next(s);
    cp_async_commit();
  }
  for (uint32_t st = 0; st < nst; ++st) {
    asm volatile("cp.async.wait_group %0;" ::"n"(kMmaStages - 2) : "memory");
    __syncthreads();  // stage st has landed for every thread; stage st - 1 is consumed
    {
      const uint32_t nx = st + kMmaStages - 1;
      if (nx < nst) load_next(nx % kMmaStages);
      cp_async_commit();
    }
    const uint8_t* As = mma_smem + (st % kMmaStages) * kMmaStageBytes;
    const uint16_t* Ss = (const uint16_t*)(As + kMmaAStage);
    const uint8_t* Bs = As + kMmaAStage + kMmaSStage;
#pragma unroll
    for (int kb = 0; kb < kMmaKB; ++kb) {
      uint32_t af[4];
      {
        const uint32_t row = 16 * warp + ((lane >> 3) & 1) * 8 + (lane & 7), c = 2 * kb + (lane >> 4);
        ldmatrix_x4(af, As + row * 128 + ((c ^ (row & 7)) << 4));
      }
      int32_t m[2], e[2], mp[2];
      bool fast[2];
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const uint16_t bits = Ss[(16 * warp + g + 8 * r) * 4 + kb];
        q8_scale_parts_finite(bits, &m[r], &e[r]);  // checked at upload (padding: 0)
        fast[r] = e[r] <= kMmaEFast;
        mp[r] = fast[r] ? m[r] * (1 << e[r]) : 0;  // 0: the block goes the 128-bit way
      }
      const bool any_slow = __any_sync(0xffffffffu, !fast[0] || !fast[1]);
#pragma unroll
      for (int nt = 0; nt < kMmaNT; ++nt) {
        uint32_t b01[4], b23[4];
        {
          const uint32_t j = lane >> 3, tok = 8 * nt + (lane & 7), c = 2 * kb + (j & 1);
          const uint32_t pl = j >> 1;
          ldmatrix_x4(b01, Bs + (tok * 4 + pl) * 128 + ((c ^ (tok & 7)) << 4));
          ldmatrix_x4(b23, Bs + (tok * 4 + 2 + pl) * 128 + ((c ^ (tok & 7)) << 4));
        }
        int32_t d0[4], d1[4], d2[4], d3[4];
        mma_i8<false>(d0, af, b01[0], b01[1]);
        mma_i8<false>(d1, af, b01[2], b01[3]);
        mma_i8<false>(d2, af, b23[0], b23[1]);
        mma_i8<true>(d3, af, b23[2], b23[3]);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int32_t lo = d0[i] + d1[i] * 256, hi = d2[i] + d3[i] * 256;
          mac_wide(alo[nt][i], lo, mp[i >> 1]);
          mac_wide(ahi[nt][i], hi, mp[i >> 1]);
        }
        if (any_slow) {  // rare: a scale exponent above kMmaEFast somewhere in the warp
          any_slow_seen = true;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int r = i >> 1;
            if (!fast[r]) {
              const int32_t lo = d0[i] + d1[i] * 256, hi = d2[i] + d3[i] * 256;
              const int64_t p = (int64_t)lo * m[r] + (int64_t)((uint64_t)((int64_t)hi * m[r]) << 16);
              Acc128& sa = slow_s[(16 * warp + g + 8 * r) * kMmaTok + 8 * nt + 2 * t + (i & 1)];
              acc128_add_shifted(sa, p, e[r]);
            }
          }
        }
      }
    }
  }

#pragma unroll
  for (int nt = 0; nt < kMmaNT; ++nt)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      Acc128 tot = any_slow_seen ? slow_s[(16 * warp + g + 8 * (i >> 1)) * kMmaTok + 8 * nt + 2 * t + (i & 1)]
                                 : Acc128{0, 0};
      acc128_add(tot, (uint64_t)alo[nt][i], alo[nt][i] >> 63);
      acc128_add(tot, (uint64_t)ahi[nt][i] << 16, ahi[nt][i] >> 48);
      int32_t v = acc128_round_q24(tot);
      const uint32_t row = n0 + 16 * warp + g + 8 * (i >> 1), tok = m0 + 8 * nt + 2 * t + (i & 1);
      if (EPI == EPI_PARTIAL) {
        if (tok < a.tokens && row < a.rows) limbs_from_acc128(tot.lo, tot.hi, a.partial + ((size_t)tok * a.rows + row) * 4);
      } else if (EPI == EPI_QKV_ROPE || EPI == EPI_SILU_MUL || EPI == EPI_GELU_MUL) {
        const int32_t partner = __shfl_xor_sync(0xffffffffu, v, 4);  // row ^ 1, same token
        if ((g & 1) == 0 && tok < a.tokens && row + 1 < a.rows) epi_pair<EPI>(a, tok, row, v, partner);
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
}

// ---------------------------------------------------------------------------
// Launchers
// ---------------------------------------------------------------------------

int g_sms = 0;  // multiprocessors of the current device

int device_sms() {
  if (g_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&g_sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || g_sms <= 0)
      g_sms = 148;
  }
  return g_sms;
}

template <int IN, int EPI>
cudaError_t launch_gemv(const ProductArgs& a, cudaStream_t stream) {
  GemvPlan p;
  const uint32_t groups = (a.rows + kQ8TileRows - 1) / kQ8TileRows;
  const bool split = a.split_acc && a.split_count && groups <= a.split_groups;
  if (!plan_gemv(a.rows, a.cols, a.kc, device_sms(), split, &p)) return cudaErrorInvalidValue;
  if (a.uniform)
    return launch_k(q8_gemv_tma_kernel<IN, EPI, true>, dim3(p.grid), dim3(kTmaThreads), p.smem, stream, a, p);
  return launch_k(q8_gemv_tma_kernel<IN, EPI, false>, dim3(p.grid), dim3(kTmaThreads), p.smem, stream, a, p);
}

template <int IN, int EPI>
cudaError_t prepare_gemv_one() {
  cudaError_t e = cudaFuncSetAttribute(q8_gemv_tma_kernel<IN, EPI, false>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTmaSmemBudget);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(q8_gemv_tma_kernel<IN, EPI, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)kTmaSmemBudget);
  return e;
}

template <int IN>
cudaError_t prepare_gemv_in() {
  cudaError_t e = prepare_gemv_one<IN, EPI_STORE>();
  if (e == cudaSuccess) e = prepare_gemv_one<IN, EPI_RESID>();
  if (e == cudaSuccess) e = prepare_gemv_one<IN, EPI_QKV_ROPE>();
  if (e == cudaSuccess) e = prepare_gemv_one<IN, EPI_SILU_MUL>();
  if (e == cudaSuccess) e = prepare_gemv_one<IN, EPI_GELU_MUL>();
  if (e == cudaSuccess) e = prepare_gemv_one<IN, EPI_LOGITS>();
  if (e == cudaSuccess) e = prepare_gemv_one<IN, EPI_PARTIAL>();
  return e;
}

template <int EPI>
cudaError_t prepare_mma_one() {
  return cudaFuncSetAttribute(q8_gemm_mma_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kMmaSmem);
}

cudaError_t prepare_product_kernels() {
  g_sms = 0;
  device_sms();
  {
    cudaError_t e = prepare_mma_one<EPI_STORE>();
    if (e == cudaSuccess) e = prepare_mma_one<EPI_RESID>();
    if (e == cudaSuccess) e = prepare_mma_one<EPI_QKV_ROPE>();
    if (e == cudaSuccess) e = prepare_mma_one<EPI_SILU_MUL>();
    if (e == cudaSuccess) e = prepare_mma_one<EPI_GELU_MUL>();
    if (e == cudaSuccess) e = prepare_mma_one<EPI_LOGITS>();
    if (e == cudaSuccess) e = prepare_mma_one<EPI_PARTIAL>();
    if (e != cudaSuccess) return e;
  }
  cudaError_t e = prepare_gemv_in<IN_PLANES>();
  if (e == cudaSuccess) e = prepare_gemv_in<IN_NORM>();
  if (e == cudaSuccess) e = prepare_gemv_in<IN_RAW>();
  if (e == cudaSuccess) e = prepare_gemv_one<IN_POST_ATTN, EPI_GELU_MUL>();
  if (e == cudaSuccess) e = prepare_tc_kernels();
  return e;
}

template <int EPI>
cudaError_t launch_gemm(const ProductArgs& a, cudaStream_t stream) {
  // the tensor-core GEMM: whole 4-block stages inside each slice, and at most
  // 2048 blocks a row for its 64-bit accumulators
  // (and 32-bit copy offsets)
  if (a.cols % (32 * kMmaKB) == 0 && (a.kc / 32) % kMmaKB == 0 && a.cols / 32 <= 2048 &&
      (uint64_t)((a.rows + 15) / 16 * 16) * a.cols < (1ull << 32) && (uint64_t)a.tokens * 4 * a.cols < (1ull << 32)) {
    dim3 grid((a.tokens + kMmaTok - 1) / kMmaTok, (a.rows + kMmaRows - 1) / kMmaRows);
    return launch_k(q8_gemm_mma_kernel<EPI>, grid, dim3(kMmaThreads), kMmaSmem, stream, a);
  }
  dim3 grid((a.rows + kTileN - 1) / kTileN, (a.tokens + kTileM - 1) / kTileM);
  return launch_k(q8_gemm_kernel<EPI>, grid, dim3(256), 0, stream, a);
}

template <int IN>
cudaError_t dispatch_gemv(const ProductArgs& a, EpiMode epi, cudaStream_t s) {
  switch (epi) {
    case EPI_STORE: return launch_gemv<IN, EPI_STORE>(a, s);
    case EPI_RESID: return launch_gemv<IN, EPI_RESID>(a, s);
    case EPI_QKV_ROPE: return launch_gemv<IN, EPI_QKV_ROPE>(a, s);
    case EPI_SILU_MUL: return launch_gemv<IN, EPI_SILU_MUL>(a, s);
    case EPI_GELU_MUL: return launch_gemv<IN, EPI_GELU_MUL>(a, s);
    case EPI_LOGITS: return launch_gemv<IN, EPI_LOGITS>(a, s);
    case EPI_PARTIAL: return launch_gemv<IN, EPI_PARTIAL>(a, s);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_product(const ProductArgs& a0, InMode in, EpiMode epi, cudaStream_t stream,
                           int path) {
  ProductArgs a = a0;
  if (a.out_stride == 0) a.out_stride = a.rows;
  if (a.tokens == 0 || a.rows == 0) return cudaSuccess;
  if (a.cols == 0 || a.cols % 32 || a.kc == 0) return cudaErrorInvalidValue;
  const bool tc_path = path == IRIS_PATH_TC || path == IRIS_PATH_TC3;
  bool gemv = (a.tokens == 1 && path != IRIS_PATH_GEMM && !tc_path) || path == IRIS_PATH_GEMV;
  if (gemv) {
    if (a.tokens != 1) return cudaErrorInvalidValue;
    switch (in) {
      case IN_PLANES: return dispatch_gemv<IN_PLANES>(a, epi, stream);
      case IN_NORM: return dispatch_gemv<IN_NORM>(a, epi, stream);
      case IN_RAW: return dispatch_gemv<IN_RAW>(a, epi, stream);
      case IN_POST_ATTN:
        static_assert(kPostAttnMaxCols == 2 * 4 * kTmaThreads, "IN_POST_ATTN holds two int4 a thread");
        if (epi != EPI_GELU_MUL || a.cols > kPostAttnMaxCols) return cudaErrorInvalidValue;
        return launch_gemv<IN_POST_ATTN, EPI_GELU_MUL>(a, stream);
    }
    return cudaErrorInvalidValue;
  }
  if (in != IN_PLANES) return cudaErrorInvalidValue;  // callers build planes first
  if (path == IRIS_PATH_TC3 && a.tc_planes != 3) return cudaErrorInvalidValue;
  if (tc_path || (path == IRIS_PATH_AUTO && a.tokens >= kTcMinTokens && tc_usable(a)))
    return launch_gemm_tc(a, epi, stream);
  switch (epi) {
    case EPI_STORE: return launch_gemm<EPI_STORE>(a, stream);
    case EPI_RESID: return launch_gemm<EPI_RESID>(a, stream);
    case EPI_QKV_ROPE: return launch_gemm<EPI_QKV_ROPE>(a, stream);
    case EPI_SILU_MUL: return launch_gemm<EPI_SILU_MUL>(a, stream);
    case EPI_GELU_MUL: return launch_gemm<EPI_GELU_MUL>(a, stream);
    case EPI_LOGITS: return launch_gemm<EPI_LOGITS>(a, stream);
    case EPI_PARTIAL: return launch_gemm<EPI_PARTIAL>(a, stream);
  }
  return cudaErrorInvalidValue;
}

}  // namespace iris

// ===========================================================================
// C ABI: the reference's q8gpu_* (drop-in) and the device-pointer products
// ===========================================================================

using namespace iris;

namespace {
std::mutex g_product_mutex;  // the drop-in's scratch buffers (one product at a time, as gpu.rs)
int32_t* g_act = nullptr;
int32_t* g_out = nullptr;
uint8_t* g_planes = nullptr;
size_t g_act_bytes = 0, g_out_bytes = 0, g_planes_bytes = 0;

template <class T>
cudaError_t reserve(T** buf, size_t* cap, size_t bytes) {
  if (bytes <= *cap) return cudaSuccess;
  cudaFree(*buf);
  *buf = nullptr;
  *cap = 0;
  cudaError_t e = cudaMalloc((void**)buf, bytes);
  if (e == cudaSuccess) *cap = bytes;
  return e;
}

// Builds the matrix's tensor-core copy the first time a product that may use
// it runs (many tokens on the automatic path, or the tensor-core path asked
// for). The copy is a cache of the weights: the matrix stays logically const.
cudaError_t prepare_tc_for(const Q8GpuMatrix* m, uint32_t tokens, int path, cudaStream_t s) {
  if (tc_state_get(m) != 0) return cudaSuccess;
  if (path == IRIS_PATH_TC3) return tc_prepare(const_cast<Q8GpuMatrix*>(m), s, 3);
  if (path == IRIS_PATH_TC || (path == IRIS_PATH_AUTO && tokens >= kTcMinTokens))
    return tc_prepare(const_cast<Q8GpuMatrix*>(m), s);
  return cudaSuccess;
}

// The fp16 bits whose exact Q.24 value is v (inverse of q8.rs:27-43).
bool q24_to_half_bits(int64_t v, uint16_t* bits) {
  uint16_t sign = v < 0 ? 0x8000 : 0;
  uint64_t mag = v < 0 ? (uint64_t)0 - (uint64_t)v : (uint64_t)v;
  if (mag < 1024) {  // subnormal (or zero)
    *bits = sign | (uint16_t)mag;
    return true;
  }
  for (uint32_t ex = 1; ex <= 30; ++ex) {
    uint64_t unit = (uint64_t)1 << (ex - 1);
    if (mag % unit) return false;
    uint64_t m = mag / unit;
    if (m >= 1024 && m <= 2047) {
      *bits = sign | (uint16_t)(ex << 10) | (uint16_t)(m - 1024);
      return true;
    }
  }
  return false;
}
}  // namespace

extern "C" {

const char* iris_error(int code) {
  switch (code) {
    case 0: return "no error";
    case IRIS_EINVAL: return "iris: invalid argument or shape";
    case IRIS_ESCALE: return "iris: Q8_0 block scale is not finite";
    case IRIS_ERANGE: return "iris: position out of range";
    case IRIS_ESTATE: return "iris: call out of order";
    case IRIS_EWINDOW: return "iris: attention window not covered by the keys";
    case IRIS_ESTALL: return "iris: a kernel gave up a bounded wait (stalled pipeline)";
    case IRIS_ESCRATCH:
      return "iris: input larger than the fixed no-alloc scratch (tokens * cols * 4 must be <= 16 MiB)";
    default: return cudaGetErrorString((cudaError_t)code);
  }
}

const char* q8gpu_error(int code) { return iris_error(code); }

int q8gpu_init(void) {
  void* probe = nullptr;
  cudaError_t e = cudaMalloc(&probe, 1 << 20);
  if (e != cudaSuccess) return (int)e;
  e = cudaFree(probe);
  if (e == cudaSuccess) e = prepare_product_kernels();
  return (int)e;
}

void q8gpu_free(Q8GpuMatrix* matrix) { free_q8(matrix); }

int q8gpu_upload(const int8_t* weights, const int64_t* scales_q24, uint32_t rows, uint32_t cols,
                 Q8GpuMatrix** out_matrix) {
  *out_matrix = nullptr;
  if (rows == 0 || cols == 0 || cols % 32) return IRIS_EINVAL;
  size_t nblk = (size_t)rows * (cols / 32);
  std::vector<uint16_t> bits(nblk);
  for (size_t i = 0; i < nblk; ++i)
    if (!q24_to_half_bits(scales_q24[i], &bits[i])) return IRIS_ESCALE;
  cudaError_t e;
  Q8GpuMatrix* m = alloc_q8(rows, cols, &e);
  if (!m) return (int)e;
  int8_t* q_nat = nullptr;
  uint16_t* s_nat = nullptr;
  int* bad = nullptr;
  e = cudaMalloc((void**)&q_nat, (size_t)rows * cols);
  if (e == cudaSuccess) e = cudaMalloc((void**)&s_nat, nblk * 2);
  if (e == cudaSuccess) e = cudaMalloc((void**)&bad, sizeof(int));
  if (e == cudaSuccess) e = cudaMemset(bad, 0, sizeof(int));
  if (e == cudaSuccess) e = cudaMemcpy(q_nat, weights, (size_t)rows * cols, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(s_nat, bits.data(), nblk * 2, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) {
    tile_from_natural_kernel<<<(unsigned)((nblk + 255) / 256), 256>>>(q_nat, s_nat, rows, cols, m->kc, m->nslices,
                                                                      m->q, m->s, bad);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaFree(q_nat);
  cudaFree(s_nat);
  cudaFree(bad);
  if (e != cudaSuccess) {
    free_q8(m);
    return (int)e;
  }
  *out_matrix = m;
  return 0;
}

int iris_q8_upload_blocks(const uint8_t* blocks, uint32_t rows, uint32_t cols,
                          Q8GpuMatrix** out_matrix) {
  *out_matrix = nullptr;
  if (rows == 0 || cols == 0 || cols % 32) return IRIS_EINVAL;
  cudaError_t e;
  Q8GpuMatrix* m = alloc_q8(rows, cols, &e);
  if (!m) return (int)e;
  int bad = 0;
  e = upload_q8_blocks(m, blocks, rows, cols, 1, 0, &bad);
  if (e != cudaSuccess || bad) {
    free_q8(m);
    return e != cudaSuccess ? (int)e : IRIS_ESCALE;
  }
  *out_matrix = m;
  return 0;
}

int iris_q8_product_device_path(const Q8GpuMatrix* m, const int32_t* d_act, uint32_t tokens,
                                int32_t* d_out, void* stream, int path) {
  if (!m || tokens == 0) return tokens == 0 ? 0 : IRIS_EINVAL;
  if (path < IRIS_PATH_AUTO || path > IRIS_PATH_GEMV1) return IRIS_EINVAL;
  cudaStream_t s = (cudaStream_t)stream;
  bool gemv = (tokens == 1 && path != IRIS_PATH_GEMM && path != IRIS_PATH_TC && path != IRIS_PATH_TC3) ||
              path == IRIS_PATH_GEMV || path == IRIS_PATH_GEMV1;
  if (gemv) {
    ProductArgs a = product_args(m, tokens);
    a.out = d_out;
    a.x = d_act;
    if (path == IRIS_PATH_GEMV1) {
      if (tokens != 1 || !q8_uniform_cached(const_cast<Q8GpuMatrix*>(m), s)) return (int)cudaErrorInvalidValue;
      a.uniform = 1;
    }
    return (int)launch_product(a, IN_RAW, EPI_STORE, s, IRIS_PATH_GEMV);
  }
  cudaError_t e = prepare_tc_for(m, tokens, path, s);
  if (e != cudaSuccess) return (int)e;
  ProductArgs a = product_args(m, tokens);
  a.out = d_out;
  // The tiled GEMMs read byte planes: build them into the shared scratch.
  std::lock_guard<std::mutex> lock(g_product_mutex);
  e = reserve(&g_planes, &g_planes_bytes, (size_t)tokens * m->cols * 4);
  if (e == cudaSuccess) e = launch_planes(d_act, nullptr, 0, tokens, m->cols, g_planes, s);
  a.planes = g_planes;
  if (e == cudaSuccess) e = launch_product(a, IN_PLANES, EPI_STORE, s, path);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);  // scratch is reused by the next call
  return (int)e;
}

int iris_q8_product_device(const Q8GpuMatrix* m, const int32_t* d_act, uint32_t tokens,
                           int32_t* d_out, void* stream) {
  return iris_q8_product_device_path(m, d_act, tokens, d_out, stream, IRIS_PATH_AUTO);
}

// ---- the product without allocation -----------------------------------------
//
// The byte planes of the GEMM path live in a fixed device array instead of
// the grown-on-demand scratch above. Its address is looked up once per device
// (cudaGetSymbolAddress with that device current) by the first call made on
// it. Every byte a call reads is written earlier in the same call, so nothing
// needs to start at zero. Calls in flight at the same time on one device
// (other streams, other host threads) share the array and race; calls queued
// on one stream are ordered and do not.
constexpr size_t kNoAllocPlanesBytes = (size_t)16 << 20;  // tokens * cols * 4 at most
static __device__ __align__(256) uint8_t g_noalloc_planes[kNoAllocPlanesBytes];
constexpr int kNoAllocMaxDevices = 64;
static std::mutex g_noalloc_mutex;
static uint8_t* g_noalloc_addr[kNoAllocMaxDevices];

static cudaError_t noalloc_planes(uint8_t** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kNoAllocMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (!g_noalloc_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_planes);
    if (e != cudaSuccess) return e;
    g_noalloc_addr[dev] = (uint8_t*)p;
  }
  *out = g_noalloc_addr[dev];
  return cudaSuccess;
}

int iris_q8_product_device_noalloc(const Q8GpuMatrix* m, const int32_t* d_act, uint32_t tokens,
                                   int32_t* d_out, void* stream) {
  if (!m) return IRIS_EINVAL;
  if (tokens > 1 && (uint64_t)tokens * m->cols * 4 > kNoAllocPlanesBytes) return IRIS_ESCRATCH;
  uint8_t* planes = nullptr;
  cudaError_t e = noalloc_planes(&planes);
  if (e != cudaSuccess || tokens == 0) return (int)e;
  cudaStream_t s = (cudaStream_t)stream;
  ProductArgs a = product_args(m, tokens);
  a.out = d_out;
  if (tokens == 1) {
    a.x = d_act;
    return (int)launch_product(a, IN_RAW, EPI_STORE, s, IRIS_PATH_GEMV);
  }
  e = launch_planes(d_act, nullptr, 0, tokens, m->cols, planes, s);
  a.planes = planes;  // the tensor-core GEMM when its copy is already built
  if (e == cudaSuccess) e = launch_product(a, IN_PLANES, EPI_STORE, s, IRIS_PATH_AUTO);
  return (int)e;
}

int q8gpu_product(const Q8GpuMatrix* m, const int32_t* activations, uint32_t tokens, int32_t* out) {
  if (!m) return IRIS_EINVAL;
  if (tokens == 0) return 0;
  size_t act_bytes = (size_t)tokens * m->cols * 4, out_bytes = (size_t)tokens * m->rows * 4;
  std::lock_guard<std::mutex> lock(g_product_mutex);
  cudaError_t e = reserve(&g_act, &g_act_bytes, act_bytes);
  if (e == cudaSuccess) e = reserve(&g_out, &g_out_bytes, out_bytes);
  if (e == cudaSuccess && tokens > 1) e = reserve(&g_planes, &g_planes_bytes, act_bytes);
  if (e == cudaSuccess) e = cudaMemcpy(g_act, activations, act_bytes, cudaMemcpyHostToDevice);
  if (e == cudaSuccess && tokens > 1) e = prepare_tc_for(m, tokens, IRIS_PATH_AUTO, 0);
  if (e != cudaSuccess) return (int)e;
  ProductArgs a = product_args(m, tokens);
  a.out = g_out;
  if (tokens == 1) {
    a.x = g_act;
    e = launch_product(a, IN_RAW, EPI_STORE, 0, IRIS_PATH_GEMV);
  } else {
    e = launch_planes(g_act, nullptr, 0, tokens, m->cols, g_planes, 0);
    a.planes = g_planes;
    if (e == cudaSuccess) e = launch_product(a, IN_PLANES, EPI_STORE, 0, IRIS_PATH_AUTO);
  }
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpy(out, g_out, out_bytes, cudaMemcpyDeviceToHost);
  return (int)e;
}

int iris_synth_q8_block(uint64_t seed, uint32_t tensor, int32_t layer, uint32_t rows, uint32_t cols, uint32_t row0,
                        uint32_t col0, uint32_t full_cols, int per_block_scales, uint8_t* blocks) {
  if (cols == 0 || cols % 32 || col0 % 32 || (uint64_t)col0 + cols > full_cols) return IRIS_EINVAL;
  uint32_t nb = cols / 32;
  for (uint32_t r = 0; r < rows; ++r)
    for (uint32_t b = 0; b < nb; ++b) {
      uint8_t* dst = blocks + ((size_t)r * nb + b) * 34;
      const uint32_t sr = row0 + r, sb = col0 / 32 + b;
      uint16_t bits = synth_scale_bits(seed, tensor, layer, sr, sb, full_cols, per_block_scales);
      dst[0] = (uint8_t)bits;
      dst[1] = (uint8_t)(bits >> 8);
      for (uint32_t j = 0; j < 32; ++j)
        dst[2 + j] = (uint8_t)synth_q(seed, tensor, layer, sr, sb * 32 + j, full_cols);
    }
  return 0;
}

int iris_synth_q8(uint64_t seed, uint32_t tensor, int32_t layer, uint32_t rows, uint32_t cols,
                  int per_block_scales, uint8_t* blocks) {
  if (cols == 0 || cols % 32) return IRIS_EINVAL;
  uint32_t nb = cols / 32;
  for (uint32_t r = 0; r < rows; ++r)
    for (uint32_t b = 0; b < nb; ++b) {
      uint8_t* dst = blocks + ((size_t)r * nb + b) * 34;
      uint16_t bits = synth_scale_bits(seed, tensor, layer, r, b, cols, per_block_scales);
      dst[0] = (uint8_t)bits;
      dst[1] = (uint8_t)(bits >> 8);
      for (uint32_t j = 0; j < 32; ++j) dst[2 + j] = (uint8_t)synth_q(seed, tensor, layer, r, b * 32 + j, cols);
    }
  return 0;
}

int iris_synth_values(uint64_t seed, uint32_t tensor, int32_t layer, uint64_t count, uint32_t fan_in,
                      int32_t* values) {
  for (uint64_t i = 0; i < count; ++i) values[i] = synth_value(seed, tensor, layer, i, fan_in);
  return 0;
}

}  // extern "C"
