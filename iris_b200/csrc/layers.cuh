// Row-level kernels of the two layer families: attention, embeddings, norms,
// Gemma's q/k/v finishing and per-layer inputs, the head's selection.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "q8.cuh"

namespace iris {

enum ScoreMode { SCORE_MISTRAL = 0, SCORE_GEMMA = 1 };

// Attention over a linear K/V cache ([positions][kv_dim] int32 per layer).
struct AttnArgs {
  const int32_t* q;       // [tokens][heads*d]
  const int32_t* kcache;  // [positions][kvd]
  const int32_t* vcache;
  uint32_t heads, kv_heads, d, kvd;
  const uint32_t* pos_ptr;  // position of token 0 (decode), or NULL
  uint32_t pos0;
  uint32_t window;          // 0 = full causal attention
  int mode;                 // ScoreMode
  uint32_t scale_q32;       // mistral score scale
  uint8_t* ctx_planes;      // [tokens][4][heads*d]
  int32_t* ctx;             // [tokens][heads*d] or NULL
  // decode split scratch
  int32_t* scores;                 // [heads][cap]
  int64_t* terms;                  // [heads][cap]
  unsigned long long* chunk_best;  // [heads][nchunks]
  uint64_t* chunk_sum;             // [heads][nchunks]
  int32_t* wsum;                   // [heads], zero between launches
  int64_t* acc;                    // [heads][d], zero between launches
  unsigned int* counters;          // [heads], zero between launches
  uint32_t cap, nchunks;           // positions held; chunks of 64 positions
  uint32_t hpc;                    // query heads a block (attention_hpc)
  // one-launch decode (attention_cluster_plan): blocks a cluster (0 = the
  // three-launch path), query heads a block, positions a block at most
  // (even), tile buffers a block
  uint32_t cluster, chpc, span, ring;
  // one-launch decode over the whole GPU (attention_grid_plan): blocks a head
  // group (0 = not used), positions a block at most (even), the group
  // exchange words (zero between launches) and the fault word
  uint32_t chunks, ghpc, gspan;
  unsigned long long* gbest;  // [heads] first-maximum keys
  unsigned long long* gsum;   // [heads] sums of exp terms
  unsigned int* gbar;         // [2 * heads]: arrivals, then finished blocks, a head group
  unsigned int* fault;
};

// Query heads a decode-attention block handles, and the chunk count for a
// cache of `cap` positions (sizes of the scratch arrays above).
uint32_t attention_hpc(uint32_t heads, uint32_t kv_heads);
uint32_t attention_chunks(uint32_t cap);
// The one-launch (thread-block cluster) decode attention for a cache of `cap`
// positions: query heads a block, blocks a cluster (0 when the shape needs
// the three-launch path), positions a block at most and tile buffers a block.
void attention_cluster_plan(uint32_t heads, uint32_t kv_heads, uint32_t d, uint32_t cap, uint32_t* hpc,
                            uint32_t* cluster, uint32_t* span, uint32_t* ring);

// The whole-GPU decode attention for a cache of `cap` positions: query heads
// a block, blocks a head group (0 when the shape or capacity needs another
// path) and positions a block at most.
void attention_grid_plan(uint32_t heads, uint32_t kv_heads, uint32_t d, uint32_t cap, uint32_t* hpc,
                         uint32_t* chunks, uint32_t* span);

// Checks an explicit one-launch shape (blocks a cluster, query heads a block,
// tile buffers a block) for the model and capacity; sets *span.
bool attention_cluster_shape_ok(uint32_t heads, uint32_t kv_heads, uint32_t d, uint32_t cap, uint32_t cluster,
                                uint32_t hpc, uint32_t ring, uint32_t* span);

// Decode (one query): one cluster launch when a.cluster is set, else three
// launches split over kv groups x position chunks.
cudaError_t launch_attention_decode(const AttnArgs& a, cudaStream_t s);
// Many queries at positions pos0.. (prefill, chain ranges): one block a
// (query, head). max_visible bounds the shared memory.
// Scratch of the tensor-core prefill attention (attn_tc.cu), carved from one
// allocation sized for pcap positions (a multiple of 128) and qcap queries (a
// multiple of 64): scores [heads][qcap][pcap] int32, weight planes
// [heads][3][qcap][pcap], key planes [kv_heads][4][pcap][128], transposed
// value planes [kv_heads][4][128][pcap], query planes [heads][4][qcap][128].
struct AttnTcScratch {
  int32_t* s = nullptr;
  uint8_t *wp = nullptr, *kp = nullptr, *vt = nullptr, *qp = nullptr;
  uint32_t pcap = 0, qcap = 0;
};
size_t attn_tc_scratch_bytes(uint32_t heads, uint32_t kv_heads, uint32_t pcap, uint32_t qcap);
void attn_tc_scratch_carve(uint8_t* base, uint32_t heads, uint32_t kv_heads, uint32_t pcap, uint32_t qcap,
                           AttnTcScratch* sc);
// Whether the tensor-core path takes this range: head_dim 128, no sliding
// window cutting the prefix, at most 22,016 positions and the scratch's.
bool attn_tc_usable(const AttnArgs& a, uint32_t tokens, const AttnTcScratch& sc);
cudaError_t launch_attention_prefill_tc(const AttnArgs& a, uint32_t tokens, const AttnTcScratch& sc,
                                        cudaStream_t stream);
cudaError_t prepare_attn_tc_kernels();
// The device's table of softmax exp terms (filled on first use): entry i
// (1 <= i < kExpTerms) is softmax_exp_term at distance -i (Q16.16) below the
// maximum; distances of kExpTerms or more give 0, distance 0 gives 2^32.
constexpr uint32_t kExpTerms = 1u << 20;
cudaError_t exp_term_table(const uint32_t** table);
cudaError_t launch_attention_prefill(const AttnArgs& a, uint32_t tokens, uint32_t max_visible,
                                     cudaStream_t s);

// Embedding rows: out[t] = dequantize_row(embed[ids[t]]), then mul_sat by
// scale when has_scale (Gemma, direct/src/model.rs:316-330).
cudaError_t launch_embed(const Q8GpuMatrix* embed, const uint32_t* d_ids, uint32_t tokens,
                         int has_scale, int32_t scale, int32_t* out, cudaStream_t s);
// Sets the shared-memory limits of every kernel instantiation (call once per
// device before any launch or stream capture).
cudaError_t prepare_layer_kernels();
cudaError_t prepare_product_kernels();

// Resets first-maximum keys.
cudaError_t launch_fill_u64(unsigned long long* p, uint32_t n, cudaStream_t s);
// Decode bookkeeping after the head: token = argmax, pos += 1, history.
cudaError_t launch_decode_finish(const unsigned long long* best, uint32_t* d_token, uint32_t* d_pos,
                                 uint32_t* d_step, uint32_t* history, uint32_t history_cap,
                                 cudaStream_t s);

// Gemma: per-head RMSNorm (q_norm/k_norm, weightless for v), rotate-half RoPE,
// q to q_out, k and v to the cache (when kcache is not NULL).
struct QkvFinishArgs {
  const int32_t* qkv;  // [tokens][qd + 2 kvd]
  int32_t* q_out;      // [tokens][qd]
  int32_t* kcache;
  int32_t* vcache;
  const int32_t* q_norm;
  const int32_t* k_norm;
  const int64_t* inv_freq;  // [rotary_dim/2]
  uint32_t heads, kv_heads, d, rotary_dim;
  int64_t eps;
  const uint32_t* pos_ptr;
  uint32_t pos0;
};
cudaError_t launch_gemma_qkv_finish(const QkvFinishArgs& a, uint32_t tokens, cudaStream_t s);

// Gemma residual steps (prefill_range.rs:879-957), one block a token:
//   post_attn: x = add_sat(rms_norm(o, w_post_attn), x); planes = rms_norm(x, w_pre_ffw)
//   post_ffw:  xs = add_sat(rms_norm(ff, w_post_ffw), x)
//   finish:    x = [layer_scalar *] add_sat(rms_norm(proj, w_ple_post), xs)
cudaError_t launch_gemma_post_attn(const int32_t* o, int32_t* x, const int32_t* w_post_attn,
                                   const int32_t* w_pre_ffw, int64_t eps, uint32_t tokens,
                                   uint32_t hidden, uint8_t* planes, cudaStream_t s);
cudaError_t launch_gemma_post_ffw(const int32_t* ff, const int32_t* x, const int32_t* w_post_ffw,
                                  int64_t eps, uint32_t tokens, uint32_t hidden, int32_t* xs,
                                  cudaStream_t s);
cudaError_t launch_gemma_finish(const int32_t* proj, const int32_t* xs, const int32_t* w_ple_post,
                                int64_t eps, int32_t layer_scalar, uint32_t tokens, uint32_t hidden,
                                int32_t* x_out, cudaStream_t s);
// The gemma norm kernels hold a row of at most kNormPer * kNormThreads values
// in registers (larger rows go through shared memory).
constexpr uint32_t kNormPer = 8;
constexpr uint32_t kNormThreads = 256;
// One token: post_ffw and the PLE gate product in one launch. Every block
// computes xs = add_sat(rms_norm(ff, w_post_ffw), x) itself (block 0 also
// stores it), then its rows of pg = mul_sat(gelu(dot_bits(xs, w_gate[r])),
// gate_rows[r]). hidden <= 2048 (kNormPer * kNormThreads), else refused
// with cudaErrorInvalidValue (the two-launch path serves it).
cudaError_t launch_gemma_post_ffw_ple_gate(const int32_t* ff, const int32_t* x, const int32_t* w_post_ffw,
                                          int64_t eps, uint32_t hidden, int32_t* xs, const int32_t* w_gate,
                                          uint32_t P, const int32_t* gate_rows, int32_t* pg, cudaStream_t s);
// One token: the PLE projection and the layer finish in one launch. Each
// warp writes rows proj[r] = dot_bits(pg, w_proj[r]); the block that
// completes the row (the last to add to *done, which it clears again) then
// writes x = [layer_scalar *] add_sat(rms_norm(proj, w_ple_post), xs).
// hidden <= kNormPer * kNormThreads, else refused with cudaErrorInvalidValue.
cudaError_t launch_gemma_ple_proj_finish(const int32_t* pg, const int32_t* w_proj, uint32_t P, uint32_t hidden,
                                         int32_t* proj, const int32_t* xs, const int32_t* w_ple_post, int64_t eps,
                                         int32_t layer_scalar, int32_t* x_out, unsigned int* done,
                                         cudaStream_t s);
// The Q2.30 sine and cosine (sin_cos_q30, mistral.rs:84-110) of each of
// `half` inverse frequencies at the positions of `tokens` tokens from
// (*pos_ptr or pos0): out[t][i][0..1], for the many-token q|k|v epilogue.
cudaError_t launch_rope_table(const int64_t* freqs, uint32_t half, const uint32_t* pos_ptr, uint32_t pos0,
                              uint32_t tokens, int64_t* out, cudaStream_t s);
// Dense Q16.16 products: out[t][r] = dot_bits(in[t], w[r]) (tensor.rs:522-528),
// optionally gated: out = mul_sat(gelu(dot), gate_rows[t][r]).
cudaError_t launch_dense(const int32_t* w, uint32_t rows, uint32_t cols, const int32_t* in,
                         uint32_t in_stride, uint32_t tokens, int32_t* out, uint32_t out_stride,
                         const int32_t* gelu_gate, uint32_t gate_stride, cudaStream_t s);
// Gemma per-layer inputs (view_kernels.rs:59-99) for every layer at once,
// given projected = dot_bits rows of the model projection: out[t][l][P].
cudaError_t launch_ple_prepare(const int32_t* projected, const Q8GpuMatrix* ple_embed,
                               const uint32_t* d_ids, const int32_t* ple_norm, int64_t eps,
                               int32_t projection_scalar, int32_t embedding_scale,
                               int32_t input_scale, uint32_t tokens, uint32_t layers, uint32_t P,
                               int32_t* out, cudaStream_t s);

// ---- device helpers shared by the attention kernels (layers.cu, step.cu) ----

// First position of the sliding window ending at p (prefill_range.rs:866-874).
__device__ __forceinline__ uint32_t window_start(uint32_t p, uint32_t window) {
  if (window == 0) return 0;
  return p + 1 > window ? p + 1 - window : 0;
}

__device__ __forceinline__ int32_t finish_score(int64_t sum, int mode, uint32_t scale) {
  return mode == SCORE_MISTRAL ? scaled_score_finish(sum, scale) : requantize(sum);
}

// Warp-wide sums over the lanes that share lane % HPC; lane h < HPC ends with
// the sum of head h's lanes.
template <uint32_t HPC, typename T>
__device__ __forceinline__ T head_lane_sum(T v) {
#pragma unroll
  for (uint32_t off = 16; off >= HPC; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

// Device-scope acquire load, release reduction and acquire-release add of a
// global 32-bit word (arrival counters between blocks of one launch).
__device__ __forceinline__ unsigned int ld_acquire_u32(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_add_release(unsigned int* p, unsigned int v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned int atom_add_acq_rel(unsigned int* p, unsigned int v) {
  unsigned int old;
  asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

}  // namespace iris
