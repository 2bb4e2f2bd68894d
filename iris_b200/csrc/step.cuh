// The persistent decode step: one cooperative launch runs a whole
// mistral-dense decode pass (embedding, every layer, head, greedy selection).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "layers.cuh"
#include "tp.cuh"

namespace iris {

enum StepKind : uint32_t {
  STEP_EMBED = 0,  // x = dequantize_row(embed[token])
  STEP_QKV = 1,    // q|k|v = W rms_norm(x); RoPE; k, v to the cache
  STEP_ATTN = 2,   // ctx = attention(q, K/V cache) as byte planes
  STEP_O = 3,      // x = x + W_o ctx
  STEP_GU = 4,     // g = silu(W_gate m) * (W_up m), m = rms_norm(x)
  STEP_DOWN = 5,   // x = x + W_down g
  STEP_HEAD = 6,   // logits = W_head rms_norm(x); first maximum -> next token
  STEP_XCHG = 7    // tensor parallelism: x = x + round(sum over ranks of the o / down partial sums)
};

// One stage of the pass (a device array built once per session).
struct StepStage {
  const int8_t* q;         // product stages: the matrix in the tiled layout
  const uint16_t* s;
  const int32_t* norm_w;   // RMSNorm weights of a normalised input, else NULL
  uint32_t kind, layer;
  uint32_t rows, cols, kc, nslices, items;
  int32_t e_fast;
  uint32_t xj;  // tensor parallelism: the pass's exchange (1-based) an o / down product feeds or an exchange is
  uint32_t uniform;  // 1: every row of the matrix has one scale (products scaled once a tile group)
};

// Timeline stamps a block records per stage (StepArgs::trace): 0 input ready,
// 7 share written; products: 1 prologue done, 2 warp 0's last tile taken,
// 6 the producer issued the stage's last tile (normalised inputs: 3 scale
// known, 4 thread 0's planes written); attention: 1 first key slot
// landed, 2 scores done, 3 and 4 first and second group exchange passed,
// 5 value sums added, 6 the producer issued the chunk's last value row.
constexpr uint32_t kStepTraceEvents = 8;

struct StepArgs {
  const StepStage* stages;
  uint32_t nstages;
  // model
  const int8_t* embed_q;
  const uint16_t* embed_s;
  uint32_t embed_kc, embed_nslices;
  uint32_t H, heads, kv_heads, d, qd, kvd;
  int64_t eps;
  uint32_t scale_q32;
  const int64_t* freqs;
  // session buffers
  int32_t* x;            // [H] residual stream
  int32_t* q;            // [qd] rotated queries
  uint8_t* planes;       // [4][qd] attention output planes
  uint8_t* planes2;      // [4][F] gated FFN planes
  int32_t* kcache;       // [layers][cap][kvd]
  int32_t* vcache;
  uint32_t cap;
  uint32_t layers;       // model layers
  int32_t* logits;       // [V]
  unsigned long long* best;
  unsigned long long* split_acc;
  unsigned int* split_count;
  // attention exchanges of a head group (zero between stages): the blocks'
  // first-maximum keys and exp-term sums, one slot [group][chunk][head] each
  unsigned long long* kslots;
  unsigned long long* sslots;
  int32_t* wsum;
  int64_t* acc;
  unsigned int* gbar;
  const uint32_t* exp_terms;  // exp_term_table
  unsigned int* gready;  // [layers][heads / hpc] q|k|v tile groups stored for each attention group (zero between launches)
  uint32_t hpc;          // query heads an attention group
  uint32_t chunks;       // blocks a head group
  uint32_t span_max;     // positions a block at most
  // bookkeeping of the greedy loop
  uint32_t* d_token;
  uint32_t* d_pos;
  uint32_t* d_step;
  uint32_t* history;
  uint32_t history_cap;
  unsigned int* sync;    // [nstages] arrivals a stage of the running pass (zero between launches)
  unsigned long long* sumsq;  // [nstages][blocks] each block's sum of squares of the x it wrote, clamped to i64::MAX
  unsigned int* fault;
  unsigned long long* trace;  // optional timeline of the last pass: [block][stage][kStepTraceEvents] ns
  // shared-memory layout
  uint32_t ring_slots, slot_bytes, planes_bytes;
  // tensor parallelism (tp_world > 1): the peer-memory exchange of tp.cuh.
  // Exchange j of a pass has epoch *xepoch + j (the count advances by the
  // pass's exchanges when the pass finishes); its limbs sit in slot
  // epoch & 1 of every rank's xpart; flags and key slots as in tp.cu.
  uint32_t tp_rank, tp_world, xchanges;
  int64_t* xpart;
  int64_t* xpeer_part[kTpMaxWorld];
  uint32_t* xflags;
  uint32_t* xpeer_flags[kTpMaxWorld];
  uint32_t* xepoch;
};

// The launch plan of a model and cache capacity, or ok = false when the
// shape needs the kernel-per-operation pass.
struct StepPlan {
  bool ok;
  uint32_t why;  // when not ok: 1 shape, 2 no kernel for the head shape, 3 device, 4 shared memory, 5 occupancy
  uint32_t blocks, ring_slots, slot_bytes, planes_bytes, smem, chunks, span_max, hpc;
};
// kcs: the slice width of every matrix of the pass.
StepPlan plan_decode_step(uint32_t H, uint32_t F, uint32_t heads, uint32_t kv_heads, uint32_t d, uint32_t V,
                          uint32_t cap, const uint32_t* kcs, uint32_t nkcs);
// uniform: every product stage's matrix has one scale a row (StepStage::uniform).
cudaError_t launch_decode_step(const StepArgs& a, const StepPlan& p, bool uniform, cudaStream_t s);
cudaError_t prepare_step_kernels();

}  // namespace iris
