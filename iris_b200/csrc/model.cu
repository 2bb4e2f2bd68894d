// Device-resident models, decoding sessions and the chain-stage entry point.
//
// A session holds the K/V cache of every layer as int32 rows
// [layers][positions][kv_heads * head_dim] in HBM; a pass runs the layers
// over a range of rows (the prompt in ranges of up to kMaxRows, or one decode
// token) and the head over its last row. Ranges are processed position-major:
// range r goes through every layer before range r+1; since every value of a
// row depends only on its own row and the K/V of earlier positions, this
// gives the same values as the reference's layer-major order
// (crates/inference/direct/src/executor.rs:293-401; the reference's own
// executor test checks the same invariance across chunkings).
//
// A decode pass is captured once into a CUDA graph that reads the token id
// and the position from device memory, so the decode loop replays it with no
// host round trip: the head's first maximum becomes the next input token on
// the device (generation.rs:25-58).
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "../../include/iris_b200.h"
#include "layers.cuh"
#include "sha256.cuh"
#include "step.cuh"
#include "tc.cuh"
#include "tp.cuh"
#include "synth.cuh"

using namespace iris;

namespace {

constexpr uint32_t kMaxRows = 512;  // rows a prefill range holds on the device (the chain's range_size)
constexpr int kFamilyMistral = 0, kFamilyGemma = 1;

struct LayerDev {
  Q8GpuMatrix *qkv = nullptr, *o = nullptr, *gu = nullptr, *down = nullptr;
  int32_t *norm_attn = nullptr, *norm_ffn = nullptr;
  // gemma-dense
  int32_t *norm_post_attn = nullptr, *norm_post_ffw = nullptr, *q_norm = nullptr, *k_norm = nullptr,
          *ple_post_norm = nullptr, *ple_gate = nullptr, *ple_proj = nullptr;
  int64_t* inv_freq = nullptr;
  uint32_t window = 0, rotary_dim = 0, freq_base_dim = 0;
  int64_t rope_base = 0;
  int32_t kv_donor = -1, layer_scalar = 0;
};

// ---- host restatement of the rotary frequency ladder (ops.rs:558-720) ------
typedef __int128 i128;
int64_t clamp64(i128 v) {
  return v < (i128)INT64_MIN ? INT64_MIN : (v > (i128)INT64_MAX ? INT64_MAX : (int64_t)v);
}
i128 div_even(i128 n, i128 d) {  // round_ties_even_division
  i128 q = n / d, r = n % d;
  if (r == 0) return q;
  i128 twice = (r < 0 ? -r : r) * 2, ad = d < 0 ? -d : d, step = ((n < 0) != (d < 0)) ? -1 : 1;
  if (twice < ad) return q;
  if (twice > ad) return q + step;
  return (q & 1) == 0 ? q : q + step;
}
int64_t h_acc_mul(int64_t a, int64_t b) { return clamp64(div_even((i128)a * b, (i128)1 << 32)); }
int64_t h_pow(int64_t b, uint32_t e) {
  int64_t r = (int64_t)1 << 32;
  for (uint32_t i = 0; i < e; ++i) r = h_acc_mul(r, b);
  return r;
}
int64_t h_nth_root(int64_t value, uint32_t degree) {  // nth_root_acc, ops.rs:564-606
  const int64_t one = (int64_t)1 << 32;
  if (degree == 1 || value == one) return value;
  int64_t lo = 0, hi = std::max(value, one);
  while (lo < hi) {
    int64_t mid = lo + (hi - lo + 1) / 2;
    if (h_pow(mid, degree) <= value) lo = mid;
    else hi = mid - 1;
  }
  int64_t up = lo == INT64_MAX ? lo : lo + 1;
  i128 le = (i128)value - h_pow(lo, degree), ue = (i128)h_pow(up, degree) - value;
  if (le < 0) le = -le;
  if (ue < 0) ue = -ue;
  if (ue < le) return up;
  if (le < ue) return lo;
  return (lo & 1) == 0 ? lo : up;
}
// inv_frequency_i for i < half: the reference's chained acc_mul (ops.rs:178-198).
std::vector<int64_t> rope_inverse_frequencies(int64_t base, uint32_t freq_base_dim, uint32_t half) {
  int64_t step = clamp64(div_even((i128)((int64_t)1 << 32) << 32, h_nth_root(base, freq_base_dim / 2)));
  std::vector<int64_t> f(half);
  int64_t inv = (int64_t)1 << 32;
  for (uint32_t i = 0; i < half; ++i) {
    f[i] = inv;
    inv = h_acc_mul(inv, step);
  }
  return f;
}

template <class T>
cudaError_t dalloc(T** p, size_t count) {
  *p = nullptr;
  if (count == 0) return cudaSuccess;
  return cudaMalloc((void**)p, count * sizeof(T));
}

}  // namespace

constexpr uint32_t kChainTickets = 64;  // copies of chain stages a session tracks at once

struct IrisModel {
  int family = 0;
  uint32_t L = 0, H = 0, F = 0, heads = 0, kvh = 0, d = 0, V = 0, P = 0, max_positions = 0;
  uint32_t qd = 0, kvd = 0;
  int64_t eps = 0;
  uint32_t scale_q32 = 0;
  bool tied = false;
  int32_t embedding_scale = 0, ple_embedding_scale = 0, ple_projection_scalar = 0, ple_input_scale = 0,
          softcap = 0;
  Q8GpuMatrix *embed = nullptr, *head = nullptr, *ple_embed = nullptr;
  int32_t *final_norm = nullptr, *ple_model_proj = nullptr, *ple_norm = nullptr;
  int64_t* freqs = nullptr;  // mistral [d/2]
  std::vector<LayerDev> layers;
  uint64_t weight_bytes = 0;
  IrisSession* scratch = nullptr;  // for the chain-stage entry point
  // tensor parallelism: this rank's share of heads, kv heads, FFN rows and
  // vocabulary (the dimensions above are the local ones), the full
  // vocabulary (embedding table, token ids) and the NCCL communicator
  uint32_t tp_rank = 0, tp_world = 1, Vfull = 0;
  void* comm = nullptr;
  TpExchange xch{};       // peer-memory exchange of one-token row-parallel products
  bool xch_nccl = false;  // exchange one-token products over NCCL instead
  int gemm_mode = IRIS_GEMM_AUTO;  // many-token products: tensor-core GEMM where it applies, or mma.sync only
  // many-query (prefill) attention launches so far: [0] tensor-core, [1] CUDA-core
  std::atomic<uint64_t> attn_ranges[2] = {};
};

struct IrisSession {
  IrisModel* m = nullptr;
  uint32_t cap = 0, len = 0;
  // tensor-core prefill attention scratch, allocated on the first range that
  // takes it (attn_tc_state: 0 not tried, 1 ready, 2 unavailable)
  uint8_t* attn_tc_buf = nullptr;
  AttnTcScratch attn_tc;
  int attn_tc_state = 0;
  bool has_logits = false;  // a pass has run since the last reset
  int32_t *kc = nullptr, *vc = nullptr;
  int32_t *x = nullptr, *tmp = nullptr, *q = nullptr, *qkv = nullptr, *xs = nullptr, *pg = nullptr,
          *ple_rows = nullptr, *ple_proj = nullptr, *logits = nullptr;
  uint8_t *planes = nullptr, *planes2 = nullptr;
  unsigned long long* best = nullptr;
  uint32_t *d_ids = nullptr, *d_pos = nullptr, *d_token = nullptr, *d_step = nullptr, *d_history = nullptr;
  uint32_t history_cap = 0;
  // decode attention scratch
  int32_t* scores = nullptr;
  int64_t* terms = nullptr;
  unsigned long long* chunk_best = nullptr;
  uint64_t* chunk_sum = nullptr;
  int32_t* wsum = nullptr;
  int64_t* acc = nullptr;
  unsigned int* counters = nullptr;
  unsigned int* ple_done = nullptr;
  int32_t* xa = nullptr;  // gemma, one token: the residual row after attention (IN_POST_ATTN)
  int64_t* rope_sc = nullptr;  // mistral: [rows][d / 2][2] sines and cosines of a range's positions  // gemma: blocks done with the PLE projection (zero between launches)
  uint32_t nchunks = 0, hpc = 1;
  uint32_t cluster = 0, chpc = 1, span = 0, ring = 0;  // one-launch cluster decode attention
  uint32_t chunks = 0, ghpc = 1, gspan = 0;               // one-launch whole-GPU decode attention
  unsigned long long *gbest = nullptr, *gsum = nullptr;
  unsigned int* gbar = nullptr;
  unsigned int* fault = nullptr;
  int64_t* partial = nullptr;     // tensor parallelism: [kMaxRows][H][4] limbs
  int32_t* logits_full = nullptr; // tensor parallelism: the gathered vocabulary
  // decode GEMV split scratch (zero between launches)
  unsigned long long* split_acc = nullptr;
  unsigned int* split_count = nullptr;
  uint32_t split_groups = 0;
  // persistent decode step (step.cu): its plan, stage list and arrival counter
  StepPlan step{};
  const uint32_t* exp_terms = nullptr;  // the device's exp-term table (the step's attention)
  StepStage* stages = nullptr;
  uint32_t nstages = 0;
  // host copy of the stage list, the matrix of each product stage and the
  // weights version its one-scale-a-row flag was taken at
  std::vector<StepStage> step_host;
  std::vector<const Q8GpuMatrix*> step_mats;
  std::vector<uint32_t> step_versions;
  unsigned int* sync = nullptr;  // [nstages] arrival counters
  unsigned int* gready = nullptr;  // [layers][heads / hpc] the attention groups' q|k|v tile groups stored
  unsigned long long* trace = nullptr;  // optional per-stage timeline of the last pass
  unsigned long long* sumsq = nullptr;  // [nstages][blocks] sums of squares of the residual stream
  unsigned long long *kslots = nullptr, *sslots = nullptr;  // attention exchange slots [heads][blocks]
  uint32_t xchanges = 0;                // tensor parallelism: exchanges a pass
  int decode_mode = IRIS_DECODE_AUTO;
  int attn_mode = IRIS_ATTN_AUTO;
  bool use_step = false;
  cudaStream_t stream = nullptr;
  cudaGraphExec_t graph = nullptr;
  // device-resident chain ranges (iris_session_range_*): rows of the range in
  // progress (0: none), the next layer to run, and the events behind tickets
  uint32_t range_n = 0, range_layer = 0;
  cudaEvent_t tickets[kChainTickets] = {};
  std::atomic<uint32_t> next_ticket{0};  // read by threads waiting for tickets
  // the stages' copies run on their own stream: the rows go through one of
  // two device staging buffers (the next layer overwrites x), K/V straight
  // from the cache; staged: the compute stream's "rows staged" event,
  // stage_read[b]: the copy stream finished reading buffer b
  cudaStream_t copy_stream = nullptr;
  int32_t* stage_rows[2] = {};
  uint8_t* stage_leaves[2] = {};  // iris_session_range_layer_leaves: the stage's leaf digests
  uint32_t leaves_cap = 0;        // leaf digests each holds
  cudaEvent_t staged = nullptr, stage_read[2] = {};
};

namespace {

size_t kv_offset(const IrisSession* s, uint32_t l) { return (size_t)l * s->cap * s->m->kvd; }

void free_session(IrisSession* s) {
  if (!s) return;
  if (s->graph) cudaGraphExecDestroy(s->graph);
  void* ptrs[] = {s->kc, s->vc, s->x, s->tmp, s->q, s->qkv, s->xs, s->pg, s->ple_rows, s->ple_proj,
                  s->logits, s->planes, s->planes2, s->best, s->d_ids, s->d_pos, s->d_token, s->d_step,
                  s->d_history, s->scores, s->terms, s->chunk_best, s->chunk_sum, s->wsum,
                  s->acc, s->counters, s->split_acc, s->split_count, s->gbest, s->gsum, s->gbar, s->partial, s->logits_full,
                  s->stages, s->sync, s->gready, s->trace, s->sumsq, s->kslots, s->sslots, s->attn_tc_buf,
                  s->ple_done, s->xa, s->rope_sc};
  if (s->copy_stream) cudaStreamSynchronize(s->copy_stream);
  for (int b = 0; b < 2; ++b) cudaFree(s->stage_leaves[b]);
  for (void* p : ptrs) cudaFree(p);
  for (int32_t* p : s->stage_rows) cudaFree(p);
  for (cudaEvent_t ev : s->tickets)
    if (ev) cudaEventDestroy(ev);
  for (cudaEvent_t ev : {s->staged, s->stage_read[0], s->stage_read[1]})
    if (ev) cudaEventDestroy(ev);
  if (s->copy_stream) cudaStreamDestroy(s->copy_stream);
  if (s->stream) cudaStreamDestroy(s->stream);
  delete s;
}

// The stage list and launch plan of the persistent decode step
// (mistral-dense without tensor parallelism); s->step.ok stays false when the
// model or capacity needs the kernel-per-operation pass.
cudaError_t setup_step(IrisSession* s) {
  IrisModel* m = s->m;
  s->step.why = 6;  // not a mistral-dense model (with the peer-memory exchange when tensor-parallel)
  if (m->family != kFamilyMistral || !m->embed || !m->head) return cudaSuccess;
  if (m->tp_world > 1 && (!m->xch.part || m->tp_world > kTpMaxWorld)) return cudaSuccess;
  std::vector<StepStage> st;
  std::vector<uint32_t> kcs;
  std::vector<const Q8GpuMatrix*> mats;
  auto product = [&](uint32_t kind, uint32_t layer, const Q8GpuMatrix* w, const int32_t* norm) {
    mats.resize(st.size());
    mats.push_back(w);
    StepStage x{};
    x.q = w->q;
    x.s = w->s;
    x.norm_w = norm;
    x.kind = kind;
    x.layer = layer;
    x.rows = w->rows;
    x.cols = w->cols;
    x.kc = w->kc;
    x.nslices = w->nslices;
    x.items = w->groups * w->nslices;
    uint32_t lg = 0;  // as plan_gemv: S terms a lane stay below 2^62 for e <= 15 - ceil(log2 S)
    while ((1u << lg) < w->nslices) ++lg;
    x.e_fast = 15 - (int32_t)lg;
    st.push_back(x);
    kcs.push_back(w->kc);
  };
  auto plain = [&](uint32_t kind, uint32_t layer) {
    StepStage x{};
    x.kind = kind;
    x.layer = layer;
    st.push_back(x);
  };
  // with tensor parallelism o and down leave partial sums that an exchange
  // stage sums over the ranks (exchange j feeds on the product tagged j)
  const bool tp = m->tp_world > 1;
  uint32_t xj = 0;
  auto exchange = [&](uint32_t layer) {
    st.back().xj = ++xj;
    StepStage x{};
    x.kind = STEP_XCHG;
    x.layer = layer;
    x.xj = xj;
    st.push_back(x);
  };
  plain(STEP_EMBED, 0);
  for (uint32_t l = 0; l < m->L; ++l) {
    const LayerDev& L = m->layers[l];
    if (!L.qkv || !L.o || !L.gu || !L.down) return cudaSuccess;
    product(STEP_QKV, l, L.qkv, L.norm_attn);
    plain(STEP_ATTN, l);
    product(STEP_O, l, L.o, nullptr);
    if (tp) exchange(l);
    product(STEP_GU, l, L.gu, L.norm_ffn);
    product(STEP_DOWN, l, L.down, nullptr);
    if (tp) exchange(l);
  }
  product(STEP_HEAD, 0, m->head, m->final_norm);
  if (cudaError_t e = exp_term_table(&s->exp_terms); e != cudaSuccess) return e;
  StepPlan plan = plan_decode_step(m->H, m->F, m->heads, m->kvh, m->d, m->V, s->cap, kcs.data(), (uint32_t)kcs.size());
  if (!plan.ok) {
    s->step = plan;
    return cudaSuccess;
  }
  mats.resize(st.size());
  s->step_host = st;
  s->step_mats = mats;
  s->step_versions.assign(st.size(), UINT32_MAX);  // flags taken before the first pass
  cudaError_t e = dalloc(&s->stages, st.size());
  if (e == cudaSuccess) e = cudaMemcpy(s->stages, st.data(), st.size() * sizeof(StepStage), cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = dalloc(&s->sync, st.size());
  if (e == cudaSuccess) e = cudaMemset(s->sync, 0, st.size() * sizeof(unsigned int));
  const size_t ngready = (size_t)m->L * (m->heads / plan.hpc);
  if (e == cudaSuccess) e = dalloc(&s->gready, ngready);
  if (e == cudaSuccess) e = cudaMemset(s->gready, 0, ngready * sizeof(unsigned int));
  const size_t nslots = (size_t)m->heads * plan.blocks;
  if (e == cudaSuccess) e = dalloc(&s->kslots, nslots);
  if (e == cudaSuccess) e = dalloc(&s->sslots, nslots);
  if (e == cudaSuccess) e = cudaMemset(s->kslots, 0, nslots * sizeof(unsigned long long));
  if (e == cudaSuccess) e = cudaMemset(s->sslots, 0, nslots * sizeof(unsigned long long));
  if (e == cudaSuccess) e = dalloc(&s->sumsq, st.size() * plan.blocks);
  if (e == cudaSuccess) e = cudaMemset(s->sumsq, 0, st.size() * plan.blocks * sizeof(unsigned long long));
  if (e != cudaSuccess) return e;
  s->nstages = (uint32_t)st.size();
  s->xchanges = xj;
  s->step = plan;
  s->use_step = true;
  return cudaSuccess;
}

// Arguments of one persistent decode step.
StepArgs step_args(IrisSession* s) {
  IrisModel* m = s->m;
  StepArgs a{};
  a.stages = s->stages;
  a.nstages = s->nstages;
  a.embed_q = m->embed->q;
  a.embed_s = m->embed->s;
  a.embed_kc = m->embed->kc;
  a.embed_nslices = m->embed->nslices;
  a.H = m->H;
  a.layers = m->L;
  a.heads = m->heads;
  a.kv_heads = m->kvh;
  a.d = m->d;
  a.qd = m->qd;
  a.kvd = m->kvd;
  a.eps = m->eps;
  a.scale_q32 = m->scale_q32;
  a.freqs = m->freqs;
  a.x = s->x;
  a.q = s->q;
  a.planes = s->planes;
  a.planes2 = s->planes2;
  a.kcache = s->kc;
  a.vcache = s->vc;
  a.cap = s->cap;
  a.logits = s->logits;
  a.best = s->best;
  a.split_acc = s->split_acc;
  a.split_count = s->split_count;
  a.kslots = s->kslots;
  a.sslots = s->sslots;
  a.wsum = s->wsum;
  a.acc = s->acc;
  a.gbar = s->gbar;
  a.chunks = s->step.chunks;
  a.span_max = s->step.span_max;
  a.gready = s->gready;
  a.hpc = s->step.hpc;
  a.exp_terms = s->exp_terms;
  a.d_token = s->d_token;
  a.d_pos = s->d_pos;
  a.d_step = s->d_step;
  a.history = s->d_history;
  a.history_cap = s->history_cap;
  a.sync = s->sync;
  a.fault = s->fault;
  a.trace = s->trace;
  a.sumsq = s->sumsq;
  if (m->tp_world > 1) {
    a.tp_rank = m->tp_rank;
    a.tp_world = m->tp_world;
    a.xchanges = s->xchanges;
    a.xpart = m->xch.part;
    a.xflags = m->xch.flags;
    a.xepoch = m->xch.epoch;
    for (uint32_t j = 0; j < m->tp_world; ++j) {
      a.xpeer_part[j] = m->xch.peer_part[j];
      a.xpeer_flags[j] = m->xch.peer_flags[j];
    }
  } else {
    a.tp_world = 1;
  }
  a.ring_slots = s->step.ring_slots;
  a.slot_bytes = s->step.slot_bytes;
  a.planes_bytes = s->step.planes_bytes;
  return a;
}

int create_session(IrisModel* m, uint32_t cap, IrisSession** out) {
  *out = nullptr;
  if (cap == 0) return IRIS_EINVAL;
  IrisSession* s = new IrisSession();
  s->m = m;
  s->cap = cap;
  const uint32_t R = kMaxRows;
  size_t wide = std::max({m->H, m->qd, m->F, m->P ? m->P : 1u});
  cudaError_t e = cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking);
  size_t kv = (size_t)m->L * cap * m->kvd;
  if (e == cudaSuccess) e = dalloc(&s->kc, kv);
  if (e == cudaSuccess) e = dalloc(&s->vc, kv);
  if (e == cudaSuccess) e = dalloc(&s->x, (size_t)R * m->H);
  if (e == cudaSuccess) e = dalloc(&s->tmp, (size_t)R * m->H);
  if (e == cudaSuccess) e = dalloc(&s->q, (size_t)R * m->qd);
  if (e == cudaSuccess) e = dalloc(&s->planes, (size_t)R * 4 * wide);
  if (e == cudaSuccess) e = dalloc(&s->planes2, (size_t)R * 4 * wide);
  if (e == cudaSuccess) e = dalloc(&s->logits, (size_t)m->V);
  if (m->tp_world > 1) {
    if (e == cudaSuccess) e = dalloc(&s->partial, (size_t)R * m->H * 4);
    if (e == cudaSuccess) e = dalloc(&s->logits_full, (size_t)m->Vfull);
  }
  if (e == cudaSuccess) e = dalloc(&s->best, R);
  if (e == cudaSuccess) e = dalloc(&s->d_ids, R);
  if (e == cudaSuccess) e = dalloc(&s->d_pos, 1);
  if (e == cudaSuccess) e = dalloc(&s->d_token, 1);
  if (e == cudaSuccess) e = dalloc(&s->d_step, 1);
  if (m->family == kFamilyGemma) {
    if (e == cudaSuccess) e = dalloc(&s->qkv, (size_t)R * (m->qd + 2 * m->kvd));
    if (e == cudaSuccess) e = dalloc(&s->xs, (size_t)R * m->H);
    if (e == cudaSuccess) e = dalloc(&s->pg, (size_t)R * m->P);
    if (e == cudaSuccess) e = dalloc(&s->ple_rows, (size_t)R * m->L * m->P);
    if (e == cudaSuccess) e = dalloc(&s->ple_proj, (size_t)R * m->L * m->P);
    if (e == cudaSuccess) e = dalloc(&s->ple_done, 1);
    if (e == cudaSuccess) e = dalloc(&s->xa, (size_t)m->H);
    if (e == cudaSuccess) e = cudaMemset(s->ple_done, 0, sizeof(unsigned int));
  } else if (m->freqs) {
    if (e == cudaSuccess) e = dalloc(&s->rope_sc, (size_t)R * (m->d / 2) * 2);
  }
  s->nchunks = attention_chunks(cap);
  s->hpc = attention_hpc(m->heads, m->kvh);
  attention_cluster_plan(m->heads, m->kvh, m->d, cap, &s->chpc, &s->cluster, &s->span, &s->ring);
  attention_grid_plan(m->heads, m->kvh, m->d, cap, &s->ghpc, &s->chunks, &s->gspan);
  s->fault = device_fault_word();
  if (e == cudaSuccess) e = dalloc(&s->gbest, m->heads);
  if (e == cudaSuccess) e = dalloc(&s->gsum, m->heads);
  if (e == cudaSuccess) e = dalloc(&s->gbar, 2 * m->heads);
  if (e == cudaSuccess) e = cudaMemset(s->gbest, 0, m->heads * sizeof(unsigned long long));
  if (e == cudaSuccess) e = cudaMemset(s->gsum, 0, m->heads * sizeof(unsigned long long));
  if (e == cudaSuccess) e = cudaMemset(s->gbar, 0, 2 * m->heads * sizeof(unsigned int));
  if (e == cudaSuccess) e = dalloc(&s->scores, (size_t)m->heads * cap);
  if (e == cudaSuccess) e = dalloc(&s->terms, (size_t)m->heads * cap);
  if (e == cudaSuccess) e = dalloc(&s->chunk_best, (size_t)m->heads * s->nchunks);
  if (e == cudaSuccess) e = dalloc(&s->chunk_sum, (size_t)m->heads * s->nchunks);
  if (e == cudaSuccess) e = dalloc(&s->wsum, m->heads);
  if (e == cudaSuccess) e = dalloc(&s->acc, (size_t)m->heads * m->d);
  if (e == cudaSuccess) e = cudaMemset(s->wsum, 0, m->heads * sizeof(int32_t));
  if (e == cudaSuccess) e = cudaMemset(s->acc, 0, (size_t)m->heads * m->d * sizeof(int64_t));
  if (e == cudaSuccess) e = dalloc(&s->counters, m->heads);
  if (e == cudaSuccess) e = cudaMemset(s->counters, 0, m->heads * sizeof(unsigned int));
  s->split_groups = (std::max({m->qd + 2 * m->kvd, m->H, 2 * m->F, m->V}) + kQ8TileRows - 1) / kQ8TileRows;
  if (e == cudaSuccess) e = dalloc(&s->split_acc, (size_t)s->split_groups * kQ8TileRows * 2);
  if (e == cudaSuccess) e = dalloc(&s->split_count, s->split_groups);
  if (e == cudaSuccess)
    e = cudaMemset(s->split_acc, 0, (size_t)s->split_groups * kQ8TileRows * 2 * sizeof(unsigned long long));
  if (e == cudaSuccess) e = cudaMemset(s->split_count, 0, s->split_groups * sizeof(unsigned int));
  if (e == cudaSuccess) e = cudaMemset(s->best, 0, R * sizeof(unsigned long long));
  if (e == cudaSuccess) e = cudaMemset(s->d_pos, 0, 4);
  if (e == cudaSuccess) e = cudaMemset(s->d_step, 0, 4);
  if (e == cudaSuccess) e = setup_step(s);
  if (e != cudaSuccess) {
    free_session(s);
    return (int)e;
  }
  *out = s;
  return 0;
}

// Whether decode passes run as the persistent step (tensor-parallel models:
// only with the peer-memory exchange).
void choose_decode_path(IrisSession* s) {
  const bool nccl_exchange = s->m->tp_world > 1 && s->m->xch_nccl;
  s->use_step = s->step.ok && !nccl_exchange && s->decode_mode != IRIS_DECODE_GRAPH &&
                s->attn_mode == IRIS_ATTN_AUTO;
}

// Product arguments with the session's GEMV split scratch.
ProductArgs session_product_args(IrisSession* s, const Q8GpuMatrix* w, uint32_t tokens) {
  // many-token products: the tensor-core copy of the weights, built on first use
  const bool tc = s->m->gemm_mode == IRIS_GEMM_AUTO && tokens >= kTcMinTokens;
  if (tc && tc_state_get(w) == 0) tc_prepare(const_cast<Q8GpuMatrix*>(w), s->stream);
  ProductArgs a = product_args(w, tokens);
  if (!tc) {
    a.tc = nullptr;
    a.tc_shift = nullptr;
    a.tc_mant = nullptr;
    a.tc_rows = 0;
    a.tc_planes = 0;
  }
  a.split_acc = s->split_acc;
  a.split_count = s->split_count;
  a.split_groups = s->split_groups;
  if (tokens == 1) a.uniform = q8_uniform_cached(const_cast<Q8GpuMatrix*>(w), s->stream) ? 1u : 0u;
  return a;
}

AttnArgs attn_args(IrisSession* s, uint32_t l, const uint32_t* pos_ptr, uint32_t pos0) {
  IrisModel* m = s->m;
  const LayerDev& L = m->layers[l];
  uint32_t src = (m->family == kFamilyGemma && L.kv_donor >= 0) ? (uint32_t)L.kv_donor : l;
  AttnArgs a{};
  a.q = s->q;
  a.kcache = s->kc + kv_offset(s, src);
  a.vcache = s->vc + kv_offset(s, src);
  a.heads = m->heads;
  a.kv_heads = m->kvh;
  a.d = m->d;
  a.kvd = m->kvd;
  a.pos_ptr = pos_ptr;
  a.pos0 = pos0;
  a.window = m->family == kFamilyGemma ? L.window : 0;
  a.mode = m->family == kFamilyGemma ? SCORE_GEMMA : SCORE_MISTRAL;
  a.scale_q32 = m->scale_q32;
  a.ctx_planes = s->planes;
  a.scores = s->scores;
  a.terms = s->terms;
  a.chunk_best = s->chunk_best;
  a.chunk_sum = s->chunk_sum;
  a.wsum = s->wsum;
  a.acc = s->acc;
  a.counters = s->counters;
  a.cap = s->cap;
  a.nchunks = s->nchunks;
  a.hpc = s->hpc;
  a.cluster = s->cluster;
  a.chpc = s->chpc;
  a.span = s->span;
  a.ring = s->ring;
  a.chunks = s->chunks;
  a.ghpc = s->ghpc;
  a.gspan = s->gspan;
  a.gbest = s->gbest;
  a.gsum = s->gsum;
  a.gbar = s->gbar;
  a.fault = s->fault;
  return a;
}


// One mistral-dense layer (mistral/layer.rs:107-270) over `tokens` rows in
// s->x at positions pos0.. (or *pos_ptr for the decode pass).
// x = x + W in (in as byte planes): one product, or with tensor parallelism
// the rank's columns as exact partial sums, their sum over the ranks, then
// one rounding and the residual.
cudaError_t row_parallel_resid(IrisSession* s, ProductArgs a, uint32_t tokens) {
  IrisModel* m = s->m;
  if (m->tp_world == 1) {
    a.out = s->x;
    a.resid = s->x;
    return launch_product(a, IN_PLANES, EPI_RESID, s->stream);
  }
  if (tokens == 1 && !m->xch_nccl) {  // one token: the peer-memory exchange
    a.partial = m->xch.part;
    a.xepoch = m->xch.epoch;
    cudaError_t e = launch_product(a, IN_PLANES, EPI_PARTIAL, s->stream);
    if (e == cudaSuccess) e = launch_tp_p2p_finish(m->xch, m->H, s->x, s->x, s->stream);
    return e;
  }
  a.partial = s->partial;
  cudaError_t e = launch_product(a, IN_PLANES, EPI_PARTIAL, s->stream);
  if (e == cudaSuccess) e = tp_sum_limbs(m->comm, s->partial, (size_t)tokens * m->H * 4, s->stream);
  if (e == cudaSuccess) e = launch_tp_finish(s->partial, tokens, m->H, s->x, s->x, s->stream);
  return e;
}

// Many-query attention of a mistral range: the tensor-core kernels where the
// shape allows (head_dim 128, no window cutting the prefix) and the model's
// many-token products are on the tensor cores, else the CUDA-core kernel.
cudaError_t launch_prefill_attention(IrisSession* s, const AttnArgs& at, uint32_t tokens, cudaStream_t st) {
  IrisModel* m = s->m;
  if (m->gemm_mode == IRIS_GEMM_AUTO && tokens >= kTcMinTokens && s->attn_tc_state != 2) {
    if (s->attn_tc_state == 0) {
      s->attn_tc_state = 2;
      const uint32_t pcap = (std::min<uint32_t>(s->cap, 22016) + 127) / 128 * 128;
      const uint32_t qcap = (kMaxRows + 63) / 64 * 64;
      const size_t bytes = attn_tc_scratch_bytes(m->heads, m->kvh, pcap, qcap);
      if (m->d == 128 && cudaMalloc((void**)&s->attn_tc_buf, bytes) == cudaSuccess) {
        attn_tc_scratch_carve(s->attn_tc_buf, m->heads, m->kvh, pcap, qcap, &s->attn_tc);
        s->attn_tc_state = 1;
      } else {
        cudaGetLastError();  // no room: the CUDA-core kernel serves this session
      }
    }
    if (s->attn_tc_state == 1 && attn_tc_usable(at, tokens, s->attn_tc)) {
      m->attn_ranges[0].fetch_add(1, std::memory_order_relaxed);
      return launch_attention_prefill_tc(at, tokens, s->attn_tc, st);
    }
  }
  m->attn_ranges[1].fetch_add(1, std::memory_order_relaxed);
  return launch_attention_prefill(at, tokens, at.pos0 + tokens, st);
}

cudaError_t mistral_layer(IrisSession* s, uint32_t l, uint32_t tokens, const uint32_t* pos_ptr,
                          uint32_t pos0) {
  IrisModel* m = s->m;
  const LayerDev& L = m->layers[l];
  cudaStream_t st = s->stream;
  cudaError_t e = cudaSuccess;
  bool one = tokens == 1;
  // n = rms_norm(x); q, k, v = W n; rope(q), rope(k); k, v to the cache
  ProductArgs a = session_product_args(s, L.qkv, tokens);
  a.out = s->q;
  a.out_stride = m->qd;
  a.freqs = m->freqs;
  a.head_dim = m->d;
  a.qd = m->qd;
  a.kvd = m->kvd;
  a.kcache = s->kc + kv_offset(s, l);
  a.vcache = s->vc + kv_offset(s, l);
  a.pos_ptr = pos_ptr;
  a.pos0 = pos0;
  if (one) {
    a.x = s->x;
    a.norm_w = L.norm_attn;
    a.eps = m->eps;
    e = launch_product(a, IN_NORM, EPI_QKV_ROPE, st);
  } else {
    e = launch_planes(s->x, L.norm_attn, m->eps, tokens, m->H, s->planes, st);
    a.planes = s->planes;
    if (e == cudaSuccess && s->rope_sc) {  // each position's rotations once, not once a row pair
      e = launch_rope_table(m->freqs, m->d / 2, pos_ptr, pos0, tokens, s->rope_sc, st);
      a.rope_sc = s->rope_sc;
    }
    if (e == cudaSuccess) e = launch_product(a, IN_PLANES, EPI_QKV_ROPE, st);
  }
  if (e != cudaSuccess) return e;
  // attention over positions 0..=p, context as planes
  AttnArgs at = attn_args(s, l, pos_ptr, pos0);
  e = one ? launch_attention_decode(at, st) : launch_prefill_attention(s, at, tokens, st);
  if (e != cudaSuccess) return e;
  // x = x + W_o ctx
  ProductArgs o = session_product_args(s, L.o, tokens);
  o.planes = s->planes;
  e = row_parallel_resid(s, o, tokens);
  if (e != cudaSuccess) return e;
  // g = silu(W_gate m) * (W_up m), m = rms_norm(x)
  ProductArgs g = session_product_args(s, L.gu, tokens);
  g.out_planes = s->planes2;
  if (one) {
    g.x = s->x;
    g.norm_w = L.norm_ffn;
    g.eps = m->eps;
    e = launch_product(g, IN_NORM, EPI_SILU_MUL, st);
  } else {
    e = launch_planes(s->x, L.norm_ffn, m->eps, tokens, m->H, s->planes, st);
    g.planes = s->planes;
    if (e == cudaSuccess) e = launch_product(g, IN_PLANES, EPI_SILU_MUL, st);
  }
  if (e != cudaSuccess) return e;
  // x = x + W_down g
  ProductArgs dn = session_product_args(s, L.down, tokens);
  dn.planes = s->planes2;
  return row_parallel_resid(s, dn, tokens);
}

// One gemma-dense layer (prefill_range.rs:307-333, 497-741, 879-957). A
// layer that shares its donor's K/V attends over the donor's cache; with
// keep_own_kv its own (unused) keys and values are still stored in its own
// cache rows (the chain stage hands them on, prefill_range.rs:542-575).
cudaError_t gemma_layer(IrisSession* s, uint32_t l, uint32_t tokens, const uint32_t* pos_ptr,
                        uint32_t pos0, bool keep_own_kv = false) {
  IrisModel* m = s->m;
  const LayerDev& L = m->layers[l];
  cudaStream_t st = s->stream;
  cudaError_t e;
  bool one = tokens == 1;
  ProductArgs a = session_product_args(s, L.qkv, tokens);
  a.out = s->qkv;
  if (one) {
    a.x = s->x;
    a.norm_w = L.norm_attn;
    a.eps = m->eps;
    e = launch_product(a, IN_NORM, EPI_STORE, st);
  } else {
    e = launch_planes(s->x, L.norm_attn, m->eps, tokens, m->H, s->planes, st);
    a.planes = s->planes;
    if (e == cudaSuccess) e = launch_product(a, IN_PLANES, EPI_STORE, st);
  }
  if (e != cudaSuccess) return e;
  QkvFinishArgs f{};
  f.qkv = s->qkv;
  f.q_out = s->q;
  bool own = L.kv_donor < 0 || keep_own_kv;  // a sharing layer attends over its donor's cache
  f.kcache = own ? s->kc + kv_offset(s, l) : nullptr;
  f.vcache = own ? s->vc + kv_offset(s, l) : nullptr;
  f.q_norm = L.q_norm;
  f.k_norm = L.k_norm;
  f.inv_freq = L.inv_freq;
  f.heads = m->heads;
  f.kv_heads = m->kvh;
  f.d = m->d;
  f.rotary_dim = L.rotary_dim;
  f.eps = m->eps;
  f.pos_ptr = pos_ptr;
  f.pos0 = pos0;
  e = launch_gemma_qkv_finish(f, tokens, st);
  if (e != cudaSuccess) return e;
  AttnArgs at = attn_args(s, l, pos_ptr, pos0);
  uint32_t max_vis = L.window ? std::min(L.window, pos0 + tokens) : pos0 + tokens;
  if (!one) m->attn_ranges[1].fetch_add(1, std::memory_order_relaxed);
  e = one ? launch_attention_decode(at, st) : launch_attention_prefill(at, tokens, max_vis, st);
  if (e != cudaSuccess) return e;
  ProductArgs o = session_product_args(s, L.o, tokens);
  o.planes = s->planes;
  o.out = s->tmp;
  e = launch_product(o, IN_PLANES, EPI_STORE, st);
  if (e != cudaSuccess) return e;
  ProductArgs g = session_product_args(s, L.gu, tokens);
  g.out_planes = s->planes2;
  // One token: the post-attention norms run in the gate|up product's
  // prologue (IN_POST_ATTN), the new residual row going to xa
  const bool post_fused = tokens == 1 && m->H <= kPostAttnMaxCols;
  const int32_t* x_attn = post_fused ? s->xa : s->x;  // the residual row after attention
  if (post_fused) {
    g.post_o = s->tmp;
    g.post_w = L.norm_post_attn;
    g.post_x = s->xa;
    g.x = s->x;
    g.norm_w = L.norm_ffn;
    g.eps = m->eps;
    e = launch_product(g, IN_POST_ATTN, EPI_GELU_MUL, st);
  } else {
    e = launch_gemma_post_attn(s->tmp, s->x, L.norm_post_attn, L.norm_ffn, m->eps, tokens, m->H, s->planes, st);
    g.planes = s->planes;
    if (e == cudaSuccess) e = launch_product(g, IN_PLANES, EPI_GELU_MUL, st);
  }
  if (e != cudaSuccess) return e;
  ProductArgs dn = session_product_args(s, L.down, tokens);
  dn.planes = s->planes2;
  dn.out = s->tmp;
  e = launch_product(dn, IN_PLANES, EPI_STORE, st);
  if (e != cudaSuccess) return e;
  if (tokens == 1 && m->P && m->H <= kNormPer * kNormThreads) {  // one launch for post_ffw and the PLE gate
    e = launch_gemma_post_ffw_ple_gate(s->tmp, x_attn, L.norm_post_ffw, m->eps, m->H, s->xs, L.ple_gate, m->P,
                                       s->ple_rows + (size_t)l * m->P, s->pg, st);
  } else {
    e = launch_gemma_post_ffw(s->tmp, x_attn, L.norm_post_ffw, m->eps, tokens, m->H, s->xs, st);
    if (e == cudaSuccess)
      e = launch_dense(L.ple_gate, m->P, m->H, s->xs, m->H, tokens, s->pg, m->P,
                       s->ple_rows + (size_t)l * m->P, m->L * m->P, st);
  }
  if (e != cudaSuccess) return e;
  // one launch for the PLE projection and the finish where the row is wide
  // (measured: Gemma-2B's 2048 values 586 -> 593 tok/s; the tiny config's 256
  // were 2 % slower, the finishing block's norm then outlasting a launch)
  if (tokens == 1 && m->P && m->H >= 1024 && m->H <= kNormPer * kNormThreads)
    return launch_gemma_ple_proj_finish(s->pg, L.ple_proj, m->P, m->H, s->tmp, s->xs, L.ple_post_norm, m->eps,
                                        L.layer_scalar, s->x, s->ple_done, st);
  e = launch_dense(L.ple_proj, m->H, m->P, s->pg, m->P, tokens, s->tmp, m->H, nullptr, 0, st);
  if (e == cudaSuccess)
    e = launch_gemma_finish(s->tmp, s->xs, L.ple_post_norm, m->eps, L.layer_scalar, tokens, m->H, s->x, st);
  return e;
}

// Embeds the ids in s->d_ids (or *d_token) into s->x, prepares Gemma's
// per-layer inputs, runs every layer and the head over the last row.
cudaError_t run_pass(IrisSession* s, uint32_t tokens, const uint32_t* ids_dev, const uint32_t* pos_ptr,
                     uint32_t pos0, bool head, bool store_logits) {
  IrisModel* m = s->m;
  cudaStream_t st = s->stream;
  bool gemma = m->family == kFamilyGemma;
  cudaError_t e = launch_embed(m->embed, ids_dev, tokens, gemma, m->embedding_scale, s->x, st);
  if (e != cudaSuccess) return e;
  if (gemma) {  // view_kernels.rs:59-99, every layer's PLE row for these tokens
    e = launch_dense(m->ple_model_proj, m->L * m->P, m->H, s->x, m->H, tokens, s->ple_proj, m->L * m->P,
                     nullptr, 0, st);
    if (e == cudaSuccess)
      e = launch_ple_prepare(s->ple_proj, m->ple_embed, ids_dev, m->ple_norm, m->eps, m->ple_projection_scalar,
                             m->ple_embedding_scale, m->ple_input_scale, tokens, m->L, m->P, s->ple_rows, st);
    if (e != cudaSuccess) return e;
  }
  for (uint32_t l = 0; l < m->L; ++l) {
    e = gemma ? gemma_layer(s, l, tokens, pos_ptr, pos0) : mistral_layer(s, l, tokens, pos_ptr, pos0);
    if (e != cudaSuccess) return e;
  }
  if (!head) return cudaSuccess;
  // head: rms_norm(final) -> dot_row over the vocabulary -> softcap -> first max
  ProductArgs h = session_product_args(s, m->head, 1);
  h.x = s->x + (size_t)(tokens - 1) * m->H;
  h.norm_w = m->final_norm;
  h.eps = m->eps;
  h.out = store_logits ? s->logits : nullptr;
  h.best = s->best;
  h.softcap = m->softcap;
  h.row_base = m->tp_rank * m->V;  // vocabulary shard
  e = launch_product(h, IN_NORM, EPI_LOGITS, st, IRIS_PATH_GEMV);
  if (e == cudaSuccess && m->tp_world > 1) e = tp_max_keys(m->comm, s->best, 1, st);
  return e;
}

// IRIS_ESTALL when a kernel recorded a given-up wait since the last check.
int check_fault() {
  uint32_t fault = 0;
  cudaError_t e = take_device_fault(&fault);
  if (e != cudaSuccess) return (int)e;
  return fault ? IRIS_ESTALL : 0;
}

// The last pass's logits (the whole vocabulary) to the host, asynchronously on
// the session stream; every rank of a tensor-parallel model takes part.
cudaError_t copy_logits(IrisSession* s, int32_t* host) {
  IrisModel* m = s->m;
  if (m->tp_world > 1) {
    cudaError_t e = tp_gather_i32(m->comm, s->logits, s->logits_full, m->V, s->stream);
    if (e != cudaSuccess) return e;
    return cudaMemcpyAsync(host, s->logits_full, (size_t)m->Vfull * 4, cudaMemcpyDeviceToHost, s->stream);
  }
  return cudaMemcpyAsync(host, s->logits, (size_t)m->V * 4, cudaMemcpyDeviceToHost, s->stream);
}

int prefill_ids(IrisSession* s, const uint32_t* ids, uint32_t n, int32_t* logits, uint32_t* token) {
  IrisModel* m = s->m;
  if (n == 0) return IRIS_EINVAL;
  if ((uint64_t)s->len + n > s->cap || (uint64_t)s->len + n > m->max_positions) return IRIS_ERANGE;
  for (uint32_t i = 0; i < n; ++i)
    if (ids[i] >= m->Vfull) return IRIS_EINVAL;
  cudaError_t e = cudaSuccess;
  for (uint32_t r0 = 0; r0 < n && e == cudaSuccess; r0 += kMaxRows) {
    uint32_t cnt = std::min(kMaxRows, n - r0);
    e = cudaMemcpyAsync(s->d_ids, ids + r0, cnt * 4, cudaMemcpyHostToDevice, s->stream);
    bool last = r0 + cnt == n;
    if (e == cudaSuccess) e = run_pass(s, cnt, s->d_ids, nullptr, s->len + r0, last, logits != nullptr);
  }
  unsigned long long key = 0;
  if (e == cudaSuccess) e = cudaMemcpyAsync(&key, s->best, 8, cudaMemcpyDeviceToHost, s->stream);
  if (e == cudaSuccess && logits) e = copy_logits(s, logits);
  if (e == cudaSuccess) e = launch_fill_u64(s->best, 1, s->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s->stream);
  if (e != cudaSuccess) return (int)e;
  int rc = check_fault();
  if (rc) return rc;
  s->len += n;
  s->has_logits = true;
  uint32_t tok = best_key_token(key);
  if (token) *token = tok;
  // device state for the decode graph: next input token and its position
  uint32_t state[2] = {tok, s->len};
  e = cudaMemcpy(s->d_token, &state[0], 4, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(s->d_pos, &state[1], 4, cudaMemcpyHostToDevice);
  return (int)e;
}

int ensure_graph(IrisSession* s) {
  if (s->graph) return 0;
  {  // the one-scale-a-row flags of the pass's products, taken before the capture
    IrisModel* m = s->m;
    for (uint32_t l = 0; l < m->L; ++l)
      for (Q8GpuMatrix* w : {m->layers[l].qkv, m->layers[l].o, m->layers[l].gu, m->layers[l].down})
        if (w) q8_uniform_cached(w, s->stream);
    if (m->head) q8_uniform_cached(m->head, s->stream);
  }
  cudaGraph_t g = nullptr;
  cudaError_t e = cudaStreamBeginCapture(s->stream, cudaStreamCaptureModeThreadLocal);
  if (e != cudaSuccess) return (int)e;
  cudaError_t body = run_pass(s, 1, s->d_token, s->d_pos, 0, true, true);
  if (body == cudaSuccess)
    body = launch_decode_finish(s->best, s->d_token, s->d_pos, s->d_step, s->d_history, s->history_cap, s->stream);
  e = cudaStreamEndCapture(s->stream, &g);
  if (body != cudaSuccess) {
    if (g) cudaGraphDestroy(g);
    return (int)body;
  }
  if (e != cudaSuccess) return (int)e;
  e = cudaGraphInstantiate(&s->graph, g, 0);
  cudaGraphDestroy(g);
  return (int)e;
}

// The persistent step's one-scale-a-row flags of every product stage whose
// matrix changed since they were taken (weights written after the session
// was made), copied to the device stage list before the next pass.
cudaError_t refresh_step_flags(IrisSession* s) {
  bool stale = false;
  for (size_t i = 0; i < s->step_mats.size(); ++i)
    stale |= s->step_mats[i] && q8_version(s->step_mats[i]) != s->step_versions[i];
  if (!stale) return cudaSuccess;
  cudaError_t e = cudaDeviceSynchronize();  // weight writes may have run on any stream
  for (size_t i = 0; i < s->step_mats.size() && e == cudaSuccess; ++i) {
    const Q8GpuMatrix* w = s->step_mats[i];
    if (!w) continue;
    const uint32_t v = q8_version(w);
    if (v == s->step_versions[i]) continue;
    s->step_host[i].uniform = q8_uniform_cached(const_cast<Q8GpuMatrix*>(w), s->stream) ? 1u : 0u;
    s->step_versions[i] = v;
  }
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(s->stages, s->step_host.data(), s->step_host.size() * sizeof(StepStage),
                        cudaMemcpyHostToDevice, s->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s->stream);  // the host copy may change again
  return e;
}

// Replays the decode graph `steps` times (positions len, len+1, ...).
int decode_steps(IrisSession* s, uint32_t steps) {
  if (!s->has_logits) return IRIS_ESTATE;
  if ((uint64_t)s->len + steps > s->cap || (uint64_t)s->len + steps > s->m->max_positions) return IRIS_ERANGE;
  choose_decode_path(s);
  if (s->use_step) {
    const StepArgs a = step_args(s);
    cudaError_t e = refresh_step_flags(s);
    bool uniform = true;
    for (size_t i = 0; i < s->step_mats.size(); ++i) uniform &= !s->step_mats[i] || s->step_host[i].uniform;
    if (e == cudaSuccess) e = cudaMemsetAsync(s->sync, 0, s->nstages * sizeof(unsigned int), s->stream);
    if (e == cudaSuccess)
      e = cudaMemsetAsync(s->gready, 0, (size_t)s->m->L * (s->m->heads / s->step.hpc) * sizeof(unsigned int),
                          s->stream);
    for (uint32_t i = 0; i < steps && e == cudaSuccess; ++i) e = launch_decode_step(a, s->step, uniform, s->stream);
    if (e != cudaSuccess) return (int)e;
    s->len += steps;
    return 0;
  }
  int rc = ensure_graph(s);
  if (rc) return rc;
  for (uint32_t i = 0; i < steps; ++i) {
    cudaError_t e = cudaGraphLaunch(s->graph, s->stream);
    if (e != cudaSuccess) return (int)e;
  }
  s->len += steps;
  return 0;
}

int check_model_ready(const IrisModel* m) {
  if (!m->embed || !m->head || !m->final_norm) return IRIS_ESTATE;
  for (const LayerDev& L : m->layers)
    if (!L.qkv || !L.o || !L.gu || !L.down || !L.norm_attn || !L.norm_ffn) return IRIS_ESTATE;
  return 0;
}

// Model tensor plumbing ------------------------------------------------------

struct Q8Target {
  Q8GpuMatrix* m;
  uint32_t rows, cols, stride, offset;
  // the block of the full tensor these rows hold (tensor-parallel shards)
  uint32_t src_row0 = 0, src_col0 = 0, full_cols = 0;
};

int q8_target(IrisModel* m, int tensor, int32_t layer, Q8Target* t) {
  const uint32_t r = m->tp_rank, W = m->tp_world;
  auto set = [&](Q8GpuMatrix* mat, uint32_t rows, uint32_t cols, uint32_t stride, uint32_t offset, uint32_t row0,
                 uint32_t col0, uint32_t full_cols) {
    t->m = mat;
    t->rows = rows;
    t->cols = cols;
    t->stride = stride;
    t->offset = offset;
    t->src_row0 = row0;
    t->src_col0 = col0;
    t->full_cols = full_cols;
    return 0;
  };
  if (tensor == IRIS_T_EMBED) return set(m->embed, m->Vfull, m->H, 1, 0, 0, 0, m->H);
  if (tensor == IRIS_T_HEAD) {
    if (m->tied) return IRIS_EINVAL;
    return set(m->head, m->V, m->H, 1, 0, r * m->V, 0, m->H);
  }
  if (tensor == IRIS_T_PLE_EMBED) {
    if (m->family != kFamilyGemma) return IRIS_EINVAL;
    return set(m->ple_embed, m->V, m->L * m->P, 1, 0, 0, 0, m->L * m->P);
  }
  if (layer < 0 || (uint32_t)layer >= m->L) return IRIS_EINVAL;
  LayerDev& L = m->layers[layer];
  switch (tensor) {
    case IRIS_T_W_Q: return set(L.qkv, m->qd, m->H, 1, 0, r * m->qd, 0, m->H);
    case IRIS_T_W_K: return set(L.qkv, m->kvd, m->H, 1, m->qd, r * m->kvd, 0, m->H);
    case IRIS_T_W_V: return set(L.qkv, m->kvd, m->H, 1, m->qd + m->kvd, r * m->kvd, 0, m->H);
    case IRIS_T_W_O: return set(L.o, m->H, m->qd, 1, 0, 0, r * m->qd, W * m->qd);
    case IRIS_T_W_GATE: return set(L.gu, m->F, m->H, 2, 0, r * m->F, 0, m->H);
    case IRIS_T_W_UP: return set(L.gu, m->F, m->H, 2, 1, r * m->F, 0, m->H);
    case IRIS_T_W_DOWN: return set(L.down, m->H, m->F, 1, 0, 0, r * m->F, W * m->F);
  }
  return IRIS_EINVAL;
}

int32_t** value_target(IrisModel* m, int tensor, int32_t layer, uint64_t* count, uint32_t* fan_in) {
  *fan_in = 0;
  if (tensor == IRIS_T_FINAL_NORM) { *count = m->H; return &m->final_norm; }
  if (tensor == IRIS_T_PLE_MODEL_PROJECTION && m->family == kFamilyGemma) {
    *count = (uint64_t)m->L * m->P * m->H;
    *fan_in = m->H;
    return &m->ple_model_proj;
  }
  if (tensor == IRIS_T_PLE_NORM && m->family == kFamilyGemma) { *count = m->P; return &m->ple_norm; }
  if (layer < 0 || (uint32_t)layer >= m->L) return nullptr;
  LayerDev& L = m->layers[layer];
  bool g = m->family == kFamilyGemma;
  switch (tensor) {
    case IRIS_T_NORM_ATTN: *count = m->H; return &L.norm_attn;
    case IRIS_T_NORM_FFN: *count = m->H; return &L.norm_ffn;
  }
  if (!g) return nullptr;
  switch (tensor) {
    case IRIS_T_NORM_POST_ATTN: *count = m->H; return &L.norm_post_attn;
    case IRIS_T_NORM_POST_FFW: *count = m->H; return &L.norm_post_ffw;
    case IRIS_T_Q_NORM: *count = m->d; return &L.q_norm;
    case IRIS_T_K_NORM: *count = m->d; return &L.k_norm;
    case IRIS_T_PLE_POST_NORM: *count = m->H; return &L.ple_post_norm;
    case IRIS_T_PLE_INPUT_GATE: *count = (uint64_t)m->P * m->H; *fan_in = m->H; return &L.ple_gate;
    case IRIS_T_PLE_LAYER_PROJECTION: *count = (uint64_t)m->H * m->P; *fan_in = m->P; return &L.ple_proj;
  }
  return nullptr;
}

int alloc_layers(IrisModel* m) {
  cudaError_t e = cudaSuccess;
  auto q8 = [&](uint32_t rows, uint32_t cols) -> Q8GpuMatrix* {
    if (e != cudaSuccess) return nullptr;
    Q8GpuMatrix* r = alloc_q8(rows, cols, &e);
    if (r) m->weight_bytes += (uint64_t)rows * cols + (uint64_t)rows * (cols / 32) * 2;
    return r;
  };
  m->embed = q8(m->Vfull, m->H);
  m->head = m->tied ? m->embed : q8(m->V, m->H);
  if (e == cudaSuccess) e = dalloc(&m->final_norm, m->H);
  for (uint32_t l = 0; l < m->L; ++l) {
    LayerDev& L = m->layers[l];
    L.qkv = q8(m->qd + 2 * m->kvd, m->H);
    L.o = q8(m->H, m->qd);
    L.gu = q8(2 * m->F, m->H);
    L.down = q8(m->H, m->F);
    if (e == cudaSuccess) e = dalloc(&L.norm_attn, m->H);
    if (e == cudaSuccess) e = dalloc(&L.norm_ffn, m->H);
    if (m->family == kFamilyGemma) {
      if (e == cudaSuccess) e = dalloc(&L.norm_post_attn, m->H);
      if (e == cudaSuccess) e = dalloc(&L.norm_post_ffw, m->H);
      if (e == cudaSuccess) e = dalloc(&L.q_norm, m->d);
      if (e == cudaSuccess) e = dalloc(&L.k_norm, m->d);
      if (e == cudaSuccess) e = dalloc(&L.ple_post_norm, m->H);
      if (e == cudaSuccess) e = dalloc(&L.ple_gate, (size_t)m->P * m->H);
      if (e == cudaSuccess) e = dalloc(&L.ple_proj, (size_t)m->H * m->P);
      m->weight_bytes += (uint64_t)2 * m->P * m->H * 4;
    }
  }
  if (m->family == kFamilyGemma) {
    m->ple_embed = q8(m->V, m->L * m->P);
    if (e == cudaSuccess) e = dalloc(&m->ple_model_proj, (size_t)m->L * m->P * m->H);
    if (e == cudaSuccess) e = dalloc(&m->ple_norm, m->P);
    m->weight_bytes += (uint64_t)m->L * m->P * m->H * 4;
  }
  if (e == cudaSuccess) e = prepare_product_kernels();
  if (e == cudaSuccess) e = prepare_layer_kernels();
  if (e == cudaSuccess) e = prepare_attn_tc_kernels();
  return (int)e;
}

}  // namespace

extern "C" {

void iris_model_free(IrisModel* m) {
  if (!m) return;
  free_session(m->scratch);
  if (m->head != m->embed) free_q8(m->head);
  free_q8(m->embed);
  free_q8(m->ple_embed);
  cudaFree(m->final_norm);
  cudaFree(m->ple_model_proj);
  cudaFree(m->ple_norm);
  cudaFree(m->freqs);
  for (LayerDev& L : m->layers) {
    free_q8(L.qkv);
    free_q8(L.o);
    free_q8(L.gu);
    free_q8(L.down);
    void* ptrs[] = {L.norm_attn, L.norm_ffn, L.norm_post_attn, L.norm_post_ffw, L.q_norm, L.k_norm,
                    L.ple_post_norm, L.ple_gate, L.ple_proj, L.inv_freq};
    for (void* p : ptrs) cudaFree(p);
  }
  if (m->xch.world) tp_exchange_free(&m->xch);
  tp_comm_free(m->comm);
  delete m;
}

static int create_mistral(const IrisMistralShape* sh, uint32_t rank, uint32_t world, const uint8_t* nccl_id,
                          IrisModel** out) {
  *out = nullptr;
  if (!sh || !sh->layers || !sh->hidden || !sh->ffn || !sh->heads || !sh->kv_heads || !sh->head_dim ||
      !sh->vocab || sh->heads % sh->kv_heads || sh->head_dim % 4 || sh->hidden % 32 || sh->ffn % 32 ||
      (sh->heads * sh->head_dim) % 32 || sh->norm_eps < 0 || !sh->rope_inverse_frequencies ||
      sh->heads / sh->kv_heads > 16)
    return IRIS_EINVAL;
  // a shard: whole kv groups, FFN rows and vocabulary rows in 32-multiples
  // where they are product columns (o, down); the tied head is not sharded
  if (world == 0 || rank >= world ||
      (world > 1 && (sh->kv_heads % world || sh->ffn % (32 * world) || sh->vocab % world || sh->tied_head ||
                     ((sh->heads / world) * sh->head_dim) % 32 || !nccl_id)))
    return IRIS_EINVAL;
  for (uint32_t i = 0; i < sh->head_dim / 2; ++i)  // layer.rs:71-78
    if (sh->rope_inverse_frequencies[i] < 0 || sh->rope_inverse_frequencies[i] > ((int64_t)1 << 32))
      return IRIS_EINVAL;
  IrisModel* m = new IrisModel();
  m->family = kFamilyMistral;
  m->tp_rank = rank;
  m->tp_world = world;
  m->L = sh->layers;
  m->H = sh->hidden;
  m->F = sh->ffn / world;
  m->heads = sh->heads / world;
  m->kvh = sh->kv_heads / world;
  m->d = sh->head_dim;
  m->V = sh->vocab / world;
  m->Vfull = sh->vocab;
  m->max_positions = sh->max_positions;
  m->qd = m->heads * m->d;
  m->kvd = m->kvh * m->d;
  m->eps = sh->norm_eps;
  m->scale_q32 = sh->attention_scale_q32;
  m->tied = sh->tied_head != 0;
  m->layers.resize(m->L);
  int rc = 0;
  if (world > 1) rc = (int)tp_comm_init(&m->comm, rank, world, nccl_id);
  if (world > 1 && rc == 0) rc = (int)tp_exchange_setup(m->comm, rank, world, m->H, &m->xch, device_fault_word());
  if (rc == 0) rc = alloc_layers(m);
  if (rc == 0) rc = (int)dalloc(&m->freqs, m->d / 2);
  if (rc == 0)
    rc = (int)cudaMemcpy(m->freqs, sh->rope_inverse_frequencies, (m->d / 2) * 8, cudaMemcpyHostToDevice);
  if (rc) {
    iris_model_free(m);
    return rc;
  }
  *out = m;
  return 0;
}

int iris_model_create_mistral(const IrisMistralShape* sh, IrisModel** out) {
  if (!out) return IRIS_EINVAL;
  return create_mistral(sh, 0, 1, nullptr, out);
}

int iris_model_create_mistral_tp(const IrisMistralShape* sh, uint32_t rank, uint32_t world, const uint8_t* nccl_id,
                                 IrisModel** out) {
  if (!out || world > kTpMaxWorld) return IRIS_EINVAL;
  return create_mistral(sh, rank, world, nccl_id, out);
}

int iris_model_set_tp_exchange(IrisModel* m, int mode) {
  if (!m || m->tp_world < 2 || (mode != IRIS_TP_PEER && mode != IRIS_TP_NCCL)) return IRIS_EINVAL;
  m->xch_nccl = mode == IRIS_TP_NCCL;
  return 0;
}

int iris_model_create_gemma(const IrisGemmaShape* sh, IrisModel** out) {
  *out = nullptr;
  if (!sh || !sh->layers || !sh->hidden || !sh->ffn || !sh->heads || !sh->kv_heads || !sh->head_dim ||
      !sh->vocab || !sh->ple_width || sh->heads % sh->kv_heads || sh->head_dim % 4 || sh->hidden % 32 ||
      sh->ffn % 32 || (sh->heads * sh->head_dim) % 32 || sh->ple_width % 32 || sh->norm_eps < 0 ||
      sh->heads / sh->kv_heads > 16 || !sh->sliding_window || !sh->rope_base || !sh->rotary_dim ||
      !sh->rope_freq_base_dim || !sh->kv_donor_layer || !sh->layer_scalar)
    return IRIS_EINVAL;
  for (uint32_t l = 0; l < sh->layers; ++l) {  // prefill_range.rs:403-484
    uint32_t rd = sh->rotary_dim[l], fbd = sh->rope_freq_base_dim[l];
    if (rd % 2 || rd > sh->head_dim) return IRIS_EINVAL;
    if (rd && (fbd < 2 || fbd % 2 || sh->rope_base[l] <= 0)) return IRIS_EINVAL;
    int32_t donor = sh->kv_donor_layer[l];
    if (donor >= (int32_t)l || donor < -1) return IRIS_EINVAL;
    if (donor >= 0 && sh->kv_donor_layer[donor] >= 0) return IRIS_EINVAL;
  }
  IrisModel* m = new IrisModel();
  m->family = kFamilyGemma;
  m->L = sh->layers;
  m->H = sh->hidden;
  m->F = sh->ffn;
  m->heads = sh->heads;
  m->kvh = sh->kv_heads;
  m->d = sh->head_dim;
  m->V = sh->vocab;
  m->Vfull = sh->vocab;
  m->P = sh->ple_width;
  m->max_positions = UINT32_MAX;
  m->qd = m->heads * m->d;
  m->kvd = m->kvh * m->d;
  m->eps = sh->norm_eps;
  m->tied = sh->tied_head != 0;  // direct/src/model.rs:577-597 (tie_word_embeddings)
  m->embedding_scale = sh->embedding_scale;
  m->ple_embedding_scale = sh->ple_embedding_scale;
  m->ple_projection_scalar = sh->ple_projection_scalar;
  m->ple_input_scale = sh->ple_input_scale;
  m->softcap = sh->final_logit_softcap;
  m->layers.resize(m->L);
  int rc = alloc_layers(m);
  for (uint32_t l = 0; l < m->L && rc == 0; ++l) {
    LayerDev& L = m->layers[l];
    L.window = sh->sliding_window[l];
    L.rotary_dim = sh->rotary_dim[l];
    L.freq_base_dim = sh->rope_freq_base_dim[l];
    L.rope_base = sh->rope_base[l];
    L.kv_donor = sh->kv_donor_layer[l];
    L.layer_scalar = sh->layer_scalar[l];
    uint32_t half = L.rotary_dim / 2;
    if (half) {
      std::vector<int64_t> f = rope_inverse_frequencies(L.rope_base, L.freq_base_dim, half);
      rc = (int)dalloc(&L.inv_freq, half);
      if (rc == 0) rc = (int)cudaMemcpy(L.inv_freq, f.data(), half * 8, cudaMemcpyHostToDevice);
    }
  }
  if (rc) {
    iris_model_free(m);
    return rc;
  }
  *out = m;
  return 0;
}

int iris_model_set_q8(IrisModel* m, int tensor, int32_t layer, const uint8_t* blocks, uint64_t bytes) {
  if (!m || !blocks || m->tp_world > 1) return IRIS_EINVAL;  // shards are synthesized on the device
  Q8Target t;
  int rc = q8_target(m, tensor, layer, &t);
  if (rc) return rc;
  if (bytes != (uint64_t)t.rows * (t.cols / 32) * 34) return IRIS_EINVAL;
  int bad = 0;
  cudaError_t e = upload_q8_blocks(t.m, blocks, t.rows, t.cols, t.stride, t.offset, &bad);
  if (e != cudaSuccess) return (int)e;
  return bad ? IRIS_ESCALE : 0;
}

int iris_model_get_q8(const IrisModel* mc, int tensor, int32_t layer, uint8_t* blocks, uint64_t bytes) {
  IrisModel* m = const_cast<IrisModel*>(mc);
  if (!m || !blocks || m->tp_world > 1) return IRIS_EINVAL;
  Q8Target t;
  int rc = q8_target(m, tensor, layer, &t);
  if (tensor == IRIS_T_HEAD && m->tied) {
    t = Q8Target{m->head, m->V, m->H, 1, 0};
    rc = 0;
  }
  if (rc) return rc;
  if (bytes != (uint64_t)t.rows * (t.cols / 32) * 34) return IRIS_EINVAL;
  return (int)download_q8_blocks(t.m, blocks, t.rows, t.cols, t.stride, t.offset);
}

int iris_model_set_values(IrisModel* m, int tensor, int32_t layer, const int32_t* values, uint64_t count) {
  if (!m || !values) return IRIS_EINVAL;
  uint64_t want;
  uint32_t fan;
  int32_t** dst = value_target(m, tensor, layer, &want, &fan);
  if (!dst || count != want) return IRIS_EINVAL;
  return (int)cudaMemcpy(*dst, values, count * 4, cudaMemcpyHostToDevice);
}

int iris_model_get_values(const IrisModel* mc, int tensor, int32_t layer, int32_t* values, uint64_t count) {
  IrisModel* m = const_cast<IrisModel*>(mc);
  if (!m || !values) return IRIS_EINVAL;
  uint64_t want;
  uint32_t fan;
  int32_t** src = value_target(m, tensor, layer, &want, &fan);
  if (!src || count != want) return IRIS_EINVAL;
  return (int)cudaMemcpy(values, *src, count * 4, cudaMemcpyDeviceToHost);
}

int iris_model_synthesize(IrisModel* m, uint64_t seed, int per_block) {
  if (!m) return IRIS_EINVAL;
  cudaError_t e = cudaSuccess;
  auto q8 = [&](int tensor, int32_t layer) {
    Q8Target t;
    if (e != cudaSuccess || q8_target(m, tensor, layer, &t)) return;
    e = synth_q8_block(t.m, seed, (uint32_t)tensor, layer, t.rows, t.cols, t.src_row0, t.src_col0, t.full_cols,
                       t.stride, t.offset, per_block, 0);
  };
  auto vals = [&](int tensor, int32_t layer) {
    uint64_t count;
    uint32_t fan;
    int32_t** dst = value_target(m, tensor, layer, &count, &fan);
    if (e != cudaSuccess || !dst) return;
    e = synth_values_dev(*dst, seed, (uint32_t)tensor, layer, count, fan, 0);
  };
  q8(IRIS_T_EMBED, -1);
  if (!m->tied) q8(IRIS_T_HEAD, -1);
  vals(IRIS_T_FINAL_NORM, -1);
  if (m->family == kFamilyGemma) {
    q8(IRIS_T_PLE_EMBED, -1);
    vals(IRIS_T_PLE_MODEL_PROJECTION, -1);
    vals(IRIS_T_PLE_NORM, -1);
  }
  for (uint32_t l = 0; l < m->L; ++l) {
    for (int t : {IRIS_T_W_Q, IRIS_T_W_K, IRIS_T_W_V, IRIS_T_W_O, IRIS_T_W_GATE, IRIS_T_W_UP, IRIS_T_W_DOWN})
      q8(t, (int32_t)l);
    for (int t : {IRIS_T_NORM_ATTN, IRIS_T_NORM_FFN, IRIS_T_NORM_POST_ATTN, IRIS_T_NORM_POST_FFW, IRIS_T_Q_NORM,
                  IRIS_T_K_NORM, IRIS_T_PLE_POST_NORM, IRIS_T_PLE_INPUT_GATE, IRIS_T_PLE_LAYER_PROJECTION})
      vals(t, (int32_t)l);
  }
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  return (int)e;
}

uint64_t iris_model_weight_bytes(const IrisModel* m) { return m ? m->weight_bytes : 0; }

int iris_model_set_gemm(IrisModel* m, int mode) {
  if (!m || (mode != IRIS_GEMM_AUTO && mode != IRIS_GEMM_MMA)) return IRIS_EINVAL;
  m->gemm_mode = mode;
  return 0;
}

int iris_model_prepare_gemm(IrisModel* m) {
  if (!m) return IRIS_EINVAL;
  if (m->gemm_mode != IRIS_GEMM_AUTO) return 0;
  cudaError_t e = cudaSuccess;
  for (LayerDev& L : m->layers)
    for (Q8GpuMatrix* w : {L.qkv, L.o, L.gu, L.down})
      if (w && e == cudaSuccess) e = tc_prepare(w, 0);
  return (int)e;
}

int iris_model_tc_matrices(const IrisModel* m, uint64_t* bytes) {
  if (!m) return -1;
  int n = 0;
  uint64_t b = 0;
  auto count = [&](const Q8GpuMatrix* w) {
    if (w && tc_state_get(w) == 1) {
      ++n;
      b += (uint64_t)w->tc_planes * w->tc_rows * w->cols + 3ull * w->tc_rows;
    }
  };
  for (const LayerDev& L : m->layers) {
    count(L.qkv);
    count(L.o);
    count(L.gu);
    count(L.down);
  }
  count(m->head);
  if (bytes) *bytes = b;
  return n;
}

int iris_model_attention_ranges(const IrisModel* m, uint64_t* counts) {
  if (!m || !counts) return IRIS_EINVAL;
  counts[0] = m->attn_ranges[0].load(std::memory_order_relaxed);
  counts[1] = m->attn_ranges[1].load(std::memory_order_relaxed);
  return 0;
}

int iris_session_create(IrisModel* m, uint32_t max_positions, IrisSession** out) {
  if (!m || !out) return IRIS_EINVAL;
  int rc = check_model_ready(m);
  if (rc) return rc;
  return create_session(m, max_positions, out);
}

int iris_session_reset(IrisSession* s) {
  if (!s) return IRIS_EINVAL;
  if (s->copy_stream) {  // chain copies still reading the cache
    cudaError_t e = cudaStreamSynchronize(s->copy_stream);
    if (e != cudaSuccess) return (int)e;
  }
  s->len = 0;
  s->has_logits = false;
  s->range_n = 0;
  cudaError_t e = cudaMemsetAsync(s->d_pos, 0, 4, s->stream);
  if (e == cudaSuccess) e = cudaMemsetAsync(s->d_step, 0, 4, s->stream);
  if (e == cudaSuccess) e = launch_fill_u64(s->best, kMaxRows, s->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s->stream);
  return (int)e;
}

int iris_session_prefill(IrisSession* s, const uint32_t* ids, uint32_t n, int32_t* logits, uint32_t* token) {
  if (!s || !ids) return IRIS_EINVAL;
  return prefill_ids(s, ids, n, logits, token);
}

// ---- the chain's ranges, device-resident ---------------------------------

int iris_session_range_begin(IrisSession* s, const uint32_t* ids, uint32_t n) {
  if (!s || !ids || n == 0 || n > kMaxRows || s->range_n || s->m->tp_world > 1) return IRIS_EINVAL;
  IrisModel* m = s->m;
  if ((uint64_t)s->len + n > s->cap || (uint64_t)s->len + n > m->max_positions) return IRIS_ERANGE;
  for (uint32_t i = 0; i < n; ++i)
    if (ids[i] >= m->Vfull) return IRIS_EINVAL;
  cudaError_t e = cudaSuccess;
  if (!s->copy_stream) {  // the stages' copy stream, staging buffers and events, on first use
    e = cudaStreamCreateWithFlags(&s->copy_stream, cudaStreamNonBlocking);
    for (int b = 0; b < 2 && e == cudaSuccess; ++b) {
      e = dalloc(&s->stage_rows[b], (size_t)kMaxRows * m->H);
      if (e == cudaSuccess) e = cudaEventCreateWithFlags(&s->stage_read[b], cudaEventDisableTiming);
    }
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&s->staged, cudaEventDisableTiming);
    // both staging buffers start unread
    for (int b = 0; b < 2 && e == cudaSuccess; ++b) e = cudaEventRecord(s->stage_read[b], s->copy_stream);
    if (e != cudaSuccess) return (int)e;
  }
  if (e == cudaSuccess) e = cudaMemcpyAsync(s->d_ids, ids, (size_t)n * 4, cudaMemcpyHostToDevice, s->stream);
  const bool gemma = m->family == kFamilyGemma;
  if (e == cudaSuccess) e = launch_embed(m->embed, s->d_ids, n, gemma, m->embedding_scale, s->x, s->stream);
  if (gemma && e == cudaSuccess) {  // view_kernels.rs:59-99, every layer's PLE row of the range
    e = launch_dense(m->ple_model_proj, m->L * m->P, m->H, s->x, m->H, n, s->ple_proj, m->L * m->P, nullptr, 0,
                     s->stream);
    if (e == cudaSuccess)
      e = launch_ple_prepare(s->ple_proj, m->ple_embed, s->d_ids, m->ple_norm, m->eps, m->ple_projection_scalar,
                             m->ple_embedding_scale, m->ple_input_scale, n, m->L, m->P, s->ple_rows, s->stream);
  }
  if (e != cudaSuccess) return (int)e;
  s->range_n = n;
  s->range_layer = 0;
  return 0;
}

namespace {

// One leaf a thread: the SHA-256 of bytes [j leaf, min((j + 1) leaf, bytes))
// of segment s (the stage's rows, then its K rows, then its V rows), leaf
// digest i = first[s] + j at out + 32 i.
struct LeafSegments {
  const uint32_t* p[3];
  uint32_t bytes[3];
  uint32_t first[4];  // first leaf of each segment; first[3]: all leaves
};

__global__ void __launch_bounds__(128) record_leaves_kernel(LeafSegments g, uint32_t leaf, uint8_t* out) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= g.first[3]) return;
  const uint32_t sg = i < g.first[1] ? 0 : i < g.first[2] ? 1 : 2;
  const uint32_t off = (i - g.first[sg]) * leaf;
  sha256_words(g.p[sg] + off / 4, min(leaf, g.bytes[sg] - off), out + (size_t)32 * i);
}

uint32_t leaves_of(uint64_t bytes, uint32_t leaf) { return (uint32_t)((bytes + leaf - 1) / leaf); }

// A chain stage: run `layer` over the range, then on the copy stream either
// copy its rows and own K/V to the host (leaf == 0) or hash them on the
// device into leaf digests and copy those (leaf > 0); a ticket's event marks
// the copies done.
int range_layer(IrisSession* s, uint32_t layer, int32_t* rows_out, int32_t* own_k, int32_t* own_v, uint32_t leaf,
                uint8_t* leaves_out, uint32_t* ticket) {
  if (!s || !s->range_n || layer != s->range_layer) return s ? IRIS_ESTATE : IRIS_EINVAL;
  IrisModel* m = s->m;
  const uint32_t n = s->range_n, start = s->len;
  const size_t kvd = m->kvd;
  cudaError_t e = cudaSuccess;
  if (leaf) {  // leaf digest buffers for a whole range at this leaf size
    const uint32_t need = leaves_of((uint64_t)kMaxRows * m->H * 4, leaf) + 2 * leaves_of((uint64_t)kMaxRows * kvd * 4, leaf);
    if (need > s->leaves_cap) {
      e = cudaStreamSynchronize(s->copy_stream);
      for (int b = 0; b < 2 && e == cudaSuccess; ++b) {
        cudaFree(s->stage_leaves[b]);
        s->stage_leaves[b] = nullptr;
        e = dalloc(&s->stage_leaves[b], (size_t)need * 32);
      }
      if (e != cudaSuccess) return (int)e;
      s->leaves_cap = need;
    }
  }
  e = m->family == kFamilyGemma ? gemma_layer(s, layer, n, nullptr, start, true)
                                : mistral_layer(s, layer, n, nullptr, start);
  // the stage's rows into staging buffer b once the copy stream has read it,
  // then every copy (or the hashing) on the copy stream while the next layer runs
  const uint32_t t = s->next_ticket.load(), b = t & 1;
  if (e == cudaSuccess) e = cudaStreamWaitEvent(s->stream, s->stage_read[b], 0);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(s->stage_rows[b], s->x, (size_t)n * m->H * 4, cudaMemcpyDeviceToDevice, s->stream);
  if (e == cudaSuccess) e = cudaEventRecord(s->staged, s->stream);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(s->copy_stream, s->staged, 0);
  const int32_t* kown = s->kc + kv_offset(s, layer) + (size_t)start * kvd;
  const int32_t* vown = s->vc + kv_offset(s, layer) + (size_t)start * kvd;
  if (leaf) {
    LeafSegments g{};
    g.p[0] = (const uint32_t*)s->stage_rows[b];
    g.p[1] = (const uint32_t*)kown;
    g.p[2] = (const uint32_t*)vown;
    g.bytes[0] = n * m->H * 4;
    g.bytes[1] = g.bytes[2] = (uint32_t)(n * kvd * 4);
    g.first[0] = 0;
    for (int sg = 0; sg < 3; ++sg) g.first[sg + 1] = g.first[sg] + leaves_of(g.bytes[sg], leaf);
    if (e == cudaSuccess)
      e = launch_k(record_leaves_kernel, dim3((g.first[3] + 127) / 128), dim3(128), 0, s->copy_stream, g, leaf,
                   s->stage_leaves[b]);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(leaves_out, s->stage_leaves[b], (size_t)g.first[3] * 32, cudaMemcpyDeviceToHost,
                          s->copy_stream);
  } else {
    if (e == cudaSuccess && rows_out)
      e = cudaMemcpyAsync(rows_out, s->stage_rows[b], (size_t)n * m->H * 4, cudaMemcpyDeviceToHost,
                          s->copy_stream);
    if (e == cudaSuccess && own_k)
      e = cudaMemcpyAsync(own_k, kown, (size_t)n * kvd * 4, cudaMemcpyDeviceToHost, s->copy_stream);
    if (e == cudaSuccess && own_v)
      e = cudaMemcpyAsync(own_v, vown, (size_t)n * kvd * 4, cudaMemcpyDeviceToHost, s->copy_stream);
  }
  if (e == cudaSuccess) e = cudaEventRecord(s->stage_read[b], s->copy_stream);
  if (e == cudaSuccess) {
    cudaEvent_t& ev = s->tickets[t % kChainTickets];
    // a thread waiting on a ticket sleeps (blocking sync) instead of spinning
    // on a host core the record hashing needs
    if (!ev) e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming | cudaEventBlockingSync);
    if (e == cudaSuccess) e = cudaEventRecord(ev, s->copy_stream);
    if (e == cudaSuccess) s->next_ticket.store(t + 1);  // published after the event is recorded
    if (ticket) *ticket = t;
  }
  if (e != cudaSuccess) return (int)e;
  s->range_layer = layer + 1;
  return 0;
}

}  // namespace

int iris_session_range_layer(IrisSession* s, uint32_t layer, int32_t* rows_out, int32_t* own_k, int32_t* own_v,
                             uint32_t* ticket) {
  return range_layer(s, layer, rows_out, own_k, own_v, 0, nullptr, ticket);
}

int iris_session_range_layer_leaves(IrisSession* s, uint32_t layer, uint32_t leaf_bytes, uint8_t* leaves_out,
                                    uint32_t* ticket) {
  if (!leaves_out || leaf_bytes < 64 || leaf_bytes % 64 || leaf_bytes > (1u << 20)) return IRIS_EINVAL;
  return range_layer(s, layer, nullptr, nullptr, nullptr, leaf_bytes, leaves_out, ticket);
}

int iris_session_range_layers_leaves(IrisSession* s, uint32_t count, uint32_t leaf_bytes, uint8_t* const* leaves_out,
                                     uint32_t* tickets) {
  if (!s || !leaves_out || !tickets || count > kChainTickets) return IRIS_EINVAL;
  for (uint32_t i = 0; i < count; ++i) {
    const int rc = iris_session_range_layer_leaves(s, s->range_layer, leaf_bytes, leaves_out[i], tickets + i);
    if (rc) return rc;
  }
  return 0;
}

int iris_session_ticket_wait(IrisSession* s, uint32_t ticket) {
  if (!s) return IRIS_EINVAL;
  const uint32_t issued = s->next_ticket.load();
  if (ticket >= issued || issued - ticket > kChainTickets) return IRIS_EINVAL;
  cudaEvent_t ev = s->tickets[ticket % kChainTickets];
  return ev ? (int)cudaEventSynchronize(ev) : IRIS_EINVAL;
}

int iris_session_range_end(IrisSession* s, uint32_t* token_ids, int32_t* values) {
  if (!s) return IRIS_EINVAL;
  IrisModel* m = s->m;
  if (!s->range_n || s->range_layer != m->L) return IRIS_ESTATE;
  const uint32_t n = s->range_n;
  cudaStream_t st = s->stream;
  cudaError_t e = cudaSuccess;
  std::vector<unsigned long long> keys(n);
  if (token_ids) {  // rms_norm(final), the head, softcap, first maximum per row (sequence_check.rs:232-300)
    e = launch_planes(s->x, m->final_norm, m->eps, n, m->H, s->planes, st);
    if (e == cudaSuccess) e = launch_fill_u64(s->best, n, st);
    if (e == cudaSuccess) {
      ProductArgs h = session_product_args(s, m->head, n);
      h.planes = s->planes;
      h.out = nullptr;
      h.best = s->best;
      h.softcap = m->softcap;
      e = launch_product(h, IN_PLANES, EPI_LOGITS, st);
    }
    if (e == cudaSuccess) e = cudaMemcpyAsync(keys.data(), s->best, (size_t)n * 8, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = launch_fill_u64(s->best, n, st);
  }
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return (int)e;
  int rc = check_fault();
  if (rc) return rc;
  for (uint32_t i = 0; token_ids && i < n; ++i) {
    token_ids[i] = best_key_token(keys[i]);
    if (values) values[i] = best_key_value(keys[i]);
  }
  s->len += n;
  s->range_n = 0;
  s->has_logits = false;  // a decode pass needs a prefill's state
  return 0;
}

int iris_host_alloc(uint64_t bytes, void** out) {
  if (!out) return IRIS_EINVAL;
  *out = nullptr;
  return (int)cudaHostAlloc(out, bytes ? bytes : 1, cudaHostAllocDefault);
}

void iris_host_free(void* p) {
  if (p) cudaFreeHost(p);
}

int iris_session_decode(IrisSession* s, uint32_t token_in, int32_t* logits, uint32_t* token_out) {
  if (!s) return IRIS_EINVAL;
  if (token_in >= s->m->Vfull) return IRIS_EINVAL;
  if (!s->has_logits) return IRIS_ESTATE;
  cudaError_t e = cudaMemcpyAsync(s->d_token, &token_in, 4, cudaMemcpyHostToDevice, s->stream);
  if (e != cudaSuccess) return (int)e;
  int rc = decode_steps(s, 1);
  if (rc) return rc;
  uint32_t tok = 0;
  e = cudaMemcpyAsync(&tok, s->d_token, 4, cudaMemcpyDeviceToHost, s->stream);
  if (e == cudaSuccess && logits) e = copy_logits(s, logits);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s->stream);
  if (e == cudaSuccess && token_out) *token_out = tok;
  return (int)e;
}

int iris_generate(IrisSession* s, const uint32_t* prompt, uint32_t n_prompt, uint32_t max_tokens,
                  const uint32_t* eos, uint32_t n_eos, uint32_t* out_tokens, uint32_t* out_count,
                  int32_t* out_logits) {
  if (!s || !prompt || !out_tokens || !out_count) return IRIS_EINVAL;
  *out_count = 0;
  if (max_tokens == 0) return 0;
  int rc = iris_session_reset(s);
  if (rc) return rc;
  const uint32_t V = s->m->Vfull;
  uint32_t tok = 0;
  rc = prefill_ids(s, prompt, n_prompt, out_logits, &tok);
  if (rc) return rc;
  auto is_eos = [&](uint32_t t) {
    for (uint32_t i = 0; i < n_eos; ++i)
      if (eos[i] == t) return true;
    return false;
  };
  uint32_t count = 0;
  out_tokens[count++] = tok;  // executor.rs:157-171
  if (is_eos(tok) || count == max_tokens) {
    *out_count = count;
    return 0;
  }
  if (out_logits) {  // one pass at a time, every pass's logits copied out
    while (true) {
      rc = iris_session_decode(s, tok, out_logits + (size_t)count * V, &tok);
      if (rc) return rc;
      out_tokens[count++] = tok;
      if (is_eos(tok) || count == max_tokens) break;
    }
    *out_count = count;
    return 0;
  }
  // Batches of graph replays, the token staying on the device; the history
  // buffer records each pass's selection.
  const uint32_t batch = 16;
  if (s->history_cap < batch) {
    cudaFree(s->d_history);
    s->d_history = nullptr;
    if (s->graph) {
      cudaGraphExecDestroy(s->graph);
      s->graph = nullptr;
    }
    cudaError_t e = dalloc(&s->d_history, batch);
    if (e != cudaSuccess) return (int)e;
    s->history_cap = batch;
  }
  std::vector<uint32_t> hist(batch);
  while (count < max_tokens) {
    uint32_t n = std::min(batch, max_tokens - count);
    cudaError_t e = cudaMemsetAsync(s->d_step, 0, 4, s->stream);
    if (e != cudaSuccess) return (int)e;
    uint32_t len0 = s->len;
    rc = decode_steps(s, n);
    if (rc) return rc;
    e = cudaMemcpyAsync(hist.data(), s->d_history, n * 4, cudaMemcpyDeviceToHost, s->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s->stream);
    if (e != cudaSuccess) return (int)e;
    for (uint32_t i = 0; i < n; ++i) {
      out_tokens[count++] = hist[i];
      if (is_eos(hist[i]) || count == max_tokens) {
        // passes after this one were not the reference's: forget them
        s->len = len0 + i + 1;
        uint32_t state[2] = {hist[i], s->len};
        e = cudaMemcpy(s->d_token, &state[0], 4, cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = cudaMemcpy(s->d_pos, &state[1], 4, cudaMemcpyHostToDevice);
        *out_count = count;
        return e != cudaSuccess ? (int)e : check_fault();
      }
    }
  }
  *out_count = count;
  return check_fault();
}

uint32_t iris_session_length(const IrisSession* s) { return s ? s->len : 0; }

int iris_session_decode_steps(IrisSession* s, uint32_t steps) {
  if (!s) return IRIS_EINVAL;
  return decode_steps(s, steps);
}

int iris_session_synchronize(IrisSession* s) {
  if (!s) return IRIS_EINVAL;
  cudaError_t e = cudaStreamSynchronize(s->stream);
  if (e != cudaSuccess) return (int)e;
  return check_fault();
}

void* iris_session_stream(IrisSession* s) { return s ? (void*)s->stream : nullptr; }

uint32_t iris_session_graph_kernels(IrisSession* s) {
  if (s && s->use_step) return 1;
  if (!s || ensure_graph(s)) return 0;
  cudaGraph_t g = nullptr;
  // Count kernel nodes by re-capturing the pass into a throwaway graph
  // (capture records launches without running them).
  if (cudaStreamBeginCapture(s->stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) return 0;
  cudaError_t body = run_pass(s, 1, s->d_token, s->d_pos, 0, true, true);
  if (body == cudaSuccess)
    body = launch_decode_finish(s->best, s->d_token, s->d_pos, s->d_step, s->d_history, s->history_cap, s->stream);
  if (cudaStreamEndCapture(s->stream, &g) != cudaSuccess || body != cudaSuccess || !g) return 0;
  size_t n = 0;
  cudaGraphGetNodes(g, nullptr, &n);
  std::vector<cudaGraphNode_t> nodes(n);
  cudaGraphGetNodes(g, nodes.data(), &n);
  uint32_t kernels = 0;
  for (cudaGraphNode_t nd : nodes) {
    cudaGraphNodeType t;
    if (cudaGraphNodeGetType(nd, &t) == cudaSuccess && t == cudaGraphNodeTypeKernel) ++kernels;
  }
  cudaGraphDestroy(g);
  return kernels;
}

int iris_session_attention(IrisSession* s, uint32_t layer) {
  if (!s || layer >= s->m->L || s->len == 0) return IRIS_EINVAL;
  AttnArgs a = attn_args(s, layer, nullptr, s->len - 1);
  return (int)launch_attention_decode(a, s->stream);
}

static int rebuild_graph_later(IrisSession* s) {
  if (!s->graph) return 0;
  cudaError_t e = cudaStreamSynchronize(s->stream);
  if (e != cudaSuccess) return (int)e;
  cudaGraphExecDestroy(s->graph);
  s->graph = nullptr;
  return 0;
}

int iris_session_set_attention(IrisSession* s, int mode) {
  if (!s || mode < IRIS_ATTN_AUTO || mode > IRIS_ATTN_CLUSTER) return IRIS_EINVAL;
  IrisModel* m = s->m;
  s->chunks = 0;
  s->cluster = 0;
  if (mode != IRIS_ATTN_SPLIT)
    attention_cluster_plan(m->heads, m->kvh, m->d, s->cap, &s->chpc, &s->cluster, &s->span, &s->ring);
  if (mode == IRIS_ATTN_AUTO) attention_grid_plan(m->heads, m->kvh, m->d, s->cap, &s->ghpc, &s->chunks, &s->gspan);
  s->attn_mode = mode;
  choose_decode_path(s);
  return rebuild_graph_later(s);
}

int iris_session_set_decode_path(IrisSession* s, int mode) {
  if (!s || mode < IRIS_DECODE_AUTO || mode > IRIS_DECODE_STEP) return IRIS_EINVAL;
  if (mode == IRIS_DECODE_STEP && !s->step.ok) return IRIS_EINVAL;
  s->decode_mode = mode;
  if (mode == IRIS_DECODE_STEP) s->attn_mode = IRIS_ATTN_AUTO;
  choose_decode_path(s);
  return 0;
}

int iris_session_decode_path(const IrisSession* s) {
  if (!s) return IRIS_EINVAL;
  return s->use_step ? IRIS_DECODE_STEP : IRIS_DECODE_GRAPH;
}

int iris_session_step_trace(IrisSession* s, int enable) {
  if (!s || !s->step.ok) return IRIS_EINVAL;
  cudaError_t e = cudaStreamSynchronize(s->stream);
  if (e != cudaSuccess) return (int)e;
  cudaFree(s->trace);
  s->trace = nullptr;
  if (!enable) return 0;
  const size_t n = (size_t)s->step.blocks * s->nstages * kStepTraceEvents;
  e = dalloc(&s->trace, n);
  if (e == cudaSuccess) e = cudaMemset(s->trace, 0, n * sizeof(unsigned long long));
  return (int)e;
}

int iris_session_get_step_trace(const IrisSession* s, uint64_t* out, uint64_t count) {
  if (!s || !s->trace || !out) return IRIS_EINVAL;
  const size_t n = (size_t)s->step.blocks * s->nstages * kStepTraceEvents;
  if (count < n) return IRIS_EINVAL;
  return (int)cudaMemcpy(out, s->trace, n * sizeof(uint64_t), cudaMemcpyDeviceToHost);
}

int iris_session_step_plan(const IrisSession* s, uint32_t* plan) {
  if (!s || !plan) return IRIS_EINVAL;
  const StepPlan& p = s->step;
  const uint32_t v[8] = {p.ok ? 0u : (p.why ? p.why : 1u), p.blocks, p.ring_slots, p.slot_bytes, p.planes_bytes,
                         p.smem, p.chunks, p.span_max};
  for (int i = 0; i < 8; ++i) plan[i] = v[i];
  return 0;
}

int iris_session_attention_plan(const IrisSession* s, uint32_t* plan) {
  if (!s || !plan) return IRIS_EINVAL;
  if (s->use_step) {
    plan[0] = 4;
    plan[1] = s->step.hpc;
    plan[2] = s->step.chunks;
    plan[3] = s->step.span_max;
    return 0;
  }
  plan[0] = s->chunks ? 3 : s->cluster ? 2 : 1;
  plan[1] = s->chunks ? s->ghpc : s->cluster ? s->chpc : s->hpc;
  plan[2] = s->chunks ? s->chunks : s->cluster;
  plan[3] = s->chunks ? s->gspan : s->span;
  return 0;
}

int iris_session_set_attention_shape(IrisSession* s, uint32_t cluster, uint32_t hpc, uint32_t ring) {
  if (!s) return IRIS_EINVAL;
  IrisModel* m = s->m;
  uint32_t span = 0;
  if (!attention_cluster_shape_ok(m->heads, m->kvh, m->d, s->cap, cluster, hpc, ring, &span)) return IRIS_EINVAL;
  s->cluster = cluster;
  s->chpc = hpc;
  s->ring = ring;
  s->span = span;
  s->chunks = 0;
  s->attn_mode = IRIS_ATTN_CLUSTER;
  choose_decode_path(s);
  return rebuild_graph_later(s);
}

int iris_session_product(IrisSession* s, uint32_t layer, int which) {
  if (!s || layer >= s->m->L || which < 0 || which > 4) return IRIS_EINVAL;
  IrisModel* m = s->m;
  const LayerDev& L = m->layers[layer];
  const Q8GpuMatrix* w = which == 0 ? L.qkv : which == 1 ? L.o : which == 2 ? L.gu : which == 3 ? L.down : m->head;
  ProductArgs a = session_product_args(s, w, 1);
  if (which == 1 || which == 3) {  // inputs from byte planes, as in the pass
    a.planes = which == 1 ? s->planes : s->planes2;
    a.out = s->tmp;
    return (int)launch_product(a, IN_PLANES, EPI_STORE, s->stream);
  }
  a.x = s->x;
  a.norm_w = which == 4 ? m->final_norm : L.norm_attn;
  a.eps = m->eps;
  if (which == 2) {
    a.out_planes = s->planes;
    return (int)launch_product(a, IN_NORM, m->family == kFamilyGemma ? EPI_GELU_MUL : EPI_SILU_MUL, s->stream);
  }
  if (which == 4) {
    a.out = s->logits;
    a.best = s->best + 1;  // not the decode pass's key
    return (int)launch_product(a, IN_NORM, EPI_LOGITS, s->stream);
  }
  a.out = s->tmp;  // kMaxRows * hidden values >= one token's q|k|v rows
  return (int)launch_product(a, IN_NORM, EPI_STORE, s->stream);
}

int iris_session_get_kv(const IrisSession* s, uint32_t layer, uint32_t first, uint32_t count, int32_t* k,
                        int32_t* v) {
  if (!s || layer >= s->m->L || (uint64_t)first + count > s->len) return IRIS_EINVAL;
  size_t off = kv_offset(s, layer) + (size_t)first * s->m->kvd, n = (size_t)count * s->m->kvd * 4;
  cudaError_t e = cudaSuccess;
  if (k) e = cudaMemcpy(k, s->kc + off, n, cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && v) e = cudaMemcpy(v, s->vc + off, n, cudaMemcpyDeviceToHost);
  return (int)e;
}

void iris_session_free(IrisSession* s) { free_session(s); }

int iris_capture_begin(void* stream) {
  if (!stream) return IRIS_EINVAL;  // the legacy default stream cannot be captured
  return (int)cudaStreamBeginCapture((cudaStream_t)stream, cudaStreamCaptureModeThreadLocal);
}

int iris_capture_end(void* stream, void** graph_exec) {
  if (!stream || !graph_exec) return IRIS_EINVAL;
  *graph_exec = nullptr;
  cudaGraph_t g = nullptr;
  cudaError_t e = cudaStreamEndCapture((cudaStream_t)stream, &g);
  if (e != cudaSuccess) return (int)e;
  cudaGraphExec_t x = nullptr;
  e = cudaGraphInstantiate(&x, g, 0);
  cudaGraphDestroy(g);
  if (e == cudaSuccess) *graph_exec = (void*)x;
  return (int)e;
}

int iris_graph_launch(void* graph_exec, void* stream) {
  if (!graph_exec) return IRIS_EINVAL;
  return (int)cudaGraphLaunch((cudaGraphExec_t)graph_exec, (cudaStream_t)stream);
}

void iris_graph_free(void* graph_exec) {
  if (graph_exec) cudaGraphExecDestroy((cudaGraphExec_t)graph_exec);
}

int iris_model_embed(IrisModel* m, const uint32_t* ids, uint32_t n, int32_t* rows) {
  if (!m || !ids || !rows || m->tp_world > 1) return IRIS_EINVAL;
  if (n == 0) return 0;
  for (uint32_t i = 0; i < n; ++i)
    if (ids[i] >= m->Vfull) return IRIS_EINVAL;
  int rc = check_model_ready(m);
  if (rc) return rc;
  if (!m->scratch) {
    rc = create_session(m, 512, &m->scratch);
    if (rc) return rc;
  }
  IrisSession* s = m->scratch;
  const bool gemma = m->family == kFamilyGemma;
  cudaError_t e = cudaSuccess;
  for (uint32_t r0 = 0; r0 < n && e == cudaSuccess; r0 += kMaxRows) {
    const uint32_t cnt = std::min(kMaxRows, n - r0);
    e = cudaMemcpyAsync(s->d_ids, ids + r0, (size_t)cnt * 4, cudaMemcpyHostToDevice, s->stream);
    if (e == cudaSuccess) e = launch_embed(m->embed, s->d_ids, cnt, gemma, m->embedding_scale, s->x, s->stream);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(rows + (size_t)r0 * m->H, s->x, (size_t)cnt * m->H * 4, cudaMemcpyDeviceToHost, s->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s->stream);
  }
  return (int)e;
}

int iris_model_ple_rows(IrisModel* m, const uint32_t* ids, uint32_t n, int32_t* out) {
  if (!m || !ids || !out || m->family != kFamilyGemma || m->tp_world > 1) return IRIS_EINVAL;
  if (n == 0) return 0;
  for (uint32_t i = 0; i < n; ++i)
    if (ids[i] >= m->Vfull) return IRIS_EINVAL;
  int rc = check_model_ready(m);
  if (rc) return rc;
  if (!m->scratch) {
    rc = create_session(m, 512, &m->scratch);
    if (rc) return rc;
  }
  IrisSession* s = m->scratch;
  const size_t LP = (size_t)m->L * m->P;
  cudaError_t e = cudaSuccess;
  for (uint32_t r0 = 0; r0 < n && e == cudaSuccess; r0 += kMaxRows) {
    const uint32_t cnt = std::min(kMaxRows, n - r0);
    e = cudaMemcpyAsync(s->d_ids, ids + r0, (size_t)cnt * 4, cudaMemcpyHostToDevice, s->stream);
    if (e == cudaSuccess) e = launch_embed(m->embed, s->d_ids, cnt, true, m->embedding_scale, s->x, s->stream);
    if (e == cudaSuccess)
      e = launch_dense(m->ple_model_proj, m->L * m->P, m->H, s->x, m->H, cnt, s->ple_proj, m->L * m->P, nullptr, 0,
                       s->stream);
    if (e == cudaSuccess)
      e = launch_ple_prepare(s->ple_proj, m->ple_embed, s->d_ids, m->ple_norm, m->eps, m->ple_projection_scalar,
                             m->ple_embedding_scale, m->ple_input_scale, cnt, m->L, m->P, s->ple_rows, s->stream);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(out + (size_t)r0 * LP, s->ple_rows, (size_t)cnt * LP * 4, cudaMemcpyDeviceToHost, s->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s->stream);
  }
  return (int)e;
}

namespace {
// Keys given as (count, positions): consecutive positions (each one more than
// the one before) that cover [lo, hi). Empty coverage (lo == hi) needs no keys.
bool keys_cover(uint32_t count, const uint32_t* pos, uint32_t lo, uint32_t hi) {
  if (lo >= hi) return true;
  if (count == 0 || !pos) return false;
  for (uint32_t i = 1; i < count; ++i)
    if (pos[i] != pos[i - 1] + 1) return false;
  return pos[0] <= lo && (uint64_t)pos[0] + count >= hi;
}
}  // namespace

int iris_gemma_layer_range(IrisModel* m, uint32_t layer, const int32_t* rows_in, uint32_t n, uint32_t start,
                           const int32_t* ple_rows, uint32_t n_prior, const uint32_t* prior_pos,
                           const int32_t* prior_k, const int32_t* prior_v, uint32_t n_donor,
                           const uint32_t* donor_pos, const int32_t* donor_k, const int32_t* donor_v,
                           int32_t* rows_out, int32_t* own_k, int32_t* own_v) {
  if (!m || m->family != kFamilyGemma || layer >= m->L || m->tp_world > 1) return IRIS_EINVAL;
  if (n == 0) return 0;  // prefill_range.rs:141-155: a range with no rows produces nothing
  if (!rows_in || !rows_out || !ple_rows) return IRIS_EINVAL;
  if ((uint64_t)start + n > 0xFFFFFFFFull) return IRIS_ERANGE;
  const LayerDev& L = m->layers[layer];
  // the positions the first query sees before itself, and those the last sees
  const uint32_t w = L.window;
  const uint32_t first_vis = w == 0 ? 0 : (start + 1 > w ? start + 1 - w : 0);
  const bool shares = L.kv_donor >= 0;
  if (!shares) {
    if (n_prior && (!prior_k || !prior_v)) return IRIS_EINVAL;
    if (!keys_cover(n_prior, prior_pos, first_vis, start)) return IRIS_EWINDOW;
    if (n_prior && prior_pos[n_prior - 1] + 1 != start) return IRIS_EWINDOW;  // nothing at or past the range
  } else {
    if (n_donor && (!donor_k || !donor_v)) return IRIS_EINVAL;
    if (!keys_cover(n_donor, donor_pos, first_vis, start + n)) return IRIS_EWINDOW;
  }
  int rc = check_model_ready(m);
  if (rc) return rc;
  const uint32_t cap_needed = std::max(start + n, shares && n_donor ? donor_pos[0] + n_donor : 0u);
  if (!m->scratch || m->scratch->cap < cap_needed) {
    free_session(m->scratch);
    m->scratch = nullptr;
    rc = create_session(m, std::max<uint32_t>(cap_needed, 512), &m->scratch);
    if (rc) return rc;
  }
  IrisSession* s = m->scratch;
  const size_t kvd = m->kvd, H = m->H, P = m->P, LP = (size_t)m->L * m->P;
  cudaError_t e = cudaSuccess;
  // the keys the layer attends over, at their positions in the cache
  const uint32_t src_layer = shares ? (uint32_t)L.kv_donor : layer;
  const uint32_t nk = shares ? n_donor : n_prior;
  if (nk) {
    const uint32_t p0 = shares ? donor_pos[0] : prior_pos[0];
    int32_t* kc = s->kc + kv_offset(s, src_layer) + (size_t)p0 * kvd;
    int32_t* vc = s->vc + kv_offset(s, src_layer) + (size_t)p0 * kvd;
    e = cudaMemcpyAsync(kc, shares ? donor_k : prior_k, (size_t)nk * kvd * 4, cudaMemcpyHostToDevice, s->stream);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(vc, shares ? donor_v : prior_v, (size_t)nk * kvd * 4, cudaMemcpyHostToDevice, s->stream);
  }
  for (uint32_t r0 = 0; r0 < n && e == cudaSuccess; r0 += kMaxRows) {
    const uint32_t cnt = std::min(kMaxRows, n - r0);
    e = cudaMemcpyAsync(s->x, rows_in + (size_t)r0 * H, (size_t)cnt * H * 4, cudaMemcpyHostToDevice, s->stream);
    if (e == cudaSuccess)
      e = cudaMemcpy2DAsync(s->ple_rows + (size_t)layer * P, LP * 4, ple_rows + (size_t)r0 * P, P * 4, P * 4, cnt,
                            cudaMemcpyHostToDevice, s->stream);
    if (e == cudaSuccess) e = gemma_layer(s, layer, cnt, nullptr, start + r0, true);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(rows_out + (size_t)r0 * H, s->x, (size_t)cnt * H * 4, cudaMemcpyDeviceToHost, s->stream);
  }
  int32_t* kc = s->kc + kv_offset(s, layer) + (size_t)start * kvd;
  int32_t* vc = s->vc + kv_offset(s, layer) + (size_t)start * kvd;
  if (e == cudaSuccess && own_k) e = cudaMemcpyAsync(own_k, kc, (size_t)n * kvd * 4, cudaMemcpyDeviceToHost, s->stream);
  if (e == cudaSuccess && own_v) e = cudaMemcpyAsync(own_v, vc, (size_t)n * kvd * 4, cudaMemcpyDeviceToHost, s->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s->stream);
  if (e == cudaSuccess) {
    rc = check_fault();
    if (rc) return rc;
  }
  return (int)e;
}

int iris_sequence_check_select(IrisModel* m, const int32_t* rows, uint32_t n, uint32_t* token_ids,
                               int32_t* values) {
  if (!m || !rows || !token_ids) return IRIS_EINVAL;
  if (n == 0) return 0;
  int rc = check_model_ready(m);
  if (rc) return rc;
  if (!m->scratch) {
    rc = create_session(m, 512, &m->scratch);
    if (rc) return rc;
  }
  IrisSession* s = m->scratch;
  cudaStream_t st = s->stream;
  std::vector<unsigned long long> keys(kMaxRows);
  cudaError_t e = cudaSuccess;
  for (uint32_t r0 = 0; r0 < n && e == cudaSuccess; r0 += kMaxRows) {
    const uint32_t cnt = std::min(kMaxRows, n - r0);
    e = cudaMemcpyAsync(s->x, rows + (size_t)r0 * m->H, (size_t)cnt * m->H * 4, cudaMemcpyHostToDevice, st);
    // rms_norm with the final norm (sequence_check.rs:118-125), as byte planes
    if (e == cudaSuccess) e = launch_planes(s->x, m->final_norm, m->eps, cnt, m->H, s->planes, st);
    if (e == cudaSuccess) e = launch_fill_u64(s->best, cnt, st);
    if (e == cudaSuccess) {
      // every vocabulary row's dot_row, softcap, first maximum (sequence_check.rs:274-288)
      ProductArgs h = session_product_args(s, m->head, cnt);
      h.planes = s->planes;
      h.out = nullptr;
      h.best = s->best;
      h.softcap = m->softcap;
      h.row_base = m->tp_rank * m->V;  // vocabulary shard
      e = launch_product(h, IN_PLANES, EPI_LOGITS, st);
    }
    if (e == cudaSuccess && m->tp_world > 1) e = tp_max_keys(m->comm, s->best, cnt, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(keys.data(), s->best, (size_t)cnt * 8, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    for (uint32_t i = 0; i < cnt && e == cudaSuccess; ++i) {
      token_ids[r0 + i] = best_key_token(keys[i]);
      if (values) values[r0 + i] = best_key_value(keys[i]);
    }
  }
  if (e != cudaSuccess) return (int)e;
  return check_fault();
}

int iris_mistral_layer_range(IrisModel* m, uint32_t layer, const int32_t* rows_in, uint32_t n, uint32_t start,
                             const int32_t* prior_k, const int32_t* prior_v, int32_t* rows_out, int32_t* own_k,
                             int32_t* own_v) {
  // the chain stage runs whole models (claims are spread data-parallel)
  if (!m || m->family != kFamilyMistral || layer >= m->L || !rows_in || !rows_out || m->tp_world > 1)
    return IRIS_EINVAL;
  if (n == 0) return 0;  // layer.rs:117-119: a range with no rows produces nothing
  if ((uint64_t)start + n > m->max_positions) return IRIS_ERANGE;  // layer.rs:121-127
  if (start && (!prior_k || !prior_v)) return IRIS_EINVAL;
  int rc = check_model_ready(m);
  if (rc) return rc;
  if (!m->scratch || m->scratch->cap < start + n) {
    free_session(m->scratch);
    m->scratch = nullptr;
    rc = create_session(m, std::max<uint32_t>(start + n, 512), &m->scratch);
    if (rc) return rc;
  }
  IrisSession* s = m->scratch;
  size_t kvd = m->kvd, H = m->H;
  int32_t* kc = s->kc + kv_offset(s, layer);
  int32_t* vc = s->vc + kv_offset(s, layer);
  cudaError_t e = cudaSuccess;
  if (start) {
    e = cudaMemcpyAsync(kc, prior_k, (size_t)start * kvd * 4, cudaMemcpyHostToDevice, s->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(vc, prior_v, (size_t)start * kvd * 4, cudaMemcpyHostToDevice, s->stream);
  }
  for (uint32_t r0 = 0; r0 < n && e == cudaSuccess; r0 += kMaxRows) {
    uint32_t cnt = std::min(kMaxRows, n - r0);
    e = cudaMemcpyAsync(s->x, rows_in + (size_t)r0 * H, (size_t)cnt * H * 4, cudaMemcpyHostToDevice, s->stream);
    if (e == cudaSuccess) e = mistral_layer(s, layer, cnt, nullptr, start + r0);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(rows_out + (size_t)r0 * H, s->x, (size_t)cnt * H * 4, cudaMemcpyDeviceToHost, s->stream);
  }
  if (e == cudaSuccess && own_k)
    e = cudaMemcpyAsync(own_k, kc + (size_t)start * kvd, (size_t)n * kvd * 4, cudaMemcpyDeviceToHost, s->stream);
  if (e == cudaSuccess && own_v)
    e = cudaMemcpyAsync(own_v, vc + (size_t)start * kvd, (size_t)n * kvd * 4, cudaMemcpyDeviceToHost, s->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s->stream);
  return (int)e;
}

}  // extern "C"
