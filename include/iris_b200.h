/*
 * iris_b200 — C ABI of the B200-native exact-integer inference path.
 *
 * Conventions (those of the reference's crates/inference/kernels/cuda/
 * q8_product.cu:129-197 and its Rust binding crates/inference/kernels/src/
 * gpu.rs:45-62):
 *   - every entry point returns an int status: 0 on success, otherwise a
 *     cudaError_t value or one of the IRIS_E* codes below; iris_error() (or
 *     q8gpu_error()) turns it into a static string;
 *   - host buffers are owned by the caller and only borrowed for the call;
 *   - device state lives behind opaque handles freed by the matching *_free;
 *   - activations are Q16.16 int32, accumulators Q32.32 int64, weights Q8_0
 *     (34-byte GGUF blocks: little-endian fp16 scale bits, then 32 int8) or
 *     dense Q16.16 int32;
 *   - no floating point anywhere: every value equals the reference's Rust CPU
 *     path (det-num) bit for bit.
 * A handle may be used by one host thread at a time.
 */
#ifndef IRIS_B200_H
#define IRIS_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

/* Status codes beyond cudaError_t (all >= 10000). */
#define IRIS_EINVAL 10001   /* bad argument, shape or parameter */
#define IRIS_ESCALE 10002   /* a Q8_0 scale is Inf/NaN (q8.rs:46-48 rejects it) */
#define IRIS_ERANGE 10003   /* a position past max_positions or the KV capacity */
#define IRIS_ESTATE 10004   /* call out of order (e.g. decode before prefill) */
#define IRIS_EWINDOW 10005  /* attention window not covered by the given keys */
#define IRIS_ESTALL 10006   /* a kernel gave up a bounded wait (pipeline stalled) */
#define IRIS_ESCRATCH 10007 /* input larger than a fixed scratch array */

/* ---------------------------------------------------------------------------
 * 1. Drop-in for the reference's q8gpu_* FFI. Same names, signatures and
 *    semantics as crates/inference/kernels/cuda/q8_product.cu:129-197, so the
 *    unchanged `extern "C"` block of gpu.rs:45-62 links against this library.
 * ------------------------------------------------------------------------- */
typedef struct Q8GpuMatrix Q8GpuMatrix;

/* q8_product.cu:131 — message for a status code (static storage). */
const char* q8gpu_error(int code);
/* q8_product.cu:134-139 — 0 when a device is usable. */
int q8gpu_init(void);
/* q8_product.cu:141-146 — frees a matrix from q8gpu_upload (NULL is a no-op). */
void q8gpu_free(Q8GpuMatrix* matrix);
/* q8_product.cu:150-171 — weights: rows*cols int8 row-major; scales_q24: one
 * decoded Q.24 block scale per 32 weights (q8.rs:27-43). Each scale must be
 * the exact image of a finite fp16 scale (what gpu.rs:175-186 passes);
 * anything else returns IRIS_ESCALE. */
int q8gpu_upload(const int8_t* weights, const int64_t* scales_q24, uint32_t rows, uint32_t cols,
                 Q8GpuMatrix** out_matrix);
/* q8_product.cu:175-195 — out[token*rows + row] = dot_row(activations[token],
 * row) (q8.rs:56-72) for tokens x cols host activations. */
int q8gpu_product(const Q8GpuMatrix* matrix, const int32_t* activations, uint32_t tokens,
                  int32_t* out);

/* ---------------------------------------------------------------------------
 * 2. Q8_0 products without the host round trip.
 * ------------------------------------------------------------------------- */
/* Uploads a matrix from its committed Q8_0 bytes (Q8Source parts concatenated,
 * crates/inference/kernels/src/tensor.rs:110-115): rows*cols/32*34 bytes.
 * Replaces the host-side scale decoding of gpu.rs:175-186. */
int iris_q8_upload_blocks(const uint8_t* blocks, uint32_t rows, uint32_t cols,
                          Q8GpuMatrix** out_matrix);
/* The same product as q8gpu_product with device pointers on a CUDA stream
 * (cudaStream_t passed as void*, NULL = default stream). One token is
 * asynchronous; more tokens build their byte planes in a scratch buffer the
 * next call reuses, so the call waits for the stream before it returns (and
 * the first many-token call on a matrix builds its tensor-core copy). */
int iris_q8_product_device(const Q8GpuMatrix* matrix, const int32_t* d_activations,
                           uint32_t tokens, int32_t* d_out, void* stream);
/* Generic-kernel timing hooks for the Q8 sweep: same product, forced through
 * the decode GEMV (tokens must be 1), the mma.sync GEMM or the tcgen05
 * tensor-core GEMM. The automatic path takes the tensor-core GEMM for 32 or
 * more tokens when the matrix qualifies (cols <= 18848, and either every row
 * has one scale, or every row's block-scale exponents lie within 5 of each
 * other), building its copy on the first such call: 1 byte a weight where
 * every row has one scale (four MMAs a 32-column step), else 3 bytes a
 * weight (twelve). IRIS_PATH_TC3 builds and uses the 3-byte form in any case
 * (measurement; it fails if another form was built first). IRIS_PATH_TC or
 * IRIS_PATH_TC3 on a matrix that does not qualify fails with
 * cudaErrorInvalidValue. IRIS_PATH_GEMV1 forces the decode GEMV's
 * one-scale-a-row form (int32 plane sums over a tile group, each row scaled
 * once: the form a session's one-token products take for such matrices);
 * tokens must be 1, every row must have one scale and cols <= 32768, else it
 * fails with cudaErrorInvalidValue. */
int iris_q8_product_device_path(const Q8GpuMatrix* matrix, const int32_t* d_activations,
                                uint32_t tokens, int32_t* d_out, void* stream, int path);
#define IRIS_PATH_AUTO 0
#define IRIS_PATH_GEMV 1
#define IRIS_PATH_GEMM 2
#define IRIS_PATH_TC 3
#define IRIS_PATH_TC3 4
#define IRIS_PATH_GEMV1 5
/* No counterpart in the reference. The same product as
 * iris_q8_product_device, allocating nothing: the GEMM path's byte planes
 * live in a fixed 16 MiB device array, so tokens > 1 needs
 * tokens * cols * 4 <= 16 MiB (else IRIS_ESCRATCH, nothing launched); one
 * token needs no scratch. The first call on each device looks the array's
 * address up (make it before any stream capture begins) and keeps it for the
 * life of the process: a cudaDeviceReset, which also frees every uploaded
 * matrix, ends the use of this entry point on that device. Nothing must start
 * at zero. Asynchronous and not synchronized: calls in flight at the same time
 * on one device (other streams or host threads) share the array and race;
 * calls on one stream are ordered. It never builds a matrix's tensor-core
 * copy (that allocates): 32 or more tokens take the tcgen05 GEMM when an
 * earlier call of another entry point built the copy, else the mma.sync
 * GEMM; both give the same values. */
int iris_q8_product_device_noalloc(const Q8GpuMatrix* matrix, const int32_t* d_activations,
                                   uint32_t tokens, int32_t* d_out, void* stream);

/* ---------------------------------------------------------------------------
 * 3. Device-resident models, sessions and the decode loop.
 * ------------------------------------------------------------------------- */
typedef struct IrisModel IrisModel;
typedef struct IrisSession IrisSession;

/* mistral-dense shape (crates/inference/artifacts/src/direct.rs:267-287). */
typedef struct {
  uint32_t layers, hidden, ffn, heads, kv_heads, head_dim, vocab;
  uint32_t max_positions;        /* positions from here on are refused */
  int64_t norm_eps;              /* Acc bits */
  uint32_t attention_scale_q32;  /* mistral.rs:148-160 */
  uint32_t tied_head;            /* head = embedding table */
  const int64_t* rope_inverse_frequencies; /* head_dim/2 Q32.32 values, copied */
} IrisMistralShape;

/* gemma-dense shape (direct.rs:241-262) with the per-layer values the
 * reference derives from it (direct/src/model.rs:802-871). */
typedef struct {
  uint32_t layers, hidden, ffn, heads, kv_heads, head_dim, vocab, ple_width;
  int64_t norm_eps;
  int32_t embedding_scale, ple_embedding_scale, ple_projection_scalar, ple_input_scale;
  int32_t final_logit_softcap; /* 0 disables */
  /* per layer (arrays of `layers` entries, copied) */
  const uint32_t* sliding_window;     /* 0 = full attention */
  const int64_t* rope_base;           /* Acc bits */
  const uint32_t* rotary_dim;
  const uint32_t* rope_freq_base_dim;
  const int32_t* kv_donor_layer;      /* -1 = own K/V */
  const int32_t* layer_scalar;        /* 0 = none */
  uint32_t tied_head;                 /* head = embedding table (tie_word_embeddings) */
} IrisGemmaShape;

/* Tensor kinds for iris_model_set_q8 / iris_model_set_values. */
enum {
  IRIS_T_EMBED = 0,       /* [vocab][hidden] Q8_0 */
  IRIS_T_HEAD = 1,        /* [vocab][hidden] Q8_0 (untied models) */
  IRIS_T_FINAL_NORM = 2,  /* [hidden] */
  IRIS_T_W_Q = 3, IRIS_T_W_K = 4, IRIS_T_W_V = 5, IRIS_T_W_O = 6,
  IRIS_T_W_GATE = 7, IRIS_T_W_UP = 8, IRIS_T_W_DOWN = 9,
  IRIS_T_NORM_ATTN = 10,  /* mistral input_layernorm / gemma norm_input */
  IRIS_T_NORM_FFN = 11,   /* mistral pre_feedforward / gemma norm_pre_ffw */
  IRIS_T_NORM_POST_ATTN = 12, IRIS_T_NORM_POST_FFW = 13,
  IRIS_T_Q_NORM = 14, IRIS_T_K_NORM = 15, IRIS_T_PLE_POST_NORM = 16,
  IRIS_T_PLE_INPUT_GATE = 17,       /* [ple][hidden] dense */
  IRIS_T_PLE_LAYER_PROJECTION = 18, /* [hidden][ple] dense */
  IRIS_T_PLE_EMBED = 19,            /* [vocab][layers*ple] Q8_0 */
  IRIS_T_PLE_MODEL_PROJECTION = 20, /* [layers*ple][hidden] dense */
  IRIS_T_PLE_NORM = 21,             /* [ple] */
  IRIS_T_COUNT = 22
};

int iris_model_create_mistral(const IrisMistralShape* shape, IrisModel** out);
int iris_model_create_gemma(const IrisGemmaShape* shape, IrisModel** out);
/* No counterpart in the reference (its tensor-parallel plan). Rank `rank` of a
 * `world`-way tensor-parallel mistral-dense model: kv groups, FFN rows and
 * vocabulary split evenly (kv_heads, ffn / 32 and vocab divisible by world;
 * no tied head), the row-parallel o and down products exchanging exact
 * partial sums over NCCL (communicator from the 128-byte id of
 * iris_tp_unique_id, the same on every rank). Every rank makes the same calls
 * in the same order; tensors are synthesized on the device
 * (iris_model_synthesize); logits, tokens and positions are the whole
 * model's. */
int iris_model_create_mistral_tp(const IrisMistralShape* shape, uint32_t rank, uint32_t world,
                                 const uint8_t* nccl_id, IrisModel** out);
/* A fresh NCCL unique id (128 bytes) for iris_model_create_mistral_tp. */
int iris_tp_unique_id(uint8_t* out);
/* How a tensor-parallel model exchanges the partial sums of its one-token
 * (decode) row-parallel products: IRIS_TP_PEER (default; loads of the peers'
 * memory over NVLink, world <= 8) or IRIS_TP_NCCL (an NCCL sum). Many-token
 * passes always use NCCL. Sessions of a tensor-parallel model are used one at
 * a time; sessions whose captured pass predates a change are rebuilt by the
 * caller (iris_session_set_attention). */
int iris_model_set_tp_exchange(IrisModel* model, int mode);
#define IRIS_TP_PEER 0
#define IRIS_TP_NCCL 1
/* Uploads one Q8_0 tensor (layer = -1 for model-level tensors). */
int iris_model_set_q8(IrisModel* model, int tensor, int32_t layer, const uint8_t* blocks,
                      uint64_t bytes);
/* Uploads one dense Q16.16 tensor (norm weights, PLE matrices). */
int iris_model_set_values(IrisModel* model, int tensor, int32_t layer, const int32_t* values,
                          uint64_t count);
/* Fills every tensor with the seeded synthetic weights of iris_synth_* on the
 * device (no host copy). */
int iris_model_synthesize(IrisModel* model, uint64_t seed, int per_block_scales);
/* Reads a tensor back: Q8_0 bytes or int32 values. */
int iris_model_get_q8(const IrisModel* model, int tensor, int32_t layer, uint8_t* blocks,
                      uint64_t bytes);
int iris_model_get_values(const IrisModel* model, int tensor, int32_t layer, int32_t* values,
                          uint64_t count);
/* Device bytes held by the model's weights. */
uint64_t iris_model_weight_bytes(const IrisModel* model);
/* Many-token products (prefill, layer ranges) of a model: IRIS_GEMM_AUTO
 * (default) runs them on the tcgen05 tensor-core GEMM for ranges of 32 or
 * more tokens, over a copy of each qualifying matrix built on its first such
 * product (freed with the model: 1 byte a weight where every row has one
 * scale, else 3 bytes a weight of pre-scaled weights; a matrix whose rows'
 * block-scale exponents spread by more than 5 keeps the mma.sync GEMM);
 * IRIS_GEMM_MMA runs them all on the mma.sync GEMM. */
int iris_model_set_gemm(IrisModel* model, int mode);
#define IRIS_GEMM_AUTO 0
#define IRIS_GEMM_MMA 1
/* Builds the tensor-core copies of every layer matrix now (otherwise the
 * first many-token product of each builds its own), so that a timed or
 * latency-bound prefill does not pay for them. Synchronous. */
int iris_model_prepare_gemm(IrisModel* model);
/* Number of the model's matrices holding a tensor-core copy; *bytes (if not
 * NULL) receives the device bytes those copies take. */
int iris_model_tc_matrices(const IrisModel* model, uint64_t* bytes);
/* No counterpart in the reference (inspection). counts[0] = many-query
 * (prefill and chain-range) attention launches of this model that ran on the
 * tensor cores, counts[1] = those that ran on the CUDA-core kernel. */
int iris_model_attention_ranges(const IrisModel* model, uint64_t* counts);
void iris_model_free(IrisModel* model);

/* A decoding session: the K/V cache for up to max_positions positions. */
int iris_session_create(IrisModel* model, uint32_t max_positions, IrisSession** out);
/* Forgets every position. */
int iris_session_reset(IrisSession* session);
/* Prompt pass (executor.rs:143-152): the prompt rows through every layer, K/V
 * kept, then the head over the last row. logits (vocab values, may be NULL)
 * and *token (its first maximum, generation.rs:25-58). */
int iris_session_prefill(IrisSession* session, const uint32_t* ids, uint32_t n, int32_t* logits,
                         uint32_t* token);
/* One decode pass (executor.rs:172-184): token_in at the next position, then
 * the head. */
int iris_session_decode(IrisSession* session, uint32_t token_in, int32_t* logits,
                        uint32_t* token_out);
/* The direct decode loop (executor.rs:136-186): prefill, then up to
 * max_tokens greedy selections, stopping after an EOS id or the budget (no
 * pass for the last token). out_tokens holds max_tokens entries; out_logits
 * (may be NULL) receives [passes][vocab], pass p being the scores that chose
 * out_tokens[p]. Decode passes run on the device back to back (persistent
 * step launches or graph replays) with the token id kept on the device. */
int iris_generate(IrisSession* session, const uint32_t* prompt, uint32_t n_prompt,
                  uint32_t max_tokens, const uint32_t* eos, uint32_t n_eos, uint32_t* out_tokens,
                  uint32_t* out_count, int32_t* out_logits);
/* Positions currently held. */
uint32_t iris_session_length(const IrisSession* session);
/* Device-resident decode loop: runs the decode pass `steps` times on the
 * session's stream without waiting (each pass feeds its first-maximum
 * token to the next). iris_session_synchronize waits for them. */
int iris_session_decode_steps(IrisSession* session, uint32_t steps);
int iris_session_synchronize(IrisSession* session);
/* The session's CUDA stream (cudaStream_t as void*), for timing with events. */
void* iris_session_stream(IrisSession* session);
/* Kernel launches in one decode pass (1 for the persistent step). */
uint32_t iris_session_graph_kernels(IrisSession* session);
/* Launches one decode product of layer `layer` on the session's stream
 * (which: 0 = fused q|k|v, 1 = o, 2 = gate|up, 3 = down, 4 = head) with the
 * session's current activations; the result is discarded. For timing. */
int iris_session_product(IrisSession* session, uint32_t layer, int which);
/* Launches one single-query attention of layer `layer` on the session's
 * stream: the last held position attends over the positions before it, with
 * the session's current query rows; the context is discarded. For timing. */
int iris_session_attention(IrisSession* session, uint32_t layer);
/* Selects the decode attention kernels of the kernel-per-operation decode
 * pass: IRIS_ATTN_AUTO (one launch over the whole GPU where the shape and
 * capacity allow it, else one thread-block-cluster launch, else three
 * launches), IRIS_ATTN_SPLIT (three launches over position chunks) or
 * IRIS_ATTN_CLUSTER (the cluster launch where possible). All give the same
 * values; the captured decode pass is rebuilt. SPLIT and CLUSTER also select
 * that pass (IRIS_DECODE_GRAPH) over the persistent step. */
int iris_session_set_attention(IrisSession* session, int mode);
#define IRIS_ATTN_AUTO 0
#define IRIS_ATTN_SPLIT 1
#define IRIS_ATTN_CLUSTER 2
/* Tuning hook: an explicit one-launch decode attention shape - blocks a
 * cluster (4, 8 or 16), query heads a block (1, 2 or 4, dividing the group)
 * and shared-memory tile buffers a block (2..12). IRIS_EINVAL when the shape
 * does not fit the model, the capacity or the device. */
int iris_session_set_attention_shape(IrisSession* session, uint32_t cluster, uint32_t hpc, uint32_t ring);
/* The decode attention in use: plan[0] = 4 (inside the persistent step), 3
 * (whole-GPU launch), 2 (cluster launch) or 1 (three launches); plan[1] query
 * heads a block; plan[2] blocks a head group (step, whole-GPU) or a cluster;
 * plan[3] positions a block at most. */
int iris_session_attention_plan(const IrisSession* session, uint32_t* plan);
/* How decode passes run: IRIS_DECODE_AUTO (default: the persistent step where
 * the model allows it, else the graph), IRIS_DECODE_GRAPH (a CUDA graph of
 * one kernel per operation, ~5 a layer) or IRIS_DECODE_STEP (one cooperative
 * launch a pass, one block a multiprocessor streaming every layer's weights
 * through one shared-memory ring; mistral-dense without tensor parallelism;
 * IRIS_EINVAL where the shape, capacity or device does not allow it). Both
 * give the same values. */
int iris_session_set_decode_path(IrisSession* session, int mode);
#define IRIS_DECODE_AUTO 0
#define IRIS_DECODE_GRAPH 1
#define IRIS_DECODE_STEP 2
/* The decode path in use: IRIS_DECODE_GRAPH or IRIS_DECODE_STEP. */
int iris_session_decode_path(const IrisSession* session);
/* The persistent step's launch plan: plan[0] = 0 when the session can use it,
 * else why not (1 shape, 2 no kernel for the head shape, 3 device, 4 shared
 * memory, 5 occupancy, 6 not a single-GPU mistral-dense model); then blocks,
 * ring slots, bytes a slot, bytes of the planes region, dynamic shared
 * memory, blocks a head group, positions a block at most (8 values). */
int iris_session_step_plan(const IrisSession* session, uint32_t* plan);
/* Profiling hook of the persistent step: with enable != 0 every pass records
 * global-timer stamps (ns) per block and stage into a device buffer of
 * blocks * stages * 8 values (blocks = plan[1], stages = 2 + 5 layers):
 * 0 input ready, 7 share written; products: 1 prologue done, 2 warp 0's last
 * tile taken, 6 the producer issued the last tile; attention: 1 first key
 * slot landed, 2 scores done, 3 and 4 group exchanges passed, 5 value sums
 * added, 6 the producer issued the last value row. iris_session_get_step_trace
 * copies the last pass's out. */
int iris_session_step_trace(IrisSession* session, int enable);
int iris_session_get_step_trace(const IrisSession* session, uint64_t* out, uint64_t count);
/* Reads count K/V rows of one layer starting at position first
 * (kv_heads*head_dim values each). For a gemma sliding layer these are the
 * positions the window still holds. */
int iris_session_get_kv(const IrisSession* session, uint32_t layer, uint32_t first, uint32_t count,
                        int32_t* k, int32_t* v);
void iris_session_free(IrisSession* session);

/* Stream capture for replaying a sequence of this library's launches as one
 * CUDA graph (timing, serving loops). Between begin and end, launches on
 * `stream` (cudaStream_t as void*) from this thread are recorded, not run. */
int iris_capture_begin(void* stream);
int iris_capture_end(void* stream, void** graph_exec);
int iris_graph_launch(void* graph_exec, void* stream);
void iris_graph_free(void* graph_exec);

/* ---------------------------------------------------------------------------
 * 4. The teacher-forced chain stage: one layer over one range of rows
 *    (mistral/layer.rs:107-270 via stage.rs:172-226; gemma
 *    prefill_range.rs:307-333). Host buffers in and out.
 * ------------------------------------------------------------------------- */
/* The embedding rows of token ids (direct/src/view_kernels.rs:37-57 ->
 * model.rs:316-330 dequantize_row; gemma-dense times embedding_scale):
 * rows[i*H ..] for ids[i], host buffers. The chain's first stage takes these
 * rows as its input. Single-GPU models. */
int iris_model_embed(IrisModel* model, const uint32_t* ids, uint32_t n, int32_t* rows);
/* The chain's head check (kernels/src/kernels/sequence_check.rs:232-300,
 * run_sequence_check_direct): for each of the n predicting rows (H values
 * each; check_positions at sequence_check.rs:89-125 lists them: the
 * previous range's last row, then this range's rows), rms_norm with the
 * model's final norm, the exact dot_row against every vocabulary row of the
 * head, softcap, and the first maximum (Argmax, sequence_check.rs:55-70):
 * token_ids[i] and (if values is not NULL) values[i] = its score. Ranges of
 * 32 or more rows run on the tensor-core GEMM (logits epilogue). The
 * selection bookkeeping around it (decode_edge, faults, the transcript) is
 * the caller's. Tensor-parallel models: every rank calls it. */
int iris_sequence_check_select(IrisModel* model, const int32_t* rows, uint32_t n, uint32_t* token_ids,
                               int32_t* values);
/* mistral-dense: prior_k/prior_v hold the layer's keys for positions
 * 0..start (start rows). Writes m output rows and the range's own K/V. */
int iris_mistral_layer_range(IrisModel* model, uint32_t layer, const int32_t* rows_in, uint32_t m,
                             uint32_t start, const int32_t* prior_k, const int32_t* prior_v,
                             int32_t* rows_out, int32_t* own_k, int32_t* own_v);
/* gemma-dense: the per-layer inputs of token ids (direct/src/view_kernels.rs:
 * 59-99, prefill_prepare_aux: embedding row, model projection, norm, scales
 * and the PLE embedding): out[i*layers*ple + l*ple ..] is layer l's PLE row
 * of ids[i]. Single-GPU models. */
int iris_model_ple_rows(IrisModel* model, const uint32_t* ids, uint32_t n, int32_t* out);
/* gemma-dense: one layer over one range of m rows starting at position start
 * (kernels/src/prefill_range.rs:82-172, run_prefill_range_direct_with_weight_
 * cache; the layer prefill_range.rs:307-957). ple_rows: the range's PLE rows
 * of this layer ([m][ple], from iris_model_ple_rows). A layer with its own
 * K/V takes the keys carried from the ranges before (n_prior rows at
 * consecutive positions prior_pos[0].., kv_heads*head_dim values each) and
 * must be given every position its window still holds before the range,
 * [max(0, start + 1 - window), start) (window 0: [0, start)), ending at
 * start - 1; a layer that shares a donor's K/V (kv_donor_layer >= 0) takes
 * the donor layer's keys for this range instead (n_donor rows at consecutive
 * positions covering [max(0, start + 1 - window), start + m)). Keys that do
 * not cover those positions are refused with IRIS_EWINDOW before anything
 * runs: the reference's cache-coverage fault (prefill-range/src/lib.rs:
 * 1237-1288), which it reports as empty rows with the carried K/V handed
 * on. Writes m output rows and the range's own K/V (sharing layers compute
 * theirs too). The keys this range hands to the next one are the carried
 * keys from position max(0, start + 1 - window) on, then its own
 * (prefill_range.rs:849-860, output_kv); the caller assembles them. */
int iris_gemma_layer_range(IrisModel* model, uint32_t layer, const int32_t* rows_in, uint32_t m,
                           uint32_t start, const int32_t* ple_rows, uint32_t n_prior, const uint32_t* prior_pos,
                           const int32_t* prior_k, const int32_t* prior_v, uint32_t n_donor,
                           const uint32_t* donor_pos, const int32_t* donor_k, const int32_t* donor_v,
                           int32_t* rows_out, int32_t* own_k, int32_t* own_v);

/* The claim's teacher-forced pass range by range on a session (device-
 * resident: the session's cache carries every layer's K/V from range to
 * range; kernels/src/mistral/stage.rs:172-226, prefill_range.rs:82-172 per
 * stage, chain_runner.rs:503-597 for the order). A range of n <= 512 rows at
 * positions [length, length + n): iris_session_range_begin embeds the ids
 * (gemma: also every layer's PLE rows); iris_session_range_layer runs layer
 * `layer` (0, 1, ... in order) and queues asynchronous copies of the
 * stage's output rows ([n][hidden]) and own K/V ([n][kv_heads*head_dim]
 * each) into the host buffers given (NULL skips one; pinned memory from
 * iris_host_alloc keeps the copies asynchronous; they run on a copy stream
 * of the session's, beside the next layers), and returns a ticket that
 * iris_session_ticket_wait waits for (the buffers may be read, or reused,
 * after that; a session tracks the last 64 tickets); iris_session_range_end,
 * after the last layer, runs the head check over the range's final rows
 * (rms_norm(final), the head, softcap, first maximum per row,
 * sequence_check.rs:232-300) into token_ids / values (NULL skips it), waits
 * for the range and advances the session's length by n. Single-GPU models;
 * IRIS_ESTATE when called out of order. */
int iris_session_range_begin(IrisSession* session, const uint32_t* ids, uint32_t n);
int iris_session_range_layer(IrisSession* session, uint32_t layer, int32_t* rows_out, int32_t* own_k,
                             int32_t* own_v, uint32_t* ticket);
/* As iris_session_range_layer, but the stage's rows, own K and own V are
 * hashed on the device instead of copied out: leaves_out receives the
 * SHA-256 (FIPS 180-4) of every consecutive leaf_bytes piece of the rows'
 * bytes, then of the K rows', then of the V rows' (the last piece of each
 * shorter), 32 bytes a digest: ceil(n*hidden*4 / leaf_bytes) +
 * 2 ceil(n*kv_heads*head_dim*4 / leaf_bytes) digests. leaf_bytes: a
 * multiple of 64 up to 1 MiB. The leaf digests of a stage record whose
 * digest is taken on the host (the two-level canonical record). */
int iris_session_range_layer_leaves(IrisSession* session, uint32_t layer, uint32_t leaf_bytes, uint8_t* leaves_out,
                                    uint32_t* ticket);
/* The next `count` layers of the range (count <= 64) in one call, as
 * iris_session_range_layer_leaves each: leaves_out[i] and tickets[i] are
 * layer i's (fewer host calls a range). */
int iris_session_range_layers_leaves(IrisSession* session, uint32_t count, uint32_t leaf_bytes,
                                     uint8_t* const* leaves_out, uint32_t* tickets);
int iris_session_ticket_wait(IrisSession* session, uint32_t ticket);
int iris_session_range_end(IrisSession* session, uint32_t* token_ids, int32_t* values);
/* Page-locked host memory for the copies above (cudaHostAlloc). */
int iris_host_alloc(uint64_t bytes, void** out);
void iris_host_free(void* ptr);

/* ---------------------------------------------------------------------------
 * 5. Seeded synthetic weights (the benchmark configs' inputs). Host copies of
 *    the generator the device uses in iris_model_synthesize.
 * ------------------------------------------------------------------------- */
int iris_synth_q8(uint64_t seed, uint32_t tensor, int32_t layer, uint32_t rows, uint32_t cols,
                  int per_block_scales, uint8_t* blocks);
/* Rows [row0, row0 + rows) x columns [col0, col0 + cols) of the synthetic
 * tensor with full_cols columns (a tensor-parallel shard), as Q8_0 blocks. */
int iris_synth_q8_block(uint64_t seed, uint32_t tensor, int32_t layer, uint32_t rows, uint32_t cols,
                        uint32_t row0, uint32_t col0, uint32_t full_cols, int per_block_scales,
                        uint8_t* blocks);
int iris_synth_values(uint64_t seed, uint32_t tensor, int32_t layer, uint64_t count, uint32_t fan_in,
                      int32_t* values);

/* No counterpart in the reference (inspection of the softmax_exp_term
 * table, det-num ops.rs:508-556). out[i] = the exp term the many-query
 * softmax uses for a score first+i below the maximum (2^32 at distance 0, 0
 * from 2^20 = 16.0 on), read through the same device lookup. Fills the
 * current device's table if needed; synchronous; first + count <= 2^31. */
int iris_softmax_exp_terms(uint32_t first, uint32_t count, uint64_t* out);

/* No counterpart in the reference (the reference has no device waits; its
 * host side latches a failed device call and falls back, gpu.rs:126-134).
 * Runs the library's two bounded device waits alone in one small kernel on
 * the current device: kind 0 an mbarrier phase (the TMA and tensor-core
 * pipelines), kind 1 a global arrival counter (the persistent step's
 * stages). With release != 0 another thread completes the wait and the call
 * returns 0; with release == 0 nothing does, the wait gives up after about a
 * second and the call returns IRIS_ESTALL, the device staying usable.
 * Synchronous; clears the library's fault word before and after. */
int iris_wait_probe(int kind, int release);

/* Message for any status this library returns. */
const char* iris_error(int code);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
#ifdef __cplusplus
}
#endif
#endif /* IRIS_B200_H */
