// Q8_0 matrices on the device and the exact products over them.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

// Device layout of a Q8_0 matrix, chosen for the products that stream it.
//
// The 34-byte GGUF blocks are split into int8 values and fp16 scale bits, and
// both are stored tile by tile: a tile is kQ8TileRows consecutive rows times
// kc consecutive columns (a "slice", kc a multiple of 32 dividing cols), and
// the tiles of a matrix follow each other group-major, slice-minor:
//
//   values: tile (g, s) at ((g * nslices + s) * kQ8TileRows) * kc bytes,
//           row r of the tile at + r * kc, column c of the slice at + c;
//   scales: tile (g, s) at ((g * nslices + s) * kQ8TileRows) * (kc / 32)
//           entries, row r at + r * (kc / 32), block b of the slice at + b.
//
// So every tile is one contiguous run of values (16 kc bytes) and one of
// scales (kc bytes): the decode GEMV moves a tile with two bulk copies. The
// rows are padded to a whole tile group with zeros. 1.0625 bytes a weight.
constexpr uint32_t kQ8TileRows = 16;

struct Q8GpuMatrix {
  int8_t* q;
  uint16_t* s;
  uint32_t rows, cols;
  uint32_t kc, nslices, groups;
  bool owns;
  // Tensor-core copy for many-token products (built on first use), in one of
  // two forms (tc_planes), tc_rows = rows rounded up to 128:
  //  - 1: every row has one scale (each block with a non-zero scale has the
  //    same scale bits): the signed byte plane W'[r][k] = q (0 in blocks
  //    whose scale is zero) at tc + r * cols, the row's scale as the signed
  //    mantissa tc_mant[r] and exponent tc_shift[r] (q8_scale_parts);
  //  - 3: byte planes p of W'[r][k] = q m 2^(e - shift[r]) at
  //    tc + (p * tc_rows + r) * cols (planes 0 and 1 unsigned, plane 2
  //    signed), tc_mant unused.
  // tc_state: 0 not built, 1 ready, 2 not usable.
  uint8_t* tc;
  uint8_t* tc_shift;
  int16_t* tc_mant;
  uint32_t tc_rows, tc_planes;
  int tc_state;  // read and written only through tc_state_get / _set / _claim
  uint32_t version;  // bumped whenever the weights change (tc_invalidate); read through q8_version
  uint64_t uniform_cache;  // q8_uniform_cached: ((version + 1) << 1) | one scale a row, 0 when not taken
};

namespace iris {

// A matrix may be used from several host threads at once (one product builds
// the tensor-core copy while another reads the state): the state word is
// published with release after tc / tc_shift / tc_rows are written, and read
// with acquire before they are used. Building starts by claiming 0 -> 2, so
// two threads never build one copy twice.
inline int tc_state_get(const Q8GpuMatrix* m) { return __atomic_load_n(&m->tc_state, __ATOMIC_ACQUIRE); }
inline void tc_state_set(Q8GpuMatrix* m, int v) { __atomic_store_n(&m->tc_state, v, __ATOMIC_RELEASE); }
inline uint32_t q8_version(const Q8GpuMatrix* m) { return __atomic_load_n(&m->version, __ATOMIC_ACQUIRE); }
inline bool tc_state_claim(Q8GpuMatrix* m) {
  int expected = 0;
  return __atomic_compare_exchange_n(&m->tc_state, &expected, 2, false, __ATOMIC_ACQ_REL, __ATOMIC_ACQUIRE);
}

// Slice width for a matrix of `cols` columns (cols a multiple of 32).
__host__ __device__ inline uint32_t q8_slice_cols(uint32_t cols) {
  if (cols % 2048 == 0) return 2048;
  if (cols % 1024 == 0) return 1024;
  if (cols <= 2048) return cols;
  for (uint32_t kc = 2048; kc >= 32; kc -= 32)
    if (cols % kc == 0) return kc;
  return 32;
}
__host__ __device__ inline size_t q8_value_offset(uint32_t kc, uint32_t nslices, uint32_t row, uint32_t col) {
  size_t tile = (size_t)(row / kQ8TileRows) * nslices + col / kc;
  return (tile * kQ8TileRows + row % kQ8TileRows) * kc + col % kc;
}
__host__ __device__ inline size_t q8_scale_offset(uint32_t kc, uint32_t nslices, uint32_t row, uint32_t block) {
  const uint32_t bps = kc / 32;
  size_t tile = (size_t)(row / kQ8TileRows) * nslices + block / bps;
  return (tile * kQ8TileRows + row % kQ8TileRows) * bps + block % bps;
}

enum InMode {
  IN_PLANES = 0,
  IN_NORM = 1,
  IN_RAW = 2,
  // gemma, one token: planes of rms_norm(x', norm_w), x' = add_sat(rms_norm(post_o,
  // post_w), x); block 0 stores x' to post_x (decode GEMV with EPI_GELU_MUL only)
  IN_POST_ATTN = 3
};
constexpr uint32_t kPostAttnMaxCols = 4608;  // IN_POST_ATTN rows: two int4 a thread of the decode GEMV
enum EpiMode {
  EPI_STORE = 0,     // out[row] = v
  EPI_RESID = 1,     // out[row] = add_sat(v, resid[row])
  EPI_QKV_ROPE = 2,  // mistral fused q|k|v rows: RoPE q,k; k,v into the cache
  EPI_SILU_MUL = 3,  // interleaved gate|up rows: planes of mul_sat(silu(g), u)
  EPI_GELU_MUL = 4,  // interleaved gate|up rows: planes of mul_sat(gelu(g), u)
  EPI_LOGITS = 5,    // logits (+softcap) and a first-maximum key
  EPI_PARTIAL = 6    // the unrounded 128-bit sums as four 32-bit limbs in int64 (tensor parallelism)
};

struct ProductArgs {
  const int8_t* q;
  const uint16_t* s;
  uint32_t rows, cols, tokens;
  uint32_t kc, nslices;    // tile layout of q and s
  // input: planes [tokens][4][cols], or raw / to-be-normed int32 [tokens][cols]
  const uint8_t* planes;
  const int32_t* x;
  const int32_t* norm_w;
  int64_t eps;
  // epilogue
  int32_t* out;            // [tokens][rows] (STORE/RESID/LOGITS), q rows for QKV
  uint32_t out_stride;     // values between tokens in out (default rows)
  const int32_t* resid;    // [tokens][rows]
  uint8_t* out_planes;     // [tokens][4][rows/2] for the gated products
  const int64_t* freqs;    // mistral inverse frequencies [head_dim/2]
  uint32_t head_dim, qd, kvd;
  int32_t* kcache;         // [positions][kvd]
  int32_t* vcache;
  const uint32_t* pos_ptr; // device position of token 0 (decode), or NULL
  uint32_t pos0;           // position of token 0 when pos_ptr is NULL
  unsigned long long* best;  // first-maximum key per token
  int32_t softcap;
  uint32_t row_base;         // global index of row 0 in first-maximum keys (vocabulary shards)
  int64_t* partial;          // EPI_PARTIAL: [tokens][rows][4] limbs
  unsigned long long* sumsq; // decode EPI_RESID (optional): receives the sum of the squares of the
                             // values this block wrote, clamped to i64::MAX
  const uint32_t* xepoch;    // EPI_PARTIAL into a peer-exchange slot: partial + ((epoch + 1) & 1) rows 4
  // Decode GEMV split scratch (optional): 2 words a row and a slice count a
  // tile group for split_groups groups, all zero between launches.
  unsigned long long* split_acc;
  unsigned int* split_count;
  uint32_t split_groups;
  // The matrix's tensor-core copy (Q8GpuMatrix::tc), or NULL
  const uint8_t* tc;
  const uint8_t* tc_shift;
  const int16_t* tc_mant;
  uint32_t tc_rows, tc_planes;
  // One-token products: every row of the matrix has one scale
  // (q8_uniform_cached), so the GEMV scales each row once a tile group
  uint32_t uniform;
  // Decode EPI_QKV_ROPE in the persistent step (optional): a release add on
  // gready[attention group] for each finished tile group of rows, for every
  // group of gready_hpc query heads that reads those rows
  unsigned int* gready;
  uint32_t gready_hpc;
  // Many-token EPI_QKV_ROPE (optional): the Q2.30 sine and cosine of every
  // frequency at each token's position, [tokens][head_dim / 2][2]
  const int64_t* rope_sc;
  // IN_POST_ATTN: the attention output product's row, its norm weights, and
  // where block 0 stores the new residual row (not x: other blocks read x)
  const int32_t* post_o;
  const int32_t* post_w;
  int32_t* post_x;
};

ProductArgs product_args(const Q8GpuMatrix* w, uint32_t tokens);

// Launches the product over args.tokens tokens: the decode GEMV for one token,
// the tiled GEMM otherwise (path forces one of them).
cudaError_t launch_product(const ProductArgs& a, InMode in, EpiMode epi, cudaStream_t stream,
                           int path = 0);
// int32 rows -> byte planes (optionally RMS-normalised), one block a token.
cudaError_t launch_planes(const int32_t* x, const int32_t* norm_w, int64_t eps, uint32_t tokens,
                          uint32_t cols, uint8_t* planes, cudaStream_t stream);

// Decodes a first-maximum key (value, lowest index) into its token id.
__host__ __device__ inline uint32_t best_key_token(unsigned long long key) {
  return 0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull);
}
__host__ __device__ inline int32_t best_key_value(unsigned long long key) {
  return (int32_t)((uint32_t)(key >> 32) ^ 0x80000000u);
}
__host__ __device__ inline unsigned long long best_key(int32_t v, uint32_t idx) {
  return ((unsigned long long)((uint32_t)v ^ 0x80000000u) << 32) | (0xFFFFFFFFu - idx);
}

// Non-zero once a kernel gave up a bounded wait (a stalled pipeline); read and
// cleared by the host.
cudaError_t take_device_fault(uint32_t* fault);
// Device address of that fault word (kernels of other files record into it);
// looked up once per device, before any stream capture.
unsigned int* device_fault_word();

// Uploads raw Q8_0 blocks into rows [row_offset + i*row_stride] of dst.
cudaError_t upload_q8_blocks(Q8GpuMatrix* dst, const uint8_t* host_blocks, uint32_t rows,
                             uint32_t cols, uint32_t row_stride, uint32_t row_offset,
                             int* bad_scale);
// Reads rows back as raw Q8_0 blocks.
cudaError_t download_q8_blocks(const Q8GpuMatrix* src, uint8_t* host_blocks, uint32_t rows,
                               uint32_t cols, uint32_t row_stride, uint32_t row_offset);
// Fills rows with the synthetic generator (synth.cuh).
cudaError_t synth_q8_rows(Q8GpuMatrix* dst, uint64_t seed, uint32_t tensor, int32_t layer,
                          uint32_t rows, uint32_t cols, uint32_t row_stride, uint32_t row_offset,
                          int per_block, cudaStream_t stream);
// Rows [row0, row0 + rows) x columns [col0, col0 + cols) of the synthetic
// tensor with full_cols columns (a tensor-parallel shard).
cudaError_t synth_q8_block(Q8GpuMatrix* dst, uint64_t seed, uint32_t tensor, int32_t layer, uint32_t rows,
                           uint32_t cols, uint32_t row0, uint32_t col0, uint32_t full_cols, uint32_t row_stride,
                           uint32_t row_offset, int per_block, cudaStream_t stream);
cudaError_t synth_values_dev(int32_t* dst, uint64_t seed, uint32_t tensor, int32_t layer,
                             uint64_t count, uint32_t fan_in, cudaStream_t stream);
Q8GpuMatrix* alloc_q8(uint32_t rows, uint32_t cols, cudaError_t* err);
void free_q8(Q8GpuMatrix* m);
// Whether every row of the matrix has one scale (all its blocks' scale bits
// equal) and cols <= 32768, so that a decode product may scale each row once
// (gemv_flush_uniform); runs a scan on `stream` and waits for it.
cudaError_t q8_rows_uniform(const Q8GpuMatrix* m, cudaStream_t stream, bool* uniform);
// q8_rows_uniform cached by weights version (a scan after a device-wide
// synchronisation when the cache is stale); false, without a scan, while
// `stream` is capturing a graph.
bool q8_uniform_cached(Q8GpuMatrix* m, cudaStream_t stream);

}  // namespace iris
