// Q8_0 matrices on the device and the exact products over them.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

// Repacked device layout of a Q8_0 matrix: the 34-byte GGUF blocks split into
// int8 values [rows][cols] (16-byte aligned rows, coalesced 128-bit loads and
// bulk copies) and fp16 scale bits [rows][spitch], spitch = cols/32 rounded
// up to 8 entries so that every row of scales starts on a 16-byte boundary.
// 1.0625 bytes a weight, as in Q8_0, for the widths models use.
struct Q8GpuMatrix {
  int8_t* q;
  uint16_t* s;
  uint32_t rows, cols, spitch;
  bool owns;
};

namespace iris {

enum InMode { IN_PLANES = 0, IN_NORM = 1, IN_RAW = 2 };
enum EpiMode {
  EPI_STORE = 0,     // out[row] = v
  EPI_RESID = 1,     // out[row] = add_sat(v, resid[row])
  EPI_QKV_ROPE = 2,  // mistral fused q|k|v rows: RoPE q,k; k,v into the cache
  EPI_SILU_MUL = 3,  // interleaved gate|up rows: planes of mul_sat(silu(g), u)
  EPI_GELU_MUL = 4,  // interleaved gate|up rows: planes of mul_sat(gelu(g), u)
  EPI_LOGITS = 5     // logits (+softcap) and a first-maximum key
};

__host__ __device__ inline uint32_t q8_scale_pitch(uint32_t cols) { return ((cols / 32 + 7) / 8) * 8; }

struct ProductArgs {
  const int8_t* q;
  const uint16_t* s;
  uint32_t rows, cols, tokens;
  uint32_t spitch;         // scale entries per row (q8_scale_pitch(cols))
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
};

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
cudaError_t synth_values_dev(int32_t* dst, uint64_t seed, uint32_t tensor, int32_t layer,
                             uint64_t count, uint32_t fan_in, cudaStream_t stream);
Q8GpuMatrix* alloc_q8(uint32_t rows, uint32_t cols, cudaError_t* err);
void free_q8(Q8GpuMatrix* m);

}  // namespace iris
