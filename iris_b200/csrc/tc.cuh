// Many-token Q8_0 products on the fifth-generation tensor cores (tcgen05,
// kind::i8), over a per-row pre-scaled copy of the weights.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "q8.cuh"

namespace iris {

// Tile of one block: 128 weight rows (the MMA's M, one TMEM lane a row) by
// 128 tokens (one-plane copies) or kTcTok = 64 tokens (three-plane copies),
// K staged 128 bytes at a time.
constexpr uint32_t kTcRows = 128, kTcTok = 64, kTcKChunk = 128;
// Widest K: the largest diagonal sum (three byte-plane products a column)
// spans less than 2^32, so its int32 accumulator is exact modulo 2^32.
constexpr uint32_t kTcMaxCols = 18848;
// Fewest tokens worth a tensor-core launch (below: the mma.sync GEMM).
constexpr uint32_t kTcMinTokens = 32;
// Widest spread of a row's block-scale exponents that the three weight
// planes hold (|q m 2^spread| < 2^23).
constexpr int32_t kTcMaxSpread = 5;

// Builds the tensor-core copy of a matrix once: one signed byte plane and a
// (mantissa, exponent) a row where every row has one scale, else three byte
// planes of the pre-scaled weights and a shift a row (planes = 3 asks for
// the three-plane form in any case, for measurement). Sets m->tc_state to 1
// when the copy is usable, 2 when the matrix does not qualify (three planes
// needed and a row's scale exponents spread wider than kTcMaxSpread, K above
// kTcMaxCols) or the device has no room for it; only a launch failure is an
// error. Synchronises `stream`.
cudaError_t tc_prepare(Q8GpuMatrix* m, cudaStream_t stream, int planes = 0);
// Whether the tensor-core GEMM takes this product.
bool tc_usable(const ProductArgs& a);
cudaError_t launch_gemm_tc(const ProductArgs& a, EpiMode epi, cudaStream_t stream);
cudaError_t prepare_tc_kernels();
// Multiprocessors of the current device (q8.cu).
int device_sms();

}  // namespace iris
