// Tensor parallelism over NCCL (tp.cu).
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace iris {

constexpr uint32_t kTpMaxWorld = 8;

// Peer-memory exchange of one-token row-parallel products (tp.cu). Passed
// by value to the finish kernel.
struct TpExchange {
  uint32_t rank, world, rows;
  int64_t* part;                    // this rank's two slots [2][rows][4] limbs, then the key slots
  uint32_t* flags;                  // [world]: the last epoch each peer published
  uint32_t* epoch;                  // exchanges finished; epoch + 1 is the coming one
  uint32_t* done;                   // finish blocks done (last block advances the epoch)
  int64_t* peer_part[kTpMaxWorld];  // every rank's slots (this rank's own at [rank])
  uint32_t* peer_flags[kTpMaxWorld];
  unsigned int* fault;
};
// The first-maximum key slots of a rank (after its limb slots): [world][2] =
// (key, epoch) written by each peer, epoch last with release semantics.
__host__ __device__ inline unsigned long long* tp_key_slots(int64_t* part, uint32_t rows) {
  return (unsigned long long*)(part + (size_t)2 * rows * 4);
}
// Allocates the slots and flags, opens every peer's over CUDA IPC (handles
// gathered over NCCL). Every rank calls it together.
cudaError_t tp_exchange_setup(void* comm, uint32_t rank, uint32_t world, uint32_t rows, TpExchange* x,
                              unsigned int* fault);
void tp_exchange_free(TpExchange* x);
// out[row] = add_sat(round_q24(sum over ranks of the slot limbs), resid[row]).
cudaError_t launch_tp_p2p_finish(const TpExchange& x, uint32_t rows, const int32_t* resid, int32_t* out,
                                 cudaStream_t s);

bool tp_available();
cudaError_t tp_unique_id(uint8_t* out);  // 128 bytes
cudaError_t tp_comm_init(void** comm, uint32_t rank, uint32_t world, const uint8_t* id);
void tp_comm_free(void* comm);
// In-place sums of int64 limbs / maxima of first-maximum keys over the ranks.
cudaError_t tp_sum_limbs(void* comm, int64_t* limbs, size_t count, cudaStream_t s);
cudaError_t tp_max_keys(void* comm, unsigned long long* keys, size_t count, cudaStream_t s);
// Rank-major concatenation of every rank's `count` values.
cudaError_t tp_gather_i32(void* comm, const int32_t* part, int32_t* full, size_t count, cudaStream_t s);
// out[t][row] = add_sat(round_q24(sum of limbs), resid[t][row]).
cudaError_t launch_tp_finish(const int64_t* limbs, uint32_t tokens, uint32_t rows, const int32_t* resid,
                             int32_t* out, cudaStream_t s);

}  // namespace iris
