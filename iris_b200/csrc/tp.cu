// Tensor parallelism of the decode and range passes over NCCL.
//
// A rank holds the query heads and key/value heads of its share of the kv
// groups (column-parallel q|k|v), its share of the FFN rows (column-parallel
// gate|up), the matching input columns of o and down (row-parallel) and its
// share of the vocabulary (head). A row-parallel product leaves every output
// row's unrounded 128-bit sum over the rank's columns as four 32-bit limbs in
// int64 (EPI_PARTIAL); an NCCL sum over the ranks adds the limbs exactly
// (integer addition is associative and the limb sums cannot overflow), and
// tp_finish rebuilds the 128-bit total, rounds it once (q8.rs:69-71) and adds
// the residual. The head's first-maximum keys carry global token ids and meet
// in an NCCL max. NCCL is loaded at run time (the library torch loaded, else
// the system's), so the library itself links no NCCL.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>

#include "../../include/iris_b200.h"
#include "detnum.cuh"
#include "q8.cuh"
#include "tp.cuh"

namespace iris {

namespace {

struct NcclApi {
  bool ok = false;
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
};

NcclApi g_nccl;
std::once_flag g_nccl_once;

void load_nccl() {
  void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);  // the copy already in the process
  if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
  if (!h) return;
  g_nccl.get_unique_id = (decltype(g_nccl.get_unique_id))dlsym(h, "ncclGetUniqueId");
  g_nccl.comm_init_rank = (decltype(g_nccl.comm_init_rank))dlsym(h, "ncclCommInitRank");
  g_nccl.comm_destroy = (decltype(g_nccl.comm_destroy))dlsym(h, "ncclCommDestroy");
  g_nccl.all_reduce = (decltype(g_nccl.all_reduce))dlsym(h, "ncclAllReduce");
  g_nccl.all_gather = (decltype(g_nccl.all_gather))dlsym(h, "ncclAllGather");
  g_nccl.ok = g_nccl.get_unique_id && g_nccl.comm_init_rank && g_nccl.comm_destroy && g_nccl.all_reduce &&
              g_nccl.all_gather;
}

const NcclApi* nccl() {
  std::call_once(g_nccl_once, load_nccl);
  return g_nccl.ok ? &g_nccl : nullptr;
}

cudaError_t from_nccl(ncclResult_t r) { return r == ncclSuccess ? cudaSuccess : cudaErrorUnknown; }

// out[t][row] = add_sat(round_q24(total), resid[t][row]) from the summed limbs.
__global__ void tp_finish_kernel(const int64_t* __restrict__ limbs, uint32_t tokens, uint32_t rows,
                                 const int32_t* resid, int32_t* out) {
  pdl_wait();
  pdl_trigger();
  const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (uint64_t)tokens * rows) return;
  const int64_t* l = limbs + i * 4;
  // total = l0 + 2^32 l1 + 2^64 l2 + 2^96 l3; l0, l1, l2 are sums of unsigned
  // 32-bit limbs (non-negative, below 2^63), l3 of signed ones
  Acc128 acc{(uint64_t)l[0], 0};
  acc128_add(acc, (uint64_t)l[1] << 32, (int64_t)((uint64_t)l[1] >> 32));
  acc128_add(acc, 0, l[2]);
  acc128_add(acc, 0, (int64_t)((uint64_t)l[3] << 32));
  out[i] = add_sat(acc128_round_q24(acc), resid[i]);
}

}  // namespace

bool tp_available() { return nccl() != nullptr; }

cudaError_t tp_unique_id(uint8_t* out) {
  const NcclApi* n = nccl();
  if (!n) return cudaErrorNotSupported;
  ncclUniqueId id;
  cudaError_t e = from_nccl(n->get_unique_id(&id));
  if (e == cudaSuccess) memcpy(out, id.internal, NCCL_UNIQUE_ID_BYTES);
  return e;
}

cudaError_t tp_comm_init(void** comm, uint32_t rank, uint32_t world, const uint8_t* id_bytes) {
  const NcclApi* n = nccl();
  if (!n) return cudaErrorNotSupported;
  ncclUniqueId id;
  memcpy(id.internal, id_bytes, NCCL_UNIQUE_ID_BYTES);
  ncclComm_t c = nullptr;
  cudaError_t e = from_nccl(n->comm_init_rank(&c, (int)world, id, (int)rank));
  *comm = e == cudaSuccess ? (void*)c : nullptr;
  return e;
}

void tp_comm_free(void* comm) {
  const NcclApi* n = nccl();
  if (n && comm) n->comm_destroy((ncclComm_t)comm);
}

cudaError_t tp_sum_limbs(void* comm, int64_t* limbs, size_t count, cudaStream_t s) {
  return from_nccl(nccl()->all_reduce(limbs, limbs, count, ncclInt64, ncclSum, (ncclComm_t)comm, s));
}

cudaError_t tp_max_keys(void* comm, unsigned long long* keys, size_t count, cudaStream_t s) {
  return from_nccl(nccl()->all_reduce(keys, keys, count, ncclUint64, ncclMax, (ncclComm_t)comm, s));
}

cudaError_t tp_gather_i32(void* comm, const int32_t* part, int32_t* full, size_t count, cudaStream_t s) {
  return from_nccl(nccl()->all_gather(part, full, count, ncclInt32, (ncclComm_t)comm, s));
}

cudaError_t launch_tp_finish(const int64_t* limbs, uint32_t tokens, uint32_t rows, const int32_t* resid,
                             int32_t* out, cudaStream_t s) {
  const uint64_t n = (uint64_t)tokens * rows;
  if (n == 0) return cudaSuccess;
  return launch_k(tp_finish_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, s, limbs, tokens, rows, resid,
                  out);
}

}  // namespace iris

extern "C" int iris_tp_unique_id(uint8_t* out) {
  if (!out) return IRIS_EINVAL;
  return (int)iris::tp_unique_id(out);
}
