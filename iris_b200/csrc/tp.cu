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
#include <vector>

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
  Acc128 acc{0, 0};
  acc128_add_limbs(acc, l[0], l[1], l[2], l[3]);
  out[i] = add_sat(acc128_round_q24(acc), resid[i]);
}

__device__ __forceinline__ uint64_t ns_now() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// The peer-memory exchange of one row-parallel product (one token): this
// rank's limbs are in its slot `parity` (written by the product); block 0
// publishes them to every peer (release flag in the peer's memory), every
// block waits - bounded - until every peer has published the same epoch,
// then each thread sums its row's limbs over the ranks with loads from the
// peers' memory (NVLink), rounds once and adds the residual. The last block
// advances the epoch. Slots alternate by epoch parity: a rank rewrites a slot
// only after every peer has published the next epoch, i.e. finished reading
// this one.
__global__ void tp_p2p_finish_kernel(TpExchange x, uint32_t rows, const int32_t* resid, int32_t* out) {
  pdl_wait();
  pdl_trigger();
  __shared__ bool last_s;
  const uint32_t epoch = *x.epoch + 1, parity = epoch & 1;
  // The release store is cumulative over the product grid's writes of this
  // rank's limbs, which the grid dependency made visible to this thread; a
  // separate system fence before it cost ~3% of a decode step and adds nothing.
  if (blockIdx.x == 0 && threadIdx.x < x.world && threadIdx.x != x.rank)
    st_release_sys(x.peer_flags[threadIdx.x] + x.rank, epoch);
  if (threadIdx.x < x.world && threadIdx.x != x.rank) {
    const uint32_t* f = x.flags + threadIdx.x;
    if (ld_acquire_sys(f) < epoch) {
      const uint64_t t0 = ns_now();
      for (uint32_t i = 1;; ++i) {  // the flag is in this GPU's memory: a tight poll stays in L2
        if (ld_acquire_sys(f) >= epoch) break;
        if ((i & 255) == 0 && ns_now() - t0 > 1000000000ull) {
          if (x.fault) atomicOr(x.fault, 1u);
          break;
        }
      }
    }
  }
  __syncthreads();
  const uint32_t row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row < rows) {
    Acc128 acc{0, 0};
    for (uint32_t j = 0; j < x.world; ++j) {
      const int64_t* src = (j == x.rank ? x.part : x.peer_part[j]) + ((size_t)parity * rows + row) * 4;
      const longlong2 a = __ldcg((const longlong2*)src), b = __ldcg((const longlong2*)(src + 2));
      acc128_add_limbs(acc, a.x, a.y, b.x, b.y);
    }
    out[row] = add_sat(acc128_round_q24(acc), resid[row]);
  }
  __syncthreads();
  if (threadIdx.x == 0) last_s = atomicAdd(x.done, 1u) == gridDim.x - 1;
  __syncthreads();
  if (last_s && threadIdx.x == 0) {
    *x.done = 0;
    *x.epoch = epoch;
  }
}

}  // namespace

bool tp_available() { return nccl() != nullptr; }

cudaError_t tp_exchange_setup(void* comm, uint32_t rank, uint32_t world, uint32_t rows, TpExchange* x,
                              unsigned int* fault) {
  *x = TpExchange{};
  x->rank = rank;
  x->world = world;
  x->rows = rows;
  x->fault = fault;
  if (world > kTpMaxWorld) return cudaErrorInvalidValue;
  const size_t part_words = (size_t)2 * rows * 4 + 2 * kTpMaxWorld;  // limb slots, then key slots
  cudaError_t e = cudaMalloc((void**)&x->part, part_words * sizeof(int64_t));
  if (e == cudaSuccess) e = cudaMemset(x->part, 0, part_words * sizeof(int64_t));
  if (e == cudaSuccess) e = cudaMalloc((void**)&x->flags, kTpMaxWorld * sizeof(uint32_t));
  if (e == cudaSuccess) e = cudaMalloc((void**)&x->epoch, 2 * sizeof(uint32_t));
  if (e == cudaSuccess) e = cudaMemset(x->flags, 0, kTpMaxWorld * sizeof(uint32_t));
  if (e == cudaSuccess) e = cudaMemset(x->epoch, 0, 2 * sizeof(uint32_t));
  x->done = x->epoch + 1;
  // every rank's two IPC handles, gathered over NCCL
  cudaIpcMemHandle_t mine[2];
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&mine[0], x->part);
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&mine[1], x->flags);
  uint8_t* dev = nullptr;
  const size_t per = sizeof(mine);
  if (e == cudaSuccess) e = cudaMalloc((void**)&dev, per * (world + 1));
  if (e == cudaSuccess) e = cudaMemcpy(dev + per * world, mine, per, cudaMemcpyHostToDevice);
  if (e == cudaSuccess)
    e = from_nccl(nccl()->all_gather(dev + per * world, dev, per, ncclInt8, (ncclComm_t)comm, 0));
  std::vector<cudaIpcMemHandle_t> all(2 * world);
  if (e == cudaSuccess) e = cudaMemcpy(all.data(), dev, per * world, cudaMemcpyDeviceToHost);
  cudaFree(dev);
  for (uint32_t j = 0; j < world && e == cudaSuccess; ++j) {
    if (j == rank) {
      x->peer_part[j] = x->part;
      x->peer_flags[j] = x->flags;
      continue;
    }
    void* p = nullptr;
    e = cudaIpcOpenMemHandle(&p, all[2 * j], cudaIpcMemLazyEnablePeerAccess);
    x->peer_part[j] = (int64_t*)p;
    if (e == cudaSuccess) e = cudaIpcOpenMemHandle(&p, all[2 * j + 1], cudaIpcMemLazyEnablePeerAccess);
    x->peer_flags[j] = (uint32_t*)p;
  }
  return e;
}

void tp_exchange_free(TpExchange* x) {
  for (uint32_t j = 0; j < x->world; ++j) {
    if (j == x->rank) continue;
    if (x->peer_part[j]) cudaIpcCloseMemHandle(x->peer_part[j]);
    if (x->peer_flags[j]) cudaIpcCloseMemHandle(x->peer_flags[j]);
  }
  cudaFree(x->part);
  cudaFree(x->flags);
  cudaFree(x->epoch);
  *x = TpExchange{};
}

cudaError_t launch_tp_p2p_finish(const TpExchange& x, uint32_t rows, const int32_t* resid, int32_t* out,
                                 cudaStream_t s) {
  return launch_k(tp_p2p_finish_kernel, dim3((rows + 255) / 256), dim3(256), 0, s, x, rows, resid, out);
}

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
