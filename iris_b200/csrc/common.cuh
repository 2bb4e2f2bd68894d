// Shared device helpers: error plumbing, PTX wrappers and the byte-plane
// activation format the Q8 kernels consume.
//
// Byte planes. A Q16.16 activation a (int32) is split into four bytes
// a = b0 + 2^8 b1 + 2^16 b2 + 2^24 b3 with b0..b2 unsigned and b3 signed. A
// vector of K activations is stored as four K-byte planes, plane p holding
// byte p of every value. A Q8_0 block sum sum_j q_j a_j then becomes four
// dp4a chains, each exact in int32 (|q| <= 128, b <= 255, 16 or 32 terms),
// recombined exactly in 64 bits. Planes are written once per activation row
// and read by every block of the product that consumes it.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "detnum.cuh"

namespace iris {

#define IRIS_CHECK(expr)                         \
  do {                                           \
    cudaError_t _e = (expr);                     \
    if (_e != cudaSuccess) return (int)_e;       \
  } while (0)

// ---- programmatic dependent launch ------------------------------------------
//
// Kernels on the inference path are launched with programmatic stream
// serialization: kernel N+1 may be scheduled while kernel N finishes. Every
// such kernel calls pdl_wait() before it reads anything its predecessor wrote
// or writes anything an earlier kernel may still read, and pdl_trigger()
// right after it (its successor may then launch). So when a kernel starts,
// every kernel before its predecessor has completed: work placed before
// pdl_wait() may read data written two or more kernels earlier (the decode
// position, cached K/V rows of earlier positions) and immutable data
// (weights).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                     Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

__device__ __forceinline__ int dp4a_su(uint32_t w_s8, uint32_t a_u8, int c) {
  int d;
  asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(w_s8), "r"(a_u8), "r"(c));
  return d;
}
__device__ __forceinline__ int dp4a_ss(uint32_t w_s8, uint32_t a_s8, int c) {
  int d;
  asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(w_s8), "r"(a_s8), "r"(c));
  return d;
}

// Streaming 16-byte load that bypasses L1 (weights are read once per pass).
__device__ __forceinline__ uint4 ld_stream_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ uint16_t ld_stream_u16(const uint16_t* p) {
  uint16_t v;
  asm volatile("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(v) : "l"(p));
  return v;
}

// ---- mbarrier + bulk-copy (TMA) pipeline primitives ------------------------

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// try_wait that may suspend the thread for up to 20 us while the phase is
// incomplete (it resumes as soon as the phase completes), so that waiting
// warps do not take issue slots from the working ones.
__device__ __forceinline__ bool mbar_try_wait_suspend(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity), "r"(20000u)
      : "memory");
  return ok != 0;
}
// Waits for the phase of `bar` with the given parity to complete, giving up
// after about one second; a give-up is recorded in *fault.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, unsigned int* fault) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait_suspend(bar, parity)) return true;
    if ((i & 15) == 0 && global_ns() - t0 > 1000000000ull) {
      atomicOr(fault, 1u);
      return false;
    }
  }
}
// System-scope release store / acquire load of a global word: flags that
// another GPU writes into this GPU's memory (or this GPU into a peer's) over
// NVLink.
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// 16-byte asynchronous global -> shared copy (cp.async) and its commit.
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }

// L2 policy for data read once per pass (weights): evict first.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
// Bulk copy global -> shared (no multicast), completing on `bar`. Both
// addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                          uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
      ::"r"(smem_addr(dst)), "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

// acc += a * b, the 32 x 32 -> 64-bit product added with 64-bit wraparound
// (one multiply-add).
__device__ __forceinline__ void mac_wide(int64_t& acc, int32_t a, int32_t b) {
  asm("mad.wide.s32 %0, %1, %2, %0;" : "+l"(acc) : "r"(a), "r"(b));
}

// Sixteen weights (one uint4) against the four planes of the same sixteen
// activations: the exact 64-bit partial block sum.
__device__ __forceinline__ int64_t q8_partial16(uint4 w, uint4 p0, uint4 p1, uint4 p2, uint4 p3) {
  int s0 = dp4a_su(w.x, p0.x, 0);
  s0 = dp4a_su(w.y, p0.y, s0);
  s0 = dp4a_su(w.z, p0.z, s0);
  s0 = dp4a_su(w.w, p0.w, s0);
  int s1 = dp4a_su(w.x, p1.x, 0);
  s1 = dp4a_su(w.y, p1.y, s1);
  s1 = dp4a_su(w.z, p1.z, s1);
  s1 = dp4a_su(w.w, p1.w, s1);
  int s2 = dp4a_su(w.x, p2.x, 0);
  s2 = dp4a_su(w.y, p2.y, s2);
  s2 = dp4a_su(w.z, p2.z, s2);
  s2 = dp4a_su(w.w, p2.w, s2);
  int s3 = dp4a_ss(w.x, p3.x, 0);
  s3 = dp4a_ss(w.y, p3.y, s3);
  s3 = dp4a_ss(w.z, p3.z, s3);
  s3 = dp4a_ss(w.w, p3.w, s3);
  // |s0 + 256 s1| < 2^28 and |s2 + 256 s3| < 2^27: both exact in int32.
  return (int64_t)(s0 + s1 * 256) + ((int64_t)(s2 + s3 * 256) << 16);
}

// Three planes suffice when |a| < 2^23: a = b0 + 2^8 b1 + 2^16 b2 with b2 the
// signed byte a >> 16, which is byte 2 of a (byte 3 is its sign extension).
__device__ __forceinline__ bool fits_three_planes(int32_t a) { return a >= -(1 << 23) && a < (1 << 23); }
// Every byte of plane 3 is the sign extension of the same value's plane-2 byte.
__device__ __forceinline__ bool planes_sign_extended(uint32_t p2, uint32_t p3) {
  // per byte: 0xFF where the plane-2 byte is negative, else 0x00
  uint32_t ext = ((p2 >> 7) & 0x01010101u) * 0xFFu;
  return p3 == ext;
}
__device__ __forceinline__ int64_t q8_partial16_three(uint4 w, uint4 p0, uint4 p1, uint4 p2) {
  int s0 = dp4a_su(w.x, p0.x, 0);
  s0 = dp4a_su(w.y, p0.y, s0);
  s0 = dp4a_su(w.z, p0.z, s0);
  s0 = dp4a_su(w.w, p0.w, s0);
  int s1 = dp4a_su(w.x, p1.x, 0);
  s1 = dp4a_su(w.y, p1.y, s1);
  s1 = dp4a_su(w.z, p1.z, s1);
  s1 = dp4a_su(w.w, p1.w, s1);
  int s2 = dp4a_ss(w.x, p2.x, 0);
  s2 = dp4a_ss(w.y, p2.y, s2);
  s2 = dp4a_ss(w.z, p2.z, s2);
  s2 = dp4a_ss(w.w, p2.w, s2);
  return (int64_t)(s0 + s1 * 256) + ((int64_t)s2 << 16);
}

// Warp-wide sum of a 128-bit accumulator (every lane ends with the total).
__device__ __forceinline__ Acc128 warp_sum_acc128(Acc128 a) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    uint64_t lo = __shfl_xor_sync(0xffffffffu, a.lo, off);
    int64_t hi = __shfl_xor_sync(0xffffffffu, a.hi, off);
    acc128_add(a, lo, hi);
  }
  return a;
}

__device__ __forceinline__ int64_t warp_sum_i64(int64_t v) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1)
    v = (int64_t)((uint64_t)v + (uint64_t)__shfl_xor_sync(0xffffffffu, v, off));
  return v;
}
__device__ __forceinline__ uint64_t warp_sum_sat_nonneg(uint64_t v) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) v = add_sat_nonneg(v, __shfl_xor_sync(0xffffffffu, v, off));
  return v;
}

// inv_sqrt_acc (ops.rs:722-771) by a warp: the largest c with c^2 x <= 2^64
// is found five bits a round (lane j tests the next five bits = j; the
// predicate falls with c, so the lanes that pass are a prefix), then the same
// tie-break. Every lane passes the same x and gets the same value.
__device__ __forceinline__ int32_t inv_sqrt_acc_warp(int64_t xs) {
  if (xs <= 0) return INT32_MAX;
  const uint64_t x = (uint64_t)xs;
  if (inv_sqrt_le_target((uint32_t)INT32_MAX, x)) return INT32_MAX;
  const uint32_t lane = threadIdx.x & 31;
  uint32_t base = 0;  // c^2 x <= 2^64 holds at base
#pragma unroll
  for (int shift = 26; shift >= 1; shift -= 5) {
    const uint32_t ok = __ballot_sync(0xffffffffu, inv_sqrt_le_target(base + (lane << shift), x));
    base += (uint32_t)(__popc(ok) - 1) << shift;
  }
  if (inv_sqrt_le_target(base + 1, x)) base += 1;
  return inv_sqrt_pick(base, x);
}

// Writes one activation into the four planes of a K-wide row.
__device__ __forceinline__ void put_planes(uint8_t* planes, uint32_t k, uint32_t idx, int32_t v) {
  uint32_t u = (uint32_t)v;
  planes[idx] = (uint8_t)u;
  planes[k + idx] = (uint8_t)(u >> 8);
  planes[2 * k + idx] = (uint8_t)(u >> 16);
  planes[3 * k + idx] = (uint8_t)(u >> 24);
}
// Four consecutive activations as one 32-bit word per plane.
__device__ __forceinline__ void put_planes4(uint8_t* planes, uint32_t k, uint32_t idx, int4 v) {
  uint32_t a = (uint32_t)v.x, b = (uint32_t)v.y, c = (uint32_t)v.z, d = (uint32_t)v.w;
  uint32_t w0 = __byte_perm(__byte_perm(a, b, 0x0040), __byte_perm(c, d, 0x0040), 0x5410);
  uint32_t w1 = __byte_perm(__byte_perm(a, b, 0x0051), __byte_perm(c, d, 0x0051), 0x5410);
  uint32_t w2 = __byte_perm(__byte_perm(a, b, 0x0062), __byte_perm(c, d, 0x0062), 0x5410);
  uint32_t w3 = __byte_perm(__byte_perm(a, b, 0x0073), __byte_perm(c, d, 0x0073), 0x5410);
  *(uint32_t*)(planes + idx) = w0;
  *(uint32_t*)(planes + k + idx) = w1;
  *(uint32_t*)(planes + 2 * k + idx) = w2;
  *(uint32_t*)(planes + 3 * k + idx) = w3;
}

}  // namespace iris
