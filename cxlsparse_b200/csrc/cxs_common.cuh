// Shared device/host helpers for the cxlsparse_b200 sm_100a kernels.
//
// PTX wrappers for mbarriers, 1-D bulk copies (TMA bulk), 2-D tensor TMA,
// acquire/release flags and bounded waits. A bounded wait never traps: on
// timeout it records an error code in a device error word and returns false,
// so the kernel can finish and the host can report the failure.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "cxlsparse.h"

namespace cxs {

constexpr int kTokenBytes = 256;  // one KV token: K[64] then V[64], bf16
constexpr int kDim = 64;
constexpr int kGroups = 16;       // query heads per KV head (GQA group)
constexpr int32_t kInt32Max = 2147483647;

// Device error word bits (also documented in include/cxlsparse.h).
constexpr int kErrReadyTimeout = CXS_DEVICE_ERR_READY_TIMEOUT;
constexpr int kErrCopyTimeout = CXS_DEVICE_ERR_COPY_TIMEOUT;
constexpr int kErrBadBlock = CXS_DEVICE_ERR_BAD_BLOCK;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, int arrivals) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(arrivals)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(phase)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// Bounded wait on an mbarrier phase. Returns false (and sets *error) on timeout.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t phase, long long limit,
                                                  int* error) {
  long long start = clock64();
  while (!mbar_try_wait(bar, phase)) {
    if (clock64() - start > limit) {
      atomicOr(error, kErrCopyTimeout);
      return false;
    }
  }
  return true;
}

// 1-D bulk copy global -> shared, completing on an mbarrier (TMA bulk).
// Source and destination 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// 1-D bulk copy shared -> global in a bulk group, then wait for completion of
// the writes themselves (not only the shared-memory reads).
__device__ __forceinline__ void bulk_s2g_and_wait(void* dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst),
               "r"(smem_addr(src)), "r"(bytes)
               : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// 2-D tensor TMA load (no multicast) into shared memory, completing on an mbarrier.
__device__ __forceinline__ void tma_load_2d(void* dst, const void* tensor_map, int x, int y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cta.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3}], [%4];" ::"r"(smem_addr(dst)),
      "l"(tensor_map), "r"(x), "r"(y), "r"(smem_addr(bar))
      : "memory");
}

// 3-D tensor TMA load (no multicast): coordinates {x, y, z}.
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const void* tensor_map, int x, int y,
                                            int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cta.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst),
      "l"(tensor_map), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const void* tensor_map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(tensor_map) : "memory");
}

__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Relaxed load at GPU scope: a poll of a flag whose value is consumed later;
// a value seen set becomes an acquire with fence_acq_rel_gpu().
__device__ __forceinline__ int ld_relaxed(const int* p) {
  int v;
  asm volatile("ld.relaxed.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void fence_acq_rel_gpu() {
  asm volatile("fence.acq_rel.gpu;" ::: "memory");
}

__device__ __forceinline__ void st_release(int* p, int v) {
  asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Bounded acquire-spin on a ready flag. Returns false (and sets *error) on timeout.
__device__ __forceinline__ bool wait_ready_bounded(const int* flag, long long limit, int* error) {
  if (ld_acquire(flag)) return true;
  long long start = clock64();
  while (!ld_acquire(flag)) {
    __nanosleep(64);
    // Give up at once when another warp has already failed: the launch is
    // invalid and the host will raise, so waiting longer only delays that.
    if (*reinterpret_cast<volatile int*>(error) != 0 || clock64() - start > limit) {
      atomicOr(error, kErrReadyTimeout);
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ float2 unpack_bf16(uint32_t v) {
  __nv_bfloat162 h = *reinterpret_cast<__nv_bfloat162*>(&v);
  return __bfloat1622float2(h);
}

__device__ __forceinline__ float bf16_round(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

__device__ __forceinline__ int warp_sum(int v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

}  // namespace cxs

// Host-side status helpers (defined in capi.cu).
namespace cxs_host {
int set_error(int code, const char* fmt, ...);
int check_cuda(cudaError_t err, const char* what);
void count_launch();  // one kernel enqueued by this library
}  // namespace cxs_host

#define CXS_CUDA(call)                                                     \
  do {                                                                     \
    cudaError_t _e = (call);                                               \
    if (_e != cudaSuccess) return cxs_host::check_cuda(_e, #call);         \
  } while (0)

#define CXS_LAUNCH_CHECK(what)                                             \
  do {                                                                     \
    cudaError_t _e = cudaGetLastError();                                   \
    if (_e != cudaSuccess) return cxs_host::check_cuda(_e, what);          \
    cxs_host::count_launch();                                              \
  } while (0)
