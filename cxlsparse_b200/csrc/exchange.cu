// KV-head split exchange over NVLink: CUDA IPC sharing of gather buffers and
// flag arrays, and a bounded pair barrier (see cxs_exchange_barrier in
// include/cxlsparse.h). The attention launch itself stores every output row
// into the local and the peer gather buffer; this barrier only announces it.
#include <string.h>

#include "cxs_common.cuh"

using cxs_host::set_error;

namespace {

constexpr int kMaxRanks = 8;

struct PeerFlags {
  int32_t* flags[kMaxRanks];
};

__global__ void exchange_barrier_kernel(int32_t* counter, PeerFlags peers, int32_t* flags,
                                        int rank, int ranks, long long spin_limit,
                                        int32_t* error) {
  if (threadIdx.x != 0) return;
  const int step = *counter + 1;
  *counter = step;
  __threadfence_system();
  for (int p = 0; p < ranks; ++p) {
    if (p == rank) continue;
    asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(peers.flags[p] + rank), "r"(step)
                 : "memory");
  }
  for (int p = 0; p < ranks; ++p) {
    if (p == rank) continue;
    const long long begin = clock64();
    while (true) {
      int seen;
      asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(seen) : "l"(flags + p) : "memory");
      if (seen >= step) break;
      if (clock64() - begin > spin_limit) {
        atomicOr(error, CXS_DEVICE_ERR_READY_TIMEOUT);
        return;
      }
      __nanosleep(64);
    }
  }
}

}  // namespace

extern "C" int cxs_device_alloc(size_t bytes, void** ptr) {
  if (!bytes || !ptr) return set_error(CXS_ERR_INVALID, "empty device allocation");
  CXS_CUDA(cudaMalloc(ptr, bytes));
  CXS_CUDA(cudaMemset(*ptr, 0, bytes));
  return CXS_OK;
}

extern "C" int cxs_device_free(void* ptr) {
  if (ptr) CXS_CUDA(cudaFree(ptr));
  return CXS_OK;
}

extern "C" int cxs_ipc_get_handle(const void* ptr, void* handle) {
  if (!ptr || !handle) return set_error(CXS_ERR_INVALID, "null IPC argument");
  cudaIpcMemHandle_t h;
  CXS_CUDA(cudaIpcGetMemHandle(&h, const_cast<void*>(ptr)));
  static_assert(sizeof(h) == 64, "CUDA IPC handles are 64 bytes");
  memcpy(handle, &h, sizeof(h));
  return CXS_OK;
}

extern "C" int cxs_ipc_open_handle(const void* handle, void** ptr) {
  if (!ptr || !handle) return set_error(CXS_ERR_INVALID, "null IPC argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  CXS_CUDA(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return CXS_OK;
}

extern "C" int cxs_ipc_close(void* ptr) {
  if (ptr) CXS_CUDA(cudaIpcCloseMemHandle(ptr));
  return CXS_OK;
}

extern "C" int cxs_exchange_barrier(int32_t* counter, int32_t* const* peer_flags, int32_t* flags,
                                    int32_t rank, int32_t ranks, int64_t spin_limit,
                                    int32_t* error, void* stream) {
  if (ranks < 2 || ranks > kMaxRanks || rank < 0 || rank >= ranks)
    return set_error(CXS_ERR_INVALID, "exchange needs 2..%d ranks", kMaxRanks);
  if (!counter || !peer_flags || !flags || !error)
    return set_error(CXS_ERR_INVALID, "null exchange argument");
  PeerFlags peers = {};
  for (int p = 0; p < ranks; ++p) {
    if (p != rank && !peer_flags[p]) return set_error(CXS_ERR_INVALID, "missing peer flags");
    peers.flags[p] = peer_flags[p];
  }
  exchange_barrier_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(
      counter, peers, flags, rank, ranks, spin_limit > 0 ? spin_limit : (1ll << 31), error);
  CXS_LAUNCH_CHECK("exchange_barrier_kernel");
  return CXS_OK;
}
