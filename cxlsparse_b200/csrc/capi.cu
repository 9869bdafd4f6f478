// Error reporting, backing-pool allocation/registration and the pool write path.
#include <errno.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/syscall.h>
#include <unistd.h>

#include "cxs_common.cuh"

namespace cxs_host {

static thread_local char g_error[512] = "";

int set_error(int code, const char* fmt, ...) {
  va_list args;
  va_start(args, fmt);
  vsnprintf(g_error, sizeof(g_error), fmt, args);
  va_end(args);
  return code;
}

int check_cuda(cudaError_t err, const char* what) {
  return set_error(CXS_ERR_CUDA, "%s: %s", what, cudaGetErrorString(err));
}

static unsigned long long g_launches = 0;

void count_launch() { __atomic_add_fetch(&g_launches, 1ull, __ATOMIC_RELAXED); }

}  // namespace cxs_host

using cxs_host::set_error;

extern "C" int cxs_abi_version(void) { return CXS_ABI_VERSION; }

extern "C" const char* cxs_last_error(void) { return cxs_host::g_error; }

extern "C" int64_t cxs_launch_count(void) {
  return (int64_t)__atomic_load_n(&cxs_host::g_launches, __ATOMIC_RELAXED);
}

// ------------------------------------------------------------------- pool ---

extern "C" int cxs_device_numa_node(int device) {
  char bus[32];
  if (cudaDeviceGetPCIBusId(bus, sizeof(bus), device) != cudaSuccess) {
    cudaGetLastError();
    return -1;
  }
  for (char* c = bus; *c; ++c) *c = (*c >= 'A' && *c <= 'F') ? *c - 'A' + 'a' : *c;
  char path[128];
  snprintf(path, sizeof(path), "/sys/bus/pci/devices/%s/numa_node", bus);
  FILE* f = fopen(path, "r");
  if (!f) return -1;
  int node = -1;
  if (fscanf(f, "%d", &node) != 1) node = -1;
  fclose(f);
  return node;
}

static int register_checked(void* base, size_t bytes) {
  cudaError_t e = cudaHostRegister(base, bytes, cudaHostRegisterMapped | cudaHostRegisterPortable);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_error(CXS_ERR_REGISTRATION, "cudaHostRegister(%p, %zu): %s", base, bytes,
                     cudaGetErrorString(e));
  }
  void* device = nullptr;
  e = cudaHostGetDevicePointer(&device, base, 0);
  if (e != cudaSuccess || device != base) {
    cudaGetLastError();
    cudaHostUnregister(base);
    return set_error(CXS_ERR_REGISTRATION,
                     "pool mapping needs identical host and device addresses (%p vs %p)", base,
                     device);
  }
  return CXS_OK;
}

extern "C" int cxs_pool_register(void* host_base, size_t bytes) {
  if (!host_base || !bytes) return set_error(CXS_ERR_INVALID, "empty pool registration");
  return register_checked(host_base, bytes);
}

extern "C" int cxs_pool_unregister(void* host_base) {
  cudaError_t e = cudaHostUnregister(host_base);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_error(CXS_ERR_REGISTRATION, "cudaHostUnregister(%p): %s", host_base,
                     cudaGetErrorString(e));
  }
  return CXS_OK;
}

extern "C" int cxs_pool_create(size_t bytes, int device, int numa_node, void** host_base,
                               int* bound_node) {
  if (!bytes || !host_base) return set_error(CXS_ERR_INVALID, "empty pool allocation");
  size_t page = (size_t)sysconf(_SC_PAGESIZE);
  size_t length = (bytes + page - 1) / page * page;
  void* base = mmap(nullptr, length, PROT_READ | PROT_WRITE, MAP_PRIVATE | MAP_ANONYMOUS, -1, 0);
  if (base == MAP_FAILED)
    return set_error(CXS_ERR_REGISTRATION, "mmap(%zu): %s", length, strerror(errno));
  int node = numa_node >= 0 ? numa_node : cxs_device_numa_node(device);
  int bound = -1;
  if (node >= 0 && node < 64) {
    // MPOL_BIND = 2; bind before first touch so pages land on the GPU's node.
    unsigned long mask = 1ul << node;
    long rc = syscall(SYS_mbind, base, length, 2, &mask, 64, 0);
    if (rc == 0) bound = node;
  }
  memset(base, 0, length);  // first touch
  int status = register_checked(base, length);
  if (status != CXS_OK) {
    munmap(base, length);
    return status;
  }
  *host_base = base;
  if (bound_node) *bound_node = bound;
  return CXS_OK;
}

extern "C" int cxs_pool_destroy(void* host_base, size_t bytes) {
  if (!host_base) return CXS_OK;
  int status = cxs_pool_unregister(host_base);
  size_t page = (size_t)sysconf(_SC_PAGESIZE);
  size_t length = (bytes + page - 1) / page * page;
  if (munmap(host_base, length) != 0 && status == CXS_OK)
    status = set_error(CXS_ERR_REGISTRATION, "munmap: %s", strerror(errno));
  return status;
}

// One warp per token record: 16 lanes x 16 bytes = 256 bytes; two tokens per warp.
__global__ void pool_write_kernel(const uint4* __restrict__ records,
                                  const int64_t* __restrict__ slots, int64_t count,
                                  const int64_t* __restrict__ bases, int regions, int page_size) {
  int64_t token = (int64_t)blockIdx.x * (blockDim.x / 16) + threadIdx.x / 16;
  int lane = threadIdx.x % 16;
  if (token >= count) return;
  int64_t slot = slots[token];
  int64_t page = slot / page_size;
  int region = (int)(page % regions);
  int64_t local = (page / regions) * page_size + slot % page_size;
  uint4* dst = reinterpret_cast<uint4*>(bases[region] + local * cxs::kTokenBytes);
  dst[lane] = records[token * 16 + lane];
}

extern "C" int cxs_pool_write(const void* records, const int64_t* slots, int64_t count,
                              const int64_t* region_bases, int regions, int page_size,
                              void* stream) {
  if (count < 0 || regions < 1 || page_size < 1)
    return set_error(CXS_ERR_INVALID, "invalid pool write geometry");
  if (!count) return CXS_OK;
  if (((uintptr_t)records) & 15) return set_error(CXS_ERR_INVALID, "records must be 16B aligned");
  int threads = 256;
  int64_t grid = (count + threads / 16 - 1) / (threads / 16);
  pool_write_kernel<<<(unsigned)grid, threads, 0, (cudaStream_t)stream>>>(
      (const uint4*)records, slots, count, region_bases, regions, page_size);
  CXS_LAUNCH_CHECK("pool_write_kernel");
  return CXS_OK;
}

// Mean of BS consecutive tokens per (summary, head, channel), fp32 accumulate.
// 128 channels x 8 token groups per CTA; partial sums reduced in shared memory.
// Grid (summary, head, run): run z reads tokens + z * token_stride records and
// writes out + z * summary_stride records.
__global__ void block_summaries_kernel(const __nv_bfloat16* __restrict__ tokens, int heads,
                                       int bs, __nv_bfloat16* __restrict__ out,
                                       int64_t token_stride, int64_t summary_stride) {
  __shared__ float partial[8][128];
  int summary = blockIdx.x, head = blockIdx.y;
  tokens += (int64_t)blockIdx.z * token_stride * heads * 128;
  out += (int64_t)blockIdx.z * summary_stride * heads * 128;
  int c = threadIdx.x & 127, group = threadIdx.x >> 7;
  const __nv_bfloat16* base = tokens + ((int64_t)summary * bs * heads + head) * 128 + c;
  float acc = 0.f;
  for (int t = group; t < bs; t += 8) acc += __bfloat162float(base[(int64_t)t * heads * 128]);
  partial[group][c] = acc;
  __syncthreads();
  if (group == 0) {
    float sum = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) sum += partial[k][c];
    out[((int64_t)summary * heads + head) * 128 + c] = __float2bfloat16_rn(sum / (float)bs);
  }
}

extern "C" int cxs_block_summaries_segments(const void* tokens, int64_t count, int32_t heads,
                                            int32_t block_size, void* summaries,
                                            int32_t segments, int64_t token_stride,
                                            int64_t summary_stride, void* stream) {
  if (count < 0 || heads < 1 || block_size < 1 || segments < 1 || segments > 65535 ||
      token_stride < 0 || summary_stride < 0)
    return set_error(CXS_ERR_INVALID, "invalid summary geometry");
  int64_t n = count / block_size;
  if (!n) return CXS_OK;
  if (segments > 1 && (token_stride < count || summary_stride < n))
    return set_error(CXS_ERR_INVALID, "summary runs overlap");
  dim3 grid((unsigned)n, heads, segments);
  block_summaries_kernel<<<grid, 1024, 0, (cudaStream_t)stream>>>(
      (const __nv_bfloat16*)tokens, heads, block_size, (__nv_bfloat16*)summaries, token_stride,
      summary_stride);
  CXS_LAUNCH_CHECK("block_summaries_kernel");
  return CXS_OK;
}

extern "C" int cxs_block_summaries(const void* tokens, int64_t count, int32_t heads,
                                   int32_t block_size, void* summaries, void* stream) {
  return cxs_block_summaries_segments(tokens, count, heads, block_size, summaries, 1, 0, 0,
                                      stream);
}
