// Block-source preparation and the persistent IO + attention kernel.
//
// Reference behaviour: tma/transport.py:17-112 (_prepare_sources, execute)
// and the staged TMA kernel tma/pipeline.py:96-742 (IO CTAs :347-421,
// consumer CTAs :436-655, online-softmax block step :172-257). This is a new
// sm_100a design: one cooperative launch whose CTAs each run one IO warp and
// eight attention warps; see cxs_fetch_attend in include/cxlsparse.h.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "cxs_common.cuh"
#include "tile_attn.cuh"

using cxs::kTokenBytes;
using cxs::Softmax;
using cxs::bf16_round;
using cxs::unpack_bf16;
using cxs_host::set_error;

namespace {

constexpr int kAttnWarps = 8;
constexpr int kThreads = 32 * (1 + kAttnWarps);

struct AttendArgs {
  int Q, H, W, BS, P, window, window_len, gate;
  long long window_start, spin_limit;
  int consumers;  // attention warps that own rows: min(rows, grid * kAttnWarps)
  const __nv_bfloat16* query;
  __nv_bfloat16* kv;
  const int32_t* all_ids;
  const int32_t* all_counts;
  const int32_t* row_positions;
  const int32_t* starts;
  const int32_t* valid;
  const int32_t* ioids;
  const int32_t* missing;
  const int64_t* address;
  const int64_t* sources;
  const int32_t* kinds;
  int32_t* ready;
  int32_t* control;
  int32_t* error;
  const __nv_bfloat16* compressed;
  const __nv_bfloat16* gates;
  __nv_bfloat16* out;
};

// Warp gather of one BS-token block: token t comes from address[t] (HBM or
// host-mapped pool memory, 256 contiguous bytes) when t < count and the
// address is set, otherwise zeros. Loads are issued in independent batches of
// eight 16-byte vectors per lane so that their latencies overlap.
template <int BS>
__device__ __forceinline__ void gather_block(const int64_t* __restrict__ address, int count,
                                             uint4* __restrict__ dst, int lane) {
  constexpr int kPerLane = BS * 16 / 32;  // 16-byte vectors per lane
  constexpr int kBatch = kPerLane < 8 ? kPerLane : 8;
#pragma unroll
  for (int b0 = 0; b0 < kPerLane; b0 += kBatch) {
    uint4 value[kBatch];
#pragma unroll
    for (int k = 0; k < kBatch; ++k) {
      int i = lane + 32 * (b0 + k);
      int t = i >> 4, v = i & 15;
      long long src = address[t];
      value[k] = make_uint4(0, 0, 0, 0);
      if (t < count && src != 0) value[k] = __ldcv(reinterpret_cast<const uint4*>(src) + v);
    }
#pragma unroll
    for (int k = 0; k < kBatch; ++k) dst[lane + 32 * (b0 + k)] = value[k];
  }
}

// ---------------------------------------------------------------- prepare ---
// One warp per physical block: classify (0 resident, 1 full contiguous
// aligned external block, 2 mixed/tail external block), gather resident
// blocks into the staging buffer (tail zero-filled), initialise ready flags.
__global__ void prepare_kernel(int P, int BS, const int64_t* __restrict__ address,
                               const int32_t* __restrict__ valid,
                               const int32_t* __restrict__ flags, uint4* __restrict__ kv,
                               int64_t* __restrict__ sources, int32_t* __restrict__ kinds,
                               int32_t* __restrict__ ready, int32_t* control, int32_t* error) {
  int p = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  int lane = threadIdx.x % 32;
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    control[0] = 0;
    control[1] = 0;
    error[0] = 0;
  }
  if (p >= P) return;
  const int64_t* a = address + (long long)p * BS;
  long long first = a[0];
  int count = valid[p];
  bool missing = flags[p] != 0;
  bool contiguous = true;
  for (int t = lane; t < BS; t += 32) contiguous &= a[t] == first + (long long)t * kTokenBytes;
  contiguous = __all_sync(0xffffffffu, contiguous);
  bool full = missing && count == BS && first != 0 && (first % 16) == 0 && contiguous;
  uint4* dst = kv + (long long)p * BS * 16;
  if (lane == 0) {
    sources[p] = full ? first : (long long)(uintptr_t)dst;
    kinds[p] = missing ? (full ? 1 : 2) : 0;
    ready[p] = missing ? 0 : 1;
  }
  if (missing || count <= 0) return;
  // Resident block: every token comes from HBM (hot replica or current KV).
  switch (BS) {
    case 16: gather_block<16>(a, count, dst, lane); break;
    case 32: gather_block<32>(a, count, dst, lane); break;
    default: gather_block<64>(a, count, dst, lane); break;
  }
}

// ------------------------------------------------------ IO + attention ---
template <int BS>
__global__ void __launch_bounds__(kThreads, 1)
    fetch_attend_kernel(const __grid_constant__ CUtensorMap kv_map,
                        const __grid_constant__ CUtensorMap win_map, AttendArgs a) {
  constexpr int kTile = BS * 128;    // one K or V tile (BS rows x 128 bytes)
  constexpr int kBlockBytes = BS * kTokenBytes;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* io_buf = smem;                                   // kBlockBytes
  uint8_t* tiles = smem + ((kBlockBytes + 1023) & ~1023);   // kAttnWarps x (K, V)
  uint64_t* bars = reinterpret_cast<uint64_t*>(tiles + kAttnWarps * 2 * kTile);
  int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    for (int i = 0; i <= kAttnWarps; ++i) cxs::mbar_init(&bars[i], 1);
    cxs::fence_mbar_init();
  }
  __syncthreads();

  if (warp == 0) {
    // ------------------------------------------------------------ IO warp
    uint32_t phase = 0;
    int missing = a.missing[0];
    while (true) {
      int rank = 0;
      if (lane == 0) rank = atomicAdd(&a.control[0], 1);
      rank = __shfl_sync(0xffffffffu, rank, 0);
      if (rank >= missing) break;
      int block = a.ioids[rank];
      if (block < 0 || block >= a.P) {
        if (lane == 0) atomicOr(a.error, cxs::kErrBadBlock);
        continue;
      }
      int kind = a.kinds[block];
      uint8_t* dst = reinterpret_cast<uint8_t*>(a.kv) + (long long)block * kBlockBytes;
      if (kind == 1) {
        if (lane == 0) {
          const void* src = reinterpret_cast<const void*>(a.sources[block]);
          cxs::fence_proxy_async_shared();
          cxs::mbar_expect_tx(&bars[kAttnWarps], kBlockBytes);
          cxs::bulk_g2s(io_buf, src, kBlockBytes, &bars[kAttnWarps]);
          if (cxs::mbar_wait_bounded(&bars[kAttnWarps], phase, a.spin_limit, a.error)) {
            cxs::bulk_s2g_and_wait(dst, io_buf, kBlockBytes);
          } else {
            cxs::mbar_wait_bounded(&bars[kAttnWarps], phase, a.spin_limit, a.error);
          }
          cxs::fence_proxy_async_global();
        }
        phase ^= 1;
      } else {
        // Mixed-tier or tail block: 16-byte vector gathers, tail zero-filled.
        gather_block<BS>(a.address + (long long)block * BS, a.valid[block],
                         reinterpret_cast<uint4*>(dst), lane);
        __threadfence();
        cxs::fence_proxy_async_global();
        __syncwarp();
      }
      if (lane == 0) cxs::st_release(&a.ready[block], 1);
    }
    return;
  }

  // ------------------------------------------------------- attention warps
  int aw = blockIdx.x * kAttnWarps + (warp - 1);
  if (aw >= a.consumers) return;
  uint8_t* k_tile = tiles + (warp - 1) * 2 * kTile;
  uint8_t* v_tile = k_tile + kTile;
  uint32_t k_addr = cxs::smem_addr(k_tile), v_addr = cxs::smem_addr(v_tile);
  uint64_t* bar = &bars[warp - 1];
  uint32_t phase = 0;
  int rows = a.Q * a.H;
  int g = lane >> 2, c = lane & 3;
  if (lane == 0) {
    cxs::tma_prefetch_desc(&kv_map);
    if (a.window) cxs::tma_prefetch_desc(&win_map);
  }
  for (int row = aw; row < rows; row += a.consumers) {
    int h = row % a.H;
    int pos = a.row_positions[row];
    uint32_t qa[4][4];
    cxs::load_query(a.query + (long long)row * cxs::kGroups * cxs::kDim, lane, qa);
    Softmax<BS> sm;
    uint32_t win_out[8][2];
    bool have_window = a.window > 0 && pos >= 0;
    if (have_window) {
      sm.reset();
      long long lo = (long long)pos - a.window + 1;
      int tiles_n = (a.window + BS - 1) / BS;
      for (int j = 0; j < tiles_n; ++j) {
        long long t0 = lo + (long long)j * BS;
        if (t0 + BS - 1 < 0) continue;  // whole tile before position 0
        long long local0 = t0 - a.window_start;
        if (lane == 0) {
          cxs::fence_proxy_async_shared();
          cxs::mbar_expect_tx(bar, 2 * kTile);
          // 3-D map {channel, head, record}: x channel, y head, z record.
          cxs::tma_load_3d(k_addr, &win_map, 0, h, (int)local0, bar);
          cxs::tma_load_3d(v_addr, &win_map, 64, h, (int)local0, bar);
        }
        __syncwarp();
        if (!cxs::mbar_wait_bounded(bar, phase, a.spin_limit, a.error)) {
          cxs::mbar_wait_bounded(bar, phase, a.spin_limit, a.error);  // drain the copy
          return;
        }
        phase ^= 1;
        long long win_lo = lo, win_len = a.window_len, wstart = a.window_start;
        sm.step(qa, k_addr, v_addr, lane, [&](int t) {
          long long logical = t0 + t;
          long long local = logical - wstart;
          return logical >= 0 && logical >= win_lo && logical <= pos && local >= 0 &&
                 local < win_len;
        });
        __syncwarp();
      }
      sm.finish(win_out);
    }
    // Selected blocks in original order, each gated on ready[b].
    sm.reset();
    int count = pos >= 0 ? a.all_counts[row] : 0;
    const int32_t* ids = a.all_ids + (long long)row * a.W;
    for (int i = 0; i < count; ++i) {
      int block = ids[i];
      if (block < 0 || block >= a.P) {
        if (lane == 0) atomicOr(a.error, cxs::kErrBadBlock);
        continue;
      }
      bool ok = true;
      if (lane == 0) {
        ok = cxs::wait_ready_bounded(&a.ready[block], a.spin_limit, a.error);
        if (ok) {
          cxs::fence_proxy_async_global();
          cxs::fence_proxy_async_shared();
          cxs::mbar_expect_tx(bar, 2 * kTile);
          cxs::tma_load_2d(k_tile, &kv_map, 0, block * BS, bar);
          cxs::tma_load_2d(v_tile, &kv_map, 64, block * BS, bar);
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) return;  // ready timeout (or an earlier failure): the launch is invalid
      if (!cxs::mbar_wait_bounded(bar, phase, a.spin_limit, a.error)) {
        cxs::mbar_wait_bounded(bar, phase, a.spin_limit, a.error);  // drain the copy
        return;
      }
      phase ^= 1;
      int start = a.starts[block];
      sm.step(qa, k_addr, v_addr, lane, [&](int t) { return start + t <= pos; });
      __syncwarp();
    }
    uint32_t sel_out[8][2];
    sm.finish(sel_out);
    // Epilogue: selected output, or the gate mix of the three branches in the
    // reference's bf16 rounding sequence (models/nsa/model.py:470-473).
    __nv_bfloat16* orow = a.out + (long long)row * cxs::kGroups * cxs::kDim;
    if (!a.gate) {
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        *reinterpret_cast<uint32_t*>(orow + g * 64 + n * 8 + 2 * c) = sel_out[n][0];
        *reinterpret_cast<uint32_t*>(orow + (g + 8) * 64 + n * 8 + 2 * c) = sel_out[n][1];
      }
    } else {
      const __nv_bfloat16* crow = a.compressed + (long long)row * cxs::kGroups * cxs::kDim;
      const __nv_bfloat16* grow = a.gates + (long long)row * cxs::kGroups * 3;
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        int head = g + r * 8;
        float g0 = __bfloat162float(grow[head * 3 + 0]);
        float g1 = __bfloat162float(grow[head * 3 + 1]);
        float g2 = __bfloat162float(grow[head * 3 + 2]);
#pragma unroll
        for (int n = 0; n < 8; ++n) {
          int dim = n * 8 + 2 * c;
          float2 sel = unpack_bf16(sel_out[n][r]);
          float2 win = have_window ? unpack_bf16(win_out[n][r]) : make_float2(0.f, 0.f);
          float2 cmp = unpack_bf16(*reinterpret_cast<const uint32_t*>(crow + head * 64 + dim));
          float x0 = bf16_round(sel.x * g1), x1 = bf16_round(sel.y * g1);
          x0 = bf16_round(x0 + cmp.x * g0);
          x1 = bf16_round(x1 + cmp.y * g0);
          x0 = x0 + win.x * g2;
          x1 = x1 + win.y * g2;
          *reinterpret_cast<uint32_t*>(orow + head * 64 + dim) = cxs::pack_bf16(x0, x1);
        }
      }
    }
  }
}

// ------------------------------------------------------- host: tensor maps ---
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    else
      cudaGetLastError();
  }
  return fn;
}

int encode_kv_map(CUtensorMap* map, void* kv, long long rows, int bs) {
  auto fn = encode_fn();
  if (!fn) return set_error(CXS_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {128, (cuuint64_t)rows};
  cuuint64_t strides[1] = {256};
  cuuint32_t box[2] = {64, (cuuint32_t)bs};
  cuuint32_t elem[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, kv, dims, strides, box, elem,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(CXS_ERR_CUDA, "kv tensor map encode failed (%d)", r);
  return CXS_OK;
}

int encode_window_map(CUtensorMap* map, const void* records, int heads, int records_n, int bs) {
  auto fn = encode_fn();
  if (!fn) return set_error(CXS_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[3] = {128, (cuuint64_t)heads, (cuuint64_t)records_n};
  cuuint64_t strides[2] = {256, (cuuint64_t)heads * 256};
  cuuint32_t box[3] = {64, 1, (cuuint32_t)bs};
  cuuint32_t elem[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(records), dims,
                  strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(CXS_ERR_CUDA, "window tensor map encode failed (%d)", r);
  return CXS_OK;
}

template <int BS>
size_t smem_bytes() {
  size_t io = ((size_t)BS * kTokenBytes + 1023) & ~(size_t)1023;
  return 1024 + io + (size_t)kAttnWarps * 2 * BS * 128 + (kAttnWarps + 1) * 8;
}

struct GridInfo {
  int grid = 0;
  int sms = 0;
};

template <int BS>
int grid_size(int* grid) {
  static int cached[64] = {0};
  int device = 0;
  CXS_CUDA(cudaGetDevice(&device));
  if (device < 64 && cached[device]) {
    *grid = cached[device];
    return CXS_OK;
  }
  size_t smem = smem_bytes<BS>();
  CXS_CUDA(cudaFuncSetAttribute(fetch_attend_kernel<BS>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  int per_sm = 0, sms = 0;
  CXS_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fetch_attend_kernel<BS>,
                                                         kThreads, smem));
  CXS_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
  if (per_sm < 1) return set_error(CXS_ERR_UNSUPPORTED, "fetch_attend kernel cannot be resident");
  *grid = per_sm * sms;
  if (device < 64) cached[device] = *grid;
  return CXS_OK;
}

template <int BS>
int launch(const cxs_attend_geometry& g, const cxs_attend_buffers& b, cudaStream_t stream) {
  int grid = 0;
  int status = grid_size<BS>(&grid);
  if (status != CXS_OK) return status;
  CUtensorMap kv_map, win_map;
  status = encode_kv_map(&kv_map, b.kv, (long long)g.physical * BS, BS);
  if (status != CXS_OK) return status;
  if (g.window > 0) {
    status = encode_window_map(&win_map, b.window_kv, g.heads, g.window_len, BS);
    if (status != CXS_OK) return status;
  } else {
    win_map = kv_map;
  }
  AttendArgs a;
  a.Q = g.queries;
  a.H = g.heads;
  a.W = g.width;
  a.BS = BS;
  a.P = g.physical;
  a.window = g.window;
  a.window_len = g.window_len;
  a.gate = g.gate;
  a.window_start = g.window_start;
  a.spin_limit = g.spin_limit > 0 ? g.spin_limit : (1ll << 31);
  int rows = g.queries * g.heads;
  a.consumers = rows < grid * kAttnWarps ? rows : grid * kAttnWarps;
  a.query = (const __nv_bfloat16*)b.query;
  a.kv = (__nv_bfloat16*)b.kv;
  a.all_ids = b.all_ids;
  a.all_counts = b.all_counts;
  a.row_positions = b.row_positions;
  a.starts = b.starts;
  a.valid = b.valid;
  a.ioids = b.ioids;
  a.missing = b.missing;
  a.address = b.address;
  a.sources = b.sources;
  a.kinds = b.kinds;
  a.ready = b.ready;
  a.control = b.control;
  a.error = b.error;
  a.compressed = (const __nv_bfloat16*)b.compressed;
  a.gates = (const __nv_bfloat16*)b.gates;
  a.out = (__nv_bfloat16*)b.out;

  int prep_grid = (g.physical + 7) / 8;
  prepare_kernel<<<prep_grid > 0 ? prep_grid : 1, 256, 0, stream>>>(
      g.physical, BS, b.address, b.valid, b.flags, (uint4*)b.kv, b.sources, b.kinds, b.ready,
      b.control, b.error);
  CXS_LAUNCH_CHECK("prepare_kernel");

  cudaLaunchConfig_t config = {};
  config.gridDim = dim3(grid);
  config.blockDim = dim3(kThreads);
  config.dynamicSmemBytes = smem_bytes<BS>();
  config.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  config.attrs = attr;
  config.numAttrs = 1;
  CXS_CUDA(cudaLaunchKernelEx(&config, fetch_attend_kernel<BS>, kv_map, win_map, a));
  cxs_host::count_launch();
  return CXS_OK;
}

}  // namespace

extern "C" int cxs_fetch_attend(const cxs_attend_geometry* geometry,
                                const cxs_attend_buffers* buffers, void* stream) {
  if (!geometry || !buffers) return set_error(CXS_ERR_INVALID, "null attend argument");
  const cxs_attend_geometry& g = *geometry;
  const cxs_attend_buffers& b = *buffers;
  if (g.queries < 1 || g.heads < 1 || g.width < 1 || g.physical < 1)
    return set_error(CXS_ERR_INVALID, "nonempty attend geometry required");
  if (g.window < 0 || (g.window > 0 && (!b.window_kv || g.window_len < 1)))
    return set_error(CXS_ERR_INVALID, "window branch needs a window buffer");
  if (g.gate && (!b.compressed || !b.gates))
    return set_error(CXS_ERR_INVALID, "gate mix needs compressed output and gates");
  if (((uintptr_t)b.kv & 15) || ((uintptr_t)b.query & 15) || ((uintptr_t)b.out & 15))
    return set_error(CXS_ERR_INVALID, "kv/query/out must be 16-byte aligned");
  if (g.window > 0 && ((uintptr_t)b.window_kv & 15))
    return set_error(CXS_ERR_INVALID, "window buffer must be 16-byte aligned");
  switch (g.block_size) {
    case 16: return launch<16>(g, b, (cudaStream_t)stream);
    case 32: return launch<32>(g, b, (cudaStream_t)stream);
    case 64: return launch<64>(g, b, (cudaStream_t)stream);
    default: return set_error(CXS_ERR_INVALID, "block_size must be 16, 32 or 64");
  }
}

extern "C" int cxs_attend_capacity(int32_t block_size, int32_t* attention_warps) {
  if (!attention_warps) return set_error(CXS_ERR_INVALID, "null output");
  int grid = 0, status;
  switch (block_size) {
    case 16: status = grid_size<16>(&grid); break;
    case 32: status = grid_size<32>(&grid); break;
    case 64: status = grid_size<64>(&grid); break;
    default: return set_error(CXS_ERR_INVALID, "block_size must be 16, 32 or 64");
  }
  if (status != CXS_OK) return status;
  *attention_warps = grid * kAttnWarps;
  return CXS_OK;
}

// ------------------------------------------------ allocation-free variant ---
// Scratch for cxs_fetch_attend_noalloc: per-block bulk sources, source kinds
// and ready flags plus the IO work cursor, for at most
// CXS_NOALLOC_MAX_PHYSICAL blocks. Every GPU that loads this library holds it
// until the process exits; all calls on a device share it.
namespace {

constexpr size_t kScratchSources = 0;
constexpr size_t kScratchKinds = kScratchSources + 8ull * CXS_NOALLOC_MAX_PHYSICAL;
constexpr size_t kScratchReady = kScratchKinds + 4ull * CXS_NOALLOC_MAX_PHYSICAL;
constexpr size_t kScratchControl = kScratchReady + 4ull * CXS_NOALLOC_MAX_PHYSICAL;
constexpr size_t kScratchBytes = kScratchControl + 256;

static __device__ __align__(256) unsigned char g_attend_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mutex;
unsigned char* g_scratch_address[kMaxDevices] = {nullptr};

// Device address of the scratch array on the current device, looked up once
// per device (the host-side symbol itself is not a device address).
int scratch_address(unsigned char** out) {
  int device = 0;
  CXS_CUDA(cudaGetDevice(&device));
  if (device < 0 || device >= kMaxDevices)
    return set_error(CXS_ERR_UNSUPPORTED, "device index %d beyond %d", device, kMaxDevices);
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (!g_scratch_address[device]) {
    void* address = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&address, g_attend_scratch);
    if (e != cudaSuccess) {
      cudaGetLastError();
      return set_error(CXS_ERR_CUDA, "cudaGetSymbolAddress(scratch): %s", cudaGetErrorString(e));
    }
    g_scratch_address[device] = static_cast<unsigned char*>(address);
  }
  *out = g_scratch_address[device];
  return CXS_OK;
}

}  // namespace

extern "C" int cxs_fetch_attend_noalloc(const cxs_attend_geometry* geometry,
                                        const cxs_attend_buffers* buffers, void* stream) {
  if (!geometry || !buffers) return set_error(CXS_ERR_INVALID, "null attend argument");
  if (geometry->physical > CXS_NOALLOC_MAX_PHYSICAL)
    return set_error(CXS_ERR_CAPACITY,
                     "cxs_fetch_attend_noalloc handles at most %d physical blocks (got %d); "
                     "use cxs_fetch_attend with caller-provided scratch",
                     CXS_NOALLOC_MAX_PHYSICAL, geometry->physical);
  if (!buffers->error) return set_error(CXS_ERR_INVALID, "error word output required");
  unsigned char* scratch = nullptr;
  int status = scratch_address(&scratch);
  if (status != CXS_OK) return status;
  // Same launches as cxs_fetch_attend; only the scratch arrays change. The
  // prepare kernel rewrites sources, kinds and ready for every block and
  // zeroes the IO cursor and the error word before the IO/attention kernel.
  cxs_attend_buffers b = *buffers;
  b.sources = reinterpret_cast<int64_t*>(scratch + kScratchSources);
  b.kinds = reinterpret_cast<int32_t*>(scratch + kScratchKinds);
  b.ready = reinterpret_cast<int32_t*>(scratch + kScratchReady);
  b.control = reinterpret_cast<int32_t*>(scratch + kScratchControl);
  return cxs_fetch_attend(geometry, &b, stream);
}
