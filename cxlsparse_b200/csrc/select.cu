// Compressed-token attention + top-n block selection.
//
// Reference semantics: models/nsa/ops.py:73-123 (torch path) and the FLA
// kernels third_party/nsa_runtime/kernels.py:13-230 used on the GPU:
//  - attention of the 16-head group over complete summaries
//    c < (pos + 1) // BS, output normalised per head;
//  - block score = sum over the 16 heads of the normalised probabilities;
//  - selection: the current block pos // BS first, then blocks before it by
//    score descending with ties to the lower block id; width =
//    min(count, ceil(total / BS)); remaining entries -1.
//
// One CTA of 4 warps per (query row, KV head); the warps split the 64-summary
// tiles (staged by 3-D tensor TMA). Pass 1: per-warp online softmax + PV,
// merged across warps in shared memory (compressed branch output). Pass 2:
// scores recomputed with the merged per-head max / normaliser, reduced over
// heads; warp 0 selects the top-n.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "cxs_common.cuh"
#include "tile_attn.cuh"

using cxs_host::set_error;

namespace {

constexpr int kWarps = 4;
constexpr int kTileKeys = 64;
constexpr int kTileBytes = kTileKeys * 128;

// Error sink for the kernel's bounded copy waits (its copies read device
// memory only, so a timeout indicates a broken launch, not a slow link).
__device__ int g_select_error;

struct SelectArgs {
  int Q, H, C, BS, count, width, score_len;
  long long total;
  const __nv_bfloat16* query;
  const int32_t* positions;
  __nv_bfloat16* out;
  int32_t* blocks;
  float* scores;
  int* error;
};

__global__ void __launch_bounds__(kWarps * 32)
    compressed_select_kernel(const __grid_constant__ CUtensorMap map, SelectArgs a) {
  // One CTA per (query row, KV head); warp w owns summary tiles w, w + 4, ...
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  int score_len = a.score_len;
  uint8_t* k_tile = smem + warp * 2 * kTileBytes;
  uint8_t* v_tile = k_tile + kTileBytes;
  float* scores = reinterpret_cast<float*>(smem + kWarps * 2 * kTileBytes);
  float* merge = scores + score_len;                    // [kWarps][16 m | 16 l | 16x64 o]
  uint64_t* bars = reinterpret_cast<uint64_t*>(merge + kWarps * (32 + 16 * 64));
  uint64_t* bar = &bars[warp];
  if (lane == 0) {
    cxs::mbar_init(bar, 1);
    cxs::fence_mbar_init();
  }
  __syncwarp();
  uint32_t k_addr = cxs::smem_addr(k_tile), v_addr = cxs::smem_addr(v_tile);
  uint32_t phase = 0;
  int row = blockIdx.x;
  int q = row / a.H, h = row % a.H;
  int pos = a.positions[q];
  int g = lane >> 2, c = lane & 3;
  int nc = pos >= 0 ? min((pos + 1) / a.BS, a.C) : 0;  // complete summaries
  int tiles = (nc + kTileKeys - 1) / kTileKeys;
  long long spin = 1ll << 31;
  for (int i = threadIdx.x; i < score_len; i += blockDim.x) scores[i] = 0.f;
  uint32_t qa[4][4];
  cxs::load_query(a.query + (long long)row * cxs::kGroups * cxs::kDim, lane, qa);
  // Pass 1: each warp runs online softmax + PV over its tiles.
  cxs::Softmax<kTileKeys> sm;
  sm.reset();
  bool ok = true;
  for (int t = warp; t < tiles && ok; t += kWarps) {
    if (lane == 0) {
      cxs::fence_proxy_async_shared();
      cxs::mbar_expect_tx(bar, 2 * kTileBytes);
      cxs::tma_load_3d(k_addr, &map, 0, h, t * kTileKeys, bar);
      cxs::tma_load_3d(v_addr, &map, 64, h, t * kTileKeys, bar);
    }
    __syncwarp();
    if (!cxs::mbar_wait_bounded(bar, phase, spin, a.error)) {
      cxs::mbar_wait_bounded(bar, phase, spin, a.error);
      ok = false;
      break;
    }
    phase ^= 1;
    int base = t * kTileKeys;
    sm.step(qa, k_addr, v_addr, lane, [&](int k) { return base + k < nc; });
    __syncwarp();
  }
  // Merge the warps' (max, sum, accumulator) per head through shared memory.
  float* mine = merge + warp * (32 + 16 * 64);
  if (c == 0) {
    mine[g] = sm.m[0];
    mine[g + 8] = sm.m[1];
    mine[16 + g] = sm.l[0];
    mine[16 + g + 8] = sm.l[1];
  }
#pragma unroll
  for (int n = 0; n < 8; ++n) {
    int dim = n * 8 + 2 * c;
    mine[32 + g * 64 + dim] = sm.o[n][0];
    mine[32 + g * 64 + dim + 1] = sm.o[n][1];
    mine[32 + (g + 8) * 64 + dim] = sm.o[n][2];
    mine[32 + (g + 8) * 64 + dim + 1] = sm.o[n][3];
  }
  __syncthreads();
  // Global per-head max / normaliser (every warp needs them for pass 2).
  float gm[2], gl[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    int head = g + r * 8;
    float m = -INFINITY;
    for (int w = 0; w < kWarps; ++w) m = fmaxf(m, merge[w * (32 + 16 * 64) + head]);
    float l = 0.f;
    for (int w = 0; w < kWarps; ++w) {
      float mw = merge[w * (32 + 16 * 64) + head];
      if (mw != -INFINITY) l += merge[w * (32 + 16 * 64) + 16 + head] * expf(mw - m);
    }
    gm[r] = m;
    gl[r] = l;
  }
  // Output: 16 heads x 64 dims spread over the CTA's 128 threads.
  __nv_bfloat16* orow = a.out + (long long)row * cxs::kGroups * cxs::kDim;
  for (int e = threadIdx.x; e < 16 * 64; e += blockDim.x) {
    int head = e / 64;
    float m = -INFINITY, l = 0.f, acc = 0.f;
    for (int w = 0; w < kWarps; ++w) m = fmaxf(m, merge[w * (32 + 16 * 64) + head]);
    for (int w = 0; w < kWarps; ++w) {
      const float* part = merge + w * (32 + 16 * 64);
      if (part[head] == -INFINITY) continue;
      float f = expf(part[head] - m);
      l += part[16 + head] * f;
      acc += part[32 + e] * f;
    }
    orow[e] = __float2bfloat16_rn(l > 0.f ? acc / l : 0.f);
  }
  // Pass 2: block scores = sum over heads of exp(s - M) / L with the merged M, L.
  float inv[2] = {gl[0] > 0.f ? 1.f / gl[0] : 0.f, gl[1] > 0.f ? 1.f / gl[1] : 0.f};
  for (int t = warp; t < tiles && ok; t += kWarps) {
    if (lane == 0) {
      cxs::fence_proxy_async_shared();
      cxs::mbar_expect_tx(bar, kTileBytes);
      cxs::tma_load_3d(k_addr, &map, 0, h, t * kTileKeys, bar);
    }
    __syncwarp();
    if (!cxs::mbar_wait_bounded(bar, phase, spin, a.error)) {
      cxs::mbar_wait_bounded(bar, phase, spin, a.error);
      ok = false;
      break;
    }
    phase ^= 1;
    float sc[kTileKeys / 8][4];
    cxs::score_tile<kTileKeys>(qa, k_addr, lane, sc);
#pragma unroll
    for (int nt = 0; nt < kTileKeys / 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        int key = t * kTileKeys + nt * 8 + 2 * c + e;
        float p = 0.f;
        if (key < nc)
          p = expf(sc[nt][e] - gm[0]) * inv[0] + expf(sc[nt][e + 2] - gm[1]) * inv[1];
        p += __shfl_xor_sync(0xffffffffu, p, 4);
        p += __shfl_xor_sync(0xffffffffu, p, 8);
        p += __shfl_xor_sync(0xffffffffu, p, 16);
        if (g == 0 && key < a.C) scores[key] = p;
      }
    }
    __syncwarp();
  }
  __syncthreads();
  if (a.scores) {
    float* srow = a.scores + (long long)row * a.C;
    for (int i = threadIdx.x; i < a.C; i += blockDim.x) srow[i] = scores[i];
  }
  __syncthreads();
  if (warp != 0) return;
  // Top-n: current block first, then (score desc, block asc) among earlier blocks.
  int32_t* brow = a.blocks + (long long)row * a.width;
  int current = pos >= 0 ? pos / a.BS : -1;
  int limit = min(current, score_len);  // candidates: blocks before the current one
  if (lane == 0) brow[0] = current >= 0 ? current : -1;
  for (int k = 1; k < a.width; ++k) {
    float best = -1.f;
    int best_idx = 0x7fffffff;
    for (int i = lane; i < limit; i += 32) {
      float v = scores[i];
      if (v > best || (v == best && i < best_idx)) {
        best = v;
        best_idx = i;
      }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      float ov = __shfl_xor_sync(0xffffffffu, best, o);
      int oi = __shfl_xor_sync(0xffffffffu, best_idx, o);
      if (ov > best || (ov == best && oi < best_idx)) {
        best = ov;
        best_idx = oi;
      }
    }
    if (lane == 0) {
      brow[k] = best_idx < limit ? best_idx : -1;
      if (best_idx < limit) scores[best_idx] = -2.f;  // taken
    }
    __syncwarp();
  }
}

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

}  // namespace

extern "C" int cxs_compressed_select(const void* query, const void* compressed, int32_t summaries,
                                     const int32_t* positions, int32_t queries, int32_t heads,
                                     int32_t block_size, int32_t count, int64_t total, void* out,
                                     int32_t* blocks, float* scores, void* stream) {
  if (queries < 1 || heads < 1 || block_size < 1 || count < 1 || total < 1 || summaries < 0)
    return set_error(CXS_ERR_INVALID, "invalid compressed-select geometry");
  if (!query || !out || !blocks || !positions || (summaries > 0 && !compressed))
    return set_error(CXS_ERR_INVALID, "null compressed-select argument");
  if (((uintptr_t)compressed & 15) || ((uintptr_t)query & 15) || ((uintptr_t)out & 3))
    return set_error(CXS_ERR_INVALID, "query/compressed must be 16-byte aligned");
  long long blocks_total = (total + block_size - 1) / block_size;
  int width = (int)(count < blocks_total ? count : blocks_total);
  if (summaries > (1 << 20)) return set_error(CXS_ERR_CAPACITY, "too many summaries");
  auto fn = encode_fn();
  if (!fn) return set_error(CXS_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled unavailable");
  CUtensorMap map;
  // With no summary yet no tile is ever loaded; the map only needs a valid
  // base, so it points at the query buffer (at least heads * 256 bytes).
  const void* base = summaries ? compressed : query;
  int records = summaries ? summaries : 1;
  cuuint64_t dims[3] = {128, (cuuint64_t)heads, (cuuint64_t)records};
  cuuint64_t strides[2] = {256, (cuuint64_t)heads * 256};
  cuuint32_t box[3] = {64, 1, (cuuint32_t)kTileKeys};
  cuuint32_t elem[3] = {1, 1, 1};
  CUresult r = fn(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides,
                  box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(CXS_ERR_CUDA, "summary tensor map encode failed (%d)", r);
  SelectArgs a;
  a.Q = queries;
  a.H = heads;
  a.C = summaries;
  a.BS = block_size;
  a.count = count;
  a.width = width;
  a.total = total;
  a.query = (const __nv_bfloat16*)query;
  a.positions = positions;
  a.out = (__nv_bfloat16*)out;
  a.blocks = blocks;
  a.scores = scores;
  int* error_word = nullptr;
  CXS_CUDA(cudaGetSymbolAddress((void**)&error_word, g_select_error));
  a.error = error_word;
  long long longest = summaries > blocks_total ? summaries : blocks_total;
  if (longest > (1 << 20)) return set_error(CXS_ERR_CAPACITY, "too many blocks");
  int score_len = (int)((longest + 3) & ~3ll);
  a.score_len = score_len;
  size_t smem = 1024 + (size_t)kWarps * 2 * kTileBytes + (size_t)score_len * 4 +
                (size_t)kWarps * (32 + 16 * 64) * 4 + kWarps * 8;
  if (smem > 227 * 1024) return set_error(CXS_ERR_CAPACITY, "too many summaries for one warp");
  CXS_CUDA(cudaFuncSetAttribute(compressed_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)smem));
  int rows = queries * heads;
  compressed_select_kernel<<<rows, kWarps * 32, smem, (cudaStream_t)stream>>>(
      map, a);
  CXS_LAUNCH_CHECK("compressed_select_kernel");
  return CXS_OK;
}
