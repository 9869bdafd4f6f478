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
// One kernel, compressed_select_tc_kernel (tcgen05 / TMEM, 8 query rows per
// CTA, 16 warps), serves every geometry: the per-row key and block scores
// live in shared memory up to 2048 columns, and in a per-device global
// scratch beyond that (the BASELINE MLP compression at H = 128K has ~8K
// keys).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "cxs_common.cuh"
#include "tile_tc.cuh"

using cxs_host::set_error;

namespace {

constexpr int kTileKeys = 64;

// Error sink for the kernels' bounded copy waits (their copies read device
// memory only, so a timeout indicates a broken launch, not a slow link).
__device__ int g_select_error;

constexpr int kMaxDevices = 64;
constexpr int kMaxSmem = 227 * 1024;
bool g_select_ready[kMaxDevices] = {false};
int* g_select_error_address[kMaxDevices] = {nullptr};

// Per-device global scratch for the score rows of long key lists, grown on
// demand. Growing allocates, which stream capture forbids: a first call of
// at least the same size must come before any capture.
float* g_score_scratch[kMaxDevices] = {nullptr};
size_t g_score_scratch_bytes[kMaxDevices] = {0};
std::mutex g_score_scratch_mutex;

int score_scratch(int device, size_t bytes, cudaStream_t stream, float** out) {
  std::lock_guard<std::mutex> lock(g_score_scratch_mutex);
  if (g_score_scratch_bytes[device] < bytes) {
    cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
    CXS_CUDA(cudaStreamIsCapturing(stream, &capture));
    if (capture != cudaStreamCaptureStatusNone)
      return set_error(CXS_ERR_CAPACITY,
                       "compressed select needs %zu bytes of score scratch on device %d; make "
                       "one call of this size before capturing a graph", bytes, device);
    if (g_score_scratch[device]) {
      CXS_CUDA(cudaDeviceSynchronize());  // a launch may still use the old scratch
      CXS_CUDA(cudaFree(g_score_scratch[device]));
      g_score_scratch[device] = nullptr;
      g_score_scratch_bytes[device] = 0;
    }
    CXS_CUDA(cudaMalloc((void**)&g_score_scratch[device], bytes));
    g_score_scratch_bytes[device] = bytes;
  }
  *out = g_score_scratch[device];
  return CXS_OK;
}

struct SelectArgs {
  int Q, H, C, BS, count, width, score_len;
  int seg_block, seg_blocks;  // candidate segments in blocks (seg_blocks 0: one suffix)
  int seg_key, seg_keys;      // the same in compressed-key slots
  int cmp_block, cmp_stride;  // compressed window l and stride d (key i: [i d, i d + l))
  int identity;               // l == d == BS: key i is block i (the reference geometry)
  int forced;                 // 1: previous block and block 0 follow the current block
  int nb, nb_len;             // block-score columns (non-identity), padded length
  long long total;
  const __nv_bfloat16* query;
  const int32_t* positions;
  __nv_bfloat16* out;
  int32_t* blocks;
  float* scores;
  float* row_scores;  // global per-row score rows (long key lists), or null: shared memory
  int* error;
};

// What one query row sees. Positions, block ids and key slots use the
// candidate-segment layout when seg_blocks > 0: history below seg_block (key
// slots below seg_key) is shared, candidate s owns seg_blocks blocks (seg_keys
// key slots) after it, and a row of candidate s > 0 never sees the segments
// before its own (the gaps). Without segments the row sees keys [0, nc).
struct Gap {
  int lo = 0, hi = 0;
  __device__ __forceinline__ bool hides(int c) const { return c >= lo && c < hi; }
};

struct RowGeo {
  int nc = 0;       // key slots [0, nc) minus the key gap: complete windows by the row
  Gap keys, blocks;  // other candidates' key slots / blocks
  int s = 0;        // the row's candidate segment (0 outside segments)
  int current = -1, previous = -1, first = -1;  // block ids of the true current,
                                                // previous and first blocks
  // Bit i: key slot col0 + i visible (one mask per 32 columns, so that the
  // unrolled column loops test a bit instead of three bounds).
  __device__ __forceinline__ uint32_t visible_bits(int col0) const {
    auto below = [](int n) -> uint32_t {
      return n <= 0 ? 0u : (n >= 32 ? 0xffffffffu : (1u << n) - 1u);
    };
    uint32_t m = below(nc - col0);
    if (keys.hi > keys.lo) m &= ~(below(keys.hi - col0) & ~below(keys.lo - col0));
    return m;
  }
};

__device__ __forceinline__ RowGeo row_geo(const SelectArgs& a, int pos) {
  RowGeo r;
  if (pos < 0) return r;
  const int bs = a.BS;
  const bool in_segment = a.seg_blocks > 0 && pos / bs >= a.seg_block;
  int truth = pos;
  if (in_segment) {
    const int start = a.seg_block * bs, span = a.seg_blocks * bs;
    r.s = (pos - start) / span;
    truth = start + (pos - start) % span;
    if (r.s > 0) {
      r.keys.lo = a.seg_key;
      r.keys.hi = a.seg_key + r.s * a.seg_keys;
      r.blocks.lo = a.seg_block;
      r.blocks.hi = a.seg_block + r.s * a.seg_blocks;
    }
  }
  // Complete windows i * d + l <= truth + 1, as key slots.
  const int complete =
      truth + 1 >= a.cmp_block ? (truth + 1 - a.cmp_block) / a.cmp_stride + 1 : 0;
  r.nc = in_segment && complete > a.seg_key
             ? a.seg_key + r.s * a.seg_keys + (complete - a.seg_key)
             : complete;
  r.nc = min(r.nc, a.C);
  auto block_id = [&](int true_block) {  // true block -> this row's block id
    return in_segment && true_block >= a.seg_block
               ? a.seg_block + r.s * a.seg_blocks + (true_block - a.seg_block)
               : true_block;
  };
  r.current = pos / bs;
  r.previous = truth / bs >= 1 ? block_id(truth / bs - 1) : -1;
  r.first = block_id(0);
  return r;
}

// Selection-block scores of one row from its compressed-key scores when the
// windows are not the blocks (l, d != BS): block j sums, in ascending window
// order, the scores of the windows that overlap it, each weighted by the
// number of its stride steps inside the block. Only candidates (blocks before
// the current one, outside the gap) are computed; other entries are 0.
__device__ __forceinline__ void aggregate_blocks(const SelectArgs& a, const RowGeo& r,
                                                 const float* key_scores, float* out, int lane) {
  const int bs = a.BS, l = a.cmp_block, d = a.cmp_stride;
  for (int j = lane; j < a.nb; j += 32) {
    float acc = 0.f;
    if (j < r.current && !r.blocks.hides(j)) {
      const bool own = a.seg_blocks > 0 && j >= a.seg_block;
      const int jt = own ? a.seg_block + (j - a.seg_block) % a.seg_blocks : j;
      const int lo = jt * bs, hi = lo + bs;
      const int first = lo - l + 1 > 0 ? (lo - l + 1 + d - 1) / d : 0;
      const int last = (hi - 1) / d;
      for (int i = first; i <= last; ++i) {
        const int w = (min(i * d + l, hi) - max(i * d, lo)) / d;
        if (w <= 0) continue;
        const int slot = a.seg_blocks > 0 && i >= a.seg_key
                             ? a.seg_key + r.s * a.seg_keys + (i - a.seg_key)
                             : i;
        if (slot < a.C) acc += (float)w * key_scores[slot];
      }
    }
    out[j] = acc;
  }
}

// Entries written before the ranked picks: the current block, then (forced)
// the previous block and the first block, each once and only if before the
// current one; the forced blocks are marked taken (-1) in `sc`. Returns the
// number of entries written. Warp-collective.
__device__ __forceinline__ int forced_picks(const SelectArgs& a, const RowGeo& r, int32_t* brow,
                                            float* sc, int lane) {
  int k = 0;
  if (lane == 0) brow[0] = r.current;
  ++k;
  if (a.forced) {
    const int picks[2] = {r.previous, r.first};
    for (int f = 0; f < 2; ++f) {
      const int b = picks[f];
      if (b < 0 || b >= r.current || (f == 1 && b == r.previous)) continue;
      if (k < a.width && lane == 0) brow[k] = b;
      if (lane == 0) sc[b] = -2.f;  // taken
      ++k;
    }
  }
  __syncwarp();
  return k < a.width ? k : a.width;
}

// ------------------------------------------------- tcgen05 / TMEM variant ---
// One CTA of 16 warps per (8 query rows, KV head h). The 8 rows x 16 GQA
// heads form the M = 128 rows of the A operand: TMEM lane m (warps m / 32,
// m / 32 + 4, + 8, + 12, which may all read that lane group) is query row
// q0 + m / 16, head m % 16. The four warps of a lane group split every
// 256-record summary chunk by columns: column quarter cq = warp / 4 owns
// columns 64 cq .. 64 cq + 63, i.e. P sub-tile cq. Summary chunks are staged
// by 3-D tensor TMA (K: channels 0-63, V: 64-127, 128-byte swizzle).
//   S[128 x 256] = Q . K^T             tcgen05.mma kind::f16, N = 64 x tiles
//   pass 1: row max and normaliser from S (TMEM reads, online over chunks,
//           the four column quarters combined through shared memory)
//   pass 2: P = exp(S - max) -> bf16 shared tile; O[128 x 64] += P . V on
//           tcgen05; block score = sum over the 16 heads of P / normaliser
//           (shuffle reduce-scatter across the 16 lanes of a row)
// then one warp per row picks the top-n from the scores in shared memory.
// K and V stay resident across both passes when the summaries fit two
// chunks (and shared memory); longer histories reload them per chunk.
constexpr int kTcRows = 8;
constexpr int kTcThreads = 512;
constexpr int kTcChunk = 256;
constexpr int kTcTileBytes = 64 * 128;              // one 64-record K or V box
constexpr int kTcQBytes = 128 * 128;                // Q: 128 rows x 64 dims bf16
constexpr int kTcChunkBytes = kTcChunk * 128;       // K or V of one chunk
constexpr int kTcPBytes = 128 * kTcChunk * 2;       // P: 4 swizzled [128 x 64] sub-tiles
constexpr int kTcMaxResident = 2;                   // K chunks kept for pass 2
constexpr int kTcTmemCols = 512;                    // S (256) + O (64), power of two
constexpr int kTcMaxScores = 2048;                  // per-row score slots in shared memory
constexpr int kTcReduceBytes = 2 * 4 * 128 * 4;     // per-quarter row max / sum

// Bytes of the K (or V) staging region: one chunk buffer, or with several
// chunks resident (kres > 1) the tiles of every summary, chunk j at
// j * kTcChunkBytes (only the last chunk is partial).
__host__ __device__ __forceinline__ size_t tc_kv_region(int kres, int summaries) {
  return kres > 1 ? (size_t)((summaries + 63) / 64) * kTcTileBytes : (size_t)kTcChunkBytes;
}

size_t tc_smem_bytes(int kres, int summaries, int score_len, int nb_len) {
  return 1024 + (size_t)kTcQBytes + 2 * tc_kv_region(kres, summaries) + kTcPBytes +
         kTcReduceBytes + (size_t)kTcRows * (score_len + nb_len) * 4 + 64;
}

// Top-n key of a score: non-negative scores order like their bit patterns;
// taken (-1) and NaN entries get key 0 and are never picked.
__device__ __forceinline__ uint32_t topn_key(float v) {
  return v >= 0.f ? (__float_as_uint(v) & 0x7fffffffu) + 1u : 0u;
}

// Ranked picks k .. width - 1 of one row (warp-collective). Lane l keeps
// its own candidates l, l + 32, ... below `limit` (visible, not taken) as a
// list sorted by (key descending, block ascending) in registers, at most L
// long: no more than width - k <= L picks can come from one lane. Each pick
// is two warp reductions (the largest head key, then the lowest block id
// holding it) and a shift of the owner's list, so the cost does not grow
// with the number of candidates beyond building the lists.
template <int L>
__device__ __forceinline__ void ranked_picks(const RowGeo& wr, const float* sc, int limit,
                                             int32_t* brow, int k, int width, int lane) {
  uint32_t key[L], idx[L];
#pragma unroll
  for (int j = 0; j < L; ++j) {
    key[j] = 0u;
    idx[j] = 0xffffffffu;
  }
  for (int i = lane; i < limit; i += 32) {
    uint32_t nk = wr.blocks.hides(i) ? 0u : topn_key(sc[i]), ni = (uint32_t)i;
    if (nk == 0u) continue;
    // Candidates arrive in ascending block order, so a strict comparison
    // keeps equal keys in ascending block order.
#pragma unroll
    for (int j = 0; j < L; ++j) {
      const bool swap = nk > key[j];
      const uint32_t tk = swap ? key[j] : nk, ti = swap ? idx[j] : ni;
      key[j] = swap ? nk : key[j];
      idx[j] = swap ? ni : idx[j];
      nk = tk;
      ni = ti;
    }
  }
  for (; k < width; ++k) {
    const uint32_t top = __reduce_max_sync(0xffffffffu, key[0]);
    const uint32_t pick = __reduce_min_sync(0xffffffffu, key[0] == top ? idx[0] : 0xffffffffu);
    if (lane == 0) brow[k] = top ? (int32_t)pick : -1;
    if (top && idx[0] == pick) {  // the owner drops its head
#pragma unroll
      for (int j = 0; j + 1 < L; ++j) {
        key[j] = key[j + 1];
        idx[j] = idx[j + 1];
      }
      key[L - 1] = 0u;
      idx[L - 1] = 0xffffffffu;
    }
  }
}

__global__ void __launch_bounds__(kTcThreads, 1)
    compressed_select_tc_kernel(const __grid_constant__ CUtensorMap map, SelectArgs a,
                                int kres) {
  namespace tc = cxs::tc;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const int H = a.H, C = a.C, score_len = a.score_len;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int lg = warp & 3, cq = warp >> 2;  // TMEM lane group, column quarter
  const int m = 32 * lg + lane;             // A row / TMEM lane of this thread
  const int h = blockIdx.x % H;
  const int q0 = (blockIdx.x / H) * kTcRows;
  // Position of the row this warp ranks (warps 0 .. kTcRows - 1), read once
  // here so the load overlaps the score pass.
  const bool ranks_row = warp < kTcRows && q0 + warp < a.Q;
  const int rank_pos = ranks_row ? a.positions[q0 + warp] : 0;
  uint8_t* q_tile = smem;
  uint8_t* k_base = q_tile + kTcQBytes;
  uint8_t* v_base = k_base + tc_kv_region(kres, C);
  uint8_t* p_tile = v_base + tc_kv_region(kres, C);
  float* red_max = reinterpret_cast<float*>(p_tile + kTcPBytes);  // [4][128]
  float* red_sum = red_max + 4 * 128;                               // [4][128]
  // Per-row key scores [kTcRows][score_len] and block scores
  // [kTcRows][nb_len]: in shared memory, or, for long key lists, in this
  // CTA's rows of the global score scratch (L2-resident; every access is
  // ordered by the same CTA barriers).
  float* const rows_smem = red_sum + 4 * 128;
  const long long row_floats = (long long)kTcRows * (score_len + a.nb_len);
  float* scores = a.row_scores ? a.row_scores + (long long)blockIdx.x * row_floats : rows_smem;
  float* bscores = scores + kTcRows * score_len;
  uint64_t* tma_bar =
      reinterpret_cast<uint64_t*>(a.row_scores ? rows_smem : rows_smem + row_floats);
  uint64_t* mma_bar = tma_bar + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_bar + 1);

  // Every chunk of summaries is processed (rows mask what lies at or beyond
  // their own complete-block count), so the copies can start at once.
  const int chunks = (C + kTcChunk - 1) / kTcChunk;
  const bool resident = chunks <= kres;  // K and V of every chunk stay in shared memory
  // Two chunks whose second holds at most 192 summaries (H = 16384 with the
  // extend's new blocks gives 260): both S chunks stay in TMEM (columns
  // [0, 256) and [256, 448), O in [448, 512)), computed once for both passes.
  const bool s_resident = resident && chunks == 2 && C <= kTcChunk + 192;
  auto s_of = [&](int j) { return s_resident ? (uint32_t)(kTcChunk * j) : 0u; };
  auto tiles_of = [&](int j) { return min(4, (C - kTcChunk * j + 63) / 64); };
  auto load_half = [&](int j, uint8_t* dst, int channel) {
    for (int t = 0; t < tiles_of(j); ++t)
      cxs::tma_load_3d(cxs::smem_addr(dst + t * kTcTileBytes), &map, channel, h,
                       kTcChunk * j + 64 * t, tma_bar);
  };
  auto k_of = [&](int j) { return k_base + (resident ? j : 0) * kTcChunkBytes; };
  auto v_of = [&](int j) { return v_base + (resident ? j : 0) * kTcChunkBytes; };

  if (tid == 0) {
    cxs::mbar_init(tma_bar, 1);
    cxs::mbar_init(mma_bar, 1);
    cxs::fence_mbar_init();
    if (chunks > 0) {
      const int first = resident ? chunks : 1;
      uint32_t bytes = 0;
      for (int j = 0; j < first; ++j) bytes += 2 * tiles_of(j) * kTcTileBytes;
      cxs::mbar_expect_tx(tma_bar, bytes);
      for (int j = 0; j < first; ++j) {
        load_half(j, k_of(j), 0);
        load_half(j, v_of(j), 64);
      }
    }
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     cxs::smem_addr(tmem_slot)),
                 "r"(kTcTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  for (int i = tid; i < kTcRows * score_len; i += kTcThreads) scores[i] = 0.f;
  // Row m of Q (pre-scaled by 1/8 and rounded to bf16); this thread writes
  // 16-byte chunks 2 cq and 2 cq + 1 of it.
  const int ql = m >> 4, g = m & 15, q = q0 + ql;
  const bool row_ok = q < a.Q;
  const int pos = row_ok ? a.positions[q] : -1;
  const RowGeo rg = row_geo(a, pos);
  const long long qrow = ((long long)q * H + h) * cxs::kGroups + g;  // [Q, H, 16] row index
#pragma unroll
  for (int c = 2 * cq; c < 2 * cq + 2; ++c) {
    uint4 out = make_uint4(0, 0, 0, 0);
    if (row_ok) {
      const uint4 in = reinterpret_cast<const uint4*>(a.query + qrow * cxs::kDim)[c];
      const uint32_t* w = reinterpret_cast<const uint32_t*>(&in);
      uint32_t* o = reinterpret_cast<uint32_t*>(&out);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = cxs::unpack_bf16(w[e]);
        o[e] = cxs::pack_bf16(f.x * 0.125f, f.y * 0.125f);
      }
    }
    *reinterpret_cast<uint4*>(q_tile + tc::sw128_chunk(m, c)) = out;
  }
  cxs::fence_proxy_async_shared();
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t lane_off = (uint32_t)(32 * lg) << 16;
  const uint32_t s_col = tmem, o_col = tmem + (s_resident ? 448 : kTcChunk);
  const uint32_t s_addr = s_col + lane_off, o_addr = o_col + lane_off;
  const uint32_t q_addr = cxs::smem_addr(q_tile), p_addr = cxs::smem_addr(p_tile);
  const long long spin = 1ll << 31;
  uint32_t tph = 0, mph = 0;
  bool ok = true;

  // Every thread waits; the CTA then agrees on the outcome, so a timeout
  // (a broken launch: these copies read device memory only) leaves all
  // threads on the same path.
  auto wait_tma = [&]() {
    bool done = ok && tc::bounded_wait(tma_bar, tph, spin, a.error, cxs::kErrCopyTimeout);
    tph ^= 1;
    ok = __syncthreads_and(done);
  };
  auto wait_mma = [&]() {
    bool done = ok && tc::bounded_wait(mma_bar, mph, spin, a.error, cxs::kErrCopyTimeout);
    mph ^= 1;
    ok = __syncthreads_and(done);
    tc::fence_after();
  };
  auto mma_scores = [&](int j) {  // S = Q . K_j^T, N = 64 x tiles (both chunks if TMEM-resident)
    if (tid == 0) {
      tc::fence_after();
      for (int c = j; c < (s_resident ? chunks : j + 1); ++c) {
        const uint32_t ka = cxs::smem_addr(k_of(c));
        const uint32_t id = tc::idesc_bf16(128, 64 * tiles_of(c), 0, 0);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          tc::mma(s_col + s_of(c), tc::desc_sw128(q_addr + 32 * k, 16, 1024),
                  tc::desc_sw128(ka + 32 * k, 16, 1024), id, k);
      }
      tc::commit(mma_bar);
    }
    wait_mma();
  };
  auto cta_sync = [&]() {
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
  };

  // Pass 1: per-row max and normaliser over every chunk. With a single chunk
  // (the common case) the probabilities computed for the normaliser stay in
  // registers for pass 2 (same values: the chunk's max is the final max).
  float m_run = -INFINITY, l_run = 0.f;
  const bool single = chunks == 1;
  float v0[32], v1[32];
  for (int j = 0; j < chunks && ok; ++j) {
    if (j > 0 && !resident) {
      if (tid == 0) {
        cxs::mbar_expect_tx(tma_bar, tiles_of(j) * kTcTileBytes);
        load_half(j, k_base, 0);
      }
    }
    if (j == 0 || !resident) wait_tma();
    if (!ok) break;
    if (!s_resident || j == 0) mma_scores(j);
    // This warp's column groups (32 columns each) of the chunk: 2 cq, 2 cq + 1.
    const bool mine = cq < tiles_of(j);
    const int col0 = kTcChunk * j + 64 * cq;
    if (mine) {  // warp-uniform
      tc::ld32(s_addr + s_of(j) + 64 * cq, v0);
      tc::ld32(s_addr + s_of(j) + 64 * cq + 32, v1);
    }
    float mt = -INFINITY;
    const uint32_t vis0 = rg.visible_bits(col0), vis1 = rg.visible_bits(col0 + 32);
    if (mine) {
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        if ((vis0 >> i) & 1u) mt = fmaxf(mt, v0[i]);
        if ((vis1 >> i) & 1u) mt = fmaxf(mt, v1[i]);
      }
    }
    red_max[cq * 128 + m] = mt;
    cta_sync();  // every thread has read S (the next chunk overwrites it) and posted its max
    const float m_new = fmaxf(m_run, fmaxf(fmaxf(red_max[m], red_max[128 + m]),
                                           fmaxf(red_max[256 + m], red_max[384 + m])));
    const float off = m_new == -INFINITY ? 0.f : m_new * tc::kLog2e;
    float sum = 0.f;
    if (mine) {
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float p0 = (vis0 >> i) & 1u ? tc::ex2(fmaf(v0[i], tc::kLog2e, -off)) : 0.f;
        const float p1 = (vis1 >> i) & 1u ? tc::ex2(fmaf(v1[i], tc::kLog2e, -off)) : 0.f;
        sum += p0;
        sum += p1;
        if (single) {
          v0[i] = p0;
          v1[i] = p1;
        }
      }
    }
    red_sum[cq * 128 + m] = sum;
    __syncthreads();
    if (m_new != -INFINITY) {
      const float total = (red_sum[m] + red_sum[128 + m]) + (red_sum[256 + m] + red_sum[384 + m]);
      l_run = (m_run == -INFINITY ? 0.f : l_run * tc::ex2((m_run - m_new) * tc::kLog2e)) + total;
      m_run = m_new;
    }
    __syncthreads();  // red_max / red_sum are reused by the next chunk
  }

  // Pass 2: probabilities -> P . V and the per-block scores.
  const float offset = m_run == -INFINITY ? 0.f : m_run * tc::kLog2e;
  const float inv_l = l_run > 0.f ? 1.f / l_run : 0.f;
  float* my_scores = scores + ql * score_len;
  for (int j = 0; j < chunks && ok; ++j) {
    if (chunks > 1 && !s_resident) {
      if (!resident) {
        if (tid == 0) {
          cxs::mbar_expect_tx(tma_bar, 2 * tiles_of(j) * kTcTileBytes);
          load_half(j, k_base, 0);
          load_half(j, v_base, 64);
        }
        wait_tma();
        if (!ok) break;
      }
      mma_scores(j);
    }
    if (cq < tiles_of(j)) {  // warp-uniform
      uint8_t* sub = p_tile + cq * (128 * 128);
#pragma unroll 1
      for (int half = 0; half < 2; ++half) {
        const int col0 = kTcChunk * j + 64 * cq + 32 * half;
        float v[32];
        if (single) {  // pass 1's probabilities (offset = its maximum)
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = half ? v1[i] : v0[i];
        } else {
          tc::ld32(s_addr + s_of(j) + 64 * cq + 32 * half, v);
          const uint32_t vis = rg.visible_bits(col0);
#pragma unroll
          for (int i = 0; i < 32; ++i)
            v[i] = (vis >> i) & 1u ? tc::ex2(fmaf(v[i], tc::kLog2e, -offset)) : 0.f;
        }
        // P (bf16): 16-byte chunks 4 half .. 4 half + 3 of row m of sub-tile cq.
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint4 chunk = make_uint4(cxs::pack_bf16(v[8 * k + 0], v[8 * k + 1]),
                                         cxs::pack_bf16(v[8 * k + 2], v[8 * k + 3]),
                                         cxs::pack_bf16(v[8 * k + 4], v[8 * k + 5]),
                                         cxs::pack_bf16(v[8 * k + 6], v[8 * k + 7]));
          *reinterpret_cast<uint4*>(sub + tc::sw128_chunk(m, 4 * half + k)) = chunk;
        }
        // Normalised probabilities summed over the row's 16 heads: a
        // reduce-scatter across lanes (xor 8, 4, 2, 1) leaves lane l of the
        // half-warp with columns 2 (l % 16) and 2 (l % 16) + 1 of the group.
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] *= inv_l;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const bool up = lane & 8;
          const float send = up ? v[i] : v[16 + i];
          v[i] = (up ? v[16 + i] : v[i]) + __shfl_xor_sync(0xffffffffu, send, 8);
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const bool up = lane & 4;
          const float send = up ? v[i] : v[8 + i];
          v[i] = (up ? v[8 + i] : v[i]) + __shfl_xor_sync(0xffffffffu, send, 4);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const bool up = lane & 2;
          const float send = up ? v[i] : v[4 + i];
          v[i] = (up ? v[4 + i] : v[i]) + __shfl_xor_sync(0xffffffffu, send, 2);
        }
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const bool up = lane & 1;
          const float send = up ? v[i] : v[2 + i];
          v[i] = (up ? v[2 + i] : v[i]) + __shfl_xor_sync(0xffffffffu, send, 1);
        }
        const int col = col0 + 2 * g;
        if (col < C) my_scores[col] = v[0];
        if (col + 1 < C) my_scores[col + 1] = v[1];
      }
    }
    cxs::fence_proxy_async_shared();
    cta_sync();
    if (tid == 0) {
      const uint32_t id = tc::idesc_bf16(128, 64, 0, 1);
      const uint32_t v_addr = cxs::smem_addr(v_of(j));
      for (int kk = 0; kk < 4 * tiles_of(j); ++kk)
        tc::mma(o_col, tc::desc_sw128(p_addr + (kk >> 2) * (128 * 128) + 32 * (kk & 3), 16, 1024),
                tc::desc_sw128(v_addr + (kk >> 2) * kTcTileBytes + 2048 * (kk & 3), 16, 1024), id,
                j > 0 || kk > 0);
      tc::commit(mma_bar);
    }
    wait_mma();
  }

  // Compressed-branch output: O / normaliser, bf16; this thread writes dims
  // 16 cq .. 16 cq + 15 of row m.
  if (row_ok) {
    uint4* dst = reinterpret_cast<uint4*>(a.out + qrow * cxs::kDim + 16 * cq);
    dst[0] = make_uint4(0, 0, 0, 0);
    dst[1] = make_uint4(0, 0, 0, 0);
  }
  if (chunks > 0 && ok) {
    float o[16];
    tc::ld16(o_addr + 16 * cq, o);
    if (row_ok) {
      uint4* dst = reinterpret_cast<uint4*>(a.out + qrow * cxs::kDim + 16 * cq);
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        uint32_t r[4];
#pragma unroll
        for (int e = 0; e < 4; ++e)
          r[e] = cxs::pack_bf16(l_run > 0.f ? o[8 * k + 2 * e] / l_run : 0.f,
                                l_run > 0.f ? o[8 * k + 2 * e + 1] / l_run : 0.f);
        dst[k] = make_uint4(r[0], r[1], r[2], r[3]);
      }
    }
  }
  __syncthreads();
  // Block scores of each row: its key scores in the reference geometry, else
  // aggregated by warp r for row r.
  const bool rank_keys = a.identity;
  if (!rank_keys) {
    if (ranks_row) {
      const RowGeo wr = row_geo(a, rank_pos);
      aggregate_blocks(a, wr, scores + warp * score_len, bscores + warp * a.nb_len, lane);
    }
    __syncthreads();
  }
  float* const ranked = rank_keys ? scores : bscores;
  const int ranked_len = rank_keys ? score_len : a.nb_len;
  const int columns = rank_keys ? C : a.nb;
  if (a.scores) {
    for (int r = 0; r < kTcRows; ++r) {
      if (q0 + r >= a.Q) break;
      float* srow = a.scores + ((long long)(q0 + r) * H + h) * columns;
      for (int i = tid; i < columns; i += kTcThreads) srow[i] = ranked[r * ranked_len + i];
    }
    __syncthreads();
  }
  // Top-n, warp r for row r: the current block first, then earlier blocks by
  // (score descending, block ascending).
  if (ranks_row) {
    const int qq = q0 + warp;
    const RowGeo wr = row_geo(a, rank_pos);
    const int limit = min(wr.current, ranked_len);
    float* sc = ranked + warp * ranked_len;
    int32_t* brow = a.blocks + ((long long)qq * H + h) * a.width;
    int k = 1;
    if (wr.current < 0) {
      if (lane == 0) brow[0] = -1;
    } else {
      k = forced_picks(a, wr, brow, sc, lane);
    }
    if (a.width <= 16)
      ranked_picks<16>(wr, sc, limit, brow, k, a.width, lane);
    else
      ranked_picks<32>(wr, sc, limit, brow, k, a.width, lane);
  }
  tc::fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTcTmemCols));
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

extern "C" int cxs_select_score_columns(const cxs_select_geometry* geometry,
                                        int32_t* columns) {
  if (!geometry || !columns) return set_error(CXS_ERR_INVALID, "null argument");
  const cxs_select_geometry& g = *geometry;
  const int bs = g.block_size, l = g.window, d = g.stride;
  if (bs < 1 || l < 1 || d < 1 || g.summaries < 0 || g.total < 1)
    return set_error(CXS_ERR_INVALID, "invalid compressed-select geometry");
  if (l == bs && d == bs) {
    *columns = g.summaries;
  } else if (g.segment_tokens > 0) {
    const long long seg_key = g.segment_start >= l ? (g.segment_start - l) / d + 1 : 0;
    const long long seg_keys = g.segment_tokens / d;
    const long long segments = seg_keys ? (g.summaries - seg_key + seg_keys - 1) / seg_keys : 0;
    *columns = (int32_t)(g.segment_start / bs + (segments > 0 ? segments : 0) *
                                                    (g.segment_tokens / bs));
  } else {
    *columns = (int32_t)((g.total + bs - 1) / bs);
  }
  return CXS_OK;
}

extern "C" int cxs_compressed_select_nsa(const cxs_select_geometry* geometry, const void* query,
                                         const void* compressed, const int32_t* positions,
                                         void* out, int32_t* blocks, float* scores,
                                         void* stream) {
  if (!geometry) return set_error(CXS_ERR_INVALID, "null compressed-select geometry");
  const cxs_select_geometry& g = *geometry;
  const int queries = g.queries, heads = g.heads, block_size = g.block_size, count = g.count;
  const int summaries = g.summaries, l = g.window, d = g.stride;
  const long long total = g.total, segment_start = g.segment_start,
                  segment_tokens = g.segment_tokens;
  if (queries < 1 || heads < 1 || block_size < 1 || count < 1 || total < 1 || summaries < 0)
    return set_error(CXS_ERR_INVALID, "invalid compressed-select geometry");
  if (d < 1 || l < d || l % d || block_size % d || (g.forced != 0 && g.forced != 1))
    return set_error(CXS_ERR_INVALID,
                     "window must be a multiple of the stride, the block a multiple of the "
                     "stride, forced 0 or 1");
  if (segment_tokens < 0 || segment_start < 0 ||
      (segment_tokens > 0 && (segment_start % block_size || segment_tokens % block_size ||
                              segment_start + segment_tokens * (long long)queries > INT32_MAX)))
    return set_error(CXS_ERR_INVALID,
                     "segment_start / segment_tokens must be block multiples and fit int32");
  if (!query || !out || !blocks || !positions || (summaries > 0 && !compressed))
    return set_error(CXS_ERR_INVALID, "null compressed-select argument");
  if (((uintptr_t)compressed & 15) || ((uintptr_t)query & 15) || ((uintptr_t)out & 15))
    return set_error(CXS_ERR_INVALID, "query/compressed/out must be 16-byte aligned");
  if (count > 32) return set_error(CXS_ERR_INVALID, "count (top-n) must be at most 32");
  long long blocks_total = (total + block_size - 1) / block_size;
  int width = (int)(count < blocks_total ? count : blocks_total);
  if (summaries > (1 << 20)) return set_error(CXS_ERR_CAPACITY, "too many summaries");
  int32_t columns = 0;
  int status = cxs_select_score_columns(geometry, &columns);
  if (status != CXS_OK) return status;
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
  a.seg_block = segment_tokens > 0 ? (int)(segment_start / block_size) : 0;
  a.seg_blocks = (int)(segment_tokens / block_size);
  a.seg_key = segment_tokens > 0 ? (int)(segment_start >= l ? (segment_start - l) / d + 1 : 0) : 0;
  a.seg_keys = (int)(segment_tokens / d);
  a.cmp_block = l;
  a.cmp_stride = d;
  a.identity = l == block_size && d == block_size;
  a.forced = g.forced;
  a.nb = a.identity ? 0 : columns;
  a.nb_len = a.identity ? 0 : (columns + 3) & ~3;
  a.query = (const __nv_bfloat16*)query;
  a.positions = positions;
  a.out = (__nv_bfloat16*)out;
  a.blocks = blocks;
  a.scores = scores;
  int device = 0;
  CXS_CUDA(cudaGetDevice(&device));
  if (device < 0 || device >= kMaxDevices)
    return set_error(CXS_ERR_UNSUPPORTED, "device index %d beyond %d", device, kMaxDevices);
  if (!g_select_ready[device]) {
    // Once per device: the error sink's device address and the shared-memory
    // opt-in (up to the per-block maximum).
    CXS_CUDA(cudaGetSymbolAddress((void**)&g_select_error_address[device], g_select_error));
    CXS_CUDA(cudaFuncSetAttribute(compressed_select_tc_kernel,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem));
    g_select_ready[device] = true;
  }
  a.error = g_select_error_address[device];
  long long longest = summaries > blocks_total ? summaries : blocks_total;
  if (longest > (1 << 20) || columns > (1 << 20))
    return set_error(CXS_ERR_CAPACITY, "too many blocks");
  int score_len = (int)((longest + 3) & ~3ll);
  a.score_len = score_len;
  a.row_scores = nullptr;
  const int grid = ((queries + kTcRows - 1) / kTcRows) * heads;
  int chunks = (summaries + kTcChunk - 1) / kTcChunk;
  int kres = chunks <= kTcMaxResident ? (chunks > 0 ? chunks : 1) : 1;
  if (kres > 1 && tc_smem_bytes(kres, summaries, score_len, a.nb_len) > (size_t)kMaxSmem) kres = 1;
  size_t tc_smem = tc_smem_bytes(kres, summaries, score_len, a.nb_len);
  if (score_len > kTcMaxScores || tc_smem > (size_t)kMaxSmem) {
    // Long key lists: the score rows go to the device's global scratch.
    const size_t need = (size_t)grid * kTcRows * (score_len + a.nb_len) * sizeof(float);
    int status = score_scratch(device, need, (cudaStream_t)stream, &a.row_scores);
    if (status != CXS_OK) return status;
    kres = chunks <= kTcMaxResident && tc_smem_bytes(chunks, summaries, 0, 0) <= (size_t)kMaxSmem
               ? (chunks > 0 ? chunks : 1) : 1;
    tc_smem = tc_smem_bytes(kres, summaries, 0, 0);
  }
  compressed_select_tc_kernel<<<grid, kTcThreads, tc_smem, (cudaStream_t)stream>>>(map, a, kres);
  CXS_LAUNCH_CHECK("compressed_select_tc_kernel");
  return CXS_OK;
}

extern "C" int cxs_compressed_select_segments(
    const void* query, const void* compressed, int32_t summaries, const int32_t* positions,
    int32_t queries, int32_t heads, int32_t block_size, int32_t count, int64_t total,
    int64_t segment_start, int64_t segment_tokens, void* out, int32_t* blocks, float* scores,
    void* stream) {
  cxs_select_geometry g = {};
  g.queries = queries;
  g.heads = heads;
  g.block_size = block_size;
  g.count = count;
  g.summaries = summaries;
  g.window = block_size;
  g.stride = block_size;
  g.forced = 0;
  g.total = total;
  g.segment_start = segment_start;
  g.segment_tokens = segment_tokens;
  return cxs_compressed_select_nsa(&g, query, compressed, positions, out, blocks, scores, stream);
}

extern "C" int cxs_compressed_select(const void* query, const void* compressed, int32_t summaries,
                                     const int32_t* positions, int32_t queries, int32_t heads,
                                     int32_t block_size, int32_t count, int64_t total, void* out,
                                     int32_t* blocks, float* scores, void* stream) {
  return cxs_compressed_select_segments(query, compressed, summaries, positions, queries, heads,
                                        block_size, count, total, 0, 0, out, blocks, scores,
                                        stream);
}
