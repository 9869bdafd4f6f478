// Block-source preparation and the persistent IO + attention kernel.
//
// Reference behaviour: tma/transport.py:17-112 (_prepare_sources, execute)
// and the staged TMA kernel tma/pipeline.py:96-742 (IO CTAs :347-421,
// consumer CTAs :436-655, online-softmax block step :172-257). This is a new
// sm_100a design: one cooperative launch whose CTAs each run one IO warp and
// four tcgen05 attention warps; see cxs_fetch_attend in include/cxlsparse.h.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <climits>
#include <mutex>

#include "cxs_common.cuh"
#include "tile_tc.cuh"

using cxs::kTokenBytes;
using cxs::bf16_round;
using cxs::unpack_bf16;
using cxs_host::set_error;

namespace {

constexpr int kAttnWarps = cxs::tc::kEngines;     // one per TMEM subpartition
constexpr int kTmemAlloc = kAttnWarps * cxs::tc::kTmemCols;  // 512: all of TMEM
constexpr int kThreads = 32 * (1 + kAttnWarps);

struct AttendArgs {
  int Q, H, W, BS, P, window, window_len, gate;
  long long window_start, spin_limit;
  int seg_start, seg_tokens;  // candidate segments (seg_tokens 0: one suffix)
  int consumers;  // attention warps of the launch: grid * kAttnWarps
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
  __nv_bfloat16* out_peer;  // optional second copy of every output row (a peer GPU's buffer)
  int out_heads, out_head0;  // output row of (q, h): q * out_heads + out_head0 + h
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

// ------------------------------------------------------- attention warps ---
// One attention warp (engine `w` of its CTA): query rows with index
// w * gridDim.x + blockIdx.x + k * consumers. Per row it runs the
// sliding-window tiles, then the row's selected occurrences in list order
// (duplicates attended again, as the reference does), on the tcgen05 engine
// of tile_tc.cuh, and writes the (gate-mixed) output.
//
// Tile t uses K buffer t % 2 and V buffer t % 2; one mbarrier commit C_t per
// tile covers P.V of tile t-1 and S of tile t. Lane 0 keeps the copies ahead:
// K of tile j may start once S of tile j-2 is done, V of tile j once P.V of
// tile j-2 is, and a selected block only after its ready flag is set.
//   A  every lane waits C_t; lane 0 starts what is free and known ready
//   B  softmax of S(t) -> P, running max/denominator, O rescale in TMEM
//   C  lane 0 makes sure K of tile t+1 is under way (acquire-waiting on its
//      ready flag); the warp agrees on every wait's status, and a failure
//      ends the launch for this warp once its copies have landed
//   D  lane 0 issues O += P.V(t) and S(t+1) as their copies land, commits
template <int BS>
__device__ __forceinline__ void attention_warp(const CUtensorMap& kv_map,
                                               const CUtensorMap& win_map, const AttendArgs& a,
                                               uint8_t* q_tile, uint8_t* p_tile, uint8_t* wbase,
                                               int w, uint32_t tmem) {
  namespace tc = cxs::tc;
  const tc::WarpSmem ws{wbase};
  const int lane = threadIdx.x % 32, half = lane >> 4;
  const bool leader = lane == 0;
  const int m = 32 * w + lane;  // this lane's row of the Q / P tiles and of S / O
  const uint32_t lane_off = (uint32_t)(32 * w) << 16;
  const uint32_t s_col = tmem, o_col = tmem + 64;  // MMA destinations
  const uint32_t s_addr = s_col + lane_off, o_addr = o_col + lane_off;
  const uint32_t id_s = tc::idesc_bf16(128, 64, 0, 0), id_o = tc::idesc_bf16(128, 64, 0, 1);
  const uint32_t q_addr = cxs::smem_addr(q_tile), p_addr = cxs::smem_addr(p_tile);
  uint32_t k_phase = 0, v_phase = 0, mma_phase = 0;  // bit b: phase of buffer b
  const int rows = a.Q * a.H;
  if (leader) {
    cxs::tma_prefetch_desc(&kv_map);
    if (a.window) cxs::tma_prefetch_desc(&win_map);
  }
  auto mma_scores = [&](int b) {  // S = Q . K(b)^T
    const uint32_t ka = cxs::smem_addr(ws.k(b));
#pragma unroll
    for (int k = 0; k < 4; ++k)
      tc::mma(s_col, tc::desc_sw128(q_addr + 32 * k, 16, 1024),
              tc::desc_sw128(ka + 32 * k, 16, 1024), id_s, k);
  };
  auto mma_output = [&](int b, bool accumulate) {  // O (+)= P . V(b)
    const uint32_t va = cxs::smem_addr(ws.v(b));
#pragma unroll
    for (int k = 0; k < 4; ++k)
      tc::mma(o_col, tc::desc_sw128(p_addr + 32 * k, 16, 1024),
              tc::desc_sw128(va + 2048 * k, 16, 1024), id_o, accumulate || k > 0);
  };
  for (int row = w * gridDim.x + blockIdx.x; row < rows; row += a.consumers) {
    const int h = row % a.H;
    const int pos = a.row_positions[row];
    // Window: positions [w_lo, w_hi], then [o_lo, o_hi] (positions and window
    // bounds fit int32: host-checked), each in tiles of 64 from its start.
    // With candidate segments, a row of segment s sees the history below
    // seg_start, then its own segment, which starts at seg_start + s *
    // seg_tokens (true position = seg_start + offset into the segment); every
    // segment row splits its window there, whatever s, so that a candidate's
    // tiles (and roundings) do not depend on its segment index. Without
    // segments the window is one contiguous range.
    int w_lo = 1, w_hi = 0, o_lo = 1, o_hi = 0;
    if (a.window > 0 && pos >= 0) {
      const int w_first = (int)a.window_start, w_last = w_first + a.window_len - 1;
      int own = -1, real = pos;
      if (a.seg_tokens > 0 && pos >= a.seg_start) {
        own = a.seg_start + (pos - a.seg_start) / a.seg_tokens * a.seg_tokens;
        real = a.seg_start + (pos - own);
      }
      w_lo = max(max(real - a.window + 1, 0), w_first);
      if (own < 0) {
        w_hi = min(pos, w_last);
      } else {
        w_hi = min(a.seg_start - 1, w_last);
        o_lo = max(own + max(real - a.window + 1 - a.seg_start, 0), w_first);
        o_hi = min(pos, w_last);
      }
    }
    const int n_hist = w_lo <= w_hi ? (w_hi - w_lo) / tc::kTileRows + 1 : 0;
    const int n_win = n_hist + (o_lo <= o_hi ? (o_hi - o_lo) / tc::kTileRows + 1 : 0);
    // First position and last position of window tile j.
    auto win_first = [&](int j) {
      return j < n_hist ? w_lo + j * tc::kTileRows : o_lo + (j - n_hist) * tc::kTileRows;
    };
    auto win_last = [&](int j) { return j < n_hist ? w_hi : o_hi; };
    const int count = pos >= 0 ? min(a.all_counts[row], a.W) : 0;
    const int total = n_win + count;
    // Lane i holds selected occurrence i (block id and first position).
    int my_block = -1, my_start = 0;
    if (lane < count) {
      my_block = a.all_ids[(long long)row * a.W + lane];
      if (my_block >= 0 && my_block < a.P) my_start = a.starts[my_block];
    }
    // Block of tile j (all lanes; -1 for window tiles and past the end).
    auto block_of = [&](int j) {
      const int b = __shfl_sync(0xffffffffu, my_block, (j - n_win) & 31);
      return (j >= n_win && j < total) ? b : -1;
    };
    tc::write_query_row(q_tile, a.query, row, m, lane);
    cxs::fence_proxy_async_shared();
    __syncwarp();
    // Lane 0's copy schedule for this row: K / V copies of tiles [0, kn) /
    // [0, vn) started, [0, kw) / [0, vw) landed.
    int kn = 0, vn = 0, kw = 0, vw = 0;
    int pf_tile = -1, pf_ready = 0;  // ready flag of tile pf_tile, acquire-loaded earlier
    bool failed = false;
    auto start_copy = [&](int j, int blk, bool value) {
      const int b = j & 1;
      uint64_t* bar = value ? ws.vbar(b) : ws.kbar(b);
      uint8_t* dst = value ? ws.v(b) : ws.k(b);
      if (j < n_win) {
        cxs::mbar_expect_tx(bar, tc::kTileBytes);
        tc::window_load(dst, &win_map, value ? 64 : 0, h, win_first(j) - (int)a.window_start,
                        bar);
      } else {
        cxs::mbar_expect_tx(bar, BS * 128);
        cxs::tma_load_2d(dst, &kv_map, value ? 64 : 0, blk * BS, bar);
      }
    };
    // Start every copy that is free during step t (K of tiles <= t + 2, V of
    // tiles <= t + 1 whose K is under way) and whose block is known ready;
    // with `need_k`, K of tile t + 1 is started even if that means waiting
    // for its ready flag. b1..b3: blocks of tiles t + 1 .. t + 3.
    auto pump = [&](int t, int b1, int b2, int b3, bool need_k) {
      while (!failed && kn < total && kn <= t + 2) {
        const int j = kn, blk = j == t + 1 ? b1 : b2;
        if (j >= n_win) {
          if (j < t + 1 || blk < 0 || blk >= a.P) {
            atomicOr(a.error, cxs::kErrBadBlock);
            failed = true;
            break;
          }
          if (!(pf_tile == j && pf_ready)) {
            if (!(need_k && j == t + 1)) break;
            if (!cxs::wait_ready_bounded(&a.ready[blk], a.spin_limit, a.error)) {
              failed = true;
              break;
            }
          }
          cxs::fence_proxy_async_global();
        }
        start_copy(j, blk, false);
        ++kn;
      }
      while (!failed && vn < kn && vn <= t + 1) {
        const int blk = vn == t + 1 ? b1 : -1;
        if (vn >= n_win && (blk < 0 || blk >= a.P)) {
          atomicOr(a.error, cxs::kErrBadBlock);
          failed = true;
          break;
        }
        start_copy(vn, blk, true);
        ++vn;
      }
      // Acquire-load the ready flag of the next K tile now; it is read at
      // the next call, after its latency has passed.
      if (!failed && kn < total && kn >= n_win && !(pf_tile == kn && pf_ready)) {
        const int blk = kn == t + 1 ? b1 : (kn == t + 2 ? b2 : b3);
        if (blk >= 0 && blk < a.P) {
          pf_tile = kn;
          pf_ready = cxs::ld_acquire(&a.ready[blk]);
        }
      }
    };
    // Lane 0: let every started copy land (bounded) before giving up the row.
    auto drain = [&]() {
      for (; kw < kn; ++kw) {
        tc::bounded_wait(ws.kbar(kw & 1), (k_phase >> (kw & 1)) & 1u, a.spin_limit, a.error,
                         cxs::kErrCopyTimeout);
        k_phase ^= 1u << (kw & 1);
      }
      for (; vw < vn; ++vw) {
        tc::bounded_wait(ws.vbar(vw & 1), (v_phase >> (vw & 1)) & 1u, a.spin_limit, a.error,
                         cxs::kErrCopyTimeout);
        v_phase ^= 1u << (vw & 1);
      }
    };
    auto land = [&](bool value) -> bool {  // lane 0: wait for the next K or V copy
      int& done = value ? vw : kw;
      uint32_t& phase = value ? v_phase : k_phase;
      const int b = done & 1;
      const bool ok = tc::bounded_wait(value ? ws.vbar(b) : ws.kbar(b), (phase >> b) & 1u,
                                       a.spin_limit, a.error, cxs::kErrCopyTimeout);
      phase ^= 1u << b;
      ++done;
      return ok;
    };
    bool alive = true;
    float m_run = -INFINITY, l_run = 0.f;
    uint32_t win_packed[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) win_packed[i] = 0;
    if (total > 0) {
      {
        const int b0 = block_of(0), b1 = block_of(1), b2 = block_of(2);
        if (leader) {
          pump(-1, b0, b1, b2, true);
          if (!failed) failed = !land(false);
          if (!failed) {
            tc::fence_after();
            mma_scores(0);
          }
          tc::commit(ws.mma_bar());
        }
      }
      for (int t = 0; t < total; ++t) {
        const bool first_of_branch = t == 0 || t == n_win;
        const int b1 = block_of(t + 1), b2 = block_of(t + 2), b3 = block_of(t + 3);
        const int cur_block = __shfl_sync(0xffffffffu, my_block, (t - n_win) & 31);
        const int cur_start = __shfl_sync(0xffffffffu, my_start, (t - n_win) & 31);
        // A
        const bool waited = tc::bounded_wait(ws.mma_bar(), mma_phase, a.spin_limit, a.error,
                                             cxs::kErrCopyTimeout);
        mma_phase ^= 1;
        tc::fence_after();
        if (t == n_win && n_win > 0) {
          // Window branch complete: keep its normalised bf16 output, restart.
          float o[32];
          tc::combine_o(o_addr, half, o);
          const float den = l_run > 0.f ? l_run : 1.f;
#pragma unroll
          for (int i = 0; i < 16; ++i)
            win_packed[i] = cxs::pack_bf16(o[2 * i] / den, o[2 * i + 1] / den);
          m_run = -INFINITY;
          l_run = 0.f;
        }
        if (leader) pump(t, b1, b2, b3, false);
        // B
        int lo = 0, hi = -1;
        if (t < n_win) {
          hi = min(win_last(t) - win_first(t), tc::kTileRows - 1);
        } else if (cur_block >= 0 && cur_block < a.P) {
          hi = min(pos - cur_start, BS - 1);
        }
        const float m_old = m_run;
        const float factor = tc::softmax_half(p_tile, s_addr, lo, hi, m_run, l_run, m, half);
        if (!first_of_branch) tc::rescale_o(o_addr, factor, m_old != -INFINITY && factor != 1.f);
        cxs::fence_proxy_async_shared();
        tc::fence_before();
        // C
        if (leader) pump(t, b1, b2, b3, true);
        const bool ok = __all_sync(0xffffffffu, waited) && !__shfl_sync(0xffffffffu, failed, 0);
        if (!ok) {
          if (leader) drain();
          alive = false;
          break;
        }
        // D
        if (leader) {
          tc::fence_after();
          if (land(true)) {
            mma_output(t & 1, !first_of_branch);
            if (t + 1 < total) {
              if (land(false))
                mma_scores((t + 1) & 1);
              else
                failed = true;
            }
          } else {
            failed = true;
          }
          tc::commit(ws.mma_bar());
        }
        __syncwarp();
      }
      if (alive && __shfl_sync(0xffffffffu, failed, 0)) {
        if (leader) drain();
        alive = false;
      }
      if (!alive) break;
      // E: the last P.V is complete.
      tc::bounded_wait(ws.mma_bar(), mma_phase, a.spin_limit, a.error, cxs::kErrCopyTimeout);
      mma_phase ^= 1;
      tc::fence_after();
      if (n_win > 0 && total == n_win) {
        float o[32];
        tc::combine_o(o_addr, half, o);
        const float den = l_run > 0.f ? l_run : 1.f;
#pragma unroll
        for (int i = 0; i < 16; ++i)
          win_packed[i] = cxs::pack_bf16(o[2 * i] / den, o[2 * i + 1] / den);
        l_run = 0.f;
      }
    }
    // Epilogue: lane writes dims 32 * half .. 32 * half + 31 of head (lane & 15).
    float o[32];
    if (total > n_win) {
      tc::combine_o(o_addr, half, o);
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) o[i] = 0.f;
    }
    const long long off = ((long long)row * 16 + (lane & 15)) * 64 + 32 * half;
    const float den = l_run > 0.f ? l_run : 1.f;
    const long long out_row = (long long)(row / a.H) * a.out_heads + a.out_head0 + row % a.H;
    const long long ooff = (out_row * 16 + (lane & 15)) * 64 + 32 * half;
    uint4* dst = reinterpret_cast<uint4*>(a.out + ooff);
    uint4* peer = a.out_peer ? reinterpret_cast<uint4*>(a.out_peer + ooff) : nullptr;
    if (!a.gate) {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t r[4];
#pragma unroll
        for (int e = 0; e < 4; ++e)
          r[e] = cxs::pack_bf16(bf16_round(o[8 * c + 2 * e] / den),
                                bf16_round(o[8 * c + 2 * e + 1] / den));
        dst[c] = make_uint4(r[0], r[1], r[2], r[3]);
        if (peer) peer[c] = make_uint4(r[0], r[1], r[2], r[3]);
      }
    } else {
      // Gate mix in the reference's bf16 rounding sequence (model.py:470-473).
      const __nv_bfloat16* gp = a.gates + ((long long)row * 16 + (lane & 15)) * 3;
      const float g0 = __bfloat162float(gp[0]), g1 = __bfloat162float(gp[1]),
                  g2 = __bfloat162float(gp[2]);
      const uint4* cmp = reinterpret_cast<const uint4*>(a.compressed + off);
      const bool have_window = a.window > 0 && pos >= 0;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const uint4 cv = cmp[c];
        const uint32_t* cp = reinterpret_cast<const uint32_t*>(&cv);
        uint32_t r[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 c2 = unpack_bf16(cp[e]);
          const float2 w2 = have_window ? unpack_bf16(win_packed[4 * c + e]) : make_float2(0.f, 0.f);
          float x0 = bf16_round(bf16_round(o[8 * c + 2 * e] / den) * g1);
          float x1 = bf16_round(bf16_round(o[8 * c + 2 * e + 1] / den) * g1);
          x0 = bf16_round(x0 + c2.x * g0);
          x1 = bf16_round(x1 + c2.y * g0);
          r[e] = cxs::pack_bf16(x0 + w2.x * g2, x1 + w2.y * g2);
        }
        dst[c] = make_uint4(r[0], r[1], r[2], r[3]);
        if (peer) peer[c] = make_uint4(r[0], r[1], r[2], r[3]);
      }
    }
    // Peer stores travel over NVLink: make them visible system-wide before
    // the exchange barrier that follows this launch announces them.
    if (peer) __threadfence_system();
    __syncwarp();  // TMEM reads done before the next row's MMAs
  }
}

// ------------------------------------------------------ IO + attention ---
// Warps 0-3: attention warps (tcgen05 engine, tile_tc.cuh), one query row at
// a time each. Warp 4: the IO warp.
template <int BS>
__global__ void __launch_bounds__(kThreads, 1)
    fetch_attend_kernel(const __grid_constant__ CUtensorMap kv_map,
                        const __grid_constant__ CUtensorMap win_map, AttendArgs a) {
  namespace tc = cxs::tc;
  constexpr int kBlockBytes = BS * kTokenBytes;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* io_buf = smem;
  uint8_t* q_tile = smem + ((kBlockBytes + 1023) & ~1023);
  uint8_t* p_tile = q_tile + tc::kRowTileBytes;
  uint8_t* warps_base = p_tile + tc::kRowTileBytes;
  uint8_t* ctrl = warps_base + kAttnWarps * tc::WarpSmem::kBytes;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ctrl);
  uint64_t* io_bar = reinterpret_cast<uint64_t*>(ctrl + 64);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    cxs::mbar_init(io_bar, 1);
    for (int w = 0; w < kAttnWarps; ++w) {
      tc::WarpSmem ws{warps_base + w * tc::WarpSmem::kBytes};
      for (int b = 0; b < 2; ++b) {
        cxs::mbar_init(ws.kbar(b), 1);
        cxs::mbar_init(ws.vbar(b), 1);
      }
      cxs::mbar_init(ws.mma_bar(), 1);
    }
    cxs::fence_mbar_init();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     cxs::smem_addr(tmem_slot)),
                 "r"(kTmemAlloc));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  // Zero the P tile (each lane only ever writes its own half of its row) and
  // the K/V stages (rows beyond a short block, BS < 64, start at zero and
  // afterwards only hold finite key/value data).
  if (warp < kAttnWarps) {
    for (int i = threadIdx.x; i < tc::kRowTileBytes / 16; i += 32 * kAttnWarps)
      reinterpret_cast<uint4*>(p_tile)[i] = make_uint4(0, 0, 0, 0);
    for (int w = 0; w < kAttnWarps; ++w)
      for (int i = threadIdx.x; i < 4 * tc::kTileBytes / 16; i += 32 * kAttnWarps)
        reinterpret_cast<uint4*>(warps_base + w * tc::WarpSmem::kBytes)[i] =
            make_uint4(0, 0, 0, 0);
  }
  cxs::fence_proxy_async_shared();
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == kAttnWarps) {
    // ------------------------------------------------------------ IO warp
    uint64_t* bar = io_bar;
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
          cxs::mbar_expect_tx(bar, kBlockBytes);
          cxs::bulk_g2s(io_buf, src, kBlockBytes, bar);
          if (cxs::mbar_wait_bounded(bar, phase, a.spin_limit, a.error)) {
            cxs::bulk_s2g_and_wait(dst, io_buf, kBlockBytes);
          } else {
            cxs::mbar_wait_bounded(bar, phase, a.spin_limit, a.error);
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
  } else {
    attention_warp<BS>(kv_map, win_map, a, q_tile, p_tile, warps_base + warp * tc::WarpSmem::kBytes,
                       warp, tmem_base + warp * tc::kTmemCols);
  }
  // All warps (IO included) meet before the TMEM columns are released.
  tc::fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(kTmemAlloc));
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
  cuuint32_t box[3] = {64, 1, 64};  // window tiles are always 64 records
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
  size_t tiles = 2 * (size_t)cxs::tc::kRowTileBytes;
  size_t warps = (size_t)kAttnWarps * cxs::tc::WarpSmem::kBytes;
  return 1024 + io + tiles + warps + 128;
}

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
  if (g.ctas > 0 && g.ctas < grid) grid = g.ctas;
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
  a.seg_start = (int)g.segment_start;
  a.seg_tokens = (int)g.segment_tokens;
  a.spin_limit = g.spin_limit > 0 ? g.spin_limit : (1ll << 31);
  a.consumers = grid * kAttnWarps;
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
  a.out_peer = (__nv_bfloat16*)b.out_peer;
  a.out_heads = g.out_heads > 0 ? g.out_heads : g.heads;
  a.out_head0 = g.out_heads > 0 ? g.out_head0 : 0;

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
  if (g.width > 32)
    return set_error(CXS_ERR_INVALID, "width (top-n) must be at most 32");
  if (g.window < 0 || (g.window > 0 && (!b.window_kv || g.window_len < 1)))
    return set_error(CXS_ERR_INVALID, "window branch needs a window buffer");
  // window_start may be negative: records before position 0 are padding that
  // no window reaches (a window never starts below position 0).
  if (g.window > 0 && (g.window_start < -(long long)g.window_len ||
                       g.window_start + g.window_len > INT32_MAX))
    return set_error(CXS_ERR_INVALID, "window positions must fit int32");
  if (g.segment_tokens < 0 || g.segment_start < 0 ||
      (g.segment_tokens > 0 &&
       (g.segment_start % g.block_size || g.segment_tokens % g.block_size ||
        g.segment_start + (long long)g.segment_tokens * g.queries > INT32_MAX)))
    return set_error(CXS_ERR_INVALID,
                     "segment_start / segment_tokens must be block multiples and fit int32");
  if (g.gate && (!b.compressed || !b.gates))
    return set_error(CXS_ERR_INVALID, "gate mix needs compressed output and gates");
  if (((uintptr_t)b.kv & 15) || ((uintptr_t)b.query & 15) || ((uintptr_t)b.out & 15))
    return set_error(CXS_ERR_INVALID, "kv/query/out must be 16-byte aligned");
  if (g.window > 0 && ((uintptr_t)b.window_kv & 15))
    return set_error(CXS_ERR_INVALID, "window buffer must be 16-byte aligned");
  if (g.out_heads < 0 || (g.out_heads > 0 && (g.out_head0 < 0 ||
                                              g.out_head0 + g.heads > g.out_heads)))
    return set_error(CXS_ERR_INVALID, "output heads must hold this call's heads");
  if ((uintptr_t)b.out_peer & 15) return set_error(CXS_ERR_INVALID, "out_peer must be 16-byte aligned");
  if (g.ctas < 0) return set_error(CXS_ERR_INVALID, "ctas must be >= 0 (0: every SM)");
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
static_assert(kScratchBytes == 16ull * CXS_NOALLOC_MAX_PHYSICAL + 256,
              "scratch layout: 8 + 4 + 4 bytes per block plus the 256-byte control word area");

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
