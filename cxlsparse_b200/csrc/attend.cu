// Block-source preparation and the persistent IO + attention kernel.
//
// Reference behaviour: tma/transport.py:17-112 (_prepare_sources, execute)
// and the staged TMA kernel tma/pipeline.py:96-742 (IO CTAs :347-421,
// consumer CTAs :436-655, online-softmax block step :172-257). This is a new
// sm_100a design: one cooperative launch whose CTAs each run one IO warp and
// four tcgen05 attention warps; see cxs_fetch_attend in include/cxlsparse.h.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <climits>
#include <mutex>

#include "cxs_common.cuh"
#include "tile_tc.cuh"

using cxs::kTokenBytes;
using cxs::bf16_round;
using cxs::unpack_bf16;
using cxs_host::set_error;

namespace {

constexpr int kAttnWarps = cxs::tc::kEngines;     // engines (warp pairs) per CTA
constexpr int kTmemAlloc = kAttnWarps * cxs::tc::kTmemCols;  // 512: all of TMEM
constexpr int kIoWarp = 2 * kAttnWarps;           // warps 0-3 softmax, 4-7 engine, 8 IO
constexpr int kThreads = 32 * (kIoWarp + 1);
// Host-link requests kept in flight by the IO warps of a launch. Every IO
// warp has one block copy outstanding, and the link shares its bandwidth
// among them, so a block arrives after about (IO warps x block bytes) /
// bandwidth. Far above the link's bandwidth-delay product (about 110 KB at
// 55 GB/s and 2 us), more warps only delay the first blocks of the
// consumption order, which the attention warps wait on. Measured at
// H=16384 / E=256 / BS=64 on one B200: 37 IO warps (this budget) take the
// 16-layer step from 4.80 to 4.68 ms against one IO warp per SM; 17 are
// slower again (mixed-source gathers need the warps).
constexpr int kIoInflightBytes = 512 * 1024;

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
  const int32_t* first_depth;  // read-order key of every block, or NULL (list order)
  const int32_t* near;
  int32_t* ready;
  int32_t* control;
  int32_t* error;
  const __nv_bfloat16* compressed;
  const __nv_bfloat16* gates;
  __nv_bfloat16* out;
  __nv_bfloat16* out_peer;  // optional second copy of every output row (a peer GPU's buffer)
  int out_heads, out_head0;  // output row of (q, h): q * out_heads + out_head0 + h
  int io_stride;             // CTAs whose blockIdx.x is a multiple of this run the IO loop
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

// ------------------------------------------------------- attention pairs ---
// One engine (a warp pair, tile_tc.cuh) per query row at a time: rows
// e * gridDim.x + blockIdx.x + k * consumers for engine e of the CTA. Per row
// the sliding-window tiles come first, then the row's selected occurrences
// by the plan's read-order key (duplicates attended again, as the reference
// does); the softmax warp writes the (gate-mixed) output.

// Tiles of one query row, computed alike by both warps of an engine.
// Position of this lane's selected occurrence in its row's processing order:
// by the plan's read-order key (first consumption depth, more near consumers
// first, block), the key the IO warps fetch missing blocks by, so that an
// engine takes its blocks in the order they arrive; equal keys keep list
// order. The plan gives every block this key whatever its residency, so the
// order (and the result) does not depend on which blocks are resident or on
// arrival times. Without the key (NULL) the order is the list order. Lanes at
// or beyond `count` keep their own slot. The key packs depth (24 bits),
// near consumers (16 bits, inverted) and block (24 bits); a field beyond its
// width saturates, which still gives one fixed order.
struct SlotFields {
  int depth = -1, near = 0, block = 0;  // depth -1: no key (list order)
};

__device__ __forceinline__ SlotFields slot_fields(const AttendArgs& a, int block) {
  SlotFields f;
  if (a.first_depth && block >= 0 && block < a.P) {
    f.depth = a.first_depth[block];
    f.near = a.near ? a.near[block] : 0;
    f.block = block;
  }
  return f;
}

__device__ __forceinline__ unsigned long long slot_key(SlotFields f) {
  if (f.depth < 0) return 0ull;
  const unsigned long long depth = (unsigned)min(f.depth, 0xffffff);
  const unsigned long long near = (unsigned)min(max(f.near, 0), 0xffff);
  return depth << 40 | (0xffffull - near) << 24 | (unsigned)min(f.block, 0xffffff);
}

__device__ __forceinline__ int process_slot(unsigned long long key, int count, int lane) {
  int slot = 0;
#pragma unroll 4
  for (int j = 0; j < count; ++j) {
    const unsigned long long kj = __shfl_sync(0xffffffffu, key, j);
    slot += kj < key || (kj == key && j < lane);
  }
  return lane < count ? slot : lane;
}

struct RowTiles {
  int h, pos, count, n_hist, n_win, total;
  int w_lo, w_hi, o_lo, o_hi;
  // First and last position of window tile j.
  __device__ __forceinline__ int win_first(int j) const {
    return j < n_hist ? w_lo + j * cxs::tc::kTileRows : o_lo + (j - n_hist) * cxs::tc::kTileRows;
  }
  __device__ __forceinline__ int win_last(int j) const { return j < n_hist ? w_hi : o_hi; }
};

// Window: positions [w_lo, w_hi], then [o_lo, o_hi] (positions and window
// bounds fit int32: host-checked), each in tiles of 64 from its start. With
// candidate segments, a row of segment s sees the history below seg_start,
// then its own segment, which starts at seg_start + s * seg_tokens (true
// position = seg_start + offset into the segment); every segment row splits
// its window there, whatever s, so that a candidate's tiles (and roundings)
// do not depend on its segment index. Without segments the window is one
// contiguous range.
__device__ __forceinline__ RowTiles row_tiles(const AttendArgs& a, int row) {
  RowTiles r;
  r.h = row % a.H;
  r.pos = a.row_positions[row];
  r.w_lo = 1, r.w_hi = 0, r.o_lo = 1, r.o_hi = 0;
  if (a.window > 0 && r.pos >= 0) {
    const int pos = r.pos;
    const int w_first = (int)a.window_start, w_last = w_first + a.window_len - 1;
    int own = -1, real = pos;
    if (a.seg_tokens > 0 && pos >= a.seg_start) {
      own = a.seg_start + (pos - a.seg_start) / a.seg_tokens * a.seg_tokens;
      real = a.seg_start + (pos - own);
    }
    r.w_lo = max(max(real - a.window + 1, 0), w_first);
    if (own < 0) {
      r.w_hi = min(pos, w_last);
    } else {
      r.w_hi = min(a.seg_start - 1, w_last);
      r.o_lo = max(own + max(real - a.window + 1 - a.seg_start, 0), w_first);
      r.o_hi = min(pos, w_last);
    }
  }
  constexpr int kRows = cxs::tc::kTileRows;
  r.n_hist = r.w_lo <= r.w_hi ? (r.w_hi - r.w_lo) / kRows + 1 : 0;
  r.n_win = r.n_hist + (r.o_lo <= r.o_hi ? (r.o_hi - r.o_lo) / kRows + 1 : 0);
  r.count = r.pos >= 0 ? min(a.all_counts[row], a.W) : 0;
  r.total = r.n_win + r.count;
  return r;
}

// Engine warp: copies and MMAs of its engine's rows, issued by lane 0.
//   K of tile j goes to K buffer (j mod 3) once S of tile j - 3 has been read
//   (the softmax warp's "S read" arrival), at most two tiles ahead; a
//   selected block's copy needs its ready flag (skipped for blocks resident
//   before the launch, kind 0), polled with relaxed loads issued one tile
//   early and made an acquire by a fence once seen set.
//   V of tile j goes to V buffer (j mod 2) once P.V of tile j - 2 is done.
//   Per tile t: wait "S(t - 1) read", issue S(t) (commit: sbar), then wait
//   "P(t - 1) written" and issue O (+)= P.V(t - 1) (commit: obar), then
//   start V(t) (P.V(t - 2) was issued a tile earlier, so rarely waited for).
// Every wait is bounded; a timeout or the partner's abort ends the launch
// for the engine after its copies and MMAs in flight have drained.
template <int BS>
__device__ __forceinline__ void engine_warp(const CUtensorMap& kv_map, const CUtensorMap& win_map,
                                            const AttendArgs& a, const uint8_t* q_tile,
                                            const uint8_t* p_tile, const cxs::tc::PairSmem ps,
                                            int e, uint32_t tmem) {
  namespace tc = cxs::tc;
  const int lane = threadIdx.x % 32;
  const uint32_t s_col = tmem, o_col = tmem + 64;
  const uint32_t id_s = tc::idesc_bf16(128, 64, 0, 0), id_o = tc::idesc_bf16(128, 64, 0, 1);
  const uint32_t q_addr = cxs::smem_addr(q_tile), p_addr = cxs::smem_addr(p_tile);
  volatile int* abort = ps.abort_flag();
  const long long spin = a.spin_limit;
  if (lane == 0) {
    cxs::tma_prefetch_desc(&kv_map);
    if (a.window) cxs::tma_prefetch_desc(&win_map);
  }
  // Running counts over the engine's rows: K / V copies started and landed
  // (buffer = count mod 3 / mod 2, phase bit per buffer), P.V issued and
  // seen complete, barrier phases of the softmax warp's arrivals.
  int k_started = 0, k_landed = 0, v_started = 0, v_landed = 0, pv_issued = 0, pv_seen = 0;
  uint32_t k_phase = 0, v_phase = 0, sfree_phase = 0, pfull_phase = 0;
  bool failed = false, first_row = true;
  const int rows = a.Q * a.H;
  for (int row = e * gridDim.x + blockIdx.x; row < rows && !failed; row += a.consumers) {
    const RowTiles rt = row_tiles(a, row);
    {  // stage the row's selected blocks and their source kinds, in processing order
      int block = -1, kind = 0;
      if (lane < rt.count) {
        block = a.all_ids[(long long)row * a.W + lane];
        if (block >= 0 && block < a.P) kind = a.kinds[block];
      }
      const int slot = process_slot(slot_key(slot_fields(a, block)), rt.count, lane);
      ps.blocks()[slot] = block;
      ps.kinds()[slot] = kind;
    }
    __syncwarp();
    if (lane == 0 && rt.total > 0) {
      const int total = rt.total, n_win = rt.n_win, h = rt.h;
      const int k0 = k_started, v0 = v_started;  // this row's tile j: K copy k0 + j, V copy v0 + j
      const int count = rt.count;
      auto block_of = [&](int j) { return ps.blocks()[j - n_win]; };
      // Selected occurrences [0, acq) are acquired (or resident). The ready
      // flags of the next kProbe are read with relaxed loads a tile before
      // they are needed (probe_base: first of them, -1: none pending); a
      // run of them seen set becomes an acquire with one fence.
      constexpr int kProbe = 4;
      int acq = 0, probe_base = -1;
      int probe[kProbe];
      auto take_probe = [&]() {
        if (probe_base < 0) return;
        bool cold = false;
        while (acq < count) {
          const int i = acq - probe_base;
          if (ps.kinds()[acq] == 0) {
            ++acq;
            continue;
          }
          bool seen = false;
#pragma unroll
          for (int q = 0; q < kProbe; ++q) seen |= q == i && probe[q] != 0;
          if (!seen) break;
          ++acq;
          cold = true;
        }
        probe_base = -1;
        if (cold) {
          cxs::fence_acq_rel_gpu();
          cxs::fence_proxy_async_global();
        }
      };
      auto issue_probe = [&]() {
        if (probe_base >= 0 || acq >= count) return;
        probe_base = acq;
#pragma unroll
        for (int q = 0; q < kProbe; ++q) {
          const int o = acq + q;
          const int block = o < count ? ps.blocks()[o] : -1;
          probe[q] = 0;
          if (block >= 0 && block < a.P && ps.kinds()[o] != 0)
            probe[q] = cxs::ld_relaxed(&a.ready[block]);
        }
      };
      auto copy = [&](int j, bool value) {
        const int b = value ? (v0 + j) % tc::PairSmem::kVBufs : (k0 + j) % tc::PairSmem::kKBufs;
        uint64_t* bar = value ? ps.vbar(b) : ps.kbar(b);
        uint8_t* dst = value ? ps.v(b) : ps.k(b);
        if (j < n_win) {
          cxs::mbar_expect_tx(bar, tc::kTileBytes);
          tc::window_load(dst, &win_map, value ? 64 : 0, h, rt.win_first(j) - (int)a.window_start,
                          bar);
        } else {
          cxs::mbar_expect_tx(bar, BS * 128);
          cxs::tma_load_2d(dst, &kv_map, value ? 64 : 0, block_of(j) * BS, bar);
        }
      };
      // Start K copies of tiles up to `upto`; tile `need` (and any before it)
      // must start now, waiting (bounded) for its ready flag.
      auto start_k = [&](int upto, int need) -> bool {
        while (k_started - k0 <= upto && k_started - k0 < total) {
          const int j = k_started - k0;
          if (j >= n_win) {
            const int o = j - n_win, block = block_of(j);
            if (block < 0 || block >= a.P) {
              atomicOr(a.error, cxs::kErrBadBlock);
              return false;
            }
            // Every earlier occurrence has started, so acq >= o here.
            if (o >= acq) take_probe();
            while (acq < count && acq <= o && ps.kinds()[acq] == 0) ++acq;
            if (o >= acq) {
              if (j > need) break;  // not known ready: retry at the next tile
              if (!cxs::wait_ready_bounded(&a.ready[block], spin, a.error)) return false;
              cxs::fence_proxy_async_global();
              acq = o + 1;
            }
          }
          copy(j, false);
          ++k_started;
        }
        return true;
      };
      // Start V copies of tiles up to `upto` whose K copy has started (its
      // block is ready); V buffer reuse waits for the P.V two copies back.
      auto start_v = [&](int upto) -> bool {
        while (v_started - v0 <= upto && v_started < k_started) {
          const int need_done = v_started - 1;  // P.V of V copy v_started - 2 complete
          while (pv_seen < need_done) {
            if (!tc::pair_wait(ps.obar(), pv_seen & 1, abort, spin, a.error, cxs::kErrCopyTimeout))
              return false;
            ++pv_seen;
          }
          copy(v_started - v0, true);
          ++v_started;
        }
        return true;
      };
      auto land = [&](bool value) -> bool {
        int& done = value ? v_landed : k_landed;
        uint32_t& phase = value ? v_phase : k_phase;
        const int b = value ? done % tc::PairSmem::kVBufs : done % tc::PairSmem::kKBufs;
        const bool ok = tc::pair_wait(value ? ps.vbar(b) : ps.kbar(b), (phase >> b) & 1u, abort,
                                      spin, a.error, cxs::kErrCopyTimeout);
        phase ^= 1u << b;
        ++done;
        return ok;
      };
      auto softmax_arrival = [&](uint64_t* bar, uint32_t& phase) -> bool {
        const bool ok = tc::pair_wait(bar, phase, abort, spin, a.error, cxs::kErrReadyTimeout);
        phase ^= 1u;
        return ok;
      };
      // O (+)= P . V(j). Every earlier P.V is seen complete first (one was
      // issued a tile ago), so the engine's count of obar phases never lags
      // two behind, which a parity wait could not tell apart.
      auto issue_pv = [&](int j) -> bool {
        while (pv_seen < pv_issued) {
          if (!tc::pair_wait(ps.obar(), pv_seen & 1, abort, spin, a.error, cxs::kErrCopyTimeout))
            return false;
          ++pv_seen;
        }
        const uint32_t va = cxs::smem_addr(ps.v((v0 + j) % tc::PairSmem::kVBufs));
        const bool accumulate = !(j == 0 || j == n_win);
        tc::fence_after();
#pragma unroll
        for (int k = 0; k < 4; ++k)
          tc::mma(o_col, tc::desc_sw128(p_addr + 32 * k, 16, 1024),
                  tc::desc_sw128(va + 2048 * k, 16, 1024), id_o, accumulate || k > 0);
        tc::commit(ps.obar());
        ++pv_issued;
        return true;
      };
      // Previous rows are complete (the softmax warp has written this row's
      // Q after its last epilogue), so every buffer is free: P.V seen.
      bool ok = true;
      if (!first_row) ok = softmax_arrival(ps.sfree(), sfree_phase);  // this row's Q written
      pv_seen = pv_issued;
      ok = ok && start_k(2, 0) && start_v(0);
      if (ok && first_row) ok = softmax_arrival(ps.sfree(), sfree_phase);
      first_row = false;
      for (int t = 0; t < total && ok; ++t) {
        if (t > 0) ok = softmax_arrival(ps.sfree(), sfree_phase);  // S(t - 1) read
        ok = ok && start_k(t + 2, t) && land(false);  // K(t)
        if (!ok) break;
        {  // S = Q . K(t)^T
          const uint32_t ka = cxs::smem_addr(ps.k((k0 + t) % tc::PairSmem::kKBufs));
          tc::fence_after();
#pragma unroll
          for (int k = 0; k < 4; ++k)
            tc::mma(s_col, tc::desc_sw128(q_addr + 32 * k, 16, 1024),
                    tc::desc_sw128(ka + 32 * k, 16, 1024), id_s, k);
          tc::commit(ps.sbar());
        }
        if (t > 0) {
          ok = softmax_arrival(ps.pfull(), pfull_phase) && land(true)  // P(t-1), V(t-1)
               && issue_pv(t - 1);
        }
        // V(t): its buffer's last P.V (tile t - 2) was issued a tile ago.
        ok = ok && start_v(t);
        // Poll the next ready flags now; they are read at the next tile,
        // after their latency has passed.
        if (ok) issue_probe();
      }
      if (ok) {
        ok = start_v(total - 1) && softmax_arrival(ps.pfull(), pfull_phase) && land(true) &&
             issue_pv(total - 1);
      }
      if (!ok) {
        *abort = 1;
        failed = true;
      }
    }
    __syncwarp();
    failed = __shfl_sync(0xffffffffu, failed, 0);
  }
  if (lane == 0) {
    // Let every copy this engine started land, and every MMA it issued
    // complete, before the CTA releases shared memory and TMEM (bounded).
    while (k_landed < k_started) {
      const int b = k_landed % tc::PairSmem::kKBufs;
      tc::bounded_wait(ps.kbar(b), (k_phase >> b) & 1u, spin, a.error, cxs::kErrCopyTimeout);
      k_phase ^= 1u << b;
      ++k_landed;
    }
    while (v_landed < v_started) {
      const int b = v_landed % tc::PairSmem::kVBufs;
      tc::bounded_wait(ps.vbar(b), (v_phase >> b) & 1u, spin, a.error, cxs::kErrCopyTimeout);
      v_phase ^= 1u << b;
      ++v_landed;
    }
    tc::commit(ps.drain());
    tc::bounded_wait(ps.drain(), 0, spin, a.error, cxs::kErrCopyTimeout);
  }
}

// Softmax warp: S tiles of its engine's rows from TMEM, online softmax, P to
// shared memory, O rescale, and the epilogue (normalisation, gate mix,
// output rows; lane writes dims 32 * half .. 32 * half + 31 of head
// (lane & 15)).
template <int BS>
__device__ __forceinline__ void softmax_warp(const AttendArgs& a, uint8_t* q_tile,
                                             uint8_t* p_tile, const cxs::tc::PairSmem ps, int e,
                                             uint32_t tmem) {
  namespace tc = cxs::tc;
  const int lane = threadIdx.x % 32, half = lane >> 4;
  const bool leader = lane == 0;
  const int m = 32 * e + lane;  // this lane's row of the Q / P tiles and of S / O
  const uint32_t lane_off = (uint32_t)(32 * e) << 16;
  const uint32_t s_addr = tmem + lane_off, o_addr = tmem + 64 + lane_off;
  volatile int* abort = ps.abort_flag();
  const long long spin = a.spin_limit;
  uint32_t s_phase = 0, o_phase = 0;
  const int rows = a.Q * a.H;
  auto agree_wait = [&](uint64_t* bar, uint32_t& phase) -> bool {
    bool ok = tc::pair_wait(bar, phase, abort, spin, a.error, cxs::kErrCopyTimeout);
    phase ^= 1u;
    ok = __all_sync(0xffffffffu, ok);
    tc::fence_after();
    return ok;
  };
  for (int row = e * gridDim.x + blockIdx.x; row < rows; row += a.consumers) {
    // The query row first (its loads do not depend on the plan's tables), so
    // the engine can start S(0) as soon as its first K tile lands.
    tc::write_query_row(q_tile, a.query, row, m, lane);
    const RowTiles rt = row_tiles(a, row);
    const int total = rt.total, n_win = rt.n_win, pos = rt.pos;
    // Lane i holds selected occurrence i's block, first position and slot in
    // the processing order (the engine warp computes the same slots).
    int my_block = -1, my_start = 0;
    if (lane < rt.count) {
      my_block = a.all_ids[(long long)row * a.W + lane];
      if (my_block >= 0 && my_block < a.P) my_start = a.starts[my_block];
    }
    cxs::fence_proxy_async_shared();
    __syncwarp();
    if (total > 0 && leader) cxs::mbar_arrive(ps.sfree());  // Q written
    // The order is first needed at the first selected tile, after the window.
    const int my_slot = process_slot(slot_key(slot_fields(a, my_block)), rt.count, lane);
    float m_run = -INFINITY, l_run = 0.f;
    uint32_t win_packed[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) win_packed[i] = 0;
    auto window_output = [&](float l_win) {  // normalised bf16 output of the window branch
      float o[32];
      tc::combine_o(o_addr, half, o);
      const float den = l_win > 0.f ? l_win : 1.f;
#pragma unroll
      for (int i = 0; i < 16; ++i) win_packed[i] = cxs::pack_bf16(o[2 * i] / den, o[2 * i + 1] / den);
    };
    bool alive = true;
    for (int t = 0; t < total; ++t) {
      const bool first_of_branch = t == 0 || t == n_win;
      if (!agree_wait(ps.sbar(), s_phase)) {  // S(t)
        alive = false;
        break;
      }
      float sv[32];
      tc::load_s(s_addr, half, sv);
      tc::fence_before();
      __syncwarp();
      if (t + 1 < total && leader) cxs::mbar_arrive(ps.sfree());  // S(t) read
      const float l_prev = l_run;
      if (t == n_win && n_win > 0) {  // window branch complete: the selected branch restarts
        m_run = -INFINITY;
        l_run = 0.f;
      }
      int lo = 0, hi = -1;
      if (t < n_win) {
        hi = min(rt.win_last(t) - rt.win_first(t), tc::kTileRows - 1);
      } else {
        const uint32_t holder = __ballot_sync(0xffffffffu, my_slot == t - n_win);
        const int src = holder ? __ffs(holder) - 1 : 0;
        const int cur_block = __shfl_sync(0xffffffffu, my_block, src);
        const int cur_start = __shfl_sync(0xffffffffu, my_start, src);
        if (holder && cur_block >= 0 && cur_block < a.P) hi = min(pos - cur_start, BS - 1);
      }
      const float m_old = m_run;
      const float factor = tc::softmax_regs(sv, lo, hi, m_run, l_run, half);
      // P.V(t - 1) runs under the softmax above; it must be done before P(t)
      // overwrites the P tile, O is rescaled or the window branch's O is read.
      if (t > 0 && !agree_wait(ps.obar(), o_phase)) {
        alive = false;
        break;
      }
      if (t == n_win && n_win > 0) window_output(l_prev);  // keep the window branch's output
      if (!first_of_branch) tc::rescale_o(o_addr, factor, m_old != -INFINITY && factor != 1.f);
      tc::store_p(p_tile, m, half, sv);
      cxs::fence_proxy_async_shared();
      tc::fence_before();
      __syncwarp();
      if (leader) cxs::mbar_arrive(ps.pfull());  // P(t) written
    }
    if (!alive) break;
    // The gate-mix inputs load while the last P.V completes.
    const long long off = ((long long)row * 16 + (lane & 15)) * 64 + 32 * half;
    float g0 = 0.f, g1 = 0.f, g2 = 0.f;
    uint4 cmp[4];
    if (a.gate) {
      const __nv_bfloat16* gp = a.gates + ((long long)row * 16 + (lane & 15)) * 3;
      g0 = __bfloat162float(gp[0]);
      g1 = __bfloat162float(gp[1]);
      g2 = __bfloat162float(gp[2]);
      const uint4* src = reinterpret_cast<const uint4*>(a.compressed + off);
#pragma unroll
      for (int c = 0; c < 4; ++c) cmp[c] = src[c];
    }
    if (total > 0) {
      if (!agree_wait(ps.obar(), o_phase)) break;  // the last P.V
      if (total == n_win && n_win > 0) {
        window_output(l_run);
        l_run = 0.f;
      }
    }
    float o[32];
    if (total > n_win) {
      tc::combine_o(o_addr, half, o);
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) o[i] = 0.f;
    }
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
        for (int q = 0; q < 4; ++q)
          r[q] = cxs::pack_bf16(bf16_round(o[8 * c + 2 * q] / den),
                                bf16_round(o[8 * c + 2 * q + 1] / den));
        dst[c] = make_uint4(r[0], r[1], r[2], r[3]);
        if (peer) peer[c] = make_uint4(r[0], r[1], r[2], r[3]);
      }
    } else {
      // Gate mix in the reference's bf16 rounding sequence (model.py:470-473).
      const bool have_window = a.window > 0 && pos >= 0;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const uint4 cv = cmp[c];
        const uint32_t* cp = reinterpret_cast<const uint32_t*>(&cv);
        uint32_t r[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 c2 = unpack_bf16(cp[q]);
          const float2 w2 = have_window ? unpack_bf16(win_packed[4 * c + q]) : make_float2(0.f, 0.f);
          float x0 = bf16_round(bf16_round(o[8 * c + 2 * q] / den) * g1);
          float x1 = bf16_round(bf16_round(o[8 * c + 2 * q + 1] / den) * g1);
          x0 = bf16_round(x0 + c2.x * g0);
          x1 = bf16_round(x1 + c2.y * g0);
          r[q] = cxs::pack_bf16(x0 + w2.x * g2, x1 + w2.y * g2);
        }
        dst[c] = make_uint4(r[0], r[1], r[2], r[3]);
        if (peer) peer[c] = make_uint4(r[0], r[1], r[2], r[3]);
      }
    }
    // Peer stores travel over NVLink: make them visible system-wide before
    // the exchange barrier that follows this launch announces them.
    if (peer) __threadfence_system();
    tc::fence_before();  // TMEM reads done before the next row's MMAs
    __syncwarp();
  }
}

// ------------------------------------------------------ IO + attention ---
// Warps 0-3: softmax warps, warps 4-7: engine warps (warp w + 4 serves
// softmax warp w; tcgen05 engines of tile_tc.cuh, one query row at a time
// each). Warp 8: the IO warp.
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
  uint8_t* pairs_base = p_tile + tc::kRowTileBytes;
  uint8_t* ctrl = pairs_base + kAttnWarps * tc::PairSmem::kBytes;
  auto pair = [&](int e) { return tc::PairSmem{pairs_base + e * tc::PairSmem::kBytes}; };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ctrl);
  uint64_t* io_bar = reinterpret_cast<uint64_t*>(ctrl + 64);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    cxs::mbar_init(io_bar, 1);
    for (int e = 0; e < kAttnWarps; ++e) {
      for (int i = 0; i < tc::PairSmem::kNumBars; ++i) cxs::mbar_init(pair(e).bar(i), 1);
      *pair(e).abort_flag() = 0;
    }
    cxs::fence_mbar_init();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     cxs::smem_addr(tmem_slot)),
                 "r"(kTmemAlloc));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  // Zero the P tile (each lane only ever writes its own half of its row) and,
  // for blocks shorter than a tile (BS < 64), the K/V stages: the rows beyond
  // such a block start at zero and afterwards only hold finite key/value data.
  if (warp < kIoWarp) {
    constexpr int kStaged = tc::PairSmem::kKBufs + tc::PairSmem::kVBufs;
    for (int i = threadIdx.x; i < tc::kRowTileBytes / 16; i += 32 * kIoWarp)
      reinterpret_cast<uint4*>(p_tile)[i] = make_uint4(0, 0, 0, 0);
    if (BS < tc::kTileRows)
      for (int e = 0; e < kAttnWarps; ++e)
        for (int i = threadIdx.x; i < kStaged * tc::kTileBytes / 16; i += 32 * kIoWarp)
          reinterpret_cast<uint4*>(pair(e).base)[i] = make_uint4(0, 0, 0, 0);
  }
  cxs::fence_proxy_async_shared();
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == kIoWarp) {
    if (blockIdx.x % a.io_stride == 0) {
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
    }
  } else {
    const int e = warp % kAttnWarps;
    if (warp < kAttnWarps)
      softmax_warp<BS>(a, q_tile, p_tile, pair(e), e, tmem_base + e * tc::kTmemCols);
    else
      engine_warp<BS>(kv_map, win_map, a, q_tile, p_tile, pair(e), e, tmem_base + e * tc::kTmemCols);
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
  size_t warps = (size_t)kAttnWarps * cxs::tc::PairSmem::kBytes;
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
  // IO warps on every io_stride-th CTA, spread over the grid: about
  // kIoInflightBytes of block copies in flight (IO ranks come from an atomic
  // cursor, so any number of IO warps fetches every block).
  const int io_ctas = std::max(1, kIoInflightBytes / (BS * kTokenBytes));
  a.io_stride = std::max(1, grid / io_ctas);
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
  a.first_depth = b.first_depth;
  a.near = b.near_consumers;
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
