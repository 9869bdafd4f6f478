// Device-side fetch planner for the NSA GR selected-block path.
//
// Deduplicating plan: planning/active.py:21-500, 670-907 (reference).
// Query-private plan: planning/query_private.py:29-216, 258-457.
// Occurrence rows: planning/occurrences.py:7-35.
// Consumption-depth read order: planning/dependencies.py:37-300.
//
// Every launch only enqueues work on the caller's stream (graph-capturable),
// uses fixed-size caller buffers and never downloads data to the host.
#include <cub/block/block_radix_sort.cuh>
#include <cub/block/block_reduce.cuh>
#include <cub/block/block_scan.cuh>

#include "cxs_common.cuh"

using cxs::kInt32Max;
using cxs::kTokenBytes;
using cxs_host::set_error;

namespace {

constexpr int kNearWindow = 4;  // planning/dependencies.py:14
constexpr int kMaxMapBlocks = 1 << 18;  // bitmap compaction limit (32 KiB of shared memory)
constexpr int kMaxPhysical = 16384;     // single-CTA publish sort limit
constexpr int kMaxHot = 4096;           // shared-memory hot hash / hot sort limit

struct Geo {
  int Q, H, W, BS, MAP, CAP, SORT, HOT, MAXH, REGIONS, PAGE, CONSUMERS, ORDER, PRIVATE, MODE;
  int HASH, P, R;
  int PAGE_SHIFT, REGION_SHIFT;  // log2 of PAGE / REGIONS when powers of two, else -1
  long long POOL;
};

// Backing-pool address of token slot `source` (>= 0): page source / PAGE,
// pages striped round-robin over the regions (mempool/cxl.py:110-113).
// Shifts and masks replace the 64-bit division when PAGE / REGIONS are
// powers of two; the values are the same.
__device__ __forceinline__ long long pool_address(const Geo& g, const int64_t* bases,
                                                  long long source, int* region_out) {
  long long page, offset, local_page;
  int region;
  if (g.PAGE_SHIFT >= 0) {
    page = source >> g.PAGE_SHIFT;
    offset = source & (g.PAGE - 1);
  } else {
    page = source / g.PAGE;
    offset = source % g.PAGE;
  }
  if (g.REGION_SHIFT >= 0) {
    region = (int)(page & (g.REGIONS - 1));
    local_page = page >> g.REGION_SHIFT;
  } else {
    region = (int)(page % g.REGIONS);
    local_page = page / g.REGIONS;
  }
  *region_out = region;
  return bases[region] + (local_page * g.PAGE + offset) * kTokenBytes;
}

__device__ __forceinline__ bool occurrence_valid(int block, int pos, int total, const Geo& g) {
  return pos >= 0 && block >= 0 && block < g.MAP && (long long)block * g.BS <= pos &&
         (long long)block * g.BS < total;
}

// ------------------------------------------------------------------ reset ---
// Scratch fills (active.py:21-53) plus clearing the mapping entries named by
// this request (active.py:56-77). No read-after-write dependency inside.
__global__ void reset_kernel(Geo g, cxs_plan_buffers b, int max_depth) {
  long long tid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  long long stride = (long long)gridDim.x * blockDim.x;
  long long hc = (long long)g.H * g.CAP;
  long long hs = (long long)g.H * g.SORT;
  long long rw = (long long)g.R * g.W;
  for (long long i = tid; i < hc; i += stride) {
    b.required[i] = 0;
    b.insert_keys[i] = kInt32Max;
    if (g.PRIVATE) b.private_required[i] = 0;
  }
  for (long long i = tid; i < hs; i += stride) {
    b.frequencies[i] = 0;
    if (g.PRIVATE) b.canonical[i] = kInt32Max;
  }
  for (long long i = tid; i < rw; i += stride) b.all_ids[i] = -1;
  for (long long i = tid; i < g.R; i += stride) b.all_counts[i] = 0;
  for (long long i = tid; i < g.P; i += stride) {
    b.ioids[i] = -1;
    b.ranks[i] = -1;
    b.first_depth[i] = max_depth;
    b.near_consumers[i] = 0;
  }
  for (long long i = tid; i < g.H; i += stride) b.active_counts[i] = 0;
  for (long long i = tid; i < (long long)g.H * 7; i += stride) b.stats[i] = 0;
  for (long long i = tid; i < g.REGIONS; i += stride) b.region_counts[i] = 0;
  if (tid == 0) b.missing[0] = 0;
  if (!g.PRIVATE) {
    // Clear mapping entries of every valid selection and set the sentinel.
    for (long long i = tid; i < (long long)g.Q * g.H * g.W; i += stride) {
      int q = (int)(i / ((long long)g.H * g.W));
      int h = (int)((i / g.W) % g.H);
      int block = b.blocks[i];
      int pos = b.positions[q];
      int total = (int)(b.desc[h * 5 + 1] + b.desc[h * 5 + 4]);
      if (occurrence_valid(block, pos, total, g)) b.mapping[(long long)h * (g.MAP + 1) + block] = -1;
    }
    for (long long i = tid; i < g.H; i += stride)
      b.mapping[i * (g.MAP + 1) + g.MAP] = -2;
  }
}

// ------------------------------------------------------------ dedup insert ---
// First CAS winner of (head, block) claims a compact slot (active.py:80-114).
__global__ void insert_kernel(Geo g, cxs_plan_buffers b) {
  int warp = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  int lane = threadIdx.x % 32;
  if (warp >= g.Q * g.H) return;
  int q = warp / g.H, h = warp % g.H;
  int pos = b.positions[q];
  int total = (int)(b.desc[h * 5 + 1] + b.desc[h * 5 + 4]);
  int errors = 0;
  for (int i0 = 0; i0 < g.W; i0 += 32) {
    int i = i0 + lane;
    if (i >= g.W) continue;
    int block = b.blocks[(long long)warp * g.W + i];
    bool valid = occurrence_valid(block, pos, total, g);
    if (valid) {
      int prev = atomicCAS(&b.mapping[(long long)h * (g.MAP + 1) + block], -1, -2);
      if (prev == -1) {
        int compact = atomicAdd(&b.active_counts[h], 1);
        if (compact < g.CAP) b.insert_keys[(long long)h * g.CAP + compact] = block;
        else ++errors;
      }
    } else if (block >= 0 && pos >= 0) {
      ++errors;
    }
  }
  errors = cxs::warp_sum(errors);
  if (lane == 0 && errors) atomicAdd(&b.stats[h * 7 + 6], errors);
}

// --------------------------------------------------- sorted compaction ---
// Compact index = rank of the block among the head's active keys, i.e. the
// sorted-key layout of active.py:117-131, 440-446, built from a bitmap.
__global__ void compact_kernel(Geo g, cxs_plan_buffers b) {
  extern __shared__ uint32_t bits[];
  int h = blockIdx.x;
  int words = (g.MAP + 31) / 32;
  for (int w = threadIdx.x; w < words; w += blockDim.x) bits[w] = 0;
  __syncthreads();
  int count = min(b.active_counts[h], g.CAP);
  for (int i = threadIdx.x; i < count; i += blockDim.x) {
    int block = b.insert_keys[(long long)h * g.CAP + i];
    atomicOr(&bits[block >> 5], 1u << (block & 31));
  }
  __syncthreads();
  // Each thread owns a contiguous run of words; exclusive scan of popcounts.
  int per = (words + blockDim.x - 1) / blockDim.x;
  int begin = threadIdx.x * per, end = min(words, begin + per);
  int local = 0;
  for (int w = begin; w < end; ++w) local += __popc(bits[w]);
  typedef cub::BlockScan<int, 1024> Scan;
  __shared__ typename Scan::TempStorage scan;
  int offset;
  Scan(scan).ExclusiveSum(local, offset);
  for (int w = begin; w < end; ++w) {
    uint32_t word = bits[w];
    while (word) {
      int bit = __ffs(word) - 1;
      word &= word - 1;
      int block = w * 32 + bit;
      b.active_keys[(long long)h * g.CAP + offset] = block;
      b.mapping[(long long)h * (g.MAP + 1) + block] = offset;
      ++offset;
    }
  }
  for (int c = count + threadIdx.x; c < g.CAP; c += blockDim.x)
    b.active_keys[(long long)h * g.CAP + c] = kInt32Max;
}

// -------------------------------------------------------------- references ---
// required = max causal prefix; per-token frequencies of historical tokens;
// stats[4] old refs / stats[5] local refs (active.py:168-206).
__global__ void references_kernel(Geo g, cxs_plan_buffers b) {
  int warp = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  int lane = threadIdx.x % 32;
  if (warp >= g.Q * g.H) return;
  int q = warp / g.H, h = warp % g.H;
  int pos = b.positions[q];
  int old = (int)b.desc[h * 5 + 1];
  int history = (int)b.desc[h * 5 + 2];
  int total = old + (int)b.desc[h * 5 + 4];
  int old_refs = 0, local_refs = 0;
  for (int i = 0; i < g.W; ++i) {
    int block = b.blocks[(long long)warp * g.W + i];
    if (!occurrence_valid(block, pos, total, g)) continue;
    int compact = b.mapping[(long long)h * (g.MAP + 1) + block];
    if (compact < 0 || compact >= g.CAP) continue;
    int start = block * g.BS;
    int req = min(g.BS, min(pos + 1, total) - start);
    if (lane == 0) {
      atomicMax(&b.required[(long long)h * g.CAP + compact], req);
      int olds = min(max(old - start, 0), req);
      old_refs += olds;
      local_refs += req - olds;
    }
    int historical = min(max(history - start, 0), req);
    int32_t* freq = b.frequencies + (long long)h * g.SORT + (long long)compact * g.BS;
    for (int o = lane; o < historical; o += 32) atomicAdd(&freq[o], 1);
  }
  if (lane == 0) {
    if (old_refs) atomicAdd(&b.stats[h * 7 + 4], old_refs);
    if (local_refs) atomicAdd(&b.stats[h * 7 + 5], local_refs);
  }
}

// ------------------------------------------------------ source resolution ---
// Per compact block: current suffix KV, hot replica or backing-pool slot for
// each required token (active.py:134-165 hot hash, 209-295 addresses).
__device__ __forceinline__ uint32_t hash_slot(int token, int mask) {
  return ((uint32_t)token * 2654435761u) & (uint32_t)mask;
}

__global__ void addresses_kernel(Geo g, cxs_plan_buffers b) {
  extern __shared__ int hash_mem[];
  int* hkeys = hash_mem;
  int* hvals = hash_mem + g.HASH;
  int h = blockIdx.y;
  int row = (int)b.desc[h * 5];
  int old = (int)b.desc[h * 5 + 1];
  long long pointer = b.desc[h * 5 + 3];
  // With a residency table every history token is looked up directly; the
  // hot hash is only built from the tags otherwise.
  const int32_t* table = b.hbm_locs ? b.hbm_locs + (long long)row * g.MAXH : nullptr;
  for (int i = threadIdx.x; i < g.HASH; i += blockDim.x) hkeys[i] = -1;
  __syncthreads();
  const int32_t* tags = b.tags + (long long)row * (g.HOT + 1);
  const int32_t* locs = b.locs + (long long)row * (g.HOT + 1);
  for (int i = threadIdx.x; i < (table ? 0 : g.HOT); i += blockDim.x) {
    int token = tags[i];
    if (token < 0 || token >= old) continue;
    uint32_t s = hash_slot(token, g.HASH - 1);
    for (int probe = 0; probe < g.HASH; ++probe) {
      int prev = atomicCAS(&hkeys[s], -1, token);
      if (prev == -1) {
        hvals[s] = locs[i];
        break;
      }
      if (prev == token) break;  // duplicate tag: keep the first location
      s = (s + 1) & (g.HASH - 1);
    }
  }
  __syncthreads();
  int warps = blockDim.x / 32;
  int lane = threadIdx.x % 32;
  int c = blockIdx.x * warps + threadIdx.x / 32;
  if (c >= g.CAP) return;
  long long p = (long long)h * g.CAP + c;
  bool active = c < b.active_counts[h];
  int block = active ? b.active_keys[p] : -1;
  int req = active ? b.required[p] : 0;
  const char* hot_data = static_cast<const char*>(b.hot_data);
  int n_valid = 0, n_prev = 0, n_hot = 0, n_ext = 0, n_err = 0;
  int region_mask_counts[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (int o = lane; o < g.BS; o += 32) {
    long long token = (long long)block * g.BS + o;
    bool valid = active && o < req;
    bool previous = valid && token < old;
    int location = -1;
    if (previous && table) {
      location = token < g.MAXH ? table[token] : -1;
    } else if (previous) {
      uint32_t s = hash_slot((int)token, g.HASH - 1);
      for (int probe = 0; probe < g.HASH; ++probe) {
        int key = hkeys[s];
        if (key == (int)token) {
          location = hvals[s];
          break;
        }
        if (key == -1) break;
        s = (s + 1) & (g.HASH - 1);
      }
    }
    bool external = previous && location < 0;
    long long source = -1;
    if (external && token >= 0 && token < g.MAXH) source = b.host_locs[(long long)row * g.MAXH + token];
    bool error = external && (source < 0 || source >= g.POOL);
    bool safe = external && !error;
    long long hbm = 0;
    if (valid && !external)
      hbm = previous ? (long long)(hot_data + (long long)location * kTokenBytes) - 0
                     : pointer + (token - old) * kTokenBytes;
    long long address = hbm;
    if (safe) {
      int region;
      address = pool_address(g, b.bases, source, &region);
      if (region < 8) region_mask_counts[region] += 1;
      else atomicAdd(&b.region_counts[region], 1);
    }
    long long idx = p * g.BS + o;
    b.address[idx] = address;
    b.hbm[idx] = hbm;
    b.slots[idx] = safe ? source : -1;
    n_valid += valid;
    n_prev += previous;
    n_hot += previous && !external;
    n_ext += external;
    n_err += error;
  }
  n_valid = cxs::warp_sum(n_valid);
  n_prev = cxs::warp_sum(n_prev);
  n_hot = cxs::warp_sum(n_hot);
  n_ext = cxs::warp_sum(n_ext);
  n_err = cxs::warp_sum(n_err);
  int regions8 = min(g.REGIONS, 8);
  for (int r = 0; r < regions8; ++r) {
    int cnt = cxs::warp_sum(region_mask_counts[r]);
    if (lane == 0 && cnt) atomicAdd(&b.region_counts[r], cnt);
  }
  if (lane == 0) {
    b.valid[p] = (active && n_err == 0) ? req : 0;
    b.starts[p] = active ? block * g.BS : 0;
    b.flags[p] = n_ext > 0;
    if (n_valid) atomicAdd(&b.stats[h * 7 + 0], n_valid);
    if (n_prev) atomicAdd(&b.stats[h * 7 + 1], n_prev);
    if (n_hot) atomicAdd(&b.stats[h * 7 + 2], n_hot);
    if (n_ext) atomicAdd(&b.stats[h * 7 + 3], n_ext);
    if (n_err) atomicAdd(&b.stats[h * 7 + 6], n_err);
  }
}

// ------------------------------------------------------------- occurrences ---
// Original-order occurrence rows with duplicates kept (occurrences.py:7-35).
__global__ void occurrences_kernel(Geo g, cxs_plan_buffers b) {
  int r = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  int lane = threadIdx.x % 32;
  if (r >= g.R) return;
  int q = r / g.H, h = r % g.H;
  int pos = b.positions[q];
  bool head_ok = b.stats[h * 7 + 6] == 0;
  int count = 0;
  for (int i0 = 0; i0 < g.W; i0 += 32) {
    int i = i0 + lane;
    bool valid = false;
    int physical = 0;
    if (i < g.W && head_ok) {
      if (!g.PRIVATE) {
        int block = b.blocks[(long long)r * g.W + i];
        valid = pos >= 0 && block >= 0 && block < g.MAP && (long long)block * g.BS <= pos;
        if (valid) {
          int compact = b.mapping[(long long)h * (g.MAP + 1) + block];
          valid = compact >= 0 && compact < g.CAP;
          physical = h * g.CAP + compact;
        }
      } else {
        int origin = b.private_occurrences[(long long)r * g.W + i];
        valid = origin >= 0;
        if (valid) {
          int compact = b.mapping[(long long)h * g.CAP + origin];
          valid = compact >= 0;
          physical = h * g.CAP + compact;
        }
      }
    }
    unsigned mask = __ballot_sync(0xffffffffu, valid);
    if (valid) b.all_ids[(long long)r * g.W + count + __popc(mask & ((1u << lane) - 1))] = physical;
    count += __popc(mask);
  }
  if (lane == 0) {
    b.all_counts[r] = count;
    b.row_positions[r] = pos;
  }
}

// ------------------------------------------------------ consumption depth ---
// Depth of each row along its consumer's serial row stream, counting resident
// steps; first depth at which each block is consumed (dependencies.py:47-75,
// which keeps it for missing blocks; resident blocks get it too, so that the
// attention launch can order every row's blocks by the read-order key
// whatever their residency).
__global__ void depth_kernel(Geo g, cxs_plan_buffers b) {
  int r = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  int lane = threadIdx.x % 32;
  if (r >= g.R) return;
  int consumers = g.CONSUMERS;
  int depth = 0;
  for (int prev = r % consumers + lane * consumers; prev < r; prev += 32 * consumers)
    if (b.row_positions[prev] >= 0) depth += b.all_counts[prev];
  depth = cxs::warp_sum(depth);
  if (lane == 0) b.row_depth[r] = depth;
  if (b.row_positions[r] < 0) return;
  int count = min(g.W, b.all_counts[r]);
  for (int col = lane; col < count; col += 32) {
    int block = b.all_ids[(long long)r * g.W + col];
    if (block >= 0 && block < g.P) atomicMin(&b.first_depth[block], depth + col);
  }
}

// Distinct rows consuming a block within NEAR_WINDOW steps of its first depth
// (dependencies.py:78-112; every block, as for the first depth).
__global__ void near_kernel(Geo g, cxs_plan_buffers b) {
  int r = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  int lane = threadIdx.x % 32;
  if (r >= g.R || b.row_positions[r] < 0) return;
  int count = min(g.W, b.all_counts[r]);
  int depth0 = b.row_depth[r];
  const int32_t* ids = b.all_ids + (long long)r * g.W;
  for (int col = lane; col < count; col += 32) {
    int block = ids[col];
    if (block < 0 || block >= g.P) continue;
    int first = b.first_depth[block];
    int depth = depth0 + col;
    if (depth < first || depth >= first + kNearWindow) continue;
    bool unique = true;
    for (int back = 1; back < kNearWindow; ++back)
      if (col >= back && ids[col - back] == block) unique = false;
    if (unique) atomicAdd(&b.near_consumers[block], 1);
  }
}

// ----------------------------------------------------------------- publish ---
// Stable IOIDs/Ranks: missing blocks by (first depth, -near, block); physical
// order is the special case of a zero depth (dependencies.py:115-191,
// active.py:298-305). One CTA, CUB block radix sort on unique 64-bit keys.
template <int ITEMS>
__global__ void __launch_bounds__(1024) publish_kernel(Geo g, cxs_plan_buffers b,
                                                       unsigned long long bound, int end_bit) {
  typedef cub::BlockRadixSort<unsigned long long, 1024, ITEMS> Sort;
  typedef cub::BlockReduce<int, 1024> Reduce;
  extern __shared__ __align__(16) unsigned char sort_mem[];
  auto& temp = *reinterpret_cast<typename Sort::TempStorage*>(sort_mem);
  __shared__ typename Reduce::TempStorage reduce;
  __shared__ int total_missing;
  unsigned long long keys[ITEMS];
  int missing = 0;
  const unsigned long long P = (unsigned long long)g.P;
  const unsigned long long rows = (unsigned long long)g.R;
#pragma unroll
  for (int k = 0; k < ITEMS; ++k) {
    int block = threadIdx.x * ITEMS + k;
    if (block < g.P) {
      bool miss = b.flags[block] != 0;
      missing += miss;
      if (!miss) {
        keys[k] = bound + (unsigned long long)block;
      } else if (g.ORDER == CXS_ORDER_PHYSICAL) {
        keys[k] = (unsigned long long)block;
      } else {
        unsigned long long first = (unsigned long long)b.first_depth[block];
        unsigned long long near =
            g.ORDER == CXS_ORDER_DEPTH_SHARED ? (unsigned long long)b.near_consumers[block] : 0ull;
        keys[k] = (first * (rows + 1) + rows - near) * P + (unsigned long long)block;
      }
    } else {
      keys[k] = ~0ull;  // padding sorts last
    }
  }
  int total = Reduce(reduce).Sum(missing);
  if (threadIdx.x == 0) {
    total_missing = total;
    b.missing[0] = total;
  }
  Sort(temp).SortBlockedToStriped(keys, 0, end_bit);
  __syncthreads();
  int count = total_missing;
#pragma unroll
  for (int k = 0; k < ITEMS; ++k) {
    int rank = k * 1024 + threadIdx.x;  // striped arrangement
    if (rank < count) {
      int block = (int)(keys[k] % P);
      b.ioids[rank] = block;
      b.ranks[block] = rank;
    }
  }
}

// Physical-order publish for plans beyond one CTA (active.py:298-305): chunk
// counts of missing blocks, a scan over chunks, then an ordered compaction.
constexpr int kChunk = 1024;

__global__ void __launch_bounds__(kChunk) chunk_count_kernel(Geo g, cxs_plan_buffers b,
                                                             int32_t* chunk_counts) {
  typedef cub::BlockReduce<int, kChunk> Reduce;
  __shared__ typename Reduce::TempStorage reduce;
  int i = blockIdx.x * kChunk + threadIdx.x;
  int miss = i < g.P && b.flags[i] != 0;
  int total = Reduce(reduce).Sum(miss);
  if (threadIdx.x == 0) chunk_counts[blockIdx.x] = total;
}

__global__ void __launch_bounds__(kChunk) chunk_compact_kernel(Geo g, cxs_plan_buffers b,
                                                               const int32_t* chunk_counts,
                                                               int chunks) {
  typedef cub::BlockScan<int, kChunk> Scan;
  __shared__ typename Scan::TempStorage scan;
  __shared__ int base;
  if (threadIdx.x == 0) {
    int sum = 0, all = 0;
    for (int c = 0; c < chunks; ++c) {
      if (c < (int)blockIdx.x) sum += chunk_counts[c];
      all += chunk_counts[c];
    }
    base = sum;
    if (blockIdx.x == 0) b.missing[0] = all;
  }
  __syncthreads();
  int i = blockIdx.x * kChunk + threadIdx.x;
  int miss = i < g.P && b.flags[i] != 0;
  int prefix;
  Scan(scan).ExclusiveSum(miss, prefix);
  if (miss) {
    b.ioids[base + prefix] = i;
    b.ranks[i] = base + prefix;
  }
}

// --------------------------------------------------------------- hot top-k ---
// Top-`hot` indices of a head's frequency table by (frequency desc, index asc)
// (active.py:449-500; stable argsort fallback active.py:884-888): find the
// threshold frequency by a radix select over the significant bytes of the
// maximum, keep every larger frequency and the lowest-index ties (an ordered
// warp-segmented gather), then sort the `hot` winners (rank counting up to
// 1024 of them, a block radix sort above). Histograms use warp-aggregated
// shared atomics because most frequencies share a few small values. When the
// table fits (`staged`), one pass with eight loads in flight per thread copies
// it into shared memory (after the sort storage) and every later pass reads
// it there instead of making a round of dependent global loads per stride.
template <int ITEMS>
__global__ void __launch_bounds__(1024) hot_select_kernel(Geo g, cxs_plan_buffers b, int staged) {
  typedef cub::BlockRadixSort<unsigned long long, 1024, ITEMS> Sort;
  typedef cub::BlockReduce<unsigned int, 1024> Reduce;
  extern __shared__ __align__(16) unsigned char sort_mem[];
  auto& temp = *reinterpret_cast<typename Sort::TempStorage*>(sort_mem);
  __shared__ typename Reduce::TempStorage reduce;
  __shared__ int hist[256];
  __shared__ unsigned int prefix_s, mask_s, max_s;
  __shared__ int remaining_s;
  __shared__ unsigned long long cand[kMaxHot];
  int h = blockIdx.x;
  int lane = threadIdx.x & 31;
  const int32_t* freq = b.frequencies + (long long)h * g.SORT;
  int n = g.SORT;
  unsigned int local_max = 0;
  if (staged) {
    constexpr size_t kTemp = (sizeof(typename Sort::TempStorage) + 15) & ~size_t(15);
    int32_t* stage = reinterpret_cast<int32_t*>(sort_mem + kTemp);
    for (int base = 0; base < n; base += 8 * 1024) {
      int v[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int i = base + k * 1024 + threadIdx.x;
        v[k] = i < n ? freq[i] : 0;
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int i = base + k * 1024 + threadIdx.x;
        if (i < n) stage[i] = v[k];
        local_max = max(local_max, (unsigned)v[k]);
      }
    }
    freq = stage;
  } else {
    for (int i = threadIdx.x; i < n; i += blockDim.x) local_max = max(local_max, (unsigned)freq[i]);
  }
  unsigned int fmax = Reduce(reduce).Reduce(local_max, cub::Max());
  if (threadIdx.x == 0) {
    max_s = fmax;
    prefix_s = 0;
    remaining_s = g.HOT;
    int top = 0;  // highest byte holding a set bit of the maximum
    while (top < 24 && (fmax >> (top + 8))) top += 8;
    mask_s = top >= 24 ? 0u : ~((1u << (top + 8)) - 1u);  // bytes above `top` are zero
    hist[0] = top;                                        // smuggle `top` to all threads
  }
  __syncthreads();
  int top = hist[0];
  __syncthreads();
  for (int shift = top; shift >= 0; shift -= 8) {
    for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    unsigned int prefix = prefix_s, mask = mask_s;
    for (int base = 0; base < n; base += blockDim.x) {
      int i = base + threadIdx.x;
      unsigned int f = i < n ? (unsigned)freq[i] : 0u;
      bool active = i < n && (f & mask) == prefix;
      unsigned int digit = active ? (f >> shift) & 255u : 256u + lane;
      unsigned peers = __match_any_sync(0xffffffffu, digit);
      if (active && lane == __ffs(peers) - 1) atomicAdd(&hist[digit], __popc(peers));
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int remaining = remaining_s;
      int digit = 255;
      for (; digit > 0; --digit) {
        if (hist[digit] >= remaining) break;
        remaining -= hist[digit];
      }
      prefix_s = prefix | ((unsigned int)digit << shift);
      mask_s = mask | (255u << shift);
      remaining_s = remaining;
    }
    __syncthreads();
  }
  unsigned int threshold = prefix_s;
  int need_eq = remaining_s;                 // ties at the threshold, lowest indices first
  int greater_total = g.HOT - need_eq;       // every frequency above the threshold
  // Ordered gather: warp w owns the contiguous segment [s0, s1); a counting
  // pass and a scan over the 32 warps give each warp its output offsets.
  const int warp = threadIdx.x >> 5;
  const int seg = (n + 31) / 32, s0 = min(n, warp * seg), s1 = min(n, s0 + seg);
  const unsigned lower = (1u << lane) - 1u;
  int count_g = 0, count_e = 0;
  for (int i = s0 + lane; i < s1; i += 32) {
    unsigned int f = (unsigned)freq[i];
    count_g += f > threshold;
    count_e += f == threshold;
  }
  for (int o = 16; o; o >>= 1) {
    count_g += __shfl_xor_sync(0xffffffffu, count_g, o);
    count_e += __shfl_xor_sync(0xffffffffu, count_e, o);
  }
  if (lane == 0) {
    hist[warp] = count_g;
    hist[32 + warp] = count_e;
  }
  __syncthreads();
  if (warp < 2) {  // warp 0: greater offsets, warp 1: equal offsets (exclusive scans)
    int own = hist[32 * warp + lane], inclusive = own;
    for (int o = 1; o < 32; o <<= 1) {
      int other = __shfl_up_sync(0xffffffffu, inclusive, o);
      if (lane >= o) inclusive += other;
    }
    hist[64 + 32 * warp + lane] = inclusive - own;
  }
  __syncthreads();
  int g_at = hist[64 + warp], e_at = hist[96 + warp];
  for (int i0 = s0; i0 < s1; i0 += 32) {
    int i = i0 + lane;
    unsigned int f = i < s1 ? (unsigned)freq[i] : 0u;
    bool greater = i < s1 && f > threshold;
    bool equal = i < s1 && f == threshold;
    unsigned mg = __ballot_sync(0xffffffffu, greater), me = __ballot_sync(0xffffffffu, equal);
    unsigned long long key = ((unsigned long long)(0x7FFFFFFFu - f) << 32) | (unsigned int)i;
    if (greater) cand[g_at + __popc(mg & lower)] = key;
    int eq_rank = e_at + __popc(me & lower);
    if (equal && eq_rank < need_eq) cand[greater_total + eq_rank] = key;
    g_at += __popc(mg);
    e_at += __popc(me);
  }
  __syncthreads();
  if (g.HOT <= 1024) {
    // Rank sort of the (distinct) winner keys: rank = number of smaller keys.
    if (threadIdx.x < g.HOT) {
      unsigned long long key = cand[threadIdx.x];
      int rank = 0;
      for (int j = 0; j < g.HOT; ++j) rank += cand[j] < key;
      b.chosen[(long long)h * g.HOT + rank] = (int)(key & 0xFFFFFFFFull);
    }
    return;
  }
  unsigned long long keys[ITEMS];
#pragma unroll
  for (int k = 0; k < ITEMS; ++k) {
    int idx = threadIdx.x * ITEMS + k;
    keys[k] = idx < g.HOT ? cand[idx] : ~0ull;
  }
  __syncthreads();
  Sort(temp).SortBlockedToStriped(keys);
#pragma unroll
  for (int k = 0; k < ITEMS; ++k) {
    int rank = k * 1024 + threadIdx.x;
    if (rank < g.HOT) b.chosen[(long long)h * g.HOT + rank] = (int)(keys[k] & 0xFFFFFFFFull);
  }
}

// ------------------------------------------------------ query-private plan ---
// Per (query, head): first-occurrence ownership, sorted private keys,
// occurrence origins, absolute-token frequencies with a canonical source
// (query_private.py:29-105). Requires W <= 32.
__global__ void private_references_kernel(Geo g, cxs_plan_buffers b) {
  int warp = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  int lane = threadIdx.x % 32;
  if (warp >= g.Q * g.H) return;
  int q = warp / g.H, h = warp % g.H;
  int pos = b.positions[q];
  int old = (int)b.desc[h * 5 + 1];
  int history = (int)b.desc[h * 5 + 2];
  int total = old + (int)b.desc[h * 5 + 4];
  bool in_row = lane < g.W;
  int block = in_row ? b.blocks[(long long)warp * g.W + lane] : (-1 - lane) - 64;
  bool valid = in_row && occurrence_valid(block, pos, total, g);
  unsigned same = __match_any_sync(0xffffffffu, block);
  bool own = valid && (__ffs(same) - 1) == lane;
  unsigned own_mask = __ballot_sync(0xffffffffu, own);
  int n_own = __popc(own_mask);
  // local rank = number of owned blocks smaller than this lane's block
  int local = 0;
  for (int j = 0; j < 32; ++j) {
    int other = __shfl_sync(0xffffffffu, block, j);
    if ((own_mask >> j) & 1u) local += other < block;
  }
  long long base = (long long)h * g.CAP + (long long)q * g.W;
  if (own) {
    b.insert_keys[base + local] = block;
    b.private_required[base + local] = min(g.BS, min(pos + 1, total) - block * g.BS);
  }
  if (in_row && lane >= n_own) {
    b.insert_keys[base + lane] = kInt32Max;
    b.private_required[base + lane] = 0;
  }
  if (in_row) b.private_occurrences[(long long)warp * g.W + lane] = valid ? q * g.W + local : -1;
  int old_refs = 0, local_refs = 0, errors = 0;
  if (in_row && !valid && block >= 0 && pos >= 0) errors = 1;
  // Frequencies / canonical sources: each valid occurrence, lanes over tokens.
  for (int i = 0; i < g.W; ++i) {
    int bi = __shfl_sync(0xffffffffu, block, i);
    bool vi = __shfl_sync(0xffffffffu, valid, i);
    int li = __shfl_sync(0xffffffffu, local, i);
    if (!vi) continue;
    int start = bi * g.BS;
    int req = min(g.BS, min(pos + 1, total) - start);
    if (lane == 0) {
      int olds = min(max(old - start, 0), req);
      old_refs += olds;
      local_refs += req - olds;
    }
    int historical = min(max(history - start, 0), req);
    int origin = q * g.W + li;
    for (int o = lane; o < historical; o += 32) {
      long long t = (long long)h * g.SORT + start + o;
      atomicAdd(&b.frequencies[t], 1);
      atomicMin(&b.canonical[t], origin * g.BS + o);
    }
  }
  errors = cxs::warp_sum(errors);
  if (lane == 0) {
    if (old_refs) atomicAdd(&b.stats[h * 7 + 4], old_refs);
    if (local_refs) atomicAdd(&b.stats[h * 7 + 5], local_refs);
    if (errors) atomicAdd(&b.stats[h * 7 + 6], errors);
  }
}

// Ordered compaction of nonempty private slots (query_private.py:108-128).
__global__ void private_compact_kernel(Geo g, cxs_plan_buffers b) {
  typedef cub::BlockScan<int, 1024> Scan;
  __shared__ typename Scan::TempStorage scan;
  __shared__ int running;
  int h = blockIdx.x;
  if (threadIdx.x == 0) running = 0;
  __syncthreads();
  for (int base = 0; base < g.CAP; base += blockDim.x) {
    int i = base + threadIdx.x;
    long long idx = (long long)h * g.CAP + i;
    int length = i < g.CAP ? b.private_required[idx] : 0;
    bool valid = length > 0;
    int prefix, sum;
    Scan(scan).ExclusiveSum((int)valid, prefix, sum);
    int rank = running + prefix;
    if (valid) {
      b.active_keys[(long long)h * g.CAP + rank] = b.insert_keys[idx];
      b.required[(long long)h * g.CAP + rank] = length;
    }
    if (i < g.CAP) b.mapping[idx] = valid ? rank : -1;
    __syncthreads();
    if (threadIdx.x == 0) running += sum;
    __syncthreads();
  }
  if (threadIdx.x == 0) b.active_counts[h] = running;
}

// ------------------------------------------------------------ hot commit ---
// One warp per (head, hot slot): tag update and 256-byte payload copy from the
// staging buffer (active.py:410-437; query_private.py:188-216).
__global__ void commit_kernel(Geo g, cxs_plan_buffers b, const uint4* __restrict__ kv,
                              int32_t* tags, uint4* data) {
  int warp = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  int lane = threadIdx.x % 32;
  if (warp >= g.H * g.HOT) return;
  int h = warp / g.HOT, slot = warp % g.HOT;
  int row = (int)b.desc[h * 5];
  int ct = b.chosen[(long long)h * g.HOT + slot];
  bool selected = ct >= 0 && ct < g.SORT && b.frequencies[(long long)h * g.SORT + ct] > 0;
  int token = -1;
  long long source = -1;
  if (selected) {
    if (!g.PRIVATE) {
      int compact = ct / g.BS;
      if (compact < g.CAP) {
        token = b.active_keys[(long long)h * g.CAP + compact] * g.BS + ct % g.BS;
        source = ((long long)h * g.CAP + compact) * g.BS + ct % g.BS;
      } else {
        selected = false;
      }
    } else {
      token = ct;
      int original = b.canonical[(long long)h * g.SORT + ct];
      int compact = b.mapping[(long long)h * g.CAP + original / g.BS];
      source = ((long long)h * g.CAP + compact) * g.BS + original % g.BS;
    }
  }
  long long index = (long long)row * (g.HOT + 1) + slot;
  if (lane == 0) tags[index] = selected ? token : -1;
  if (selected && lane < 16) {
    int location = b.locs[index];
    data[(long long)location * 16 + lane] = kv[source * 16 + lane];
  }
}

// -------------------------------------------------------------- fused plan ---
// The deduplicating plan in one launch of a single thread-block cluster
// (16 CTAs of 512 threads where the GPU allows, else 8), its phases
// separated by the cluster's hardware barrier instead of kernel boundaries.
// Same arrays, same values as the kernels above:
//   0 reset                                   (reset_kernel)
//   1 dedup insert                            (insert_kernel)
//   2 compact ranks + references: every CTA rebuilds the per-head bitmap of
//     inserted blocks and its word prefix counts in shared memory, so a
//     block's compact index (its rank among the head's keys) is known without
//     waiting for the mapping; CTA h writes head h's active_keys / mapping
//                                             (compact_kernel, references_kernel)
//   3 source resolution, missing count        (addresses_kernel)
//   4 occurrence rows, consumption depth: a row's depth recounts the valid
//     occurrences of the earlier rows of its consumer (at most 8 of them),
//     so both fit one phase; longer consumer chains take two
//                                             (occurrences_kernel, depth_kernel)
//   5 near consumers (shared order only)      (near_kernel)
//   6 IOIDs / Ranks: each missing block's rank is the number of missing
//     blocks with a smaller unique key, counted against all keys staged in
//     shared memory                           (publish_kernel)
constexpr int kFusedThreads = 512;
constexpr int kFusedWarps = kFusedThreads / 32;
constexpr int kFusedMaxPhysical = 8192;
constexpr int kFusedMaxMap = 65536;
constexpr int kFusedMaxChain = 8;  // earlier rows per consumer recounted in phase 4
constexpr int kFusedMaxHeads = 8;
constexpr int kFusedRegions = 32;  // pool region bases kept in shared memory

// Hardware barrier over the CTAs of the cluster, ordering their memory
// accesses (shared and global) at cluster scope.
__device__ __forceinline__ void cluster_sync() {
  asm volatile(
      "barrier.cluster.arrive.release.aligned;\n"
      "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Distributed shared memory: the address of the same shared-memory offset
// in CTA `cta` of the cluster, a fire-and-forget OR into it and a load.
__device__ __forceinline__ uint32_t cluster_map(uint32_t local, uint32_t cta) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local), "r"(cta));
  return remote;
}
__device__ __forceinline__ void cluster_or(uint32_t remote, uint32_t value) {
  asm volatile("red.shared::cluster.or.b32 [%0], %1;" ::"r"(remote), "r"(value) : "memory");
}
__device__ __forceinline__ uint32_t cluster_ld(uint32_t remote) {
  uint32_t value;
  asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(value) : "r"(remote) : "memory");
  return value;
}

// Valid, mapped occurrences of row r (warp-collective): the occurrence-row
// length of occurrences_kernel for a deduplicating plan; compact(h, block)
// gives the compact index or -1.
template <typename Compact>
__device__ __forceinline__ int row_occurrences(const Geo& g, const cxs_plan_buffers& b, int r,
                                               int lane, Compact compact, int32_t* out) {
  const int q = r / g.H, h = r % g.H;
  const int pos = b.positions[q];
  const bool head_ok = b.stats[h * 7 + 6] == 0;
  int count = 0;
  for (int i0 = 0; i0 < g.W; i0 += 32) {
    const int i = i0 + lane;
    bool valid = false;
    int physical = 0;
    if (i < g.W && head_ok) {
      const int block = b.blocks[(long long)r * g.W + i];
      valid = pos >= 0 && block >= 0 && block < g.MAP && (long long)block * g.BS <= pos;
      if (valid) {
        const int c = compact(h, block);
        valid = c >= 0 && c < g.CAP;
        physical = h * g.CAP + c;
      }
    }
    const unsigned mask = __ballot_sync(0xffffffffu, valid);
    if (out && valid) out[count + __popc(mask & ((1u << lane) - 1))] = physical;
    count += __popc(mask);
  }
  return count;
}

__global__ void __launch_bounds__(kFusedThreads, 1)
    plan_fused_kernel(Geo g, cxs_plan_buffers b, int max_depth, int merged_depth) {
  extern __shared__ __align__(16) unsigned char fused_mem[];
  const int ctas = gridDim.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const long long gtid = (long long)blockIdx.x * kFusedThreads + threadIdx.x;
  const long long gthreads = (long long)ctas * kFusedThreads;
  const int gwarp = blockIdx.x * kFusedWarps + warp, gwarps = ctas * kFusedWarps;

  // Per-CTA counters: phases add into shared memory and flush one global
  // atomic per counter per CTA (the stats words are shared by every block
  // and row of a head, so direct global atomics would serialise at L2).
  __shared__ int cta_stats[kFusedMaxHeads * 7];
  __shared__ int cta_regions[8];
  __shared__ int cta_missing;
  auto clear_counters = [&]() {
    for (int i = threadIdx.x; i < kFusedMaxHeads * 7; i += kFusedThreads) cta_stats[i] = 0;
    if (threadIdx.x < 8) cta_regions[threadIdx.x] = 0;
    if (threadIdx.x == 0) cta_missing = 0;
  };
  auto flush_counters = [&]() {  // after a __syncthreads
    for (int i = threadIdx.x; i < g.H * 7; i += kFusedThreads)
      if (cta_stats[i]) atomicAdd(&b.stats[i], cta_stats[i]);
    if (threadIdx.x < min(g.REGIONS, 8) && cta_regions[threadIdx.x])
      atomicAdd(&b.region_counts[threadIdx.x], cta_regions[threadIdx.x]);
    if (threadIdx.x == 0 && cta_missing) atomicAdd(b.missing, cta_missing);
  };
  // CTA h (h < H) keeps head h's claim bitmap at the start of its shared
  // memory; every CTA reaches it through distributed shared memory.
  const int words = (g.MAP + 31) / 32;
  uint32_t* claim = reinterpret_cast<uint32_t*>(fused_mem);
  unsigned char* scratch = fused_mem + (((size_t)words * 4 + 15) & ~(size_t)15);
  // Scratch: the claim bitmaps and word prefix counts of every head (phases
  // 2-3), the hot hash of this CTA's phase-3 head (built in phase 1) and the
  // CTA's required lengths and full-history reference counts per physical
  // block (phase 2); phase 6 reuses it all for the unique keys.
  const size_t layout_bytes = ((size_t)2 * g.H * words * 4 + 15) & ~(size_t)15;
  int* hkeys = reinterpret_cast<int*>(scratch + layout_bytes);
  int* hvals = hkeys + g.HASH;
  int* cta_required = hvals + g.HASH;  // [P]
  int* cta_full = cta_required + g.P;  // [P]
  const int per_head = ctas / g.H;  // phase-3 CTAs per head
  const bool resolver = (int)blockIdx.x < per_head * g.H;
  const bool hot_hash = resolver && !b.hbm_locs;
  // Pool region bases (phase 3 address arithmetic) in shared memory.
  __shared__ int64_t region_bases[kFusedRegions];
  const int64_t* bases = g.REGIONS <= kFusedRegions ? region_bases : b.bases;
  for (int i = threadIdx.x; i < min(g.REGIONS, kFusedRegions); i += kFusedThreads)
    region_bases[i] = b.bases[i];

  // ---- 0: reset. The claim bitmaps are cleared first and announced with a
  // split cluster barrier, so the global resets below overlap the barrier's
  // latency (they are ordered before phase 2 by the barrier after phase 1).
  {
    clear_counters();
    if ((int)blockIdx.x < g.H)
      for (int i = threadIdx.x; i < words; i += kFusedThreads) claim[i] = 0;
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
    if (hot_hash)
      for (int i = threadIdx.x; i < g.HASH; i += kFusedThreads) hkeys[i] = -1;
    for (int i = threadIdx.x; i < g.P; i += kFusedThreads) {
      cta_required[i] = 0;
      cta_full[i] = 0;
    }
    const long long hc = (long long)g.H * g.CAP, hs = (long long)g.H * g.SORT;
    const long long rw = (long long)g.R * g.W;
    for (long long i = gtid; i < hc; i += gthreads) {
      b.required[i] = 0;
      b.insert_keys[i] = kInt32Max;
    }
    for (long long i = gtid; i < hs; i += gthreads) b.frequencies[i] = 0;
    for (long long i = gtid; i < rw; i += gthreads) b.all_ids[i] = -1;
    for (long long i = gtid; i < g.R; i += gthreads) b.all_counts[i] = 0;
    for (long long i = gtid; i < g.P; i += gthreads) {
      b.ioids[i] = -1;
      b.ranks[i] = -1;
      b.first_depth[i] = max_depth;
      b.near_consumers[i] = 0;
    }
    for (long long i = gtid; i < g.H; i += gthreads) b.active_counts[i] = 0;
    for (long long i = gtid; i < (long long)g.H * 7; i += gthreads) b.stats[i] = 0;
    for (long long i = gtid; i < g.REGIONS; i += gthreads) b.region_counts[i] = 0;
    if (gtid == 0) b.missing[0] = 0;
    // Every mapping entry of a valid selection is rewritten in phase 2 (all
    // valid blocks are claimed), so only the sentinel is set here.
    for (long long i = gtid; i < g.H; i += gthreads) b.mapping[i * (g.MAP + 1) + g.MAP] = -2;
  }
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
  __syncthreads();  // this CTA's shared-memory resets (hot hash, tallies) done

  // ---- 1: dedup claims: each valid occurrence sets its block's bit in the
  // head's claim bitmap (CTA h's shared memory); duplicates set it again.
  for (int r = gwarp; r < g.R; r += gwarps) {
    const int q = r / g.H, h = r % g.H;
    const int pos = b.positions[q];
    const int total = (int)(b.desc[h * 5 + 1] + b.desc[h * 5 + 4]);
    const uint32_t remote = cluster_map(cxs::smem_addr(claim), h);
    int errors = 0;
    for (int i = lane; i < g.W; i += 32) {
      const int block = b.blocks[(long long)r * g.W + i];
      if (occurrence_valid(block, pos, total, g))
        cluster_or(remote + (uint32_t)(block >> 5) * 4, 1u << (block & 31));
      else if (block >= 0 && pos >= 0)
        ++errors;
    }
    errors = cxs::warp_sum(errors);
    if (lane == 0 && errors) atomicAdd(&cta_stats[h * 7 + 6], errors);
  }
  // The hot hash of this CTA's phase-3 head: token -> replica location of
  // the tags below the cached length (the first location of a duplicate tag).
  if (hot_hash) {
    const int h = blockIdx.x % g.H;
    const int row = (int)b.desc[h * 5];
    const int old = (int)b.desc[h * 5 + 1];
    const int32_t* tags = b.tags + (long long)row * (g.HOT + 1);
    const int32_t* locs = b.locs + (long long)row * (g.HOT + 1);
    for (int i = threadIdx.x; i < g.HOT; i += kFusedThreads) {
      const int token = tags[i];
      if (token < 0 || token >= old) continue;
      uint32_t s = hash_slot(token, g.HASH - 1);
      for (int probe = 0; probe < g.HASH; ++probe) {
        const int prev = atomicCAS(&hkeys[s], -1, token);
        if (prev == -1) {
          hvals[s] = locs[i];
          break;
        }
        if (prev == token) break;  // duplicate tag: keep the first location
        s = (s + 1) & (g.HASH - 1);
      }
    }
  }
  __syncthreads();
  flush_counters();
  __syncthreads();
  clear_counters();
  cluster_sync();

  // ---- 2: claim bitmaps copied into every CTA with word prefix counts, so
  // a block's compact index (its rank among the head's claimed blocks) is
  // known locally; CTA h publishes head h's compact layout; references.
  uint32_t* bits = reinterpret_cast<uint32_t*>(scratch);                // [H][words]
  int* prefix = reinterpret_cast<int*>(bits + (long long)g.H * words);  // [H][words]
  for (int h = 0; h < g.H; ++h) {
    const uint32_t remote = cluster_map(cxs::smem_addr(claim), h);
    for (int i = threadIdx.x; i < words; i += kFusedThreads)
      bits[h * words + i] = cluster_ld(remote + (uint32_t)i * 4);
  }
  __syncthreads();
  // Word prefix counts of head h: warp h scans the head's words 32 at a time.
  if (warp < g.H) {
    const int h = warp;
    int carry = 0;
    for (int base = 0; base < words; base += 32) {
      const int w = base + lane;
      const int c = w < words ? __popc(bits[h * words + w]) : 0;
      int incl = c;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int other = __shfl_up_sync(0xffffffffu, incl, d);
        if (lane >= d) incl += other;
      }
      if (w < words) prefix[h * words + w] = carry + incl - c;
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
  }
  __syncthreads();
  auto rank_of = [&](int h, int block) -> int {
    const uint32_t word = bits[h * words + (block >> 5)];
    const uint32_t bit = 1u << (block & 31);
    if (!(word & bit)) return -1;
    return prefix[h * words + (block >> 5)] + __popc(word & (bit - 1));
  };
  if ((int)blockIdx.x < g.H) {  // CTA h publishes head h's compact layout
    const int h = blockIdx.x;
    const int count = prefix[h * words + words - 1] + __popc(bits[h * words + words - 1]);
    if (threadIdx.x == 0) {
      b.active_counts[h] = count;
      if (count > g.CAP) atomicAdd(&b.stats[h * 7 + 6], count - g.CAP);  // no slot left
    }
    // One thread per block id: claimed blocks write their compact slot.
    for (int block = threadIdx.x; block < g.MAP; block += kFusedThreads) {
      const int offset = rank_of(h, block);
      if (offset < 0) continue;
      if (offset < g.CAP) {
        b.active_keys[(long long)h * g.CAP + offset] = block;
        b.insert_keys[(long long)h * g.CAP + offset] = block;
        b.mapping[(long long)h * (g.MAP + 1) + block] = offset;
      } else {
        b.mapping[(long long)h * (g.MAP + 1) + block] = -2;
      }
    }
    for (int c = min(count, g.CAP) + threadIdx.x; c < g.CAP; c += kFusedThreads)
      b.active_keys[(long long)h * g.CAP + c] = kInt32Max;
  }
  // References, one occurrence per lane (required = causal prefix maximum,
  // old / local token counts, one frequency-run count per occurrence). The
  // required maximum and the counts of full-history occurrences gather in
  // shared memory and reach global memory once per block and CTA: a block
  // that every row selects would otherwise queue hundreds of atomics on one
  // word at L2, and phase 3's reads of that word wait behind them.
  for (int r = gwarp; r < g.R; r += gwarps) {
    const int q = r / g.H, h = r % g.H;
    const int pos = b.positions[q];
    const int old = (int)b.desc[h * 5 + 1];
    const int history = (int)b.desc[h * 5 + 2];
    const int total = old + (int)b.desc[h * 5 + 4];
    int old_refs = 0, local_refs = 0;
    for (int i = lane; i < g.W; i += 32) {
      const int block = b.blocks[(long long)r * g.W + i];
      if (!occurrence_valid(block, pos, total, g)) continue;
      const int compact = rank_of(h, block);
      if (compact < 0 || compact >= g.CAP) continue;
      const int start = block * g.BS;
      const int req = min(g.BS, min(pos + 1, total) - start);
      atomicMax(&cta_required[h * g.CAP + compact], req);
      const int olds = min(max(old - start, 0), req);
      old_refs += olds;
      local_refs += req - olds;
      // One count per occurrence at slot (historical - 1) of the block's
      // frequency run; phase 3 turns the run into per-token frequencies
      // (token o is counted by every occurrence covering more than o
      // historical tokens: a suffix sum).
      const int historical = min(max(history - start, 0), req);
      if (historical == g.BS)
        atomicAdd(&cta_full[h * g.CAP + compact], 1);
      else if (historical > 0)
        atomicAdd(&b.frequencies[(long long)h * g.SORT + (long long)compact * g.BS +
                                 historical - 1], 1);
    }
    old_refs = cxs::warp_sum(old_refs);
    local_refs = cxs::warp_sum(local_refs);
    if (lane == 0) {
      if (old_refs) atomicAdd(&cta_stats[h * 7 + 4], old_refs);
      if (local_refs) atomicAdd(&cta_stats[h * 7 + 5], local_refs);
    }
  }
  __syncthreads();
  int* cta_first = cta_required;  // reused in phase 4: the CTA's first consumption depths
  for (int p = threadIdx.x; p < g.P; p += kFusedThreads) {
    if (cta_required[p]) atomicMax(&b.required[p], cta_required[p]);
    if (cta_full[p])
      atomicAdd(&b.frequencies[(long long)(p / g.CAP) * g.SORT + (long long)(p % g.CAP) * g.BS +
                               g.BS - 1],
                cta_full[p]);
    cta_first[p] = max_depth;
  }
  flush_counters();
  __syncthreads();
  clear_counters();
  cluster_sync();

  // ---- 3: source resolution; CTAs split by head, one compact block per
  // warp at a time (lane l owns tokens l and l + 32 of the block). The compact
  // layout of phase 2 (claim bitmaps, word prefix counts) is still in shared
  // memory and the hot hash was built in phase 1, so a block's id, the head's
  // block count and hot locations are shared-memory lookups; every global
  // load of a block (required length, frequency run, pool slots, residency
  // table) is in flight before the first of them is used. The block loop is
  // not unrolled: this phase runs once per launch, from a cold instruction
  // cache, so its code is kept short.
  if (resolver) {
    const int h = blockIdx.x % g.H, k = blockIdx.x / g.H;
    const int row = (int)b.desc[h * 5];
    const int old = (int)b.desc[h * 5 + 1];
    const long long pointer = b.desc[h * 5 + 3];
    const int32_t* table = b.hbm_locs ? b.hbm_locs + (long long)row * g.MAXH : nullptr;
    const int64_t* row_slots = b.host_locs + (long long)row * g.MAXH;
    const char* hot_data = static_cast<const char*>(b.hot_data);
    const uint32_t* hbits = bits + (long long)h * words;
    const int* hprefix = prefix + (long long)h * words;
    const int count = hprefix[words - 1] + __popc(hbits[words - 1]);
    const int regions8 = min(g.REGIONS, 8);
#pragma unroll 1
    for (int c = k * kFusedWarps + warp; c < g.CAP; c += per_head * kFusedWarps) {
      const bool active = c < count;
      const long long p = (long long)h * g.CAP + c;
      int32_t* run = b.frequencies + (long long)h * g.SORT + (long long)c * g.BS;
      // Block id of compact index c: the c-th claimed block of the head.
      int block = -1;
      if (active) {
        int lo = 0, hi = words - 1;  // last word whose prefix count is <= c
        while (lo < hi) {
          const int mid = (lo + hi + 1) >> 1;
          if (hprefix[mid] <= c) lo = mid;
          else hi = mid - 1;
        }
        uint32_t word = hbits[lo];
        for (int skip = c - hprefix[lo]; skip > 0; --skip) word &= word - 1;
        block = lo * 32 + __ffs(word) - 1;
      }
      const int req = active ? b.required[p] : 0;
      int fv[2];
      long long slot[2];
      int table_loc[2];
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        const int o = lane + 32 * t;
        const long long token = (long long)block * g.BS + o;
        const bool history = active && o < g.BS && token < old && token < g.MAXH;
        fv[t] = o < g.BS ? run[o] : 0;
        slot[t] = history ? row_slots[token] : -1;
        table_loc[t] = history && table ? table[token] : -1;
      }
      // Hot locations (shared memory) while the loads are in flight.
      int hot_loc[2] = {-1, -1};
      if (!table) {
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          const int o = lane + 32 * t;
          const long long token = (long long)block * g.BS + o;
          if (!(active && o < g.BS && token < old)) continue;
          uint32_t s = hash_slot((int)token, g.HASH - 1);
          for (int probe = 0; probe < g.HASH; ++probe) {
            const int key = hkeys[s];
            if (key == (int)token) {
              hot_loc[t] = hvals[s];
              break;
            }
            if (key == -1) break;
            s = (s + 1) & (g.HASH - 1);
          }
        }
      }
      // Frequency run: per-token frequencies are suffix sums of the
      // per-length counts (token o: counts at slots >= o).
      {
        int lo_sum = fv[0], hi_sum = fv[1];
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
          const int lo_other = __shfl_down_sync(0xffffffffu, lo_sum, d);
          const int hi_other = __shfl_down_sync(0xffffffffu, hi_sum, d);
          if (lane + d < 32) {
            lo_sum += lo_other;
            hi_sum += hi_other;
          }
        }
        const int hi_total = __shfl_sync(0xffffffffu, hi_sum, 0);
        if (lane < g.BS) run[lane] = lo_sum + hi_total;
        if (lane + 32 < g.BS) run[lane + 32] = hi_sum;
      }
      unsigned packed = 0;  // n_valid | n_prev << 8 | n_hot << 16 | n_ext << 24
      int n_err = 0, region_of[2] = {-1, -1};
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        const int o = lane + 32 * t;
        if (o >= g.BS) continue;
        const long long token = (long long)block * g.BS + o;
        const bool valid = active && o < req;
        const bool previous = valid && token < old;
        int location = -1;
        long long source = -1;
        if (previous) {
          location = table ? (token < g.MAXH ? table_loc[t] : -1) : hot_loc[t];
          if (location < 0 && token < g.MAXH) source = slot[t];
        }
        const bool external = previous && location < 0;
        const bool error = external && (source < 0 || source >= g.POOL);
        const bool safe = external && !error;
        long long hbm = 0;
        if (valid && !external)
          hbm = previous ? (long long)(hot_data + (long long)location * kTokenBytes)
                         : pointer + (token - old) * kTokenBytes;
        long long address = hbm;
        if (safe) {
          int region;
          address = pool_address(g, bases, source, &region);
          if (region < 8) region_of[t] = region;
          else atomicAdd(&b.region_counts[region], 1);
        }
        const long long idx = p * g.BS + o;
        b.address[idx] = address;
        b.hbm[idx] = hbm;
        b.slots[idx] = safe ? source : -1;
        packed += (unsigned)valid | ((unsigned)previous << 8) |
                  ((unsigned)(previous && !external) << 16) | ((unsigned)external << 24);
        n_err += error;
      }
      // Block totals over the warp (every count is at most 64).
#pragma unroll
      for (int d = 16; d; d >>= 1) {
        packed += __shfl_xor_sync(0xffffffffu, packed, d);
        n_err += __shfl_xor_sync(0xffffffffu, n_err, d);
      }
#pragma unroll 1
      for (int r = 0; r < regions8; ++r) {
        const int cnt = __popc(__ballot_sync(0xffffffffu, region_of[0] == r)) +
                        __popc(__ballot_sync(0xffffffffu, region_of[1] == r));
        if (lane == 0 && cnt) atomicAdd(&cta_regions[r], cnt);
      }
      if (lane == 0) {
        const int n_valid = packed & 255u, n_prev = (packed >> 8) & 255u;
        const int n_hot = (packed >> 16) & 255u, n_ext = packed >> 24;
        b.valid[p] = (active && n_err == 0) ? req : 0;
        b.starts[p] = active ? block * g.BS : 0;
        b.flags[p] = n_ext > 0;
        if (n_ext > 0) atomicAdd(&cta_missing, 1);
        if (n_valid) atomicAdd(&cta_stats[h * 7 + 0], n_valid);
        if (n_prev) atomicAdd(&cta_stats[h * 7 + 1], n_prev);
        if (n_hot) atomicAdd(&cta_stats[h * 7 + 2], n_hot);
        if (n_ext) atomicAdd(&cta_stats[h * 7 + 3], n_ext);
        if (n_err) atomicAdd(&cta_stats[h * 7 + 6], n_err);
      }
    }
  }
  __syncthreads();
  flush_counters();
  cluster_sync();

  // ---- 4: occurrence rows (+ consumption depth)
  // A block's compact index from the claim bitmaps still in shared memory
  // (the same value phase 2 wrote into the mapping).
  auto mapped = [&](int h, int block) { return rank_of(h, block); };
  const bool by_depth = g.ORDER != CXS_ORDER_PHYSICAL;
  for (int r = gwarp; r < g.R; r += gwarps) {
    int32_t* ids = b.all_ids + (long long)r * g.W;
    const int count = row_occurrences(g, b, r, lane, mapped, ids);
    const int pos = b.positions[r / g.H];
    if (lane == 0) {
      b.all_counts[r] = count;
      b.row_positions[r] = pos;
    }
    if (!by_depth || !merged_depth) continue;
    int depth = 0;
    for (int prev = r % g.CONSUMERS; prev < r; prev += g.CONSUMERS)
      depth += row_occurrences(g, b, prev, lane, mapped, nullptr);
    if (lane == 0) b.row_depth[r] = depth;
    __syncwarp();
    if (pos < 0) continue;
    for (int col = lane; col < min(g.W, count); col += 32) {
      const int block = ids[col];
      if (block >= 0 && block < g.P) atomicMin(&cta_first[block], depth + col);
    }
  }
  if (by_depth && !merged_depth) {
    cluster_sync();
    for (int r = gwarp; r < g.R; r += gwarps) {
      int depth = 0;
      for (int prev = r % g.CONSUMERS + lane * g.CONSUMERS; prev < r; prev += 32 * g.CONSUMERS)
        if (b.row_positions[prev] >= 0) depth += b.all_counts[prev];
      depth = cxs::warp_sum(depth);
      if (lane == 0) b.row_depth[r] = depth;
      if (b.row_positions[r] < 0) continue;
      const int count = min(g.W, b.all_counts[r]);
      for (int col = lane; col < count; col += 32) {
        const int block = b.all_ids[(long long)r * g.W + col];
        if (block >= 0 && block < g.P) atomicMin(&cta_first[block], depth + col);
      }
    }
  }
  // First depths reach global memory once per block and CTA (as in phase 2).
  if (by_depth) {
    __syncthreads();
    for (int p = threadIdx.x; p < g.P; p += kFusedThreads)
      if (cta_first[p] < max_depth) atomicMin(&b.first_depth[p], cta_first[p]);
  }
  cluster_sync();

  // ---- 5: near consumers (shared consumption-depth order)
  if (g.ORDER == CXS_ORDER_DEPTH_SHARED) {
    for (int r = gwarp; r < g.R; r += gwarps) {
      if (b.row_positions[r] < 0) continue;
      const int count = min(g.W, b.all_counts[r]);
      const int depth0 = b.row_depth[r];
      const int32_t* ids = b.all_ids + (long long)r * g.W;
      for (int col = lane; col < count; col += 32) {
        const int block = ids[col];
        if (block < 0 || block >= g.P) continue;
        const int first = b.first_depth[block];
        const int depth = depth0 + col;
        if (depth < first || depth >= first + kNearWindow) continue;
        bool unique = true;
        for (int back = 1; back < kNearWindow; ++back)
          if (col >= back && ids[col - back] == block) unique = false;
        if (unique) atomicAdd(&b.near_consumers[block], 1);
      }
    }
    cluster_sync();
  }

  // ---- 6: IOIDs / Ranks by counting smaller unique keys
  unsigned long long* keys = reinterpret_cast<unsigned long long*>(scratch);
  const unsigned long long P = (unsigned long long)g.P, rows = (unsigned long long)g.R;
  for (int p = threadIdx.x; p < g.P; p += kFusedThreads) {
    unsigned long long key = ~0ull;
    if (b.flags[p]) {
      if (g.ORDER == CXS_ORDER_PHYSICAL) {
        key = (unsigned long long)p;
      } else {
        const unsigned long long first = (unsigned long long)b.first_depth[p];
        const unsigned long long near =
            g.ORDER == CXS_ORDER_DEPTH_SHARED ? (unsigned long long)b.near_consumers[p] : 0ull;
        key = (first * (rows + 1) + rows - near) * P + (unsigned long long)p;
      }
    }
    keys[p] = key;
  }
  __syncthreads();
  // One warp per missing block (blocks spread over the CTAs); the lanes
  // split the keys and the warp sums their counts.
  for (int p = warp * ctas + blockIdx.x; p < g.P; p += gwarps) {
    const unsigned long long key = keys[p];
    if (key == ~0ull) continue;
    int rank = 0;
    for (int j = lane; j < g.P; j += 32) rank += keys[j] < key;
    rank = cxs::warp_sum(rank);
    if (lane == 0) {
      b.ioids[rank] = p;
      b.ranks[p] = rank;
    }
  }
}

int sort_items(int n) {
  int items = 1;
  while (items * 1024 < n) items *= 2;
  return items;
}

template <template <int> class K>
struct Dummy {};

int check_geometry(const cxs_plan_geometry* geo, Geo* out) {
  if (!geo) return set_error(CXS_ERR_INVALID, "null plan geometry");
  Geo g{};
  g.Q = geo->queries;
  g.H = geo->heads;
  g.W = geo->width;
  g.BS = geo->block_size;
  g.MAP = geo->map_blocks;
  g.CAP = geo->per_head;
  g.SORT = geo->sort_extent;
  g.HOT = geo->hot;
  g.MAXH = geo->max_history;
  g.REGIONS = geo->regions;
  g.PAGE = geo->page_size;
  g.CONSUMERS = geo->consumer_ctas;
  g.ORDER = geo->read_order;
  g.PRIVATE = geo->private_plan;
  g.MODE = geo->launch_mode;
  g.POOL = geo->pool_tokens;
  if (g.Q < 1 || g.H < 1 || g.W < 1 || g.BS < 1 || (g.BS & (g.BS - 1)) || g.MAP < 1 ||
      g.CAP < 1 || g.HOT < 1 || g.REGIONS < 1 || g.PAGE < 1 || g.CONSUMERS < 1)
    return set_error(CXS_ERR_INVALID, "nonempty plan geometry and power-of-two BS required");
  if (g.MODE < 0 || g.MODE > 1) return set_error(CXS_ERR_INVALID, "launch_mode must be 0 or 1");
  if (g.ORDER < CXS_ORDER_PHYSICAL || g.ORDER > CXS_ORDER_DEPTH_SHARED)
    return set_error(CXS_ERR_INVALID, "unknown read order %d", g.ORDER);
  if ((long long)g.MAP * g.BS > kInt32Max)
    return set_error(CXS_ERR_INVALID, "absolute token addressing must fit int32");
  if (g.SORT < g.HOT) return set_error(CXS_ERR_INVALID, "sort_extent must cover hot");
  g.P = g.H * g.CAP;
  g.R = g.Q * g.H;
  auto log2_or_minus = [](int v) {
    if (v < 1 || (v & (v - 1))) return -1;
    int shift = 0;
    while ((1 << shift) < v) ++shift;
    return shift;
  };
  g.PAGE_SHIFT = log2_or_minus(g.PAGE);
  g.REGION_SHIFT = log2_or_minus(g.REGIONS);
  g.HASH = 1;
  while (g.HASH < 2 * g.HOT) g.HASH *= 2;
  if (g.MAP + 1 > kMaxMapBlocks)
    return set_error(CXS_ERR_CAPACITY, "map_blocks %d exceeds %d", g.MAP, kMaxMapBlocks - 1);
  if (g.P > kMaxPhysical && g.ORDER != CXS_ORDER_PHYSICAL)
    return set_error(CXS_ERR_CAPACITY,
                     "consumption-depth order supports at most %d physical blocks (got %d)",
                     kMaxPhysical, g.P);
  if (g.P > kMaxPhysical && (g.P + kChunk - 1) / kChunk > g.R)
    return set_error(CXS_ERR_CAPACITY, "physical blocks %d need more rows of scratch", g.P);
  if (g.P > (1 << 24))
    return set_error(CXS_ERR_CAPACITY, "physical blocks %d exceed %d", g.P, 1 << 24);
  if (g.HOT > kMaxHot) return set_error(CXS_ERR_CAPACITY, "hot %d exceeds %d", g.HOT, kMaxHot);
  if (g.PRIVATE && g.W > 32)
    return set_error(CXS_ERR_CAPACITY, "query-private plan supports width <= 32");
  if (g.PRIVATE && g.CAP != g.Q * g.W)
    return set_error(CXS_ERR_INVALID, "query-private per_head must equal queries * width");
  if (!g.PRIVATE && g.CAP > g.MAP)
    return set_error(CXS_ERR_INVALID, "per_head cannot exceed map_blocks");
  *out = g;
  return CXS_OK;
}

template <int ITEMS>
int launch_publish(const Geo& g, const cxs_plan_buffers& b, unsigned long long bound, int end_bit,
                   cudaStream_t stream) {
  size_t smem = sizeof(typename cub::BlockRadixSort<unsigned long long, 1024, ITEMS>::TempStorage);
  CXS_CUDA(cudaFuncSetAttribute(publish_kernel<ITEMS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)smem));
  publish_kernel<ITEMS><<<1, 1024, smem, stream>>>(g, b, bound, end_bit);
  CXS_LAUNCH_CHECK("publish_kernel");
  return CXS_OK;
}

template <int ITEMS>
int launch_hot(const Geo& g, const cxs_plan_buffers& b, cudaStream_t stream) {
  const size_t temp =
      (sizeof(typename cub::BlockRadixSort<unsigned long long, 1024, ITEMS>::TempStorage) + 15) &
      ~size_t(15);
  // Stage the frequency table in shared memory when it fits beside the sort
  // storage and the kernel's static arrays (kMaxHot candidates, histograms).
  const size_t table = (size_t)g.SORT * sizeof(int32_t);
  const bool staged = temp + table + kMaxHot * sizeof(unsigned long long) + 8192 <= 200 * 1024;
  const size_t smem = staged ? temp + table : temp;
  CXS_CUDA(cudaFuncSetAttribute(hot_select_kernel<ITEMS>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  hot_select_kernel<ITEMS><<<g.H, 1024, smem, stream>>>(g, b, staged ? 1 : 0);
  CXS_LAUNCH_CHECK("hot_select_kernel");
  return CXS_OK;
}

// The single-cluster plan when the geometry allows it (deduplicating plan,
// launch_mode 0, at most kFusedMaxPhysical blocks, BS <= 64, shared-memory
// tables within bounds); *launched reports whether it ran.
int launch_fused(const Geo& g, const cxs_plan_buffers& b, int max_depth, cudaStream_t stream,
                 int* launched) {
  *launched = 0;
  if (g.PRIVATE || g.MODE != 0 || g.P > kFusedMaxPhysical || g.MAP + 1 > kFusedMaxMap ||
      g.BS > 64)
    return CXS_OK;
  if (g.H > kFusedMaxHeads) return CXS_OK;
  const size_t words = (size_t)(g.MAP + 31) / 32;
  // Claim bitmap, then the compact layout of every head, the hot hash and the
  // per-CTA reference tallies (phases 1-3), or the unique keys (phase 6).
  size_t smem = (((size_t)2 * g.H * words * 4 + 15) & ~(size_t)15) + (size_t)g.HASH * 8 +
                (size_t)g.P * 8;
  smem += ((words * 4 + 15) & ~(size_t)15) + 16;  // the claim bitmap in front
  constexpr size_t kMaxFusedSmem = 160 * 1024;
  if (smem > kMaxFusedSmem) return CXS_OK;
  static int cluster_cache[64] = {0};  // CTAs per cluster for this device (-1: none)
  int device = 0;
  CXS_CUDA(cudaGetDevice(&device));
  if (device < 0 || device >= 64) return CXS_OK;
  cudaLaunchConfig_t config = {};
  config.blockDim = dim3(kFusedThreads);
  config.dynamicSmemBytes = kMaxFusedSmem;
  config.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  config.attrs = attr;
  config.numAttrs = 1;
  if (!cluster_cache[device]) {
    CXS_CUDA(cudaFuncSetAttribute(plan_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)kMaxFusedSmem));
    if (cudaFuncSetAttribute(plan_fused_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed,
                             1) != cudaSuccess)
      cudaGetLastError();
    cluster_cache[device] = -1;
    for (int size : {16, 8}) {
      config.gridDim = dim3(size);
      attr[0].val.clusterDim.x = size;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      int clusters = 0;
      if (cudaOccupancyMaxActiveClusters(&clusters, plan_fused_kernel, &config) == cudaSuccess &&
          clusters >= 1) {
        cluster_cache[device] = size;
        break;
      }
      cudaGetLastError();
    }
  }
  const int ctas = cluster_cache[device];
  if (ctas < g.H) return CXS_OK;
  const int chain = (g.R + g.CONSUMERS - 1) / g.CONSUMERS - 1;  // earlier rows per consumer
  const int merged = chain <= kFusedMaxChain;
  config.gridDim = dim3(ctas);
  config.dynamicSmemBytes = smem;
  attr[0].val.clusterDim.x = ctas;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  CXS_CUDA(cudaLaunchKernelEx(&config, plan_fused_kernel, g, b, max_depth, merged));
  cxs_host::count_launch();
  *launched = 1;
  return CXS_OK;
}

}  // namespace

extern "C" int cxs_plan_check(const cxs_plan_geometry* geometry) {
  Geo g;
  return check_geometry(geometry, &g);
}

static int plan_impl(const cxs_plan_geometry* geometry, const cxs_plan_buffers* buffers,
                     void* stream_ptr, bool hot);

extern "C" int cxs_plan(const cxs_plan_geometry* geometry, const cxs_plan_buffers* buffers,
                        void* stream_ptr) {
  return plan_impl(geometry, buffers, stream_ptr, true);
}

extern "C" int cxs_plan_core(const cxs_plan_geometry* geometry, const cxs_plan_buffers* buffers,
                             void* stream_ptr) {
  return plan_impl(geometry, buffers, stream_ptr, false);
}

static int plan_impl(const cxs_plan_geometry* geometry, const cxs_plan_buffers* buffers,
                     void* stream_ptr, bool hot) {
  Geo g;
  int status = check_geometry(geometry, &g);
  if (status != CXS_OK) return status;
  if (!buffers) return set_error(CXS_ERR_INVALID, "null plan buffers");
  const cxs_plan_buffers& b = *buffers;
  if (g.PRIVATE && (!b.private_required || !b.private_occurrences || !b.canonical))
    return set_error(CXS_ERR_INVALID, "query-private plan buffers missing");
  cudaStream_t stream = (cudaStream_t)stream_ptr;
  int max_depth = ((g.R + g.CONSUMERS - 1) / g.CONSUMERS) * g.W;
  int fused = 0;
  status = launch_fused(g, b, max_depth, stream, &fused);
  if (status != CXS_OK) return status;
  if (fused) {
    if (!hot) return CXS_OK;
    switch (sort_items(g.HOT)) {
      case 1: return launch_hot<1>(g, b, stream);
      case 2: return launch_hot<2>(g, b, stream);
      default: return launch_hot<4>(g, b, stream);
    }
  }
  int warps_per_cta = 8;
  int row_grid = (g.Q * g.H + warps_per_cta - 1) / warps_per_cta;
  int r_grid = (g.R + warps_per_cta - 1) / warps_per_cta;

  reset_kernel<<<296, 512, 0, stream>>>(g, b, max_depth);
  CXS_LAUNCH_CHECK("reset_kernel");
  if (!g.PRIVATE) {
    insert_kernel<<<row_grid, warps_per_cta * 32, 0, stream>>>(g, b);
    CXS_LAUNCH_CHECK("insert_kernel");
    size_t bitmap = (size_t)((g.MAP + 31) / 32) * 4;
    if (bitmap > 48 * 1024)
      CXS_CUDA(cudaFuncSetAttribute(compact_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)bitmap));
    compact_kernel<<<g.H, 1024, bitmap, stream>>>(g, b);
    CXS_LAUNCH_CHECK("compact_kernel");
    references_kernel<<<row_grid, warps_per_cta * 32, 0, stream>>>(g, b);
    CXS_LAUNCH_CHECK("references_kernel");
  } else {
    private_references_kernel<<<row_grid, warps_per_cta * 32, 0, stream>>>(g, b);
    CXS_LAUNCH_CHECK("private_references_kernel");
    private_compact_kernel<<<g.H, 1024, 0, stream>>>(g, b);
    CXS_LAUNCH_CHECK("private_compact_kernel");
  }
  {
    dim3 grid((g.CAP + warps_per_cta - 1) / warps_per_cta, g.H);
    size_t smem = (size_t)g.HASH * 8;
    if (smem > 48 * 1024)
      CXS_CUDA(cudaFuncSetAttribute(addresses_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)smem));
    addresses_kernel<<<grid, warps_per_cta * 32, smem, stream>>>(g, b);
    CXS_LAUNCH_CHECK("addresses_kernel");
  }
  occurrences_kernel<<<r_grid, warps_per_cta * 32, 0, stream>>>(g, b);
  CXS_LAUNCH_CHECK("occurrences_kernel");
  unsigned long long bound;
  if (g.ORDER == CXS_ORDER_PHYSICAL) {
    bound = (unsigned long long)g.P;
  } else {
    depth_kernel<<<r_grid, warps_per_cta * 32, 0, stream>>>(g, b);
    CXS_LAUNCH_CHECK("depth_kernel");
    if (g.ORDER == CXS_ORDER_DEPTH_SHARED) {
      near_kernel<<<r_grid, warps_per_cta * 32, 0, stream>>>(g, b);
      CXS_LAUNCH_CHECK("near_kernel");
    }
    bound = ((unsigned long long)(max_depth + 1) * (unsigned long long)(g.R + 1) +
             (unsigned long long)g.R) *
            (unsigned long long)g.P;
  }
  int end_bit = 1;
  while (end_bit < 64 && ((bound + (unsigned long long)g.P) >> end_bit)) ++end_bit;
  if (g.P > kMaxPhysical) {
    // Only physical order reaches here (check_geometry): chunked compaction.
    int chunks = (g.P + kChunk - 1) / kChunk;
    int32_t* chunk_counts = b.row_depth;  // unused by the physical order; >= chunks entries
    chunk_count_kernel<<<chunks, kChunk, 0, stream>>>(g, b, chunk_counts);
    CXS_LAUNCH_CHECK("chunk_count_kernel");
    chunk_compact_kernel<<<chunks, kChunk, 0, stream>>>(g, b, chunk_counts, chunks);
    CXS_LAUNCH_CHECK("chunk_compact_kernel");
    status = CXS_OK;
  } else switch (sort_items(g.P)) {
    case 1: status = launch_publish<1>(g, b, bound, end_bit, stream); break;
    case 2: status = launch_publish<2>(g, b, bound, end_bit, stream); break;
    case 4: status = launch_publish<4>(g, b, bound, end_bit, stream); break;
    case 8: status = launch_publish<8>(g, b, bound, end_bit, stream); break;
    default: status = launch_publish<16>(g, b, bound, end_bit, stream); break;
  }
  if (status != CXS_OK || !hot) return status;
  switch (sort_items(g.HOT)) {
    case 1: status = launch_hot<1>(g, b, stream); break;
    case 2: status = launch_hot<2>(g, b, stream); break;
    default: status = launch_hot<4>(g, b, stream); break;
  }
  return status;
}

extern "C" int cxs_plan_select_commit_hot(const cxs_plan_geometry* geometry,
                                          const cxs_plan_buffers* buffers, const void* kv,
                                          int32_t* tags, void* hot_data, void* stream_ptr) {
  Geo g;
  int status = check_geometry(geometry, &g);
  if (status != CXS_OK) return status;
  if (!buffers) return set_error(CXS_ERR_INVALID, "null plan buffers");
  cudaStream_t stream = (cudaStream_t)stream_ptr;
  switch (sort_items(g.HOT)) {
    case 1: status = launch_hot<1>(g, *buffers, stream); break;
    case 2: status = launch_hot<2>(g, *buffers, stream); break;
    default: status = launch_hot<4>(g, *buffers, stream); break;
  }
  if (status != CXS_OK) return status;
  return cxs_plan_commit_hot(geometry, buffers, kv, tags, hot_data, stream_ptr);
}

extern "C" int cxs_plan_commit_hot(const cxs_plan_geometry* geometry,
                                   const cxs_plan_buffers* buffers, const void* kv, int32_t* tags,
                                   void* hot_data, void* stream_ptr) {
  Geo g;
  int status = check_geometry(geometry, &g);
  if (status != CXS_OK) return status;
  if (!buffers || !kv || !tags || !hot_data)
    return set_error(CXS_ERR_INVALID, "null commit argument");
  int warps = g.H * g.HOT;
  commit_kernel<<<(warps + 7) / 8, 256, 0, (cudaStream_t)stream_ptr>>>(
      g, *buffers, (const uint4*)kv, tags, (uint4*)hot_data);
  CXS_LAUNCH_CHECK("commit_kernel");
  return CXS_OK;
}
