// tcgen05 / TMEM attention engine: one warp pair per query row (sm_100a).
//
// Each engine of a CTA is a pair of warps that owns one query row (16 GQA
// heads of one KV head) at a time:
//   - the engine warp keeps the row's K/V tiles (64 tokens of K and V,
//     staged in shared memory by TMA with a 128-byte swizzle) coming and
//     issues every MMA of the row:
//       S[128 x 64 tok]  = Q[128 x 64 dim] . K^T   tcgen05.mma kind::f16, M=128 N=64
//       O[128 x 64 dim] += P[128 x 64 tok] . V      tcgen05.mma kind::f16, M=128 N=64
//   - the softmax warp reads S from TMEM, runs the online softmax in
//     registers, writes P to shared memory and rescales O in TMEM.
// S(t + 1) is computed while the softmax of tile t runs, and neither warp
// waits for its own MMA issue or copy bookkeeping: the pair hands tiles over
// through shared-memory mbarriers (S computed, S read, P written, P.V done).
// Both accumulators live in the pair's 128 TMEM columns (S: 64, O: 64). With
// M = 128, row r of an accumulator is TMEM lane r, and the softmax warp of
// engine w can read lanes 32w .. 32w + 31 only, so the engine's rows are
// 32w .. 32w + 31 of the A tiles (Q and P, shared by the four engines; each
// MMA reads all 128 rows but only the issuing engine's 32 rows of D are
// used). Rows 32w + i and 32w + 16 + i both hold head i: lane i handles
// tokens 0-31 of each tile and lane 16 + i tokens 32-63, with one shuffle to
// combine maxima and sums. P row 32w + lane carries only the lane's own 32
// tokens (the other half stays zero), so the two O rows of a head are
// partial sums that the epilogue adds. Q (pre-scaled by 0.125, bf16) and P
// (bf16 probabilities, as the reference rounds them, tma/pipeline.py:250-253)
// are written in the swizzled K-major layout the MMA descriptors describe; V
// is read MN-major.
#pragma once

#include "cxs_common.cuh"

namespace cxs {
namespace tc {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLazyRescale = 8.f / kLog2e;  // natural-log units: a factor of 2^8
constexpr int kEngines = 4;                    // warp pairs per CTA (softmax warp w reads TMEM subpartition w)
constexpr int kTileRows = 64;                  // tokens per key tile (N of S, K of P.V)
constexpr int kTileBytes = kTileRows * 128;    // one K or V tile
constexpr int kRowTileBytes = 128 * 128;       // Q or P tile: 128 rows of 64 bf16
constexpr int kTmemCols = 128;                 // per engine: S (64) + O (64)

// Shared-memory matrix descriptor, 128-byte swizzle, sm_100 version bits.
__device__ __forceinline__ uint64_t desc_sw128(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor: kind::f16 with bf16 A/B, fp32 accumulate.
__device__ __forceinline__ uint32_t idesc_bf16(int M, int N, int a_mn_major, int b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)a_mn_major << 15) |
         ((uint32_t)b_mn_major << 16) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void mma(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                    int accumulate) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(
          d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0));
}

__device__ __forceinline__ void commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// 32 consecutive fp32 columns of this warp's 32 TMEM lanes (warp-collective).
__device__ __forceinline__ void ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Store 32 fp32 columns back (warp-collective); the caller waits with wait_st().
__device__ __forceinline__ void st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,"
      "%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(
          taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}
__device__ __forceinline__ void wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 16-column variants of ld32 / st32.
__device__ __forceinline__ void ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void st16(uint32_t taddr, const float (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,"
      "%13,%14,%15,%16};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15]))
      : "memory");
}

// Byte offset of 16-byte chunk `chunk` (8 bf16) of row `row` in a [rows x 64]
// bf16 tile with 128-byte swizzle.
__device__ __forceinline__ uint32_t sw128_chunk(int row, int chunk) {
  return (uint32_t)(row * 128 + ((chunk ^ (row & 7)) << 4));
}

// Shared memory of one engine (warp pair): three K buffers, two V buffers,
// the mbarriers that hand tiles between the two warps, an abort word and the
// row's selected blocks with their source kinds (staged by the engine warp).
struct PairSmem {
  static constexpr int kKBufs = 3, kVBufs = 2;
  static constexpr int kBars = (kKBufs + kVBufs) * kTileBytes;
  static constexpr int kBytes = kBars + 1024;  // keeps the next engine 1024-aligned
  uint8_t* base;
  __device__ __forceinline__ uint8_t* k(int b) const { return base + b * kTileBytes; }
  __device__ __forceinline__ uint8_t* v(int b) const { return base + (kKBufs + b) * kTileBytes; }
  __device__ __forceinline__ uint64_t* bar(int i) const {
    return reinterpret_cast<uint64_t*>(base + kBars) + i;
  }
  __device__ __forceinline__ uint64_t* kbar(int b) const { return bar(b); }
  __device__ __forceinline__ uint64_t* vbar(int b) const { return bar(kKBufs + b); }
  // S(t) computed (MMA commit) / P.V(t) done (MMA commit) / S read or Q
  // written (softmax warp) / P(t) written (softmax warp) / final MMA drain.
  __device__ __forceinline__ uint64_t* sbar() const { return bar(5); }
  __device__ __forceinline__ uint64_t* obar() const { return bar(6); }
  __device__ __forceinline__ uint64_t* sfree() const { return bar(7); }
  __device__ __forceinline__ uint64_t* pfull() const { return bar(8); }
  __device__ __forceinline__ uint64_t* drain() const { return bar(9); }
  static constexpr int kNumBars = 10;
  __device__ __forceinline__ volatile int* abort_flag() const {
    return reinterpret_cast<volatile int*>(base + kBars + 96);
  }
  __device__ __forceinline__ int* blocks() const { return reinterpret_cast<int*>(base + kBars + 128); }
  __device__ __forceinline__ int* kinds() const { return reinterpret_cast<int*>(base + kBars + 256); }
};

// Bounded wait on an mbarrier phase that the partner warp of an engine
// completes. Gives up at once when the partner has aborted, or after `limit`
// cycles: then it records `code` in the device error word and aborts the
// engine (both warps then leave the launch).
__device__ __forceinline__ bool pair_wait(uint64_t* bar, uint32_t phase, volatile int* abort,
                                          long long limit, int* error, int code) {
  if (mbar_try_wait(bar, phase)) return true;
  const long long start = clock64();
  while (!mbar_try_wait(bar, phase)) {
    if (*abort) return false;
    if (clock64() - start > limit) {
      atomicOr(error, code);
      *abort = 1;
      return false;
    }
  }
  return true;
}

// Bounded wait on an mbarrier phase. On a timeout it records `code` in the
// device error word, drains with a second bounded wait and returns false.
__device__ __forceinline__ bool bounded_wait(uint64_t* bar, uint32_t phase, long long limit,
                                             int* error, int code) {
  long long start = clock64();
  while (!mbar_try_wait(bar, phase)) {
    if (clock64() - start > limit) {
      atomicOr(error, code);
      long long again = clock64();
      while (!mbar_try_wait(bar, phase) && clock64() - again <= limit) {
      }
      return false;
    }
  }
  return true;
}

// Half (K: channels 0-63, V: 64-127) of a window tile: 64 records of KV head
// `head` from record `record0` (3-D map {channel, head, record};
// out-of-range records are zero-filled).
__device__ __forceinline__ void window_load(uint8_t* dst, const void* map, int channel, int head,
                                            int record0, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cta.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_addr(dst)),
      "l"(map), "r"(channel), "r"(head), "r"(record0), "r"(smem_addr(bar))
      : "memory");
}

// Q row 32w + lane of the shared Q tile: GQA head (lane & 15) of query row
// `row` (bf16 [row][16][64]), scaled by 0.125 and rounded to bf16.
__device__ __forceinline__ void write_query_row(uint8_t* q_tile, const __nv_bfloat16* query,
                                                long long row, int m, int lane) {
  const uint4* src = reinterpret_cast<const uint4*>(query + (row * 16 + (lane & 15)) * 64);
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    uint4 in = src[c], out;
    const uint32_t* w = reinterpret_cast<const uint32_t*>(&in);
    uint32_t* o = reinterpret_cast<uint32_t*>(&out);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const __nv_bfloat162 h2 = *reinterpret_cast<const __nv_bfloat162*>(&w[e]);
      o[e] = pack_bf16(__low2float(h2) * 0.125f, __high2float(h2) * 0.125f);
    }
    *reinterpret_cast<uint4*>(q_tile + sw128_chunk(m, c)) = out;
  }
}

// 2^x with the hardware approximation (flushes results below 2^-126 to 0,
// far below what a bf16 probability or an fp32 denominator resolves here).
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Scores of this lane's half (tokens 32 * half .. 32 * half + 31) of its
// head's row of S (warp-collective TMEM reads of both halves).
__device__ __forceinline__ void load_s(uint32_t s_addr, int half, float (&sv)[32]) {
  uint32_t r0[32], r1[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r0[0]), "=r"(r0[1]), "=r"(r0[2]), "=r"(r0[3]), "=r"(r0[4]), "=r"(r0[5]),
        "=r"(r0[6]), "=r"(r0[7]), "=r"(r0[8]), "=r"(r0[9]), "=r"(r0[10]), "=r"(r0[11]),
        "=r"(r0[12]), "=r"(r0[13]), "=r"(r0[14]), "=r"(r0[15]), "=r"(r0[16]), "=r"(r0[17]),
        "=r"(r0[18]), "=r"(r0[19]), "=r"(r0[20]), "=r"(r0[21]), "=r"(r0[22]), "=r"(r0[23]),
        "=r"(r0[24]), "=r"(r0[25]), "=r"(r0[26]), "=r"(r0[27]), "=r"(r0[28]), "=r"(r0[29]),
        "=r"(r0[30]), "=r"(r0[31])
      : "r"(s_addr));
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r1[0]), "=r"(r1[1]), "=r"(r1[2]), "=r"(r1[3]), "=r"(r1[4]), "=r"(r1[5]),
        "=r"(r1[6]), "=r"(r1[7]), "=r"(r1[8]), "=r"(r1[9]), "=r"(r1[10]), "=r"(r1[11]),
        "=r"(r1[12]), "=r"(r1[13]), "=r"(r1[14]), "=r"(r1[15]), "=r"(r1[16]), "=r"(r1[17]),
        "=r"(r1[18]), "=r"(r1[19]), "=r"(r1[20]), "=r"(r1[21]), "=r"(r1[22]), "=r"(r1[23]),
        "=r"(r1[24]), "=r"(r1[25]), "=r"(r1[26]), "=r"(r1[27]), "=r"(r1[28]), "=r"(r1[29]),
        "=r"(r1[30]), "=r"(r1[31])
      : "r"(s_addr + 32));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) sv[i] = __uint_as_float(half ? r1[i] : r0[i]);
}

// Online softmax over one tile for this lane's half of its head's row;
// tokens outside [lo, hi] are masked. The lane and its partner (lane ^ 16)
// agree on the tile max and sum. Leaves the lane's 32 probabilities in `sv`
// and returns the factor the running output must be scaled by (1 unless the
// reference maximum moved). p = 2^(s log2e - m log2e), the exp2 form of the
// reference's exp(s - m), with m the running reference maximum.
__device__ __forceinline__ float softmax_regs(float (&sv)[32], int lo, int hi, float& m_run,
                                              float& l_run, int half) {
  // This lane's valid tokens: [lo_l, hi_l] within its 32.
  const int lo_l = lo - 32 * half, hi_l = hi - 32 * half;
  const bool whole = lo_l <= 0 && hi_l >= 31;
  if (!__all_sync(0xffffffffu, whole)) {
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (i < lo_l || i > hi_l) sv[i] = -INFINITY;
  }
  float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
  for (int i = 0; i < 32; ++i) mx[i & 3] = fmaxf(mx[i & 3], sv[i]);
  float mt = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
  mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 16));
  // The reference maximum moves only when a score exceeds it by more than
  // 2^8 in probability (so p <= 256 in between, exact in bf16's exponent
  // range): most tiles then need no rescale of O in TMEM.
  const float updated = mt > m_run + kLazyRescale ? mt : m_run;
  const float factor = m_run == -INFINITY ? 0.f
                       : updated == m_run ? 1.f
                                          : ex2((m_run - updated) * kLog2e);
  m_run = updated;
  // A fully masked row so far (updated = -inf) gets p = 0 everywhere.
  const float offset = updated == -INFINITY ? 0.f : updated * kLog2e;
  float sm[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const float v = ex2(fmaf(sv[i], kLog2e, -offset));  // masked: 2^-inf = 0
    sv[i] = v;
    sm[i & 3] += v;
  }
  float sum = (sm[0] + sm[1]) + (sm[2] + sm[3]);
  sum += __shfl_xor_sync(0xffffffffu, sum, 16);
  l_run = l_run * factor + sum;
  return factor;
}

// The lane's 32 probabilities as bf16 into its half of P row `m`.
__device__ __forceinline__ void store_p(uint8_t* p_tile, int m, int half, const float (&sv)[32]) {
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    uint4 chunk = make_uint4(pack_bf16(sv[8 * c + 0], sv[8 * c + 1]),
                             pack_bf16(sv[8 * c + 2], sv[8 * c + 3]),
                             pack_bf16(sv[8 * c + 4], sv[8 * c + 5]),
                             pack_bf16(sv[8 * c + 6], sv[8 * c + 7]));
    *reinterpret_cast<uint4*>(p_tile + sw128_chunk(m, 4 * half + c)) = chunk;
  }
}

// Scale this warp's O rows by `factor` in TMEM (warp-collective; lanes that
// need no rescale pass 1). Skipped when no lane of the warp needs it.
__device__ __forceinline__ void rescale_o(uint32_t o_addr, float factor, bool need) {
  if (!__any_sync(0xffffffffu, need)) return;
  const float f = need ? factor : 1.f;
#pragma unroll
  for (int part = 0; part < 4; ++part) {
    float v[16];
    ld16(o_addr + 16 * part, v);
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] *= f;
    st16(o_addr + 16 * part, v);
  }
  wait_st();
}

// Output of this lane's head for dims 32 * half .. 32 * half + 31: the two
// partial O rows of the head (this lane's and its partner's) added
// (warp-collective TMEM reads and shuffles).
__device__ __forceinline__ void combine_o(uint32_t o_addr, int half, float (&out)[32]) {
  float lo_cols[32], hi_cols[32];
  ld32(o_addr, lo_cols);
  ld32(o_addr + 32, hi_cols);
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const float keep = half ? hi_cols[i] : lo_cols[i];
    const float send = half ? lo_cols[i] : hi_cols[i];
    out[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
}

}  // namespace tc
}  // namespace cxs
