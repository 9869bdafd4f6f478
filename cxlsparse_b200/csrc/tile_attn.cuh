// Warp-level tensor-core attention tile shared by the attention kernels.
//
// One warp computes 16 query heads (the GQA group, M = 16) against a tile of
// BS key tokens staged in shared memory by TMA with 128-byte swizzle:
// S = Q K^T with mma.m16n8k16 (K via ldmatrix), online softmax in registers,
// O += P V (V via ldmatrix.trans, P reused from the S accumulators).
#pragma once

#include "cxs_common.cuh"

namespace cxs {

constexpr float kLog2e = 1.4426950408889634f;

// ------------------------------------------------------- PTX fragments ---
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Byte offset of (row, 16-byte chunk) inside a 128-byte-swizzled TMA tile.
__device__ __forceinline__ uint32_t sw128(int row, int chunk) {
  return (uint32_t)(row * 128 + ((chunk ^ (row & 7)) << 4));
}

// Online-softmax state of one attention branch for the warp's 16 query heads.
// Lane (g = lane/4, c = lane%4) owns heads g and g+8.
template <int BS>
struct Softmax {
  float o[8][4];
  float m[2], l[2];
  __device__ __forceinline__ void reset() {
#pragma unroll
    for (int n = 0; n < 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
    m[0] = m[1] = -INFINITY;
    l[0] = l[1] = 0.f;
  }
  // One BS-token tile: K at `k_tile`, V at `v_tile` (shared, SW128), masked
  // by `keep(token)` for the tile-relative token index.
  template <typename Keep>
  __device__ __forceinline__ void step(const uint32_t (&qa)[4][4], uint32_t k_tile, uint32_t v_tile,
                                       int lane, Keep keep) {
    constexpr int NT = BS / 8, KT = BS / 16;
    float s[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
      int token = nt * 8 + (lane & 7);
      uint32_t b[8];
      ldsm_x4(k_tile + sw128(token, (lane >> 3)), b[0], b[1], b[2], b[3]);
      ldsm_x4(k_tile + sw128(token, 4 + (lane >> 3)), b[4], b[5], b[6], b[7]);
#pragma unroll
      for (int kt = 0; kt < 4; ++kt) mma_bf16(s[nt], qa[kt], b[2 * kt], b[2 * kt + 1]);
    }
    int c = lane & 3;
    // Zero V rows of masked tokens so a non-finite value beyond a row's
    // position cannot reach the PV product through 0 * NaN.
    bool masked_any = false;
    for (int t = lane; t < BS; t += 32) masked_any |= !keep(t);
    if (__any_sync(0xffffffffu, masked_any)) {
      for (int i = lane; i < BS * 8; i += 32) {
        int t = i / 8;
        if (!keep(t)) {
          uint32_t addr = v_tile + t * 128 + (i % 8) * 16;
          asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(addr), "r"(0) : "memory");
        }
      }
      cxs::fence_proxy_async_shared();
      __syncwarp();
    }
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        int token = nt * 8 + 2 * c + (e & 1);
        if (!keep(token)) s[nt][e] = -INFINITY;
        mx[e >> 1] = fmaxf(mx[e >> 1], s[nt][e]);
      }
    }
    float factor[2], sum[2] = {0.f, 0.f};
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
      float updated = fmaxf(m[r], mx[r]);
      factor[r] = m[r] == -INFINITY ? 0.f : exp2f((m[r] - updated) * kLog2e);
      m[r] = updated;
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float v = s[nt][e] == -INFINITY ? 0.f : exp2f((s[nt][e] - m[e >> 1]) * kLog2e);
        s[nt][e] = v;
        sum[e >> 1] += v;
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      sum[r] += __shfl_xor_sync(0xffffffffu, sum[r], 1);
      sum[r] += __shfl_xor_sync(0xffffffffu, sum[r], 2);
      l[r] = l[r] * factor[r] + sum[r];
    }
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      o[n][0] *= factor[0];
      o[n][1] *= factor[0];
      o[n][2] *= factor[1];
      o[n][3] *= factor[1];
    }
#pragma unroll
    for (int kt = 0; kt < KT; ++kt) {
      uint32_t pa[4] = {cxs::pack_bf16(s[2 * kt][0], s[2 * kt][1]),
                        cxs::pack_bf16(s[2 * kt][2], s[2 * kt][3]),
                        cxs::pack_bf16(s[2 * kt + 1][0], s[2 * kt + 1][1]),
                        cxs::pack_bf16(s[2 * kt + 1][2], s[2 * kt + 1][3])};
      int sel = lane >> 3;
      int token = kt * 16 + (sel & 1) * 8 + (lane & 7);
#pragma unroll
      for (int nd = 0; nd < 8; nd += 2) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(v_tile + sw128(token, nd + (sel >> 1)), b0, b1, b2, b3);
        mma_bf16(o[nd], pa, b0, b1);
        mma_bf16(o[nd + 1], pa, b2, b3);
      }
    }
  }
  // Normalised bf16 output fragment: 2 heads x 8 dim pairs.
  __device__ __forceinline__ void finish(uint32_t (&packed)[8][2]) const {
    float inv0 = 1.f / (l[0] > 0.f ? l[0] : 1.f);
    float inv1 = 1.f / (l[1] > 0.f ? l[1] : 1.f);
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      packed[n][0] = cxs::pack_bf16(o[n][0] * inv0, o[n][1] * inv0);
      packed[n][1] = cxs::pack_bf16(o[n][2] * inv1, o[n][3] * inv1);
    }
  }
};

__device__ __forceinline__ float2 unpack_bf16(uint32_t v) {
  __nv_bfloat162 h = *reinterpret_cast<__nv_bfloat162*>(&v);
  return __bfloat1622float2(h);
}

__device__ __forceinline__ float bf16_round(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}


// S tile only (no softmax): s[nt][e] for heads g/g+8 and tokens 8nt+2c+(e&1).
template <int BS>
__device__ __forceinline__ void score_tile(const uint32_t (&qa)[4][4], uint32_t k_tile, int lane,
                                           float (&s)[BS / 8][4]) {
#pragma unroll
  for (int nt = 0; nt < BS / 8; ++nt) {
    s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
    int token = nt * 8 + (lane & 7);
    uint32_t b[8];
    ldsm_x4(k_tile + sw128(token, (lane >> 3)), b[0], b[1], b[2], b[3]);
    ldsm_x4(k_tile + sw128(token, 4 + (lane >> 3)), b[4], b[5], b[6], b[7]);
#pragma unroll
    for (int kt = 0; kt < 4; ++kt) mma_bf16(s[nt], qa[kt], b[2 * kt], b[2 * kt + 1]);
  }
}

// Q A-fragments for 16 heads x 64 dims, pre-scaled by 0.125 and rounded to bf16
// (q = bf16(Q * 1/sqrt(64)), tma/pipeline.py:444-445).
__device__ __forceinline__ void load_query(const __nv_bfloat16* qrow, int lane, uint32_t (&qa)[4][4]) {
  int g = lane >> 2, c = lane & 3;
#pragma unroll
  for (int kt = 0; kt < 4; ++kt) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      int head = g + (e & 1) * 8;
      int dim = kt * 16 + (e >> 1) * 8 + 2 * c;
      float2 v = unpack_bf16(*reinterpret_cast<const uint32_t*>(qrow + head * 64 + dim));
      qa[kt][e] = pack_bf16(bf16_round(v.x * 0.125f), bf16_round(v.y * 0.125f));
    }
  }
}

// 3-D tensor TMA load (no multicast): coordinates {x, y, z}.
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const void* tensor_map, int x, int y, int z,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cta.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst),
      "l"(tensor_map), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar))
      : "memory");
}

}  // namespace cxs
