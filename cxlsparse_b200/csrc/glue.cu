// Fused elementwise glue around the cuBLAS projections of one NSA layer.
//
// Reference arithmetic: models/tensor_ops.py (rms_norm, rotary) and
// models/nsa/model.py:440-492 (_project: sigmoid gates, q/k/v views;
// _finish_prepare: SiLU(gate) * up). Every rounding step of the reference's
// bf16 torch sequence is kept: each bf16 tensor op rounds once.
#include "cxs_common.cuh"

using cxs_host::set_error;

namespace {

__device__ __forceinline__ float rbf(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// Eight bf16 values <-> floats.
__device__ __forceinline__ void unpack8(const uint4& v, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __low2float(h[i]);
    f[2 * i + 1] = __high2float(h[i]);
  }
}
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint4 v;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  return v;
}

__device__ __forceinline__ float block_sum(float v, float* partial) {
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((threadIdx.x & 31) == 0) partial[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    v = threadIdx.x < (blockDim.x >> 5) ? partial[threadIdx.x] : 0.f;
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (threadIdx.x == 0) partial[0] = v;
  }
  __syncthreads();
  return partial[0];
}

// One CTA per row: out = bf16(bf16(x * rsqrt(mean(x^2) + eps)) * w).
// VEC: the row is read once as 16-byte vectors (dim % 8 == 0, aligned rows,
// at most kMaxChunks vectors per thread) and kept in registers.
constexpr int kMaxChunks = 4;
template <bool VEC>
__global__ void rms_norm_kernel(const __nv_bfloat16* __restrict__ x,
                                const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ out,
                                int dim, float eps) {
  __shared__ float partial[32];
  const __nv_bfloat16* row = x + (long long)blockIdx.x * dim;
  __nv_bfloat16* orow = out + (long long)blockIdx.x * dim;
  if (VEC) {
    const int chunks = dim / 8;
    float v[kMaxChunks][8];
    float sum = 0.f;
#pragma unroll
    for (int k = 0; k < kMaxChunks; ++k) {
      const int c = threadIdx.x + k * blockDim.x;
      if (c < chunks) {
        unpack8(reinterpret_cast<const uint4*>(row)[c], v[k]);
#pragma unroll
        for (int i = 0; i < 8; ++i) sum += v[k][i] * v[k][i];
      }
    }
    const float scale = rsqrtf(block_sum(sum, partial) / (float)dim + eps);
#pragma unroll
    for (int k = 0; k < kMaxChunks; ++k) {
      const int c = threadIdx.x + k * blockDim.x;
      if (c < chunks) {
        float wv[8], o[8];
        unpack8(reinterpret_cast<const uint4*>(w)[c], wv);
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = rbf(v[k][i] * scale) * wv[i];
        reinterpret_cast<uint4*>(orow)[c] = pack8(o);
      }
    }
    return;
  }
  float sum = 0.f;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) {
    float v = __bfloat162float(row[i]);
    sum += v * v;
  }
  const float scale = rsqrtf(block_sum(sum, partial) / (float)dim + eps);
  for (int i = threadIdx.x; i < dim; i += blockDim.x) {
    float v = rbf(__bfloat162float(row[i]) * scale);
    orow[i] = __float2bfloat16_rn(v * __bfloat162float(w[i]));
  }
}

// One CTA per row: the residual add of the preceding projection and the
// RMSNorm that follows it, in the reference's bf16 sequence
// (models/nsa/model.py: hidden = hidden + F.linear(...), then rms_norm):
//   h = bf16(hidden + delta), written back to `hidden`;
//   out = bf16(bf16(h * rsqrt(mean(h^2) + eps)) * w).
// The row is read as 16-byte vectors and kept in registers (dim % 8 == 0,
// aligned rows, at most kMaxChunks vectors per thread; checked by the host).
__global__ void residual_rms_norm_kernel(__nv_bfloat16* hidden, const __nv_bfloat16* delta,
                                         const __nv_bfloat16* __restrict__ w,
                                         __nv_bfloat16* __restrict__ out, int dim, float eps) {
  __shared__ float partial[32];
  uint4* row = reinterpret_cast<uint4*>(hidden + (long long)blockIdx.x * dim);
  const uint4* drow = reinterpret_cast<const uint4*>(delta + (long long)blockIdx.x * dim);
  uint4* orow = reinterpret_cast<uint4*>(out + (long long)blockIdx.x * dim);
  const int chunks = dim / 8;
  float v[kMaxChunks][8];
  float sum = 0.f;
#pragma unroll
  for (int k = 0; k < kMaxChunks; ++k) {
    const int c = threadIdx.x + k * blockDim.x;
    if (c < chunks) {
      float d[8];
      unpack8(row[c], v[k]);
      unpack8(drow[c], d);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        v[k][i] = rbf(v[k][i] + d[i]);
        sum += v[k][i] * v[k][i];
      }
      row[c] = pack8(v[k]);
    }
  }
  const float scale = rsqrtf(block_sum(sum, partial) / (float)dim + eps);
#pragma unroll
  for (int k = 0; k < kMaxChunks; ++k) {
    const int c = threadIdx.x + k * blockDim.x;
    if (c < chunks) {
      float wv[8], o[8];
      unpack8(reinterpret_cast<const uint4*>(w)[c], wv);
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = rbf(v[k][i] * scale) * wv[i];
      orow[c] = pack8(o);
    }
  }
}

// RoPE (rotate-half, bf16 rounding per op) + sigmoid gates + output packing
// from the fused projection [E, Hq*64 | Hkv*64 | Hkv*64 | Hq*3]. One CTA per
// token; the token's 32 (cos, sin) pairs are computed once and shared by all heads.
__global__ void qkv_rope_kernel(const __nv_bfloat16* __restrict__ proj, int proj_stride,
                                const int32_t* __restrict__ positions,
                                const float* __restrict__ inv_freq, int q_heads, int kv_heads,
                                __nv_bfloat16* __restrict__ query, __nv_bfloat16* __restrict__ records,
                                int records_stride, __nv_bfloat16* __restrict__ current,
                                int current_stride, __nv_bfloat16* __restrict__ gates,
                                int segment_rows, int segment_stride) {
  __shared__ float cos_s[32], sin_s[32];
  int t = blockIdx.x;
  // Destination row of this token's record / current KV (candidate segments).
  const long long d =
      segment_rows > 0 ? (long long)(t / segment_rows) * segment_stride + t % segment_rows : t;
  const __nv_bfloat16* p = proj + (long long)t * proj_stride;
  if (threadIdx.x < 32) {
    const float angle = (float)positions[t] * inv_freq[threadIdx.x];
    cos_s[threadIdx.x] = rbf(cosf(angle));
    sin_s[threadIdx.x] = rbf(sinf(angle));
  }
  __syncthreads();
  int q_cols = q_heads * 64, kv_cols = kv_heads * 64;
  // q and k: rotate pairs (i, i + 32) of each 64-wide head.
  for (int idx = threadIdx.x; idx < (q_heads + kv_heads) * 32; idx += blockDim.x) {
    int head = idx / 32, i = idx % 32;
    bool is_q = head < q_heads;
    const __nv_bfloat16* src = is_q ? p + head * 64 : p + q_cols + (head - q_heads) * 64;
    float cosv = cos_s[i], sinv = sin_s[i];
    float left = __bfloat162float(src[i]), right = __bfloat162float(src[i + 32]);
    float out_left = rbf(rbf(left * cosv) + rbf(-right * sinv));
    float out_right = rbf(rbf(right * cosv) + rbf(left * sinv));
    if (is_q) {
      __nv_bfloat16* dst = query + ((long long)t * q_heads + head) * 64;
      dst[i] = __float2bfloat16_rn(out_left);
      dst[i + 32] = __float2bfloat16_rn(out_right);
    } else {
      int kh = head - q_heads;
      __nv_bfloat16* rec = records + d * records_stride + kh * 128;
      rec[i] = __float2bfloat16_rn(out_left);
      rec[i + 32] = __float2bfloat16_rn(out_right);
      __nv_bfloat16* cur = current + (long long)kh * current_stride + d * 128;
      cur[i] = __float2bfloat16_rn(out_left);
      cur[i + 32] = __float2bfloat16_rn(out_right);
    }
  }
  // v: copied into records / current (second 64 of each 128-wide record).
  for (int idx = threadIdx.x; idx < kv_cols; idx += blockDim.x) {
    int kh = idx / 64, i = idx % 64;
    __nv_bfloat16 v = p[q_cols + kv_cols + idx];
    records[d * records_stride + kh * 128 + 64 + i] = v;
    current[(long long)kh * current_stride + d * 128 + 64 + i] = v;
  }
  // gates: sigmoid, [Hkv, Hq/Hkv, 3] per token.
  for (int idx = threadIdx.x; idx < q_heads * 3; idx += blockDim.x) {
    float g = __bfloat162float(p[q_cols + 2 * kv_cols + idx]);
    gates[(long long)t * q_heads * 3 + idx] = __float2bfloat16_rn(1.f / (1.f + expf(-g)));
  }
}

// out = bf16(silu(gate)) * up, rounded once more (F.silu(a) * b on bf16 tensors).
// Grid (column chunks, rows); VEC: 8 columns per thread as 16-byte vectors.
template <bool VEC>
__global__ void silu_mul_kernel(const __nv_bfloat16* __restrict__ gate_up, int ffn,
                                __nv_bfloat16* __restrict__ out) {
  const int row = blockIdx.y;
  const __nv_bfloat16* p = gate_up + (long long)row * 2 * ffn;
  __nv_bfloat16* o = out + (long long)row * ffn;
  if (VEC) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= ffn / 8) return;
    float g[8], u[8], r[8];
    unpack8(reinterpret_cast<const uint4*>(p)[c], g);
    unpack8(reinterpret_cast<const uint4*>(p + ffn)[c], u);
#pragma unroll
    for (int i = 0; i < 8; ++i) r[i] = rbf(g[i] / (1.f + expf(-g[i]))) * u[i];
    reinterpret_cast<uint4*>(o)[c] = pack8(r);
    return;
  }
  const int col = blockIdx.x * blockDim.x + threadIdx.x;
  if (col >= ffn) return;
  float a = __bfloat162float(p[col]);
  float s = rbf(a / (1.f + expf(-a)));
  o[col] = __float2bfloat16_rn(s * __bfloat162float(p[ffn + col]));
}

// Window compression, stage 1: act = bf16(silu(bf16(W1 vec(x)))) for every
// window, x = bf16(window records + position encoding) (one K or V half).
// CTA (unit chunk, head, part) owns kCmpUnits hidden units; windows go
// through shared memory in tiles of kCmpTile, so every W1 row is read once
// per tile and reused for all of its windows; a lane keeps the CPL 16-byte
// chunks of the row it needs in registers (all loads in flight together).
constexpr int kCmpTile = 16;
constexpr int kCmpUnits = 16;
constexpr int kCmpWarps = 8;

template <int CPL>
__global__ void __launch_bounds__(kCmpWarps * 32, 1)
    compress_hidden_kernel(const __nv_bfloat16* __restrict__ records,
                           const int64_t* __restrict__ rows, int n, int heads, int hidden,
                           const __nv_bfloat16* __restrict__ pe,
                           const __nv_bfloat16* __restrict__ w1, float* __restrict__ act) {
  extern __shared__ uint4 xs[];  // [kCmpTile][in / 8]: bf16 x, 8 values per chunk
  constexpr int kIn = CPL * 256, kChunks = kIn / 8, kL = kIn / 64;
  static_assert(kChunks == kCmpWarps * 32, "one staged chunk per thread");
  const int part = blockIdx.z, h = blockIdx.y, j0 = blockIdx.x * kCmpUnits;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint4* pe_p = reinterpret_cast<const uint4*>(pe + (long long)part * kIn);
  // Thread k stages chunk k (8 channels of token k / 8) of every window of the
  // tile: the row indices, then the records, all loads issued before use.
  const int k = threadIdx.x, t = k / 8, c8 = (k % 8) * 8;
  float q[8];
  unpack8(pe_p[k], q);
  for (int w0 = 0; w0 < n; w0 += kCmpTile) {
    const int nt = min(kCmpTile, n - w0);
    long long row[kCmpTile];
#pragma unroll
    for (int w = 0; w < kCmpTile; ++w) row[w] = w < nt ? rows[(long long)(w0 + w) * kL + t] : 0;
    uint4 rv[kCmpTile];
#pragma unroll
    for (int w = 0; w < kCmpTile; ++w)
      if (w < nt)
        rv[w] = *reinterpret_cast<const uint4*>(records + (row[w] * heads + h) * 128 +
                                                part * 64 + c8);
#pragma unroll
    for (int w = 0; w < kCmpTile; ++w) {
      if (w < nt) {
        float r[8];
        unpack8(rv[w], r);
#pragma unroll
        for (int e = 0; e < 8; ++e) r[e] += q[e];
        xs[w * kChunks + k] = pack8(r);  // rounded to bf16, as the reference adds bf16 tensors
      }
    }
    __syncthreads();
    for (int u = warp; u < kCmpUnits; u += kCmpWarps) {
      const int j = j0 + u;
      if (j >= hidden) break;
      const uint4* wr = reinterpret_cast<const uint4*>(w1 + ((long long)part * hidden + j) * kIn);
      uint4 wv[CPL];
#pragma unroll
      for (int c = 0; c < CPL; ++c) wv[c] = wr[lane + 32 * c];
      float acc[kCmpTile];
#pragma unroll
      for (int w = 0; w < kCmpTile; ++w) acc[w] = 0.f;
#pragma unroll
      for (int c = 0; c < CPL; ++c) {
        float wf[8];
        unpack8(wv[c], wf);
#pragma unroll
        for (int w = 0; w < kCmpTile; ++w) {
          if (w < nt) {
            float xf[8];
            unpack8(xs[w * kChunks + lane + 32 * c], xf);
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[w] = fmaf(wf[e], xf[e], acc[w]);
          }
        }
      }
      float mine = 0.f;
#pragma unroll
      for (int w = 0; w < kCmpTile; ++w) {
        float v = acc[w];
#pragma unroll
        for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (w == lane) mine = v;
      }
      if (lane < nt) {
        const float hv = rbf(mine);
        act[(((long long)part * heads + h) * n + w0 + lane) * hidden + j] =
            rbf(hv / (1.f + expf(-hv)));
      }
    }
    __syncthreads();
  }
}

// Stage 2: key half = bf16(W2 act) into key slot slots[window]. CTA (window,
// head, part) of 4 warps; warp w computes outputs 16 w .. 16 w + 15, lanes
// split the hidden units, and the 16 W2 chunks of a lane load together.
constexpr int kOutPerWarp = 16;

__global__ void __launch_bounds__(128)
    compress_out_kernel(int n, int heads, int hidden, const __nv_bfloat16* __restrict__ w2,
                        const float* __restrict__ act, __nv_bfloat16* __restrict__ keys,
                        const int64_t* __restrict__ slots) {
  const int window = blockIdx.x, h = blockIdx.y, part = blockIdx.z;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const float4* a = reinterpret_cast<const float4*>(
      act + (((long long)part * heads + h) * n + window) * hidden);
  const int c0 = warp * kOutPerWarp;
  const uint4* wbase = reinterpret_cast<const uint4*>(w2 + ((long long)part * 64 + c0) * hidden);
  const int chunks = hidden / 8;
  float acc[kOutPerWarp];
#pragma unroll
  for (int u = 0; u < kOutPerWarp; ++u) acc[u] = 0.f;
  for (int k = lane; k < chunks; k += 32) {
    const float4 a0 = a[2 * k], a1 = a[2 * k + 1];
    uint4 wv[kOutPerWarp];
#pragma unroll
    for (int u = 0; u < kOutPerWarp; ++u) wv[u] = wbase[(long long)u * chunks + k];
#pragma unroll
    for (int u = 0; u < kOutPerWarp; ++u) {
      float wf[8];
      unpack8(wv[u], wf);
      acc[u] = fmaf(wf[0], a0.x, acc[u]);
      acc[u] = fmaf(wf[1], a0.y, acc[u]);
      acc[u] = fmaf(wf[2], a0.z, acc[u]);
      acc[u] = fmaf(wf[3], a0.w, acc[u]);
      acc[u] = fmaf(wf[4], a1.x, acc[u]);
      acc[u] = fmaf(wf[5], a1.y, acc[u]);
      acc[u] = fmaf(wf[6], a1.z, acc[u]);
      acc[u] = fmaf(wf[7], a1.w, acc[u]);
    }
  }
  float mine = 0.f;
#pragma unroll
  for (int u = 0; u < kOutPerWarp; ++u) {
    float v = acc[u];
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (u == lane) mine = v;
  }
  if (lane < kOutPerWarp)
    keys[(slots[window] * heads + h) * 128 + part * 64 + c0 + lane] = __float2bfloat16_rn(mine);
}

}  // namespace

extern "C" int cxs_compress_windows(const void* records, const int64_t* rows, int32_t windows,
                                    int32_t heads, int32_t window, int32_t hidden,
                                    const void* pe, const void* w1, const void* w2,
                                    void* scratch, void* keys, const int64_t* slots,
                                    void* stream) {
  if (windows < 0 || heads < 1 || heads > 65535 || hidden < 8 || hidden % 8 || window != 32)
    return set_error(CXS_ERR_INVALID, "window-compression geometry: window 32, "
                                      "hidden a multiple of 8");
  if (!windows) return CXS_OK;
  if (!records || !rows || !pe || !w1 || !w2 || !scratch || !keys || !slots)
    return set_error(CXS_ERR_INVALID, "null window-compression argument");
  if (((uintptr_t)records | (uintptr_t)pe | (uintptr_t)w1 | (uintptr_t)w2 |
       (uintptr_t)scratch) & 15)
    return set_error(CXS_ERR_INVALID, "window-compression buffers must be 16-byte aligned");
  const int in = window * 64;
  const size_t smem = (size_t)kCmpTile * in * 2;
  dim3 grid1((hidden + kCmpUnits - 1) / kCmpUnits, heads, 2);
  auto* act = static_cast<float*>(scratch);
  CXS_CUDA(cudaFuncSetAttribute(compress_hidden_kernel<8>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  compress_hidden_kernel<8><<<grid1, kCmpWarps * 32, smem, (cudaStream_t)stream>>>(
      (const __nv_bfloat16*)records, rows, windows, heads, hidden, (const __nv_bfloat16*)pe,
      (const __nv_bfloat16*)w1, act);
  CXS_LAUNCH_CHECK("compress_hidden_kernel");
  compress_out_kernel<<<dim3(windows, heads, 2), 128, 0, (cudaStream_t)stream>>>(
      windows, heads, hidden, (const __nv_bfloat16*)w2, act, (__nv_bfloat16*)keys, slots);
  CXS_LAUNCH_CHECK("compress_out_kernel");
  return CXS_OK;
}

extern "C" int cxs_rms_norm(const void* x, const void* weight, void* out, int32_t rows,
                            int32_t dim, float eps, void* stream) {
  if (rows < 0 || dim < 1) return set_error(CXS_ERR_INVALID, "invalid rms_norm geometry");
  if (!rows) return CXS_OK;
  const bool vec = dim % 8 == 0 && dim / 8 <= 256 * kMaxChunks &&
                   !(((uintptr_t)x | (uintptr_t)weight | (uintptr_t)out) & 15);
  if (vec)
    rms_norm_kernel<true><<<rows, 256, 0, (cudaStream_t)stream>>>(
        (const __nv_bfloat16*)x, (const __nv_bfloat16*)weight, (__nv_bfloat16*)out, dim, eps);
  else
    rms_norm_kernel<false><<<rows, 256, 0, (cudaStream_t)stream>>>(
        (const __nv_bfloat16*)x, (const __nv_bfloat16*)weight, (__nv_bfloat16*)out, dim, eps);
  CXS_LAUNCH_CHECK("rms_norm_kernel");
  return CXS_OK;
}

extern "C" int cxs_residual_rms_norm(void* hidden, const void* delta, const void* weight,
                                     void* out, int32_t rows, int32_t dim, float eps,
                                     void* stream) {
  if (rows < 0 || dim < 1) return set_error(CXS_ERR_INVALID, "invalid rms_norm geometry");
  if (!hidden || !delta || !weight || !out)
    return set_error(CXS_ERR_INVALID, "null residual rms_norm argument");
  if (dim % 8 || dim / 8 > 256 * kMaxChunks ||
      (((uintptr_t)hidden | (uintptr_t)delta | (uintptr_t)weight | (uintptr_t)out) & 15))
    return set_error(CXS_ERR_INVALID,
                     "residual rms_norm needs 16-byte aligned rows of at most %d, dim a multiple of 8",
                     8 * 256 * kMaxChunks);
  if (!rows) return CXS_OK;
  residual_rms_norm_kernel<<<rows, 256, 0, (cudaStream_t)stream>>>(
      (__nv_bfloat16*)hidden, (const __nv_bfloat16*)delta, (const __nv_bfloat16*)weight,
      (__nv_bfloat16*)out, dim, eps);
  CXS_LAUNCH_CHECK("residual_rms_norm_kernel");
  return CXS_OK;
}

extern "C" int cxs_qkv_rope_segments(const void* proj, int32_t proj_stride,
                                     const int32_t* positions, const float* inv_freq,
                                     int32_t tokens, int32_t q_heads, int32_t kv_heads,
                                     void* query, void* records, int32_t records_stride,
                                     void* current, int32_t current_stride, void* gates,
                                     int32_t segment_rows, int32_t segment_stride, void* stream) {
  if (tokens < 0 || q_heads < 1 || kv_heads < 1 || segment_rows < 0 ||
      (segment_rows > 0 && segment_stride < segment_rows))
    return set_error(CXS_ERR_INVALID, "invalid qkv_rope geometry");
  if (!tokens) return CXS_OK;
  qkv_rope_kernel<<<tokens, 256, 0, (cudaStream_t)stream>>>(
      (const __nv_bfloat16*)proj, proj_stride, positions, inv_freq, q_heads, kv_heads,
      (__nv_bfloat16*)query, (__nv_bfloat16*)records, records_stride, (__nv_bfloat16*)current,
      current_stride, (__nv_bfloat16*)gates, segment_rows, segment_stride);
  CXS_LAUNCH_CHECK("qkv_rope_kernel");
  return CXS_OK;
}

extern "C" int cxs_qkv_rope(const void* proj, int32_t proj_stride, const int32_t* positions,
                            const float* inv_freq, int32_t tokens, int32_t q_heads,
                            int32_t kv_heads, void* query, void* records, int32_t records_stride,
                            void* current, int32_t current_stride, void* gates, void* stream) {
  return cxs_qkv_rope_segments(proj, proj_stride, positions, inv_freq, tokens, q_heads,
                               kv_heads, query, records, records_stride, current, current_stride,
                               gates, 0, 0, stream);
}

extern "C" int cxs_silu_mul(const void* gate_up, int32_t rows, int32_t ffn, void* out,
                            void* stream) {
  if (rows < 0 || ffn < 1) return set_error(CXS_ERR_INVALID, "invalid silu_mul geometry");
  if (!rows) return CXS_OK;
  if (rows > 65535) return set_error(CXS_ERR_CAPACITY, "silu_mul supports at most 65535 rows");
  const bool vec = ffn % 8 == 0 && !(((uintptr_t)gate_up | (uintptr_t)out) & 15);
  if (vec) {
    dim3 grid((ffn / 8 + 127) / 128, rows);
    silu_mul_kernel<true><<<grid, 128, 0, (cudaStream_t)stream>>>(
        (const __nv_bfloat16*)gate_up, ffn, (__nv_bfloat16*)out);
  } else {
    dim3 grid((ffn + 255) / 256, rows);
    silu_mul_kernel<false><<<grid, 256, 0, (cudaStream_t)stream>>>(
        (const __nv_bfloat16*)gate_up, ffn, (__nv_bfloat16*)out);
  }
  CXS_LAUNCH_CHECK("silu_mul_kernel");
  return CXS_OK;
}
