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

}  // namespace

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
