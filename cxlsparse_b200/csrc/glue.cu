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

// One CTA per row: out = bf16(bf16(x * rsqrt(mean(x^2) + eps)) * w).
__global__ void rms_norm_kernel(const __nv_bfloat16* __restrict__ x,
                                const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ out,
                                int dim, float eps) {
  const __nv_bfloat16* row = x + (long long)blockIdx.x * dim;
  __nv_bfloat16* orow = out + (long long)blockIdx.x * dim;
  float sum = 0.f;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) {
    float v = __bfloat162float(row[i]);
    sum += v * v;
  }
  __shared__ float partial[32];
  for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if ((threadIdx.x & 31) == 0) partial[threadIdx.x >> 5] = sum;
  __syncthreads();
  if (threadIdx.x < 32) {
    sum = threadIdx.x < (blockDim.x >> 5) ? partial[threadIdx.x] : 0.f;
    for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (threadIdx.x == 0) partial[0] = sum;
  }
  __syncthreads();
  float scale = rsqrtf(partial[0] / (float)dim + eps);
  for (int i = threadIdx.x; i < dim; i += blockDim.x) {
    float v = rbf(__bfloat162float(row[i]) * scale);
    orow[i] = __float2bfloat16_rn(v * __bfloat162float(w[i]));
  }
}

// RoPE (rotate-half, bf16 rounding per op) + sigmoid gates + output packing
// from the fused projection [E, Hq*64 | Hkv*64 | Hkv*64 | Hq*3]. One CTA per token.
__global__ void qkv_rope_kernel(const __nv_bfloat16* __restrict__ proj, int proj_stride,
                                const int32_t* __restrict__ positions,
                                const float* __restrict__ inv_freq, int q_heads, int kv_heads,
                                __nv_bfloat16* __restrict__ query, __nv_bfloat16* __restrict__ records,
                                int records_stride, __nv_bfloat16* __restrict__ current,
                                int current_stride, __nv_bfloat16* __restrict__ gates) {
  int t = blockIdx.x;
  const __nv_bfloat16* p = proj + (long long)t * proj_stride;
  float pos = (float)positions[t];
  int q_cols = q_heads * 64, kv_cols = kv_heads * 64;
  // q and k: rotate pairs (i, i + 32) of each 64-wide head.
  for (int idx = threadIdx.x; idx < (q_heads + kv_heads) * 32; idx += blockDim.x) {
    int head = idx / 32, i = idx % 32;
    bool is_q = head < q_heads;
    const __nv_bfloat16* src = is_q ? p + head * 64 : p + q_cols + (head - q_heads) * 64;
    float cosv = rbf(cosf(pos * inv_freq[i])), sinv = rbf(sinf(pos * inv_freq[i]));
    float left = __bfloat162float(src[i]), right = __bfloat162float(src[i + 32]);
    float out_left = rbf(rbf(left * cosv) + rbf(-right * sinv));
    float out_right = rbf(rbf(right * cosv) + rbf(left * sinv));
    if (is_q) {
      __nv_bfloat16* dst = query + ((long long)t * q_heads + head) * 64;
      dst[i] = __float2bfloat16_rn(out_left);
      dst[i + 32] = __float2bfloat16_rn(out_right);
    } else {
      int kh = head - q_heads;
      __nv_bfloat16* rec = records + (long long)t * records_stride + kh * 128;
      rec[i] = __float2bfloat16_rn(out_left);
      rec[i + 32] = __float2bfloat16_rn(out_right);
      __nv_bfloat16* cur = current + (long long)kh * current_stride + (long long)t * 128;
      cur[i] = __float2bfloat16_rn(out_left);
      cur[i + 32] = __float2bfloat16_rn(out_right);
    }
  }
  // v: copied into records / current (second 64 of each 128-wide record).
  for (int idx = threadIdx.x; idx < kv_cols; idx += blockDim.x) {
    int kh = idx / 64, i = idx % 64;
    __nv_bfloat16 v = p[q_cols + kv_cols + idx];
    records[(long long)t * records_stride + kh * 128 + 64 + i] = v;
    current[(long long)kh * current_stride + (long long)t * 128 + 64 + i] = v;
  }
  // gates: sigmoid, [Hkv, Hq/Hkv, 3] per token.
  for (int idx = threadIdx.x; idx < q_heads * 3; idx += blockDim.x) {
    float g = __bfloat162float(p[q_cols + 2 * kv_cols + idx]);
    gates[(long long)t * q_heads * 3 + idx] = __float2bfloat16_rn(1.f / (1.f + expf(-g)));
  }
}

// out = bf16(silu(gate)) * up, rounded once more (F.silu(a) * b on bf16 tensors).
__global__ void silu_mul_kernel(const __nv_bfloat16* __restrict__ gate_up, int ffn,
                                __nv_bfloat16* __restrict__ out, long long total) {
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  long long row = i / ffn, col = i % ffn;
  const __nv_bfloat16* p = gate_up + row * 2 * ffn;
  float a = __bfloat162float(p[col]);
  float s = rbf(a / (1.f + expf(-a)));
  out[i] = __float2bfloat16_rn(s * __bfloat162float(p[ffn + col]));
}

}  // namespace

extern "C" int cxs_rms_norm(const void* x, const void* weight, void* out, int32_t rows,
                            int32_t dim, float eps, void* stream) {
  if (rows < 0 || dim < 1) return set_error(CXS_ERR_INVALID, "invalid rms_norm geometry");
  if (!rows) return CXS_OK;
  rms_norm_kernel<<<rows, 256, 0, (cudaStream_t)stream>>>(
      (const __nv_bfloat16*)x, (const __nv_bfloat16*)weight, (__nv_bfloat16*)out, dim, eps);
  CXS_LAUNCH_CHECK("rms_norm_kernel");
  return CXS_OK;
}

extern "C" int cxs_qkv_rope(const void* proj, int32_t proj_stride, const int32_t* positions,
                            const float* inv_freq, int32_t tokens, int32_t q_heads,
                            int32_t kv_heads, void* query, void* records, int32_t records_stride,
                            void* current, int32_t current_stride, void* gates, void* stream) {
  if (tokens < 0 || q_heads < 1 || kv_heads < 1)
    return set_error(CXS_ERR_INVALID, "invalid qkv_rope geometry");
  if (!tokens) return CXS_OK;
  qkv_rope_kernel<<<tokens, 256, 0, (cudaStream_t)stream>>>(
      (const __nv_bfloat16*)proj, proj_stride, positions, inv_freq, q_heads, kv_heads,
      (__nv_bfloat16*)query, (__nv_bfloat16*)records, records_stride, (__nv_bfloat16*)current,
      current_stride, (__nv_bfloat16*)gates);
  CXS_LAUNCH_CHECK("qkv_rope_kernel");
  return CXS_OK;
}

extern "C" int cxs_silu_mul(const void* gate_up, int32_t rows, int32_t ffn, void* out,
                            void* stream) {
  if (rows < 0 || ffn < 1) return set_error(CXS_ERR_INVALID, "invalid silu_mul geometry");
  long long total = (long long)rows * ffn;
  if (!total) return CXS_OK;
  silu_mul_kernel<<<(unsigned)((total + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
      (const __nv_bfloat16*)gate_up, ffn, (__nv_bfloat16*)out, total);
  CXS_LAUNCH_CHECK("silu_mul_kernel");
  return CXS_OK;
}
