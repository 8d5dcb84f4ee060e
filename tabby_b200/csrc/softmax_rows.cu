// Row softmax with the reference's causal mask, in place (softmax_rows.wgsl:1-60,
// restated on the CPU by cpu.ts:softmaxRows). It is the kernel next to the sampling pass
// in the reference's decode step: the same max / sum-exp skeleton over attention scores.
//
// Row r of an [n_rows, row_len] fp32 tensor keeps its first `valid` entries, with
// valid = causal_offset + (r % causal_period) + 1 when causal_period != 0 (rows laid out
// as (head, query)) and valid = row_len otherwise; those become exp(x - max) / sum, the
// rest become 0.
//
// Roofline: HBM-bound, 8 bytes per element (one read, one write). One CTA of 256 threads
// per row; rows of up to 8192 valid entries stay in registers between the max, the sum
// and the write (one read of the row), longer rows are read three times.
#include <cuda_runtime.h>
#include <stdint.h>

#include "sampler_internal.h"
#include "tabby_sample.h"

namespace tabby {
namespace {

constexpr int kSmThreads = 256;
constexpr int kSmWarps = kSmThreads / 32;

__device__ __forceinline__ int valid_len(int row, int row_len, int period, int offset) {
  return period != 0 ? offset + (row % period) + 1 : row_len;
}

// Block-wide max / sum of one value a thread (block-uniform call).
__device__ __forceinline__ float block_max(float v, float *red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();  // red is free (its previous use is complete)
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  v = red[0];
#pragma unroll
  for (int w = 1; w < kSmWarps; w++) v = fmaxf(v, red[w]);
  return v;
}
__device__ __forceinline__ float block_sum(float v, float *red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  v = 0.f;
#pragma unroll
  for (int w = 0; w < kSmWarps; w++) v += red[w];
  return v;
}

// Rows whose valid part fits in VPT values a thread: one read, one write.
template <int VPT>
__global__ void __launch_bounds__(kSmThreads) softmax_rows_reg(float *x, int n_rows, int row_len,
                                                               int period, int offset) {
  __shared__ float red[kSmWarps];
  const int row = blockIdx.x;
  const int tid = threadIdx.x;
  float *p = x + (int64_t)row * row_len;
  const int valid = min(valid_len(row, row_len, period, offset), row_len);
  float v[VPT];
  float m = -__int_as_float(0x7f800000);
#pragma unroll
  for (int j = 0; j < VPT; j++) {
    const int i = tid + j * kSmThreads;
    v[j] = i < valid ? p[i] : -__int_as_float(0x7f800000);
    m = fmaxf(m, v[j]);
  }
  m = block_max(m, red);
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < VPT; j++) {
    const int i = tid + j * kSmThreads;
    v[j] = i < valid ? expf(v[j] - m) : 0.f;
    s += v[j];
  }
  s = block_sum(s, red);
  const float inv = 1.0f / s;
#pragma unroll
  for (int j = 0; j < VPT; j++) {
    const int i = tid + j * kSmThreads;
    if (i < valid) p[i] = v[j] * inv;
  }
  for (int i = valid + tid; i < row_len; i += kSmThreads) p[i] = 0.f;  // masked tail
}

// The same with float4 loads and stores (row_len a multiple of 4, x 16-byte aligned):
// V4 groups of four a thread; kept entries and the zeroed tail are written together.
template <int V4>
__global__ void __launch_bounds__(kSmThreads) softmax_rows_reg4(float *x, int n_rows,
                                                                int row_len, int period,
                                                                int offset) {
  __shared__ float red[kSmWarps];
  const int row = blockIdx.x;
  const int tid = threadIdx.x;
  float4 *p = reinterpret_cast<float4 *>(x + (int64_t)row * row_len);
  const int valid = min(valid_len(row, row_len, period, offset), row_len);
  const int nv4 = (valid + 3) >> 2;    // groups holding kept entries
  const int n4 = row_len >> 2;         // groups of the row
  const float ninf = -__int_as_float(0x7f800000);
  float4 v[V4];
  float m = ninf;
#pragma unroll
  for (int j = 0; j < V4; j++) {
    const int g = tid + j * kSmThreads;
    v[j] = make_float4(ninf, ninf, ninf, ninf);
    if (g < nv4) {
      v[j] = p[g];
      const int e = 4 * g;  // entries past the prefix do not count
      if (e + 1 >= valid) v[j].y = ninf;
      if (e + 2 >= valid) v[j].z = ninf;
      if (e + 3 >= valid) v[j].w = ninf;
    }
    m = fmaxf(m, fmaxf(fmaxf(v[j].x, v[j].y), fmaxf(v[j].z, v[j].w)));
  }
  m = block_max(m, red);
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < V4; j++) {
    const int g = tid + j * kSmThreads;
    const int e = 4 * g;
    v[j].x = e < valid ? expf(v[j].x - m) : 0.f;
    v[j].y = e + 1 < valid ? expf(v[j].y - m) : 0.f;
    v[j].z = e + 2 < valid ? expf(v[j].z - m) : 0.f;
    v[j].w = e + 3 < valid ? expf(v[j].w - m) : 0.f;
    s += (v[j].x + v[j].y) + (v[j].z + v[j].w);
  }
  s = block_sum(s, red);
  const float inv = 1.0f / s;
#pragma unroll
  for (int j = 0; j < V4; j++) {
    const int g = tid + j * kSmThreads;
    if (g < n4)  // zeros past the prefix come from the masked exps above
      p[g] = make_float4(v[j].x * inv, v[j].y * inv, v[j].z * inv, v[j].w * inv);
  }
  for (int g = V4 * kSmThreads + tid; g < n4; g += kSmThreads)
    p[g] = make_float4(0.f, 0.f, 0.f, 0.f);  // masked tail beyond the registers
}

// Longer rows: max, then sum of exp, then the write, each a pass over the row.
__global__ void __launch_bounds__(kSmThreads) softmax_rows_loop(float *x, int n_rows, int row_len,
                                                                int period, int offset) {
  __shared__ float red[kSmWarps];
  const int row = blockIdx.x;
  const int tid = threadIdx.x;
  float *p = x + (int64_t)row * row_len;
  const int valid = min(valid_len(row, row_len, period, offset), row_len);
  float m = -__int_as_float(0x7f800000);
  for (int i = tid; i < valid; i += kSmThreads) m = fmaxf(m, p[i]);
  m = block_max(m, red);
  float s = 0.f;
  for (int i = tid; i < valid; i += kSmThreads) s += expf(p[i] - m);
  s = block_sum(s, red);
  const float inv = 1.0f / s;
  for (int i = tid; i < valid; i += kSmThreads) p[i] = expf(p[i] - m) * inv;
  for (int i = valid + tid; i < row_len; i += kSmThreads) p[i] = 0.f;
}

}  // namespace
}  // namespace tabby

extern "C" int tabby_softmax_rows_async(float *d_x, int32_t n_rows, int32_t row_len,
                                        int32_t causal_period, int32_t causal_offset,
                                        void *stream) {
  using namespace tabby;
  if (n_rows < 0 || row_len < 1)
    return set_error(TABBY_EINVAL, "softmax_rows: n_rows must be >= 0 and row_len >= 1");
  if (causal_period < 0 || causal_offset < 0)
    return set_error(TABBY_EINVAL, "softmax_rows: causal_period and causal_offset must be >= 0");
  // The reference reads past the row when offset + period > row_len; refused here.
  if (causal_period != 0 && (int64_t)causal_offset + causal_period > row_len)
    return set_error(TABBY_EINVAL, "softmax_rows: causal_offset + causal_period > row_len");
  if (n_rows == 0) return TABBY_OK;
  if (!d_x || (reinterpret_cast<uintptr_t>(d_x) & 3u))
    return set_error(TABBY_EINVAL, "softmax_rows: x must be a non-NULL 4-byte aligned pointer");
  const int max_valid = causal_period != 0 ? causal_offset + causal_period : row_len;
  cudaStream_t s = (cudaStream_t)stream;
  const dim3 grid((unsigned)n_rows);
  const bool vec = (row_len & 3) == 0 && (reinterpret_cast<uintptr_t>(d_x) & 15u) == 0;
  if (vec && max_valid <= 4 * kSmThreads)
    softmax_rows_reg4<1><<<grid, kSmThreads, 0, s>>>(d_x, n_rows, row_len, causal_period,
                                                     causal_offset);
  else if (vec && max_valid <= 16 * kSmThreads)
    softmax_rows_reg4<4><<<grid, kSmThreads, 0, s>>>(d_x, n_rows, row_len, causal_period,
                                                     causal_offset);
  else if (vec && max_valid <= 32 * kSmThreads)
    softmax_rows_reg4<8><<<grid, kSmThreads, 0, s>>>(d_x, n_rows, row_len, causal_period,
                                                     causal_offset);
  else if (max_valid <= 4 * kSmThreads)
    softmax_rows_reg<4><<<grid, kSmThreads, 0, s>>>(d_x, n_rows, row_len, causal_period,
                                                    causal_offset);
  else if (max_valid <= 16 * kSmThreads)
    softmax_rows_reg<16><<<grid, kSmThreads, 0, s>>>(d_x, n_rows, row_len, causal_period,
                                                     causal_offset);
  else if (max_valid <= 32 * kSmThreads)
    softmax_rows_reg<32><<<grid, kSmThreads, 0, s>>>(d_x, n_rows, row_len, causal_period,
                                                     causal_offset);
  else
    softmax_rows_loop<<<grid, kSmThreads, 0, s>>>(d_x, n_rows, row_len, causal_period,
                                                  causal_offset);
  const cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return set_error(TABBY_ECUDA, cudaGetErrorString(err));
  return TABBY_OK;
}
