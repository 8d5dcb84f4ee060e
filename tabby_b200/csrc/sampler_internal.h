// Internal launch interface between the C ABI (capi.cu) and the kernels
// (sampler_kernels.cu). Not installed; the public surface is include/tabby_sample.h.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "tabby_sample.h"

namespace tabby {

enum Mode : int32_t {
  kModeSample = 0,  // pool rule + top-k + sampleFromTopK  -> tabby_sample_outcome
  kModeTopK = 1,    // fixed k -> [maxLogit, sumExp, (value, index) * k] block
  kModeShard = 2    // fixed k = 64, global indices -> block for the all-gather
};

struct RowLaunch {
  const float *logits = nullptr;
  int64_t row_stride = 0;
  int32_t rows = 0;
  int32_t vocab = 0;
  int32_t mode = kModeSample;
  int32_t cap = TABBY_DEFAULT_MAX_TOP_K;  // pool-rule cap (kModeSample)
  int32_t fixed_k = 0;                    // kModeTopK / kModeShard
  int64_t index_offset = 0;               // kModeShard
  const tabby_sampling_params *params = nullptr;
  const double *uniforms = nullptr;
  tabby_sample_outcome *out = nullptr;
  int32_t *topk_ids = nullptr;
  float *topk_values = nullptr;
  int32_t topk_ld = 0;
  float *block = nullptr;
  int32_t block_ld = 0;
};

struct MergeLaunch {
  const float *gathered = nullptr;
  int32_t shards = 0;
  int32_t rows = 0;
  int32_t block_ld = 0;
  const tabby_sampling_params *params = nullptr;
  const double *uniforms = nullptr;
  tabby_sample_outcome *out = nullptr;
  int32_t *topk_ids = nullptr;
  float *topk_values = nullptr;
  int32_t topk_ld = 0;
};

// Geometry of one stream_kernel launch: the row is cut into `nslices` slices of
// `slice` logits, one CTA each.
struct RowGeometry {
  int32_t slice = 0;        // logits per CTA (multiple of 4)
  int32_t nslices = 0;      // CTAs per row
  int32_t data_floats = 0;  // shared-memory staging region, floats
  size_t smem_bytes = 0;
};

// Global scratch of the row kernel, owned by the sampler handle. Row counters and
// thresholds must be zero before a launch; the kernel leaves them zero again.
struct Scratch {
  uint32_t *row_count = nullptr;             // [max_rows] slices finished
  unsigned long long *row_tau = nullptr;     // [max_rows] exact lower bound of the k-th
  float2 *slice_stats = nullptr;             // [max_rows * max_slices] (max, sum-exp)
  uint2 *slice_meta = nullptr;               // [max_rows * max_slices] (count, flags)
  unsigned long long *slice_cand = nullptr;  // [max_rows * max_slices * cand_ld]
  int32_t cand_ld = 0;                       // candidates a slice may write (>= k)
  int32_t max_rows = 0;
  int32_t max_slices = 0;
};

int32_t max_slices(int32_t vocab, int32_t cap);
cudaError_t plan_rows(int32_t sms, int32_t rows, int32_t vocab, int32_t cap, RowGeometry *geo);
cudaError_t launch_rows(const RowLaunch &a, const RowGeometry &geo, const Scratch &scr,
                        cudaStream_t stream);
cudaError_t launch_merge(const MergeLaunch &a, cudaStream_t stream);

// Records `msg` as the calling thread's tabby_last_error() and returns `status`.
int set_error(int status, const char *msg);

// Host float64 finalize with the device's arithmetic (sampler.ts:147-212).
int host_sample_from_topk(const int32_t *ids, const float *logits, int32_t n, float max_logit,
                          float sum_exp, double temperature, double top_p, double u,
                          tabby_sample_outcome *out);

}  // namespace tabby
