// C ABI of libtabbysample.so (declared in include/tabby_sample.h).
//
// Host-side validation mirrors the reference's errors: ForwardError for a k outside
// [0, MAX_TOP_K] (xOAviOx/tabby src/engine/forward.ts:348-351), 'sampleFromTopK: empty
// candidate set' (src/engine/sampler.ts:153), RangeError for launch limits
// (src/engine/kernels.ts:370-388). Errors are status codes plus a thread-local message;
// nothing aborts.
#include <cuda_runtime.h>
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>

#include "sampler_internal.h"
#include "tabby_sample.h"

using tabby::MergeLaunch;
using tabby::RowGeometry;
using tabby::RowLaunch;
using tabby::Scratch;
using tabby::DeviceScope;

struct tabby_sampler {
  int32_t device;
  int32_t cap;
  int32_t max_rows;
  int32_t max_vocab;
  int32_t sms;
  Scratch scratch;     // per-row state of the row pass, carved from scratch_mem
  void *scratch_mem;
  cudaStream_t stream;  // used by the host-buffer entry points
  float *d_logits;
  tabby_sampling_params *d_params;
  double *d_uniforms;
  tabby_sample_outcome *d_out;
  int32_t *d_ids;
  float *d_values;
};

namespace {

thread_local char g_error[512] = "";

int fail(int status, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_error, sizeof(g_error), fmt, ap);
  va_end(ap);
  return status;
}

int cuda_fail(cudaError_t err, const char *what) {
  return fail(TABBY_ECUDA, "%s: %s (%s)", what, cudaGetErrorName(err), cudaGetErrorString(err));
}


bool aligned4(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 3u) == 0; }

int check_rows(const tabby_sampler *s, const float *logits, int64_t row_stride, int32_t rows,
               int32_t vocab) {
  if (!s) return fail(TABBY_EINVAL, "sampler is NULL");
  if (rows < 0) return fail(TABBY_EINVAL, "rows must be >= 0, got %d", rows);
  if (vocab < 1 || vocab > (1 << 30))
    return fail(TABBY_EINVAL, "vocab must be in [1, 2^30], got %d", vocab);
  if (row_stride < vocab)
    return fail(TABBY_EINVAL, "row_stride (%lld) must be >= vocab (%d)", (long long)row_stride,
                vocab);
  if (rows > 0 && !logits) return fail(TABBY_EINVAL, "logits is NULL");
  if (!aligned4(logits)) return fail(TABBY_EINVAL, "logits must be 4-byte aligned");
  return TABBY_OK;
}

int check_params_host(const tabby_sampling_params *p, int32_t rows) {
  for (int32_t r = 0; r < rows; r++) {
    if (isnan(p[r].temperature) || isnan(p[r].top_p))
      return fail(TABBY_EINVAL, "row %d: temperature and top_p must not be NaN", r);
  }
  return TABBY_OK;
}

// Launches the row kernel over `rows` rows in batches of the scratch capacity.
cudaError_t plan_and_launch(tabby_sampler *s, const RowLaunch &l, cudaStream_t stream) {
  for (int32_t r0 = 0; r0 < l.rows; r0 += s->scratch.max_rows) {
    RowLaunch b = l;
    b.rows = std::min(l.rows - r0, s->scratch.max_rows);
    b.logits = l.logits + (int64_t)r0 * l.row_stride;
    if (b.params) b.params = l.params + r0;
    if (b.uniforms) b.uniforms = l.uniforms + r0;
    if (b.rng_state) b.rng_state = l.rng_state + r0;
    if (b.out) b.out = l.out + r0;
    if (b.topk_ids) b.topk_ids = l.topk_ids + (int64_t)r0 * l.topk_ld;
    if (b.topk_values) b.topk_values = l.topk_values + (int64_t)r0 * l.topk_ld;
    if (b.block) b.block = l.block + (int64_t)r0 * l.block_ld;
    RowGeometry geo;
    cudaError_t err = tabby::plan_rows(s->sms, b.rows, b.vocab, s->cap, &geo);
    if (err != cudaSuccess) return err;
    err = tabby::launch_rows(b, geo, s->scratch, stream);
    if (err != cudaSuccess) return err;
  }
  return cudaSuccess;
}

int check_vocab_capacity(const tabby_sampler *s, int32_t vocab) {
  if (vocab > s->max_vocab)
    return fail(TABBY_EINVAL, "vocab %d exceeds the handle's max_vocab %d", vocab, s->max_vocab);
  return TABBY_OK;
}

}  // namespace

int tabby::set_error(int status, const char *msg) { return fail(status, "%s", msg); }

extern "C" {

int32_t tabby_abi_version(void) { return TABBY_ABI_VERSION; }

const char *tabby_last_error(void) { return g_error; }

int32_t tabby_pool_size(double temperature, int32_t top_k, int32_t max_top_k) {
  if (temperature <= 0) return 1;
  int32_t k = top_k != 0 ? top_k : max_top_k;
  if (k < 1) k = 1;
  return k < max_top_k ? k : max_top_k;
}

int tabby_sampler_create(const tabby_sampler_config *config, tabby_sampler **out) {
  if (!config || !out) return fail(TABBY_EINVAL, "config and out must not be NULL");
  *out = nullptr;
  tabby_sampler_config c = *config;
  if (c.max_top_k == 0) c.max_top_k = TABBY_DEFAULT_MAX_TOP_K;
  if (c.max_rows == 0) c.max_rows = 256;
  if (c.max_vocab == 0) c.max_vocab = 151936;
  if (c.max_top_k < 1 || c.max_top_k > TABBY_MAX_TOP_K_LIMIT)
    return fail(TABBY_EINVAL, "max_top_k must be in [1, %d], got %d", TABBY_MAX_TOP_K_LIMIT,
                c.max_top_k);
  if (c.max_rows < 1 || c.max_vocab < 1 || c.max_vocab > (1 << 30))
    return fail(TABBY_EINVAL, "max_rows and max_vocab must be positive (max_vocab <= 2^30)");
  int ndev = 0;
  cudaError_t err = cudaGetDeviceCount(&ndev);
  if (err != cudaSuccess) return cuda_fail(err, "cudaGetDeviceCount");
  if (c.device < 0 || c.device >= ndev)
    return fail(TABBY_EINVAL, "device %d out of range (%d devices)", c.device, ndev);
  DeviceScope scope(c.device);
  if (scope.err != cudaSuccess) return cuda_fail(scope.err, "cudaSetDevice");
  cudaDeviceProp prop;
  err = cudaGetDeviceProperties(&prop, c.device);
  if (err != cudaSuccess) return cuda_fail(err, "cudaGetDeviceProperties");
  if (prop.major < 10)
    return fail(TABBY_ECUDA, "device %d is sm_%d%d; this library is built for sm_100a",
                c.device, prop.major, prop.minor);

  tabby_sampler *s = new tabby_sampler();
  memset(s, 0, sizeof(*s));
  s->device = c.device;
  s->cap = c.max_top_k;
  s->max_rows = c.max_rows;
  s->max_vocab = c.max_vocab;
  s->sms = prop.multiProcessorCount;
  const size_t nlog = (size_t)c.max_rows * (size_t)c.max_vocab;
  // Row state for at most 1024 rows a launch; larger batches run in several launches.
  const int32_t scratch_rows = std::min(c.max_rows, (int32_t)1024);
  if ((err = cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking)) != cudaSuccess ||
      (err = cudaMalloc(&s->d_logits, nlog * sizeof(float))) != cudaSuccess ||
      (err = cudaMalloc(&s->d_params, (size_t)c.max_rows * sizeof(tabby_sampling_params))) !=
          cudaSuccess ||
      (err = cudaMalloc(&s->d_uniforms, (size_t)c.max_rows * sizeof(double))) != cudaSuccess ||
      (err = cudaMalloc(&s->d_out, (size_t)c.max_rows * sizeof(tabby_sample_outcome))) !=
          cudaSuccess ||
      (err = cudaMalloc(&s->d_ids, (size_t)c.max_rows * c.max_top_k * sizeof(int32_t))) !=
          cudaSuccess ||
      (err = cudaMalloc(&s->d_values, (size_t)c.max_rows * c.max_top_k * sizeof(float))) !=
          cudaSuccess ||
      (err = cudaMalloc(&s->scratch_mem, Scratch::bytes(scratch_rows))) != cudaSuccess ||
      (err = cudaMemset(s->scratch_mem, 0, Scratch::bytes(scratch_rows))) != cudaSuccess ||
      (err = cudaDeviceSynchronize()) != cudaSuccess) {
    tabby_sampler_destroy(s);
    cudaGetLastError();
    return fail(TABBY_ENOMEM, "allocation of sampler buffers failed: %s", cudaGetErrorString(err));
  }
  s->scratch = Scratch::carve(s->scratch_mem, scratch_rows);
  *out = s;
  return TABBY_OK;
}

int tabby_sampler_destroy(tabby_sampler *s) {
  if (!s) return TABBY_OK;
  DeviceScope scope(s->device);
  if (s->d_logits) cudaFree(s->d_logits);
  if (s->d_params) cudaFree(s->d_params);
  if (s->d_uniforms) cudaFree(s->d_uniforms);
  if (s->d_out) cudaFree(s->d_out);
  if (s->d_ids) cudaFree(s->d_ids);
  if (s->d_values) cudaFree(s->d_values);
  if (s->scratch_mem) cudaFree(s->scratch_mem);
  if (s->stream) cudaStreamDestroy(s->stream);
  delete s;
  return TABBY_OK;
}

int tabby_sample_rows_async(tabby_sampler *s, const float *d_logits, int64_t row_stride,
                            int32_t rows, int32_t vocab, const tabby_sampling_params *d_params,
                            const double *d_uniforms, tabby_sample_outcome *d_out,
                            int32_t *d_topk_ids, float *d_topk_values, int32_t topk_ld,
                            void *stream) {
  int st = check_rows(s, d_logits, row_stride, rows, vocab);
  if (st) return st;
  if (rows > 0 && (!d_params || !d_uniforms || !d_out))
    return fail(TABBY_EINVAL, "params, uniforms and out must not be NULL");
  if ((d_topk_ids || d_topk_values) && topk_ld < s->cap)
    return fail(TABBY_EINVAL, "topk_ld (%d) must be >= max_top_k (%d)", topk_ld, s->cap);
  if ((st = check_vocab_capacity(s, vocab))) return st;
  DeviceScope scope(s->device);
  if (scope.err != cudaSuccess) return cuda_fail(scope.err, "cudaSetDevice");
  RowLaunch l;
  l.logits = d_logits;
  l.row_stride = row_stride;
  l.rows = rows;
  l.vocab = vocab;
  l.mode = tabby::kModeSample;
  l.cap = s->cap;
  l.params = d_params;
  l.uniforms = d_uniforms;
  l.out = d_out;
  l.topk_ids = d_topk_ids;
  l.topk_values = d_topk_values;
  l.topk_ld = topk_ld;
  cudaError_t err = plan_and_launch(s, l, (cudaStream_t)stream);
  if (err != cudaSuccess) return cuda_fail(err, "row_kernel launch");
  return TABBY_OK;
}

int tabby_sample_rows_rng_async(tabby_sampler *s, const float *d_logits, int64_t row_stride,
                                int32_t rows, int32_t vocab, const tabby_sampling_params *d_params,
                                uint32_t *d_rng_state, tabby_sample_outcome *d_out,
                                int32_t *d_topk_ids, float *d_topk_values, int32_t topk_ld,
                                void *stream) {
  int st = check_rows(s, d_logits, row_stride, rows, vocab);
  if (st) return st;
  if (rows > 0 && (!d_params || !d_rng_state || !d_out))
    return fail(TABBY_EINVAL, "params, rng_state and out must not be NULL");
  if ((d_topk_ids || d_topk_values) && topk_ld < s->cap)
    return fail(TABBY_EINVAL, "topk_ld (%d) must be >= max_top_k (%d)", topk_ld, s->cap);
  if ((st = check_vocab_capacity(s, vocab))) return st;
  DeviceScope scope(s->device);
  if (scope.err != cudaSuccess) return cuda_fail(scope.err, "cudaSetDevice");
  RowLaunch l;
  l.logits = d_logits;
  l.row_stride = row_stride;
  l.rows = rows;
  l.vocab = vocab;
  l.mode = tabby::kModeSample;
  l.cap = s->cap;
  l.params = d_params;
  l.rng_state = d_rng_state;
  l.out = d_out;
  l.topk_ids = d_topk_ids;
  l.topk_values = d_topk_values;
  l.topk_ld = topk_ld;
  cudaError_t err = plan_and_launch(s, l, (cudaStream_t)stream);
  if (err != cudaSuccess) return cuda_fail(err, "row_kernel launch");
  return TABBY_OK;
}

int tabby_sample_rows_debug_async(tabby_sampler *s, const float *d_logits, int64_t row_stride,
                                  int32_t rows, int32_t vocab,
                                  const tabby_sampling_params *d_params,
                                  const double *d_uniforms, tabby_sample_outcome *d_out,
                                  uint32_t spin_limit, int32_t withhold_row, void *stream) {
  int st = check_rows(s, d_logits, row_stride, rows, vocab);
  if (st) return st;
  if (rows > 0 && (!d_params || !d_uniforms || !d_out))
    return fail(TABBY_EINVAL, "params, uniforms and out must not be NULL");
  if (spin_limit < 1) return fail(TABBY_EINVAL, "spin_limit must be >= 1");
  if ((st = check_vocab_capacity(s, vocab))) return st;
  DeviceScope scope(s->device);
  if (scope.err != cudaSuccess) return cuda_fail(scope.err, "cudaSetDevice");
  RowLaunch l;
  l.logits = d_logits;
  l.row_stride = row_stride;
  l.rows = rows;
  l.vocab = vocab;
  l.mode = tabby::kModeSample;
  l.cap = s->cap;
  l.params = d_params;
  l.uniforms = d_uniforms;
  l.out = d_out;
  l.spin_limit = spin_limit;
  l.withhold_row = withhold_row;
  cudaError_t err = plan_and_launch(s, l, (cudaStream_t)stream);
  if (err != cudaSuccess) return cuda_fail(err, "row_kernel launch");
  return TABBY_OK;
}

int tabby_sample_rows(tabby_sampler *s, const float *h_logits, int64_t row_stride, int32_t rows,
                      int32_t vocab, const tabby_sampling_params *h_params,
                      const double *h_uniforms, tabby_sample_outcome *h_out,
                      int32_t *h_topk_ids, float *h_topk_values, int32_t topk_ld) {
  int st = check_rows(s, h_logits, row_stride, rows, vocab);
  if (st) return st;
  if (rows > s->max_rows || vocab > s->max_vocab)
    return fail(TABBY_EINVAL, "rows %d / vocab %d exceed the handle's capacity %d / %d", rows,
                vocab, s->max_rows, s->max_vocab);
  if (rows > 0 && (!h_params || !h_uniforms || !h_out))
    return fail(TABBY_EINVAL, "params, uniforms and out must not be NULL");
  if ((h_topk_ids || h_topk_values) && topk_ld < s->cap)
    return fail(TABBY_EINVAL, "topk_ld (%d) must be >= max_top_k (%d)", topk_ld, s->cap);
  if ((st = check_params_host(h_params, rows))) return st;
  if (rows == 0) return TABBY_OK;
  DeviceScope scope(s->device);
  if (scope.err != cudaSuccess) return cuda_fail(scope.err, "cudaSetDevice");
  cudaStream_t q = s->stream;
  cudaError_t err;
  if (row_stride == vocab)
    err = cudaMemcpyAsync(s->d_logits, h_logits, (size_t)rows * vocab * sizeof(float),
                          cudaMemcpyHostToDevice, q);
  else
    err = cudaMemcpy2DAsync(s->d_logits, (size_t)vocab * sizeof(float), h_logits,
                            (size_t)row_stride * sizeof(float), (size_t)vocab * sizeof(float),
                            (size_t)rows, cudaMemcpyHostToDevice, q);
  if (err != cudaSuccess) return cuda_fail(err, "copy logits to device");
  if ((err = cudaMemcpyAsync(s->d_params, h_params, (size_t)rows * sizeof(*h_params),
                             cudaMemcpyHostToDevice, q)) != cudaSuccess ||
      (err = cudaMemcpyAsync(s->d_uniforms, h_uniforms, (size_t)rows * sizeof(double),
                             cudaMemcpyHostToDevice, q)) != cudaSuccess)
    return cuda_fail(err, "copy params to device");
  const bool want_topk = h_topk_ids || h_topk_values;
  st = tabby_sample_rows_async(s, s->d_logits, vocab, rows, vocab, s->d_params, s->d_uniforms,
                               s->d_out, want_topk ? s->d_ids : nullptr,
                               want_topk ? s->d_values : nullptr, s->cap, q);
  if (st) return st;
  if ((err = cudaMemcpyAsync(h_out, s->d_out, (size_t)rows * sizeof(*h_out),
                             cudaMemcpyDeviceToHost, q)) != cudaSuccess)
    return cuda_fail(err, "copy outcomes to host");
  if (h_topk_ids &&
      (err = cudaMemcpy2DAsync(h_topk_ids, (size_t)topk_ld * 4, s->d_ids, (size_t)s->cap * 4,
                               (size_t)s->cap * 4, (size_t)rows, cudaMemcpyDeviceToHost, q)) !=
          cudaSuccess)
    return cuda_fail(err, "copy candidate ids to host");
  if (h_topk_values &&
      (err = cudaMemcpy2DAsync(h_topk_values, (size_t)topk_ld * 4, s->d_values,
                               (size_t)s->cap * 4, (size_t)s->cap * 4, (size_t)rows,
                               cudaMemcpyDeviceToHost, q)) != cudaSuccess)
    return cuda_fail(err, "copy candidate values to host");
  if ((err = cudaStreamSynchronize(q)) != cudaSuccess) return cuda_fail(err, "synchronize");
  for (int32_t r = 0; r < rows; r++)
    if (h_out[r].status != TABBY_OK)
      return fail(h_out[r].status, "row %d: %s", r,
                  h_out[r].status == TABBY_EINPUT
                      ? "logits hold NaN, +-inf or a value <= -3.0e38"
                  : h_out[r].status == TABBY_EINVAL ? "temperature or top_p is NaN"
                  : h_out[r].status == TABBY_ETIMEOUT
                      ? "a bounded device wait timed out"
                      : "sampleFromTopK: empty candidate set");
  return TABBY_OK;
}

int tabby_topk_rows_async(tabby_sampler *s, const float *d_logits, int64_t row_stride,
                          int32_t rows, int32_t vocab, int32_t k, float *d_block,
                          int32_t block_ld, void *stream) {
  int st = check_rows(s, d_logits, row_stride, rows, vocab);
  if (st) return st;
  if (k < 0 || k > s->cap)
    return fail(TABBY_EINVAL, "topK must be between 0 and %d, got %d", s->cap, k);
  if (k > vocab) return fail(TABBY_EINVAL, "topK (%d) exceeds vocab (%d)", k, vocab);
  if (rows > 0 && !d_block) return fail(TABBY_EINVAL, "block is NULL");
  if (block_ld < 2 + 2 * k)
    return fail(TABBY_EINVAL, "block_ld (%d) must be >= 2 + 2k (%d)", block_ld, 2 + 2 * k);
  if ((st = check_vocab_capacity(s, vocab))) return st;
  DeviceScope scope(s->device);
  if (scope.err != cudaSuccess) return cuda_fail(scope.err, "cudaSetDevice");
  RowLaunch l;
  l.logits = d_logits;
  l.row_stride = row_stride;
  l.rows = rows;
  l.vocab = vocab;
  l.mode = tabby::kModeTopK;
  l.cap = s->cap;
  l.fixed_k = k;
  l.block = d_block;
  l.block_ld = block_ld;
  cudaError_t err = plan_and_launch(s, l, (cudaStream_t)stream);
  if (err != cudaSuccess) return cuda_fail(err, "row_kernel launch");
  return TABBY_OK;
}

int tabby_shard_local_async(tabby_sampler *s, const float *d_logits, int64_t row_stride,
                            int32_t rows, int32_t shard_vocab, int64_t vocab_offset,
                            float *d_block, int32_t block_ld, void *stream) {
  int st = check_rows(s, d_logits, row_stride, rows, shard_vocab);
  if (st) return st;
  if (vocab_offset < 0 || vocab_offset + shard_vocab > ((int64_t)1 << 31) - 1)
    return fail(TABBY_EINVAL, "vocab_offset %lld out of range", (long long)vocab_offset);
  if (rows > 0 && !d_block) return fail(TABBY_EINVAL, "block is NULL");
  if (block_ld < 2 + 2 * TABBY_SHARD_TOP_K)
    return fail(TABBY_EINVAL, "block_ld (%d) must be >= %d", block_ld, 2 + 2 * TABBY_SHARD_TOP_K);
  if ((st = check_vocab_capacity(s, shard_vocab))) return st;
  DeviceScope scope(s->device);
  if (scope.err != cudaSuccess) return cuda_fail(scope.err, "cudaSetDevice");
  RowLaunch l;
  l.logits = d_logits;
  l.row_stride = row_stride;
  l.rows = rows;
  l.vocab = shard_vocab;
  l.mode = tabby::kModeShard;
  l.cap = s->cap;
  l.fixed_k = TABBY_SHARD_TOP_K;
  l.index_offset = vocab_offset;
  l.block = d_block;
  l.block_ld = block_ld;
  cudaError_t err = plan_and_launch(s, l, (cudaStream_t)stream);
  if (err != cudaSuccess) return cuda_fail(err, "row_kernel launch");
  return TABBY_OK;
}

int tabby_shard_merge_async(tabby_sampler *s, const float *d_gathered, int32_t shards,
                            int32_t rows, int32_t block_ld, const tabby_sampling_params *d_params,
                            const double *d_uniforms, tabby_sample_outcome *d_out,
                            int32_t *d_topk_ids, float *d_topk_values, int32_t topk_ld,
                            void *stream) {
  if (!s) return fail(TABBY_EINVAL, "sampler is NULL");
  if (shards < 1 || shards > 16) return fail(TABBY_EINVAL, "shards must be in [1, 16]");
  if (rows < 0) return fail(TABBY_EINVAL, "rows must be >= 0");
  if (block_ld < 2 + 2 * TABBY_SHARD_TOP_K)
    return fail(TABBY_EINVAL, "block_ld (%d) must be >= %d", block_ld, 2 + 2 * TABBY_SHARD_TOP_K);
  if (rows > 0 && (!d_gathered || !d_params || !d_uniforms || !d_out))
    return fail(TABBY_EINVAL, "gathered, params, uniforms and out must not be NULL");
  if ((d_topk_ids || d_topk_values) && topk_ld < TABBY_SHARD_TOP_K)
    return fail(TABBY_EINVAL, "topk_ld (%d) must be >= %d", topk_ld, TABBY_SHARD_TOP_K);
  DeviceScope scope(s->device);
  if (scope.err != cudaSuccess) return cuda_fail(scope.err, "cudaSetDevice");
  MergeLaunch l;
  l.gathered = d_gathered;
  l.shards = shards;
  l.rows = rows;
  l.block_ld = block_ld;
  l.params = d_params;
  l.uniforms = d_uniforms;
  l.out = d_out;
  l.topk_ids = d_topk_ids;
  l.topk_values = d_topk_values;
  l.topk_ld = topk_ld;
  cudaError_t err = tabby::launch_merge(l, (cudaStream_t)stream);
  if (err != cudaSuccess) return cuda_fail(err, "merge_kernel launch");
  return TABBY_OK;
}

int tabby_sample_from_topk(const int32_t *ids, const float *logits, int32_t n, float max_logit,
                           float sum_exp, const tabby_sampling_params *params, double uniform,
                           tabby_sample_outcome *out) {
  if (!out || !params) return fail(TABBY_EINVAL, "params and out must not be NULL");
  if (n <= 0 || !ids || !logits) return fail(TABBY_EEMPTY, "sampleFromTopK: empty candidate set");
  if (isnan(params->temperature) || isnan(params->top_p))
    return fail(TABBY_EINVAL, "temperature and top_p must not be NaN");
  return tabby::host_sample_from_topk(ids, logits, n, max_logit, sum_exp, params->temperature,
                                      params->top_p, uniform, out);
}

}  // extern "C"
