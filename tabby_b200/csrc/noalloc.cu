// tabby_sample_rows_noalloc: the batched sampler without any device allocation.
//
// Some callers cannot call cudaMalloc at all: code running under an allocator that
// owns the whole device memory pool, plug-in hosts that forbid allocation on their
// request path, or capture-style callers that must not add allocations between steps.
// For them this entry point runs the same row kernel as tabby_sample_rows_async but
// keeps the kernel's global scratch (per-row counters and per-slice candidate lists) in
// a file-scope device array instead of a handle's cudaMalloc'd buffers.
//
// Limits: max_top_k <= TABBY_NOALLOC_MAX_TOP_K (256); rows are processed in launches of
// at most kNoAllocRows. The array lives on every GPU that loads this library until the
// process exits.
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <mutex>

#include "sampler_internal.h"
#include "tabby_sample.h"

namespace tabby {
namespace {

constexpr int kNoAllocRows = 32;  // rows a launch; larger batches run in several launches
constexpr size_t kScratchBytes = Scratch::layout_bytes(kNoAllocRows);  // ~5.4 MB

// The scratch itself. In host code this name is only a stand-in for the symbol; its
// device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
struct DeviceState {
  bool ready = false;
  unsigned char *scratch = nullptr;  // device address of g_noalloc_scratch on this device
  int sms = 0;
};
DeviceState g_devices[kMaxDevices];
std::mutex g_setup_mutex;

int fail(int status, const char *fmt, ...) {
  char msg[256];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(msg, sizeof(msg), fmt, ap);
  va_end(ap);
  return set_error(status, msg);
}

// Once per device, with that device current: resolve the array's device address.
int setup_current_device(DeviceState **out) {
  int dev = -1;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return fail(TABBY_ECUDA, "cudaGetDevice: %s", cudaGetErrorString(err));
  if (dev < 0 || dev >= kMaxDevices) return fail(TABBY_EINVAL, "device %d unsupported", dev);
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  DeviceState &st = g_devices[dev];
  if (!st.ready) {
    void *ptr = nullptr;
    err = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (err != cudaSuccess)
      return fail(TABBY_ECUDA, "cudaGetSymbolAddress: %s", cudaGetErrorString(err));
    int sms = 0;
    err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (err != cudaSuccess)
      return fail(TABBY_ECUDA, "cudaDeviceGetAttribute: %s", cudaGetErrorString(err));
    st.scratch = static_cast<unsigned char *>(ptr);
    st.sms = sms;
    st.ready = true;
  }
  *out = &st;
  return TABBY_OK;
}

}  // namespace
}  // namespace tabby

extern "C" int tabby_sample_rows_noalloc(const float *d_logits, int64_t row_stride, int32_t rows,
                                         int32_t vocab, int32_t max_top_k,
                                         const tabby_sampling_params *d_params,
                                         const double *d_uniforms, tabby_sample_outcome *d_out,
                                         int32_t *d_topk_ids, float *d_topk_values,
                                         int32_t topk_ld, void *stream) {
  using namespace tabby;
  if (rows < 0) return fail(TABBY_EINVAL, "rows must be >= 0, got %d", rows);
  if (vocab < 1 || vocab > (1 << 30))
    return fail(TABBY_EINVAL, "vocab must be in [1, 2^30], got %d", vocab);
  if (row_stride < vocab) return fail(TABBY_EINVAL, "row_stride must be >= vocab");
  if (max_top_k < 1 || max_top_k > TABBY_NOALLOC_MAX_TOP_K)
    return fail(TABBY_EINVAL,
                "max_top_k %d is beyond this entry point's limit of %d (its scratch array is "
                "fixed); use tabby_sample_rows_async with a sampler handle for larger pools",
                max_top_k, TABBY_NOALLOC_MAX_TOP_K);
  if (rows > 0 && (!d_logits || !d_params || !d_uniforms || !d_out))
    return fail(TABBY_EINVAL, "logits, params, uniforms and out must not be NULL");
  if ((reinterpret_cast<uintptr_t>(d_logits) & 3u) != 0)
    return fail(TABBY_EINVAL, "logits must be 4-byte aligned");
  if ((d_topk_ids || d_topk_values) && topk_ld < max_top_k)
    return fail(TABBY_EINVAL, "topk_ld (%d) must be >= max_top_k (%d)", topk_ld, max_top_k);
  if (rows == 0) return TABBY_OK;
  DeviceState *st = nullptr;
  int rc = setup_current_device(&st);
  if (rc) return rc;
  const Scratch scr = Scratch::carve(st->scratch, kNoAllocRows);
  cudaStream_t q = (cudaStream_t)stream;

  RowLaunch l;
  l.logits = d_logits;
  l.row_stride = row_stride;
  l.vocab = vocab;
  l.mode = kModeSample;
  l.cap = max_top_k;
  l.params = d_params;
  l.uniforms = d_uniforms;
  l.out = d_out;
  l.topk_ids = d_topk_ids;
  l.topk_values = d_topk_values;
  l.topk_ld = topk_ld;

  // No clearing is needed: the array is zero when the library loads; every launch resets
  // a row's counters before using the row (the plan phase of chunked launches, the unit
  // start of whole-row launches), its last unit take resets the unit counter, and plan
  // entries carry the launch number kept in the array.
  cudaError_t err = cudaSuccess;
  for (int32_t r0 = 0; r0 < rows; r0 += kNoAllocRows) {
    RowLaunch b = l;
    b.rows = std::min(rows - r0, (int32_t)kNoAllocRows);
    b.logits = d_logits + (int64_t)r0 * row_stride;
    b.params = d_params + r0;
    b.uniforms = d_uniforms + r0;
    b.out = d_out + r0;
    if (b.topk_ids) b.topk_ids = d_topk_ids + (int64_t)r0 * topk_ld;
    if (b.topk_values) b.topk_values = d_topk_values + (int64_t)r0 * topk_ld;
    RowGeometry geo;
    err = plan_rows(st->sms, b.rows, vocab, max_top_k, &geo);
    if (err != cudaSuccess) return fail(TABBY_ECUDA, "row pass setup: %s", cudaGetErrorString(err));
    err = launch_rows(b, geo, scr, q);
    if (err != cudaSuccess)
      return fail(TABBY_ECUDA, "row kernel launch: %s", cudaGetErrorString(err));
  }
  return TABBY_OK;
}
