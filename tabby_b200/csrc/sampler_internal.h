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
  uint32_t *rng_state = nullptr;  // kModeSample: per-row mulberry32 state on the device; u
                                  // is drawn and the state advanced in place (no uniforms)
  uint32_t spin_limit = 1u << 24;  // polls of the bounded wait for a row's plan entry
  int32_t withhold_row = -1;       // tests only: the plan of this row is never published
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

// The vocab-sharded merge with its exchange over peer memory (xmerge_kernel). Each rank's
// exchange buffer holds two block buffers [max_rows][block_ld] (a step writes the one of
// its epoch's parity) and `world` arrive words (slot q written by rank q with the epoch
// of the step whose blocks it has published).
struct XMergeLaunch {
  MergeLaunch m;  // rows = all rows; gathered unused; out = the caller's
  // Every rank's block buffer of this step, by rank (kernel parameters: no dependent load
  // to find them).
  const float *peer_blocks[TABBY_EXCHANGE_MAX_WORLD] = {};
  uint32_t *peer_flags[TABBY_EXCHANGE_MAX_WORLD] = {};  // every rank's arrive words
  uint32_t *flags = nullptr;                            // this rank's arrive words
  int32_t rank = 0;
  int32_t world = 1;
  uint32_t epoch = 0;
  uint64_t timeout_ns = 0;
};
cudaError_t launch_xmerge(const XMergeLaunch &l, cudaStream_t stream);

// Partial results of the fused LM-head kernel (lmhead.cu), per (row, CTA): the CTA's
// (max, sum-exp) of the row over its vocabulary range and its kLmCands best logits of the
// row as (raw float bits << 32 | vocab index); unused slots hold index 0xffffffff.
constexpr int32_t kLmCands = 64;
struct LmheadMergeLaunch {
  const float2 *stats = nullptr;               // [stat_n][stats_ld]: (max, sum-exp) entries
  int32_t stat_n = 0;
  int32_t stats_ld = 0;
  const unsigned long long *cands = nullptr;   // [rows][parts][kLmCands]
  int32_t parts = 0;
  int32_t rows = 0;
  int32_t vocab = 0;
  const tabby_sampling_params *params = nullptr;
  const double *uniforms = nullptr;
  uint32_t *rng_state = nullptr;
  tabby_sample_outcome *out = nullptr;
  int32_t *topk_ids = nullptr;
  float *topk_values = nullptr;
  int32_t topk_ld = 0;
  const uint32_t *error = nullptr;  // == epoch: a bounded wait of the fused kernel ran out
  // keep < kLmCands (the fast pass): each part kept only its best `keep`; the merge checks
  // that no part's last kept candidate lies above the row's k-th best and, where one does,
  // sets row_flag[row] and *any_flag to the epoch so the exact pass recomputes the row.
  // keep == kLmCands with row_flag set (the exact pass's merge): only the rows flagged with
  // this epoch are finished.
  int32_t keep = kLmCands;
  uint32_t *row_flag = nullptr;
  uint32_t *any_flag = nullptr;
  uint32_t epoch = 0;  // the call's tag: error, row_flag and any_flag hold the epoch they refer to
};
cudaError_t launch_lmhead_merge(const LmheadMergeLaunch &l, cudaStream_t stream);

// Geometry of one row pass: rows are cut into `nch` chunks of `chunk` logits; `grid`
// persistent CTAs work through the rows * nch (row, chunk) units.
struct RowGeometry {
  int32_t chunk = 0;  // logits a unit (multiple of 4)
  int32_t nch = 0;    // units a row
  int32_t grid = 0;   // CTAs of the row kernel
  int32_t whole = 0;  // 1: one CTA a row, threshold from the stream, no plan phase
  size_t smem_bytes = 0;
};

constexpr int32_t kScratchGroups = 8192;      // candidate groups a row may collect
constexpr int32_t kScratchChunks = 32;        // chunks a row may have (kMaxChunks)
constexpr int32_t kScratchWarps = 16;         // warps a CTA has

// Global scratch of the row pass for up to max_rows rows, carved from one device
// allocation (every section 256-byte aligned). It must be zero when first used; after
// that every launch resets the row counters it plans, the launch's last take of a unit
// resets the unit counter, and plan entries carry the launch's epoch, so no clearing is
// needed between launches. The epoch lives in the scratch itself (sched[2]): a chunked
// launch runs as epoch sched[2] + 1 (never 0) and its last take stores that number, so
// the kernel's arguments do not change from call to call and a captured CUDA graph
// replays correctly.
struct Scratch {
  uint32_t *sched = nullptr;                 // [4] unit counter, -, the last chunked
                                             // launch's epoch, -
  unsigned long long *pos_entry = nullptr;   // [max_rows][2] epoch-tagged plan by position
  uint32_t *row_done = nullptr;              // [max_rows] chunks finished
  uint32_t *warp_cnt = nullptr;              // [max_rows][kScratchChunks * kScratchWarps]
  uint32_t *row_flags = nullptr;             // [max_rows] bad input / overflow
  float *row_tf = nullptr;                   // [max_rows] estimated threshold
  float *row_tf_lo = nullptr;                // [max_rows] the re-filter's starting threshold
  float2 *warp_stats = nullptr;              // [max_rows][kScratchChunks][kScratchWarps]
  float4 *row_gval = nullptr;                // [max_rows][kScratchGroups] group values
  int32_t *row_gidx = nullptr;               // [max_rows][kScratchGroups] group first index
  int32_t max_rows = 0;

  static constexpr size_t section(size_t bytes) { return (bytes + 255) / 256 * 256; }
  static constexpr size_t layout_bytes(int32_t rows) {
    return section(16) + section(16 * (size_t)rows) + 4 * section(4 * (size_t)rows) +
           section(4 * (size_t)rows * kScratchChunks * kScratchWarps) +
           section(8 * (size_t)rows * kScratchChunks * kScratchWarps) +
           section(16 * (size_t)rows * kScratchGroups) + section(4 * (size_t)rows * kScratchGroups);
  }
  static size_t bytes(int32_t rows) { return layout_bytes(rows); }
  static Scratch carve(void *base, int32_t rows) {
    Scratch s;
    unsigned char *p = static_cast<unsigned char *>(base);
    const size_t r = (size_t)rows;
    s.sched = reinterpret_cast<uint32_t *>(p);
    p += section(16);
    s.pos_entry = reinterpret_cast<unsigned long long *>(p);
    p += section(16 * r);
    s.row_done = reinterpret_cast<uint32_t *>(p);
    p += section(4 * r);
    s.warp_cnt = reinterpret_cast<uint32_t *>(p);
    p += section(4 * r * kScratchChunks * kScratchWarps);
    s.row_flags = reinterpret_cast<uint32_t *>(p);
    p += section(4 * r);
    s.row_tf = reinterpret_cast<float *>(p);
    p += section(4 * r);
    s.row_tf_lo = reinterpret_cast<float *>(p);
    p += section(4 * r);
    s.warp_stats = reinterpret_cast<float2 *>(p);
    p += section(8 * r * kScratchChunks * kScratchWarps);
    s.row_gval = reinterpret_cast<float4 *>(p);
    p += section(16 * r * kScratchGroups);
    s.row_gidx = reinterpret_cast<int32_t *>(p);
    s.max_rows = rows;
    return s;
  }
};

cudaError_t plan_rows(int32_t sms, int32_t rows, int32_t vocab, int32_t cap, RowGeometry *geo);
cudaError_t launch_rows(const RowLaunch &a, const RowGeometry &geo, const Scratch &scr,
                        cudaStream_t stream);
cudaError_t launch_merge(const MergeLaunch &a, cudaStream_t stream);

// Makes a device current for the scope of a C-ABI call and restores the caller's.
struct DeviceScope {
  int prev = -1;
  cudaError_t err = cudaSuccess;
  explicit DeviceScope(int dev) {
    err = cudaGetDevice(&prev);
    if (err == cudaSuccess && prev != dev) err = cudaSetDevice(dev);
  }
  ~DeviceScope() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

// Records `msg` as the calling thread's tabby_last_error() and returns `status`.
int set_error(int status, const char *msg);

// Host float64 finalize with the device's arithmetic (sampler.ts:147-212).
int host_sample_from_topk(const int32_t *ids, const float *logits, int32_t n, float max_logit,
                          float sum_exp, double temperature, double top_p, double u,
                          tabby_sample_outcome *out);

}  // namespace tabby
