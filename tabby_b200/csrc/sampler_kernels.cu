// B200 (sm_100a) kernels of the token sampler.
//
// Replaces the reference's sampling dispatches (xOAviOx/tabby src/engine/forward.ts
// :520-601): a logits copy, reduce_max x2, reduce_sumexp x2 and k rounds of
// topk_partial + topk_select, i.e. k+4 passes over the row. Here each row is read from
// HBM once:
//
//   row_kernel   one thread-block cluster of C CTAs per row. CTA q stages columns
//                [q*slice, (q+1)*slice) in shared memory with 1-D TMA bulk copies
//                (cp.async.bulk, mbarrier completion) and, while the chunks land,
//                takes the max and an 11-bit digit histogram of order-preserving keys.
//                The cluster merges histograms in rank 0's shared memory over DSMEM
//                and picks the digit bucket that holds the k-th largest key (radix
//                select, digits 11/11/10 bits, at most three levels). Later passes run
//                over shared memory only: sum(exp(x - max)), the next digit histogram,
//                and finally the gather of the candidates into rank 0, which sorts
//                them by (value desc, index asc) and runs sampleFromTopK in float64.
//   merge_kernel the vocab-sharded finish: merges all-gathered per-shard blocks.
//
// Selection works on the raw logits; temperature only enters the float64 finalize,
// exactly as sampler.ts:144-146 and :170 do. Ties go to the lower index, as
// topk_partial.wgsl:40-42 and sampler.ts:28 order them.
#include <cooperative_groups.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "finalize.cuh"
#include "sampler_internal.h"

namespace cg = cooperative_groups;

namespace tabby {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kBins = 2048;      // widest radix digit: 11 bits
constexpr int kCandCap = 2048;   // candidates rank 0 can hold and sort
constexpr int kChunks = 4;       // bulk-copy chunks per CTA, one mbarrier each
constexpr int kMaxCluster = 16;
constexpr int kMergeThreads = 256;
constexpr float kNegSentinel = -3.0e38f;  // NEG_INF of reduce_max.wgsl:13

enum Decide : int32_t { kContinue = 0, kGather = 1, kExact = 2, kNone = 3 };
enum Flags : uint32_t { kFlagBadInput = 1u, kFlagTimeout = 2u, kFlagBadParams = 4u };

// Per-row cluster state. Every CTA has one; rank 0's copy collects the merges.
struct RowCtrl {
  uint32_t max_key;
  uint32_t flags;
  uint32_t cand_count;
  int32_t decision;
  uint32_t prefix;    // digits fixed before the current level
  int32_t remaining;  // keys still to take from inside the current prefix bucket
  uint32_t thresh;    // kGather: take key >= thresh; kExact: the tie key
  int32_t need;       // kExact: how many tie keys to take, lowest index first
  uint32_t bucket;    // digit chosen at the deciding level
  int32_t k_eff;
  float row_max;
  float sums[kMaxCluster];
};

// ------------------------------------------------------------------------------------
// Small device helpers
// ------------------------------------------------------------------------------------

// Order-preserving key: larger float -> larger key. -0 is folded onto +0 so equal values
// tie on the index, as the reference's `b.value - a.value || a.id - b.id` does.
__device__ __forceinline__ uint32_t key_of(float x) {
  uint32_t b = __float_as_uint(x);
  b = (b == 0x80000000u) ? 0u : b;
  const uint32_t mask = (uint32_t)((int32_t)b >> 31) | 0x80000000u;
  return b ^ mask;
}

__device__ __forceinline__ float float_of_key(uint32_t k) {
  const uint32_t mask = (k >> 31) ? 0x80000000u : 0xffffffffu;
  return __uint_as_float(k ^ mask);
}

__device__ __forceinline__ bool bad_logit(float x) {
  // NaN, +-inf and values at or below the reference's -3.0e38 sentinel
  // (topk_select.wgsl:65 masks with it) have no defined result in the reference.
  return !(x > kNegSentinel && x <= 3.40282347e38f);
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t cluster_nctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}

__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void cluster_sync_all() {
  cluster_arrive();
  cluster_wait();
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: gives up after ~2^22 polls (each poll may suspend briefly) and reports
// failure instead of spinning forever.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity) {
  for (uint32_t i = 0; i < (1u << 22); i++)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

// 1-D TMA bulk copy global -> this CTA's shared memory (no multicast).
__device__ __forceinline__ void bulk_copy_g2s(void *dst, const void *src, uint32_t bytes,
                                              uint64_t *bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint64_t evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Block-wide sum of one float per thread, fixed order (deterministic).
__device__ float block_sum_f32(float v, float *red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float total = 0.f;
  if (threadIdx.x == 0)
    for (int i = 0; i < kWarps; i++) total += red[i];
  return total;  // valid in thread 0 only
}

// Block-wide exclusive prefix sum of one int per thread in thread order.
__device__ int block_exclusive_scan(int v, int *red, int *total) {
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  int inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(0xffffffffu, inc, o);
    if (l >= o) inc += n;
  }
  __syncthreads();
  if (l == 31) red[w] = inc;
  __syncthreads();
  int before = 0, all = 0;
  for (int i = 0; i < kWarps; i++) {
    const int s = red[i];
    before += (i < w) ? s : 0;
    all += s;
  }
  *total = all;
  return before + inc - v;
}

// Bitonic sort of a[0, N) descending, N a power of two, in shared memory.
__device__ void block_sort_desc(uint64_t *a, int N) {
  for (int size = 2; size <= N; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < (N >> 1); i += blockDim.x) {
        const int lo = 2 * i - (i & (stride - 1));
        const int hi = lo + stride;
        const bool desc = (lo & size) == 0;
        const uint64_t x = a[lo], y = a[hi];
        if ((x < y) == desc) {
          a[lo] = y;
          a[hi] = x;
        }
      }
      __syncthreads();
    }
  }
}

__device__ __forceinline__ int next_pow2(int n) {
  int p = 2;
  while (p < n) p <<= 1;
  return p;
}

// Pool-size rule of the worker (inference.worker.ts:120-123).
__host__ __device__ __forceinline__ int32_t pool_rule(double temperature, int32_t top_k,
                                                      int32_t cap) {
  if (temperature <= 0) return 1;
  int32_t k = top_k != 0 ? top_k : cap;
  if (k < 1) k = 1;
  return k < cap ? k : cap;
}

// ------------------------------------------------------------------------------------
// Candidate push into rank 0's shared memory (warp-aggregated slot reservation).
// ------------------------------------------------------------------------------------
__device__ __forceinline__ void push_candidate(bool pred, uint32_t key, uint32_t idx,
                                               uint32_t *r0_count, uint64_t *r0_cand) {
  const uint32_t mask = __ballot_sync(0xffffffffu, pred);
  if (mask == 0) return;
  const int lane = threadIdx.x & 31;
  const int leader = __ffs(mask) - 1;
  uint32_t base = 0;
  if (lane == leader) base = atomicAdd(r0_count, (uint32_t)__popc(mask));
  base = __shfl_sync(0xffffffffu, base, leader);
  if (pred) {
    const uint32_t slot = base + __popc(mask & ((1u << lane) - 1u));
    if (slot < (uint32_t)kCandCap) r0_cand[slot] = ((uint64_t)key << 32) | (uint64_t)(~idx);
  }
}

// ------------------------------------------------------------------------------------
// Rank 0: pick the digit bucket that holds the k-th largest key.
// ------------------------------------------------------------------------------------
__device__ void decide_level(RowCtrl *ctrl, uint32_t *merged, int level, int *red) {
  const int width = level == 2 ? 10 : 11;
  const int shift = level == 0 ? 21 : (level == 1 ? 10 : 0);
  const int tid = threadIdx.x;
  // Inputs of this level, read before anyone can overwrite them.
  const uint32_t R = (uint32_t)ctrl->remaining;
  const uint32_t k_eff = (uint32_t)ctrl->k_eff;
  const uint32_t prefix = ctrl->prefix;
  // Thread t owns bins [4t, 4t+4); sum of everything above them (descending order).
  uint32_t h[4];
  uint32_t mine = 0;
#pragma unroll
  for (int j = 0; j < 4; j++) {
    h[j] = merged[4 * tid + j];
    mine += h[j];
  }
  // Suffix sum over threads > tid.
  const int lane = tid & 31, w = tid >> 5;
  uint32_t inc = mine;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t n = __shfl_down_sync(0xffffffffu, inc, o);
    if (lane + o < 32) inc += n;
  }
  __syncthreads();
  if (lane == 0) red[w] = (int)inc;
  // No crossing found (inconsistent counts) ends the selection instead of looping.
  if (tid == 0) ctrl->decision = kNone;
  __syncthreads();
  uint32_t above = inc - mine;
  for (int i = w + 1; i < kWarps; i++) above += (uint32_t)red[i];

  if (above < R && above + mine >= R) {
    // The crossing is in this thread's bins: scan them from the top.
    int b = 3;
    for (; b > 0; b--) {
      if (above + h[b] >= R) break;
      above += h[b];
    }
    const uint32_t bin = 4 * tid + b;
    const uint32_t inb = h[b];
    const uint32_t taken = k_eff - R;
    const uint32_t n_stop = taken + above + inb;
    const uint32_t stop_limit = min((uint32_t)kCandCap, max(2u * k_eff, 128u));
    const uint32_t full = (prefix << width) | bin;
    ctrl->bucket = bin;
    if (n_stop <= stop_limit) {
      ctrl->decision = kGather;
      ctrl->thresh = full << shift;
    } else if (level == 2) {
      ctrl->decision = kExact;
      ctrl->thresh = full;
      ctrl->need = (int32_t)(R - above);
    } else {
      ctrl->decision = kContinue;
      ctrl->prefix = full;
      ctrl->remaining = (int32_t)(R - above);
    }
  }
  __syncthreads();
  // Clear the merge area for the next level's histogram.
  if (ctrl->decision == kContinue)
    for (int i = tid; i < kBins; i += kThreads) merged[i] = 0;
}

// ------------------------------------------------------------------------------------
// The row kernel.
// ------------------------------------------------------------------------------------
struct RowArgs {
  const float *logits;
  int64_t row_stride;
  int32_t rows, vocab, slice, data_floats;
  int32_t mode, cap, fixed_k;
  int64_t index_offset;
  const tabby_sampling_params *params;
  const double *uniforms;
  tabby_sample_outcome *out;
  int32_t *topk_ids;
  float *topk_values;
  int32_t topk_ld;
  float *block;
  int32_t block_ld;
};

// One pass over the staged slice: optional sum(exp(x - M)), optional digit histogram of
// the keys inside `prefix`, optional gather of keys >= thresh into rank 0.
template <bool kSum, bool kHist, bool kGather>
__device__ float slice_pass(const float *data, int mis, int n, int lo, float row_max,
                            uint32_t *hist, int level, uint32_t prefix, uint32_t thresh,
                            uint32_t *r0_count, uint64_t *r0_cand) {
  const int width = level == 2 ? 10 : 11;
  const int shift = level == 0 ? 21 : (level == 1 ? 10 : 0);
  const uint32_t dmask = (1u << width) - 1u;
  const float4 *d4 = reinterpret_cast<const float4 *>(data);
  const int G = (mis + n + 3) >> 2;
  float s = 0.f;
  for (int base = 0; base < G; base += kThreads) {
    const int g = base + threadIdx.x;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (g < G) v = d4[g];
    const float xs[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int e = 0; e < 4; e++) {
      const int idx = 4 * g + e;
      const bool valid = g < G && idx >= mis && idx < mis + n;
      const float x = xs[e];
      const uint32_t key = key_of(x);
      if (kSum) {
        if (valid) s += __expf(x - row_max);
      }
      if (kHist) {
        if (valid && (key >> (shift + width)) == prefix)
          atomicAdd(&hist[(key >> shift) & dmask], 1u);
      }
      if (kGather) {
        push_candidate(valid && key >= thresh, key, (uint32_t)(lo + idx - mis), r0_count,
                       r0_cand);
      }
    }
  }
  return s;
}

__global__ void __launch_bounds__(kThreads, 2) row_kernel(RowArgs a) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  float *data = reinterpret_cast<float *>(smem_raw);
  uint32_t *hist = reinterpret_cast<uint32_t *>(smem_raw + (size_t)a.data_floats * 4);
  uint64_t *cand = reinterpret_cast<uint64_t *>(hist + kBins);  // also the merged histogram
  uint32_t *merged = reinterpret_cast<uint32_t *>(cand);
  uint64_t *bars = cand + kCandCap;
  RowCtrl *ctrl = reinterpret_cast<RowCtrl *>(bars + kChunks);
  int *red = reinterpret_cast<int *>(ctrl + 1);

  cg::cluster_group cluster = cg::this_cluster();
  const uint32_t rank = cluster_ctarank();
  const uint32_t csize = cluster_nctarank();
  const int row = (int)cluster_id_x();
  const int tid = threadIdx.x;

  RowCtrl *r0 = cluster.map_shared_rank(ctrl, 0);
  uint32_t *r0_merged = cluster.map_shared_rank(merged, 0);
  uint64_t *r0_cand = cluster.map_shared_rank(cand, 0);

  const float *rowp = a.logits + (int64_t)row * a.row_stride;
  const int lo = (int)rank * a.slice;
  const int hi = min(lo + a.slice, a.vocab);
  const int n = max(hi - lo, 0);
  const int mis = n > 0 ? (int)((reinterpret_cast<uintptr_t>(rowp + lo) >> 2) & 3) : 0;
  int a0 = lo + ((4 - mis) & 3);
  if (a0 > hi) a0 = hi;
  const int a1 = a0 + ((hi - a0) & ~3);
  const int ng = (a1 - a0) >> 2;  // 16-byte groups moved by TMA
  const int gb0 = (a0 - lo + mis) >> 2;

  // ---- set-up: local state, mbarriers, then start the bulk copies at once ----
  for (int i = tid; i < kBins; i += kThreads) hist[i] = 0;
  if (rank == 0)
    for (int i = tid; i < kBins; i += kThreads) merged[i] = 0;
  if (tid == 0) {
    RowCtrl c = {};
    c.max_key = 0;
    c.decision = kContinue;
    *ctrl = c;
    for (int c2 = 0; c2 < kChunks; c2++) mbar_init(&bars[c2], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (tid == 0 && ng > 0) {
    const uint64_t policy = evict_first_policy();
    for (int c2 = 0; c2 < kChunks; c2++) {
      const int g0 = (ng * c2) / kChunks, g1 = (ng * (c2 + 1)) / kChunks;
      const uint32_t bytes = (uint32_t)(g1 - g0) * 16u;
      mbar_expect_tx(&bars[c2], bytes);
      if (bytes) bulk_copy_g2s(data + 4 * (gb0 + g0), rowp + a0 + 4 * g0, bytes, &bars[c2], policy);
    }
  }
  // Every CTA of the cluster must be running before any DSMEM access: arrive now, wait
  // just before the first remote operation.
  cluster_arrive();

  // ---- pass A: max, bad-input check and level-0 histogram as chunks arrive ----
  uint32_t kmax = 0;
  bool bad = false;
  // Ragged head/tail elements (fewer than 4 at each end) come in through plain loads.
  if (tid < 8) {
    const int e = tid < 4 ? lo + tid : a1 + (tid - 4);
    const bool in = tid < 4 ? (e < a0) : (e < hi);
    if (in) {
      const float x = __ldg(rowp + e);
      data[e - lo + mis] = x;
      const uint32_t key = key_of(x);
      kmax = max(kmax, key);
      bad |= bad_logit(x);
      atomicAdd(&hist[key >> 21], 1u);
    }
  }
  bool timed_out = false;
  const float4 *d4 = reinterpret_cast<const float4 *>(data);
  for (int c2 = 0; c2 < kChunks && ng > 0; c2++) {
    if (!mbar_wait_bounded(&bars[c2], 0)) timed_out = true;
    const int g0 = gb0 + (ng * c2) / kChunks, g1 = gb0 + (ng * (c2 + 1)) / kChunks;
    for (int g = g0 + tid; g < g1; g += kThreads) {
      const float4 v = d4[g];
      const float xs[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const uint32_t key = key_of(xs[e]);
        kmax = max(kmax, key);
        bad |= bad_logit(xs[e]);
        atomicAdd(&hist[key >> 21], 1u);
      }
    }
  }
  kmax = __reduce_max_sync(0xffffffffu, kmax);
  const int any_bad = __syncthreads_or(bad ? 1 : 0);
  const int any_timeout = __syncthreads_or(timed_out ? 1 : 0);

  cluster_wait();  // peers are alive; rank 0's merge area is cleared

  // ---- level loop: merge histograms in rank 0, decide, maybe refine ----
  int level = 0;
  float row_max = 0.f;
  bool sum_done = false;
  float my_sum = 0.f;
  RowCtrl c;
  for (;;) {
    for (int i = tid; i < kBins; i += kThreads) {
      const uint32_t v = hist[i];
      if (v) atomicAdd(&r0_merged[i], v);
    }
    if (level == 0) {
      if ((tid & 31) == 0) atomicMax(&r0->max_key, kmax);
      if (tid == 0 && (any_bad || any_timeout))
        atomicOr(&r0->flags, (any_bad ? kFlagBadInput : 0u) | (any_timeout ? kFlagTimeout : 0u));
    }
    cluster_sync_all();
    if (rank == 0) {
      if (level == 0) {
        if (tid == 0) {
          int32_t k;
          if (a.mode == kModeSample) {
            const tabby_sampling_params p = a.params[row];
            k = pool_rule(p.temperature, p.top_k, a.cap);
            if (isnan(p.temperature) || isnan(p.top_p)) ctrl->flags |= kFlagBadParams;
          } else {
            k = a.fixed_k;
          }
          k = min(k, a.vocab);
          ctrl->k_eff = k;
          ctrl->remaining = k;
          ctrl->prefix = 0;
          ctrl->row_max = float_of_key(ctrl->max_key);
          if (k <= 0) ctrl->decision = kNone;
        }
        __syncthreads();
      }
      if (ctrl->decision != kNone) decide_level(ctrl, merged, level, red);
      __syncthreads();
    }
    cluster_sync_all();
    // Decision of this level; rank 0 writes no decision field again before the next
    // cluster barrier. One thread fetches it over DSMEM for the whole CTA.
    if (rank != 0 && tid == 0) *ctrl = *r0;
    __syncthreads();
    c = *ctrl;
    if (level == 0) row_max = c.row_max;
    if (c.decision != kContinue) break;
    level++;
    for (int i = tid; i < kBins; i += kThreads) hist[i] = 0;
    __syncthreads();
    if (!sum_done) {
      my_sum = slice_pass<true, true, false>(data, mis, n, lo, row_max, hist, level, c.prefix, 0,
                                             nullptr, nullptr);
      sum_done = true;
    } else {
      slice_pass<false, true, false>(data, mis, n, lo, row_max, hist, level, c.prefix, 0, nullptr,
                                     nullptr);
    }
    __syncthreads();
  }

  // ---- final pass: gather candidates into rank 0 ----
  uint32_t *r0_count = &r0->cand_count;
  if (c.decision == kGather) {
    if (!sum_done) {
      my_sum = slice_pass<true, false, true>(data, mis, n, lo, row_max, hist, 0, 0, c.thresh,
                                             r0_count, r0_cand);
      sum_done = true;
    } else {
      slice_pass<false, false, true>(data, mis, n, lo, row_max, hist, 0, 0, c.thresh, r0_count,
                                     r0_cand);
    }
  } else {
    if (!sum_done) {
      my_sum = slice_pass<true, false, false>(data, mis, n, lo, row_max, hist, 0, 0, 0, nullptr,
                                              nullptr);
      sum_done = true;
    }
    if (c.decision == kExact) {
      // Keys above the tie key all go; of the keys equal to it, the `need` lowest
      // indices go. CTAs cover ascending column ranges, so this CTA's first tie has rank
      // (ties held by lower ranks).
      int offset = 0;
      for (uint32_t p = 0; p < rank; p++) offset += (int)*cluster.map_shared_rank(&hist[c.bucket], p);
      const int G = (mis + n + 3) >> 2;
      int running = 0;
      for (int base = 0; base < G; base += kThreads) {
        const int g = base + tid;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (g < G) v = d4[g];
        const float xs[4] = {v.x, v.y, v.z, v.w};
        int ties = 0;
        bool is_tie[4], is_above[4];
#pragma unroll
        for (int e = 0; e < 4; e++) {
          const int idx = 4 * g + e;
          const bool valid = g < G && idx >= mis && idx < mis + n;
          const uint32_t key = key_of(xs[e]);
          is_tie[e] = valid && key == c.thresh;
          is_above[e] = valid && key > c.thresh;
          ties += is_tie[e] ? 1 : 0;
        }
        int tile_total;
        const int before = block_exclusive_scan(ties, red, &tile_total);
        int r = offset + running + before;
#pragma unroll
        for (int e = 0; e < 4; e++) {
          const uint32_t idx = (uint32_t)(lo + 4 * g + e - mis);
          const bool take_tie = is_tie[e] && r < c.need;
          r += is_tie[e] ? 1 : 0;
          push_candidate(is_above[e] || take_tie, key_of(xs[e]), idx, r0_count, r0_cand);
        }
        running += tile_total;
      }
    }
  }
  {
    const float total = block_sum_f32(my_sum, reinterpret_cast<float *>(red));
    if (tid == 0) r0->sums[rank] = total;
  }
  cluster_sync_all();  // every candidate and partial sum is in rank 0
  if (rank != 0) return;

  // ---- rank 0: sort the candidates, then the epilogue of the mode ----
  const RowCtrl fin = *ctrl;
  const int k = fin.k_eff;
  int nc = (int)min(fin.cand_count, (uint32_t)kCandCap);
  if (fin.decision == kNone) nc = 0;
  double sum_d = 0.0;
  for (uint32_t q = 0; q < csize; q++) sum_d += (double)fin.sums[q];
  const float sum_exp = (float)sum_d;
  const uint32_t status = (fin.flags & kFlagBadInput)    ? (uint32_t)TABBY_EINPUT
                          : (fin.flags & kFlagBadParams) ? (uint32_t)TABBY_EINVAL
                          : (fin.flags & kFlagTimeout)   ? (uint32_t)TABBY_ETIMEOUT
                                                         : (uint32_t)TABBY_OK;
  if (nc > 0) {
    const int N = next_pow2(nc);
    for (int i = nc + tid; i < N; i += kThreads) cand[i] = 0ull;
    __syncthreads();
    block_sort_desc(cand, N);
  }
  const int kk = min(k, nc);
  // Unpack the first kk candidates into (id, value); the finalize arrays reuse the
  // (no longer needed) data region.
  double *exact = reinterpret_cast<double *>(data);
  double *scaled = exact + kk;
  int32_t *ids = reinterpret_cast<int32_t *>(scaled + kk);
  float *vals = reinterpret_cast<float *>(ids + kk);
  for (int i = tid; i < kk; i += kThreads) {
    const uint64_t e = cand[i];
    const uint32_t key = (uint32_t)(e >> 32);
    const uint32_t idx = ~(uint32_t)e;
    float v = float_of_key(key);
    if (key == 0x80000000u) v = rowp[idx];  // keep the sign of a zero logit
    ids[i] = (int32_t)idx;
    vals[i] = v;
  }
  __syncthreads();
  const float max_logit = kk > 0 ? vals[0] : fin.row_max;

  if (a.mode == kModeTopK || a.mode == kModeShard) {
    float *blk = a.block + (int64_t)row * a.block_ld;
    const int slots = a.mode == kModeShard ? TABBY_SHARD_TOP_K : k;
    if (tid == 0) {
      blk[0] = status == TABBY_OK ? max_logit : __int_as_float(0x7fc00000);
      blk[1] = sum_exp;
    }
    for (int i = tid; i < slots; i += kThreads) {
      float v = __int_as_float(0xff800000);  // -inf pad
      uint32_t gi = 0xffffffffu;
      if (i < kk) {
        v = vals[i];
        gi = (uint32_t)((int64_t)ids[i] + a.index_offset);
      }
      blk[2 + 2 * i] = v;
      blk[3 + 2 * i] = __uint_as_float(gi);
    }
    return;
  }

  // kModeSample
  if (a.topk_ids)
    for (int i = tid; i < kk; i += kThreads) a.topk_ids[(int64_t)row * a.topk_ld + i] = ids[i];
  if (a.topk_values)
    for (int i = tid; i < kk; i += kThreads) a.topk_values[(int64_t)row * a.topk_ld + i] = vals[i];
  const tabby_sampling_params p = a.params[row];
  const double u = a.uniforms[row];
  for (int i = tid; i < kk; i += kThreads) {
    exact[i] = exact_prob(vals[i], max_logit, sum_exp);
    scaled[i] = p.temperature > 0 ? scaled_weight(vals[i], max_logit, p.temperature) : 0.0;
  }
  __syncthreads();
  if (tid == 0) {
    tabby_sample_outcome o;
    o.pool_size = kk;
    o.max_logit = max_logit;
    o.sum_exp = sum_exp;
    o.reserved = 0;
    if (status != TABBY_OK || kk == 0) {
      o.id = -1;
      o.considered_count = 0;
      o.probability = 0.0;
      o.pool_mass = 0.0;
      o.pool_exhausted = 0;
      o.status = status != TABBY_OK ? (int32_t)status : (int32_t)TABBY_EEMPTY;
    } else {
      const Decision d = decide_sequential(exact, scaled, scaled, kk, p.temperature, p.top_p, u);
      o.id = ids[d.chosen];
      o.considered_count = d.cut;
      o.probability = exact[d.chosen];
      o.pool_mass = d.pool_mass;
      o.pool_exhausted = d.pool_exhausted;
      o.status = TABBY_OK;
    }
    a.out[row] = o;
  }
}

// ------------------------------------------------------------------------------------
// Vocab-sharded finish: one CTA per row over the all-gathered shard blocks.
// ------------------------------------------------------------------------------------
__global__ void __launch_bounds__(kMergeThreads) merge_kernel(MergeLaunch a) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  const int row = blockIdx.x;
  const int tid = threadIdx.x;
  const int total = a.shards * TABBY_SHARD_TOP_K;
  const int N = next_pow2(total);
  uint64_t *cand = reinterpret_cast<uint64_t *>(smem_raw);
  double *exact = reinterpret_cast<double *>(cand + N);
  double *scaled = exact + TABBY_SHARD_TOP_K;
  int32_t *ids = reinterpret_cast<int32_t *>(scaled + TABBY_SHARD_TOP_K);
  float *vals = reinterpret_cast<float *>(ids + TABBY_SHARD_TOP_K);
  __shared__ float s_max;
  __shared__ float s_sum;
  __shared__ int s_bad;
  __shared__ int s_count;

  if (tid == 0) {
    // M = max m_s; S = sum s_s * exp(m_s - M), shards in rank order.
    float m = -3.40282347e38f;
    int bad = 0;
    for (int s = 0; s < a.shards; s++) {
      const float ms = a.gathered[((int64_t)s * a.rows + row) * a.block_ld];
      if (ms != ms) bad = 1;
      m = fmaxf(m, ms);
    }
    double S = 0.0;
    for (int s = 0; s < a.shards; s++) {
      const float *b = a.gathered + ((int64_t)s * a.rows + row) * a.block_ld;
      S = JS_ADD(S, JS_MUL((double)b[1], js_exp(JS_SUB((double)b[0], (double)m))));
    }
    s_max = m;
    s_sum = (float)S;
    const tabby_sampling_params p0 = a.params[row];
    if (isnan(p0.temperature) || isnan(p0.top_p)) bad = 2;
    s_bad = bad;
    s_count = 0;
  }
  __syncthreads();
  for (int i = tid; i < N; i += kMergeThreads) {
    uint64_t e = 0;
    if (i < total) {
      const int s = i / TABBY_SHARD_TOP_K, j = i % TABBY_SHARD_TOP_K;
      const float *b = a.gathered + ((int64_t)s * a.rows + row) * a.block_ld;
      const uint32_t gi = __float_as_uint(b[3 + 2 * j]);
      if (gi != 0xffffffffu) e = ((uint64_t)key_of(b[2 + 2 * j]) << 32) | (uint64_t)(~gi);
      if (gi != 0xffffffffu) atomicAdd(&s_count, 1);
    }
    cand[i] = e;
  }
  __syncthreads();
  block_sort_desc(cand, N);
  const tabby_sampling_params p = a.params[row];
  int k = pool_rule(p.temperature, p.top_k, TABBY_SHARD_TOP_K);
  const int kk = min(k, s_count);
  for (int i = tid; i < kk; i += kMergeThreads) {
    const uint64_t e = cand[i];
    const uint32_t key = (uint32_t)(e >> 32);
    const uint32_t gi = ~(uint32_t)e;
    float v = float_of_key(key);
    if (key == 0x80000000u) {
      // Recover the sign of a zero from the shard block that holds it.
      for (int s = 0; s < a.shards; s++) {
        const float *b = a.gathered + ((int64_t)s * a.rows + row) * a.block_ld;
        for (int j = 0; j < TABBY_SHARD_TOP_K; j++)
          if (__float_as_uint(b[3 + 2 * j]) == gi) v = b[2 + 2 * j];
      }
    }
    ids[i] = (int32_t)gi;
    vals[i] = v;
  }
  __syncthreads();
  const float max_logit = kk > 0 ? vals[0] : s_max;
  const float sum_exp = s_sum;
  if (a.topk_ids)
    for (int i = tid; i < kk; i += kMergeThreads) a.topk_ids[(int64_t)row * a.topk_ld + i] = ids[i];
  if (a.topk_values)
    for (int i = tid; i < kk; i += kMergeThreads)
      a.topk_values[(int64_t)row * a.topk_ld + i] = vals[i];
  const double u = a.uniforms[row];
  for (int i = tid; i < kk; i += kMergeThreads) {
    exact[i] = exact_prob(vals[i], max_logit, sum_exp);
    scaled[i] = p.temperature > 0 ? scaled_weight(vals[i], max_logit, p.temperature) : 0.0;
  }
  __syncthreads();
  if (tid == 0) {
    tabby_sample_outcome o;
    o.pool_size = kk;
    o.max_logit = max_logit;
    o.sum_exp = sum_exp;
    o.reserved = 0;
    if (s_bad || kk == 0) {
      o.id = -1;
      o.considered_count = 0;
      o.probability = 0.0;
      o.pool_mass = 0.0;
      o.pool_exhausted = 0;
      o.status = s_bad == 1 ? TABBY_EINPUT : s_bad == 2 ? TABBY_EINVAL : TABBY_EEMPTY;
    } else {
      const Decision d = decide_sequential(exact, scaled, scaled, kk, p.temperature, p.top_p, u);
      o.id = ids[d.chosen];
      o.considered_count = d.cut;
      o.probability = exact[d.chosen];
      o.pool_mass = d.pool_mass;
      o.pool_exhausted = d.pool_exhausted;
      o.status = TABBY_OK;
    }
    a.out[row] = o;
  }
}

// ------------------------------------------------------------------------------------
// Host side: geometry and launches.
// ------------------------------------------------------------------------------------
static size_t row_smem_bytes(int data_floats) {
  return (size_t)data_floats * 4 + (size_t)kBins * 4 + (size_t)kCandCap * 8 +
         (size_t)kChunks * 8 + sizeof(RowCtrl) + (size_t)kWarps * 4 + 64;
}

static int round_up(int x, int m) { return (x + m - 1) / m * m; }

cudaError_t plan_rows(int32_t sms, int32_t max_smem_optin, int32_t rows, int32_t vocab,
                      int32_t cap, int32_t max_cluster, RowGeometry *geo) {
  // Shared memory per CTA that still lets two CTAs share an SM (one streams its slice in
  // while the other works on shared memory), and the hard per-CTA limit beyond that.
  const size_t two_per_sm = 112 * 1024;
  const size_t one_per_sm = (size_t)max_smem_optin;
  const int finalize_floats = 6 * min(max(cap, (int32_t)TABBY_SHARD_TOP_K), vocab) + 16;
  auto geometry = [&](int C) {
    RowGeometry g;
    g.cluster = C;
    g.slice = round_up((vocab + C - 1) / C, 4);
    g.data_floats = round_up(max(g.slice + 8, finalize_floats), 32);
    g.smem_bytes = row_smem_bytes(g.data_floats);
    return g;
  };
  if (max_cluster > kMaxCluster) max_cluster = kMaxCluster;
  int C = 1;
  while (C < max_cluster && geometry(C).smem_bytes > two_per_sm) C <<= 1;
  if (geometry(C).smem_bytes > one_per_sm) return cudaErrorInvalidValue;
  // Spread small batches over more SMs: aim for >= 2 CTAs per SM in flight, but keep
  // at least ~4K logits per CTA.
  while (C < max_cluster && (int64_t)rows * C < 2 * (int64_t)sms &&
         geometry(2 * C).slice >= 4096)
    C <<= 1;
  *geo = geometry(C);
  return cudaSuccess;
}

// Raises the kernel's dynamic shared-memory limit once per process to the largest size
// ever asked for, and allows clusters of 16 CTAs.
static cudaError_t prepare_row_kernel(size_t smem_bytes) {
  static size_t configured = 0;
  static bool nonportable = false;
  if (!nonportable) {
    cudaError_t err =
        cudaFuncSetAttribute(row_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (err != cudaSuccess) return err;
    nonportable = true;
  }
  if (smem_bytes > configured) {
    cudaError_t err = cudaFuncSetAttribute(
        row_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_bytes);
    if (err != cudaSuccess) return err;
    configured = smem_bytes;
  }
  return cudaSuccess;
}

cudaError_t max_active_clusters(const RowGeometry &geo, int *count) {
  cudaError_t err = prepare_row_kernel(geo.smem_bytes);
  if (err != cudaSuccess) return err;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)geo.cluster, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = geo.smem_bytes;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)geo.cluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaOccupancyMaxActiveClusters(count, row_kernel, &cfg);
}

cudaError_t launch_rows(const RowLaunch &l, const RowGeometry &geo, cudaStream_t stream) {
  if (l.rows == 0) return cudaSuccess;
  RowArgs a;
  a.logits = l.logits;
  a.row_stride = l.row_stride;
  a.rows = l.rows;
  a.vocab = l.vocab;
  a.slice = geo.slice;
  a.data_floats = geo.data_floats;
  a.mode = l.mode;
  a.cap = l.cap;
  a.fixed_k = l.fixed_k;
  a.index_offset = l.index_offset;
  a.params = l.params;
  a.uniforms = l.uniforms;
  a.out = l.out;
  a.topk_ids = l.topk_ids;
  a.topk_values = l.topk_values;
  a.topk_ld = l.topk_ld;
  a.block = l.block;
  a.block_ld = l.block_ld;

  cudaError_t err = prepare_row_kernel(geo.smem_bytes);
  if (err != cudaSuccess) return err;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(l.rows * geo.cluster), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = geo.smem_bytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)geo.cluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, row_kernel, a);
}

cudaError_t launch_merge(const MergeLaunch &l, cudaStream_t stream) {
  if (l.rows == 0) return cudaSuccess;
  const int total = l.shards * TABBY_SHARD_TOP_K;
  int N = 2;
  while (N < total) N <<= 1;
  const size_t smem = (size_t)N * 8 + (size_t)TABBY_SHARD_TOP_K * (8 + 8 + 4 + 4);
  cudaError_t err =
      cudaFuncSetAttribute(merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (err != cudaSuccess) return err;
  merge_kernel<<<l.rows, kMergeThreads, smem, stream>>>(l);
  return cudaGetLastError();
}

int host_sample_from_topk(const int32_t *ids, const float *logits, int32_t n, float max_logit,
                          float sum_exp, double temperature, double top_p, double u,
                          tabby_sample_outcome *out) {
  if (n <= 0) return TABBY_EEMPTY;
  double *exact = new double[n];
  double *scaled = new double[n];
  for (int32_t i = 0; i < n; i++) {
    exact[i] = exact_prob(logits[i], max_logit, sum_exp);
    scaled[i] = temperature > 0 ? scaled_weight(logits[i], max_logit, temperature) : 0.0;
  }
  const Decision d = decide_sequential(exact, scaled, scaled, n, temperature, top_p, u);
  out->id = ids[d.chosen];
  out->considered_count = d.cut;
  out->probability = exact[d.chosen];
  out->pool_mass = d.pool_mass;
  out->pool_exhausted = d.pool_exhausted;
  out->pool_size = n;
  out->max_logit = max_logit;
  out->sum_exp = sum_exp;
  out->status = TABBY_OK;
  out->reserved = 0;
  delete[] exact;
  delete[] scaled;
  return TABBY_OK;
}

}  // namespace tabby
