// B200 (sm_100a) kernels of the token sampler.
//
// Replaces the reference's sampling dispatches (xOAviOx/tabby src/engine/forward.ts
// :520-601): a logits copy, reduce_max x2, reduce_sumexp x2 and k rounds of
// topk_partial + topk_select, i.e. k+4 passes over the row. Here every logit is read
// from HBM once, in one streaming pass:
//
//   row_kernel     one launch, at most two 512-thread CTAs per SM. Rows are cut into
//                  chunks only until the units cover ~0.8 of the resident CTAs.
//     whole rows   (large batches) CTAs take rows from a counter; each warp streams its
//                  16th of the row; the threshold comes from every warp's first
//                  iteration (8192 logits spread over the row) while the second is in
//                  flight; the CTA finishes its own row. No inter-CTA waits.
//     chunked      (small batches) a plan phase (CTA c plans rows c, c + grid, ...:
//                  resets the row's counters, fixes its pool size and its place in the
//                  processing order, estimates the threshold from 2048 logits sampled
//                  in 32 runs, publishes epoch-tagged entries), then CTAs take (row,
//                  chunk) units, waiting only for their own row's entry (cooperative
//                  launch: all CTAs resident); the unit that completes a row finishes it.
//     streaming    each warp streams through a 3-stage cp.async ring in shared memory,
//                  keeps online max and sum(exp(x - max)) per thread (packed f32x2
//                  arithmetic) and appends every float4 group holding a logit at or
//                  above the threshold to its own region of the row's candidate list;
//                  no block barrier until the segment ends.
//     finish       merges the per-warp statistics, expands the groups into 64-bit
//                  composites (order-preserving key, inverted index), checks the
//                  estimate (falling back to an exact re-filter), keeps and sorts the k
//                  best (binned ranking) and runs sampleFromTopK in float64
//                  (finalize.cuh); with a device RNG state the draw is made here.
//   merge_kernel   the vocab-sharded finish: one warp a row merges the all-gathered
//                  per-shard blocks (register bitonic merges) and runs finalize_warp.
//   xmerge_kernel  the same merge with the exchange inside: the peers' blocks read over
//                  NVLink after one release/acquire handshake (exchange.cu).
//
// Selection works on the raw logits; temperature only enters the float64 finalize,
// exactly as sampler.ts:144-146 and :170 do. Ties go to the lower index, as
// topk_partial.wgsl:40-42 and sampler.ts:28 order them: the composite
// (key << 32 | ~index) is unique per logit and orders exactly like that.
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <mutex>
#include <type_traits>

#include "finalize.cuh"
#include "warp_sort.cuh"
#include "sampler_internal.h"

namespace tabby {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kVec = 4;                   // float4 loads in flight per thread per iteration
constexpr int kWarpIter = 32 * kVec;      // float4 groups a warp reads per iteration (2 KB)
constexpr int kRowGroups = 8192;   // candidate groups (float4 + index) a row's global list holds
constexpr int kStages = 3;         // cp.async stages of the streaming loop
constexpr int kStageBytes = kStages * 4 * 512 * 16;  // the stages (kStages x kVec x kThreads)
// The finish reuses the stage region: composites first, the histogram at its end.
constexpr int kFinishCap = (kStageBytes - 2048 * 4) / 8;
constexpr int kBins = 2048;               // radix digit: 11 bits
constexpr int kMaxChunks = 32;            // chunks of one row (warp stats: chunks x 16 <= 512)
constexpr int kMinChunk = 8192;           // logits: below this a row is not split further
constexpr int kMaxShards = 16;           // shards the merge takes (tabby_shard_merge_async's limit)
static_assert(kRowGroups == kScratchGroups && kFinishCap >= 8192 &&
                  kRowGroups / (kMaxChunks * kWarps) >= 16 && kMaxChunks == kScratchChunks &&
                  kWarps == kScratchWarps && kMaxChunks * kWarps <= kThreads,
              "scratch layout and kernel constants disagree");
constexpr float kNegSentinel = -3.0e38f;  // NEG_INF of reduce_max.wgsl:13

enum Flags : uint32_t { kFlagBadInput = 1u, kFlagTimeout = 2u, kFlagBadParams = 4u };


// Opt-in self-checks for debugging builds (-DTABBY_CHECKS=1): shared-memory candidate
// writes of the selection are validated first; a violation is recorded (first one wins)
// and the access is skipped instead of faulting.
#ifdef TABBY_CHECKS
__device__ unsigned long long g_check[4];  // code, blockIdx, a, b
__device__ __forceinline__ bool check_ok(bool ok, unsigned code, unsigned long long x,
                                         unsigned long long y) {
  if (!ok && atomicCAS(&g_check[0], 0ull, (unsigned long long)code) == 0ull) {
    g_check[1] = blockIdx.x;
    g_check[2] = x;
    g_check[3] = y;
  }
  return ok;
}
#define CHECK(ok, code, x, y) check_ok((ok), (code), (unsigned long long)(x), (unsigned long long)(y))
#else
#define CHECK(ok, code, x, y) ((void)0, true)
#endif

// ------------------------------------------------------------------------------------
// Keys and small device helpers
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

// Unique, totally ordered candidate: value first, then the lower index.
__device__ __forceinline__ uint64_t composite(uint32_t key, uint32_t idx) {
  return ((uint64_t)key << 32) | (uint64_t)(~idx);
}

__device__ __forceinline__ bool bad_logit(float x) {
  // NaN, +-inf and values at or below the reference's -3.0e38 sentinel
  // (topk_select.wgsl:65 masks with it) have no defined result in the reference.
  return !(x > kNegSentinel && x <= 3.40282347e38f);
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

// 16-byte asynchronous global -> shared copy (cp.async, L2 only), tracked per thread by
// commit groups.
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_group 0;" ::: "memory");
}
// An L2 policy for data read once: its lines go first when L2 needs room, so the code and
// the small buffers the finish uses stay in L2.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ void cp_async16_u32(uint32_t dst, const void *src, uint64_t pol) {
  asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;" ::"r"(dst),
               "l"(src), "l"(pol)
               : "memory");
}
__device__ __forceinline__ void st_shared_f4(uint32_t dst, float4 v) {
  asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(dst), "f"(v.x), "f"(v.y),
               "f"(v.z), "f"(v.w)
               : "memory");
}
__device__ __forceinline__ float4 ld_shared_f4(uint32_t src) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(src)
               : "memory");
  return v;
}
__device__ __forceinline__ void st_release_u64(unsigned long long *p, unsigned long long v) {
  asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
template <int N>
__device__ __forceinline__ void cp_async_wait_group() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Three-input float max / min (sm_100 max.f32 / min.f32 with three sources).
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
__device__ __forceinline__ float min3f(float a, float b, float c) {
  float d;
  asm("min.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// 2^x by the MUFU.EX2 approximation (flush-to-zero).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint64_t ld_cg_u64(const unsigned long long *p) {
  return (uint64_t)__ldcg(p);
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

// Shared scalars of a CTA (block-uniform values and reduction scratch).
struct Shared {
  uint32_t count;   // candidates in the buffer
  uint32_t count2;  // compaction write cursor
  uint32_t bucket;
  uint32_t above;
  uint32_t inb;
  uint32_t last;  // this CTA finishes the row
  float2 wst[kWarps];        // whole rows: each warp's (max, sum-exp)
  uint32_t wgroups[kWarps];  // whole rows: candidate groups in each warp's region
  uint32_t unit;  // the unit this CTA works on
  int32_t urow, uk;  // its row and pool size
  int32_t plan_red[3][kWarps];  // plan: per-warp counts for the row order
  float utf;         // its threshold
  uint32_t base;  // where the unit's candidates go in the row's list
  int32_t cut_claim;
  int32_t chosen_claim;
  int32_t fallback;
  uint32_t flags;
  uint32_t overflow;  // an insert found the candidate buffer full
  uint64_t tau;  // accept composites >= tau
  float red_f[kWarps];
  float red_f2[kWarps];
  uint32_t red_u[kWarps];
  uint32_t red_u2[kWarps];
  double red_d[kWarps];
  float merge_max;
  float merge_sum;
  uint64_t samp[64];  // sorted sample of the candidate buffer
  int32_t off[32];  // merge: first candidate of each slice
  int32_t cnt[32];  // merge: candidates of each slice
  double rng_u;     // the row's draw in device-RNG mode
  uint32_t epoch;   // this launch's number (thread 0's copy for the plan)
};

// ------------------------------------------------------------------------------------
// Block primitives (blockDim.x == 512)
// ------------------------------------------------------------------------------------

// Warp-wide reductions of the 16 per-warp partials a block left in shared memory:
// every lane reads one partial, so the result costs one load and one reduction
// instead of a loop over the warps. Same value in every thread.
__device__ __forceinline__ uint32_t partials_min_u32(const uint32_t *p) {
  const int lane = threadIdx.x & 31;
  return __reduce_min_sync(0xffffffffu, lane < kWarps ? p[lane] : 0xffffffffu);
}
__device__ __forceinline__ uint32_t partials_max_u32(const uint32_t *p) {
  const int lane = threadIdx.x & 31;
  return __reduce_max_sync(0xffffffffu, lane < kWarps ? p[lane] : 0u);
}
// Sum of the partials of warps above w (w = this thread's warp).
__device__ __forceinline__ uint32_t partials_sum_above_u32(const uint32_t *p, int w) {
  const int lane = threadIdx.x & 31;
  return __reduce_add_sync(0xffffffffu, (lane > w && lane < kWarps) ? p[lane] : 0u);
}


// Deterministic block sum of one double per thread: a fixed shuffle tree in each warp,
// then the same tree over the 16 warp sums (one per lane). Same value in every thread.
__device__ double block_sum_f64(double v, Shared *sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = JS_ADD(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) sh->red_d[w] = v;
  __syncthreads();
  double total = l < kWarps ? sh->red_d[l] : 0.0;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) total = JS_ADD(total, __shfl_xor_sync(0xffffffffu, total, o));
  return total;
}

// Exclusive block scan of one double per thread in thread order.
__device__ double block_exclusive_scan_f64(double v, Shared *sh) {
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  double inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double n = __shfl_up_sync(0xffffffffu, inc, o);
    if (l >= o) inc = JS_ADD(inc, n);
  }
  __syncthreads();
  if (l == 31) sh->red_d[w] = inc;
  __syncthreads();
  // Sum of the warps before this one, one warp total a lane.
  double before = l < w ? sh->red_d[l] : 0.0;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) before = JS_ADD(before, __shfl_xor_sync(0xffffffffu, before, o));
  return JS_ADD(before, JS_SUB(inc, v));
}

// Finds the digit bucket b holding the R-th largest element of hist (scanning from the
// top): above = elements in buckets > b, inb = hist[b]. Results land in sh.
__device__ void find_bucket(const uint32_t *hist, uint32_t R, Shared *sh) {
  const int tid = threadIdx.x;
  const int lane = tid & 31, w = tid >> 5;
  uint32_t h[4];
  uint32_t mine = 0;
#pragma unroll
  for (int j = 0; j < 4; j++) {
    h[j] = hist[4 * tid + j];
    mine += h[j];
  }
  uint32_t inc = mine;  // suffix sum over this lane and the lanes above it
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t n = __shfl_down_sync(0xffffffffu, inc, o);
    if (lane + o < 32) inc += n;
  }
  __syncthreads();
  if (lane == 0) sh->red_u[w] = inc;
  __syncthreads();
  uint32_t above = inc - mine + partials_sum_above_u32(sh->red_u, w);
  if (above < R && above + mine >= R) {
    int b = 3;
    for (; b > 0; b--) {
      if (above + h[b] >= R) break;
      above += h[b];
    }
    sh->bucket = 4 * tid + b;
    sh->above = above;
    sh->inb = h[b];
  }
  __syncthreads();
}

// Keeps the k largest of cand[0, n) (n > k >= 1, k <= 1024) in cand[0, k), by radix
// select over the 64-bit composites (11-bit digits, most significant first). Histogram
// increments are aggregated per warp over equal digits (__match_any_sync), so runs of equal
// logits do not serialise on one counter. Returns the lower bound of the kept set: every
// kept composite is >= it and every dropped one is below it.
__device__ __noinline__ uint64_t select_top(uint64_t *cand, int n, int k, uint32_t *hist, Shared *sh) {
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  uint64_t prefix = 0;
  int pbits = 0;
  uint32_t R = (uint32_t)k;
  const int nround = (n + kThreads - 1) / kThreads * kThreads;  // warp-uniform trip count
  for (;;) {
    const int w = min(11, 64 - pbits);
    const int shift = 64 - pbits - w;
    const uint64_t dmask = (1ull << w) - 1ull;
    for (int i = tid; i < kBins; i += kThreads) hist[i] = 0;
    __syncthreads();
    for (int i = tid; i < nround; i += kThreads) {
      bool in = false;
      uint32_t digit = 0;
      if (i < n) {
        const uint64_t c = cand[i];
        in = pbits == 0 || (c >> (64 - pbits)) == prefix;
        digit = (uint32_t)((c >> shift) & dmask);
      }
      const uint32_t act = __ballot_sync(0xffffffffu, in);
      if (in) {
        const uint32_t peers = __match_any_sync(act, digit);
        if (lane == __ffs(peers) - 1) atomicAdd(&hist[digit], (uint32_t)__popc(peers));
      }
    }
    __syncthreads();
    find_bucket(hist, R, sh);
    const uint32_t b = sh->bucket, above = sh->above, inb = sh->inb;
    R -= above;
    prefix = (prefix << w) | b;
    pbits += w;
    if (inb == R || pbits == 64) break;  // the bucket is taken whole
  }
  const uint64_t thr = pbits == 64 ? prefix : (prefix << (64 - pbits));
  // Exactly k composites are >= thr: collect them in the histogram space (1024 slots),
  // then copy them to the front of the buffer.
  uint64_t *tmp = reinterpret_cast<uint64_t *>(hist);
  if (tid == 0) sh->count2 = 0;
  __syncthreads();
  for (int i = tid; i < nround; i += kThreads) {
    const uint64_t c = i < n ? cand[i] : 0ull;
    const bool keep = i < n && c >= thr;
    const uint32_t mask = __ballot_sync(0xffffffffu, keep);
    if (mask) {
      const int leader = __ffs(mask) - 1;
      uint32_t base = 0;
      if (lane == leader) base = atomicAdd(&sh->count2, (uint32_t)__popc(mask));
      base = __shfl_sync(0xffffffffu, base, leader);
      const uint32_t slot = base + __popc(mask & ((1u << lane) - 1u));
      if (keep && CHECK(slot < (uint32_t)(kBins / 2), 4, slot, n)) tmp[slot] = c;
    }
  }
  __syncthreads();
  for (int i = tid; i < k; i += kThreads) cand[i] = tmp[i];
  __syncthreads();
  return thr;
}


// Bitonic network for N (a power of two, 128..1024) values held two per thread of a
// 512-thread block (elements 2t, 2t+1), descending. Fully unrolled: strides up to 32
// exchange through warp shuffles, larger ones through shared memory `a`.
template <int N>
__device__ __forceinline__ void sort_pow2_desc(uint64_t *a, uint64_t &v0, uint64_t &v1) {
  const int j0 = 2 * threadIdx.x, j1 = j0 + 1;
#pragma unroll
  for (int size = 2; size <= N; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      uint64_t p0, p1;
      if (stride == 1) {
        p0 = v1;
        p1 = v0;
      } else if (stride <= 32) {
        p0 = __shfl_xor_sync(0xffffffffu, v0, stride >> 1);
        p1 = __shfl_xor_sync(0xffffffffu, v1, stride >> 1);
      } else {
        __syncthreads();
        if (j0 < N) {
          a[j0] = v0;
          a[j1] = v1;
        }
        __syncthreads();
        p0 = j0 < N ? a[j0 ^ stride] : 0ull;
        p1 = j1 < N ? a[j1 ^ stride] : 0ull;
      }
      const bool lower0 = (j0 & stride) == 0, desc0 = (j0 & size) == 0;
      const bool lower1 = (j1 & stride) == 0, desc1 = (j1 & size) == 0;
      v0 = (lower0 == desc0) ? (v0 > p0 ? v0 : p0) : (v0 < p0 ? v0 : p0);
      v1 = (lower1 == desc1) ? (v1 > p1 ? v1 : p1) : (v1 < p1 ? v1 : p1);
    }
  }
}

// Sorts a[0, n) descending, n <= 1024 (block-uniform call, 512 threads): one warp for
// n <= 64, otherwise the smallest unrolled network that holds n.
__device__ __noinline__ void block_sort_desc(uint64_t *a, int n) {
  const int tid = threadIdx.x;
  if (n <= 1) {
    __syncthreads();
    return;
  }
  if (n <= 64) {
    if (tid < 32) {
      uint64_t v0 = 2 * tid < n ? a[2 * tid] : 0ull;
      uint64_t v1 = 2 * tid + 1 < n ? a[2 * tid + 1] : 0ull;
      warp_sort64_desc(v0, v1);
      if (2 * tid < n) a[2 * tid] = v0;
      if (2 * tid + 1 < n) a[2 * tid + 1] = v1;
    }
    __syncthreads();
    return;
  }
  const int j0 = 2 * tid, j1 = j0 + 1;
  uint64_t v0 = j0 < n ? a[j0] : 0ull;
  uint64_t v1 = j1 < n ? a[j1] : 0ull;
  if (n <= 128)
    sort_pow2_desc<128>(a, v0, v1);
  else if (n <= 256)
    sort_pow2_desc<256>(a, v0, v1);
  else if (n <= 512)
    sort_pow2_desc<512>(a, v0, v1);
  else
    sort_pow2_desc<1024>(a, v0, v1);
  __syncthreads();
  if (j0 < n) a[j0] = v0;
  if (j1 < n) a[j1] = v1;
  __syncthreads();
}

// 2048-element variant: four values a thread (elements 4t..4t+3), unrolled.
__device__ __forceinline__ void sort2048_desc(uint64_t *a, uint64_t (&v)[4]) {
  const int jb = 4 * threadIdx.x;
#pragma unroll
  for (int size = 2; size <= 2048; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      uint64_t p[4];
      if (stride <= 2) {
#pragma unroll
        for (int e = 0; e < 4; e++) p[e] = v[e ^ stride];
      } else if (stride <= 64) {
#pragma unroll
        for (int e = 0; e < 4; e++) p[e] = __shfl_xor_sync(0xffffffffu, v[e], stride >> 2);
      } else {
        __syncthreads();
#pragma unroll
        for (int e = 0; e < 4; e++) a[jb + e] = v[e];
        __syncthreads();
#pragma unroll
        for (int e = 0; e < 4; e++) p[e] = a[(jb + e) ^ stride];
      }
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const int j = jb + e;
        const bool lower = (j & stride) == 0, desc = (j & size) == 0;
        v[e] = (lower == desc) ? (v[e] > p[e] ? v[e] : p[e]) : (v[e] < p[e] ? v[e] : p[e]);
      }
    }
  }
}

// Sorts a[0, n) descending for n <= 2048 (block-uniform call).
__device__ __noinline__ void block_sort_desc_2k(uint64_t *a, int n) {
  if (n <= 1024) {
    block_sort_desc(a, n);
    return;
  }
  const int jb = 4 * threadIdx.x;
  uint64_t v[4];
#pragma unroll
  for (int e = 0; e < 4; e++) v[e] = jb + e < n ? a[jb + e] : 0ull;
  sort2048_desc(a, v);
  __syncthreads();
#pragma unroll
  for (int e = 0; e < 4; e++)
    if (jb + e < n) a[jb + e] = v[e];
  __syncthreads();
}

// Number of composites >= t in cand[0, n), the same in every thread.
__device__ __noinline__ int block_count_ge(const uint64_t *cand, int n, uint64_t t, Shared *sh) {
  int c = 0;
  for (int i = threadIdx.x; i < n; i += kThreads) c += cand[i] >= t ? 1 : 0;
  c = __reduce_add_sync(0xffffffffu, c);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) sh->red_u[threadIdx.x >> 5] = (uint32_t)c;
  __syncthreads();
  return (int)__reduce_add_sync(0xffffffffu, (threadIdx.x & 31) < kWarps ? sh->red_u[threadIdx.x & 31] : 0u);
}

// Keeps the composites >= t of cand[0, n) at the front, in order, in place: chunk by chunk
// every thread reads its element, a block scan gives the new positions (never past the
// chunk being read), then the kept elements are written. Returns how many were kept.
__device__ __noinline__ int block_keep_ge(uint64_t *cand, int n, uint64_t t, Shared *sh) {
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  int out = 0;
  for (int base = 0; base < n; base += kThreads) {
    const int i = base + tid;
    const uint64_t c = i < n ? cand[i] : 0ull;
    const bool keep = i < n && c >= t;
    const uint32_t mask = __ballot_sync(0xffffffffu, keep);
    __syncthreads();  // everyone has read this chunk (and the previous red_u is consumed)
    if (lane == 0) sh->red_u[w] = (uint32_t)__popc(mask);
    __syncthreads();
    int before = 0, all = 0;
#pragma unroll
    for (int q = 0; q < kWarps; q++) {
      const int cq = (int)sh->red_u[q];
      before += q < w ? cq : 0;
      all += cq;
    }
    if (keep) cand[out + before + __popc(mask & ((1u << lane) - 1u))] = c;
    out += all;
  }
  __syncthreads();
  return out;
}

// Shrinks cand[0, n) (n > limit >= k) to between k and `limit` composites that include its
// k largest. A sorted sample of 64 candidates proposes actual candidates as thresholds; a
// block count accepts one or moves the sample rank. Returns the threshold (a valid lower
// bound of the k-th largest: at least k composites are >= it); falls back to the exact
// radix select when no sampled rank fits.
__device__ __noinline__ uint64_t shrink_to(uint64_t *cand, int n, int k, int limit, uint32_t *hist,
                              Shared *sh, int *kept) {
  const int tid = threadIdx.x;
  if (tid < 32) {
    uint64_t v0 = cand[(int)(((int64_t)(2 * tid) * n) >> 6)];
    uint64_t v1 = cand[(int)(((int64_t)(2 * tid + 1) * n) >> 6)];
    warp_sort64_desc(v0, v1);
    sh->samp[2 * tid] = v0;
    sh->samp[2 * tid + 1] = v1;
  }
  __syncthreads();
  // Sample rank r stands for about (r + 1) * n / 64 candidates; aim between k and limit.
  const int target = (k + limit) / 2;
  int r = (int)(((int64_t)target * 64) / n) - 1;
  r = min(max(r, 0), 63);
  for (int round = 0; round < 6; round++) {
    const uint64_t t = sh->samp[r];
    const int c = block_count_ge(cand, n, t, sh);
    if (c >= k && c <= limit) {
      *kept = block_keep_ge(cand, n, t, sh);
      return t;
    }
    if (c < k) {
      if (r == 63) break;
      r = min(63, r + max(1, (int)(((int64_t)(k - c) * 64 + n - 1) / n)));
    } else {
      if (r == 0) break;
      r = max(0, r - max(1, (int)(((int64_t)(c - limit) * 64 + n - 1) / n)));
    }
  }
  const uint64_t thr = select_top(cand, n, k, hist, sh);
  *kept = k;
  return thr;
}

// ------------------------------------------------------------------------------------
// sampleFromTopK on the device (sampler.ts:147-212).
//
// The reference makes three decisions from left-to-right float64 sums: the top-p cut,
// the drawn candidate and poolExhausted. Here those sums come from parallel trees /
// scans of fast estimates of the terms (approx_exact / approx_scaled); each decision is
// taken from them only when its margin exceeds decision_bound(n), a rigorous bound on
// the difference to the reference's sums, otherwise thread 0 replays the reference's
// arithmetic (decide_sequential). The token id, considered count and poolExhausted
// therefore always equal the reference's; the reported probability is the reference's
// exp(l - max) / sumExp of the chosen candidate, computed exactly (js_exp); poolMass is
// the parallel sum (within 1e-12 relative of the reference's) unless the replay ran.
// ------------------------------------------------------------------------------------
__device__ __noinline__ void finalize_sample(const int32_t *ids, const float *vals, int n,
                                             float max_logit, float sum_exp,
                                             tabby_sampling_params p, double u, double *cum,
                                             double *work, Shared *sh,
                                             tabby_sample_outcome *out, uint32_t status) {
  const int tid = threadIdx.x;
  if (status != TABBY_OK || n == 0) {
    if (tid == 0) {
      tabby_sample_outcome o;
      o.id = -1;
      o.considered_count = 0;
      o.probability = 0.0;
      o.pool_mass = 0.0;
      o.pool_exhausted = 0;
      o.pool_size = n;
      o.max_logit = max_logit;
      o.sum_exp = sum_exp;
      o.status = status != TABBY_OK ? (int32_t)status : (int32_t)TABBY_EEMPTY;
      o.reserved = 0;
      *out = o;
    }
    return;
  }
  const bool sample = p.temperature > 0;
  const double inv_sum = 1.0 / (double)sum_exp;
  const double inv_t = sample ? 1.0 / p.temperature : 0.0;
  // Two consecutive candidates a thread (n <= 2 * blockDim.x).
  const int i0 = 2 * tid, i1 = 2 * tid + 1;
  double e0 = 0.0, e1 = 0.0, s0 = 0.0, s1 = 0.0;
  if (i0 < n) {
    e0 = approx_exact(vals[i0], max_logit, inv_sum);
    if (sample) s0 = approx_scaled(vals[i0], max_logit, inv_t);
  }
  if (i1 < n) {
    e1 = approx_exact(vals[i1], max_logit, inv_sum);
    if (sample) s1 = approx_scaled(vals[i1], max_logit, inv_t);
  }
  const double pool_mass = block_sum_f64(e0 + e1, sh);
  const double bound = decision_bound(n);

  int32_t cut = 1, chosen = 0, exhausted = 0;
  bool fallback = false;
  if (sample) {
    const double st = block_sum_f64(s0 + s1, sh);
    const double inv_st = 1.0 / st;
    const double w0 = i0 < n ? s0 * inv_st : 0.0;
    const double w1 = i1 < n ? s1 * inv_st : 0.0;
    const double before = block_exclusive_scan_f64(w0 + w1, sh);
    const double c0 = before + w0;
    const double c1 = c0 + w1;
    if (i0 < n) cum[i0] = c0;
    if (i1 < n) cum[i1] = c1;
    if (tid == 0) {
      sh->cut_claim = n;
      sh->chosen_claim = n;
      sh->fallback = 0;
    }
    __syncthreads();
    cut = n;
    if (p.top_p < 1) {
      // First i with cumulative >= top_p (sampler.ts:175-189).
      if (i0 < n && c0 >= p.top_p)
        atomicMin(&sh->cut_claim, i0);
      else if (i1 < n && c1 >= p.top_p)
        atomicMin(&sh->cut_claim, i1);
      if (pool_mass < p.top_p) exhausted = 1;
      __syncthreads();
      const int ci = sh->cut_claim;
      if (tid == 0) {
        bool ok = fabs(pool_mass - p.top_p) > bound;
        if (ci < n)
          ok = ok && (cum[ci] - p.top_p > bound) && (ci == 0 || p.top_p - cum[ci - 1] > bound);
        else
          ok = ok && (p.top_p - cum[n - 1] > bound);
        if (!ok) sh->fallback = 1;
      }
      cut = ci < n ? ci + 1 : n;
    }
    // target = u * total; first i < cut with target < cumulative (sampler.ts:191-203).
    const double total = cum[cut - 1];
    const double target = u * total;
    if (i0 < cut && target < c0)
      atomicMin(&sh->chosen_claim, i0);
    else if (i1 < cut && target < c1)
      atomicMin(&sh->chosen_claim, i1);
    __syncthreads();
    const int ch = sh->chosen_claim;
    if (tid == 0) {
      bool ok = ch < cut;
      if (ok)
        ok = (cum[ch] - target > 2 * bound) && (ch == 0 || target - cum[ch - 1] > 2 * bound);
      if (!ok) sh->fallback = 1;
    }
    __syncthreads();
    chosen = ch < cut ? ch : cut - 1;
    fallback = sh->fallback != 0;
  }
  if (tid == 0) {
    tabby_sample_outcome o;
    double pm = pool_mass;
    if (fallback) {
      const Decision d =
          decide_sequential(vals, n, max_logit, sum_exp, p.temperature, p.top_p, u, work);
      chosen = d.chosen;
      cut = d.cut;
      exhausted = d.pool_exhausted;
      pm = d.pool_mass;
    }
    o.id = ids[chosen];
    o.considered_count = cut;
    o.probability = exact_prob(vals[chosen], max_logit, sum_exp);
    o.pool_mass = pm;
    o.pool_exhausted = exhausted;
    o.pool_size = n;
    o.max_logit = max_logit;
    o.sum_exp = sum_exp;
    o.status = TABBY_OK;
    o.reserved = fallback ? 1 : 0;  // 1 when the sequential replay decided
    *out = o;
  }
}


// The min(64, n) largest of cand[0, n), sorted descending, into cand[0, 64) (zeros past
// n). Block-uniform call. Every warp keeps a running top 64 of its share in registers
// (sort 64, merge); a four-level tree then merges the 16 lists through tmp (960 slots),
// one barrier a level.
__device__ __noinline__ void top64_sorted(uint64_t *cand, int n, uint64_t *tmp) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int per = ((n + kWarps - 1) / kWarps + 63) & ~63;
  const int b0 = min(n, warp * per), b1 = min(n, b0 + per);
  uint64_t a0 = 0, a1 = 0;
  for (int base = b0; base < b1; base += 64) {
    uint64_t c0 = base + 2 * lane < b1 ? cand[base + 2 * lane] : 0ull;
    uint64_t c1 = base + 2 * lane + 1 < b1 ? cand[base + 2 * lane + 1] : 0ull;
    warp_sort64_desc(c0, c1);
    if (base == b0) {
      a0 = c0;
      a1 = c1;
    } else {
      warp_merge64_desc(a0, a1, c0, c1);
    }
  }
  int off = 0;
#pragma unroll
  for (int h = kWarps / 2; h >= 1; h >>= 1) {
    if (warp >= h && warp < 2 * h) {
      tmp[off + (warp - h) * 64 + 2 * lane] = a0;
      tmp[off + (warp - h) * 64 + 2 * lane + 1] = a1;
    }
    __syncthreads();
    if (warp < h)
      warp_merge64_desc(a0, a1, tmp[off + warp * 64 + 2 * lane], tmp[off + warp * 64 + 2 * lane + 1]);
    off += h * 64;
  }
  if (warp == 0) {
    cand[2 * lane] = a0;
    cand[2 * lane + 1] = a1;
  }
  __syncthreads();
}

// sampleFromTopK for n <= 64 candidates in one warp (lane l holds candidates 2l, 2l+1:
// logits x0, x1), with warp shuffles only. Same float64 arithmetic, the same error bound
// on the parallel sums and the same sequential replay as finalize_sample; `scratch`
// holds 192 doubles for the replay.
__device__ __noinline__ void finalize_warp(int32_t id0, int32_t id1, float x0, float x1, int n,
                                           float max_logit, float sum_exp,
                                           tabby_sampling_params p, double u, double *scratch,
                                           tabby_sample_outcome *out, uint32_t status) {
  const unsigned kAll = 0xffffffffu;
  const int lane = threadIdx.x & 31;
  if (status != TABBY_OK || n == 0) {
    if (lane == 0) {
      tabby_sample_outcome o;
      o.id = -1;
      o.considered_count = 0;
      o.probability = 0.0;
      o.pool_mass = 0.0;
      o.pool_exhausted = 0;
      o.pool_size = n;
      o.max_logit = max_logit;
      o.sum_exp = sum_exp;
      o.status = status != TABBY_OK ? (int32_t)status : (int32_t)TABBY_EEMPTY;
      o.reserved = 0;
      *out = o;
    }
    return;
  }
  const bool sample = p.temperature > 0;
  const int i0 = 2 * lane, i1 = i0 + 1;
  const double inv_sum = 1.0 / (double)sum_exp;
  const double inv_t = sample ? 1.0 / p.temperature : 0.0;
  const double e0 = i0 < n ? approx_exact(x0, max_logit, inv_sum) : 0.0;
  const double e1 = i1 < n ? approx_exact(x1, max_logit, inv_sum) : 0.0;
  const double s0 = (sample && i0 < n) ? approx_scaled(x0, max_logit, inv_t) : 0.0;
  const double s1 = (sample && i1 < n) ? approx_scaled(x1, max_logit, inv_t) : 0.0;
  double pm = e0 + e1;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) pm += __shfl_xor_sync(kAll, pm, o);
  const double bound = decision_bound(n);

  int32_t cut = 1, chosen = 0, exhausted = 0;
  bool fallback = false;
  double c0 = 0.0, c1 = 0.0;
  // cum[i] from the lane that holds it (i warp-uniform).
  auto cum_at = [&](int i) -> double {
    const double a = __shfl_sync(kAll, c0, (i >> 1) & 31);
    const double b = __shfl_sync(kAll, c1, (i >> 1) & 31);
    return (i & 1) ? b : a;
  };
  if (sample) {
    double st = s0 + s1;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) st += __shfl_xor_sync(kAll, st, o);
    const double inv_st = 1.0 / st;
    const double w0 = i0 < n ? s0 * inv_st : 0.0;
    const double w1 = i1 < n ? s1 * inv_st : 0.0;
    double incl = w0 + w1;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double t = __shfl_up_sync(kAll, incl, o);
      if (lane >= o) incl += t;
    }
    double excl = __shfl_up_sync(kAll, incl, 1);
    if (lane == 0) excl = 0.0;
    c0 = excl + w0;
    c1 = c0 + w1;
    cut = n;
    if (p.top_p < 1) {
      // First i with cumulative >= top_p (sampler.ts:175-189).
      const bool h0 = i0 < n && c0 >= p.top_p, h1 = i1 < n && c1 >= p.top_p;
      const unsigned bal = __ballot_sync(kAll, h0 || h1);
      int ci = n;
      if (bal) {
        const int L = __ffs(bal) - 1;
        ci = __shfl_sync(kAll, h0 ? 1 : 0, L) ? 2 * L : 2 * L + 1;
      }
      exhausted = pm < p.top_p ? 1 : 0;
      bool ok = fabs(pm - p.top_p) > bound;
      if (ci < n) {
        const double here = cum_at(ci), prev = cum_at(ci > 0 ? ci - 1 : 0);
        ok = ok && (here - p.top_p > bound) && (ci == 0 || p.top_p - prev > bound);
      } else {
        ok = ok && (p.top_p - cum_at(n - 1) > bound);
      }
      fallback = !ok;
      cut = ci < n ? ci + 1 : n;
    }
    // target = u * total; first i < cut with target < cumulative (sampler.ts:191-203).
    const double target = u * cum_at(cut - 1);
    const bool g0 = i0 < cut && target < c0, g1 = i1 < cut && target < c1;
    const unsigned bal = __ballot_sync(kAll, g0 || g1);
    int ch = cut;
    if (bal) {
      const int L = __ffs(bal) - 1;
      ch = __shfl_sync(kAll, g0 ? 1 : 0, L) ? 2 * L : 2 * L + 1;
    }
    bool ok = ch < cut;
    if (ok) {
      const double here = cum_at(ch), prev = cum_at(ch > 0 ? ch - 1 : 0);
      ok = (here - target > 2 * bound) && (ch == 0 || target - prev > 2 * bound);
    }
    fallback = fallback || !ok;
    chosen = ch < cut ? ch : cut - 1;
  }
  if (fallback) {
    // Exact replay of the reference's left-to-right float64 arithmetic.
    float *xs = reinterpret_cast<float *>(scratch);
    double *wk = scratch + 32;
    if (i0 < n) xs[i0] = x0;
    if (i1 < n) xs[i1] = x1;
    __syncwarp();
    int32_t dv[3] = {0, 0, 0};
    double dpm = 0.0;
    if (lane == 0) {
      const Decision d =
          decide_sequential(xs, n, max_logit, sum_exp, p.temperature, p.top_p, u, wk);
      dv[0] = d.chosen;
      dv[1] = d.cut;
      dv[2] = d.pool_exhausted;
      dpm = d.pool_mass;
    }
    chosen = __shfl_sync(kAll, dv[0], 0);
    cut = __shfl_sync(kAll, dv[1], 0);
    exhausted = __shfl_sync(kAll, dv[2], 0);
    pm = __shfl_sync(kAll, dpm, 0);
  }
  const int32_t cid = __shfl_sync(kAll, (chosen & 1) ? id1 : id0, (chosen >> 1) & 31);
  const float cx = __shfl_sync(kAll, (chosen & 1) ? x1 : x0, (chosen >> 1) & 31);
  if (lane == 0) {
    tabby_sample_outcome o;
    o.id = cid;
    o.considered_count = cut;
    o.probability = exact_prob(cx, max_logit, sum_exp);
    o.pool_mass = pm;
    o.pool_exhausted = exhausted;
    o.pool_size = n;
    o.max_logit = max_logit;
    o.sum_exp = sum_exp;
    o.status = TABBY_OK;
    o.reserved = fallback ? 1 : 0;  // 1 when the sequential replay decided
    *out = o;
  }
}

// Sorts cand[0, n) descending into out[0, min(n, R)) for n <= kThreads by rank: each
// thread counts the composites above its own (broadcast reads of the whole list).
// Block-uniform call; out must not overlap cand[0, n).
__device__ __forceinline__ void rank_sort_small(const uint64_t *cand, int n, int R, uint64_t *out) {
  const int tid = threadIdx.x;
  if (tid < n) {
    const uint64_t c = cand[tid];
    int r = 0;
    for (int q = 0; q < n; q++) r += cand[q] > c ? 1 : 0;
    if (r < R) out[r] = c;
  }
  __syncthreads();
}

constexpr int kRankSortMax = 160;  // lists ranked by all-pairs counting (rank_sort_small)

// Exact top-R (R = min(k, n)) with its order. Candidates are binned on their key
// relative to the smallest one (2048 bins, the shift set by the key range); bins are
// counted and turned into offsets in descending order; the bins down to the one that
// holds the R-th are scattered into a grouped list behind the input; every element's
// position is its bin's offset plus the number of larger composites in its bin. Writes
// the R largest of cand[0, n), sorted descending, to cand[0, R) and returns R; returns
// -1 without changing cand when the grouped list does not fit behind the input (cand
// holds `capacity` slots) or a bin
// holds more than 512 elements (long runs of equal logits), for the caller's fallback.
// Block-uniform call.
__device__ __noinline__ int bin_rank_topk(uint64_t *cand, int n, int k, int capacity,
                                          uint32_t *hist, Shared *sh) {
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int R = min(k, n);
  // Key range.
  uint32_t kmin = 0xffffffffu, kmax = 0u;
  for (int i = tid; i < n; i += kThreads) {
    const uint32_t key = (uint32_t)(cand[i] >> 32);
    kmin = min(kmin, key);
    kmax = max(kmax, key);
  }
  kmin = __reduce_min_sync(0xffffffffu, kmin);
  kmax = __reduce_max_sync(0xffffffffu, kmax);
  if (lane == 0) {
    sh->red_u[w] = kmin;
    sh->red_u2[w] = kmax;
  }
  for (int i = tid; i < kBins; i += kThreads) hist[i] = 0;
  __syncthreads();
  kmin = partials_min_u32(sh->red_u);
  kmax = partials_max_u32(sh->red_u2);
  const uint32_t range = kmax - kmin;
  const int shift = max(0, 32 - __clz((int)range) - 11);  // (range >> shift) < 2048
  for (int i = tid; i < n; i += kThreads)
    atomicAdd(&hist[((uint32_t)(cand[i] >> 32) - kmin) >> shift], 1u);
  __syncthreads();
  // In place: hist[b] = elements in bins above b (exclusive suffix sum, high bins first).
  uint32_t h[4], mine = 0, big = 0;
#pragma unroll
  for (int j = 0; j < 4; j++) {
    h[j] = hist[4 * tid + j];
    mine += h[j];
    big = max(big, h[j]);
  }
  uint32_t inc = mine;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t t = __shfl_down_sync(0xffffffffu, inc, o);
    if (lane + o < 32) inc += t;
  }
  big = __reduce_max_sync(0xffffffffu, big);
  __syncthreads();  // everyone has read hist and the red arrays
  if (lane == 0) {
    sh->red_u[w] = inc;
    sh->red_u2[w] = big;
  }
  __syncthreads();
  big = partials_max_u32(sh->red_u2);
  if (big > 512u) return -1;  // block-uniform
  uint32_t off = inc - mine + partials_sum_above_u32(sh->red_u, w);
  for (int j = 3; j >= 0; j--) {
    if (off < (uint32_t)R && off + h[j] >= (uint32_t)R) {
      sh->bucket = 4 * tid + j;
      sh->above = off;
      sh->inb = h[j];
    }
    hist[4 * tid + j] = off;
    off += h[j];
  }
  __syncthreads();
  const uint32_t kb = sh->bucket;
  const int kept = (int)(sh->above + sh->inb);  // elements in bins >= kb
  if (n + kept > capacity) return -1;  // block-uniform
  uint64_t *g = cand + n;
  for (int i = tid; i < n; i += kThreads) {
    const uint64_t c = cand[i];
    const uint32_t b = ((uint32_t)(c >> 32) - kmin) >> shift;
    if (b >= kb) g[atomicAdd(&hist[b], 1u)] = c;
  }
  __syncthreads();
  // Now hist[b] is the end of bin b and hist[b + 1] its start.
  for (int p = tid; p < kept; p += kThreads) {
    const uint64_t c = g[p];
    const uint32_t b = ((uint32_t)(c >> 32) - kmin) >> shift;
    const int s = b + 1 < (uint32_t)kBins ? (int)hist[b + 1] : 0;
    const int e = (int)hist[b];
    int r = 0;
    for (int q = s; q < e; q++) r += g[q] > c ? 1 : 0;
    if (s + r < R) cand[s + r] = c;
  }
  __syncthreads();
  return R;
}

// The min(k, n) largest of cand[0, n) (k <= 1024), sorted descending, at cand[0, ...);
// returns how many. Block-uniform call. Lists of at most kRankSortMax are ranked directly,
// longer ones through the binned ranking; long runs of equal logits fall back to the
// per-warp top-64 tree (pools up to 64) or the exact radix select and a sort.
__device__ __forceinline__ int top_sorted(uint64_t *cand, int n, int k, int capacity,
                                          uint32_t *hist, Shared *sh) {
  if (k <= 0 || n <= 0) {
    __syncthreads();
    return 0;
  }
  if (n <= kRankSortMax && 2 * n <= capacity) {
    // Short lists: rank every element against all the others (a pass over the list per
    // thread; the binned ranking's fixed cost is lower from about 160 elements on), then
    // move the result to the front.
    rank_sort_small(cand, n, min(k, n), cand + n);
    const int R = min(k, n);
    for (int i = threadIdx.x; i < R; i += kThreads) cand[i] = cand[n + i];
    __syncthreads();
    return R;
  }
  const int r = bin_rank_topk(cand, n, k, capacity, hist, sh);
  if (r >= 0) return r;
  if (k <= 64) {
    top64_sorted(cand, n, reinterpret_cast<uint64_t *>(hist));
    return min(k, n);
  }
  if (n > k) {
    select_top(cand, n, k, hist, sh);
    n = k;
  }
  block_sort_desc(cand, n);
  return n;
}

// ------------------------------------------------------------------------------------
// The row pass: one cooperative row_kernel launch, a plan phase then the units.
//
// plan_row (one CTA a row) resets the row's counters, fixes its pool size k and its
// place in the processing order (rows with pools above 64 first, so that the rows whose
// finish is cheap come last), and estimates a threshold from a sample of 512 float4
// groups in 32 runs spread over the row: a logit with about rr sample logits at or above
// it, rr = min(k, mu + 4 sqrt(mu) + 6), mu the expected sample count above the row's
// k-th largest, so that the row holds at least k logits at or above it with near
// certainty (rr = k never fails: the sample is part of the row). It publishes the row
// as its position entry, tagged with the epoch.
//
// The units: every CTA takes (row, chunk) units from a global counter in that order, so
// fast CTAs take more. A unit streams its chunk once, appends its candidate groups to
// its warps' regions of the row's list and its per-warp statistics to the row's table;
// the unit that completes a row finishes it: it checks the estimate (at least min(k, V)
// candidates and no overflow, else the row is filtered again exactly), keeps the k
// best, sorts them and runs sampleFromTopK. Rows finish while other rows still stream.
// ------------------------------------------------------------------------------------
struct PassArgs {
  const float *logits;
  int64_t row_stride;
  int32_t rows, vocab;
  int32_t nch, chunk;  // chunks a row, logits a chunk (a multiple of 4)
  int32_t whole;       // 1: whole rows a CTA, threshold from the stream (no plan phase)
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
  uint32_t *sched;       // [0] unit counter, [2] the last chunked launch's epoch (the
                         // launch's last take of a unit resets [0] and stores [2])
  unsigned long long *pos_entry;  // [rows][2] by processing position, each word tagged
                                 // with the epoch: (epoch, row << 12 | k), (epoch, tf)
  uint32_t *rng_state;   // kModeSample: per-row mulberry32 state, or NULL (uniforms)
  uint32_t *row_done;    // [rows] chunks finished
  uint32_t *warp_cnt;    // [rows][nch * kWarps] candidate groups of each (chunk, warp)
  uint32_t *row_flags;   // [rows] kFlagBadInput | kRowOverflow
  float *row_tf;         // [rows] threshold, by row
  float *row_tf_lo;      // [rows] a lower threshold (far safer rank), by row
  float2 *warp_stats;    // [rows][nch][kWarps] (max, sum-exp)
  float4 *row_gval;      // [rows][kRowGroups] candidate groups: warp w of chunk c owns the
  int32_t *row_gidx;     //   region (c * kWarps + w) of region_slots() slots
  uint32_t spin_limit;   // polls of the bounded wait for a row's plan entry
  int32_t withhold_row;  // tests only: this row's plan entry is never published (-1: none)
};

// Candidate slots of the row's list each chunk owns.
__device__ __forceinline__ int region_slots(const PassArgs &a) {
  return kRowGroups / (a.nch * kWarps);
}

constexpr uint32_t kRowOverflow = 8u;  // the row's candidates did not fit: filter it again

// Appends c to the candidate buffer when pred holds (warp-uniform call). Slots past
// `cap` are not written; the overflow flag records the loss.
__device__ __forceinline__ void insert_candidate(bool pred, uint64_t c, uint64_t *cand, int cap,
                                                 uint32_t *count, uint32_t *overflow) {
  const uint32_t mask = __ballot_sync(0xffffffffu, pred);
  if (mask == 0) return;
  const int lane = threadIdx.x & 31;
  const int leader = __ffs(mask) - 1;
  uint32_t base = 0;
  if (lane == leader) base = atomicAdd(count, (uint32_t)__popc(mask));
  base = __shfl_sync(0xffffffffu, base, leader);
  const uint32_t slot = base + __popc(mask & ((1u << lane) - 1u));
  if (pred) {
    if (slot < (uint32_t)cap)
      cand[slot] = c;
    else
      *overflow = 1u;
  }
}

// Pool size of a row (inference.worker.ts:120-123 with the handle's cap in sample mode).
__device__ __forceinline__ int32_t row_pool(const PassArgs &a, int row, uint32_t *pflags) {
  if (a.mode == kModeSample) {
    const tabby_sampling_params p = a.params[row];
    if (isnan(p.temperature) || isnan(p.top_p)) *pflags = kFlagBadParams;
    return min(pool_rule(p.temperature, p.top_k, a.cap), a.vocab);
  }
  return min(a.fixed_k, a.vocab);
}

// First float4-aligned logit of [lo, hi) and the number of whole float4 groups after it.
struct Span {
  int a0, a1, ngroups;
};
__device__ __forceinline__ Span aligned_span(const float *rowp, int lo, int hi) {
  const int mis = (int)((reinterpret_cast<uintptr_t>(rowp + lo) >> 2) & 3);
  Span s;
  s.a0 = min(lo + ((4 - mis) & 3), hi);
  s.a1 = s.a0 + ((hi - s.a0) & ~3);
  s.ngroups = (s.a1 - s.a0) >> 2;
  return s;
}

// The row the plan puts at processing position `pos` (thread-level call): rows with pools
// above 64 first, each group in row order, as plan_row orders them. Used only when the
// wait for a plan entry runs out.
__device__ __noinline__ int row_at_position(const PassArgs &a, int pos) {
  int large = 0;
  for (int r = 0; r < a.rows; r++) {
    uint32_t f = 0;
    large += row_pool(a, r, &f) > 64 ? 1 : 0;
  }
  int lb = 0, sb = 0;
  for (int r = 0; r < a.rows; r++) {
    uint32_t f = 0;
    const bool lg = row_pool(a, r, &f) > 64;
    if ((lg ? lb : large + sb) == pos) return r;
    lb += lg ? 1 : 0;
    sb += lg ? 0 : 1;
  }
  return 0;
}

// Plans one row (block-uniform call): resets its counters, fixes its pool size and its
// place in the processing order, estimates its threshold, then publishes the row's
// position entry, tagged with the epoch (release). cand holds 2048 slots.
__device__ __noinline__ void plan_row(const PassArgs &a, int row, uint64_t *cand,
                                      uint32_t *hist, Shared *sh) {
  int (*red)[kWarps] = sh->plan_red;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float *rowp = a.logits + (int64_t)row * a.row_stride;
  uint32_t pf = 0;
  const int k = row_pool(a, row, &pf);
  if (tid == 0) {
    a.row_done[row] = 0;
    a.row_flags[row] = 0;
  }
  // The sample: 32 runs of 16 consecutive float4 groups (256 contiguous bytes, whole DRAM
  // bursts), spread evenly over the aligned middle of the row; one group a thread, its
  // load in flight while the row order is worked out.
  const Span sp = aligned_span(rowp, 0, a.vocab);
  constexpr int kPlanSample = kThreads;  // float4 groups sampled
  constexpr int kPlanRun = 16;
  constexpr int kPlanRuns = kPlanSample / kPlanRun;
  const int S = min(kPlanSample, sp.ngroups);
  int g = tid;  // short rows: every group
  if (S == kPlanSample) {
    const int run = tid / kPlanRun;
    const int start = (int)(((2LL * run + 1) * sp.ngroups) / (2LL * kPlanRuns)) - kPlanRun / 2;
    g = max(0, min(start, sp.ngroups - kPlanRun)) + tid % kPlanRun;
  }
  const bool sampled = k > 0 && tid < S;
  float4 sv = make_float4(0.f, 0.f, 0.f, 0.f);
  if (sampled) sv = __ldg(reinterpret_cast<const float4 *>(rowp + sp.a0) + g);
  // Place in the order: rows with k > 64 first, each group in row order.
  int large = 0, large_before = 0, small_before = 0;
  for (int r = tid; r < a.rows; r += kThreads) {
    uint32_t f = 0;
    const int lg = row_pool(a, r, &f) > 64 ? 1 : 0;
    large += lg;
    if (r < row) {
      large_before += lg;
      small_before += 1 - lg;
    }
  }
  large = __reduce_add_sync(0xffffffffu, large);
  large_before = __reduce_add_sync(0xffffffffu, large_before);
  small_before = __reduce_add_sync(0xffffffffu, small_before);
  if (lane == 0) {
    red[0][warp] = large;
    red[1][warp] = large_before;
    red[2][warp] = small_before;
  }
  uint64_t t1 = 0, t2 = 0;
  if (sampled) {
    const float xs[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
    for (int e = 0; e < 4; e++) {
      const uint64_t c = composite(key_of(xs[e]), (uint32_t)(sp.a0 + 4 * g + e));
      if (c > t1) {
        t2 = t1;
        t1 = c;
      } else if (c > t2) {
        t2 = c;
      }
    }
  }
  cand[2 * tid] = t1;
  cand[2 * tid + 1] = t2;
  __syncthreads();
  if (tid == 0) {
    int lt = 0, lb = 0, sb = 0;
    for (int w = 0; w < kWarps; w++) {
      lt += red[0][w];
      lb += red[1][w];
      sb += red[2][w];
    }
    sh->unit = (uint32_t)(k > 64 ? lb : lt + sb);  // this row's processing position
  }
  float tf = -__int_as_float(0x7f800000);  // no estimate: every logit is a candidate
  float tf_lo = tf;
  if (k > 0) {
    const int ns = 4 * S;
    const float mu = (float)k * (float)ns / (float)a.vocab;
    // The sample is part of the row, so rr = k can never fail; for larger k the
    // statistical rank is smaller (and the check at the end of the pass guards it).
    const int rr = min(k, (int)ceilf(mu + 4.f * sqrtf(mu) + 6.f));
    // The per-thread top two stand in for the sample's top (at least rr sample logits
    // are at or above their rr-th largest).
    if (rr >= 1 && rr < 2 * min(S, kThreads) && rr < ns) {
      // rr2: a far safer rank, the starting threshold of the exact re-filter.
      const int rr2 = min(4 * rr, 2 * min(S, kThreads) - 1);
      uint64_t thr, thr2;
      if (bin_rank_topk(cand, 2 * kThreads, rr2, 4 * kThreads, hist, sh) >= 0) {
        thr = cand[rr - 1];
        thr2 = cand[rr2 - 1];
      } else {
        thr = thr2 = select_top(cand, 2 * kThreads, rr, hist, sh);
      }
      if ((thr >> 32) != 0ull) tf = float_of_key((uint32_t)(thr >> 32));
      if ((thr2 >> 32) != 0ull) tf_lo = float_of_key((uint32_t)(thr2 >> 32));
    }
  }
  if (tid == 0 && row != a.withhold_row) {
    const int pos = (int)sh->unit;
    a.row_tf[row] = tf;
    a.row_tf_lo[row] = tf_lo;
    __threadfence();
    const unsigned long long tag = (unsigned long long)sh->epoch << 32;
    st_release_u64(&a.pos_entry[2 * pos], tag | ((unsigned long long)row << 12) | (uint32_t)k);
    st_release_u64(&a.pos_entry[2 * pos + 1], tag | __float_as_uint(tf));
  }
  __syncthreads();  // the slots and sh are free again
}

// Filters a whole row again, exactly (block-uniform call): candidates are the logits
// >= start_tf (a threshold of far safer rank than the failed estimate), and when those
// are fewer than k, every logit; compaction (keep a superset of the k best, raise the
// threshold) makes room. Returns the candidate count (at least min(k, vocab)).
__device__ __noinline__ int rescan_row(const float *rowp, int vocab, int k, float start_tf,
                                       uint64_t *cand, uint32_t *hist, Shared *sh) {
  const int tid = threadIdx.x, warp = tid >> 5;
  const Span sp = aligned_span(rowp, 0, vocab);
  const float4 *p4 = reinterpret_cast<const float4 *>(rowp + sp.a0);
  const float kNegInf = -__int_as_float(0x7f800000);
  for (int attempt = 0; attempt < 2; attempt++) {
    float tf = attempt == 0 ? start_tf : kNegInf;
    uint64_t tau = tf == kNegInf ? 0ull : ((uint64_t)key_of(tf) << 32);
    __syncthreads();
    if (tid == 0) {
      sh->count = 0;
      sh->overflow = 0;
    }
    __syncthreads();
    if (warp == 0) {
      const int e = tid < 4 ? tid : sp.a1 + (tid - 4);
      const bool in = tid < 8 && (tid < 4 ? (e < sp.a0) : (e < vocab));
      const float x = in ? __ldcg(rowp + e) : 0.f;
      const uint64_t c = composite(key_of(x), (uint32_t)(in ? e : 0));
      insert_candidate(in && c >= tau, c, cand, kFinishCap, &sh->count, &sh->overflow);
    }
    for (int base = 0; base < sp.ngroups; base += kThreads) {
      __syncthreads();
      if (sh->count > (uint32_t)(kFinishCap - 4 * kThreads)) {
        int kept;
        const uint64_t thr =
            shrink_to(cand, (int)sh->count, k, max(2 * k, 1024), hist, sh, &kept);
        if (tid == 0) sh->count = (uint32_t)kept;
        __syncthreads();
        tau = thr;
        tf = float_of_key((uint32_t)(thr >> 32));
      }
      const int g = base + tid;
      const float4 w = g < sp.ngroups ? __ldcg(p4 + g) : make_float4(0.f, 0.f, 0.f, 0.f);
      const bool hit = g < sp.ngroups && max3f(w.x, w.y, fmaxf(w.z, w.w)) >= tf;
      if (__any_sync(0xffffffffu, hit)) {
        const float xs[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int e = 0; e < 4; e++) {
          const uint64_t c = composite(key_of(xs[e]), (uint32_t)(sp.a0 + 4 * g + e));
          insert_candidate(hit && c >= tau, c, cand, kFinishCap, &sh->count, &sh->overflow);
        }
      }
    }
    __syncthreads();
    if ((int)sh->count >= min(k, vocab)) break;  // block-uniform
  }
  return (int)sh->count;
}

// SeededRandom.next() (sampler.ts:112-118, mulberry32) on a device-resident state: advances
// the state and returns u32 / 2^32.
__device__ __forceinline__ double rng_next(uint32_t *state) {
  const uint32_t s = *state + 0x6d2b79f5u;
  *state = s;
  uint32_t t = s;
  t = (t ^ (t >> 15)) * (t | 1u);
  t ^= t + (t ^ (t >> 7)) * (t | 61u);
  return (double)(t ^ (t >> 14)) / 4294967296.0;
}

// The finish of one row, run by the CTA whose unit completed it (block-uniform call).
__device__ __noinline__ void finish_row(const PassArgs &a, int row, int k, uint64_t *cand,
                                        uint32_t *hist, Shared *sh) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const float *rowp = a.logits + (int64_t)row * a.row_stride;
  uint32_t pflags = 0;
  // Everything the finish reads from global memory, issued together.
  const int np = a.nch * kWarps;
  float2 st = make_float2(-3.40282347e38f, 0.f);
  int rcount = 0;
  if (a.whole) {  // the CTA's own warps: their tables are in shared memory
    if (tid < kWarps) {
      st = sh->wst[tid];
      rcount = (int)sh->wgroups[tid];
    }
  } else if (tid < np) {
    st = __ldcg(&a.warp_stats[(int64_t)row * np + tid]);
    rcount = (int)__ldcg(&a.warp_cnt[(int64_t)row * np + tid]);
  }
  const uint32_t rflags = __ldcg(&a.row_flags[row]);
  const float tf = a.row_tf[row];
  tabby_sampling_params prm = {};
  double uni = 0.0;
  if (a.mode == kModeSample) {
    prm = a.params[row];
    if (!a.rng_state) uni = a.uniforms[row];
    if (isnan(prm.temperature) || isnan(prm.top_p)) pflags = kFlagBadParams;
  }
  // Region counts (one a thread) and their exclusive offsets in the gathered list, kept
  // in the histogram space (np <= 512 entries).
  uint32_t *roff = hist;
  int rincl = rcount;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, rincl, o);
    if (lane >= o) rincl += t;
  }
  if (lane == 31) sh->red_u2[warp] = (uint32_t)rincl;
  // Statistics of every warp of every chunk, merged in a fixed order.
  float bm = st.x;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, o));
  if (lane == 0) sh->red_f[warp] = bm;
  __syncthreads();
  float M = lane < kWarps ? sh->red_f[lane] : -3.40282347e38f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
  float contrib = st.y > 0.f ? st.y * __expf(st.x - M) : 0.f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) contrib += __shfl_xor_sync(0xffffffffu, contrib, o);
  if (lane == 0) sh->red_f2[warp] = contrib;
  __syncthreads();
  float S = lane < kWarps ? sh->red_f2[lane] : 0.f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) S += __shfl_xor_sync(0xffffffffu, S, o);
  const float row_max = M, sum_exp = S;
  // The region offsets (sh->red_u2 was published by the barriers above).
  const int rbefore = (int)partials_sum_above_u32(sh->red_u2, -1) -
                      (int)partials_sum_above_u32(sh->red_u2, warp - 1);
  if (tid < np) roff[tid] = (uint32_t)(rbefore + rincl - rcount);
  const int total = (int)partials_sum_above_u32(sh->red_u2, -1);  // candidate groups of the row
  __syncthreads();

  int n = 0;
  if (k > 0 && !(rflags & kFlagTimeout)) {
    bool ok = !(rflags & kRowOverflow);
    if (ok) {
      // Expand the groups into composites of their logits >= tf. Every group is one
      // independent pair of loads; a warp reserves its slots with one atomic.
      if (tid == 0) {
        sh->count = 0;
        sh->overflow = 0;
      }
      __syncthreads();
      const int regsize = region_slots(a);
      const float4 *gv = a.row_gval + (int64_t)row * kRowGroups;
      const int32_t *gi = a.row_gidx + (int64_t)row * kRowGroups;
      // Four groups a thread in flight at once, then their logits >= tf as composites.
      constexpr int kBatch = 4;
      for (int r0 = 0; r0 < total; r0 += kBatch * kThreads) {
        float4 xb[kBatch];
        int bb[kBatch];
#pragma unroll
        for (int j = 0; j < kBatch; j++) {
          const int i = r0 + j * kThreads + tid;
          xb[j] = make_float4(kNegSentinel, kNegSentinel, kNegSentinel, kNegSentinel);
          bb[j] = 0;
          if (i < total) {
            // The region holding gathered element i: the last offset <= i.
            int lo_r = 0, hi_r = np - 1;
            while (lo_r < hi_r) {
              const int mid = (lo_r + hi_r + 1) >> 1;
              if ((int)roff[mid] <= i)
                lo_r = mid;
              else
                hi_r = mid - 1;
            }
            const int64_t at = (int64_t)lo_r * regsize + (i - (int)roff[lo_r]);
            xb[j] = __ldcg(gv + at);
            bb[j] = __ldcg(gi + at);
          }
        }
        // This thread's logits >= tf over its batch, one warp scan and one atomic.
        uint32_t hm = 0;  // 4 bits a group
#pragma unroll
        for (int j = 0; j < kBatch; j++) {
          const float4 x = xb[j];
          if (r0 + j * kThreads + tid < total)
            hm |= ((x.x >= tf ? 1u : 0u) | (x.y >= tf ? 2u : 0u) | (x.z >= tf ? 4u : 0u) |
                   (x.w >= tf ? 8u : 0u))
                  << (4 * j);
        }
        const int nh = __popc(hm);
        int incl = nh;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int t = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += t;
        }
        const int wtotal = __shfl_sync(0xffffffffu, incl, 31);
        uint32_t wb = 0;
        if (lane == 31 && wtotal > 0) wb = atomicAdd(&sh->count, (uint32_t)wtotal);
        wb = __shfl_sync(0xffffffffu, wb, 31);
        uint32_t slot = wb + (uint32_t)(incl - nh);
#pragma unroll
        for (int j = 0; j < kBatch; j++) {
          const uint32_t jm = (hm >> (4 * j)) & 15u;
          if (jm) {
            const float4 x = xb[j];
#pragma unroll
            for (int e = 0; e < 4; e++) {
              if ((jm >> e) & 1u) {
                const float xe = e == 0 ? x.x : e == 1 ? x.y : e == 2 ? x.z : x.w;
                if (slot < (uint32_t)kFinishCap)
                  cand[slot] = composite(key_of(xe), (uint32_t)(bb[j] + e));
                else
                  sh->overflow = 1u;
                slot++;
              }
            }
          }
        }
      }
      __syncthreads();
      n = (int)sh->count;
      ok = sh->overflow == 0u && n >= k;
      __syncthreads();
    }
    if (!ok) n = rescan_row(rowp, a.vocab, k, __ldcg(&a.row_tf_lo[row]), cand, hist, sh);
  }
  const int kk = top_sorted(cand, n, k, kFinishCap, hist, sh);
  const uint32_t flags = (rflags & (kFlagBadInput | kFlagTimeout)) | pflags;
  const uint32_t status = (flags & kFlagTimeout)     ? (uint32_t)TABBY_ETIMEOUT
                          : (flags & kFlagBadInput)  ? (uint32_t)TABBY_EINPUT
                          : (flags & kFlagBadParams) ? (uint32_t)TABBY_EINVAL
                                                     : (uint32_t)TABBY_OK;
  if (k <= 64) {
    // Small pools: warp 0 finishes the row alone.
    if (warp != 0) return;
    const uint64_t c0 = cand[2 * lane], c1 = cand[2 * lane + 1];
    const int32_t id0 = (int32_t)~(uint32_t)c0, id1 = (int32_t)~(uint32_t)c1;
    float x0 = float_of_key((uint32_t)(c0 >> 32)), x1 = float_of_key((uint32_t)(c1 >> 32));
    if (2 * lane < kk && (uint32_t)(c0 >> 32) == 0x80000000u) x0 = rowp[id0];  // sign of a zero
    if (2 * lane + 1 < kk && (uint32_t)(c1 >> 32) == 0x80000000u) x1 = rowp[id1];
    const float max_logit = kk > 0 ? __shfl_sync(0xffffffffu, x0, 0) : row_max;
    if (a.mode == kModeTopK || a.mode == kModeShard) {
      float *blk = a.block + (int64_t)row * a.block_ld;
      const int slots = a.mode == kModeShard ? TABBY_SHARD_TOP_K : k;
      if (lane == 0) {
        blk[0] = status == TABBY_OK ? max_logit : __int_as_float(0x7fc00000);
        blk[1] = sum_exp;
      }
#pragma unroll
      for (int e = 0; e < 2; e++) {
        const int i = 2 * lane + e;
        if (i < slots) {
          const bool in = i < kk;
          blk[2 + 2 * i] = in ? (e ? x1 : x0) : __int_as_float(0xff800000);  // -inf pad
          blk[3 + 2 * i] = __uint_as_float(
              in ? (uint32_t)((int64_t)(e ? id1 : id0) + a.index_offset) : 0xffffffffu);
        }
      }
      return;
    }
    if (a.topk_ids) {
      if (2 * lane < kk) a.topk_ids[(int64_t)row * a.topk_ld + 2 * lane] = id0;
      if (2 * lane + 1 < kk) a.topk_ids[(int64_t)row * a.topk_ld + 2 * lane + 1] = id1;
    }
    if (a.topk_values) {
      if (2 * lane < kk) a.topk_values[(int64_t)row * a.topk_ld + 2 * lane] = x0;
      if (2 * lane + 1 < kk) a.topk_values[(int64_t)row * a.topk_ld + 2 * lane + 1] = x1;
    }
    if (a.rng_state) {
      // The reference draws only when it samples: after the empty-pool throw and the
      // greedy return (sampler.ts:153,159-167).
      double un = 0.0;
      if (lane == 0 && status == TABBY_OK && kk > 0 && prm.temperature > 0)
        un = rng_next(&a.rng_state[row]);
      uni = __shfl_sync(0xffffffffu, un, 0);
    }
    finalize_warp(id0, id1, x0, x1, kk, max_logit, sum_exp, prm, uni,
                  reinterpret_cast<double *>(hist), &a.out[row], status);
    return;
  }
  // Unpack into (id, value) in the histogram space; once that is done the candidate
  // buffer holds the float64 finalize arrays.
  int32_t *ids = reinterpret_cast<int32_t *>(hist);
  float *vals = reinterpret_cast<float *>(ids + kk);
  double *cum = reinterpret_cast<double *>(cand);
  double *scaled = cum + kk;  // the replay's work space
  uint64_t mine[2];
  for (int j = 0; j < 2; j++) mine[j] = tid + j * kThreads < kk ? cand[tid + j * kThreads] : 0ull;
  __syncthreads();
  for (int j = 0; j < 2; j++) {
    const int i = tid + j * kThreads;
    if (i < kk) {
      const uint32_t key = (uint32_t)(mine[j] >> 32);
      const uint32_t idx = ~(uint32_t)mine[j];
      float v = float_of_key(key);
      if (key == 0x80000000u) v = rowp[idx];  // keep the sign of a zero logit
      ids[i] = (int32_t)idx;
      vals[i] = v;
    }
  }
  __syncthreads();
  const float max_logit = kk > 0 ? vals[0] : row_max;
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
  if (a.topk_ids)
    for (int i = tid; i < kk; i += kThreads) a.topk_ids[(int64_t)row * a.topk_ld + i] = ids[i];
  if (a.topk_values)
    for (int i = tid; i < kk; i += kThreads) a.topk_values[(int64_t)row * a.topk_ld + i] = vals[i];
  if (a.rng_state) {  // drawn only when the reference draws (see the warp path)
    if (tid == 0)
      sh->rng_u = status == TABBY_OK && kk > 0 && prm.temperature > 0
                      ? rng_next(&a.rng_state[row])
                      : 0.0;
    __syncthreads();
    uni = sh->rng_u;
  }
  finalize_sample(ids, vals, kk, max_logit, sum_exp, prm, uni, cum, scaled, sh,
                  &a.out[row], status);
}

// Packed pair arithmetic of sm_100 (two fp32 lanes in one 64-bit register pair).
__device__ __forceinline__ unsigned long long f2_pack(float lo, float hi) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_unpack(unsigned long long v, float &lo, float &hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ unsigned long long f2_fma(unsigned long long a, unsigned long long b,
                                                     unsigned long long c) {
  unsigned long long r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ unsigned long long f2_add(unsigned long long a, unsigned long long b) {
  unsigned long long r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ unsigned long long f2_mul(unsigned long long a, unsigned long long b) {
  unsigned long long r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
// 2^x of both lanes (two MUFU.EX2), packed again.
__device__ __forceinline__ unsigned long long f2_ex2(unsigned long long v) {
  float lo, hi;
  f2_unpack(v, lo, hi);
  return f2_pack(ex2_approx(lo), ex2_approx(hi));
}

// Threshold of a row streamed whole by one CTA, from the first iteration of every warp's
// segment (16 runs of up to 512 contiguous logits spread evenly over the row), which
// stage 0 holds when this runs (block-uniform call). Each thread keeps the top two
// composites of its up to 16 logits; the rr-th largest of those 1024 is at or below the
// sample's rr-th largest, so the estimate errs towards more candidates. The rank rule is
// the plan's (rr = min(k, ceil(mu + 4 sqrt(mu) + 6)), mu = k * sample / vocab). buf
// (2048 slots) and hist must not overlap stages 0 and 1.
__device__ __noinline__ float whole_threshold(const PassArgs &a, int row, int k, uint32_t sslot0,
                                              int wn, int seg, int ngroups, int gbase,
                                              uint64_t *buf, uint32_t *hist, Shared *sh) {
  const int tid = threadIdx.x, lane = tid & 31;
  uint64_t t1 = 0, t2 = 0;
#pragma unroll
  for (int q = 0; q < kVec; q++) {
    if (q * 32 + lane < wn) {
      const float4 v = ld_shared_f4(sslot0 + (uint32_t)(q * kThreads * 16));
      const float xs[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const uint64_t c = composite(key_of(xs[e]), (uint32_t)(gbase + 4 * (q * 32 + lane) + e));
        if (c > t1) {
          t2 = t1;
          t1 = c;
        } else if (c > t2) {
          t2 = c;
        }
      }
    }
  }
  buf[2 * tid] = t1;
  buf[2 * tid + 1] = t2;
  int ns = 0;  // logits sampled (the same arithmetic for every thread)
  for (int w = 0; w < kWarps; w++) {
    const int g0 = min(w * seg, ngroups);
    ns += 4 * min(kWarpIter, min(g0 + seg, ngroups) - g0);
  }
  __syncthreads();
  float tf = -__int_as_float(0x7f800000);  // no estimate: every logit is a candidate
  if (k > 0) {
    const float mu = (float)k * (float)ns / (float)a.vocab;
    const int rr = min(k, (int)ceilf(mu + 4.f * sqrtf(mu) + 6.f));
    if (rr >= 1 && rr < 2 * kThreads && rr < ns) {
      // Only rank rr is ranked (a ranking down to a safer rank cost more than the rare
      // re-filter it would shorten): the re-filter of a whole row starts from every logit.
      uint64_t thr;
      if (bin_rank_topk(buf, 2 * kThreads, rr, 4 * kThreads, hist, sh) >= 0)
        thr = buf[rr - 1];
      else
        thr = select_top(buf, 2 * kThreads, rr, hist, sh);
      if ((thr >> 32) != 0ull) tf = float_of_key((uint32_t)(thr >> 32));
    }
  }
  if (tid == 0) {
    a.row_tf[row] = tf;
    a.row_tf_lo[row] = -__int_as_float(0x7f800000);
  }
  __syncthreads();  // buf and hist are free again
  return tf;
}

__global__ void __launch_bounds__(kThreads, 2) row_kernel(const __grid_constant__ PassArgs a) {
  // Shared memory: the cp.async stages of the streaming loop; the finish reuses them as
  // its composite buffer (kFinishCap) followed by the histogram.
  extern __shared__ __align__(128) unsigned char smem_raw[];
  float4 *stage = reinterpret_cast<float4 *>(smem_raw);  // [kStages][kVec][kThreads]
  uint64_t *fin = reinterpret_cast<uint64_t *>(smem_raw);
  uint32_t *hist = reinterpret_cast<uint32_t *>(fin + kFinishCap);
  Shared *sh = reinterpret_cast<Shared *>(smem_raw + kStageBytes);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int units = a.rows * a.nch;
  constexpr float kLog2e = 1.44269504088896341f;
  const float kNaN = __int_as_float(0x7fc00000);
  const float4 kPast = make_float4(-3.40282347e38f, -3.40282347e38f, -3.40282347e38f,
                                   -3.40282347e38f);
  // Plan phase: every CTA plans rows blockIdx.x, blockIdx.x + gridDim.x, ... and
  // publishes each as an epoch-tagged position entry; a unit waits only for its own row's entry, so
  // streaming starts as soon as the first rows are planned. The launch is cooperative:
  // every CTA is resident, so every awaited row gets planned.
  uint32_t *sched = a.sched;  // the unit counter
  // Chunked rows need this launch's epoch (one more than the last chunked launch's, kept
  // in the scratch; never 0), which tags the plan entries; whole rows have no plan.
  if (tid == 0 && !a.whole) {
    uint32_t e = __ldcg(&a.sched[2]) + 1u;
    sh->epoch = e == 0u ? 1u : e;  // read before this CTA's first unit is taken
  }
  // Every CTA takes units until one lies past the end, so a launch makes exactly
  // units + gridDim.x takes; the last one resets the counter for the next launch and
  // records the epoch (every CTA has read it by then).
  auto take = [&]() -> int {  // thread 0 only
    const uint32_t t = atomicAdd(sched, 1u);
    if (t == (uint32_t)(a.rows * a.nch) + gridDim.x - 1u) {
      *sched = 0u;
      if (!a.whole) a.sched[2] = sh->epoch;
    }
    return (int)t;
  };
  if (!a.whole)
    for (int r = blockIdx.x; r < a.rows; r += gridDim.x) plan_row(a, r, fin, hist, sh);

  // Unit schedule, kept by thread 0: at the end of a unit it counts the unit into its row
  // (the unit that completes a row finishes it at once), then takes the next unit and its
  // row data.
  int nid = 0, nrow = 0, nk = 0;
  float ntf = 0.f;
  // Thread 0: the row data of unit nid, once its row is planned. The wait is bounded:
  // when it runs out, the unit's row is worked out from the parameters, flagged with
  // kFlagTimeout and the unit streamed with no candidates (threshold +inf), so the row
  // still completes and its finish reports TABBY_ETIMEOUT; the counters stay exact.
  auto unit_info = [&]() {
    if (nid >= units) return;
    if (a.whole) {  // unit = row; the threshold comes from the stream
      uint32_t f = 0;
      nrow = nid;
      nk = row_pool(a, nid, &f);
      ntf = 0.f;
      return;
    }
    const int ri = nid / a.nch;
    uint32_t spins = 0;
    unsigned long long w0, w1;
    for (;;) {  // both words of this launch's entry: one round trip once planned
      w0 = ld_acquire_u64(&a.pos_entry[2 * ri]);
      w1 = ld_acquire_u64(&a.pos_entry[2 * ri + 1]);
      if ((uint32_t)(w0 >> 32) == sh->epoch && (uint32_t)(w1 >> 32) == sh->epoch) break;
      if (++spins > a.spin_limit) {
        uint32_t f = 0;
        nrow = row_at_position(a, ri);
        nk = row_pool(a, nrow, &f);
        ntf = __int_as_float(0x7f800000);
        atomicOr(&a.row_flags[nrow], kFlagTimeout);
        return;
      }
      __nanosleep(100);
    }
    nrow = (int)((uint32_t)w0 >> 12);
    nk = (int)((uint32_t)w0 & 0xfffu);
    ntf = __uint_as_float((uint32_t)w1);
  };
  if (tid == 0) {
    nid = take();
    unit_info();
    sh->unit = (uint32_t)nid;
    sh->urow = nrow;
    sh->uk = nk;
    sh->utf = ntf;
  }
  __syncthreads();
  for (;;) {
    if (sh->unit == 0xffffffffu) {
      // The previous unit finished a row without asking for its successor: ask now, so
      // a CTA busy finishing never holds on to a unit other CTAs could take.
      __syncthreads();
      if (tid == 0) {
        nid = take();
        unit_info();
        sh->unit = (uint32_t)nid;
        sh->urow = nrow;
        sh->uk = nk;
        sh->utf = ntf;
      }
      __syncthreads();
    }
    const int unit = (int)sh->unit;
    const int row = sh->urow;
    const int k = sh->uk;
    float tf = sh->utf;
    if (unit >= units) break;
    const int ri = unit / a.nch;
    const int chunk = unit - ri * a.nch;
    const float *rowp = a.logits + (int64_t)row * a.row_stride;
    const int lo = chunk * a.chunk;
    const int hi = min(lo + a.chunk, a.vocab);
    const Span sp = aligned_span(rowp, lo, hi);
    const float4 *p4 = reinterpret_cast<const float4 *>(rowp + sp.a0);

    // Per-thread online statistics, two packed lanes: s = sum exp(x - m) as
    // 2^((x - m) * log2(e)).
    float m = -3.40282347e38f;
    unsigned long long s2 = 0ull;  // (0.f, 0.f)
    float mL = 0.f;      // rn(m * log2(e)) for the FFMA form of the exponent argument
    bool small = false;  // |m| small enough for the FFMA form
    float mn = 3.40282347e38f;  // running min: catches -inf and the -3e38 sentinel

    // Candidate groups go straight to this warp's region of the row's global list; the
    // warp counts them (wcnt, warp-uniform). A full region sends the row to the exact
    // re-filter.
    const int regsize = region_slots(a);
    const int64_t region = (int64_t)row * kRowGroups + (int64_t)(chunk * kWarps + warp) * regsize;
    float4 *rgv = a.row_gval + region;
    int32_t *rgi = a.row_gidx + region;
    int wcnt = 0;

    // Warp segments: warp w streams the float4 groups [sg0, sg0 + wn) of the chunk's
    // aligned middle, 128 groups (2 KB, four 512-byte coalesced loads) an iteration.
    const int seg = (sp.ngroups + kWarps - 1) / kWarps;
    const int sg0 = min(warp * seg, sp.ngroups);
    const int wn = min(sg0 + seg, sp.ngroups) - sg0;
    const int wit = (wn + kWarpIter - 1) / kWarpIter;
    const float4 *wp = p4 + sg0;
    const int gbase = sp.a0 + 4 * sg0;  // logit index of this warp's first group

    // Iteration it's groups of this thread go to its own slots of stage it % kStages by
    // cp.async (one commit group an iteration); slots of groups past the segment get
    // -FLT_MAX instead. They come back into registers once the group has landed.
    const uint32_t sslot = smem_u32(stage + tid);  // slot (s, q) at + (s * kVec + q) * 8 KB
    const float4 *gsrc = wp + lane;                // this thread's group of the next issue
    const uint64_t pol = l2_evict_first_policy();  // the logits are read once
    int inext = 0;                                 // iteration of the next issue
    // Issues iteration inext into stage S (compile-time) and advances. Slots of groups
    // past the segment get -FLT_MAX.
    auto issue = [&](auto SC) {
      constexpr int S = decltype(SC)::value;
      if (inext + 1 < wit) {
#pragma unroll
        for (int q = 0; q < kVec; q++)
          cp_async16_u32(sslot + (uint32_t)((S * kVec + q) * kThreads * 16), gsrc + q * 32, pol);
      } else if (inext < wit) {
        const int rem = wn - inext * kWarpIter - lane;
#pragma unroll
        for (int q = 0; q < kVec; q++) {
          const uint32_t dst = sslot + (uint32_t)((S * kVec + q) * kThreads * 16);
          if (q * 32 < rem)
            cp_async16_u32(dst, gsrc + q * 32, pol);
          else
            st_shared_f4(dst, kPast);
        }
      }
      cp_async_commit();  // one group an iteration, empty past the segment
      gsrc += kWarpIter;
      inext++;
    };
    // One iteration from stage S: statistics, the refill of the stage, the filter.
    auto step = [&](auto SC, int it) {
      constexpr int S = decltype(SC)::value;
      cp_async_wait_group<kStages - 1>();  // iteration it has landed
      float4 v[kVec];
#pragma unroll
      for (int q = 0; q < kVec; q++)
        v[q] = ld_shared_f4(sslot + (uint32_t)((S * kVec + q) * kThreads * 16));
      const bool full = it + 1 < wit;
      // Group maxima, iteration max and min. Groups past the segment hold -FLT_MAX: they
      // never raise the max, add exp(-huge) = 0 to the sum and are skipped by the min.
      float gm[kVec];
#pragma unroll
      for (int q = 0; q < kVec; q++) gm[q] = max3f(v[q].x, v[q].y, fmaxf(v[q].z, v[q].w));
      const float im = max3f(gm[0], gm[1], fmaxf(gm[2], gm[3]));
      if (full) {
        float l = min3f(min3f(v[0].x, v[0].y, v[0].z), min3f(v[0].w, v[1].x, v[1].y),
                        min3f(v[1].z, v[1].w, v[2].x));
        l = min3f(l, min3f(v[2].y, v[2].z, v[2].w),
                  min3f(v[3].x, v[3].y, min3f(v[3].z, v[3].w, l)));
        mn = fminf(mn, l);
      } else {
#pragma unroll
        for (int q = 0; q < kVec; q++)
          if (it * kWarpIter + q * 32 + lane < wn)
            mn = min3f(mn, min3f(v[q].x, v[q].y, v[q].z), v[q].w);
      }
      if (im > m) {
        const float r = ex2_approx((m - im) * kLog2e);
        s2 = f2_mul(s2, f2_pack(r, r));
        m = im;
        mL = m * kLog2e;
        // fma(x, L, -rn(m*L)) differs from (x - m)*L by the rounding of m*L, at most
        // 2^-20 for |m| <= 16: every term then carries a factor within 7e-7 of 1 (well
        // inside the 1e-5 budget). Larger |m| uses the subtraction form.
        small = fabsf(m) <= 16.f;
      }
      if (small) {
        const unsigned long long L2 = f2_pack(kLog2e, kLog2e), nmL2 = f2_pack(-mL, -mL);
#pragma unroll
        for (int q = 0; q < kVec; q++) {
          const unsigned long long e01 = f2_ex2(f2_fma(f2_pack(v[q].x, v[q].y), L2, nmL2));
          const unsigned long long e23 = f2_ex2(f2_fma(f2_pack(v[q].z, v[q].w), L2, nmL2));
          s2 = f2_add(s2, f2_add(e01, e23));
        }
      } else {
        const unsigned long long L2 = f2_pack(kLog2e, kLog2e), nm2 = f2_pack(-m, -m);
#pragma unroll
        for (int q = 0; q < kVec; q++) {
          const unsigned long long e01 =
              f2_ex2(f2_mul(f2_add(f2_pack(v[q].x, v[q].y), nm2), L2));
          const unsigned long long e23 =
              f2_ex2(f2_mul(f2_add(f2_pack(v[q].z, v[q].w), nm2), L2));
          s2 = f2_add(s2, f2_add(e01, e23));
        }
      }
      issue(SC);  // refills stage S (its values are in registers and in use above)
      // Groups holding a logit >= tf go to the warp's region whole (the value check per
      // logit happens in the finish).
      if (k > 0 && __any_sync(0xffffffffu, im >= tf)) {
        const int rem = full ? kWarpIter : wn - it * kWarpIter - lane;
        const int base0 = gbase + 4 * (it * kWarpIter + lane);
        const uint32_t below = (1u << lane) - 1u;
        // One ballot a column of groups: slots in (column, lane) order.
#pragma unroll
        for (int q = 0; q < kVec; q++) {
          const bool hit = gm[q] >= tf && q * 32 < rem;
          const uint32_t mask = __ballot_sync(0xffffffffu, hit);
          if (hit) {
            const int slot = wcnt + __popc(mask & below);
            if (slot < regsize) {
              rgv[slot] = v[q];
              rgi[slot] = base0 + 4 * 32 * q;
            }
          }
          wcnt += __popc(mask);
        }
      }
    };
    using I0 = std::integral_constant<int, 0>;
    using I1 = std::integral_constant<int, 1>;
    using I2 = std::integral_constant<int, 2>;
    static_assert(kStages == 3, "the loop below is unrolled for three stages");
    issue(I0{});
    issue(I1{});
    if (a.whole) {
      // Whole rows: the threshold from iteration 0 (stage 0), while iteration 1 is in
      // flight; stage 2's region holds the selection until iteration 2 is issued.
      if (tid == 0) a.row_flags[row] = 0;
      cp_async_wait_group<1>();
      __syncthreads();
      uint64_t *sel = reinterpret_cast<uint64_t *>(smem_raw + 2 * (kStageBytes / kStages));
      tf = whole_threshold(a, row, k, sslot, wn, seg, sp.ngroups, gbase, sel,
                           reinterpret_cast<uint32_t *>(sel + 4 * kThreads), sh);
    }
    issue(I2{});
    // Ragged ends of the chunk: at most 3 logits before a0 and 3 after a1, one per lane
    // of warp 0, each kept as a group of its own (the other three slots NaN, which no
    // threshold admits).
    if (warp == 0) {
      const int e = lane < 4 ? lo + lane : sp.a1 + (lane - 4);
      const bool in = lane < 8 && (lane < 4 ? (e < sp.a0) : (e < hi));
      float rx = 0.f;
      if (in) {
        rx = __ldg(rowp + e);
        m = rx;
        mL = m * kLog2e;
        small = fabsf(m) <= 16.f;
        s2 = f2_pack(1.f, 0.f);
        mn = rx;
      }
      const bool take = in && k > 0 && rx >= tf;
      const uint32_t mask = __ballot_sync(0xffffffffu, take);
      if (take) {
        const int slot = wcnt + __popc(mask & ((1u << lane) - 1u));
        if (slot < regsize) {
          rgv[slot] = make_float4(rx, kNaN, kNaN, kNaN);
          rgi[slot] = e;
        }
      }
      wcnt += __popc(mask);
    }

    for (int it = 0; it < wit; it += kStages) {
      step(I0{}, it);
      if (it + 1 < wit) step(I1{}, it + 1);
      if (it + 2 < wit) step(I2{}, it + 2);
    }
    cp_async_wait_group<0>();

    // Per-warp statistics into the row's table.
    {
      float s_lo, s_hi;
      f2_unpack(s2, s_lo, s_hi);
      const float s = s_lo + s_hi;
      float wm = m;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) wm = fmaxf(wm, __shfl_xor_sync(0xffffffffu, wm, o));
      float ws = s > 0.f ? s * __expf(m - wm) : 0.f;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ws += __shfl_xor_sync(0xffffffffu, ws, o);
      // NaN or +inf logits leave s or m non-finite; -inf and values at or below the
      // reference's -3.0e38 sentinel show in the running min.
      const bool bad = !(s == s) || !(m <= 3.40282347e38f) || !(mn > kNegSentinel) ||
                       !(s <= 3.40282347e38f);
      const bool wbad = __any_sync(0xffffffffu, bad);
      if (lane == 0) {
        if (a.whole) {
          sh->wst[warp] = make_float2(wm, ws);
          sh->wgroups[warp] = (uint32_t)min(wcnt, regsize);
        } else {
          const int64_t at = ((int64_t)row * a.nch + chunk) * kWarps + warp;
          a.warp_stats[at] = make_float2(wm, ws);
          a.warp_cnt[at] = (uint32_t)min(wcnt, regsize);
        }
        const uint32_t f = (wbad ? kFlagBadInput : 0u) | (wcnt > regsize ? kRowOverflow : 0u);
        if (f) atomicOr(&a.row_flags[row], f);
      }
    }
    __syncthreads();  // every thread's candidate groups and statistics are written
    if (tid == 0) {
      if (!a.whole) __threadfence();  // ... and visible before the count (release)
      const bool last =
          a.whole || atomicAdd(&a.row_done[row], 1u) == (uint32_t)(a.nch - 1);
      // A unit that completes a row asks for its successor only after the finish, so a
      // CTA busy finishing never holds on to a unit other CTAs could take.
      if (!last) {
        nid = take();
        unit_info();  // the next unit's row data
      }
      sh->last = last ? 1u : 0u;
      sh->unit = last ? 0xffffffffu : (uint32_t)nid;
      sh->urow = nrow;
      sh->uk = nk;
      sh->utf = ntf;
    }
    __syncthreads();
    if (sh->last) {
      __threadfence();
      finish_row(a, row, k, fin, hist, sh);
      __syncthreads();  // the finish is done with the stage region before the loads reuse it
    }
  }
}

// ------------------------------------------------------------------------------------
// Vocab-sharded finish: one warp per row over the shard blocks (all-gathered, or in peer memory).
// ------------------------------------------------------------------------------------
// One row of the vocab-sharded merge by one warp: block s of the row is at
// bases[s] + src_row * a.block_ld. The shards' candidate lists (at most 64 each, sorted)
// are merged into the row's best 64 in registers (lane l holds 2l and 2l + 1), the
// (max, sum-exp) pairs are combined in shard order, and finalize_warp samples. Writes the
// outcome to *out; `status_in` (TABBY_OK or an error found by the
// caller) overrides the outcome's status. `scratch`: 192 doubles of this warp.
__device__ __noinline__ void merge_row_warp(const MergeLaunch &a, int row, int src_row,
                                            const float *const *bases, uint32_t status_in,
                                            tabby_sample_outcome *out, double *scratch) {
  const unsigned kAll = 0xffffffffu;
  const int lane = threadIdx.x & 31;
  const tabby_sampling_params p = a.params[row];
  auto blk = [&](int s) { return bases[s] + (int64_t)src_row * a.block_ld; };
  // Every load of the row's blocks is issued before any result is used (the blocks may
  // be in a peer's memory, a round trip over NVLink): lane s takes shard s's (max,
  // sum-exp); the candidates come four shards at a time, two a lane.
  float2 stat = make_float2(-3.40282347e38f, 0.f);
  if (lane < a.shards) stat = *reinterpret_cast<const float2 *>(blk(lane));
  uint64_t v0 = 0, v1 = 0;  // the best 64 composites of all shards so far (0 = empty slot)
  for (int s0 = 0; s0 < a.shards; s0 += 4) {
    float2 lo[4], hi[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
      if (s0 + j < a.shards) {
        const float2 *q = reinterpret_cast<const float2 *>(blk(s0 + j) + 2) + 2 * lane;
        lo[j] = q[0];  // (value, index bits) of candidate 2l
        hi[j] = q[1];  // ... of candidate 2l + 1
      }
    }
#pragma unroll
    for (int j = 0; j < 4; j++) {
      if (s0 + j < a.shards) {
        uint64_t c0 = 0, c1 = 0;
        const uint32_t g0 = __float_as_uint(lo[j].y), g1 = __float_as_uint(hi[j].y);
        if (g0 != 0xffffffffu) c0 = composite(key_of(lo[j].x), g0);
        if (g1 != 0xffffffffu) c1 = composite(key_of(hi[j].x), g1);
        warp_sort64_desc(c0, c1);
        if (s0 + j == 0) {
          v0 = c0;
          v1 = c1;
        } else {
          warp_merge64_desc(v0, v1, c0, c1);
        }
      }
    }
  }
  // M = max m_s; S = sum s_s * exp(m_s - M), shards in rank order (every lane computes
  // the same values from the pairs the lanes hold).
  float mx = -3.40282347e38f;
  double S = 0.0;
  uint32_t bad = 0;
  for (int s = 0; s < a.shards; s++) {
    const float ms = __shfl_sync(kAll, stat.x, s);
    if (ms != ms) bad = kFlagBadInput;
    mx = fmaxf(mx, ms);
  }
  for (int s = 0; s < a.shards; s++) {
    const float ms = __shfl_sync(kAll, stat.x, s), ss = __shfl_sync(kAll, stat.y, s);
    if (ss > 0.f) S = JS_ADD(S, JS_MUL((double)ss, js_exp(JS_SUB((double)ms, (double)mx))));
  }
  if (isnan(p.temperature) || isnan(p.top_p)) bad |= kFlagBadParams;
  const int nc = __popc(__ballot_sync(kAll, v0 != 0)) + __popc(__ballot_sync(kAll, v1 != 0));
  const int k = pool_rule(p.temperature, p.top_k, TABBY_SHARD_TOP_K);
  const int kk = min(k, nc);
  const int32_t id0 = (int32_t)~(uint32_t)v0, id1 = (int32_t)~(uint32_t)v1;
  float x0 = float_of_key((uint32_t)(v0 >> 32)), x1 = float_of_key((uint32_t)(v1 >> 32));
  // Recover the sign of a zero logit from the shard block that holds it (rare).
  for (int e = 0; e < 2; e++) {
    const uint64_t c = e ? v1 : v0;
    if (2 * lane + e < kk && (uint32_t)(c >> 32) == 0x80000000u) {
      const uint32_t gi = ~(uint32_t)c;
      for (int s = 0; s < a.shards; s++) {
        const float *b = blk(s);
        for (int j = 0; j < TABBY_SHARD_TOP_K; j++)
          if (__float_as_uint(b[3 + 2 * j]) == gi) {
            if (e)
              x1 = b[2 + 2 * j];
            else
              x0 = b[2 + 2 * j];
          }
      }
    }
  }
  const float max_logit = kk > 0 ? __shfl_sync(kAll, x0, 0) : mx;
  const uint32_t status = status_in != TABBY_OK        ? status_in
                          : (bad & kFlagBadInput)    ? (uint32_t)TABBY_EINPUT
                          : (bad & kFlagBadParams) ? (uint32_t)TABBY_EINVAL
                                                   : (uint32_t)TABBY_OK;
  if (a.topk_ids) {
    if (2 * lane < kk) a.topk_ids[(int64_t)row * a.topk_ld + 2 * lane] = id0;
    if (2 * lane + 1 < kk) a.topk_ids[(int64_t)row * a.topk_ld + 2 * lane + 1] = id1;
  }
  if (a.topk_values) {
    if (2 * lane < kk) a.topk_values[(int64_t)row * a.topk_ld + 2 * lane] = x0;
    if (2 * lane + 1 < kk) a.topk_values[(int64_t)row * a.topk_ld + 2 * lane + 1] = x1;
  }
  finalize_warp(id0, id1, x0, x1, kk, max_logit, (float)S, p, a.uniforms[row], scratch, out,
                status);
}

constexpr int kMergeWarps = 4;  // rows a merge CTA (one warp a row)

__global__ void __launch_bounds__(32 * kMergeWarps) merge_kernel(MergeLaunch a) {
  __shared__ const float *bases[kMaxShards];
  __shared__ double scratch[kMergeWarps][192];
  if (threadIdx.x < a.shards)
    bases[threadIdx.x] = a.gathered + (int64_t)threadIdx.x * a.rows * a.block_ld;
  __syncthreads();
  const int warp = threadIdx.x >> 5;
  const int row = blockIdx.x * kMergeWarps + warp;
  if (row < a.rows)
    merge_row_warp(a, row, row, bases, TABBY_OK, &a.out[row], scratch[warp]);
}

// ------------------------------------------------------------------------------------
// Vocab-sharded merge with the exchange over NVLink peer memory (one launch a rank).
//
// Every rank's local pass has written its blocks into its own exchange buffer (the one
// of the step's parity). This kernel (1) tells every peer that this rank's blocks of the
// step are ready (a system-scope fence, then a release store of the step's epoch into
// the peer's arrive word for this rank), (2) waits until every peer's arrive word here
// holds the epoch, and (3) merges every row, one warp a row, reading the peers' blocks
// straight from their buffers over NVLink. Every rank computes the same outcomes, so
// nothing else is exchanged. A rank rewrites a block buffer two steps later; by then
// every peer has announced the step in between, which it does only after its merge of
// this step has returned, so nobody still reads it. Every wait polls at most
// `timeout_ns` of %globaltimer; when a peer's word does not arrive in time every row
// reports TABBY_ETIMEOUT.
// ------------------------------------------------------------------------------------
__device__ __forceinline__ void st_release_sys_u32(uint32_t *p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Waits until flags[i] == epoch for i in [0, n), i != skip (one thread). Returns the mask
// of the slots that did not reach it in time.
__device__ uint32_t wait_flags(const uint32_t *flags, int n, int skip, uint32_t epoch,
                               uint64_t timeout_ns) {
  const uint64_t t0 = global_ns();
  uint32_t missing = (n >= 32 ? 0xffffffffu : ((1u << n) - 1u)) & ~(1u << skip);
  if (!missing) return 0u;
  for (;;) {
    for (int i = 0; i < n; i++)
      if (((missing >> i) & 1u) && ld_acquire_sys_u32(&flags[i]) == epoch) missing &= ~(1u << i);
    if (!missing || global_ns() - t0 > timeout_ns) return missing;
    __nanosleep(64);
  }
}


// Element q of a per-rank pointer array held in the kernel parameters, selected with
// constant indices (a dynamic index into the parameters would copy them to local memory).
template <typename T>
__device__ __forceinline__ T pick(const T (&arr)[TABBY_EXCHANGE_MAX_WORLD], int q) {
  T v = arr[0];
#pragma unroll
  for (int i = 1; i < TABBY_EXCHANGE_MAX_WORLD; i++)
    if (q == i) v = arr[i];
  return v;
}

__global__ void __launch_bounds__(32 * kMergeWarps) xmerge_kernel(const __grid_constant__ XMergeLaunch x) {
  __shared__ const float *bases[kMaxShards];
  __shared__ double scratch[kMergeWarps][192];
  __shared__ uint32_t missing;
  const MergeLaunch &a = x.m;
  const int tid = threadIdx.x;
  if (tid < x.world) bases[tid] = pick(x.peer_blocks, tid);
  if (blockIdx.x == 0 && tid < x.world && tid != x.rank) {
    // The local pass (the previous launch on this stream) has written the blocks.
    __threadfence_system();
    st_release_sys_u32(pick(x.peer_flags, tid) + x.rank, x.epoch);
  }
  // This rank's own blocks are ready by stream order; only the peers' are waited for.
  if (tid == 0) missing = wait_flags(x.flags, x.world, x.rank, x.epoch, x.timeout_ns);
  __syncthreads();
  const int warp = tid >> 5;
  const int row = (int)blockIdx.x * kMergeWarps + warp;
  if (row < a.rows)
    merge_row_warp(a, row, row, bases, missing ? (uint32_t)TABBY_ETIMEOUT : (uint32_t)TABBY_OK,
                   &a.out[row], scratch[warp]);
}

// ------------------------------------------------------------------------------------
// Host side: geometry and launches.
// ------------------------------------------------------------------------------------
static int round_up(int x, int m) { return (x + m - 1) / m * m; }

static size_t row_smem_bytes() {
  return (size_t)kStageBytes + sizeof(Shared) + 64;
}

// Units a CTA should see on average: enough for the dynamic schedule to even out the
// CTAs' speeds, few enough that the per-unit overhead stays small.
// Rows are split into chunks only until the units cover about 0.8 of the resident CTAs:
// every extra unit pays a pipeline refill and a cross-CTA hand-off to the row's finish,
// which measured dearer than leaving a few CTAs idle (B=256 on 296 CTAs runs fastest
// with whole rows).
constexpr int kUnitsPerCtaX10 = 8;

constexpr int kMaxDevices = 64;

namespace {
// Per-device set-up of the row kernel: the dynamic shared-memory attribute and the
// occupancy are properties of the kernel on one device, so each device is set up once,
// with that device current (the callers make it current), under std::call_once.
struct RowKernelSetup {
  std::once_flag once;
  cudaError_t err = cudaSuccess;
  int per_sm = 0;
};
RowKernelSetup g_row_setup[kMaxDevices];

cudaError_t row_kernel_setup(int *per_sm) {
  int dev = -1;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  RowKernelSetup &s = g_row_setup[dev];
  std::call_once(s.once, [&]() {
    s.err = cudaFuncSetAttribute(row_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)row_smem_bytes());
    int occ = 0;
    if (s.err == cudaSuccess)
      s.err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, row_kernel, kThreads,
                                                            row_smem_bytes());
    if (s.err == cudaSuccess && occ < 1) s.err = cudaErrorInvalidConfiguration;
    if (s.err == cudaSuccess) s.per_sm = std::min(occ, 2);
  });
  *per_sm = s.per_sm;
  return s.err;
}
}  // namespace

cudaError_t plan_rows(int32_t sms, int32_t rows, int32_t vocab, int32_t cap, RowGeometry *geo) {
  (void)cap;
  // Resident CTAs a SM (two 512-thread CTAs by design); the cooperative launch needs the
  // grid to fit at once.
  int per_sm = 0;
  cudaError_t err = row_kernel_setup(&per_sm);
  if (err != cudaSuccess) return err;
  const int ctas = per_sm * std::max(sms, 1);
  const int max_by_size = std::max(1, vocab / kMinChunk);
  int nch = (kUnitsPerCtaX10 * ctas + 10 * std::max(rows, 1) - 1) / (10 * std::max(rows, 1));
  nch = std::max(1, std::min(nch, std::min(kMaxChunks, max_by_size)));
  RowGeometry g;
  g.chunk = round_up((vocab + nch - 1) / nch, 4);
  g.nch = (vocab + g.chunk - 1) / g.chunk;
  g.grid = (int32_t)std::min<int64_t>((int64_t)rows * g.nch, ctas);
  g.whole = g.nch == 1 ? 1 : 0;
  g.smem_bytes = row_smem_bytes();
  *geo = g;
  return cudaSuccess;
}

cudaError_t launch_rows(const RowLaunch &l, const RowGeometry &geo, const Scratch &scr,
                        cudaStream_t stream) {
  if (l.rows == 0) return cudaSuccess;
  if (l.rows > scr.max_rows || geo.nch > kMaxChunks) return cudaErrorInvalidValue;
  PassArgs a;
  a.logits = l.logits;
  a.row_stride = l.row_stride;
  a.rows = l.rows;
  a.vocab = l.vocab;
  a.nch = geo.nch;
  a.chunk = geo.chunk;
  a.whole = geo.whole;
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
  a.sched = scr.sched;
  a.row_done = scr.row_done;
  a.warp_cnt = scr.warp_cnt;
  a.row_flags = scr.row_flags;
  a.row_tf = scr.row_tf;
  a.row_tf_lo = scr.row_tf_lo;
  a.pos_entry = scr.pos_entry;
  a.warp_stats = scr.warp_stats;
  a.row_gval = scr.row_gval;
  a.row_gidx = scr.row_gidx;
  a.rng_state = l.rng_state;
  a.spin_limit = l.spin_limit;
  a.withhold_row = l.withhold_row;
  int per_sm = 0;
  cudaError_t err = row_kernel_setup(&per_sm);
  if (err != cudaSuccess) return err;
  // Cooperative launch: all CTAs resident at once (units wait on rows other CTAs plan).
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)geo.grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = geo.smem_bytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, row_kernel, a);
}

cudaError_t launch_xmerge(const XMergeLaunch &l, cudaStream_t stream) {
  const int grid = std::max((l.m.rows + kMergeWarps - 1) / kMergeWarps, 1);
  xmerge_kernel<<<grid, 32 * kMergeWarps, 0, stream>>>(l);
  return cudaGetLastError();
}

cudaError_t launch_merge(const MergeLaunch &l, cudaStream_t stream) {
  if (l.rows == 0) return cudaSuccess;
  merge_kernel<<<(l.rows + kMergeWarps - 1) / kMergeWarps, 32 * kMergeWarps, 0, stream>>>(l);
  return cudaGetLastError();
}


// ------------------------------------------------------------------------------------
// Fused LM-head finish: one CTA a row over the per-CTA partials of lmhead_kernel
// (lmhead.cu). M = max m_c, S = sum s_c exp(m_c - M) in a fixed order, the global top-k
// (k <= kLmCands, the reference's MAX_TOP_K) of the CTAs' best logits by (value desc,
// index asc), then sampleFromTopK exactly as the row pass does.
// ------------------------------------------------------------------------------------
__host__ __device__ __forceinline__ int lm_merge_cap(int parts, int keep) {
  return max(kFinishCap, parts * min(max(keep, 1), kLmCands));
}

__global__ void __launch_bounds__(kThreads) lmhead_merge_kernel(LmheadMergeLaunch a) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  __shared__ Shared sh_s;
  Shared *sh = &sh_s;
  // Room for every entry the parts wrote (at least kFinishCap), then the histogram.
  const int cap = lm_merge_cap(a.parts, a.keep);
  uint64_t *cand = reinterpret_cast<uint64_t *>(smem_raw);
  uint32_t *hist = reinterpret_cast<uint32_t *>(cand + cap);
  const int row = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool exact_pass = a.keep >= kLmCands && a.row_flag != nullptr;
  // Launched with programmatic stream serialization (its launch overlaps the previous
  // kernel's tail): wait for the previous kernel in the stream to complete.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (exact_pass && __ldcg(a.row_flag + row) != a.epoch) return;  // settled by the fast pass
  const tabby_sampling_params prm = a.params[row];
  uint32_t pflags = (isnan(prm.temperature) || isnan(prm.top_p)) ? kFlagBadParams : 0u;
  const int k = min(pool_rule(prm.temperature, prm.top_k, kLmCands), a.vocab);
  double uni = (!a.rng_state && a.uniforms) ? a.uniforms[row] : 0.0;
  // The parts' candidates: raw value bits << 32 | id, each part's list sorted best first;
  // the first batch of loads is issued before anything waits on memory.
  const int total = a.parts * kLmCands;
  const unsigned long long *rc = a.cands + (int64_t)row * total;
  const int keep = min(a.keep, kLmCands);
  const int nent = a.parts * keep;  // the entries the parts wrote
  constexpr int kBatch = 10;        // a thread's loads in flight at once
  unsigned long long w[kBatch];
  auto load_batch = [&](int base) {
#pragma unroll
    for (int u = 0; u < kBatch; u++) {
      const int i = base + u * kThreads + tid;
      w[u] = i < nent ? __ldcg(rc + (i / keep) * kLmCands + i % keep) : 0xffffffffull;
    }
  };
  load_batch(0);
  auto comp_of = [](unsigned long long e) -> uint64_t {
    return (uint32_t)e == 0xffffffffu
               ? 0ull
               : composite(key_of(__uint_as_float((uint32_t)(e >> 32))), (uint32_t)e);
  };
  // Each part's best entry; the (max, sum-exp) entries combined in a fixed order (entry
  // i by thread i mod kThreads, in increasing i, then the block's trees), so the sum does
  // not depend on which CTA produced which entry.
  uint64_t *heads = reinterpret_cast<uint64_t *>(hist);  // [parts]: free until the top-k
  uint64_t hv = 0ull;
  if (tid < a.parts) {
    hv = comp_of(__ldcg(rc + (int64_t)tid * kLmCands));
    heads[tid] = hv;
  }
  float2 st = make_float2(-3.40282347e38f, 0.f);
  bool bad_part = false;
  constexpr int kStatBatch = 8;
  for (int base = 0; base < a.stat_n; base += kStatBatch * kThreads) {
    float2 e[kStatBatch];
#pragma unroll
    for (int u = 0; u < kStatBatch; u++) {
      const int i = base + u * kThreads + tid;
      e[u] = i < a.stat_n ? __ldcg(a.stats + (int64_t)i * a.stats_ld + row)
                          : make_float2(-3.40282347e38f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < kStatBatch; u++) {
      bad_part = bad_part || e[u].y != e[u].y || !(e[u].x <= 3.40282347e38f);
      if (e[u].y > 0.f) {
        const float mm = fmaxf(st.x, e[u].x);
        st.y = st.y * __expf(st.x - mm) + e[u].y * __expf(e[u].x - mm);
        st.x = mm;
      }
    }
  }
  float bm = st.x;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, o));
  if (lane == 0) sh->red_f[warp] = bm;
  if (tid == 0) {
    sh->count = 0;
    sh->tau = 0ull;
  }
  __syncthreads();
  // A lower bound on the row's k-th best: the k-th best of the parts' heads (k parts hold a
  // candidate at or above it), found by counting; nothing below it can be in the top k.
  if (hv != 0ull && a.parts >= k && k > 0) {
    int above = 0;
    for (int q = 0; q < a.parts; q++) above += heads[q] > hv ? 1 : 0;
    if (above == k - 1) sh->tau = hv;
  }
  float M = lane < kWarps ? sh->red_f[lane] : -3.40282347e38f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
  float contrib = st.y > 0.f ? st.y * __expf(st.x - M) : 0.f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) contrib += __shfl_xor_sync(0xffffffffu, contrib, o);
  const bool wbad = __any_sync(0xffffffffu, bad_part);
  if (lane == 0) {
    sh->red_f2[warp] = contrib;
    sh->red_u[warp] = wbad ? 1u : 0u;
  }
  __syncthreads();
  // The candidates at or above the bound as composites (order-preserving key, inverted
  // id); a warp appends its batch with one shared-memory atomic.
  const uint64_t tau = sh->tau;
  for (int base = 0; base < nent; base += kBatch * kThreads) {
    if (base > 0) load_batch(base);
#pragma unroll
    for (int u = 0; u < kBatch; u++) {
      const uint64_t c = comp_of(w[u]);
      const bool valid = c != 0ull && c >= tau;
      const uint32_t ball = __ballot_sync(0xffffffffu, valid);
      if (ball == 0u) continue;
      uint32_t first = 0;
      if (lane == 0) first = atomicAdd(&sh->count, (uint32_t)__popc(ball));
      first = __shfl_sync(0xffffffffu, first, 0);
      const uint32_t slot = first + (uint32_t)__popc(ball & ((1u << lane) - 1u));
      if (valid && slot < (uint32_t)cap) cand[slot] = c;
    }
  }
  __syncthreads();
  float S = lane < kWarps ? sh->red_f2[lane] : 0.f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) S += __shfl_xor_sync(0xffffffffu, S, o);
  const bool bad = __any_sync(0xffffffffu, lane < kWarps && sh->red_u[lane] != 0u) ||
                   !(S <= 3.40282347e38f) || !(M <= 3.40282347e38f);
  const int n = min((int)sh->count, cap);
  const bool timed_out = a.error && *a.error == a.epoch;
  int kk = 0;
  if (!timed_out && !bad && k > 0) kk = top_sorted(cand, n, k, cap, hist, sh);
  else __syncthreads();
  if (a.keep < kLmCands && a.row_flag) {
    // The fast pass: a part whose last kept candidate lies above the k-th best may have
    // dropped one of the top k; such a row goes to the exact pass.
    const uint64_t kth = (kk == k && k > 0) ? cand[k - 1] : 0ull;
    bool unsettled = false;
    if (tid < a.parts && k > 0 && !timed_out && !bad) {
      const unsigned long long w = rc[(int64_t)tid * kLmCands + a.keep - 1];
      if ((uint32_t)w != 0xffffffffu &&
          composite(key_of(__uint_as_float((uint32_t)(w >> 32))), (uint32_t)w) > kth)
        unsettled = true;
    }
    if (__syncthreads_or(unsettled ? 1 : 0)) {
      if (tid == 0) {
        a.row_flag[row] = a.epoch;
        *a.any_flag = a.epoch;
      }
      return;  // the exact pass writes this row
    }
  }
  const uint32_t status = timed_out ? (uint32_t)TABBY_ETIMEOUT
                          : bad     ? (uint32_t)TABBY_EINPUT
                          : pflags  ? (uint32_t)TABBY_EINVAL
                                    : (uint32_t)TABBY_OK;
  if (warp != 0) return;
  const uint64_t c0 = cand[2 * lane], c1 = cand[2 * lane + 1];
  const int32_t id0 = (int32_t)~(uint32_t)c0, id1 = (int32_t)~(uint32_t)c1;
  float x0 = float_of_key((uint32_t)(c0 >> 32)), x1 = float_of_key((uint32_t)(c1 >> 32));
  // A zero logit keeps its sign: look its raw bits up among the partials (rare).
  for (int e = 0; e < 2; e++) {
    const int i = 2 * lane + e;
    const uint64_t c = e ? c1 : c0;
    if (i < kk && (uint32_t)(c >> 32) == 0x80000000u) {
      const uint32_t want = ~(uint32_t)c;
      for (int i2 = 0; i2 < a.parts * keep; i2++) {  // the entries the parts wrote
        const unsigned long long w = rc[(i2 / keep) * kLmCands + i2 % keep];
        if ((uint32_t)w == want) {
          if (e) x1 = __uint_as_float((uint32_t)(w >> 32));
          else x0 = __uint_as_float((uint32_t)(w >> 32));
          break;
        }
      }
    }
  }
  const float max_logit = kk > 0 ? __shfl_sync(0xffffffffu, x0, 0) : M;
  if (a.topk_ids) {
    if (2 * lane < kk) a.topk_ids[(int64_t)row * a.topk_ld + 2 * lane] = id0;
    if (2 * lane + 1 < kk) a.topk_ids[(int64_t)row * a.topk_ld + 2 * lane + 1] = id1;
  }
  if (a.topk_values) {
    if (2 * lane < kk) a.topk_values[(int64_t)row * a.topk_ld + 2 * lane] = x0;
    if (2 * lane + 1 < kk) a.topk_values[(int64_t)row * a.topk_ld + 2 * lane + 1] = x1;
  }
  if (a.rng_state) {  // drawn only where sampleFromTopK draws (sampler.ts:153,159-167,194)
    double un = 0.0;
    if (lane == 0 && status == TABBY_OK && kk > 0 && prm.temperature > 0)
      un = rng_next(&a.rng_state[row]);
    uni = __shfl_sync(0xffffffffu, un, 0);
  }
  double *scratch = reinterpret_cast<double *>(hist);
  finalize_warp(id0, id1, x0, x1, kk, max_logit, S, prm, uni, scratch, &a.out[row], status);
}

cudaError_t launch_lmhead_merge(const LmheadMergeLaunch &l, cudaStream_t stream) {
  if (l.rows == 0) return cudaSuccess;
  if (l.parts < 1 || l.parts > kThreads) return cudaErrorInvalidValue;
  const size_t smem = (size_t)lm_merge_cap(l.parts, l.keep) * 8 + (size_t)kBins * 4;
  // The attribute is raised per device to the largest size launched so far.
  static std::mutex mu;
  static size_t set_to[64];
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  {
    std::lock_guard<std::mutex> g(mu);
    if (set_to[dev] < smem) {
      err = cudaFuncSetAttribute(lmhead_merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem);
      if (err != cudaSuccess) return err;
      set_to[dev] = smem;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)l.rows);
  cfg.blockDim = dim3((unsigned)kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, lmhead_merge_kernel, l);
}

int host_sample_from_topk(const int32_t *ids, const float *logits, int32_t n, float max_logit,
                          float sum_exp, double temperature, double top_p, double u,
                          tabby_sample_outcome *out) {
  if (n <= 0) return TABBY_EEMPTY;
  double *exact = new double[n];
  double *scaled = new double[n];
  for (int32_t i = 0; i < n; i++) exact[i] = exact_prob(logits[i], max_logit, sum_exp);
  const Decision d = decide_sequential(logits, n, max_logit, sum_exp, temperature, top_p, u, scaled);
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


#ifdef TABBY_CHECKS
extern "C" __attribute__((visibility("default"))) int tabby_debug_checks(unsigned long long *host) {
  return (int)cudaMemcpyFromSymbol(host, tabby::g_check, sizeof(unsigned long long) * 4);
}
#endif
