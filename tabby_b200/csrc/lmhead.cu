// Fused LM head + sampling on sm_100a: logits = hidden x weight^T computed with tcgen05
// tensor-core MMAs and consumed in the epilogue, so they never reach HBM.
//
// Replaces, for the decode step, the reference's lm_head dispatch
// (xOAviOx/tabby src/engine/forward.ts:418-428: encodeMatmul(... 'lm_head') with
// src/shaders/matmul_f16.wgsl / matvec_q4.wgsl into this.logits) followed by the sampling
// dispatches (forward.ts:520-601) and sampleFromTopK (src/engine/sampler.ts:147-212).
//
//   lmhead_kernel   one CTA a SM, 320 threads. Vocabulary tiles of 128 rows (the last one
//                   narrower, a multiple of 16) are taken from a global counter, so SMs
//                   that stream faster take more of them.
//                   warp 0 (one lane)  TMA producer: cp.async.bulk.tensor 2-D loads of the
//                                      weight stages (128 rows x 64 bf16, 128-byte swizzle,
//                                      from HBM) and of the hidden states (the batch's rows
//                                      rounded up to 8; resident in shared memory when all
//                                      K blocks fit, else a ring), mbarrier transaction
//                                      counts; every CTA loads only its own tiles.
//                   warp 1 (one lane)  tcgen05.mma.cta_group::1.kind::f16, M = 128 token rows
//                                      (rows past the batch are never read back), N = the
//                                      tile's rows, K = 16 a step, fp32 accumulators in TMEM,
//                                      double-buffered (2 x 128 columns); tcgen05.commit
//                                      frees a stage and hands a finished tile over.
//                   warps 2-9          epilogue, one thread a (token row, half of the tile's
//                                      columns): tcgen05.ld 32x32b, online max and
//                                      sum(exp(x - max)) with tree reductions, and the best
//                                      16 logits in registers (a parallel insertion); at the
//                                      end the two halves merge, and the CTA's (max,
//                                      sum-exp) and best 16 go to a partials buffer
//                                      (optionally the logits themselves, for tests).
//   lmhead_merge_kernel (sampler_kernels.cu) finishes every row: merged statistics, the
//                   global top-k of the candidates, sampleFromTopK in float64, and flags
//                   rows where a CTA's 16th best lies above the row's k-th best. For those
//                   (rare) rows the exact variant (the best 64 a CTA, in a shared-memory
//                   table) and its merge run; both launches return at once otherwise.
// Every mbarrier wait is bounded; a wait that runs out sets an error word and the rows
// report TABBY_ETIMEOUT.
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <mutex>

#include "sampler_internal.h"
#include "tabby_sample.h"
#include "warp_sort.cuh"

namespace tabby {
namespace {

constexpr int kLmM = 128;          // token rows of a tile (the MMA's M)
constexpr int kLmN = 256;          // vocabulary rows of a full tile (the MMA's N, its largest)
constexpr int kLmSmallUnits = 4;   // the schedule's tail: tiles of 4 units (64 rows)
constexpr int kLmK = 64;           // hidden elements a stage (128 bytes of bf16: one swizzle row)
constexpr int kLmUnit = 16;        // CTAs own vocabulary ranges in units of 16 rows (the MMA's
                                   // smallest N), so the last tile of a range may be narrower
constexpr int kTileBytes = kLmM * kLmK * 2;   // 16 KB: a hidden-state tile
constexpr int kWTileBytes = kLmN * kLmK * 2;  // 32 KB: a weight stage
constexpr int kLmThreads = 320;    // TMA producer, MMA issuer, 8 epilogue warps
constexpr int kEpiThreads = 256;   // two epilogue warps a TMEM lane quarter
constexpr int kTmemCols = 2 * kLmN;
constexpr unsigned long long kWaitNs = 500000000ull;  // a bounded wait gives up after 0.5 s
// Candidate slots a row: its best 64 so far, sorted (slots 0-63), then up to 63 pending
// composites above the 64th (slots 64-127), merged in by the warp once 32 are pending.
constexpr int kLmBuf = 128;
// The two variants of the kernel: the fast pass keeps a row's best kFastKeep logits of a
// CTA's range in registers; the exact pass (run only for rows the fast pass could not
// settle) keeps the best kLmCands in a shared-memory table.
constexpr int kFastKeep = 16;
// The hidden-state ring holds kAStages full (128-row) boxes; smaller batches fit more, up to
// kAMaxStages boxes of 8 rows, and when every K block fits the states stay resident.
constexpr int kAMaxStages = 64;
template <int KL> struct LmVariant;
// The weight tiles (from HBM) get a deeper ring than the hidden-state tiles (from L2).
template <> struct LmVariant<kFastKeep> {
  static constexpr int kWStages = 4;
  static constexpr int kAStages = 4;
  static constexpr size_t kTable = (size_t)32 * kEpiThreads * 4;  // staged logits [32][256]
};
template <> struct LmVariant<kLmCands> {
  static constexpr int kWStages = 2;
  static constexpr int kAStages = 2;
  static constexpr size_t kTable = (size_t)kLmBuf * kLmM * 8;  // [kLmBuf][kLmM]
};
// Dynamic shared memory: the stages, the candidate table, barriers.
template <int KL>
constexpr size_t lm_smem() {
  return 1024 + (size_t)LmVariant<KL>::kWStages * kWTileBytes +
         (size_t)LmVariant<KL>::kAStages * kTileBytes + LmVariant<KL>::kTable + 2048;
}

struct LmArgs {
  int32_t rows, vocab, hidden;
  int32_t units;                 // vocabulary rows in units of kLmUnit
  int32_t ntiles;                // tiles: big_tiles of kLmN rows, then tiles of 64 rows
  int32_t big_tiles;
  uint32_t *tile_ctr;            // [0] next tile, [1] CTAs done: zero between launches
  uint32_t a_bytes;              // bytes of a hidden-state box: round_up(rows, 8) x 128
  float2 *stats;                 // [ntiles][2][stats_ld]: (max, sum-exp) a tile and half
  int32_t stats_ld;
  unsigned long long *cands;     // [rows][gridDim.x][kLmCands]
  float *logits_out;             // tests only: [rows][vocab] fp32, or NULL
  uint32_t *error;               // set to `epoch` when a bounded wait runs out
  const uint32_t *gate;          // non-NULL: run only when *gate == epoch (the exact pass)
  uint32_t epoch;                // the call's tag: flags from earlier calls never match it
};

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mb_init(uint64_t *b, uint32_t n) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(b)), "r"(n) : "memory");
}
__device__ __forceinline__ void mb_arrive_expect(uint64_t *b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(b)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mb_arrive(uint64_t *b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(b)) : "memory");
}
__device__ __forceinline__ unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ bool mb_try(uint64_t *b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(b)), "r"(parity)
      : "memory");
  return ok != 0u;
}
// The clock is read only once a first attempt has failed (reading it costs tens of ns).
__device__ __forceinline__ bool mb_wait(uint64_t *b, uint32_t parity) {
  if (mb_try(b, parity)) return true;
  const unsigned long long t0 = now_ns();
  for (uint32_t i = 0;; i++) {
    if ((i & 1023u) == 1023u && now_ns() - t0 > kWaitNs) return false;
    if (mb_try(b, parity)) return true;
  }
}
// 2-D TMA load of one box into this CTA's shared memory (coordinates: inner, outer).
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y,
                                            uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, "
      "{%3, %4}], [%2];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(x), "r"(y)
      : "memory");
}
// The same with an L2 cache policy: the weights are read once a call, so their lines go
// first when L2 needs room and the small buffers and code the other kernels use stay.
__device__ __forceinline__ uint64_t l2_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ void tma_load_2d_hint(void *dst, const CUtensorMap *map, int x, int y,
                                                 uint64_t *bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(x), "r"(y), "l"(pol)
      : "memory");
}
// Shared-memory matrix descriptor of a K-major tile written by TMA with 128-byte swizzle:
// rows of 128 bytes, 8-row groups 1024 bytes apart (stride byte offset), descriptor
// version 1 (sm_100), layout type 2 (SWIZZLE_128B). The tile base is 1024-byte aligned.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFFu);         // start address
  d |= (uint64_t)1u << 16;                         // leading byte offset (unused here)
  d |= (uint64_t)(1024u >> 4) << 32;               // stride byte offset
  d |= (uint64_t)1u << 46;                         // version
  d |= (uint64_t)2u << 61;                         // SWIZZLE_128B
  return d;
}
// Instruction descriptor of kind::f16: bf16 A and B, fp32 accumulate, both K-major.
// N (a multiple of 16, at most kLmN) is the tile's width.
__device__ __forceinline__ uint32_t idesc_n(int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(kLmM >> 4) << 24);
}

__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                         uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_addr(bar))
      : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
      "%28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ float ex2_fast(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Order-preserving key with -0 folded onto +0 (ties then go to the lower index), as the
// row pass orders candidates (sampler.ts:28: b.value - a.value || a.id - b.id).
__device__ __forceinline__ uint32_t lm_key(float x) {
  uint32_t b = __float_as_uint(x);
  b = (b == 0x80000000u) ? 0u : b;
  return b ^ ((uint32_t)((int32_t)b >> 31) | 0x80000000u);
}

// Index of (slot, row) in the candidate table. Rows are XOR-swizzled by the slot pair so
// that both access patterns are free of bank conflicts: a warp's threads each on their own
// row at one slot, and one warp walking one row's slots (two a lane).
__device__ __forceinline__ int cidx(int slot, int row) {
  return slot * kLmM + (row ^ ((slot >> 1) & 31));
}

// Merges the pending composites of row `rr` (one of this warp's 32 rows; `np` of them)
// into its sorted best 64 (warp-uniform call): the pending ones are sorted by a bitonic
// network, the two sorted lists merged keeping the 64 largest. Returns the 64th largest
// (0 while fewer than 64 are kept).
__device__ __forceinline__ uint64_t merge_pending(unsigned long long *tab, int rr, int np) {
  const int lane = threadIdx.x & 31;
  uint64_t w0 = 2 * lane < np ? tab[cidx(kLmCands + 2 * lane, rr)] : 0ull;
  uint64_t w1 = 2 * lane + 1 < np ? tab[cidx(kLmCands + 2 * lane + 1, rr)] : 0ull;
  warp_sort64_desc(w0, w1);
  uint64_t a0 = tab[cidx(2 * lane, rr)], a1 = tab[cidx(2 * lane + 1, rr)];
  warp_merge64_desc(a0, a1, w0, w1);
  tab[cidx(2 * lane, rr)] = a0;
  tab[cidx(2 * lane + 1, rr)] = a1;
  return __shfl_sync(0xffffffffu, a1, 31);
}

template <int KL>
__global__ void __launch_bounds__(kLmThreads, 1)
    lmhead_kernel(const __grid_constant__ CUtensorMap map_h, const __grid_constant__ CUtensorMap map_w,
                  const __grid_constant__ CUtensorMap map_w16, const __grid_constant__ LmArgs a) {
  constexpr int kW = LmVariant<KL>::kWStages, kA = LmVariant<KL>::kAStages;
  // Launched with programmatic stream serialization (its launch overlaps the previous
  // kernel's tail): wait for the previous kernel in the stream to complete.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (a.gate && *a.gate != a.epoch) return;  // the exact pass, not needed this call
  extern __shared__ unsigned char smem_dyn[];
  unsigned char *base = reinterpret_cast<unsigned char *>(
      (reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~(uintptr_t)1023);
  constexpr int kRing = kW * kWTileBytes + kA * kTileBytes;  // both rings' bytes
  constexpr int kWMax = kRing / kWTileBytes;
  unsigned long long *cand =
      reinterpret_cast<unsigned long long *>(base + kRing);
  uint64_t *bars = reinterpret_cast<uint64_t *>(base + kRing + LmVariant<KL>::kTable);
  uint64_t *wfull = bars, *wempty = bars + kWMax;
  uint64_t *afull = bars + 2 * kWMax, *aempty = afull + kAMaxStages;
  uint64_t *tfull = aempty + kAMaxStages, *tempty = tfull + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(tempty + 2);
  volatile uint32_t *err = tmem_slot + 1;
  // Which tile a weight stage belongs to (-1: no more tiles), and which tile each
  // accumulator holds, handed from the producer to the MMA issuer to the epilogue.
  volatile int32_t *stage_tile = reinterpret_cast<volatile int32_t *>(tmem_slot + 2);
  volatile int32_t *acc_tile = stage_tile + kWMax;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // Tiles are taken from a global counter, so SMs that stream faster take more of them;
  // a CTA's tiles come in increasing order. The schedule: big_tiles tiles of kLmN rows,
  // then tiles of 64 rows for the last two rounds (so CTAs end within a small tile of one
  // another); the vocabulary's last tile may be narrower (a multiple of 16 rows).
  auto tile_v0 = [&](int g) {
    return g < a.big_tiles ? g * kLmN
                           : (a.big_tiles * (kLmN / kLmUnit) + (g - a.big_tiles) * kLmSmallUnits) *
                                 kLmUnit;
  };
  auto tile_width = [&](int g) {
    return min(g < a.big_tiles ? kLmN : kLmSmallUnits * kLmUnit, a.units * kLmUnit - tile_v0(g));
  };
  const int kb_n = a.hidden / kLmK;
  // The rings share kRing bytes. When every K block of the batch's hidden states fits
  // beside kW weight stages, the states stay resident (loaded once, never released) and
  // the weight ring takes the rest; otherwise the hidden-state ring holds as many boxes as
  // kA full ones would, refilled once the MMAs of a stage complete.
  const int a_all = kb_n * (int)a.a_bytes;
  const bool a_res = a_all <= kRing - kW * kWTileBytes && kb_n <= kAMaxStages;
  const int dA = a_res ? kb_n : min(kAMaxStages, (kA * kTileBytes) / (int)a.a_bytes);
  const int dW = a_res ? (kRing - a_all) / kWTileBytes : kW;
  unsigned char *wring = base;                      // [dW] weight tiles
  unsigned char *aring = base + dW * kWTileBytes;   // [dA] hidden-state boxes

  if (tid == 0) {
    for (int s = 0; s < kWMax; s++) {
      mb_init(&wfull[s], 1);
      mb_init(&wempty[s], 1);
    }
    for (int s = 0; s < kAMaxStages; s++) {
      mb_init(&afull[s], 1);
      mb_init(&aempty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      mb_init(&tfull[b], 2);  // the MMAs' completion and the issuer's tile hand-over
      mb_init(&tempty[b], kEpiThreads / 32);  // one arrival an epilogue warp
    }
    *err = 0u;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {  // TMEM: two accumulators of 128 columns
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_addr(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---- TMA producer (one lane): takes a tile, then streams its weight stages and, per
    // stage, the hidden-state box (resident states: only with the first tile) ----
    if (lane == 0) {
      int sw = 0, sa = 0, nw = 0, na = 0;
      uint32_t pw = 0, pa = 0;  // round parities; a fresh barrier passes a wait on parity 1
      bool a_loaded = false, ok = true, ended = false;
      const uint64_t pol = l2_evict_first();
      // The next tile is asked for one tile ahead, so the counter's round trip overlaps
      // the current tile's loads.
      int g_next = (int)atomicAdd(a.tile_ctr, 1u);
      while (ok) {
        int g = g_next;
        if (g >= a.ntiles || *err) g = -1;
        else g_next = (int)atomicAdd(a.tile_ctr, 1u);
        if (!mb_wait(&wempty[sw], pw ^ 1u)) break;
        if (g < 0) {  // the end: a stage with no data carries the mark
          stage_tile[sw] = -1;
          mb_arrive(&wfull[sw]);
          nw++;
          if (++sw == dW) {
            sw = 0;
            pw ^= 1u;
          }
          ended = true;
          break;
        }
        const int v0 = tile_v0(g), n = tile_width(g);
        for (int kb = 0; kb < kb_n; kb++) {
          if (kb > 0 && !mb_wait(&wempty[sw], pw ^ 1u)) {
            ok = false;
            break;
          }
          if (!a_res || !a_loaded) {  // only the batch's rows (rounded up to 8)
            if (!mb_wait(&aempty[sa], pa ^ 1u)) {
              ok = false;
              break;
            }
            mb_arrive_expect(&afull[sa], a.a_bytes);
            tma_load_2d(aring + sa * (int)a.a_bytes, &map_h, kb * kLmK, 0, &afull[sa]);
            na++;
            if (++sa == dA) {
              sa = 0;
              pa ^= 1u;
            }
          }
          stage_tile[sw] = g;
          unsigned char *dst = wring + sw * kWTileBytes;
          if (n == kLmN) {
            mb_arrive_expect(&wfull[sw], (uint32_t)kWTileBytes);
            tma_load_2d_hint(dst, &map_w, kb * kLmK, v0, &wfull[sw], pol);
          } else {  // a narrow last tile: boxes of 16 rows, 2 KB apart (same swizzle phase)
            mb_arrive_expect(&wfull[sw], (uint32_t)(n * kLmK * 2));
            for (int j = 0; j < n; j += kLmUnit)
              tma_load_2d_hint(dst + j * kLmK * 2, &map_w16, kb * kLmK, v0 + j, &wfull[sw], pol);
          }
          nw++;
          if (++sw == dW) {
            sw = 0;
            pw ^= 1u;
          }
        }
        a_loaded = true;
      }
      if (!ended) *err = 1u;  // a wait ran out
      // Every issued load has landed before the CTA may exit (bounded): the last stages
      // of each ring, newest first.
      for (int j = 0; j < min(nw, dW); j++) {
        if (sw == 0) {
          sw = dW;
          pw ^= 1u;
        }
        sw--;
        mb_wait(&wfull[sw], pw);
      }
      for (int j = 0; j < min(na, dA); j++) {
        if (sa == 0) {
          sa = dA;
          pa ^= 1u;
        }
        sa--;
        mb_wait(&afull[sa], pa);
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer (one lane) ----
    if (lane == 0) {
      int sw = 0, sa = 0;
      uint32_t pw = 0, pa = 0;  // round parities of the two rings
      for (int t = 0; !*err; t++) {
        const int b = t & 1;
        if (t >= 2 && !mb_wait(&tempty[b], ((t >> 1) - 1) & 1)) {
          *err = 1u;
          break;
        }
        if (!mb_wait(&wfull[sw], pw)) {
          *err = 1u;
          break;
        }
        const int g = stage_tile[sw];
        acc_tile[b] = g;
        if (g < 0) {  // no more tiles: both arrivals, so the epilogue sees the mark
          mb_arrive(&tfull[b]);
          mb_arrive(&tfull[b]);
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(b * kLmN);
        const uint32_t idesc = idesc_n(tile_width(g));
        for (int kb = 0; kb < kb_n; kb++) {
          if ((kb > 0 && !mb_wait(&wfull[sw], pw)) || !mb_wait(&afull[sa], pa)) {
            *err = 1u;
            break;
          }
          tc_fence_after();
          const uint32_t wa = smem_addr(wring + sw * kWTileBytes);
          const uint32_t ha = smem_addr(aring + sa * (int)a.a_bytes);
#pragma unroll
          for (int kk = 0; kk < kLmK / 16; kk++)  // 16 bf16 = 32 bytes a step along K
            mma_bf16(d, smem_desc(ha + 32 * kk), smem_desc(wa + 32 * kk), idesc,
                   (kb | kk) != 0 ? 1u : 0u);
          mma_commit(&wempty[sw]);  // the stages are free once these MMAs have read them
          if (!a_res) mma_commit(&aempty[sa]);
          if (++sw == dW) {
            sw = 0;
            pw ^= 1u;
          }
          if (++sa == dA) {  // resident states: every tile reads the same stages, round 0
            sa = 0;
            if (!a_res) pa ^= 1u;
          }
        }
        if (*err) break;
        mb_arrive(&tfull[b]);   // the tile number in acc_tile[b] is published
        mma_commit(&tfull[b]);  // the tile's accumulator is complete
      }
    }
  } else {
    // ---- epilogue: thread = token row (TMEM lane 32 * (warp % 4) + lane); the two warps
    // of a lane quarter take the two halves of every tile's columns, each its own part ----
    const int q = warp & 3;
    const int row = 32 * q + lane;
    const int et = tid - 64;        // epilogue thread
    const int hf = et >> 7;         // which half of the columns
    const int parts = gridDim.x;  // one part a CTA: the two halves merge at the end
    const int pi = blockIdx.x;
    const bool live = row < a.rows;
    float m = -3.40282347e38f, s = 0.f;
    constexpr float kLog2e = 1.44269504088896341f;
    if constexpr (KL == kFastKeep) {
      // The row's best kFastKeep composites of this CTA's range, sorted in registers;
      // a logit above the last one is inserted by one branch-free pass.
      float *stage_f = reinterpret_cast<float *>(cand);  // the variant's table: [32][256]
      // Values and vocabulary ids, best first. The scan visits ids in increasing order, so
      // a value equal to a kept one ranks after it: the order is (value desc, id asc), the
      // candidates' order, with value comparisons alone.
      float bv[kFastKeep];
      uint32_t bi[kFastKeep];
#pragma unroll
      for (int e = 0; e < kFastKeep; e++) {
        bv[e] = -INFINITY;
        bi[e] = 0xffffffffu;
      }
      float thr_val = -INFINITY;  // bv[kFastKeep - 1]: a logit must exceed it to enter
      for (int t = 0;; t++) {
        const int b = t & 1;
        if (!mb_wait(&tfull[b], (t >> 1) & 1)) {
          *err = 1u;
          break;
        }
        tc_fence_after();
        const int g = acc_tile[b];
        if (g < 0) break;  // no more tiles
        const int v0 = tile_v0(g), vend = min(a.vocab, v0 + tile_width(g));
        // Statistics a tile and half, so that the merge combines them in a fixed order
        // whichever CTA took the tile.
        m = -3.40282347e38f;
        s = 0.f;
        // The halves take alternate 32-column chunks (so narrow tiles split evenly too);
        // each thread still visits its vocabulary ids in increasing order.
#pragma unroll 1
        for (int c = hf; c < kLmN / 32; c += 2) {
          const int vb = v0 + 32 * c;
          if (vb >= vend) break;  // past a narrow tile's columns (warp-uniform)
          uint32_t r[32];
          tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(b * kLmN + 32 * c), r);
          const int nv = live ? min(32, vend - vb) : 0;
          if (nv <= 0) continue;
          if (nv < 32) {  // columns past the vocabulary count as -inf: no max, exp 0, no hit
#pragma unroll
            for (int j = 0; j < 32; j++)
              if (j >= nv) r[j] = 0xff800000u;
          }
          // Reductions as trees (independent operations, not one dependent chain).
          float tm[16];
#pragma unroll
          for (int j = 0; j < 16; j++) tm[j] = fmaxf(__uint_as_float(r[j]), __uint_as_float(r[j + 16]));
#pragma unroll
          for (int w = 8; w > 0; w >>= 1)
#pragma unroll
            for (int j = 0; j < w; j++) tm[j] = fmaxf(tm[j], tm[j + w]);
          const float cm = tm[0];
          if (cm > m) {
            s *= ex2_fast((m - cm) * kLog2e);
            m = cm;
          }
          const float mL = m * kLog2e;
          float te[16];
#pragma unroll
          for (int j = 0; j < 16; j++)
            te[j] = ex2_fast(fmaf(__uint_as_float(r[j]), kLog2e, -mL)) +
                    ex2_fast(fmaf(__uint_as_float(r[j + 16]), kLog2e, -mL));
#pragma unroll
          for (int w = 8; w > 0; w >>= 1)
#pragma unroll
            for (int j = 0; j < w; j++) te[j] += te[j + w];
          s += te[0];
          if (a.logits_out) {
#pragma unroll
            for (int j = 0; j < 32; j++)
              if (j < nv) a.logits_out[(int64_t)row * a.vocab + vb + j] = __uint_as_float(r[j]);
          }
          if (cm > thr_val) {
            // The logits above the threshold: a mask, then one compact loop over
            // them (staged in shared memory) for the insertions.
            uint32_t hq[4] = {0u, 0u, 0u, 0u};
#pragma unroll
            for (int j = 0; j < 32; j++)
              hq[j & 3] |= (__uint_as_float(r[j]) > thr_val) ? (1u << j) : 0u;
            uint32_t hits = (hq[0] | hq[1]) | (hq[2] | hq[3]);
#pragma unroll
            for (int j = 0; j < 32; j++)
              if ((hits >> j) & 1u) stage_f[j * kEpiThreads + et] = __uint_as_float(r[j]);
            while (hits) {
              const int j = __ffs(hits) - 1;
              hits &= hits - 1;
              const float x = stage_f[j * kEpiThreads + et];
              if (x > thr_val) {
                // Insertion with every slot computed from the old list at once (no chain
                // of dependent compare-and-swaps): slot e keeps its value if that is >= x,
                // takes x if slot e-1 keeps its own, else shifts down slot e-1's.
                const uint32_t id = (uint32_t)(vb + j);
                bool g[kFastKeep];
#pragma unroll
                for (int e = 0; e < kFastKeep; e++) g[e] = bv[e] >= x;
#pragma unroll
                for (int e = kFastKeep - 1; e > 0; e--) {
                  bv[e] = g[e] ? bv[e] : (g[e - 1] ? x : bv[e - 1]);
                  bi[e] = g[e] ? bi[e] : (g[e - 1] ? id : bi[e - 1]);
                }
                bv[0] = g[0] ? bv[0] : x;
                bi[0] = g[0] ? bi[0] : id;
                thr_val = bv[kFastKeep - 1];
              }
            }
          }
        }
        if (live) a.stats[((int64_t)g * 2 + hf) * a.stats_ld + row] = make_float2(m, s);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mb_arrive(&tempty[b]);  // the accumulator may be overwritten
      }
      // The second half's threads hand their lists over through shared
      // memory (the staging area, free now: a barrier of the 256 epilogue threads first);
      // the first half's merge them, the lists by (value desc, id asc).
      float *xv = stage_f;                                           // [kFastKeep][kLmM]
      uint32_t *xi = reinterpret_cast<uint32_t *>(xv + kFastKeep * kLmM);
      asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory");
      if (hf == 1) {
#pragma unroll
        for (int e = 0; e < kFastKeep; e++) {
          xv[e * kLmM + row] = bv[e];
          xi[e * kLmM + row] = bi[e];
        }
      }
      asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory");
      if (hf == 0 && live) {
        // Two-pointer merge: this thread's list pops from the front of its registers (a
        // shift), the other half's list is read from shared memory.
        float ov[kFastKeep];
        uint32_t oi[kFastKeep];
        int jb = 0;
        float x = xv[row];
        uint32_t id = xi[row];
#pragma unroll
        for (int e = 0; e < kFastKeep; e++) {
          const bool take_a = bv[0] > x || (bv[0] == x && bi[0] < id);
          ov[e] = take_a ? bv[0] : x;
          oi[e] = take_a ? bi[0] : id;
          if (take_a) {
#pragma unroll
            for (int f = 0; f < kFastKeep - 1; f++) {
              bv[f] = bv[f + 1];
              bi[f] = bi[f + 1];
            }
            bv[kFastKeep - 1] = -INFINITY;
            bi[kFastKeep - 1] = 0xffffffffu;
          } else {
            jb++;
            x = jb < kFastKeep ? xv[jb * kLmM + row] : -INFINITY;
            id = jb < kFastKeep ? xi[jb * kLmM + row] : 0xffffffffu;
          }
        }
#pragma unroll
        for (int e = 0; e < kFastKeep; e++) {
          bv[e] = ov[e];
          bi[e] = oi[e];
        }
        unsigned long long *dst = a.cands + ((int64_t)row * parts + pi) * kLmCands;
#pragma unroll
        for (int e = 0; e < kFastKeep; e++)  // the merge reads the first kFastKeep entries
          dst[e] = bi[e] != 0xffffffffu
                       ? (((uint64_t)__float_as_uint(bv[e]) << 32) | (uint64_t)bi[e])
                       : 0xffffffffull;
      }
    } else {
    int pend = 0;                     // this row's pending composites
    uint64_t thr = 0ull;              // candidates must exceed the row's 64th best
    float thr_val = -3.40282347e38f;  // its value: a cheap first filter (>=)
    // The exact pass uses the first warp of each lane quarter for all columns; the second
    // only releases the accumulators and reports an empty part.
    if (hf == 0)
      for (int e = 0; e < kLmCands; e++) cand[cidx(e, row)] = 0ull;  // nothing kept yet
    __syncwarp();
    // Merges, for every row of this warp with at least `at_least` pending, the pending
    // composites into the row's best 64, and raises its thresholds.
    auto merge_rows = [&](int at_least) {
      uint32_t need = __ballot_sync(0xffffffffu, pend >= at_least && pend > 0);
      while (need) {
        const int rr = __ffs(need) - 1;
        need &= need - 1;
        const int np = __shfl_sync(0xffffffffu, pend, rr);
        const uint64_t t = merge_pending(cand, 32 * q + rr, np);
        if (lane == rr) {
          pend = 0;
          if (t != 0ull) {
            thr = t;
            const uint32_t kk = (uint32_t)(t >> 32);
            thr_val = __uint_as_float(kk ^ ((kk >> 31) ? 0x80000000u : 0xffffffffu));
          }
        }
        __syncwarp();
      }
    };
    for (int t = 0;; t++) {
      const int b = t & 1;
      if (!mb_wait(&tfull[b], (t >> 1) & 1)) {
        *err = 1u;
        break;
      }
      tc_fence_after();
      const int g = acc_tile[b];
      if (g < 0) break;  // no more tiles
      const int v0 = tile_v0(g), vend = min(a.vocab, v0 + tile_width(g));
      m = -3.40282347e38f;  // statistics a tile (the second half's slot stays empty)
      s = 0.f;
#pragma unroll 1
      for (int c = 0; c < (hf == 0 ? (vend - v0 + 31) / 32 : 0); c++) {
        uint32_t r[32];
        tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(b * kLmN + 32 * c), r);
        const int vb = v0 + 32 * c;
        const int nv = live ? min(32, vend - vb) : 0;
        if (nv > 0) {
          float cm = -3.40282347e38f;
#pragma unroll
          for (int j = 0; j < 32; j++)
            if (j < nv) cm = fmaxf(cm, __uint_as_float(r[j]));
          if (cm > m) {
            s *= ex2_fast((m - cm) * kLog2e);
            m = cm;
          }
          const float mL = m * kLog2e;
          float acc = 0.f;
#pragma unroll
          for (int j = 0; j < 32; j++)
            if (j < nv) acc += ex2_fast(fmaf(__uint_as_float(r[j]), kLog2e, -mL));
          s += acc;
          if (a.logits_out) {
#pragma unroll
            for (int j = 0; j < 32; j++)
              if (j < nv) a.logits_out[(int64_t)row * a.vocab + vb + j] = __uint_as_float(r[j]);
          }
          if (cm >= thr_val) {
#pragma unroll
            for (int j = 0; j < 32; j++) {
              const float x = __uint_as_float(r[j]);
              if (j < nv && x >= thr_val) {
                const uint64_t cmp = ((uint64_t)lm_key(x) << 32) | (uint64_t)(~(uint32_t)(vb + j));
                if (cmp > thr) cand[cidx(kLmCands + pend++, row)] = cmp;
              }
            }
          }
        }
        merge_rows(32);  // keeps every row's pending list below 64
      }
      if (live) a.stats[((int64_t)g * 2 + hf) * a.stats_ld + row] = make_float2(m, s);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mb_arrive(&tempty[b]);  // the accumulator may be overwritten
    }
    if (hf == 0) merge_rows(1);  // the last pending composites of every row
    if (live && hf == 0) {
      unsigned long long *dst = a.cands + ((int64_t)row * parts + pi) * kLmCands;
      for (int e = 0; e < kLmCands; e++) {
        // composite: raw value bits from the key (+0 for a -0 logit, the one value the key folds)
        const uint64_t c = cand[cidx(e, row)];
        const uint32_t kk = (uint32_t)(c >> 32);
        const uint32_t raw = kk ^ ((kk >> 31) ? 0x80000000u : 0xffffffffu);
        dst[e] = c != 0ull ? (((uint64_t)raw << 32) | (uint64_t)(~(uint32_t)c)) : 0xffffffffull;
      }
    }
      }
  }
  tc_fence_before();
  __syncthreads();
  if (tid == 0) {
    if (*err) *a.error = a.epoch;
    // The last CTA to finish zeroes the tile counter for the next launch (every CTA has
    // taken its last tile by now).
    if (atomicAdd(a.tile_ctr + 1, 1u) == gridDim.x - 1) {
      a.tile_ctr[0] = 0u;
      a.tile_ctr[1] = 0u;
    }
  }
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols)
                 : "memory");
  }
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link to libcuda).
using EncodeTiled = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                 const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                 const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                 CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encode_fn() {
  static std::once_flag once;
  static EncodeTiled fn = nullptr;
  std::call_once(once, []() {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiled>(p);
  });
  return fn;
}

// K-major bf16 matrix [outer][inner] with boxes of 64 x box_rows (inner x outer), 128-byte
// swizzle, zero fill out of bounds.
bool make_map(CUtensorMap *m, const void *ptr, uint64_t inner, uint64_t outer, uint32_t box_rows) {
  EncodeTiled enc = encode_fn();
  if (!enc) return false;
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {inner * 2};
  const cuuint32_t box[2] = {(cuuint32_t)kLmK, box_rows};
  const cuuint32_t elem[2] = {1u, 1u};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(ptr), dims, strides, box,
             elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

// A launch with programmatic stream serialization: the kernel may start before the previous
// one in the stream completes and orders itself with griddepcontrol.wait.
template <typename... Args>
cudaError_t launch_pdl(void (*kernel)(Args...), int grid, int block, size_t smem,
                       cudaStream_t stream, const Args &...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3((unsigned)block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

int lfail(int status, const char *fmt, ...) {
  char msg[256];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(msg, sizeof(msg), fmt, ap);
  va_end(ap);
  return set_error(status, msg);
}

}  // namespace
}  // namespace tabby

struct tabby_lmhead {
  CUtensorMap map_h;       // over the last hidden-state pointer and batch: boxes of the
                           // batch's rows rounded up to 8 (the rest zero-filled by TMA)
  const void *map_h_ptr;
  int32_t map_h_rows;
  uint32_t epoch;          // the last call's tag (never 0: the flags start zeroed)
  CUtensorMap map_w;       // over the last weight pointer: boxes of 128 rows
  CUtensorMap map_w16;     // the same, boxes of 16 rows (the narrow last tile of a range)
  const void *map_w_ptr;
  int32_t device;
  int32_t max_rows;
  int32_t vocab;
  int32_t hidden;
  int32_t grid;
  int32_t units;
  float2 *stats;
  unsigned long long *cands;
  uint32_t *error;  // [0] = the epoch of a call whose bounded wait ran out, [1] = the
                    // epoch of a call with a row for the exact pass
  uint32_t *flags;  // [max_rows] = the epoch of a call whose exact pass recomputes the row
  uint32_t *tile_ctr;  // the kernels' tile counter (zeroed by the last CTA of each launch)
  int32_t ntiles;
  int32_t big_tiles;
};

extern "C" {

int tabby_lmhead_create(int32_t device, int32_t max_rows, int32_t vocab, int32_t hidden,
                        tabby_lmhead **out) {
  using namespace tabby;
  if (!out) return lfail(TABBY_EINVAL, "out must not be NULL");
  *out = nullptr;
  if (max_rows < 1 || max_rows > kLmM)
    return lfail(TABBY_EINVAL, "max_rows must be in [1, %d], got %d", kLmM, max_rows);
  if (vocab < 1 || vocab > TABBY_MAX_VOCAB_LMHEAD)
    return lfail(TABBY_EINVAL, "vocab must be in [1, %d], got %d", TABBY_MAX_VOCAB_LMHEAD, vocab);
  if (hidden < kLmK || hidden % kLmK != 0 || hidden > 65536)
    return lfail(TABBY_EINVAL, "hidden must be a positive multiple of %d (<= 65536), got %d",
                 kLmK, hidden);
  int cur = 0;
  cudaError_t err = cudaGetDevice(&cur);
  if (err == cudaSuccess && cur != device) err = cudaSetDevice(device);
  if (err != cudaSuccess) return lfail(TABBY_ECUDA, "cudaSetDevice: %s", cudaGetErrorString(err));
  int sms = 0, major = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
  if (major < 10) {
    if (cur != device) cudaSetDevice(cur);
    return lfail(TABBY_ECUDA, "device %d is not sm_100", device);
  }
  tabby_lmhead *h = new tabby_lmhead();
  memset(h, 0, sizeof(*h));
  h->device = device;
  h->max_rows = max_rows;
  h->vocab = vocab;
  h->hidden = hidden;
  h->units = (vocab + kLmUnit - 1) / kLmUnit;
  // Tiles of 64 rows cover the last two rounds (8 units a CTA); big tiles the rest.
  {
    const int grid_guess = std::max(std::min(sms, (h->units + kLmSmallUnits - 1) / kLmSmallUnits), 1);
    const int tail_units = std::min(h->units, 2 * kLmSmallUnits * grid_guess);
    h->big_tiles = (h->units - tail_units) / (kLmN / kLmUnit);
    const int rest = h->units - h->big_tiles * (kLmN / kLmUnit);
    h->ntiles = h->big_tiles + (rest + kLmSmallUnits - 1) / kLmSmallUnits;
  }
  // Every SM, an even share of the 16-row units each (at least a full tile's worth).
  h->grid = std::min(h->ntiles, std::max(sms, 1));
  const size_t nst = (size_t)max_rows * h->grid;  // one candidate part a CTA
  if ((err = cudaMalloc(&h->stats, (size_t)max_rows * h->ntiles * 2 * sizeof(float2))) !=
          cudaSuccess ||
      (err = cudaMalloc(&h->cands, nst * kLmCands * 8)) != cudaSuccess ||
      (err = cudaMalloc(&h->error, 16)) != cudaSuccess ||
      (err = cudaMemset(h->error, 0, 16)) != cudaSuccess ||
      (err = cudaMalloc(&h->flags, (size_t)max_rows * 4)) != cudaSuccess ||
      (err = cudaMalloc(&h->tile_ctr, 8)) != cudaSuccess ||
      (err = cudaMemset(h->tile_ctr, 0, 8)) != cudaSuccess ||
      (err = cudaMemset(h->flags, 0, (size_t)max_rows * 4)) != cudaSuccess ||
      (err = cudaFuncSetAttribute(lmhead_kernel<kFastKeep>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)lm_smem<kFastKeep>())) != cudaSuccess ||
      (err = cudaFuncSetAttribute(lmhead_kernel<kLmCands>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)lm_smem<kLmCands>())) != cudaSuccess) {
    if (h->flags) cudaFree(h->flags);
    if (h->tile_ctr) cudaFree(h->tile_ctr);
    if (h->stats) cudaFree(h->stats);
    if (h->cands) cudaFree(h->cands);
    if (h->error) cudaFree(h->error);
    delete h;
    if (cur != device) cudaSetDevice(cur);
    return lfail(TABBY_ENOMEM, "LM-head set-up failed: %s", cudaGetErrorString(err));
  }
  if (cur != device) cudaSetDevice(cur);
  *out = h;
  return TABBY_OK;
}

int tabby_lmhead_destroy(tabby_lmhead *h) {
  if (!h) return TABBY_OK;
  int cur = 0;
  cudaGetDevice(&cur);
  if (cur != h->device) cudaSetDevice(h->device);
  cudaFree(h->stats);
  cudaFree(h->cands);
  cudaFree(h->error);
  cudaFree(h->flags);
  cudaFree(h->tile_ctr);
  if (cur != h->device) cudaSetDevice(cur);
  delete h;
  return TABBY_OK;
}

int tabby_lmhead_sample_async(tabby_lmhead *h, const void *d_hidden, const void *d_weight,
                              int32_t rows, const tabby_sampling_params *d_params,
                              const double *d_uniforms, tabby_sample_outcome *d_out,
                              int32_t *d_topk_ids, float *d_topk_values, int32_t topk_ld,
                              float *d_logits_out, void *stream) {
  using namespace tabby;
  if (!h) return lfail(TABBY_EINVAL, "lmhead handle is NULL");
  if (rows < 0 || rows > h->max_rows)
    return lfail(TABBY_EINVAL, "rows must be in [0, %d], got %d", h->max_rows, rows);
  if (rows == 0) return TABBY_OK;
  if (!d_hidden || !d_weight || !d_params || !d_uniforms || !d_out)
    return lfail(TABBY_EINVAL, "hidden, weight, params, uniforms and out must not be NULL");
  if ((reinterpret_cast<uintptr_t>(d_hidden) | reinterpret_cast<uintptr_t>(d_weight)) & 15u)
    return lfail(TABBY_EINVAL, "hidden and weight must be 16-byte aligned");
  if ((d_topk_ids || d_topk_values) && topk_ld < kLmCands)
    return lfail(TABBY_EINVAL, "topk_ld (%d) must be >= %d", topk_ld, kLmCands);
  int cur = 0;
  cudaError_t err = cudaGetDevice(&cur);
  if (err == cudaSuccess && cur != h->device) err = cudaSetDevice(h->device);
  if (err != cudaSuccess) return lfail(TABBY_ECUDA, "cudaSetDevice: %s", cudaGetErrorString(err));
  if (d_weight != h->map_w_ptr) {
    if (!make_map(&h->map_w, d_weight, (uint64_t)h->hidden, (uint64_t)h->vocab, (uint32_t)kLmN) ||
        !make_map(&h->map_w16, d_weight, (uint64_t)h->hidden, (uint64_t)h->vocab,
                  (uint32_t)kLmUnit)) {
      h->map_w_ptr = nullptr;
      if (cur != h->device) cudaSetDevice(cur);
      return lfail(TABBY_ECUDA, "cuTensorMapEncodeTiled failed");
    }
    h->map_w_ptr = d_weight;
  }
  const int mb = (rows + 7) / 8;  // hidden-state boxes of 8 * mb rows
  if (d_hidden != h->map_h_ptr || rows != h->map_h_rows) {
    if (!make_map(&h->map_h, d_hidden, (uint64_t)h->hidden, (uint64_t)rows, (uint32_t)(8 * mb))) {
      h->map_h_ptr = nullptr;
      if (cur != h->device) cudaSetDevice(cur);
      return lfail(TABBY_ECUDA, "cuTensorMapEncodeTiled failed");
    }
    h->map_h_ptr = d_hidden;
    h->map_h_rows = rows;
  }
  if (++h->epoch == 0u) h->epoch = 1u;
  const CUtensorMap &mh = h->map_h, &mw = h->map_w, &mw16 = h->map_w16;
  cudaStream_t q = (cudaStream_t)stream;
  LmArgs a;
  a.rows = rows;
  a.vocab = h->vocab;
  a.hidden = h->hidden;
  a.units = h->units;
  a.ntiles = h->ntiles;
  a.big_tiles = h->big_tiles;
  a.tile_ctr = h->tile_ctr;
  a.a_bytes = (uint32_t)(8 * mb * kLmK * 2);
  a.stats = h->stats;
  a.stats_ld = h->max_rows;
  a.cands = h->cands;
  a.logits_out = d_logits_out;
  a.error = h->error;
  a.epoch = h->epoch;
  // The fast pass and its merge; then the exact pass and its merge, which return at once
  // unless the fast merge flagged a row (a part's 16th best above the row's k-th best).
  a.gate = nullptr;
  LmheadMergeLaunch l;
  l.stats = h->stats;
  l.cands = h->cands;
  l.parts = h->grid;
  l.stat_n = 2 * h->ntiles;
  l.stats_ld = h->max_rows;
  l.rows = rows;
  l.vocab = h->vocab;
  l.params = d_params;
  l.uniforms = d_uniforms;
  l.out = d_out;
  l.topk_ids = d_topk_ids;
  l.topk_values = d_topk_values;
  l.topk_ld = topk_ld;
  l.error = h->error;
  l.row_flag = h->flags;
  l.any_flag = h->error + 1;
  l.epoch = h->epoch;
  if (err == cudaSuccess)
    err = launch_pdl(lmhead_kernel<kFastKeep>, h->grid, kLmThreads, lm_smem<kFastKeep>(), q, mh,
                     mw, mw16, a);
  if (err == cudaSuccess) {
    l.keep = kFastKeep;
    err = launch_lmhead_merge(l, q);
  }
  if (err == cudaSuccess) {
    a.gate = h->error + 1;
    err = launch_pdl(lmhead_kernel<kLmCands>, h->grid, kLmThreads, lm_smem<kLmCands>(), q, mh, mw,
                     mw16, a);
  }
  if (err == cudaSuccess) {
    l.keep = kLmCands;
    err = launch_lmhead_merge(l, q);
  }
  if (cur != h->device) cudaSetDevice(cur);
  if (err != cudaSuccess)
    return lfail(TABBY_ECUDA, "LM-head launch: %s", cudaGetErrorString(err));
  return TABBY_OK;
}

}  // extern "C"
