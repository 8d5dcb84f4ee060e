// Fused LM head + sampling on sm_100a: logits = hidden x weight^T computed with tcgen05
// tensor-core MMAs and consumed in the epilogue, so they never reach HBM.
//
// Replaces, for the decode step, the reference's lm_head dispatch
// (xOAviOx/tabby src/engine/forward.ts:418-428: encodeMatmul(... 'lm_head') with
// src/shaders/matmul_f16.wgsl / matvec_q4.wgsl into this.logits) followed by the sampling
// dispatches (forward.ts:520-601) and sampleFromTopK (src/engine/sampler.ts:147-212).
//
//   lmhead_kernel   one CTA a SM, each a contiguous range of vocabulary tiles of 128 rows.
//                   warp 0 (one lane)  TMA producer: cp.async.bulk.tensor 2-D loads of the
//                                      hidden tile (128 x 64 bf16) and the weight tile
//                                      (128 x 64 bf16), 128-byte swizzle, into a 4-stage
//                                      ring (mbarrier transaction counts). No multicast.
//                   warp 1 (one lane)  tcgen05.mma.cta_group::1.kind::f16, M = 128 token rows
//                                      (rows past the batch are zero-filled by TMA), N = 128
//                                      vocabulary rows, K = 16 a step, fp32 accumulators in
//                                      TMEM, double-buffered (2 x 128 columns); tcgen05.commit
//                                      frees a stage and hands a finished tile over.
//                   warps 2-5          epilogue: tcgen05.ld 32x32b of the accumulator, one
//                                      thread a token row: online max and sum(exp(x - max)),
//                                      and the row's 64 best logits of the CTA's range kept
//                                      in shared memory (replace-the-minimum), then the
//                                      CTA's (max, sum-exp) and candidates to a partials
//                                      buffer (optionally the logits themselves, for tests).
//   lmhead_merge_kernel (sampler_kernels.cu) finishes every row: merged statistics, the
//                   global top-k of the candidates, sampleFromTopK in float64.
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

namespace tabby {
namespace {

constexpr int kLmM = 128;          // token rows of a tile (the MMA's M)
constexpr int kLmN = 128;          // vocabulary rows of a tile (the MMA's N)
constexpr int kLmK = 64;           // hidden elements a stage (128 bytes of bf16: one swizzle row)
constexpr int kLmStages = 4;
constexpr int kTileBytes = kLmM * kLmK * 2;  // 16 KB, A and B alike
constexpr int kStageBytes2 = 2 * kTileBytes;
constexpr int kLmThreads = 192;    // producer warp, MMA warp, 4 epilogue warps
constexpr int kTmemCols = 2 * kLmN;
constexpr unsigned long long kWaitNs = 500000000ull;  // a bounded wait gives up after 0.5 s
// Dynamic shared memory: the stages, the candidate table [kLmCands][kLmM], barriers.
constexpr size_t kLmSmem = 1024 + (size_t)kLmStages * kStageBytes2 + (size_t)kLmCands * kLmM * 8 + 256;

struct LmArgs {
  int32_t rows, vocab, hidden;
  int32_t tiles_per_cta;
  int32_t ntiles;
  float2 *stats;                 // [rows][gridDim.x]
  unsigned long long *cands;     // [rows][gridDim.x][kLmCands]
  float *logits_out;             // tests only: [rows][vocab] fp32, or NULL
  uint32_t *error;
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
__device__ __forceinline__ bool mb_wait(uint64_t *b, uint32_t parity) {
  const unsigned long long t0 = now_ns();
  for (uint32_t i = 0;; i++) {
    if ((i & 1023u) == 1023u && now_ns() - t0 > kWaitNs) return false;
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(b)), "r"(parity)
        : "memory");
    if (ok) return true;
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
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kLmN >> 3) << 17) |
                            ((uint32_t)(kLmM >> 4) << 24);

__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(kIdesc), "r"(acc)
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
__device__ __forceinline__ uint64_t lm_comp(uint64_t raw_idx) {  // raw << 32 | idx
  return ((uint64_t)lm_key(__uint_as_float((uint32_t)(raw_idx >> 32))) << 32) |
         (uint64_t)(~(uint32_t)raw_idx);
}

__global__ void __launch_bounds__(kLmThreads, 1)
    lmhead_kernel(const __grid_constant__ CUtensorMap map_h, const __grid_constant__ CUtensorMap map_w,
                  const __grid_constant__ LmArgs a) {
  extern __shared__ unsigned char smem_dyn[];
  unsigned char *base = reinterpret_cast<unsigned char *>(
      (reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~(uintptr_t)1023);
  unsigned char *stages = base;  // [stage]{A 16 KB, B 16 KB}
  unsigned long long *cand =
      reinterpret_cast<unsigned long long *>(base + kLmStages * kStageBytes2);  // [64][128]
  uint64_t *bars = reinterpret_cast<uint64_t *>(cand + kLmCands * kLmM);
  uint64_t *full = bars, *empty = bars + kLmStages;
  uint64_t *tfull = bars + 2 * kLmStages, *tempty = tfull + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(tempty + 2);
  volatile uint32_t *err = tmem_slot + 1;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int t0 = blockIdx.x * a.tiles_per_cta;
  const int nt = max(0, min(a.tiles_per_cta, a.ntiles - t0));
  const int kb_n = a.hidden / kLmK;

  if (tid == 0) {
    for (int s = 0; s < kLmStages; s++) {
      mb_init(&full[s], 1);
      mb_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      mb_init(&tfull[b], 1);
      mb_init(&tempty[b], 128);
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
    // ---- TMA producer ----
    if (lane == 0) {
      int it = 0;
      for (int t = 0; t < nt && !*err; t++) {
        const int v0 = (t0 + t) * kLmN;
        for (int kb = 0; kb < kb_n; kb++, it++) {
          const int s = it % kLmStages;
          if (it >= kLmStages && !mb_wait(&empty[s], ((it / kLmStages) - 1) & 1)) {
            *err = 1u;
            break;
          }
          unsigned char *st = stages + s * kStageBytes2;
          mb_arrive_expect(&full[s], kStageBytes2);
          tma_load_2d(st, &map_h, kb * kLmK, 0, &full[s]);
          tma_load_2d(st + kTileBytes, &map_w, kb * kLmK, v0, &full[s]);
        }
      }
      // Every issued load has landed before the CTA may exit (bounded).
      for (int j = max(0, it - kLmStages); j < it; j++)
        mb_wait(&full[j % kLmStages], (j / kLmStages) & 1);
    }
  } else if (warp == 1) {
    // ---- MMA issuer ----
    if (lane == 0) {
      int it = 0;
      for (int t = 0; t < nt && !*err; t++) {
        const int b = t & 1;
        if (t >= 2 && !mb_wait(&tempty[b], ((t >> 1) - 1) & 1)) {
          *err = 1u;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(b * kLmN);
        for (int kb = 0; kb < kb_n; kb++, it++) {
          const int s = it % kLmStages;
          if (!mb_wait(&full[s], (it / kLmStages) & 1)) {
            *err = 1u;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_addr(stages + s * kStageBytes2);
#pragma unroll
          for (int kk = 0; kk < kLmK / 16; kk++)  // 16 bf16 = 32 bytes a step along K
            mma_bf16(d, smem_desc(sa + 32 * kk), smem_desc(sa + kTileBytes + 32 * kk),
                     (kb | kk) != 0 ? 1u : 0u);
          mma_commit(&empty[s]);  // the stage is free once these MMAs have read it
        }
        if (*err) break;
        mma_commit(&tfull[b]);  // the tile's accumulator is complete
      }
    }
  } else {
    // ---- epilogue: thread = token row (TMEM lane 32 * (warp % 4) + lane) ----
    const int q = warp & 3;
    const int row = 32 * q + lane;
    const bool live = row < a.rows;
    float m = -3.40282347e38f, s = 0.f;
    int filled = 0, min_slot = 0;
    uint64_t min_c = 0ull;  // composite of the smallest kept candidate
    constexpr float kLog2e = 1.44269504088896341f;
    for (int t = 0; t < nt; t++) {
      const int b = t & 1;
      if (!mb_wait(&tfull[b], (t >> 1) & 1)) {
        *err = 1u;
        break;
      }
      tc_fence_after();
      const int v0 = (t0 + t) * kLmN;
#pragma unroll 1
      for (int c = 0; c < kLmN / 32; c++) {
        uint32_t r[32];
        tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(b * kLmN + 32 * c), r);
        if (!live) continue;
        const int vb = v0 + 32 * c;
        const int nv = min(32, a.vocab - vb);
        if (nv <= 0) continue;
        float cm = -3.40282347e38f;
#pragma unroll
        for (int j = 0; j < 32; j++)
          if (j < nv) cm = fmaxf(cm, __uint_as_float(r[j]));
        if (cm > m) {
          s *= exp2f((m - cm) * kLog2e);
          m = cm;
        }
        const float mL = m * kLog2e;
#pragma unroll
        for (int j = 0; j < 32; j++)
          if (j < nv) s += exp2f(fmaf(__uint_as_float(r[j]), kLog2e, -mL));
        if (a.logits_out) {
#pragma unroll
          for (int j = 0; j < 32; j++)
            if (j < nv) a.logits_out[(int64_t)row * a.vocab + vb + j] = __uint_as_float(r[j]);
        }
        // The row's 64 best of this CTA: fill, then replace the smallest.
#pragma unroll 1
        for (int j = 0; j < nv; j++) {
          const uint64_t raw = ((uint64_t)r[j] << 32) | (uint32_t)(vb + j);
          const uint64_t cmp = lm_comp(raw);
          if (filled < kLmCands) {
            cand[filled * kLmM + row] = raw;
            if (filled == 0 || cmp < min_c) {
              min_c = cmp;
              min_slot = filled;
            }
            filled++;
          } else if (cmp > min_c) {
            cand[min_slot * kLmM + row] = raw;
            min_c = ~0ull;
            for (int e = 0; e < kLmCands; e++) {
              const uint64_t ce = lm_comp(cand[e * kLmM + row]);
              if (ce < min_c) {
                min_c = ce;
                min_slot = e;
              }
            }
          }
        }
      }
      tc_fence_before();
      mb_arrive(&tempty[b]);  // the accumulator may be overwritten
    }
    if (live) {
      const int parts = gridDim.x;
      a.stats[(int64_t)row * parts + blockIdx.x] = make_float2(m, s);
      unsigned long long *dst = a.cands + ((int64_t)row * parts + blockIdx.x) * kLmCands;
      for (int e = 0; e < kLmCands; e++)
        dst[e] = e < filled ? cand[e * kLmM + row] : 0xffffffffull;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (*err && tid == 0) atomicOr(a.error, 1u);
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

// K-major bf16 matrix [outer][inner] with boxes of 64 x 128 (inner x outer), 128-byte
// swizzle, zero fill out of bounds.
bool make_map(CUtensorMap *m, const void *ptr, uint64_t inner, uint64_t outer) {
  EncodeTiled enc = encode_fn();
  if (!enc) return false;
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {inner * 2};
  const cuuint32_t box[2] = {(cuuint32_t)kLmK, 128u};
  const cuuint32_t elem[2] = {1u, 1u};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(ptr), dims, strides, box,
             elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
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
  int32_t device;
  int32_t max_rows;
  int32_t vocab;
  int32_t hidden;
  int32_t grid;
  int32_t tiles_per_cta;
  int32_t ntiles;
  float2 *stats;
  unsigned long long *cands;
  uint32_t *error;
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
  h->ntiles = (vocab + kLmN - 1) / kLmN;
  h->tiles_per_cta = (h->ntiles + sms - 1) / std::max(sms, 1);
  h->grid = (h->ntiles + h->tiles_per_cta - 1) / h->tiles_per_cta;
  const size_t nst = (size_t)max_rows * h->grid;
  if ((err = cudaMalloc(&h->stats, nst * sizeof(float2))) != cudaSuccess ||
      (err = cudaMalloc(&h->cands, nst * kLmCands * 8)) != cudaSuccess ||
      (err = cudaMalloc(&h->error, 16)) != cudaSuccess ||
      (err = cudaMemset(h->error, 0, 16)) != cudaSuccess ||
      (err = cudaFuncSetAttribute(lmhead_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)kLmSmem)) != cudaSuccess) {
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
  CUtensorMap mh, mw;
  if (!make_map(&mh, d_hidden, (uint64_t)h->hidden, (uint64_t)rows) ||
      !make_map(&mw, d_weight, (uint64_t)h->hidden, (uint64_t)h->vocab)) {
    if (cur != h->device) cudaSetDevice(cur);
    return lfail(TABBY_ECUDA, "cuTensorMapEncodeTiled failed");
  }
  cudaStream_t q = (cudaStream_t)stream;
  LmArgs a;
  a.rows = rows;
  a.vocab = h->vocab;
  a.hidden = h->hidden;
  a.tiles_per_cta = h->tiles_per_cta;
  a.ntiles = h->ntiles;
  a.stats = h->stats;
  a.cands = h->cands;
  a.logits_out = d_logits_out;
  a.error = h->error;
  err = cudaMemsetAsync(h->error, 0, 4, q);
  if (err == cudaSuccess) {
    lmhead_kernel<<<h->grid, kLmThreads, kLmSmem, q>>>(mh, mw, a);
    err = cudaGetLastError();
  }
  if (err == cudaSuccess) {
    LmheadMergeLaunch l;
    l.stats = h->stats;
    l.cands = h->cands;
    l.parts = h->grid;
    l.rows = rows;
    l.vocab = h->vocab;
    l.params = d_params;
    l.uniforms = d_uniforms;
    l.out = d_out;
    l.topk_ids = d_topk_ids;
    l.topk_values = d_topk_values;
    l.topk_ld = topk_ld;
    l.error = h->error;
    err = launch_lmhead_merge(l, q);
  }
  if (cur != h->device) cudaSetDevice(cur);
  if (err != cudaSuccess)
    return lfail(TABBY_ECUDA, "LM-head launch: %s", cudaGetErrorString(err));
  return TABBY_OK;
}

}  // extern "C"
