/*
 * tabby_sample.h -- C ABI of the B200 token sampler (libtabbysample.so).
 *
 * Drop-in for the GPU sampling path of xOAviOx/tabby ("browser-llm"). The reference
 * splits that path in two:
 *   - device side: ForwardPass.encodeSampling (src/engine/forward.ts:520-601) records
 *     reduce_max, reduce_sumexp and k rounds of topk_partial/topk_select
 *     (the WGSL files under src/shaders) and reads back [maxLogit, sumExp, (value, index) * k]
 *     (forward.ts:126-157) as a TopKResult (forward.ts:94-103);
 *   - host side: sampleFromTopK(top, params, random) (src/engine/sampler.ts:147-212)
 *     turns that block into a SampleOutcome, with the candidate pool sized by the
 *     worker's rule (src/worker/inference.worker.ts:120-123).
 * This library runs both halves on the GPU, batched over rows, in one launch.
 *
 * Conventions: every function returns a tabby_status; on failure tabby_last_error()
 * returns a message for the calling thread. Pointers named d_* are device pointers,
 * h_* host pointers. `stream` is a cudaStream_t passed as void* (NULL = legacy stream).
 * Nothing here aborts the process. A sampler handle is bound to one device and is not
 * thread-safe: use one handle per thread or stream.
 */
#ifndef TABBY_SAMPLE_H
#define TABBY_SAMPLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TABBY_ABI_VERSION 1

#if defined(__GNUC__)
#define TABBY_API __attribute__((visibility("default")))
#else
#define TABBY_API
#endif

/* Largest candidate pool the kernels extract. The reference caps k at MAX_TOP_K = 64
 * (src/engine/kernels.ts:448); this build raises the cap to 1024 and keeps 64 as the
 * default so an unmodified caller sees the reference's behaviour. */
#define TABBY_MAX_TOP_K_LIMIT 1024
#define TABBY_DEFAULT_MAX_TOP_K 64
/* Local pool each vocab shard contributes in the sharded path. */
#define TABBY_SHARD_TOP_K 64

typedef enum tabby_status {
  TABBY_OK = 0,
  TABBY_EINVAL = 1,    /* bad argument: ForwardError / RangeError in the reference */
  TABBY_ECUDA = 2,     /* a CUDA runtime call failed */
  TABBY_ENOMEM = 3,    /* device or pinned allocation failed */
  TABBY_EINPUT = 4,    /* a logits row held NaN, +-inf or a value <= -3.0e38 */
  TABBY_ETIMEOUT = 5,  /* a bounded device-side wait gave up; the context stays usable */
  TABBY_EEMPTY = 6     /* 'sampleFromTopK: empty candidate set' (sampler.ts:153) */
} tabby_status;

/* SamplingParams (sampler.ts:83-91) minus `seed`: the caller draws one uniform per row
 * from its SeededRandom and passes it in `uniforms`. */
typedef struct tabby_sampling_params {
  double temperature; /* <= 0 selects the argmax (sampler.ts:159-167) */
  double top_p;       /* nucleus threshold; >= 1 disables it (sampler.ts:175) */
  int32_t top_k;      /* pool size request; 0 = the sampler's max_top_k (worker :120-123) */
  int32_t reserved;   /* must be 0 */
} tabby_sampling_params; /* 24 bytes */

/* SampleOutcome (sampler.ts:121-135) plus the TopKResult statistics it came from. */
typedef struct tabby_sample_outcome {
  int32_t id;               /* sampled token id */
  int32_t considered_count; /* candidates that survived top-p */
  double probability;       /* full-vocabulary probability of `id` */
  double pool_mass;         /* full-vocabulary mass held by the pool */
  int32_t pool_exhausted;   /* 1 when top-p asked for more mass than the pool held */
  int32_t pool_size;        /* k actually extracted: min(pool rule, vocab) */
  float max_logit;          /* TopKResult.maxLogit */
  float sum_exp;            /* TopKResult.sumExp: sum(exp(x - maxLogit)), f32 */
  int32_t status;           /* tabby_status of this row */
  int32_t reserved;
} tabby_sample_outcome; /* 48 bytes */

typedef struct tabby_sampler_config {
  int32_t device;     /* CUDA device ordinal the handle is bound to */
  int32_t max_top_k;  /* MAX_TOP_K: 1..TABBY_MAX_TOP_K_LIMIT (0 = default 64) */
  int32_t max_rows;   /* capacity of the host-buffer entry points (0 = 256) */
  int32_t max_vocab;  /* capacity of the host-buffer entry points (0 = 151936) */
} tabby_sampler_config;

typedef struct tabby_sampler tabby_sampler;

/* ABI version of the loaded library (TABBY_ABI_VERSION). */
TABBY_API int32_t tabby_abi_version(void);

/* Thread-local message for the last failing call on this thread ("" if none). */
TABBY_API const char *tabby_last_error(void);

/* Creates a handle. Replaces ForwardPass.create's sampling buffers (forward.ts:240-248):
 * device and pinned staging for the host-buffer entry points are owned by the handle. */
TABBY_API int tabby_sampler_create(const tabby_sampler_config *config, tabby_sampler **out);

/* Frees everything the handle owns (ForwardPass.destroy, forward.ts:311-317). */
TABBY_API int tabby_sampler_destroy(tabby_sampler *sampler);

/*
 * The batched sampler, all buffers on the device, asynchronous on `stream`.
 * Per row r (logits row at d_logits + r * row_stride, `vocab` floats):
 *   k = pool rule(params[r].temperature, params[r].top_k, max_top_k), clipped to vocab;
 *   maxLogit, sumExp, exact top-k by (value desc, index asc) on the raw logits
 *     (forward.ts:520-601, the four sampling WGSL kernels);
 *   sampleFromTopK(top, params[r], u = d_uniforms[r]) (sampler.ts:147-212) in float64.
 * Writes d_out[r]; when d_topk_ids / d_topk_values are non-NULL also the k candidates
 * (ids int32, raw logits f32) at stride topk_ld (>= max_top_k) in candidate order.
 * Per-row failures (non-finite logits) are reported in d_out[r].status.
 * Requirements: d_logits 4-byte aligned, row_stride >= vocab, 1 <= vocab <= 2^30.
 */
TABBY_API int tabby_sample_rows_async(tabby_sampler *sampler, const float *d_logits, int64_t row_stride,
                            int32_t rows, int32_t vocab, const tabby_sampling_params *d_params,
                            const double *d_uniforms, tabby_sample_outcome *d_out,
                            int32_t *d_topk_ids, float *d_topk_values, int32_t topk_ld,
                            void *stream);

/*
 * tabby_sample_rows_async with the draws made on the device: d_rng_state[r] is row r's
 * SeededRandom state (sampler.ts:105-119; a new generator of seed s starts at s as
 * uint32). Where sampleFromTopK calls random.next() -- a row with temperature > 0, a
 * non-empty pool and no error -- the kernel advances d_rng_state[r] by one mulberry32
 * step and uses u32 / 2^32 as u; greedy and failed rows leave it unchanged (the
 * reference returns before drawing, sampler.ts:153,159-167). Nothing in the call
 * depends on host state that changes between calls, so a decode step that calls it can
 * be captured once in a CUDA graph and replayed (the per-launch epoch lives in the
 * handle's device scratch). Moves the worker's per-token draw (inference.worker.ts:142,
 * 165) onto the GPU.
 */
TABBY_API int tabby_sample_rows_rng_async(tabby_sampler *sampler, const float *d_logits,
                                int64_t row_stride, int32_t rows, int32_t vocab,
                                const tabby_sampling_params *d_params, uint32_t *d_rng_state,
                                tabby_sample_outcome *d_out, int32_t *d_topk_ids,
                                float *d_topk_values, int32_t topk_ld, void *stream);

/*
 * Same computation from and to HOST buffers: copies logits/params/uniforms in, runs,
 * copies outcomes (and candidates when h_topk_ids/h_topk_values are non-NULL) back and
 * synchronises. Returns the first failing row's status (TABBY_EINPUT, ...) if any.
 * rows <= max_rows and vocab <= max_vocab of the handle; row_stride is the host stride.
 * This is the call sampler.ts's sample() reaches through the N-API addon.
 */
TABBY_API int tabby_sample_rows(tabby_sampler *sampler, const float *h_logits, int64_t row_stride,
                      int32_t rows, int32_t vocab, const tabby_sampling_params *h_params,
                      const double *h_uniforms, tabby_sample_outcome *h_out,
                      int32_t *h_topk_ids, float *h_topk_values, int32_t topk_ld);

/*
 * Top-k block only, the TopKResult of ForwardPass.runFull(ids, {topK: k})
 * (forward.ts:339-350, 430-448): per row writes (2 + 2k) 32-bit words at
 * d_block + r * block_ld:  [maxLogit, sumExp, (value f32, index u32 bits) * k]
 * exactly as topk_select.wgsl:60-64 lays them out. 0 <= k <= max_top_k, k <= vocab
 * (k > max_top_k is rejected like forward.ts:348-351); block_ld >= 2 + 2k.
 * Row failures set maxLogit to NaN.
 */
TABBY_API int tabby_topk_rows_async(tabby_sampler *sampler, const float *d_logits, int64_t row_stride,
                          int32_t rows, int32_t vocab, int32_t k, float *d_block,
                          int32_t block_ld, void *stream);

/*
 * Vocab-sharded sampling, step 1 (new in this build; the reference has no multi-GPU
 * path). This rank holds columns [vocab_offset, vocab_offset + shard_vocab) of every
 * row. Writes per row (2 + 2 * TABBY_SHARD_TOP_K) words at d_block + r * block_ld:
 * [local max, local sum(exp(x - local max)), (value, GLOBAL index bits) * 64], unused
 * slots padded with (-inf, 0xffffffff). The blocks of all ranks are then all-gathered.
 */
TABBY_API int tabby_shard_local_async(tabby_sampler *sampler, const float *d_logits, int64_t row_stride,
                            int32_t rows, int32_t shard_vocab, int64_t vocab_offset,
                            float *d_block, int32_t block_ld, void *stream);

/*
 * Vocab-sharded sampling, step 2: d_gathered holds `shards` blocks per row as
 * all-gathered rank-major: block of (shard s, row r) at d_gathered + (s*rows + r)*block_ld.
 * Merges (max, sum-exp) pairs as M = max m_s, S = sum s_s exp(m_s - M), takes the global
 * top-k of the candidates by (value desc, global index asc), and runs sampleFromTopK
 * with params[r] and uniforms[r]. Pool sizes above TABBY_SHARD_TOP_K are clipped to it.
 * 1 <= shards <= 16.
 */
TABBY_API int tabby_shard_merge_async(tabby_sampler *sampler, const float *d_gathered, int32_t shards,
                            int32_t rows, int32_t block_ld, const tabby_sampling_params *d_params,
                            const double *d_uniforms, tabby_sample_outcome *d_out,
                            int32_t *d_topk_ids, float *d_topk_values, int32_t topk_ld,
                            void *stream);

/*
 * Vocab-sharded sampling with the exchange done by the merge kernel itself over NVLink
 * peer memory, in place of the all-gather between tabby_shard_local_async and
 * tabby_shard_merge_async (new in this build; the reference has no multi-GPU path). One
 * exchange object per rank of a job of `world` ranks (one process per GPU):
 *   1. tabby_exchange_create; tabby_exchange_ipc_handle gives this rank's
 *      TABBY_EXCHANGE_HANDLE_BYTES-byte CUDA IPC handle; the caller moves the handles
 *      between processes (rank-major) and passes all of them to tabby_exchange_open;
 *   2. every step: tabby_shard_local_async writes this rank's blocks into the buffer
 *      tabby_exchange_blocks returns (ask before every step: two buffers alternate), then
 *      tabby_exchange_merge_async on the same stream. It announces this rank's blocks to
 *      every peer (a release store into the peer's flag word), waits for every peer's
 *      word, then merges every row reading the peers' blocks over NVLink, and writes all
 *      `rows` outcomes to d_out, the same on every rank. Every rank must make the same
 *      calls in the same order with the same `rows`, params and uniforms. A wait that
 *      runs out (0.5 s) gives every row status TABBY_ETIMEOUT; the kernel always returns.
 *   3. tabby_exchange_destroy only after every rank's last merge has completed (e.g. after
 *      a device synchronize and a barrier between the processes).
 * 1 <= world <= TABBY_EXCHANGE_MAX_WORLD; pool sizes above TABBY_SHARD_TOP_K are clipped.
 */
#define TABBY_EXCHANGE_MAX_WORLD 16
#define TABBY_EXCHANGE_HANDLE_BYTES 64
typedef struct tabby_exchange tabby_exchange;
TABBY_API int tabby_exchange_create(int32_t device, int32_t world, int32_t rank, int32_t max_rows,
                          tabby_exchange **out);
TABBY_API int tabby_exchange_ipc_handle(tabby_exchange *exchange, void *handle);
TABBY_API int tabby_exchange_open(tabby_exchange *exchange, const void *handles);
TABBY_API int tabby_exchange_blocks(tabby_exchange *exchange, float **d_blocks, int32_t *block_ld);
TABBY_API int tabby_exchange_merge_async(tabby_exchange *exchange, int32_t rows,
                               const tabby_sampling_params *d_params, const double *d_uniforms,
                               tabby_sample_outcome *d_out, void *stream);
TABBY_API int tabby_exchange_destroy(tabby_exchange *exchange);

/*
 * Host-side sampleFromTopK on a TopKResult (sampler.ts:147-212) with the same float64
 * arithmetic the device finalize uses; no GPU involved. For callers that already hold
 * a TopKResult (e.g. from tabby_topk_rows_async).
 */
TABBY_API int tabby_sample_from_topk(const int32_t *ids, const float *logits, int32_t n, float max_logit,
                           float sum_exp, const tabby_sampling_params *params, double uniform,
                           tabby_sample_outcome *out);

/*
 * Row softmax in place over d_x [n_rows, row_len] fp32 (softmax_rows.wgsl, the attention
 * score softmax of ForwardPass; CPU form cpu.ts softmaxRows). With causal_period != 0 row
 * r keeps its first causal_offset + (r % causal_period) + 1 entries (rows are (head,
 * query)) and the rest are set to 0; causal_period == 0 softmaxes whole rows. Entries:
 * exp(x - max) / sum over the kept part, fp32. Requires row_len >= 1 and
 * causal_offset + causal_period <= row_len (the shader would read past the row).
 * No handle needed; asynchronous on `stream`.
 */
TABBY_API int tabby_softmax_rows_async(float *d_x, int32_t n_rows, int32_t row_len,
                                int32_t causal_period, int32_t causal_offset, void *stream);

/*
 * Test entry for the failure path of the row pass: tabby_sample_rows_async (in the chunked
 * schedule, which batches below the resident CTA count use) with the bounded wait for a
 * row's plan limited to `spin_limit` polls and the plan of row `withhold_row` never
 * published (-1: none). The waits for that row run out; the kernel still returns, the row
 * reports TABBY_ETIMEOUT in its outcome, every other row is sampled normally and the
 * handle stays usable. The reference surfaces device failure as an error the same way
 * (src/worker/inference.worker.ts:55-58, onDeviceLost -> fail). Not for production use.
 */
TABBY_API int tabby_sample_rows_debug_async(tabby_sampler *sampler, const float *d_logits,
                                  int64_t row_stride, int32_t rows, int32_t vocab,
                                  const tabby_sampling_params *d_params,
                                  const double *d_uniforms, tabby_sample_outcome *d_out,
                                  uint32_t spin_limit, int32_t withhold_row, void *stream);

/* Largest max_top_k tabby_sample_rows_noalloc accepts (its scratch array is fixed). */
#define TABBY_NOALLOC_MAX_TOP_K 256

/*
 * tabby_sample_rows_async without a sampler handle and without any device allocation.
 * No counterpart in the reference: it exists for callers that cannot call cudaMalloc
 * (code running under an allocator that owns all device memory, plug-in hosts that
 * forbid allocation on their request path, callers that must not add allocations
 * between steps). The row kernel's global scratch -- per-row counters and per-slice
 * candidate lists, about 5.4 MB -- lives in a file-scope __device__ array that every GPU
 * loading the library keeps until the process exits. Same inputs, outputs and results
 * as tabby_sample_rows_async with max_top_k as the pool cap; max_top_k must be
 * 1..TABBY_NOALLOC_MAX_TOP_K, larger values are rejected with TABBY_EINVAL.
 * Runs on the current device. The first call on a device looks up the array's device
 * address (cudaGetSymbolAddress): make that first call before any stream capture.
 * All calls on a device share the one array. No call clears it: it is zero when the
 * library loads, and every launch leaves it ready for the next (the launch's last unit
 * take resets the unit counter, each row's counters are reset before the row is used,
 * and plan entries carry a launch number kept in the array). Calls that overlap on the
 * GPU -- concurrent streams or threads -- race and must be serialised by the caller.
 */
TABBY_API int tabby_sample_rows_noalloc(const float *d_logits, int64_t row_stride, int32_t rows,
                                        int32_t vocab, int32_t max_top_k,
                                        const tabby_sampling_params *d_params,
                                        const double *d_uniforms, tabby_sample_outcome *d_out,
                                        int32_t *d_topk_ids, float *d_topk_values,
                                        int32_t topk_ld, void *stream);

/*
 * Fused LM head + sampling for the decode step (new in this build): replaces the
 * reference's lm_head matmul into `this.logits` (src/engine/forward.ts:418-428,
 * src/shaders/matmul_f16.wgsl / matvec_q4.wgsl) followed by the sampling dispatches
 * (forward.ts:520-601) and sampleFromTopK (src/engine/sampler.ts:147-212). Logits
 * hidden[r] . weight[v] (bf16 inputs, fp32 accumulation on the tensor cores) are consumed
 * in the GEMM's epilogue and never written to HBM; the pool cap is the reference's
 * MAX_TOP_K = 64 (kernels.ts:448).
 * A handle holds the per-CTA partials for up to max_rows (<= TABBY_LMHEAD_MAX_ROWS) rows of
 * a fixed vocab (<= TABBY_MAX_VOCAB_LMHEAD) and hidden size (a multiple of 64).
 */
#define TABBY_LMHEAD_MAX_ROWS 128
#define TABBY_MAX_VOCAB_LMHEAD 16777216
typedef struct tabby_lmhead tabby_lmhead;
TABBY_API int tabby_lmhead_create(int32_t device, int32_t max_rows, int32_t vocab,
                                  int32_t hidden, tabby_lmhead **out);
TABBY_API int tabby_lmhead_destroy(tabby_lmhead *lmhead);
/*
 * d_hidden: bf16 [rows][hidden] row-major; d_weight: bf16 [vocab][hidden] row-major (the
 * lm_head / tied embedding matrix); both 16-byte aligned. Per row: pool rule with cap 64,
 * max and sum-exp of the row's logits, exact top-k (value desc, index asc), then
 * sampleFromTopK with d_uniforms[r]; writes d_out[r] and, when non-NULL, the candidates
 * (d_topk_ids / d_topk_values at stride topk_ld >= 64). d_logits_out (tests; normally
 * NULL) receives the fp32 logits [rows][vocab] the epilogue saw. Asynchronous on `stream`.
 */
TABBY_API int tabby_lmhead_sample_async(tabby_lmhead *lmhead, const void *d_hidden,
                                        const void *d_weight, int32_t rows,
                                        const tabby_sampling_params *d_params,
                                        const double *d_uniforms, tabby_sample_outcome *d_out,
                                        int32_t *d_topk_ids, float *d_topk_values,
                                        int32_t topk_ld, float *d_logits_out, void *stream);

/* Pool-size rule of the worker (inference.worker.ts:120-123) with the handle's cap. */
TABBY_API int32_t tabby_pool_size(double temperature, int32_t top_k, int32_t max_top_k);

#ifdef __cplusplus
}
#endif
#endif /* TABBY_SAMPLE_H */
