/*
 * TEST INFRASTRUCTURE ONLY -- the parity checker, never the product.
 *
 * CPU restatement of the reference's token-sampling path (xOAviOx/tabby, TypeScript):
 *   src/engine/sampler.ts      argmax :13-23, topK :26-30, SeededRandom :105-119,
 *                              sampleFromTopK :147-212
 *   src/worker/inference.worker.ts  pool-size rule :120-123
 *   src/engine/forward.ts      TopKResult :94-103, sample block layout :126-157
 *   src/shaders/reduce_max.wgsl, reduce_sumexp.wgsl, topk_partial.wgsl,
 *   topk_select.wgsl           max / sum-exp / top-k semantics (lower index wins ties)
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg may load this.
 */
#ifndef TABBY_ORACLE_SAMPLER_REF_H
#define TABBY_ORACLE_SAMPLER_REF_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
  double temperature;
  double top_p;
  int32_t top_k;
  int32_t reserved;
} or_params;

typedef struct {
  int32_t id;
  int32_t considered_count;
  double probability;
  double pool_mass;
  int32_t pool_exhausted;
  int32_t pool_size;
  float max_logit;
  float sum_exp;
  int32_t status;
  int32_t reserved;
} or_outcome;

/* mulberry32 (sampler.ts:105-119, tests/support.ts:7-16). */
uint32_t or_mulberry32_u32(uint32_t *state);
double or_mulberry32_next(uint32_t *state);

/* exp(x) by the fdlibm e_exp method, which is what V8's Math.exp evaluates. */
double or_js_exp(double x);

/* Strictly-greater argmax: lowest index on ties (sampler.ts:13-23). */
int32_t or_argmax(const float *logits, int64_t n);

/* Full sort by (value desc, id asc), first k (sampler.ts:26-30). k is clipped to n. */
int32_t or_topk(const float *logits, int64_t n, int32_t k, int32_t *ids, float *values);

/* Worker pool rule (inference.worker.ts:120-123) with cap = MAX_TOP_K. */
int32_t or_pool_size(double temperature, int32_t top_k, int32_t cap);

float or_row_max(const float *logits, int64_t n);
/* sum(exp(x - max)) in float64 (the "unlimited precision" mode of cpu.ts:1-17). */
double or_sum_exp_f64(const float *logits, int64_t n, float max_value);
/* The same sum in f32 with reduce_sumexp.wgsl's two-stage order (256 groups x 256 lanes). */
float or_sum_exp_wgsl_f32(const float *logits, int64_t n, float max_value);

/* sampleFromTopK (sampler.ts:147-212), float64 throughout. Returns 0, or -1 on n == 0. */
int or_sample_from_topk(const int32_t *ids, const float *logits, int32_t n, float max_logit,
                        float sum_exp, double temperature, double top_p, double u,
                        or_outcome *out);

/*
 * Whole path per row: pool rule, row max, f64 sum-exp rounded to f32, top-k full sort,
 * sampleFromTopK with the row's uniform. topk_ids/topk_values get pool_size entries per
 * row at stride topk_ld (may be NULL). Returns 0, or -1 on invalid arguments.
 */
int or_sample_rows(const float *logits, int64_t row_stride, int32_t rows, int32_t vocab,
                   const or_params *params, const double *uniforms, int32_t cap,
                   or_outcome *out, int32_t *topk_ids, float *topk_values, int32_t topk_ld,
                   int32_t threads);

/* Time the reference CPU path (full sort + sampleFromTopK) on `rows` rows. */
double or_bench_rows(const float *logits, int64_t row_stride, int32_t rows, int32_t vocab,
                     const or_params *params, const double *uniforms, int32_t cap,
                     int32_t threads);

#ifdef __cplusplus
}
#endif
#endif
