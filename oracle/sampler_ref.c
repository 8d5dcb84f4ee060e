/*
 * TEST INFRASTRUCTURE ONLY -- the parity checker and the timed CPU baseline, never the
 * product. Compiled with -ffp-contract=off so every float64 operation rounds exactly as
 * JavaScript's does (no fused multiply-add).
 *
 * Each function cites the reference lines it restates (paths inside xOAviOx/tabby).
 */
#include "sampler_ref.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

/* ---------------------------------------------------------------------------------- */
/* SeededRandom / tests/support.ts rng: mulberry32 (sampler.ts:105-119).               */
/* ---------------------------------------------------------------------------------- */
uint32_t or_mulberry32_u32(uint32_t *state) {
  *state = *state + 0x6d2b79f5u;                      /* (state + 0x6d2b79f5) >>> 0 */
  uint32_t t = *state;
  t = (t ^ (t >> 15)) * (t | 1u);                     /* Math.imul(t ^ (t >>> 15), t | 1) */
  t ^= t + (t ^ (t >> 7)) * (t | 61u);                /* t ^= t + Math.imul(t ^ t>>>7, t|61) */
  return t ^ (t >> 14);                               /* (t ^ (t >>> 14)) >>> 0 */
}

double or_mulberry32_next(uint32_t *state) {
  return (double)or_mulberry32_u32(state) / 4294967296.0;
}

/* ---------------------------------------------------------------------------------- */
/* Math.exp. V8 evaluates it with the fdlibm e_exp algorithm (Sun Microsystems, 1993):  */
/*   reduce x = k*ln2 + r with ln2 split into a high part with trailing zero bits and a  */
/*   low correction, |r| <= ln2/2; approximate exp(r) = 1 + r + r*c/(2 - c) with         */
/*   c = r - r^2*R(r^2), R a degree-5 Remez polynomial; scale by 2^k in the exponent.    */
/* Restated here from that published method; tests check it against glibc's exp.       */
/* ---------------------------------------------------------------------------------- */
static const double kLn2Hi = 6.93147180369123816490e-01;
static const double kLn2Lo = 1.90821492927058770002e-10;
static const double kInvLn2 = 1.44269504088896338700e+00;
static const double kR1 = 1.66666666666666019037e-01;
static const double kR2 = -2.77777777770155933842e-03;
static const double kR3 = 6.61375632143793436117e-05;
static const double kR4 = -1.65339022054652515390e-06;
static const double kR5 = 4.13813679705723846039e-08;
static const double kOverflow = 7.09782712893383973096e+02;
static const double kUnderflow = -7.45133219101941108420e+02;

static inline uint64_t d2u(double x) { uint64_t u; memcpy(&u, &x, 8); return u; }
static inline double u2d(uint64_t u) { double x; memcpy(&x, &u, 8); return x; }

double or_js_exp(double x) {
  uint64_t bits = d2u(x);
  uint32_t hx = (uint32_t)(bits >> 32);
  int negative = (int)(hx >> 31);
  hx &= 0x7fffffffu;

  if (hx >= 0x40862E42u) {                 /* |x| >= 709.78 */
    if (hx >= 0x7ff00000u) {
      if (((hx & 0xfffffu) | (uint32_t)bits) != 0) return x + x;   /* NaN */
      return negative ? 0.0 : x;                                    /* exp(+-inf) */
    }
    if (x > kOverflow) return INFINITY;
    if (x < kUnderflow) return 0.0;
  }

  double hi = 0.0, lo = 0.0, r;
  int k = 0;
  if (hx > 0x3fd62e42u) {                  /* |x| > ln2/2 */
    if (hx < 0x3FF0A2B2u) {                /* |x| < 1.5 ln2: k = +-1 */
      k = negative ? -1 : 1;
      hi = negative ? x + kLn2Hi : x - kLn2Hi;
      lo = negative ? -kLn2Lo : kLn2Lo;
    } else {
      k = (int)(kInvLn2 * x + (negative ? -0.5 : 0.5));
      double t = (double)k;
      hi = x - t * kLn2Hi;                 /* exact: kLn2Hi has trailing zero bits */
      lo = t * kLn2Lo;
    }
    r = hi - lo;
  } else if (hx < 0x3e300000u) {           /* |x| < 2^-28 */
    return 1.0 + x;
  } else {
    r = x;
  }

  double r2 = r * r;
  double c = r - r2 * (kR1 + r2 * (kR2 + r2 * (kR3 + r2 * (kR4 + r2 * kR5))));
  if (k == 0) return 1.0 - ((r * c) / (c - 2.0) - r);
  double y = 1.0 - ((lo - (r * c) / (2.0 - c)) - hi);
  if (k >= -1021) {
    return u2d(d2u(y) + ((uint64_t)(int64_t)k << 52));
  }
  /* Result is subnormal: scale in two steps so the final rounding happens once. */
  return u2d(d2u(y) + ((uint64_t)(int64_t)(k + 1000) << 52)) * u2d(0x0170000000000000ull);
}

/* ---------------------------------------------------------------------------------- */
/* argmax (sampler.ts:13-23): strictly greater keeps the lowest index on ties.          */
/* ---------------------------------------------------------------------------------- */
int32_t or_argmax(const float *logits, int64_t n) {
  int32_t best = 0;
  float best_value = logits[0];
  for (int64_t i = 1; i < n; i++) {
    if (logits[i] > best_value) {
      best_value = logits[i];
      best = (int32_t)i;
    }
  }
  return best;
}

/* ---------------------------------------------------------------------------------- */
/* topK (sampler.ts:26-30): sort by b.value - a.value || a.id - b.id, then slice(0, k). */
/* A zero difference (equal values, +0 and -0 included) falls through to the id order.  */
/* ---------------------------------------------------------------------------------- */
typedef struct { float value; int32_t id; } or_entry;

static int cmp_entry(const void *pa, const void *pb) {
  const or_entry *a = (const or_entry *)pa, *b = (const or_entry *)pb;
  double d = (double)b->value - (double)a->value;
  if (d != 0.0) return d > 0 ? 1 : -1;
  return (a->id > b->id) - (a->id < b->id);
}

int32_t or_topk(const float *logits, int64_t n, int32_t k, int32_t *ids, float *values) {
  if (k > n) k = (int32_t)n;
  if (k <= 0) return 0;
  or_entry *all = (or_entry *)malloc((size_t)n * sizeof(or_entry));
  for (int64_t i = 0; i < n; i++) { all[i].value = logits[i]; all[i].id = (int32_t)i; }
  qsort(all, (size_t)n, sizeof(or_entry), cmp_entry);
  for (int32_t i = 0; i < k; i++) {
    if (ids) ids[i] = all[i].id;
    if (values) values[i] = all[i].value;
  }
  free(all);
  return k;
}

/* ---------------------------------------------------------------------------------- */
/* Pool size (inference.worker.ts:120-123):                                             */
/*   temperature <= 0 ? 1 : min(MAX_TOP_K, max(1, topK || MAX_TOP_K))                  */
/* ---------------------------------------------------------------------------------- */
int32_t or_pool_size(double temperature, int32_t top_k, int32_t cap) {
  if (temperature <= 0) return 1;
  int32_t k = top_k != 0 ? top_k : cap;
  if (k < 1) k = 1;
  return k < cap ? k : cap;
}

/* ---------------------------------------------------------------------------------- */
/* reduce_max.wgsl / reduce_sumexp.wgsl semantics.                                      */
/* ---------------------------------------------------------------------------------- */
float or_row_max(const float *logits, int64_t n) {
  float best = -3.0e38f;                   /* NEG_INF sentinel, reduce_max.wgsl:13 */
  for (int64_t i = 0; i < n; i++) best = logits[i] > best ? logits[i] : best;
  return best;
}

double or_sum_exp_f64(const float *logits, int64_t n, float max_value) {
  double total = 0.0;
  for (int64_t i = 0; i < n; i++) total += exp((double)logits[i] - (double)max_value);
  return total;
}

float or_sum_exp_wgsl_f32(const float *logits, int64_t n, float max_value) {
  /* Stage 1 (reduce_sumexp.wgsl:36-64): 256 groups, chunk = ceil(n/256), lanes stride
   * 256 inside a chunk, then a shared-memory tree per group. Stage 2: the same over the
   * 256 partials without exp. */
  const int groups = 256, lanes = 256;
  float partial[256];
  int64_t chunk = (n + groups - 1) / groups;
  for (int g = 0; g < groups; g++) {
    float scratch[256];
    int64_t start = g * chunk, end = start + chunk < n ? start + chunk : n;
    for (int l = 0; l < lanes; l++) {
      float total = 0.0f;
      for (int64_t i = start + l; i < end; i += lanes) total += expf(logits[i] - max_value);
      scratch[l] = total;
    }
    for (int stride = lanes / 2; stride > 0; stride >>= 1)
      for (int l = 0; l < stride; l++) scratch[l] = scratch[l] + scratch[l + stride];
    partial[g] = scratch[0];
  }
  float scratch[256];
  for (int l = 0; l < lanes; l++) scratch[l] = partial[l];
  for (int stride = lanes / 2; stride > 0; stride >>= 1)
    for (int l = 0; l < stride; l++) scratch[l] = scratch[l] + scratch[l + stride];
  return scratch[0];
}

/* ---------------------------------------------------------------------------------- */
/* sampleFromTopK (sampler.ts:147-212), statement by statement in float64.             */
/* ---------------------------------------------------------------------------------- */
int or_sample_from_topk(const int32_t *ids, const float *logits, int32_t n, float max_logit,
                        float sum_exp, double temperature, double top_p, double u,
                        or_outcome *out) {
  if (n <= 0) return -1;                   /* 'sampleFromTopK: empty candidate set' */
  double *exact = (double *)malloc((size_t)n * sizeof(double));
  double *weights = (double *)malloc((size_t)n * sizeof(double));
  const double m = (double)max_logit, s = (double)sum_exp;

  double pool_mass = 0.0;                  /* exact.reduce((a, b) => a + b, 0) */
  for (int32_t i = 0; i < n; i++) {
    exact[i] = or_js_exp((double)logits[i] - m) / s;
    pool_mass += exact[i];
  }
  memset(out, 0, sizeof(*out));
  out->pool_mass = pool_mass;
  out->max_logit = max_logit;
  out->sum_exp = sum_exp;

  if (temperature <= 0) {
    out->id = ids[0];
    out->probability = exact[0];
    out->considered_count = 1;
    out->pool_exhausted = 0;
    free(exact); free(weights);
    return 0;
  }

  double scaled_total = 0.0;
  for (int32_t i = 0; i < n; i++) {
    weights[i] = or_js_exp(((double)logits[i] - m) / temperature);
    scaled_total += weights[i];
  }
  for (int32_t i = 0; i < n; i++) weights[i] = weights[i] / scaled_total;

  int32_t cut = n;
  int pool_exhausted = 0;
  if (top_p < 1) {
    double cumulative = 0.0;
    for (int32_t i = 0; i < n; i++) {
      cumulative += weights[i];
      if (cumulative >= top_p) { cut = i + 1; break; }
    }
    if (pool_mass < top_p) pool_exhausted = 1;
  }

  double total = 0.0;
  for (int32_t i = 0; i < cut; i++) total += weights[i];
  double target = u * total;
  double running = 0.0;
  int32_t chosen = cut - 1;
  for (int32_t i = 0; i < cut; i++) {
    running += weights[i];
    if (target < running) { chosen = i; break; }
  }

  out->id = ids[chosen];
  out->probability = exact[chosen];
  out->considered_count = cut;
  out->pool_exhausted = pool_exhausted;
  free(exact); free(weights);
  return 0;
}

/* ---------------------------------------------------------------------------------- */
/* Whole path per row (forward.ts:520-601 then inference.worker.ts:162-168).          */
/* ---------------------------------------------------------------------------------- */
typedef struct {
  const float *logits; int64_t row_stride; int32_t row0, row1, vocab;
  const or_params *params; const double *uniforms; int32_t cap;
  or_outcome *out; int32_t *topk_ids; float *topk_values; int32_t topk_ld;
} or_job;

static void run_row(const or_job *j, int32_t r, int32_t *ids, float *vals) {
  const float *row = j->logits + (int64_t)r * j->row_stride;
  const or_params *p = &j->params[r];
  int32_t k = or_pool_size(p->temperature, p->top_k, j->cap);
  int32_t n = or_topk(row, j->vocab, k, ids, vals);
  float mx = or_row_max(row, j->vocab);
  float se = (float)or_sum_exp_f64(row, j->vocab, mx);
  or_outcome *o = &j->out[r];
  or_sample_from_topk(ids, vals, n, mx, se, p->temperature, p->top_p, j->uniforms[r], o);
  o->pool_size = n;
  if (j->topk_ids)
    for (int32_t i = 0; i < n; i++) j->topk_ids[(int64_t)r * j->topk_ld + i] = ids[i];
  if (j->topk_values)
    for (int32_t i = 0; i < n; i++) j->topk_values[(int64_t)r * j->topk_ld + i] = vals[i];
}

static void *run_job(void *arg) {
  const or_job *j = (const or_job *)arg;
  int32_t *ids = (int32_t *)malloc((size_t)j->cap * sizeof(int32_t));
  float *vals = (float *)malloc((size_t)j->cap * sizeof(float));
  for (int32_t r = j->row0; r < j->row1; r++) run_row(j, r, ids, vals);
  free(ids); free(vals);
  return NULL;
}

static int run_rows(const float *logits, int64_t row_stride, int32_t rows, int32_t vocab,
                    const or_params *params, const double *uniforms, int32_t cap,
                    or_outcome *out, int32_t *topk_ids, float *topk_values, int32_t topk_ld,
                    int32_t threads) {
  if (rows < 0 || vocab <= 0 || cap <= 0 || !logits || !params || !uniforms || !out) return -1;
  if (threads < 1) threads = 1;
  if (threads > rows) threads = rows > 0 ? rows : 1;
  or_job jobs[256];
  pthread_t tids[256];
  if (threads > 256) threads = 256;
  for (int t = 0; t < threads; t++) {
    or_job j = {logits, row_stride, (int32_t)((int64_t)rows * t / threads),
                (int32_t)((int64_t)rows * (t + 1) / threads), vocab, params, uniforms, cap,
                out, topk_ids, topk_values, topk_ld};
    jobs[t] = j;
  }
  for (int t = 1; t < threads; t++) pthread_create(&tids[t], NULL, run_job, &jobs[t]);
  run_job(&jobs[0]);
  for (int t = 1; t < threads; t++) pthread_join(tids[t], NULL);
  return 0;
}

int or_sample_rows(const float *logits, int64_t row_stride, int32_t rows, int32_t vocab,
                   const or_params *params, const double *uniforms, int32_t cap,
                   or_outcome *out, int32_t *topk_ids, float *topk_values, int32_t topk_ld,
                   int32_t threads) {
  return run_rows(logits, row_stride, rows, vocab, params, uniforms, cap, out, topk_ids,
                  topk_values, topk_ld, threads);
}

double or_bench_rows(const float *logits, int64_t row_stride, int32_t rows, int32_t vocab,
                     const or_params *params, const double *uniforms, int32_t cap,
                     int32_t threads) {
  or_outcome *out = (or_outcome *)malloc((size_t)(rows > 0 ? rows : 1) * sizeof(or_outcome));
  struct timespec a, b;
  clock_gettime(CLOCK_MONOTONIC, &a);
  run_rows(logits, row_stride, rows, vocab, params, uniforms, cap, out, NULL, NULL, 0, threads);
  clock_gettime(CLOCK_MONOTONIC, &b);
  free(out);
  return (double)(b.tv_sec - a.tv_sec) + 1e-9 * (double)(b.tv_nsec - a.tv_nsec);
}
