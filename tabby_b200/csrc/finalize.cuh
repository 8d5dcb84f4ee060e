// sampleFromTopK (xOAviOx/tabby src/engine/sampler.ts:147-212) on candidates already
// sorted by (logit desc, id asc), in float64 with JavaScript's rounding (js_math.cuh).
//
// The device takes the decisions from parallel sums of fast estimates and checks their
// margins against a rigorous error bound; when a margin is too small it replays the
// reference's left-to-right float64 arithmetic (decide_sequential), so the token, the
// cut and poolExhausted always equal the reference's.
#pragma once

#include "js_math.cuh"

namespace tabby {

// exact[i] = exp(l_i - max) / sumExp            (sampler.ts:156)
JS_FN double exact_prob(float logit, float max_logit, float sum_exp) {
  return JS_DIV(js_exp(JS_SUB((double)logit, (double)max_logit)), (double)sum_exp);
}

// scaled[i] = exp((l_i - max) / T)              (sampler.ts:170)
JS_FN double scaled_weight(float logit, float max_logit, double temperature) {
  return js_exp(JS_DIV(JS_SUB((double)logit, (double)max_logit), temperature));
}

struct Decision {
  int32_t chosen;
  int32_t cut;
  double pool_mass;
  int32_t pool_exhausted;
};

// sampleFromTopK's decisions replayed in the reference's order and rounding from the
// candidate logits (n >= 1): poolMass left to right, scaledTotal left to right, weights,
// the top-p cut and the draw (sampler.ts:156-203). `work` holds n doubles.
JS_FN Decision decide_sequential(const float *logits, int32_t n, float max_logit, float sum_exp,
                                 double temperature, double top_p, double u, double *work) {
  Decision d;
  double pool_mass = 0.0;  // exact.reduce((a, b) => a + b, 0)
  for (int32_t i = 0; i < n; i++) pool_mass = JS_ADD(pool_mass, exact_prob(logits[i], max_logit, sum_exp));
  d.pool_mass = pool_mass;
  if (temperature <= 0) {  // sampler.ts:159-167
    d.chosen = 0;
    d.cut = 1;
    d.pool_exhausted = 0;
    return d;
  }
  double scaled_total = 0.0;  // sampler.ts:170-171
  for (int32_t i = 0; i < n; i++) {
    work[i] = scaled_weight(logits[i], max_logit, temperature);
    scaled_total = JS_ADD(scaled_total, work[i]);
  }
  for (int32_t i = 0; i < n; i++) work[i] = JS_DIV(work[i], scaled_total);  // weights

  int32_t cut = n;  // sampler.ts:175-189
  int32_t exhausted = 0;
  if (top_p < 1) {
    double cumulative = 0.0;
    for (int32_t i = 0; i < n; i++) {
      cumulative = JS_ADD(cumulative, work[i]);
      if (cumulative >= top_p) {
        cut = i + 1;
        break;
      }
    }
    if (pool_mass < top_p) exhausted = 1;
  }
  double total = 0.0;  // sampler.ts:191-192
  for (int32_t i = 0; i < cut; i++) total = JS_ADD(total, work[i]);
  const double target = JS_MUL(u, total);  // sampler.ts:194
  double running = 0.0;
  int32_t chosen = cut - 1;
  for (int32_t i = 0; i < cut; i++) {  // sampler.ts:196-203
    running = JS_ADD(running, work[i]);
    if (target < running) {
      chosen = i;
      break;
    }
  }
  d.chosen = chosen;
  d.cut = cut;
  d.pool_exhausted = exhausted;
  return d;
}

#if defined(__CUDACC__)
// Fast float64 estimates for the parallel decisions: CUDA's exp (within 1 ulp) instead of
// the JS-rounded js_exp, and multiplications by reciprocals instead of divisions. An
// estimate of exact[i] or weight[i] is within 8 ulp of the JS value; exp's argument
// error from the reciprocal of T moves a weight w by at most |x| w 2^-52 <= 2^-52 / e
// absolute. The decision margin bound (decision_bound) covers both.
__device__ __forceinline__ double approx_exact(float logit, float max_logit, double inv_sum) {
  return exp((double)logit - (double)max_logit) * inv_sum;
}
__device__ __forceinline__ double approx_scaled(float logit, float max_logit, double inv_t) {
  return exp(((double)logit - (double)max_logit) * inv_t);
}
// Largest difference between a parallel cumulative sum of n estimated terms and the
// reference's left-to-right sum of exact terms, with a factor 4 of headroom.
__device__ __forceinline__ double decision_bound(int n) {
  return 4.0 * (double)(12 * n + 64) * 1.1102230246251565e-16;
}
#endif

}  // namespace tabby
