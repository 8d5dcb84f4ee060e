// sampleFromTopK (xOAviOx/tabby src/engine/sampler.ts:147-212) on candidates already
// sorted by (logit desc, id asc), in float64 with JavaScript's rounding (js_math.cuh).
//
// The per-candidate exponentials are independent, so the device computes them with
// all threads; the sums that decide the token are then replayed in the reference's
// left-to-right order, because a different summation order could move a cumulative
// sum across top_p or across the drawn target.
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

// Sequential remainder of sampleFromTopK given exact[] and scaled[] (n >= 1).
// `weights` may alias `scaled`; it receives scaled[i] / scaledTotal.
JS_FN Decision decide_sequential(const double *exact, const double *scaled, double *weights,
                                 int32_t n, double temperature, double top_p, double u) {
  Decision d;
  double pool_mass = 0.0;  // exact.reduce((a, b) => a + b, 0)
  for (int32_t i = 0; i < n; i++) pool_mass = JS_ADD(pool_mass, exact[i]);
  d.pool_mass = pool_mass;
  if (temperature <= 0) {  // sampler.ts:159-167
    d.chosen = 0;
    d.cut = 1;
    d.pool_exhausted = 0;
    return d;
  }
  double scaled_total = 0.0;  // sampler.ts:171
  for (int32_t i = 0; i < n; i++) scaled_total = JS_ADD(scaled_total, scaled[i]);
  for (int32_t i = 0; i < n; i++) weights[i] = JS_DIV(scaled[i], scaled_total);

  int32_t cut = n;  // sampler.ts:175-189
  int32_t exhausted = 0;
  if (top_p < 1) {
    double cumulative = 0.0;
    for (int32_t i = 0; i < n; i++) {
      cumulative = JS_ADD(cumulative, weights[i]);
      if (cumulative >= top_p) {
        cut = i + 1;
        break;
      }
    }
    if (pool_mass < top_p) exhausted = 1;
  }
  double total = 0.0;  // sampler.ts:191-192
  for (int32_t i = 0; i < cut; i++) total = JS_ADD(total, weights[i]);
  const double target = JS_MUL(u, total);  // sampler.ts:194
  double running = 0.0;
  int32_t chosen = cut - 1;
  for (int32_t i = 0; i < cut; i++) {  // sampler.ts:196-203
    running = JS_ADD(running, weights[i]);
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

}  // namespace tabby
