// Float64 arithmetic that rounds exactly like JavaScript's, on host and device.
//
// sampleFromTopK (xOAviOx/tabby src/engine/sampler.ts:147-212) runs in float64 with
// Math.exp. Token ids must match it bit for bit, so the finalize kernel evaluates the
// same expressions with the same rounding: every multiply and add below is a separately
// rounded IEEE operation (__dmul_rn / __dadd_rn on the device, which the compiler never
// fuses; plain operators on the host, which this library compiles with
// -ffp-contract=off).
//
// js_exp is exp(x) by the fdlibm e_exp method (Sun Microsystems, 1993), which is the
// algorithm V8 evaluates for Math.exp: x = k*ln2 + r with ln2 split into a high part
// whose trailing bits are zero and a low correction, |r| <= ln2/2; exp(r) =
// 1 + r + r*c/(2 - c) with c = r - r^2*R(r^2), R a degree-5 Remez polynomial in r^2;
// then 2^k is added to the exponent. Written here from that published description.
#pragma once

#include <stdint.h>

#if defined(__CUDA_ARCH__)
#define JS_MUL(a, b) __dmul_rn((a), (b))
#define JS_ADD(a, b) __dadd_rn((a), (b))
#define JS_SUB(a, b) __dsub_rn((a), (b))
#define JS_DIV(a, b) __ddiv_rn((a), (b))
#else
#define JS_MUL(a, b) ((a) * (b))
#define JS_ADD(a, b) ((a) + (b))
#define JS_SUB(a, b) ((a) - (b))
#define JS_DIV(a, b) ((a) / (b))
#endif

#if defined(__CUDACC__)
#define JS_FN __host__ __device__ __forceinline__
#else
#define JS_FN static inline
#endif

namespace tabby {

JS_FN uint64_t js_bits(double x) {
#if defined(__CUDA_ARCH__)
  return (uint64_t)__double_as_longlong(x);
#else
  uint64_t u;
  __builtin_memcpy(&u, &x, 8);
  return u;
#endif
}

JS_FN double js_from_bits(uint64_t u) {
#if defined(__CUDA_ARCH__)
  return __longlong_as_double((long long)u);
#else
  double x;
  __builtin_memcpy(&x, &u, 8);
  return x;
#endif
}

JS_FN double js_exp(double x) {
  const double ln2_hi = 6.93147180369123816490e-01;   // 0x3fe62e42fee00000
  const double ln2_lo = 1.90821492927058770002e-10;   // 0x3dea39ef35793c76
  const double inv_ln2 = 1.44269504088896338700e+00;
  const double r1 = 1.66666666666666019037e-01;
  const double r2 = -2.77777777770155933842e-03;
  const double r3 = 6.61375632143793436117e-05;
  const double r4 = -1.65339022054652515390e-06;
  const double r5 = 4.13813679705723846039e-08;
  const double overflow = 7.09782712893383973096e+02;
  const double underflow = -7.45133219101941108420e+02;

  const uint64_t bits = js_bits(x);
  uint32_t hx = (uint32_t)(bits >> 32);
  const bool negative = (hx >> 31) != 0;
  hx &= 0x7fffffffu;

  if (hx >= 0x40862E42u) {  // |x| >= 709.78
    if (hx >= 0x7ff00000u) {
      if (((hx & 0xfffffu) | (uint32_t)bits) != 0) return JS_ADD(x, x);  // NaN
      return negative ? 0.0 : x;
    }
    if (x > overflow) return js_from_bits(0x7ff0000000000000ull);
    if (x < underflow) return 0.0;
  }

  double hi = 0.0, lo = 0.0, r;
  int k = 0;
  if (hx > 0x3fd62e42u) {  // |x| > ln2/2
    if (hx < 0x3FF0A2B2u) {  // |x| < 1.5*ln2
      k = negative ? -1 : 1;
      hi = negative ? JS_ADD(x, ln2_hi) : JS_SUB(x, ln2_hi);
      lo = negative ? -ln2_lo : ln2_lo;
    } else {
      k = (int)JS_ADD(JS_MUL(inv_ln2, x), negative ? -0.5 : 0.5);
      const double t = (double)k;
      hi = JS_SUB(x, JS_MUL(t, ln2_hi));
      lo = JS_MUL(t, ln2_lo);
    }
    r = JS_SUB(hi, lo);
  } else if (hx < 0x3e300000u) {  // |x| < 2^-28
    return JS_ADD(1.0, x);
  } else {
    r = x;
  }

  const double rr = JS_MUL(r, r);
  double poly = JS_ADD(r4, JS_MUL(rr, r5));
  poly = JS_ADD(r3, JS_MUL(rr, poly));
  poly = JS_ADD(r2, JS_MUL(rr, poly));
  poly = JS_ADD(r1, JS_MUL(rr, poly));
  const double c = JS_SUB(r, JS_MUL(rr, poly));
  if (k == 0) return JS_SUB(1.0, JS_SUB(JS_DIV(JS_MUL(r, c), JS_SUB(c, 2.0)), r));
  const double y = JS_SUB(1.0, JS_SUB(JS_SUB(lo, JS_DIV(JS_MUL(r, c), JS_SUB(2.0, c))), hi));
  if (k >= -1021) return js_from_bits(js_bits(y) + ((uint64_t)(int64_t)k << 52));
  // Subnormal result: scale by 2^(k+1000) in the exponent, then by 2^-1000 once.
  return JS_MUL(js_from_bits(js_bits(y) + ((uint64_t)(int64_t)(k + 1000) << 52)),
                js_from_bits(0x0170000000000000ull));
}

}  // namespace tabby
