// Elementary functions with a fixed fp32 operation sequence, shared
// verbatim by the CUDA kernels and the CPU oracle so that both round
// identically (no library exp/erf, whose last bits differ between libm and
// the device). Compile the CPU side with -ffp-contract=off.
//
//  mt_exp_f32: Cody–Waite reduction x = k ln2 + r (ln2 split into an exactly
//   representable high part and a low part), |r| <= ln2/2, then the degree-7
//   Taylor polynomial of e^r in Horner form, scaled by 2^k. Truncation error
//   r^8/8! < 6e-9 relative; total error a few ulp.
//  mt_erf_f32: Abramowitz & Stegun, Handbook of Mathematical Functions,
//   formula 7.1.26 (Hastings' rational approximation), |error| <= 1.5e-7,
//   odd extension for x < 0.
#pragma once
#include <math.h>

#if defined(__CUDACC__)
#define MT_HD __host__ __device__ __forceinline__
#else
#define MT_HD static inline
#endif

// Plain products and sums that must not be fused into an FMA by the compiler.
#if defined(__CUDA_ARCH__)
#define MT_MUL(a, b) __fmul_rn((a), (b))
#define MT_SUB(a, b) __fsub_rn((a), (b))
#define MT_ADD(a, b) __fadd_rn((a), (b))
#else
#define MT_MUL(a, b) ((a) * (b))
#define MT_SUB(a, b) ((a) - (b))
#define MT_ADD(a, b) ((a) + (b))
#endif

MT_HD float mt_exp_f32(float x) {
  if (x != x) return x;
  if (x > 88.7228394f) return INFINITY;
  if (x < -103.972084f) return 0.0f;
  const float k = rintf(MT_MUL(x, 1.44269504088896341f));
  float r = fmaf(-k, 0.693145751953125f, x);
  r = fmaf(-k, 1.42860682030941723e-06f, r);
  float p = 1.0f / 5040.0f;
  p = fmaf(p, r, 1.0f / 720.0f);
  p = fmaf(p, r, 1.0f / 120.0f);
  p = fmaf(p, r, 1.0f / 24.0f);
  p = fmaf(p, r, 1.0f / 6.0f);
  p = fmaf(p, r, 0.5f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  return ldexpf(p, (int)k);
}

MT_HD float mt_erf_f32(float x) {
  const float ax = fabsf(x);
  const float t = 1.0f / fmaf(0.3275911f, ax, 1.0f);
  float poly = 1.061405429f;
  poly = fmaf(poly, t, -1.453152027f);
  poly = fmaf(poly, t, 1.421413741f);
  poly = fmaf(poly, t, -0.284496736f);
  poly = fmaf(poly, t, 0.254829592f);
  poly = MT_MUL(poly, t);
  const float e = mt_exp_f32(-MT_MUL(ax, ax));
  const float y = MT_SUB(1.0f, MT_MUL(poly, e));
  return x < 0.0f ? -y : y;
}

// mlx.nn.gelu: x * (1 + erf(x / sqrt(2))) / 2
MT_HD float mt_gelu_f32(float x) {
  const float u = MT_ADD(1.0f, mt_erf_f32(x / 1.41421356237309505f));
  return MT_MUL(x, u) / 2.0f;
}
