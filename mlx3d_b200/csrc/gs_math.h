// Exactly-rounded float32 arithmetic shared by the sm_100a kernels and the CPU
// oracle.
//
// The splatting path has discontinuous cut-offs (radius = ceil(...), tile
// bounds = floor(...), alpha < 1/255, T < 1e-4).  A one-ulp difference between
// two implementations can flip one of them, so every expression whose result
// feeds a cut-off is evaluated here with one IEEE rounding per operation, in
// the same order as the reference's elementwise MLX expressions
// (src/mlx3d/splatting/projection.py:56-146, tiles.py:54-65, rasterize.py:74-87).
//
// * On the device, gs_mul/gs_add/... map to the __f*_rn intrinsics, which the
//   compiler never contracts into FMAs.
// * On the host (oracle, built with -ffp-contract=off and without fast-math),
//   the plain operators give the same IEEE binary32 results.
//
// gs_expf is this project's own exponential (Cody & Waite 1980 range reduction
// followed by the degree-7 Taylor polynomial of e^r on |r| <= ln2/2, evaluated
// with correctly rounded fused multiply-adds).  It is bit-identical on host and
// device because it uses only IEEE-exact primitives (fmaf, rintf, exact
// power-of-two scaling).  Its error against the true exponential is below
// 2 ulp on the whole float range; tests/test_oracle.py checks this.
#pragma once

#include <stdint.h>
#include <string.h>
#include <math.h>

#if defined(__CUDACC__)
#define GS_HD __host__ __device__ __forceinline__
#else
#define GS_HD static inline
#endif

GS_HD float gs_mul(float a, float b) {
#if defined(__CUDA_ARCH__)
  return __fmul_rn(a, b);
#else
  return a * b;
#endif
}
GS_HD float gs_add(float a, float b) {
#if defined(__CUDA_ARCH__)
  return __fadd_rn(a, b);
#else
  return a + b;
#endif
}
GS_HD float gs_sub(float a, float b) {
#if defined(__CUDA_ARCH__)
  return __fsub_rn(a, b);
#else
  return a - b;
#endif
}
GS_HD float gs_div(float a, float b) {
#if defined(__CUDA_ARCH__)
  return __fdiv_rn(a, b);
#else
  return a / b;
#endif
}
GS_HD float gs_sqrt(float a) {
#if defined(__CUDA_ARCH__)
  return __fsqrt_rn(a);
#else
  return sqrtf(a);
#endif
}
GS_HD float gs_fma(float a, float b, float c) {
#if defined(__CUDA_ARCH__)
  return __fmaf_rn(a, b, c);
#else
  return fmaf(a, b, c);
#endif
}
GS_HD float gs_maxf(float a, float b) { return a > b ? a : b; }
GS_HD float gs_minf(float a, float b) { return a < b ? a : b; }

GS_HD float gs_bits_to_float(uint32_t u) {
#if defined(__CUDA_ARCH__)
  return __uint_as_float(u);
#else
  float f;
  memcpy(&f, &u, 4);
  return f;
#endif
}
GS_HD uint32_t gs_float_to_bits(float f) {
#if defined(__CUDA_ARCH__)
  return __float_as_uint(f);
#else
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
#endif
}

// 2^k for -126 <= k <= 127, built from the exponent field (exact).
GS_HD float gs_pow2i(int k) { return gs_bits_to_float((uint32_t)(k + 127) << 23); }

// e^x.  Method: x = n*ln2 + r with n = rint(x*log2(e)) and r reduced with a
// two-part ln2 (Cody & Waite); e^r from its Taylor series to degree 7
// (truncation error < 5e-9 relative for |r| <= 0.347); result scaled by 2^n
// in at most two exact power-of-two steps so sub-normal results round once.
GS_HD float gs_expf(float x) {
  const float kLog2e = 1.44269502162933349609375f;   // nearest float to 1/ln2
  const float kLn2Hi = 0.693147182464599609375f;     // nearest float to ln2
  const float kLn2Lo = -1.904654299957768e-09f;      // ln2 - kLn2Hi
  float n = rintf(gs_mul(x, kLog2e));
  float r = gs_fma(-n, kLn2Hi, x);
  r = gs_fma(-n, kLn2Lo, r);
  // Taylor coefficients 1/k!, k = 7..0.
  float p = 1.98412698412698412e-4f;          // 1/5040
  p = gs_fma(p, r, 1.38888888888888889e-3f);  // 1/720
  p = gs_fma(p, r, 8.33333333333333333e-3f);  // 1/120
  p = gs_fma(p, r, 4.16666666666666667e-2f);  // 1/24
  p = gs_fma(p, r, 1.66666666666666667e-1f);  // 1/6
  p = gs_fma(p, r, 0.5f);
  p = gs_fma(p, r, 1.0f);
  p = gs_fma(p, r, 1.0f);
  // Fast path: n in [-126, 127], one exact power-of-two scaling.
  if (x >= -87.0f && x <= 88.0f) return gs_mul(p, gs_pow2i((int)n));
  if (x != x) return x;                       // NaN
  if (x > 88.72283935546875f) return INFINITY;  // above ln(FLT_MAX)
  if (x < -103.972084045410156f) return 0.0f;  // below ln(smallest denormal / 2)
  int k = (int)n;
  if (k > 127) return gs_mul(gs_mul(p, gs_pow2i(127)), gs_pow2i(k - 127));
  if (k >= -126) return gs_mul(p, gs_pow2i(k));
  // Sub-normal result: scale by 2^(k+64) exactly, then by 2^-64 (one rounding).
  return gs_mul(gs_mul(p, gs_pow2i(k + 64)), gs_pow2i(-64));
}

// e^x for -87 <= x <= 0: the operations of gs_expf's fast path, with n =
// rint(x log2e) taken by the round-to-nearest-even addition of 1.5 * 2^23
// (exact for |x log2e| < 2^22; the sum's low mantissa bits hold n, from
// which 2^n is built with one integer multiply-add) instead of rintf and a
// float-to-int conversion.  Bit-identical to gs_expf on that
// interval (tests/test_oracle.py checks every float in it).
GS_HD float gs_expf_nonpos(float x) {
  const float kLog2e = 1.44269502162933349609375f;
  const float kLn2Hi = 0.693147182464599609375f;
  const float kLn2Lo = -1.904654299957768e-09f;
  const float kShift = 12582912.0f;  // 1.5 * 2^23
  const float s = gs_add(gs_mul(x, kLog2e), kShift);
  const float n = gs_sub(s, kShift);
  const uint32_t sb = gs_float_to_bits(s);  // low mantissa bits hold n
  float r = gs_fma(-n, kLn2Hi, x);
  r = gs_fma(-n, kLn2Lo, r);
  float p = 1.98412698412698412e-4f;
  p = gs_fma(p, r, 1.38888888888888889e-3f);
  p = gs_fma(p, r, 8.33333333333333333e-3f);
  p = gs_fma(p, r, 4.16666666666666667e-2f);
  p = gs_fma(p, r, 1.66666666666666667e-1f);
  p = gs_fma(p, r, 0.5f);
  p = gs_fma(p, r, 1.0f);
  p = gs_fma(p, r, 1.0f);
  // 2^n as a float: its bits (n + 127) << 23 equal sb * 2^23 + 0x3F800000
  // modulo 2^32 (sb = 0x4B400000 + n), one integer multiply-add.
  return gs_mul(p, gs_bits_to_float(sb * 8388608u + 0x3F800000u));
}

// Logistic sigmoid 1 / (1 + e^-x) on top of gs_expf (model activations,
// src/mlx3d/splatting/model.py:120-122).
GS_HD float gs_sigmoidf(float x) { return gs_div(1.0f, gs_add(1.0f, gs_expf(-x))); }

// ---------------------------------------------------------------------------
// Constants of the path.
#define GS_TILE 16
#define GS_BLOCK 256
// 1/255 as a float32 literal, the alpha skip threshold of rasterize.py:81.
#define GS_ALPHA_MIN (1.0f / 255.0f)
#define GS_ALPHA_MAX 0.99f
#define GS_T_MIN 1e-4f
