// Deterministic float arithmetic shared by the CUDA kernels and the C oracle.
//
// Every rounding step is one IEEE-754 binary32 operation (add, sub, mul, div, sqrt, fma) in
// round-to-nearest-even, written as an explicit call so that neither nvcc nor gcc may contract
// or reorder it (the oracle is built with -ffp-contract=off, the kernels use the _rn
// intrinsics). The transcendental functions are this project's own, built only from those
// operations, so the GPU and the CPU restatement produce the same bits:
//
//   exp    Cody & Waite range reduction (x = n ln2 + r, ln2 split in two parts), then the degree-7
//          Taylor polynomial of e^r on |r| <= ln2/2 by Horner with fma, then scaling by 2^n
//          (two steps near the subnormal range, so the result rounds once).
//   log    u = m 2^e with m in [sqrt(1/2), sqrt(2)); log m = 2 atanh(s), s = (m-1)/(m+1), by its
//          odd series to s^11; e ln2 added in two parts.
//   log1p  Goldberg's method (D. Goldberg, "What every computer scientist should know about
//          floating-point arithmetic", 1991, theorem 4): log1p(y) = log(u) * y / (u - 1), u = 1 + y.
//
// The stock model computes these with torch's own exp/log1p (within an ulp or so); the bf16
// roundings that follow almost always absorb that difference, and the parity tests state their
// tolerance for the fp32 recurrent state.
//
// bf16 conversion is round-to-nearest-even on the bit pattern, as torch's float -> bfloat16
// (a NaN becomes the canonical bf16 NaN 0x7fff, where torch writes 0x7fc0).
#pragma once
#include <stdint.h>

#ifdef __CUDACC__
#define LXB_FN __host__ __device__ __forceinline__
#else
#define LXB_FN static inline
#include <math.h>
#include <string.h>
#endif

typedef uint16_t lxb_bf16;

LXB_FN uint32_t lxb_fbits(float x) {
#ifdef __CUDA_ARCH__
  return __float_as_uint(x);
#else
  uint32_t u;
  memcpy(&u, &x, 4);
  return u;
#endif
}
LXB_FN float lxb_bitsf(uint32_t u) {
#ifdef __CUDA_ARCH__
  return __uint_as_float(u);
#else
  float x;
  memcpy(&x, &u, 4);
  return x;
#endif
}

// --- one rounding each --------------------------------------------------------------------------
#ifdef __CUDA_ARCH__
LXB_FN float lx_add(float a, float b) { return __fadd_rn(a, b); }
LXB_FN float lx_sub(float a, float b) { return __fsub_rn(a, b); }
LXB_FN float lx_mul(float a, float b) { return __fmul_rn(a, b); }
LXB_FN float lx_div(float a, float b) { return __fdiv_rn(a, b); }
LXB_FN float lx_fma(float a, float b, float c) { return __fmaf_rn(a, b, c); }
LXB_FN float lx_sqrt(float a) { return __fsqrt_rn(a); }
#else
LXB_FN float lx_add(float a, float b) { return a + b; }
LXB_FN float lx_sub(float a, float b) { return a - b; }
LXB_FN float lx_mul(float a, float b) { return a * b; }
LXB_FN float lx_div(float a, float b) { return a / b; }
LXB_FN float lx_fma(float a, float b, float c) { return fmaf(a, b, c); }
LXB_FN float lx_sqrt(float a) { return sqrtf(a); }
#endif

// --- bf16 ---------------------------------------------------------------------------------------
LXB_FN float lx_f(lxb_bf16 b) { return lxb_bitsf(((uint32_t)b) << 16); }
// On the device this is the hardware conversion (cvt.rn.bf16.f32): the same bits as the form
// below for every non-NaN float (all 2^32 inputs checked on the B200), and 0x7fff for every NaN,
// which the form below returns too (a NaN never arises from a valid machine state).
LXB_FN lxb_bf16 lx_rb(float x) {
#ifdef __CUDA_ARCH__
  uint16_t r;
  asm("cvt.rn.bf16.f32 %0, %1;" : "=h"(r) : "f"(x));
  return r;
#else
  uint32_t u = lxb_fbits(x);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (lxb_bf16)0x7fffu;  // NaN: the canonical bf16 NaN
  u += 0x7fffu + ((u >> 16) & 1u);
  return (lxb_bf16)(u >> 16);
#endif
}
LXB_FN float lx_rbf(float x) { return lx_f(lx_rb(x)); }

// --- exp, log, log1p --------------------------------------------------------------------------
#define LXB_INF lxb_bitsf(0x7f800000u)

LXB_FN float lx_pow2i(int n) { return lxb_bitsf((uint32_t)(n + 127) << 23); }  // -126 <= n <= 127

LXB_FN float lx_exp(float x) {
  if (x != x) return x;
  if (x > 88.72283935546875f) return LXB_INF;
  if (x < -103.97208404541015625f) return 0.0f;
  // n = round(x / ln2): the 1.5 * 2^23 trick rounds to nearest even for |t| < 2^22
  const float t = lx_mul(x, 1.44269502162933349609375f);
  const float n = lx_sub(lx_add(t, 12582912.0f), 12582912.0f);
  // r = x - n ln2, ln2 = 0.693145751953125 + 1.428606765330187e-06 (the first part exact in
  // 16 bits, so n * hi is exact and the first fma exact)
  float r = lx_fma(-n, 0.693145751953125f, x);
  r = lx_fma(-n, 1.428606765330187e-06f, r);
  float p = 1.9841269841e-4f;                 // 1/5040
  p = lx_fma(p, r, 1.3888888889e-3f);         // 1/720
  p = lx_fma(p, r, 8.3333333333e-3f);         // 1/120
  p = lx_fma(p, r, 4.1666666667e-2f);         // 1/24
  p = lx_fma(p, r, 1.6666666667e-1f);         // 1/6
  p = lx_fma(p, r, 0.5f);
  p = lx_fma(p, r, 1.0f);
  p = lx_fma(p, r, 1.0f);
  const int ni = (int)n;
  if (ni > 127) return lx_mul(lx_mul(p, lx_pow2i(127)), lx_pow2i(ni - 127));
  if (ni < -126) return lx_mul(lx_mul(p, lx_pow2i(-64)), lx_pow2i(ni + 64));
  return lx_mul(p, lx_pow2i(ni));
}

// natural log for finite x > 0 (x = 0 -> -inf, inf -> inf, negative/NaN -> NaN)
LXB_FN float lx_log(float x) {
  if (x != x || x < 0.0f) return lxb_bitsf(0x7fc00000u);
  if (x == 0.0f) return -LXB_INF;
  if (x == LXB_INF) return x;
  int e = 0;
  if (x < 1.17549435e-38f) {  // subnormal: scale into the normal range first
    x = lx_mul(x, 16777216.0f);
    e = -24;
  }
  uint32_t u = lxb_fbits(x);
  e += (int)((u >> 23) & 0xff) - 127;
  float m = lxb_bitsf((u & 0x007fffffu) | 0x3f800000u);  // [1, 2)
  if (m > 1.41421353816986083984375f) {
    m = lx_mul(m, 0.5f);
    e += 1;
  }
  const float f = lx_sub(m, 1.0f);
  const float s = lx_div(f, lx_add(2.0f, f));
  const float s2 = lx_mul(s, s);
  float q = 0.0909090909f;               // 1/11
  q = lx_fma(q, s2, 0.1111111111f);      // 1/9
  q = lx_fma(q, s2, 0.1428571429f);      // 1/7
  q = lx_fma(q, s2, 0.2f);
  q = lx_fma(q, s2, 0.3333333333f);
  // log m = 2s + 2s * s2 * q
  const float two_s = lx_add(s, s);
  const float lm = lx_fma(lx_mul(two_s, s2), q, two_s);
  const float fe = (float)e;
  return lx_add(lx_fma(fe, 0.693145751953125f, 0.0f), lx_fma(fe, 1.428606765330187e-06f, lm));
}

LXB_FN float lx_log1p(float y) {
  if (y != y) return y;
  const float u = lx_add(1.0f, y);
  if (u == 1.0f) return y;
  if (u == LXB_INF) return u;
  return lx_mul(lx_log(u), lx_div(y, lx_sub(u, 1.0f)));
}

// --- the stock model's elementwise functions, fp32 in and out ----------------------------------
// torch: silu(x) = x / (1 + exp(-x)); sigmoid(x) = 1 / (1 + exp(-x)); softplus (beta 1,
// threshold 20) = x > 20 ? x : log1p(exp(x)); rsqrt(x) = 1 / sqrt(x).
LXB_FN float lx_silu(float x) { return lx_div(x, lx_add(1.0f, lx_exp(-x))); }
LXB_FN float lx_sigmoid(float x) { return lx_div(1.0f, lx_add(1.0f, lx_exp(-x))); }
LXB_FN float lx_softplus(float x) { return x > 20.0f ? x : lx_log1p(lx_exp(x)); }
LXB_FN float lx_rsqrt(float x) { return lx_div(1.0f, lx_sqrt(x)); }
