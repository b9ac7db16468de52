// GELU for 16-bit tensors and the fused GeGLU epilogue, shared by the GEMM,
// elementwise and GeGLU kernels.
#pragma once
#include "lc_sm100.cuh"

using sm100::add2;
using sm100::fma2;
using sm100::mul2;

// GELU, 0.5·x·(1 + erf(x/√2)), used where the result is stored in f16 / bf16 (the fused
// encoder's GeGLU epilogue, gelu and geglu on 16-bit tensors; f32 and f64 keep
// the library erf) — packages/backend-webgpu/src/kernels.ts:102 likewise
// computes GELU with its own erf approximation, for two values as packed pairs. erf(z) by the
// rational approximation of Abramowitz & Stegun, Handbook of Mathematical
// Functions (1964), eq. 7.1.26 (after C. Hastings):
// erf(z) = 1 − (a1·t + a2·t² + a3·t³ + a4·t⁴ + a5·t⁵)·exp(−z²), t = 1/(1 + p·z),
// z >= 0, |error| <= 1.5e-7, odd extension for z < 0. Two MUFU operations
// (reciprocal, exp2) per value.
__device__ __forceinline__ float2 gelu_as2(float2 x) {
  const float2 z = mul2(x, make_float2(0.7071067811865476f, 0.7071067811865476f));
  const float2 az = make_float2(fabsf(z.x), fabsf(z.y));
  const float2 den = fma2(make_float2(0.3275911f, 0.3275911f), az, make_float2(1.f, 1.f));
  float2 t;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(t.x) : "f"(den.x));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(t.y) : "f"(den.y));
  float2 q = fma2(make_float2(1.061405429f, 1.061405429f), t, make_float2(-1.453152027f, -1.453152027f));
  q = fma2(q, t, make_float2(1.421413741f, 1.421413741f));
  q = fma2(q, t, make_float2(-0.284496736f, -0.284496736f));
  q = fma2(q, t, make_float2(0.254829592f, 0.254829592f));
  q = mul2(q, t);
  const float2 g = mul2(az, mul2(az, make_float2(-1.4426950408889634f, -1.4426950408889634f)));
  float2 e;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e.x) : "f"(g.x));
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e.y) : "f"(g.y));
  const float2 r = fma2(make_float2(-q.x, -q.y), e, make_float2(1.f, 1.f));  // erf(|z|)
  const float2 erf = make_float2(copysignf(r.x, z.x), copysignf(r.y, z.y));
  const float2 h = mul2(x, make_float2(0.5f, 0.5f));
  return fma2(h, erf, h);
}
