// Packed two-lane float32 arithmetic (sm_100: one fma/mul/add instruction on a register pair).
//
// The scans keep each thread's states as pairs and step both with one instruction; every lane is
// an ordinary round-to-nearest float32 operation, so a packed op gives the same bits as the two
// scalar ones.
#pragma once
#include "common.cuh"

namespace pgf {

__device__ __forceinline__ float2 f2(float v) { return make_float2(v, v); }
__device__ __forceinline__ float2 f2(float x, float y) { return make_float2(x, y); }
__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 add2(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float2 exp2_2(float2 x) { return make_float2(exp2f(x.x), exp2f(x.y)); }
__device__ __forceinline__ float hsum2(float2 a) { return a.x + a.y; }
__device__ __forceinline__ float2 lo2(float4 v) { return make_float2(v.x, v.y); }
__device__ __forceinline__ float2 hi2(float4 v) { return make_float2(v.z, v.w); }

__device__ __forceinline__ float2 ex2_2(float2 x) { return make_float2(ex2f(x.x), ex2f(x.y)); }
// The same, never merged with an equal expression elsewhere: a kernel that re-derives a value instead
// of keeping it live in registers uses this so that the compiler cannot reuse the earlier result.
__device__ __forceinline__ float ex2f_fresh(float x) {
  float y;
  asm volatile("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float2 ex2_2_fresh(float2 x) { return make_float2(ex2f_fresh(x.x), ex2f_fresh(x.y)); }

// phi_1(z) = (e^z - 1)/z and phi_1'(z) = (e^z - phi_1(z))/z given e = e^z and rz = 1/z.
// |z| < 1/8: Taylor series to z^4 (truncation < 5e-8); elsewhere the closed forms.  With e accurate
// to 2 ulp the worst relative error is ~1.1e-6 for phi_1 and ~5.4e-6 for phi_1' (at the switch).
// Both forms are evaluated, then one is selected (cheaper than a divergent branch).  The series run
// as scalar FMAs so that their coefficients stay immediate operands instead of register pairs.
__device__ __forceinline__ float phi1_s(float z) {
  float p = fmaf(z, 1.0f / 120.0f, 1.0f / 24.0f);
  p = fmaf(p, z, 1.0f / 6.0f);
  p = fmaf(p, z, 0.5f);
  return fmaf(p, z, 1.0f);
}
__device__ __forceinline__ float phi1p_s(float z) {
  float p = fmaf(z, 5.0f / 720.0f, 4.0f / 120.0f);
  p = fmaf(p, z, 3.0f / 24.0f);
  p = fmaf(p, z, 2.0f / 6.0f);
  return fmaf(p, z, 0.5f);
}
__device__ __forceinline__ float pick(float z, float series, float closed) {
  return fabsf(z) < 0.125f ? series : closed;
}
__device__ __forceinline__ float phi1(float z, float e, float rz) {
  const float p = phi1_s(z), c = (e - 1.0f) * rz;
  return pick(z, p, c);
}
__device__ __forceinline__ float phi1p(float z, float e, float p1, float rz) {
  const float p = phi1p_s(z), c = (e - p1) * rz;
  return pick(z, p, c);
}
__device__ __forceinline__ float2 phi1_2(float2 z, float2 e, float2 rz) {
  const float2 p = f2(phi1_s(z.x), phi1_s(z.y));
  const float2 c = mul2(add2(e, f2(-1.0f)), rz);
  return f2(pick(z.x, p.x, c.x), pick(z.y, p.y, c.y));
}
__device__ __forceinline__ float2 phi1p_2(float2 z, float2 e, float2 p1, float2 rz) {
  const float2 p = f2(phi1p_s(z.x), phi1p_s(z.y));
  const float2 c = mul2(fma2(p1, f2(-1.0f), e), rz);
  return f2(pick(z.x, p.x, c.x), pick(z.y, p.y, c.y));
}

}  // namespace pgf
