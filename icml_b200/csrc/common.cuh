// Shared helpers for the PGF sm_100a kernels: error reporting through the C-ABI,
// dtype access, and the scalar math of the PGF recurrence.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdio.h>
#include <stdarg.h>

#include "../../include/pgf.h"

namespace pgf {

// ---------------------------------------------------------------------------
// Error handling: every entry point returns 0 or a PGF_ERR_* code and leaves a
// message readable through pgf_last_error() (thread-local).
// ---------------------------------------------------------------------------
void set_error(const char* fmt, ...);
void clear_error();

#define PGF_CHECK_ARG(cond, ...)                     \
  do {                                               \
    if (!(cond)) {                                   \
      ::pgf::set_error(__VA_ARGS__);                 \
      return PGF_ERR_INVALID;                        \
    }                                                \
  } while (0)

#define PGF_CUDA(call)                                                        \
  do {                                                                        \
    cudaError_t e_ = (call);                                                  \
    if (e_ != cudaSuccess) {                                                  \
      ::pgf::set_error("%s:%d %s: %s", __FILE__, __LINE__, #call,             \
                       cudaGetErrorString(e_));                               \
      return PGF_ERR_CUDA;                                                    \
    }                                                                         \
  } while (0)

// Kernel-launch accounting and optional CUDA-event timing of selected kernels (abi.cu).
enum ProfId {
  PROF_SSM_CHUNK_FWD = 0, PROF_SSM_COMPOSE, PROF_SSM_OUT_FWD, PROF_SSM_CHUNK_BWD, PROF_SSM_MAIN_BWD,
  PROF_GEMM_TC, PROF_GEMM_SIMT, PROF_RMSNORM_FWD, PROF_RMSNORM_BWD, PROF_EMBEDDING, PROF_CE, PROF_OPTIM,
  PROF_COUNT
};
void count_launch();
void prof_begin(int id, cudaStream_t s);
// `work`: algorithmic FLOPs (dense products) or bytes (bandwidth kernels) of the launch
void prof_end(int id, cudaStream_t s, double work);

#define PGF_LAUNCH_CHECK()                                                    \
  do {                                                                        \
    ::pgf::count_launch();                                                    \
    cudaError_t e_ = cudaGetLastError();                                      \
    if (e_ != cudaSuccess) {                                                  \
      ::pgf::set_error("%s:%d kernel launch: %s", __FILE__, __LINE__,         \
                       cudaGetErrorString(e_));                               \
      return PGF_ERR_CUDA;                                                    \
    }                                                                         \
  } while (0)

#define PGF_TRY(expr)            \
  do {                           \
    int rc_ = (expr);            \
    if (rc_ != PGF_OK) return rc_; \
  } while (0)

static inline cudaStream_t as_stream(pgf_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

static inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Raises `kernel`'s dynamic shared-memory limit to `bytes` the first time a launch needs more than
// the limit already set through `limit` (one per kernel, per process; the default limit is 48 KB
// minus the kernel's static shared memory, so any size is set once).  Calls that need no more
// touch nothing, so launches inside a CUDA-graph capture make no runtime calls beyond the launch.
template <class Kernel>
static inline cudaError_t ensure_dynamic_smem(Kernel kernel, size_t bytes, int& limit) {
  if (int(bytes) <= limit) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(bytes));
  if (e == cudaSuccess) limit = int(bytes);
  return e;
}

// Bump allocator over a caller-provided workspace.  Keeps every sub-buffer 256-byte aligned.
struct Workspace {
  char* base;
  size_t cap;
  size_t used;
  Workspace(void* p, size_t n) : base(static_cast<char*>(p)), cap(n), used(0) {}
  template <class T>
  T* take(size_t count) {
    size_t off = (used + 255) & ~size_t(255);
    size_t bytes = count * sizeof(T);
    if (off + bytes > cap) return nullptr;
    used = off + bytes;
    return reinterpret_cast<T*>(base + off);
  }
  static size_t round(size_t bytes) { return (bytes + 255) & ~size_t(255); }
};

// ---------------------------------------------------------------------------
// dtype access
// ---------------------------------------------------------------------------
__device__ __forceinline__ float ld(const float* p, int64_t i) { return p[i]; }
__device__ __forceinline__ float ld(const __nv_bfloat16* p, int64_t i) { return __bfloat162float(p[i]); }
__device__ __forceinline__ void st(float* p, int64_t i, float v) { p[i] = v; }
__device__ __forceinline__ void st(__nv_bfloat16* p, int64_t i, float v) { p[i] = __float2bfloat16_rn(v); }
// v as it reads back after a store to a T (bf16: rounded to nearest even; float: unchanged)
template <class T> __device__ __forceinline__ float rounded(float v);
template <> __device__ __forceinline__ float rounded<float>(float v) { return v; }
template <> __device__ __forceinline__ float rounded<__nv_bfloat16>(float v) {
  return __bfloat162float(__float2bfloat16_rn(v));
}

__device__ __forceinline__ float ldv(const void* p, int bf16, int64_t i) {
  return bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i])
              : reinterpret_cast<const float*>(p)[i];
}
__device__ __forceinline__ void stv(void* p, int bf16, int64_t i, float v) {
  if (bf16) reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else reinterpret_cast<float*>(p)[i] = v;
}

// ---------------------------------------------------------------------------
// Scalar math of the recurrence (train_singlemamba_optimized.py:13-27, 140-144;
// pgf_ffn.py:16-26).  phi_1 and phi_1' use their Taylor series near 0, which is
// accurate where the closed forms cancel; elsewhere the closed forms with the
// CUDA math library's expf.
// ---------------------------------------------------------------------------

// phi_1(z) = (e^z - 1)/z given e = e^z.
// Series: sum_{k>=0} z^k/(k+1)!, truncated after z^7 for |z| < 1/4 (error < 5e-11).
__device__ __forceinline__ float phi1_from_exp(float z, float e) {
  if (fabsf(z) < 0.25f) {
    float p = 1.0f / 40320.0f;
    p = fmaf(p, z, 1.0f / 5040.0f);
    p = fmaf(p, z, 1.0f / 720.0f);
    p = fmaf(p, z, 1.0f / 120.0f);
    p = fmaf(p, z, 1.0f / 24.0f);
    p = fmaf(p, z, 1.0f / 6.0f);
    p = fmaf(p, z, 0.5f);
    return fmaf(p, z, 1.0f);
  }
  return (e - 1.0f) / z;
}

// phi_1'(z) = ((z-1)e^z + 1)/z^2 given e = e^z.
// Series: sum_{k>=1} k z^(k-1)/(k+1)!, truncated after z^8 for |z| < 1/2 (error < 5e-10).
__device__ __forceinline__ float phi1p_from_exp(float z, float e) {
  if (fabsf(z) < 0.5f) {
    float p = 9.0f / 3628800.0f;
    p = fmaf(p, z, 8.0f / 362880.0f);
    p = fmaf(p, z, 7.0f / 40320.0f);
    p = fmaf(p, z, 6.0f / 5040.0f);
    p = fmaf(p, z, 5.0f / 720.0f);
    p = fmaf(p, z, 4.0f / 120.0f);
    p = fmaf(p, z, 3.0f / 24.0f);
    p = fmaf(p, z, 2.0f / 6.0f);
    return fmaf(p, z, 0.5f);
  }
  return fmaf(z - 1.0f, e, 1.0f) / (z * z);
}

// torch.nn.functional.softplus with beta=1, threshold=20.
__device__ __forceinline__ float softplus_f(float x) { return x > 20.0f ? x : log1pf(expf(x)); }

// 2^x by the hardware approximation (ex2.approx.ftz: ~2 ulp; results below 2^-126 flush to zero,
// which for the decays exp(dt A) <= 1 of the scans changes nothing that is added to a state).
__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// 1/x by the hardware approximation (rcp.approx.ftz: <= 1 ulp; denormal inputs count as zero).
__device__ __forceinline__ float rcpf(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// softplus(x) = max(x, 0) + log1p(y), y = exp(-|x|) in (0, 1], branch-free:
//   y = 2^t (1 + r ln 2) with t = -|x| log2(e) rounded and r its rounding residual (two FMAs: the
//   product's error and the tail of log2(e)), so the exponent's rounding does not grow with |x|;
//   log1p(y) = 2 atanh(s), s = y / (2 + y) <= 1/3, by its odd series to s^13.
// Relative error <= 2.8e-7 with an exact 2^t and <= 5.4e-7 with the 2-ulp hardware ex2, over
// x in [-87, 100] (below -87.3 the result flushes to zero).  About 20 instructions, where
// log1pf(expf(x)) takes several times that with branches.  The scans derive dt = softplus(dt_in)
// with it for every (token, channel) they stage.
__device__ __forceinline__ float exp_neg_abs(float x) {
  constexpr float L2E = 1.4426950408889634f, L2E_LO = 1.925963033500011e-08f, LN2 = 0.6931471805599453f;
  const float na = -fabsf(x);
  const float t = na * L2E;
  float r = fmaf(na, L2E, -t);
  r = fmaf(na, L2E_LO, r);
  const float y0 = ex2f(t);
  return fmaf(y0, r * LN2, y0);
}
__device__ __forceinline__ float softplus_from(float x, float y) {
  const float s = y * rcpf(2.0f + y);
  const float s2 = s * s;
  float p = fmaf(s2, 1.0f / 13.0f, 1.0f / 11.0f);
  p = fmaf(p, s2, 1.0f / 9.0f);
  p = fmaf(p, s2, 1.0f / 7.0f);
  p = fmaf(p, s2, 1.0f / 5.0f);
  p = fmaf(p, s2, 1.0f / 3.0f);
  p = fmaf(p, s2, 1.0f);
  return fmaxf(x, 0.0f) + 2.0f * s * p;
}
__device__ __forceinline__ float softplus_fast(float x) { return softplus_from(x, exp_neg_abs(x)); }
// sigmoid(x) from the same y = exp(-|x|): 1/(1+y) for x >= 0, y/(1+y) otherwise (~3 ulp).
__device__ __forceinline__ float sigmoid_from(float x, float y) { return (x >= 0.0f ? 1.0f : y) * rcpf(1.0f + y); }
__device__ __forceinline__ float sigmoid_f(float x) { return 1.0f / (1.0f + expf(-x)); }

// tanh-approximated GELU and its derivative, constants of pgf_ffn.py:16-26.
#define PGF_GELU_C 0.7978845608f
#define PGF_GELU_A 0.044715f
__device__ __forceinline__ float gelu_f(float x) {
  return 0.5f * x * (1.0f + tanhf(PGF_GELU_C * (x + PGF_GELU_A * x * x * x)));
}
__device__ __forceinline__ float gelu_prime_f(float x) {
  float t = tanhf(PGF_GELU_C * (x + PGF_GELU_A * x * x * x));
  float sech2 = 1.0f - t * t;
  return 0.5f * (1.0f + t) + 0.5f * x * sech2 * (PGF_GELU_C * (1.0f + 3.0f * PGF_GELU_A * x * x));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

static inline int ceil_div(int64_t a, int64_t b) { return int((a + b - 1) / b); }

}  // namespace pgf
