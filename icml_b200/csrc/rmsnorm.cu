// RMSNorm forward / backward (pgf_rmsnorm.py:10-51).
//
// One warp per row; the row lives in registers (VPL values per lane, columns lane + 32*j), so x
// and g are read once.  grad_weight is reduced deterministically: each CTA sums its warps'
// register partials through shared memory in warp order and writes one partial row; a second
// kernel adds the CTA partials in CTA order.
#include "gemm.cuh"

namespace pgf {

constexpr int RMS_WARPS = 8;
constexpr int RMS_ROWS_PER_WARP = 4;  // rows handled by a warp in the backward (one CTA = 32 rows)

template <int VPL, class T>
__global__ void __launch_bounds__(RMS_WARPS * 32)
rmsnorm_fwd_kernel(const T* __restrict__ x, const float* __restrict__ w, T* __restrict__ y,
                   int64_t rows, int dim, float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t row = int64_t(blockIdx.x) * RMS_WARPS + (threadIdx.x >> 5);
  if (row >= rows) return;
  const T* xr = x + row * dim;
  float v[VPL];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    int c = j * 32 + lane;
    v[j] = c < dim ? ld(xr, c) : 0.f;
    ss = fmaf(v[j], v[j], ss);
  }
  ss = warp_sum(ss);
  const float rms = sqrtf(ss / float(dim) + eps);
  T* yr = y + row * dim;
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    int c = j * 32 + lane;
    if (c < dim) st(yr, c, (v[j] / rms) * w[c]);
  }
}

template <int VPL, class T>
__global__ void __launch_bounds__(RMS_WARPS * 32)
rmsnorm_bwd_kernel(const T* __restrict__ x, const T* __restrict__ g, const float* __restrict__ w,
                   T* __restrict__ gx, float* __restrict__ gw_part, int64_t rows, int dim,
                   float eps) {
  extern __shared__ float sm_gw[];  // [RMS_WARPS][dim]
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  float acc[VPL];
#pragma unroll
  for (int j = 0; j < VPL; ++j) acc[j] = 0.f;
  float wv[VPL];
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    int c = j * 32 + lane;
    wv[j] = c < dim ? w[c] : 0.f;
  }
  const int64_t row0 = (int64_t(blockIdx.x) * RMS_WARPS + warp) * RMS_ROWS_PER_WARP;
  for (int r = 0; r < RMS_ROWS_PER_WARP; ++r) {
    const int64_t row = row0 + r;
    if (row >= rows) break;
    const T* xr = x + row * dim;
    const T* gr = g + row * dim;
    float xv[VPL], gv[VPL];
    float ss = 0.f, dot = 0.f;
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      int c = j * 32 + lane;
      xv[j] = c < dim ? ld(xr, c) : 0.f;
      gv[j] = c < dim ? ld(gr, c) : 0.f;
      ss = fmaf(xv[j], xv[j], ss);
      dot = fmaf(gv[j] * wv[j], xv[j], dot);
    }
    ss = warp_sum(ss);
    dot = warp_sum(dot);
    const float rms = sqrtf(ss / float(dim) + eps);
    const float rinv = 1.0f / rms;
    const float r3 = rinv * rinv * rinv;
    if (gx) {
      T* gxr = gx + row * dim;
#pragma unroll
      for (int j = 0; j < VPL; ++j) {
        int c = j * 32 + lane;
        if (c < dim) st(gxr, c, (gv[j] * wv[j]) * rinv - (xv[j] * dot) * r3 / float(dim));
      }
    }
#pragma unroll
    for (int j = 0; j < VPL; ++j) acc[j] = fmaf(gv[j], xv[j] * rinv, acc[j]);
  }
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    int c = j * 32 + lane;
    if (c < dim) sm_gw[warp * dim + c] = acc[j];
  }
  __syncthreads();
  for (int c = threadIdx.x; c < dim; c += blockDim.x) {
    float s = 0.f;
    for (int k = 0; k < RMS_WARPS; ++k) s += sm_gw[k * dim + c];
    gw_part[int64_t(blockIdx.x) * dim + c] = s;
  }
}

template <class T>
static int rms_fwd_dispatch(const T* x, const float* w, T* y, int64_t rows, int dim, float eps,
                            cudaStream_t s) {
  dim3 grid(ceil_div(rows, RMS_WARPS)), block(RMS_WARPS * 32);
  int vpl = ceil_div(dim, 32);
#define PGF_RMS_F(V)                                                                  \
  do {                                                                                \
    prof_begin(PROF_RMSNORM_FWD, s);                                                  \
    rmsnorm_fwd_kernel<V, T><<<grid, block, 0, s>>>(x, w, y, rows, dim, eps);         \
    prof_end(PROF_RMSNORM_FWD, s, double(rows) * dim * 2.0 * sizeof(T) + dim * 4.0);    \
  } while (0)
  if (vpl <= 1) PGF_RMS_F(1);
  else if (vpl <= 2) PGF_RMS_F(2);
  else if (vpl <= 4) PGF_RMS_F(4);
  else if (vpl <= 8) PGF_RMS_F(8);
  else if (vpl <= 16) PGF_RMS_F(16);
  else if (vpl <= 32) PGF_RMS_F(32);
  else if (vpl <= 64) PGF_RMS_F(64);
  else if (vpl <= 128) PGF_RMS_F(128);
  else { set_error("rmsnorm: dim %d > 4096 unsupported", dim); return PGF_ERR_UNSUPPORTED; }
#undef PGF_RMS_F
  PGF_LAUNCH_CHECK();
  return PGF_OK;
}

static int64_t rms_bwd_ctas(int64_t rows) { return ceil_div(rows, RMS_WARPS * RMS_ROWS_PER_WARP); }

template <class T>
static int rms_bwd_dispatch(const T* x, const T* g, const float* w, T* gx, float* gw, int acc,
                            int64_t rows, int dim, float eps, float* part, cudaStream_t s) {
  int64_t nct = rms_bwd_ctas(rows);
  dim3 grid((unsigned)nct), block(RMS_WARPS * 32);
  size_t smem = size_t(RMS_WARPS) * dim * sizeof(float);
  int vpl = ceil_div(dim, 32);
#define PGF_RMS_B(V)                                                                           \
  do {                                                                                         \
    static int smem_limit_##V = 0;                                                             \
    PGF_CUDA(ensure_dynamic_smem(rmsnorm_bwd_kernel<V, T>, smem, smem_limit_##V));             \
    prof_begin(PROF_RMSNORM_BWD, s);                                                           \
    rmsnorm_bwd_kernel<V, T><<<grid, block, smem, s>>>(x, g, w, gx, part, rows, dim, eps);     \
    prof_end(PROF_RMSNORM_BWD, s, double(rows) * dim * 3.0 * sizeof(T) + dim * 4.0);           \
  } while (0)
  if (vpl <= 1) PGF_RMS_B(1);
  else if (vpl <= 2) PGF_RMS_B(2);
  else if (vpl <= 4) PGF_RMS_B(4);
  else if (vpl <= 8) PGF_RMS_B(8);
  else if (vpl <= 16) PGF_RMS_B(16);
  else if (vpl <= 32) PGF_RMS_B(32);
  else if (vpl <= 64) PGF_RMS_B(64);
  else if (vpl <= 128) PGF_RMS_B(128);
  else { set_error("rmsnorm: dim %d > 4096 unsupported", dim); return PGF_ERR_UNSUPPORTED; }
#undef PGF_RMS_B
  PGF_LAUNCH_CHECK();
  PGF_TRY(column_reduce(part, nct, dim, gw, acc, s));
  return PGF_OK;
}

}  // namespace pgf

using namespace pgf;

extern "C" int pgf_rmsnorm_fwd(const void* x, const float* weight, void* y, int64_t rows,
                               int64_t dim, float eps, int dtype, pgf_stream_t stream) {
  PGF_CHECK_ARG(rows >= 0 && dim > 0 && dim <= 4096, "rmsnorm_fwd: bad shape rows=%lld dim=%lld",
                (long long)rows, (long long)dim);
  if (rows == 0) return PGF_OK;
  PGF_CHECK_ARG(x && weight && y, "rmsnorm_fwd: null pointer");
  cudaStream_t s = as_stream(stream);
  if (dtype == PGF_DTYPE_F32)
    return rms_fwd_dispatch((const float*)x, weight, (float*)y, rows, int(dim), eps, s);
  if (dtype == PGF_DTYPE_BF16)
    return rms_fwd_dispatch((const __nv_bfloat16*)x, weight, (__nv_bfloat16*)y, rows, int(dim),
                            eps, s);
  set_error("rmsnorm_fwd: bad dtype %d", dtype);
  return PGF_ERR_INVALID;
}

extern "C" size_t pgf_rmsnorm_bwd_workspace(int64_t rows, int64_t dim) {
  return Workspace::round(size_t(rms_bwd_ctas(rows < 1 ? 1 : rows)) * size_t(dim) * sizeof(float));
}

extern "C" int pgf_rmsnorm_bwd(const void* x, const void* g, const float* weight, void* grad_x,
                               float* grad_weight, int accumulate, int64_t rows, int64_t dim,
                               float eps, int dtype, void* ws, size_t ws_bytes,
                               pgf_stream_t stream) {
  PGF_CHECK_ARG(weight && grad_weight, "rmsnorm_bwd: null pointer");
  PGF_CHECK_ARG(rows >= 0 && dim > 0 && dim <= 4096, "rmsnorm_bwd: bad shape");
  cudaStream_t s = as_stream(stream);
  if (rows > 0) PGF_CHECK_ARG(x && g, "rmsnorm_bwd: null pointer");
  if (rows == 0) {
    if (!accumulate) PGF_CUDA(cudaMemsetAsync(grad_weight, 0, dim * sizeof(float), s));
    return PGF_OK;
  }
  Workspace W(ws, ws_bytes);
  float* part = W.take<float>(size_t(rms_bwd_ctas(rows)) * dim);
  if (!part) { set_error("rmsnorm_bwd: workspace too small (%zu)", ws_bytes); return PGF_ERR_WORKSPACE; }
  if (dtype == PGF_DTYPE_F32)
    return rms_bwd_dispatch((const float*)x, (const float*)g, weight, (float*)grad_x, grad_weight,
                            accumulate, rows, int(dim), eps, part, s);
  if (dtype == PGF_DTYPE_BF16)
    return rms_bwd_dispatch((const __nv_bfloat16*)x, (const __nv_bfloat16*)g, weight,
                            (__nv_bfloat16*)grad_x, grad_weight, accumulate, rows, int(dim), eps,
                            part, s);
  set_error("rmsnorm_bwd: bad dtype %d", dtype);
  return PGF_ERR_INVALID;
}

// ---------------------------------------------------------------------------------------------
// RMSNorm backward without a caller workspace.
//
// For callers that cannot call cudaMalloc: a plugin inside an engine that plans and owns all
// device memory and forbids allocation from its operators, or a latency-critical loop that must
// not enter the allocator.  The grad-weight partials live in the file-scope array below instead
// of a workspace: NOALLOC_RMS_FLOATS floats (4 MiB), held by every GPU that loads this library
// until the process exits.  A call needs ceil(rows / 32) * dim of them.
//
// The host cannot pass the array's name to a kernel (in host code it is only a stand-in for the
// device symbol): the first call on each device, with that device current, looks up the device
// address with cudaGetSymbolAddress and caches it.  Make that first call before any stream
// capture.  Every call overwrites all the partial slots it reads, so nothing needs clearing, but
// the calls share the one array: calls that overlap on the GPU (other streams, other threads)
// race on it and must be serialised by the caller.
// ---------------------------------------------------------------------------------------------
#include <mutex>

namespace pgf {

constexpr size_t NOALLOC_RMS_FLOATS = size_t(1) << 20;
static __device__ __align__(256) float g_rms_noalloc_scratch[NOALLOC_RMS_FLOATS];

constexpr int NOALLOC_MAX_DEVICES = 64;
static std::mutex g_noalloc_mu;
static float* g_noalloc_ptr[NOALLOC_MAX_DEVICES] = {};

// Device address of the scratch array on the current device (looked up once per device).
static int noalloc_scratch(float** out) {
  int dev = 0;
  PGF_CUDA(cudaGetDevice(&dev));
  PGF_CHECK_ARG(dev >= 0 && dev < NOALLOC_MAX_DEVICES, "rmsnorm_bwd_noalloc: device %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_rms_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      set_error("rmsnorm_bwd_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
      return PGF_ERR_CUDA;
    }
    g_noalloc_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_noalloc_ptr[dev];
  return PGF_OK;
}

}  // namespace pgf

extern "C" int pgf_rmsnorm_bwd_noalloc(const void* x, const void* g, const float* weight, void* grad_x,
                                       float* grad_weight, int accumulate, int64_t rows, int64_t dim,
                                       float eps, int dtype, pgf_stream_t stream) {
  PGF_CHECK_ARG(weight && grad_weight, "rmsnorm_bwd_noalloc: null pointer");
  PGF_CHECK_ARG(rows >= 0 && dim > 0 && dim <= 4096, "rmsnorm_bwd_noalloc: bad shape");
  const size_t need = size_t(rms_bwd_ctas(rows < 1 ? 1 : rows)) * size_t(dim);
  PGF_CHECK_ARG(need <= NOALLOC_RMS_FLOATS,
                "rmsnorm_bwd_noalloc: ceil(rows/32)*dim = %zu floats exceeds the static scratch of %zu "
                "floats (4 MiB); use pgf_rmsnorm_bwd with a caller workspace",
                need, NOALLOC_RMS_FLOATS);
  cudaStream_t s = as_stream(stream);
  if (rows == 0) {
    if (!accumulate) PGF_CUDA(cudaMemsetAsync(grad_weight, 0, dim * sizeof(float), s));
    return PGF_OK;
  }
  PGF_CHECK_ARG(x && g, "rmsnorm_bwd_noalloc: null pointer");
  float* part = nullptr;
  PGF_TRY(noalloc_scratch(&part));
  if (dtype == PGF_DTYPE_F32)
    return rms_bwd_dispatch((const float*)x, (const float*)g, weight, (float*)grad_x, grad_weight,
                            accumulate, rows, int(dim), eps, part, s);
  if (dtype == PGF_DTYPE_BF16)
    return rms_bwd_dispatch((const __nv_bfloat16*)x, (const __nv_bfloat16*)g, weight,
                            (__nv_bfloat16*)grad_x, grad_weight, accumulate, rows, int(dim), eps,
                            part, s);
  set_error("rmsnorm_bwd_noalloc: bad dtype %d", dtype);
  return PGF_ERR_INVALID;
}
