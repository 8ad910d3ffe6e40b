// RMSNorm forward / backward (pgf_rmsnorm.py:10-51).
//
// One warp per row; the row lives in registers (VPL values per lane, columns lane + 32*j), so x
// and g are read once.  The forward can take a residual (sum = x + res, written out in the
// activation type and normalised: the block's `y + x` then norm2 in one pass); the backward can
// add a gradient to grad_x (the block's `norm.grad_x + g` skip connections).  Both round where the
// separate add would, so the fused forms give the same bits.  grad_weight is reduced deterministically: each CTA sums its warps'
// register partials through shared memory in warp order and writes one partial row; a second
// kernel adds the CTA partials in CTA order.
#include "gemm.cuh"

namespace pgf {

constexpr int RMS_WARPS = 8;
constexpr int RMS_ROWS_PER_WARP = 4;  // rows handled by a warp in the backward (one CTA = 32 rows)

template <int VPL, class T>
__global__ void __launch_bounds__(RMS_WARPS * 32)
rmsnorm_fwd_kernel(const T* __restrict__ x, const T* __restrict__ res, T* __restrict__ sum_out,
                   const float* __restrict__ w, T* __restrict__ y, int64_t rows, int dim, float eps) {
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
    if (res && c < dim) {
      // the sum rounded to T, as the separate add stores it, then normalised
      v[j] = rounded<T>(v[j] + ld(res + row * dim, c));
      st(sum_out + row * dim, c, v[j]);
    }
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
                   const T* __restrict__ gadd, T* __restrict__ gx, float* __restrict__ gw_part, int64_t rows, int dim,
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
    float xv[VPL], gv[VPL], av[VPL];
    float ss = 0.f, dot = 0.f;
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      int c = j * 32 + lane;
      xv[j] = c < dim ? ld(xr, c) : 0.f;
      gv[j] = c < dim ? ld(gr, c) : 0.f;
      av[j] = (gadd && c < dim) ? ld(gadd + row * dim, c) : 0.f;  // loaded with x and g
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
        if (c < dim) {
          const float v = (gv[j] * wv[j]) * rinv - (xv[j] * dot) * r3 / float(dim);
          // with an addend: grad_x rounded to T as a separate operator would return it, then added
          st(gxr, c, gadd ? rounded<T>(v) + av[j] : v);
        }
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

// ---- vector forms: a lane owns CPL 16-byte chunks of a row (chunk k = columns (32k + lane) VW ..
// + VW, VW = 16 / sizeof(T)), so a row is CPL coalesced 512-byte loads per tensor; a warp takes
// RPW rows and issues every load of them before any arithmetic.  Used when dim is a multiple of
// 32 VW and every row starts on a 16-byte boundary.
template <class T> struct Vec16;
template <> struct Vec16<float> {
  static constexpr int VW = 4;
  __device__ static void unpack(const uint4 q, float* o) {
    o[0] = __uint_as_float(q.x); o[1] = __uint_as_float(q.y); o[2] = __uint_as_float(q.z); o[3] = __uint_as_float(q.w);
  }
  __device__ static uint4 pack(const float* v) {
    return make_uint4(__float_as_uint(v[0]), __float_as_uint(v[1]), __float_as_uint(v[2]), __float_as_uint(v[3]));
  }
};
template <> struct Vec16<__nv_bfloat16> {
  static constexpr int VW = 8;
  __device__ static void unpack(const uint4 q, float* o) {
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      o[2 * k] = __uint_as_float(w[k] << 16);
      o[2 * k + 1] = __uint_as_float(w[k] & 0xFFFF0000u);
    }
  }
  __device__ static uint32_t pk(float a, float b) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
  __device__ static uint4 pack(const float* v) {
    return make_uint4(pk(v[0], v[1]), pk(v[2], v[3]), pk(v[4], v[5]), pk(v[6], v[7]));
  }
};

template <int CPL, int RPW, class T>
__global__ void __launch_bounds__(RMS_WARPS * 32)
rmsnorm_fwd_vec_kernel(const T* __restrict__ x, const T* __restrict__ res, T* __restrict__ sum_out,
                       const float* __restrict__ w, T* __restrict__ y, int64_t rows, int dim, float eps) {
  using V = Vec16<T>;
  constexpr int VW = V::VW;
  const int lane = threadIdx.x & 31;
  const int64_t row0 = (int64_t(blockIdx.x) * RMS_WARPS + (threadIdx.x >> 5)) * RPW;
  if (row0 >= rows) return;
  uint4 qx[RPW][CPL], qr[RPW][CPL];
#pragma unroll
  for (int r = 0; r < RPW; ++r)
#pragma unroll
    for (int k = 0; k < CPL; ++k) {
      const int64_t off = (row0 + r) * dim + int64_t(k * 32 + lane) * VW;
      const bool ok = row0 + r < rows;
      qx[r][k] = ok ? __ldg(reinterpret_cast<const uint4*>(x + off)) : make_uint4(0, 0, 0, 0);
      qr[r][k] = (ok && res) ? __ldg(reinterpret_cast<const uint4*>(res + off)) : make_uint4(0, 0, 0, 0);
    }
  // the weight slice of this lane, once for all of the warp's rows (one row per warp: read in place)
  constexpr bool HOIST_W = RPW > 1;
  float wv[HOIST_W ? CPL : 1][VW];
  if (HOIST_W) {
#pragma unroll
    for (int k = 0; k < (HOIST_W ? CPL : 1); ++k)
#pragma unroll
      for (int e = 0; e < VW; ++e) wv[k][e] = __ldg(w + (k * 32 + lane) * VW + e);
  }
  // sums of squares of all the warp's rows first, then their warp reductions side by side (the
  // same butterfly order per row), then the per-row divides: the rows' dependent chains overlap
  float v[RPW][CPL][VW];
  float ss[RPW];
#pragma unroll
  for (int r = 0; r < RPW; ++r) {
    const int64_t row = row0 + r;
    ss[r] = 0.f;
#pragma unroll
    for (int k = 0; k < CPL; ++k) {
      V::unpack(qx[r][k], v[r][k]);
      if (res) {
        float a[VW];
        V::unpack(qr[r][k], a);
#pragma unroll
        for (int e = 0; e < VW; ++e) v[r][k][e] = rounded<T>(v[r][k][e] + a[e]);
        if (row < rows)
          *reinterpret_cast<uint4*>(sum_out + row * dim + int64_t(k * 32 + lane) * VW) = V::pack(v[r][k]);
      }
#pragma unroll
      for (int e = 0; e < VW; ++e) ss[r] = fmaf(v[r][k][e], v[r][k][e], ss[r]);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
#pragma unroll
    for (int r = 0; r < RPW; ++r) ss[r] += __shfl_xor_sync(0xffffffffu, ss[r], o);
#pragma unroll
  for (int r = 0; r < RPW; ++r) {
    const int64_t row = row0 + r;
    const float rinv = 1.0f / sqrtf(ss[r] / float(dim) + eps);  // one divide per row
    if (row >= rows) continue;
#pragma unroll
    for (int k = 0; k < CPL; ++k) {
      const int c0 = (k * 32 + lane) * VW;
      float o[VW];
#pragma unroll
      for (int e = 0; e < VW; ++e) o[e] = (v[r][k][e] * rinv) * (HOIST_W ? wv[HOIST_W ? k : 0][e] : __ldg(w + c0 + e));
      *reinterpret_cast<uint4*>(y + row * dim + c0) = V::pack(o);
    }
  }
}

template <int CPL, class T>
__global__ void __launch_bounds__(RMS_WARPS * 32, CPL == 1 ? 3 : 1)  // 1 chunk per lane: 3 CTAs per SM
rmsnorm_bwd_vec_kernel(const T* __restrict__ x, const T* __restrict__ g, const float* __restrict__ w,
                       const T* __restrict__ gadd, T* __restrict__ gx, float* __restrict__ gw_part, int64_t rows,
                       int dim, float eps) {
  using V = Vec16<T>;
  constexpr int VW = V::VW;
  extern __shared__ float sm_gw[];  // [RMS_WARPS][dim]
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  // rows whose loads are issued together: four 16-byte chunks of each tensor per lane in flight,
  // eight at 4 chunks per lane (two rows: one CTA per SM either way, 222 registers)
  constexpr int RB = CPL >= 4 ? 2 : 4 / CPL;
  float acc[CPL][VW];
#pragma unroll
  for (int k = 0; k < CPL; ++k)
#pragma unroll
    for (int e = 0; e < VW; ++e) acc[k][e] = 0.f;
  const int64_t row0 = (int64_t(blockIdx.x) * RMS_WARPS + warp) * RMS_ROWS_PER_WARP;
  // the weight slice of this lane, once per warp where it fits beside the row group's loads;
  // at 4 chunks per lane it is re-read (from L1) per row
  constexpr bool HOIST_W = CPL <= 2;
  float wh[HOIST_W ? CPL : 1][VW];
  if (HOIST_W) {
#pragma unroll
    for (int k = 0; k < (HOIST_W ? CPL : 1); ++k)
#pragma unroll
      for (int e = 0; e < VW; ++e) wh[k][e] = __ldg(w + (k * 32 + lane) * VW + e);
  }
#pragma unroll 1
  for (int rb = 0; rb < RMS_ROWS_PER_WARP; rb += RB) {
  uint4 qx[RB][CPL], qg[RB][CPL], qa[RB][CPL];
#pragma unroll
  for (int r = 0; r < RB; ++r)
#pragma unroll
    for (int k = 0; k < CPL; ++k) {
      const int64_t off = (row0 + rb + r) * dim + int64_t(k * 32 + lane) * VW;
      const bool ok = row0 + rb + r < rows;
      qx[r][k] = ok ? __ldg(reinterpret_cast<const uint4*>(x + off)) : make_uint4(0, 0, 0, 0);
      qg[r][k] = ok ? __ldg(reinterpret_cast<const uint4*>(g + off)) : make_uint4(0, 0, 0, 0);
      qa[r][k] = (ok && gadd) ? __ldg(reinterpret_cast<const uint4*>(gadd + off)) : make_uint4(0, 0, 0, 0);
    }
  // the group's sums (x.x and (g w).x) first, then their warp reductions side by side (each row's
  // butterfly in the same order as a lone row's), then the per-row divides and outputs: the rows'
  // shuffle and divide chains overlap instead of running one after another.  Rows past the end
  // hold zeros and are reduced too, but write nothing.
  float ss[RB], dot[RB];
#pragma unroll
  for (int r = 0; r < RB; ++r) {
    ss[r] = 0.f;
    dot[r] = 0.f;
#pragma unroll
    for (int k = 0; k < CPL; ++k) {
      float xv[VW], gv[VW];
      V::unpack(qx[r][k], xv);
      V::unpack(qg[r][k], gv);
#pragma unroll
      for (int e = 0; e < VW; ++e) {
        const float wk = HOIST_W ? wh[HOIST_W ? k : 0][e] : __ldg(w + (k * 32 + lane) * VW + e);
        ss[r] = fmaf(xv[e], xv[e], ss[r]);
        dot[r] = fmaf(gv[e] * wk, xv[e], dot[r]);
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
#pragma unroll
    for (int r = 0; r < RB; ++r) {
      ss[r] += __shfl_xor_sync(0xffffffffu, ss[r], o);
      dot[r] += __shfl_xor_sync(0xffffffffu, dot[r], o);
    }
  // with several rows in the group, unpack again below rather than keep the unpacked rows alive
  // across the reductions (twice the registers of the packed ones): an empty asm makes the packed
  // words opaque to the compiler
  if constexpr (RB > 1) {
#pragma unroll
    for (int r = 0; r < RB; ++r)
#pragma unroll
      for (int k = 0; k < CPL; ++k) {
        asm volatile("" : "+r"(qx[r][k].x), "+r"(qx[r][k].y), "+r"(qx[r][k].z), "+r"(qx[r][k].w));
        asm volatile("" : "+r"(qg[r][k].x), "+r"(qg[r][k].y), "+r"(qg[r][k].z), "+r"(qg[r][k].w));
      }
  }
#pragma unroll
  for (int r = 0; r < RB; ++r) {
    const int64_t row = row0 + rb + r;
    if (row >= rows) break;
    float wv[CPL][VW];
#pragma unroll
    for (int k = 0; k < CPL; ++k)
#pragma unroll
      for (int e = 0; e < VW; ++e) wv[k][e] = HOIST_W ? wh[HOIST_W ? k : 0][e] : __ldg(w + (k * 32 + lane) * VW + e);
    float xv[CPL][VW], gv[CPL][VW];
#pragma unroll
    for (int k = 0; k < CPL; ++k) {
      V::unpack(qx[r][k], xv[k]);
      V::unpack(qg[r][k], gv[k]);
    }
    const float rinv = 1.0f / sqrtf(ss[r] / float(dim) + eps);
    const float kx = dot[r] * (rinv * rinv * rinv) / float(dim);  // per row: no divide per element
    if (gx) {
#pragma unroll
      for (int k = 0; k < CPL; ++k) {
        float o[VW], a[VW];
        V::unpack(qa[r][k], a);
#pragma unroll
        for (int e = 0; e < VW; ++e) {
          const float v = fmaf(gv[k][e] * wv[k][e], rinv, -xv[k][e] * kx);
          o[e] = gadd ? rounded<T>(v) + a[e] : v;
        }
        *reinterpret_cast<uint4*>(gx + row * dim + int64_t(k * 32 + lane) * VW) = V::pack(o);
      }
    }
#pragma unroll
    for (int k = 0; k < CPL; ++k)
#pragma unroll
      for (int e = 0; e < VW; ++e) acc[k][e] = fmaf(gv[k][e], xv[k][e] * rinv, acc[k][e]);
  }
  }  // row groups
#pragma unroll
  for (int k = 0; k < CPL; ++k)
#pragma unroll
    for (int e = 0; e < VW; ++e) sm_gw[warp * dim + (k * 32 + lane) * VW + e] = acc[k][e];
  __syncthreads();
  for (int c = threadIdx.x; c < dim; c += blockDim.x) {
    float s = 0.f;
    for (int q = 0; q < RMS_WARPS; ++q) s += sm_gw[q * dim + c];
    gw_part[int64_t(blockIdx.x) * dim + c] = s;
  }
}

// Forward-mode derivative (RMSNorm.pgf_jvp, pgf_rmsnorm.py:54-72): along (x_dot, w_dot),
//   y = x w / rms,  rms' = mean(x x_dot) / rms,
//   y_dot = (x_dot / rms - x rms' / rms^2) w + x w_dot / rms.
template <int VPL, class T>
__global__ void __launch_bounds__(RMS_WARPS * 32)
rmsnorm_jvp_kernel(const T* __restrict__ x, const T* __restrict__ xd, const float* __restrict__ w,
                   const float* __restrict__ wd, T* __restrict__ y, T* __restrict__ yd, int64_t rows, int dim,
                   float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t row = int64_t(blockIdx.x) * RMS_WARPS + (threadIdx.x >> 5);
  if (row >= rows) return;
  float v[VPL], t[VPL];
  float ss = 0.f, sd = 0.f;
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    const int c = j * 32 + lane;
    v[j] = c < dim ? ld(x + row * dim, c) : 0.f;
    t[j] = c < dim ? ld(xd + row * dim, c) : 0.f;
    ss = fmaf(v[j], v[j], ss);
    sd = fmaf(v[j], t[j], sd);
  }
  ss = warp_sum(ss);
  sd = warp_sum(sd);
  const float rinv = 1.0f / sqrtf(ss / float(dim) + eps);
  const float rdot = (sd / float(dim)) * rinv;  // rms'
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    const int c = j * 32 + lane;
    if (c < dim) {
      const float wc = w[c];
      st(y + row * dim, c, (v[j] * rinv) * wc);
      st(yd + row * dim, c, fmaf(t[j], rinv, -v[j] * rdot * rinv * rinv) * wc + (v[j] * rinv) * wd[c]);
    }
  }
}

template <class T>
static int rms_jvp_dispatch(const T* x, const T* xd, const float* w, const float* wd, T* y, T* yd, int64_t rows,
                            int dim, float eps, cudaStream_t s) {
  dim3 grid(ceil_div(rows, RMS_WARPS)), block(RMS_WARPS * 32);
  const int vpl = ceil_div(dim, 32);
#define PGF_RMS_J(V) rmsnorm_jvp_kernel<V, T><<<grid, block, 0, s>>>(x, xd, w, wd, y, yd, rows, dim, eps)
  if (vpl <= 1) PGF_RMS_J(1);
  else if (vpl <= 2) PGF_RMS_J(2);
  else if (vpl <= 4) PGF_RMS_J(4);
  else if (vpl <= 8) PGF_RMS_J(8);
  else if (vpl <= 16) PGF_RMS_J(16);
  else if (vpl <= 32) PGF_RMS_J(32);
  else if (vpl <= 64) PGF_RMS_J(64);
  else if (vpl <= 128) PGF_RMS_J(128);
  else { set_error("rmsnorm_jvp: dim %d > 4096 unsupported", dim); return PGF_ERR_UNSUPPORTED; }
#undef PGF_RMS_J
  PGF_LAUNCH_CHECK();
  return PGF_OK;
}

// chunks per lane of the vector forms (0: use the scalar kernels)
template <class T>
static int rms_vec_cpl(const void* a, const void* b, const void* c, const void* d, int64_t dim) {
  constexpr int VW = 16 / int(sizeof(T));
  if (dim % (32 * VW)) return 0;
  const int cpl = int(dim / (32 * VW));
  if (cpl != 1 && cpl != 2 && cpl != 4) return 0;
  for (const void* p : {a, b, c, d})
    if (p && !aligned(p, 16)) return 0;
  return cpl;
}

template <class T>
static int rms_fwd_dispatch(const T* x, const T* res, T* sum_out, const float* w, T* y, int64_t rows, int dim,
                            float eps, cudaStream_t s) {
  const int cpl = rms_vec_cpl<T>(x, res, sum_out, y, dim);
  if (cpl) {
    const double work = double(rows) * dim * (res ? 4.0 : 2.0) * sizeof(T) + dim * 4.0;
#define PGF_RMS_FV(C, R)                                                                                   \
  do {                                                                                                     \
    prof_begin(PROF_RMSNORM_FWD, s);                                                                       \
    rmsnorm_fwd_vec_kernel<C, R, T><<<unsigned(ceil_div(rows, RMS_WARPS * R)), RMS_WARPS * 32, 0, s>>>(     \
        x, res, sum_out, w, y, rows, dim, eps);                                                            \
    prof_end(PROF_RMSNORM_FWD, s, work);                                                                   \
  } while (0)
    if (cpl == 1) PGF_RMS_FV(1, 4);
    else if (cpl == 2) PGF_RMS_FV(2, 2);
    else PGF_RMS_FV(4, 1);
#undef PGF_RMS_FV
    PGF_LAUNCH_CHECK();
    return PGF_OK;
  }
  dim3 grid(ceil_div(rows, RMS_WARPS)), block(RMS_WARPS * 32);
  int vpl = ceil_div(dim, 32);
#define PGF_RMS_F(V)                                                                  \
  do {                                                                                \
    prof_begin(PROF_RMSNORM_FWD, s);                                                  \
    rmsnorm_fwd_kernel<V, T><<<grid, block, 0, s>>>(x, res, sum_out, w, y, rows, dim, eps); \
    prof_end(PROF_RMSNORM_FWD, s, double(rows) * dim * (res ? 4.0 : 2.0) * sizeof(T) + dim * 4.0); \
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
static int rms_bwd_dispatch(const T* x, const T* g, const float* w, const T* gadd, T* gx, float* gw, int acc,
                            int64_t rows, int dim, float eps, float* part, cudaStream_t s) {
  int64_t nct = rms_bwd_ctas(rows);
  dim3 grid((unsigned)nct), block(RMS_WARPS * 32);
  size_t smem = size_t(RMS_WARPS) * dim * sizeof(float);
  const int cpl = rms_vec_cpl<T>(x, g, gadd, gx, dim);
  if (cpl) {
    const double work = double(rows) * dim * (gadd ? 4.0 : 3.0) * sizeof(T) + dim * 4.0;
#define PGF_RMS_BV(C)                                                                                 \
  do {                                                                                                \
    static int smem_limit_v##C = 0;                                                                   \
    PGF_CUDA(ensure_dynamic_smem(rmsnorm_bwd_vec_kernel<C, T>, smem, smem_limit_v##C));               \
    prof_begin(PROF_RMSNORM_BWD, s);                                                                  \
    rmsnorm_bwd_vec_kernel<C, T><<<grid, block, smem, s>>>(x, g, w, gadd, gx, part, rows, dim, eps);  \
    prof_end(PROF_RMSNORM_BWD, s, work);                                                              \
  } while (0)
    if (cpl == 1) PGF_RMS_BV(1);
    else if (cpl == 2) PGF_RMS_BV(2);
    else PGF_RMS_BV(4);
#undef PGF_RMS_BV
    PGF_LAUNCH_CHECK();
    PGF_TRY(column_reduce(part, nct, dim, gw, acc, s));
    return PGF_OK;
  }
  int vpl = ceil_div(dim, 32);
#define PGF_RMS_B(V)                                                                           \
  do {                                                                                         \
    static int smem_limit_##V = 0;                                                             \
    PGF_CUDA(ensure_dynamic_smem(rmsnorm_bwd_kernel<V, T>, smem, smem_limit_##V));             \
    prof_begin(PROF_RMSNORM_BWD, s);                                                           \
    rmsnorm_bwd_kernel<V, T><<<grid, block, smem, s>>>(x, g, w, gadd, gx, part, rows, dim, eps); \
    prof_end(PROF_RMSNORM_BWD, s, double(rows) * dim * (gadd ? 4.0 : 3.0) * sizeof(T) + dim * 4.0); \
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
    return rms_fwd_dispatch((const float*)x, (const float*)nullptr, (float*)nullptr, weight, (float*)y, rows,
                            int(dim), eps, s);
  if (dtype == PGF_DTYPE_BF16)
    return rms_fwd_dispatch((const __nv_bfloat16*)x, (const __nv_bfloat16*)nullptr, (__nv_bfloat16*)nullptr,
                            weight, (__nv_bfloat16*)y, rows, int(dim), eps, s);
  set_error("rmsnorm_fwd: bad dtype %d", dtype);
  return PGF_ERR_INVALID;
}

extern "C" int pgf_rmsnorm_jvp(const void* x, const void* x_dot, const float* weight, const float* weight_dot,
                               void* y, void* y_dot, int64_t rows, int64_t dim, float eps, int dtype,
                               pgf_stream_t stream) {
  PGF_CHECK_ARG(rows >= 0 && dim > 0 && dim <= 4096, "rmsnorm_jvp: bad shape rows=%lld dim=%lld", (long long)rows,
                (long long)dim);
  if (rows == 0) return PGF_OK;
  PGF_CHECK_ARG(x && x_dot && weight && weight_dot && y && y_dot, "rmsnorm_jvp: null pointer");
  cudaStream_t s = as_stream(stream);
  if (dtype == PGF_DTYPE_F32)
    return rms_jvp_dispatch((const float*)x, (const float*)x_dot, weight, weight_dot, (float*)y, (float*)y_dot, rows,
                            int(dim), eps, s);
  if (dtype == PGF_DTYPE_BF16)
    return rms_jvp_dispatch((const __nv_bfloat16*)x, (const __nv_bfloat16*)x_dot, weight, weight_dot,
                            (__nv_bfloat16*)y, (__nv_bfloat16*)y_dot, rows, int(dim), eps, s);
  set_error("rmsnorm_jvp: bad dtype %d", dtype);
  return PGF_ERR_INVALID;
}

extern "C" int pgf_rmsnorm_fwd_res(const void* x, const void* res, const float* weight, void* sum_out, void* y,
                                   int64_t rows, int64_t dim, float eps, int dtype, pgf_stream_t stream) {
  PGF_CHECK_ARG(rows >= 0 && dim > 0 && dim <= 4096, "rmsnorm_fwd_res: bad shape rows=%lld dim=%lld",
                (long long)rows, (long long)dim);
  if (rows == 0) return PGF_OK;
  PGF_CHECK_ARG(x && res && weight && sum_out && y, "rmsnorm_fwd_res: null pointer");
  PGF_CHECK_ARG(sum_out != x && sum_out != res, "rmsnorm_fwd_res: sum_out must not alias the inputs");
  cudaStream_t s = as_stream(stream);
  if (dtype == PGF_DTYPE_F32)
    return rms_fwd_dispatch((const float*)x, (const float*)res, (float*)sum_out, weight, (float*)y, rows, int(dim),
                            eps, s);
  if (dtype == PGF_DTYPE_BF16)
    return rms_fwd_dispatch((const __nv_bfloat16*)x, (const __nv_bfloat16*)res, (__nv_bfloat16*)sum_out, weight,
                            (__nv_bfloat16*)y, rows, int(dim), eps, s);
  set_error("rmsnorm_fwd_res: bad dtype %d", dtype);
  return PGF_ERR_INVALID;
}

extern "C" size_t pgf_rmsnorm_bwd_workspace(int64_t rows, int64_t dim) {
  return Workspace::round(size_t(rms_bwd_ctas(rows < 1 ? 1 : rows)) * size_t(dim) * sizeof(float));
}

static int rmsnorm_bwd_impl(const void* x, const void* g, const float* weight, const void* g_add, void* grad_x,
                            float* grad_weight, int accumulate, int64_t rows, int64_t dim, float eps, int dtype,
                            void* ws, size_t ws_bytes, pgf_stream_t stream) {
  PGF_CHECK_ARG(weight && grad_weight, "rmsnorm_bwd: null pointer");
  PGF_CHECK_ARG(!g_add || grad_x, "rmsnorm_bwd: an addend needs grad_x");
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
    return rms_bwd_dispatch((const float*)x, (const float*)g, weight, (const float*)g_add, (float*)grad_x,
                            grad_weight, accumulate, rows, int(dim), eps, part, s);
  if (dtype == PGF_DTYPE_BF16)
    return rms_bwd_dispatch((const __nv_bfloat16*)x, (const __nv_bfloat16*)g, weight,
                            (const __nv_bfloat16*)g_add, (__nv_bfloat16*)grad_x, grad_weight, accumulate, rows,
                            int(dim), eps, part, s);
  set_error("rmsnorm_bwd: bad dtype %d", dtype);
  return PGF_ERR_INVALID;
}

extern "C" int pgf_rmsnorm_bwd(const void* x, const void* g, const float* weight, void* grad_x, float* grad_weight,
                               int accumulate, int64_t rows, int64_t dim, float eps, int dtype, void* ws,
                               size_t ws_bytes, pgf_stream_t stream) {
  return rmsnorm_bwd_impl(x, g, weight, nullptr, grad_x, grad_weight, accumulate, rows, dim, eps, dtype, ws,
                          ws_bytes, stream);
}

extern "C" int pgf_rmsnorm_bwd_add(const void* x, const void* g, const float* weight, const void* g_add,
                                   void* grad_x, float* grad_weight, int accumulate, int64_t rows, int64_t dim,
                                   float eps, int dtype, void* ws, size_t ws_bytes, pgf_stream_t stream) {
  PGF_CHECK_ARG(g_add && grad_x, "rmsnorm_bwd_add: null pointer");
  return rmsnorm_bwd_impl(x, g, weight, g_add, grad_x, grad_weight, accumulate, rows, dim, eps, dtype, ws,
                          ws_bytes, stream);
}

// ---------------------------------------------------------------------------------------------
// RMSNorm backward without a caller workspace.
//
// For callers that cannot call cudaMalloc: a plugin inside an engine that plans and owns all
// device memory and forbids allocation from its operators, or a latency-critical loop that must
// not enter the allocator.  The grad-weight partials live in the file-scope array below instead
// of a workspace: NOALLOC_RMS_FLOATS floats (4 MiB), held by every GPU that loads this library
// until the process exits.  A call needs ceil(rows / 32) * dim of them, and dim <= 4096.
//
// The host cannot pass the array's name to a kernel (in host code it is only a stand-in for the
// device symbol): every call looks up the array's device address with cudaGetSymbolAddress in the
// calling thread's current context, so the address always belongs to the context the kernel runs
// in (a non-primary context, or a primary context re-created after cudaDeviceReset, included).  The
// lookup is a table read once the library's module is loaded in that context; the first call in a
// context may load it, so make that first call before any stream capture.  Every call overwrites
// all the partial slots it reads, so nothing needs clearing, but the calls share the one array:
// calls that overlap on the GPU (other streams, other threads) race on it and must be serialised
// by the caller.
// ---------------------------------------------------------------------------------------------
namespace pgf {

constexpr size_t NOALLOC_RMS_FLOATS = size_t(1) << 20;
static __device__ __align__(256) float g_rms_noalloc_scratch[NOALLOC_RMS_FLOATS];

// Device address of the scratch array in the current context.
static int noalloc_scratch(float** out) {
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_rms_noalloc_scratch);
  if (e != cudaSuccess || !p) {
    set_error("rmsnorm_bwd_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
    return PGF_ERR_CUDA;
  }
  *out = static_cast<float*>(p);
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
    return rms_bwd_dispatch((const float*)x, (const float*)g, weight, (const float*)nullptr, (float*)grad_x,
                            grad_weight, accumulate, rows, int(dim), eps, part, s);
  if (dtype == PGF_DTYPE_BF16)
    return rms_bwd_dispatch((const __nv_bfloat16*)x, (const __nv_bfloat16*)g, weight,
                            (const __nv_bfloat16*)nullptr, (__nv_bfloat16*)grad_x, grad_weight, accumulate, rows,
                            int(dim), eps, part, s);
  set_error("rmsnorm_bwd_noalloc: bad dtype %d", dtype);
  return PGF_ERR_INVALID;
}
