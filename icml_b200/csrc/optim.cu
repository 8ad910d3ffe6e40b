// The step on either side of the training path: AdamW over one flat float32 parameter buffer and
// the global gradient norm (clip_grad_norm_ semantics), both HBM-bound single passes.
//
// The reference steps torch.optim.AdamW(params, lr=1e-3, weight_decay=0.01) with default betas and
// eps after every PGF step (train_wikitext_rebuttal.py:77,148).  pgf_adamw_step follows that
// optimizer's arithmetic per element, in float32:
//   p <- p (1 - lr wd);  m <- m + (1 - b1)(g - m);  v <- b2 v + (1 - b2) g^2;
//   p <- p - (lr / (1 - b1^t)) m / (sqrt(v) / sqrt(1 - b2^t) + eps)
// with t the step count, kept on the device (so a captured step replays with the right t) and
// g optionally multiplied by a device scalar (the clip factor from pgf_grad_norm).
#include "gemm.cuh"

namespace pgf {

constexpr int OPT_THREADS = 256;
constexpr int NORM_BLOCKS = 592;  // fixed, so the summation order does not depend on the GPU

struct AdamHyper {
  float lr, b1, b2, eps, wd;
};

__device__ __forceinline__ void adam_elem(float& p, float g, float& m, float& v, const AdamHyper& h, float step_size,
                                          float rbc2_sqrt) {
  p *= 1.0f - h.lr * h.wd;
  m = fmaf(1.0f - h.b1, g - m, m);
  v = fmaf(h.b2, v, (1.0f - h.b2) * g * g);
  const float denom = sqrtf(v) * rbc2_sqrt + h.eps;
  p = fmaf(-step_size, m / denom, p);
}

__global__ void __launch_bounds__(OPT_THREADS) adamw_kernel(float* __restrict__ p, const float* __restrict__ g,
                                                            float* __restrict__ m, float* __restrict__ v, int64_t n,
                                                            AdamHyper h, const float* __restrict__ step,
                                                            const float* __restrict__ gscale) {
  const float t = *step + 1.0f;
  const float bc1 = 1.0f - powf(h.b1, t), bc2 = 1.0f - powf(h.b2, t);
  const float step_size = h.lr / bc1;
  const float rbc2_sqrt = 1.0f / sqrtf(bc2);
  const float s = gscale ? *gscale : 1.0f;
  const int64_t n4 = n / 4;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  float4* p4 = reinterpret_cast<float4*>(p);
  float4* m4 = reinterpret_cast<float4*>(m);
  float4* v4 = reinterpret_cast<float4*>(v);
  const float4* g4 = reinterpret_cast<const float4*>(g);
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n4; i += stride) {
    float4 pp = p4[i], mm = m4[i], vv = v4[i];
    const float4 gg = g4[i];
    adam_elem(pp.x, gg.x * s, mm.x, vv.x, h, step_size, rbc2_sqrt);
    adam_elem(pp.y, gg.y * s, mm.y, vv.y, h, step_size, rbc2_sqrt);
    adam_elem(pp.z, gg.z * s, mm.z, vv.z, h, step_size, rbc2_sqrt);
    adam_elem(pp.w, gg.w * s, mm.w, vv.w, h, step_size, rbc2_sqrt);
    p4[i] = pp;
    m4[i] = mm;
    v4[i] = vv;
  }
  for (int64_t i = n4 * 4 + int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
    adam_elem(p[i], g[i] * s, m[i], v[i], h, step_size, rbc2_sqrt);
}

__global__ void step_increment_kernel(float* step) { *step += 1.0f; }

// Multi-tensor form: the gradients stay in their own tensors.  The host cuts every tensor into
// chunks of at most MT_CHUNK elements and passes the chunk table by value (one CTA per chunk, up
// to MT_MAX chunks per launch): gradient source, offset in the flat buffers, length.  A null
// source is a zero gradient.
constexpr int MT_MAX = 1000;       // 24 KB of kernel parameters
constexpr int64_t MT_CHUNK = 32768;
struct MtItem {
  const float* src;
  int64_t off;
  int64_t len;
};
struct MtTable {
  MtItem it[MT_MAX];
};

__global__ void __launch_bounds__(OPT_THREADS) adamw_multi_kernel(float* __restrict__ p, float* __restrict__ m,
                                                                  float* __restrict__ v, const __grid_constant__ MtTable tab,
                                                                  AdamHyper h, const float* __restrict__ step,
                                                                  const float* __restrict__ gscale) {
  const MtItem w = tab.it[blockIdx.x];
  const float t = *step + 1.0f;
  const float bc1 = 1.0f - powf(h.b1, t), bc2 = 1.0f - powf(h.b2, t);
  const float step_size = h.lr / bc1;
  const float rbc2_sqrt = 1.0f / sqrtf(bc2);
  const float s = gscale ? *gscale : 1.0f;
  float* pp = p + w.off;
  float* mp = m + w.off;
  float* vp = v + w.off;
  const bool vec = (reinterpret_cast<uintptr_t>(w.src) & 15) == 0;  // flat offsets are multiples of 4
  const int64_t n4 = vec ? w.len / 4 : 0;
  for (int64_t i = threadIdx.x; i < n4; i += OPT_THREADS) {
    float4 a = reinterpret_cast<float4*>(pp)[i], mm = reinterpret_cast<float4*>(mp)[i],
           vv = reinterpret_cast<float4*>(vp)[i];
    const float4 gg = w.src ? reinterpret_cast<const float4*>(w.src)[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    adam_elem(a.x, gg.x * s, mm.x, vv.x, h, step_size, rbc2_sqrt);
    adam_elem(a.y, gg.y * s, mm.y, vv.y, h, step_size, rbc2_sqrt);
    adam_elem(a.z, gg.z * s, mm.z, vv.z, h, step_size, rbc2_sqrt);
    adam_elem(a.w, gg.w * s, mm.w, vv.w, h, step_size, rbc2_sqrt);
    reinterpret_cast<float4*>(pp)[i] = a;
    reinterpret_cast<float4*>(mp)[i] = mm;
    reinterpret_cast<float4*>(vp)[i] = vv;
  }
  for (int64_t i = n4 * 4 + threadIdx.x; i < w.len; i += OPT_THREADS)
    adam_elem(pp[i], (w.src ? w.src[i] : 0.f) * s, mp[i], vp[i], h, step_size, rbc2_sqrt);
}

__global__ void __launch_bounds__(OPT_THREADS) gather_multi_kernel(float* __restrict__ dst,
                                                                   const __grid_constant__ MtTable tab) {
  const MtItem w = tab.it[blockIdx.x];
  float* d = dst + w.off;
  const bool vec = (reinterpret_cast<uintptr_t>(w.src) & 15) == 0;
  const int64_t n4 = vec ? w.len / 4 : 0;
  for (int64_t i = threadIdx.x; i < n4; i += OPT_THREADS)
    reinterpret_cast<float4*>(d)[i] =
        w.src ? reinterpret_cast<const float4*>(w.src)[i] : make_float4(0.f, 0.f, 0.f, 0.f);
  for (int64_t i = n4 * 4 + threadIdx.x; i < w.len; i += OPT_THREADS) d[i] = w.src ? w.src[i] : 0.f;
}

// Cuts tensors [first, count) into chunks, fills `tab` (at most MT_MAX items) and returns the
// number of items; `first` / `done` advance to where the next launch resumes.
static int mt_fill(MtTable& tab, const float* const* srcs, const int64_t* offs, const int64_t* sizes, int count,
                   int& first, int64_t& done) {
  int k = 0;
  while (first < count && k < MT_MAX) {
    const int64_t rem = sizes[first] - done;
    if (rem <= 0) {
      ++first;
      done = 0;
      continue;
    }
    const int64_t len = rem < MT_CHUNK ? rem : MT_CHUNK;
    tab.it[k].src = srcs[first] ? srcs[first] + done : nullptr;
    tab.it[k].off = offs[first] + done;
    tab.it[k].len = len;
    ++k;
    done += len;
  }
  return k;
}

// Sum of squares: block b covers a fixed grid-stride share, its partial (double) goes to part[b].
__global__ void __launch_bounds__(OPT_THREADS) sumsq_part_kernel(const float* __restrict__ g, int64_t n,
                                                                 double* __restrict__ part) {
  __shared__ double red[OPT_THREADS / 32];
  float acc = 0.f;
  const int64_t n4 = n / 4;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  const float4* g4 = reinterpret_cast<const float4*>(g);
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n4; i += stride) {
    const float4 x = g4[i];
    acc = fmaf(x.x, x.x, acc);
    acc = fmaf(x.y, x.y, acc);
    acc = fmaf(x.z, x.z, acc);
    acc = fmaf(x.w, x.w, acc);
  }
  for (int64_t i = n4 * 4 + int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
    acc = fmaf(g[i], g[i], acc);
  double d = acc;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = d;
  __syncthreads();
  if (threadIdx.x == 0) {
    double s = 0.0;
    for (int w = 0; w < OPT_THREADS / 32; ++w) s += red[w];
    part[blockIdx.x] = s;
  }
}

// norm = sqrt(sum of the partials, in block order); clip = min(1, max_norm / (norm + 1e-6)).
__global__ void __launch_bounds__(OPT_THREADS) sumsq_final_kernel(const double* __restrict__ part, int nb,
                                                                  float* __restrict__ norm, float max_norm,
                                                                  float* __restrict__ clip) {
  __shared__ double red[OPT_THREADS];
  double s = 0.0;
  for (int i = threadIdx.x; i < nb; i += OPT_THREADS) s += part[i];
  red[threadIdx.x] = s;
  __syncthreads();
  for (int w = OPT_THREADS / 2; w > 0; w >>= 1) {
    if (threadIdx.x < w) red[threadIdx.x] += red[threadIdx.x + w];
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    const float nrm = float(sqrt(red[0]));
    if (norm) *norm = nrm;
    if (clip) *clip = fminf(1.0f, max_norm / (nrm + 1e-6f));
  }
}

static unsigned opt_grid(int64_t n) {
  const int64_t want = (n / 4 + OPT_THREADS - 1) / OPT_THREADS;
  const int64_t cap = int64_t(sm_count()) * 8;
  return unsigned(want < 1 ? 1 : (want < cap ? want : cap));
}

}  // namespace pgf

using namespace pgf;

extern "C" int pgf_adamw_step(float* param, const float* grad, float* exp_avg, float* exp_avg_sq, int64_t n,
                              float lr, float beta1, float beta2, float eps, float weight_decay, float* step,
                              const float* grad_scale, pgf_stream_t stream) {
  PGF_CHECK_ARG(n >= 0, "adamw: negative size");
  PGF_CHECK_ARG(step, "adamw: null step counter");
  if (n == 0) return PGF_OK;
  PGF_CHECK_ARG(param && grad && exp_avg && exp_avg_sq, "adamw: null pointer");
  PGF_CHECK_ARG(aligned(param, 16) && aligned(grad, 16) && aligned(exp_avg, 16) && aligned(exp_avg_sq, 16),
                "adamw: buffers must be 16-byte aligned");
  PGF_CHECK_ARG(beta1 >= 0.f && beta1 < 1.f && beta2 >= 0.f && beta2 < 1.f && eps > 0.f, "adamw: bad hyperparameters");
  cudaStream_t s = as_stream(stream);
  AdamHyper h{lr, beta1, beta2, eps, weight_decay};
  prof_begin(PROF_OPTIM, s);
  adamw_kernel<<<opt_grid(n), OPT_THREADS, 0, s>>>(param, grad, exp_avg, exp_avg_sq, n, h, step, grad_scale);
  prof_end(PROF_OPTIM, s, 28.0 * double(n));  // read p, g, m, v; write p, m, v
  PGF_LAUNCH_CHECK();
  step_increment_kernel<<<1, 1, 0, s>>>(step);
  PGF_LAUNCH_CHECK();
  return PGF_OK;
}

static int check_table(const float* const* srcs, const int64_t* offs, const int64_t* sizes, int count, int64_t n) {
  PGF_CHECK_ARG(count >= 0 && (count == 0 || (srcs && offs && sizes)), "multi-tensor: null table");
  for (int i = 0; i < count; ++i) {
    PGF_CHECK_ARG(sizes[i] >= 0 && offs[i] >= 0 && offs[i] + sizes[i] <= n, "multi-tensor: tensor %d outside the buffer", i);
    PGF_CHECK_ARG(offs[i] % 4 == 0, "multi-tensor: offset of tensor %d not a multiple of 4", i);
  }
  return PGF_OK;
}

extern "C" int pgf_adamw_step_multi(float* param, float* exp_avg, float* exp_avg_sq, int64_t n,
                                    const float* const* grads, const int64_t* offsets, const int64_t* sizes,
                                    int count, float lr, float beta1, float beta2, float eps, float weight_decay,
                                    float* step, const float* grad_scale, pgf_stream_t stream) {
  PGF_CHECK_ARG(n >= 0 && step, "adamw: bad size or null step counter");
  PGF_CHECK_ARG(param && exp_avg && exp_avg_sq, "adamw: null pointer");
  PGF_CHECK_ARG(aligned(param, 16) && aligned(exp_avg, 16) && aligned(exp_avg_sq, 16),
                "adamw: buffers must be 16-byte aligned");
  PGF_CHECK_ARG(beta1 >= 0.f && beta1 < 1.f && beta2 >= 0.f && beta2 < 1.f && eps > 0.f, "adamw: bad hyperparameters");
  PGF_TRY(check_table(grads, offsets, sizes, count, n));
  cudaStream_t s = as_stream(stream);
  AdamHyper h{lr, beta1, beta2, eps, weight_decay};
  MtTable tab;  // the launch parameters (24 KB, on the caller's stack: calls may run concurrently)
  int first = 0;
  int64_t done = 0, total = 0;
  for (int i = 0; i < count; ++i) total += sizes[i];
  prof_begin(PROF_OPTIM, s);
  while (true) {
    const int k = mt_fill(tab, grads, offsets, sizes, count, first, done);
    if (k == 0) break;
    adamw_multi_kernel<<<k, OPT_THREADS, 0, s>>>(param, exp_avg, exp_avg_sq, tab, h, step, grad_scale);
    PGF_LAUNCH_CHECK();
  }
  prof_end(PROF_OPTIM, s, 28.0 * double(total));
  step_increment_kernel<<<1, 1, 0, s>>>(step);
  PGF_LAUNCH_CHECK();
  return PGF_OK;
}

extern "C" int pgf_gather_multi(float* dst, int64_t n, const float* const* srcs, const int64_t* offsets,
                                const int64_t* sizes, int count, pgf_stream_t stream) {
  PGF_CHECK_ARG(n >= 0 && (dst || n == 0), "gather: null destination");
  PGF_CHECK_ARG(!dst || aligned(dst, 16), "gather: destination must be 16-byte aligned");
  PGF_TRY(check_table(srcs, offsets, sizes, count, n));
  cudaStream_t s = as_stream(stream);
  MtTable tab;
  int first = 0;
  int64_t done = 0;
  while (true) {
    const int k = mt_fill(tab, srcs, offsets, sizes, count, first, done);
    if (k == 0) break;
    gather_multi_kernel<<<k, OPT_THREADS, 0, s>>>(dst, tab);
    PGF_LAUNCH_CHECK();
  }
  return PGF_OK;
}

extern "C" size_t pgf_grad_norm_workspace(int64_t n) {
  (void)n;
  return size_t(NORM_BLOCKS) * sizeof(double);
}

extern "C" int pgf_grad_norm(const float* grad, int64_t n, float* norm, float max_norm, float* clip, void* ws,
                             size_t ws_bytes, pgf_stream_t stream) {
  PGF_CHECK_ARG(n >= 0, "grad_norm: negative size");
  PGF_CHECK_ARG(grad || n == 0, "grad_norm: null gradient");
  PGF_CHECK_ARG(norm || clip, "grad_norm: no output");
  PGF_CHECK_ARG(ws && ws_bytes >= pgf_grad_norm_workspace(n) && aligned(ws, 8), "grad_norm: workspace too small");
  PGF_CHECK_ARG(aligned(grad, 16) || n == 0, "grad_norm: gradient must be 16-byte aligned");
  PGF_CHECK_ARG(!clip || max_norm > 0.f, "grad_norm: max_norm must be positive");
  cudaStream_t s = as_stream(stream);
  double* part = static_cast<double*>(ws);
  sumsq_part_kernel<<<NORM_BLOCKS, OPT_THREADS, 0, s>>>(grad, n, part);
  PGF_LAUNCH_CHECK();
  sumsq_final_kernel<<<1, OPT_THREADS, 0, s>>>(part, NORM_BLOCKS, norm, max_norm, clip);
  PGF_LAUNCH_CHECK();
  return PGF_OK;
}
