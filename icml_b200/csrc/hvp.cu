// State Hessian-vector product of the selective scan (SingleLayerMambaPGF.compute_state_hvp,
// train_singlemamba_optimized.py:563-685, with _pass2_block's HVP branch :249-275): the
// trajectory zeta (L, B, D, N) of d^2 Loss / dh^2 . v_h for the MSE loss against `target`.
//
//   xi_t = exp(A P_t) v_h,  P_t = sum_{s <= t} dt_s            (the tangent scan, closed form)
//   S_t = hf_t (C_t . xi_t) C_t,  hf = l'' or l'' act'(C.h)^2 + grad_y act''(C.h)
//   zeta_t = exp(A dt_{t+1}) zeta_{t+1} + S_t,  zeta_L = 0, no decay after the last token.
//
// zeta is a reverse scan of the same form as the training backward's adjoint, so it is chunked the
// same way: per-chunk dt statistics, a prefix of dt over chunks (for xi), a reverse pass per chunk
// from a zero carry, the segmented reverse compose of scan_compose.cuh, and the output pass that
// re-runs each chunk from its carry and writes zeta.  A thread owns 4 states of one channel, a CTA
// 64 channels x one chunk; tokens are staged 8 at a time in shared memory.
#include "gemm.cuh"
#include "scan_compose.cuh"
#include "f32x2.cuh"

namespace pgf {
namespace hvp {

constexpr int NST = 16, NQ = 4, NS = NST / NQ, DC = 64, THREADS = DC * NQ, ST = 8, TC = 128, KS = TC / ST;
constexpr float LOG2E = 1.4426950408889634f;

struct Args {
  int64_t Bsz, L, D, P, nC, G;
  const float* proj;          // (B, L, P): [dt_in | B | C]
  const float* hf;            // (B, L, D) Hessian factor, or null: the constant l2
  float l2;
  const float* A_log;
  const float* v;             // (B, D, N)
  float* sdt; float* sdt2; float* dt0; float* P0;  // (B, nC, D)
  float* dloc; float* X;      // (B, nC, D, N)
  float* out;                 // (L, B, D, N)
};

struct Stage {
  float dt[ST][DC];
  float hf[ST][DC];
  float4 C[ST][NQ];
};

__device__ __forceinline__ float dt_of(const Args& a, int64_t b, int64_t t, int64_t d) {
  return softplus_fast(a.proj[(b * a.L + t) * a.P + d]);
}

// ---- per-chunk dt statistics: sum, sum without the first token, first dt
__global__ void __launch_bounds__(256) chunk_dt_kernel(const Args a) {
  const int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;  // (b, c, d)
  if (idx >= a.Bsz * a.nC * a.D) return;
  const int64_t d = idx % a.D, c = (idx / a.D) % a.nC, b = idx / (a.D * a.nC);
  const int64_t s = c * TC, e = s + TC < a.L ? s + TC : a.L;
  float first = dt_of(a, b, s, d), sum2 = 0.f;
  for (int64_t t = s + 1; t < e; ++t) sum2 += dt_of(a, b, t, d);
  a.sdt[idx] = first + sum2;
  a.sdt2[idx] = sum2;
  a.dt0[idx] = first;
}

// ---- exclusive prefix of the chunk sums over chunks, per (b, d)
__global__ void __launch_bounds__(256) chunk_prefix_kernel(const Args a) {
  const int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;  // (b, d)
  if (idx >= a.Bsz * a.D) return;
  const int64_t d = idx % a.D, b = idx / a.D;
  float p = 0.f;
  for (int64_t c = 0; c < a.nC; ++c) {
    const int64_t o = (b * a.nC + c) * a.D + d;
    a.P0[o] = p;
    p += a.sdt[o];
  }
}

// ---- reverse pass over one chunk: OUT = false from a zero carry (writes the chunk-start zeta to
// dloc), OUT = true from the composed carry X (writes the trajectory)
template <bool OUT>
__global__ void __launch_bounds__(THREADS) pass_kernel(const Args a) {
  __shared__ Stage stg;
  __shared__ float subP[KS][DC];  // P just before each sub-chunk
  const int tid = threadIdx.x, dl = tid / NQ, nq = tid % NQ;
  const int64_t c = blockIdx.x, b = blockIdx.y, d = int64_t(blockIdx.z) * DC + dl;
  const bool ch = d < a.D;
  const int64_t s = c * TC, e = s + TC < a.L ? s + TC : a.L;
  const int nsub = int((e - s + ST - 1) / ST);
  float A[NS], A2[NS], v[NS];
#pragma unroll
  for (int j = 0; j < NS; ++j) {
    A[j] = -expf(a.A_log[nq * NS + j]);
    A2[j] = A[j] * LOG2E;
    v[j] = ch ? a.v[(b * a.D + d) * NST + nq * NS + j] : 0.f;
  }
  // sub-chunk sums of dt (lane nq takes sub-chunks nq, nq+4, ...), then their prefix from P0
  for (int k = nq; k < nsub; k += NQ) {
    float sm = 0.f;
    for (int i = 0; i < ST; ++i) {
      const int64_t t = s + int64_t(k) * ST + i;
      if (t < e && ch) sm += dt_of(a, b, t, d);
    }
    subP[k][dl] = sm;
  }
  __syncthreads();
  if (nq == 0) {
    float p = ch ? a.P0[(b * a.nC + c) * a.D + d] : 0.f;
    for (int k = 0; k < nsub; ++k) {
      const float sm = subP[k][dl];
      subP[k][dl] = p;
      p += sm;
    }
  }
  float z[NS];
  const int64_t so = ((b * a.nC + c) * a.D + (ch ? d : 0)) * NST + nq * NS;
#pragma unroll
  for (int j = 0; j < NS; ++j) z[j] = (OUT && ch) ? a.X[so + j] : 0.f;
  float dt_next = 0.f;  // dt of the token after the current one (0: none, the carry holds the decay)
  for (int k = nsub - 1; k >= 0; --k) {
    __syncthreads();  // the previous sub-chunk's stage (and subP's prefix) are settled
    // stage: dt and hf of 8 tokens x 64 channels (two per thread), C of 8 tokens (one value per thread)
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const int idx = tid + q * THREADS;
      const int t = idx / DC, cl = idx % DC;
      const int64_t tok = s + int64_t(k) * ST + t, dd = int64_t(blockIdx.z) * DC + cl;
      const bool ok = tok < e && dd < a.D;
      stg.dt[t][cl] = ok ? dt_of(a, b, tok, dd) : 0.f;
      stg.hf[t][cl] = ok ? (a.hf ? a.hf[(b * a.L + tok) * a.D + dd] : a.l2) : 0.f;
    }
    if (tid < ST * NST) {
      const int t = tid / NST, n = tid % NST;
      const int64_t tok = s + int64_t(k) * ST + t;
      reinterpret_cast<float*>(&stg.C[t][0])[n] = tok < e ? a.proj[(b * a.L + tok) * a.P + a.D + NST + n] : 0.f;
    }
    __syncthreads();
    const int64_t rem = e - (s + int64_t(k) * ST);
    const int nt = rem < ST ? int(rem) : ST;
    float cum[ST];  // P_t within the sub-chunk (inclusive)
    {
      float p = subP[k][dl];
#pragma unroll
      for (int i = 0; i < ST; ++i) {
        p += stg.dt[i][dl];
        cum[i] = p;
      }
    }
#pragma unroll
    for (int i = ST - 1; i >= 0; --i) {
      if (i < nt) {
        const float4 Cq = stg.C[i][nq];
        const float Cv[NS] = {Cq.x, Cq.y, Cq.z, Cq.w};
        float cx = 0.f;
#pragma unroll
        for (int j = 0; j < NS; ++j) cx = fmaf(Cv[j], ex2f(A2[j] * cum[i]) * v[j], cx);
        cx += __shfl_xor_sync(0xffffffffu, cx, 1);
        cx += __shfl_xor_sync(0xffffffffu, cx, 2);
        const float w = stg.hf[i][dl] * cx;
#pragma unroll
        for (int j = 0; j < NS; ++j) z[j] = fmaf(ex2f(A2[j] * dt_next), z[j], w * Cv[j]);
        if (OUT && ch) {
          const int64_t tok = s + int64_t(k) * ST + i;
          *reinterpret_cast<float4*>(a.out + ((tok * a.Bsz + b) * a.D + d) * NST + nq * NS) =
              make_float4(z[0], z[1], z[2], z[3]);
        }
        dt_next = stg.dt[i][dl];
      }
    }
  }
  if (!OUT && ch) {
#pragma unroll
    for (int j = 0; j < NS; ++j) a.dloc[so + j] = z[j];
  }
}

// ---- carries X entering each chunk from the right (zero after the last token, no decay there)
__global__ void __launch_bounds__(32 * CSEG) compose_kernel(const Args a) {
  const int64_t idx = int64_t(blockIdx.x) * 32 + (threadIdx.x & 31);  // (b, d, n)
  const bool valid = idx < a.Bsz * a.D * NST;
  const int64_t ii = valid ? idx : 0;
  const int n = int(ii % NST);
  const int64_t d = (ii / NST) % a.D, b = ii / (NST * a.D);
  const float A2 = -expf(a.A_log[n]) * LOG2E;
  float aE0;
  compose_bwd_segmented(valid, a.sdt2 + b * a.nC * a.D + d, a.dt0 + b * a.nC * a.D + d, a.D,
                        a.dloc + (b * a.nC * a.D + d) * NST + n, a.D * NST, a.X + (b * a.nC * a.D + d) * NST + n, A2,
                        0.f, 1.f, a.nC, &aE0);
}

// Hessian factor from C.h (in place): hf = l2 act'(hc)^2 + grad_y act''(hc),
// grad_y = sc ((act(hc) + D u) scale - target)  (train_singlemamba_optimized.py:213-232, 258-265)
__global__ void __launch_bounds__(256) factor_kernel(float* __restrict__ hc, const float* __restrict__ u,
                                                     const float* __restrict__ target, const float* __restrict__ Dp,
                                                     const float* __restrict__ scale, int64_t n, int64_t D, int act,
                                                     float sc, float l2) {
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t d = i % D;
    const float x = hc[i];
    float f, fp, fpp;
    if (act == PGF_ACT_TANH) {
      f = tanhf(x);
      fp = 1.f - f * f;
      fpp = -2.f * f * fp;
    } else {  // relu
      f = x > 0.f ? x : 0.f;
      fp = x > 0.f ? 1.f : 0.f;
      fpp = 0.f;
    }
    const float gy = sc * ((f + Dp[d] * u[i]) * scale[d] - target[i]);
    hc[i] = l2 * fp * fp + gy * fpp;
  }
}

__global__ void fill_kernel(float* p, int64_t n, float v) {
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) p[i] = v;
}

struct Plan {
  int64_t Bsz, L, D, P, nC, G;
};
static Plan plan_of(int64_t Bsz, int64_t L, int64_t D) {
  Plan p{Bsz, L, D, D + 2 * NST, (L + TC - 1) / TC, (D + DC - 1) / DC};
  return p;
}
static size_t ws_bytes(const Plan& p, int act) {
  const size_t BL = size_t(p.Bsz) * p.L, st = size_t(p.Bsz) * p.nC * p.D;
  size_t b = Workspace::round(BL * p.P * 4) + Workspace::round(st * 4) * 4 + Workspace::round(st * NST * 4) * 2;
  if (act != PGF_ACT_NONE) {
    b += Workspace::round(BL * p.D * 4) + Workspace::round(size_t(p.D) * 4) * 2;
    b += Workspace::round(pgf_ssm_workspace(p.Bsz, p.L, p.D, NST, 0, 0));
  }
  return b + 1024;
}

}  // namespace hvp
}  // namespace pgf

using namespace pgf;

extern "C" size_t pgf_ssm_state_hvp_workspace(int64_t Bsz, int64_t L, int64_t D, int64_t N, int act) {
  (void)N;
  return hvp::ws_bytes(hvp::plan_of(Bsz < 1 ? 1 : Bsz, L < 1 ? 1 : L, D < 1 ? 1 : D), act);
}

extern "C" int pgf_ssm_state_hvp(const float* u, const float* target, const float* W_cat, const float* b_cat,
                                 const float* A_log, const float* Dp, const float* scale, const float* v_h, float* out,
                                 int64_t Bsz, int64_t L, int64_t D, int64_t N, int act, void* ws, size_t ws_bytes,
                                 pgf_stream_t stream) {
  using namespace hvp;
  PGF_CHECK_ARG(N == NST, "ssm_state_hvp: d_state must be %d (got %lld)", NST, (long long)N);
  PGF_CHECK_ARG(Bsz > 0 && L >= 0 && D > 0 && Bsz <= 65535, "ssm_state_hvp: bad shape");
  PGF_CHECK_ARG(act == PGF_ACT_NONE || act == PGF_ACT_RELU || act == PGF_ACT_TANH, "ssm_state_hvp: bad act");
  PGF_CHECK_ARG(u && target && W_cat && b_cat && A_log && Dp && scale && v_h && (out || L == 0),
                "ssm_state_hvp: null pointer");
  if (L == 0) return PGF_OK;
  cudaStream_t s = as_stream(stream);
  const Plan p = plan_of(Bsz, L, D);
  Workspace W(ws, ws_bytes);
  Args a = {};
  a.Bsz = Bsz; a.L = L; a.D = D; a.P = p.P; a.nC = p.nC; a.G = p.G;
  a.A_log = A_log; a.v = v_h; a.out = out;
  const float sc = 2.0f / float(double(L) * double(D) * double(Bsz));
  a.l2 = 2.0f * sc;
  const size_t BL = size_t(Bsz) * L, st = size_t(Bsz) * p.nC * D;
  float* proj = W.take<float>(BL * p.P);
  a.sdt = W.take<float>(st); a.sdt2 = W.take<float>(st); a.dt0 = W.take<float>(st); a.P0 = W.take<float>(st);
  a.dloc = W.take<float>(st * NST); a.X = W.take<float>(st * NST);
  if (!proj || !a.sdt || !a.sdt2 || !a.dt0 || !a.P0 || !a.dloc || !a.X) {
    set_error("ssm_state_hvp: workspace too small (%zu)", ws_bytes);
    return PGF_ERR_WORKSPACE;
  }
  a.proj = proj;
  // [dt_in | B | C] = u W_cat^T + b_cat  (train_singlemamba_optimized.py:116-124)
  Gemm g = gemm_make(int64_t(BL), p.P, D, u, 0, D, 0, W_cat, 0, D, 0, proj, 0, p.P);
  g.epi.bias = b_cat;
  PGF_TRY(run_gemm(g, s));
  if (act != PGF_ACT_NONE) {
    // C.h from a zero state: the scan's forward with D = 0, scale = 1 and no activation
    float* hc = W.take<float>(BL * D);
    float* zero = W.take<float>(size_t(D));
    float* one = W.take<float>(size_t(D));
    const size_t fws = pgf_ssm_workspace(Bsz, L, D, NST, 0, 0);
    void* fw = W.take<char>(fws);
    if (!hc || !zero || !one || !fw) {
      set_error("ssm_state_hvp: workspace too small (%zu)", ws_bytes);
      return PGF_ERR_WORKSPACE;
    }
    PGF_CUDA(cudaMemsetAsync(zero, 0, D * 4, s));
    fill_kernel<<<unsigned((D + 255) / 256), 256, 0, s>>>(one, D, 1.0f);
    PGF_LAUNCH_CHECK();
    PGF_TRY(pgf_ssm_fwd(u, W_cat, b_cat, A_log, zero, one, nullptr, hc, nullptr, Bsz, L, D, NST, PGF_ACT_NONE,
                        PGF_DTYPE_F32, fw, fws, stream));
    const int64_t n = int64_t(BL) * D;
    int64_t blocks = (n + 255) / 256;
    if (blocks > int64_t(sm_count()) * 16) blocks = int64_t(sm_count()) * 16;
    factor_kernel<<<unsigned(blocks), 256, 0, s>>>(hc, u, target, Dp, scale, n, D, act, sc, a.l2);
    PGF_LAUNCH_CHECK();
    a.hf = hc;
  }
  chunk_dt_kernel<<<unsigned((st + 255) / 256), 256, 0, s>>>(a);
  PGF_LAUNCH_CHECK();
  chunk_prefix_kernel<<<unsigned((Bsz * D + 255) / 256), 256, 0, s>>>(a);
  PGF_LAUNCH_CHECK();
  const dim3 grid(unsigned(p.nC), unsigned(Bsz), unsigned(p.G));
  pass_kernel<false><<<grid, THREADS, 0, s>>>(a);
  PGF_LAUNCH_CHECK();
  compose_kernel<<<unsigned((Bsz * D * NST + 31) / 32), 32 * CSEG, 0, s>>>(a);
  PGF_LAUNCH_CHECK();
  pass_kernel<true><<<grid, THREADS, 0, s>>>(a);
  PGF_LAUNCH_CHECK();
  return PGF_OK;
}
