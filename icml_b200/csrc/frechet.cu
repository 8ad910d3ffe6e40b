// Forward-mode (JVP) scan of the Frechet operator (FrechetMambaOperator.pgf_forward,
// pgf_mamba.py:69-139): the selective scan of pgf_mamba.py:89-110 and its directional derivative
// along (h0_dot, u_dot) with the parameters fixed, for a whole sequence at once.
//
// Per token t, channel d, state n (p = [dt_in | B | C] = u W_cat^T + b_cat, pd = u_dot W_cat^T):
//   dt = softplus(p_dt), dt' = sigmoid(p_dt) pd_dt, z = dt A_n, z' = dt' A_n, e = exp(z),
//   h' = e h' + e z' h + (phi_1'(z) z' B + phi_1(z) B') u + phi_1(z) B u';   h = e h + phi_1(z) B u
//   y = softplus(C.h + D u) s,  y' = sigmoid(C.h + D u) (C'.h + C.h' + D u') s,  s = max(scale, 0.5).
// The pair (h, h') follows a linear recurrence with the lower-triangular transition
// [[e, 0], [e z', e]], so the sequence is cut into chunks exactly like the training scan:
//   1. chunk pass: every chunk from a zero pair; its end pair and sum of dt, dt';
//   2. compose: a chunk's transition is [[E, 0], [E A S', E]] with E = exp(A S) (S, S' the sums of
//      dt, dt'), folded in chunk order from (h0, h0') into every chunk's start pair;
//   3. output pass: every chunk again from its start pair, forming y and y'.
// A thread owns 4 states of one channel (4 lanes per channel), a CTA 64 channels x one chunk;
// inputs are staged 8 tokens at a time in shared memory with a register prefetch.
#include "gemm.cuh"
#include "f32x2.cuh"

namespace pgf {
namespace fjvp {

constexpr int NST = 16, NQ = 4, NS = NST / NQ, DC = 64, THREADS = DC * NQ, ST = 8;
constexpr float LOG2E = 1.4426950408889634f;

struct Args {
  int64_t L, D, P, Tc, nC, G;
  const float* u; const float* ud;
  const float* proj; const float* projd;    // (L, P): [dt_in | B | C] and its tangent
  const float* A_log; const float* Dp; const float* scale;
  const float* h0; const float* hd0;        // (D, N) or null (zero)
  float* hloc; float* hdloc;                // (nC, D, N) chunk-local end pairs
  float* sdt; float* sdtd;                  // (nC, D) sums of dt, dt'
  float* hC; float* hdC;                    // (nC, D, N) chunk start pairs
  float* h_end; float* hd_end;              // (D, N) or null
  float* y; float* yd;                      // (L, D)
};

struct Stage {
  float dt[ST][DC], dtd[ST][DC], rdt[ST][DC], u[ST][DC], ud[ST][DC];
  float4 B[ST][NQ], Bd[ST][NQ], C[ST][NQ], Cd[ST][NQ];
};

struct Pref {
  float p[2], pd[2], u[2], ud[2];
  float bc[2], bcd[2];
};

struct Lane {
  int tid, dl, nq, grp;
  int64_t c, d, s, e;
  bool ch;
};

__device__ __forceinline__ Lane lane_of(const Args& a) {
  Lane l;
  l.tid = threadIdx.x;
  l.dl = l.tid / NQ;
  l.nq = l.tid % NQ;
  l.c = blockIdx.x;
  l.grp = blockIdx.y;
  l.d = int64_t(l.grp) * DC + l.dl;
  l.ch = l.d < a.D;
  l.s = l.c * a.Tc;
  l.e = l.s + a.Tc < a.L ? l.s + a.Tc : a.L;
  return l;
}

struct AConst {
  float A[NS], A2[NS], rA[NS];
};
__device__ __forceinline__ AConst load_A(const Args& a, int nq) {
  AConst c;
#pragma unroll
  for (int j = 0; j < NS; ++j) {
    c.A[j] = -expf(a.A_log[nq * NS + j]);
    c.A2[j] = c.A[j] * LOG2E;
    c.rA[j] = 1.0f / c.A[j];
  }
  return c;
}

__device__ __forceinline__ void pref_load(const Args& a, const Lane& l, int64_t s0, Pref& r) {
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const int idx = l.tid + q * THREADS;
    const int t = idx / DC, dl = idx % DC;
    const int64_t tok = s0 + t;
    const int64_t d = int64_t(l.grp) * DC + dl;
    const bool v = tok < l.e && d < a.D;
    r.p[q] = v ? a.proj[tok * a.P + d] : 0.f;
    r.pd[q] = v ? a.projd[tok * a.P + d] : 0.f;
    r.u[q] = v ? a.u[tok * a.D + d] : 0.f;
    r.ud[q] = v ? a.ud[tok * a.D + d] : 0.f;
    // B and C of the sub-chunk's tokens: 8 tokens x 32 values, two per thread
    const int bt = idx >> 5, j = idx & 31;  // idx < 512: token bt (0..15, only < ST used), value j
    const int64_t btok = s0 + bt;
    const bool bv = bt < ST && btok < l.e;
    r.bc[q] = bv ? a.proj[btok * a.P + a.D + j] : 0.f;
    r.bcd[q] = bv ? a.projd[btok * a.P + a.D + j] : 0.f;
  }
}

__device__ __forceinline__ void pref_store(const Pref& r, const Lane& l, Stage& st) {
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const int idx = l.tid + q * THREADS;
    const int t = idx / DC, dl = idx % DC;
    const float y = exp_neg_abs(r.p[q]);
    const float dt = softplus_from(r.p[q], y);
    st.dt[t][dl] = dt;
    st.dtd[t][dl] = sigmoid_from(r.p[q], y) * r.pd[q];
    st.rdt[t][dl] = rcpf(dt);
    st.u[t][dl] = r.u[q];
    st.ud[t][dl] = r.ud[q];
    const int bt = idx >> 5, j = idx & 31;
    if (bt < ST) {
      float* dB = j < NST ? reinterpret_cast<float*>(&st.B[bt][0]) + j : reinterpret_cast<float*>(&st.C[bt][0]) + (j - NST);
      float* dBd = j < NST ? reinterpret_cast<float*>(&st.Bd[bt][0]) + j
                           : reinterpret_cast<float*>(&st.Cd[bt][0]) + (j - NST);
      *dB = r.bc[q];
      *dBd = r.bcd[q];
    }
  }
}

// One step of the thread's states (and tangents) on staged token i.
__device__ __forceinline__ void step(const Stage& S, int i, const Lane& l, const AConst& K, float h[NS],
                                     float hd[NS]) {
  const float dt = S.dt[i][l.dl], dtd = S.dtd[i][l.dl], rdt = S.rdt[i][l.dl];
  const float uu = S.u[i][l.dl], ud = S.ud[i][l.dl];
  const float4 Bq = S.B[i][l.nq], Bdq = S.Bd[i][l.nq];
  const float Bv[NS] = {Bq.x, Bq.y, Bq.z, Bq.w}, Bdv[NS] = {Bdq.x, Bdq.y, Bdq.z, Bdq.w};
#pragma unroll
  for (int j = 0; j < NS; ++j) {
    const float z = dt * K.A[j], zd = dtd * K.A[j];
    const float e = ex2f(dt * K.A2[j]);
    const float rz = rdt * K.rA[j];
    const float p1 = phi1(z, e, rz);
    const float p1p = phi1p(z, e, p1, rz);
    const float bu = Bv[j] * uu;
    const float bdu = fmaf(Bdv[j], uu, Bv[j] * ud);
    hd[j] = fmaf(e, hd[j], fmaf(e * zd, h[j], fmaf(p1p * zd, bu, p1 * bdu)));
    h[j] = fmaf(e, h[j], p1 * bu);
  }
}

// ---- 1. chunk pass from a zero pair
__global__ void __launch_bounds__(THREADS) chunk_kernel(const Args a) {
  __shared__ Stage stg[2];
  const Lane l = lane_of(a);
  const AConst K = load_A(a, l.nq);
  float h[NS] = {0.f, 0.f, 0.f, 0.f}, hd[NS] = {0.f, 0.f, 0.f, 0.f};
  float S = 0.f, Sd = 0.f;
  const int nsub = int((l.e - l.s + ST - 1) / ST);
  Pref r;
  pref_load(a, l, l.s, r);
  pref_store(r, l, stg[0]);
  __syncthreads();
  for (int k = 0; k < nsub; ++k) {
    const int64_t rem = l.e - (l.s + int64_t(k) * ST);
    const int nt = rem < ST ? int(rem) : ST;
    if (k + 1 < nsub) pref_load(a, l, l.s + int64_t(k + 1) * ST, r);
    const Stage& St = stg[k & 1];
#pragma unroll
    for (int i = 0; i < ST; ++i)
      if (i < nt) {
        step(St, i, l, K, h, hd);
        S += St.dt[i][l.dl];
        Sd += St.dtd[i][l.dl];
      }
    if (k + 1 < nsub) pref_store(r, l, stg[(k + 1) & 1]);
    __syncthreads();
  }
  if (!l.ch) return;
  const int64_t o = (l.c * a.D + l.d) * NST + l.nq * NS;
#pragma unroll
  for (int j = 0; j < NS; ++j) {
    a.hloc[o + j] = h[j];
    a.hdloc[o + j] = hd[j];
  }
  if (l.nq == 0) {
    a.sdt[l.c * a.D + l.d] = S;
    a.sdtd[l.c * a.D + l.d] = Sd;
  }
}

// ---- 2. compose over chunks, one thread per (d, n)
__global__ void __launch_bounds__(256) compose_kernel(const Args a) {
  const int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= a.D * NST) return;
  const int n = int(idx % NST);
  const int64_t d = idx / NST;
  const float A = -expf(a.A_log[n]);
  float h = a.h0 ? a.h0[idx] : 0.f, hd = a.hd0 ? a.hd0[idx] : 0.f;
  for (int64_t c = 0; c < a.nC; ++c) {
    const int64_t o = c * a.D * NST + idx;
    a.hC[o] = h;
    a.hdC[o] = hd;
    const float S = a.sdt[c * a.D + d], Sd = a.sdtd[c * a.D + d];
    const float E = expf(A * S);
    const float Ed = E * A * Sd;
    const float hn = fmaf(E, h, a.hloc[o]);
    hd = fmaf(Ed, h, fmaf(E, hd, a.hdloc[o]));
    h = hn;
  }
  if (a.h_end) a.h_end[idx] = h;
  if (a.hd_end) a.hd_end[idx] = hd;
}

// ---- 3. output pass from the chunk start pairs
__global__ void __launch_bounds__(THREADS) out_kernel(const Args a) {
  __shared__ Stage stg[2];
  __shared__ float ybuf[2][ST][DC], ydbuf[2][ST][DC];
  const Lane l = lane_of(a);
  const AConst K = load_A(a, l.nq);
  float h[NS], hd[NS];
  const int64_t o = (l.c * a.D + (l.ch ? l.d : 0)) * NST + l.nq * NS;
#pragma unroll
  for (int j = 0; j < NS; ++j) {
    h[j] = l.ch ? a.hC[o + j] : 0.f;
    hd[j] = l.ch ? a.hdC[o + j] : 0.f;
  }
  const float Dd = l.ch ? a.Dp[l.d] : 0.f;
  const float sc = fmaxf(a.scale[0], 0.5f);
  const int nsub = int((l.e - l.s + ST - 1) / ST);
  Pref r;
  pref_load(a, l, l.s, r);
  pref_store(r, l, stg[0]);
  __syncthreads();
  for (int k = 0; k < nsub; ++k) {
    const int64_t rem = l.e - (l.s + int64_t(k) * ST);
    const int nt = rem < ST ? int(rem) : ST;
    if (k + 1 < nsub) pref_load(a, l, l.s + int64_t(k + 1) * ST, r);
    const Stage& St = stg[k & 1];
#pragma unroll
    for (int i = 0; i < ST; ++i) {
      if (i < nt) {
        step(St, i, l, K, h, hd);
        const float4 Cq = St.C[i][l.nq], Cdq = St.Cd[i][l.nq];
        const float Cv[NS] = {Cq.x, Cq.y, Cq.z, Cq.w}, Cdv[NS] = {Cdq.x, Cdq.y, Cdq.z, Cdq.w};
        float yc = 0.f, ydc = 0.f;
#pragma unroll
        for (int j = 0; j < NS; ++j) {
          yc = fmaf(Cv[j], h[j], yc);
          ydc = fmaf(Cdv[j], h[j], fmaf(Cv[j], hd[j], ydc));
        }
        yc += __shfl_xor_sync(0xffffffffu, yc, 1);
        yc += __shfl_xor_sync(0xffffffffu, yc, 2);
        ydc += __shfl_xor_sync(0xffffffffu, ydc, 1);
        ydc += __shfl_xor_sync(0xffffffffu, ydc, 2);
        if (l.nq == 0) {
          const float yr = fmaf(Dd, St.u[i][l.dl], yc);
          const float yrd = fmaf(Dd, St.ud[i][l.dl], ydc);
          const float ey = exp_neg_abs(yr);
          ybuf[k & 1][i][l.dl] = softplus_from(yr, ey) * sc;
          ydbuf[k & 1][i][l.dl] = sigmoid_from(yr, ey) * yrd * sc;
        }
      }
    }
    if (k + 1 < nsub) pref_store(r, l, stg[(k + 1) & 1]);
    __syncthreads();
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const int idx = l.tid + q * THREADS;
      const int t = idx / DC, dl = idx % DC;
      const int64_t tok = l.s + int64_t(k) * ST + t;
      const int64_t d = int64_t(l.grp) * DC + dl;
      if (tok < l.e && d < a.D) {
        a.y[tok * a.D + d] = ybuf[k & 1][t][dl];
        a.yd[tok * a.D + d] = ydbuf[k & 1][t][dl];
      }
    }
  }
}

struct Plan {
  int64_t L, D, P, Tc, nC, G;
};
static Plan plan_of(int64_t L, int64_t D) {
  Plan p;
  p.L = L;
  p.D = D;
  p.P = D + 2 * NST;
  p.G = (D + DC - 1) / DC;
  // chunks small enough that the chunk and output passes give every SM a few CTAs
  p.Tc = 128;
  const int64_t want = int64_t(sm_count()) * 4;
  while (p.Tc > 16 && ((L + p.Tc - 1) / p.Tc) * p.G < want) p.Tc /= 2;
  p.nC = (L + p.Tc - 1) / p.Tc;
  return p;
}
static size_t ws_bytes(const Plan& p) {
  const size_t L = size_t(p.L), P = size_t(p.P), st = size_t(p.nC) * p.D * NST, sd = size_t(p.nC) * p.D;
  return Workspace::round(L * P * 4) * 2 + Workspace::round(st * 4) * 4 + Workspace::round(sd * 4) * 2 + 1024;
}

}  // namespace fjvp
}  // namespace pgf

using namespace pgf;

extern "C" size_t pgf_frechet_jvp_workspace(int64_t L, int64_t D, int64_t N) {
  (void)N;
  return fjvp::ws_bytes(fjvp::plan_of(L < 1 ? 1 : L, D < 1 ? 1 : D));
}

extern "C" int pgf_frechet_jvp(const float* u, const float* u_dot, const float* W_cat, const float* b_cat,
                               const float* A_log, const float* Dp, const float* scale, const float* h0,
                               const float* h0_dot, float* y, float* y_dot, float* h_end, float* h_end_dot,
                               int64_t L, int64_t D, int64_t N, void* ws, size_t ws_bytes, pgf_stream_t stream) {
  using namespace fjvp;
  PGF_CHECK_ARG(N == NST, "frechet_jvp: d_state must be %d (got %lld)", NST, (long long)N);
  PGF_CHECK_ARG(L >= 0 && D > 0, "frechet_jvp: bad shape");
  PGF_CHECK_ARG(u && u_dot && W_cat && b_cat && A_log && Dp && scale && y && y_dot, "frechet_jvp: null pointer");
  cudaStream_t s = as_stream(stream);
  if (L == 0) {
    if (h_end) {
      if (h0) PGF_CUDA(cudaMemcpyAsync(h_end, h0, D * NST * 4, cudaMemcpyDeviceToDevice, s));
      else PGF_CUDA(cudaMemsetAsync(h_end, 0, D * NST * 4, s));
    }
    if (h_end_dot) {
      if (h0_dot) PGF_CUDA(cudaMemcpyAsync(h_end_dot, h0_dot, D * NST * 4, cudaMemcpyDeviceToDevice, s));
      else PGF_CUDA(cudaMemsetAsync(h_end_dot, 0, D * NST * 4, s));
    }
    return PGF_OK;
  }
  const Plan p = plan_of(L, D);
  Workspace W(ws, ws_bytes);
  Args a = {};
  a.L = L; a.D = D; a.P = p.P; a.Tc = p.Tc; a.nC = p.nC; a.G = p.G;
  a.u = u; a.ud = u_dot; a.A_log = A_log; a.Dp = Dp; a.scale = scale; a.h0 = h0; a.hd0 = h0_dot;
  float* proj = W.take<float>(size_t(L) * p.P);
  float* projd = W.take<float>(size_t(L) * p.P);
  const size_t st = size_t(p.nC) * D * NST, sd = size_t(p.nC) * D;
  a.hloc = W.take<float>(st); a.hdloc = W.take<float>(st);
  a.hC = W.take<float>(st); a.hdC = W.take<float>(st);
  a.sdt = W.take<float>(sd); a.sdtd = W.take<float>(sd);
  if (!proj || !projd || !a.hloc || !a.hdloc || !a.hC || !a.hdC || !a.sdt || !a.sdtd) {
    set_error("frechet_jvp: workspace too small (%zu)", ws_bytes);
    return PGF_ERR_WORKSPACE;
  }
  a.proj = proj; a.projd = projd; a.h_end = h_end; a.hd_end = h_end_dot; a.y = y; a.yd = y_dot;
  // [dt_in | B | C] = u W_cat^T + b_cat (pgf_mamba.py:92-94) and its tangent u_dot W_cat^T
  Gemm g = gemm_make(L, p.P, D, u, 0, D, 0, W_cat, 0, D, 0, proj, 0, p.P);
  g.epi.bias = b_cat;
  PGF_TRY(run_gemm(g, s));
  Gemm gd = gemm_make(L, p.P, D, u_dot, 0, D, 0, W_cat, 0, D, 0, projd, 0, p.P);
  PGF_TRY(run_gemm(gd, s));
  const dim3 grid(unsigned(p.nC), unsigned(p.G));
  chunk_kernel<<<grid, THREADS, 0, s>>>(a);
  PGF_LAUNCH_CHECK();
  compose_kernel<<<unsigned((D * NST + 255) / 256), 256, 0, s>>>(a);
  PGF_LAUNCH_CHECK();
  out_kernel<<<grid, THREADS, 0, s>>>(a);
  PGF_LAUNCH_CHECK();
  return PGF_OK;
}
