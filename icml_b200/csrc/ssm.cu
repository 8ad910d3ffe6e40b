// Selective-scan layer of SingleLayerMambaPGF (train_singlemamba_optimized.py:88-472) on sm_100a.
//
// Layout: u, y, g: (Bsz, L, D); proj = u W_cat^T + b_cat: (Bsz, L, P = D + 2N) float32 with
// columns [dt_in | B | C].  The recurrence h_t = exp(dt_t A) h_{t-1} + phi_1(dt_t A) B_t u_t runs
// per (batch, channel, state); a thread owns NS = 4 states of one channel, four adjacent lanes
// cover the N = 16 states, a CTA covers DC = 64 channels of one time chunk of Tc tokens.
//
// Inputs reach the kernels through shared memory, ST tokens at a time: the CTA loads the next
// sub-chunk into registers while it computes the current one, then stores it, already
// transformed once per (token, channel) -- dt = softplus(dt_in), 1/dt, delta_in -- so the four
// lanes of a channel never repeat that work.  exp(dt A_n) is exp2(dt * A_n log2 e) and 1/(dt A_n)
// is (1/dt)(1/A_n): no division per state.
//
// Forward (3 kernels): chunk summaries from a zero state (local end state + sum of dt, because
// prod_t exp(dt_t A_n) = exp(A_n sum_t dt_t)), a sequential compose over chunks giving every
// chunk's start state (the PGF boundary states), and the output pass re-running each chunk from
// its start state.
// Backward (3 kernels + 2 reductions): reverse chunk summaries of the adjoint
// delta_h_t = exp(dt_{t+1} A) delta_h_{t+1} + delta_in_t C_t from a zero carry, a reverse compose
// giving each chunk's incoming carry, and the main kernel: it re-runs the chunk from its boundary
// state keeping a checkpoint every ST tokens in shared memory, then walks the sub-chunks in
// reverse, re-running each one into registers (state and exp(dt A) per token) and stepping the
// adjoint back through it while it forms every gradient of _pass2_block_direct_grad (:350-472).
// Sums over channels (grad B, grad C) and over tokens (grad A_log, D, scale) go through
// fixed-order partial buffers: results are bitwise reproducible.
#include "gemm.cuh"
#include "scan_compose.cuh"
#include "f32x2.cuh"

namespace pgf {

constexpr int NST = 16;              // d_state
constexpr int NQ = 4;                // threads per channel
constexpr int NS = NST / NQ;         // states per thread
constexpr int NP = NS / 2;           // state pairs per thread (packed f32x2 arithmetic)
constexpr int DC = 64;               // channels per CTA
constexpr int SSM_THREADS = DC * NQ; // 256
constexpr int SSM_WARPS = SSM_THREADS / 32;
constexpr int ST = 8;                // tokens per staged sub-chunk (= backward register trajectory)
constexpr int TC_MAX = 128;
constexpr float LOG2E = 1.4426950408889634f;

struct SsmArgs {
  const void* u; int u_bf16;
  const float* proj;
  const void* g; int g_bf16;
  const float* A_log; const float* Dp; const float* scale;
  int act;
  int64_t Bsz, L, D, P, Tc, nC, G;
  const float* h_init;
  float* hloc; float* sdt; float* hC;
  float* dloc; float* sdt2; float* dt0; float* X;
  void* y; int y_bf16;
  float* actp;
  float* gstack; float* gu_scan; float* dbc_part;
  __nv_bfloat16* gstack_bf;  // bf16 copy of gstack (bf16 runs), operand of the tensor-core GEMMs
  float* partA; float* partD; float* partS;
  // states at the start of every ST-token sub-chunk, (Bsz, nC, Tc/ST, D, N): written by the output
  // pass when ckpt_write, read by the main backward kernel instead of its own forward pass
  float* ckpt_g; int ckpt_write;
  // zero-start forward (chunk_y0 / out_corr): y0 = C h0 per (token, channel), float32 (Bsz, L, D);
  // ckpt_s = sum of dt inside the chunk before each ST-token sub-chunk, (Bsz, nC, Tc/ST, D).  With
  // them the saved checkpoints hold zero-start states h0, and a state is h0 + exp(A S) H_chunk.
  float* y0;
  float* ckpt_s;
};

// One staged sub-chunk: ST tokens x DC channels (+ the token's B and C rows).
struct Stage {
  float dt[ST][DC];
  float rdt[ST][DC];
  float u[ST][DC];
  float gg[ST][DC];    // backward: incoming gradient g
  float dh[ST][DC];    // backward: delta_in_h = g * scale * act'(C h)
  float rs[ST][DC];    // backward: d dt / d dt_in divided by dt = sigmoid(dt_in) / softplus(dt_in)
  float4 B[ST][NQ];
  float4 C[ST][NQ];
};

// Registers that carry the next sub-chunk from global memory to the stage.
struct Pref {
  float dtin[2], u[2], g[2], ap[2], sc[2];
  float bc;
};

__device__ __forceinline__ float act_apply(int act, float x) {
  if (act == PGF_ACT_RELU) return x > 0.f ? x : 0.f;
  if (act == PGF_ACT_TANH) return tanhf(x);
  return x;
}
__device__ __forceinline__ float act_deriv(int act, float x) {
  if (act == PGF_ACT_RELU) return x > 0.f ? 1.f : 0.f;
  if (act == PGF_ACT_TANH) { float t = tanhf(x); return 1.f - t * t; }
  return 1.f;
}

struct Lane {
  int tid, dl, nq;
  int64_t c, b, d, s, e;
  int grp;
  bool ch;
};

__device__ __forceinline__ Lane lane_of(const SsmArgs& a) {
  Lane l;
  l.tid = threadIdx.x;
  l.dl = l.tid / NQ;
  l.nq = l.tid % NQ;
  l.c = blockIdx.x;
  l.b = blockIdx.y;
  l.grp = blockIdx.z;
  l.d = int64_t(l.grp) * DC + l.dl;
  l.ch = l.d < a.D;
  l.s = l.c * a.Tc;
  l.e = l.s + a.Tc < a.L ? l.s + a.Tc : a.L;
  return l;
}

// Tokens of sub-chunk k that lie inside the chunk (ST except in a ragged last sub-chunk).
__device__ __forceinline__ int sub_len(const Lane& l, int k) {
  const int64_t r = l.e - (l.s + int64_t(k) * ST);
  return r < ST ? int(r) : ST;
}

// per-thread state constants, as pairs of states: A_n, A_n log2(e), 1/A_n
struct AConst {
  float2 A[NP], A2[NP], rA[NP];
};
__device__ __forceinline__ AConst load_A(const SsmArgs& a, int nq) {
  AConst c;
#pragma unroll
  for (int p = 0; p < NP; ++p) {
    const float a0 = -expf(a.A_log[nq * NS + 2 * p]), a1 = -expf(a.A_log[nq * NS + 2 * p + 1]);
    c.A[p] = f2(a0, a1);
    c.A2[p] = f2(a0 * LOG2E, a1 * LOG2E);
    c.rA[p] = f2(1.0f / a0, 1.0f / a1);
  }
  return c;
}

// The thread's NS states of row `o` (o = first state) as pairs; stores likewise.
__device__ __forceinline__ void ld_states(const float* __restrict__ src, float2 v[NP]) {
  const float4 q = *reinterpret_cast<const float4*>(src);
  v[0] = lo2(q);
  v[1] = hi2(q);
}
__device__ __forceinline__ void st_states(float* __restrict__ dst, const float2 v[NP]) {
  *reinterpret_cast<float4*>(dst) = make_float4(v[0].x, v[0].y, v[1].x, v[1].y);
}

__device__ __forceinline__ void pref_load(const SsmArgs& a, const Lane& l, int64_t s0, bool bwd, Pref& r) {
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const int idx = l.tid + q * SSM_THREADS;
    const int t = idx / DC, dl = idx % DC;
    const int64_t tok = s0 + t;
    const int64_t d = int64_t(l.grp) * DC + dl;
    const bool v = tok < l.e && d < a.D;
    const int64_t row = l.b * a.L + tok;
    r.dtin[q] = v ? a.proj[row * a.P + d] : 0.f;
    r.u[q] = v ? ldv(a.u, a.u_bf16, row * a.D + d) : 0.f;
    if (bwd) {
      r.g[q] = v ? ldv(a.g, a.g_bf16, row * a.D + d) : 0.f;
      r.ap[q] = (v && a.actp) ? a.actp[row * a.D + d] : 1.f;
      r.sc[q] = v ? a.scale[d] : 0.f;
    }
  }
  {
    const int t = l.tid >> 5, j = l.tid & 31;
    const int64_t tok = s0 + t;
    r.bc = (t < ST && tok < l.e) ? a.proj[(l.b * a.L + tok) * a.P + a.D + j] : 0.f;
  }
}

__device__ __forceinline__ void pref_store(const Pref& r, const Lane& l, bool bwd, Stage& st) {
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const int idx = l.tid + q * SSM_THREADS;
    const int t = idx / DC, dl = idx % DC;
    const float y = exp_neg_abs(r.dtin[q]);
    const float dt = softplus_from(r.dtin[q], y);
    st.dt[t][dl] = dt;
    st.rdt[t][dl] = rcpf(dt);
    st.u[t][dl] = r.u[q];
    if (bwd) {
      st.gg[t][dl] = r.g[q];
      st.dh[t][dl] = r.g[q] * r.sc[q] * r.ap[q];
      // sigmoid(x) / softplus(x) tends to 1 as x -> -inf, where dt flushes to zero (and 1/dt to inf)
      st.rs[t][dl] = dt > 0.f ? sigmoid_from(r.dtin[q], y) * rcpf(dt) : 1.f;
    }
  }
  {
    const int t = l.tid >> 5, j = l.tid & 31;
    if (t < ST) {
      float* dst = j < NST ? reinterpret_cast<float*>(&st.B[t][0]) + j
                           : reinterpret_cast<float*>(&st.C[t][0]) + (j - NST);
      *dst = r.bc;
    }
  }
}

// Untransformed inputs of one backward sub-chunk, copied global -> shared by cp.async in 16-byte
// pieces two sub-chunks ahead of their use, so that no thread holds them in registers or waits for
// them: projection columns dt_in and [B | C], u and g (bf16 rows fill the first half of each row),
// act'(C h) with an output activation, and the forward's checkpoint (h0, S) of the 64 channels.
struct Raw {
  float dtin[ST][DC];
  float bc[ST][32];
  float u[ST][DC];
  float g[ST][DC];
  float ap[ST][DC];
  float ckh[DC * NST];
  float cks[DC];
};

__device__ __forceinline__ void cp16(void* dst, const void* src, bool valid) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(valid ? 16 : 0) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// Issue the copies of sub-chunk k into R (every thread takes every 256th 16-byte piece): dt_in and
// [B | C] always, u, g, act' and the checkpoint as `fl` asks (RAW_* bits; act' only when the
// layer has an output activation).  Pieces of tokens past the chunk or channels past D are
// zero-filled (nothing is read for them).  Needs D a multiple of 8 and 16-byte aligned rows (the
// host checks).
enum { RAW_U = 1, RAW_G = 2, RAW_AP = 4, RAW_CK = 8 };
__device__ __forceinline__ void raw_issue(const SsmArgs& a, const Lane& l, int k, Raw& R, int fl) {
  const int es = a.u_bf16 ? 2 : 4;
  const int pu = DC * es / 16;                      // pieces per token row of u (and of g)
  const int n_dt = ST * 16, n_bc = ST * 8;
  const int n_u = (fl & RAW_U) ? ST * pu : 0, n_g = (fl & RAW_G) ? ST * pu : 0;
  const int n_ap = ((fl & RAW_AP) && a.actp) ? ST * 16 : 0;
  const int n_ck = ((fl & RAW_CK) && a.ckpt_g) ? DC * NST / 4 + DC / 4 : 0;
  const int total = n_dt + n_bc + n_u + n_g + n_ap + n_ck;
  const int64_t t0 = l.s + int64_t(k) * ST, c0 = int64_t(l.grp) * DC;
  const int KS = int((a.Tc + ST - 1) / ST);
  const int64_t ck = (l.b * a.nC + l.c) * KS + k;
  for (int pc = l.tid; pc < total; pc += SSM_THREADS) {
    int q = pc;
    if (q < n_dt) {
      const int t = q >> 4, c = (q & 15) * 4;
      const int64_t tok = t0 + t;
      const bool v = tok < l.e && c0 + c < a.D;
      cp16(&R.dtin[t][c], v ? a.proj + (l.b * a.L + tok) * a.P + c0 + c : a.proj, v);
      continue;
    }
    q -= n_dt;
    if (q < n_bc) {
      const int t = q >> 3, c = (q & 7) * 4;
      const int64_t tok = t0 + t;
      const bool v = tok < l.e;
      cp16(&R.bc[t][c], v ? a.proj + (l.b * a.L + tok) * a.P + a.D + c : a.proj, v);
      continue;
    }
    q -= n_bc;
    if (q < n_u + n_g) {
      const bool isg = q >= n_u;
      if (isg) q -= n_u;
      const int t = q / pu, c = (q % pu) * (16 / es);
      const int64_t tok = t0 + t;
      const bool v = tok < l.e && c0 + c < a.D;
      const char* base = static_cast<const char*>(isg ? a.g : a.u);
      float* dst = isg ? &R.g[t][0] : &R.u[t][0];
      cp16(reinterpret_cast<char*>(dst) + c * es, v ? base + ((l.b * a.L + tok) * a.D + c0 + c) * es : base, v);
      continue;
    }
    q -= n_u + n_g;
    if (q < n_ap) {
      const int t = q >> 4, c = (q & 15) * 4;
      const int64_t tok = t0 + t;
      const bool v = tok < l.e && c0 + c < a.D;
      cp16(&R.ap[t][c], v ? a.actp + (l.b * a.L + tok) * a.D + c0 + c : a.actp, v);
      continue;
    }
    q -= n_ap;
    if (q < DC * NST / 4) {
      const int c = q >> 2;  // channel; four pieces of four states each
      const bool v = c0 + c < a.D;
      cp16(&R.ckh[q * 4], v ? a.ckpt_g + (ck * a.D + c0) * NST + q * 4 : a.ckpt_g, v);
      continue;
    }
    q -= DC * NST / 4;
    {
      const int c = q * 4;
      const bool v = c0 + c < a.D;
      cp16(&R.cks[c], v ? a.ckpt_s + ck * a.D + c0 + c : a.ckpt_s, v);
    }
  }
  cp_commit();
}

// The stage of a backward sub-chunk from its raw inputs (the transform of pref_store); sc_ch is the
// scale of the thread's write-out channel (the same channel for both of its slots).
__device__ __forceinline__ void raw_store(const SsmArgs& a, const Raw& R, const Lane& l, float sc_ch, Stage& st) {
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const int idx = l.tid + q * SSM_THREADS;
    const int t = idx / DC, dl = idx % DC;
    const float x = R.dtin[t][dl];
    const float uu = a.u_bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(&R.u[t][0])[dl]) : R.u[t][dl];
    const float gg = a.g_bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(&R.g[t][0])[dl]) : R.g[t][dl];
    const float ap = a.actp ? R.ap[t][dl] : 1.f;
    const float y = exp_neg_abs(x);
    const float dt = softplus_from(x, y);
    st.dt[t][dl] = dt;
    st.rdt[t][dl] = rcpf(dt);
    st.u[t][dl] = uu;
    st.gg[t][dl] = gg;
    st.dh[t][dl] = gg * sc_ch * ap;
    st.rs[t][dl] = dt > 0.f ? sigmoid_from(x, y) * rcpf(dt) : 1.f;
  }
  const int t = l.tid >> 5, j = l.tid & 31;
  if (t < ST) {
    float* dst = j < NST ? reinterpret_cast<float*>(&st.B[t][0]) + j
                         : reinterpret_cast<float*>(&st.C[t][0]) + (j - NST);
    *dst = R.bc[t][j];
  }
}

// Forward-order staging of a chunk's sub-chunks into stg[k & 1]: the inputs come through registers
// one sub-chunk ahead.  Per sub-chunk k: before(k), the compute on stg[k & 1], then after(k), which
// ends with the sub-chunk's barrier (stg[(k + 1) & 1] is then ready).  (Staging these by cp.async,
// as the backward kernels do, measured slower: they are issue-bound and rarely wait on loads.)
struct FwdStager {
  const SsmArgs& a;
  const Lane& l;
  Stage* stg;
  int nsub;
  Pref r;
  __device__ FwdStager(const SsmArgs& a_, const Lane& l_, Stage* stg_, int nsub_)
      : a(a_), l(l_), stg(stg_), nsub(nsub_) {}
  __device__ void begin() {
    pref_load(a, l, l.s, false, r);
    pref_store(r, l, false, stg[0]);
    __syncthreads();
  }
  __device__ void before(int k) {
    if (k + 1 < nsub) pref_load(a, l, l.s + int64_t(k + 1) * ST, false, r);
  }
  __device__ void after(int k) {
    if (k + 1 < nsub) pref_store(r, l, false, stg[(k + 1) & 1]);
    __syncthreads();
  }
};

// One forward step of the thread's NS states (as pairs) on staged token i:
// h = exp(dt A) h + phi_1(dt A) B u; returns phi_1(dt A) per state.
template <bool OUT_E = false>
__device__ __forceinline__ void step_fwd(const Stage& st, int i, int dl, int nq, const AConst& K,
                                         float2 h[NP], float2 p1_out[NP]) {
  const float2 dt = f2(st.dt[i][dl]), rdt = f2(st.rdt[i][dl]), uu = f2(st.u[i][dl]);
  const float4 Bq = st.B[i][nq];
  const float2 Bv[NP] = {lo2(Bq), hi2(Bq)};
#pragma unroll
  for (int p = 0; p < NP; ++p) {
    const float2 z = mul2(dt, K.A[p]);
    const float2 ez = ex2_2(mul2(dt, K.A2[p]));
    const float2 p1 = phi1_2(z, ez, mul2(rdt, K.rA[p]));
    h[p] = fma2(ez, h[p], mul2(mul2(p1, Bv[p]), uu));
    p1_out[p] = OUT_E ? ez : p1;
  }
}

// C . h over the thread's states (the pair sums, then the two lanes).
__device__ __forceinline__ float dot_c(const float4 Cq, const float2 h[NP]) {
  return hsum2(fma2(hi2(Cq), h[1], mul2(lo2(Cq), h[0])));
}

// ---------------------------------------------------------------------------------------------
// forward
// ---------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(SSM_THREADS) ssm_chunk_fwd_kernel(const SsmArgs a) {
  __shared__ Stage stg[2];
  const Lane l = lane_of(a);
  const AConst K = load_A(a, l.nq);
  float2 h[NP] = {f2(0.f), f2(0.f)}, e[NP];
  float sdt = 0.f;
  const int nsub = int((l.e - l.s + ST - 1) / ST);
  FwdStager fs(a, l, stg, nsub);
  fs.begin();
  for (int k = 0; k < nsub; ++k) {
    const int nt = sub_len(l, k);
    fs.before(k);
    const Stage& S = stg[k & 1];
#pragma unroll
    for (int i = 0; i < ST; ++i) {
      if (i < nt) {
        step_fwd(S, i, l.dl, l.nq, K, h, e);
        sdt += S.dt[i][l.dl];
      }
    }
    fs.after(k);
  }
  if (!l.ch) return;
  const int64_t cb = l.b * a.nC + l.c;
  st_states(a.hloc + (cb * a.D + l.d) * NST + l.nq * NS, h);
  if (l.nq == 0) a.sdt[cb * a.D + l.d] = sdt;
}

// Chunk start states: H_{c+1} = exp(A_n * sum_dt_c) H_c + hloc_c from h_init (or zero), segmented
// over the block's warps (scan_compose.cuh); optionally the end state and the total sum of dt.
__global__ void __launch_bounds__(32 * CSEG) ssm_compose_fwd_kernel(const SsmArgs a, float* __restrict__ h_final,
                                                                    float* __restrict__ sum_dt) {
  const int64_t idx = int64_t(blockIdx.x) * 32 + (threadIdx.x & 31);
  const bool valid = idx < a.Bsz * a.D * NST;
  const int64_t ii = valid ? idx : 0;
  const int n = int(ii % NST);
  const int64_t d = (ii / NST) % a.D;
  const int64_t b = ii / (NST * a.D);
  const float A2 = -expf(a.A_log[n]) * LOG2E;
  const float H0 = (valid && a.h_init) ? a.h_init[(b * a.D + d) * NST + n] : 0.f;
  float tot = 0.f;
  const float Hend = compose_fwd_segmented(valid, a.sdt + b * a.nC * a.D + d, a.D,
                                           a.hloc + (b * a.nC * a.D + d) * NST + n, a.D * NST,
                                           a.hC + (b * (a.nC + 1) * a.D + d) * NST + n, A2, H0, a.nC, &tot);
  if (valid && threadIdx.x < 32) {
    if (h_final) h_final[(b * a.D + d) * NST + n] = Hend;
    if (sum_dt && n == 0) sum_dt[b * a.D + d] = tot;
  }
}

// Forward in two light passes instead of summary + full re-run.  The recurrence is linear in the
// state: from the chunk's true start state H, h_t = h0_t + exp(A S_t) H with h0 the trajectory
// from a zero state and S_t the sum of dt over the chunk's tokens up to t.  Pass 1 (this kernel)
// runs the chunk from zero: its end state and sum of dt (the compose inputs), y0 = C h0 for every
// token and, when checkpoints are kept, h0 and S at every sub-chunk start.  Pass 2
// (ssm_out_corr_kernel) adds C_t (exp(A S_t) H) -- an exp2 and two FMAs per state instead of the
// whole step -- and forms the output.
__global__ void __launch_bounds__(SSM_THREADS) ssm_chunk_y0_kernel(const SsmArgs a) {
  __shared__ Stage stg[2];
  __shared__ float ybuf[2][ST][DC];
  const Lane l = lane_of(a);
  const AConst K = load_A(a, l.nq);
  float2 h[NP] = {f2(0.f), f2(0.f)}, e[NP];
  float sdt = 0.f;
  const int nsub = int((l.e - l.s + ST - 1) / ST);
  const int KS = int((a.Tc + ST - 1) / ST);
  FwdStager fs(a, l, stg, nsub);
  fs.begin();
  for (int k = 0; k < nsub; ++k) {
    const int nt = sub_len(l, k);
    fs.before(k);
    if (a.ckpt_write && l.ch) {
      const int64_t ck = (l.b * a.nC + l.c) * KS + k;
      st_states(a.ckpt_g + (ck * a.D + l.d) * NST + l.nq * NS, h);
      if (l.nq == 0) a.ckpt_s[ck * a.D + l.d] = sdt;
    }
    const Stage& S = stg[k & 1];
#pragma unroll
    for (int i = 0; i < ST; ++i) {
      if (i < nt) {
        step_fwd(S, i, l.dl, l.nq, K, h, e);
        sdt += S.dt[i][l.dl];
        float yc = dot_c(S.C[i][l.nq], h);
        yc += __shfl_xor_sync(0xffffffffu, yc, 1);
        yc += __shfl_xor_sync(0xffffffffu, yc, 2);
        if (l.nq == 0) ybuf[k & 1][i][l.dl] = yc;
      }
    }
    fs.after(k);
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const int idx = l.tid + q * SSM_THREADS;
      const int t = idx / DC, dl = idx % DC;
      const int64_t tok = l.s + int64_t(k) * ST + t;
      const int64_t d = int64_t(l.grp) * DC + dl;
      if (tok < l.e && d < a.D) a.y0[(l.b * a.L + tok) * a.D + d] = ybuf[k & 1][t][dl];
    }
  }
  if (!l.ch) return;
  const int64_t cb = l.b * a.nC + l.c;
  st_states(a.hloc + (cb * a.D + l.d) * NST + l.nq * NS, h);
  if (l.nq == 0) a.sdt[cb * a.D + l.d] = sdt;
}

// Pass 2 of the forward: y = (act(y0 + C_t (exp(A S_t) H)) + D u) scale, H the chunk's start state.
__global__ void __launch_bounds__(SSM_THREADS) ssm_out_corr_kernel(const SsmArgs a) {
  __shared__ Stage stg[2];
  __shared__ float ybuf[2][ST][DC];
  const Lane l = lane_of(a);
  const AConst K = load_A(a, l.nq);
  float2 H[NP] = {f2(0.f), f2(0.f)};
  if (l.ch) ld_states(a.hC + ((l.b * (a.nC + 1) + l.c) * a.D + l.d) * NST + l.nq * NS, H);
  float S_run = 0.f;
  const int nsub = int((l.e - l.s + ST - 1) / ST);
  // write-out operands of this thread's two (token, channel) slots per sub-chunk -- the slots its
  // staging loads cover -- held in registers: u from those loads, y0 loaded with them (a sub-chunk
  // ahead), D and scale of its fixed channel
  const int64_t d_out = int64_t(l.grp) * DC + l.tid % DC;
  const float D_out = d_out < a.D ? a.Dp[d_out] : 0.f, sc_out = d_out < a.D ? a.scale[d_out] : 0.f;
  auto load_y0 = [&](int64_t s0, float y0v[2]) {
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const int64_t tok = s0 + (l.tid + q * SSM_THREADS) / DC;
      y0v[q] = (tok < l.e && d_out < a.D) ? a.y0[(l.b * a.L + tok) * a.D + d_out] : 0.f;
    }
  };
  float y0c[2], y0n[2], uc[2];
  FwdStager fs(a, l, stg, nsub);
  load_y0(l.s, y0c);
  fs.begin();
  for (int k = 0; k < nsub; ++k) {
    const int nt = sub_len(l, k);
    fs.before(k);
    if (k + 1 < nsub) load_y0(l.s + int64_t(k + 1) * ST, y0n);
    const Stage& S = stg[k & 1];
    // u of the thread's write-out slots, from the stage before the barrier lets it be refilled
#pragma unroll
    for (int q = 0; q < 2; ++q) uc[q] = S.u[(l.tid + q * SSM_THREADS) / DC][l.tid % DC];
#pragma unroll
    for (int i = 0; i < ST; ++i) {
      if (i < nt) {
        S_run += S.dt[i][l.dl];
        const float2 s2 = f2(S_run);
        const float2 hs[NP] = {mul2(ex2_2(mul2(K.A2[0], s2)), H[0]), mul2(ex2_2(mul2(K.A2[1], s2)), H[1])};
        float yc = dot_c(S.C[i][l.nq], hs);
        yc += __shfl_xor_sync(0xffffffffu, yc, 1);
        yc += __shfl_xor_sync(0xffffffffu, yc, 2);
        if (l.nq == 0) ybuf[k & 1][i][l.dl] = yc;
      }
    }
    fs.after(k);
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const int idx = l.tid + q * SSM_THREADS;
      const int t = idx / DC, dl = idx % DC;
      const int64_t tok = l.s + int64_t(k) * ST + t;
      if (tok < l.e && d_out < a.D) {
        const int64_t o = (l.b * a.L + tok) * a.D + d_out;
        const float yc = y0c[q] + ybuf[k & 1][t][dl];
        stv(a.y, a.y_bf16, o, (act_apply(a.act, yc) + D_out * uc[q]) * sc_out);
      }
    }
    if (k + 1 < nsub) {
      y0c[0] = y0n[0]; y0c[1] = y0n[1];
    }
  }
}

__global__ void __launch_bounds__(SSM_THREADS) ssm_out_fwd_kernel(const SsmArgs a) {
  __shared__ Stage stg[2];
  __shared__ float ybuf[2][ST][DC];
  const Lane l = lane_of(a);
  const AConst K = load_A(a, l.nq);
  float2 h[NP] = {f2(0.f), f2(0.f)}, e[NP];
  if (l.ch) ld_states(a.hC + ((l.b * (a.nC + 1) + l.c) * a.D + l.d) * NST + l.nq * NS, h);
  const float2 h_start[NP] = {h[0], h[1]};
  // D and scale only enter the output (a.y); the act'(C h) mode (a.y == nullptr) may run without them
  const float Dd = (l.ch && a.y) ? a.Dp[l.d] : 0.f;
  const float sc = (l.ch && a.y) ? a.scale[l.d] : 0.f;
  const int nsub = int((l.e - l.s + ST - 1) / ST);
  FwdStager fs(a, l, stg, nsub);
  fs.begin();
  const int KS = int((a.Tc + ST - 1) / ST);
  for (int k = 0; k < nsub; ++k) {
    const int nt = sub_len(l, k);
    fs.before(k);
    if (a.ckpt_write && l.ch) {
      const int64_t ck = (l.b * a.nC + l.c) * KS + k;
      if (a.ckpt_write == 2) {
        // the layout the main backward reads: a state is ckpt + exp(A S) H_chunk; with S = 0 the
        // checkpoint is the state's offset from the chunk start state
        const float2 off[NP] = {fma2(h_start[0], f2(-1.f), h[0]), fma2(h_start[1], f2(-1.f), h[1])};
        st_states(a.ckpt_g + (ck * a.D + l.d) * NST + l.nq * NS, off);
        if (l.nq == 0) a.ckpt_s[ck * a.D + l.d] = 0.f;
      } else {
        st_states(a.ckpt_g + (ck * a.D + l.d) * NST + l.nq * NS, h);
      }
    }
    const Stage& S = stg[k & 1];
#pragma unroll
    for (int i = 0; i < ST; ++i) {
      if (i < nt) {
        step_fwd(S, i, l.dl, l.nq, K, h, e);
        float yc = dot_c(S.C[i][l.nq], h);
        yc += __shfl_xor_sync(0xffffffffu, yc, 1);
        yc += __shfl_xor_sync(0xffffffffu, yc, 2);
        if (l.nq == 0) {
          ybuf[k & 1][i][l.dl] = a.y ? (act_apply(a.act, yc) + Dd * S.u[i][l.dl]) * sc
                                     : act_deriv(a.act, yc);
        }
      }
    }
    fs.after(k);
    // coalesced write-out of the sub-chunk (y, or act'(C h) for the backward)
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const int idx = l.tid + q * SSM_THREADS;
      const int t = idx / DC, dl = idx % DC;
      const int64_t tok = l.s + int64_t(k) * ST + t;
      const int64_t d = int64_t(l.grp) * DC + dl;
      if (tok < l.e && d < a.D) {
        const int64_t o = (l.b * a.L + tok) * a.D + d;
        if (a.y) stv(a.y, a.y_bf16, o, ybuf[k & 1][t][dl]);
        else a.actp[o] = ybuf[k & 1][t][dl];
      }
    }
  }
}

// ---------------------------------------------------------------------------------------------
// backward
// ---------------------------------------------------------------------------------------------
// Bytes of a Raw buffer the adjoint-only pass uses (its leading fields up to act'; u is not filled).
constexpr size_t RAW_ADJ_BYTES = offsetof(Raw, ckh);
__device__ __forceinline__ Raw& raw_at(float* smr, size_t stride, int k) {
  return *reinterpret_cast<Raw*>(reinterpret_cast<char*>(smr) + (k & 1) * stride);
}

// The parts of a backward stage the adjoint-only pass reads (dt, delta_in_h, C) from raw inputs.
__device__ __forceinline__ void raw_store_adj(const SsmArgs& a, const Raw& R, const Lane& l, float sc_ch, Stage& st) {
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const int idx = l.tid + q * SSM_THREADS;
    const int t = idx / DC, dl = idx % DC;
    const float gg = a.g_bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(&R.g[t][0])[dl]) : R.g[t][dl];
    const float ap = a.actp ? R.ap[t][dl] : 1.f;
    st.dt[t][dl] = softplus_fast(R.dtin[t][dl]);
    st.dh[t][dl] = gg * sc_ch * ap;
  }
  const int t = l.tid >> 5, j = l.tid & 31;
  if (t < ST && j >= NST) reinterpret_cast<float*>(&st.C[t][0])[j - NST] = R.bc[t][j];
}

// Reverse chunk summaries of the adjoint from a zero carry.  ASYNC (D a multiple of 8, aligned rows):
// inputs staged by cp.async into two Raw buffers in dynamic shared memory, three sub-chunks ahead
// of their use, one barrier per sub-chunk.
template <bool ASYNC>
__global__ void __launch_bounds__(SSM_THREADS, 4) ssm_chunk_bwd_kernel(const SsmArgs a) {
  extern __shared__ __align__(16) float smr[];
  __shared__ Stage stg[2];
  auto raw = [&](int k) -> Raw& { return raw_at(smr, RAW_ADJ_BYTES, k); };
  const Lane l = lane_of(a);
  const AConst K = load_A(a, l.nq);
  float2 dlt[NP] = {f2(0.f), f2(0.f)};
  float2 anext[NP] = {f2(1.f), f2(1.f)};
  float sdt2 = 0.f, dt_first = 0.f;
  const int nsub = int((l.e - l.s + ST - 1) / ST);
  const int64_t c_out = int64_t(l.grp) * DC + l.tid % DC;
  const float sc_ch = c_out < a.D ? a.scale[c_out] : 0.f;
  Pref r;
  if (ASYNC) {
    raw_issue(a, l, nsub - 1, raw(nsub - 1), RAW_G | RAW_AP);
    if (nsub > 1) raw_issue(a, l, nsub - 2, raw(nsub - 2), RAW_G | RAW_AP);
    cp_wait_all();
    __syncthreads();
    raw_store_adj(a, raw(nsub - 1), l, sc_ch, stg[(nsub - 1) & 1]);
    __syncthreads();
    if (nsub > 2) raw_issue(a, l, nsub - 3, raw(nsub - 3), RAW_G | RAW_AP);
  } else {
    pref_load(a, l, l.s + int64_t(nsub - 1) * ST, true, r);
    pref_store(r, l, true, stg[(nsub - 1) & 1]);
    __syncthreads();
  }
  for (int k = nsub - 1; k >= 0; --k) {
    if (!ASYNC && k > 0) pref_load(a, l, l.s + int64_t(k - 1) * ST, true, r);
    const Stage& S = stg[k & 1];
#pragma unroll
    for (int i = ST - 1; i >= 0; --i) {
      const int64_t t = l.s + int64_t(k) * ST + i;
      if (t < l.e) {
        const float dt = S.dt[i][l.dl];
        const float2 dh = f2(S.dh[i][l.dl]);
        const float4 Cq = S.C[i][l.nq];
        const float2 Cv[NP] = {lo2(Cq), hi2(Cq)};
#pragma unroll
        for (int p = 0; p < NP; ++p) {
          dlt[p] = fma2(anext[p], dlt[p], mul2(dh, Cv[p]));
          anext[p] = ex2_2(mul2(f2(dt), K.A2[p]));
        }
        if (t > l.s) sdt2 += dt;
        dt_first = dt;
      }
    }
    if (ASYNC) {
      // stage k-1 from its raw inputs (landed by the previous barrier); raw k-2 lands by this one
      if (k > 0) raw_store_adj(a, raw(k - 1), l, sc_ch, stg[(k - 1) & 1]);
      cp_wait_all();
      __syncthreads();
      if (k > 2) raw_issue(a, l, k - 3, raw(k - 3), RAW_G | RAW_AP);
    } else {
      if (k > 0) pref_store(r, l, true, stg[(k - 1) & 1]);
      __syncthreads();
    }
  }
  if (!l.ch) return;
  const int64_t cb = l.b * a.nC + l.c;
  st_states(a.dloc + (cb * a.D + l.d) * NST + l.nq * NS, dlt);
  if (l.nq == 0) {
    a.sdt2[cb * a.D + l.d] = sdt2;
    a.dt0[cb * a.D + l.d] = dt_first;
  }
}

// Launch of the reverse chunk summaries: the cp.async form when the rows allow it.
static int launch_chunk_bwd(const SsmArgs& a, dim3 grid, cudaStream_t s) {
  auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  const bool async = a.D % 8 == 0 && al16(a.proj) && al16(a.g) && (!a.actp || al16(a.actp));
  if (async) {
    static int lim = 0;
    PGF_CUDA(ensure_dynamic_smem(ssm_chunk_bwd_kernel<true>, 2 * RAW_ADJ_BYTES, lim));
    ssm_chunk_bwd_kernel<true><<<grid, SSM_THREADS, 2 * RAW_ADJ_BYTES, s>>>(a);
  } else {
    ssm_chunk_bwd_kernel<false><<<grid, SSM_THREADS, 0, s>>>(a);
  }
  PGF_LAUNCH_CHECK();
  return PGF_OK;
}

// Adjoint carries X entering each chunk from the right, from (dh_end, dA_end) or (0, 1), segmented
// over the block's warps (scan_compose.cuh); optionally the carry and decay at the first token
// (dh_start, dA_start) and the sum of dt over every token but the first.
__global__ void __launch_bounds__(32 * CSEG) ssm_compose_bwd_kernel(const SsmArgs a, const float* __restrict__ dh_end,
                                                                    const float* __restrict__ dA_end,
                                                                    float* __restrict__ dh_start,
                                                                    float* __restrict__ dA_start,
                                                                    float* __restrict__ sum_dt_excl) {
  __shared__ float sSum[CSEG][32];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int64_t idx = int64_t(blockIdx.x) * 32 + lane;
  const bool valid = idx < a.Bsz * a.D * NST;
  const int64_t ii = valid ? idx : 0;
  const int n = int(ii % NST);
  const int64_t d = (ii / NST) % a.D;
  const int64_t b = ii / (NST * a.D);
  const float A2 = -expf(a.A_log[n]) * LOG2E;
  const int64_t o = (b * a.D + d) * NST + n;
  const float* sdt2 = a.sdt2 + b * a.nC * a.D + d;
  const float* dt0 = a.dt0 + b * a.nC * a.D + d;
  const float G_end = (valid && dh_end) ? dh_end[o] : 0.f;
  const float aE_end = (valid && dA_end) ? dA_end[o] : 1.f;
  float aE0 = 1.f;
  const float G0 = compose_bwd_segmented(valid, sdt2, dt0, a.D, a.dloc + (b * a.nC * a.D + d) * NST + n, a.D * NST,
                                         a.X + (b * a.nC * a.D + d) * NST + n, A2, G_end, aE_end, a.nC, &aE0);
  if (valid && w == 0) {
    if (dh_start) dh_start[o] = G0;
    if (dA_start) dA_start[o] = aE0;
  }
  if (sum_dt_excl) {
    // sum of dt over every token but the first: the within-chunk sums plus the later chunks' first dt,
    // per run of chunks, then the runs in order
    const int64_t run = (a.nC + CSEG - 1) / CSEG;
    const int64_t c0 = w * run < a.nC ? w * run : a.nC;
    const int64_t c1 = c0 + run < a.nC ? c0 + run : a.nC;
    float t = 0.f;
    if (valid && n == 0)
      for (int64_t k = c0; k < c1; ++k) t += sdt2[k * a.D] + (k > 0 ? dt0[k * a.D] : 0.f);
    sSum[w][lane] = t;
    __syncthreads();
    if (valid && w == 0 && n == 0) {
      float tot = 0.f;
      for (int v = 0; v < CSEG; ++v) tot += sSum[v][lane];
      sum_dt_excl[b * a.D + d] = tot;
    }
  }
}

// Main backward kernel.  Shared memory (dynamic): ckpt [Tc/ST][SSM_THREADS][NS] floats (only when
// the forward's checkpoints are not given), then red [ST][SSM_WARPS][32], then gbuf [2][ST][DC]
// (grad_dt_in, grad_u_scan of the sub-chunk).
//
// Per state and token the adjoint step needs h_{t-1}, h_t, phi_1(z) and e^z (z = dt A).  The
// sub-chunk re-run keeps h and phi_1 of every token in registers, and e^z = 1 + z phi_1 is rebuilt
// from them (absolute error ~1e-7; the decays are <= 1), so phi_1 is evaluated once per state update
// and no exponential runs in the adjoint loop.  The z-derivative of the step,
// dh_t/dz = e^z h_{t-1} + phi_1'(z) B u, enters the gradients only through
//   w = delta_h z dh_t/dz = delta_h (z e^z h_{t-1} + (e^z - phi_1) B u)     (z phi_1'(z) = e^z - phi_1)
// as grad A_log_n = sum w (dz/dA_log = z) and grad dt = sum_n w / dt (dz/ddt = A = z/dt), so phi_1'
// is never formed.  Both passes step the thread's states as packed f32x2 pairs.
//
// ASYNC (saved checkpoints, D a multiple of 8, aligned rows): the inputs of each sub-chunk arrive by
// cp.async into two Raw buffers after gbuf (see Raw), issued two sub-chunks ahead; otherwise they
// are prefetched through registers one sub-chunk ahead.
template <bool ASYNC>
__global__ void __launch_bounds__(SSM_THREADS, 2) ssm_main_bwd_kernel(const SsmArgs a) {
  extern __shared__ __align__(16) float sm[];
  __shared__ Stage stg[2];
  const Lane l = lane_of(a);
  const int KS = int((a.Tc + ST - 1) / ST);
  const bool saved = ASYNC || a.ckpt_g != nullptr;  // checkpoints come from the forward output pass
  float* ckpt = sm;
  float* red = ckpt + (saved ? size_t(0) : size_t(KS) * SSM_THREADS * NS);
  float* gbuf = red + ST * SSM_WARPS * 32;  // [2][ST][DC]
  Raw* raw = reinterpret_cast<Raw*>(gbuf + 2 * 2 * ST * DC);  // [2], ASYNC only
  const int lane = l.tid & 31, warp = l.tid >> 5;
  const AConst K = load_A(a, l.nq);
  // one forward step of the thread's state pairs on staged token i; p1o = phi_1(dt A) per state
  auto step = [&](const Stage& st, int i, float2 hh[NP], float2 p1o[NP]) {
    const float2 dt = f2(st.dt[i][l.dl]), rdt = f2(st.rdt[i][l.dl]), uu = f2(st.u[i][l.dl]);
    const float4 Bq = st.B[i][l.nq];
    const float2 Bv[NP] = {lo2(Bq), hi2(Bq)};
#pragma unroll
    for (int p = 0; p < NP; ++p) {
      const float2 z = mul2(dt, K.A[p]);
      const float2 ez = ex2_2(mul2(dt, K.A2[p]));
      const float2 p1 = phi1_2(z, ez, mul2(rdt, K.rA[p]));
      hh[p] = fma2(ez, hh[p], mul2(p1, mul2(Bv[p], uu)));
      p1o[p] = p1;
    }
  };
  const float Dd = l.ch ? a.Dp[l.d] : 0.f;
  const float sc = l.ch ? a.scale[l.d] : 0.f;  // in a register: the loop's stores may alias a.scale
  const int64_t cb = l.b * a.nC + l.c;
  const int nsub = int((l.e - l.s + ST - 1) / ST);

  float2 h[NP] = {f2(0.f), f2(0.f)}, carry[NP] = {f2(0.f), f2(0.f)};
  if (l.ch) {
    ld_states(a.hC + ((l.b * (a.nC + 1) + l.c) * a.D + l.d) * NST + l.nq * NS, h);
    ld_states(a.X + (cb * a.D + l.d) * NST + l.nq * NS, carry);
  }
  // ---- pass 1 (no saved checkpoints): forward through the chunk, checkpoint every sub-chunk start
  Pref r;
  if (!saved) {
    pref_load(a, l, l.s, false, r);
    pref_store(r, l, false, stg[0]);
    __syncthreads();
    float2 unused[NP];
    for (int k = 0; k < nsub; ++k) {
      if (k + 1 < nsub) pref_load(a, l, l.s + int64_t(k + 1) * ST, false, r);
      st_states(ckpt + (size_t(k) * SSM_THREADS + l.tid) * NS, h);
      const Stage& S = stg[k & 1];
#pragma unroll
      for (int i = 0; i < ST; ++i)
        if (l.s + int64_t(k) * ST + i < l.e) step(S, i, h, unused);
      if (k + 1 < nsub) pref_store(r, l, false, stg[(k + 1) & 1]);
      __syncthreads();
    }
  }

  // ---- pass 2: sub-chunks in reverse
  // saved checkpoints (zero-start h0 and S), loaded one sub-chunk ahead so the re-run never waits
  float2 ck_h[NP] = {f2(0.f), f2(0.f)};
  float ck_s = 0.f;
  auto ckpt_at = [&](int kk) {
    if (!l.ch) return;
    const int64_t ck = (l.b * a.nC + l.c) * KS + kk;
    ld_states(a.ckpt_g + (ck * a.D + l.d) * NST + l.nq * NS, ck_h);
    ck_s = a.ckpt_s[ck * a.D + l.d];
  };
  // ASYNC: the start state of the next sub-chunk to run, formed from its raw checkpoint when its
  // stage is filled (the raw buffer is refilled before that sub-chunk runs)
  float2 tr0n[NP] = {f2(0.f), f2(0.f)};
  const float sc_ch = (int64_t(l.grp) * DC + l.tid % DC) < a.D ? a.scale[int64_t(l.grp) * DC + l.tid % DC] : 0.f;
  auto fill = [&](int kk) {  // stage kk from raw buffer kk & 1 (ASYNC)
    const Raw& R = raw[kk & 1];
    raw_store(a, R, l, sc_ch, stg[kk & 1]);
    const float4 q = *reinterpret_cast<const float4*>(&R.ckh[l.dl * NST + l.nq * NS]);
    const float2 s2 = f2(R.cks[l.dl]);
    tr0n[0] = l.ch ? fma2(ex2_2(mul2(K.A2[0], s2)), h[0], lo2(q)) : f2(0.f);
    tr0n[1] = l.ch ? fma2(ex2_2(mul2(K.A2[1], s2)), h[1], hi2(q)) : f2(0.f);
  };
  if (!ASYNC && saved) ckpt_at(nsub - 1);
  float2 accA[NP] = {f2(0.f), f2(0.f)};
  float accD = 0.f, accS = 0.f;
  const int b4 = (lane >> 4) & 1, b3 = (lane >> 3) & 1, b2 = (lane >> 2) & 1;
  if (ASYNC) {
    raw_issue(a, l, nsub - 1, raw[(nsub - 1) & 1], RAW_U | RAW_G | RAW_AP | RAW_CK);
    cp_wait_all();
    __syncthreads();
    fill(nsub - 1);
    __syncthreads();
    if (nsub > 1) raw_issue(a, l, nsub - 2, raw[(nsub - 2) & 1], RAW_U | RAW_G | RAW_AP | RAW_CK);
  } else {
    pref_load(a, l, l.s + int64_t(nsub - 1) * ST, true, r);
    pref_store(r, l, true, stg[(nsub - 1) & 1]);
    __syncthreads();
  }
  for (int k = nsub - 1; k >= 0; --k) {
    if (!ASYNC && k > 0) pref_load(a, l, l.s + int64_t(k - 1) * ST, true, r);
    const Stage& S = stg[k & 1];
    float* gb = gbuf + (k & 1) * (2 * ST * DC);
    // re-run the sub-chunk into registers: tr[i] = state before token i, ph[i] = phi_1(dt_i A)
    float2 tr[ST + 1][NP], ph[ST][NP];
    if (ASYNC) {
      tr[0][0] = tr0n[0];
      tr[0][1] = tr0n[1];
    } else if (saved) {
      // zero-start checkpoint h0 of the forward (prefetched one sub-chunk ahead), moved onto the
      // chunk's start state h (= hC): state = h0 + exp(A S) h, S = sum of dt before this sub-chunk
      const float2 s2 = f2(ck_s);
#pragma unroll
      for (int p = 0; p < NP; ++p) tr[0][p] = l.ch ? fma2(ex2_2(mul2(K.A2[p], s2)), h[p], ck_h[p]) : f2(0.f);
      if (k > 0) ckpt_at(k - 1);
    } else {
      ld_states(ckpt + (size_t(k) * SSM_THREADS + l.tid) * NS, tr[0]);
    }
#pragma unroll
    for (int i = 0; i < ST; ++i) {
#pragma unroll
      for (int p = 0; p < NP; ++p) {
        tr[i + 1][p] = tr[i][p];
        ph[i][p] = f2(0.f);
      }
      if (l.s + int64_t(k) * ST + i < l.e) step(S, i, tr[i + 1], ph[i]);
    }
#pragma unroll
    for (int i = ST - 1; i >= 0; --i) {
      const bool valid = l.s + int64_t(k) * ST + i < l.e;  // uniform across the CTA
      float2 vB[NP] = {f2(0.f), f2(0.f)}, vC[NP] = {f2(0.f), f2(0.f)};
      float2 ws = f2(0.f), gu2 = f2(0.f), hc2 = f2(0.f);
      if (valid) {
        const float2 dt = f2(S.dt[i][l.dl]), uu = f2(S.u[i][l.dl]), dh = f2(S.dh[i][l.dl]);
        const float4 Bq = S.B[i][l.nq], Cq = S.C[i][l.nq];
        const float2 Bv[NP] = {lo2(Bq), hi2(Bq)};
        const float2 Cv[NP] = {lo2(Cq), hi2(Cq)};
#pragma unroll
        for (int p = 0; p < NP; ++p) {
          const float2 z = mul2(dt, K.A[p]);
          const float2 E = fma2(z, ph[i][p], f2(1.f));        // e^z = 1 + z phi_1
          const float2 dlt = fma2(dh, Cv[p], carry[p]);       // delta_h_t
          const float2 pd = mul2(dlt, ph[i][p]);
          gu2 = fma2(pd, Bv[p], gu2);                         // grad u (scan part)
          vB[p] = mul2(pd, uu);                               // grad B, this channel's term
          vC[p] = mul2(dh, tr[i + 1][p]);                     // grad C, this channel's term
          hc2 = fma2(Cv[p], tr[i + 1][p], hc2);               // C h_t
          const float2 em = fma2(ph[i][p], f2(-1.f), E);      // e^z - phi_1 = z phi_1'(z)
          const float2 t = fma2(mul2(z, E), tr[i][p], mul2(em, mul2(Bv[p], uu)));
          const float2 w = mul2(dlt, t);
          accA[p] = add2(accA[p], w);
          ws = add2(ws, w);
          carry[p] = mul2(E, dlt);
        }
      }
      float gdt = hsum2(ws), gur = hsum2(gu2), hc = hsum2(hc2);
      gdt += __shfl_xor_sync(0xffffffffu, gdt, 1);
      gdt += __shfl_xor_sync(0xffffffffu, gdt, 2);
      gur += __shfl_xor_sync(0xffffffffu, gur, 1);
      gur += __shfl_xor_sync(0xffffffffu, gur, 2);
      hc += __shfl_xor_sync(0xffffffffu, hc, 1);
      hc += __shfl_xor_sync(0xffffffffu, hc, 2);
      if (valid && l.nq == 0) {
        const float gg = S.gg[i][l.dl], uu = S.u[i][l.dl];
        const float din = gg * sc;
        gb[i * DC + l.dl] = gdt * S.rs[i][l.dl];  // (sum_n w / dt) sigmoid(dt_in)
        gb[ST * DC + i * DC + l.dl] = din * Dd + gur;
        accD = fmaf(din, uu, accD);
        accS = fmaf(gg, act_apply(a.act, hc) + Dd * uu, accS);
      }
      // sum the 8 grad-B / grad-C terms over the warp's 8 channels (lane bits 2..4)
      const float v8[8] = {vB[0].x, vB[0].y, vB[1].x, vB[1].y, vC[0].x, vC[0].y, vC[1].x, vC[1].y};
      float w4[4], w2[2];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float keep = b4 ? v8[4 + q] : v8[q];
        const float send = b4 ? v8[q] : v8[4 + q];
        w4[q] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
      }
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const float keep = b3 ? w4[2 + q] : w4[q];
        const float send = b3 ? w4[q] : w4[2 + q];
        w2[q] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
      }
      const float keep = b2 ? w2[1] : w2[0];
      const float send = b2 ? w2[0] : w2[1];
      red[(i * SSM_WARPS + warp) * 32 + lane] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
    }
    if (ASYNC) {
      if (k > 0) cp_wait_all();  // sub-chunk k-1's raw inputs (issued a sub-chunk ago) have landed
      __syncthreads();
      if (k > 0) fill(k - 1);
    } else {
      if (k > 0) pref_store(r, l, true, stg[(k - 1) & 1]);
      __syncthreads();
    }
    // grad B / grad C of the sub-chunk: sum over the CTA's warps, one partial per channel group
    {
      const int i = l.tid >> 5, ln = l.tid & 31;
      const int64_t t = l.s + int64_t(k) * ST + i;
      if (i < ST && t < l.e) {
        float sum = 0.f;
#pragma unroll
        for (int w = 0; w < SSM_WARPS; ++w) sum += red[(i * SSM_WARPS + w) * 32 + ln];
        const int vi = (ln >> 2) & 7, nqq = ln & 3;
        const int n = nqq * NS + (vi & 3);
        const int which = vi >> 2;
        a.dbc_part[((int64_t(l.grp) * a.Bsz + l.b) * a.L + t) * 32 + which * NST + n] = sum;
      }
    }
    // grad dt_in and grad_u (scan part) of the sub-chunk, coalesced
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const int idx = l.tid + q * SSM_THREADS;
      const int t = idx / DC, dl = idx % DC;
      const int64_t tok = l.s + int64_t(k) * ST + t;
      const int64_t d = int64_t(l.grp) * DC + dl;
      if (tok < l.e && d < a.D) {
        const int64_t row = l.b * a.L + tok;
        const float gd = gb[t * DC + dl];
        a.gstack[row * a.P + d] = gd;
        if (a.gstack_bf) a.gstack_bf[row * a.P + d] = __float2bfloat16_rn(gd);
        a.gu_scan[row * a.D + d] = gb[ST * DC + t * DC + dl];
      }
    }
    __syncthreads();
    // raw buffer (k - 2) & 1 held sub-chunk k, whose stage was filled a sub-chunk ago
    if (ASYNC && k > 1) raw_issue(a, l, k - 2, raw[k & 1], RAW_U | RAW_G | RAW_AP | RAW_CK);
  }
  // per-CTA parameter partials
  float* sA = sm;  // [SSM_THREADS][NS]; checkpoints are no longer needed
  if (!l.ch) accA[0] = accA[1] = f2(0.f);
  st_states(sA + l.tid * NS, accA);
  __syncthreads();
  if (l.tid < NST) {
    const int n = l.tid, nqq = n / NS, j = n % NS;
    float s = 0.f;
    for (int dl = 0; dl < DC; ++dl) s += sA[(dl * NQ + nqq) * NS + j];
    a.partA[((l.c * a.Bsz + l.b) * a.G + l.grp) * NST + n] = s;
  }
  if (l.nq == 0 && l.ch) {
    a.partD[(l.c * a.Bsz + l.b) * a.D + l.d] = accD;
    a.partS[(l.c * a.Bsz + l.b) * a.D + l.d] = accS;
  }
}

// grad B / grad C columns of gstack: sum of the channel-group partials, in group order.
__global__ void ssm_bc_reduce_kernel(const SsmArgs a) {
  const int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t rows = a.Bsz * a.L;
  if (idx >= rows * 32) return;
  const int64_t row = idx / 32;
  const int m = int(idx % 32);
  float s = 0.f;
  for (int64_t gi = 0; gi < a.G; ++gi) s += a.dbc_part[(gi * rows + row) * 32 + m];
  a.gstack[row * a.P + a.D + m] = s;
  if (a.gstack_bf) a.gstack_bf[row * a.P + a.D + m] = __float2bfloat16_rn(s);
}

// grad A_log / D / scale from the per-CTA partials, in a fixed order.
// grad A_log from the per-CTA partials (A is shared by the channels: one block per state n, the
// partials summed in a fixed order).  grad D and grad scale are column reductions (column_reduce).
__global__ void ssm_param_reduce_kernel(const SsmArgs a, float* __restrict__ gA, int accumulate) {
  __shared__ float red[256];
  const int n = blockIdx.x;
  const int64_t cnt = a.nC * a.Bsz * a.G;
  float s = 0.f;
  for (int64_t i = threadIdx.x; i < cnt; i += blockDim.x) s += a.partA[i * NST + n];
  red[threadIdx.x] = s;
  __syncthreads();
  for (int o = blockDim.x / 2; o > 0; o >>= 1) {
    if (int(threadIdx.x) < o) red[threadIdx.x] += red[threadIdx.x + o];
    __syncthreads();
  }
  if (threadIdx.x == 0) gA[n] = accumulate ? gA[n] + red[0] : red[0];
}

// ---------------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------------
// Algorithmic HBM bytes of the scan kernels (each mandatory tensor once, activations at `es`
// bytes, boundary states in float32): the denominators of their roofline.
static double bytes_chunk_fwd(const SsmArgs& a, int es) {
  const double T = double(a.Bsz) * a.L;
  return T * es * (2.0 * a.D + NST) + double(a.Bsz) * a.nC * a.D * (NST + 1) * 4.0;
}
static double bytes_out_fwd(const SsmArgs& a, int es) {
  const double T = double(a.Bsz) * a.L;
  return T * es * (3.0 * a.D + 2.0 * NST) + double(a.Bsz) * a.nC * a.D * NST * 4.0;
}
static double bytes_chunk_bwd(const SsmArgs& a, int es) {
  const double T = double(a.Bsz) * a.L;
  return T * es * (2.0 * a.D + NST) + double(a.Bsz) * a.nC * a.D * (NST + 2) * 4.0;
}
static double bytes_main_bwd(const SsmArgs& a, int es) {
  // read u, dt_in, g, B, C; write grad_dt_in, grad_u, grad_B, grad_C; boundary state + carry
  const double T = double(a.Bsz) * a.L;
  return T * es * (5.0 * a.D + 4.0 * NST) + double(a.Bsz) * a.nC * a.D * NST * 4.0 * 2.0;
}
static double bytes_compose(const SsmArgs& a) { return double(a.Bsz) * a.nC * a.D * NST * 4.0 * 2.0; }
static int64_t pick_tc(int64_t Bsz, int64_t L, int64_t G) {
  int64_t tc = TC_MAX;
  const int64_t target = 4 * 148;
  while (tc > 32 && ((L + tc - 1) / tc) * Bsz * G < target) tc /= 2;
  return tc;
}

struct SsmPlan {
  int64_t Bsz, L, D, P, Tc, nC, G;
};

static SsmPlan plan_of(int64_t Bsz, int64_t L, int64_t D) {
  SsmPlan p;
  p.Bsz = Bsz; p.L = L; p.D = D; p.P = D + 2 * NST;
  p.G = (D + DC - 1) / DC;
  p.Tc = pick_tc(Bsz, L, p.G);
  p.nC = (L + p.Tc - 1) / p.Tc;
  return p;
}

static size_t ssm_ws(const SsmPlan& p, int dtype, int backward, int act) {
  const size_t BL = size_t(p.Bsz) * p.L;
  size_t b = 0;
  b += Workspace::round(BL * p.P * 4);                                  // proj
  b += Workspace::round(BL * p.D * 4);                                  // y0 (forward)
  b += Workspace::round(size_t(p.Bsz) * p.nC * p.D * NST * 4);          // hloc
  b += Workspace::round(size_t(p.Bsz) * p.nC * p.D * 4);                // sdt
  b += Workspace::round(size_t(p.Bsz) * (p.nC + 1) * p.D * NST * 4);    // hC
  if (dtype) b += Workspace::round(size_t(p.P) * p.D * 2);              // W_cat bf16
  if (backward) {
    b += Workspace::round(BL * p.P * 4);                                // gstack
    if (dtype) b += Workspace::round(BL * p.P * 2);                     // gstack bf16 copy
    b += Workspace::round(BL * p.D * 4);                                // gu_scan
    b += Workspace::round(size_t(p.G) * BL * 32 * 4);                   // dbc_part
    if (act != PGF_ACT_NONE) b += Workspace::round(BL * p.D * 4);       // actp
    b += Workspace::round(size_t(p.Bsz) * p.nC * p.D * NST * 4) * 2;    // dloc, X
    b += Workspace::round(size_t(p.Bsz) * p.nC * p.D * 4) * 2;          // sdt2, dt0
    b += Workspace::round(size_t(p.nC) * p.Bsz * p.G * NST * 4);        // partA
    b += Workspace::round(size_t(p.nC) * p.Bsz * p.D * 4) * 2;          // partD, partS
    b += colsum_ws(int64_t(BL), p.P);
    b += Workspace::round(gemm_split_ws(p.P, p.D, int64_t(BL)));        // split-K partials of grad W_cat
  }
  return b + 4096;
}

// Floats of the saved-state buffer: boundary states, then the sub-chunk checkpoints.
static size_t saved_hc_floats(const SsmPlan& p) { return size_t(p.Bsz) * (p.nC + 1) * p.D * NST; }
static size_t saved_ckpt_floats(const SsmPlan& p) {
  return size_t(p.Bsz) * p.nC * size_t((p.Tc + ST - 1) / ST) * p.D * NST;
}
static size_t saved_s_floats(const SsmPlan& p) { return size_t(p.Bsz) * p.nC * size_t((p.Tc + ST - 1) / ST) * p.D; }
static size_t saved_floats(const SsmPlan& p) { return saved_hc_floats(p) + saved_ckpt_floats(p) + saved_s_floats(p); }

// Carves the buffers every pass shares (projection, chunk summaries, start states, bf16 W_cat) in a
// fixed order, and -- when `fill` -- computes the projection and the bf16 weights.  A staged call
// (begin / finish on one workspace) carves the same layout again with fill = false.
static int ssm_common(SsmArgs& a, const SsmPlan& p, Workspace& W, const void* u, int dtype,
                      const float* W_cat, const float* b_cat, const void** wcat_op, cudaStream_t s,
                      float* hC_ext = nullptr, bool fill = true) {
  const size_t BL = size_t(p.Bsz) * p.L;
  a.Bsz = p.Bsz; a.L = p.L; a.D = p.D; a.P = p.P; a.Tc = p.Tc; a.nC = p.nC; a.G = p.G;
  a.u = u; a.u_bf16 = dtype;
  float* proj = W.take<float>(BL * p.P);
  a.hloc = W.take<float>(size_t(p.Bsz) * p.nC * p.D * NST);
  a.sdt = W.take<float>(size_t(p.Bsz) * p.nC * p.D);
  a.hC = hC_ext ? hC_ext : W.take<float>(size_t(p.Bsz) * (p.nC + 1) * p.D * NST);
  __nv_bfloat16* wb = dtype ? W.take<__nv_bfloat16>(size_t(p.P) * p.D) : nullptr;
  if (!proj || !a.hloc || !a.sdt || !a.hC || (dtype && !wb)) {
    set_error("ssm: workspace too small (%zu)", W.cap);
    return PGF_ERR_WORKSPACE;
  }
  a.proj = proj;
  const void* w = W_cat;
  if (dtype) {
    if (fill) PGF_TRY(to_bf16(W_cat, wb, p.P * p.D, s));
    w = wb;
  }
  *wcat_op = w;
  if (!fill) return PGF_OK;
  // proj = u W_cat^T + b_cat   (train_singlemamba_optimized.py:116-124)
  Gemm g = gemm_make(int64_t(BL), p.P, p.D, u, dtype, p.D, 0, w, dtype, p.D, 0, proj, 0, p.P);
  g.epi.bias = b_cat;
  return run_gemm(g, s);
}

static int ssm_forward_states(const SsmArgs& a, const SsmPlan& p, float* h_final, cudaStream_t s,
                              float* sum_dt = nullptr) {
  dim3 grid(unsigned(p.nC), unsigned(p.Bsz), unsigned(p.G));
  prof_begin(PROF_SSM_CHUNK_FWD, s);
  ssm_chunk_fwd_kernel<<<grid, SSM_THREADS, 0, s>>>(a);
  prof_end(PROF_SSM_CHUNK_FWD, s, bytes_chunk_fwd(a, a.u_bf16 ? 2 : 4));
  PGF_LAUNCH_CHECK();
  const int64_t nth = p.Bsz * p.D * NST;
  prof_begin(PROF_SSM_COMPOSE, s);
  ssm_compose_fwd_kernel<<<ceil_div(nth, 32), 32 * CSEG, 0, s>>>(a, h_final, sum_dt);
  prof_end(PROF_SSM_COMPOSE, s, bytes_compose(a));
  PGF_LAUNCH_CHECK();
  return PGF_OK;
}

static int check_common(int64_t Bsz, int64_t L, int64_t D, int64_t N, int act, int dtype) {
  PGF_CHECK_ARG(N == NST, "ssm: d_state must be %d (got %lld)", NST, (long long)N);
  PGF_CHECK_ARG(Bsz > 0 && L >= 0 && D > 0, "ssm: bad shape");
  PGF_CHECK_ARG(Bsz <= 65535, "ssm: batch too large");
  PGF_CHECK_ARG(act == PGF_ACT_NONE || act == PGF_ACT_RELU || act == PGF_ACT_TANH, "ssm: bad act");
  PGF_CHECK_ARG(dtype == 0 || dtype == 1, "ssm: bad dtype");
  return PGF_OK;
}

}  // namespace pgf

using namespace pgf;

extern "C" size_t pgf_ssm_workspace(int64_t Bsz, int64_t L, int64_t D, int64_t N, int dtype,
                                    int backward) {
  (void)N;
  SsmPlan p = plan_of(Bsz < 1 ? 1 : Bsz, L < 1 ? 1 : L, D < 1 ? 1 : D);
  return ssm_ws(p, dtype, backward, PGF_ACT_TANH);
}

namespace pgf {
// Forward stages: ALL (one call), BEGIN (projection, zero-start pass, summary of the segment from a
// zero start into h_out / sum_dt), FINISH (on BEGIN's workspace: start states from h_init, output).
enum { STAGE_ALL = 0, STAGE_BEGIN = 1, STAGE_FINISH = 2 };

static int ssm_fwd_impl(const void* u, const float* W_cat, const float* b_cat, const float* A_log,
                        const float* Dp, const float* scale, const float* h_init, void* y,
                        float* h_final, int64_t Bsz, int64_t L, int64_t D, int64_t N, int act,
                        int dtype, void* ws, size_t ws_bytes, pgf_stream_t stream, float* saved,
                        int stage = STAGE_ALL, float* sum_dt = nullptr, float* states_out = nullptr) {
  PGF_TRY(check_common(Bsz, L, D, N, act, dtype));
  PGF_CHECK_ARG(u && W_cat && b_cat && A_log, "ssm_fwd: null pointer");
  PGF_CHECK_ARG(stage == STAGE_BEGIN || (Dp && scale && y), "ssm_fwd: null pointer");
  cudaStream_t s = as_stream(stream);
  if (L == 0) {
    if (h_final) {
      if (h_init && stage != STAGE_BEGIN)
        PGF_CUDA(cudaMemcpyAsync(h_final, h_init, Bsz * D * NST * 4, cudaMemcpyDeviceToDevice, s));
      else PGF_CUDA(cudaMemsetAsync(h_final, 0, Bsz * D * NST * 4, s));
    }
    if (sum_dt) PGF_CUDA(cudaMemsetAsync(sum_dt, 0, Bsz * D * 4, s));
    return PGF_OK;
  }
  SsmPlan p = plan_of(Bsz, L, D);
  Workspace W(ws, ws_bytes);
  SsmArgs a = {};
  a.A_log = A_log; a.Dp = Dp; a.scale = scale; a.act = act;
  a.h_init = stage == STAGE_BEGIN ? nullptr : h_init;
  const void* wop;
  // (a staged call keeps the start states in the workspace, whose layout BEGIN and FINISH share)
  PGF_TRY(ssm_common(a, p, W, u, dtype, W_cat, b_cat, &wop, s,
                     saved ? saved : (stage == STAGE_ALL ? states_out : nullptr), stage != STAGE_FINISH));
  a.y0 = W.take<float>(size_t(Bsz) * L * D);
  if (!a.y0) { set_error("ssm_fwd: workspace too small (%zu)", ws_bytes); return PGF_ERR_WORKSPACE; }
  a.y = y;
  a.y_bf16 = dtype;
  if (saved) {
    a.ckpt_g = saved + saved_hc_floats(p);
    a.ckpt_s = a.ckpt_g + saved_ckpt_floats(p);
    a.ckpt_write = 1;
  }
  dim3 grid(unsigned(p.nC), unsigned(p.Bsz), unsigned(p.G));
  if (stage != STAGE_FINISH) {
    // zero-start pass (y0, summaries, checkpoints): independent of the start state
    prof_begin(PROF_SSM_CHUNK_FWD, s);
    ssm_chunk_y0_kernel<<<grid, SSM_THREADS, 0, s>>>(a);
    prof_end(PROF_SSM_CHUNK_FWD, s, bytes_chunk_fwd(a, a.u_bf16 ? 2 : 4) + double(Bsz) * L * D * 4.0);
    PGF_LAUNCH_CHECK();
  }
  // chunk start states (from h_init; from zero in BEGIN, whose end state and sum of dt are the summary)
  const int64_t nth = p.Bsz * p.D * NST;
  prof_begin(PROF_SSM_COMPOSE, s);
  ssm_compose_fwd_kernel<<<ceil_div(nth, 32), 32 * CSEG, 0, s>>>(a, h_final, stage == STAGE_BEGIN ? sum_dt : nullptr);
  prof_end(PROF_SSM_COMPOSE, s, bytes_compose(a));
  PGF_LAUNCH_CHECK();
  if (stage == STAGE_BEGIN) return PGF_OK;
  if (states_out && states_out != a.hC)
    PGF_CUDA(cudaMemcpyAsync(states_out, a.hC, saved_hc_floats(p) * sizeof(float), cudaMemcpyDeviceToDevice, s));
  prof_begin(PROF_SSM_OUT_FWD, s);
  ssm_out_corr_kernel<<<grid, SSM_THREADS, 0, s>>>(a);
  prof_end(PROF_SSM_OUT_FWD, s, bytes_out_fwd(a, a.u_bf16 ? 2 : 4) + double(Bsz) * L * D * 4.0);
  PGF_LAUNCH_CHECK();
  return PGF_OK;
}
}  // namespace pgf

extern "C" int pgf_ssm_fwd(const void* u, const float* W_cat, const float* b_cat,
                           const float* A_log, const float* Dp, const float* scale,
                           const float* h_init, void* y, float* h_final, int64_t Bsz, int64_t L,
                           int64_t D, int64_t N, int act, int dtype, void* ws, size_t ws_bytes,
                           pgf_stream_t stream) {
  return ssm_fwd_impl(u, W_cat, b_cat, A_log, Dp, scale, h_init, y, h_final, Bsz, L, D, N, act, dtype,
                      ws, ws_bytes, stream, nullptr);
}

extern "C" size_t pgf_ssm_states_size(int64_t Bsz, int64_t L, int64_t D, int64_t N) {
  (void)N;
  SsmPlan p = plan_of(Bsz < 1 ? 1 : Bsz, L < 1 ? 1 : L, D < 1 ? 1 : D);
  return saved_hc_floats(p) * sizeof(float);
}

extern "C" int pgf_ssm_fwd_states(const void* u, const float* W_cat, const float* b_cat, const float* A_log,
                                  const float* Dp, const float* scale, const float* h_init, void* y, float* states,
                                  int64_t Bsz, int64_t L, int64_t D, int64_t N, int act, int dtype, void* ws,
                                  size_t ws_bytes, pgf_stream_t stream) {
  PGF_CHECK_ARG(states, "ssm_fwd_states: null state buffer");
  PGF_CHECK_ARG(L > 0, "ssm_fwd_states: empty sequence");
  return ssm_fwd_impl(u, W_cat, b_cat, A_log, Dp, scale, h_init, y, nullptr, Bsz, L, D, N, act, dtype, ws, ws_bytes,
                      stream, nullptr, STAGE_ALL, nullptr, states);
}

extern "C" int pgf_ssm_fwd_save_states(const void* u, const float* W_cat, const float* b_cat, const float* A_log,
                                       const float* Dp, const float* scale, const float* states, void* y,
                                       float* saved, int64_t Bsz, int64_t L, int64_t D, int64_t N, int act,
                                       int dtype, void* ws, size_t ws_bytes, pgf_stream_t stream) {
  PGF_TRY(check_common(Bsz, L, D, N, act, dtype));
  PGF_CHECK_ARG(u && W_cat && b_cat && A_log && Dp && scale && states && y && saved, "ssm_fwd_save_states: null pointer");
  PGF_CHECK_ARG(L > 0, "ssm_fwd_save_states: empty sequence");
  cudaStream_t s = as_stream(stream);
  SsmPlan p = plan_of(Bsz, L, D);
  Workspace W(ws, ws_bytes);
  SsmArgs a = {};
  a.A_log = A_log; a.Dp = Dp; a.scale = scale; a.act = act;
  const void* wop;
  // projection; the boundary states come from the caller (copied where the backward reads them)
  PGF_TRY(ssm_common(a, p, W, u, dtype, W_cat, b_cat, &wop, s, saved, true));
  PGF_CUDA(cudaMemcpyAsync(saved, states, saved_hc_floats(p) * sizeof(float), cudaMemcpyDeviceToDevice, s));
  a.y = y;
  a.y_bf16 = dtype;
  a.ckpt_g = saved + saved_hc_floats(p);
  a.ckpt_s = a.ckpt_g + saved_ckpt_floats(p);
  a.ckpt_write = 2;
  dim3 grid(unsigned(p.nC), unsigned(p.Bsz), unsigned(p.G));
  prof_begin(PROF_SSM_OUT_FWD, s);
  ssm_out_fwd_kernel<<<grid, SSM_THREADS, 0, s>>>(a);
  prof_end(PROF_SSM_OUT_FWD, s, bytes_out_fwd(a, a.u_bf16 ? 2 : 4));
  PGF_LAUNCH_CHECK();
  return PGF_OK;
}

extern "C" size_t pgf_ssm_saved_size(int64_t Bsz, int64_t L, int64_t D, int64_t N) {
  (void)N;
  SsmPlan p = plan_of(Bsz < 1 ? 1 : Bsz, L < 1 ? 1 : L, D < 1 ? 1 : D);
  return saved_floats(p) * sizeof(float);
}

extern "C" int pgf_ssm_fwd_save(const void* u, const float* W_cat, const float* b_cat,
                                const float* A_log, const float* Dp, const float* scale,
                                const float* h_init, void* y, float* saved, int64_t Bsz, int64_t L,
                                int64_t D, int64_t N, int act, int dtype, void* ws, size_t ws_bytes,
                                pgf_stream_t stream) {
  PGF_CHECK_ARG(saved, "ssm_fwd_save: null saved-state buffer");
  PGF_CHECK_ARG(L > 0, "ssm_fwd_save: empty sequence");
  return ssm_fwd_impl(u, W_cat, b_cat, A_log, Dp, scale, h_init, y, nullptr, Bsz, L, D, N, act, dtype,
                      ws, ws_bytes, stream, saved);
}

namespace pgf {
static int ssm_bwd_impl(const void* u, const void* g, const float* W_cat, const float* b_cat,
                        const float* A_log, const float* Dp, const float* scale, const float* h_init,
                        const float* dh_end, const float* dA_end, float* gW_cat, float* gb_cat,
                        float* gA_log, float* gDp, float* gscale, void* gu, float* dh_start,
                        float* dA_start, int accumulate, int64_t Bsz, int64_t L, int64_t D, int64_t N,
                        int act, int dtype, void* ws, size_t ws_bytes, pgf_stream_t stream,
                        const float* saved, int stage = STAGE_ALL, float* sum_dt_excl = nullptr) {
  PGF_TRY(check_common(Bsz, L, D, N, act, dtype));
  PGF_CHECK_ARG(u && g && W_cat && b_cat && A_log && scale, "ssm_bwd: null pointer");
  PGF_CHECK_ARG(stage == STAGE_BEGIN || (Dp && gW_cat && gb_cat && gA_log && gDp && gscale && gu),
                "ssm_bwd: null pointer");
  PGF_CHECK_ARG(stage == STAGE_ALL || saved, "ssm_bwd: a staged backward needs the saved forward states");
  PGF_CHECK_ARG(L > 0, "ssm_bwd: empty sequence");
  cudaStream_t s = as_stream(stream);
  SsmPlan p = plan_of(Bsz, L, D);
  Workspace W(ws, ws_bytes);
  SsmArgs a = {};
  a.A_log = A_log; a.Dp = Dp; a.scale = scale; a.act = act; a.h_init = h_init;
  a.g = g; a.g_bf16 = dtype;
  const void* wop;
  PGF_TRY(ssm_common(a, p, W, u, dtype, W_cat, b_cat, &wop, s, const_cast<float*>(saved), stage != STAGE_FINISH));
  const size_t BL = size_t(Bsz) * L;
  a.gstack = W.take<float>(BL * p.P);
  a.gstack_bf = dtype ? W.take<__nv_bfloat16>(BL * p.P) : nullptr;
  a.gu_scan = W.take<float>(BL * p.D);
  a.dbc_part = W.take<float>(size_t(p.G) * BL * 32);
  a.actp = act != PGF_ACT_NONE ? W.take<float>(BL * p.D) : nullptr;
  a.dloc = W.take<float>(size_t(Bsz) * p.nC * D * NST);
  a.X = W.take<float>(size_t(Bsz) * p.nC * D * NST);
  a.sdt2 = W.take<float>(size_t(Bsz) * p.nC * D);
  a.dt0 = W.take<float>(size_t(Bsz) * p.nC * D);
  a.partA = W.take<float>(size_t(p.nC) * Bsz * p.G * NST);
  a.partD = W.take<float>(size_t(p.nC) * Bsz * D);
  a.partS = W.take<float>(size_t(p.nC) * Bsz * D);
  const size_t csb = colsum_ws(int64_t(BL), p.P);
  void* cs = W.take<char>(csb);
  const size_t split_ws_bytes = gemm_split_ws(p.P, D, int64_t(BL));
  void* split_ws = split_ws_bytes ? W.take<char>(split_ws_bytes) : nullptr;
  if ((split_ws_bytes && !split_ws) || !a.gstack || (dtype && !a.gstack_bf) || !a.gu_scan || !a.dbc_part || (act != PGF_ACT_NONE && !a.actp) || !a.dloc ||
      !a.X || !a.sdt2 || !a.dt0 || !a.partA || !a.partD || !a.partS || !cs) {
    set_error("ssm_bwd: workspace too small (%zu)", ws_bytes);
    return PGF_ERR_WORKSPACE;
  }
  dim3 grid(unsigned(p.nC), unsigned(p.Bsz), unsigned(p.G));
  if (stage != STAGE_FINISH) {
    if (!saved) PGF_TRY(ssm_forward_states(a, p, nullptr, s));
    if (act != PGF_ACT_NONE) {
      a.y = nullptr;
      ssm_out_fwd_kernel<<<grid, SSM_THREADS, 0, s>>>(a);  // act'(C h) per token and channel
      PGF_LAUNCH_CHECK();
    }
  }
  if (saved) {
    a.ckpt_g = const_cast<float*>(saved) + saved_hc_floats(p);
    a.ckpt_s = a.ckpt_g + saved_ckpt_floats(p);
  }
  if (stage != STAGE_FINISH) {
    // reverse chunk summaries from a zero carry: independent of the carry entering from the right
    prof_begin(PROF_SSM_CHUNK_BWD, s);
    PGF_TRY(launch_chunk_bwd(a, grid, s));
    prof_end(PROF_SSM_CHUNK_BWD, s, bytes_chunk_bwd(a, a.u_bf16 ? 2 : 4));
  }
  const int64_t nth = Bsz * D * NST;
  if (stage == STAGE_BEGIN) {
    // the segment's adjoint summary from a zero end carry
    ssm_compose_bwd_kernel<<<ceil_div(nth, 32), 32 * CSEG, 0, s>>>(a, nullptr, nullptr, dh_start, dA_start,
                                                              sum_dt_excl);
    PGF_LAUNCH_CHECK();
    return PGF_OK;
  }
  ssm_compose_bwd_kernel<<<ceil_div(nth, 32), 32 * CSEG, 0, s>>>(a, dh_end, dA_end, dh_start, dA_start,
                                                            nullptr);
  PGF_LAUNCH_CHECK();
  const int KS = int((p.Tc + ST - 1) / ST);
  // cp.async staging: saved checkpoints, whole 16-byte pieces per row (D a multiple of 8) and
  // 16-byte aligned bases
  auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  const bool async = saved && D % 8 == 0 && al16(u) && al16(g) && al16(a.proj) && al16(a.ckpt_g) &&
                     al16(a.ckpt_s) && (!a.actp || al16(a.actp));
  const size_t smem = ((saved ? size_t(0) : size_t(KS) * SSM_THREADS * NS) + size_t(ST) * SSM_WARPS * 32 +
                       2 * 2 * ST * DC) * 4 + (async ? 2 * sizeof(Raw) : 0);
  prof_begin(PROF_SSM_MAIN_BWD, s);
  if (async) {
    static int smem_limit_async = 0;
    PGF_CUDA(ensure_dynamic_smem(ssm_main_bwd_kernel<true>, smem, smem_limit_async));
    ssm_main_bwd_kernel<true><<<grid, SSM_THREADS, smem, s>>>(a);
  } else {
    static int smem_limit = 0;
    PGF_CUDA(ensure_dynamic_smem(ssm_main_bwd_kernel<false>, smem, smem_limit));
    ssm_main_bwd_kernel<false><<<grid, SSM_THREADS, smem, s>>>(a);
  }
  prof_end(PROF_SSM_MAIN_BWD, s, bytes_main_bwd(a, a.u_bf16 ? 2 : 4));
  PGF_LAUNCH_CHECK();
  ssm_bc_reduce_kernel<<<ceil_div(int64_t(BL) * 32, 256), 256, 0, s>>>(a);
  PGF_LAUNCH_CHECK();
  ssm_param_reduce_kernel<<<NST, 256, 0, s>>>(a, gA_log, accumulate);
  PGF_LAUNCH_CHECK();
  PGF_TRY(column_reduce(a.partD, p.nC * Bsz, D, gDp, accumulate, s));
  PGF_TRY(column_reduce(a.partS, p.nC * Bsz, D, gscale, accumulate, s));
  // grad W_cat (+)= gstack^T u ;  grad b_cat (+)= colsum(gstack)   (:438-451)
  Gemm gw = gemm_make(p.P, D, int64_t(BL), dtype ? (const void*)a.gstack_bf : (const void*)a.gstack, dtype, p.P,
                      1, u, dtype, D, 1, gW_cat, 0, D);
  gw.epi.accumulate = accumulate;
  gw.ws = split_ws; gw.ws_bytes = split_ws_bytes;
  PGF_TRY(run_gemm(gw, s));
  PGF_TRY(colsum(a.gstack, 0, int64_t(BL), p.P, p.P, gb_cat, accumulate, cs, csb, s));
  // grad_u = gstack W_cat + (delta_in*D + sum_n delta_h phi_1 B)   (:453-463)
  Gemm gx = gemm_make(int64_t(BL), D, p.P, dtype ? (const void*)a.gstack_bf : (const void*)a.gstack, dtype, p.P,
                      0, wop, dtype, D, 1, gu, dtype, D);
  gx.epi.addend = a.gu_scan;
  gx.epi.addend_dtype = 0;
  gx.epi.ld_addend = D;
  PGF_TRY(run_gemm(gx, s));
  return PGF_OK;
}
}  // namespace pgf

extern "C" int pgf_ssm_bwd(const void* u, const void* g, const float* W_cat, const float* b_cat,
                           const float* A_log, const float* Dp, const float* scale,
                           const float* h_init, const float* dh_end, const float* dA_end,
                           float* gW_cat, float* gb_cat, float* gA_log, float* gDp, float* gscale,
                           void* gu, float* dh_start, float* dA_start, int accumulate, int64_t Bsz,
                           int64_t L, int64_t D, int64_t N, int act, int dtype, void* ws,
                           size_t ws_bytes, pgf_stream_t stream) {
  return ssm_bwd_impl(u, g, W_cat, b_cat, A_log, Dp, scale, h_init, dh_end, dA_end, gW_cat, gb_cat, gA_log,
                      gDp, gscale, gu, dh_start, dA_start, accumulate, Bsz, L, D, N, act, dtype, ws, ws_bytes,
                      stream, nullptr);
}

extern "C" int pgf_ssm_bwd_saved(const void* u, const void* g, const float* W_cat, const float* b_cat,
                                 const float* A_log, const float* Dp, const float* scale,
                                 const float* saved, const float* dh_end, const float* dA_end,
                                 float* gW_cat, float* gb_cat, float* gA_log, float* gDp, float* gscale,
                                 void* gu, float* dh_start, float* dA_start, int accumulate, int64_t Bsz,
                                 int64_t L, int64_t D, int64_t N, int act, int dtype, void* ws,
                                 size_t ws_bytes, pgf_stream_t stream) {
  PGF_CHECK_ARG(saved, "ssm_bwd_saved: null saved-state buffer");
  return ssm_bwd_impl(u, g, W_cat, b_cat, A_log, Dp, scale, nullptr, dh_end, dA_end, gW_cat, gb_cat, gA_log,
                      gDp, gscale, gu, dh_start, dA_start, accumulate, Bsz, L, D, N, act, dtype, ws, ws_bytes,
                      stream, saved);
}

// ---------------------------------------------------------------------------------------------
// Segment summaries for a sequence sharded across ranks (affine-recurrence composition).
// ---------------------------------------------------------------------------------------------
extern "C" int pgf_ssm_summary(const void* u, const float* W_cat, const float* b_cat, const float* A_log,
                               const float* h_init, float* h_final, float* sum_dt, int64_t Bsz, int64_t L,
                               int64_t D, int64_t N, int dtype, void* ws, size_t ws_bytes,
                               pgf_stream_t stream) {
  PGF_TRY(check_common(Bsz, L, D, N, PGF_ACT_NONE, dtype));
  PGF_CHECK_ARG(u && W_cat && b_cat && A_log && h_final && sum_dt, "ssm_summary: null pointer");
  PGF_CHECK_ARG(L > 0, "ssm_summary: empty segment");
  cudaStream_t s = as_stream(stream);
  SsmPlan p = plan_of(Bsz, L, D);
  Workspace W(ws, ws_bytes);
  SsmArgs a = {};
  a.A_log = A_log; a.act = PGF_ACT_NONE; a.h_init = h_init;
  const void* wop;
  PGF_TRY(ssm_common(a, p, W, u, dtype, W_cat, b_cat, &wop, s));
  return ssm_forward_states(a, p, h_final, s, sum_dt);
}

extern "C" int pgf_ssm_fwd_begin(const void* u, const float* W_cat, const float* b_cat, const float* A_log,
                                 float* h_seg, float* sum_dt, int64_t Bsz, int64_t L, int64_t D, int64_t N,
                                 int dtype, void* ws, size_t ws_bytes, pgf_stream_t stream) {
  PGF_CHECK_ARG(h_seg && sum_dt, "ssm_fwd_begin: null pointer");
  return ssm_fwd_impl(u, W_cat, b_cat, A_log, nullptr, nullptr, nullptr, nullptr, h_seg, Bsz, L, D, N, PGF_ACT_NONE,
                      dtype, ws, ws_bytes, stream, nullptr, STAGE_BEGIN, sum_dt);
}

extern "C" int pgf_ssm_fwd_finish(const void* u, const float* W_cat, const float* b_cat, const float* A_log,
                                  const float* Dp, const float* scale, const float* h_init, void* y,
                                  float* h_final, int64_t Bsz, int64_t L, int64_t D, int64_t N, int act, int dtype,
                                  void* ws, size_t ws_bytes, pgf_stream_t stream) {
  return ssm_fwd_impl(u, W_cat, b_cat, A_log, Dp, scale, h_init, y, h_final, Bsz, L, D, N, act, dtype, ws,
                      ws_bytes, stream, nullptr, STAGE_FINISH);
}

extern "C" int pgf_ssm_fwd_finish_states(const void* u, const float* W_cat, const float* b_cat, const float* A_log,
                                         const float* Dp, const float* scale, const float* h_init, void* y,
                                         float* states, int64_t Bsz, int64_t L, int64_t D, int64_t N, int act,
                                         int dtype, void* ws, size_t ws_bytes, pgf_stream_t stream) {
  PGF_CHECK_ARG(states, "ssm_fwd_finish_states: null state buffer");
  PGF_CHECK_ARG(L > 0, "ssm_fwd_finish_states: empty sequence");
  return ssm_fwd_impl(u, W_cat, b_cat, A_log, Dp, scale, h_init, y, nullptr, Bsz, L, D, N, act, dtype, ws,
                      ws_bytes, stream, nullptr, STAGE_FINISH, nullptr, states);
}

extern "C" int pgf_ssm_bwd_begin(const void* u, const void* g, const float* W_cat, const float* b_cat,
                                 const float* A_log, const float* scale, const float* h_init, const float* saved,
                                 float* dh_start, float* dA_start, float* sum_dt_excl, int64_t Bsz, int64_t L,
                                 int64_t D, int64_t N, int act, int dtype, void* ws, size_t ws_bytes,
                                 pgf_stream_t stream) {
  PGF_CHECK_ARG(dh_start && dA_start && sum_dt_excl, "ssm_bwd_begin: null pointer");
  return ssm_bwd_impl(u, g, W_cat, b_cat, A_log, nullptr, scale, h_init, nullptr, nullptr, nullptr, nullptr,
                      nullptr, nullptr, nullptr, nullptr, dh_start, dA_start, 0, Bsz, L, D, N, act, dtype, ws,
                      ws_bytes, stream, saved, STAGE_BEGIN, sum_dt_excl);
}

extern "C" int pgf_ssm_bwd_finish(const void* u, const void* g, const float* W_cat, const float* b_cat,
                                  const float* A_log, const float* Dp, const float* scale, const float* h_init,
                                  const float* saved, const float* dh_end, const float* dA_end, float* gW_cat,
                                  float* gb_cat, float* gA_log, float* gDp, float* gscale, void* gu,
                                  float* dh_start, float* dA_start, int accumulate, int64_t Bsz, int64_t L,
                                  int64_t D, int64_t N, int act, int dtype, void* ws, size_t ws_bytes,
                                  pgf_stream_t stream) {
  return ssm_bwd_impl(u, g, W_cat, b_cat, A_log, Dp, scale, h_init, dh_end, dA_end, gW_cat, gb_cat, gA_log, gDp,
                      gscale, gu, dh_start, dA_start, accumulate, Bsz, L, D, N, act, dtype, ws, ws_bytes, stream,
                      saved, STAGE_FINISH);
}

extern "C" int pgf_ssm_bwd_summary(const void* u, const void* g, const float* W_cat, const float* b_cat,
                                   const float* A_log, const float* scale, const float* h_init,
                                   float* dh_start, float* dA_start, float* sum_dt_excl, int64_t Bsz,
                                   int64_t L, int64_t D, int64_t N, int act, int dtype, void* ws,
                                   size_t ws_bytes, pgf_stream_t stream) {
  PGF_TRY(check_common(Bsz, L, D, N, act, dtype));
  PGF_CHECK_ARG(u && g && W_cat && b_cat && A_log && scale && dh_start && dA_start && sum_dt_excl,
                "ssm_bwd_summary: null pointer");
  PGF_CHECK_ARG(L > 0, "ssm_bwd_summary: empty segment");
  cudaStream_t s = as_stream(stream);
  SsmPlan p = plan_of(Bsz, L, D);
  Workspace W(ws, ws_bytes);
  SsmArgs a = {};
  a.A_log = A_log; a.scale = scale; a.act = act; a.h_init = h_init;
  a.g = g; a.g_bf16 = dtype;
  const void* wop;
  PGF_TRY(ssm_common(a, p, W, u, dtype, W_cat, b_cat, &wop, s));
  const size_t BL = size_t(Bsz) * L;
  a.actp = act != PGF_ACT_NONE ? W.take<float>(BL * p.D) : nullptr;
  a.dloc = W.take<float>(size_t(Bsz) * p.nC * D * NST);
  a.X = W.take<float>(size_t(Bsz) * p.nC * D * NST);
  a.sdt2 = W.take<float>(size_t(Bsz) * p.nC * D);
  a.dt0 = W.take<float>(size_t(Bsz) * p.nC * D);
  if ((act != PGF_ACT_NONE && !a.actp) || !a.dloc || !a.X || !a.sdt2 || !a.dt0) {
    set_error("ssm_bwd_summary: workspace too small (%zu)", ws_bytes);
    return PGF_ERR_WORKSPACE;
  }
  dim3 grid(unsigned(p.nC), unsigned(p.Bsz), unsigned(p.G));
  if (act != PGF_ACT_NONE) {
    PGF_TRY(ssm_forward_states(a, p, nullptr, s));
    a.y = nullptr;
    ssm_out_fwd_kernel<<<grid, SSM_THREADS, 0, s>>>(a);
    PGF_LAUNCH_CHECK();
  }
  PGF_TRY(launch_chunk_bwd(a, grid, s));
  const int64_t nth = Bsz * D * NST;
  ssm_compose_bwd_kernel<<<ceil_div(nth, 32), 32 * CSEG, 0, s>>>(a, nullptr, nullptr, dh_start, dA_start,
                                                            sum_dt_excl);
  PGF_LAUNCH_CHECK();
  return PGF_OK;
}

// ---------------------------------------------------------------------------------------------
// Composition of the ranks' segment summaries (sequence sharding): one thread per (b, d, n) folds
// the P summaries gathered into one buffer, in rank order, instead of a host loop of small ops.
// ---------------------------------------------------------------------------------------------
namespace pgf {

__global__ void compose_ranks_fwd_kernel(const float* __restrict__ gat, int64_t stride, int P, int rank,
                                         const float* __restrict__ A_log, int a_pc, float* __restrict__ h_in,
                                         int64_t Bsz, int64_t D, int64_t N) {
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t nth = Bsz * D * N;
  if (i >= nth) return;
  const int64_t n = i % N, bd = i / N, d = bd % D;
  const float A = -expf(A_log[a_pc ? d * N + n : n]);
  float H = 0.f;
  for (int j = 0; j < rank && j < P; ++j) {
    const float* g = gat + int64_t(j) * stride;
    H = fmaf(expf(A * g[nth + bd]), H, g[i]);
  }
  h_in[i] = H;
}

__global__ void compose_ranks_bwd_kernel(const float* __restrict__ gat, int64_t stride, int P, int rank,
                                         const float* __restrict__ A_log, int a_pc, float* __restrict__ dh_end,
                                         float* __restrict__ dA_end, int64_t Bsz, int64_t D, int64_t N) {
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t nth = Bsz * D * N;
  if (i >= nth) return;
  const int64_t n = i % N, bd = i / N, d = bd % D;
  const float A = -expf(A_log[a_pc ? d * N + n : n]);
  float G = 0.f, aE = 1.f;
  for (int j = P - 1; j > rank; --j) {
    const float* g = gat + int64_t(j) * stride;
    G = fmaf(expf(A * g[2 * nth + bd]), aE * G, g[i]);
    aE = g[nth + i];
  }
  dh_end[i] = G;
  dA_end[i] = aE;
}

}  // namespace pgf

extern "C" int pgf_ssm_compose_ranks_fwd(const float* gathered, int64_t stride, int P, int rank, const float* A_log,
                                         int a_per_channel, float* h_in, int64_t Bsz, int64_t D, int64_t N,
                                         pgf_stream_t stream) {
  PGF_CHECK_ARG(gathered && A_log && h_in, "ssm_compose_ranks_fwd: null pointer");
  PGF_CHECK_ARG(P >= 1 && rank >= 0 && rank < P && Bsz > 0 && D > 0 && N > 0, "ssm_compose_ranks_fwd: bad shape");
  PGF_CHECK_ARG(stride >= Bsz * D * (N + 1), "ssm_compose_ranks_fwd: stride %lld below one summary",
                (long long)stride);
  const int64_t nth = Bsz * D * N;
  compose_ranks_fwd_kernel<<<ceil_div(nth, 256), 256, 0, as_stream(stream)>>>(gathered, stride, P, rank, A_log,
                                                                              a_per_channel, h_in, Bsz, D, N);
  PGF_LAUNCH_CHECK();
  return PGF_OK;
}

extern "C" int pgf_ssm_compose_ranks_bwd(const float* gathered, int64_t stride, int P, int rank, const float* A_log,
                                         int a_per_channel, float* dh_end, float* dA_end, int64_t Bsz, int64_t D,
                                         int64_t N, pgf_stream_t stream) {
  PGF_CHECK_ARG(gathered && A_log && dh_end && dA_end, "ssm_compose_ranks_bwd: null pointer");
  PGF_CHECK_ARG(P >= 1 && rank >= 0 && rank < P && Bsz > 0 && D > 0 && N > 0, "ssm_compose_ranks_bwd: bad shape");
  PGF_CHECK_ARG(stride >= Bsz * D * (2 * N + 1), "ssm_compose_ranks_bwd: stride %lld below one summary",
                (long long)stride);
  const int64_t nth = Bsz * D * N;
  compose_ranks_bwd_kernel<<<ceil_div(nth, 256), 256, 0, as_stream(stream)>>>(gathered, stride, P, rank, A_log,
                                                                              a_per_channel, dh_end, dA_end, Bsz, D,
                                                                              N);
  PGF_LAUNCH_CHECK();
  return PGF_OK;
}
