// Internal dense-product interface shared by the composite operators.
#pragma once
#include "common.cuh"

namespace pgf {

struct Gemm {
  int64_t M, N, K;
  const void* A; int a_bf16; int64_t lda; int a_trans;
  const void* B; int b_bf16; int64_t ldb; int b_trans;
  void* D; int d_bf16; int64_t ldd;
  pgf_epilogue epi;
  // Optional scratch for split-K (>= gemm_split_ws(M, N, K) bytes).  When the output has too few
  // tiles to fill the GPU, K is cut into slices whose float32 partial products land here and are
  // summed in slice order (deterministic) by the epilogue pass; without it the product is not split.
  void* ws; size_t ws_bytes;
};

static inline pgf_epilogue epi_default() {
  pgf_epilogue e;
  e.kind = PGF_EPI_NONE; e.alpha = 1.f; e.bias = nullptr;
  e.aux = nullptr; e.aux_dtype = 0; e.ld_aux = 0;
  e.aux_out = nullptr; e.aux_out_dtype = 0; e.ld_aux_out = 0;
  e.addend = nullptr; e.addend_dtype = 0; e.ld_addend = 0;
  e.accumulate = 0;
  return e;
}

static inline Gemm gemm_make(int64_t M, int64_t N, int64_t K, const void* A, int abf, int64_t lda, int at,
                             const void* B, int bbf, int64_t ldb, int bt, void* D, int dbf, int64_t ldd) {
  Gemm g;
  g.M = M; g.N = N; g.K = K;
  g.A = A; g.a_bf16 = abf; g.lda = lda; g.a_trans = at;
  g.B = B; g.b_bf16 = bbf; g.ldb = ldb; g.b_trans = bt;
  g.D = D; g.d_bf16 = dbf; g.ldd = ldd;
  g.epi = epi_default();
  g.ws = nullptr; g.ws_bytes = 0;
  return g;
}

// D = epi(opA * opB^T); picks the tensor-core path when the operands allow it.
int run_gemm(const Gemm& g, cudaStream_t s);
// Split-K scratch bytes run_gemm may use for an (M x N, depth K) product on either engine.
size_t gemm_split_ws(int64_t M, int64_t N, int64_t K);
// Number of K slices each engine uses for the product (1 = no split).
int split_slices_tc(int64_t M, int64_t N, int64_t K);
int sm_count();  // streaming multiprocessors of the current device (cached)
int split_slices_simt(int64_t M, int64_t N, int64_t K);
// Engine entry points for one split: slice z covers k-range [z*kchunk, (z+1)*kchunk) and writes its
// float32 partial to part + z*M*N (row pitch N).  They return the number of slices launched.
int run_gemm_tc_split(const Gemm& g, int slices, float* part, int* launched, cudaStream_t s);
// SIMT path (any dtype mix, any layout): the float32 reference-precision engine.
int run_gemm_simt(const Gemm& g, cudaStream_t s);
// tcgen05 path; returns PGF_ERR_UNSUPPORTED when the call does not fit it.
int run_gemm_tc(const Gemm& g, cudaStream_t s);
bool tc_usable(const Gemm& g);
// Two products into one (M x N) output tile, on the tcgen05 engine, for the FFN backward: with
//   z = A1 B1^T + bias  (A1: M x K1, B1: N x K1, or K1 x N when b1_trans),
//   d = A2 B2^T         (A2: M x K2, B2: N x K2, or K2 x N when b2_trans),
// it writes H = act(z) and DZ = d * act'(z) (act = GELU (tanh form) or ReLU), all bf16; z itself is
// never stored.  PGF_ERR_UNSUPPORTED when the operands do not suit the engine.
struct DualGemm {
  int64_t M, N, K1, K2;
  const void* A1; int64_t lda1;
  const void* B1; int64_t ldb1; int b1_trans;
  const void* A2; int64_t lda2;
  const void* B2; int64_t ldb2; int b2_trans;
  const float* bias;  // (N,) or NULL
  int kind;           // PGF_EPI_GELU or PGF_EPI_RELU
  void* H; int64_t ldh;
  void* DZ; int64_t lddz;
};
int run_gemm_tc_dual(const DualGemm& g, cudaStream_t s);
// Fused LM-head + cross-entropy passes on the tcgen05 engine (g: logits = h W^T, N = vocab).
// Forward: per row and per group of `ng` 128-column tiles, the running max / sum of exp of the
// logits (part_m, part_s: (M, n_groups)) and the target logit; the logits are never stored.
int tc_ce_fwd(const Gemm& g, int ng, const int64_t* targets, float* part_m, float* part_s,
              float* tgt_logit, int* n_groups_out, cudaStream_t s);
// Backward: G[m, v] = (exp(logit - lse[m]) - [v == target[m]]) * scale as bf16, pitch ldg.
int tc_ce_bwd(const Gemm& g, const int64_t* targets, const float* lse, float scale, __nv_bfloat16* G,
              int64_t ldg, cudaStream_t s);

// Fault flag of the fused LM-head kernels (lmhead_tc.cu): read and cleared; -1 on a CUDA error.
int lmhead_tc_fault();
// Fused CE backward over M rows (lmhead_tc.cu): G = (softmax(h W^T) - onehot) * scale as bf16 (rows x
// ldg, for grad W) and dh = G W (bf16, M x d) in one pass, G never re-read for dh.  d % 64 == 0,
// d <= 256, 16-byte aligned operands; PGF_ERR_UNSUPPORTED otherwise.
bool ce_bwd_dh_usable(const void* h, const void* Wb, const void* G, int64_t ldg, const void* dh, int64_t d);
int ce_bwd_dh(const __nv_bfloat16* h, const __nv_bfloat16* Wb, const int64_t* targets, const float* lse, float scale,
              __nv_bfloat16* G, int64_t ldg, __nv_bfloat16* dh, int64_t M, int64_t V, int64_t d, cudaStream_t s);

// out[n] (+)= sum_m X[m*ld+n] with `ws` >= colsum_ws(M, N) bytes.
size_t colsum_ws(int64_t M, int64_t N);
int colsum(const void* X, int bf16, int64_t M, int64_t N, int64_t ld, float* out, int accumulate,
           void* ws, size_t ws_bytes, cudaStream_t s);

// out[n] (+)= sum_p part[p*N + n] for p = 0 .. nparts-1, deterministic (fixed assignment and order).
int column_reduce(const float* part, int64_t nparts, int64_t N, float* out, int accumulate, cudaStream_t s);

// dst[i] = bf16(src[i]) (weights to the tensor-core operand type)
int to_bf16(const float* src, __nv_bfloat16* dst, int64_t n, cudaStream_t s);
// the same for up to MAX tensors in one launch (tensor t: src[t] -> dst[t], n[t] elements)
struct Bf16Casts {
  static constexpr int MAX = 4;
  const float* src[MAX];
  __nv_bfloat16* dst[MAX];
  int64_t n[MAX];
  int count;
};
int to_bf16_multi(const Bf16Casts& c, cudaStream_t s);

// GELU / GELU' with the hardware tanh approximation (tanh.approx.f32, relative error ~2^-11): used
// only where the result is rounded to bf16 (8-bit mantissa) anyway.
__device__ __forceinline__ float tanh_approx(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float gelu_bf(float x) {
  return 0.5f * x * (1.0f + tanh_approx(PGF_GELU_C * (x + PGF_GELU_A * x * x * x)));
}
__device__ __forceinline__ float gelu_prime_bf(float x) {
  const float t = tanh_approx(PGF_GELU_C * (x + PGF_GELU_A * x * x * x));
  return 0.5f * (1.0f + t) + 0.5f * x * (1.0f - t * t) * (PGF_GELU_C * (1.0f + 3.0f * PGF_GELU_A * x * x));
}

// Epilogue applied to one accumulator element, the column's bias already loaded.
__device__ __forceinline__ void epi_store_biased(const pgf_epilogue& e, void* D, int d_bf16, int64_t ldd,
                                                 int64_t m, int64_t n, float acc, float bias_n) {
  float v = fmaf(e.alpha, acc, bias_n);
  switch (e.kind) {
    case PGF_EPI_GELU:
      if (e.aux_out) stv(e.aux_out, e.aux_out_dtype, m * e.ld_aux_out + n, v);
      v = d_bf16 ? gelu_bf(v) : gelu_f(v);
      break;
    case PGF_EPI_RELU:
      if (e.aux_out) stv(e.aux_out, e.aux_out_dtype, m * e.ld_aux_out + n, v);
      v = v > 0.f ? v : 0.f;
      break;
    case PGF_EPI_DGELU: {
      const float zz = ldv(e.aux, e.aux_dtype, m * e.ld_aux + n);
      v *= d_bf16 ? gelu_prime_bf(zz) : gelu_prime_f(zz);
      break;
    }
    case PGF_EPI_DRELU:
      v *= ldv(e.aux, e.aux_dtype, m * e.ld_aux + n) > 0.f ? 1.f : 0.f;
      break;
    default:
      break;
  }
  if (e.addend) v += ldv(e.addend, e.addend_dtype, m * e.ld_addend + n);
  const int64_t o = m * ldd + n;
  if (e.accumulate) v += reinterpret_cast<float*>(D)[o];
  stv(D, d_bf16, o, v);
}

// Epilogue applied to one accumulator element.
__device__ __forceinline__ void epi_store(const pgf_epilogue& e, void* D, int d_bf16, int64_t ldd,
                                          int64_t m, int64_t n, float acc) {
  epi_store_biased(e, D, d_bf16, ldd, m, n, acc, e.bias ? e.bias[n] : 0.f);
}

}  // namespace pgf
