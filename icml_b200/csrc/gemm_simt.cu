// SIMT dense product (float32 FMA on the CUDA cores) with the fused epilogues, column sums and
// the public pgf_gemm / pgf_colsum entry points.
//
// The SIMT engine is the reference-precision path: float32 inputs are multiplied and summed in
// float32, which keeps the float32 operators within the 1e-5 parity bound.  bf16 operands go to
// the tcgen05 engine (gemm_tc.cu) when their shapes fit it.
#include "gemm.cuh"

namespace pgf {

constexpr int SG_BM = 64, SG_BN = 64, SG_BK = 16, SG_THREADS = 256;

// blockIdx.z = K slice: k in [z*kchunk, min(K, (z+1)*kchunk)); slice z > 0 writes at D + z*split_stride
// (float32 partials; only used with the plain epilogue).
__global__ void __launch_bounds__(SG_THREADS) gemm_simt_kernel(const Gemm g, int64_t kchunk, int64_t split_stride) {
  __shared__ __align__(16) float As[SG_BK][SG_BM + 4];
  __shared__ __align__(16) float Bs[SG_BK][SG_BN + 4];
  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const int64_t m0 = int64_t(blockIdx.y) * SG_BM, n0 = int64_t(blockIdx.x) * SG_BN;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;

  const int64_t kbeg = int64_t(blockIdx.z) * kchunk;
  const int64_t kend = kbeg + kchunk < g.K ? kbeg + kchunk : g.K;
  for (int64_t k0 = kbeg; k0 < kend; k0 += SG_BK) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int li = tid + i * SG_THREADS;
      int mm, kk;
      if (!g.a_trans) { kk = li % SG_BK; mm = li / SG_BK; } else { mm = li % SG_BM; kk = li / SG_BM; }
      const int64_t gm = m0 + mm, gk = k0 + kk;
      float v = 0.f;
      if (gm < g.M && gk < kend)
        v = ldv(g.A, g.a_bf16, g.a_trans ? gk * g.lda + gm : gm * g.lda + gk);
      As[kk][mm] = v;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int li = tid + i * SG_THREADS;
      int nn, kk;
      if (!g.b_trans) { kk = li % SG_BK; nn = li / SG_BK; } else { nn = li % SG_BN; kk = li / SG_BN; }
      const int64_t gn = n0 + nn, gk = k0 + kk;
      float v = 0.f;
      if (gn < g.N && gk < kend)
        v = ldv(g.B, g.b_bf16, g.b_trans ? gk * g.ldb + gn : gn * g.ldb + gk);
      Bs[kk][nn] = v;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < SG_BK; ++kk) {
      const float4 a = *reinterpret_cast<const float4*>(&As[kk][ty * 4]);
      const float4 b = *reinterpret_cast<const float4*>(&Bs[kk][tx * 4]);
      const float av[4] = {a.x, a.y, a.z, a.w};
      const float bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
  }
  void* D = blockIdx.z ? static_cast<void*>(static_cast<float*>(g.D) + blockIdx.z * split_stride) : g.D;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t m = m0 + ty * 4 + i;
    if (m >= g.M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t n = n0 + tx * 4 + j;
      if (n < g.N) epi_store(g.epi, D, g.d_bf16, g.ldd, m, n, acc[i][j]);
    }
  }
}

int run_gemm_simt(const Gemm& g, cudaStream_t s) {
  if (g.M == 0 || g.N == 0) return PGF_OK;
  dim3 grid(ceil_div(g.N, SG_BN), ceil_div(g.M, SG_BM));
  if (grid.y > 65535u) {
    // split M into launches of at most 65535 row tiles
    const int64_t rows_per = int64_t(65535) * SG_BM;
    for (int64_t r = 0; r < g.M; r += rows_per) {
      Gemm h = g;
      h.M = (g.M - r) < rows_per ? (g.M - r) : rows_per;
      const int64_t ea = g.a_bf16 ? 2 : 4, ed = g.d_bf16 ? 2 : 4;
      h.A = static_cast<const char*>(g.A) + (g.a_trans ? r : r * g.lda) * ea;
      h.D = static_cast<char*>(g.D) + r * g.ldd * ed;
      if (h.epi.aux) h.epi.aux = static_cast<const char*>(g.epi.aux) + r * g.epi.ld_aux * (g.epi.aux_dtype ? 2 : 4);
      if (h.epi.aux_out) h.epi.aux_out = static_cast<char*>(g.epi.aux_out) + r * g.epi.ld_aux_out * (g.epi.aux_out_dtype ? 2 : 4);
      if (h.epi.addend) h.epi.addend = static_cast<const char*>(g.epi.addend) + r * g.epi.ld_addend * (g.epi.addend_dtype ? 2 : 4);
      PGF_TRY(run_gemm_simt(h, s));
    }
    return PGF_OK;
  }
  prof_begin(PROF_GEMM_SIMT, s);
  gemm_simt_kernel<<<grid, SG_THREADS, 0, s>>>(g, g.K, 0);
  prof_end(PROF_GEMM_SIMT, s, 2.0 * double(g.M) * double(g.N) * double(g.K));
  PGF_LAUNCH_CHECK();
  return PGF_OK;
}

int split_slices_simt(int64_t M, int64_t N, int64_t K) {
  const int64_t tiles = ceil_div(M, SG_BM) * ceil_div(N, SG_BN);
  const int64_t target = int64_t(sm_count()) * 4;  // resident 256-thread CTAs to aim for
  if (tiles * 2 > target) return 1;
  int64_t S = ceil_div(target, tiles);
  if (S > K / 256) S = K / 256;  // at least 256 deep per slice
  if (S > 64) S = 64;
  return S < 1 ? 1 : int(S);
}

size_t gemm_split_ws(int64_t M, int64_t N, int64_t K) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  const int a = split_slices_tc(M, N, K), b = split_slices_simt(M, N, K);
  const int S = a > b ? a : b;
  return S > 1 ? size_t(S) * size_t(M) * size_t(N) * 4 : 0;
}

static int run_gemm_simt_split(const Gemm& g, int slices, float* part, int* launched, cudaStream_t s) {
  int64_t kchunk = ceil_div(ceil_div(g.K, slices), SG_BK) * SG_BK;
  const int used = int(ceil_div(g.K, kchunk));
  Gemm h = g;
  h.D = part; h.d_bf16 = 0; h.ldd = g.N;
  h.epi = epi_default();
  dim3 grid(ceil_div(g.N, SG_BN), ceil_div(g.M, SG_BM), unsigned(used));
  prof_begin(PROF_GEMM_SIMT, s);
  gemm_simt_kernel<<<grid, SG_THREADS, 0, s>>>(h, kchunk, g.M * g.N);
  prof_end(PROF_GEMM_SIMT, s, 2.0 * double(g.M) * double(g.N) * double(g.K));
  PGF_LAUNCH_CHECK();
  *launched = used;
  return PGF_OK;
}

// D = epi(sum over slices of the partial products), slices added in index order.
// Sum of the K slices' partial products, in slice order, then the epilogue.  A thread owns VEC
// adjacent outputs (float4 loads when N % 4 == 0) and keeps SK slices' loads in flight before it
// adds them (the adds stay in slice order: the same sum as one slice at a time).
template <int VEC>
__global__ void splitk_reduce_kernel(const float* __restrict__ part, int slices, int64_t M, int64_t N,
                                     const pgf_epilogue e, void* D, int d_bf16, int64_t ldd) {
  constexpr int SK = 8;
  const int64_t MN = M * N, nv = MN / VEC;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < nv; i += int64_t(gridDim.x) * blockDim.x) {
    float v[VEC];
#pragma unroll
    for (int k = 0; k < VEC; ++k) v[k] = 0.f;
    int z = 0;
    for (; z + SK <= slices; z += SK) {
      float a[SK][VEC];
#pragma unroll
      for (int q = 0; q < SK; ++q) {
        if (VEC == 4) {
          const float4 t = __ldg(reinterpret_cast<const float4*>(part + (z + q) * MN) + i);
          a[q][0] = t.x; a[q][VEC > 1 ? 1 : 0] = t.y; a[q][VEC > 2 ? 2 : 0] = t.z; a[q][VEC > 3 ? 3 : 0] = t.w;
        } else {
          a[q][0] = __ldg(part + (z + q) * MN + i);
        }
      }
#pragma unroll
      for (int q = 0; q < SK; ++q)
#pragma unroll
        for (int k = 0; k < VEC; ++k) v[k] += a[q][k];
    }
    for (; z < slices; ++z)
#pragma unroll
      for (int k = 0; k < VEC; ++k) v[k] += __ldg(part + z * MN + i * VEC + k);
#pragma unroll
    for (int k = 0; k < VEC; ++k) {
      const int64_t j = i * VEC + k;
      const int64_t m = j / N, n = j - m * N;
      epi_store(e, D, d_bf16, ldd, m, n, v[k]);
    }
  }
}

static int splitk_finish(const Gemm& g, const float* part, int used, cudaStream_t s) {
  const bool vec = g.N % 4 == 0 && aligned(part, 16);
  int64_t blocks = ceil_div(g.M * g.N / (vec ? 4 : 1), 256);
  if (blocks > int64_t(sm_count()) * 8) blocks = int64_t(sm_count()) * 8;
  if (blocks < 1) blocks = 1;
  if (vec)
    splitk_reduce_kernel<4><<<unsigned(blocks), 256, 0, s>>>(part, used, g.M, g.N, g.epi, g.D, g.d_bf16, g.ldd);
  else
    splitk_reduce_kernel<1><<<unsigned(blocks), 256, 0, s>>>(part, used, g.M, g.N, g.epi, g.D, g.d_bf16, g.ldd);
  PGF_LAUNCH_CHECK();
  return PGF_OK;
}

int run_gemm(const Gemm& g, cudaStream_t s) {
  const size_t per = size_t(g.M > 0 ? g.M : 0) * size_t(g.N > 0 ? g.N : 0) * 4;
  const size_t fit_sz = (g.ws && per) ? g.ws_bytes / per : 0;
  const int fit = fit_sz > 64 ? 64 : int(fit_sz);  // slices the scratch can hold
  float* part = static_cast<float*>(g.ws);
  int used = 0;
  if (tc_usable(g)) {
    int S = split_slices_tc(g.M, g.N, g.K);
    if (S > fit) S = fit;
    const int rc = S > 1 ? run_gemm_tc_split(g, S, part, &used, s) : run_gemm_tc(g, s);
    if (rc == PGF_OK) return S > 1 ? splitk_finish(g, part, used, s) : PGF_OK;
    if (rc != PGF_ERR_UNSUPPORTED) return rc;
    clear_error();
  }
  int S = split_slices_simt(g.M, g.N, g.K);
  if (S > fit) S = fit;
  if (S > 1) {
    PGF_TRY(run_gemm_simt_split(g, S, part, &used, s));
    return splitk_finish(g, part, used, s);
  }
  return run_gemm_simt(g, s);
}

// ---------------------------------------------------------------------------
// column sums, fixed two-level order
// ---------------------------------------------------------------------------
constexpr int CS_ROWS = 256;

__global__ void colsum_part_kernel(const void* __restrict__ X, int bf16, int64_t M, int64_t N,
                                   int64_t ld, int64_t rows, float* __restrict__ part) {
  const int64_t n = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (n >= N) return;
  const int64_t r0 = int64_t(blockIdx.y) * rows;
  const int64_t r1 = r0 + rows < M ? r0 + rows : M;
  float s = 0.f;
  for (int64_t r = r0; r < r1; ++r) s += ldv(X, bf16, r * ld + n);
  part[int64_t(blockIdx.y) * N + n] = s;
}

// out[c] (+)= sum_p part[p*N + c].  A CTA owns 32 columns; warp w sums parts w, w+32, w+64, ... in
// order (coalesced 128 B rows), then the 32 warp sums are added in warp order: deterministic.
constexpr int CR_WARPS = 32;
__global__ void __launch_bounds__(CR_WARPS * 32)
column_reduce_kernel(const float* __restrict__ part, int64_t nparts, int64_t N, float* __restrict__ out,
                     int accumulate) {
  __shared__ float sm[CR_WARPS][33];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t c = int64_t(blockIdx.x) * 32 + lane;
  float s = 0.f;
  if (c < N) {
    int64_t p = warp;
    for (; p + 7 * CR_WARPS < nparts; p += 8 * CR_WARPS) {
      float a[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) a[q] = __ldg(part + (p + q * CR_WARPS) * N + c);
#pragma unroll
      for (int q = 0; q < 8; ++q) s += a[q];
    }
    for (; p < nparts; p += CR_WARPS) s += part[p * N + c];
  }
  sm[warp][lane] = s;
  __syncthreads();
  if (warp == 0 && c < N) {
    float t = 0.f;
#pragma unroll 8
    for (int w = 0; w < CR_WARPS; ++w) t += sm[w][lane];
    out[c] = accumulate ? out[c] + t : t;
  }
}

int column_reduce(const float* part, int64_t nparts, int64_t N, float* out, int accumulate, cudaStream_t s) {
  if (N <= 0) return PGF_OK;
  column_reduce_kernel<<<unsigned(ceil_div(N, 32)), CR_WARPS * 32, 0, s>>>(part, nparts, N, out, accumulate);
  PGF_LAUNCH_CHECK();
  return PGF_OK;
}

// Rows per slab (one partial row each): CS_ROWS, halved (down to 32) while the vector kernel's grid
// would not give every SM four CTAs, so narrow outputs (a few hundred columns) still fill the GPU.
static int64_t colsum_rows(int64_t M, int64_t N) {
  int64_t rows = CS_ROWS;
  const int64_t want = int64_t(sm_count()) * 4;
  while (rows > 32 && ceil_div(N, 256) * ceil_div(M < 1 ? 1 : M, rows) < want) rows /= 2;
  return rows;
}

size_t colsum_ws(int64_t M, int64_t N) {
  return Workspace::round(size_t(ceil_div(M < 1 ? 1 : M, colsum_rows(M, N))) * size_t(N) * 4);
}

// Vector form: a CTA sums a slab of `rows` rows of 256 columns; a thread owns 8 adjacent columns
// (one 16-byte load per row in bf16, two in float32), warp w takes rows w, w+8, ... of the slab in
// order, and the 8 warp partials are added in warp order.  Needs N % 8 == 0 and 16-byte aligned rows.
constexpr int CSV_WARPS = 8;
__global__ void __launch_bounds__(CSV_WARPS * 32)
colsum_part_vec_kernel(const void* __restrict__ X, int bf16, int64_t M, int64_t N, int64_t ld, int64_t rows,
                       float* __restrict__ part) {
  __shared__ float sm[CSV_WARPS][256 + 4];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t c0 = int64_t(blockIdx.x) * 256 + lane * 8;
  const int64_t r0 = int64_t(blockIdx.y) * rows;
  const int64_t r1 = r0 + rows < M ? r0 + rows : M;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (c0 < N) {
    if (bf16) {
      const __nv_bfloat16* Xb = static_cast<const __nv_bfloat16*>(X);
#pragma unroll 4
      for (int64_t r = r0 + warp; r < r1; r += CSV_WARPS) {
        const uint4 v = __ldg(reinterpret_cast<const uint4*>(Xb + r * ld + c0));
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          acc[2 * k] += __uint_as_float(w[k] << 16);
          acc[2 * k + 1] += __uint_as_float(w[k] & 0xFFFF0000u);
        }
      }
    } else {
      const float* Xf = static_cast<const float*>(X);
#pragma unroll 4
      for (int64_t r = r0 + warp; r < r1; r += CSV_WARPS) {
        const float4 a = __ldg(reinterpret_cast<const float4*>(Xf + r * ld + c0));
        const float4 b = __ldg(reinterpret_cast<const float4*>(Xf + r * ld + c0 + 4));
        acc[0] += a.x; acc[1] += a.y; acc[2] += a.z; acc[3] += a.w;
        acc[4] += b.x; acc[5] += b.y; acc[6] += b.z; acc[7] += b.w;
      }
    }
  }
#pragma unroll
  for (int k = 0; k < 8; ++k) sm[warp][lane * 8 + k] = acc[k];
  __syncthreads();
  const int64_t c = int64_t(blockIdx.x) * 256 + threadIdx.x;
  if (c < N) {
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < CSV_WARPS; ++w) t += sm[w][threadIdx.x];
    part[int64_t(blockIdx.y) * N + c] = t;
  }
}

int colsum(const void* X, int bf16, int64_t M, int64_t N, int64_t ld, float* out, int accumulate,
           void* ws, size_t ws_bytes, cudaStream_t s) {
  if (N == 0) return PGF_OK;
  if (M == 0) {
    if (!accumulate) PGF_CUDA(cudaMemsetAsync(out, 0, N * 4, s));
    return PGF_OK;
  }
  const int64_t rows = colsum_rows(M, N);
  const int64_t np = ceil_div(M, rows);
  if (size_t(np) * N * 4 > ws_bytes) { set_error("colsum: workspace too small"); return PGF_ERR_WORKSPACE; }
  if (np > 65535) { set_error("colsum: too many rows"); return PGF_ERR_UNSUPPORTED; }
  float* part = static_cast<float*>(ws);
  const int64_t es = bf16 ? 2 : 4;
  if (N % 8 == 0 && aligned(X, 16) && (ld * es) % 16 == 0) {
    colsum_part_vec_kernel<<<dim3(ceil_div(N, 256), unsigned(np)), CSV_WARPS * 32, 0, s>>>(X, bf16, M, N, ld, rows,
                                                                                          part);
  } else {
    colsum_part_kernel<<<dim3(ceil_div(N, 128), unsigned(np)), 128, 0, s>>>(X, bf16, M, N, ld, rows, part);
  }
  PGF_LAUNCH_CHECK();
  return column_reduce(part, np, N, out, accumulate, s);
}

__global__ void to_bf16_kernel(const float* __restrict__ src, __nv_bfloat16* __restrict__ dst, int64_t n) {
  int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (; i < n; i += stride) dst[i] = __float2bfloat16_rn(src[i]);
}

int to_bf16(const float* src, __nv_bfloat16* dst, int64_t n, cudaStream_t s) {
  if (n == 0) return PGF_OK;
  int blocks = ceil_div(n, 256);
  if (blocks > 148 * 16) blocks = 148 * 16;
  to_bf16_kernel<<<blocks, 256, 0, s>>>(src, dst, n);
  PGF_LAUNCH_CHECK();
  return PGF_OK;
}

// Several tensors in one launch: grid row blockIdx.y converts tensor blockIdx.y (the per-element
// loop of to_bf16_kernel), so a call's weight copies cost one launch instead of one each.
__global__ void to_bf16_multi_kernel(Bf16Casts c) {
  const int t = blockIdx.y;
  const float* __restrict__ src = c.src[t];
  __nv_bfloat16* __restrict__ dst = c.dst[t];
  const int64_t n = c.n[t];
  int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (; i < n; i += stride) dst[i] = __float2bfloat16_rn(src[i]);
}

int to_bf16_multi(const Bf16Casts& c, cudaStream_t s) {
  if (c.count < 1 || c.count > Bf16Casts::MAX) {
    set_error("to_bf16_multi: %d tensors (1..%d)", c.count, Bf16Casts::MAX);
    return PGF_ERR_INVALID;
  }
  int64_t most = 0;
  for (int t = 0; t < c.count; ++t) most = c.n[t] > most ? c.n[t] : most;
  if (most == 0) return PGF_OK;
  int blocks = ceil_div(most, 256);
  if (blocks > 148 * 16) blocks = 148 * 16;
  to_bf16_multi_kernel<<<dim3(unsigned(blocks), unsigned(c.count)), 256, 0, s>>>(c);
  PGF_LAUNCH_CHECK();
  return PGF_OK;
}

}  // namespace pgf

using namespace pgf;

extern "C" int pgf_gemm(int64_t M, int64_t N, int64_t K, const void* A, int a_dtype, int64_t lda,
                        int a_trans, const void* B, int b_dtype, int64_t ldb, int b_trans, void* D,
                        int d_dtype, int64_t ldd, const pgf_epilogue* epi, pgf_stream_t stream) {
  return pgf_gemm_ex(M, N, K, A, a_dtype, lda, a_trans, B, b_dtype, ldb, b_trans, D, d_dtype, ldd, epi, nullptr, 0,
                     stream);
}

extern "C" size_t pgf_gemm_workspace(int64_t M, int64_t N, int64_t K) { return gemm_split_ws(M, N, K); }

extern "C" int pgf_gemm_ex(int64_t M, int64_t N, int64_t K, const void* A, int a_dtype, int64_t lda, int a_trans,
                           const void* B, int b_dtype, int64_t ldb, int b_trans, void* D, int d_dtype, int64_t ldd,
                           const pgf_epilogue* epi, void* ws, size_t ws_bytes, pgf_stream_t stream) {
  PGF_CHECK_ARG(M >= 0 && N >= 0 && K >= 0, "gemm: negative size");
  PGF_CHECK_ARG((M == 0 || N == 0 || K == 0) || (A && B), "gemm: null operand");
  PGF_CHECK_ARG(D || M == 0 || N == 0, "gemm: null output");
  PGF_CHECK_ARG((a_dtype == 0 || a_dtype == 1) && (b_dtype == 0 || b_dtype == 1) &&
                    (d_dtype == 0 || d_dtype == 1),
                "gemm: bad dtype");
  Gemm g = gemm_make(M, N, K, A, a_dtype, lda, a_trans, B, b_dtype, ldb, b_trans, D, d_dtype, ldd);
  if (epi) g.epi = *epi;
  PGF_CHECK_ARG(!g.epi.accumulate || d_dtype == PGF_DTYPE_F32, "gemm: accumulate needs float32 D");
  PGF_CHECK_ARG(g.epi.kind >= PGF_EPI_NONE && g.epi.kind <= PGF_EPI_DRELU, "gemm: bad epilogue kind %d",
                g.epi.kind);
  PGF_CHECK_ARG(!(g.epi.kind == PGF_EPI_DGELU || g.epi.kind == PGF_EPI_DRELU) || g.epi.aux,
                "gemm: DGELU/DRELU need aux");
  PGF_CHECK_ARG(!ws || (reinterpret_cast<uintptr_t>(ws) & 15) == 0, "gemm: workspace must be 16-byte aligned");
  g.ws = ws;
  g.ws_bytes = ws ? ws_bytes : 0;
  return run_gemm(g, as_stream(stream));
}

extern "C" size_t pgf_colsum_workspace(int64_t M, int64_t N) { return colsum_ws(M, N); }

extern "C" int pgf_colsum(const void* X, int dtype, int64_t M, int64_t N, int64_t ld, float* out,
                          int accumulate, void* ws, size_t ws_bytes, pgf_stream_t stream) {
  PGF_CHECK_ARG(out && (X || M == 0), "colsum: null pointer");
  return colsum(X, dtype, M, N, ld, out, accumulate, ws, ws_bytes, as_stream(stream));
}
