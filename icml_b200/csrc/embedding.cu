// Embedding gather and its deterministic gradient (pgf_embedding.py:7-71).
//
// Gradient = stable LSD radix sort of (id, token) pairs, 8-bit digits, then a segmented sum of
// the gradient rows in sorted (= ascending token) order.  The sorted array is cut into tiles of
// SEG_TILE entries; segments that stay inside a tile are written directly, segments that cross
// tiles leave per-tile partials that the tile holding the segment's first entry adds up in tile
// order.  Every sum therefore runs in one fixed order: the result is bitwise reproducible.
#include "common.cuh"

namespace pgf {

constexpr int RADIX_TILE = 2048;      // elements ranked by one warp, in order
constexpr int RADIX_WARPS = 4;        // tiles per CTA
constexpr int SEG_TILE = 256;         // sorted entries per segment-sum tile
constexpr int SEG_THREADS = 256;
constexpr int SEG_BATCH = 8;          // gradient rows loaded together per thread

// Out-of-range ids give zero rows (the API does not synchronise to report them).
template <class T>
__global__ void embedding_fwd_kernel(const int64_t* __restrict__ ids, const float* __restrict__ W,
                                     T* __restrict__ y, int64_t n, int64_t vocab, int dim) {
  int64_t t = blockIdx.x;
  int64_t id = ids[t];
  T* yr = y + t * dim;
  if (id < 0 || id >= vocab) {
    for (int c = threadIdx.x; c < dim; c += blockDim.x) st(yr, c, 0.f);
    return;
  }
  const float* wr = W + id * dim;
  for (int c = threadIdx.x; c < dim; c += blockDim.x) st(yr, c, wr[c]);
}

// The same with a warp per token and 16-byte rows pieces (dim a multiple of 4, aligned rows): eight
// tokens per CTA instead of one CTA per token.
__device__ __forceinline__ void st4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }
__device__ __forceinline__ void st4(__nv_bfloat16* p, float4 v) {
  const __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
  uint2 u;
  u.x = *reinterpret_cast<const uint32_t*>(&a);
  u.y = *reinterpret_cast<const uint32_t*>(&b);
  *reinterpret_cast<uint2*>(p) = u;
}
template <class T>
__global__ void __launch_bounds__(256) embedding_fwd_vec_kernel(const int64_t* __restrict__ ids,
                                                                 const float* __restrict__ W, T* __restrict__ y,
                                                                 int64_t n, int64_t vocab, int dim) {
  const int64_t t = int64_t(blockIdx.x) * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= n) return;
  const int64_t id = ids[t];
  const bool ok = id >= 0 && id < vocab;
  const float4* wr = reinterpret_cast<const float4*>(W + (ok ? id : 0) * dim);
  T* yr = y + t * dim;
  for (int c4 = lane; c4 < dim / 4; c4 += 32) st4(yr + 4 * c4, ok ? __ldg(wr + c4) : make_float4(0.f, 0.f, 0.f, 0.f));
}

__global__ void make_keys_kernel(const int64_t* __restrict__ ids, uint32_t* __restrict__ keys,
                                 uint32_t* __restrict__ vals, int64_t n, int64_t vocab,
                                 int* __restrict__ bad) {
  int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  int64_t id = ids[i];
  if (id < 0 || id >= vocab) {
    atomicExch(bad, 1);
    id = vocab;  // sorts after every valid id; its segment is skipped
  }
  keys[i] = uint32_t(id);
  vals[i] = uint32_t(i);
}

// hist[digit * ntiles + tile] = count of `digit` in tile.
__global__ void radix_hist_kernel(const uint32_t* __restrict__ keys, int64_t n, int shift,
                                  int ntiles, uint32_t* __restrict__ hist) {
  __shared__ uint32_t h[RADIX_WARPS][256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < RADIX_WARPS * 256; i += blockDim.x) (&h[0][0])[i] = 0;
  __syncthreads();
  const int tile = blockIdx.x * RADIX_WARPS + warp;
  if (tile < ntiles) {
    int64_t a = int64_t(tile) * RADIX_TILE;
    int64_t b = a + RADIX_TILE < n ? a + RADIX_TILE : n;
    for (int64_t i = a + lane; i < b; i += 32) atomicAdd(&h[warp][(keys[i] >> shift) & 255u], 1u);
  }
  __syncwarp();
  if (tile < ntiles)
    for (int dgt = lane; dgt < 256; dgt += 32) hist[int64_t(dgt) * ntiles + tile] = h[warp][dgt];
}

// In-place exclusive scan of `a` (length m) with one CTA of 1024 threads.
__global__ void exclusive_scan_kernel(uint32_t* __restrict__ a, int64_t m) {
  __shared__ uint32_t part[1024];
  const int tid = threadIdx.x;
  int64_t per = (m + 1023) / 1024;
  int64_t lo = tid * per, hi = lo + per < m ? lo + per : m;
  uint32_t s = 0;
  for (int64_t i = lo; i < hi; ++i) s += a[i];
  part[tid] = s;
  __syncthreads();
  for (int o = 1; o < 1024; o <<= 1) {
    uint32_t v = tid >= o ? part[tid - o] : 0u;
    __syncthreads();
    part[tid] += v;
    __syncthreads();
  }
  uint32_t run = tid ? part[tid - 1] : 0u;
  for (int64_t i = lo; i < hi; ++i) {
    uint32_t v = a[i];
    a[i] = run;
    run += v;
  }
}

// Stable scatter: one warp walks its tile 32 entries at a time, in order.
__global__ void radix_scatter_kernel(const uint32_t* __restrict__ kin, const uint32_t* __restrict__ vin,
                                     uint32_t* __restrict__ kout, uint32_t* __restrict__ vout,
                                     int64_t n, int shift, int ntiles,
                                     const uint32_t* __restrict__ offs) {
  __shared__ uint32_t base[RADIX_WARPS][256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x * RADIX_WARPS + warp;
  if (tile >= ntiles) return;
  for (int dgt = lane; dgt < 256; dgt += 32) base[warp][dgt] = offs[int64_t(dgt) * ntiles + tile];
  __syncwarp();
  int64_t a = int64_t(tile) * RADIX_TILE;
  int64_t b = a + RADIX_TILE < n ? a + RADIX_TILE : n;
  const unsigned lt = (1u << lane) - 1u;
  // the next 32 keys and values are loaded while the current ones are ranked and stored
  uint32_t kn = a + lane < b ? kin[a + lane] : 0u, vn = a + lane < b ? vin[a + lane] : 0u;
  for (int64_t i0 = a; i0 < b; i0 += 32) {
    int64_t i = i0 + lane;
    bool valid = i < b;
    const uint32_t k = kn, v = vn;
    if (i + 32 < b) {
      kn = kin[i + 32];
      vn = vin[i + 32];
    }
    int dgt = valid ? int((k >> shift) & 255u) : 256 + lane;  // invalid lanes match nobody
    unsigned peers = __match_any_sync(0xffffffffu, dgt);
    uint32_t pos = 0;
    if (valid) pos = base[warp][dgt] + __popc(peers & lt);
    __syncwarp();
    if (valid) {
      kout[pos] = k;
      vout[pos] = v;
      int leader = __ffs(peers) - 1;
      if (lane == leader) base[warp][dgt] += __popc(peers);
    }
    __syncwarp();
  }
}

// Segment sums over one tile of sorted entries.  Writes finished segments to grad_weight and
// leaves head/tail partials for segments that cross the tile's edges.
template <class T>
__global__ void __launch_bounds__(SEG_THREADS)
seg_tile_kernel(const uint32_t* __restrict__ keys, const uint32_t* __restrict__ pos, int64_t n,
                const T* __restrict__ g, int dim, uint32_t vocab, float* __restrict__ gw,
                int accumulate, float* __restrict__ head, float* __restrict__ tail) {
  const int tile = blockIdx.x;
  const int64_t a = int64_t(tile) * SEG_TILE;
  const int64_t b = a + SEG_TILE < n ? a + SEG_TILE : n;
  const bool head_cont = a > 0 && keys[a - 1] == keys[a];
  const bool tail_cont = b < n && keys[b] == keys[b - 1];
  for (int c = threadIdx.x; c < dim; c += blockDim.x) {
    float s = 0.f;
    bool first = true;  // current segment is the tile's first
    // entries are taken SEG_BATCH at a time: their gradient rows are loaded together (independent
    // loads in flight), then summed in order, so the sums are those of the one-by-one loop
    for (int64_t i0 = a; i0 < b; i0 += SEG_BATCH) {
      float v[SEG_BATCH];
#pragma unroll
      for (int q = 0; q < SEG_BATCH; ++q) v[q] = i0 + q < b ? ld(g, int64_t(pos[i0 + q]) * dim + c) : 0.f;
#pragma unroll
      for (int q = 0; q < SEG_BATCH; ++q) {
        const int64_t i = i0 + q;
        if (i >= b) break;
        s += v[q];
        const bool seg_end = (i + 1 == b) || keys[i + 1] != keys[i];
        if (!seg_end) continue;
        const uint32_t k = keys[i];
        const bool last = (i + 1 == b);
        if (first && head_cont) {
          head[int64_t(tile) * dim + c] = s;          // piece of a segment owned by an earlier tile
        } else if (last && tail_cont) {
          tail[int64_t(tile) * dim + c] = s;          // this tile owns a segment that continues
        } else if (k < vocab) {
          float* dst = gw + int64_t(k) * dim + c;     // segment entirely inside the tile
          *dst = accumulate ? *dst + s : s;
        }
        s = 0.f;
        first = false;
      }
    }
  }
}

// Owner tiles (last segment continues past the tile) add the following tiles' head partials.
__global__ void seg_fixup_kernel(const uint32_t* __restrict__ keys, int64_t n, int ntiles, int dim,
                                 uint32_t vocab, float* __restrict__ gw, int accumulate,
                                 const float* __restrict__ head, const float* __restrict__ tail) {
  const int tile = blockIdx.x;
  const int64_t a = int64_t(tile) * SEG_TILE;
  const int64_t b = a + SEG_TILE < n ? a + SEG_TILE : n;
  if (!(b < n && keys[b] == keys[b - 1])) return;
  const bool head_cont = a > 0 && keys[a - 1] == keys[a];
  // a tile whose single segment started earlier is not an owner
  if (head_cont && keys[a] == keys[b - 1]) return;
  const uint32_t k = keys[b - 1];
  for (int c = threadIdx.x; c < dim; c += blockDim.x) {
    float s = tail[int64_t(tile) * dim + c];
    for (int t2 = tile + 1; t2 < ntiles; ++t2) {
      s += head[int64_t(t2) * dim + c];
      int64_t a2 = int64_t(t2) * SEG_TILE;
      int64_t b2 = a2 + SEG_TILE < n ? a2 + SEG_TILE : n;
      if (!(b2 < n && keys[b2] == k)) break;  // segment ends inside tile t2
    }
    if (k < vocab) {
      float* dst = gw + int64_t(k) * dim + c;
      *dst = accumulate ? *dst + s : s;
    }
  }
}

struct EmbWs {
  uint32_t *k0, *v0, *k1, *v1, *hist;
  float *head, *tail;
  int* bad;
};

static int radix_ntiles(int64_t n) { return ceil_div(n, RADIX_TILE); }
static int seg_ntiles(int64_t n) { return ceil_div(n, SEG_TILE); }

static bool carve(Workspace& W, EmbWs& e, int64_t n, int64_t dim) {
  e.k0 = W.take<uint32_t>(n);
  e.v0 = W.take<uint32_t>(n);
  e.k1 = W.take<uint32_t>(n);
  e.v1 = W.take<uint32_t>(n);
  e.hist = W.take<uint32_t>(size_t(256) * radix_ntiles(n));
  e.head = W.take<float>(size_t(seg_ntiles(n)) * dim);
  e.tail = W.take<float>(size_t(seg_ntiles(n)) * dim);
  e.bad = W.take<int>(1);
  return e.k0 && e.v0 && e.k1 && e.v1 && e.hist && e.head && e.tail && e.bad;
}

template <class T>
static int emb_bwd_impl(const int64_t* ids, const T* g, float* gw, int accumulate, int64_t n,
                        int64_t vocab, int dim, EmbWs& e, cudaStream_t s) {
  PGF_CUDA(cudaMemsetAsync(e.bad, 0, sizeof(int), s));
  make_keys_kernel<<<ceil_div(n, 256), 256, 0, s>>>(ids, e.k0, e.v0, n, vocab, e.bad);
  PGF_LAUNCH_CHECK();
  int bits = 1;
  while ((int64_t(1) << bits) <= vocab) ++bits;  // keys lie in [0, vocab]
  const int passes = (bits + 7) / 8;
  const int nt = radix_ntiles(n);
  uint32_t *kin = e.k0, *vin = e.v0, *kout = e.k1, *vout = e.v1;
  for (int p = 0; p < passes; ++p) {
    const int shift = 8 * p;
    radix_hist_kernel<<<ceil_div(nt, RADIX_WARPS), RADIX_WARPS * 32, 0, s>>>(kin, n, shift, nt, e.hist);
    PGF_LAUNCH_CHECK();
    exclusive_scan_kernel<<<1, 1024, 0, s>>>(e.hist, int64_t(256) * nt);
    PGF_LAUNCH_CHECK();
    radix_scatter_kernel<<<ceil_div(nt, RADIX_WARPS), RADIX_WARPS * 32, 0, s>>>(kin, vin, kout, vout, n,
                                                                              shift, nt, e.hist);
    PGF_LAUNCH_CHECK();
    uint32_t* t;
    t = kin; kin = kout; kout = t;
    t = vin; vin = vout; vout = t;
  }
  if (!accumulate) PGF_CUDA(cudaMemsetAsync(gw, 0, size_t(vocab) * dim * sizeof(float), s));
  const int st = seg_ntiles(n);
  seg_tile_kernel<T><<<st, SEG_THREADS, 0, s>>>(kin, vin, n, g, dim, uint32_t(vocab), gw, 1,
                                               e.head, e.tail);
  PGF_LAUNCH_CHECK();
  seg_fixup_kernel<<<st, SEG_THREADS, 0, s>>>(kin, n, st, dim, uint32_t(vocab), gw, 1, e.head, e.tail);
  PGF_LAUNCH_CHECK();
  return PGF_OK;
}

}  // namespace pgf

using namespace pgf;

extern "C" int pgf_embedding_fwd(const int64_t* ids, const float* weight, void* y, int64_t n_tokens,
                                 int64_t vocab, int64_t dim, int dtype, pgf_stream_t stream) {
  PGF_CHECK_ARG(ids && weight && y, "embedding_fwd: null pointer");
  PGF_CHECK_ARG(n_tokens >= 0 && vocab > 0 && dim > 0 && n_tokens < (int64_t(1) << 31),
                "embedding_fwd: bad shape");
  if (n_tokens == 0) return PGF_OK;
  cudaStream_t s = as_stream(stream);
  const size_t ya = dtype == PGF_DTYPE_F32 ? 16 : 8;
  if (dim % 4 == 0 && reinterpret_cast<uintptr_t>(weight) % 16 == 0 && reinterpret_cast<uintptr_t>(y) % ya == 0 &&
      (dtype == PGF_DTYPE_F32 || dtype == PGF_DTYPE_BF16)) {
    const unsigned grid = unsigned((n_tokens + 7) / 8);
    if (dtype == PGF_DTYPE_F32)
      embedding_fwd_vec_kernel<float><<<grid, 256, 0, s>>>(ids, weight, (float*)y, n_tokens, vocab, int(dim));
    else
      embedding_fwd_vec_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(ids, weight, (__nv_bfloat16*)y, n_tokens,
                                                                   vocab, int(dim));
    PGF_LAUNCH_CHECK();
    return PGF_OK;
  }
  int threads = dim >= 256 ? 256 : int((dim + 31) / 32 * 32);
  if (dtype == PGF_DTYPE_F32)
    embedding_fwd_kernel<float><<<unsigned(n_tokens), threads, 0, s>>>(ids, weight, (float*)y,
                                                                       n_tokens, vocab, int(dim));
  else if (dtype == PGF_DTYPE_BF16)
    embedding_fwd_kernel<__nv_bfloat16><<<unsigned(n_tokens), threads, 0, s>>>(
        ids, weight, (__nv_bfloat16*)y, n_tokens, vocab, int(dim));
  else { set_error("embedding_fwd: bad dtype"); return PGF_ERR_INVALID; }
  PGF_LAUNCH_CHECK();
  return PGF_OK;
}

extern "C" size_t pgf_embedding_bwd_workspace(int64_t n, int64_t vocab, int64_t dim) {
  (void)vocab;
  if (n < 1) n = 1;
  size_t b = 0;
  b += 4 * Workspace::round(size_t(n) * 4);
  b += Workspace::round(size_t(256) * radix_ntiles(n) * 4);
  b += 2 * Workspace::round(size_t(seg_ntiles(n)) * dim * 4);
  b += Workspace::round(4);
  return b + 256;
}

extern "C" int pgf_embedding_bwd(const int64_t* ids, const void* g, float* grad_weight,
                                 int accumulate, int64_t n, int64_t vocab, int64_t dim, int dtype,
                                 void* ws, size_t ws_bytes, pgf_stream_t stream) {
  PGF_CHECK_ARG(ids && g && grad_weight, "embedding_bwd: null pointer");
  PGF_CHECK_ARG(n >= 0 && vocab > 0 && vocab < (int64_t(1) << 30) && dim > 0 &&
                    n < (int64_t(1) << 31),
                "embedding_bwd: bad shape");
  cudaStream_t s = as_stream(stream);
  if (n == 0) {
    if (!accumulate) PGF_CUDA(cudaMemsetAsync(grad_weight, 0, size_t(vocab) * dim * 4, s));
    return PGF_OK;
  }
  Workspace W(ws, ws_bytes);
  EmbWs e;
  if (!carve(W, e, n, dim)) { set_error("embedding_bwd: workspace too small"); return PGF_ERR_WORKSPACE; }
  if (dtype == PGF_DTYPE_F32)
    return emb_bwd_impl(ids, (const float*)g, grad_weight, accumulate, n, vocab, int(dim), e, s);
  if (dtype == PGF_DTYPE_BF16)
    return emb_bwd_impl(ids, (const __nv_bfloat16*)g, grad_weight, accumulate, n, vocab, int(dim), e, s);
  set_error("embedding_bwd: bad dtype");
  return PGF_ERR_INVALID;
}
