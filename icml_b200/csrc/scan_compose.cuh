// Chunk-state composition of the chunked selective scans, segmented over the warps of a block.
//
// Both scan variants summarise every chunk of Tc tokens from a zero state, then need the state
// entering each chunk: a first-order linear recurrence over chunks, one per (batch, channel, state)
// chain.  A block owns 32 consecutive chains (one per lane) and splits the chunk sequence into
// CSEG contiguous runs, one per warp:
//   1. each warp composes its run from a zero state into an affine summary (multiplier, offset);
//   2. each warp folds the summaries of the runs before it (in run order) into its incoming state;
//   3. each warp walks its run again from that state and writes the per-chunk states.
// The per-chunk inputs are re-read in step 3 (from L2); the dependent chain per thread is
// 2 * nC / CSEG steps instead of nC, and the block has CSEG times more threads in flight.
// Results are deterministic (fixed run boundaries and fold order).
#pragma once
#include "common.cuh"

namespace pgf {

constexpr int CSEG = 16;         // warps (chunk runs) per compose block
constexpr int CSEG_PF = 8;       // chunks whose inputs are loaded ahead of the dependent chain

// Forward: H_{c+1} = exp2(A2 * sdt[c*cs]) * H_c + hloc[c*hs], H_0 = H0; hC[c*hs] = H_c for
// c = 0 .. nC.  Returns H_nC and, through sum_out, sum_c sdt[c*cs] (valid in every lane of every
// warp).  All threads of the block must call it (it synchronises the block).
__device__ __forceinline__ float compose_fwd_segmented(bool valid, const float* __restrict__ sdt, int64_t cs,
                                                       const float* __restrict__ hloc, int64_t hs,
                                                       float* __restrict__ hC, float A2, float H0, int64_t nC,
                                                       float* sum_out) {
  __shared__ float sP[CSEG][32], sH[CSEG][32], sS[CSEG][32];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int64_t run = (nC + CSEG - 1) / CSEG;
  const int64_t c0 = w * run < nC ? w * run : nC;
  const int64_t c1 = c0 + run < nC ? c0 + run : nC;
  float P = 1.f, H = 0.f, S = 0.f;
  if (valid) {
    int64_t c = c0;
    for (; c + CSEG_PF <= c1; c += CSEG_PF) {
      float sd[CSEG_PF], hl[CSEG_PF];
#pragma unroll
      for (int q = 0; q < CSEG_PF; ++q) {
        sd[q] = sdt[(c + q) * cs];
        hl[q] = hloc[(c + q) * hs];
      }
#pragma unroll
      for (int q = 0; q < CSEG_PF; ++q) {
        const float m = exp2f(A2 * sd[q]);
        H = m * H + hl[q];
        P *= m;
        S += sd[q];
      }
    }
    for (; c < c1; ++c) {
      const float sd = sdt[c * cs];
      const float m = exp2f(A2 * sd);
      H = m * H + hloc[c * hs];
      P *= m;
      S += sd;
    }
  }
  sP[w][lane] = P;
  sH[w][lane] = H;
  sS[w][lane] = S;
  __syncthreads();
  float Hin = H0, tot = 0.f;
  for (int v = 0; v < w; ++v) Hin = sP[v][lane] * Hin + sH[v][lane];
  float Hend = Hin;
  for (int v = w; v < CSEG; ++v) Hend = sP[v][lane] * Hend + sH[v][lane];
  for (int v = 0; v < CSEG; ++v) tot += sS[v][lane];
  if (valid) {
    if (w == 0) hC[0] = H0;
    H = Hin;
    int64_t c = c0;
    for (; c + CSEG_PF <= c1; c += CSEG_PF) {
      float sd[CSEG_PF], hl[CSEG_PF];
#pragma unroll
      for (int q = 0; q < CSEG_PF; ++q) {
        sd[q] = sdt[(c + q) * cs];
        hl[q] = hloc[(c + q) * hs];
      }
#pragma unroll
      for (int q = 0; q < CSEG_PF; ++q) {
        H = exp2f(A2 * sd[q]) * H + hl[q];
        hC[(c + q + 1) * hs] = H;
      }
    }
    for (; c < c1; ++c) {
      H = exp2f(A2 * sdt[c * cs]) * H + hloc[c * hs];
      hC[(c + 1) * hs] = H;
    }
  }
  if (sum_out) *sum_out = tot;
  return Hend;
}

// Backward (reverse over chunks): with G_nC = G_end and aE_nC = aE_end,
//   x_c = aE_{c+1} G_{c+1};  X[c*hs] = x_c;  G_c = exp2(A2 sdt2[c*cs]) x_c + dloc[c*hs];
//   aE_c = exp2(A2 dt0[c*cs]).
// Returns G_0 and aE_0 (through aE_out).  All threads of the block must call it.
__device__ __forceinline__ float compose_bwd_segmented(bool valid, const float* __restrict__ sdt2,
                                                       const float* __restrict__ dt0, int64_t cs,
                                                       const float* __restrict__ dloc, int64_t hs,
                                                       float* __restrict__ X, float A2, float G_end, float aE_end,
                                                       int64_t nC, float* aE_out) {
  __shared__ float sM[CSEG][32], sG[CSEG][32];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int64_t run = (nC + CSEG - 1) / CSEG;
  const int64_t c0 = w * run < nC ? w * run : nC;
  const int64_t c1 = c0 + run < nC ? c0 + run : nC;
  // aE entering the run from the right: the first dt of the chunk after it, or aE_end
  float aE_right = aE_end;
  if (valid && c1 < nC) aE_right = exp2f(A2 * dt0[c1 * cs]);
  float M = 1.f, G = 0.f;
  if (valid) {
    float aE = aE_right;
    int64_t c = c1 - 1;
    for (; c - CSEG_PF + 1 >= c0; c -= CSEG_PF) {
      float s2[CSEG_PF], d0[CSEG_PF], dl[CSEG_PF];
#pragma unroll
      for (int q = 0; q < CSEG_PF; ++q) {
        s2[q] = sdt2[(c - q) * cs];
        d0[q] = dt0[(c - q) * cs];
        dl[q] = dloc[(c - q) * hs];
      }
#pragma unroll
      for (int q = 0; q < CSEG_PF; ++q) {
        const float m = exp2f(A2 * s2[q]) * aE;
        G = m * G + dl[q];
        M *= m;
        aE = exp2f(A2 * d0[q]);
      }
    }
    for (; c >= c0; --c) {
      const float m = exp2f(A2 * sdt2[c * cs]) * aE;
      G = m * G + dloc[c * hs];
      M *= m;
      aE = exp2f(A2 * dt0[c * cs]);
    }
  }
  sM[w][lane] = M;
  sG[w][lane] = G;
  __syncthreads();
  float Gin = G_end;
  for (int v = CSEG - 1; v > w; --v) Gin = sM[v][lane] * Gin + sG[v][lane];
  float aE = aE_right;
  G = Gin;
  if (valid) {
    int64_t c = c1 - 1;
    for (; c - CSEG_PF + 1 >= c0; c -= CSEG_PF) {
      float s2[CSEG_PF], d0[CSEG_PF], dl[CSEG_PF];
#pragma unroll
      for (int q = 0; q < CSEG_PF; ++q) {
        s2[q] = sdt2[(c - q) * cs];
        d0[q] = dt0[(c - q) * cs];
        dl[q] = dloc[(c - q) * hs];
      }
#pragma unroll
      for (int q = 0; q < CSEG_PF; ++q) {
        const float x = aE * G;
        X[(c - q) * hs] = x;
        G = exp2f(A2 * s2[q]) * x + dl[q];
        aE = exp2f(d0[q] * A2);
      }
    }
    for (; c >= c0; --c) {
      const float x = aE * G;
      X[c * hs] = x;
      G = exp2f(A2 * sdt2[c * cs]) * x + dloc[c * hs];
      aE = exp2f(dt0[c * cs] * A2);
    }
  }
  if (aE_out) *aE_out = aE;
  return G;
}

}  // namespace pgf
