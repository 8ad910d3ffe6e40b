// tcgen05 / TMEM dense product for bf16 operands on sm_100a.
//
// Persistent, warp-specialised kernel, one CTA per SM, 320 threads:
//   * warp 0 (one lane): TMA producer.  Operand tiles arrive 128B-swizzled through a TC_STAGES-deep
//     mbarrier ring.  A K-major operand is one box {64 k, 128 rows}; an MN-major operand (stored
//     transposed) is two boxes {64 rows, 64 k} side by side, so no operand is ever transposed in
//     memory.
//   * warp 1 (one lane): issues tcgen05.mma (kind::f16, bf16 x bf16 -> f32, M=128, N=128, K=16)
//     into one of two TMEM accumulators (2 x 128 columns), frees smem stages with tcgen05.commit
//     on their "empty" barriers and hands finished accumulators to the epilogue.
//   * warps 2..9: epilogue.  Warp w reads TMEM lanes 32*(w%4).. (tile rows) of one 64-column half
//     with tcgen05.ld while the MMA warp already fills the other accumulator.  Modes:
//       GENERIC  - row-per-thread epilogue in registers (bias, GELU / GELU', addend, accumulate),
//                  rows staged 128B-swizzled in shared memory and written by TMA bulk-tensor
//                  stores (D and the pre-activation aux_out); outputs whose pitch or base does not
//                  suit TMA take a 32x32 shared-memory transpose and coalesced row stores instead;
//       CE_FWD   - online log-sum-exp of each row over the CTA's vocabulary range plus the target
//                  logit; the logits never leave TMEM;
//       CE_BWD   - g = (softmax - onehot) * scale from the recomputed logits and the saved lse,
//                  stored as bf16 through the transpose;
//       DUAL     - two products per output tile into two accumulators (z = A1 B1^T and
//                  d = A2 B2^T, 128 columns each, four TMEM accumulators in all), stored as
//                  act(z + bias) and d * act'(z + bias): the FFN backward's recomputed hidden
//                  activation and its pre-activation gradient, z never leaving TMEM.
// Work unit = (128-row block, group of `ng` consecutive 128-column tiles); CTAs stride over units.
// Every mbarrier wait is bounded by a clock budget; on expiry the kernel records a fault in
// g_tc_fault and stops issuing work.
#include "f32x2.cuh"
#include "gemm.cuh"
#include "tc_common.cuh"

#include <cuda.h>
#include <math.h>

#include <mutex>
#include <string.h>

namespace pgf {

constexpr int TC_BM = 128, TC_BN = 128, TC_BK = 64;  // TC_BN: the CE modes' (and narrow outputs') tile width
constexpr int TC_THREADS = 320;  // TMA warp, MMA warp, 8 epilogue warps
constexpr int TILE_A_BYTES = TC_BM * TC_BK * 2;

// Tile width BN = 128 or 256 output columns.  At N = 256 a K = 16 MMA reads 12 KB of operands for
// 1 MFLOP (8 KB for 0.5 MFLOP at N = 128), which keeps the tensor pipe ahead of the operand reads;
// the price is all 512 TMEM columns (two accumulators).  Four operand stages either way: at N = 256
// they leave room for one 4 KB epilogue staging buffer per warp instead of two (measured: the fourth
// stage, which hides more of the operand fetch latency, is worth more than the second buffer).
// Every epilogue warp has at least 4 KB (the transpose path uses the first 32 x 33 floats).
// PAIR: a cluster of two CTAs computes a 256-row tile with tcgen05.mma.cta_group::2; each CTA holds
// its 128 rows of A and half of the tile's B columns, so a stage is 32 KB and six fit.
template <int BN, bool PAIR = false>
struct TcCfg {
  static constexpr int TILE_B = (PAIR ? BN / 2 : BN) * TC_BK * 2;
  static constexpr int STAGES = PAIR ? 6 : 4;
  static constexpr int STAGE = TILE_A_BYTES + TILE_B;
  static constexpr int NBUF = BN == 256 ? 1 : 2;      // epilogue staging buffers per warp
  static constexpr int EPI_WARP = NBUF * 4096;
  static constexpr size_t SMEM = size_t(STAGES) * STAGE + 8 * EPI_WARP + 256 /* barriers */ + 1024 /* align */;
  static_assert(SMEM <= 232448, "shared memory per CTA");
};

enum { TC_GENERIC = 0, TC_CE_FWD = 1, TC_CE_BWD = 2 };

// Epilogue families, one kernel instantiation each (a kernel carries only its own epilogue code:
// the single all-modes kernel spent a measurable share of its issue slots on instruction-cache misses):
//   PLAIN: generic, no activation (bias / addend / accumulate);  ACT: GELU or ReLU (+ pre-activation);
//   DACT: GELU' or ReLU' with the saved pre-activation;  CE_FWD / CE_BWD: the cross-entropy modes.
enum { EK_PLAIN = 0, EK_ACT = 1, EK_DACT = 2, EK_CE_FWD = 3, EK_CE_BWD = 4, EK_DUAL = 5 };

// The bf16-output GELU and GELU' (tanh form) on a pair of columns with packed float32 instructions:
// GELU(x) = hx + hx tanh(u) with hx = x/2, u = C x (1 + A x^2);
// GELU'(x) = (1 + tanh(u))/2 + hx (1 - tanh(u)^2) (C + 3AC x^2).
__device__ __forceinline__ float2 gelu2_bf(float2 x) {
  const float2 q = fma2(mul2(x, x), f2(PGF_GELU_A), f2(1.0f));
  const float2 u = mul2(mul2(x, f2(PGF_GELU_C)), q);
  const float2 t = f2(tanh_approx(u.x), tanh_approx(u.y));
  const float2 hx = mul2(x, f2(0.5f));
  return fma2(hx, t, hx);
}
__device__ __forceinline__ float2 gelu_prime2_bf(float2 x) {
  const float2 x2 = mul2(x, x);
  const float2 u = mul2(mul2(x, f2(PGF_GELU_C)), fma2(x2, f2(PGF_GELU_A), f2(1.0f)));
  const float2 t = f2(tanh_approx(u.x), tanh_approx(u.y));
  const float2 w = fma2(x2, f2(3.0f * PGF_GELU_A * PGF_GELU_C), f2(PGF_GELU_C));
  const float2 hs = mul2(mul2(x, f2(0.5f)), fma2(t, f2(-t.x, -t.y), f2(1.0f)));
  return fma2(hs, w, fma2(t, f2(0.5f), f2(0.5f)));
}
// GELU(x) and GELU'(x) from one tanh per element.
__device__ __forceinline__ void gelu_and_prime2(float2 x, float2& g, float2& gp) {
  const float2 x2 = mul2(x, x);
  const float2 u = mul2(mul2(x, f2(PGF_GELU_C)), fma2(x2, f2(PGF_GELU_A), f2(1.0f)));
  const float2 t = f2(tanh_approx(u.x), tanh_approx(u.y));
  const float2 hx = mul2(x, f2(0.5f));
  g = fma2(hx, t, hx);
  const float2 w = fma2(x2, f2(3.0f * PGF_GELU_A * PGF_GELU_C), f2(PGF_GELU_C));
  const float2 hs = mul2(hx, fma2(t, f2(-t.x, -t.y), f2(1.0f)));
  gp = fma2(hs, w, fma2(t, f2(0.5f), f2(0.5f)));
}


struct TcParams {
  int64_t M, N, K;
  int a_mn, b_mn;
  int64_t K2;          // DUAL: depth of the second product (operands tmA2 / tmB2)
  int a2_mn, b2_mn;
  int mode;
  int ng;              // 128-column tiles per work unit
  int n_groups;        // work units per row block
  int64_t tiles;       // work units per K slice (row blocks x column groups)
  int64_t units;       // tiles x ksplit
  int ksplit;          // K slices (1 = whole K per unit)
  int kper;            // 64-deep k-blocks per slice
  int64_t split_stride;  // floats between the partial products of consecutive slices
  int fast;            // 1: row-per-thread epilogue with TMA stores (maps tmD / tmZ valid)
  int z_bf16;          // aux_out element type on the fast path
  void* D;
  int d_bf16;
  int64_t ldd;
  pgf_epilogue epi;
  // cross-entropy modes (columns are vocabulary ids)
  const int64_t* targets;  // (M,)
  const float* lse;        // (M,)  CE_BWD
  float scale;             // CE_BWD
  float* part_m;           // (M, n_groups)  CE_FWD
  float* part_s;           // (M, n_groups)  CE_FWD
  float* tgt_logit;        // (M,)  CE_FWD
};

template <int BN, int EK, bool PAIR = false>
__global__ void __launch_bounds__(TC_THREADS, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
               const __grid_constant__ CUtensorMap tmD, const __grid_constant__ CUtensorMap tmZ,
               const __grid_constant__ CUtensorMap tmA2, const __grid_constant__ CUtensorMap tmB2, const TcParams p) {
  using C = TcCfg<BN, PAIR>;
  static_assert(EK != EK_DUAL || BN == 128, "the dual product runs 128-column tiles");
  static_assert(!PAIR || (BN == 256 && (EK == EK_PLAIN || EK == EK_ACT || EK == EK_DACT)),
                "CTA pairs run 256-column generic products");
  // PAIR: rank 0 of the pair (the leader) holds the stage barriers and issues the MMAs
  const uint32_t crank = PAIR ? cluster_rank() : 0u;
  const int64_t u_first = PAIR ? int64_t(blockIdx.x >> 1) : int64_t(blockIdx.x);
  const int64_t u_step = PAIR ? int64_t(gridDim.x >> 1) : int64_t(gridDim.x);
  constexpr int BMU = PAIR ? 2 * TC_BM : TC_BM;        // rows of one work unit
  const int64_t row_off = int64_t(crank) * TC_BM;      // this CTA's rows within the unit
  constexpr int NPROD = EK == EK_DUAL ? 2 : 1;        // products per output tile
  constexpr uint32_t ABUF = uint32_t(NPROD * BN);     // TMEM columns of one accumulator set
  constexpr uint32_t NCOL = 2 * ABUF;                 // two sets: the MMA fills one while the epilogue drains the other
  constexpr int MODE = EK == EK_CE_FWD ? TC_CE_FWD : (EK == EK_CE_BWD ? TC_CE_BWD : TC_GENERIC);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* tiles = smem;
  float* epi_buf = reinterpret_cast<float*>(tiles + C::STAGES * C::STAGE);
  uint64_t* full = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(epi_buf) + 8 * C::EPI_WARP);
  uint64_t* empty = full + C::STAGES;
  uint64_t* tfull = empty + C::STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nk = int((p.K + TC_BK - 1) / TC_BK);
  const int nk2 = EK == EK_DUAL ? int((p.K2 + TC_BK - 1) / TC_BK) : 0;
  const int n_tiles = int((p.N + BN - 1) / BN);

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], PAIR ? 16 : 8);  // the epilogue warps of both CTAs arrive on the leader's
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmB)) : "memory");
    if (EK == EK_DUAL) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA2)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmB2)) : "memory");
    }
  }
  if (PAIR) cluster_sync();  // both CTAs' barriers are initialised before either signals the other's
  if (warp == 0) {
    if (PAIR) {
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;"
                   ::"r"(smem_u32(tslot)), "r"(NCOL));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    } else {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                   ::"r"(smem_u32(tslot)), "r"(NCOL));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tslot;

  if (warp == 0) {
    // ---- TMA producer: the whole warp runs the loop and waits, one elected lane issues the copies
    const bool leader = elect_one();
    uint32_t it = 0;
    bool ok = true;
    for (int64_t u = u_first; u < p.units && ok; u += u_step) {
      const int ks = int(u / p.tiles), ut = int(u % p.tiles);
      const int mb = ut / p.n_groups, ng = ut % p.n_groups;
      const int nt0 = ng * p.ng, nt1 = min(nt0 + p.ng, n_tiles);
      const int m0 = int(int64_t(mb) * BMU + row_off);
      const int kb0 = ks * p.kper, kb1 = min(nk, kb0 + p.kper);
      for (int nt = nt0; nt < nt1 && ok; ++nt) {
        const int n0 = nt * BN;
        for (int pr = 0; pr < NPROD && ok; ++pr) {
          const CUtensorMap* mA = pr ? &tmA2 : &tmA;
          const CUtensorMap* mB = pr ? &tmB2 : &tmB;
          const int amn = pr ? p.a2_mn : p.a_mn, bmn = pr ? p.b2_mn : p.b_mn;
          const int kbs = pr ? 0 : kb0, kbe = pr ? nk2 : kb1;
          for (int kb = kbs; kb < kbe; ++kb, ++it) {
            const int s = int(it % C::STAGES), r = int(it / C::STAGES);
            if (r > 0 && !mbar_wait_warp(&empty[s], uint32_t((r - 1) & 1))) { ok = false; break; }
            if (PAIR) {
              // both CTAs' copies complete on the leader's barrier; the leader expects both
              if (leader) {
                if (crank == 0) mbar_expect_tx(&full[s], 2 * C::STAGE);
                const uint32_t fb = cluster_addr(&full[s], 0);
                uint8_t* sa = tiles + s * C::STAGE;
                uint8_t* sb = sa + TILE_A_BYTES;
                const int k0 = kb * TC_BK;
                const int nb0 = n0 + int(crank) * (BN / 2);
                if (!amn) {
                  tma_load_2d_pair(sa, mA, fb, k0, m0);
                } else {
                  tma_load_2d_pair(sa, mA, fb, m0, k0);
                  tma_load_2d_pair(sa + TILE_A_BYTES / 2, mA, fb, m0 + 64, k0);
                }
                if (!bmn) {
                  tma_load_2d_pair(sb, mB, fb, k0, nb0);
                } else {
#pragma unroll
                  for (int i = 0; i < BN / 128; ++i) tma_load_2d_pair(sb + i * 8192, mB, fb, nb0 + 64 * i, k0);
                }
              }
            } else if (leader) {
              mbar_expect_tx(&full[s], C::STAGE);
              uint8_t* sa = tiles + s * C::STAGE;
              uint8_t* sb = sa + TILE_A_BYTES;
              const int k0 = kb * TC_BK;
              if (!amn) {
                tma_load_2d(sa, mA, &full[s], k0, m0);
              } else {
                tma_load_2d(sa, mA, &full[s], m0, k0);
                tma_load_2d(sa + TILE_A_BYTES / 2, mA, &full[s], m0 + 64, k0);
              }
              if (!bmn) {
                tma_load_2d(sb, mB, &full[s], k0, n0);
              } else {
#pragma unroll
                for (int i = 0; i < BN / 64; ++i) tma_load_2d(sb + i * 8192, mB, &full[s], n0 + 64 * i, k0);
              }
            }
            __syncwarp();
          }
        }
      }
    }
  } else if (warp == 1 && (!PAIR || crank == 0)) {
    // ---- MMA issuer: the whole warp runs the loop and waits (descriptors stay warp-uniform), one
    //      elected lane issues every tcgen05.mma and tcgen05.commit (commits track that lane's MMAs).
    //      PAIR: the leader's warp issues the pair's MMAs (M = 256) and signals both CTAs' barriers.
    const bool leader = elect_one();
    const uint32_t idesc_base = (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(BN >> 3) << 17) |
                                (uint32_t(BMU >> 4) << 24);
    // commit: this CTA's barrier, and in a pair the peer's too
    auto commit = [&](uint64_t* bar) {
      if (PAIR) {
        umma_commit_pair(cluster_addr(bar, 0));
        umma_commit_pair(cluster_addr(bar, 1));
      } else {
        umma_commit(bar);
      }
    };
    uint32_t it = 0, tt = 0;
    bool ok = true;
    for (int64_t u = u_first; u < p.units && ok; u += u_step) {
      const int ks = int(u / p.tiles), ng = int(u % p.tiles) % p.n_groups;
      const int nt0 = ng * p.ng, nt1 = min(nt0 + p.ng, n_tiles);
      const int kb0 = ks * p.kper, kb1 = min(nk, kb0 + p.kper);
      for (int nt = nt0; nt < nt1 && ok; ++nt, ++tt) {
        const uint32_t buf = tt & 1, use = tt >> 1;
        if (use > 0 && !mbar_wait_warp(&tempty[buf], (use - 1) & 1)) { ok = false; break; }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        for (int pr = 0; pr < NPROD && ok; ++pr) {
          const uint32_t dcol = tmem + buf * ABUF + uint32_t(pr * BN);
          const int amn = pr ? p.a2_mn : p.a_mn, bmn = pr ? p.b2_mn : p.b_mn;
          const uint32_t idesc = idesc_base | (uint32_t(amn) << 15) | (uint32_t(bmn) << 16);
          const int kbs = pr ? 0 : kb0, kbe = pr ? nk2 : kb1;
          for (int kb = kbs; kb < kbe; ++kb, ++it) {
            const int s = int(it % C::STAGES), r = int(it / C::STAGES);
            if (!mbar_wait_warp(&full[s], uint32_t(r & 1))) { ok = false; break; }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t a_base = smem_u32(tiles + s * C::STAGE);
            const uint32_t b_base = a_base + TILE_A_BYTES;
#pragma unroll
            for (int kk = 0; kk < TC_BK / 16; ++kk) {
              // K-major: advance 16 elements (32 B) inside the 128B swizzle row;
              // MN-major: advance 16 k-rows (2 KB), two 8-row atoms apart by SBO = 1 KB.
              const uint64_t ad = amn ? sdesc(a_base + kk * 2048, TILE_A_BYTES / 2, 1024)
                                      : sdesc(a_base + kk * 32, 16, 1024);
              const uint64_t bd = bmn ? sdesc(b_base + kk * 2048, 8192, 1024)
                                      : sdesc(b_base + kk * 32, 16, 1024);
              if (leader) {
                if (PAIR) umma_bf16_pair(dcol, ad, bd, idesc, (kb != kbs) || (kk != 0));
                else umma_bf16(dcol, ad, bd, idesc, (kb != kbs) || (kk != 0));
              }
            }
            if (leader) commit(&empty[s]);
            __syncwarp();
          }
        }
        if (!ok) break;
        if (leader) commit(&tfull[buf]);
        __syncwarp();
      }
    }
  } else if (warp >= 2) {
    // ---- epilogue warps 2..9: TMEM lane quarter q = warp % 4 (rows 32q..32q+31), column half
    //      hf = (warp - 2) / 4 (columns 64hf..64hf+63 of the 128-column tile)
    const int q = warp & 3;
    const int hf = (warp - 2) >> 2;
    // the accumulator buffer is drained: tell the MMA warp (the leader's, in a pair)
    auto release_acc = [&](uint32_t b) {
      if (PAIR) mbar_arrive_cluster(cluster_addr(&tempty[b], 0));
      else mbar_arrive(&tempty[b]);
    };
    uint8_t* stg = reinterpret_cast<uint8_t*>(epi_buf) + (warp - 2) * C::EPI_WARP;
    float* tb = reinterpret_cast<float*>(stg);
    uint32_t sq = 0;  // staging buffers taken by this warp
    uint32_t tt = 0;
    bool ok = true;
    for (int64_t u = u_first; u < p.units && ok; u += u_step) {
      const int ks = int(u / p.tiles), ut = int(u % p.tiles);
      const int mb = ut / p.n_groups, ng = ut % p.n_groups;
      const int nt0 = ng * p.ng, nt1 = min(nt0 + p.ng, n_tiles);
      // a K slice stores its plain float32 partial product; the reduction applies the epilogue
      void* Dst = p.ksplit > 1 ? static_cast<void*>(static_cast<float*>(p.D) + ks * p.split_stride) : p.D;
      const int64_t row = (int64_t(mb) * BMU + row_off) + q * 32 + lane;  // this thread's row (CE modes)
      const bool row_ok = row < p.M;
      float run_m = -INFINITY, run_s = 0.f;
      int64_t tgt = -1;
      float row_lse = 0.f;
      if (MODE != TC_GENERIC && row_ok) {
        tgt = p.targets[row];
        if (MODE == TC_CE_BWD) row_lse = p.lse[row];
      }
      for (int nt = nt0; nt < nt1; ++nt, ++tt) {
        const uint32_t buf = tt & 1, use = tt >> 1;
        // DUAL: the tile's 64 bias values of this warp's columns, loaded while the MMA runs
        float bias_pre[64];
        if (EK == EK_DUAL) {
          const int64_t nh = int64_t(nt) * BN + hf * 64;
          const float* bias = p.epi.bias;
          if (bias && nh + 64 <= p.N && ((reinterpret_cast<uintptr_t>(bias + nh) & 15) == 0)) {
            const float4* bq = reinterpret_cast<const float4*>(bias + nh);
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const float4 b4 = __ldg(bq + j);
              bias_pre[4 * j] = b4.x; bias_pre[4 * j + 1] = b4.y; bias_pre[4 * j + 2] = b4.z; bias_pre[4 * j + 3] = b4.w;
            }
          } else {
#pragma unroll
            for (int j = 0; j < 64; ++j) bias_pre[j] = (bias && nh + j < p.N) ? __ldg(bias + nh + j) : 0.f;
          }
        }
        if (!mbar_wait_warp(&tfull[buf], use & 1)) { ok = false; break; }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const int64_t n0 = int64_t(nt) * BN;
        if (EK == EK_DUAL) {
          // ---- two accumulators per tile: z (columns 0..127 of the set) and d (128..255); this
          //      thread owns row `row` and the warp's 64 columns nh .. nh+63 of both
          const int64_t row0 = (int64_t(mb) * BMU + row_off) + q * 32;
          const bool box_live = row0 < p.M;
          const int64_t nh = n0 + hf * 64;
          const uint32_t tq = tmem + buf * ABUF + (uint32_t(q * 32) << 16) + uint32_t(hf * 64);
          uint32_t hpk[32], dpk[32];  // bf16 pairs of act(z) and d * act'(z)
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            uint32_t rz[32], rd[32];
            tmem_ld32_nowait(tq + uint32_t(c * 32), rz);
            tmem_ld32_nowait(tq + uint32_t(BN + c * 32), rd);
            tmem_wait_ld();
            if (c == 1) {
              asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
              __syncwarp();
              if (lane == 0) release_acc(buf);
            }
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const float2 z = add2(f2(__uint_as_float(rz[2 * j]), __uint_as_float(rz[2 * j + 1])),
                                    f2(bias_pre[c * 32 + 2 * j], bias_pre[c * 32 + 2 * j + 1]));
              const float2 d = f2(__uint_as_float(rd[2 * j]), __uint_as_float(rd[2 * j + 1]));
              float2 h, gz;
              if (p.epi.kind == PGF_EPI_GELU) {
                float2 gp;
                gelu_and_prime2(z, h, gp);
                gz = mul2(d, gp);
              } else {
                h = f2(fmaxf(z.x, 0.f), fmaxf(z.y, 0.f));
                gz = f2(z.x > 0.f ? d.x : 0.f, z.y > 0.f ? d.y : 0.f);
              }
              hpk[c * 16 + j] = pack_bf16(h.x, h.y);
              dpk[c * 16 + j] = pack_bf16(gz.x, gz.y);
            }
          }
          // boxes start inside the output (the TMA clips their far edges)
          if (box_live && nh < p.N) {
            uint8_t* b = stage_acquire<C::NBUF>(stg, sq, lane);
            stage_row(b, lane, hpk);
            stage_store(b, &tmD, nh, row0, 0, lane);
            b = stage_acquire<C::NBUF>(stg, sq, lane);
            stage_row(b, lane, dpk);
            stage_store(b, &tmZ, nh, row0, 0, lane);
          }
          continue;
        }
        if (EK != EK_CE_FWD && p.fast) {
          // ---- row-per-thread epilogue: this thread owns row `row` and the warp's BN/2 columns,
          //      taken 64 at a time (nh .. nh+63)
          const int64_t row0 = (int64_t(mb) * BMU + row_off) + q * 32;
          const bool box_live = row0 < p.M;  // rows of this quarter exist (TMA clips the rest)
#pragma unroll 1
          for (int g64 = 0; g64 < BN / 128; ++g64) {
          const int64_t nh = n0 + hf * (BN / 2) + g64 * 64;
          const uint32_t tcol = uint32_t(hf * (BN / 2) + g64 * 64);
          uint32_t dpk[32], zpk[32];          // bf16 pairs of D / aux_out for the 64 columns
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            uint32_t r[32];
            tmem_ld32(tmem + buf * ABUF + (uint32_t(q * 32) << 16) + tcol + uint32_t(c * 32), r);
            if (c == 1 && g64 == BN / 128 - 1) {
              // both chunks are in registers: hand the accumulator back to the MMA warp
              asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
              __syncwarp();
              if (lane == 0) release_acc(buf);
            }
            const int64_t nb = nh + c * 32;
            float v[32];
            if (MODE == TC_CE_BWD) {
              constexpr float L2E = 1.4426950408889634f;
              const float ll = row_lse * L2E;
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                float g = exp2f(fmaf(__uint_as_float(r[j]), L2E, -ll));
                if (tgt == nb + j) g -= 1.0f;
                v[j] = g * p.scale;
              }
            } else {
              const pgf_epilogue& e = p.epi;
              if (e.bias) {
                if (nb + 32 <= p.N && ((reinterpret_cast<uintptr_t>(e.bias + nb) & 15) == 0)) {
                  const float4* bq = reinterpret_cast<const float4*>(e.bias + nb);
#pragma unroll
                  for (int j = 0; j < 8; ++j) {
                    const float4 b4 = __ldg(bq + j);
                    const float2 lo = fma2(f2(e.alpha), f2(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1])),
                                           lo2(b4));
                    const float2 hi = fma2(f2(e.alpha), f2(__uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3])),
                                           hi2(b4));
                    v[4 * j] = lo.x; v[4 * j + 1] = lo.y; v[4 * j + 2] = hi.x; v[4 * j + 3] = hi.y;
                  }
                } else {
#pragma unroll
                  for (int j = 0; j < 32; ++j)
                    v[j] = fmaf(e.alpha, __uint_as_float(r[j]), nb + j < p.N ? __ldg(e.bias + nb + j) : 0.f);
                }
              } else {
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] = e.alpha * __uint_as_float(r[j]);
              }
              if (EK == EK_ACT) {
                if (e.aux_out) {
                  if (p.z_bf16) {
#pragma unroll
                    for (int j = 0; j < 16; ++j) zpk[c * 16 + j] = pack_bf16(v[2 * j], v[2 * j + 1]);
                  } else if (box_live && nb < p.N) {
                    uint32_t w[32];
#pragma unroll
                    for (int j = 0; j < 32; ++j) w[j] = __float_as_uint(v[j]);
                    uint8_t* b = stage_acquire<C::NBUF>(stg, sq, lane);
                    stage_row(b, lane, w);
                    stage_store(b, &tmZ, nb, row0, 0, lane);
                  }
                }
                if (e.kind == PGF_EPI_GELU) {
                  if (p.d_bf16) {
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                      const float2 g = gelu2_bf(f2(v[2 * j], v[2 * j + 1]));
                      v[2 * j] = g.x; v[2 * j + 1] = g.y;
                    }
                  } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j) v[j] = gelu_f(v[j]);
                  }
                } else {
#pragma unroll
                  for (int j = 0; j < 32; ++j) v[j] = fmaxf(v[j], 0.f);
                }
              } else if (EK == EK_DACT) {
                float a[32];
                load_seg(e.aux, e.aux_dtype, e.ld_aux, row, nb, p.M, p.N, a);
                if (e.kind == PGF_EPI_DRELU) {
#pragma unroll
                  for (int j = 0; j < 32; ++j) v[j] = a[j] > 0.f ? v[j] : 0.f;
                } else if (p.d_bf16) {
#pragma unroll
                  for (int j = 0; j < 16; ++j) {
                    const float2 g = mul2(f2(v[2 * j], v[2 * j + 1]), gelu_prime2_bf(f2(a[2 * j], a[2 * j + 1])));
                    v[2 * j] = g.x; v[2 * j + 1] = g.y;
                  }
                } else {
#pragma unroll
                  for (int j = 0; j < 32; ++j) v[j] *= gelu_prime_f(a[j]);
                }
              }
              if (e.addend) {
                float a[32];
                load_seg(e.addend, e.addend_dtype, e.ld_addend, row, nb, p.M, p.N, a);
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] += a[j];
              }
              if (e.accumulate) {
                float a[32];
                load_seg(p.D, 0, p.ldd, row, nb, p.M, p.N, a);
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] += a[j];
              }
            }
            if (p.d_bf16) {
#pragma unroll
              for (int j = 0; j < 16; ++j) dpk[c * 16 + j] = pack_bf16(v[2 * j], v[2 * j + 1]);
            } else if (box_live && nb < p.N) {
              uint32_t w[32];
#pragma unroll
              for (int j = 0; j < 32; ++j) w[j] = __float_as_uint(v[j]);
              uint8_t* b = stage_acquire<C::NBUF>(stg, sq, lane);
              stage_row(b, lane, w);
              stage_store(b, &tmD, nb, row0, ks, lane);
            }
          }
          // boxes start inside the output (the TMA clips their far edges)
          if (box_live && nh < p.N && p.d_bf16) {
            uint8_t* b = stage_acquire<C::NBUF>(stg, sq, lane);
            stage_row(b, lane, dpk);
            stage_store(b, &tmD, nh, row0, ks, lane);
          }
          if (box_live && nh < p.N && MODE == TC_GENERIC && p.epi.aux_out && p.z_bf16 &&
              (EK == EK_ACT)) {
            uint8_t* b = stage_acquire<C::NBUF>(stg, sq, lane);
            stage_row(b, lane, zpk);
            stage_store(b, &tmZ, nh, row0, 0, lane);
          }
          }  // g64
          continue;
        }
        // column-chunk path: the CE forward at either width, the transposed store only in 128-wide
        // tiles (the host sends 256-wide generic and CE-backward tiles to the row-per-thread path)
#pragma unroll 1
        for (int c = hf * (BN / 64); c < (BN == 128 || EK == EK_CE_FWD ? (hf + 1) * (BN / 64) : 0); ++c) {
          uint32_t r[32];
          tmem_ld32(tmem + buf * ABUF + (uint32_t(q * 32) << 16) + uint32_t(c * 32), r);
          const int64_t nc = n0 + c * 32;
          if (MODE == TC_CE_FWD) {
            // online log-sum-exp in base 2: exp(v - m) = exp2(v log2e - m log2e)
            constexpr float L2E = 1.4426950408889634f;
            if (nc + 32 > p.N) {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (nc + j >= p.N) r[j] = __float_as_uint(-INFINITY);
            }
            float mx = __uint_as_float(r[0]);
#pragma unroll
            for (int j = 1; j < 32; ++j) mx = fmaxf(mx, __uint_as_float(r[j]));
            if (mx > -INFINITY) {
              const float m1 = fmaxf(run_m, mx);
              const float ml = m1 * L2E;
              float s0 = 0.f, s1 = 0.f;
#pragma unroll
              for (int j = 0; j < 32; j += 2) {
                s0 += ex2f(fmaf(__uint_as_float(r[j]), L2E, -ml));
                s1 += ex2f(fmaf(__uint_as_float(r[j + 1]), L2E, -ml));
              }
              run_s = run_s * ex2f((run_m - m1) * L2E) + (s0 + s1);
              run_m = m1;
            }
            if (tgt >= nc && tgt < nc + 32 && tgt < p.N) {  // a target >= N stays unwritten (NaN loss)
              float v = 0.f;
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (tgt == nc + j) v = __uint_as_float(r[j]);
              if (row_ok) p.tgt_logit[row] = v;
            }
            continue;
          }
          if (MODE == TC_CE_BWD) {
            constexpr float L2E = 1.4426950408889634f;
            const float ll = row_lse * L2E;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              float g = exp2f(fmaf(__uint_as_float(r[j]), L2E, -ll));
              if (tgt == nc + j) g -= 1.0f;
              r[j] = __float_as_uint(g * p.scale);
            }
          }
          // transpose the 32x32 block through shared memory, then store row segments
#pragma unroll
          for (int j = 0; j < 32; ++j) tb[lane * 33 + j] = __uint_as_float(r[j]);
          __syncwarp();
          const int64_t n = nc + lane;
          const bool n_ok = n < p.N;
          const int64_t mbase = (int64_t(mb) * BMU + row_off) + q * 32;
          if (MODE == TC_GENERIC) {
            const float bias_n = (p.epi.bias && n_ok) ? p.epi.bias[n] : 0.f;
#pragma unroll 8
            for (int rr = 0; rr < 32; ++rr) {
              const int64_t m = mbase + rr;
              if (m < p.M && n_ok) epi_store_biased(p.epi, Dst, p.d_bf16, p.ldd, m, n, tb[rr * 33 + lane], bias_n);
            }
          } else {
            __nv_bfloat16* G = reinterpret_cast<__nv_bfloat16*>(p.D);
#pragma unroll 8
            for (int rr = 0; rr < 32; ++rr) {
              const int64_t m = mbase + rr;
              if (m < p.M && n_ok) G[m * p.ldd + n] = __float2bfloat16_rn(tb[rr * 33 + lane]);
            }
          }
          __syncwarp();
        }
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncwarp();
        if (lane == 0) release_acc(buf);
      }
      if (MODE == TC_CE_FWD && row_ok && ok) {
        p.part_m[row * (2 * p.n_groups) + 2 * ng + hf] = run_m;
        p.part_s[row * (2 * p.n_groups) + 2 * ng + hf] = run_s;
      }
    }
    // all TMA stores of this warp complete before the CTA leaves
    if (p.fast && lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  if (PAIR) {
    // neither CTA leaves (or frees its tensor memory) while the other may still signal its barriers
    // or the pair's MMAs may still write it
    cluster_sync();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(NCOL));
  } else {
    __syncthreads();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(NCOL));
  }
}

// ---------------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------------
static bool fast_epilogue_disabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("PGF_TC_TRANSPOSE_EPILOGUE");
    v = (e && e[0] == '1') ? 1 : 0;
  }
  return v == 1;
}

static bool tc_disabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("PGF_DISABLE_TC");
    v = (e && e[0] == '1') ? 1 : 0;
  }
  return v == 1;
}

int sm_count() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
  }
  return n;
}

bool tc_usable(const Gemm& g) {
  if (tc_disabled() || !g.a_bf16 || !g.b_bf16 || g.K == 0) return false;
  if (!aligned(g.A, 16) || !aligned(g.B, 16) || (g.lda * 2) % 16 || (g.ldb * 2) % 16) return false;
  if (g.M > (int64_t(1) << 31) || g.N > (int64_t(1) << 31) || g.K > (int64_t(1) << 31)) return false;
  return true;
}

// Launch over the whole (M x N) output with the given mode; `ng` = column tiles per work unit.
// Tile width of a launch: 256 columns for generic products whose width pads no further at 256
// than at 128 (N mod 256 = 0 or > 128; PGF_TC_BN128=1 keeps 128), else 128; the cross-entropy
// modes always use 128.
static int tile_bn(int mode, int64_t N) {
  static int force128 = -1;
  if (force128 < 0) {
    const char* e = getenv("PGF_TC_BN128");
    force128 = (e && e[0] == '1') ? 1 : 0;
  }
  if (force128 || N <= 128) return 128;
  if (mode == TC_CE_FWD) return 256;  // no stored output: the wider tile only saves operand reads
  const bool wide = ((N + 255) / 256) * 256 <= ((N + 127) / 128) * 128;
  return (mode == TC_GENERIC && wide) ? 256 : 128;
}

static int ek_of(const TcParams& p) {
  if (p.mode == TC_CE_FWD) return EK_CE_FWD;
  if (p.mode == TC_CE_BWD) return EK_CE_BWD;
  switch (p.epi.kind) {
    case PGF_EPI_GELU: case PGF_EPI_RELU: return EK_ACT;
    case PGF_EPI_DGELU: case PGF_EPI_DRELU: return EK_DACT;
    default: return EK_PLAIN;
  }
}

// ma2 / mb2: the second product's operands (DUAL; other modes pass copies of ma / mb, unused).
template <int BN, int EK>
static int launch_tc_kernel(unsigned grid, cudaStream_t s, const CUtensorMap& ma, const CUtensorMap& mb,
                            const CUtensorMap& md, const CUtensorMap& mz, const TcParams& p,
                            const CUtensorMap* ma2 = nullptr, const CUtensorMap* mb2 = nullptr) {
  using C = TcCfg<BN>;
  static int smem_limit = 0;
  PGF_CUDA(ensure_dynamic_smem(gemm_tc_kernel<BN, EK>, C::SMEM, smem_limit));
  gemm_tc_kernel<BN, EK><<<grid, TC_THREADS, C::SMEM, s>>>(ma, mb, md, mz, ma2 ? *ma2 : ma, mb2 ? *mb2 : mb, p);
  return PGF_OK;
}

static bool pair_disabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("PGF_TC_NO_PAIR");
    v = (e && e[0] == '1') ? 1 : 0;
  }
  return v == 1;
}

// A 256-column generic product on CTA pairs: `pairs` clusters of two CTAs.
template <int EK>
static int launch_tc_pair_kernel(unsigned pairs, cudaStream_t s, const CUtensorMap& ma, const CUtensorMap& mb,
                                 const CUtensorMap& md, const CUtensorMap& mz, const TcParams& p) {
  using C = TcCfg<256, true>;
  static int smem_limit = 0;
  PGF_CUDA(ensure_dynamic_smem(gemm_tc_kernel<256, EK, true>, C::SMEM, smem_limit));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs);
  cfg.blockDim = dim3(TC_THREADS);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  PGF_CUDA(cudaLaunchKernelEx(&cfg, gemm_tc_kernel<256, EK, true>, ma, mb, md, mz, ma, mb, p));
  return PGF_OK;
}

template <int BN>
static int launch_tc_bn(const Gemm& g, TcParams& p, cudaStream_t s, int prof_id) {
  using C = TcCfg<BN>;
  (void)sizeof(C);
  CUtensorMap ma, mb;
  const bool oka = g.a_trans ? make_map(&ma, g.A, g.M, g.K, g.lda, 64, 64)
                             : make_map(&ma, g.A, g.K, g.M, g.lda, 64, TC_BM);
  const bool okb = g.b_trans ? make_map(&mb, g.B, g.N, g.K, g.ldb, 64, 64)
                             : make_map(&mb, g.B, g.K, g.N, g.ldb, 64, BN);
  if (!oka || !okb) return PGF_ERR_UNSUPPORTED;
  p.M = g.M; p.N = g.N; p.K = g.K;
  p.a_mn = g.a_trans; p.b_mn = g.b_trans;
  const int64_t n_tiles = (g.N + BN - 1) / BN;
  const int64_t m_blocks = (g.M + TC_BM - 1) / TC_BM;
  const int nk = int((g.K + TC_BK - 1) / TC_BK);
  p.n_groups = int((n_tiles + p.ng - 1) / p.ng);
  p.tiles = m_blocks * p.n_groups;
  if (p.ksplit < 1) {
    p.ksplit = 1;
    p.kper = nk;
  }
  p.units = p.tiles * p.ksplit;
  // output maps of the row-per-thread epilogue (GENERIC / CE_BWD)
  CUtensorMap md, mz;
  memset(&md, 0, sizeof md);
  memset(&mz, 0, sizeof mz);
  p.fast = 0;
  if ((p.mode == TC_GENERIC || p.mode == TC_CE_BWD) && !fast_epilogue_disabled()) {
    const int64_t es = p.d_bf16 ? 2 : 4;
    bool ok = aligned(p.D, 16) && (p.ldd * es) % 16 == 0 && (p.ksplit == 1 || (p.split_stride * es) % 16 == 0) &&
              make_out_map(&md, p.D, p.d_bf16, g.N, g.M, p.ldd, p.ksplit, p.split_stride);
    const bool want_z = p.mode == TC_GENERIC && p.epi.aux_out &&
                        (p.epi.kind == PGF_EPI_GELU || p.epi.kind == PGF_EPI_RELU);
    if (ok && want_z) {
      const int64_t ez = p.epi.aux_out_dtype ? 2 : 4;
      p.z_bf16 = p.epi.aux_out_dtype ? 1 : 0;
      ok = aligned(p.epi.aux_out, 16) && (p.epi.ld_aux_out * ez) % 16 == 0 &&
           make_out_map(&mz, p.epi.aux_out, p.z_bf16, g.N, g.M, p.epi.ld_aux_out, 1, 0);
    }
    p.fast = ok ? 1 : 0;
  }
  // 256-wide tiles: generic products through the TMA-store epilogue, and the CE forward (no stored
  // output); the transpose epilogue is only used at 128
  if (BN == 256 && ((p.mode == TC_GENERIC && !p.fast) || p.mode == TC_CE_BWD)) return PGF_ERR_UNSUPPORTED;
  const int ek = ek_of(p);
  // CTA pairs: 256-column generic products of at least two 128-row blocks and a depth of at least
  // 512 per unit (at shallower depths the two CTAs' epilogues, which must both drain an accumulator
  // before it is reused, bound the product and the pair was measured slower: FFN up at K = 256
  // 74 -> 84 us; at K = 1024 133 -> 119 us; the FFN 1024 -> 4096 weight gradients, depth 16384,
  // 121 -> 102 us)
  if (BN == 256 && p.mode == TC_GENERIC && p.fast && m_blocks >= 2 && !pair_disabled() &&
      int64_t(p.kper) * TC_BK >= 512 &&
      (ek == EK_PLAIN || ek == EK_ACT || ek == EK_DACT)) {
    CUtensorMap mbp;  // a K-major B operand is loaded in halves of BN / 2 rows
    const bool okp = g.b_trans ? true : make_map(&mbp, g.B, g.K, g.N, g.ldb, 64, BN / 2);
    if (okp) {
      if (g.b_trans) mbp = mb;
      TcParams q = p;
      q.tiles = ((g.M + 2 * TC_BM - 1) / (2 * TC_BM)) * q.n_groups;
      q.units = q.tiles * q.ksplit;
      const int64_t max_pairs = sm_count() / 2;
      const unsigned pairs = unsigned(q.units < max_pairs ? q.units : max_pairs);
      prof_begin(prof_id, s);
      int rc = PGF_OK;
      if (ek == EK_PLAIN) rc = launch_tc_pair_kernel<EK_PLAIN>(pairs, s, ma, mbp, md, mz, q);
      else if (ek == EK_ACT) rc = launch_tc_pair_kernel<EK_ACT>(pairs, s, ma, mbp, md, mz, q);
      else rc = launch_tc_pair_kernel<EK_DACT>(pairs, s, ma, mbp, md, mz, q);
      PGF_TRY(rc);
      prof_end(prof_id, s, 2.0 * double(g.M) * double(g.N) * double(g.K));
      PGF_LAUNCH_CHECK();
      return PGF_OK;
    }
  }
  const unsigned grid = unsigned(p.units < sm_count() ? p.units : sm_count());
  prof_begin(prof_id, s);
  int rc = PGF_OK;
  switch (ek) {
    case EK_PLAIN: rc = launch_tc_kernel<BN, EK_PLAIN>(grid, s, ma, mb, md, mz, p); break;
    case EK_ACT: rc = launch_tc_kernel<BN, EK_ACT>(grid, s, ma, mb, md, mz, p); break;
    case EK_DACT: rc = launch_tc_kernel<BN, EK_DACT>(grid, s, ma, mb, md, mz, p); break;
    case EK_CE_FWD: rc = launch_tc_kernel<BN, EK_CE_FWD>(grid, s, ma, mb, md, mz, p); break;
    default: rc = launch_tc_kernel<BN, EK_CE_BWD>(grid, s, ma, mb, md, mz, p); break;
  }
  PGF_TRY(rc);
  prof_end(prof_id, s, 2.0 * double(g.M) * double(g.N) * double(g.K));
  PGF_LAUNCH_CHECK();
  return PGF_OK;
}

static int launch_tc(const Gemm& g, TcParams& p, cudaStream_t s, int prof_id) {
  if (tile_bn(p.mode, g.N) == 256) {
    TcParams q = p;
    const int rc = launch_tc_bn<256>(g, q, s, prof_id);
    if (rc != PGF_ERR_UNSUPPORTED) return rc;
    clear_error();
  }
  return launch_tc_bn<128>(g, p, s, prof_id);
}

int run_gemm_tc(const Gemm& g, cudaStream_t s) {
  if (!tc_usable(g)) return PGF_ERR_UNSUPPORTED;
  if (g.M == 0 || g.N == 0) return PGF_OK;
  TcParams p = {};
  p.mode = TC_GENERIC;
  p.ng = 1;
  p.D = g.D; p.d_bf16 = g.d_bf16; p.ldd = g.ldd;
  p.epi = g.epi;
  return launch_tc(g, p, s, PROF_GEMM_TC);
}

int run_gemm_tc_dual(const DualGemm& g, cudaStream_t s) {
  if (g.M == 0 || g.N == 0) return PGF_OK;
  if (g.kind != PGF_EPI_GELU && g.kind != PGF_EPI_RELU) return PGF_ERR_UNSUPPORTED;
  // both products must suit the engine on their own (bf16 operands, 16-byte aligned rows)
  const Gemm p1 = gemm_make(g.M, g.N, g.K1, g.A1, 1, g.lda1, 0, g.B1, 1, g.ldb1, g.b1_trans, g.H, 1, g.ldh);
  const Gemm p2 = gemm_make(g.M, g.N, g.K2, g.A2, 1, g.lda2, 0, g.B2, 1, g.ldb2, g.b2_trans, g.DZ, 1, g.lddz);
  if (!tc_usable(p1) || !tc_usable(p2) || fast_epilogue_disabled()) return PGF_ERR_UNSUPPORTED;
  if (!aligned(g.H, 16) || !aligned(g.DZ, 16) || (g.ldh * 2) % 16 || (g.lddz * 2) % 16) return PGF_ERR_UNSUPPORTED;
  CUtensorMap ma, mb, ma2, mb2, md, mz;
  memset(&md, 0, sizeof md);
  memset(&mz, 0, sizeof mz);
  const bool ok = make_map(&ma, g.A1, g.K1, g.M, g.lda1, 64, TC_BM) &&
                  (g.b1_trans ? make_map(&mb, g.B1, g.N, g.K1, g.ldb1, 64, 64)
                              : make_map(&mb, g.B1, g.K1, g.N, g.ldb1, 64, TC_BN)) &&
                  make_map(&ma2, g.A2, g.K2, g.M, g.lda2, 64, TC_BM) &&
                  (g.b2_trans ? make_map(&mb2, g.B2, g.N, g.K2, g.ldb2, 64, 64)
                              : make_map(&mb2, g.B2, g.K2, g.N, g.ldb2, 64, TC_BN)) &&
                  make_out_map(&md, g.H, 1, g.N, g.M, g.ldh, 1, 0) &&
                  make_out_map(&mz, g.DZ, 1, g.N, g.M, g.lddz, 1, 0);
  if (!ok) return PGF_ERR_UNSUPPORTED;
  TcParams p = {};
  p.mode = TC_GENERIC;
  p.M = g.M; p.N = g.N; p.K = g.K1; p.K2 = g.K2;
  p.a_mn = 0; p.b_mn = g.b1_trans;
  p.a2_mn = 0; p.b2_mn = g.b2_trans;
  p.ng = 1;
  const int64_t n_tiles = (g.N + TC_BN - 1) / TC_BN;
  p.n_groups = int(n_tiles);
  p.tiles = ((g.M + TC_BM - 1) / TC_BM) * n_tiles;
  p.ksplit = 1;
  p.kper = int((g.K1 + TC_BK - 1) / TC_BK);
  p.units = p.tiles;
  p.fast = 1;
  p.z_bf16 = 1;
  p.D = g.H; p.d_bf16 = 1; p.ldd = g.ldh;
  p.epi = epi_default();
  p.epi.kind = g.kind;
  p.epi.bias = g.bias;
  const unsigned grid = unsigned(p.units < sm_count() ? p.units : sm_count());
  prof_begin(PROF_GEMM_TC, s);
  PGF_TRY((launch_tc_kernel<TC_BN, EK_DUAL>(grid, s, ma, mb, md, mz, p, &ma2, &mb2)));
  prof_end(PROF_GEMM_TC, s, 2.0 * double(g.M) * double(g.N) * double(g.K1 + g.K2));
  PGF_LAUNCH_CHECK();
  return PGF_OK;
}

int split_slices_tc(int64_t M, int64_t N, int64_t K) {
  const int bn = tile_bn(TC_GENERIC, N);
  const int64_t tiles = ((M + TC_BM - 1) / TC_BM) * ((N + bn - 1) / bn);
  const int64_t nk = (K + TC_BK - 1) / TC_BK;
  const int64_t sm = sm_count();
  if (tiles * 2 > sm) return 1;
  int64_t S = sm / tiles;
  if (S > nk / 4) S = nk / 4;  // at least four k-blocks (256 deep) per slice
  if (S > 32) S = 32;
  return S < 1 ? 1 : int(S);
}

int run_gemm_tc_split(const Gemm& g, int slices, float* part, int* launched, cudaStream_t s) {
  if (!tc_usable(g)) return PGF_ERR_UNSUPPORTED;
  const int nk = int((g.K + TC_BK - 1) / TC_BK);
  TcParams p = {};
  p.mode = TC_GENERIC;
  p.ng = 1;
  p.kper = (nk + slices - 1) / slices;
  p.ksplit = (nk + p.kper - 1) / p.kper;
  p.split_stride = g.M * g.N;
  p.D = part; p.d_bf16 = 0; p.ldd = g.N;
  p.epi = epi_default();
  *launched = p.ksplit;
  return launch_tc(g, p, s, PROF_GEMM_TC);
}

int tc_ce_fwd(const Gemm& g, int ng, const int64_t* targets, float* part_m, float* part_s,
              float* tgt_logit, int* n_groups_out, cudaStream_t s) {
  if (!tc_usable(g)) return PGF_ERR_UNSUPPORTED;
  TcParams p = {};
  p.mode = TC_CE_FWD;
  p.ng = ng;
  p.targets = targets;
  p.part_m = part_m; p.part_s = part_s; p.tgt_logit = tgt_logit;
  // `ng` counts 128-wide tiles; a 256-wide launch covers the same columns per unit with ng / 2
  const int bn = tile_bn(TC_CE_FWD, g.N);
  if (bn == 256) {
    TcParams q = p;
    q.ng = ng / 2 > 0 ? ng / 2 : 1;
    const int64_t n_tiles = (g.N + 255) / 256;
    *n_groups_out = 2 * int((n_tiles + q.ng - 1) / q.ng);  // two column halves per unit
    const int rc = launch_tc_bn<256>(g, q, s, PROF_CE);
    if (rc != PGF_ERR_UNSUPPORTED) return rc;
    clear_error();
  }
  const int64_t n_tiles = (g.N + TC_BN - 1) / TC_BN;
  *n_groups_out = 2 * int((n_tiles + ng - 1) / ng);  // two column halves per unit
  return launch_tc_bn<128>(g, p, s, PROF_CE);
}

int tc_ce_bwd(const Gemm& g, const int64_t* targets, const float* lse, float scale, __nv_bfloat16* G,
              int64_t ldg, cudaStream_t s) {
  if (!tc_usable(g)) return PGF_ERR_UNSUPPORTED;
  TcParams p = {};
  p.mode = TC_CE_BWD;
  p.ng = 1;
  p.targets = targets; p.lse = lse; p.scale = scale;
  p.D = G; p.d_bf16 = 1; p.ldd = ldg;
  return launch_tc(g, p, s, PROF_CE);
}

}  // namespace pgf

// Reads and clears the tensor-core kernels' fault flags (1 = a bounded wait expired).  Synchronous.
extern "C" int pgf_tc_fault(void) {
  const int a = pgf::take_tc_fault();
  const int b = pgf::lmhead_tc_fault();
  if (a < 0 || b < 0) return -1;
  return (a || b) ? 1 : 0;
}
