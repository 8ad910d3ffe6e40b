// Fused LM-head + cross-entropy backward on tcgen05 (bf16 activations), for a chunk of M rows:
//
//   for every 128-row block (one work unit of a persistent CTA) and every 128-wide vocabulary tile j:
//     L_j  = h_rows W_j^T                          tcgen05.mma, accumulator in TMEM (2 buffers)
//     G_j  = (exp(L_j - lse) - onehot) * scale     epilogue warps, rounded to bf16
//     dh  += G_j W_j                               tcgen05.mma, accumulator in TMEM over all tiles
//
// G_j is written once, into shared memory in the tensor cores' K-major 128B-swizzled operand layout;
// the dh product reads it from there, and a TMA bulk-tensor store copies the same buffer to global
// memory for grad W = G^T h (a separate product over all rows).  Compared with materialising G and
// running dh = G W as a separate GEMM, G is never read back from HBM for dh and one pass over the
// logits serves both.  The W tile of the logits product (K-major, K = d) is reused, viewed MN-major,
// as the B operand of the dh product (N = d, K = vocabulary).
//
// Roles (320 threads): warp 0 lane 0 issues the TMA loads (h rows once per unit, W tiles into two
// slots); warp 1 lane 0 issues the MMAs (logits of tile j, then dh of tile j-1); warps 2..9 are the
// epilogue (warp w: TMEM lanes 32 (w % 4) .., vocabulary half (w - 2) / 4 of the tile).  Every
// mbarrier wait is bounded and records a fault in this unit's g_tc_fault on expiry.
//
// Shared memory: h rows (d * 256 B), two W slots (d * 256 B each), the G tile (32 KB): 224 KB at
// d = 256.  TMEM: 512 columns (logits 2 x 128, dh d <= 256).
#include "tc_common.cuh"

namespace pgf {
namespace lmh {

constexpr int BM = 128;            // rows per work unit
constexpr int BV = 128;            // vocabulary ids per tile
constexpr int THREADS = 320;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t G_BYTES = BM * BV * 2;
constexpr int NBARS = 16;

struct Params {
  int64_t M;             // rows of the chunk
  int64_t V;             // vocabulary size
  int d;                 // model width: a multiple of 64, at most 256
  int n_tiles;           // ceil(V / BV)
  int64_t units;         // ceil(M / BM)
  const int64_t* targets;
  const float* lse;
  float scale;
  __nv_bfloat16* dh;     // (M, d) bf16, row pitch d
};

__global__ void __launch_bounds__(THREADS, 1)
ce_bwd_dh_kernel(const __grid_constant__ CUtensorMap tmH, const __grid_constant__ CUtensorMap tmW,
                 const __grid_constant__ CUtensorMap tmG, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int dch = p.d / 64;                       // 64-wide K chunks of d
  const uint32_t HB = uint32_t(dch) * 16384u;     // bytes of the h rows and of one W slot
  uint8_t* sH = base;
  uint8_t* sW = base + HB;                        // slots 0, 1
  uint8_t* sG = base + 3 * HB;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sG + G_BYTES);
  uint64_t* hfull = bars + 0;
  uint64_t* hempty = bars + 1;
  uint64_t* wfull = bars + 2;    // [2]
  uint64_t* wempty = bars + 4;   // [2]
  uint64_t* tfull = bars + 6;    // [2]
  uint64_t* tempty = bars + 8;   // [2]
  uint64_t* gready = bars + 10;
  uint64_t* gfree = bars + 11;
  uint64_t* dhdone = bars + 12;
  uint64_t* dhfree = bars + 13;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + NBARS);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(hfull, 1);
    mbar_init(hempty, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&wfull[s], 1);
      mbar_init(&wempty[s], 1);
      mbar_init(&tfull[s], 1);
      mbar_init(&tempty[s], 8);
    }
    mbar_init(gready, 8);
    mbar_init(gfree, 1);
    mbar_init(dhdone, 1);
    mbar_init(dhfree, 8);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmH)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmW)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmG)) : "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(smem_u32(tslot)), "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tslot;
  const uint32_t tmem_dh = tmem + 2 * BV;

  if (warp == 0) {
    if (lane == 0) {
      // ---- TMA producer
      uint32_t jj = 0, uu = 0;
      bool ok = true;
      for (int64_t u = blockIdx.x; u < p.units && ok; u += gridDim.x, ++uu) {
        const int m0 = int(u * BM);
        if (uu > 0 && !mbar_wait(hempty, (uu - 1) & 1)) { ok = false; break; }
        mbar_expect_tx(hfull, HB);
        for (int c = 0; c < dch; ++c) tma_load_2d(sH + c * 16384, &tmH, hfull, c * 64, m0);
        for (int j = 0; j < p.n_tiles; ++j, ++jj) {
          const uint32_t s = jj & 1, r = jj >> 1;
          if (r > 0 && !mbar_wait(&wempty[s], (r - 1) & 1)) { ok = false; break; }
          mbar_expect_tx(&wfull[s], HB);
          for (int c = 0; c < dch; ++c) tma_load_2d(sW + s * HB + c * 16384, &tmW, &wfull[s], c * 64, j * BV);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---- MMA issuer: logits of tile j, then dh of tile j-1 (whose G the epilogue has written)
      const uint32_t idesc_l = (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(BV >> 3) << 17) |
                               (uint32_t(BM >> 4) << 24);
      const uint32_t idesc_d = (1u << 4) | (1u << 7) | (1u << 10) | (1u << 16) | (uint32_t(p.d >> 3) << 17) |
                               (uint32_t(BM >> 4) << 24);
      uint32_t jj = 0, tt = 0, uu = 0;
      bool ok = true;
      // dh product of the tile with global index t, W slot s; `first`: the unit's first tile
      auto issue_dh = [&](uint32_t t, uint32_t s, bool first) -> bool {
        if (!mbar_wait(gready, t & 1)) return false;
        if (first && uu > 0 && !mbar_wait(dhfree, (uu - 1) & 1)) return false;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t g_base = smem_u32(sG), w_base = smem_u32(sW + s * HB);
#pragma unroll
        for (int kk = 0; kk < BV / 16; ++kk) {
          // A = G (K-major, K = vocabulary: two 64-wide chunks 16 KB apart); B = W tile viewed
          // MN-major (N = d in 64-wide blocks 16 KB apart, K = vocabulary rows, 16 rows = 2 KB)
          const uint64_t ad = sdesc(g_base + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = sdesc(w_base + kk * 2048, 16384, 1024);
          umma_bf16(tmem_dh, ad, bd, idesc_d, (!first || kk > 0) ? 1u : 0u);
        }
        umma_commit(&wempty[s]);
        umma_commit(gfree);
        return true;
      };
      for (int64_t u = blockIdx.x; u < p.units && ok; u += gridDim.x, ++uu) {
        if (!mbar_wait(hfull, uu & 1)) { ok = false; break; }
        uint32_t prev_t = 0, prev_s = 0;
        for (int j = 0; j < p.n_tiles && ok; ++j, ++jj, ++tt) {
          const uint32_t s = jj & 1, r = jj >> 1;
          const uint32_t buf = tt & 1, use = tt >> 1;
          if (!mbar_wait(&wfull[s], r & 1)) { ok = false; break; }
          if (use > 0 && !mbar_wait(&tempty[buf], (use - 1) & 1)) { ok = false; break; }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t h_base = smem_u32(sH), w_base = smem_u32(sW + s * HB);
          for (int kk = 0; kk < 4 * dch; ++kk) {
            const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
            umma_bf16(tmem + buf * BV, sdesc(h_base + off, 16, 1024), sdesc(w_base + off, 16, 1024), idesc_l,
                      kk > 0 ? 1u : 0u);
          }
          umma_commit(&tfull[buf]);
          if (j == p.n_tiles - 1) umma_commit(hempty);  // the unit's h rows are no longer read
          if (j > 0 && !issue_dh(prev_t, prev_s, j == 1)) { ok = false; break; }
          prev_t = tt;
          prev_s = s;
        }
        if (!ok) break;
        if (!issue_dh(prev_t, prev_s, p.n_tiles == 1)) { ok = false; break; }
        umma_commit(dhdone);
      }
    }
  } else {
    // ---- epilogue warps 2..9
    const int q = warp & 3;
    const int hf = (warp - 2) >> 2;
    constexpr float L2E = 1.4426950408889634f;
    uint32_t tt = 0, uu = 0;
    bool ok = true;
    for (int64_t u = blockIdx.x; u < p.units && ok; u += gridDim.x, ++uu) {
      const int64_t m0 = u * BM;
      const int64_t row = m0 + q * 32 + lane;
      const bool row_ok = row < p.M;
      const int64_t tgt = row_ok ? p.targets[row] : -1;
      const float ll = row_ok ? p.lse[row] * L2E : 0.f;
      for (int j = 0; j < p.n_tiles; ++j, ++tt) {
        const uint32_t buf = tt & 1, use = tt >> 1;
        if (!mbar_wait_warp(&tfull[buf], use & 1)) { ok = false; break; }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        uint32_t r0[32], r1[32];
        const uint32_t ta = tmem + buf * BV + (uint32_t(q * 32) << 16) + uint32_t(hf * 64);
        tmem_ld32(ta, r0);
        tmem_ld32(ta + 32, r1);
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[buf]);
        const int64_t nb = int64_t(j) * BV + hf * 64;
        uint32_t pk[32];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float g0 = exp2f(fmaf(__uint_as_float(r0[2 * i]), L2E, -ll));
          float g1 = exp2f(fmaf(__uint_as_float(r0[2 * i + 1]), L2E, -ll));
          if (tgt == nb + 2 * i) g0 -= 1.0f;
          if (tgt == nb + 2 * i + 1) g1 -= 1.0f;
          pk[i] = pack_bf16(g0 * p.scale, g1 * p.scale);
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float g0 = exp2f(fmaf(__uint_as_float(r1[2 * i]), L2E, -ll));
          float g1 = exp2f(fmaf(__uint_as_float(r1[2 * i + 1]), L2E, -ll));
          if (tgt == nb + 32 + 2 * i) g0 -= 1.0f;
          if (tgt == nb + 32 + 2 * i + 1) g1 -= 1.0f;
          pk[16 + i] = pack_bf16(g0 * p.scale, g1 * p.scale);
        }
        // the G tile is free once the dh product of the previous tile is done and the previous
        // TMA store has read it
        if (tt > 0 && !mbar_wait_warp(gfree, (tt - 1) & 1)) { ok = false; break; }
        if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
        __syncwarp();
        uint8_t* gb = sG + hf * 16384 + q * 4096;
        stage_row(gb, lane, pk);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) {
          if (m0 + q * 32 < p.M && nb < p.V) {
            asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%1, %2, %3}], [%4];"
                         ::"l"(reinterpret_cast<uint64_t>(&tmG)), "r"(int(nb)), "r"(int(m0 + q * 32)), "r"(0),
                         "r"(smem_u32(gb))
                         : "memory");
            asm volatile("cp.async.bulk.commit_group;" ::: "memory");
          }
          mbar_arrive(gready);
        }
      }
      if (!ok) break;
      // the unit's dh: TMEM lanes of this warp, columns hf * d/2 .. (bf16, 16-byte stores)
      if (!mbar_wait_warp(dhdone, uu & 1)) { ok = false; break; }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const int half = p.d / 2;
      for (int c = 0; c < half; c += 32) {
        uint32_t r[32];
        tmem_ld32(tmem_dh + (uint32_t(q * 32) << 16) + uint32_t(hf * half + c), r);
        if (row_ok) {
          uint4* dst = reinterpret_cast<uint4*>(p.dh + row * p.d + hf * half + c);
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            uint4 w;
            w.x = pack_bf16(__uint_as_float(r[8 * v]), __uint_as_float(r[8 * v + 1]));
            w.y = pack_bf16(__uint_as_float(r[8 * v + 2]), __uint_as_float(r[8 * v + 3]));
            w.z = pack_bf16(__uint_as_float(r[8 * v + 4]), __uint_as_float(r[8 * v + 5]));
            w.w = pack_bf16(__uint_as_float(r[8 * v + 6]), __uint_as_float(r[8 * v + 7]));
            dst[v] = w;
          }
        }
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(dhfree);
    }
    if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
  }
}

// The same product with the h rows in tensor memory instead of shared memory.  With two W slots and
// the dh product one tile behind the logits, the TMA load of tile j+2 can only start once dh(j) has
// released its slot, which is the product just before logits(j+2): every tile waited for a W load.
// Here the unit's h rows sit in TMEM (d/2 columns, the A operand of the logits product) and the
// 64 KB they took in shared memory hold a third W slot, so W(j+2) loads while logits(j+1) and dh(j)
// run.  TMEM: logits 128 columns (one buffer: the epilogue reads it out right after it completes,
// while dh of the previous tile runs), dh d columns, h d/2 columns: 512 at d = 256.
// The epilogue warps write the h rows into TMEM (tcgen05.st) at the start of each unit.
constexpr int NSLOT3 = 3;

struct Params3 {
  int64_t M, V;
  int d, n_tiles;
  int64_t units;
  const __nv_bfloat16* h;  // (M, d) bf16, row pitch d
  const int64_t* targets;
  const float* lse;
  float scale;
  float log2_scale;        // log2(scale): the scale is folded into the exponent
  __nv_bfloat16* dh;
};

__global__ void __launch_bounds__(THREADS, 1)
ce_bwd_dh3_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmG,
                  const Params3 p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int dch = p.d / 64;
  const uint32_t HB = uint32_t(dch) * 16384u;     // bytes of one W slot
  uint8_t* sW = base;                             // slots 0..2
  uint8_t* sG = base + NSLOT3 * HB;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sG + G_BYTES);
  uint64_t* wfull = bars + 0;    // [3]
  uint64_t* wempty = bars + 3;   // [3]
  uint64_t* tfull = bars + 6;
  uint64_t* tempty = bars + 7;
  uint64_t* hready = bars + 8;
  uint64_t* hfree = bars + 9;
  uint64_t* gready = bars + 10;
  uint64_t* gfree = bars + 11;
  uint64_t* dhdone = bars + 12;
  uint64_t* dhfree = bars + 13;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + NBARS);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < NSLOT3; ++s) {
      mbar_init(&wfull[s], 1);
      mbar_init(&wempty[s], 1);
    }
    mbar_init(tfull, 1);
    mbar_init(tempty, 8);
    mbar_init(hready, 8);
    mbar_init(hfree, 1);
    mbar_init(gready, 8);
    mbar_init(gfree, 1);
    mbar_init(dhdone, 1);
    mbar_init(dhfree, 8);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmW)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmG)) : "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(smem_u32(tslot)), "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tslot;
  const uint32_t tmem_l = tmem;                    // logits, BV columns
  const uint32_t tmem_dh = tmem + BV;              // dh, d columns
  const uint32_t tmem_h = tmem + BV + 256;         // h rows, d/2 columns

  if (warp == 0) {
    // ---- TMA producer: W tiles through the three slots (the whole warp waits, one lane issues)
    const bool leader = elect_one();
    uint32_t jj = 0;
    bool ok = true;
    for (int64_t u = blockIdx.x; u < p.units && ok; u += gridDim.x) {
      for (int j = 0; j < p.n_tiles; ++j, ++jj) {
        const uint32_t s = jj % NSLOT3, r = jj / NSLOT3;
        if (r > 0 && !mbar_wait_warp(&wempty[s], (r - 1) & 1)) { ok = false; break; }
        if (leader) {
          mbar_expect_tx(&wfull[s], HB);
          for (int c = 0; c < dch; ++c) tma_load_2d(sW + s * HB + c * 16384, &tmW, &wfull[s], c * 64, j * BV);
        }
        __syncwarp();
      }
    }
  } else if (warp == 1) {
    {
      // ---- MMA issuer: logits of tile j (A = h rows in TMEM), then dh of tile j-1; the whole warp
      //      runs the loop and waits, one elected lane issues every MMA and commit
      const bool leader = elect_one();
      const uint32_t idesc_l = (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(BV >> 3) << 17) |
                               (uint32_t(BM >> 4) << 24);
      const uint32_t idesc_d = (1u << 4) | (1u << 7) | (1u << 10) | (1u << 16) | (uint32_t(p.d >> 3) << 17) |
                               (uint32_t(BM >> 4) << 24);
      uint32_t jj = 0, tt = 0, uu = 0;
      bool ok = true;
      auto issue_dh = [&](uint32_t t, uint32_t s, bool first) -> bool {
        if (!mbar_wait_warp(gready, t & 1)) return false;
        if (first && uu > 0 && !mbar_wait_warp(dhfree, (uu - 1) & 1)) return false;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t g_base = smem_u32(sG), w_base = smem_u32(sW + s * HB);
#pragma unroll
        for (int kk = 0; kk < BV / 16; ++kk) {
          const uint64_t ad = sdesc(g_base + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = sdesc(w_base + kk * 2048, 16384, 1024);
          if (leader) umma_bf16(tmem_dh, ad, bd, idesc_d, (!first || kk > 0) ? 1u : 0u);
        }
        if (leader) {
          umma_commit(&wempty[s]);
          umma_commit(gfree);
        }
        __syncwarp();
        return true;
      };
      for (int64_t u = blockIdx.x; u < p.units && ok; u += gridDim.x, ++uu) {
        if (!mbar_wait_warp(hready, uu & 1)) { ok = false; break; }
        uint32_t prev_t = 0, prev_s = 0;
        for (int j = 0; j < p.n_tiles && ok; ++j, ++jj, ++tt) {
          const uint32_t s = jj % NSLOT3, r = jj / NSLOT3;
          if (!mbar_wait_warp(&wfull[s], r & 1)) { ok = false; break; }
          if (tt > 0 && !mbar_wait_warp(tempty, (tt - 1) & 1)) { ok = false; break; }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t w_base = smem_u32(sW + s * HB);
          for (int kk = 0; kk < 4 * dch; ++kk) {
            const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
            if (leader)
              umma_bf16_ta(tmem_l, tmem_h + uint32_t(8 * kk), sdesc(w_base + off, 16, 1024), idesc_l,
                           kk > 0 ? 1u : 0u);
          }
          if (leader) {
            umma_commit(tfull);
            if (j == p.n_tiles - 1) umma_commit(hfree);  // the unit's h rows are no longer read
          }
          __syncwarp();
          if (j > 0 && !issue_dh(prev_t, prev_s, j == 1)) { ok = false; break; }
          prev_t = tt;
          prev_s = s;
        }
        if (!ok) break;
        if (!issue_dh(prev_t, prev_s, p.n_tiles == 1)) { ok = false; break; }
        if (leader) umma_commit(dhdone);
        __syncwarp();
      }
    }
  } else {
    // ---- epilogue warps 2..9: TMEM lane quarter q, vocabulary half hf of each tile
    const int q = warp & 3;
    const int hf = (warp - 2) >> 2;
    const int dq = p.d / 4;  // TMEM columns of h rows written by this warp
    constexpr float L2E = 1.4426950408889634f;
    uint32_t tt = 0, uu = 0;
    bool ok = true;
    for (int64_t u = blockIdx.x; u < p.units && ok; u += gridDim.x, ++uu) {
      const int64_t m0 = u * BM;
      const int64_t row = m0 + q * 32 + lane;
      const bool row_ok = row < p.M;
      const int64_t tgt = row_ok ? p.targets[row] : -1;
      // g = scale exp(l - lse) = exp2(l log2e - (lse log2e - log2 scale))
      const float lls = row_ok ? fmaf(p.lse[row], L2E, -p.log2_scale) : 0.f;
      // the unit's h rows into TMEM: this thread's row, elements 2 hf dq .. 2 (hf + 1) dq (zero past M)
      if (uu > 0 && !mbar_wait_warp(hfree, (uu - 1) & 1)) { ok = false; break; }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      for (int c = 0; c < dq; c += 16) {
        uint32_t v[16];
        if (row_ok) {
          const uint4* src = reinterpret_cast<const uint4*>(p.h + row * p.d + 2 * (hf * dq + c));
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const uint4 t = __ldg(src + i);
            v[4 * i] = t.x; v[4 * i + 1] = t.y; v[4 * i + 2] = t.z; v[4 * i + 3] = t.w;
          }
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) v[i] = 0u;
        }
        tmem_st16(tmem_h + (uint32_t(q * 32) << 16) + uint32_t(hf * dq + c), v);
      }
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(hready);
      for (int j = 0; j < p.n_tiles; ++j, ++tt) {
        if (!mbar_wait_warp(tfull, tt & 1)) { ok = false; break; }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        uint32_t r0[32], r1[32];
        const uint32_t ta = tmem_l + (uint32_t(q * 32) << 16) + uint32_t(hf * 64);
        tmem_ld32(ta, r0);
        tmem_ld32(ta + 32, r1);
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(tempty);
        const int64_t nb = int64_t(j) * BV + hf * 64;
        uint32_t pk[32];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          pk[i] = pack_bf16(ex2f(fmaf(__uint_as_float(r0[2 * i]), L2E, -lls)),
                            ex2f(fmaf(__uint_as_float(r0[2 * i + 1]), L2E, -lls)));
          pk[16 + i] = pack_bf16(ex2f(fmaf(__uint_as_float(r1[2 * i]), L2E, -lls)),
                                 ex2f(fmaf(__uint_as_float(r1[2 * i + 1]), L2E, -lls)));
        }
        // the one-hot term: a row meets its target in one tile of the vocabulary, so this branch is
        // rare.  The target's value (with scale subtracted) is formed here and written over its
        // element of the staged tile below: fix = column << 16 | bf16 bits, or ~0 for none.
        const int64_t off = tgt - nb;
        const bool hit = off >= 0 && off < 64;
        uint32_t fix = 0xFFFFFFFFu;
        if (__any_sync(0xffffffffu, hit)) {
          if (hit) {
            const int e = int(off);
            float x = 0.f;
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              x = e == i ? __uint_as_float(r0[i]) : x;
              x = e == 32 + i ? __uint_as_float(r1[i]) : x;
            }
            const float g = ex2f(fmaf(x, L2E, -lls)) - p.scale;
            fix = (uint32_t(e) << 16) | uint32_t(__bfloat16_as_ushort(__float2bfloat16_rn(g)));
          }
        }
        if (tt > 0 && !mbar_wait_warp(gfree, (tt - 1) & 1)) { ok = false; break; }
        if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
        __syncwarp();
        uint8_t* gb = sG + hf * 16384 + q * 4096;
        stage_row(gb, lane, pk);
        if (fix != 0xFFFFFFFFu) {
          // element e of this lane's row: 16-byte chunk e / 8 (swizzled by the row), bf16 e % 8
          const uint32_t e = fix >> 16;
          const uint32_t addr = smem_u32(gb) + uint32_t(lane) * 128u + (((e >> 3) ^ uint32_t(lane & 7)) << 4) +
                                (e & 7u) * 2u;
          asm volatile("st.shared.b16 [%0], %1;" ::"r"(addr), "h"(static_cast<unsigned short>(fix & 0xFFFFu))
                       : "memory");
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) {
          if (m0 + q * 32 < p.M && nb < p.V) {
            asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%1, %2, %3}], [%4];"
                         ::"l"(reinterpret_cast<uint64_t>(&tmG)), "r"(int(nb)), "r"(int(m0 + q * 32)), "r"(0),
                         "r"(smem_u32(gb))
                         : "memory");
            asm volatile("cp.async.bulk.commit_group;" ::: "memory");
          }
          mbar_arrive(gready);
        }
      }
      if (!ok) break;
      if (!mbar_wait_warp(dhdone, uu & 1)) { ok = false; break; }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const int half = p.d / 2;
      for (int c = 0; c < half; c += 32) {
        uint32_t r[32];
        tmem_ld32(tmem_dh + (uint32_t(q * 32) << 16) + uint32_t(hf * half + c), r);
        if (row_ok) {
          uint4* dst = reinterpret_cast<uint4*>(p.dh + row * p.d + hf * half + c);
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            uint4 w;
            w.x = pack_bf16(__uint_as_float(r[8 * v]), __uint_as_float(r[8 * v + 1]));
            w.y = pack_bf16(__uint_as_float(r[8 * v + 2]), __uint_as_float(r[8 * v + 3]));
            w.z = pack_bf16(__uint_as_float(r[8 * v + 4]), __uint_as_float(r[8 * v + 5]));
            w.w = pack_bf16(__uint_as_float(r[8 * v + 6]), __uint_as_float(r[8 * v + 7]));
            dst[v] = w;
          }
        }
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(dhfree);
    }
    if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
  }
}

}  // namespace lmh

static size_t ce_bwd_dh_smem(int d) { return size_t(3) * (d / 64) * 16384 + lmh::G_BYTES + 8 * lmh::NBARS + 64 + 1024; }
static size_t ce_bwd_dh3_smem(int d) {
  return size_t(lmh::NSLOT3) * (d / 64) * 16384 + lmh::G_BYTES + 8 * lmh::NBARS + 64 + 1024;
}
// PGF_CE_BWD_TWO_SLOTS=1 selects the kernel with the h rows in shared memory and two W slots.
static bool ce_bwd_two_slots() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("PGF_CE_BWD_TWO_SLOTS");
    v = (e && e[0] == '1') ? 1 : 0;
  }
  return v == 1;
}

bool ce_bwd_dh_usable(const void* h, const void* Wb, const void* G, int64_t ldg, const void* dh, int64_t d) {
  if (d % 64 != 0 || d < 64 || d > 256) return false;
  if (!aligned(h, 16) || !aligned(Wb, 16) || !aligned(G, 16) || !aligned(dh, 16) || (ldg * 2) % 16) return false;
  return encode_fn() != nullptr;
}

// G (bf16, rows x ldg) and dh = G W (bf16, rows x d) for M rows of h; see the kernel's comment.
int ce_bwd_dh(const __nv_bfloat16* h, const __nv_bfloat16* Wb, const int64_t* targets, const float* lse, float scale,
              __nv_bfloat16* G, int64_t ldg, __nv_bfloat16* dh, int64_t M, int64_t V, int64_t d, cudaStream_t s) {
  if (M == 0) return PGF_OK;
  if (!ce_bwd_dh_usable(h, Wb, G, ldg, dh, d)) return PGF_ERR_UNSUPPORTED;
  CUtensorMap mh, mw, mg;
  if (!make_map(&mh, h, d, M, d, 64, lmh::BM) || !make_map(&mw, Wb, d, V, d, 64, lmh::BV) ||
      !make_out_map(&mg, G, 1, V, M, ldg, 1, 0))
    return PGF_ERR_UNSUPPORTED;
  lmh::Params p;
  p.M = M;
  p.V = V;
  p.d = int(d);
  p.n_tiles = int((V + lmh::BV - 1) / lmh::BV);
  p.units = (M + lmh::BM - 1) / lmh::BM;
  p.targets = targets;
  p.lse = lse;
  p.scale = scale;
  p.dh = dh;
  const int64_t grid = p.units < sm_count() ? p.units : sm_count();
  // (the scale is folded into the exponent, so a scale that is not positive takes the other kernel)
  if (!ce_bwd_two_slots() && scale > 0.f) {
    lmh::Params3 p3;
    p3.M = M; p3.V = V; p3.d = int(d); p3.n_tiles = p.n_tiles; p3.units = p.units;
    p3.h = h; p3.targets = targets; p3.lse = lse; p3.scale = scale; p3.dh = dh;
    p3.log2_scale = float(log2(double(scale)));
    const size_t smem3 = ce_bwd_dh3_smem(int(d));
    static int smem_limit3 = 0;
    PGF_CUDA(ensure_dynamic_smem(lmh::ce_bwd_dh3_kernel, smem3, smem_limit3));
    prof_begin(PROF_CE, s);
    lmh::ce_bwd_dh3_kernel<<<unsigned(grid), lmh::THREADS, smem3, s>>>(mw, mg, p3);
    prof_end(PROF_CE, s, 4.0 * double(M) * double(V) * double(d));
    PGF_LAUNCH_CHECK();
    return PGF_OK;
  }
  const size_t smem = ce_bwd_dh_smem(int(d));
  static int smem_limit = 0;
  PGF_CUDA(ensure_dynamic_smem(lmh::ce_bwd_dh_kernel, smem, smem_limit));
  prof_begin(PROF_CE, s);
  lmh::ce_bwd_dh_kernel<<<unsigned(grid), lmh::THREADS, smem, s>>>(mh, mw, mg, p);
  prof_end(PROF_CE, s, 4.0 * double(M) * double(V) * double(d));
  PGF_LAUNCH_CHECK();
  return PGF_OK;
}

int lmhead_tc_fault() { return take_tc_fault(); }

}  // namespace pgf
