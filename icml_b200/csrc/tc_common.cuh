// Building blocks of the tcgen05 / TMEM / TMA kernels (sm_100a): mbarriers with bounded waits,
// 2-D TMA tile loads, shared-memory matrix descriptors (128B swizzle), tcgen05.mma / commit / ld,
// the 128B-swizzled epilogue staging rows stored by TMA bulk-tensor stores, and the host-side
// tensor-map encoders.
#pragma once
#include "gemm.cuh"

#include <cuda.h>
#include <math.h>
#include <string.h>

#include <mutex>

namespace pgf {

constexpr long long WAIT_CYCLES = 4000000000ll;  // about 2 s at the B200 clock

// Set (never cleared by a kernel) when a bounded mbarrier wait expires.  One flag per translation
// unit (the library is compiled without relocatable device code, so device variables do not link
// across units); take_tc_fault() reads and
// clears this unit's flag, and pgf_tc_fault() combines the units.
static __device__ int g_tc_fault;

static inline int take_tc_fault() {
  int v = 0, z = 0;
  if (cudaMemcpyFromSymbol(&v, g_tc_fault, sizeof(int)) != cudaSuccess) return -1;
  cudaMemcpyToSymbol(g_tc_fault, &z, sizeof(int));
  return v;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// One lane of a converged warp (the same lane on every call): issues the single-thread tcgen05 / TMA
// instructions while the whole warp runs the loop around them, so that their operands (descriptors,
// coordinates, addresses) are warp-uniform values.
__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "elect.sync _|P, 0xffffffff;\n\t"
      "selp.b32 %0, 1, 0, P;\n\t}\n"
      : "=r"(pred));
  return pred != 0;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Bounded wait for the phase of parity `parity` to complete; false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t addr = smem_u32(bar);
  const long long t0 = clock64();
  while (true) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(done)
        : "r"(addr), "r"(parity)
        : "memory");
    if (done) return true;
    if (clock64() - t0 > WAIT_CYCLES) {
      atomicExch(&g_tc_fault, 1);
      return false;
    }
  }
}

// Bounded mbarrier wait whose outcome is the same in every lane of the warp (for whole-warp roles
// that go on to warp-synchronous instructions).
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity)) != 0;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

// ---- CTA pairs (a cluster of two CTAs sharing one tcgen05.mma.cta_group::2 per tile)
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// The shared::cluster address of the same shared-memory object in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t cluster_addr(const void* p, uint32_t rank) {
  uint32_t a;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_u32(p)), "r"(rank));
  return a;
}
// Every thread of every CTA of the cluster.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}
// 2-D tile load into this CTA's shared memory whose completion is counted on a barrier of either
// CTA of the pair (`cluster_bar`, a shared::cluster address); the data lands in this CTA only.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t cluster_bar, int c0,
                                                 int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(cluster_bar), "r"(c0), "r"(c1)
      : "memory");
}
__device__ __forceinline__ void umma_bf16_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                               uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum));
}
// Arrive on a barrier (shared::cluster address, either CTA) when this thread's pair MMAs complete.
__device__ __forceinline__ void umma_commit_pair(uint32_t cluster_bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               ::"r"(cluster_bar) : "memory");
}

// Shared-memory matrix descriptor, 128B swizzle (layout type 2), descriptor version 1.
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return uint64_t((saddr >> 4) & 0x3FFFu) | (uint64_t((lbo >> 4) & 0x3FFFu) << 16) |
         (uint64_t((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum));
}

// The same product with A read from tensor memory (K-major: row m of A in TMEM lane m, K elements
// packed two per 32-bit column, the lower K index in the low half).
__device__ __forceinline__ void umma_bf16_ta(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n"
      ::"r"(tmem_d), "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accum));
}

// 16 consecutive 32-bit TMEM columns of this thread's lane (the warp's 32-lane quarter).
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};"
      ::"r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
        "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
        "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
        "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// The same load without its wait: issue several, then tmem_wait_ld() once before reading any of them.
__device__ __forceinline__ void tmem_ld32_nowait(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
        "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
        "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// ---- epilogue staging: 32 rows x 128 B, 128B-swizzled (16-byte chunk j of row r at j ^ (r % 8)),
//      written by the warp and stored to global memory by one TMA bulk-tensor store.
// NB = 2: two 4 KB buffers taken in turn (the store issued from a buffer two stagings ago must have
// finished reading it); NB = 1: one buffer (the previous store must have finished reading it).
template <int NB = 2>
__device__ __forceinline__ uint8_t* stage_acquire(uint8_t* stg, uint32_t& sq, int lane) {
  static_assert(NB == 1 || NB == 2, "one or two staging buffers");
  uint8_t* b = stg + (sq % uint32_t(NB)) * 4096u;
  if (lane == 0) {
    if (NB == 2)
      asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
    else
      asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
  }
  __syncwarp();
  ++sq;
  return b;
}

__device__ __forceinline__ void stage_row(uint8_t* b, int lane, const uint32_t (&w)[32]) {
  const uint32_t row = smem_u32(b) + uint32_t(lane) * 128u;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint32_t a = row + ((uint32_t(j) ^ uint32_t(lane & 7)) << 4);
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(w[4 * j]), "r"(w[4 * j + 1]),
                 "r"(w[4 * j + 2]), "r"(w[4 * j + 3])
                 : "memory");
  }
}

// 3-D output map {columns, rows, K slice}: a box of 32 rows x 128 B at (col, row, slice).
__device__ __forceinline__ void stage_store(uint8_t* b, const CUtensorMap* map, int64_t col, int64_t row, int slice,
                                            int lane) {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  __syncwarp();
  if (lane == 0) {
    asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%1, %2, %3}], [%4];"
                 ::"l"(reinterpret_cast<uint64_t>(map)), "r"(int(col)), "r"(int(row)), "r"(slice),
                 "r"(smem_u32(b))
                 : "memory");
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
  }
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// 32 consecutive elements of row m from column nb (zeros outside M x N); vector loads when the whole
// segment is in range and 16-byte aligned.
__device__ __forceinline__ void load_seg(const void* base, int bf16, int64_t ld, int64_t m, int64_t nb, int64_t M,
                                         int64_t N, float (&o)[32]) {
  const int64_t off = m * ld + nb;
  const bool full = m < M && nb + 32 <= N;
  if (full && !bf16 && ((reinterpret_cast<uintptr_t>(static_cast<const float*>(base) + off) & 15) == 0)) {
    const float4* q = reinterpret_cast<const float4*>(static_cast<const float*>(base) + off);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float4 t = __ldg(q + j);
      o[4 * j] = t.x; o[4 * j + 1] = t.y; o[4 * j + 2] = t.z; o[4 * j + 3] = t.w;
    }
  } else if (full && bf16 && ((reinterpret_cast<uintptr_t>(static_cast<const __nv_bfloat16*>(base) + off) & 15) == 0)) {
    const uint4* q = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(base) + off);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint4 t = __ldg(q + j);
      const uint32_t w[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        o[8 * j + 2 * k] = __uint_as_float(w[k] << 16);
        o[8 * j + 2 * k + 1] = __uint_as_float(w[k] & 0xFFFF0000u);
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) o[j] = (m < M && nb + j < N) ? ldv(base, bf16, off + j) : 0.f;
  }
}


// ---- host side: tensor maps
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*,
                                  CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                  CUtensorMapFloatOOBfill);

static inline EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// 2-D bf16 tensor map: `inner` contiguous elements per row, `outer` rows, row pitch `ld` elements.
static inline bool make_map(CUtensorMap* m, const void* ptr, int64_t inner, int64_t outer, int64_t ld,
                     uint32_t box_inner, uint32_t box_outer) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {cuuint64_t(inner), cuuint64_t(outer)};
  cuuint64_t strides[1] = {cuuint64_t(ld) * 2};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t es[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 3-D output map {cols, rows, slices} (float32 or bf16) with a 128-byte x 32-row box, 128B swizzle:
// the store side of the row-per-thread epilogue.  slice_stride in elements (slices > 1: split-K).
static inline bool make_out_map(CUtensorMap* m, void* ptr, int bf16, int64_t cols, int64_t rows, int64_t ld,
                         int64_t slices, int64_t slice_stride) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const int64_t es = bf16 ? 2 : 4;
  cuuint64_t dims[3] = {cuuint64_t(cols), cuuint64_t(rows), cuuint64_t(slices)};
  cuuint64_t strides[2] = {cuuint64_t(ld * es), cuuint64_t((slices > 1 ? slice_stride : ld * rows) * es)};
  cuuint32_t box[3] = {cuuint32_t(128 / es), 32, 1};
  cuuint32_t est[3] = {1, 1, 1};
  return fn(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, ptr, dims, strides, box,
            est, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}


}  // namespace pgf
