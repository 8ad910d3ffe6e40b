// tcgen05 / TMEM dense product for bf16 operands on sm_100a.
//
// One CTA computes a 128 x 128 output tile, fp32 accumulation in tensor memory (TMEM):
//   * warp 0, one lane: TMA producer.  Operand tiles arrive 128B-swizzled through a TC_STAGES-deep
//     mbarrier ring.  A K-major operand is one box {64 k, 128 rows}; an MN-major operand (stored
//     transposed) is two boxes {64 rows, 64 k} side by side, so no operand is ever transposed in
//     memory.
//   * warp 1, one lane: issues tcgen05.mma (kind::f16, bf16 x bf16 -> f32, M=128, N=128, K=16)
//     and frees each smem stage with tcgen05.commit onto its "empty" mbarrier.
//   * all 4 warps: epilogue.  Warp w reads TMEM lanes 32w..32w+31 (tile rows) with tcgen05.ld and
//     applies the shared epilogue (bias, GELU / GELU', addend, accumulate) from gemm.cuh.
// Every mbarrier wait is bounded by a clock budget; on expiry the kernel records a fault in
// g_tc_fault, skips the epilogue, releases its TMEM and returns.
#include "gemm.cuh"

#include <cuda.h>

#include <mutex>

namespace pgf {

constexpr int TC_BM = 128, TC_BN = 128, TC_BK = 64;
constexpr int TC_STAGES = 3;
constexpr int TC_THREADS = 128;
constexpr int TILE_A_BYTES = TC_BM * TC_BK * 2;
constexpr int TILE_B_BYTES = TC_BN * TC_BK * 2;
constexpr int STAGE_BYTES = TILE_A_BYTES + TILE_B_BYTES;
constexpr uint32_t TMEM_COLS = 128;
constexpr size_t TC_SMEM = size_t(TC_STAGES) * STAGE_BYTES + 1024 /* align */ + 256 /* barriers */;
constexpr long long WAIT_CYCLES = 4000000000ll;  // about 2 s at the B200 clock

__device__ int g_tc_fault;

struct TcParams {
  int64_t M, N, K;
  int a_mn, b_mn;
  void* D;
  int d_bf16;
  int64_t ldd;
  pgf_epilogue epi;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
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

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
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

__global__ void __launch_bounds__(TC_THREADS, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
               const TcParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* tiles = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(tiles + TC_STAGES * STAGE_BYTES);
  uint64_t* empty = full + TC_STAGES;
  uint64_t* accb = empty + TC_STAGES;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(accb + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t m0 = int64_t(blockIdx.y) * TC_BM, n0 = int64_t(blockIdx.x) * TC_BN;
  const int nk = int((p.K + TC_BK - 1) / TC_BK);

  if (threadIdx.x == 0) {
    for (int s = 0; s < TC_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accb, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmB)) : "memory");
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

  if (warp == 0 && lane == 0) {
    // ---- TMA producer
    for (int kb = 0; kb < nk; ++kb) {
      const int s = kb % TC_STAGES, r = kb / TC_STAGES;
      if (r > 0 && !mbar_wait(&empty[s], uint32_t((r - 1) & 1))) break;
      mbar_expect_tx(&full[s], STAGE_BYTES);
      uint8_t* sa = tiles + s * STAGE_BYTES;
      uint8_t* sb = sa + TILE_A_BYTES;
      const int k0 = kb * TC_BK;
      if (!p.a_mn) {
        tma_load_2d(sa, &tmA, &full[s], k0, int(m0));
      } else {
        tma_load_2d(sa, &tmA, &full[s], int(m0), k0);
        tma_load_2d(sa + TILE_A_BYTES / 2, &tmA, &full[s], int(m0) + 64, k0);
      }
      if (!p.b_mn) {
        tma_load_2d(sb, &tmB, &full[s], k0, int(n0));
      } else {
        tma_load_2d(sb, &tmB, &full[s], int(n0), k0);
        tma_load_2d(sb + TILE_B_BYTES / 2, &tmB, &full[s], int(n0) + 64, k0);
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer
    const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(p.a_mn) << 15) |
                           (uint32_t(p.b_mn) << 16) | (uint32_t(TC_BN >> 3) << 17) |
                           (uint32_t(TC_BM >> 4) << 24);
    for (int kb = 0; kb < nk; ++kb) {
      const int s = kb % TC_STAGES, r = kb / TC_STAGES;
      if (!mbar_wait(&full[s], uint32_t(r & 1))) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t a_base = smem_u32(tiles + s * STAGE_BYTES);
      const uint32_t b_base = a_base + TILE_A_BYTES;
#pragma unroll
      for (int kk = 0; kk < TC_BK / 16; ++kk) {
        // K-major: advance 16 elements (32 B) inside the 128B swizzle row;
        // MN-major: advance 16 k-rows (2 KB), two 8-row atoms apart by SBO = 1 KB.
        const uint64_t ad = p.a_mn ? sdesc(a_base + kk * 2048, TILE_A_BYTES / 2, 1024)
                                   : sdesc(a_base + kk * 32, 16, 1024);
        const uint64_t bd = p.b_mn ? sdesc(b_base + kk * 2048, TILE_B_BYTES / 2, 1024)
                                   : sdesc(b_base + kk * 32, 16, 1024);
        umma_bf16(tmem, ad, bd, idesc, (kb | kk) != 0);
      }
      umma_commit(&empty[s]);
    }
    umma_commit(accb);
  }
  __syncwarp();

  // ---- epilogue
  const bool ok = mbar_wait(accb, 0);
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (ok) {
    const int64_t m = m0 + warp * 32 + lane;
#pragma unroll 1
    for (int c = 0; c < TC_BN / 32; ++c) {
      uint32_t r[32];
      tmem_ld32(tmem + (uint32_t(warp * 32) << 16) + uint32_t(c * 32), r);
      if (m < p.M) {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int64_t n = n0 + c * 32 + j;
          if (n < p.N) epi_store(p.epi, p.D, p.d_bf16, p.ldd, m, n, __uint_as_float(r[j]));
        }
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
  }
}

// ---------------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*,
                                  CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                  CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
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
static bool make_map(CUtensorMap* m, const void* ptr, int64_t inner, int64_t outer, int64_t ld,
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

static bool tc_disabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("PGF_DISABLE_TC");
    v = (e && e[0] == '1') ? 1 : 0;
  }
  return v == 1;
}

int run_gemm_tc(const Gemm& g, cudaStream_t s) {
  if (tc_disabled() || !g.a_bf16 || !g.b_bf16) return PGF_ERR_UNSUPPORTED;
  if (g.M == 0 || g.N == 0) return PGF_OK;
  if (g.K == 0) return PGF_ERR_UNSUPPORTED;
  if (!aligned(g.A, 16) || !aligned(g.B, 16) || (g.lda * 2) % 16 || (g.ldb * 2) % 16) return PGF_ERR_UNSUPPORTED;
  if (g.M > (int64_t(1) << 31) || g.N > (int64_t(1) << 31) || g.K > (int64_t(1) << 31)) return PGF_ERR_UNSUPPORTED;
  if (ceil_div(g.M, TC_BM) > 65535) return PGF_ERR_UNSUPPORTED;
  CUtensorMap ma, mb;
  const bool oka = g.a_trans ? make_map(&ma, g.A, g.M, g.K, g.lda, 64, 64)
                             : make_map(&ma, g.A, g.K, g.M, g.lda, 64, TC_BM);
  const bool okb = g.b_trans ? make_map(&mb, g.B, g.N, g.K, g.ldb, 64, 64)
                             : make_map(&mb, g.B, g.K, g.N, g.ldb, 64, TC_BN);
  if (!oka || !okb) return PGF_ERR_UNSUPPORTED;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [] {
    attr_err = cudaFuncSetAttribute(gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(TC_SMEM));
  });
  if (attr_err != cudaSuccess) {
    set_error("gemm_tc: smem attribute: %s", cudaGetErrorString(attr_err));
    return PGF_ERR_CUDA;
  }
  TcParams p;
  p.M = g.M; p.N = g.N; p.K = g.K;
  p.a_mn = g.a_trans; p.b_mn = g.b_trans;
  p.D = g.D; p.d_bf16 = g.d_bf16; p.ldd = g.ldd;
  p.epi = g.epi;
  dim3 grid(ceil_div(g.N, TC_BN), ceil_div(g.M, TC_BM));
  prof_begin(PROF_GEMM_TC, s);
  gemm_tc_kernel<<<grid, TC_THREADS, TC_SMEM, s>>>(ma, mb, p);
  prof_end(PROF_GEMM_TC, s, 2.0 * double(g.M) * double(g.N) * double(g.K));
  PGF_LAUNCH_CHECK();
  return PGF_OK;
}

}  // namespace pgf

// Reads and clears the tensor-core engine's fault flag (1 = a bounded wait expired).  Synchronous.
extern "C" int pgf_tc_fault(void) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, pgf::g_tc_fault, sizeof(int)) != cudaSuccess) return -1;
  int z = 0;
  cudaMemcpyToSymbol(pgf::g_tc_fault, &z, sizeof(int));
  return v;
}
