// tcgen05 / TMEM dense-product engine for bf16 operands (placeholder: not yet enabled).
#include "gemm.cuh"

namespace pgf {

int run_gemm_tc(const Gemm& g, cudaStream_t s) {
  (void)g;
  (void)s;
  return PGF_ERR_UNSUPPORTED;
}

}  // namespace pgf
