// mr_gemv_mx.cu — the MXFP4 instantiation of the TMA dequant-GEMV (e2m1
// codes, e8m0 exponents per 32 elements, store epilogue).
#include "mr_launch.h"

namespace mr {

cudaError_t launch_tma_mx(const GemvParams& p, const TmaMaps& m, int nt, int xs, int grid,
                          cudaStream_t s) {
  if (nt != 1) return cudaErrorInvalidValue;  // one 8-column tile per segment
  return xs == 2 ? launch_tma_inst<4, MR_DTYPE_E8M0, EPI_STORE, 1, 2>(p, m, grid, s)
                 : launch_tma_inst<4, MR_DTYPE_E8M0, EPI_STORE, 1, 1>(p, m, grid, s);
}

}  // namespace mr
