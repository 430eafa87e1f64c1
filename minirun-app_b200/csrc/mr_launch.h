// mr_launch.h — host launchers of the templated kernels (one .cu per bit
// width, compiled in parallel).
#pragma once

#include "mr_gemv.cuh"

namespace mr {

constexpr int kPrefetch = 4;  // groups of codes in flight per lane

cudaError_t launch_gemv_b2(const GemvParams& p, int sd, int epi, int nt, int grid, cudaStream_t s);
cudaError_t launch_gemv_b4(const GemvParams& p, int sd, int epi, int nt, int grid, cudaStream_t s);
cudaError_t launch_gemv_b8(const GemvParams& p, int sd, int epi, int nt, int grid, cudaStream_t s);

inline cudaError_t launch_gemv(const GemvParams& p, int bits, int sd, int epi, int nt, int grid,
                               cudaStream_t s) {
  switch (bits) {
    case 2: return launch_gemv_b2(p, sd, epi, nt, grid, s);
    case 4: return launch_gemv_b4(p, sd, epi, nt, grid, s);
    case 8: return launch_gemv_b8(p, sd, epi, nt, grid, s);
    default: return cudaErrorInvalidValue;
  }
}

inline int pick_nt(int max_cols) {
  const int tiles = (max_cols + 7) / 8;
  return tiles <= 1 ? 1 : (tiles <= 2 ? 2 : 8);
}

}  // namespace mr

// Instantiates launch_gemv_b<BITS> in a translation unit.
#define MR_DEFINE_GEMV_LAUNCHER(BITS)                                                          \
  namespace mr {                                                                               \
  template <int SD, int EPI>                                                                   \
  static cudaError_t launch_nt_##BITS(const GemvParams& p, int nt, int grid, cudaStream_t s) { \
    switch (nt) {                                                                              \
      case 1: gemv_kernel<BITS, SD, EPI, 1, kPrefetch><<<grid, kGemvThreads, 0, s>>>(p); break; \
      case 2: gemv_kernel<BITS, SD, EPI, 2, kPrefetch><<<grid, kGemvThreads, 0, s>>>(p); break; \
      default: gemv_kernel<BITS, SD, EPI, 8, kPrefetch><<<grid, kGemvThreads, 0, s>>>(p); break; \
    }                                                                                          \
    return cudaGetLastError();                                                                 \
  }                                                                                            \
  template <int SD>                                                                            \
  static cudaError_t launch_epi_##BITS(const GemvParams& p, int epi, int nt, int grid,         \
                                       cudaStream_t s) {                                       \
    switch (epi) {                                                                             \
      case EPI_STORE: return launch_nt_##BITS<SD, EPI_STORE>(p, nt, grid, s);                  \
      case EPI_SWIGLU: return launch_nt_##BITS<SD, EPI_SWIGLU>(p, nt, grid, s);                \
      default: return launch_nt_##BITS<SD, EPI_PARTIAL>(p, nt, grid, s);                       \
    }                                                                                          \
  }                                                                                            \
  cudaError_t launch_gemv_b##BITS(const GemvParams& p, int sd, int epi, int nt, int grid,      \
                                  cudaStream_t s) {                                            \
    switch (sd) {                                                                              \
      case MR_DTYPE_BF16: return launch_epi_##BITS<MR_DTYPE_BF16>(p, epi, nt, grid, s);        \
      case MR_DTYPE_F16: return launch_epi_##BITS<MR_DTYPE_F16>(p, epi, nt, grid, s);          \
      default: return launch_epi_##BITS<MR_DTYPE_F32>(p, epi, nt, grid, s);                    \
    }                                                                                          \
  }                                                                                            \
  }
