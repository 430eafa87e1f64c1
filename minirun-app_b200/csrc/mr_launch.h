// mr_launch.h — host launchers of the templated GEMV kernels (one .cu per bit
// width, compiled in parallel).
#pragma once

#include "mr_gemv.cuh"
#include "mr_gemv_tma.cuh"
#include "mr_gemv_v2.cuh"
#include "mr_gemv_umma.cuh"
#include "mr_gemm_umma.cuh"

namespace mr {

constexpr int kPrefetch = 4;  // groups of codes in flight per lane (register kernel)

// Register-streaming kernel (any in % 64 == 0).
cudaError_t launch_gemv_b2(const GemvParams& p, int sd, int epi, int nt, int grid, cudaStream_t s);
cudaError_t launch_gemv_b4(const GemvParams& p, int sd, int epi, int nt, int grid, cudaStream_t s);
cudaError_t launch_gemv_b8(const GemvParams& p, int sd, int epi, int nt, int grid, cudaStream_t s);
// TMA-pipelined persistent kernel (in % 512 == 0).
cudaError_t launch_tma_b2(const GemvParams& p, const TmaMaps& m, int sd, int epi, int nt, int grid,
                          cudaStream_t s);
cudaError_t launch_tma_b4(const GemvParams& p, const TmaMaps& m, int sd, int epi, int nt, int grid,
                          cudaStream_t s);
cudaError_t launch_tma_b8(const GemvParams& p, const TmaMaps& m, int sd, int epi, int nt, int grid,
                          cudaStream_t s);

// Staged-activation TMA kernel (in % 512 == 0, 2-D tensor-map stacks; nt = 1
// or 2 mma tiles of 8 columns per segment).
cudaError_t launch_v2_b2(const GemvParams& p, const TmaMaps& m, int sd, int epi, int nt, int grid,
                         cudaStream_t s);
cudaError_t launch_v2_b4(const GemvParams& p, const TmaMaps& m, int sd, int epi, int nt, int grid,
                         cudaStream_t s);
cudaError_t launch_v2_b8(const GemvParams& p, const TmaMaps& m, int sd, int epi, int nt, int grid,
                         cudaStream_t s);

inline cudaError_t launch_v2(const GemvParams& p, const TmaMaps& m, int bits, int sd, int epi,
                             int nt, int grid, cudaStream_t s) {
  switch (bits) {
    case 2: return launch_v2_b2(p, m, sd, epi, nt, grid, s);
    case 4: return launch_v2_b4(p, m, sd, epi, nt, grid, s);
    case 8: return launch_v2_b8(p, m, sd, epi, nt, grid, s);
    default: return cudaErrorInvalidValue;
  }
}

// MXFP4 form of the TMA kernel (in % 512 == 0, store epilogue, nt == 1);
// xs = 1: bf16 activations, xs = 2: fp32 activations as two f16 terms.
cudaError_t launch_tma_mx(const GemvParams& p, const TmaMaps& m, int nt, int xs, int grid,
                          cudaStream_t s);

// tcgen05 kernel (in % 512 == 0, activations through tensor maps).
cudaError_t launch_umma_b2(const GemvParams& p, const UmMaps& m, int sd, int epi, int grid,
                           cudaStream_t s);
cudaError_t launch_umma_b4(const GemvParams& p, const UmMaps& m, int sd, int epi, int grid,
                           cudaStream_t s);
cudaError_t launch_umma_b8(const GemvParams& p, const UmMaps& m, int sd, int epi, int grid,
                           cudaStream_t s);

inline cudaError_t launch_umma(const GemvParams& p, const UmMaps& m, int bits, int sd, int epi,
                               int grid, cudaStream_t s) {
  switch (bits) {
    case 2: return launch_umma_b2(p, m, sd, epi, grid, s);
    case 4: return launch_umma_b4(p, m, sd, epi, grid, s);
    case 8: return launch_umma_b8(p, m, sd, epi, grid, s);
    default: return cudaErrorInvalidValue;
  }
}

// tcgen05 prefill GEMM (4/8-bit, in % 256 == 0, activations through tensor maps).
cudaError_t launch_pf_b4(const GemvParams& p, const UmMaps& m, int sd, int epi, int grid,
                         cudaStream_t s);
cudaError_t launch_pf_b8(const GemvParams& p, const UmMaps& m, int sd, int epi, int grid,
                         cudaStream_t s);

inline cudaError_t launch_pf(const GemvParams& p, const UmMaps& m, int bits, int sd, int epi,
                             int grid, cudaStream_t s) {
  switch (bits) {
    case 4: return launch_pf_b4(p, m, sd, epi, grid, s);
    case 8: return launch_pf_b8(p, m, sd, epi, grid, s);
    default: return cudaErrorInvalidValue;
  }
}

inline cudaError_t launch_gemv(const GemvParams& p, int bits, int sd, int epi, int nt, int grid,
                               cudaStream_t s) {
  switch (bits) {
    case 2: return launch_gemv_b2(p, sd, epi, nt, grid, s);
    case 4: return launch_gemv_b4(p, sd, epi, nt, grid, s);
    case 8: return launch_gemv_b8(p, sd, epi, nt, grid, s);
    default: return cudaErrorInvalidValue;
  }
}

inline cudaError_t launch_tma(const GemvParams& p, const TmaMaps& m, int bits, int sd, int epi,
                              int nt, int grid, cudaStream_t s) {
  switch (bits) {
    case 2: return launch_tma_b2(p, m, sd, epi, nt, grid, s);
    case 4: return launch_tma_b4(p, m, sd, epi, nt, grid, s);
    case 8: return launch_tma_b8(p, m, sd, epi, nt, grid, s);
    default: return cudaErrorInvalidValue;
  }
}

// Columns per segment: one 8-column mma tile. An expert with more columns
// gets several segments (its weights are re-read, mostly from L2): measured
// on config 1 at T = 64, one tile per segment is 1.55x faster than two,
// because decode segments hold 1-4 columns and every mma.sync costs the same
// whatever the number of live columns.
inline int pick_seg_cols(int64_t max_cols) {
  (void)max_cols;
  return 8;
}

// Sets the dynamic shared-memory opt-in of `kernel` once per device; `done`
// must be owned by that one kernel.
template <class K>
inline cudaError_t opt_in_smem(K kernel, int bytes, bool (&done)[64]) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev >= 0 && dev < 64 && done[dev]) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess && dev >= 0 && dev < 64) done[dev] = true;
  return e;
}

template <int BITS, int SD, int EPI, int NT, int XS = 1>
inline cudaError_t launch_tma_inst(const GemvParams& p, const TmaMaps& m, int grid,
                                   cudaStream_t s) {
  static bool done[64] = {};  // one per instantiation
  const int nst = tma_stages<BITS, SD, EPI, NT>();
  const int smem = tma_smem_bytes<BITS, SD, EPI, NT>(nst);
  auto kern = gemv_tma_kernel<BITS, SD, EPI, NT, XS>;
  cudaError_t e = opt_in_smem(kern, smem, done);
  if (e != cudaSuccess) return e;
  return launch_pdl(kern, grid, kTmaThreads, smem, s, p, m, nst);
}

template <int BITS, int SD, int EPI, int NT, int MT, bool XH = false>
inline cudaError_t launch_v2_inst(const GemvParams& p, const TmaMaps& m, int grid,
                                  cudaStream_t s) {
  static bool done[64] = {};  // one per instantiation
  constexpr int RT = MT % kV2RT == 0 ? kV2RT : 1;
  const int nst = v2_stages<BITS, SD, EPI, NT, MT, XH>();
  const int smem = v2_smem_bytes<BITS, SD, EPI, NT, MT, XH>(nst);
  auto kern = gemv_v2_kernel<BITS, SD, EPI, NT, MT, XH, RT>;
  cudaError_t e = opt_in_smem(kern, smem, done);
  if (e != cudaSuccess) return e;
  return launch_pdl(kern, grid, v2_threads(RT), smem, s, p, m, nst);
}

template <int BITS, int SD, int EPI>
inline cudaError_t launch_umma_inst(const GemvParams& p, const UmMaps& m, int grid,
                                    cudaStream_t s) {
  static bool done[64] = {};  // one per instantiation
  const int nst = um_stages<BITS, SD, EPI>();
  const int smem = um_smem_bytes<BITS, SD, EPI>(nst);
  auto kern = gemv_umma_kernel<BITS, SD, EPI>;
  cudaError_t e = opt_in_smem(kern, smem, done);
  if (e != cudaSuccess) return e;
  kern<<<grid, kUmThreads, smem, s>>>(p, m, nst);
  return cudaGetLastError();
}

template <int BITS, int SD>
inline cudaError_t launch_umma_epi(const GemvParams& p, const UmMaps& m, int epi, int grid,
                                   cudaStream_t s) {
  switch (epi) {
    case EPI_STORE: return launch_umma_inst<BITS, SD, EPI_STORE>(p, m, grid, s);
    case EPI_SWIGLU: return launch_umma_inst<BITS, SD, EPI_SWIGLU>(p, m, grid, s);
    default: return launch_umma_inst<BITS, SD, EPI_PARTIAL>(p, m, grid, s);
  }
}

template <int BITS, int SD, int EPI>
inline cudaError_t launch_pf_inst(const GemvParams& p, const UmMaps& m, int grid,
                                  cudaStream_t s) {
  static bool done[64] = {};  // one per instantiation
  const int nst = pf_stages<BITS, SD, EPI>();
  const int smem = pf_smem_bytes<BITS, SD, EPI>(nst);
  auto kern = gemm_umma_kernel<BITS, SD, EPI>;
  cudaError_t e = opt_in_smem(kern, smem, done);
  if (e != cudaSuccess) return e;
  kern<<<grid, kPfThreads, smem, s>>>(p, m, nst);
  return cudaGetLastError();
}

template <int BITS, int SD>
inline cudaError_t launch_pf_epi(const GemvParams& p, const UmMaps& m, int epi, int grid,
                                 cudaStream_t s) {
  switch (epi) {
    case EPI_STORE: return launch_pf_inst<BITS, SD, EPI_STORE>(p, m, grid, s);
    case EPI_SWIGLU: return launch_pf_inst<BITS, SD, EPI_SWIGLU>(p, m, grid, s);
    default: return launch_pf_inst<BITS, SD, EPI_PARTIAL>(p, m, grid, s);
  }
}

}  // namespace mr

// Instantiates launch_pf_b<BITS> in a translation unit.
#define MR_DEFINE_PF_LAUNCHER(BITS)                                                           \
  namespace mr {                                                                              \
  cudaError_t launch_pf_b##BITS(const GemvParams& p, const UmMaps& m, int sd, int epi,        \
                                int grid, cudaStream_t s) {                                   \
    switch (sd) {                                                                             \
      case MR_DTYPE_BF16: return launch_pf_epi<BITS, MR_DTYPE_BF16>(p, m, epi, grid, s);      \
      case MR_DTYPE_F16: return launch_pf_epi<BITS, MR_DTYPE_F16>(p, m, epi, grid, s);        \
      default: return launch_pf_epi<BITS, MR_DTYPE_F32>(p, m, epi, grid, s);                  \
    }                                                                                         \
  }                                                                                           \
  }

// Instantiates launch_umma_b<BITS> in a translation unit.
#define MR_DEFINE_UMMA_LAUNCHER(BITS)                                                         \
  namespace mr {                                                                              \
  cudaError_t launch_umma_b##BITS(const GemvParams& p, const UmMaps& m, int sd, int epi,      \
                                  int grid, cudaStream_t s) {                                 \
    switch (sd) {                                                                             \
      case MR_DTYPE_BF16: return launch_umma_epi<BITS, MR_DTYPE_BF16>(p, m, epi, grid, s);    \
      case MR_DTYPE_F16: return launch_umma_epi<BITS, MR_DTYPE_F16>(p, m, epi, grid, s);      \
      default: return launch_umma_epi<BITS, MR_DTYPE_F32>(p, m, epi, grid, s);                \
    }                                                                                         \
  }                                                                                           \
  }

// Instantiates launch_gemv_b<BITS> and launch_tma_b<BITS> in a translation unit.
#define MR_DEFINE_GEMV_LAUNCHER(BITS)                                                          \
  namespace mr {                                                                               \
  template <int SD, int EPI>                                                                   \
  static cudaError_t launch_nt_##BITS(const GemvParams& p, int nt, int grid, cudaStream_t s) { \
    if (nt == 1)                                                                               \
      gemv_kernel<BITS, SD, EPI, 1, kPrefetch><<<grid, kGemvThreads, 0, s>>>(p);               \
    else                                                                                       \
      gemv_kernel<BITS, SD, EPI, 2, kPrefetch><<<grid, kGemvThreads, 0, s>>>(p);               \
    return cudaGetLastError();                                                                 \
  }                                                                                            \
  template <int SD, int EPI>                                                                   \
  static cudaError_t tma_nt_##BITS(const GemvParams& p, const TmaMaps& m, int nt, int grid,    \
                                   cudaStream_t s) {                                           \
    return nt == 1 ? launch_tma_inst<BITS, SD, EPI, 1>(p, m, grid, s)                          \
                   : launch_tma_inst<BITS, SD, EPI, 2>(p, m, grid, s);                         \
  }                                                                                            \
  template <int SD>                                                                            \
  static cudaError_t launch_epi_##BITS(const GemvParams& p, const TmaMaps* m, int epi, int nt, \
                                       int grid, cudaStream_t s) {                             \
    switch (epi) {                                                                             \
      case EPI_STORE:                                                                          \
        return m ? tma_nt_##BITS<SD, EPI_STORE>(p, *m, nt, grid, s)                            \
                 : launch_nt_##BITS<SD, EPI_STORE>(p, nt, grid, s);                            \
      case EPI_SWIGLU:                                                                         \
        return m ? tma_nt_##BITS<SD, EPI_SWIGLU>(p, *m, nt, grid, s)                           \
                 : launch_nt_##BITS<SD, EPI_SWIGLU>(p, nt, grid, s);                           \
      default:                                                                                 \
        return m ? tma_nt_##BITS<SD, EPI_PARTIAL>(p, *m, nt, grid, s)                          \
                 : launch_nt_##BITS<SD, EPI_PARTIAL>(p, nt, grid, s);                          \
    }                                                                                          \
  }                                                                                            \
  static cudaError_t dispatch_##BITS(const GemvParams& p, const TmaMaps* m, int sd, int epi,   \
                                     int nt, int grid, cudaStream_t s) {                       \
    switch (sd) {                                                                              \
      case MR_DTYPE_BF16: return launch_epi_##BITS<MR_DTYPE_BF16>(p, m, epi, nt, grid, s);     \
      case MR_DTYPE_F16: return launch_epi_##BITS<MR_DTYPE_F16>(p, m, epi, nt, grid, s);       \
      default: return launch_epi_##BITS<MR_DTYPE_F32>(p, m, epi, nt, grid, s);                 \
    }                                                                                          \
  }                                                                                            \
  cudaError_t launch_gemv_b##BITS(const GemvParams& p, int sd, int epi, int nt, int grid,      \
                                  cudaStream_t s) {                                            \
    return dispatch_##BITS(p, nullptr, sd, epi, nt, grid, s);                                  \
  }                                                                                            \
  cudaError_t launch_tma_b##BITS(const GemvParams& p, const TmaMaps& m, int sd, int epi,       \
                                 int nt, int grid, cudaStream_t s) {                           \
    return dispatch_##BITS(p, &m, sd, epi, nt, grid, s);                                       \
  }                                                                                            \
  template <int SD, int EPI, int MT>                                                           \
  static cudaError_t v2_mt_##BITS(const GemvParams& p, const TmaMaps& m, int nt, int grid,     \
                                  cudaStream_t s) {                                            \
    if constexpr (EPI != EPI_STORE && (BITS == 4 || BITS == 8)) {                              \
      if (p.x_f16)                                                                             \
        return nt == 1 ? launch_v2_inst<BITS, SD, EPI, 1, MT, true>(p, m, grid, s)             \
                       : launch_v2_inst<BITS, SD, EPI, 2, MT, true>(p, m, grid, s);            \
    }                                                                                          \
    if (p.x_f16) return cudaErrorInvalidValue;                                                 \
    return nt == 1 ? launch_v2_inst<BITS, SD, EPI, 1, MT>(p, m, grid, s)                       \
                   : launch_v2_inst<BITS, SD, EPI, 2, MT>(p, m, grid, s);                      \
  }                                                                                            \
  template <int SD, int EPI>                                                                   \
  static cudaError_t v2_nt_##BITS(const GemvParams& p, const TmaMaps& m, int nt, int grid,     \
                                  cudaStream_t s) {                                            \
    if constexpr (EPI == EPI_PARTIAL)                                                          \
      return v2_mt_##BITS<SD, EPI, v2_down_mt(BITS)>(p, m, nt, grid, s);                       \
    if constexpr (EPI == EPI_SWIGLU) {                                                         \
      if (v2_up_wide(BITS, p.rows)) return v2_mt_##BITS<SD, EPI, v2_up_mt(BITS)>(p, m, nt, grid, s); \
    }                                                                                          \
    return v2_mt_##BITS<SD, EPI, 4>(p, m, nt, grid, s);                                        \
  }                                                                                            \
  template <int SD>                                                                            \
  static cudaError_t v2_epi_##BITS(const GemvParams& p, const TmaMaps& m, int epi, int nt,     \
                                   int grid, cudaStream_t s) {                                 \
    switch (epi) {                                                                             \
      case EPI_STORE: return v2_nt_##BITS<SD, EPI_STORE>(p, m, nt, grid, s);                   \
      case EPI_SWIGLU: return v2_nt_##BITS<SD, EPI_SWIGLU>(p, m, nt, grid, s);                 \
      default: return v2_nt_##BITS<SD, EPI_PARTIAL>(p, m, nt, grid, s);                        \
    }                                                                                          \
  }                                                                                            \
  cudaError_t launch_v2_b##BITS(const GemvParams& p, const TmaMaps& m, int sd, int epi, int nt, \
                                int grid, cudaStream_t s) {                                    \
    switch (sd) {                                                                              \
      case MR_DTYPE_BF16: return v2_epi_##BITS<MR_DTYPE_BF16>(p, m, epi, nt, grid, s);         \
      case MR_DTYPE_F16: return v2_epi_##BITS<MR_DTYPE_F16>(p, m, epi, nt, grid, s);           \
      default: return v2_epi_##BITS<MR_DTYPE_F32>(p, m, epi, nt, grid, s);                     \
    }                                                                                          \
  }                                                                                            \
  }
