// mr_gemm_b8.cu — 8-bit instantiations of the tcgen05 prefill GEMM.
#include "mr_launch.h"

MR_DEFINE_PF_LAUNCHER(8)
