// mr_gemm_b4.cu — 4-bit instantiations of the tcgen05 prefill GEMM.
#include "mr_launch.h"

MR_DEFINE_PF_LAUNCHER(4)
