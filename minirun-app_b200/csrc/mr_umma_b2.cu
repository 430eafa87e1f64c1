// mr_umma_b2.cu — 2-bit instantiations of the tcgen05 dequant-GEMV.
#include "mr_launch.h"

MR_DEFINE_UMMA_LAUNCHER(2)
