// mr_umma_b8.cu — 8-bit instantiations of the tcgen05 dequant-GEMV.
#include "mr_launch.h"

MR_DEFINE_UMMA_LAUNCHER(8)
