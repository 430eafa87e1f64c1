// mr_umma_b4.cu — 4-bit instantiations of the tcgen05 dequant-GEMV.
#include "mr_launch.h"

MR_DEFINE_UMMA_LAUNCHER(4)
