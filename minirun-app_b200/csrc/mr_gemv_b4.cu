// mr_gemv_b4.cu — 4-bit instantiations of the dequant-GEMV.
#include "mr_launch.h"

MR_DEFINE_GEMV_LAUNCHER(4)
