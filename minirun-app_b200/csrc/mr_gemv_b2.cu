// mr_gemv_b2.cu — 2-bit instantiations of the dequant-GEMV.
#include "mr_launch.h"

MR_DEFINE_GEMV_LAUNCHER(2)
