// mr_gemv_b8.cu — 8-bit instantiations of the dequant-GEMV.
#include "mr_launch.h"

MR_DEFINE_GEMV_LAUNCHER(8)
