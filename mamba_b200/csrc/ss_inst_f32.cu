// Kernel instantiations for fp32 I/O.
#include "ss_launch.cuh"
SSB_INSTANTIATE(float)
