// Kernel instantiations for bf16 I/O.
#include "ss_launch.cuh"
SSB_INSTANTIATE(__nv_bfloat16)
