// Kernel instantiations for fp16 I/O.
#include "ss_launch.cuh"
SSB_INSTANTIATE(__half)
