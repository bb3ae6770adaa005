// Single translation unit of libxp_cuda.so (kernels are defined in headers).
#include "capi.cuh"
#include "engine.cuh"
