// gemm_kind2.cu — tile-GEMM kernels and launchers for int8 inputs.
#include "launch_impl.cuh"

HX_INSTANTIATE_KIND(2)
