// gemm_kind1.cu — tile-GEMM kernels and launchers for bf16 inputs.
#include "launch_impl.cuh"

HX_INSTANTIATE_KIND(1)
