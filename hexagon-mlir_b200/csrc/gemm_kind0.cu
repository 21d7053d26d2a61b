// gemm_kind0.cu — tile-GEMM kernels and launchers for fp16 inputs.
#include "launch_impl.cuh"

HX_INSTANTIATE_KIND(0)
