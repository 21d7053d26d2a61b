// gemm_simt.cuh — CUDA-core GEMM for shapes the TMA path cannot take
// (row strides or base pointers that are not 16-byte aligned, K = 0).
//
// This is the analogue of the reference's remainder handling when a tile
// does not divide the problem (lib/Transforms/TilingPass.cpp:170-246): it is
// still device code, fed from the same descriptor and the same fused
// epilogue, and it is never a host fallback.  It also serves as an
// independent second kernel in the tests.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <type_traits>

#include "epilogue.cuh"

namespace hx {

struct SimtParams {
  int32_t M, N, K;
  const void *A;
  int64_t lda;
  const void *B;
  int64_t ldb;
  int32_t ab_dtype;     // HX_F16 | HX_BF16 | HX_S8
  int32_t b_kn;         // 1: B[K,N]; 0: W[N,K]
  int32_t n_half;       // SWIGLU: first row of the "up" half of W
  EpiArgs epi;
};

__device__ __forceinline__ float ld_ab(const void *p, int dtype, int64_t i) {
  switch (dtype) {
    case HX_F16: return __half2float(static_cast<const __half *>(p)[i]);
    case HX_BF16: return __bfloat162float(static_cast<const __nv_bfloat16 *>(p)[i]);
    case HX_S8: return static_cast<float>(static_cast<const int8_t *>(p)[i]);
    default: return 0.f;
  }
}

constexpr int kSimtTile = 64;
constexpr int kSimtBK = 16;

// 64x64 output tile per 256-thread block; each thread owns a 4x4 patch.
// ACC = float for f16/bf16 (fp32 accumulate), int for s8 (exact int32).
template <typename ACC, bool SWIGLU>
__global__ void __launch_bounds__(256) hx_gemm_simt_kernel(const SimtParams p) {
  __shared__ ACC sA[kSimtBK][kSimtTile + 1];
  __shared__ ACC sB[kSimtBK][kSimtTile + 1];
  __shared__ ACC sU[SWIGLU ? kSimtBK : 1][SWIGLU ? kSimtTile + 1 : 1];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int m0 = blockIdx.y * kSimtTile, n0 = blockIdx.x * kSimtTile;
  ACC acc[4][4] = {};
  ACC accu[4][4] = {};
  for (int k0 = 0; k0 < p.K; k0 += kSimtBK) {
    for (int i = threadIdx.x; i < kSimtBK * kSimtTile; i += 256) {
      const int kk = i % kSimtBK, r = i / kSimtBK;
      const int m = m0 + r, k = k0 + kk;
      sA[kk][r] = (m < p.M && k < p.K) ? static_cast<ACC>(ld_ab(p.A, p.ab_dtype, m * p.lda + k))
                                       : ACC(0);
      const int n = n0 + r;
      ACC bv = ACC(0), uv = ACC(0);
      if (n < p.N && k < p.K) {
        if (p.b_kn)
          bv = static_cast<ACC>(ld_ab(p.B, p.ab_dtype, static_cast<int64_t>(k) * p.ldb + n));
        else
          bv = static_cast<ACC>(ld_ab(p.B, p.ab_dtype, static_cast<int64_t>(n) * p.ldb + k));
        if (SWIGLU)
          uv = static_cast<ACC>(
              ld_ab(p.B, p.ab_dtype, static_cast<int64_t>(p.n_half + n) * p.ldb + k));
      }
      sB[kk][r] = bv;
      if (SWIGLU) sU[kk][r] = uv;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kSimtBK; ++kk) {
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          acc[i][j] += sA[kk][ty * 4 + i] * sB[kk][tx * 4 + j];
          if (SWIGLU) accu[i][j] += sA[kk][ty * 4 + i] * sU[kk][tx * 4 + j];
        }
    }
    __syncthreads();
  }
  constexpr bool kIntAcc = std::is_same<ACC, int>::value;
  const bool raw_int = kIntAcc && p.epi.c_dtype == HX_S32 && p.epi.epi == HX_EPI_NONE;
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int m = m0 + ty * 4 + i, n = n0 + tx * 4 + j;
      if (m < p.M && n < p.N) {
        const float v = raw_int ? 0.f
                                : epi_scalar(p.epi, static_cast<float>(acc[i][j]),
                                             static_cast<float>(accu[i][j]), m, n);
        epi_store_scalar(p.epi, v, static_cast<int32_t>(acc[i][j]), raw_int, m, n);
      }
    }
}

}  // namespace hx
