// gemv_w8a16.cuh — memory-bound skinny-M W8A16 decode GEMM on CUDA cores.
//
// y[M,N] = x[M,K] . (W[N,K] * scale[N])^T (+ bias), W int8 per-output-channel
// quantised, x / y / scale fp16, fp32 accumulate.  The reference lowers
// quantised ops to dequantise-then-float-matmul
// (lib/Conversion/LinalgToLLVM/LinalgToLLVMPass.cpp:203-209) and turns a
// unit-M matvec into a dot reduction (ReduceContractionRankPass.cpp:38-47,
// split reduction TilingPass.cpp:266-279).  Here the weight stream is the
// whole cost: each warp streams ROWS weight rows with 128-bit loads, keeps
// the M activation rows in shared memory, reduces with warp shuffles and
// applies the per-channel scale once per output.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

#include "ptx.cuh"

namespace hx {

struct GemvParams {
  int32_t M, N, K;
  const __half *x;
  int64_t ldx;
  const int8_t *W;
  int64_t ldw;
  const __half *scale;
  const __half *bias;
  __half *y;
  int64_t ldy;
};

__device__ __forceinline__ void i8x4_to_f32(uint32_t w, float (&f)[4]) {
  f[0] = static_cast<float>(static_cast<int8_t>(w & 0xFF));
  f[1] = static_cast<float>(static_cast<int8_t>((w >> 8) & 0xFF));
  f[2] = static_cast<float>(static_cast<int8_t>((w >> 16) & 0xFF));
  f[3] = static_cast<float>(static_cast<int8_t>(w >> 24));
}

// Vector kernel: requires K % 16 == 0, ldw % 16 == 0, ldx % 8 == 0 and
// 16-byte aligned W / x.  Block = 4 warps; warp w owns ROWS consecutive rows.
// MC activation rows are processed per pass (M is looped in chunks of MC).
template <int ROWS, int MC>
__global__ void __launch_bounds__(128) hx_gemv_w8a16_kernel(const GemvParams p) {
  extern __shared__ __align__(16) __half xs[];  // [MC][K]
  grid_dep_launch_dependents();
  grid_dep_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = (blockIdx.x * 4 + warp) * ROWS;
  const int kvec = p.K / 16;
  for (int mc0 = 0; mc0 < p.M; mc0 += MC) {
    const int mcount = min(MC, p.M - mc0);
    __syncthreads();
    for (int i = threadIdx.x; i < MC * (p.K / 8); i += blockDim.x) {
      const int r = i / (p.K / 8), c = i % (p.K / 8);
      uint4 v = make_uint4(0, 0, 0, 0);
      if (r < mcount) v = *reinterpret_cast<const uint4 *>(p.x + (mc0 + r) * p.ldx + c * 8);
      reinterpret_cast<uint4 *>(xs + r * p.K)[c] = v;
    }
    __syncthreads();
    float acc[ROWS][MC];
#pragma unroll
    for (int r = 0; r < ROWS; ++r)
#pragma unroll
      for (int m = 0; m < MC; ++m) acc[r][m] = 0.f;
    for (int kv = lane; kv < kvec; kv += 32) {
      uint4 w[ROWS];
#pragma unroll
      for (int r = 0; r < ROWS; ++r) {
        const int n = min(row0 + r, p.N - 1);
        w[r] = __ldg(reinterpret_cast<const uint4 *>(p.W + n * p.ldw) + kv);
      }
#pragma unroll
      for (int m = 0; m < MC; ++m) {
        const uint4 *xp = reinterpret_cast<const uint4 *>(xs + m * p.K + kv * 16);
        const uint4 xa = xp[0], xb = xp[1];
        const uint32_t xw[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
        float xf[16];
#pragma unroll
        for (int h = 0; h < 8; ++h) {
          const __half2 hv = *reinterpret_cast<const __half2 *>(&xw[h]);
          xf[2 * h] = __low2float(hv);
          xf[2 * h + 1] = __high2float(hv);
        }
#pragma unroll
        for (int r = 0; r < ROWS; ++r) {
          const uint32_t ww[4] = {w[r].x, w[r].y, w[r].z, w[r].w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            float f[4];
            i8x4_to_f32(ww[q], f);
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[r][m] = fmaf(f[e], xf[q * 4 + e], acc[r][m]);
          }
        }
      }
    }
#pragma unroll
    for (int r = 0; r < ROWS; ++r)
#pragma unroll
      for (int m = 0; m < MC; ++m) {
        float v = acc[r][m];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        acc[r][m] = v;
      }
    if (lane == 0) {
#pragma unroll
      for (int r = 0; r < ROWS; ++r) {
        const int n = row0 + r;
        if (n >= p.N) continue;
        const float s = __half2float(p.scale[n]);
        const float b = p.bias ? __half2float(p.bias[n]) : 0.f;
#pragma unroll
        for (int m = 0; m < MC; ++m)
          if (m < mcount) p.y[(mc0 + m) * p.ldy + n] = __float2half_rn(acc[r][m] * s + b);
      }
    }
  }
}

// Scalar kernel for unaligned shapes: one warp per (m, n) output.
__global__ void __launch_bounds__(128) hx_gemv_w8a16_scalar_kernel(const GemvParams p) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const int64_t total = static_cast<int64_t>(p.M) * p.N;
  if (warp >= total) return;
  const int m = warp / p.N, n = warp % p.N;
  float acc = 0.f;
  for (int k = lane; k < p.K; k += 32)
    acc = fmaf(static_cast<float>(p.W[n * p.ldw + k]), __half2float(p.x[m * p.ldx + k]), acc);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) {
    const float b = p.bias ? __half2float(p.bias[n]) : 0.f;
    p.y[m * p.ldy + n] = __float2half_rn(acc * __half2float(p.scale[n]) + b);
  }
}

}  // namespace hx
