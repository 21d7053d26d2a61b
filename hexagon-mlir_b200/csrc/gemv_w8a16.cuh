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

// Four int8 -> four fp32, exactly, with the magic-number method: flipping
// the sign bit maps v in [-128, 127] to u = v + 128 in [0, 255]; the fp32 bit
// pattern 0x4B000000 | u is exactly 2^23 + u, so subtracting 2^23 + 128
// leaves v.  One prmt places each byte under the 0x4B exponent byte.
__device__ __forceinline__ void i8x4_to_f32(uint32_t w, float (&f)[4]) {
  const uint32_t u = w ^ 0x80808080u;
  uint32_t b0, b1, b2, b3;
  asm("prmt.b32 %0, %1, %2, 0x7650;" : "=r"(b0) : "r"(u), "r"(0x4B000000u));
  asm("prmt.b32 %0, %1, %2, 0x7651;" : "=r"(b1) : "r"(u), "r"(0x4B000000u));
  asm("prmt.b32 %0, %1, %2, 0x7652;" : "=r"(b2) : "r"(u), "r"(0x4B000000u));
  asm("prmt.b32 %0, %1, %2, 0x7653;" : "=r"(b3) : "r"(u), "r"(0x4B000000u));
  const float k = 8388736.0f;  // 2^23 + 128
  f[0] = __uint_as_float(b0) - k;
  f[1] = __uint_as_float(b1) - k;
  f[2] = __uint_as_float(b2) - k;
  f[3] = __uint_as_float(b3) - k;
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


// 1-D bulk copy global -> shared completing on an mbarrier (16-byte aligned
// addresses, size a multiple of 16).

struct GemvStreamParams {
  GemvParams g;
  int32_t rows_per_cta;   // R in {8, 16, 32}
  int32_t weights_const;  // copy W before waiting on the previous kernel
  uint64_t timeout;
};

// Streaming W8A16 GEMV for M <= MC <= 8.  Each CTA (8 warps) owns R weight
// rows and copies all R x K int8 of them into shared memory with one bulk
// copy per row.  With weights_const the copies are issued before
// griddepcontrol.wait, so under programmatic dependent launch this
// kernel's weights stream from HBM while the previous kernel is still
// running; after the wait only x (L2-resident) is read.  Each warp computes
// R/8 rows x MC batch rows, lanes striding over K in 16-byte chunks, then a
// shuffle reduction; the per-channel scale (and bias) is applied once.
template <int MC>
__global__ void __launch_bounds__(256) hx_gemv_w8a16_stream_kernel(const GemvStreamParams sp) {
  const GemvParams &p = sp.g;
  extern __shared__ __align__(16) uint8_t wsm[];  // [R][K] int8, then the mbarrier
  const int R = sp.rows_per_cta;
  uint64_t *bar = reinterpret_cast<uint64_t *>(wsm + R * p.K);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = blockIdx.x * R;
  const int nrows = min(R, p.N - row0);
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  grid_dep_launch_dependents();
  auto issue = [&]() {
    if (threadIdx.x == 0) {
      mbar_arrive_expect_tx(bar, static_cast<uint32_t>(nrows) * p.K);
      for (int r = 0; r < nrows; ++r)
        bulk_load_1d(wsm + r * p.K, p.W + static_cast<int64_t>(row0 + r) * p.ldw, p.K, bar);
    }
  };
  if (sp.weights_const) issue();
  grid_dep_wait();
  if (!sp.weights_const) issue();
  int dummy_abort = 0;
  const bool have = mbar_wait(bar, 0, sp.timeout, &dummy_abort);

  const int rpw = R / 8;  // rows per warp (1, 2 or 4)
  float acc[4][MC];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int m = 0; m < MC; ++m) acc[i][m] = 0.f;
  const int kvec = p.K / 16;
  for (int kv = lane; kv < kvec; kv += 32) {
    float xf[MC][16];
#pragma unroll
    for (int m = 0; m < MC; ++m) {
      uint4 xa = make_uint4(0, 0, 0, 0), xb = make_uint4(0, 0, 0, 0);
      if (m < p.M) {
        const uint4 *xp = reinterpret_cast<const uint4 *>(p.x + m * p.ldx + kv * 16);
        xa = __ldg(xp);
        xb = __ldg(xp + 1);
      }
      const uint32_t xw[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
      for (int h = 0; h < 8; ++h) {
        const __half2 hv = *reinterpret_cast<const __half2 *>(&xw[h]);
        xf[m][2 * h] = __low2float(hv);
        xf[m][2 * h + 1] = __high2float(hv);
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (i >= rpw) break;
      const int r = warp * rpw + i;
      const uint4 wv = *reinterpret_cast<const uint4 *>(wsm + r * p.K + kv * 16);
      const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float f[4];
        i8x4_to_f32(ww[q], f);
#pragma unroll
        for (int m = 0; m < MC; ++m)
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[i][m] = fmaf(f[e], xf[m][q * 4 + e], acc[i][m]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (i >= rpw) break;
    const int r = warp * rpw + i;
#pragma unroll
    for (int m = 0; m < MC; ++m) {
      float v = acc[i][m];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      acc[i][m] = v;
    }
    if (lane == 0 && r < nrows && have) {
      const int n = row0 + r;
      const float sc = __half2float(p.scale[n]);
      const float b = p.bias ? __half2float(p.bias[n]) : 0.f;
#pragma unroll
      for (int m = 0; m < MC; ++m)
        if (m < p.M) p.y[m * p.ldy + n] = __float2half_rn(acc[i][m] * sc + b);
    }
  }
}

}  // namespace hx
