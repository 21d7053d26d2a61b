// epilogue.cuh — the fused elementwise epilogue of the linear layer.
//
// In the reference the matmul and its elementwise linalg.generic (bias add,
// GELU-tanh, SiLU*mul, residual add, cast) are NOT fused: FusionPass only
// fuses producer/consumer pairs that are both all-parallel
// (lib/Conversion/LinalgToLLVM/FusionPass.cpp:163,176-179), so the epilogue
// is a second tiled loop nest over the stored C.  Here it runs on the fp32
// accumulator in registers, straight out of TMEM, before the single store.
//
// Math follows the reference's golden (PyTorch): F.gelu(approximate="tanh")
// (test/python/triton/test_gelu.py:72) and F.silu (test_silu.py:63), both
// evaluated in fp32 with CUDA's expf/tanhf.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "hx_gemm.h"

namespace hx {

struct EpiArgs {
  void *C;
  int64_t ldc;
  const void *bias;
  const void *residual;
  int64_t ldr;
  const void *scale;
  int32_t c_dtype, bias_dtype, scale_dtype, epi;
  int32_t M, N;        // output extent (columns of C)
  int32_t c_vec_ok;    // C rows are 16-byte aligned: vector stores allowed
  int32_t r_vec_ok;    // residual rows are 16-byte aligned
};

__device__ __forceinline__ float ld_as_float(const void *p, int dtype, int64_t i) {
  switch (dtype) {
    case HX_F16: return __half2float(static_cast<const __half *>(p)[i]);
    case HX_BF16: return __bfloat162float(static_cast<const __nv_bfloat16 *>(p)[i]);
    case HX_F32: return static_cast<const float *>(p)[i];
    case HX_S32: return static_cast<float>(static_cast<const int32_t *>(p)[i]);
    default: return 0.f;
  }
}

__device__ __forceinline__ float gelu_tanh(float x) {
  // 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3)))
  const float k0 = 0.7978845608028654f;
  const float k1 = 0.044715f;
  return 0.5f * x * (1.f + tanhf(k0 * (x + k1 * x * x * x)));
}
__device__ __forceinline__ float silu(float x) { return x / (1.f + expf(-x)); }

// Apply the epilogue to 32 consecutive output columns of one row.
//   v[j]   : accumulator for column n0 + j (gate half for SWIGLU)
//   up[j]  : "up" accumulator for SWIGLU (ignored otherwise)
__device__ __forceinline__ void epi_transform32(const EpiArgs &e, float (&v)[32],
                                                const float (&up)[32], int m, int n0) {
  const bool full = (n0 + 32 <= e.N);
  const int epi = e.epi;
  if (epi == HX_EPI_SWIGLU) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = silu(v[j]) * up[j];
    return;
  }
  if (epi == HX_EPI_DEQUANT_SCALE) {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int n = (full || n0 + j < e.N) ? n0 + j : e.N - 1;
      v[j] *= ld_as_float(e.scale, e.scale_dtype, n);
    }
  }
  const bool has_bias = e.bias != nullptr &&
                        (epi == HX_EPI_BIAS || epi == HX_EPI_BIAS_GELU_TANH ||
                         epi == HX_EPI_BIAS_RESIDUAL || epi == HX_EPI_DEQUANT_SCALE ||
                         epi == HX_EPI_BIAS_SILU);
  if (has_bias) {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int n = (full || n0 + j < e.N) ? n0 + j : e.N - 1;
      v[j] += ld_as_float(e.bias, e.bias_dtype, n);
    }
  }
  if ((epi == HX_EPI_BIAS_RESIDUAL || epi == HX_EPI_RESIDUAL) && e.residual != nullptr &&
      m < e.M) {
    const int64_t base = static_cast<int64_t>(m) * e.ldr + n0;
    if (full && e.r_vec_ok && (e.c_dtype == HX_F16 || e.c_dtype == HX_BF16)) {
      const uint4 *rp = reinterpret_cast<const uint4 *>(
          static_cast<const uint16_t *>(e.residual) + base);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint4 w = __ldg(rp + q);
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          float lo, hi;
          if (e.c_dtype == HX_F16) {
            const __half2 p = *reinterpret_cast<const __half2 *>(&ws[h]);
            lo = __low2float(p);
            hi = __high2float(p);
          } else {
            const __nv_bfloat162 p = *reinterpret_cast<const __nv_bfloat162 *>(&ws[h]);
            lo = __low2float(p);
            hi = __high2float(p);
          }
          v[q * 8 + h * 2] += lo;
          v[q * 8 + h * 2 + 1] += hi;
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (n0 + j < e.N) v[j] += ld_as_float(e.residual, e.c_dtype, base + j);
    }
  }
  if (epi == HX_EPI_BIAS_GELU_TANH) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = gelu_tanh(v[j]);
  } else if (epi == HX_EPI_BIAS_SILU) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = silu(v[j]);
  }
}

// Store 32 float values (or raw int32 bits) of row m, columns n0.. n0+31.
__device__ __forceinline__ void epi_store32(const EpiArgs &e, const float (&v)[32],
                                            const uint32_t (&raw)[32], bool raw_int, int m,
                                            int n0) {
  if (m >= e.M) return;
  const bool full = (n0 + 32 <= e.N);
  const int64_t base = static_cast<int64_t>(m) * e.ldc + n0;
  switch (e.c_dtype) {
    case HX_F16:
    case HX_BF16: {
      uint32_t pk[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        if (e.c_dtype == HX_F16) {
          __half2 h = __floats2half2_rn(v[2 * j], v[2 * j + 1]);
          pk[j] = *reinterpret_cast<uint32_t *>(&h);
        } else {
          __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
          pk[j] = *reinterpret_cast<uint32_t *>(&h);
        }
      }
      uint16_t *cp = static_cast<uint16_t *>(e.C) + base;
      if (full && e.c_vec_ok) {
        uint4 *dst = reinterpret_cast<uint4 *>(cp);
#pragma unroll
        for (int q = 0; q < 4; ++q)
          dst[q] = make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (n0 + j < e.N) cp[j] = static_cast<uint16_t>(pk[j >> 1] >> ((j & 1) * 16));
      }
      break;
    }
    case HX_F32:
    case HX_S32: {
      uint32_t w[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        if (e.c_dtype == HX_F32)
          w[j] = __float_as_uint(v[j]);
        else
          w[j] = raw_int ? raw[j] : static_cast<uint32_t>(__float2int_rn(v[j]));
      }
      uint32_t *cp = static_cast<uint32_t *>(e.C) + base;
      if (full && e.c_vec_ok) {
        uint4 *dst = reinterpret_cast<uint4 *>(cp);
#pragma unroll
        for (int q = 0; q < 8; ++q)
          dst[q] = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (n0 + j < e.N) cp[j] = w[j];
      }
      break;
    }
    default: break;
  }
}

// Scalar form used by the CUDA-core fallback kernel.
__device__ __forceinline__ float epi_scalar(const EpiArgs &e, float acc, float up, int m, int n) {
  const int epi = e.epi;
  if (epi == HX_EPI_SWIGLU) return silu(acc) * up;
  float v = acc;
  if (epi == HX_EPI_DEQUANT_SCALE) v *= ld_as_float(e.scale, e.scale_dtype, n);
  if (e.bias != nullptr &&
      (epi == HX_EPI_BIAS || epi == HX_EPI_BIAS_GELU_TANH || epi == HX_EPI_BIAS_RESIDUAL ||
       epi == HX_EPI_DEQUANT_SCALE || epi == HX_EPI_BIAS_SILU))
    v += ld_as_float(e.bias, e.bias_dtype, n);
  if ((epi == HX_EPI_BIAS_RESIDUAL || epi == HX_EPI_RESIDUAL) && e.residual != nullptr)
    v += ld_as_float(e.residual, e.c_dtype, static_cast<int64_t>(m) * e.ldr + n);
  if (epi == HX_EPI_BIAS_GELU_TANH) v = gelu_tanh(v);
  if (epi == HX_EPI_BIAS_SILU) v = silu(v);
  return v;
}

__device__ __forceinline__ void epi_store_scalar(const EpiArgs &e, float v, int32_t iv,
                                                 bool raw_int, int m, int n) {
  const int64_t i = static_cast<int64_t>(m) * e.ldc + n;
  switch (e.c_dtype) {
    case HX_F16: static_cast<__half *>(e.C)[i] = __float2half_rn(v); break;
    case HX_BF16: static_cast<__nv_bfloat16 *>(e.C)[i] = __float2bfloat16_rn(v); break;
    case HX_F32: static_cast<float *>(e.C)[i] = v; break;
    case HX_S32: static_cast<int32_t *>(e.C)[i] = raw_int ? iv : __float2int_rn(v); break;
    default: break;
  }
}

}  // namespace hx
