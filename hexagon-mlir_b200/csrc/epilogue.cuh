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
// evaluated in fp32 (CUDA's __expf; GELU through an exact identity below).
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
  int32_t b_vec_ok;    // bias is 16-byte aligned
  int32_t s_vec_ok;    // scale is 16-byte aligned
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

// GELU-tanh through the identity 0.5 * (1 + tanh(y)) = 1 / (1 + exp(-2y)):
//   gelu_tanh(x) = x / (1 + exp(-2 * sqrt(2/pi) * (x + 0.044715 x^3)))
// which needs one exponential (CUDA's __expf) and one fast division.
__device__ __forceinline__ float gelu_tanh(float x) {
  const float k0x2 = 1.5957691216057308f;  // 2 * sqrt(2/pi)
  const float k1 = 0.044715f;
  const float y = k0x2 * fmaf(k1 * x, x * x, x);
  return __fdividef(x, 1.f + __expf(-y));
}
__device__ __forceinline__ float silu(float x) { return __fdividef(x, 1.f + __expf(-x)); }

// Load 32 consecutive elements v[j] = p[n0 + j] as float, j < 32 (columns
// >= N read as 0).  `vec_ok`: p is 16-byte aligned (n0 is a multiple of 32).
// COHERENT: read through L2 only (data another CTA of the same launch may
// have written); otherwise the read-only path.
template <bool COHERENT = false>
__device__ __forceinline__ void load_row32(const void *p, int dtype, int64_t base, int n0, int N,
                                           bool vec_ok, float (&v)[32]) {
  if (vec_ok && n0 + 32 <= N && (dtype == HX_F16 || dtype == HX_BF16)) {
    const uint4 *q = reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(p) + base + n0);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint4 w = COHERENT ? __ldcg(q + i) : __ldg(q + i);
      const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        if (dtype == HX_F16) {
          const __half2 t = *reinterpret_cast<const __half2 *>(&ws[h]);
          v[i * 8 + 2 * h] = __low2float(t);
          v[i * 8 + 2 * h + 1] = __high2float(t);
        } else {
          const __nv_bfloat162 t = *reinterpret_cast<const __nv_bfloat162 *>(&ws[h]);
          v[i * 8 + 2 * h] = __low2float(t);
          v[i * 8 + 2 * h + 1] = __high2float(t);
        }
      }
    }
    return;
  }
  if (vec_ok && n0 + 32 <= N && dtype == HX_F32) {
    const float4 *q = reinterpret_cast<const float4 *>(static_cast<const float *>(p) + base + n0);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 w = COHERENT ? __ldcg(q + i) : __ldg(q + i);
      v[4 * i] = w.x;
      v[4 * i + 1] = w.y;
      v[4 * i + 2] = w.z;
      v[4 * i + 3] = w.w;
    }
    return;
  }
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = (n0 + j < N) ? ld_as_float(p, dtype, base + n0 + j) : 0.f;
}

// Apply the epilogue to 32 consecutive output columns of one row.
//   v[j]   : accumulator for column n0 + j (gate half for SWIGLU)
//   up[j]  : "up" accumulator for SWIGLU (ignored otherwise)
// Every switch below is on a value uniform across the CTA; the per-element
// loops inside each case are straight-line code.
__device__ __forceinline__ void epi_transform32(const EpiArgs &e, float (&v)[32],
                                                const float (&up)[32], int m, int n0) {
  const int epi = e.epi;
  if (epi == HX_EPI_NONE) return;
  if (epi == HX_EPI_SWIGLU) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = silu(v[j]) * up[j];
    return;
  }
  float t[32];
  if (epi == HX_EPI_DEQUANT_SCALE) {
    load_row32(e.scale, e.scale_dtype, 0, n0, e.N, e.s_vec_ok, t);
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] *= t[j];
  }
  if (e.bias != nullptr && epi != HX_EPI_RESIDUAL) {
    load_row32(e.bias, e.bias_dtype, 0, n0, e.N, e.b_vec_ok, t);
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] += t[j];
  }
  if ((epi == HX_EPI_BIAS_RESIDUAL || epi == HX_EPI_RESIDUAL) && m < e.M) {
    load_row32<true>(e.residual, e.c_dtype, static_cast<int64_t>(m) * e.ldr, n0, e.N, e.r_vec_ok, t);
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] += t[j];
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
