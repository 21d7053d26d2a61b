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
// evaluated in fp32.  For fp32 outputs through CUDA's __expf (GELU via an
// exact identity below); for 16-bit outputs through the hardware tanh.approx
// (relative error about 2^-11, below half an fp16 ulp of the result scale),
// one special-function op per element instead of two.
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
  int32_t n_peers;     // > 0: every stored chunk also goes to peer_C[0..n_peers)
  void *peer_C[7];     //   (other GPUs' buffers, same offsets and ldc as C)
  int32_t pre16;       // every operand the epilogue reads (scale, bias,
                       // residual) is 16-bit and 16-byte aligned: full
                       // 32-column chunks may be prefetched raw (Pre16)
  // A normalisation of the rows of A folded into this GEMM (0 = none,
  // 1 + HX_NORM_LAYER / HX_NORM_RMS): before the rest of the epilogue,
  // acc = acc * rstd[m] - rstd[m] * mean[m] * col_sum[n] (the second term for
  // LayerNorm only; SWIGLU: col_sum[N + n] for the up half).
  int32_t norm;
  const float *row_stats;  // [M][2]: mean, rstd
  const float *col_sum;    // [N] (SWIGLU: [2N]) row sums of the folded weight
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

__device__ __forceinline__ float tanh_hw(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// 0.5 x (1 + tanh(y)) with one hardware tanh (16-bit outputs).
__device__ __forceinline__ float gelu_tanh_hw(float x) {
  const float k0 = 0.7978845608028654f;  // sqrt(2/pi)
  const float k1 = 0.044715f;
  const float hx = 0.5f * x;
  return fmaf(hx, tanh_hw(k0 * fmaf(k1 * x, x * x, x)), hx);
}
// x * sigmoid(x) = 0.5 x (1 + tanh(x / 2)).
__device__ __forceinline__ float silu_hw(float x) {
  const float hx = 0.5f * x;
  return fmaf(hx, tanh_hw(hx), hx);
}

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

// Final activation of BIAS_GELU_TANH / BIAS_SILU (identity otherwise).
__device__ __forceinline__ void epi_activate32(const EpiArgs &e, float (&v)[32]) {
  const bool hw = (e.c_dtype != HX_F32);
  if (e.epi == HX_EPI_BIAS_GELU_TANH) {
    if (hw) {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = gelu_tanh_hw(v[j]);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = gelu_tanh(v[j]);
    }
  } else if (e.epi == HX_EPI_BIAS_SILU) {
    if (hw) {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = silu_hw(v[j]);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = silu(v[j]);
    }
  }
}

__device__ __forceinline__ void swiglu32(const EpiArgs &e, float (&v)[32], const float (&up)[32]) {
  if (e.c_dtype != HX_F32) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = silu_hw(v[j]) * up[j];
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = silu(v[j]) * up[j];
  }
}

// Raw 16-bit operands of one full 32-column chunk, loaded ahead of the
// accumulator so their global-memory latency overlaps other work.
//   a: scale (DEQUANT_SCALE) or bias;   b: bias (DEQUANT_SCALE) or residual row
struct Pre16 {
  uint4 a[4];
  uint4 b[4];
};

template <bool COHERENT>
__device__ __forceinline__ void ld_raw16x32(const void *p, int64_t off, uint4 (&w)[4]) {
  const uint4 *q = reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(p) + off);
#pragma unroll
  for (int i = 0; i < 4; ++i) w[i] = COHERENT ? __ldcg(q + i) : __ldg(q + i);
}

__device__ __forceinline__ void raw16_to_f32(const uint4 (&w)[4], int dtype, float (&t)[32]) {
  if (dtype == HX_F16) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t ws[4] = {w[i].x, w[i].y, w[i].z, w[i].w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const __half2 x = *reinterpret_cast<const __half2 *>(&ws[h]);
        t[i * 8 + 2 * h] = __low2float(x);
        t[i * 8 + 2 * h + 1] = __high2float(x);
      }
    }
  } else {  // bf16: the value is the upper half of an fp32
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t ws[4] = {w[i].x, w[i].y, w[i].z, w[i].w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        t[i * 8 + 2 * h] = __uint_as_float(ws[h] << 16);
        t[i * 8 + 2 * h + 1] = __uint_as_float(ws[h] & 0xffff0000u);
      }
    }
  }
}

// The residual chunk of a warp's 32 rows, loaded coalesced: lane l holds
// rows i * 8 + l / 4 (i < 4), 16-byte column chunk l % 4 — whole 64-byte row
// segments per instruction.  residual_to_rows() transposes it through the
// warp's staging buffer to one row per lane.  Rows >= M read as zero.
__device__ __forceinline__ void ld_residual_coalesced(const EpiArgs &e, int m, int n0, uint4 (&w)[4]) {
  const int lane = threadIdx.x & 31;
  const int m0 = m - lane;
  const uint16_t *base = static_cast<const uint16_t *>(e.residual) + n0 + (lane & 3) * 8;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = i * 8 + (lane >> 2);
    w[i] = (m0 + r < e.M) ? __ldcg(reinterpret_cast<const uint4 *>(base + static_cast<int64_t>(m0 + r) * e.ldr))
                          : make_uint4(0u, 0u, 0u, 0u);
  }
}

__device__ __forceinline__ void residual_to_rows(const uint4 (&w)[4], uint8_t *stg, uint4 (&row)[4]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = i * 8 + (lane >> 2), q = lane & 3;
    *reinterpret_cast<uint4 *>(stg + r * 64 + ((q ^ ((r >> 1) & 3)) << 4)) = w[i];
  }
  __syncwarp();
  const int sw = (lane >> 1) & 3;
#pragma unroll
  for (int q = 0; q < 4; ++q) row[q] = *reinterpret_cast<const uint4 *>(stg + lane * 64 + ((q ^ sw) << 4));
  __syncwarp();  // stg is free again
}

// Valid when e.pre16 and n0 + 32 <= e.N.
__device__ __forceinline__ void epi_prefetch16(const EpiArgs &e, int m, int n0, Pre16 &f) {
  const int epi = e.epi;
  if (epi == HX_EPI_NONE || epi == HX_EPI_SWIGLU) return;
  const bool residual = (epi == HX_EPI_BIAS_RESIDUAL || epi == HX_EPI_RESIDUAL);
  if (epi == HX_EPI_DEQUANT_SCALE)
    ld_raw16x32<false>(e.scale, n0, f.a);
  else if (e.bias != nullptr && epi != HX_EPI_RESIDUAL)
    ld_raw16x32<false>(e.bias, n0, f.a);
  if (epi == HX_EPI_DEQUANT_SCALE && e.bias != nullptr)
    ld_raw16x32<false>(e.bias, n0, f.b);
  else if (residual)
    ld_residual_coalesced(e, m, n0, f.b);  // warp-collective
}

// Compile-time specialised epilogue of one full 32-column chunk on
// prefetched operands (valid when e.pre16): EPI is the epilogue, CT the
// output dtype.  The hot loop instantiates exactly one of these, so its
// instruction footprint holds only the path that runs.
template <int EPI>
__device__ __forceinline__ void epi_prefetch_t(const EpiArgs &e, int m, int n0, Pre16 &f) {
  if constexpr (EPI == HX_EPI_DEQUANT_SCALE) {
    ld_raw16x32<false>(e.scale, n0, f.a);
    if (e.bias != nullptr) ld_raw16x32<false>(e.bias, n0, f.b);
  } else if constexpr (EPI == HX_EPI_BIAS || EPI == HX_EPI_BIAS_GELU_TANH ||
                       EPI == HX_EPI_BIAS_SILU || EPI == HX_EPI_BIAS_RESIDUAL) {
    if (e.bias != nullptr) ld_raw16x32<false>(e.bias, n0, f.a);
  }
  if constexpr (EPI == HX_EPI_BIAS_RESIDUAL || EPI == HX_EPI_RESIDUAL) {
    ld_residual_coalesced(e, m, n0, f.b);
  }
}

template <int EPI, int CT>
__device__ __forceinline__ void epi_apply_t(const EpiArgs &e, float (&v)[32], const float (&up)[32],
                                            int m, const Pre16 &f, uint8_t *stg) {
  constexpr bool kHw = (CT != HX_F32);  // hardware tanh for 16-bit outputs
  if constexpr (EPI == HX_EPI_SWIGLU) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = (kHw ? silu_hw(v[j]) : silu(v[j])) * up[j];
  } else if constexpr (EPI != HX_EPI_NONE) {
    float t[32];
    if constexpr (EPI == HX_EPI_DEQUANT_SCALE) {
      raw16_to_f32(f.a, e.scale_dtype, t);
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] *= t[j];
      if (e.bias != nullptr) {
        raw16_to_f32(f.b, e.bias_dtype, t);
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] += t[j];
      }
    } else {
      if constexpr (EPI != HX_EPI_RESIDUAL) {
        if (e.bias != nullptr) {
          raw16_to_f32(f.a, e.bias_dtype, t);
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] += t[j];
        }
      }
      if constexpr (EPI == HX_EPI_BIAS_RESIDUAL || EPI == HX_EPI_RESIDUAL) {
        uint4 rrow[4];
        residual_to_rows(f.b, stg, rrow);
        raw16_to_f32(rrow, CT, t);
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] += t[j];
      }
      if constexpr (EPI == HX_EPI_BIAS_GELU_TANH) {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = kHw ? gelu_tanh_hw(v[j]) : gelu_tanh(v[j]);
      } else if constexpr (EPI == HX_EPI_BIAS_SILU) {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = kHw ? silu_hw(v[j]) : silu(v[j]);
      }
    }
  }
}

// Apply the epilogue to 32 consecutive output columns of one row.
//   v[j]   : accumulator for column n0 + j (gate half for SWIGLU)
//   up[j]  : "up" accumulator for SWIGLU (ignored otherwise)
// Every switch below is on a value uniform across the CTA; the per-element
// loops inside each case are straight-line code.
// The folded row normalisation of one 32-column chunk (e.norm != 0).
__device__ __forceinline__ void epi_norm32(const EpiArgs &e, float (&v)[32], float (&up)[32], int m, int n0) {
  if (m >= e.M) return;
  const float2 st = reinterpret_cast<const float2 *>(e.row_stats)[m];
  const float rstd = st.y;
  if (e.norm == 1 + HX_NORM_RMS) {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      v[j] *= rstd;
      up[j] *= rstd;
    }
    return;
  }
  const float shift = rstd * st.x;
  const bool sw = e.epi == HX_EPI_SWIGLU;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const int n = n0 + j;
    const float cs = n < e.N ? e.col_sum[n] : 0.f;
    v[j] = v[j] * rstd - shift * cs;
    if (sw) up[j] = up[j] * rstd - shift * (n < e.N ? e.col_sum[e.N + n] : 0.f);
  }
}

__device__ __forceinline__ void epi_transform32(const EpiArgs &e, float (&v)[32],
                                                float (&up)[32], int m, int n0) {
  if (e.norm) epi_norm32(e, v, up, m, n0);
  const int epi = e.epi;
  if (epi == HX_EPI_NONE) return;
  if (epi == HX_EPI_SWIGLU) {
    swiglu32(e, v, up);
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
  epi_activate32(e, v);
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
      for (int tgt = -1; tgt < e.n_peers; ++tgt) {  // C, then the peers' copies
        uint16_t *cp = static_cast<uint16_t *>(tgt < 0 ? e.C : e.peer_C[tgt]) + base;
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
      for (int tgt = -1; tgt < e.n_peers; ++tgt) {  // C, then the peers' copies
        uint32_t *cp = static_cast<uint32_t *>(tgt < 0 ? e.C : e.peer_C[tgt]) + base;
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
      }
      break;
    }
    default: break;
  }
}

// Scalar form used by the CUDA-core fallback kernel.
__device__ __forceinline__ float epi_scalar(const EpiArgs &e, float acc, float up, int m, int n) {
  const int epi = e.epi;
  if (e.norm && m < e.M) {
    const float2 st = reinterpret_cast<const float2 *>(e.row_stats)[m];
    acc *= st.y;
    up *= st.y;
    if (e.norm == 1 + HX_NORM_LAYER) {
      acc -= st.y * st.x * e.col_sum[n];
      if (epi == HX_EPI_SWIGLU) up -= st.y * st.x * e.col_sum[e.N + n];
    }
  }
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


// Store (to C only) of one full 32-column chunk for a whole warp through its 4 KB
// staging buffer `stg`: each thread parks its row segment in shared memory,
// then the warp writes 8 rows x 64 B (16-bit C) or 4 rows x 128 B (32-bit C)
// per store instruction instead of 32 rows x 16 B.  The 16-byte chunks of a
// row are XOR-swizzled by row so both shared-memory phases are free of bank
// conflicts.  All 32 lanes call it with the same n0 and m0 = the warp's first
// row; requires e.c_vec_ok and n0 + 32 <= e.N.  RAW: v is ignored and the
// int32 bits in raw are stored.
template <int CT, bool RAW>
__device__ __forceinline__ void epi_store32_staged_t(const EpiArgs &e, const float (&v)[32],
                                                     const uint32_t (&raw)[32], int m0, int n0,
                                                     uint8_t *stg) {
  const int lane = threadIdx.x & 31;
  if constexpr (CT == HX_F16 || CT == HX_BF16) {
    uint32_t pk[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      if constexpr (CT == HX_F16) {
        __half2 h = __floats2half2_rn(v[2 * j], v[2 * j + 1]);
        pk[j] = *reinterpret_cast<uint32_t *>(&h);
      } else {
        __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
        pk[j] = *reinterpret_cast<uint32_t *>(&h);
      }
    }
    uint8_t *row = stg + lane * 64;
    const int sw = (lane >> 1) & 3;
#pragma unroll
    for (int q = 0; q < 4; ++q)
      *reinterpret_cast<uint4 *>(row + ((q ^ sw) << 4)) =
          make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
    __syncwarp();
    const int qq = lane & 3;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = i * 8 + (lane >> 2);
      const uint4 x = *reinterpret_cast<const uint4 *>(stg + r * 64 + ((qq ^ ((r >> 1) & 3)) << 4));
      if (m0 + r < e.M) {
        const int64_t off = static_cast<int64_t>(m0 + r) * e.ldc + n0 + qq * 8;
        *reinterpret_cast<uint4 *>(static_cast<uint16_t *>(e.C) + off) = x;
      }
    }
  } else {
    uint32_t w[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if constexpr (RAW)
        w[j] = raw[j];
      else if constexpr (CT == HX_F32)
        w[j] = __float_as_uint(v[j]);
      else
        w[j] = static_cast<uint32_t>(__float2int_rn(v[j]));
    }
    uint8_t *row = stg + lane * 128;
    const int sw = lane & 7;
#pragma unroll
    for (int q = 0; q < 8; ++q)
      *reinterpret_cast<uint4 *>(row + ((q ^ sw) << 4)) =
          make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
    __syncwarp();
    const int qq = lane & 7;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int r = i * 4 + (lane >> 3);
      const uint4 x = *reinterpret_cast<const uint4 *>(stg + r * 128 + ((qq ^ (r & 7)) << 4));
      if (m0 + r < e.M) {
        const int64_t off = static_cast<int64_t>(m0 + r) * e.ldc + n0 + qq * 4;
        *reinterpret_cast<uint4 *>(static_cast<uint32_t *>(e.C) + off) = x;
      }
    }
  }
  __syncwarp();  // the next chunk may overwrite stg
}


// Staged store of one full 32-column chunk to C and to every peer copy
// (fused all-gather), for a whole warp; runtime output dtype.  The row
// segments leave as whole 64 / 128-byte pieces, which matters more over
// NVLink than locally.  Same preconditions as epi_store32_staged_t.
inline __device__ __noinline__ void epi_store32_staged_all(const EpiArgs &e, const float (&v)[32],
                                                    const uint32_t (&raw)[32], bool raw_int, int m0,
                                                    int n0, uint8_t *stg) {
  const int lane = threadIdx.x & 31;
  const bool b16 = (e.c_dtype == HX_F16 || e.c_dtype == HX_BF16);
  uint32_t w[32];
  if (b16) {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      if (e.c_dtype == HX_F16) {
        __half2 h = __floats2half2_rn(v[2 * j], v[2 * j + 1]);
        w[j] = *reinterpret_cast<uint32_t *>(&h);
      } else {
        __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
        w[j] = *reinterpret_cast<uint32_t *>(&h);
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      w[j] = raw_int ? raw[j]
                     : (e.c_dtype == HX_F32 ? __float_as_uint(v[j]) : static_cast<uint32_t>(__float2int_rn(v[j])));
  }
  const int row_bytes = b16 ? 64 : 128;     // bytes of the chunk in one row
  const int cpr = row_bytes / 16;           // 16-byte pieces per row
  const int esz = b16 ? 2 : 4;
  uint8_t *row = stg + lane * row_bytes;
  for (int q = 0; q < cpr; ++q) {
    const int sw = b16 ? ((lane >> 1) & 3) : (lane & 7);
    *reinterpret_cast<uint4 *>(row + ((q ^ sw) << 4)) = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
  }
  __syncwarp();
  const int rpi = 32 / cpr;  // rows per warp instruction
  const int qq = lane % cpr;
  for (int i = 0; i < cpr; ++i) {
    const int r = i * rpi + lane / cpr;
    const int sw = b16 ? ((r >> 1) & 3) : (r & 7);
    const uint4 x = *reinterpret_cast<const uint4 *>(stg + r * row_bytes + ((qq ^ sw) << 4));
    if (m0 + r < e.M) {
      const int64_t off = (static_cast<int64_t>(m0 + r) * e.ldc + n0) * esz + qq * 16;
      *reinterpret_cast<uint4 *>(static_cast<uint8_t *>(e.C) + off) = x;
      for (int t = 0; t < e.n_peers; ++t)
        *reinterpret_cast<uint4 *>(static_cast<uint8_t *>(e.peer_C[t]) + off) = x;
    }
  }
  __syncwarp();  // the next chunk may overwrite stg
}

}  // namespace hx
