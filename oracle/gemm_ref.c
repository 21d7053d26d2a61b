/*
 * gemm_ref.c - plain-C CPU oracle of the linear-layer GEMM path.
 * TEST INFRASTRUCTURE ONLY: loaded by tests/ (ctypes) as a second,
 * independent checker beside oracle/gemm_oracle.py; never by the product.
 *
 * Restates, in C, the reference's CPU check of its HMX matmul
 * (test/python/mlir/hexkl_linalg_matmul/wrapper.cpp:47-66): for every
 * output, a float accumulator summing (float)act[row,k] * (float)W[k,col]
 * over k in order.  Here the same loop covers both B layouts, bf16 as well
 * as f16 operands, the fused epilogues the GPU kernels implement (bias,
 * GELU-tanh, SiLU, residual, SwiGLU, per-channel scale; PyTorch's formulas,
 * test/python/triton/test_gelu.py:72, test_silu.py:63), and the exact int32
 * product of int8 operands.  Half/bfloat16 decoding is by bit manipulation.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#define REF_BF16 1
#define REF_B_NK 0
#define EPI_BIAS 1
#define EPI_BIAS_GELU_TANH 2
#define EPI_BIAS_RESIDUAL 3
#define EPI_RESIDUAL 4
#define EPI_SWIGLU 5
#define EPI_DEQUANT_SCALE 6
#define EPI_BIAS_SILU 7

static float bits_to_f32(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* IEEE binary16 -> binary32 (exact). */
float hx_ref_f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h >> 15) << 31;
  uint32_t exp = (h >> 10) & 0x1F;
  uint32_t man = h & 0x3FF;
  if (exp == 0) {
    if (man == 0) return bits_to_f32(sign);
    float v = (float)man * 5.9604644775390625e-08f; /* man * 2^-24 */
    return sign ? -v : v;
  }
  if (exp == 31) return bits_to_f32(sign | 0x7F800000u | (man << 13));
  return bits_to_f32(sign | ((exp + 112) << 23) | (man << 13));
}

/* bfloat16 -> binary32: the upper half of the float's bits (exact). */
float hx_ref_bf16_to_f32(uint16_t b) { return bits_to_f32((uint32_t)b << 16); }

static float load16(const uint16_t *p, int dtype, int64_t i) {
  return dtype == REF_BF16 ? hx_ref_bf16_to_f32(p[i]) : hx_ref_f16_to_f32(p[i]);
}

static float gelu_tanh(float x) {
  return 0.5f * x * (1.0f + tanhf(0.7978845608028654f * (x + 0.044715f * x * x * x)));
}
static float silu(float x) { return x / (1.0f + expf(-x)); }

/* C[M,N] (f32) = epilogue(A[M,K] . B), fp32 accumulation in k order.
   bias/scale: [N] f32 or NULL; residual: [M,N] f32 or NULL.
   SWIGLU: B is W[2N,K] = [gate; up]. */
void hx_ref_gemm(int64_t M, int64_t N, int64_t K, const uint16_t *A, const uint16_t *B,
                 int dtype, int b_layout, int epilogue, const float *bias, const float *residual,
                 const float *scale, float *C) {
  for (int64_t m = 0; m < M; ++m) {
    for (int64_t n = 0; n < N; ++n) {
      float acc = 0.0f, up = 0.0f;
      for (int64_t k = 0; k < K; ++k) {
        float a = load16(A, dtype, m * K + k);
        float b = b_layout == REF_B_NK ? load16(B, dtype, n * K + k) : load16(B, dtype, k * N + n);
        acc += a * b;
        if (epilogue == EPI_SWIGLU) up += a * load16(B, dtype, (N + n) * K + k);
      }
      float v = acc;
      switch (epilogue) {
        case EPI_SWIGLU: v = silu(acc) * up; break;
        case EPI_DEQUANT_SCALE: v = acc * scale[n] + (bias ? bias[n] : 0.0f); break;
        case EPI_BIAS: v = acc + bias[n]; break;
        case EPI_BIAS_GELU_TANH: v = gelu_tanh(acc + (bias ? bias[n] : 0.0f)); break;
        case EPI_BIAS_SILU: v = silu(acc + (bias ? bias[n] : 0.0f)); break;
        case EPI_BIAS_RESIDUAL: v = acc + bias[n] + residual[m * N + n]; break;
        case EPI_RESIDUAL: v = acc + residual[m * N + n]; break;
        default: break;
      }
      C[m * N + n] = v;
    }
  }
}

/* Exact int32 C = A . B for int8 operands (int64 accumulation). */
void hx_ref_gemm_s8(int64_t M, int64_t N, int64_t K, const int8_t *A, const int8_t *B,
                    int b_layout, int32_t *C) {
  for (int64_t m = 0; m < M; ++m)
    for (int64_t n = 0; n < N; ++n) {
      int64_t acc = 0;
      for (int64_t k = 0; k < K; ++k)
        acc += (int64_t)A[m * K + k] *
               (int64_t)(b_layout == REF_B_NK ? B[n * K + k] : B[k * N + n]);
      C[m * N + n] = (int32_t)acc;
    }
}

/* W8A16: y[M,N] = sum_k x[m,k] * (W[n,k] * scale[n]) in fp32, x / scale f16 bits. */
void hx_ref_w8a16(int64_t M, int64_t N, int64_t K, const uint16_t *x, const int8_t *W,
                  const uint16_t *scale, float *y) {
  for (int64_t m = 0; m < M; ++m)
    for (int64_t n = 0; n < N; ++n) {
      float s = hx_ref_f16_to_f32(scale[n]);
      float acc = 0.0f;
      for (int64_t k = 0; k < K; ++k)
        acc += hx_ref_f16_to_f32(x[m * K + k]) * ((float)W[n * K + k] * s);
      y[m * N + n] = acc;
    }
}
