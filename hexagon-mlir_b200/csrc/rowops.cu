// rowops.cu — row-wise kernels either side of the linear layer:
//
//   * softmax over the vocabulary of LM-head logits, also when the vocabulary
//     is split across ranks (vocab-parallel): each rank reduces its shard of a
//     row to (max, sum of exp(x - max)), the ranks exchange these two floats
//     per row, and each rank normalises its own shard.  The full [M, N] logits
//     never have to be gathered.  Reference: the softmax kernels of
//     test/python/triton/test_softmax.py and the two-phase online softmax of
//     test/python/triton/test_online_softmax.py (running max and rescaled sum,
//     then exp(x - max) / sum).
//   * the per-row statistics of LayerNorm (mean, 1/sqrt(var + eps)) and
//     RMSNorm (1/sqrt(mean(x^2) + eps)) that let the normalisation be folded
//     into the following GEMM (its epilogue applies them), as
//     test/python/triton/test_layer_norm.py and test_rms_norm.py define them.
//
// All are HBM-bound streaming kernels: one CTA per row (grid-stride over rows,
// up to four 512-thread CTAs per SM), 16-byte loads where rows are aligned, fp32 arithmetic.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include <algorithm>
#include <type_traits>

#include "hx_gemm.h"
#include "launch.cuh"

namespace hx {
namespace {

constexpr int kRowThreads = 512;

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }

template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <>
__device__ __forceinline__ float from_f<float>(float v) { return v; }

// (max, sum of exp(x - max)) pairs: merging two partial reductions.
struct MaxSum {
  float m, s;
};
__device__ __forceinline__ MaxSum ms_merge(MaxSum a, MaxSum b) {
  if (a.m == -INFINITY) return b;
  if (b.m == -INFINITY) return a;
  const float m = fmaxf(a.m, b.m);
  return {m, a.s * __expf(a.m - m) + b.s * __expf(b.m - m)};
}
__device__ __forceinline__ MaxSum ms_add(MaxSum a, float x) {
  if (x == -INFINITY) return a;  // contributes exp(-inf) = 0
  if (x <= a.m) return {a.m, a.s + __expf(x - a.m)};
  return {x, (a.m == -INFINITY ? 0.f : a.s * __expf(a.m - x)) + 1.f};
}

// Block-wide reductions (kRowThreads threads); `red` holds 2 floats per warp.
__device__ __forceinline__ MaxSum block_merge(MaxSum v, float *red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    MaxSum w{__shfl_xor_sync(0xffffffffu, v.m, o), __shfl_xor_sync(0xffffffffu, v.s, o)};
    v = ms_merge(v, w);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();  // red may still be read from the previous row
  if (lane == 0) {
    red[2 * warp] = v.m;
    red[2 * warp + 1] = v.s;
  }
  __syncthreads();
  MaxSum r{-INFINITY, 0.f};
  for (int w = 0; w < kRowThreads / 32; ++w) r = ms_merge(r, MaxSum{red[2 * w], red[2 * w + 1]});
  return r;
}
__device__ __forceinline__ float2 block_sum2(float a, float b, float *red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    a += __shfl_xor_sync(0xffffffffu, a, o);
    b += __shfl_xor_sync(0xffffffffu, b, o);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) {
    red[2 * warp] = a;
    red[2 * warp + 1] = b;
  }
  __syncthreads();
  float2 r = make_float2(0.f, 0.f);
  for (int w = 0; w < kRowThreads / 32; ++w) {
    r.x += red[2 * w];
    r.y += red[2 * w + 1];
  }
  return r;
}

// Visit the N elements of a row: 16-byte vectors when `vec` (four loads in
// flight per thread, so a few CTAs per SM keep HBM busy), else scalars.
template <typename T, typename F>
__device__ __forceinline__ void for_row(const T *row, int64_t N, bool vec, F &&f) {
  constexpr int V = 16 / sizeof(T);
  constexpr int U = 4;
  if (vec) {
    const int64_t nv = N / V;
    const uint4 *r4 = reinterpret_cast<const uint4 *>(row);
    int64_t i = threadIdx.x;
    for (; i + (U - 1) * kRowThreads < nv; i += U * kRowThreads) {
      uint4 u[U];
#pragma unroll
      for (int j = 0; j < U; ++j) u[j] = __ldcs(r4 + i + j * kRowThreads);  // streamed once
#pragma unroll
      for (int j = 0; j < U; ++j) {
        const T *e = reinterpret_cast<const T *>(&u[j]);
#pragma unroll
        for (int q = 0; q < V; ++q) f((i + j * kRowThreads) * V + q, to_f<T>(e[q]));
      }
    }
    for (; i < nv; i += kRowThreads) {
      const uint4 u = __ldcs(r4 + i);
      const T *e = reinterpret_cast<const T *>(&u);
#pragma unroll
      for (int q = 0; q < V; ++q) f(i * V + q, to_f<T>(e[q]));
    }
    for (int64_t k = nv * V + threadIdx.x; k < N; k += kRowThreads) f(k, to_f<T>(row[k]));
  } else {
    for (int64_t k = threadIdx.x; k < N; k += kRowThreads) f(k, to_f<T>(row[k]));
  }
}

// Visit a row 16 bytes at a time: fv(first index, float v[VT]) for whole
// vectors (four loads in flight per thread), fs(index, v) for a ragged tail
// or an unaligned row.
template <typename T, typename FV, typename FS>
__device__ __forceinline__ void for_row_vec(const T *row, int64_t N, bool vec, FV &&fv, FS &&fs) {
  constexpr int V = 16 / sizeof(T);
  constexpr int U = 4;
  if (!vec) {
    for (int64_t k = threadIdx.x; k < N; k += kRowThreads) fs(k, to_f<T>(row[k]));
    return;
  }
  const int64_t nv = N / V;
  const uint4 *r4 = reinterpret_cast<const uint4 *>(row);
  int64_t i = threadIdx.x;
  for (; i + (U - 1) * kRowThreads < nv; i += U * kRowThreads) {
    uint4 u[U];
#pragma unroll
    for (int j = 0; j < U; ++j) u[j] = __ldcs(r4 + i + j * kRowThreads);
#pragma unroll
    for (int j = 0; j < U; ++j) {
      const T *e = reinterpret_cast<const T *>(&u[j]);
      float v[V];
#pragma unroll
      for (int q = 0; q < V; ++q) v[q] = to_f<T>(e[q]);
      fv((i + j * kRowThreads) * V, u[j], v);
    }
  }
  for (; i < nv; i += kRowThreads) {
    const uint4 u = __ldcs(r4 + i);
    const T *e = reinterpret_cast<const T *>(&u);
    float v[V];
#pragma unroll
    for (int q = 0; q < V; ++q) v[q] = to_f<T>(e[q]);
    fv(i * V, u, v);
  }
  for (int64_t k = nv * V + threadIdx.x; k < N; k += kRowThreads) fs(k, to_f<T>(row[k]));
}

// Fold V values into a running {max, sum}: one max over the vector, one
// rescale of the sum, then V exponentials.
template <int V>
__device__ __forceinline__ MaxSum ms_add_vec(MaxSum a, const float (&v)[V]) {
  float mx = v[0];
#pragma unroll
  for (int q = 1; q < V; ++q) mx = fmaxf(mx, v[q]);
  if (mx == -INFINITY) return a;
  const float m = fmaxf(a.m, mx);
  float s = a.m == -INFINITY ? 0.f : a.s * __expf(a.m - m);
#pragma unroll
  for (int q = 0; q < V; ++q) s += __expf(v[q] - m);
  return {m, s};
}

template <typename T>
__global__ void __launch_bounds__(kRowThreads) softmax_stats_kernel(const T *x, int64_t M, int64_t N,
                                                                    int64_t ldx, bool vec, float *stats) {
  __shared__ float red[2 * kRowThreads / 32];
  for (int64_t m = blockIdx.x; m < M; m += gridDim.x) {
    MaxSum acc{-INFINITY, 0.f};
    for_row_vec(x + m * ldx, N, vec, [&](int64_t, const uint4 &, const float (&v)[16 / sizeof(T)]) {
      acc = ms_add_vec(acc, v);
    }, [&](int64_t, float v) { acc = ms_add(acc, v); });
    const MaxSum r = block_merge(acc, red);
    if (threadIdx.x == 0) {
      stats[2 * m] = r.m;
      stats[2 * m + 1] = r.s;
    }
  }
}

__global__ void softmax_combine_kernel(const float *all, int world, int64_t M, float *stats) {
  for (int64_t m = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; m < M; m += int64_t(gridDim.x) * blockDim.x) {
    MaxSum r{-INFINITY, 0.f};
    for (int w = 0; w < world; ++w) r = ms_merge(r, MaxSum{all[(w * M + m) * 2], all[(w * M + m) * 2 + 1]});
    stats[2 * m] = r.m;
    stats[2 * m + 1] = r.s;
  }
}

template <typename T, typename U>
__global__ void __launch_bounds__(kRowThreads) softmax_apply_kernel(const T *x, int64_t M, int64_t N, int64_t ldx,
                                                                    bool vec, const float *stats, U *y,
                                                                    int64_t ldy, bool log_out) {
  for (int64_t m = blockIdx.x; m < M; m += gridDim.x) {
    const float mx = stats[2 * m], sum = stats[2 * m + 1];
    const float inv = 1.f / sum, lse = mx + logf(sum);
    U *yr = y + m * ldy;
    for_row(x + m * ldx, N, vec, [&](int64_t i, float v) {
      yr[i] = from_f<U>(log_out ? v - lse : __expf(v - mx) * inv);
    });
  }
}

// VT = 16 / sizeof(T) outputs from VT inputs: one 16-byte store per VT * 2
// bytes of 16-bit U (two for float U) when the output row is aligned.
template <typename T, typename U>
__device__ __forceinline__ void store_outs(U *dst, const float (&o)[16 / sizeof(T)], bool yvec) {
  constexpr int VT = 16 / sizeof(T);
  if (yvec && (VT * sizeof(U)) % 16 == 0) {
    U pk[VT];
#pragma unroll
    for (int q = 0; q < VT; ++q) pk[q] = from_f<U>(o[q]);
#pragma unroll
    for (int q = 0; q < int(VT * sizeof(U) / 16); ++q)
      reinterpret_cast<uint4 *>(dst)[q] = reinterpret_cast<const uint4 *>(pk)[q];
  } else {
#pragma unroll
    for (int q = 0; q < VT; ++q) dst[q] = from_f<U>(o[q]);
  }
}

// Whole softmax of a row in one CTA: the row is read once and kept in shared
// memory (in its own dtype) when it fits in kSmemRow bytes, small enough for
// two CTAs per SM, else read twice.
constexpr int kSmemRow = 112 * 1024;
template <typename T, typename U>
__global__ void __launch_bounds__(kRowThreads) softmax_rows_kernel(const T *x, int64_t M, int64_t N, int64_t ldx,
                                                                   bool vec, U *y, int64_t ldy, bool log_out,
                                                                   bool yvec) {
  extern __shared__ __align__(16) uint8_t srow_raw[];  // the row, when it fits
  T *srow = reinterpret_cast<T *>(srow_raw);
  __shared__ float red[2 * kRowThreads / 32];
  constexpr int VT = 16 / sizeof(T);
  const bool cache = N * int64_t(sizeof(T)) <= kSmemRow;
  for (int64_t m = blockIdx.x; m < M; m += gridDim.x) {
    MaxSum acc{-INFINITY, 0.f};
    for_row_vec(x + m * ldx, N, vec, [&](int64_t i, const uint4 &u, const float (&v)[VT]) {
      acc = ms_add_vec(acc, v);
      if (cache) *reinterpret_cast<uint4 *>(srow + i) = u;  // the raw vector
    }, [&](int64_t i, float v) {
      acc = ms_add(acc, v);
      if (cache) srow[i] = from_f<T>(v);  // exact: v came from a T
    });
    const MaxSum r = block_merge(acc, red);  // its barriers also order the srow writes
    const float inv = 1.f / r.s, lse = r.m + logf(r.s);
    U *yr = y + m * ldy;
    if (cache) {
      const int64_t nv = N / VT;  // shared memory rows are 16-byte aligned
      for (int64_t i = threadIdx.x; i < nv; i += kRowThreads) {
        const uint4 u = reinterpret_cast<const uint4 *>(srow)[i];
        const T *e = reinterpret_cast<const T *>(&u);
        float o[VT];
#pragma unroll
        for (int q = 0; q < VT; ++q) {
          const float v = to_f<T>(e[q]);
          o[q] = log_out ? v - lse : __expf(v - r.m) * inv;
        }
        store_outs<T, U>(yr + i * VT, o, yvec);
      }
      for (int64_t i = nv * VT + threadIdx.x; i < N; i += kRowThreads) {
        const float v = to_f<T>(srow[i]);
        yr[i] = from_f<U>(log_out ? v - lse : __expf(v - r.m) * inv);
      }
      __syncthreads();  // srow is rewritten by the next row
    } else {
      for_row(x + m * ldx, N, vec, [&](int64_t i, float v) {
        yr[i] = from_f<U>(log_out ? v - lse : __expf(v - r.m) * inv);
      });
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kRowThreads) row_norm_stats_kernel(const T *x, int64_t M, int64_t K, int64_t ldx,
                                                                     bool vec, int kind, float eps, float *stats) {
  __shared__ float red[2 * kRowThreads / 32];
  for (int64_t m = blockIdx.x; m < M; m += gridDim.x) {
    // Shifted sums (shift = the row's first element) keep the variance
    // accurate when the mean is large against the spread.
    const float shift = kind == HX_NORM_LAYER ? to_f<T>(x[m * ldx]) : 0.f;
    float s1 = 0.f, s2 = 0.f;
    for_row(x + m * ldx, K, vec, [&](int64_t, float v) {
      const float d = v - shift;
      s1 += d;
      s2 += d * d;
    });
    const float2 r = block_sum2(s1, s2, red);
    if (threadIdx.x == 0) {
      const float inv_k = 1.f / static_cast<float>(K);
      float mean = 0.f, var;
      if (kind == HX_NORM_LAYER) {
        const float dm = r.x * inv_k;
        mean = shift + dm;
        var = fmaxf(r.y * inv_k - dm * dm, 0.f);
      } else {
        var = r.y * inv_k;  // mean of squares
      }
      stats[2 * m] = mean;
      stats[2 * m + 1] = rsqrtf(var + eps);
    }
  }
}

int row_grid(int64_t M) {
  int sms = 148;
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(M, int64_t(sms) * (2048 / kRowThreads))));
}

bool row_vec(const void *p, int64_t ld, int esz) {
  return (reinterpret_cast<uintptr_t>(p) & 15) == 0 && (ld * esz) % 16 == 0;
}

int esz_of(int dt) { return dt == HX_F32 ? 4 : ((dt == HX_F16 || dt == HX_BF16) ? 2 : 0); }

template <typename F>
int by_dtype(int dt, F &&f) {
  switch (dt) {
    case HX_F16: return f(static_cast<const __half *>(nullptr));
    case HX_BF16: return f(static_cast<const __nv_bfloat16 *>(nullptr));
    case HX_F32: return f(static_cast<const float *>(nullptr));
    default: return unsupported("row kernels take f16, bf16 or f32");
  }
}

int check_launch(const char *what) {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? HX_OK : cuda_fail(e, what);
}

}  // namespace
}  // namespace hx

extern "C" {

int hx_softmax_stats(const void *x, int dtype, int64_t M, int64_t N, int64_t ldx, float *stats, void *stream) {
  hx::g_last_error.clear();
  if (M < 0 || N <= 0 || ldx < N || (M > 0 && (!x || !stats))) return HX_E_INVALID_ARG;
  if (M == 0) return HX_OK;
  const int ez = hx::esz_of(dtype);
  const bool vec = hx::row_vec(x, ldx, ez);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return hx::by_dtype(dtype, [&](auto tag) {
    using T = std::remove_const_t<std::remove_pointer_t<decltype(tag)>>;
    hx::softmax_stats_kernel<T><<<hx::row_grid(M), hx::kRowThreads, 0, s>>>(static_cast<const T *>(x), M, N,
                                                                            ldx, vec, stats);
    return hx::check_launch("softmax_stats_kernel");
  });
}

int hx_softmax_combine(const float *stats_all, int world, int64_t M, float *stats, void *stream) {
  hx::g_last_error.clear();
  if (world < 1 || M < 0 || (M > 0 && (!stats_all || !stats))) return HX_E_INVALID_ARG;
  if (M == 0) return HX_OK;
  const int blocks = static_cast<int>(std::min<int64_t>((M + 255) / 256, 148 * 4));
  hx::softmax_combine_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(stats_all, world, M, stats);
  return hx::check_launch("softmax_combine_kernel");
}

int hx_softmax_apply(const void *x, int dtype, int64_t M, int64_t N, int64_t ldx, const float *stats, void *y,
                     int y_dtype, int64_t ldy, int log_softmax, void *stream) {
  hx::g_last_error.clear();
  if (M < 0 || N <= 0 || ldx < N || ldy < N || (M > 0 && (!x || !stats || !y))) return HX_E_INVALID_ARG;
  if (M == 0) return HX_OK;
  const bool vec = hx::row_vec(x, ldx, hx::esz_of(dtype));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return hx::by_dtype(dtype, [&](auto tag) {
    using T = std::remove_const_t<std::remove_pointer_t<decltype(tag)>>;
    return hx::by_dtype(y_dtype, [&](auto tag2) {
      using U = std::remove_const_t<std::remove_pointer_t<decltype(tag2)>>;
      hx::softmax_apply_kernel<T, U><<<hx::row_grid(M), hx::kRowThreads, 0, s>>>(
          static_cast<const T *>(x), M, N, ldx, vec, stats, static_cast<U *>(y), ldy, log_softmax != 0);
      return hx::check_launch("softmax_apply_kernel");
    });
  });
}

int hx_softmax(const void *x, int dtype, int64_t M, int64_t N, int64_t ldx, void *y, int y_dtype, int64_t ldy,
               int log_softmax, void *stream) {
  hx::g_last_error.clear();
  if (M < 0 || N <= 0 || ldx < N || ldy < N || (M > 0 && (!x || !y))) return HX_E_INVALID_ARG;
  if (M == 0) return HX_OK;
  const bool vec = hx::row_vec(x, ldx, hx::esz_of(dtype));
  const bool yvec = hx::row_vec(y, ldy, hx::esz_of(y_dtype));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return hx::by_dtype(dtype, [&](auto tag) {
    using T = std::remove_const_t<std::remove_pointer_t<decltype(tag)>>;
    const size_t smem = N * sizeof(T) <= static_cast<size_t>(hx::kSmemRow) ? N * sizeof(T) : 0;
    return hx::by_dtype(y_dtype, [&](auto tag2) {
      using U = std::remove_const_t<std::remove_pointer_t<decltype(tag2)>>;
      auto kern = hx::softmax_rows_kernel<T, U>;
      static hx::SmemAttrOnce once;
      cudaError_t e = hx::ensure_max_smem(kern, once, hx::kSmemRow);
      if (e != cudaSuccess) return hx::cuda_fail(e, "cudaFuncSetAttribute(softmax)");
      kern<<<hx::row_grid(M), hx::kRowThreads, smem, s>>>(static_cast<const T *>(x), M, N, ldx, vec,
                                                          static_cast<U *>(y), ldy, log_softmax != 0, yvec);
      return hx::check_launch("softmax_rows_kernel");
    });
  });
}

int hx_row_norm_stats(const void *x, int dtype, int64_t M, int64_t K, int64_t ldx, int kind, float eps,
                      float *stats, void *stream) {
  hx::g_last_error.clear();
  if (M < 0 || K <= 0 || ldx < K || (kind != HX_NORM_LAYER && kind != HX_NORM_RMS) || !(eps >= 0.f) ||
      (M > 0 && (!x || !stats)))
    return HX_E_INVALID_ARG;
  if (M == 0) return HX_OK;
  const bool vec = hx::row_vec(x, ldx, hx::esz_of(dtype));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return hx::by_dtype(dtype, [&](auto tag) {
    using T = std::remove_const_t<std::remove_pointer_t<decltype(tag)>>;
    hx::row_norm_stats_kernel<T><<<hx::row_grid(M), hx::kRowThreads, 0, s>>>(static_cast<const T *>(x), M, K,
                                                                             ldx, vec, kind, eps, stats);
    return hx::check_launch("row_norm_stats_kernel");
  });
}

}  // extern "C"
