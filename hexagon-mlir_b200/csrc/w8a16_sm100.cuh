// w8a16_sm100.cuh — W8A16 skinny-M GEMM on tcgen05 tensor cores (swap-AB,
// split-K over a thread-block cluster, DSMEM reduction).
//
//   y[M, N] = x[M, K] . (W[N, K] * scale[N])^T (+ bias[N])
//   W int8 (per-output-channel symmetric), x / y / scale / bias fp16,
//   fp32 accumulation; M <= 256 (decode batch).
//
// Reference: the reference has no int8 GEMM; it lowers quantised ops to
// dequantise + float matmul (lib/Conversion/LinalgToLLVM/
// LinalgToLLVMPass.cpp:203-209) and turns unit-M matvec into a dot reduction
// split across threads (ReduceContractionRankPass.cpp:38-47,
// TilingPass.cpp:266-279).  At M = 8..64 the dequantised product needs
// 2*M flops per weight byte, more than CUDA cores deliver at HBM speed, so
// the product runs on the tensor cores with the operands swapped:
//   D^T[n, m] = W[n, :] . x[m, :]   (UMMA M = 128 weight rows,
//                                    UMMA N = M padded to MPAD)
// The int8 -> fp16 conversion is exact (|w| <= 127), and the per-channel
// scale is applied once to the fp32 result (scale[n] is a row factor of D^T),
// so the numbers equal dequantise-then-fp32-matmul up to summation order.
//
// One cluster of S CTAs owns 128 weight rows; CTA s of the cluster owns a
// contiguous share of the K blocks.  Roles (192 threads per CTA):
//   warp 0      TMA producer: raw int8 W box (128 rows x 128 K) and the two
//               fp16 x boxes (MPAD rows x 64 K) of each stage
//   warp 1      TMEM allocator + UMMA issuer
//   warps 2..5  converters (int8 smem -> fp16 128B-swizzled smem), then the
//               epilogue: TMEM -> smem partials, cluster barrier, each CTA
//               sums its share of batch rows over the S partials through
//               distributed shared memory, scales, stores y.
// With `weights_const`, the W loads of the first stages are issued before
// griddepcontrol.wait, overlapping the previous kernel in the stream.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

#include "ptx.cuh"

namespace hx {

struct W8A16Params {
  int32_t M, N, K;
  int32_t k_blocks;        // ceil(K / 128)
  int32_t splits;          // cluster size S
  int32_t stages;
  int32_t weights_const;   // prefetch W before waiting on the previous kernel
  const __half *scale;
  const __half *bias;
  __half *y;
  int64_t ldy;
  uint64_t timeout;
  int32_t *err_flag;
};

constexpr int kW8Threads = 192;
constexpr int kW8KBlock = 128;   // K elements per stage

template <int MPAD>
struct W8Cfg {
  static constexpr int kRawBytes = 128 * 128;          // int8 W box
  static constexpr int kConvBytes = 2 * 128 * 128;     // fp16, two 64-K halves
  static constexpr int kXHalfBytes = MPAD * 128;       // fp16 x, one 64-K half
  static constexpr int kXBytes = 2 * kXHalfBytes;
  static constexpr int kStageBytes = kRawBytes + kConvBytes + kXBytes;
  static constexpr int kTmemCols = MPAD < 32 ? 32 : MPAD;
  static constexpr int kRedBytes = MPAD * 128 * 4;     // fp32 partials
  static constexpr uint32_t kIdesc = make_idesc(0, false, 128, MPAD);
  static constexpr int smem_bytes(int stages) {
    const int ring = stages * kStageBytes;
    return (ring > kRedBytes ? ring : kRedBytes) + 1024 + 256;
  }
  static_assert(MPAD == 16 || MPAD == 32 || MPAD == 64 || MPAD == 128 || MPAD == 256, "MPAD");
};

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}
__device__ __forceinline__ uint32_t map_peer_smem(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
__device__ __forceinline__ float ld_cluster_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32"
      " {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// Convert 16 int8 (one 16-byte chunk) to 16 fp16 packed in two uint4.
// Exact magic-number conversion: for v in [-128, 127], u = v + 128 (flip the
// sign bit) is an 8-bit unsigned value, the fp16 bit pattern 0x6400 | u is
// exactly 1024 + u, and subtracting 1152 (= 1024 + 128) leaves v.  prmt
// places two bytes into the low halves of two 16-bit lanes.
__device__ __forceinline__ uint32_t i8x2_to_f16x2(uint32_t w_flipped, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(w_flipped), "r"(0x64646464u), "r"(sel));
  __half2 h = *reinterpret_cast<__half2 *>(&r);
  const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));  // 1152
  h = __hsub2(h, bias);
  return *reinterpret_cast<uint32_t *>(&h);
}
__device__ __forceinline__ void i8x16_to_f16(const uint4 w, uint4 &lo, uint4 &hi) {
  const uint32_t ws[4] = {w.x ^ 0x80808080u, w.y ^ 0x80808080u, w.z ^ 0x80808080u,
                          w.w ^ 0x80808080u};
  uint32_t o[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    o[2 * i] = i8x2_to_f16x2(ws[i], 0x5150u);      // bytes 0,1 -> lanes (b0|0x64, b1|0x64)
    o[2 * i + 1] = i8x2_to_f16x2(ws[i], 0x5352u);  // bytes 2,3
  }
  lo = make_uint4(o[0], o[1], o[2], o[3]);
  hi = make_uint4(o[4], o[5], o[6], o[7]);
}

template <int MPAD>
__global__ void __launch_bounds__(kW8Threads, 1)
    hx_w8a16_tc_kernel(const __grid_constant__ CUtensorMap tmW,
                       const __grid_constant__ CUtensorMap tmX,
                       const __grid_constant__ W8A16Params p) {
  using Cfg = W8Cfg<MPAD>;
  const int STAGES = p.stages;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int ring = STAGES * Cfg::kStageBytes;
  uint8_t *tail = smem + (ring > Cfg::kRedBytes ? ring : Cfg::kRedBytes);
  uint64_t *full_bar = reinterpret_cast<uint64_t *>(tail);
  uint64_t *conv_bar = full_bar + STAGES;
  uint64_t *empty_bar = conv_bar + STAGES;
  uint64_t *tfull_bar = empty_bar + STAGES;
  uint64_t *drain_bar = tfull_bar + 1;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain_bar + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
  // stage s: [conv (32 KB) | x (2 * MPAD * 128) | raw W (16 KB)], each 1024-aligned
  auto conv_of = [&](int s) { return smem + s * Cfg::kStageBytes; };
  auto x_of = [&](int s) { return smem + s * Cfg::kStageBytes + Cfg::kConvBytes; };
  auto raw_of = [&](int s) { return smem + s * Cfg::kStageBytes + Cfg::kConvBytes + Cfg::kXBytes; };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t split = cluster_ctarank();
  const int tile = blockIdx.x / p.splits;
  const int n0 = tile * 128;
  // this CTA's K blocks: [kb0, kb1)
  const int per = p.k_blocks / p.splits, rem = p.k_blocks % p.splits;
  const int kb0 = split * per + min(static_cast<int>(split), rem);
  const int kb1 = kb0 + per + (static_cast<int>(split) < rem ? 1 : 0);
  const int nkb = kb1 - kb0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&conv_bar[s], 4);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(tfull_bar, 1);
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  grid_dep_launch_dependents();

  bool ok = true;
  if (warp == 0) {
    // ------------------------------------------------------------ producer
    const int pre = (p.weights_const && nkb > 0) ? min(STAGES, nkb) : 0;
    if (lane == 0) {
      tma_prefetch_desc(&tmW);
      tma_prefetch_desc(&tmX);
      for (int i = 0; i < pre; ++i) {  // constant weights: start streaming now
        mbar_arrive_expect_tx(&full_bar[i], Cfg::kRawBytes + Cfg::kXBytes);
        tma_load_2d(raw_of(i), &tmW, &full_bar[i], (kb0 + i) * kW8KBlock, n0);
      }
    }
    grid_dep_wait();
    int stage = 0;
    uint32_t phase = 0;
    int issued = pre;
    for (int i = 0; i < nkb; ++i) {
      const int kx = (kb0 + i) * kW8KBlock;
      if (i >= pre) {
        bool w = (lane == 0) ? mbar_wait(&empty_bar[stage], phase ^ 1, p.timeout, abort_flag) : true;
        w = __shfl_sync(0xffffffffu, w, 0);
        if (!w) {
          if (lane == 0) {
            *abort_flag = 1;
            if (p.err_flag) atomicExch(p.err_flag, 11);
          }
          ok = false;
          break;
        }
        if (lane == 0) {
          mbar_arrive_expect_tx(&full_bar[stage], Cfg::kRawBytes + Cfg::kXBytes);
          tma_load_2d(raw_of(stage), &tmW, &full_bar[stage], kx, n0);
        }
        ++issued;
      }
      if (lane == 0) {
        tma_load_2d(x_of(stage), &tmX, &full_bar[stage], kx, 0);
        tma_load_2d(x_of(stage) + Cfg::kXHalfBytes, &tmX, &full_bar[stage], kx + 64, 0);
      }
      __syncwarp();
      if (++stage == STAGES) {
        stage = 0;
        phase ^= 1;
      }
    }
    if (!ok && lane == 0) {  // drain loads still in flight
      int dummy = 0;
      for (int j = (issued > STAGES ? issued - STAGES : 0); j < issued; ++j)
        mbar_wait(&full_bar[j % STAGES], static_cast<uint32_t>((j / STAGES) & 1), p.timeout, &dummy);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ UMMA issuer
    grid_dep_wait();
    int stage = 0;
    uint32_t phase = 0;
    bool any = false;
    for (int i = 0; i < nkb; ++i) {
      bool w = (lane == 0) ? mbar_wait(&conv_bar[stage], phase, p.timeout, abort_flag) : true;
      w = __shfl_sync(0xffffffffu, w, 0);
      if (!w) {
        if (lane == 0) {
          *abort_flag = 1;
          if (p.err_flag) atomicExch(p.err_flag, 12);
        }
        ok = false;
        break;
      }
      tc_fence_after();
      if (lane == 0) {
        const uint32_t a_base = smem_u32(conv_of(stage));
        const uint32_t b_base = smem_u32(x_of(stage));
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint64_t ad = sdesc_kmajor_sw128(a_base + h * (128 * 128) + k * 32);
            const uint64_t bd = sdesc_kmajor_sw128(b_base + h * Cfg::kXHalfBytes + k * 32);
            umma_f16(tmem_base, ad, bd, Cfg::kIdesc, (i > 0 || h > 0 || k > 0) ? 1u : 0u);
          }
        umma_commit(&empty_bar[stage]);
        any = true;
      }
      __syncwarp();
      if (++stage == STAGES) {
        stage = 0;
        phase ^= 1;
      }
    }
    if (lane == 0) {
      if (ok) {
        umma_commit(tfull_bar);
      } else if (any) {
        umma_commit(drain_bar);
        int dummy = 0;
        mbar_wait(drain_bar, 0, p.timeout, &dummy);
      }
    }
  } else {
    // ------------------------------------------------------------ converters
    grid_dep_wait();
    const int r = (warp & 3) * 32 + lane;  // weight row of the tile this thread converts
    int stage = 0;
    uint32_t phase = 0;
    for (int i = 0; i < nkb; ++i) {
      bool w = (lane == 0) ? mbar_wait(&full_bar[stage], phase, p.timeout, abort_flag) : true;
      w = __shfl_sync(0xffffffffu, w, 0);
      if (!w) {
        if (lane == 0) {
          *abort_flag = 1;
          if (p.err_flag) atomicExch(p.err_flag, 13);
        }
        ok = false;
        break;
      }
      const uint8_t *raw = raw_of(stage) + r * 128;
      uint8_t *conv = conv_of(stage) + r * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        // raw box is 128B-swizzled by TMA: logical chunk c sits at c ^ (r & 7)
        const uint4 wv = *reinterpret_cast<const uint4 *>(raw + ((c ^ (r & 7)) << 4));
        uint4 lo, hi;
        i8x16_to_f16(wv, lo, hi);
        // fp16 K = 16c .. 16c+15 -> half h = c/4, 16-byte chunks 2(c%4), 2(c%4)+1
        uint8_t *dst = conv + (c >> 2) * (128 * 128);
        const int j0 = (c & 3) * 2;
        *reinterpret_cast<uint4 *>(dst + ((j0 ^ (r & 7)) << 4)) = lo;
        *reinterpret_cast<uint4 *>(dst + (((j0 + 1) ^ (r & 7)) << 4)) = hi;
      }
      fence_proxy_async_smem();  // generic smem writes -> visible to UMMA
      __syncwarp();
      if (lane == 0) mbar_arrive(&conv_bar[stage]);
      if (++stage == STAGES) {
        stage = 0;
        phase ^= 1;
      }
    }
    // ------------------------------------------------------------ epilogue part 1
    float *red = reinterpret_cast<float *>(smem);  // [MPAD][128] fp32 partials
    bool have = ok && nkb > 0;
    if (have) {
      bool w = (lane == 0) ? mbar_wait(tfull_bar, 0, p.timeout, abort_flag) : true;
      w = __shfl_sync(0xffffffffu, w, 0);
      if (!w) {
        if (lane == 0) {
          *abort_flag = 1;
          if (p.err_flag) atomicExch(p.err_flag, 14);
        }
        have = false;
      }
    }
    // Named barrier over the 4 epilogue warps: every converter finished
    // reading the ring before the partials overwrite it.
    asm volatile("bar.sync 1, 128;" ::: "memory");
    tc_fence_after();
    const uint32_t t_row = tmem_base + (static_cast<uint32_t>((warp & 3) * 32) << 16);
#pragma unroll
    for (int c = 0; c < MPAD; c += 16) {
      uint32_t v[16];
      tmem_ld_32x32b_x16(t_row + c, v);
      tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < 16; ++j) red[(c + j) * 128 + r] = have ? __uint_as_float(v[j]) : 0.f;
    }
    tc_fence_before();
  }

  // ---------------------------------------------------------------- reduce
  __syncthreads();
  cluster_sync();  // every CTA's partials are written
  if (warp >= 2) {
    const int r = (warp & 3) * 32 + threadIdx.x % 32;
    const int n = n0 + r;
    const uint32_t my_red = smem_u32(smem);
    if (n < p.N) {
      const float sc = __half2float(p.scale[n]);
      const float bi = p.bias ? __half2float(p.bias[n]) : 0.f;
      for (int m = split; m < p.M; m += p.splits) {
        const uint32_t a = my_red + (m * 128 + r) * 4;
        float part[8];
#pragma unroll
        for (int s = 0; s < 8; ++s)  // independent DSMEM loads, issued together
          part[s] = s < p.splits ? ld_cluster_f32(map_peer_smem(a, s)) : 0.f;
        float acc = 0.f;
#pragma unroll
        for (int s = 0; s < 8; ++s) acc += part[s];
        p.y[static_cast<int64_t>(m) * p.ldy + n] = __float2half_rn(acc * sc + bi);
      }
    }
  }
  cluster_sync();  // peers keep their smem until every CTA finished reading
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, Cfg::kTmemCols);
}

}  // namespace hx
