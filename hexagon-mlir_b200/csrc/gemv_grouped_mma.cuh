// gemv_grouped_mma.cuh — a decode step's W8A16 projections in one persistent
// launch, weights converted in registers and multiplied on the tensor cores
// through warp-level register-operand MMAs (mma.sync m16n8k16, fp32
// accumulate).  Used for batches M <= 16 (wider batches measured slower than
// the tcgen05 kernel: the warp-level MMA rate, not HBM, bounds them).
//
// Same contract as hx_gemv_w8a16_grouped_kernel (gemv_grouped.cuh): a list of
// projections y_g[M, N_g] = x_g[M, K_g] . (W_g * scale_g)^T (+ bias_g), W int8
// per-output-channel, x / y / scale / bias fp16, fp32 accumulation, optional
// dependencies (x_g is the y of an earlier projection).
//
// Why not tcgen05 here: with the batch as the UMMA N (16 at M <= 16), one
// tcgen05.mma covers 128 weight rows x 16 K = 2 KB of int8 weights, and the
// measured cost per instruction stays near 170 SM cycles for N = 16 .. 64
// wherever A lives (shared memory or TMEM).  That caps the tcgen05 decode
// kernel (gemv_grouped_tc.cuh) near 3.4 TB/s, about half of HBM.  A
// warp-level MMA takes its A fragment straight from the registers the int8 ->
// fp16 conversion writes, so the weights cross no shared memory and no
// tensor-memory stage:
//   * each lane loads 16 P contiguous int8 weights of each of its rows per
//     chunk of 64 P K (128-bit streaming loads; a lane quad covers a 64 P-byte
//     row segment: P = 2 gives 128-byte runs, which HBM serves measurably
//     better than 64-byte ones), converts them exactly (byte permute + fp16
//     subtract) and feeds 4 P MMAs;
//   * the reduction order over K is permuted inside each chunk so that a
//     lane's A fragment is its own contiguous bytes: MMA j of a chunk takes,
//     for lane quad q, K = 16 P q + 4 j + {0, 1, 2, 3}; x is read with the same
//     permutation (the dot product does not depend on the order);
//   * a register ring of weight loads keeps 8 KB in flight per warp, 128 KB
//     per SM (two CTAs of eight warps).
// Work item = (projection g, block of 32 weight rows), one warp per item.
// Items are handed out in list order by a ticket counter (an atomic add on
// the last projection's counter, which no projection signals): with static
// round-robin the items' sizes (K = 2048 vs 5632) left the busiest warp
// ~1.5x the average.  A dependent projection's warp first waits (bounded
// spin, acquire) until every item of its producer projection has signalled
// its counter; every warp of the grid is resident and tickets rise, so the
// lowest unfinished item's dependencies are finished and it can proceed.
//
// Reference counterpart: dequantise + matmul (lib/Conversion/LinalgToLLVM/
// LinalgToLLVMPass.cpp:203-209); the conversion is exact and the scale is a
// per-row factor applied to the fp32 accumulator, so results equal
// dequantise-then-fp32-matmul up to summation order.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

#include "gemv_grouped.cuh"
#include "ptx.cuh"
#include "w8a16_sm100.cuh"

namespace hx {

constexpr int kGmWarps = 8;   // warps per CTA

__device__ __forceinline__ uint4 ld_stream_u4(const void *p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// D (4 x fp32) += A (16 x 16 fp16, 4 regs) * B (16 x 8 fp16, 2 regs).
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9},"
      " {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t u4_word(const uint4 &v, int j) {
  return j == 0 ? v.x : (j == 1 ? v.y : (j == 2 ? v.z : v.w));
}

// NB: batch blocks of 8 (M <= 8 NB).  RB: 16-row blocks per item; lane
// (g8 = lane / 4, q = lane % 4) owns rows g8 and g8 + 8 of each block.
// P: 16-byte pieces of a row per lane per chunk (a chunk is 64 P of K).
template <int NB, int RB, int P>
__global__ void __launch_bounds__(kGmWarps * 32, 2)
    hx_gemv_w8a16_grouped_mma_kernel(const __grid_constant__ GroupParams p) {
  constexpr int kGmRows = 16 * RB;
  constexpr int kSeg = 16 * P;                                   // row bytes per lane per chunk
  constexpr int kChunk = 4 * kSeg;                               // K per chunk
  constexpr int kDepth = 8 / (RB * P) < 2 ? 2 : 8 / (RB * P);    // chunks in flight per lane
  const int lane = threadIdx.x & 31;
  const int g8 = lane >> 2, q = lane & 3;
  grid_dep_launch_dependents();
  grid_dep_wait();  // counters zeroed and inputs written by the preceding work
  int32_t *ticket = p.counters + (p.G - 1);

  while (true) {
    int item = 0;
    if (lane == 0) item = atomicAdd(ticket, 1);
    item = __shfl_sync(0xffffffffu, item, 0);
    if (item >= p.total_items) break;
    const int g = group_find(p, item);
    const GroupDesc &d = p.d[g];
    const int row0 = (item - d.item_begin) * kGmRows;
    if (d.dep >= 0) {  // x is an earlier projection's y: wait until all of it is stored
      const GroupDesc &dd = p.d[d.dep];
      const int target = (dd.N + kGmRows - 1) / kGmRows;
      bool ok = true;
      if (lane == 0) {
        const uint64_t t0 = clock64();
        while (ld_acquire_gpu(p.counters + d.dep) < target) {
          if (static_cast<uint64_t>(clock64() - t0) > p.timeout) {
            ok = false;
            break;
          }
          __nanosleep(64);
        }
        if (!ok && p.err_flag) atomicExch(p.err_flag, 21);
      }
      if (!__shfl_sync(0xffffffffu, ok, 0)) return;
    }

    // the lane's weight rows (rows past N re-read row N-1; not stored)
    const int8_t *wr[RB][2];
#pragma unroll
    for (int rb = 0; rb < RB; ++rb)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh)
        wr[rb][hh] = d.W + static_cast<int64_t>(min(row0 + 16 * rb + 8 * hh + g8, d.N - 1)) * d.ldw + kSeg * q;
    // the lane's batch rows of x (rows >= M read as zero)
    const __half *xr[NB];
    bool xv_ok[NB];
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) {
      const int m = 8 * nb + g8;
      xv_ok[nb] = m < p.M;
      xr[nb] = d.x + static_cast<int64_t>(xv_ok[nb] ? m : 0) * d.ldx + kSeg * q;
    }

    float acc[RB][NB][4];
#pragma unroll
    for (int rb = 0; rb < RB; ++rb)
#pragma unroll
      for (int nb = 0; nb < NB; ++nb)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[rb][nb][i] = 0.f;

    const int nch = d.K / kChunk;
    uint4 wb[kDepth][RB][2][P];
#pragma unroll
    for (int s = 0; s < kDepth; ++s)
      if (s < nch)
#pragma unroll
        for (int rb = 0; rb < RB; ++rb)
#pragma unroll
          for (int hh = 0; hh < 2; ++hh)
#pragma unroll
            for (int pp = 0; pp < P; ++pp) wb[s][rb][hh][pp] = ld_stream_u4(wr[rb][hh] + s * kChunk + 16 * pp);

    for (int c0 = 0; c0 < nch; c0 += kDepth) {
#pragma unroll
      for (int s = 0; s < kDepth; ++s) {
        const int c = c0 + s;
        if (c < nch) {
          const uint4 (&w)[RB][2][P] = wb[s];
          // x[m][kChunk c + kSeg q .. + kSeg - 1] (fp16): words 2j, 2j+1 feed MMA j
          uint4 xs[NB][2 * P];
#pragma unroll
          for (int nb = 0; nb < NB; ++nb)
#pragma unroll
            for (int i = 0; i < 2 * P; ++i) {
              xs[nb][i] = make_uint4(0u, 0u, 0u, 0u);
              if (xv_ok[nb]) {
                const uint4 *xp = reinterpret_cast<const uint4 *>(xr[nb] + c * kChunk) + i;
                xs[nb][i] = d.dep < 0 ? __ldg(xp) : __ldcg(xp);  // written earlier in this launch: from L2
              }
            }
#pragma unroll
          for (int j = 0; j < 4 * P; ++j) {
            uint32_t b0[NB], b1[NB];
#pragma unroll
            for (int nb = 0; nb < NB; ++nb) {
              b0[nb] = u4_word(xs[nb][j >> 1], (2 * j) & 3);
              b1[nb] = u4_word(xs[nb][j >> 1], (2 * j + 1) & 3);
            }
#pragma unroll
            for (int rb = 0; rb < RB; ++rb) {
              // exact int8 -> fp16 pairs: K kSeg q + 4j + {0,1} and + {2,3} of rows g8, g8+8
              const uint32_t lo = u4_word(w[rb][0][j >> 2], j & 3) ^ 0x80808080u;
              const uint32_t hi = u4_word(w[rb][1][j >> 2], j & 3) ^ 0x80808080u;
              const uint32_t a0 = i8x2_to_f16x2(lo, 0x5150u), a2 = i8x2_to_f16x2(lo, 0x5352u);
              const uint32_t a1 = i8x2_to_f16x2(hi, 0x5150u), a3 = i8x2_to_f16x2(hi, 0x5352u);
#pragma unroll
              for (int nb = 0; nb < NB; ++nb) mma_16816(acc[rb][nb], a0, a1, a2, a3, b0[nb], b1[nb]);
            }
          }
          // the slot is consumed: refill it with chunk c + depth
          if (c + kDepth < nch) {
#pragma unroll
            for (int rb = 0; rb < RB; ++rb)
#pragma unroll
              for (int hh = 0; hh < 2; ++hh)
#pragma unroll
                for (int pp = 0; pp < P; ++pp)
                  wb[s][rb][hh][pp] = ld_stream_u4(wr[rb][hh] + (c + kDepth) * kChunk + 16 * pp);
          }
        }
      }
    }

    // epilogue: lane holds D[row g8 (+8)][batch 2q, 2q+1] of each block
#pragma unroll
    for (int rb = 0; rb < RB; ++rb)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int n = row0 + 16 * rb + 8 * hh + g8;
        if (n < d.N) {
          const float sc = __half2float(d.scale[n]);
          const float bs = d.bias ? __half2float(d.bias[n]) : 0.f;
#pragma unroll
          for (int nb = 0; nb < NB; ++nb)
#pragma unroll
            for (int cc = 0; cc < 2; ++cc) {
              const int m = 8 * nb + 2 * q + cc;
              if (m < p.M)
                d.y[static_cast<int64_t>(m) * d.ldy + n] = __float2half_rn(acc[rb][nb][2 * hh + cc] * sc + bs);
            }
        }
      }
    if (d.signal) {  // this warp's y stores, then the count
      __syncwarp();
      if (lane == 0) {
        asm volatile("fence.acq_rel.gpu;" ::: "memory");
        red_release_gpu_add(p.counters + g, 1);
      }
    }
  }
}

}  // namespace hx
