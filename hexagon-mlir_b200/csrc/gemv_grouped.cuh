// gemv_grouped.cuh — many W8A16 decode projections in one persistent launch.
//
// A decode step is a chain of skinny GEMMs (22 layers x 7 projections for
// the TinyLlama shapes), each only a few MB of int8 weights.  Launched one by
// one, every projection pays a dependent-launch latency that is larger than
// its HBM time.  Here one persistent grid walks the whole list:
//   * work item = (projection g, block of R weight rows); items are numbered
//     in list order and CTA c takes items c, c + grid, c + 2*grid, ...;
//   * each CTA keeps a ring of D shared-memory slots; thread 0 bulk-copies
//     the weight rows of its next D items ahead of use, so the weight stream
//     from HBM never waits on compute or on dependencies;
//   * projection g may read the output of an earlier projection dep(g): before
//     reading x, the CTA waits (bounded spin, acquire) until every row block of
//     dep(g) has signalled completion through a counter in `counters`;
//   * the counters are the only scratch; the host zeroes them before launch.
// Progress: the lowest-numbered unfinished item only depends on lower-
// numbered items, which are finished, and its CTA has nothing earlier left
// to do, so it proceeds (all CTAs of the persistent grid are resident).
//
// Reference counterpart: the same per-projection math as hx_gemv_w8a16
// (dequantise-then-matmul, lib/Conversion/LinalgToLLVM/LinalgToLLVMPass.cpp:
// 203-209); the grouping is B200-side scheduling with no reference analogue.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

#include "gemv_w8a16.cuh"
#include "ptx.cuh"
#include "w8a16_sm100.cuh"

namespace hx {

constexpr int kGroupMax = 256;       // projections per launch
constexpr int kGroupSlotBytes = 56 * 1024;
constexpr int kGroupSlots = 2;       // ring depth (two CTAs per SM)
constexpr int kGroupThreads = 256;  // compute threads (a producer warp is added)

struct GroupDesc {
  const int8_t *W;
  const __half *scale;
  const __half *bias;
  const __half *x;
  __half *y;
  int32_t N, K, ldw, ldx, ldy;
  int32_t dep;          // index of the projection whose y is this x, or -1
  int32_t item_begin;   // first global item number of this projection
  int32_t rows;         // R: weight rows per item (R * K <= slot bytes, R * MC <= 32)
  int32_t signal;       // 1 if a later projection depends on this one
  int32_t x_in_slot;    // x (M x K fp16) is staged in the slot after the weights
};

struct GroupParams {
  int32_t G, M, total_items;
  int32_t *counters;    // [G] completed row blocks per projection (zeroed)
  int32_t *err_flag;    // optional
  uint64_t timeout;     // cycles per bounded wait
  GroupDesc d[kGroupMax];
};

__device__ __forceinline__ int group_find(const GroupParams &p, int item) {
  int lo = 0, hi = p.G - 1;
  while (lo < hi) {  // last g with item_begin <= item
    const int mid = (lo + hi + 1) >> 1;
    if (p.d[mid].item_begin <= item) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

// c + a.lo * b.lo + a.hi * b.hi for fp16 pairs a, b, accumulated in fp32
// (fma.rn.f32.f16: the fp16 product is exact in fp32, one rounding per step).
__device__ __forceinline__ float fma2_f16_f32(uint32_t a2, uint32_t b2, float c) {
  float d;
  asm("{\n\t.reg .f16 al, ah, bl, bh;\n\t.reg .f32 t;\n\t"
      "mov.b32 {al, ah}, %1;\n\tmov.b32 {bl, bh}, %2;\n\t"
      "fma.rn.f32.f16 t, al, bl, %3;\n\tfma.rn.f32.f16 %0, ah, bh, t;\n\t}"
      : "=f"(d)
      : "r"(a2), "r"(b2), "f"(c));
  return d;
}

__device__ __forceinline__ int ld_acquire_gpu(const int32_t *p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_gpu_add(int32_t *p, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Warp roles: warps 0..7 compute, warp 8 produces.  For item t (slot t % D):
//   producer  waits empty[slot] (every compute warp released it), then
//             bulk-copies the item's R weight rows (one copy when the rows are
//             contiguous) into the slot;
//   compute   warp w waits full[slot] (and, for a dependent projection, the
//             producer projection's counter), computes rows [w*R/8, (w+1)*R/8)
//             for all M batch rows with lanes striding over K, releases the
//             slot, reduces across lanes, scales and stores y, and, when a
//             later projection depends on this one, signals the counter.
constexpr int kGroupComputeWarps = kGroupThreads / 32;

template <int MC, int RMAX>
__global__ void __launch_bounds__(kGroupThreads + 32, 2)
    hx_gemv_w8a16_grouped_kernel(const __grid_constant__ GroupParams p) {
  extern __shared__ __align__(16) uint8_t gsm[];
  uint64_t *full = reinterpret_cast<uint64_t *>(gsm + kGroupSlots * kGroupSlotBytes);
  uint64_t *empty = full + kGroupSlots;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kGroupSlots; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kGroupComputeWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();
  grid_dep_launch_dependents();
  grid_dep_wait();  // counters were zeroed by the preceding memset

  int dummy_abort = 0;
  if (warp == kGroupComputeWarps) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      for (int t = 0;; ++t) {
        const int item = blockIdx.x + t * gridDim.x;
        if (item >= p.total_items) break;
        const GroupDesc &d = p.d[group_find(p, item)];
        const int row0 = (item - d.item_begin) * d.rows;
        const int nrows = min(d.rows, d.N - row0);
        const int s = t % kGroupSlots;
        if (!mbar_wait(&empty[s], static_cast<uint32_t>(((t / kGroupSlots) & 1) ^ 1), p.timeout,
                       &dummy_abort)) {
          if (p.err_flag) atomicExch(p.err_flag, 22);
          break;
        }
        uint8_t *dst = gsm + s * kGroupSlotBytes;
        const uint32_t xbytes = static_cast<uint32_t>(p.M) * d.K * 2;
        const bool x_now = d.x_in_slot && d.dep < 0;
        // one arrival per phase, expecting the weight rows and (maybe) x
        mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(nrows) * d.K + (x_now ? xbytes : 0u));
        if (x_now) {
          uint8_t *xdst = dst + ((static_cast<uint32_t>(d.rows) * d.K + 15) & ~15u);
          if (d.ldx == d.K)
            bulk_load_1d(xdst, d.x, xbytes, &full[s]);
          else
            for (int m = 0; m < p.M; ++m)
              bulk_load_1d(xdst + m * d.K * 2, d.x + static_cast<int64_t>(m) * d.ldx, d.K * 2, &full[s]);
        }
        if (d.ldw == d.K) {  // the item's rows are one contiguous block
          bulk_load_1d(dst, d.W + static_cast<int64_t>(row0) * d.K, static_cast<uint32_t>(nrows) * d.K,
                       &full[s]);
        } else {
          for (int r = 0; r < nrows; ++r)
            bulk_load_1d(dst + r * d.K, d.W + static_cast<int64_t>(row0 + r) * d.ldw, d.K, &full[s]);
        }
      }
    }
    return;  // the producer takes no part in the compute warps' barriers
  }

  // ------------------------------------------------------------ compute
  for (int t = 0;; ++t) {
    const int item = blockIdx.x + t * gridDim.x;
    if (item >= p.total_items) break;
    const int g = group_find(p, item);
    const GroupDesc &d = p.d[g];
    const int s = t % kGroupSlots;
    const uint8_t *wsm = gsm + s * kGroupSlotBytes;
    const int row0 = (item - d.item_begin) * d.rows;
    const int nrows = min(d.rows, d.N - row0);
    const int R = d.rows;

    bool ok = true;
    if (lane == 0) {
      ok = mbar_wait(&full[s], static_cast<uint32_t>((t / kGroupSlots) & 1), p.timeout, &dummy_abort);
      if (ok && d.dep >= 0) {
        const GroupDesc &dd = p.d[d.dep];
        // every compute warp of every item of the producer projection signals once
        const int target = ((dd.N + dd.rows - 1) / dd.rows) * kGroupComputeWarps;
        const uint64_t t0 = clock64();
        while (ld_acquire_gpu(p.counters + d.dep) < target) {
          if (static_cast<uint64_t>(clock64() - t0) > p.timeout) {
            ok = false;
            break;
          }
          __nanosleep(32);
        }
      }
      if (!ok && p.err_flag) atomicExch(p.err_flag, 21);
    }
    ok = __shfl_sync(0xffffffffu, ok, 0);

    // x: staged in the slot (by the producer, or here for a dependent
    // projection once its input is complete), else read from L2.
    const __half *xs = d.x;
    int64_t ldxs = d.ldx;
    if (d.x_in_slot) {
      __half *xslot = reinterpret_cast<__half *>(
          const_cast<uint8_t *>(wsm) + ((static_cast<uint32_t>(d.rows) * d.K + 15) & ~15u));
      if (d.dep >= 0) {
        asm volatile("bar.sync 1, %0;" ::"n"(kGroupThreads) : "memory");  // every warp saw the counter
        const int per_row = d.K / 8;  // uint4 per batch row
        for (int i = threadIdx.x; i < p.M * per_row; i += kGroupThreads) {
          const int m = i / per_row, c = i % per_row;
          reinterpret_cast<uint4 *>(xslot + m * d.K)[c] =
              __ldcg(reinterpret_cast<const uint4 *>(d.x + static_cast<int64_t>(m) * d.ldx) + c);
        }
        asm volatile("bar.sync 1, %0;" ::"n"(kGroupThreads) : "memory");
      }
      xs = xslot;
      ldxs = d.K;
    }
    // Warp w owns rows [w*rpw, (w+1)*rpw) of the item; lanes stride over K.
    const int rpw = R / kGroupComputeWarps;
    const int kvec = d.K / 16;
    float acc[RMAX][MC];
#pragma unroll
    for (int r = 0; r < RMAX; ++r)
#pragma unroll
      for (int m = 0; m < MC; ++m) acc[r][m] = 0.f;
    if (ok) {
      for (int kv = lane; kv < kvec; kv += 32) {
        uint4 wv[RMAX];
#pragma unroll
        for (int r = 0; r < RMAX; ++r)
          if (r < rpw) wv[r] = *reinterpret_cast<const uint4 *>(wsm + (warp * rpw + r) * d.K + kv * 16);
        // four weights (one 32-bit word per row) at a time keeps MC x 4 x-values live
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint2 xh[MC];  // four fp16 x values of batch row m
#pragma unroll
          for (int m = 0; m < MC; ++m) {
            xh[m] = make_uint2(0, 0);
            // shared memory, or L2-coherent global loads (x may have been
            // written earlier in this launch)
            if (m < p.M) {
              const uint2 *xp = reinterpret_cast<const uint2 *>(xs + m * ldxs + kv * 16 + q * 4);
              xh[m] = d.x_in_slot ? *xp : __ldcg(xp);
            }
          }
#pragma unroll
          for (int r = 0; r < RMAX; ++r) {
            if (r >= rpw) break;
            const uint32_t word = q == 0 ? wv[r].x : (q == 1 ? wv[r].y : (q == 2 ? wv[r].z : wv[r].w));
            // exact int8 -> fp16 pairs (weights 0,1 and 2,3), then fp16 x fp16
            // products (exact in fp32) accumulated in fp32: the same numbers as
            // fmaf on the converted floats, in half the instructions
            const uint32_t u = word ^ 0x80808080u;
            const uint32_t w01 = i8x2_to_f16x2(u, 0x5150u);
            const uint32_t w23 = i8x2_to_f16x2(u, 0x5352u);
#pragma unroll
            for (int m = 0; m < MC; ++m)
              acc[r][m] = fma2_f16_f32(w23, xh[m].y, fma2_f16_f32(w01, xh[m].x, acc[r][m]));
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);  // this warp is done with the slot
#pragma unroll
    for (int r = 0; r < RMAX; ++r) {
      if (r >= rpw) break;
#pragma unroll
      for (int m = 0; m < MC; ++m) {
        float v = acc[r][m];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        acc[r][m] = v;
      }
      const int rr = warp * rpw + r;
      if (lane == 0 && ok && rr < nrows) {
        const int n = row0 + rr;
        const float sc = __half2float(d.scale[n]);
        const float b = d.bias ? __half2float(d.bias[n]) : 0.f;
#pragma unroll
        for (int m = 0; m < MC; ++m)
          if (m < p.M) d.y[static_cast<int64_t>(m) * d.ldy + n] = __float2half_rn(acc[r][m] * sc + b);
      }
    }
    if (d.signal && lane == 0) {  // per-warp completion: its y stores, then the count
      asm volatile("fence.acq_rel.gpu;" ::: "memory");
      red_release_gpu_add(p.counters + g, 1);
    }
  }
}

}  // namespace hx
