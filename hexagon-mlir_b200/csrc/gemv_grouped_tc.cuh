// gemv_grouped_tc.cuh — a decode step's W8A16 projections in one persistent
// launch, on the tcgen05 tensor cores.
//
// Same contract as hx_gemv_w8a16_grouped_kernel (gemv_grouped.cuh): a list of
// projections y_g[M, N_g] = x_g[M, K_g] . (W_g * scale_g)^T (+ bias_g), W int8
// per-output-channel, x / y / scale / bias fp16, fp32 accumulation, optional
// dependencies (x_g is the y of an earlier projection).  On CUDA cores the
// dequantise-and-multiply costs several instructions per weight byte, which
// caps that kernel near 40% of HBM bandwidth; here the weights only pass
// through an exact int8 -> fp16 conversion and the products run on the tensor
// cores with the operands swapped (as in w8a16_sm100.cuh):
//   D^T[n, m] = W[n, :] . x[m, :]   (UMMA M = 128 weight rows, N = M padded
//                                    to 16, 32 or 64)
//
// Work item = (projection g, block of 128 weight rows); CTA c of the
// persistent grid (one per SM) takes items c, c + grid, ...  Roles (448 threads):
//   warp 0      producer: one 3-D TMA load per 4 K blocks (128 rows x 512 B =
//               64 KB of int8) into a 2-stage ring; never waits on
//               dependencies, so the weight stream runs ahead of the math
//   warp 1      TMEM allocator + UMMA issuer (2 accumulators of N columns)
//   warps 2..9  converters (two per row quarter, half a row each):
//               int8 (TMA 128B-swizzled) -> fp16 A tile, and the x rows of the
//               K block -> fp16 B tile (rows >= M zero), both 128B-swizzled
//               K-major; a dependent projection first waits (bounded,
//               acquire) on its producer projection's counter.  Eight
//               warps, two per scheduler, hide the shared-memory latency of
//               the conversion (measured: 4 -> 8 warps +48%, 16 warps slower)
//   warps 10..13 epilogue: TMEM -> scale, bias -> y; then, if a later
//               projection depends on this one, a release-add on its counter
// Reference counterpart: dequantise + matmul (lib/Conversion/LinalgToLLVM/
// LinalgToLLVMPass.cpp:203-209); the conversion is exact and the scale is a
// row factor of D^T, so results equal dequantise-then-fp32-matmul up to
// summation order.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "gemv_grouped.cuh"
#include "ptx.cuh"
#include "w8a16_sm100.cuh"

namespace hx {

constexpr int kGtMaxProj = 156;                          // projections per launch (param space)
constexpr int kGtConvWarps = 8;
constexpr int kGtThreads = (2 + kGtConvWarps + 4) * 32;
constexpr int kGtMaxM = 64;                              // largest batch (UMMA N <= 64)
constexpr int kGtKbStage = 4;                            // 128-byte K blocks per W stage
constexpr int kGtWStages = 2;
constexpr int kGtCStages = 2;
constexpr int kGtWStageBytes = kGtKbStage * 128 * 128;   // 64 KB of int8 W
constexpr int kGtABytes = 2 * 128 * 128;                 // fp16 W, 128 rows x 128 K
constexpr int kGtEpiWarps = 4;

// MPAD: the batch M padded to the UMMA N (16, 32 or 64).
template <int MPAD>
struct GtCfg {
  static constexpr int kXBytes = 2 * MPAD * 128;                  // fp16 x, MPAD rows x 128 K
  static constexpr int kCStageBytes = kGtABytes + kXBytes;        // 36 / 40 / 48 KB
  static constexpr int kSmemBytes = kGtWStages * kGtWStageBytes + kGtCStages * kCStageBytes + 1024 + 256;
  static constexpr uint32_t kIdesc = make_idesc(0, false, 128, MPAD);
  static constexpr int kTmemCols = 2 * MPAD < 32 ? 32 : 2 * MPAD;  // two accumulators
  static constexpr int kXPieces = MPAD * 16 / 256;                // 16-byte x pieces per converter thread
  static_assert(MPAD == 16 || MPAD == 32 || MPAD == 64, "MPAD");
  static_assert(kSmemBytes <= 232448, "shared memory");
};

struct GtDesc {
  const __half *x;
  const __half *scale;
  const __half *bias;
  __half *y;
  int32_t N, K, ldx, ldy;
  int32_t dep;          // index of the projection whose y is this x, or -1
  int32_t item_begin;   // first global item of this projection
  int32_t kblocks;      // K / 128
  int32_t signal;       // 1 if a later projection depends on this one
};

struct GtParams {
  CUtensorMap tmW[kGtMaxProj];  // 3-D {128 B, N rows, K / 128}, box {128, 128, 4}, 128B swizzle
  GtDesc d[kGtMaxProj];
  int32_t G, M, total_items, pad;
  int32_t *counters;            // [G] completed (item, epilogue warp) pairs; zeroed by the host
  int32_t *err_flag;
  uint64_t timeout;
};

__device__ __forceinline__ int gt_find(const GtParams &p, int item) {
  int lo = 0, hi = p.G - 1;
  while (lo < hi) {  // last g with item_begin <= item
    const int mid = (lo + hi + 1) >> 1;
    if (p.d[mid].item_begin <= item) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

#ifdef HX_GT_PROF
__device__ unsigned long long g_gt_prof[1024][8];
#define GT_T0() const long long gt_t0_ = clock64()
#define GT_ACC(slot) atomicAdd(&g_gt_prof[blockIdx.x][slot], (unsigned long long)(clock64() - gt_t0_))
#define GT_WAIT(slot, expr) ([&]() { GT_T0(); const bool r_ = (expr); GT_ACC(slot); return r_; }())
#else
#define GT_WAIT(slot, expr) (expr)
#define GT_T0() \
  do {          \
  } while (0)
#define GT_ACC(slot) \
  do {               \
  } while (0)
#endif

__device__ __forceinline__ void gt_fail(volatile int *abort_flag, int32_t *err, int code) {
  *abort_flag = 1;
  if (err) atomicExch(err, code);
}

template <int MPAD>
__global__ void __launch_bounds__(kGtThreads, 1)
    hx_gemv_w8a16_grouped_tc_kernel(const __grid_constant__ GtParams p) {
  using Cfg = GtCfg<MPAD>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t *wring = smem;
  uint8_t *cring = smem + kGtWStages * kGtWStageBytes;
  uint64_t *wfull = reinterpret_cast<uint64_t *>(cring + kGtCStages * Cfg::kCStageBytes);
  uint64_t *wempty = wfull + kGtWStages;   // converters finished a W stage (8 arrivals)
  uint64_t *cfull = wempty + kGtWStages;   // converted A + x ready (8 arrivals)
  uint64_t *cempty = cfull + kGtCStages;   // UMMAs finished reading (commit)
  uint64_t *tfull = cempty + kGtCStages;   // [2] accumulator ready (commit)
  uint64_t *tempty = tfull + 2;            // [2] epilogue read the accumulator (4 arrivals)
  uint64_t *drain = tempty + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kGtWStages; ++s) {
      mbar_init(&wfull[s], 1);
      mbar_init(&wempty[s], kGtConvWarps);
    }
    for (int s = 0; s < kGtCStages; ++s) {
      mbar_init(&cfull[s], kGtConvWarps);
      mbar_init(&cempty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], kGtEpiWarps);
    }
    mbar_init(drain, 1);
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
  grid_dep_wait();  // counters zeroed and inputs written by the preceding work
#ifdef HX_GT_PROF
  const long long gt_start_ = clock64();
#endif

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int ws = 0;
      uint32_t wph = 0;
      uint32_t last_phase[kGtWStages];  // phase of each stage's latest load
      bool issued[kGtWStages];
      for (int i = 0; i < kGtWStages; ++i) issued[i] = false;
      bool ok = true;
      for (int t = 0; ok; ++t) {
        const int item = blockIdx.x + t * gridDim.x;
        if (item >= p.total_items) break;
        const int g = gt_find(p, item);
        const GtDesc &d = p.d[g];
        const int row0 = (item - d.item_begin) * 128;
        if (t == 0) tma_prefetch_desc(&p.tmW[g]);
        for (int kb = 0; kb < d.kblocks; kb += kGtKbStage) {
          if (!GT_WAIT(0, mbar_wait(&wempty[ws], wph ^ 1, p.timeout, abort_flag))) {
            gt_fail(abort_flag, p.err_flag, 31);
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&wfull[ws], kGtWStageBytes);  // OOB parts of the box are zero-filled
          tma_load_3d(wring + ws * kGtWStageBytes, &p.tmW[g], &wfull[ws], 0, row0, kb);
          issued[ws] = true;
          last_phase[ws] = wph;
          if (++ws == kGtWStages) {
            ws = 0;
            wph ^= 1;
          }
        }
      }
      if (!ok) {  // let the loads still in flight land before the CTA exits
        int ignored = 0;
        for (int i = 0; i < kGtWStages; ++i)
          if (issued[i]) mbar_wait(&wfull[i], last_phase[i], p.timeout, &ignored);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ UMMA issuer
    int cs = 0;
    uint32_t cph = 0;
    bool ok = true, any = false;
    for (int t = 0; ok; ++t) {
      const int item = blockIdx.x + t * gridDim.x;
      if (item >= p.total_items) break;
      const GtDesc &d = p.d[gt_find(p, item)];
      const int acc = t & 1;
      bool w = (lane == 0) ? GT_WAIT(1, mbar_wait(&tempty[acc], ((t >> 1) & 1) ^ 1, p.timeout, abort_flag)) : true;
      w = __shfl_sync(0xffffffffu, w, 0);
      if (!w) {
        if (lane == 0) gt_fail(abort_flag, p.err_flag, 32);
        ok = false;
        break;
      }
      tc_fence_after();
      for (int kb = 0; kb < d.kblocks; ++kb) {
        w = (lane == 0) ? GT_WAIT(2, mbar_wait(&cfull[cs], cph, p.timeout, abort_flag)) : true;
        w = __shfl_sync(0xffffffffu, w, 0);
        if (!w) {
          if (lane == 0) gt_fail(abort_flag, p.err_flag, 33);
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t a_base = smem_u32(cring + cs * Cfg::kCStageBytes);
          const uint32_t b_base = a_base + kGtABytes;
#pragma unroll
          for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int k = 0; k < 4; ++k)
              umma_f16(tmem_base + acc * MPAD, sdesc_kmajor_sw128(a_base + h * (128 * 128) + k * 32),
                       sdesc_kmajor_sw128(b_base + h * (MPAD * 128) + k * 32), Cfg::kIdesc,
                       (kb > 0 || h > 0 || k > 0) ? 1u : 0u);
          umma_commit(&cempty[cs]);
          any = true;
        }
        __syncwarp();
        if (++cs == kGtCStages) {
          cs = 0;
          cph ^= 1;
        }
      }
      if (ok && lane == 0) umma_commit(&tfull[acc]);
      __syncwarp();
    }
    if (!ok && any && lane == 0) {  // every issued UMMA completes before TMEM is freed
      umma_commit(drain);
      int ignored = 0;
      mbar_wait(drain, 0, p.timeout, &ignored);
    }
  } else if (warp < 2 + kGtConvWarps) {
    // ------------------------------------------------------------ converters
    constexpr int kCPT = 8 * 4 / kGtConvWarps;  // 16-byte chunks of a row per thread
    const int cw = warp - 2;                // 0 .. kGtConvWarps-1
    const int r = (cw & 3) * 32 + lane;     // weight row this thread converts
    const int c_lo = (cw >> 2) * kCPT;      // its chunks of the row: c_lo .. c_lo+kCPT-1
    const int tid = cw * 32 + lane;         // < 256: one 16-byte piece of the K block's x tile
    int ws = 0, cs = 0;
    uint32_t wph = 0, cph = 0;
    bool ok = true;
    for (int t = 0; ok; ++t) {
      const int item = blockIdx.x + t * gridDim.x;
      if (item >= p.total_items) break;
      const GtDesc &d = p.d[gt_find(p, item)];
      if (d.dep >= 0) {  // x is an earlier projection's y: wait until all of it is stored
        const GtDesc &dd = p.d[d.dep];
        const int target = ((dd.N + 127) / 128) * kGtEpiWarps;
        bool w = true;
        if (lane == 0) {
          const uint64_t t0 = clock64();
          while (ld_acquire_gpu(p.counters + d.dep) < target) {
            if (*abort_flag || static_cast<uint64_t>(clock64() - t0) > p.timeout) {
              w = false;
              break;
            }
            __nanosleep(64);
          }
        }
        w = __shfl_sync(0xffffffffu, w, 0);
        if (!w) {
          if (lane == 0) gt_fail(abort_flag, p.err_flag, 34);
          ok = false;
          break;
        }
      }
      for (int kb0 = 0; kb0 < d.kblocks && ok; kb0 += kGtKbStage) {
        bool w = (lane == 0) ? GT_WAIT(3, mbar_wait(&wfull[ws], wph, p.timeout, abort_flag)) : true;
        w = __shfl_sync(0xffffffffu, w, 0);
        if (!w) {
          if (lane == 0) gt_fail(abort_flag, p.err_flag, 35);
          ok = false;
          break;
        }
        const int nk = min(kGtKbStage, d.kblocks - kb0);
        for (int j = 0; j < nk; ++j) {
          // this thread's x piece: through L1 when x predates the launch, else
          // coherent from L2; its latency overlaps the slot wait and conversion
          uint4 xv[Cfg::kXPieces];
#pragma unroll
          for (int i = 0; i < Cfg::kXPieces; ++i) {
            const int pc = tid + i * 256;
            const int xm = pc >> 4, xh = (pc >> 3) & 1, xc = pc & 7;
            xv[i] = make_uint4(0u, 0u, 0u, 0u);
            if (xm < p.M) {
              const uint4 *xp = reinterpret_cast<const uint4 *>(
                  d.x + static_cast<int64_t>(xm) * d.ldx + (kb0 + j) * 128 + xh * 64 + xc * 8);
              xv[i] = d.dep < 0 ? __ldg(xp) : __ldcg(xp);
            }
          }
          w = (lane == 0) ? GT_WAIT(4, mbar_wait(&cempty[cs], cph ^ 1, p.timeout, abort_flag)) : true;
          w = __shfl_sync(0xffffffffu, w, 0);
          if (!w) {
            if (lane == 0) gt_fail(abort_flag, p.err_flag, 36);
            ok = false;
            break;
          }
          uint8_t *cst = cring + cs * Cfg::kCStageBytes;
          // weight row r, chunks c_lo.. : int8 (TMA 128B-swizzled) -> fp16 in the
          // 64-K half c_lo / 4
          const uint8_t *raw = wring + ws * kGtWStageBytes + j * (128 * 128) + r * 128;
          uint8_t *dst = cst + (c_lo >> 2) * (128 * 128) + r * 128;
#pragma unroll
          for (int ci = 0; ci < kCPT; ++ci) {
            const int c = c_lo + ci;
            const uint4 wv = *reinterpret_cast<const uint4 *>(raw + ((c ^ (r & 7)) << 4));
            uint4 lo, hi;
            i8x16_to_f16(wv, lo, hi);
            const int j0 = (c & 3) * 2;
            *reinterpret_cast<uint4 *>(dst + ((j0 ^ (r & 7)) << 4)) = lo;
            *reinterpret_cast<uint4 *>(dst + (((j0 + 1) ^ (r & 7)) << 4)) = hi;
          }
          // x rows of this K block (fp16, MPAD rows x 2 halves x 8 chunks; rows >= M zero)
#pragma unroll
          for (int i = 0; i < Cfg::kXPieces; ++i) {
            const int pc = tid + i * 256;
            const int xm = pc >> 4, xh = (pc >> 3) & 1, xc = pc & 7;
            *reinterpret_cast<uint4 *>(cst + kGtABytes + xh * (MPAD * 128) + xm * 128 +
                                       ((xc ^ (xm & 7)) << 4)) = xv[i];
          }
          fence_proxy_async_smem();  // generic smem writes -> visible to the UMMAs
          __syncwarp();
          if (lane == 0) mbar_arrive(&cfull[cs]);
          if (++cs == kGtCStages) {
            cs = 0;
            cph ^= 1;
          }
        }
        if (!ok) break;
        __syncwarp();
        if (lane == 0) mbar_arrive(&wempty[ws]);
        if (++ws == kGtWStages) {
          ws = 0;
          wph ^= 1;
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    for (int t = 0;; ++t) {
      const int item = blockIdx.x + t * gridDim.x;
      if (item >= p.total_items) break;
      const int g = gt_find(p, item);
      const GtDesc &d = p.d[g];
      const int acc = t & 1;
      bool w = (lane == 0) ? GT_WAIT(5, mbar_wait(&tfull[acc], (t >> 1) & 1, p.timeout, abort_flag)) : true;
      w = __shfl_sync(0xffffffffu, w, 0);
      if (!w) {
        if (lane == 0) gt_fail(abort_flag, p.err_flag, 37);
        break;
      }
      tc_fence_after();
      const int n = (item - d.item_begin) * 128 + q * 32 + lane;
      const float sc = n < d.N ? __half2float(d.scale[n]) : 0.f;
      const float b = (n < d.N && d.bias) ? __half2float(d.bias[n]) : 0.f;
#pragma unroll
      for (int c = 0; c < MPAD / 16; ++c) {
        if (c * 16 >= p.M) break;
        uint32_t v[16];
        tmem_ld_32x32b_x16(tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * MPAD + c * 16, v);
        tmem_ld_wait();
        if (n < d.N) {
#pragma unroll
          for (int m = 0; m < 16; ++m)
            if (c * 16 + m < p.M)
              d.y[static_cast<int64_t>(c * 16 + m) * d.ldy + n] = __float2half_rn(__uint_as_float(v[m]) * sc + b);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);  // the accumulator may be reused
      if (d.signal) {  // this warp's y stores, then one count
        __syncwarp();
        if (lane == 0) {
          asm volatile("fence.acq_rel.gpu;" ::: "memory");
          red_release_gpu_add(p.counters + g, 1);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
#ifdef HX_GT_PROF
  if (threadIdx.x == 0) atomicAdd(&g_gt_prof[blockIdx.x][6], (unsigned long long)(clock64() - gt_start_));
#endif
  if (warp == 1) tmem_dealloc(tmem_base, Cfg::kTmemCols);
}

}  // namespace hx
