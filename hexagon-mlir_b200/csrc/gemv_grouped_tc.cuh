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
//   warp 0      producer: one 3-D TMA load per KBS K blocks (128 rows x 128 B
//               each) into a 128 KB int8 ring; never waits on dependencies,
//               so the weight stream runs ahead of the math
//   warp 1      TMEM allocator + UMMA issuer: per K block, eight
//               tcgen05.mma (M = 128, N = MPAD, K = 16) with A read from TMEM
//               and B (x) from shared memory, into one of 2 accumulators
//   warps 2..9  converters in two groups of four warps (one per TMEM lane
//               quarter): group h converts the 64-K half h of every K block,
//               one weight row per thread, int8 (TMA 128B-swizzled, shared
//               memory) -> fp16 in registers -> tcgen05.st into a ring of
//               4-6 TMEM A stages (64 columns each); it also copies its half of
//               the K block's x rows into the matching shared-memory B stage
//               (rows >= M zero); a dependent projection first waits
//               (bounded, acquire) on its producer projection's counter
//   warps 10..13 epilogue: TMEM -> scale, bias -> y; then, if a later
//               projection depends on this one, a release-add on its counter
// Keeping the converted weights in TMEM removes their shared-memory round
// trip: with A in shared memory, every N = 16 MMA re-reads a 4 KB A slice
// there, and the MMA issue rate, not HBM, bounded the launch.
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
constexpr int kGtWRingBytes = 128 * 1024;                // int8 W ring
constexpr int kGtTmemCols = 512;
constexpr int kGtEpiWarps = 4;

// MPAD: the batch M padded to the UMMA N (16, 32 or 64); KBS: 128-byte K
// blocks per W stage (one TMA instruction), the ring holding 8 / KBS stages;
// NACC: accumulators per item, taken in turn by consecutive MMAs so that
// back-to-back N = MPAD MMAs do not wait on one another's accumulator.
template <int MPAD, int KBS, int NACC>
struct GtCfg {
  static constexpr int kKbStage = KBS;
  static constexpr int kWStageBytes = KBS * 128 * 128;
  static constexpr int kWStages = kGtWRingBytes / kWStageBytes;
  static constexpr int kAccCols = NACC * MPAD;                    // one item's accumulators
  static constexpr int kAColBase = 2 * kAccCols < 128 ? 128 : 2 * kAccCols;  // A ring after two items' accumulators
  static constexpr int kAStages = (kGtTmemCols - kAColBase) / 64 > 6 ? 6 : (kGtTmemCols - kAColBase) / 64;
  static constexpr int kXBytes = 2 * MPAD * 128;                  // fp16 x, MPAD rows x 128 K (two 64-K tiles)
  static constexpr int kSmemBytes = kGtWRingBytes + kAStages * kXBytes + 1024 + 256;
  static constexpr uint32_t kIdesc = make_idesc(0, false, 128, MPAD);
  static constexpr int kXPieces = MPAD * 8 / 128;                 // 16-byte x pieces per converter thread
  static_assert(MPAD == 16 || MPAD == 32 || MPAD == 64, "MPAD");
  static_assert(NACC == 1 || NACC == 2 || NACC == 4, "NACC");
  static_assert(kAStages >= 3, "TMEM A ring");
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

__device__ __forceinline__ void gt_fail(volatile int *abort_flag, int32_t *err, int code) {
  *abort_flag = 1;
  if (err) atomicExch(err, code);
}

template <int MPAD, int KBS, int NACC>
__global__ void __launch_bounds__(kGtThreads, 1)
    hx_gemv_w8a16_grouped_tc_kernel(const __grid_constant__ GtParams p) {
  using Cfg = GtCfg<MPAD, KBS, NACC>;
  constexpr int NA = Cfg::kAStages;
  constexpr int kGtAColBase = Cfg::kAColBase;
  constexpr int kKbStage = Cfg::kKbStage;
  constexpr int kWStages = Cfg::kWStages;
  constexpr int kWStageBytes = Cfg::kWStageBytes;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t *wring = smem;
  uint8_t *xring = smem + kGtWRingBytes;
  uint64_t *wfull = reinterpret_cast<uint64_t *>(xring + NA * Cfg::kXBytes);
  uint64_t *wempty = wfull + kWStages;     // converters finished a W stage (8 arrivals)
  uint64_t *cfull = wempty + kWStages;     // A stage (TMEM) + x stage (smem) ready (8 arrivals)
  uint64_t *cempty = cfull + NA;           // UMMAs finished reading them (commit)
  uint64_t *tfull = cempty + NA;           // [2] accumulator ready (commit)
  uint64_t *tempty = tfull + 2;            // [2] epilogue read the accumulator (4 arrivals)
  uint64_t *drain = tempty + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kWStages; ++s) {
      mbar_init(&wfull[s], 1);
      mbar_init(&wempty[s], kGtConvWarps);
    }
    for (int s = 0; s < NA; ++s) {
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
    tmem_alloc(tmem_slot, kGtTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  grid_dep_launch_dependents();
  grid_dep_wait();  // counters zeroed and inputs written by the preceding work

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int ws = 0;
      uint32_t wph = 0;
      uint32_t last_phase[kWStages];  // phase of each stage's latest load
      bool issued[kWStages];
      for (int i = 0; i < kWStages; ++i) issued[i] = false;
      bool ok = true;
      for (int t = 0; ok; ++t) {
        const int item = blockIdx.x + t * gridDim.x;
        if (item >= p.total_items) break;
        const int g = gt_find(p, item);
        const GtDesc &d = p.d[g];
        const int row0 = (item - d.item_begin) * 128;
        if (t == 0) tma_prefetch_desc(&p.tmW[g]);
        for (int kb = 0; kb < d.kblocks; kb += kKbStage) {
          if (!mbar_wait(&wempty[ws], wph ^ 1, p.timeout, abort_flag)) {
            gt_fail(abort_flag, p.err_flag, 31);
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&wfull[ws], kWStageBytes);  // OOB parts of the box are zero-filled
          tma_load_3d(wring + ws * kWStageBytes, &p.tmW[g], &wfull[ws], 0, row0, kb);
          issued[ws] = true;
          last_phase[ws] = wph;
          if (++ws == kWStages) {
            ws = 0;
            wph ^= 1;
          }
        }
      }
      if (!ok) {  // let the loads still in flight land before the CTA exits
        int ignored = 0;
        for (int i = 0; i < kWStages; ++i)
          if (issued[i]) mbar_wait(&wfull[i], last_phase[i], p.timeout, &ignored);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ UMMA issuer
    // K block number q counts over the CTA's whole item sequence; block q
    // uses A stage and x stage q % NA.
    uint32_t q = 0;
    bool ok = true, any = false;
    for (int t = 0; ok; ++t) {
      const int item = blockIdx.x + t * gridDim.x;
      if (item >= p.total_items) break;
      const GtDesc &d = p.d[gt_find(p, item)];
      const int acc = t & 1;
      bool w = (lane == 0) ? mbar_wait(&tempty[acc], ((t >> 1) & 1) ^ 1, p.timeout, abort_flag) : true;
      w = __shfl_sync(0xffffffffu, w, 0);
      if (!w) {
        if (lane == 0) gt_fail(abort_flag, p.err_flag, 32);
        ok = false;
        break;
      }
      tc_fence_after();
      for (int kb = 0; kb < d.kblocks; ++kb, ++q) {
        const int cs = static_cast<int>(q % NA);
        const uint32_t cph = (q / NA) & 1u;
        w = (lane == 0) ? mbar_wait(&cfull[cs], cph, p.timeout, abort_flag) : true;
        w = __shfl_sync(0xffffffffu, w, 0);
        if (!w) {
          if (lane == 0) gt_fail(abort_flag, p.err_flag, 33);
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t a_col = tmem_base + kGtAColBase + cs * 64;
          const uint32_t b_base = smem_u32(xring + cs * Cfg::kXBytes);
#pragma unroll
          for (int k = 0; k < 8; ++k)
            umma_f16_ts(tmem_base + acc * Cfg::kAccCols + (k % NACC) * MPAD, a_col + k * 8,
                        sdesc_kmajor_sw128(b_base + (k >> 2) * (MPAD * 128) + (k & 3) * 32), Cfg::kIdesc,
                        (kb > 0 || k >= NACC) ? 1u : 0u);
          umma_commit(&cempty[cs]);
          any = true;
        }
        __syncwarp();
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
    // Warp w may access TMEM lanes 32 (w % 4) .. +31, so thread (w, lane)
    // owns weight row r = 32 (w % 4) + lane.  Group h = (w - 2) / 4 converts
    // the 64-K half h of each K block: int8 chunks 4h .. 4h+3 of the row
    // (TMA 128B swizzle: chunk c of row r at ((c ^ (r & 7)) << 4)) become
    // 32 columns of fp16 pairs at A-stage columns 32h .. 32h+31.
    const int cw = warp - 2;                // 0 .. kGtConvWarps-1
    const int h = cw >> 2;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const int gtid = (cw & 3) * 32 + lane;  // thread index within the group (< 128)
    int ws = 0;
    uint32_t wph = 0;
    uint32_t q = 0;                         // K block number (see the UMMA issuer)
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
      for (int kb0 = 0; kb0 < d.kblocks && ok; kb0 += kKbStage) {
        bool w = (lane == 0) ? mbar_wait(&wfull[ws], wph, p.timeout, abort_flag) : true;
        w = __shfl_sync(0xffffffffu, w, 0);
        if (!w) {
          if (lane == 0) gt_fail(abort_flag, p.err_flag, 35);
          ok = false;
          break;
        }
        const int nk = min(kKbStage, d.kblocks - kb0);
        for (int j = 0; j < nk; ++j, ++q) {
          // this thread's x pieces: through L1 when x predates the launch, else
          // coherent from L2; their latency overlaps the slot wait and conversion
          uint4 xv[Cfg::kXPieces];
#pragma unroll
          for (int i = 0; i < Cfg::kXPieces; ++i) {
            const int pc = gtid + i * 128;
            const int xm = pc >> 3, xc = pc & 7;
            xv[i] = make_uint4(0u, 0u, 0u, 0u);
            if (xm < p.M) {
              const uint4 *xp = reinterpret_cast<const uint4 *>(
                  d.x + static_cast<int64_t>(xm) * d.ldx + (kb0 + j) * 128 + h * 64 + xc * 8);
              xv[i] = d.dep < 0 ? __ldg(xp) : __ldcg(xp);
            }
          }
          // int8 -> fp16 pairs of this row's half block, in K order
          const uint8_t *raw = wring + ws * kWStageBytes + j * (128 * 128) + r * 128;
          uint32_t a[32];
#pragma unroll
          for (int ci = 0; ci < 4; ++ci) {
            const uint4 wv = *reinterpret_cast<const uint4 *>(raw + (((4 * h + ci) ^ (r & 7)) << 4));
            uint4 lo, hi;
            i8x16_to_f16(wv, lo, hi);
            a[8 * ci + 0] = lo.x;
            a[8 * ci + 1] = lo.y;
            a[8 * ci + 2] = lo.z;
            a[8 * ci + 3] = lo.w;
            a[8 * ci + 4] = hi.x;
            a[8 * ci + 5] = hi.y;
            a[8 * ci + 6] = hi.z;
            a[8 * ci + 7] = hi.w;
          }
          const int cs = static_cast<int>(q % NA);
          const uint32_t cph = (q / NA) & 1u;
          w = (lane == 0) ? mbar_wait(&cempty[cs], cph ^ 1, p.timeout, abort_flag) : true;
          w = __shfl_sync(0xffffffffu, w, 0);
          if (!w) {
            if (lane == 0) gt_fail(abort_flag, p.err_flag, 36);
            ok = false;
            break;
          }
          tc_fence_after();
          tmem_st_32x32b_x32(tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + kGtAColBase + cs * 64 + h * 32,
                             a);
          // x rows of this half block (fp16, MPAD rows x 8 chunks; rows >= M zero)
          uint8_t *xst = xring + cs * Cfg::kXBytes + h * (MPAD * 128);
#pragma unroll
          for (int i = 0; i < Cfg::kXPieces; ++i) {
            const int pc = gtid + i * 128;
            const int xm = pc >> 3, xc = pc & 7;
            *reinterpret_cast<uint4 *>(xst + xm * 128 + ((xc ^ (xm & 7)) << 4)) = xv[i];
          }
          fence_proxy_async_smem();  // generic smem writes -> visible to the UMMAs
          tmem_st_wait();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&cfull[cs]);
        }
        if (!ok) break;
        __syncwarp();
        if (lane == 0) mbar_arrive(&wempty[ws]);
        if (++ws == kWStages) {
          ws = 0;
          wph ^= 1;
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int qd = warp & 3;  // TMEM lane quarter this warp may access
    for (int t = 0;; ++t) {
      const int item = blockIdx.x + t * gridDim.x;
      if (item >= p.total_items) break;
      const int g = gt_find(p, item);
      const GtDesc &d = p.d[g];
      const int acc = t & 1;
      bool w = (lane == 0) ? mbar_wait(&tfull[acc], (t >> 1) & 1, p.timeout, abort_flag) : true;
      w = __shfl_sync(0xffffffffu, w, 0);
      if (!w) {
        if (lane == 0) gt_fail(abort_flag, p.err_flag, 37);
        break;
      }
      tc_fence_after();
      const int n = (item - d.item_begin) * 128 + qd * 32 + lane;
      const float sc = n < d.N ? __half2float(d.scale[n]) : 0.f;
      const float b = (n < d.N && d.bias) ? __half2float(d.bias[n]) : 0.f;
#pragma unroll
      for (int c = 0; c < MPAD / 16; ++c) {
        if (c * 16 >= p.M) break;
        float sum[16];
#pragma unroll
        for (int j = 0; j < NACC; ++j) {  // the item's partial accumulators
          uint32_t v[16];
          tmem_ld_32x32b_x16(tmem_base + (static_cast<uint32_t>(qd * 32) << 16) + acc * Cfg::kAccCols + j * MPAD +
                                 c * 16,
                             v);
          tmem_ld_wait();
#pragma unroll
          for (int m = 0; m < 16; ++m) sum[m] = j == 0 ? __uint_as_float(v[m]) : sum[m] + __uint_as_float(v[m]);
        }
        if (n < d.N) {
#pragma unroll
          for (int m = 0; m < 16; ++m)
            if (c * 16 + m < p.M)
              d.y[static_cast<int64_t>(c * 16 + m) * d.ldy + n] = __float2half_rn(sum[m] * sc + b);
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
  if (warp == 1) tmem_dealloc(tmem_base, kGtTmemCols);
}

}  // namespace hx
