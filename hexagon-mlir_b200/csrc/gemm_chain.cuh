// gemm_chain.cuh — a stack of fused linear layers as one persistent launch.
//
// A transformer block's linears (GPT-2: QKV, attn-out + residual, MLP-up +
// GELU, MLP-down + residual; 12 blocks) are GEMMs of 1-5 GFLOP each, a few
// microseconds of tensor-core time, and launched one by one each pays its own
// ramp-up, first-load latency and tail.  In the reference these are separate
// linalg.matmul + linalg.generic ops compiled and run one after the other
// (lib/Conversion/LinalgToLLVM/LinalgToLLVMPass.cpp:188-400).  Here the whole
// list runs in one persistent grid:
//   * tiles are numbered GEMM-major, then row block m, then column block n;
//     CTA c takes tiles c, c + grid, c + 2*grid, ...;
//   * GEMM g may read (as its A operand, or as the residual of its epilogue)
//     the output of an earlier GEMM; before loading a tile of row block m the
//     producer warp waits (bounded spin, acquire) until that earlier GEMM has
//     finished all column blocks of row block m, counted in `counters`;
//   * after storing a tile the epilogue warps fence their stores and add one
//     to counter[g][m] (release).
// The lowest-numbered unfinished tile only waits on lower-numbered tiles,
// which are done, and nothing in its CTA is ahead of it, so the grid always
// progresses (all CTAs are resident: one per SM).
//
// The mainloop and epilogue are those of gemm_sm100.cuh (TMA ring, tcgen05
// UMMA into double-buffered TMEM, 8 epilogue warps), with the per-GEMM
// parameters (tensor maps, sizes, instruction descriptor, SwiGLU, epilogue)
// read from the launch's parameter block.  As there:
//   * A and B come through 3-D tensor maps, KBS 128-byte K blocks per TMA
//     instruction (TMA throughput here is per instruction, not per byte);
//   * the weights (B) of a tile's first stages are requested before the
//     producer waits for the tile's dependencies, so they are in flight
//     while the producing GEMM finishes its row block;
//   * full 32-column chunks leave through a per-warp staging buffer, so a
//     store instruction writes whole 64 / 128-byte row segments.
#pragma once
#include <cuda.h>
#include <stdint.h>

#include "epilogue.cuh"
#include "gemm_sm100.cuh"
#include "ptx.cuh"

namespace hx {

constexpr int kChainMax = 64;  // GEMMs per launch (parameter block < 32 KB)

struct ChainGemm {
  int32_t m_tiles, n_tiles, k_blocks;
  int32_t n_half;      // SWIGLU: first row of the "up" half of B
  int32_t swiglu;      // 1: B tile = [gate rows; up rows], output BN/2 columns
  int32_t a_dep;       // GEMM whose output is this A, or -1
  int32_t r_dep;       // GEMM whose output is this residual, or -1
  int32_t tile_begin;  // first global tile number
  int32_t ctr_begin;   // first counter (one per row block)
  uint32_t idesc;      // UMMA instruction descriptor (f16 / bf16)
  uint32_t idesc_half; // SWIGLU: the gate / up halves (N = BN / 2)
  EpiArgs epi;
};

struct ChainParams {
  CUtensorMap tma[kChainMax];   // A operand maps, 3-D {64 elements, rows, K blocks}
  CUtensorMap tmb[kChainMax];   // B operand maps, same form
  ChainGemm g[kChainMax];
  int32_t count, total_tiles, stages;  // stages of KBS K blocks each
  int32_t *counters;            // zeroed before launch
  int32_t *err_flag;
  uint64_t timeout;
};

__device__ __forceinline__ int chain_find(const ChainParams &p, int t) {
  int lo = 0, hi = p.count - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (p.g[mid].tile_begin <= t) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

__device__ __forceinline__ int ld_acquire_gpu_i32(const int32_t *p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Bounded wait until counter >= target.
__device__ __forceinline__ bool wait_counter(const int32_t *c, int target, uint64_t timeout,
                                             volatile int *abort_flag) {
  if (ld_acquire_gpu_i32(c) >= target) return true;
  const uint64_t t0 = clock64();
  while (ld_acquire_gpu_i32(c) < target) {
    if (*abort_flag) return false;
    if (static_cast<uint64_t>(clock64() - t0) > timeout) return false;
    __nanosleep(64);
  }
  return true;
}

template <int BN, int KBS>
__global__ void __launch_bounds__(kThreads, 1)
    hx_gemm_chain_kernel(const __grid_constant__ ChainParams p) {
  constexpr int kABytes = kBM * kKBytes;           // one K block of A
  constexpr int kBBytes = BN * kKBytes;            // one K block of B
  constexpr int A_ST = KBS * kABytes, B_ST = KBS * kBBytes;
  constexpr int kStageBytes = A_ST + B_ST;
  const int STAGES = p.stages;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t *sA = smem;
  uint8_t *sB = smem + STAGES * A_ST;
  uint64_t *full_bar = reinterpret_cast<uint64_t *>(smem + STAGES * kStageBytes);
  uint64_t *empty_bar = full_bar + STAGES;
  uint64_t *tfull_bar = empty_bar + STAGES;
  uint64_t *tempty_bar = tfull_bar + 2;
  uint64_t *drain_bar = tempty_bar + 2;
  uint64_t *stored_bar = drain_bar + 1;  // [2] the 8 epilogue warps stored a tile
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(stored_bar + 2);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
  uint8_t *stage_out = reinterpret_cast<uint8_t *>(full_bar) + kBarBytes;  // 8 x 4 KB
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], kEpiWarps);
      mbar_init(&stored_bar[a], kEpiWarps);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 2 * BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  grid_dep_launch_dependents();
  grid_dep_wait();  // counters were zeroed by the preceding memset

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    int stage = 0;
    uint32_t phase = 0;
    int64_t issued = 0;
    bool ok = true;
    auto advance = [&](int &st, uint32_t &ph) {
      if (++st == STAGES) {
        st = 0;
        ph ^= 1;
      }
    };
    for (int t = blockIdx.x; t < p.total_tiles && ok; t += gridDim.x) {
      const int gi = chain_find(p, t);
      const ChainGemm &g = p.g[gi];
      const int local = t - g.tile_begin;
      const int m_blk = local / g.n_tiles, n_blk = local % g.n_tiles;
      const int stage_blocks = (g.k_blocks + KBS - 1) / KBS;
      auto load_b = [&](uint64_t *fb, int st, int sb) {
        uint8_t *dstB = sB + st * B_ST;
        if (g.swiglu) {
          const int n0 = n_blk * (BN / 2);
          tma_load_3d(dstB, &p.tmb[gi], fb, 0, n0, sb * KBS);
          tma_load_3d(dstB + B_ST / 2, &p.tmb[gi], fb, 0, g.n_half + n0, sb * KBS);
        } else {
          tma_load_3d(dstB, &p.tmb[gi], fb, 0, n_blk * BN, sb * KBS);
        }
      };
      // 1. weights of the first stages, before any dependency wait
      const int pre = min(STAGES, stage_blocks);
      const int st0 = stage;
      for (int i = 0; i < pre && ok; ++i) {
        bool w = (lane == 0) ? mbar_wait(&empty_bar[stage], phase ^ 1, p.timeout, abort_flag) : true;
        w = __shfl_sync(0xffffffffu, w, 0);
        if (!w) {
          if (lane == 0) raise_abort(abort_flag, p.err_flag, 32);
          ok = false;
          break;
        }
        if (lane == 0) {
          mbar_arrive_expect_tx(&full_bar[stage], kStageBytes);
          load_b(&full_bar[stage], stage, i);
        }
        __syncwarp();
        ++issued;
        advance(stage, phase);
      }
      if (!ok) break;
      // 2. dependencies: full row block m of the producers of A and residual
      if (lane == 0) {
        if (g.a_dep >= 0)
          ok = wait_counter(p.counters + p.g[g.a_dep].ctr_begin + m_blk, p.g[g.a_dep].n_tiles,
                            p.timeout, abort_flag);
        if (ok && g.r_dep >= 0)
          ok = wait_counter(p.counters + p.g[g.r_dep].ctr_begin + m_blk, p.g[g.r_dep].n_tiles,
                            p.timeout, abort_flag);
        if (ok && (g.a_dep >= 0 || g.r_dep >= 0))
          asm volatile("fence.proxy.async.global;" ::: "memory");  // generic writes -> TMA reads
        if (!ok) raise_abort(abort_flag, p.err_flag, 31);
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) {
        // the armed stages still expect their A bytes: fill them so the
        // drain below completes (A's rows are valid memory)
        if (lane == 0)
          for (int i = 0, st = st0; i < pre; ++i, st = (st + 1 == STAGES ? 0 : st + 1))
            tma_load_3d(sA + st * A_ST, &p.tma[gi], &full_bar[st], 0, m_blk * kBM, i * KBS);
        break;
      }
      // 3. activations of those stages
      if (lane == 0)
        for (int i = 0, st = st0; i < pre; ++i, st = (st + 1 == STAGES ? 0 : st + 1))
          tma_load_3d(sA + st * A_ST, &p.tma[gi], &full_bar[st], 0, m_blk * kBM, i * KBS);
      __syncwarp();
      // 4. the remaining stages
      for (int sb = pre; sb < stage_blocks; ++sb) {
        bool w = (lane == 0) ? mbar_wait(&empty_bar[stage], phase ^ 1, p.timeout, abort_flag) : true;
        w = __shfl_sync(0xffffffffu, w, 0);
        if (!w) {
          if (lane == 0) raise_abort(abort_flag, p.err_flag, 32);
          ok = false;
          break;
        }
        if (lane == 0) {
          uint64_t *fb = &full_bar[stage];
          mbar_arrive_expect_tx(fb, kStageBytes);
          tma_load_3d(sA + stage * A_ST, &p.tma[gi], fb, 0, m_blk * kBM, sb * KBS);
          load_b(fb, stage, sb);
        }
        __syncwarp();
        ++issued;
        advance(stage, phase);
      }
    }
    if (!ok && lane == 0) {
      const int64_t first = issued > STAGES ? issued - STAGES : 0;
      for (int64_t i = first; i < issued; ++i) {
        int dummy = 0;
        mbar_wait(&full_bar[i % STAGES], static_cast<uint32_t>((i / STAGES) & 1), p.timeout, &dummy);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ UMMA issuer
    int stage = 0;
    uint32_t phase = 0;
    int it = 0;
    bool ok = true, any = false;
    for (int t = blockIdx.x; t < p.total_tiles && ok; t += gridDim.x, ++it) {
      const ChainGemm &g = p.g[chain_find(p, t)];
      const int stage_blocks = (g.k_blocks + KBS - 1) / KBS;
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      bool w = (lane == 0) ? mbar_wait(&tempty_bar[acc], acc_phase ^ 1, p.timeout, abort_flag) : true;
      w = __shfl_sync(0xffffffffu, w, 0);
      if (!w) {
        if (lane == 0) raise_abort(abort_flag, p.err_flag, 33);
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + acc * BN;
      for (int sb = 0; sb < stage_blocks; ++sb) {
        bool f = (lane == 0) ? mbar_wait(&full_bar[stage], phase, p.timeout, abort_flag) : true;
        f = __shfl_sync(0xffffffffu, f, 0);
        if (!f) {
          if (lane == 0) raise_abort(abort_flag, p.err_flag, 34);
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t a_base = smem_u32(sA + stage * A_ST);
          const uint32_t b_base = smem_u32(sB + stage * B_ST);
          const int nj = min(KBS, g.k_blocks - sb * KBS);  // K blocks past K are zero-filled anyway
          for (int j = 0; j < nj; ++j) {
#pragma unroll
            for (int k = 0; k < kKBytes / kUmmaKBytes; ++k) {
              const uint64_t ad = sdesc_kmajor_sw128(a_base + j * kABytes + k * kUmmaKBytes);
              const uint32_t accum = (sb > 0 || j > 0 || k > 0) ? 1u : 0u;
              if (g.swiglu) {
                const uint32_t hb = (BN / 2) * kKBytes;
                const uint64_t gd = sdesc_kmajor_sw128(b_base + j * hb + k * kUmmaKBytes);
                const uint64_t ud = sdesc_kmajor_sw128(b_base + B_ST / 2 + j * hb + k * kUmmaKBytes);
                umma_f16(d_tmem, ad, gd, g.idesc_half, accum);
                umma_f16(d_tmem + BN / 2, ad, ud, g.idesc_half, accum);
              } else {
                umma_f16(d_tmem, ad, sdesc_kmajor_sw128(b_base + j * kBBytes + k * kUmmaKBytes), g.idesc,
                         accum);
              }
            }
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
      if (!ok) break;
      if (lane == 0) umma_commit(&tfull_bar[acc]);
      __syncwarp();
    }
    if (!ok && lane == 0 && any) {
      umma_commit(drain_bar);
      int dummy = 0;
      mbar_wait(drain_bar, 0, p.timeout, &dummy);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int row_in_tile = q * 32 + lane;
    uint8_t *stg = stage_out + (warp - 2) * 4096;
    int it = 0;
    for (int t = blockIdx.x; t < p.total_tiles; t += gridDim.x, ++it) {
      const int gi = chain_find(p, t);
      const ChainGemm &g = p.g[gi];
      const int local = t - g.tile_begin;
      const int m_blk = local / g.n_tiles, n_blk = local % g.n_tiles;
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      bool w = (lane == 0) ? mbar_wait(&tfull_bar[acc], acc_phase, p.timeout, abort_flag) : true;
      w = __shfl_sync(0xffffffffu, w, 0);
      if (!w) {
        if (lane == 0) raise_abort(abort_flag, p.err_flag, 35);
        break;
      }
      tc_fence_after();
      const int out_w = g.swiglu ? BN / 2 : BN;
      const int m = m_blk * kBM + row_in_tile;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN;
#pragma unroll 1
      for (int c = (warp - 2) / 4; c < out_w / 32; c += 2) {
        uint32_t r[32], r2[32];
        tmem_ld_32x32b_x32(t_row + c * 32, r);
        if (g.swiglu) tmem_ld_32x32b_x32(t_row + BN / 2 + c * 32, r2);
        tmem_ld_wait();
        float v[32], up[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          v[j] = __uint_as_float(r[j]);
          up[j] = g.swiglu ? __uint_as_float(r2[j]) : 0.f;
        }
        const int n0 = n_blk * out_w + c * 32;
        epi_transform32(g.epi, v, up, m, n0);
        if (g.epi.c_vec_ok && n0 + 32 <= g.epi.N)
          epi_store32_staged_rt(g.epi, v, r, false, m - lane, n0, stg);
        else
          epi_store32(g.epi, v, r, false, m, n0);
      }
      tc_fence_before();
      // Stores of this thread, then visible to later TMA (async-proxy) reads.
      asm volatile("fence.proxy.async.global;" ::: "memory");
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&tempty_bar[acc]);
        mbar_arrive(&stored_bar[acc]);
      }
      // When all 8 epilogue warps stored the tile, one lane counts it for row
      // block m (bounded wait; on timeout the tile is never counted and its
      // consumers time out too).
      if (warp == 2 && lane == 0) {
        if (mbar_wait(&stored_bar[acc], acc_phase, p.timeout, abort_flag)) {
          asm volatile("fence.acq_rel.gpu;" ::: "memory");
          asm volatile("red.relaxed.gpu.global.add.s32 [%0], 1;" ::"l"(p.counters + g.ctr_begin + m_blk)
                       : "memory");
        } else {
          raise_abort(abort_flag, p.err_flag, 36);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, 2 * BN);
}

}  // namespace hx
