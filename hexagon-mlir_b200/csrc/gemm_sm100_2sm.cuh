// gemm_sm100_2sm.cuh — the GEMM of gemm_sm100.cuh on CTA pairs (tcgen05
// cta_group::2): one 256 x BN tile per pair of SMs.
//
// Why: a 128 x BN tile on one SM must bring in 128 rows of A and BN rows of B
// per K block; TMA ingest, not the tensor core, bounds the large GEMMs (the
// LM head).  With cta_group::2 each CTA brings its own 128 rows of A and
// only BN/2 rows of B, and one UMMA (M = 256) reads both CTAs' halves, so the
// bytes each SM ingests per flop drop by 1/3 at BN = 256.
//
// Pair protocol (cluster of 2, CTA rank 0 = leader):
//   * TMEM: both CTAs allocate with cta_group::2 (same columns in both).
//   * loads: each CTA's producer TMA-loads its A rows and its B half into its
//     own smem; every load completes on the LEADER's full barrier (the leader
//     alone arms it with the pair's byte count).  No load is shared between
//     CTAs (no multicast loads).
//   * MMA: the leader's single thread issues tcgen05.mma.cta_group::2 with
//     descriptors of its own smem; the same offsets in the peer supply the
//     other halves.  Commits are multicast to both CTAs' barriers (empty
//     stage, accumulator full).
//   * epilogue: each CTA drains its own 128 accumulator rows from its own TMEM;
//     both CTAs' epilogue warps arrive on the leader's accumulator-empty barrier.
// Every wait is bounded as in gemm_sm100.cuh.
#pragma once
#include <cuda.h>
#include <stdint.h>

#include "epilogue.cuh"
#include "gemm_sm100.cuh"
#include "ptx.cuh"

namespace hx {

__device__ __forceinline__ void tma_load_3d_pair(void *smem_dst, const CUtensorMap *map,
                                                 uint32_t leader_bar, int32_t x, int32_t y,
                                                 int32_t z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(leader_bar), "r"(x), "r"(y), "r"(z)
      : "memory");
}
__device__ __forceinline__ void umma_f16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                              uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_i8_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on the barrier at this smem offset in every CTA of `mask` once all
// prior tcgen05 ops of the pair have completed.
__device__ __forceinline__ void umma_commit_pair(uint64_t *bar, uint16_t mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(smem_u32(bar)),
      "h"(mask)
      : "memory");
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t *dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// BN = UMMA N of the pair (each CTA holds BN/2 rows of B); K blocks are
// always loaded through 3-D maps (kbs per stage).
template <int BN, int KIND, bool SWIGLU>
__global__ void __launch_bounds__(kThreads, 1)
    hx_gemm_sm100_2sm_kernel(const __grid_constant__ CUtensorMap tmA,
                             const __grid_constant__ CUtensorMap tmB,
                             const __grid_constant__ GemmParams p) {
  constexpr int kElem = (KIND == 2) ? 1 : 2;
  constexpr int kUmmaKBytesC = kUmmaKBytes;
  constexpr int kABytes = kBM * kKBytes;            // per CTA per K block
  constexpr int kBBytes = (BN / 2) * kKBytes;       // per CTA per K block
  constexpr int kBNOut = SWIGLU ? BN / 2 : BN;
  constexpr int kTmemCols = 2 * BN;
  constexpr uint32_t kIdesc = make_idesc(KIND, false, 2 * kBM, BN);
  const int STAGES = p.stages;
  const int A_ST = p.kbs * kABytes, B_ST = p.kbs * kBBytes;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t *sA = smem;
  uint8_t *sB = smem + STAGES * A_ST;
  uint64_t *full_bar = reinterpret_cast<uint64_t *>(smem + STAGES * (A_ST + B_ST));
  uint64_t *empty_bar = full_bar + STAGES;
  uint64_t *tfull_bar = empty_bar + STAGES;   // [2]
  uint64_t *tempty_bar = tfull_bar + 2;       // [2] (used in the leader)
  uint64_t *drain_bar = tempty_bar + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain_bar + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
  uint8_t *stage_out = reinterpret_cast<uint8_t *>(full_bar) + kBarBytes;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = gemm_cluster_rank();   // 0 = leader
  const bool leader = rank == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 2 * kEpiWarps);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  gemm_cluster_sync();  // both CTAs' barriers are initialised before any remote use
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  grid_dep_launch_dependents();
  grid_dep_wait();

  const int t_first = blockIdx.x / 2, t_step = gridDim.x / 2;
  const uint32_t leader_full0 = gemm_peer_addr(smem_u32(full_bar), 0);
  const uint32_t leader_tempty0 = gemm_peer_addr(smem_u32(tempty_bar), 0);

  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    int stage = 0;
    uint32_t phase = 0;
    int64_t issued = 0;
    bool ok = true;
    for (int t = t_first; t < p.total_tiles && ok; t += t_step) {
      int m_blk, n_blk;
      tile_coords(t, p, m_blk, n_blk);
      const int m0 = m_blk * (2 * kBM) + static_cast<int>(rank) * kBM;
      for (int sb = 0; sb < p.stage_blocks; ++sb) {
        bool w = (lane == 0) ? mbar_wait(&empty_bar[stage], phase ^ 1, p.timeout, abort_flag) : true;
        w = __shfl_sync(0xffffffffu, w, 0);
        if (!w) {
          if (lane == 0) raise_abort(abort_flag, p.err_flag, 41);
          ok = false;
          break;
        }
        if (lane == 0) {
          if (leader) mbar_arrive_expect_tx(&full_bar[stage], 2 * (A_ST + B_ST));
          const uint32_t lbar = leader_full0 + stage * 8;
          const int kz = sb * p.kbs;
          tma_load_3d_pair(sA + stage * A_ST, &tmA, lbar, 0, m0, kz);
          int brow;
          if constexpr (SWIGLU)  // rank 0 holds the gate rows, rank 1 the up rows
            brow = (rank == 0 ? 0 : p.n_half) + n_blk * (BN / 2);
          else
            brow = n_blk * BN + static_cast<int>(rank) * (BN / 2);
          tma_load_3d_pair(sB + stage * B_ST, &tmB, lbar, 0, brow, kz);
        }
        __syncwarp();
        ++issued;
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
    if (!ok && lane == 0 && leader) {  // the leader's barrier counts the pair's loads
      const int64_t first = issued > STAGES ? issued - STAGES : 0;
      for (int64_t i = first; i < issued; ++i) {
        int dummy = 0;
        mbar_wait(&full_bar[i % STAGES], static_cast<uint32_t>((i / STAGES) & 1), p.timeout, &dummy);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ UMMA issuer (leader)
    if (leader) {
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true, any = false;
      for (int t = t_first; t < p.total_tiles && ok; t += t_step, ++it) {
        const int acc = it & 1;
        const uint32_t acc_phase = (it >> 1) & 1;
        bool w = (lane == 0) ? mbar_wait(&tempty_bar[acc], acc_phase ^ 1, p.timeout, abort_flag) : true;
        w = __shfl_sync(0xffffffffu, w, 0);
        if (!w) {
          if (lane == 0) raise_abort(abort_flag, p.err_flag, 42);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int sb = 0; sb < p.stage_blocks; ++sb) {
          bool f = (lane == 0) ? mbar_wait(&full_bar[stage], phase, p.timeout, abort_flag) : true;
          f = __shfl_sync(0xffffffffu, f, 0);
          if (!f) {
            if (lane == 0) raise_abort(abort_flag, p.err_flag, 43);
            ok = false;
            break;
          }
          tc_fence_after();
          if (lane == 0) {
            const uint32_t a_base = smem_u32(sA + stage * A_ST);
            const uint32_t b_base = smem_u32(sB + stage * B_ST);
            for (int j = 0; j < p.kbs; ++j) {
#pragma unroll
              for (int k = 0; k < kKBytes / kUmmaKBytesC; ++k) {
                const uint64_t ad = sdesc_kmajor_sw128(a_base + j * kABytes + k * kUmmaKBytesC);
                const uint64_t bd = sdesc_kmajor_sw128(b_base + j * kBBytes + k * kUmmaKBytesC);
                const uint32_t accum = (sb > 0 || j > 0 || k > 0) ? 1u : 0u;
                if constexpr (KIND == 2)
                  umma_i8_pair(d_tmem, ad, bd, kIdesc, accum);
                else
                  umma_f16_pair(d_tmem, ad, bd, kIdesc, accum);
              }
            }
            umma_commit_pair(&empty_bar[stage], 0x3);  // both CTAs' stage is free
            any = true;
          }
          __syncwarp();
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        if (lane == 0) umma_commit_pair(&tfull_bar[acc], 0x3);  // both halves ready
        __syncwarp();
      }
      if (!ok && lane == 0 && any) {
        umma_commit_pair(drain_bar, 0x1);
        int dummy = 0;
        mbar_wait(drain_bar, 0, p.timeout, &dummy);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    (void)kElem;
    const int q = warp & 3;
    const int row_in_tile = q * 32 + lane;
    int it = 0;
    for (int t = t_first; t < p.total_tiles; t += t_step, ++it) {
      int m_blk, n_blk;
      tile_coords(t, p, m_blk, n_blk);
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      const int m = m_blk * (2 * kBM) + static_cast<int>(rank) * kBM + row_in_tile;
      const int c0 = (warp - 2) / 4;
      Pre16 pf;
      epi_row_prefetch<SWIGLU>(p.epi, m, n_blk * kBNOut + c0 * 32, pf);
      bool w = (lane == 0) ? mbar_wait(&tfull_bar[acc], acc_phase, p.timeout, abort_flag) : true;
      w = __shfl_sync(0xffffffffu, w, 0);
      if (!w) {
        if (lane == 0) raise_abort(abort_flag, p.err_flag, 44);
        break;
      }
      tc_fence_after();
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN;
      epi_row<BN, kBNOut, KIND, SWIGLU>(p.epi, t_row, m, n_blk * kBNOut, c0, pf,
                                        stage_out + (warp - 2) * 4096);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (leader)
          mbar_arrive(&tempty_bar[acc]);
        else
          mbar_arrive_remote(leader_tempty0 + acc * 8);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  gemm_cluster_sync();  // the pair finished: no more remote arrivals or UMMA writes
  tc_fence_after();
  // fused all-gather: peer stores are visible system-wide before the grid ends
  if (p.epi.n_peers > 0) __threadfence_system();
  if (warp == 1) tmem_dealloc_pair(tmem_base, kTmemCols);
}

}  // namespace hx
