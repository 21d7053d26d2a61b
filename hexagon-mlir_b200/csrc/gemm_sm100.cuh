// gemm_sm100.cuh — persistent, warp-specialised tcgen05 GEMM for sm_100a.
//
// What it replaces in the reference (hustc12/hexagon-mlir):
//   * the VTCM tile scheduler (lib/Conversion/LinalgToLLVM/VTCMTiling.cpp:231-266,
//     VTCMTilingOptions.cpp:374-432): tiles are 128 x BN x (128 bytes of K),
//     sized to the 227 KB of shared memory instead of the 2 MB VTCM;
//   * the DDR->VTCM DMA prefetch + double buffering
//     (HexmemCpyToDMA.cpp:50-80, DoubleBufferGenericS1.cpp:10-19,
//     UserDMA.cc:27,94,167): a STAGES-deep ring of TMA box loads completing
//     on mbarriers, issued by one producer warp;
//   * the HVX/HMX inner loop (TilingPass.cpp:108-292,
//     DecomposeHexKLMatmulPass.cpp:148-222): tcgen05.mma 128xBNx(32 bytes)
//     issued by one thread, accumulating in TMEM;
//   * the 4-thread scf.forall split (FormVirtualThreadsPass.cpp:51-202):
//     a persistent grid of one CTA per SM walking a grouped tile order;
//   * the unfused epilogue generic (FusionPass.cpp:163,176-179): applied to
//     the accumulator in registers by eight epilogue warps.
//
// Warp roles (320 threads):
//   warp 0      TMA producer (lane 0 issues)
//   warp 1      TMEM allocator + UMMA issuer (lane 0 issues)
//   warps 2..9  epilogue: TMEM -> registers -> fused epilogue -> global;
//               warp w reads TMEM lane quarter w % 4 and every other
//               32-column chunk ((w - 2) / 4 picks which)
// TMEM holds two BN-column fp32/s32 accumulators so the epilogue of tile i
// overlaps the mainloop of tile i+1.
#pragma once
#include <cuda.h>
#include <stdint.h>

#include "epilogue.cuh"
#include "ptx.cuh"

namespace hx {

constexpr int kBM = 128;          // UMMA M (rows of A per tile)
constexpr int kKBytes = 128;      // K bytes per stage (one 128B swizzle row)
constexpr int kUmmaKBytes = 32;   // K bytes per UMMA instruction
constexpr int kThreads = 320;
constexpr int kEpiWarps = 8;
constexpr int kBarBytes = 256;                   // mbarriers + TMEM slot + abort word
constexpr int kStageOutBytes = kEpiWarps * 4096; // per-epilogue-warp output staging

// Per-phase %globaltimer stamps of each CTA (prologue, first stage, last UMMA,
// accumulator ready, epilogue chunks) for latency studies; compiled in only
// with -DHX_GEMM_TRACE.
#ifdef HX_GEMM_TRACE
__device__ unsigned long long g_gemm_trace[1024][16];
#define HX_GEMM_STAMP(i)                                         \
  do {                                                           \
    unsigned long long t_;                                       \
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));       \
    if (blockIdx.x < 1024) g_gemm_trace[blockIdx.x][i] = t_;     \
  } while (0)
#else
#define HX_GEMM_STAMP(i) \
  do {                   \
  } while (0)
#endif

struct GemmParams {
  int32_t M, K;                   // rows of A/C, reduction length
  int32_t n_tiles, m_tiles, k_blocks;
  int32_t n_half;                 // SWIGLU: first row of the "up" half of B
  int32_t group_m;                // grouped raster: m-tiles per group
  int32_t total_tiles;
  int32_t stages;                 // depth of the smem ring
  int32_t kbs;                    // 128-byte K blocks per stage (one TMA load each for A, B)
  int32_t stage_blocks;           // stages per tile: ceil(k_blocks / kbs)
  int32_t use3d;                  // 3-D maps (K blocks as the third dimension)
  int32_t splits;                 // split-K: CTAs per cluster sharing one tile (1 = none)
  uint64_t timeout;               // cycles per bounded wait
  int32_t *err_flag;              // optional global error word
  uint4 *ws;                      // split-K: [tile][rank][BN/32][8][128] x 16 B of partials
  int32_t red_smem;               // split-K: fetch remote partials into the ring (else read L2)
  int32_t b_const;                // B is constant: fetch the first B tiles before the dependency wait
  // Batched GEMM (batch > 1): tile t belongs to item t / batch_tiles; A and B
  // are 3-D tensor maps (item as the outer dimension, 2-D K-block loads) and
  // C / residual rows are flattened, item b's row r at b * batch_rows + r.
  int32_t batch;                  // items (1 = a plain GEMM)
  int32_t batch_tiles;            // m_tiles * n_tiles of one item
  int32_t batch_rows;             // rows of one item (a multiple of kBM)
  // Implicit-GEMM convolution (conv != 0): A is the NHWC activation through a
  // 4-D map {C, W, H, N}; output row m is pixel m of NHWC order (tiles of
  // kBM consecutive pixels = whole rows of the image); K block kb is filter
  // tap kb / conv_cpb (kh * KW + kw) and channels 64 * (kb % conv_cpb) + [0, 64).
  int32_t conv;
  int32_t conv_H, conv_W, conv_KW, conv_cpb, conv_pad_h, conv_pad_w;
  EpiArgs epi;
};

template <int BN, int KIND, bool B_MN, bool SWIGLU>
struct GemmCfg {
  static constexpr int kElem = (KIND == 2) ? 1 : 2;
  static constexpr int kBKElems = kKBytes / kElem;               // 64 or 128
  static constexpr int kUmmaK = kUmmaKBytes / kElem;              // 16 or 32
  static constexpr int kABytes = kBM * kKBytes;                   // 16 KB
  static constexpr int kBBytes = BN * kKBytes;                    // BN * 128 B
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kBNOut = SWIGLU ? BN / 2 : BN;             // output columns / tile
  // double-buffered accumulator; allocations are powers of two columns
  static constexpr int kTmemCols = 2 * BN <= 128 ? 128 : (2 * BN <= 256 ? 256 : 512);
  static constexpr int kMNChunk = kKBytes / kElem;                // MN elems per 128 B
  static constexpr int smem_bytes(int stages) { return stages * kStageBytes + 1024 /*align*/ + kBarBytes + kStageOutBytes; }
  static constexpr uint32_t kIdesc = make_idesc(KIND, B_MN, kBM, BN);
  // split-K: ring bytes that receive the remote partials of a rank's chunks
  __host__ __device__ static constexpr int red_bytes(int splits) {
    return ((kBNOut / 32 + splits - 1) / splits) * (splits - 1) * (SWIGLU ? 2 : 1) * 8 * kBM * 16;
  }
  static constexpr uint32_t kIdescHalf = make_idesc(KIND, B_MN, kBM, BN / 2);  // SWIGLU halves
  static_assert(BN == 64 || BN == 96 || BN == 128 || BN == 192 || BN == 256, "BN");
  static_assert(BN % 64 == 0 || !(B_MN || SWIGLU), "BN 96 / 192: W[N,K] only; SWIGLU needs BN / 2 % 32 == 0");
  static_assert(!(SWIGLU && B_MN), "SWIGLU needs the W[N,K] layout");
  static_assert(kTmemCols >= 32 && kTmemCols <= 512, "TMEM columns");
};

__device__ __forceinline__ void tile_coords(int t, const GemmParams &p, int &m_blk, int &n_blk) {
  const int per_group = p.group_m * p.n_tiles;
  const int g = t / per_group;
  const int first_m = g * p.group_m;
  const int gsize = min(p.m_tiles - first_m, p.group_m);
  const int r = t - g * per_group;
  m_blk = first_m + r % gsize;
  n_blk = r / gsize;
}

// Tile t of a (possibly batched) launch: item b and its m / n blocks.
__device__ __forceinline__ void tile_coords_b(int t, const GemmParams &p, int &b, int &m_blk, int &n_blk) {
  b = 0;
  if (p.batch > 1) {
    b = t / p.batch_tiles;
    t -= b * p.batch_tiles;
  }
  tile_coords(t, p, m_blk, n_blk);
}

__device__ __forceinline__ uint32_t gemm_cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void gemm_cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}
__device__ __forceinline__ uint32_t gemm_peer_addr(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
__device__ __forceinline__ uint32_t ld_cluster_u32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
  return v;
}

__device__ __forceinline__ void raise_abort(volatile int *abort_flag, int32_t *err, int code) {
  *abort_flag = 1;
  if (err != nullptr) atomicExch(err, code);
}

// A raw-accumulator argument for store paths that do not read it.
__device__ __forceinline__ const uint32_t (&v_as_raw_unused())[32] {
  static __device__ const uint32_t kNone[32] = {};
  return kNone;
}

// Epilogue of one accumulator row (TMEM lane quarter row, every other
// 32-column chunk from c0): TMEM -> registers -> fused epilogue -> global.
// With 16-bit operands (e.pre16) the scale / bias / residual of each chunk
// are loaded one chunk ahead, the first by epi_row_prefetch before the
// accumulator wait, so their latency overlaps the previous chunk's stores.
template <bool SWIGLU>
__device__ __forceinline__ void epi_row_prefetch(const EpiArgs &e, int m, int n0, Pre16 &pf) {
  if (!SWIGLU && e.pre16 && n0 + 32 <= e.N) epi_prefetch16(e, m, n0, pf);
}

// The loop for one (epilogue, output dtype) pair, fixed at compile time, for
// rows whose chunks are all full and whose operands are 16-bit and aligned
// (e.pre16, e.c_vec_ok): nothing in it calls out, so its registers stay put.
template <int BN, int BN_OUT, int KIND, bool SWIGLU, int EPI, int CT>
__device__ __forceinline__ void epi_row_t(const EpiArgs &e, uint32_t t_row, int m, int n_base, int c0,
                                          Pre16 &pf, uint8_t *stg) {
  constexpr bool kRaw = (KIND == 2) && (CT == HX_S32) && (EPI == HX_EPI_NONE);
  constexpr bool kPre = !(EPI == HX_EPI_NONE || EPI == HX_EPI_SWIGLU);  // operands to prefetch
#ifndef HX_EPI_NO_TMEM_PIPE
  if constexpr (!SWIGLU && !kRaw) {
    // The next chunk's TMEM load is in flight while this chunk is finished
    // and stored (tcgen05.wait::ld waits for every earlier load, so the next
    // load is issued only after this chunk's registers are consumed).
    uint32_t r[32];
    if (c0 < BN_OUT / 32) tmem_ld_32x32b_x32(t_row + c0 * 32, r);
#pragma unroll 1
    for (int c = c0; c < BN_OUT / 32; c += 2) {
      const int n0 = n_base + c * 32;
      tmem_ld_wait();
      float v[32], up[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        if constexpr (KIND == 2)
          v[j] = static_cast<float>(static_cast<int32_t>(r[j]));
        else
          v[j] = __uint_as_float(r[j]);
        up[j] = 0.f;
      }
      if (c + 2 < BN_OUT / 32) tmem_ld_32x32b_x32(t_row + (c + 2) * 32, r);
      epi_apply_t<EPI, CT>(e, v, up, m, pf, stg);
      if constexpr (kPre) {
        if (c + 2 < BN_OUT / 32) epi_prefetch_t<EPI>(e, m, n0 + 64, pf);
      }
      epi_store32_staged_t<CT, false>(e, v, v_as_raw_unused(), m - static_cast<int>(threadIdx.x & 31), n0, stg);
    }
  } else
#endif
  {
#pragma unroll 1
  for (int c = c0; c < BN_OUT / 32; c += 2) {
    uint32_t r[32], r2[32];
    tmem_ld_32x32b_x32(t_row + c * 32, r);
    if constexpr (SWIGLU) tmem_ld_32x32b_x32(t_row + BN / 2 + c * 32, r2);
    const int n0 = n_base + c * 32;
    tmem_ld_wait();
    if (threadIdx.x == 64 && c < 8) HX_GEMM_STAMP(8 + c);
    float v[32], up[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if constexpr (KIND == 2)
        v[j] = static_cast<float>(static_cast<int32_t>(r[j]));
      else
        v[j] = __uint_as_float(r[j]);
      if constexpr (SWIGLU)
        up[j] = __uint_as_float(r2[j]);
      else
        up[j] = 0.f;
    }
    if constexpr (!kRaw) epi_apply_t<EPI, CT>(e, v, up, m, pf, stg);
    // The next chunk's operands load while this chunk is stored.
    if constexpr (kPre) {
      if (c + 2 < BN_OUT / 32) epi_prefetch_t<EPI>(e, m, n0 + 64, pf);
    }
    epi_store32_staged_t<CT, kRaw>(e, v, r, m - static_cast<int>(threadIdx.x & 31), n0, stg);
    if (threadIdx.x == 64 && c < 8) HX_GEMM_STAMP(9 + c);
  }
  }
}

// Every other row (a partial last tile, unaligned C, 32-bit operands): the
// runtime-dispatched epilogue and row stores, out of line.
template <int BN, int BN_OUT, int KIND, bool SWIGLU>
__device__ __noinline__ void epi_row_generic(const EpiArgs &e, uint32_t t_row, int m, int n_base, int c0,
                                             uint8_t *stg) {
  const bool raw_int = (KIND == 2) && (e.c_dtype == HX_S32) && (e.epi == HX_EPI_NONE);
#pragma unroll 1
  for (int c = c0; c < BN_OUT / 32; c += 2) {
    uint32_t r[32], r2[32];
    tmem_ld_32x32b_x32(t_row + c * 32, r);
    if constexpr (SWIGLU) tmem_ld_32x32b_x32(t_row + BN / 2 + c * 32, r2);
    tmem_ld_wait();
    float v[32], up[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if constexpr (KIND == 2)
        v[j] = static_cast<float>(static_cast<int32_t>(r[j]));
      else
        v[j] = __uint_as_float(r[j]);
      if constexpr (SWIGLU)
        up[j] = __uint_as_float(r2[j]);
      else
        up[j] = 0.f;
    }
    const int n0 = n_base + c * 32;
    if (!raw_int) epi_transform32(e, v, up, m, n0);
    if (e.n_peers > 0 && e.c_vec_ok && n0 + 32 <= e.N)  // fused all-gather: coalesced stores
      epi_store32_staged_all(e, v, r, raw_int, m - static_cast<int>(threadIdx.x & 31), n0, stg);
    else
      epi_store32(e, v, r, raw_int, m, n0);
  }
}

template <int BN, int BN_OUT, int KIND, bool SWIGLU, int CT>
__device__ __forceinline__ void epi_row_ct(const EpiArgs &e, uint32_t t_row, int m, int n_base, int c0,
                                           Pre16 &pf, uint8_t *stg) {
#define HX_EPI_ROW(E) epi_row_t<BN, BN_OUT, KIND, SWIGLU, E, CT>(e, t_row, m, n_base, c0, pf, stg)
  if constexpr (SWIGLU) {
    HX_EPI_ROW(HX_EPI_SWIGLU);
  } else if constexpr (CT == HX_S32) {
    HX_EPI_ROW(HX_EPI_NONE);  // int32 output: int8 inputs, no epilogue
  } else {
    switch (e.epi) {
      case HX_EPI_NONE: HX_EPI_ROW(HX_EPI_NONE); break;
      case HX_EPI_BIAS: HX_EPI_ROW(HX_EPI_BIAS); break;
      case HX_EPI_BIAS_GELU_TANH: HX_EPI_ROW(HX_EPI_BIAS_GELU_TANH); break;
      case HX_EPI_BIAS_RESIDUAL: HX_EPI_ROW(HX_EPI_BIAS_RESIDUAL); break;
      case HX_EPI_RESIDUAL: HX_EPI_ROW(HX_EPI_RESIDUAL); break;
      case HX_EPI_BIAS_SILU: HX_EPI_ROW(HX_EPI_BIAS_SILU); break;
      case HX_EPI_DEQUANT_SCALE:
        if constexpr (KIND == 2) HX_EPI_ROW(HX_EPI_DEQUANT_SCALE);
        break;
      default: break;
    }
  }
#undef HX_EPI_ROW
}

// Epilogue of one accumulator row (TMEM lane quarter row, every other
// 32-column chunk from c0): rows of full tiles with aligned 16-bit operands
// dispatch once on the output dtype and the epilogue to a loop specialised
// for that pair; the rest take the generic loop.
template <int BN, int BN_OUT, int KIND, bool SWIGLU>
__device__ __forceinline__ void epi_row(const EpiArgs &e, uint32_t t_row, int m, int n_base, int c0,
                                        Pre16 &pf, uint8_t *stg) {
  // rows whose chunks also go to peers (fused all-gather) take the generic
  // loop, which stores to every target; the specialised loop stores C only.
  // So do GEMMs with a folded row normalisation.
  if (!(e.pre16 && e.c_vec_ok && n_base + BN_OUT <= e.N) || e.n_peers > 0 || e.norm) {
    epi_row_generic<BN, BN_OUT, KIND, SWIGLU>(e, t_row, m, n_base, c0, stg);
    return;
  }
  switch (e.c_dtype) {
    case HX_F16: epi_row_ct<BN, BN_OUT, KIND, SWIGLU, HX_F16>(e, t_row, m, n_base, c0, pf, stg); break;
    case HX_BF16: epi_row_ct<BN, BN_OUT, KIND, SWIGLU, HX_BF16>(e, t_row, m, n_base, c0, pf, stg); break;
    case HX_F32: epi_row_ct<BN, BN_OUT, KIND, SWIGLU, HX_F32>(e, t_row, m, n_base, c0, pf, stg); break;
    case HX_S32:
      if constexpr (KIND == 2 && !SWIGLU) epi_row_ct<BN, BN_OUT, KIND, SWIGLU, HX_S32>(e, t_row, m, n_base, c0, pf, stg);
      break;
    default: break;
  }
}

// Runtime-dispatched staged store for the split-K reduction.
__device__ __forceinline__ void epi_store32_staged_rt(const EpiArgs &e, const float (&v)[32],
                                                      const uint32_t (&raw)[32], bool raw_int, int m0,
                                                      int n0, uint8_t *stg) {
  switch (e.c_dtype) {
    case HX_F16: epi_store32_staged_t<HX_F16, false>(e, v, raw, m0, n0, stg); break;
    case HX_BF16: epi_store32_staged_t<HX_BF16, false>(e, v, raw, m0, n0, stg); break;
    case HX_F32: epi_store32_staged_t<HX_F32, false>(e, v, raw, m0, n0, stg); break;
    default:
      if (raw_int) epi_store32_staged_t<HX_S32, true>(e, v, raw, m0, n0, stg);
      else epi_store32_staged_t<HX_S32, false>(e, v, raw, m0, n0, stg);
      break;
  }
}

template <int BN, int KIND, bool B_MN, bool SWIGLU>
__global__ void __launch_bounds__(kThreads, 1)
    hx_gemm_sm100_kernel(const __grid_constant__ CUtensorMap tmA,
                         const __grid_constant__ CUtensorMap tmB,
                         const __grid_constant__ GemmParams p) {
  using Cfg = GemmCfg<BN, KIND, B_MN, SWIGLU>;
  const int STAGES = p.stages;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte alignment for the 128B-swizzle atoms.
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int A_ST = p.kbs * Cfg::kABytes;  // bytes of A per stage
  const int B_ST = p.kbs * Cfg::kBBytes;  // bytes of B per stage
  uint8_t *sA = smem;
  uint8_t *sB = smem + STAGES * A_ST;
  // Split-K lands remote partials in the ring once the mainloop is done: the
  // barriers go after whichever of the two is larger.
  const int ring_bytes = STAGES * (A_ST + B_ST);
  const int red_bytes = (p.splits > 1 && p.red_smem) ? Cfg::red_bytes(p.splits) : 0;
  uint64_t *full_bar = reinterpret_cast<uint64_t *>(smem + (ring_bytes > red_bytes ? ring_bytes : red_bytes));
  uint64_t *empty_bar = full_bar + STAGES;
  uint64_t *tfull_bar = empty_bar + STAGES;   // [2]
  uint64_t *tempty_bar = tfull_bar + 2;       // [2]
  uint64_t *drain_bar = tempty_bar + 2;       // [1]
  uint64_t *red_bar = drain_bar + 1;          // [1] split-K: remote partials landed
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(red_bar + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
  uint8_t *stage_out = reinterpret_cast<uint8_t *>(full_bar) + kBarBytes;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) HX_GEMM_STAMP(0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], kEpiWarps);
    }
    mbar_init(drain_bar, 1);
    mbar_init(red_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Prologue done: let the next kernel in the stream start its own.  The
  // producer and the epilogue wait for the previous one before touching
  // global memory (griddepcontrol.wait below); the UMMA warp touches none.
  grid_dep_launch_dependents();
  if (threadIdx.x == 0) HX_GEMM_STAMP(1);

  // Split-K: the CTAs of a cluster share each tile; CTA `rank` streams stage
  // blocks [sb_begin, sb_end) of it.  Without split-K: the whole K range.
  const int S = p.splits;
  const uint32_t rank = S > 1 ? gemm_cluster_rank() : 0u;
  const int t_first = blockIdx.x / S, t_step = gridDim.x / S;
  const int sper = p.stage_blocks / S, srem = p.stage_blocks % S;
  const int sb_begin = static_cast<int>(rank) * sper + min(static_cast<int>(rank), srem);
  const int sb_end = sb_begin + sper + (static_cast<int>(rank) < srem ? 1 : 0);

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    auto load_a = [&](uint64_t *fb, int stage, int m0, int sb, int b) {
      uint8_t *dstA = sA + stage * A_ST;
      if (p.conv) {  // kbs == 1: one filter tap x 64 channels of 128 pixels
        const int hw = p.conv_H * p.conv_W;
        const int img = m0 / hw, rem = m0 - img * hw;
        const int h0 = rem / p.conv_W, w0 = rem - h0 * p.conv_W;
        const int tap = sb / p.conv_cpb, cb = sb - tap * p.conv_cpb;
        const int kh = tap / p.conv_KW, kw = tap - kh * p.conv_KW;
        tma_load_4d(dstA, &tmA, fb, cb * Cfg::kBKElems, w0 + kw - p.conv_pad_w, h0 + kh - p.conv_pad_h, img);
      } else if (p.batch > 1)
        tma_load_3d(dstA, &tmA, fb, sb * Cfg::kBKElems, m0, b);
      else if (!B_MN && p.use3d)
        tma_load_3d(dstA, &tmA, fb, 0, m0, sb * p.kbs);
      else
        tma_load_2d(dstA, &tmA, fb, sb * Cfg::kBKElems, m0);
    };
    auto load_b = [&](uint64_t *fb, int stage, int n_blk, int sb, int b) {
      uint8_t *dstB = sB + stage * B_ST;
      if constexpr (B_MN) {  // kbs == 1, 2-D maps (3-D with the batch item outermost)
        const int kx = sb * Cfg::kBKElems;
        const int n0 = n_blk * BN;
#pragma unroll
        for (int j = 0; j < BN / Cfg::kMNChunk; ++j) {
          if (p.batch > 1)
            tma_load_3d(dstB + j * (Cfg::kBKElems * 128), &tmB, fb, n0 + j * Cfg::kMNChunk, kx, b);
          else
            tma_load_2d(dstB + j * (Cfg::kBKElems * 128), &tmB, fb, n0 + j * Cfg::kMNChunk, kx);
        }
      } else if (p.batch > 1) {  // kbs == 1, no SWIGLU
        tma_load_3d(dstB, &tmB, fb, sb * Cfg::kBKElems, n_blk * BN, b);
      } else if (p.use3d) {
        const int kz = sb * p.kbs;
        if constexpr (SWIGLU) {
          const int n0 = n_blk * (BN / 2);
          tma_load_3d(dstB, &tmB, fb, 0, n0, kz);
          tma_load_3d(dstB + B_ST / 2, &tmB, fb, 0, p.n_half + n0, kz);
        } else {
          tma_load_3d(dstB, &tmB, fb, 0, n_blk * BN, kz);
        }
      } else {  // kbs == 1, 2-D maps
        const int kx = sb * Cfg::kBKElems;
        if constexpr (SWIGLU) {
          const int n0 = n_blk * (BN / 2);
          tma_load_2d(dstB, &tmB, fb, kx, n0);
          tma_load_2d(dstB + B_ST / 2, &tmB, fb, kx, p.n_half + n0);
        } else {
          tma_load_2d(dstB, &tmB, fb, kx, n_blk * BN);
        }
      }
    };
    // Constant B (model weights): the first tile's first stages of B are
    // fetched before waiting for the previous kernel, overlapping its tail.
    int pre = 0;
    if (p.b_const && t_first < p.total_tiles) pre = min(STAGES, sb_end - sb_begin);
    if (lane == 0 && pre > 0) {
      int b, m_blk, n_blk;
      tile_coords_b(t_first, p, b, m_blk, n_blk);
      for (int i = 0; i < pre; ++i) {
        mbar_arrive_expect_tx(&full_bar[i], A_ST + B_ST);
        load_b(&full_bar[i], i, n_blk, sb_begin + i, b);
      }
    }
    grid_dep_wait();
    if (threadIdx.x == 0) HX_GEMM_STAMP(2);
    int stage = 0;
    uint32_t phase = 0;
    int64_t issued = pre;
    bool ok = true;
    for (int t = t_first; t < p.total_tiles && ok; t += t_step) {
      int b, m_blk, n_blk;
      tile_coords_b(t, p, b, m_blk, n_blk);
      const int m0 = m_blk * kBM;
      for (int sb = sb_begin; sb < sb_end; ++sb) {
        const bool early = (t == t_first) && (sb - sb_begin < pre);  // B already in flight
        if (!early) {
          bool w = (lane == 0) ? mbar_wait(&empty_bar[stage], phase ^ 1, p.timeout, abort_flag)
                               : true;
          w = __shfl_sync(0xffffffffu, w, 0);
          if (!w) {
            if (lane == 0) raise_abort(abort_flag, p.err_flag, 1);
            ok = false;
            break;
          }
        }
        if (lane == 0) {
          uint64_t *fb = &full_bar[stage];
          if (!early) mbar_arrive_expect_tx(fb, A_ST + B_ST);
          load_a(fb, stage, m0, sb, b);
          if (!early) load_b(fb, stage, n_blk, sb, b);
        }
        __syncwarp();
        if (!early) ++issued;
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
    if (!ok && lane == 0) {
      // Drain: every load still in flight lands before the CTA exits.
      const int64_t first = issued > STAGES ? issued - STAGES : 0;
      for (int64_t i = first; i < issued; ++i) {
        int dummy_abort = 0;
        mbar_wait(&full_bar[i % STAGES], static_cast<uint32_t>((i / STAGES) & 1), p.timeout,
                  &dummy_abort);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ UMMA issuer
    int stage = 0;
    uint32_t phase = 0;
    int it = 0;
    bool ok = true;
    bool any_mma = false;
    for (int t = t_first; t < p.total_tiles && ok; t += t_step, ++it) {
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      bool w = (lane == 0) ? mbar_wait(&tempty_bar[acc], acc_phase ^ 1, p.timeout, abort_flag)
                           : true;
      w = __shfl_sync(0xffffffffu, w, 0);
      if (!w) {
        if (lane == 0) raise_abort(abort_flag, p.err_flag, 2);
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + acc * BN;
      for (int sb = sb_begin; sb < sb_end; ++sb) {
        bool f = (lane == 0) ? mbar_wait(&full_bar[stage], phase, p.timeout, abort_flag) : true;
        if (it == 0 && sb == sb_begin && lane == 0) HX_GEMM_STAMP(3);
        f = __shfl_sync(0xffffffffu, f, 0);
        if (!f) {
          if (lane == 0) raise_abort(abort_flag, p.err_flag, 3);
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t a_base = smem_u32(sA + stage * A_ST);
          const uint32_t b_base = smem_u32(sB + stage * B_ST);
          for (int j = 0; j < p.kbs; ++j) {
#pragma unroll
            for (int k = 0; k < kKBytes / kUmmaKBytes; ++k) {
              const uint64_t adesc = sdesc_kmajor_sw128(a_base + j * Cfg::kABytes + k * kUmmaKBytes);
              const uint32_t accum = (sb > sb_begin || j > 0 || k > 0) ? 1u : 0u;
              if constexpr (B_MN) {
                // UMMA K step = kUmmaK rows of K = kUmmaK/8 swizzle atoms of 1024 B.
                const uint64_t bdesc = sdesc_mnmajor_sw128(b_base + k * (Cfg::kUmmaK / 8) * 1024,
                                                           Cfg::kBKElems * 128);
                if constexpr (KIND == 2)
                  umma_i8(d_tmem, adesc, bdesc, Cfg::kIdesc, accum);
                else
                  umma_f16(d_tmem, adesc, bdesc, Cfg::kIdesc, accum);
              } else if constexpr (SWIGLU) {
                // gate rows and up rows are separate boxes: two N/2 products
                const uint32_t hb = (BN / 2) * kKBytes;
                const uint64_t gdesc = sdesc_kmajor_sw128(b_base + j * hb + k * kUmmaKBytes);
                const uint64_t udesc =
                    sdesc_kmajor_sw128(b_base + B_ST / 2 + j * hb + k * kUmmaKBytes);
                umma_f16(d_tmem, adesc, gdesc, Cfg::kIdescHalf, accum);
                umma_f16(d_tmem + BN / 2, adesc, udesc, Cfg::kIdescHalf, accum);
              } else {
                const uint64_t bdesc =
                    sdesc_kmajor_sw128(b_base + j * Cfg::kBBytes + k * kUmmaKBytes);
                if constexpr (KIND == 2)
                  umma_i8(d_tmem, adesc, bdesc, Cfg::kIdesc, accum);
                else
                  umma_f16(d_tmem, adesc, bdesc, Cfg::kIdesc, accum);
              }
            }
          }
          umma_commit(&empty_bar[stage]);  // frees the smem stage when read
          any_mma = true;
        }
        __syncwarp();
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (!ok) break;
      if (lane == 0) umma_commit(&tfull_bar[acc]);  // accumulator ready
      if (it == 0 && lane == 0) HX_GEMM_STAMP(4);
      __syncwarp();
    }
    if (!ok && lane == 0 && any_mma) {
      // Drain: wait until every issued UMMA has finished before TMEM is freed.
      umma_commit(drain_bar);
      int dummy_abort = 0;
      mbar_wait(drain_bar, 0, p.timeout, &dummy_abort);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    grid_dep_wait();  // C / residual / bias may come from the previous kernel
    const int q = warp & 3;                   // TMEM lane quarter this warp may access
    const int row_in_tile = q * 32 + lane;
    int it = 0;
    for (int t = t_first; t < p.total_tiles; t += t_step, ++it) {
      int b, m_blk, n_blk;
      tile_coords_b(t, p, b, m_blk, n_blk);
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      const int m = b * p.batch_rows + m_blk * kBM + row_in_tile;  // flattened row of C
      const int c0 = (warp - 2) / 4;
      Pre16 pf;
      if (S == 1) epi_row_prefetch<SWIGLU>(p.epi, m, n_blk * Cfg::kBNOut + c0 * 32, pf);
      bool w = (lane == 0) ? mbar_wait(&tfull_bar[acc], acc_phase, p.timeout, abort_flag) : true;
      w = __shfl_sync(0xffffffffu, w, 0);
      if (!w) {
        if (lane == 0) raise_abort(abort_flag, p.err_flag, 4);
        break;
      }
      if (it == 0 && warp == 2 && lane == 0) HX_GEMM_STAMP(5);
      tc_fence_after();
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN;
      if (S > 1) {
        // Split-K: write the partial columns that other ranks own to this
        // CTA's slot of the L2 workspace (raw fp32 / int32 bits), laid out
        // [column chunk][4-column group][row] in 16-byte units so a warp's 32
        // rows fill 512 contiguous bytes.  Chunks this rank owns stay in TMEM
        // (one tile per cluster: the accumulator is not released).
        uint4 *slot = p.ws + (static_cast<size_t>(t) * S + rank) * (BN / 32) * 8 * kBM;
#pragma unroll 1
        for (int c = (warp - 2) / 4; c < BN / 32; c += 2) {
          if ((c % (Cfg::kBNOut / 32)) % S == static_cast<int>(rank)) continue;
          uint32_t r[32];
          tmem_ld_32x32b_x32(t_row + c * 32, r);
          tmem_ld_wait();
#pragma unroll
          for (int g = 0; g < 8; ++g)
            slot[(c * 8 + g) * kBM + row_in_tile] = make_uint4(r[4 * g], r[4 * g + 1], r[4 * g + 2], r[4 * g + 3]);
        }
        if (it == 0 && warp == 2 && lane == 0) HX_GEMM_STAMP(6);
        continue;
      }
      epi_row<BN, Cfg::kBNOut, KIND, SWIGLU>(p.epi, t_row, m, n_blk * Cfg::kBNOut, c0, pf,
                                             stage_out + (warp - 2) * 4096);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty_bar[acc]);
      if (it == 0 && warp == 2 && lane == 0) HX_GEMM_STAMP(6);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  if (S > 1) {
    // Every CTA's non-owned partials are in the workspace (the cluster
    // barrier's release / acquire makes them visible).  Each CTA fetches the
    // partials of the output chunks it owns (chunk oc belongs to rank oc % S)
    // into its idle stage ring with 16 KB bulk copies, then reduces them in
    // rank order — its own straight from TMEM — applies the epilogue once and
    // stores.  Ring slot of (owned chunk j, remote rank index ri, half h):
    // ((j * (S - 1) + ri) * H + h) * 16 KB, H = 2 for SWIGLU (gate, up).
    constexpr int kH = SWIGLU ? 2 : 1;
    constexpr int kChunkBytes = 8 * kBM * 16;
    constexpr int kUpChunk = Cfg::kBNOut / 32;  // SWIGLU: up half starts here
    const int n_own = (Cfg::kBNOut / 32 - static_cast<int>(rank) + S - 1) / S;
    if (threadIdx.x == 0) HX_GEMM_STAMP(12);
    gemm_cluster_sync();
    if (threadIdx.x == 64) HX_GEMM_STAMP(13);
    const bool via_smem = p.red_smem != 0;
    if (threadIdx.x == 64 && via_smem) {
      asm volatile("fence.proxy.async.global;" ::: "memory");  // generic writes -> bulk reads
      const uint32_t bytes = static_cast<uint32_t>(n_own * (S - 1) * kH * kChunkBytes);
      if (bytes > 0) {
        mbar_arrive_expect_tx(red_bar, bytes);
        for (int t = t_first; t < p.total_tiles; t += t_step) {  // one tile per cluster
          for (int j = 0; j < n_own; ++j) {
            const int oc = static_cast<int>(rank) + j * S;
            int ri = 0;
            for (int rr = 0; rr < S; ++rr) {
              if (rr == static_cast<int>(rank)) continue;
              const uint4 *src = p.ws + (static_cast<size_t>(t) * S + rr) * (BN / 32) * 8 * kBM;
              for (int h = 0; h < kH; ++h)
                bulk_load_1d(smem + ((j * (S - 1) + ri) * kH + h) * kChunkBytes,
                             src + (h ? kUpChunk + oc : oc) * 8 * kBM, kChunkBytes, red_bar);
              ++ri;
            }
          }
        }
      }
    }
    if (warp >= 2) {
      const int q = warp & 3;
      const int row_in_tile = q * 32 + lane;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16);  // accumulator 0
      const bool raw_int = (KIND == 2) && (p.epi.c_dtype == HX_S32) && (p.epi.epi == HX_EPI_NONE);
      bool landed = (n_own == 0 || !via_smem) || (lane == 0 ? mbar_wait(red_bar, 0, p.timeout, abort_flag) : true);
      landed = __shfl_sync(0xffffffffu, landed, 0);
      if (!landed && lane == 0) {
        raise_abort(abort_flag, p.err_flag, 5);
        int ignored = 0;  // let copies still in flight land before the CTA exits
        if (warp == 2) mbar_wait(red_bar, 0, p.timeout, &ignored);
      }
      for (int t = t_first; landed && t < p.total_tiles; t += t_step) {  // one tile per cluster
        int m_blk, n_blk;
        tile_coords(t, p, m_blk, n_blk);
        const int m = m_blk * kBM + row_in_tile;
#pragma unroll 1
        for (int j = (warp - 2) / 4; j < n_own; j += 2) {  // two warps per row quarter
          const int oc = static_cast<int>(rank) + j * S;
          uint32_t own[32], ownu[32];
          tmem_ld_32x32b_x32(t_row + oc * 32, own);
          if constexpr (SWIGLU) tmem_ld_32x32b_x32(t_row + (kUpChunk + oc) * 32, ownu);
          tmem_ld_wait();
          uint32_t r[32];
          float v[32], up[32];
#pragma unroll
          for (int jj = 0; jj < 32; ++jj) {
            r[jj] = 0u;
            v[jj] = 0.f;
            up[jj] = 0.f;
          }
          int ri = 0;
#pragma unroll 1
          for (int rr = 0; rr < S; ++rr) {
            uint32_t x[32], u[32];
            if (rr == static_cast<int>(rank)) {
#pragma unroll
              for (int jj = 0; jj < 32; ++jj) {
                x[jj] = own[jj];
                u[jj] = SWIGLU ? ownu[jj] : 0u;
              }
            } else if (!via_smem) {  // partials too large for the ring: read them from L2
              const uint4 *src = p.ws + (static_cast<size_t>(t) * S + rr) * (BN / 32) * 8 * kBM + row_in_tile;
#pragma unroll
              for (int g = 0; g < 8; ++g) {
                const uint4 w = __ldcg(src + (oc * 8 + g) * kBM);
                x[4 * g] = w.x;
                x[4 * g + 1] = w.y;
                x[4 * g + 2] = w.z;
                x[4 * g + 3] = w.w;
              }
              if constexpr (SWIGLU) {
#pragma unroll
                for (int g = 0; g < 8; ++g) {
                  const uint4 w = __ldcg(src + ((kUpChunk + oc) * 8 + g) * kBM);
                  u[4 * g] = w.x;
                  u[4 * g + 1] = w.y;
                  u[4 * g + 2] = w.z;
                  u[4 * g + 3] = w.w;
                }
              }
            } else {
              const uint8_t *slot = smem + ((j * (S - 1) + ri) * kH) * kChunkBytes + row_in_tile * 16;
#pragma unroll
              for (int g = 0; g < 8; ++g) {
                const uint4 w = *reinterpret_cast<const uint4 *>(slot + g * kBM * 16);
                x[4 * g] = w.x;
                x[4 * g + 1] = w.y;
                x[4 * g + 2] = w.z;
                x[4 * g + 3] = w.w;
              }
              if constexpr (SWIGLU) {
#pragma unroll
                for (int g = 0; g < 8; ++g) {
                  const uint4 w = *reinterpret_cast<const uint4 *>(slot + kChunkBytes + g * kBM * 16);
                  u[4 * g] = w.x;
                  u[4 * g + 1] = w.y;
                  u[4 * g + 2] = w.z;
                  u[4 * g + 3] = w.w;
                }
              }
              ++ri;
            }
#pragma unroll
            for (int jj = 0; jj < 32; ++jj) {
              if constexpr (KIND == 2) r[jj] += x[jj];
              else v[jj] += __uint_as_float(x[jj]);
              if constexpr (SWIGLU) up[jj] += __uint_as_float(u[jj]);
            }
          }
          if constexpr (KIND == 2) {
#pragma unroll
            for (int jj = 0; jj < 32; ++jj) v[jj] = static_cast<float>(static_cast<int32_t>(r[jj]));
          }
          const int n0 = n_blk * Cfg::kBNOut + oc * 32;
          if (!raw_int) epi_transform32(p.epi, v, up, m, n0);
          if (p.epi.c_vec_ok && n0 + 32 <= p.epi.N && p.epi.n_peers == 0)
            epi_store32_staged_rt(p.epi, v, r, raw_int, m - lane, n0, stage_out + (warp - 2) * 4096);
          else
            epi_store32(p.epi, v, r, raw_int, m, n0);
        }
      }
    }
    if (threadIdx.x == 64) HX_GEMM_STAMP(14);
    // the reduction read this CTA's own partial from TMEM: free it only after
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
  }

  // fused all-gather: peer stores are visible system-wide before the grid ends
  if (p.epi.n_peers > 0) __threadfence_system();
  if (warp == 1) tmem_dealloc(tmem_base, Cfg::kTmemCols);
  if (threadIdx.x == 0) HX_GEMM_STAMP(7);
}

}  // namespace hx
