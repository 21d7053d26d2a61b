// launch_impl.cuh — tile-GEMM launchers; included only by gemm_kind*.cu,
// each of which instantiates one input kind.
#pragma once
#include <algorithm>
#include "gemm_sm100.cuh"
#include "gemm_sm100_2sm.cuh"
#include "launch.cuh"

namespace hx {

template <int BN, int KIND, bool BMN, bool SW>
int launch_tc(const CUtensorMap &ta, const CUtensorMap &tb, const GemmParams &p, int grid,
              cudaStream_t s) {
  using Cfg = GemmCfg<BN, KIND, BMN, SW>;
  auto kern = hx_gemm_sm100_kernel<BN, KIND, BMN, SW>;
  const int ring = p.stages * p.kbs * Cfg::kStageBytes;
  const int fixed = 1024 + kBarBytes + kStageOutBytes;
  GemmParams q = p;
  q.red_smem = (p.splits > 1 && Cfg::red_bytes(p.splits) + fixed <= kMaxDynSmem) ? 1 : 0;
  const int smem = std::max(ring, q.red_smem ? Cfg::red_bytes(p.splits) : 0) + fixed;
  if (smem > kMaxDynSmem) return unsupported("shared memory for this tile plan exceeds 227 KB");
  static SmemAttrOnce attr_once;
  {
    cudaError_t e = ensure_max_smem(kern, attr_once);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute");
  }
  cudaError_t e;
  if (p.splits > 1) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = p.splits;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    // Split-K runs one tile per cluster; clusters that do not all fit at once
    // would run as a second wave, so such plans fall back to no split.
    // The resident-cluster count depends on the device, so it is cached per ordinal.
    static std::atomic<int> max_clusters[kMaxDevices][9];
    const int dev = current_device_ordinal();
    int mc = dev >= 0 ? max_clusters[dev][p.splits].load(std::memory_order_acquire) : 0;
    if (mc == 0) {
      e = cudaOccupancyMaxActiveClusters(&mc, kern, &cfg);
      if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveClusters");
      mc = std::max(mc, 1);
      if (dev >= 0) max_clusters[dev][p.splits].store(mc, std::memory_order_release);
    }
    if (grid / p.splits > mc) return kNeedsNoSplit;
    cfg.numAttrs = 2;
    e = cudaLaunchKernelEx(&cfg, kern, ta, tb, q);
  } else {
    e = launch_pdl(kern, dim3(grid), dim3(kThreads), smem, s, ta, tb, q);
  }
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "hx_gemm_sm100_kernel launch");
  return HX_OK;
}

template <int BN, int KIND, bool SW>
int launch_pair(const CUtensorMap &ta, const CUtensorMap &tb, const GemmParams &p, int grid,
                cudaStream_t s) {
  auto kern = hx_gemm_sm100_2sm_kernel<BN, KIND, SW>;
  const int stage = p.kbs * (kBM * kKBytes + (BN / 2) * kKBytes);
  const int smem = p.stages * stage + 1024 + kBarBytes + kStageOutBytes;
  if (smem > kMaxDynSmem) return unsupported("shared memory for this pair plan exceeds 227 KB");
  static SmemAttrOnce attr_once;
  {
    cudaError_t e = ensure_max_smem(kern, attr_once);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(pair)");
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, ta, tb, p);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "hx_gemm_sm100_2sm_kernel launch");
  return HX_OK;
}

template <int KIND>
int dispatch_pair_kind(int bn, bool sw, const CUtensorMap &ta, const CUtensorMap &tb,
                       const GemmParams &p, int grid, cudaStream_t s) {
  if (bn != 256) return unsupported("pair tiles use tile_n 256");
  if (sw) {
    if constexpr (KIND == 2) return unsupported("SWIGLU with int8 inputs");
    else return launch_pair<256, KIND, true>(ta, tb, p, grid, s);
  }
  return launch_pair<256, KIND, false>(ta, tb, p, grid, s);
}

template <int KIND, bool BMN, bool SW>
int dispatch_bn(int bn, const CUtensorMap &ta, const CUtensorMap &tb, const GemmParams &p,
                int grid, cudaStream_t s) {
  switch (bn) {
    case 64:
      if constexpr (!(BMN && KIND == 2)) return launch_tc<64, KIND, BMN, SW>(ta, tb, p, grid, s);
      return unsupported("tile_n 64 with int8 B[K,N]");
    case 96:
      if constexpr (!BMN && !SW) return launch_tc<96, KIND, BMN, SW>(ta, tb, p, grid, s);
      return unsupported("tile_n 96 with B[K,N] or SWIGLU");
    case 128: return launch_tc<128, KIND, BMN, SW>(ta, tb, p, grid, s);
    case 192:
      if constexpr (!BMN) return launch_tc<192, KIND, BMN, SW>(ta, tb, p, grid, s);
      return unsupported("tile_n 192 with B[K,N]");
    case 256: return launch_tc<256, KIND, BMN, SW>(ta, tb, p, grid, s);
    default: return unsupported("tile_n");
  }
}

template <int KIND>
int dispatch_kind(int bn, bool bmn, bool sw, const CUtensorMap &ta, const CUtensorMap &tb,
                  const GemmParams &p, int grid, cudaStream_t s) {
  if (bmn) return dispatch_bn<KIND, true, false>(bn, ta, tb, p, grid, s);
  if (sw) {
    if constexpr (KIND == 2) return unsupported("SWIGLU with int8 inputs");
    else return dispatch_bn<KIND, false, true>(bn, ta, tb, p, grid, s);
  }
  return dispatch_bn<KIND, false, false>(bn, ta, tb, p, grid, s);
}


}  // namespace hx

#define HX_INSTANTIATE_KIND(K)                                                                  \
  template int hx::dispatch_kind<K>(int, bool, bool, const CUtensorMap &, const CUtensorMap &,  \
                                    const hx::GemmParams &, int, cudaStream_t);                 \
  template int hx::dispatch_pair_kind<K>(int, bool, const CUtensorMap &, const CUtensorMap &,   \
                                         const hx::GemmParams &, int, cudaStream_t);
