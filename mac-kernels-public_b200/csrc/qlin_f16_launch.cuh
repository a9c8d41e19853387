// Launch templates of the weight-only (kind::f16) fused dequantize + GEMM, shared by the
// translation units that instantiate it: qlin_f16.cu (INT8, Q8_0, Q4_0, IQ4_NL), qlin_f16_blk.cu
// (Q4_1, Q5_0, Q5_1, IQ4_XS) and qlin_f16_kq.cu (Q2_K .. Q6_K), which compile in parallel.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "qlin_gemm.cuh"
#include "qlin_internal.h"

namespace qlin {

template <class Dec, int TM, int STAGES, bool PAIR, bool ROT = false>
static int launch_one(const CUtensorMap& tx, const CUtensorMap& tw, const CUtensorMap& tp, const CUtensorMap& tt,
                      const PeerMaps& maps,
                      const GemmParams& p, cudaStream_t stream) {
  constexpr int smem = qgemm_f16_smem_bytes<Dec, TM, STAGES, PAIR>();
  static_assert(smem <= 232448, "shared memory per CTA");
  auto kern = qgemm_f16_kernel<Dec, TM, STAGES, PAIR, ROT>;
  static bool attr_done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_done[dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) {
      set_error("cudaFuncSetAttribute(max dynamic smem %d) failed", smem);
      return 3;
    }
    attr_done[dev] = true;
  }
  constexpr int kCtas = PAIR ? 2 : 1;
  const int tiles = p.m_tiles * (p.n_tiles / kCtas) * p.k_splits;
  const int grid = kCtas * std::min(tiles, sm_count() / kCtas);
  cudaError_t e;
  if constexpr (PAIR) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(F16Cfg<TM, STAGES, PAIR>::kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, kern, tx, tw, tp, tt, maps, p);
  } else {
    kern<<<grid, F16Cfg<TM, STAGES, PAIR>::kThreads, smem, stream>>>(tx, tw, tp, tt, maps, p);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) {
    set_error("qgemm_f16 launch failed: %s", cudaGetErrorString(e));
    return 3;
  }
  return 0;
}

template <class Dec, int TM, bool ROT = false>
static int launch_tm(const CUtensorMap& tx, const CUtensorMap& tw, const CUtensorMap& tp, const CUtensorMap& tt,
                      const PeerMaps& maps,
                     const GemmParams& p, bool pair, cudaStream_t stream) {
  if constexpr (TM >= 128) {
    if (pair) return launch_one<Dec, TM, qgemm_f16_stages<Dec, TM, true>(), true, ROT>(tx, tw, tp, tt, maps, p, stream);
  }
  return launch_one<Dec, TM, qgemm_f16_stages<Dec, TM, false>(), false, ROT>(tx, tw, tp, tt, maps, p, stream);
}

template <class Dec, bool ROT = false>
static int dispatch_tm(const CUtensorMap& tx, const CUtensorMap& tw, const CUtensorMap& tp, const CUtensorMap& tt,
                      const PeerMaps& maps,
                       const GemmParams& p, int tm, bool pair, cudaStream_t stream) {
  switch (tm) {
    case 16: return launch_tm<Dec, 16, ROT>(tx, tw, tp, tt, maps, p, pair, stream);
    case 32: return launch_tm<Dec, 32, ROT>(tx, tw, tp, tt, maps, p, pair, stream);
    case 64: return launch_tm<Dec, 64, ROT>(tx, tw, tp, tt, maps, p, pair, stream);
    case 128: return launch_tm<Dec, 128, ROT>(tx, tw, tp, tt, maps, p, pair, stream);
    case 192: return launch_tm<Dec, 192, ROT>(tx, tw, tp, tt, maps, p, pair, stream);
    case 256: return launch_tm<Dec, 256, ROT>(tx, tw, tp, tt, maps, p, pair, stream);
    default: set_error("unsupported token tile %d", tm); return 2;
  }
}

// Per-format dispatch of the other translation units; -1 when the format is not theirs.
int dispatch_f16_blk(int fmt, const CUtensorMap& tx, const CUtensorMap& tw, const CUtensorMap& tp,
                     const CUtensorMap& tt, const PeerMaps& maps, const GemmParams& p, int tm, bool pair,
                     cudaStream_t stream);
int dispatch_f16_kq(int fmt, const CUtensorMap& tx, const CUtensorMap& tw, const CUtensorMap& tp,
                    const CUtensorMap& tt, const PeerMaps& maps, const GemmParams& p, int tm, bool pair,
                    cudaStream_t stream);

}  // namespace qlin
