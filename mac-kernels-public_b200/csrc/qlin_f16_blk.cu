// Instantiations of the weight-only (kind::f16) fused dequantize + GEMM for the 32-value block formats
// Q4_1, Q5_0, Q5_1 and IQ4_XS.
#include <cuda_runtime.h>

#include "qlin_f16_launch.cuh"

namespace qlin {

int dispatch_f16_blk(int fmt, const CUtensorMap& tx, const CUtensorMap& tw, const CUtensorMap& tp,
                     const CUtensorMap& tt, const PeerMaps& maps, const GemmParams& p, int tm, bool pair, cudaStream_t stream) {
  switch (fmt) {
    case WF_Q4_1: return dispatch_tm<DecQ4_1>(tx, tw, tp, tt, maps, p, tm, pair, stream);
    case WF_Q5_0: return dispatch_tm<DecQ5Block<false>>(tx, tw, tp, tt, maps, p, tm, pair, stream);
    case WF_Q5_1: return dispatch_tm<DecQ5Block<true>>(tx, tw, tp, tt, maps, p, tm, pair, stream);
    case WF_IQ4_XS: return dispatch_tm<DecIQ4<true>>(tx, tw, tp, tt, maps, p, tm, pair, stream);
    default: return -1;
  }
}

// This translation unit's bounds record (QLIN_CHECKS build).
QLIN_BOUNDS_READER(bounds_read_f16_blk)

}  // namespace qlin
