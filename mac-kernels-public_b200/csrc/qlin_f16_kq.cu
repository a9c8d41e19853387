// Instantiations of the weight-only (kind::f16) fused dequantize + GEMM for the K-quant formats Q2_K,
// Q3_K, Q4_K, Q5_K and Q6_K.
#include <cuda_runtime.h>

#include "qlin_f16_launch.cuh"

namespace qlin {

int dispatch_f16_kq(int fmt, const CUtensorMap& tx, const CUtensorMap& tw, const CUtensorMap& tp,
                    const CUtensorMap& tt, const PeerMaps& maps, const GemmParams& p, int tm, bool pair, cudaStream_t stream) {
  switch (fmt) {
    case WF_Q2_K: return dispatch_tm<DecQ23_K<false>>(tx, tw, tp, tt, maps, p, tm, pair, stream);
    case WF_Q3_K: return dispatch_tm<DecQ23_K<true>>(tx, tw, tp, tt, maps, p, tm, pair, stream);
    case WF_Q4_K: return dispatch_tm<DecQ4_K>(tx, tw, tp, tt, maps, p, tm, pair, stream);
    case WF_Q5_K: return dispatch_tm<DecQ5_K>(tx, tw, tp, tt, maps, p, tm, pair, stream);
    case WF_Q6_K: return dispatch_tm<DecQ6_K>(tx, tw, tp, tt, maps, p, tm, pair, stream);
    default: return -1;
  }
}

// This translation unit's bounds record (QLIN_CHECKS build).
QLIN_BOUNDS_READER(bounds_read_f16_kq)

}  // namespace qlin
