// Host launcher of the W4A8 / W6A8 kind::i8 GEMM and the one-time 6-bit repack.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "qlin_gemm_i8.cuh"
#include "qlin_gemm_i8p.cuh"
#include "qlin_internal.h"

namespace qlin {

int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elem, uint64_t cols, uint64_t rows,
                 uint64_t pitch_bytes, uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle swz);

// 6-bit weights -> "W6 planes" stage chunks (layout documented at DecW6).
//   layout 0: four values per three bytes, u0 | u1<<6 | u2<<12 | u3<<18 little-endian, u = q + 32
//   layout 1: comfy-kitchen planar (modal/weight_error_app.py:145-152): K/2 nibble bytes, then K/4
//             bytes of 2-bit high planes; codes are used as stored (u = code)
// grid = (K/128, n_tiles), block = 128 (one weight row per thread).
__global__ void w6_repack_kernel(const uint8_t* __restrict__ src, int layout, int N, int K, int num_k_stages,
                                 uint8_t* __restrict__ out, long long out_bytes) {
  const int kst = blockIdx.x, nt = blockIdx.y, r = threadIdx.x;
  const int n = nt * 128 + r;
  uint8_t* st = out + ((size_t)nt * num_k_stages + kst) * (128 * 96);
  uint32_t L[16], T[8];
#pragma unroll
  for (int i = 0; i < 16; ++i) L[i] = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) T[i] = 0;
  if (n < N) {
    const size_t row_bytes = (size_t)K * 3 / 4;
    const uint8_t* row = src + (size_t)n * row_bytes;
    for (int u = 0; u < 8; ++u) {
      uint32_t code[16];
      for (int i = 0; i < 16; ++i) {
        const int k = kst * 128 + u * 16 + i;
        uint32_t c = 0;
        const long long src_bytes = (long long)N * row_bytes;
        if (layout == 0) {
          if (!qchk_span(BS_REPACK_SRC, (long long)n * row_bytes + (k / 4) * 3, 3, src_bytes)) continue;
          const uint8_t* w = row + (k / 4) * 3;
          const uint32_t word = w[0] | (w[1] << 8) | (w[2] << 16);
          c = (word >> (6 * (k & 3))) & 0x3F;
        } else {
          if (!qchk(BS_REPACK_SRC, (long long)n * row_bytes + k / 2, src_bytes) ||
              !qchk(BS_REPACK_SRC, (long long)n * row_bytes + K / 2 + k / 4, src_bytes))
            continue;
          const uint32_t lo = (row[k / 2] >> (4 * (k & 1))) & 0xF;
          const uint32_t hi = (row[K / 2 + k / 4] >> (2 * (k & 3))) & 0x3;
          c = lo | (hi << 4);
        }
        code[i] = c;
      }
      uint32_t l0 = 0, l1 = 0, t = 0;
      for (int i = 0; i < 8; ++i) {
        l0 |= (code[i] & 0xF) << (4 * i);
        l1 |= (code[8 + i] & 0xF) << (4 * i);
      }
      for (int b = 0; b < 4; ++b) {
        const uint32_t byte = (code[2 * b] >> 4) | ((code[2 * b + 1] >> 4) << 2) | ((code[8 + 2 * b] >> 4) << 4) |
                              ((code[9 + 2 * b] >> 4) << 6);
        t |= byte << (8 * b);
      }
      L[2 * u] = l0;
      L[2 * u + 1] = l1;
      T[u] = t;
    }
  }
  const long long st_off = ((long long)nt * num_k_stages + kst) * (128 * 96);
  for (int j = 0; j < 4; ++j)
    if (qchk_span(BS_REPACK_DST, st_off + (j * 128 + r) * 16, 16, out_bytes))
      *reinterpret_cast<uint4*>(st + (j * 128 + r) * 16) = make_uint4(L[4 * j], L[4 * j + 1], L[4 * j + 2], L[4 * j + 3]);
  for (int j = 0; j < 2; ++j)
    if (qchk_span(BS_REPACK_DST, st_off + ((4 + j) * 128 + r) * 16, 16, out_bytes))
      *reinterpret_cast<uint4*>(st + ((4 + j) * 128 + r) * 16) =
          make_uint4(T[4 * j], T[4 * j + 1], T[4 * j + 2], T[4 * j + 3]);
}

// Stage chunks for whole pairs of 128-row tiles (the CTA-pair kernel reads both tiles of a pair);
// rows past N are zero.
void launch_w6_repack(const uint8_t* src, int layout, int N, int K, uint8_t* out, cudaStream_t s) {
  const int kst = K / 128, nt = (N + 255) / 256 * 2;
  if (kst == 0 || nt == 0) return;
  w6_repack_kernel<<<dim3(kst, nt), 128, 0, s>>>(src, layout, N, K, kst, out, (long long)w6_repacked_bytes(N, K));
}

size_t w6_repacked_bytes(int N, int K) { return (size_t)((N + 255) / 256 * 2) * (K / 128) * 128 * 96; }

template <class Dec, int TM, int STAGES>
static int launch_i8(const CUtensorMap& tx, const CUtensorMap& tw, const GemmI8Params& p, cudaStream_t stream) {
  constexpr int smem = qgemm_i8_smem_bytes<Dec, TM, STAGES>();
  auto kern = qgemm_i8_kernel<Dec, TM, STAGES>;
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
  const int tiles = p.m_tiles * p.n_tiles;
  const int grid = std::min(tiles, sm_count());
  kern<<<grid, I8Cfg<TM, STAGES>::kThreads, smem, stream>>>(tx, tw, p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("qgemm_i8 launch failed: %s", cudaGetErrorString(e));
    return 3;
  }
  return 0;
}

template <class Dec>
static int dispatch_i8(int tm, const CUtensorMap& tx, const CUtensorMap& tw, const GemmI8Params& p,
                       cudaStream_t stream) {
  switch (tm) {
    case 32: return launch_i8<Dec, 32, 8>(tx, tw, p, stream);
    case 64: return launch_i8<Dec, 64, 8>(tx, tw, p, stream);
    case 128: return launch_i8<Dec, 128, 6>(tx, tw, p, stream);
    default: set_error("unsupported token tile %d", tm); return 2;
  }
}

template <class Dec, int TN, int GPS>
static int launch_i8p(const CUtensorMap& tx, const CUtensorMap& tw, const GemmI8Params& p, cudaStream_t stream) {
  constexpr int STAGES = qgemm_i8p_stages<Dec, TN>();
  constexpr int smem = qgemm_i8p_smem_bytes<Dec, TN, STAGES>();
  static_assert(smem <= 232448, "shared memory per CTA");
  auto kern = qgemm_i8p_kernel<Dec, TN, GPS, STAGES>;
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
  const int tiles = p.m_tiles * ((p.N + 255) / 256);
  const int grid = 2 * std::min(tiles, sm_count() / 2);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(I8PCfg<TN, GPS>::kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, tx, tw, p);
  if (e != cudaSuccess) {
    set_error("qgemm_i8p launch failed: %s", cudaGetErrorString(e));
    return 3;
  }
  return 0;
}

// The CTA-pair kernel takes token counts above 64 with groups of 64 or whole multiples of 128
// values (per-channel scales included): 256-token tiles above 128 tokens, else 128.
// Tuning knob: QLIN_I8_PAIR=0 keeps the single-CTA kernel for A/B runs.
static int plan_i8_pair(int M, int group) {
  static const bool enabled = [] {
    const char* e = getenv("QLIN_I8_PAIR");
    return !(e && atoi(e) == 0);
  }();
  if (!enabled || M <= 64) return 0;
  if (group == 64) return 128;
  if (group % 128 != 0) return 0;
  static const int forced = [] {
    const char* e = getenv("QLIN_I8_TN");  // tuning knob: force the pair kernel's token tile
    return e ? atoi(e) : 0;
  }();
  if (forced == 128 || forced == 256) return forced;
  return M > 128 ? 256 : 128;
}

int plan_i8_tm(int M) {
  static const int forced = [] {
    const char* e = getenv("QLIN_TM_I8");
    return e ? atoi(e) : 0;
  }();
  if (forced == 32 || forced == 64 || forced == 128) return forced;
  if (M <= 32) return 32;
  if (M <= 64) return 64;
  return 128;
}

// xq: int8 [M, Kp] (columns permuted per 8), sx: fp32 [M]; w: raw W4 [N, K/2] or W6 planes.
int run_i8_gemm(int bits, const void* xq, long long kp, const float* sx, int M, int N, int K, const void* w, int group,
                const void* scales, int scale_kind, const void* bias, int bias_kind, void* y, int y_dtype,
                long long ldy, cudaStream_t stream) {
  if (M == 0 || N == 0) return 0;
  const int tn = plan_i8_pair(M, group);
  const int tm = tn ? tn : plan_i8_tm(M);
  GemmI8Params p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.num_k_stages = K / 128;
  p.m_tiles = (M + tm - 1) / tm;
  p.n_tiles = (N + 127) / 128;
  p.group = group;
  p.groups_per_row = K / group;
  p.w_stages = reinterpret_cast<const uint8_t*>(w);
  p.scales = scales;
  p.scale_kind = scale_kind;
  p.inv_scale = bits == 4 ? DecW4::kInvScale : DecW6::kInvScale;
  p.x_scale = sx;
  p.bias = bias;
  p.bias_kind = bias_kind;
  p.y = y;
  p.y_dtype = y_dtype;
  p.ldy = ldy;
  p.status = reinterpret_cast<DeviceStatus*>(device_status_ptr());
  p.lim_y = (long long)(M - 1) * ldy + N;
  p.lim_w_bytes = bits == 4 ? (long long)N * K / 2 : (long long)w6_repacked_bytes(N, K);
  p.lim_scales = scale_kind == I8S_GROUP_F16 ? (long long)N * p.groups_per_row : (long long)N;
  CUtensorMap tx, tw;
  // activation box: the token tile (the pair kernel: half of it per CTA)
  int rc = make_tmap_2d(&tx, xq, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)kp, (uint64_t)M, (uint64_t)kp, 128,
                        (uint32_t)(tn ? tn / 2 : tm), CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  if (bits == 4) {
    rc = make_tmap_2d(&tw, w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)K / 2, (uint64_t)N, (uint64_t)K / 2, 64,
                      128, CU_TENSOR_MAP_SWIZZLE_64B);
    if (rc) return rc;
    if (tn == 256) return launch_i8p<DecW4, 256, 1>(tx, tw, p, stream);
    if (tn == 128) return group == 64 ? launch_i8p<DecW4, 128, 2>(tx, tw, p, stream) : launch_i8p<DecW4, 128, 1>(tx, tw, p, stream);
    return dispatch_i8<DecW4>(tm, tx, tw, p, stream);
  }
  tw = tx;
  if (tn == 256) return launch_i8p<DecW6, 256, 1>(tx, tw, p, stream);
  if (tn == 128) return group == 64 ? launch_i8p<DecW6, 128, 2>(tx, tw, p, stream) : launch_i8p<DecW6, 128, 1>(tx, tw, p, stream);
  return dispatch_i8<DecW6>(tm, tx, tw, p, stream);
}

// This translation unit's bounds record (QLIN_CHECKS build).
QLIN_BOUNDS_READER(bounds_read_i8)

}  // namespace qlin
