// Small-M path (one token, weights of up to 4096 x 8192: text tokens, adapter side paths): a
// weight-streaming kernel on the CUDA cores instead of the tensor-core GEMM, whose fixed costs
// (pipeline fill, K split and its finalize pass) dominate when the MMA work is a few microseconds.
//
// A CTA takes 16 output rows and 32 half-warps split the K stages between them; every thread
// decodes its row's 64 values per stage with the same decoders as the GEMM (reading the repacked
// GGUF stage layout, or the row-major int8 weight, straight from global memory: each half-warp load
// is 16 consecutive 16-byte pieces) and accumulates the dot products with the M activation rows
// (staged once per CTA in shared memory as fp32) with packed fp32 FMAs.  The warps' partial sums are reduced in a fixed order in shared memory (the result
// does not depend on scheduling), then the epilogue of the GEMM (column scale, row power of two,
// bias, one rounding) writes the outputs.  No workspace and one launch.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>

#include "qlin_decode.cuh"
#include "qlin_internal.h"

namespace qlin {

namespace {

constexpr int kGemvWarps = 16;

struct GemvParams {
  int M, N, K, num_k_stages;
  const uint8_t* w;          // GGUF: repacked stages [n_tile][k_stage][stage]; INT8: row-major [N, K]
  const int32_t* w_row_exp;
  const void* col_scale;
  int col_scale_kind;
  const __half* x;           // fp16 activations [M, ldx]
  long long ldx;
  const int32_t* x_row_exp;  // or null
  const void* bias;
  int bias_kind;
  void* y;
  int y_dtype;
  long long ldy;
  // Element counts of the caller's buffers for the QLIN_CHECKS build (unused otherwise).
  long long lim_w_bytes, lim_x, lim_y;
};

__device__ __forceinline__ float gemv_colscale(const GemvParams& p, int n) {
  if (!qchk(BS_GEMV_Y, n, p.N)) return 1.f;
  switch (p.col_scale_kind) {
    case CS_F16: return __half2float(reinterpret_cast<const __half*>(p.col_scale)[n]);
    case CS_F32: return reinterpret_cast<const float*>(p.col_scale)[n];
    case CS_EXP2: return exp2i(p.w_row_exp[n]);
    default: return 1.f;
  }
}

// Row r of an int8 [N, K] weight, K values k0 .. k0+63, as 32 packed fp16 pairs (exact).
__device__ __forceinline__ void decode_int8_row(const uint8_t* row, uint32_t (&out)[32]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(row) + j);
    s8x4_to_f16x4(v.x, out[8 * j + 0], out[8 * j + 1]);
    s8x4_to_f16x4(v.y, out[8 * j + 2], out[8 * j + 3]);
    s8x4_to_f16x4(v.z, out[8 * j + 4], out[8 * j + 5]);
    s8x4_to_f16x4(v.w, out[8 * j + 6], out[8 * j + 7]);
  }
}

__device__ __forceinline__ void ffma2(float2& acc, float2 a, float2 b) {
  asm("{\n\t.reg .b64 x, y, z;\n\t"
      "mov.b64 x, {%2, %3};\n\t"
      "mov.b64 y, {%4, %5};\n\t"
      "mov.b64 z, {%0, %1};\n\t"
      "fma.rn.f32x2 z, x, y, z;\n\t"
      "mov.b64 {%0, %1}, z;\n\t}"
      : "+f"(acc.x), "+f"(acc.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
}

// CTA: 16 output rows; lane l handles row l % 16 and the K stages of parity l / 16 among those of
// its warp (warp w: stages w, w + kGemvWarps, ...).  The activations are staged once per CTA in
// shared memory as fp32 [M][K].
template <class Dec, int MT, bool INT8>
__global__ void __launch_bounds__(32 * kGemvWarps) gemv_kernel(const GemvParams p) {
  extern __shared__ float xs[];                 // [MT][K]
  __shared__ float red[2 * kGemvWarps][MT][16];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int half = lane >> 4;
  const int n = blockIdx.x * 16 + (lane & 15);
  const bool n_ok = n < p.N;
  const int nt = n >> 7, r = n & 127;
  float rscale = 1.f;
  if (!INT8 && p.w_row_exp != nullptr && p.col_scale_kind == CS_EXP2 && qchk(BS_GEMV_Y, min(n, p.N - 1), p.N))
    rscale = exp2i(-p.w_row_exp[min(n, p.N - 1)]);
  auto decode = [&](int kst, uint32_t (&w)[32]) {
    if constexpr (INT8) {
      const long long off = (long long)n * p.K + kst * 64;
      if (qchk_span(BS_GEMV_W, off, 64, p.lim_w_bytes)) decode_int8_row(p.w + off, w);
    } else {
      const long long off = ((long long)nt * p.num_k_stages + kst) * Dec::kStageBytes;
      if (qchk_span(BS_GEMV_W, off, Dec::kStageBytes, p.lim_w_bytes)) Dec::decode(p.w + off, r, rscale, w);
    }
  };
  // The first stage's weights are fetched and decoded while the activations are staged.
  const int kst0 = warp + half * kGemvWarps;
  uint32_t w[32];
  if (n_ok && kst0 < p.num_k_stages) decode(kst0, w);
  for (int i = threadIdx.x; i < p.M * (p.K / 2); i += blockDim.x) {
    const int m = i / (p.K / 2), c = i - m * (p.K / 2);
    if (!qchk_span(BS_GEMV_X, (long long)m * p.ldx + 2 * c, 2, p.lim_x) ||
        !qchk_smem(BS_GEMV_X, xs, xs + (size_t)m * p.K + 2 * c, 8))
      continue;
    const float2 v = __half22float2(reinterpret_cast<const __half2*>(p.x + (size_t)m * p.ldx)[c]);
    reinterpret_cast<float2*>(xs + (size_t)m * p.K)[c] = v;
  }
  float2 acc[MT];
#pragma unroll
  for (int m = 0; m < MT; ++m) acc[m] = make_float2(0.f, 0.f);
  __syncthreads();
  if (n_ok) {
    for (int kst = kst0; kst < p.num_k_stages; kst += 2 * kGemvWarps) {
      if (kst != kst0) decode(kst, w);
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float2 wf = __half22float2(*reinterpret_cast<const __half2*>(&w[j]));
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          if (m < p.M) ffma2(acc[m], wf, reinterpret_cast<const float2*>(xs + (size_t)m * p.K + kst * 64)[j]);
        }
      }
    }
  }
#pragma unroll
  for (int m = 0; m < MT; ++m) red[2 * warp + half][m][lane & 15] = __fadd_rn(acc[m].x, acc[m].y);
  __syncthreads();
  if (threadIdx.x < MT * 16) {
    const int m = threadIdx.x >> 4, nn = blockIdx.x * 16 + (threadIdx.x & 15);
    if (m < p.M && nn < p.N) {
      float s = 0.f;
#pragma unroll
      for (int w = 0; w < 2 * kGemvWarps; ++w) s = __fadd_rn(s, red[w][m][threadIdx.x & 15]);
      float o = __fmul_rn(s, gemv_colscale(p, nn));
      if (p.x_row_exp != nullptr && qchk(BS_GEMV_Y, m, p.M)) o = __fmul_rn(o, exp2i(p.x_row_exp[m]));
      float b = 0.f;
      if (p.bias_kind != 0 && !qchk(BS_GEMV_Y, nn, p.N)) b = 0.f;
      else if (p.bias_kind == 1) b = __half2float(reinterpret_cast<const __half*>(p.bias)[nn]);
      else if (p.bias_kind == 2) b = reinterpret_cast<const float*>(p.bias)[nn];
      else if (p.bias_kind == 3) b = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p.bias)[nn]);
      o = __fadd_rn(o, b);
      const long long idx = (long long)m * p.ldy + nn;
      if (qchk(BS_GEMV_Y, idx, p.lim_y)) {
        if (p.y_dtype == OUT_F16) reinterpret_cast<__half*>(p.y)[idx] = __float2half_rn(o);
        else if (p.y_dtype == OUT_BF16) reinterpret_cast<__nv_bfloat16*>(p.y)[idx] = __float2bfloat16_rn(o);
        else reinterpret_cast<float*>(p.y)[idx] = o;
      }
    }
  }
}

constexpr int kGemvMaxXBytes = 48 * 1024;  // fp32 activations staged per CTA

template <class Dec, int MT, bool INT8>
int launch_gemv_mt(const GemvParams& p, cudaStream_t stream) {
  auto kern = gemv_kernel<Dec, MT, INT8>;
  static bool attr_done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_done[dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemvMaxXBytes) != cudaSuccess) {
      set_error("cudaFuncSetAttribute (gemv shared memory) failed");
      return 3;
    }
    attr_done[dev] = true;
  }
  kern<<<(p.N + 15) / 16, 32 * kGemvWarps, (size_t)p.M * p.K * sizeof(float), stream>>>(p);
  return 0;
}

template <class Dec, bool INT8>
int launch_gemv(const GemvParams& p, cudaStream_t stream) {
  const int rc = launch_gemv_mt<Dec, 1, INT8>(p, stream);
  if (rc) return rc;
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("gemv launch failed: %s", cudaGetErrorString(e));
    return 3;
  }
  return 0;
}

}  // namespace

// Returns -1 when the small-M kernel does not apply (the caller then runs the GEMM).
int run_gemv(const F16GemmArgs& a, cudaStream_t stream) {
  static const bool disabled = [] {
    const char* e = getenv("QLIN_NO_GEMV");  // tuning knob: force the tensor-core GEMM for small M
    return e && atoi(e) != 0;
  }();
  // Measured against the tensor-core GEMM on weights cold in L2 (graphs of calls over weight copies,
  // all twelve GGUF types): faster at M = 1 on 3072 x 3072 weights (7.7-8.7 against 10.8-11.6 us),
  // equal or slower at N = 12288 or K = 12288 (more CTAs than one wave, longer rows per thread),
  // and slower at M = 2 for every type but Q3_K / Q5_K (15.7 against 11.2 us for most).
  if (disabled || a.M != 1 || a.N > 4096 || a.K > 8192 || a.out != nullptr || (a.x_slabs > 1) || a.K % 64 != 0 || a.ldx % 8 != 0 ||
      (reinterpret_cast<uintptr_t>(a.x) & 15) || (size_t)a.M * a.K * sizeof(float) > kGemvMaxXBytes)
    return -1;
  if (a.fmt == WF_INT8 && (reinterpret_cast<uintptr_t>(a.w) & 15)) return -1;
  GemvParams p{};
  p.M = a.M;
  p.N = a.N;
  p.K = a.K;
  p.num_k_stages = a.K / 64;
  p.w = reinterpret_cast<const uint8_t*>(a.w);
  p.w_row_exp = a.w_row_exp;
  p.col_scale = a.col_scale;
  p.col_scale_kind = a.col_scale_kind;
  p.x = reinterpret_cast<const __half*>(a.x);
  p.ldx = a.ldx;
  p.x_row_exp = a.x_row_exp;
  p.bias = a.bias;
  p.bias_kind = a.bias_kind;
  p.y = a.y;
  p.y_dtype = a.y_dtype;
  p.ldy = a.ldy;
  p.lim_w_bytes = a.fmt == WF_INT8 ? (long long)a.N * a.K : a.w_bytes;
  p.lim_x = (long long)(a.M - 1) * a.ldx + a.K;
  p.lim_y = (long long)(a.M - 1) * a.ldy + a.N;
  switch (a.fmt) {
    case WF_INT8: return launch_gemv<DecInt8, true>(p, stream);
    case WF_Q8_0: return launch_gemv<DecQ8_0, false>(p, stream);
    case WF_Q4_0: return launch_gemv<DecQ4_0, false>(p, stream);
    case WF_IQ4_NL: return launch_gemv<DecIQ4<false>, false>(p, stream);
    case WF_Q4_K: return launch_gemv<DecQ4_K, false>(p, stream);
    case WF_Q6_K: return launch_gemv<DecQ6_K, false>(p, stream);
    case WF_Q4_1: return launch_gemv<DecQ4_1, false>(p, stream);
    case WF_Q5_0: return launch_gemv<DecQ5Block<false>, false>(p, stream);
    case WF_Q5_1: return launch_gemv<DecQ5Block<true>, false>(p, stream);
    case WF_Q2_K: return launch_gemv<DecQ23_K<false>, false>(p, stream);
    case WF_Q3_K: return launch_gemv<DecQ23_K<true>, false>(p, stream);
    case WF_Q5_K: return launch_gemv<DecQ5_K, false>(p, stream);
    case WF_IQ4_XS: return launch_gemv<DecIQ4<true>, false>(p, stream);
    default: return -1;
  }
}

// This translation unit's bounds record (QLIN_CHECKS build).
QLIN_BOUNDS_READER(bounds_read_gemv)

}  // namespace qlin
