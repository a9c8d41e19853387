// Bandwidth-bound helper kernels around the tensor-core GEMMs:
//   * activation prologues: optional block-Hadamard (ConvRot) rotation, then either
//       - a per-row power-of-two normalization and one rounding to fp16 (kind::f16 operand), or
//       - per-token absmax INT8 quantization with the reference's rounding (kind::i8 operand);
//   * GGUF decode-only (bit-exact with gguf-py 0.19.0), the one-time repack into pipeline
//     stages, and the per-row exponent pass;
//   * the deterministic split-K reduction + epilogue.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <algorithm>
#include <cstdlib>
#include <cstdint>

#include "qlin_decode.cuh"
#include "qlin_hadamard.cuh"
#include "qlin_peer.cuh"
#include "qlin_internal.h"

namespace qlin {

__device__ __forceinline__ float load_x(const void* x, int dtype, long long idx) {
  if (dtype == 1) return __half2float(reinterpret_cast<const __half*>(x)[idx]);
  if (dtype == 2) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(x)[idx]);
  return reinterpret_cast<const float*>(x)[idx];
}

// Loads E consecutive elements of row `row` starting at column c (zeros past K).
template <int E>
__device__ __forceinline__ void load_vals(const void* x, int dtype, long long ldx, int row, int c, int K, float (&v)[E]) {
#pragma unroll
  for (int e = 0; e < E; ++e) v[e] = (c + e < K) ? load_x(x, dtype, (long long)row * ldx + c + e) : 0.f;
}

__device__ __forceinline__ float block_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) red[w] = v;
  __syncthreads();
  if (w == 0) {
    v = (l < (int)(blockDim.x >> 5)) ? red[l] : 0.f;
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (l == 0) red[32] = v;
  }
  __syncthreads();
  const float r = red[32];
  __syncthreads();
  return r;
}

// v * 2^-f, exactly as ldexpf(v, -f): one multiply by the power of two when 2^-f is a normal
// float (every row whose max is a normal number), the library call otherwise.
__device__ __forceinline__ float scale_pow2(float v, int f) {
  return (f >= -127 && f <= 126) ? __fmul_rn(v, exp2i(-f)) : ldexpf(v, -f);
}

// Rounds a float to the input dtype (fp16 / bf16 / fp32) and back.
__device__ __forceinline__ float round_to(float v, int dtype) {
  if (dtype == 1) return __half2float(__float2half_rn(v));
  if (dtype == 2) return __bfloat162float(__float2bfloat16_rn(v));
  return v;
}

// Loads E consecutive elements with one vector load when the row is 16-byte aligned (fp16 / bf16 /
// fp32 inputs), else element by element; zeros past K.
template <int E>
__device__ __forceinline__ void load_vec(const void* x, int dtype, long long ldx, int row, int c, int K, bool vec,
                                         float (&v)[E]) {
  if (vec && c + E <= K) {
    if (dtype == 0) {
      const float* p = reinterpret_cast<const float*>(x) + (long long)row * ldx + c;
      if constexpr (E >= 4) {
#pragma unroll
        for (int e = 0; e < E; e += 4) {
          const float4 f = *reinterpret_cast<const float4*>(p + e);
          v[e] = f.x; v[e + 1] = f.y; v[e + 2] = f.z; v[e + 3] = f.w;
        }
      } else {
#pragma unroll
        for (int e = 0; e < E; ++e) v[e] = p[e];
      }
      return;
    }
    const uint16_t* p = reinterpret_cast<const uint16_t*>(x) + (long long)row * ldx + c;
    uint32_t w[E / 2 > 0 ? E / 2 : 1];
    if constexpr (E == 8) {
      const uint4 q = *reinterpret_cast<const uint4*>(p);
      w[0] = q.x; w[1] = q.y; w[2] = q.z; w[3] = q.w;
    } else if constexpr (E == 4) {
      const uint2 q = *reinterpret_cast<const uint2*>(p);
      w[0] = q.x; w[1] = q.y;
    } else if constexpr (E == 2) {
      w[0] = *reinterpret_cast<const uint32_t*>(p);
    } else {
      w[0] = p[0];
    }
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const unsigned short h = (unsigned short)((w[e >> 1] >> (16 * (e & 1))) & 0xFFFF);
      v[e] = dtype == 1 ? __half2float(__ushort_as_half(h)) : __bfloat162float(__ushort_as_bfloat16(h));
    }
    return;
  }
  load_vals<E>(x, dtype, ldx, row, c, K, v);
}

// Both prologues: walk the row in warp-sized blocks of G = 32*E values (rotated when rotate != 0).
// When `staged`, pass 1 keeps the rotated row in shared memory (fp32) and pass 2 reads it from
// there; otherwise pass 2 reloads and re-rotates.  Pass 2 writes 8 consecutive columns per thread
// (one 16-byte fp16 store or one 8-byte int8 store).
template <int E, int MODE>  // MODE 0: fp16 normalize; MODE 1: int8 per-token quantize
__global__ void __launch_bounds__(256) prologue_kernel(const void* __restrict__ x, int x_dtype, long long ldx, int M,
                                                        int K, int Kp, int rotate_kind, int rotate,
                                                        void* __restrict__ out, int32_t* __restrict__ row_exp,
                                                        float* __restrict__ row_scale, int perm, int staged,
                                                        int vec) {
  extern __shared__ float srow[];
  __shared__ float red[33];
  const int row = blockIdx.x;
  if (!qchk(BS_PRO_X, row, M)) return;  // the whole block: row is uniform
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = blockDim.x >> 5;
  constexpr int G = 32 * E;
  const int nblk = (Kp + G - 1) / G;
  float amax = 0.f;
  for (int b = warp; b < nblk; b += nwarps) {
    float v[E];
    const int c = b * G + lane * E;
    load_vec<E>(x, x_dtype, ldx, row, c, K, vec != 0, v);
    if (rotate) block_hadamard<E>(v, rotate_kind, lane);
#pragma unroll
    for (int e = 0; e < E; ++e) {
      float t = (MODE == 1) ? round_to(v[e], x_dtype) : v[e];
      amax = fmaxf(amax, fabsf(t));
      if (staged && qchk_smem(BS_PRO_OUT, srow, srow + c + e, 4)) srow[c + e] = v[e];
    }
  }
  amax = block_max(amax, red);  // contains __syncthreads, so srow is complete afterwards
  // Pass 2 helpers
  auto value_at = [&](int c, float (&v8)[8]) {
    if (staged) {
#pragma unroll
      for (int e = 0; e < 8; ++e) v8[e] = qchk_smem(BS_PRO_OUT, srow, srow + c + e, 4) ? srow[c + e] : 0.f;
    }
  };
  if (MODE == 0) {
    int f = 0;
    if (amax > 0.f && amax <= 3.402823466e38f) {
      int ex;
      frexpf(amax, &ex);
      f = ex - 15;
    }
    if (threadIdx.x == 0) row_exp[row] = f;
    __half* o = reinterpret_cast<__half*>(out) + (long long)row * Kp;
    if (staged) {
      for (int c = threadIdx.x * 8; c < Kp; c += blockDim.x * 8) {
        float v8[8];
        value_at(c, v8);
        uint4 pk;
        uint32_t* pw = reinterpret_cast<uint32_t*>(&pk);
#pragma unroll
        for (int e = 0; e < 4; ++e) pw[e] = pack_f16x2(scale_pow2(v8[2 * e], f), scale_pow2(v8[2 * e + 1], f));
        if (qchk_span(BS_PRO_OUT, (long long)row * Kp + c, 8, (long long)M * Kp)) *reinterpret_cast<uint4*>(o + c) = pk;
      }
    } else {
      for (int b = warp; b < nblk; b += nwarps) {
        float v[E];
        const int c = b * G + lane * E;
        load_vec<E>(x, x_dtype, ldx, row, c, K, vec != 0, v);
        if (rotate) block_hadamard<E>(v, rotate_kind, lane);
#pragma unroll
        for (int e = 0; e < E; ++e)
          if (c + e < Kp) o[c + e] = __float2half_rn(scale_pow2(v[e], f));
      }
    }
  } else {
    // quantize_int8_rowwise semantics (modal/weight_error_app.py:109-115) in the input dtype.
    float scale = fmaxf(__fdiv_rn(amax, 127.f), 1e-30f);
    float s = round_to(scale, x_dtype);
    if (s == 0.f) s = (x_dtype == 1) ? 6.103515625e-05f : 1.17549435e-38f;
    if (threadIdx.x == 0) row_scale[row] = scale;
    int8_t* o = reinterpret_cast<int8_t*>(out) + (long long)row * Kp;
    auto quant = [&](float v) {
      const float xv = round_to(v, x_dtype);
      const float qv = rintf(round_to(__fdiv_rn(xv, s), x_dtype));
      return (int)fminf(fmaxf(qv, -128.f), 127.f);
    };
    if (staged) {
      for (int c = threadIdx.x * 8; c < Kp; c += blockDim.x * 8) {
        float v8[8];
        value_at(c, v8);
        int q[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) q[e] = (c + e < K) ? quant(v8[e]) : 0;
        // perm: within each group of 8 columns, even columns first (0,2,4,6,1,3,5,7)
        uint32_t lo, hi;
        if (perm) {
          lo = (q[0] & 0xFF) | ((q[2] & 0xFF) << 8) | ((q[4] & 0xFF) << 16) | ((uint32_t)(q[6] & 0xFF) << 24);
          hi = (q[1] & 0xFF) | ((q[3] & 0xFF) << 8) | ((q[5] & 0xFF) << 16) | ((uint32_t)(q[7] & 0xFF) << 24);
        } else {
          lo = (q[0] & 0xFF) | ((q[1] & 0xFF) << 8) | ((q[2] & 0xFF) << 16) | ((uint32_t)(q[3] & 0xFF) << 24);
          hi = (q[4] & 0xFF) | ((q[5] & 0xFF) << 8) | ((q[6] & 0xFF) << 16) | ((uint32_t)(q[7] & 0xFF) << 24);
        }
        if (qchk_span(BS_PRO_OUT, (long long)row * Kp + c, 8, (long long)M * Kp))
          *reinterpret_cast<uint2*>(o + c) = make_uint2(lo, hi);
      }
    } else {
      for (int b = warp; b < nblk; b += nwarps) {
        float v[E];
        const int c = b * G + lane * E;
        load_vec<E>(x, x_dtype, ldx, row, c, K, vec != 0, v);
        if (rotate) block_hadamard<E>(v, rotate_kind, lane);
#pragma unroll
        for (int e = 0; e < E; ++e) {
          const int col = c + e;
          const int dst = perm ? ((col & ~7) | ((col & 1) ? 4 + ((col & 7) >> 1) : ((col & 7) >> 1))) : col;
          if (col < Kp && qchk(BS_PRO_OUT, (long long)row * Kp + dst, (long long)M * Kp))
            o[dst] = (col < K) ? static_cast<int8_t>(quant(v[e])) : 0;
        }
      }
    }
  }
}

// Register-resident variant: each warp keeps its BPW blocks (E values per lane each) in registers
// between the row-max pass and the write pass, so the row is read from HBM once.  Used when
// ceil(Kp / G) <= 8 * BPW.  Stores are E-wide vectors (fp16) or, for int8, 8-column groups.
template <int E, int MODE, int BPW>
__global__ void __launch_bounds__(512) prologue_reg_kernel(const void* __restrict__ x, int x_dtype, long long ldx,
                                                            int M, int K, int Kp, int rotate_kind, int rotate,
                                                            void* __restrict__ out, int32_t* __restrict__ row_exp,
                                                            float* __restrict__ row_scale, int perm, int vec) {
  __shared__ float red[33];
  const int row = blockIdx.x;
  if (!qchk(BS_PRO_X, row, M)) return;  // the whole block: row is uniform
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nw = blockDim.x >> 5;
  constexpr int G = 32 * E;
  const int nblk = (Kp + G - 1) / G;
  float v[BPW][E];
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < BPW; ++i) {
    const int b = warp + nw * i;
    if (b < nblk) {
      const int c = b * G + lane * E;
      load_vec<E>(x, x_dtype, ldx, row, c, K, vec != 0, v[i]);
      if (rotate) block_hadamard<E>(v[i], rotate_kind, lane);
#pragma unroll
      for (int e = 0; e < E; ++e) {
        if (MODE == 1) v[i][e] = round_to(v[i][e], x_dtype);
        amax = fmaxf(amax, fabsf(v[i][e]));
      }
    }
  }
  amax = block_max(amax, red);
  if (MODE == 0) {
    int f = 0;
    if (amax > 0.f && amax <= 3.402823466e38f) {
      int ex;
      frexpf(amax, &ex);
      f = ex - 15;
    }
    if (threadIdx.x == 0) row_exp[row] = f;
    __half* o = reinterpret_cast<__half*>(out) + (long long)row * Kp;
#pragma unroll
    for (int i = 0; i < BPW; ++i) {
      const int b = warp + nw * i;
      if (b < nblk) {
        const int c = b * G + lane * E;
        if (c + E <= Kp && qchk_span(BS_PRO_OUT, (long long)row * Kp + c, E, (long long)M * Kp)) {
          uint32_t w[(E + 1) / 2];
#pragma unroll
          for (int e = 0; e < E; e += 2)
            w[e / 2] = pack_f16x2(scale_pow2(v[i][e], f), E > 1 ? scale_pow2(v[i][e + 1 < E ? e + 1 : e], f) : 0.f);
          if constexpr (E == 8) *reinterpret_cast<uint4*>(o + c) = make_uint4(w[0], w[1], w[2], w[3]);
          else if constexpr (E == 4) *reinterpret_cast<uint2*>(o + c) = make_uint2(w[0], w[1]);
          else if constexpr (E == 2) *reinterpret_cast<uint32_t*>(o + c) = w[0];
          else o[c] = __float2half_rn(scale_pow2(v[i][0], f));
        }
      }
    }
  } else {
    float scale = fmaxf(__fdiv_rn(amax, 127.f), 1e-30f);
    float s = round_to(scale, x_dtype);
    if (s == 0.f) s = (x_dtype == 1) ? 6.103515625e-05f : 1.17549435e-38f;
    if (threadIdx.x == 0) row_scale[row] = scale;
    int8_t* o = reinterpret_cast<int8_t*>(out) + (long long)row * Kp;
#pragma unroll
    for (int i = 0; i < BPW; ++i) {
      const int b = warp + nw * i;
      if (b < nblk) {
        const int c = b * G + lane * E;
        int q[E];
#pragma unroll
        for (int e = 0; e < E; ++e) {
          const float qv = rintf(round_to(__fdiv_rn(v[i][e], s), x_dtype));
          q[e] = (c + e < K) ? (int)fminf(fmaxf(qv, -128.f), 127.f) : 0;
        }
        if constexpr (E == 8) {
          uint32_t lo, hi;
          if (perm) {  // even columns first within the group of 8
            lo = (q[0] & 0xFF) | ((q[2] & 0xFF) << 8) | ((q[4] & 0xFF) << 16) | ((uint32_t)(q[6] & 0xFF) << 24);
            hi = (q[1] & 0xFF) | ((q[3] & 0xFF) << 8) | ((q[5] & 0xFF) << 16) | ((uint32_t)(q[7] & 0xFF) << 24);
          } else {
            lo = (q[0] & 0xFF) | ((q[1] & 0xFF) << 8) | ((q[2] & 0xFF) << 16) | ((uint32_t)(q[3] & 0xFF) << 24);
            hi = (q[4] & 0xFF) | ((q[5] & 0xFF) << 8) | ((q[6] & 0xFF) << 16) | ((uint32_t)(q[7] & 0xFF) << 24);
          }
          if (c + 8 <= Kp && qchk_span(BS_PRO_OUT, (long long)row * Kp + c, 8, (long long)M * Kp))
            *reinterpret_cast<uint2*>(o + c) = make_uint2(lo, hi);
        } else {
#pragma unroll
          for (int e = 0; e < E; ++e) {
            const int col = c + e;
            const int dst = perm ? ((col & ~7) | ((col & 1) ? 4 + ((col & 7) >> 1) : ((col & 7) >> 1))) : col;
            if (col < Kp && qchk(BS_PRO_OUT, (long long)row * Kp + dst, (long long)M * Kp))
              o[dst] = static_cast<int8_t>(q[e]);
          }
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------------------------
// Per-token int8 codes of fp16 / bf16 rows without rotation (the A8 activations of the W4A8 /
// W6A8 linears and quantize_int8_rowwise).  The codes are those of prologue_reg_kernel<E, 1, ..>,
// with about a quarter of its instructions per value and half its registers, so that several rows
// are in flight per SM and the pass streams at HBM rate:
//  * each thread keeps its NV 16-byte vectors (8 values each) of the row in registers as loaded;
//  * the row maximum is taken on packed pairs (max.f16x2 / max.bf16x2 return the non-NaN operand,
//    as fmaxf does);
//  * x / s, the correctly rounded fp32 quotient, comes from Markstein's correction (P. Markstein,
//    IBM J. Res. Dev. 34(1), 1990): y = RN(1/s) once per row, then q0 = RN(x*y), r = x - s*q0 (one
//    fma, exact) and q = RN(q0 + r*y), two values per packed fp32 instruction.  Over every fp16 /
//    bf16 pair that a row can hold (|x| <= 256 s, s >= RN(1e-30)) this equals RN(x/s) wherever
//    |x/s| >= 1/16 and gives the same code everywhere (tests/quotient_check.c checks every pair);
//    a row with s > 1e37 (an infinite maximum) divides;
//  * the quotient is rounded to the input dtype two at a time, clamped to [-128, 127] there and
//    rounded half-to-even to an integer by adding 1.5 * 2^10 in fp16 (spacing 1 on [1024, 2048))
//    or 1.5 * 2^23 in fp32 (bf16 rows): the low byte of the sum's bits is the two's-complement code.
// ---------------------------------------------------------------------------------------------
template <bool BF16>
__device__ __forceinline__ uint32_t max2_bits(uint32_t a, uint32_t b) {
  uint32_t d;
  if constexpr (BF16) asm("max.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  else asm("max.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

template <bool BF16>
__device__ __forceinline__ float bits_lo_f32(uint32_t w) {
  if constexpr (BF16) return __uint_as_float(w << 16);
  else return __half2float(__ushort_as_half((unsigned short)(w & 0xFFFFu)));
}

template <bool BF16>
__device__ __forceinline__ float bits_hi_f32(uint32_t w) {
  if constexpr (BF16) return __uint_as_float(w & 0xFFFF0000u);
  else return __half2float(__ushort_as_half((unsigned short)(w >> 16)));
}

// (a, b) <- (RN(a/s), RN(b/s)) by Markstein's correction; y = RN(1/s), ns = -s.
__device__ __forceinline__ void div2_markstein(float& a, float& b, float y, float ns) {
  asm("{\n\t.reg .b64 x, q, r, yy, nn;\n\t"
      "mov.b64 x, {%0, %1};\n\t"
      "mov.b64 yy, {%2, %2};\n\t"
      "mov.b64 nn, {%3, %3};\n\t"
      "mul.rn.f32x2 q, x, yy;\n\t"
      "fma.rn.f32x2 r, q, nn, x;\n\t"
      "fma.rn.f32x2 q, r, yy, q;\n\t"
      "mov.b64 {%0, %1}, q;\n\t}"
      : "+f"(a), "+f"(b)
      : "f"(y), "f"(ns));
}

// Codes of two quotients: byte 0 holds a's, byte 2 b's.
template <bool BF16>
__device__ __forceinline__ uint32_t codes2(float a, float b) {
  uint32_t h, d;
  if constexpr (BF16) {
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(h) : "f"(b), "f"(a));
    asm("max.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(h), "r"(0xC300C300u));  // -128
    asm("min.bf16x2 %0, %0, %1;" : "+r"(d) : "r"(0x42FE42FEu));          // 127
    const uint32_t ca = __float_as_uint(__fadd_rn(__uint_as_float(d << 16), 12582912.f));
    const uint32_t cb = __float_as_uint(__fadd_rn(__uint_as_float(d & 0xFFFF0000u), 12582912.f));
    return __byte_perm(ca, cb, 0x0400);
  } else {
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(h) : "f"(b), "f"(a));
    asm("max.f16x2 %0, %1, %2;" : "=r"(d) : "r"(h), "r"(0xD800D800u));  // -128
    asm("min.f16x2 %0, %0, %1;" : "+r"(d) : "r"(0x57F057F0u));          // 127
    asm("add.rn.f16x2 %0, %0, %1;" : "+r"(d) : "r"(0x66006600u));       // + 1536
    return d;
  }
}

template <int NV, bool BF16>
__global__ void __launch_bounds__(512) quant_rows16_kernel(const uint16_t* __restrict__ x, long long ldx, int M,
                                                           int K, int Kp, int8_t* __restrict__ out,
                                                           float* __restrict__ row_scale, int perm) {
  __shared__ float red[33];
  const int row = blockIdx.x;
  if (!qchk(BS_PRO_X, row, M)) return;  // the whole block: row is uniform
  const int nvec = K >> 3, nvp = Kp >> 3;
  const uint16_t* xr = x + (long long)row * ldx;
  uint4 v[NV];
  uint32_t mx = 0u;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int j = threadIdx.x + i * blockDim.x;
    v[i] = (j < nvec) ? __ldcs(reinterpret_cast<const uint4*>(xr) + j) : make_uint4(0u, 0u, 0u, 0u);
    mx = max2_bits<BF16>(mx, v[i].x & 0x7FFF7FFFu);
    mx = max2_bits<BF16>(mx, v[i].y & 0x7FFF7FFFu);
    mx = max2_bits<BF16>(mx, v[i].z & 0x7FFF7FFFu);
    mx = max2_bits<BF16>(mx, v[i].w & 0x7FFF7FFFu);
  }
  const float amax = block_max(fmaxf(bits_lo_f32<BF16>(mx), bits_hi_f32<BF16>(mx)), red);
  const float scale = fmaxf(__fdiv_rn(amax, 127.f), 1e-30f);
  float s = BF16 ? __bfloat162float(__float2bfloat16_rn(scale)) : __half2float(__float2half_rn(scale));
  if (s == 0.f) s = BF16 ? 1.17549435e-38f : 6.103515625e-05f;
  if (threadIdx.x == 0) row_scale[row] = scale;
  const bool fast = s <= 1e37f;
  const float y = __frcp_rn(s), ns = -s;
  int8_t* o = out + (long long)row * Kp;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int j = threadIdx.x + i * blockDim.x;
    if (j < nvp) {
      const uint32_t in[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
      uint32_t w[4];
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        float a = bits_lo_f32<BF16>(in[p]), b = bits_hi_f32<BF16>(in[p]);
        if (fast) {
          div2_markstein(a, b, y, ns);
        } else {
          a = __fdiv_rn(a, s);
          b = __fdiv_rn(b, s);
        }
        w[p] = codes2<BF16>(a, b);
      }
      uint32_t lo, hi;
      if (perm) {  // even columns first within the group of 8
        const uint32_t e = __byte_perm(w[0], w[1], 0x6240), f = __byte_perm(w[2], w[3], 0x6240);
        lo = __byte_perm(e, f, 0x5410);
        hi = __byte_perm(e, f, 0x7632);
      } else {
        lo = __byte_perm(w[0], w[1], 0x6420);
        hi = __byte_perm(w[2], w[3], 0x6420);
      }
      if (qchk_span(BS_PRO_OUT, (long long)row * Kp + 8 * j, 8, (long long)M * Kp))
        *reinterpret_cast<uint2*>(o + 8 * j) = make_uint2(lo, hi);
    }
  }
}

// ---------------------------------------------------------------------------------------------
// GGUF decode-only: one thread per 4 consecutive values of the flat tensor (blocks are indexed
// by flat element, so rows may straddle blocks).  fp32 results are bit-exact with gguf-py.
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ float f16_at(const uint8_t* p) {
  return __half2float(__ushort_as_half((unsigned short)(p[0] | (p[1] << 8))));
}

__host__ __device__ constexpr int gguf_qk(int qtype) {
  return (qtype == GGUF_Q2_K || qtype == GGUF_Q3_K || qtype == GGUF_Q4_K || qtype == GGUF_Q5_K ||
          qtype == GGUF_Q6_K || qtype == GGUF_IQ4_XS) ? 256 : 32;
}

__host__ __device__ constexpr int gguf_ts(int qtype) {
  return qtype == GGUF_Q4_0 || qtype == GGUF_IQ4_NL ? 18 : qtype == GGUF_Q4_1 ? 20 : qtype == GGUF_Q5_0 ? 22
       : qtype == GGUF_Q5_1 ? 24 : qtype == GGUF_Q8_0 ? 34 : qtype == GGUF_Q2_K ? 84 : qtype == GGUF_Q3_K ? 110
       : qtype == GGUF_Q4_K ? 144 : qtype == GGUF_Q5_K ? 176 : qtype == GGUF_Q6_K ? 210 : 136;
}

__device__ __forceinline__ uint32_t u32_at(const uint8_t* p) {  // little-endian, any alignment
  return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

// 6-bit (scale, min) of sub-block `sub` from the 12 packed bytes of a Q4_K / Q5_K superblock
// (`gguf/quants.py:478-500`).
__device__ __forceinline__ void k4_scale_min(const uint8_t* sc, int sub, int& s, int& m) {
  if (sub < 4) {
    s = sc[sub] & 0x3F;
    m = sc[sub + 4] & 0x3F;
  } else {
    s = (sc[sub + 4] & 0x0F) | ((sc[sub - 4] >> 2) & 0x30);
    m = (sc[sub + 4] >> 4) | ((sc[sub] >> 2) & 0x30);
  }
}

// Signed 6-bit scale of 16-value group i of a Q3_K superblock (`gguf/quants.py:456-463`).
__device__ __forceinline__ int q3k_scale(const uint8_t* sc, int i) {
  const int lo = i < 8 ? (sc[i] & 0xF) : (sc[i - 8] >> 4);
  const int hi = (sc[8 + (i & 3)] >> (2 * (i >> 2))) & 3;
  return (lo | (hi << 4)) - 32;
}

// Signed 6-bit scale of sub-block i of an IQ4_XS superblock (`gguf/quants.py:1363-1369`).
__device__ __forceinline__ int iq4xs_scale(const uint8_t* b, int i) {
  const int lo = (b[4 + (i >> 1)] >> (4 * (i & 1))) & 0xF;
  const int hi = ((b[2] | (b[3] << 8)) >> (2 * i)) & 3;
  return (lo | (hi << 4)) - 32;
}

// 2-bit code of value j (0..255) of a Q2_K / Q3_K code array (`gguf/quants.py:422-424`).
__device__ __forceinline__ int crumb_at(const uint8_t* qs, int j) {
  return (qs[32 * (j >> 7) + (j & 31)] >> (2 * ((j & 127) >> 5))) & 3;
}

__device__ float gguf_value(const uint8_t* __restrict__ raw, int qtype, long long idx) {
  switch (qtype) {
    case GGUF_Q4_1:
    case GGUF_Q5_0:
    case GGUF_Q5_1: {
      const int ts = gguf_ts(qtype);
      const uint8_t* b = raw + (idx / 32) * ts;
      const int j = (int)(idx % 32);
      const int qs = ts - 16;
      const uint8_t byte = b[qs + (j & 15)];
      int q = (j < 16) ? (byte & 0xF) : (byte >> 4);
      if (qtype != GGUF_Q4_1) q |= (int)((u32_at(b + qs - 4) >> j) & 1) << 4;
      const float d = f16_at(b);
      if (qtype == GGUF_Q5_0) return __fmul_rn(d, (float)(q - 16));
      return __fadd_rn(__fmul_rn(d, (float)q), f16_at(b + 2));
    }
    case GGUF_Q2_K: {
      const uint8_t* b = raw + (idx / 256) * 84;
      const int j = (int)(idx % 256);
      const int sc = b[j / 16];
      const float dl = __fmul_rn(f16_at(b + 80), (float)(sc & 0xF));
      const float ml = __fmul_rn(f16_at(b + 82), (float)(sc >> 4));
      return __fsub_rn(__fmul_rn(dl, (float)crumb_at(b + 16, j)), ml);
    }
    case GGUF_Q3_K: {
      const uint8_t* b = raw + (idx / 256) * 110;
      const int j = (int)(idx % 256);
      const int q = crumb_at(b + 32, j) - (((b[j & 31] >> (j >> 5)) & 1) ? 0 : 4);
      const float dl = __fmul_rn(f16_at(b + 108), (float)q3k_scale(b + 96, j / 16));
      return __fmul_rn(dl, (float)q);
    }
    case GGUF_Q5_K: {
      const uint8_t* b = raw + (idx / 256) * 176;
      const int j = (int)(idx % 256);
      const int sub = j / 32, l = j % 32;
      int s, m;
      k4_scale_min(b + 4, sub, s, m);
      const int q = ((b[48 + 32 * (sub / 2) + l] >> (4 * (sub & 1))) & 0xF) | (((b[16 + l] >> sub) & 1) << 4);
      const float ds = __fmul_rn(f16_at(b), (float)s);
      const float dm = __fmul_rn(f16_at(b + 2), (float)m);
      return __fsub_rn(__fmul_rn(ds, (float)q), dm);
    }
    case GGUF_IQ4_XS: {
      const uint8_t* b = raw + (idx / 256) * 136;
      const int j = (int)(idx % 256);
      const int sub = j / 32, l = j % 32;
      const uint8_t byte = b[8 + 16 * sub + (l & 15)];
      const int nib = (l < 16) ? (byte & 0xF) : (byte >> 4);
      constexpr int8_t kv[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};
      const float dl = __fmul_rn(f16_at(b), (float)iq4xs_scale(b, sub));
      return __fmul_rn(dl, (float)kv[nib]);
    }
    case GGUF_Q4_0:
    case GGUF_IQ4_NL: {
      const uint8_t* b = raw + (idx / 32) * 18;
      const int j = (int)(idx % 32);
      const uint8_t byte = b[2 + (j & 15)];
      const int nib = (j < 16) ? (byte & 0xF) : (byte >> 4);
      const float d = f16_at(b);
      if (qtype == GGUF_Q4_0) return __fmul_rn(d, (float)(nib - 8));
      constexpr int8_t kv[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};
      return __fmul_rn(d, (float)kv[nib]);
    }
    case GGUF_Q8_0: {
      const uint8_t* b = raw + (idx / 32) * 34;
      return __fmul_rn((float)(int8_t)b[2 + idx % 32], f16_at(b));
    }
    case GGUF_Q4_K: {
      const uint8_t* b = raw + (idx / 256) * 144;
      const int j = (int)(idx % 256);
      const int sub = j / 32;
      int s, m;
      k4_scale_min(b + 4, sub, s, m);
      const uint8_t byte = b[16 + (sub / 2) * 32 + (j % 32)];
      const int q = (sub & 1) ? (byte >> 4) : (byte & 0xF);
      const float ds = __fmul_rn(f16_at(b), (float)s);
      const float dm = __fmul_rn(f16_at(b + 2), (float)m);
      return __fsub_rn(__fmul_rn(ds, (float)q), dm);
    }
    case GGUF_Q6_K: {
      const uint8_t* b = raw + (idx / 256) * 210;
      const int j = (int)(idx % 256);
      const int h = j / 128, r = j % 128;
      const int lo = (b[64 * h + (r % 64)] >> (4 * (r / 64))) & 0xF;
      const int hi = (b[128 + 32 * h + (r % 32)] >> (2 * (r / 32))) & 0x3;
      const int q = (lo | (hi << 4)) - 32;
      const float ds = __fmul_rn(f16_at(b + 208), (float)(int8_t)b[192 + j / 16]);
      return __fmul_rn(ds, (float)q);
    }
  }
  return 0.f;
}

__global__ void gguf_dequant_kernel(const uint8_t* __restrict__ raw, int qtype, long long total, void* __restrict__ out,
                                    int out_dtype) {
  const long long i0 = ((long long)blockIdx.x * blockDim.x + threadIdx.x) * 4;
  for (int t = 0; t < 4; ++t) {
    const long long i = i0 + t;
    if (i >= total) return;
    const int qk = gguf_qk(qtype), ts = gguf_ts(qtype);
    if (!qchk_span(BS_REPACK_SRC, (i / qk) * ts, ts, (total + qk - 1) / qk * ts)) return;
    const float v = gguf_value(raw, qtype, i);
    if (out_dtype == 0) reinterpret_cast<float*>(out)[i] = v;
    else if (out_dtype == 1) reinterpret_cast<__half*>(out)[i] = __float2half_rn(v);
    else reinterpret_cast<__nv_bfloat16*>(out)[i] = __float2bfloat16_rn(v);
  }
}

// Upper bound on |w| over one block, from its scales only (float64, as the oracle computes it).
__device__ double gguf_block_bound(const uint8_t* b, int qtype) {
  switch (qtype) {
    case GGUF_Q4_0: return fabs((double)f16_at(b)) * 8.0;
    case GGUF_Q4_1: return fabs((double)f16_at(b)) * 15.0 + fabs((double)f16_at(b + 2));
    case GGUF_Q5_0: return fabs((double)f16_at(b)) * 16.0;
    case GGUF_Q5_1: return fabs((double)f16_at(b)) * 31.0 + fabs((double)f16_at(b + 2));
    case GGUF_Q8_0: return fabs((double)f16_at(b)) * 128.0;
    case GGUF_IQ4_NL: return fabs((double)f16_at(b)) * 127.0;
    case GGUF_Q2_K: {
      const double d = fabs((double)f16_at(b + 80)), dmin = fabs((double)f16_at(b + 82));
      double v = 0.0;
      for (int t = 0; t < 16; ++t) v = fmax(v, d * (b[t] & 0xF) * 3.0 + dmin * (b[t] >> 4));
      return v;
    }
    case GGUF_Q3_K: {
      const double d = fabs((double)f16_at(b + 108));
      double v = 0.0;
      for (int t = 0; t < 16; ++t) v = fmax(v, d * abs(q3k_scale(b + 96, t)) * 4.0);
      return v;
    }
    case GGUF_Q4_K:
    case GGUF_Q5_K: {
      const double d = fabs((double)f16_at(b)), dmin = fabs((double)f16_at(b + 2));
      const double qmax = qtype == GGUF_Q4_K ? 15.0 : 31.0;
      double v = 0.0;
      for (int sub = 0; sub < 8; ++sub) {
        int s, m;
        k4_scale_min(b + 4, sub, s, m);
        v = fmax(v, d * s * qmax + dmin * m);
      }
      return v;
    }
    case GGUF_Q6_K: {
      const double d = fabs((double)f16_at(b + 208));
      double v = 0.0;
      for (int t = 0; t < 16; ++t) v = fmax(v, d * fabs((double)(int8_t)b[192 + t]) * 32.0);
      return v;
    }
    case GGUF_IQ4_XS: {
      const double d = fabs((double)f16_at(b));
      double v = 0.0;
      for (int sub = 0; sub < 8; ++sub) v = fmax(v, d * abs(iq4xs_scale(b, sub)) * 127.0);
      return v;
    }
  }
  return 0.0;
}

// Per-row exponent: e = frexp(bound).exp - 15 with bound an upper bound on |w| over the row's
// blocks read from block scales only (float64, as the oracle computes it).
__global__ void gguf_row_exp_kernel(const uint8_t* __restrict__ raw, int qtype, int N, int K, int n_pad,
                                    int32_t* __restrict__ row_exp) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= n_pad) return;
  double bound = 0.0;
  if (row < N) {
    const int qk = gguf_qk(qtype), ts = gguf_ts(qtype);
    const int nb = K / qk;
    const uint8_t* r = raw + (long long)row * nb * ts;
    for (int blk = lane; blk < nb; blk += 32)
      if (qchk_span(BS_REPACK_SRC, ((long long)row * nb + blk) * ts, ts, (long long)N * nb * ts))
        bound = fmax(bound, gguf_block_bound(r + (long long)blk * ts, qtype));
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) bound = fmax(bound, __shfl_xor_sync(0xffffffffu, bound, o));
  if (lane == 0 && qchk(BS_REPACK_DST, row, n_pad)) {
    int e = 0;
    if (bound > 0.0 && bound < 1e300) {
      int ex;
      frexp(bound, &ex);
      e = ex - 15;
    }
    row_exp[row] = e;
  }
}

// H word of a stage layout from 32 per-value bits (bit v = the extra bit of value v): bit 8b + g
// of H is the bit of value 4g + b.
__device__ __forceinline__ uint32_t h_transpose(uint32_t bits) {
  uint32_t h = 0;
#pragma unroll
  for (int v = 0; v < 32; ++v) h |= ((bits >> v) & 1u) << (8 * (v & 3) + (v >> 2));
  return h;
}

__device__ __forceinline__ void put_u32(uint8_t* p, uint32_t v) {
  for (int i = 0; i < 4; ++i) p[i] = (uint8_t)(v >> (8 * i));
}

// A run of 32 IQ4 codes (ggml order: byte i holds value i in its low nibble, value i+16 in its
// high nibble) -> 4 words in selector order: word t = codes of values 4t..4t+3 in bits 0-15 and
// 16+4t..16+4t+3 in bits 16-31, value 4t+k in nibble k, each code with its bits 2 and 3 swapped
// (the two-permute level lookup of the decoder relies on it).
__device__ __forceinline__ uint32_t iq4_swap23(uint32_t c) { return (c & 3u) | ((c & 4u) << 1) | ((c & 8u) >> 1); }

__device__ __forceinline__ void iq4_selector_order(const uint8_t* qs, uint8_t* out) {
  for (int t = 0; t < 4; ++t) {
    uint32_t w = 0;
    for (int k = 0; k < 4; ++k)
      w |= (iq4_swap23(qs[4 * t + k] & 0xFu) << (4 * k)) | (iq4_swap23((uint32_t)qs[4 * t + k] >> 4) << (16 + 4 * k));
    put_u32(out + 4 * t, w);
  }
}

// One-time repack of raw GGUF rows into the pipeline-stage layout documented in qlin_decode.cuh.
// grid = (num_k_stages, n_tiles), block = 128 (one thread per weight row of the tile).
__global__ void gguf_repack_kernel(const uint8_t* __restrict__ raw, int qtype, int N, int K, int num_k_stages,
                                   uint8_t* __restrict__ out, uint32_t stage_bytes, int P, int S, long long out_bytes) {
  const int kst = blockIdx.x, nt = blockIdx.y, r = threadIdx.x;
  const int n = nt * 128 + r;
  uint8_t* st = out + ((size_t)nt * num_k_stages + kst) * stage_bytes;
  uint8_t payload[64];
  uint8_t side[16];
#pragma unroll
  for (int i = 0; i < 64; ++i) payload[i] = 0;
#pragma unroll
  for (int i = 0; i < 16; ++i) side[i] = 0;
  const int k0 = kst * 64;
  if (n < N && k0 < K) {
    const int ts = gguf_ts(qtype);
    if (gguf_qk(qtype) == 32) {
      const uint8_t* row = raw + (long long)n * (K / 32) * ts;
      for (int blk = 0; blk < 2; ++blk) {
        const int kb = k0 / 32 + blk;
        if (kb * 32 >= K) break;
        const uint8_t* b = row + (long long)kb * ts;
        if (!qchk_span(BS_REPACK_SRC, ((long long)n * (K / 32) + kb) * ts, ts, (long long)N * (K / 32) * ts)) break;
        switch (qtype) {
          case GGUF_Q8_0:
          case GGUF_Q4_0: {
            const int qsb = ts - 2;
            side[2 * blk] = b[0];
            side[2 * blk + 1] = b[1];
            for (int i = 0; i < qsb; ++i) payload[blk * qsb + i] = b[2 + i];
            break;
          }
          case GGUF_IQ4_NL:
            side[2 * blk] = b[0];
            side[2 * blk + 1] = b[1];
            iq4_selector_order(b + 2, payload + 16 * blk);
            break;
          case GGUF_Q4_1:
            for (int i = 0; i < 4; ++i) side[4 * blk + i] = b[i];  // d, m
            for (int i = 0; i < 16; ++i) payload[16 * blk + i] = b[4 + i];
            break;
          case GGUF_Q5_0:
            side[2 * blk] = b[0];
            side[2 * blk + 1] = b[1];
            put_u32(side + 4 + 4 * blk, h_transpose(u32_at(b + 2)));
            for (int i = 0; i < 16; ++i) payload[16 * blk + i] = b[6 + i];
            break;
          case GGUF_Q5_1:
            for (int i = 0; i < 4; ++i) side[4 * blk + i] = b[i];  // d, m
            put_u32(side + 8 + 4 * blk, h_transpose(u32_at(b + 4)));
            for (int i = 0; i < 16; ++i) payload[16 * blk + i] = b[8 + i];
            break;
        }
      }
    } else {
      const uint8_t* b = raw + ((long long)n * (K / 256) + k0 / 256) * ts;
      const int c = (k0 % 256) / 64;  // the stage holds superblock values 64c .. 64c+63
      const bool b_in =
          qchk_span(BS_REPACK_SRC, ((long long)n * (K / 256) + k0 / 256) * ts, ts, (long long)N * (K / 256) * ts);
      switch (b_in ? qtype : -1) {
        case GGUF_Q2_K:
        case GGUF_Q3_K: {
          const uint8_t* qs = b + (qtype == GGUF_Q2_K ? 16 : 32);
          for (int i = 0; i < 64; ++i)  // word i/16, byte i%4, bits 2*((i%16)/4)
            payload[4 * (i >> 4) + (i & 3)] |= (uint8_t)(crumb_at(qs, 64 * c + i) << (2 * ((i & 15) >> 2)));
          if (qtype == GGUF_Q2_K) {
            for (int i = 0; i < 4; ++i) side[i] = b[80 + i];  // d, dmin
            for (int t = 0; t < 4; ++t) side[4 + t] = b[4 * c + t];
          } else {
            side[0] = b[108];
            side[1] = b[109];
            for (int t = 0; t < 4; ++t) side[2 + t] = (uint8_t)(int8_t)q3k_scale(b + 96, 4 * c + t);
            for (int w = 0; w < 2; ++w) {
              uint32_t bits = 0;
              for (int l = 0; l < 32; ++l) bits |= (uint32_t)((b[l] >> (2 * c + w)) & 1) << l;
              put_u32(side + 8 + 4 * w, h_transpose(bits));
            }
          }
          break;
        }
        case GGUF_Q4_K:
        case GGUF_Q5_K: {
          const int qs = qtype == GGUF_Q4_K ? 16 : 48;
          for (int i = 0; i < 32; ++i) payload[i] = b[qs + c * 32 + i];
          int s0, m0, s1, m1;
          k4_scale_min(b + 4, 2 * c, s0, m0);
          k4_scale_min(b + 4, 2 * c + 1, s1, m1);
          for (int i = 0; i < 4; ++i) side[i] = b[i];  // d, dmin
          side[4] = (uint8_t)s0;
          side[5] = (uint8_t)s1;
          side[6] = (uint8_t)m0;
          side[7] = (uint8_t)m1;
          if (qtype == GGUF_Q5_K) {
            for (int w = 0; w < 2; ++w) {  // sub-block 2c + w: bit (2c + w) of qh[l]
              uint32_t bits = 0;
              for (int l = 0; l < 32; ++l) bits |= (uint32_t)((b[16 + l] >> (2 * c + w)) & 1) << l;
              put_u32(side + 8 + 4 * w, h_transpose(bits));
            }
          }
          break;
        }
        case GGUF_Q6_K: {
          const int base = 64 * c;
          uint8_t v[64];
          for (int i = 0; i < 64; ++i) {
            const int j = base + i;
            const int h = j / 128, rr = j % 128;
            const int lo = (b[64 * h + (rr % 64)] >> (4 * (rr / 64))) & 0xF;
            const int hi = (b[128 + 32 * h + (rr % 32)] >> (2 * (rr / 32))) & 0x3;
            v[i] = (uint8_t)(lo | (hi << 4));
          }
          for (int i = 0; i < 64; ++i) payload[i] = v[i];  // one byte per code
          for (int t = 0; t < 4; ++t) side[t] = b[192 + base / 16 + t];
          side[4] = b[208];
          side[5] = b[209];
          break;
        }
        case GGUF_IQ4_XS:
          iq4_selector_order(b + 8 + 32 * c, payload);  // sub-blocks 2c, 2c+1
          iq4_selector_order(b + 8 + 32 * c + 16, payload + 16);
          side[0] = b[0];
          side[1] = b[1];
          side[2] = (uint8_t)(int8_t)iq4xs_scale(b, 2 * c);
          side[3] = (uint8_t)(int8_t)iq4xs_scale(b, 2 * c + 1);
          break;
      }
    }
  }
  const long long st_off = ((long long)nt * num_k_stages + kst) * stage_bytes;
  for (int j = 0; j < P; ++j)
    for (int i = 0; i < 16; ++i)
      if (qchk(BS_REPACK_DST, (j * 128 + r) * 16 + i, stage_bytes) &&
          qchk(BS_REPACK_DST, st_off + (j * 128 + r) * 16 + i, out_bytes))
        st[(j * 128 + r) * 16 + i] = payload[j * 16 + i];
  for (int i = 0; i < S; ++i)
    if (qchk(BS_REPACK_DST, 128 * 16 * P + r * S + i, stage_bytes) &&
        qchk(BS_REPACK_DST, st_off + 128 * 16 * P + r * S + i, out_bytes))
      st[128 * 16 * P + r * S + i] = side[i];
}

// Split-K: y[m,n] = (sum_s partial[s][n][m]) * colscale[n] * 2^f[m] + bias[n], summed in split
// order (deterministic).  The partials are n-major ([split][N][Mp], Mp a multiple of 16) so the GEMM
// epilogue writes each thread's tokens contiguously.  A CTA takes a TT-token x 64-channel tile
// (TT = 16, 32 or 64, the smallest that holds M, so small batches keep every thread busy): pass 1
// sums the splits with 16-byte loads, four splits' loads in flight before their adds, into a
// shared-memory tile; pass 2 reads it transposed and writes 8 consecutive channels of a token per
// thread (one 16-byte store for 2-byte outputs).  (Launching it as a programmatic dependent of the
// GEMM measured 0.5-0.7 us slower per call at M = 16 .. 256.)  grid = (ceil(M/TT), ceil(N/64)),
// block = 256.
template <int TT>
__global__ void __launch_bounds__(256) splitk_finalize_kernel(
    const float* __restrict__ partial, int splits, int M, int N, int Mp, const void* col_scale, int col_scale_kind,
    const int32_t* w_row_exp, const int32_t* x_row_exp, const float* x_row_scale, const void* bias, int bias_kind,
    void* y, int y_dtype, long long ldy, const PeerOut po, int lora, long long lim_partial, int vec_out) {
  constexpr int kQ = TT / 4;          // float4 columns of a channel's tokens
  constexpr int kTasks = 64 * kQ / 256;  // pass-1 tasks per thread (1, 2 or 4)
  __shared__ float tile[64][TT + 1];  // [channel][token]; the odd pitch keeps pass 2 conflict-free
  const int m0 = blockIdx.x * TT, n0 = blockIdx.y * 64;
  const int t = threadIdx.x;
  const long long plane = (long long)N * Mp;
  long long off[kTasks];
  bool in[kTasks];
  float4 acc[kTasks];
#pragma unroll
  for (int i = 0; i < kTasks; ++i) {
    const int task = t + 256 * i, nl = task / kQ, m = m0 + (task % kQ) * 4, n = n0 + nl;
    off[i] = (long long)n * Mp + m;
    in[i] = n < N && m < Mp;
    acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  for (int s0 = 0; s0 < splits; s0 += 4) {
    float4 v[4][kTasks];
#pragma unroll
    for (int u = 0; u < 4; ++u)
#pragma unroll
      for (int i = 0; i < kTasks; ++i) {
        const long long o = (s0 + u) * plane + off[i];
        v[u][i] = (s0 + u < splits && in[i] && qchk_span(BS_FINAL, o, 4, lim_partial))
                      ? *reinterpret_cast<const float4*>(partial + o) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
    for (int u = 0; u < 4; ++u)
#pragma unroll
      for (int i = 0; i < kTasks; ++i) {
        if (s0 + u >= splits) continue;
        acc[i].x = __fadd_rn(acc[i].x, v[u][i].x);
        acc[i].y = __fadd_rn(acc[i].y, v[u][i].y);
        acc[i].z = __fadd_rn(acc[i].z, v[u][i].z);
        acc[i].w = __fadd_rn(acc[i].w, v[u][i].w);
      }
  }
#pragma unroll
  for (int i = 0; i < kTasks; ++i) {
    const int task = t + 256 * i, nl = task / kQ, ml = (task % kQ) * 4;
    tile[nl][ml] = acc[i].x;
    tile[nl][ml + 1] = acc[i].y;
    tile[nl][ml + 2] = acc[i].z;
    tile[nl][ml + 3] = acc[i].w;
  }
  __syncthreads();
  // pass 2: task (token ml, channels 8g .. 8g+7), 8 * TT tasks
  for (int task = t; task < 8 * TT; task += 256) {
    const int ml = task >> 3, g = task & 7;
    const int m = m0 + ml, nb = n0 + 8 * g;
    if (m >= M || nb >= N) continue;
    const bool has_e = x_row_exp != nullptr && qchk(BS_FINAL, m, M);
    const bool has_s = x_row_scale != nullptr && qchk(BS_FINAL, m, M);
    const float re = has_e ? exp2i(x_row_exp[m]) : 1.f;
    const float rsc = has_s ? x_row_scale[m] : 1.f;
    float o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int n = nb + j;
      if (n >= N) { o[j] = 0.f; continue; }
      float cs = 1.f;
      if (col_scale_kind == 1) cs = __half2float(reinterpret_cast<const __half*>(col_scale)[n]);
      else if (col_scale_kind == 2) cs = reinterpret_cast<const float*>(col_scale)[n];
      else if (col_scale_kind == 3) cs = exp2i(w_row_exp[n]);
      if (lora) cs = lora_safe_scale(cs);
      float v = __fmul_rn(tile[8 * g + j][ml], cs);
      if (has_e) v = __fmul_rn(v, re);
      if (has_s) v = __fmul_rn(v, rsc);
      float b = 0.f;
      if (bias_kind == 1) b = __half2float(reinterpret_cast<const __half*>(bias)[n]);
      else if (bias_kind == 2) b = reinterpret_cast<const float*>(bias)[n];
      else if (bias_kind == 3) b = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(bias)[n]);
      o[j] = __fadd_rn(v, b);
    }
    const long long oi = (long long)m * ldy + nb;
    const int cnt = min(8, N - nb);
    if (!qchk_span(BS_FINAL, oi, cnt, (long long)(M - 1) * ldy + N)) continue;
    if (po.ndst > 0 || y_dtype != 0) {
      uint16_t bits[8];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        bits[j] = y_dtype == 2 ? __bfloat16_as_ushort(__float2bfloat16_rn(o[j])) : __half_as_ushort(__float2half_rn(o[j]));
      const int nd = po.ndst > 0 ? po.ndst : 1;
#pragma unroll
      for (int d = 0; d < kMaxPeers; ++d) {
        if (d >= nd) break;
        uint16_t* dst = reinterpret_cast<uint16_t*>(po.ndst > 0 ? po.dst[d] : y) + oi;
        if (vec_out && cnt == 8) {
          *reinterpret_cast<uint4*>(dst) = make_uint4(bits[0] | ((uint32_t)bits[1] << 16), bits[2] | ((uint32_t)bits[3] << 16),
                                                      bits[4] | ((uint32_t)bits[5] << 16), bits[6] | ((uint32_t)bits[7] << 16));
        } else {
          for (int j = 0; j < cnt; ++j) dst[j] = bits[j];
        }
      }
    } else {
      float* dst = reinterpret_cast<float*>(y) + oi;
      if (vec_out && cnt == 8) {
        *reinterpret_cast<float4*>(dst) = make_float4(o[0], o[1], o[2], o[3]);
        *reinterpret_cast<float4*>(dst + 4) = make_float4(o[4], o[5], o[6], o[7]);
      } else {
        for (int j = 0; j < cnt; ++j) dst[j] = o[j];
      }
    }
  }
  if (po.signal) {
    __syncthreads();
    if (t == 0) peer_signal_last_cta(po);
  }
}

// ---------------------------------------------------------------------------------------------
// Tensor-core block-Hadamard prologue for fp16 / bf16 activations (fp16 output, per-row power of
// two).  A group of G = 16 * A values factors as H_G = H_A (x) H_16 (index i = 16 a + b): the
// 16-point factor runs on mma.sync (m16n8k16, fp32 accumulate, entries +-1 exact), the A-point
// factor as butterflies on the accumulators, which hold all A chunks of the same (row, column)
// position in one thread.  A CTA takes 16 rows: the tile is staged in shared memory once, pass 1
// finds the row maxima, pass 2 recomputes the rotation, scales, rounds to fp16 in place and the
// tile is stored with 16-byte writes.  KIND 0: Sylvester; KIND 1: H4 (x) H4 (x) H4 (G = 64).
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

template <int KIND>
__device__ __forceinline__ float hadamard16_entry(int k, int n) {
  if constexpr (KIND == 0) return (__popc(k & n) & 1) ? -1.f : 1.f;
  const float a = ((n >> 2) == 3 - (k >> 2)) ? -1.f : 1.f;
  const float b = ((n & 3) == 3 - (k & 3)) ? -1.f : 1.f;
  return a * b;
}

template <bool BF16>
__device__ __forceinline__ uint32_t pack_pm1(float lo, float hi) {
  if constexpr (BF16) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  } else {
    return pack_f16x2(lo, hi);
  }
}

template <bool BF16>
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  if constexpr (BF16) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%10,%10,%10,%10};"
                 : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(0.f));
  } else {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%10,%10,%10,%10};"
                 : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(0.f));
  }
}

// Rotated values of group g for this lane: z[a][nb][c] = row (lane/4 + 8*(c>>1)),
// column 16a + 8nb + 2*(lane%4) + (c&1) of the group, not yet normalized: the caller multiplies by
// prologue_norm<A>() = 1/sqrt(G), folded into its power-of-two scale.
template <int A>
__device__ __forceinline__ constexpr float prologue_norm() {
  return A == 2 ? 0.17677669529663687f : A == 4 ? 0.125f : 0.08838834764831845f;
}

template <int A, int KIND, bool BF16>
__device__ __forceinline__ void rotate_group(const uint8_t* tile, int pitch, int g, int lane,
                                             const uint32_t (&hb)[2][2], float (&z)[A][2][4]) {
  const int row = (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
  for (int a = 0; a < A; ++a) {
    const int col = g * 16 * A + 16 * a + (lane >> 4) * 8;
    uint32_t fr[4];
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(fr[0]), "=r"(fr[1]), "=r"(fr[2]), "=r"(fr[3])
                 : "r"(smem_u32(tile + row * pitch + col * 2)));
    mma_16816<BF16>(z[a][0], fr, hb[0][0], hb[0][1]);
    mma_16816<BF16>(z[a][1], fr, hb[1][0], hb[1][1]);
  }
#pragma unroll
  for (int nb = 0; nb < 2; ++nb) {
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      if constexpr (KIND == 0) {
#pragma unroll
        for (int st = 1; st < A; st <<= 1) {
#pragma unroll
          for (int a = 0; a < A; ++a) {
            if (a & st) continue;
            const float u = z[a][nb][c], v = z[a + st][nb][c];
            z[a][nb][c] = __fadd_rn(u, v);
            z[a + st][nb][c] = __fsub_rn(u, v);
          }
        }
      } else {
        const float t = __fadd_rn(__fadd_rn(z[0][nb][c], z[1][nb][c]), __fadd_rn(z[2][nb][c], z[3][nb][c]));
        float y[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) y[k] = __fsub_rn(t, __fmul_rn(2.f, z[3 - k][nb][c]));
#pragma unroll
        for (int k = 0; k < 4; ++k) z[k][nb][c] = y[k];
      }
    }
  }
}

// Exponent e with |v| * 2^-e in [2^14, 2^15) for the largest |v| = amax (0 for zero / non-finite).
__device__ __forceinline__ int pow2_exponent(float amax) {
  int f = 0;
  if (amax > 0.f && amax <= 3.402823466e38f) {
    int ex;
    frexpf(amax, &ex);
    f = ex - 15;
  }
  return f;
}

// Group exponent records of the single-pass prologue: a group of zeros and a group holding a
// non-finite value are marked (their values were scaled by 2^0).
constexpr int kGroupZero = -(1 << 20), kGroupNonFinite = 1 << 20;
__device__ __forceinline__ int group_exponent_code(float amax, int f) {
  return amax == 0.f ? kGroupZero : !(amax <= 3.402823466e38f) ? kGroupNonFinite : f;
}

// One pass over the tile: each warp rotates its groups once, scales each (row, group) by its own
// power of two (the group's maximum into [2^14, 2^15)), rounds to fp16 in place and records the
// exponent.  The row exponent is the largest of its groups' (the exponent of the row maximum);
// the store loop multiplies each group by 2^(group - row) on the way out, exact in fp16 except for
// results below the fp16 normal range (|v| < 2^-14 against a row maximum of at least 2^14).  The
// tile arrives in rounds of 8 groups (one per warp) so the first rotations overlap later loads.
template <int A, int KIND, bool BF16>
__global__ void __launch_bounds__(256) prologue_mma_kernel(const void* __restrict__ x, long long ldx, int M, int K,
                                                           __half* __restrict__ out, long long ldo,
                                                           int32_t* __restrict__ row_exp) {
  extern __shared__ __align__(16) uint8_t psm[];
  const int pitch = K * 2 + 16;
  const int groups = K / (16 * A);
  uint8_t* tile = psm;
  int* gexp = reinterpret_cast<int*>(psm + 16 * pitch);  // [16 rows][groups]
  int* rexp = gexp + 16 * groups;                          // [16 rows]
  const int row0 = blockIdx.x * 16;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr int kGroupCols = 16 * A;
  const int rounds = (groups + 7) / 8;
  // Loads, one commit group per round of 8 groups.  (row, chunk) advance without divisions.
  for (int j = 0; j < rounds; ++j) {
    const int c0 = j * kGroupCols, c1 = min(groups, j * 8 + 8) * kGroupCols / 8;  // 16-byte chunks
    const int cpr = c1 - c0;
    const int dr = 256 / cpr, dc = 256 - dr * cpr;
    int r = tid / cpr, c = tid - r * cpr;
    for (; r < 16; r += dr, c += dc) {
      if (c >= cpr) {
        c -= cpr;
        if (++r >= 16) break;
      }
      uint8_t* dst = tile + r * pitch + (c0 + c) * 16;
      if (!qchk_smem(BS_PRO_OUT, psm, dst, 16)) continue;
      if (row0 + r < M) {
        if (qchk_span(BS_PRO_X, (long long)(row0 + r) * ldx + (c0 + c) * 8, 8, (long long)(M - 1) * ldx + K))
          cp_async16(dst, reinterpret_cast<const uint8_t*>(x) + ((long long)(row0 + r) * ldx + (c0 + c) * 8) * 2);
      } else {
        *reinterpret_cast<uint4*>(dst) = make_uint4(0u, 0u, 0u, 0u);
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  }
  // B fragments of H16 (symmetric): n-block nb, k rows 2(lane%4)+{0,1} and +8, column lane/4.
  uint32_t hb[2][2];
#pragma unroll
  for (int nb = 0; nb < 2; ++nb) {
    const int n = nb * 8 + (lane >> 2), k0 = 2 * (lane & 3);
    hb[nb][0] = pack_pm1<BF16>(hadamard16_entry<KIND>(k0, n), hadamard16_entry<KIND>(k0 + 1, n));
    hb[nb][1] = pack_pm1<BF16>(hadamard16_entry<KIND>(k0 + 8, n), hadamard16_entry<KIND>(k0 + 9, n));
  }
  constexpr float kNorm = prologue_norm<A>();
  for (int j = 0; j < rounds; ++j) {
    const int pending = rounds - 1 - j;  // commit groups still allowed in flight
    if (pending >= 2) asm volatile("cp.async.wait_group 2;" ::: "memory");
    else if (pending == 1) asm volatile("cp.async.wait_group 1;" ::: "memory");
    else asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    const int g = j * 8 + warp;
    if (g < groups) {
      float z[A][2][4];
      rotate_group<A, KIND, BF16>(tile, pitch, g, lane, hb, z);
      float m_lo = 0.f, m_hi = 0.f;
#pragma unroll
      for (int a = 0; a < A; ++a)
#pragma unroll
        for (int nb = 0; nb < 2; ++nb) {
          m_lo = fmaxf(m_lo, fmaxf(fabsf(z[a][nb][0]), fabsf(z[a][nb][1])));
          m_hi = fmaxf(m_hi, fmaxf(fabsf(z[a][nb][2]), fabsf(z[a][nb][3])));
        }
#pragma unroll
      for (int o = 1; o <= 2; o <<= 1) {
        m_lo = fmaxf(m_lo, __shfl_xor_sync(0xffffffffu, m_lo, o));
        m_hi = fmaxf(m_hi, __shfl_xor_sync(0xffffffffu, m_hi, o));
      }
      // max |z * kNorm| = RN(max|z| * kNorm): rounding is monotonic
      const float a_lo = __fmul_rn(m_lo, kNorm), a_hi = __fmul_rn(m_hi, kNorm);
      const int f_lo = pow2_exponent(a_lo), f_hi = pow2_exponent(a_hi);
      if ((lane & 3) == 0 && qchk_smem(BS_PRO_OUT, psm, gexp + ((lane >> 2) + 8) * groups + g, 4)) {
        gexp[(lane >> 2) * groups + g] = group_exponent_code(a_lo, f_lo);
        gexp[((lane >> 2) + 8) * groups + g] = group_exponent_code(a_hi, f_hi);
      }
      // z * (kNorm * 2^-f) = RN(z * kNorm) * 2^-f while the scale is a normal fp32 number; rows
      // of extreme exponents take the two-step form (a warp-uniform branch around whole loops)
      const bool fast = __all_sync(0xffffffffu, f_lo >= -100 && f_lo <= 100 && f_hi >= -100 && f_hi <= 100);
      if (fast) {
        const float s_lo = exp2i(-f_lo) * kNorm, s_hi = exp2i(-f_hi) * kNorm;
#pragma unroll
        for (int a = 0; a < A; ++a)
#pragma unroll
          for (int nb = 0; nb < 2; ++nb) {
            const int col = g * kGroupCols + 16 * a + 8 * nb + 2 * (lane & 3);
            if (!qchk_smem(BS_PRO_OUT, psm, tile + ((lane >> 2) + 8) * pitch + col * 2, 4)) continue;
            *reinterpret_cast<uint32_t*>(tile + (lane >> 2) * pitch + col * 2) =
                pack_f16x2(__fmul_rn(z[a][nb][0], s_lo), __fmul_rn(z[a][nb][1], s_lo));
            *reinterpret_cast<uint32_t*>(tile + ((lane >> 2) + 8) * pitch + col * 2) =
                pack_f16x2(__fmul_rn(z[a][nb][2], s_hi), __fmul_rn(z[a][nb][3], s_hi));
          }
      } else {
#pragma unroll
        for (int a = 0; a < A; ++a)
#pragma unroll
          for (int nb = 0; nb < 2; ++nb) {
            const int col = g * kGroupCols + 16 * a + 8 * nb + 2 * (lane & 3);
            if (!qchk_smem(BS_PRO_OUT, psm, tile + ((lane >> 2) + 8) * pitch + col * 2, 4)) continue;
            *reinterpret_cast<uint32_t*>(tile + (lane >> 2) * pitch + col * 2) =
                pack_f16x2(scale_pow2(__fmul_rn(z[a][nb][0], kNorm), f_lo), scale_pow2(__fmul_rn(z[a][nb][1], kNorm), f_lo));
            *reinterpret_cast<uint32_t*>(tile + ((lane >> 2) + 8) * pitch + col * 2) =
                pack_f16x2(scale_pow2(__fmul_rn(z[a][nb][2], kNorm), f_hi), scale_pow2(__fmul_rn(z[a][nb][3], kNorm), f_hi));
          }
      }
    }
  }
  __syncthreads();
  if (tid < 16) {
    // the exponent of the row maximum: the largest over nonzero groups; 0 for a zero row or a row
    // with a non-finite value (as the exponent of the row maximum itself)
    int f = kGroupZero;
    for (int g = 0; g < groups; ++g) f = max(f, gexp[tid * groups + g]);
    if (f == kGroupZero || f == kGroupNonFinite) f = 0;
    if (qchk_smem(BS_PRO_OUT, psm, rexp + tid, 4)) rexp[tid] = f;
    if (row0 + tid < M) row_exp[row0 + tid] = f;
  }
  __syncthreads();
  const int cpr = K / 8;
  const int dr = 256 / cpr, dc = 256 - dr * cpr;
  int r = tid / cpr, c = tid - r * cpr;
  for (; r < 16; r += dr, c += dc) {
    if (c >= cpr) {
      c -= cpr;
      if (++r >= 16) break;
    }
    if (row0 + r >= M) break;
    if (!qchk_smem(BS_PRO_OUT, psm, tile + r * pitch + c * 16, 16) ||
        !qchk_span(BS_PRO_OUT, (long long)(row0 + r) * ldo + c * 8, 8, (long long)M * ldo))
      continue;
    uint4 v = *reinterpret_cast<const uint4*>(tile + r * pitch + c * 16);
    const int code = gexp[r * groups + (c * 8) / kGroupCols];
    const int d = (code == kGroupZero ? rexp[r] : code == kGroupNonFinite ? 0 : code) - rexp[r];
    if (d != 0) {
      uint32_t* w = reinterpret_cast<uint32_t*>(&v);
      if (d >= -14 && d < 0) {
        const __half2 sc = __half2half2(__ushort_as_half((unsigned short)((d + 15) << 10)));  // 2^d
#pragma unroll
        for (int e = 0; e < 4; ++e) w[e] = hmul2_u32(w[e], sc);
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f2 = __half22float2(*reinterpret_cast<const __half2*>(&w[e]));
          w[e] = pack_f16x2(scale_pow2(f2.x, -d), scale_pow2(f2.y, -d));
        }
      }
    }
    *reinterpret_cast<uint4*>(out + (long long)(row0 + r) * ldo + c * 8) = v;
  }
}

// Launches the tensor-core prologue when it applies (fp16 / bf16 input, fp16 output, groups of
// 32 / 128 (Sylvester) or 64 (H4 (x) H4 (x) H4), whole groups, 16-byte aligned rows, the tile in
// shared memory); returns false otherwise.
static bool launch_prologue_mma(const void* x, int x_dtype, long long ldx, int M, int K, int Kp, int group, int kind,
                                void* out, int32_t* row_exp, cudaStream_t stream) {
  if ((x_dtype != 1 && x_dtype != 2) || K != Kp || K % group != 0 || K % 8 != 0 || ldx % 8 != 0 ||
      (reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(out) & 15))
    return false;
  const size_t smem = 16 * ((size_t)K * 2 + 16) + 4 * (16 * (size_t)(K / group) + 16);
  if (smem > 200 * 1024) return false;
  const bool bf = x_dtype == 2;
  const dim3 grid((M + 15) / 16);
  __half* o = reinterpret_cast<__half*>(out);
#define QLIN_MMA_PRO(AA, KK, BB)                                                                           \
  do {                                                                                                     \
    auto kern = prologue_mma_kernel<AA, KK, BB>;                                                           \
    static bool attr_done[64] = {false};                                                                   \
    int dev = 0;                                                                                           \
    cudaGetDevice(&dev);                                                                                   \
    if (dev >= 0 && dev < 64 && !attr_done[dev]) {                                                         \
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024 + 64) !=      \
          cudaSuccess)                                                                                     \
        return false;                                                                                      \
      attr_done[dev] = true;                                                                               \
    }                                                                                                      \
    kern<<<grid, 256, smem, stream>>>(x, ldx, M, K, o, Kp, row_exp);                                       \
  } while (0)
  if (group == 128 && kind == 0) {
    if (bf) QLIN_MMA_PRO(8, 0, true); else QLIN_MMA_PRO(8, 0, false);
  } else if (group == 32 && kind == 0) {
    if (bf) QLIN_MMA_PRO(2, 0, true); else QLIN_MMA_PRO(2, 0, false);
  } else if (group == 64 && kind == 1) {
    if (bf) QLIN_MMA_PRO(4, 1, true); else QLIN_MMA_PRO(4, 1, false);
  } else {
    return false;
  }
#undef QLIN_MMA_PRO
  return true;
}

// ---------------------------------------------------------------------------------------------
// Kitchen W4A8 / W6A8 (AsymW4A8Int8Layout, symmetric) -> its int8 weight grid, bit-exact:
// grid = clamp(rint(level[code] * s_rel), +-127) in fp32 (`modal/weight_error_app.py:326-336`).
// Codes: planar packing, K/2 bytes of nibble pairs (even column low), then for 6 bits K/4 bytes of
// 2-bit high planes (column 4j+i at bits 2i..2i+1 of byte j).  s_rel: float8_e4m3fn per group.
// One thread per 16 consecutive values of a row; the level table (<= 64 fp32) sits in shared memory.
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ float e4m3_to_float(uint32_t b) {
  const uint32_t e = (b >> 3) & 0xF, m = b & 7;
  float v = e == 0 ? (float)m * 0.001953125f                              // m/8 * 2^-6
                   : __uint_as_float(((e + 120u) << 23) | (m << 20));     // (1 + m/8) * 2^(e-7)
  if ((b & 0x7F) == 0x7F) v = __uint_as_float(0x7FC00000u);
  return (b & 0x80) ? -v : v;
}

__global__ void kitchen_grid_kernel(const uint8_t* __restrict__ q, const uint8_t* __restrict__ s_rel,
                                    const float* __restrict__ codebook, int bits, int group, int N, int K,
                                    int8_t* __restrict__ out) {
  __shared__ float levels[64];
  const int nlev = 1 << bits;
  if (threadIdx.x < nlev && qchk(BS_KITCHEN, threadIdx.x, 64))
    levels[threadIdx.x] = codebook ? codebook[threadIdx.x] : (float)((int)threadIdx.x - nlev / 2);
  __syncthreads();
  const int gpr = K / 16;
  const long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= (long long)N * gpr) return;
  const int row = (int)(t / gpr), c0 = (int)(t - (long long)row * gpr) * 16;
  const long long pitch = (long long)K * bits / 8;
  const uint8_t* qr = q + row * pitch;
  if (!qchk_span(BS_KITCHEN, row * pitch + c0 / 2, 8, (long long)N * pitch) ||
      (bits == 6 && !qchk_span(BS_KITCHEN, row * pitch + K / 2 + c0 / 4, 4, (long long)N * pitch)) ||
      !qchk(BS_KITCHEN, (long long)row * (K / group) + c0 / group, (long long)N * (K / group)) ||
      !qchk_span(BS_KITCHEN, (long long)row * K + c0, 16, (long long)N * K))
    return;
  const uint2 lo = *reinterpret_cast<const uint2*>(qr + c0 / 2);
  uint32_t hi = 0;
  if (bits == 6) hi = *reinterpret_cast<const uint32_t*>(qr + K / 2 + c0 / 4);
  const float sc = e4m3_to_float(s_rel[(long long)row * (K / group) + c0 / group]);
  uint32_t w[4] = {0, 0, 0, 0};
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const uint32_t byte = ((i < 8 ? lo.x : lo.y) >> (8 * ((i >> 1) & 3))) & 0xFF;
    uint32_t code = (i & 1) ? (byte >> 4) : (byte & 0xF);
    if (bits == 6) code |= ((hi >> (2 * i)) & 3) << 4;
    const float v = qchk(BS_KITCHEN, code, nlev) ? fminf(fmaxf(rintf(__fmul_rn(levels[code], sc)), -127.f), 127.f) : 0.f;
    w[i >> 2] |= ((uint32_t)(int)v & 0xFF) << (8 * (i & 3));
  }
  *reinterpret_cast<uint4*>(out + (long long)row * K + c0) = make_uint4(w[0], w[1], w[2], w[3]);
}

// Uniform levels, two values at a time in fp16, exactly: the codes go under the fp16 magic exponent
// (0x64XX is 1024 + XX), lose their offset (1024 + 8 or 1024 + 32), are multiplied by the e4m3
// scale and clamped to [-127, 127]; every product is exact in fp16 (a level of at most 6 bits times
// a 4-bit significand, |v| <= 14336, nonzero |v| >= 2^-9), so this equals the fp32 product of the
// reference.  Adding 1.5 * 2^10 then rounds half-to-even to an integer (fp16 spacing 1 on
// [1024, 2048)) and leaves the two's-complement code in the low byte of each half.
// p: two codes as (1024 + code) fp16 pairs; s: the scale as an fp16 pair.
template <int BITS>
__device__ __forceinline__ uint32_t kitchen_uniform2(uint32_t p, uint32_t s) {
  constexpr uint32_t kOff = BITS == 4 ? 0x64086408u : 0x64206420u;  // 1024 + 8 / 1024 + 32
  uint32_t d;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(p), "r"(kOff));
  asm("mul.rn.f16x2 %0, %0, %1;" : "+r"(d) : "r"(s));
  asm("max.f16x2 %0, %0, %1;" : "+r"(d) : "r"(0xD7F0D7F0u));  // -127
  asm("min.f16x2 %0, %0, %1;" : "+r"(d) : "r"(0x57F057F0u));  // 127
  asm("add.rn.f16x2 %0, %0, %1;" : "+r"(d) : "r"(0x66006600u));  // + 1536
  return d;
}

// Packed fp32 (a.x * s, a.y * s) and (a.x + c, a.y + c), each correctly rounded.
__device__ __forceinline__ float2 mul2_rn(float2 a, float s) {
  asm("{\n\t.reg .b64 x, y;\n\t"
      "mov.b64 x, {%0, %1};\n\t"
      "mov.b64 y, {%2, %2};\n\t"
      "mul.rn.f32x2 x, x, y;\n\t"
      "mov.b64 {%0, %1}, x;\n\t}"
      : "+f"(a.x), "+f"(a.y)
      : "f"(s));
  return a;
}
__device__ __forceinline__ float2 add2_rn(float2 a, float c) {
  asm("{\n\t.reg .b64 x, y;\n\t"
      "mov.b64 x, {%0, %1};\n\t"
      "mov.b64 y, {%2, %2};\n\t"
      "add.rn.f32x2 x, x, y;\n\t"
      "mov.b64 {%0, %1}, x;\n\t}"
      : "+f"(a.x), "+f"(a.y)
      : "f"(c));
  return a;
}

// 2-bit fields at bits 4k..4k+1 (k = 0..3) of the low 16 bits of h -> bits 8k+4..8k+5: the high
// planes of four 6-bit codes moved above their nibbles.  With each field alone in its nibble the
// fields are byte selectors (0..3) into the table {0x00, 0x10, 0x20, 0x30}: one byte permute.
__device__ __forceinline__ uint32_t kitchen_spread_hi(uint32_t h) {
  return __byte_perm(0x30201000u, 0u, h & 0x3333u);
}

// The same grid for K a multiple of 32 (8-byte aligned code rows), 32 values of a row per thread:
// 16 code bytes, 8 high-plane bytes for 6 bits and one or two scale bytes in, two 16-byte stores
// out.  Uniform levels take the packed fp16 form above (about four instructions per value, no
// conversions); codebook levels are looked up and multiplied in fp32 (packed pairs), clamped, and
// rounded half-to-even by adding 1.5 * 2^23 (the code is then the low byte of the sum).  Clamping
// before rounding gives the same integers as rounding first: both give +-127 whenever
// |x| >= 127.5.  (Two 32-value chunks per thread, with the loads of both issued first, measured
// ~10 % slower.)
template <int BITS, bool CB>
__global__ void __launch_bounds__(256) kitchen_grid32_kernel(const uint8_t* __restrict__ q,
                                                             const uint8_t* __restrict__ s_rel,
                                                             const float* __restrict__ codebook, int group, int N,
                                                             int K, int8_t* __restrict__ out) {
  constexpr int kLevels = 1 << BITS;
  __shared__ float levels[kLevels];
  if (CB && threadIdx.x < kLevels) levels[threadIdx.x] = codebook[threadIdx.x];
  if (CB) __syncthreads();
  // 32-bit unit index (the launcher keeps N * K / 32 below 2^31): a 64-bit division per thread
  // is a visible share of this short pass
  const unsigned gpr = (unsigned)K / 32u;
  const unsigned t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= (unsigned)N * gpr) return;
  const int row = (int)(t / gpr), c0 = (int)(t - (unsigned)row * gpr) * 32;
  const long long pitch = (long long)K * BITS / 8;
  const uint8_t* qr = q + row * pitch;
  if (!qchk_span(BS_KITCHEN, row * pitch + c0 / 2, 16, (long long)N * pitch) ||
      (BITS == 6 && !qchk_span(BS_KITCHEN, row * pitch + K / 2 + c0 / 4, 8, (long long)N * pitch)) ||
      !qchk_span(BS_KITCHEN, (long long)row * (K / group) + c0 / group, group == 16 ? 2 : 1,
                 (long long)N * (K / group)) ||
      !qchk_span(BS_KITCHEN, (long long)row * K + c0, 32, (long long)N * K))
    return;
  const uint2 lo0 = *reinterpret_cast<const uint2*>(qr + c0 / 2);
  const uint2 lo1 = *reinterpret_cast<const uint2*>(qr + c0 / 2 + 8);
  const uint32_t lw[4] = {lo0.x, lo0.y, lo1.x, lo1.y};
  uint2 hi = make_uint2(0u, 0u);
  if (BITS == 6) hi = *reinterpret_cast<const uint2*>(qr + K / 2 + c0 / 4);
  const long long sbase = (long long)row * (K / group) + c0 / group;
  const float sc0 = e4m3_to_float(s_rel[sbase]);
  const float sc1 = group == 16 ? e4m3_to_float(s_rel[sbase + 1]) : sc0;
  uint32_t w[8];
  if constexpr (!CB) {
    const __half h0 = __float2half_rn(sc0), h1 = __float2half_rn(sc1);  // exact: e4m3 values are fp16 values
    const uint32_t s0 = (uint32_t)__half_as_ushort(h0) * 0x10001u, s1 = (uint32_t)__half_as_ushort(h1) * 0x10001u;
#pragma unroll
    for (int t = 0; t < 4; ++t) {  // word t: values 8t .. 8t+7 (value 8t+2b in the low nibble of byte b)
      uint32_t a = lw[t] & 0x0F0F0F0Fu, b = (lw[t] >> 4) & 0x0F0F0F0Fu;  // even / odd values, one per byte
      if (BITS == 6) {
        const uint32_t hw = ((t < 2 ? hi.x : hi.y) >> (16 * (t & 1))) & 0xFFFFu;  // value 8t+i at bits 2i..2i+1
        a |= kitchen_spread_hi(hw);
        b |= kitchen_spread_hi(hw >> 2);
      }
      const uint32_t s = t < 2 ? s0 : s1;
      const uint32_t ca0 = kitchen_uniform2<BITS>(__byte_perm(a, 0x64646464u, 0x4140), s);  // values 8t, 8t+2
      const uint32_t ca1 = kitchen_uniform2<BITS>(__byte_perm(a, 0x64646464u, 0x4342), s);  // 8t+4, 8t+6
      const uint32_t cb0 = kitchen_uniform2<BITS>(__byte_perm(b, 0x64646464u, 0x4140), s);  // 8t+1, 8t+3
      const uint32_t cb1 = kitchen_uniform2<BITS>(__byte_perm(b, 0x64646464u, 0x4342), s);  // 8t+5, 8t+7
      w[2 * t] = __byte_perm(ca0, cb0, 0x6240);
      w[2 * t + 1] = __byte_perm(ca1, cb1, 0x6240);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) {  // values 4j .. 4j+3
      float v[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = 4 * j + e;
        uint32_t code = (lw[i >> 3] >> (4 * (i & 7))) & 0xF;
        if (BITS == 6) code |= (((i < 16 ? hi.x : hi.y) >> (2 * (i & 15))) & 3) << 4;
        v[e] = levels[code];
      }
      const float sc = j < 4 ? sc0 : sc1;
      uint32_t c[4];
#pragma unroll
      for (int e = 0; e < 4; e += 2) {
        float2 x = mul2_rn(make_float2(v[e], v[e + 1]), sc);
        x.x = fminf(fmaxf(x.x, -127.f), 127.f);
        x.y = fminf(fmaxf(x.y, -127.f), 127.f);
        x = add2_rn(x, 12582912.f);  // 1.5 * 2^23 + rint(v): the code in byte 0
        c[e] = __float_as_uint(x.x);
        c[e + 1] = __float_as_uint(x.y);
      }
      w[j] = __byte_perm(__byte_perm(c[0], c[1], 0x0040), __byte_perm(c[2], c[3], 0x0040), 0x5410);
    }
  }
  uint4* o = reinterpret_cast<uint4*>(out + (long long)row * K + c0);
  o[0] = make_uint4(w[0], w[1], w[2], w[3]);
  o[1] = make_uint4(w[4], w[5], w[6], w[7]);
}

// ---------------------------------------------------------------------------------------------
// Fused-LoRA operands (bf16): T'[m][r] = t[m][r] * 2^-f[m] (the activation's row exponent, so the
// GEMM epilogue's 2^f restores t) and U'[n][r] = up[n][r] * scale / cs[n] (the column scale the
// epilogue applies), zero-padded to rk columns and n_pad rows.
// ---------------------------------------------------------------------------------------------
__global__ void lora_t_kernel(const void* __restrict__ t, int t_dtype, long long ldt, int M, int R, int rk,
                              const int32_t* __restrict__ x_row_exp, __nv_bfloat16* __restrict__ out) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)M * rk) return;
  const int m = (int)(i / rk), r = (int)(i - (long long)m * rk);
  float v = (r < R && qchk(BS_LORA, (long long)m * ldt + r, (long long)(M - 1) * ldt + R))
                ? load_x(t, t_dtype, (long long)m * ldt + r) : 0.f;
  if (x_row_exp != nullptr && qchk(BS_LORA, m, M)) v = scale_pow2(v, x_row_exp[m]);
  out[i] = __float2bfloat16_rn(v);
}

__global__ void lora_u_kernel(const void* __restrict__ up, int up_dtype, long long ldu, int N, int n_pad, int R,
                              int rk, float scale, const void* __restrict__ cs, int cs_kind,
                              const int32_t* __restrict__ w_row_exp, __nv_bfloat16* __restrict__ out) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)n_pad * rk) return;
  const int n = (int)(i / rk), r = (int)(i - (long long)n * rk);
  float v = 0.f;
  if (n < N && r < R && qchk(BS_LORA, (long long)n * ldu + r, (long long)(N - 1) * ldu + R)) {
    v = __fmul_rn(load_x(up, up_dtype, (long long)n * ldu + r), scale);
    if (cs_kind == 1) v = __fdiv_rn(v, lora_safe_scale(__half2float(reinterpret_cast<const __half*>(cs)[n])));
    else if (cs_kind == 2) v = __fdiv_rn(v, lora_safe_scale(reinterpret_cast<const float*>(cs)[n]));
    else if (cs_kind == 3) v = scale_pow2(v, w_row_exp[n]);
  }
  out[i] = __float2bfloat16_rn(v);
}

// ---------------------------------------------------------------------------------------------
// Host launchers
// ---------------------------------------------------------------------------------------------
template <int E, int MODE, int BPW>
static void launch_reg(const void* x, int x_dtype, long long ldx, int M, int K, int Kp, int kind, int rotate,
                       void* out, int32_t* row_exp, float* row_scale, int perm, int vec, cudaStream_t stream) {
  const int nblk = (Kp + 32 * E - 1) / (32 * E);
  const int warps = std::min(16, std::max(1, (nblk + BPW - 1) / BPW));
  prologue_reg_kernel<E, MODE, BPW>
      <<<M, 32 * warps, 0, stream>>>(x, x_dtype, ldx, M, K, Kp, kind, rotate, out, row_exp, row_scale, perm, vec);
}

template <int E, int MODE>
static void launch_prologue_e(const void* x, int x_dtype, long long ldx, int M, int K, int Kp, int kind, int rotate,
                              void* out, int32_t* row_exp, float* row_scale, int perm, cudaStream_t stream) {
  const int esz = x_dtype == 0 ? 4 : 2;
  const bool vec = ((reinterpret_cast<uintptr_t>(x) | (uintptr_t)(ldx * esz)) & 15) == 0;
  const bool out_ok = (reinterpret_cast<uintptr_t>(out) & 15) == 0 && Kp % 8 == 0;
  const int nblk = (Kp + 32 * E - 1) / (32 * E);
  constexpr int kMaxBpw = 64 / E;  // at most 64 staged values per thread
  if (out_ok && nblk <= 16 * kMaxBpw) {
    // up to 16 warps per row; the fewest blocks per warp that cover the row
    const int bpw = (nblk + 15) / 16;
    if (bpw <= 1) return launch_reg<E, MODE, 1>(x, x_dtype, ldx, M, K, Kp, kind, rotate, out, row_exp, row_scale, perm, vec, stream);
    if (bpw <= 2) return launch_reg<E, MODE, 2>(x, x_dtype, ldx, M, K, Kp, kind, rotate, out, row_exp, row_scale, perm, vec, stream);
    if (bpw <= 4) return launch_reg<E, MODE, 4>(x, x_dtype, ldx, M, K, Kp, kind, rotate, out, row_exp, row_scale, perm, vec, stream);
    if (bpw <= 8) return launch_reg<E, MODE, (8 <= kMaxBpw ? 8 : kMaxBpw)>(x, x_dtype, ldx, M, K, Kp, kind, rotate, out, row_exp, row_scale, perm, vec, stream);
    if constexpr (kMaxBpw >= 16) {
      if (bpw <= 16) return launch_reg<E, MODE, 16>(x, x_dtype, ldx, M, K, Kp, kind, rotate, out, row_exp, row_scale, perm, vec, stream);
    }
    if constexpr (kMaxBpw >= 32) {
      if (bpw <= 32) return launch_reg<E, MODE, 32>(x, x_dtype, ldx, M, K, Kp, kind, rotate, out, row_exp, row_scale, perm, vec, stream);
    }
    if constexpr (kMaxBpw >= 64) {
      return launch_reg<E, MODE, 64>(x, x_dtype, ldx, M, K, Kp, kind, rotate, out, row_exp, row_scale, perm, vec, stream);
    }
  }
  // Long rows: two passes over global memory (the second mostly from L2).
  prologue_kernel<E, MODE><<<M, 256, 0, stream>>>(x, x_dtype, ldx, M, K, Kp, kind, rotate, out, row_exp, row_scale,
                                                  perm, 0, vec ? 1 : 0);
}

int launch_prologue(const void* x, int x_dtype, long long ldx, int M, int K, int Kp, int group, int mode, void* out,
                    int32_t* row_exp, float* row_scale, int perm, cudaStream_t stream) {
  if (M == 0) return 0;
  const int rotate = group > 0;
  int E = 8, kind = 0;
  if (rotate) {
    switch (group) {
      case 32: E = 1; kind = 0; break;
      case 64: E = 2; kind = 1; break;
      case 128: E = 4; kind = 0; break;
      case 256: E = 8; kind = 1; break;
      default: return -1;
    }
  }
  // Unrotated int8 codes of fp16 / bf16 rows: the packed quantizer when the rows are 16-byte
  // vectors and one CTA of at most 512 threads holds a row in 8 vectors per thread or fewer.
  if (mode == 1 && !rotate && (x_dtype == 1 || x_dtype == 2) && K % 8 == 0 && Kp % 8 == 0 && Kp <= 32768 &&
      ((reinterpret_cast<uintptr_t>(x) | (uintptr_t)(ldx * 2)) & 15) == 0 &&
      (reinterpret_cast<uintptr_t>(out) & 7) == 0) {
    const int nvp = Kp / 8;
    const int nv = nvp <= 512 ? 1 : nvp <= 1024 ? 2 : nvp <= 2048 ? 4 : 8;
    const int threads = ((nvp + nv - 1) / nv + 31) / 32 * 32;
    const uint16_t* xs = reinterpret_cast<const uint16_t*>(x);
    int8_t* o = reinterpret_cast<int8_t*>(out);
#define QLIN_Q16(NV)                                                                                  \
  do {                                                                                                \
    if (x_dtype == 2) quant_rows16_kernel<NV, true><<<M, threads, 0, stream>>>(xs, ldx, M, K, Kp, o, row_scale, perm); \
    else quant_rows16_kernel<NV, false><<<M, threads, 0, stream>>>(xs, ldx, M, K, Kp, o, row_scale, perm); \
  } while (0)
    switch (nv) {
      case 1: QLIN_Q16(1); break;
      case 2: QLIN_Q16(2); break;
      case 4: QLIN_Q16(4); break;
      default: QLIN_Q16(8); break;
    }
#undef QLIN_Q16
    return 0;
  }
  // Tuning knob: QLIN_FWHT_PROLOGUE=1 keeps the shuffle-butterfly rotation for comparisons.
  static const bool fwht_only = getenv("QLIN_FWHT_PROLOGUE") != nullptr;
  if (mode == 0 && rotate && !fwht_only &&
      launch_prologue_mma(x, x_dtype, ldx, M, K, Kp, group, kind, out, row_exp, stream))
    return 0;
#define QLIN_PRO(EE)                                                                                       \
  do {                                                                                                     \
    if (mode == 0) launch_prologue_e<EE, 0>(x, x_dtype, ldx, M, K, Kp, kind, rotate, out, row_exp, row_scale, perm, stream); \
    else launch_prologue_e<EE, 1>(x, x_dtype, ldx, M, K, Kp, kind, rotate, out, row_exp, row_scale, perm, stream); \
  } while (0)
  switch (E) {
    case 1: QLIN_PRO(1); break;
    case 2: QLIN_PRO(2); break;
    case 4: QLIN_PRO(4); break;
    default: QLIN_PRO(8); break;
  }
#undef QLIN_PRO
  return 0;
}

// GGUF weights whose rows straddle blocks (K not a whole number of blocks; the blocks run over
// the flattened [N, K] tensor): decoded once by flat element into plain fp16 rows w * 2^-e, [n_pad,
// ldw] (zeros past K and past N), with e the row exponent of the row's largest |w| (as for the
// other layouts: that weight lands in [2^14, 2^15)).  One CTA per row: a max pass, then the writes.
__global__ void gguf_straddle_repack_kernel(const uint8_t* __restrict__ raw, int qtype, int N, int K, int ldw,
                                            __half* __restrict__ out, int32_t* __restrict__ row_exp,
                                            long long out_elems) {
  const int n = blockIdx.x;
  __shared__ float red[32];
  __shared__ int e_row;
  const int qk = gguf_qk(qtype), ts = gguf_ts(qtype);
  const long long raw_bytes = (long long)N * K / qk * ts;
  float mx = 0.f;
  if (n < N)
    for (int k = threadIdx.x; k < K; k += blockDim.x)
      if (qchk_span(BS_REPACK_SRC, ((long long)n * K + k) / qk * ts, ts, raw_bytes))
        mx = fmaxf(mx, fabsf(gguf_value(raw, qtype, (long long)n * K + k)));
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  if (threadIdx.x == 0) {
    float m = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) m = fmaxf(m, red[w]);
    int ex = 0;
    if (m > 0.f) frexpf(m, &ex);
    e_row = m > 0.f ? ex - 15 : 0;
    if (qchk(BS_REPACK_DST, n, gridDim.x)) row_exp[n] = e_row;
  }
  __syncthreads();
  const float sc = exp2i(-e_row);
  for (int k = threadIdx.x; k < ldw; k += blockDim.x) {
    float v = 0.f;
    if (n < N && k < K && qchk_span(BS_REPACK_SRC, ((long long)n * K + k) / qk * ts, ts, raw_bytes))
      v = __fmul_rn(gguf_value(raw, qtype, (long long)n * K + k), sc);
    if (qchk(BS_REPACK_DST, (long long)n * ldw + k, out_elems)) out[(size_t)n * ldw + k] = __float2half_rn(v);
  }
}

void launch_gguf_straddle_repack(const uint8_t* raw, int qtype, int N, int K, int n_pad, int ldw, void* out,
                                 size_t out_bytes, int32_t* row_exp, cudaStream_t s) {
  if (n_pad == 0) return;
  gguf_straddle_repack_kernel<<<n_pad, 256, 0, s>>>(raw, qtype, N, K, ldw, reinterpret_cast<__half*>(out), row_exp,
                                                    (long long)(out_bytes / 2));
}

void launch_gguf_dequant(const uint8_t* raw, int qtype, long long total, void* out, int out_dtype, cudaStream_t s) {
  if (total == 0) return;
  const long long threads = (total + 3) / 4;
  gguf_dequant_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(raw, qtype, total, out, out_dtype);
}

void launch_gguf_row_exp(const uint8_t* raw, int qtype, int N, int K, int n_pad, int32_t* row_exp, cudaStream_t s) {
  if (n_pad == 0) return;
  gguf_row_exp_kernel<<<(n_pad + 7) / 8, 256, 0, s>>>(raw, qtype, N, K, n_pad, row_exp);
}

void launch_gguf_repack(const uint8_t* raw, int qtype, int N, int K, int num_k_stages, int n_tiles, uint8_t* out,
                        size_t out_bytes, uint32_t stage_bytes, int P, int S, cudaStream_t s) {
  if (num_k_stages == 0 || n_tiles == 0) return;
  dim3 grid(num_k_stages, n_tiles);
  gguf_repack_kernel<<<grid, 128, 0, s>>>(raw, qtype, N, K, num_k_stages, out, stage_bytes, P, S, (long long)out_bytes);
}

void launch_splitk_finalize(const float* partial, int splits, int M, int N, int Mp, const void* col_scale,
                            int cs_kind, const int32_t* w_row_exp, const int32_t* x_row_exp,
                            const float* x_row_scale, const void* bias, int bias_kind, void* y, int y_dtype,
                            long long ldy, cudaStream_t s, const PeerOut* out, int lora, size_t partial_bytes) {
  if (M == 0 || N == 0) return;
  PeerOut po{};
  bool aligned = ldy % 8 == 0 && (reinterpret_cast<uintptr_t>(y) & 15) == 0;
  if (out != nullptr) {
    po = *out;
    po.wait = 0;  // the GEMM that produced the partials waited
    for (int d = 0; d < po.ndst && d < kMaxPeers; ++d) aligned = aligned && (reinterpret_cast<uintptr_t>(po.dst[d]) & 15) == 0;
  }
  const long long lim = partial_bytes ? (long long)(partial_bytes / sizeof(float)) : (long long)splits * N * Mp;
  const int tt = M <= 16 ? 16 : M <= 32 ? 32 : 64;
  auto kern = tt == 16 ? splitk_finalize_kernel<16> : tt == 32 ? splitk_finalize_kernel<32> : splitk_finalize_kernel<64>;
  kern<<<dim3((M + tt - 1) / tt, (N + 63) / 64), 256, 0, s>>>(partial, splits, M, N, Mp, col_scale, cs_kind, w_row_exp,
                                                              x_row_exp, x_row_scale, bias, bias_kind, y, y_dtype, ldy,
                                                              po, lora, lim, aligned ? 1 : 0);
}

void launch_kitchen_grid(const uint8_t* q, const uint8_t* s_rel, const float* codebook, int bits, int group, int N,
                         int K, int8_t* out, cudaStream_t s) {
  if (K % 32 == 0 && (group == 16 || group % 32 == 0) && (bits == 4 || (K * 3 / 4) % 8 == 0) &&
      (long long)N * (K / 32) < (1ll << 31)) {
    const long long threads = (long long)N * (K / 32);
    if (threads == 0) return;
    const unsigned blocks = (unsigned)((threads + 255) / 256);
    if (bits == 4) {
      if (codebook) kitchen_grid32_kernel<4, true><<<blocks, 256, 0, s>>>(q, s_rel, codebook, group, N, K, out);
      else kitchen_grid32_kernel<4, false><<<blocks, 256, 0, s>>>(q, s_rel, codebook, group, N, K, out);
    } else {
      if (codebook) kitchen_grid32_kernel<6, true><<<blocks, 256, 0, s>>>(q, s_rel, codebook, group, N, K, out);
      else kitchen_grid32_kernel<6, false><<<blocks, 256, 0, s>>>(q, s_rel, codebook, group, N, K, out);
    }
    return;
  }
  const long long threads = (long long)N * (K / 16);
  if (threads == 0) return;
  kitchen_grid_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(q, s_rel, codebook, bits, group, N, K, out);
}

void launch_lora_operands(const void* t, int t_dtype, long long ldt, int M, const void* up, int up_dtype,
                          long long ldu, int N, int n_pad, int R, int rk, float scale, const void* cs, int cs_kind,
                          const int32_t* w_row_exp, const int32_t* x_row_exp, void* t_out, void* u_out,
                          cudaStream_t s) {
  const long long nt = (long long)M * rk, nu = (long long)n_pad * rk;
  if (nt > 0)
    lora_t_kernel<<<(unsigned)((nt + 255) / 256), 256, 0, s>>>(t, t_dtype, ldt, M, R, rk, x_row_exp,
                                                               reinterpret_cast<__nv_bfloat16*>(t_out));
  if (nu > 0)
    lora_u_kernel<<<(unsigned)((nu + 255) / 256), 256, 0, s>>>(up, up_dtype, ldu, N, n_pad, R, rk, scale, cs, cs_kind,
                                                               w_row_exp, reinterpret_cast<__nv_bfloat16*>(u_out));
}


// ---------------------------------------------------------------------------------------------
// Input gradient of the weight-only INT8 linear for a frozen weight (comfy-kitchen's
// int8_linear_grad_input): dX = dY . W with W = (q * s) un-rotated per block, W = W_rot . H (H the
// symmetric block Hadamard of the forward).  The contraction runs along N, so the GEMM reads a
// transposed copy of q made once; the per-channel scale s moves onto dY's columns.
// ---------------------------------------------------------------------------------------------

// q int8 [N, K] -> qt int8 [K, ldt] (ldt a multiple of 64 >= N, zeros in columns N .. ldt-1).
// grid = (ceil(K / 64), ldt / 64), block = 256: a 64 x 64 byte tile through shared memory.
__global__ void __launch_bounds__(256) int8_transpose_kernel(const int8_t* __restrict__ q, int N, int K,
                                                             int8_t* __restrict__ qt, int ldt) {
  __shared__ uint8_t tile[64][65];  // [n][k]
  const int k0 = blockIdx.x * 64, n0 = blockIdx.y * 64;
  const int t = threadIdx.x;
  {
    const int r = t >> 2, c = (t & 3) * 16;
    const int n = n0 + r;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int k = k0 + c + i;
      tile[r][c + i] = (n < N && k < K && qchk(BS_GRAD, (long long)n * K + k, (long long)N * K))
                           ? (uint8_t)q[(size_t)n * K + k] : 0;
    }
  }
  __syncthreads();
  const int r = t >> 2, c = (t & 3) * 16;  // output row k0 + r, columns n0 + c .. + 15
  const int k = k0 + r;
  if (k >= K) return;
  uint32_t w[4];
#pragma unroll
  for (int j = 0; j < 4; ++j)
    w[j] = (uint32_t)tile[c + 4 * j][r] | ((uint32_t)tile[c + 4 * j + 1][r] << 8) |
           ((uint32_t)tile[c + 4 * j + 2][r] << 16) | ((uint32_t)tile[c + 4 * j + 3][r] << 24);
  if (qchk_span(BS_GRAD, (long long)k * ldt + n0 + c, 16, (long long)K * ldt))
    *reinterpret_cast<uint4*>(qt + (size_t)k * ldt + n0 + c) = make_uint4(w[0], w[1], w[2], w[3]);
}

// dY' = dY * s per column, normalized per row like the forward's activation operand: a power of
// two 2^f from the row's largest |dY * s| (f = exponent - 15), one rounding to fp16, zeros in
// columns N .. Np-1.  One CTA per row; the second pass rereads the row (mostly from L2).
__global__ void __launch_bounds__(256) grad_prologue_kernel(const void* __restrict__ dy, int dy_dtype, long long lddy,
                                                            int N, int Np, const void* __restrict__ s, int s_f16,
                                                            __half* __restrict__ out, int32_t* __restrict__ row_exp) {
  __shared__ float red[33];
  const int row = blockIdx.x;
  const long long lim_dy = (long long)(gridDim.x - 1) * lddy + N;  // one CTA per row of dY [M, lddy]
  auto value = [&](int c) {
    if (!qchk(BS_GRAD, c, N) || !qchk(BS_GRAD, (long long)row * lddy + c, lim_dy)) return 0.f;
    const float sc = s_f16 ? __half2float(reinterpret_cast<const __half*>(s)[c]) : reinterpret_cast<const float*>(s)[c];
    return __fmul_rn(load_x(dy, dy_dtype, (long long)row * lddy + c), sc);
  };
  float amax = 0.f;
  for (int c = threadIdx.x; c < N; c += blockDim.x) amax = fmaxf(amax, fabsf(value(c)));
  amax = block_max(amax, red);
  int f = 0;
  if (amax > 0.f && amax <= 3.402823466e38f) {
    int ex;
    frexpf(amax, &ex);
    f = ex - 15;
  }
  if (threadIdx.x == 0) row_exp[row] = f;
  __half* o = out + (long long)row * Np;
  for (int c = 2 * threadIdx.x; c < Np; c += 2 * blockDim.x) {
    const float v0 = c < N ? scale_pow2(value(c), f) : 0.f;
    const float v1 = c + 1 < N ? scale_pow2(value(c + 1), f) : 0.f;
    if (qchk_span(BS_GRAD, (long long)row * Np + c, 2, (long long)gridDim.x * Np))
      *reinterpret_cast<__half2*>(o + c) = __floats2half2_rn(v0, v1);
  }
}

// 8 consecutive values of a 16-byte aligned row (f16 / bf16 / f32) as floats.
__device__ __forceinline__ void load8(const void* base, int dtype, long long idx, float (&v)[8]) {
  if (dtype == 0) {
    const float4 a = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + idx);
    const float4 b = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + idx + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    return;
  }
  const uint4 w = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(base) + idx);
  const uint32_t p[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const unsigned short lo = (unsigned short)(p[e] & 0xFFFF), hi = (unsigned short)(p[e] >> 16);
    v[2 * e] = dtype == 1 ? __half2float(__ushort_as_half(lo)) : __bfloat162float(__ushort_as_bfloat16(lo));
    v[2 * e + 1] = dtype == 1 ? __half2float(__ushort_as_half(hi)) : __bfloat162float(__ushort_as_bfloat16(hi));
  }
}

// The same operand with 16-byte loads and stores: each thread keeps CH chunks of 8 columns in
// registers between the max pass and the write pass, so dY is read once; 16-bit inputs are kept
// as loaded (4 registers a chunk) and the products dY * s recomputed in the write pass, the same
// fp32 products as in the max pass.  Needs N % 8 == 0, 16-byte aligned rows of dy and s, and
// CH * blockDim.x * 8 >= Np.
template <int CH, bool F32>
__global__ void __launch_bounds__(512) grad_prologue_vec_kernel(const void* __restrict__ dy, int dy_dtype,
                                                                long long lddy, int N, int Np,
                                                                const void* __restrict__ s, int s_f16,
                                                                __half* __restrict__ out, int32_t* __restrict__ row_exp) {
  __shared__ float red[33];
  const int row = blockIdx.x;
  constexpr int W = F32 ? 8 : 4;  // registers a chunk
  uint32_t raw[CH][W];
  auto products = [&](int j, int c, float (&v)[8]) {
    if constexpr (F32) {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = __uint_as_float(raw[j][e]);
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const unsigned short lo = (unsigned short)(raw[j][e] & 0xFFFF), hi = (unsigned short)(raw[j][e] >> 16);
        v[2 * e] = dy_dtype == 1 ? __half2float(__ushort_as_half(lo)) : __bfloat162float(__ushort_as_bfloat16(lo));
        v[2 * e + 1] = dy_dtype == 1 ? __half2float(__ushort_as_half(hi)) : __bfloat162float(__ushort_as_bfloat16(hi));
      }
    }
    float sc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (qchk_span(BS_GRAD, c, 8, N)) load8(s, s_f16 ? 1 : 0, c, sc);
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = __fmul_rn(v[e], sc[e]);
  };
  float amax = 0.f;
#pragma unroll
  for (int j = 0; j < CH; ++j) {
    const int c = (j * (int)blockDim.x + (int)threadIdx.x) * 8;
    if (c < N && qchk_span(BS_GRAD, (long long)row * lddy + c, 8, (long long)(gridDim.x - 1) * lddy + N)) {
      if constexpr (F32) {
        const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const float*>(dy) + (long long)row * lddy + c);
        const uint4 a = src[0], b = src[1];
        raw[j][0] = a.x; raw[j][1] = a.y; raw[j][2] = a.z; raw[j][3] = a.w;
        raw[j][4] = b.x; raw[j][5] = b.y; raw[j][6] = b.z; raw[j][7] = b.w;
      } else {
        const uint4 a = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(dy) + (long long)row * lddy + c);
        raw[j][0] = a.x; raw[j][1] = a.y; raw[j][2] = a.z; raw[j][3] = a.w;
      }
      float v[8];
      products(j, c, v);
#pragma unroll
      for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(v[e]));
    }
  }
  amax = block_max(amax, red);
  int f = 0;
  if (amax > 0.f && amax <= 3.402823466e38f) {
    int ex;
    frexpf(amax, &ex);
    f = ex - 15;
  }
  if (threadIdx.x == 0) row_exp[row] = f;
#pragma unroll
  for (int j = 0; j < CH; ++j) {
    const int c = (j * (int)blockDim.x + (int)threadIdx.x) * 8;
    if (c < Np) {
      float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      if (c < N) products(j, c, v);
      uint4 pk;
      uint32_t* pw = reinterpret_cast<uint32_t*>(&pk);
#pragma unroll
      for (int e = 0; e < 4; ++e) pw[e] = pack_f16x2(scale_pow2(v[2 * e], f), scale_pow2(v[2 * e + 1], f));
      if (qchk_span(BS_GRAD, (long long)row * Np + c, 8, (long long)gridDim.x * Np))
        *reinterpret_cast<uint4*>(out + (long long)row * Np + c) = pk;
    }
  }
}

// Rows of dX (fp32 [M, K]) times the block Hadamard, written in the output dtype: each warp
// rotates R blocks of G = 32 * E values (all loads issued before the butterflies), lane l holding
// values l*E .. l*E+E-1 of a block.  `vec`: 16-byte aligned output rows, stored as whole vectors.
template <int E, int R>
__global__ void __launch_bounds__(256) grad_rotate_kernel(const float* __restrict__ in, int M, int K, int kind,
                                                          void* __restrict__ out, int out_dtype, long long ldo,
                                                          int vec) {
  constexpr int G = 32 * E;
  const int nblk = K / G;
  const long long total = (long long)M * nblk;
  const long long w0 = ((long long)blockIdx.x * 8 + (threadIdx.x >> 5)) * R;
  const int lane = threadIdx.x & 31;
  if (w0 >= total) return;  // uniform per warp
  float v[R][E];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const long long wg = w0 + r;
    if (wg < total && qchk_span(BS_GRAD, (wg / nblk) * K + (wg % nblk) * G + lane * E, E, (long long)M * K)) {
      const float* src = in + (size_t)(wg / nblk) * K + (int)(wg % nblk) * G + lane * E;
      if constexpr (E >= 4) {
#pragma unroll
        for (int e = 0; e < E; e += 4) {
          const float4 t = *reinterpret_cast<const float4*>(src + e);
          v[r][e] = t.x; v[r][e + 1] = t.y; v[r][e + 2] = t.z; v[r][e + 3] = t.w;
        }
      } else {
#pragma unroll
        for (int e = 0; e < E; ++e) v[r][e] = src[e];
      }
    } else {
#pragma unroll
      for (int e = 0; e < E; ++e) v[r][e] = 0.f;
    }
  }
#pragma unroll
  for (int r = 0; r < R; ++r) block_hadamard<E>(v[r], kind, lane);  // every lane joins the shuffles
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const long long wg = w0 + r;
    if (wg >= total) break;
    const long long o = (long long)(wg / nblk) * ldo + (int)(wg % nblk) * G + lane * E;
    if (!qchk_span(BS_GRAD, o, E, (long long)(M - 1) * ldo + K)) continue;
    bool done = false;
    if constexpr (E >= 4) {
      if (vec && out_dtype != OUT_F32) {
        uint32_t pw[E / 2];
#pragma unroll
        for (int e = 0; e < E / 2; ++e)
          pw[e] = out_dtype == OUT_F16 ? pack_f16x2(v[r][2 * e], v[r][2 * e + 1])
                                       : pack_bf16x2(v[r][2 * e], v[r][2 * e + 1]);
        uint16_t* dst = reinterpret_cast<uint16_t*>(out) + o;
#pragma unroll
        for (int e = 0; e < E / 2; e += 2) *reinterpret_cast<uint2*>(dst + 2 * e) = make_uint2(pw[e], pw[e + 1]);
        done = true;
      } else if (vec) {
        float* dst = reinterpret_cast<float*>(out) + o;
#pragma unroll
        for (int e = 0; e < E; e += 4)
          *reinterpret_cast<float4*>(dst + e) = make_float4(v[r][e], v[r][e + 1], v[r][e + 2], v[r][e + 3]);
        done = true;
      }
    }
    if (!done) {
#pragma unroll
      for (int e = 0; e < E; ++e) {
        if (out_dtype == OUT_F16) reinterpret_cast<__half*>(out)[o + e] = __float2half_rn(v[r][e]);
        else if (out_dtype == OUT_BF16) reinterpret_cast<__nv_bfloat16*>(out)[o + e] = __float2bfloat16_rn(v[r][e]);
        else reinterpret_cast<float*>(out)[o + e] = v[r][e];
      }
    }
  }
}

void launch_int8_transpose(const int8_t* q, int N, int K, int8_t* qt, int ldt, cudaStream_t s) {
  if (N == 0 || K == 0) return;
  int8_transpose_kernel<<<dim3((K + 63) / 64, ldt / 64), 256, 0, s>>>(q, N, K, qt, ldt);
}

void launch_grad_prologue(const void* dy, int dy_dtype, long long lddy, int M, int N, int Np, const void* scale,
                          int scale_f16, void* out, int32_t* row_exp, cudaStream_t s) {
  if (M == 0) return;
  const int esz = dy_dtype == 0 ? 4 : 2;
  const bool vec = N % 8 == 0 && ((reinterpret_cast<uintptr_t>(dy) | (uintptr_t)(lddy * esz)) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(scale) & 15) == 0;
  __half* o = reinterpret_cast<__half*>(out);
  if (vec) {
    const int chunks = (Np + 512 * 8 - 1) / (512 * 8);
#define QLIN_GRAD_PRO(CH)                                                                                          \
    if (chunks <= CH) {                                                                                            \
      if (dy_dtype == 0) grad_prologue_vec_kernel<CH, true><<<M, 512, 0, s>>>(dy, dy_dtype, lddy, N, Np, scale, scale_f16, o, row_exp); \
      else grad_prologue_vec_kernel<CH, false><<<M, 512, 0, s>>>(dy, dy_dtype, lddy, N, Np, scale, scale_f16, o, row_exp); \
      return;                                                                                                      \
    }
    QLIN_GRAD_PRO(1)
    QLIN_GRAD_PRO(2)
    QLIN_GRAD_PRO(4)
    QLIN_GRAD_PRO(8)
#undef QLIN_GRAD_PRO
  }
  grad_prologue_kernel<<<M, 256, 0, s>>>(dy, dy_dtype, lddy, N, Np, scale, scale_f16, o, row_exp);
}

int launch_grad_rotate(const float* in, int M, int K, int group, void* out, int out_dtype, long long ldo,
                       cudaStream_t s) {
  if (M == 0 || K == 0) return 0;
  constexpr int R = 4;  // blocks per warp
  const long long warps = ((long long)M * (K / group) + R - 1) / R;
  const unsigned blocks = (unsigned)((warps + 7) / 8);
  const int esz = out_dtype == OUT_F32 ? 4 : 2;
  const int vec = ((reinterpret_cast<uintptr_t>(out) | (uintptr_t)(ldo * esz)) & 15) == 0 ? 1 : 0;
  switch (group) {  // the forward prologue's rotation for each group size
    case 32: grad_rotate_kernel<1, R><<<blocks, 256, 0, s>>>(in, M, K, 0, out, out_dtype, ldo, vec); return 0;
    case 64: grad_rotate_kernel<2, R><<<blocks, 256, 0, s>>>(in, M, K, 1, out, out_dtype, ldo, vec); return 0;
    case 128: grad_rotate_kernel<4, R><<<blocks, 256, 0, s>>>(in, M, K, 0, out, out_dtype, ldo, vec); return 0;
    case 256: grad_rotate_kernel<8, R><<<blocks, 256, 0, s>>>(in, M, K, 1, out, out_dtype, ldo, vec); return 0;
    default: return -1;
  }
}

// This translation unit's bounds record (QLIN_CHECKS build).
QLIN_BOUNDS_READER(bounds_read_aux)

}  // namespace qlin
