// Block-Hadamard rotation of values held across a warp, shared by the activation prologues, the
// input-gradient rotation and the GEMM epilogue that rotates its output rows.
#pragma once

namespace qlin {

// ---------------------------------------------------------------------------------------------
// Block-Hadamard rotation in a warp: a block of G = 32*E values, lane l holding elements
// l*E .. l*E+E-1.  y[p] = sum_i H[p][i] x[i] / sqrt(G) with
//   kind 0: Sylvester H2 (x) ... (x) H2 (H2 = [[1,1],[1,-1]]), any power of two;
//   kind 1: H4 (x) ... (x) H4 with the regular H4 = J - 2*antidiag (the reference's
//           build_hadamard, modal/weight_error_app.py:90-98), powers of four.
// ---------------------------------------------------------------------------------------------
template <int E>
__device__ __forceinline__ float partner(const float (&x)[E], int e, int mask) {
  constexpr int LE = (E == 1) ? 0 : (E == 2) ? 1 : (E == 4) ? 2 : 3;
  const int rm = mask & (E - 1);
  const int lm = mask >> LE;
  float v = x[e ^ rm];
  if (lm) v = __shfl_xor_sync(0xffffffffu, v, lm);
  return v;
}

template <int E>
__device__ __forceinline__ void block_hadamard(float (&x)[E], int kind, int lane) {
  constexpr int LE = (E == 1) ? 0 : (E == 2) ? 1 : (E == 4) ? 2 : 3;
  constexpr int LG = LE + 5;
  if (kind == 0) {
#pragma unroll
    for (int t = 0; t < LG; ++t) {
      float y[E];
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const int i = lane * E + e;
        const float p = partner<E>(x, e, 1 << t);
        y[e] = (i >> t) & 1 ? __fsub_rn(p, x[e]) : __fadd_rn(x[e], p);
      }
#pragma unroll
      for (int e = 0; e < E; ++e) x[e] = y[e];
    }
  } else {
#pragma unroll
    for (int t = 0; t < LG / 2; ++t) {
      float y[E];
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const float p1 = partner<E>(x, e, 1 << (2 * t));
        const float p2 = partner<E>(x, e, 2 << (2 * t));
        const float p3 = partner<E>(x, e, 3 << (2 * t));
        const float s = __fadd_rn(__fadd_rn(x[e], p1), __fadd_rn(p2, p3));
        y[e] = __fsub_rn(s, __fmul_rn(2.f, p3));
      }
#pragma unroll
      for (int e = 0; e < E; ++e) x[e] = y[e];
    }
  }
  const float norm = (E == 1) ? 0.17677669529663687f : (E == 2) ? 0.125f : (E == 4) ? 0.08838834764831845f : 0.0625f;
#pragma unroll
  for (int e = 0; e < E; ++e) x[e] = __fmul_rn(x[e], norm);
}

// Sylvester butterflies over 2^LG values held four per lane, for R independent rows at once
// (stage by stage, so the rows' shuffle chains overlap); both the sum and the difference are
// formed and one is selected by the element's bit t, so a lane-dependent choice never becomes a
// divergent branch.
template <int R, int LG>
__device__ __forceinline__ void sylvester_rows4(float (&x)[R][4], int lane) {
#pragma unroll
  for (int t = 0; t < LG; ++t) {
    float y[R][4];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float p = partner<4>(x[r], e, 1 << t);
        const float a = __fadd_rn(x[r][e], p), b = __fsub_rn(p, x[r][e]);
        y[r][e] = (((lane * 4 + e) >> t) & 1) ? b : a;
      }
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int e = 0; e < 4; ++e) x[r][e] = y[r][e];
  }
}

// The H4 Kronecker power over blocks of 64 values held four per lane (base-4 digits 0, 1, 2),
// R rows at once.
template <int R>
__device__ __forceinline__ void h4_rows4_64(float (&x)[R][4]) {
#pragma unroll
  for (int t = 0; t < 3; ++t) {
    float y[R][4];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float p1 = partner<4>(x[r], e, 1 << (2 * t));
        const float p2 = partner<4>(x[r], e, 2 << (2 * t));
        const float p3 = partner<4>(x[r], e, 3 << (2 * t));
        const float s = __fadd_rn(__fadd_rn(x[r][e], p1), __fadd_rn(p2, p3));
        y[r][e] = __fsub_rn(s, __fmul_rn(2.f, p3));
      }
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int e = 0; e < 4; ++e) x[r][e] = y[r][e];
  }
}

// R rows of 128 values, each held four per lane (lane l: elements 4l .. 4l+3), rotated in blocks
// of G = 32 / 128 (Sylvester) or 64 (the H4 Kronecker power), the forward prologue's matrices for
// those sizes.  The butterfly stages run in the same order and with the same operations as
// block_hadamard's, so each block's result is the same, value for value, as block_hadamard over
// that block.
template <int R>
__device__ __forceinline__ void rows_hadamard4(float (&x)[R][4], int G, int lane) {
  if (G == 128) sylvester_rows4<R, 7>(x, lane);
  else if (G == 64) h4_rows4_64<R>(x);
  else sylvester_rows4<R, 5>(x, lane);
  const float norm = G == 128 ? 0.08838834764831845f : G == 64 ? 0.125f : 0.17677669529663687f;
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int e = 0; e < 4; ++e) x[r][e] = __fmul_rn(x[r][e], norm);
}

}  // namespace qlin
