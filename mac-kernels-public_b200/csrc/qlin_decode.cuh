// Per-format weight decoders.  Each decoder turns one pipeline stage of packed weights in
// shared memory into the tensor-core A operand for one weight row (one TMEM lane):
//   * f16 family (kind::f16): 64 K-values -> 32 words of packed fp16 pairs (even k in the low half)
//   * i8 family (kind::i8):  128 K-values -> 32 words of packed int8 quads (k%4 = byte index)
//
// Stage layouts in shared memory (and, for repacked formats, in global memory):
//   INT8 (raw [N,K] int8 via a 2-D TMA box {64 B, 128 rows}, 64-byte swizzle):
//     row r, 16-byte chunk j at r*64 + 16*(j ^ ((r >> 1) & 3)).
//   Repacked GGUF stage ("plane" layout): P chunks of 16 bytes per row stored chunk-major,
//     [P][128 rows][16 B], followed by a side record of S bytes per row, [128 rows][S B].
//     Q8_0   P=4 (qs of two blocks)                     S=4 (d0, d1 fp16)
//     Q4_0   P=2 (qs of two blocks, ggml nibble order)   S=4 (d0, d1 fp16)
//     IQ4_NL P=2 (two runs of 32 in "selector order": word t of a run holds the nibbles of values
//            4t..4t+3 in bits 0-15 and 16+4t..16+4t+3 in bits 16-31, value 4t+k in nibble k;
//            each code with its bits 2 and 3 swapped)
//                                                       S=4 (d0, d1 fp16)
//     Q4_K   P=2 (the 32-byte qs chunk of sub-blocks 2c, 2c+1)  S=8 (d, dmin fp16, sc0, sc1, m0, m1 u8)
//     Q6_K   P=4 (one byte per value: the unsigned 6-bit code)  S=8 (sc0..sc3 int8, d fp16, pad)
//     Q4_1   P=2 (qs of two blocks)                     S=8 (d0, m0, d1, m1 fp16)
//     Q5_0   P=2 (qs of two blocks)                     S=12 (d0, d1 fp16, H0, H1)
//     Q5_1   P=2 (qs of two blocks)                     S=16 (d0, m0, d1, m1 fp16, H0, H1)
//     Q2_K   P=1 (2-bit codes: word u, byte b, bits 2s..2s+1 = value 16u+4s+b)
//                                                       S=8 (d, dmin fp16, the 4 scale bytes)
//     Q3_K   P=1 (low 2 bits, as Q2_K)                  S=16 (d fp16, 4 int8 scales sc-32, pad 2,
//                                                              H0, H1: the hmask bits)
//     Q5_K   P=2 (as Q4_K)                              S=16 (d, dmin fp16, sc0, sc1, m0, m1, H0, H1)
//     IQ4_XS P=2 (sub-blocks 2c, 2c+1, selector order as IQ4_NL)  S=4 (d fp16, 2 int8 scales sc-32)
//   "H" words carry one extra bit per value, transposed so that one shift and one mask place the
//   bits of four consecutive values (4g .. 4g+3, g = 0..7 within the word) at the same bit of
//   four bytes: bit 8b + g of H is the bit of value 4g + b.
//   W4 nibbles (raw [N,K/2] via TMA box {64 B, 128 rows}, 64-byte swizzle): 128 values per stage.
//   W6 planar (kitchen layout): low-nibble plane box {64 B, 128 rows} followed by the 2-bit plane
//     box {32 B, 128 rows}, both 64-/32-byte swizzled.
//
// GGUF values are computed in fp32 in the operation order of gguf-py 0.19.0 (bit-exact), then
// scaled by the row's power of two 2^-e (exact) and rounded once to fp16.
#pragma once
#include "qlin_ptx.cuh"

namespace qlin {

enum GgufType : int {
  GGUF_Q4_0 = 2, GGUF_Q4_1 = 3, GGUF_Q5_0 = 6, GGUF_Q5_1 = 7, GGUF_Q8_0 = 8, GGUF_Q2_K = 10, GGUF_Q3_K = 11,
  GGUF_Q4_K = 12, GGUF_Q5_K = 13, GGUF_Q6_K = 14, GGUF_IQ4_NL = 20, GGUF_IQ4_XS = 23
};

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

// Four signed bytes -> two words of packed fp16 pairs, exactly: 0x64XX is the fp16 1024 + XX,
// so (byte ^ 0x80) placed under 0x64 and minus 1152 is the signed value.
__device__ __forceinline__ void s8x4_to_f16x4(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t u = w ^ 0x80808080u;
  const uint32_t a = prmt(u, 0x64646464u, 0x5140u);
  const uint32_t b = prmt(u, 0x64646464u, 0x7362u);
  const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));
  __half2 ha = __hsub2(*reinterpret_cast<const __half2*>(&a), bias);
  __half2 hb = __hsub2(*reinterpret_cast<const __half2*>(&b), bias);
  lo = *reinterpret_cast<uint32_t*>(&ha);
  hi = *reinterpret_cast<uint32_t*>(&hb);
}

__device__ __forceinline__ uint32_t pack_f16x2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);  // a -> low half
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);  // a -> low half
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ float exp2i(int e) {  // 2^e for -126 <= e <= 127
  return __int_as_float((e + 127) << 23);
}

// With a fused LoRA the accumulator holds base + LoRA / colscale, so a column scale of (nearly)
// zero is raised to +-2^-100: the base term still vanishes in the output and the LoRA term stays
// finite (the LoRA operand is divided by the same raised scale).
__device__ __forceinline__ float lora_safe_scale(float cs) {
  return fabsf(cs) >= 7.888609052210118e-31f ? cs : copysignf(7.888609052210118e-31f, cs);
}

__device__ __forceinline__ float half_bits_to_float(uint32_t bits16) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16 & 0xFFFF)));
}

// ---------------------------------------------------------------------------------------------
// f16 family (64 values per stage)
// ---------------------------------------------------------------------------------------------
struct DecInt8 {
  static constexpr int kP = 4;  // informational: 64 bytes per row
  static constexpr uint32_t kStageBytes = 128 * 64;
  static constexpr bool kTma = true;
  __device__ __forceinline__ static void decode(const uint8_t* st, int r, float /*row_scale*/, uint32_t (&out)[32]) {
    const uint8_t* row = st + r * 64;
    const int sw = (r >> 1) & 3;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint4 v = *reinterpret_cast<const uint4*>(row + ((j ^ sw) << 4));
      s8x4_to_f16x4(v.x, out[8 * j + 0], out[8 * j + 1]);
      s8x4_to_f16x4(v.y, out[8 * j + 2], out[8 * j + 3]);
      s8x4_to_f16x4(v.z, out[8 * j + 4], out[8 * j + 5]);
      s8x4_to_f16x4(v.w, out[8 * j + 6], out[8 * j + 7]);
    }
  }
};

// Plain fp16 weights (the LoRA down factor after the activation prologue, and GGUF rows that
// straddle blocks after their one-time decode to w * 2^-e): [N, ldw] row-major via a TMA box
// {64 values, 128 rows} with 128-byte swizzle, so 16-byte chunk j of row r sits at
// r * 128 + 16 * (j ^ (r & 7)).  The values are the operand already: the decode is a copy.
struct DecF16 {
  static constexpr uint32_t kStageBytes = 128 * 128;
  static constexpr bool kTma = true;
  __device__ __forceinline__ static void decode(const uint8_t* st, int r, float /*row_scale*/, uint32_t (&out)[32]) {
    const uint8_t* row = st + r * 128;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint4 v = *reinterpret_cast<const uint4*>(row + ((j ^ (r & 7)) << 4));
      out[4 * j] = v.x;
      out[4 * j + 1] = v.y;
      out[4 * j + 2] = v.z;
      out[4 * j + 3] = v.w;
    }
  }
};

template <int P, int S>
struct PlaneStage {
  static constexpr uint32_t kStageBytes = 128 * (16 * P + S);
  __device__ __forceinline__ static uint4 chunk(const uint8_t* st, int j, int r) {
    return *reinterpret_cast<const uint4*>(st + (j * 128 + r) * 16);
  }
  __device__ __forceinline__ static const uint8_t* side(const uint8_t* st, int r) {
    return st + 128 * 16 * P + r * S;
  }
};

// Scale d * 2^-e as an fp16 pair.  Exact whenever d * 2^-e is a normal fp16 (the row exponent
// puts the row's largest |w| in [2^14, 2^15), so only blocks more than ~2^22 smaller than the
// row's largest can fall below the normal range).
__device__ __forceinline__ __half2 scale_pair(uint32_t d_bits, float rscale) {
  const __half h = __float2half_rn(__fmul_rn(half_bits_to_float(d_bits), rscale));
  return __halves2half2(h, h);
}

__device__ __forceinline__ uint32_t hmul2_u32(uint32_t a, __half2 d) {
  __half2 r = __hmul2(*reinterpret_cast<const __half2*>(&a), d);
  return *reinterpret_cast<uint32_t*>(&r);
}

// Four unsigned bytes b (0..255) -> (b0 - off, b1 - off) and (b2 - off, b3 - off) as exact fp16
// pairs, off in 0..1024: 0x64XX is the fp16 1024 + XX.
__device__ __forceinline__ void u8x4_to_f16x4(uint32_t u, uint32_t bias_pair, uint32_t& lo, uint32_t& hi) {
  const uint32_t a = prmt(u, 0x64646464u, 0x5140u);
  const uint32_t b = prmt(u, 0x64646464u, 0x7362u);
  const __half2 bias = *reinterpret_cast<const __half2*>(&bias_pair);
  __half2 ha = __hsub2(*reinterpret_cast<const __half2*>(&a), bias);
  __half2 hb = __hsub2(*reinterpret_cast<const __half2*>(&b), bias);
  lo = *reinterpret_cast<uint32_t*>(&ha);
  hi = *reinterpret_cast<uint32_t*>(&hb);
}

// Q8_0: w = q * d.  int8 -> fp16 exactly, then one correctly rounded fp16 multiply by d * 2^-e:
// RN16(q * d * 2^-e), the same single rounding as the fp32 decode followed by the fp16 cast.
struct DecQ8_0 : PlaneStage<4, 4> {
  static constexpr bool kTma = false;
  __device__ __forceinline__ static void decode(const uint8_t* st, int r, float rscale, uint32_t (&out)[32]) {
    const uint32_t dd = *reinterpret_cast<const uint32_t*>(side(st, r));
    const __half2 d0 = scale_pair(dd & 0xFFFF, rscale), d1 = scale_pair(dd >> 16, rscale);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint4 v = chunk(st, j, r);
      const __half2 d = j < 2 ? d0 : d1;
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        uint32_t lo, hi;
        s8x4_to_f16x4(w[t], lo, hi);
        out[8 * j + 2 * t + 0] = hmul2_u32(lo, d);
        out[8 * j + 2 * t + 1] = hmul2_u32(hi, d);
      }
    }
  }
};

// Packed fp16 arithmetic on words holding two fp16 values.
__device__ __forceinline__ uint32_t hsub2_u32(uint32_t a, uint32_t b) {
  __half2 r = __hsub2(*reinterpret_cast<const __half2*>(&a), *reinterpret_cast<const __half2*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}
__device__ __forceinline__ uint32_t hfma2_u32(uint32_t a, __half2 s, __half2 c) {
  __half2 r = __hfma2(*reinterpret_cast<const __half2*>(&a), s, c);
  return *reinterpret_cast<uint32_t*>(&r);
}

// Q4_0: block of 32 values, byte i holds value i (low nibble) and value i+16 (high); value =
// nib - 8 (exact fp16 via the magic number with offset 1032), times the exact fp16 d*2^-e.
struct DecQ4_0 : PlaneStage<2, 4> {
  static constexpr bool kTma = false;
  __device__ __forceinline__ static void decode(const uint8_t* st, int r, float rscale, uint32_t (&out)[32]) {
    const uint32_t dd = *reinterpret_cast<const uint32_t*>(side(st, r));
#pragma unroll
    for (int blk = 0; blk < 2; ++blk) {
      const __half2 d = scale_pair(blk ? (dd >> 16) : (dd & 0xFFFF), rscale);
      const uint4 v = chunk(st, blk, r);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        uint32_t a0, a1, b0, b1;
        u8x4_to_f16x4(w[t] & 0x0F0F0F0Fu, 0x64086408u, a0, a1);         // values 4t..; 1032 = 1024 + 8
        u8x4_to_f16x4((w[t] >> 4) & 0x0F0F0F0Fu, 0x64086408u, b0, b1);  // values 16+4t..
        out[16 * blk + 2 * t + 0] = hmul2_u32(a0, d);
        out[16 * blk + 2 * t + 1] = hmul2_u32(a1, d);
        out[16 * blk + 8 + 2 * t + 0] = hmul2_u32(b0, d);
        out[16 * blk + 8 + 2 * t + 1] = hmul2_u32(b1, d);
      }
    }
  }
};

// The IQ4 non-linear levels (gguf/quants.py:1331) of four 4-bit codes -> two exact fp16 pairs.
// f holds four codes in its nibbles 0-3 ("selector order", written by the repack), each with its
// bits 2 and 3 swapped: stored code s stands for level L(swap(s)).  The levels + 128 as bytes
// (B = L + 128, 1..241) are looked up with two byte permutes:
//   lookup A (selectors s): s < 8 picks A[s] = B(swap(s)); s >= 8 replicates the sign bit of
//     A[s & 7], which is 0 for s = 8..11 and 1 for s = 12..15 (A[0..3] < 128 <= A[4..7]);
//   lookup H (selectors s ^ 8): s >= 8 picks H[s & 7] = B(swap(s)) ^ (that replicated byte);
//     s < 8 replicates the sign bit of H[s], and every H entry is below 128, so 0.
// A ^ H is B(swap(s)) for every s: the swap pairs codes j and j + 8 whose levels have the same
// sign, which is what keeps all of H below 128.  The bytes then go under the 0x64 magic byte:
// (1024 + L + 128) - 1152 = L exactly.
__device__ __forceinline__ void iq4_levels_f16(uint32_t f, uint32_t fx, uint32_t& lo, uint32_t& hi) {
  const uint32_t v = prmt(0x3F2D1801u, 0xA6998D81u, f) ^ prmt(0x766A5D4Fu, 0x0E263A4Au, fx);  // fx = f ^ 0x8888
  const uint32_t bias = 0x64806480u;  // fp16 (1152, 1152)
  lo = hsub2_u32(prmt(v, 0x64646464u, 0x5140u), bias);
  hi = hsub2_u32(prmt(v, 0x64646464u, 0x7362u), bias);
}

// IQ4_NL (one fp16 scale per run of 32, exact: RN16(d*L*2^-e)) and IQ4_XS (sub-block scale
// d*(sc-32) formed in fp32, rounded once to fp16; gguf/quants.py:1352-1377): two runs of 32 per
// stage in selector order, one fp16 multiply per value.
template <bool kXS>
struct DecIQ4 : PlaneStage<2, 4> {
  static constexpr bool kTma = false;
  __device__ __forceinline__ static void decode(const uint8_t* st, int r, float rscale, uint32_t (&out)[32]) {
    const uint32_t sd = *reinterpret_cast<const uint32_t*>(side(st, r));
#pragma unroll
    for (int blk = 0; blk < 2; ++blk) {
      __half2 d;
      if constexpr (kXS) {
        const float dx = __fmul_rn(half_bits_to_float(sd), rscale);
        d = __float2half2_rn(__fmul_rn(dx, (float)(int8_t)((sd >> (16 + 8 * blk)) & 0xFF)));
      } else {
        d = scale_pair(blk ? (sd >> 16) : (sd & 0xFFFF), rscale);
      }
      const uint4 v = chunk(st, blk, r);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        uint32_t a0, a1, b0, b1;
        const uint32_t wx = w[t] ^ 0x88888888u;
        iq4_levels_f16(w[t], wx, a0, a1);              // values 4t .. 4t+3
        iq4_levels_f16(w[t] >> 16, wx >> 16, b0, b1);  // values 16+4t .. 16+4t+3
        out[16 * blk + 2 * t + 0] = hmul2_u32(a0, d);
        out[16 * blk + 2 * t + 1] = hmul2_u32(a1, d);
        out[16 * blk + 8 + 2 * t + 0] = hmul2_u32(b0, d);
        out[16 * blk + 8 + 2 * t + 1] = hmul2_u32(b1, d);
      }
    }
  }
};

// Q4_K: w = (d*sc)*q - dmin*m per 32-value sub-block (gguf/quants.py:504-522), in packed fp16.
// Nibbles become exact fp16 pairs through the 0x64 magic byte (1024 + q, minus 1024); the high
// nibble of a byte is kept in place as 16*q and its scale divided by 16 (exact).  The products
// d*sc*2^-e and dmin*m*2^-e are formed in fp32 and rounded once to fp16, then one fp16 fma per
// value: each weight is within two fp16 rounding steps of the exact dequantized value.
struct DecQ4_K : PlaneStage<2, 8> {
  static constexpr bool kTma = false;
  __device__ __forceinline__ static void decode(const uint8_t* st, int r, float rscale, uint32_t (&out)[32]) {
    const uint2 sd = *reinterpret_cast<const uint2*>(side(st, r));
    const float d = __fmul_rn(half_bits_to_float(sd.x), rscale), dmin = __fmul_rn(half_bits_to_float(sd.x >> 16), rscale);
    const __half2 ds0 = __float2half2_rn(__fmul_rn(d, (float)(sd.y & 0xFF)));
    const __half2 ds1 = __float2half2_rn(__fmul_rn(__fmul_rn(d, (float)((sd.y >> 8) & 0xFF)), 0.0625f));
    const __half2 dm0 = __float2half2_rn(-__fmul_rn(dmin, (float)((sd.y >> 16) & 0xFF)));
    const __half2 dm1 = __float2half2_rn(-__fmul_rn(dmin, (float)(sd.y >> 24)));
    constexpr uint32_t kMagic = 0x64006400u;  // fp16 (1024, 1024)
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const uint4 v = chunk(st, j, r);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        // bytes (0,1) and (2,3) of the word under the magic byte: (1024 + byte) pairs
        const uint32_t a = prmt(w[t], 0x64646464u, 0x5140u), b = prmt(w[t], 0x64646464u, 0x7362u);
        // low nibbles: values 16j+4t.. of sub-block 2c; high nibbles (x16): sub-block 2c+1
        out[8 * j + 2 * t + 0] = hfma2_u32(hsub2_u32(a & 0xFF0FFF0Fu, kMagic), ds0, dm0);
        out[8 * j + 2 * t + 1] = hfma2_u32(hsub2_u32(b & 0xFF0FFF0Fu, kMagic), ds0, dm0);
        out[16 + 8 * j + 2 * t + 0] = hfma2_u32(hsub2_u32(a & 0xFFF0FFF0u, kMagic), ds1, dm1);
        out[16 + 8 * j + 2 * t + 1] = hfma2_u32(hsub2_u32(b & 0xFFF0FFF0u, kMagic), ds1, dm1);
      }
    }
  }
};

// Q6_K: w = (d*sc)*(q-32) per 16 values (gguf/quants.py:552-574).  The repack stores each 6-bit
// code in a byte (1.125 bytes per value with the scales, +37% over the raw blocks, for the decode
// cost of Q8_0): the code goes under the 0x64 magic byte, (1024 + q) - 1056 = q - 32 is exact, and
// one fp16 multiply by d*sc*2^-e (formed in fp32, rounded once to fp16).
struct DecQ6_K : PlaneStage<4, 8> {
  static constexpr bool kTma = false;
  __device__ __forceinline__ static void decode(const uint8_t* st, int r, float rscale, uint32_t (&out)[32]) {
    const uint2 sd = *reinterpret_cast<const uint2*>(side(st, r));
    const float d = __fmul_rn(half_bits_to_float(sd.y), rscale);
    constexpr uint32_t kBias = 0x64206420u;  // fp16 (1056, 1056) = 1024 + 32
#pragma unroll
    for (int j = 0; j < 4; ++j) {  // chunk j = the 16-value group j
      const __half2 ds = __float2half2_rn(__fmul_rn(d, (float)(int8_t)((sd.x >> (8 * j)) & 0xFF)));
      const uint4 v = chunk(st, j, r);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        uint32_t lo, hi;
        u8x4_to_f16x4(w[t], kBias, lo, hi);
        out[8 * j + 2 * t + 0] = hmul2_u32(lo, ds);
        out[8 * j + 2 * t + 1] = hmul2_u32(hi, ds);
      }
    }
  }
};

// The bits of values 4g .. 4g+3 of an H word (bit 8b + g = value 4g + b) moved to bit `kAt` of
// bytes 0..3.
template <int kAt>
__device__ __forceinline__ uint32_t h_bits(uint32_t h, int g) {
  return (g <= kAt ? (h << (kAt - g)) : (h >> (g - kAt))) & (0x01010101u << kAt);
}

// Q4_1: w = d*q + m per 32-value block (gguf/quants.py:275-288).  Nibbles under the magic byte as
// in Q4_K (high nibbles in place, scale divided by 16); d*2^-e and m*2^-e are exact fp16 (normal
// range), so one fp16 fma gives RN16((d*q + m) * 2^-e).
struct DecQ4_1 : PlaneStage<2, 8> {
  static constexpr bool kTma = false;
  __device__ __forceinline__ static void decode(const uint8_t* st, int r, float rscale, uint32_t (&out)[32]) {
    const uint2 sd = *reinterpret_cast<const uint2*>(side(st, r));
    constexpr uint32_t kMagic = 0x64006400u;
#pragma unroll
    for (int blk = 0; blk < 2; ++blk) {
      const uint32_t dm = blk ? sd.y : sd.x;
      const float d = __fmul_rn(half_bits_to_float(dm), rscale);
      const __half2 d0 = __float2half2_rn(d), d1 = __float2half2_rn(__fmul_rn(d, 0.0625f));
      const __half2 m = __float2half2_rn(__fmul_rn(half_bits_to_float(dm >> 16), rscale));
      const uint4 v = chunk(st, blk, r);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const uint32_t a = prmt(w[t], 0x64646464u, 0x5140u), b = prmt(w[t], 0x64646464u, 0x7362u);
        out[16 * blk + 2 * t + 0] = hfma2_u32(hsub2_u32(a & 0xFF0FFF0Fu, kMagic), d0, m);
        out[16 * blk + 2 * t + 1] = hfma2_u32(hsub2_u32(b & 0xFF0FFF0Fu, kMagic), d0, m);
        out[16 * blk + 8 + 2 * t + 0] = hfma2_u32(hsub2_u32(a & 0xFFF0FFF0u, kMagic), d1, m);
        out[16 * blk + 8 + 2 * t + 1] = hfma2_u32(hsub2_u32(b & 0xFFF0FFF0u, kMagic), d1, m);
      }
    }
  }
};

// Q5_0 / Q5_1: the Q4 nibble plus a fifth bit from the block's qh word (gguf/quants.py:313-330,
// 356-375), assembled under the magic byte.  Q5_0: (1024 + q) - 1040 = q - 16 exactly, times the
// exact fp16 d*2^-e: RN16(d*(q-16)*2^-e), bit-exact.  Q5_1: one fp16 fma q*d' + m'.
template <bool kMin>
struct DecQ5Block : PlaneStage<2, kMin ? 16 : 12> {
  using Base = PlaneStage<2, kMin ? 16 : 12>;
  static constexpr bool kTma = false;
  __device__ __forceinline__ static void decode(const uint8_t* st, int r, float rscale, uint32_t (&out)[32]) {
    const uint32_t* sd = reinterpret_cast<const uint32_t*>(Base::side(st, r));
    uint32_t dw[2], hw[2];
    if constexpr (kMin) {
      const uint4 v = *reinterpret_cast<const uint4*>(sd);
      dw[0] = v.x;
      dw[1] = v.y;
      hw[0] = v.z;
      hw[1] = v.w;
    } else {
      dw[0] = sd[0] & 0xFFFF;
      dw[1] = sd[0] >> 16;
      hw[0] = sd[1];
      hw[1] = sd[2];
    }
    const uint32_t bias = kMin ? 0x64006400u : 0x64106410u;  // fp16 1024 / 1040 = 1024 + 16
#pragma unroll
    for (int blk = 0; blk < 2; ++blk) {
      const __half2 d = scale_pair(dw[blk] & 0xFFFF, rscale);
      const __half2 m = kMin ? scale_pair(dw[blk] >> 16, rscale) : __half2{};
      const uint4 v = Base::chunk(st, blk, r);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const uint32_t qlo = (w[t] & 0x0F0F0F0Fu) | h_bits<4>(hw[blk], t);             // values 4t..
        const uint32_t qhi = ((w[t] >> 4) & 0x0F0F0F0Fu) | h_bits<4>(hw[blk], 4 + t);  // 16+4t..
        uint32_t a0, a1, b0, b1;
        u8x4_to_f16x4(qlo, bias, a0, a1);
        u8x4_to_f16x4(qhi, bias, b0, b1);
        if constexpr (kMin) {
          out[16 * blk + 2 * t + 0] = hfma2_u32(a0, d, m);
          out[16 * blk + 2 * t + 1] = hfma2_u32(a1, d, m);
          out[16 * blk + 8 + 2 * t + 0] = hfma2_u32(b0, d, m);
          out[16 * blk + 8 + 2 * t + 1] = hfma2_u32(b1, d, m);
        } else {
          out[16 * blk + 2 * t + 0] = hmul2_u32(a0, d);
          out[16 * blk + 2 * t + 1] = hmul2_u32(a1, d);
          out[16 * blk + 8 + 2 * t + 0] = hmul2_u32(b0, d);
          out[16 * blk + 8 + 2 * t + 1] = hmul2_u32(b1, d);
        }
      }
    }
  }
};

// Q2_K / Q3_K: 2-bit codes, 16-value groups with their own scale (gguf/quants.py:405-428,
// 432-472).  Word u of the code chunk holds the group u (values 16u .. 16u+15); shifting it by 2s
// and masking gives values 16u+4s .. 16u+4s+3, one per byte, under the magic byte.
//   Q2_K: w = (d*sc)*q - dmin*m, scale and min in packed fp16 (each rounded once from fp32), one
//         fp16 fma per value.
//   Q3_K: q = code | hbit<<2, minus 4 (exact), times RN16(d*sc*2^-e): one fp16 multiply.
template <bool kQ3>
struct DecQ23_K : PlaneStage<1, kQ3 ? 16 : 8> {
  using Base = PlaneStage<1, kQ3 ? 16 : 8>;
  static constexpr bool kTma = false;
  __device__ __forceinline__ static void decode(const uint8_t* st, int r, float rscale, uint32_t (&out)[32]) {
    const uint4 v = Base::chunk(st, 0, r);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    constexpr uint32_t kMagic = 0x64006400u;
    if constexpr (kQ3) {
      const uint4 sd = *reinterpret_cast<const uint4*>(Base::side(st, r));
      const float d = __fmul_rn(half_bits_to_float(sd.x), rscale);
      const uint32_t scs = (sd.x >> 16) | (sd.y << 16);  // four int8 scales
      const uint32_t hw[2] = {sd.z, sd.w};
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const __half2 dl = __float2half2_rn(__fmul_rn(d, (float)(int8_t)((scs >> (8 * u)) & 0xFF)));
#pragma unroll
        for (int s = 0; s < 4; ++s) {
          const int g = 4 * u + s;
          const uint32_t x = ((w[u] >> (2 * s)) & 0x03030303u) | h_bits<2>(hw[g >> 3], g & 7);
          uint32_t a0, a1;
          u8x4_to_f16x4(x, 0x64046404u, a0, a1);  // fp16 1028 = 1024 + 4
          out[8 * u + 2 * s + 0] = hmul2_u32(a0, dl);
          out[8 * u + 2 * s + 1] = hmul2_u32(a1, dl);
        }
      }
    } else {
      const uint2 sd = *reinterpret_cast<const uint2*>(Base::side(st, r));
      const float d = __fmul_rn(half_bits_to_float(sd.x), rscale);
      const float dmin = __fmul_rn(half_bits_to_float(sd.x >> 16), rscale);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const uint32_t sc = (sd.y >> (8 * u)) & 0xFF;
        const __half2 dl = __float2half2_rn(__fmul_rn(d, (float)(sc & 0xF)));
        const __half2 ml = __float2half2_rn(-__fmul_rn(dmin, (float)(sc >> 4)));
#pragma unroll
        for (int s = 0; s < 4; ++s) {
          const uint32_t x = (w[u] >> (2 * s)) & 0x03030303u;
          const uint32_t a = prmt(x, 0x64646464u, 0x5140u), b = prmt(x, 0x64646464u, 0x7362u);
          out[8 * u + 2 * s + 0] = hfma2_u32(hsub2_u32(a, kMagic), dl, ml);
          out[8 * u + 2 * s + 1] = hfma2_u32(hsub2_u32(b, kMagic), dl, ml);
        }
      }
    }
  }
};

// Q5_K: Q4_K with a fifth bit per value (gguf/quants.py:526-549).  The 5-bit code is assembled
// under the magic byte (the high nibble shifted down, the H bit ORed in at bit 4), then one fp16
// fma with the fp16-rounded d*sc*2^-e and -dmin*m*2^-e, as for Q4_K.
struct DecQ5_K : PlaneStage<2, 16> {
  static constexpr bool kTma = false;
  __device__ __forceinline__ static void decode(const uint8_t* st, int r, float rscale, uint32_t (&out)[32]) {
    const uint4 sd = *reinterpret_cast<const uint4*>(side(st, r));
    const float d = __fmul_rn(half_bits_to_float(sd.x), rscale), dmin = __fmul_rn(half_bits_to_float(sd.x >> 16), rscale);
    const __half2 ds0 = __float2half2_rn(__fmul_rn(d, (float)(sd.y & 0xFF)));
    const __half2 ds1 = __float2half2_rn(__fmul_rn(d, (float)((sd.y >> 8) & 0xFF)));
    const __half2 dm0 = __float2half2_rn(-__fmul_rn(dmin, (float)((sd.y >> 16) & 0xFF)));
    const __half2 dm1 = __float2half2_rn(-__fmul_rn(dmin, (float)(sd.y >> 24)));
    constexpr uint32_t kMagic = 0x64006400u;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const uint4 v = chunk(st, j, r);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const uint32_t qlo = (w[t] & 0x0F0F0F0Fu) | h_bits<4>(sd.z, 4 * j + t);         // values 16j+4t..
        const uint32_t qhi = ((w[t] >> 4) & 0x0F0F0F0Fu) | h_bits<4>(sd.w, 4 * j + t);  // 32+16j+4t..
        const uint32_t a = prmt(qlo, 0x64646464u, 0x5140u), b = prmt(qlo, 0x64646464u, 0x7362u);
        const uint32_t c = prmt(qhi, 0x64646464u, 0x5140u), e = prmt(qhi, 0x64646464u, 0x7362u);
        out[8 * j + 2 * t + 0] = hfma2_u32(hsub2_u32(a, kMagic), ds0, dm0);
        out[8 * j + 2 * t + 1] = hfma2_u32(hsub2_u32(b, kMagic), ds0, dm0);
        out[16 + 8 * j + 2 * t + 0] = hfma2_u32(hsub2_u32(c, kMagic), ds1, dm1);
        out[16 + 8 * j + 2 * t + 1] = hfma2_u32(hsub2_u32(e, kMagic), ds1, dm1);
      }
    }
  }
};

}  // namespace qlin

namespace qlin {

// ---------------------------------------------------------------------------------------------
// i8 family (kind::i8, 128 K-values per stage).  The activation operand is stored with every
// group of 8 columns permuted to 0,2,4,6,1,3,5,7, so TMEM column 2j holds the weights of
// columns 8j+{0,2,4,6} and column 2j+1 those of 8j+{1,3,5,7}.
// ---------------------------------------------------------------------------------------------

// Symmetric 4-bit weights stored as unsigned nibbles u = q + 8 (even column in the low nibble),
// raw [N, K/2] bytes via a TMA box {64 B, 128 rows} with 64-byte swizzle.  Output bytes are
// 16*q (exact in int8); the epilogue divides by 16.
struct DecW4 {
  static constexpr uint32_t kStageBytes = 128 * 64;
  static constexpr bool kTma = true;
  static constexpr float kInvScale = 1.0f / 16.0f;
  __device__ __forceinline__ static void decode(const uint8_t* st, int r, uint32_t (&out)[32]) {
    const uint8_t* row = st + r * 64;
    const int sw = (r >> 1) & 3;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint4 v = *reinterpret_cast<const uint4*>(row + ((j ^ sw) << 4));
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const uint32_t s = w[t] ^ 0x88888888u;  // nibble = two's complement of q
        out[8 * j + 2 * t + 0] = (s << 4) & 0xF0F0F0F0u;  // columns 0,2,4,6 of these 8
        out[8 * j + 2 * t + 1] = s & 0xF0F0F0F0u;         // columns 1,3,5,7
      }
    }
  }
};

// Symmetric 6-bit weights in the repacked "W6 planes" layout (one stage = 128 values per row):
// per unit u of 16 values, L0 / L1 hold the low nibbles of values 0-7 / 8-15 (value i in nibble
// i) and T holds the high 2 bits: byte b bits 0-1 = value 2b, 2-3 = 2b+1, 4-5 = 8+2b, 6-7 = 9+2b.
// Stage chunk: [6 planes][128 rows][16 B]; planes 0-3 carry L0,L1 of units 0..7, planes 4-5 the T
// words of units 0..7.  Output bytes are 4*q = (4u) ^ 0x80; the epilogue divides by 4.
struct DecW6 {
  static constexpr uint32_t kStageBytes = 128 * 96;
  static constexpr bool kTma = false;
  static constexpr float kInvScale = 0.25f;
  __device__ __forceinline__ static void decode(const uint8_t* st, int r, uint32_t (&out)[32]) {
    uint32_t L[16], T[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint4 v = *reinterpret_cast<const uint4*>(st + (j * 128 + r) * 16);
      L[4 * j] = v.x;
      L[4 * j + 1] = v.y;
      L[4 * j + 2] = v.z;
      L[4 * j + 3] = v.w;
    }
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const uint4 v = *reinterpret_cast<const uint4*>(st + ((4 + j) * 128 + r) * 16);
      T[4 * j] = v.x;
      T[4 * j + 1] = v.y;
      T[4 * j + 2] = v.z;
      T[4 * j + 3] = v.w;
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const uint32_t l0 = L[2 * u], l1 = L[2 * u + 1], t = T[u];
      const uint32_t o0 = (l0 & 0x0F0F0F0Fu) | ((t & 0x03030303u) << 4);
      const uint32_t o1 = ((l0 >> 4) & 0x0F0F0F0Fu) | ((t & 0x0C0C0C0Cu) << 2);
      const uint32_t o2 = (l1 & 0x0F0F0F0Fu) | (t & 0x30303030u);
      const uint32_t o3 = ((l1 >> 4) & 0x0F0F0F0Fu) | ((t >> 2) & 0x30303030u);
      out[4 * u + 0] = (o0 << 2) ^ 0x80808080u;
      out[4 * u + 1] = (o1 << 2) ^ 0x80808080u;
      out[4 * u + 2] = (o2 << 2) ^ 0x80808080u;
      out[4 * u + 3] = (o3 << 2) ^ 0x80808080u;
    }
  }
};

}  // namespace qlin
