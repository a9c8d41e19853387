// W4A8 / W6A8 on the integer tensor cores (tcgen05.mma kind::i8, int32 accumulation).
//
//   Y[m, n] = sx[m] * inv * sum_g s[n, g] * P_g[m, n]  (+ bias[n]),
//   P_g[m, n] = sum_{k in group g} xq[m, k] * wq'[n, k]   (exact int32)
//
// xq are the per-token INT8 activations (prologue), wq' = D * wq the decoded weights scaled by
// an exact power of two D (16 for 4-bit, 4 for 6-bit) so the decode needs no shuffles, and
// inv = 1/D.  Every K-group accumulates into its own int32 TMEM buffer (double-buffered); the
// rescale warps fold s[n, g] * P_g into fp32 registers while the tensor cores run the next
// group.  With one group spanning all of K (per-channel scales) this is a plain int8 GEMM with
// the scale in the epilogue.
//
// The rescale is the per-group serial step (its cost grows with every value of every group), so
// it is kept to one exact int32 -> fp32 conversion per value and one packed fp32 FMA per two
// values (ffma2_cvt).  The first MMA of a group overwrites its buffer; the rescale warps hand the
// buffer back as soon as its values are in registers.
//
// Warp roles (448 threads, one CTA per SM, persistent):
//   warp 0        TMA producer            warp 1   TMEM alloc + MMA issuer
//   warps 2..5    decoders -> TMEM A operand (int8); each pass decodes two consecutive stages
//                 and waits for both TMEM stores at once, which hides the store latency
//   warps 6..13   rescale + epilogue: two warps per TMEM lane quarter, half the columns each
#pragma once
#include <cuda.h>

#include "qlin_decode.cuh"

namespace qlin {

enum I8ScaleKind : int { I8S_GROUP_F16 = 0, I8S_CHANNEL_F32 = 1 };

struct GemmI8Params {
  int M, N, K;        // K = padded K (multiple of 128)
  int num_k_stages;   // K / 128
  int m_tiles, n_tiles;
  int group;          // K-values per scale group (multiple of 32); == K for per-channel scales
  int groups_per_row; // K / group
  const uint8_t* w_stages;  // repacked stage chunks for non-TMA decoders
  const void* scales;       // fp16 [N, groups_per_row] or fp32 [N]
  int scale_kind;
  float inv_scale;          // 1 / D of the decoder
  const float* x_scale;     // per-token activation scale [M]
  const void* bias;
  int bias_kind;
  void* y;
  int y_dtype;
  long long ldy;
  DeviceStatus* status;
  // Element counts of the caller's buffers for the QLIN_CHECKS build (unused otherwise).
  long long lim_y;        // output elements reachable from y
  long long lim_w_bytes;  // bytes of w_stages
  long long lim_scales;   // scale entries (N * groups_per_row, or N per channel)
};

// Output element idx (checked against the caller's buffer in the QLIN_CHECKS build).
__device__ __forceinline__ void store_out_i8(const GemmI8Params& p, long long idx, float o) {
  if (!qchk(BS_I8_Y, idx, p.lim_y)) return;
  if (p.y_dtype == OUT_F16) reinterpret_cast<__half*>(p.y)[idx] = __float2half_rn(o);
  else if (p.y_dtype == OUT_BF16) reinterpret_cast<__nv_bfloat16*>(p.y)[idx] = __float2bfloat16_rn(o);
  else reinterpret_cast<float*>(p.y)[idx] = o;
}

__device__ __forceinline__ float load_bias_i8(const void* bias, int kind, int n, int lim) {
  if (kind != 0 && !qchk(BS_I8_SCALE, n, lim)) return 0.f;
  if (kind == 1) return __half2float(reinterpret_cast<const __half*>(bias)[n]);
  if (kind == 2) return reinterpret_cast<const float*>(bias)[n];
  if (kind == 3) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(bias)[n]);
  return 0.f;
}

// (a0, a1) += s * (float(p0), float(p1)) for int32 group sums p: two exact conversions (|p| <= 2^24
// for every group of up to 1024 values of these formats; cvt.rn beyond) and one packed fp32 FMA.
// Measured against the magic-number form (p + the bits of 1.5 * 2^23, an exact fp32 subtraction,
// then the FMA): 15-25% faster kernels at configurations 3 and 4, the rescale being the FMA-pipe
// bound part of the loop.
__device__ __forceinline__ void ffma2_cvt(float s, uint32_t p0, uint32_t p1, float& a0, float& a1) {
  const float f0 = (float)(int32_t)p0, f1 = (float)(int32_t)p1;
  asm("{\n\t.reg .b64 f, sc, acc;\n\t"
      "mov.b64 f, {%2, %3};\n\t"
      "mov.b64 sc, {%4, %4};\n\t"
      "mov.b64 acc, {%0, %1};\n\t"
      "fma.rn.f32x2 acc, sc, f, acc;\n\t"
      "mov.b64 {%0, %1}, acc;\n\t}"
      : "+f"(a0), "+f"(a1)
      : "f"(f0), "f"(f1), "f"(s));
}

template <int TM, int STAGES>
struct I8Cfg {
  static constexpr int kDecGroups = 1;
  static constexpr int kEpiWarps = 8;
  static constexpr int kEpiParts = kEpiWarps / 4;  // rescale warps per TMEM lane quarter
  static constexpr int kThreads = 32 * (2 + 4 * kDecGroups + kEpiWarps);
  static constexpr int kXStageBytes = TM * 128;  // TM rows x 128 int8
  static constexpr int kACol0 = 2 * TM;
  static constexpr uint32_t kTmemCols = 512;
  static_assert(2 * TM + STAGES * 32 <= 512, "TMEM budget");
  static_assert(TM / kEpiParts >= 8 && (TM / kEpiParts <= 32 || TM / kEpiParts % 32 == 0),
                "each rescale warp reads its columns in chunks of 8, 16 or 32");
};

template <class Dec, int TM, int STAGES>
__global__ void __launch_bounds__(I8Cfg<TM, STAGES>::kThreads, 1)
qgemm_i8_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                const GemmI8Params p) {
  using Cfg = I8Cfg<TM, STAGES>;
  constexpr uint32_t kWStage = (Dec::kStageBytes + 1023) / 1024 * 1024;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sx = smem;
  uint8_t* sw = sx + STAGES * Cfg::kXStageBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sw + STAGES * kWStage);
  uint64_t* full = bars;
  uint64_t* a_full = full + STAGES;
  uint64_t* empty = a_full + STAGES;
  uint64_t* acc_full = empty + STAGES;  // [2]
  uint64_t* acc_empty = acc_full + 2;   // [2]
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_tiles = p.m_tiles * p.n_tiles;
  const int groups_per_tile = p.groups_per_row;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&a_full[s], 4);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], Cfg::kEpiWarps);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    // the carve-out (rings, barriers, flags) lies inside the launch's shared memory
    if (!qchk_smem(BS_I8_SMEM, smem_raw, bars, reinterpret_cast<volatile uint8_t*>(abort_flag + 1) -
                                         reinterpret_cast<volatile uint8_t*>(bars)))
      *abort_flag = 1;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmap_x);
    if constexpr (Dec::kTma) prefetch_tmap(&tmap_w);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (warp == 0) {
    if (elect_one()) {
      uint32_t it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        const int mt = t % p.m_tiles;
        const int nt = t / p.m_tiles;
        for (int kst = 0; kst < p.num_k_stages; ++kst, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, p.status, 11)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[s], Cfg::kXStageBytes + Dec::kStageBytes);
          tma_load_2d(sx + s * Cfg::kXStageBytes, &tmap_x, &full[s], kst * 128, mt * TM);
          if constexpr (Dec::kTma) {
            tma_load_2d(sw + s * kWStage, &tmap_w, &full[s], kst * 64, nt * 128);
          } else {
            const long long off = ((long long)nt * p.num_k_stages + kst) * Dec::kStageBytes;
            // out of range: copy stage 0 instead, so the pipeline keeps its byte count
            const bool in = qchk_span(BS_I8_WBULK, off, Dec::kStageBytes, p.lim_w_bytes);
            bulk_load(sw + s * kWStage, p.w_stages + (in ? off : 0), Dec::kStageBytes, &full[s]);
          }
        }
      }
      if (!ok) {
        for (uint32_t j = (it >= (uint32_t)STAGES ? it - STAGES : 0); j < it; ++j) {
          const uint64_t t0 = globaltimer();
          while (!mbar_try_wait(smem_u32(&full[j % STAGES]), (j / STAGES) & 1)) {
            if (globaltimer() - t0 > QLIN_WAIT_TIMEOUT_NS) break;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idesc = idesc_s8_s32(128, TM);
      uint32_t it = 0, g_all = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        uint32_t b = 0;
        int gk = 0;  // K position inside the current group (no divisions on this thread's path)
        for (int kst = 0; kst < p.num_k_stages && ok; ++kst, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(&a_full[s], ph, abort_flag, p.status, 12)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_tmem = tmem_base + Cfg::kACol0 + s * 32;
          const uint64_t b_desc = smem_desc_sw128(smem_u32(sx + s * Cfg::kXStageBytes));
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            if (gk == 0) {  // first MMA of a group: wait for its accumulator buffer, which it overwrites
              b = g_all & 1;
              if (!mbar_wait(&acc_empty[b], ((g_all >> 1) & 1) ^ 1, abort_flag, p.status, 13)) { ok = false; break; }
              tc_fence_after();
            }
            mma_i8_ts(tmem_base + b * TM, a_tmem + kk * 8, b_desc + (uint64_t)(kk * 2), idesc, gk > 0 ? 1u : 0u);
            gk += 32;
            if (gk == p.group) {
              tc_commit(&acc_full[b]);
              ++g_all;
              gk = 0;
            }
          }
          if (!ok) break;
          tc_commit(&empty[s]);
        }
      }
      tc_commit(drain);
      const uint64_t t0 = globaltimer();
      while (!mbar_try_wait(smem_u32(drain), 0)) {
        if (globaltimer() - t0 > QLIN_WAIT_TIMEOUT_NS) break;
      }
    }
  } else if (warp < 2 + 4 * Cfg::kDecGroups) {
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lanes = (uint32_t)(quarter * 32) << 16;
    uint32_t it = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
      for (int kst = 0; kst < p.num_k_stages; kst += 2) {
        const bool two = kst + 1 < p.num_k_stages;
        const int s0 = it % STAGES, s1 = (it + 1) % STAGES;
        if (!mbar_wait_sleep(&full[s0], (it / STAGES) & 1, abort_flag, p.status, 14)) { ok = false; break; }
        uint32_t a[32];
        Dec::decode(sw + s0 * kWStage, r, a);
        tmem_st32(tmem_base + lanes + Cfg::kACol0 + s0 * 32, a);
        if (two) {
          if (!mbar_wait_sleep(&full[s1], ((it + 1) / STAGES) & 1, abort_flag, p.status, 14)) { ok = false; break; }
          uint32_t a1[32];
          Dec::decode(sw + s1 * kWStage, r, a1);
          tmem_st32(tmem_base + lanes + Cfg::kACol0 + s1 * 32, a1);
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&a_full[s0]);
          if (two) mbar_arrive(&a_full[s1]);
        }
        it += two ? 2 : 1;
      }
    }
  } else {
    // ----------------------------------------------------------------- rescale + epilogue
    constexpr int kCols = TM / Cfg::kEpiParts;  // tokens per rescale warp
    constexpr int kChunk = kCols < 16 ? kCols : 16;  // columns per TMEM load (register budget)
    const int ew = warp - (2 + 4 * Cfg::kDecGroups);
    const int quarter = warp & 3;
    const int part = ew >> 2;
    const int r = quarter * 32 + lane;
    uint32_t g_all = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
      const int mt = t % p.m_tiles;
      const int nt = t / p.m_tiles;
      const int n = nt * 128 + r;
      const bool n_ok = n < p.N;
      float accf[kCols];
#pragma unroll
      for (int j = 0; j < kCols; ++j) accf[j] = 0.f;
      const __half* gscale = reinterpret_cast<const __half*>(p.scales) + (size_t)min(n, p.N - 1) * p.groups_per_row;
      float s_next = 0.f;
      const long long gbase = (long long)min(n, p.N - 1) * p.groups_per_row;
      if (n_ok && qchk(BS_I8_SCALE, p.scale_kind == I8S_GROUP_F16 ? gbase : n, p.lim_scales))
        s_next = (p.scale_kind == I8S_GROUP_F16) ? __half2float(gscale[0]) : reinterpret_cast<const float*>(p.scales)[n];
      for (int g = 0; g < groups_per_tile; ++g, ++g_all) {
        const float sg = s_next;
        if (n_ok && p.scale_kind == I8S_GROUP_F16 && g + 1 < groups_per_tile &&
            qchk(BS_I8_SCALE, gbase + g + 1, p.lim_scales))
          s_next = __half2float(gscale[g + 1]);
        const uint32_t b = g_all & 1;
        if (!mbar_wait_sleep(&acc_full[b], (g_all >> 1) & 1, abort_flag, p.status, 15)) { ok = false; break; }
        tc_fence_after();
        const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + b * TM + part * kCols;
#pragma unroll
        for (int c0 = 0; c0 < kCols; c0 += kChunk) {
          uint32_t v[kChunk];
          tmem_ld_cols<kChunk>(taddr + c0, v);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < kChunk; j += 2) ffma2_cvt(sg, v[j], v[j + 1], accf[c0 + j], accf[c0 + j + 1]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[b]);
      }
      if (!ok) break;
      const float bias = n_ok ? load_bias_i8(p.bias, p.bias_kind, n, p.N) : 0.f;
#pragma unroll
      for (int c0 = 0; c0 < kCols; c0 += kChunk) {
        const int m0 = mt * TM + part * kCols + c0;
        const float sx_lane = (lane < kChunk && m0 + lane < p.M && qchk(BS_I8_SCALE, m0 + lane, p.M))
                                  ? __ldg(&p.x_scale[m0 + lane]) * p.inv_scale : 0.f;
#pragma unroll
        for (int j = 0; j < kChunk; ++j) {
          const float sxm = __shfl_sync(0xffffffffu, sx_lane, j);
          const int m = m0 + j;
          if (n_ok && m < p.M) {
            const float o = __fadd_rn(__fmul_rn(accf[c0 + j], sxm), bias);
            store_out_i8(p, (long long)m * p.ldy + n, o);
          }
        }
      }
    }
  }

  // Warps 0 and 1 ran their loops on one elected lane; reconverge before the block barrier
  // (barrier.sync is .aligned) and before the warp-wide TMEM dealloc.
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}

template <class Dec, int TM, int STAGES>
constexpr int qgemm_i8_smem_bytes() {
  constexpr int kWStage = (Dec::kStageBytes + 1023) / 1024 * 1024;
  return 1024 + STAGES * (TM * 128 + kWStage) + (3 * STAGES + 5) * 8 + 16;
}

}  // namespace qlin
