// Fused dequantize + GEMM on the 5th-generation tensor cores (sm_100a).
//
//   Y[m, n] = colscale[n] * rowscale[m] * sum_k Wdec[n, k] * X[m, k]  (+ bias[n])
//
// Weight-stationary orientation: the decoded weight tile is the MMA's A operand and lives in
// tensor memory (TMEM), written by decoder warps with tcgen05.st; the activation tile is the B
// operand, streamed by TMA into 128-byte-swizzled shared memory; the fp32 accumulator D[n, m]
// is in TMEM too.  A weight tile is 128 rows (the MMA's M); a token tile is TM rows (the
// MMA's N, 16..256), so small batches only shrink the MMA's N while the weight stream stays
// the same.  Keeping A in TMEM leaves shared-memory bandwidth to the activation operand.
//
// Warp roles (448 threads, one CTA per SM, persistent over tiles):
//   warp 0       TMA producer (activations via tensor map; weights via tensor map or bulk copy)
//   warp 1       TMEM allocator + single-thread MMA issuer
//   warps 2..9   decoders, two groups of four that take alternate pipeline stages: one weight
//                row per thread, smem -> registers -> TMEM (A operand)
//   warps 10..13 epilogue: TMEM -> registers, scales, bias, cast, global stores
// Pipelines: STAGES-deep ring (full / a_full / empty) and a double-buffered accumulator
// (acc_full / acc_empty) so the epilogue of one tile overlaps the MMAs of the next.
#pragma once
#include <cuda.h>

#include "qlin_decode.cuh"
#include "qlin_peer.cuh"

namespace qlin {


struct GemmParams {
  int M, N, K;
  int num_k_stages;  // stages over the padded K
  int k_slab;        // K columns per activation slab (the activation is [slabs][M][k_slab]; slabs = 1
                     // for an ordinary row-major X).  A multiple of 64 when there is more than one slab.
  int m_tiles, n_tiles, k_splits;
  int stages_per_split;
  // weights
  const uint8_t* w_stages;  // repacked stage chunks [n_tile][k_stage][stage_bytes] (non-TMA decoders)
  const int32_t* w_row_exp;  // per weight row exponent e (2^-e applied at decode, 2^e in epilogue)
  // epilogue
  const void* col_scale;
  int col_scale_kind;
  const int32_t* x_row_exp;  // per token exponent f (activation was scaled by 2^-f), or null
  const void* bias;
  int bias_kind;  // 0 none, 1 fp16, 2 fp32, 3 bf16
  void* y;
  int y_dtype;
  long long ldy;
  float* partial;  // split-K partial sums, n-major [k_splits][N][Mp]; null when k_splits == 1
  int Mp;          // M rounded up to the token tile (row pitch of the partials)
  DeviceStatus* status;
  // Staged 2-byte output: out.ndst > 0 writes each finished 32-token chunk through shared memory
  // with 16-byte stores to every destination (this rank's slab in each rank's gathered buffer);
  // out.wait / out.signal run the cross-rank flag protocol of qlin_peer.cuh.
  PeerOut out;
};

template <int TM, int STAGES>
struct F16Cfg {
  static constexpr int kDecGroups = 2;
  static constexpr int kThreads = 32 * (2 + 4 * kDecGroups + 4);
  static constexpr int kXStageBytes = TM * 128;  // TM rows x 64 fp16
  static constexpr int kAccBufs = (2 * TM + STAGES * 32 <= 512) ? 2 : 1;
  static constexpr int kAccCols = TM;
  static constexpr int kACol0 = kAccBufs * TM;  // first TMEM column of the A stages
  static constexpr uint32_t kTmemCols = 512;
};

__device__ __forceinline__ float load_bias(const void* bias, int kind, int n) {
  if (kind == 1) return __half2float(reinterpret_cast<const __half*>(bias)[n]);
  if (kind == 2) return reinterpret_cast<const float*>(bias)[n];
  if (kind == 3) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(bias)[n]);
  return 0.f;
}

__device__ __forceinline__ float load_colscale(const GemmParams& p, int n) {
  switch (p.col_scale_kind) {
    case CS_F16: return __half2float(reinterpret_cast<const __half*>(p.col_scale)[n]);
    case CS_F32: return reinterpret_cast<const float*>(p.col_scale)[n];
    case CS_EXP2: return exp2i(p.w_row_exp[n]);
    default: return 1.f;
  }
}

__device__ __forceinline__ void store_out(void* y, int dtype, long long idx, float v) {
  if (dtype == OUT_F16) reinterpret_cast<__half*>(y)[idx] = __float2half_rn(v);
  else if (dtype == OUT_BF16) reinterpret_cast<__nv_bfloat16*>(y)[idx] = __float2bfloat16_rn(v);
  else reinterpret_cast<float*>(y)[idx] = v;
}

template <class Dec, int TM, int STAGES>
__global__ void __launch_bounds__(448, 1)
qgemm_f16_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                 const __grid_constant__ CUtensorMap tmap_p, const GemmParams p) {
  using Cfg = F16Cfg<TM, STAGES>;
  constexpr uint32_t kWStage = (Dec::kStageBytes + 1023) / 1024 * 1024;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sx = smem;                                 // STAGES x kXStageBytes
  uint8_t* sw = sx + STAGES * Cfg::kXStageBytes;      // STAGES x kWStage
  uint64_t* bars = reinterpret_cast<uint64_t*>(sw + STAGES * kWStage);
  uint64_t* full = bars;                    // [STAGES]
  uint64_t* a_full = full + STAGES;         // [STAGES]
  uint64_t* empty = a_full + STAGES;        // [STAGES]
  uint64_t* acc_full = empty + STAGES;      // [2]
  uint64_t* acc_empty = acc_full + 2;       // [2]
  uint64_t* drain = acc_empty + 2;          // [1]
  uint64_t* epi_bar = drain + 1;            // [1] epilogue warps' barrier (bounded, unlike bar.sync)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(epi_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // Split-K epilogue staging: two 16 KB tiles (128 rows x 32 fp32, 128-byte swizzled) written by
  // the epilogue warps and stored to the partials with one TMA tensor store each.
  uint8_t* sepi = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(tmem_slot + 2) + 1023) & ~uintptr_t(1023));

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_tiles = p.m_tiles * p.n_tiles * p.k_splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&a_full[s], 4);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    mbar_init(drain, 1);
    mbar_init(epi_bar, 4);
    *abort_flag = 0;
    // Before any activation is read: every rank finished the previous output-writing kernel.
    if (p.out.wait && !peer_wait(p.out, p.status, 6)) *abort_flag = 1;
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
    // ----------------------------------------------------------------- producer
    if (elect_one()) {
      uint32_t it = 0;
      bool ok = *abort_flag == 0;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        const int mt = t % p.m_tiles;
        const int rest = t / p.m_tiles;
        const int nt = rest % p.n_tiles;
        const int ks = rest / p.n_tiles;
        const int s0 = ks * p.stages_per_split;
        const int s1 = min(p.num_k_stages, s0 + p.stages_per_split);
        for (int kst = s0; kst < s1; ++kst, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, p.status, 1)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[s], Cfg::kXStageBytes + Dec::kStageBytes);
          {
            const int k0 = kst * 64;
            const int slab = k0 / p.k_slab;
            tma_load_3d(sx + s * Cfg::kXStageBytes, &tmap_x, &full[s], k0 - slab * p.k_slab, mt * TM, slab);
          }
          if constexpr (Dec::kTma) {
            tma_load_2d(sw + s * kWStage, &tmap_w, &full[s], kst * 64, nt * 128);
          } else {
            const uint8_t* src = p.w_stages + ((size_t)nt * p.num_k_stages + kst) * Dec::kStageBytes;
            bulk_load(sw + s * kWStage, src, Dec::kStageBytes, &full[s]);
          }
        }
      }
      if (!ok) {
        // Let copies already in flight land before the CTA's shared memory goes away.
        for (uint32_t j = (it >= (uint32_t)STAGES ? it - STAGES : 0); j < it; ++j) {
          const uint64_t t0 = globaltimer();
          while (!mbar_try_wait(smem_u32(&full[j % STAGES]), (j / STAGES) & 1)) {
            if (globaltimer() - t0 > QLIN_WAIT_TIMEOUT_NS) break;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------------- MMA issuer
    if (elect_one()) {
      constexpr uint32_t idesc = idesc_f16_f32(128, TM);
      uint32_t it = 0, tile_i = 0;
      bool ok = *abort_flag == 0;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++tile_i) {
        const int ks = (t / p.m_tiles) / p.n_tiles;
        const int s0 = ks * p.stages_per_split;
        const int s1 = min(p.num_k_stages, s0 + p.stages_per_split);
        const int b = (Cfg::kAccBufs == 2) ? (tile_i & 1) : 0;
        const uint32_t aph = (Cfg::kAccBufs == 2) ? ((tile_i >> 1) & 1) : (tile_i & 1);
        if (!mbar_wait(&acc_empty[b], aph ^ 1, abort_flag, p.status, 2)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + b * Cfg::kAccCols;
        for (int kst = s0; kst < s1; ++kst, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(&a_full[s], ph, abort_flag, p.status, 3)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_tmem = tmem_base + Cfg::kACol0 + s * 32;
          const uint64_t b_desc = smem_desc_sw128(smem_u32(sx + s * Cfg::kXStageBytes));
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            mma_f16_ts(d_tmem, a_tmem + kk * 8, b_desc + (uint64_t)(kk * 2), idesc, (kst > s0 || kk > 0) ? 1u : 0u);
          }
          tc_commit(&empty[s]);
        }
        if (!ok) break;
        tc_commit(&acc_full[b]);
      }
      // Wait until every MMA this thread issued has completed before TMEM is released.
      tc_commit(drain);
      const uint64_t t0 = globaltimer();
      while (!mbar_try_wait(smem_u32(drain), 0)) {
        if (globaltimer() - t0 > QLIN_WAIT_TIMEOUT_NS) break;
      }
    }
  } else if (warp < 2 + 4 * Cfg::kDecGroups) {
    // ----------------------------------------------------------------- decoders
    const int quarter = warp & 3;
    const int group = (warp - 2) >> 2;  // takes ring iterations it with it % kDecGroups == group
    const int r = quarter * 32 + lane;  // weight row within the tile == TMEM lane
    uint32_t it = 0;
    bool ok = *abort_flag == 0;
    for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
      const int nt = (t / p.m_tiles) % p.n_tiles;
      const int ks = (t / p.m_tiles) / p.n_tiles;
      const int s0 = ks * p.stages_per_split;
      const int s1 = min(p.num_k_stages, s0 + p.stages_per_split);
      const int n = nt * 128 + r;
      float rscale = 1.f;
      if (p.w_row_exp != nullptr && p.col_scale_kind == CS_EXP2) rscale = exp2i(-p.w_row_exp[min(n, p.N - 1)]);
      for (int kst = s0; kst < s1; ++kst, ++it) {
        if ((int)(it % Cfg::kDecGroups) != group) continue;
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1;
        if (!mbar_wait(&full[s], ph, abort_flag, p.status, 4)) { ok = false; break; }
        uint32_t a[32];
        Dec::decode(sw + s * kWStage, r, rscale, a);
        tmem_st32(tmem_base + ((uint32_t)(quarter * 32) << 16) + Cfg::kACol0 + s * 32, a);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&a_full[s]);
      }
    }
  } else {
    // ----------------------------------------------------------------- epilogue
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    uint32_t tile_i = 0;
    uint32_t epi_chunk = 0, epi_phase = 0;
    // Barrier of the four epilogue warps.  A bounded mbarrier wait instead of a named barrier:
    // if another role gives up, the warps leave on the abort flag instead of waiting for a warp
    // that already left the loop.
    auto epi_sync = [&]() -> bool {
      __syncwarp();
      if (lane == 0) mbar_arrive(epi_bar);
      const bool ok = mbar_wait(epi_bar, epi_phase & 1, abort_flag, p.status, 7);
      ++epi_phase;
      return ok;
    };
    bool epi_ok = true;
    const int etid = threadIdx.x - 32 * (2 + 4 * Cfg::kDecGroups);  // 0..127
    for (int t = blockIdx.x; t < num_tiles && epi_ok && *abort_flag == 0; t += gridDim.x, ++tile_i) {
      const int mt = t % p.m_tiles;
      const int nt = (t / p.m_tiles) % p.n_tiles;
      const int ks = (t / p.m_tiles) / p.n_tiles;
      const int b = (Cfg::kAccBufs == 2) ? (tile_i & 1) : 0;
      const uint32_t aph = (Cfg::kAccBufs == 2) ? ((tile_i >> 1) & 1) : (tile_i & 1);
      if (!mbar_wait(&acc_full[b], aph, abort_flag, p.status, 5)) break;
      tc_fence_after();
      const int n = nt * 128 + r;
      const bool n_ok = n < p.N;
      float cs = 1.f, bias = 0.f;
      if (p.k_splits == 1 && n_ok) {
        cs = load_colscale(p, n);
        bias = load_bias(p.bias, p.bias_kind, n);
      }
#pragma unroll 1
      for (int c0 = 0; c0 < TM; c0 += 32) {
        uint32_t v[32];
        tmem_ld32(tmem_base + ((uint32_t)(quarter * 32) << 16) + b * Cfg::kAccCols + c0, v);
        if (p.k_splits > 1) {
          // n-major partials [split][N][Mp]: this thread's 32 tokens are one 128-byte row of a
          // swizzled staging tile; one TMA store per chunk writes whole lines
          tmem_wait_ld();
          if constexpr (TM >= 32) {
            const bool issuer = (warp == 2 + 4 * Cfg::kDecGroups) && lane == 0;
            uint8_t* buf = sepi + (epi_chunk & 1) * 16384;
            if (issuer) bulk_wait_read<1>();  // the store that last read this buffer is done
            if (!(epi_ok = epi_sync())) break;
            uint8_t* rowp = buf + r * 128;
#pragma unroll
            for (int j = 0; j < 8; ++j)
              *reinterpret_cast<float4*>(rowp + ((j ^ (r & 7)) << 4)) =
                  make_float4(__uint_as_float(v[4 * j]), __uint_as_float(v[4 * j + 1]),
                              __uint_as_float(v[4 * j + 2]), __uint_as_float(v[4 * j + 3]));
            fence_proxy_async_smem();
            if (!(epi_ok = epi_sync())) break;
            if (issuer) {
              tma_store_3d(&tmap_p, buf, mt * TM + c0, nt * 128, ks);
              bulk_commit();
            }
            ++epi_chunk;
          } else {
            if (n_ok) {
              float4* dst = reinterpret_cast<float4*>(p.partial + ((size_t)ks * p.N + n) * p.Mp + mt * TM + c0);
#pragma unroll
              for (int j = 0; j < TM / 4; ++j)
                dst[j] = make_float4(__uint_as_float(v[4 * j]), __uint_as_float(v[4 * j + 1]),
                                     __uint_as_float(v[4 * j + 2]), __uint_as_float(v[4 * j + 3]));
            }
          }
          continue;
        }
        // per-token power of two for the 32 columns of this chunk: lane j holds column j's
        constexpr int kCh = TM < 32 ? TM : 32;  // tokens of this tile in the chunk
        const int mj = mt * TM + c0 + lane;
        const float rs_lane = (p.x_row_exp != nullptr && mj < p.M && lane < kCh) ? exp2i(__ldg(&p.x_row_exp[mj])) : 1.f;
        tmem_wait_ld();
        if (p.out.ndst > 0) {
          // Stage the chunk as [kCh tokens][128 channels] 2-byte values, then copy whole 16-byte
          // pieces of token rows to every destination.  Two buffers: the barrier after staging
          // one also orders every thread's reads of the other before it is staged again.
          uint16_t* buf = reinterpret_cast<uint16_t*>(sepi + (epi_chunk & 1) * 8192);
#pragma unroll
          for (int j = 0; j < kCh; ++j) {
            const float rs = __shfl_sync(0xffffffffu, rs_lane, j);
            float o = __fmul_rn(__fmul_rn(__uint_as_float(v[j]), cs), rs);
            o = __fadd_rn(o, bias);
            buf[j * 128 + r] = p.y_dtype == OUT_BF16 ? __bfloat16_as_ushort(__float2bfloat16_rn(o))
                                                     : __half_as_ushort(__float2half_rn(o));
          }
          if (!(epi_ok = epi_sync())) break;
#pragma unroll
          for (int i = etid; i < kCh * 16; i += 128) {
            const int m = mt * TM + c0 + (i >> 4);
            const int n0 = nt * 128 + (i & 15) * 8;
            if (m < p.M && n0 < p.N) {
              const uint4 val = reinterpret_cast<const uint4*>(buf)[i];
              const long long off = (long long)m * p.ldy + n0;
#pragma unroll
              for (int d = 0; d < kMaxPeers; ++d)
                if (d < p.out.ndst) reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(p.out.dst[d]) + off)[0] = val;
            }
          }
          ++epi_chunk;
          continue;
        }
#pragma unroll
        for (int j = 0; j < kCh; ++j) {
          const int m = mt * TM + c0 + j;
          const float rs = __shfl_sync(0xffffffffu, rs_lane, j);
          if (n_ok && m < p.M) {
            float o = __fmul_rn(__fmul_rn(__uint_as_float(v[j]), cs), rs);
            o = __fadd_rn(o, bias);
            store_out(p.y, p.y_dtype, (long long)m * p.ldy + n, o);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);
    }
    if (warp == 2 + 4 * Cfg::kDecGroups && lane == 0) bulk_wait_all();  // partial stores complete
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
  if (p.out.signal && threadIdx.x == 0) peer_signal_last_cta(p.out);
}

template <class Dec, int TM, int STAGES>
constexpr int qgemm_f16_smem_bytes() {
  constexpr int kWStage = (Dec::kStageBytes + 1023) / 1024 * 1024;
  return 1024 /*align slack*/ + STAGES * (TM * 128 + kWStage) + 1024 /*barriers, aligned*/ + 2 * 16384;
}

}  // namespace qlin
