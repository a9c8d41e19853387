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
// Pipelines: a STAGES-deep shared-memory ring (full / empty), a ring of decoded-weight slots in
// TMEM (a_full / a_empty) and a double-buffered accumulator
// (acc_full / acc_empty) so the epilogue of one tile overlaps the MMAs of the next.
#pragma once
#include <cuda.h>

#include "qlin_decode.cuh"
#include "qlin_hadamard.cuh"
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
  // Unmerged LoRA fused as extra K stages: stages [main_k_stages, num_k_stages) multiply the bf16
  // low-rank activation T' (tensor map tmap_t) by the bf16 up-projection U' [n_tiles*128][lora_k]
  // into the same accumulator (main_k_stages == num_k_stages: no LoRA).
  int main_k_stages;
  const __nv_bfloat16* lora_u;
  int lora_k;
  // ROT kernels only: each output row is multiplied by the block Hadamard of rot_group (32, 64 or
  // 128) channels, in fp32, before its one rounding (the staged 2-byte output path, no K split).
  int rot_group;
  DeviceStatus* status;
  // Element counts of the caller's buffers, derived on the host from the C-ABI arguments; the
  // QLIN_CHECKS build tests every plain access against them (unused otherwise).
  long long lim_y;        // output elements reachable from y (and from each out.dst[d])
  long long lim_w_bytes;  // bytes of w_stages (bulk-copied weight stages)
  long long lim_partial;  // fp32 elements of partial
  long long lim_lora_u;   // bf16 elements of lora_u
  // Staged 2-byte output: out.ndst > 0 writes each finished 32-token chunk through shared memory
  // with 16-byte stores to every destination (this rank's slab in each rank's gathered buffer);
  // out.wait / out.signal run the cross-rank flag protocol of qlin_peer.cuh.
  PeerOut out;
};

// Two rings: STAGES shared-memory stages (activation tile + packed weights, filled by TMA) and
// kASlots decoded-weight slots in TMEM (32 columns each).  TMEM holds the accumulators too, so
// it bounds the slots; the shared-memory ring can run deeper and keep more loads in flight.
//
// PAIR: the CTAs of a 2-CTA cluster share cta_group::2 MMAs of 256 weight rows (128 decoded into
// each CTA's TMEM) by TM tokens (TM/2 loaded into each CTA's shared memory), so each SM streams
// half of the activation tile per MMA.  The even CTA issues the MMAs; decoders and epilogues of
// both CTAs arrive on its barriers, and its commits arrive on the barriers of both.
template <int TM, int STAGES, bool PAIR = false>
struct F16Cfg {
  static constexpr int kCtas = PAIR ? 2 : 1;
  static constexpr int kDecGroups = 2;
  static constexpr int kThreads = 32 * (2 + 4 * kDecGroups + 4);
  static constexpr int kXRows = TM / kCtas;              // activation rows this CTA loads per stage
  static constexpr int kXStageBytes = kXRows * 128;      // kXRows rows x 64 fp16
  static constexpr int kAccBufs = (2 * TM + 4 * 32 <= 512) ? 2 : 1;
  static constexpr int kAccCols = TM;
  static constexpr int kACol0 = kAccBufs * TM;  // first TMEM column of the A slots
  static constexpr int kASlotsMax = (512 - kAccBufs * TM) / 32;
  static constexpr int kASlots = STAGES < kASlotsMax ? STAGES : (kASlotsMax < 8 ? kASlotsMax : 8);
  static constexpr uint32_t kTmemCols = 512;
  static_assert(kASlots >= 2, "at least two decoded-weight slots");
};

__device__ __forceinline__ float load_bias(const void* bias, int kind, int n, int lim) {
  if (kind != 0 && !qchk(BS_GEMM_BIAS, n, lim)) return 0.f;
  if (kind == 1) return __half2float(reinterpret_cast<const __half*>(bias)[n]);
  if (kind == 2) return reinterpret_cast<const float*>(bias)[n];
  if (kind == 3) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(bias)[n]);
  return 0.f;
}

__device__ __forceinline__ float load_colscale(const GemmParams& p, int n) {
  if (!qchk(BS_GEMM_BIAS, n, p.N)) return 1.f;
  switch (p.col_scale_kind) {
    case CS_F16: return __half2float(reinterpret_cast<const __half*>(p.col_scale)[n]);
    case CS_F32: return reinterpret_cast<const float*>(p.col_scale)[n];
    case CS_EXP2: return exp2i(p.w_row_exp[n]);
    default: return 1.f;
  }
}

__device__ __forceinline__ void store_out(void* y, int dtype, long long idx, float v, long long lim) {
  if (!qchk(BS_GEMM_Y, idx, lim)) return;
  if (dtype == OUT_F16) reinterpret_cast<__half*>(y)[idx] = __float2half_rn(v);
  else if (dtype == OUT_BF16) reinterpret_cast<__nv_bfloat16*>(y)[idx] = __float2bfloat16_rn(v);
  else reinterpret_cast<float*>(y)[idx] = v;
}

template <class Dec, int TM, int STAGES, bool PAIR, bool ROT = false>
__global__ void __launch_bounds__(448, 1)
qgemm_f16_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                 const __grid_constant__ CUtensorMap tmap_p, const __grid_constant__ CUtensorMap tmap_t,
                 const __grid_constant__ PeerMaps out_maps, const GemmParams p) {
  using Cfg = F16Cfg<TM, STAGES, PAIR>;
  constexpr uint32_t kWStage = (Dec::kStageBytes + 1023) / 1024 * 1024;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sx = smem;                                 // STAGES x kXStageBytes
  uint8_t* sw = sx + STAGES * Cfg::kXStageBytes;      // STAGES x kWStage
  uint64_t* bars = reinterpret_cast<uint64_t*>(sw + STAGES * kWStage);
  uint64_t* full = bars;                    // [STAGES] X + W landed
  uint64_t* empty = full + STAGES;          // [STAGES] MMAs that read the stage completed
  uint64_t* a_full = empty + STAGES;        // [kASlots] decoded weights written to TMEM
  uint64_t* a_empty = a_full + Cfg::kASlots;  // [kASlots] MMAs that read the slot completed
  uint64_t* acc_full = a_empty + Cfg::kASlots;  // [2]
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
  // Tiles are (token tile, group of kCtas weight tiles, K split); a CTA of a pair takes weight
  // tile 2 * group + rank.  Pairs (or single CTAs) walk the tiles persistently.
  const uint32_t rank = PAIR ? cluster_ctarank() : 0;
  const bool leader = rank == 0;
  const int n_groups = p.n_tiles / Cfg::kCtas;
  const int num_tiles = p.m_tiles * n_groups * p.k_splits;
  const int tile0 = blockIdx.x / Cfg::kCtas;
  const int tile_step = gridDim.x / Cfg::kCtas;
  auto tile_nt = [&](int t) { return ((t / p.m_tiles) % n_groups) * Cfg::kCtas + (int)rank; };
  auto tile_ks = [&](int t) { return (t / p.m_tiles) / n_groups; };
  // Arrivals that the MMA issuer waits for go to the even CTA's barriers; in a single CTA these
  // are its own.
  auto arrive_leader = [&](uint64_t* bar) {
    if constexpr (PAIR) mbar_arrive_cluster(cluster_map(bar, 0));
    else mbar_arrive(bar);
  };
  // MMA completion arrives on the barrier in every CTA of the pair.
  auto commit_all = [&](uint64_t* bar) {
    if constexpr (PAIR) {
      tc_commit_pair(cluster_map(bar, 0));
      tc_commit_pair(cluster_map(bar, 1));
    } else {
      tc_commit(bar);
    }
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < Cfg::kASlots; ++a) {
      mbar_init(&a_full[a], 4 * Cfg::kCtas);
      mbar_init(&a_empty[a], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4 * Cfg::kCtas);
    }
    mbar_init(drain, 1);
    mbar_init(epi_bar, 4);
    *abort_flag = 0;
    // the carve-out (rings, barriers, epilogue staging) lies inside the launch's shared memory
    if (!qchk_smem(BS_GEMM_SMEM, smem_raw, sepi, 2 * 16384)) *abort_flag = 1;
    // Before any activation is read: every rank finished the previous output-writing kernel.
    if (p.out.wait && !peer_wait(p.out, p.status, 6)) *abort_flag = 1;
    fence_mbar_init();
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_slot, Cfg::kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, Cfg::kTmemCols);
      tmem_relinquish();
    }
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmap_x);
    if constexpr (Dec::kTma) prefetch_tmap(&tmap_w);
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync();  // both CTAs' barriers are initialized before any remote arrive
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ----------------------------------------------------------------- producer
    if (elect_one()) {
      uint32_t it = 0;
      bool ok = *abort_flag == 0;
      for (int t = tile0; t < num_tiles && ok; t += tile_step) {
        const int mt = t % p.m_tiles;
        const int nt = tile_nt(t);
        const int ks = tile_ks(t);
        const int s0 = ks * p.stages_per_split;
        const int s1 = min(p.num_k_stages, s0 + p.stages_per_split);
        // weight stages, then (fused LoRA) the low-rank stages in a loop of their own, so the
        // weight-stage loop is the same code with or without LoRA support
        const int s_main = min(s1, p.main_k_stages);
        for (int kst = s0; kst < s_main; ++kst, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, p.status, 1)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[s], Cfg::kXStageBytes + Dec::kStageBytes);
          {
            const int k0 = kst * 64;
            const int slab = k0 / p.k_slab;
            // fp16 x coordinate: 8 elements per 16 bytes (a misaligned copy is skipped and the
            // stage's barrier then runs out its bounded wait)
            if (qchk_align(BS_TMA_ALIGN, (long long)(k0 - slab * p.k_slab) * 2, 16))
              tma_load_3d(sx + s * Cfg::kXStageBytes, &tmap_x, &full[s], k0 - slab * p.k_slab,
                          mt * TM + (int)rank * Cfg::kXRows, slab);
          }
          if constexpr (Dec::kTma) {
            tma_load_2d(sw + s * kWStage, &tmap_w, &full[s], kst * 64, nt * 128);
          } else {
            const long long off = ((long long)nt * p.main_k_stages + kst) * Dec::kStageBytes;
            // out of range: copy stage 0 instead, so the pipeline keeps its byte count
            const bool in = qchk_span(BS_GEMM_WBULK, off, Dec::kStageBytes, p.lim_w_bytes);
            bulk_load(sw + s * kWStage, p.w_stages + (in ? off : 0), Dec::kStageBytes, &full[s]);
          }
        }
        for (int kst = max(s0, p.main_k_stages); kst < s1 && ok; ++kst, ++it) {  // LoRA: T' only
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, p.status, 1)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[s], Cfg::kXStageBytes);
          if (qchk_align(BS_TMA_ALIGN, (long long)(kst - p.main_k_stages) * 64 * 2, 16))
            tma_load_2d(sx + s * Cfg::kXStageBytes, &tmap_t, &full[s], (kst - p.main_k_stages) * 64,
                        mt * TM + (int)rank * Cfg::kXRows);
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
    if (leader && elect_one()) {
      constexpr uint32_t idesc_main = idesc_f16_f32(128 * Cfg::kCtas, TM);
      constexpr uint32_t idesc_lora = idesc_bf16_f32(128 * Cfg::kCtas, TM);
      uint32_t it = 0, tile_i = 0;
      bool ok = *abort_flag == 0;
      for (int t = tile0; t < num_tiles && ok; t += tile_step, ++tile_i) {
        const int ks = tile_ks(t);
        const int s0 = ks * p.stages_per_split;
        const int s1 = min(p.num_k_stages, s0 + p.stages_per_split);
        const int b = (Cfg::kAccBufs == 2) ? (tile_i & 1) : 0;
        const uint32_t aph = (Cfg::kAccBufs == 2) ? ((tile_i >> 1) & 1) : (tile_i & 1);
        if (!mbar_wait(&acc_empty[b], aph ^ 1, abort_flag, p.status, 2)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + b * Cfg::kAccCols;
        const int s_main = min(s1, p.main_k_stages);
        for (int kst = s0; kst < s_main; ++kst, ++it) {
          const int s = it % STAGES;
          const int as = it % Cfg::kASlots;
          if (!mbar_wait(&a_full[as], (it / Cfg::kASlots) & 1, abort_flag, p.status, 3)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_tmem = tmem_base + Cfg::kACol0 + as * 32;
          const uint64_t b_desc = smem_desc_sw128(smem_u32(sx + s * Cfg::kXStageBytes));
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint32_t acc = (kst > s0 || kk > 0) ? 1u : 0u;
            if constexpr (PAIR) mma_f16_ts_pair(d_tmem, a_tmem + kk * 8, b_desc + (uint64_t)(kk * 2), idesc_main, acc);
            else mma_f16_ts(d_tmem, a_tmem + kk * 8, b_desc + (uint64_t)(kk * 2), idesc_main, acc);
          }
          commit_all(&empty[s]);
          commit_all(&a_empty[as]);
        }
        for (int kst = max(s0, p.main_k_stages); kst < s1 && ok; ++kst, ++it) {  // LoRA: bf16 operands
          const int s = it % STAGES;
          const int as = it % Cfg::kASlots;
          if (!mbar_wait(&a_full[as], (it / Cfg::kASlots) & 1, abort_flag, p.status, 3)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_tmem = tmem_base + Cfg::kACol0 + as * 32;
          const uint64_t b_desc = smem_desc_sw128(smem_u32(sx + s * Cfg::kXStageBytes));
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint32_t acc = (kst > s0 || kk > 0) ? 1u : 0u;
            if constexpr (PAIR) mma_f16_ts_pair(d_tmem, a_tmem + kk * 8, b_desc + (uint64_t)(kk * 2), idesc_lora, acc);
            else mma_f16_ts(d_tmem, a_tmem + kk * 8, b_desc + (uint64_t)(kk * 2), idesc_lora, acc);
          }
          commit_all(&empty[s]);
          commit_all(&a_empty[as]);
        }
        if (!ok) break;
        commit_all(&acc_full[b]);
      }
      // Wait until every MMA this thread issued has completed before TMEM is released.
      if constexpr (PAIR) tc_commit_pair(cluster_map(drain, 0));
      else tc_commit(drain);
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
    for (int t = tile0; t < num_tiles && ok; t += tile_step) {
      const int nt = tile_nt(t);
      const int ks = tile_ks(t);
      const int s0 = ks * p.stages_per_split;
      const int s1 = min(p.num_k_stages, s0 + p.stages_per_split);
      const int n = nt * 128 + r;
      float rscale = 1.f;
      if (p.w_row_exp != nullptr && p.col_scale_kind == CS_EXP2 && qchk(BS_GEMM_BIAS, min(n, p.N - 1), p.N))
        rscale = exp2i(-p.w_row_exp[min(n, p.N - 1)]);
      const int s_main = min(s1, p.main_k_stages);
      for (int kst = s0; kst < s_main; ++kst, ++it) {
        if ((int)(it % Cfg::kDecGroups) != group) continue;
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1;
        if (!mbar_wait(&full[s], ph, abort_flag, p.status, 4)) { ok = false; break; }
        uint32_t a[32];
        Dec::decode(sw + s * kWStage, r, rscale, a);
        // the slot's previous weights have been consumed by their MMAs
        const int as = it % Cfg::kASlots;
        if (!mbar_wait(&a_empty[as], ((it / Cfg::kASlots) & 1) ^ 1, abort_flag, p.status, 8)) { ok = false; break; }
        tc_fence_after();
        tmem_st32(tmem_base + ((uint32_t)(quarter * 32) << 16) + Cfg::kACol0 + as * 32, a);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) arrive_leader(&a_full[as]);
      }
      for (int kst = max(s0, p.main_k_stages); kst < s1 && ok; ++kst, ++it) {
        if ((int)(it % Cfg::kDecGroups) != group) continue;
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1;
        if (!mbar_wait(&full[s], ph, abort_flag, p.status, 4)) { ok = false; break; }
        uint32_t a[32];  // LoRA stage: 64 bf16 values of this row of U', as stored
        const long long uoff = (long long)n * p.lora_k + (kst - p.main_k_stages) * 64;
        const uint4* u = reinterpret_cast<const uint4*>(p.lora_u + uoff);
        const bool u_in = qchk_span(BS_GEMM_LORA_U, uoff, 64, p.lim_lora_u);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint4 v = u_in ? __ldg(u + j) : make_uint4(0u, 0u, 0u, 0u);
          a[4 * j] = v.x; a[4 * j + 1] = v.y; a[4 * j + 2] = v.z; a[4 * j + 3] = v.w;
        }
        const int as = it % Cfg::kASlots;
        if (!mbar_wait(&a_empty[as], ((it / Cfg::kASlots) & 1) ^ 1, abort_flag, p.status, 8)) { ok = false; break; }
        tc_fence_after();
        tmem_st32(tmem_base + ((uint32_t)(quarter * 32) << 16) + Cfg::kACol0 + as * 32, a);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) arrive_leader(&a_full[as]);
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
    for (int t = tile0; t < num_tiles && epi_ok && *abort_flag == 0; t += tile_step, ++tile_i) {
      const int mt = t % p.m_tiles;
      const int nt = tile_nt(t);
      const int ks = tile_ks(t);
      const int b = (Cfg::kAccBufs == 2) ? (tile_i & 1) : 0;
      const uint32_t aph = (Cfg::kAccBufs == 2) ? ((tile_i >> 1) & 1) : (tile_i & 1);
      if (!mbar_wait(&acc_full[b], aph, abort_flag, p.status, 5)) break;
      tc_fence_after();
      const int n = nt * 128 + r;
      const bool n_ok = n < p.N;
      float cs = 1.f, bias = 0.f;
      if (p.k_splits == 1 && n_ok) {
        cs = load_colscale(p, n);
        if (p.lora_k > 0) cs = lora_safe_scale(cs);
        bias = load_bias(p.bias, p.bias_kind, n, p.N);
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
              if (qchk_align(BS_TMA_ALIGN, (long long)(mt * TM + c0) * 4, 16))
                tma_store_3d(&tmap_p, buf, mt * TM + c0, nt * 128, ks);
              bulk_commit();
            }
            ++epi_chunk;
          } else {
            if (n_ok && qchk_span(BS_GEMM_PARTIAL, ((long long)ks * p.N + n) * p.Mp + mt * TM + c0, TM, p.lim_partial)) {
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
        const float rs_lane = (p.x_row_exp != nullptr && mj < p.M && lane < kCh && qchk(BS_GEMM_XEXP, mj, p.M))
                                  ? exp2i(__ldg(&p.x_row_exp[mj])) : 1.f;
        tmem_wait_ld();
        if (p.out.ndst > 0) {
          // Stage the chunk as [kCh tokens][128 channels] 2-byte values, then copy whole 16-byte
          // pieces of token rows to every destination (or one TMA tensor store per destination).
          // Two buffers: the barrier after staging one also orders every thread's reads of the
          // other (or the TMA stores that read it, waited for by the issuer) before it is staged again.
          uint16_t* buf = reinterpret_cast<uint16_t*>(sepi + (epi_chunk & 1) * 8192);
          const bool use_tma = TM >= 32 && p.out.tma;
          const bool issuer = (warp == 2 + 4 * Cfg::kDecGroups) && lane == 0;
          if (use_tma) {
            if (issuer) bulk_wait_read<1>();  // the stores that last read this buffer are done with it
            if (!(epi_ok = epi_sync())) break;
          }
          if constexpr (ROT) {
            // fp32 chunk [kCh tokens][128 channels] in the upper half of the staging area (free on
            // this path), then each warp rotates whole token rows: lane l holds channels
            // 4l .. 4l+3, i.e. one 128-block, two 64-blocks or four 32-blocks of the row.
            float* frot = reinterpret_cast<float*>(sepi + 16384);
#pragma unroll
            for (int j = 0; j < kCh; ++j) {
              const float rs = __shfl_sync(0xffffffffu, rs_lane, j);
              if (qchk(BS_GEMM_SMEM, j * 128 + r, 4096)) frot[j * 128 + r] = __fadd_rn(__fmul_rn(__fmul_rn(__uint_as_float(v[j]), cs), rs), bias);
            }
            if (!(epi_ok = epi_sync())) break;
            constexpr int kRows = (kCh + 3) / 4;  // token rows of this warp: quarter, quarter + 4, ...
            float o4[kRows][4];
#pragma unroll
            for (int jj = 0; jj < kRows; ++jj) {
              const int j = jj * 4 + quarter;
              float4 t4 = make_float4(0.f, 0.f, 0.f, 0.f);
              if (j < kCh) t4 = *reinterpret_cast<const float4*>(frot + j * 128 + 4 * lane);
              o4[jj][0] = t4.x; o4[jj][1] = t4.y; o4[jj][2] = t4.z; o4[jj][3] = t4.w;
            }
            rows_hadamard4<kRows>(o4, p.rot_group, lane);  // the rows' butterfly chains overlap
#pragma unroll
            for (int jj = 0; jj < kRows; ++jj) {
              const int j = jj * 4 + quarter;
              if (j < kCh) {
                const uint32_t w0 = p.y_dtype == OUT_BF16 ? pack_bf16x2(o4[jj][0], o4[jj][1]) : pack_f16x2(o4[jj][0], o4[jj][1]);
                const uint32_t w1 = p.y_dtype == OUT_BF16 ? pack_bf16x2(o4[jj][2], o4[jj][3]) : pack_f16x2(o4[jj][2], o4[jj][3]);
                if (qchk_span(BS_GEMM_SMEM, j * 128 + 4 * lane, 4, 4096))
                  *reinterpret_cast<uint2*>(buf + j * 128 + 4 * lane) = make_uint2(w0, w1);
              }
            }
          } else {
#pragma unroll
            for (int j = 0; j < kCh; ++j) {
              const float rs = __shfl_sync(0xffffffffu, rs_lane, j);
              float o = __fmul_rn(__fmul_rn(__uint_as_float(v[j]), cs), rs);
              o = __fadd_rn(o, bias);
              if (qchk(BS_GEMM_SMEM, j * 128 + r, 4096))
                buf[j * 128 + r] = p.y_dtype == OUT_BF16 ? __bfloat16_as_ushort(__float2bfloat16_rn(o))
                                                       : __half_as_ushort(__float2half_rn(o));
            }
          }
          if (use_tma) {
            fence_proxy_async_smem();
            if (!(epi_ok = epi_sync())) break;
            if (issuer) {
#pragma unroll
              for (int d = 0; d < kMaxPeers; ++d)
                if (d < p.out.ndst && qchk_align(BS_TMA_ALIGN, (long long)nt * 128 * 2, 16))
                tma_store_2d(&out_maps.m[d], buf, nt * 128, mt * TM + c0);
              bulk_commit();
            }
            ++epi_chunk;
            continue;
          }
          if (!(epi_ok = epi_sync())) break;
#pragma unroll
          for (int i = etid; i < kCh * 16; i += 128) {
            const int m = mt * TM + c0 + (i >> 4);
            const int n0 = nt * 128 + (i & 15) * 8;
            if (m < p.M && n0 < p.N) {
              const uint4 val = reinterpret_cast<const uint4*>(buf)[i];
              const long long off = (long long)m * p.ldy + n0;
              if (qchk_span(BS_GEMM_PEER, off, 8, p.lim_y)) {
#pragma unroll
                for (int d = 0; d < kMaxPeers; ++d)
                  if (d < p.out.ndst) reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(p.out.dst[d]) + off)[0] = val;
              }
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
            store_out(p.y, p.y_dtype, (long long)m * p.ldy + n, o, p.lim_y);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) arrive_leader(&acc_empty[b]);
    }
    if (warp == 2 + 4 * Cfg::kDecGroups && lane == 0) {
      bulk_wait_all();  // partial / output tensor stores complete
      fence_proxy_async_global();
    }
  }

  // Warps 0 and 1 ran their loops on one elected lane; reconverge before the block barrier
  // (barrier.sync is .aligned) and before the warp-wide TMEM dealloc.
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  // A pair: the even CTA's MMAs (which write the odd CTA's TMEM and read its shared memory) have
  // all completed once its issuer's drain wait returned; neither CTA frees TMEM or exits before.
  if constexpr (PAIR) cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR) tmem_dealloc_pair(tmem_base, Cfg::kTmemCols);
    else tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
  if (p.out.signal && threadIdx.x == 0) peer_signal_last_cta(p.out);
}

template <class Dec, int TM, int STAGES, bool PAIR>
constexpr int qgemm_f16_smem_bytes() {
  constexpr int kWStage = (Dec::kStageBytes + 1023) / 1024 * 1024;
  return 1024 /*align slack*/ + STAGES * (F16Cfg<TM, STAGES, PAIR>::kXStageBytes + kWStage) +
         1024 /*barriers, aligned*/ + 2 * 16384;
}

// Deepest shared-memory ring (at most 8 stages) that fits the 227 KB a CTA may use.
template <class Dec, int TM, bool PAIR>
constexpr int qgemm_f16_stages() {
  constexpr int kWStage = (Dec::kStageBytes + 1023) / 1024 * 1024;
  constexpr int fit = (232448 - 1024 - 1024 - 2 * 16384) / ((PAIR ? TM / 2 : TM) * 128 + kWStage);
  return fit < 8 ? fit : 8;
}

}  // namespace qlin
