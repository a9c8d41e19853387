// W4A8 / W6A8 on pairs of SMs (tcgen05.mma.cta_group::2.kind::i8, int32 accumulation).
//
//   Y[m, n] = sx[m] * inv * sum_g s[n, g] * P_g[m, n]  (+ bias[n]),
//   P_g[m, n] = sum_{k in group g} xq[m, k] * wq'[n, k]   (exact int32)
//
// Same arithmetic as qgemm_i8_kernel (qlin_gemm_i8.cuh); this kernel is built for the pace of the
// tensor core on large token counts.  Measured on B200: a single thread issues every MMA of a CTA,
// and each observed commit (an accumulator handed to the rescale warps and back) costs a fixed
// few hundred clocks that more accumulator buffers do not hide at 128-token MMAs.  So the work
// behind each issued instruction and each observed commit is made as large as the exact
// per-group sums allow:
//   * the two CTAs of a cluster share cta_group::2 MMAs of 256 weight rows (128 decoded into each
//     CTA's shared memory, the SS form) by TN tokens (TN/2 loaded into each CTA), issued by one
//     thread for both SMs;
//   * TN = 256 with two int32 accumulator buffers (all 512 TMEM columns) for groups of 128 values
//     or more: one observed commit per 4 MMAs of 256 x 256 x 32 per group of 128;
//   * TN = 128 with four buffers for groups of 64: the two groups of a 128-deep stage go to two
//     buffers behind one commit.
// The first MMA of a group overwrites its buffer; the rescale hands the buffer back as soon as
// its last columns are in registers and folds s[n, g] * P into fp32 registers with one exact
// int32 -> fp32 conversion per value and one packed fma per two values (ffma2_cvt).  Measured
// alternatives: the magic-number conversion (P plus the bit pattern of 1.5 * 2^23 with an integer
// add, then an exact packed subtraction) was 15-25% slower, the extra FMA-pipe subtraction being
// on the bound path; re-biasing the buffers in TMEM instead of the integer add measured 1.7x slower
// (the stores and their completion wait sit on the buffer's round trip back to the issuer).
//
// Warp roles (512 threads, one CTA per SM, persistent over tiles; registers rebalanced per
// warpgroup with setmaxnreg: 40 / 72 / 200 / 200 per thread, 65,536 in all):
//   warpgroup 0: warp 0 TMA producer, warp 1 TMEM allocator + MMA issuer (even CTA), warps 2-3 idle
//   warpgroup 1: decoders, one weight row per thread: packed stage -> 128 int8 (the activation
//                prologue's column order) -> the 128-byte-swizzled A tile in shared memory
//   warpgroups 2-3: rescale + epilogue, two warps per TMEM lane quarter, TN/2 columns each
#pragma once
#include <cuda.h>

#include "qlin_gemm_i8.cuh"

namespace qlin {

template <int TN, int GPS>
struct I8PCfg {
  static constexpr int kThreads = 512;
  static constexpr int kNB = 512 / TN;          // int32 accumulator buffers in TMEM
  static constexpr int kNBatch = kNB / GPS;     // buffers handed over per commit: GPS
  static constexpr int kXRows = TN / 2;         // tokens this CTA loads per stage
  static constexpr uint32_t kXStage = kXRows * 128;
  static constexpr uint32_t kAStage = 128 * 128;  // 128 weight rows x 128 int8
  static constexpr int kCols = TN / 2;          // accumulator columns per rescale warp
  static_assert(TN == 128 || TN == 256, "token tiles of 128 or 256");
  static_assert(GPS == 1 || (GPS == 2 && TN == 128), "two groups per stage need four buffers");
};

__device__ __forceinline__ void mma_i8_ss_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

template <int N>
__device__ __forceinline__ void setmaxnreg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void setmaxnreg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

template <class Dec, int TN, int GPS, int STAGES>
__global__ void __launch_bounds__(512, 1)
qgemm_i8p_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                 const GemmI8Params p) {
  using Cfg = I8PCfg<TN, GPS>;
  constexpr uint32_t kWStage = (Dec::kStageBytes + 1023) / 1024 * 1024;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sx = smem;                                // STAGES x kXStage
  uint8_t* sa = sx + STAGES * Cfg::kXStage;          // STAGES x kAStage (decoded weights)
  uint8_t* sw = sa + STAGES * Cfg::kAStage;          // STAGES x kWStage (packed weights)
  uint64_t* bars = reinterpret_cast<uint64_t*>(sw + STAGES * kWStage);
  uint64_t* full = bars;                        // [STAGES] X + W landed (this CTA)
  uint64_t* empty = full + STAGES;              // [STAGES] MMAs that read the stage completed (this CTA)
  uint64_t* a_full = empty + STAGES;            // [STAGES] decoded A of both CTAs written (even CTA's)
  uint64_t* acc_full = a_full + STAGES;         // [kNBatch] accumulators ready (this CTA)
  uint64_t* acc_empty = acc_full + Cfg::kNBatch;  // [kNBatch] read out by the rescale warps of both CTAs (even CTA's)
  uint64_t* drain = acc_empty + Cfg::kNBatch;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int n_pairs = (p.N + 255) / 256;
  const int num_tiles = p.m_tiles * n_pairs;
  const int tile0 = blockIdx.x >> 1;
  const int tile_step = gridDim.x >> 1;
  const int nks = p.num_k_stages;
  const int gs = p.group >= 128 ? p.group / 128 : 1;  // stages per group (GPS == 1)
  const int groups = p.groups_per_row;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&a_full[s], 4 * 2);
    }
    for (int b = 0; b < Cfg::kNBatch; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 8 * 2);
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
    tmem_alloc_pair(tmem_slot, 512);
    tmem_relinquish_pair();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmap_x);
    if constexpr (Dec::kTma) prefetch_tmap(&tmap_w);
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers are initialized before any remote arrive
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp < 4) {
    setmaxnreg_dec<40>();
    if (warp == 0) {
      // ------------------------------------------------------------------- producer (both CTAs)
      if (elect_one()) {
        uint32_t it = 0;
        bool ok = true;
        for (int t = tile0; t < num_tiles && ok; t += tile_step) {
          const int mt = t % p.m_tiles;
          const int nt = (t / p.m_tiles) * 2 + (int)rank;  // this CTA's 128-row weight tile
          for (int kst = 0; kst < nks; ++kst, ++it) {
            const int s = it % STAGES;
            if (!mbar_wait(&empty[s], ((it / STAGES) & 1) ^ 1, abort_flag, p.status, 0x21)) { ok = false; break; }
            mbar_arrive_expect_tx(&full[s], Cfg::kXStage + Dec::kStageBytes);
            tma_load_2d(sx + s * Cfg::kXStage, &tmap_x, &full[s], kst * 128, mt * TN + (int)rank * Cfg::kXRows);
            if constexpr (Dec::kTma) {
              tma_load_2d(sw + s * kWStage, &tmap_w, &full[s], kst * 64, nt * 128);
            } else {
              const long long off = ((long long)nt * nks + kst) * Dec::kStageBytes;
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
      // ------------------------------------------------------------------- MMA issuer (even CTA)
      if (leader && elect_one()) {
        constexpr uint32_t idesc = idesc_s8_s32(256, TN);
        const uint32_t sx_u = smem_u32(sx), sa_u = smem_u32(sa);
        uint32_t it = 0, bc = 0;
        bool ok = true;
        for (int t = tile0; t < num_tiles && ok; t += tile_step) {
          int gk = 0;
          for (int kst = 0; kst < nks; ++kst, ++it) {
            const int s = it % STAGES;
            if (!mbar_wait(&a_full[s], (it / STAGES) & 1, abort_flag, p.status, 0x22)) { ok = false; break; }
            tc_fence_after();
            const uint64_t a_desc = smem_desc_sw128(sa_u + s * Cfg::kAStage);
            const uint64_t b_desc = smem_desc_sw128(sx_u + s * Cfg::kXStage);
            const uint32_t bt = bc % Cfg::kNBatch;
            if (GPS == 2 || gk == 0) {  // first MMA of a batch: its (re-biased) buffers are free
              if (!mbar_wait(&acc_empty[bt], (bc / Cfg::kNBatch) & 1, abort_flag, p.status, 0x23)) {
                ok = false;
                break;
              }
              tc_fence_after();
            }
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint32_t buf = GPS == 2 ? bt * 2 + (kk >> 1) : bt;
              // the first MMA of a group overwrites its buffer
              const uint32_t accum = GPS == 2 ? (uint32_t)(kk & 1) : (uint32_t)(gk > 0 || kk > 0);
              mma_i8_ss_pair(tmem_base + buf * TN, a_desc + (uint64_t)(kk * 2), b_desc + (uint64_t)(kk * 2), idesc,
                             accum);
            }
            if (GPS == 2 || ++gk == gs) {
              tc_commit_pair(cluster_map(&acc_full[bt], 0));
              tc_commit_pair(cluster_map(&acc_full[bt], 1));
              ++bc;
              gk = 0;
            }
            tc_commit_pair(cluster_map(&empty[s], 0));
            tc_commit_pair(cluster_map(&empty[s], 1));
          }
        }
        tc_commit_pair(cluster_map(drain, 0));
        const uint64_t t0 = globaltimer();
        while (!mbar_try_wait(smem_u32(drain), 0)) {
          if (globaltimer() - t0 > QLIN_WAIT_TIMEOUT_NS) break;
        }
      }
    }
  } else if (warp < 8) {
    // --------------------------------------------------------------------- decoders (both CTAs)
    setmaxnreg_dec<72>();
    const int r = threadIdx.x - 128;  // weight row within this CTA's tile
    const uint32_t a_full_leader = cluster_map(a_full, 0);
    uint32_t it = 0;
    bool ok = true;
    for (int t = tile0; t < num_tiles && ok; t += tile_step) {
      for (int kst = 0; kst < nks; ++kst, ++it) {
        const int s = it % STAGES;
        if (!mbar_wait(&full[s], (it / STAGES) & 1, abort_flag, p.status, 0x24)) { ok = false; break; }
        uint32_t a[32];
        Dec::decode(sw + s * kWStage, r, a);
        uint8_t* row = sa + s * Cfg::kAStage + r * 128;
        if (qchk_smem(BS_I8_SMEM, smem_raw, row, 128) && qchk(BS_I8_SMEM, (row - sa) + 128, sw - sa + 1)) {
#pragma unroll
          for (int ch = 0; ch < 8; ++ch)
            *reinterpret_cast<uint4*>(row + ((ch ^ (r & 7)) << 4)) = make_uint4(a[4 * ch], a[4 * ch + 1],
                                                                              a[4 * ch + 2], a[4 * ch + 3]);
        }
        fence_proxy_async_smem();  // the MMA reads the tile through the async proxy
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(a_full_leader + (uint32_t)(s * 8));
      }
    }
  } else {
    // --------------------------------------------------------------------- rescale + epilogue
    setmaxnreg_inc<200>();
    constexpr int kCols = Cfg::kCols;
    const int quarter = warp & 3;
    const int part = (warp - 8) >> 2;
    const int r = quarter * 32 + lane;  // TMEM lane == weight row within this CTA's tile
    const uint32_t lanes = (uint32_t)(quarter * 32) << 16;
    // The same arithmetic either way; at 256 tokens groups above 128 values take the scalar FMA,
    // a form with which ptxas fits the 128 running sums with fewer spills (measured: 0.33 against
    // 0.43 ms at configuration 3), while the 128-token kernels run fastest with the packed form
    // alone (0.66 against 0.72 ms at configuration 4).
    const bool paired = p.group <= 128;
    const uint32_t acc_empty_leader = cluster_map(acc_empty, 0);
    // release each batch once so its first use can start
    if (lane == 0)
      for (int b = 0; b < Cfg::kNBatch; ++b) mbar_arrive_cluster(acc_empty_leader + (uint32_t)(b * 8));
    uint32_t bc = 0;
    bool ok = true;
    for (int t = tile0; t < num_tiles && ok; t += tile_step) {
      const int mt = t % p.m_tiles;
      const int nt = (t / p.m_tiles) * 2 + (int)rank;
      const int n = nt * 128 + r;
      const bool n_ok = n < p.N;
      float accf[kCols];
#pragma unroll
      for (int j = 0; j < kCols; ++j) accf[j] = 0.f;
      const unsigned short* gscale =
          reinterpret_cast<const unsigned short*>(p.scales) + (size_t)min(n, p.N - 1) * p.groups_per_row;
      const bool group_scales = p.scale_kind == I8S_GROUP_F16;
      const long long gbase = (long long)min(n, p.N - 1) * p.groups_per_row;
      const float s_channel =
          (n_ok && !group_scales && qchk(BS_I8_SCALE, n, p.lim_scales)) ? reinterpret_cast<const float*>(p.scales)[n] : 0.f;
      // the next group's scale stays raw (a load in flight across a whole group) until it is used
      unsigned short s_raw =
          (n_ok && group_scales && qchk(BS_I8_SCALE, gbase, p.lim_scales)) ? __ldg(gscale) : (unsigned short)0;
      for (int g = 0; g < groups; ++g) {
        const float sg = group_scales ? __half2float(__ushort_as_half(s_raw)) : s_channel;
        if (n_ok && group_scales && g + 1 < groups && qchk(BS_I8_SCALE, gbase + g + 1, p.lim_scales))
          s_raw = __ldg(gscale + g + 1);
        const uint32_t bt = bc % Cfg::kNBatch;
        const int sub = GPS == 2 ? (g & 1) : 0;
        if (sub == 0) {
          if (!mbar_wait(&acc_full[bt], (bc / Cfg::kNBatch) & 1, abort_flag, p.status, 0x25)) {
            ok = false;
            break;
          }
          tc_fence_after();
        }
        const uint32_t taddr = tmem_base + lanes + (bt * GPS + sub) * TN + part * kCols;
        // kChunk columns per TMEM round trip (64 at TN = 128: two loads, one wait; 32 at TN = 256,
        // where 128 running sums leave no registers for more); the batch's buffers go back to the
        // issuer as soon as their last values are in registers, before the arithmetic
        constexpr int kChunk = TN == 256 ? 32 : 64;
#pragma unroll
        for (int c0 = 0; c0 < kCols; c0 += kChunk) {
          uint32_t v[kChunk];
          tmem_ld32(taddr + c0, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
          if constexpr (kChunk == 64) tmem_ld32(taddr + c0 + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
          tmem_wait_ld();
          if (c0 + kChunk >= kCols && sub == GPS - 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(acc_empty_leader + (uint32_t)(bt * 8));
          }
          if (TN == 128 || paired) {
#pragma unroll
            for (int j = 0; j < kChunk; j += 2) ffma2_cvt(sg, v[j], v[j + 1], accf[c0 + j], accf[c0 + j + 1]);
          } else {
#pragma unroll
            for (int j = 0; j < kChunk; ++j) accf[c0 + j] = fmaf(sg, (float)(int32_t)v[j], accf[c0 + j]);
          }
        }
        if (sub == GPS - 1) {
          ++bc;
        }
      }
      if (!ok) break;
      const float bias = n_ok ? load_bias_i8(p.bias, p.bias_kind, n, p.N) : 0.f;
#pragma unroll
      for (int c0 = 0; c0 < kCols; c0 += 32) {
        const int m0 = mt * TN + part * kCols + c0;
        const float sx_lane =
            (m0 + lane < p.M && qchk(BS_I8_SCALE, m0 + lane, p.M)) ? __ldg(&p.x_scale[m0 + lane]) * p.inv_scale : 0.f;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
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
  // The even CTA's MMAs (which write the odd CTA's TMEM and read its shared memory) have all
  // completed once its issuer's drain wait returned; neither CTA frees TMEM or exits before.
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, 512);
  }
}

template <class Dec, int TN, int STAGES>
constexpr int qgemm_i8p_smem_bytes() {
  constexpr int kWStage = (Dec::kStageBytes + 1023) / 1024 * 1024;
  return 1024 + STAGES * ((TN / 2) * 128 + 128 * 128 + kWStage) + 1024;
}

// Deepest ring (at most 6 stages) that fits the 227 KB a CTA may use.
template <class Dec, int TN>
constexpr int qgemm_i8p_stages() {
  constexpr int kWStage = (Dec::kStageBytes + 1023) / 1024 * 1024;
  constexpr int fit = (232448 - 2048) / ((TN / 2) * 128 + 128 * 128 + kWStage);
  return fit < 6 ? fit : 6;
}

}  // namespace qlin
