// Instantiations and host launcher of the weight-only (kind::f16) fused dequantize + GEMM.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "qlin_f16_launch.cuh"

namespace qlin {

// Device status word written by timed-out waits in every kernel of this library.
__device__ DeviceStatus g_status;

void* device_status_ptr() {
  // Looked up once per CUDA context (keyed by the context's unique id, so a context created after
  // cudaDeviceReset, or a non-primary context the caller made current, gets its own lookup).
  static std::mutex mu;
  struct Entry {
    unsigned long long ctx;
    void* addr;
  };
  static Entry cache[64] = {};
  static int next = 0;
  std::lock_guard<std::mutex> lock(mu);
  unsigned long long id = current_context_id();
  if (id != 0)
    for (const Entry& e : cache)
      if (e.ctx == id) return e.addr;
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_status) != cudaSuccess) return nullptr;  // also makes the context current
  if (id == 0) id = current_context_id();
  if (id != 0) {
    cache[next] = Entry{id, p};
    next = (next + 1) % 64;
  }
  return p;
}

int sm_count() {
  static int cache[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && cache[dev] == 0) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = v > 0 ? v : 148;
  }
  return (dev >= 0 && dev < 64) ? cache[dev] : 148;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link needed).
typedef CUresult (*PFN_encodeTiled_t)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                      const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                      CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static PFN_encodeTiled_t encode_fn() {
  static PFN_encodeTiled_t fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_encodeTiled_t>(p);
  });
  return fn;
}

// 2-D tile map over a row-major matrix [rows, cols] of `elem` bytes with row pitch `pitch_bytes`.
int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elem, uint64_t cols, uint64_t rows,
                 uint64_t pitch_bytes, uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle swz) {
  PFN_encodeTiled_t fn = encode_fn();
  if (fn == nullptr) {
    set_error("cuTensorMapEncodeTiled is unavailable");
    return 3;
  }
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || pitch_bytes % 16 != 0) {
    set_error("TMA operand needs a 16-byte aligned base and row pitch (pitch %llu bytes)",
              (unsigned long long)pitch_bytes);
    return 1;
  }
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {pitch_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  (void)elem;
  CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d): cols %llu rows %llu pitch %llu box %u x %u", (int)r,
              (unsigned long long)cols, (unsigned long long)rows, (unsigned long long)pitch_bytes, box_cols, box_rows);
    return 3;
  }
  return 0;
}

// 3-D tile map over a dense [d2][d1][d0] array of `elem`-byte elements (d0 contiguous).
int make_tmap_3d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elem, uint64_t d0, uint64_t d1,
                 uint64_t d2, uint32_t b0, uint32_t b1, CUtensorMapSwizzle swz) {
  PFN_encodeTiled_t fn = encode_fn();
  if (fn == nullptr) {
    set_error("cuTensorMapEncodeTiled is unavailable");
    return 3;
  }
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {d0 * elem, d0 * d1 * elem};
  cuuint32_t box[3] = {b0, b1, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || strides[0] % 16 != 0) {
    set_error("TMA store target needs 16-byte alignment");
    return 1;
  }
  CUresult r = fn(map, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled (3-D) failed (%d)", (int)r);
    return 3;
  }
  return 0;
}

// 3-D tile map with explicit byte strides: dims {d0, d1, d2}, d0 contiguous.
int make_tmap_3d_strided(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elem, uint64_t d0,
                         uint64_t d1, uint64_t d2, uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t b0,
                         uint32_t b1, CUtensorMapSwizzle swz) {
  PFN_encodeTiled_t fn = encode_fn();
  if (fn == nullptr) {
    set_error("cuTensorMapEncodeTiled is unavailable");
    return 3;
  }
  (void)elem;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || stride1_bytes % 16 != 0 || stride2_bytes % 16 != 0) {
    set_error("TMA operand needs a 16-byte aligned base and strides (row pitch %llu, slab stride %llu bytes)",
              (unsigned long long)stride1_bytes, (unsigned long long)stride2_bytes);
    return 1;
  }
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
  cuuint32_t box[3] = {b0, b1, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled (3-D) failed (%d): %llu x %llu x %llu", (int)r, (unsigned long long)d0,
              (unsigned long long)d1, (unsigned long long)d2);
    return 3;
  }
  return 0;
}

uint32_t gguf_stage_bytes(int qtype, int* P, int* S) {
  int p = 0, s = 0;
  switch (qtype) {
    case WF_Q8_0: p = 4; s = 4; break;
    case WF_Q4_0:
    case WF_IQ4_NL:
    case WF_IQ4_XS: p = 2; s = 4; break;
    case WF_Q4_1:
    case WF_Q4_K: p = 2; s = 8; break;
    case WF_Q5_0: p = 2; s = 12; break;
    case WF_Q5_1:
    case WF_Q5_K: p = 2; s = 16; break;
    case WF_Q2_K: p = 1; s = 8; break;
    case WF_Q3_K: p = 1; s = 16; break;
    case WF_Q6_K: p = 4; s = 8; break;
    default: return 0;
  }
  if (P) *P = p;
  if (S) *S = s;
  return 128u * (16u * p + s);
}

int gguf_block_values(int qtype) {
  switch (qtype) {
    case WF_Q4_0: case WF_Q4_1: case WF_Q5_0: case WF_Q5_1: case WF_Q8_0: case WF_IQ4_NL: return 32;
    case WF_Q2_K: case WF_Q3_K: case WF_Q4_K: case WF_Q5_K: case WF_Q6_K: case WF_IQ4_XS: return 256;
    default: return 0;
  }
}

int gguf_type_size(int qtype) {
  switch (qtype) {
    case WF_Q4_0: case WF_IQ4_NL: return 18;
    case WF_Q4_1: return 20;
    case WF_Q5_0: return 22;
    case WF_Q5_1: return 24;
    case WF_Q8_0: return 34;
    case WF_Q2_K: return 84;
    case WF_Q3_K: return 110;
    case WF_Q4_K: return 144;
    case WF_Q5_K: return 176;
    case WF_Q6_K: return 210;
    case WF_IQ4_XS: return 136;
    default: return 0;
  }
}

// Pairs of CTAs (cta_group::2 MMAs, half the activation tile per SM) for token tiles of 128 and
// more, when the weight tiles pair up.  Tuning knob: QLIN_PAIR=0 keeps single-CTA MMAs for sweeps.
static bool use_pair(int tm, int n_tiles) {
  static const bool enabled = [] {
    const char* e = getenv("QLIN_PAIR");
    return !(e && atoi(e) == 0);
  }();
  return enabled && tm >= 128 && n_tiles % 2 == 0;
}

// Relative decode cost of a 64-deep stage per format (the 4-bit formats are the unit; measured at
// configuration-2 shape: the formats that insert a fifth / third bit are ~4% slower, the IQ4
// codebook lookups ~25%).
static double fmt_stage_cost(int fmt) {
  switch (fmt) {
    case WF_IQ4_NL: case WF_IQ4_XS: return 1.12;
    case WF_Q5_0: case WF_Q5_1: case WF_Q5_K: case WF_Q3_K: return 1.04;
    case WF_Q2_K: case WF_Q8_0: case WF_Q6_K: return 1.02;
    default: return 1.0;
  }
}

// Modelled time of one plan (microseconds at the boost clock), from measured per-stage costs of
// the persistent kernel on B200: a 64-deep K stage of one tile costs c(TM), the 256-token tile
// (single-buffered accumulator) adds an exposed epilogue per tile, the format scales the stage cost
// (fmt_stage_cost), and a K split adds the finalize pass over the fp32 partials.
static double plan_cost(int M, int N, int kst, int fmt, int tm, int splits, int sms) {
  const int n_tiles = (N + 127) / 128;
  const bool pair = use_pair(tm, n_tiles);
  const long long units = (long long)((M + tm - 1) / tm) * (pair ? n_tiles / 2 : n_tiles) * splits;
  const int slots = pair ? sms / 2 : sms;
  const long long waves = (units + slots - 1) / slots;
  double c = tm <= 64 ? 0.30 : tm == 128 ? 0.33 : tm == 192 ? 0.38 : 0.45;
  if (!pair) c *= 1.03;
  c *= fmt_stage_cost(fmt);
  const double epi = tm == 256 ? 6.0 : 0.0;
  const int per = (kst + splits - 1) / splits;
  double t = (double)waves * (per * c + epi);
  if (splits > 1) t += ((double)splits * N * M * 4 + (double)N * M * 2) / 5.0e6 + 3.0;
  return t;
}

// Token tile and K-split plan.  M <= 256: the smallest tile that holds M and K split across
// CTAs until the grid covers the SMs.  Larger M: the tile (128 / 192 / 256) and split with the
// lowest modelled time, which weighs per-stage cost against wave quantization on the SMs.
void plan_f16(int M, int N, int K, int fmt, int* tm_out, int* splits_out) {
  int tm = *tm_out;
  // Tuning knob: QLIN_TM forces the token tile (16, 32, 64, 128, 192 or 256) for sweeps.
  if (tm == 0) {
    static const int forced = [] {
      const char* e = getenv("QLIN_TM");
      return e ? atoi(e) : 0;
    }();
    if (forced == 16 || forced == 32 || forced == 64 || forced == 128 || forced == 192 || forced == 256) tm = forced;
  }
  int splits = *splits_out;
  const int kst = (K + 63) / 64;
  if (splits == 0) {
    // Tuning knob: QLIN_SPLITS forces the number of K splits for sweeps.
    static const int forced_splits = [] {
      const char* e = getenv("QLIN_SPLITS");
      return e ? atoi(e) : 0;
    }();
    if (forced_splits > 0) splits = forced_splits;
  }
  const int sms = sm_count();
  if (tm == 0 && M > 256) {
    double best = 1e30;
    int best_tm = 192, best_splits = 1;
    for (int cand : {128, 192, 256}) {
      for (int sp = 1; sp <= 4; ++sp) {
        if (splits != 0 && sp != splits) continue;
        if (sp > 1 && kst / sp < 8) break;
        const double t = plan_cost(M, N, kst, fmt, cand, sp, sms);
        if (t < best) {
          best = t;
          best_tm = cand;
          best_splits = sp;
        }
      }
    }
    tm = best_tm;
    if (splits == 0) splits = best_splits;
  }
  if (tm == 0) {
    if (M <= 16) tm = 16;
    else if (M <= 32) tm = 32;
    else if (M <= 64) tm = 64;
    else if (M <= 128) tm = 128;
    else tm = 256;  // one token tile; the grid is filled by splitting K
  }
  if (splits == 0) {
    // Fewer output tiles than SMs: split K.  The CTAs are persistent over (tile, split) units, so
    // the time goes as rounds x stages per split, ceil(tiles * s / sms) * ceil(kst / s), plus a
    // fixed cost for the finalize pass once s > 1 (about five stages' time).  The plain rule
    // s = sms / tiles left a third of the SMs idle at 96 tiles (M = 16, N = 12288); measured there:
    // 20.6 us with one split against ~14 us with three.
    const int tiles = ((N + 127) / 128) * ((M + tm - 1) / tm);
    splits = 1;
    if (tiles < sms) {
      const int max_s = std::min(16, std::max(1, kst / 4));  // keep >= 4 stages per split
      long best = (long)kst;
      for (int sp = 2; sp <= max_s; ++sp) {
        const long cost = (long)((tiles * sp + sms - 1) / sms) * ((kst + sp - 1) / sp) + 5;
        if (cost < best) {
          best = cost;
          splits = sp;
        }
      }
    }
  }
  splits = std::max(1, std::min(splits, kst));
  // normalize so every split has work
  const int per = (kst + splits - 1) / splits;
  splits = (kst + per - 1) / per;
  *tm_out = tm;
  *splits_out = splits;
}

size_t f16_gemm_partial_bytes(int M, int N, int K, int fmt, int tm, int k_splits) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;  // nothing to plan (the callers return before any launch)
  plan_f16(M, N, K, fmt, &tm, &k_splits);
  const size_t mp = (size_t)(M + tm - 1) / tm * tm;
  return k_splits > 1 ? (size_t)k_splits * N * mp * sizeof(float) : 0;
}



// Whole 16-byte pieces of 2-byte output rows can be stored from the shared-memory staging tile.
// Tuning knob: QLIN_STAGED_OUT=0 keeps per-element stores for sweeps.
static bool staged_output_ok(const F16GemmArgs& a) {
  static const bool enabled = [] {
    const char* e = getenv("QLIN_STAGED_OUT");
    return !(e && atoi(e) == 0);
  }();
  return enabled && (a.y_dtype == OUT_F16 || a.y_dtype == OUT_BF16) && a.N % 8 == 0 && a.ldy % 8 == 0 &&
         (reinterpret_cast<uintptr_t>(a.y) & 15) == 0;
}

bool f16_gemm_can_rotate(const F16GemmArgs& a) {
  static const bool disabled = [] {
    const char* e = getenv("QLIN_NO_ROT_EPILOGUE");  // tuning knob: rotate in a separate pass
    return e && atoi(e) != 0;
  }();
  if (disabled || a.fmt != WF_INT8 || a.out != nullptr || a.lora_k != 0 || a.M <= 1 || a.N == 0 ||
      (a.rot_group != 32 && a.rot_group != 64 && a.rot_group != 128) || !staged_output_ok(a))
    return false;
  int tm = a.tm, splits = a.k_splits;
  plan_f16(a.M, a.N, a.K, a.fmt, &tm, &splits);
  return splits == 1;
}

int run_f16_gemm(const F16GemmArgs& a, cudaStream_t stream) {
  if (a.M == 0 || a.N == 0) return 0;
  if (a.M == 1 && a.lora_k == 0 && a.rot_group == 0) {
    const int rc = run_gemv(a, stream);
    if (rc >= 0) return rc;
  }
  int tm = a.tm, splits = a.k_splits;
  plan_f16(a.M, a.N, a.K + a.lora_k, a.fmt, &tm, &splits);
  GemmParams p{};
  p.M = a.M;
  p.N = a.N;
  p.K = a.K;
  p.main_k_stages = (a.K + 63) / 64;
  p.num_k_stages = p.main_k_stages + a.lora_k / 64;
  p.lora_u = reinterpret_cast<const __nv_bfloat16*>(a.lora_u_ptr);
  p.lora_k = a.lora_k;
  p.m_tiles = (a.M + tm - 1) / tm;
  p.n_tiles = (a.N + 127) / 128;
  p.k_splits = splits;
  p.stages_per_split = (p.num_k_stages + splits - 1) / splits;
  p.w_stages = reinterpret_cast<const uint8_t*>(a.w);
  p.w_row_exp = a.w_row_exp;
  p.col_scale = a.col_scale;
  p.col_scale_kind = a.col_scale_kind;
  p.x_row_exp = a.x_row_exp;
  p.bias = a.bias;
  p.bias_kind = a.bias_kind;
  p.y = a.y;
  p.y_dtype = a.y_dtype;
  p.ldy = a.ldy;
  p.rot_group = a.rot_group;
  p.partial = nullptr;
  p.status = reinterpret_cast<DeviceStatus*>(device_status_ptr());
  p.Mp = p.m_tiles * tm;
  p.lim_y = (long long)(a.M - 1) * a.ldy + a.N;
  p.lim_w_bytes = a.w_bytes;
  p.lim_partial = (long long)(a.partial_bytes / sizeof(float));
  p.lim_lora_u = (long long)p.n_tiles * 128 * a.lora_k;
  PeerMaps maps;
  memset(&maps, 0, sizeof(maps));
  if (a.out != nullptr) {
    p.out = *a.out;
    if (splits > 1) {
      p.out.ndst = 0;  // the GEMM writes partials; the finalize kernel stores the output and signals
      p.out.signal = 0;
      p.out.tma = 0;
    } else if (p.out.tma) {
      if (a.out_maps == nullptr || tm < 32) p.out.tma = 0;
      else maps = *a.out_maps;
    }
  } else if (splits == 1 && staged_output_ok(a)) {
    // the staged output goes out as one TMA tensor store per 32-token chunk (box 128 channels x 32
    // tokens) instead of 16-byte stores from every epilogue thread: 3-6 % faster GEMMs at the
    // configuration-2 and -5 shapes (same-box A/B)
    p.out.ndst = 1;
    p.out.dst[0] = a.y;
    if (tm >= 32 && make_tmap_2d(&maps.m[0], a.y, a.y_dtype == OUT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                                       : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                                 2, (uint64_t)a.N, (uint64_t)a.M, (uint64_t)a.ldy * 2, 128, 32,
                                 CU_TENSOR_MAP_SWIZZLE_NONE) == 0)
      p.out.tma = 1;
  }
  if (splits > 1) {
    const size_t need = (size_t)splits * a.N * p.Mp * sizeof(float);
    if (a.partial == nullptr || a.partial_bytes < need) {
      set_error("split-K workspace too small: need %zu bytes", need);
      return 2;
    }
    p.partial = a.partial;
  }
  CUtensorMap tx, tw;
  // Activation map: 3-D {K per slab, M, slabs}; an ordinary X is one slab.
  const int slabs = a.x_slabs > 0 ? a.x_slabs : 1;
  const long long k_slab = a.K / slabs;
  if (slabs > 1 && (a.K % slabs != 0 || k_slab % 64 != 0)) {
    set_error("slab width %lld must be a multiple of 64", k_slab);
    return 1;
  }
  p.k_slab = (int)k_slab;
  const bool pair = use_pair(tm, p.n_tiles);
  int rc = make_tmap_3d_strided(&tx, a.x, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (uint64_t)k_slab, (uint64_t)a.M,
                                (uint64_t)slabs, (uint64_t)a.ldx * 2,
                                (uint64_t)(slabs > 1 ? a.x_slab_stride : (long long)a.ldx * a.M) * 2, 64,
                                (uint32_t)(pair ? tm / 2 : tm), CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  if (a.fmt == WF_INT8) {
    rc = make_tmap_2d(&tw, a.w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)a.K, (uint64_t)a.N, (uint64_t)a.K, 64,
                      128, CU_TENSOR_MAP_SWIZZLE_64B);
    if (rc) return rc;
  } else if (a.fmt == WF_F16) {
    const long long ldw = a.ldw > 0 ? a.ldw : a.K;
    rc = make_tmap_2d(&tw, a.w, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (uint64_t)a.K, (uint64_t)a.N, (uint64_t)ldw * 2,
                      64, 128, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  } else {
    tw = tx;  // unused by bulk-copy decoders
  }
  CUtensorMap tt = tx;  // LoRA low-rank activation T' [M][lora_k] bf16, box {64, token rows per CTA}
  if (a.lora_k > 0) {
    rc = make_tmap_2d(&tt, a.lora_t, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)a.lora_k, (uint64_t)a.M,
                      (uint64_t)a.lora_k * 2, 64, (uint32_t)(pair ? tm / 2 : tm), CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  CUtensorMap tp = tx;  // split-K partials [splits][N][Mp] fp32, box {32 tokens, 128 rows}
  if (splits > 1 && tm >= 32) {
    rc = make_tmap_3d(&tp, p.partial, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (uint64_t)p.Mp, (uint64_t)a.N,
                      (uint64_t)splits, 32, 128, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  switch (a.fmt) {
    case WF_INT8:
      if (a.rot_group != 0) {
        if (!f16_gemm_can_rotate(a)) {
          set_error("output rotation needs the staged single-pass epilogue");
          return 2;
        }
        rc = dispatch_tm<DecInt8, true>(tx, tw, tp, tt, maps, p, tm, pair, stream);
      } else {
        rc = dispatch_tm<DecInt8>(tx, tw, tp, tt, maps, p, tm, pair, stream);
      }
      break;
    case WF_F16: rc = dispatch_tm<DecF16>(tx, tw, tp, tt, maps, p, tm, pair, stream); break;
    case WF_Q8_0: rc = dispatch_tm<DecQ8_0>(tx, tw, tp, tt, maps, p, tm, pair, stream); break;
    case WF_Q4_0: rc = dispatch_tm<DecQ4_0>(tx, tw, tp, tt, maps, p, tm, pair, stream); break;
    case WF_IQ4_NL: rc = dispatch_tm<DecIQ4<false>>(tx, tw, tp, tt, maps, p, tm, pair, stream); break;
    default:
      rc = dispatch_f16_blk(a.fmt, tx, tw, tp, tt, maps, p, tm, pair, stream);
      if (rc < 0) rc = dispatch_f16_kq(a.fmt, tx, tw, tp, tt, maps, p, tm, pair, stream);
      if (rc < 0) {
        set_error("unsupported weight format %d", a.fmt);
        rc = 2;
      }
  }
  if (rc) return rc;
  if (splits > 1) {
    launch_splitk_finalize(p.partial, splits, a.M, a.N, p.Mp, a.col_scale, a.col_scale_kind, a.w_row_exp,
                           a.x_row_exp, nullptr, a.bias, a.bias_kind, a.y, a.y_dtype, a.ldy, stream, a.out,
                           a.lora_k > 0, a.partial_bytes);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
      set_error("split-K finalize launch failed: %s", cudaGetErrorString(e));
      return 3;
    }
  }
  return 0;
}

// This translation unit's bounds record (QLIN_CHECKS build).
QLIN_BOUNDS_READER(bounds_read_f16)

}  // namespace qlin
