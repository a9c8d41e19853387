// Bounds checks of the QLIN_CHECKS build (libqlin_checked.so).
//
// compute-sanitizer's memcheck is not available to this project's test runs, so the library can
// be built with -DQLIN_CHECKS instead: every global access that the hardware does not bound by
// itself (plain loads and stores, untiled bulk copies; TMA tensor copies are clipped to their
// tensor map) and every computed shared-memory index is tested against a limit that the host
// derives from the C-ABI arguments -- the number of elements the caller's buffer holds -- rather
// than from the kernel's own index arithmetic.  A failed check records the first offender (site,
// index, limit, block) in a device word and SKIPS the access; it never traps, so the context stays
// usable and the host reads the record with qlin_bounds_check().  TMA coordinates are also checked
// for the 16-byte alignment of the innermost coordinate.
//
// In the ordinary build every check is the constant `true` and compiles away.
#pragma once
#include <cstdint>

namespace qlin {

struct BoundsRecord {
  unsigned int count;   // failed checks since the last reset
  unsigned int site;    // BoundsSite of the first failure
  unsigned int block;   // blockIdx.x of the first failure
  unsigned int thread;  // threadIdx.x of the first failure
  long long index;      // offending index (elements or bytes, as the site counts)
  long long limit;      // the limit it was checked against
};

// Sites: which access failed.  Keep in step with SITE_NAMES in qlin/__init__.py.
enum BoundsSite : unsigned int {
  BS_NONE = 0,
  BS_GEMM_Y = 1,          // f16 GEMM epilogue: output element
  BS_GEMM_BIAS = 2,       // f16 GEMM epilogue: bias / column scale / row exponent of a channel
  BS_GEMM_XEXP = 3,       // f16 GEMM epilogue: per-token exponent
  BS_GEMM_PARTIAL = 4,    // f16 GEMM split-K partial (direct store)
  BS_GEMM_WBULK = 5,      // f16 GEMM bulk copy of a repacked weight stage (byte range)
  BS_GEMM_LORA_U = 6,     // f16 GEMM LoRA up-projection row read
  BS_GEMM_PEER = 7,       // f16 GEMM staged store to a destination (own or peer output)
  BS_GEMM_SMEM = 8,       // f16 GEMM shared-memory layout / staging index
  BS_TMA_ALIGN = 9,       // a TMA coordinate whose innermost byte offset is not 16-byte aligned
  BS_I8_Y = 10,           // int8 GEMM epilogue output element
  BS_I8_SCALE = 11,       // int8 GEMM group / channel scale, bias, token scale
  BS_I8_WBULK = 12,       // int8 GEMM bulk copy of a weight stage
  BS_I8_SMEM = 13,        // int8 GEMM shared-memory layout
  BS_GEMV_W = 14,         // small-M kernel weight bytes
  BS_GEMV_X = 15,         // small-M kernel activation
  BS_GEMV_Y = 16,         // small-M kernel output / bias / scales
  BS_PRO_X = 17,          // activation prologue: input element
  BS_PRO_OUT = 18,        // activation prologue: operand / exponent / scale output
  BS_REPACK_SRC = 19,     // weight repack / row exponent / decode kernels: source bytes
  BS_REPACK_DST = 20,     // weight repack / decode kernels: destination
  BS_FINAL = 21,          // split-K finalize: partial read / output write
  BS_LORA = 22,           // LoRA packing kernels
  BS_GRAD = 23,           // gradient prologue / transpose / rotation kernels
  BS_KITCHEN = 24,        // kitchen int8 grid kernel
  BS_PEER_FLAG = 25,      // peer flag words
};

#ifdef QLIN_CHECKS
// One record per translation unit (each .cu is its own device module); qlin_bounds_check()
// gathers them through each unit's reader.
static __device__ BoundsRecord g_bounds;

__device__ __noinline__ inline bool bounds_fail(unsigned int site, long long idx, long long lim) {
  if (atomicAdd(&g_bounds.count, 1u) == 0u) {
    g_bounds.site = site;
    g_bounds.block = blockIdx.x;
    g_bounds.thread = threadIdx.x;
    g_bounds.index = idx;
    g_bounds.limit = lim;
  }
  return false;
}

// idx in [0, lim)
__device__ __forceinline__ bool qchk(unsigned int site, long long idx, long long lim) {
  return (idx >= 0 && idx < lim) ? true : bounds_fail(site, idx, lim);
}
// [idx, idx + len) inside [0, lim)
__device__ __forceinline__ bool qchk_span(unsigned int site, long long idx, long long len, long long lim) {
  return (idx >= 0 && len >= 0 && idx + len <= lim) ? true : bounds_fail(site, idx + len, lim);
}
// value a multiple of `align`
__device__ __forceinline__ bool qchk_align(unsigned int site, long long value, long long align) {
  return (value % align == 0) ? true : bounds_fail(site, value, align);
}
// The dynamic shared memory this launch was given, in bytes.
__device__ __forceinline__ unsigned int dyn_smem_bytes() {
  unsigned int v;
  asm volatile("mov.u32 %0, %%dynamic_smem_size;" : "=r"(v));
  return v;
}
// [p, p + bytes) inside the launch's dynamic shared memory that starts at `base`.
__device__ __forceinline__ bool qchk_smem(unsigned int site, const void* base, const void* p, long long bytes) {
  const long long off = (long long)(reinterpret_cast<const uint8_t*>(p) - reinterpret_cast<const uint8_t*>(base));
  return qchk_span(site, off, bytes, (long long)dyn_smem_bytes());
}

// Host side: defines `int NAME(BoundsRecord* out, int reset)` reading (and optionally clearing)
// this translation unit's record.
#define QLIN_BOUNDS_READER(NAME)                                                              \
  int NAME(::qlin::BoundsRecord* out, int reset) {                                            \
    ::qlin::BoundsRecord r{};                                                                 \
    if (cudaMemcpyFromSymbol(&r, ::qlin::g_bounds, sizeof(r)) != cudaSuccess) return -1;      \
    if (out) *out = r;                                                                        \
    if (reset) {                                                                              \
      ::qlin::BoundsRecord z{};                                                               \
      if (cudaMemcpyToSymbol(::qlin::g_bounds, &z, sizeof(z)) != cudaSuccess) return -1;      \
    }                                                                                         \
    return 0;                                                                                 \
  }
#else
__device__ __forceinline__ constexpr bool qchk(unsigned int, long long, long long) { return true; }
__device__ __forceinline__ constexpr bool qchk_span(unsigned int, long long, long long, long long) { return true; }
__device__ __forceinline__ constexpr bool qchk_align(unsigned int, long long, long long) { return true; }
__device__ __forceinline__ constexpr bool qchk_smem(unsigned int, const void*, const void*, long long) { return true; }
#define QLIN_BOUNDS_READER(NAME)                                                              \
  int NAME(::qlin::BoundsRecord* out, int) {                                                  \
    if (out) *out = ::qlin::BoundsRecord{};                                                   \
    return 1;                                                                                 \
  }
#endif

}  // namespace qlin
