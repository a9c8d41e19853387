// The C ABI (include/qlin.h): argument checks, workspace carving, prologue + GEMM sequencing.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "../../include/qlin.h"
#include "qlin_internal.h"
#include "qlin_ptx.cuh"
#include "qlin_gemm_i8.cuh"
#include "qlin_peer.cuh"

namespace qlin {

static thread_local char g_err[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

static inline size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

// Workspace carving: consecutive 256-byte aligned regions.
struct Carver {
  uint8_t* base;
  size_t cap, off = 0;
  void* take(size_t bytes) {
    void* p = base ? base + off : nullptr;
    off = align256(off + bytes);
    return p;
  }
};

static bool is_float_dtype(int d) { return d == QLIN_F32 || d == QLIN_F16 || d == QLIN_BF16; }
static int bias_kind_of(const void* bias, int dt) {
  if (bias == nullptr) return 0;
  return dt == QLIN_F16 ? 1 : dt == QLIN_F32 ? 2 : dt == QLIN_BF16 ? 3 : -1;
}
static int out_kind_of(int dt) { return dt == QLIN_F32 ? 0 : dt == QLIN_F16 ? 1 : dt == QLIN_BF16 ? 2 : -1; }

static int check_cuda(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s: %s", what, cudaGetErrorString(e));
    return QLIN_ECUDA;
  }
  return QLIN_OK;
}

static int64_t round_up(int64_t v, int64_t a) { return (v + a - 1) / a * a; }

// Activation operand for the f16 family: fp16 [m, kp] + row exponents, produced by the prologue
// unless x is already a suitable fp16 tensor and no rotation is requested.
struct F16Operand {
  const void* x;
  long long ldx;
  const int32_t* row_exp;
};

static size_t f16_operand_bytes(int64_t m, int64_t k) {
  return align256((size_t)m * round_up(k, 64) * 2) + align256((size_t)m * 4);
}

static int make_f16_operand(const void* x, int x_dtype, int64_t m, int64_t k, int64_t ldx, int group, Carver& ws,
                            cudaStream_t stream, F16Operand* out) {
  const bool direct = x_dtype == QLIN_F16 && group == 0 && ldx % 8 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0;
  if (direct) {
    out->x = x;
    out->ldx = ldx;
    out->row_exp = nullptr;
    return QLIN_OK;
  }
  const int64_t kp = round_up(k, 64);
  void* xr = ws.take((size_t)m * kp * 2);
  int32_t* rexp = reinterpret_cast<int32_t*>(ws.take((size_t)m * 4));
  if (ws.off > ws.cap) {
    set_error("workspace too small: need %zu bytes", ws.off);
    return QLIN_EINVAL;
  }
  if (launch_prologue(x, x_dtype, ldx, (int)m, (int)k, (int)kp, group, 0, xr, rexp, nullptr, 0, stream) != 0) {
    set_error("unsupported rotation group %d", group);
    return QLIN_EDECLINE;
  }
  int rc = check_cuda("prologue launch");
  if (rc) return rc;
  out->x = xr;
  out->ldx = kp;
  out->row_exp = rexp;
  return QLIN_OK;
}

static bool valid_group(int g) { return g == 0 || g == 32 || g == 64 || g == 128 || g == 256; }

// Scratch for qlin_gguf_linear_noalloc: a fixed 16 MiB array in every device's global memory,
// reserved when the library's module is loaded on that device and held until the process exits.
// It replaces the caller's workspace (the fp16 activation copy and the split-K partial sums).
constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Unique id of the calling thread's current CUDA context (cuCtxGetId: never reused within the
// process, unlike a context handle or a device index), through the runtime's driver entry points;
// 0 when no context is current yet.
typedef CUresult (*PFN_ctxGetCurrent_t)(CUcontext*);
typedef CUresult (*PFN_ctxGetId_t)(CUcontext, unsigned long long*);

unsigned long long current_context_id() {
  static PFN_ctxGetCurrent_t get_current = nullptr;
  static PFN_ctxGetId_t get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<PFN_ctxGetCurrent_t>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<PFN_ctxGetId_t>(p);
  });
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (get_current == nullptr || get_id == nullptr || get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr ||
      get_id(ctx, &id) != CUDA_SUCCESS)
    return 0;
  return id;
}

// Device address of g_noalloc_scratch in the current context.  In host code the symbol is only a
// host-side stand-in; the real address comes from cudaGetSymbolAddress, looked up once per CUDA
// context (keyed by the context's unique id, so a context created after cudaDeviceReset, or a
// non-primary context the caller made current, gets its own lookup) with that context current.
static int noalloc_scratch(void** out) {
  static std::mutex mu;
  struct Entry {
    unsigned long long ctx;
    void* addr;
  };
  static Entry cache[64] = {};
  static int next = 0;
  std::lock_guard<std::mutex> lock(mu);
  unsigned long long id = current_context_id();
  if (id != 0) {
    for (const Entry& e : cache)
      if (e.ctx == id) {
        *out = e.addr;
        return QLIN_OK;
      }
  }
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);  // also makes the context current
  if (e != cudaSuccess || p == nullptr) {
    int dev = -1;
    cudaGetDevice(&dev);
    set_error("qlin_gguf_linear_noalloc: cudaGetSymbolAddress failed on device %d: %s", dev, cudaGetErrorString(e));
    return QLIN_ECUDA;
  }
  if (id == 0) id = current_context_id();
  if (id != 0) {
    cache[next] = Entry{id, p};
    next = (next + 1) % 64;
  }
  *out = p;
  return QLIN_OK;
}

// This translation unit's bounds record (QLIN_CHECKS build).
QLIN_BOUNDS_READER(bounds_read_api)

}  // namespace qlin

using namespace qlin;

static int gguf_slabs_impl(const void* x, int64_t m, int64_t k, int64_t ldx, int x_slabs, int64_t x_slab_stride,
                           const void* packed, const int32_t* row_exp, int qtype, int64_t n, const void* bias,
                           int bias_dtype, void* y, int y_dtype, int64_t ldy, void* workspace, size_t workspace_bytes,
                           void* stream_, const PeerOut* out, const PeerMaps* out_maps = nullptr) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (m < 0 || n < 0 || k <= 0 || x_slabs < 1 || k % x_slabs != 0 || ldx < k / x_slabs || ldy < n ||
      (x_slabs > 1 && x_slab_stride < m * ldx)) {
    set_error("bad slab sizes");
    return QLIN_EINVAL;
  }
  if (m == 0 || n == 0) return QLIN_OK;
  if (gguf_stage_bytes(qtype, nullptr, nullptr) == 0 || k % gguf_block_values(qtype) != 0 ||
      out_kind_of(y_dtype) < 0 || bias_kind_of(bias, bias_dtype) < 0 || (k / x_slabs) % 64 != 0 || ldx % 8 != 0 ||
      x_slab_stride % 8 != 0 || (reinterpret_cast<uintptr_t>(x) & 15)) {
    set_error("unsupported slab operand (fp16 slabs of a multiple of 64 columns, 16-byte aligned)");
    return QLIN_EDECLINE;
  }
  Carver ws{reinterpret_cast<uint8_t*>(workspace), workspace_bytes};
  F16GemmArgs a{};
  a.fmt = qtype;
  a.x = x;
  a.ldx = ldx;
  a.x_slabs = x_slabs;
  a.x_slab_stride = x_slab_stride;
  a.M = (int)m;
  a.N = (int)n;
  a.K = (int)k;
  a.w = packed;
  {
    size_t wb = 0;
    if (qlin_gguf_repacked_bytes(qtype, n, k, &wb, nullptr) == QLIN_OK) a.w_bytes = (long long)wb;
  }
  a.w_row_exp = row_exp;
  a.col_scale_kind = CS_EXP2;
  a.bias = bias;
  a.bias_kind = bias_kind_of(bias, bias_dtype);
  a.y = y;
  a.y_dtype = out_kind_of(y_dtype);
  a.ldy = ldy;
  const size_t pb = f16_gemm_partial_bytes((int)m, (int)n, (int)k, qtype, 0, 0);
  a.partial = reinterpret_cast<float*>(ws.take(pb));
  a.partial_bytes = pb;
  if (ws.off > ws.cap && pb > 0) {
    set_error("workspace too small: need %zu bytes", ws.off);
    return QLIN_EINVAL;
  }
  a.out = out;
  a.out_maps = out_maps;
  return run_f16_gemm(a, stream);
}

// Unmerged LoRA (y += scale * t . up^T with t = x . down^T computed by the caller) fused into the
// linear as extra K stages; see GemmParams::main_k_stages.
struct LoraArgs {
  const void* t;
  int t_dtype;
  int64_t ldt;
  const void* up;
  int up_dtype;
  int64_t ldu;
  int64_t rank;
  float scale;
};

static int64_t lora_k_of(const LoraArgs* l) { return l == nullptr ? 0 : round_up(l->rank, 64); }

static size_t lora_bytes(int64_t m, int64_t n, const LoraArgs* l) {
  const int64_t rk = lora_k_of(l);
  return rk == 0 ? 0 : align256((size_t)m * rk * 2) + align256((size_t)round_up(n, 128) * rk * 2);
}

// The LoRA down factor given instead of t = x . down^T: t is computed here, by the same tensor-core
// GEMM on the activation operand (rotated, per-row normalized fp16) against the down factor put
// through the same prologue (x . down^T = rot(x) . rot(down)^T for the orthonormal rotation).
struct LoraDown {
  const void* down;  // [rank, k], row pitch ldd
  int dtype;
  int64_t ldd;
};

static size_t lora_down_bytes(int64_t m, int64_t k, int64_t rank) {
  const int64_t kp = round_up(k, 64);
  return align256((size_t)rank * kp * 2) + align256((size_t)rank * 4) + align256((size_t)m * rank * 4) +
         align256(f16_gemm_partial_bytes((int)m, (int)rank, (int)k, WF_F16, 0, 0));
}

// t [m, rank] fp32 into the workspace; returns QLIN_OK and *t_out, or an error.
static int compute_lora_t(const void* x, int64_t ldx, const int32_t* x_row_exp, int64_t m, int64_t k, int group,
                          const LoraDown& d, int64_t rank, Carver& ws, cudaStream_t stream, float** t_out) {
  if (rank <= 0 || rank > 256 || d.down == nullptr || !is_float_dtype(d.dtype) || d.ldd < k) {
    set_error("lora: rank 1..256 and a float down factor [rank, k]");
    return QLIN_EDECLINE;
  }
  const int64_t kp = round_up(k, 64);
  void* dn = ws.take((size_t)rank * kp * 2);
  int32_t* dexp = reinterpret_cast<int32_t*>(ws.take((size_t)rank * 4));
  float* t = reinterpret_cast<float*>(ws.take((size_t)m * rank * 4));
  const size_t pb = f16_gemm_partial_bytes((int)m, (int)rank, (int)k, WF_F16, 0, 0);
  float* part = reinterpret_cast<float*>(ws.take(pb));
  if (ws.off > ws.cap) {
    set_error("workspace too small: need %zu bytes", ws.off);
    return QLIN_EINVAL;
  }
  if (launch_prologue(d.down, d.dtype, d.ldd, (int)rank, (int)k, (int)kp, group, 0, dn, dexp, nullptr, 0, stream) != 0) {
    set_error("lora: unsupported rotation group %d", group);
    return QLIN_EDECLINE;
  }
  int rc = check_cuda("lora down prologue launch");
  if (rc) return rc;
  F16GemmArgs b{};
  b.fmt = WF_F16;
  b.x = x;
  b.ldx = ldx;
  b.M = (int)m;
  b.N = (int)rank;
  b.K = (int)k;
  b.w = dn;
  b.ldw = kp;
  b.w_row_exp = dexp;
  b.col_scale = nullptr;
  b.col_scale_kind = CS_EXP2;
  b.x_row_exp = x_row_exp;
  b.bias = nullptr;
  b.bias_kind = 0;
  b.y = t;
  b.y_dtype = OUT_F32;
  b.ldy = rank;
  b.partial = part;
  b.partial_bytes = pb;
  rc = run_f16_gemm(b, stream);
  if (rc) return rc;
  *t_out = t;
  return QLIN_OK;
}

static int attach_lora(const LoraArgs* l, F16GemmArgs& a, Carver& ws, cudaStream_t stream) {
  if (l == nullptr) return QLIN_OK;
  if (l->rank <= 0 || l->rank > 256 || !is_float_dtype(l->t_dtype) || !is_float_dtype(l->up_dtype) ||
      l->t == nullptr || l->up == nullptr || l->ldt < l->rank || l->ldu < l->rank) {
    set_error("lora: rank 1..256, float t [m, rank] and up [n, rank]");
    return QLIN_EDECLINE;
  }
  const int rk = (int)lora_k_of(l);
  const int n_pad = (int)round_up(a.N, 128);
  void* t_out = ws.take((size_t)a.M * rk * 2);
  void* u_out = ws.take((size_t)n_pad * rk * 2);
  if (ws.off > ws.cap) {
    set_error("workspace too small: need %zu bytes", ws.off);
    return QLIN_EINVAL;
  }
  launch_lora_operands(l->t, l->t_dtype, l->ldt, a.M, l->up, l->up_dtype, l->ldu, a.N, n_pad, (int)l->rank, rk,
                       l->scale, a.col_scale, a.col_scale_kind, a.w_row_exp, a.x_row_exp, t_out, u_out, stream);
  const int rc = check_cuda("lora operand launch");
  if (rc) return rc;
  a.lora_t = t_out;
  a.lora_u_ptr = u_out;
  a.lora_k = rk;
  return QLIN_OK;
}

extern "C" {

const char* qlin_version(void) { return "qlin 0.1 (sm_100a, tcgen05)"; }

const char* qlin_last_error(void) { return g_err; }

int qlin_bounds_check(int reset, uint32_t* count, uint32_t* site, int64_t* index, int64_t* limit, uint32_t* block) {
  int (*const readers[])(BoundsRecord*, int) = {bounds_read_api, bounds_read_aux,  bounds_read_f16, bounds_read_f16_blk,
                                                bounds_read_f16_kq, bounds_read_gemv, bounds_read_i8};
  uint32_t total = 0;
  BoundsRecord first{};
  for (auto rd : readers) {
    BoundsRecord r{};
    const int rc = rd(&r, reset);
    if (rc < 0) return check_cuda("bounds record read");
    if (rc > 0) {
      set_error("this library was built without QLIN_CHECKS");
      return QLIN_EDECLINE;
    }
    if (r.count > 0 && total == 0) first = r;
    total += r.count;
  }
  if (count) *count = total;
  if (site) *site = first.site;
  if (index) *index = first.index;
  if (limit) *limit = first.limit;
  if (block) *block = first.block;
  return QLIN_OK;
}

int qlin_device_status(int reset, uint32_t* where) {
  void* p = device_status_ptr();
  if (p == nullptr) {
    set_error("device status word unavailable");
    return QLIN_ECUDA;
  }
  DeviceStatus st{};
  if (cudaMemcpy(&st, p, sizeof(st), cudaMemcpyDeviceToHost) != cudaSuccess) return check_cuda("status read");
  if (where) *where = st.where;
  if (reset) {
    DeviceStatus z{};
    if (cudaMemcpy(p, &z, sizeof(z), cudaMemcpyHostToDevice) != cudaSuccess) return check_cuda("status reset");
  }
  return st.timed_out ? QLIN_ETIMEOUT : QLIN_OK;
}

// ------------------------------------------------------------------------------------------ INT8
size_t qlin_int8_linear_workspace(int64_t m, int64_t n, int64_t k) {
  return f16_operand_bytes(m, k) + align256(f16_gemm_partial_bytes((int)m, (int)n, (int)k, WF_INT8, 0, 0));
}

static int int8_linear_impl(const void* x, int x_dtype, int64_t m, int64_t k, int64_t ldx, const int8_t* q,
                            int64_t n, const void* scale, int scale_dtype, const void* bias, int bias_dtype,
                            int convrot_group, void* y, int y_dtype, int64_t ldy, void* workspace,
                            size_t workspace_bytes, void* stream_, const LoraArgs* lora,
                            const LoraDown* down = nullptr) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (m < 0 || n < 0 || k < 0 || ldx < k || ldy < n) {
    set_error("bad sizes m=%lld n=%lld k=%lld ldx=%lld ldy=%lld", (long long)m, (long long)n, (long long)k,
              (long long)ldx, (long long)ldy);
    return QLIN_EINVAL;
  }
  if (m == 0 || n == 0) return QLIN_OK;
  if (!is_float_dtype(x_dtype) || out_kind_of(y_dtype) < 0 || (scale_dtype != QLIN_F16 && scale_dtype != QLIN_F32) ||
      bias_kind_of(bias, bias_dtype) < 0) {
    set_error("unsupported dtype combination");
    return QLIN_EDECLINE;
  }
  if (k == 0 || k % 16 != 0 || !valid_group(convrot_group) || (convrot_group && k % convrot_group) ||
      m > 0x7fffffff || n > 0x7fffffff || k > 0x7fffffff) {
    set_error("unsupported shape: k=%lld group=%d (k must be a multiple of 16 and of the group)", (long long)k,
              convrot_group);
    return QLIN_EDECLINE;
  }
  if (x == nullptr || q == nullptr || scale == nullptr || y == nullptr || (reinterpret_cast<uintptr_t>(q) & 15)) {
    set_error("null or misaligned pointer (q needs 16-byte alignment)");
    return QLIN_EINVAL;
  }
  Carver ws{reinterpret_cast<uint8_t*>(workspace), workspace_bytes};
  F16Operand op;
  int rc = make_f16_operand(x, x_dtype, m, k, ldx, convrot_group, ws, stream, &op);
  if (rc) return rc;
  F16GemmArgs a{};
  a.fmt = WF_INT8;
  a.x = op.x;
  a.ldx = op.ldx;
  a.M = (int)m;
  a.N = (int)n;
  a.K = (int)k;
  a.w = q;
  a.w_row_exp = nullptr;
  a.col_scale = scale;
  a.col_scale_kind = scale_dtype == QLIN_F16 ? CS_F16 : CS_F32;
  a.x_row_exp = op.row_exp;
  a.bias = bias;
  a.bias_kind = bias_kind_of(bias, bias_dtype);
  a.y = y;
  a.y_dtype = out_kind_of(y_dtype);
  a.ldy = ldy;
  const size_t pb = f16_gemm_partial_bytes((int)m, (int)n, (int)(k + lora_k_of(lora)), WF_INT8, 0, 0);
  a.partial = reinterpret_cast<float*>(ws.take(pb));
  a.partial_bytes = pb;
  if (ws.off > ws.cap && pb > 0) {
    set_error("workspace too small: need %zu bytes", ws.off);
    return QLIN_EINVAL;
  }
  LoraArgs with_t;
  if (down != nullptr && lora != nullptr) {
    float* t = nullptr;
    rc = compute_lora_t(op.x, op.ldx, op.row_exp, m, k, convrot_group, *down, lora->rank, ws, stream, &t);
    if (rc) return rc;
    with_t = *lora;
    with_t.t = t;
    with_t.t_dtype = QLIN_F32;
    with_t.ldt = lora->rank;
    lora = &with_t;
  }
  rc = attach_lora(lora, a, ws, stream);
  if (rc) return rc;
  return run_f16_gemm(a, stream);
}

int qlin_int8_linear(const void* x, int x_dtype, int64_t m, int64_t k, int64_t ldx, const int8_t* q, int64_t n,
                     const void* scale, int scale_dtype, const void* bias, int bias_dtype, int convrot_group, void* y,
                     int y_dtype, int64_t ldy, void* workspace, size_t workspace_bytes, void* stream) {
  return int8_linear_impl(x, x_dtype, m, k, ldx, q, n, scale, scale_dtype, bias, bias_dtype, convrot_group, y, y_dtype,
                          ldy, workspace, workspace_bytes, stream, nullptr);
}

size_t qlin_int8_linear_lora_workspace(int64_t m, int64_t n, int64_t k, int64_t rank) {
  LoraArgs l{};
  l.rank = rank;
  return f16_operand_bytes(m, k) +
         align256(f16_gemm_partial_bytes((int)m, (int)n, (int)(k + lora_k_of(&l)), WF_INT8, 0, 0)) +
         lora_bytes(m, n, &l);
}

size_t qlin_int8_linear_lora_down_workspace(int64_t m, int64_t n, int64_t k, int64_t rank) {
  return qlin_int8_linear_lora_workspace(m, n, k, rank) + lora_down_bytes(m, k, rank);
}

int qlin_int8_linear_lora_down(const void* x, int x_dtype, int64_t m, int64_t k, int64_t ldx, const int8_t* q,
                               int64_t n, const void* scale, int scale_dtype, const void* bias, int bias_dtype,
                               int convrot_group, const void* lora_down, int lora_down_dtype, int64_t ldd,
                               const void* lora_up, int lora_up_dtype, int64_t ldu, int64_t rank, float lora_scale,
                               void* y, int y_dtype, int64_t ldy, void* workspace, size_t workspace_bytes,
                               void* stream) {
  // t is filled in by the impl; the LoraArgs carry up, rank and scale
  const LoraArgs l{lora_down, QLIN_F32, rank, lora_up, lora_up_dtype, ldu, rank, lora_scale};
  const LoraDown d{lora_down, lora_down_dtype, ldd};
  return int8_linear_impl(x, x_dtype, m, k, ldx, q, n, scale, scale_dtype, bias, bias_dtype, convrot_group, y, y_dtype,
                          ldy, workspace, workspace_bytes, stream, &l, &d);
}

int qlin_int8_linear_lora(const void* x, int x_dtype, int64_t m, int64_t k, int64_t ldx, const int8_t* q, int64_t n,
                          const void* scale, int scale_dtype, const void* bias, int bias_dtype, int convrot_group,
                          const void* lora_t, int lora_t_dtype, int64_t ldt, const void* lora_up, int lora_up_dtype,
                          int64_t ldu, int64_t rank, float lora_scale, void* y, int y_dtype, int64_t ldy,
                          void* workspace, size_t workspace_bytes, void* stream) {
  const LoraArgs l{lora_t, lora_t_dtype, ldt, lora_up, lora_up_dtype, ldu, rank, lora_scale};
  return int8_linear_impl(x, x_dtype, m, k, ldx, q, n, scale, scale_dtype, bias, bias_dtype, convrot_group, y, y_dtype,
                          ldy, workspace, workspace_bytes, stream, &l);
}

// ------------------------------------------------------------------------ INT8 input gradient
size_t qlin_int8_grad_weight_bytes(int64_t n, int64_t k) {
  return n <= 0 || k <= 0 ? 0 : (size_t)k * (size_t)round_up(n, 64);
}

int qlin_int8_grad_weight(const int8_t* q, int64_t n, int64_t k, int8_t* qt, size_t qt_bytes, void* stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (n <= 0 || k <= 0 || n > 0x7fffffff || k > 0x7fffffff) {
    set_error("bad sizes n=%lld k=%lld", (long long)n, (long long)k);
    return QLIN_EINVAL;
  }
  if (q == nullptr || qt == nullptr || (reinterpret_cast<uintptr_t>(qt) & 15) || qt_bytes < qlin_int8_grad_weight_bytes(n, k)) {
    set_error("null or misaligned pointer, or qt smaller than qlin_int8_grad_weight_bytes");
    return QLIN_EINVAL;
  }
  launch_int8_transpose(q, (int)n, (int)k, qt, (int)round_up(n, 64), stream);
  return check_cuda("int8 transpose launch");
}

size_t qlin_int8_linear_grad_input_workspace(int64_t m, int64_t n, int64_t k, int rotate_group) {
  if (m <= 0 || n <= 0 || k <= 0) return 0;
  const int64_t np = round_up(n, 64);
  size_t b = f16_operand_bytes(m, np) + align256(f16_gemm_partial_bytes((int)m, (int)k, (int)np, WF_INT8, 0, 0));
  if (rotate_group) b += align256((size_t)m * k * 4);
  return b;
}

int qlin_int8_linear_grad_input(const void* dy, int dy_dtype, int64_t m, int64_t n, int64_t lddy, const int8_t* qt,
                                int64_t k, const void* scale, int scale_dtype, int rotate_group, void* dx,
                                int dx_dtype, int64_t lddx, void* workspace, size_t workspace_bytes, void* stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (m < 0 || n < 0 || k < 0 || lddy < n || lddx < k || m > 0x7fffffff || n > 0x7fffffff || k > 0x7fffffff) {
    set_error("bad sizes m=%lld n=%lld k=%lld lddy=%lld lddx=%lld", (long long)m, (long long)n, (long long)k,
              (long long)lddy, (long long)lddx);
    return QLIN_EINVAL;
  }
  if (!is_float_dtype(dy_dtype) || out_kind_of(dx_dtype) < 0 || (scale_dtype != QLIN_F16 && scale_dtype != QLIN_F32)) {
    set_error("unsupported dtype combination");
    return QLIN_EDECLINE;
  }
  if (k % 16 != 0 || !valid_group(rotate_group) || (rotate_group && k % rotate_group)) {
    set_error("unsupported shape: k=%lld group=%d (k must be a multiple of 16 and of the group)", (long long)k,
              rotate_group);
    return QLIN_EDECLINE;
  }
  if (m == 0 || k == 0) return QLIN_OK;
  if (dx == nullptr) {
    set_error("null dx");
    return QLIN_EINVAL;
  }
  const int esz = dx_dtype == QLIN_F32 ? 4 : 2;
  if (n == 0) {  // empty contraction: dX = 0
    if (cudaMemset2DAsync(dx, (size_t)lddx * esz, 0, (size_t)k * esz, (size_t)m, stream) != cudaSuccess)
      return check_cuda("dx clear");
    return QLIN_OK;
  }
  if (dy == nullptr || qt == nullptr || scale == nullptr || (reinterpret_cast<uintptr_t>(qt) & 15)) {
    set_error("null or misaligned pointer (qt needs 16-byte alignment)");
    return QLIN_EINVAL;
  }
  const int64_t np = round_up(n, 64);
  Carver ws{reinterpret_cast<uint8_t*>(workspace), workspace_bytes};
  void* xr = ws.take((size_t)m * np * 2);
  int32_t* rexp = reinterpret_cast<int32_t*>(ws.take((size_t)m * 4));
  const size_t pb = f16_gemm_partial_bytes((int)m, (int)k, (int)np, WF_INT8, 0, 0);
  float* partial = reinterpret_cast<float*>(ws.take(pb));
  float* unrot = rotate_group ? reinterpret_cast<float*>(ws.take((size_t)m * k * 4)) : nullptr;
  if (ws.off > ws.cap) {
    set_error("workspace too small: need %zu bytes", ws.off);
    return QLIN_EINVAL;
  }
  launch_grad_prologue(dy, dy_dtype, lddy, (int)m, (int)n, (int)np, scale, scale_dtype == QLIN_F16 ? 1 : 0, xr, rexp,
                       stream);
  int rc = check_cuda("gradient prologue launch");
  if (rc) return rc;
  F16GemmArgs a{};
  a.fmt = WF_INT8;
  a.x = xr;
  a.ldx = np;
  a.M = (int)m;
  a.N = (int)k;
  a.K = (int)np;
  a.w = qt;
  a.w_row_exp = nullptr;
  a.col_scale = nullptr;
  a.col_scale_kind = CS_NONE;
  a.x_row_exp = rexp;
  a.bias = nullptr;
  a.bias_kind = 0;
  a.partial = partial;
  a.partial_bytes = pb;
  // The rotation runs in the GEMM's epilogue where it can (groups up to 128, 2-byte dx, no K
  // split); otherwise the GEMM writes fp32 dx and a separate pass rotates it.  Both apply the
  // same butterflies to the same fp32 values.
  a.y = dx;
  a.y_dtype = out_kind_of(dx_dtype);
  a.ldy = lddx;
  a.rot_group = rotate_group;
  if (rotate_group == 0 || f16_gemm_can_rotate(a)) return run_f16_gemm(a, stream);
  a.rot_group = 0;
  a.y = unrot;
  a.y_dtype = OUT_F32;
  a.ldy = k;
  rc = run_f16_gemm(a, stream);
  if (rc) return rc;
  launch_grad_rotate(unrot, (int)m, (int)k, rotate_group, dx, out_kind_of(dx_dtype), lddx, stream);
  return check_cuda("gradient rotation launch");
}

// ------------------------------------------------------------------------------------------ GGUF
int qlin_gguf_repacked_bytes(int qtype, int64_t n, int64_t k, size_t* bytes, int64_t* padded_n) {
  const uint32_t sb = gguf_stage_bytes(qtype, nullptr, nullptr);
  if (sb == 0) {
    set_error("unsupported GGUF type %d", qtype);
    return QLIN_EDECLINE;
  }
  const int qk = gguf_block_values(qtype);
  if (n < 0 || k <= 0 || (n * k) % qk != 0 || k % 8 != 0) {
    set_error("n*k=%lld is not a whole number of %d-value blocks (or k is not a multiple of 8)", (long long)(n * k),
              qk);
    return QLIN_EDECLINE;
  }
  const int64_t nt = (n + 127) / 128;
  if (k % qk != 0) {
    // rows straddle blocks: plain fp16 rows w * 2^-e, pitch roundup(k, 64)
    if (bytes) *bytes = (size_t)nt * 128 * (size_t)round_up(k, 64) * 2;
  } else {
    if (bytes) *bytes = (size_t)nt * ((k + 63) / 64) * sb;
  }
  if (padded_n) *padded_n = nt * 128;
  return QLIN_OK;
}

int qlin_gguf_repack(const void* raw, int qtype, int64_t n, int64_t k, void* packed, size_t packed_bytes,
                     int32_t* row_exp, int64_t row_exp_len, void* stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  size_t need = 0;
  int64_t npad = 0;
  int rc = qlin_gguf_repacked_bytes(qtype, n, k, &need, &npad);
  if (rc) return rc;
  if (packed_bytes < need || row_exp_len < npad || raw == nullptr || packed == nullptr || row_exp == nullptr ||
      (reinterpret_cast<uintptr_t>(packed) & 15)) {
    set_error("repack buffers: need %zu bytes (16-byte aligned) and %lld exponents", need, (long long)npad);
    return QLIN_EINVAL;
  }
  if (k % gguf_block_values(qtype) != 0) {
    launch_gguf_straddle_repack(reinterpret_cast<const uint8_t*>(raw), qtype, (int)n, (int)k, (int)npad,
                                (int)round_up(k, 64), packed, packed_bytes, row_exp, stream);
    return check_cuda("gguf straddle repack launch");
  }
  int P = 0, S = 0;
  const uint32_t sb = gguf_stage_bytes(qtype, &P, &S);
  launch_gguf_repack(reinterpret_cast<const uint8_t*>(raw), qtype, (int)n, (int)k, (int)((k + 63) / 64),
                     (int)(npad / 128), reinterpret_cast<uint8_t*>(packed), packed_bytes, sb, P, S, stream);
  launch_gguf_row_exp(reinterpret_cast<const uint8_t*>(raw), qtype, (int)n, (int)k, (int)npad, row_exp, stream);
  return check_cuda("gguf repack launch");
}

static constexpr int kGgufFormats[] = {WF_F16, WF_Q4_0, WF_Q4_1, WF_Q5_0, WF_Q5_1, WF_Q8_0, WF_Q2_K,
                                       WF_Q3_K, WF_Q4_K, WF_Q5_K, WF_Q6_K, WF_IQ4_NL, WF_IQ4_XS};

// Workspace of the GGUF linear for any of the supported types (the largest plan's partials).
size_t qlin_gguf_linear_workspace(int64_t m, int64_t n, int64_t k, int x_dtype, int64_t ldx) {
  (void)x_dtype;
  (void)ldx;
  size_t pb = 0;
  for (int fmt : kGgufFormats)
    pb = std::max(pb, f16_gemm_partial_bytes((int)m, (int)n, (int)k, fmt, 0, 0));
  return f16_operand_bytes(m, k) + align256(pb);
}

static int gguf_linear_impl(const void* x, int x_dtype, int64_t m, int64_t k, int64_t ldx, const void* packed,
                            const int32_t* row_exp, int qtype, int64_t n, const void* bias, int bias_dtype, void* y,
                            int y_dtype, int64_t ldy, void* workspace, size_t workspace_bytes, void* stream_,
                            const LoraArgs* lora, const LoraDown* down = nullptr) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (m < 0 || n < 0 || k < 0 || ldx < k || ldy < n) {
    set_error("bad sizes");
    return QLIN_EINVAL;
  }
  if (m == 0 || n == 0) return QLIN_OK;
  if (gguf_stage_bytes(qtype, nullptr, nullptr) == 0 || (k % gguf_block_values(qtype) != 0 && k % 8 != 0) ||
      !is_float_dtype(x_dtype) || out_kind_of(y_dtype) < 0 || bias_kind_of(bias, bias_dtype) < 0) {
    set_error("unsupported GGUF type/shape/dtype (type %d, k %lld)", qtype, (long long)k);
    return QLIN_EDECLINE;
  }
  // rows that straddle blocks were repacked to plain fp16 rows (qlin_gguf_repack)
  const bool straddle = k % gguf_block_values(qtype) != 0;
  if (x == nullptr || packed == nullptr || row_exp == nullptr || y == nullptr) {
    set_error("null pointer");
    return QLIN_EINVAL;
  }
  Carver ws{reinterpret_cast<uint8_t*>(workspace), workspace_bytes};
  F16Operand op;
  int rc = make_f16_operand(x, x_dtype, m, k, ldx, 0, ws, stream, &op);
  if (rc) return rc;
  F16GemmArgs a{};
  a.fmt = straddle ? (int)WF_F16 : qtype;
  a.ldw = straddle ? round_up(k, 64) : 0;
  a.x = op.x;
  a.ldx = op.ldx;
  a.M = (int)m;
  a.N = (int)n;
  a.K = (int)k;
  a.w = packed;
  {
    size_t wb = 0;
    if (qlin_gguf_repacked_bytes(qtype, n, k, &wb, nullptr) == QLIN_OK) a.w_bytes = (long long)wb;
  }
  a.w_row_exp = row_exp;
  a.col_scale = nullptr;
  a.col_scale_kind = CS_EXP2;
  a.x_row_exp = op.row_exp;
  a.bias = bias;
  a.bias_kind = bias_kind_of(bias, bias_dtype);
  a.y = y;
  a.y_dtype = out_kind_of(y_dtype);
  a.ldy = ldy;
  const size_t pb = f16_gemm_partial_bytes((int)m, (int)n, (int)(k + lora_k_of(lora)), a.fmt, 0, 0);
  a.partial = reinterpret_cast<float*>(ws.take(pb));
  a.partial_bytes = pb;
  if (ws.off > ws.cap && pb > 0) {
    set_error("workspace too small: need %zu bytes", ws.off);
    return QLIN_EINVAL;
  }
  LoraArgs with_t;
  if (down != nullptr && lora != nullptr) {
    float* t = nullptr;
    rc = compute_lora_t(op.x, op.ldx, op.row_exp, m, k, 0, *down, lora->rank, ws, stream, &t);
    if (rc) return rc;
    with_t = *lora;
    with_t.t = t;
    with_t.t_dtype = QLIN_F32;
    with_t.ldt = lora->rank;
    lora = &with_t;
  }
  rc = attach_lora(lora, a, ws, stream);
  if (rc) return rc;
  return run_f16_gemm(a, stream);
}

int qlin_gguf_linear(const void* x, int x_dtype, int64_t m, int64_t k, int64_t ldx, const void* packed,
                     const int32_t* row_exp, int qtype, int64_t n, const void* bias, int bias_dtype, void* y,
                     int y_dtype, int64_t ldy, void* workspace, size_t workspace_bytes, void* stream) {
  return gguf_linear_impl(x, x_dtype, m, k, ldx, packed, row_exp, qtype, n, bias, bias_dtype, y, y_dtype, ldy,
                          workspace, workspace_bytes, stream, nullptr);
}

size_t qlin_gguf_linear_lora_workspace(int64_t m, int64_t n, int64_t k, int x_dtype, int64_t ldx, int64_t rank) {
  (void)x_dtype;
  (void)ldx;
  LoraArgs l{};
  l.rank = rank;
  size_t pb = 0;
  for (int fmt : kGgufFormats)
    pb = std::max(pb, f16_gemm_partial_bytes((int)m, (int)n, (int)(k + lora_k_of(&l)), fmt, 0, 0));
  return f16_operand_bytes(m, k) + align256(pb) + lora_bytes(m, n, &l);
}

size_t qlin_gguf_linear_lora_down_workspace(int64_t m, int64_t n, int64_t k, int x_dtype, int64_t ldx, int64_t rank) {
  return qlin_gguf_linear_lora_workspace(m, n, k, x_dtype, ldx, rank) + lora_down_bytes(m, k, rank);
}

int qlin_gguf_linear_lora_down(const void* x, int x_dtype, int64_t m, int64_t k, int64_t ldx, const void* packed,
                               const int32_t* row_exp, int qtype, int64_t n, const void* bias, int bias_dtype,
                               const void* lora_down, int lora_down_dtype, int64_t ldd, const void* lora_up,
                               int lora_up_dtype, int64_t ldu, int64_t rank, float lora_scale, void* y, int y_dtype,
                               int64_t ldy, void* workspace, size_t workspace_bytes, void* stream) {
  const LoraArgs l{lora_down, QLIN_F32, rank, lora_up, lora_up_dtype, ldu, rank, lora_scale};
  const LoraDown d{lora_down, lora_down_dtype, ldd};
  return gguf_linear_impl(x, x_dtype, m, k, ldx, packed, row_exp, qtype, n, bias, bias_dtype, y, y_dtype, ldy,
                          workspace, workspace_bytes, stream, &l, &d);
}

int qlin_gguf_linear_lora(const void* x, int x_dtype, int64_t m, int64_t k, int64_t ldx, const void* packed,
                          const int32_t* row_exp, int qtype, int64_t n, const void* bias, int bias_dtype,
                          const void* lora_t, int lora_t_dtype, int64_t ldt, const void* lora_up, int lora_up_dtype,
                          int64_t ldu, int64_t rank, float lora_scale, void* y, int y_dtype, int64_t ldy,
                          void* workspace, size_t workspace_bytes, void* stream) {
  const LoraArgs l{lora_t, lora_t_dtype, ldt, lora_up, lora_up_dtype, ldu, rank, lora_scale};
  return gguf_linear_impl(x, x_dtype, m, k, ldx, packed, row_exp, qtype, n, bias, bias_dtype, y, y_dtype, ldy,
                          workspace, workspace_bytes, stream, &l);
}

int qlin_gguf_linear_slabs(const void* x, int64_t m, int64_t k, int64_t ldx, int x_slabs, int64_t x_slab_stride,
                           const void* packed, const int32_t* row_exp, int qtype, int64_t n, const void* bias,
                           int bias_dtype, void* y, int y_dtype, int64_t ldy, void* workspace, size_t workspace_bytes,
                           void* stream) {
  return gguf_slabs_impl(x, m, k, ldx, x_slabs, x_slab_stride, packed, row_exp, qtype, n, bias, bias_dtype, y, y_dtype,
                         ldy, workspace, workspace_bytes, stream, nullptr);
}

int qlin_gguf_linear_allgather(const void* x, int64_t m, int64_t k, int64_t ldx, int x_slabs, int64_t x_slab_stride,
                               const void* packed, const int32_t* row_exp, int qtype, int64_t n, const void* bias,
                               int bias_dtype, int world, int rank, void* const* y_ranks, int y_dtype, int64_t ldy,
                               void* const* sync_ranks, uint32_t timeout_ms, void* workspace, size_t workspace_bytes,
                               void* stream) {
  if (world < 1 || world > kMaxPeers || rank < 0 || rank >= world || y_ranks == nullptr || sync_ranks == nullptr) {
    set_error("allgather: world must be 1..%d with 0 <= rank < world and per-rank pointer arrays", kMaxPeers);
    return QLIN_EINVAL;
  }
  if ((y_dtype != QLIN_F16 && y_dtype != QLIN_BF16) || n % 8 != 0 || ldy % 8 != 0) {
    set_error("allgather: fp16/bf16 output with n and ldy multiples of 8");
    return QLIN_EDECLINE;
  }
  PeerOut po{};
  po.ndst = world;
  po.world = world;
  po.self = rank;
  po.wait = 1;
  po.signal = 1;
  po.timeout_ms = timeout_ms;
  for (int r = 0; r < world; ++r) {
    if (y_ranks[r] == nullptr || sync_ranks[r] == nullptr || (reinterpret_cast<uintptr_t>(y_ranks[r]) & 15) ||
        (reinterpret_cast<uintptr_t>(sync_ranks[r]) & 63)) {
      set_error("allgather: rank %d output (16-byte) or pad (64-byte) pointer missing or misaligned", r);
      return QLIN_EINVAL;
    }
    po.dst[r] = y_ranks[r];
    po.sync[r] = reinterpret_cast<PeerSync*>(sync_ranks[r]);
  }
  po.own = po.sync[rank];
  // Destination tensor maps for the TMA-store epilogue: {n, m} over each slab, boxes of 128
  // channels x 32 tokens (the staged chunk).
  PeerMaps maps;
  memset(&maps, 0, sizeof(maps));
  po.tma = 1;
  for (int r = 0; r < world && po.tma; ++r) {
    if (make_tmap_2d(&maps.m[r], y_ranks[r], y_dtype == QLIN_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                                   : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                     2, (uint64_t)n, (uint64_t)m, (uint64_t)ldy * 2, 128, 32, CU_TENSOR_MAP_SWIZZLE_NONE) != 0)
      po.tma = 0;  // fall back to element stores
  }
  if (m == 0 || n == 0) {
    set_error("allgather: empty shapes are not supported (every rank must take part in every step)");
    return QLIN_EINVAL;
  }
  return gguf_slabs_impl(x, m, k, ldx, x_slabs, x_slab_stride, packed, row_exp, qtype, n, bias, bias_dtype,
                         y_ranks[rank], y_dtype, ldy, workspace, workspace_bytes, stream, &po, &maps);
}

int qlin_kitchen_w4a8_grid(const void* qdata, int bits, const void* s_rel, const float* codebook, int group,
                           int64_t n, int64_t k, int8_t* out, void* stream) {
  if ((bits != 4 && bits != 6) || n < 0 || k < 0 || group < 16 || group % 16 != 0 || k % group != 0 ||
      (bits == 6 && k % 32 != 0) || (n > 0 && k > 0 && (qdata == nullptr || s_rel == nullptr || out == nullptr))) {
    set_error("kitchen grid: bits 4 or 6, group a multiple of 16 dividing k (k a multiple of 32 for 6 bits)");
    return QLIN_EINVAL;
  }
  if ((reinterpret_cast<uintptr_t>(qdata) & 7) || (reinterpret_cast<uintptr_t>(out) & 15) ||
      (bits == 6 && ((k / 2) % 4 != 0 || (n > 1 && ((k * 6 / 8) % 8 != 0))))) {
    set_error("kitchen grid: qdata rows must be 8-byte aligned and out 16-byte aligned");
    return QLIN_EDECLINE;
  }
  launch_kitchen_grid(reinterpret_cast<const uint8_t*>(qdata), reinterpret_cast<const uint8_t*>(s_rel), codebook,
                      bits, group, (int)n, (int)k, out, reinterpret_cast<cudaStream_t>(stream));
  return check_cuda("kitchen grid launch");
}

size_t qlin_peer_sync_bytes(void) { return sizeof(PeerSync); }

int qlin_peer_alloc(size_t bytes, void** ptr) {
  if (ptr == nullptr || bytes == 0) {
    set_error("peer_alloc: null result pointer or zero size");
    return QLIN_EINVAL;
  }
  *ptr = nullptr;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return check_cuda("cudaMalloc (peer buffer)");
  if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
    cudaFree(p);
    return check_cuda("cudaMemset (peer buffer)");
  }
  *ptr = p;
  return QLIN_OK;
}

int qlin_peer_free(void* ptr) {
  if (ptr != nullptr && cudaFree(ptr) != cudaSuccess) return check_cuda("cudaFree (peer buffer)");
  return QLIN_OK;
}

int qlin_peer_export(const void* ptr, void* handle) {
  if (ptr == nullptr || handle == nullptr) {
    set_error("peer_export: null pointer");
    return QLIN_EINVAL;
  }
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, const_cast<void*>(ptr)) != cudaSuccess) return check_cuda("cudaIpcGetMemHandle");
  static_assert(sizeof(h) == QLIN_PEER_HANDLE_BYTES, "IPC handle size");
  memcpy(handle, &h, sizeof(h));
  return QLIN_OK;
}

int qlin_peer_import(const void* handle, void** ptr) {
  if (ptr == nullptr || handle == nullptr) {
    set_error("peer_import: null pointer");
    return QLIN_EINVAL;
  }
  *ptr = nullptr;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  if (cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
    return check_cuda("cudaIpcOpenMemHandle");
  return QLIN_OK;
}

int qlin_peer_close(void* ptr) {
  if (ptr != nullptr && cudaIpcCloseMemHandle(ptr) != cudaSuccess) return check_cuda("cudaIpcCloseMemHandle");
  return QLIN_OK;
}

namespace {
// One thread: the bounded wait of the flag protocol, without computing or publishing anything.
__global__ void peer_wait_kernel(const PeerOut po, DeviceStatus* status) {
  if (threadIdx.x == 0) peer_wait(po, status, 9);
}
}  // namespace

int qlin_peer_wait(int world, int rank, void* const* sync_ranks, uint32_t timeout_ms, void* stream) {
  if (world < 1 || world > kMaxPeers || rank < 0 || rank >= world || sync_ranks == nullptr) {
    set_error("peer_wait: 1 <= world <= %d, 0 <= rank < world and one flag pad per rank", kMaxPeers);
    return QLIN_EINVAL;
  }
  PeerOut po;
  memset(&po, 0, sizeof(po));
  po.world = world;
  po.self = rank;
  po.timeout_ms = timeout_ms;
  for (int r = 0; r < world; ++r) {
    if (sync_ranks[r] == nullptr) {
      set_error("peer_wait: null flag pad for rank %d", r);
      return QLIN_EINVAL;
    }
    po.sync[r] = reinterpret_cast<PeerSync*>(sync_ranks[r]);
  }
  po.own = po.sync[rank];
  peer_wait_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      po, reinterpret_cast<DeviceStatus*>(device_status_ptr()));
  return check_cuda("peer wait launch");
}

// Same computation as qlin_gguf_linear, with the workspace taken from the library's static device
// scratch instead of the caller.  Nothing is allocated, so it suits callers that cannot allocate
// device memory at call time.  The first call in a CUDA context (once per device, again after a
// reset or under another context) looks up the scratch address (make it before any stream
// capture).  All calls on a device share one scratch: calls that overlap on
// the GPU (different streams, or other threads) race and must be ordered by the caller.
// Every scratch byte a call reads is written earlier in the same call, so stale contents from a
// previous call are never read and nothing needs clearing.
int qlin_gguf_linear_noalloc(const void* x, int x_dtype, int64_t m, int64_t k, int64_t ldx, const void* packed,
                             const int32_t* row_exp, int qtype, int64_t n, const void* bias, int bias_dtype, void* y,
                             int y_dtype, int64_t ldy, void* stream) {
  if (m < 0 || n < 0 || k < 0) {
    set_error("qlin_gguf_linear_noalloc: bad sizes");
    return QLIN_EINVAL;
  }
  const size_t need = qlin_gguf_linear_workspace(m, n, k, x_dtype, ldx);
  if (need > kNoAllocScratchBytes) {
    set_error("qlin_gguf_linear_noalloc: this call needs %zu bytes of scratch, more than the fixed %zu bytes "
              "(16 MiB); use qlin_gguf_linear with a caller workspace",
              need, kNoAllocScratchBytes);
    return QLIN_EINVAL;
  }
  void* scratch = nullptr;
  int rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  return qlin_gguf_linear(x, x_dtype, m, k, ldx, packed, row_exp, qtype, n, bias, bias_dtype, y, y_dtype, ldy,
                          scratch, kNoAllocScratchBytes, stream);
}

int qlin_gguf_dequantize(const void* raw, int qtype, int64_t n, int64_t k, void* out, int out_dtype, void* stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  const int qk = gguf_block_values(qtype);
  if (qk == 0 || out_kind_of(out_dtype) < 0) {
    set_error("unsupported GGUF type %d or out dtype %d", qtype, out_dtype);
    return QLIN_EDECLINE;
  }
  if (n < 0 || k < 0 || (n * k) % qk != 0) {
    set_error("n*k must be a whole number of blocks");
    return QLIN_EINVAL;
  }
  if (n * k == 0) return QLIN_OK;
  launch_gguf_dequant(reinterpret_cast<const uint8_t*>(raw), qtype, (long long)(n * k), out, out_kind_of(out_dtype),
                      stream);
  return check_cuda("gguf dequantize launch");
}

// ------------------------------------------------------------------------------------------ W4A8 / W6A8
int qlin_w4a8_repacked_bytes(int bits, int layout, int64_t n, int64_t k, size_t* bytes) {
  if ((bits != 4 && bits != 6) || layout < 0 || layout > 1 || (bits == 4 && layout != 0) || n < 0 || k <= 0 ||
      k % 128 != 0) {
    set_error("unsupported packed-weight format bits=%d layout=%d k=%lld (k must be a multiple of 128)", bits, layout,
              (long long)k);
    return QLIN_EDECLINE;
  }
  if (bytes) *bytes = bits == 4 ? (size_t)n * k / 2 : w6_repacked_bytes((int)n, (int)k);
  return QLIN_OK;
}

int qlin_w4a8_repack(const void* packed, int bits, int layout, int64_t n, int64_t k, void* out, size_t out_bytes,
                     void* stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  size_t need = 0;
  int rc = qlin_w4a8_repacked_bytes(bits, layout, n, k, &need);
  if (rc) return rc;
  if (out_bytes < need || packed == nullptr || out == nullptr || (reinterpret_cast<uintptr_t>(out) & 15)) {
    set_error("repack output needs %zu bytes, 16-byte aligned", need);
    return QLIN_EINVAL;
  }
  if (need == 0) return QLIN_OK;
  if (bits == 4) {
    if (cudaMemcpyAsync(out, packed, need, cudaMemcpyDeviceToDevice, stream) != cudaSuccess)
      return check_cuda("w4 repack copy");
    return QLIN_OK;
  }
  launch_w6_repack(reinterpret_cast<const uint8_t*>(packed), layout, (int)n, (int)k, reinterpret_cast<uint8_t*>(out),
                   stream);
  return check_cuda("w6 repack launch");
}

size_t qlin_w4a8_linear_workspace(int64_t m, int64_t n, int64_t k, int rotate_group) {
  (void)n;
  (void)rotate_group;
  return align256((size_t)m * round_up(k, 128)) + align256((size_t)m * 4);
}

int qlin_w4a8_linear(const void* x, int x_dtype, int64_t m, int64_t k, int64_t ldx, const void* w, int bits, int group,
                     int64_t n, const void* scales, int scale_dtype, int rotate_group, const void* bias,
                     int bias_dtype, void* y, int y_dtype, int64_t ldy, void* workspace, size_t workspace_bytes,
                     void* stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (m < 0 || n < 0 || k < 0 || ldx < k || ldy < n) {
    set_error("bad sizes");
    return QLIN_EINVAL;
  }
  if (m == 0 || n == 0) return QLIN_OK;
  const bool per_channel = group == 0;
  if ((bits != 4 && bits != 6) || k % 128 != 0 || !is_float_dtype(x_dtype) || out_kind_of(y_dtype) < 0 ||
      bias_kind_of(bias, bias_dtype) < 0 || !valid_group(rotate_group) || (rotate_group && k % rotate_group) ||
      (per_channel ? scale_dtype != QLIN_F32 : (scale_dtype != QLIN_F16 || group % 32 != 0 || k % group != 0)) ||
      m > 0x7fffffff || n > 0x7fffffff || k > 0x7fffffff) {
    set_error("unsupported W%dA8 arguments: k=%lld group=%d scale dtype %d (k must be a multiple of 128 and of "
              "the group; group scales fp16, per-channel scales fp32)",
              bits, (long long)k, group, scale_dtype);
    return QLIN_EDECLINE;
  }
  if (x == nullptr || w == nullptr || scales == nullptr || y == nullptr || (reinterpret_cast<uintptr_t>(w) & 15)) {
    set_error("null or misaligned pointer (weights need 16-byte alignment)");
    return QLIN_EINVAL;
  }
  Carver ws{reinterpret_cast<uint8_t*>(workspace), workspace_bytes};
  const int64_t kp = round_up(k, 128);
  int8_t* xq = reinterpret_cast<int8_t*>(ws.take((size_t)m * kp));
  float* sx = reinterpret_cast<float*>(ws.take((size_t)m * 4));
  if (ws.off > ws.cap || workspace == nullptr) {
    set_error("workspace too small: need %zu bytes", ws.off);
    return QLIN_EINVAL;
  }
  if (launch_prologue(x, x_dtype, ldx, (int)m, (int)k, (int)kp, rotate_group, 1, xq, nullptr, sx, 1, stream) != 0) {
    set_error("unsupported rotation group %d", rotate_group);
    return QLIN_EDECLINE;
  }
  int rc = check_cuda("quantize launch");
  if (rc) return rc;
  return run_i8_gemm(bits, xq, kp, sx, (int)m, (int)n, (int)k, w, per_channel ? (int)k : group, scales,
                     per_channel ? I8S_CHANNEL_F32 : I8S_GROUP_F16, bias, bias_kind_of(bias, bias_dtype), y,
                     out_kind_of(y_dtype), ldy, stream);
}

// ------------------------------------------------------------------------------------------ prologues
int qlin_prologue_f16(const void* x, int x_dtype, int64_t m, int64_t k, int64_t ldx, int rotate_group, void* out,
                      int64_t ldo, int32_t* row_exp, void* stream_) {
  if (!is_float_dtype(x_dtype) || !valid_group(rotate_group) || (rotate_group && k % rotate_group) || ldo < k) {
    set_error("unsupported prologue arguments");
    return QLIN_EDECLINE;
  }
  if (m == 0) return QLIN_OK;
  launch_prologue(x, x_dtype, ldx, (int)m, (int)k, (int)ldo, rotate_group, 0, out, row_exp, nullptr, 0,
                  reinterpret_cast<cudaStream_t>(stream_));
  return check_cuda("prologue launch");
}

int qlin_quantize_rows_int8(const void* x, int x_dtype, int64_t m, int64_t k, int64_t ldx, int rotate_group, int perm,
                            int8_t* out, int64_t ldo, float* scale, void* stream_) {
  if (!is_float_dtype(x_dtype) || !valid_group(rotate_group) || (rotate_group && k % rotate_group) || ldo < k ||
      (perm && ldo % 8)) {
    set_error("unsupported quantize arguments");
    return QLIN_EDECLINE;
  }
  if (m == 0) return QLIN_OK;
  launch_prologue(x, x_dtype, ldx, (int)m, (int)k, (int)ldo, rotate_group, 1, out, nullptr, scale, perm,
                  reinterpret_cast<cudaStream_t>(stream_));
  return check_cuda("quantize launch");
}

}  // extern "C"
