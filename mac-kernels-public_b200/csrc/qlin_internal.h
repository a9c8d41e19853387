// Host-side declarations shared by the library's translation units (not part of the ABI).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>

namespace qlin {

struct PeerOut;
struct PeerMaps;

int launch_prologue(const void* x, int x_dtype, long long ldx, int M, int K, int Kp, int group, int mode, void* out,
                    int32_t* row_exp, float* row_scale, int perm, cudaStream_t stream);
void launch_gguf_dequant(const uint8_t* raw, int qtype, long long total, void* out, int out_dtype, cudaStream_t s);
void launch_gguf_row_exp(const uint8_t* raw, int qtype, int N, int K, int n_pad, int32_t* row_exp, cudaStream_t s);
void launch_gguf_straddle_repack(const uint8_t* raw, int qtype, int N, int K, int n_pad, int ldw, void* out,
                                 size_t out_bytes, int32_t* row_exp, cudaStream_t s);
void launch_gguf_repack(const uint8_t* raw, int qtype, int N, int K, int num_k_stages, int n_tiles, uint8_t* out,
                        size_t out_bytes, uint32_t stage_bytes, int P, int S, cudaStream_t s);
void launch_splitk_finalize(const float* partial, int splits, int M, int N, int Mp, const void* col_scale,
                            int cs_kind, const int32_t* w_row_exp, const int32_t* x_row_exp,
                            const float* x_row_scale, const void* bias, int bias_kind, void* y, int y_dtype,
                            long long ldy, cudaStream_t s,
                            const PeerOut* out = nullptr, int lora = 0, size_t partial_bytes = 0);

// Fused-LoRA operands: T'[m][r] = bf16(t[m][r] * 2^-f[m]) and U'[n][r] = bf16(up[n][r] * scale / cs[n])
// (cs: the linear's column scale; 2^e[n] for GGUF), zero past r = R and n = N.
void launch_lora_operands(const void* t, int t_dtype, long long ldt, int M, const void* up, int up_dtype,
                          long long ldu, int N, int n_pad, int R, int rk, float scale, const void* cs, int cs_kind,
                          const int32_t* w_row_exp, const int32_t* x_row_exp, void* t_out, void* u_out,
                          cudaStream_t s);
// INT8 input gradient (dX = dY . W): the transposed weight copy, dY * s normalized to fp16, and the
// block Hadamard of dX's rows (group 32, 64, 128 or 256; returns -1 for other groups).
void launch_int8_transpose(const int8_t* q, int N, int K, int8_t* qt, int ldt, cudaStream_t s);
void launch_grad_prologue(const void* dy, int dy_dtype, long long lddy, int M, int N, int Np, const void* scale,
                          int scale_f16, void* out, int32_t* row_exp, cudaStream_t s);
int launch_grad_rotate(const float* in, int M, int K, int group, void* out, int out_dtype, long long ldo,
                       cudaStream_t s);
void launch_kitchen_grid(const uint8_t* q, const uint8_t* s_rel, const float* codebook, int bits, int group, int N,
                         int K, int8_t* out, cudaStream_t s);

// Weight formats of the f16 (weight-only) GEMM family.
enum WFormat : int {
  WF_INT8 = 0, WF_F16 = 1, WF_Q4_0 = 2, WF_Q4_1 = 3, WF_Q5_0 = 6, WF_Q5_1 = 7, WF_Q8_0 = 8, WF_Q2_K = 10, WF_Q3_K = 11,
  WF_Q4_K = 12, WF_Q5_K = 13, WF_Q6_K = 14, WF_IQ4_NL = 20, WF_IQ4_XS = 23
};

struct F16GemmArgs {
  int fmt;
  const void* x;  // fp16 activations [M, ldx] (prologue output or caller's fp16 tensor)
  long long ldx;
  int x_slabs = 1;             // > 1: X is [x_slabs][M][K / x_slabs] (e.g. an all-gather of column shards)
  long long x_slab_stride = 0;  // elements between slabs
  int M, N, K;
  const void* w;  // INT8: raw int8 [N, K]; F16: fp16 [N, ldw]; GGUF: repacked stages
  long long w_bytes = 0;  // GGUF: bytes of the repacked stages (the bounds-checked build tests copies against it)
  long long ldw = 0;  // F16 weights: row pitch in elements (0: K)
  const int32_t* w_row_exp;
  const void* col_scale;
  int col_scale_kind;
  const int32_t* x_row_exp;
  const void* bias;
  int bias_kind;
  void* y;
  int y_dtype;
  long long ldy;
  float* partial;  // split-K workspace (or null)
  size_t partial_bytes;
  int tm;           // token tile (0 = auto)
  int k_splits;     // 0 = auto
  const PeerOut* out = nullptr;  // peer destinations + flag protocol (null: plain output to y)
  const PeerMaps* out_maps = nullptr;  // destination tensor maps when out->tma
  // Fused unmerged LoRA: T' bf16 [M][lora_k] and U' bf16 [n_tiles * 128][lora_k] (lora_k a
  // multiple of 64; 0 = none), prepared by launch_lora_operands.
  const void* lora_t = nullptr;
  const void* lora_u_ptr = nullptr;
  int lora_k = 0;
  // > 0: every output row times the block Hadamard of rot_group channels (32, 64 or 128) before
  // its one rounding, in the GEMM epilogue; only where f16_gemm_can_rotate() says so.
  int rot_group = 0;
};

// Returns 0 on success, a positive QLIN_* code on failure (message via set_error).
int run_f16_gemm(const F16GemmArgs& a, cudaStream_t stream);
// Whether run_f16_gemm can apply a.rot_group in its epilogue: INT8 weights, groups of 32, 64 or
// 128 (one 128-row weight tile), no small-M kernel, no K split, the staged 2-byte output path, a
// plain output.
bool f16_gemm_can_rotate(const F16GemmArgs& a);
// Small-M (M = 1) weight-streaming kernel; -1 when it does not apply.
int run_gemv(const F16GemmArgs& a, cudaStream_t stream);
size_t f16_gemm_partial_bytes(int M, int N, int K, int fmt, int tm, int k_splits);
void plan_f16(int M, int N, int K, int fmt, int* tm, int* k_splits);

uint32_t gguf_stage_bytes(int qtype, int* P, int* S);
int gguf_block_values(int qtype);
int gguf_type_size(int qtype);

void launch_w6_repack(const uint8_t* src, int layout, int N, int K, uint8_t* out, cudaStream_t s);
size_t w6_repacked_bytes(int N, int K);
int plan_i8_tm(int M);
int run_i8_gemm(int bits, const void* xq, long long kp, const float* sx, int M, int N, int K, const void* w, int group,
                const void* scales, int scale_kind, const void* bias, int bias_kind, void* y, int y_dtype,
                long long ldy, cudaStream_t stream);

void set_error(const char* fmt, ...);
int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elem, uint64_t cols, uint64_t rows,
                 uint64_t pitch_bytes, uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle swz);
int sm_count();
void* device_status_ptr();
// Unique id of the calling thread's current CUDA context (0 when there is none); the key of the
// per-context caches of device-symbol addresses.
unsigned long long current_context_id();

// Bounds records of the QLIN_CHECKS build, one reader per translation unit that launches
// kernels (qlin_checks.cuh); each returns 0, 1 in the unchecked build, -1 on a CUDA error.
struct BoundsRecord;
int bounds_read_api(BoundsRecord* out, int reset);
int bounds_read_aux(BoundsRecord* out, int reset);
int bounds_read_f16(BoundsRecord* out, int reset);
int bounds_read_f16_blk(BoundsRecord* out, int reset);
int bounds_read_f16_kq(BoundsRecord* out, int reset);
int bounds_read_gemv(BoundsRecord* out, int reset);
int bounds_read_i8(BoundsRecord* out, int reset);

}  // namespace qlin
