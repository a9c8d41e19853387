/* qlin: B200 (sm_100a) fused dequantize-and-GEMM linears for quantized diffusion-model weights.
 *
 * C ABI of libqlin.so.  Plain pointers and sizes only; every pointer named "device" is CUDA device
 * memory on the current device, and `stream` is a cudaStream_t (NULL = legacy default stream).
 *
 * Ownership: the caller allocates every input, output and workspace.  The library never
 * allocates, keeps no per-call state and launches only on `stream` (stream-ordered, re-entrant).
 * Errors: functions return QLIN_OK or a positive qlin_status; qlin_last_error() gives a message
 * for the calling thread.  QLIN_EDECLINE means "unsupported input, use the stock path" and
 * mirrors the reference's `mps.linear(layer, x) -> None` decline
 * (docs/research/2026-10-03-gguf-on-metal.md:117 in roblennon/mac-kernels-public).
 *
 * Dtype codes: 0 f32, 1 f16, 2 bf16, 3 int8, 4 uint8, 5 int32, 6 float8_e4m3fn.
 * Shapes: X [m, k] row-major with row pitch ldx elements; Y [m, n] row-major with pitch ldy.
 * Y = X . W^T (+ bias) with W [n, k].
 */
#ifndef QLIN_H_
#define QLIN_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum qlin_status {
  QLIN_OK = 0,
  QLIN_EDECLINE = 1, /* unsupported dtype / format / alignment: caller takes the stock path   */
  QLIN_EINVAL = 2,   /* inconsistent arguments (sizes, null pointers, workspace too small)    */
  QLIN_ECUDA = 3,    /* a CUDA runtime call failed; see qlin_last_error()                     */
  QLIN_ETIMEOUT = 4  /* a kernel gave up a bounded wait (reported by qlin_device_status)      */
};

enum qlin_dtype { QLIN_F32 = 0, QLIN_F16 = 1, QLIN_BF16 = 2, QLIN_I8 = 3, QLIN_U8 = 4, QLIN_I32 = 5, QLIN_E4M3 = 6 };

/* ggml type ids accepted by the GGUF entry points. */
enum qlin_gguf_type {
  QLIN_Q4_0 = 2, QLIN_Q4_1 = 3, QLIN_Q5_0 = 6, QLIN_Q5_1 = 7, QLIN_Q8_0 = 8, QLIN_Q2_K = 10, QLIN_Q3_K = 11,
  QLIN_Q4_K = 12, QLIN_Q5_K = 13, QLIN_Q6_K = 14, QLIN_IQ4_NL = 20, QLIN_IQ4_XS = 23
};

const char* qlin_version(void);
const char* qlin_last_error(void);

/* Reads the device-side status word of the current device (synchronizes the device).  Returns
 * 0 when no kernel timed out, else QLIN_ETIMEOUT and *where = (block << 8) | site.  reset != 0
 * clears it. */
int qlin_device_status(int reset, uint32_t* where);

/* Bounds record of the library built with -DQLIN_CHECKS (libqlin_checked.so; the library is
 * otherwise the same).  That build tests every global access the hardware does not bound by
 * itself, and every computed shared-memory index, against limits the host derives from the
 * arguments of each call; a failed check skips the access and is recorded, never trapped.
 * Writes the number of failed checks since the last reset to *count and the first failure's site
 * (see qlin_checks.cuh), index, limit and block.  Returns QLIN_OK, or QLIN_EDECLINE from a library
 * built without checks.  reset != 0 clears the record.  Synchronizes the device.  No counterpart
 * in the reference (it has no such build). */
int qlin_bounds_check(int reset, uint32_t* count, uint32_t* site, int64_t* index, int64_t* limit, uint32_t* block);

/* ------------------------------------------------------------------------------------------
 * INT8 ConvRot weight-only linear.
 * Replaces comfy-kitchen `int8_linear(x, qdata, scale, bias, out_dtype, convrot, convrot_groupsize)`
 * (call sites bench/bench_ck01_int8.py:57, bench/bench_lora_fused_rank.py:39; contract
 * docs/upstream/comfy-kitchen-mps-backend.md:44-56 in the reference).
 *   q      int8 [n, k] row-major, stored already rotated (W_rot = W . H^T per group)
 *   scale  per-output-channel scale [n] (dtype f32 or f16)
 *   bias   [n] (f16 / f32 / bf16) or NULL
 *   convrot_group  0 (no rotation) or the Hadamard block size: 32 / 128 (Sylvester) or 64 / 256
 *                  (the reference's H4 Kronecker construction, modal/weight_error_app.py:90-98)
 * x dtype f16 / bf16 / f32; y dtype f16 / bf16 / f32.  Requires k % 16 == 0 (and % group).
 * ------------------------------------------------------------------------------------------ */
size_t qlin_int8_linear_workspace(int64_t m, int64_t n, int64_t k);
int qlin_int8_linear(const void* x, int x_dtype, int64_t m, int64_t k, int64_t ldx, const int8_t* q, int64_t n,
                     const void* scale, int scale_dtype, const void* bias, int bias_dtype, int convrot_group,
                     void* y, int y_dtype, int64_t ldy, void* workspace, size_t workspace_bytes, void* stream);

/* The INT8 linear with an unmerged LoRA fused in: y = (linear) + lora_scale * t . up^T, where
 * t = x . down^T [m, rank] is computed by the caller (a plain GEMM, e.g. cuBLAS) and passed with its
 * row pitch ldt; up [n, rank] with pitch ldu (dtypes f32 / f16 / bf16), rank <= 256.  The LoRA
 * term runs as extra K stages of the same tensor-core GEMM (bf16 operands, fp32 accumulator), so it
 * is added before the output's single rounding.  Replaces the fused LoRA epilogue of the reference's
 * backend (`lora_down`, `lora_up`, `lora_scale`; docs/upstream/comfy-kitchen-mps-backend.md:35,
 * docs/findings.md:251-273). */
size_t qlin_int8_linear_lora_workspace(int64_t m, int64_t n, int64_t k, int64_t rank);
int qlin_int8_linear_lora(const void* x, int x_dtype, int64_t m, int64_t k, int64_t ldx, const int8_t* q, int64_t n,
                          const void* scale, int scale_dtype, const void* bias, int bias_dtype, int convrot_group,
                          const void* lora_t, int lora_t_dtype, int64_t ldt, const void* lora_up, int lora_up_dtype,
                          int64_t ldu, int64_t rank, float lora_scale, void* y, int y_dtype, int64_t ldy,
                          void* workspace, size_t workspace_bytes, void* stream);

/* The INT8 LoRA linear with the down factor itself instead of t: down [rank, k] with row pitch ldd
 * (f32 / f16 / bf16), rank <= 256.  t = x . down^T is computed inside the library by the same
 * tensor-core GEMM on the rotated, per-row normalized fp16 activation against the down factor put
 * through the same prologue (x . down^T = rot(x) . rot(down)^T for the orthonormal block rotation),
 * fp32 accumulation; then the fused up-projection stages as in qlin_int8_linear_lora.  No library
 * GEMM runs.  Replaces the reference backend's fused LoRA, whose down factor rides along the main
 * GEMM (docs/upstream/comfy-kitchen-mps-backend.md:52-53). */
size_t qlin_int8_linear_lora_down_workspace(int64_t m, int64_t n, int64_t k, int64_t rank);
int qlin_int8_linear_lora_down(const void* x, int x_dtype, int64_t m, int64_t k, int64_t ldx, const int8_t* q,
                               int64_t n, const void* scale, int scale_dtype, const void* bias, int bias_dtype,
                               int convrot_group, const void* lora_down, int lora_down_dtype, int64_t ldd,
                               const void* lora_up, int lora_up_dtype, int64_t ldu, int64_t rank, float lora_scale,
                               void* y, int y_dtype, int64_t ldy, void* workspace, size_t workspace_bytes,
                               void* stream);

/* ------------------------------------------------------------------------------------------
 * Input gradient of the INT8 ConvRot linear for a frozen weight: dx = dy . W, where
 * W = (q * scale) un-rotated per block (W = W_rot . H; H symmetric, the forward's rotation).
 * Replaces comfy-kitchen's MPS `int8_linear_grad_input(dy, q, s, convrot, convrot_groupsize,
 * out_dtype)` (call sites bench/bench_int8_backward.py:52, bench/probe_packed_backward_real_k.py:151
 * in the reference; its W4A8 twin `w4a8_linear_grad_input` runs on the kitchen layout's int8 grid).
 *
 * qlin_int8_grad_weight writes, once per weight, the transposed copy the gradient GEMM reads:
 * qt int8 [k, roundup(n, 64)] (zeros past column n), qlin_int8_grad_weight_bytes(n, k) bytes,
 * 16-byte aligned.  qlin_int8_linear_grad_input then runs dy * scale (per column) normalized to
 * fp16 per row, the tensor-core GEMM over n, and, when rotate_group != 0, the block Hadamard of
 * every row of dx (computed in fp32, rounded once to dx's dtype).
 *   dy  [m, n] with row pitch lddy (f16 / bf16 / f32); scale [n] (f16 / f32)
 *   dx  [m, k] with row pitch lddx (f16 / bf16 / f32); k % 16 == 0 (and % rotate_group)
 * n == 0 writes zeros.  The workspace holds the fp16 operand, split-K partials and, with a
 * rotation, the fp32 dx before it.
 * ------------------------------------------------------------------------------------------ */
size_t qlin_int8_grad_weight_bytes(int64_t n, int64_t k);
int qlin_int8_grad_weight(const int8_t* q, int64_t n, int64_t k, int8_t* qt, size_t qt_bytes, void* stream);
size_t qlin_int8_linear_grad_input_workspace(int64_t m, int64_t n, int64_t k, int rotate_group);
int qlin_int8_linear_grad_input(const void* dy, int dy_dtype, int64_t m, int64_t n, int64_t lddy, const int8_t* qt,
                                int64_t k, const void* scale, int scale_dtype, int rotate_group, void* dx,
                                int dx_dtype, int64_t lddx, void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------------------------
 * GGUF block-format linear: the twelve types of the reference's kernel, Q4_0, Q4_1, Q5_0, Q5_1,
 * Q8_0, Q2_K, Q3_K, Q4_K, Q5_K, Q6_K, IQ4_NL, IQ4_XS (docs/research/2026-10-03-gguf-on-metal.md:59).
 * Replaces comfy-kitchen `gguf_linear(x, weight, qtype, shape, bias, out_dtype)` and its decode
 * helpers `_decode` / `gguf_row_exp_<type>` (bench/bench_gguf_linear.py:120-127; design
 * docs/research/2026-10-03-gguf-on-metal.md:83-97 in the reference).
 *
 * qlin_gguf_repack turns raw ggml blocks [n rows of k/QK blocks] into the resident stage layout
 * (one time per weight) and writes the per-row exponents e (row_exp, length padded_n = n rounded
 * up to 128).  The linear feeds the tensor cores fp16 weights w * 2^-e, where w is gguf-py 0.19.0's
 * fp32 value: exactly RN16(w * 2^-e) for Q8_0, Q4_0, Q5_0 and IQ4_NL; one fp16 fma of exact fp16
 * factors (the exact value rounded once) for Q4_1 and Q5_1; within two fp16 rounding steps (block
 * scale products rounded once to fp16, then one fp16 multiply or fma) for the K-quants and IQ4_XS.
 * The epilogue restores 2^e, adds bias in fp32 and rounds once to the output dtype.
 * qlin_gguf_dequantize is bit-exact with gguf-py for every type.  Requires k to be a whole number
 * of blocks per row.
 * ------------------------------------------------------------------------------------------ */
int qlin_gguf_repacked_bytes(int qtype, int64_t n, int64_t k, size_t* bytes, int64_t* padded_n);
int qlin_gguf_repack(const void* raw, int qtype, int64_t n, int64_t k, void* packed, size_t packed_bytes,
                     int32_t* row_exp, int64_t row_exp_len, void* stream);
size_t qlin_gguf_linear_workspace(int64_t m, int64_t n, int64_t k, int x_dtype, int64_t ldx);
int qlin_gguf_linear(const void* x, int x_dtype, int64_t m, int64_t k, int64_t ldx, const void* packed,
                     const int32_t* row_exp, int qtype, int64_t n, const void* bias, int bias_dtype, void* y,
                     int y_dtype, int64_t ldy, void* workspace, size_t workspace_bytes, void* stream);

/* The GGUF linear with an unmerged LoRA fused in (as qlin_int8_linear_lora). */
size_t qlin_gguf_linear_lora_workspace(int64_t m, int64_t n, int64_t k, int x_dtype, int64_t ldx, int64_t rank);
int qlin_gguf_linear_lora(const void* x, int x_dtype, int64_t m, int64_t k, int64_t ldx, const void* packed,
                          const int32_t* row_exp, int qtype, int64_t n, const void* bias, int bias_dtype,
                          const void* lora_t, int lora_t_dtype, int64_t ldt, const void* lora_up, int lora_up_dtype,
                          int64_t ldu, int64_t rank, float lora_scale, void* y, int y_dtype, int64_t ldy,
                          void* workspace, size_t workspace_bytes, void* stream);

/* The GGUF LoRA linear with the down factor itself (as qlin_int8_linear_lora_down, no rotation). */
size_t qlin_gguf_linear_lora_down_workspace(int64_t m, int64_t n, int64_t k, int x_dtype, int64_t ldx, int64_t rank);
int qlin_gguf_linear_lora_down(const void* x, int x_dtype, int64_t m, int64_t k, int64_t ldx, const void* packed,
                               const int32_t* row_exp, int qtype, int64_t n, const void* bias, int bias_dtype,
                               const void* lora_down, int lora_down_dtype, int64_t ldd, const void* lora_up,
                               int lora_up_dtype, int64_t ldu, int64_t rank, float lora_scale, void* y, int y_dtype,
                               int64_t ldy, void* workspace, size_t workspace_bytes, void* stream);

/* The GGUF linear with the fp16 activation given as x_slabs column slabs, [x_slabs][m][k / x_slabs]
 * (slab i holds columns i*k/x_slabs ...; rows ldx apart, slabs x_slab_stride elements apart) —
 * the layout an all-gather of column shards produces, consumed in place by the N-sharded multi-GPU
 * stack.  No counterpart in the reference (which runs on one GPU).  k / x_slabs must be a multiple
 * of 64.  Workspace: qlin_gguf_linear_workspace(m, n, k, QLIN_F16, ldx). */
int qlin_gguf_linear_slabs(const void* x, int64_t m, int64_t k, int64_t ldx, int x_slabs, int64_t x_slab_stride,
                           const void* packed, const int32_t* row_exp, int qtype, int64_t n, const void* bias,
                           int bias_dtype, void* y, int y_dtype, int64_t ldy, void* workspace, size_t workspace_bytes,
                           void* stream);

/* ------------------------------------------------------------------------------------------
 * Sharded linear fused with the all-gather of its output (one process per GPU of a node).
 * No counterpart in the reference (which runs on one GPU); it replaces the slab linear above
 * followed by an all-gather of the world ranks' [m, n] output shards into [world][m][n] slabs.
 *
 * Each rank computes its [m, n] shard and its epilogue stores every finished tile into all
 * ranks' gathered buffers over NVLink: y_ranks[r] is this rank's slab inside rank r's buffer
 * (row pitch ldy; a peer buffer mapped into this process with qlin_peer_import, or local for
 * r == rank).  sync_ranks[r] is rank r's flag pad (qlin_peer_sync_bytes() bytes of a buffer
 * from qlin_peer_alloc, zero at start; mapped likewise).  Before reading x the kernel waits until
 * every rank finished its previous call of this function; every rank must therefore make the same
 * sequence of calls.  The wait is bounded by timeout_ms (0: 10 s): on expiry the call's tiles are
 * skipped and qlin_device_status reports QLIN_ETIMEOUT; the pads are then out of step and must be
 * reallocated.  Output fp16/bf16 with n and ldy multiples of 8; m, n > 0.
 * Workspace: qlin_gguf_linear_workspace(m, n, k, QLIN_F16, ldx).
 * ------------------------------------------------------------------------------------------ */
#define QLIN_PEER_HANDLE_BYTES 64
int qlin_gguf_linear_allgather(const void* x, int64_t m, int64_t k, int64_t ldx, int x_slabs, int64_t x_slab_stride,
                               const void* packed, const int32_t* row_exp, int qtype, int64_t n, const void* bias,
                               int bias_dtype, int world, int rank, void* const* y_ranks, int y_dtype, int64_t ldy,
                               void* const* sync_ranks, uint32_t timeout_ms, void* workspace, size_t workspace_bytes,
                               void* stream);
size_t qlin_peer_sync_bytes(void);
/* Zero-filled device memory on the current device that other processes can map (cudaMalloc). */
int qlin_peer_alloc(size_t bytes, void** ptr);
int qlin_peer_free(void* ptr);
/* handle: QLIN_PEER_HANDLE_BYTES bytes (a CUDA IPC memory handle of ptr's allocation, which must
 * start at ptr: a qlin_peer_alloc pointer).  qlin_peer_import maps another process's buffer
 * into this one (peer access enabled on first use); qlin_peer_close unmaps it. */
int qlin_peer_export(const void* ptr, void* handle);
int qlin_peer_import(const void* handle, void** ptr);
int qlin_peer_close(void* ptr);
/* Stream-ordered: waits (one-thread kernel, bounded by timeout_ms, 0: 10 s) until every rank has
 * finished as many qlin_gguf_linear_allgather calls as this rank, i.e. until the other ranks'
 * stores into this rank's gathered buffers from those calls are complete.  Call it before
 * reading a gathered output that no later all-gather call waits for (the last one of a
 * sequence).  On expiry qlin_device_status reports QLIN_ETIMEOUT.  No counterpart in the
 * reference (which runs on one GPU). */
int qlin_peer_wait(int world, int rank, void* const* sync_ranks, uint32_t timeout_ms, void* stream);

/* The GGUF linear above with no workspace argument: the scratch (fp16 activation copy and split-K
 * partial sums) lives in a fixed 16 MiB array in device memory that the library reserves on every
 * device that loads it, until the process exits.  It has no counterpart in the reference; it is
 * for callers that cannot allocate device memory at call time: hosts without a caching allocator
 * (cudaMalloc synchronizes the device and costs far more than the layer) and hosts with a fixed
 * memory budget or allocation-free steady state.  Calls whose scratch need exceeds 16 MiB are
 * rejected with QLIN_EINVAL and a message; nothing is allocated.  The first call in a CUDA
 * context (per device, and again after cudaDeviceReset or under another context the caller made
 * current) looks up the scratch address (make that call before any stream capture).  Calls on one
 * device share the scratch, so calls that overlap on the GPU race: order them on one stream. */
int qlin_gguf_linear_noalloc(const void* x, int x_dtype, int64_t m, int64_t k, int64_t ldx, const void* packed,
                             const int32_t* row_exp, int qtype, int64_t n, const void* bias, int bias_dtype, void* y,
                             int y_dtype, int64_t ldy, void* stream);

/* Decode-only, bit-exact with gguf-py 0.19.0 (f32 out; f16 / bf16 out = that value rounded once).
 * Blocks are indexed by flat element, so rows may straddle blocks.  Replaces comfy-kitchen
 * `dequantize_gguf(weight, qtype, shape, out_dtype)` (docs/upstream/comfy-kitchen-mps-followups.md:43). */
int qlin_gguf_dequantize(const void* raw, int qtype, int64_t n, int64_t k, void* out, int out_dtype, void* stream);

/* ------------------------------------------------------------------------------------------
 * W4A8 / W6A8 packed-weight linears on the integer tensor cores (kind::i8, int32 accumulation).
 * Replaces comfy-kitchen `w4a8_int8_linear(x, qdata, s_rel, s_channel, ..., group_size,
 * convrot_groupsize, out_dtype)` (bench/bench_lora_fused_rank.py:42-44; positional form
 * bench/bench_lora_sidepath_kernel.py:78) for symmetric uniform weights:
 *   bits 4: values in [-8, 7] stored as nibbles u = q + 8, two per byte, even column in the low
 *           nibble (the kitchen's nibble order, modal/weight_error_app.py:145-152), [n, k/2] bytes;
 *   bits 6: values in [-32, 31]; qlin_w4a8_repack converts layout 0 (four values per three bytes:
 *           u0 | u1<<6 | u2<<12 | u3<<18 little-endian, u = q + 32) or layout 1 (the kitchen planar
 *           6-bit packing, modal/weight_error_app.py:145-152) into the kernel's stage layout.
 * Scales: group != 0 -> fp16 group scales [n, k/group] (group a multiple of 32 dividing k);
 *         group == 0 -> fp32 per-channel scales [n].
 * Activations are rotated (rotate_group, 0 = none) and quantized per token exactly like
 * qlin_quantize_rows_int8; each group's int32 sum is exact; Y = sx[m] * sum_g s[n,g] * P_g + bias
 * in fp32, rounded once.  Requires k % 128 == 0.
 * ------------------------------------------------------------------------------------------ */
int qlin_w4a8_repacked_bytes(int bits, int layout, int64_t n, int64_t k, size_t* bytes);
int qlin_w4a8_repack(const void* packed, int bits, int layout, int64_t n, int64_t k, void* out, size_t out_bytes,
                     void* stream);
size_t qlin_w4a8_linear_workspace(int64_t m, int64_t n, int64_t k, int rotate_group);
int qlin_w4a8_linear(const void* x, int x_dtype, int64_t m, int64_t k, int64_t ldx, const void* w, int bits, int group,
                     int64_t n, const void* scales, int scale_dtype, int rotate_group, const void* bias,
                     int bias_dtype, void* y, int y_dtype, int64_t ldy, void* workspace, size_t workspace_bytes,
                     void* stream);

/* The kitchen's AsymW4A8Int8Layout weight (symmetric form) -> its int8 weight grid, bit-exact:
 * grid[n, k] = clamp(rint(level[code] * s_rel[n, k / group]), -127, 127) in fp32, with
 * level = codebook (1 << bits fp32 entries) or code - 2^(bits-1).  qdata int8 [n, k * bits / 8]
 * in the kitchen's planar packing, s_rel float8_e4m3fn [n, k / group], out int8 [n, k].
 * Replaces the decode of `dequantize_w4a8` / the kitchen's w4a8_int8_linear
 * (modal/weight_error_app.py:326-336, bench/bench_w4a8_linear.py:98-99); the linear is then the
 * INT8 ConvRot linear with s_channel as the per-channel scale (the reference backend is weight-only:
 * docs/upstream/comfy-kitchen-mps-backend.md:42). */
int qlin_kitchen_w4a8_grid(const void* qdata, int bits, const void* s_rel, const float* codebook, int group,
                           int64_t n, int64_t k, int8_t* out, void* stream);

/* ------------------------------------------------------------------------------------------
 * Activation prologues (exposed for tests and for callers that reuse one prologue across
 * several linears sharing an input).
 *   qlin_prologue_f16: optional block-Hadamard rotation, then per-row power-of-two scaling
 *     (row max mapped into [2^14, 2^15)) and one rounding to fp16.  out [m, ldo] fp16,
 *     row_exp[m] = f (the row was multiplied by 2^-f).
 *   qlin_quantize_rows_int8: optional rotation, then quantize_int8_rowwise semantics
 *     (modal/weight_error_app.py:109-115): scale = max(absmax/127, 1e-30) in fp32, quotient
 *     formed in x's dtype, round half-to-even, clamp [-128, 127].  out int8 [m, ldo], scale[m] f32.
 *     perm != 0 writes each group of 8 columns in the order 0,2,4,6,1,3,5,7 (the operand order of
 *     the packed-weight kernels).
 * ------------------------------------------------------------------------------------------ */
int qlin_prologue_f16(const void* x, int x_dtype, int64_t m, int64_t k, int64_t ldx, int rotate_group, void* out,
                      int64_t ldo, int32_t* row_exp, void* stream);
int qlin_quantize_rows_int8(const void* x, int x_dtype, int64_t m, int64_t k, int64_t ldx, int rotate_group,
                            int perm, int8_t* out, int64_t ldo, float* scale, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* QLIN_H_ */
