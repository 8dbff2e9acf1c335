/*
 * h3b.h -- C ABI of libh3b.so, the B200-native (sm_100a) W4A8 ConvRot quantised linear.
 *
 * Every pointer argument is a device pointer unless the name ends in `_host`.  The caller owns every buffer, including
 * outputs and scratch ("workspace"): no entry point allocates device memory.  Work is enqueued on `stream` (a
 * cudaStream_t; NULL means the legacy default stream) and the call returns without synchronising.  Weight tensors may be
 * views into a larger byte buffer (256-byte aligned rows are enough).
 *
 * Return value: H3B_OK (0) or a positive H3B_ERR_* code; h3b_last_error() then returns a message (thread-local, valid
 * until the next call on the same thread).  H3B_ERR_ARG means the arguments are invalid (the Python layer raises
 * ValueError); every other code is a device or build failure (RuntimeError).
 *
 * Numerics (all entry points): identical to the reference's "ck" profile of h3turbo/h3/qlinear.py.  The int4->int8 decode,
 * the int32 accumulation and every epilogue rounding are bit-exact; the only float step that is not the reference's
 * correctly rounded fp64 computation is the ConvRot rotation, done as an fp32 fast Walsh-Hadamard transform.
 *
 * Reference interfaces named below are file:line in the reference project (Alexpoopy1/MiniMax-H3-Turbo).
 */
#ifndef H3B_H
#define H3B_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define H3B_ABI_VERSION 1

enum h3b_status {
  H3B_OK = 0,
  H3B_ERR_ARG = 1,          /* invalid argument (shape, dtype, size, alignment) */
  H3B_ERR_CUDA = 2,         /* a CUDA runtime call failed */
  H3B_ERR_UNSUPPORTED = 3,  /* valid for the reference, not supported by this build (e.g. convrot 1024) */
  H3B_ERR_DEVICE = 4        /* a kernel reported a failure (a bounded wait timed out); see h3b_device_error */
};

enum h3b_dtype {
  H3B_BF16 = 0,
  H3B_FP16 = 1,
  H3B_FP32 = 2,
  H3B_FP8_E4M3 = 3, /* float8_e4m3fn group scales (raw bytes) */
  H3B_INT32 = 4     /* int32 accumulator output (parity dump) */
};

enum h3b_quant_mode {
  H3B_QMODE_CK = 0,    /* absmax of the unrounded rotation; epilogue (acc * xs) * s_ch   (qlinear.py:278-283, :400-401) */
  H3B_QMODE_EAGER = 1  /* absmax of the dtype-rounded rotation; epilogue acc * (xs * s_ch) (qlinear.py:284-287, :402-403) */
};

/* ABI version (H3B_ABI_VERSION) and the last error message of this thread. */
int h3b_version(void);
const char* h3b_last_error(void);

/* Rotate + per-token int8 quantisation of activations (kernel KA).
 * Replaces quantize_activation / _quantize_rows (qlinear.py:267-303), the activation half of comfy_kitchen's fused
 * w4a8_int8_linear reached through _run_ck (qlinear.py:427-429).
 *   x      [M, ldx] of x_dtype (bf16/fp16/fp32); the row holds K features, or [gate | up] (2K) when swiglu != 0
 *          (input_act="swiglu", qlinear.py:376-379: silu(gate) * up in x_dtype, applied before the rotation).
 *   convrot 4, 16, 64 or 256 (the ConvRot block; K % convrot == 0).
 *   q      [M, ldq] int8 codes out; xs [M] fp32 per-row scales out. */
int h3b_rotq(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx, int convrot, int swiglu, int quant_mode,
             int8_t* q, int64_t ldq, float* xs, void* stream);

/* Block rotation only: y = per-convrot-block x @ H in y_dtype (one rounding of the fp32 transform).
 * Replaces rotate (qlinear.py:118-132). */
int h3b_rotate(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx, int convrot, void* y, int y_dtype,
               int64_t ldy, void* stream);

/* Per-head RMSNorm + split-half rotary embedding of q and k, in place (both, or one of them with the other NULL).
 * Replaces comfy_kitchen's rms_rope_split_half_ (called at layout.py:343) with the bit-exact semantics of the
 * reference's "torch" form of that kernel, norm_rope_ (layout.py:329-356) with rms_norm_fused_order (layout.py:309-326).
 *   q, k      [S, heads, head_dim] of x_dtype (bf16 or fp16), heads contiguous, token strides ldq / ldk (elements);
 *             head_dim 32, 64, 128 or 256
 *   wq, wk    [head_dim] of w_dtype;  eps as the fp32 value of the model's qk_norm_eps
 *   cos, sin  [S, half] of t_dtype, rows ldt elements apart; channel j < half pairs with j + half; 2 * half <= head_dim */
int h3b_qk_norm_rope(void* q, int64_t ldq, void* k, int64_t ldk, int x_dtype, int64_t S, int heads, int head_dim,
                     const void* wq, const void* wk, int w_dtype, float eps, const void* cos_t, const void* sin_t,
                     int64_t ldt, int t_dtype, int half, void* stream);

/* RMSNorm + AdaLN modulation of the residual stream: h = scale_shift(rms(x)).  Replaces _rms followed by _scale_shift_
 * (model.py:64-66, 106-109): n = dt((x * rsqrt(mean(x^2) + eps)) * w), then for a token with modulation row `row`
 * h = dt(dt(n * dt(1 + dt(scale[row]))) + dt(shift[row])); tokens without a row keep n.  The row sum's order is this
 * kernel's own (torch's F.rms_norm reduces in another order: rare one-ulp differences of n).
 *   x, h          [M, hidden] of x_dtype (bf16 or fp16), rows ldx / ldh elements apart; hidden a multiple of 8
 *   w             [hidden] of w_dtype;  shift, scale: [n_rows, hidden] of m_dtype, rows ldm elements apart
 *   segments      HOST table of n_segments <= H3B_MAX_SEGMENTS x (first token, end token, row), int32
 *   token_rows    optional DEVICE int32 [M] row per token (negative: none, else < n_rows, which the caller guarantees);
 *                 used instead of the segments when given
 *   every device pointer 16-byte aligned */
#define H3B_MAX_SEGMENTS 16
int h3b_rms_modulate(const void* x, int x_dtype, int64_t ldx, int64_t M, int hidden, const void* w, int w_dtype,
                     float eps, const void* shift, const void* scale, int64_t ldm, int64_t n_rows, int m_dtype,
                     const int32_t* segments, int n_segments, const int32_t* token_rows, void* h, int64_t ldh,
                     void* stream);

/* RMSNorm + AdaLN modulation fused into the rotate+quantise kernel: the codes and scales of h = _scale_shift_(_rms(x))
 * (model.py:64-66, 106-109, 239-241) without writing h; the activation side of the qkv and fc1 linears of a block.
 * Bit-identical to h3b_rms_modulate (bf16) followed by h3b_rotq on its output.  Every tensor bf16:
 *   x          [M, K], rows ldx elements apart; K a multiple of 256, at most 6144; convrot 256
 *   w          [K] norm weight (the reference rounds it to x's dtype first)
 *   shift      [n_rows, K] dt(shift);  scale1: [n_rows, K] dt(1 + dt(scale)), the factor _scale_shift_ multiplies by;
 *              rows ldm elements apart
 *   segments / token_rows as h3b_rms_modulate;  q [M, ldq] int8 codes, xs [M] fp32 scales as h3b_rotq
 *   every device pointer 16-byte aligned */
int h3b_rotq_rms_modulate(const void* x, int64_t M, int64_t K, int64_t ldx, const void* w, float eps, const void* shift,
                          const void* scale1, int64_t ldm, int64_t n_rows, const int32_t* segments, int n_segments,
                          const int32_t* token_rows, int convrot, int quant_mode, int8_t* q, int64_t ldq, float* xs,
                          void* stream);

/* Gated residual update, in place: x = dt(x + other * dt(gate[row])) for tokens with a modulation row, others
 * unchanged.  Replaces _gate_ (model.py:111-115; torch's addcmul_, bit-identical).  Arguments as h3b_rms_modulate;
 * other: [M, hidden] of x_dtype, rows ldo elements apart. */
int h3b_gate_residual(void* x, int x_dtype, int64_t ldx, const void* other, int64_t ldo, int64_t M, int hidden,
                      const void* gate, int64_t ldm, int64_t n_rows, int m_dtype, const int32_t* segments, int n_segments,
                      const int32_t* token_rows, void* stream);

/* Merge softmax attention computed over disjoint key sets (no reference counterpart: the ring key/value exchange of
 * the token-sharded DiT block, whose single-GPU form is one attention call, model.py:196-228).  For every head h and
 * query q: L' = log(exp(L) + exp(l)), A = A exp(L - L') + fp32(o) exp(l - L'), L = L'.
 *   acc    fp32 [heads, queries, head_dim] running output;  acc_lse fp32 [heads, queries] running log-sum-exp
 *   o      attention output over the next key set, element (h, q, d) at o + h*o_head_stride + q*o_query_stride + d;
 *          o_dtype must be H3B_BF16 (anything else is refused with H3B_ERR_ARG)
 *   lse    fp32 [heads, queries] its log-sum-exp (natural log);  first != 0: (acc, acc_lse) = (o, lse)
 *          a query with no keys on either side (both log-sum-exps -inf) gets a zero output
 *   out    optional bf16 [queries, heads * head_dim] (row stride ldo): the merged result, written instead of acc */
int h3b_attn_merge(float* acc, float* acc_lse, const void* o, int64_t o_head_stride, int64_t o_query_stride, int o_dtype,
                   const float* lse, int64_t heads, int64_t queries, int head_dim, int first, void* out, int64_t ldo,
                   void* stream);

/* int4 codebook indices + group scales -> the exact int8 grid [N, K] (row stride ldg bytes).
 * Replaces decode_int8_grid / _decode_rows / _pair_lut (qlinear.py:157-204).
 *   q4     [N, ldq4 bytes] packed nibbles, low nibble first (types.py:14-16)
 *   s_rel  [N, lds elements] of s_dtype (fp8 e4m3 bytes, fp16, bf16 or fp32), K / group per row
 *   codebook fp32 [16]; group >= 4 dividing 16 or a multiple of 16 (qlinear.py:146). */
int h3b_decode_grid(const void* q4, int64_t N, int64_t K, int64_t ldq4, const void* s_rel, int s_dtype, int64_t lds,
                    const float* codebook, int group, int8_t* grid, int64_t ldg, void* stream);

/* Exact int32 a[M, K] @ b[N, K]^T for int8 operands on the tcgen05 tensor cores (parity of the integer accumulator).
 * Replaces _int8_mm (qlinear.py:236-254).  lda/ldb in bytes (multiples of 16), ldc in elements. */
int h3b_int8_gemm_s32(const int8_t* a, int64_t lda, int64_t M, const int8_t* b, int64_t ldb, int64_t N, int64_t K,
                      int32_t* c, int64_t ldc, void* stream);

/* Scratch bytes h3b_w4a8_gemm / h3b_w4a8_linear need for these sizes (0 is a valid answer). */
size_t h3b_gemm_workspace_bytes(int64_t M, int64_t N, int64_t K);
size_t h3b_linear_workspace_bytes(int64_t M, int64_t N, int64_t K);

/* W4A8 GEMM + epilogue on already-quantised activation codes (kernel KB).
 * Replaces the int8 GEMM and epilogue of _TorchRunner._a8 (qlinear.py:396-405):
 *   out = out_dtype( (fp32(acc) * xs[m]) * s_ch[n] )            quant_mode CK
 *   out = out_dtype(  fp32(acc) * (xs[m] * s_ch[n]) )           quant_mode EAGER
 *   out = out_dtype( fp32(out) + fp32(bias[n]) )                 when bias != NULL (bias already of out_dtype)
 * out_dtype H3B_INT32 stores the raw accumulator instead (xs, s_ch, bias ignored).
 *   qa [M, lda bytes] int8 codes, xs [M] fp32; weight as in h3b_decode_grid; out [M, ldo elements]. */
int h3b_w4a8_gemm(const int8_t* qa, int64_t lda, const float* xs, int64_t M, const void* q4, int64_t ldq4,
                  const void* s_rel, int s_dtype, int64_t lds, const float* s_ch, const float* codebook, int group,
                  const void* bias, void* out, int out_dtype, int64_t ldo, int64_t N, int64_t K, int quant_mode,
                  void* workspace, size_t ws_bytes, void* stream);

/* GEMM + epilogue on an already-decoded int8 weight grid [N, ldg bytes] (same epilogue contract as h3b_w4a8_gemm).
 * For callers that keep decoded grids resident (weights that never stream); no workspace.  Same reference lines as
 * h3b_w4a8_gemm (qlinear.py:396-405) with the decode (qlinear.py:194-204) hoisted out. */
/* 1 when h3b_w4a8_gemm (and so h3b_w4a8_linear) decodes the int4 weight inside the GEMM's producer warps for this
 * problem (few M tiles; fp8 e4m3 scales with group 16 or fp16/bf16/fp32 scales with group 128; 16-byte aligned packed
 * rows), 0 when it runs a separate decode pass into the workspace first.  No reference counterpart (introspection). */
int h3b_w4a8_gemm_decodes_in_kernel(int64_t M, int64_t N, int64_t K, const void* q4, int64_t ldq4, int s_dtype,
                                    int group);

int h3b_int8_gemm_epilogue(const int8_t* qa, int64_t lda, const float* xs, int64_t M, const int8_t* grid, int64_t ldg,
                           const float* s_ch, const void* bias, void* out, int out_dtype, int64_t ldo, int64_t N,
                           int64_t K, int quant_mode, void* stream);

/* The whole W4A8 linear: (swiglu) -> rotate+quantise -> GEMM -> epilogue.  The seam the reference hands to
 * comfy_kitchen: _run_ck -> w4a8_int8_linear(x2, w.q, s_rel, w.s_ch, codebook, bias, group_size, convrot_groupsize,
 * out_dtype) (qlinear.py:427-429, result contract :446-451).  workspace >= h3b_linear_workspace_bytes(M, N, K). */
int h3b_w4a8_linear(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx, int swiglu, const void* q4,
                    int64_t ldq4, const void* s_rel, int s_dtype, int64_t lds, const float* s_ch, const float* codebook,
                    int group, int convrot, const void* bias, void* out, int out_dtype, int64_t ldo, int64_t N,
                    int quant_mode, void* workspace, size_t ws_bytes, void* stream);

/* Allocation-free W4A8 GEMM + epilogue: h3b_w4a8_gemm without the workspace argument.  No counterpart in the
 * reference.  For callers that cannot allocate device memory: code running inside a host framework or plugin that
 * gives it no device allocator, a C/FFI caller with no CUDA memory pool of its own, or a latency-critical loop that must
 * not call cudaMalloc (it can synchronise the whole device).  The decoded weight rows live in one file-scope device
 * array of H3B_NOALLOC_SCRATCH_BYTES that every GPU using the library holds until the process exits; the weight is
 * decoded and multiplied in slabs of rows that fit in it, so any N works, and K may be at most
 * H3B_NOALLOC_SCRATCH_BYTES / 32 (larger K is rejected with H3B_ERR_ARG).  Every call looks up the array's device
 * address in the current device's context (cudaGetSymbolAddress; the first call on a device loads the module there, so
 * make that first call before any stream capture).  All calls share the one
 * array: calls that may overlap on the GPU (different streams, or different host threads) race on it and must be
 * serialised by the caller.  Nothing in it needs to start at zero (each slab is fully rewritten before it is read). */
#define H3B_NOALLOC_SCRATCH_BYTES (16u << 20)
int h3b_w4a8_gemm_noalloc(const int8_t* qa, int64_t lda, const float* xs, int64_t M, const void* q4, int64_t ldq4,
                          const void* s_rel, int s_dtype, int64_t lds, const float* s_ch, const float* codebook, int group,
                          const void* bias, void* out, int out_dtype, int64_t ldo, int64_t N, int64_t K, int quant_mode,
                          void* stream);

/* ---- block streamer: the copy path of StreamingProvider (stream.py:115-623; copies and slot events :333-362,
 * acquire/release ordering :376-437).  An engine owns a copy stream, per-slot `ready`/`done` events and page-locked host
 * staging buffers; the caller owns the device slots.  Slot s's copy waits on the device for done[s] (recorded by
 * release on the compute stream), and acquire makes the compute stream wait for ready[s].  Host waits are bounded. */
typedef struct h3b_streamer h3b_streamer;
enum h3b_copy_mode {
  H3B_COPY_DIRECT = 0,   /* source is page-locked (registered or pinned): one async copy */
  H3B_COPY_STAGED = 1,   /* pageable source: multi-threaded memcpy into a staging buffer, then an async copy */
  H3B_COPY_PAGEABLE = 2  /* pageable source copied by the driver (returns once the source has been read) */
};
int h3b_streamer_create(int device, int n_slots, int n_staging, size_t staging_bytes, int memcpy_threads,
                        h3b_streamer** out);
int h3b_streamer_destroy(h3b_streamer* s);
int h3b_streamer_copy(h3b_streamer* s, int slot, void* dst, const void* src_host, size_t bytes, int mode);
/* A caller-driven copy (a custom transfer) on the engine's copy stream: begin (the stream waits for done[slot]),
 * enqueue the copy on h3b_streamer_stream(s), end (ready[slot] recorded). */
int h3b_streamer_begin(h3b_streamer* s, int slot);
int h3b_streamer_end(h3b_streamer* s, int slot, size_t bytes);
void* h3b_streamer_stream(h3b_streamer* s);
int h3b_streamer_acquire(h3b_streamer* s, int slot, void* stream);
int h3b_streamer_release(h3b_streamer* s, int slot, void* stream);
int h3b_streamer_wait(h3b_streamer* s, int slot, double timeout_s);
int h3b_streamer_stats(h3b_streamer* s, uint64_t* copies, uint64_t* bytes, double* busy_s);
/* Page-lock / unlock a host range in place (read_only != 0 for a read-only file mapping: cudaHostRegisterReadOnly).
 * Replaces the reference's torch.cuda.cudart().cudaHostRegister calls (stream.py:208-217, :232-238). */
int h3b_host_register(void* ptr, size_t bytes, int read_only);
int h3b_host_unregister(void* ptr);

/* Self-test of the bounded-wait failure path (no reference counterpart): one thread waits on an mbarrier that nothing
 * arrives on, gives up after limit_s (0 < limit_s <= 10) of GPU time, raises bit 0 of the device flag and writes 1 to
 * *gave_up_device (device memory).  The context stays usable; read and clear the flag with h3b_device_error(1). */
int h3b_selftest_wait_timeout(double limit_s, int* gave_up_device, void* stream);

/* Device-side failure flag of the current device: a kernel whose bounded wait ran out sets it (and returns instead of
 * hanging).  Returns the flag and, when clear != 0, resets it.  Synchronises the device. */
int h3b_device_error(int clear);

#ifdef __cplusplus
}
#endif

#endif /* H3B_H */
