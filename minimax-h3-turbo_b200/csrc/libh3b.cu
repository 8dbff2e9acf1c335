// libh3b.so: the C ABI declared in include/h3b.h, argument validation and error state, the block streamer and the
// wait self-test.  The kernels live in the k_*.cu translation units (launch.h lists what each exports).
#include <cstdio>
#include <mutex>
#include <string>

#include "h3b_common.cuh"

namespace h3b {

static thread_local std::string g_err;

void set_error(const std::string& msg) { g_err = msg; }
int fail(int code, const std::string& msg) {
  g_err = msg;
  return code;
}
int cuda_fail(cudaError_t e, const char* what) {
  g_err = std::string(what) + ": " + cudaGetErrorString(e);
  return H3B_ERR_CUDA;
}
int check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, what);
  return H3B_OK;
}

}  // namespace h3b

#include "launch.h"
#include "streamer.cuh"

namespace h3b {

static bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }
static size_t act_size(int dt) { return dt == H3B_FP32 ? 4 : 2; }
static bool is_act(int dt) { return dt == H3B_BF16 || dt == H3B_FP16 || dt == H3B_FP32; }
static bool is_scale(int dt) { return dt == H3B_FP8_E4M3 || is_act(dt); }
static size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// qlinear.py:146 -- K divisible by 16, group and convrot; group >= 4 dividing 16 or a multiple of 16.
static int check_weight_geometry(int64_t K, int group) {
  if (group < 4 || K % 16 || K % group || ((16 % group) && (group % 16)))
    return fail(H3B_ERR_ARG, "K=" + std::to_string(K) + " must be divisible by 16 and group_size=" + std::to_string(group) +
                                 "; group_size >= 4 dividing 16 or a multiple of 16");
  return H3B_OK;
}

static int check_rotq_args(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx, int convrot, int swiglu) {
  if (!is_act(x_dtype)) return fail(H3B_ERR_ARG, "activation dtype must be bf16, fp16 or fp32");
  if (M < 0 || K <= 0) return fail(H3B_ERR_ARG, "M must be >= 0 and K > 0");
  if (convrot != 4 && convrot != 16 && convrot != 64 && convrot != 256) {
    int n = convrot;
    while (n > 1 && n % 4 == 0) n /= 4;
    if (convrot < 4 || n != 1)
      return fail(H3B_ERR_ARG, "regular Hadamard size must be a power of 4 (>= 4), got " + std::to_string(convrot));
    return fail(H3B_ERR_UNSUPPORTED, "convrot " + std::to_string(convrot) + " is not supported by the b200 backend (4, 16, 64, 256)");
  }
  if (K % convrot) return fail(H3B_ERR_ARG, "last dim " + std::to_string(K) + " is not a multiple of the rotation block " + std::to_string(convrot));
  if (K % 16) return fail(H3B_ERR_ARG, "K must be a multiple of 16");
  if (K / 16 > 1024) return fail(H3B_ERR_UNSUPPORTED, "K > 16384 is not supported by the rotate+quantise kernel");
  if (M > 0x7FFFFFFF) return fail(H3B_ERR_UNSUPPORTED, "M >= 2^31 rows");
  const int64_t row_elems = swiglu ? 2 * K : K;
  if (ldx < row_elems) return fail(H3B_ERR_ARG, "ldx is smaller than the row width");
  if (!aligned(x, 16) || (ldx * static_cast<int64_t>(act_size(x_dtype))) % 16)
    return fail(H3B_ERR_ARG, "x must be 16-byte aligned with a row stride that is a multiple of 16 bytes");
  return H3B_OK;
}

static int check_weight_args(const void* q4, int64_t N, int64_t K, int64_t ldq4, const void* s_rel, int s_dtype,
                             int64_t lds, const float* codebook, int group) {
  if (N < 0) return fail(H3B_ERR_ARG, "N must be >= 0");
  int rc = check_weight_geometry(K, group);
  if (rc) return rc;
  if (!is_scale(s_dtype)) return fail(H3B_ERR_ARG, "group scale dtype must be fp8_e4m3, fp16, bf16 or fp32");
  if (ldq4 < K / 2 || ldq4 % 8 || !aligned(q4, 8)) return fail(H3B_ERR_ARG, "q must be 8-byte aligned with a row stride >= K/2 and a multiple of 8 bytes");
  if (lds < K / group) return fail(H3B_ERR_ARG, "s_rel row stride is smaller than K / group_size");
  if (!s_rel || !codebook) return fail(H3B_ERR_ARG, "s_rel and codebook must be given");
  return H3B_OK;
}

}  // namespace h3b

// ------------------------------------------------------------------------------------------------ allocation-free GEMM
// h3b_w4a8_gemm_noalloc: the same decode + GEMM + epilogue as h3b_w4a8_gemm, for callers that cannot allocate device
// memory (see include/h3b.h).  Its scratch -- the decoded int8 weight rows -- is this file-scope device array.  In host
// code `g_noalloc_grid` names a host-side stand-in, not device memory, so its device address is looked up with
// cudaGetSymbolAddress (with the caller's device current) and only that address is handed to the kernels.
static __device__ __align__(256) int8_t g_noalloc_grid[H3B_NOALLOC_SCRATCH_BYTES];

namespace h3b {
// The array's device address in the current device's current context.  Looked up on every call (cheap once the module
// is loaded) rather than cached, so a device reset or a different context on the same ordinal never sees a stale address.
static int noalloc_scratch(void** addr) {
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_grid);
  if (e != cudaSuccess || !p) return cuda_fail(e, "cudaGetSymbolAddress(allocation-free scratch)");
  *addr = p;
  return H3B_OK;
}
// The failure path of the bounded waits, exercised on purpose: one thread waits on an mbarrier that nothing arrives on;
// after `limit_ns` of %globaltimer time it gives up, raises bit 0 of the device flag and returns (no trap, no fault).
__global__ void wait_timeout_selftest_kernel(unsigned long long limit_ns, int* gave_up) {
  __shared__ uint64_t bar;
  mbar_init(&bar, 1);
  mbar_fence_init();
  const unsigned long long t0 = globaltimer_ns();
  bool done = false;
  for (uint32_t i = 0; !done; ++i) {
    if (mbar_try_wait(&bar, 0)) break;
    if ((i & 63) == 0 && globaltimer_ns() - t0 > limit_ns) {
      atomicOr(&g_device_error, 1u);
      *gave_up = 1;
      done = true;
    }
  }
}
static H3B_DEVICE_ERROR_ACCESSOR(device_error_abi)
}  // namespace h3b

using namespace h3b;

extern "C" {

int h3b_selftest_wait_timeout(double limit_s, int* gave_up_device, void* stream) {
  if (!(limit_s > 0.0 && limit_s <= 10.0) || !gave_up_device) return fail(H3B_ERR_ARG, "selftest: limit must be in (0, 10] s");
  wait_timeout_selftest_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<unsigned long long>(limit_s * 1e9), gave_up_device);
  return check_launch("wait_timeout_selftest_kernel");
}

int h3b_version(void) { return H3B_ABI_VERSION; }

const char* h3b_last_error(void) { return g_err.c_str(); }

int h3b_rotq(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx, int convrot, int swiglu, int quant_mode,
             int8_t* q, int64_t ldq, float* xs, void* stream) {
  int rc = check_rotq_args(x, x_dtype, M, K, ldx, convrot, swiglu);
  if (rc) return rc;
  if (quant_mode != H3B_QMODE_CK && quant_mode != H3B_QMODE_EAGER) return fail(H3B_ERR_ARG, "quant_mode must be 'ck' or 'eager'");
  if (ldq < K || ldq % 16 || !aligned(q, 16)) return fail(H3B_ERR_ARG, "q must be 16-byte aligned with a row stride >= K, multiple of 16");
  if (M == 0) return H3B_OK;
  return rotq_launch(x, x_dtype, M, K, ldx, convrot, swiglu, quant_mode, q, ldq, xs, nullptr, 0, 0,
                     static_cast<cudaStream_t>(stream));
}

int h3b_rotate(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx, int convrot, void* y, int y_dtype,
               int64_t ldy, void* stream) {
  int rc = check_rotq_args(x, x_dtype, M, K, ldx, convrot, 0);
  if (rc) return rc;
  if (!is_act(y_dtype)) return fail(H3B_ERR_ARG, "output dtype must be bf16, fp16 or fp32");
  if (ldy < K) return fail(H3B_ERR_ARG, "ldy is smaller than K");
  if (M == 0) return H3B_OK;
  return rotq_launch(x, x_dtype, M, K, ldx, convrot, 0, MODE_ROTATE, nullptr, 0, nullptr, y, y_dtype, ldy,
                     static_cast<cudaStream_t>(stream));
}

int h3b_qk_norm_rope(void* q, int64_t ldq, void* k, int64_t ldk, int x_dtype, int64_t S, int heads, int head_dim,
                     const void* wq, const void* wk, int w_dtype, float eps, const void* cos_t, const void* sin_t,
                     int64_t ldt, int t_dtype, int half, void* stream) {
  if (S == 0) return H3B_OK;  // empty sequence (torch hands out null pointers for empty tensors)
  if (!q && !k) return fail(H3B_ERR_ARG, "qk_norm_rope: q and k are both null");
  if ((q && !wq) || (k && !wk)) return fail(H3B_ERR_ARG, "qk_norm_rope: a norm weight is missing");
  if (S < 0 || heads < 1 || head_dim < 1) return fail(H3B_ERR_ARG, "qk_norm_rope: bad shape");
  if ((q && ldq < static_cast<int64_t>(heads) * head_dim) || (k && ldk < static_cast<int64_t>(heads) * head_dim))
    return fail(H3B_ERR_ARG, "qk_norm_rope: token stride is smaller than heads * head_dim");
  if (!is_act(w_dtype) || !is_act(t_dtype)) return fail(H3B_ERR_ARG, "qk_norm_rope: weight/table dtype must be bf16, fp16 or fp32");
  if (half < 0 || 2 * half > head_dim) return fail(H3B_ERR_ARG, "qk_norm_rope: 2 * half exceeds head_dim");
  if (half > 0 && (!cos_t || !sin_t || ldt < half)) return fail(H3B_ERR_ARG, "qk_norm_rope: cos/sin tables missing or too narrow");
  return qk_norm_rope_launch(q, ldq, k, ldk, x_dtype, S, heads, head_dim, wq, wk, w_dtype, eps, cos_t, sin_t, ldt, t_dtype,
                             half, static_cast<cudaStream_t>(stream));
}

int h3b_rms_modulate(const void* x, int x_dtype, int64_t ldx, int64_t M, int hidden, const void* w, int w_dtype,
                     float eps, const void* shift, const void* scale, int64_t ldm, int64_t n_rows, int m_dtype,
                     const int32_t* segments, int n_segments, const int32_t* token_rows, void* h, int64_t ldh,
                     void* stream) {
  if (M < 0 || hidden < 8 || hidden % 8) return fail(H3B_ERR_ARG, "rms_modulate: hidden must be a positive multiple of 8");
  if (M == 0) return H3B_OK;
  if (!x || !w || !h) return fail(H3B_ERR_ARG, "rms_modulate: null x, weight or output");
  if (ldx < hidden || ldh < hidden || ldx % 8 || ldh % 8 || !aligned(x, 16) || !aligned(h, 16) || !aligned(w, 16))
    return fail(H3B_ERR_ARG, "rms_modulate: x / h / weight must be 16-byte aligned with row strides >= hidden, multiples of 8");
  if (n_segments < 0 || n_segments > H3B_MAX_SEGMENTS || (n_segments > 0 && !segments))
    return fail(H3B_ERR_ARG, "rms_modulate: at most H3B_MAX_SEGMENTS segments, given as a host table");
  const bool mod = n_segments > 0 || token_rows;
  if (!is_act(w_dtype) || (mod && !is_act(m_dtype))) return fail(H3B_ERR_ARG, "rms_modulate: bad weight / modulation dtype");
  if (mod && (!shift || !scale || ldm < hidden || ldm % 8 || !aligned(shift, 16) || !aligned(scale, 16)))
    return fail(H3B_ERR_ARG, "rms_modulate: shift/scale must be 16-byte aligned rows of >= hidden, stride a multiple of 8");
  for (int i = 0; i < n_segments; ++i)
    if (segments[3 * i] < 0 || segments[3 * i + 1] < segments[3 * i] || segments[3 * i + 2] < 0 ||
        segments[3 * i + 2] >= n_rows)
      return fail(H3B_ERR_ARG, "rms_modulate: a segment has a negative bound, ends before it starts, or names a row >= n_rows");
  return rms_modulate_launch(x, x_dtype, ldx, M, hidden, w, w_dtype, eps, shift, scale, ldm, m_dtype, segments, n_segments,
                             token_rows, h, ldh, static_cast<cudaStream_t>(stream));
}

int h3b_rotq_rms_modulate(const void* x, int64_t M, int64_t K, int64_t ldx, const void* w, float eps, const void* shift,
                          const void* scale1, int64_t ldm, int64_t n_rows, const int32_t* segments, int n_segments,
                          const int32_t* token_rows, int convrot, int quant_mode, int8_t* q, int64_t ldq, float* xs,
                          void* stream) {
  if (M < 0 || K <= 0 || !rotq_rmsmod_supported(K))
    return fail(H3B_ERR_ARG, "rotq_rms_modulate: K must be a positive multiple of 256, at most 6144");
  if (convrot != 256) return fail(H3B_ERR_UNSUPPORTED, "rotq_rms_modulate: convrot must be 256");
  if (quant_mode != H3B_QMODE_CK && quant_mode != H3B_QMODE_EAGER) return fail(H3B_ERR_ARG, "quant_mode must be 'ck' or 'eager'");
  if (M == 0) return H3B_OK;
  if (!x || !w || !q || !xs) return fail(H3B_ERR_ARG, "rotq_rms_modulate: null x, weight, codes or scales");
  if (ldx < K || ldx % 8 || !aligned(x, 16) || !aligned(w, 16))
    return fail(H3B_ERR_ARG, "rotq_rms_modulate: x / weight must be 16-byte aligned, x rows >= K elements apart, a multiple of 8");
  if (ldq < K || ldq % 16 || !aligned(q, 16)) return fail(H3B_ERR_ARG, "q must be 16-byte aligned with a row stride >= K, multiple of 16");
  if (n_segments < 0 || n_segments > H3B_MAX_SEGMENTS || (n_segments > 0 && !segments))
    return fail(H3B_ERR_ARG, "rotq_rms_modulate: at most H3B_MAX_SEGMENTS segments, given as a host table");
  const bool mod = n_segments > 0 || token_rows;
  if (mod && (!shift || !scale1 || ldm < K || ldm % 8 || !aligned(shift, 16) || !aligned(scale1, 16)))
    return fail(H3B_ERR_ARG, "rotq_rms_modulate: shift/scale1 must be 16-byte aligned rows of >= K, stride a multiple of 8");
  RowNorm nrm{};
  nrm.w = static_cast<const __nv_bfloat16*>(w);
  nrm.shift = static_cast<const __nv_bfloat16*>(shift);
  nrm.scale1 = static_cast<const __nv_bfloat16*>(scale1);
  nrm.ldm = ldm;
  nrm.eps = eps;
  nrm.token_rows = token_rows;
  nrm.segs.n = n_segments;
  for (int i = 0; i < n_segments; ++i) {
    if (segments[3 * i] < 0 || segments[3 * i + 1] < segments[3 * i] || segments[3 * i + 2] < 0 ||
        segments[3 * i + 2] >= n_rows)
      return fail(H3B_ERR_ARG, "rotq_rms_modulate: a segment has a negative bound, ends before it starts, or names a row >= n_rows");
    nrm.segs.first[i] = segments[3 * i];
    nrm.segs.end[i] = segments[3 * i + 1];
    nrm.segs.row[i] = segments[3 * i + 2];
  }
  return rotq_rmsmod_launch(x, ldx, M, K, nrm, quant_mode, q, ldq, xs, static_cast<cudaStream_t>(stream));
}

int h3b_gate_residual(void* x, int x_dtype, int64_t ldx, const void* other, int64_t ldo, int64_t M, int hidden,
                      const void* gate, int64_t ldm, int64_t n_rows, int m_dtype, const int32_t* segments, int n_segments,
                      const int32_t* token_rows, void* stream) {
  if (M < 0 || hidden < 8 || hidden % 8) return fail(H3B_ERR_ARG, "gate_residual: hidden must be a positive multiple of 8");
  if (M == 0 || (n_segments == 0 && !token_rows)) return H3B_OK;
  if (!x || !other || !gate) return fail(H3B_ERR_ARG, "gate_residual: null x, other or gate");
  if (ldx < hidden || ldo < hidden || ldm < hidden || ldx % 8 || ldo % 8 || ldm % 8 || !aligned(x, 16) ||
      !aligned(other, 16) || !aligned(gate, 16))
    return fail(H3B_ERR_ARG, "gate_residual: 16-byte aligned rows with strides >= hidden, multiples of 8, are required");
  if (!is_act(m_dtype)) return fail(H3B_ERR_ARG, "gate_residual: bad gate dtype");
  if (n_segments < 0 || n_segments > H3B_MAX_SEGMENTS || (n_segments > 0 && !segments))
    return fail(H3B_ERR_ARG, "gate_residual: at most H3B_MAX_SEGMENTS segments, given as a host table");
  for (int i = 0; i < n_segments; ++i)
    if (segments[3 * i] < 0 || segments[3 * i + 1] < segments[3 * i] || segments[3 * i + 2] < 0 ||
        segments[3 * i + 2] >= n_rows)
      return fail(H3B_ERR_ARG, "gate_residual: a segment has a negative bound, ends before it starts, or names a row >= n_rows");
  return gate_residual_launch(x, x_dtype, ldx, other, ldo, M, hidden, gate, ldm, m_dtype, segments, n_segments, token_rows,
                              static_cast<cudaStream_t>(stream));
}

int h3b_attn_merge(float* acc, float* acc_lse, const void* o, int64_t o_head_stride, int64_t o_query_stride, int o_dtype,
                   const float* lse, int64_t heads, int64_t queries, int head_dim, int first, void* out, int64_t ldo,
                   void* stream) {
  if (o_dtype != H3B_BF16) return fail(H3B_ERR_ARG, "attn_merge: the attention output (and the merged output) must be bf16");
  if (heads < 0 || queries < 0) return fail(H3B_ERR_ARG, "attn_merge: negative size");
  if (heads == 0 || queries == 0) return H3B_OK;
  if (!acc || !acc_lse || !o || !lse) return fail(H3B_ERR_ARG, "attn_merge: null pointer");
  if (out && ldo < heads * head_dim) return fail(H3B_ERR_ARG, "attn_merge: output row stride below heads * head_dim");
  return attn_merge_launch(acc, acc_lse, o, o_head_stride, o_query_stride, lse, heads, queries, head_dim, first, out, ldo,
                           static_cast<cudaStream_t>(stream));
}

int h3b_decode_grid(const void* q4, int64_t N, int64_t K, int64_t ldq4, const void* s_rel, int s_dtype, int64_t lds,
                    const float* codebook, int group, int8_t* grid, int64_t ldg, void* stream) {
  int rc = check_weight_args(q4, N, K, ldq4, s_rel, s_dtype, lds, codebook, group);
  if (rc) return rc;
  if (ldg < K || ldg % 16 || !aligned(grid, 16)) return fail(H3B_ERR_ARG, "grid must be 16-byte aligned with a row stride >= K, multiple of 16");
  return decode_launch(q4, N, K, ldq4, s_rel, s_dtype, lds, codebook, group, grid, ldg, static_cast<cudaStream_t>(stream));
}

int h3b_int8_gemm_s32(const int8_t* a, int64_t lda, int64_t M, const int8_t* b, int64_t ldb, int64_t N, int64_t K,
                      int32_t* c, int64_t ldc, void* stream) {
  if (M < 0 || N < 0 || K <= 0 || K % 16) return fail(H3B_ERR_ARG, "need M, N >= 0 and K a positive multiple of 16");
  if (lda < K || ldb < K || lda % 16 || ldb % 16 || !aligned(a, 16) || !aligned(b, 16))
    return fail(H3B_ERR_ARG, "a and b must be 16-byte aligned with row strides >= K, multiples of 16 bytes");
  if (ldc < N) return fail(H3B_ERR_ARG, "ldc is smaller than N");
  if (M == 0 || N == 0) return H3B_OK;
  return gemm_launch(a, lda, b, ldb, nullptr, nullptr, nullptr, c, H3B_INT32, ldc, M, N, K, H3B_QMODE_CK,
                     static_cast<cudaStream_t>(stream));
}

size_t h3b_gemm_workspace_bytes(int64_t M, int64_t N, int64_t K) {
  (void)M;
  return round_up(static_cast<size_t>(N) * static_cast<size_t>(K), 256);  // the decoded int8 grid (separate decode pass)
}

size_t h3b_linear_workspace_bytes(int64_t M, int64_t N, int64_t K) {
  return round_up(static_cast<size_t>(M) * static_cast<size_t>(K), 256)  // activation codes
         + round_up(static_cast<size_t>(M) * 4, 256)                    // per-row scales
         + h3b_gemm_workspace_bytes(M, N, K);
}

int h3b_w4a8_gemm(const int8_t* qa, int64_t lda, const float* xs, int64_t M, const void* q4, int64_t ldq4,
                  const void* s_rel, int s_dtype, int64_t lds, const float* s_ch, const float* codebook, int group,
                  const void* bias, void* out, int out_dtype, int64_t ldo, int64_t N, int64_t K, int quant_mode,
                  void* workspace, size_t ws_bytes, void* stream) {
  int rc = check_weight_args(q4, N, K, ldq4, s_rel, s_dtype, lds, codebook, group);
  if (rc) return rc;
  if (M < 0) return fail(H3B_ERR_ARG, "M must be >= 0");
  if (out_dtype != H3B_BF16 && out_dtype != H3B_FP16 && out_dtype != H3B_FP32 && out_dtype != H3B_INT32)
    return fail(H3B_ERR_ARG, "out dtype must be bf16, fp16, fp32 or int32");
  if (quant_mode != H3B_QMODE_CK && quant_mode != H3B_QMODE_EAGER) return fail(H3B_ERR_ARG, "quant_mode must be 'ck' or 'eager'");
  if (lda < K || lda % 16 || !aligned(qa, 16)) return fail(H3B_ERR_ARG, "activation codes must be 16-byte aligned with a row stride >= K, multiple of 16");
  if (ldo < N) return fail(H3B_ERR_ARG, "ldo is smaller than N");
  if (out_dtype != H3B_INT32 && (!s_ch || !xs)) return fail(H3B_ERR_ARG, "xs and s_ch must be given");
  if (M == 0 || N == 0) return H3B_OK;
  const size_t need = h3b_gemm_workspace_bytes(M, N, K);
  if (!workspace || ws_bytes < need || !aligned(workspace, 256))
    return fail(H3B_ERR_ARG, "workspace must be 256-byte aligned and hold h3b_gemm_workspace_bytes() = " + std::to_string(need) + " bytes");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (w4_fused_ok(M, N, K, q4, ldq4, s_dtype, group))  // few M tiles: decode inside the GEMM's producer warps
    return gemm_w4_launch(qa, lda, q4, ldq4, s_rel, s_dtype, lds, codebook, xs, s_ch, bias, out, out_dtype, ldo, M, N, K,
                          quant_mode, st);
  int8_t* grid = static_cast<int8_t*>(workspace);
  rc = decode_launch(q4, N, K, ldq4, s_rel, s_dtype, lds, codebook, group, grid, K, st);
  if (rc) return rc;
  return gemm_launch(qa, lda, grid, K, xs, s_ch, bias, out, out_dtype, ldo, M, N, K, quant_mode, st);
}

int h3b_w4a8_gemm_decodes_in_kernel(int64_t M, int64_t N, int64_t K, const void* q4, int64_t ldq4, int s_dtype,
                                    int group) {
  return w4_fused_ok(M, N, K, q4, ldq4, s_dtype, group) ? 1 : 0;
}

int h3b_int8_gemm_epilogue(const int8_t* qa, int64_t lda, const float* xs, int64_t M, const int8_t* grid, int64_t ldg,
                           const float* s_ch, const void* bias, void* out, int out_dtype, int64_t ldo, int64_t N,
                           int64_t K, int quant_mode, void* stream) {
  if (M < 0 || N < 0 || K <= 0 || K % 16) return fail(H3B_ERR_ARG, "need M, N >= 0 and K a positive multiple of 16");
  if (out_dtype != H3B_BF16 && out_dtype != H3B_FP16 && out_dtype != H3B_FP32 && out_dtype != H3B_INT32)
    return fail(H3B_ERR_ARG, "out dtype must be bf16, fp16, fp32 or int32");
  if (quant_mode != H3B_QMODE_CK && quant_mode != H3B_QMODE_EAGER) return fail(H3B_ERR_ARG, "quant_mode must be 'ck' or 'eager'");
  if (lda < K || ldg < K || lda % 16 || ldg % 16 || !aligned(qa, 16) || !aligned(grid, 16))
    return fail(H3B_ERR_ARG, "codes and grid must be 16-byte aligned with row strides >= K, multiples of 16 bytes");
  if (ldo < N) return fail(H3B_ERR_ARG, "ldo is smaller than N");
  if (out_dtype != H3B_INT32 && (!s_ch || !xs)) return fail(H3B_ERR_ARG, "xs and s_ch must be given");
  if (M == 0 || N == 0) return H3B_OK;
  return gemm_launch(qa, lda, grid, ldg, xs, s_ch, bias, out, out_dtype, ldo, M, N, K, quant_mode,
                     static_cast<cudaStream_t>(stream));
}

int h3b_w4a8_linear(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx, int swiglu, const void* q4,
                    int64_t ldq4, const void* s_rel, int s_dtype, int64_t lds, const float* s_ch, const float* codebook,
                    int group, int convrot, const void* bias, void* out, int out_dtype, int64_t ldo, int64_t N,
                    int quant_mode, void* workspace, size_t ws_bytes, void* stream) {
  int rc = check_rotq_args(x, x_dtype, M, K, ldx, convrot, swiglu);
  if (rc) return rc;
  rc = check_weight_args(q4, N, K, ldq4, s_rel, s_dtype, lds, codebook, group);
  if (rc) return rc;
  if (out_dtype != H3B_BF16 && out_dtype != H3B_FP16 && out_dtype != H3B_FP32)
    return fail(H3B_ERR_ARG, "out dtype must be bf16, fp16 or fp32");
  if (quant_mode != H3B_QMODE_CK && quant_mode != H3B_QMODE_EAGER) return fail(H3B_ERR_ARG, "quant_mode must be 'ck' or 'eager'");
  if (ldo < N) return fail(H3B_ERR_ARG, "ldo is smaller than N");
  if (!s_ch) return fail(H3B_ERR_ARG, "s_ch must be given");
  if (M == 0 || N == 0) return H3B_OK;
  const size_t need = h3b_linear_workspace_bytes(M, N, K);
  if (!workspace || ws_bytes < need || !aligned(workspace, 256))
    return fail(H3B_ERR_ARG, "workspace must be 256-byte aligned and hold h3b_linear_workspace_bytes() = " + std::to_string(need) + " bytes");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  int8_t* qa = reinterpret_cast<int8_t*>(ws);
  float* xs = reinterpret_cast<float*>(ws + round_up(static_cast<size_t>(M) * K, 256));
  char* rest = ws + round_up(static_cast<size_t>(M) * K, 256) + round_up(static_cast<size_t>(M) * 4, 256);
  rc = rotq_launch(x, x_dtype, M, K, ldx, convrot, swiglu, quant_mode, qa, K, xs, nullptr, 0, 0, st);
  if (rc) return rc;
  return h3b_w4a8_gemm(qa, K, xs, M, q4, ldq4, s_rel, s_dtype, lds, s_ch, codebook, group, bias, out, out_dtype, ldo, N,
                       K, quant_mode, rest, ws_bytes - static_cast<size_t>(rest - ws), stream);
}

int h3b_w4a8_gemm_noalloc(const int8_t* qa, int64_t lda, const float* xs, int64_t M, const void* q4, int64_t ldq4,
                          const void* s_rel, int s_dtype, int64_t lds, const float* s_ch, const float* codebook, int group,
                          const void* bias, void* out, int out_dtype, int64_t ldo, int64_t N, int64_t K, int quant_mode,
                          void* stream) {
  int rc = check_weight_args(q4, N, K, ldq4, s_rel, s_dtype, lds, codebook, group);
  if (rc) return rc;
  if (M < 0) return fail(H3B_ERR_ARG, "M must be >= 0");
  if (out_dtype != H3B_BF16 && out_dtype != H3B_FP16 && out_dtype != H3B_FP32 && out_dtype != H3B_INT32)
    return fail(H3B_ERR_ARG, "out dtype must be bf16, fp16, fp32 or int32");
  if (quant_mode != H3B_QMODE_CK && quant_mode != H3B_QMODE_EAGER) return fail(H3B_ERR_ARG, "quant_mode must be 'ck' or 'eager'");
  if (lda < K || lda % 16 || !aligned(qa, 16)) return fail(H3B_ERR_ARG, "activation codes must be 16-byte aligned with a row stride >= K, multiple of 16");
  if (ldo < N) return fail(H3B_ERR_ARG, "ldo is smaller than N");
  if (out_dtype != H3B_INT32 && (!s_ch || !xs)) return fail(H3B_ERR_ARG, "xs and s_ch must be given");
  // slabs of `rows` weight rows (a multiple of 32, so every slab's output columns stay 16-byte aligned)
  const int64_t rows = (static_cast<int64_t>(H3B_NOALLOC_SCRATCH_BYTES) / K) / 32 * 32;
  if (rows < 32)
    return fail(H3B_ERR_ARG, "K=" + std::to_string(K) + " exceeds the allocation-free limit: 32 decoded rows of K bytes must fit in the " +
                                 std::to_string(H3B_NOALLOC_SCRATCH_BYTES) + "-byte scratch (K <= " +
                                 std::to_string(H3B_NOALLOC_SCRATCH_BYTES / 32) + ")");
  if (M == 0 || N == 0) return H3B_OK;
  void* scratch = nullptr;
  rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int8_t* grid = static_cast<int8_t*>(scratch);
  const size_t ssz = s_dtype == H3B_FP8_E4M3 ? 1 : (s_dtype == H3B_FP32 ? 4 : 2);
  const size_t osz = (out_dtype == H3B_FP32 || out_dtype == H3B_INT32) ? 4 : 2;
  for (int64_t n0 = 0; n0 < N; n0 += rows) {
    const int64_t nr = N - n0 < rows ? N - n0 : rows;
    rc = decode_launch(static_cast<const uint8_t*>(q4) + n0 * ldq4, nr, K, ldq4,
                       static_cast<const char*>(s_rel) + static_cast<size_t>(n0 * lds) * ssz, s_dtype, lds, codebook,
                       group, grid, K, st);
    if (rc) return rc;
    rc = gemm_launch(qa, lda, grid, K, xs, s_ch ? s_ch + n0 : nullptr,
                     bias ? static_cast<const char*>(bias) + static_cast<size_t>(n0) * osz : nullptr,
                     static_cast<char*>(out) + static_cast<size_t>(n0) * osz, out_dtype, ldo, M, nr, K, quant_mode, st);
    if (rc) return rc;
  }
  return H3B_OK;
}

// ------------------------------------------------------------------------------------------------ block streamer
struct h3b_streamer {
  h3b::StreamEngine* e;
};

int h3b_streamer_create(int device, int n_slots, int n_staging, size_t staging_bytes, int memcpy_threads,
                        h3b_streamer** out) {
  if (!out || n_slots < 0 || n_staging < 0 || (n_staging > 0 && staging_bytes == 0))
    return fail(H3B_ERR_ARG, "streamer: need out, n_slots >= 0, n_staging >= 0 and staging_bytes > 0 with staging");
  *out = nullptr;
  cudaError_t err = cudaSetDevice(device);
  if (err != cudaSuccess) return cuda_fail(err, "cudaSetDevice");
  auto* e = new h3b::StreamEngine();
  e->device = device;
  e->memcpy_threads = memcpy_threads > 0 ? memcpy_threads : 8;
  auto bail = [&](cudaError_t er, const char* what) {
    const int rc = cuda_fail(er, what);
    h3b::engine_free(e);
    return rc;
  };
  if ((err = cudaStreamCreateWithFlags(&e->copy, cudaStreamNonBlocking)) != cudaSuccess) return bail(err, "cudaStreamCreate");
  e->ready.assign(n_slots, nullptr);
  e->done.assign(n_slots, nullptr);
  e->done_set.assign(n_slots, 0);
  for (int i = 0; i < n_slots; ++i) {
    if ((err = cudaEventCreateWithFlags(&e->ready[i], cudaEventDisableTiming)) != cudaSuccess) return bail(err, "cudaEventCreate");
    if ((err = cudaEventCreateWithFlags(&e->done[i], cudaEventDisableTiming)) != cudaSuccess) return bail(err, "cudaEventCreate");
  }
  e->stage_bytes = staging_bytes;
  for (int i = 0; i < n_staging; ++i) {
    void* p = nullptr;
    if ((err = cudaHostAlloc(&p, staging_bytes, cudaHostAllocDefault)) != cudaSuccess) {
      cudaGetLastError();  // a refused page-lock is not sticky; run with fewer staging buffers
      break;
    }
    e->staging.push_back(p);
    cudaEvent_t ev;
    if ((err = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming)) != cudaSuccess) return bail(err, "cudaEventCreate");
    e->stage_ev.push_back(ev);
    e->stage_used.push_back(0);
  }
  *out = new h3b_streamer{e};
  return H3B_OK;
}

int h3b_streamer_destroy(h3b_streamer* s) {
  if (!s) return H3B_OK;
  h3b::engine_free(s->e);
  delete s;
  return H3B_OK;
}

int h3b_streamer_copy(h3b_streamer* s, int slot, void* dst, const void* src, size_t bytes, int mode) {
  if (!s || slot < 0 || slot >= static_cast<int>(s->e->ready.size()) || !dst || !src)
    return fail(H3B_ERR_ARG, "streamer_copy: bad engine, slot or pointer");
  h3b::StreamEngine* e = s->e;
  const double t0 = h3b::now_s();
  cudaError_t err = cudaSetDevice(e->device);
  if (err != cudaSuccess) return cuda_fail(err, "cudaSetDevice");
  if (mode == H3B_COPY_STAGED && (e->staging.empty() || bytes > e->stage_bytes)) mode = H3B_COPY_PAGEABLE;
  if (e->done_set[slot] && (err = cudaStreamWaitEvent(e->copy, e->done[slot], 0)) != cudaSuccess)
    return cuda_fail(err, "cudaStreamWaitEvent(done)");
  if (mode == H3B_COPY_STAGED) {
    int k;
    {
      std::lock_guard<std::mutex> lock(e->mu);
      k = e->stage_next;
      e->stage_next = (k + 1) % static_cast<int>(e->staging.size());
    }
    if (e->stage_used[k]) {  // the previous copy out of this staging buffer must have finished
      const int rc = h3b::event_wait(e->stage_ev[k], 600.0, "streamer staging buffer");
      if (rc) return rc;
    }
    h3b::parallel_memcpy(e->staging[k], src, bytes, e->memcpy_threads);
    if ((err = cudaMemcpyAsync(dst, e->staging[k], bytes, cudaMemcpyHostToDevice, e->copy)) != cudaSuccess)
      return cuda_fail(err, "cudaMemcpyAsync(staged)");
    if ((err = cudaEventRecord(e->stage_ev[k], e->copy)) != cudaSuccess) return cuda_fail(err, "cudaEventRecord");
    e->stage_used[k] = 1;
  } else if ((err = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, e->copy)) != cudaSuccess) {
    return cuda_fail(err, "cudaMemcpyAsync");
  }
  if ((err = cudaEventRecord(e->ready[slot], e->copy)) != cudaSuccess) return cuda_fail(err, "cudaEventRecord(ready)");
  e->copies += 1;
  e->bytes += bytes;
  e->busy_ns += static_cast<unsigned long long>((h3b::now_s() - t0) * 1e9);
  return H3B_OK;
}

int h3b_streamer_begin(h3b_streamer* s, int slot) {
  if (!s || slot < 0 || slot >= static_cast<int>(s->e->ready.size())) return fail(H3B_ERR_ARG, "streamer_begin: bad slot");
  cudaError_t err = cudaSetDevice(s->e->device);
  if (err == cudaSuccess && s->e->done_set[slot]) err = cudaStreamWaitEvent(s->e->copy, s->e->done[slot], 0);
  return err == cudaSuccess ? H3B_OK : cuda_fail(err, "streamer_begin");
}

int h3b_streamer_end(h3b_streamer* s, int slot, size_t bytes) {
  if (!s || slot < 0 || slot >= static_cast<int>(s->e->ready.size())) return fail(H3B_ERR_ARG, "streamer_end: bad slot");
  const cudaError_t err = cudaEventRecord(s->e->ready[slot], s->e->copy);
  if (err != cudaSuccess) return cuda_fail(err, "cudaEventRecord(ready)");
  s->e->copies += 1;
  s->e->bytes += bytes;
  return H3B_OK;
}

void* h3b_streamer_stream(h3b_streamer* s) { return s ? static_cast<void*>(s->e->copy) : nullptr; }

int h3b_streamer_acquire(h3b_streamer* s, int slot, void* stream) {
  if (!s || slot < 0 || slot >= static_cast<int>(s->e->ready.size())) return fail(H3B_ERR_ARG, "streamer_acquire: bad slot");
  const cudaError_t err = cudaStreamWaitEvent(static_cast<cudaStream_t>(stream), s->e->ready[slot], 0);
  return err == cudaSuccess ? H3B_OK : cuda_fail(err, "cudaStreamWaitEvent(ready)");
}

int h3b_streamer_release(h3b_streamer* s, int slot, void* stream) {
  if (!s || slot < 0 || slot >= static_cast<int>(s->e->done.size())) return fail(H3B_ERR_ARG, "streamer_release: bad slot");
  const cudaError_t err = cudaEventRecord(s->e->done[slot], static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail(err, "cudaEventRecord(done)");
  s->e->done_set[slot] = 1;
  return H3B_OK;
}

int h3b_streamer_wait(h3b_streamer* s, int slot, double timeout_s) {
  if (!s || slot < 0 || slot >= static_cast<int>(s->e->ready.size())) return fail(H3B_ERR_ARG, "streamer_wait: bad slot");
  return h3b::event_wait(s->e->ready[slot], timeout_s, "streamer copy");
}

int h3b_streamer_stats(h3b_streamer* s, uint64_t* copies, uint64_t* bytes, double* busy_s) {
  if (!s) return fail(H3B_ERR_ARG, "streamer_stats: bad engine");
  if (copies) *copies = s->e->copies.load();
  if (bytes) *bytes = s->e->bytes.load();
  if (busy_s) *busy_s = s->e->busy_ns.load() * 1e-9;
  return H3B_OK;
}

int h3b_host_register(void* ptr, size_t bytes, int read_only) {
  if (!ptr || bytes == 0) return fail(H3B_ERR_ARG, "host_register: empty range");
  const cudaError_t err = cudaHostRegister(ptr, bytes, read_only ? cudaHostRegisterReadOnly : cudaHostRegisterDefault);
  if (err != cudaSuccess) {
    cudaGetLastError();  // not sticky: the caller falls back to a pinned copy or staging
    return cuda_fail(err, "cudaHostRegister");
  }
  return H3B_OK;
}

int h3b_host_unregister(void* ptr) {
  const cudaError_t err = cudaHostUnregister(ptr);
  if (err != cudaSuccess) {
    cudaGetLastError();
    return cuda_fail(err, "cudaHostUnregister");
  }
  return H3B_OK;
}

int h3b_device_error(int clear) {
  unsigned int v = 0;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return -static_cast<int>(cuda_fail(e, "cudaDeviceSynchronize"));
  cudaError_t (*const units[])(unsigned*, int) = {device_error_abi, device_error_act, device_error_decode,
                                                  device_error_gemm, device_error_w4, device_error_w4_fp8,
                                                  device_error_w4_fp16, device_error_w4_bf16, device_error_w4_fp32};
  for (auto unit : units) {
    unsigned u = 0;
    e = unit(&u, clear);
    if (e != cudaSuccess) return -static_cast<int>(cuda_fail(e, "device failure flag"));
    v |= u;
  }
  return static_cast<int>(v);
}

}  // extern "C"
