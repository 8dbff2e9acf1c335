// Host-side interface between the translation units of libh3b.so: the launch functions each kernel file exports to the
// C ABI (libh3b.cu), the small argument structs they share, and the per-unit device failure flags.
//
// Translation units (compiled in parallel, linked into one library without relocatable device code):
//   k_act.cu      rotate + quantise (rotq.cuh), RMSNorm + modulation (rmsmod.cuh), q/k norm + RoPE (rope.cuh),
//                 attention merge (attn_merge.cuh)
//   k_decode.cu   int4 -> int8 grid decode (decode.cuh)
//   k_gemm.cu     int8 GEMM + epilogue, 1-CTA and CTA-pair kernels (gemm_sm100.cuh)
//   k_w4.cu       dispatch of the decode-in-producer W4A8 GEMM for few M tiles (gemm_w4.cuh), instantiated per group
//                 scale dtype in k_w4_fp8.cu, k_w4_fp16.cu, k_w4_bf16.cu, k_w4_fp32.cu
//   libh3b.cu     the C ABI, argument checks, the block streamer, the wait self-test
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/h3b.h"

namespace h3b {

enum { MODE_CK = 0, MODE_EAGER = 1, MODE_ROTATE = 2 };

// Token segments passed by value (no device table to upload per call).
constexpr int MAX_SEGMENTS = H3B_MAX_SEGMENTS;
struct SegTable {
  int n;
  int64_t first[MAX_SEGMENTS], end[MAX_SEGMENTS];
  int row[MAX_SEGMENTS];
};

// Operands of the RMSNorm + modulation prologue fused into the quantiser: h = dt(dt(dt((x rs) w) s1) + sh) per token,
// rs = rsqrt(mean(x^2) + eps), the steps and roundings of rms_modulate_warp_kernel (model.py:_rms :64-66,
// _scale_shift_ :106-109).  All bf16; scale1 is dt(1 + dt(scale)), the factor _scale_shift_ multiplies by; a token
// outside every segment (row < 0) keeps n.
struct RowNorm {
  const __nv_bfloat16* w;       // [K]
  const __nv_bfloat16* shift;   // [rows][ldm]
  const __nv_bfloat16* scale1;  // [rows][ldm]
  int64_t ldm;
  float eps;
  const int* token_rows;  // per-token modulation row (negative: none), or null: the segments decide
  SegTable segs;
};

// ---- k_act.cu
int rotq_launch(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx, int convrot, int swiglu, int mode,
                int8_t* q, int64_t ldq, float* xs, void* y, int y_dtype, int64_t ldy, cudaStream_t st);
bool rotq_rmsmod_supported(int64_t K);
int rotq_rmsmod_launch(const void* x, int64_t ldx, int64_t M, int64_t K, const RowNorm& nrm, int mode, int8_t* q,
                       int64_t ldq, float* xs, cudaStream_t st);
int rms_modulate_launch(const void* x, int x_dtype, int64_t ldx, int64_t M, int H, const void* w, int w_dtype, float eps,
                        const void* shift, const void* scale, int64_t ldm, int m_dtype, const int32_t* segments,
                        int n_segments, const int32_t* token_rows, void* h, int64_t ldh, cudaStream_t st);
int gate_residual_launch(void* x, int x_dtype, int64_t ldx, const void* other, int64_t ldo, int64_t M, int H,
                         const void* gate, int64_t ldm, int m_dtype, const int32_t* segments, int n_segments,
                         const int32_t* token_rows, cudaStream_t st);
int qk_norm_rope_launch(void* q, int64_t ldq, void* k, int64_t ldk, int x_dtype, int64_t S, int heads, int D,
                        const void* wq, const void* wk, int w_dtype, float eps, const void* cos_t, const void* sin_t,
                        int64_t ldt, int t_dtype, int half, cudaStream_t st);
int attn_merge_launch(float* acc, float* acc_lse, const void* o, int64_t o_sh, int64_t o_sq, const float* lse, int64_t H,
                      int64_t Q, int D, int first, void* out, int64_t ldo, cudaStream_t st);

// ---- k_decode.cu
int decode_launch(const void* q4, int64_t N, int64_t K, int64_t ldq4, const void* s_rel, int s_dtype, int64_t lds,
                  const float* codebook, int group, int8_t* grid, int64_t ldg, cudaStream_t st);

// ---- k_gemm.cu
int gemm_launch(const int8_t* a, int64_t lda, const int8_t* b, int64_t ldb, const float* xs, const float* sch,
                const void* bias, void* out, int out_dtype, int64_t ldo, int64_t M, int64_t N, int64_t K, int qmode,
                cudaStream_t st);

// ---- k_w4.cu
bool w4_fused_ok(int64_t M, int64_t N, int64_t K, const void* q4, int64_t ldq4, int s_dtype, int group);
// The decode-in-producer GEMM; it needs no scratch (the small-M kernel reduces its K splits inside a cluster).
int gemm_w4_launch(const int8_t* a, int64_t lda, const void* q4, int64_t ldq4, const void* s_rel, int s_dtype,
                   int64_t lds, const float* codebook, const float* xs, const float* sch, const void* bias, void* out,
                   int out_dtype, int64_t ldo, int64_t M, int64_t N, int64_t K, int qmode, cudaStream_t st);

// ---- device failure flags: every translation unit has its own copy of the flag (h3b_common.cuh); each returns its
// value (after synchronising nothing: the caller synchronises first) and clears it when asked.  0 or a CUDA error.
cudaError_t device_error_act(unsigned* v, int clear);
cudaError_t device_error_decode(unsigned* v, int clear);
cudaError_t device_error_gemm(unsigned* v, int clear);
cudaError_t device_error_w4(unsigned* v, int clear);
cudaError_t device_error_w4_fp8(unsigned* v, int clear);
cudaError_t device_error_w4_fp16(unsigned* v, int clear);
cudaError_t device_error_w4_bf16(unsigned* v, int clear);
cudaError_t device_error_w4_fp32(unsigned* v, int clear);

}  // namespace h3b
