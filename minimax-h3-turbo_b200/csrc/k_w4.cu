// Translation unit: the W4A8 GEMM that decodes the int4 weight in its producer warps (gemm_w4.cuh).
#include "gemm_w4.cuh"
#include "launch.h"

namespace h3b {

extern template int w4_launch_sdt<H3B_FP8_E4M3>(int, int, int, const int8_t*, int64_t, const void*, int64_t, const void*,
                                                int64_t, const float*, const float*, const float*, const void*, void*,
                                                int64_t, int, int, int, cudaStream_t);
extern template int w4_launch_sdt<H3B_FP16>(int, int, int, const int8_t*, int64_t, const void*, int64_t, const void*,
                                            int64_t, const float*, const float*, const float*, const void*, void*,
                                            int64_t, int, int, int, cudaStream_t);
extern template int w4_launch_sdt<H3B_BF16>(int, int, int, const int8_t*, int64_t, const void*, int64_t, const void*,
                                            int64_t, const float*, const float*, const float*, const void*, void*,
                                            int64_t, int, int, int, cudaStream_t);
extern template int w4_launch_sdt<H3B_FP32>(int, int, int, const int8_t*, int64_t, const void*, int64_t, const void*,
                                            int64_t, const float*, const float*, const float*, const void*, void*,
                                            int64_t, int, int, int, cudaStream_t);

// Whether the decode-in-producer kernel takes this problem: few M tiles (the 1-CTA kernel's regime), a supported
// weight format, and a packed weight TMA can read (16-byte aligned rows).
bool w4_fused_ok(int64_t M, int64_t N, int64_t K, const void* q4, int64_t ldq4, int s_dtype, int group) {
  const bool fmt = (s_dtype == H3B_FP8_E4M3 && group == 16) ||
                   ((s_dtype == H3B_FP16 || s_dtype == H3B_BF16 || s_dtype == H3B_FP32) && group == 128);
  if (!fmt || ldq4 % 16 || (reinterpret_cast<uintptr_t>(q4) & 15) || K % 16) return false;
  const int bn = pick_bn(static_cast<int>(M), static_cast<int>(N));
  return bn <= 192 && M <= 1024;
}

size_t w4_workspace_bytes(int64_t M, int64_t N, int64_t K) {
  (void)M;
  (void)N;
  (void)K;
  return 0;
}

int gemm_w4_launch(const int8_t* a, int64_t lda, const void* q4, int64_t ldq4, const void* s_rel, int s_dtype,
                   int64_t lds, const float* codebook, const float* xs, const float* sch, const void* bias, void* out,
                   int out_dtype, int64_t ldo, int64_t M, int64_t N, int64_t K, int qmode, void* ws, size_t ws_bytes,
                   cudaStream_t st) {
  (void)ws;
  (void)ws_bytes;
  const int m = static_cast<int>(M), n = static_cast<int>(N), k = static_cast<int>(K);
  const int bn = pick_bn(m, n);
  switch (s_dtype) {
    case H3B_FP8_E4M3:
      return w4_launch_sdt<H3B_FP8_E4M3>(out_dtype, qmode, bn, a, lda, q4, ldq4, s_rel, lds, codebook, xs, sch, bias, out, ldo, m, n, k, st);
    case H3B_FP16:
      return w4_launch_sdt<H3B_FP16>(out_dtype, qmode, bn, a, lda, q4, ldq4, s_rel, lds, codebook, xs, sch, bias, out, ldo, m, n, k, st);
    case H3B_BF16:
      return w4_launch_sdt<H3B_BF16>(out_dtype, qmode, bn, a, lda, q4, ldq4, s_rel, lds, codebook, xs, sch, bias, out, ldo, m, n, k, st);
    case H3B_FP32:
      return w4_launch_sdt<H3B_FP32>(out_dtype, qmode, bn, a, lda, q4, ldq4, s_rel, lds, codebook, xs, sch, bias, out, ldo, m, n, k, st);
    default: return fail(H3B_ERR_ARG, "group scale dtype must be fp8_e4m3, fp16, bf16 or fp32");
  }
}

H3B_DEVICE_ERROR_ACCESSOR(device_error_w4)

}  // namespace h3b
