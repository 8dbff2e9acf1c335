// Translation unit: dispatch of the W4A8 GEMMs that decode the int4 weight in their producer warps -- the small-M
// split-K kernel (gemm_w4s.cuh, M <= 256) and the tile kernel for up to 1024 rows (gemm_w4.cuh); the kernels are
// instantiated per group-scale dtype in k_w4_<dtype>.cu.
#include "gemm_w4.cuh"
#include "gemm_w4s.cuh"
#include "launch.h"

#include <cstdio>
#include <cstdlib>

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

extern template int w4s_launch_sdt<H3B_FP8_E4M3>(const W4sPlan*, const int8_t*, int64_t, const void*, int64_t, const void*,
                                                 int64_t, const float*, const W4sEpi&, int, int, int, cudaStream_t);
extern template int w4s_launch_sdt<H3B_FP16>(const W4sPlan*, const int8_t*, int64_t, const void*, int64_t, const void*,
                                             int64_t, const float*, const W4sEpi&, int, int, int, cudaStream_t);
extern template int w4s_launch_sdt<H3B_BF16>(const W4sPlan*, const int8_t*, int64_t, const void*, int64_t, const void*,
                                             int64_t, const float*, const W4sEpi&, int, int, int, cudaStream_t);
extern template int w4s_launch_sdt<H3B_FP32>(const W4sPlan*, const int8_t*, int64_t, const void*, int64_t, const void*,
                                             int64_t, const float*, const W4sEpi&, int, int, int, cudaStream_t);

// The small-M split-K kernel serves M <= 256 (H3B_W4S=0 in the environment turns it off: read once per process; for
// comparisons).
static bool w4s_enabled(int64_t M) {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("H3B_W4S");
    v = (e && e[0] == '0') ? 0 : 1;
  }
  return v == 1 && M >= 1 && M <= 2 * BM;
}

// Whether the decode-in-producer kernel takes this problem: few M tiles (the 1-CTA kernel's regime), a supported
// weight format, and a packed weight TMA can read (16-byte aligned rows).
bool w4_fused_ok(int64_t M, int64_t N, int64_t K, const void* q4, int64_t ldq4, int s_dtype, int group) {
  const bool fmt = (s_dtype == H3B_FP8_E4M3 && group == 16) ||
                   ((s_dtype == H3B_FP16 || s_dtype == H3B_BF16 || s_dtype == H3B_FP32) && group == 128);
  if (!fmt || ldq4 % 16 || (reinterpret_cast<uintptr_t>(q4) & 15) || K % 16) return false;
  if (w4s_enabled(M)) return true;
  const int bn = pick_bn(static_cast<int>(M), static_cast<int>(N));
  return bn <= 192 && M <= 1024;
}

int gemm_w4_launch(const int8_t* a, int64_t lda, const void* q4, int64_t ldq4, const void* s_rel, int s_dtype,
                   int64_t lds, const float* codebook, const float* xs, const float* sch, const void* bias, void* out,
                   int out_dtype, int64_t ldo, int64_t M, int64_t N, int64_t K, int qmode, cudaStream_t st) {
  const int m = static_cast<int>(M), n = static_cast<int>(N), k = static_cast<int>(K);
  if (w4s_enabled(M)) {
    // H3B_W4S_PLAN="bn,splits,subtiles" in the environment replaces the planner's choice (read per call; for tile
    // sweeps)
    W4sPlan forced{0, 0, 0};
    const W4sPlan* plan = nullptr;
    if (const char* e = getenv("H3B_W4S_PLAN")) {
      int bn = 0, sp = 0, ms = 0;
      if (sscanf(e, "%d,%d,%d", &bn, &sp, &ms) == 3 && bn == W4S_BN && sp >= 1 && sp <= 8 &&
          sp <= static_cast<int>((K + BK - 1) / BK) && (ms == 1 || (ms == 2 && M <= 2 * BM))) {
        forced = W4sPlan{bn, ms, sp};
        plan = &forced;
      }
    }
    const W4sEpi epi{xs, sch, bias, out, ldo, out_dtype, qmode};
    switch (s_dtype) {
      case H3B_FP8_E4M3: return w4s_launch_sdt<H3B_FP8_E4M3>(plan, a, lda, q4, ldq4, s_rel, lds, codebook, epi, m, n, k, st);
      case H3B_FP16: return w4s_launch_sdt<H3B_FP16>(plan, a, lda, q4, ldq4, s_rel, lds, codebook, epi, m, n, k, st);
      case H3B_BF16: return w4s_launch_sdt<H3B_BF16>(plan, a, lda, q4, ldq4, s_rel, lds, codebook, epi, m, n, k, st);
      case H3B_FP32: return w4s_launch_sdt<H3B_FP32>(plan, a, lda, q4, ldq4, s_rel, lds, codebook, epi, m, n, k, st);
      default: return fail(H3B_ERR_ARG, "group scale dtype must be fp8_e4m3, fp16, bf16 or fp32");
    }
  }
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
