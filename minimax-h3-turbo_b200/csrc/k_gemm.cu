// Translation unit: the int8 GEMM + epilogue, 1-CTA and CTA-pair kernels (gemm_sm100.cuh), and their dispatch.
#include "gemm_sm100.cuh"
#include "launch.h"

namespace h3b {

// Bytes of weight rows one super-column of output tiles may span (the CTAs working at the same time read them all, so
// they should stay in L2 while the activation rows stream past).  H3B_GEMM_GN_MB in the environment overrides the
// default (read once per process; for sweeps).
static int64_t gn_budget() {
  static int64_t v = -1;
  if (v < 0) {
    const char* e = getenv("H3B_GEMM_GN_MB");
    const long mb = e ? atol(e) : 0;
    v = (mb > 0 ? mb : 24) << 20;
  }
  return v;
}

template <int BN, int OUT, bool BIAS, int QMODE>
static int launch_gemm(const int8_t* a, int64_t lda, const int8_t* b, int64_t ldb, const float* xs, const float* sch,
                       const void* bias, void* out, int64_t ldo, int M, int N, int K, cudaStream_t st) {
  using C = GemmCfg<BN>;
  CUtensorMap ta, tb;
  int rc = make_map(&ta, a, K, M, lda, BM);
  if (rc) return rc;
  rc = make_map(&tb, b, K, N, ldb, BN);
  if (rc) return rc;
  auto kern = gemm_i8_kernel<BN, OUT, BIAS, QMODE>;
  static std::atomic<unsigned long long> attr_done{0};  // one bit per device, per instantiation
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned long long bit = 1ull << (dev & 63);
  if (!(attr_done.load() & bit)) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(gemm)");
    attr_done.fetch_or(bit);
  }
  const int tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  const int sms = num_sms();
  const int grid = tiles < sms ? tiles : sms;
  // weight block per super-column <= gn_budget() bytes of int8 rows, so it stays in L2 while every M tile passes over it
  const int n_tiles = (N + BN - 1) / BN;
  int gn = static_cast<int>(gn_budget() / (static_cast<int64_t>(BN) * K));
  gn = gn < 1 ? 1 : (gn > n_tiles ? n_tiles : gn);
  kern<<<grid, 192, C::SMEM, st>>>(ta, tb, xs, sch, bias, out, ldo, M, N, K, gn);
  return check_launch("gemm_i8_kernel");
}

template <int OUT, bool BIAS, int QMODE>
static int launch_gemm_pair(const int8_t* a, int64_t lda, const int8_t* b, int64_t ldb, const float* xs, const float* sch,
                            const void* bias, void* out, int64_t ldo, int M, int N, int K, cudaStream_t st) {
  CUtensorMap ta, tb;
  int rc = make_map(&ta, a, K, M, lda, BM);
  if (rc) return rc;
  rc = make_map(&tb, b, K, N, ldb, P_BN / 2);
  if (rc) return rc;
  auto kern = gemm_i8_pair_kernel<OUT, BIAS, QMODE>;
  static std::atomic<unsigned long long> attr_done{0};
  static int max_pairs[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned long long bit = 1ull << (dev & 63);
  if (!(attr_done.load() & bit)) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, P_SMEM);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(gemm pair)");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * 74, 1, 1);
    cfg.blockDim = dim3(192, 1, 1);
    cfg.dynamicSmemBytes = P_SMEM;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 2;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int n = 0;
    e = cudaOccupancyMaxActiveClusters(&n, kern, &cfg);
    if (e != cudaSuccess || n < 1) {
      cudaGetLastError();
      n = num_sms() / 2;
    }
    max_pairs[dev & 63] = n;
    attr_done.fetch_or(bit);
  }
  const int tiles = ((M + P_BM - 1) / P_BM) * ((N + P_BN - 1) / P_BN);
  const int pairs = tiles < max_pairs[dev & 63] ? tiles : max_pairs[dev & 63];
  const int n_tiles = (N + P_BN - 1) / P_BN;
  int gn = static_cast<int>(gn_budget() / (static_cast<int64_t>(P_BN) * K));
  gn = gn < 1 ? 1 : (gn > n_tiles ? n_tiles : gn);
  kern<<<2 * pairs, 192, P_SMEM, st>>>(ta, tb, xs, sch, bias, out, ldo, M, N, K, gn);
  return check_launch("gemm_i8_pair_kernel");
}

// The CTA-pair kernel for shapes that fill the GPU with 256 x 256 tiles; H3B_GEMM_PAIR=0 in the environment keeps the
// 1-CTA kernel (read once per process; for comparisons).
static bool pair_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("H3B_GEMM_PAIR");
    v = (e && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

template <int OUT, bool BIAS, int QMODE>
static int dispatch_bn(int bn, const int8_t* a, int64_t lda, const int8_t* b, int64_t ldb, const float* xs,
                       const float* sch, const void* bias, void* out, int64_t ldo, int M, int N, int K, cudaStream_t st) {
  if (bn == 256 && M >= P_BM && pair_enabled())
    return launch_gemm_pair<OUT, BIAS, QMODE>(a, lda, b, ldb, xs, sch, bias, out, ldo, M, N, K, st);
  switch (bn) {
    case 256: return launch_gemm<256, OUT, BIAS, QMODE>(a, lda, b, ldb, xs, sch, bias, out, ldo, M, N, K, st);
    case 192: return launch_gemm<192, OUT, BIAS, QMODE>(a, lda, b, ldb, xs, sch, bias, out, ldo, M, N, K, st);
    case 128: return launch_gemm<128, OUT, BIAS, QMODE>(a, lda, b, ldb, xs, sch, bias, out, ldo, M, N, K, st);
    case 96: return launch_gemm<96, OUT, BIAS, QMODE>(a, lda, b, ldb, xs, sch, bias, out, ldo, M, N, K, st);
    case 64: return launch_gemm<64, OUT, BIAS, QMODE>(a, lda, b, ldb, xs, sch, bias, out, ldo, M, N, K, st);
    default: return launch_gemm<32, OUT, BIAS, QMODE>(a, lda, b, ldb, xs, sch, bias, out, ldo, M, N, K, st);
  }
}

template <int OUT>
static int dispatch_epi(bool has_bias, int qmode, int bn, const int8_t* a, int64_t lda, const int8_t* b, int64_t ldb,
                        const float* xs, const float* sch, const void* bias, void* out, int64_t ldo, int M, int N, int K,
                        cudaStream_t st) {
  if (qmode == H3B_QMODE_CK)
    return has_bias ? dispatch_bn<OUT, true, 0>(bn, a, lda, b, ldb, xs, sch, bias, out, ldo, M, N, K, st)
                    : dispatch_bn<OUT, false, 0>(bn, a, lda, b, ldb, xs, sch, bias, out, ldo, M, N, K, st);
  return has_bias ? dispatch_bn<OUT, true, 1>(bn, a, lda, b, ldb, xs, sch, bias, out, ldo, M, N, K, st)
                  : dispatch_bn<OUT, false, 1>(bn, a, lda, b, ldb, xs, sch, bias, out, ldo, M, N, K, st);
}

int gemm_launch(const int8_t* a, int64_t lda, const int8_t* b, int64_t ldb, const float* xs, const float* sch,
                const void* bias, void* out, int out_dtype, int64_t ldo, int64_t M, int64_t N, int64_t K, int qmode,
                cudaStream_t st) {
  const int bn = pick_bn(static_cast<int>(M), static_cast<int>(N));
  const int m = static_cast<int>(M), n = static_cast<int>(N), k = static_cast<int>(K);
  switch (out_dtype) {
    case H3B_BF16: return dispatch_epi<OUT_BF16>(bias != nullptr, qmode, bn, a, lda, b, ldb, xs, sch, bias, out, ldo, m, n, k, st);
    case H3B_FP16: return dispatch_epi<OUT_FP16>(bias != nullptr, qmode, bn, a, lda, b, ldb, xs, sch, bias, out, ldo, m, n, k, st);
    case H3B_FP32: return dispatch_epi<OUT_FP32>(bias != nullptr, qmode, bn, a, lda, b, ldb, xs, sch, bias, out, ldo, m, n, k, st);
    case H3B_INT32: return dispatch_bn<OUT_S32, false, 0>(bn, a, lda, b, ldb, xs, sch, nullptr, out, ldo, m, n, k, st);
    default: return fail(H3B_ERR_ARG, "out dtype must be bf16, fp16, fp32 or int32");
  }
}

H3B_DEVICE_ERROR_ACCESSOR(device_error_gemm)

}  // namespace h3b
