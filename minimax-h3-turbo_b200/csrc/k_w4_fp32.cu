// Translation unit: the decode-in-producer W4A8 GEMMs (gemm_w4.cuh, and the small-M split-K gemm_w4s.cuh) for fp32 group scales, every epilogue variant.
#include "gemm_w4.cuh"
#include "gemm_w4s.cuh"

namespace h3b {

template int w4_launch_sdt<H3B_FP32>(int, int, int, const int8_t*, int64_t, const void*, int64_t, const void*, int64_t,
                                  const float*, const float*, const float*, const void*, void*, int64_t, int, int, int,
                                  cudaStream_t);

template int w4s_launch_sdt<H3B_FP32>(const W4sPlan*, const int8_t*, int64_t, const void*, int64_t, const void*, int64_t,
                                   const float*, const W4sEpi&, int, int, int, cudaStream_t);

H3B_DEVICE_ERROR_ACCESSOR(device_error_w4_fp32)

}  // namespace h3b
