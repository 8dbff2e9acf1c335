// Translation unit: the int4 -> int8 grid decode (decode.cuh).
#include "decode.cuh"
#include "launch.h"

namespace h3b {

int decode_launch(const void* q4, int64_t N, int64_t K, int64_t ldq4, const void* s_rel, int s_dtype, int64_t lds,
                  const float* codebook, int group, int8_t* grid, int64_t ldg, cudaStream_t st) {
  const int64_t total = N * (K / 16);
  if (total == 0) return H3B_OK;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (group % 16 == 0) {
    const int64_t segs = N * ((K + SEG - 1) / SEG);
    const int64_t want_t = (segs + 255) / 256;
    const int nb = static_cast<int>(want_t < 16ll * sms ? want_t : 16ll * sms);
    const uint8_t* qt = static_cast<const uint8_t*>(q4);
    switch (s_dtype) {
      case H3B_FP8_E4M3: decode_tab_kernel<H3B_FP8_E4M3><<<nb, 256, 0, st>>>(qt, N, K, ldq4, s_rel, lds, codebook, group, grid, ldg); break;
      case H3B_FP16: decode_tab_kernel<H3B_FP16><<<nb, 256, 0, st>>>(qt, N, K, ldq4, s_rel, lds, codebook, group, grid, ldg); break;
      case H3B_BF16: decode_tab_kernel<H3B_BF16><<<nb, 256, 0, st>>>(qt, N, K, ldq4, s_rel, lds, codebook, group, grid, ldg); break;
      case H3B_FP32: decode_tab_kernel<H3B_FP32><<<nb, 256, 0, st>>>(qt, N, K, ldq4, s_rel, lds, codebook, group, grid, ldg); break;
      default: return fail(H3B_ERR_ARG, "group scale dtype must be fp8_e4m3, fp16, bf16 or fp32");
    }
    return check_launch("decode_tab_kernel");
  }
  const int64_t want = (total + 255) / 256;
  const int blocks = static_cast<int>(want < 16ll * sms ? want : 16ll * sms);
  const uint8_t* q = static_cast<const uint8_t*>(q4);
  switch (s_dtype) {
    case H3B_FP8_E4M3: decode_kernel<H3B_FP8_E4M3><<<blocks, 256, 0, st>>>(q, N, K, ldq4, s_rel, lds, codebook, group, grid, ldg); break;
    case H3B_FP16: decode_kernel<H3B_FP16><<<blocks, 256, 0, st>>>(q, N, K, ldq4, s_rel, lds, codebook, group, grid, ldg); break;
    case H3B_BF16: decode_kernel<H3B_BF16><<<blocks, 256, 0, st>>>(q, N, K, ldq4, s_rel, lds, codebook, group, grid, ldg); break;
    case H3B_FP32: decode_kernel<H3B_FP32><<<blocks, 256, 0, st>>>(q, N, K, ldq4, s_rel, lds, codebook, group, grid, ldg); break;
    default: return fail(H3B_ERR_ARG, "group scale dtype must be fp8_e4m3, fp16, bf16 or fp32");
  }
  return check_launch("decode_kernel");
}

H3B_DEVICE_ERROR_ACCESSOR(device_error_decode)

}  // namespace h3b
