// int4 codebook indices + group scales -> the exact int8 weight grid.
//
// Reference semantics (h3turbo/h3/qlinear.py:157-204, format types.py:14-16):
//   nibble[n, 2j] = low nibble of q[n, j], nibble[n, 2j + 1] = high nibble
//   level[n, k]   = clamp(rint(fp32(codebook[nibble]) * fp32(s_rel[n, k / group])), -127, 127)   (half-to-even)
//   fp8 scale bytes that are NaN decode to level 0 (the pair table's nan_to_num, :162).
// One thread decodes 16 consecutive weights (8 packed bytes) of one row and stores them as one 16-byte vector.
#include "h3b_common.cuh"

namespace h3b {

template <int SDT>
__device__ __forceinline__ float scale_at(const void* s, int64_t idx) {
  if constexpr (SDT == H3B_FP8_E4M3) return fp8e4m3_to_f32(static_cast<const uint8_t*>(s)[idx]);
  else if constexpr (SDT == H3B_FP16) return __half2float(static_cast<const __half*>(s)[idx]);
  else if constexpr (SDT == H3B_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(s)[idx]);
  else return static_cast<const float*>(s)[idx];
}

// level = clamp(rint(cb * s), -127, 127); NaN -> 0.  cvt.rni.sat.s8 rounds half-to-even, saturates to [-128, 127]
// and maps NaN to 0; the lower clamp to -127 is the reference's symmetric range.
__device__ __forceinline__ uint32_t level_of(float cb, float s) {
  const float prod = __fmul_rn(cb, s);
  int l;
  asm("cvt.rni.sat.s8.f32 %0, %1;" : "=r"(l) : "f"(prod));
  l = max(l, -127);
  return static_cast<uint32_t>(l) & 0xFFu;
}

template <int SDT>
__global__ void __launch_bounds__(256) decode_kernel(const uint8_t* __restrict__ q4, int64_t N, int64_t K, int64_t ldq4,
                                                     const void* __restrict__ s_rel, int64_t lds,
                                                     const float* __restrict__ codebook, int group,
                                                     int8_t* __restrict__ grid, int64_t ldg) {
  __shared__ float cbs[16];
  if (threadIdx.x < 16) cbs[threadIdx.x] = codebook[threadIdx.x];
  __syncthreads();
  const int64_t chunks_per_row = K / 16;
  const int64_t total = N * chunks_per_row;
  for (int64_t c = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; c < total;
       c += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t n = c / chunks_per_row;
    const int64_t k0 = (c - n * chunks_per_row) * 16;
    const uint2 packed = *reinterpret_cast<const uint2*>(q4 + n * ldq4 + k0 / 2);
    const uint32_t pw[2] = {packed.x, packed.y};
    const int64_t srow = n * lds;
    float s16[4];
    if (group % 16 == 0) {
      const float s = scale_at<SDT>(s_rel, srow + k0 / group);
      s16[0] = s16[1] = s16[2] = s16[3] = s;
    } else {  // group 4 or 8: 16 / group scales in this chunk
#pragma unroll
      for (int i = 0; i < 4; ++i) s16[i] = scale_at<SDT>(s_rel, srow + (k0 + 4 * i) / group);
    }
    uint32_t out[4];
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const uint32_t bytes = pw[w >> 1] >> (16 * (w & 1));  // 2 packed bytes = 4 weights
      const float s = s16[w];
      const uint32_t l0 = level_of(cbs[bytes & 0xF], s);
      const uint32_t l1 = level_of(cbs[(bytes >> 4) & 0xF], s);
      const uint32_t l2 = level_of(cbs[(bytes >> 8) & 0xF], s);
      const uint32_t l3 = level_of(cbs[(bytes >> 12) & 0xF], s);
      out[w] = l0 | (l1 << 8) | (l2 << 16) | (l3 << 24);
    }
    *reinterpret_cast<uint4*>(grid + n * ldg + k0) = make_uint4(out[0], out[1], out[2], out[3]);
  }
}

int decode_launch(const void* q4, int64_t N, int64_t K, int64_t ldq4, const void* s_rel, int s_dtype, int64_t lds,
                  const float* codebook, int group, int8_t* grid, int64_t ldg, cudaStream_t st) {
  const int64_t total = N * (K / 16);
  if (total == 0) return H3B_OK;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
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

}  // namespace h3b
