// int4 codebook indices + group scales -> the exact int8 weight grid.
//
// Reference semantics (h3turbo/h3/qlinear.py:157-204, format types.py:14-16):
//   nibble[n, 2j] = low nibble of q[n, j], nibble[n, 2j + 1] = high nibble
//   level[n, k]   = clamp(rint(fp32(codebook[nibble]) * fp32(s_rel[n, k / group])), -127, 127)   (half-to-even)
//   fp8 scale bytes that are NaN decode to level 0 (the pair table's nan_to_num, :162).
// One thread decodes 16 consecutive weights (8 packed bytes) of one row and stores them as one 16-byte vector.
#pragma once

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

// ------------------------------------------------------------------------------------------------ table decode
// For groups of 16 or more weights the 16 possible levels of a scale are computed once (a "level table": byte j of
// word w = level of codebook index 4 w + j) and the nibbles are translated by byte permutes, 1.5 instructions per
// weight instead of a float product and a conversion each.  fp8 scales: the 256 tables of every scale byte are built
// once per CTA in shared memory.  Same levels as level_of, bit for bit.
__device__ __forceinline__ uint32_t pack4(uint32_t l0, uint32_t l1, uint32_t l2, uint32_t l3) {
  return __byte_perm(__byte_perm(l0, l1, 0x0040), __byte_perm(l2, l3, 0x0040), 0x5410);
}
__device__ __forceinline__ uint4 level_table(const float (&cb)[16], float s) {
  uint32_t t[4];
#pragma unroll
  for (int w = 0; w < 4; ++w)
    t[w] = pack4(level_of(cb[4 * w], s), level_of(cb[4 * w + 1], s), level_of(cb[4 * w + 2], s), level_of(cb[4 * w + 3], s));
  return make_uint4(t[0], t[1], t[2], t[3]);
}
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));  // selector bit 3: replicate the byte's sign bit
  return d;
}
// 8 nibbles (low nibble first) -> 8 level bytes (two words), by table lookups
__device__ __forceinline__ uint2 decode8(uint32_t w, const uint4& t) {
  const uint32_t sel = w & 0x77777777u;          // codebook index mod 8 per nibble: a byte of {t.x, t.y} or {t.z, t.w}
  const uint32_t y = w & 0x88888888u, y4 = y << 4;  // bit 3 of nibble i at the top of a byte of y4 (even i) / y (odd i)
  const uint32_t lo0 = prmt(t.x, t.y, sel), hi0 = prmt(t.z, t.w, sel);
  const uint32_t m0 = prmt(y4, y, 0xD9C8u);      // 0xFF bytes where the index is >= 8
  const uint32_t sh = sel >> 16;
  const uint32_t lo1 = prmt(t.x, t.y, sh), hi1 = prmt(t.z, t.w, sh);
  const uint32_t m1 = prmt(y4, y, 0xFBEAu);
  return make_uint2((hi0 & m0) | (lo0 & ~m0), (hi1 & m1) | (lo1 & ~m1));
}

constexpr int SEG = 128;  // weights per thread (8 chunks of 16)

template <int SDT>
__global__ void __launch_bounds__(256) decode_tab_kernel(const uint8_t* __restrict__ q4, int64_t N, int64_t K, int64_t ldq4,
                                                         const void* __restrict__ s_rel, int64_t lds,
                                                         const float* __restrict__ codebook, int group,
                                                         int8_t* __restrict__ grid, int64_t ldg) {
  __shared__ float cbs[16];
  __shared__ uint4 lut[SDT == H3B_FP8_E4M3 ? 256 : 1];
  if (threadIdx.x < 16) cbs[threadIdx.x] = codebook[threadIdx.x];
  __syncthreads();
  float cb[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) cb[i] = cbs[i];
  if constexpr (SDT == H3B_FP8_E4M3) {
    for (int b = threadIdx.x; b < 256; b += blockDim.x) lut[b] = level_table(cb, fp8e4m3_to_f32(static_cast<uint32_t>(b)));
    __syncthreads();
  }
  const int64_t segs_per_row = (K + SEG - 1) / SEG;
  const int64_t total = N * segs_per_row;
  for (int64_t c = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; c < total;
       c += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t n = c / segs_per_row;
    const int64_t k0 = (c - n * segs_per_row) * SEG;
    const int nch = static_cast<int>(K - k0 >= SEG ? 8 : (K - k0) / 16);
    const uint8_t* qrow = q4 + n * ldq4 + k0 / 2;
    uint2 pk[8];
    if (nch == 8 && (reinterpret_cast<uintptr_t>(qrow) & 15) == 0) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint4 v = __ldg(reinterpret_cast<const uint4*>(qrow) + i);
        pk[2 * i] = make_uint2(v.x, v.y);
        pk[2 * i + 1] = make_uint2(v.z, v.w);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) pk[i] = i < nch ? __ldg(reinterpret_cast<const uint2*>(qrow) + i) : make_uint2(0, 0);
    }
    const int64_t srow = n * lds;
    uint4 t = make_uint4(0, 0, 0, 0);
    int64_t cur = -1;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (i >= nch) break;
      const int64_t e0 = k0 + 16 * i;
      const int64_t gi = e0 / group;
      if (gi != cur) {
        cur = gi;
        if constexpr (SDT == H3B_FP8_E4M3) t = lut[static_cast<const uint8_t*>(s_rel)[srow + gi]];
        else t = level_table(cb, scale_at<SDT>(s_rel, srow + gi));
      }
      const uint2 a = decode8(pk[i].x, t), b = decode8(pk[i].y, t);
      *reinterpret_cast<uint4*>(grid + n * ldg + e0) = make_uint4(a.x, a.y, b.x, b.y);
    }
  }
}

}  // namespace h3b
