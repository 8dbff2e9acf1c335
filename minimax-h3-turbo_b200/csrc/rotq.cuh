// Kernel KA: ConvRot rotation + per-token int8 quantisation (and the rotation-only variant).
//
// Reference semantics (h3turbo/h3/qlinear.py):
//   y32  = per-`convrot`-block x @ H, H = kron(H4, ..., H4) / sqrt(convrot)          _rot32 / hadamard_regular :44-115
//   amax = max |y32| over the whole row ("ck") or max |dt(y32)| ("eager")           _quantize_rows :278-287
//   xs   = max(amax / 127, 1e-30) (fp32); s = dt(xs), 0 -> finfo(dt).tiny           :288-290
//   q    = clamp(rint(dt(fp32(dt(y32)) / s)), -128, 127)                              :291-292
//   with input_act="swiglu": x <- dt(dt(silu(gate)) * up) first                       _swiglu :376-379
//
// Layout.  bf16/fp16: a thread owns TWO 16-element chunks ("lanes"), so every butterfly and quantiser FMA is a packed
// fp32x2 instruction with lane 0 in .x and lane 1 in .y.  In split mode both lanes are the same row, K/2 elements apart
// (K/32 threads per row; needs K to be a multiple of 32 x the threads of a ConvRot block so both lanes sit at the same
// position of their blocks); otherwise the lanes are the same chunk of two rows (a row pair, K/16 threads).  fp32
// activations: one chunk of one row per thread and the transform in fp64 -- exact for any fp32 input whose 256-block
// spans under ~21 binades, i.e. the reference's correctly rounded fp64 rotation.  An exchanged value is 8 bytes
// (float2 or double) either way.
// Inside a ConvRot block of CR = 4^n elements, element e has base-4 digits d0..d(n-1).  The chunk's 16 elements are
// digits d0, d1 (in registers); the CR/16 threads of a block hold digits d2, d3.  Stage A transforms d0, d1 in registers;
// a padded shared-memory exchange regroups the block so each thread holds all values of d2, d3 for a fixed (d0, d1);
// stage B transforms those.  The regular H4 butterfly is (H4 a)_i = S - 2 a_{3-i}, S = (a0 + a1) + (a2 + a3); the
// 1/sqrt(CR) normalisation (a power of two) is folded into the last stage, which is exact.
//
// Pipelining.  CTAs are persistent: each loops over row groups, and every thread loads its chunks of the NEXT group into
// registers before transforming the current one, so HBM reads overlap the arithmetic and the CTA-wide row-max barrier.
//
// Division: s is constant per row.  bf16: RNbf16(RN(b r)) with r = RN(1/s) equals RNbf16(RN(b / s)) for every pair of
// bf16 significands (checked exhaustively), so one multiply suffices.  fp16: r and one Markstein correction
// (q0 = RN(b r), e = b - q0 s exactly, q1 = RN(q0 + e r)) -- the correctly rounded quotient for every pair of fp16
// operands (checked exhaustively).  fp32 activations use the IEEE division.
// Rounding the dt quotient to an integer uses the fp32 magic constant 1.5 * 2^23 (round half-to-even), after clamping
// at 127 in the dt domain; the int8 code is the low byte of the sum's bit pattern.
#include <type_traits>

#include "h3b_common.cuh"

// Threads a CTA should at least have: row groups are added to a CTA until it reaches this (build-time tuning knob).
#ifndef H3B_ROTQ_MIN_THREADS
#define H3B_ROTQ_MIN_THREADS 128
#endif

namespace h3b {

enum { DT_BF16 = 0, DT_FP16 = 1, DT_FP32 = 2 };
enum { MODE_CK = 0, MODE_EAGER = 1, MODE_ROTATE = 2 };

// ------------------------------------------------------------------------------------------------ dtype helpers
template <int DT>
__device__ __forceinline__ float round_dt(float v) {
  if constexpr (DT == DT_BF16) return __bfloat162float(__float2bfloat16_rn(v));
  else if constexpr (DT == DT_FP16) return __half2float(__float2half_rn(v));
  else return v;
}
template <int DT>
__device__ __forceinline__ float tiny_dt() {
  return DT == DT_FP16 ? 6.103515625e-05f : 1.1754943508222875e-38f;  // torch.finfo(dt).tiny
}
// bf16x2 / fp16x2 bit pattern -> the two values as fp32 (exact, integer ops for bf16)
template <int DT>
__device__ __forceinline__ float2 unpack2(uint32_t w) {
  if constexpr (DT == DT_BF16) {
    return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
  } else {
    return __half22float2(*reinterpret_cast<const __half2*>(&w));
  }
}
// two fp32 values -> dt, packed (round to nearest even)
template <int DT>
__device__ __forceinline__ uint32_t pack2(float2 v) {
  if constexpr (DT == DT_BF16) {
    const __nv_bfloat162 h = __float22bfloat162_rn(v);
    return *reinterpret_cast<const uint32_t*>(&h);
  } else {
    const __half2 h = __float22half2_rn(v);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
}
// Packed clamp of the dt quotient before rounding.  bf16: |b / s| <= 127 (1 + 2^-8)^2 / (1 - 2^-24) < 128.5, so only
// the top needs a clamp (rint(127.5) = 128 -> 127); fp16 also clamps at -128 (an overflowed fp16 rotation can reach it).
template <int DT>
__device__ __forceinline__ uint32_t clamp_q2(uint32_t w) {
  if constexpr (DT == DT_BF16) {
    const __nv_bfloat162 r = __hmin2(*reinterpret_cast<const __nv_bfloat162*>(&w), __float2bfloat162_rn(127.0f));
    return *reinterpret_cast<const uint32_t*>(&r);
  } else {
    const __half2 r = __hmax2(__hmin2(*reinterpret_cast<const __half2*>(&w), __float2half2_rn(127.0f)), __float2half2_rn(-128.0f));
    return *reinterpret_cast<const uint32_t*>(&r);
  }
}
// Round two fp32 values to the nearest bf16 (ties to even), returned as fp32, on the FMA pipe: Veltkamp splitting with
// C = 2^16 + 1 (g = v C, d = v - g, h = g + d; each step rounded once, never contracted).  Equal to round-to-nearest-even
// for every fp32 significand whenever all intermediates are normal and finite, i.e. for |v| in [2^-125, 2^111) (checked
// exhaustively by tests/test_numerics.py); callers use it only below 2^100 -- values under 2^-110 quantise to code 0
// whatever their last bf16 bit.
__device__ __forceinline__ float2 rne_bf16_fma(float2 v) {
  const float2 g = __fmul2_rn(v, make_float2(65537.0f, 65537.0f));
  const float2 d = __ffma2_rn(g, make_float2(-1.0f, -1.0f), v);
  return __fadd2_rn(g, d);
}
constexpr float VELTKAMP_MAX = 1.2676506002282294e30f;  // 2^100

// max(a, b, c), NaN operands ignored like fmaxf (one three-input instruction on sm_100)
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}
// round half-to-even and saturate to [-128, 127]; the code in the low byte
__device__ __forceinline__ uint32_t sat_s8(float v) {
  int r;
  asm("cvt.rni.sat.s8.f32 %0, %1;" : "=r"(r) : "f"(v));
  return static_cast<uint32_t>(r);
}
constexpr float RINT_MAGIC = 12582912.0f;  // 1.5 * 2^23: x + M rounds x to an integer (half-to-even) for |x| < 2^22

// silu(gate) * up in dt, as torch computes it: x / (1 + exp(-x)) in fp32, rounded to dt; the product of the two dt
// values in fp32, rounded to dt.
template <int DT>
__device__ __forceinline__ float swiglu1(float g, float u) {
  const float sl = round_dt<DT>(g / (1.0f + expf(-g)));
  return round_dt<DT>(sl * u);
}

// ------------------------------------------------------------------------------------------------ lanes
// A thread's inputs: L lanes (2 for bf16/fp16, 1 for fp32) of 16 elements; each lane is (row offset, column offset)
// from the thread's (row0, col): split mode (0, l K/2), pair mode (l, 0).
template <int DT, bool SW>
struct Raw {
  static constexpr int L = DT == DT_FP32 ? 1 : 2;
  static constexpr int ESZ = DT == DT_FP32 ? 4 : 2;      // bytes per element
  static constexpr int V16 = ESZ;                        // uint4 per 16 elements (32 or 64 bytes)
  uint4 u[L * V16 * (SW ? 2 : 1)];
};

template <int DT, bool SW, bool SPLIT>
__device__ __forceinline__ void load_raw(Raw<DT, SW>& raw, const void* x, int64_t ldx, int64_t row0, int M, int64_t col,
                                         int K) {
  using RW = Raw<DT, SW>;
#pragma unroll
  for (int l = 0; l < RW::L; ++l) {
    const int64_t row = row0 + (SPLIT ? 0 : l);
    const int64_t c0 = col + (SPLIT ? l * (K / 2) : 0);
    const bool valid = row < M;
    const char* base = static_cast<const char*>(x) + static_cast<size_t>(valid ? row : 0) * static_cast<size_t>(ldx) * RW::ESZ;
#pragma unroll
    for (int h = 0; h < (SW ? 2 : 1); ++h) {
      const uint4* ptr = reinterpret_cast<const uint4*>(base + static_cast<size_t>(c0 + h * K) * RW::ESZ);
#pragma unroll
      for (int i = 0; i < RW::V16; ++i)
        raw.u[(l * (SW ? 2 : 1) + h) * RW::V16 + i] = valid ? __ldg(ptr + i) : make_uint4(0, 0, 0, 0);
    }
  }
}

// lane l of `raw` -> 16 fp32 values (SwiGLU applied)
template <int DT, bool SW>
__device__ __forceinline__ void lane_f32(const Raw<DT, SW>& raw, int l, float (&v)[16]) {
  using RW = Raw<DT, SW>;
  float u[SW ? 16 : 1];
#pragma unroll
  for (int h = 0; h < (SW ? 2 : 1); ++h) {
    float* dst = h == 0 ? v : u;
    const uint4* src = raw.u + (l * (SW ? 2 : 1) + h) * RW::V16;
    if constexpr (DT == DT_FP32) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        dst[4 * i] = __uint_as_float(src[i].x); dst[4 * i + 1] = __uint_as_float(src[i].y);
        dst[4 * i + 2] = __uint_as_float(src[i].z); dst[4 * i + 3] = __uint_as_float(src[i].w);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const uint32_t w[4] = {src[i].x, src[i].y, src[i].z, src[i].w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 f = unpack2<DT>(w[k]);
          dst[8 * i + 2 * k] = f.x;
          dst[8 * i + 2 * k + 1] = f.y;
        }
      }
    }
  }
  if constexpr (SW) {
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = swiglu1<DT>(v[i], u[i]);
  }
}

// ------------------------------------------------------------------------------------------------ butterflies
// float2: two rows in lockstep (packed fp32x2); double: one fp32-input row in fp64.
__device__ __forceinline__ void h4(float2& a0, float2& a1, float2& a2, float2& a3, float sc) {
  float2 s = __fadd2_rn(__fadd2_rn(a0, a1), __fadd2_rn(a2, a3));
  if (sc != 1.0f) s = __fmul2_rn(s, make_float2(sc, sc));
  const float2 m2 = make_float2(-2.f * sc, -2.f * sc);
  const float2 y0 = __ffma2_rn(m2, a3, s), y1 = __ffma2_rn(m2, a2, s);
  const float2 y2 = __ffma2_rn(m2, a1, s), y3 = __ffma2_rn(m2, a0, s);
  a0 = y0; a1 = y1; a2 = y2; a3 = y3;
}
__device__ __forceinline__ void h4(double& a0, double& a1, double& a2, double& a3, float sc) {
  const double s = ((a0 + a1) + (a2 + a3)) * static_cast<double>(sc);
  const double m2 = -2.0 * static_cast<double>(sc);
  const double y0 = fma(m2, a3, s), y1 = fma(m2, a2, s), y2 = fma(m2, a1, s), y3 = fma(m2, a0, s);
  a0 = y0; a1 = y1; a2 = y2; a3 = y3;
}

// ------------------------------------------------------------------------------------------------ exchange layout
// Per ConvRot block of G threads: owner t's 16 values (8 bytes each) in row t of a [G][18] array of 8-byte slots
// (144-byte rows: 16-byte aligned, and consecutive rows shift by one 16-byte bank group, so both the owners' 16-byte
// stores and the readers' 8-byte loads are conflict-free).  Blocks are g x 144 + 64 bytes apart (a half-bank shift).
constexpr int XROW = 18;                       // 8-byte slots per owner row
__host__ __device__ constexpr int xgrp(int g) { return g * XROW + 8; }  // 8-byte slots per ConvRot block of g threads
// Code regroup: 16 chunks of 16 x (A, B) byte pairs, chunk stride 48 bytes (conflict-free 16-byte reads).
constexpr int CSTRIDE = 48;

// ------------------------------------------------------------------------------------------------ the kernel
// blockDim.x = tpr * groups_per_cta; tpr = K / 32 (split) or K / 16 threads per row group; a row group is 1 row (split,
// fp32) or 2 rows (pair).  Persistent: group g = blockIdx.x * groups_per_cta + p, then += gridDim.x * groups_per_cta.
template <int DT, int CR, int MODE, bool SW, bool SPLIT>
__global__ void __launch_bounds__(SPLIT ? 512 : 1024) rotq_kernel(const void* __restrict__ x, int64_t ldx, int M, int K,
                                                                   int tpr, int pairs, int8_t* __restrict__ q, int64_t ldq,
                                                                   float* __restrict__ xs_out, void* __restrict__ y_out,
                                                                   int y_dtype, int64_t ldy) {
  constexpr int G = CR >= 256 ? 16 : (CR == 64 ? 4 : 1);  // threads per ConvRot block
  constexpr float SCALE = CR == 256 ? 0.0625f : CR == 64 ? 0.125f : CR == 16 ? 0.25f : 0.5f;
  constexpr int L = DT == DT_FP32 ? 1 : 2;                // lanes per thread
  constexpr int RG = (SPLIT || L == 1) ? 1 : 2;           // rows per row group
  using T = typename std::conditional<DT == DT_FP32, double, float2>::type;
  extern __shared__ __align__(16) unsigned char rotq_smem[];
  unsigned int* rowmax = reinterpret_cast<unsigned int*>(rotq_smem);  // [3 slots][pairs * RG]
  T* xbuf = reinterpret_cast<T*>(rotq_smem + 16 * ((3 * pairs * RG * 4 + 15) / 16));

  const int tid = threadIdx.x;
  const int p = tid / tpr, tr = tid - p * tpr;
  const int t = tr % G;                                  // thread within the ConvRot block
  const int64_t col = 16ll * tr;                         // lane 0's first element
  const int64_t blk0 = static_cast<int64_t>(tr - t) * 16;  // first element of lane 0's ConvRot block
  T* gbuf = xbuf + static_cast<size_t>((tid - t) / G) * xgrp(G);
  const int64_t ngroups = (static_cast<int64_t>(M) + RG - 1) / RG;
  const int64_t gstep = static_cast<int64_t>(gridDim.x) * pairs;
  const int64_t lane_col = SPLIT ? K / 2 : 0;            // lane 1's column offset

  auto elem = [&](int i) -> int64_t {  // lane-0 element (within the row) of register i after the transform
    if constexpr (G == 16) return blk0 + t + 16 * i;
    else if constexpr (G == 4) return blk0 + 16 * (i >> 2) + 4 * t + (i & 3);
    else return col + i;
  };

  for (int s = tid; s < 3 * pairs * RG; s += blockDim.x) rowmax[s] = 0u;
  __syncthreads();

  int64_t g = static_cast<int64_t>(blockIdx.x) * pairs + p;
  Raw<DT, SW> raw;
  load_raw<DT, SW, SPLIT>(raw, x, ldx, g * RG, M, col, K);
  int slot = 0;
  for (int64_t gbase = static_cast<int64_t>(blockIdx.x) * pairs; gbase < ngroups; gbase += gstep, g += gstep) {
    const int64_t row0 = g * RG;
    // ---- this group's values, then prefetch the next group's raw inputs into the same registers
    T v[16];
    if constexpr (DT == DT_FP32) {
      float f[16];
      lane_f32<DT, SW>(raw, 0, f);
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] = static_cast<double>(f[i]);
    } else if constexpr (!SW) {
#pragma unroll
      for (int i = 0; i < 2; ++i) {  // words of lane 0 (raw.u[0..1]) and lane 1 (raw.u[2..3]), 2 elements per word
        const uint32_t wa[4] = {raw.u[i].x, raw.u[i].y, raw.u[i].z, raw.u[i].w};
        const uint32_t wb[4] = {raw.u[2 + i].x, raw.u[2 + i].y, raw.u[2 + i].z, raw.u[2 + i].w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 a = unpack2<DT>(wa[k]), b = unpack2<DT>(wb[k]);
          v[8 * i + 2 * k] = make_float2(a.x, b.x);
          v[8 * i + 2 * k + 1] = make_float2(a.y, b.y);
        }
      }
    } else {
      float f[16];
      lane_f32<DT, SW>(raw, 0, f);
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i].x = f[i];
      lane_f32<DT, SW>(raw, 1, f);
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i].y = f[i];
    }
    if (gbase + gstep < ngroups) load_raw<DT, SW, SPLIT>(raw, x, ldx, (g + gstep) * RG, M, col, K);

    // ---- stage A: digits d0 (register bits 0-1) and d1 (register bits 2-3)
    if constexpr (CR == 4) {
#pragma unroll
      for (int a = 0; a < 4; ++a) h4(v[4 * a], v[4 * a + 1], v[4 * a + 2], v[4 * a + 3], SCALE);
    } else {
#pragma unroll
      for (int a = 0; a < 4; ++a) h4(v[4 * a], v[4 * a + 1], v[4 * a + 2], v[4 * a + 3], 1.0f);
#pragma unroll
      for (int d = 0; d < 4; ++d) h4(v[d], v[d + 4], v[d + 8], v[d + 12], CR == 16 ? SCALE : 1.0f);
    }
    // ---- exchange + stage B (digits d2, d3 across the G threads of the block)
    if constexpr (G > 1) {
      float4* wr = reinterpret_cast<float4*>(gbuf + t * XROW);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if constexpr (DT == DT_FP32) {
          wr[i] = make_float4(__int_as_float(__double2loint(v[2 * i])), __int_as_float(__double2hiint(v[2 * i])),
                              __int_as_float(__double2loint(v[2 * i + 1])), __int_as_float(__double2hiint(v[2 * i + 1])));
        } else {
          wr[i] = make_float4(v[2 * i].x, v[2 * i].y, v[2 * i + 1].x, v[2 * i + 1].y);
        }
      }
      __syncwarp();
      if constexpr (G == 16) {
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = gbuf[j * XROW + t];  // owner j's element r = t (register j = d2 + 4 d3)
        __syncwarp();
#pragma unroll
        for (int a = 0; a < 4; ++a) h4(v[4 * a], v[4 * a + 1], v[4 * a + 2], v[4 * a + 3], 1.0f);
#pragma unroll
        for (int d = 0; d < 4; ++d) h4(v[d], v[d + 4], v[d + 8], v[d + 12], SCALE);
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
#pragma unroll
          for (int d = 0; d < 4; ++d) v[4 * j + d] = gbuf[j * XROW + 4 * t + d];  // owner j's r = 4t + d0
        }
        __syncwarp();
#pragma unroll
        for (int d = 0; d < 4; ++d) h4(v[d], v[d + 4], v[d + 8], v[d + 12], SCALE);
      }
    }

    if constexpr (MODE == MODE_ROTATE) {
      const size_t ysz = y_dtype == H3B_FP32 ? 4 : 2;
#pragma unroll
      for (int l = 0; l < L; ++l) {
        const int64_t row = row0 + (SPLIT ? 0 : l);
        if (row >= M) continue;
        char* yr = static_cast<char*>(y_out) + static_cast<size_t>(row) * static_cast<size_t>(ldy) * ysz;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float val;
          if constexpr (DT == DT_FP32) val = static_cast<float>(v[i]);
          else val = l == 0 ? v[i].x : v[i].y;
          const int64_t e = elem(i) + l * lane_col;
          if (y_dtype == H3B_BF16) reinterpret_cast<__nv_bfloat16*>(yr)[e] = __float2bfloat16_rn(val);
          else if (y_dtype == H3B_FP16) reinterpret_cast<__half*>(yr)[e] = __float2half_rn(val);
          else reinterpret_cast<float*>(yr)[e] = val;
        }
      }
      continue;
    } else {
      // ---- dt rounding (b, kept as fp32 values) and the local absmax
      float2 b2[16];       // bf16/fp16: dt(y) of (lane 0, lane 1)
      uint32_t bw[16];     // fp32 activations: the fp32 value of the single lane
      float mA = 0.f, mB = 0.f;
      if constexpr (DT == DT_FP32) {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float y = static_cast<float>(v[i]);
          bw[i] = __float_as_uint(y);
          mA = fmaxf(mA, fabsf(y));
        }
      } else if constexpr (DT == DT_BF16 && MODE == MODE_CK) {
        if constexpr (RG == 1) {  // split: both lanes are the same row
#pragma unroll
          for (int i = 0; i < 16; ++i) mA = max3f(mA, fabsf(v[i].x), fabsf(v[i].y));
        } else {
#pragma unroll
          for (int i = 0; i < 16; i += 2) {
            mA = max3f(mA, fabsf(v[i].x), fabsf(v[i + 1].x));
            mB = max3f(mB, fabsf(v[i].y), fabsf(v[i + 1].y));
          }
        }
        if (fmaxf(mA, mB) < VELTKAMP_MAX) {
#pragma unroll
          for (int i = 0; i < 16; ++i) b2[i] = rne_bf16_fma(v[i]);
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) b2[i] = unpack2<DT>(pack2<DT>(v[i]));
        }
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          b2[i] = unpack2<DT>(pack2<DT>(v[i]));
          const float2 src = MODE == MODE_CK ? v[i] : b2[i];
          mA = fmaxf(mA, fabsf(src.x));
          mB = fmaxf(mB, fabsf(src.y));
        }
      }
      if constexpr (RG == 1 && L == 2) mA = fmaxf(mA, mB);  // split: both lanes are the same row
      unsigned int* rm = rowmax + slot * pairs * RG + p * RG;
      if ((tpr & 31) == 0) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          mA = fmaxf(mA, __shfl_xor_sync(0xffffffffu, mA, o));
          if (RG == 2) mB = fmaxf(mB, __shfl_xor_sync(0xffffffffu, mB, o));
        }
        if ((tid & 31) == 0) {
          atomicMax(&rm[0], __float_as_uint(mA));
          if (RG == 2) atomicMax(&rm[RG - 1], __float_as_uint(mB));
        }
      } else {
        atomicMax(&rm[0], __float_as_uint(mA));
        if (RG == 2) atomicMax(&rm[RG - 1], __float_as_uint(mB));
      }
      __syncthreads();
      // slot (slot + 2) % 3 was last read before the previous barrier and is next written after the next one
      {
        const int clr = slot == 0 ? 2 : slot - 1;
        for (int s2 = tid; s2 < pairs * RG; s2 += blockDim.x) rowmax[clr * pairs * RG + s2] = 0u;
      }
      const float amaxA = __uint_as_float(rm[0]), amaxB = __uint_as_float(rm[RG - 1]);
      slot = slot == 2 ? 0 : slot + 1;
      const float xsA = fmaxf(__fdiv_rn(amaxA, 127.0f), 1e-30f);
      const float xsB = RG == 2 ? fmaxf(__fdiv_rn(amaxB, 127.0f), 1e-30f) : xsA;
      float sA = round_dt<DT>(xsA);
      if (sA == 0.f) sA = tiny_dt<DT>();
      float sB = sA;
      if (RG == 2) {
        sB = round_dt<DT>(xsB);
        if (sB == 0.f) sB = tiny_dt<DT>();
      }
      if (tr == 0) {
        if (row0 < M) xs_out[row0] = xsA;
        if (RG == 2 && row0 + 1 < M) xs_out[row0 + 1] = xsB;
      }

      // ---- quantise: code = sat_s8(rint(dt(RN(b / s)))); cpair(i) = lane 0 code | lane 1 code << 8
      unsigned char* cbuf = reinterpret_cast<unsigned char*>(gbuf);  // G > 1: regroup area (the exchange is done)
      // (lane 0, lane 1) byte pairs by element e of the block; the 16 elements of chunk c at c * CSTRIDE bytes.
      // G = 16: register i is element t + 16 i (chunk i, slot t); G = 4: 16 (i >> 2) + 4 t + (i & 3).
      unsigned char* cb_t = cbuf + (G == 16 ? 2 * t : 8 * t);
      uint32_t wA[4] = {0, 0, 0, 0}, wB[4] = {0, 0, 0, 0};
      auto put = [&](int i, uint32_t cpair) {
        if constexpr (G == 1) {  // own 16 contiguous elements: pack in registers
          wA[i >> 2] |= (cpair & 0xFFu) << (8 * (i & 3));
          wB[i >> 2] |= ((cpair >> 8) & 0xFFu) << (8 * (i & 3));
        } else if constexpr (G == 16) {
          *reinterpret_cast<uint16_t*>(cb_t + i * CSTRIDE) = static_cast<uint16_t>(cpair);
        } else {
          *reinterpret_cast<uint16_t*>(cb_t + (i >> 2) * CSTRIDE + 2 * (i & 3)) = static_cast<uint16_t>(cpair);
        }
      };
      if constexpr (DT == DT_FP32) {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float qv = fminf(__fdiv_rn(__uint_as_float(bw[i]), sA), 127.0f);
          qv = fmaxf(qv, -128.0f);
          put(i, __float_as_uint(qv + RINT_MAGIC) & 0xFFu);
        }
      } else {
        const float2 nS2 = make_float2(-sA, -sB);
        const float rA = __frcp_rn(sA);
        const float2 R2 = make_float2(rA, RG == 2 ? __frcp_rn(sB) : rA);
        const float2 MG = make_float2(RINT_MAGIC, RINT_MAGIC);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float2 b = b2[i];
          const float2 q0 = __fmul2_rn(b, R2);
          float2 qd;
          if constexpr (DT == DT_BF16) {
            // RNbf16(q0) is RNbf16(b / s); the saturating conversion rounds half-to-even and clamps to [-128, 127]
            // (on the XU pipe, which the rest of the kernel leaves idle)
            qd = rne_bf16_fma(q0);
            put(i, __byte_perm(sat_s8(qd.x), sat_s8(qd.y), 0x0040));
          } else {
            const float2 e = __ffma2_rn(q0, nS2, b);
            qd = unpack2<DT>(clamp_q2<DT>(pack2<DT>(__ffma2_rn(e, R2, q0))));  // dt(RN(b / s)), clamped
            const float2 rr = __fadd2_rn(qd, MG);  // rint, half-to-even
            put(i, __byte_perm(__float_as_uint(rr.x), __float_as_uint(rr.y), 0x0040));
          }
        }
      }
      if constexpr (G > 1) {
        __syncwarp();
        const uint4* rd = reinterpret_cast<const uint4*>(cbuf + t * CSTRIDE);
        const uint4 u0 = rd[0], u1 = rd[1];
        const uint32_t w8[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          wA[w] = __byte_perm(w8[2 * w], w8[2 * w + 1], 0x6420);
          wB[w] = __byte_perm(w8[2 * w], w8[2 * w + 1], 0x7531);
        }
        __syncwarp();
      }
      // ---- store: lane 0 -> (row0, col), lane 1 -> split: (row0, col + K/2), pair: (row0 + 1, col)
      if (row0 < M) *reinterpret_cast<uint4*>(q + row0 * ldq + col) = make_uint4(wA[0], wA[1], wA[2], wA[3]);
      if constexpr (L == 2) {
        const int64_t row1 = row0 + (SPLIT ? 0 : 1);
        if (row1 < M) *reinterpret_cast<uint4*>(q + row1 * ldq + col + lane_col) = make_uint4(wB[0], wB[1], wB[2], wB[3]);
      }
    }
  }
}

// ------------------------------------------------------------------------------------------------ launcher
template <int DT, int CR, int MODE, bool SW, bool SPLIT>
static int launch_t(const void* x, int64_t ldx, int64_t M, int64_t K, int8_t* q, int64_t ldq, float* xs, void* y,
                    int ydt, int64_t ldy, cudaStream_t st) {
  constexpr int L = DT == DT_FP32 ? 1 : 2;
  constexpr int RG = (SPLIT || L == 1) ? 1 : 2;
  constexpr int G = CR >= 256 ? 16 : (CR == 64 ? 4 : 1);
  constexpr int MAXT = SPLIT ? 512 : 1024;
  using T = typename std::conditional<DT == DT_FP32, double, float2>::type;
  const int tpr = static_cast<int>(SPLIT ? K / 32 : K / 16);
  int pairs = tpr >= H3B_ROTQ_MIN_THREADS ? 1 : (H3B_ROTQ_MIN_THREADS + tpr - 1) / tpr;
  while (pairs > 1 && pairs * tpr > MAXT) --pairs;
  const int threads = pairs * tpr;
  const size_t nblk = G > 1 ? static_cast<size_t>(threads) / G : 0;  // no exchange for blocks inside one thread
  const size_t smem = 16 * ((3 * pairs * RG * 4 + 15) / 16) + nblk * xgrp(G) * sizeof(T);
  auto kern = rotq_kernel<DT, CR, MODE, SW, SPLIT>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(rotq)");
  }
  cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);  // several CTAs' exchange buffers
  int dev = 0, sms = 148, per_sm = 1;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, smem);
  if (e != cudaSuccess || per_sm < 1) per_sm = 1;
  const int64_t groups = (M + RG - 1) / RG;
  const int64_t want = (groups + pairs - 1) / pairs;
  const int64_t cap = static_cast<int64_t>(sms) * per_sm;
  const int blocks = static_cast<int>(want < cap ? want : cap);
  kern<<<blocks, threads, smem, st>>>(x, ldx, static_cast<int>(M), static_cast<int>(K), tpr, pairs, q, ldq, xs, y, ydt, ldy);
  return check_launch("rotq_kernel");
}

// split mode when both lanes of a thread can be the same row (K a multiple of 32 x the block's threads, <= 512 threads)
template <int DT, int CR, int MODE, bool SW>
static int launch_split(const void* x, int64_t ldx, int64_t M, int64_t K, int8_t* q, int64_t ldq, float* xs, void* y,
                        int ydt, int64_t ldy, cudaStream_t st) {
  constexpr int G = CR >= 256 ? 16 : (CR == 64 ? 4 : 1);
  if constexpr (DT != DT_FP32) {
    if (K % (32 * G) == 0 && K / 32 <= 512) return launch_t<DT, CR, MODE, SW, true>(x, ldx, M, K, q, ldq, xs, y, ydt, ldy, st);
  }
  return launch_t<DT, CR, MODE, SW, false>(x, ldx, M, K, q, ldq, xs, y, ydt, ldy, st);
}

template <int DT, int MODE, bool SW>
static int launch_cr(int cr, const void* x, int64_t ldx, int64_t M, int64_t K, int8_t* q, int64_t ldq, float* xs, void* y,
                     int ydt, int64_t ldy, cudaStream_t st) {
  switch (cr) {
    case 4: return launch_split<DT, 4, MODE, SW>(x, ldx, M, K, q, ldq, xs, y, ydt, ldy, st);
    case 16: return launch_split<DT, 16, MODE, SW>(x, ldx, M, K, q, ldq, xs, y, ydt, ldy, st);
    case 64: return launch_split<DT, 64, MODE, SW>(x, ldx, M, K, q, ldq, xs, y, ydt, ldy, st);
    case 256: return launch_split<DT, 256, MODE, SW>(x, ldx, M, K, q, ldq, xs, y, ydt, ldy, st);
    default: return fail(H3B_ERR_UNSUPPORTED, "convrot must be 4, 16, 64 or 256 on the b200 backend");
  }
}

template <int MODE, bool SW>
static int launch_dt(int dt, int cr, const void* x, int64_t ldx, int64_t M, int64_t K, int8_t* q, int64_t ldq, float* xs,
                     void* y, int ydt, int64_t ldy, cudaStream_t st) {
  switch (dt) {
    case H3B_BF16: return launch_cr<DT_BF16, MODE, SW>(cr, x, ldx, M, K, q, ldq, xs, y, ydt, ldy, st);
    case H3B_FP16: return launch_cr<DT_FP16, MODE, SW>(cr, x, ldx, M, K, q, ldq, xs, y, ydt, ldy, st);
    case H3B_FP32: return launch_cr<DT_FP32, MODE, SW>(cr, x, ldx, M, K, q, ldq, xs, y, ydt, ldy, st);
    default: return fail(H3B_ERR_ARG, "activation dtype must be bf16, fp16 or fp32");
  }
}

int rotq_launch(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx, int convrot, int swiglu, int mode,
                int8_t* q, int64_t ldq, float* xs, void* y, int y_dtype, int64_t ldy, cudaStream_t st) {
  if (mode == MODE_ROTATE) return launch_dt<MODE_ROTATE, false>(x_dtype, convrot, x, ldx, M, K, q, ldq, xs, y, y_dtype, ldy, st);
  if (mode == MODE_CK)
    return swiglu ? launch_dt<MODE_CK, true>(x_dtype, convrot, x, ldx, M, K, q, ldq, xs, y, y_dtype, ldy, st)
                  : launch_dt<MODE_CK, false>(x_dtype, convrot, x, ldx, M, K, q, ldq, xs, y, y_dtype, ldy, st);
  return swiglu ? launch_dt<MODE_EAGER, true>(x_dtype, convrot, x, ldx, M, K, q, ldq, xs, y, y_dtype, ldy, st)
                : launch_dt<MODE_EAGER, false>(x_dtype, convrot, x, ldx, M, K, q, ldq, xs, y, y_dtype, ldy, st);
}

}  // namespace h3b
