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
// Rounding to dt uses the hardware round-to-nearest-even pack (cvt.rn.bf16x2.f32 / f16x2).  bf16 codes: the packed
// quotient goes straight to integers (cvt.rni.s32.bf16, half-to-even) and a saturating byte pack (cvt.pack.sat.s8);
// fp16 and fp32: the fp32 magic constant 1.5 * 2^23 rounds half-to-even after a clamp in the dt domain, and the code is
// the low byte of the sum's bit pattern.
#include <mutex>
#include <type_traits>

#include "h3b_common.cuh"
#include "rmsmod.cuh"

// Threads a CTA should at least have: row groups are added to a CTA until it reaches this (build-time tuning knob).
#ifndef H3B_ROTQ_MIN_THREADS
#define H3B_ROTQ_MIN_THREADS 128
#endif

namespace h3b {

enum { DT_BF16 = 0, DT_FP16 = 1, DT_FP32 = 2 };

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
__device__ __forceinline__ float2 rnd_bf16x2(float2 v) { return unpack2<DT_BF16>(pack2<DT_BF16>(v)); }

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
// max(a, b, c), NaN operands ignored like fmaxf (one three-input instruction on sm_100)
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}
constexpr float RINT_MAGIC = 12582912.0f;  // 1.5 * 2^23: x + M rounds x to an integer (half-to-even) for |x| < 2^22

// Codes of a bf16 pair of quotients (element 0 in the low half): each half rounded half-to-even to an integer
// (cvt.rni.s32.bf16; NaN -> 0), saturated to [-128, 127] and packed as bytes: code0 | code1 << 8 | c << 16.
__device__ __forceinline__ uint32_t codes2_bf16(uint32_t qb, uint32_t c) {
  uint32_t d;
  asm("{\n\t.reg .b16 lo, hi;\n\t.reg .s32 k0, k1;\n\tmov.b32 {lo, hi}, %1;\n\tcvt.rni.s32.bf16 k0, lo;\n\t"
      "cvt.rni.s32.bf16 k1, hi;\n\tcvt.pack.sat.s8.s32.b32 %0, k1, k0, %2;\n\t}"
      : "=r"(d) : "r"(qb), "r"(c));
  return d;
}
// Codes of four elements given as the low (HI = false) or high halves of four bf16 pairs, the same rounding and
// saturation: c0 | c1 << 8 | c2 << 16 | c3 << 24.
#define H3B_CODES4_ASM(H)                                                                                     \
  "{\n\t.reg .b16 a0, a1, a2, a3, b0, b1, b2, b3;\n\t.reg .s32 k0, k1, k2, k3, t;\n\t"                       \
  "mov.b32 {a0, b0}, %1;\n\tmov.b32 {a1, b1}, %2;\n\tmov.b32 {a2, b2}, %3;\n\tmov.b32 {a3, b3}, %4;\n\t"      \
  "cvt.rni.s32.bf16 k0, " H "0;\n\tcvt.rni.s32.bf16 k1, " H "1;\n\tcvt.rni.s32.bf16 k2, " H "2;\n\t"            \
  "cvt.rni.s32.bf16 k3, " H "3;\n\tcvt.pack.sat.s8.s32.b32 t, k3, k2, 0;\n\tcvt.pack.sat.s8.s32.b32 %0, k1, k0, t;\n\t}"
template <bool HI>
__device__ __forceinline__ uint32_t codes4_bf16(uint32_t p0, uint32_t p1, uint32_t p2, uint32_t p3) {
  uint32_t d;
  if constexpr (HI) asm(H3B_CODES4_ASM("b") : "=r"(d) : "r"(p0), "r"(p1), "r"(p2), "r"(p3));
  else asm(H3B_CODES4_ASM("a") : "=r"(d) : "r"(p0), "r"(p1), "r"(p2), "r"(p3));
  return d;
}
#undef H3B_CODES4_ASM

// silu(gate) * up in dt, as torch computes it: x / (1 + exp(-x)) in fp32, rounded to dt; the product of the two dt
// values in fp32, rounded to dt.
template <int DT>
__device__ __forceinline__ float swiglu1(float g, float u) {
  const float sl = round_dt<DT>(g / (1.0f + expf(-g)));
  return round_dt<DT>(sl * u);
}
// The same for bf16, on (lane 0, lane 1) pairs.  silu's quotient matters only through its rounding to bf16, so it is
// taken from __fdividef (within 2 ulp of g / d for d in [2^-126, 2^126]) unless that result lies within 4 ulp of a bf16
// rounding midpoint (low 16 bits in [0x7FFC, 0x8004]) or g is outside (-87, 1e30) (d beyond 2^125, g infinite or NaN):
// then both the approximation and the IEEE quotient RN(g / d) (within 0.5 ulp of g / d) round to the same bf16 value, or
// the IEEE division is taken.  Every bf16 gate value is checked against torch's silu by tests/test_swiglu_gpu.py.
__device__ __forceinline__ float silu_quot_bf16(float g, float d) {
  float qt = __fdividef(g, d);
  if (!(g > -87.0f && g < 1.0e30f) || ((__float_as_uint(qt) & 0xFFFFu) - 0x7FFCu) < 9u) qt = __fdiv_rn(g, d);
  return qt;
}
__device__ __forceinline__ float2 swiglu2_bf16(float2 g, float2 u) {
  const float2 d = __fadd2_rn(make_float2(1.0f, 1.0f), make_float2(expf(-g.x), expf(-g.y)));
  const float2 sl = rnd_bf16x2(make_float2(silu_quot_bf16(g.x, d.x), silu_quot_bf16(g.y, d.y)));
  return rnd_bf16x2(__fmul2_rn(sl, u));
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
    // a row past the end reads the last row instead: its values only ever reach its own row group's scale slot and
    // stores, which are skipped for rows past the end
    const int64_t row = row0 + (SPLIT ? 0 : l) < M ? row0 + (SPLIT ? 0 : l) : M - 1;
    const int64_t c0 = col + (SPLIT ? l * (K / 2) : 0);
    const char* base = static_cast<const char*>(x) + static_cast<size_t>(row) * static_cast<size_t>(ldx) * RW::ESZ;
#pragma unroll
    for (int h = 0; h < (SW ? 2 : 1); ++h) {
      const uint4* ptr = reinterpret_cast<const uint4*>(base + static_cast<size_t>(c0 + h * K) * RW::ESZ);
#pragma unroll
      for (int i = 0; i < RW::V16; ++i) raw.u[(l * (SW ? 2 : 1) + h) * RW::V16 + i] = __ldg(ptr + i);
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

// Both lanes' 16 SwiGLU values as (lane 0, lane 1) pairs.  raw.u: lane 0 gate [0, 1], lane 0 up [2, 3], lane 1 gate
// [4, 5], lane 1 up [6, 7] (16-bit activations).
template <int DT>
__device__ __forceinline__ void swiglu_lanes(const Raw<DT, true>& raw, float2 (&v)[16]) {
  if constexpr (DT == DT_BF16) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const uint4 ga = raw.u[i], ua = raw.u[2 + i], gb = raw.u[4 + i], ub = raw.u[6 + i];
      const uint32_t g0[4] = {ga.x, ga.y, ga.z, ga.w}, u0[4] = {ua.x, ua.y, ua.z, ua.w};
      const uint32_t g1[4] = {gb.x, gb.y, gb.z, gb.w}, u1[4] = {ub.x, ub.y, ub.z, ub.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 a = unpack2<DT>(g0[k]), b = unpack2<DT>(g1[k]), c = unpack2<DT>(u0[k]), e = unpack2<DT>(u1[k]);
        v[8 * i + 2 * k] = swiglu2_bf16(make_float2(a.x, b.x), make_float2(c.x, e.x));
        v[8 * i + 2 * k + 1] = swiglu2_bf16(make_float2(a.y, b.y), make_float2(c.y, e.y));
      }
    }
  } else {
    float f[16];
    lane_f32<DT, true>(raw, 0, f);
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i].x = f[i];
    lane_f32<DT, true>(raw, 1, f);
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i].y = f[i];
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
      swiglu_lanes<DT>(raw, v);
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
        if constexpr (RG == 1) {  // split: both lanes are the same row; four independent chains
          float m4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int i = 0; i < 16; ++i) m4[i & 3] = max3f(m4[i & 3], fabsf(v[i].x), fabsf(v[i].y));
          mA = max3f(m4[0], m4[1], fmaxf(m4[2], m4[3]));
        } else {
#pragma unroll
          for (int i = 0; i < 16; i += 2) {
            mA = max3f(mA, fabsf(v[i].x), fabsf(v[i + 1].x));
            mB = max3f(mB, fabsf(v[i].y), fabsf(v[i + 1].y));
          }
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) b2[i] = unpack2<DT>(pack2<DT>(v[i]));
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

      // ---- quantise: code = sat(rint(dt(RN(b / s)))); cpair(i) = lane 0 code | lane 1 code << 8
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
          if constexpr (DT == DT_BF16) {
            // RNbf16(q0) is RNbf16(b / s) (the hardware pack rounds to nearest even); the codes round it half-to-even
            // to an integer and saturate to [-128, 127]
            put(i, codes2_bf16(pack2<DT>(q0), 0u));
          } else {
            const float2 e = __ffma2_rn(q0, nS2, b);
            const float2 qd = unpack2<DT>(clamp_q2<DT>(pack2<DT>(__ffma2_rn(e, R2, q0))));  // dt(RN(b / s)), clamped
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

// ------------------------------------------------------------------------------------------------ warp-per-row kernel
// bf16 activations, ConvRot 256, K a multiple of 256, quantise modes.  One warp owns a whole row.  Pass p transforms
// chunk pair c = 32 p + lane (lane 0 at column 16 c, lane 1 at rowk_off(K) + 16 c) like rotq_kernel's split mode,
// keeps dt(y) as bf16 pairs in the warp's row buffer in shared memory (64 bytes per thread per pass, so 2 K bytes per
// row) and the running absmax in a register.  After the last pass a warp shuffle gives the row's amax, and a second
// sweep over the buffer quantises and stores.  No CTA barrier: each warp runs its rows on its own, and the per-row
// scalar work (the scale's division and reciprocal) is spread over the whole row instead of 32 elements per thread.
// The same roundings as rotq_kernel (dt(y) is the hardware round-to-nearest-even pack), so the codes are identical.
constexpr int ROWK_PASS = 1024;  // elements of a row per pass (32 threads x 2 lanes x 16)
// The row kernel serves M >= ROWK_MIN_ROWS (below, a CTA per row spreads each row over more SMs) and rows whose buffer
// leaves room for several warps per SM.
#ifndef H3B_ROTQ_ROW_MIN_ROWS
#define H3B_ROTQ_ROW_MIN_ROWS 4096
#endif
constexpr int64_t ROWK_MIN_ROWS = H3B_ROTQ_ROW_MIN_ROWS;
constexpr size_t ROWK_MAX_WARP_BYTES = 16 * 1024;  // K <= 5120 (at 8192 and above the CTA kernel is faster)
__host__ __device__ constexpr int rowk_xbytes() { return 2 * xgrp(16) * 8; }  // a warp's exchange area (two blocks)
// Row buffer of a pass: per ConvRot block a 16 x 16 matrix of bf16 pairs (row i = elements 16 i .. 16 i + 15 of the
// block), the four 16-byte chunks of row i stored in the order j ^ ((i >> 1) & 3), blocks 272 words apart: the
// transform's column writes (16 threads, element t + 16 i) and the quantiser's row reads (thread t', 16-byte chunks of
// row t') are both free of bank conflicts.
constexpr int ROWK_BLOCK_WORDS = 16 * 16 + 16;
constexpr int ROWK_PASS_BYTES = 2 * ROWK_BLOCK_WORDS * 4;  // a pass's part of the row buffer (two blocks)
// A thread's two lanes are the same row, `rowk_off(K)` elements apart: K / 2 when K is a multiple of 512, otherwise
// (K a multiple of 256 only, e.g. the official width 5376 = 21 x 256) half a ConvRot block more, so that both lanes sit
// at the same position of their blocks; the upper lane then runs off the end of the row for the last 128 elements of
// the lower half, where it loads zeros (no effect on the transform of other blocks or on the absmax) and stores nothing.
__host__ __device__ constexpr int64_t rowk_off(int64_t K) { return (K + 511) / 512 * 256; }
__host__ __device__ constexpr int rowk_passes(int64_t K) { return static_cast<int>((2 * rowk_off(K) + ROWK_PASS - 1) / ROWK_PASS); }
// A warp's shared memory: the row buffer, then a tail.  Pass p's exchange area starts where the pass's part of the row
// buffer starts: that part and those of the later passes hold nothing yet (the pass writes its part only after the
// exchange is read back), so only the last pass's exchange reaches past the row buffer, into the tail.
__host__ __device__ inline size_t rowk_warp_bytes(int64_t K) {
  return static_cast<size_t>(rowk_passes(K)) * ROWK_PASS_BYTES +
         (rowk_xbytes() > ROWK_PASS_BYTES ? rowk_xbytes() - ROWK_PASS_BYTES : 0);
}
__device__ __forceinline__ int rowk_word(int i, int col) { return 16 * i + 4 * ((col >> 2) ^ ((i >> 1) & 3)) + (col & 3); }


// 16 bf16 values from element e of a bf16 array (16-byte aligned) for lane 0 and from element e + off for lane 1, as
// (lane 0, lane 1) pairs; lane 1 reads zeros when e + off is past the row (hi_ok false)
__device__ __forceinline__ void load_pairs16(const __nv_bfloat16* p, int64_t e, int64_t off, bool hi_ok, float2 (&out)[16]) {
  const uint4* a = reinterpret_cast<const uint4*>(p + e);
  const uint4* b = reinterpret_cast<const uint4*>(p + e + off);
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const uint4 ua = __ldg(a + i), ub = hi_ok ? __ldg(b + i) : make_uint4(0u, 0u, 0u, 0u);
    const uint32_t wa[4] = {ua.x, ua.y, ua.z, ua.w}, wb[4] = {ub.x, ub.y, ub.z, ub.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 fa = unpack2<DT_BF16>(wa[k]), fb = unpack2<DT_BF16>(wb[k]);
      out[8 * i + 2 * k] = make_float2(fa.x, fb.x);
      out[8 * i + 2 * k + 1] = make_float2(fa.y, fb.y);
    }
  }
}

template <int MODE, bool SW, bool NORM>
__global__ void __launch_bounds__(256) rotq_row_kernel(const void* __restrict__ x, int64_t ldx, int M, int K,
                                                       int8_t* __restrict__ q, int64_t ldq, float* __restrict__ xs_out,
                                                       const RowNorm nrm) {
  static_assert(!(SW && NORM), "the norm prologue reads the block's residual stream, not a SwiGLU input");
  constexpr int DT = DT_BF16;
  constexpr float SCALE = 0.0625f;
  extern __shared__ __align__(16) unsigned char rotq_smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int64_t half = rowk_off(K);  // lane 1's offset from lane 0 (K / 2 when K is a multiple of 512)
  const int P = rowk_passes(K);
  const int nchunk = static_cast<int>(half / 16);  // chunk pairs per row; a multiple of 16, so a pass is full or its
                                                   // upper half-warp idles
  unsigned char* wbase = rotq_smem + static_cast<size_t>(warp) * rowk_warp_bytes(K);
  const int t = lane & 15;
  // this half-warp's block in the row buffer of pass 0 (passes are 2 blocks apart), and its exchange area in pass 0
  // (the exchange of pass p sits ROWK_PASS_BYTES * p further on)
  uint32_t* bblk = reinterpret_cast<uint32_t*>(wbase) + (lane >> 4) * ROWK_BLOCK_WORDS;
  float2* gbuf0 = reinterpret_cast<float2*>(wbase) + (lane >> 4) * xgrp(16);
  const int64_t rstep = static_cast<int64_t>(gridDim.x) * nw;
  int64_t row = static_cast<int64_t>(blockIdx.x) * nw + warp;

  Raw<DT, SW> raw;
  auto load = [&](int64_t r, int p) {  // r < M; the idle half-warp of a row's last pass re-reads chunk nchunk - 1
    const int c = 32 * p + lane;
    const int64_t e = 16ll * (c < nchunk ? c : nchunk - 1);
    const char* base = static_cast<const char*>(x) + static_cast<size_t>(r) * static_cast<size_t>(ldx) * 2;
#pragma unroll
    for (int h = 0; h < (SW ? 2 : 1); ++h) {  // SwiGLU rows hold [gate | up], K elements apart
      const uint4* lo = reinterpret_cast<const uint4*>(base + static_cast<size_t>(e + h * K) * 2);
      const uint4* hi = reinterpret_cast<const uint4*>(base + static_cast<size_t>(e + half + h * K) * 2);
      const bool hi_ok = e + half < K;
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        raw.u[h * 2 + i] = __ldg(lo + i);
        raw.u[((SW ? 2 : 1) + h) * 2 + i] = hi_ok ? __ldg(hi + i) : make_uint4(0u, 0u, 0u, 0u);
      }
    }
  };
  // the four swizzled column offsets of this thread's element column t (row i uses colw[(i >> 1) & 3])
  int colw[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) colw[j] = 4 * ((t >> 2) ^ j) + (t & 3);
  int rowr[4];  // and the word offsets of the four 16-byte chunks of row t
#pragma unroll
  for (int j = 0; j < 4; ++j) rowr[j] = rowk_word(t, 4 * j);
  if (row < M) load(row, 0);
  for (; row < M; row += rstep) {
    float mA = 0.f;
    float2 RS2 = make_float2(0.f, 0.f);
    int mrow = -1;
    if constexpr (NORM) {
      // sum of squares in rms_modulate_warp_kernel's order: lane l adds its 8-element vectors l, l + 32, ... in turn,
      // then an xor-shuffle tree; the loads go out four vectors at a time
      const uint4* xr = reinterpret_cast<const uint4*>(static_cast<const char*>(x) + row * ldx * 2);
      const int vpw = K >> 8;
      float ss = 0.f;
      int v0 = 0;
      for (; v0 + 4 <= vpw; v0 += 4) {
        uint4 u[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) u[j] = __ldg(xr + lane + 32 * (v0 + j));
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float f[8];
          unpack8<H3B_BF16>(u[j], f);
#pragma unroll
          for (int i = 0; i < 8; ++i) ss = __fmaf_rn(f[i], f[i], ss);
        }
      }
      for (; v0 < vpw; ++v0) {
        float f[8];
        unpack8<H3B_BF16>(__ldg(xr + lane + 32 * v0), f);
#pragma unroll
        for (int i = 0; i < 8; ++i) ss = __fmaf_rn(f[i], f[i], ss);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
      const float rs = rsqrtf(__fadd_rn(__fdiv_rn(ss, static_cast<float>(K)), nrm.eps));
      RS2 = make_float2(rs, rs);
      if (nrm.token_rows) {
        mrow = nrm.token_rows[row];
      } else {
        for (int s2 = 0; s2 < nrm.segs.n; ++s2)
          if (row >= nrm.segs.first[s2] && row < nrm.segs.end[s2]) mrow = nrm.segs.row[s2];
      }
    }
    for (int p = 0; p < P; ++p) {
      float2 v[16];
      if constexpr (!SW) {
#pragma unroll
        for (int i = 0; i < 2; ++i) {
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
        swiglu_lanes<DT>(raw, v);
      }
      if (p + 1 < P) load(row, p + 1);
      else if (row + rstep < M) load(row + rstep, 0);
      if constexpr (NORM) {  // x -> h: n = dt((x rs) w); h = dt(dt(n s1) + sh) for a modulated token
        const int64_t e = 16ll * ((32 * p + lane) < nchunk ? 32 * p + lane : nchunk - 1);
        const bool hi_ok = e + half < K;
        float2 a[16];
        load_pairs16(nrm.w, e, half, hi_ok, a);
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = rnd_bf16x2(__fmul2_rn(__fmul2_rn(v[i], RS2), a[i]));
        if (mrow >= 0) {
          load_pairs16(nrm.scale1 + mrow * nrm.ldm, e, half, hi_ok, a);
#pragma unroll
          for (int i = 0; i < 16; ++i) v[i] = rnd_bf16x2(__fmul2_rn(v[i], a[i]));
          load_pairs16(nrm.shift + mrow * nrm.ldm, e, half, hi_ok, a);
#pragma unroll
          for (int i = 0; i < 16; ++i) v[i] = rnd_bf16x2(__fadd2_rn(v[i], a[i]));
        }
      }

      // stage A (digits d0, d1 in registers), exchange, stage B (d2, d3 across the 16 threads of the block)
#pragma unroll
      for (int a = 0; a < 4; ++a) h4(v[4 * a], v[4 * a + 1], v[4 * a + 2], v[4 * a + 3], 1.0f);
#pragma unroll
      for (int d = 0; d < 4; ++d) h4(v[d], v[d + 4], v[d + 8], v[d + 12], 1.0f);
      {
        float2* gbuf = gbuf0 + p * (ROWK_PASS_BYTES / 8);
        float4* wr = reinterpret_cast<float4*>(gbuf + t * XROW);
#pragma unroll
        for (int i = 0; i < 8; ++i) wr[i] = make_float4(v[2 * i].x, v[2 * i].y, v[2 * i + 1].x, v[2 * i + 1].y);
        __syncwarp();
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = gbuf[j * XROW + t];
        __syncwarp();
      }
#pragma unroll
      for (int a = 0; a < 4; ++a) h4(v[4 * a], v[4 * a + 1], v[4 * a + 2], v[4 * a + 3], 1.0f);
#pragma unroll
      for (int d = 0; d < 4; ++d) h4(v[d], v[d + 4], v[d + 8], v[d + 12], SCALE);

      // dt(y) as bf16 pairs (lane 0 low, lane 1 high) into the row buffer; absmax of y (ck) or of dt(y) (eager)
      uint32_t bw[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) bw[i] = pack2<DT>(v[i]);
      float m4[4] = {0.f, 0.f, 0.f, 0.f};  // four independent chains
      if constexpr (MODE == MODE_CK) {
#pragma unroll
        for (int i = 0; i < 16; ++i) m4[i & 3] = max3f(m4[i & 3], fabsf(v[i].x), fabsf(v[i].y));
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float2 b = unpack2<DT>(bw[i]);
          m4[i & 3] = max3f(m4[i & 3], fabsf(b.x), fabsf(b.y));
        }
      }
      const float mP = max3f(m4[0], m4[1], fmaxf(m4[2], m4[3]));
      if (32 * p + lane < nchunk) mA = fmaxf(mA, mP);
      uint32_t* bp = bblk + p * (2 * ROWK_BLOCK_WORDS);
#pragma unroll
      for (int i = 0; i < 16; ++i) bp[16 * i + colw[(i >> 1) & 3]] = bw[i];  // element t + 16 i: row i, column t
    }
    __syncwarp();  // the quantiser reads rows that other threads of the half-warp wrote

    // the row's scale
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mA = fmaxf(mA, __shfl_xor_sync(0xffffffffu, mA, o));
    const float xs = fmaxf(__fdiv_rn(mA, 127.0f), 1e-30f);
    float s = round_dt<DT>(xs);
    if (s == 0.f) s = tiny_dt<DT>();
    if (lane == 0) xs_out[row] = xs;
    const float r = __frcp_rn(s);
    const float2 R2 = make_float2(r, r);

    // quantise: code = sat(rint(dt(RN(b / s)))) with RNbf16(RN(b RN(1/s))) = RNbf16(RN(b / s)).  Thread t' takes row
    // t' of its block, i.e. its own chunk pair c = 32 p + lane in element order, so its codes pack straight into words.
    int8_t* qrow = q + row * ldq;
    for (int p = 0; p < P; ++p) {
      const uint32_t* bp = bblk + p * (2 * ROWK_BLOCK_WORDS);
      uint32_t qb[16];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint4 u = *reinterpret_cast<const uint4*>(bp + rowr[j]);
        qb[4 * j] = u.x; qb[4 * j + 1] = u.y; qb[4 * j + 2] = u.z; qb[4 * j + 3] = u.w;
      }
#pragma unroll
      for (int e = 0; e < 16; ++e) qb[e] = pack2<DT>(__fmul2_rn(unpack2<DT>(qb[e]), R2));
      uint32_t wA[4], wB[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        wA[u] = codes4_bf16<false>(qb[4 * u], qb[4 * u + 1], qb[4 * u + 2], qb[4 * u + 3]);
        wB[u] = codes4_bf16<true>(qb[4 * u], qb[4 * u + 1], qb[4 * u + 2], qb[4 * u + 3]);
      }
      const int c = 32 * p + lane;
      if (c < nchunk) {
        *reinterpret_cast<uint4*>(qrow + 16ll * c) = make_uint4(wA[0], wA[1], wA[2], wA[3]);
        if (half + 16ll * c < K) *reinterpret_cast<uint4*>(qrow + half + 16ll * c) = make_uint4(wB[0], wB[1], wB[2], wB[3]);
      }
    }
    __syncwarp();  // the next row's first exchange overwrites row buffer parts that the loop above read
  }
}

// H3B_ROTQ_ROW=0 in the environment keeps rotq_kernel for every shape (read once per process; for comparisons).
static bool rowk_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("H3B_ROTQ_ROW");
    v = (e && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

// Warps per CTA for the row kernel: the most warps per SM that the row buffers allow (ties: more warps per CTA).
// Chosen once per K and kept (a few entries; the device is the same kind on every call).
struct RowkShape { int64_t K; int nw, ctas_per_sm, sms; };

template <int MODE, bool SW, bool NORM>
static int rowk_shape(int64_t K, RowkShape& out) {
  static std::mutex mu;
  static RowkShape cache[8];
  static int n_cached = 0;
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < n_cached; ++i)
    if (cache[i].K == K) { out = cache[i]; return 0; }
  auto kern = rotq_row_kernel<MODE, SW, NORM>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(rotq_row)");
  cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const size_t per_warp = rowk_warp_bytes(K);
  RowkShape best{K, 0, 0, sms};
  for (int nw = 8; nw >= 1; --nw) {
    const size_t smem = per_warp * nw;
    if (smem > 227 * 1024) continue;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 32 * nw, smem);
    if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor(rotq_row)");
    if (per_sm * nw > best.nw * best.ctas_per_sm) { best.nw = nw; best.ctas_per_sm = per_sm; }
  }
  if (best.nw == 0) return fail(H3B_ERR_UNSUPPORTED, "rotq_row: the row buffer does not fit in shared memory");
  cache[n_cached < 8 ? n_cached++ : 7] = best;
  out = best;
  return 0;
}

template <int MODE, bool SW, bool NORM = false>
static int rowk_launch(const void* x, int64_t ldx, int64_t M, int64_t K, int8_t* q, int64_t ldq, float* xs,
                       cudaStream_t st, const RowNorm& nrm = RowNorm{}) {
  RowkShape sh;
  if (int rc = rowk_shape<MODE, SW, NORM>(K, sh)) return rc;
  const size_t smem = rowk_warp_bytes(K) * sh.nw;
  const int64_t want = (M + sh.nw - 1) / sh.nw, cap = static_cast<int64_t>(sh.sms) * sh.ctas_per_sm;
  const int blocks = static_cast<int>(want < cap ? want : cap);
  rotq_row_kernel<MODE, SW, NORM><<<blocks, 32 * sh.nw, smem, st>>>(x, ldx, static_cast<int>(M), static_cast<int>(K), q,
                                                                      ldq, xs, nrm);
  return check_launch("rotq_row_kernel");
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
  if constexpr (DT == DT_BF16 && CR == 256 && MODE != MODE_ROTATE) {
    if (K % 256 == 0 && M >= ROWK_MIN_ROWS && rowk_warp_bytes(K) <= ROWK_MAX_WARP_BYTES && rowk_enabled())
      return rowk_launch<MODE, SW>(x, ldx, M, K, q, ldq, xs, st);
  }
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

// RMSNorm + modulation fused into the quantiser (bf16 x, ConvRot 256, K a multiple of 256 and <= 6144: the shapes the
// norm's warp-per-row kernel serves, whose sum order this reproduces).  Codes and scales are bit-identical to
// rms_modulate_launch followed by rotq_launch on its output.
bool rotq_rmsmod_supported(int64_t K) { return K > 0 && K % 256 == 0 && K <= 6144; }

int rotq_rmsmod_launch(const void* x, int64_t ldx, int64_t M, int64_t K, const RowNorm& nrm, int mode, int8_t* q,
                       int64_t ldq, float* xs, cudaStream_t st) {
  if (!rotq_rmsmod_supported(K)) return fail(H3B_ERR_UNSUPPORTED, "rotq_rms_modulate: K must be a multiple of 256, at most 6144");
  if (mode == MODE_CK) return rowk_launch<MODE_CK, false, true>(x, ldx, M, K, q, ldq, xs, st, nrm);
  if (mode == MODE_EAGER) return rowk_launch<MODE_EAGER, false, true>(x, ldx, M, K, q, ldq, xs, st, nrm);
  return fail(H3B_ERR_ARG, "rotq_rms_modulate: quant_mode must be ck or eager");
}

}  // namespace h3b
