// Kernel KA: ConvRot rotation + per-token int8 quantisation (and the rotation-only variant).
//
// Reference semantics (h3turbo/h3/qlinear.py):
//   y32  = per-`convrot`-block x @ H, H = kron(H4, ..., H4) / sqrt(convrot)          _rot32 / hadamard_regular :44-115
//   amax = max |y32| over the whole row ("ck") or max |dt(y32)| ("eager")           _quantize_rows :278-287
//   xs   = max(amax / 127, 1e-30) (fp32); s = dt(xs), 0 -> finfo(dt).tiny           :288-290
//   q    = clamp(rint(dt(fp32(dt(y32)) / s)), -128, 127)                              :291-292
//   with input_act="swiglu": x <- dt(dt(silu(gate)) * up) first                       _swiglu :376-379
//
// Layout.  A thread owns a 16-element chunk of TWO rows (a row pair), so every butterfly and every quantiser FMA is a
// packed fp32x2 instruction with row A in .x and row B in .y.  Inside a ConvRot block of CR = 4^n elements, element
// e has base-4 digits d0..d(n-1).  The chunk's 16 elements are digits d0, d1 (in registers); the CR/16 threads of a
// block hold digits d2, d3.  Stage A transforms d0, d1 in registers; a swizzled shared-memory exchange regroups the
// block so each thread holds all values of d2, d3 for a fixed (d0, d1); stage B transforms those.  The regular H4
// butterfly is (H4 a)_i = S - 2 a_{3-i}, S = (a0 + a1) + (a2 + a3); the 1/sqrt(CR) normalisation (a power of two) is
// folded into the last stage, which is exact.
//
// Division: s is constant per row, so q = dt(RN(b / s)) uses r = RN(1 / s) and one Markstein correction
// (q0 = RN(b r), e = b - q0 s exactly, q1 = RN(q0 + e r)), which returns the correctly rounded quotient for every pair
// of bf16 / fp16 operands (checked exhaustively over all significand pairs by tests/test_numerics.py); fp32
// activations use the IEEE division directly.
#include "h3b_common.cuh"

namespace h3b {

enum { DT_BF16 = 0, DT_FP16 = 1, DT_FP32 = 2 };
enum { MODE_CK = 0, MODE_EAGER = 1, MODE_ROTATE = 2 };

// ------------------------------------------------------------------------------------------------ dtype helpers
template <int DT>
__device__ __forceinline__ float2 round_dt2(float2 v) {
  if constexpr (DT == DT_BF16) {
    const __nv_bfloat162 h = __float22bfloat162_rn(v);
    return __bfloat1622float2(h);
  } else if constexpr (DT == DT_FP16) {
    const __half2 h = __float22half2_rn(v);
    return __half22float2(h);
  } else {
    return v;
  }
}
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

// 16 consecutive activations of one row starting at element `off` -> fp32 (exact).  Row pointer 16-byte aligned.
template <int DT>
__device__ __forceinline__ void load16(const void* row, int64_t off, float (&v)[16]) {
  if constexpr (DT == DT_FP32) {
    const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(row) + off);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4 f = __ldg(p + i);
      v[4 * i] = f.x; v[4 * i + 1] = f.y; v[4 * i + 2] = f.z; v[4 * i + 3] = f.w;
    }
  } else {
    const uint4* p = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(row) + off);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const uint4 u = __ldg(p + i);
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if constexpr (DT == DT_BF16) {
          v[8 * i + 2 * k] = __int_as_float(w[k] << 16);
          v[8 * i + 2 * k + 1] = __int_as_float(w[k] & 0xFFFF0000u);
        } else {
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[k]));
          v[8 * i + 2 * k] = f.x;
          v[8 * i + 2 * k + 1] = f.y;
        }
      }
    }
  }
}

// silu(gate) * up in dt, as torch computes it: x / (1 + exp(-x)) in fp32, rounded to dt; the product of the two dt
// values in fp32, rounded to dt.
template <int DT>
__device__ __forceinline__ float swiglu1(float g, float u) {
  const float sl = round_dt<DT>(g / (1.0f + expf(-g)));
  return round_dt<DT>(sl * u);
}

template <int DT, bool SWIGLU>
__device__ __forceinline__ void load_chunk(const void* x, int64_t ldx, int64_t row, bool valid, int64_t col, int K,
                                           float (&v)[16]) {
  if (!valid) {
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = 0.f;
    return;
  }
  const size_t esz = DT == DT_FP32 ? 4 : 2;
  const char* r = static_cast<const char*>(x) + static_cast<size_t>(row) * static_cast<size_t>(ldx) * esz;
  load16<DT>(r, col, v);
  if constexpr (SWIGLU) {
    float u[16];
    load16<DT>(r, col + K, u);
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = swiglu1<DT>(v[i], u[i]);
  }
}

// ------------------------------------------------------------------------------------------------ butterflies
__device__ __forceinline__ void h4x2(float2& a0, float2& a1, float2& a2, float2& a3) {
  const float2 s = __fadd2_rn(__fadd2_rn(a0, a1), __fadd2_rn(a2, a3));
  const float2 m2 = make_float2(-2.f, -2.f);
  const float2 y0 = __ffma2_rn(m2, a3, s), y1 = __ffma2_rn(m2, a2, s);
  const float2 y2 = __ffma2_rn(m2, a1, s), y3 = __ffma2_rn(m2, a0, s);
  a0 = y0; a1 = y1; a2 = y2; a3 = y3;
}
// Same butterfly, result scaled by the power of two `sc` (exact).
__device__ __forceinline__ void h4x2s(float2& a0, float2& a1, float2& a2, float2& a3, float sc) {
  const float2 s = __fmul2_rn(__fadd2_rn(__fadd2_rn(a0, a1), __fadd2_rn(a2, a3)), make_float2(sc, sc));
  const float2 m2 = make_float2(-2.f * sc, -2.f * sc);
  const float2 y0 = __ffma2_rn(m2, a3, s), y1 = __ffma2_rn(m2, a2, s);
  const float2 y2 = __ffma2_rn(m2, a1, s), y3 = __ffma2_rn(m2, a0, s);
  a0 = y0; a1 = y1; a2 = y2; a3 = y3;
}

// ------------------------------------------------------------------------------------------------ the kernel
// blockDim.x = tpr * pairs; tpr = K / 16 threads per row pair.  Row pair p of the CTA: rows 2(blockIdx.x*pairs+p)+{0,1}.
template <int DT, int CR, int MODE, bool SWIGLU>
__global__ void __launch_bounds__(1024) rotq_kernel(const void* __restrict__ x, int64_t ldx, int M, int K, int tpr,
                                                     int pairs, int8_t* __restrict__ q, int64_t ldq,
                                                     float* __restrict__ xs_out, void* __restrict__ y_out,
                                                     int y_dtype, int64_t ldy) {
  constexpr int G = CR >= 256 ? 16 : (CR == 64 ? 4 : 1);  // threads per ConvRot block
  constexpr float SCALE = CR == 256 ? 0.0625f : CR == 64 ? 0.125f : CR == 16 ? 0.25f : 0.5f;
  extern __shared__ __align__(16) unsigned char rotq_smem[];
  unsigned int* rowmax = reinterpret_cast<unsigned int*>(rotq_smem);  // [2 * pairs]
  float2* xbuf = reinterpret_cast<float2*>(rotq_smem + 16 * ((2 * pairs * 4 + 15) / 16));  // [blockDim][16]

  const int tid = threadIdx.x;
  const int p = tid / tpr, tr = tid - p * tpr;  // pair in CTA, thread in row
  const int64_t rowA = 2ll * (static_cast<int64_t>(blockIdx.x) * pairs + p);
  const bool vA = rowA < M, vB = rowA + 1 < M;
  const int64_t col = 16ll * tr;

  if (tid < 2 * pairs) rowmax[tid] = 0u;

  float2 v[16];
  {
    float a[16], b[16];
    load_chunk<DT, SWIGLU>(x, ldx, rowA, vA, col, K, a);
    load_chunk<DT, SWIGLU>(x, ldx, rowA + 1, vB, col, K, b);
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = make_float2(a[i], b[i]);
  }

  // ---- stage A: digits d0 (register bits 0-1) and d1 (register bits 2-3)
  if constexpr (CR == 4) {
#pragma unroll
    for (int g = 0; g < 4; ++g) h4x2s(v[4 * g], v[4 * g + 1], v[4 * g + 2], v[4 * g + 3], SCALE);
  } else {
#pragma unroll
    for (int g = 0; g < 4; ++g) h4x2(v[4 * g], v[4 * g + 1], v[4 * g + 2], v[4 * g + 3]);
#pragma unroll
    for (int d = 0; d < 4; ++d) {
      if constexpr (CR == 16) h4x2s(v[d], v[d + 4], v[d + 8], v[d + 12], SCALE);
      else h4x2(v[d], v[d + 4], v[d + 8], v[d + 12]);
    }
  }

  // ---- exchange + stage B (digits d2, d3 across the G threads of the block)
  const int t = tr % G;                       // thread within the ConvRot block
  float2* gbuf = xbuf + static_cast<size_t>(tid - t) * 16;  // this block's G x 16 float2
  if constexpr (G > 1) {
    // write own 16 values as eight 16-byte chunks, chunk index XOR-swizzled by the owner so stores are conflict-free
    float4* wr = reinterpret_cast<float4*>(gbuf + t * 16);
#pragma unroll
    for (int i = 0; i < 8; ++i)
      wr[i ^ (t & 7)] = make_float4(v[2 * i].x, v[2 * i].y, v[2 * i + 1].x, v[2 * i + 1].y);
    __syncwarp();
    if constexpr (G == 16) {
      // v[j] <- owner j's element r = t   (register j = d2 + 4 d3)
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float2* src = gbuf + j * 16;
        v[j] = src[2 * ((t >> 1) ^ (j & 7)) + (t & 1)];
      }
      __syncwarp();
#pragma unroll
      for (int g = 0; g < 4; ++g) h4x2(v[4 * g], v[4 * g + 1], v[4 * g + 2], v[4 * g + 3]);
#pragma unroll
      for (int d = 0; d < 4; ++d) h4x2s(v[d], v[d + 4], v[d + 8], v[d + 12], SCALE);
    } else {
      // G == 4: v[4 j + d0] <- owner j's elements r = 4t + d0  (register 4j + d0; digit d2 = j)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float4* src = reinterpret_cast<const float4*>(gbuf + j * 16);
        const float4 c0 = src[(2 * t) ^ (j & 7)], c1 = src[(2 * t + 1) ^ (j & 7)];
        v[4 * j + 0] = make_float2(c0.x, c0.y);
        v[4 * j + 1] = make_float2(c0.z, c0.w);
        v[4 * j + 2] = make_float2(c1.x, c1.y);
        v[4 * j + 3] = make_float2(c1.z, c1.w);
      }
      __syncwarp();
#pragma unroll
      for (int d = 0; d < 4; ++d) h4x2s(v[d], v[d + 4], v[d + 8], v[d + 12], SCALE);
    }
  }
  // element index (within the row) of register i
  const int64_t blk0 = static_cast<int64_t>(tr - t) * 16;  // first element of this ConvRot block
  auto elem = [&](int i) -> int64_t {
    if constexpr (G == 16) return blk0 + t + 16 * i;
    else if constexpr (G == 4) return blk0 + 16 * (i >> 2) + 4 * t + (i & 3);
    else return col + i;
  };

  if constexpr (MODE == MODE_ROTATE) {
    const size_t ysz = y_dtype == 2 ? 4 : 2;
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      if (!(rr == 0 ? vA : vB)) continue;
      char* yr = static_cast<char*>(y_out) + static_cast<size_t>(rowA + rr) * static_cast<size_t>(ldy) * ysz;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float val = rr == 0 ? v[i].x : v[i].y;
        const int64_t e = elem(i);
        if (y_dtype == 0) reinterpret_cast<__nv_bfloat16*>(yr)[e] = __float2bfloat16_rn(val);
        else if (y_dtype == 1) reinterpret_cast<__half*>(yr)[e] = __float2half_rn(val);
        else reinterpret_cast<float*>(yr)[e] = val;
      }
    }
    return;
  } else {
    // ---- dt rounding and the row absmax
    float2 b[16];
    float mA = 0.f, mB = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      b[i] = round_dt2<DT>(v[i]);
      const float2 src = MODE == MODE_CK ? v[i] : b[i];
      mA = fmaxf(mA, fabsf(src.x));
      mB = fmaxf(mB, fabsf(src.y));
    }
    __syncthreads();  // rowmax initialised
    if ((tpr & 31) == 0) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        mA = fmaxf(mA, __shfl_xor_sync(0xffffffffu, mA, o));
        mB = fmaxf(mB, __shfl_xor_sync(0xffffffffu, mB, o));
      }
      if ((tid & 31) == 0) {
        atomicMax(&rowmax[2 * p], __float_as_uint(mA));
        atomicMax(&rowmax[2 * p + 1], __float_as_uint(mB));
      }
    } else {
      atomicMax(&rowmax[2 * p], __float_as_uint(mA));
      atomicMax(&rowmax[2 * p + 1], __float_as_uint(mB));
    }
    __syncthreads();
    const float amaxA = __uint_as_float(rowmax[2 * p]), amaxB = __uint_as_float(rowmax[2 * p + 1]);
    const float xsA = fmaxf(__fdiv_rn(amaxA, 127.0f), 1e-30f), xsB = fmaxf(__fdiv_rn(amaxB, 127.0f), 1e-30f);
    float sA = round_dt<DT>(xsA), sB = round_dt<DT>(xsB);
    if (sA == 0.f) sA = tiny_dt<DT>();
    if (sB == 0.f) sB = tiny_dt<DT>();
    if (tr == 0) {
      if (vA) xs_out[rowA] = xsA;
      if (vB) xs_out[rowA + 1] = xsB;
    }

    // ---- quantise: c = sat_s8(rint(dt(RN(b / s))))
    uint32_t c[16];
    if constexpr (DT == DT_FP32) {
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float qa = __fdiv_rn(b[i].x, sA), qb = __fdiv_rn(b[i].y, sB);
        int ia, ib;
        asm("cvt.rni.sat.s8.f32 %0, %1;" : "=r"(ia) : "f"(qa));
        asm("cvt.rni.sat.s8.f32 %0, %1;" : "=r"(ib) : "f"(qb));
        c[i] = (static_cast<uint32_t>(ia) & 0xFFu) | ((static_cast<uint32_t>(ib) & 0xFFu) << 8);
      }
    } else {
      const float2 S2 = make_float2(sA, sB), nS2 = make_float2(-sA, -sB);
      const float2 R2 = make_float2(__frcp_rn(sA), __frcp_rn(sB));
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float2 q0 = __fmul2_rn(b[i], R2);
        const float2 e = __ffma2_rn(q0, nS2, b[i]);
        const float2 q1 = round_dt2<DT>(__ffma2_rn(e, R2, q0));
        int ia, ib;
        asm("cvt.rni.sat.s8.f32 %0, %1;" : "=r"(ia) : "f"(q1.x));
        asm("cvt.rni.sat.s8.f32 %0, %1;" : "=r"(ib) : "f"(q1.y));
        c[i] = (static_cast<uint32_t>(ia) & 0xFFu) | ((static_cast<uint32_t>(ib) & 0xFFu) << 8);
      }
      (void)S2;
    }

    // ---- store the codes of both rows (16 contiguous bytes each)
    uint32_t wA[4], wB[4];
    if constexpr (G == 1) {
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        wA[w] = __byte_perm(__byte_perm(c[4 * w], c[4 * w + 1], 0x0040), __byte_perm(c[4 * w + 2], c[4 * w + 3], 0x0040), 0x5410);
        wB[w] = __byte_perm(__byte_perm(c[4 * w], c[4 * w + 1], 0x0051), __byte_perm(c[4 * w + 2], c[4 * w + 3], 0x0051), 0x5410);
      }
    } else {
      // regroup through shared memory: interleaved (A, B) byte pairs at each element of this block
      uint16_t* cb = reinterpret_cast<uint16_t*>(gbuf);
#pragma unroll
      for (int i = 0; i < 16; ++i) cb[elem(i) - blk0] = static_cast<uint16_t>(c[i]);
      __syncwarp();
      const uint4* rd = reinterpret_cast<const uint4*>(cb + 16 * t);
      const uint4 u0 = rd[0], u1 = rd[1];
      const uint32_t w8[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        wA[w] = __byte_perm(w8[2 * w], w8[2 * w + 1], 0x6420);
        wB[w] = __byte_perm(w8[2 * w], w8[2 * w + 1], 0x7531);
      }
    }
    if (vA) *reinterpret_cast<uint4*>(q + rowA * ldq + col) = make_uint4(wA[0], wA[1], wA[2], wA[3]);
    if (vB) *reinterpret_cast<uint4*>(q + (rowA + 1) * ldq + col) = make_uint4(wB[0], wB[1], wB[2], wB[3]);
  }
}

// ------------------------------------------------------------------------------------------------ launcher
struct RotqLaunch {
  int tpr, pairs, threads, blocks;
  size_t smem;
};

static RotqLaunch plan(int64_t M, int64_t K) {
  RotqLaunch L;
  L.tpr = static_cast<int>(K / 16);
  L.pairs = L.tpr >= 256 ? 1 : (256 + L.tpr - 1) / L.tpr;
  while (L.pairs > 1 && L.pairs * L.tpr > 1024) --L.pairs;
  L.threads = L.pairs * L.tpr;
  const int64_t row_pairs = (M + 1) / 2;
  L.blocks = static_cast<int>((row_pairs + L.pairs - 1) / L.pairs);
  L.smem = 16 * ((2 * L.pairs * 4 + 15) / 16) + static_cast<size_t>(L.threads) * 16 * sizeof(float2);
  return L;
}

template <int DT, int CR, int MODE, bool SW>
static int launch_t(const void* x, int64_t ldx, int64_t M, int64_t K, int8_t* q, int64_t ldq, float* xs, void* y,
                    int ydt, int64_t ldy, cudaStream_t st) {
  const RotqLaunch L = plan(M, K);
  auto kern = rotq_kernel<DT, CR, MODE, SW>;
  if (L.smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(L.smem));
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(rotq)");
  }
  kern<<<L.blocks, L.threads, L.smem, st>>>(x, ldx, static_cast<int>(M), static_cast<int>(K), L.tpr, L.pairs, q, ldq, xs,
                                            y, ydt, ldy);
  return check_launch("rotq_kernel");
}

template <int DT, int MODE, bool SW>
static int launch_cr(int cr, const void* x, int64_t ldx, int64_t M, int64_t K, int8_t* q, int64_t ldq, float* xs, void* y,
                     int ydt, int64_t ldy, cudaStream_t st) {
  switch (cr) {
    case 4: return launch_t<DT, 4, MODE, SW>(x, ldx, M, K, q, ldq, xs, y, ydt, ldy, st);
    case 16: return launch_t<DT, 16, MODE, SW>(x, ldx, M, K, q, ldq, xs, y, ydt, ldy, st);
    case 64: return launch_t<DT, 64, MODE, SW>(x, ldx, M, K, q, ldq, xs, y, ydt, ldy, st);
    case 256: return launch_t<DT, 256, MODE, SW>(x, ldx, M, K, q, ldq, xs, y, ydt, ldy, st);
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
