// Fused RMSNorm + AdaLN modulation of the DiT block's residual stream: h = scale_shift(rms(x)).
//
// Reference semantics (h3turbo/h3/model.py):
//   _rms (:64-66):            n = dt((x * rsqrt(mean(x^2) + eps)) * w), w first rounded to dt, fp32 math, one rounding
//                             (torch's fused F.rms_norm; its reduction order is its own, so a row's rsqrt can differ
//                             from this kernel's in the last fp32 bit: about 4 elements per million flip one dt ulp)
//   _scale_shift_ (:106-109): for token segments (a, b, row):  h = dt(n * dt(1 + dt(scale[row])));  h = dt(h + dt(shift[row]))
//   tokens outside every segment keep n.
// One CTA per row (persistent over rows): 16-byte loads, fp32 sum of squares per thread, warp shuffles and one shared
// memory pass for the row total.  HBM-bound: 2 H bytes read + 2 H written per token (the modulation rows stay in L2).
#pragma once
#include "h3b_common.cuh"
#include "launch.h"

namespace h3b {

template <int DT>
__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if constexpr (DT == H3B_BF16) {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    } else {
      const float2 v = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
      f[2 * i] = v.x;
      f[2 * i + 1] = v.y;
    }
  }
}
template <int DT>
__device__ __forceinline__ float rnd_dt(float v) {
  if constexpr (DT == H3B_BF16) return __bfloat162float(__float2bfloat16_rn(v));
  else return __half2float(__float2half_rn(v));
}
template <int DT>
__device__ __forceinline__ uint32_t pack_dt2(float a, float b) {
  if constexpr (DT == H3B_BF16) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
  } else {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
}
template <int DT>
__device__ __forceinline__ void unpack2w(uint32_t w, float (&f)[2]) {
  if constexpr (DT == H3B_BF16) {
    f[0] = __uint_as_float(w << 16);
    f[1] = __uint_as_float(w & 0xFFFF0000u);
  } else {
    const float2 v = __half22float2(*reinterpret_cast<const __half2*>(&w));
    f[0] = v.x;
    f[1] = v.y;
  }
}
// 8 consecutive values from element e (a multiple of 8) of a bf16 / fp16 / fp32 array with a 16-byte aligned base
__device__ __forceinline__ void load8(const void* p, int64_t e, int dt, float (&f)[8]) {
  if (dt == H3B_FP32) {
    const float4* q = reinterpret_cast<const float4*>(static_cast<const float*>(p) + e);
    const float4 a = __ldg(q), b = __ldg(q + 1);
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  } else {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(static_cast<const char*>(p) + e * 2));
    if (dt == H3B_BF16) unpack8<H3B_BF16>(u, f);
    else unpack8<H3B_FP16>(u, f);
  }
}


// VPT = 8-element vectors per thread; blockDim.x * VPT * 8 >= H.  The modulation row of token r is token_rows[r] when
// that map is given (negative: none), else the row of the segment holding r.
template <int DT, int VPT>
__global__ void __launch_bounds__(1024) rms_modulate_kernel(const void* __restrict__ x, int64_t ldx, int64_t M, int H,
                                                            const void* __restrict__ w, int w_dtype, float eps,
                                                            const void* __restrict__ shift, const void* __restrict__ scale,
                                                            int64_t ldm, int m_dtype, const SegTable segs,
                                                            const int* __restrict__ token_rows, void* __restrict__ h,
                                                            int64_t ldh) {
  __shared__ float part[32];
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5, nw = (blockDim.x + 31) >> 5;
  const int nvec = H >> 3;
  for (int64_t r = blockIdx.x; r < M; r += gridDim.x) {
    const uint4* xr = reinterpret_cast<const uint4*>(static_cast<const char*>(x) + r * ldx * 2);
    uint4 raw[VPT];
    float ss = 0.f;
#pragma unroll
    for (int v = 0; v < VPT; ++v) {
      const int c = tid + v * blockDim.x;
      raw[v] = c < nvec ? __ldg(xr + c) : make_uint4(0, 0, 0, 0);
      float f[8];
      unpack8<DT>(raw[v], f);
#pragma unroll
      for (int i = 0; i < 8; ++i) ss = __fmaf_rn(f[i], f[i], ss);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
    if (lane == 0) part[wid] = ss;
    __syncthreads();
    float tot = 0.f;
    for (int i = 0; i < nw; ++i) tot = __fadd_rn(tot, part[i]);
    __syncthreads();  // part[] is rewritten by the next row
    const float rs = rsqrtf(__fadd_rn(__fdiv_rn(tot, static_cast<float>(H)), eps));
    int mrow = -1;
    if (token_rows) {
      mrow = token_rows[r];
    } else {
      for (int s = 0; s < segs.n; ++s)
        if (r >= segs.first[s] && r < segs.end[s]) mrow = segs.row[s];
    }
    uint4* hr = reinterpret_cast<uint4*>(static_cast<char*>(h) + r * ldh * 2);
#pragma unroll
    for (int v = 0; v < VPT; ++v) {
      const int c = tid + v * blockDim.x;
      if (c >= nvec) continue;
      float f[8], wv[8], sc[8], sh[8];
      unpack8<DT>(raw[v], f);
      load8(w, 8 * c, w_dtype, wv);
      if (mrow >= 0) {
        load8(scale, mrow * ldm + 8 * c, m_dtype, sc);
        load8(shift, mrow * ldm + 8 * c, m_dtype, sh);
      }
      float o[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float n = rnd_dt<DT>(__fmul_rn(__fmul_rn(f[i], rs), rnd_dt<DT>(wv[i])));
        if (mrow >= 0) {
          const float s1 = rnd_dt<DT>(__fadd_rn(1.0f, rnd_dt<DT>(sc[i])));
          n = rnd_dt<DT>(__fadd_rn(rnd_dt<DT>(__fmul_rn(n, s1)), rnd_dt<DT>(sh[i])));
        }
        o[i] = n;
      }
      hr[c] = make_uint4(pack_dt2<DT>(o[0], o[1]), pack_dt2<DT>(o[2], o[3]), pack_dt2<DT>(o[4], o[5]), pack_dt2<DT>(o[6], o[7]));
    }
  }
}

// Warp-per-row variant for hidden = 256 * VPW (VPW <= 32): lane l holds 8-element vectors l, l + 32, ...; the row sum is
// a per-lane fp32 sum and an xor-shuffle tree, so rows never wait on a CTA barrier and each SM keeps many rows in flight.
template <int DT, int VPW>
__global__ void __launch_bounds__(256) rms_modulate_warp_kernel(const void* __restrict__ x, int64_t ldx, int64_t M,
                                                                const void* __restrict__ w, int w_dtype, float eps,
                                                                const void* __restrict__ shift,
                                                                const void* __restrict__ scale, int64_t ldm, int m_dtype,
                                                                const SegTable segs, const int* __restrict__ token_rows,
                                                                void* __restrict__ h, int64_t ldh) {
  constexpr int H = 256 * VPW;
  const int lane = threadIdx.x & 31;
  const int64_t warp0 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  const bool same_w = w_dtype == DT, same_m = m_dtype == DT;
  for (int64_t r = warp0; r < M; r += nwarps) {
    const uint4* xr = reinterpret_cast<const uint4*>(static_cast<const char*>(x) + r * ldx * 2);
    uint4 raw[VPW];
#pragma unroll
    for (int v = 0; v < VPW; ++v) raw[v] = __ldg(xr + lane + 32 * v);
    float ss = 0.f;
#pragma unroll
    for (int v = 0; v < VPW; ++v) {
      float f[8];
      unpack8<DT>(raw[v], f);
#pragma unroll
      for (int i = 0; i < 8; ++i) ss = __fmaf_rn(f[i], f[i], ss);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
    const float rs = rsqrtf(__fadd_rn(__fdiv_rn(ss, static_cast<float>(H)), eps));
    int mrow = -1;
    if (token_rows) {
      mrow = token_rows[r];
    } else {
      for (int s = 0; s < segs.n; ++s)
        if (r >= segs.first[s] && r < segs.end[s]) mrow = segs.row[s];
    }
    uint4* hr = reinterpret_cast<uint4*>(static_cast<char*>(h) + r * ldh * 2);
    // second pass re-reads the row (an L1/L2 hit) instead of holding VPW vectors across the loop
#pragma unroll 2
    for (int v = 0; v < VPW; ++v) {
      const int c = lane + 32 * v;
      float f[8], wv[8];
      unpack8<DT>(__ldg(xr + c), f);
      load8(w, 8 * c, w_dtype, wv);
      uint32_t o[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float w0 = wv[2 * i], w1 = wv[2 * i + 1];
        if (!same_w) { w0 = rnd_dt<DT>(w0); w1 = rnd_dt<DT>(w1); }
        o[i] = pack_dt2<DT>(__fmul_rn(__fmul_rn(f[2 * i], rs), w0), __fmul_rn(__fmul_rn(f[2 * i + 1], rs), w1));
      }
      if (mrow >= 0) {
        float sc[8], sh[8];
        load8(scale, mrow * ldm + 8 * c, m_dtype, sc);
        load8(shift, mrow * ldm + 8 * c, m_dtype, sh);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          float c0 = sc[2 * i], c1 = sc[2 * i + 1], h0 = sh[2 * i], h1 = sh[2 * i + 1];
          if (!same_m) { c0 = rnd_dt<DT>(c0); c1 = rnd_dt<DT>(c1); h0 = rnd_dt<DT>(h0); h1 = rnd_dt<DT>(h1); }
          float n[2], s1[2], p[2];
          unpack2w<DT>(o[i], n);
          unpack2w<DT>(pack_dt2<DT>(__fadd_rn(1.0f, c0), __fadd_rn(1.0f, c1)), s1);
          unpack2w<DT>(pack_dt2<DT>(__fmul_rn(n[0], s1[0]), __fmul_rn(n[1], s1[1])), p);
          o[i] = pack_dt2<DT>(__fadd_rn(p[0], h0), __fadd_rn(p[1], h1));
        }
      }
      hr[c] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

// Gated residual update of the block (model.py:_gate_ :111-115): for a token with modulation row `row`,
// x = dt(x + other * dt(gate[row])) in fp32 (the product of two dt values is exact in fp32); other tokens unchanged.
template <int DT>
__global__ void __launch_bounds__(256) gate_residual_kernel(void* __restrict__ x, int64_t ldx, const void* __restrict__ other,
                                                            int64_t ldo, int64_t M, int H, const void* __restrict__ gate,
                                                            int64_t ldm, int m_dtype, const SegTable segs,
                                                            const int* __restrict__ token_rows) {
  const int nv = H >> 3;
  const int64_t total = M * nv;
  const bool same_m = m_dtype == DT;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / nv;
    const int c = static_cast<int>(i - r * nv);
    int mrow = -1;
    if (token_rows) {
      mrow = token_rows[r];
    } else {
      for (int s = 0; s < segs.n; ++s)
        if (r >= segs.first[s] && r < segs.end[s]) mrow = segs.row[s];
    }
    if (mrow < 0) continue;
    uint4* xp = reinterpret_cast<uint4*>(static_cast<char*>(x) + (r * ldx + 8 * c) * 2);
    float xv[8], ov[8], gv[8];
    unpack8<DT>(*xp, xv);
    unpack8<DT>(__ldg(reinterpret_cast<const uint4*>(static_cast<const char*>(other) + (r * ldo + 8 * c) * 2)), ov);
    load8(gate, mrow * ldm + 8 * c, m_dtype, gv);
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float g0 = gv[2 * j], g1 = gv[2 * j + 1];
      if (!same_m) { g0 = rnd_dt<DT>(g0); g1 = rnd_dt<DT>(g1); }
      o[j] = pack_dt2<DT>(__fadd_rn(xv[2 * j], __fmul_rn(ov[2 * j], g0)), __fadd_rn(xv[2 * j + 1], __fmul_rn(ov[2 * j + 1], g1)));
    }
    *xp = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

template <int DT>
static int rms_mod_launch_t(const void* x, int64_t ldx, int64_t M, int H, const void* w, int w_dtype, float eps,
                            const void* shift, const void* scale, int64_t ldm, int m_dtype, const SegTable& segs,
                            const int* token_rows, void* h, int64_t ldh, cudaStream_t st) {
  int dev0 = 0, sms0 = 148;
  cudaGetDevice(&dev0);
  cudaDeviceGetAttribute(&sms0, cudaDevAttrMultiProcessorCount, dev0);
  if (H % 256 == 0 && H <= 256 * 32) {
    const int64_t want = (M + 7) / 8;
    const int64_t cap = static_cast<int64_t>(sms0) * 8;
    const int nb = static_cast<int>(want < cap ? want : cap);
#define H3B_RMSW(V) case V: rms_modulate_warp_kernel<DT, V><<<nb, 256, 0, st>>>(x, ldx, M, w, w_dtype, eps, shift, scale, ldm, m_dtype, segs, token_rows, h, ldh); break
    switch (H / 256) {
      H3B_RMSW(1); H3B_RMSW(2); H3B_RMSW(3); H3B_RMSW(4); H3B_RMSW(5); H3B_RMSW(6); H3B_RMSW(7); H3B_RMSW(8);
      H3B_RMSW(9); H3B_RMSW(10); H3B_RMSW(11); H3B_RMSW(12); H3B_RMSW(13); H3B_RMSW(14); H3B_RMSW(15); H3B_RMSW(16);
      H3B_RMSW(17); H3B_RMSW(18); H3B_RMSW(19); H3B_RMSW(20); H3B_RMSW(21); H3B_RMSW(22); H3B_RMSW(23); H3B_RMSW(24);
      default: goto cta_path;
    }
#undef H3B_RMSW
    return check_launch("rms_modulate_warp_kernel");
  }
cta_path:
  const int nvec = H / 8;
  int threads = nvec < 1024 ? ((nvec + 31) / 32) * 32 : 1024;
  const int vpt = (nvec + threads - 1) / threads;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t cap = static_cast<int64_t>(sms) * (2048 / threads);
  const int blocks = static_cast<int>(M < cap ? M : cap);
#define H3B_RMSMOD(V) rms_modulate_kernel<DT, V><<<blocks, threads, 0, st>>>(x, ldx, M, H, w, w_dtype, eps, shift, scale, ldm, m_dtype, segs, token_rows, h, ldh)
  switch (vpt) {
    case 1: H3B_RMSMOD(1); break;
    case 2: H3B_RMSMOD(2); break;
    case 3: H3B_RMSMOD(3); break;
    case 4: H3B_RMSMOD(4); break;
    default: return fail(H3B_ERR_UNSUPPORTED, "rms_modulate: hidden size above 32768");
  }
#undef H3B_RMSMOD
  return check_launch("rms_modulate_kernel");
}

int gate_residual_launch(void* x, int x_dtype, int64_t ldx, const void* other, int64_t ldo, int64_t M, int H,
                         const void* gate, int64_t ldm, int m_dtype, const int32_t* segs, int nseg,
                         const int32_t* token_rows, cudaStream_t st) {
  SegTable t{};
  t.n = nseg;
  for (int i = 0; i < nseg; ++i) {
    t.first[i] = segs[3 * i];
    t.end[i] = segs[3 * i + 1];
    t.row[i] = segs[3 * i + 2];
  }
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t total = M * (H / 8);
  const int64_t want = (total + 255) / 256, cap = static_cast<int64_t>(sms) * 8;
  const int nb = static_cast<int>(want < cap ? want : cap);
  if (x_dtype == H3B_BF16) gate_residual_kernel<H3B_BF16><<<nb, 256, 0, st>>>(x, ldx, other, ldo, M, H, gate, ldm, m_dtype, t, token_rows);
  else if (x_dtype == H3B_FP16) gate_residual_kernel<H3B_FP16><<<nb, 256, 0, st>>>(x, ldx, other, ldo, M, H, gate, ldm, m_dtype, t, token_rows);
  else return fail(H3B_ERR_UNSUPPORTED, "gate_residual: x must be bf16 or fp16");
  return check_launch("gate_residual_kernel");
}

int rms_modulate_launch(const void* x, int x_dtype, int64_t ldx, int64_t M, int H, const void* w, int w_dtype, float eps,
                        const void* shift, const void* scale, int64_t ldm, int m_dtype, const int32_t* segs, int nseg,
                        const int32_t* token_rows, void* h, int64_t ldh, cudaStream_t st) {
  SegTable t{};
  t.n = nseg;
  for (int i = 0; i < nseg; ++i) {
    t.first[i] = segs[3 * i];
    t.end[i] = segs[3 * i + 1];
    t.row[i] = segs[3 * i + 2];
  }
  if (x_dtype == H3B_BF16) return rms_mod_launch_t<H3B_BF16>(x, ldx, M, H, w, w_dtype, eps, shift, scale, ldm, m_dtype, t, token_rows, h, ldh, st);
  if (x_dtype == H3B_FP16) return rms_mod_launch_t<H3B_FP16>(x, ldx, M, H, w, w_dtype, eps, shift, scale, ldm, m_dtype, t, token_rows, h, ldh, st);
  return fail(H3B_ERR_UNSUPPORTED, "rms_modulate: x must be bf16 or fp16");
}

}  // namespace h3b
