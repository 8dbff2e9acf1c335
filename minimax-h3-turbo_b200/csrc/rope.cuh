// Fused per-head RMSNorm + split-half rotary embedding of q and k, in place.
//
// Reference semantics (h3turbo/h3/layout.py, the bit-exact "torch" form of the fused kernel, :309-326 and :348-355):
//   per head of D channels:  lane l (of 32) sums x_{l}^2, x_{l+32}^2, ... sequentially in fp32; a halving tree over the
//   lanes (acc[i] += acc[i + off], off = 16 .. 1) gives the sum;  n = dt((x * rsqrt(sum / D + eps)) * w), each product
//   rounded once in fp32;  then with half = cos.shape[1], for j < half:
//     o_j        = dt(n_j c - n_{j+half} s),   o_{j+half} = dt(n_j s + n_{j+half} c)      (fp32 products, one rounding)
//   and channels >= 2 half keep n.
// One warp per (token, head): lane l holds channels l + 32 i, exactly the reference's lanes, so the sum needs no
// reordering; the normalised head is staged in shared memory (one row per warp) so each lane can read its rotation
// partner.  HBM-bound: 2 * 2 * D bytes per head (read + write of q and k), the cos/sin rows come from L2.
#include "h3b_common.cuh"

namespace h3b {

template <int DT>
__device__ __forceinline__ float ld_act(const void* p, int64_t i) {
  if constexpr (DT == H3B_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
  else if constexpr (DT == H3B_FP16) return __half2float(static_cast<const __half*>(p)[i]);
  else return static_cast<const float*>(p)[i];
}
template <int DT>
__device__ __forceinline__ float rnd_act(float v) {
  if constexpr (DT == H3B_BF16) return __bfloat162float(__float2bfloat16_rn(v));
  else return __half2float(__float2half_rn(v));
}
template <int DT>
__device__ __forceinline__ void st_act(void* p, int64_t i, float v) {
  if constexpr (DT == H3B_BF16) static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else static_cast<__half*>(p)[i] = __float2half_rn(v);
}
__device__ __forceinline__ float ld_any(const void* p, int64_t i, int dt) {
  switch (dt) {
    case H3B_BF16: return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
    case H3B_FP16: return __half2float(static_cast<const __half*>(p)[i]);
    default: return static_cast<const float*>(p)[i];
  }
}

template <int TDT>  // the cos / sin tables' dtype, fixed per launch
__device__ __forceinline__ float ld_tab(const void* p, int64_t i) {
  if constexpr (TDT == H3B_BF16) return __bfloat162float(__ldg(static_cast<const __nv_bfloat16*>(p) + i));
  else if constexpr (TDT == H3B_FP16) return __half2float(__ldg(static_cast<const __half*>(p) + i));
  else return __ldg(static_cast<const float*>(p) + i);
}

constexpr int ROPE_WARPS = 8;

// NI = D / 32 channels per lane; HPI heads of one token per warp item (their loads are issued together).
// Items: (token, head group) of q, then of k.
template <int DT, int NI, int HPI, int TDT>
__global__ void __launch_bounds__(32 * ROPE_WARPS) qk_norm_rope_kernel(
    void* __restrict__ q, int64_t ldq, void* __restrict__ k, int64_t ldk, int64_t S, int heads,
    const void* __restrict__ wq, const void* __restrict__ wk, int w_dtype, float eps, const void* __restrict__ cs,
    const void* __restrict__ sn, int64_t ldt, int t_dtype, int half) {
  constexpr int D = 32 * NI;
  __shared__ float stage[ROPE_WARPS][HPI][D];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int groups = heads / HPI;
  const int64_t per = S * groups;
  const int64_t items = (q ? per : 0) + (k ? per : 0);
  const float inv_d = 1.0f / static_cast<float>(D);  // exact: D is a power of two
  float wv[2][NI];
#pragma unroll
  for (int i = 0; i < NI; ++i) {
    wv[0][i] = q ? ld_any(wq, lane + 32 * i, w_dtype) : 0.f;
    wv[1][i] = k ? ld_any(wk, lane + 32 * i, w_dtype) : 0.f;
  }
  for (int64_t it = static_cast<int64_t>(blockIdx.x) * ROPE_WARPS + wid; it < items;
       it += static_cast<int64_t>(gridDim.x) * ROPE_WARPS) {
    const bool is_k = !q || it >= per;
    const int64_t r = (q && it >= per) ? it - per : it;
    const int64_t tok = r / groups, h0 = (r - tok * groups) * HPI;
    void* base = is_k ? k : q;
    const int64_t off = tok * (is_k ? ldk : ldq) + h0 * D;
    float x[HPI][NI];
#pragma unroll
    for (int hh = 0; hh < HPI; ++hh)
#pragma unroll
      for (int i = 0; i < NI; ++i) x[hh][i] = ld_act<DT>(base, off + hh * D + lane + 32 * i);
    float acc[HPI];
#pragma unroll
    for (int hh = 0; hh < HPI; ++hh) {
      acc[hh] = __fmul_rn(x[hh][0], x[hh][0]);
#pragma unroll
      for (int i = 1; i < NI; ++i) acc[hh] = __fadd_rn(acc[hh], __fmul_rn(x[hh][i], x[hh][i]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int hh = 0; hh < HPI; ++hh) acc[hh] = __fadd_rn(acc[hh], __shfl_down_sync(0xffffffffu, acc[hh], o));
    float n[HPI][NI];
#pragma unroll
    for (int hh = 0; hh < HPI; ++hh) {
      const float rs = rsqrtf(__fadd_rn(__fmul_rn(__shfl_sync(0xffffffffu, acc[hh], 0), inv_d), eps));
#pragma unroll
      for (int i = 0; i < NI; ++i) {
        n[hh][i] = rnd_act<DT>(__fmul_rn(__fmul_rn(x[hh][i], rs), is_k ? wv[1][i] : wv[0][i]));
        stage[wid][hh][lane + 32 * i] = n[hh][i];
      }
    }
    __syncwarp();
    const int64_t trow = tok * ldt;
#pragma unroll
    for (int i = 0; i < NI; ++i) {
      const int c = lane + 32 * i;
      float cv = 0.f, sv = 0.f;
      if (c < 2 * half) {
        const int j = c < half ? c : c - half;
        cv = ld_tab<TDT>(cs, trow + j);
        sv = ld_tab<TDT>(sn, trow + j);
      }
#pragma unroll
      for (int hh = 0; hh < HPI; ++hh) {
        float o = n[hh][i];
        if (c < half) o = __fsub_rn(__fmul_rn(n[hh][i], cv), __fmul_rn(stage[wid][hh][c + half], sv));
        else if (c < 2 * half) o = __fadd_rn(__fmul_rn(stage[wid][hh][c - half], sv), __fmul_rn(n[hh][i], cv));
        st_act<DT>(base, off + hh * D + c, o);
      }
    }
    __syncwarp();  // the next item overwrites this warp's staging rows
  }
}

template <int DT>
static int qk_launch_d(void* q, int64_t ldq, void* k, int64_t ldk, int64_t S, int heads, int D, const void* wq,
                       const void* wk, int w_dtype, float eps, const void* cs, const void* sn, int64_t ldt, int t_dtype,
                       int half, cudaStream_t st) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int hpi = heads % 4 == 0 && D <= 128 ? 4 : heads % 2 == 0 ? 2 : 1;
  const int64_t items = S * (heads / hpi) * ((q ? 1 : 0) + (k ? 1 : 0));
  const int64_t want = (items + ROPE_WARPS - 1) / ROPE_WARPS;
  const int64_t cap = static_cast<int64_t>(sms) * 8;  // 8 resident 256-thread CTAs per SM
  const int blocks = static_cast<int>(want < cap ? want : cap);
#define H3B_QKR_T(NI, HPI, TDT) qk_norm_rope_kernel<DT, NI, HPI, TDT><<<blocks, 32 * ROPE_WARPS, 0, st>>>(q, ldq, k, ldk, S, heads, wq, wk, w_dtype, eps, cs, sn, ldt, t_dtype, half)
#define H3B_QKR(NI, HPI) do { if (t_dtype == H3B_BF16) H3B_QKR_T(NI, HPI, H3B_BF16); else if (t_dtype == H3B_FP16) H3B_QKR_T(NI, HPI, H3B_FP16); else H3B_QKR_T(NI, HPI, H3B_FP32); } while (0)
#define H3B_QKR_H(NI) if (hpi == 4) H3B_QKR(NI, 4); else if (hpi == 2) H3B_QKR(NI, 2); else H3B_QKR(NI, 1)
  switch (D) {
    case 32: H3B_QKR_H(1); break;
    case 64: H3B_QKR_H(2); break;
    case 128: H3B_QKR_H(4); break;
    case 256: if (hpi == 1) H3B_QKR(8, 1); else H3B_QKR(8, 2); break;
    default: return fail(H3B_ERR_UNSUPPORTED, "qk_norm_rope: head_dim must be 32, 64, 128 or 256");
  }
#undef H3B_QKR_H
#undef H3B_QKR
#undef H3B_QKR_T
  return check_launch("qk_norm_rope_kernel");
}

int qk_norm_rope_launch(void* q, int64_t ldq, void* k, int64_t ldk, int x_dtype, int64_t S, int heads, int D,
                        const void* wq, const void* wk, int w_dtype, float eps, const void* cs, const void* sn,
                        int64_t ldt, int t_dtype, int half, cudaStream_t st) {
  if (x_dtype == H3B_BF16) return qk_launch_d<H3B_BF16>(q, ldq, k, ldk, S, heads, D, wq, wk, w_dtype, eps, cs, sn, ldt, t_dtype, half, st);
  if (x_dtype == H3B_FP16) return qk_launch_d<H3B_FP16>(q, ldq, k, ldk, S, heads, D, wq, wk, w_dtype, eps, cs, sn, ldt, t_dtype, half, st);
  return fail(H3B_ERR_UNSUPPORTED, "qk_norm_rope: q/k must be bf16 or fp16 (fp32 takes the reference's eager form)");
}

}  // namespace h3b
