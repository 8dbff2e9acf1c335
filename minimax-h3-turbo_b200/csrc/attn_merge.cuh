// Merge of softmax attention computed over disjoint key sets (the ring key/value exchange of the token-sharded block).
//
// For each (head h, query q):  new = log(exp(L) + exp(l)),  A = A * exp(L - new) + fp32(o) * exp(l - new),  L = new
// where (A, L) is the running fp32 output and log-sum-exp and (o, l) the attention over the next key set.  `first`
// initialises (A, L) from (o, l); `out` (optional) receives dt(A) transposed to [Sq, H * D] rows, the layout the output
// projection reads.  One warp per (h, q); D/32 values per lane; HBM-bound (4 + 2 + 4 bytes per value, +2 with `out`).
#include "h3b_common.cuh"

namespace h3b {

template <int VPL>  // values per lane = D / 32
__global__ void __launch_bounds__(256) attn_merge_kernel(float* __restrict__ acc, float* __restrict__ acc_lse,
                                                         const __nv_bfloat16* __restrict__ o, int64_t o_sh, int64_t o_sq,
                                                         const float* __restrict__ lse, int64_t H, int64_t Sq, int first,
                                                         __nv_bfloat16* __restrict__ out, int64_t ldo) {
  constexpr int D = 32 * VPL;
  const int lane = threadIdx.x & 31;
  const int64_t rows = H * Sq;
  for (int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; row < rows;
       row += (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5) {
    const int64_t h = row / Sq, q = row - h * Sq;
    const __nv_bfloat16* orow = o + h * o_sh + q * o_sq;
    float* arow = acc + row * D;
    const float l = lse[row];
    float res[VPL];
    if (first) {
#pragma unroll
      for (int i = 0; i < VPL; ++i) res[i] = __bfloat162float(orow[lane + 32 * i]);
      if (lane == 0) acc_lse[row] = l;
    } else {
      const float L = acc_lse[row];
      const float m = fmaxf(L, l);
      if (m == -INFINITY) {  // neither key set had a key for this query (empty shards): nothing to weigh, output 0
#pragma unroll
        for (int i = 0; i < VPL; ++i) res[i] = 0.f;
      } else {
        // log(exp(L) + exp(l)) = m + log(exp(L - m) + exp(l - m)), both exponents <= 0; an empty side has weight 0
        const float ea = expf(L - m), eb = expf(l - m);
        const float sum = ea + eb;
        const float wa = ea / sum, wb = eb / sum;
#pragma unroll
        for (int i = 0; i < VPL; ++i)
          res[i] = fmaf(wa == 0.f ? 0.f : arow[lane + 32 * i], wa, wb == 0.f ? 0.f : __bfloat162float(orow[lane + 32 * i]) * wb);
        if (lane == 0) acc_lse[row] = m + logf(sum);
      }
    }
    if (out) {
      __nv_bfloat16* dst = out + q * ldo + h * D;
#pragma unroll
      for (int i = 0; i < VPL; ++i) dst[lane + 32 * i] = __float2bfloat16_rn(res[i]);
    } else {
#pragma unroll
      for (int i = 0; i < VPL; ++i) arow[lane + 32 * i] = res[i];
    }
  }
}

int attn_merge_launch(float* acc, float* acc_lse, const void* o, int64_t o_sh, int64_t o_sq, const float* lse, int64_t H,
                      int64_t Sq, int D, int first, void* out, int64_t ldo, cudaStream_t st) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t warps = H * Sq;
  const int64_t want = (warps + 7) / 8, cap = static_cast<int64_t>(sms) * 8;
  const int nb = static_cast<int>(want < cap ? want : cap);
  const auto* ob = static_cast<const __nv_bfloat16*>(o);
  auto* outb = static_cast<__nv_bfloat16*>(out);
  switch (D) {
    case 64: attn_merge_kernel<2><<<nb, 256, 0, st>>>(acc, acc_lse, ob, o_sh, o_sq, lse, H, Sq, first, outb, ldo); break;
    case 128: attn_merge_kernel<4><<<nb, 256, 0, st>>>(acc, acc_lse, ob, o_sh, o_sq, lse, H, Sq, first, outb, ldo); break;
    case 256: attn_merge_kernel<8><<<nb, 256, 0, st>>>(acc, acc_lse, ob, o_sh, o_sq, lse, H, Sq, first, outb, ldo); break;
    default: return fail(H3B_ERR_UNSUPPORTED, "attn_merge: head_dim must be 64, 128 or 256");
  }
  return check_launch("attn_merge_kernel");
}

}  // namespace h3b
