// Kernel KB, small-M form: the W4A8 GEMM for M <= 256 tokens, int4 weight decoded in the producer warps, K split
// across CTAs so that every SM works although N / BN weight tiles alone would leave many idle.
//
// At small M the weight dominates the bytes and every output tile needs the whole K: one CTA per (N tile) gives
// 20-108 CTAs for N = 5120-13824 on 148 SMs, each walking all of K.  Here a work unit is (N tile, K range): CTA u owns
// output columns [BN nt, BN nt + BN) for ALL M rows (up to two 128-row subtiles, so each weight tile is decoded once)
// and the k-blocks [kb0, kb1) of split s.  Integer partial sums are exact, so splitting K changes no bit of the result.
//
//   warp 0      TMA producer of the packed int4 weight tiles (BN x 64 bytes per k-block) into a deep ring (P ring)
//   warp 6      TMA producer of the activation-code tiles (MS x 128 x 128 bytes per k-block) into the AB ring
//   warps 7..   decoders: a P stage -> the BN x 128 int8 B tile of an AB stage (level tables + byte permutes, exactly
//               decode.cuh's levels, 128-byte swizzle), then fence.proxy.async and an arrival per warp
//   warp 1      MMA issuer: per k-block and M subtile 4 x tcgen05.mma.kind::i8 (K = 32 each) into its TMEM accumulator
//   warps 2-5   epilogue: wait for the accumulator, then (with every warp of the CTA, after the roles) stage and store.
//               The S CTAs of one output tile (S K splits; S = 1 included) form a thread-block cluster: CTA p owns 1/S
//               of the tile's rows, every CTA stores its raw int32 partial sums of each row straight from TMEM into
//               the owner's (by then idle) ring memory (distributed shared memory stores, posted; its own rows
//               locally), and after a cluster barrier each owner adds up its rows over the S slots in rank order from
//               its own shared memory and all its warps apply the W4A8 epilogue (as gemm_sm100.cuh) and store the
//               output -- no partial sums in HBM, no second kernel, no remote loads.
// The P ring is separate from (and deeper than) the AB ring, so weight bytes keep streaming from HBM while the tensor
// core works on earlier k-blocks.  One work unit per CTA; every mbarrier wait bounded (h3b_common.cuh), and every CTA
// reaches every cluster barrier whatever happened before, so no CTA waits for a peer that left; after the last one no
// CTA touches another's shared memory.
#pragma once

#include "decode.cuh"
#include "gemm_sm100.cuh"
#include "gemm_w4.cuh"

namespace h3b {

// Epilogue parameters, runtime values: one kernel instantiation serves every output dtype, quant mode and bias choice.
struct W4sEpi {
  const float* xs;     // [M] per-row activation scales (unused for int32 output)
  const float* sch;    // [N] per-channel weight scales
  const void* bias;    // [N] of the output dtype, or null
  void* out;           // [M, ldo] output
  int64_t ldo;
  int out_dtype;       // H3B_BF16 / H3B_FP16 / H3B_FP32 / H3B_INT32
  int qmode;           // H3B_QMODE_CK / H3B_QMODE_EAGER
};

template <int BN, int MS>
struct W4sCfg {
  // 16-weight chunks per decoder thread per k-block: 16 decoder warps for BN 128 and 256, 12 for 192 -- enough warps
  // per scheduler to hide the shared-memory and permute latencies of the decode behind each other
  static constexpr int CPT = BN == 128 ? 2 : 4;
  static constexpr int DWARPS = BN * 8 / (32 * CPT);  // decoder warps (a thread owns CPT chunks of one B row)
  static constexpr int LA = 4;                        // k-blocks of group scales each decoder thread loads ahead
  static constexpr int A_BYTES = BM * BK;             // one 128-row activation subtile of one k-block
  static constexpr int B_BYTES = BN * BK;
  static constexpr int P_BYTES = BN * (BK / 2);
  static constexpr int BUDGET = 210 * 1024;
  // Three rings.  The activation tiles come from L2 with a latency of a few microseconds when every SM streams at
  // once, so their ring is the deepest the budget allows; the decoded weight tiles are produced in shared memory and
  // need only double buffering; the packed weight tiles take the rest.
  static constexpr int A_STAGES = MS == 1 ? 6 : (BN == 128 ? 4 : 3);
  static constexpr int B_STAGES = MS == 1 && BN == 128 ? 3 : 2;
  static constexpr int P_LEFT = (BUDGET - A_STAGES * MS * A_BYTES - B_STAGES * B_BYTES) / P_BYTES;
  static constexpr int P_STAGES = P_LEFT > 10 ? 10 : P_LEFT;
  static constexpr int TMEM_COLS = MS * BN <= 128 ? 128 : (MS * BN <= 256 ? 256 : 512);
  static constexpr int THREADS = 32 * (7 + DWARPS);
  static constexpr int SMEM = 1024 + A_STAGES * MS * A_BYTES + B_STAGES * B_BYTES + P_STAGES * P_BYTES + 4096 + 512;
  static constexpr uint32_t IDESC = idesc_i8(BM, BN);
  static_assert(P_STAGES >= 2 && CPT * 32 * DWARPS == BN * 8 && 8 % CPT == 0, "bad small-M GEMM configuration");
  // the split-K receive area of one 128-row subtile, in the rings: [S][ceil(128 / S)][BN + 4] int32 (rows 16 bytes
  // apart in bank terms); S ceil(128 / S) <= 128 + 7 rows for S <= 8
  static constexpr int RED_STRIDE = BN + 4;
  static constexpr int RED_WORDS = (BM + 7) * RED_STRIDE;  // one subtile's receive area
  static constexpr int RING_BYTES = A_STAGES * MS * A_BYTES + B_STAGES * B_BYTES + P_STAGES * P_BYTES;
  static_assert(RED_WORDS * 4 <= RING_BYTES, "the split-K receive area lives in the ring memory");
  static_assert(SMEM <= 227 * 1024, "shared memory");
  static_assert(2 * BN + MS * BM <= 1024, "the epilogue constants fit the 4 KB level-table area");
};

// 16 bytes into this CTA's shared memory (`addr`: a shared::cta address)
__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}
// 16 bytes into a cluster CTA's shared memory (`addr`: a shared::cluster address; a posted store)
__device__ __forceinline__ void st_cluster_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared::cluster.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

// The W4A8 epilogue of `n` (<= 8) consecutive accumulators of one row, runtime dtype / mode (the same operations, in the
// same order, as epilogue_row32: (fp32(acc) * xs) * s_ch or fp32(acc) * (xs * s_ch), rounded to the output dtype, then
// + bias and a second rounding), stored at column n0 of `orow`.  `sch` / `bias`: the channel scales and the bias (as
// fp32, exact for every bias dtype; null without a bias) of these columns, staged in shared memory.
__device__ __forceinline__ void w4s_store8(const int32_t (&a)[8], int n, float xsr, const float* sch, const float* bias,
                                           int out_dtype, int qmode, char* orow, int64_t n0, bool vec) {
  if (out_dtype == H3B_INT32) {
    int32_t* o = reinterpret_cast<int32_t*>(orow) + n0;
    if (vec) {
      reinterpret_cast<int4*>(o)[0] = make_int4(a[0], a[1], a[2], a[3]);
      reinterpret_cast<int4*>(o)[1] = make_int4(a[4], a[5], a[6], a[7]);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (j < n) o[j] = a[j];
    }
    return;
  }
  const float4 s0 = reinterpret_cast<const float4*>(sch)[0], s1 = reinterpret_cast<const float4*>(sch)[1];
  const float sv[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
  float bv[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (bias) {
    const float4 b0 = reinterpret_cast<const float4*>(bias)[0], b1 = reinterpret_cast<const float4*>(bias)[1];
    bv[0] = b0.x; bv[1] = b0.y; bv[2] = b0.z; bv[3] = b0.w; bv[4] = b1.x; bv[5] = b1.y; bv[6] = b1.z; bv[7] = b1.w;
  }
  float v[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float f = __int2float_rn(a[j]);
    v[j] = qmode == H3B_QMODE_CK ? __fmul_rn(__fmul_rn(f, xsr), sv[j]) : __fmul_rn(f, __fmul_rn(xsr, sv[j]));
  }
  if (out_dtype == H3B_FP32) {
    if (bias) {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = __fadd_rn(v[j], bv[j]);
    }
    float* o = reinterpret_cast<float*>(orow) + n0;
    if (vec) {
      reinterpret_cast<float4*>(o)[0] = make_float4(v[0], v[1], v[2], v[3]);
      reinterpret_cast<float4*>(o)[1] = make_float4(v[4], v[5], v[6], v[7]);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (j < n) o[j] = v[j];
    }
    return;
  }
  const bool bf = out_dtype == H3B_BF16;
  uint16_t h[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    float r = bf ? __bfloat162float(__float2bfloat16_rn(v[j])) : __half2float(__float2half_rn(v[j]));
    if (bias) r = __fadd_rn(r, bv[j]);
    if (bf) {
      const __nv_bfloat16 t = __float2bfloat16_rn(r);
      h[j] = *reinterpret_cast<const uint16_t*>(&t);
    } else {
      const __half t = __float2half_rn(r);
      h[j] = *reinterpret_cast<const uint16_t*>(&t);
    }
  }
  uint16_t* o = reinterpret_cast<uint16_t*>(orow) + n0;
  if (vec) {
    *reinterpret_cast<uint4*>(o) = make_uint4(h[0] | (uint32_t(h[1]) << 16), h[2] | (uint32_t(h[3]) << 16),
                                              h[4] | (uint32_t(h[5]) << 16), h[6] | (uint32_t(h[7]) << 16));
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (j < n) o[j] = h[j];
  }
}

template <int BN, int MS, int SDT>
__global__ void __launch_bounds__(W4sCfg<BN, MS>::THREADS, 1)
    gemm_w4s_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmP,
                    const void* __restrict__ s_rel, int64_t lds, const float* __restrict__ codebook, const W4sEpi epi,
                    int M, int N, int K, int splits, int m_tiles) {
  using C = W4sCfg<BN, MS>;
  constexpr int GROUP = SDT == H3B_FP8_E4M3 ? 16 : 128;
  extern __shared__ __align__(1024) unsigned char w4s_smem[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(w4s_smem) + 1023) & ~uintptr_t(1023));
  unsigned char* sA = smem;                                    // [A_STAGES][MS][A_BYTES]
  unsigned char* sB = sA + C::A_STAGES * MS * C::A_BYTES;      // [B_STAGES][B_BYTES]
  unsigned char* sP = sB + C::B_STAGES * C::B_BYTES;           // [P_STAGES][P_BYTES]
  uint4* lut = reinterpret_cast<uint4*>(sP + C::P_STAGES * C::P_BYTES);  // fp8: the 256 level tables
  uint64_t* pkfull = reinterpret_cast<uint64_t*>(lut + 256);
  uint64_t* pkempty = pkfull + C::P_STAGES;
  uint64_t* afull = pkempty + C::P_STAGES;
  uint64_t* aempty = afull + C::A_STAGES;
  uint64_t* bfull = aempty + C::A_STAGES;
  uint64_t* bempty = bfull + C::B_STAGES;
  uint64_t* tfull = bempty + C::B_STAGES;
  uint64_t* mdone = tfull + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mdone + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tiles = (N + BN - 1) / BN;
  // unit = (M tile, N tile, split), split fastest: the S splits of one output tile are one cluster, split = cluster rank
  const int split = blockIdx.x % splits, tile = blockIdx.x / splits;
  const int nt = tile % n_tiles, mt = tile / n_tiles;
  const int row_base = mt * MS * BM;  // first activation / output row of this CTA
  const int num_kb = (K + BK - 1) / BK;
  const int kb0 = static_cast<int>(static_cast<int64_t>(split) * num_kb / splits);
  const int kb1 = static_cast<int>(static_cast<int64_t>(split + 1) * num_kb / splits);
  const int nkb = kb1 - kb0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::P_STAGES; ++s) {
      mbar_init(&pkfull[s], 1);
      mbar_init(&pkempty[s], C::DWARPS);
    }
    for (int s = 0; s < C::A_STAGES; ++s) {
      mbar_init(&afull[s], 1);
      mbar_init(&aempty[s], 1);
    }
    for (int s = 0; s < C::B_STAGES; ++s) {
      mbar_init(&bfull[s], C::DWARPS);
      mbar_init(&bempty[s], 1);
    }
    mbar_init(tfull, 1);
    mbar_init(mdone, 1);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if constexpr (SDT == H3B_FP8_E4M3) {
    if (warp >= 7) {
      float cb[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) cb[i] = __ldg(codebook + i);
      for (int b = threadIdx.x - 224; b < 256; b += 32 * C::DWARPS) lut[b] = level_table(cb, fp8e4m3_to_f32(static_cast<uint32_t>(b)));
    }
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmP);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {  // ------------------------------------------------------ packed weight tiles -> P ring
      int ps = 0;
      uint32_t ph = 0;
      int fills = 0;
      for (int i = 0; i < nkb; ++i) {
        if (!mbar_wait(&pkempty[ps], ph ^ 1u, abort_flag)) break;
        mbar_arrive_expect_tx(&pkfull[ps], C::P_BYTES);
        tma_load_2d(sP + ps * C::P_BYTES, &tmP, &pkfull[ps], (kb0 + i) * (BK / 2), nt * BN);
        ++fills;
        if (++ps == C::P_STAGES) { ps = 0; ph ^= 1u; }
      }
      for (int j = fills > C::P_STAGES ? fills - C::P_STAGES : 0; j < fills; ++j)  // drain this CTA's own copies
        if (!mbar_wait_drain(&pkfull[j % C::P_STAGES], static_cast<uint32_t>((j / C::P_STAGES) & 1))) break;
    }
  } else if (warp == 6) {
    if (lane == 0) {  // ------------------------------------------------------ activation tiles -> A ring
      int as = 0;
      uint32_t ph = 0;
      int fills = 0;
      for (int i = 0; i < nkb; ++i) {
        if (!mbar_wait(&aempty[as], ph ^ 1u, abort_flag)) break;
        mbar_arrive_expect_tx(&afull[as], MS * C::A_BYTES);
#pragma unroll
        for (int ms = 0; ms < MS; ++ms)
          tma_load_2d(sA + (as * MS + ms) * C::A_BYTES, &tmA, &afull[as], (kb0 + i) * BK, row_base + ms * BM);
        ++fills;
        if (++as == C::A_STAGES) { as = 0; ph ^= 1u; }
      }
      for (int j = fills > C::A_STAGES ? fills - C::A_STAGES : 0; j < fills; ++j)
        if (!mbar_wait_drain(&afull[j % C::A_STAGES], static_cast<uint32_t>((j / C::A_STAGES) & 1))) break;
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ------------------------------------------------------ MMA issuer
      int as = 0, bs = 0;
      uint32_t aph = 0, bph = 0;
      bool ok = true;
      for (int i = 0; i < nkb && ok; ++i) {
        if (!mbar_wait(&afull[as], aph, abort_flag) || !mbar_wait(&bfull[bs], bph, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t b0 = smem_u32(sB + bs * C::B_BYTES);
#pragma unroll
        for (int ms = 0; ms < MS; ++ms) {
          const uint32_t a0 = smem_u32(sA + (as * MS + ms) * C::A_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 32; ++k)
            mma_i8(tmem_base + static_cast<uint32_t>(ms * BN), smem_desc_sw128(a0 + 32 * k), smem_desc_sw128(b0 + 32 * k),
                   C::IDESC, (i | k) != 0);
        }
        mma_commit(&aempty[as]);  // both slots free once these MMAs complete
        mma_commit(&bempty[bs]);
        if (++as == C::A_STAGES) { as = 0; aph ^= 1u; }
        if (++bs == C::B_STAGES) { bs = 0; bph ^= 1u; }
      }
      if (ok) mma_commit(tfull);
      mma_commit(mdone);
      mbar_wait_drain(mdone, 0);
    }
  } else if (warp < 6) {  // ------------------------------------------------------------------- epilogue
    // the accumulator is complete once the last MMA has committed; the epilogue proper runs after the roles, with every
    // warp of the CTA (below)
    mbar_wait(tfull, 0, abort_flag);
  } else {  // -------------------------------------------------------------------------------------- decoders
    const int dt = threadIdx.x - 224;             // 0 .. 32 DWARPS - 1
    const int r_loc = (dt * C::CPT) >> 3;         // this thread's row of the B tile
    const int j0 = (dt * C::CPT) & 7;             // its first 16-weight chunk in the row
    // group-128 scales: the TPR adjacent lanes of one weight row build its level table together, WPT of the four
    // table words each, and exchange them by shuffles
    constexpr int TPR = 8 / C::CPT, WPT = 4 / TPR;
    float cbm[4 * WPT];  // the codebook entries of this lane's table words
    if constexpr (SDT != H3B_FP8_E4M3) {
#pragma unroll
      for (int e = 0; e < 4 * WPT; ++e) cbm[e] = __ldg(codebook + 4 * WPT * (lane % TPR) + e);
    }
    auto table = [&](float sc) -> uint4 {
      uint32_t mine[WPT];
#pragma unroll
      for (int w = 0; w < WPT; ++w)
        mine[w] = pack4(level_of(cbm[4 * w], sc), level_of(cbm[4 * w + 1], sc), level_of(cbm[4 * w + 2], sc),
                        level_of(cbm[4 * w + 3], sc));
      uint32_t tw[4];
#pragma unroll
      for (int w = 0; w < 4; ++w) tw[w] = __shfl_sync(0xffffffffu, mine[w % WPT], (lane & ~(TPR - 1)) | (w / WPT));
      return make_uint4(tw[0], tw[1], tw[2], tw[3]);
    };
    const int n = nt * BN + r_loc;
    const bool row_ok = n < N;
    const unsigned char* srow = static_cast<const unsigned char*>(s_rel) +
                                static_cast<int64_t>(row_ok ? n : 0) * lds * (SDT == H3B_FP8_E4M3 ? 1 : (SDT == H3B_FP32 ? 4 : 2));
    // this thread's group scales of k-block i: the one scale of its row (group-128 formats, as a float) or the scale
    // byte of each of its chunks (fp8 group 16); plain global loads, issued LA k-blocks before their use
    auto load_scales = [&](int i, float& g, uint32_t (&f8)[C::CPT]) {
      const int64_t kbase = static_cast<int64_t>(kb0 + i) * BK;
      if constexpr (SDT == H3B_FP8_E4M3) {
#pragma unroll
        for (int c = 0; c < C::CPT; ++c) {
          const int64_t e0 = kbase + 16 * (j0 + c);
          f8[c] = (row_ok && i < nkb && e0 < K) ? static_cast<uint32_t>(srow[e0 / GROUP]) : 0u;
        }
      } else {
        const int64_t e0 = kbase + 16 * j0;
        g = (row_ok && i < nkb && e0 < K) ? scale_at<SDT>(srow, e0 / GROUP) : 0.f;
      }
    };
    float sg[C::LA];
    uint32_t s8[C::LA][C::CPT];
#pragma unroll
    for (int u = 0; u < C::LA; ++u) {
      sg[u] = 0.f;
#pragma unroll
      for (int c = 0; c < C::CPT; ++c) s8[u][c] = 0u;
      load_scales(u, sg[u], s8[u]);
    }
    int ps = 0, bs = 0;
    uint32_t pph = 0, bph = 0;
    bool ok = true;
    for (int i0 = 0; i0 < nkb && ok; i0 += C::LA) {
#pragma unroll
      for (int u = 0; u < C::LA; ++u) {  // unrolled, so the scale ring stays in registers
        const int i = i0 + u;
        if (i >= nkb) break;
        // warp-uniform outcome, so that no lane leaves while the others wait in the table's shuffles
        const bool got = mbar_wait(&pkfull[ps], pph, abort_flag) && mbar_wait(&bempty[bs], bph ^ 1u, abort_flag);
        if (!__all_sync(0xffffffffu, got)) { ok = false; break; }
        uint4 t = make_uint4(0, 0, 0, 0);
        if constexpr (SDT != H3B_FP8_E4M3) t = table(sg[u]);
        const unsigned char* prow = sP + ps * C::P_BYTES + r_loc * (BK / 2);
        unsigned char* brow = sB + bs * C::B_BYTES + r_loc * BK;
#pragma unroll
        for (int c = 0; c < C::CPT; ++c) {
          const int j = j0 + c;
          if constexpr (SDT == H3B_FP8_E4M3) t = lut[s8[u][c]];
          const uint2 pk = *reinterpret_cast<const uint2*>(prow + 8 * j);
          const uint2 lo = decode8(pk.x, t), hi = decode8(pk.y, t);
          *reinterpret_cast<uint4*>(brow + ((j ^ (r_loc & 7)) << 4)) = make_uint4(lo.x, lo.y, hi.x, hi.y);
        }
        fence_proxy_async_smem();  // the tensor core reads these bytes through the async proxy
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&bfull[bs]);
          mbar_arrive(&pkempty[ps]);
        }
        if (++ps == C::P_STAGES) { ps = 0; pph ^= 1u; }
        if (++bs == C::B_STAGES) { bs = 0; bph ^= 1u; }
        load_scales(i + C::LA, sg[u], s8[u]);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  {  // -------------------------------------------------------------------- staging, split-K reduction and epilogue
    tc_fence_after();
    // receive area [source rank][row - first row of this CTA][column]; every ring is idle now (all MMAs and copies
    // have completed)
    int32_t* red = reinterpret_cast<int32_t*>(sA);
    const uint32_t red_u32 = smem_u32(red);
    const int rows_max = (BM + splits - 1) / splits;
    // subtiles staged and reduced per round: both at once when their receive areas fit the rings (one pair of cluster
    // barriers instead of two)
    const int sub_words = splits * rows_max * C::RED_STRIDE;
    const int spr = MS * sub_words * 4 <= C::RING_BYTES ? MS : 1;
    const int r0 = BM * split / splits, r1 = BM * (split + 1) / splits;  // this CTA's rows of each subtile
    constexpr int VPR = BN / 8;
    const size_t osz = epi.out_dtype == H3B_FP32 || epi.out_dtype == H3B_INT32 ? 4 : 2;
    const bool vec_ok = (epi.ldo % (16 / static_cast<int64_t>(osz))) == 0 && (reinterpret_cast<uintptr_t>(epi.out) & 15) == 0;
    const bool ok = *abort_flag == 0;
    // the epilogue's per-column and per-row constants, staged once in the (now idle) level-table area: channel scales
    // and bias of the BN columns (zero past N), activation scales of this CTA's rows of each subtile; visible to every
    // thread after the first cluster barrier below
    float* e_sch = reinterpret_cast<float*>(lut);  // [BN]
    float* e_bias = e_sch + BN;                    // [BN]
    float* e_xs = e_bias + BN;                     // [MS][rows_max]
    const bool scaled = epi.out_dtype != H3B_INT32, has_bias = scaled && epi.bias != nullptr;
    for (int i = threadIdx.x; i < BN; i += blockDim.x) {
      const int64_t n = static_cast<int64_t>(nt) * BN + i;
      float sv = 0.f, bv = 0.f;
      if (scaled && n < N) {
        sv = __ldg(epi.sch + n);
        if (has_bias)
          bv = epi.out_dtype == H3B_FP32   ? static_cast<const float*>(epi.bias)[n]
               : epi.out_dtype == H3B_BF16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(epi.bias)[n])
                                           : __half2float(static_cast<const __half*>(epi.bias)[n]);
      }
      e_sch[i] = sv;
      e_bias[i] = bv;
    }
    for (int i = threadIdx.x; i < MS * rows_max; i += blockDim.x) {
      const int q = i / rows_max, rl = i - q * rows_max;
      const int row = row_base + q * BM + r0 + rl;
      e_xs[i] = (scaled && rl < r1 - r0 && row < M) ? epi.xs[row] : 0.f;
    }
#pragma unroll 1
    for (int m0 = 0; m0 < MS; m0 += spr) {
      // before any push: every CTA of the cluster is done with its rings (they receive the pushes) and, after the first
      // round, has read the previous round's subtiles out of its receive area
      cluster_sync();
      {
        // push: TMEM lane (quad * 32 + lane) = subtile row r; every warp of the CTA takes part, the warps of one lane
        // quadrant (warp % 4) sharing its 32-column chunks, and stores them straight into the receive area of the CTA
        // that owns row r, in this CTA's slot (posted stores, no round trip)
        const int quad = warp & 3, r = quad * 32 + lane;
        const int wq = warp >> 2, nwq = (C::THREADS / 32 - 1 - quad) / 4 + 1;  // this warp's rank in its quadrant
        int owner = (r * splits) / BM;  // the owner p has BM p / S <= r < BM (p + 1) / S
        while (BM * (owner + 1) / splits <= r) ++owner;
        while (BM * owner / splits > r) --owner;
        const uint32_t local = red_u32 + static_cast<uint32_t>(((split * rows_max + (r - BM * owner / splits)) * C::RED_STRIDE) * 4);
        const bool mine = owner == split;  // this CTA's own rows stay on the local path
        const uint32_t dst0 = mine ? local : mapa_rank(local, static_cast<uint32_t>(owner));
        constexpr int CHUNKS = BN / 32;
#pragma unroll 1
        for (int it = wq; it < spr * CHUNKS; it += nwq) {
          const int q = it / CHUNKS, c = it - q * CHUNKS;
          const uint32_t dst = dst0 + static_cast<uint32_t>(q * sub_words * 4);
          uint32_t v[32];
          tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>((m0 + q) * BN + c * 32), v);
          tmem_ld_wait();
          if (mine) {
#pragma unroll
            for (int j = 0; j < 8; ++j)
              st_shared_v4(dst + static_cast<uint32_t>((c * 32 + 4 * j) * 4), v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
          } else {
#pragma unroll
            for (int j = 0; j < 8; ++j)
              st_cluster_v4(dst + static_cast<uint32_t>((c * 32 + 4 * j) * 4), v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
          }
        }
      }
      cluster_sync();  // every CTA's rows of this round's subtiles have landed in their owners' receive areas
      if (ok) {
        const int per_sub = (r1 - r0) * VPR;
        for (int it = threadIdx.x; it < spr * per_sub; it += blockDim.x) {
          const int q = it / per_sub, rem = it - q * per_sub;
          const int rl = rem / VPR, g = rem - rl * VPR;
          const int row = row_base + (m0 + q) * BM + r0 + rl;
          const int64_t n0 = static_cast<int64_t>(nt) * BN + 8 * g;
          if (row >= M || n0 >= N) continue;
          const int32_t* src = red + q * sub_words + rl * C::RED_STRIDE + 8 * g;
          int32_t a[8] = {0, 0, 0, 0, 0, 0, 0, 0};
          for (int p = 0; p < splits; ++p) {  // rank order, the same sum on every run
            const int4 x = reinterpret_cast<const int4*>(src + p * rows_max * C::RED_STRIDE)[0];
            const int4 y = reinterpret_cast<const int4*>(src + p * rows_max * C::RED_STRIDE)[1];
            a[0] += x.x; a[1] += x.y; a[2] += x.z; a[3] += x.w;
            a[4] += y.x; a[5] += y.y; a[6] += y.z; a[7] += y.w;
          }
          const int nn = N - n0 < 8 ? static_cast<int>(N - n0) : 8;
          char* orow = static_cast<char*>(epi.out) + static_cast<size_t>(row) * static_cast<size_t>(epi.ldo) * osz;
          w4s_store8(a, nn, e_xs[(m0 + q) * rows_max + rl], e_sch + 8 * g, has_bias ? e_bias + 8 * g : nullptr,
                     epi.out_dtype, epi.qmode, orow, n0, vec_ok && nn == 8);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// ------------------------------------------------------------------------------------------------ host side
// The work split: all M rows per CTA (MS subtiles) or one CTA per 128-row M tile, then the N tile width and the number
// of K splits S <= 4 (larger clusters measured slower: fewer of them fit the GPCs at once) with the shortest estimated
// time -- one wave of at most cap[S] CTAs (clusters of S CTAs that can be resident at once; several waves only without
// a split), each doing ceil(num_kb / S) k-blocks.  The terms, in microseconds, were fitted to %globaltimer stamps per CTA
// phase and graph-timed sweeps of forced plans on B200 (M = 256; (K, N) = (5120, 5120), (5120, 13824), (13824, 5120) and
// the official fp8 shapes): a k-block costs 0.45 / 0.6 / 0.8 us for one 128-row subtile and BN = 128 / 192 / 256
// columns, 0.72 / 0.9 / 1.02 us for two (the decode of the weight tile is the bound; two subtiles share it), stretched
// when fewer than 64 CTAs run; start-up takes 2 us, and each wave ends with the staging and the epilogue: 8.5 us +
// 0.026 us per subtile column across a cluster, 3 us + 0.055 us per subtile column without a split (measured; the
// single-CTA epilogue of a whole 128- or 256-row tile is slower per column than a cluster member's share).
struct W4sPlan {
  int bn, ms, splits;  // N tile, 128-row M subtiles per CTA (1: one CTA per M tile), K splits
};

inline W4sPlan w4s_plan(int64_t M, int64_t N, int64_t K, const int (&cap)[9]) {
  const int64_t num_kb = (K + BK - 1) / BK;
  W4sPlan best{128, M <= BM ? 1 : 2, 1};
  double best_t = -1;
  for (int ms : {1, 2}) {
    if (ms == 2 && M <= BM) continue;
    const int64_t m_tiles = ms == 1 ? (M + BM - 1) / BM : 1;
    for (int bn : {256, 192, 128}) {
      const int64_t n_tiles = (N + bn - 1) / bn;
      for (int s = 1; s <= 4 && s <= num_kb; ++s) {
        if (cap[s] < s) continue;
        const int64_t units = m_tiles * n_tiles * s;
        const int64_t waves = (units + cap[s] - 1) / cap[s];
        if (waves > 1 && s > 1) break;
        double per_kb = ms == 2 ? (bn == 128 ? 0.72 : bn == 192 ? 0.9 : 1.02) : (bn == 128 ? 0.45 : bn == 192 ? 0.6 : 0.8);
        if (units < 64) per_kb *= 64.0 / static_cast<double>(units);
        // every wave pays its k-blocks and its epilogue; start-up once
        const double epi = s > 1 ? 8.5 + 0.026 * ms * bn : 3.0 + 0.055 * ms * bn;
        const double t = 2.0 + static_cast<double>(waves) * (((num_kb + s - 1) / s) * per_kb + epi);
        if (best_t < 0 || t < best_t) {
          best_t = t;
          best = W4sPlan{bn, ms, s};
        }
      }
    }
  }
  return best;
}

template <int BN, int MS, int SDT>
static int w4s_set_attrs() {
  using C = W4sCfg<BN, MS>;
  static std::atomic<unsigned long long> attr_done{0};  // one bit per device
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned long long bit = 1ull << (dev & 63);
  if (!(attr_done.load() & bit)) {
    const cudaError_t e = cudaFuncSetAttribute(gemm_w4s_kernel<BN, MS, SDT>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(gemm w4s)");
    attr_done.fetch_or(bit);
  }
  return 0;
}

// CTAs that can be resident at once for each cluster size 1..8 (every configuration takes one CTA per SM), queried
// once per device on the 256-column one-subtile kernel.
template <int SDT>
static int w4s_capacity(int (&cap)[9]) {
  static std::mutex mu;
  static int cached[64][9];
  static unsigned long long done = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  if (!(done & (1ull << (dev & 63)))) {
    if (int rc = w4s_set_attrs<256, 1, SDT>()) return rc;
    int* c = cached[dev & 63];
    c[0] = 0;
    c[1] = num_sms();
    for (int s = 2; s <= 8; ++s) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(static_cast<unsigned>(s), 1, 1);
      cfg.blockDim = dim3(W4sCfg<256, 1>::THREADS, 1, 1);
      cfg.dynamicSmemBytes = W4sCfg<256, 1>::SMEM;
      cudaLaunchAttribute attr;
      attr.id = cudaLaunchAttributeClusterDimension;
      attr.val.clusterDim.x = static_cast<unsigned>(s);
      attr.val.clusterDim.y = 1;
      attr.val.clusterDim.z = 1;
      cfg.attrs = &attr;
      cfg.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, gemm_w4s_kernel<256, 1, SDT>, &cfg) != cudaSuccess) {
        cudaGetLastError();
        n = 0;
      }
      c[s] = n * s;
    }
    done |= 1ull << (dev & 63);
  }
  for (int s = 0; s < 9; ++s) cap[s] = cached[dev & 63][s];
  return 0;
}

template <int BN, int MS, int SDT>
static int w4s_launch_cfg(int splits, const CUtensorMap& ta, const CUtensorMap& tp, const void* s_rel, int64_t lds,
                          const float* codebook, const W4sEpi& epi, int M, int N, int K, cudaStream_t st) {
  using C = W4sCfg<BN, MS>;
  if (int rc = w4s_set_attrs<BN, MS, SDT>()) return rc;
  const int m_tiles = MS == 1 ? (M + BM - 1) / BM : 1;
  const int units = ((N + BN - 1) / BN) * m_tiles * splits;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(units), 1, 1);
  cfg.blockDim = dim3(C::THREADS, 1, 1);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeClusterDimension;  // the splits of one output tile are one cluster
  attr.val.clusterDim.x = static_cast<unsigned>(splits);
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_w4s_kernel<BN, MS, SDT>, ta, tp, s_rel, lds, codebook, epi, M, N, K,
                                           splits, m_tiles);
  if (e != cudaSuccess) return cuda_fail(e, "cudaLaunchKernelEx(gemm_w4s_kernel)");
  return check_launch("gemm_w4s_kernel");
}

// The small-M GEMM of one scale dtype: plan (or `force`, when not null), then one clustered launch.
template <int SDT>
int w4s_launch_sdt(const W4sPlan* force, const int8_t* a, int64_t lda, const void* q4, int64_t ldq4, const void* s_rel,
                   int64_t lds, const float* codebook, const W4sEpi& epi, int M, int N, int K, cudaStream_t st) {
  int cap[9];
  if (int rc = w4s_capacity<SDT>(cap)) return rc;
  const W4sPlan plan = force ? *force : w4s_plan(M, N, K, cap);
  if (plan.splits < 1 || plan.splits > 8) return fail(H3B_ERR_ARG, "small-M GEMM: 1 to 8 K splits");
  CUtensorMap ta, tp;
  int rc = make_map(&ta, a, K, M, lda, BM);
  if (rc) return rc;
  rc = make_map_packed(&tp, q4, K / 2, N, ldq4, plan.bn);
  if (rc) return rc;
#define H3B_W4S(B, S) if (plan.bn == B && plan.ms == S) return w4s_launch_cfg<B, S, SDT>(plan.splits, ta, tp, s_rel, lds, codebook, epi, M, N, K, st);
  H3B_W4S(256, 2) H3B_W4S(192, 2) H3B_W4S(128, 2) H3B_W4S(256, 1) H3B_W4S(192, 1) H3B_W4S(128, 1)
#undef H3B_W4S
  return fail(H3B_ERR_ARG, "small-M GEMM: unsupported tile plan");
}

}  // namespace h3b
