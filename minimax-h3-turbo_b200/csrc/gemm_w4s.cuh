// Kernel KB, small-M form: the W4A8 GEMM for M <= 256 tokens, int4 weight decoded in the producer warps, K split
// across CTAs so that every SM works although N / 128 weight tiles alone would leave many idle.
//
// At small M the weight dominates the bytes and every output tile needs the whole K.  Here a work unit is (128 weight
// rows, K range): CTA u owns output columns [128 nt, 128 nt + 128) for ALL M tokens (up to two 128-token subtiles, so
// each weight tile is decoded once) and the k-blocks [kb0, kb1) of split s.  Integer partial sums are exact, so
// splitting K changes no bit of the result.
//
// The tensor core computes the transposed product D[n, m] = sum_k W[n, k] X[m, k]: the decoded weight tile is the
// MMA's A operand (M = 128 weight rows) and lives in tensor memory, the activation codes are its B operand (N = 128 or
// 256 tokens) in shared memory.  With the weight as B in shared memory instead, each k-block took two 128 x 128 MMAs
// whose shared-memory operand reads paced the loop (measured on B200 at 2.9 int8 POP/s over all SMs, against 4.3 for
// one 128 x 256 MMA with A in TMEM); here the tensor core reads half the shared-memory bytes per multiply-add, and the
// decoded bytes never pass through shared memory.
//
//   warp 0      TMA producer of the packed int4 weight tiles (128 x 64 bytes per k-block, 64-byte swizzle) -> P ring
//   warp 6      TMA producer of the activation-code tiles (MS x 128 x 128 bytes per k-block) -> A ring
//   warps 7-18  decoders, three groups of four warps: group g decodes the k-blocks i = g (mod 3), each warp the 32
//               weight rows of its TMEM lane quadrant (warp % 4), one row per thread (level tables + byte permutes,
//               exactly decode.cuh's levels), and stores them with tcgen05.st into the group's TMEM stage
//   warp 1      MMA issuer: per k-block 4 x tcgen05.mma.kind::i8 (K = 32 each, A from TMEM) into the accumulator
//   warps 2-5   epilogue: stage the channel scales, bias and token scales in shared memory while the main loop runs,
//               wait for the accumulator, then (with every warp of the CTA, after the roles) apply the W4A8 epilogue
//               (as gemm_sm100.cuh).  Without a split straight from TMEM to the output.  With S K splits the S CTAs of
//               one output tile form a thread-block cluster: CTA p owns 1/S of the tile's token rows, every CTA stores
//               its raw int32 partial sums straight from TMEM into the owner's (by then idle) ring memory (distributed
//               shared memory stores, posted; 128 contiguous bytes of one token row per warp store; its own rows
//               locally), and after a cluster barrier each owner adds up its rows over the S slots in rank order from
//               its own shared memory -- no partial sums in HBM, no second kernel.
// One work unit per CTA; every mbarrier wait bounded (h3b_common.cuh), and every CTA reaches every cluster barrier
// whatever happened before, so no CTA waits for a peer that left; after the last one no CTA touches another's shared
// memory.
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

constexpr int W4S_BN = 128;  // weight rows (output columns) per CTA: the MMA's M

template <int MS>
struct W4sCfg {
  static constexpr int BN = W4S_BN;
  static constexpr int DEPTH = 3;                  // k-blocks decoded ahead: TMEM stages = decoder warp groups
                                                   // (3 measured 1-4 % faster than 4 and than 2)
  static constexpr int DWARPS = 4 * DEPTH;         // one warp per (group, TMEM lane quadrant)
  static constexpr int LA = 1;                     // look-ahead of a decoder's scale loads, in its own k-blocks
                                                   // (1 measured 0-3 % faster than 2 and 3)
  static constexpr int A_BYTES = BM * BK;          // one 128-token activation subtile of one k-block
  static constexpr int P_BYTES = BN * (BK / 2);    // one packed weight tile
  static constexpr int BUDGET = 210 * 1024;
  // The activation tiles come from L2 with a latency of a few microseconds when every SM streams at once, so they get
  // 128 KB of ring; the packed weight tiles the rest.
  static constexpr int A_STAGES = MS == 1 ? 8 : 4;
  static constexpr int P_LEFT = (BUDGET - A_STAGES * MS * A_BYTES) / P_BYTES;
  static constexpr int P_STAGES = P_LEFT > 12 ? 12 : P_LEFT;
  static constexpr int ACC_COLS = MS * BM;         // the accumulator: TMEM lane = weight row, column = token
  static constexpr int A_COL0 = ACC_COLS;          // then DEPTH decoded stages of 32 columns (128 int8 per row)
  static constexpr int TMEM_COLS = ACC_COLS + DEPTH * 32 <= 256 ? 256 : 512;
  static constexpr int THREADS = 32 * (7 + DWARPS);
  static constexpr int RING_BYTES = A_STAGES * MS * A_BYTES + P_STAGES * P_BYTES;
  static constexpr int SMEM = 1024 + RING_BYTES + 4096 + 512 + 2048;  // rings, fp8 level tables, barriers, epilogue constants
  static constexpr uint32_t IDESC = idesc_i8(BN, MS * BM);
  // the split-K receive area of one 128-token subtile, in the rings: [S][ceil(128 / S)][BN + 4] int32 (rows 16 bytes
  // apart in bank terms); S ceil(128 / S) <= 128 + 7 rows for S <= 8
  static constexpr int RED_STRIDE = BN + 4;
  static constexpr int RED_WORDS = (BM + 7) * RED_STRIDE;
  static_assert(P_STAGES >= DEPTH + 2, "bad small-M GEMM configuration");
  static_assert(2 * RED_WORDS * 4 <= RING_BYTES, "the split-K receive areas of both subtiles live in the ring memory");
  static_assert(SMEM <= 227 * 1024, "shared memory");
  static_assert((2 * BN + MS * BM) * 4 <= 2048, "the epilogue constants");
  static_assert(ACC_COLS + DEPTH * 32 <= TMEM_COLS, "tensor memory");
};

// 4 bytes into this CTA's / a cluster CTA's shared memory (`addr`: a shared::cta / shared::cluster address; the
// remote store is posted)
__device__ __forceinline__ void st_shared_u32(uint32_t addr, uint32_t v) {
  asm volatile("st.shared.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ void st_cluster_u32(uint32_t addr, uint32_t v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}
// 32 lanes x 8 consecutive 32-bit columns of tensor memory into registers: thread i of the warp gets its lane's.
__device__ __forceinline__ void tmem_ld_32x32b_x8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr)
               : "memory");
}
// 32 lanes x 8 consecutive 32-bit columns of tensor memory from registers: thread i of the warp writes its lane.
__device__ __forceinline__ void tmem_st_32x32b_x8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr), "r"(r[0]),
               "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// D[tmem] (+)= A[tmem] * B[smem desc]^T, int8 x int8 -> int32, one CTA: row r of A in TMEM lane r, its K bytes packed
// four to a 32-bit column (lowest k in the lowest byte).
__device__ __forceinline__ void mma_i8_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
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

// The same epilogue for one accumulator: column n of `orow`, channel scale `s`, bias `b` (used when `bias`).
__device__ __forceinline__ void w4s_store1(int32_t a, float xsr, float s, float b, bool bias, int out_dtype, int qmode,
                                           char* orow, int64_t n) {
  if (out_dtype == H3B_INT32) {
    reinterpret_cast<int32_t*>(orow)[n] = a;
    return;
  }
  const float f = __int2float_rn(a);
  float v = qmode == H3B_QMODE_CK ? __fmul_rn(__fmul_rn(f, xsr), s) : __fmul_rn(f, __fmul_rn(xsr, s));
  if (out_dtype == H3B_FP32) {
    if (bias) v = __fadd_rn(v, b);
    reinterpret_cast<float*>(orow)[n] = v;
    return;
  }
  if (out_dtype == H3B_BF16) {
    float r = __bfloat162float(__float2bfloat16_rn(v));
    if (bias) r = __fadd_rn(r, b);
    reinterpret_cast<__nv_bfloat16*>(orow)[n] = __float2bfloat16_rn(r);
  } else {
    float r = __half2float(__float2half_rn(v));
    if (bias) r = __fadd_rn(r, b);
    reinterpret_cast<__half*>(orow)[n] = __float2half_rn(r);
  }
}

template <int MS, int SDT>
__global__ void __launch_bounds__(W4sCfg<MS>::THREADS, 1)
    gemm_w4s_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmP,
                    const void* __restrict__ s_rel, int64_t lds, const float* __restrict__ codebook, const W4sEpi epi,
                    int M, int N, int K, int splits, int m_tiles) {
  using C = W4sCfg<MS>;
  constexpr int BN = C::BN;
  constexpr int GROUP = SDT == H3B_FP8_E4M3 ? 16 : 128;
  extern __shared__ __align__(1024) unsigned char w4s_smem[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(w4s_smem) + 1023) & ~uintptr_t(1023));
  unsigned char* sA = smem;                                    // [A_STAGES][MS][A_BYTES]
  unsigned char* sP = sA + C::A_STAGES * MS * C::A_BYTES;      // [P_STAGES][P_BYTES]
  uint4* lut = reinterpret_cast<uint4*>(sP + C::P_STAGES * C::P_BYTES);  // fp8: the 256 level tables
  uint64_t* pkfull = reinterpret_cast<uint64_t*>(lut + 256);
  uint64_t* pkempty = pkfull + C::P_STAGES;
  uint64_t* afull = pkempty + C::P_STAGES;
  uint64_t* aempty = afull + C::A_STAGES;
  uint64_t* dfull = aempty + C::A_STAGES;   // a decoded weight stage in TMEM is complete
  uint64_t* dempty = dfull + C::DEPTH;      // the MMAs of a decoded stage are done with it
  uint64_t* tfull = dempty + C::DEPTH;
  uint64_t* mdone = tfull + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mdone + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* econst = reinterpret_cast<float*>(reinterpret_cast<unsigned char*>(lut) + 4096 + 512);  // epilogue constants

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
      mbar_init(&pkempty[s], 4);  // the four quadrant warps of the group that decodes it
    }
    for (int s = 0; s < C::A_STAGES; ++s) {
      mbar_init(&afull[s], 1);
      mbar_init(&aempty[s], 1);
    }
    for (int s = 0; s < C::DEPTH; ++s) {
      mbar_init(&dfull[s], 4);
      mbar_init(&dempty[s], 1);
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
      int as = 0;
      uint32_t aph = 0;
      bool ok = true;
      for (int i = 0; i < nkb && ok; ++i) {
        const int ds = i % C::DEPTH;
        const uint32_t dph = static_cast<uint32_t>((i / C::DEPTH) & 1);
        if (!mbar_wait(&afull[as], aph, abort_flag) || !mbar_wait(&dfull[ds], dph, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t b0 = smem_u32(sA + as * MS * C::A_BYTES);  // the MS subtiles: one K-major tile of MS x 128 rows
        const uint32_t a0 = tmem_base + static_cast<uint32_t>(C::A_COL0 + 32 * ds);
#pragma unroll
        for (int k = 0; k < BK / 32; ++k)
          mma_i8_ts(tmem_base, a0 + static_cast<uint32_t>(8 * k), smem_desc_sw128(b0 + 32 * k), C::IDESC, (i | k) != 0);
        mma_commit(&aempty[as]);  // the activation slot and the decoded stage are free once these MMAs complete
        mma_commit(&dempty[ds]);
        if (++as == C::A_STAGES) { as = 0; aph ^= 1u; }
      }
      if (ok) mma_commit(tfull);
      mma_commit(mdone);
      mbar_wait_drain(mdone, 0);
    }
  } else if (warp < 6) {  // ------------------------------------------------------------------- epilogue
    // while the main loop runs: stage the epilogue's constants -- channel scales and bias (as fp32, exact for every bias
    // dtype) of the BN columns, zero past N; activation scales of this CTA's token rows of each subtile
    {
      const int rows_max = (BM + splits - 1) / splits;
      const int r0 = BM * split / splits, r1 = BM * (split + 1) / splits;
      float* e_sch = econst;
      float* e_bias = e_sch + BN;
      float* e_xs = e_bias + BN;
      const bool scaled = epi.out_dtype != H3B_INT32, has_bias = scaled && epi.bias != nullptr;
      for (int i = threadIdx.x - 64; i < BN; i += 128) {
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
      for (int i = threadIdx.x - 64; i < MS * rows_max; i += 128) {
        const int q = i / rows_max, rl = i - q * rows_max;
        const int row = row_base + q * BM + r0 + rl;
        e_xs[i] = (scaled && rl < r1 - r0 && row < M) ? epi.xs[row] : 0.f;
      }
    }
    // the accumulator is complete once the last MMA has committed; the epilogue proper runs after the roles, with every
    // warp of the CTA (below)
    mbar_wait(tfull, 0, abort_flag);
  } else {  // -------------------------------------------------------------------------------------- decoders
    const int grp = (warp - 7) >> 2;      // this warp decodes the k-blocks i = grp (mod DEPTH) into TMEM stage grp
    const int quad = warp & 3;            // its TMEM lane quadrant
    const int r_loc = quad * 32 + lane;   // this thread's weight row of the tile = its TMEM lane
    const int n = nt * BN + r_loc;
    const bool row_ok = n < N;
    const unsigned char* srow = static_cast<const unsigned char*>(s_rel) +
                                static_cast<int64_t>(row_ok ? n : 0) * lds * (SDT == H3B_FP8_E4M3 ? 1 : (SDT == H3B_FP32 ? 4 : 2));
    float cb[16];
    if constexpr (SDT != H3B_FP8_E4M3) {
#pragma unroll
      for (int e = 0; e < 16; ++e) cb[e] = __ldg(codebook + e);
    }
    // the group scales of k-block i: the one scale of this row (group-128 formats, as a float) or its 8 scale bytes
    // (fp8 group 16); plain global loads, issued LA of this warp's k-blocks before their use
    auto load_scales = [&](int i, float& g, uint2& f8) {
      const int64_t kbase = static_cast<int64_t>(kb0 + i) * BK;
      if constexpr (SDT == H3B_FP8_E4M3) {
        uint32_t b[8];
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const int64_t e0 = kbase + 16 * c;
          b[c] = (row_ok && i < nkb && e0 < K) ? static_cast<uint32_t>(srow[e0 / GROUP]) : 0u;
        }
        f8 = make_uint2(b[0] | (b[1] << 8) | (b[2] << 16) | (b[3] << 24), b[4] | (b[5] << 8) | (b[6] << 16) | (b[7] << 24));
      } else {
        g = (row_ok && i < nkb && kbase < K) ? scale_at<SDT>(srow, kbase / GROUP) : 0.f;
      }
    };
    float sg[C::LA];
    uint2 s8[C::LA];
#pragma unroll
    for (int u = 0; u < C::LA; ++u) {
      sg[u] = 0.f;
      s8[u] = make_uint2(0u, 0u);
      load_scales(grp + u * C::DEPTH, sg[u], s8[u]);
    }
    const uint32_t tstage = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(C::A_COL0 + 32 * grp);
    const int sw = (r_loc >> 1) & 3;  // 64-byte swizzle: 16-byte chunk c of packed row r sits at chunk c ^ ((r >> 1) & 3)
    bool ok = true;
    for (int i0 = grp; i0 < nkb && ok; i0 += C::LA * C::DEPTH) {
#pragma unroll
      for (int u = 0; u < C::LA; ++u) {  // unrolled, so the scale ring stays in registers
        const int i = i0 + u * C::DEPTH;
        if (i >= nkb) break;
        const int ps = i % C::P_STAGES;
        const uint32_t pph = static_cast<uint32_t>((i / C::P_STAGES) & 1);
        const uint32_t dph = static_cast<uint32_t>(((i / C::DEPTH) & 1) ^ 1);
        // warp-uniform outcome: tcgen05.st below is a whole-warp instruction
        const bool got = mbar_wait(&pkfull[ps], pph, abort_flag) && mbar_wait(&dempty[grp], dph, abort_flag);
        if (!__all_sync(0xffffffffu, got)) { ok = false; break; }
        tc_fence_after();
        uint4 t = make_uint4(0, 0, 0, 0);
        if constexpr (SDT != H3B_FP8_E4M3) t = level_table(cb, sg[u]);
        const unsigned char* prow = sP + ps * C::P_BYTES + r_loc * (BK / 2);
#pragma unroll
        for (int c = 0; c < 4; ++c) {  // 16 packed bytes = 32 weights = 8 TMEM columns
          const uint4 pk = *reinterpret_cast<const uint4*>(prow + ((c ^ sw) << 4));
          uint4 t0 = t, t1 = t;
          if constexpr (SDT == H3B_FP8_E4M3) {
            const uint32_t sb = c < 2 ? s8[u].x : s8[u].y;
            t0 = lut[(sb >> (16 * (c & 1))) & 0xFFu];
            t1 = lut[(sb >> (16 * (c & 1) + 8)) & 0xFFu];
          }
          const uint2 d0 = decode8(pk.x, t0), d1 = decode8(pk.y, t0), d2 = decode8(pk.z, t1), d3 = decode8(pk.w, t1);
          const uint32_t w[8] = {d0.x, d0.y, d1.x, d1.y, d2.x, d2.y, d3.x, d3.y};
          tmem_st_32x32b_x8(tstage + static_cast<uint32_t>(8 * c), w);
        }
        tmem_st_wait();
        tc_fence_before();  // the MMA issuer reads these columns after the arrival below
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&dfull[grp]);
          mbar_arrive(&pkempty[ps]);
        }
        load_scales(i + C::LA * C::DEPTH, sg[u], s8[u]);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  {  // -------------------------------------------------------------------- staging, split-K reduction and epilogue
    tc_fence_after();
    // receive area [subtile][source rank][token row - first row of this CTA][column]; every ring is idle now (all MMAs
    // and copies have completed)
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
    // the epilogue's constants, staged by the epilogue warps during the main loop
    const float* e_sch = econst;
    const float* e_bias = e_sch + BN;
    const float* e_xs = e_bias + BN;
    const bool has_bias = epi.out_dtype != H3B_INT32 && epi.bias != nullptr;
    const int quad = warp & 3, n_loc = quad * 32 + lane;  // this thread's TMEM lane = output column of the tile
    const int wq = warp >> 2, nwq = (C::THREADS / 32 - 1 - quad) / 4 + 1;  // this warp's rank in its lane quadrant
    constexpr int CHUNKS = BM / 32;
    if (splits == 1) {
      // one split: the accumulator is the result; every warp applies the epilogue straight from TMEM, the warps of one
      // lane quadrant sharing its 32-token chunks, one token row of 32 output columns per warp store
      const int64_t n = static_cast<int64_t>(nt) * BN + n_loc;
      const float sv = e_sch[n_loc], bv = e_bias[n_loc];
      // (8 tokens per TMEM load and a rolled loop over them: the unrolled body stays small enough for the instruction
      // cache, which a fully unrolled 32-token body did not)
#pragma unroll 1
      for (int it = wq; it < MS * CHUNKS * 4; it += nwq) {
        const int q = it / (CHUNKS * 4), t0 = (it - q * CHUNKS * 4) * 8;  // subtile, first token of the 8
        uint32_t v[8];  // v[j] = D[n_loc][token t0 + j of subtile q]
        tmem_ld_32x32b_x8(tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(q * BM + t0), v);
        tmem_ld_wait();
        if (ok && n < N) {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int row = row_base + q * BM + t0 + j;
            if (row < M)
              w4s_store1(static_cast<int32_t>(v[j]), e_xs[q * rows_max + t0 + j], sv, bv, has_bias, epi.out_dtype,
                         epi.qmode, static_cast<char*>(epi.out) + static_cast<size_t>(row) * static_cast<size_t>(epi.ldo) * osz, n);
          }
        }
        __syncwarp();
      }
    } else {
#pragma unroll 1
    for (int m0 = 0; m0 < MS; m0 += spr) {
      // before any push: every CTA of the cluster is done with its rings (they receive the pushes) and, after the first
      // round, has read the previous round's subtiles out of its receive area
      cluster_sync();
      {
        // push: TMEM lane (quad * 32 + lane) = output column n_loc of the tile, TMEM column = token; every warp of the
        // CTA takes part, the warps of one lane quadrant (warp % 4) sharing its 32-token chunks.  Each token row goes
        // to the CTA that owns it, into this CTA's slot: for one token the 32 lanes of a warp store 128 contiguous
        // bytes (posted stores, no round trip); own rows stay local
#pragma unroll 1
        for (int it = wq; it < spr * CHUNKS; it += nwq) {
          const int q = it / CHUNKS, c = it - q * CHUNKS;
          uint32_t v[32];  // v[j] = D[n_loc][token 32 c + j of subtile m0 + q]
          tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>((m0 + q) * BM + c * 32), v);
          tmem_ld_wait();
          const uint32_t qoff = red_u32 + static_cast<uint32_t>((q * sub_words + n_loc) * 4);
          // the chunk's 32 token rows belong to at most three owners (S <= 8: at least 16 rows each): o0, o0 + 1 from
          // row j1 on, o0 + 2 from row j2 on; base[k] + j RS 4 is row j's address in owner o0 + k's slot of this CTA
          const int c0 = c * 32;
          int o0 = (c0 * splits) / BM;  // the owner p has BM p / S <= r < BM (p + 1) / S
          while (BM * (o0 + 1) / splits <= c0) ++o0;
          while (BM * o0 / splits > c0) --o0;
          const int j1 = BM * (o0 + 1) / splits - c0, j2 = BM * (o0 + 2) / splits - c0;
          uint32_t base[3];
#pragma unroll
          for (int k = 0; k < 3; ++k) {
            const int o = o0 + k;
            base[k] = 0;
            if (o < splits) {
              const int rf = max(c0, BM * o / splits);  // the owner's first row in this chunk
              const uint32_t first = qoff + static_cast<uint32_t>(((split * rows_max + rf - BM * o / splits) * C::RED_STRIDE) * 4);
              base[k] = (o == split ? first : mapa_rank(first, static_cast<uint32_t>(o))) -
                        static_cast<uint32_t>((rf - c0) * C::RED_STRIDE * 4);
            }
          }
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int k = (j >= j1) + (j >= j2);  // warp-uniform
            const uint32_t addr = (k == 0 ? base[0] : (k == 1 ? base[1] : base[2])) + static_cast<uint32_t>(j * C::RED_STRIDE * 4);
            if (o0 + k == split)
              st_shared_u32(addr, v[j]);
            else
              st_cluster_u32(addr, v[j]);
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
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// ------------------------------------------------------------------------------------------------ host side
// The work split: all M rows per CTA (MS subtiles) or one CTA per 128-row M tile, then the number of K splits S <= 4
// (larger clusters measured slower: fewer of them fit the GPCs at once) with the shortest estimated time -- waves of at
// most cap[S] CTAs (clusters of S CTAs that can be resident at once; several waves only without a split), each doing
// ceil(num_kb / S) k-blocks.  The terms, in microseconds, were fitted to graph-timed sweeps of forced plans on B200
// (M = 128 and 256; (K, N) = (5120, 5120), (5120, 13824), (13824, 5120) with fp16 group scales and the official fp8
// shapes): a k-block costs 0.45 us with group-128 scales and about 0.62 us with fp8 group-16 scales (a level table per 16
// weights), for one or two 128-token subtiles alike (the decode paces it, not the tensor core), whatever the number of
// CTAs; start-up takes 2 us; each wave ends with the epilogue, 3.7 + 2.0 MS us without a split (straight from TMEM)
// and 4.2 + 4.0 MS us with one (cluster barriers, the push of the partial sums, the reduction).
struct W4sPlan {
  int bn, ms, splits;  // N tile (always W4S_BN), 128-row M subtiles per CTA (1: one CTA per M tile), K splits
};

inline W4sPlan w4s_plan(int64_t M, int64_t N, int64_t K, bool fp8_scales, const int (&cap)[9]) {
  const double per_kb = fp8_scales ? 0.62 : 0.45;
  const int64_t num_kb = (K + BK - 1) / BK;
  const int64_t n_tiles = (N + W4S_BN - 1) / W4S_BN;
  W4sPlan best{W4S_BN, M <= BM ? 1 : 2, 1};
  double best_t = -1;
  for (int ms : {1, 2}) {
    if (ms == 2 && M <= BM) continue;
    const int64_t m_tiles = ms == 1 ? (M + BM - 1) / BM : 1;
    for (int s = 1; s <= 4 && s <= num_kb; ++s) {
      if (cap[s] < s) continue;
      const int64_t units = m_tiles * n_tiles * s;
      const int64_t waves = (units + cap[s] - 1) / cap[s];
      if (waves > 1 && s > 1) break;
      const double epi = s > 1 ? 4.2 + 4.0 * ms : 3.7 + 2.0 * ms;
      const double t = 2.0 + static_cast<double>(waves) * (((num_kb + s - 1) / s) * per_kb + epi);
      if (best_t < 0 || t < best_t) {
        best_t = t;
        best = W4sPlan{W4S_BN, ms, s};
      }
    }
  }
  return best;
}

// 2-D uint8 tensor map over the packed weight for this kernel: box 64 bytes x 128 rows, 64-byte swizzle (so that the
// decoders' 16-byte row reads of one column of chunks spread over all banks), zero fill.
static int make_map_packed_sw64(CUtensorMap* map, const void* base, int64_t inner, int64_t rows, int64_t ld) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(H3B_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable (driver too old?)");
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld)};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(BK / 2), static_cast<cuuint32_t>(W4S_BN)};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(H3B_ERR_CUDA, "cuTensorMapEncodeTiled (packed, swizzled) failed (code " + std::to_string(int(r)) + ")");
  return H3B_OK;
}

template <int MS, int SDT>
static int w4s_set_attrs() {
  using C = W4sCfg<MS>;
  static std::atomic<unsigned long long> attr_done{0};  // one bit per device
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned long long bit = 1ull << (dev & 63);
  if (!(attr_done.load() & bit)) {
    const cudaError_t e = cudaFuncSetAttribute(gemm_w4s_kernel<MS, SDT>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(gemm w4s)");
    attr_done.fetch_or(bit);
  }
  return 0;
}

// CTAs that can be resident at once for each cluster size 1..8 (every configuration takes one CTA per SM), queried
// once per device on the one-subtile kernel.
template <int SDT>
static int w4s_capacity(int (&cap)[9]) {
  static std::mutex mu;
  static int cached[64][9];
  static unsigned long long done = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  if (!(done & (1ull << (dev & 63)))) {
    if (int rc = w4s_set_attrs<1, SDT>()) return rc;
    int* c = cached[dev & 63];
    c[0] = 0;
    c[1] = num_sms();
    for (int s = 2; s <= 8; ++s) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(static_cast<unsigned>(s), 1, 1);
      cfg.blockDim = dim3(W4sCfg<1>::THREADS, 1, 1);
      cfg.dynamicSmemBytes = W4sCfg<1>::SMEM;
      cudaLaunchAttribute attr;
      attr.id = cudaLaunchAttributeClusterDimension;
      attr.val.clusterDim.x = static_cast<unsigned>(s);
      attr.val.clusterDim.y = 1;
      attr.val.clusterDim.z = 1;
      cfg.attrs = &attr;
      cfg.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, gemm_w4s_kernel<1, SDT>, &cfg) != cudaSuccess) {
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

template <int MS, int SDT>
static int w4s_launch_cfg(int splits, const CUtensorMap& ta, const CUtensorMap& tp, const void* s_rel, int64_t lds,
                          const float* codebook, const W4sEpi& epi, int M, int N, int K, cudaStream_t st) {
  using C = W4sCfg<MS>;
  if (int rc = w4s_set_attrs<MS, SDT>()) return rc;
  const int m_tiles = MS == 1 ? (M + BM - 1) / BM : 1;
  const int units = ((N + C::BN - 1) / C::BN) * m_tiles * splits;
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
  const cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_w4s_kernel<MS, SDT>, ta, tp, s_rel, lds, codebook, epi, M, N, K,
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
  const W4sPlan plan = force ? *force : w4s_plan(M, N, K, SDT == H3B_FP8_E4M3, cap);
  if (plan.splits < 1 || plan.splits > 8) return fail(H3B_ERR_ARG, "small-M GEMM: 1 to 8 K splits");
  if (plan.bn != W4S_BN) return fail(H3B_ERR_ARG, "small-M GEMM: the N tile is 128");
  CUtensorMap ta, tp;
  int rc = make_map(&ta, a, K, M, lda, BM);
  if (rc) return rc;
  rc = make_map_packed_sw64(&tp, q4, K / 2, N, ldq4);
  if (rc) return rc;
  if (plan.ms == 2) return w4s_launch_cfg<2, SDT>(plan.splits, ta, tp, s_rel, lds, codebook, epi, M, N, K, st);
  if (plan.ms == 1) return w4s_launch_cfg<1, SDT>(plan.splits, ta, tp, s_rel, lds, codebook, epi, M, N, K, st);
  return fail(H3B_ERR_ARG, "small-M GEMM: unsupported tile plan");
}

}  // namespace h3b
