// Kernel KB: int8 x int8 -> int32 GEMM on the sm_100a tensor cores (tcgen05.mma kind::i8, TMEM accumulators) with the
// W4A8 epilogue fused.
//
//   acc[m, n] = sum_k a[m, k] * b[n, k]           a = activation codes [M, K], b = int8 weight grid [N, K], both K-major
//   out[m, n] = dt((fp32(acc) * xs[m]) * s_ch[n])      ("ck",    h3turbo/h3/qlinear.py:400-401)
//             = dt(fp32(acc) * (xs[m] * s_ch[n]))      ("eager", qlinear.py:402-403)
//   out      <- dt(fp32(out) + fp32(bias[n]))          (bias after the output rounding, qlinear.py:404-405)
//
// Persistent, warp-specialised CTA of 192 threads, one per SM:
//   warp 0      TMA producer: 128 x 128-byte A tile + BN x 128-byte B tile per stage, 128-byte swizzle, STAGES-deep ring
//   warp 1      MMA issuer: 4 x tcgen05.mma (K = 32 each) per stage into a TMEM accumulator; tcgen05.commit frees the
//               stage and, after the last k-block, hands the accumulator to the epilogue
//   warps 2-5   epilogue: tcgen05.ld 32 columns at a time, scales, rounding, bias, 16-byte stores
// Two TMEM accumulators (2 x BN columns) let the epilogue of tile i overlap the mainloop of tile i + 1.
// Every mbarrier wait is bounded (h3b_common.cuh): a lost arrival makes the kernel raise the device flag and exit.
#pragma once

#include <atomic>
#include <cstdlib>
#include <mutex>

#include "h3b_common.cuh"

namespace h3b {

constexpr int BM = 128;
constexpr int BK = 128;  // int8 elements (= bytes) of K per stage: one 128-byte swizzle row

template <int BN>
struct GemmCfg {
  static constexpr int STAGES = BN >= 256 ? 4 : (BN >= 192 ? 5 : (BN >= 128 ? 6 : (BN >= 96 ? 7 : 8)));
  static constexpr int A_BYTES = BM * BK;
  static constexpr int B_BYTES = BN * BK;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  // TMEM is allocated in power-of-two column counts (>= 32) holding two BN-column accumulators
  static constexpr int TMEM_COLS = 2 * BN <= 32 ? 32 : (2 * BN <= 64 ? 64 : (2 * BN <= 128 ? 128 : (2 * BN <= 256 ? 256 : 512)));
  static constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + 256;  // alignment slack + ring + barriers
  static constexpr uint32_t IDESC = idesc_i8(BM, BN);
};

enum { OUT_BF16 = 0, OUT_FP16 = 1, OUT_FP32 = 2, OUT_S32 = 4 };

template <int OUT>
__device__ __forceinline__ float round_out(float v) {
  if constexpr (OUT == OUT_BF16) return __bfloat162float(__float2bfloat16_rn(v));
  else if constexpr (OUT == OUT_FP16) return __half2float(__float2half_rn(v));
  else return v;
}
template <int OUT>
__device__ __forceinline__ float bias_at(const void* bias, int n) {
  if constexpr (OUT == OUT_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(bias)[n]);
  else if constexpr (OUT == OUT_FP16) return __half2float(static_cast<const __half*>(bias)[n]);
  else return static_cast<const float*>(bias)[n];
}

// One row's 32 accumulator columns -> output.  ncols <= 32 valid columns starting at global column n0.
template <int OUT, bool BIAS, int QMODE>
__device__ __forceinline__ void epilogue_row32(const uint32_t (&r)[32], float xsr, const float* __restrict__ sch,
                                               const void* __restrict__ bias, char* orow, int n0, int ncols,
                                               bool vec_ok) {
  if constexpr (OUT == OUT_S32) {
    int32_t* o = reinterpret_cast<int32_t*>(orow) + n0;
    if (vec_ok && ncols == 32) {
#pragma unroll
      for (int j = 0; j < 32; j += 4)
        *reinterpret_cast<int4*>(o + j) = make_int4(int(r[j]), int(r[j + 1]), int(r[j + 2]), int(r[j + 3]));
    } else {
      for (int j = 0; j < ncols; ++j) o[j] = int(r[j]);
    }
    return;
  } else {
    float v[32];
    if (ncols == 32) {
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        const float4 s4 = __ldg(reinterpret_cast<const float4*>(sch + n0 + j));
        const float sv[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float a = __int2float_rn(int(r[j + u]));
          v[j + u] = QMODE == 0 ? __fmul_rn(__fmul_rn(a, xsr), sv[u]) : __fmul_rn(a, __fmul_rn(xsr, sv[u]));
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float s = j < ncols ? __ldg(sch + n0 + j) : 0.f;
        const float a = __int2float_rn(int(r[j]));
        v[j] = QMODE == 0 ? __fmul_rn(__fmul_rn(a, xsr), s) : __fmul_rn(a, __fmul_rn(xsr, s));
      }
    }
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      v[j] = round_out<OUT>(v[j]);
      if constexpr (BIAS) {
        if (j < ncols) v[j] = round_out<OUT>(v[j] + bias_at<OUT>(bias, n0 + j));
      }
    }
    if constexpr (OUT == OUT_FP32) {
      float* o = reinterpret_cast<float*>(orow) + n0;
      if (vec_ok && ncols == 32) {
#pragma unroll
        for (int j = 0; j < 32; j += 4) *reinterpret_cast<float4*>(o + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
      } else {
        for (int j = 0; j < ncols; ++j) o[j] = v[j];
      }
    } else {
      uint32_t w[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        if constexpr (OUT == OUT_BF16) {
          const __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);  // exact: values already bf16
          w[j] = *reinterpret_cast<const uint32_t*>(&h);
        } else {
          const __half2 h = __floats2half2_rn(v[2 * j], v[2 * j + 1]);
          w[j] = *reinterpret_cast<const uint32_t*>(&h);
        }
      }
      uint16_t* o = reinterpret_cast<uint16_t*>(orow) + n0;
      if (vec_ok && ncols == 32) {
#pragma unroll
        for (int j = 0; j < 16; j += 4) *reinterpret_cast<uint4*>(o + 2 * j) = make_uint4(w[j], w[j + 1], w[j + 2], w[j + 3]);
      } else {
        for (int j = 0; j < ncols; ++j) o[j] = static_cast<uint16_t>(w[j >> 1] >> (16 * (j & 1)));
      }
    }
  }
}

// Tile order: "super-columns" of `gn` N tiles; inside one, N runs fastest and M next, so the CTAs working at the same
// time share a weight block of gn x BN rows (sized by the host to stay resident in L2) and a slab of activation rows.
__device__ __forceinline__ void tile_coords(int tile, int m_tiles, int n_tiles, int gn, int& mt, int& nt) {
  const int group = tile / (gn * m_tiles);
  const int first_n = group * gn;
  const int width = min(gn, n_tiles - first_n);
  const int local = tile - group * gn * m_tiles;
  mt = local / width;
  nt = first_n + (local - mt * width);
}

template <int BN, int OUT, bool BIAS, int QMODE>
__global__ void __launch_bounds__(192, 1)
    gemm_i8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const float* __restrict__ xs, const float* __restrict__ sch, const void* __restrict__ bias,
                   void* __restrict__ out, int64_t ldo, int M, int N, int K, int gn) {
  using C = GemmCfg<BN>;
  extern __shared__ __align__(1024) unsigned char gemm_smem[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(gemm_smem) + 1023) & ~uintptr_t(1023));
  unsigned char* sA = smem;
  unsigned char* sB = smem + C::STAGES * C::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + C::STAGES * C::B_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* tfull = empty + C::STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* mdone = tempty + 2;  // MMA drain before TMEM is freed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mdone + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m_tiles = (M + BM - 1) / BM, n_tiles = (N + BN - 1) / BN;
  const int num_tiles = m_tiles * n_tiles;
  const int num_kb = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 128);
    }
    mbar_init(mdone, 1);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
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
    if (lane == 0) {  // ---------------------------------------------------------------- TMA producer
      int stage = 0;
      uint32_t phase = 0;
      long long fills = 0;
      for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
        int mt, nt;
        tile_coords(tile, m_tiles, n_tiles, gn, mt, nt);
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
          tma_load_2d(sA + stage * C::A_BYTES, &tmA, &full[stage], kb * BK, mt * BM);
          tma_load_2d(sB + stage * C::B_BYTES, &tmB, &full[stage], kb * BK, nt * BN);
          ++fills;
          if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
      }
      // drain: the last STAGES loads issued must have landed before the CTA may exit (bounded)
      for (long long j = fills > C::STAGES ? fills - C::STAGES : 0; j < fills; ++j)
        if (!mbar_wait_drain(&full[j % C::STAGES], static_cast<uint32_t>((j / C::STAGES) & 1))) break;
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ---------------------------------------------------------------- MMA issuer
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++it) {
        const int buf = it & 1;
        if (!mbar_wait(&tempty[buf], ((it >> 1) & 1) ^ 1, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * BN);
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + stage * C::A_BYTES), b0 = smem_u32(sB + stage * C::B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 32; ++k)
            mma_i8(d_tmem, smem_desc_sw128(a0 + 32 * k), smem_desc_sw128(b0 + 32 * k), C::IDESC, (kb | k) != 0);
          mma_commit(&empty[stage]);
          if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        mma_commit(&tfull[buf]);
      }
      mma_commit(mdone);  // completes when every MMA issued above has finished
      mbar_wait_drain(mdone, 0);
    }
  } else {  // -------------------------------------------------------------------------------------- epilogue
    const int quad = warp & 3;  // TMEM lanes [32 quad, 32 quad + 32) are this warp's
    const size_t osz = OUT == OUT_FP32 || OUT == OUT_S32 ? 4 : 2;
    const bool vec_ok = (ldo % (16 / static_cast<int64_t>(osz))) == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0;
    int it = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++it) {
      const int buf = it & 1;
      const bool ok = mbar_wait(&tfull[buf], (it >> 1) & 1, abort_flag);
      if (!__all_sync(0xffffffffu, ok)) break;  // tcgen05.ld below is warp-collective: leave together
      tc_fence_after();
      int mt, nt;
      tile_coords(tile, m_tiles, n_tiles, gn, mt, nt);
      const int row = mt * BM + quad * 32 + lane;
      const float xsr = (OUT != OUT_S32 && row < M) ? xs[row] : 0.f;
      char* orow = static_cast<char*>(out) + static_cast<size_t>(row) * static_cast<size_t>(ldo) * osz;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(buf * BN + c * 32), r);
        tmem_ld_wait();
        const int n0 = nt * BN + c * 32;
        if (row < M && n0 < N) epilogue_row32<OUT, BIAS, QMODE>(r, xsr, sch, bias, orow, n0, min(32, N - n0), vec_ok);
      }
      tc_fence_before();
      mbar_arrive(&tempty[buf]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// ------------------------------------------------------------------------------------------------ CTA-pair variant
// 256 x 256 output tiles on a cluster of two CTAs (one per SM of a TPC) with tcgen05.mma.cta_group::2: CTA r holds A rows
// [128 r, 128 r + 128) and B rows (= output columns) [128 r, 128 r + 128) of the tile in its own shared memory, the
// leader (rank 0) issues one 256 x 256 x 32 MMA that reads both CTAs' halves, and each CTA's TMEM receives its 128 rows
// x 256 columns.  Per SM and per MMA the tensor core reads 4 KB of A and 4 KB of B from shared memory (the 1-CTA
// 128 x 256 tile reads 4 + 8 KB), the co-limit the 1-CTA kernel hits.
//   full[s]    leader only: one arrive.expect_tx (both CTAs' bytes) + the TMA bytes of both CTAs
//   empty[s]   both CTAs: the leader's tcgen05.commit arrives on both
//   tfull[b]   both CTAs: accumulator b is complete (leader's commit, both CTAs)
//   tempty[b]  leader only: 2 x 128 epilogue threads (the peer's arrive remotely) have drained accumulator b
constexpr int P_BN = 256;      // output columns per pair tile (N of the MMA)
constexpr int P_BM = 2 * BM;   // output rows per pair tile
#ifndef H3B_PAIR_STAGES
#define H3B_PAIR_STAGES 6  // build-time tuning knob: TMA/MMA ring depth of the CTA-pair kernel (7 measured the same)
#endif
constexpr int P_STAGES = H3B_PAIR_STAGES;
constexpr int P_A_BYTES = BM * BK;           // this CTA's A half per stage
constexpr int P_B_BYTES = (P_BN / 2) * BK;   // this CTA's B half per stage
constexpr int P_STAGE_BYTES = P_A_BYTES + P_B_BYTES;
constexpr int P_TMEM_COLS = 2 * P_BN;
constexpr int P_SMEM = 1024 + P_STAGES * P_STAGE_BYTES + 256;
constexpr uint32_t P_IDESC = idesc_i8(P_BM, P_BN);

template <int OUT, bool BIAS, int QMODE>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(192, 1)
    gemm_i8_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const float* __restrict__ xs, const float* __restrict__ sch, const void* __restrict__ bias,
                        void* __restrict__ out, int64_t ldo, int M, int N, int K, int gn) {
  extern __shared__ __align__(1024) unsigned char gemm_smem[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(gemm_smem) + 1023) & ~uintptr_t(1023));
  unsigned char* sA = smem;
  unsigned char* sB = smem + P_STAGES * P_A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + P_STAGES * P_B_BYTES);
  uint64_t* empty = full + P_STAGES;
  uint64_t* tfull = empty + P_STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* mdone = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mdone + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int m_tiles = (M + P_BM - 1) / P_BM, n_tiles = (N + P_BN - 1) / P_BN;
  const int num_tiles = m_tiles * n_tiles;
  const int num_kb = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < P_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 2 * 128);
    }
    mbar_init(mdone, 1);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, P_TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers initialised and TMEM allocated before any remote arrive or MMA
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {  // ---------------------------------------------------------------- TMA producer (both CTAs)
      int stage = 0;
      uint32_t phase = 0;
      long long fills = 0;
      for (int tile = pair; tile < num_tiles; tile += npairs) {
        int mt, nt;
        tile_coords(tile, m_tiles, n_tiles, gn, mt, nt);
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) { ok = false; break; }
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * P_STAGE_BYTES);
          const uint32_t bar = mapa_rank(smem_u32(&full[stage]), 0);
          tma_load_2d_pair(sA + stage * P_A_BYTES, &tmA, bar, kb * BK, mt * P_BM + static_cast<int>(rank) * BM);
          tma_load_2d_pair(sB + stage * P_B_BYTES, &tmB, bar, kb * BK, nt * P_BN + static_cast<int>(rank) * (P_BN / 2));
          ++fills;
          if (++stage == P_STAGES) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
      }
      // drain: this CTA's last loads must have landed before it may exit.  Their bytes count on the leader's full
      // barriers, which only the leader can wait on; the peer waits for the leader's MMAs to release the stages instead.
      for (long long j = fills > P_STAGES ? fills - P_STAGES : 0; j < fills; ++j) {
        if (leader) {
          if (!mbar_wait_drain(&full[j % P_STAGES], static_cast<uint32_t>((j / P_STAGES) & 1))) break;
        } else {
          if (!mbar_wait_drain(&empty[j % P_STAGES], static_cast<uint32_t>((j / P_STAGES) & 1))) break;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {  // ------------------------------------------------------- MMA issuer (leader only)
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      for (int tile = pair; tile < num_tiles; tile += npairs, ++it) {
        const int buf = it & 1;
        if (!mbar_wait_cl(&tempty[buf], ((it >> 1) & 1) ^ 1, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * P_BN);
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + stage * P_A_BYTES), b0 = smem_u32(sB + stage * P_B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 32; ++k)
            mma_i8_pair(d_tmem, smem_desc_sw128(a0 + 32 * k), smem_desc_sw128(b0 + 32 * k), P_IDESC, (kb | k) != 0);
          mma_commit_pair(&empty[stage], 0x3);
          if (++stage == P_STAGES) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        mma_commit_pair(&tfull[buf], 0x3);
      }
      mma_commit_pair(mdone, 0x1);  // completes when every MMA issued above has finished
      mbar_wait_drain(mdone, 0);
    }
  } else {  // -------------------------------------------------------------------------------------- epilogue (both CTAs)
    const int quad = warp & 3;
    const size_t osz = OUT == OUT_FP32 || OUT == OUT_S32 ? 4 : 2;
    const bool vec_ok = (ldo % (16 / static_cast<int64_t>(osz))) == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0;
    const uint32_t tempty_leader0 = mapa_rank(smem_u32(&tempty[0]), 0), tempty_leader1 = mapa_rank(smem_u32(&tempty[1]), 0);
    int it = 0;
    for (int tile = pair; tile < num_tiles; tile += npairs, ++it) {
      const int buf = it & 1;
      const bool ok = mbar_wait(&tfull[buf], (it >> 1) & 1, abort_flag);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      int mt, nt;
      tile_coords(tile, m_tiles, n_tiles, gn, mt, nt);
      const int row = mt * P_BM + static_cast<int>(rank) * BM + quad * 32 + lane;
      const float xsr = (OUT != OUT_S32 && row < M) ? xs[row] : 0.f;
      char* orow = static_cast<char*>(out) + static_cast<size_t>(row) * static_cast<size_t>(ldo) * osz;
#pragma unroll 1
      for (int c = 0; c < P_BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(buf * P_BN + c * 32), r);
        tmem_ld_wait();
        const int n0 = nt * P_BN + c * 32;
        if (row < M && n0 < N) epilogue_row32<OUT, BIAS, QMODE>(r, xsr, sch, bias, orow, n0, min(32, N - n0), vec_ok);
      }
      tc_fence_before();
      mbar_arrive_cluster(buf ? tempty_leader1 : tempty_leader0);
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no CTA leaves while its pair may still read its shared memory or arrive on its barriers
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, P_TMEM_COLS);
  }
}

// ------------------------------------------------------------------------------------------------ host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 2-D uint8 tensor map over rows of `inner` bytes (row stride `ld` bytes), box = 128 bytes x box_rows, 128-byte swizzle,
// out-of-range elements read as zero.
static int make_map(CUtensorMap* map, const void* base, int64_t inner, int64_t rows, int64_t ld, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(H3B_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable (driver too old?)");
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld)};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(BK), static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(H3B_ERR_CUDA, "cuTensorMapEncodeTiled failed (code " + std::to_string(int(r)) + ")");
  return H3B_OK;
}

static int num_sms() {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

// Largest N tile that still gives every SM a tile; the smallest one otherwise.
// N tile of a GEMM: 256 when 256-wide tiles give every SM work (the CTA-pair kernel's regime); otherwise the width that
// minimises waves x width -- the time of the busiest SM -- so that small-M problems neither leave SMs idle nor run a
// nearly empty last wave (wider on ties: fewer re-reads of A).
static int pick_bn(int M, int N) {
  const int sms = num_sms();
  const int64_t mt = (M + BM - 1) / BM;
  if (mt * ((N + 255) / 256) >= sms) return 256;
  int best = 32;
  int64_t best_cost = -1;
  for (int bn : {256, 192, 128, 96, 64, 32}) {
    const int64_t tiles = mt * ((N + bn - 1) / bn);
    const int64_t cost = ((tiles + sms - 1) / sms) * bn;
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best = bn;
    }
  }
  return best;
}

}  // namespace h3b
