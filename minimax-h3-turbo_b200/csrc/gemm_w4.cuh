// Kernel KB with the int4 weight decode in its producer warps (the small-M, weight-bandwidth-bound regime).
//
// Same product and epilogue as gemm_i8_kernel, but B arrives as the packed int4 codebook indices of the weight: TMA
// brings a BN x 64-byte tile of packed nibbles per stage, eight decoder warps turn it into the BN x 128 int8 levels the
// tensor core reads (level tables per scale group and byte permutes, exactly decode.cuh's levels), write them into the
// stage's 128-byte-swizzled B tile, and arrive on the stage's barrier after a generic->async proxy fence.  The weight
// crosses HBM once at 0.5 byte per element and no int8 grid is written.  Used when the M tiles are few (each B tile is
// decoded once per M tile); for large M a separate decode pass followed by the CTA-pair kernel does less work.
//
// Warps: 0 TMA producer (A tile + packed B tile), 1 MMA issuer, 2-5 epilogue, 6-13 decoders (448 threads).
//   pkfull[s]  packed tile of stage s landed (TMA bytes)
//   full[s]    A bytes (TMA) + one arrival per decoder warp: the stage is ready for the MMA
//   empty[s]   the MMAs of stage s finished (tcgen05.commit): A, B and the packed tile may be refilled
// Formats: scales fp16 / bf16 / fp32 with group 128, or fp8 e4m3 with group 16 (the benchmark and checkpoint formats).
#pragma once

#include "decode.cuh"
#include "gemm_sm100.cuh"

namespace h3b {

template <int BN>
struct W4Cfg {
  static constexpr int STAGES = BN >= 192 ? 4 : (BN >= 128 ? 4 : (BN >= 96 ? 5 : 6));
  static constexpr int A_BYTES = BM * BK;
  static constexpr int B_BYTES = BN * BK;
  static constexpr int P_BYTES = BN * (BK / 2);
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES + P_BYTES;
  static constexpr int TMEM_COLS = GemmCfg<BN>::TMEM_COLS;
  static constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + 4096 + 512;  // ring + fp8 level tables + barriers
  static constexpr uint32_t IDESC = idesc_i8(BM, BN);
  // decoder warps: 8, or 6 when BN is a multiple of 96, so that a thread's CPT chunks (CPT dividing the 8 chunks
  // of a row) lie in one row of the B tile
  static constexpr int DWARPS = BN % 96 == 0 ? 6 : 8;
  static constexpr int CPT = BN * 8 / (32 * DWARPS);  // 16-weight chunks per decoder thread and stage
  static_assert(CPT >= 1 && 8 % CPT == 0 && CPT * 32 * DWARPS == BN * 8, "decoder chunks must tile the rows");
};

template <int BN, int OUT, bool BIAS, int QMODE, int SDT>
__global__ void __launch_bounds__(192 + 32 * W4Cfg<BN>::DWARPS, 1)
    gemm_w4_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmP,
                   const void* __restrict__ s_rel, int64_t lds, const float* __restrict__ codebook,
                   const float* __restrict__ xs, const float* __restrict__ sch, const void* __restrict__ bias,
                   void* __restrict__ out, int64_t ldo, int M, int N, int K, int gn) {
  using C = W4Cfg<BN>;
  constexpr int GROUP = SDT == H3B_FP8_E4M3 ? 16 : 128;
  extern __shared__ __align__(1024) unsigned char gemm_smem[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(gemm_smem) + 1023) & ~uintptr_t(1023));
  unsigned char* sA = smem;
  unsigned char* sB = smem + C::STAGES * C::A_BYTES;
  unsigned char* sP = sB + C::STAGES * C::B_BYTES;
  uint4* lut = reinterpret_cast<uint4*>(sP + C::STAGES * C::P_BYTES);  // fp8: 256 level tables
  uint64_t* full = reinterpret_cast<uint64_t*>(lut + 256);
  uint64_t* pkfull = full + C::STAGES;
  uint64_t* empty = pkfull + C::STAGES;
  uint64_t* tfull = empty + C::STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* mdone = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mdone + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m_tiles = (M + BM - 1) / BM, n_tiles = (N + BN - 1) / BN;
  const int num_tiles = m_tiles * n_tiles;
  const int num_kb = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1 + C::DWARPS);
      mbar_init(&pkfull[s], 1);
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
  float cb[16];
  if (warp >= 6) {
#pragma unroll
    for (int i = 0; i < 16; ++i) cb[i] = __ldg(codebook + i);
    if constexpr (SDT == H3B_FP8_E4M3) {
      for (int b = threadIdx.x - 192; b < 256; b += 32 * C::DWARPS) lut[b] = level_table(cb, fp8e4m3_to_f32(static_cast<uint32_t>(b)));
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
          mbar_arrive_expect_tx(&full[stage], C::A_BYTES);
          tma_load_2d(sA + stage * C::A_BYTES, &tmA, &full[stage], kb * BK, mt * BM);
          mbar_arrive_expect_tx(&pkfull[stage], C::P_BYTES);
          tma_load_2d(sP + stage * C::P_BYTES, &tmP, &pkfull[stage], kb * (BK / 2), nt * BN);
          ++fills;
          if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
      }
      for (long long j = fills > C::STAGES ? fills - C::STAGES : 0; j < fills; ++j) {  // drain (bounded)
        const uint32_t par = static_cast<uint32_t>((j / C::STAGES) & 1);
        if (!mbar_wait_drain(&pkfull[j % C::STAGES], par)) break;
        if (!mbar_wait_drain(&empty[j % C::STAGES], par)) break;
      }
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
      mma_commit(mdone);
      mbar_wait_drain(mdone, 0);
    }
  } else if (warp < 6) {  // ------------------------------------------------------------------ epilogue
    const int quad = warp & 3;
    const size_t osz = OUT == OUT_FP32 || OUT == OUT_S32 ? 4 : 2;
    const bool vec_ok = (ldo % (16 / static_cast<int64_t>(osz))) == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0;
    int it = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++it) {
      const int buf = it & 1;
      const bool ok = mbar_wait(&tfull[buf], (it >> 1) & 1, abort_flag);
      if (!__all_sync(0xffffffffu, ok)) break;
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
  } else {  // ----------------------------------------------------------------------------------- decoders
    const int dt = threadIdx.x - 192;                 // 0 .. 32 DWARPS - 1
    const int r_loc = (dt * C::CPT) >> 3;             // this thread's row of the B tile
    const int j0 = (dt * C::CPT) & 7;                 // its first 16-weight chunk in the row
    struct Scales {
      float g;                 // group-128 formats: the stage's one scale of this row
      uint32_t f8[C::CPT];     // fp8 group 16: the scale byte of each chunk
    };
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
      int mt, nt;
      tile_coords(tile, m_tiles, n_tiles, gn, mt, nt);
      const int n = nt * BN + r_loc;
      const bool row_ok = n < N;
      const unsigned char* srow = static_cast<const unsigned char*>(s_rel) +
                                  static_cast<int64_t>(row_ok ? n : 0) * lds * (SDT == H3B_FP8_E4M3 ? 1 : (SDT == H3B_FP32 ? 4 : 2));
      // scales are global loads: they are issued two stages before they are used, so their latency hides behind the
      // decode of the stages in between
      auto load_scales = [&](int kb) {
        Scales sc;
        sc.g = 0.f;
        if constexpr (SDT == H3B_FP8_E4M3) {
#pragma unroll
          for (int i = 0; i < C::CPT; ++i) {
            const int64_t e0 = static_cast<int64_t>(kb) * BK + 16 * (j0 + i);
            sc.f8[i] = (row_ok && e0 < K) ? static_cast<uint32_t>(srow[e0 / GROUP]) : 0u;
          }
        } else {
#pragma unroll
          for (int i = 0; i < C::CPT; ++i) sc.f8[i] = 0u;
          const int64_t e0 = static_cast<int64_t>(kb) * BK + 16 * j0;
          sc.g = (row_ok && e0 < K) ? scale_at<SDT>(srow, e0 / GROUP) : 0.f;
        }
        return sc;
      };
      auto decode_stage = [&](const Scales& sc) -> bool {
        if (!mbar_wait(&pkfull[stage], phase, abort_flag)) return false;
        uint4 t = make_uint4(0, 0, 0, 0);
        if constexpr (SDT != H3B_FP8_E4M3) t = level_table(cb, sc.g);
        const unsigned char* prow = sP + stage * C::P_BYTES + r_loc * (BK / 2);
        unsigned char* brow = sB + stage * C::B_BYTES + r_loc * BK;
#pragma unroll
        for (int i = 0; i < C::CPT; ++i) {
          const int j = j0 + i;
          if constexpr (SDT == H3B_FP8_E4M3) t = lut[sc.f8[i]];
          const uint2 pk = *reinterpret_cast<const uint2*>(prow + 8 * j);
          const uint2 a = decode8(pk.x, t), b = decode8(pk.y, t);
          *reinterpret_cast<uint4*>(brow + ((j ^ (r_loc & 7)) << 4)) = make_uint4(a.x, a.y, b.x, b.y);
        }
        fence_proxy_async_smem();  // the tensor core reads these bytes through the async proxy
        __syncwarp();
        if (lane == 0) mbar_arrive(&full[stage]);
        if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
        return true;
      };
      Scales s0 = load_scales(0), s1 = load_scales(1);
      for (int kb = 0; kb < num_kb; kb += 2) {
        const Scales s2 = load_scales(kb + 2);
        if (!decode_stage(s0)) { ok = false; break; }
        const Scales s3 = load_scales(kb + 3);
        if (kb + 1 < num_kb && !decode_stage(s1)) { ok = false; break; }
        s0 = s2;
        s1 = s3;
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

// 2-D uint8 tensor map over the packed weight: rows of K/2 bytes, box 64 bytes x box_rows, no swizzle, zero fill.
static int make_map_packed(CUtensorMap* map, const void* base, int64_t inner, int64_t rows, int64_t ld, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(H3B_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable (driver too old?)");
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld)};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(BK / 2), static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(H3B_ERR_CUDA, "cuTensorMapEncodeTiled (packed) failed (code " + std::to_string(int(r)) + ")");
  return H3B_OK;
}

template <int BN, int OUT, bool BIAS, int QMODE, int SDT>
static int launch_w4(const int8_t* a, int64_t lda, const void* q4, int64_t ldq4, const void* s_rel, int64_t lds,
                     const float* codebook, const float* xs, const float* sch, const void* bias, void* out, int64_t ldo,
                     int M, int N, int K, cudaStream_t st) {
  using C = W4Cfg<BN>;
  CUtensorMap ta, tp;
  int rc = make_map(&ta, a, K, M, lda, BM);
  if (rc) return rc;
  rc = make_map_packed(&tp, q4, K / 2, N, ldq4, BN);
  if (rc) return rc;
  auto kern = gemm_w4_kernel<BN, OUT, BIAS, QMODE, SDT>;
  static std::atomic<unsigned long long> attr_done{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned long long bit = 1ull << (dev & 63);
  if (!(attr_done.load() & bit)) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(gemm w4)");
    attr_done.fetch_or(bit);
  }
  const int tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  const int sms = num_sms();
  const int grid = tiles < sms ? tiles : sms;
  const int n_tiles = (N + BN - 1) / BN;
  int gn = static_cast<int>((24ll << 20) / (static_cast<int64_t>(BN) * K));
  gn = gn < 1 ? 1 : (gn > n_tiles ? n_tiles : gn);
  kern<<<grid, 192 + 32 * C::DWARPS, C::SMEM, st>>>(ta, tp, s_rel, lds, codebook, xs, sch, bias, out, ldo, M, N, K, gn);
  return check_launch("gemm_w4_kernel");
}

template <int OUT, bool BIAS, int QMODE, int SDT>
static int w4_dispatch_bn(int bn, const int8_t* a, int64_t lda, const void* q4, int64_t ldq4, const void* s_rel,
                          int64_t lds, const float* codebook, const float* xs, const float* sch, const void* bias, void* out,
                          int64_t ldo, int M, int N, int K, cudaStream_t st) {
  switch (bn) {
    case 192: return launch_w4<192, OUT, BIAS, QMODE, SDT>(a, lda, q4, ldq4, s_rel, lds, codebook, xs, sch, bias, out, ldo, M, N, K, st);
    case 128: return launch_w4<128, OUT, BIAS, QMODE, SDT>(a, lda, q4, ldq4, s_rel, lds, codebook, xs, sch, bias, out, ldo, M, N, K, st);
    case 96: return launch_w4<96, OUT, BIAS, QMODE, SDT>(a, lda, q4, ldq4, s_rel, lds, codebook, xs, sch, bias, out, ldo, M, N, K, st);
    case 64: return launch_w4<64, OUT, BIAS, QMODE, SDT>(a, lda, q4, ldq4, s_rel, lds, codebook, xs, sch, bias, out, ldo, M, N, K, st);
    default: return launch_w4<32, OUT, BIAS, QMODE, SDT>(a, lda, q4, ldq4, s_rel, lds, codebook, xs, sch, bias, out, ldo, M, N, K, st);
  }
}

// Every epilogue variant of the kernel for one scale dtype.  Each scale dtype is instantiated in its own translation
// unit (k_w4_<dtype>.cu) so the units compile in parallel.
template <int SDT>
int w4_launch_sdt(int out_dtype, int qmode, int bn, const int8_t* a, int64_t lda, const void* q4, int64_t ldq4,
                  const void* s_rel, int64_t lds, const float* codebook, const float* xs, const float* sch,
                  const void* bias, void* out, int64_t ldo, int M, int N, int K, cudaStream_t st) {
  const bool b = bias != nullptr;
#define H3B_W4(OUTT)                                                                                                   \
  (qmode == H3B_QMODE_CK                                                                                               \
       ? (b ? w4_dispatch_bn<OUTT, true, 0, SDT>(bn, a, lda, q4, ldq4, s_rel, lds, codebook, xs, sch, bias, out, ldo, M, N, K, st) \
            : w4_dispatch_bn<OUTT, false, 0, SDT>(bn, a, lda, q4, ldq4, s_rel, lds, codebook, xs, sch, bias, out, ldo, M, N, K, st)) \
       : (b ? w4_dispatch_bn<OUTT, true, 1, SDT>(bn, a, lda, q4, ldq4, s_rel, lds, codebook, xs, sch, bias, out, ldo, M, N, K, st) \
            : w4_dispatch_bn<OUTT, false, 1, SDT>(bn, a, lda, q4, ldq4, s_rel, lds, codebook, xs, sch, bias, out, ldo, M, N, K, st)))
  switch (out_dtype) {
    case H3B_BF16: return H3B_W4(OUT_BF16);
    case H3B_FP16: return H3B_W4(OUT_FP16);
    case H3B_FP32: return H3B_W4(OUT_FP32);
    case H3B_INT32: return w4_dispatch_bn<OUT_S32, false, 0, SDT>(bn, a, lda, q4, ldq4, s_rel, lds, codebook, xs, sch, nullptr, out, ldo, M, N, K, st);
    default: return fail(H3B_ERR_ARG, "out dtype must be bf16, fp16, fp32 or int32");
  }
#undef H3B_W4
}

}  // namespace h3b
