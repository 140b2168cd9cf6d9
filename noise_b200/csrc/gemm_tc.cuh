// Persistent tcgen05 GEMM engine for the population forward: C[M, N] = A[M, K] * B[N, K]^T with
// bf16 operands in HBM, fp32 accumulators in tensor memory, and a pluggable epilogue that turns each
// accumulator row into the layer's outputs (rank-1 draw terms, RoPE, norms, residual mixing, ...).
//
// Roles (10 warps, one CTA per SM):
//   warp 0      TMA producer: streams 128x64 A tiles and 256x64 B tiles into a ring of smem stages.
//   warp 1      MMA issuer: one thread issues tcgen05.mma (M=128, N=256, K=16) into one of two TMEM
//               accumulators (2 x 256 fp32 columns = all 512 columns), commits stage releases.
//   warps 2..9  epilogue: warp w reads TMEM lanes 32*(w%4).. of column half (w-2)/4 and hands 64-column
//               groups to the epilogue functor, then releases the accumulator.
// Tile schedule, chosen per epilogue (Epi::kInterleaveN):
//   false  a CTA owns whole M tiles: all N tiles of an M tile run back to back on one CTA, so per-row
//          state can live in epilogue registers across the N loop and A stays hot in L2;
//   true   tiles t = m * n_tiles + n are dealt round-robin, so the n_tiles CTAs that share an A tile
//          run at the same time and the A tile is read from DRAM once (for large-K, few-N GEMMs).
// A "unit" is one M tile (false) or one tile (true); row state is set up per unit.
//
// Epilogue functor contract (all methods run on every epilogue thread; `row` is global):
//   static constexpr int kSmemBytes;                 shared memory the functor needs
//   static constexpr bool kInterleaveN;              tile schedule above
//   __device__ Epi(const Params&, uint8_t* smem, int epi_warp, int lane)
//   __device__ void begin_mtile(int m_tile, int row)               once per unit
//   __device__ void begin_tile(int m_tile, int n_tile, int col0)   warp-uniform; may __syncwarp
//   __device__ void group(int row, int col, float (&v)[64])        64 consecutive columns of `row`
//   __device__ void end_mtile(int m_tile, int n_tile, int row)     once per unit (n_tile = last one)
// Optional:
//   static constexpr bool kTf32;                     true: A and B are fp32 in HBM and the MMAs run
//                                                    kind::tf32 (32 K elements per 128-byte row)
//   __device__ void finish()                                       once, after the last unit
//   __device__ void next_unit(int m_tile, int n_begin)             at the start of each unit: the 128-row
//                  tile and first N tile of this CTA's next unit (m_tile = -1: none), for prefetches
#pragma once

#include <type_traits>

#include "profile.cuh"
#include "ptx.cuh"

namespace noise {

struct GemmShape {
  int M, N, K;
  int m_tiles, n_tiles, k_blocks;
  int* status;
  // Batched (block-diagonal) products, whole-M-tile schedule only: with batch_m_tiles > 0, rows
  // [b * batch_m_tiles * 128, (b + 1) * batch_m_tiles * 128) of A meet only rows
  // [b * batch_n_tiles * 256, (b + 1) * batch_n_tiles * 256) of B: batch b's own product.
  int batch_m_tiles = 0, batch_n_tiles = 0;
};

// The tiles of one schedule unit (see the header comment).
template <bool kInterleaveN>
struct TileUnit {
  int m, n_begin, n_end;
  __device__ __forceinline__ TileUnit(int u, const GemmShape& s) {
    if (kInterleaveN) {
      m = u / s.n_tiles;
      n_begin = u % s.n_tiles;
      n_end = n_begin + 1;
    } else if (s.batch_m_tiles > 0) {
      m = u;
      n_begin = (u / s.batch_m_tiles) * s.batch_n_tiles;
      n_end = n_begin + s.batch_n_tiles;
    } else {
      m = u;
      n_begin = 0;
      n_end = s.n_tiles;
    }
  }
  __host__ __device__ static int count(const GemmShape& s) { return kInterleaveN ? s.m_tiles * s.n_tiles : s.m_tiles; }
};

template <class E, class = void>
struct HasNextUnit : std::false_type {};
template <class E>
struct HasNextUnit<E, std::void_t<decltype(&E::next_unit)>> : std::true_type {};

template <class E, class = void>
struct OperandTf32 : std::false_type {};
template <class E>
struct OperandTf32<E, std::void_t<decltype(E::kTf32)>> : std::integral_constant<bool, E::kTf32> {};

// Self-test traits (the wait-timeout test instantiation): kWaitBudget replaces the cycle budget of
// every wait; kSkipLoads makes the producer arm its barriers without issuing the copies, so the MMA
// warp's first wait runs out and the kernel ends through its timeout path.
template <class E, class = void>
struct WaitBudget : std::integral_constant<long long, kWaitCycleBudget> {};
template <class E>
struct WaitBudget<E, std::void_t<decltype(E::kWaitBudget)>> : std::integral_constant<long long, E::kWaitBudget> {};

template <class E, class = void>
struct SkipsLoads : std::false_type {};
template <class E>
struct SkipsLoads<E, std::void_t<decltype(E::kSkipLoads)>> : std::integral_constant<bool, E::kSkipLoads> {};

template <class E, class = void>
struct HasFinish : std::false_type {};
template <class E>
struct HasFinish<E, std::void_t<decltype(&E::finish)>> : std::true_type {};

// Tiles are 128 bytes of K per row: 64 bf16 or 32 fp32 (tf32) elements; one MMA consumes 32 bytes of K
// (K = 16 bf16 or K = 8 tf32), so a stage is always 4 MMAs.
template <int kStages, int kElemBytes = 2>
struct GemmLayout {
  static constexpr int BM = 128, BN = 256, BK = 128 / kElemBytes;
  static constexpr int kEpiWarps = 8;
  static constexpr int kThreads = (2 + kEpiWarps) * 32;
  static constexpr int kABytes = BM * 128;
  static constexpr int kBBytes = BN * 128;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kBarrierBytes = 256;
  static constexpr int kCoreBytes = kStages * kStageBytes + kBarrierBytes;
};

template <class Epi, int kStages>
__global__ void __launch_bounds__(GemmLayout<kStages>::kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const GemmShape shape, const __grid_constant__ typename Epi::Params ep) {
  constexpr bool kTf32 = OperandTf32<Epi>::value;
  constexpr long long kBudget = WaitBudget<Epi>::value;
  using L = GemmLayout<kStages, kTf32 ? 4 : 2>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = base;
  uint8_t* sB = base + kStages * L::kABytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + kStages * L::kStageBytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + kStages;
  uint64_t* tfull = bars + 2 * kStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint8_t* epi_smem = base + L::kCoreBytes;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int* status = shape.status;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], L::kEpiWarps);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
    prefetch_tensormap(&tmA);
    prefetch_tensormap(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      uint32_t stage = 0, phase = 0;
      uint32_t issued_phase[kStages];
      bool issued[kStages];
      for (int s = 0; s < kStages; ++s) issued[s] = false, issued_phase[s] = 0;
      const uint64_t keep = l2_policy_evict_last();  // weights: every CTA re-reads them
      bool ok = true;
      const int units = TileUnit<Epi::kInterleaveN>::count(shape);
      for (int u = blockIdx.x; ok && u < units; u += gridDim.x) {
        const TileUnit<Epi::kInterleaveN> tu(u, shape);
        const int m = tu.m;
        for (int n = tu.n_begin; ok && n < tu.n_end; ++n) {
          for (int kb = 0; kb < shape.k_blocks; ++kb) {
            if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, status, kBudget)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&full[stage], L::kStageBytes);
            if constexpr (SkipsLoads<Epi>::value) {
              if (++stage == kStages) stage = 0, phase ^= 1;
              continue;  // self-test: the barrier waits for bytes that never come
            }
            tma_load_2d(sA + stage * L::kABytes, &tmA, &full[stage], kb * L::BK, m * L::BM);
            tma_load_2d_hint(sB + stage * L::kBBytes, &tmB, &full[stage], kb * L::BK, n * L::BN, keep);
            issued[stage] = true;
            issued_phase[stage] = phase;
            if (++stage == kStages) stage = 0, phase ^= 1;
          }
        }
      }
      // Every copy this thread started lands before the CTA can exit.
      for (int s = 0; s < kStages; ++s)
        if (issued[s]) mbar_wait(&full[s], issued_phase[s], abort_flag, status, kBudget);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      const uint32_t idesc = make_idesc(kTf32 ? 2 : 1, L::BM, L::BN);
      uint32_t stage = 0, phase = 0, t = 0;
      bool ok = true;
      const int units = TileUnit<Epi::kInterleaveN>::count(shape);
      for (int u = blockIdx.x; ok && u < units; u += gridDim.x) {
        const TileUnit<Epi::kInterleaveN> tu(u, shape);
        for (int n = tu.n_begin; ok && n < tu.n_end; ++n, ++t) {
          const uint32_t acc = t & 1, acc_phase = (t >> 1) & 1;
          if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag, status, kBudget)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem_base + acc * L::BN;
          for (int kb = 0; kb < shape.k_blocks; ++kb) {
            if (!mbar_wait(&full[stage], phase, abort_flag, status, kBudget)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint64_t da = smem_desc_sw128(sA + stage * L::kABytes);
            const uint64_t db = smem_desc_sw128(sB + stage * L::kBBytes);
#pragma unroll
            for (int k = 0; k < 4; ++k) {  // 32 bytes of K per MMA: descriptor start + 2 (16-byte units)
              if constexpr (kTf32) tc_mma_tf32(d, da + 2 * k, db + 2 * k, idesc, (kb | k) != 0 ? 1u : 0u);
              else tc_mma_f16(d, da + 2 * k, db + 2 * k, idesc, (kb | k) != 0 ? 1u : 0u);
            }
            tc_commit(&empty[stage]);
            if (++stage == kStages) stage = 0, phase ^= 1;
          }
          if (ok) tc_commit(&tfull[acc]);
        }
      }
      // No MMA may still be writing TMEM when it is freed.
      tc_commit(drain);
      mbar_wait(drain, 0, abort_flag, status, kBudget);
    }
    __syncwarp();
  } else {
    // ---------------- epilogue ----------------
    const int ew = warp - 2;
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    const int half = ew >> 2;      // column half of the 256-wide tile
    Epi epi(ep, epi_smem, ew, lane);
    uint32_t t = 0;
    bool ok = true;
    const int units = TileUnit<Epi::kInterleaveN>::count(shape);
    for (int u = blockIdx.x; ok && u < units; u += gridDim.x) {
      const TileUnit<Epi::kInterleaveN> tu(u, shape);
      const int m = tu.m;
      const int row = m * L::BM + quarter * 32 + lane;
      if constexpr (HasNextUnit<Epi>::value) {
        const int un = u + (int)gridDim.x;
        if (un < units) {
          const TileUnit<Epi::kInterleaveN> tn(un, shape);
          epi.next_unit(tn.m, tn.n_begin);
        } else {
          epi.next_unit(-1, 0);
        }
      }
      epi.begin_mtile(m, row);
      for (int n = tu.n_begin; n < tu.n_end; ++n, ++t) {
        const uint32_t acc = t & 1, acc_phase = (t >> 1) & 1;
        if (!mbar_wait(&tfull[acc], acc_phase, abort_flag, status, kBudget)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int col0 = half * (L::BN / 2);
        epi.begin_tile(m, n, n * L::BN + col0);
        const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * L::BN + col0;
#pragma unroll 1
        for (int g = 0; g < L::BN / 2 / 64; ++g) {
          float v[64];
          tmem_ld64(taddr + g * 64, v);
          if (g == L::BN / 2 / 64 - 1) {
            // All TMEM reads of this tile are done: hand the accumulator back to the MMA warp.
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[acc]);
          }
          epi.group(row, n * L::BN + col0 + g * 64, v);
        }
      }
      if (ok) epi.end_mtile(m, tu.n_end - 1, row);
    }
    if constexpr (HasFinish<Epi>::value) epi.finish();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

// ---------------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled_fn();
int device_sm_count();

// Tensor map of a row-major [rows, cols] matrix read in boxes of box_rows x box_cols elements with
// 128-byte swizzle (box_cols * element size must be 128 bytes).
int make_tmap_2d(CUtensorMap* map, const void* ptr, CUtensorMapDataType dtype, int elem_bytes, uint64_t rows,
                 uint64_t cols, uint64_t row_stride_elems, uint32_t box_rows, uint32_t box_cols);

template <class Epi, int kStages>
int launch_gemm_tc(const void* A, const void* B, int M, int N, int K, int lda, int ldb,
                   const typename Epi::Params& ep, int* status, cudaStream_t stream, int kind = kKindOther,
                   int max_ctas = 0, int batch_m = 0, int batch_n = 0) {
  constexpr bool kTf32 = OperandTf32<Epi>::value;
  constexpr int kElem = kTf32 ? 4 : 2;
  using L = GemmLayout<kStages, kElem>;
  const CUtensorMapDataType dt = kTf32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  if (M <= 0 || N <= 0 || K <= 0 || M % L::BM || N % L::BN || K % L::BK) return kStatusBadArgument;
  if ((reinterpret_cast<uintptr_t>(A) & 15) || (reinterpret_cast<uintptr_t>(B) & 15)) return kStatusBadArgument;
  if (((int64_t)lda * kElem) % 16 || ((int64_t)ldb * kElem) % 16 || lda < K || ldb < K) return kStatusBadArgument;
  CUtensorMap ta, tb;
  if (make_tmap_2d(&ta, A, dt, kElem, M, K, lda, L::BM, L::BK)) return kStatusBadArgument;
  if (make_tmap_2d(&tb, B, dt, kElem, N, K, ldb, L::BN, L::BK)) return kStatusBadArgument;
  GemmShape shape{M, N, K, M / L::BM, N / L::BN, K / L::BK, status};
  if (batch_m > 0) {  // batch_m rows of A against batch_n rows of B, batch by batch
    if (Epi::kInterleaveN || batch_m % L::BM || batch_n % L::BN || M % batch_m || N % batch_n ||
        M / batch_m != N / batch_n)
      return kStatusBadArgument;
    shape.batch_m_tiles = batch_m / L::BM;
    shape.batch_n_tiles = batch_n / L::BN;
  }
  const int smem = 1024 + L::kCoreBytes + Epi::kSmemBytes;
  static bool configured = false;  // one instantiation = one kernel
  if (!configured) {
    if (cudaFuncSetAttribute(gemm_tc_kernel<Epi, kStages>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
        cudaSuccess)
      return kStatusLaunchFailed;
    configured = true;
  }
  int grid = device_sm_count();
  if (max_ctas > 0 && max_ctas < grid) grid = max_ctas;
  const int units = Epi::kInterleaveN ? shape.m_tiles * shape.n_tiles : shape.m_tiles;
  if (grid > units) grid = units;
  LaunchScope scope(kind, stream);
  gemm_tc_kernel<Epi, kStages><<<grid, L::kThreads, smem, stream>>>(ta, tb, shape, ep);
  return cudaGetLastError() == cudaSuccess ? kStatusOk : kStatusLaunchFailed;
}

}  // namespace noise
