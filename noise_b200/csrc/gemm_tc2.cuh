// The GEMM engine on CTA pairs: C[M, N] = A[M, K] * B[N, K]^T with the 2-SM tensor-core MMA
// (tcgen05 .cta_group::2). A cluster of two CTAs on two SMs computes 256 x 256 tiles: each CTA
// streams its own 128 rows of A and half (128 rows) of B's 256 per k-block, and one thread of the
// leader (cluster rank 0) issues M = 256, N = 256 MMAs that read both CTAs' shared memory and
// accumulate each CTA's 128 rows in its own TMEM. Against the single-SM engine (gemm_tc.cuh) every
// SM moves 32 KiB instead of 48 KiB from L2 per 4.2 MFLOP, which is what bounds these GEMMs.
//
// Roles per CTA (10 warps): warp 0 TMA producer (both CTAs; completions counted on the leader's
// `full` barriers), warp 1 MMA issuer (leader only; commits multicast to both CTAs' `empty`/`tfull`
// barriers) and TMEM owner, warps 2..9 epilogue with the same functor contract as gemm_tc.cuh (the
// m_tile it sees is the 128-row tile index 2 * pair_tile + rank). The leader's `tempty` barriers
// count the epilogue warps of both CTAs. Every wait is bounded; both CTAs always reach the same
// cluster barriers.
#pragma once

#include "gemm_tc.cuh"

namespace noise {

template <int kStages, int kAccs>
struct Gemm2Layout {
  static constexpr int BM = 128;   // rows per CTA (a pair covers 256)
  static constexpr int BN = 256;   // columns per pair tile
  static constexpr int BNH = 128;  // rows of B held by each CTA
  static constexpr int BK = 64;
  static constexpr int kEpiWarps = 8;
  static constexpr int kThreads = (2 + kEpiWarps) * 32;
  static constexpr int kABytes = BM * BK * 2;
  static constexpr int kBBytes = BNH * BK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kBarrierBytes = 256;
  static constexpr int kCoreBytes = kStages * kStageBytes + kBarrierBytes;
  static constexpr uint32_t kTmemCols = kAccs * BN;
};

template <class Epi, int kStages, int kAccs>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(Gemm2Layout<kStages, kAccs>::kThreads, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const GemmShape shape, const __grid_constant__ typename Epi::Params ep) {
  using L = Gemm2Layout<kStages, kAccs>;
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
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int cluster = blockIdx.x >> 1, clusters = gridDim.x >> 1;
  int* status = shape.status;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 2 * L::kEpiWarps);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
    prefetch_tensormap(&tmA);
    prefetch_tensormap(&tmB);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, L::kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers and TMEM exist before any cross-CTA traffic
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // The pair MMA writes the same TMEM columns in both SMs: refuse to run if the CTAs disagree.
  const bool paired = ld_cluster_u32(cluster_addr(tmem_slot, rank ^ 1u)) == tmem_base;
  if (!paired && threadIdx.x == 0) atomicExch(status, kStatusUnsupported);
  const int units = paired ? TileUnit<Epi::kInterleaveN>::count(shape) : 0;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer (both CTAs) ----------------
      uint32_t stage = 0, phase = 0;
      uint32_t issued_phase[kStages];
      bool issued[kStages];
      for (int s = 0; s < kStages; ++s) issued[s] = false, issued_phase[s] = 0;
      const uint64_t keep = l2_policy_evict_last();  // weights: every pair re-reads them
      const uint32_t full0 = cluster_addr(&full[0], 0);  // the leader's barriers count both CTAs' bytes
      bool ok = true;
      for (int u = cluster; ok && u < units; u += clusters) {
        const TileUnit<Epi::kInterleaveN> tu(u, shape);
        const int arow = tu.m * 2 * L::BM + (int)rank * L::BM;
        for (int n = tu.n_begin; ok && n < tu.n_end; ++n) {
          const int brow = n * L::BN + (int)rank * L::BNH;
          for (int kb = 0; kb < shape.k_blocks; ++kb) {
            if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, status)) {
              ok = false;
              break;
            }
            if (leader) mbar_arrive_expect_tx(&full[stage], 2 * L::kStageBytes);
            tma_load_2d_pair(sA + stage * L::kABytes, &tmA, full0 + 8 * stage, kb * L::BK, arow);
            tma_load_2d_pair(sB + stage * L::kBBytes, &tmB, full0 + 8 * stage, kb * L::BK, brow, keep);
            issued[stage] = true;
            issued_phase[stage] = phase;
            if (++stage == kStages) stage = 0, phase ^= 1;
          }
        }
      }
      // This CTA's copies have landed once the MMAs that read them completed.
      for (int s = 0; s < kStages; ++s)
        if (issued[s]) mbar_wait(&empty[s], issued_phase[s], abort_flag, status);
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ---------------- MMA issuer (leader) ----------------
      const uint32_t idesc = make_idesc(1, 2 * L::BM, L::BN);
      uint32_t stage = 0, phase = 0, t = 0;
      bool ok = true;
      for (int u = cluster; ok && u < units; u += clusters) {
        const TileUnit<Epi::kInterleaveN> tu(u, shape);
        for (int n = tu.n_begin; ok && n < tu.n_end; ++n, ++t) {
          const uint32_t acc = t % kAccs, acc_phase = (t / kAccs) & 1;
          if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag, status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem_base + acc * L::BN;
          for (int kb = 0; kb < shape.k_blocks; ++kb) {
            if (!mbar_wait(&full[stage], phase, abort_flag, status)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint64_t da = smem_desc_sw128(sA + stage * L::kABytes);
            const uint64_t db = smem_desc_sw128(sB + stage * L::kBBytes);
#pragma unroll
            for (int k = 0; k < L::BK / 16; ++k)
              tc_mma_f16_pair(d, da + 2 * k, db + 2 * k, idesc, (kb | k) != 0 ? 1u : 0u);
            tc_commit_pair(&empty[stage], 0x3);
            if (++stage == kStages) stage = 0, phase ^= 1;
          }
          if (ok) tc_commit_pair(&tfull[acc], 0x3);
        }
      }
      // No MMA may still be writing TMEM (or arriving on the peer's barriers) past this point.
      tc_commit_pair(drain, 0x1);
      mbar_wait(drain, 0, abort_flag, status);
    }
    __syncwarp();
  } else {
    // ---------------- epilogue (both CTAs) ----------------
    const int ew = warp - 2;
    const int quarter = warp & 3;
    const int half = ew >> 2;
    const uint32_t tempty0 = cluster_addr(&tempty[0], 0);
    Epi epi(ep, epi_smem, ew, lane);
    uint32_t t = 0;
    bool ok = true;
    for (int u = cluster; ok && u < units; u += clusters) {
      const TileUnit<Epi::kInterleaveN> tu(u, shape);
      const int m = 2 * tu.m + (int)rank;  // this CTA's 128-row tile
      const int row = m * L::BM + quarter * 32 + lane;
      if constexpr (HasNextUnit<Epi>::value) {
        const int un = u + clusters;
        if (un < units) {
          const TileUnit<Epi::kInterleaveN> tn(un, shape);
          epi.next_unit(2 * tn.m + (int)rank, tn.n_begin);
        } else {
          epi.next_unit(-1, 0);
        }
      }
      epi.begin_mtile(m, row);
      for (int n = tu.n_begin; n < tu.n_end; ++n, ++t) {
        const uint32_t acc = t % kAccs, acc_phase = (t / kAccs) & 1;
        if (!mbar_wait(&tfull[acc], acc_phase, abort_flag, status)) {
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
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(tempty0 + 8 * acc);
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
  cluster_sync();  // the peer's remote arrivals and the leader's commits are done
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, L::kTmemCols);
  }
}

template <class Epi, int kStages, int kAccs>
int launch_gemm_tc2(const void* A, const void* B, int M, int N, int K, int lda, int ldb,
                    const typename Epi::Params& ep, int* status, cudaStream_t stream, int kind = kKindOther) {
  using L = Gemm2Layout<kStages, kAccs>;
  if (M <= 0 || N <= 0 || K <= 0 || M % (2 * L::BM) || N % L::BN || K % L::BK) return kStatusBadArgument;
  if ((reinterpret_cast<uintptr_t>(A) & 15) || (reinterpret_cast<uintptr_t>(B) & 15)) return kStatusBadArgument;
  if ((lda * 2) % 16 || (ldb * 2) % 16 || lda < K || ldb < K) return kStatusBadArgument;
  CUtensorMap ta, tb;
  if (make_tmap_2d(&ta, A, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, M, K, lda, L::BM, L::BK)) return kStatusBadArgument;
  if (make_tmap_2d(&tb, B, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, N, K, ldb, L::BNH, L::BK)) return kStatusBadArgument;
  GemmShape shape{M, N, K, M / (2 * L::BM), N / L::BN, K / L::BK, status};
  const int smem = 1024 + L::kCoreBytes + Epi::kSmemBytes;
  static bool configured = false;
  if (!configured) {
    if (cudaFuncSetAttribute(gemm_tc2_kernel<Epi, kStages, kAccs>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             smem) != cudaSuccess)
      return kStatusLaunchFailed;
    configured = true;
  }
  int clusters = device_sm_count() / 2;
  const int units = Epi::kInterleaveN ? shape.m_tiles * shape.n_tiles : shape.m_tiles;
  if (clusters > units) clusters = units;
  LaunchScope scope(kind, stream);
  gemm_tc2_kernel<Epi, kStages, kAccs><<<2 * clusters, L::kThreads, smem, stream>>>(ta, tb, shape, ep);
  return cudaGetLastError() == cudaSuccess ? kStatusOk : kStatusLaunchFailed;
}

constexpr int kPairStages = 4;
constexpr int kPairAccs = 2;

template <class E, class = void>
struct PrefersPair : std::false_type {};
template <class E>
struct PrefersPair<E, std::void_t<decltype(E::kPair)>> : std::integral_constant<bool, E::kPair> {};

// Epilogues that set kPair (long-K GEMMs, whose MMAs are fed from L2) run on CTA pairs; the others,
// bound by their epilogue rather than by the operand feed, keep the single-SM engine.
template <class Epi, int kSingleStages>
int launch_gemm(const void* A, const void* B, int M, int N, int K, int lda, int ldb, const typename Epi::Params& ep,
                int* status, cudaStream_t stream, int kind) {
  // only bf16 epilogues that ask for it instantiate the pair engine (it has no tf32 operand mode)
  if constexpr (PrefersPair<Epi>::value && !OperandTf32<Epi>::value) {
    if (M % 256 == 0)
      return launch_gemm_tc2<Epi, kPairStages, kPairAccs>(A, B, M, N, K, lda, ldb, ep, status, stream, kind);
  }
  return launch_gemm_tc<Epi, kSingleStages>(A, B, M, N, K, lda, ldb, ep, status, stream, kind);
}

}  // namespace noise
