// Plain GEMM through the tcgen05 engine: C = alpha * A * B^T, stored as fp32 or bf16. It has no
// counterpart on the reference's path; it exists so the engine itself can be checked in isolation
// (tests/test_gemm_gpu.py) before the fused epilogues are layered on it.
#include "gemm_tc2.cuh"
#include "noise_b200.h"

namespace noise {

struct EpiStore {
  struct Params {
    void* C;
    int ldc;
    float alpha;
    int out_bf16;
  };
  static constexpr int kSmemBytes = 0;
  static constexpr bool kInterleaveN = false;
  static constexpr bool kPair = true;
  const Params& p;
  __device__ EpiStore(const Params& p_, uint8_t*, int, int) : p(p_) {}
  __device__ void begin_mtile(int, int) {}
  __device__ void begin_tile(int, int, int) {}
  __device__ void end_mtile(int, int, int) {}
  __device__ void group(int row, int col, float (&v)[64]) {
    if (p.out_bf16) {
      __nv_bfloat16* c = reinterpret_cast<__nv_bfloat16*>(p.C) + (size_t)row * p.ldc + col;
#pragma unroll
      for (int j = 0; j < 64; j += 8)
        st_global_v4(c + j, pack_bf16x2(p.alpha * v[j], p.alpha * v[j + 1]),
                     pack_bf16x2(p.alpha * v[j + 2], p.alpha * v[j + 3]),
                     pack_bf16x2(p.alpha * v[j + 4], p.alpha * v[j + 5]),
                     pack_bf16x2(p.alpha * v[j + 6], p.alpha * v[j + 7]));
    } else {
      float* c = reinterpret_cast<float*>(p.C) + (size_t)row * p.ldc + col;
#pragma unroll
      for (int j = 0; j < 64; j += 4)
        st_global_v4f(c + j, p.alpha * v[j], p.alpha * v[j + 1], p.alpha * v[j + 2], p.alpha * v[j + 3]);
    }
  }
};

// The engine's failure path, exercised without a fault: the producer arms the operand barrier but
// issues no copy, so the MMA warp's wait for the first stage runs out after kWaitBudget cycles
// (about 10 ms), sets the abort flag and the status word, and every role leaves its loop, drains and
// frees tensor memory. Nothing is stored.
struct EpiWaitTimeout {
  struct Params {};
  static constexpr int kSmemBytes = 0;
  static constexpr bool kInterleaveN = false;
  static constexpr bool kSkipLoads = true;
  static constexpr long long kWaitBudget = 20ll * 1000 * 1000;
  __device__ EpiWaitTimeout(const Params&, uint8_t*, int, int) {}
  __device__ void begin_mtile(int, int) {}
  __device__ void begin_tile(int, int, int) {}
  __device__ void end_mtile(int, int, int) {}
  __device__ void group(int, int, float (&)[64]) {}
};

}  // namespace noise

extern "C" int noise_selftest_wait_timeout(const void* A, const void* B, int* status, void* stream) {
  if (!A || !B || !status) return noise::kStatusBadArgument;
  noise::EpiWaitTimeout::Params ep{};
  return noise::launch_gemm_tc<noise::EpiWaitTimeout, 3>(A, B, 128, 256, 64, 64, 64, ep, status,
                                                          reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int noise_gemm_bf16(const void* A, const void* B, void* C, int M, int N, int K, float alpha,
                               int out_bf16, int* status, void* stream) {
  noise::EpiStore::Params ep{C, N, alpha, out_bf16};
  return noise::launch_gemm<noise::EpiStore, 4>(A, B, M, N, K, K, K, ep, status,
                                                   reinterpret_cast<cudaStream_t>(stream), noise::kKindOther);
}
