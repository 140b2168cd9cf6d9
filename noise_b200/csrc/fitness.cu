// Fitness shaping: per-member losses -> per-direction weights.
//
//   mode 0 (z-score, train/val/eggroll.py:151-154): f_i = L[2i+1] - L[2i] for the i-th antithetic
//           member pair, f /= (unbiased std(f) + 1e-8), weight[d] = sum of f_i over i = d (mod P).
//   mode 1 (centred rank): rank_j of L_j in ascending order (NaN last, ties by member index),
//           c_j = rank_j / (N - 1) - 0.5, f_i = c[2i+1] - c[2i], weight[d] as above.
//
// Ranks are integer counts of strictly smaller keys, so they are exact and independent of thread
// order. Pair differences are taken with a lane-xor-1 shuffle (members 2i and 2i+1 sit in adjacent
// lanes); reductions use warp shuffles and fp64 accumulation.
#include "noise_b200.h"
#include "profile.cuh"
#include "ptx.cuh"

namespace noise {

// Total order on losses: NaN after every number, -0 == +0, then member index.
__device__ __forceinline__ uint32_t order_key(float x) {
  if (x != x) return 0xFFFFFFFFu;
  if (x == 0.0f) x = 0.0f;
  const uint32_t u = __float_as_uint(x);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

constexpr int kRankTile = 2048;

__global__ void __launch_bounds__(256) rank_kernel(const float* __restrict__ losses, int n, int32_t* __restrict__ ranks) {
  __shared__ uint32_t keys[kRankTile];
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  const uint32_t kj = j < n ? order_key(losses[j]) : 0xFFFFFFFFu;
  int count = 0;
  for (int t0 = 0; t0 < n; t0 += kRankTile) {
    __syncthreads();
    for (int k = threadIdx.x; k < kRankTile; k += blockDim.x) keys[k] = t0 + k < n ? order_key(losses[t0 + k]) : 0xFFFFFFFFu;
    __syncthreads();
    const int lim = min(kRankTile, n - t0);
    for (int k = 0; k < lim; ++k) {
      const uint32_t kk = keys[k];
      count += (kk < kj) || (kk == kj && t0 + k < j);
    }
  }
  if (j < n) ranks[j] = count;
}

// pair differences f_i (fp64 in scratch): mode 0 from losses, mode 1 from centred ranks
__global__ void pair_diff_kernel(const float* __restrict__ losses, const int32_t* __restrict__ ranks, int n, int mode,
                                 double* __restrict__ f) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x;  // member; n is even so pairs never straddle warps
  double v = 0.0;
  if (j < n) v = mode == 0 ? (double)losses[j] : (double)ranks[j] / (double)(n > 1 ? n - 1 : 1) - 0.5;
  const double partner = __shfl_xor_sync(0xffffffffu, v, 1);
  if (j < n && (j & 1)) f[j >> 1] = v - partner;
}

__device__ __forceinline__ double block_sum(double v, double* red) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  double s = 0.0;
  if (threadIdx.x < 32) {
    s = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0;
#pragma unroll
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (threadIdx.x == 0) red[32] = s;
  }
  __syncthreads();
  return red[32];
}

// one CTA: z-score (mode 0) then fold onto directions
__global__ void __launch_bounds__(1024) fold_kernel(const double* __restrict__ f, int nf, int pairs, int mode,
                                                    float* __restrict__ weights) {
  __shared__ double red[33];
  double scale = 1.0;
  if (mode == 0) {
    double s = 0.0;
    for (int i = threadIdx.x; i < nf; i += blockDim.x) s += f[i];
    const double mean = block_sum(s, red) / nf;
    double q = 0.0;
    for (int i = threadIdx.x; i < nf; i += blockDim.x) q += (f[i] - mean) * (f[i] - mean);
    const double var = block_sum(q, red) / (nf > 1 ? nf - 1 : 1);
    scale = 1.0 / (sqrt(var) + 1e-8);
  }
  for (int d = threadIdx.x; d < pairs; d += blockDim.x) {
    double w = 0.0;
    for (int i = d; i < nf; i += pairs) w += f[i] * scale;
    weights[d] = (float)w;
  }
}

}  // namespace noise

using namespace noise;

extern "C" size_t noise_fitness_workspace_bytes(int members) {
  return ((size_t)members * sizeof(int32_t) + 255) / 256 * 256 + (size_t)(members / 2 + 1) * sizeof(double);
}

extern "C" int noise_fitness(const float* losses, int members, int pairs, int mode, float* weights, int32_t* ranks,
                             void* workspace, size_t workspace_bytes, void* stream) {
  if (!losses || !weights || !workspace || members < 2 || (members & 1) || pairs <= 0 || (mode != 0 && mode != 1))
    return kStatusBadArgument;
  if (workspace_bytes < noise_fitness_workspace_bytes(members)) return kStatusWorkspaceTooSmall;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int32_t* rk = reinterpret_cast<int32_t*>(workspace);
  double* f = reinterpret_cast<double*>(reinterpret_cast<uint8_t*>(workspace) +
                                        ((size_t)members * sizeof(int32_t) + 255) / 256 * 256);
  const int blocks = (members + 255) / 256;
  LaunchScope scope(kKindFitness, s, (mode == 1 || ranks) ? 3 : 2);
  if (mode == 1 || ranks) rank_kernel<<<blocks, 256, 0, s>>>(losses, members, rk);
  pair_diff_kernel<<<blocks, 256, 0, s>>>(losses, rk, members, mode, f);
  fold_kernel<<<1, 1024, 0, s>>>(f, members / 2, pairs, mode, weights);
  if (ranks) cudaMemcpyAsync(ranks, rk, (size_t)members * sizeof(int32_t), cudaMemcpyDeviceToDevice, s);
  return cudaGetLastError() == cudaSuccess ? kStatusOk : kStatusLaunchFailed;
}
