// noise_fitness_static: the fitness-shaping entry point for callers that cannot allocate device
// memory — for example a host-language binding (a Go, Java or Node FFI shim) that has no device
// allocator of its own, or a serving process whose device memory is entirely reserved by another
// allocator's pool, so that neither can hand noise_fitness its scratch buffer.
//
// It runs the same kernels as noise_fitness (fitness.cu), with the scratch (exact ranks and
// per-pair differences) taken from a file-scope __device__ array instead of a caller's buffer:
//   - capacity: kStaticMaxMembers = 262,144 members (131,072 antithetic pairs, the reference's
//     PAIRS), 2 MiB + 256 B of device memory that every GPU loading the library keeps until exit;
//     larger populations are rejected with NOISE_SCRATCH_LIMIT before anything is launched;
//   - set-up: the first call on a device, with that device current, looks up the array's device
//     address with cudaGetSymbolAddress (the host-side name of a __device__ array is only a host
//     stand-in, never a device address); make that first call before any stream capture;
//   - sharing: all calls on a device use the same array and it keeps the last call's contents.
//     No entry has to start at zero — each call writes every rank and difference it later reads —
//     but calls that overlap on the GPU (other streams, other threads) race on the array: serialise
//     them on one stream.
// Nothing here calls cudaMalloc, cudaFree or any allocating library routine.
#include <mutex>

#include "noise_b200.h"
#include "profile.cuh"
#include "ptx.cuh"

namespace noise {

// kernels of fitness.cu
__global__ void rank_kernel(const float* __restrict__ losses, int n, int32_t* __restrict__ ranks);
__global__ void pair_diff_kernel(const float* __restrict__ losses, const int32_t* __restrict__ ranks, int n, int mode,
                                 double* __restrict__ f);
__global__ void fold_kernel(const double* __restrict__ f, int nf, int pairs, int mode, float* __restrict__ weights);

constexpr int kStaticMaxMembers = 262144;
constexpr size_t kStaticRankBytes = (size_t)kStaticMaxMembers * sizeof(int32_t);  // 256-byte multiple
constexpr size_t kStaticScratchBytes = kStaticRankBytes + ((size_t)kStaticMaxMembers / 2 + 1) * sizeof(double);

static __device__ __align__(256) uint8_t g_fitness_scratch[(kStaticScratchBytes + 255) / 256 * 256];

constexpr int kMaxDevices = 64;
static std::mutex g_static_mu;
static void* g_static_addr[kMaxDevices];

// Device address of g_fitness_scratch on the current device (looked up once per device).
static int static_scratch(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return kStatusLaunchFailed;
  std::lock_guard<std::mutex> lk(g_static_mu);
  if (!g_static_addr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_fitness_scratch) != cudaSuccess || p == nullptr) return kStatusLaunchFailed;
    g_static_addr[dev] = p;
  }
  *out = g_static_addr[dev];
  return kStatusOk;
}

}  // namespace noise

using namespace noise;

extern "C" int noise_fitness_static_max_members(void) { return kStaticMaxMembers; }

extern "C" int noise_fitness_static(const float* losses, int members, int pairs, int mode, float* weights,
                                    int32_t* ranks, void* stream) {
  if (!losses || !weights || members < 2 || (members & 1) || pairs <= 0 || (mode != 0 && mode != 1))
    return kStatusBadArgument;
  if (members > kStaticMaxMembers) return NOISE_SCRATCH_LIMIT;
  void* scratch = nullptr;
  if (int rc = static_scratch(&scratch)) return rc;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int32_t* rk = reinterpret_cast<int32_t*>(scratch);
  double* f = reinterpret_cast<double*>(reinterpret_cast<uint8_t*>(scratch) + kStaticRankBytes);
  const int blocks = (members + 255) / 256;
  LaunchScope scope(kKindFitness, s, (mode == 1 || ranks) ? 3 : 2);
  if (mode == 1 || ranks) rank_kernel<<<blocks, 256, 0, s>>>(losses, members, rk);
  pair_diff_kernel<<<blocks, 256, 0, s>>>(losses, rk, members, mode, f);
  fold_kernel<<<1, 1024, 0, s>>>(f, members / 2, pairs, mode, weights);
  if (ranks) cudaMemcpyAsync(ranks, rk, (size_t)members * sizeof(int32_t), cudaMemcpyDeviceToDevice, s);
  return cudaGetLastError() == cudaSuccess ? kStatusOk : kStatusLaunchFailed;
}
