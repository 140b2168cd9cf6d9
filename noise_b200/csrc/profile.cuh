// Launch accounting shared by every launcher (see host_util.cu).
#pragma once

#include <cuda_runtime.h>

namespace noise {

// Kernel kinds reported by noise_profile_read (index = kind).
enum LaunchKind : int {
  kKindEmbed = 0,
  kKindQkv = 1,
  kKindAttention = 2,
  kKindProj = 3,
  kKindFc = 4,
  kKindMlp = 5,
  kKindHead = 6,
  kKindLoss = 7,
  kKindFitness = 8,
  kKindUpdate = 9,
  kKindPack = 10,
  kKindOther = 11,
  kNumKinds = 12,
};

// One scope brackets the launches of one library call; `kernels` is how many kernels it launches
// (the count noise_launch_count reports), the timing covers them together.
class LaunchScope {
 public:
  LaunchScope(int kind, cudaStream_t s, int kernels = 1);
  ~LaunchScope();

 private:
  int kind_;
  cudaStream_t s_;
  int idx_;
};

}  // namespace noise
