// ANVIL II's `polar` (train/val/run.py:572-580) on the block matrices of a region, on the tcgen05
// engine: every matrix in its wide form X [R, C] (R <= C: the matrix itself, or the transpose of a
// tall c_fc), normalised and cast to bf16 by noise_anvil_region_prepare, goes through six quintic
// maps
//     S = X X^T,   X <- a X + (b S + c S S) X
// in bf16 storage with fp32 accumulation. Matrices of one wide shape are stacked and each map is
// three batched (block-diagonal) GEMMs whose operands are all K-major:
//     G1  S   = X X^T                     A = X,   B = X     (K = C)
//     G2  Bm  = b S + c S S               A = S,   B = S     (K = R; S is symmetric, so B = S^T = S)
//     G3  X'^T = a X^T + X^T Bm           A = X^T, B = Bm    (K = R; Bm is symmetric: X^T Bm = (Bm X)^T)
// G3's epilogue writes X'^T and, transposed, X' (a warp's 32 rows are 32 consecutive columns of
// X', so each of its stores is 64 contiguous bytes), which the next map's G1 reads. X and X^T
// ping-pong between two buffers so no GEMM reads what its own epilogue writes.
#include "gemm_tc2.cuh"
#include "model_layout.cuh"
#include "noise_b200.h"

namespace noise {

constexpr int kPolarR = 512;          // the short side of every block matrix
constexpr int kPolarMaxMatrices = 48;

struct EpiGram {
  struct Params {
    __nv_bfloat16* S;  // [n * R, R]
    int R;
  };
  static constexpr int kSmemBytes = 0;
  static constexpr bool kInterleaveN = false;
  const Params& p;
  __device__ EpiGram(const Params& p_, uint8_t*, int, int) : p(p_) {}
  __device__ void begin_mtile(int, int) {}
  __device__ void begin_tile(int, int, int) {}
  __device__ void end_mtile(int, int, int) {}
  __device__ void group(int row, int col, float (&v)[64]) {
    const int lc = col - (row / p.R) * p.R;
    st_bf16x64(p.S + (size_t)row * p.R + lc, v);
  }
};

struct EpiPoly {
  struct Params {
    const __nv_bfloat16* S;  // [n * R, R]
    __nv_bfloat16* Bm;       // [n * R, R]
    int R;
    float b, c;
  };
  static constexpr int kSmemBytes = 0;
  static constexpr bool kInterleaveN = false;
  const Params& p;
  __device__ EpiPoly(const Params& p_, uint8_t*, int, int) : p(p_) {}
  __device__ void begin_mtile(int, int) {}
  __device__ void begin_tile(int, int, int) {}
  __device__ void end_mtile(int, int, int) {}
  __device__ void group(int row, int col, float (&v)[64]) {
    const size_t at = (size_t)row * p.R + (col - (row / p.R) * p.R);
    const uint4* s = reinterpret_cast<const uint4*>(p.S + at);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const uint4 u = s[q];
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
        v[8 * q + 2 * i] = p.b * f.x + p.c * v[8 * q + 2 * i];
        v[8 * q + 2 * i + 1] = p.b * f.y + p.c * v[8 * q + 2 * i + 1];
      }
    }
    st_bf16x64(p.Bm + at, v);
  }
};

struct EpiApply {
  struct Params {
    const __nv_bfloat16* XT;  // [n * C, R] this map's X^T
    __nv_bfloat16* XT_out;    // [n * C, R]
    __nv_bfloat16* X_out;     // [n * R, C]
    int R, C;
    float a;
  };
  static constexpr int kSmemBytes = 0;
  static constexpr bool kInterleaveN = false;
  const Params& p;
  __device__ EpiApply(const Params& p_, uint8_t*, int, int) : p(p_) {}
  __device__ void begin_mtile(int, int) {}
  __device__ void begin_tile(int, int, int) {}
  __device__ void end_mtile(int, int, int) {}
  __device__ void group(int row, int col, float (&v)[64]) {
    const int b = row / p.C, n = row - b * p.C;
    const int m0 = col - b * p.R;
    const size_t at = (size_t)row * p.R + m0;
    const uint4* x = reinterpret_cast<const uint4*>(p.XT + at);
    uint32_t w[32];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const uint4 u = x[q];
      const uint32_t in[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&in[i]));
        w[4 * q + i] = pack_bf16x2(p.a * f.x + v[8 * q + 2 * i], p.a * f.y + v[8 * q + 2 * i + 1]);
      }
    }
#pragma unroll
    for (int q = 0; q < 8; ++q)
      reinterpret_cast<uint4*>(p.XT_out + at)[q] = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
    __nv_bfloat16* xo = p.X_out + ((size_t)b * p.R + m0) * p.C + n;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162*>(&w[j]);
      xo[(size_t)(2 * j) * p.C] = h.x;
      xo[(size_t)(2 * j + 1) * p.C] = h.y;
    }
  }
};

// One block matrix of a polar group: where it sits in the region buffer, its natural shape, and its
// slot in the stacked wide-form buffers.
struct PolarItem {
  int64_t src;  // element offset in the region buffer
  int rows, cols;
};

struct PolarCopy {
  PolarItem item[kPolarMaxMatrices];
  int count;
  int R, C;               // wide form
  __nv_bfloat16* X;       // [count * R, C]
  __nv_bfloat16* XT;      // [count * C, R]
  __nv_bfloat16* region;  // the region's bf16 buffer
};

// blockIdx.z = matrix; 32 x 32 tiles of the matrix's natural [rows, cols]. gather (to_region = 0):
// natural -> the stacked buffer of the same orientation (X for a wide matrix, X^T for a tall one)
// and its transpose into the other; scatter (to_region = 1): the same-orientation buffer -> natural.
__global__ void __launch_bounds__(256) polar_copy_kernel(const __grid_constant__ PolarCopy p, int to_region) {
  __shared__ __nv_bfloat16 tile[32][34];
  const PolarItem it = p.item[blockIdx.z];
  const int r0 = blockIdx.y * 32, c0 = blockIdx.x * 32;
  if (r0 >= it.rows || c0 >= it.cols) return;
  const bool wide = it.rows <= it.cols;
  __nv_bfloat16* same = wide ? p.X + (size_t)blockIdx.z * p.R * p.C : p.XT + (size_t)blockIdx.z * p.C * p.R;
  __nv_bfloat16* other = wide ? p.XT + (size_t)blockIdx.z * p.C * p.R : p.X + (size_t)blockIdx.z * p.R * p.C;
  __nv_bfloat16* nat = p.region + it.src;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  for (int r = ty; r < 32; r += 8) {
    const size_t at = (size_t)(r0 + r) * it.cols + c0 + tx;
    if (to_region) {
      nat[at] = same[at];
    } else {
      const __nv_bfloat16 v = nat[at];
      same[at] = v;
      tile[r][tx] = v;
    }
  }
  if (to_region) return;
  __syncthreads();
  for (int r = ty; r < 32; r += 8) other[(size_t)(c0 + r) * it.rows + r0 + tx] = tile[tx][r];
}

struct PolarGroups {
  PolarCopy g[2];  // [0] 512 x 512, [1] 512 x 2048 (wide form)
  size_t bytes;
};

bool is_block_matrix(int tid) {
  for (int l = 0; l < kLayers; ++l)
    if ((uint32_t)tid == tid_q(l) || (uint32_t)tid == tid_k(l) || (uint32_t)tid == tid_v(l) ||
        (uint32_t)tid == tid_proj(l) || (uint32_t)tid == tid_fc(l) || (uint32_t)tid == tid_mlp(l))
      return true;
  return false;
}

static size_t polar_group_bytes(int n, int R, int C) {
  return (size_t)n * (4 * (size_t)R * C + 2 * (size_t)R * R) * 2;
}

// The region's matrices by wide shape, and (with ws) the stacked buffers carved from the workspace.
PolarGroups polar_groups(const NoiseRegion& region, void* x, void* ws) {
  static const ParamLayout L = make_param_layout();
  PolarGroups G{};
  G.g[0].R = kPolarR, G.g[0].C = kPolarR;
  G.g[1].R = kPolarR, G.g[1].C = 4 * kPolarR;
  for (int tid = region.tensor_begin; tid < region.tensor_end; ++tid) {
    if (!is_block_matrix(tid)) continue;
    const int big = L.rows[tid] > L.cols[tid] ? L.rows[tid] : L.cols[tid];
    PolarCopy& c = G.g[big == kPolarR ? 0 : 1];
    c.item[c.count++] = PolarItem{L.offset[tid] - region.base, L.rows[tid], L.cols[tid]};
  }
  size_t off = 0;
  for (PolarCopy& c : G.g) {
    c.region = reinterpret_cast<__nv_bfloat16*>(x);
    // X[0], X[1], XT[0], XT[1], S, Bm follow; a size query (no workspace) carves nothing
    c.X = ws ? reinterpret_cast<__nv_bfloat16*>(reinterpret_cast<uint8_t*>(ws) + off) : nullptr;
    off += polar_group_bytes(c.count, c.R, c.C);
  }
  G.bytes = off;
  return G;
}

}  // namespace noise

using namespace noise;

extern "C" int64_t noise_anvil_polar_workspace_bytes(const NoiseRegion* region) {
  if (!region || region->tensor_begin < 0 || region->tensor_end > kNumTensors) return -1;
  return (int64_t)polar_groups(*region, nullptr, nullptr).bytes;
}

extern "C" int noise_anvil_region_polar(const NoiseRegion* region, void* x, const float* maps, int nmaps,
                                        void* workspace, size_t workspace_bytes, int* status, void* stream) {
  if (!region || !x || !maps || nmaps <= 0 || region->tensor_begin < 0 || region->tensor_end > kNumTensors ||
      region->tensor_begin > region->tensor_end)
    return kStatusBadArgument;
  PolarGroups G = polar_groups(*region, x, workspace);
  if (G.bytes > 0 && (!workspace || G.bytes > workspace_bytes)) return kStatusWorkspaceTooSmall;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  for (PolarCopy& c : G.g) {
    const int n = c.count;
    if (n == 0) continue;
    const size_t xs = (size_t)n * c.R * c.C;
    __nv_bfloat16* X[2] = {c.X, c.X + xs};
    __nv_bfloat16* XT[2] = {c.X + 2 * xs, c.X + 3 * xs};
    __nv_bfloat16* S = c.X + 4 * xs;
    __nv_bfloat16* Bm = S + (size_t)n * c.R * c.R;
    const dim3 grid(c.C / 32, c.C / 32, n);  // covers either orientation; blocks outside a matrix return
    {
      PolarCopy g = c;
      g.XT = XT[0];
      LaunchScope scope(kKindUpdate, s);
      polar_copy_kernel<<<grid, 256, 0, s>>>(g, 0);
      if (cudaGetLastError() != cudaSuccess) return kStatusLaunchFailed;
    }
    int cur = 0;
    for (int k = 0; k < nmaps; ++k, cur ^= 1) {
      const float a = maps[3 * k], b = maps[3 * k + 1], cc = maps[3 * k + 2];
      int rc;
      EpiGram::Params g1{S, c.R};
      if ((rc = launch_gemm_tc<EpiGram, 3>(X[cur], X[cur], n * c.R, n * c.R, c.C, c.C, c.C, g1, status, s,
                                           kKindUpdate, 0, c.R, c.R)))
        return rc;
      EpiPoly::Params g2{S, Bm, c.R, b, cc};
      if ((rc = launch_gemm_tc<EpiPoly, 3>(S, S, n * c.R, n * c.R, c.R, c.R, c.R, g2, status, s, kKindUpdate, 0,
                                           c.R, c.R)))
        return rc;
      EpiApply::Params g3{XT[cur], XT[cur ^ 1], X[cur ^ 1], c.R, c.C, a};
      if ((rc = launch_gemm_tc<EpiApply, 3>(XT[cur], Bm, n * c.C, n * c.R, c.R, c.R, c.R, g3, status, s,
                                            kKindUpdate, 0, c.C, c.R)))
        return rc;
    }
    {
      PolarCopy g = c;
      g.X = X[cur];
      g.XT = XT[cur];
      LaunchScope scope(kKindUpdate, s);
      polar_copy_kernel<<<grid, 256, 0, s>>>(g, 1);
      if (cudaGetLastError() != cudaSuccess) return kStatusLaunchFailed;
    }
  }
  return kStatusOk;
}
