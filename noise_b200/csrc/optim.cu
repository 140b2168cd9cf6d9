// Optimizer kernels for dense gradients (the DUST estimator's reassembled gradients):
//
// Each runs on a region of the flat layout (NoiseRegion: tensors [tensor_begin, tensor_end), their
// optimizer buffers holding flat indices from `base` on), the whole buffer being one region; the
// sharded update gives each rank the region of whole tensors it owns.
//
// noise_adamw_dense: torch.optim.AdamW over a subset of the flat parameter buffer, with one lr
//   multiplier per tensor (train/val/run.py:643-656: embeddings x300, mixing scalars x30, the rest
//   x1; block matrices excluded when they go to ANVIL).
// noise_anvil_prepare / noise_anvil_finish: the elementwise and reduction passes of ANVIL II
//   (train/val/run.py:583-626) batched over every block matrix; the six quintic maps of `polar`
//   (:572-580) run between them as bf16 GEMMs (cuBLAS through the host).
//   prepare: fast/slow EMAs, m = g.lerp(blend, beta), x = bf16(m / (1.05 |m| + 1e-6))
//   finish:  lane energy EMA of the polar update u, gained = u / sqrt(energy),
//            u' = gained |u| / |gained|, p -= lr sqrt(max(1, rows/cols)) (u' + (slow w >= 0) w wd lr)
// Reductions are per block into fixed slots and summed in a fixed order, so results do not depend
// on scheduling.
#include "model_layout.cuh"
#include "noise_b200.h"
#include "profile.cuh"
#include "ptx.cuh"

namespace noise {

constexpr int kOptBlock = 256, kOptPerThread = 8, kOptTile = kOptBlock * kOptPerThread;
constexpr int kMaxMatrices = 64;

// torch's lerp: self + w (end - self) for w < 0.5, else end - (end - self) (1 - w)
__device__ __forceinline__ float torch_lerp(float self, float end, float w) {
  return w < 0.5f ? self + w * (end - self) : end - (end - self) * (1.0f - w);
}

struct TensorSpan {
  int64_t offset, n;
  int tile_begin;
};

// ---------------------------------------------------------------------------------------------
// AdamW on dense gradients
// ---------------------------------------------------------------------------------------------
struct AdamDenseParams {
  TensorSpan t[kNumTensors];
  int count;
  int tensor_id[kNumTensors];
  int64_t packed[kNumTensors];
  float* params;
  __nv_bfloat16* packed_w;
  float* m;           // m, v, grad: element i holds flat index base + i (a region of the flat layout)
  float* v;
  const float* grad;
  int64_t base;
  float lr[kNumTensors];
  float beta1, beta2, eps, wd, bc1, bc2_sqrt;
};

__global__ void __launch_bounds__(kOptBlock) adamw_dense_kernel(const __grid_constant__ AdamDenseParams p) {
  int k = 0;
  while (k + 1 < p.count && (int)blockIdx.x >= p.t[k + 1].tile_begin) ++k;
  const TensorSpan s = p.t[k];
  const int64_t base = (int64_t)(blockIdx.x - s.tile_begin) * kOptTile;
  const float lr = p.lr[k], step = lr / p.bc1;
  for (int u = 0; u < kOptPerThread; ++u) {
    const int64_t i = base + u * kOptBlock + threadIdx.x;
    if (i >= s.n) break;
    const int64_t idx = s.offset + i, r = idx - p.base;
    const float g = p.grad[r];
    float w = p.params[idx];
    if (p.wd != 0.f) w *= 1.0f - lr * p.wd;
    const float m = torch_lerp(p.m[r], g, 1.0f - p.beta1);
    const float v = p.v[r] * p.beta2 + (1.0f - p.beta2) * g * g;
    w -= step * (m / (sqrtf(v) / p.bc2_sqrt + p.eps));
    p.params[idx] = w;
    p.m[r] = m;
    p.v[r] = v;
    if (p.packed[k] >= 0 && p.packed_w) p.packed_w[p.packed[k] + i] = __float2bfloat16_rn(w);
  }
}

// ---------------------------------------------------------------------------------------------
// ANVIL II
// ---------------------------------------------------------------------------------------------
struct AnvilMatrix {
  int64_t offset;       // in the flat buffers (params, grad, fast, slow, scratch)
  int64_t packed;       // packed bf16 offset or -1
  int rows, cols;
  int tile_begin;       // first elementwise tile
  int lane_begin;       // first lane (row if rows >= cols, else column) in the energy buffer
};

struct AnvilParams {
  AnvilMatrix m[kMaxMatrices];
  int count, tiles, lanes;
  float* params;
  __nv_bfloat16* packed_w;
  // grad, fast, slow, mbuf and x: element i holds flat index base + i (a region of the flat layout)
  int64_t base;
  const float* grad;
  float* fast;
  float* slow;
  float* mbuf;                 // scratch: m (prepare), then reused
  __nv_bfloat16* x;            // bf16 polar input / output
  float* energy;               // [lanes]
  float* partial;              // [tiles] per-tile partial sums
  float* partial2;             // [tiles]
  float* scale;                // [count] per-matrix scalars
  float fast_beta, slow_beta, beta, weight, lane_beta, lr, wd;
};

__device__ __forceinline__ int anvil_matrix_of(const AnvilParams& p, int tile) {
  int k = 0;
  while (k + 1 < p.count && tile >= p.m[k + 1].tile_begin) ++k;
  return k;
}

__device__ __forceinline__ float block_reduce_sum(float v) {
  __shared__ float red[kOptBlock / 32];
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float s = 0.f;
  if (threadIdx.x == 0)
    for (int w = 0; w < kOptBlock / 32; ++w) s += red[w];
  __syncthreads();
  return s;  // valid on thread 0
}

// fast/slow EMAs and the blended matrix m; per-tile sum of m^2
__global__ void __launch_bounds__(kOptBlock) anvil_blend_kernel(const __grid_constant__ AnvilParams p) {
  const int k = anvil_matrix_of(p, blockIdx.x);
  const AnvilMatrix M = p.m[k];
  const int64_t n = (int64_t)M.rows * M.cols;
  const int64_t base = (int64_t)(blockIdx.x - M.tile_begin) * kOptTile;
  float ss = 0.f;
  for (int u = 0; u < kOptPerThread; ++u) {
    const int64_t i = base + u * kOptBlock + threadIdx.x;
    if (i >= n) break;
    const int64_t idx = M.offset + i - p.base;
    const float g = p.grad[idx];
    const float f = torch_lerp(p.fast[idx], g, 1.0f - p.fast_beta);
    const float s = torch_lerp(p.slow[idx], g, 1.0f - p.slow_beta);
    p.fast[idx] = f;
    p.slow[idx] = s;
    const float blend = p.weight * f + (1.0f - p.weight) * s;
    const float m = torch_lerp(g, blend, p.beta);
    p.mbuf[idx] = m;
    ss += m * m;
  }
  const float t = block_reduce_sum(ss);
  if (threadIdx.x == 0) p.partial[blockIdx.x] = t;
}

// per-matrix scalar from the per-tile partials, in tile order: mode 0 -> 1.05 |m| + 1e-6,
// mode 1 -> |u| / max(|gained|, 1e-10) from (partial = sum u^2, partial2 = sum gained^2)
__global__ void anvil_scalar_kernel(const __grid_constant__ AnvilParams p, int mode) {
  const int k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= p.count) return;
  const int t0 = p.m[k].tile_begin, t1 = k + 1 < p.count ? p.m[k + 1].tile_begin : p.tiles;
  double a = 0.0, b = 0.0;
  for (int t = t0; t < t1; ++t) a += p.partial[t], b += mode ? p.partial2[t] : 0.0;
  if (mode == 0)
    p.scale[k] = (float)(1.05 * sqrt(a) + 1e-6);
  else
    p.scale[k] = (float)(sqrt(a) / fmax(sqrt(b), 1e-10));
}

__global__ void __launch_bounds__(kOptBlock) anvil_cast_kernel(const __grid_constant__ AnvilParams p) {
  const int k = anvil_matrix_of(p, blockIdx.x);
  const AnvilMatrix M = p.m[k];
  const int64_t n = (int64_t)M.rows * M.cols;
  const int64_t base = (int64_t)(blockIdx.x - M.tile_begin) * kOptTile;
  const float denom = p.scale[k];
  for (int u = 0; u < kOptPerThread; ++u) {
    const int64_t i = base + u * kOptBlock + threadIdx.x;
    if (i >= n) break;
    p.x[M.offset + i - p.base] = __float2bfloat16_rn(p.mbuf[M.offset + i - p.base] / denom);
  }
}

// one block per lane: energy = lerp(energy, mean(u^2 over the lane), 1 - lane_beta)
__global__ void __launch_bounds__(kOptBlock) anvil_energy_kernel(const __grid_constant__ AnvilParams p) {
  int k = 0;
  while (k + 1 < p.count && (int)blockIdx.x >= p.m[k + 1].lane_begin) ++k;
  const AnvilMatrix M = p.m[k];
  const int lane = blockIdx.x - M.lane_begin;
  const bool rows_are_lanes = M.rows >= M.cols;  // lanes = 1: mean over columns, one value per row
  const int len = rows_are_lanes ? M.cols : M.rows;
  float ss = 0.f;
  for (int j = threadIdx.x; j < len; j += blockDim.x) {
    const int64_t i = rows_are_lanes ? (int64_t)lane * M.cols + j : (int64_t)j * M.cols + lane;
    const float u = __bfloat162float(p.x[M.offset + i - p.base]);
    ss += u * u;
  }
  const float t = block_reduce_sum(ss);
  if (threadIdx.x == 0) p.energy[blockIdx.x] = torch_lerp(p.energy[blockIdx.x], t / (float)len, 1.0f - p.lane_beta);
}

// per-tile sums of u^2 and of gained^2
__global__ void __launch_bounds__(kOptBlock) anvil_norms_kernel(const __grid_constant__ AnvilParams p) {
  const int k = anvil_matrix_of(p, blockIdx.x);
  const AnvilMatrix M = p.m[k];
  const int64_t n = (int64_t)M.rows * M.cols;
  const int64_t base = (int64_t)(blockIdx.x - M.tile_begin) * kOptTile;
  const bool rows_are_lanes = M.rows >= M.cols;
  float su = 0.f, sg = 0.f;
  for (int uu = 0; uu < kOptPerThread; ++uu) {
    const int64_t i = base + uu * kOptBlock + threadIdx.x;
    if (i >= n) break;
    const float u = __bfloat162float(p.x[M.offset + i - p.base]);
    const int lane = rows_are_lanes ? (int)(i / M.cols) : (int)(i % M.cols);
    const float g = u * rsqrtf(fmaxf(p.energy[M.lane_begin + lane], 1e-10f));
    su += u * u;
    sg += g * g;
  }
  const float a = block_reduce_sum(su);
  const float b = block_reduce_sum(sg);
  if (threadIdx.x == 0) p.partial[blockIdx.x] = a, p.partial2[blockIdx.x] = b;
}

__global__ void __launch_bounds__(kOptBlock) anvil_apply_kernel(const __grid_constant__ AnvilParams p) {
  const int k = anvil_matrix_of(p, blockIdx.x);
  const AnvilMatrix M = p.m[k];
  const int64_t n = (int64_t)M.rows * M.cols;
  const int64_t base = (int64_t)(blockIdx.x - M.tile_begin) * kOptTile;
  const bool rows_are_lanes = M.rows >= M.cols;
  const float ratio = p.scale[k];
  const float lr_eff = p.lr * sqrtf(fmaxf(1.0f, (float)M.rows / (float)M.cols));
  for (int uu = 0; uu < kOptPerThread; ++uu) {
    const int64_t i = base + uu * kOptBlock + threadIdx.x;
    if (i >= n) break;
    const int64_t idx = M.offset + i, r = idx - p.base;
    const float u = __bfloat162float(p.x[r]);
    const int lane = rows_are_lanes ? (int)(i / M.cols) : (int)(i % M.cols);
    const float upd = u * rsqrtf(fmaxf(p.energy[M.lane_begin + lane], 1e-10f)) * ratio;
    const float w = p.params[idx];
    const float decay = (p.slow[r] * w >= 0.f) ? w * (p.wd * p.lr) : 0.f;
    const float nw = w - lr_eff * (upd + decay);
    p.params[idx] = nw;
    if (M.packed >= 0 && p.packed_w) p.packed_w[M.packed + i] = __float2bfloat16_rn(nw);
  }
}

int64_t packed_offset(int tid) {
  for (int l = 0; l < kLayers; ++l) {
    const int64_t b = l * kPackLayer;
    if ((uint32_t)tid == tid_q(l)) return b + kPackQkv;
    if ((uint32_t)tid == tid_k(l)) return b + kPackQkv + kWidth * kWidth;
    if ((uint32_t)tid == tid_v(l)) return b + kPackQkv + 2 * kWidth * kWidth;
    if ((uint32_t)tid == tid_proj(l)) return b + kPackProj;
    if ((uint32_t)tid == tid_fc(l)) return b + kPackFc;
    if ((uint32_t)tid == tid_mlp(l)) return b + kPackMlp;
  }
  if ((uint32_t)tid == kTidHead) return kPackHead;
  return -1;
}

bool is_anvil_matrix(int tid) {  // transformer.h.* 2-D parameters except ve_gate (run.py:647)
  for (int l = 0; l < kLayers; ++l)
    if ((uint32_t)tid == tid_q(l) || (uint32_t)tid == tid_k(l) || (uint32_t)tid == tid_v(l) ||
        (uint32_t)tid == tid_proj(l) || (uint32_t)tid == tid_fc(l) || (uint32_t)tid == tid_mlp(l))
      return true;
  return false;
}

// The block matrices of tensors [region.tensor_begin, region.tensor_end), in flat order.
AnvilParams make_anvil_params(const NoiseRegion& region, float* params, void* packed, const float* grad, float* fast,
                              float* slow, float* scratch, void* x, float* energy, float* partials, float* scalars) {
  static const ParamLayout L = make_param_layout();
  AnvilParams p{};
  p.base = region.base;
  int tiles = 0, lanes = 0;
  for (int tid = region.tensor_begin; tid < region.tensor_end; ++tid) {
    if (!is_anvil_matrix(tid)) continue;
    AnvilMatrix& M = p.m[p.count++];
    M.offset = L.offset[tid];
    M.packed = packed_offset(tid);
    M.rows = L.rows[tid];
    M.cols = L.cols[tid];
    M.tile_begin = tiles;
    M.lane_begin = lanes;
    tiles += (int)(((int64_t)M.rows * M.cols + kOptTile - 1) / kOptTile);
    lanes += M.rows >= M.cols ? M.rows : M.cols;
  }
  p.tiles = tiles;
  p.lanes = lanes;
  p.params = params;
  p.packed_w = reinterpret_cast<__nv_bfloat16*>(packed);
  p.grad = grad;
  p.fast = fast;
  p.slow = slow;
  p.mbuf = scratch;
  p.x = reinterpret_cast<__nv_bfloat16*>(x);
  p.energy = energy;
  p.partial = partials;
  p.partial2 = partials + tiles;
  p.scale = scalars;
  return p;
}

}  // namespace noise

using namespace noise;

static const NoiseRegion kAllTensors = {0, kNumTensors, 0};

static bool region_ok(const NoiseRegion* r) {
  static const ParamLayout L = make_param_layout();
  if (!r || r->tensor_begin < 0 || r->tensor_end > kNumTensors || r->tensor_begin > r->tensor_end) return false;
  return r->tensor_begin == r->tensor_end || r->base <= L.offset[r->tensor_begin];
}

extern "C" int noise_adamw_region(float* params, void* packed, float* exp_avg, float* exp_avg_sq, const float* grad,
                                  const NoiseRegion* region, const float* lr_per_tensor, float beta1, float beta2,
                                  float eps, float weight_decay, int adam_t, void* stream) {
  if (!params || !exp_avg || !exp_avg_sq || !grad || !lr_per_tensor || adam_t <= 0 || !region_ok(region))
    return kStatusBadArgument;
  static const ParamLayout L = make_param_layout();
  AdamDenseParams p{};
  int tiles = 0;
  for (int tid = region->tensor_begin; tid < region->tensor_end; ++tid) {
    if (lr_per_tensor[tid] < 0.f) continue;  // tensors another optimizer owns
    TensorSpan& s = p.t[p.count];
    s.offset = L.offset[tid];
    s.n = (int64_t)L.rows[tid] * L.cols[tid];
    s.tile_begin = tiles;
    p.tensor_id[p.count] = tid;
    p.packed[p.count] = packed_offset(tid);
    p.lr[p.count] = lr_per_tensor[tid];
    ++p.count;
    tiles += (int)((s.n + kOptTile - 1) / kOptTile);
  }
  if (p.count == 0) return kStatusOk;
  p.params = params;
  p.packed_w = reinterpret_cast<__nv_bfloat16*>(packed);
  p.m = exp_avg;
  p.v = exp_avg_sq;
  p.grad = grad;
  p.base = region->base;
  p.beta1 = beta1, p.beta2 = beta2, p.eps = eps, p.wd = weight_decay;
  p.bc1 = (float)(1.0 - pow((double)beta1, adam_t));
  p.bc2_sqrt = (float)sqrt(1.0 - pow((double)beta2, adam_t));
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  LaunchScope scope(kKindUpdate, s);
  adamw_dense_kernel<<<tiles, kOptBlock, 0, s>>>(p);
  return cudaGetLastError() == cudaSuccess ? kStatusOk : kStatusLaunchFailed;
}

extern "C" int noise_adamw_dense(float* params, void* packed, float* exp_avg, float* exp_avg_sq, const float* grad,
                                 const float* lr_per_tensor, float beta1, float beta2, float eps, float weight_decay,
                                 int adam_t, void* stream) {
  return noise_adamw_region(params, packed, exp_avg, exp_avg_sq, grad, &kAllTensors, lr_per_tensor, beta1, beta2, eps,
                            weight_decay, adam_t, stream);
}

extern "C" int noise_anvil_region_sizes(const NoiseRegion* region, int64_t* tiles, int64_t* lanes, int* matrices) {
  if (!region_ok(region) || !tiles || !lanes || !matrices) return kStatusBadArgument;
  AnvilParams p = make_anvil_params(*region, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr,
                                    nullptr, nullptr);
  *tiles = p.tiles;
  *lanes = p.lanes;
  *matrices = p.count;
  return kStatusOk;
}

extern "C" int noise_anvil_sizes(int64_t* tiles, int64_t* lanes, int* matrices) {
  return noise_anvil_region_sizes(&kAllTensors, tiles, lanes, matrices);
}

extern "C" int noise_anvil_region_prepare(const NoiseRegion* region, const float* grad, float* fast, float* slow,
                                          float* scratch, void* x, float* partials, float* scalars, float fast_beta,
                                          float slow_beta, float beta, float weight, void* stream) {
  if (!grad || !fast || !slow || !scratch || !x || !partials || !scalars || !region_ok(region))
    return kStatusBadArgument;
  AnvilParams p = make_anvil_params(*region, nullptr, nullptr, grad, fast, slow, scratch, x, nullptr, partials, scalars);
  if (p.count == 0) return kStatusOk;
  p.fast_beta = fast_beta, p.slow_beta = slow_beta, p.beta = beta, p.weight = weight;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  LaunchScope scope(kKindUpdate, s, 3);
  anvil_blend_kernel<<<p.tiles, kOptBlock, 0, s>>>(p);
  anvil_scalar_kernel<<<1, kMaxMatrices, 0, s>>>(p, 0);
  anvil_cast_kernel<<<p.tiles, kOptBlock, 0, s>>>(p);
  return cudaGetLastError() == cudaSuccess ? kStatusOk : kStatusLaunchFailed;
}

extern "C" int noise_anvil_prepare(const float* grad, float* fast, float* slow, float* scratch, void* x,
                                   float* partials, float* scalars, float fast_beta, float slow_beta, float beta,
                                   float weight, void* stream) {
  return noise_anvil_region_prepare(&kAllTensors, grad, fast, slow, scratch, x, partials, scalars, fast_beta,
                                    slow_beta, beta, weight, stream);
}

extern "C" int noise_anvil_region_finish(const NoiseRegion* region, float* params, void* packed, const float* slow,
                                         const void* update, float* energy, float* partials, float* scalars,
                                         float lane_beta, float lr, float weight_decay, void* stream) {
  if (!params || !slow || !update || !energy || !partials || !scalars || !region_ok(region))
    return kStatusBadArgument;
  AnvilParams p = make_anvil_params(*region, params, packed, nullptr, nullptr, const_cast<float*>(slow), nullptr,
                                    const_cast<void*>(update), energy, partials, scalars);
  if (p.count == 0) return kStatusOk;
  p.lane_beta = lane_beta, p.lr = lr, p.wd = weight_decay;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  LaunchScope scope(kKindUpdate, s, 4);
  anvil_energy_kernel<<<p.lanes, kOptBlock, 0, s>>>(p);
  anvil_norms_kernel<<<p.tiles, kOptBlock, 0, s>>>(p);
  anvil_scalar_kernel<<<1, kMaxMatrices, 0, s>>>(p, 1);
  anvil_apply_kernel<<<p.tiles, kOptBlock, 0, s>>>(p);
  return cudaGetLastError() == cudaSuccess ? kStatusOk : kStatusLaunchFailed;
}

extern "C" int noise_anvil_finish(float* params, void* packed, const float* slow, const void* update, float* energy,
                                  float* partials, float* scalars, float lane_beta, float lr, float weight_decay,
                                  void* stream) {
  return noise_anvil_region_finish(&kAllTensors, params, packed, slow, update, energy, partials, scalars, lane_beta, lr,
                                   weight_decay, stream);
}
