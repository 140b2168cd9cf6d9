// Update reconstruction fused with AdamW, and its partial form for the sharded update.
//
// For every parameter tensor, the estimated gradient of train/val/eggroll.py:155-166,
//     g = -scale * sum_d w_d a_d b_d^T     (matrices and embeddings: rank-1 factors a_d, b_d)
//     g = -scale * sum_d w_d eps_d         (mixing-scalar vectors)
// is accumulated tile by tile with the draws regenerated from the counter-based stream (no noise
// tensor is stored), then the AdamW step of torch.optim.AdamW (decoupled decay, m lerp, v update,
// bias-corrected step) is applied to the tile, and the packed bf16 GEMM copy is refreshed.
//
// noise_sum_fe_partial writes g alone for a range of directions, each tensor at a caller-given offset:
// a rank's share of the sum, laid out for the reduce-scatter of the sharded update.
//
// Tiles are 128 x 128; 256 threads hold 8 rows x 8 columns each (rows ty + 16 i, columns
// 4 tx + 64 j .. +3), so global reads and writes are 256-byte contiguous per half-warp. Draws for 8
// directions at a time are generated into shared memory.
#include "model_layout.cuh"
#include "noise_b200.h"
#include "profile.cuh"
#include "ptx.cuh"

namespace noise {

struct UpdTensor {
  int64_t offset;   // in the flat master buffer
  int64_t out;      // where g of this tensor starts in grad_out
  int64_t packed;   // packed bf16 destination offset, or -1
  int rows, cols;   // cols == 1: a vector of eps draws
  int tile_begin;   // first tile index of this tensor
  int tiles_c;      // tiles along columns
};

struct UpdParams {
  UpdTensor t[kNumTensors];
  int ntensors;
  float* params;
  __nv_bfloat16* packed;
  float* exp_avg;
  float* exp_avg_sq;
  float* grad_out;
  const float* weights;
  const float* lr_mult;  // per-tensor lr multiplier or nullptr
  int dir_begin, dir_end;  // the directions contracted: weights[d] for d in [dir_begin, dir_end)
  float scale;
  PhiloxKey key;
  float lr, beta1, beta2, eps, weight_decay, bc1, bc2_sqrt;
  int apply_adam;
};

constexpr int kUpdTile = 128;
constexpr int kUpdBatch = 8;

__global__ void __launch_bounds__(256) sum_fe_adamw_kernel(const __grid_constant__ UpdParams p) {
  __shared__ float4 sa[kUpdBatch][kUpdTile / 4];
  __shared__ float4 sb[kUpdBatch][kUpdTile / 4];
  __shared__ float sw[kUpdBatch];
  int ti = 0;
  while (ti + 1 < p.ntensors && (int)blockIdx.x >= p.t[ti + 1].tile_begin) ++ti;
  const UpdTensor T = p.t[ti];
  const int local = blockIdx.x - T.tile_begin;
  const int r0 = (local / T.tiles_c) * kUpdTile, c0 = (local % T.tiles_c) * kUpdTile;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const bool vec1d = T.cols == 1;

  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

  for (int d0 = p.dir_begin; d0 < p.dir_end; d0 += kUpdBatch) {
    __syncthreads();
    {
      // 8 directions x (32 a-blocks + 32 b-blocks) = 512 Philox blocks, two per thread
      for (int q = threadIdx.x; q < kUpdBatch * 64; q += 256) {
        const int dd = q >> 6, which = (q >> 5) & 1, blk = q & 31;
        const int d = d0 + dd;
        float4 g = make_float4(0.f, 0.f, 0.f, 0.f);
        if (d < p.dir_end) {
          if (which == 0) {
            const int e0 = r0 + 4 * blk;
            if (e0 < T.rows) g = gauss4(p.key, (uint32_t)(e0 >> 2), (uint32_t)ti, 0, (uint32_t)d);
          } else if (!vec1d) {
            const int e0 = c0 + 4 * blk;
            if (e0 < T.cols) g = gauss4(p.key, (uint32_t)(e0 >> 2), (uint32_t)ti, 1, (uint32_t)d);
          } else {
            g = make_float4(1.f, 1.f, 1.f, 1.f);  // a vector's "column factor" is 1
          }
        }
        (which == 0 ? sa : sb)[dd][blk] = g;
      }
      if (threadIdx.x < kUpdBatch) sw[threadIdx.x] = d0 + threadIdx.x < p.dir_end ? p.weights[d0 + threadIdx.x] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int dd = 0; dd < kUpdBatch; ++dd) {
      const float w = sw[dd];
      const float* a = reinterpret_cast<const float*>(sa[dd]);
      float bcol[8];
      const float4 b0 = sb[dd][tx], b1 = sb[dd][16 + tx];
      bcol[0] = b0.x, bcol[1] = b0.y, bcol[2] = b0.z, bcol[3] = b0.w;
      bcol[4] = b1.x, bcol[5] = b1.y, bcol[6] = b1.z, bcol[7] = b1.w;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float wa = w * a[ty + 16 * i];
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] += wa * bcol[j];
      }
    }
  }

  const float lr = p.lr * (p.lr_mult ? p.lr_mult[ti] : 1.0f);
  const float step = lr / p.bc1;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = r0 + ty + 16 * i;
    if (r >= T.rows) continue;
#pragma unroll
    for (int jj = 0; jj < 2; ++jj) {
      const int c = c0 + 4 * tx + 64 * jj;
      const int ncols = vec1d ? 1 : T.cols;
      if (c >= ncols) continue;
      const int64_t idx = T.offset + (int64_t)r * ncols + c;
      const int nv = min(4, ncols - c);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (u >= nv) break;
        const float g = -p.scale * acc[i][4 * jj + u];
        if (p.grad_out) p.grad_out[T.out + (idx - T.offset) + u] = g;
        if (!p.apply_adam) continue;
        float w = p.params[idx + u];
        if (p.weight_decay != 0.f) w *= 1.0f - lr * p.weight_decay;
        float m = p.exp_avg[idx + u], v = p.exp_avg_sq[idx + u];
        const float wgt = 1.0f - p.beta1;  // torch lerp: weight < 0.5 uses the first form
        m = wgt < 0.5f ? m + wgt * (g - m) : g - (g - m) * (1.0f - wgt);
        v = v * p.beta2 + (1.0f - p.beta2) * g * g;
        const float denom = sqrtf(v) / p.bc2_sqrt + p.eps;
        w -= step * (m / denom);
        p.params[idx + u] = w;
        p.exp_avg[idx + u] = m;
        p.exp_avg_sq[idx + u] = v;
        if (T.packed >= 0 && p.packed) p.packed[T.packed + (int64_t)r * ncols + c + u] = __float2bfloat16_rn(w);
      }
    }
  }
}

}  // namespace noise

using namespace noise;

static int64_t packed_offset_of(int tid) {
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

// The tensor table of every parameter: tiles, packed offsets, and g's destination (out_offsets[tid], or
// the flat layout when null).
static int build_tensors(UpdParams& p, const int64_t* out_offsets) {
  static const ParamLayout L = make_param_layout();
  int tiles = 0;
  for (int i = 0; i < kNumTensors; ++i) {
    UpdTensor& t = p.t[i];
    t.offset = L.offset[i];
    t.out = out_offsets ? out_offsets[i] : L.offset[i];
    t.rows = L.rows[i];
    t.cols = L.cols[i];
    t.packed = packed_offset_of(i);
    t.tiles_c = (t.cols + kUpdTile - 1) / kUpdTile;
    t.tile_begin = tiles;
    tiles += ((t.rows + kUpdTile - 1) / kUpdTile) * t.tiles_c;
  }
  p.ntensors = kNumTensors;
  return tiles;
}

extern "C" int noise_update_sum_fe_adamw(float* params, void* packed, float* exp_avg, float* exp_avg_sq,
                                         const float* weights, int pairs, float grad_scale, uint32_t seed,
                                         uint32_t step, const float* lr_mult, float lr, float beta1, float beta2,
                                         float eps, float weight_decay, int adam_t, float* grad_out, void* stream) {
  if (!params || !weights || pairs <= 0) return kStatusBadArgument;
  const bool adam = adam_t > 0;
  if (adam && (!exp_avg || !exp_avg_sq)) return kStatusBadArgument;
  if (!adam && !grad_out) return kStatusBadArgument;
  UpdParams p{};
  const int tiles = build_tensors(p, nullptr);
  p.params = params;
  p.packed = reinterpret_cast<__nv_bfloat16*>(packed);
  p.exp_avg = exp_avg;
  p.exp_avg_sq = exp_avg_sq;
  p.grad_out = grad_out;
  p.weights = weights;
  p.lr_mult = lr_mult;
  p.dir_begin = 0, p.dir_end = pairs;
  p.scale = grad_scale;
  p.key = PhiloxKey{seed, step};
  p.lr = lr, p.beta1 = beta1, p.beta2 = beta2, p.eps = eps, p.weight_decay = weight_decay;
  p.apply_adam = adam ? 1 : 0;
  if (adam) {
    p.bc1 = (float)(1.0 - pow((double)beta1, adam_t));
    p.bc2_sqrt = (float)sqrt(1.0 - pow((double)beta2, adam_t));
  } else {
    p.bc1 = 1.f, p.bc2_sqrt = 1.f;
  }
  LaunchScope scope(kKindUpdate, reinterpret_cast<cudaStream_t>(stream));
  sum_fe_adamw_kernel<<<tiles, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(p);
  return cudaGetLastError() == cudaSuccess ? kStatusOk : kStatusLaunchFailed;
}

extern "C" int noise_sum_fe_partial(const float* weights, int pairs, int dir_begin, int dir_count, float grad_scale,
                                    uint32_t seed, uint32_t step, const int64_t* out_offsets, float* out,
                                    void* stream) {
  if (!weights || !out || pairs <= 0 || dir_begin < 0 || dir_count < 0 || dir_begin + dir_count > pairs)
    return kStatusBadArgument;
  if (out_offsets)
    for (int i = 0; i < kNumTensors; ++i)
      if (out_offsets[i] < 0) return kStatusBadArgument;
  UpdParams p{};
  const int tiles = build_tensors(p, out_offsets);
  p.grad_out = out;
  p.weights = weights;
  p.dir_begin = dir_begin, p.dir_end = dir_begin + dir_count;
  p.scale = grad_scale;
  p.key = PhiloxKey{seed, step};
  p.apply_adam = 0;
  p.bc1 = 1.f, p.bc2_sqrt = 1.f;
  LaunchScope scope(kKindUpdate, reinterpret_cast<cudaStream_t>(stream));
  sum_fe_adamw_kernel<<<tiles, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(p);
  return cudaGetLastError() == cudaSuccess ? kStatusOk : kStatusLaunchFailed;
}
