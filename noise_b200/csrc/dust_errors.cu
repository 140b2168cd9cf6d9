// DUST's per-token error estimates from rerun losses, and the head's coordinate differences.
//
// noise_dust_errors (train/val/run.py:347-373): for draws [draw_begin, draw_begin + N) of one site,
// in chunks of n consecutive draws,
//     reward_i(t) = clean(t) - perturbed_i(t), centred over the chunk's draws,
//     optionally replaced by its reward-to-go sum_k gamma^k reward_i(t + k) (run.py:81-86),
//     plus, with credit-memory priors mu_s, the centred predicted drop sigma sum_s a_i,s(t) . mu_s(t),
//     errors(t, c) -= sum_i reward_i(t) * a_i(t, c) * live(t, c) / sigma
// with a_i regenerated from the counter-based stream (csrc/dust.cuh). One CTA per token; the
// draws' weights are staged in shared memory, the columns are spread over the threads. For an
// orthogonal draw a . mu = s H[row] . (pattern * mu), so one in-place Walsh-Hadamard transform of
// pattern * mu per token and draw cycle yields the predicted drop of every draw in that cycle.
//
// noise_coordinate_differences (run.py:120-137): for every token and every logit j, the central
// difference of the soft-capped cross-entropy along raw logit j, in closed form from the clean
// softmax; zero at ignored targets (< 0).
#include <math.h>

#include "dust.cuh"
#include "model_layout.cuh"
#include "noise_b200.h"
#include "profile.cuh"
#include "ptx.cuh"

namespace noise {

constexpr int kErrMaxDraws = 2048;
constexpr int kErrThreads = 256;
constexpr int kErrMaxPriorWidth = 2048;

struct ErrParams {
  const float* clean;        // [B*T]
  const float* perturbed;    // [N][B*T]
  const __nv_bfloat16* live; // [B*T][d] or nullptr
  float* errors;             // [B*T][d], accumulated
  int N, n, T, BT, d;
  uint32_t draw_begin, site;
  float gamma, inv_sigma;
  int lags;
  PhiloxKey key;
  int n_prior;
  uint32_t prior_site[2];
  int prior_d[2];
  const float* prior_mu[2];
  float sigma;
};

__global__ void __launch_bounds__(kErrThreads) dust_errors_kernel(const __grid_constant__ ErrParams p) {
  __shared__ float w[kErrMaxDraws];      // reward weight of each draw at this token
  __shared__ uint32_t hrow[kErrMaxDraws];
  __shared__ float pred[kErrMaxDraws];   // prior-predicted loss drop of each draw
  __shared__ float fw[kErrMaxPriorWidth];
  const int e = blockIdx.x;              // token (b * T + t)
  const int t = e % p.T;
  // 0. predicted drops sigma sum_s a_i,s . mu_s, through one transform per site and draw cycle
  if (p.n_prior > 0) {
    for (int i = threadIdx.x; i < p.N; i += blockDim.x) pred[i] = 0.f;
    for (int s = 0; s < p.n_prior; ++s) {
      const int d = p.prior_d[s];
      const float* mu = p.prior_mu[s] + (int64_t)e * d;
      const uint32_t c_lo = p.draw_begin / (uint32_t)d, c_hi = (p.draw_begin + (uint32_t)p.N - 1) / (uint32_t)d;
      for (uint32_t cyc = c_lo; cyc <= c_hi; ++cyc) {
        __syncthreads();  // fw and pred free
        for (int c = threadIdx.x; c < d; c += blockDim.x) {
          const uint32_t pat = pattern_word(p.key, p.prior_site[s], cyc, (uint32_t)c >> 5);
          fw[c] = ((pat >> (c & 31)) & 1u) ? -mu[c] : mu[c];
        }
        for (int h = 1; h < d; h <<= 1) {  // y[r] = sum_c (-1)^popcount(r & c) x[c]
          __syncthreads();
          for (int k = threadIdx.x; k < d / 2; k += blockDim.x) {
            const int i0 = (k / h) * 2 * h + (k % h), i1 = i0 + h;
            const float a = fw[i0], b = fw[i1];
            fw[i0] = a + b;
            fw[i1] = a - b;
          }
        }
        __syncthreads();
        for (int i = threadIdx.x; i < p.N; i += blockDim.x) {
          const uint32_t idx = p.draw_begin + (uint32_t)i;
          if (idx / (uint32_t)d != cyc) continue;
          const DrawRow r = draw_row(p.key, p.prior_site[s], idx, (uint32_t)e, (uint32_t)d);
          pred[i] += p.sigma * (r.sbit ? -fw[r.hrow] : fw[r.hrow]);
        }
      }
    }
    __syncthreads();
  }
  // 1. centred (and discounted) rewards of every draw at token e
  for (int i = threadIdx.x; i < p.N; i += blockDim.x) {
    const int c0 = (i / p.n) * p.n, c1 = min(p.N, c0 + p.n);
    const int lags = p.gamma != 0.f ? p.lags : 1;
    float acc = 0.f, g = 1.f;
    for (int k = 0; k < lags && t + k < p.T; ++k, g *= p.gamma) {
      const int ek = e + k;
      float mean = 0.f;
      if (c1 - c0 > 1) {
        for (int j = c0; j < c1; ++j) mean += p.clean[ek] - p.perturbed[(size_t)j * p.BT + ek];
        mean /= (float)(c1 - c0);
      }
      acc += g * ((p.clean[ek] - p.perturbed[(size_t)i * p.BT + ek]) - mean);
    }
    if (p.n_prior > 0) {  // the prior's predicted drop, centred like the reward, after the reward-to-go
      float pm = 0.f;
      if (c1 - c0 > 1) {
        for (int j = c0; j < c1; ++j) pm += pred[j];
        pm /= (float)(c1 - c0);
      }
      acc += pred[i] - pm;
    }
    const DrawRow r = draw_row(p.key, p.site, p.draw_begin + i, e, p.d);
    w[i] = r.sbit ? -acc * p.inv_sigma : acc * p.inv_sigma;  // fold the draw's sign in
    hrow[i] = r.hrow | (r.cycle << 16);
  }
  __syncthreads();
  // 2. errors(e, c) -= sum_i w_i * H[hrow_i][c] * pattern[cycle_i][c]
  for (int c = threadIdx.x; c < p.d; c += blockDim.x) {
    float acc = 0.f;
    uint32_t cur_cycle = 0xFFFFFFFFu, pat = 0;
    for (int i = 0; i < p.N; ++i) {
      const uint32_t hc = hrow[i];
      const uint32_t cyc = hc >> 16;
      if (cyc != cur_cycle) {
        cur_cycle = cyc;
        pat = pattern_word(p.key, p.site, cyc, (uint32_t)c >> 5);
      }
      const uint32_t neg = (__popc((hc & 0xFFFFu) & (uint32_t)c) ^ (pat >> (c & 31))) & 1u;
      acc += neg ? -w[i] : w[i];
    }
    if (p.live && !(__bfloat162float(p.live[(size_t)e * p.d + c]) > 0.f)) acc = 0.f;
    p.errors[(size_t)e * p.d + c] -= acc;
  }
}

// log-sum-exp of the soft-capped row, then the per-logit central differences
__global__ void __launch_bounds__(256) coordinate_differences_kernel(const float* __restrict__ raw,
                                                                     const int* __restrict__ targets, int V,
                                                                     float sigma, float* __restrict__ out) {
  const int64_t row = blockIdx.x;
  const float* r = raw + row * V;
  float* o = out + row * V;
  const int tgt = targets[row];
  __shared__ float red[32];
  auto cap = [](float v) { return kSoftCap * tanhf(v / kSoftCap); };
  float m = -INFINITY;
  for (int j = threadIdx.x; j < V; j += blockDim.x) m = fmaxf(m, cap(r[j]));
  for (int s = 16; s; s >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, s));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  m = red[0];
  for (int k = 1; k < (int)(blockDim.x >> 5); ++k) m = fmaxf(m, red[k]);
  __syncthreads();
  float z = 0.f;
  for (int j = threadIdx.x; j < V; j += blockDim.x) z += expf(cap(r[j]) - m);
  for (int s = 16; s; s >>= 1) z += __shfl_xor_sync(0xffffffffu, z, s);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = z;
  __syncthreads();
  z = 0.f;
  for (int k = 0; k < (int)(blockDim.x >> 5); ++k) z += red[k];
  const float inv2s = 1.0f / (2.0f * sigma);
  for (int j = threadIdx.x; j < V; j += blockDim.x) {
    if (tgt < 0) {
      o[j] = 0.f;
      continue;
    }
    const float zj = cap(r[j]), up = cap(r[j] + sigma), dn = cap(r[j] - sigma);
    const float wj = expf(zj - m) / z;  // the clean forward's probability of logit j
    float change = log1pf(wj * expm1f(up - zj)) - log1pf(wj * expm1f(dn - zj));
    if (j == tgt) change -= up - dn;  // the target logit's own term
    o[j] = change * inv2s;
  }
}

}  // namespace noise

using namespace noise;

extern "C" int noise_dust_errors(const float* clean, const float* perturbed, int draws, int chunk, int B, int T,
                                 int64_t draw_begin, uint32_t site, int d, float sigma, float gamma, const void* live,
                                 const NoisePrior* prior, uint32_t seed, uint32_t step, float* errors, void* stream) {
  if (!clean || !perturbed || !errors || draws <= 0 || draws > kErrMaxDraws || chunk <= 0 || B <= 0 || T <= 0)
    return kStatusBadArgument;
  if (d <= 0 || (d & (d - 1)) || d > 65536 || sigma == 0.f || draw_begin < 0) return kStatusBadArgument;
  if (draw_begin + draws > (int64_t)UINT32_MAX) return kStatusBadArgument;
  ErrParams p{};
  if (prior && prior->count > 0) {
    if (prior->count > 2) return kStatusBadArgument;
    for (int s = 0; s < prior->count; ++s) {
      const int pd = prior->d[s];
      if (!prior->mu[s] || pd < 2 || (pd & (pd - 1)) || pd > kErrMaxPriorWidth) return kStatusBadArgument;
      p.prior_site[s] = prior->site[s];
      p.prior_d[s] = pd;
      p.prior_mu[s] = prior->mu[s];
    }
    p.n_prior = prior->count;
  }
  p.sigma = sigma;
  p.clean = clean;
  p.perturbed = perturbed;
  p.live = reinterpret_cast<const __nv_bfloat16*>(live);
  p.errors = errors;
  p.N = draws, p.n = chunk, p.T = T, p.BT = B * T, p.d = d;
  p.draw_begin = (uint32_t)draw_begin, p.site = site;
  p.gamma = gamma, p.inv_sigma = 1.0f / sigma;
  p.lags = gamma != 0.f ? (int)ceil(log(1e-6) / log((double)gamma)) : 1;
  p.key = PhiloxKey{seed, step};
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  LaunchScope scope(kKindOther, s);
  dust_errors_kernel<<<B * T, kErrThreads, 0, s>>>(p);
  return cudaGetLastError() == cudaSuccess ? kStatusOk : kStatusLaunchFailed;
}

extern "C" int noise_coordinate_differences(const float* raw, const int32_t* targets, int64_t rows, float sigma,
                                            float* out, void* stream) {
  if (!raw || !targets || !out || rows <= 0 || sigma == 0.f) return kStatusBadArgument;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  LaunchScope scope(kKindOther, s);
  coordinate_differences_kernel<<<(unsigned)rows, 256, 0, s>>>(raw, targets, kVocab, sigma, out);
  return cudaGetLastError() == cudaSuccess ? kStatusOk : kStatusLaunchFailed;
}
