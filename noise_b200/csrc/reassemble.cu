// Reassembly of a weight gradient from an output error and the module's cached input
// (train/val/run.py:465-471, DUST.reassemble: einsum('btd,bti->di', error, x) in float32, which the
// reference's set_float32_matmul_precision('high') runs on TF32 tensor cores):
//
//     g[o, i] = sum_k err[k, o] * x[k, i]         k over the B*T tokens (16,384 at the reference's batch)
//
// Both operands arrive token-major (the contraction index is their row), so a transpose kernel first
// writes them K-major in fp32 (bf16 inputs widened, and the input rows optionally scaled by 1/rms
// for the sites whose module input is a normalised stream: mlp.c_fc, lm_head, the attention
// projections). The tcgen05 engine then runs the product on kind::tf32 MMAs with an fp32-store
// epilogue. A site's output is only out / 128 M tiles (4 for a 512-row weight) against a long K, so
// K is split: the transposes write each operand as S blocks of K / S tokens, the engine's batched
// (block-diagonal) mode multiplies block s of the error with block s of the input, the epilogue
// stores each partial product compactly, and a reduction adds the S partials in order (deterministic).
// S is the smallest power of two that gives the engine at least one 128-row unit per SM, with at
// least 256 tokens per block. Shapes the 128 x 256 tiles do not divide (the 8 x 32 ve_gate) take an
// fp32 CUDA-core kernel instead.
#include "gemm_tc2.cuh"
#include "noise_b200.h"

namespace noise {

struct EpiStoreF32 {
  struct Params {
    float* C;
    int ldc;
    int out, in;  // with K split: partial s of C[out, in] at C + s * out * in (row b * out + r of the batch)
  };
  static constexpr int kSmemBytes = 0;
  static constexpr bool kInterleaveN = false;
  static constexpr bool kTf32 = true;
  const Params& p;
  __device__ EpiStoreF32(const Params& p_, uint8_t*, int, int) : p(p_) {}
  __device__ void begin_mtile(int, int) {}
  __device__ void begin_tile(int, int, int) {}
  __device__ void end_mtile(int, int, int) {}
  __device__ void group(int row, int col, float (&v)[64]) {
    const int b = row / p.out;  // batch (K block): 0 when K is not split
    float* c = p.C + ((size_t)b * p.out + (row - b * p.out)) * p.ldc + (col - b * p.in);
#pragma unroll
    for (int j = 0; j < 64; j += 8) st_global_v8f(c + j, v + j);
  }
};

// g[i] = sum over s of part[s * n + i], s in order
__global__ void __launch_bounds__(256) sum_splits_kernel(const float* __restrict__ part, int splits, int64_t n,
                                                         float* __restrict__ g) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float acc = 0.f;
  for (int sp = 0; sp < splits; ++sp) acc += part[sp * n + i];
  g[i] = acc;
}

// scale[k] = 1 / rms(x[k, 0 .. width)), one warp per row
__global__ void __launch_bounds__(256) row_rms_kernel(const void* __restrict__ x, int x_bf16, int ld, int width,
                                                      int rows, float* __restrict__ scale) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= rows) return;
  float ss = 0.f;
  for (int j = lane; j < width; j += 32) {
    const float v = x_bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(x)[(size_t)row * ld + j])
                           : reinterpret_cast<const float*>(x)[(size_t)row * ld + j];
    ss += v * v;
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (lane == 0) scale[row] = rsqrtf(ss / (float)width + 1.1920928955078125e-07f);
}

// out[k / kc][c][k % kc] = in[k, c] * (scale ? scale[k] : 1) for k < rows, c < cols (kc = rows: the plain
// transpose); fp32 or bf16 in, fp32 out
__global__ void __launch_bounds__(256) transpose_kernel(const void* __restrict__ in, int in_bf16, int ld, int rows,
                                                        int cols, const float* __restrict__ scale, int kc,
                                                        float* __restrict__ out) {
  __shared__ float tile[32][33];
  const int c0 = blockIdx.x * 32, k0 = blockIdx.y * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  for (int r = ty; r < 32; r += 8) {
    const int k = k0 + r, c = c0 + tx;
    float v = 0.f;
    if (k < rows && c < cols) {
      v = in_bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(in)[(size_t)k * ld + c])
                  : reinterpret_cast<const float*>(in)[(size_t)k * ld + c];
      if (scale) v *= scale[k];
    }
    tile[r][tx] = v;
  }
  __syncthreads();
  for (int r = ty; r < 32; r += 8) {
    const int c = c0 + r, k = k0 + tx;
    if (c < cols && k < rows) out[((size_t)(k / kc) * cols + c) * kc + k % kc] = tile[tx][r];
  }
}

// fp32 CUDA-core path: one block per output element, the block's threads split the K sum
__global__ void __launch_bounds__(256) small_contract_kernel(const float* __restrict__ err, int err_ld,
                                                             const void* __restrict__ x, int x_bf16, int x_ld,
                                                             const float* __restrict__ scale, int K, int in,
                                                             float* __restrict__ g) {
  const int o = blockIdx.x / in, i = blockIdx.x % in;
  float acc = 0.f;
  for (int k = threadIdx.x; k < K; k += blockDim.x) {
    float v = x_bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(x)[(size_t)k * x_ld + i])
                     : reinterpret_cast<const float*>(x)[(size_t)k * x_ld + i];
    if (scale) v *= scale[k];
    acc += err[(size_t)k * err_ld + o] * v;
  }
  __shared__ float red[8];
#pragma unroll
  for (int s = 16; s; s >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, s);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < 8; ++w) t += red[w];
    g[blockIdx.x] = t;
  }
}

static bool tensor_core_shape(int K, int out, int in) { return out % 128 == 0 && in % 256 == 0 && K % 32 == 0; }

// K blocks of the split product (1: not split); a power of two dividing K into blocks of >= 256 tokens
// (a multiple of the tf32 tile's 32), the smallest that gives at least 148 units of 128 rows
static int k_splits(int K, int out) {
  int sp = 1;
  while (sp * (out / 128) < 148 && K % (sp * 2 * 32) == 0 && K / (sp * 2) >= 256) sp *= 2;
  return sp;
}

static size_t align256(size_t b) { return (b + 255) / 256 * 256; }

}  // namespace noise

using namespace noise;

extern "C" int64_t noise_reassemble_workspace_bytes(int K, int out, int in) {
  if (K <= 0 || out <= 0 || in <= 0) return -1;
  size_t b = align256((size_t)K * 4);  // row scales
  if (tensor_core_shape(K, out, in)) {
    b += align256((size_t)out * K * 4) + align256((size_t)in * K * 4);
    const int sp = k_splits(K, out);
    if (sp > 1) b += align256((size_t)sp * out * in * 4);  // the partial products
  }
  return (int64_t)b;
}

extern "C" int noise_reassemble(const float* err, int err_ld, int K, int out, const void* x, int x_bf16, int x_ld,
                                int in, int x_norm, float* g, void* workspace, size_t workspace_bytes, int* status,
                                void* stream) {
  if (!err || !x || !g || !workspace || K <= 0 || out <= 0 || in <= 0 || err_ld < out || x_ld < in)
    return kStatusBadArgument;
  const int64_t need = noise_reassemble_workspace_bytes(K, out, in);
  if (need < 0 || (size_t)need > workspace_bytes) return kStatusWorkspaceTooSmall;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
  float* scale = x_norm ? reinterpret_cast<float*>(ws) : nullptr;
  const bool tc = tensor_core_shape(K, out, in);
  float* errT = reinterpret_cast<float*>(ws + align256((size_t)K * 4));
  float* xT = reinterpret_cast<float*>(ws + align256((size_t)K * 4) + align256((size_t)out * K * 4));
  const int sp = tc ? k_splits(K, out) : 1, kc = K / sp;
  float* part = reinterpret_cast<float*>(ws + align256((size_t)K * 4) + align256((size_t)out * K * 4) +
                                         align256((size_t)in * K * 4));
  {
    LaunchScope scope(kKindOther, s, (x_norm ? 1 : 0) + (tc ? 2 : 1));
    if (x_norm) row_rms_kernel<<<(K + 7) / 8, 256, 0, s>>>(x, x_bf16, x_ld, x_ld, K, scale);
    if (!tc) {
      small_contract_kernel<<<out * in, 256, 0, s>>>(err, err_ld, x, x_bf16, x_ld, scale, K, in, g);
      return cudaGetLastError() == cudaSuccess ? kStatusOk : kStatusLaunchFailed;
    }
    transpose_kernel<<<dim3((out + 31) / 32, (K + 31) / 32), 256, 0, s>>>(err, 0, err_ld, K, out, nullptr, kc, errT);
    transpose_kernel<<<dim3((in + 31) / 32, (K + 31) / 32), 256, 0, s>>>(x, x_bf16, x_ld, K, in, scale, kc, xT);
    if (cudaGetLastError() != cudaSuccess) return kStatusLaunchFailed;
  }
  if (sp == 1) {
    EpiStoreF32::Params ep{g, in, out, in};
    return launch_gemm<EpiStoreF32, 3>(errT, xT, out, in, K, K, K, ep, status, s, kKindOther);
  }
  EpiStoreF32::Params ep{part, in, out, in};
  const int rc = launch_gemm_tc<EpiStoreF32, 3>(errT, xT, sp * out, sp * in, kc, kc, kc, ep, status, s, kKindOther, 0,
                                                 out, in);
  if (rc != kStatusOk) return rc;
  const int64_t n = (int64_t)out * in;
  LaunchScope scope(kKindOther, s);
  sum_splits_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(part, sp, n, g);
  return cudaGetLastError() == cudaSuccess ? kStatusOk : kStatusLaunchFailed;
}
