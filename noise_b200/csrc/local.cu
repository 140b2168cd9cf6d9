// DUST's attention-internal (local) errors: attention reruns of one block with a perturbed side,
// scored against the block's hub target (train/val/run.py:391-463).
//
// For a block of draws [draw_begin, draw_begin + N) of one kind at one layer:
//   1. local_prep_kernel writes each draw's operand, [N][B*T][512] bf16:
//        q, k   rms_norm(rope(raw + sigma a)) per head (the moved queries or keys)
//        v      sigma a                                  (the value change)
//        ve     sigma a * 2 sigmoid(z)
//        gate   (2 sigmoid(z + sigma a) - 2 sigmoid(z - sigma a)) * ve     (a: one value per head)
//      with a the orthogonal draw regenerated from the counter-based stream (csrc/dust.cuh).
//   2. attention_tc_kernel in score mode reruns the attention with that operand in place of the clean
//      one and writes score[j][b][t][h] = <target, O> - base, base = the clean attention's score
//      (kinds q, k; the value kinds are linear in the change and have no baseline).
//   3. local_credit_kernel (all kinds but q) spreads each score back over the earlier tokens that
//      see it: credit(t) = sum_{s = t .. t + window} gamma^(s - t) score(s), by a reverse linear
//      recurrence per (draw, sequence, head).
//   4. local_contract_kernel accumulates errors[e][c] += sum_j score_j(e, head(c)) a_j(e, c) / divisor.
// The host divides by the draw count once all blocks of draws are in.
#include <math.h>

#include "attention_tc.cuh"
#include "dust.cuh"
#include "model_layout.cuh"
#include "noise_b200.h"
#include "profile.cuh"
#include "ptx.cuh"

namespace noise {

enum : int { kLocalQ = 0, kLocalK = 1, kLocalV = 2, kLocalGate = 3, kLocalVe = 4 };
constexpr int kLocalMaxDraws = 1024;

int make_tmap_2d(CUtensorMap* map, const void* ptr, CUtensorMapDataType dtype, int elem_bytes, uint64_t rows,
                 uint64_t cols, uint64_t row_stride_elems, uint32_t box_rows, uint32_t box_cols);

struct LocalPrep {
  int kind;
  uint32_t site;
  float sigma;
  const __nv_bfloat16* raw;  // q, k: [BT][512]
  const float* z;            // gate, ve: [BT][8]
  const float* ve;           // gate, ve: [BT][512]
  const float* rope;         // [T][64] cos | sin
  __nv_bfloat16* out;        // [draws][BT][512]
  int BT, T, draws;
  uint32_t draw_begin;
  PhiloxKey key;
};

__device__ __forceinline__ float sigmoid2(float x) { return 2.0f / (1.0f + expf(-x)); }

// One warp per (draw, token); lane -> head lane / 4 and columns c0 .. c0 + 7, c0 + 32 .. c0 + 39 of
// that head (c0 = head * 64 + (lane % 4) * 8), so each RoPE pair and each head's norm stay in 4 lanes.
__global__ void __launch_bounds__(256) local_prep_kernel(const __grid_constant__ LocalPrep p) {
  const int64_t wid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (wid >= (int64_t)p.draws * p.BT) return;
  const int j = (int)(wid / p.BT), e = (int)(wid % p.BT);
  const int lane = threadIdx.x & 31, head = lane >> 2, part = lane & 3;
  const int c0 = head * kHeadDim + part * 8;
  const uint32_t idx = p.draw_begin + (uint32_t)j;
  const bool moved = p.sigma != 0.f;
  float a[16];
  if (!moved) {
#pragma unroll
    for (int i = 0; i < 16; ++i) a[i] = 0.f;
  } else if (p.kind == kLocalGate) {
    // width 8: one draw value per head; lane 0 fetches the row state and the cycle's pattern word
    uint32_t hrow = 0, sbit = 0, pat = 0;
    if (lane == 0) {
      const DrawRow r = draw_row(p.key, p.site, idx, (uint32_t)e, kHeads);
      hrow = r.hrow, sbit = r.sbit;
      pat = pattern_word(p.key, p.site, r.cycle, 0);
    }
    hrow = __shfl_sync(0xffffffffu, hrow, 0);
    sbit = __shfl_sync(0xffffffffu, sbit, 0);
    pat = __shfl_sync(0xffffffffu, pat, 0);
    const float ah = ((__popc(hrow & (uint32_t)head) ^ sbit ^ (pat >> head)) & 1u) ? -1.f : 1.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) a[i] = ah;
  } else {
    // width 512: the Hadamard row offset (lane 0), the draw sign (lane 1), pattern word w (lane w % 16)
    const uint32_t cycle = idx / kWidth;
    uint32_t mine = 0;
    if (lane == 0) mine = draw_offset(p.key, p.site, (uint32_t)e, kWidth);
    else if (lane == 1) mine = draw_sign_bit(p.key, p.site, idx, (uint32_t)e);
    const uint32_t patw = pattern_word(p.key, p.site, cycle, (uint32_t)(lane & 15));
    const uint32_t off = __shfl_sync(0xffffffffu, mine, 0);
    const uint32_t sbit = __shfl_sync(0xffffffffu, mine, 1);
    const uint32_t w_lo = __shfl_sync(0xffffffffu, patw, 2 * head);
    const uint32_t w_hi = __shfl_sync(0xffffffffu, patw, 2 * head + 1);
    DrawRow r;
    r.hrow = (off + idx) & (kWidth - 1), r.sbit = sbit, r.cycle = cycle;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      a[i] = draw_value(r, (uint32_t)(c0 + i), w_lo);
      a[8 + i] = draw_value(r, (uint32_t)(c0 + 32 + i), w_hi);
    }
  }
  float x[16];
  const int64_t row = (int64_t)e * kWidth;
  if (p.kind == kLocalQ || p.kind == kLocalK) {
    const uint4 lo = __ldg(reinterpret_cast<const uint4*>(p.raw + row + c0));
    const uint4 hi = __ldg(reinterpret_cast<const uint4*>(p.raw + row + c0 + 32));
    const uint32_t wl[4] = {lo.x, lo.y, lo.z, lo.w}, wh[4] = {hi.x, hi.y, hi.z, hi.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 fl = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&wl[i]));
      const float2 fh = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&wh[i]));
      x[2 * i] = fl.x + p.sigma * a[2 * i];
      x[2 * i + 1] = fl.y + p.sigma * a[2 * i + 1];
      x[8 + 2 * i] = fh.x + p.sigma * a[8 + 2 * i];
      x[8 + 2 * i + 1] = fh.y + p.sigma * a[8 + 2 * i + 1];
    }
    // RoPE (utils/model.py:55-58): (x1, x2) -> (x1 cos + x2 sin, -x1 sin + x2 cos), frequency part * 8 + i
    const float* cs = p.rope + (int64_t)(e % p.T) * kHeadDim + part * 8;
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float c = __ldg(cs + i), s = __ldg(cs + 32 + i);
      const float x1 = x[i], x2 = x[8 + i];
      x[i] = x1 * c + x2 * s;
      x[8 + i] = x1 * -s + x2 * c;
      ss += x[i] * x[i] + x[8 + i] * x[8 + i];
    }
    ss += __shfl_xor_sync(0xffffffffu, ss, 1);
    ss += __shfl_xor_sync(0xffffffffu, ss, 2);
    const float inv = rsqrtf(ss / (float)kHeadDim + kNormEps);
#pragma unroll
    for (int i = 0; i < 16; ++i) x[i] *= inv;
  } else if (p.kind == kLocalV) {
#pragma unroll
    for (int i = 0; i < 16; ++i) x[i] = p.sigma * a[i];
  } else {
    const float zh = __ldg(p.z + (int64_t)e * kHeads + head);
    const float* ve = p.ve + row;
    if (p.kind == kLocalVe) {
      const float g = sigmoid2(zh);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        x[i] = p.sigma * a[i] * g;
        x[8 + i] = p.sigma * a[8 + i] * g;
      }
    } else {
      const float dg = sigmoid2(zh + p.sigma * a[0]) - sigmoid2(zh - p.sigma * a[0]);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        x[i] = dg * __ldg(ve + c0 + i);
        x[8 + i] = dg * __ldg(ve + c0 + 32 + i);
      }
    }
  }
  __nv_bfloat16* o = p.out + ((int64_t)j * p.BT + e) * kWidth;
  uint4 lo, hi;
  lo.x = pack_bf16x2(x[0], x[1]), lo.y = pack_bf16x2(x[2], x[3]);
  lo.z = pack_bf16x2(x[4], x[5]), lo.w = pack_bf16x2(x[6], x[7]);
  hi.x = pack_bf16x2(x[8], x[9]), hi.y = pack_bf16x2(x[10], x[11]);
  hi.z = pack_bf16x2(x[12], x[13]), hi.w = pack_bf16x2(x[14], x[15]);
  *reinterpret_cast<uint4*>(o + c0) = lo;
  *reinterpret_cast<uint4*>(o + c0 + 32) = hi;
}

struct LocalCredit {
  const float* score;  // [Z][T][8]
  float* out;          // [Z][T][8]
  int Z, T, window;
  float gamma, tail;   // tail = gamma^(window + 1)
};

// One CTA per row block z; T is cut into 32 chunks of L = T / 32 tokens. Thread (warp w, lane l)
// takes head l % 8 of chunk 4 w + l / 8, so that each load of a warp reads the 8 heads of one token
// (32 contiguous bytes) in each of 4 chunks. credit(t) = c(t) + gamma credit(t + 1) with
// c(t) = score(t) - gamma^(window+1) score(t + window + 1): every thread runs the recurrence over its
// chunk from zero, one thread per head carries the chunks' start values back through the chunks in
// shared memory, and a second pass adds gamma^(chunk end - t) times the carry of the next chunk.
__global__ void __launch_bounds__(256) local_credit_kernel(const __grid_constant__ LocalCredit p) {
  __shared__ float start[kHeads][32], carry[kHeads][32];
  const int64_t z = blockIdx.x;
  const int head = threadIdx.x & 7, chunk = threadIdx.x >> 3;
  const float* s = p.score + z * p.T * kHeads + head;
  float* o = p.out + z * p.T * kHeads + head;
  const int L = p.T / 32, t0 = chunk * L;
  float y = 0.f;
  for (int t = t0 + L - 1; t >= t0; --t) {
    float c = s[(int64_t)t * kHeads];
    if (t + p.window + 1 < p.T) c -= p.tail * s[(int64_t)(t + p.window + 1) * kHeads];
    y = c + p.gamma * y;
    o[(int64_t)t * kHeads] = y;
  }
  start[head][chunk] = y;
  __syncthreads();
  if (threadIdx.x < kHeads) {  // thread h: carry[h][k] = credit at the first token of chunk k + 1
    float gL = 1.f;
    for (int i = 0; i < L; ++i) gL *= p.gamma;
    float c = 0.f;
    carry[threadIdx.x][31] = 0.f;
    for (int k = 30; k >= 0; --k) {
      c = start[threadIdx.x][k + 1] + gL * c;
      carry[threadIdx.x][k] = c;
    }
  }
  __syncthreads();
  const float cr = carry[head][chunk];
  float f = 1.f;
  for (int t = t0 + L - 1; t >= t0; --t) {
    f *= p.gamma;
    o[(int64_t)t * kHeads] += f * cr;
  }
}

struct LocalContract {
  const float* w;   // [draws][BT][8]
  float* errors;    // [BT][width]
  int draws, BT, width;
  uint32_t draw_begin, site;
  float inv_div;
  PhiloxKey key;
};

// One CTA per token: the draws' per-head weights and Hadamard rows in shared memory, the columns
// over the threads.
__global__ void __launch_bounds__(256) local_contract_kernel(const __grid_constant__ LocalContract p) {
  __shared__ float sw[kLocalMaxDraws * kHeads];
  __shared__ uint32_t srow[kLocalMaxDraws];
  const int e = blockIdx.x;
  for (int i = threadIdx.x; i < p.draws; i += blockDim.x) {
    const DrawRow r = draw_row(p.key, p.site, p.draw_begin + (uint32_t)i, (uint32_t)e, (uint32_t)p.width);
    const float4* src = reinterpret_cast<const float4*>(p.w + ((int64_t)i * p.BT + e) * kHeads);
    const float4 u = __ldg(src), v = __ldg(src + 1);
    const float sg = (r.sbit ? -1.f : 1.f) * p.inv_div;
    float* d = sw + i * kHeads;
    d[0] = u.x * sg, d[1] = u.y * sg, d[2] = u.z * sg, d[3] = u.w * sg;
    d[4] = v.x * sg, d[5] = v.y * sg, d[6] = v.z * sg, d[7] = v.w * sg;
    srow[i] = r.hrow | (r.cycle << 16);
  }
  __syncthreads();
  for (int c = threadIdx.x; c < p.width; c += blockDim.x) {
    const int h = p.width == kHeads ? c : c / kHeadDim;
    float acc = 0.f;
    uint32_t cur = 0xFFFFFFFFu, pat = 0;
    for (int i = 0; i < p.draws; ++i) {
      const uint32_t hc = srow[i];
      if ((hc >> 16) != cur) {
        cur = hc >> 16;
        pat = pattern_word(p.key, p.site, cur, (uint32_t)c >> 5);
      }
      const uint32_t neg = (__popc((hc & 0xFFFFu) & (uint32_t)c) ^ (pat >> (c & 31))) & 1u;
      const float wv = sw[i * kHeads + h];
      acc += neg ? -wv : wv;
    }
    p.errors[(int64_t)e * p.width + c] += acc;
  }
}

constexpr int kLocalKeyTile = 64;  // as the population forward's attention (population.cu)

template <int G, int KT>
int launch_local_attention_g(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                             const AttnTcParams& ap, int Z, cudaStream_t stream) {
  using L = AttnTcLayout<G, KT>;
  static bool configured = false;
  if (!configured) {
    if (cudaFuncSetAttribute(attention_tc_kernel<G, KT, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kSmem) !=
        cudaSuccess)
      return kStatusLaunchFailed;
    configured = true;
  }
  dim3 grid(ap.ctx.T / (kAtQ * G), kHeads, (unsigned)Z);
  LaunchScope scope(kKindAttention, stream);
  attention_tc_kernel<G, KT, true><<<grid, L::kThreads, L::kSmem, stream>>>(tq, tk, tv, ap);
  return cudaGetLastError() == cudaSuccess ? kStatusOk : kStatusLaunchFailed;
}

// Score-mode attention over Z = draws * B row blocks; a null moved operand keeps the clean one.
int launch_local_attention(const NoiseLocal* s, int B, int T, int Z, const __nv_bfloat16* moved, int moved_kind,
                           const float* base, float* score, int* status, cudaStream_t stream) {
  const uint64_t clean_rows = (uint64_t)B * T, moved_rows = (uint64_t)Z * T;
  const void* src[3] = {s->q, s->k, s->values};
  int slot = -1;
  if (moved) slot = moved_kind == kLocalQ ? 0 : moved_kind == kLocalK ? 1 : 2;
  CUtensorMap tm[3];
  int mod[3];
  for (int i = 0; i < 3; ++i) {
    const bool m = i == slot;
    if (make_tmap_2d(&tm[i], m ? (const void*)moved : src[i], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                     m ? moved_rows : clean_rows, kWidth, kWidth, 64, kHeadDim))
      return kStatusBadArgument;
    mod[i] = m ? 0 : B;
  }
  AttnTcParams ap{};
  ap.ctx.T = T, ap.ctx.B = B;
  ap.layer = s->layer, ap.window = layer_window(s->layer), ap.status = status;
  ap.col_q = ap.col_k = ap.col_v = 0;
  ap.mod_q = mod[0], ap.mod_k = mod[1], ap.mod_v = mod[2];
  ap.target = reinterpret_cast<const __nv_bfloat16*>(s->target);
  ap.base = base, ap.score = score, ap.seqs = B;
  const int n_qt = T / kAtQ;
  if (kLocalKeyTile == 128) return launch_local_attention_g<1, 128>(tm[0], tm[1], tm[2], ap, Z, stream);
  if (n_qt % 2 == 0) return launch_local_attention_g<2, 64>(tm[0], tm[1], tm[2], ap, Z, stream);
  return launch_local_attention_g<1, 64>(tm[0], tm[1], tm[2], ap, Z, stream);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

int check_local(const NoiseLocal* s, int B, int T) {
  if (!s || B <= 0 || T <= 0 || T % kAtQ || (int64_t)B * T > (1 << 24)) return kStatusBadArgument;
  if (s->kind < kLocalQ || s->kind > kLocalVe || s->layer < 0 || s->layer >= kLayers) return kStatusBadArgument;
  if ((s->kind == kLocalGate || s->kind == kLocalVe) && !has_ve(s->layer)) return kStatusBadArgument;
  if (!s->q || !s->k || !s->values || !s->target) return kStatusBadArgument;
  if (!aligned16(s->q) || !aligned16(s->k) || !aligned16(s->values) || !aligned16(s->target)) return kStatusBadArgument;
  return kStatusOk;
}

}  // namespace noise

using namespace noise;

extern "C" int64_t noise_local_workspace_bytes(int B, int T, int draws) {
  if (B <= 0 || T <= 0 || draws <= 0) return -1;
  const int64_t rows = (int64_t)draws * B * T;
  return rows * kWidth * 2 + 2 * rows * kHeads * 4 + 1024;
}

extern "C" int noise_local_process(const void* raw, const float* rope, int B, int T, void* out, void* stream) {
  if (!raw || !rope || !out || B <= 0 || T <= 0 || !aligned16(raw) || !aligned16(out)) return kStatusBadArgument;
  LocalPrep lp{};
  lp.kind = kLocalQ, lp.sigma = 0.f;
  lp.raw = reinterpret_cast<const __nv_bfloat16*>(raw);
  lp.rope = rope;
  lp.out = reinterpret_cast<__nv_bfloat16*>(out);
  lp.BT = B * T, lp.T = T, lp.draws = 1;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  LaunchScope scope(kKindOther, st);
  local_prep_kernel<<<(unsigned)(((int64_t)B * T * 32 + 255) / 256), 256, 0, st>>>(lp);
  return cudaGetLastError() == cudaSuccess ? kStatusOk : kStatusLaunchFailed;
}

extern "C" int noise_local_baseline(const NoiseLocal* s, int B, int T, float* base, int* status, void* stream) {
  int rc = check_local(s, B, T);
  if (rc) return rc;
  if (!base || !status) return kStatusBadArgument;
  return launch_local_attention(s, B, T, B, nullptr, 0, nullptr, base, status, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int noise_local_errors(const NoiseLocal* s, const float* rope, int B, int T, int64_t draw_begin, int draws,
                                  uint32_t seed, uint32_t step, float* errors, void* workspace, size_t ws_bytes,
                                  int* status, void* stream) {
  int rc = check_local(s, B, T);
  if (rc) return rc;
  if (!errors || !workspace || !status || draws <= 0 || draws > kLocalMaxDraws || draw_begin < 0) return kStatusBadArgument;
  if ((int64_t)draws * B > 65535 || draw_begin + draws > (int64_t)UINT32_MAX) return kStatusBadArgument;
  const bool qk = s->kind == kLocalQ || s->kind == kLocalK;
  if (qk && (!s->raw || !rope || !s->base || !aligned16(s->raw))) return kStatusBadArgument;
  if (!qk && (s->kind != kLocalV) && (!s->gate_logits || !s->ve)) return kStatusBadArgument;
  const int64_t need = noise_local_workspace_bytes(B, T, draws);
  if ((int64_t)ws_bytes < need) return kStatusBadArgument;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int64_t BT = (int64_t)B * T, rows = (int64_t)draws * BT;
  uint8_t* ws = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(workspace) + 1023) & ~uintptr_t(1023));
  __nv_bfloat16* op = reinterpret_cast<__nv_bfloat16*>(ws);
  float* score = reinterpret_cast<float*>(ws + rows * kWidth * 2);
  float* credit = score + rows * kHeads;
  const PhiloxKey key{seed, step};

  LocalPrep lp{};
  lp.kind = s->kind, lp.site = s->site, lp.sigma = s->sigma;
  lp.raw = reinterpret_cast<const __nv_bfloat16*>(s->raw);
  lp.z = s->gate_logits, lp.ve = s->ve, lp.rope = rope, lp.out = op;
  lp.BT = (int)BT, lp.T = T, lp.draws = draws, lp.draw_begin = (uint32_t)draw_begin, lp.key = key;
  {
    LaunchScope scope(kKindOther, st);
    local_prep_kernel<<<(unsigned)((rows * 32 + 255) / 256), 256, 0, st>>>(lp);
    if (cudaGetLastError() != cudaSuccess) return kStatusLaunchFailed;
  }
  rc = launch_local_attention(s, B, T, draws * B, op, s->kind, qk ? s->base : nullptr, score, status, st);
  if (rc) return rc;
  const float* w = score;
  if (s->kind != kLocalQ) {
    LocalCredit lc{};
    lc.score = score, lc.out = credit, lc.Z = draws * B, lc.T = T, lc.window = layer_window(s->layer);
    lc.gamma = s->gamma;
    lc.tail = (float)pow((double)s->gamma, (double)(lc.window + 1));
    LaunchScope scope(kKindOther, st);
    local_credit_kernel<<<(unsigned)lc.Z, 256, 0, st>>>(lc);
    if (cudaGetLastError() != cudaSuccess) return kStatusLaunchFailed;
    w = credit;
  }
  LocalContract lc{};
  lc.w = w, lc.errors = errors, lc.draws = draws, lc.BT = (int)BT;
  lc.width = s->kind == kLocalGate ? kHeads : kWidth;
  lc.draw_begin = (uint32_t)draw_begin, lc.site = s->site;
  lc.inv_div = 1.0f / (s->kind == kLocalGate ? 2.0f * s->sigma : s->sigma);
  lc.key = key;
  LaunchScope scope(kKindOther, st);
  local_contract_kernel<<<(unsigned)BT, 256, 0, st>>>(lc);
  return cudaGetLastError() == cudaSuccess ? kStatusOk : kStatusLaunchFailed;
}
