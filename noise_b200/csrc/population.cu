// Population forward of the rank-1 (EGGROLL) estimator: the perturbed forward of
// `population_loss` (train/val/eggroll.py:66-103) for a contiguous range of members, each member
// evaluating every row of a [B, T] token batch, reduced to one mean cross-entropy per member.
//
// Kernel sequence per chunk of members (rows ordered member, sequence, token):
//   embed            x0 = norm(wte[id] + s a_id b) and block 0's input, with its row statistics
//   8 x { QKV GEMM   q, k (RoPE + QK-norm), v (+ gated value embedding)
//         attention  sliding window, writes y and y.b_proj
//         proj GEMM  x += y Wp^T (+rank-1); FC input + stats
//         FC GEMM    relu^2 hidden (bf16) + hidden.b_mlp
//         MLP GEMM   x += hidden Wm^T (+rank-1); next block's mixed input + stats }
//   head GEMM        soft-capped logits -> per-row log-sum-exp pieces
//   member loss      mean over the member's B*T rows
// No noise tensor is ever materialised: the draws are the counter-based stream of (seed, step,
// direction, tensor). Each chunk starts with draw_table_kernel, which writes the rank-1 vectors of
// the directions it spans (a few hundred KB each) for the epilogues, the embedding and the attention
// to read; the direct-mode jitter is regenerated where it is added.
#include "attention_tc.cuh"
#include "epilogues.cuh"
#include "gemm_tc2.cuh"
#include "noise_b200.h"

namespace noise {

// ------------------------------------------------------------------------------------------------
// embedding + block-0 input
// ------------------------------------------------------------------------------------------------
struct EmbedParams {
  PopCtx ctx;
  const float* wte;
  const float* lambdas;  // resid[8] | x0[8]
  float* x;
  __nv_bfloat16* xb;
  float* inv0;
  float* stats;   // stats_a: [rows][4][16]
  float* x0_out;  // [rows, 512] normalised embedding (capture only), or nullptr
};

constexpr int kEmbedRows = 64;

__global__ void __launch_bounds__(256) embed_kernel(const __grid_constant__ EmbedParams p) {
  __shared__ float4 sv[4][kWidth / 4];  // b_wte, b_q0, b_k0, b_v0
  __shared__ uint32_t patw[kWidth / 32];  // direct mode: pattern words of the embedding draw
  const int64_t row0 = (int64_t)blockIdx.x * kEmbedRows;
  const RowInfo r0 = row_info(p.ctx, row0);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int i = tid; i < 4 * (kWidth / 4); i += blockDim.x) {
    const int v = i / (kWidth / 4), blk = i % (kWidth / 4);
    const uint32_t tensor = v == 0 ? kTidWte : v == 1 ? tid_q(0) : v == 2 ? tid_k(0) : tid_v(0);
    sv[v][blk] = p.ctx.sigma != 0.f ? draw4(p.ctx, r0.slot, tensor, 1, blk) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  const SiteJitter j0 = site_jitter(p.ctx, -1, kSiteWte, row0, kWidth);  // same draw for the whole CTA
  if (j0.on && tid < kWidth / 128) {
    uint32_t w[4];
    site_patterns(p.ctx, kSiteWte, j0.r, tid * 128, w);
    for (int k = 0; k < 4; ++k) patw[tid * 4 + k] = w[k];
  }
  __syncthreads();
  const float mix = p.lambdas[0] + r0.sign * draw1(p.ctx, r0.slot, kTidResid, 0, 0) + p.lambdas[kLayers] +
                    r0.sign * draw1(p.ctx, r0.slot, kTidX0, 0, 0);
  for (int rr = warp; rr < kEmbedRows; rr += 8) {
    const int64_t row = row0 + rr;
    const RowInfo ri = row_info(p.ctx, row);
    const float sa = p.ctx.sigma != 0.f ? ri.sign * draw1(p.ctx, ri.slot, kTidWte, 0, ri.tok) : 0.f;
    const SiteJitter jit = site_jitter(p.ctx, -1, kSiteWte, row, kWidth);
    const float4* w = reinterpret_cast<const float4*>(p.wte + (size_t)ri.tok * kWidth);
    float4 e[4];
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int c4 = lane + 32 * k;
      const float4 wv = __ldg(w + c4), bv = sv[0][c4];
      e[k] = make_float4(wv.x + sa * bv.x, wv.y + sa * bv.y, wv.z + sa * bv.z, wv.w + sa * bv.w);
      if (jit.on) {
        const uint32_t c = 4 * c4;
        const uint32_t pw = patw[c >> 5];
        e[k].x += jit.scale * draw_value(jit.r, c, pw);
        e[k].y += jit.scale * draw_value(jit.r, c + 1, pw);
        e[k].z += jit.scale * draw_value(jit.r, c + 2, pw);
        e[k].w += jit.scale * draw_value(jit.r, c + 3, pw);
      }
      ss += e[k].x * e[k].x + e[k].y * e[k].y + e[k].z * e[k].z + e[k].w * e[k].w;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float i0 = rms_scale(ss, kWidth);
    float ssx = 0.f, dq = 0.f, dk = 0.f, dv = 0.f;
    float4* xo = reinterpret_cast<float4*>(p.x + (size_t)row * kWidth);
    uint2* xbo = reinterpret_cast<uint2*>(p.xb + (size_t)row * kWidth);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int c4 = lane + 32 * k;
      const float4 x0v = make_float4(e[k].x * i0, e[k].y * i0, e[k].z * i0, e[k].w * i0);
      if (p.x0_out) reinterpret_cast<float4*>(p.x0_out + (size_t)row * kWidth)[c4] = x0v;
      const float4 xi = make_float4(mix * x0v.x, mix * x0v.y, mix * x0v.z, mix * x0v.w);
      xo[c4] = xi;
      ssx += xi.x * xi.x + xi.y * xi.y + xi.z * xi.z + xi.w * xi.w;
      const float r[4] = {bf16_round(xi.x), bf16_round(xi.y), bf16_round(xi.z), bf16_round(xi.w)};
      xbo[c4] = make_uint2(pack_bf16x2(r[0], r[1]), pack_bf16x2(r[2], r[3]));
      const float4 bq = sv[1][c4], bk = sv[2][c4], bvv = sv[3][c4];
      dq += r[0] * bq.x + r[1] * bq.y + r[2] * bq.z + r[3] * bq.w;
      dk += r[0] * bk.x + r[1] * bk.y + r[2] * bk.z + r[3] * bk.w;
      dv += r[0] * bvv.x + r[1] * bvv.y + r[2] * bvv.z + r[3] * bvv.w;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      ssx += __shfl_xor_sync(0xffffffffu, ssx, o);
      dq += __shfl_xor_sync(0xffffffffu, dq, o);
      dk += __shfl_xor_sync(0xffffffffu, dk, o);
      dv += __shfl_xor_sync(0xffffffffu, dv, o);
    }
    const float vals[4] = {ssx, dq, dk, dv};
    float* st = p.stats + (size_t)row * kStatParts * kStatStride;  // part 0 holds the sums, parts 1..3 zero
    st[lane] = lane < 4 ? vals[lane] : 0.f;
    st[32 + lane] = 0.f;
    if (lane == 0) p.inv0[row] = i0;
  }
}

// ------------------------------------------------------------------------------------------------
// direct mode from block `entry` >= 0: every draw starts from the clean input of that block
// ------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) direct_start_kernel(const __grid_constant__ EmbedParams p, int64_t rows) {
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int64_t seq = row % ((int64_t)p.ctx.B * p.ctx.T);
  const float4* src = reinterpret_cast<const float4*>(p.ctx.dir.x_entry + (size_t)seq * kWidth);
  float4* xo = reinterpret_cast<float4*>(p.x + (size_t)row * kWidth);
  uint2* xbo = reinterpret_cast<uint2*>(p.xb + (size_t)row * kWidth);
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int c4 = lane + 32 * k;
    const float4 v = __ldg(src + c4);
    xo[c4] = v;
    xbo[c4] = make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
    ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  float* st = p.stats + (size_t)row * kStatParts * kStatStride;
  st[lane] = lane == 0 ? ss : 0.f;
  st[32 + lane] = 0.f;
  if (lane == 0) p.inv0[row] = p.ctx.dir.inv0[seq];
}

// per-token cross-entropy from the head's pieces; ignored targets (< 0) score 0
__global__ void token_loss_kernel(const float* part, const int* targets, int64_t rows, int64_t seq_rows, float* out) {
  const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  const float4 q = reinterpret_cast<const float4*>(part)[r];
  out[r] = targets[r % seq_rows] < 0 ? 0.f : logf(q.x + q.z) + kSoftCap - (q.y + q.w);
}

// ------------------------------------------------------------------------------------------------
// per-member mean cross-entropy from the head's per-row pieces
// ------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) member_loss_kernel(const float* part, int64_t rows_per_member, float* losses) {
  const int m = blockIdx.x;
  const float* pm = part + (size_t)m * rows_per_member * 4;
  double acc = 0.0;
  for (int64_t r = threadIdx.x; r < rows_per_member; r += blockDim.x) {
    const float4 q = reinterpret_cast<const float4*>(pm)[r];
    acc += (double)(logf(q.x + q.z) + kSoftCap - (q.y + q.w));
  }
  __shared__ double red[256];
  red[threadIdx.x] = acc;
  __syncthreads();
  for (int s = 128; s; s >>= 1) {
    if (threadIdx.x < s) red[threadIdx.x] += red[threadIdx.x + s];
    __syncthreads();
  }
  if (threadIdx.x == 0) losses[m] = (float)(red[0] / (double)rows_per_member);
}

// ------------------------------------------------------------------------------------------------
// master fp32 -> packed bf16 GEMM weights
// ------------------------------------------------------------------------------------------------
struct PackJob {
  int64_t src, dst, n;
};
constexpr int kMaxPackJobs = 8 * 6 + 1;
struct PackJobs {
  PackJob job[kMaxPackJobs];
  int count;
};

__global__ void pack_weights_kernel(const float* __restrict__ params, __nv_bfloat16* __restrict__ packed,
                                    const __grid_constant__ PackJobs jobs) {
  const PackJob j = jobs.job[blockIdx.y];
  for (int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 4; i < j.n; i += (int64_t)gridDim.x * blockDim.x * 4) {
    const float4 v = *reinterpret_cast<const float4*>(params + j.src + i);
    *reinterpret_cast<uint2*>(packed + j.dst + i) = make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
  }
}

PackJobs make_pack_jobs() {
  const ParamLayout L = make_param_layout();
  PackJobs jobs{};
  auto add = [&](uint32_t tid, int64_t dst) {
    jobs.job[jobs.count++] = PackJob{L.offset[tid], dst, (int64_t)L.rows[tid] * L.cols[tid]};
  };
  for (int l = 0; l < kLayers; ++l) {
    const int64_t b = l * kPackLayer;
    add(tid_q(l), b + kPackQkv);
    add(tid_k(l), b + kPackQkv + kWidth * kWidth);
    add(tid_v(l), b + kPackQkv + 2 * kWidth * kWidth);
    add(tid_proj(l), b + kPackProj);
    add(tid_fc(l), b + kPackFc);
    add(tid_mlp(l), b + kPackMlp);
  }
  add(kTidHead, kPackHead);
  return jobs;
}

// ------------------------------------------------------------------------------------------------
// workspace
// ------------------------------------------------------------------------------------------------
struct PopWorkspace {
  float* x;
  __nv_bfloat16* xb;
  __nv_bfloat16* qkv;
  __nv_bfloat16* y;
  __nv_bfloat16* hidden;
  float* st_a;
  float* st_b;
  float* ystats;
  float* hstats;
  float* inv0;
  float* part;
  __nv_bfloat16* rope_bf16;  // [T][64] cos | sin as bf16 (the QKV epilogue's staged rotary rows)
  float* draws;              // [slots][kDrawPerSlot] the chunk's draw table
};

// bytes per row of each buffer, in carve order
static const size_t kRowBytes[] = {
    kWidth * 4, kWidth * 2, 3 * kWidth * 2, kWidth * 2, kHidden * 2, kStatParts * kStatStride * 4, 2 * 2 * 4,
    kHeads * 4, 2 * 4, 4, 4 * 4};

constexpr int kMaxT = 20480;
constexpr size_t kRopeBf16Bytes = (size_t)kMaxT * kHeadDim * 2;

// Draw-table slots a workspace for `rows` rows holds: a chunk of m members spans at most m / 2 + 1
// directions and has at least 128 rows per member.
int64_t draw_capacity(int64_t rows) {
  const int64_t cap = rows / 256 + 2;
  return cap < kDrawMaxSlots ? cap : kDrawMaxSlots;
}

size_t pop_workspace_bytes(int64_t rows) {
  size_t total = kRopeBf16Bytes + ((draw_capacity(rows) * kDrawPerSlot * 4 + 255) / 256) * 256;
  for (size_t b : kRowBytes) total += ((b * rows + 255) / 256) * 256;
  return total;
}

PopWorkspace carve(void* ws, int64_t rows) {
  uint8_t* p = reinterpret_cast<uint8_t*>(ws);
  void* out[11];
  for (int i = 0; i < 11; ++i) {
    out[i] = p;
    p += ((kRowBytes[i] * rows + 255) / 256) * 256;
  }
  return PopWorkspace{(float*)out[0], (__nv_bfloat16*)out[1], (__nv_bfloat16*)out[2], (__nv_bfloat16*)out[3],
                      (__nv_bfloat16*)out[4], (float*)out[5], (float*)out[6], (float*)out[7], (float*)out[8],
                      (float*)out[9], (float*)out[10], (__nv_bfloat16*)p, (float*)(p + kRopeBf16Bytes)};
}

// Point a chunk's context at its draw table (filled by draw_table_kernel at the start of the chunk).
void attach_draws(PopCtx& c, const PopWorkspace& w, int members) {
  c.draws = w.draws;
  c.dir_first = (c.member_begin % (2 * (int64_t)c.pairs)) >> 1;
  c.slots = draw_slots(c.member_begin, members, c.pairs);
}

// Block (x, tensor * 2 + vec, slot): float4 x of the vector, the same gauss4 the epilogues used to draw.
__global__ void __launch_bounds__(256) draw_table_kernel(PhiloxKey key, int64_t dir_first, int pairs,
                                                         float* __restrict__ table) {
  const int t = blockIdx.y >> 1, v = blockIdx.y & 1;
  const int blk = blockIdx.x * blockDim.x + threadIdx.x;
  if (blk * 4 >= draw_len(t, v)) return;
  const uint32_t slot = blockIdx.z;
  const uint32_t direction = (uint32_t)((dir_first + slot) % pairs);
  reinterpret_cast<float4*>(table + (size_t)slot * kDrawPerSlot + kDrawTableDev.off[t][v])[blk] =
      gauss4(key, (uint32_t)blk, (uint32_t)t, (uint32_t)v, direction);
}

constexpr int kGemmStages = 3;  // 3 beats 4: the smaller carve-out leaves L1 to the epilogues' table loads

// 64: two query tiles per CTA, 64-key tiles (measured 695 ms per bench step); 128: one query tile,
// 128-key tiles, half the hand-offs per key (parity-tested, measured slower: 923 ms)
constexpr int kAttnKeyTile = 64;

template <int G, int KT, bool kDirect>
int launch_attention_g(const CUtensorMap& tm, const AttnTcParams& ap, int64_t rows, cudaStream_t stream) {
  using L = AttnTcLayout<G, KT>;
  static bool configured = false;
  if (!configured) {
    if (cudaFuncSetAttribute(attention_tc_kernel<G, KT, false, kDirect>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kSmem) !=
        cudaSuccess)
      return kStatusLaunchFailed;
    configured = true;
  }
  dim3 grid(ap.ctx.T / (kAtQ * G), kHeads, (unsigned)(rows / ap.ctx.T));
  LaunchScope scope(kKindAttention, stream);
  attention_tc_kernel<G, KT, false, kDirect><<<grid, L::kThreads, L::kSmem, stream>>>(tm, tm, tm, ap);
  return cudaGetLastError() == cudaSuccess ? kStatusOk : kStatusLaunchFailed;
}

int launch_attention(const PopCtx& ctx, const __nv_bfloat16* qkv, PopWorkspace& w, int64_t rows, int layer,
                     int* status, cudaStream_t stream) {
  CUtensorMap tm;
  if (make_tmap_2d(&tm, qkv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, rows, 3 * kWidth, 3 * kWidth, 64, kHeadDim))
    return kStatusBadArgument;
  AttnTcParams ap{};
  ap.ctx = ctx, ap.y = w.y, ap.ystats = w.ystats, ap.layer = layer, ap.window = layer_window(layer);
  ap.status = status;
  ap.col_q = 0, ap.col_k = kWidth, ap.col_v = 2 * kWidth;
  const int n_qt = ctx.T / kAtQ;  // query tiles per sequence; a CTA takes 2 or 1 of them
  // only block `entry` of a direct rerun adds a draw here (site 'o')
  if (ctx.dir.on && layer == ctx.dir.entry && ((ctx.dir.mask >> kSiteO) & 1u)) {
    if (kAttnKeyTile == 128) return launch_attention_g<1, 128, true>(tm, ap, rows, stream);
    if (n_qt % 2 == 0) return launch_attention_g<2, 64, true>(tm, ap, rows, stream);
    return launch_attention_g<1, 64, true>(tm, ap, rows, stream);
  }
  if (kAttnKeyTile == 128) return launch_attention_g<1, 128, false>(tm, ap, rows, stream);
  if (n_qt % 2 == 0) return launch_attention_g<2, 64, false>(tm, ap, rows, stream);
  return launch_attention_g<1, 64, false>(tm, ap, rows, stream);
}

// Optional copies of the clean forward's intermediates (one member, sigma = 0): what DUST's
// reruns and reassembly need (train/val/run.py:189-209, :244-254).
struct CaptureBufs {
  float* blocks;           // [8][rows][512] block inputs after the x0 mixing
  float* x0;               // [rows][512]
  float* inv0;             // [rows]
  __nv_bfloat16* y;        // [8][rows][512] attention outputs (c_proj inputs)
  float* mid;              // [8][rows][512] residual stream after the attention (c_fc input before its norm)
  __nv_bfloat16* hidden;   // [8][rows][2048] relu^2 hidden (mlp.c_proj inputs; > 0 marks live units)
  float* final_x;          // [rows][512] residual stream after the last block
  float* logits;           // [rows][4096] raw logits before the soft cap
};

// Direct reruns from block `entry`: every draw's attention output of that block is the clean one
// (no site changes its q, k or v), plus the draw at site 'o' when that site is jittered; the rank-1
// statistics of the (unperturbed) projection are zero. Eight columns per thread.
__global__ void __launch_bounds__(256) direct_y_kernel(const __grid_constant__ PopCtx ctx, int layer,
                                                       __nv_bfloat16* __restrict__ y, float* __restrict__ ystats,
                                                       int64_t rows) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * (kWidth / 8)) return;
  const int64_t row = i / (kWidth / 8);
  const int c0 = (int)(i % (kWidth / 8)) * 8;
  const int64_t e = row % ((int64_t)ctx.B * ctx.T);
  const uint4 u = __ldg(reinterpret_cast<const uint4*>(ctx.dir.y_entry + e * kWidth + c0));
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
  float v[8];
#pragma unroll
  for (int k = 0; k < 4; ++k) v[2 * k] = __uint_as_float(w[k] << 16), v[2 * k + 1] = __uint_as_float(w[k] & 0xFFFF0000u);
  const SiteJitter jit = site_jitter(ctx, layer, kSiteO, row, kWidth);
  if (jit.on) {
    const uint32_t pat = pattern_word(ctx.key, ctx.dir.site[kSiteO], jit.r.cycle, (uint32_t)c0 >> 5);
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] += jit.scale * draw_value(jit.r, c0 + k, pat);
  }
  uint4 o;
  o.x = pack_bf16x2(v[0], v[1]), o.y = pack_bf16x2(v[2], v[3]), o.z = pack_bf16x2(v[4], v[5]), o.w = pack_bf16x2(v[6], v[7]);
  *reinterpret_cast<uint4*>(y + row * kWidth + c0) = o;
  if (c0 == 0)  // one thread per row clears the row's per-head statistics
#pragma unroll
    for (int k = 0; k < kHeads; ++k) ystats[row * kHeads + k] = 0.f;
}

// The rotary table's bf16 copy (its values are bf16 already: exact).
__global__ void rope_bf16_kernel(const float* __restrict__ rope, __nv_bfloat16* __restrict__ out, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = __float2bfloat16_rn(rope[i]);
}

int pop_forward_chunk(const float* params, const __nv_bfloat16* packed, const float* rope, const PopCtx& ctx,
                      int members, float* losses, PopWorkspace& w, int* status, cudaStream_t stream,
                      const CaptureBufs* cap = nullptr) {
  static const ParamLayout L = make_param_layout();
  const int64_t rows = (int64_t)members * ctx.B * ctx.T;
  const float* wte = params + L.offset[kTidWte];
  const float* lambdas = params + L.offset[kTidResid];  // resid_lambdas then x0_lambdas, contiguous
  const bool direct = ctx.dir.on != 0;
  const int first = (direct && ctx.dir.entry >= 0) ? ctx.dir.entry : 0;
  auto copy = [&](void* dst, const void* src, size_t bytes) {
    return cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, stream) == cudaSuccess;
  };
  int rc;
  {
    const int n = ctx.T * kHeadDim;
    LaunchScope scope(kKindOther, stream);
    rope_bf16_kernel<<<(n + 255) / 256, 256, 0, stream>>>(rope, w.rope_bf16, n);
  }
  if (ctx.draws != w.draws || ctx.slots <= 0 || ctx.slots > draw_capacity(rows)) return kStatusBadArgument;
  {
    LaunchScope scope(kKindOther, stream);
    const dim3 grid((kVocab / 4 + 255) / 256, 2 * kNumTensors, (unsigned)ctx.slots);
    draw_table_kernel<<<grid, 256, 0, stream>>>(ctx.key, ctx.dir_first, ctx.pairs, w.draws);
    if (cudaGetLastError() != cudaSuccess) return kStatusLaunchFailed;
  }
  CUtensorMap tm_rope;
  if (make_tmap_2d(&tm_rope, w.rope_bf16, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, ctx.T, kHeadDim, kHeadDim, 32, 64))
    return kStatusBadArgument;
  {
    EmbedParams ep{ctx, wte, lambdas, w.x, w.xb, w.inv0, w.st_a, cap ? cap->x0 : nullptr};
    if (first > 0 || (direct && ctx.dir.entry == 0)) {
      LaunchScope scope(kKindEmbed, stream);
      direct_start_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, stream>>>(ep, rows);
    } else {
      LaunchScope scope(kKindEmbed, stream);
      embed_kernel<<<(unsigned)(rows / kEmbedRows), 256, 0, stream>>>(ep);
    }
    if (cudaGetLastError() != cudaSuccess) return kStatusLaunchFailed;
    if (cap && !(copy(cap->inv0, w.inv0, rows * 4) && copy(cap->blocks, w.x, rows * kWidth * 4)))
      return kStatusLaunchFailed;
  }
  for (int l = first; l < kLayers; ++l) {
    const __nv_bfloat16* wl = packed + l * kPackLayer;
    EpiQkv::Params q{{}, tm_rope, status, ctx, w.qkv, w.st_a, has_ve(l) ? params + L.offset[tid_ve(l)] : nullptr, l};
    if (make_tmap_2d(&q.tm_qkv, w.qkv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, rows, 3 * kWidth, 3 * kWidth, 32, 64))
      return kStatusBadArgument;
    if (direct && l == ctx.dir.entry && ctx.dir.y_entry) {
      LaunchScope scope(kKindAttention, stream);
      direct_y_kernel<<<(unsigned)((rows * (kWidth / 8) + 255) / 256), 256, 0, stream>>>(ctx, l, w.y, w.ystats, rows);
      if (cudaGetLastError() != cudaSuccess) return kStatusLaunchFailed;
    } else {
      if ((rc = launch_gemm<EpiQkv, kGemmStages>(w.xb, wl + kPackQkv, (int)rows, 3 * kWidth, kWidth, kWidth, kWidth,
                                                    q, status, stream, kKindQkv)))
        return rc;
      if ((rc = launch_attention(ctx, w.qkv, w, rows, l, status, stream))) return rc;
    }
    if (cap && !copy(cap->y + (size_t)l * rows * kWidth, w.y, rows * kWidth * 2)) return kStatusLaunchFailed;
    EpiProj::Params pp{{}, status, ctx, w.x, w.xb, w.ystats, w.st_b, l};
    if (make_tmap_2d(&pp.tm_x, w.x, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, rows, kWidth, kWidth, 32, 32))
      return kStatusBadArgument;
    if ((rc = launch_gemm<EpiProj, kGemmStages>(w.y, wl + kPackProj, (int)rows, kWidth, kWidth, kWidth, kWidth, pp,
                                                   status, stream, kKindProj)))
      return rc;
    if (cap && !copy(cap->mid + (size_t)l * rows * kWidth, w.x, rows * kWidth * 4)) return kStatusLaunchFailed;
    EpiFc::Params fp{{}, ctx, w.hidden, w.st_b, w.hstats, l};
    if (make_tmap_2d(&fp.tm_hidden, w.hidden, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, rows, kHidden, kHidden, 32, 64))
      return kStatusBadArgument;
    if ((rc = launch_gemm<EpiFc, kGemmStages>(w.xb, wl + kPackFc, (int)rows, kHidden, kWidth, kWidth, kWidth, fp,
                                                 status, stream, kKindFc)))
      return rc;
    if (cap && !copy(cap->hidden + (size_t)l * rows * kHidden, w.hidden, rows * kHidden * 2)) return kStatusLaunchFailed;
    const float* wg_next = (l + 1 < kLayers && has_ve(l + 1)) ? params + L.offset[tid_gate(l + 1)] : nullptr;
    // after the last block: the capture keeps the fp32 final stream; a direct rerun's fp32 head reads it
    // from the residual buffer itself
    float* x_final = l == kLayers - 1 ? (cap ? cap->final_x : direct ? w.x : nullptr) : nullptr;
    EpiMlpOut::Params mp{ctx, w.x, w.xb, w.hstats, w.st_a, wte, w.inv0, lambdas, wg_next, x_final, l};
    // the direct instantiation where this block adds a draw: site 'mlp' of block `entry`, or the
    // embedding draw inside x0 in every block of a rerun from the embedding
    const bool jitter_here = direct && (l == ctx.dir.entry || ctx.dir.entry < 0);
    rc = jitter_here ? launch_gemm<EpiMlpOutDirect, kGemmStages>(w.hidden, wl + kPackMlp, (int)rows, kWidth, kHidden,
                                                            kHidden, kHidden, mp, status, stream, kKindMlp)
                : launch_gemm<EpiMlpOut, kGemmStages>(w.hidden, wl + kPackMlp, (int)rows, kWidth, kHidden, kHidden,
                                                      kHidden, mp, status, stream, kKindMlp);
    if (rc) return rc;
    if (cap && l + 1 < kLayers && !copy(cap->blocks + (size_t)(l + 1) * rows * kWidth, w.x, rows * kWidth * 4))
      return kStatusLaunchFailed;
  }
  EpiHead::Params hp{ctx, w.st_a, w.part, cap ? cap->logits : nullptr};
  // direct reruns: fp32 operands (the final stream and the lm_head master) on kind::tf32, as the
  // reference's float32 rerun head (train/val/run.py:272-278); the population forward and the capture
  // keep the autocast head on bf16 operands
  rc = direct ? launch_gemm<EpiHeadF32, kGemmStages>(w.x, params + L.offset[kTidHead], (int)rows, kVocab, kWidth,
                                                      kWidth, kWidth, hp, status, stream, kKindHead)
              : launch_gemm<EpiHead, kGemmStages>(w.xb, packed + kPackHead, (int)rows, kVocab, kWidth, kWidth, kWidth,
                                                  hp, status, stream, kKindHead);
  if (rc) return rc;
  {
    LaunchScope scope(kKindLoss, stream);
    if (direct || cap)
      token_loss_kernel<<<(unsigned)((rows + 255) / 256), 256, 0, stream>>>(
          w.part, ctx.targets, rows, (int64_t)ctx.B * ctx.T, direct ? ctx.dir.token_loss : losses);
    else
      member_loss_kernel<<<members, 256, 0, stream>>>(w.part, (int64_t)ctx.B * ctx.T, losses);
  }
  return cudaGetLastError() == cudaSuccess ? kStatusOk : kStatusLaunchFailed;
}

int check_pop_shape(int B, int T, int members) {
  if (B <= 0 || T <= 0 || T % kAtQ || ((int64_t)B * T) % 128 || members <= 0 || T > kMaxT) return kStatusBadArgument;
  return kStatusOk;
}

int pop_chunk_members(int64_t rows_per_member, int members, int pairs, size_t workspace_bytes) {
  int chunk = members;
  while (chunk > 0 && pop_workspace_bytes(rows_per_member * chunk) > workspace_bytes) --chunk;
  // the chunk's directions fit the draw table (at most chunk / 2 + 1 of them, and at most P)
  while (chunk > 0 && draw_slots(1, chunk, pairs) > draw_capacity(rows_per_member * chunk)) --chunk;
  while (chunk > 0 && (int64_t)chunk * rows_per_member > (int64_t)1 << 30) --chunk;  // int32 GEMM row indices
  if (chunk == 0) return 0;
  // as many chunks as the largest fitting one needs, of equal size: no short tail chunk
  const int n = (members + chunk - 1) / chunk;
  return (members + n - 1) / n;
}

}  // namespace noise

using namespace noise;

extern "C" size_t noise_pop_workspace_bytes(int64_t rows) { return pop_workspace_bytes(rows); }

extern "C" int noise_pop_chunk_members(int64_t rows_per_member, int members, int pairs, size_t workspace_bytes) {
  if (rows_per_member <= 0 || members <= 0 || pairs <= 0) return 0;
  return pop_chunk_members(rows_per_member, members, pairs, workspace_bytes);
}

extern "C" int64_t noise_param_count(void) { return make_param_layout().total; }

extern "C" int64_t noise_packed_count(void) { return kPackTotal; }

extern "C" int noise_pack_weights(const float* params, void* packed, void* stream) {
  static const PackJobs jobs = make_pack_jobs();
  dim3 grid(64, jobs.count);
  LaunchScope scope(kKindPack, reinterpret_cast<cudaStream_t>(stream));
  pack_weights_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      params, reinterpret_cast<__nv_bfloat16*>(packed), jobs);
  return cudaGetLastError() == cudaSuccess ? kStatusOk : kStatusLaunchFailed;
}

extern "C" int noise_pop_forward_lowrank(const float* params, const void* packed, const float* rope,
                                         const int32_t* tokens, const int32_t* targets, int B, int T,
                                         int64_t member_begin, int members, int pairs, float sigma, uint32_t seed,
                                         uint32_t step, float* losses, void* workspace, size_t workspace_bytes,
                                         int* status, void* stream) {
  if (!params || !packed || !rope || !tokens || !targets || !losses || !workspace) return kStatusBadArgument;
  if (check_pop_shape(B, T, members) || pairs <= 0 || member_begin < 0) return kStatusBadArgument;
  const int64_t rows_per_member = (int64_t)B * T;
  const int chunk = pop_chunk_members(rows_per_member, members, pairs, workspace_bytes);
  if (chunk == 0) return kStatusWorkspaceTooSmall;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  for (int m0 = 0; m0 < members; m0 += chunk) {
    const int mc = members - m0 < chunk ? members - m0 : chunk;
    PopCtx ctx{tokens, targets, T, B, member_begin + m0, pairs, sigma, PhiloxKey{seed, step}, DirectSpec{}};
    PopWorkspace w = carve(workspace, rows_per_member * mc);
    attach_draws(ctx, w, mc);
    const int rc = pop_forward_chunk(params, reinterpret_cast<const __nv_bfloat16*>(packed), rope, ctx, mc,
                                     losses + m0, w, status, s);
    if (rc) return rc;
  }
  return kStatusOk;
}

extern "C" int noise_pop_forward_direct(const float* params, const void* packed, const float* rope,
                                        const int32_t* tokens, const int32_t* targets, int B, int T,
                                        int64_t draw_begin, int draws, const NoiseDirect* spec, uint32_t seed,
                                        uint32_t step, float* token_loss, void* workspace, size_t workspace_bytes,
                                        int* status, void* stream) {
  if (!params || !packed || !rope || !tokens || !targets || !token_loss || !workspace || !spec) return kStatusBadArgument;
  if (check_pop_shape(B, T, draws) || draw_begin < 0) return kStatusBadArgument;
  if (spec->entry < -1 || spec->entry >= kLayers || (spec->mask >> kSiteKinds)) return kStatusBadArgument;
  if (spec->entry == -1 && spec->mask != (1u << kSiteWte) && spec->mask != 0) return kStatusBadArgument;
  if (spec->entry >= 0 && spec->mask == 0) return kStatusBadArgument;
  if (spec->entry >= 0 && ((spec->mask & 1u) || !spec->x_entry || !spec->inv0)) return kStatusBadArgument;
  if (((spec->mask >> kSiteFc) & 1u) && !spec->live) return kStatusBadArgument;
  const int64_t rows_per_member = (int64_t)B * T;
  const int chunk = pop_chunk_members(rows_per_member, draws, 1, workspace_bytes);
  if (chunk == 0) return kStatusWorkspaceTooSmall;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  for (int m0 = 0; m0 < draws; m0 += chunk) {
    const int mc = draws - m0 < chunk ? draws - m0 : chunk;
    DirectSpec d{};
    d.on = 1;
    d.entry = spec->entry;
    d.mask = spec->mask;
    for (int k = 0; k < kSiteKinds; ++k) d.site[k] = spec->site[k];
    d.sigma = spec->sigma;
    d.x_entry = spec->x_entry;
    d.inv0 = spec->inv0;
    d.live = reinterpret_cast<const __nv_bfloat16*>(spec->live);
    d.y_entry = spec->entry >= 0 ? reinterpret_cast<const __nv_bfloat16*>(spec->y_entry) : nullptr;
    d.token_loss = token_loss + m0 * rows_per_member;
    PopCtx ctx{tokens, targets, T, B, draw_begin + m0, 1, 0.0f, PhiloxKey{seed, step}, d};
    PopWorkspace w = carve(workspace, rows_per_member * mc);
    attach_draws(ctx, w, mc);
    const int rc = pop_forward_chunk(params, reinterpret_cast<const __nv_bfloat16*>(packed), rope, ctx, mc, nullptr,
                                     w, status, s);
    if (rc) return rc;
  }
  return kStatusOk;
}

extern "C" int noise_pop_capture(const float* params, const void* packed, const float* rope, const int32_t* tokens,
                                 const int32_t* targets, int B, int T, const NoiseCapture* out, void* workspace,
                                 size_t workspace_bytes, int* status, void* stream) {
  if (!params || !packed || !rope || !tokens || !targets || !out || !workspace) return kStatusBadArgument;
  if (!out->blocks || !out->x0 || !out->inv0 || !out->y || !out->mid || !out->hidden || !out->final_x ||
      !out->logits || !out->token_loss)
    return kStatusBadArgument;
  if (check_pop_shape(B, T, 1)) return kStatusBadArgument;
  const int64_t rows = (int64_t)B * T;
  if (pop_workspace_bytes(rows) > workspace_bytes) return kStatusWorkspaceTooSmall;
  CaptureBufs cap{out->blocks, out->x0, out->inv0, reinterpret_cast<__nv_bfloat16*>(out->y), out->mid,
                  reinterpret_cast<__nv_bfloat16*>(out->hidden), out->final_x, out->logits};
  PopCtx ctx{tokens, targets, T, B, 0, 1, 0.0f, PhiloxKey{0, 0}, DirectSpec{}};
  PopWorkspace w = carve(workspace, rows);
  attach_draws(ctx, w, 1);
  return pop_forward_chunk(params, reinterpret_cast<const __nv_bfloat16*>(packed), rope, ctx, 1, out->token_loss, w,
                           status, reinterpret_cast<cudaStream_t>(stream), &cap);
}
