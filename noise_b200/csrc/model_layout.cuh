// The fixed model's shapes, the flat parameter layout and the draw-stream tensor ids.
//
// Master parameters are one fp32 buffer in `GPT.named_parameters()` order (utils/model.py:123-147:
// resid_lambdas, x0_lambdas, transformer.wte, blocks h.0..h.7 as c_q, c_k, c_v, c_proj, [ve_gate],
// c_fc, mlp.c_proj, then lm_head and value_embeds.{1,3,5,7}); the index of a parameter in that order
// is its draw-stream tensor id. The GEMMs read a packed bf16 copy of the matrices:
//   per layer: [c_q; c_k; c_v] (1536 x 512) | c_proj (512 x 512) | c_fc (2048 x 512) | mlp.c_proj (512 x 2048)
//   then lm_head (4096 x 512).
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

#include "dust.cuh"
#include "philox.cuh"

namespace noise {

constexpr int kLayers = 8, kWidth = 512, kVocab = 4096, kHidden = 2048, kHeads = 8, kHeadDim = 64;
constexpr int kGateChannels = 32;
constexpr float kSoftCap = 15.0f;
constexpr float kNormEps = 1.1920928955078125e-07f;  // float32 epsilon, F.rms_norm's default

__host__ __device__ constexpr bool has_ve(int layer) { return (layer & 1) == 1; }  // utils/model.py:50-52
__host__ __device__ constexpr int layer_window(int layer) { return (layer % 4 == 3 || layer == kLayers - 1) ? 2048 : 1024; }

// draw-stream tensor ids (= index in named_parameters order)
constexpr uint32_t kTidResid = 0, kTidX0 = 1, kTidWte = 2, kTidHead = 55;
__host__ __device__ constexpr uint32_t tid_base(int layer) { return 3 + 6 * layer + layer / 2; }
__host__ __device__ constexpr uint32_t tid_q(int l) { return tid_base(l); }
__host__ __device__ constexpr uint32_t tid_k(int l) { return tid_base(l) + 1; }
__host__ __device__ constexpr uint32_t tid_v(int l) { return tid_base(l) + 2; }
__host__ __device__ constexpr uint32_t tid_proj(int l) { return tid_base(l) + 3; }
__host__ __device__ constexpr uint32_t tid_gate(int l) { return tid_base(l) + 4; }
__host__ __device__ constexpr uint32_t tid_fc(int l) { return tid_base(l) + 4 + (has_ve(l) ? 1 : 0); }
__host__ __device__ constexpr uint32_t tid_mlp(int l) { return tid_base(l) + 5 + (has_ve(l) ? 1 : 0); }
__host__ __device__ constexpr uint32_t tid_ve(int l) { return 56 + l / 2; }
constexpr int kNumTensors = 60;

// Offsets (in floats) of every tensor in the flat master buffer.
struct ParamLayout {
  int64_t offset[kNumTensors];
  int rows[kNumTensors];
  int cols[kNumTensors];  // 1 for vectors
  int64_t total;
};

inline ParamLayout make_param_layout() {
  ParamLayout L{};
  int n = 0;
  auto add = [&](int r, int c) {
    L.rows[n] = r;
    L.cols[n] = c;
    ++n;
  };
  add(kLayers, 1);
  add(kLayers, 1);
  add(kVocab, kWidth);
  for (int l = 0; l < kLayers; ++l) {
    add(kWidth, kWidth);
    add(kWidth, kWidth);
    add(kWidth, kWidth);
    add(kWidth, kWidth);
    if (has_ve(l)) add(kHeads, kGateChannels);
    add(kHidden, kWidth);
    add(kWidth, kHidden);
  }
  add(kVocab, kWidth);
  for (int l = 1; l < kLayers; l += 2) add(kVocab, kWidth);
  int64_t off = 0;
  for (int i = 0; i < n; ++i) {
    L.offset[i] = off;
    off += (int64_t)L.rows[i] * L.cols[i];
  }
  L.total = off;
  return L;
}

// packed bf16 GEMM weights
constexpr int64_t kPackQkv = 0;
constexpr int64_t kPackProj = 3 * kWidth * kWidth;
constexpr int64_t kPackFc = kPackProj + kWidth * kWidth;
constexpr int64_t kPackMlp = kPackFc + (int64_t)kHidden * kWidth;
constexpr int64_t kPackLayer = kPackMlp + (int64_t)kWidth * kHidden;
constexpr int64_t kPackHead = kLayers * kPackLayer;
constexpr int64_t kPackTotal = kPackHead + (int64_t)kVocab * kWidth;

// Direct-draw (DUST rerun) mode: weights unperturbed, member j of the call is draw
// member_begin + j, rerun from block `entry` (-1: from the embedding) with the orthogonal draws
// of the sites in `mask` added in that block (train/val/run.py:256-279, block_forward :102-117).
struct DirectSpec {
  int on;
  int entry;
  uint32_t mask;                  // bits kSiteWte, kSiteO, kSiteAttn, kSiteFc, kSiteMlp
  uint32_t site[kSiteKinds];      // stream site id per site kind
  float sigma;                    // jitter scale (the draws are +-1)
  const float* x_entry;           // [B*T, 512] clean input of block `entry` (entry >= 0)
  const float* inv0;              // [B*T] clean 1/rms of the embedding rows (entry >= 0)
  const __nv_bfloat16* live;      // [B*T, 2048] clean relu^2 hidden of block `entry`: > 0 marks live units
  const __nv_bfloat16* y_entry;   // [B*T, 512] clean attention output of block `entry`, or nullptr
  float* token_loss;              // [members, B, T] per-token cross-entropy
};

// Everything a kernel needs to place a row of the population batch: rows are ordered
// (member, sequence, token), member j = member_begin + row / (B * T).
struct PopCtx {
  const int* tokens;   // [B, T] input ids
  const int* targets;  // [B, T] next-token ids
  int T, B;
  int64_t member_begin;
  int pairs;           // antithetic directions P: member j uses direction (j mod 2P) / 2
  float sigma;         // member j perturbs by +sigma (even j) or -sigma (odd j); 0 in direct mode
  PhiloxKey key;
  DirectSpec dir;
  // The chunk's draw table (see DrawTable): slot s holds direction (dir_first + s) mod P.
  const float* draws = nullptr;
  int64_t dir_first = 0;
  int slots = 0;
};

// ---------------------------------------------------------------------------------------------
// Draw table. Every rank-1 draw vector a (vec 0, length out) and b (vec 1, length in) of every
// tensor depends only on (key, tensor, vec, direction), yet the GEMM epilogues need the same
// 128-column slices for every 128-row tile of a member. One kernel per chunk writes each direction's
// vectors once (gauss4 of the same counters, so the values are identical) and the epilogues load
// them: [slot][tensor][vec][len], lengths padded to 4 floats.
// ---------------------------------------------------------------------------------------------
__host__ __device__ constexpr int draw_len(int t, int v) {
  if (t == (int)kTidResid || t == (int)kTidX0) return v ? 4 : kLayers;
  if (t == (int)kTidWte || t == (int)kTidHead || t >= (int)tid_ve(0)) return v ? kWidth : kVocab;  // by token
  for (int l = 0; l < kLayers; ++l) {
    const int k = t - (int)tid_base(l);
    if (k < 0 || k > (has_ve(l) ? 6 : 5)) continue;
    if (k < 4) return kWidth;                                       // c_q, c_k, c_v, c_proj
    if (has_ve(l) && k == 4) return v ? kGateChannels : kHeads;     // ve_gate [8, 32]
    const bool fc = k == (has_ve(l) ? 5 : 4);
    return fc ? (v ? kWidth : kHidden) : (v ? kHidden : kWidth);   // c_fc [2048, 512], mlp.c_proj [512, 2048]
  }
  return 0;
}

struct DrawTable {
  int32_t off[kNumTensors][2];
  int32_t per_slot;
};

__host__ __device__ constexpr DrawTable make_draw_table() {
  DrawTable d{};
  int32_t o = 0;
  for (int t = 0; t < kNumTensors; ++t)
    for (int v = 0; v < 2; ++v) {
      d.off[t][v] = o;
      o += draw_len(t, v);
    }
  d.per_slot = o;
  return d;
}

__host__ __device__ constexpr bool draw_lengths_aligned() {
  for (int t = 0; t < kNumTensors; ++t)
    if (draw_len(t, 0) % 4 || draw_len(t, 1) % 4 || draw_len(t, 0) == 0) return false;
  return true;
}
static_assert(draw_lengths_aligned(), "draw vectors are read as float4 and every tensor has one");

constexpr int kDrawPerSlot = make_draw_table().per_slot;  // floats per direction
static_assert(kDrawPerSlot == 101560, "the documented draw-table size (406,240 B per direction)");
constexpr int kDrawMaxSlots = 512;                        // directions one chunk may span
static __constant__ DrawTable kDrawTableDev = make_draw_table();

// Slots a chunk of `members` members starting at member_begin spans.
__host__ __device__ inline int draw_slots(int64_t member_begin, int members, int pairs) {
  const int span = (int)((members + (member_begin & 1) + 1) / 2);
  return span < pairs ? span : pairs;
}

__device__ __forceinline__ const float* draw_ptr(const PopCtx& c, uint32_t slot, uint32_t tensor, uint32_t vec) {
  return c.draws + (size_t)slot * kDrawPerSlot + kDrawTableDev.off[tensor][vec];
}

// element i of draw vector (tensor, vec) of a slot; four elements from 4 * blk
__device__ __forceinline__ float draw1(const PopCtx& c, uint32_t slot, uint32_t tensor, uint32_t vec, uint32_t i) {
  return __ldg(draw_ptr(c, slot, tensor, vec) + i);
}
__device__ __forceinline__ float4 draw4(const PopCtx& c, uint32_t slot, uint32_t tensor, uint32_t vec, uint32_t blk) {
  return __ldg(reinterpret_cast<const float4*>(draw_ptr(c, slot, tensor, vec)) + blk);
}

// Jitter of a direct-mode site in one row: the draw's Hadamard row and sign, and scale.
struct SiteJitter {
  bool on;
  DrawRow r;
  float scale;
};

__device__ __forceinline__ SiteJitter site_jitter(const PopCtx& c, int layer, uint32_t kind, int64_t row,
                                                  uint32_t d) {
  SiteJitter j;
  j.on = c.dir.on && layer == c.dir.entry && ((c.dir.mask >> kind) & 1u);
  j.scale = c.dir.sigma;
  if (j.on) {
    const int64_t seq_rows = (int64_t)c.B * c.T;
    const uint32_t idx = (uint32_t)(c.member_begin + row / seq_rows);
    j.r = draw_row(c.key, c.dir.site[kind], idx, (uint32_t)(row % seq_rows), d);
  }
  return j;
}

// The 4 pattern words of columns [c0, c0 + 128) (c0 % 128 == 0) for the row's draw cycle.
__device__ __forceinline__ void site_patterns(const PopCtx& c, uint32_t kind, const DrawRow& r, uint32_t c0,
                                              uint32_t (&w)[4]) {
  uint32_t x[4];
  philox4x32_10(c0 >> 7, (c.dir.site[kind] << 2) | 1u, r.cycle, kDomainDirect, c.key.k0, c.key.k1, x);
  w[0] = x[0], w[1] = x[1], w[2] = x[2], w[3] = x[3];
}

struct RowInfo {
  uint32_t direction;
  uint32_t slot;  // the direction's slot in the chunk's draw table
  float sign;
  int t;    // position in the sequence
  int tok;  // input token id
  int tgt;  // target id
};

__device__ __forceinline__ RowInfo row_info(const PopCtx& c, int64_t row) {
  RowInfo r;
  const int64_t seq_rows = (int64_t)c.B * c.T;
  const int64_t j = c.member_begin + row / seq_rows;
  const int64_t within = row % seq_rows;
  r.direction = (uint32_t)((j % (2 * (int64_t)c.pairs)) >> 1);
  const int64_t s = (int64_t)r.direction - c.dir_first;
  r.slot = (uint32_t)(s < 0 ? s + c.pairs : s);
  r.sign = (j & 1) ? -c.sigma : c.sigma;
  r.t = (int)(within % c.T);
  r.tok = __ldg(c.tokens + within);
  r.tgt = __ldg(c.targets + within);
  return r;
}

// Fill dst[0..127] (per-warp shared memory) with elements e0 .. e0+127 of draw vector (tensor, vec)
// of a slot of the draw table; e0 % 4 == 0. Caller brackets with __syncwarp().
__device__ __forceinline__ void warp_draw128(float* dst, const PopCtx& c, uint32_t slot, uint32_t tensor, uint32_t vec,
                                             uint32_t e0, int lane) {
  reinterpret_cast<float4*>(dst)[lane] = draw4(c, slot, tensor, vec, (e0 >> 2) + lane);
}

}  // namespace noise
