// Epilogues of the population GEMMs. Each one finishes a perturbed linear layer of
// `population_loss` (train/val/eggroll.py:66-103) on a 64-column group of one accumulator row:
//
//   y = s * (x W^T + s_m (x b_m) a_m^T)        (train/val/eggroll.py:56-58, lowrank)
//
// where the row scale s is the RMS-norm of the layer input (applied here instead of on the operand:
// norm(x) W^T = (x W^T) / rms(x)), s_m = +-sigma is the member's sign, and x . b_m is a per-row scalar
// that the *producer* of x computed as a side statistic, so the GEMM itself is the plain shared-weight
// product. a_m is regenerated from the counter-based stream into per-warp shared memory.
//
// Row statistics travel between kernels as two partial sums per row, `float [rows][2][16]`:
//   stats for a QKV / head input x:  [0] sum x^2, [1..3] x.b_q, x.b_k, x.b_v (or [1] x.b_head),
//                                     [4] x[:32].b_gate, [5..12] x[:32].W_gate^T (value-embedding layers)
//   stats for an FC input x:         [0] sum x^2, [1] x.b_fc
// Dot products use the bf16 values the next GEMM reads; sums of squares use the fp32 stream.
#pragma once

#include "gemm_tc.cuh"
#include "model_layout.cuh"

namespace noise {

constexpr int kStatStride = 16;  // floats per partial

__device__ __forceinline__ float rms_scale(float ssq, int n) { return rsqrtf(ssq / (float)n + kNormEps); }

// Per-warp vector slots in the epilogue's shared memory.
constexpr int kWarpVecs = 6;
constexpr int kEpiVecBytes = 8 * kWarpVecs * 128 * 4;

// ---------------------------------------------------------------------------------------------
// QKV: q, k through RoPE and a per-head RMS norm; v plus the gated value embedding.
// ---------------------------------------------------------------------------------------------
struct EpiQkv {
  struct Params {
    PopCtx ctx;
    __nv_bfloat16* qkv;     // [rows, 1536]
    const float* stats;     // [rows][2][16]
    const float* rope;      // [T][64]: cos[0..31] | sin[0..31]
    const float* ve_table;  // [4096, 512] or nullptr
    int layer;
  };
  static constexpr int kSmemBytes = kEpiVecBytes;
  const Params& p;
  float* vec;  // this warp's slots: [0] a of the tile's tensor, [1] b_ve
  int lane;
  RowInfo ri;
  float inv, xb[3], gate[kHeads], a_ve_tok;

  __device__ EpiQkv(const Params& p_, uint8_t* smem, int ew, int lane_)
      : p(p_), vec(reinterpret_cast<float*>(smem) + ew * kWarpVecs * 128), lane(lane_) {}

  __device__ void begin_mtile(int, int row) {
    ri = row_info(p.ctx, row);
    const float* s0 = p.stats + (size_t)row * 2 * kStatStride;
    const float* s1 = s0 + kStatStride;
    inv = rms_scale(s0[0] + s1[0], kWidth);
#pragma unroll
    for (int i = 0; i < 3; ++i) xb[i] = s0[1 + i] + s1[1 + i];
    if (has_ve(p.layer)) {
      const float xg = s0[4] + s1[4];
      const float4 ag0 = gauss4(p.ctx.key, 0, tid_gate(p.layer), 0, ri.direction);
      const float4 ag1 = gauss4(p.ctx.key, 1, tid_gate(p.layer), 0, ri.direction);
      const float ag[8] = {ag0.x, ag0.y, ag0.z, ag0.w, ag1.x, ag1.y, ag1.z, ag1.w};
#pragma unroll
      for (int h = 0; h < kHeads; ++h) {
        const float pre = inv * (s0[5 + h] + s1[5 + h] + ri.sign * xg * ag[h]);
        gate[h] = 2.0f / (1.0f + expf(-pre));
      }
      a_ve_tok = gauss1(p.ctx.key, ri.tok, tid_ve(p.layer), 0, ri.direction);
    }
  }

  __device__ void begin_tile(int m_tile, int, int col0) {
    // all rows of an M tile belong to one member
    const RowInfo r0 = row_info(p.ctx, (int64_t)m_tile * 128);
    const int which = col0 / kWidth, local = col0 % kWidth;
    const uint32_t tid = which == 0 ? tid_q(p.layer) : which == 1 ? tid_k(p.layer) : tid_v(p.layer);
    __syncwarp();
    warp_gauss128(vec, p.ctx.key, tid, 0, r0.direction, local, lane);
    if (which == 2 && has_ve(p.layer)) warp_gauss128(vec + 128, p.ctx.key, tid_ve(p.layer), 1, r0.direction, local, lane);
    __syncwarp();
  }

  __device__ void group(int row, int col, float (&v)[64]) {
    const int which = col / kWidth, local = col % kWidth, head = local / kHeadDim;
    const float* a = vec + (local & 127);
    const float c2 = ri.sign * xb[which];
    __nv_bfloat16* out = p.qkv + (size_t)row * (3 * kWidth) + col;
#pragma unroll
    for (int j = 0; j < 64; ++j) v[j] = inv * (v[j] + c2 * a[j]);
    if (which < 2) {
      const float4* cs = reinterpret_cast<const float4*>(p.rope + (size_t)ri.t * 64);
      float cr[32], sr[32];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float4 c4 = __ldg(cs + j), s4 = __ldg(cs + 8 + j);
        cr[4 * j] = c4.x, cr[4 * j + 1] = c4.y, cr[4 * j + 2] = c4.z, cr[4 * j + 3] = c4.w;
        sr[4 * j] = s4.x, sr[4 * j + 1] = s4.y, sr[4 * j + 2] = s4.z, sr[4 * j + 3] = s4.w;
      }
      float ss = 0.f;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float c = cr[j], s = sr[j];
        const float x1 = v[j], x2 = v[j + 32];
        v[j] = x1 * c + x2 * s;
        v[j + 32] = x2 * c - x1 * s;
        ss += v[j] * v[j] + v[j + 32] * v[j + 32];
      }
      const float r = rms_scale(ss, kHeadDim);
#pragma unroll
      for (int j = 0; j < 64; ++j) v[j] *= r;
    } else if (has_ve(p.layer)) {
      const float* ve = p.ve_table + (size_t)ri.tok * kWidth + local;
      const float* bve = vec + 128 + (local & 127);
      const float g = gate[head], sa = ri.sign * a_ve_tok;
#pragma unroll
      for (int j = 0; j < 64; j += 4) {
        const float4 e = __ldg(reinterpret_cast<const float4*>(ve + j));
        v[j] += g * (e.x + sa * bve[j]);
        v[j + 1] += g * (e.y + sa * bve[j + 1]);
        v[j + 2] += g * (e.z + sa * bve[j + 2]);
        v[j + 3] += g * (e.w + sa * bve[j + 3]);
      }
    }
#pragma unroll
    for (int j = 0; j < 64; j += 8)
      st_global_v4(out + j, pack_bf16x2(v[j], v[j + 1]), pack_bf16x2(v[j + 2], v[j + 3]),
                   pack_bf16x2(v[j + 4], v[j + 5]), pack_bf16x2(v[j + 6], v[j + 7]));
  }

  __device__ void end_mtile(int, int) {}
};

// ---------------------------------------------------------------------------------------------
// attention projection + residual: x += y Wp^T + s (y.b_p) a_p; emits the FC input and its stats.
// ---------------------------------------------------------------------------------------------
struct EpiProj {
  struct Params {
    PopCtx ctx;
    float* x;                // [rows, 512] fp32 residual stream, updated in place
    __nv_bfloat16* xb;       // [rows, 512] bf16 copy for the FC GEMM
    const float* ystats;     // [rows][8] per-head y.b_proj from the attention kernel
    float* stats_out;        // [rows][2][16]: sum x^2, x.b_fc
    int layer;
  };
  static constexpr int kSmemBytes = kEpiVecBytes;
  const Params& p;
  float* vec;  // [0] a_proj, [1] b_fc
  int lane, half;
  RowInfo ri;
  float c2, ssq, dfc;

  __device__ EpiProj(const Params& p_, uint8_t* smem, int ew, int lane_)
      : p(p_), vec(reinterpret_cast<float*>(smem) + ew * kWarpVecs * 128), lane(lane_), half(ew >> 2) {}

  __device__ void begin_mtile(int, int row) {
    ri = row_info(p.ctx, row);
    const float4* ys = reinterpret_cast<const float4*>(p.ystats + (size_t)row * kHeads);
    const float4 y0 = ys[0], y1 = ys[1];
    c2 = ri.sign * (y0.x + y0.y + y0.z + y0.w + y1.x + y1.y + y1.z + y1.w);
    ssq = 0.f;
    dfc = 0.f;
  }

  __device__ void begin_tile(int m_tile, int, int col0) {
    const RowInfo r0 = row_info(p.ctx, (int64_t)m_tile * 128);
    __syncwarp();
    warp_gauss128(vec, p.ctx.key, tid_proj(p.layer), 0, r0.direction, col0, lane);
    warp_gauss128(vec + 128, p.ctx.key, tid_fc(p.layer), 1, r0.direction, col0, lane);
    __syncwarp();
  }

  __device__ void group(int row, int col, float (&v)[64]) {
    const float* a = vec + (col & 127);
    const float* b = vec + 128 + (col & 127);
    float* __restrict__ xr = p.x + (size_t)row * kWidth + col;
    __nv_bfloat16* __restrict__ xo = p.xb + (size_t)row * kWidth + col;
    // all loads of the row segment first, so they are in flight together
    float4 x4[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) x4[j] = reinterpret_cast<const float4*>(xr)[j];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      v[4 * j] += x4[j].x + c2 * a[4 * j];
      v[4 * j + 1] += x4[j].y + c2 * a[4 * j + 1];
      v[4 * j + 2] += x4[j].z + c2 * a[4 * j + 2];
      v[4 * j + 3] += x4[j].w + c2 * a[4 * j + 3];
    }
#pragma unroll
    for (int j = 0; j < 16; ++j)
      reinterpret_cast<float4*>(xr)[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
#pragma unroll
    for (int j = 0; j < 64; ++j) {
      ssq += v[j] * v[j];
      v[j] = bf16_round(v[j]);
      dfc += v[j] * b[j];
    }
#pragma unroll
    for (int j = 0; j < 64; j += 8)
      st_global_v4(xo + j, pack_bf16x2(v[j], v[j + 1]), pack_bf16x2(v[j + 2], v[j + 3]),
                   pack_bf16x2(v[j + 4], v[j + 5]), pack_bf16x2(v[j + 6], v[j + 7]));
  }

  __device__ void end_mtile(int, int row) {
    float* s = p.stats_out + ((size_t)row * 2 + half) * kStatStride;
    s[0] = ssq;
    s[1] = dfc;
  }
};

// ---------------------------------------------------------------------------------------------
// FC: hidden = relu(norm(x) Wfc^T + rank-1)^2 in bf16, plus the hidden.b_mlp statistic.
// ---------------------------------------------------------------------------------------------
struct EpiFc {
  struct Params {
    PopCtx ctx;
    __nv_bfloat16* hidden;  // [rows, 2048]
    const float* stats;     // [rows][2][16] from EpiProj
    float* hstats;          // [rows][2] partial hidden.b_mlp
    int layer;
  };
  static constexpr int kSmemBytes = kEpiVecBytes;
  const Params& p;
  float* vec;  // [0] a_fc, [1] b_mlp
  int lane, half;
  RowInfo ri;
  float inv, c2, dmp;

  __device__ EpiFc(const Params& p_, uint8_t* smem, int ew, int lane_)
      : p(p_), vec(reinterpret_cast<float*>(smem) + ew * kWarpVecs * 128), lane(lane_), half(ew >> 2) {}

  __device__ void begin_mtile(int, int row) {
    ri = row_info(p.ctx, row);
    const float* s0 = p.stats + (size_t)row * 2 * kStatStride;
    const float* s1 = s0 + kStatStride;
    inv = rms_scale(s0[0] + s1[0], kWidth);
    c2 = ri.sign * (s0[1] + s1[1]);
    dmp = 0.f;
  }

  __device__ void begin_tile(int m_tile, int, int col0) {
    const RowInfo r0 = row_info(p.ctx, (int64_t)m_tile * 128);
    __syncwarp();
    warp_gauss128(vec, p.ctx.key, tid_fc(p.layer), 0, r0.direction, col0, lane);
    warp_gauss128(vec + 128, p.ctx.key, tid_mlp(p.layer), 1, r0.direction, col0, lane);
    __syncwarp();
  }

  __device__ void group(int row, int col, float (&v)[64]) {
    const float* a = vec + (col & 127);
    const float* b = vec + 128 + (col & 127);
    __nv_bfloat16* out = p.hidden + (size_t)row * kHidden + col;
#pragma unroll
    for (int j = 0; j < 64; ++j) {
      const float pre = inv * (v[j] + c2 * a[j]);
      const float r = fmaxf(pre, 0.f);
      v[j] = bf16_round(r * r);
      dmp += v[j] * b[j];
    }
#pragma unroll
    for (int j = 0; j < 64; j += 8)
      st_global_v4(out + j, pack_bf16x2(v[j], v[j + 1]), pack_bf16x2(v[j + 2], v[j + 3]),
                   pack_bf16x2(v[j + 4], v[j + 5]), pack_bf16x2(v[j + 6], v[j + 7]));
  }

  __device__ void end_mtile(int, int row) { p.hstats[(size_t)row * 2 + half] = dmp; }
};

// ---------------------------------------------------------------------------------------------
// MLP out + residual, then the next block's x0 mixing (utils/model.py:199) and its input stats;
// after the last block, the head's input and stats.
// ---------------------------------------------------------------------------------------------
struct EpiMlpOut {
  struct Params {
    PopCtx ctx;
    float* x;               // [rows, 512] residual stream, in place
    __nv_bfloat16* xb;      // [rows, 512] next GEMM's operand
    const float* hstats;    // [rows][2]
    float* stats_out;       // [rows][2][16]
    const float* wte;       // [4096, 512] fp32 token embedding (x0 recomputation)
    const float* inv0;      // [rows] 1/rms of the perturbed embedding row
    const float* lambdas;   // resid_lambdas[8] | x0_lambdas[8]
    const float* wgate_next;  // [8, 32] fp32 of the next block, or nullptr
    int layer;
  };
  static constexpr int kSmemBytes = kEpiVecBytes;
  const Params& p;
  float* vec;  // [0] a_mlp, [1] b_wte, [2..4] next b_q, b_k, b_v (or [2] b_head), [5] next b_gate
  int lane, half;
  bool last;
  RowInfo ri;
  float c2, lr, l0, sa_wte, i0, ssq, d[3], dg, gp[kHeads];

  __device__ EpiMlpOut(const Params& p_, uint8_t* smem, int ew, int lane_)
      : p(p_), vec(reinterpret_cast<float*>(smem) + ew * kWarpVecs * 128), lane(lane_), half(ew >> 2),
        last(p_.layer == kLayers - 1) {}

  __device__ void begin_mtile(int, int row) {
    ri = row_info(p.ctx, row);
    c2 = ri.sign * (p.hstats[(size_t)row * 2] + p.hstats[(size_t)row * 2 + 1]);
    ssq = 0.f, d[0] = d[1] = d[2] = 0.f, dg = 0.f;
#pragma unroll
    for (int h = 0; h < kHeads; ++h) gp[h] = 0.f;
    if (!last) {
      const int nl = p.layer + 1;
      lr = p.lambdas[nl] + ri.sign * gauss1(p.ctx.key, nl, kTidResid, 0, ri.direction);
      l0 = p.lambdas[kLayers + nl] + ri.sign * gauss1(p.ctx.key, nl, kTidX0, 0, ri.direction);
      sa_wte = ri.sign * gauss1(p.ctx.key, ri.tok, kTidWte, 0, ri.direction);
      i0 = p.inv0[row];
    }
  }

  __device__ void begin_tile(int m_tile, int, int col0) {
    const RowInfo r0 = row_info(p.ctx, (int64_t)m_tile * 128);
    const uint32_t dir = r0.direction;
    __syncwarp();
    warp_gauss128(vec, p.ctx.key, tid_mlp(p.layer), 0, dir, col0, lane);
    if (!last) {
      const int nl = p.layer + 1;
      warp_gauss128(vec + 128, p.ctx.key, kTidWte, 1, dir, col0, lane);
      warp_gauss128(vec + 256, p.ctx.key, tid_q(nl), 1, dir, col0, lane);
      warp_gauss128(vec + 384, p.ctx.key, tid_k(nl), 1, dir, col0, lane);
      warp_gauss128(vec + 512, p.ctx.key, tid_v(nl), 1, dir, col0, lane);
      if (has_ve(nl) && col0 == 0 && lane < 8)  // b_gate has 32 entries
        reinterpret_cast<float4*>(vec + 640)[lane] = gauss4(p.ctx.key, lane, tid_gate(nl), 1, dir);
    } else {
      warp_gauss128(vec + 256, p.ctx.key, kTidHead, 1, dir, col0, lane);
    }
    __syncwarp();
  }

  __device__ void group(int row, int col, float (&v)[64]) {
    const int c = col & 127;
    const float* a = vec + c;
    float* __restrict__ xr = p.x + (size_t)row * kWidth + col;
    __nv_bfloat16* __restrict__ xo = p.xb + (size_t)row * kWidth + col;
    {
      float4 x4[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) x4[j] = reinterpret_cast<const float4*>(xr)[j];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        v[4 * j] += x4[j].x + c2 * a[4 * j];
        v[4 * j + 1] += x4[j].y + c2 * a[4 * j + 1];
        v[4 * j + 2] += x4[j].z + c2 * a[4 * j + 2];
        v[4 * j + 3] += x4[j].w + c2 * a[4 * j + 3];
      }
    }
    if (!last) {
      const float* bw = vec + 128 + c;
      const float* bq = vec + 256 + c;
      const float* bk = vec + 384 + c;
      const float* bv = vec + 512 + c;
      const float* __restrict__ e = p.wte + (size_t)ri.tok * kWidth + col;
#pragma unroll
      for (int h = 0; h < 64; h += 32) {
        float4 e4[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) e4[j] = __ldg(reinterpret_cast<const float4*>(e + h) + j);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float ev[4] = {e4[j].x, e4[j].y, e4[j].z, e4[j].w};
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int k = h + 4 * j + u;
            const float x0 = (ev[u] + sa_wte * bw[k]) * i0;
            v[k] = lr * v[k] + l0 * x0;
          }
        }
      }
#pragma unroll
      for (int j = 0; j < 16; ++j)
        reinterpret_cast<float4*>(xr)[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
#pragma unroll
      for (int j = 0; j < 64; ++j) {
        ssq += v[j] * v[j];
        v[j] = bf16_round(v[j]);
        d[0] += v[j] * bq[j];
        d[1] += v[j] * bk[j];
        d[2] += v[j] * bv[j];
      }
      if (has_ve(p.layer + 1) && col == 0) {
        const float* bg = vec + 640;
        const float* wg = p.wgate_next;
#pragma unroll
        for (int j = 0; j < kGateChannels; ++j) {
          dg += v[j] * bg[j];
#pragma unroll
          for (int h = 0; h < kHeads; ++h) gp[h] += v[j] * __ldg(wg + h * kGateChannels + j);
        }
      }
    } else {
      const float* bh = vec + 256 + c;
#pragma unroll
      for (int j = 0; j < 64; ++j) {
        ssq += v[j] * v[j];
        v[j] = bf16_round(v[j]);
        d[0] += v[j] * bh[j];
      }
    }
#pragma unroll
    for (int j = 0; j < 64; j += 8)
      st_global_v4(xo + j, pack_bf16x2(v[j], v[j + 1]), pack_bf16x2(v[j + 2], v[j + 3]),
                   pack_bf16x2(v[j + 4], v[j + 5]), pack_bf16x2(v[j + 6], v[j + 7]));
  }

  __device__ void end_mtile(int, int row) {
    float* s = p.stats_out + ((size_t)row * 2 + half) * kStatStride;
    s[0] = ssq;
    s[1] = d[0];
    s[2] = d[1];
    s[3] = d[2];
    s[4] = dg;
#pragma unroll
    for (int h = 0; h < kHeads; ++h) s[5 + h] = gp[h];
  }
};

// ---------------------------------------------------------------------------------------------
// Head: soft-capped logits of the whole vocabulary, reduced on the fly to the row's cross-entropy
// pieces. |z| <= 15 after the soft cap, so sum exp(z - 15) needs no running maximum.
// ---------------------------------------------------------------------------------------------
struct EpiHead {
  struct Params {
    PopCtx ctx;
    const float* stats;  // [rows][2][16]: sum x^2, x.b_head
    float* part;         // [rows][2][2]: sum exp(z - 15), z[target] (0 if not in this half)
  };
  static constexpr int kSmemBytes = kEpiVecBytes;
  const Params& p;
  float* vec;
  int lane, half;
  RowInfo ri;
  float inv, c2, se, zt;

  __device__ EpiHead(const Params& p_, uint8_t* smem, int ew, int lane_)
      : p(p_), vec(reinterpret_cast<float*>(smem) + ew * kWarpVecs * 128), lane(lane_), half(ew >> 2) {}

  __device__ void begin_mtile(int, int row) {
    ri = row_info(p.ctx, row);
    const float* s0 = p.stats + (size_t)row * 2 * kStatStride;
    const float* s1 = s0 + kStatStride;
    inv = rms_scale(s0[0] + s1[0], kWidth);
    c2 = ri.sign * (s0[1] + s1[1]);
    se = 0.f;
    zt = 0.f;
  }

  __device__ void begin_tile(int m_tile, int, int col0) {
    const RowInfo r0 = row_info(p.ctx, (int64_t)m_tile * 128);
    __syncwarp();
    warp_gauss128(vec, p.ctx.key, kTidHead, 0, r0.direction, col0, lane);
    __syncwarp();
  }

  __device__ void group(int, int col, float (&v)[64]) {
    const float* a = vec + (col & 127);
#pragma unroll
    for (int j = 0; j < 64; ++j) {
      const float logit = inv * (v[j] + c2 * a[j]);
      const float z = kSoftCap * tanhf(logit * (1.0f / kSoftCap));
      se += expf(z - kSoftCap);
      if (col + j == ri.tgt) zt = z;
    }
  }

  __device__ void end_mtile(int, int row) {
    float* o = p.part + ((size_t)row * 2 + half) * 2;
    o[0] = se;
    o[1] = zt;
  }
};

}  // namespace noise
