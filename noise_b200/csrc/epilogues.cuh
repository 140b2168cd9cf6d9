// Epilogues of the population GEMMs. Each one finishes a perturbed linear layer of
// `population_loss` (train/val/eggroll.py:66-103) on a 64-column group of one accumulator row:
//
//   y = s * (x W^T + s_m (x b_m) a_m^T)        (train/val/eggroll.py:56-58, lowrank)
//
// where the row scale s is the RMS-norm of the layer input (applied here instead of on the operand:
// norm(x) W^T = (x W^T) / rms(x)), s_m = +-sigma is the member's sign, and x . b_m is a per-row scalar
// that the *producer* of x computed as a side statistic, so the GEMM itself is the plain shared-weight
// product. a_m's 128-column slice is copied into per-warp shared memory from the chunk's draw table
// (the counter-based stream, written once per chunk by draw_table_kernel).
//
// Row statistics travel between kernels as partial sums (the consumer adds the parts):
//   stats_a (QKV / head input x), float [rows][4][16]:
//       [0] sum x^2, [1..3] x.b_q, x.b_k, x.b_v (or [1] x.b_head),
//       [4] x[:32].b_gate, [5..12] x[:32].W_gate^T (value-embedding blocks)
//   stats_b (FC input x), float [rows][2][2]: sum x^2, x.b_fc
//   hstats (MLP-out input), float [rows][2]: hidden.b_mlp
// Dot products use the bf16 values the next GEMM reads; sums of squares use the fp32 stream.
// Row segments move through 32-byte (full-sector) per-thread loads and stores, or through TMA where
// an epilogue stages them (QKV and FC outputs, proj's residual rows, QKV's rotary rows).
#pragma once

#include "gemm_tc.cuh"
#include "model_layout.cuh"

namespace noise {

constexpr int kStatStride = 16;  // floats per stats_a part
constexpr int kStatParts = 4;    // stats_a parts per row

__device__ __forceinline__ float rms_scale(float ssq, int n) { return rsqrtf(ssq / (float)n + kNormEps); }

// Per-warp vector slots in the epilogue's shared memory.
template <int kVecs>
struct WarpVecs {
  static constexpr int kBytes = 8 * kVecs * 128 * 4;
};

// Output staging for TMA stores: each epilogue warp owns two 4 KiB tiles of 32 rows x 128 bytes in the
// 128-byte-swizzled layout of a {64 bf16, 32 rows} tensor-map box. A group's bf16 row segment is written
// by its thread (16-byte chunk c of row r at position c ^ (r % 8): conflict-free), then lane 0 stores
// the box with cp.async.bulk.tensor; a tile is rewritten only after the store issued from it two
// groups earlier has read it.
template <int kTiles>
struct StoreStageT {
  static constexpr int kTileBytes = 32 * 128;
  static constexpr int kBytes = 8 * kTiles * kTileBytes + 1024;  // 8 warps x kTiles tiles, plus alignment slack
  uint8_t* tile[kTiles];
  int next = 0;
  __device__ void init(uint8_t* region, int ew) {
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(region) + 1023) & ~uintptr_t(1023));
    for (int i = 0; i < kTiles; ++i) tile[i] = base + (ew * kTiles + i) * kTileBytes;
  }
  // v[0..63] of row (row0 + lane) -> global columns [col, col + 64) through the map
  __device__ void store64(const CUtensorMap* map, const float (&v)[64], int lane, int col, int row0) {
    uint8_t* t = tile[next];
    next = (next + 1) % kTiles;
    if (lane == 0) tma_store_wait_read<kTiles - 1>();
    __syncwarp();
    uint8_t* r = t + lane * 128;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      uint4 w;
      w.x = pack_bf16x2(v[8 * c + 0], v[8 * c + 1]);
      w.y = pack_bf16x2(v[8 * c + 2], v[8 * c + 3]);
      w.z = pack_bf16x2(v[8 * c + 4], v[8 * c + 5]);
      w.w = pack_bf16x2(v[8 * c + 6], v[8 * c + 7]);
      *reinterpret_cast<uint4*>(r + ((c ^ (lane & 7)) << 4)) = w;
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_2d(map, t, col, row0);
      tma_store_commit();
    }
  }
  // the same with the 64 values already packed to bf16 pairs
  __device__ void store64_packed(const CUtensorMap* map, const uint32_t (&w)[32], int lane, int col, int row0) {
    uint8_t* t = tile[next];
    next = (next + 1) % kTiles;
    if (lane == 0) tma_store_wait_read<kTiles - 1>();
    __syncwarp();
    uint8_t* r = t + lane * 128;
#pragma unroll
    for (int c = 0; c < 8; ++c)
      *reinterpret_cast<uint4*>(r + ((c ^ (lane & 7)) << 4)) = make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_2d(map, t, col, row0);
      tma_store_commit();
    }
  }
  // every store has completed (before the CTA's shared memory goes away)
  __device__ void drain(int lane) {
    if (lane == 0) tma_store_wait_all<0>();
    __syncwarp();
  }
};

using StoreStage = StoreStageT<2>;

// Input staging for the fp32 residual rows an epilogue reads: each epilogue warp owns one 8 KiB tile
// of 32 rows x 64 floats, filled by two {32 fp32, 32 rows} tensor-map boxes (128-byte swizzle: the
// 16-byte chunk c of row r of box b sits at b * 4 KiB + r * 128 + (c ^ (r % 8)) * 16, so the warp's
// row-per-thread reads are conflict-free). The next group's load is issued as soon as the current
// group has read its tile, so it overlaps the group's math and the next accumulator wait.
struct LoadStage {
  static constexpr int kTileBytes = 32 * 64 * 4;
  static constexpr int kBytes = 8 * kTileBytes + 8 * 8 + 1024;  // tiles, one mbarrier per warp, alignment
  uint8_t* tile;
  uint64_t* bar;
  uint32_t phase = 0;
  bool pending = false;
  __device__ void init(uint8_t* region, int ew, int lane) {
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(region) + 1023) & ~uintptr_t(1023));
    tile = base + ew * kTileBytes;
    bar = reinterpret_cast<uint64_t*>(base + 8 * kTileBytes) + ew;
    if (lane == 0) {
      mbar_init(bar, 1);
      fence_mbarrier_init();
    }
    __syncwarp();
  }
  // warp-uniform: columns [col, col + 64) of rows [row0, row0 + 32)
  __device__ void issue(const CUtensorMap* map, int col, int row0, int lane) {
    fence_proxy_async_smem();  // this warp's reads of the tile come before the copy overwrites it
    __syncwarp();
    if (lane == 0) {
      mbar_arrive_expect_tx(bar, kTileBytes);
      tma_load_2d(tile, map, bar, col, row0);
      tma_load_2d(tile + kTileBytes / 2, map, bar, col + 32, row0);
    }
    pending = true;
  }
  // bounded wait for the issued load; false (and the status word set) when it timed out
  __device__ bool wait(int* status) {
    pending = false;
    const uint32_t par = phase;
    phase ^= 1u;
    if (mbar_try_wait(bar, par)) return true;
    const long long start = clock64();
    while (!mbar_try_wait_sleep(bar, par, 20000u)) {
      if (clock64() - start > kWaitCycleBudget) {
        if (status) atomicExch(status, kStatusWaitTimeout);
        return false;
      }
    }
    return true;
  }
  // floats 4 q .. 4 q + 3 of this thread's row (q = 0 .. 15)
  __device__ float4 read4(int lane, int q) const {
    return *reinterpret_cast<const float4*>(tile + (q >> 3) * (kTileBytes / 2) + lane * 128 +
                                            (((q & 7) ^ (lane & 7)) << 4));
  }
};

// The rotary table rows (bf16 cos[0..31] | sin[0..31], one 128-byte swizzled row per position) of a
// warp's 32 consecutive positions, loaded once per M tile by one tensor-map box and read by every q
// and k head of those rows.
struct RopeStage {
  static constexpr int kTileBytes = 32 * 128;
  static constexpr int kBytes = 8 * kTileBytes + 8 * 8 + 1024;
  uint8_t* tile;
  uint64_t* bar;
  uint32_t phase = 0;
  bool pending = false;
  __device__ void init(uint8_t* region, int ew, int lane) {
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(region) + 1023) & ~uintptr_t(1023));
    tile = base + ew * kTileBytes;
    bar = reinterpret_cast<uint64_t*>(base + 8 * kTileBytes) + ew;
    if (lane == 0) {
      mbar_init(bar, 1);
      fence_mbarrier_init();
    }
    __syncwarp();
  }
  __device__ void issue(const CUtensorMap* map, int t0, int lane) {
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      mbar_arrive_expect_tx(bar, kTileBytes);
      tma_load_2d(tile, map, bar, 0, t0);
    }
    pending = true;
  }
  __device__ void wait(int* status) {
    pending = false;
    const uint32_t par = phase;
    phase ^= 1u;
    if (mbar_try_wait(bar, par)) return;
    const long long start = clock64();
    while (!mbar_try_wait_sleep(bar, par, 20000u)) {
      if (clock64() - start > kWaitCycleBudget) {
        if (status) atomicExch(status, kStatusWaitTimeout);
        return;
      }
    }
  }
  // cos (half 0) or sin (half 1) of frequencies 8 c .. 8 c + 7 (c = 0 .. 3) for this thread's position
  __device__ void read8(int lane, int half, int c, float (&out)[8]) const {
    const uint4 u = *reinterpret_cast<const uint4*>(tile + lane * 128 + (((4 * half + c) ^ (lane & 7)) << 4));
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) out[2 * i] = __uint_as_float(w[i] << 16), out[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
};

// Sum the kStatParts parts of a stats_a row into out[0..15].
__device__ __forceinline__ void load_stats_a(const float* stats, int64_t row, float (&out)[16]) {
  const float* s = stats + (size_t)row * kStatParts * kStatStride;
  ld_global_v8f(s, *reinterpret_cast<float(*)[8]>(&out[0]));
  ld_global_v8f(s + 8, *reinterpret_cast<float(*)[8]>(&out[8]));
#pragma unroll
  for (int p = 1; p < kStatParts; ++p) {
    float a[8], b[8];
    ld_global_v8f(s + p * kStatStride, a);
    ld_global_v8f(s + p * kStatStride + 8, b);
#pragma unroll
    for (int i = 0; i < 8; ++i) out[i] += a[i], out[8 + i] += b[i];
  }
}

// ---------------------------------------------------------------------------------------------
// QKV: q, k through RoPE and a per-head RMS norm; v plus the gated value embedding.
// ---------------------------------------------------------------------------------------------
struct EpiQkv {
  struct Params {
    CUtensorMap tm_qkv;     // qkv [rows, 1536] bf16, boxes of {64, 32}
    CUtensorMap tm_rope;    // [T, 64] bf16 cos | sin, boxes of {64, 32}
    int* status;
    PopCtx ctx;
    __nv_bfloat16* qkv;     // [rows, 1536]
    const float* stats;     // stats_a
    const float* ve_table;  // [4096, 512] or nullptr
    int layer;
  };
  // one store tile per warp: with the rotary rows staged too, a second would not fit beside 3 operand stages
  static constexpr int kSmemBytes = WarpVecs<2>::kBytes + StoreStageT<1>::kBytes + RopeStage::kBytes;
  static constexpr bool kInterleaveN = false;
  const Params& p;
  float* vec;  // this warp's slots: [0] a of the tile's tensor, [1] b_ve
  int lane, half;
  RowInfo ri;
  float inv, xb[3], gate[kHeads], a_ve_tok;
  StoreStageT<1> out;
  RopeStage rs;
  int m_next = -1;  // this CTA's next 128-row tile

  __device__ EpiQkv(const Params& p_, uint8_t* smem, int ew, int lane_)
      : p(p_), vec(reinterpret_cast<float*>(smem) + ew * 2 * 128), lane(lane_), half(ew >> 2) {
    out.init(smem + WarpVecs<2>::kBytes, ew);
    rs.init(smem + WarpVecs<2>::kBytes + StoreStageT<1>::kBytes, ew, lane);
  }

  __device__ void next_unit(int m, int) { m_next = m; }

  __device__ void begin_mtile(int, int row) {
    if (!rs.pending) rs.issue(&p.tm_rope, (row - lane) % p.ctx.T, lane);  // the first unit's rows
    ri = row_info(p.ctx, row);
    float st[16];
    load_stats_a(p.stats, row, st);
    inv = rms_scale(st[0], kWidth);
#pragma unroll
    for (int i = 0; i < 3; ++i) xb[i] = st[1 + i];
    if (has_ve(p.layer)) {
      const float4 ag0 = draw4(p.ctx, ri.slot, tid_gate(p.layer), 0, 0);
      const float4 ag1 = draw4(p.ctx, ri.slot, tid_gate(p.layer), 0, 1);
      const float ag[8] = {ag0.x, ag0.y, ag0.z, ag0.w, ag1.x, ag1.y, ag1.z, ag1.w};
#pragma unroll
      for (int h = 0; h < kHeads; ++h) {
        const float pre = inv * (st[5 + h] + ri.sign * st[4] * ag[h]);
        gate[h] = 2.0f / (1.0f + expf(-pre));
      }
      a_ve_tok = draw1(p.ctx, ri.slot, tid_ve(p.layer), 0, ri.tok);
    }
  }

  __device__ void begin_tile(int m_tile, int, int col0) {
    // all rows of an M tile belong to one member
    const RowInfo r0 = row_info(p.ctx, (int64_t)m_tile * 128);
    const int which = col0 / kWidth, local = col0 % kWidth;
    const uint32_t tid = which == 0 ? tid_q(p.layer) : which == 1 ? tid_k(p.layer) : tid_v(p.layer);
    __syncwarp();
    warp_draw128(vec, p.ctx, r0.slot, tid, 0, local, lane);
    if (which == 2 && has_ve(p.layer)) warp_draw128(vec + 128, p.ctx, r0.slot, tid_ve(p.layer), 1, local, lane);
    __syncwarp();
  }

  __device__ void group(int row, int col, float (&v)[64]) {
    const int which = col / kWidth, local = col % kWidth, head = local / kHeadDim;
    const float* a = vec + (local & 127);
    const float c2 = ri.sign * xb[which];
#pragma unroll
    for (int j = 0; j < 64; ++j) v[j] = inv * (v[j] + c2 * a[j]);
    if (which < 2) {
      if (rs.pending) rs.wait(p.status);  // the M tile's first q or k group
      float ss = 0.f;
#pragma unroll
      for (int j0 = 0; j0 < 32; j0 += 8) {
        float c[8], s[8];
        rs.read8(lane, 0, j0 >> 3, c);
        rs.read8(lane, 1, j0 >> 3, s);
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int j = j0 + u;
          const float x1 = v[j], x2 = v[j + 32];
          v[j] = x1 * c[u] + x2 * s[u];
          v[j + 32] = x2 * c[u] - x1 * s[u];
          ss += v[j] * v[j] + v[j + 32] * v[j + 32];
        }
      }
      const float r = rms_scale(ss, kHeadDim);
#pragma unroll
      for (int j = 0; j < 64; ++j) v[j] *= r;
      // after this warp's last k group of the M tile the rows are free: fetch the next unit's
      if (which == 1 && local == 256 + half * 128 + 64 && m_next >= 0)
        rs.issue(&p.tm_rope, (m_next * 128 + ((row - lane) & 127)) % p.ctx.T, lane);
    } else if (has_ve(p.layer)) {
      const float* ve = p.ve_table + (size_t)ri.tok * kWidth + local;
      const float* bve = vec + 128 + (local & 127);
      const float g = gate[head], sa = ri.sign * a_ve_tok;
#pragma unroll
      for (int j = 0; j < 64; j += 8) {
        float e[8];
        ld_global_nc_v8f(ve + j, e);
#pragma unroll
        for (int u = 0; u < 8; ++u) v[j + u] += g * (e[u] + sa * bve[j + u]);
      }
    }
    out.store64(&p.tm_qkv, v, lane, col, row - lane);
  }

  __device__ void end_mtile(int, int, int) {}
  __device__ void finish() {
    if (rs.pending) rs.wait(p.status);  // a load issued for a unit that never ran lands before exit
    out.drain(lane);
  }
};

// ---------------------------------------------------------------------------------------------
// attention projection + residual: x += y Wp^T + s (y.b_p) a_p; emits the FC input and its stats.
// ---------------------------------------------------------------------------------------------
struct EpiProj {
  struct Params {
    CUtensorMap tm_x;        // x [rows, 512] fp32, boxes of {32, 32}
    int* status;
    PopCtx ctx;
    float* x;                // [rows, 512] fp32 residual stream, updated in place
    __nv_bfloat16* xb;       // [rows, 512] bf16 copy for the FC GEMM
    const float* ystats;     // [rows][8] per-head y.b_proj from the attention kernel
    float* stats_out;        // stats_b
    int layer;
  };
  static constexpr int kSmemBytes = WarpVecs<2>::kBytes + LoadStage::kBytes;
  static constexpr bool kInterleaveN = false;
  const Params& p;
  float* vec;  // [0] a_proj, [1] b_fc
  int lane, half;
  RowInfo ri;
  float c2, ssq, dfc;
  SiteJitter jit;  // direct mode: draw added to the c_proj output (site 'attn')
  uint32_t patw[4];
  LoadStage xs;     // the residual rows
  int m_next = -1;  // this CTA's next 128-row tile

  __device__ EpiProj(const Params& p_, uint8_t* smem, int ew, int lane_)
      : p(p_), vec(reinterpret_cast<float*>(smem) + ew * 2 * 128), lane(lane_), half(ew >> 2) {
    xs.init(smem + WarpVecs<2>::kBytes, ew, lane);
  }

  __device__ void next_unit(int m, int) { m_next = m; }

  __device__ void begin_mtile(int, int row) {
    if (!xs.pending) xs.issue(&p.tm_x, half * 128, row - lane, lane);  // the first group of the first unit
    ri = row_info(p.ctx, row);
    float ys[8];
    ld_global_v8f(p.ystats + (size_t)row * kHeads, ys);
    c2 = ri.sign * (ys[0] + ys[1] + ys[2] + ys[3] + ys[4] + ys[5] + ys[6] + ys[7]);
    ssq = 0.f;
    dfc = 0.f;
    jit = site_jitter(p.ctx, p.layer, kSiteAttn, row, kWidth);
  }

  __device__ void begin_tile(int m_tile, int, int col0) {
    const RowInfo r0 = row_info(p.ctx, (int64_t)m_tile * 128);
    __syncwarp();
    warp_draw128(vec, p.ctx, r0.slot, tid_proj(p.layer), 0, col0, lane);
    warp_draw128(vec + 128, p.ctx, r0.slot, tid_fc(p.layer), 1, col0, lane);
    __syncwarp();
    if (jit.on) site_patterns(p.ctx, kSiteAttn, jit.r, col0, patw);
  }

  __device__ void group(int row, int col, float (&v)[64]) {
    const float* a = vec + (col & 127);
    const float* b = vec + 128 + (col & 127);
    if (jit.on) {
#pragma unroll
      for (int j = 0; j < 64; ++j)
        v[j] += jit.scale * draw_value(jit.r, col + j, patw[((col + j) & 127) >> 5]);
    }
    float* xr = p.x + (size_t)row * kWidth + col;
    xs.wait(p.status);
#pragma unroll
    for (int q = 0; q < 16; ++q) {
      const float4 x4 = xs.read4(lane, q);
      v[4 * q] += x4.x + c2 * a[4 * q];
      v[4 * q + 1] += x4.y + c2 * a[4 * q + 1];
      v[4 * q + 2] += x4.z + c2 * a[4 * q + 2];
      v[4 * q + 3] += x4.w + c2 * a[4 * q + 3];
    }
    // the next group of this warp: the other 64 columns of its half, the next N tile, or the next unit
    {
      const int g = (col >> 6) & 1, n = col >> 8;
      const int row0 = row - lane;
      if (g == 0) xs.issue(&p.tm_x, col + 64, row0, lane);
      else if (n + 1 < kWidth / 256) xs.issue(&p.tm_x, (n + 1) * 256 + half * 128, row0, lane);
      else if (m_next >= 0) xs.issue(&p.tm_x, half * 128, m_next * 128 + (row0 & 127), lane);
    }
#pragma unroll
    for (int j = 0; j < 64; j += 8) st_global_v8f(xr + j, v + j);
#pragma unroll
    for (int j = 0; j < 64; ++j) {
      ssq += v[j] * v[j];
      v[j] = bf16_round(v[j]);
      dfc += v[j] * b[j];
    }
    st_bf16x64(p.xb + (size_t)row * kWidth + col, v);
  }

  __device__ void end_mtile(int, int, int row) {
    *reinterpret_cast<float2*>(p.stats_out + ((size_t)row * 2 + half) * 2) = make_float2(ssq, dfc);
  }

  // a load issued for a group that never ran (a timed-out pipeline) lands before the CTA exits
  __device__ void finish() {
    if (xs.pending) xs.wait(p.status);
  }
};

// ---------------------------------------------------------------------------------------------
// FC: hidden = relu(norm(x) Wfc^T + rank-1)^2 in bf16, plus the hidden.b_mlp statistic.
// ---------------------------------------------------------------------------------------------
struct EpiFc {
  struct Params {
    CUtensorMap tm_hidden;  // hidden [rows, 2048] bf16, boxes of {64, 32}
    PopCtx ctx;
    __nv_bfloat16* hidden;  // [rows, 2048]
    const float* stats;     // stats_b
    float* hstats;          // [rows][2] partial hidden.b_mlp
    int layer;
  };
  static constexpr int kSmemBytes = WarpVecs<2>::kBytes + StoreStage::kBytes;
  static constexpr bool kInterleaveN = false;
  const Params& p;
  float* vec;  // [0] a_fc, [1] b_mlp
  int lane, half;
  RowInfo ri;
  float inv, c2, dmp;
  SiteJitter jit;  // direct mode: draw added to the live units' pre-activation (site 'fc')
  uint32_t patw[4];
  StoreStage out;

  __device__ EpiFc(const Params& p_, uint8_t* smem, int ew, int lane_)
      : p(p_), vec(reinterpret_cast<float*>(smem) + ew * 2 * 128), lane(lane_), half(ew >> 2) {
    out.init(smem + WarpVecs<2>::kBytes, ew);
  }

  __device__ void begin_mtile(int, int row) {
    ri = row_info(p.ctx, row);
    const float4 s = *reinterpret_cast<const float4*>(p.stats + (size_t)row * 4);
    inv = rms_scale(s.x + s.z, kWidth);
    c2 = ri.sign * (s.y + s.w);
    dmp = 0.f;
    jit = site_jitter(p.ctx, p.layer, kSiteFc, row, kHidden);
  }

  __device__ void begin_tile(int m_tile, int, int col0) {
    const RowInfo r0 = row_info(p.ctx, (int64_t)m_tile * 128);
    __syncwarp();
    warp_draw128(vec, p.ctx, r0.slot, tid_fc(p.layer), 0, col0, lane);
    warp_draw128(vec + 128, p.ctx, r0.slot, tid_mlp(p.layer), 1, col0, lane);
    __syncwarp();
    if (jit.on) site_patterns(p.ctx, kSiteFc, jit.r, col0, patw);
  }

  __device__ void group(int row, int col, float (&v)[64]) {
    const float* a = vec + (col & 127);
    const float* b = vec + 128 + (col & 127);
    if (jit.on) {  // direct mode: the draw joins the normalised pre-activation of live units
      const int64_t seq_rows = (int64_t)p.ctx.B * p.ctx.T;
      const __nv_bfloat16* lv = p.ctx.dir.live + (size_t)(row % seq_rows) * kHidden + col;
#pragma unroll
      for (int j = 0; j < 64; ++j) {
        v[j] = inv * (v[j] + c2 * a[j]);
        if (__bfloat162float(lv[j]) > 0.f) v[j] += jit.scale * draw_value(jit.r, col + j, patw[((col + j) & 127) >> 5]);
        const float r = fmaxf(v[j], 0.f);
        v[j] = r * r;
      }
    } else {
      // relu(inv (x + c2 a))^2 = inv^2 relu(x + c2 a)^2 for inv > 0
      const float inv2 = inv * inv;
#pragma unroll
      for (int j = 0; j < 64; ++j) {
        const float r = fmaxf(v[j] + c2 * a[j], 0.f);
        v[j] = (r * r) * inv2;
      }
    }
    // bf16 hidden once; its statistic hidden . b_mlp is taken from the rounded values
    uint32_t w[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      w[i] = pack_bf16x2(v[2 * i], v[2 * i + 1]);
      dmp += __uint_as_float(w[i] << 16) * b[2 * i] + __uint_as_float(w[i] & 0xFFFF0000u) * b[2 * i + 1];
    }
    out.store64_packed(&p.tm_hidden, w, lane, col, row - lane);
  }

  __device__ void end_mtile(int, int, int row) { p.hstats[(size_t)row * 2 + half] = dmp; }
  __device__ void finish() { out.drain(lane); }
};

// ---------------------------------------------------------------------------------------------
// MLP out + residual, then the next block's x0 mixing (utils/model.py:199) and its input stats;
// after the last block, the head's input and stats. N-interleaved schedule: the two CTAs of an
// M tile run together so the 512 KiB hidden tile is read from DRAM once.
// ---------------------------------------------------------------------------------------------
struct MlpOutParams {
  PopCtx ctx;
  float* x;               // [rows, 512] residual stream, in place
  __nv_bfloat16* xb;      // [rows, 512] next GEMM's operand
  const float* hstats;    // [rows][2]
  float* stats_out;       // stats_a
  const float* wte;       // [4096, 512] fp32 token embedding (x0 recomputation)
  const float* inv0;      // [rows] 1/rms of the perturbed embedding row
  const float* lambdas;   // resid_lambdas[8] | x0_lambdas[8]
  const float* wgate_next;  // [8, 32] fp32 of the next block, or nullptr
  float* x_final;         // [rows, 512] fp32 output of the last block (capture only), or nullptr
  int layer;
};

template <bool kDirect>
struct EpiMlpOutT {
  using Params = MlpOutParams;
  static constexpr int kSmemBytes = WarpVecs<6>::kBytes;
  static constexpr bool kInterleaveN = true;
  static constexpr bool kPair = true;  // K = 2048: the 2-SM engine halves the weight traffic per MMA
  const Params& p;
  float* vec;  // [0] a_mlp, [1] b_wte, [2..4] next b_q, b_k, b_v (or [2] b_head), [5] next b_gate
  int lane, half;
  bool last;
  RowInfo ri;
  float c2, lr, l0, sa_wte, i0, ssq, d[3], dg, gp[kHeads];
  SiteJitter jit, jit_wte;  // direct mode: site 'mlp' in this block; the embedding draw inside x0
  uint32_t patw[4], patw_wte[4];

  __device__ EpiMlpOutT(const Params& p_, uint8_t* smem, int ew, int lane_)
      : p(p_), vec(reinterpret_cast<float*>(smem) + ew * 6 * 128), lane(lane_), half(ew >> 2),
        last(p_.layer == kLayers - 1) {}

  __device__ void begin_mtile(int, int row) {
    ri = row_info(p.ctx, row);
    const float2 h = *reinterpret_cast<const float2*>(p.hstats + (size_t)row * 2);
    c2 = ri.sign * (h.x + h.y);
    ssq = 0.f, d[0] = d[1] = d[2] = 0.f, dg = 0.f;
#pragma unroll
    for (int h = 0; h < kHeads; ++h) gp[h] = 0.f;
    if (!last) {
      const int nl = p.layer + 1;
      lr = p.lambdas[nl] + ri.sign * draw1(p.ctx, ri.slot, kTidResid, 0, nl);
      l0 = p.lambdas[kLayers + nl] + ri.sign * draw1(p.ctx, ri.slot, kTidX0, 0, nl);
      sa_wte = ri.sign * draw1(p.ctx, ri.slot, kTidWte, 0, ri.tok);
      i0 = p.inv0[row];
    }
    if constexpr (kDirect) {
      jit = site_jitter(p.ctx, p.layer, kSiteMlp, row, kWidth);
      jit_wte = site_jitter(p.ctx, -1, kSiteWte, row, kWidth);  // on for every block when rerun from the embedding
    }
  }

  __device__ void begin_tile(int m_tile, int, int col0) {
    const RowInfo r0 = row_info(p.ctx, (int64_t)m_tile * 128);
    const uint32_t slot = r0.slot, e4 = (col0 >> 2) + lane;
    // every vector's load is issued before the first store, so the loads overlap one another and the
    // warp's wait for the previous tile's readers of vec
    const float4 d_mlp = draw4(p.ctx, slot, tid_mlp(p.layer), 0, e4);
    float4 d_wte, d_q, d_k, d_v, d_gate;
    const bool gate = !last && has_ve(p.layer + 1) && col0 == 0 && lane < 8;  // b_gate has 32 entries
    if (!last) {
      const int nl = p.layer + 1;
      d_wte = draw4(p.ctx, slot, kTidWte, 1, e4);
      d_q = draw4(p.ctx, slot, tid_q(nl), 1, e4);
      d_k = draw4(p.ctx, slot, tid_k(nl), 1, e4);
      d_v = draw4(p.ctx, slot, tid_v(nl), 1, e4);
      if (gate) d_gate = draw4(p.ctx, slot, tid_gate(nl), 1, lane);
    } else {
      d_q = draw4(p.ctx, slot, kTidHead, 1, e4);
    }
    __syncwarp();
    float4* v4 = reinterpret_cast<float4*>(vec);  // [0] a_mlp, [32] b_wte, [64] b_q or b_head, ...
    v4[lane] = d_mlp;
    v4[64 + lane] = d_q;
    if (!last) {
      v4[32 + lane] = d_wte;
      v4[96 + lane] = d_k;
      v4[128 + lane] = d_v;
      if (gate) v4[160 + lane] = d_gate;
    }
    __syncwarp();
    if constexpr (kDirect) {
      if (jit.on) site_patterns(p.ctx, kSiteMlp, jit.r, col0, patw);
      if (jit_wte.on) site_patterns(p.ctx, kSiteWte, jit_wte.r, col0, patw_wte);
    }
  }

  __device__ void group(int row, int col, float (&v)[64]) {
    const int c = col & 127;
    const float* a = vec + c;
    if constexpr (kDirect) {
      if (jit.on) {
#pragma unroll
        for (int j = 0; j < 64; ++j) v[j] += jit.scale * draw_value(jit.r, col + j, patw[((col + j) & 127) >> 5]);
      }
    }
    float* xr = p.x + (size_t)row * kWidth + col;
#pragma unroll
    for (int h = 0; h < 64; h += 32) {  // two 32-column halves keep fewer loads live
      float x8[4][8];
#pragma unroll
      for (int j = 0; j < 4; ++j) ld_global_v8f(xr + h + 8 * j, x8[j]);
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int u = 0; u < 8; ++u) v[h + 8 * j + u] += x8[j][u] + c2 * a[h + 8 * j + u];
    }
    if (!last) {
      const float* bw = vec + 128 + c;
      const float* bq = vec + 256 + c;
      const float* bk = vec + 384 + c;
      const float* bv = vec + 512 + c;
      const float* e = p.wte + (size_t)ri.tok * kWidth + col;
#pragma unroll
      for (int h = 0; h < 64; h += 32) {
        float e8[4][8];
#pragma unroll
        for (int j = 0; j < 4; ++j) ld_global_nc_v8f(e + h + 8 * j, e8[j]);
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const int k = h + 8 * j + u;
            float ek = e8[j][u] + sa_wte * bw[k];
            if constexpr (kDirect)
              if (jit_wte.on) ek += jit_wte.scale * draw_value(jit_wte.r, col + k, patw_wte[((col + k) & 127) >> 5]);
            const float x0 = ek * i0;
            v[k] = lr * v[k] + l0 * x0;
          }
      }
#pragma unroll
      for (int j = 0; j < 64; j += 8) st_global_v8f(xr + j, v + j);
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
      if (p.x_final) {
#pragma unroll
        for (int j = 0; j < 64; j += 8) st_global_v8f(p.x_final + (size_t)row * kWidth + col + j, v + j);
      }
#pragma unroll
      for (int j = 0; j < 64; ++j) {
        ssq += v[j] * v[j];
        v[j] = bf16_round(v[j]);
        d[0] += v[j] * bh[j];
      }
    }
    st_bf16x64(p.xb + (size_t)row * kWidth + col, v);
  }

  __device__ void end_mtile(int, int n, int row) {
    float* s = p.stats_out + ((size_t)row * kStatParts + 2 * n + half) * kStatStride;
    const float w0[8] = {ssq, d[0], d[1], d[2], dg, gp[0], gp[1], gp[2]};
    const float w1[8] = {gp[3], gp[4], gp[5], gp[6], gp[7], 0.f, 0.f, 0.f};
    st_global_v8f(s, w0);
    st_global_v8f(s + 8, w1);
  }
};

// ---------------------------------------------------------------------------------------------

// the population forward (rank-1 members) and the direct-draw reruns (site jitter) instantiate it apart,
// so the former carries none of the jitter state
using EpiMlpOut = EpiMlpOutT<false>;
using EpiMlpOutDirect = EpiMlpOutT<true>;

// Head: soft-capped logits of the whole vocabulary, reduced on the fly to the row's cross-entropy
// pieces. |z| <= 15 after the soft cap, so sum exp(z - 15) needs no running maximum.
// kF32: the GEMM reads the fp32 final stream and the fp32 lm_head master through kind::tf32 MMAs (the
// direct reruns' head, which train/val/run.py:272-278 runs in float32 with autocast off); otherwise
// the bf16 stream copy and the packed bf16 head (the population forward's autocast head).
// ---------------------------------------------------------------------------------------------
struct HeadParams {
  PopCtx ctx;
  const float* stats;  // stats_a: sum x^2, x.b_head
  float* part;         // [rows][2][2]: sum exp(z - 15), z[target] (0 if not in this half)
  float* logits;       // [rows, 4096] raw logits before the soft cap (capture only), or nullptr
};

template <bool kF32>
struct EpiHeadT {
  static constexpr bool kTf32 = kF32;
  using Params = HeadParams;
  static constexpr int kSmemBytes = WarpVecs<1>::kBytes;
  static constexpr bool kInterleaveN = false;
  const Params& p;
  float* vec;
  int lane, half;
  RowInfo ri;
  float inv, c2, se, zt;

  __device__ EpiHeadT(const Params& p_, uint8_t* smem, int ew, int lane_)
      : p(p_), vec(reinterpret_cast<float*>(smem) + ew * 128), lane(lane_), half(ew >> 2) {}

  __device__ void begin_mtile(int, int row) {
    ri = row_info(p.ctx, row);
    float st[16];
    load_stats_a(p.stats, row, st);
    inv = rms_scale(st[0], kWidth);
    c2 = ri.sign * st[1];
    se = 0.f;
    zt = 0.f;
  }

  __device__ void begin_tile(int m_tile, int, int col0) {
    const RowInfo r0 = row_info(p.ctx, (int64_t)m_tile * 128);
    __syncwarp();
    warp_draw128(vec, p.ctx, r0.slot, kTidHead, 0, col0, lane);
    __syncwarp();
  }

  __device__ void group(int row, int col, float (&v)[64]) {
    const float* a = vec + (col & 127);
    if (p.logits) {
      float lg[64];
#pragma unroll
      for (int j = 0; j < 64; ++j) lg[j] = inv * (v[j] + c2 * a[j]);
#pragma unroll
      for (int j = 0; j < 64; j += 8) st_global_v8f(p.logits + (size_t)row * kVocab + col + j, lg + j);
    }
    // exp(z - 15) with z = 15 tanh(l / 15): since tanh(u) - 1 = -2 / (e^(2u) + 1),
    // z - 15 = -30 / (e^(2 l / 15) + 1), i.e. two base-2 exponentials and one reciprocal per logit.
    const float k_in = 2.0f / kSoftCap * 1.4426950408889634f;
    const float k_out = -2.0f * kSoftCap * 1.4426950408889634f;
    float lt = 0.f;
    bool mine = false;
#pragma unroll
    for (int j = 0; j < 64; ++j) {
      const float logit = inv * (v[j] + c2 * a[j]);
      se += ex2_approx(k_out * rcp_approx(ex2_approx(logit * k_in) + 1.0f));
      if (col + j == ri.tgt) lt = logit, mine = true;
    }
    if (mine) zt = kSoftCap * tanhf(lt * (1.0f / kSoftCap));  // the target's capped logit, once per row
  }

  __device__ void end_mtile(int, int, int row) {
    *reinterpret_cast<float2*>(p.part + ((size_t)row * 2 + half) * 2) = make_float2(se, zt);
  }
};

using EpiHead = EpiHeadT<false>;
using EpiHeadF32 = EpiHeadT<true>;

}  // namespace noise
