// Sliding-window causal attention of the population forward (utils/model.py:17-31, 81-97):
// query s sees keys s - window .. s, softmax scale 1/sqrt(64), q and k already RoPE'd and
// RMS-normalised per head by the QKV epilogue.
//
// Because q and k are unit-RMS, |q.k| / 8 <= 8 (up to bf16 rounding), so the softmax runs with a
// fixed offset of 8 instead of a running maximum: exp(s/8 - 8) never overflows and the diagonal key
// keeps every row sum >= e^-16. No rescaling of the output accumulator is needed.
//
// One CTA = 64 queries x one head x one (member, sequence) row block; 4 warps x 16 queries. Q, K, V
// tiles arrive by TMA (128-byte swizzle) into a 2-stage ring; S = Q K^T and O += P V use
// mma.sync m16n8k16 (bf16 in, fp32 accumulate) with ldmatrix from the swizzled tiles. Key tiles
// outside [q0 - window, q0 + 63] are never loaded. The epilogue writes y in bf16 and, per head,
// the dot product of the rounded y with the member's c_proj column factor b, which the projection
// GEMM needs for its rank-1 term.
#pragma once

#include "model_layout.cuh"
#include "ptx.cuh"

namespace noise {

struct AttnParams {
  PopCtx ctx;
  __nv_bfloat16* y;  // [rows, 512]
  float* ystats;     // [rows][8]
  int layer, window;
  int* status;
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma_bf16_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// byte offset of (row, 16-byte chunk) in a 64-row x 128-byte tile written by TMA with SWIZZLE_128B
__device__ __forceinline__ uint32_t sw128(int row, int chunk) { return row * 128 + ((chunk ^ (row & 7)) << 4); }

constexpr int kAttnTile = 64;
constexpr int kAttnThreads = 128;
constexpr int kAttnTileBytes = kAttnTile * kHeadDim * 2;           // 8 KB
constexpr int kAttnSmem = 1024 + 5 * kAttnTileBytes + 256 + 64 * 4;  // Q + 2 x (K, V) + barriers + b_proj

__global__ void __launch_bounds__(kAttnThreads)
    attention_window_kernel(const __grid_constant__ CUtensorMap tm_qkv, const __grid_constant__ AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = base;
  uint8_t* sK = base + kAttnTileBytes;       // stage s at sK + s * 2 * tile
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + 5 * kAttnTileBytes);
  uint64_t* qbar = bars;
  uint64_t* kvbar = bars + 1;  // [2]
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 3);
  float* bproj = reinterpret_cast<float*>(base + 5 * kAttnTileBytes + 256);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int T = p.ctx.T;
  const int n_qt = T / kAttnTile;
  const int qt = n_qt - 1 - blockIdx.x;  // longest key ranges first
  const int head = blockIdx.y;
  const int64_t seq = blockIdx.z;
  const int64_t row_base = seq * T;
  const int q0 = qt * kAttnTile;
  const int kt_begin = max(0, q0 - p.window) / kAttnTile;
  const int n_kt = qt - kt_begin + 1;

  if (tid == 0) {
    mbar_init(qbar, 1);
    mbar_init(&kvbar[0], 1);
    mbar_init(&kvbar[1], 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  // member's c_proj column factor for this head's 64 columns
  if (tid < 16) {
    const RowInfo r0 = row_info(p.ctx, row_base);
    reinterpret_cast<float4*>(bproj)[tid] =
        gauss4(p.ctx.key, (head * kHeadDim >> 2) + tid, tid_proj(p.layer), 1, r0.direction);
  }
  __syncthreads();

  const int qcol = head * kHeadDim, kcol = kWidth + head * kHeadDim, vcol = 2 * kWidth + head * kHeadDim;
  if (tid == 0) {
    mbar_arrive_expect_tx(qbar, kAttnTileBytes);
    tma_load_2d(sQ, &tm_qkv, qbar, qcol, (int)(row_base + q0));
    for (int s = 0; s < 2 && s < n_kt; ++s) {
      mbar_arrive_expect_tx(&kvbar[s], 2 * kAttnTileBytes);
      const int r = (int)(row_base + (kt_begin + s) * kAttnTile);
      tma_load_2d(sK + s * 2 * kAttnTileBytes, &tm_qkv, &kvbar[s], kcol, r);
      tma_load_2d(sK + s * 2 * kAttnTileBytes + kAttnTileBytes, &tm_qkv, &kvbar[s], vcol, r);
    }
  }

  bool ok = mbar_wait(qbar, 0, abort_flag, p.status);
  uint32_t qf[4][4];
  const uint32_t sq = smem_u32(sQ);
  if (ok) {
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const int r = warp * 16 + (lane & 15);
      ldsm_x4(sq + sw128(r, 2 * kk + (lane >> 4)), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
    }
  }

  float o[8][4];
#pragma unroll
  for (int j = 0; j < 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float l0 = 0.f, l1 = 0.f;
  const float kScaleLog2 = 0.125f * 1.4426950408889634f;
  const float kOffsetLog2 = 8.0f * 1.4426950408889634f;
  const int qa = q0 + warp * 16 + g, qb = qa + 8;

  int issued = min(2, n_kt);
  for (int i = 0; ok && i < n_kt; ++i) {
    const int s = i & 1;
    if (!mbar_wait(&kvbar[s], (i >> 1) & 1, abort_flag, p.status)) {
      ok = false;
      break;
    }
    const uint32_t sk = smem_u32(sK + s * 2 * kAttnTileBytes);
    const uint32_t sv = sk + kAttnTileBytes;
    const int kt = kt_begin + i;
    float sc[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        uint32_t b0, b1, b2, b3;
        const int r = 16 * jj + (lane & 7) + ((lane >> 4) << 3);
        ldsm_x4(sk + sw128(r, 2 * kk + ((lane >> 3) & 1)), b0, b1, b2, b3);
        mma_bf16_16816(sc[2 * jj], qf[kk], b0, b1);
        mma_bf16_16816(sc[2 * jj + 1], qf[kk], b2, b3);
      }
    }
    const bool need_mask = (kt * kAttnTile + kAttnTile - 1 > q0) || (q0 + kAttnTile - 1 - kt * kAttnTile > p.window);
    uint32_t pf[4][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float e[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        e[u] = exp2f(sc[j][u] * kScaleLog2 - kOffsetLog2);
        if (need_mask) {
          const int key = kt * kAttnTile + 8 * j + 2 * t4 + (u & 1);
          const int q = (u < 2) ? qa : qb;
          if (key > q || q - key > p.window) e[u] = 0.f;
        }
      }
      // round to the bf16 the P.V product uses, so the normaliser matches the numerator
      const uint32_t lo = pack_bf16x2(e[0], e[1]), hi = pack_bf16x2(e[2], e[3]);
      const __nv_bfloat162 blo = *reinterpret_cast<const __nv_bfloat162*>(&lo);
      const __nv_bfloat162 bhi = *reinterpret_cast<const __nv_bfloat162*>(&hi);
      l0 += __low2float(blo) + __high2float(blo);
      l1 += __low2float(bhi) + __high2float(bhi);
      pf[j >> 1][(j & 1) * 2 + 0] = lo;
      pf[j >> 1][(j & 1) * 2 + 1] = hi;
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const uint32_t a[4] = {pf[kk][0], pf[kk][1], pf[kk][2], pf[kk][3]};
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        uint32_t b0, b1, b2, b3;
        const int r = 16 * kk + (lane & 7) + (((lane >> 3) & 1) << 3);
        ldsm_x4_t(sv + sw128(r, 2 * jj + (lane >> 4)), b0, b1, b2, b3);
        mma_bf16_16816(o[2 * jj], a, b0, b1);
        mma_bf16_16816(o[2 * jj + 1], a, b2, b3);
      }
    }
    __syncthreads();  // every warp is done with stage s
    if (tid == 0 && i + 2 < n_kt) {
      mbar_arrive_expect_tx(&kvbar[s], 2 * kAttnTileBytes);
      const int r = (int)(row_base + (kt + 2) * kAttnTile);
      tma_load_2d(sK + s * 2 * kAttnTileBytes, &tm_qkv, &kvbar[s], kcol, r);
      tma_load_2d(sK + s * 2 * kAttnTileBytes + kAttnTileBytes, &tm_qkv, &kvbar[s], vcol, r);
      ++issued;
    }
  }
  if (tid == 0) {  // copies still in flight land before the CTA exits
    for (int i = n_kt; i < issued; ++i) mbar_wait(&kvbar[i & 1], (i >> 1) & 1, abort_flag, p.status);
  }
  if (!ok) return;

  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float r0 = 1.0f / l0, r1 = 1.0f / l1;
  __nv_bfloat16* ya = p.y + (row_base + qa) * kWidth + head * kHeadDim;
  __nv_bfloat16* yb = p.y + (row_base + qb) * kWidth + head * kHeadDim;
  float da = 0.f, db = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int c = 8 * j + 2 * t4;
    const uint32_t pa = pack_bf16x2(o[j][0] * r0, o[j][1] * r0);
    const uint32_t pb = pack_bf16x2(o[j][2] * r1, o[j][3] * r1);
    *reinterpret_cast<uint32_t*>(ya + c) = pa;
    *reinterpret_cast<uint32_t*>(yb + c) = pb;
    const __nv_bfloat162 ha = *reinterpret_cast<const __nv_bfloat162*>(&pa);
    const __nv_bfloat162 hb = *reinterpret_cast<const __nv_bfloat162*>(&pb);
    da += __low2float(ha) * bproj[c] + __high2float(ha) * bproj[c + 1];
    db += __low2float(hb) * bproj[c] + __high2float(hb) * bproj[c + 1];
  }
  da += __shfl_xor_sync(0xffffffffu, da, 1);
  da += __shfl_xor_sync(0xffffffffu, da, 2);
  db += __shfl_xor_sync(0xffffffffu, db, 1);
  db += __shfl_xor_sync(0xffffffffu, db, 2);
  if (t4 == 0) {
    p.ystats[(row_base + qa) * kHeads + head] = da;
    p.ystats[(row_base + qb) * kHeads + head] = db;
  }
}

}  // namespace noise
