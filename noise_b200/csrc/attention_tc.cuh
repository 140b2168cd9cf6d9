// Sliding-window causal attention on the 5th-generation tensor cores (utils/model.py:17-31, 81-97):
// query s sees keys s - window .. s, softmax scale 1/sqrt(64), q and k already RoPE'd and
// RMS-normalised per head by the QKV epilogue.
//
// One CTA = G consecutive 128-query tiles x one head x one (member, sequence) row block. The G tiles
// share every K/V tile the CTA streams. The kernel is bound by the latency of each query tile's
// S -> softmax -> P -> PV cycle, not by the tensor or exp2 units, so it holds as many query tiles per
// SM as TMEM allows: G = 2, 96 registers, a 3-stage K ring and a 2-stage V ring (2 CTAs and 20 warps
// per SM; G = 1 when the tile count is odd). Warps:
//   warp 0       TMA producer: the G Q tiles once, then 64-key K and V tiles, K two tiles ahead of V
//   warp 1       TMEM owner and MMA issuer (one thread), per key tile j and query tile g:
//                  O_g += P_g V_{j-1}  tcgen05.mma M=128 N=64 K=64, A = P_g from TMEM, B = V (MN-major smem)
//                  S_g  = Q_g K_j^T    tcgen05.mma M=128 N=64 K=64, A and B K-major smem
//   warps 2..    softmax group g = 4 warps, one query row per thread: S_g from TMEM -> p = exp(s/8 - 8)
//                (masked) -> bf16 P_g written back over S_g's first 32 TMEM columns; at the end
//                O_g / sum(p) -> y, y.b_proj.
// P never passes through shared memory: the PV product reads it from TMEM, and S_g of the next key
// tile is issued after that product (the tensor core runs one thread's products in issue order).
// The groups run out of phase with each other, so the tensor core serves one group's products while
// the special-function unit works through another's exponentials.
// Because q and k are unit-RMS, |q.k| / 8 <= 8 (up to bf16 rounding), so the softmax uses the fixed
// offset 8: no running maximum and no rescaling of the TMEM accumulator. Each query tile walks only
// the key tiles its window reaches; 32-key chunks outside a warp's rows' windows skip their
// exponentials. TMEM: group g uses S (then P) at 128g and O at 128g + 64.
// Every wait is bounded (status word on timeout).
//
// Score mode (kScore, DUST's attention reruns, train/val/run.py:391-463): Q, K and V each come from
// their own [rows, 512] map, and CTA row block z reads operand X's sequence z % mod_X (mod 0: z), so
// per-draw operands and shared clean ones mix in one launch. Instead of y, each query row writes
// score[z * T + q][head] = <target, O> - base (target and base of the clean sequence z % seqs).
#pragma once

#include "model_layout.cuh"
#include "ptx.cuh"

namespace noise {

struct AttnTcParams {
  PopCtx ctx;
  __nv_bfloat16* y;  // [rows, 512]
  float* ystats;     // [rows][8]
  int layer, window;
  int* status;
  int col_q, col_k, col_v;  // column of head 0 in each operand's map
  int mod_q, mod_k, mod_v;  // row block of operand X = blockIdx.z % mod_X (0: blockIdx.z)
  // score mode
  const __nv_bfloat16* target;  // [seqs * T, 512]
  const float* base;            // [seqs * T][8] or nullptr
  float* score;                 // [gridDim.z * T][8]
  int seqs;
};

constexpr int kAtQ = 128;
constexpr int kAtQBytes = kAtQ * kHeadDim * 2;  // 16 KB

// G query tiles per CTA, key tiles of KT keys (64 or 128). A K or V tile is KT rows x 128 B. TMEM per
// query tile: S (KT columns, P over its first KT / 2 once S is read), then O.
// K and V have rings of their own: a K stage is free once the S products have read it, a V stage
// once the PV products have, and the producer keeps K kKStages - 1 tiles ahead of V.
template <int G, int KT>
struct AttnTcLayout {
  static constexpr int kThreads = (2 + 4 * G) * 32;
  static constexpr int kTileBytes = KT * kHeadDim * 2;
  static constexpr int kKStages = KT == 64 ? 3 : 2, kVStages = 2;
  static constexpr int kCore = G * kAtQBytes + (kKStages + kVStages) * kTileBytes;
  static constexpr int kSmem = 1024 + kCore + 512 + kHeadDim * 4;  // 1 KB for the 1024-byte alignment
  static constexpr uint32_t kGroupCols = KT == 64 ? 128 : 256;
  static constexpr uint32_t kTmemCols = kGroupCols * G;
};

// kDirect (population mode only): the DUST reruns' instantiation, which adds the 'o'-site draw.
template <int G, int KT, bool kScore, bool kDirect = false>
__global__ void __launch_bounds__(AttnTcLayout<G, KT>::kThreads, G == 1 && KT == 64 ? 3 : 2)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ AttnTcParams p) {
  using L = AttnTcLayout<G, KT>;
  constexpr int kAtK = KT, kAtTileBytes = L::kTileBytes;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = base;                              // [g] 16 KB
  constexpr int KS = L::kKStages, VS = L::kVStages;
  uint8_t* sK = sQ + G * kAtQBytes;         // [stage] KT x 128 B
  uint8_t* sV = sK + KS * kAtTileBytes;     // [stage] KT x 128 B
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + L::kCore);
  uint64_t* q_full = bars;
  uint64_t* k_full = q_full + 1;      // [KS]
  uint64_t* k_empty = k_full + KS;    // [KS]
  uint64_t* v_full = k_empty + KS;    // [VS]
  uint64_t* v_empty = v_full + VS;    // [VS]
  uint64_t* s_full = v_empty + VS;    // [G]
  uint64_t* p_full = s_full + G;      // [G]
  uint64_t* o_full = p_full + G;      // [G]
  uint64_t* drain = o_full + G;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* bproj = reinterpret_cast<float*>(base + L::kCore + 512);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int T = p.ctx.T;
  const int n_units = T / (kAtQ * G);
  const int unit = n_units - 1 - blockIdx.x;  // longest key ranges first
  const int head = blockIdx.y;
  const int64_t row_base = (int64_t)blockIdx.z * T;
  auto operand_rows = [&](int mod) { return (int64_t)(mod ? (int)blockIdx.z % mod : (int)blockIdx.z) * T; };
  const int q0 = unit * kAtQ * G;  // first query of the CTA
  const int kt_begin = max(0, q0 - p.window) / kAtK;
  const int kt_end = (q0 + kAtQ * G - 1) / kAtK;
  const int n_kt = kt_end - kt_begin + 1;
  // Each query tile g needs only key tiles [g_lo(g), g_hi(g)] of the CTA's range (relative indices):
  // the tiles before its window are skipped by the MMA and softmax roles alike.
  auto g_lo = [&](int g) { return max(0, q0 + kAtQ * g - p.window) / kAtK - kt_begin; };
  auto g_hi = [&](int g) { return (q0 + kAtQ * g + kAtQ - 1) / kAtK - kt_begin; };
  int* status = p.status;

  if (tid == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < KS; ++s) mbar_init(&k_full[s], 1), mbar_init(&k_empty[s], 1);
    for (int s = 0; s < VS; ++s) mbar_init(&v_full[s], 1), mbar_init(&v_empty[s], 1);
    for (int g = 0; g < G; ++g) {
      mbar_init(&s_full[g], 1);
      mbar_init(&p_full[g], 4);
    }
    for (int g = 0; g < G; ++g) mbar_init(&o_full[g], 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
    prefetch_tensormap(&tm_q);
    prefetch_tensormap(&tm_k);
    prefetch_tensormap(&tm_v);
  }
  if (!kScore && tid >= 64 && tid < 80) {  // the member's c_proj column factor for this head's 64 columns
    const RowInfo r0 = row_info(p.ctx, row_base);
    reinterpret_cast<float4*>(bproj)[tid - 64] =
        draw4(p.ctx, r0.slot, tid_proj(p.layer), 1, (head * kHeadDim >> 2) + (tid - 64));
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, L::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const int qcol = p.col_q + head * kHeadDim, kcol = p.col_k + head * kHeadDim, vcol = p.col_v + head * kHeadDim;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      const int64_t rq = operand_rows(p.mod_q), rk = operand_rows(p.mod_k), rv = operand_rows(p.mod_v);
      mbar_arrive_expect_tx(q_full, G * kAtQBytes);
      for (int b = 0; b < 2 * G; ++b)
        tma_load_2d(sQ + b * (kAtQBytes / 2), &tm_q, q_full, qcol, (int)(rq + q0 + 64 * b));
      // order K(0) .. K(KS - 2), then K(j + KS - 1) before V(j): each wait is for a stage that the
      // products issued before the one the next copy feeds have released
      int nk = 0, nv = 0;
      bool ok = true;
      auto load = [&](bool key, int j) {
        const int stages = key ? KS : VS, st = j % stages;
        uint64_t* full = key ? &k_full[st] : &v_full[st];
        if (!mbar_wait(key ? &k_empty[st] : &v_empty[st], ((j / stages) & 1) ^ 1, abort_flag, status)) return false;
        mbar_arrive_expect_tx(full, kAtTileBytes);
        uint8_t* dst = (key ? sK : sV) + st * kAtTileBytes;
        const int r = (kt_begin + j) * kAtK;
        for (int h = 0; h < KT / 64; ++h)  // boxes of 64 rows
          tma_load_2d(dst + h * 8192, key ? &tm_k : &tm_v, full, key ? kcol : vcol, (int)((key ? rk : rv) + r + 64 * h));
        return true;
      };
      while (ok && nv < n_kt) {
        if (nk < n_kt && nk < nv + KS - 1) ok = load(true, nk++);
        else ok = load(false, nv++);
      }
      // copies in flight land before the CTA can exit
      mbar_wait(q_full, 0, abort_flag, status);
      for (int j = max(0, nk - KS); j < nk; ++j) mbar_wait(&k_full[j % KS], (j / KS) & 1, abort_flag, status);
      for (int j = max(0, nv - VS); j < nv; ++j) mbar_wait(&v_full[j % VS], (j / VS) & 1, abort_flag, status);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      // Per key tile j, for each query tile g: PV(j - 1), then S(j). P(j - 1) lies in the TMEM columns
      // of S(j - 1), so S(j) is issued only after the PV product that reads them (the tensor core
      // runs one thread's products in issue order).
      const uint32_t idesc_s = make_idesc(1, kAtQ, kAtK);
      const uint32_t idesc_o = make_idesc(1, kAtQ, kHeadDim, 0, 1);  // B = V is MN-major
      bool ok = mbar_wait(q_full, 0, abort_flag, status);
      tc_fence_after();
      for (int j = 0; ok && j <= n_kt; ++j) {
        const int jj = j - 1;
        bool v_ready = false, k_ready = false;
        for (int g = 0; g < G && ok; ++g) {
          const int lo = g_lo(g), hi = g_hi(g);
          const uint32_t tG = tmem + L::kGroupCols * g;  // S, then P over its first columns
          if (jj >= lo && jj <= hi) {
            if (!v_ready && !(v_ready = mbar_wait(&v_full[jj % VS], (jj / VS) & 1, abort_flag, status))) {
              ok = false;
              break;
            }
            if (!mbar_wait(&p_full[g], (jj - lo) & 1, abort_flag, status)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint64_t dv = smem_desc_sw128_mn(sV + (jj % VS) * kAtTileBytes);
#pragma unroll
            for (int k = 0; k < kAtK / 16; ++k)  // 16 keys of P = 8 TMEM columns
              tc_mma_f16_ts(tG + KT, tG + 8 * k, dv + (uint64_t)(2048 >> 4) * k, idesc_o, (jj > lo || k > 0) ? 1u : 0u);
            if (jj == hi) tc_commit(&o_full[g]);  // this query tile's output is complete
          }
          if (j < n_kt && j >= lo && j <= hi) {
            if (!k_ready) {
              if (!(k_ready = mbar_wait(&k_full[j % KS], (j / KS) & 1, abort_flag, status))) {
                ok = false;
                break;
              }
              tc_fence_after();
            }
            const uint64_t dk = smem_desc_sw128(sK + (j % KS) * kAtTileBytes);
            const uint64_t dq = smem_desc_sw128(sQ + g * kAtQBytes);
#pragma unroll
            for (int k = 0; k < kHeadDim / 16; ++k)
              tc_mma_f16(tG, dq + 2 * k, dk + 2 * k, idesc_s, k > 0 ? 1u : 0u);
            tc_commit(&s_full[g]);
          }
        }
        if (!ok) break;
        // every tile of [0, n_kt) is used by at least one query tile
        if (jj >= 0) tc_commit(&v_empty[jj % VS]);
        if (j < n_kt) tc_commit(&k_empty[j % KS]);
      }
      tc_commit(drain);
      mbar_wait(drain, 0, abort_flag, status);
    }
    __syncwarp();
  } else {
    // ---------------- softmax + output ----------------
    const int g = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;      // row of query tile g = TMEM lane
    const int qg = q0 + kAtQ * g;           // first query of tile g
    const int q = qg + r;
    const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
    const uint32_t tS = tmem + L::kGroupCols * g, tO = tS + KT;
    const float kScaleLog2 = 0.125f * 1.4426950408889634f;
    const float kOffsetLog2 = 8.0f * 1.4426950408889634f;
    // packed fp32 pairs (sm_100 f32x2 FMA / add): two independent partial row sums of two lanes each
    const float2 kScale2 = make_float2(kScaleLog2, kScaleLog2), kNegOffset2 = make_float2(-kOffsetLog2, -kOffsetLog2);
    float2 lsum[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
    bool ok = true;
    const int qlo = qg + quarter * 32, qhi = qlo + 31;  // this warp's rows
    const int j_lo = g_lo(g), j_hi = g_hi(g);
    for (int j = j_lo; j <= j_hi; ++j) {
      const int k0 = (kt_begin + j) * kAtK;
      const uint32_t par = (uint32_t)(j - j_lo) & 1u;
      if (!mbar_wait(&s_full[g], par, abort_flag, status)) {
        ok = false;
        break;
      }
      tc_fence_after();
#pragma unroll 1
      for (int h = 0; h < KT / 64; ++h) {  // 64-key parts of S; P (bf16 pairs) goes over S's first columns
        {
          float sv[64];
          tmem_ld64(tS + lane_addr + 64 * h, sv);
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const int kc = k0 + 64 * h + 32 * c;
            // warp-uniform classification of the 32 x 32 block (this warp's rows x the chunk's keys):
            // fully visible blocks take a path without per-key masks
            const bool none = kc > qhi || qlo - (kc + 31) > p.window;
            const bool all = (kc + 31 <= qlo) && (qhi - kc <= p.window);
            uint32_t pw[16];
            if (all) {
#pragma unroll
              for (int u = 0; u < 16; ++u) {
                const int i = 32 * c + 2 * u;
                const float2 x = __ffma2_rn(make_float2(sv[i], sv[i + 1]), kScale2, kNegOffset2);
                const float2 e = make_float2(ex2_approx(x.x), ex2_approx(x.y));
                lsum[u & 1] = __fadd2_rn(lsum[u & 1], e);
                pw[u] = pack_bf16x2(e.x, e.y);
              }
            } else if (none) {
#pragma unroll
              for (int u = 0; u < 16; ++u) pw[u] = 0u;
            } else {
#pragma unroll
              for (int u = 0; u < 16; ++u) {
                const int i = 32 * c + 2 * u;
                const float2 x = __ffma2_rn(make_float2(sv[i], sv[i + 1]), kScale2, kNegOffset2);
                float2 e = make_float2(ex2_approx(x.x), ex2_approx(x.y));
                const int key = kc + 2 * u;
                if (key > q || q - key > p.window) e.x = 0.f;
                if (key + 1 > q || q - key - 1 > p.window) e.y = 0.f;
                lsum[u & 1] = __fadd2_rn(lsum[u & 1], e);
                pw[u] = pack_bf16x2(e.x, e.y);
              }
            }
            // P's columns 32h + 16c .. + 15 hold S values this part or the one before it has read
            tmem_st16(tS + lane_addr + 32 * h + 16 * c, pw);
          }
        }
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[g]);
    }
    if (kScore) {
      if (ok && mbar_wait(&o_full[g], 0, abort_flag, status)) {
        tc_fence_after();
        float o[64];
        tmem_ld64(tO + lane_addr, o);
        const float inv = 1.0f / ((lsum[0].x + lsum[0].y) + (lsum[1].x + lsum[1].y));
        const int64_t trow = (int64_t)((int)blockIdx.z % p.seqs) * T + q;
        const uint4* tg = reinterpret_cast<const uint4*>(p.target + trow * kWidth + head * kHeadDim);
        float d = 0.f;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint4 u = __ldg(tg + c);
          const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w4[i]));
            d += o[8 * c + 2 * i] * f.x + o[8 * c + 2 * i + 1] * f.y;
          }
        }
        d *= inv;
        if (p.base) d -= __ldg(p.base + trow * kHeads + head);
        p.score[(row_base + q) * kHeads + head] = d;
      }
    } else if (ok && mbar_wait(&o_full[g], 0, abort_flag, status)) {
      tc_fence_after();
      float o[64];
      tmem_ld64(tO + lane_addr, o);
      const float inv = 1.0f / ((lsum[0].x + lsum[0].y) + (lsum[1].x + lsum[1].y));
      float d = 0.f;
      if constexpr (kDirect) {
        // direct mode: the draw added to the attention output (site 'o', before c_proj)
        const SiteJitter jit = site_jitter(p.ctx, p.layer, kSiteO, row_base + q, kWidth);
        uint32_t patw[4] = {0u, 0u, 0u, 0u};
        if (jit.on) site_patterns(p.ctx, kSiteO, jit.r, (head * kHeadDim) & ~127, patw);
#pragma unroll
        for (int j = 0; j < 64; ++j) {
          const int col = head * kHeadDim + j;
          const float jv = jit.on ? jit.scale * draw_value(jit.r, col, patw[(col & 127) >> 5]) : 0.f;
          o[j] = bf16_round(o[j] * inv + jv);
          d += o[j] * bproj[j];
        }
      } else {
#pragma unroll
        for (int j = 0; j < 64; ++j) {
          o[j] = bf16_round(o[j] * inv);
          d += o[j] * bproj[j];
        }
      }
      st_bf16x64(p.y + (row_base + q) * kWidth + head * kHeadDim, o);
      p.ystats[(row_base + q) * kHeads + head] = d;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, L::kTmemCols);
  }
}

}  // namespace noise
