// Orthogonal direct draws of the DUST estimator (train/val/run.py:218-238), regenerated in-kernel.
//
// Draw idx of a site at token e = b * T + t is the row (offset[e] + idx) mod d of the Sylvester
// Hadamard matrix, H[r][c] = (-1)^popcount(r & c), times the site's sign pattern of cycle idx / d,
// times a per-(draw, token) sign:
//     a[idx][e][c] = H[(offset[e] + idx) & (d - 1)][c] * pattern[idx / d][c] * s[idx][e]
// Patterns, offsets and signs are bits of the counter-based stream (domain kDomainDirect, key
// (seed, step)); counter = (block, site << 2 | kind, direction):
//     kind 1 pattern bits  (block = c / 128, direction = cycle),   bit c % 128
//     kind 2 offsets       (block = e / 4,   direction = 0),       lane e % 4, low log2(d) bits
//     kind 3 draw signs    (block = e / 128, direction = idx),     bit e % 128
// A set bit means -1. The draw index is global (rank-independent), so every rank regenerates any
// draw; oracle/dust.py restates the same bits.
#pragma once

#include "philox.cuh"

namespace noise {

// site kinds of a direct rerun (bit positions in DirectSpec::site_mask)
enum : uint32_t { kSiteWte = 0, kSiteO = 1, kSiteAttn = 2, kSiteFc = 3, kSiteMlp = 4, kSiteKinds = 5 };

__device__ __forceinline__ uint32_t direct_word(PhiloxKey key, uint32_t block, uint32_t site, uint32_t kind,
                                                uint32_t direction, uint32_t word) {
  uint32_t x[4];
  philox4x32_10(block, (site << 2) | kind, direction, kDomainDirect, key.k0, key.k1, x);
  return x[word & 3];
}

// 32 pattern bits of columns [32 w, 32 w + 32) for cycle `cycle` (bit j <-> column 32 w + j)
__device__ __forceinline__ uint32_t pattern_word(PhiloxKey key, uint32_t site, uint32_t cycle, uint32_t w) {
  return direct_word(key, w >> 2, site, 1, cycle, w);
}

__device__ __forceinline__ uint32_t draw_offset(PhiloxKey key, uint32_t site, uint32_t e, uint32_t d) {
  return direct_word(key, e >> 2, site, 2, 0, e) & (d - 1);
}

__device__ __forceinline__ uint32_t draw_sign_bit(PhiloxKey key, uint32_t site, uint32_t idx, uint32_t e) {
  return (direct_word(key, e >> 7, site, 3, idx, e >> 5) >> (e & 31)) & 1u;
}

// Row state of one (draw, token): the Hadamard row and the combined sign bit (draw sign).
struct DrawRow {
  uint32_t hrow;   // (offset + idx) & (d - 1)
  uint32_t sbit;   // draw sign bit (1 = negative)
  uint32_t cycle;  // idx / d
};

__device__ __forceinline__ DrawRow draw_row(PhiloxKey key, uint32_t site, uint32_t idx, uint32_t e, uint32_t d) {
  DrawRow r;
  r.hrow = (draw_offset(key, site, e, d) + idx) & (d - 1);
  r.sbit = draw_sign_bit(key, site, idx, e);
  r.cycle = idx / d;
  return r;
}

// a at column c given the row state and the 32 pattern bits covering c (pat >> (c & 31) & 1).
__device__ __forceinline__ float draw_value(const DrawRow& r, uint32_t c, uint32_t pat_word) {
  const uint32_t neg = (__popc(r.hrow & c) ^ r.sbit ^ (pat_word >> (c & 31))) & 1u;
  return neg ? -1.0f : 1.0f;
}

}  // namespace noise
