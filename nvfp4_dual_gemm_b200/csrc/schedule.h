// schedule.h — persistent tile scheduler of the dual GEMM, shared by the
// device kernel and the host (planning, workspace sizing, tests).
//
// The output is cut into 128 x BN tiles (BN columns of each GEMM); a tile
// needs `kblocks` = K/256 main-loop iterations.  The reference launches one
// CTA per tile and never splits K (nvfp4_dual_gemm.cu:95-97, 368-372), which
// leaves 20-52 of the 148 SMs idle on its decode shapes.  Here a persistent
// grid of `grid` CTAs (at most one per SM) works through:
//   1. data-parallel (DP) tiles: tile t < dp_tiles goes whole to CTA t % grid;
//   2. stream-K (SK) tiles: the remaining tiles' iterations, laid end to end,
//      are cut into `grid` equal contiguous ranges, CTA b taking
//      [lo(b), lo(b+1)), lo(b) = b * sk_iters / grid.
// A tile whose iterations span CTAs b_first..b_last is finished by b_first,
// which holds the tile's first K blocks as the LAST item of its range, while
// for every other contributor its segment is the FIRST item of its range:
// those write their fp32 partial accumulators to workspace slots and bump the
// tile's counter; b_first waits (bounded) for the count, adds the partials to
// its own accumulator in a fixed order and runs the SiLU epilogue.  Waits
// only go from a CTA's last item to other CTAs' first items, so none can
// wait on a CTA that waits, and in practice the partials are already there.
#pragma once

#include <cstdint>

#if defined(__CUDACC__)
#define NVFP4DG_HD __host__ __device__ __forceinline__
#else
#define NVFP4DG_HD inline
#endif

namespace nvfp4dg {

struct Plan {
  int m_tiles;      // ceil(M / (128 * ctas))
  int n_tiles;      // N / BN
  int kblocks;      // K / 256
  int num_tiles;    // L * m_tiles * n_tiles
  int grid;         // persistent work units (CTAs, or CTA pairs)
  int dp_tiles;     // whole tiles handed out round-robin (multiple of grid)
  int bn;           // tile width per GEMM (64 or 128)
  int ctas;         // CTAs per work unit: 1, or 2 for a 2-SM pair (M = 256)
  long long sk_iters;  // (num_tiles - dp_tiles) * kblocks
  int split;        // 2: the two CTAs of a cluster split each tile's K range
                    // (unit b = CTA b: tile b / 2, K half b % 2); else 0
  // tile / m_tiles as (umulhi(tile, mt_mul) + tile) >> mt_shift (set by
  // set_tile_div; a division by a run-time value is a long dependent chain
  // on the producers' way to their first copy)
  uint32_t mt_mul;
  int mt_shift;
  int L;            // batch count (independent problems of one shape)
  // (tile / m_tiles) / n_tiles, the batch of a tile, likewise (L > 1)
  uint32_t nt_mul;
  int nt_shift;
};

// Division by d >= 1 through a multiply-high: shift = ceil(log2 d),
// mul = floor(2^32 (2^shift - d) / d) + 1; exact for every n < 2^31
// (Granlund and Montgomery, "Division by invariant integers using
// multiplication", 1994, round-up variant).
inline void set_div(unsigned long long d, uint32_t& mul, int& shift_out) {
  int shift = 0;
  while ((1ull << shift) < d) ++shift;
  shift_out = shift;
  mul = static_cast<uint32_t>(((1ull << 32) * ((1ull << shift) - d)) / d +
                              1ull);
}

inline void set_tile_div(Plan& p) {
  if (p.L < 1) p.L = 1;
  set_div(static_cast<unsigned long long>(p.m_tiles), p.mt_mul, p.mt_shift);
  set_div(static_cast<unsigned long long>(p.n_tiles), p.nt_mul, p.nt_shift);
}

NVFP4DG_HD uint32_t div_by(uint32_t t, uint32_t mul, int shift) {
#if defined(__CUDA_ARCH__)
  const uint32_t hi = __umulhi(t, mul);
#else
  const uint32_t hi =
      static_cast<uint32_t>((static_cast<unsigned long long>(t) * mul) >> 32);
#endif
  return (hi + t) >> shift;
}

// (batch, m_tile, n_tile) of linear tile index `tile`: m fastest, then n,
// then the batch.
NVFP4DG_HD void tile_lmn(const Plan& p, int tile, int& l, int& m_tile,
                         int& n_tile) {
  const uint32_t t = static_cast<uint32_t>(tile);
  const int u = static_cast<int>(div_by(t, p.mt_mul, p.mt_shift));
  m_tile = tile - u * p.m_tiles;
  if (p.L == 1) {
    l = 0;
    n_tile = u;
  } else {
    l = static_cast<int>(div_by(static_cast<uint32_t>(u), p.nt_mul,
                                p.nt_shift));
    n_tile = u - l * p.n_tiles;
  }
}


struct Work {
  int tile;  // linear tile index; m fastest: m = tile % m_tiles
  int kb0;   // first 256-wide K block
  int kb1;   // one past the last K block
  int slot;  // workspace slot of the partial, -1 for a whole tile
};

NVFP4DG_HD long long sk_lo(const Plan& p, int b) {
  return static_cast<long long>(b) * p.sk_iters / p.grid;
}

// CTA whose stream-K range holds iteration x.
NVFP4DG_HD int sk_owner(const Plan& p, long long x) {
  return static_cast<int>(((x + 1) * p.grid - 1) / p.sk_iters);
}

// Workspace slot used by CTA b for its segment of stream-K tile ts
// (ts counted from the first SK tile): slot 2b for the CTA's first segment,
// 2b + 1 for its last one.
NVFP4DG_HD int sk_slot(const Plan& p, int b, long long ts) {
  const long long first_ts = sk_lo(p, b) / p.kblocks;
  return 2 * b + (first_ts == ts ? 0 : 1);
}

struct WorkIter {
  int b;
  int dp_next;
  int first_sk;
  int pad;
  long long it;
  long long it_end;
};

NVFP4DG_HD void work_begin(const Plan& p, int b, WorkIter& s) {
  s.b = b;
  s.dp_next = b;
  s.first_sk = 1;
  s.pad = 0;
  if (p.sk_iters > 0) {
    s.it = sk_lo(p, b);
    s.it_end = sk_lo(p, b + 1);
  } else {
    s.it = 0;
    s.it_end = 0;
  }
}

NVFP4DG_HD bool work_next(const Plan& p, WorkIter& s, Work& w) {
  if (p.split == 2) {
    // Cluster split-K: one work item per CTA, K blocks [0, h) on the even
    // CTA and [h, kblocks) on the odd one (kblocks >= 2).
    if (!s.first_sk) return false;
    s.first_sk = 0;
    const int h = (p.kblocks + 1) / 2;
    w.tile = s.b / 2;
    w.kb0 = (s.b & 1) ? h : 0;
    w.kb1 = (s.b & 1) ? p.kblocks : h;
    w.slot = -1;
    return true;
  }
  if (s.dp_next < p.dp_tiles) {
    w.tile = s.dp_next;
    w.kb0 = 0;
    w.kb1 = p.kblocks;
    w.slot = -1;
    s.dp_next += p.grid;
    return true;
  }
  if (s.it >= s.it_end) return false;
  const long long ts = s.it / p.kblocks;
  const int kb0 = static_cast<int>(s.it - ts * p.kblocks);
  const long long left = s.it_end - s.it;
  const int kb1 = (kb0 + left < p.kblocks) ? static_cast<int>(kb0 + left)
                                           : p.kblocks;
  w.tile = p.dp_tiles + static_cast<int>(ts);
  w.kb0 = kb0;
  w.kb1 = kb1;
  const bool whole = (kb0 == 0 && kb1 == p.kblocks);
  w.slot = whole ? -1 : 2 * s.b + (s.first_sk ? 0 : 1);
  s.first_sk = 0;
  s.it += kb1 - kb0;
  return true;
}

// CTAs [*b_first, *b_last] hold the segments of stream-K tile ts.
NVFP4DG_HD void sk_tile_owners(const Plan& p, long long ts, int* b_first,
                               int* b_last) {
  *b_first = sk_owner(p, ts * p.kblocks);
  *b_last = sk_owner(p, ts * p.kblocks + p.kblocks - 1);
}

// Workspace layout, independent of the plan so that one buffer serves calls
// with different plans: [counters: kCounterBytes, one int per stream-K tile
// and CTA of its work unit, always left at zero by a completed call]
// [partials: 2 slots per CTA of 128 x 2*BN fp32].
constexpr long long kCounterBytes = 64ll * 1024;  // 16384 >= 2 * 2 * 4095
NVFP4DG_HD long long partial_slot_floats(const Plan& p) {
  return 128ll * 2 * p.bn;
}
NVFP4DG_HD long long workspace_partials_offset(const Plan&) {
  return kCounterBytes;
}
NVFP4DG_HD long long workspace_bytes(const Plan& p) {
  if (p.sk_iters == 0) return 0;
  return kCounterBytes +
         2ll * p.grid * p.ctas * partial_slot_floats(p) * 4;
}
// Partial slot of CTA `rank` of the unit whose unit-level slot is `unit_slot`
// (2 * unit + which).
NVFP4DG_HD long long cta_slot(const Plan& p, int unit_slot, int rank) {
  return 2ll * ((unit_slot >> 1) * p.ctas + rank) + (unit_slot & 1);
}

}  // namespace nvfp4dg
