// Persistent tile scheduler: data-parallel full tiles, then a stream-K
// remainder. Shared by the host (planning, workspace sizing, CPU tests of the
// partition) and the device (every role of every CTA walks the same list).
//
// Replaces the reference's one-program-per-tile grid and its tile raster
// (kernels/gemm/utils/common.py:38-83 get_pids: XCD remap + GROUP_SIZE_M
// swizzle). On B200 the grid is one work unit per SM (cta_group::1) or per SM
// pair (cta_group::2); a unit walks its tiles in the same GROUP_M-swizzled
// raster so concurrently running units share A and B panels in L2.
//
// Three ways to spread the tiles left after the full data-parallel waves:
//   stream-K (modes 1, 2): their (tile, k) iteration space is cut into equal
//     contiguous ranges, one per unit;
//   split (mode 3): every leftover tile is cut into S equal k-chunks and chunk
//     s of leftover tile j goes to unit s * leftover + j, so units running at
//     the same time stream the same k-range of neighbouring tiles (their A and
//     B panels stay shared in L2, which contiguous ranges lose);
//   half (mode 4, and mode 3 when the tiles are too short to split in K;
//     both only when twice the leftover tiles fit on the units): every
//     leftover tile runs as two independent half-width tiles (N = 128, whole
//     K) on units 2j and 2j + 1, with no partial-tile reduction. An N = 128
//     MMA takes half the time of an N = 256 one, but a half tile still loads
//     its whole A panel, so it takes well over half a tile: splitting in K
//     (same bytes shared by two units) is preferred where a tile is long.
// Ownership rule (stream-K, and splits into more than two pieces): the unit
// that runs k-iteration 0 of a split tile owns it. Every other unit touching
// the tile does so in the FIRST segment of its range, writes an fp32 partial
// to its own workspace slot and raises a flag; the owner adds the partials in
// increasing unit order (deterministic) after its own accumulation and stores
// C. Contributors never wait and always have larger unit numbers than the
// owner, so the waits cannot form a cycle.
// K direction (serpentine): with `serpentine` set, the data-parallel tiles of
// odd waves walk their k-iterations from the last down to the first, so each
// wave starts on the k-chunks of the panels the previous wave read last, which
// are still in L2 (FP16 4096 x 4096 x 8192: 323 -> 251 MB read from DRAM per
// launch). The fp32 sums of those tiles are taken in the opposite order.
// Bit 1 extends the rule to the leftover items (split pieces, half tiles,
// stream-K segments), which run as the wave after the data-parallel ones.
// Pair rule (a tile split into two pieces): each piece reduces half of the
// tile's columns. Piece s keeps columns [128 s, 128 s + 128): it publishes its
// partial of the other half, raises its flag, then waits for its peer's flag
// and adds the peer's partial of its own half (peer partial + own, in that
// order on both sides: deterministic). Both publish before waiting, so the
// waits cannot form a cycle, and the two halves are reduced in parallel.
#pragma once

#include <stdint.h>

#if defined(__CUDACC__)
#define B2G_HD __host__ __device__ __forceinline__
#else
#define B2G_HD inline
#endif

namespace b2g {

enum : int { kRoleFull = 0, kRoleOwner = 1, kRoleContrib = 2, kRolePair = 3 };

struct SkPlan {
  int32_t tiles_m, tiles_n;  // output tile grid
  int32_t k_iters;           // k-iterations (pipeline stages) per tile
  int32_t units;             // persistent work units launched
  int32_t dp_tiles;          // tiles [0, dp_tiles) are data-parallel
  int32_t sk_units;          // units [0, sk_units) share the leftover tiles
  int64_t sk_iters;          // (tiles - dp_tiles) * k_iters
  int32_t group_m;           // raster group height in tiles
  int32_t splits;            // split mode: k-chunks per leftover tile (0 = stream-K)
  int32_t half;              // 1: leftover tiles run as half-width items (units [0, sk_units))
  int32_t serpentine;        // bit 0: data-parallel tiles of odd waves walk K backwards;
                             // bit 1: so do the leftover items when their wave is odd
};

struct WorkItem {
  int32_t tile;      // raster index
  int32_t tm, tn;    // tile coordinates
  int32_t k_begin;   // first k-iteration (inclusive)
  int32_t k_end;     // last k-iteration (exclusive)
  int32_t role;      // kRoleFull / kRoleOwner / kRoleContrib
  // owner only: contributing units first, first + stride, ... (n_contrib of them)
  int32_t first_contrib, n_contrib, contrib_stride;
  int32_t nh;        // -1: whole tile; 0 / 1: columns [0, 128) / [128, 256) of the tile
  // pair only: the half this piece reduces (0 / 1); its peer is first_contrib
  int32_t pair_half;
  int32_t k_desc;    // 1: k-iterations run from k_end - 1 down to k_begin
};

B2G_HD int32_t plan_tiles(const SkPlan& p) { return p.tiles_m * p.tiles_n; }

B2G_HD void tile_coords(const SkPlan& p, int32_t t, int32_t& tm, int32_t& tn) {
  const int32_t per_group = p.group_m * p.tiles_n;
  const int32_t g = t / per_group;
  const int32_t first_m = g * p.group_m;
  int32_t gm = p.tiles_m - first_m;
  if (gm > p.group_m) gm = p.group_m;
  const int32_t r = t - g * per_group;
  tm = first_m + r % gm;
  tn = r / gm;
}

B2G_HD int64_t sk_range_begin(const SkPlan& p, int32_t u) {
  return (p.sk_iters * u) / p.sk_units;
}

// Builds the plan. `sk_mode`: 0 = no splitting (all tiles data-parallel, the
// last wave partial); 1 = stream-K over the partial last wave only;
// 2 = stream-K over the last full wave plus the partial one; 3 = split the
// tiles of the partial last wave into equal k-chunks; 4 = run them as
// half-width tiles when they fit, else as mode 3.
inline SkPlan make_plan(int32_t tiles_m, int32_t tiles_n, int32_t k_iters, int32_t units,
                        int32_t group_m, int32_t sk_mode, int32_t min_sk_iters) {
  SkPlan p{};
  p.tiles_m = tiles_m;
  p.tiles_n = tiles_n;
  p.k_iters = k_iters;
  p.units = units;
  p.group_m = group_m < 1 ? 1 : group_m;
  if (min_sk_iters < 1) min_sk_iters = 1;
  const int32_t tiles = tiles_m * tiles_n;
  int32_t dp = tiles;
  if (sk_mode != 0 && tiles % units != 0) {
    int32_t waves = tiles / units;
    if (sk_mode == 2 && waves >= 1) waves -= 1;
    dp = waves * units;
  }
  p.dp_tiles = dp;
  const int32_t left = tiles - dp;
  p.sk_iters = static_cast<int64_t>(left) * k_iters;
  p.sk_units = 0;
  p.splits = 0;
  p.half = 0;
  if (left == 0) return p;
  if (sk_mode == 4 && 2 * left <= units) {
    p.half = 1;
    p.sk_units = 2 * left;
    return p;
  }
  if (sk_mode == 3 || sk_mode == 4) {
    // At most kMaxSplits pieces per leftover tile: the owner adds every
    // contributor's fp32 partial tile after its own k-range, and with more
    // than one contributor that serial reduction costs more than the shorter
    // pieces save (3840 x 3840 x 8192 fp16, 3 leftover tiles: 16 pieces 368 us,
    // 4 pieces 193 us, 2 pieces 188 us).
    constexpr int32_t kMaxSplits = 2;
    int32_t s = units / left;
    const int32_t s_max = k_iters / min_sk_iters;
    if (s > s_max) s = s_max;
    if (s > kMaxSplits) s = kMaxSplits;
    if (s < 1) s = 1;
    if (s == 1 && 2 * left <= units) {
      // too short to split in K (MXFP4 at K = 8192: 16 stages): half-width
      // tiles still put the idle units to work (58.3 against 59.3 us)
      p.half = 1;
      p.sk_units = 2 * left;
      return p;
    }
    p.splits = s;
    p.sk_units = left * s;
    return p;
  }
  int64_t su = p.sk_iters / min_sk_iters;
  if (su > units) su = units;
  if (su < 1) su = 1;
  p.sk_units = static_cast<int32_t>(su);
  return p;
}

// Iterates the work items of unit `u` in execution order.
struct WorkCursor {
  int32_t dp_next;   // next data-parallel tile index
  int64_t sk_pos;    // next stream-K iteration
  int64_t sk_end;    // end of this unit's stream-K range
};

B2G_HD WorkCursor cursor_begin(const SkPlan& p, int32_t u) {
  WorkCursor c;
  c.dp_next = u;
  if (p.half && u < p.sk_units) {
    c.sk_pos = 0;  // one half-width item
    c.sk_end = 1;
  } else if (u < p.sk_units) {
    c.sk_pos = sk_range_begin(p, u);
    c.sk_end = sk_range_begin(p, u + 1);
  } else {
    c.sk_pos = 0;
    c.sk_end = 0;
  }
  return c;
}

B2G_HD bool cursor_next(const SkPlan& p, int32_t u, WorkCursor& c, WorkItem& w) {
  w.first_contrib = -1;
  w.n_contrib = 0;
  w.contrib_stride = 1;
  w.nh = -1;
  w.pair_half = -1;
  w.k_desc = 0;
  if (c.dp_next < p.dp_tiles) {
    w.tile = c.dp_next;
    w.k_begin = 0;
    w.k_end = p.k_iters;
    w.role = kRoleFull;
    w.k_desc = p.serpentine & (w.tile / p.units) & 1;
    c.dp_next += p.units;
    tile_coords(p, w.tile, w.tm, w.tn);
    return true;
  }
  if (c.sk_pos >= c.sk_end) return false;
  // the leftover items run as wave dp_tiles / units
  w.k_desc = (p.serpentine >> 1) & (p.dp_tiles / p.units) & 1;
  if (p.half) {
    // half mode: units 2j, 2j + 1 take the two column halves of leftover tile j
    w.tile = p.dp_tiles + (u >> 1);
    w.nh = u & 1;
    w.k_begin = 0;
    w.k_end = p.k_iters;
    w.role = kRoleFull;
    c.sk_pos = c.sk_end;
    tile_coords(p, w.tile, w.tm, w.tn);
    return true;
  }
  if (p.splits > 0) {
    // split mode: exactly one chunk per unit
    const int32_t left = p.sk_units / p.splits;
    const int32_t j = u % left, s = u / left;
    w.tile = p.dp_tiles + j;
    w.k_begin = static_cast<int32_t>((static_cast<int64_t>(p.k_iters) * s) / p.splits);
    w.k_end = static_cast<int32_t>((static_cast<int64_t>(p.k_iters) * (s + 1)) / p.splits);
    if (p.splits == 1) {
      w.role = kRoleFull;
    } else if (p.splits == 2) {
      w.role = kRolePair;
      w.pair_half = s;
      w.first_contrib = s == 0 ? u + left : u - left;
      w.n_contrib = 1;
    } else if (s == 0) {
      w.role = kRoleOwner;
      w.first_contrib = u + left;
      w.n_contrib = p.splits - 1;
      w.contrib_stride = left;
    } else {
      w.role = kRoleContrib;
    }
    c.sk_pos = c.sk_end;
    tile_coords(p, w.tile, w.tm, w.tn);
    return true;
  }
  const int64_t local_tile = c.sk_pos / p.k_iters;
  const int64_t tile_begin = local_tile * p.k_iters;
  const int64_t tile_end = tile_begin + p.k_iters;
  const int64_t seg_end = c.sk_end < tile_end ? c.sk_end : tile_end;
  w.tile = p.dp_tiles + static_cast<int32_t>(local_tile);
  w.k_begin = static_cast<int32_t>(c.sk_pos - tile_begin);
  w.k_end = static_cast<int32_t>(seg_end - tile_begin);
  if (w.k_begin > 0) {
    w.role = kRoleContrib;
  } else if (w.k_end == p.k_iters) {
    w.role = kRoleFull;
  } else {
    w.role = kRoleOwner;
    int32_t v = u + 1;
    w.first_contrib = v;
    while (v < p.sk_units && sk_range_begin(p, v) < tile_end) ++v;
    w.n_contrib = v - w.first_contrib;
  }
  c.sk_pos = seg_end;
  tile_coords(p, w.tile, w.tm, w.tn);
  return true;
}

}  // namespace b2g
