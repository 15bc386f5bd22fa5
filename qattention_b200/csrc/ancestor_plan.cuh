// Level planning shared by the ancestor-walk kernels.
//
// In a complete b-ary BFS tree, parent(a) = (a-1)/b for a >= 1, and the step-s
// ancestors of a contiguous node range [lo, hi] form the contiguous range
// [anc^s(lo'), anc^s(hi)] (lo' skips nodes whose walk already ended at the
// root). A CTA that owns queries [q_lo, q_lo+nq) therefore needs, per walk
// level s = 0..L-1, one contiguous range of K/V rows. Ranges only move towards
// the root as s grows, so overlapping or touching neighbours merge into
// windows; every window is staged once in shared memory and level s gets one
// offset with   slot = lv_off[s] + node.
#pragma once

#include "qa_common.cuh"

#include <type_traits>

namespace qa {

constexpr int kMaxLevels = 32;  // walk levels (including the own level) planned per CTA

// Computes, on one thread, the staged levels and windows of a query tile.
// max_depth = 0 plans only the own level. Levels are dropped from the deep
// end until the windows fit in rows_cap rows; n_levels reports how many fit.
QA_DEVINL void plan_levels(int q_lo, int nq, int max_depth, FastDiv div_b, int rows_cap,
                           int* lv_off, int* win_lo, int* win_base, int& n_levels,
                           int& n_windows) {
  int rlo[kMaxLevels], rhi[kMaxLevels], lev_win[kMaxLevels];
  int L = 1;
  rlo[0] = q_lo;
  rhi[0] = q_lo + nq - 1;
  while (L < kMaxLevels && L <= max_depth && rhi[L - 1] > 0) {
    rlo[L] = int(fast_div(uint32_t(max(rlo[L - 1], 1) - 1), div_b));
    rhi[L] = int(fast_div(uint32_t(rhi[L - 1] - 1), div_b));
    ++L;
  }
  int nw, cum;
  for (;;) {
    nw = 0;
    cum = 0;
    int wlo = rlo[0], whi = rhi[0];
    lev_win[0] = 0;
    for (int s = 1; s < L; ++s) {
      if (rhi[s] >= wlo - 1) {
        wlo = min(wlo, rlo[s]);
      } else {
        win_lo[nw] = wlo;
        win_base[nw] = cum;
        cum += whi - wlo + 1;
        ++nw;
        wlo = rlo[s];
        whi = rhi[s];
      }
      lev_win[s] = nw;
    }
    win_lo[nw] = wlo;
    win_base[nw] = cum;
    cum += whi - wlo + 1;
    ++nw;
    if (cum <= rows_cap || L == 1) break;
    --L;
  }
  for (int s = 0; s < L; ++s) lv_off[s] = win_base[lev_win[s]] - win_lo[lev_win[s]];
  win_base[nw] = cum;
  n_levels = L;
  n_windows = nw;
}

// Single-pass form of plan_levels for callers that know every level fits
// (no capacity check, no local arrays): ranges only move towards the root, so
// each new range either extends the open window downwards or closes it.
QA_DEVINL void plan_levels_fit(int q_lo, int nq, int max_depth, FastDiv div_b, int* lv_off,
                               int* win_lo, int* win_base, int& n_levels, int& n_windows) {
  int lo = q_lo, hi = q_lo + nq - 1;
  int wlo = lo, whi = hi, nw = 0, cum = 0, L = 1;
  lv_off[0] = 0;  // provisional window index, turned into an offset below
  while (L < kMaxLevels && L <= max_depth && hi > 0) {
    lo = int(fast_div(uint32_t(max(lo, 1) - 1), div_b));
    hi = int(fast_div(uint32_t(hi - 1), div_b));
    if (hi >= wlo - 1) {
      wlo = min(wlo, lo);
    } else {
      win_lo[nw] = wlo;
      win_base[nw] = cum;
      cum += whi - wlo + 1;
      ++nw;
      wlo = lo;
      whi = hi;
    }
    lv_off[L++] = nw;
  }
  win_lo[nw] = wlo;
  win_base[nw] = cum;
  cum += whi - wlo + 1;
  ++nw;
  win_base[nw] = cum;
  for (int s = 0; s < L; ++s) lv_off[s] = win_base[lv_off[s]] - win_lo[lv_off[s]];
  n_levels = L;
  n_windows = nw;
}

// Upper bound on the K/V rows plan_levels needs for a tile of mq queries.
// If level s-1 spans nodes [lo, lo + span], its parents span at most
// floor(span / b) + 1 nodes more than one, so span_s <= span_{s-1} / b + 1 and
// level s has at most span_s + 1 rows. A chain (b = 1) needs mq + depth rows:
// its levels overlap into one window.
inline int rows_needed(int mq, int b, int max_depth, bool parents) {
  if (parents || max_depth == 0) return mq;
  const int levels = max_depth < kMaxLevels - 1 ? max_depth : kMaxLevels - 1;
  if (b == 1) return mq + levels;
  int rows = mq, span = mq - 1;
  for (int s = 1; s <= levels; ++s) {
    span = span / b + 1;
    rows += span + 1;
  }
  return rows;
}

inline FastDiv make_fast_div(uint32_t d) {
  uint32_t l = 0;
  while ((1ull << l) < d) ++l;
  const uint64_t m = ((uint64_t(1) << 32) * ((uint64_t(1) << l) - d)) / d + 1;
  return FastDiv{uint32_t(m), l};
}

// ---------------------------------------------------------------------------
// Tile geometry of the tensor-core kernel (ancestor_tc.cu).
//
// A tile is up to kTileRows queries, listed in BFS order as level segments
// (each a contiguous node range inside one tree level). Two tilings:
//   * contiguous: tile t = nodes [64 t, 64 t + 64), split at level boundaries;
//   * subtree: the levels are cut, from the bottom, into bands of h levels
//     (h = the most levels whose complete subtree has at most 64 nodes; the
//     top band keeps the remainder), and each band into complete subtrees
//     rooted on its first level; a tile holds k sibling subtrees (roots
//     [F(R) + u k, + k) on the band's root level R), one segment per level.
//     Such a tile is closed under the parent rule except for its roots' path
//     to the root, so it stages ~its own rows plus a few path rows, where a
//     contiguous tile of a deep binary tree stages its own rows plus about as
//     many ancestors again.
// The staged K/V rows of a tile, and the key list of each warp, are planned
// level by level from the deepest level up: needed(L) = own(L) + parents of
// needed(L + 1), kept as at most two intervals (the closest ones merged when
// there are more: staging a few extra rows is harmless), merged into windows
// of consecutive nodes in descending node order. The host runs the same
// planner over every tile of the launch's tree to size shared memory and the
// key lists exactly.
// ---------------------------------------------------------------------------
#define QA_HD __host__ __device__ __forceinline__

constexpr int kTileRows = 64;
constexpr int kMaxWin = 32;  // windows per plan (the last one absorbs any excess)

constexpr int kMaxBands = 8;

struct TileGeom {
  int32_t b;
  int32_t levels;      // levels of a tree of max_seqlen nodes
  int32_t top_tiles;   // contiguous tiles over nodes [0, top_nodes) (contiguous tiling)
  int32_t top_nodes;
  int32_t bands;       // subtree bands, top first (0: contiguous tiling)
  int32_t tiles;       // tiles per sequence
  int32_t band_root[kMaxBands];   // root level R of the band
  int32_t band_h[kMaxBands];      // levels per subtree
  int32_t band_k[kMaxBands];      // subtrees (roots) per tile
  int32_t band_tile0[kMaxBands + 1];  // first tile of the band
  int32_t first[kMaxLevels + 1];  // first node of each level (F(L)), saturated
};

struct HostDivB {
  uint32_t b;
  QA_HD uint32_t operator()(uint32_t x) const { return x / b; }
};
struct DevDivB {
  FastDiv f;
  QA_HD uint32_t operator()(uint32_t x) const {
#ifdef __CUDA_ARCH__
    return fast_div(x, f);
#else
    return uint32_t(((uint64_t(x) * f.m >> 32) + x) >> f.l);
#endif
  }
};

// Level segments of tile `tile` of a sequence of len nodes, in row order:
// seg_lo[i] first node, seg_row[i] first tile row, seg_row[nseg] = rows.
QA_HD int tile_segments(const TileGeom& g, int tile, int len, int* seg_lo, int* seg_row) {
  int n = 0, rows = 0;
  if (tile < g.top_tiles) {
    int lo = tile * kTileRows;
    const int hi = min(min(lo + kTileRows, g.top_nodes), len);  // exclusive
    int L = 0;
    while (L + 1 < g.levels && g.first[L + 1] <= lo) ++L;
    while (lo < hi) {
      const int end = min(hi, g.first[L + 1]);
      seg_lo[n] = lo;
      seg_row[n] = rows;
      rows += end - lo;
      ++n;
      lo = end;
      ++L;
    }
  } else {
    int bd = 0;
    while (bd + 1 < g.bands && g.band_tile0[bd + 1] <= tile) ++bd;
    const int u = tile - g.band_tile0[bd], R = g.band_root[bd];
    const int width = g.first[R + 1] - g.first[R];  // b^R roots
    const int k = min(g.band_k[bd], width - u * g.band_k[bd]);
    int off = u * g.band_k[bd], cnt = k;  // offset and count inside the level
    for (int i = 0; i < g.band_h[bd] && k > 0; ++i) {
      const int L = R + i;
      const int lo = g.first[L] + off;
      const int hi = min(lo + cnt, len);
      if (hi <= lo) break;
      seg_lo[n] = lo;
      seg_row[n] = rows;
      rows += hi - lo;
      ++n;
      if (hi < lo + cnt) break;  // the sequence ends inside this level
      off *= g.b;
      cnt *= g.b;
    }
  }
  seg_row[n] = rows;
  return n;
}

// Level of the node (first[L] <= node < first[L + 1]).
QA_HD int node_level(const TileGeom& g, int node) {
  int L = 0;
  while (L + 1 < g.levels && g.first[L + 1] <= node) ++L;
  return L;
}

// Windows (descending node order) holding every ancestor, within max_depth
// steps, of tile rows [r0, r1); segment i lies on level level(seg 0) + i.
// Returns the number of staged rows; win_base[nwin] = that count. The needed
// nodes of a level are kept as at most two intervals A (upper) and B (lower)
// in registers; a third disjoint interval is merged into its nearer
// neighbour (a few extra staged rows, never a missing one).
template <class DivB>
QA_HD int plan_rows(const TileGeom& g, const int* seg_lo, const int* seg_row, int nseg, int r0, int r1,
                    int max_depth, DivB divb, int* win_lo, int* win_base, int& nwin) {
  nwin = 0;
  if (r1 <= r0 || nseg <= 0) {
    win_base[0] = 0;
    return 0;
  }
  int i0 = 0;
  while (i0 + 1 < nseg && seg_row[i0 + 1] <= r0) ++i0;
  int i1 = i0;
  while (i1 + 1 < nseg && seg_row[i1 + 1] < r1) ++i1;
  const int lev0 = node_level(g, seg_lo[0]);
  const int lev_min = max(0, lev0 + i0 - max_depth);
  int alo = 0, ahi = -1, blo = 0, bhi = -1;  // empty when hi < lo
  int open_hi = -1, cum = 0;
  for (int i = i1, L = lev0 + i1; L >= lev_min; --L, --i) {
    if (ahi >= alo) {  // parents of level L + 1 (every node there is >= 1)
      alo = int(divb(uint32_t(alo - 1)));
      ahi = int(divb(uint32_t(ahi - 1)));
    }
    if (bhi >= blo) {
      blo = int(divb(uint32_t(blo - 1)));
      bhi = int(divb(uint32_t(bhi - 1)));
      if (bhi >= alo - 1) {
        alo = min(alo, blo);
        blo = 0;
        bhi = -1;
      }
    }
    if (i >= i0) {  // the rows' own piece of this level
      const int olo = seg_lo[i] + max(r0 - seg_row[i], 0);
      const int ohi = seg_lo[i] + min(r1, seg_row[i + 1]) - 1 - seg_row[i];
      int clo = 0, chi = -1;
      if (ahi < alo) {
        alo = olo;
        ahi = ohi;
      } else if (ohi > ahi) {
        clo = blo; chi = bhi; blo = alo; bhi = ahi; alo = olo; ahi = ohi;
      } else if (bhi < blo || ohi > bhi) {
        clo = blo; chi = bhi; blo = olo; bhi = ohi;
      } else {
        clo = olo; chi = ohi;
      }
      // A, B, C sorted by upper end: merge touching neighbours
      if (bhi >= blo && bhi >= alo - 1) {
        alo = min(alo, blo);
        blo = clo; bhi = chi; clo = 0; chi = -1;
      }
      if (bhi >= blo && bhi >= alo - 1) {
        alo = min(alo, blo);
        blo = 0; bhi = -1;
      }
      if (chi >= clo && chi >= blo - 1) {
        blo = min(blo, clo);
        clo = 0; chi = -1;
      }
      if (chi >= clo) {  // three disjoint intervals: close the smaller gap
        if (alo - bhi <= blo - chi) {
          alo = blo; blo = clo; bhi = chi;
        } else {
          blo = clo;
        }
      }
    }
    // append A then B to the windows (levels below hold smaller nodes)
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int lo = k ? blo : alo, hi = k ? bhi : ahi;
      if (hi < lo) continue;
      if (nwin > 0 && (hi >= win_lo[nwin - 1] - 1 || nwin == kMaxWin)) {
        win_lo[nwin - 1] = min(win_lo[nwin - 1], lo);
      } else {
        if (nwin > 0) cum += open_hi - win_lo[nwin - 1] + 1;
        win_lo[nwin] = lo;
        win_base[nwin] = cum;
        open_hi = hi;
        ++nwin;
      }
    }
    if ((bhi >= blo ? blo : alo) == 0) break;  // the root is planned
  }
  cum += open_hi - win_lo[nwin - 1] + 1;
  win_base[nwin] = cum;
  return cum;
}

// Geometry for a tree of n nodes (n >= 1, b >= 2): contiguous tiling, plus the
// subtree tiling when it applies (bands > 0).
inline TileGeom make_tile_geom(int b, int n, bool subtree) {
  TileGeom g{};
  g.b = b;
  int L = 0;
  int64_t f = 0;
  g.first[0] = 0;
  while (f < n && L < kMaxLevels) {
    f = f * b + 1;
    ++L;
    g.first[L] = int(f < (int64_t(1) << 30) ? f : (int64_t(1) << 30));
  }
  for (int i = L + 1; i <= kMaxLevels; ++i) g.first[i] = 1 << 30;
  g.levels = L;
  g.top_nodes = n;
  g.top_tiles = (n + kTileRows - 1) / kTileRows;
  g.bands = 0;
  g.tiles = g.top_tiles;
  if (subtree && b >= 2) {
    int h = 1;
    while (h + 1 <= L && g.first[h + 1] <= kTileRows) ++h;  // F(h) nodes per subtree
    const int nb = (L + h - 1) / h;                          // bands; the top one keeps L - (nb-1) h levels
    if (nb >= 2 && nb <= kMaxBands) {
      g.top_nodes = 0;
      g.top_tiles = 0;
      g.bands = nb;
      int tiles = 0;
      for (int i = 0; i < nb; ++i) {
        const int R = i == 0 ? 0 : L - (nb - i) * h;
        const int H = i == 0 ? L - (nb - 1) * h : h;
        g.band_root[i] = R;
        g.band_h[i] = H;
        g.band_k[i] = kTileRows / g.first[H];
        g.band_tile0[i] = tiles;
        const int roots = g.first[R + 1] - g.first[R];
        tiles += (roots + g.band_k[i] - 1) / g.band_k[i];
      }
      g.band_tile0[nb] = tiles;
      g.tiles = tiles;
    }
  }
  return g;
}

// Largest staged-row count of a tile and key-list length of a 16-row warp
// over every tile of an n-node tree (shorter sequences plan subsets).
inline void tile_geom_caps(const TileGeom& g, int n, int max_depth, int& rows_cap, int& keys_cap) {
  int seg_lo[kMaxLevels + 1], seg_row[kMaxLevels + 2], wl[kMaxWin + 1], wb[kMaxWin + 1], nw = 0;
  rows_cap = 0;
  keys_cap = 0;
  const HostDivB div{uint32_t(g.b)};
  for (int t = 0; t < g.tiles; ++t) {
    const int ns = tile_segments(g, t, n, seg_lo, seg_row);
    const int rows = seg_row[ns];
    if (rows == 0) continue;
    rows_cap = max(rows_cap, plan_rows(g, seg_lo, seg_row, ns, 0, rows, max_depth, div, wl, wb, nw));
    for (int w = 0; w * 16 < rows; ++w)
      keys_cap = max(keys_cap, plan_rows(g, seg_lo, seg_row, ns, 16 * w, min(rows, 16 * w + 16), max_depth, div,
                                         wl, wb, nw));
  }
}

// Tensor-core level kernel for complete-tree mode (ancestor_tc.cu): returns
// QA_OK / a QA_ERR_* code, or kTcNotApplicable when the scalar walk must run.
constexpr int kTcNotApplicable = 1;
int ancestor_tc_launch(const qa_ancestor_args& a, cudaStream_t stream);

}  // namespace qa
