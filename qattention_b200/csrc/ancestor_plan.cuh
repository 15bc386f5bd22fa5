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

// Tensor-core level kernel for complete-tree mode (ancestor_tc.cu): returns
// QA_OK / a QA_ERR_* code, or kTcNotApplicable when the scalar walk must run.
constexpr int kTcNotApplicable = 1;
int ancestor_tc_launch(const qa_ancestor_args& a, cudaStream_t stream);

}  // namespace qa
