// Ancestor-walk attention for tree verification (kernel A1), sm_100a.
//
// Behaviour follows the reference's Triton kernels
//   _ragged_attn_sparse_kernel      src/ragged_attn.py:267-387  (formula parents)
//   _ragged_attn_sparse_kernel_lse  src/ragged_attn.py:401-496  (+ LSE)
//   _ragged_attn_parents_kernel_lse src/ragged_attn.py:593-713  (explicit parents)
// i.e. softmax attention of each query over its own row and its ancestors,
// with the parent rule parent(a) = max(a-1,0)/b applied before the divide
// (:333-337, :377), max_depth+1 walk steps, and the walk ending where a step
// would revisit the previous node (:340: root, or a root self-loop in parents
// mode). The reference's `l == 0 -> 1` guard (:380) cannot trigger: every
// valid query attends at least to itself.
//
// B200 design (not a translation of the Triton tiling):
//   * One CTA = (sequence, query head, tile of MQ consecutive BFS queries),
//     CTAs ordered head-fastest so concurrently running CTAs stream the same
//     tokens' rows of all heads (contiguous [T, H, D] memory).
//   * In a complete b-ary BFS tree the step-s ancestors of a contiguous query
//     range are the contiguous node range [anc^s(first), anc^s(last)]. The CTA
//     computes these level ranges, merges overlapping ones into windows, and
//     stages the tile's Q rows plus every window's K and V rows in shared
//     memory with 16-byte cp.async copies issued all at once (maximal bytes in
//     flight, no register cost). Each level s then has one offset with
//     slot = off[s] + node, so the walk loop addresses shared memory
//     uniformly: no per-step branches or range checks. Ancestor rows are other
//     tiles' own rows, so the extra reads hit L2; HBM sees each row once.
//   * Walk: parent by multiply-high division (no integer divide), q.k and p.v
//     with sm_100 mixed-precision FMA (16-bit inputs, fp32 accumulation, no
//     conversions on the fp16 path), and a lazy online softmax that rescales
//     the running sum only when a score exceeds the reference maximum by more
//     than 2^8 (the result is exact: only the reference point moves).
//   * D/16 lanes per query, 16 elements per lane as two 16-byte chunks at
//     element 8*lane and D/2 + 8*lane (conflict-free shared loads).
//   * Explicit-parent mode and levels beyond the staged ones (very deep
//     walks) read ancestor rows from global memory in a second loop.
//   * No tensor cores (a gather with ~2.8 flop per HBM byte), no global
//     scratch, no atomics, no spin-waits.
#include "ancestor_plan.cuh"

namespace qa {
namespace {

constexpr int kThreads = 256;
constexpr int kOwnBytes = 16 * 1024;  // Q rows per tile: MQ = kOwnBytes / (2 * D)
constexpr float kLazy = 8.f;          // rescale threshold, log2 units

struct AncParams {
  qa_ancestor_args a;
  float scale_log2;   // scale * log2(e)
  int32_t tiles_per_seq;
  int32_t head_ratio;
  int32_t rows_cap;   // K/V rows of shared memory per CTA
  FastDiv div_b;      // division by the branching factor
};

template <int D> struct Tile {
  static constexpr int LPI = D / 16;              // lanes per query
  static constexpr int QPP = kThreads / LPI;      // queries per pass
  static constexpr int MQ = kOwnBytes / (2 * D);  // queries per tile
  static constexpr int RC = D / 8;                // 16-byte chunks per row
};

template <typename T, int D>
QA_DEVINL void lds_row(const T* row, int li, uint4& lo, uint4& hi) {
  lo = *reinterpret_cast<const uint4*>(row + li * 8);
  hi = *reinterpret_cast<const uint4*>(row + D / 2 + li * 8);
}

template <typename T, int D>
QA_DEVINL void ldg_row(const T* row, int li, uint4& lo, uint4& hi) {
  lo = ld_shared_row(row + li * 8);
  hi = ld_shared_row(row + D / 2 + li * 8);
}

template <typename T>
QA_DEVINL float dot16(const uint4& qa, const uint4& qb, const uint4& ka, const uint4& kb) {
  float s0 = 0.f, s1 = 0.f;
  dot_pair<T>(s0, qa.x, ka.x);
  dot_pair<T>(s1, qa.y, ka.y);
  dot_pair<T>(s0, qa.z, ka.z);
  dot_pair<T>(s1, qa.w, ka.w);
  dot_pair<T>(s0, qb.x, kb.x);
  dot_pair<T>(s1, qb.y, kb.y);
  dot_pair<T>(s0, qb.z, kb.z);
  dot_pair<T>(s1, qb.w, kb.w);
  return s0 + s1;
}

// acc += p * v over 16 elements; returns the weight actually applied.
// fp16: p is rounded to fp16 once and applied with mixed-precision FMA (the
// same rounded weight enters the softmax denominator, so the normalisation is
// consistent). bf16: V is widened to fp32 (exact) and p stays fp32.
template <typename T> struct PV;
template <> struct PV<__half> {
  QA_DEVINL static float apply(float (&acc)[16], float p, const uint4& va, const uint4& vb) {
    const __half ph = __float2half_rn(p);
    const unsigned short pb = __half_as_ushort(ph);
    const uint32_t w[8] = {va.x, va.y, va.z, va.w, vb.x, vb.y, vb.z, vb.w};
#pragma unroll
    for (int i = 0; i < 8; ++i)
      asm("{.reg .b16 v0, v1;\n\t"
          "mov.b32 {v0, v1}, %2;\n\t"
          "fma.rn.f32.f16 %0, v0, %3, %0;\n\t"
          "fma.rn.f32.f16 %1, v1, %3, %1;}"
          : "+f"(acc[2 * i]), "+f"(acc[2 * i + 1]) : "r"(w[i]), "h"(pb));
    return p;  // the denominator keeps the exact weight (LSE stays fp32-accurate)
  }
};
template <> struct PV<__nv_bfloat16> {
  QA_DEVINL static float apply(float (&acc)[16], float p, const uint4& va, const uint4& vb) {
    const uint32_t w[8] = {va.x, va.y, va.z, va.w, vb.x, vb.y, vb.z, vb.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      acc[2 * i] = fmaf(p, __uint_as_float(w[i] << 16), acc[2 * i]);
      acc[2 * i + 1] = fmaf(p, __uint_as_float(w[i] & 0xffff0000u), acc[2 * i + 1]);
    }
    return p;
  }
};

// Running softmax state of one query (log2 units, lazy reference maximum).
struct SoftState {
  float m;  // reference maximum (-inf before the first key)
  float l;  // sum of weights relative to m
  float acc[16];
};

template <typename T, int LPI>
QA_DEVINL void softmax_step(SoftState& st, float s, const uint4& va, const uint4& vb) {
  if (s > st.m + kLazy) {  // also taken for the first key (m = -inf)
    const float alpha = fast_exp2(st.m - s);
    st.l *= alpha;
#pragma unroll
    for (int e = 0; e < 16; ++e) st.acc[e] *= alpha;
    st.m = s;
  }
  st.l += PV<T>::apply(st.acc, fast_exp2(s - st.m), va, vb);
}

template <int LPI>
QA_DEVINL float reduce_lanes(float s, unsigned mask) {
#pragma unroll
  for (int off = LPI / 2; off > 0; off >>= 1) s += __shfl_xor_sync(mask, s, off);
  return s;
}

// Element offsets of the K and V rows of sequence `seq`'s node `node`: packed
// K/V at token kv0 + node, or (paged) slot (kv_offset + node) % page_size of the
// physical page the sequence's page-table row names for it.
QA_DEVINL void kv_offsets(const qa_ancestor_args& a, int seq, int kv0, int node, int64_t& ko, int64_t& vo) {
  if (a.page_table == nullptr) {
    const int64_t tk = int64_t(kv0) + node;
    ko = tk * a.k_stride_t;
    vo = tk * a.v_stride_t;
  } else {
    const int pos = a.kv_offset + node;
    const int64_t page = __ldg(a.page_table + int64_t(seq) * a.page_table_stride + pos / a.page_size);
    const int slot = pos % a.page_size;
    ko = page * a.k_stride_page + int64_t(slot) * a.k_stride_t;
    vo = page * a.v_stride_page + int64_t(slot) * a.v_stride_t;
  }
}

template <typename T, int D, bool PARENTS>
__global__ void __launch_bounds__(kThreads) ancestor_attn_kernel(const AncParams p) {
  using TL = Tile<D>;
  constexpr int LPI = TL::LPI, MQ = TL::MQ, RC = TL::RC;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  T* sQ = reinterpret_cast<T*>(smem_raw);
  T* sK = sQ + MQ * D;
  T* sV = sK + p.rows_cap * D;
  __shared__ int lv_off[kMaxLevels];      // slot = lv_off[s] + node for staged level s
  __shared__ int win_lo[kMaxLevels + 1];  // staged windows: first node, first slot
  __shared__ int win_base[kMaxLevels + 1];
  __shared__ int n_staged, n_win;

  const qa_ancestor_args& a = p.a;
  const int h = int(blockIdx.x % unsigned(a.num_q_heads));
  const int rest = int(blockIdx.x / unsigned(a.num_q_heads));
  const int tile = rest % p.tiles_per_seq;
  const int seq = rest / p.tiles_per_seq;
  const int q0 = __ldg(a.cu_seqlens_q + seq);
  const int len = __ldg(a.cu_seqlens_q + seq + 1) - q0;
  const int q_lo = tile * MQ;
  if (q_lo >= len) return;  // uniform over the CTA
  const int nq = min(MQ, len - q_lo);
  const int kv0 = (a.cu_seqlens_kv ? __ldg(a.cu_seqlens_kv + seq) : q0) + a.kv_offset;
  const int hk = h / p.head_ratio;
  const T* Qh = reinterpret_cast<const T*>(a.q) + int64_t(h) * a.q_stride_h;
  const T* Kh = reinterpret_cast<const T*>(a.k) + int64_t(hk) * a.k_stride_h;
  const T* Vh = reinterpret_cast<const T*>(a.v) + int64_t(hk) * a.v_stride_h;
  const int tid = threadIdx.x;

  // ---- plan: level ranges -> merged windows -> slot offsets (one thread) ----
  if (tid == 0) {
    int ns = 0, nw = 0;
    plan_levels(q_lo, nq, PARENTS ? 0 : a.max_depth, p.div_b, p.rows_cap, lv_off, win_lo, win_base, ns, nw);
    n_staged = ns;
    n_win = nw;
  }

  // ---- stage the tile's Q rows ----
  for (int c = tid; c < nq * RC; c += kThreads) {
    const int r = c / RC, cc = c - r * RC;
    cp_async16(sQ + r * D + cc * 8, Qh + q_seq_off(a, seq, q0) + int64_t(q_lo + r) * a.q_stride_t + cc * 8);
  }
  __syncthreads();
  // ---- stage every window's K and V rows ----
  const int nw = n_win, nrows = win_base[nw];
  for (int c = tid; c < nrows * RC; c += kThreads) {
    const int j = c / RC, cc = c - j * RC;
    int w = 0;
    while (w + 1 < nw && win_base[w + 1] <= j) ++w;
    int64_t ko, vo;
    kv_offsets(a, seq, kv0, win_lo[w] + (j - win_base[w]), ko, vo);
    cp_async16(sK + j * D + cc * 8, Kh + ko + cc * 8);
    cp_async16(sV + j * D + cc * 8, Vh + vo + cc * 8);
  }
  cp_async_wait_all();
  __syncthreads();

  // ---- walk: LPI lanes per query, 16 elements per lane ----
  const int lane = tid & 31;
  const int li = lane & (LPI - 1);
  const unsigned mask =
      (LPI == 32) ? 0xffffffffu : (((1u << LPI) - 1u) << (lane & ~(LPI - 1)));
  const int nst = n_staged;
  // next node of the walk, or -1 where the walk ends (root / self-loop / depth)
  auto advance = [&](int node, int s) -> int {
    if (s >= a.max_depth) return -1;
    if constexpr (PARENTS) {
      const int nx = __ldg(a.parents + q0 + node);
      return (nx == node || nx < 0 || nx >= len) ? -1 : nx;
    } else {
      return node == 0 ? -1 : int(fast_div(uint32_t(node - 1), p.div_b));
    }
  };
  for (int qi = tid / LPI; qi < nq; qi += TL::QPP) {  // uniform over a query's lanes
    const int q = q_lo + qi;
    const int64_t t = int64_t(q0) + q;
    uint4 qa, qb;
    lds_row<T, D>(sQ + qi * D, li, qa, qb);
    SoftState st;
    st.m = -INFINITY;
    st.l = 0.f;
#pragma unroll
    for (int e = 0; e < 16; ++e) st.acc[e] = 0.f;
    if (a.prefix_o != nullptr) {
      // merge source: a prior result over other keys = one extra key of
      // weight exp(prefix_lse) and value prefix_o
      const float pl = __ldg(a.prefix_lse + t * a.prefix_lse_stride_t + int64_t(h) * a.prefix_lse_stride_h);
      if (pl > -INFINITY) {
        uint4 pa, pb;
        ldg_row<T, D>(reinterpret_cast<const T*>(a.prefix_o) + t * a.prefix_o_stride_t +
                          int64_t(h) * a.prefix_o_stride_h, li, pa, pb);
        float f[8];
        Vec8<T>::to_f32(pa, f);
#pragma unroll
        for (int e = 0; e < 8; ++e) st.acc[e] = f[e];
        Vec8<T>::to_f32(pb, f);
#pragma unroll
        for (int e = 0; e < 8; ++e) st.acc[8 + e] = f[e];
        st.m = pl * kLog2e;
        st.l = 1.f;
      }
    }

    int node = q, s = 0;
    while (node >= 0 && s < nst) {  // staged levels: shared memory only
      const int slot = lv_off[s] + node;
      uint4 ka, kb, va, vb;
      lds_row<T, D>(sK + slot * D, li, ka, kb);
      lds_row<T, D>(sV + slot * D, li, va, vb);
      const float sc = reduce_lanes<LPI>(dot16<T>(qa, qb, ka, kb), mask) * p.scale_log2;
      softmax_step<T, LPI>(st, sc, va, vb);
      node = advance(node, s);
      ++s;
    }
    while (node >= 0) {  // explicit parents / levels past the staged ones
      int64_t ko, vo;
      kv_offsets(a, seq, kv0, node, ko, vo);
      uint4 ka, kb, va, vb;
      ldg_row<T, D>(Kh + ko, li, ka, kb);
      ldg_row<T, D>(Vh + vo, li, va, vb);
      const float sc = reduce_lanes<LPI>(dot16<T>(qa, qb, ka, kb), mask) * p.scale_log2;
      softmax_step<T, LPI>(st, sc, va, vb);
      node = advance(node, s);
      ++s;
    }

    // ---- epilogue: normalise, store O (and LSE) ----
    const float inv = 1.f / st.l;
    float o0[8], o1[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      o0[e] = st.acc[e] * inv;
      o1[e] = st.acc[8 + e] * inv;
    }
    T* ob = reinterpret_cast<T*>(a.o) + t * a.o_stride_t + int64_t(h) * a.o_stride_h;
    st_stream(ob + li * 8, Vec8<T>::from_f32(o0));
    st_stream(ob + D / 2 + li * 8, Vec8<T>::from_f32(o1));
    if (a.lse != nullptr && li == 0)
      a.lse[t * a.lse_stride_t + int64_t(h) * a.lse_stride_h] = (st.m + __log2f(st.l)) * kLn2;
  }
}

constexpr int kMaxSmem = 200 * 1024;

template <typename T, int D>
cudaError_t launch_d(AncParams& p, bool parents, cudaStream_t st) {
  using TL = Tile<D>;
  const int64_t blocks = int64_t(p.a.batch) * p.tiles_per_seq * p.a.num_q_heads;
  if (blocks > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
  const int row_bytes = 2 * D * int(sizeof(T));  // one K row + one V row
  const int cap_max = (kMaxSmem - TL::MQ * D * int(sizeof(T))) / row_bytes;
  int cap = rows_needed(TL::MQ, p.a.branching, p.a.max_depth, parents);
  p.rows_cap = cap < cap_max ? cap : cap_max;
  const int smem = TL::MQ * D * int(sizeof(T)) + p.rows_cap * row_bytes;
  auto kern = parents ? ancestor_attn_kernel<T, D, true> : ancestor_attn_kernel<T, D, false>;
  {
    const cudaError_t e = qa_smem_attr(reinterpret_cast<const void*>(kern), kMaxSmem);
    if (e != cudaSuccess) return e;
  }
  kern<<<dim3{unsigned(blocks)}, kThreads, smem, st>>>(p);
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_t(AncParams& p, bool parents, cudaStream_t st) {
  switch (p.a.head_dim) {
    case 32: return launch_d<T, 32>(p, parents, st);
    case 64: return launch_d<T, 64>(p, parents, st);
    case 128: return launch_d<T, 128>(p, parents, st);
    default: return launch_d<T, 256>(p, parents, st);
  }
}

bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }
bool stride_ok(int64_t s) { return (s % 8) == 0; }  // 8 elements = 16 bytes

}  // namespace
}  // namespace qa

extern "C" int qa_ancestor_attn(const qa_ancestor_args* args, void* stream) {
  using namespace qa;
  if (args == nullptr) return QA_ERR_INVALID;
  const qa_ancestor_args& a = *args;
  if (a.batch < 0 || a.num_q_heads <= 0 || a.num_kv_heads <= 0 || a.max_depth < 0 ||
      a.max_seqlen < 0)
    return QA_ERR_INVALID;
  if (a.num_q_heads % a.num_kv_heads != 0) return QA_ERR_INVALID;
  if (a.parents == nullptr && a.branching < 1) return QA_ERR_INVALID;
  if (a.dtype != QA_DTYPE_F16 && a.dtype != QA_DTYPE_BF16) return QA_ERR_UNSUPPORTED;
  if (a.head_dim != 32 && a.head_dim != 64 && a.head_dim != 128 && a.head_dim != 256)
    return QA_ERR_UNSUPPORTED;
  if (a.batch == 0 || a.max_seqlen == 0) return QA_OK;
  if (!a.q || !a.k || !a.v || !a.o || !a.cu_seqlens_q) return QA_ERR_INVALID;
  if ((a.prefix_o == nullptr) != (a.prefix_lse == nullptr)) return QA_ERR_INVALID;
  if (!aligned16(a.q) || !aligned16(a.k) || !aligned16(a.v) || !aligned16(a.o) ||
      (a.prefix_o && !aligned16(a.prefix_o)))
    return QA_ERR_ALIGN;
  if (!stride_ok(a.q_stride_t) || !stride_ok(a.q_stride_h) || !stride_ok(a.q_stride_b) || !stride_ok(a.k_stride_t) ||
      !stride_ok(a.k_stride_h) || !stride_ok(a.v_stride_t) || !stride_ok(a.v_stride_h) ||
      !stride_ok(a.o_stride_t) || !stride_ok(a.o_stride_h))
    return QA_ERR_ALIGN;
  if (a.prefix_o && (!stride_ok(a.prefix_o_stride_t) || !stride_ok(a.prefix_o_stride_h)))
    return QA_ERR_ALIGN;

  AncParams p;
  p.a = a;
  p.scale_log2 = a.scale * kLog2e;
  p.head_ratio = a.num_q_heads / a.num_kv_heads;
  const int mq = kOwnBytes / (2 * a.head_dim);
  p.tiles_per_seq = (a.max_seqlen + mq - 1) / mq;
  const bool parents = a.parents != nullptr;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (a.page_table != nullptr) {  // paged K/V: both kernels look the rows up in the page table
    if (a.page_size <= 0 || a.page_table_stride < 0) return QA_ERR_INVALID;
    if (!stride_ok(a.k_stride_page) || !stride_ok(a.v_stride_page)) return QA_ERR_ALIGN;
  }
  const int tc = ancestor_tc_launch(a, st);
  if (tc != kTcNotApplicable) return tc;
  p.div_b = make_fast_div(uint32_t(parents ? 1 : a.branching));
  cudaError_t e = (a.dtype == QA_DTYPE_F16) ? launch_t<__half>(p, parents, st)
                                            : launch_t<__nv_bfloat16>(p, parents, st);
  return e == cudaSuccess ? QA_OK : QA_ERR_LAUNCH;
}
