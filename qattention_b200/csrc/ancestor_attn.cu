// Ancestor-walk attention for tree verification (kernel A1), sm_100a.
//
// Behaviour follows the reference's Triton kernels
//   _ragged_attn_sparse_kernel      src/ragged_attn.py:267-387  (formula parents)
//   _ragged_attn_sparse_kernel_lse  src/ragged_attn.py:401-496  (+ LSE)
//   _ragged_attn_parents_kernel_lse src/ragged_attn.py:593-713  (explicit parents)
// i.e. FlashAttention-2 online softmax over the query's own row and its
// ancestors, with the parent rule parent(a) = max(a-1,0)/b applied before the
// divide (:333-337, :377) and a step skipped when it revisits the previous
// node (:340). The reference's `l == 0 -> 1` guard (:380) cannot trigger here
// because every valid query attends at least to itself.
//
// B200 design (not a translation of the Triton tiling):
//   * Work item = (sequence, sibling group, query head). In a complete b-ary
//     BFS tree the children of node p are the consecutive nodes
//     p*b+1 .. p*b+b, and from step 1 on they share every ancestor. One item
//     holds up to G siblings' queries in registers and streams each shared
//     ancestor K/V row once for all of them, so on-chip traffic for the
//     ancestor part drops by G. Own rows (step 0) are read with L1 bypass
//     since no other item needs them; ancestor rows go through L1/L2.
//   * D/8 lanes per item, each lane owning 8 contiguous elements (one 16-byte
//     vector) of the head dimension. Items are ordered head-fastest, so one
//     warp instruction touches adjacent heads of the same token: contiguous
//     512 B - 1 KB of the [T, H, D] row-major layout.
//   * Ancestor indices of the formula mode are pure arithmetic, so the K and V
//     rows of P ancestor steps are issued back to back before any math
//     (memory-level parallelism instead of a dependent load chain).
//   * No tensor cores: the work is a gather with ~2.8 flop per HBM byte.
//   * No scratch memory, no atomics, no spin-waits.
#include "qa_common.cuh"

#include <algorithm>

namespace qa {
namespace {

struct AncParams {
  qa_ancestor_args a;
  float scale_log2;  // scale * log2(e)
  int32_t groups_per_seq;
  int32_t chunks;    // sibling chunks per parent (formula mode)
  int32_t head_ratio;
  int64_t total_items;
};

constexpr int kThreads = 256;
constexpr int kBatch = 4;  // ancestor steps whose rows are loaded together

template <typename T, int D, int G, bool PARENTS>
__global__ void __launch_bounds__(kThreads) ancestor_attn_kernel(const AncParams p) {
  constexpr int LPI = D / 8;            // lanes per item
  const int lane = threadIdx.x & 31;
  const int li = lane & (LPI - 1);      // lane within item
  const unsigned mask =
      (LPI == 32) ? 0xffffffffu : (((1u << LPI) - 1u) << (lane & ~(LPI - 1)));

  const int64_t item = (int64_t(blockIdx.x) * kThreads + threadIdx.x) / LPI;
  if (item >= p.total_items) return;
  const qa_ancestor_args& a = p.a;
  const int h = int(item % a.num_q_heads);
  const int64_t rest = item / a.num_q_heads;
  const int grp = int(rest % p.groups_per_seq);
  const int seq = int(rest / p.groups_per_seq);

  const int q0 = __ldg(a.cu_seqlens_q + seq);
  const int len = __ldg(a.cu_seqlens_q + seq + 1) - q0;
  const int kv0 = (a.cu_seqlens_kv ? __ldg(a.cu_seqlens_kv + seq) : q0) + a.kv_offset;

  // ---- which queries this item owns, and their shared first ancestor ----
  int first, cnt, par;
  if constexpr (PARENTS) {
    first = grp;
    if (first >= len) return;
    cnt = 1;
    const int pp = __ldg(a.parents + q0 + first);
    par = (pp == first || pp < 0 || pp >= len) ? -1 : pp;
  } else {
    const int b = a.branching;
    if (grp == 0) {
      first = 0;
      cnt = 1;
      par = -1;  // root: max(0-1,0)/b == 0 revisits itself
    } else {
      const int pg = (grp - 1) / p.chunks;
      const int c = (grp - 1) - pg * p.chunks;
      first = pg * b + 1 + c * G;
      if (first >= len) return;
      cnt = min(min(G, b - c * G), len - first);
      par = pg;
    }
  }
  if (a.max_depth == 0) par = -1;

  const int hk = h / p.head_ratio;
  const T* qb = reinterpret_cast<const T*>(a.q) + int64_t(h) * a.q_stride_h + li * 8;
  const T* kb = reinterpret_cast<const T*>(a.k) + int64_t(hk) * a.k_stride_h + li * 8;
  const T* vb = reinterpret_cast<const T*>(a.v) + int64_t(hk) * a.v_stride_h + li * 8;

  // ---- own rows (step 0): Q, K, V of each sibling ----
  float q[G][8];
  float m[G], l[G], acc[G][8];
  uint4 kown[G], vown[G];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    if (g < cnt) {
      const int64_t t = int64_t(q0) + first + g;
      const int64_t tk = int64_t(kv0) + first + g;
      uint4 qr = ld_stream(qb + t * a.q_stride_t);
      kown[g] = ld_stream(kb + tk * a.k_stride_t);
      vown[g] = ld_stream(vb + tk * a.v_stride_t);
      Vec8<T>::to_f32(qr, q[g]);
    } else {
      kown[g] = vown[g] = make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int e = 0; e < 8; ++e) q[g][e] = 0.f;
    }
  }
  // Optional merge source: a prior attention result over other keys, folded in
  // as one extra "key" whose weight is exp(prefix_lse) and value is prefix_o.
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[g][e] = 0.f;
    if (a.prefix_o != nullptr && g < cnt) {
      const int64_t t = int64_t(q0) + first + g;
      const float pl = __ldg(a.prefix_lse + t * a.prefix_lse_stride_t +
                             int64_t(h) * a.prefix_lse_stride_h);
      if (pl > -INFINITY) {
        const T* po = reinterpret_cast<const T*>(a.prefix_o) + t * a.prefix_o_stride_t +
                      int64_t(h) * a.prefix_o_stride_h + li * 8;
        uint4 pr = ld_stream(po);
        Vec8<T>::to_f32(pr, acc[g]);
        m[g] = pl * kLog2e;
        l[g] = 1.f;
      }
    }
  }

  // step 0 update
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float kf[8], vf[8];
    Vec8<T>::to_f32(kown[g], kf);
    float s = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) s = fmaf(q[g][e], kf[e], s);
#pragma unroll
    for (int off = LPI / 2; off > 0; off >>= 1) s += __shfl_xor_sync(mask, s, off);
    s *= p.scale_log2;
    if (g < cnt) {
      Vec8<T>::to_f32(vown[g], vf);
      const float mx = fmaxf(m[g], s);
      const float alpha = fast_exp2(m[g] - mx);
      const float pr = fast_exp2(s - mx);
      l[g] = l[g] * alpha + pr;
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[g][e] = fmaf(pr, vf[e], acc[g][e] * alpha);
      m[g] = mx;
    }
  }

  // ---- shared ancestor steps 1..max_depth, kBatch rows at a time ----
  int anc = par;
  int remaining = a.max_depth;
  while (anc >= 0 && remaining > 0) {
    int idx[kBatch];
    bool val[kBatch];
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      val[j] = (anc >= 0) && (j < remaining);
      idx[j] = anc;
      if (val[j]) {
        int nx;
        if constexpr (PARENTS) {
          nx = __ldg(a.parents + q0 + anc);
          if (nx == anc || nx < 0 || nx >= len) nx = -1;
        } else {
          nx = (anc == 0) ? -1 : (anc - 1) / a.branching;
        }
        anc = nx;
      }
    }
    remaining -= kBatch;
    uint4 kr[kBatch], vr[kBatch];
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      if (val[j]) {
        const int64_t tk = int64_t(kv0) + idx[j];
        kr[j] = ld_shared_row(kb + tk * a.k_stride_t);
        vr[j] = ld_shared_row(vb + tk * a.v_stride_t);
      } else {
        kr[j] = vr[j] = make_uint4(0, 0, 0, 0);
      }
    }
    float sc[G][kBatch];
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      float kf[8];
      Vec8<T>::to_f32(kr[j], kf);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float s = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) s = fmaf(q[g][e], kf[e], s);
        sc[g][j] = s;
      }
    }
#pragma unroll
    for (int j = 0; j < kBatch; ++j)
#pragma unroll
      for (int g = 0; g < G; ++g) {
#pragma unroll
        for (int off = LPI / 2; off > 0; off >>= 1)
          sc[g][j] += __shfl_xor_sync(mask, sc[g][j], off);
        sc[g][j] = val[j] ? sc[g][j] * p.scale_log2 : -INFINITY;
      }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float mx = m[g];
#pragma unroll
      for (int j = 0; j < kBatch; ++j) mx = fmaxf(mx, sc[g][j]);
      const float alpha = fast_exp2(m[g] - mx);
      l[g] *= alpha;
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[g][e] *= alpha;
      m[g] = mx;
    }
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      float vf[8];
      Vec8<T>::to_f32(vr[j], vf);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float pr = fast_exp2(sc[g][j] - m[g]);  // 0 for masked steps
        l[g] += pr;
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[g][e] = fmaf(pr, vf[e], acc[g][e]);
      }
    }
  }

  // ---- epilogue: normalise, store O (and LSE) ----
#pragma unroll
  for (int g = 0; g < G; ++g) {
    if (g < cnt) {
      const int64_t t = int64_t(q0) + first + g;
      const float inv = 1.f / l[g];
      float o[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = acc[g][e] * inv;
      T* ob = reinterpret_cast<T*>(a.o) + t * a.o_stride_t + int64_t(h) * a.o_stride_h + li * 8;
      st_stream(ob, Vec8<T>::from_f32(o));
      if (a.lse != nullptr && li == 0)
        a.lse[t * a.lse_stride_t + int64_t(h) * a.lse_stride_h] = (m[g] + __log2f(l[g])) * kLn2;
    }
  }
}

template <typename T, int D>
cudaError_t launch_d(const AncParams& p, int G, bool parents, cudaStream_t st) {
  constexpr int LPI = D / 8;
  const int64_t threads = p.total_items * LPI;
  const int64_t blocks = (threads + kThreads - 1) / kThreads;
  if (blocks > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
  const dim3 grid{unsigned(blocks)};
  if (parents) {
    ancestor_attn_kernel<T, D, 1, true><<<grid, kThreads, 0, st>>>(p);
  } else if (G == 1) {
    ancestor_attn_kernel<T, D, 1, false><<<grid, kThreads, 0, st>>>(p);
  } else if (G == 2) {
    ancestor_attn_kernel<T, D, 2, false><<<grid, kThreads, 0, st>>>(p);
  } else {
    ancestor_attn_kernel<T, D, 4, false><<<grid, kThreads, 0, st>>>(p);
  }
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_t(const AncParams& p, int G, bool parents, cudaStream_t st) {
  switch (p.a.head_dim) {
    case 32: return launch_d<T, 32>(p, G, parents, st);
    case 64: return launch_d<T, 64>(p, G, parents, st);
    case 128: return launch_d<T, 128>(p, G, parents, st);
    default: return launch_d<T, 256>(p, G, parents, st);
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
  if (!stride_ok(a.q_stride_t) || !stride_ok(a.q_stride_h) || !stride_ok(a.k_stride_t) ||
      !stride_ok(a.k_stride_h) || !stride_ok(a.v_stride_t) || !stride_ok(a.v_stride_h) ||
      !stride_ok(a.o_stride_t) || !stride_ok(a.o_stride_h))
    return QA_ERR_ALIGN;
  if (a.prefix_o && (!stride_ok(a.prefix_o_stride_t) || !stride_ok(a.prefix_o_stride_h)))
    return QA_ERR_ALIGN;

  AncParams p;
  p.a = a;
  p.scale_log2 = a.scale * kLog2e;
  p.head_ratio = a.num_q_heads / a.num_kv_heads;
  const bool parents = a.parents != nullptr;
  int G = 1;
  if (parents) {
    p.chunks = 1;
    p.groups_per_seq = a.max_seqlen;
  } else {
    const int b = a.branching;
    G = (b == 1) ? 1 : (b == 2 ? 2 : 4);
    p.chunks = (b + G - 1) / G;
    // group 0 = root, then `chunks` groups per parent p for p with p*b+1 < max_seqlen
    const int64_t parents_needed = a.max_seqlen > 1 ? (int64_t(a.max_seqlen) - 2) / b + 1 : 0;
    const int64_t gps = 1 + parents_needed * p.chunks;
    if (gps > 0x7fffffffLL) return QA_ERR_INVALID;
    p.groups_per_seq = int32_t(gps);
  }
  p.total_items = int64_t(a.batch) * p.groups_per_seq * a.num_q_heads;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e = (a.dtype == QA_DTYPE_F16) ? launch_t<__half>(p, G, parents, st)
                                            : launch_t<__nv_bfloat16>(p, G, parents, st);
  return e == cudaSuccess ? QA_OK : QA_ERR_LAUNCH;
}
