// Ancestor-walk attention, complete-tree mode, on tensor cores (mma.sync).
//
// Same result as the scalar walk in ancestor_attn.cu (and as the reference's
// _ragged_attn_sparse_kernel(_lse), src/ragged_attn.py:267-496, and its paged
// variant, :827-1004), organised so that per-query overhead disappears:
//   * Work item = (sequence, tile of <= 64 queries, query head). Tiles are
//     64 consecutive BFS nodes, or (deep trees) sibling subtrees cut from
//     bands of levels plus their root path (ancestor_plan.cuh), whichever
//     stages fewer rows. A persistent grid (one CTA per resident slot) takes
//     equal contiguous ranges of the items, tile-major, or one (tile, head
//     chunk) unit per CTA when that balances better; a tile is planned once
//     for all of its heads.
//   * Plan: the walk keys of a tile's rows form a few windows of consecutive
//     nodes (ancestor_plan.cuh); their K/V rows are staged in shared memory
//     once per head (through a page table when K/V are paged).
//   * A warp owns 16 queries; their keys over all levels form one key list
//     (<= 128 columns). S = Q . K_list^T runs as mma.sync m16n8k16 (fp32
//     accumulate) with S kept in registers; a per-thread bitmask (built once
//     per tile) keeps exactly each row's walk keys, so the softmax (exact, row
//     max over the walk) sees the reference's key set. P is normalised, rounded
//     to fp16 (bf16: hi + lo split) and reused from the S registers as the A
//     operand of O = P . V_list.
//   * The head loop is software-pipelined with two cp.async groups per head
//     (next head's Q/K during this head's P.V and epilogue, its V during its
//     own S and softmax).
//   * Tensor cores here only cut instruction count: the pass is a gather bound
//     by HBM bandwidth (~2.8 flop per byte).
//   * Shared rows use a 16-byte-chunk XOR swizzle (chunk ^ (row & 7)), unrolled
//     into the ldmatrix/stmatrix addresses, so row reads are bank-conflict
//     free; the output tile leaves through stmatrix and 16-byte streaming
//     stores.
// Used for branching >= 2 when a tile's rows and a warp's key list fit (the
// host plans every tile's capacity), for head_dim 64, 128 and 256; chains and
// explicit parents take the scalar walk.
#include <atomic>
#include <cstdlib>
#include <mutex>

#include "ancestor_plan.cuh"

namespace qa {

// First failed plan check of the tensor-core ancestor kernel since the last
// read: [0] check (1 sizes, 2 query row, 3 key slot, 4 staged row), [1] tile,
// [2] sequence, [3] offending value, [4] plan from the table, [5] sequence
// length, [6] tile rows, [7] staged rows. Read and cleared by
// qa_ancestor_diagnostics; [0] also sets bit 4 of qa_check_device_error.
__device__ int g_anc_diag[8];

namespace {

constexpr int kWarps = 4;
constexpr int kTcThreads = kWarps * 32;
constexpr int kTcMQ = kWarps * 16;  // queries per CTA
constexpr int kTcMaxSmem = 200 * 1024;
constexpr int kTcMaxKeys = 128;  // key-list columns per warp (all walk levels of 16 queries)

struct TcParams {
  qa_ancestor_args a;
  float scale_log2;
  TileGeom geom;  // tiling of every sequence's tree
  int32_t head_ratio;
  int32_t rows_cap;
  int32_t kw_cap;  // key-list columns per warp (multiple of 16)
  int32_t num_sms;     // host-side launch planning only
  int32_t unit_heads;  // > 0: CTA x runs unit x = (tile, chunk of unit_heads heads)
  FastDiv div_b;
  // Tile-plan table (plans of a full-length tree, one record per tile; see
  // TilePlanRec): read when plan != nullptr, or written (and nothing else
  // done) by a launch with plan_out = 1 and one CTA per tile.
  uint32_t* plan;
  int32_t plan_stride;  // words per record
  uint32_t plan_key;    // word 0 of a valid record of this launch's table
  int32_t plan_out;
  // Explicit parents: per-call plans, one record per (sequence, tile), written
  // by ancestor_parents_plan_kernel just before this launch (read after the
  // programmatic-launch wait). Warps flagged in a record's word 1 ("walk warps")
  // attend their rows with a per-row walk over global memory instead.
  const uint32_t* par_plan;
};

// One tile's plan in the table (32-bit words): [0] key, [1] plan_tile_word, [2] rows of
// the tile, [3] staged K/V rows, [4 + w] warp w's rows | key columns << 16,
// [8 + r] tree node of tile row r, [72 + 64 w + c / 2] staged slot of warp w's
// key column c (16 bits each), [328 + 2 t + h] thread t's walk-key mask of its
// row g + 8 h, [584 + j] tree node of staged row j.
// Record check words: a table assignment's key is a well-mixed 32-bit value
// and word 1 mixes it with the tile index, so stale words of an earlier table
// in the same slot (node numbers, masks, small counts) do not pass for a record.
__host__ __device__ inline uint32_t plan_mix(uint32_t x) {  // a 32-bit finaliser (MurmurHash3 fmix32)
  x ^= x >> 16;
  x *= 0x85ebca6bu;
  x ^= x >> 13;
  x *= 0xc2b2ae35u;
  x ^= x >> 16;
  return x;
}
__host__ __device__ inline uint32_t plan_tile_word(uint32_t key, int tile) {
  return plan_mix(key ^ (0x9e3779b9u * uint32_t(tile + 1)));
}

struct TilePlanRec {
  static constexpr int kRows = 8, kSlots = 72, kSel = 328, kStaged = 584;
  static int words(int rows_cap) { return (kStaged + rows_cap + 3) & ~3; }
};

QA_DEVINL uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

QA_DEVINL void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
QA_DEVINL void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}

QA_DEVINL void stsm_x4(uint32_t addr, uint32_t r0, uint32_t r1, uint32_t r2, uint32_t r3) {
  asm volatile("stmatrix.sync.aligned.m8n8.x4.shared.b16 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(r0), "r"(r1),
               "r"(r2), "r"(r3)
               : "memory");
}
QA_DEVINL uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}
QA_DEVINL void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> QA_DEVINL void cp_async_wait_group() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
// 16-byte cp.async.cg to a shared-window address
QA_DEVINL void cp_async16_s(uint32_t saddr, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(saddr), "l"(gmem) : "memory");
}

template <typename T> QA_DEVINL void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1);
template <> QA_DEVINL void mma16816<__half>(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <> QA_DEVINL void mma16816<__nv_bfloat16>(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Two fp32 -> packed pair of T (low element first).
template <typename T> QA_DEVINL uint32_t pack2(float lo, float hi);
template <> QA_DEVINL uint32_t pack2<__half>(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
template <> QA_DEVINL uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
// Byte offset of 16-byte chunk c of row r in a swizzled [rows][D] tile.
template <int D> QA_DEVINL uint32_t swz(int r, int c) {
  return uint32_t(r) * (D * 2) + uint32_t((c ^ (r & 7)) * 16);
}

// Dynamic shared memory of one CTA (bytes): Q tile, staged K and V rows, and
// the K and V element offsets of every staged row.
template <int D> struct TcSmem {
  __host__ __device__ static int k_off() { return kTcMQ * D * 2; }
  __host__ __device__ static int v_off(int rows) { return k_off() + rows * D * 2; }
  __host__ __device__ static int tok_off(int rows) { return v_off(rows) + rows * D * 2; }
  // + 128: room to align the tiles to 128 bytes
  __host__ __device__ static int total(int rows) { return tok_off(rows) + rows * 16 + 128; }
};

// Per-row walk of one warp over global memory (explicit-parent tiles whose
// key lists do not fit the staged rows): rows [node_lo, node_lo + n) of
// sequence `seq`, query head h. Lanes split head_dim (D/32 elements each);
// the walk follows parents[] as the scalar kernel does (ends at a self-loop,
// a parent outside the sequence, or max_depth steps); exact online softmax in
// fp32 with the prefix result (if any) merged in as one extra key.
template <typename T, int D>
__device__ __noinline__ void walk_rows(const TcParams& p, int h, int seq, int q0, int len, int kv0, int node_lo,
                                       int n, int lane) {
  constexpr int E = D / 32;  // elements per lane (2, 4 or 8)
  const qa_ancestor_args& a = p.a;
  const int hk = h / p.head_ratio;
  auto load = [&](const void* base, int64_t elem_off, float (&f)[E]) {
    const T* src = reinterpret_cast<const T*>(base) + elem_off + lane * E;
#pragma unroll
    for (int i = 0; i < E / 2; ++i) {
      const float2 v = pair_to_f32<T>(__ldg(reinterpret_cast<const unsigned int*>(src) + i));
      f[2 * i] = v.x;
      f[2 * i + 1] = v.y;
    }
  };
  auto kv_off = [&](int node, int64_t& ko, int64_t& vo) {
    if (a.page_table == nullptr) {
      const int64_t tk = int64_t(kv0) + node;
      ko = tk * a.k_stride_t;
      vo = tk * a.v_stride_t;
    } else {
      const int pos = a.kv_offset + node;
      const int64_t page = __ldg(a.page_table + int64_t(seq) * a.page_table_stride + pos / a.page_size);
      ko = page * a.k_stride_page + int64_t(pos % a.page_size) * a.k_stride_t;
      vo = page * a.v_stride_page + int64_t(pos % a.page_size) * a.v_stride_t;
    }
    ko += int64_t(hk) * a.k_stride_h;
    vo += int64_t(hk) * a.v_stride_h;
  };
  for (int i = 0; i < n; ++i) {
    const int q = node_lo + i;
    const int64_t t = int64_t(q0) + q;
    float qf[E], acc[E];
    load(a.q, q_seq_off(a, seq, q0) + int64_t(q) * a.q_stride_t + int64_t(h) * a.q_stride_h, qf);
    float m = -INFINITY, l = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) acc[e] = 0.f;
    if (a.prefix_o != nullptr) {
      const float pl = __ldg(a.prefix_lse + t * a.prefix_lse_stride_t + int64_t(h) * a.prefix_lse_stride_h);
      if (pl > -INFINITY) {
        load(a.prefix_o, t * a.prefix_o_stride_t + int64_t(h) * a.prefix_o_stride_h, acc);
        m = pl * kLog2e;
        l = 1.f;
      }
    }
    int node = q;
    for (int s = 0;; ++s) {
      int64_t ko, vo;
      kv_off(node, ko, vo);
      float kf[E], vf[E];
      load(a.k, ko, kf);
      load(a.v, vo, vf);
      float d = 0.f;
#pragma unroll
      for (int e = 0; e < E; ++e) d = fmaf(qf[e], kf[e], d);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) d += __shfl_xor_sync(0xffffffffu, d, off);
      const float sc = d * p.scale_log2;
      if (sc > m) {
        const float alpha = fast_exp2(m - sc);
        l *= alpha;
#pragma unroll
        for (int e = 0; e < E; ++e) acc[e] *= alpha;
        m = sc;
      }
      const float w = fast_exp2(sc - m);
      l += w;
#pragma unroll
      for (int e = 0; e < E; ++e) acc[e] = fmaf(w, vf[e], acc[e]);
      if (s >= a.max_depth) break;
      const int nx = __ldg(a.parents + q0 + node);
      if (nx == node || nx < 0 || nx >= len) break;
      node = nx;
    }
    const float inv = 1.f / l;
    T* o = reinterpret_cast<T*>(a.o) + t * a.o_stride_t + int64_t(h) * a.o_stride_h + lane * E;
#pragma unroll
    for (int e = 0; e < E; e += 2)
      *reinterpret_cast<uint32_t*>(o + e) = pack2<T>(acc[e] * inv, acc[e + 1] * inv);
    if (a.lse != nullptr && lane == 0)
      a.lse[t * a.lse_stride_t + int64_t(h) * a.lse_stride_h] = (m + __log2f(l)) * kLn2;
  }
}

// MINB = CTAs per SM the register allocation must allow (1, 3 or 4; chosen
// per launch by launch_tc_minb).
template <typename T, int D, int NBK, int MINB, int MODE>
__global__ void __launch_bounds__(kTcThreads, MINB) ancestor_tc_kernel(const TcParams p) {
  constexpr bool SUB = MODE == 1;  // subtree tiles
  constexpr bool PAR = MODE == 2;  // explicit parents: per-call plans, walk warps
  using SM = TcSmem<D>;
  constexpr int RC = D / 8;   // 16-byte chunks per row
  constexpr int KB = D / 16;  // k16 steps of q.k
  constexpr int NB = D / 8;   // n8 blocks of the output
  extern __shared__ __align__(128) unsigned char smem_raw[];
  // tiles start on a 128-byte boundary: the unrolled swizzle XORs address bits 4-6
  unsigned char* smem_base = smem_raw + ((128u - (smem_u32(smem_raw) & 127u)) & 127u);
  unsigned char* sQ = smem_base;
  unsigned char* sK = smem_base + SM::k_off();
  unsigned char* sV = smem_base + SM::v_off(p.rows_cap);
  int64_t* row_off = reinterpret_cast<int64_t*>(smem_base + SM::tok_off(p.rows_cap));
  __shared__ int seg_lo[kMaxLevels + 1], seg_row[kMaxLevels + 2], n_seg;  // the tile's level segments
  __shared__ int q_node[kTcMQ];                   // tree node of every tile row
  __shared__ int win_lo[kMaxWin + 1];             // staged windows (descending nodes)
  __shared__ int win_base[kMaxWin + 1];
  __shared__ int n_win;
  __shared__ int w_lo[kWarps][kMaxWin + 1];       // per-warp key windows
  __shared__ int w_base[kWarps][kMaxWin + 1];
  __shared__ int w_nwin[kWarps];
  __shared__ int lv_off[kMaxLevels];              // contiguous tiles: CTA level offsets (unused after planning)
  __shared__ int w_col[kWarps][kMaxLevels];       // contiguous tiles: column = w_col[s] + node, per warp
  __shared__ int w_levels[kWarps];
  __shared__ int kslot[kWarps][kTcMaxKeys];       // staged K/V row of each key column
  __shared__ bool table_hit;                      // this tile's plan is in the table

  if (threadIdx.x == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");  // a following GEMM may stage
  const qa_ancestor_args& a = p.a;
  // Work of this CTA: either an equal contiguous range of the (tile, head)
  // items, tile-major (a persistent grid; the range touches one or two
  // tiles), or one unit = one tile and a chunk of its heads. A tile is
  // planned once for all of its heads in the range.
  const int64_t items = int64_t(a.batch) * p.geom.tiles * a.num_q_heads;
  int64_t it, it_end;
  if (p.unit_heads > 0) {  // one tile, one chunk of heads: every CTA plans exactly one tile
    const int chunks = (a.num_q_heads + p.unit_heads - 1) / p.unit_heads;
    const int64_t tg = blockIdx.x / chunks;
    it = tg * a.num_q_heads + int64_t(blockIdx.x % chunks) * p.unit_heads;
    it_end = min(it + p.unit_heads, (tg + 1) * a.num_q_heads);
  } else {
    it = items * blockIdx.x / gridDim.x;
    it_end = items * (blockIdx.x + 1) / gridDim.x;
  }
  bool waited = false;  // griddepcontrol.wait done (before the first global read)
  if (p.plan_out) {  // planning launch: CTA x plans tile x of a full-length tree
    it = int64_t(blockIdx.x) * a.num_q_heads;
    it_end = it + 1;
  }
  bool from_table = false;  // this tile's plan came from the table
  const uint32_t* rec = nullptr;
  while (it < it_end) {
  const int64_t tg = it / a.num_q_heads;
  const int h_first = int(it - tg * a.num_q_heads);
  const int h_end = int(min(int64_t(a.num_q_heads), h_first + (it_end - it)));
  it += h_end - h_first;
  const int tile = int(tg % p.geom.tiles);
  const int seq = int(tg / p.geom.tiles);
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int wrow = warp * 16;  // first tile row of this warp
  const int g = lane >> 2, t = lane & 3;
  // The plan depends on the tree shape only, not on the inputs: the first tile
  // is planned for a full-length sequence before waiting for the previous
  // kernel on the stream (programmatic dependent launch), so the planning
  // overlaps that kernel's tail; it is redone if the sequence is shorter.
  int q0 = 0, len = 0, kv0 = 0;
  if (waited) {
    q0 = __ldg(a.cu_seqlens_q + seq);
    len = __ldg(a.cu_seqlens_q + seq + 1) - q0;
    kv0 = (a.cu_seqlens_kv ? __ldg(a.cu_seqlens_kv + seq) : q0) + a.kv_offset;
  }
  int len_plan = waited ? len : a.max_seqlen;
  int q_lo = 0, nq = 0, wn = 0, nw = 0, nrows = 0, nkeys = 0, kpad = 0;
  int walk_n = 0;  // explicit parents: rows of this warp attended by walk_rows
  uint32_t sel0 = 0u, sel1 = 0u;  // walk-key masks, the same for every head
  // token (relative to the sequence) of tile row r
  auto row_tok = [&](int r) -> int {
    if constexpr (SUB) return q_node[r];
    else return q_lo + r;
  };
  // token of this thread's row g (half 0) or g + 8 (half 1), clamped to the
  // warp's rows (the result is unused past them)
  auto tok_g = [&](int half) -> int { return row_tok(wrow + min(g + 8 * half, max(wn - 1, 0))); };
  for (;;) {
  __syncthreads();  // the previous plan is no longer read
  q_lo = 0;
  wn = 0;
  sel0 = sel1 = 0u;
  nkeys = kpad = 0;
  from_table = false;
  if constexpr (PAR) {
    // explicit parents: the plan kernel wrote this (sequence, tile)'s record
    // just before this launch, so read it after the programmatic-launch wait
    if (!waited) {
      asm volatile("griddepcontrol.wait;" ::: "memory");
      waited = true;
      q0 = __ldg(a.cu_seqlens_q + seq);
      len = __ldg(a.cu_seqlens_q + seq + 1) - q0;
      kv0 = (a.cu_seqlens_kv ? __ldg(a.cu_seqlens_kv + seq) : q0) + a.kv_offset;
    }
    rec = p.par_plan + (int64_t(seq) * p.geom.tiles + tile) * p.plan_stride;
    nq = min(int(__ldcg(rec + 2)), kTcMQ);
    nrows = min(int(__ldcg(rec + 3)), p.rows_cap);
    const uint32_t wk = __ldcg(rec + 4 + warp);
    wn = min(int(wk & 0xffffu), 16);
    nkeys = min(int(wk >> 16), p.kw_cap);
    if ((__ldcg(rec + 1) >> warp) & 1u) {  // a walk warp: no key list, rows go to walk_rows
      walk_n = wn;
      wn = nkeys = 0;
    }
    kpad = (nkeys + 15) & ~15;
    const uint32_t* sl = rec + TilePlanRec::kSlots + warp * (kTcMaxKeys / 2);
    for (int c = lane; c < kTcMaxKeys; c += 32) {
      const uint32_t w2 = __ldcg(sl + c / 2);
      kslot[warp][c] = min(int((c & 1) ? (w2 >> 16) : (w2 & 0xffffu)), p.rows_cap - 1);
    }
    sel0 = __ldcg(rec + TilePlanRec::kSel + 2 * tid);
    sel1 = __ldcg(rec + TilePlanRec::kSel + 2 * tid + 1);
    q_lo = tile * kTcMQ;
    from_table = true;
    __syncthreads();  // the key slots are visible
    break;
  }
  if (p.plan != nullptr && !p.plan_out && len_plan == a.max_seqlen) {
    // a full-length tree: its tile plans are in the table when the record's
    // key matches this launch's. One thread reads the key (the record may be
    // written while this CTA runs) and the barrier hands its answer, and the
    // visibility of the record it guards, to every thread.
    rec = p.plan + int64_t(tile) * p.plan_stride;
    if (tid == 0) {
      uint32_t k0;
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(k0) : "l"(rec) : "memory");
      table_hit = k0 == p.plan_key && __ldcg(rec + 1) == plan_tile_word(p.plan_key, tile);
    }
    __syncthreads();
    if (table_hit) {
      from_table = true;
      nq = min(int(__ldcg(rec + 2)), kTcMQ);
      nrows = min(int(__ldcg(rec + 3)), p.rows_cap);
      const uint32_t wk = __ldcg(rec + 4 + warp);
      wn = min(int(wk & 0xffffu), 16);
      nkeys = min(int(wk >> 16), p.kw_cap);
      kpad = (nkeys + 15) & ~15;
      if (SUB && tid < kTcMQ) q_node[tid] = int(__ldcg(rec + TilePlanRec::kRows + tid));
      const uint32_t* sl = rec + TilePlanRec::kSlots + warp * (kTcMaxKeys / 2);
      for (int c = lane; c < kTcMaxKeys; c += 32) {
        const uint32_t w2 = __ldcg(sl + c / 2);
        kslot[warp][c] = min(int((c & 1) ? (w2 >> 16) : (w2 & 0xffffu)), p.rows_cap - 1);
      }
      sel0 = __ldcg(rec + TilePlanRec::kSel + 2 * tid);
      sel1 = __ldcg(rec + TilePlanRec::kSel + 2 * tid + 1);
      q_lo = SUB ? 0 : tile * kTcMQ;
      __syncthreads();  // q_node and the key slots are visible
    }
  }
  if (from_table) {
    // planned: nothing to compute
  } else if constexpr (SUB) {
    // ---- plans, shared by every head: the tile's staged windows (thread 1)
    // and each warp's key windows (lane 0 of each warp), computed in parallel ----
    if (tid == 0) n_seg = tile_segments(p.geom, tile, len_plan, seg_lo, seg_row);
    __syncthreads();
    nq = seg_row[n_seg];
    if (nq > 0) {
      wn = max(0, min(16, nq - wrow));
      if (tid < nq) {
        int i = 0;
        while (seg_row[i + 1] <= tid) ++i;
        q_node[tid] = seg_lo[i] + tid - seg_row[i];
      }
      if ((lane == 0 && wn > 0) || tid == 1) {
        const bool cta = tid == 1;
        int nwin = 0;
        plan_rows(p.geom, seg_lo, seg_row, n_seg, cta ? 0 : wrow, cta ? nq : wrow + wn, a.max_depth,
                  DevDivB{p.div_b}, cta ? win_lo : w_lo[warp], cta ? win_base : w_base[warp], nwin);
        if (cta) n_win = nwin;
        else w_nwin[warp] = nwin;
      }
      __syncthreads();
    }
  } else {
    // ---- contiguous tile: its walk levels are contiguous node ranges
    // (plan_levels_fit), for the CTA and for each warp's 16 rows ----
    q_lo = tile * kTcMQ;
    nq = max(0, min(kTcMQ, len_plan - q_lo));
    if (nq > 0) {
      wn = max(0, min(16, nq - wrow));
      if (tid == 0) {
        int ns = 0, nwc = 0;
        plan_levels_fit(q_lo, nq, a.max_depth, p.div_b, lv_off, win_lo, win_base, ns, nwc);
        n_win = nwc;
      }
      if (lane == 0 && wn > 0 && warp > 0) {
        int L = 0, nwin = 0;
        plan_levels_fit(q_lo + wrow, wn, a.max_depth, p.div_b, w_col[warp], w_lo[warp], w_base[warp], L, nwin);
        w_levels[warp] = L;
        w_nwin[warp] = nwin;
      }
      if (tid == 32) {  // warp 0's plan, beside thread 0's
        int L = 0, nwin = 0;
        plan_levels_fit(q_lo, min(16, nq), a.max_depth, p.div_b, w_col[0], w_lo[0], w_base[0], L, nwin);
        w_levels[0] = L;
        w_nwin[0] = nwin;
      }
      __syncthreads();
    }
  }
  if (nq > 0 && !from_table) {
    nw = n_win;
    nrows = win_base[nw];
    // key column -> staged slot (columns past the list repeat its last row)
    nkeys = wn > 0 ? w_base[warp][w_nwin[warp]] : 0;
    kpad = (nkeys + 15) & ~15;
    if (wn > 0) {
      const int nwin = w_nwin[warp];
      for (int c = lane; c < kpad; c += 32) {
        const int cc = min(c, nkeys - 1);
        int wi = 0;
        while (wi + 1 < nwin && w_base[warp][wi + 1] <= cc) ++wi;
        const int node = w_lo[warp][wi] + (cc - w_base[warp][wi]);
        int cw = 0;  // the CTA window that stages this node
        while (cw + 1 < nw && node < win_lo[cw]) ++cw;  // windows descend in node order
        kslot[warp][c] = win_base[cw] + node - win_lo[cw];
      }
    }
    // ---- which fragment elements are this thread's rows' walk keys ----
    // The thread owning column c of a row holds it in block c/8, element c%2
    // when (c%8)/2 == t.
    if constexpr (SUB) {
      // row r's step-s key is the column of node_s(r) in the warp's windows (the
      // walk descends, so the window index only grows)
      if (wn > 0) {
        const int* wl = w_lo[warp];
        const int* wb = w_base[warp];
        const int nwin = w_nwin[warp];
#pragma unroll 1
        for (int half = 0; half < 2; ++half) {
          if (g + 8 * half >= wn) continue;
          int n = tok_g(half), wi = 0;
          uint32_t sel = 0u;
          for (int s = 0; s <= a.max_depth; ++s) {
            if (s > 0) {
              if (n == 0) break;  // the walk ended at the root
              n = int(fast_div(uint32_t(n - 1), p.div_b));
            }
            while (wi + 1 < nwin && n < wl[wi]) ++wi;
            const int c = wb[wi] + n - wl[wi];
            if (((c >> 1) & 3) == t) sel |= 1u << (((c >> 3) << 1) | (c & 1));
          }
          if (half) sel1 = sel; else sel0 = sel;
        }
      }
    } else {
      // row r's step-s key is column w_col[s] + node_s(r)
      if (wn > 0) {
        const int L = w_levels[warp];
        const int* wc = w_col[warp];
        int n0 = g < wn ? tok_g(0) : -1, n1 = g + 8 < wn ? tok_g(1) : -1;
        for (int s = 0; s < L; ++s) {
          if (s > 0) {
            n0 = n0 <= 0 ? -1 : int(fast_div(uint32_t(n0 - 1), p.div_b));
            n1 = n1 <= 0 ? -1 : int(fast_div(uint32_t(n1 - 1), p.div_b));
          }
          const int off = wc[s];
          const int c0 = off + n0, c1 = off + n1;
          if (n0 >= 0 && ((c0 >> 1) & 3) == t) sel0 |= 1u << (((c0 >> 3) << 1) | (c0 & 1));
          if (n1 >= 0 && ((c1 >> 1) & 3) == t) sel1 |= 1u << (((c1 >> 3) << 1) | (c1 & 1));
        }
      }
    }
  }
  if (p.plan_out) {  // write this tile's record (no input is read) and stop
    uint32_t* out = p.plan + int64_t(tile) * p.plan_stride;
    if (tid < kTcMQ) out[TilePlanRec::kRows + tid] = uint32_t(tid < nq ? row_tok(tid) : 0);
    if (tid == 0) {
      out[2] = uint32_t(nq);
      out[3] = uint32_t(nrows);
    }
    if (lane == 0) out[4 + warp] = uint32_t(wn) | (uint32_t(nkeys) << 16);
    for (int c = 2 * lane; c < kTcMaxKeys; c += 64) {
      const uint32_t lo = c < kpad ? uint32_t(kslot[warp][c]) : 0u;
      const uint32_t hi = c + 1 < kpad ? uint32_t(kslot[warp][c + 1]) : 0u;
      out[TilePlanRec::kSlots + warp * (kTcMaxKeys / 2) + c / 2] = lo | (hi << 16);
    }
    out[TilePlanRec::kSel + 2 * tid] = sel0;
    out[TilePlanRec::kSel + 2 * tid + 1] = sel1;
    for (int j = tid; j < nrows; j += kTcThreads) {
      int w = 0;
      while (w + 1 < nw && win_base[w + 1] <= j) ++w;
      out[TilePlanRec::kStaged + j] = uint32_t(win_lo[w] + (j - win_base[w]));
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
      out[1] = plan_tile_word(p.plan_key, tile);
      asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(out), "r"(p.plan_key) : "memory");
    }
    return;
  }
  if (waited) break;
  asm volatile("griddepcontrol.wait;" ::: "memory");  // inputs of the previous kernel are visible
  waited = true;
  q0 = __ldg(a.cu_seqlens_q + seq);
  len = __ldg(a.cu_seqlens_q + seq + 1) - q0;
  kv0 = (a.cu_seqlens_kv ? __ldg(a.cu_seqlens_kv + seq) : q0) + a.kv_offset;
  if (len == len_plan) break;
  len_plan = len;  // a shorter sequence: plan again
  }  // plan passes
  if (nq == 0) continue;  // uniform over the CTA
  {
    // Plan check: every row and key the tile will address lies inside its
    // sequence and its staged rows. A plan that fails (which the planner
    // should never produce) is recorded in the device diagnostics and the tile
    // is skipped instead of reading or writing out of bounds.
    int bad = 0, val = 0;
    if (nq > kTcMQ || nrows > p.rows_cap || kpad > p.kw_cap || wn > 16) bad = 1, val = nq;
    if (!bad && tid < nq) {
      const int r = row_tok(tid);
      if (r < 0 || r >= len) bad = 2, val = r;
    }
    if (!bad && wn > 0)
      for (int c = lane; c < kpad; c += 32)
        if (kslot[warp][c] < 0 || kslot[warp][c] >= nrows) bad = 3, val = kslot[warp][c];
    for (int j = tid; !bad && j < nrows; j += kTcThreads) {
      int node;
      if (from_table) {
        node = int(__ldcg(rec + TilePlanRec::kStaged + j));
      } else {
        int w = 0;
        while (w + 1 < nw && win_base[w + 1] <= j) ++w;
        node = win_lo[w] + (j - win_base[w]);
      }
      if (node < 0 || node >= len) bad = 4, val = node;
    }
    if (__syncthreads_or(bad != 0)) {
      if (bad && atomicCAS(&g_anc_diag[0], 0, bad) == 0) {
        g_anc_diag[1] = tile;
        g_anc_diag[2] = seq;
        g_anc_diag[3] = val;
        g_anc_diag[4] = from_table ? 1 : 0;
        g_anc_diag[5] = len;
        g_anc_diag[6] = nq;
        g_anc_diag[7] = nrows;
      }
      continue;
    }
  }
  for (int j = tid; j < nrows; j += kTcThreads) {  // byte offset of every staged row
    int node;
    if (from_table) {
      node = min(int(__ldcg(rec + TilePlanRec::kStaged + j)), len - 1);
    } else {
      int w = 0;
      while (w + 1 < nw && win_base[w + 1] <= j) ++w;
      node = win_lo[w] + (j - win_base[w]);
    }
    if (a.page_table == nullptr) {
      const int64_t tk = int64_t(kv0) + node;
      row_off[2 * j] = tk * a.k_stride_t * int64_t(sizeof(T));
      row_off[2 * j + 1] = tk * a.v_stride_t * int64_t(sizeof(T));
    } else {  // paged K/V: the row is a slot of the page the sequence's table names
      const int pos = a.kv_offset + node;
      const int64_t page = __ldg(a.page_table + int64_t(seq) * a.page_table_stride + pos / a.page_size);
      const int slot = pos % a.page_size;
      row_off[2 * j] = (page * a.k_stride_page + int64_t(slot) * a.k_stride_t) * int64_t(sizeof(T));
      row_off[2 * j + 1] = (page * a.v_stride_page + int64_t(slot) * a.v_stride_t) * int64_t(sizeof(T));
    }
  }
  const int* ks = kslot[warp];
  __syncthreads();  // row offsets and key slots are visible to every thread
  // Staging: thread tid copies 16-byte chunk my_cc of rows my_r0, my_r0 + RPP,
  // ...; the swizzle term of those rows is my_x, flipped by kXStep per pass
  // (RPP is a multiple of 8, or 4 for head_dim 256).
  constexpr int RPP = kTcThreads / RC;
  constexpr uint32_t kXStep = uint32_t((RPP & 7) << 4);
  constexpr uint32_t kRowStep = uint32_t(RPP * D * 2);
  const int my_cc = tid % RC, my_r0 = tid / RC;
  const uint32_t my_x = uint32_t((my_cc ^ (my_r0 & 7)) << 4);
  const uint32_t sQa = smem_u32(sQ), sKa = smem_u32(sK), sVa = smem_u32(sV);
  // Software pipeline over the heads (two cp.async groups per head): head h+1's
  // Q and K rows load during head h's P.V and epilogue, and its V rows during
  // its own S and softmax. K and V are re-staged only when the KV head changes;
  // the epilogue stages the output tile in the V rows only when they are about
  // to be replaced (otherwise it stores straight from the fragments).
  int k_staged = -1, v_staged = -1;
  auto issue_qk = [&](int hh) {
    if constexpr (SUB) {
      const char* Qh = reinterpret_cast<const char*>(a.q) +
                       int64_t(sizeof(T)) * (int64_t(hh) * a.q_stride_h + q_seq_off(a, seq, q0) + my_cc * 8);
      const int64_t tstep = a.q_stride_t * int64_t(sizeof(T));
      uint32_t d = sQa + uint32_t(my_r0 * D * 2), x = my_x;
#pragma unroll
      for (int i = 0; i < kTcMQ / RPP; ++i, d += kRowStep, x ^= kXStep) {
        const int r = my_r0 + i * RPP;
        if (r < nq) cp_async16_s(d + x, Qh + row_tok(r) * tstep);
      }
    } else {
      const char* src = reinterpret_cast<const char*>(a.q) +
                        int64_t(sizeof(T)) * (int64_t(hh) * a.q_stride_h + q_seq_off(a, seq, q0) +
                                              int64_t(q_lo + my_r0) * a.q_stride_t + my_cc * 8);
      const int64_t step = int64_t(RPP) * a.q_stride_t * int64_t(sizeof(T));
      uint32_t d = sQa + uint32_t(my_r0 * D * 2), x = my_x;
      for (int r = my_r0; r < nq; r += RPP, src += step, d += kRowStep, x ^= kXStep) cp_async16_s(d + x, src);
    }
    const int hk = hh / p.head_ratio;
    if (hk != k_staged) {
      const char* Kh = reinterpret_cast<const char*>(a.k) + int64_t(sizeof(T)) * (int64_t(hk) * a.k_stride_h + my_cc * 8);
      uint32_t dk = uint32_t(my_r0 * D * 2), xk = my_x;
      for (int j = my_r0; j < nrows; j += RPP, dk += kRowStep, xk ^= kXStep)
        cp_async16_s(sKa + dk + xk, Kh + row_off[2 * j]);
      k_staged = hk;
    }
    cp_async_commit();
  };
  auto issue_v = [&](int hh) {
    const int hk = hh / p.head_ratio;
    if (hk != v_staged) {
      const char* Vh = reinterpret_cast<const char*>(a.v) + int64_t(sizeof(T)) * (int64_t(hk) * a.v_stride_h + my_cc * 8);
      uint32_t dv = uint32_t(my_r0 * D * 2), xv = my_x;
      for (int j = my_r0; j < nrows; j += RPP, dv += kRowStep, xv ^= kXStep)
        cp_async16_s(sVa + dv + xv, Vh + row_off[2 * j + 1]);
      v_staged = hk;
    }
    cp_async_commit();
  };
  issue_qk(h_first);
  issue_v(h_first);
  for (int h = h_first; h < h_end; ++h) {
  cp_async_wait_group<1>();  // Q and K of head h (its V may still be in flight)
  __syncthreads();
  // ---- S = Q . K_list^T over every level's keys at once (registers) ----
  // A-operand (and stmatrix) lane address of 16x16 block kk of this warp's
  // rows: row wrow + (lane & 15), chunk 2kk + (lane >> 4), i.e.
  // q_off ^ ((kk & 3) << 5) plus 128 bytes per 4 blocks (swizzle unrolled).
  const uint32_t q_off = sQa + uint32_t((wrow + (lane & 15)) * D * 2) + uint32_t((((lane >> 4) ^ (lane & 7))) << 4);
  uint32_t qf[KB][4];
#pragma unroll
  for (int kk = 0; kk < KB; ++kk)
    ldsm_x4((q_off ^ uint32_t((kk & 3) << 5)) + uint32_t((kk >> 2) * 128), qf[kk][0], qf[kk][1], qf[kk][2],
            qf[kk][3]);
  float sc[NBK][4];
  // B-operand lane address of key block nb: row kslot, chunk 4k2 + (lane >> 3)
  // = k_off[nb] ^ ((k2 & 1) << 6) plus 128 bytes per 2 steps
  uint32_t k_off[NBK];
#pragma unroll
  for (int nb = 0; nb < NBK; ++nb) {
    sc[nb][0] = sc[nb][1] = sc[nb][2] = sc[nb][3] = 0.f;
    const int row = 8 * nb < kpad ? ks[8 * nb + (lane & 7)] : 0;
    k_off[nb] = uint32_t(row * D * 2) + uint32_t(((lane >> 3) ^ (row & 7)) << 4);
  }
#pragma unroll
  for (int k2 = 0; k2 < KB / 2; ++k2) {  // k outer: NBK independent accumulation chains
#pragma unroll
    for (int nb = 0; nb < NBK; ++nb) {
      if (8 * nb < kpad) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4(sKa + (k_off[nb] ^ uint32_t((k2 & 1) << 6)) + uint32_t((k2 >> 1) * 128), b0, b1, b2, b3);
        mma16816<T>(sc[nb], qf[2 * k2], b0, b1);
        mma16816<T>(sc[nb], qf[2 * k2 + 1], b2, b3);
      }
    }
  }
  // ---- exact softmax per row over its walk (a quad of threads shares a row) ----
  float mx0 = -INFINITY, mx1 = -INFINITY, pl0 = -INFINITY, pl1 = -INFINITY;
  if (a.prefix_o != nullptr) {
    const int64_t t0 = int64_t(q0) + tok_g(0);
    if (g < wn) pl0 = __ldg(a.prefix_lse + t0 * a.prefix_lse_stride_t + int64_t(h) * a.prefix_lse_stride_h) * kLog2e;
    if (g + 8 < wn) pl1 = __ldg(a.prefix_lse + (int64_t(q0) + tok_g(1)) * a.prefix_lse_stride_t + int64_t(h) * a.prefix_lse_stride_h) * kLog2e;
    mx0 = pl0;
    mx1 = pl1;
  }
#pragma unroll
  for (int nb = 0; nb < NBK; ++nb)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      sc[nb][e] *= p.scale_log2;
      sc[nb][2 + e] *= p.scale_log2;
      if ((sel0 >> (2 * nb + e)) & 1u) mx0 = fmaxf(mx0, sc[nb][e]);
      if ((sel1 >> (2 * nb + e)) & 1u) mx1 = fmaxf(mx1, sc[nb][2 + e]);
    }
  mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
  mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
  mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
  mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
  float l0 = 0.f, l1 = 0.f;
#pragma unroll
  for (int nb = 0; nb < NBK; ++nb)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      sc[nb][e] = ((sel0 >> (2 * nb + e)) & 1u) ? fast_exp2(sc[nb][e] - mx0) : 0.f;
      sc[nb][2 + e] = ((sel1 >> (2 * nb + e)) & 1u) ? fast_exp2(sc[nb][2 + e] - mx1) : 0.f;
      l0 += sc[nb][e];
      l1 += sc[nb][2 + e];
    }
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float wp0 = pl0 > -INFINITY ? fast_exp2(pl0 - mx0) : 0.f;  // prefix weights
  const float wp1 = pl1 > -INFINITY ? fast_exp2(pl1 - mx1) : 0.f;
  l0 += wp0;
  l1 += wp1;
  if (a.lse != nullptr && t == 0) {
    float* Lh = a.lse + int64_t(h) * a.lse_stride_h;
    if (g < wn) Lh[(int64_t(q0) + tok_g(0)) * a.lse_stride_t] = (mx0 + __log2f(l0)) * kLn2;
    if (g + 8 < wn) Lh[(int64_t(q0) + tok_g(1)) * a.lse_stride_t] = (mx1 + __log2f(l1)) * kLn2;
  }
  const float inv0 = g < wn ? 1.f / l0 : 0.f;
  const float inv1 = g + 8 < wn ? 1.f / l1 : 0.f;
  __syncthreads();  // every warp holds its Q fragments and is done with the K rows
  const bool next = h + 1 < h_end;
  if (next) issue_qk(h + 1); else cp_async_commit();
  cp_async_wait_group<1>();  // V of head h
  __syncthreads();

  // ---- O = prefix weight * prefix_o + P . V_list (P from the S registers) ----
  float o[NB][4];
#pragma unroll
  for (int j = 0; j < NB; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  if (a.prefix_o != nullptr) {
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int r = g + 8 * half;
      const float wgt = half ? wp1 : wp0;
      if (r >= wn || wgt == 0.f) continue;
      const float wgt_n = wgt * (half ? inv1 : inv0);
      const int64_t tq = int64_t(q0) + tok_g(half);
      const T* po = reinterpret_cast<const T*>(a.prefix_o) + tq * a.prefix_o_stride_t + int64_t(h) * a.prefix_o_stride_h;
#pragma unroll
      for (int j = 0; j < NB; ++j) {
        const float2 f = pair_to_f32<T>(__ldg(reinterpret_cast<const unsigned int*>(po + 8 * j + 2 * t)));
        o[j][2 * half] = wgt_n * f.x;
        o[j][2 * half + 1] = wgt_n * f.y;
      }
    }
  }
#pragma unroll
  for (int kp = 0; kp < NBK / 2; ++kp) {
    if (16 * kp >= kpad) break;
    // P normalised before rounding to T: O needs no rescale afterwards
    const float p00 = sc[2 * kp][0] * inv0, p01 = sc[2 * kp][1] * inv0;
    const float p02 = sc[2 * kp][2] * inv1, p03 = sc[2 * kp][3] * inv1;
    const float p10 = sc[2 * kp + 1][0] * inv0, p11 = sc[2 * kp + 1][1] * inv0;
    const float p12 = sc[2 * kp + 1][2] * inv1, p13 = sc[2 * kp + 1][3] * inv1;
    uint32_t pa[4];
    pa[0] = pack2<T>(p00, p01);
    pa[1] = pack2<T>(p02, p03);
    pa[2] = pack2<T>(p10, p11);
    pa[3] = pack2<T>(p12, p13);
    uint32_t pb[4] = {0u, 0u, 0u, 0u};
    if constexpr (std::is_same<T, __nv_bfloat16>::value) {
      // bf16 keeps 8 mantissa bits: the rounding remainder goes in a second product
      auto rem = [](float x) { return x - __bfloat162float(__float2bfloat16_rn(x)); };
      pb[0] = pack2<T>(rem(p00), rem(p01));
      pb[1] = pack2<T>(rem(p02), rem(p03));
      pb[2] = pack2<T>(rem(p10), rem(p11));
      pb[3] = pack2<T>(rem(p12), rem(p13));
    }
    // transposed B-operand lane address: row slot, chunk 2jp + (lane >> 4)
    const int slot = ks[16 * kp + (lane & 7) + 8 * ((lane >> 3) & 1)];
    const uint32_t v_off = sVa + uint32_t(slot * D * 2) + uint32_t(((lane >> 4) ^ (slot & 7)) << 4);
#pragma unroll
    for (int jp = 0; jp < D / 16; ++jp) {
      uint32_t b0, b1, b2, b3;
      ldsm_x4_t((v_off ^ uint32_t((jp & 3) << 5)) + uint32_t((jp >> 2) * 128), b0, b1, b2, b3);
      mma16816<T>(o[2 * jp], pa, b0, b1);
      mma16816<T>(o[2 * jp + 1], pa, b2, b3);
      if constexpr (std::is_same<T, __nv_bfloat16>::value) {
        mma16816<T>(o[2 * jp], pb, b0, b1);
        mma16816<T>(o[2 * jp + 1], pb, b2, b3);
      }
    }
  }

  // ---- epilogue ----
  const bool v_replaced = !next || (h + 1) / p.head_ratio != v_staged;
  if (v_replaced) {
  // stage the tile in the V rows wrow.. (stmatrix), then 16-byte row stores
  __syncthreads();  // every warp is done with the V rows
  const uint32_t e_off = q_off - sQa + sVa;
#pragma unroll
  for (int jj = 0; jj < D / 16; ++jj)
    stsm_x4((e_off ^ uint32_t((jj & 3) << 5)) + uint32_t((jj >> 2) * 128), pack2<T>(o[2 * jj][0], o[2 * jj][1]),
            pack2<T>(o[2 * jj][2], o[2 * jj][3]), pack2<T>(o[2 * jj + 1][0], o[2 * jj + 1][1]),
            pack2<T>(o[2 * jj + 1][2], o[2 * jj + 1][3]));
  __syncwarp();
  {
    constexpr int RPI = 32 / RC;  // rows per store instruction (power of two)
    const int c = lane % RC, r0 = lane / RC;
    const uint32_t s0 = sVa + uint32_t((wrow + r0) * D * 2) + uint32_t((c ^ r0) << 4);
    if constexpr (SUB) {
      const char* Oh = reinterpret_cast<const char*>(a.o) +
                       int64_t(sizeof(T)) * (int64_t(h) * a.o_stride_h + int64_t(q0) * a.o_stride_t + c * 8);
      const int64_t tstep = a.o_stride_t * int64_t(sizeof(T));
#pragma unroll
      for (int it = 0; it < 16 / RPI; ++it) {
        // row r0 + it*RPI: (r & 7) = r0 ^ ((it*RPI) & 7) since r0 < RPI
        if (r0 + it * RPI < wn)
          st_stream(const_cast<char*>(Oh + row_tok(wrow + r0 + it * RPI) * tstep),
                    lds128((s0 ^ uint32_t(((it * RPI) & 7) << 4)) + uint32_t(it * RPI * D * 2)));
      }
    } else {
      const char* dst = reinterpret_cast<const char*>(a.o) +
                        int64_t(sizeof(T)) * (int64_t(h) * a.o_stride_h + (int64_t(q0) + q_lo + wrow + r0) * a.o_stride_t + c * 8);
      const int64_t dstep = int64_t(RPI) * a.o_stride_t * int64_t(sizeof(T));
#pragma unroll
      for (int it = 0; it < 16 / RPI; ++it) {
        if (r0 + it * RPI < wn)
          st_stream(const_cast<char*>(dst), lds128((s0 ^ uint32_t(((it * RPI) & 7) << 4)) + uint32_t(it * RPI * D * 2)));
        dst += dstep;
      }
    }
  }
  __syncthreads();  // the staged tiles are read before the next V rows land
  } else {
    // V rows stay for the next head of the group: store pairs from the fragments
    T* Oh = reinterpret_cast<T*>(a.o) + int64_t(h) * a.o_stride_h + int64_t(q0) * a.o_stride_t + 2 * t;
    T* orow0 = Oh + tok_g(0) * a.o_stride_t;
    T* orow1 = Oh + tok_g(1) * a.o_stride_t;
#pragma unroll
    for (int j = 0; j < NB; ++j) {
      if (g < wn) *reinterpret_cast<uint32_t*>(orow0 + 8 * j) = pack2<T>(o[j][0], o[j][1]);
      if (g + 8 < wn) *reinterpret_cast<uint32_t*>(orow1 + 8 * j) = pack2<T>(o[j][2], o[j][3]);
    }
  }
  if constexpr (PAR) {
    if (walk_n > 0) walk_rows<T, D>(p, h, seq, q0, len, kv0, q_lo + wrow, walk_n, lane);
  }
  if (next) issue_v(h + 1); else cp_async_commit();
  }  // heads
  }  // tiles
}

// ---------------------------------------------------------------------------
// Explicit-parent plans (one CTA of 128 threads per (sequence, tile of 64
// consecutive BFS nodes)). Each row's walk follows parents[] exactly as the
// per-query kernel does; the walk nodes of each warp's 16 rows form its key
// list and the union over the warps is the tile's staged row set, both in
// ascending node order via bitmaps over the sequence's nodes (kParWords words).
// A warp whose key list exceeds the key columns, or whose keys would push the
// union past the staged rows, becomes a walk warp (walk_rows). Writes one
// TilePlanRec per (sequence, tile); word 1 holds the walk-warp mask.
// ---------------------------------------------------------------------------
constexpr int kParMaxSeq = 16384;          // nodes per sequence the plans cover
constexpr int kParWords = kParMaxSeq / 32;  // bitmap words
constexpr int kParRowsCap = 96;            // staged rows of a parents tile
constexpr int kParKeys = 64;               // key columns per warp (deep walks)

struct ParPlanSmem {
  uint32_t cta_bm[kParWords];
  uint32_t warp_bm[kWarps][kParWords];
  int cta_pref[kParWords];
  int warp_pref[kWarps][kParWords];
  int walk[kTcMQ][kMaxLevels];
  int walk_len[kTcMQ];
  int kcol[kWarps][kTcMaxKeys];
  int red[kWarps];
};

__global__ void __launch_bounds__(kTcThreads) ancestor_parents_plan_kernel(const qa_ancestor_args a, int tiles,
                                                                            int stride, int rows_cap, int kw_cap,
                                                                            uint32_t* __restrict__ plans) {
  extern __shared__ __align__(16) unsigned char par_smem[];
  ParPlanSmem& S = *reinterpret_cast<ParPlanSmem*>(par_smem);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int seq = blockIdx.x / tiles, tile = blockIdx.x % tiles;
  asm volatile("griddepcontrol.wait;" ::: "memory");  // parents / cu_seqlens may come from the previous kernel
  if (tid == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  uint32_t* out = plans + (int64_t(seq) * tiles + tile) * stride;
  const int q0 = __ldg(a.cu_seqlens_q + seq);
  const int len = min(__ldg(a.cu_seqlens_q + seq + 1) - q0, kParMaxSeq);
  const int q_lo = tile * kTcMQ;
  const int nq = max(0, min(kTcMQ, len - q_lo));
  if (nq == 0) {
    if (tid == 0) out[1] = out[2] = out[3] = 0u;
    if (tid < kWarps) out[4 + tid] = 0u;
    return;
  }
  const int words = (len + 31) / 32;
  // the sequence's parents, staged once (the walks then chase them in shared memory)
  int* par_s = reinterpret_cast<int*>(par_smem + sizeof(ParPlanSmem));
  for (int i = tid; i < len; i += kTcThreads) par_s[i] = __ldg(a.parents + q0 + i);
  for (int i = tid; i < words; i += kTcThreads) {
    S.cta_bm[i] = 0u;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) S.warp_bm[w][i] = 0u;
  }
  __syncthreads();
  const int levels = min(a.max_depth + 1, kMaxLevels);
  if (tid < nq) {  // row tid's walk
    int n = q_lo + tid, s = 0;
    for (;;) {
      S.walk[tid][s] = n;
      atomicOr(&S.warp_bm[tid >> 4][n >> 5], 1u << (n & 31));
      if (s + 1 >= levels) break;
      const int nx = par_s[n];
      if (nx == n || nx < 0 || nx >= len) break;
      n = nx;
      ++s;
    }
    S.walk_len[tid] = s + 1;
  }
  __syncthreads();
  // key-list sizes per warp, then the union, warp by warp while it fits
  uint32_t walk_mask = 0u;
  int nkeys[kWarps];
  int nrows = 0;
  for (int w = 0; w < kWarps; ++w) {
    int own = 0, uni = 0;
    for (int i = tid; i < words; i += kTcThreads) {
      own += __popc(S.warp_bm[w][i]);
      uni += __popc(S.warp_bm[w][i] | S.cta_bm[i]);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      own += __shfl_xor_sync(0xffffffffu, own, off);
      uni += __shfl_xor_sync(0xffffffffu, uni, off);
    }
    if (lane == 0) S.red[warp] = own | (uni << 16);
    __syncthreads();
    own = uni = 0;
#pragma unroll
    for (int i = 0; i < kWarps; ++i) {
      own += S.red[i] & 0xffff;
      uni += S.red[i] >> 16;
    }
    nkeys[w] = own;
    const bool rows_w = q_lo + w * 16 < q_lo + nq;
    if (rows_w && own <= kw_cap && uni <= rows_cap) {
      for (int i = tid; i < words; i += kTcThreads) S.cta_bm[i] |= S.warp_bm[w][i];
      nrows = uni;
    } else if (rows_w) {
      walk_mask |= 1u << w;
    }
    __syncthreads();
  }
  // exclusive popcount prefixes: the CTA bitmap by all threads (one word each
  // per pass, pass totals carried), each good warp's bitmap by that warp
  {
    int carry = 0;
    for (int base = 0; base < words; base += kTcThreads) {
      const int i = base + tid;
      const int c = i < words ? __popc(S.cta_bm[i]) : 0;
      int x = c;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, off);
        if (lane >= off) x += y;
      }
      if (lane == 31) S.red[warp] = x;
      __syncthreads();
      int before = carry;
      for (int w = 0; w < warp; ++w) before += S.red[w];
      if (i < words) S.cta_pref[i] = before + x - c;
      for (int w = 0; w < kWarps; ++w) carry += S.red[w];
      __syncthreads();
    }
  }
  if (!((walk_mask >> warp) & 1u)) {
    int carry = 0;
    for (int base = 0; base < words; base += 32) {
      const int i = base + lane;
      const int c = i < words ? __popc(S.warp_bm[warp][i]) : 0;
      int x = c;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, off);
        if (lane >= off) x += y;
      }
      if (i < words) S.warp_pref[warp][i] = carry + x - c;
      carry += __shfl_sync(0xffffffffu, x, 31);
    }
  }
  __syncthreads();
  auto cta_slot = [&](int n) {
    return S.cta_pref[n >> 5] + __popc(S.cta_bm[n >> 5] & ((1u << (n & 31)) - 1u));
  };
  auto warp_col = [&](int w, int n) {
    return S.warp_pref[w][n >> 5] + __popc(S.warp_bm[w][n >> 5] & ((1u << (n & 31)) - 1u));
  };
  // staged rows in ascending node order
  for (int i = tid; i < words; i += kTcThreads) {
    uint32_t bits = S.cta_bm[i];
    int slot = S.cta_pref[i];
    while (bits) {
      const int b = __ffs(bits) - 1;
      bits &= bits - 1u;
      out[TilePlanRec::kStaged + slot++] = uint32_t(32 * i + b);
    }
  }
  // key columns -> staged slots (padded columns repeat the last key)
  const bool good = !((walk_mask >> warp) & 1u);
  if (good) {
    for (int i = lane; i < words; i += 32) {
      uint32_t bits = S.warp_bm[warp][i];
      int col = S.warp_pref[warp][i];
      while (bits) {
        const int b = __ffs(bits) - 1;
        bits &= bits - 1u;
        S.kcol[warp][col++] = cta_slot(32 * i + b);
      }
    }
  }
  __syncwarp();
  const int nk = good ? nkeys[warp] : 0;
  const int kp = (nk + 15) & ~15;
  for (int c = 2 * lane; c < kTcMaxKeys; c += 64) {
    const uint32_t lo = c < kp ? uint32_t(S.kcol[warp][min(c, nk - 1)]) : 0u;
    const uint32_t hi = c + 1 < kp ? uint32_t(S.kcol[warp][min(c + 1, nk - 1)]) : 0u;
    out[TilePlanRec::kSlots + warp * (kTcMaxKeys / 2) + c / 2] = lo | (hi << 16);
  }
  // walk-key masks: thread (g, t) of the warp owns column c of rows g and g + 8
  // in block c / 8, element c % 2, when (c % 8) / 2 == t
  uint32_t sel[2] = {0u, 0u};
  const int g = lane >> 2, t = lane & 3;
  if (good) {
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int r = warp * 16 + g + 8 * half;
      if (r >= nq) continue;
      for (int s2 = 0; s2 < S.walk_len[r]; ++s2) {
        const int c = warp_col(warp, S.walk[r][s2]);
        if (((c >> 1) & 3) == t) sel[half] |= 1u << (((c >> 3) << 1) | (c & 1));
      }
    }
  }
  out[TilePlanRec::kSel + 2 * tid] = sel[0];
  out[TilePlanRec::kSel + 2 * tid + 1] = sel[1];
  if (lane == 0) {
    const int wn = max(0, min(16, nq - warp * 16));
    out[4 + warp] = uint32_t(wn) | (uint32_t(nk) << 16);
  }
  if (tid == 0) {
    out[1] = walk_mask;
    out[2] = uint32_t(nq);
    out[3] = uint32_t(nrows);
  }
}

// Resident CTAs per SM of one instantiation at this shared-memory size
// (memoised: the size depends only on the tree shape).
template <typename T, int D, int NBK, int MINB, int MODE>
int resident_ctas(int smem) {
  // (smem << 32 | occupancy) of the last query on each device; atomic so that
  // host threads launching concurrently read a consistent pair
  static std::atomic<int64_t> memo[kQaMaxDevices];
  static std::once_flag init;
  std::call_once(init, [] {
    for (auto& x : memo) x.store(-1);
  });
  const int dev = qa_current_device();
  const int64_t m = memo[dev].load(std::memory_order_relaxed);
  if (m >= 0 && int(m >> 32) == smem) return int(m & 0xffffffff);
  {
    if (qa_smem_attr(reinterpret_cast<const void*>(ancestor_tc_kernel<T, D, NBK, MINB, MODE>), kTcMaxSmem) !=
        cudaSuccess)
      return 0;
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, ancestor_tc_kernel<T, D, NBK, MINB, MODE>, kTcThreads,
                                                      smem) != cudaSuccess)
      return 0;
    memo[dev].store((int64_t(smem) << 32) | int64_t(occ), std::memory_order_relaxed);
    return occ;
  }
}

// Launched with programmatic stream serialisation: the kernel may start while
// the previous kernel on the stream finishes; it plans its first tile, then
// waits (griddepcontrol.wait) before its first read of any input.
// Tile-plan tables: kPlanSlots tables of kPlanSlotWords words in a fixed
// device array (no allocation). A table holds every tile's plan of one tree
// shape (branching, depth, length) and is filled once by a planning launch;
// each record carries the key of its table's assignment, so a launch whose
// key does not match (the slot was reassigned) plans on the device instead.
constexpr int kPlanSlots = 4;
constexpr int64_t kPlanSlotWords = int64_t(128) << 10;  // 512 KB per table
__device__ __align__(16) uint32_t g_tile_plans[kPlanSlots * kPlanSlotWords];

struct PlanSlot {
  int dev = -1, b = 0, d = 0, n = 0, sub = 0, rows_cap = 0, kw_cap = 0;
  uint32_t key = 0;
  uint64_t last_use = 0;
};

template <typename T, int D, int NBK, int MINB, int MODE>
int launch_tc(TcParams& p, int64_t blocks, int smem, cudaStream_t st, bool pdl = true);

// Table of this tree shape on the current device, planned on first use with a
// launch on `st` ahead of the attention launch (not while `st` is being
// captured: a captured planning launch would only run when the graph does).
// Returns false when the plans do not fit a table; p.plan stays null then.
// The registry of table assignments: one for the whole library (every kernel
// instantiation shares the tables), keyed by device and tree shape.
struct PlanRegistry {
  std::mutex mu;
  PlanSlot slots[kQaMaxDevices][kPlanSlots];
  uint32_t* base[kQaMaxDevices] = {nullptr};
  uint32_t gen[kQaMaxDevices] = {0};
  uint64_t clock = 0;
};
PlanRegistry& plan_registry() {
  static PlanRegistry r;
  return r;
}

// Table of this tree shape on the current device, planned on first use with a
// launch on `st` ahead of the attention launch (not while `st` is being
// captured: a captured planning launch would only run when the graph does).
// Returns false when the plans do not fit a table; p.plan stays null then.
template <typename T, int D, int NBK, int MINB, int MODE>
bool attach_plan_table(TcParams& p, int smem, cudaStream_t st) {
  p.plan = nullptr;
  p.plan_out = 0;
  if (p.par_plan != nullptr) return false;  // explicit parents carry their own per-call plans
  static const bool disabled = [] {  // QA_TILE_PLAN_TABLES=0 plans every tile on the device
    const char* e = std::getenv("QA_TILE_PLAN_TABLES");
    return e != nullptr && e[0] == '0';
  }();
  if (disabled) return false;
  const int stride = TilePlanRec::words(p.rows_cap);
  if (int64_t(p.geom.tiles) * stride > kPlanSlotWords) return false;
  const int dev = qa_current_device();
  PlanRegistry& R = plan_registry();
  std::lock_guard<std::mutex> lock(R.mu);
  if (R.base[dev] == nullptr) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_tile_plans) != cudaSuccess || ptr == nullptr) return false;
    R.base[dev] = static_cast<uint32_t*>(ptr);
  }
  PlanSlot* slots = R.slots[dev];
  PlanSlot* hit = nullptr;
  for (int i = 0; i < kPlanSlots; ++i) {
    const PlanSlot& sl = slots[i];
    if (sl.key != 0 && sl.b == p.a.branching && sl.d == p.a.max_depth && sl.n == p.a.max_seqlen &&
        sl.sub == MODE && sl.rows_cap == p.rows_cap && sl.kw_cap == p.kw_cap)
      hit = &slots[i];
  }
  if (hit == nullptr) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(st, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) return false;
    hit = &slots[0];  // a free slot, else the least recently used one
    for (int i = 0; i < kPlanSlots; ++i)
      if (slots[i].key == 0 || slots[i].last_use < hit->last_use) hit = &slots[i];
    uint32_t key = 0;
    while (key == 0) key = plan_mix(++R.gen[dev] * 0x9e3779b9u + uint32_t(dev) * 0x7f4a7c15u + 0x6a09e667u);
    TcParams q = p;
    q.plan = R.base[dev] + int64_t(hit - slots) * kPlanSlotWords;
    q.plan_stride = stride;
    q.plan_key = key;
    q.plan_out = 1;
    q.unit_heads = 0;
    hit->key = 0;  // invalid until the planning launch is queued
    // Clear the slot first: the new records do not cover every word of the old
    // ones (different record strides, unwritten tails), and a launch captured
    // in a graph while the old table was valid must find no intact old record.
    if (cudaMemsetAsync(q.plan, 0, size_t(kPlanSlotWords) * sizeof(uint32_t), st) != cudaSuccess) return false;
    if (launch_tc<T, D, NBK, MINB, MODE>(q, p.geom.tiles, smem, st, false) != QA_OK) return false;
    *hit = PlanSlot{dev, p.a.branching, p.a.max_depth, p.a.max_seqlen, MODE, p.rows_cap, p.kw_cap, key, 0};
  }
  hit->last_use = ++R.clock;
  p.plan = R.base[dev] + int64_t(hit - slots) * kPlanSlotWords;
  p.plan_stride = stride;
  p.plan_key = hit->key;
  return true;
}

template <typename T, int D, int NBK, int MINB, int MODE>
int launch_tc(TcParams& p, int64_t blocks, int smem, cudaStream_t st, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(blocks));
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = size_t(smem);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  if (cudaLaunchKernelEx(&cfg, ancestor_tc_kernel<T, D, NBK, MINB, MODE>, p) != cudaSuccess) return QA_ERR_LAUNCH;
  return cudaGetLastError() == cudaSuccess ? QA_OK : QA_ERR_LAUNCH;
}

// Picks the register budget and the persistent grid (one CTA per resident
// slot). The kernel is latency-bound, so resident warps count: the builds
// capped for 3 and 4 CTAs per SM (168 and 128 registers) are used only when
// they raise residency; at equal residency the build with more registers runs
// faster. head_dim 256 is held to <= 2 CTAs by shared memory and uses the
// unconstrained build only.
template <typename T, int D, int NBK, int MODE>
int launch_tc_minb(TcParams& p, cudaStream_t st) {
  const int64_t items = int64_t(p.a.batch) * p.geom.tiles * p.a.num_q_heads;
  const int smem = TcSmem<D>::total(p.rows_cap);
  const int occ1 = resident_ctas<T, D, NBK, 1, MODE>(smem);
  int occ = occ1, minb = 1;
  if constexpr (D <= 128) {
    const int occ3 = resident_ctas<T, D, NBK, 3, MODE>(smem);
    const int occ4 = resident_ctas<T, D, NBK, 4, MODE>(smem);
    if (occ3 > occ) occ = occ3, minb = 3;
    if (occ4 > occ) occ = occ4, minb = 4;
  }
  if (occ <= 0) return QA_ERR_LAUNCH;
  bool table = false;
  if (minb == 4) table = attach_plan_table<T, D, NBK, 4, MODE>(p, smem, st);
  else if (minb == 3) table = attach_plan_table<T, D, NBK, 3, MODE>(p, smem, st);
  else table = attach_plan_table<T, D, NBK, 1, MODE>(p, smem, st);
  int64_t blocks = min(items, int64_t(p.num_sms) * occ);
  // Work split. A tile's plan costs about as much as kPlanHeads heads (the
  // subtree planner more), so an even split of the (tile, head) items, whose
  // ranges touch one or two tiles, is compared with one (tile, head-chunk)
  // unit per CTA when every unit gets a slot; the cheaper estimate wins.
  p.unit_heads = 0;
  {
    // tile plan cost in heads (measured); a plan read from the table costs little
    const double plan = (table || MODE == 2) ? 0.3 : (MODE == 1 ? 2.0 : 1.2);
    const int H = p.a.num_q_heads;
    const int64_t tgs = int64_t(p.a.batch) * p.geom.tiles;
    const double even = double((items + blocks - 1) / blocks) + 2.0 * plan;
    double best = even;
    for (int q = H; q >= 1; --q) {
      const int chunks = (H + q - 1) / q;
      if (tgs * chunks > int64_t(p.num_sms) * occ) break;
      if ((H + chunks - 1) / chunks != q) continue;  // same chunks as a smaller q
      if (plan + q < best) {
        best = plan + q;
        p.unit_heads = q;
      }
    }
    if (p.unit_heads > 0) blocks = tgs * ((H + p.unit_heads - 1) / p.unit_heads);
  }
  if (blocks <= 0) return QA_OK;
  if (minb == 4) return launch_tc<T, D, NBK, 4, MODE>(p, blocks, smem, st);
  if (minb == 3) return launch_tc<T, D, NBK, 3, MODE>(p, blocks, smem, st);
  return launch_tc<T, D, NBK, 1, MODE>(p, blocks, smem, st);
}

template <typename T, int D, int NBK>
int launch_tc_sub(TcParams& p, cudaStream_t st) {
  if (p.par_plan != nullptr) return launch_tc_minb<T, D, NBK, 2>(p, st);
  return p.geom.bands > 0 ? launch_tc_minb<T, D, NBK, 1>(p, st) : launch_tc_minb<T, D, NBK, 0>(p, st);
}

template <typename T, int D>
int launch_tc_nbk(TcParams& p, cudaStream_t st) {
  if (p.kw_cap <= 32) return launch_tc_sub<T, D, 4>(p, st);
  if (p.kw_cap <= 48) return launch_tc_sub<T, D, 6>(p, st);  // e.g. binary trees on subtree tiles
  if (p.kw_cap <= 64) return launch_tc_sub<T, D, 8>(p, st);
  return launch_tc_sub<T, D, 16>(p, st);
}

}  // namespace

// Launches the tensor-core level kernel when it applies (complete-tree mode,
// head_dim 64/128/256, every level of a tile fits in shared memory); returns
// kTcNotApplicable otherwise so the caller runs the scalar walk. Arguments are
// already validated by qa_ancestor_attn.
// Tiling of a launch's trees (memoised per tree shape): contiguous tiles, or
// subtree tiles when they stage far fewer rows per tile (deep trees; their
// capacities come from planning every tile of a max_seqlen-node tree here).
struct TcPlan {
  TileGeom geom;
  int rows_cap = 0, kw_cap = 0;
};
bool tc_plan(int b, int max_depth, int n, TcPlan& out) {
  static std::mutex mu;
  static int key_b = -1, key_d = -1, key_n = -1;
  static TcPlan memo;
  static bool memo_ok = false;
  std::lock_guard<std::mutex> lock(mu);
  if (b != key_b || max_depth != key_d || n != key_n) {
    memo_ok = false;
    // contiguous tiles: the level-range bounds plan_levels_fit stays within
    const int rows_c = rows_needed(kTcMQ, b, max_depth, false);
    const int kw_c = (rows_needed(16, b, max_depth, false) + 15) & ~15;
    if (kw_c <= kTcMaxKeys) {
      memo.geom = make_tile_geom(b, n, false);
      memo.rows_cap = max(rows_c, kTcMQ);  // the epilogue stages the output tile in the V rows
      memo.kw_cap = kw_c;
      memo_ok = true;
    }
    // subtree tiles, when they stage under two thirds of the rows (deep
    // trees); shallower trees keep the cheaper contiguous planning
    const TileGeom gs = make_tile_geom(b, n, true);
    if (gs.bands > 0) {
      int rows = 0, keys = 0;
      tile_geom_caps(gs, n, max_depth, rows, keys);
      rows = max(rows, kTcMQ);
      const int kw = max((keys + 15) & ~15, 16);
      if (kw <= kTcMaxKeys && (!memo_ok || 3 * rows < 2 * memo.rows_cap)) {
        memo.geom = gs;
        memo.rows_cap = rows;
        memo.kw_cap = kw;
        memo_ok = true;
      }
    }
    key_b = b;
    key_d = max_depth;
    key_n = n;
  }
  out = memo;
  return memo_ok;
}

// Explicit parents on the tensor-core kernel: the per-call plans need the
// caller's workspace (qa_ancestor_workspace_bytes); 0 when the path does not
// apply (head_dim, sequence length, walk depth).
int64_t parents_workspace_bytes(const qa_ancestor_args& a) {
  if (a.head_dim != 64 && a.head_dim != 128 && a.head_dim != 256) return 0;
  if (a.max_seqlen <= 0 || a.max_seqlen > kParMaxSeq || a.max_depth + 1 > kMaxLevels || a.batch <= 0) return 0;
  const int tiles = (a.max_seqlen + kTcMQ - 1) / kTcMQ;
  return int64_t(a.batch) * tiles * TilePlanRec::words(kParRowsCap) * int64_t(sizeof(uint32_t));
}

// Explicit-parent plans of every (sequence, tile) into a.workspace.
int launch_parents_plan(const qa_ancestor_args& a, int tiles, int stride, int kw_cap, cudaStream_t st) {
  const int smem = int(sizeof(ParPlanSmem)) + a.max_seqlen * int(sizeof(int));
  if (qa_smem_attr(reinterpret_cast<const void*>(ancestor_parents_plan_kernel), smem) != cudaSuccess)
    return QA_ERR_LAUNCH;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(int64_t(a.batch) * tiles));
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = size_t(smem);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, ancestor_parents_plan_kernel, a, tiles, stride, int(kParRowsCap), kw_cap,
                         static_cast<uint32_t*>(a.workspace)) != cudaSuccess)
    return QA_ERR_LAUNCH;
  return QA_OK;
}

int ancestor_tc_parents_launch(const qa_ancestor_args& a, cudaStream_t st, bool plan_only = false) {
  const int64_t need = parents_workspace_bytes(a);
  if (need == 0 || a.workspace == nullptr || a.workspace_bytes < need ||
      (reinterpret_cast<uintptr_t>(a.workspace) & 15u))
    return kTcNotApplicable;
  TcParams p;
  p.a = a;
  p.scale_log2 = a.scale * kLog2e;
  p.geom = make_tile_geom(2, a.max_seqlen, false);
  p.head_ratio = a.num_q_heads / a.num_kv_heads;
  p.rows_cap = kParRowsCap;
  // key columns per warp: 32 (four S blocks) for shallow trees, whose 16 rows
  // rarely have more walk keys (rows that do go to walk warps), 64 for deeper
  // ones; four blocks run ~15 % faster than eight on C2-sized batches
  p.kw_cap = a.max_depth <= 6 ? 32 : kParKeys;
  p.num_sms = qa_sm_count();
  p.div_b = make_fast_div(2u);
  p.plan = nullptr;
  p.plan_key = 0;
  p.plan_out = 0;
  p.plan_stride = TilePlanRec::words(kParRowsCap);
  p.par_plan = static_cast<const uint32_t*>(a.workspace);
  // plans first (programmatic launch: it waits for the previous kernel before
  // reading parents), then the attention launch reads them after its own wait;
  // workspace_planned = 1: the workspace already holds these plans
  if (a.workspace_planned == 0 || plan_only) {
    const int st_plan = launch_parents_plan(a, int(p.geom.tiles), int(p.plan_stride), int(p.kw_cap), st);
    if (st_plan != QA_OK || plan_only) return st_plan;
  }
  const bool bf = a.dtype == QA_DTYPE_BF16;
  switch (a.head_dim) {
    case 64: return bf ? launch_tc_nbk<__nv_bfloat16, 64>(p, st) : launch_tc_nbk<__half, 64>(p, st);
    case 128: return bf ? launch_tc_nbk<__nv_bfloat16, 128>(p, st) : launch_tc_nbk<__half, 128>(p, st);
    default: return bf ? launch_tc_nbk<__nv_bfloat16, 256>(p, st) : launch_tc_nbk<__half, 256>(p, st);
  }
}

int ancestor_tc_launch(const qa_ancestor_args& a, cudaStream_t st) {
  if (a.parents != nullptr) return ancestor_tc_parents_launch(a, st);
  if (a.head_dim != 64 && a.head_dim != 128 && a.head_dim != 256) return kTcNotApplicable;
  if (a.branching < 2 || a.max_seqlen <= 0) return kTcNotApplicable;  // chains: the scalar walk
  TcPlan plan;
  if (!tc_plan(a.branching, a.max_depth, a.max_seqlen, plan)) return kTcNotApplicable;
  const int rows = plan.rows_cap;
  const int smem = a.head_dim == 64 ? TcSmem<64>::total(rows)
                 : a.head_dim == 128 ? TcSmem<128>::total(rows) : TcSmem<256>::total(rows);
  if (smem > kTcMaxSmem) return kTcNotApplicable;
  TcParams p;
  p.a = a;
  p.scale_log2 = a.scale * kLog2e;
  p.geom = plan.geom;
  p.head_ratio = a.num_q_heads / a.num_kv_heads;
  p.rows_cap = rows;
  p.kw_cap = plan.kw_cap;
  p.num_sms = qa_sm_count();
  p.div_b = make_fast_div(uint32_t(a.branching));
  p.plan = nullptr;
  p.plan_stride = 0;
  p.plan_key = 0;
  p.plan_out = 0;
  p.par_plan = nullptr;
  const bool bf = a.dtype == QA_DTYPE_BF16;
  switch (a.head_dim) {
    case 64: return bf ? launch_tc_nbk<__nv_bfloat16, 64>(p, st) : launch_tc_nbk<__half, 64>(p, st);
    case 128: return bf ? launch_tc_nbk<__nv_bfloat16, 128>(p, st) : launch_tc_nbk<__half, 128>(p, st);
    default: return bf ? launch_tc_nbk<__nv_bfloat16, 256>(p, st) : launch_tc_nbk<__half, 256>(p, st);
  }
}

}  // namespace qa

namespace qa {
// 1 when a plan check has failed since the last qa_ancestor_diagnostics, -1 on error.
int ancestor_diag_pending() {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_anc_diag, sizeof(int)) != cudaSuccess) return -1;
  return v != 0 ? 1 : 0;
}
}  // namespace qa

extern "C" int qa_ancestor_diagnostics(int32_t* out8) {
  using namespace qa;
  int v[8] = {0}, zero[8] = {0};
  if (cudaMemcpyFromSymbol(v, g_anc_diag, sizeof(v)) != cudaSuccess) return QA_ERR_LAUNCH;
  if (v[0] != 0 && cudaMemcpyToSymbol(g_anc_diag, zero, sizeof(zero)) != cudaSuccess) return QA_ERR_LAUNCH;
  if (out8 != nullptr)
    for (int i = 0; i < 8; ++i) out8[i] = v[i];
  return QA_OK;
}

extern "C" int qa_ancestor_workspace_bytes(const qa_ancestor_args* args, int64_t* bytes) {
  if (args == nullptr || bytes == nullptr) return QA_ERR_INVALID;
  *bytes = args->parents != nullptr ? qa::parents_workspace_bytes(*args) : 0;
  return QA_OK;
}

extern "C" int qa_ancestor_plan(const qa_ancestor_args* args, void* stream) {
  using namespace qa;
  if (args == nullptr || args->parents == nullptr || args->cu_seqlens_q == nullptr) return QA_ERR_INVALID;
  const int r = ancestor_tc_parents_launch(*args, reinterpret_cast<cudaStream_t>(stream), true);
  return r == kTcNotApplicable ? QA_ERR_UNSUPPORTED : r;
}
