// Shared-prefix pass (kernel P1) of tree verification, sm_100a tcgen05/TMEM.
//
// Computes, for every sequence b and query head h, attention of the tree's
// N query tokens over the L prefix keys (every prefix key is visible to every
// tree query), returning O_pre and the natural-log LSE. This is the dense
// half of tree verification that the reference runs as aten flash SDPA
// (scripts/w4a16_e2e.py:1236-1253, after repeat_kv at :1446-1447) or as the
// tl.dot loop of _ragged_attn_hybrid_kernel (src/ragged_attn.py:1761-1800).
// Its result is merged with the ancestor pass by log-sum-exp (the ancestor
// kernels take it as prefix_o / prefix_lse).
//
// B200 design:
//   * One CTA = 128 packed query rows of one (sequence, KV head): with GQA the
//     G = Hq/Hkv query heads sharing a KV head are packed as rows (token, g),
//     so K/V tiles are read once for all of them (no repeat_kv copies).
//   * TMA (5-D tensor maps over [B, tokens, heads, D] with D split into its
//     two 64-element halves, 128-byte swizzle) streams 128-key K and V tiles
//     through a 3-stage shared-memory ring, one copy per tile (both halves)
//     and K and V issued by two different threads: a single issuing thread
//     sustains only a few TMA copies per microsecond. The Q tile is loaded
//     once. Every copy lands in this CTA's own shared memory only.
//   * One thread issues tcgen05.mma: S_j = Q K_j^T into one of two TMEM
//     buffers (fp32, 128 columns), then O += P_{j-1} V_{j-1} with P read from
//     TMEM (the fp16/bf16 probabilities overwrite their S buffer) and V from
//     shared memory; commits drive the mbarriers.
//   * Four softmax warps own one accumulator row each (TMEM lane = row): read
//     S with tcgen05.ld, keep the running max and sum in fp32, write P back,
//     and rescale O in TMEM only when the max grows by more than 2^8 (lazy
//     rescale; exact result). They also run the epilogue (O / l, LSE).
//   * Every mbarrier wait is bounded: on timeout the CTA sets a device error
//     flag (qa_check_device_error), stops issuing work, waits (bounded) for
//     its in-flight copies and MMAs, frees its TMEM and exits.
#include "sm100_ptx.cuh"

#include <atomic>

#include <cudaTypedefs.h>

#include <type_traits>

namespace qa {

__device__ int g_prefix_error = 0;

namespace {

constexpr int kBM = 128;    // packed query rows per CTA (= TMEM lanes)
constexpr int kBN = 128;    // keys per tile (S MMAs with N = 128 run at the full tensor rate)
constexpr int kStages = 3;  // K/V ring depth
constexpr int kThreads = 224;  // warps 0-3 softmax, 4 Q/K producer, 5 MMA, 6 V producer
constexpr uint32_t kTmemCols = 512;  // 2 x S (128) + O (<= 128) + Q (<= 64)
constexpr uint32_t kWaitLimit = 1u << 22;
constexpr float kLazy = 8.f;

struct PfxParams {
  void* o;
  float* lse;
  int64_t o_stride_b, o_stride_t, o_stride_h;
  int64_t lse_stride_b, lse_stride_t, lse_stride_h;
  int32_t batch, nq, prefix_len, hq, hkv, group;
  int32_t m_tiles;  // per (sequence, kv head)
  int32_t n_tiles;  // key tiles
  float scale_log2;
  uint32_t wait_limit;  // polls of a pipeline wait before the kernel gives up (kWaitLimit)
};

// Pipeline-wait limit of the next launches (0 = kWaitLimit): a test hook that
// makes the bounded waits run out without a fault (qa_set_pipeline_wait_limit).
std::atomic<uint32_t> g_wait_limit{0};

template <int D> struct PfxSmem {
  static constexpr int Q_BYTES = kBM * D * 2;
  static constexpr int KV_BYTES = kBN * D * 2;  // one K or one V tile
  static constexpr int TOTAL = Q_BYTES + kStages * 2 * KV_BYTES + 1024;  // + alignment slack
};

template <typename T> QA_DEVINL uint32_t pack_pair(float lo, float hi);
template <> QA_DEVINL uint32_t pack_pair<__half>(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
template <> QA_DEVINL uint32_t pack_pair<__nv_bfloat16>(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Packed fp32 pair add (sm_100 add.f32x2: one instruction for two lanes).
QA_DEVINL float2 add2(float2 a, float2 b) {
  uint64_t r;
  asm("{.reg .b64 x, y;\n\tmov.b64 x, {%1, %2};\n\tmov.b64 y, {%3, %4};\n\t"
      "add.rn.f32x2 %0, x, y;\n\t}"
      : "=l"(r) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  float2 out;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(out.x), "=f"(out.y) : "l"(r));
  return out;
}

// Softmax / correction / epilogue role: 4 warps, thread = accumulator row.
// All tcgen05.ld/st are warp-collective, so every decision that gates them is
// made warp-uniform (__any_sync / __all_sync).
template <typename T, int D>
__device__ __forceinline__ void softmax_role(const PfxParams& p, uint32_t tbase, int warp, int lane,
                                             int b, int hk, int n0, uint64_t* s_full,
                                             uint64_t* p_full, uint64_t* o_done, uint64_t* q_smem_full,
                                             uint64_t* q_tmem_full, uint32_t sq_addr,
                                             volatile int* abort) {
  using namespace sm100;
  const uint32_t tl = tbase + (uint32_t(warp * 32) << 16);  // this warp's TMEM lanes
  const uint32_t to = tl + 2 * kBN;
  const int ntiles = p.n_tiles;
  float m = -INFINITY, l = 0.f;
  bool ok = true;
  // ---- Q into TMEM (the A operand of S = Q K^T): each thread moves its own
  // row out of the 128-byte-swizzled shared tile, so the S MMAs read only K
  // from shared memory ----
  {
    ok = __all_sync(0xffffffffu, mbar_wait(q_smem_full, 0, abort, p.wait_limit));
    if (!ok) return;
    const int r = warp * 32 + lane;
#pragma unroll
    for (int hb = 0; hb < D / 64; ++hb) {  // 64-element halves of D
      uint32_t qv[32];
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint4 v = lds128(sq_addr + hb * kBM * 128 + r * 128 + ((c ^ (r & 7)) << 4));
        qv[4 * c] = v.x; qv[4 * c + 1] = v.y; qv[4 * c + 2] = v.z; qv[4 * c + 3] = v.w;
      }
      tmem_st32(tl + 2 * kBN + D + hb * 32, qv);
    }
    tmem_wait_st();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(q_tmem_full);
  }
  for (int j = 0; j < ntiles; ++j) {
    ok = __all_sync(0xffffffffu, mbar_wait(&s_full[j & 1], (j >> 1) & 1, abort, p.wait_limit));
    if (!ok) break;
    tc_fence_after();
    constexpr int NC = kBN / 32;  // 32-column chunks of the S tile
    uint32_t r[NC][32];
#pragma unroll
    for (int ch = 0; ch < NC; ++ch) tmem_ld32(tl + (j & 1) * kBN + 32 * ch, r[ch]);
    tmem_wait_ld();
    const int kvalid = min(kBN, p.prefix_len - j * kBN);  // keys past L were zero-filled
    if (kvalid < kBN) {  // only the last tile is partial
#pragma unroll
      for (int ch = 0; ch < NC; ++ch)
#pragma unroll
        for (int c = 0; c < 32; ++c)
          if (32 * ch + c >= kvalid) r[ch][c] = __float_as_uint(-INFINITY);
    }
    // row max on raw scores (the scale is positive), scaled once
    float mxc[NC];
#pragma unroll
    for (int ch = 0; ch < NC; ++ch) {
      mxc[ch] = __uint_as_float(r[ch][0]);
#pragma unroll
      for (int c = 1; c < 32; ++c) mxc[ch] = fmaxf(mxc[ch], __uint_as_float(r[ch][c]));
    }
#pragma unroll
    for (int ch = 1; ch < NC; ++ch) mxc[0] = fmaxf(mxc[0], mxc[ch]);
    const float mx = mxc[0] * p.scale_log2;
    const float m_new = fmaxf(m, mx);
    const bool need = m_new > m + kLazy;  // always true on the first tile
    if (j > 0 && __any_sync(0xffffffffu, need)) {
      // rescale O in TMEM once P_{j-1} V_{j-1} has landed
      ok = __all_sync(0xffffffffu, mbar_wait(o_done, (j - 1) & 1, abort, p.wait_limit));
      if (!ok) break;
      tc_fence_after();
      const float alpha = need ? fast_exp2(m - m_new) : 1.f;
#pragma unroll 1
      for (int c4 = 0; c4 < D / 32; ++c4) {
        uint32_t o[32];
        tmem_ld32(to + 32 * c4, o);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
        tmem_st32(to + 32 * c4, o);
      }
      tmem_wait_st();
    }
    if (need) {
      l *= fast_exp2(m - m_new);
      m = m_new;
    }
    // p = 2^(s * scale - m): one FMA and one exponential per score; P_j
    // (two 16-bit values per column) overwrites the first kBN/2 columns of S_j
    float2 acc2 = make_float2(0.f, 0.f);
#pragma unroll
    for (int pc = 0; pc < NC / 2; ++pc) {
      uint32_t pk[32];
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        const float a = fast_exp2(fmaf(__uint_as_float(r[2 * pc][2 * c]), p.scale_log2, -m));
        const float bb = fast_exp2(fmaf(__uint_as_float(r[2 * pc][2 * c + 1]), p.scale_log2, -m));
        const float x = fast_exp2(fmaf(__uint_as_float(r[2 * pc + 1][2 * c]), p.scale_log2, -m));
        const float y = fast_exp2(fmaf(__uint_as_float(r[2 * pc + 1][2 * c + 1]), p.scale_log2, -m));
        acc2 = add2(acc2, make_float2(a + x, bb + y));
        pk[c] = pack_pair<T>(a, bb);
        pk[16 + c] = pack_pair<T>(x, y);
      }
      tmem_st32(tl + (j & 1) * kBN + 32 * pc, pk);
    }
    const float sum = acc2.x + acc2.y;
    l += sum;
    tmem_wait_st();
    tc_fence_before();
    mbar_arrive(&p_full[j & 1]);
  }
  if (ok) ok = __all_sync(0xffffffffu, mbar_wait(o_done, (ntiles - 1) & 1, abort, p.wait_limit));
  if (!ok) return;
  tc_fence_after();
  // ---- epilogue: row -> (token, head); O / l and LSE ----
  const int row = warp * 32 + lane;
  const int n = n0 + row / p.group;
  const int h = hk * p.group + row % p.group;
  const bool valid = n < p.nq;
  const float inv = 1.f / l;
  T* orow = reinterpret_cast<T*>(p.o) + int64_t(b) * p.o_stride_b + int64_t(n) * p.o_stride_t +
            int64_t(h) * p.o_stride_h;
#pragma unroll 1
  for (int c4 = 0; c4 < D / 32; ++c4) {
    uint32_t o[32];
    tmem_ld32(to + 32 * c4, o);
    tmem_wait_ld();
    if (valid) {
      uint32_t w[16];
#pragma unroll
      for (int c = 0; c < 16; ++c)
        w[c] = pack_pair<T>(__uint_as_float(o[2 * c]) * inv, __uint_as_float(o[2 * c + 1]) * inv);
      uint4* dst = reinterpret_cast<uint4*>(orow + 32 * c4);
#pragma unroll
      for (int q = 0; q < 4; ++q) dst[q] = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
    }
  }
  if (valid && p.lse != nullptr)
    p.lse[int64_t(b) * p.lse_stride_b + int64_t(n) * p.lse_stride_t + int64_t(h) * p.lse_stride_h] =
        (m + __log2f(l)) * kLn2;
}

template <typename T, int D>
__global__ void __launch_bounds__(kThreads, 1)
    prefix_attn_kernel(const __grid_constant__ CUtensorMap q_map,
                       const __grid_constant__ CUtensorMap k_map,
                       const __grid_constant__ CUtensorMap v_map, const PfxParams p) {
  using namespace sm100;
  constexpr uint32_t FMT = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* sQ = base;
  auto sK = [&](int st) { return base + PfxSmem<D>::Q_BYTES + st * 2 * PfxSmem<D>::KV_BYTES; };
  auto sV = [&](int st) { return sK(st) + PfxSmem<D>::KV_BYTES; };

  __shared__ __align__(8) uint64_t bar_q, bar_qt, bar_kv_full[kStages], bar_kv_empty[kStages];
  __shared__ __align__(8) uint64_t bar_s_full[2], bar_p_full[2], bar_o_done, bar_final;
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int mt = int(blockIdx.x % unsigned(p.m_tiles));
  const int rest = int(blockIdx.x / unsigned(p.m_tiles));
  const int hk = rest % p.hkv;
  const int b = rest / p.hkv;
  const int G = p.group;
  const int n0 = mt * (kBM / G);  // first query token of the tile
  const int ntiles = p.n_tiles;

  if (tid == 0) {
    mbar_init(&bar_q, 1);
    mbar_init(&bar_qt, 4);  // Q copied into TMEM by the four softmax warps
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bar_kv_full[s], 2);  // K producer + V producer
      mbar_init(&bar_kv_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bar_s_full[s], 1);
      mbar_init(&bar_p_full[s], 128);
    }
    mbar_init(&bar_o_done, 1);
    mbar_init(&bar_final, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 5) {
    tmem_alloc(&tmem_base_sh, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = tmem_base_sh;
  const uint32_t tmem_o = tbase + 2 * kBN;

  if (warp == 4 || warp == 6) {
    // ---------------- TMA producers: Q once + K tiles (warp 4), V tiles (warp 6) ----------------
    if (lane == 0) {
      const bool is_k = warp == 4;
      const CUtensorMap* map = is_k ? &k_map : &v_map;
      prefetch_tensormap(map);
      if (is_k) {
        prefetch_tensormap(&q_map);
        mbar_arrive_expect_tx(&bar_q, PfxSmem<D>::Q_BYTES);
        tma_load_5d(sQ, &q_map, &bar_q, 0, hk * G, n0, 0, b);
      }
      int issued = 0;
      for (int j = 0; j < ntiles; ++j) {
        const int st = j % kStages;
        if (j >= kStages && !mbar_wait(&bar_kv_empty[st], ((j / kStages) - 1) & 1, &abort_flag, p.wait_limit))
          break;
        // K and V of a stage each add their bytes to the stage's barrier (2 arrivals)
        mbar_arrive_expect_tx(&bar_kv_full[st], PfxSmem<D>::KV_BYTES);
        tma_load_5d(is_k ? sK(st) : sV(st), map, &bar_kv_full[st], 0, hk, j * kBN, 0, b);
        issued = j + 1;
      }
      if (abort_flag) {
        // drain: the copies already issued must land before shared memory is released
        if (is_k) mbar_wait(&bar_q, 0, &abort_flag, kWaitLimit);
        for (int j = max(0, issued - kStages); j < issued; ++j) {
          uint32_t n = 0;
          while (!mbar_try_wait(&bar_kv_full[j % kStages], (j / kStages) & 1) && ++n < kWaitLimit) {}
        }
      }
    }
  } else if (warp == 5) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc_s = f16_idesc(FMT, 0, 0, kBM, kBN);
      const uint32_t idesc_o = f16_idesc(FMT, 0, 1, kBM, D);
      // Descriptors are built once and advanced by constants: the 64-bit
      // bit-field assembly per MMA costs about as much issue time as the MMA.
      // Offsets go into the 16-byte-unit address field (bits 0-13), which
      // shared-memory offsets never carry out of.
      constexpr uint32_t kStageUnits = uint32_t(2 * PfxSmem<D>::KV_BYTES) >> 4;
      const uint64_t k_desc0 = sw128_desc(smem_addr(sK(0)), 16, 1024);
      const uint64_t v_desc0 = sw128_desc(smem_addr(sV(0)), kBN * 128, 1024);
      auto issue_pv = [&](int i) -> bool {
        if (!mbar_wait(&bar_p_full[i & 1], (i >> 1) & 1, &abort_flag, p.wait_limit)) return false;
        tc_fence_after();
        const uint64_t v_desc = v_desc0 + uint64_t((i % kStages) * kStageUnits);
        const uint32_t p_tmem = tbase + (i & 1) * kBN;
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk)
          mma_ts(tmem_o, p_tmem + kk * 8, v_desc + uint64_t(kk * 128), idesc_o, (i > 0 || kk > 0) ? 1u : 0u);
        mma_commit(&bar_o_done);
        mma_commit(&bar_kv_empty[i % kStages]);
        return true;
      };
      bool ok = mbar_wait(&bar_qt, 0, &abort_flag, p.wait_limit);
      const uint32_t q_tmem = tbase + 2 * kBN + D;
      for (int j = 0; ok && j < ntiles; ++j) {
        const int st = j % kStages;
        if (!mbar_wait(&bar_kv_full[st], (j / kStages) & 1, &abort_flag, p.wait_limit)) break;
        tc_fence_after();
        const uint64_t k_desc = k_desc0 + uint64_t(st * kStageUnits);
        const uint32_t s_tmem = tbase + (j & 1) * kBN;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          mma_ts(s_tmem, q_tmem + kk * 8, k_desc + uint64_t((kk / 4) * kBN * 8 + (kk % 4) * 2), idesc_s,
                 kk > 0 ? 1u : 0u);
        mma_commit(&bar_s_full[j & 1]);
        if (j >= 1) ok = issue_pv(j - 1);
      }
      if (ok && !abort_flag) issue_pv(ntiles - 1);
      // every MMA issued by this thread completes before TMEM is released
      mma_commit(&bar_final);
      uint32_t n = 0;
      while (!mbar_try_wait(&bar_final, 0) && ++n < kWaitLimit) {}
    }
  } else {
    softmax_role<T, D>(p, tbase, warp, lane, b, hk, n0, &bar_s_full[0], &bar_p_full[0], &bar_o_done, &bar_q,
                       &bar_qt, smem_addr(sQ), &abort_flag);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tbase, kTmemCols);
  }
  if (tid == 0 && abort_flag) atomicExch(&g_prefix_error, 1);
}

}  // namespace
}  // namespace qa

namespace qa {
namespace {

// cuTensorMapEncodeTiled, resolved through the runtime so that the library
// itself does not link the driver library (it loads on machines without one).
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

// 5-D tensor map over [batch, tokens, heads, D] with D split into 64-element
// halves, dims (innermost first): d within half, heads, tokens, half, batch.
// A box of (64, box_h, box_t, D/64, 1) lands as D/64 column blocks, each
// [box_h * box_t rows][128 B] with the 128-byte swizzle the UMMA descriptors expect.
bool make_map(CUtensorMap* map, const void* ptr, bool bf16, int D, int heads, int tokens, int batch,
              int64_t stride_h, int64_t stride_t, int64_t stride_b, int box_h, int box_t) {
  const cuuint64_t dims[5] = {64u, cuuint64_t(heads), cuuint64_t(tokens), cuuint64_t(D / 64), cuuint64_t(batch)};
  const cuuint64_t strides[4] = {cuuint64_t(stride_h) * 2, cuuint64_t(stride_t) * 2, 128u, cuuint64_t(stride_b) * 2};
  const cuuint32_t box[5] = {64u, cuuint32_t(box_h), cuuint32_t(box_t), cuuint32_t(D / 64), 1u};
  const cuuint32_t estr[5] = {1u, 1u, 1u, 1u, 1u};
  for (int i = 0; i < 4; ++i)
    if (strides[i] % 16 != 0 || strides[i] == 0) return false;
  const auto encode = encode_fn();
  if (encode == nullptr) return false;
  const CUresult r = encode(
      map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 5,
      const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
      CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <typename T, int D>
int launch(const qa_prefix_args& a, cudaStream_t st) {
  const bool bf = std::is_same<T, __nv_bfloat16>::value;
  const int G = a.num_q_heads / a.num_kv_heads;
  CUtensorMap qm, km, vm;
  if (!make_map(&qm, a.q, bf, D, a.num_q_heads, a.num_queries, a.batch, a.q_stride_h, a.q_stride_t,
                a.q_stride_b, G, kBM / G) ||
      !make_map(&km, a.k, bf, D, a.num_kv_heads, a.prefix_len, a.batch, a.k_stride_h, a.k_stride_t,
                a.k_stride_b, 1, kBN) ||
      !make_map(&vm, a.v, bf, D, a.num_kv_heads, a.prefix_len, a.batch, a.v_stride_h, a.v_stride_t,
                a.v_stride_b, 1, kBN))
    return QA_ERR_ALIGN;
  PfxParams p;
  p.o = a.o;
  p.lse = a.lse;
  p.o_stride_b = a.o_stride_b;
  p.o_stride_t = a.o_stride_t;
  p.o_stride_h = a.o_stride_h;
  p.lse_stride_b = a.lse_stride_b;
  p.lse_stride_t = a.lse_stride_t;
  p.lse_stride_h = a.lse_stride_h;
  p.batch = a.batch;
  p.nq = a.num_queries;
  p.prefix_len = a.prefix_len;
  p.hq = a.num_q_heads;
  p.hkv = a.num_kv_heads;
  p.group = G;
  p.m_tiles = (a.num_queries + kBM / G - 1) / (kBM / G);
  p.n_tiles = (a.prefix_len + kBN - 1) / kBN;
  p.scale_log2 = a.scale * kLog2e;
  {
    const uint32_t lim = g_wait_limit.load(std::memory_order_relaxed);
    p.wait_limit = lim != 0 ? lim : kWaitLimit;
  }
  const int64_t blocks = int64_t(a.batch) * a.num_kv_heads * p.m_tiles;
  if (blocks > 0x7fffffffLL) return QA_ERR_INVALID;
  if (qa_smem_attr(reinterpret_cast<const void*>(prefix_attn_kernel<T, D>), PfxSmem<D>::TOTAL) != cudaSuccess)
    return QA_ERR_LAUNCH;
  prefix_attn_kernel<T, D><<<dim3{unsigned(blocks)}, kThreads, PfxSmem<D>::TOTAL, st>>>(qm, km, vm, p);
  return cudaGetLastError() == cudaSuccess ? QA_OK : QA_ERR_LAUNCH;
}

}  // namespace
}  // namespace qa

extern "C" int qa_prefix_attn(const qa_prefix_args* args, void* stream) {
  using namespace qa;
  if (args == nullptr) return QA_ERR_INVALID;
  const qa_prefix_args& a = *args;
  if (a.batch < 0 || a.num_queries < 0 || a.prefix_len < 1 || a.num_q_heads <= 0 || a.num_kv_heads <= 0)
    return QA_ERR_INVALID;
  if (a.num_q_heads % a.num_kv_heads != 0) return QA_ERR_INVALID;
  const int G = a.num_q_heads / a.num_kv_heads;
  if (G > kBM || kBM % G != 0) return QA_ERR_UNSUPPORTED;
  if (a.dtype != QA_DTYPE_F16 && a.dtype != QA_DTYPE_BF16) return QA_ERR_UNSUPPORTED;
  if (a.head_dim != 64 && a.head_dim != 128) return QA_ERR_UNSUPPORTED;
  if (a.batch == 0 || a.num_queries == 0) return QA_OK;
  if (!a.q || !a.k || !a.v || !a.o) return QA_ERR_INVALID;
  for (const void* ptr : {a.q, a.k, a.v, static_cast<const void*>(a.o)})
    if (reinterpret_cast<uintptr_t>(ptr) & 15u) return QA_ERR_ALIGN;
  if ((a.o_stride_b % 8) || (a.o_stride_t % 8) || (a.o_stride_h % 8)) return QA_ERR_ALIGN;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const bool bf = a.dtype == QA_DTYPE_BF16;
  if (a.head_dim == 64) return bf ? launch<__nv_bfloat16, 64>(a, st) : launch<__half, 64>(a, st);
  return bf ? launch<__nv_bfloat16, 128>(a, st) : launch<__half, 128>(a, st);
}

namespace qa {
int w4a16_read_clear_error();  // w4a16_gemm.cu
int ancestor_diag_pending();           // ancestor_tc.cu
}

extern "C" int qa_check_device_error(int* flag) {
  if (flag == nullptr) return QA_ERR_INVALID;
  int v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, qa::g_prefix_error, sizeof(int)) != cudaSuccess) return QA_ERR_LAUNCH;
  if (v != 0 && cudaMemcpyToSymbol(qa::g_prefix_error, &zero, sizeof(int)) != cudaSuccess)
    return QA_ERR_LAUNCH;
  const int w = qa::w4a16_read_clear_error();
  if (w < 0) return QA_ERR_LAUNCH;
  const int d0 = qa::ancestor_diag_pending();
  if (d0 < 0) return QA_ERR_LAUNCH;
  *flag = v | w | (d0 != 0 ? 4 : 0);
  return QA_OK;
}

extern "C" int qa_set_pipeline_wait_limit(uint32_t polls) {
  qa::g_wait_limit.store(polls, std::memory_order_relaxed);
  return QA_OK;
}
