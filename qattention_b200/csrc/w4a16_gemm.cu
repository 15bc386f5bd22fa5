// W4A16 weight-streaming GEMM (kernel G1), sm_100a tcgen05/TMEM.
//
// Y[M, N] = X[M, K] . dequant(W)[K, N] for int4 weights (symmetric, zero point
// 8, group 128 along K, one fp16 scale per group and output column) and fp16
// activations: the verify-step linears that the reference runs as GPTQModel
// Marlin kernels (scripts/w4a16_e2e.py:698-699, format set by
// scripts/quantize_llama31.py:41-59). Packed layout: qweight int32, tile-major
// [N/128][K/128][128][16] (each 8 KB tile of one GEMM step contiguous; 8
// consecutive k per word, nibbles interleaved so that (w >> 4i) & 0x000F000F is
// the pair (2i, 2i+1)), scales fp16 [K/128, N].
//
// B200 design (128 x 128 output tile per CTA, 64-deep K steps):
//   * One bulk copy per step fetches the contiguous 8 KB packed weight tile
//     (plus a 256-byte TMA of its scales) into a deep ring; TMA streams the
//     activation tile (128-byte swizzle) into a second ring.
//   * Four dequantisation warps (thread = output column) expand 64 int4 values
//     to fp16 in registers — q | 0x6400 reads as 1024 + q, minus 1032 gives
//     q - 8 exactly, times the fp16 scale is one correctly rounded product —
//     and write them into a swizzled K-major B tile (double buffered).
//   * One thread issues tcgen05.mma (M=128, N=128, K=16) with the fp32
//     accumulator in TMEM; commits free the ring stages and B buffers.
//   * The dequant warps read the accumulator back (tcgen05.ld) and store fp16
//     Y, or fp32 partial sums when K is split across CTAs (small M: the grid
//     needs more CTAs than output tiles); a second kernel reduces the splits.
//   * HBM-bound for small M (0.5 byte per weight + 2 bytes per 128 weights),
//     tensor-core-bound for large M. Bounded waits as in the prefix pass.
#include "sm100_ptx.cuh"

#include <cudaTypedefs.h>

namespace qa {

__device__ int g_w4a16_error = 0;


namespace {

constexpr int kBM = 128, kBN = 128, kBK = 128;  // one quantisation group per K step
constexpr int kMaxStages = 8;                     // ring depths are set per launch (<= 8)
// warps 0-3: weight-ring producers (one thread each, round-robin over K steps:
// a single issuing thread sustains only a few bulk copies per microsecond),
// warp 4: activation-ring producer, warp 5: MMA issuer, warps 6-21: dequant.
constexpr int kProducers = 4;
constexpr int kXWarp = 4, kMmaWarp = 5, kDeqWarp0 = 6;
constexpr int kThreads = 704;
constexpr int kDeqThreads = 512;
constexpr uint32_t kTmemCols = 128;
constexpr uint32_t kWaitLimit = 1u << 22;
constexpr int kWBytes = kBN * (kBK / 8) * 4;    // 8 KB packed
constexpr int kSBytes = kBN * 2;                // 256 B of scales
constexpr int kWStageBytes = kWBytes + 1024;    // keep every stage 1 KB aligned
constexpr int kBBytes = kBN * kBK * 2;          // 32 KB dequantised
constexpr int kSmem = 220 * 1024;  // dynamic shared memory (static barriers use the rest); rings laid out per launch

struct W4Params {
  int32_t m_pad;     // swapped mode: X rows per tile (N of the MMA), multiple of 16
  int32_t x_stages;  // activation ring depth
  int32_t w_stages;  // packed-weight ring depth
  int32_t b_bufs;    // dequantised B tiles in flight
  const uint32_t* qweight;  // tile-major [N/128][K/128][128][16]
  const __half* scales;     // [K/128][N]
  void* y;  // fp16 [M, N] (row stride y_stride) or fp32 partials [splits, M, N]
  int64_t y_stride;
  int32_t M, N, K;
  int32_t k_tiles_per_split;
  int32_t split;  // 1 = direct fp16 output
};

// SWAP (M <= 64): D^T = W^T X^T, so the dequantised 128-column weight tile is the
// M=128 A operand and the few activation rows are the narrow B operand; the
// tensor-core time per weight byte then shrinks with M and the kernel is bound
// by the weight stream. Otherwise D = X W with 128-row activation tiles.
template <bool SPLIT, bool SWAP>
__global__ void __launch_bounds__(kThreads, 1)
    w4a16_gemm_kernel(const __grid_constant__ CUtensorMap x_map, const W4Params p) {
  using namespace sm100;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int x_rows = SWAP ? p.m_pad : kBM;  // activation rows per tile
  const int x_bytes = x_rows * kBK * 2;
  const int kXStages = p.x_stages, kWStages = p.w_stages;
  const int kB = p.b_bufs;
  auto sB = [&](int b) { return base + b * kBBytes; };
  auto sW = [&](int st) { return base + kB * kBBytes + st * kWStageBytes; };
  auto sX = [&](int st) { return base + kB * kBBytes + kWStages * kWStageBytes + st * x_bytes; };
  auto sS = [&](int st) { return sW(st) + kWBytes; };

  __shared__ __align__(8) uint64_t bar_w_full[kMaxStages], bar_w_empty[kMaxStages];
  __shared__ __align__(8) uint64_t bar_x_full[kMaxStages], bar_x_empty[kMaxStages];
  __shared__ __align__(8) uint64_t bar_deq_full[8], bar_deq_empty[8], bar_acc, bar_final;
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int mt = blockIdx.x, nt = blockIdx.y, split = blockIdx.z;
  const int k_tiles = p.K / kBK;
  const int kt0 = split * p.k_tiles_per_split;
  const int kt1 = min(k_tiles, kt0 + p.k_tiles_per_split);
  const int nk = max(0, kt1 - kt0);

  if (tid == 0) {
    for (int s = 0; s < kWStages; ++s) {
      mbar_init(&bar_w_full[s], 1);
      mbar_init(&bar_w_empty[s], kDeqThreads);
    }
    for (int s = 0; s < kXStages; ++s) {
      mbar_init(&bar_x_full[s], 1);
      mbar_init(&bar_x_empty[s], 1);
    }
    for (int b = 0; b < 8; ++b) {
      mbar_init(&bar_deq_full[b], kDeqThreads);
      mbar_init(&bar_deq_empty[b], 1);
    }
    mbar_init(&bar_acc, 1);
    mbar_init(&bar_final, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(&tmem_base_sh, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tacc = tmem_base_sh;

  if (warp < kProducers) {
    // ---------------- weight ring: packed tile (8 KB) + its scale row (256 B) ----------------
    if (lane == 0) {
      int issued = 0;
      for (int i = warp; i < nk; i += kProducers) {
        const int st = i % kWStages, kt = kt0 + i;
        if (i >= kWStages && !mbar_wait(&bar_w_empty[st], ((i / kWStages) - 1) & 1, &abort_flag, kWaitLimit)) break;
        mbar_arrive_expect_tx(&bar_w_full[st], kWBytes + kSBytes);
        bulk_load(sW(st), p.qweight + (int64_t(nt) * k_tiles + kt) * (kBN * kBK / 8), kWBytes, &bar_w_full[st]);
        bulk_load(sS(st), p.scales + int64_t(kt) * p.N + nt * kBN, kSBytes, &bar_w_full[st]);
        issued = i + 1;
      }
      if (abort_flag) {  // let this thread's issued copies land before shared memory is released
        for (int i = warp; i < issued; i += kProducers) {
          if (i + kWStages < issued) continue;
          uint32_t n = 0;
          while (!mbar_try_wait(&bar_w_full[i % kWStages], (i / kWStages) & 1) && ++n < kWaitLimit) {}
        }
      }
    }
  } else if (warp == kXWarp) {
    // ---------------- activation ring: one 3-D TMA per step (both 64-column halves) ----------------
    if (lane == 0) {
      prefetch_tensormap(&x_map);
      int issued = 0;
      for (int i = 0; i < nk; ++i) {
        const int st = i % kXStages, kt = kt0 + i;
        if (i >= kXStages && !mbar_wait(&bar_x_empty[st], ((i / kXStages) - 1) & 1, &abort_flag, kWaitLimit)) break;
        mbar_arrive_expect_tx(&bar_x_full[st], x_bytes);
        tma_load_3d(sX(st), &x_map, &bar_x_full[st], 0, mt * x_rows, kt * 2);
        issued = i + 1;
      }
      if (abort_flag) {
        for (int i = max(0, issued - kXStages); i < issued; ++i) {
          uint32_t n = 0;
          while (!mbar_try_wait(&bar_x_full[i % kXStages], (i / kXStages) & 1) && ++n < kWaitLimit) {}
        }
      }
    }
  } else if (warp == kMmaWarp) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc = SWAP ? f16_idesc(0, 0, 0, kBN, uint32_t(x_rows)) : f16_idesc(0, 0, 0, kBM, kBN);
      for (int i = 0; i < nk; ++i) {
        const int sx = i % kXStages, b = i % kB;
        if (!mbar_wait(&bar_x_full[sx], (i / kXStages) & 1, &abort_flag, kWaitLimit)) break;
        if (!mbar_wait(&bar_deq_full[b], (i / kB) & 1, &abort_flag, kWaitLimit)) break;
        tc_fence_after();
        const uint32_t xa = smem_addr(sX(sx)), ba = smem_addr(sB(b));
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk) {
          const uint64_t xd = sw128_desc(xa + (kk / 4) * x_rows * 128 + (kk % 4) * 32, 16, 1024);
          const uint64_t wd = sw128_desc(ba + (kk / 4) * kBN * 128 + (kk % 4) * 32, 16, 1024);
          if constexpr (SWAP) mma_ss(tacc, wd, xd, idesc, (i > 0 || kk > 0) ? 1u : 0u);
          else mma_ss(tacc, xd, wd, idesc, (i > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(&bar_x_empty[sx]);
        mma_commit(&bar_deq_empty[b]);
      }
      mma_commit(&bar_acc);
      mma_commit(&bar_final);
      uint32_t n = 0;
      while (!mbar_try_wait(&bar_final, 0) && ++n < kWaitLimit) {}
    }
  } else if (warp >= kDeqWarp0) {
    // ---------------- dequantisation: thread = (output column, quarter of the 128 k) ----------------
    const int t = tid - kDeqWarp0 * 32;  // 0..511
    const int nrow = t & 127, qk = t >> 7;  // k range [32 qk, 32 qk + 32)
    const int half = qk & 1;                // epilogue column half (warps 4-7 / 8-11)
    bool ok = true;
    for (int i = 0; i < nk; ++i) {
      const int st = i % kWStages, b = i % kB;
      ok = __all_sync(0xffffffffu, mbar_wait(&bar_w_full[st], (i / kWStages) & 1, &abort_flag, kWaitLimit));
      if (!ok) break;
      if (i >= kB) {
        ok = __all_sync(0xffffffffu, mbar_wait(&bar_deq_empty[b], ((i / kB) - 1) & 1, &abort_flag, kWaitLimit));
        if (!ok) break;
      }
      const uint4 w0 = lds128(smem_addr(sW(st)) + nrow * 64 + qk * 16);
      const __half sc = __ushort_as_half(lds16(smem_addr(sS(st)) + nrow * 2));
      mbar_arrive(&bar_w_empty[st]);  // packed words and scale are in registers
      const uint32_t words[4] = {w0.x, w0.y, w0.z, w0.w};
      const __half2 s2 = __halves2half2(sc, sc);
      const __half2 bias = __floats2half2_rn(1032.f, 1032.f);
      // words cover k = 32 qk .. 32 qk + 31: column block qk / 2, chunks 4 (qk % 2) .. +3
      const uint32_t row = smem_addr(sB(b)) + (qk >> 1) * (kBN * 128) + nrow * 128;
#pragma unroll
      for (int cw = 0; cw < 4; ++cw) {
        const int c = 4 * (qk & 1) + cw;
        uint32_t o[4];
#pragma unroll
        for (int i4 = 0; i4 < 4; ++i4) {
          const uint32_t bits = ((words[cw] >> (4 * i4)) & 0x000F000Fu) | 0x64006400u;
          __half2 h = __hsub2(*reinterpret_cast<const __half2*>(&bits), bias);  // q - 8, exact
          h = __hmul2(h, s2);                                                 // one rounding
          o[i4] = *reinterpret_cast<uint32_t*>(&h);
        }
        sts128(row + ((c ^ (nrow & 7)) * 16), o[0], o[1], o[2], o[3]);
      }
      fence_proxy_async_smem();  // make the B tile visible to the tensor cores
      mbar_arrive(&bar_deq_full[b]);
    }
    // ---------------- epilogue: warps 4-7 columns 0-63, warps 8-11 columns 64-127 ----------------
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&bar_acc, 0, &abort_flag, kWaitLimit));
    if (qk >= 2) ok = false;  // the second eight dequant warps do not take part in the epilogue
    if (ok && SWAP) {
      // TMEM lane = output column n, TMEM column = activation row m
      tc_fence_after();
      const int quarter = warp & 3;
      const int n = nt * kBN + quarter * 32 + lane;
#pragma unroll 1
      for (int c4 = half; c4 * 32 < x_rows; c4 += 2) {
        uint32_t acc[32];
        tmem_ld32(tacc + (uint32_t(quarter * 32) << 16) + c4 * 32, acc);
        tmem_wait_ld();
        if (n >= p.N) continue;
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const int m = mt * x_rows + c4 * 32 + c;
          if (m >= p.M || c4 * 32 + c >= x_rows) break;
          if constexpr (SPLIT)
            reinterpret_cast<float*>(p.y)[(int64_t(split) * p.M + m) * p.N + n] = __uint_as_float(acc[c]);
          else
            reinterpret_cast<__half*>(p.y)[int64_t(m) * p.y_stride + n] = __float2half_rn(__uint_as_float(acc[c]));
        }
      }
    } else if (ok) {
      tc_fence_after();
      const int quarter = warp & 3;
      const int row = quarter * 32 + lane;
      const int m = mt * kBM + row;
      const bool m_ok = m < p.M;
#pragma unroll 1
      for (int c4 = 2 * half; c4 < 2 * half + 2; ++c4) {
        uint32_t acc[32];
        tmem_ld32(tacc + (uint32_t(quarter * 32) << 16) + c4 * 32, acc);
        tmem_wait_ld();
        const int n0 = nt * kBN + c4 * 32;
        if (!m_ok || n0 >= p.N) continue;
        if constexpr (SPLIT) {
          float* dst = reinterpret_cast<float*>(p.y) + (int64_t(split) * p.M + m) * p.N + n0;
#pragma unroll
          for (int q = 0; q < 8; ++q)
            reinterpret_cast<uint4*>(dst)[q] = make_uint4(acc[4 * q], acc[4 * q + 1], acc[4 * q + 2], acc[4 * q + 3]);
        } else {
          __half* dst = reinterpret_cast<__half*>(p.y) + int64_t(m) * p.y_stride + n0;
          uint32_t hv[16];
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            __half2 v = __floats2half2_rn(__uint_as_float(acc[2 * c]), __uint_as_float(acc[2 * c + 1]));
            hv[c] = *reinterpret_cast<uint32_t*>(&v);
          }
#pragma unroll
          for (int q = 0; q < 4; ++q)
            reinterpret_cast<uint4*>(dst)[q] = make_uint4(hv[4 * q], hv[4 * q + 1], hv[4 * q + 2], hv[4 * q + 3]);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tacc, kTmemCols);
  }
  if (tid == 0 && abort_flag) atomicExch(&g_w4a16_error, 1);
}

// Y[m, n] = fp16(sum over splits of partial[s, m, n]); 8 columns per thread.
__global__ void w4a16_reduce_kernel(const float* __restrict__ part, __half* __restrict__ y, int64_t y_stride,
                                    int M, int N, int splits) {
  const int64_t idx = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) * 8;
  if (idx >= int64_t(M) * N) return;
  const int m = int(idx / N), n = int(idx % N);
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int s = 0; s < splits; ++s) {
    const float4* src = reinterpret_cast<const float4*>(part + (int64_t(s) * M + m) * N + n);
    const float4 a = src[0], b = src[1];
    acc[0] += a.x; acc[1] += a.y; acc[2] += a.z; acc[3] += a.w;
    acc[4] += b.x; acc[5] += b.y; acc[6] += b.z; acc[7] += b.w;
  }
  uint32_t h[4];
  for (int c = 0; c < 4; ++c) {
    __half2 v = __floats2half2_rn(acc[2 * c], acc[2 * c + 1]);
    h[c] = *reinterpret_cast<uint32_t*>(&v);
  }
  *reinterpret_cast<uint4*>(y + int64_t(m) * y_stride + n) = make_uint4(h[0], h[1], h[2], h[3]);
}

// W'[k, n] = fp16((q - 8) * scale): the reference dequantisation, for tests.
// qw is tile-major [N/128][K/128][128][16]; word index -> (n, 8 consecutive k).
__global__ void w4a16_dequant_kernel(const uint32_t* __restrict__ qw, const __half* __restrict__ scales,
                                     __half* __restrict__ out, int K, int N) {
  const int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;  // one word = 8 k of one n
  if (idx >= int64_t(N) * (K / 8)) return;
  const int w16 = int(idx & 15), row = int((idx >> 4) & 127);
  const int64_t tile = idx >> 11;  // (n tile, k step)
  const int kt = int(tile % (K / 128)), ntile = int(tile / (K / 128));
  const int n = ntile * 128 + row, kw = kt * 16 + w16;
  const uint32_t w = qw[idx];
  const __half sc = scales[int64_t(kw * 8 / 128) * N + n];
  const __half2 s2 = __halves2half2(sc, sc), bias = __floats2half2_rn(1032.f, 1032.f);
#pragma unroll
  for (int i4 = 0; i4 < 4; ++i4) {
    const uint32_t bits = ((w >> (4 * i4)) & 0x000F000Fu) | 0x64006400u;
    const __half2 h = __hmul2(__hsub2(*reinterpret_cast<const __half2*>(&bits), bias), s2);
    out[int64_t(kw * 8 + 2 * i4) * N + n] = __low2half(h);
    out[int64_t(kw * 8 + 2 * i4 + 1) * N + n] = __high2half(h);
  }
}

}  // namespace
}  // namespace qa

namespace qa {
namespace {

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

// Activations [M, K] fp16 viewed as (64 columns, M rows, K/64 column blocks):
// one box of (64, rows, 2) lands as two swizzled [rows][128 B] column blocks.
bool make_x_map(CUtensorMap* map, const void* x, int K, int M, int64_t x_stride, int rows) {
  const auto enc = encode_fn();
  if (enc == nullptr || (x_stride * 2) % 16 != 0) return false;
  const cuuint64_t dims[3] = {64u, cuuint64_t(M), cuuint64_t(K / 64)};
  const cuuint64_t strides[2] = {cuuint64_t(x_stride) * 2, 128u};
  const cuuint32_t box[3] = {64u, cuuint32_t(rows), 2u};
  const cuuint32_t estr[3] = {1u, 1u, 1u};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(x), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int sm_count() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
  }
  return n;
}

}  // namespace

// Split-K factor for an (M, N, K) problem: enough CTAs for every SM when the
// makespan estimate over the candidate split counts.
int w4a16_auto_splits(int M, int N, int K) {
  const int m_tile = M <= 64 ? ((M + 15) / 16) * 16 : kBM;
  const int tiles = ((M + m_tile - 1) / m_tile) * ((N + kBN - 1) / kBN);
  const int k_tiles = K / kBK;
  const int sms = sm_count();
  // minimise (waves of CTAs) x (K steps per CTA + fixed cost of ~3 steps)
  int best = 1;
  double best_cost = 1e30;
  for (int s = 1; s <= k_tiles && s <= 64; s *= 2) {
    const int per = (k_tiles + s - 1) / s;
    const int ctas = tiles * ((k_tiles + per - 1) / per);
    const double cost = double((ctas + sms - 1) / sms) * (per + 3) + (s > 1 ? 2.0 : 0.0);
    if (cost < best_cost) { best_cost = cost; best = s; }
  }
  return best;
}

int w4a16_read_clear_error() {
  int v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, g_w4a16_error, sizeof(int)) != cudaSuccess) return -1;
  if (v != 0) cudaMemcpyToSymbol(g_w4a16_error, &zero, sizeof(int));
  return v;
}

}  // namespace qa

extern "C" int qa_w4a16_plan(int32_t M, int32_t N, int32_t K, int32_t* splits, int64_t* workspace_bytes) {
  using namespace qa;
  if (M <= 0 || N <= 0 || K <= 0 || K % 128 != 0 || N % 128 != 0 || !splits || !workspace_bytes)
    return QA_ERR_INVALID;
  const int s = w4a16_auto_splits(M, N, K);
  *splits = s;
  *workspace_bytes = s > 1 ? int64_t(s) * M * N * 4 : 0;
  return QA_OK;
}

extern "C" int qa_w4a16_gemm(const qa_w4a16_args* args, void* stream) {
  using namespace qa;
  if (args == nullptr) return QA_ERR_INVALID;
  const qa_w4a16_args& a = *args;
  if (a.M < 0 || a.N <= 0 || a.K <= 0 || a.K % 128 != 0 || a.N % 128 != 0 || a.splits < 0) return QA_ERR_INVALID;
  if (a.M == 0) return QA_OK;
  if (!a.x || !a.qweight || !a.scales || !a.y) return QA_ERR_INVALID;
  if ((reinterpret_cast<uintptr_t>(a.x) | reinterpret_cast<uintptr_t>(a.qweight) |
       reinterpret_cast<uintptr_t>(a.y)) & 15u)
    return QA_ERR_ALIGN;
  if (a.x_stride % 8 != 0 || a.y_stride % 8 != 0 || a.N % 8 != 0 ||
      (reinterpret_cast<uintptr_t>(a.scales) & 15u))
    return QA_ERR_ALIGN;
  const int k_tiles = a.K / kBK;
  int splits = a.splits == 0 ? w4a16_auto_splits(a.M, a.N, a.K) : a.splits;
  splits = splits < 1 ? 1 : (splits > k_tiles ? k_tiles : splits);
  const int per = (k_tiles + splits - 1) / splits;
  splits = (k_tiles + per - 1) / per;  // no empty split
  if (splits > 1 && (a.workspace == nullptr || (reinterpret_cast<uintptr_t>(a.workspace) & 15u)))
    return QA_ERR_INVALID;
  const bool swap = a.M <= 64;
  const int m_pad = swap ? ((a.M + 15) / 16) * 16 : kBM;
  CUtensorMap xm;
  if (!make_x_map(&xm, a.x, a.K, a.M, a.x_stride, m_pad)) return QA_ERR_ALIGN;
  W4Params p;
  p.qweight = reinterpret_cast<const uint32_t*>(a.qweight);
  p.scales = reinterpret_cast<const __half*>(a.scales);
  p.m_pad = m_pad;
  {
    // shared memory: dequantised B tiles (32 KB each) + weight ring + activation ring
    const int x_bytes = m_pad * kBK * 2;
    p.b_bufs = 2;
    p.w_stages = swap ? 8 : 4;
    const int avail = kSmem - 1024 - p.b_bufs * kBBytes - p.w_stages * kWStageBytes;
    p.x_stages = avail / x_bytes < kMaxStages ? avail / x_bytes : kMaxStages;
    if (p.x_stages < 2) return QA_ERR_UNSUPPORTED;
  }
  p.M = a.M;
  p.N = a.N;
  p.K = a.K;
  p.k_tiles_per_split = per;
  p.split = splits;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const dim3 grid{unsigned((a.M + m_pad - 1) / m_pad), unsigned((a.N + kBN - 1) / kBN), unsigned(splits)};
  static bool attr[4] = {false, false, false, false};
  const bool split = splits > 1;
  auto kern = split ? (swap ? w4a16_gemm_kernel<true, true> : w4a16_gemm_kernel<true, false>)
                    : (swap ? w4a16_gemm_kernel<false, true> : w4a16_gemm_kernel<false, false>);
  if (!attr[split * 2 + swap]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem) != cudaSuccess)
      return QA_ERR_LAUNCH;
    attr[split * 2 + swap] = true;
  }
  if (split) {
    p.y = a.workspace;
    p.y_stride = a.N;
    kern<<<grid, kThreads, kSmem, st>>>(xm, p);
    const int64_t vec = int64_t(a.M) * a.N / 8;
    w4a16_reduce_kernel<<<unsigned((vec + 255) / 256), 256, 0, st>>>(
        a.workspace, reinterpret_cast<__half*>(a.y), a.y_stride, a.M, a.N, splits);
  } else {
    p.y = a.y;
    p.y_stride = a.y_stride;
    kern<<<grid, kThreads, kSmem, st>>>(xm, p);
  }
  return cudaGetLastError() == cudaSuccess ? QA_OK : QA_ERR_LAUNCH;
}

extern "C" int qa_w4a16_dequant(const int32_t* qweight, const void* scales, void* out, int32_t K, int32_t N,
                                void* stream) {
  using namespace qa;
  if (K <= 0 || N <= 0 || K % 128 != 0 || N % 128 != 0 || !qweight || !scales || !out) return QA_ERR_INVALID;
  const int64_t words = int64_t(N) * (K / 8);
  w4a16_dequant_kernel<<<unsigned((words + 255) / 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const uint32_t*>(qweight), reinterpret_cast<const __half*>(scales),
      reinterpret_cast<__half*>(out), K, N);
  return cudaGetLastError() == cudaSuccess ? QA_OK : QA_ERR_LAUNCH;
}


// ---------------------------------------------------------------------------
// No-allocation variant of qa_w4a16_gemm.
//
// The split-K path needs an fp32 workspace for its partial sums. Callers that
// cannot allocate device memory on their hot path get this entry point
// instead; its workspace is the fixed array below, which every GPU that loads
// this library holds until the process exits.
// ---------------------------------------------------------------------------
namespace qa {
namespace {

constexpr int64_t kNoAllocScratchFloats = int64_t(4) << 20;  // 16 MiB of fp32 partial sums
static __device__ __align__(256) float g_w4a16_scratch[kNoAllocScratchFloats];

constexpr int kMaxDevices = 64;
float* g_scratch_ptr[kMaxDevices] = {nullptr};

// Device address of the scratch array for the current device. In host code the
// array's name is only a host-side stand-in, so the address is looked up once
// per device (with that device current) and cached.
int scratch_for_current_device(float** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return QA_ERR_DEVICE;
  if (g_scratch_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_w4a16_scratch) != cudaSuccess || ptr == nullptr) return QA_ERR_DEVICE;
    g_scratch_ptr[dev] = static_cast<float*>(ptr);
  }
  *out = g_scratch_ptr[dev];
  return QA_OK;
}

}  // namespace
}  // namespace qa

extern "C" int qa_w4a16_gemm_noalloc(const qa_w4a16_args* args, void* stream) {
  using namespace qa;
  if (args == nullptr) return QA_ERR_INVALID;
  qa_w4a16_args a = *args;
  if (a.M < 0 || a.N <= 0 || a.K <= 0 || a.K % 128 != 0 || a.N % 128 != 0 || a.splits < 0) return QA_ERR_INVALID;
  if (a.M == 0) return QA_OK;
  // The split count the GEMM will use is at most this (it only ever lowers it).
  const int splits = a.splits == 0 ? w4a16_auto_splits(a.M, a.N, a.K) : a.splits;
  if (splits > 1) {
    if (int64_t(splits) * a.M * a.N > kNoAllocScratchFloats) return QA_ERR_INVALID;  // beyond the fixed scratch
    float* scratch = nullptr;
    const int st = scratch_for_current_device(&scratch);
    if (st != QA_OK) return st;
    a.workspace = scratch;  // every partial is written before it is read: nothing to clear
  }
  a.splits = splits;
  return qa_w4a16_gemm(&a, stream);
}
