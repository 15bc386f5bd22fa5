// W4A16 weight-streaming GEMM (kernel G1), sm_100a tcgen05/TMEM.
//
// Y[M, N] = X[M, K] . dequant(W)[K, N] for int4 weights (symmetric, zero point
// 8, group 128 along K, one fp16 scale per group and output column) and fp16
// activations: the verify-step linears that the reference runs as GPTQModel
// Marlin kernels (scripts/w4a16_e2e.py:698-699, format set by
// scripts/quantize_llama31.py:41-59). Packed layout: qweight int32 [N, K/8]
// (8 consecutive k per word, nibbles interleaved so that (w >> 4i) & 0x000F000F
// is the pair (2i, 2i+1)), scales fp16 [K/128, N].
//
// B200 design (128 x 128 output tile per CTA, 64-deep K steps):
//   * TMA streams the X tile (128 rows x 64 k, 128-byte swizzle) and the packed
//     weight tile (128 columns x 8 words) through a 4-stage ring.
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

constexpr int kBM = 128, kBN = 128, kBK = 64, kStages = 4;
constexpr int kThreads = 192;  // warp 0 TMA, warp 1 MMA, warps 2-5 dequant + epilogue
constexpr uint32_t kTmemCols = 128;
constexpr uint32_t kWaitLimit = 1u << 22;
constexpr int kXBytes = kBM * kBK * 2;      // 16 KB
constexpr int kWBytes = kBN * (kBK / 8) * 4;  // 4 KB packed
constexpr int kBBytes = kBN * kBK * 2;      // 16 KB dequantised
constexpr int kSmem = kStages * (kXBytes + kWBytes) + 2 * kBBytes + 1024;

struct W4Params {
  const __half* scales;  // [K/128, N]
  void* y;               // fp16 [M, N] (row stride y_stride) or fp32 partials [splits, M, N]
  int64_t y_stride;
  int32_t M, N, K;
  int32_t k_tiles_per_split;
  int32_t split;  // 1 = direct fp16 output
};

template <bool SPLIT>
__global__ void __launch_bounds__(kThreads, 1)
    w4a16_gemm_kernel(const __grid_constant__ CUtensorMap x_map, const __grid_constant__ CUtensorMap w_map,
                      const W4Params p) {
  using namespace sm100;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  auto sX = [&](int st) { return base + st * kXBytes; };
  auto sB = [&](int b) { return base + kStages * kXBytes + b * kBBytes; };
  auto sW = [&](int st) { return base + kStages * kXBytes + 2 * kBBytes + st * kWBytes; };

  __shared__ __align__(8) uint64_t bar_full[kStages], bar_empty[kStages];
  __shared__ __align__(8) uint64_t bar_deq_full[2], bar_deq_empty[2], bar_acc, bar_final;
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int mt = blockIdx.x, nt = blockIdx.y, split = blockIdx.z;
  const int k_tiles = p.K / kBK;
  const int kt0 = split * p.k_tiles_per_split;
  const int kt1 = min(k_tiles, kt0 + p.k_tiles_per_split);
  const int nk = max(0, kt1 - kt0);

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bar_full[s], 1);
      mbar_init(&bar_empty[s], 1 + 128);  // MMA commit + every dequant thread
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bar_deq_full[b], 128);
      mbar_init(&bar_deq_empty[b], 1);
    }
    mbar_init(&bar_acc, 1);
    mbar_init(&bar_final, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&tmem_base_sh, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tacc = tmem_base_sh;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      prefetch_tensormap(&x_map);
      prefetch_tensormap(&w_map);
      int issued = 0;
      for (int i = 0; i < nk; ++i) {
        const int st = i % kStages, kt = kt0 + i;
        if (i >= kStages && !mbar_wait(&bar_empty[st], ((i / kStages) - 1) & 1, &abort_flag, kWaitLimit)) break;
        mbar_arrive_expect_tx(&bar_full[st], kXBytes + kWBytes);
        tma_load_2d(sX(st), &x_map, &bar_full[st], kt * kBK, mt * kBM);
        tma_load_2d(sW(st), &w_map, &bar_full[st], kt * (kBK / 8), nt * kBN);
        issued = i + 1;
      }
      if (abort_flag) {  // let issued copies land before shared memory is released
        for (int i = max(0, issued - kStages); i < issued; ++i) {
          uint32_t n = 0;
          while (!mbar_try_wait(&bar_full[i % kStages], (i / kStages) & 1) && ++n < kWaitLimit) {}
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc = f16_idesc(0, 0, 0, kBM, kBN);
      for (int i = 0; i < nk; ++i) {
        const int st = i % kStages, b = i & 1;
        if (!mbar_wait(&bar_full[st], (i / kStages) & 1, &abort_flag, kWaitLimit)) break;
        if (!mbar_wait(&bar_deq_full[b], (i >> 1) & 1, &abort_flag, kWaitLimit)) break;
        tc_fence_after();
        const uint32_t xa = smem_addr(sX(st)), ba = smem_addr(sB(b));
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk)
          mma_ss(tacc, sw128_desc(xa + kk * 32, 16, 1024), sw128_desc(ba + kk * 32, 16, 1024), idesc,
                 (i > 0 || kk > 0) ? 1u : 0u);
        mma_commit(&bar_empty[st]);
        mma_commit(&bar_deq_empty[b]);
      }
      mma_commit(&bar_acc);
      mma_commit(&bar_final);
      uint32_t n = 0;
      while (!mbar_try_wait(&bar_final, 0) && ++n < kWaitLimit) {}
    }
  } else {
    // ---------------- dequantisation (thread = output column) ----------------
    const int t = tid - 64;  // 0..127
    const int n = nt * kBN + t;
    const bool n_ok = n < p.N;
    bool ok = true;
    for (int i = 0; i < nk; ++i) {
      const int st = i % kStages, b = i & 1, kt = kt0 + i;
      ok = __all_sync(0xffffffffu, mbar_wait(&bar_full[st], (i / kStages) & 1, &abort_flag, kWaitLimit));
      if (!ok) break;
      if (i >= 2) {
        ok = __all_sync(0xffffffffu, mbar_wait(&bar_deq_empty[b], ((i >> 1) - 1) & 1, &abort_flag, kWaitLimit));
        if (!ok) break;
      }
      const uint4 w0 = *reinterpret_cast<const uint4*>(sW(st) + t * 32);
      const uint4 w1 = *reinterpret_cast<const uint4*>(sW(st) + t * 32 + 16);
      const uint32_t words[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
      const __half sc = n_ok ? p.scales[int64_t(kt * kBK / 128) * p.N + n] : __float2half(0.f);
      const __half2 s2 = __halves2half2(sc, sc);
      const __half2 bias = __floats2half2_rn(1032.f, 1032.f);
      unsigned char* row = sB(b) + t * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint32_t o[4];
#pragma unroll
        for (int i4 = 0; i4 < 4; ++i4) {
          const uint32_t bits = ((words[c] >> (4 * i4)) & 0x000F000Fu) | 0x64006400u;
          __half2 h = __hsub2(*reinterpret_cast<const __half2*>(&bits), bias);  // q - 8, exact
          h = __hmul2(h, s2);                                                 // one rounding
          o[i4] = *reinterpret_cast<uint32_t*>(&h);
        }
        *reinterpret_cast<uint4*>(row + ((c ^ (t & 7)) * 16)) = make_uint4(o[0], o[1], o[2], o[3]);
      }
      fence_proxy_async_smem();  // make the B tile visible to the tensor cores
      mbar_arrive(&bar_deq_full[b]);
      mbar_arrive(&bar_empty[st]);
    }
    // ---------------- epilogue ----------------
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&bar_acc, 0, &abort_flag, kWaitLimit));
    if (ok) {
      tc_fence_after();
      const int quarter = warp & 3;  // TMEM lanes this warp may read
      const int row = quarter * 32 + lane;
      const int m = mt * kBM + row;
      const bool m_ok = m < p.M;
#pragma unroll 1
      for (int c4 = 0; c4 < kBN / 32; ++c4) {
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
          uint32_t h[16];
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            __half2 v = __floats2half2_rn(__uint_as_float(acc[2 * c]), __uint_as_float(acc[2 * c + 1]));
            h[c] = *reinterpret_cast<uint32_t*>(&v);
          }
#pragma unroll
          for (int q = 0; q < 4; ++q)
            reinterpret_cast<uint4*>(dst)[q] = make_uint4(h[4 * q], h[4 * q + 1], h[4 * q + 2], h[4 * q + 3]);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
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
__global__ void w4a16_dequant_kernel(const uint32_t* __restrict__ qw, const __half* __restrict__ scales,
                                     __half* __restrict__ out, int K, int N) {
  const int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;  // one word = 8 k of one n
  if (idx >= int64_t(N) * (K / 8)) return;
  const int n = int(idx / (K / 8)), kw = int(idx % (K / 8));
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

bool make_2d(CUtensorMap* map, const void* ptr, CUtensorMapDataType dt, uint64_t inner, uint64_t outer,
             uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle sw) {
  const auto enc = encode_fn();
  if (enc == nullptr || row_bytes % 16 != 0) return false;
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1u, 1u};
  return enc(map, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
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
// output has few 128 x 128 tiles, each split at least 8 K tiles deep.
int w4a16_auto_splits(int M, int N, int K) {
  const int tiles = ((M + kBM - 1) / kBM) * ((N + kBN - 1) / kBN);
  const int k_tiles = K / kBK;
  int s = 1;
  while (tiles * s < sm_count() && k_tiles / (2 * s) >= 8) s *= 2;
  return s;
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
  if (M <= 0 || N <= 0 || K <= 0 || K % 128 != 0 || N % 8 != 0 || !splits || !workspace_bytes)
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
  if (a.M < 0 || a.N <= 0 || a.K <= 0 || a.K % 128 != 0 || a.N % 8 != 0 || a.splits < 0) return QA_ERR_INVALID;
  if (a.M == 0) return QA_OK;
  if (!a.x || !a.qweight || !a.scales || !a.y) return QA_ERR_INVALID;
  if ((reinterpret_cast<uintptr_t>(a.x) | reinterpret_cast<uintptr_t>(a.qweight) |
       reinterpret_cast<uintptr_t>(a.y)) & 15u)
    return QA_ERR_ALIGN;
  if (a.x_stride % 8 != 0 || a.y_stride % 8 != 0) return QA_ERR_ALIGN;
  const int k_tiles = a.K / kBK;
  int splits = a.splits == 0 ? w4a16_auto_splits(a.M, a.N, a.K) : a.splits;
  splits = splits < 1 ? 1 : (splits > k_tiles ? k_tiles : splits);
  const int per = (k_tiles + splits - 1) / splits;
  splits = (k_tiles + per - 1) / per;  // no empty split
  if (splits > 1 && (a.workspace == nullptr || (reinterpret_cast<uintptr_t>(a.workspace) & 15u)))
    return QA_ERR_INVALID;
  CUtensorMap xm, wm;
  if (!make_2d(&xm, a.x, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, uint64_t(a.K), uint64_t(a.M), uint64_t(a.x_stride) * 2,
               kBK, kBM, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_2d(&wm, a.qweight, CU_TENSOR_MAP_DATA_TYPE_INT32, uint64_t(a.K / 8), uint64_t(a.N),
               uint64_t(a.K / 8) * 4, kBK / 8, kBN, CU_TENSOR_MAP_SWIZZLE_NONE))
    return QA_ERR_ALIGN;
  W4Params p;
  p.scales = reinterpret_cast<const __half*>(a.scales);
  p.M = a.M;
  p.N = a.N;
  p.K = a.K;
  p.k_tiles_per_split = per;
  p.split = splits;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const dim3 grid{unsigned((a.M + kBM - 1) / kBM), unsigned((a.N + kBN - 1) / kBN), unsigned(splits)};
  static bool attr[2] = {false, false};
  const bool split = splits > 1;
  if (!attr[split]) {
    if (cudaFuncSetAttribute(split ? w4a16_gemm_kernel<true> : w4a16_gemm_kernel<false>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem) != cudaSuccess)
      return QA_ERR_LAUNCH;
    attr[split] = true;
  }
  if (split) {
    p.y = a.workspace;
    p.y_stride = a.N;
    w4a16_gemm_kernel<true><<<grid, kThreads, kSmem, st>>>(xm, wm, p);
    const int64_t vec = int64_t(a.M) * a.N / 8;
    w4a16_reduce_kernel<<<unsigned((vec + 255) / 256), 256, 0, st>>>(
        a.workspace, reinterpret_cast<__half*>(a.y), a.y_stride, a.M, a.N, splits);
  } else {
    p.y = a.y;
    p.y_stride = a.y_stride;
    w4a16_gemm_kernel<false><<<grid, kThreads, kSmem, st>>>(xm, wm, p);
  }
  return cudaGetLastError() == cudaSuccess ? QA_OK : QA_ERR_LAUNCH;
}

extern "C" int qa_w4a16_dequant(const int32_t* qweight, const void* scales, void* out, int32_t K, int32_t N,
                                void* stream) {
  using namespace qa;
  if (K <= 0 || N <= 0 || K % 128 != 0 || !qweight || !scales || !out) return QA_ERR_INVALID;
  const int64_t words = int64_t(N) * (K / 8);
  w4a16_dequant_kernel<<<unsigned((words + 255) / 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const uint32_t*>(qweight), reinterpret_cast<const __half*>(scales),
      reinterpret_cast<__half*>(out), K, N);
  return cudaGetLastError() == cudaSuccess ? QA_OK : QA_ERR_LAUNCH;
}
