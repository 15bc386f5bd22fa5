// W4A16 weight-streaming GEMM, sm_100a tcgen05/TMEM.
//
// Y[M, N] = X[M, K] . dequant(W)[K, N] for int4 weights (symmetric, zero point
// 8, group 128 along K, one fp16 scale per group and output column) and fp16
// activations: the verify-step linears that the reference runs as GPTQModel
// Marlin kernels (scripts/w4a16_e2e.py:698-699, format set by
// scripts/quantize_llama31.py:41-59). Packed layout: qweight int32, tile-major
// [N/128][K/128][4][128][4] (each 8 KB tile of one GEMM step contiguous and
// chunk-plane-major inside: 16-byte chunk c of output column j at c*2048 + j*16;
// 8 consecutive k per word, nibbles interleaved so that bits 0-3|16-19 hold
// the pair (0,1), 4-7|20-23 (2,3), 8-11|24-27 (4,5), 12-15|28-31 (6,7)),
// scales fp16 [K/128, N]. Dequantisation w = fp16((q - 8) * scale), one rounding.
//
// The kernel computes D^T = W^T X^T with the dequantised weights as the A
// operand in TMEM (see the kernel's comment); it is HBM-bound for small M
// (0.5 byte per weight + 2 bytes per 128 weights) and tensor-bound for large M.
// Split-K partial sums (small grids) go to an fp32 workspace that a second
// kernel reduces. All waits are bounded (iteration caps, abort flag, device
// error flag read by qa_check_device_error).
#include "sm100_ptx.cuh"

#include <cudaTypedefs.h>

namespace qa {

__device__ int g_w4a16_error = 0;


namespace {

// Bounded wait with a short sleep between polls: most of this kernel's warps
// wait at any moment, and their polls take issue slots from the dequantisation
// warps (32 ns: 1-2 % faster per layer at M = 16 / 64 than none; 512 ns slower).
QA_DEVINL bool w4_wait(uint64_t* bar, uint32_t parity, volatile int* abort, uint32_t limit, uint32_t sleep_ns) {
  using namespace sm100;
  for (uint32_t i = 0; i < limit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort) return false;
    if (sleep_ns) __nanosleep(sleep_ns);
  }
  *abort = 1;
  return false;
}

constexpr int kBK = 128;  // one quantisation group per K step
constexpr uint32_t kSleepLimit = 100000;  // x 64 polls with short sleeps: a wait gives up after about a second
constexpr int kWBytes = 128 * (kBK / 8) * 4;  // 8 KB packed per 128 x 128 tile
constexpr int kSBytes = 128 * 2;              // 256 B of scales

// Y[m, n] = fp16(sum over splits of partial[s, m, n]), summed in split order
// (deterministic). Block = 32 float4 column chunks x 8 split groups: thread
// (c, g) adds splits g, g + 8, ... of its 4 outputs, then the 8 group sums are
// added in g order through shared memory. Many blocks even when M x N is small.
__global__ void __launch_bounds__(256) w4a16_reduce_kernel(const float* __restrict__ part, __half* __restrict__ y,
                                                          int64_t y_stride, int M, int N, int splits) {
  __shared__ float4 sums[8][32];
  sm100::pdl_wait();  // the partial sums are the GEMM's output
  if (threadIdx.x == 0) sm100::pdl_launch_dependents();
  const int c = threadIdx.x & 31, g = threadIdx.x >> 5;
  const int64_t q = int64_t(blockIdx.x) * 32 + c;  // float4 chunk of the M x N output
  const int64_t MN4 = int64_t(M) * N / 4;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  if (q < MN4) {
    const float4* src = reinterpret_cast<const float4*>(part) + q;
#pragma unroll 4
    for (int s = g; s < splits; s += 8) {
      const float4 v = __ldg(src + int64_t(s) * MN4);
      acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    }
  }
  sums[g][c] = acc;
  __syncthreads();
  if (g == 0 && q < MN4) {
#pragma unroll
    for (int k = 1; k < 8; ++k) {
      const float4 v = sums[k][c];
      acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    }
    const int64_t idx = q * 4;
    const int m = int(idx / N), n = int(idx % N);
    const __half2 lo = __floats2half2_rn(acc.x, acc.y), hi = __floats2half2_rn(acc.z, acc.w);
    uint2 o;
    o.x = *reinterpret_cast<const uint32_t*>(&lo);
    o.y = *reinterpret_cast<const uint32_t*>(&hi);
    *reinterpret_cast<uint2*>(y + int64_t(m) * y_stride + n) = o;
  }
}

// W'[k, n] = fp16((q - 8) * scale): the reference dequantisation, for tests.
// qw is tile-major [N/128][K/128][4][128][4]; word index -> (n, 8 consecutive k).
__global__ void w4a16_dequant_kernel(const uint32_t* __restrict__ qw, const __half* __restrict__ scales,
                                     __half* __restrict__ out, int K, int N) {
  const int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;  // one word = 8 k of one n
  if (idx >= int64_t(N) * (K / 8)) return;
  const int w4 = int(idx & 3), row = int((idx >> 2) & 127), c = int((idx >> 9) & 3);
  const int w16 = 4 * c + w4;      // word of the row
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


// ---------------------------------------------------------------------------
// GEMM kernel: dequantised weights live in TMEM (tcgen05.mma with A from TMEM).
//
// D^T[features, tokens] = W^T[features, K] . X^T: the weight tile is the M=128
// A operand and sits in tensor memory, the activation tile is the B operand in
// shared memory (TMA, 128-byte swizzle), the fp32 accumulator is in TMEM.
//   * Per K step one bulk copy per feature tile brings the packed 8 KB tile
//     (stored chunk-plane-major, [16-byte chunk][row], so every dequant thread
//     reads its row's chunks without bank conflicts) into a ring, and one more
//     brings the step's scales.
//   * Dequant thread = one output feature (TMEM lane): it expands its 128
//     int4 values to 64 fp16 pairs in registers and stores them into an A
//     buffer in TMEM (tcgen05.st): no shared-memory operand tile, no
//     generic-to-async proxy fence. NA A buffers rotate between the dequant
//     warps and the MMA thread.
//   * One thread issues the MMAs (M=128 per feature tile, N = tokens, K=16);
//     the FT feature tiles share every activation stage.
//   * Epilogue: the dequant warps read the accumulator back (tcgen05.ld).
// ---------------------------------------------------------------------------
constexpr int kMaxNA = 8;          // A buffers in TMEM
constexpr int kMaxXStages = 10;
constexpr int kMaxWStages = 10;
constexpr int kSmem = 216 * 1024;   // dynamic shared memory, one CTA per SM
constexpr int kSmem2 = 108 * 1024;  // two CTAs per SM

struct GemmParams {
  const uint32_t* qweight;  // tile-major [N/128][K/128][4][128][4]
  const __half* scales;     // [K/128][N]
  void* y;                  // fp16 [M, N] (row stride y_stride) or fp32 partials [splits, M, N]
  int64_t y_stride;
  int32_t M, N, K;
  int32_t tn;        // tokens per CTA (MMA N), multiple of 16, <= 256
  int32_t tn_cols;   // TMEM columns per accumulator (tn rounded up to 32)
  int32_t na;        // A buffers
  int32_t x_stages;
  int32_t w_stages;
  int32_t k_tiles_per_split;
  uint32_t sleep_ns;
  // split-K finished in the kernel: the last CTA of each (feature, token) tile
  // to arrive on its counter adds the tile's partial sums into y_out
  uint32_t* counters;  // nullptr: a separate reduce kernel does it
  __half* y_out;
  int64_t y_out_stride;
};

// CPS = CTAs resident per SM (1 or 2): with 2, each CTA takes half of the
// TMEM columns and of the shared memory, and two independent pipelines
// interleave on the SM (the per-step latency chain of one pipeline caps its
// weight stream well below the SM's share of HBM bandwidth).
// NP producer warps (steps i % NP), NM MMA-issuing warps (steps i % NM, one
// accumulator each) and NG dequant groups of 4 FT warps (steps i % NG): at
// small M each role's barrier round trips, not any unit's throughput, set
// the pace, so several independent chains per role raise the weight stream.
template <int FT, bool SPLIT, int CPS, int NG, int NM, int NP>
__global__ void __launch_bounds__(32 * (NP + NM) + NG * FT * 128, CPS)
    w4a16_gemm_kernel(const __grid_constant__ CUtensorMap x_map, const GemmParams p) {
  using namespace sm100;
  constexpr int kWBytesFT = FT * kWBytes;     // packed weights of one step
  constexpr int kSBytesFT = FT * kSBytes;     // their scales
  constexpr int kWStage = kWBytesFT + 1024;   // stage stride (scales after the weights, 1 KB aligned)
  extern __shared__ unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tn = p.tn;
  const int x_bytes = tn * kBK * 2;
  const int XS = p.x_stages, WS = p.w_stages, NA = p.na;
  auto sX = [&](int st) { return base + st * x_bytes; };
  auto sW = [&](int st) { return base + XS * x_bytes + st * kWStage; };

  __shared__ __align__(8) uint64_t bar_x_full[kMaxXStages], bar_x_empty[kMaxXStages];
  __shared__ __align__(8) uint64_t bar_w_full[kMaxWStages], bar_w_empty[kMaxWStages];
  __shared__ __align__(8) uint64_t bar_a_empty[kMaxNA], bar_acc, bar_step[kMaxXStages];
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int ftile = blockIdx.x, mblk = blockIdx.y, split = blockIdx.z;
  const int k_tiles = p.K / kBK;
  const int kt0 = split * p.k_tiles_per_split;
  const int nk = max(0, min(k_tiles, kt0 + p.k_tiles_per_split) - kt0);
  // Every CTA reads the same activation rows: starting the K loop of CTA x at
  // step x * nk / gridDim.x spreads those reads over the L2 slices (all CTAs
  // on one 4 KB chunk at once queue behind each other). The order of a CTA's
  // accumulation is fixed by its index, so results stay deterministic.
  const int rot = nk > 0 ? int((int64_t(ftile) * nk) / gridDim.x) % nk : 0;
  auto kt_of = [&](int i) { const int j = i + rot; return kt0 + (j >= nk ? j - nk : j); };

  if (tid == 0) {
    // bar_step: one arrival per dequant warp of the step's group, each made
    // after the warp saw the step's activation tile land (bar_x_full) and
    // stored its A rows; the MMA thread waits on it alone, once per step (a
    // wait costs a few hundred cycles in this kernel, and the MMA thread is its
    // critical path)
    for (int s = 0; s < XS; ++s) {
      mbar_init(&bar_x_full[s], 1);
      mbar_init(&bar_x_empty[s], 1);
      mbar_init(&bar_step[s], FT * 4);
    }
    for (int s = 0; s < WS; ++s) {
      mbar_init(&bar_w_full[s], 1);
      mbar_init(&bar_w_empty[s], FT * 4);  // one arrival per warp of the step's dequant group
    }
    for (int b = 0; b < NA; ++b) mbar_init(&bar_a_empty[b], 1);
    mbar_init(&bar_acc, NM);
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&tmem_base_sh, 512 / CPS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (tid == 0) pdl_launch_dependents();  // the next kernel may stage while this one runs
  const uint32_t tbase = tmem_base_sh;
  // TMEM columns: accumulators [1 or 2 MMA threads][FT][tn_cols], then A buffers [NA][FT][64]
  constexpr int nacc = NM;
  auto acc_col = [&](int ft, int par) { return uint32_t((par * FT + ft) * p.tn_cols); };
  auto a_col = [&](int b, int ft) { return uint32_t(nacc * FT * p.tn_cols + (b * FT + ft) * 64); };

  if (warp < NP) {
    // ---------------- producers: step i's activation tile and weight tiles together ----------------
    // Both rings have the same depth and are refilled in lockstep: the SM's
    // copy engine serves requests in order, so an activation tile issued
    // later than the weight stream would wait behind many steps of weights.
    if (lane == 0) {
      const int pw = warp;  // this producer issues the steps i with i % NP == pw
      if (pw == 0) prefetch_tensormap(&x_map);
      const int S = XS;  // == WS
      auto issue_w = [&](int i) {  // one 8 KB bulk copy per feature tile, then the step's scales
        const int st = i % S, kt = kt_of(i);
        mbar_arrive_expect_tx(&bar_w_full[st], kWBytesFT + kSBytesFT);
#pragma unroll
        for (int t = 0; t < FT; ++t)
          bulk_load(sW(st) + t * kWBytes, p.qweight + (int64_t(ftile * FT + t) * k_tiles + kt) * (kWBytes / 4),
                    kWBytes, &bar_w_full[st]);
        bulk_load(sW(st) + kWBytesFT, p.scales + int64_t(kt) * p.N + ftile * FT * 128, kSBytesFT, &bar_w_full[st]);
      };
      // The weights do not depend on the previous kernel: the first stages
      // stream while it finishes (programmatic dependent launch); only a few,
      // so that the first activation tile does not queue behind many of them.
      const int pre = min(nk, min(S, 3));
      for (int i = pw; i < pre; i += NP) issue_w(i);

      pdl_wait();  // the activations are the previous kernel's output
      int issued_x = 0, issued_w = pre;
      for (int i = pw; i < nk; i += NP) {
        const int st = i % S, kt = kt_of(i);
        if (i >= S) {
          const uint32_t ph = ((i / S) - 1) & 1;
          if (!w4_wait(&bar_x_empty[st], ph, &abort_flag, kSleepLimit * 64, p.sleep_ns)) break;
          if (!w4_wait(&bar_w_empty[st], ph, &abort_flag, kSleepLimit * 64, p.sleep_ns)) break;
        }
        mbar_arrive_expect_tx(&bar_x_full[st], x_bytes);
        tma_load_3d(sX(st), &x_map, &bar_x_full[st], 0, mblk * tn, kt * 2);
        issued_x = i + 1;
        if (i >= pre) {
          issue_w(i);
          issued_w = i + 1;
        }
      }
      if (abort_flag) {  // let this producer's issued copies land before shared memory is released
        for (int i = max(0, issued_x - S); i < issued_x; ++i) {
          if (i % NP != pw) continue;
          uint32_t n = 0;
          while (!mbar_try_wait(&bar_x_full[i % S], (i / S) & 1) && ++n < kSleepLimit) {}
        }
        for (int i = max(0, issued_w - S); i < issued_w; ++i) {
          if (i % NP != pw) continue;
          uint32_t n = 0;
          while (!mbar_try_wait(&bar_w_full[i % S], (i / S) & 1) && ++n < kSleepLimit) {}
        }
      }
    }
  } else if (warp < NP + NM) {
    // ---------------- MMA issuer(s) ----------------
    // With `dual`, warp 1 issues the even K steps into accumulator 0 and warp 2
    // the odd ones into accumulator 1, so one thread's barrier waits overlap the
    // other's MMAs (a single issuing thread is this kernel's critical path at
    // small M); the epilogue adds the two accumulators in a fixed order.
    // The issue loop is the throughput limit at small N (an MMA takes ~45
    // cycles at N <= 64), so descriptors are built once: the K-slice kk of
    // stage sx starts (kk / 4) * tn * 128 + (kk % 4) * 32 bytes after the
    // stage, i.e. that many 16-byte units added to the descriptor's address
    // field (bits 0-13, which these offsets never carry out of).
    if (lane == 0) {
      const int par = warp - NP, stride = NM;
      const uint32_t idesc = f16_idesc(0, 0, 0, 128, uint32_t(tn));
      const uint64_t xdesc0 = sw128_desc(smem_addr(sX(0)), 16, 1024);
      const uint32_t x_stage_units = uint32_t(x_bytes >> 4), kblk_units = uint32_t(tn * 8);
      for (int i = par; i < nk; i += stride) {
        const int sx = i % XS, b = i % NA;
        if (!w4_wait(&bar_step[sx], (i / XS) & 1, &abort_flag, kSleepLimit * 64, p.sleep_ns)) break;
        tc_fence_after();
        const uint64_t xd0 = xdesc0 + uint64_t(sx * x_stage_units);
        const uint32_t ta0 = tbase + a_col(b, 0);
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk) {
          const uint64_t xd = xd0 + uint64_t((kk / 4) * kblk_units + (kk % 4) * 2);
#pragma unroll
          for (int ft = 0; ft < FT; ++ft)
            mma_ts(tbase + acc_col(ft, par), ta0 + ft * 64 + kk * 8, xd, idesc, (i >= stride || kk > 0) ? 1u : 0u);
        }
        mma_commit(&bar_x_empty[sx]);
        mma_commit(&bar_a_empty[b]);
      }
      mma_commit(&bar_acc);
    }
  } else {
    // ---------------- dequantisation: thread = output feature, group = every other K step ----------------
    // Dequant warp dw: group gr = dw / (4 FT) takes the steps i with i % 2 == gr
    // (two steps in flight); inside a group, warp w -> feature tile (w / 4) % FT,
    // and the 4 warps of a tile cover the 4 TMEM lane quarters (warp & 3).
    const int dw = (tid - 32 * (NP + NM)) >> 5;
    const int gr = dw / (4 * FT);
    const int ft = (dw >> 2) % FT;
    const int quarter = warp & 3;          // TMEM lanes this warp may access
    const int f = quarter * 32 + lane;     // feature row inside the tile (= TMEM lane)
    const int n = (ftile * FT + ft) * 128 + f;
    // int4 -> fp16 without shifts for half of the pairs: OR-ing 0x6400 onto a
    // nibble at bits 0-3 gives 1024 + q, at bits 4-7 gives 1024 + 16 q; then
    // q - 8 = x - 1032 or x / 16 - 72, both exact in fp16 (constants 0x6408 =
    // 1032, 0x2C00 = 1/16, 0xD480 = -72).
    bool ok = true;
    for (int i = gr; i < nk; i += NG) {
      const int st = i % WS, b = i % NA;
      ok = __all_sync(0xffffffffu, w4_wait(&bar_w_full[st], (i / WS) & 1, &abort_flag, kSleepLimit * 64, p.sleep_ns));
      if (!ok) break;
      // stage layout: [tile][chunk c][row][16 B] then scales [tile][row] fp16
      const uint32_t sw = smem_addr(sW(st));
      uint32_t words[16];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const uint4 v = lds128(sw + ft * kWBytes + c * (128 * 16) + f * 16);
        words[4 * c] = v.x; words[4 * c + 1] = v.y; words[4 * c + 2] = v.z; words[4 * c + 3] = v.w;
      }
      const __half sh = __ushort_as_half(lds16(sw + kWBytesFT + (ft * 128 + f) * 2));
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar_w_empty[st]);  // words and scale are in registers
      const uint32_t s2u = uint32_t(__half_as_ushort(sh)) * 0x00010001u;  // scale in both halves
      if (i >= NA) {
        ok = __all_sync(0xffffffffu, w4_wait(&bar_a_empty[b], ((i / NA) - 1) & 1, &abort_flag, kSleepLimit * 64, p.sleep_ns));
        if (!ok) break;
        tc_fence_after();
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t o[32];
#pragma unroll
        for (int w = 0; w < 8; ++w) {
          // word w holds 8 consecutive k as the pairs (0,1) bits 0-3|16-19,
          // (2,3) bits 4-7|20-23, (4,5) and (6,7) the same 8 bits higher;
          // 13 instructions per 8 weights, written out so that nothing else
          // (moves, conversions) lands between them
          asm("{\n\t.reg .b32 hi, b0, b1, b2, b3, q0, q1, q2, q3;\n\t"
              "shr.b32 hi, %4, 8;\n\t"
              "lop3.b32 b0, %4, 0x000F000F, 0x64006400, 0xEA;\n\t"
              "lop3.b32 b1, %4, 0x00F000F0, 0x64006400, 0xEA;\n\t"
              "lop3.b32 b2, hi, 0x000F000F, 0x64006400, 0xEA;\n\t"
              "lop3.b32 b3, hi, 0x00F000F0, 0x64006400, 0xEA;\n\t"
              "sub.f16x2 q0, b0, %6;\n\t"          // 1024 + q - 1032 = q - 8
              "fma.rn.f16x2 q1, b1, %7, %8;\n\t"   // (1024 + 16 q) / 16 - 72 = q - 8
              "sub.f16x2 q2, b2, %6;\n\t"
              "fma.rn.f16x2 q3, b3, %7, %8;\n\t"
              "mul.rn.f16x2 %0, q0, %5;\n\t"       // (q - 8) * scale, one rounding
              "mul.rn.f16x2 %1, q1, %5;\n\t"
              "mul.rn.f16x2 %2, q2, %5;\n\t"
              "mul.rn.f16x2 %3, q3, %5;\n\t}"
              : "=r"(o[4 * w]), "=r"(o[4 * w + 1]), "=r"(o[4 * w + 2]), "=r"(o[4 * w + 3])
              : "r"(words[8 * h + w]), "r"(s2u), "r"(0x64086408u), "r"(0x2C002C00u), "r"(0xD480D480u));
        }
        tmem_st32(tbase + (uint32_t(quarter * 32) << 16) + a_col(b, ft) + 32 * h, o);
      }
      tmem_wait_st();
      tc_fence_before();
      // the step's activation tile (issued with its weights) has landed as well
      ok = __all_sync(0xffffffffu, w4_wait(&bar_x_full[i % XS], (i / XS) & 1, &abort_flag, kSleepLimit * 64, p.sleep_ns));
      if (!ok) break;
      if (lane == 0) mbar_arrive(&bar_step[i % XS]);  // A rows of step i are in TMEM
    }
    // ---------------- epilogue: TMEM lane = feature n, column = token ----------------
    if (ok) ok = __all_sync(0xffffffffu, w4_wait(&bar_acc, 0, &abort_flag, kSleepLimit * 64, p.sleep_ns));
    if (ok) {
      tc_fence_after();
#pragma unroll 1
      for (int c4 = gr; c4 * 32 < tn; c4 += NG) {  // the groups split the token columns
        uint32_t acc[32];
        tmem_ld32(tbase + (uint32_t(quarter * 32) << 16) + acc_col(ft, 0) + c4 * 32, acc);
#pragma unroll 1
        for (int par = 1; par < NM; ++par) {  // the other MMA warps' accumulators, in order
          if (nk <= par) break;               // (a warp with no step wrote nothing)
          uint32_t acc1[32];
          tmem_ld32(tbase + (uint32_t(quarter * 32) << 16) + acc_col(ft, par) + c4 * 32, acc1);
          tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < 32; ++c) acc[c] = __float_as_uint(__uint_as_float(acc[c]) + __uint_as_float(acc1[c]));
        }
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const int m = mblk * tn + c4 * 32 + c;
          if (c4 * 32 + c >= tn || m >= p.M) break;
          if constexpr (SPLIT)
            reinterpret_cast<float*>(p.y)[(int64_t(split) * p.M + m) * p.N + n] = __uint_as_float(acc[c]);
          else
            reinterpret_cast<__half*>(p.y)[int64_t(m) * p.y_stride + n] = __float2half_rn(__uint_as_float(acc[c]));
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, 512 / CPS);
  }
  if (tid == 0 && abort_flag) atomicExch(&g_w4a16_error, 1);
  if constexpr (SPLIT) {
    if (p.counters != nullptr) {
      // Every CTA of the tile counts in (an aborted one too, so that the
      // counter always returns to zero); the last one sums the splits' partials
      // in split order (deterministic) and writes fp16, then resets the counter.
      __shared__ int last_cta;
      __threadfence();  // this thread's partial sums are visible device-wide
      __syncthreads();
      if (tid == 0) {
        uint32_t* cnt = p.counters + (int64_t(mblk) * gridDim.x + ftile);
        const uint32_t prev = atomicAdd(cnt, 1u);
        last_cta = prev + 1 == gridDim.z;
        if (last_cta) *cnt = 0u;
      }
      __syncthreads();
      if (last_cta) {
        __threadfence();
        const int rows = min(tn, p.M - mblk * tn);
        constexpr int F4 = FT * 128 / 4;  // float4 columns of the tile
        const int n_base = ftile * FT * 128;
        const float* part = reinterpret_cast<const float*>(p.y);
        for (int e = tid; e < rows * F4; e += blockDim.x) {
          const int r = e / F4, c = e - r * F4;
          const int64_t m = int64_t(mblk) * tn + r;
          const int n0 = n_base + 4 * c;
          float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
          for (int sp = 0; sp < int(gridDim.z); ++sp) {
            const float4 v = __ldcg(reinterpret_cast<const float4*>(part + (int64_t(sp) * p.M + m) * p.N + n0));
            acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
          }
          const __half2 lo = __floats2half2_rn(acc.x, acc.y), hi = __floats2half2_rn(acc.z, acc.w);
          uint2 o;
          o.x = *reinterpret_cast<const uint32_t*>(&lo);
          o.y = *reinterpret_cast<const uint32_t*>(&hi);
          *reinterpret_cast<uint2*>(p.y_out + m * p.y_out_stride + n0) = o;
        }
      }
    }
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

int sm_count() { return qa_sm_count(); }

}  // namespace

// Tile shape: FT feature tiles of 128 x tn tokens per CTA.
struct GemmShape {
  int ft, tn, cps;  // feature tiles per CTA, tokens per CTA, CTAs per SM
  int ng = 2, nm = 1, np = 1;  // dequant groups, MMA-issuing warps, producer warps
};
GemmShape gemm_shape(int M, int N) {
  const bool ft2 = N % 256 == 0;
  // M <= 64: one CTA per SM with four producer warps, four MMA warps (one
  // accumulator each) and four dequant groups, i.e. four independent chains per
  // role (measured against two CTAs per SM with two chains each: equal at M = 16,
  // 1-8 % faster at M = 64, and one CTA per SM leaves TMEM for six A buffers)
  if (M <= 64) return {1, ((M + 15) / 16) * 16, 1, 4, 4, 4};
  if (M <= 128) return {ft2 ? 2 : 1, ((M + 15) / 16) * 16, 1};
  if (M <= 256) return {1, ((M + 15) / 16) * 16, 1};
  // up to ~2K tokens two CTAs per SM overlap one CTA's prologue/epilogue with
  // the other's main loop (+8-19 % at M = 1023); beyond that one wide CTA
  if (M <= 2048) return {1, 128, 2};
  return ft2 ? GemmShape{2, 128, 1} : GemmShape{1, 256, 1};
}

// Split-K factor for the GEMM kernel. Unit = one K step of one CTA running
// alone on its SM (~1 us); two CTAs sharing an SM each take ~1.4 units per
// step (measured), so a wave costs (steps per CTA) x (1 or 1.4, by the busiest
// SM's CTA count) + ~4 units of pipeline fill. The reduce pass reads splits x
// M x N fp32 partials (~3 TB/s) and costs a launch (~2 units). Every split
// count is tried (the best ones are often not powers of two).
int w4a16_auto_splits(int M, int N, int K) {
  const GemmShape sh = gemm_shape(M, N);
  const int tiles = ((M + sh.tn - 1) / sh.tn) * (N / (128 * sh.ft));
  const int k_tiles = K / kBK;
  const int sms = sm_count();
  int best = 1;
  double best_cost = 1e30;
  for (int s = 1; s <= k_tiles && s <= 32; ++s) {
    const int per = (k_tiles + s - 1) / s;
    const int splits = (k_tiles + per - 1) / per;
    if (splits != s) continue;  // same partition as a smaller count
    const int64_t ctas = int64_t(tiles) * splits;
    const int64_t slots = int64_t(sms) * sh.cps;
    const int64_t waves = (ctas + slots - 1) / slots;
    const int64_t in_wave = ctas < slots ? ctas : slots;
    const int busiest = int((in_wave + sms - 1) / sms);  // CTAs on the busiest SM
    const double step = busiest >= 2 ? 1.4 : 1.0;
    const double reduce = s > 1 ? 2.0 + double(s) * M * N * 4 / 3.0e12 / 1.0e-6 : 0.0;
    const double cost = double(waves) * (per * step + 4) + reduce;
    if (cost < best_cost) { best_cost = cost; best = s; }
  }
  return best;
}

// Launches the GEMM (and the split-K reduce). Arguments are validated by the caller.
int w4a16_gemm_launch(const qa_w4a16_args& a, int splits, int per, cudaStream_t st) {
  const GemmShape sh = gemm_shape(a.M, a.N);
  CUtensorMap xm;
  if (!make_x_map(&xm, a.x, a.K, a.M, a.x_stride, sh.tn)) return QA_ERR_ALIGN;
  GemmParams p;
  p.qweight = reinterpret_cast<const uint32_t*>(a.qweight);
  p.scales = reinterpret_cast<const __half*>(a.scales);
  p.M = a.M;
  p.N = a.N;
  p.K = a.K;
  p.tn = sh.tn;
  p.tn_cols = ((sh.tn + 31) / 32) * 32;
  p.na = (512 / sh.cps - sh.nm * sh.ft * p.tn_cols) / (sh.ft * 64);
  if (p.na > kMaxNA) p.na = kMaxNA;
  // Role chain c (producer, MMA warp or dequant group) handles the steps i
  // with i % chains == c and waits on ring slots by phase parity, which cannot
  // tell phase k from phase k + 2. Slot counts are therefore multiples of the
  // chain count, so that a slot is only ever reused by the chain that used it
  // last; otherwise a chain could pass its wait two phases early and overwrite
  // a slot (or an A buffer) still in use.
  const int chains = sh.np > sh.nm ? (sh.np > sh.ng ? sh.np : sh.ng) : (sh.nm > sh.ng ? sh.nm : sh.ng);
  p.na -= p.na % chains;
  if (p.na < 2) return QA_ERR_UNSUPPORTED;
  const int w_stage = sh.ft * kWBytes + 1024;
  const int x_bytes = sh.tn * kBK * 2;
  // one ring depth for both (the producer refills them in lockstep)
  const int smem = sh.cps == 2 ? kSmem2 : kSmem;
  int stages = (smem - 1024) / (x_bytes + w_stage);
  if (stages > kMaxXStages) stages = kMaxXStages;
  stages -= stages % chains;
  if (stages < 2) return QA_ERR_UNSUPPORTED;
  p.x_stages = p.w_stages = stages;
  p.k_tiles_per_split = per;
  p.sleep_ns = 32;
  const dim3 grid{unsigned(a.N / (128 * sh.ft)), unsigned((a.M + sh.tn - 1) / sh.tn), unsigned(splits)};
  const bool split = splits > 1;
  using Kern = void (*)(CUtensorMap, GemmParams);
  Kern kern = nullptr;
#define QA_W4_PICK(FT_, CPS_, NG_, NM_, NP_)                                                     \
  if (sh.ft == FT_ && sh.cps == CPS_ && sh.ng == NG_ && sh.nm == NM_ && sh.np == NP_)          \
    kern = split ? w4a16_gemm_kernel<FT_, true, CPS_, NG_, NM_, NP_>                            \
                 : w4a16_gemm_kernel<FT_, false, CPS_, NG_, NM_, NP_>;
  QA_W4_PICK(1, 1, 4, 4, 4)
  QA_W4_PICK(1, 2, 2, 1, 1)
  QA_W4_PICK(2, 1, 2, 1, 1)
  QA_W4_PICK(1, 1, 2, 1, 1)
#undef QA_W4_PICK
  if (kern == nullptr) return QA_ERR_UNSUPPORTED;
  if (qa_smem_attr(reinterpret_cast<const void*>(kern), smem) != cudaSuccess) return QA_ERR_LAUNCH;
  const int threads = 32 * (sh.np + sh.nm) + sh.ng * sh.ft * 128;
  // both kernels are launched as programmatic dependents of their predecessor
  cudaLaunchAttribute pdl[1];
  pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  pdl[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(unsigned(threads));
  cfg.dynamicSmemBytes = size_t(smem);
  cfg.stream = st;
  cfg.attrs = pdl;
  cfg.numAttrs = 1;
  p.counters = nullptr;
  p.y_out = nullptr;
  p.y_out_stride = 0;
  if (split && a.counters != nullptr) {  // one launch: the last CTA of each tile reduces
    p.y = a.workspace;
    p.y_stride = a.N;
    p.counters = a.counters;
    p.y_out = reinterpret_cast<__half*>(a.y);
    p.y_out_stride = a.y_stride;
    if (cudaLaunchKernelEx(&cfg, kern, xm, p) != cudaSuccess) return QA_ERR_LAUNCH;
  } else if (split) {
    p.y = a.workspace;
    p.y_stride = a.N;
    if (cudaLaunchKernelEx(&cfg, kern, xm, p) != cudaSuccess) return QA_ERR_LAUNCH;
    const int64_t vec = int64_t(a.M) * a.N / 4;
    cudaLaunchConfig_t rcfg = {};
    rcfg.gridDim = dim3(unsigned((vec + 31) / 32));
    rcfg.blockDim = dim3(256u);
    rcfg.stream = st;
    rcfg.attrs = pdl;
    rcfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&rcfg, w4a16_reduce_kernel, const_cast<const float*>(a.workspace),
                           reinterpret_cast<__half*>(a.y), int64_t(a.y_stride), int(a.M), int(a.N), splits) !=
        cudaSuccess)
      return QA_ERR_LAUNCH;
  } else {
    p.y = a.y;
    p.y_stride = a.y_stride;
    if (cudaLaunchKernelEx(&cfg, kern, xm, p) != cudaSuccess) return QA_ERR_LAUNCH;
  }
  return cudaGetLastError() == cudaSuccess ? QA_OK : QA_ERR_LAUNCH;
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
  return w4a16_gemm_launch(a, splits, per, reinterpret_cast<cudaStream_t>(stream));
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

// split-K tile counters of the allocation-free entry point (zero at load; each
// call leaves them zero)
constexpr int kNoAllocCounters = 1 << 16;
static __device__ __align__(256) uint32_t g_w4a16_counters[kNoAllocCounters];

constexpr int kMaxDevices = 64;
float* g_scratch_ptr[kMaxDevices] = {nullptr};
uint32_t* g_counters_ptr[kMaxDevices] = {nullptr};

// Device address of the scratch array for the current device. In host code the
// array's name is only a host-side stand-in, so the address is looked up once
// per device (with that device current) and cached.
int scratch_for_current_device(float** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return QA_ERR_DEVICE;
  if (g_scratch_ptr[dev] == nullptr) {
    void* ptr = nullptr, * cptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_w4a16_scratch) != cudaSuccess || ptr == nullptr) return QA_ERR_DEVICE;
    if (cudaGetSymbolAddress(&cptr, g_w4a16_counters) != cudaSuccess || cptr == nullptr) return QA_ERR_DEVICE;
    g_counters_ptr[dev] = static_cast<uint32_t*>(cptr);
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
  // The split count after the same clamps qa_w4a16_gemm applies (at most one
  // split per K step, no empty split), so the size check sees the count that runs.
  const int k_tiles = a.K / kBK;
  auto effective = [k_tiles](int s) {
    s = s < 1 ? 1 : (s > k_tiles ? k_tiles : s);
    const int per = (k_tiles + s - 1) / s;
    return (k_tiles + per - 1) / per;
  };
  const int64_t mn = int64_t(a.M) * a.N;
  int splits = effective(a.splits == 0 ? w4a16_auto_splits(a.M, a.N, a.K) : a.splits);
  if (splits > 1 && int64_t(splits) * mn > kNoAllocScratchFloats) {
    if (a.splits != 0) return QA_ERR_INVALID;  // an explicit split count beyond the fixed scratch
    // automatic mode: the largest split count whose partials fit (1 needs none)
    while (splits > 1 && int64_t(splits) * mn > kNoAllocScratchFloats) splits = effective(splits - 1);
  }
  if (splits > 1) {
    float* scratch = nullptr;
    const int st = scratch_for_current_device(&scratch);
    if (st != QA_OK) return st;
    a.workspace = scratch;  // every partial is written before it is read: nothing to clear
    int dev = 0;
    cudaGetDevice(&dev);
    const int64_t tiles = int64_t(a.N / 128) * ((a.M + 15) / 16);
    a.counters = tiles <= kNoAllocCounters ? g_counters_ptr[dev] : nullptr;
  }
  a.splits = splits;
  return qa_w4a16_gemm(&a, stream);
}
