// Elementwise kernels of the W4A16 verify step (bench config C5): the work
// between the GEMMs and the attention of one Llama decoder layer, each fused
// so that it reads and writes its tensors once.
//
//   qa_add_rmsnorm  h += delta (optional); out = rmsnorm(h) * w        (per token)
//   qa_rope_qkv     RoPE on the q and k heads of the fused qkv projection,
//                   q rotated in place, k (rotated) and v written into the
//                   [B, Hkv, S, D] KV cache at token offset `kv_offset`
//   qa_silu_mul     out = silu(gate) * up for the fused [gate | up] projection
//
// These follow the reference's model code path: HF Llama RMSNorm (fp32
// variance, eps inside the rsqrt), rotate-half RoPE with position
// prefix_len + depth for tree tokens (scripts/w4a16_e2e.py:1424-1431, tree
// positions :993), and the SwiGLU MLP. fp16 storage, fp32 arithmetic.
#include "qa_common.cuh"

namespace qa {
namespace {

// Lets a programmatically dependent successor (the next W4A16 GEMM, which waits
// for this kernel's output before reading it) launch and stage its weights now.
__device__ __forceinline__ void allow_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// One CTA per token row; 256 threads, 8 fp16 per 16-byte vector.
__global__ void __launch_bounds__(256) add_rmsnorm_kernel(__half* __restrict__ h, const __half* __restrict__ delta,
                                                          const __half* __restrict__ w, __half* __restrict__ out,
                                                          int hidden, float eps) {
  if (threadIdx.x == 0) allow_dependents();
  const int64_t row = blockIdx.x;
  __half* hr = h + row * hidden;
  const __half* dr = delta ? delta + row * hidden : nullptr;
  __half* orow = out + row * hidden;
  __shared__ float red[8];
  float ss = 0.f;
  for (int c = threadIdx.x * 8; c < hidden; c += 256 * 8) {
    uint4 hv = *reinterpret_cast<const uint4*>(hr + c);
    __half2* hp = reinterpret_cast<__half2*>(&hv);
    if (dr) {
      const uint4 dv = *reinterpret_cast<const uint4*>(dr + c);
      const __half2* dp = reinterpret_cast<const __half2*>(&dv);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 a = __half22float2(hp[i]), b = __half22float2(dp[i]);
        hp[i] = __floats2half2_rn(a.x + b.x, a.y + b.y);
      }
      *reinterpret_cast<uint4*>(hr + c) = hv;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 a = __half22float2(hp[i]);
      ss += a.x * a.x + a.y * a.y;
    }
  }
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) tot += red[i];
  const float inv = rsqrtf(tot / float(hidden) + eps);
  for (int c = threadIdx.x * 8; c < hidden; c += 256 * 8) {
    const uint4 hv = *reinterpret_cast<const uint4*>(hr + c);
    const uint4 wv = *reinterpret_cast<const uint4*>(w + c);
    const __half2* hp = reinterpret_cast<const __half2*>(&hv);
    const __half2* wp = reinterpret_cast<const __half2*>(&wv);
    uint4 ov;
    __half2* op = reinterpret_cast<__half2*>(&ov);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      // HF order: normalise in fp32, round to fp16, then scale by the weight
      const float2 a = __half22float2(hp[i]);
      const __half2 n = __floats2half2_rn(a.x * inv, a.y * inv);
      op[i] = __hmul2(n, wp[i]);
    }
    *reinterpret_cast<uint4*>(orow + c) = ov;
  }
}

// One warp per (token, head) of the q and k heads (and a plain copy for v):
// lane l handles the rotate-half pairs (i, i + D/2) for i = l, l + 32, ...
__global__ void __launch_bounds__(256) rope_qkv_kernel(__half* __restrict__ qkv, const int* __restrict__ pos,
                                                       const float* __restrict__ inv_freq, __half* __restrict__ kc,
                                                       __half* __restrict__ vc, int M, int n_per_seq, int hq, int hkv,
                                                       int D, int64_t kv_stride_b, int64_t kv_stride_h,
                                                       int kv_offset) {
  if (threadIdx.x == 0) allow_dependents();
  const int64_t gw = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int heads = hq + 2 * hkv;
  if (gw >= int64_t(M) * heads) return;
  const int m = int(gw / heads), hh = int(gw % heads);
  const int b = m / n_per_seq, t = m % n_per_seq;
  __half* src = qkv + int64_t(m) * heads * D + int64_t(hh) * D;
  const float p = float(pos[m]);
  const int half = D / 2;
  if (hh < hq + hkv) {
    __half* dst = hh < hq ? src : kc + b * kv_stride_b + int64_t(hh - hq) * kv_stride_h + int64_t(kv_offset + t) * D;
    for (int i = lane; i < half; i += 32) {
      float s, c;
      sincosf(p * inv_freq[i], &s, &c);
      const float x1 = __half2float(src[i]), x2 = __half2float(src[i + half]);
      dst[i] = __float2half_rn(x1 * c - x2 * s);
      dst[i + half] = __float2half_rn(x2 * c + x1 * s);
    }
  } else {
    __half* dst = vc + b * kv_stride_b + int64_t(hh - hq - hkv) * kv_stride_h + int64_t(kv_offset + t) * D;
    for (int i = lane; i < D; i += 32) dst[i] = src[i];
  }
}

__global__ void __launch_bounds__(256) silu_mul_kernel(const __half* __restrict__ gu, __half* __restrict__ out,
                                                       int64_t M, int F) {
  if (threadIdx.x == 0) allow_dependents();
  const int64_t i = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) * 8;  // 8 outputs per thread
  if (i >= M * F) return;
  const int64_t m = i / F, f = i % F;
  const uint4 gv = *reinterpret_cast<const uint4*>(gu + m * 2 * F + f);
  const uint4 uv = *reinterpret_cast<const uint4*>(gu + m * 2 * F + F + f);
  const __half2* gp = reinterpret_cast<const __half2*>(&gv);
  const __half2* up = reinterpret_cast<const __half2*>(&uv);
  uint4 ov;
  __half2* op = reinterpret_cast<__half2*>(&ov);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float2 g = __half22float2(gp[k]), u = __half22float2(up[k]);
    // silu in fp32, rounded to fp16 before the product (HF: act_fn(gate) * up in fp16)
    const __half2 sg = __floats2half2_rn(g.x / (1.f + __expf(-g.x)), g.y / (1.f + __expf(-g.y)));
    op[k] = __hmul2(sg, up[k]);
  }
  *reinterpret_cast<uint4*>(out + i) = ov;
}

}  // namespace
}  // namespace qa

extern "C" int qa_add_rmsnorm(void* h, const void* delta, const void* w, void* out, int32_t M, int32_t hidden,
                              float eps, void* stream) {
  using namespace qa;
  if (!h || !w || !out || M < 0 || hidden <= 0 || hidden % 8 != 0) return QA_ERR_INVALID;
  if ((reinterpret_cast<uintptr_t>(h) | reinterpret_cast<uintptr_t>(delta) | reinterpret_cast<uintptr_t>(w) |
       reinterpret_cast<uintptr_t>(out)) & 15u)
    return QA_ERR_ALIGN;
  if (M == 0) return QA_OK;
  add_rmsnorm_kernel<<<unsigned(M), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<__half*>(h), static_cast<const __half*>(delta), static_cast<const __half*>(w),
      static_cast<__half*>(out), hidden, eps);
  return cudaGetLastError() == cudaSuccess ? QA_OK : QA_ERR_LAUNCH;
}

extern "C" int qa_rope_qkv(void* qkv, const int32_t* pos, const float* inv_freq, void* k_cache, void* v_cache,
                           int32_t M, int32_t n_per_seq, int32_t hq, int32_t hkv, int32_t head_dim,
                           int64_t kv_stride_b, int64_t kv_stride_h, int32_t kv_offset, void* stream) {
  using namespace qa;
  if (!qkv || !pos || !inv_freq || !k_cache || !v_cache || M < 0 || n_per_seq <= 0 || hq <= 0 || hkv <= 0 ||
      head_dim <= 0 || head_dim % 2 != 0 || kv_offset < 0)
    return QA_ERR_INVALID;
  if (M == 0) return QA_OK;
  const int64_t warps = int64_t(M) * (hq + 2 * hkv);
  rope_qkv_kernel<<<unsigned((warps * 32 + 255) / 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<__half*>(qkv), pos, inv_freq, static_cast<__half*>(k_cache), static_cast<__half*>(v_cache), M,
      n_per_seq, hq, hkv, head_dim, kv_stride_b, kv_stride_h, kv_offset);
  return cudaGetLastError() == cudaSuccess ? QA_OK : QA_ERR_LAUNCH;
}

extern "C" int qa_silu_mul(const void* gate_up, void* out, int32_t M, int32_t F, void* stream) {
  using namespace qa;
  if (!gate_up || !out || M < 0 || F <= 0 || F % 8 != 0) return QA_ERR_INVALID;
  if ((reinterpret_cast<uintptr_t>(gate_up) | reinterpret_cast<uintptr_t>(out)) & 15u) return QA_ERR_ALIGN;
  if (M == 0) return QA_OK;
  const int64_t vec = int64_t(M) * F / 8;
  silu_mul_kernel<<<unsigned((vec + 255) / 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half*>(gate_up), static_cast<__half*>(out), M, F);
  return cudaGetLastError() == cudaSuccess ? QA_OK : QA_ERR_LAUNCH;
}
