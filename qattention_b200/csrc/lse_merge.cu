// Two-way log-sum-exp merge (standalone form of the merge that the ancestor
// kernel can also fuse into its epilogue). Arithmetic follows
// _fused_lse_merge_kernel, src/ragged_attn.py:1576-1616:
//   m = max(la, lb); wa = exp(la - m); wb = exp(lb - m)
//   out = (wa * oa + wb * ob) / max(wa + wb, 1e-8)
// One row (b, h, n) per D/8 lanes; 16-byte vectors; arbitrary b/h/n strides,
// so permuted [B, N, H, D] views are consumed without a layout copy.
#include "qa_common.cuh"

namespace qa {
namespace {

struct MergeParams {
  const float* la;
  const float* lb;
  const void* oa;
  const void* ob;
  void* out;
  int32_t B, H, N;
  int64_t sla[3], slb[3], soa[3], sob[3], so[3];
  int64_t rows;
};

template <typename T, int D>
__global__ void __launch_bounds__(256) lse_merge_kernel(const MergeParams p) {
  constexpr int LPI = D / 8;
  const int64_t row = (int64_t(blockIdx.x) * 256 + threadIdx.x) / LPI;
  const int li = threadIdx.x & (LPI - 1);
  if (row >= p.rows) return;
  const int n = int(row % p.N);
  const int64_t r2 = row / p.N;
  const int h = int(r2 % p.H);
  const int b = int(r2 / p.H);
  const float la = __ldg(p.la + b * p.sla[0] + h * p.sla[1] + n * p.sla[2]);
  const float lb = __ldg(p.lb + b * p.slb[0] + h * p.slb[1] + n * p.slb[2]);
  const float mx = fmaxf(la, lb);
  // exp(x) = exp2(x*log2e); inputs are natural-log LSE values.
  const float wa = fast_exp2((la - mx) * kLog2e);
  const float wb = fast_exp2((lb - mx) * kLog2e);
  const float inv = 1.f / fmaxf(wa + wb, 1e-8f);
  const T* pa = reinterpret_cast<const T*>(p.oa) + b * p.soa[0] + h * p.soa[1] + n * p.soa[2] + li * 8;
  const T* pb = reinterpret_cast<const T*>(p.ob) + b * p.sob[0] + h * p.sob[1] + n * p.sob[2] + li * 8;
  T* po = reinterpret_cast<T*>(p.out) + b * p.so[0] + h * p.so[1] + n * p.so[2] + li * 8;
  float fa[8], fb[8], r[8];
  Vec8<T>::to_f32(ld_stream(pa), fa);
  Vec8<T>::to_f32(ld_stream(pb), fb);
#pragma unroll
  for (int e = 0; e < 8; ++e) r[e] = (wa * fa[e] + wb * fb[e]) * inv;
  st_stream(po, Vec8<T>::from_f32(r));
}

template <typename T>
cudaError_t launch(const MergeParams& p, int D, cudaStream_t st) {
  const int64_t threads = p.rows * (D / 8);
  const unsigned blocks = unsigned((threads + 255) / 256);
  switch (D) {
    case 32: lse_merge_kernel<T, 32><<<blocks, 256, 0, st>>>(p); break;
    case 64: lse_merge_kernel<T, 64><<<blocks, 256, 0, st>>>(p); break;
    case 128: lse_merge_kernel<T, 128><<<blocks, 256, 0, st>>>(p); break;
    default: lse_merge_kernel<T, 256><<<blocks, 256, 0, st>>>(p); break;
  }
  return cudaGetLastError();
}

}  // namespace
}  // namespace qa

extern "C" int qa_lse_merge(const float* lse_a, const float* lse_b, const void* out_a,
                            const void* out_b, void* out, int32_t B, int32_t H, int32_t N,
                            int32_t head_dim, const int64_t* sla, const int64_t* slb,
                            const int64_t* soa, const int64_t* sob, const int64_t* so,
                            int32_t dtype, void* stream) {
  using namespace qa;
  if (B < 0 || H < 0 || N < 0) return QA_ERR_INVALID;
  if (dtype != QA_DTYPE_F16 && dtype != QA_DTYPE_BF16) return QA_ERR_UNSUPPORTED;
  if (head_dim != 32 && head_dim != 64 && head_dim != 128 && head_dim != 256)
    return QA_ERR_UNSUPPORTED;
  if (int64_t(B) * H * N == 0) return QA_OK;
  if (!lse_a || !lse_b || !out_a || !out_b || !out || !sla || !slb || !soa || !sob || !so)
    return QA_ERR_INVALID;
  for (const void* ptr : {out_a, out_b, static_cast<const void*>(out)})
    if (reinterpret_cast<uintptr_t>(ptr) & 15u) return QA_ERR_ALIGN;
  for (int i = 0; i < 3; ++i)
    if ((soa[i] % 8) || (sob[i] % 8) || (so[i] % 8)) return QA_ERR_ALIGN;
  MergeParams p;
  p.la = lse_a; p.lb = lse_b; p.oa = out_a; p.ob = out_b; p.out = out;
  p.B = B; p.H = H; p.N = N;
  for (int i = 0; i < 3; ++i) {
    p.sla[i] = sla[i]; p.slb[i] = slb[i]; p.soa[i] = soa[i]; p.sob[i] = sob[i]; p.so[i] = so[i];
  }
  p.rows = int64_t(B) * H * N;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e = dtype == QA_DTYPE_F16 ? launch<__half>(p, head_dim, st)
                                        : launch<__nv_bfloat16>(p, head_dim, st);
  return e == cudaSuccess ? QA_OK : QA_ERR_LAUNCH;
}
