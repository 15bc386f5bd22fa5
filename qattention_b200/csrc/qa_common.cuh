// Shared device helpers for the tree-verification kernels (sm_100a only).
//
// Element types: fp16 (`__half`) and bf16 (`__nv_bfloat16`) rows are moved as
// 16-byte vectors (8 elements) and widened to fp32 in registers. All softmax
// arithmetic is fp32, in log2 units (scores pre-multiplied by scale*log2(e)),
// and log-sum-exp values leave the kernels in natural-log units, which is the
// convention of the reference's `lse = m + log(l)`.
#pragma once

#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <mutex>
#include <vector>

#include "../../include/qattn_b200.h"

#define QA_DEVINL __device__ __forceinline__

namespace qa {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

template <typename T> struct Vec8;

template <> struct Vec8<__half> {
  QA_DEVINL static void to_f32(const uint4& r, float (&f)[8]) {
    const __half2* h = reinterpret_cast<const __half2*>(&r);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 t = __half22float2(h[i]);
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    }
  }
  QA_DEVINL static uint4 from_f32(const float (&f)[8]) {
    uint4 r;
    __half2* h = reinterpret_cast<__half2*>(&r);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
    return r;
  }
};

template <> struct Vec8<__nv_bfloat16> {
  QA_DEVINL static void to_f32(const uint4& r, float (&f)[8]) {
    // bf16 -> fp32 widening is exact: the bf16 bits are the top half of fp32.
    const uint32_t* w = reinterpret_cast<const uint32_t*>(&r);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  }
  QA_DEVINL static uint4 from_f32(const float (&f)[8]) {
    uint4 r;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&r);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    return r;
  }
};

// Read-only 16-byte load that is not kept in L1 (rows read exactly once).
QA_DEVINL uint4 ld_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// Read-only 16-byte load through L1 (ancestor rows shared by nearby queries).
QA_DEVINL uint4 ld_shared_row(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// Streaming 16-byte store (output rows are written once and not re-read).
QA_DEVINL void st_stream(void* p, const uint4& v) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

// acc += a.lo*b.lo + a.hi*b.hi for packed pairs of 16-bit elements, products
// and sums in fp32 (sm_100 mixed-precision FMA, no conversion instructions).
template <typename T> QA_DEVINL void dot_pair(float& acc, uint32_t a, uint32_t b);
template <> QA_DEVINL void dot_pair<__half>(float& acc, uint32_t a, uint32_t b) {
  asm("{.reg .b16 a0, a1, b0, b1;\n\t"
      "mov.b32 {a0, a1}, %1;\n\t"
      "mov.b32 {b0, b1}, %2;\n\t"
      "fma.rn.f32.f16 %0, a0, b0, %0;\n\t"
      "fma.rn.f32.f16 %0, a1, b1, %0;}"
      : "+f"(acc) : "r"(a), "r"(b));
}
template <> QA_DEVINL void dot_pair<__nv_bfloat16>(float& acc, uint32_t a, uint32_t b) {
  asm("{.reg .b16 a0, a1, b0, b1;\n\t"
      "mov.b32 {a0, a1}, %1;\n\t"
      "mov.b32 {b0, b1}, %2;\n\t"
      "fma.rn.f32.bf16 %0, a0, b0, %0;\n\t"
      "fma.rn.f32.bf16 %0, a1, b1, %0;}"
      : "+f"(acc) : "r"(a), "r"(b));
}

// Packed pair of 16-bit elements -> two fp32 (exact).
template <typename T> QA_DEVINL float2 pair_to_f32(uint32_t w);
template <> QA_DEVINL float2 pair_to_f32<__half>(uint32_t w) {
  return __half22float2(*reinterpret_cast<const __half2*>(&w));
}
template <> QA_DEVINL float2 pair_to_f32<__nv_bfloat16>(uint32_t w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}

// 16-byte asynchronous global->shared copy that bypasses L1 (cp.async.cg).
QA_DEVINL void cp_async16(void* smem, const void* gmem) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}
QA_DEVINL void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// x / d for 0 <= x < 2^31 with a precomputed multiplier (round-up method of
// Granlund & Montgomery, 1994): l = ceil(log2 d), m = floor(2^32 (2^l - d) / d) + 1,
// x / d = (umulhi(x, m) + x) >> l.
struct FastDiv {
  uint32_t m;
  uint32_t l;
};
QA_DEVINL uint32_t fast_div(uint32_t x, FastDiv f) { return (__umulhi(x, f.m) + x) >> f.l; }

// Element offset of sequence `seq`'s first query row: its own batch stride when
// the caller gave one (queries in a [B, N, ...] view whose batch pitch is not
// N token rows), else row cu_seqlens_q[seq] = q0 of the packed token axis.
QA_DEVINL int64_t q_seq_off(const qa_ancestor_args& a, int seq, int q0) {
  return a.q_stride_b != 0 ? int64_t(seq) * a.q_stride_b : int64_t(q0) * a.q_stride_t;
}

QA_DEVINL float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// ---- host-side per-device launch state --------------------------------------
// Kernel attributes (the dynamic shared-memory limit) and device properties are
// per device: a process that launches on several GPUs must set and query them
// on each. These helpers key everything by the current device and are safe to
// call from several host threads at once.
constexpr int kQaMaxDevices = 64;

inline int qa_current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kQaMaxDevices) dev = 0;
  return dev;
}

// Raises `fn`'s dynamic shared-memory limit to at least `bytes` on the current
// device (once per device, kernel and size).
inline cudaError_t qa_smem_attr(const void* fn, int bytes) {
  struct Entry {
    int dev;
    const void* fn;
    int bytes;
  };
  static std::mutex mu;
  static std::vector<Entry> done;
  const int dev = qa_current_device();
  std::lock_guard<std::mutex> lock(mu);
  for (Entry& e : done)
    if (e.dev == dev && e.fn == fn) {
      if (e.bytes >= bytes) return cudaSuccess;
      const cudaError_t r = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
      if (r == cudaSuccess) e.bytes = bytes;
      return r;
    }
  const cudaError_t r = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (r == cudaSuccess) done.push_back({dev, fn, bytes});
  return r;
}

// Streaming multiprocessors of the current device (cached per device).
inline int qa_sm_count() {
  static std::atomic<int> cache[kQaMaxDevices];
  const int dev = qa_current_device();
  int n = cache[dev].load(std::memory_order_relaxed);
  if (n > 0) return n;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
  cache[dev].store(n, std::memory_order_relaxed);
  return n;
}

}  // namespace qa
