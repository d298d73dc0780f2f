// Small device helpers shared by the kernels: element conversion, ldmatrix and the legacy
// warp-level mma.sync shapes used by ring_mma.cu.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>

namespace trr {

template <typename E>
__device__ __forceinline__ float to_f32(E v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}

template <typename E>
__device__ __forceinline__ E from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

// two floats -> packed 16-bit pair (low half = first argument)
template <typename E>
__device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
// packed 16-bit pair -> two floats (x = low half)
template <typename E>
__device__ __forceinline__ float2 unpack2(uint32_t w);
template <>
__device__ __forceinline__ float2 unpack2<__half>(uint32_t w) {
  return __half22float2(*reinterpret_cast<const __half2*>(&w));
}
template <>
__device__ __forceinline__ float2 unpack2<__nv_bfloat16>(uint32_t w) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w));
}

// ---- programmatic dependent launch: the kernels are launched so that they may start while
// the previous kernel of the stream finishes.  pdl_wait() blocks until that kernel completed
// and its memory is visible; every global-memory access of a kernel comes after it.
// pdl_trigger() lets the next kernel of the stream start (its own pdl_wait still waits for
// this whole grid).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
}

// Hint: bring the whole 16-byte units inside [p, p + bytes) into L2 (the start is rounded up
// and the end down, so nothing outside the range is touched).  Only a hint: L2 is the point of
// coherence, so it may be issued before griddepcontrol.wait even for data the previous kernel
// is still writing; the loads that follow the wait see the written values.
__device__ __forceinline__ void prefetch_l2(const void* p, size_t bytes) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uintptr_t b = (a + 15) & ~(uintptr_t)15, e = (a + bytes) & ~(uintptr_t)15;
  if (e <= b) return;
  bytes = e - b;
  const char* c = reinterpret_cast<const char*>(b);
  while (bytes > 0) {  // one bulk prefetch covers at most 2^20 - 16 bytes here
    const uint32_t n = (uint32_t)(bytes < ((1u << 20) - 16) ? bytes : ((1u << 20) - 16));
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;\n" ::"l"(c), "r"(n) : "memory");
    c += n;
    bytes -= n;
  }
}

// ---- output epilogue (struct Epi, plan.h): the value written for y[i], and the store
template <typename E, class EP>
__device__ __forceinline__ float epi_value(const EP& ep, size_t i, float v) {
  if (ep.kind == 0) return v;
  const float a = ep.aux_f32 ? static_cast<const float*>(ep.aux)[i]
                             : to_f32<E>(static_cast<const E*>(ep.aux)[i]);
  if (ep.kind == 1) return a + v;
  return a / (1.f + __expf(-a)) * v;  // silu(a) * v
}
template <typename E, class EP>
__device__ __forceinline__ void epi_store(const EP& ep, void* y, size_t i, float v) {
  const float r = epi_value<E>(ep, i, v);
  if (ep.out_f32) static_cast<float*>(y)[i] = r;
  else static_cast<E*>(y)[i] = from_f32<E>(r);
}
// N consecutive elements y[i .. i + N - 1] (N = 4 or 8; 8-byte or 16-byte aligned in E, twice
// that in fp32)
template <typename E, int N, class EP>
__device__ __forceinline__ void epi_store_vec(const EP& ep, void* y, size_t i, const float* f) {
  float r[N];
#pragma unroll
  for (int k = 0; k < N; ++k) r[k] = epi_value<E>(ep, i + k, f[k]);
  if (ep.out_f32) {
    float4* d = reinterpret_cast<float4*>(static_cast<float*>(y) + i);
#pragma unroll
    for (int k = 0; k < N / 4; ++k) d[k] = make_float4(r[4 * k], r[4 * k + 1], r[4 * k + 2], r[4 * k + 3]);
  } else if constexpr (N == 8) {
    uint4 o;
    o.x = pack2<E>(r[0], r[1]);
    o.y = pack2<E>(r[2], r[3]);
    o.z = pack2<E>(r[4], r[5]);
    o.w = pack2<E>(r[6], r[7]);
    *reinterpret_cast<uint4*>(static_cast<E*>(y) + i) = o;
  } else {
    uint2 o;
    o.x = pack2<E>(r[0], r[1]);
    o.y = pack2<E>(r[2], r[3]);
    *reinterpret_cast<uint2*>(static_cast<E*>(y) + i) = o;
  }
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  const uint32_t a = (uint32_t)__cvta_generic_to_shared(p);
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(a));
}

// D(16x8,f32) += A(16x16) * B(16x8); A, B fp16
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                          uint32_t b1, __half) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// same, bf16 operands
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                          uint32_t b1, __nv_bfloat16) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// D(16x8,f32) += A(16x8) * B(8x8); fp16
__device__ __forceinline__ void mma_1688(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5}, {%6}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(b0));
}

}  // namespace trr
