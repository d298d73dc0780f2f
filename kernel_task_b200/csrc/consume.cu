// Stand-alone consumers of fp32 forward outputs: the reference's consume_silu_mul and
// consume_add (factorized_inference/csrc/v3g/bind.cu:93-148), kept for callers that run the
// unfused order (fp32 forward, then a separate elementwise launch).  The fused form is an
// epilogue of the forward kernel itself (tr_forward_epilogue).
//
// Memory-bound: per element 8 bytes read and 8 bytes cleared (silu_mul) or 6 read + 4 cleared
// (add), plus 2 bytes written.  Each thread moves 16-byte vectors; the grid is a multiple of
// the SM count, striding over the array.
#include <cuda_runtime.h>

#include <algorithm>

#include "device_util.cuh"
#include "plan.h"

namespace trr {

template <typename E>
__global__ void __launch_bounds__(256) consume_silu_mul_kernel(float4* __restrict__ g,
                                                               float4* __restrict__ u,
                                                               uint2* __restrict__ out,
                                                               int64_t n4) {
  const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float4 a = __ldcs(g + i), b = __ldcs(u + i);
    __stcs(g + i, z);
    __stcs(u + i, z);
    uint2 o;
    o.x = pack2<E>(a.x / (1.f + __expf(-a.x)) * b.x, a.y / (1.f + __expf(-a.y)) * b.y);
    o.y = pack2<E>(a.z / (1.f + __expf(-a.z)) * b.z, a.w / (1.f + __expf(-a.w)) * b.w);
    out[i] = o;
  }
}

template <typename E>
__global__ void __launch_bounds__(256) consume_add_kernel(const uint2* __restrict__ h,
                                                          float4* __restrict__ y,
                                                          uint2* __restrict__ out, int64_t n4) {
  const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float4 v = __ldcs(y + i);
    const uint2 hv = h[i];
    __stcs(y + i, z);
    const float2 h0 = unpack2<E>(hv.x), h1 = unpack2<E>(hv.y);
    uint2 o;
    o.x = pack2<E>(h0.x + v.x, h0.y + v.y);
    o.y = pack2<E>(h1.x + v.z, h1.y + v.w);
    out[i] = o;
  }
}

static int consume_grid(int64_t n4) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t blocks = (n4 + 255) / 256;
  return (int)std::max<int64_t>(1, std::min<int64_t>(blocks, (int64_t)sms * 8));
}

static int consume_check(const void* a, const void* b, const void* out, int32_t out_dtype,
                         int64_t n, const char* what) {
  if (out_dtype != TR_F16 && out_dtype != TR_BF16) {
    set_error("%s: output dtype must be TR_F16 or TR_BF16, got %d", what, (int)out_dtype);
    return TR_ERR_INVALID;
  }
  if (n < 0 || n % 4 != 0) {
    set_error("%s: element count %lld must be a non-negative multiple of 4", what, (long long)n);
    return TR_ERR_INVALID;
  }
  if (n > 0 && (!a || !b || !out)) {
    set_error("%s: null pointer", what);
    return TR_ERR_INVALID;
  }
  if (((uintptr_t)a | (uintptr_t)b | (uintptr_t)out) & 15) {
    set_error("%s: pointers must be 16-byte aligned", what);
    return TR_ERR_ALIGN;
  }
  return TR_OK;
}

static int consume_launched(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s launch: %s", what, cudaGetErrorString(e));
    return TR_ERR_CUDA;
  }
  return TR_OK;
}

}  // namespace trr

using namespace trr;

extern "C" int tr_consume_silu_mul(float* g, float* u, void* out, int32_t out_dtype, int64_t n,
                                   void* stream) {
  const int st = consume_check(g, u, out, out_dtype, n, "tr_consume_silu_mul");
  if (st != TR_OK || n == 0) return st;
  const int64_t n4 = n / 4;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  float4* g4 = reinterpret_cast<float4*>(g);
  float4* u4 = reinterpret_cast<float4*>(u);
  uint2* o = static_cast<uint2*>(out);
  if (out_dtype == TR_F16)
    consume_silu_mul_kernel<__half><<<consume_grid(n4), 256, 0, s>>>(g4, u4, o, n4);
  else
    consume_silu_mul_kernel<__nv_bfloat16><<<consume_grid(n4), 256, 0, s>>>(g4, u4, o, n4);
  return consume_launched("tr_consume_silu_mul");
}

extern "C" int tr_consume_add(const void* h, float* y, void* out, int32_t out_dtype, int64_t n,
                              void* stream) {
  const int st = consume_check(h, y, out, out_dtype, n, "tr_consume_add");
  if (st != TR_OK || n == 0) return st;
  const int64_t n4 = n / 4;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const uint2* h2 = static_cast<const uint2*>(h);
  float4* y4 = reinterpret_cast<float4*>(y);
  uint2* o = static_cast<uint2*>(out);
  if (out_dtype == TR_F16)
    consume_add_kernel<__half><<<consume_grid(n4), 256, 0, s>>>(h2, y4, o, n4);
  else
    consume_add_kernel<__nv_bfloat16><<<consume_grid(n4), 256, 0, s>>>(h2, y4, o, n4);
  return consume_launched("tr_consume_add");
}
