// Generic tensor-ring kernel: any spec, fp32 / fp16 / bf16 storage, fp32 arithmetic on CUDA
// cores.  It serves fp32 plans (the reference's CPU checks run in fp32, reference tests
// test_correctness.py:26-46) and shapes the mma.sync kernel does not cover.
//
// One CTA owns one (token t, o1) pair and every (o2, o3) output of it, so no cross-CTA
// reduction, workspace or atomic is needed and the sum order is fixed (deterministic).  It
// walks i3 and chunks of the ring index s:
//   T1[s][i2][u] = sum_i1       x[t,i1,i2,i3] G1[s,o1,i1,u]
//   T2[s][o2][v] = sum_{i2,u}   T1[s][i2][u]  G2[u,o2,i2,v]
//   Y[o2][o3]   += sum_{s,v}    T2[s][o2][v]  G3[v,o3,i3,s]
// which is the chosen order's chain with no redundant work (each S1 value is used for all o2).
#include <cuda_runtime.h>

#include <algorithm>

#include "device_util.cuh"
#include "plan.h"

namespace trr {

struct GenericParams {
  const void* x;
  void* y;
  const void* g1;
  const void* g2;
  const void* g3;
  int I1, I2, I3, O1, O2, O3, R;
  int d_in, d_out;
  long long sx1, sx2, sx3, sy1, sy2, sy3;
  int SC;  // ring indices s per chunk held in shared memory
  Epi epi;  // what is written for each y element
};

template <typename E>
__global__ void __launch_bounds__(256) ring_generic_kernel(GenericParams p) {
  extern __shared__ float gsm[];
  const E* __restrict__ x = static_cast<const E*>(p.x);
  const E* __restrict__ g1 = static_cast<const E*>(p.g1);
  const E* __restrict__ g2 = static_cast<const E*>(p.g2);
  const E* __restrict__ g3 = static_cast<const E*>(p.g3);
  const int t = blockIdx.x / p.O1, o1 = blockIdx.x % p.O1;
  const int R = p.R;
  float* T1 = gsm;                           // [SC][I2][R]
  float* T2 = T1 + (size_t)p.SC * p.I2 * R;  // [SC][O2][R]
  float* Y = T2 + (size_t)p.SC * p.O2 * R;   // [O2][O3]
  const int nY = p.O2 * p.O3;
  for (int e = threadIdx.x; e < nY; e += blockDim.x) Y[e] = 0.f;
  const E* xr = x + (size_t)t * p.d_in;
  for (int i3 = 0; i3 < p.I3; ++i3) {
    for (int s0 = 0; s0 < R; s0 += p.SC) {
      const int sc = min(p.SC, R - s0);
      __syncthreads();  // previous chunk's T1/T2 fully consumed
      const int n1 = sc * p.I2 * R;
      for (int e = threadIdx.x; e < n1; e += blockDim.x) {
        const int u = e % R, i2 = (e / R) % p.I2, sl = e / (R * p.I2);
        const E* gp = g1 + ((size_t)(s0 + sl) * p.O1 + o1) * p.I1 * R + u;
        const E* xp = xr + i2 * p.sx2 + i3 * p.sx3;
        float acc = 0.f;
        for (int i1 = 0; i1 < p.I1; ++i1)
          acc = fmaf(to_f32<E>(xp[i1 * p.sx1]), to_f32<E>(gp[(size_t)i1 * R]), acc);
        T1[e] = acc;
      }
      __syncthreads();
      const int n2 = sc * p.O2 * R;
      for (int e = threadIdx.x; e < n2; e += blockDim.x) {
        const int v = e % R, o2 = (e / R) % p.O2, sl = e / (R * p.O2);
        const float* tp = T1 + (size_t)sl * p.I2 * R;
        float acc = 0.f;
        for (int u = 0; u < R; ++u) {
          const E* gp = g2 + (((size_t)u * p.O2 + o2) * p.I2) * R + v;
          for (int i2 = 0; i2 < p.I2; ++i2)
            acc = fmaf(tp[i2 * R + u], to_f32<E>(gp[(size_t)i2 * R]), acc);
        }
        T2[e] = acc;
      }
      __syncthreads();
      for (int e = threadIdx.x; e < nY; e += blockDim.x) {
        const int o3 = e % p.O3, o2 = e / p.O3;
        float acc = Y[e];
        for (int sl = 0; sl < sc; ++sl) {
          const float* tp = T2 + ((size_t)sl * p.O2 + o2) * R;
          for (int v = 0; v < R; ++v)
            acc = fmaf(tp[v],
                       to_f32<E>(g3[(((size_t)v * p.O3 + o3) * p.I3 + i3) * R + s0 + sl]), acc);
        }
        Y[e] = acc;
      }
    }
  }
  __syncthreads();
  const size_t yr = (size_t)t * p.d_out + (size_t)o1 * p.sy1;
  for (int e = threadIdx.x; e < nY; e += blockDim.x) {
    const int o3 = e % p.O3, o2 = e / p.O3;
    epi_store<E>(p.epi, p.y, yr + (size_t)o2 * p.sy2 + (size_t)o3 * p.sy3, Y[e]);
  }
}

int launch_generic(const Plan& p, const void* packed, const void* x, int64_t T, void* y,
                   void* stream, const Epi& epi) {
  const Canon& c = p.c;
  if (p.mma_ok) {
    set_error("fp16/bf16 plans pack the mma layout; the generic kernel needs an fp32 plan or "
              "a shape the mma kernel does not cover");
    return TR_ERR_UNSUPPORTED;
  }
  if (T * (int64_t)c.O1 > 0x7fffffffLL) {
    set_error("too many tokens for one launch");
    return TR_ERR_UNSUPPORTED;
  }
  const size_t budget = 96 * 1024;
  const size_t fixed = (size_t)c.O2 * c.O3 * 4;
  const size_t per_s = ((size_t)c.I2 * c.R + (size_t)c.O2 * c.R) * 4;
  if (fixed + per_s > budget) {
    set_error("spec too large for the generic kernel's shared memory");
    return TR_ERR_UNSUPPORTED;
  }
  const int SC = (int)std::min<size_t>((size_t)c.R, (budget - fixed) / per_s);
  const size_t smem = fixed + per_s * SC;
  const char* base = static_cast<const char*>(packed);
  GenericParams gp;
  gp.x = x;
  gp.y = y;
  gp.epi = epi;
  gp.g1 = base + p.g.off_g1;
  gp.g2 = base + p.g.off_g2;
  gp.g3 = base + p.g.off_g3;
  gp.I1 = c.I1; gp.I2 = c.I2; gp.I3 = c.I3;
  gp.O1 = c.O1; gp.O2 = c.O2; gp.O3 = c.O3;
  gp.R = c.R;
  gp.d_in = c.d_in;
  gp.d_out = c.d_out;
  gp.sx1 = c.sx1; gp.sx2 = c.sx2; gp.sx3 = c.sx3;
  gp.sy1 = c.sy1; gp.sy2 = c.sy2; gp.sy3 = c.sy3;
  gp.SC = SC;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 grid((unsigned)(T * c.O1));
  cudaError_t e = cudaSuccess;
  switch (p.dtype) {
    case TR_F32:
      e = cudaFuncSetAttribute(ring_generic_kernel<float>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e == cudaSuccess) ring_generic_kernel<float><<<grid, 256, smem, st>>>(gp);
      break;
    case TR_F16:
      e = cudaFuncSetAttribute(ring_generic_kernel<__half>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e == cudaSuccess) ring_generic_kernel<__half><<<grid, 256, smem, st>>>(gp);
      break;
    case TR_BF16:
      e = cudaFuncSetAttribute(ring_generic_kernel<__nv_bfloat16>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e == cudaSuccess) ring_generic_kernel<__nv_bfloat16><<<grid, 256, smem, st>>>(gp);
      break;
  }
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("generic kernel launch: %s", cudaGetErrorString(e));
    return TR_ERR_CUDA;
  }
  return TR_OK;
}

}  // namespace trr
