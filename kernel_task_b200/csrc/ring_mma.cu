// Fused tensor-ring kernel on warp-level tensor cores (mma.sync m16n8k16 / m16n8k8), one
// launch per call: S1 -> S2 -> S3 chained on-chip, ring trace and fp16/bf16 cast fused.
//
// Work decomposition (canonical form, see plan.h).  The sum over the ring closes through
// `pieces` (i3, s): for a fixed piece,
//   S1  T1[(t,o1),(i2,u)] = sum_i1 x[t,i1,i2,i3] G1[s,o1,i1,u]          (mma, rows (t,i2))
//   S2  D2[(t,o1),(o2,v)] = sum_(i2,u) T1 G2[u,o2,i2,v]                   (mma, A from smem)
//   S3  Y[(t,o1),(o2,o3)] += sum_v D2 G3[v,o3,i3,s]                       (mma, A = D2 regs)
// and y is the sum of Y over all I3*R pieces.  S3 contracts only v, which is the column index
// of S2's accumulator, so the S2 accumulator fragments are re-packed in registers as S3's A
// operand (m16n8 C layout == m16n8k16 A layout pairwise).  S1's output changes layout
// ((t,i2) rows -> (t,o1) rows), so it goes through shared memory (ldmatrix) once per piece.
//
// Grid: row tiles (TT tokens) x NC clusters x CL CTAs.  Each CTA takes a contiguous range of
// pieces and keeps its partial Y in registers (warp w owns o2 = w and all m16 row tiles).
// Partials are summed over the cluster through distributed shared memory; with NC == 1 the
// cluster writes y directly.  With NC > 1 each cluster stores its sum to a workspace slot and
// the last cluster to arrive on a per-slice counter adds the slots, writes y and resets the
// counter (threadfence reduction).  No spin-waits.
//
// Replaces the reference's V3 / V3T / V3G kernels (csrc/tr_ring.cu:543-751, 822-1056;
// csrc/v3g/v3g.cuh:142-431), which compute S1 on CUDA cores and reduce pieces with global
// float atomics into a zeroed workspace.
#include <cooperative_groups.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>

#include "device_util.cuh"
#include "plan.h"

namespace cg = cooperative_groups;

namespace trr {

struct MmaParams {
  const void* x;
  void* y;
  const uint2* g1f;
  const uint2* g2f;
  const uint2* g3f;
  float* slots;
  int* cnt;
  int T;
  int I1, I2, I3, O1, O2, O3, R;
  int d_in, d_out;
  int xm0, xm1, xm2;     // reference input modes
  int ym0, ym1, ym2;     // reference output modes
  int role0, role1, role2;  // reference mode index of canonical mode 1, 2, 3
  int K1P, KS1, NT1, K2P, KS2, NT2, O3P, NT3, npieces;
  int TT, MT1, MT2, CL, NC, NI3L;
  long long sy1, sy2, sy3;  // y strides of o1, o2, o3
  // shared-memory carve-up (bytes; see mma_smem_layout in plan.cpp)
  int off_t1, t1_stride, off_g2, off_pf, off_xr;
  int g1p_bytes, g3p_bytes;  // fragments of one piece: G1 of its s, then G3 of the piece
  int g2_smem, pf_smem, x_async, g2_bytes;
  int vec4;                 // d_out % 4 == 0: reductions move float4
  int flag_off;
  Epi epi;                  // what is written for each y element
};

__device__ __forceinline__ int sel3(int k, int a, int b, int c) {
  return k == 0 ? a : (k == 1 ? b : c);
}

__device__ __forceinline__ void cp_async16(uint32_t saddr, const void* g) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(saddr), "l"(g) : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;\n" ::: "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_group 0;\n" ::: "memory");
}
// All threads of the CTA copy `bytes` (multiple of 16) global -> shared, asynchronously.
__device__ __forceinline__ void copy_async(unsigned char* dst, const void* src, int bytes,
                                           int tid, int nthr) {
  const uint32_t s = (uint32_t)__cvta_generic_to_shared(dst);
  const char* g = static_cast<const char*>(src);
  for (int i = tid * 16; i < bytes; i += nthr * 16) cp_async16(s + i, g + i);
}

// S2 for one warp: D2[mi][nv] += T1[rows of tile mi] . G2[:, o2 block], G2 fragments from
// shared memory (SM) or global memory (!SM).
template <int NV, int MTW, bool SM>
__device__ __forceinline__ void s2_accumulate(float (&d2)[MTW][NV][4], const __half* t1, int T1STR,
                                              const uint2* g2w, int KS2, int NT2, int MT2,
                                              int lane) {
  for (int ks2 = 0; ks2 < KS2; ++ks2) {
    uint2 b[NV];
#pragma unroll
    for (int nv = 0; nv < NV; ++nv) {
      const uint2* src = g2w + ((size_t)ks2 * NT2 + nv) * 32;
      b[nv] = SM ? *src : __ldg(src);
    }
#pragma unroll
    for (int mi = 0; mi < MTW; ++mi) {
      if (mi < MT2) {
        uint32_t a[4];
        ldsm_x4(a, t1 + (size_t)(mi * 16 + (lane & 15)) * T1STR + ks2 * 16 + (lane >> 4) * 8);
#pragma unroll
        for (int nv = 0; nv < NV; ++nv) mma_16816(d2[mi][nv], a, b[nv].x, b[nv].y, __half());
      }
    }
  }
}

template <typename E, int RP, int MTW, int MAXT>
__global__ void __launch_bounds__(MAXT, 1) ring_mma_kernel(const MmaParams p) {
  constexpr int NV = RP / 8;                 // n8 tiles of one o2 in S2
  constexpr int KS3 = RP >= 16 ? RP / 16 : 1;
  extern __shared__ __align__(128) unsigned char smem[];
  const int tid = threadIdx.x, nthr = blockDim.x;
  const int warp = tid >> 5, lane = tid & 31, nwarps = nthr >> 5;
  const int g = lane >> 2, t4 = lane & 3;

  const int NJ = p.CL * p.NC;
  const int tile = blockIdx.x / NJ;
  const int jj = blockIdx.x - tile * NJ;
  const int crank = jj % p.CL;
  const int cl_id = jj / p.CL;
  const int pa = (int)((long long)jj * p.npieces / NJ);
  const int pb = (int)((long long)(jj + 1) * p.npieces / NJ);
  const int np = pb - pa;
  const int t0 = tile * p.TT;
  const int TTv = min(p.TT, p.T - t0);
  const int i3a = pa / p.R;
  const int i3b = np > 0 ? (pb - 1) / p.R + 1 : i3a;

  const int XSTR = p.K1P + 8;   // +16 B per row: ldmatrix rows fall in distinct banks
  const int M1P = p.MT1 * 16;
  const int T1STR = p.K2P + 8;
  const int pf_stride = p.g1p_bytes + p.g3p_bytes;
  E* xs = reinterpret_cast<E*>(smem);
  float* ys = reinterpret_cast<float*>(smem);  // [t][d_out] partial y, after the piece loop
  int* flag = reinterpret_cast<int*>(smem + p.flag_off);
  const E* xg = static_cast<const E*>(p.x) + (size_t)t0 * p.d_in;

  // ---- prologue: one burst of async copies (G2, every piece's G1/G3 fragments, x rows)
  if (p.g2_smem) copy_async(smem + p.off_g2, p.g2f, p.g2_bytes, tid, nthr);
  if (p.pf_smem) {
    for (int j = 0; j < np; ++j) {
      const int pi = pa + j;
      unsigned char* dst = smem + p.off_pf + j * pf_stride;
      copy_async(dst, p.g1f + (size_t)(pi % p.R) * p.KS1 * p.NT1 * 32, p.g1p_bytes, tid, nthr);
      copy_async(dst + p.g1p_bytes, p.g3f + (size_t)pi * KS3 * p.NT3 * 32, p.g3p_bytes, tid,
                 nthr);
    }
  }
  if (p.x_async) copy_async(smem + p.off_xr, xg, TTv * p.d_in * (int)sizeof(E), tid, nthr);
  cp_async_commit();
  {  // clear the x tile and both T1 buffers: padding rows/columns must read as zero
    uint4* z = reinterpret_cast<uint4*>(smem);
    const int n16 = (p.off_t1 + 2 * p.t1_stride) / 16;
    for (int e = tid; e < n16; e += nthr) z[e] = make_uint4(0u, 0u, 0u, 0u);
  }
  __syncthreads();
  {  // x rows -> xs[i3][(t,i2)][i1]
    const E* xsrc = p.x_async ? reinterpret_cast<const E*>(smem + p.off_xr) : xg;
    if (p.x_async) cp_async_wait_all();
    if (p.x_async) __syncthreads();
    const int n = TTv * p.d_in;
    for (int e = tid; e < n; e += nthr) {
      const int t = e / p.d_in, f = e - t * p.d_in;
      const int m2 = f % p.xm2, q = f / p.xm2;
      const int m1 = q % p.xm1, m0 = q / p.xm1;
      const int i3 = sel3(p.role2, m0, m1, m2);
      if (i3 < i3a || i3 >= i3b) continue;
      const int i1 = sel3(p.role0, m0, m1, m2);
      const int i2 = sel3(p.role1, m0, m1, m2);
      xs[((size_t)(i3 - i3a) * M1P + t * p.I2 + i2) * XSTR + i1] = xsrc[e];
    }
  }
  cp_async_wait_all();
  __syncthreads();

  const int o2 = warp;  // one o2 per warp (nwarps == O2)
  float yacc[MTW][4][4];
#pragma unroll
  for (int a = 0; a < MTW; ++a)
#pragma unroll
    for (int b = 0; b < 4; ++b)
#pragma unroll
      for (int c = 0; c < 4; ++c) yacc[a][b][c] = 0.f;

  const uint2* g2s = reinterpret_cast<const uint2*>(smem + p.off_g2) + (size_t)o2 * NV * 32 + lane;
  const uint2* g2g = p.g2f + (size_t)o2 * NV * 32 + lane;
  const int s1rows = TTv * p.I2;
  const int njobs1 = p.MT1 * p.NT1;

  // S1 of piece j+1 and S2/S3 of piece j share one iteration and one barrier (T1 is
  // double-buffered), so each warp's instruction stream carries both.
  for (int j = 0; j <= np; ++j) {
    if (j < np) {
      // ---- S1: D1[(t,i2),(o1,u)] = x_i3 . G1_s, written as T1[(t,o1)][(i2,u)] (fp16)
      const int pi = pa + j;
      const int i3 = pi / p.R;
      const uint2* g1p = p.pf_smem
          ? reinterpret_cast<const uint2*>(smem + p.off_pf + j * pf_stride) + lane
          : p.g1f + (size_t)(pi % p.R) * p.KS1 * p.NT1 * 32 + lane;
      const E* xt = xs + (size_t)(i3 - i3a) * M1P * XSTR;
      __half* t1 = reinterpret_cast<__half*>(smem + p.off_t1 + (j & 1) * p.t1_stride);
      for (int job = warp; job < njobs1; job += nwarps) {
        const int mt1 = job / p.NT1, nt1 = job - mt1 * p.NT1;
        float d[4] = {0.f, 0.f, 0.f, 0.f};
        for (int ks = 0; ks < p.KS1; ++ks) {
          uint32_t a[4];
          ldsm_x4(a, xt + (size_t)(mt1 * 16 + (lane & 15)) * XSTR + ks * 16 + (lane >> 4) * 8);
          const uint2* src = g1p + (size_t)(ks * p.NT1 + nt1) * 32;
          const uint2 b = p.pf_smem ? *src : __ldg(src);
          mma_16816(d, a, b.x, b.y, E());
        }
        const int col = nt1 * 8 + 2 * t4;
        const int o1 = col / RP, u = col % RP;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int r = mt1 * 16 + g + 8 * h;
          if (r < s1rows) {
            const int t = r / p.I2, i2 = r - t * p.I2;
            *reinterpret_cast<__half2*>(t1 + (size_t)(t * p.O1 + o1) * T1STR + i2 * RP + u) =
                __floats2half2_rn(d[2 * h], d[2 * h + 1]);
          }
        }
      }
    }
    if (j > 0 && o2 < p.O2) {
      const int jp = j - 1;
      const int pi = pa + jp;
      const __half* t1 =
          reinterpret_cast<const __half*>(smem + p.off_t1 + (jp & 1) * p.t1_stride);
      const uint2* g3p = p.pf_smem
          ? reinterpret_cast<const uint2*>(smem + p.off_pf + jp * pf_stride + p.g1p_bytes) + lane
          : p.g3f + (size_t)pi * KS3 * p.NT3 * 32 + lane;
      uint2 b3[KS3][4];
#pragma unroll
      for (int k = 0; k < KS3; ++k)
#pragma unroll
        for (int n = 0; n < 4; ++n) {
          const uint2* src = g3p + (size_t)(k * p.NT3 + n) * 32;
          b3[k][n] = n < p.NT3 ? (p.pf_smem ? *src : __ldg(src)) : make_uint2(0u, 0u);
        }
      // ---- S2: D2[(t,o1),(o2,v)] for this warp's o2, all row tiles
      float d2[MTW][NV][4];
#pragma unroll
      for (int a = 0; a < MTW; ++a)
#pragma unroll
        for (int b = 0; b < NV; ++b)
#pragma unroll
          for (int c = 0; c < 4; ++c) d2[a][b][c] = 0.f;
      if (p.g2_smem) {
        s2_accumulate<NV, MTW, true>(d2, t1, T1STR, g2s, p.KS2, p.NT2, p.MT2, lane);
      } else {
        s2_accumulate<NV, MTW, false>(d2, t1, T1STR, g2g, p.KS2, p.NT2, p.MT2, lane);
      }
      // ---- S3: Y[(t,o1),(o2,o3)] += D2 (as A, fp16) . G3_piece
#pragma unroll
      for (int mi = 0; mi < MTW; ++mi) {
        if (mi < p.MT2) {
          if constexpr (RP == 8) {
            const uint32_t a0 = pack2<__half>(d2[mi][0][0], d2[mi][0][1]);
            const uint32_t a1 = pack2<__half>(d2[mi][0][2], d2[mi][0][3]);
#pragma unroll
            for (int n = 0; n < 4; ++n)
              if (n < p.NT3) mma_1688(yacc[mi][n], a0, a1, b3[0][n].x);
          } else {
#pragma unroll
            for (int k = 0; k < KS3; ++k) {
              uint32_t a[4];
              a[0] = pack2<__half>(d2[mi][2 * k][0], d2[mi][2 * k][1]);
              a[1] = pack2<__half>(d2[mi][2 * k][2], d2[mi][2 * k][3]);
              a[2] = pack2<__half>(d2[mi][2 * k + 1][0], d2[mi][2 * k + 1][1]);
              a[3] = pack2<__half>(d2[mi][2 * k + 1][2], d2[mi][2 * k + 1][3]);
#pragma unroll
              for (int n = 0; n < 4; ++n)
                if (n < p.NT3) mma_16816(yacc[mi][n], a, b3[k][n].x, b3[k][n].y, __half());
            }
          }
        }
      }
    }
    __syncthreads();
  }

  // ---- partial Y -> ys[t][y offset]: y memory order, so the reductions below move float4
  if (o2 < p.O2) {
#pragma unroll
    for (int mi = 0; mi < MTW; ++mi) {
      if (mi < p.MT2) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int r = mi * 16 + g + 8 * h;
          const int t = r / p.O1, o1 = r - t * p.O1;
          if (t < TTv) {
            float* row = ys + (size_t)t * p.d_out + o1 * p.sy1 + o2 * p.sy2;
#pragma unroll
            for (int n = 0; n < 4; ++n) {
              const int o3 = n * 8 + 2 * t4;
              if (o3 < p.O3) row[o3 * p.sy3] = yacc[mi][n][2 * h];
              if (o3 + 1 < p.O3) row[(o3 + 1) * p.sy3] = yacc[mi][n][2 * h + 1];
            }
          }
        }
      }
    }
  }
  cg::cluster_group cluster = cg::this_cluster();
  if (p.CL > 1) {
    cluster.sync();
  } else {
    __syncthreads();
  }

  // ---- reduce this CTA's slice of the tile over the cluster (loads from every peer issued
  // together, added in rank order), then write y (NC == 1) or this cluster's workspace slot
  const size_t ybase = (size_t)t0 * p.d_out;
  const size_t sstride = (size_t)p.TT * p.d_out;
  float* slot = p.NC > 1 ? p.slots + ((size_t)tile * p.NC + cl_id) * sstride : nullptr;
  const int vw = p.vec4 ? 4 : 1;
  const int nvec = TTv * p.d_out / vw;
  const int vbeg = (int)((long long)crank * nvec / p.CL);
  const int vend = (int)((long long)(crank + 1) * nvec / p.CL);
  const float* peer[16];
#pragma unroll
  for (int r = 0; r < 16; ++r)
    peer[r] = (p.CL > 1 && r < p.CL) ? cluster.map_shared_rank(ys, r) : ys;
  if (p.vec4) {
    for (int i = vbeg + tid; i < vend; i += nthr) {
      float4 v[16];
#pragma unroll
      for (int r = 0; r < 16; ++r)
        v[r] = r < p.CL ? reinterpret_cast<const float4*>(peer[r])[i] : make_float4(0, 0, 0, 0);
      float4 s = v[0];
#pragma unroll
      for (int r = 1; r < 16; ++r) {
        s.x += v[r].x; s.y += v[r].y; s.z += v[r].z; s.w += v[r].w;
      }
      if (p.NC == 1) {
        const float f[4] = {s.x, s.y, s.z, s.w};
        epi_store_vec<E, 4>(p.epi, p.y, ybase + 4 * (size_t)i, f);
      } else {
        reinterpret_cast<float4*>(slot)[i] = s;
      }
    }
  } else {
    for (int i = vbeg + tid; i < vend; i += nthr) {
      float v[16];
#pragma unroll
      for (int r = 0; r < 16; ++r) v[r] = r < p.CL ? peer[r][i] : 0.f;
      float s = 0.f;
#pragma unroll
      for (int r = 0; r < 16; ++r) s += v[r];
      if (p.NC == 1) {
        epi_store<E>(p.epi, p.y, ybase + i, s);
      } else {
        slot[i] = s;
      }
    }
  }
  if (p.CL > 1) cluster.sync();  // peers finished reading this CTA's shared memory

  if (p.NC > 1) {
    __threadfence();  // this thread's slot stores are visible device-wide
    __syncthreads();
    if (tid == 0) {
      const int old = atomicAdd(p.cnt + tile * p.CL + crank, 1);
      *flag = (old == p.NC - 1);
    }
    __syncthreads();
    if (*flag) {  // last cluster for this slice: add the NC slots in cluster order, write y
      __threadfence();
      const float* s0 = p.slots + (size_t)tile * p.NC * sstride;
      if (p.vec4) {
        for (int i = vbeg + tid; i < vend; i += nthr) {
          float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
          for (int c0 = 0; c0 < p.NC; c0 += 8) {
            float4 v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u)
              v[u] = c0 + u < p.NC
                         ? __ldcg(reinterpret_cast<const float4*>(s0 + (c0 + u) * sstride) + i)
                         : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int u = 0; u < 8; ++u) {
              s.x += v[u].x; s.y += v[u].y; s.z += v[u].z; s.w += v[u].w;
            }
          }
          const float f[4] = {s.x, s.y, s.z, s.w};
          epi_store_vec<E, 4>(p.epi, p.y, ybase + 4 * (size_t)i, f);
        }
      } else {
        for (int i = vbeg + tid; i < vend; i += nthr) {
          float s = 0.f;
          for (int c0 = 0; c0 < p.NC; c0 += 8) {
            float v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u)
              v[u] = c0 + u < p.NC ? __ldcg(s0 + (c0 + u) * sstride + i) : 0.f;
#pragma unroll
            for (int u = 0; u < 8; ++u) s += v[u];
          }
          epi_store<E>(p.epi, p.y, ybase + i, s);
        }
      }
      if (tid == 0) atomicExch(p.cnt + tile * p.CL + crank, 0);
    }
  }
}

__global__ void empty_kernel() {}

// ------------------------------------------------------------------------------------------
template <typename E, int RP, int MTW, int MAXT>
static cudaError_t launch_variant(const MmaParams& mp, const MmaGeom& g, int device,
                                  cudaStream_t st) {
  auto kern = ring_mma_kernel<E, RP, MTW, MAXT>;
  static bool configured[64] = {};
  if (device >= 0 && device < 64 && !configured[device]) {
    int optin = 0;
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, optin);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return e;
    configured[device] = true;
  }
  if (g.NW * 32 > MAXT) return cudaErrorInvalidConfiguration;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(g.ntiles * g.NC * g.CL));
  cfg.blockDim = dim3((unsigned)(g.NW * 32));
  cfg.dynamicSmemBytes = g.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  if (g.CL > 1) {
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)g.CL;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, kern, mp);
}

template <typename E, int RP>
static cudaError_t launch_rp(const MmaParams& mp, const MmaGeom& g, int device, cudaStream_t st) {
  switch (g.MTW) {
    case 1: return launch_variant<E, RP, 1, 1024>(mp, g, device, st);
    case 2: return launch_variant<E, RP, 2, 512>(mp, g, device, st);
    default: return launch_variant<E, RP, 5, 384>(mp, g, device, st);
  }
}

template <typename E>
static cudaError_t launch_e(const Plan& p, const MmaParams& mp, const MmaGeom& g,
                            cudaStream_t st) {
  switch (p.m.RP) {
    case 8: return launch_rp<E, 8>(mp, g, p.device, st);
    case 16: return launch_rp<E, 16>(mp, g, p.device, st);
    default: return launch_rp<E, 32>(mp, g, p.device, st);
  }
}

int mma_max_threads(int MTW) { return MTW <= 1 ? 1024 : (MTW <= 2 ? 512 : 384); }

int launch_mma(const Plan& p, const MmaGeom& g, const void* packed, const void* x, int64_t T,
               void* y, void* ws, void* stream, const Epi& epi) {
  const Canon& c = p.c;
  const MmaLayout& m = p.m;
  if (T > 0x7fffffffLL / std::max(c.d_in, c.d_out)) {
    set_error("too many tokens for one launch");
    return TR_ERR_UNSUPPORTED;
  }
  if (g.NW * 32 > mma_max_threads(g.MTW)) {
    set_error("O2=%d warps exceed the %d threads of the MTW=%d variant", g.NW,
              mma_max_threads(g.MTW), g.MTW);
    return TR_ERR_UNSUPPORTED;
  }
  const char* base = static_cast<const char*>(packed);
  MmaParams mp;
  mp.x = x;
  mp.y = y;
  mp.epi = epi;
  mp.g1f = reinterpret_cast<const uint2*>(base + m.off_g1);
  mp.g2f = reinterpret_cast<const uint2*>(base + m.off_g2);
  mp.g3f = reinterpret_cast<const uint2*>(base + m.off_g3);
  if (g.NC > 1) {
    const size_t counters = ((size_t)g.ntiles * g.CL * sizeof(int) + 255) / 256 * 256;
    mp.cnt = static_cast<int*>(ws);
    mp.slots = reinterpret_cast<float*>(static_cast<char*>(ws) + counters);
  } else {
    mp.cnt = nullptr;
    mp.slots = nullptr;
  }
  mp.T = (int)T;
  mp.I1 = c.I1; mp.I2 = c.I2; mp.I3 = c.I3;
  mp.O1 = c.O1; mp.O2 = c.O2; mp.O3 = c.O3;
  mp.R = c.R;
  mp.d_in = c.d_in;
  mp.d_out = c.d_out;
  mp.xm0 = p.spec.input_modes[0]; mp.xm1 = p.spec.input_modes[1]; mp.xm2 = p.spec.input_modes[2];
  mp.ym0 = p.spec.output_modes[0]; mp.ym1 = p.spec.output_modes[1]; mp.ym2 = p.spec.output_modes[2];
  mp.role0 = c.role[0]; mp.role1 = c.role[1]; mp.role2 = c.role[2];
  mp.K1P = m.K1P; mp.KS1 = m.KS1; mp.NT1 = m.NT1;
  mp.K2P = m.K2P; mp.KS2 = m.KS2; mp.NT2 = m.NT2;
  mp.O3P = m.O3P; mp.NT3 = m.NT3; mp.npieces = m.npieces;
  mp.TT = g.TT; mp.MT1 = g.MT1; mp.MT2 = g.MT2;
  mp.CL = g.CL; mp.NC = g.NC; mp.NI3L = g.NI3L;
  mp.sy1 = c.sy1; mp.sy2 = c.sy2; mp.sy3 = c.sy3;
  mp.off_t1 = (int)g.off_t1;
  mp.t1_stride = (int)g.t1_stride;
  mp.off_g2 = (int)g.off_g2;
  mp.off_pf = (int)g.off_pf;
  mp.off_xr = (int)g.off_xr;
  mp.g1p_bytes = (int)(m.KS1 * m.NT1 * 256);
  mp.g3p_bytes = (int)(m.KS3 * m.NT3 * 256);
  mp.g2_smem = g.g2_smem;
  mp.pf_smem = g.pf_smem;
  mp.x_async = g.x_async;
  mp.g2_bytes = (int)m.bytes_g2;
  mp.vec4 = (c.d_out % 4 == 0) ? 1 : 0;
  mp.flag_off = (int)(g.smem - 128);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (p.dtype == TR_F16) {
    e = launch_e<__half>(p, mp, g, st);
  } else {
    e = launch_e<__nv_bfloat16>(p, mp, g, st);
  }
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_error("mma kernel launch (tiles=%d CL=%d NC=%d smem=%zu): %s", g.ntiles, g.CL, g.NC,
              g.smem, cudaGetErrorString(e));
    return TR_ERR_CUDA;
  }
  return TR_OK;
}

int query_max_active_clusters(const Plan& p, const MmaGeom& g, int* n) {
  (void)p;
  (void)g;
  *n = -1;
  return TR_OK;
}

// ------------------------------------------------------------------------------------------
// Scratch for tr_forward_noalloc: a fixed array in the module image, so that entry point never
// asks the allocator for memory.  Every GPU that loads this library holds kNoAllocScratchBytes
// for it until the process exits.
constexpr size_t kNoAllocScratchBytes = TR_NOALLOC_SCRATCH_BYTES;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// The array's device address on `device` (the current device).  Host code cannot use the
// symbol itself: on the host it names a stand-in object, not device memory.  Looked up once
// per device, on that device's first no-alloc call.
static int noalloc_scratch(int device, void** out) {
  static std::mutex mu;
  static void* addr[64] = {};
  if (device < 0 || device >= 64) {
    set_error("device ordinal %d out of range", device);
    return TR_ERR_INVALID;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[device]) {
    void* ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess || !ptr) {
      cudaGetLastError();
      set_error("cudaGetSymbolAddress(scratch): %s", cudaGetErrorString(e));
      return TR_ERR_CUDA;
    }
    addr[device] = ptr;
  }
  *out = addr[device];
  return TR_OK;
}

int forward_noalloc(const Plan& p, const void* packed, const void* x, int64_t T, void* y,
                    void* stream) {
  if (T == 0) return TR_OK;
  MmaGeom g;
  int st = resolve_mma_geom(p, T, nullptr, &g);
  if (st != TR_OK) return st;
  if (g.ws_bytes > kNoAllocScratchBytes) {
    set_error("%lld tokens need %zu bytes of scratch; the no-alloc entry point has %zu "
              "(use tr_forward with a caller workspace)",
              (long long)T, g.ws_bytes, kNoAllocScratchBytes);
    return TR_ERR_WORKSPACE;
  }
  int cur = -1;
  if (cudaGetDevice(&cur) != cudaSuccess || cur != p.device) {
    cudaGetLastError();
    set_error("current device %d is not the plan's device %d", cur, p.device);
    return TR_ERR_INVALID;
  }
  void* scratch = nullptr;
  st = noalloc_scratch(p.device, &scratch);
  if (st != TR_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (g.ws_bytes > 0) {
    // the arrival counters must read zero when the kernel starts
    const size_t counters = ((size_t)g.ntiles * g.CL * sizeof(int) + 255) / 256 * 256;
    const cudaError_t e = cudaMemsetAsync(scratch, 0, counters, s);
    if (e != cudaSuccess) {
      set_error("cudaMemsetAsync(scratch counters): %s", cudaGetErrorString(e));
      return TR_ERR_CUDA;
    }
  }
  return launch_mma(p, g, packed, x, T, y, scratch, stream, Epi{0, 0, 0, nullptr});
}

}  // namespace trr

extern "C" int tr_empty_launch(void* stream) {
  trr::empty_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>();
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    trr::set_error("empty launch: %s", cudaGetErrorString(e));
    return TR_ERR_CUDA;
  }
  return TR_OK;
}
