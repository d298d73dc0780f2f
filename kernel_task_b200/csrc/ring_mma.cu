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
  int flag_off;
};

__device__ __forceinline__ int sel3(int k, int a, int b, int c) {
  return k == 0 ? a : (k == 1 ? b : c);
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
  const int t0 = tile * p.TT;
  const int TTv = min(p.TT, p.T - t0);
  const int i3a = pa / p.R;
  const int i3b = pb > pa ? (pb - 1) / p.R + 1 : i3a;

  const int XSTR = p.K1P + 8;   // +16 B per row: ldmatrix rows fall in distinct banks
  const int M1P = p.MT1 * 16;
  const int T1STR = p.K2P + 8;
  const int M2P = p.MT2 * 16;
  const size_t xs_bytes = ((size_t)p.NI3L * M1P * XSTR * 2 + 127) / 128 * 128;
  const size_t t1_bytes = (size_t)2 * M2P * T1STR * 2;
  E* xs = reinterpret_cast<E*>(smem);
  __half* t1s = reinterpret_cast<__half*>(smem + xs_bytes);
  float* ys = reinterpret_cast<float*>(smem);  // reused after the piece loop
  int* flag = reinterpret_cast<int*>(smem + p.flag_off);

  // ---- clear the x tile and both T1 buffers (padding rows/columns must read as zero)
  {
    uint4* z = reinterpret_cast<uint4*>(smem);
    const int n16 = (int)((xs_bytes + t1_bytes) / 16);
    for (int e = tid; e < n16; e += nthr) z[e] = make_uint4(0u, 0u, 0u, 0u);
  }
  __syncthreads();
  // ---- x tile: read rows in memory order (coalesced), scatter to xs[i3][(t,i2)][i1]
  {
    const E* x = static_cast<const E*>(p.x) + (size_t)t0 * p.d_in;
    const int n = TTv * p.d_in;
    for (int e = tid; e < n; e += nthr) {
      const int t = e / p.d_in, f = e - t * p.d_in;
      const int m2 = f % p.xm2, q = f / p.xm2;
      const int m1 = q % p.xm1, m0 = q / p.xm1;
      const int i3 = sel3(p.role2, m0, m1, m2);
      if (i3 < i3a || i3 >= i3b) continue;
      const int i1 = sel3(p.role0, m0, m1, m2);
      const int i2 = sel3(p.role1, m0, m1, m2);
      xs[((size_t)(i3 - i3a) * M1P + t * p.I2 + i2) * XSTR + i1] = x[e];
    }
  }
  __syncthreads();

  const int o2 = warp;  // one o2 per warp (nwarps == O2)
  float yacc[MTW][4][4];
#pragma unroll
  for (int a = 0; a < MTW; ++a)
#pragma unroll
    for (int b = 0; b < 4; ++b)
#pragma unroll
      for (int c = 0; c < 4; ++c) yacc[a][b][c] = 0.f;

  const uint2* g2w = p.g2f + (size_t)o2 * NV * 32 + lane;
  const int s1rows = TTv * p.I2;
  const int njobs1 = p.MT1 * p.NT1;

  for (int pi = pa; pi < pb; ++pi) {
    const int i3 = pi / p.R, s = pi - i3 * p.R;
    const int buf = (pi - pa) & 1;
    const E* xt = xs + (size_t)(i3 - i3a) * M1P * XSTR;
    __half* t1 = t1s + (size_t)buf * M2P * T1STR;

    // ---- S1: D1[(t,i2),(o1,u)] = x_i3 . G1_s, written as T1[(t,o1)][(i2,u)] (fp16)
    const uint2* g1p = p.g1f + (size_t)s * p.KS1 * p.NT1 * 32 + lane;
    for (int job = warp; job < njobs1; job += nwarps) {
      const int mt1 = job / p.NT1, nt1 = job - mt1 * p.NT1;
      float d[4] = {0.f, 0.f, 0.f, 0.f};
      for (int ks = 0; ks < p.KS1; ++ks) {
        uint32_t a[4];
        ldsm_x4(a, xt + (size_t)(mt1 * 16 + (lane & 15)) * XSTR + ks * 16 + (lane >> 4) * 8);
        const uint2 b = __ldg(g1p + (size_t)(ks * p.NT1 + nt1) * 32);
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
    __syncthreads();  // T1[buf] complete; the other buffer is free for the next piece

    if (o2 < p.O2) {
      // G3 fragments of this piece (K = v, N = o3)
      const uint2* g3p = p.g3f + (size_t)pi * KS3 * p.NT3 * 32 + lane;
      uint2 b3[KS3][4];
#pragma unroll
      for (int k = 0; k < KS3; ++k)
#pragma unroll
        for (int n = 0; n < 4; ++n)
          b3[k][n] = n < p.NT3 ? __ldg(g3p + (size_t)(k * p.NT3 + n) * 32) : make_uint2(0u, 0u);

      // ---- S2: D2[(t,o1),(o2,v)] for this warp's o2, all row tiles
      float d2[MTW][NV][4];
#pragma unroll
      for (int a = 0; a < MTW; ++a)
#pragma unroll
        for (int b = 0; b < NV; ++b)
#pragma unroll
          for (int c = 0; c < 4; ++c) d2[a][b][c] = 0.f;
      for (int ks2 = 0; ks2 < p.KS2; ++ks2) {
        uint2 b[NV];
#pragma unroll
        for (int nv = 0; nv < NV; ++nv) b[nv] = __ldg(g2w + ((size_t)ks2 * p.NT2 + nv) * 32);
#pragma unroll
        for (int mi = 0; mi < MTW; ++mi) {
          if (mi < p.MT2) {
            uint32_t a[4];
            ldsm_x4(a, t1 + (size_t)(mi * 16 + (lane & 15)) * T1STR + ks2 * 16 + (lane >> 4) * 8);
#pragma unroll
            for (int nv = 0; nv < NV; ++nv) mma_16816(d2[mi][nv], a, b[nv].x, b[nv].y, __half());
          }
        }
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
  }
  __syncthreads();  // every warp is done with xs / T1: reuse the space for the partial Y

  // ---- partial Y -> ys[(t,o1)][o2*O3P + o3]
  const int YSTR = p.O2 * p.O3P;
  if (o2 < p.O2) {
#pragma unroll
    for (int mi = 0; mi < MTW; ++mi) {
      if (mi < p.MT2) {
#pragma unroll
        for (int n = 0; n < 4; ++n) {
          if (n < p.NT3) {
            const int col = o2 * p.O3P + n * 8 + 2 * t4;
            const int r0 = mi * 16 + g;
            *reinterpret_cast<float2*>(ys + (size_t)r0 * YSTR + col) =
                make_float2(yacc[mi][n][0], yacc[mi][n][1]);
            *reinterpret_cast<float2*>(ys + (size_t)(r0 + 8) * YSTR + col) =
                make_float2(yacc[mi][n][2], yacc[mi][n][3]);
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

  // ---- reduce this CTA's slice of the tile over the cluster, in y memory order
  const int ntot = TTv * p.d_out;
  const int ebeg = (int)((long long)crank * ntot / p.CL);
  const int eend = (int)((long long)(crank + 1) * ntot / p.CL);
  E* y = static_cast<E*>(p.y) + (size_t)t0 * p.d_out;
  float* slot =
      p.NC > 1 ? p.slots + ((size_t)tile * p.NC + cl_id) * (size_t)p.TT * p.d_out : nullptr;
  for (int e = ebeg + tid; e < eend; e += nthr) {
    const int t = e / p.d_out, f = e - t * p.d_out;
    const int m2 = f % p.ym2, q = f / p.ym2;
    const int m1 = q % p.ym1, m0 = q / p.ym1;
    const int oc1 = sel3(p.role0, m0, m1, m2);
    const int oc2 = sel3(p.role1, m0, m1, m2);
    const int oc3 = sel3(p.role2, m0, m1, m2);
    const int idx = (t * p.O1 + oc1) * YSTR + oc2 * p.O3P + oc3;
    float v;
    if (p.CL > 1) {
      v = 0.f;
      for (int r = 0; r < p.CL; ++r) v += cluster.map_shared_rank(ys, r)[idx];
    } else {
      v = ys[idx];
    }
    if (p.NC == 1) {
      y[e] = from_f32<E>(v);
    } else {
      slot[e] = v;
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
    if (*flag) {  // last cluster for this slice: add the NC slots and write y
      __threadfence();
      const float* s0 = p.slots + (size_t)tile * p.NC * (size_t)p.TT * p.d_out;
      const size_t sstride = (size_t)p.TT * p.d_out;
      for (int e = ebeg + tid; e < eend; e += nthr) {
        float v = 0.f;
        for (int c = 0; c < p.NC; ++c) v += __ldcg(s0 + c * sstride + e);
        y[e] = from_f32<E>(v);
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
               void* y, void* ws, void* stream) {
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
