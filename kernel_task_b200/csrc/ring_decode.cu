// Decode kernel: the fused tensor-ring operator for token counts whose S2 rows (t, o1) fit one
// or two m16 tiles (T * O1 <= 32: T = 1 for every benchmark shape, T = 2-3 for small decode
// batches).  One launch, no workspace, no global atomics, deterministic summation order.
//
// Work split (canonical form, plan.h):
//   * a warp owns one ring piece (i3, s) at a time and runs the whole chain for it:
//       S1  D1[(t,i2),(o1,u)] = x_i3 . G1_s          mma, A fragments loaded from x directly
//       T1  D1 -> fp16 -> the warp's own shared tile [(t,o1)][(i2,u)]      (__syncwarp only)
//       S2  D2[(t,o1),(o2,v)] = T1 . G2               mma, A by ldmatrix, B from shared memory
//       S3  Y[(t,o1),(o2,o3)] += D2 . G3_piece        mma, A = D2 re-packed in registers
//   * a thread-block cluster of CL CTAs covers all I3*R pieces for one chunk of O2C output
//     modes o2 (cluster index = o2 chunk).  Warp partials are summed in shared memory, CTA
//     partials across the cluster through distributed shared memory, and the cluster writes its
//     slice of y.  Clusters of different o2 chunks repeat S1 (cheap at decode sizes) instead of
//     reducing through global memory.
//
// Replaces the reference's T = 1 kernel tr_ring_fused_v3_kernel (csrc/tr_ring.cu:543-751),
// which splits pieces over blocks and reduces them with red.global.add into a zeroed
// workspace finished by the last block.
#include <cooperative_groups.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "device_util.cuh"
#include "plan.h"
#include "shapes.cuh"

namespace cg = cooperative_groups;

namespace trr {

template <class S>
struct DecodeParams {
  S sh;            // shape: compile-time (FixedShape) or runtime (DynShape)
  const void* x;
  void* y;
  const uint2* g1f;
  const uint2* g2f;
  const uint2* g3f;
  int T;
  int MT1;         // m16 tiles of S1 rows (t, i2)
  int MT2;         // m16 tiles of S2/S3 rows (t, o1): 1 or 2
  int CL;          // CTAs per cluster (pieces split over them)
  int O2C;         // o2 modes per cluster
  int warp_bytes;  // per-warp shared area: T1 tile, later the warp's partial Y
  int off_warps;   // offset of the per-warp areas (after the staged G2 chunk)
  int off_recv;    // receive slots of the cluster reduction (CL x slice, fp32)
  Epi epi;         // what is written for each y element
};

template <class S, typename E, int RP, int KS1M, int NT1M, int O2CM, int MAXT, int MT2M>
__global__ void __launch_bounds__(MAXT, 1) ring_decode_kernel(const DecodeParams<S> p) {
  const S& sh = p.sh;
  constexpr int NV = RP / 8;
  constexpr int KS3 = RP >= 16 ? RP / 16 : 1;
  extern __shared__ __align__(128) unsigned char smem[];
  const int tid = threadIdx.x, nthr = blockDim.x;
  const int warp = tid >> 5, lane = tid & 31, nwarps = nthr >> 5;
  const int g = lane >> 2, t4 = lane & 3;
  cg::cluster_group cluster = cg::this_cluster();
  const int crank = (int)cluster.block_rank();
  // announce that this CTA runs; the matching wait precedes the first remote store
  asm volatile("barrier.cluster.arrive.relaxed.aligned;\n" ::: "memory");
  // Programmatic dependent launch: the kernel may start while the previous kernel of the stream
  // finishes.  The packed cores (G2 staging, G1/G3 fragments) are read before griddepcontrol.wait
  // (they are written by nothing but tr_pack_cores, which ends with a normally serialized launch);
  // x, y and the epilogue operand only after it.
  bool waited = false;
  const int chunk = blockIdx.x / p.CL;
  const int o2a = chunk * p.O2C;
  const int o2n = min(p.O2C, sh.O2 - o2a);
  const int pa = (int)((long long)crank * sh.npieces / p.CL);
  const int pb = (int)((long long)(crank + 1) * sh.npieces / p.CL);
  const int T1STR = sh.K2P + 8;
  const int YSTR = O2CM * sh.O3P;          // partial Y row: this chunk's (o2, o3)
  const int rows = p.T * sh.O1;            // valid S2 rows (t, o1), <= 16 * MT2M
  const int s1rows = p.T * sh.I2;          // valid S1 rows (t, i2)

  // ---- stage this chunk's G2 fragments: per k-step, O2C*NV contiguous n-tiles
  {
    const int per_ks = o2n * NV * 256;
    const uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
    for (int ks = 0; ks < sh.KS2; ++ks) {
      const char* src = reinterpret_cast<const char*>(p.g2f + ((size_t)ks * sh.NT2 + o2a * NV) * 32);
      for (int i = tid * 16; i < per_ks; i += nthr * 16)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s + ks * per_ks + i),
                     "l"(src + i)
                     : "memory");
    }
    asm volatile("cp.async.commit_group;\n" ::: "memory");
  }
  unsigned char* wbase = smem + p.off_warps + warp * p.warp_bytes;
  __half* t1 = reinterpret_cast<__half*>(wbase);
  float* yw = reinterpret_cast<float*>(wbase);
  {  // clear this warp's T1 tile: padding rows (t,o1) >= rows and columns >= I2*RP stay zero
    uint4* z = reinterpret_cast<uint4*>(wbase);
    for (int i = lane; i < p.warp_bytes / 16; i += 32) z[i] = make_uint4(0u, 0u, 0u, 0u);
  }

  float yacc[MT2M][O2CM][4][4];
#pragma unroll
  for (int m = 0; m < MT2M; ++m)
#pragma unroll
    for (int a = 0; a < O2CM; ++a)
#pragma unroll
      for (int b = 0; b < 4; ++b)
#pragma unroll
        for (int c = 0; c < 4; ++c) yacc[m][a][b][c] = 0.f;

  const E* x = static_cast<const E*>(p.x);
  bool g2_ready = false;
  const int iters = (pb - pa + nwarps - 1) / nwarps;  // same count in every warp
  for (int it = 0; it < iters; ++it) {
    const int pi = pa + warp + it * nwarps;
    const bool active = pi < pb;
    const int i3 = active ? pi / sh.R : 0, s = active ? pi % sh.R : 0;
    // ---- operands of this piece, all loads issued before any use
    uint2 g1[KS1M][NT1M];
#pragma unroll
    for (int k = 0; k < KS1M; ++k)
#pragma unroll
      for (int n = 0; n < NT1M; ++n)
        g1[k][n] = (active && k < sh.KS1 && n < sh.NT1)
                       ? __ldg(p.g1f + (((size_t)s * sh.KS1 + k) * sh.NT1 + n) * 32 + lane)
                       : make_uint2(0u, 0u);
    uint2 b3[KS3][4];
#pragma unroll
    for (int k = 0; k < KS3; ++k)
#pragma unroll
      for (int n = 0; n < 4; ++n)
        b3[k][n] = (active && n < sh.NT3)
                       ? __ldg(p.g3f + (((size_t)pi * KS3 + k) * sh.NT3 + n) * 32 + lane)
                       : make_uint2(0u, 0u);
    if (!waited) {  // first piece: the previous kernel's x is complete and visible from here
      pdl_wait();
      waited = true;
    }
    // x A fragments: rows (t, i2) = 16*mt + g (+8), columns i1 = 16*k + 2*t4 (+1, +8, +9)
    uint32_t xa[2][KS1M][4];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int k = 0; k < KS1M; ++k)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int r = mt * 16 + g + (q & 1) * 8;
          const int c = k * 16 + 2 * t4 + (q >> 1) * 8;
          float lo = 0.f, hi = 0.f;
          if (active && mt < p.MT1 && k < sh.KS1 && r < s1rows) {
            const int t = r / sh.I2, i2 = r - t * sh.I2;
            const E* row = x + (size_t)t * sh.d_in + i2 * sh.sx2 + i3 * sh.sx3;
            if (c < sh.I1) lo = to_f32<E>(row[c * sh.sx1]);
            if (c + 1 < sh.I1) hi = to_f32<E>(row[(c + 1) * sh.sx1]);
          }
          xa[mt][k][q] = pack2<E>(lo, hi);
        }
    __syncwarp();
    // ---- S1 -> T1 (this warp's tile), one n8 column tile at a time
#pragma unroll
    for (int n = 0; n < NT1M; ++n) {
      if (n < sh.NT1) {
        const int col = n * 8 + 2 * t4;
        const int o1 = col / RP, u = col % RP;
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
          if (mt < p.MT1) {
            float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int k = 0; k < KS1M; ++k)
              if (k < sh.KS1) mma_16816(d, xa[mt][k], g1[k][n].x, g1[k][n].y, E());
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int r = mt * 16 + g + 8 * h;
              if (r < s1rows) {
                const int t = r / sh.I2, i2 = r - t * sh.I2;
                *reinterpret_cast<__half2*>(t1 + (size_t)(t * sh.O1 + o1) * T1STR + i2 * RP + u) =
                    __floats2half2_rn(d[2 * h], d[2 * h + 1]);
              }
            }
          }
        }
      }
    }
    __syncwarp();
    if (!g2_ready) {  // the staged G2 chunk: needed from here on, once
      asm volatile("cp.async.wait_group 0;\n" ::: "memory");
      __syncthreads();
      g2_ready = true;
    }
    // ---- S2 and S3 per m16 tile of rows (t, o1); S2's A fragments shared across the o2
#pragma unroll
    for (int mt = 0; mt < MT2M; ++mt) {
      if (mt * 16 >= rows) break;
      float d2[O2CM][NV][4];
#pragma unroll
      for (int a = 0; a < O2CM; ++a)
#pragma unroll
        for (int b = 0; b < NV; ++b)
#pragma unroll
          for (int c = 0; c < 4; ++c) d2[a][b][c] = 0.f;
      const uint2* g2s = reinterpret_cast<const uint2*>(smem) + lane;
      for (int ks = 0; ks < sh.KS2; ++ks) {
        uint32_t a[4];
        ldsm_x4(a, t1 + (size_t)(mt * 16 + (lane & 15)) * T1STR + ks * 16 + (lane >> 4) * 8);
#pragma unroll
        for (int o = 0; o < O2CM; ++o) {
          if (o < o2n) {
#pragma unroll
            for (int nv = 0; nv < NV; ++nv) {
              const uint2 b = g2s[((size_t)ks * o2n * NV + o * NV + nv) * 32];
              mma_16816(d2[o][nv], a, b.x, b.y, __half());
            }
          }
        }
      }
      // ---- S3
#pragma unroll
      for (int o = 0; o < O2CM; ++o) {
        if (o < o2n) {
          if constexpr (RP == 8) {
            const uint32_t a0 = pack2<__half>(d2[o][0][0], d2[o][0][1]);
            const uint32_t a1 = pack2<__half>(d2[o][0][2], d2[o][0][3]);
#pragma unroll
            for (int n = 0; n < 4; ++n)
              if (n < sh.NT3) mma_1688(yacc[mt][o][n], a0, a1, b3[0][n].x);
          } else {
#pragma unroll
            for (int k = 0; k < KS3; ++k) {
              uint32_t a[4];
              a[0] = pack2<__half>(d2[o][2 * k][0], d2[o][2 * k][1]);
              a[1] = pack2<__half>(d2[o][2 * k][2], d2[o][2 * k][3]);
              a[2] = pack2<__half>(d2[o][2 * k + 1][0], d2[o][2 * k + 1][1]);
              a[3] = pack2<__half>(d2[o][2 * k + 1][2], d2[o][2 * k + 1][3]);
#pragma unroll
              for (int n = 0; n < 4; ++n)
                if (n < sh.NT3) mma_16816(yacc[mt][o][n], a, b3[k][n].x, b3[k][n].y, __half());
            }
          }
        }
      }
    }
    __syncwarp();  // T1 fully read before the next piece overwrites it
  }
  if (!waited) pdl_wait();
  if (!g2_ready) {  // warps without pieces still take part in the CTA barrier
    asm volatile("cp.async.wait_group 0;\n" ::: "memory");
    __syncthreads();
  }

  pdl_trigger();  // the next kernel may set up while this one reduces
  // ---- warp partial -> its shared area (rows (t,o1), columns (o2 of chunk, o3))
  __syncwarp();
#pragma unroll
  for (int mt = 0; mt < MT2M; ++mt)
#pragma unroll
    for (int o = 0; o < O2CM; ++o)
#pragma unroll
      for (int n = 0; n < 4; ++n)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int r = mt * 16 + g + 8 * h;
          const int col = o * sh.O3P + n * 8 + 2 * t4;
          if (r < rows && n < sh.NT3)
            *reinterpret_cast<float2*>(yw + (size_t)r * YSTR + col) =
                make_float2(yacc[mt][o][n][2 * h], yacc[mt][o][n][2 * h + 1]);
        }
  __syncthreads();
  // ---- push: sum the warps (fixed order) for each output of the chunk and store the CTA's
  // partial into the owning CTA's receive slot (distributed shared memory).  Output e of the
  // chunk, e = (row, o2, o3) with o3 fastest, belongs to cluster rank e / SL.
  const int nout = rows * o2n * sh.O3;
  const int SL = (nout + p.CL - 1) / p.CL;
  float* recv = reinterpret_cast<float*>(smem + p.off_recv);
  asm volatile("barrier.cluster.wait.aligned;\n" ::: "memory");  // every peer has started
  for (int e = tid; e < nout; e += nthr) {
    const int o3 = e % sh.O3, q = e / sh.O3;
    const int o = q % o2n, r = q / o2n;
    const int idx = r * YSTR + o * sh.O3P + o3;
    // every warp's value in flight at once, then added in warp order
    constexpr int kMaxWarps = MAXT / 32;
    float part[kMaxWarps];
#pragma unroll
    for (int w = 0; w < kMaxWarps; ++w)
      part[w] = w < nwarps
                    ? reinterpret_cast<const float*>(smem + p.off_warps + w * p.warp_bytes)[idx]
                    : 0.f;
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kMaxWarps; ++w)
      if (w < nwarps) v += part[w];
    const int owner = e / SL;
    cluster.map_shared_rank(recv, owner)[crank * SL + (e - owner * SL)] = v;
  }
  cluster.sync();  // all partials have landed in their owners' receive slots
  // ---- own slice: add the CL partials in rank order and write y
  const int ebeg = crank * SL, eend = min(nout, ebeg + SL);
  for (int e = ebeg + tid; e < eend; e += nthr) {
    float rk[16];  // the CL partials in flight at once, added in rank order
#pragma unroll
    for (int k = 0; k < 16; ++k) rk[k] = k < p.CL ? recv[k * SL + (e - ebeg)] : 0.f;
    float sum = 0.f;
#pragma unroll
    for (int k = 0; k < 16; ++k)
      if (k < p.CL) sum += rk[k];
    const int o3 = e % sh.O3, q = e / sh.O3;
    const int o = q % o2n, r = q / o2n;
    const int t = r / sh.O1, o1 = r - t * sh.O1;
    epi_store<E>(p.epi, p.y,
                 (size_t)t * sh.d_out + o1 * sh.sy1 + (o2a + o) * sh.sy2 + o3 * sh.sy3, sum);
  }
}

// ------------------------------------------------------------------------------------------
template <class S, typename E, int RP, int KS1M, int NT1M, int O2CM, int MAXT, int MT2M>
static cudaError_t launch_decode_variant(const DecodeParams<S>& dp, const DecodeGeom& g,
                                         int device, cudaStream_t st) {
  auto kern = ring_decode_kernel<S, E, RP, KS1M, NT1M, O2CM, MAXT, MT2M>;
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
  if (g.NW * 32 > MAXT || g.O2C > O2CM || g.MT2 > MT2M) return cudaErrorInvalidConfiguration;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(g.NOC * g.CL));
  cfg.blockDim = dim3((unsigned)(g.NW * 32));
  cfg.dynamicSmemBytes = g.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)g.CL;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kern, dp);
}

// Variant = (S1 k-steps, S1 n-tiles) capacity: (1,16), (1,32), (2,32).  Threads per CTA and
// o2 modes per cluster the compiled kernels hold, by variant and S2 row tiles (MT2): one row
// tile 512 / 384 / 256 threads with 4 o2; two row tiles (twice the accumulators) 384 / 256 / 256
// threads with 2 / 2 / 1 o2.
int decode_variant(const Plan& p) {
  if (p.m.KS1 > 2 || p.m.NT1 > 32 || p.m.RP > 16) return -1;
  if (p.m.KS1 == 1 && p.m.NT1 <= 16) return 0;
  if (p.m.KS1 == 1) return 1;
  return 2;
}

int decode_max_threads(int variant, int mt2) {
  if (mt2 > 1) return variant == 0 ? 384 : 256;
  return variant == 0 ? 512 : (variant == 1 ? 384 : 256);
}

int decode_max_o2c(int variant, int mt2) { return mt2 > 1 ? (variant == 2 ? 1 : 2) : 4; }

template <class S>
static void fill_common(DecodeParams<S>& dp, const Plan& p, const DecodeGeom& g,
                        const void* packed, const void* x, int64_t T, void* y, const Epi& epi) {
  const char* base = static_cast<const char*>(packed);
  dp.x = x;
  dp.y = y;
  dp.epi = epi;
  dp.g1f = reinterpret_cast<const uint2*>(base + p.m.off_g1);
  dp.g2f = reinterpret_cast<const uint2*>(base + p.m.off_g2);
  dp.g3f = reinterpret_cast<const uint2*>(base + p.m.off_g3);
  dp.T = (int)T;
  dp.MT1 = g.MT1;
  dp.MT2 = g.MT2;
  dp.CL = g.CL;
  dp.O2C = g.O2C;
  dp.warp_bytes = (int)g.warp_bytes;
  dp.off_warps = (int)g.off_warps;
  dp.off_recv = (int)g.off_recv;
}

DynShape dyn_shape(const Plan& p) {
  const Canon& c = p.c;
  const MmaLayout& m = p.m;
  DynShape d;
  d.I1 = c.I1; d.I2 = c.I2; d.I3 = c.I3;
  d.O1 = c.O1; d.O2 = c.O2; d.O3 = c.O3;
  d.R = c.R;
  d.d_in = c.d_in;
  d.d_out = c.d_out;
  d.sx1 = c.sx1; d.sx2 = c.sx2; d.sx3 = c.sx3;
  d.sy1 = c.sy1; d.sy2 = c.sy2; d.sy3 = c.sy3;
  d.KS1 = m.KS1; d.NT1 = m.NT1; d.K2P = m.K2P; d.KS2 = m.KS2; d.NT2 = m.NT2;
  d.O3P = m.O3P; d.NT3 = m.NT3; d.npieces = m.npieces;
  d.xm1 = p.spec.input_modes[1]; d.xm2 = p.spec.input_modes[2];
  d.ym1 = p.spec.output_modes[1]; d.ym2 = p.spec.output_modes[2];
  d.role0 = c.role[0]; d.role1 = c.role[1]; d.role2 = c.role[2];
  return d;
}

template <class S>
static bool shape_matches(const Plan& p) {
  return p.spec.input_modes[0] == S::in0 && p.spec.input_modes[1] == S::in1 &&
         p.spec.input_modes[2] == S::in2 && p.spec.output_modes[0] == S::on0 &&
         p.spec.output_modes[1] == S::on1 && p.spec.output_modes[2] == S::on2 &&
         p.spec.rank == S::R && p.c.role[0] == S::role0 && p.c.role[1] == S::role1;
}

template <class S, typename E>
static cudaError_t launch_decode_fixed(const Plan& p, const DecodeGeom& g, const void* packed,
                                       const void* x, int64_t T, void* y, const Epi& epi,
                                       cudaStream_t st) {
  DecodeParams<S> dp;
  fill_common(dp, p, g, packed, x, T, y, epi);
  constexpr int V = (S::KS1 == 1 && S::NT1 <= 16) ? 0 : (S::KS1 == 1 ? 1 : 2);
  if (g.MT2 > 1)
    return launch_decode_variant<S, E, S::RPc, S::KS1, S::NT1, V == 2 ? 1 : 2,
                                 V == 0 ? 384 : 256, 2>(dp, g, p.device, st);
  return launch_decode_variant<S, E, S::RPc, S::KS1, S::NT1, 4,
                               V == 0 ? 512 : (V == 1 ? 384 : 256), 1>(dp, g, p.device, st);
}

template <typename E, int RP>
static cudaError_t launch_decode_dyn(const Plan& p, const DecodeGeom& g, const void* packed,
                                     const void* x, int64_t T, void* y, const Epi& epi,
                                     cudaStream_t st) {
  DecodeParams<DynShape> dp;
  dp.sh = dyn_shape(p);
  fill_common(dp, p, g, packed, x, T, y, epi);
  if (g.MT2 > 1) {
    switch (decode_variant(p)) {
      case 0: return launch_decode_variant<DynShape, E, RP, 1, 16, 2, 384, 2>(dp, g, p.device, st);
      case 1: return launch_decode_variant<DynShape, E, RP, 1, 32, 2, 256, 2>(dp, g, p.device, st);
      default: return launch_decode_variant<DynShape, E, RP, 2, 32, 1, 256, 2>(dp, g, p.device, st);
    }
  }
  switch (decode_variant(p)) {
    case 0: return launch_decode_variant<DynShape, E, RP, 1, 16, 4, 512, 1>(dp, g, p.device, st);
    case 1: return launch_decode_variant<DynShape, E, RP, 1, 32, 4, 384, 1>(dp, g, p.device, st);
    default: return launch_decode_variant<DynShape, E, RP, 2, 32, 4, 256, 1>(dp, g, p.device, st);
  }
}

template <typename E>
static cudaError_t launch_decode_e(const Plan& p, const DecodeGeom& g, const void* packed,
                                   const void* x, int64_t T, void* y, const Epi& epi,
                                   cudaStream_t st) {
#define TRR_TRY_FIXED(a, b, c, d, e, f, r, X, Y)                                         \
  if (shape_matches<FixedShape<a, b, c, d, e, f, r, X, Y>>(p))                           \
    return launch_decode_fixed<FixedShape<a, b, c, d, e, f, r, X, Y>, E>(p, g, packed, x, T, \
                                                                         y, epi, st);
  TRR_FIXED_SHAPES(TRR_TRY_FIXED)
#undef TRR_TRY_FIXED
  return p.m.RP == 8 ? launch_decode_dyn<E, 8>(p, g, packed, x, T, y, epi, st)
                     : launch_decode_dyn<E, 16>(p, g, packed, x, T, y, epi, st);
}

int launch_decode(const Plan& p, const DecodeGeom& g, const void* packed, const void* x,
                  int64_t T, void* y, void* stream, const Epi& epi) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const cudaError_t e = p.dtype == TR_F16
                            ? launch_decode_e<__half>(p, g, packed, x, T, y, epi, st)
                            : launch_decode_e<__nv_bfloat16>(p, g, packed, x, T, y, epi, st);
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_error("decode kernel launch (chunks=%d CL=%d warps=%d smem=%zu): %s", g.NOC, g.CL, g.NW,
              g.smem, cudaGetErrorString(e));
    return TR_ERR_CUDA;
  }
  return TR_OK;
}

}  // namespace trr
