// Fused tensor-ring kernel on the tcgen05 tensor cores for small token counts (decode).
//
// At small T the token rows cannot fill a 128-row MMA tile, so every contraction is issued
// transposed: the packed core is the A operand (M = 128 rows of (output mode, ring index)) and
// the tokens are the N side (N = 16 .. 256 columns).  The packed operands are the ones the
// tcgen05 prefill kernel uses (same K-major tiles, other roles).  Per ring piece (i3, s):
//   S1  D1[(o1,u), (t,i2)]  = G1_s[(o1,u), i1] . X_i3[(t,i2), i1]          M tiles of 128 rows
//   C1  D1 -> B2[(t,o1), (i2,u)] (fp16, shared memory)
//   S2  D2_g[(o2,v), (t,o1)] = G2_g[(o2,v), (i2,u)] . B2                    one per o2 group g
//   C2  D2_g -> A3_g[(t,o1,o2), v] (fp16)
//   S3  D3_g[(t,o1,o2), o3] += A3_g . G3_piece[o3, v]                       accumulated in TMEM
// A group holds O2G output modes o2 with O2G * RP <= 128 (S2's rows) and T * O1 * O2G <= 128
// (S3's rows).  A CTA covers NGC groups (G2 of those groups stays in shared memory) and a range
// of pieces; the clusters of the grid split the pieces, and the partial sums are added across a
// cluster through distributed shared memory (in rank order) and across clusters through
// workspace slots (in cluster order): deterministic.
//
// Stages run one after the other inside a CTA (256 threads; warp 0 issues the MMAs, all warps
// convert); the G1 slices and G3 pieces stream in through TMA bulk copies into a ring of
// buffers that is refilled as pieces finish, and the x slices of the CTA's pieces are staged
// once.  Every mbarrier wait is bounded: on expiry the CTA records TR_ERR_TIMEOUT in the status
// word, stops issuing work, drains what it issued and releases its TMEM.
#include <cooperative_groups.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <type_traits>

#include "device_util.cuh"
#include "plan.h"
#include "shapes.cuh"
#include "tc_util.cuh"

namespace cg = cooperative_groups;

namespace trr {

constexpr int kTcsThreads = 256;
constexpr int kTcsMaxRing = 16;

enum {
  TBAR_A2 = 0,     // G2 of the CTA's groups landed
  TBAR_MM = 1,     // commit after each batch of MMAs
  TBAR_DRAIN = 2,  // after a timeout: every MMA issued has completed
  TBAR_LD = 3,     // [kTcsMaxRing] G1 slice + G3 piece of ring slot k landed
  TBAR_COUNT = 3 + kTcsMaxRing
};

template <class S>
struct TcsParams {
  S sh;
  const void* x;
  void* y;
  const unsigned char* g1;  // packed G1 slices: N1P rows (o1, u) x K1P, element type E
  const unsigned char* g2;  // packed G2: rows (o2, v) x K2P, fp16
  const unsigned char* g3;  // packed G3 pieces: N3P rows o3 x K3P, fp16
  float* slots;
  int* cnt;
  int* status;
  int T, CL, NC, O2G, NG, NGC, MT1, N1P, N1C, N2C, N3P, K3P;
  int g1_bytes;   // one packed G1 slice
  int g2_rows;    // rows of packed G2 (every group, padded)
  int g3_bytes;   // one packed G3 piece
  int d1_col, d2_col, d3_col, tmem_cols;
  int off_a2, off_b1, off_a1, off_b3, off_b2, off_a3, off_ys, off_recv, off_bar;
  int a2_stride;  // bytes of one group's G2 block in shared memory (128 rows)
  int b1_bytes;   // one staged x slice
  int a1_stride;  // one ring slot of G1 (MT1 * 128 rows)
  int b3_stride;  // one ring slot of G3
  int b2_bytes, a3_stride;
  int NB;         // ring slots
  int NQ;         // x slices staged (i3 values of the CTA's piece range)
  int slot_elems;
  Epi epi;
};

template <class S, typename E, int RP>
__global__ void __launch_bounds__(kTcsThreads, 1) ring_tcs_kernel(const TcsParams<S> p) {
  static_assert(RP == 8 || RP == 16, "rank padded to 8 or 16");
  const S& sh = p.sh;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  cg::cluster_group cluster = cg::this_cluster();

  const int NJ = p.CL * p.NC;
  const int bj = blockIdx.x % NJ;
  const int gs = blockIdx.x / NJ;  // which set of NGC groups
  const int crank = bj % p.CL;
  const int cl_id = bj / p.CL;
  const int pa = (int)((long long)bj * sh.npieces / NJ);
  const int pb = (int)((long long)(bj + 1) * sh.npieces / NJ);
  const int np = pb - pa;
  const int i3a = pa / sh.R;
  const int g0 = gs * p.NGC;
  const int ngc = min(p.NGC, p.NG - g0);
  const int T = p.T;
  const int K1P = sh.KS1 * 16, K2P = sh.K2P;

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + p.off_bar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + p.off_bar + TBAR_COUNT * 8);
  int* flag = reinterpret_cast<int*>(smem + p.off_bar + TBAR_COUNT * 8 + 4);
  volatile int* abort = reinterpret_cast<volatile int*>(smem + p.off_bar + TBAR_COUNT * 8 + 8);
  auto bar = [&](int i) { return smem_u32(&bars[i]); };

  // ---- TMEM, mbarriers, zeroed operands (their padding is read by the MMAs)
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(p.tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
  }
  if (tid == 32) {
    for (int i = 0; i < TBAR_COUNT; ++i)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(bar(i)) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    *flag = 0;
    *abort = 0;
  }
  {
    uint4* z = reinterpret_cast<uint4*>(smem + p.off_b2);
    for (int i = tid; i < p.b2_bytes / 16; i += kTcsThreads) z[i] = make_uint4(0u, 0u, 0u, 0u);
    z = reinterpret_cast<uint4*>(smem + p.off_a3);
    for (int i = tid; i < p.NGC * p.a3_stride / 16; i += kTcsThreads)
      z[i] = make_uint4(0u, 0u, 0u, 0u);
  }
  // ---- the x slices of the CTA's pieces: rows (t, i2), K = i1 (zero padding)
  {
    const unsigned short* xt = static_cast<const unsigned short*>(p.x);
    const int kch = K1P / 8;
    const int per = p.N1C * kch;
    for (int e = tid; e < p.NQ * per; e += kTcsThreads) {
      const int q = e / per, r0 = e - q * per;
      const int r = r0 / kch, kc = r0 - r * kch;
      const int t = r / sh.I2, i2 = r - t * sh.I2;
      const int i3 = i3a + q;
      unsigned short v[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int i1 = kc * 8 + k;
        v[k] = (t < T && i3 < sh.I3 && i1 < sh.I1)
                   ? __ldg(xt + (size_t)t * sh.d_in + i1 * sh.sx1 + i2 * sh.sx2 + i3 * sh.sx3)
                   : (unsigned short)0;
      }
      uint4 w;
      w.x = v[0] | (uint32_t)v[1] << 16;
      w.y = v[2] | (uint32_t)v[3] << 16;
      w.z = v[4] | (uint32_t)v[5] << 16;
      w.w = v[6] | (uint32_t)v[7] << 16;
      *reinterpret_cast<uint4*>(smem + p.off_b1 + q * p.b1_bytes +
                                kmajor_offset(r, kc * 8, K1P)) = w;
    }
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;

  const uint32_t a2s = smem_u32(smem + p.off_a2);
  const uint32_t b1s = smem_u32(smem + p.off_b1);
  const uint32_t a1s = smem_u32(smem + p.off_a1);
  const uint32_t b3s = smem_u32(smem + p.off_b3);
  const uint32_t b2s = smem_u32(smem + p.off_b2);
  const uint32_t a3s = smem_u32(smem + p.off_a3);

  // ---- bulk copies: G2 of the CTA's groups once, then G1 slice + G3 piece per ring slot
  auto load_piece = [&](int j) {  // one thread
    const int pi = pa + j, slot = j % p.NB;
    const uint32_t b = bar(TBAR_LD + slot);
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(b),
                 "r"(p.g1_bytes + p.g3_bytes)
                 : "memory");
    bulk_copy(a1s + slot * p.a1_stride, p.g1 + (size_t)(pi % sh.R) * p.g1_bytes, p.g1_bytes, b);
    bulk_copy(b3s + slot * p.b3_stride, p.g3 + (size_t)pi * p.g3_bytes, p.g3_bytes, b);
  };
  if (tid == 0 && np > 0) {
    uint32_t total = 0;
    int rows[8];
    for (int g = 0; g < ngc; ++g) {
      const int r0 = (g0 + g) * p.O2G * RP;
      rows[g] = max(0, min(p.O2G * RP, p.g2_rows - r0));
      total += (uint32_t)rows[g] * K2P * 2;
    }
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar(TBAR_A2)),
                 "r"(total)
                 : "memory");
    for (int g = 0; g < ngc; ++g)
      if (rows[g] > 0)
        bulk_copy(a2s + g * p.a2_stride,
                  p.g2 + (size_t)(g0 + g) * p.O2G * RP * K2P * 2, rows[g] * K2P * 2,
                  bar(TBAR_A2));
    for (int j = 0; j < p.NB && j < np; ++j) load_piece(j);
  }

  const uint32_t sbo1 = (uint32_t)(K1P / 8) * 128;
  const uint32_t sbo2 = (uint32_t)(K2P / 8) * 128;
  const uint32_t sbo3 = (uint32_t)(p.K3P / 8) * 128;
  const uint32_t idesc1 = umma_idesc<E>(128, p.N1C);
  const uint32_t idesc2 = umma_idesc<__half>(128, p.N2C);
  const uint32_t idesc3 = umma_idesc<__half>(128, p.N3P);
  uint32_t mm_phase = 0;
  int issued = min(p.NB, np);  // pieces whose operands were requested (thread 0's count)
  // every thread waits for the commit of warp 0's latest batch of MMAs
  auto batch_wait = [&]() {
    mbar_spin(bar(TBAR_MM), mm_phase, abort);
    mm_phase ^= 1u;
    tc_fence_after();
  };
  // warp-uniform view of the abort flag (set by any thread whose wait ran out)
  auto aborted = [&]() { return __any_sync(0xffffffffu, *abort != 0); };
  // The loop runs the same barriers in every thread whatever happens: after a timeout warp 0
  // stops issuing MMAs (its commits still complete) and every later wait returns at once.
  for (int j = 0; j < np; ++j) {
    const int pi = pa + j, slot = j % p.NB;
    const int q = pi / sh.R - i3a;
    // ---- S1: M tiles of (o1, u) rows against the x slice of this i3
    if (warp == 0) {
      bool w = !aborted();
      if (w) w = warp_wait(bar(TBAR_LD + slot), (j / p.NB) & 1, abort);
      if (w && j == 0) w = warp_wait(bar(TBAR_A2), 0, abort);
      if (w) {
        tc_fence_after();
        for (int m = 0; m < p.MT1; ++m)
          for (int ks = 0; ks < K1P / 16; ++ks)
            umma_one(tmem + p.d1_col + m * p.N1C,
                     desc_plain(a1s + slot * p.a1_stride + m * 16 * sbo1 + ks * 256, 128, sbo1),
                     desc_plain(b1s + q * p.b1_bytes + ks * 256, 128, sbo1), idesc1,
                     ks > 0 ? 1u : 0u);
      }
      commit_one(bar(TBAR_MM));
    }
    batch_wait();
    // ---- C1: D1 lane (o1, u) of tile m, columns (t, i2) -> B2[(t, o1)][(i2, u)]
    if (warp < 4 * p.MT1) {
      const int m = warp >> 2;
      const int row = m * 128 + (warp & 3) * 32 + lane;
      const int o1 = row / RP, u = row - o1 * RP;
      const bool valid = o1 < sh.O1;
      for (int c0 = 0; c0 < p.N1C; c0 += 16) {
        uint32_t r[16];
        tmem_ld<16>(tmem + lane_base + p.d1_col + m * p.N1C + c0, r);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          const int col = c0 + c;
          if (valid && col < T * sh.I2) {
            const int t = col / sh.I2, i2 = col - t * sh.I2;
            *reinterpret_cast<__half*>(smem + p.off_b2 +
                                       kmajor_offset(t * sh.O1 + o1, i2 * RP + u, K2P)) =
                __float2half_rn(__uint_as_float(r[c]));
          }
        }
      }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    // ---- S2 of every group of the CTA
    if (warp == 0) {
      tc_fence_after();
      if (!aborted())
        for (int g = 0; g < ngc; ++g)
          for (int ks = 0; ks < K2P / 16; ++ks)
            umma_one(tmem + p.d2_col + g * p.N2C,
                     desc_plain(a2s + g * p.a2_stride + ks * 256, 128, sbo2),
                     desc_plain(b2s + ks * 256, 128, sbo2), idesc2, ks > 0 ? 1u : 0u);
      commit_one(bar(TBAR_MM));
    }
    batch_wait();
    // ---- C2: D2_g lane (o2, v), columns (t, o1) -> A3_g[(t, o1, o2)][v]
    for (int g = warp >> 2; g < ngc; g += kTcsThreads / 128) {
      const int row = (warp & 3) * 32 + lane;
      const int o2g = row / RP, v = row - o2g * RP;
      const bool valid = o2g < p.O2G && (g0 + g) * p.O2G + o2g < sh.O2;
      for (int c0 = 0; c0 < p.N2C; c0 += 16) {
        uint32_t r[16];
        tmem_ld<16>(tmem + lane_base + p.d2_col + g * p.N2C + c0, r);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          const int col = c0 + c;
          if (valid && col < T * sh.O1)
            *reinterpret_cast<__half*>(smem + p.off_a3 + g * p.a3_stride +
                                       kmajor_offset(col * p.O2G + o2g, v, p.K3P)) =
                __float2half_rn(__uint_as_float(r[c]));
        }
      }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    // ---- S3 of every group, accumulated over the pieces
    if (warp == 0) {
      tc_fence_after();
      if (!aborted())
        for (int g = 0; g < ngc; ++g)
          for (int ks = 0; ks < p.K3P / 16; ++ks)
            umma_one(tmem + p.d3_col + g * p.N3P,
                     desc_plain(a3s + g * p.a3_stride + ks * 256, 128, sbo3),
                     desc_plain(b3s + slot * p.b3_stride + ks * 256, 128, sbo3), idesc3,
                     (j > 0 || ks > 0) ? 1u : 0u);
      commit_one(bar(TBAR_MM));
    }
    batch_wait();
    // ---- refill the ring slot this piece used (its MMAs completed)
    if (tid == 0 && !*abort && j + p.NB < np) {
      load_piece(j + p.NB);
      issued = j + p.NB + 1;
    }
  }
  if (*abort) {  // a wait gave up: drain this CTA's own work in flight
    if (tid == 0) atomicExch(p.status, (int)TR_ERR_TIMEOUT);
    if (warp == 0) {
      commit_one(bar(TBAR_DRAIN));
      if (lane == 0) mbar_drain(bar(TBAR_DRAIN), 0);
    }
    if (tid == 0) {
      if (np > 0) mbar_drain(bar(TBAR_A2), 0);
      for (int k = 0; k < p.NB && k < issued; ++k) {
        const int last = k + ((issued - 1 - k) / p.NB) * p.NB;  // last piece loaded in slot k
        mbar_drain(bar(TBAR_LD + k), (last / p.NB) & 1);
      }
    }
  }

  // ---- D3 -> this CTA's partial sums in shared memory: ys[g][row (t, o1, o2)][o3]
  float* ys = reinterpret_cast<float*>(smem + p.off_ys);
  const int O3 = sh.O3;
  for (int g = warp >> 2; g < ngc; g += kTcsThreads / 128) {
    const int row = (warp & 3) * 32 + lane;
    for (int c0 = 0; c0 < p.N3P; c0 += 16) {
      uint32_t r[16];
      tmem_ld<16>(tmem + lane_base + p.d3_col + g * p.N3P + c0, r);
      tmem_wait_ld();
#pragma unroll
      for (int c = 0; c < 16; ++c)
        if (c0 + c < O3)
          ys[((size_t)g * 128 + row) * O3 + c0 + c] = np > 0 ? __uint_as_float(r[c]) : 0.f;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem),
                 "r"(p.tmem_cols)
                 : "memory");
  }

  // ---- reduce over the cluster: item e = (g, row, o3) belongs to rank e / SL; every CTA
  // pushes its partial of each item into the owner's receive slots, the owner adds them in rank
  // order and writes y (one cluster) or its workspace slot (NC > 1)
  const int nout = ngc * 128 * O3;
  const int SL = (nout + p.CL - 1) / p.CL;
  float* recv = reinterpret_cast<float*>(smem + p.off_recv);
  if (p.CL > 1) {
    cluster.sync();  // the receive slots overlap the peers' G2: every peer left its loop
    for (int e = tid; e < nout; e += kTcsThreads) {
      const int owner = e / SL;
      cluster.map_shared_rank(recv, owner)[crank * SL + (e - owner * SL)] = ys[e];
    }
    cluster.sync();
  }
  const int ebeg = crank * SL, eend = min(nout, ebeg + SL);
  auto store_y = [&](int e, float v) {
    const int o3 = e % O3, gr = e / O3;
    const int g = gr / 128, row = gr - g * 128;
    const int r2 = row / p.O2G, o2g = row - r2 * p.O2G;
    const int t = r2 / sh.O1, o1 = r2 - t * sh.O1;
    const int o2 = (g0 + g) * p.O2G + o2g;
    if (t < T && o2g < p.O2G && o2 < sh.O2)
      epi_store<E>(p.epi, p.y,
                   (size_t)t * sh.d_out + (size_t)o1 * sh.sy1 + (size_t)o2 * sh.sy2 +
                       (size_t)o3 * sh.sy3,
                   v);
  };
  float* slot = p.NC > 1 ? p.slots + ((size_t)gs * p.NC + cl_id) * (size_t)p.slot_elems : nullptr;
  for (int e = ebeg + tid; e < eend; e += kTcsThreads) {
    float v;
    if (p.CL > 1) {
      v = 0.f;
      for (int k = 0; k < p.CL; ++k) v += recv[k * SL + (e - ebeg)];
    } else {
      v = ys[e];
    }
    if (p.NC == 1) store_y(e, v);
    else slot[e] = v;
  }
  if (p.NC > 1) {
    __threadfence();
    __syncthreads();
    if (tid == 0) {
      const int old = atomicAdd(p.cnt + gs * p.CL + crank, 1);
      *flag = (old == p.NC - 1);
    }
    __syncthreads();
    if (*flag) {  // last cluster for this slice: add the NC slots in cluster order
      __threadfence();
      const float* s0 = p.slots + (size_t)gs * p.NC * p.slot_elems;
      for (int e = ebeg + tid; e < eend; e += kTcsThreads) {
        float v = 0.f;
        for (int c = 0; c < p.NC; ++c) v += __ldcg(s0 + (size_t)c * p.slot_elems + e);
        store_y(e, v);
      }
      if (tid == 0) atomicExch(p.cnt + gs * p.CL + crank, 0);
    }
  }
}

// ------------------------------------------------------------------------------------------
template <class S, typename E, int RP>
static cudaError_t launch_tcs_variant(const TcsParams<S>& tp, const TcsGeom& g, int device,
                                      cudaStream_t st) {
  auto kern = ring_tcs_kernel<S, E, RP>;
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
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(g.NGS * g.CL * g.NC));
  cfg.blockDim = dim3(kTcsThreads);
  cfg.dynamicSmemBytes = g.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)g.CL;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, tp);
}

DynShape dyn_shape(const Plan& p);  // ring_decode.cu

template <class S>
static void fill_tcs(TcsParams<S>& tp, const Plan& p, const TcsGeom& g, const void* packed,
                     const void* x, int64_t T, void* y, void* ws, const Epi& epi) {
  const char* base = static_cast<const char*>(packed);
  const TcLayout& t = p.t;
  tp.x = x;
  tp.y = y;
  tp.g1 = reinterpret_cast<const unsigned char*>(base + t.off_b1);
  tp.g2 = reinterpret_cast<const unsigned char*>(base + t.off_b2);
  tp.g3 = reinterpret_cast<const unsigned char*>(base + t.off_b3);
  const size_t counters = ((size_t)g.NGS * g.CL * sizeof(int) + 255) / 256 * 256;
  tp.status = static_cast<int*>(ws);
  tp.cnt = reinterpret_cast<int*>(static_cast<char*>(ws) + 256);
  tp.slots = reinterpret_cast<float*>(static_cast<char*>(ws) + 256 + counters);
  tp.T = (int)T;
  tp.CL = g.CL;
  tp.NC = g.NC;
  tp.O2G = g.O2G;
  tp.NG = g.NG;
  tp.NGC = g.NGC;
  tp.MT1 = g.MT1;
  tp.N1P = t.N1P;
  tp.N1C = g.N1C;
  tp.N2C = g.N2C;
  tp.N3P = t.N3P;
  tp.K3P = t.K3P;
  tp.g1_bytes = (int)t.bytes_b1_slice;
  tp.g2_rows = t.NG * t.N2;
  tp.g3_bytes = (int)t.bytes_b3_piece;
  tp.d1_col = g.d1_col;
  tp.d2_col = g.d2_col;
  tp.d3_col = g.d3_col;
  tp.tmem_cols = g.tmem_cols;
  tp.off_a2 = (int)g.off_a2;
  tp.off_b1 = (int)g.off_b1;
  tp.off_a1 = (int)g.off_a1;
  tp.off_b3 = (int)g.off_b3;
  tp.off_b2 = (int)g.off_b2;
  tp.off_a3 = (int)g.off_a3;
  tp.off_ys = (int)g.off_ys;
  tp.off_recv = (int)g.off_recv;
  tp.off_bar = (int)g.off_bar;
  tp.a2_stride = (int)g.a2_stride;
  tp.b1_bytes = (int)g.b1_bytes;
  tp.a1_stride = (int)g.a1_stride;
  tp.b3_stride = (int)g.b3_stride;
  tp.b2_bytes = (int)g.b2_bytes;
  tp.a3_stride = (int)g.a3_stride;
  tp.NB = g.NB;
  tp.NQ = g.NQ;
  tp.slot_elems = g.slot_elems;
  tp.epi = epi;
}

template <typename E>
static cudaError_t launch_tcs_e(const Plan& p, const TcsGeom& g, const void* packed,
                                const void* x, int64_t T, void* y, void* ws, const Epi& epi,
                                cudaStream_t st) {
  TcsParams<DynShape> tp;
  tp.sh = dyn_shape(p);
  fill_tcs(tp, p, g, packed, x, T, y, ws, epi);
  if (p.m.RP == 8) return launch_tcs_variant<DynShape, E, 8>(tp, g, p.device, st);
  return launch_tcs_variant<DynShape, E, 16>(tp, g, p.device, st);
}

int launch_tcs(const Plan& p, const TcsGeom& g, const void* packed, const void* x, int64_t T,
               void* y, void* ws, void* stream, const Epi& epi) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const cudaError_t e = p.dtype == TR_F16
                            ? launch_tcs_e<__half>(p, g, packed, x, T, y, ws, epi, st)
                            : launch_tcs_e<__nv_bfloat16>(p, g, packed, x, T, y, ws, epi, st);
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_error("tcgen05 small-T kernel launch (grid=%d CL=%d NC=%d smem=%zu): %s",
              g.NGS * g.CL * g.NC, g.CL, g.NC, g.smem, cudaGetErrorString(e));
    return TR_ERR_CUDA;
  }
  return TR_OK;
}

}  // namespace trr
