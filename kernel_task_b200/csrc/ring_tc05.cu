// Fused tensor-ring kernel on the 5th-generation tensor cores (tcgen05, TMEM accumulators) for
// token counts with several 128-row tiles of S2 rows (t, o1).  One launch per call.
//
// Per CTA: one row tile (TT tokens -> M = 128 rows (t, o1), zero-padded), one group of O2G output
// modes o2, and a contiguous range of ring pieces (i3, s).  Warp-specialised pipeline over the
// pieces, each stage handing buffers to the next through mbarriers:
//   warps 4-11  S1 (mma.sync): T1[(t,o1),(i2,u)] = sum_i1 x[t,i1,i2,i3] G1[s,o1,i1,u], written
//               straight into the K-major UMMA layout of S2's A operand (A2 ring, NA2 deep)
//   warp 12     issues every tcgen05.mma from one thread:
//               S2  D2[b] (TMEM, 2 buffers) = A2 . G2[(i2,u), (o2 of group, v)]
//               S3  D3[o2] (TMEM, accumulated over all pieces) += A3[b][o2] . G3_piece
//               and the TMA bulk copies of G2 (once) and the per-piece G3 operand (2-deep ring)
//   warps 0-3   read D2[b] from TMEM (one row per thread), round to fp16, write A3[b]
// G1 fragments of each piece arrive by TMA bulk copy (2-deep ring) issued by the S1 warps.
// After the last piece D3 is read out, summed across the cluster's CTAs through distributed
// shared memory (and across clusters through workspace slots when NC > 1) and written as y.
//
// Shared-memory operands use the no-swizzle K-major canonical layout: 8 x 16-byte core matrices,
// LBO between the K chunks of a row group, SBO between row groups.  A2 uses LBO = 144 B so that
// the S1 fragment stores of one warp (eight K chunks of one row group) hit distinct banks.
//
// Every wait on an mbarrier is bounded; on expiry the CTA raises a shared abort flag (all later
// waits return at once), records TR_ERR_TIMEOUT in the status word, still releases its TMEM and
// returns.
#include <cooperative_groups.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "device_util.cuh"
#include "plan.h"
#include "shapes.cuh"

namespace cg = cooperative_groups;

namespace trr {

constexpr int kTcThreads = 416;  // 4 converter warps + 8 S1 warps + 1 MMA warp
constexpr int kS1Threads = 256;
constexpr int kA2Lbo = 144;
constexpr unsigned kWaitLimit = 1u << 24;
// mbarrier slots
constexpr int kRing = 4;  // depth of the per-piece G1 and G3 operand rings
enum {
  BAR_A2FULL = 0,   // [2] S1 -> MMA (count 8: one arrive per S1 warp)
  BAR_A2FREE = 2,   // [2] MMA commit after S2 -> S1
  BAR_D2FULL = 4,   // [2] MMA commit after S2 -> converters
  BAR_D2FREE = 6,   // [2] converters (count 4) -> MMA
  BAR_A3FULL = 8,   // [2] converters (count 4) -> MMA
  BAR_A3FREE = 10,  // [2] MMA commit after S3 -> converters, G3 ring refill
  BAR_B3FULL = 12,  // [kRing] G3 bulk copy landed
  BAR_G1FULL = 16,  // [kRing] G1 bulk copy landed
  BAR_B2FULL = 20,  // G2 bulk copy landed
  BAR_D3DONE = 21,  // last S3 complete
  BAR_COUNT = 22
};

template <class S>
struct TcParams {
  S sh;
  const void* x;
  void* y;
  const uint2* g1f;
  const unsigned char* b2;
  const unsigned char* b3;
  float* slots;
  int* cnt;
  int* status;
  int T;
  int TT, MT1, CL, NC, NG, O2G, N2, N3P, K3P, tmem_cols;
  int g1p_bytes, b2_bytes, b3p_bytes;
  int off_xs, off_a2, off_b2, off_a3, off_g1, off_b3, off_bar;
  int NA2, a2_bytes, a3_bytes;
  int a2_sbo, slot_elems;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

// UMMA shared-memory matrix descriptor: no swizzle, K-major, sm_100 version field = 1.
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  return d;
}

// kind::f16 instruction descriptor: fp16 A and B, fp32 D, both K-major, M x N.
__host__ __device__ constexpr uint32_t umma_idesc_f16(int M, int N) {
  return (1u << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t dtmem, uint64_t da, uint64_t db, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(
          dtmem),
      "l"(da), "l"(db), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0));
}

__device__ __forceinline__ void umma_commit(uint32_t mbar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(mbar)
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
}
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}

// Bounded wait for the mbarrier phase with parity `parity` to complete: a non-blocking
// test_wait spin (a suspended try_wait wakes up late enough to dominate a short pipeline stage).
// Gives up at once when the CTA's abort flag is set, and sets it when the bound runs out.
__device__ __forceinline__ bool mbar_wait(uint32_t mbar, uint32_t parity, volatile int* abort) {
  for (unsigned i = 0; i < kWaitLimit; ++i) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(done)
        : "r"(mbar), "r"(parity)
        : "memory");
    if (done) return true;
    if ((i & 255) == 255) {
      if (*abort) return false;
      __nanosleep(32);
    }
  }
  *abort = 1;
  return false;
}

__device__ __forceinline__ void mbar_arrive(uint32_t mbar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(mbar) : "memory");
}

// One thread: TMA bulk copy of `bytes` (multiple of 16) global -> shared, completing on `mbar`.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes,
                                          uint32_t mbar) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(mbar), "r"(bytes)
               : "memory");
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::
          "r"(dst),
      "l"(src), "r"(bytes), "r"(mbar)
      : "memory");
}

__device__ __forceinline__ void s1_bar_sync() {
  asm volatile("bar.sync 1, %0;\n" ::"n"(kS1Threads) : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15}, [%16];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
}

__device__ __forceinline__ void copy_async16(unsigned char* dst, const void* src, int bytes,
                                             int tid, int nthr) {
  const uint32_t s = smem_u32(dst);
  const char* g = static_cast<const char*>(src);
  for (int i = tid * 16; i < bytes; i += nthr * 16)
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s + i), "l"(g + i)
                 : "memory");
}

template <class S, typename E, int RP>
__global__ void __launch_bounds__(kTcThreads, 1) ring_tc05_kernel(const TcParams<S> p) {
  const S& sh = p.sh;
  constexpr int K3 = RP < 16 ? 16 : RP;   // S3 K (v padded to 16)
  extern __shared__ __align__(128) unsigned char smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t4 = lane & 3;
  cg::cluster_group cluster = cg::this_cluster();

  const int NJ = p.CL * p.NC;
  const int bj = blockIdx.x % NJ;
  const int rest = blockIdx.x / NJ;
  const int grp = rest % p.NG;
  const int tile = rest / p.NG;
  const int crank = bj % p.CL;
  const int cl_id = bj / p.CL;
  const int pa = (int)((long long)bj * sh.npieces / NJ);
  const int pb = (int)((long long)(bj + 1) * sh.npieces / NJ);
  const int np = pb - pa;
  const int t0 = tile * p.TT;
  const int TTv = min(p.TT, p.T - t0);
  const int rows = TTv * sh.O1;
  const int o2a = grp * p.O2G;
  const int o2n = min(p.O2G, sh.O2 - o2a);
  const int a3_block = 128 * K3 * 2;

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + p.off_bar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + p.off_bar + BAR_COUNT * 8);
  int* flag = reinterpret_cast<int*>(smem + p.off_bar + BAR_COUNT * 8 + 4);
  volatile int* abort = reinterpret_cast<volatile int*>(smem + p.off_bar + BAR_COUNT * 8 + 8);
  auto bar = [&](int i) { return smem_u32(&bars[i]); };

  // ---- TMEM, mbarriers, zeroed operand buffers (padded rows and K columns contribute nothing)
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(p.tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
  }
  if (tid == 0) {
    const int counts[BAR_COUNT] = {8, 8, 1, 1, 1, 1, 4, 4, 4, 4, 1, 1,
                                   1, 1, 1, 1, 1, 1, 1, 1, 1, 1};
    for (int i = 0; i < BAR_COUNT; ++i)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar(i)), "r"(counts[i])
                   : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    *flag = 0;
    *abort = 0;
  }
  {
    uint4* z = reinterpret_cast<uint4*>(smem + p.off_a2);
    const int n16 = p.NA2 * p.a2_bytes / 16;
    for (int i = tid; i < n16; i += kTcThreads) z[i] = make_uint4(0u, 0u, 0u, 0u);
    uint4* z3 = reinterpret_cast<uint4*>(smem + p.off_a3);
    const int n3 = 2 * p.a3_bytes / 16;
    for (int i = tid; i < n3; i += kTcThreads) z3[i] = make_uint4(0u, 0u, 0u, 0u);
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;

  if (warp == 12) {
    // ================================ MMA issuer ================================
    if (lane == 0 && np > 0) {
      const uint32_t b2s = smem_u32(smem + p.off_b2);
      const uint32_t idesc2 = umma_idesc_f16(128, p.N2);
      const uint32_t idesc3 = umma_idesc_f16(128, p.N3P);
      const int b2_sbo = (sh.K2P / 8) * 128;
      const int b3_sbo = (K3 / 8) * 128;
      bulk_load(b2s, p.b2 + (size_t)grp * p.b2_bytes, p.b2_bytes, bar(BAR_B2FULL));
      for (int q = 0; q < kRing && q < np; ++q)
        bulk_load(smem_u32(smem + p.off_b3 + q * p.b3p_bytes),
                  p.b3 + (size_t)(pa + q) * p.b3p_bytes, p.b3p_bytes, bar(BAR_B3FULL + q));
      bool ok = mbar_wait(bar(BAR_B2FULL), 0, abort);
      for (int j = 0; j <= np && ok; ++j) {
        if (j < np) {  // ---- S2(j)
          const int ab = j % p.NA2, db = j & 1;
          ok = mbar_wait(bar(BAR_A2FULL + ab), (uint32_t)((j / p.NA2) & 1), abort);
          if (ok && j >= 2) ok = mbar_wait(bar(BAR_D2FREE + db), (uint32_t)(((j >> 1) - 1) & 1), abort);
          if (!ok) break;
          tc_fence_after();
          const uint32_t a2s = smem_u32(smem + p.off_a2 + ab * p.a2_bytes);
          for (int ks = 0; ks < sh.KS2; ++ks) {
            const uint64_t da = umma_desc(a2s + ks * 2 * kA2Lbo, kA2Lbo, p.a2_sbo);
            const uint64_t db2 = umma_desc(b2s + ks * 2 * 128, 128, b2_sbo);
            umma_f16(tmem + db * p.N2, da, db2, idesc2, ks > 0 ? 1u : 0u);
          }
          umma_commit(bar(BAR_A2FREE + ab));
          umma_commit(bar(BAR_D2FULL + db));
        }
        if (j >= 1) {  // ---- S3(j-1)
          const int jj = j - 1, bb = jj & 1, rb = jj % kRing;
          // Refill the G3 slot of piece jj-2 with piece jj+2.  S3(jj-2) completes phase
          // (jj-2)/2 of A3FREE[bb]; wait for it before S3(jj) is committed to the same barrier,
          // so the phase being waited for cannot have been overtaken by the next one.
          if (jj >= 2 && jj + 2 < np) {
            const int old = jj - 2;
            ok = mbar_wait(bar(BAR_A3FREE + bb), (uint32_t)((old >> 1) & 1), abort);
            if (!ok) break;
            const int slot = (jj + 2) % kRing;
            bulk_load(smem_u32(smem + p.off_b3 + slot * p.b3p_bytes),
                      p.b3 + (size_t)(pa + jj + 2) * p.b3p_bytes, p.b3p_bytes,
                      bar(BAR_B3FULL + slot));
          }
          ok = mbar_wait(bar(BAR_A3FULL + bb), (uint32_t)((jj >> 1) & 1), abort);
          if (ok) ok = mbar_wait(bar(BAR_B3FULL + rb), (uint32_t)((jj / kRing) & 1), abort);
          if (!ok) break;
          tc_fence_after();
          const uint32_t a3s = smem_u32(smem + p.off_a3 + bb * p.a3_bytes);
          const uint32_t b3s = smem_u32(smem + p.off_b3 + rb * p.b3p_bytes);
          for (int o = 0; o < o2n; ++o) {
#pragma unroll
            for (int ks = 0; ks < K3 / 16; ++ks) {
              const uint64_t da = umma_desc(a3s + o * a3_block + ks * 256, 128, (K3 / 8) * 128);
              const uint64_t db3 = umma_desc(b3s + ks * 256, 128, b3_sbo);
              umma_f16(tmem + 2 * p.N2 + o * p.N3P, da, db3, idesc3,
                       (jj > 0 || ks > 0) ? 1u : 0u);
            }
          }
          umma_commit(bar(BAR_A3FREE + bb));
        }
      }
      umma_commit(bar(BAR_D3DONE));
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ================================ S1 producers ================================
    const int sw = warp - 4, st = tid - 128;
    const int XSTR = (sh.KS1 * 16) + 8;
    const int M1P = p.MT1 * 16;
    const int s1rows = TTv * sh.I2;
    const int njobs1 = p.MT1 * sh.NT1;
    E* xs = reinterpret_cast<E*>(smem + p.off_xs);
    const E* x = static_cast<const E*>(p.x) + (size_t)t0 * sh.d_in;
    if (st == 0)
      for (int q = 0; q < kRing && q < np; ++q)
        bulk_load(smem_u32(smem + p.off_g1 + q * p.g1p_bytes),
                  p.g1f + (size_t)((pa + q) % sh.R) * sh.KS1 * sh.NT1 * 32, p.g1p_bytes,
                  bar(BAR_G1FULL + q));
    int cur_i3 = -1;
    bool ok = true;
    for (int j = 0; j < np; ++j) {
      const int pi = pa + j, i3 = pi / sh.R;
      if (i3 != cur_i3) {  // x slice of this i3: rows (t, i2), columns i1 (zero padded)
        s1_bar_sync();
        const int n = M1P * XSTR;
        for (int e = st; e < n; e += kS1Threads) {
          const int r = e / XSTR, c = e - r * XSTR;
          E v = from_f32<E>(0.f);
          if (r < s1rows && c < sh.I1) {
            const int t = r / sh.I2, i2 = r - t * sh.I2;
            v = x[(size_t)t * sh.d_in + c * sh.sx1 + i2 * sh.sx2 + i3 * sh.sx3];
          }
          xs[e] = v;
        }
        s1_bar_sync();
        cur_i3 = i3;
      }
      const int gb = j % kRing, ab = j % p.NA2;
      if (ok) ok = mbar_wait(bar(BAR_G1FULL + gb), (uint32_t)((j / kRing) & 1), abort);
      if (ok && j >= p.NA2)
        ok = mbar_wait(bar(BAR_A2FREE + ab), (uint32_t)(((j / p.NA2) - 1) & 1), abort);
      if (ok) {
        unsigned char* a2 = smem + p.off_a2 + ab * p.a2_bytes;
        const uint2* g1p = reinterpret_cast<const uint2*>(smem + p.off_g1 + gb * p.g1p_bytes) + lane;
        // four independent jobs at a time: (m16 tile, n8 tile) = job / NT1, job % NT1
        for (int jb = sw; jb < njobs1; jb += 4 * (kS1Threads / 32)) {
          float d[4][4];
          int jobs[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            jobs[u] = jb + u * (kS1Threads / 32);
#pragma unroll
            for (int c = 0; c < 4; ++c) d[u][c] = 0.f;
          }
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            if (jobs[u] < njobs1) {
              const int mt1 = jobs[u] / sh.NT1, nt1 = jobs[u] - mt1 * sh.NT1;
              for (int ks = 0; ks < sh.KS1; ++ks) {
                uint32_t a[4];
                ldsm_x4(a, xs + (size_t)(mt1 * 16 + (lane & 15)) * XSTR + ks * 16 +
                               (lane >> 4) * 8);
                const uint2 b = g1p[(size_t)(ks * sh.NT1 + nt1) * 32];
                mma_16816(d[u], a, b.x, b.y, E());
              }
            }
          }
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            if (jobs[u] < njobs1) {
              const int mt1 = jobs[u] / sh.NT1, nt1 = jobs[u] - mt1 * sh.NT1;
              const int col = nt1 * 8 + 2 * t4;
              const int o1 = col / RP, uu = col % RP;
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const int r = mt1 * 16 + g + 8 * h;
                if (r < s1rows) {
                  const int t = r / sh.I2, i2 = r - t * sh.I2;
                  const int row = t * sh.O1 + o1, k = i2 * RP + uu;
                  *reinterpret_cast<__half2*>(a2 + (row >> 3) * p.a2_sbo + (k >> 3) * kA2Lbo +
                                              (row & 7) * 16 + (k & 7) * 2) =
                      __floats2half2_rn(d[u][2 * h], d[u][2 * h + 1]);
                }
              }
            }
          }
        }
        fence_async_smem();
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(BAR_A2FULL + ab));
      s1_bar_sync();  // every S1 warp is done with G1 slot gb
      if (st == 0 && ok && j + kRing < np)
        bulk_load(smem_u32(smem + p.off_g1 + gb * p.g1p_bytes),
                  p.g1f + (size_t)((pa + j + kRing) % sh.R) * sh.KS1 * sh.NT1 * 32, p.g1p_bytes,
                  bar(BAR_G1FULL + gb));
    }
  } else {
    // ================================ D2 -> A3 converters ================================
    const int r = 32 * warp + lane;
    bool ok = true;
    for (int j = 0; j < np; ++j) {
      const int db = j & 1, ab = j & 1;
      if (ok) ok = mbar_wait(bar(BAR_D2FULL + db), (uint32_t)((j >> 1) & 1), abort);
      if (ok && j >= 2) ok = mbar_wait(bar(BAR_A3FREE + ab), (uint32_t)(((j >> 1) - 1) & 1), abort);
      tc_fence_after();
      if (ok) {
        const uint32_t d2 = tmem + db * p.N2 + lane_base;
        unsigned char* rowp = smem + p.off_a3 + ab * p.a3_bytes + (r >> 3) * ((K3 / 8) * 128) +
                              (r & 7) * 16;
        // 64 columns per batch: issue every TMEM load of the batch, then wait once
        for (int c0 = 0; c0 < p.N2; c0 += 64) {
          float v[4][16];
#pragma unroll
          for (int c = 0; c < 4; ++c)
            if (c0 + c * 16 < p.N2) tmem_ld16(d2 + c0 + c * 16, v[c]);
          tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < 4; ++c) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int col = c0 + c * 16 + 8 * h;  // D2 column = o * RP + v
              if (col < p.N2) {
                const int o = col / RP, vv = col % RP;
                uint4 q;
                q.x = pack2<__half>(v[c][8 * h + 0], v[c][8 * h + 1]);
                q.y = pack2<__half>(v[c][8 * h + 2], v[c][8 * h + 3]);
                q.z = pack2<__half>(v[c][8 * h + 4], v[c][8 * h + 5]);
                q.w = pack2<__half>(v[c][8 * h + 6], v[c][8 * h + 7]);
                *reinterpret_cast<uint4*>(rowp + o * a3_block + (vv >> 3) * 128) = q;
              }
            }
          }
        }
        fence_async_smem();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(bar(BAR_D2FREE + db));
        mbar_arrive(bar(BAR_A3FULL + ab));
      }
    }
  }

  // ---- D3 -> partial y of this CTA (rows (t,o1), columns (o of group, o3)), fp32 in smem.
  // Every role is past its last use of the operand space; D3DONE means every MMA completed.
  __syncthreads();
  float* ys = reinterpret_cast<float*>(smem);
  const int ystr = (p.O2G * sh.O3) | 1;  // odd row stride: one bank per row of the warp
  if (warp < 4) {
    const bool ok = np > 0 && mbar_wait(bar(BAR_D3DONE), 0, abort);
    tc_fence_after();
    const int r = 32 * warp + lane;
    for (int o = 0; o < o2n; ++o) {
      for (int c16 = 0; c16 < p.N3P / 16; ++c16) {
        float v[16];
        if (ok) {
          tmem_ld16(tmem + 2 * p.N2 + lane_base + o * p.N3P + c16 * 16, v);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) v[i] = 0.f;
        }
        if (r < rows) {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int o3 = c16 * 16 + i;
            if (o3 < sh.O3) ys[r * ystr + o * sh.O3 + o3] = v[i];
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {  // release TMEM: all reads completed (wait::ld) before the barrier
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem),
                 "r"(p.tmem_cols)
                 : "memory");
  }
  if (tid == 0 && *abort) atomicExch(p.status, (int)TR_ERR_TIMEOUT);

  // ---- reduce over the cluster: each CTA sums its slice of the tile from every peer's partial
  // (distributed shared memory, rank order), then across clusters through workspace slots
  const int nout = rows * o2n * sh.O3;
  const int SL = (nout + p.CL - 1) / p.CL;
  if (p.CL > 1) cluster.sync();  // all peers' partials are in their shared memory
  const float* peer[16];
#pragma unroll
  for (int k = 0; k < 16; ++k) peer[k] = (p.CL > 1 && k < p.CL) ? cluster.map_shared_rank(ys, k) : ys;
  E* y = static_cast<E*>(p.y) + (size_t)t0 * sh.d_out;
  const int ebeg = crank * SL;
  const int eend = min(nout, ebeg + SL);
  float* slot = p.NC > 1
      ? p.slots + (((size_t)tile * p.NG + grp) * p.NC + cl_id) * (size_t)p.slot_elems
      : nullptr;
  for (int e = ebeg + tid; e < eend; e += kTcThreads) {
    const int o3 = e % sh.O3, q = e / sh.O3;
    const int o = q % o2n, r = q / o2n;
    const int idx = r * ystr + o * sh.O3 + o3;
    float v[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) v[k] = k < p.CL ? peer[k][idx] : 0.f;
    float sum = 0.f;
#pragma unroll
    for (int k = 0; k < 16; ++k) sum += v[k];
    if (p.NC > 1) {
      slot[e] = sum;
    } else {
      const int t = r / sh.O1, o1 = r - t * sh.O1;
      y[(size_t)t * sh.d_out + o1 * sh.sy1 + (o2a + o) * sh.sy2 + o3 * sh.sy3] =
          from_f32<E>(sum);
    }
  }
  if (p.CL > 1) cluster.sync();  // peers finished reading this CTA's shared memory
  if (p.NC > 1) {
    __threadfence();
    __syncthreads();
    int* counter = p.cnt + ((size_t)tile * p.NG + grp) * p.CL + crank;
    if (tid == 0) *flag = (atomicAdd(counter, 1) == p.NC - 1);
    __syncthreads();
    if (*flag) {  // last cluster for this slice: add the NC slots in cluster order, write y
      __threadfence();
      const float* s0 = p.slots + ((size_t)tile * p.NG + grp) * p.NC * (size_t)p.slot_elems;
      for (int e = ebeg + tid; e < eend; e += kTcThreads) {
        float sum = 0.f;
        for (int c = 0; c < p.NC; ++c) sum += __ldcg(s0 + (size_t)c * p.slot_elems + e);
        const int o3 = e % sh.O3, q = e / sh.O3;
        const int o = q % o2n, r = q / o2n;
        const int t = r / sh.O1, o1 = r - t * sh.O1;
        y[(size_t)t * sh.d_out + o1 * sh.sy1 + (o2a + o) * sh.sy2 + o3 * sh.sy3] =
            from_f32<E>(sum);
      }
      if (tid == 0) atomicExch(counter, 0);
    }
  }
}

// ------------------------------------------------------------------------------------------
template <class S, typename E, int RP>
static cudaError_t launch_tc_variant(const TcParams<S>& tp, const TcGeom& g, int device,
                                     int grid, cudaStream_t st) {
  auto kern = ring_tc05_kernel<S, E, RP>;
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
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kTcThreads);
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
static void fill_tc(TcParams<S>& tp, const Plan& p, const TcGeom& g, const void* packed,
                    const void* x, int64_t T, void* y, void* ws) {
  const char* base = static_cast<const char*>(packed);
  const TcLayout& t = p.t;
  tp.x = x;
  tp.y = y;
  tp.g1f = reinterpret_cast<const uint2*>(base + p.m.off_g1);
  tp.b2 = reinterpret_cast<const unsigned char*>(base + t.off_b2);
  tp.b3 = reinterpret_cast<const unsigned char*>(base + t.off_b3);
  const size_t counters = ((size_t)g.ntiles * t.NG * g.CL * sizeof(int) + 255) / 256 * 256;
  tp.status = static_cast<int*>(ws);  // first word of the workspace
  tp.cnt = reinterpret_cast<int*>(static_cast<char*>(ws) + 256);
  tp.slots = reinterpret_cast<float*>(static_cast<char*>(ws) + 256 + counters);
  tp.T = (int)T;
  tp.TT = g.TT;
  tp.MT1 = g.MT1;
  tp.CL = g.CL;
  tp.NC = g.NC;
  tp.NG = t.NG;
  tp.O2G = t.O2G;
  tp.N2 = t.N2;
  tp.N3P = t.N3P;
  tp.K3P = t.K3P;
  tp.tmem_cols = t.tmem_cols;
  tp.g1p_bytes = p.m.KS1 * p.m.NT1 * 256;
  tp.b2_bytes = (int)t.bytes_b2_group;
  tp.b3p_bytes = (int)t.bytes_b3_piece;
  tp.off_xs = (int)g.off_xs;
  tp.off_a2 = (int)g.off_a2;
  tp.off_b2 = (int)g.off_b2;
  tp.off_a3 = (int)g.off_a3;
  tp.off_g1 = (int)g.off_pbuf;
  tp.off_b3 = (int)(g.off_pbuf + 4 * (size_t)tp.g1p_bytes);
  tp.off_bar = (int)g.off_bar;
  tp.NA2 = g.NA2;
  tp.a2_bytes = (int)g.a2_bytes;
  tp.a3_bytes = (int)(t.O2G * 128 * t.K3P * 2);
  tp.a2_sbo = (p.m.K2P / 8) * kA2Lbo;
  tp.slot_elems = 128 * t.O2G * p.c.O3;
}

template <class S, typename E>
static cudaError_t launch_tc_fixed(const Plan& p, const TcGeom& g, const void* packed,
                                   const void* x, int64_t T, void* y, void* ws, int grid,
                                   cudaStream_t st) {
  TcParams<S> tp;
  fill_tc(tp, p, g, packed, x, T, y, ws);
  return launch_tc_variant<S, E, S::RPc>(tp, g, p.device, grid, st);
}

template <class S>
static bool shape_is(const Plan& p) {
  return p.spec.input_modes[0] == S::in0 && p.spec.input_modes[1] == S::in1 &&
         p.spec.input_modes[2] == S::in2 && p.spec.output_modes[0] == S::on0 &&
         p.spec.output_modes[1] == S::on1 && p.spec.output_modes[2] == S::on2 &&
         p.spec.rank == S::R && p.c.role[0] == S::role0 && p.c.role[1] == S::role1;
}

template <typename E>
static cudaError_t launch_tc_e(const Plan& p, const TcGeom& g, const void* packed, const void* x,
                               int64_t T, void* y, void* ws, int grid, cudaStream_t st) {
#define TRR_TRY_TC(a, b, c, d, e, f, r, X, Y)                                               \
  if (shape_is<FixedShape<a, b, c, d, e, f, r, X, Y>>(p))                                 \
    return launch_tc_fixed<FixedShape<a, b, c, d, e, f, r, X, Y>, E>(p, g, packed, x, T, y, ws, \
                                                                     grid, st);
  TRR_FIXED_SHAPES(TRR_TRY_TC)
#undef TRR_TRY_TC
  TcParams<DynShape> tp;
  tp.sh = dyn_shape(p);
  fill_tc(tp, p, g, packed, x, T, y, ws);
  switch (p.m.RP) {
    case 8: return launch_tc_variant<DynShape, E, 8>(tp, g, p.device, grid, st);
    case 16: return launch_tc_variant<DynShape, E, 16>(tp, g, p.device, grid, st);
    default: return launch_tc_variant<DynShape, E, 32>(tp, g, p.device, grid, st);
  }
}

int launch_tc05(const Plan& p, const TcGeom& g, const void* packed, const void* x, int64_t T,
                void* y, void* ws, void* stream) {
  const int grid = g.ntiles * p.t.NG * g.CL * g.NC;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const cudaError_t e = p.dtype == TR_F16
                            ? launch_tc_e<__half>(p, g, packed, x, T, y, ws, grid, st)
                            : launch_tc_e<__nv_bfloat16>(p, g, packed, x, T, y, ws, grid, st);
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_error("tcgen05 kernel launch (grid=%d CL=%d NC=%d smem=%zu): %s", grid, g.CL, g.NC,
              g.smem, cudaGetErrorString(e));
    return TR_ERR_CUDA;
  }
  return TR_OK;
}

}  // namespace trr
