// Tensor-ring kernel on the 5th-generation tensor cores for ranks up to 32 and for large token
// counts: the ring rank is cut into slabs of SW = 8 or 4 ranks, and the first two stages
// advance slab by slab.  One launch per call; every contraction runs as tcgen05.mma with operands in shared
// memory and accumulators in TMEM.
//
// Per CTA: one row tile of TT tokens, one group of O2G output modes o2 and a contiguous range of
// ring pieces (i3, s).  Each piece's rank index u of the first link runs over NSL slabs of SW
// (u = SW sl + ul); slab step g = j NSL + sl of piece j:
//   S1  D1[g&1][(t,i2), (o1,ul)] = A1[(t,i2), i1] . B1_{s,sl}[(o1,ul), i1]     A1 = x slice of i3
//   C1  D1 -> A2 slot g%NA2 [(t,o1), (i2,ul)] (fp16): the transpose between S1's rows and S2's
//       rows, TMEM -> registers -> shared memory, one D1 row (t,i2) per thread
//   S2  D2[j%ND2][(t,o1), (o2,v)] += A2 slot . B2[(o2 of group, v), (sl, i2, ul)]   (K slab sl)
// and once per piece:
//   C2  D2 -> A3[o2][(t,o1), v] (fp16)
//   S3  D3[o2][(t,o1), o3] += A3[o2] . B3_piece[o3, v]                 (accumulated over pieces)
// D1 holds two slabs (2 * SW * O1 TMEM columns), so S1 of slab g+2 runs while C1 converts slab
// g+1, and S2 consumes each A2 slab as soon as it is written: the S1 -> C1 -> S2 chain overlaps
// across slabs instead of serialising per piece, at a fraction of a whole-piece D1's TMEM (the
// rest widens the o2 groups).  C1 stores one 16-byte chunk (SW 8) or half a chunk (SW 4) per o1.
// Roles (512 threads):
//   warps 0-7   C1 (warps w and w+4 read the same TMEM lanes, each half of the o1 range)
//   warps 8-11  C2, and the D3 read-out with warps 0-7 after the last piece
//   warp 12     S1 issuer: S1 of slab g once C1 has read slab g - 2 (its D1 buffer)
//   warp 13     S2 issuer: S2 of slab g once C1 has written it
//   warp 14     S3 issuer: S3 of each piece
//   warp 15     feeder: B2 once, B1 slab slices and B3 by TMA bulk copy (all at once when they
//               fit, else rings refilled as the tensor-core stages release slots), and the x
//               slice A1 of each further i3 (the first two are staged by the converter and
//               feeder warps)
// One issuing warp per stage: an issuer that waits (S2 on C2 reading D2, S3 on C2) holds up no
// other stage; measured with per-step clock marks, a single S1+S2 issuer held C1 idle most of
// each slab step behind S2's waits.
// Hand-offs are mbarriers: tcgen05.commit arrivals from the issuers (S1DONE, S2SL, S2DONE,
// S3DONE) and one arrival per converter warp (D1READ: its TMEM loads landed, the buffer may be
// overwritten; C1DONE / C2DONE: its operand slab is written).  Ring depths are chosen so that no
// barrier can complete a phase twice before its consumer tests it.  After the last piece D3 is
// summed across the cluster's CTAs through per-CTA workspace areas in L2 (lane-major, written
// straight from the TMEM loads) and across clusters through workspace slots when NC > 1, and
// written as y with the fused epilogue, as in ring_tc05.cu.  Launched with programmatic stream serialization: set-up and the first bulk
// copies of packed cores overlap the previous kernel; x, y and the workspace are touched only
// after griddepcontrol.wait.
//
// Shared-memory operand layouts (K-major):
//   A2 slot  128-byte swizzle: 64-element K slabs of 128 rows x 128 B, row groups 1024 B apart,
//            the 16-byte chunk index XOR (row & 7)
//   A1, B1, B2, A3, B3  no swizzle: 8 rows x 16 B core matrices, LBO 128 B, SBO = K/8 * 128 B
//
// Every wait is bounded (SlabParams::spin_limit polls); on expiry the CTA raises a shared abort
// flag (later waits return at once), records TR_ERR_TIMEOUT in the first workspace word, waits
// for its own bulk copies, and returns; the three issuing warps always wait for their own
// tensor-core work before the barrier that precedes the TMEM release.
#include <cooperative_groups.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "device_util.cuh"
#include "plan.h"
#include "shapes.cuh"
#include "tc_util.cuh"

namespace cg = cooperative_groups;

namespace trr {

constexpr int kSlThreads = 512;
constexpr int kSlBuildThreads = 416;  // converter and feeder warps: first x slices
constexpr unsigned kSlPollLimit = 1u << 24;  // feeder polls without progress before it gives up
constexpr int kSwSlab = 128 * 128;           // bytes of one 64-wide K slab of an A2 slot

enum {
  SB_A1FULL = 0,   // [2] x slice staged (count 1)
  SB_A1FREE = 2,   // [2] commit after the last S1 of that i3
  SB_G1FULL = 4,   // [4] B1 slab slice landed (slot 0 only when all load at once)
  SB_S1DONE = 8,   // [4] commit after S1(g), index g % 4
  SB_D1READ = 12,  // [2] C1 warps read D1 slab g (count 8), index g % 2
  SB_C1DONE = 14,  // [4] C1 warps wrote A2 slot of slab g (count 8), index g % 4
  SB_S2SL = 18,    // [4] commit after S2 of slab g: its A2 slot is free, index g % 4
  SB_S2DONE = 22,  // [2] commit after the last S2 slab of piece j, index j % 2
  SB_D2READ = 24,  // [2] C2 warps read D2(j) (count 4), index j % 2
  SB_C2DONE = 26,  // [2] C2 warps wrote A3(j) (count 4), index j % 2
  SB_S3DONE = 28,  // [16] commit after S3(j), index j % 16
  SB_B3FULL = 44,  // [16] B3 landed (slot 0 only when the whole range loads at once)
  SB_B2FULL = 60,  // B2 landed
  SB_D3DONE = 61,  // commit after the last S3: every tensor-core operation completed
  SB_DRAIN = 62,   // [3] after the piece loop: each issuing warp's own work completed
  SB_COUNT = 65
};

template <class S>
struct SlabParams {
  S sh;
  const void* x;
  void* y;
  const unsigned char* b1;
  const unsigned char* b2;
  const unsigned char* b3;
  float* slots;
  int* cnt;
  int* status;
  float* parts;    // per-CTA partial sums in the workspace (CL > 1)
  int T, TT, CL, NC, NG, O2G;
  int SW, NSL, N1S, KSS, K2S, RV, N2, ND2, N3P, K3P, d2_col, d3_col, tmem_cols;
  int b1_bytes, b2_bytes, b3_bytes;
  int off_a2, off_b2, off_a3, off_a1, off_g1, off_b3, off_bar;
  int NA2, a2_bytes, NA3, a3_bytes, a1_bytes, NB1, b1_all, NB3, b3_all;
  int ystr, vec_out, vec_out4, slot_elems, part_elems;
  int zero_a2;     // 1: A2 slots hold K columns C1 never writes (zeroed once)
  unsigned spin_limit;
  Epi epi;
};

// Eight fp32 (as raw TMEM words) -> one 16-byte chunk of fp16.
__device__ __forceinline__ uint4 sl_chunk_f16(const uint32_t* w) {
  uint4 q;
  q.x = pack2<__half>(__uint_as_float(w[0]), __uint_as_float(w[1]));
  q.y = pack2<__half>(__uint_as_float(w[2]), __uint_as_float(w[3]));
  q.z = pack2<__half>(__uint_as_float(w[4]), __uint_as_float(w[5]));
  q.w = pack2<__half>(__uint_as_float(w[6]), __uint_as_float(w[7]));
  return q;
}

// Byte offset of 16-byte chunk kc (K elements 8 kc .. 8 kc + 7) of row `row` in an A2 slot.
__device__ __forceinline__ uint32_t sl_a2_offset(int row, int kc) {
  return (uint32_t)((kc >> 3) * kSwSlab + (row >> 3) * 1024 + (row & 7) * 128 +
                    (((kc & 7) ^ (row & 7)) << 4));
}

// Stage the x slice of one i3 as S1's A operand: rows (t, i2) of the tile (zero beyond TTv
// tokens), K = i1 padded to 16 KS1.  Thread `bt` of `nb` builds 16-byte chunks bt, bt + nb, ...
template <class S>
__device__ __forceinline__ void sl_build_a1(const S& sh, unsigned char* a1,
                                            const unsigned short* xt, int TTv, int i3, int bt,
                                            int nb) {
  const int kch = sh.KS1 * 2;
  const int nchunks = 128 * kch;
  const uint32_t sbo = (uint32_t)kch * 128;
  for (int e = bt; e < nchunks; e += nb) {
    const int r = e / kch, kc = e - r * kch;
    const int t = r / sh.I2, i2 = r - t * sh.I2;
    unsigned short v[8];
    const unsigned short* row = xt + (size_t)t * sh.d_in + i2 * sh.sx2 + i3 * sh.sx3;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int i1 = kc * 8 + k;
      v[k] = (t < TTv && i1 < sh.I1) ? __ldg(row + i1 * sh.sx1) : (unsigned short)0;
    }
    uint4 q;
    q.x = v[0] | (uint32_t)v[1] << 16;
    q.y = v[2] | (uint32_t)v[3] << 16;
    q.z = v[4] | (uint32_t)v[5] << 16;
    q.w = v[6] | (uint32_t)v[7] << 16;
    *reinterpret_cast<uint4*>(a1 + (r >> 3) * sbo + kc * 128 + (r & 7) * 16) = q;
  }
}

template <class S, typename E>
__global__ void __launch_bounds__(kSlThreads, 1) ring_slab_kernel(const SlabParams<S> p) {
  const S& sh = p.sh;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  cg::cluster_group cluster = cg::this_cluster();
  const unsigned lim = p.spin_limit;

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
  const int i3a = pa / sh.R;
  const int nq = np > 0 ? (pb - 1) / sh.R - i3a + 1 : 0;  // i3 values of the range
  const int t0 = tile * p.TT;
  const int TTv = min(p.TT, p.T - t0);
  const int rows = TTv * sh.O1;
  const int o2a = grp * p.O2G;
  const int o2n = min(p.O2G, sh.O2 - o2a);
  const int NSL = p.NSL;
  const int G = np * NSL;  // slab steps of this CTA
  const int a3_block = 128 * p.K3P * 2;

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + p.off_bar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + p.off_bar + SB_COUNT * 8);
  int* flag = reinterpret_cast<int*>(smem + p.off_bar + SB_COUNT * 8 + 4);
  volatile int* abort = reinterpret_cast<volatile int*>(smem + p.off_bar + SB_COUNT * 8 + 8);
  auto bar = [&](int i) { return smem_u32(&bars[i]); };
  const unsigned short* xt = static_cast<const unsigned short*>(p.x) + (size_t)t0 * sh.d_in;
  auto d1_col = [&](int g) { return (g & 1) * p.N1S; };
  auto d2_col = [&](int j) { return p.d2_col + (j % p.ND2) * p.N2; };
  // packed B1 slice of slab step r: (s, sl) of piece r / NSL
  auto b1_slice = [&](int r) { return ((pa + r / NSL) % sh.R) * NSL + r % NSL; };

  const uint32_t a1s = smem_u32(smem + p.off_a1);
  const uint32_t g1s = smem_u32(smem + p.off_g1);
  const uint32_t a2s = smem_u32(smem + p.off_a2);
  const uint32_t b2s = smem_u32(smem + p.off_b2);
  const uint32_t a3s = smem_u32(smem + p.off_a3);
  const uint32_t b3s = smem_u32(smem + p.off_b3);

  // ---- set-up, all before one CTA barrier: warp 0 allocates TMEM; the feeder warp initialises
  // the mbarriers (one per lane: one thread initialising them all took 2 us) and sends its first
  // bulk copies of packed cores; every thread zeroes its share of the A-operand pads
  // (never-written K columns); the converter and feeder warps stage the first x slices after
  // griddepcontrol.wait, so the x gather overlaps the set-up.
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(p.tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
  }
  if (warp == 15) {
    for (int i = lane; i < SB_COUNT; i += 32) {
      int count = 1;
      if ((i >= SB_D1READ && i < SB_D1READ + 2) || (i >= SB_C1DONE && i < SB_C1DONE + 4))
        count = 8;
      if ((i >= SB_D2READ && i < SB_D2READ + 2) || (i >= SB_C2DONE && i < SB_C2DONE + 2))
        count = 4;
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar(i)), "r"(count)
                   : "memory");
    }
    // each lane's initialised barriers, visible to the async proxy before the first complete_tx
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    fence_async_smem();
    __syncwarp();
    if (lane == 0) {
      *flag = 0;
      *abort = 0;
      if (np > 0) {  // the feeder's first bulk copies go out at once
        bulk_load(b2s, p.b2 + (size_t)grp * p.b2_bytes, p.b2_bytes, bar(SB_B2FULL));
        if (p.b1_all) {
          bulk_load(g1s, p.b1, sh.R * NSL * p.b1_bytes, bar(SB_G1FULL));
        } else {
          for (int r = 0; r < p.NB1 && r < G; ++r)
            bulk_load(g1s + r * p.b1_bytes, p.b1 + (size_t)b1_slice(r) * p.b1_bytes,
                      p.b1_bytes, bar(SB_G1FULL + r));
        }
        if (p.b3_all) {
          bulk_load(b3s, p.b3 + (size_t)pa * p.b3_bytes, np * p.b3_bytes, bar(SB_B3FULL));
        } else {
          for (int q = 0; q < p.NB3 && q < np; ++q)
            bulk_load(b3s + q * p.b3_bytes, p.b3 + (size_t)(pa + q) * p.b3_bytes, p.b3_bytes,
                      bar(SB_B3FULL + q));
        }
      }
    }
    __syncwarp();
  }
  if (p.zero_a2) {
    uint4* z = reinterpret_cast<uint4*>(smem + p.off_a2);
    const int n16 = p.NA2 * p.a2_bytes / 16;
    for (int i = tid; i < n16; i += kSlThreads) z[i] = make_uint4(0u, 0u, 0u, 0u);
  }
  if (p.RV < p.K3P) {
    uint4* z = reinterpret_cast<uint4*>(smem + p.off_a3);
    const int n16 = p.NA3 * p.a3_bytes / 16;
    for (int i = tid; i < n16; i += kSlThreads) z[i] = make_uint4(0u, 0u, 0u, 0u);
  }
  if (warp < 12 || warp == 15) {  // first x slices: converter and feeder warps
    const int bt = tid < 384 ? tid : tid - 96;
    pdl_wait();
    for (int q = 0; q < 2 && q < nq; ++q)
      sl_build_a1(sh, smem + p.off_a1 + q * p.a1_bytes, xt, TTv, i3a + q, bt, kSlBuildThreads);
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (tid == 0)
    for (int q = 0; q < 2 && q < nq; ++q) mbar_arrive(bar(SB_A1FULL + q));
  const uint32_t tmem = *tmem_slot;
  const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;

  // S1 of slab step g, issued by a converged warp: waits for its x slice and B1 slab slice
  // (each only once when it does not change), accumulates into D1 slab buffer g & 1, signals
  // S1DONE (and A1FREE after the last slab of an i3).  False when a wait gave up.
  int s1_q_seen = -1;
  bool s1_b1_seen = false;
  auto issue_s1 = [&](int g) -> bool {
    const int j = g / NSL, sl = g - j * NSL;
    const int q = (pa + j) / sh.R - i3a;
    bool ok = true;
    if (q != s1_q_seen) {
      ok = warp_wait(bar(SB_A1FULL + (q & 1)), (q >> 1) & 1, abort, lim);
      s1_q_seen = q;
    }
    if (ok && !s1_b1_seen) {
      ok = p.b1_all ? warp_wait(bar(SB_G1FULL), 0, abort, lim)
                    : warp_wait(bar(SB_G1FULL + g % p.NB1), (g / p.NB1) & 1, abort, lim);
      s1_b1_seen = p.b1_all;
    }
    if (!ok) return false;
    const uint32_t a1 = a1s + (q & 1) * p.a1_bytes;
    const uint32_t b1 = g1s + (p.b1_all ? b1_slice(g) : g % p.NB1) * p.b1_bytes;
    const uint32_t sbo1 = (uint32_t)sh.KS1 * 256;
    const uint32_t idesc1 = umma_idesc<E>(128, p.N1S);
    for (int ks = 0; ks < sh.KS1; ++ks)
      umma_one(tmem + d1_col(g), desc_plain(a1 + ks * 256, 128, sbo1),
               desc_plain(b1 + ks * 256, 128, sbo1), idesc1, ks > 0 ? 1u : 0u);
    commit_one(bar(SB_S1DONE + (g & 3)));
    if (sl == NSL - 1 && (j == np - 1 || (pa + j + 1) % sh.R == 0))
      commit_one(bar(SB_A1FREE + (q & 1)));
    return true;
  };

  if (warp == 12) {
    // ===================== S1 issuer: S1 of slab g once C1 read slab g - 2 ====================
    // The whole warp runs the loop (uniform decisions); one elected lane issues.  S1 runs ahead
    // of S2 on its own: C1 is fed at its own pace, whatever S2 and C2 wait for.
    pdl_wait();
    bool ok = true;
    for (int g = 0; g < G && ok; ++g) {
      if (g >= 2) {  // the D1 slab buffer of g was read by C1 (slab g - 2)
        ok = warp_wait(bar(SB_D1READ + (g & 1)), ((g - 2) >> 1) & 1, abort, lim);
        tc_fence_after();
      }
      if (ok) ok = issue_s1(g);
    }
    // Drain this warp's tensor-core work before the CTA barrier that precedes the TMEM release,
    // whatever happened (another warp may raise the abort flag after the last MMA was issued).
    commit_one(bar(SB_DRAIN));
    if (lane == 0) mbar_drain_spin(bar(SB_DRAIN), 0);
    __syncwarp();
  } else if (warp == 13) {
    // ===================== S2 issuer: S2 of slab g once C1 wrote its A2 slot ==================
    pdl_wait();
    bool ok = true, b2ok = false;
    const uint32_t sbo2 = (uint32_t)(p.K2S / 8) * 128;
    const uint32_t idesc2 = umma_idesc<__half>(128, p.N2);
    for (int g = 0; g < G; ++g) {
      const int j = g / NSL, sl = g - j * NSL;
      if (ok) ok = warp_wait(bar(SB_C1DONE + (g & 3)), (g >> 2) & 1, abort, lim);
      if (ok && !b2ok) ok = b2ok = warp_wait(bar(SB_B2FULL), 0, abort, lim);
      if (ok && sl == 0 && j >= p.ND2) {  // the D2 buffer's previous piece was read by C2
        ok = warp_wait(bar(SB_D2READ + ((j - p.ND2) & 1)), ((j - p.ND2) >> 1) & 1, abort, lim);
        tc_fence_after();
      }
      if (ok) {
        const uint32_t a2 = a2s + (g % p.NA2) * p.a2_bytes;
        for (int ks = 0; ks < p.KSS; ++ks)
          umma_one(tmem + d2_col(j), desc_sw128(a2 + (ks >> 2) * kSwSlab + (ks & 3) * 32),
                   desc_plain(b2s + (sl * p.KSS + ks) * 256, 128, sbo2), idesc2,
                   (sl > 0 || ks > 0) ? 1u : 0u);
        commit_one(bar(SB_S2SL + (g & 3)));
        if (sl == NSL - 1) commit_one(bar(SB_S2DONE + (j & 1)));
      }
    }
    commit_one(bar(SB_DRAIN + 1));  // drain this warp's tensor-core work (as the S1 issuer)
    if (lane == 0) mbar_drain_spin(bar(SB_DRAIN + 1), 0);
    __syncwarp();
  } else if (warp == 14) {
    // ===================== S3 issuer: S3 of each piece ========================================
    pdl_wait();
    bool ok = true;
    const uint32_t sbo3 = (uint32_t)(p.K3P / 8) * 128;
    const uint32_t idesc3 = umma_idesc<__half>(128, p.N3P);
    const int KS3 = p.K3P / 16;
    for (int j = 0; j < np; ++j) {
      if (ok) ok = warp_wait(bar(SB_C2DONE + (j & 1)), (j >> 1) & 1, abort, lim);
      if (ok)
        ok = p.b3_all ? warp_wait(bar(SB_B3FULL), 0, abort, lim)
                      : warp_wait(bar(SB_B3FULL + j % p.NB3), (j / p.NB3) & 1, abort, lim);
      if (ok) {
        const uint32_t a3 = a3s + (j % p.NA3) * p.a3_bytes;
        const uint32_t b3 = b3s + (p.b3_all ? j : j % p.NB3) * p.b3_bytes;
        for (int o = 0; o < o2n; ++o)
          for (int ks = 0; ks < KS3; ++ks)
            umma_one(tmem + p.d3_col + o * p.N3P,
                     desc_plain(a3 + o * a3_block + ks * 256, 128, sbo3),
                     desc_plain(b3 + ks * 256, 128, sbo3), idesc3,
                     (j > 0 || ks > 0) ? 1u : 0u);
        commit_one(bar(SB_S3DONE + (j & 15)));
        if (j == np - 1) commit_one(bar(SB_D3DONE));
      }
    }
    commit_one(bar(SB_DRAIN + 2));  // drain this warp's tensor-core work (as the S1 issuer)
    if (lane == 0) mbar_drain_spin(bar(SB_DRAIN + 2), 0);
    __syncwarp();
  } else {
    if (warp < 8) {
      // ============================ C1: D1 slab -> A2 slot ======================================
      const int r1 = 32 * (warp & 3) + lane;  // D1 row (t, i2)
      const int tq = r1 / sh.I2, i2 = r1 - tq * sh.I2;
      const bool rvalid = tq < p.TT;
      const int h = (sh.O1 + 1) >> 1;
      const int o1a = (warp >> 2) ? h : 0, o1b = (warp >> 2) ? sh.O1 : h;
      const int SW = p.SW;                            // D1 slab columns (o1, ul): o1 * SW + ul
      const int nld = ((o1b - o1a) * SW + 15) >> 4;  // 16-column TMEM loads of this half
      constexpr int CB = 4;                          // loads in flight per wait
      bool ok = true;
      for (int g = 0; g < G; ++g) {
        if (ok) ok = mbar_spin(bar(SB_S1DONE + (g & 3)), (g >> 2) & 1, abort, lim);
        if (ok && g >= p.NA2)  // S2 of the slab that last used this A2 slot completed
          ok = mbar_spin(bar(SB_S2SL + ((g - p.NA2) & 3)), ((g - p.NA2) >> 2) & 1, abort, lim);
        bool d1_read = false;
        if (ok) {
          tc_fence_after();
          unsigned char* a2 = smem + p.off_a2 + (g % p.NA2) * p.a2_bytes;
          const uint32_t d1 = tmem + lane_base + d1_col(g) + o1a * SW;
          for (int cb = 0; cb < nld; cb += CB) {
            uint32_t v[CB][16];
#pragma unroll
            for (int c = 0; c < CB; ++c)
              if (cb + c < nld) tmem_ld<16>(d1 + (cb + c) * 16, v[c]);
            tmem_wait_ld();
            if (cb + CB >= nld) {  // last read of D1 slab g: S1(g + 2) may overwrite it
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive(bar(SB_D1READ + (g & 1)));
              d1_read = true;
            }
            if (rvalid && SW == 8) {
#pragma unroll
              for (int c = 0; c < CB; ++c) {
#pragma unroll
                for (int hh = 0; hh < 2; ++hh) {  // one load = two o1, one 16-byte chunk each
                  const int o1 = o1a + 2 * (cb + c) + hh;
                  if (cb + c < nld && o1 < o1b) {
                    const int row = tq * sh.O1 + o1;
                    *reinterpret_cast<uint4*>(a2 + sl_a2_offset(row, i2)) =
                        sl_chunk_f16(v[c] + 8 * hh);
                  }
                }
              }
            } else if (rvalid) {  // SW 4: one load = four o1, half a chunk (8 bytes) each
#pragma unroll
              for (int c = 0; c < CB; ++c) {
#pragma unroll
                for (int hh = 0; hh < 4; ++hh) {
                  const int o1 = o1a + 4 * (cb + c) + hh;
                  if (cb + c < nld && o1 < o1b) {
                    const int row = tq * sh.O1 + o1;
                    const uint32_t* w = v[c] + 4 * hh;
                    *reinterpret_cast<uint2*>(a2 + sl_a2_offset(row, i2 >> 1) + (i2 & 1) * 8) =
                        make_uint2(pack2<__half>(__uint_as_float(w[0]), __uint_as_float(w[1])),
                                   pack2<__half>(__uint_as_float(w[2]), __uint_as_float(w[3])));
                  }
                }
              }
            }
          }
          fence_async_smem();
        }
        if (!d1_read) {
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(SB_D1READ + (g & 1)));
        }
        __syncwarp();  // hand slab g to the S2 issuer
        if (lane == 0) mbar_arrive(bar(SB_C1DONE + (g & 3)));
      }
    } else if (warp < 12) {
      // ============================ C2: D2 -> A3 ============================
      const int r = 32 * (warp & 3) + lane;  // row (t, o1)
      bool ok = true;
      for (int j = 0; j < np; ++j) {
        const int db = j & 1, ab = j % p.NA3;
        if (ok) ok = mbar_spin(bar(SB_S2DONE + db), (j >> 1) & 1, abort, lim);
        if (ok && j >= p.NA3)  // S3 of the piece that last used this A3 buffer completed
          ok = mbar_spin(bar(SB_S3DONE + ((j - p.NA3) & 15)), ((j - p.NA3) >> 4) & 1, abort,
                         lim);
        if (ok) {
          tc_fence_after();
          const uint32_t d2 = tmem + lane_base + d2_col(j);
          unsigned char* rowp = smem + p.off_a3 + ab * p.a3_bytes +
                                (r >> 3) * ((p.K3P / 8) * 128) + (r & 7) * 16;
          // six 16-column loads per wait: config 3's 96 D2 columns in one wait (c3 T = 128
          // 2.80 -> 2.58 ms against four)
          constexpr int CB2 = 6;
          // D2 column = o * RV + v, walked in 8-column chunks: (o, vv) advance without division
          int o = 0, vv = 0;
          for (int c0 = 0; c0 < p.N2; c0 += 16 * CB2) {
            uint32_t v[CB2][16];
#pragma unroll
            for (int c = 0; c < CB2; ++c)
              if (c0 + c * 16 < p.N2) tmem_ld<16>(d2 + c0 + c * 16, v[c]);
            tmem_wait_ld();
            if (c0 + 16 * CB2 >= p.N2) {  // last read of D2(j): its buffer may be reused
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive(bar(SB_D2READ + db));
            }
#pragma unroll
            for (int c = 0; c < CB2; ++c) {
#pragma unroll
              for (int hh = 0; hh < 2; ++hh) {
                if (c0 + c * 16 + 8 * hh < p.N2) {
                  *reinterpret_cast<uint4*>(rowp + o * a3_block + (vv >> 3) * 128) =
                      sl_chunk_f16(v[c] + 8 * hh);
                  vv += 8;
                  if (vv == p.RV) {
                    vv = 0;
                    ++o;
                  }
                }
              }
            }
          }
          fence_async_smem();
        } else {
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(SB_D2READ + db));
        }
        __syncwarp();  // hand piece j to the S3 issuer
        if (lane == 0) mbar_arrive(bar(SB_C2DONE + (j & 1)));
      }
    } else {
      // ==================== feeder: ring refills and the x slices of further i3 ================
      // Polls; every decision is taken by all lanes together (a vote over their own tests).
      int r1 = p.b1_all ? G : min(p.NB1, G), r3 = p.b3_all ? np : min(p.NB3, np), q = 2;
      unsigned idle = 0;
      while ((q < nq || r1 < G || r3 < np) && !*abort) {
        bool prog = false;
        if (q < nq && __all_sync(0xffffffffu,
                                 mbar_test(bar(SB_A1FREE + (q & 1)), ((q >> 1) - 1) & 1))) {
          sl_build_a1(sh, smem + p.off_a1 + (q & 1) * p.a1_bytes, xt, TTv, i3a + q, lane, 32);
          fence_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(SB_A1FULL + (q & 1)));
          ++q;
          prog = true;
        }
        if (r1 < G && __all_sync(0xffffffffu, mbar_test(bar(SB_S1DONE + ((r1 - p.NB1) & 3)),
                                                        ((r1 - p.NB1) >> 2) & 1))) {
          if (lane == 0)
            bulk_load(g1s + (r1 % p.NB1) * p.b1_bytes,
                      p.b1 + (size_t)b1_slice(r1) * p.b1_bytes, p.b1_bytes,
                      bar(SB_G1FULL + r1 % p.NB1));
          __syncwarp();
          ++r1;
          prog = true;
        }
        if (r3 < np &&
            __all_sync(0xffffffffu, mbar_test(bar(SB_S3DONE + ((r3 - p.NB3) & 15)),
                                              ((r3 - p.NB3) >> 4) & 1))) {
          if (lane == 0)
            bulk_load(b3s + (r3 % p.NB3) * p.b3_bytes, p.b3 + (size_t)(pa + r3) * p.b3_bytes,
                      p.b3_bytes, bar(SB_B3FULL + r3 % p.NB3));
          __syncwarp();
          ++r3;
          prog = true;
        }
        if (prog) {
          idle = 0;
        } else if (++idle >= kSlPollLimit) {
          if (lane == 0) *abort = 1;
          __syncwarp();
        } else {
          __nanosleep(64);
        }
      }
      // wait for this CTA's bulk copies before the operand space is reused (normally each was
      // already consumed, so every test succeeds at once)
      if (lane == 0 && np > 0) {
        mbar_drain(bar(SB_B2FULL), 0);
        if (p.b1_all) mbar_drain(bar(SB_G1FULL), 0);
        else
          for (int k = max(0, r1 - p.NB1); k < r1; ++k)
            mbar_drain(bar(SB_G1FULL + k % p.NB1), (k / p.NB1) & 1);
        if (p.b3_all) mbar_drain(bar(SB_B3FULL), 0);
        else
          for (int k = max(0, r3 - p.NB3); k < r3; ++k)
            mbar_drain(bar(SB_B3FULL + k % p.NB3), (k / p.NB3) & 1);
      }
      __syncwarp();
    }
  }

  pdl_trigger();  // the next kernel may set up while this one reduces
  // ---- D3 -> partial y of this CTA (rows (t,o1), columns (o of group, o3)).
  // Cluster of CTAs with O3 a multiple of 4 (lm): straight from the TMEM loads to this CTA's
  // workspace area in L2, lane-major (float4 of column quad q = (o, o3 / 4) of row r at
  // q * RS + r), so that the stores need no staging and every warp store covers 512 contiguous
  // bytes.  Otherwise into shared memory (rows of ystr floats; the operand space is free once
  // D3DONE has completed every tensor-core operation).
  __syncthreads();
  float* ys = reinterpret_cast<float*>(smem);
  const int ystr = p.ystr;
  const bool lm = p.CL > 1 && (sh.O3 & 3) == 0;
  const int RS = p.TT * sh.O1;  // rows of a tile: the row stride of the lane-major layout
  float4* mine4 = reinterpret_cast<float4*>(p.parts + (size_t)blockIdx.x * p.part_elems);
  if (warp < 12) {
    const bool ok = np > 0 && mbar_spin(bar(SB_D3DONE), 0, abort, lim);
    tc_fence_after();
    const int r = 32 * (warp & 3) + lane;
    const bool vec4 = (sh.O3 & 3) == 0;
    const int nc16 = p.N3P / 16;
    for (int o = warp >> 2; o < o2n; o += 3) {
      // all of this o's TMEM chunks in flight at once, one wait
      uint32_t v[4][16];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        if (c < nc16 && ok) {
          tmem_ld<16>(tmem + lane_base + p.d3_col + o * p.N3P + c * 16, v[c]);
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) v[c][i] = 0u;
        }
      }
      if (ok) tmem_wait_ld();
      for (int c16 = 4; c16 < nc16; ++c16) {  // o3 beyond 64: one chunk at a time
        uint32_t w[16];
        if (ok) {
          tmem_ld<16>(tmem + lane_base + p.d3_col + o * p.N3P + c16 * 16, w);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) w[i] = 0u;
        }
        if (r < rows) {
          if (lm) {
#pragma unroll
            for (int k = 0; k < 4; ++k)
              if (c16 * 16 + 4 * k < sh.O3)
                __stcg(mine4 + (size_t)(o * (sh.O3 >> 2) + c16 * 4 + k) * RS + r,
                       make_float4(__uint_as_float(w[4 * k]), __uint_as_float(w[4 * k + 1]),
                                   __uint_as_float(w[4 * k + 2]), __uint_as_float(w[4 * k + 3])));
          } else {
            for (int i = 0; i < 16; ++i)
              if (c16 * 16 + i < sh.O3)
                ys[r * ystr + o * sh.O3 + c16 * 16 + i] = __uint_as_float(w[i]);
          }
        }
      }
      if (r < rows) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          if (c >= nc16) break;
          float* dst = ys + r * ystr + o * sh.O3 + c * 16;
          if (lm) {  // column quads (o, o3 / 4) of this row, lane-major: a warp store is 512 B
#pragma unroll
            for (int k = 0; k < 4; ++k)
              if (c * 16 + 4 * k < sh.O3)
                __stcg(mine4 + (size_t)(o * (sh.O3 >> 2) + c * 4 + k) * RS + r,
                       make_float4(__uint_as_float(v[c][4 * k]), __uint_as_float(v[c][4 * k + 1]),
                                   __uint_as_float(v[c][4 * k + 2]),
                                   __uint_as_float(v[c][4 * k + 3])));
          } else if (vec4) {
#pragma unroll
            for (int k = 0; k < 4; ++k)
              if (c * 16 + 4 * k < sh.O3)
                *reinterpret_cast<float4*>(dst + 4 * k) =
                    make_float4(__uint_as_float(v[c][4 * k]), __uint_as_float(v[c][4 * k + 1]),
                                __uint_as_float(v[c][4 * k + 2]), __uint_as_float(v[c][4 * k + 3]));
          } else {
#pragma unroll
            for (int i = 0; i < 16; ++i)
              if (c * 16 + i < sh.O3) dst[i] = __uint_as_float(v[c][i]);
          }
        }
      }
    }
  }
  if (lm) cluster_arrive_release();  // this CTA's partial sums are in L2; wait below
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {  // release TMEM: all reads completed (wait::ld) before the barrier
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem),
                 "r"(p.tmem_cols)
                 : "memory");
  }
  if (tid == 0 && *abort) atomicExch(p.status, (int)TR_ERR_TIMEOUT);

  const size_t ybase = (size_t)t0 * sh.d_out;
  if (lm) {
    // ---- reduce over the cluster, lane-major: item e = float4 of column quad q = e / rows, row
    // e % rows.  After the cluster barrier (release / acquire at cluster scope) rank r adds the
    // CL areas' values of items [r SLc, (r + 1) SLc), every rank's load in flight at once, in rank
    // order (the same order and sums as the row-major path), and writes y (one cluster per tile)
    // or its workspace slot (NC > 1; the last cluster to finish adds the NC slots in cluster
    // order).  Consecutive threads take consecutive rows: every load and slot access coalesces.
    const int nq4 = sh.O3 >> 2;
    const int nout = rows * o2n * nq4;
    const int SLc = (nout + p.CL - 1) / p.CL;
    const int ebeg = crank * SLc, eend = min(nout, ebeg + SLc);
    const size_t part4 = (size_t)p.part_elems / 4;
    const float4* parts0 = reinterpret_cast<const float4*>(p.parts) + (size_t)(blockIdx.x - crank) * part4;
    float4* slot = p.NC > 1
        ? reinterpret_cast<float4*>(p.slots) +
              (((size_t)tile * p.NG + grp) * p.NC + cl_id) * (size_t)(p.slot_elems / 4)
        : nullptr;
    const float4* s0 = reinterpret_cast<const float4*>(p.slots) +
                       ((size_t)tile * p.NG + grp) * p.NC * (size_t)(p.slot_elems / 4);
    auto store_y4 = [&](int e, float4 a) {
      const int q = e / rows, r = e - q * rows;
      const int o = q / nq4, o3 = (q - o * nq4) * 4;
      const int t = r / sh.O1, o1 = r - t * sh.O1;
      const size_t i = ybase + (size_t)t * sh.d_out + (size_t)o1 * sh.sy1 +
                       (size_t)(o2a + o) * sh.sy2 + (size_t)o3 * sh.sy3;
      const float f[4] = {a.x, a.y, a.z, a.w};
      if (p.vec_out4) {
        epi_store_vec<E, 4>(p.epi, p.y, i, f);
      } else {
#pragma unroll
        for (int k = 0; k < 4; ++k) epi_store<E>(p.epi, p.y, i + (size_t)k * sh.sy3, f[k]);
      }
    };
    cluster_wait_acquire();
    for (int e = ebeg + tid; e < eend; e += kSlThreads) {
      const int q = e / rows, r = e - q * rows;
      const float4* src = parts0 + (size_t)q * RS + r;
      float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int k0 = 0; k0 < p.CL; k0 += 8) {
        float4 u[8];
#pragma unroll
        for (int i = 0; i < 8; ++i)
          if (k0 + i < p.CL) u[i] = __ldcg(src + (size_t)(k0 + i) * part4);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          if (k0 + i < p.CL) {
            a.x += u[i].x; a.y += u[i].y; a.z += u[i].z; a.w += u[i].w;
          }
        }
      }
      if (p.NC > 1) slot[e] = a;
      else store_y4(e, a);
    }
    if (p.NC > 1) {
      // the CTA barrier gathers every thread's slot stores; thread 0's acq_rel arrival
      // publishes them at device scope and, for the last cluster, acquires the other clusters'
      // slots, which the second CTA barrier passes on to every thread
      __syncthreads();
      int* counter = p.cnt + ((size_t)tile * p.NG + grp) * p.CL + crank;
      if (tid == 0) *flag = (atom_add_acq_rel_gpu(counter, 1) == p.NC - 1);
      __syncthreads();
      if (*flag) {
        const size_t sl4 = (size_t)(p.slot_elems / 4);
        for (int e = ebeg + tid; e < eend; e += kSlThreads) {
          float4 u[5];
          float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
          for (int c0 = 0; c0 < p.NC; c0 += 5) {
#pragma unroll
            for (int i = 0; i < 5; ++i)
              if (c0 + i < p.NC) u[i] = __ldcg(s0 + (size_t)(c0 + i) * sl4 + e);
#pragma unroll
            for (int i = 0; i < 5; ++i) {
              if (c0 + i < p.NC) {
                a.x += u[i].x; a.y += u[i].y; a.z += u[i].z; a.w += u[i].w;
              }
            }
          }
          store_y4(e, a);
        }
        if (tid == 0) atomicExch(counter, 0);
      }
    }
    return;
  }

  // ---- reduce over the cluster.  Items: 8 consecutive o3 (vector path) or single elements.
  // Every CTA writes its partial sums to its own workspace area (through L2: far faster than
  // distributed shared memory for this all-to-all), then after a cluster barrier (release /
  // acquire at cluster scope) cluster rank r adds items [r SLc, (r + 1) SLc) of the CL areas in
  // rank order and writes y (one cluster per tile) or its workspace slot (NC > 1; the last
  // cluster to finish adds the NC slots in cluster order).
  const int W = p.vec_out ? 8 : 1;  // floats per item
  const int nper = p.vec_out ? sh.O3 / 8 : sh.O3;
  const int nout = rows * o2n * nper;
  const int SLc = (nout + p.CL - 1) / p.CL;
  const int ebeg = crank * SLc, eend = min(nout, ebeg + SLc);
  auto item_idx = [&](int e) {  // offset of item e inside ys (and a CTA's partial area)
    const int o3v = e % nper, q = e / nper;
    return (q / o2n) * ystr + (q % o2n) * sh.O3 + o3v * W;
  };
  const float* parts0 = p.parts + (size_t)(blockIdx.x - crank) * p.part_elems;  // rank 0's
  if (p.CL > 1) {
    float4* dst = reinterpret_cast<float4*>(p.parts + (size_t)blockIdx.x * p.part_elems);
    const float4* src = reinterpret_cast<const float4*>(ys);
    for (int i = tid; i < rows * ystr / 4; i += kSlThreads) __stcg(dst + i, src[i]);
    cluster.sync();
  }
  float* slot = p.NC > 1
      ? p.slots + (((size_t)tile * p.NG + grp) * p.NC + cl_id) * (size_t)p.slot_elems
      : nullptr;
  const float* s0 = p.slots + ((size_t)tile * p.NG + grp) * p.NC * (size_t)p.slot_elems;
  // write the 8 (or 1) finished values of item e to y
  auto store_y = [&](int e, const float* f) {
    const int o3v = e % nper, q = e / nper;
    const int o = q % o2n, r = q / o2n;
    const int t = r / sh.O1, o1 = r - t * sh.O1;
    const size_t i = ybase + (size_t)t * sh.d_out + (size_t)o1 * sh.sy1 +
                     (size_t)(o2a + o) * sh.sy2 + (size_t)o3v * W * sh.sy3;
    if (p.vec_out) {
      epi_store_vec<E, 8>(p.epi, p.y, i, f);
    } else {
      epi_store<E>(p.epi, p.y, i, f[0]);
    }
  };
  for (int e = ebeg + tid; e < eend; e += kSlThreads) {
    float f[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (p.CL > 1) {
      // four ranks' partials in flight at once (an L2 round trip each), added in rank order
      const float* src = parts0 + item_idx(e);
      for (int k0 = 0; k0 < p.CL; k0 += 4) {
        if (p.vec_out) {
          float4 u[4], w[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float4* rk =
                reinterpret_cast<const float4*>(src + (size_t)(k0 + i) * p.part_elems);
            if (k0 + i < p.CL) { u[i] = __ldcg(rk); w[i] = __ldcg(rk + 1); }
          }
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            if (k0 + i < p.CL) {
              f[0] += u[i].x; f[1] += u[i].y; f[2] += u[i].z; f[3] += u[i].w;
              f[4] += w[i].x; f[5] += w[i].y; f[6] += w[i].z; f[7] += w[i].w;
            }
          }
        } else {
          float v[4];
#pragma unroll
          for (int i = 0; i < 4; ++i)
            if (k0 + i < p.CL) v[i] = __ldcg(src + (size_t)(k0 + i) * p.part_elems);
#pragma unroll
          for (int i = 0; i < 4; ++i)
            if (k0 + i < p.CL) f[0] += v[i];
        }
      }
    } else {
      const float* src = ys + item_idx(e);
      for (int i = 0; i < W; ++i) f[i] = src[i];
    }
    if (p.NC > 1) {
      float* d = slot + (size_t)e * W;
      if (p.vec_out) {
        reinterpret_cast<float4*>(d)[0] = make_float4(f[0], f[1], f[2], f[3]);
        reinterpret_cast<float4*>(d)[1] = make_float4(f[4], f[5], f[6], f[7]);
      } else {
        *d = f[0];
      }
    } else {
      store_y(e, f);
    }
  }
  if (p.NC > 1) {
    // the CTA barrier orders every thread's slot stores before thread 0's fence and count (a
    // release at device scope); thread 0's fence after the count orders the last cluster's slot
    // reads after it (an acquire), and the barrier passes that on to the other threads
    __syncthreads();
    int* counter = p.cnt + ((size_t)tile * p.NG + grp) * p.CL + crank;
    if (tid == 0) {
      __threadfence();
      *flag = (atomicAdd(counter, 1) == p.NC - 1);
      __threadfence();
    }
    __syncthreads();
    if (*flag) {  // last cluster for this slice: add the NC slots in cluster order, write y
      for (int e = ebeg + tid; e < eend; e += kSlThreads) {
        float f[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int c = 0; c < p.NC; ++c) {
          const float* sc = s0 + (size_t)c * p.slot_elems + (size_t)e * W;
          if (p.vec_out) {
            const float4 u = __ldcg(reinterpret_cast<const float4*>(sc));
            const float4 w = __ldcg(reinterpret_cast<const float4*>(sc) + 1);
            f[0] += u.x; f[1] += u.y; f[2] += u.z; f[3] += u.w;
            f[4] += w.x; f[5] += w.y; f[6] += w.z; f[7] += w.w;
          } else {
            f[0] += __ldcg(sc);
          }
        }
        store_y(e, f);
      }
      if (tid == 0) atomicExch(counter, 0);
    }
  }
}

// ------------------------------------------------------------------------------------------
template <class S, typename E>
static cudaError_t launch_slab_variant(const SlabParams<S>& sp, const SlabGeom& g, int device,
                                       int grid, cudaStream_t st) {
  auto kern = ring_slab_kernel<S, E>;
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
  cfg.blockDim = dim3(kSlThreads);
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
  return cudaLaunchKernelEx(&cfg, kern, sp);
}

DynShape dyn_shape(const Plan& p);  // ring_decode.cu

template <class S>
static void fill_slab(SlabParams<S>& sp, const Plan& p, const SlabGeom& g, const void* packed,
                      const void* x, int64_t T, void* y, void* ws, const Epi& epi) {
  const char* base = static_cast<const char*>(packed);
  const SlabLayout& l = p.sl;
  sp.x = x;
  sp.y = y;
  sp.epi = epi;
  sp.b1 = reinterpret_cast<const unsigned char*>(base + l.off_b1);
  sp.b2 = reinterpret_cast<const unsigned char*>(base + l.off_b2);
  sp.b3 = reinterpret_cast<const unsigned char*>(base + l.off_b3);
  const size_t counters = ((size_t)g.ntiles * l.NG * g.CL * sizeof(int) + 255) / 256 * 256;
  sp.status = static_cast<int*>(ws);  // first word of the workspace
  sp.cnt = reinterpret_cast<int*>(static_cast<char*>(ws) + 256);
  sp.slots = reinterpret_cast<float*>(static_cast<char*>(ws) + 256 + counters);
  sp.parts = reinterpret_cast<float*>(static_cast<char*>(ws) + g.parts_off);
  sp.T = (int)T;
  sp.TT = g.TT;
  sp.CL = g.CL;
  sp.NC = g.NC;
  sp.NG = l.NG;
  sp.O2G = l.O2G;
  sp.SW = l.SW;
  sp.NSL = l.NSL;
  sp.N1S = l.N1S;
  sp.KSS = l.KSL / 16;
  sp.K2S = l.K2S;
  sp.RV = l.RV;
  sp.N2 = l.N2;
  sp.ND2 = l.ND2;
  sp.N3P = l.N3P;
  sp.K3P = l.K3P;
  sp.d2_col = l.d2_col;
  sp.d3_col = l.d3_col;
  sp.tmem_cols = l.tmem_cols;
  sp.b1_bytes = (int)l.bytes_b1;
  sp.b2_bytes = (int)l.bytes_b2;
  sp.b3_bytes = (int)l.bytes_b3;
  sp.off_a2 = (int)g.off_a2;
  sp.off_b2 = (int)g.off_b2;
  sp.off_a3 = (int)g.off_a3;
  sp.off_a1 = (int)g.off_a1;
  sp.off_g1 = (int)g.off_g1;
  sp.off_b3 = (int)g.off_b3;
  sp.off_bar = (int)g.off_bar;
  sp.NA2 = g.NA2;
  sp.a2_bytes = (int)g.a2_bytes;
  sp.NA3 = g.NA3;
  sp.a3_bytes = (int)g.a3_bytes;
  sp.a1_bytes = (int)g.a1_bytes;
  sp.NB1 = g.NB1;
  sp.b1_all = g.b1_all;
  sp.NB3 = g.NB3;
  sp.b3_all = g.b3_all;
  sp.ystr = g.ystr;
  sp.part_elems = (int)g.part_elems;
  sp.zero_a2 = p.c.I2 * l.SW < l.KSL;
  const Canon& c = p.c;
  sp.vec_out = c.sy3 == 1 && c.O3 % 8 == 0 && c.sy1 % 8 == 0 && c.sy2 % 8 == 0 &&
               c.d_out % 8 == 0 && (reinterpret_cast<uintptr_t>(y) & 15) == 0;
  sp.vec_out4 = c.sy3 == 1 && c.O3 % 4 == 0 && c.sy1 % 4 == 0 && c.sy2 % 4 == 0 &&
                c.d_out % 4 == 0 && (reinterpret_cast<uintptr_t>(y) & 15) == 0;
  sp.slot_elems = 128 * l.O2G * c.O3;
  sp.spin_limit = p.wait_limit ? p.wait_limit : kSpinLimit;
}

template <class S, typename E>
static cudaError_t launch_slab_fixed(const Plan& p, const SlabGeom& g, const void* packed,
                                     const void* x, int64_t T, void* y, void* ws, int grid,
                                     const Epi& epi, cudaStream_t st) {
  SlabParams<S> sp;
  fill_slab(sp, p, g, packed, x, T, y, ws, epi);
  return launch_slab_variant<S, E>(sp, g, p.device, grid, st);
}

template <class S>
static bool slab_shape_is(const Plan& p) {
  return p.spec.input_modes[0] == S::in0 && p.spec.input_modes[1] == S::in1 &&
         p.spec.input_modes[2] == S::in2 && p.spec.output_modes[0] == S::on0 &&
         p.spec.output_modes[1] == S::on1 && p.spec.output_modes[2] == S::on2 &&
         p.spec.rank == S::R && p.c.role[0] == S::role0 && p.c.role[1] == S::role1;
}

template <typename E>
static cudaError_t launch_slab_e(const Plan& p, const SlabGeom& g, const void* packed,
                                 const void* x, int64_t T, void* y, void* ws, int grid,
                                 const Epi& epi, cudaStream_t st) {
#define TRR_TRY_SLAB(a, b, c, d, e, f, r, X, Y)                                                   \
  if (slab_shape_is<FixedShape<a, b, c, d, e, f, r, X, Y>>(p))                                   \
    return launch_slab_fixed<FixedShape<a, b, c, d, e, f, r, X, Y>, E>(p, g, packed, x, T, y, ws, \
                                                                      grid, epi, st);
  TRR_SLAB_SHAPES(TRR_TRY_SLAB)
#undef TRR_TRY_SLAB
  SlabParams<DynShape> sp;
  sp.sh = dyn_shape(p);
  fill_slab(sp, p, g, packed, x, T, y, ws, epi);
  return launch_slab_variant<DynShape, E>(sp, g, p.device, grid, st);
}

int launch_slab(const Plan& p, const SlabGeom& g, const void* packed, const void* x, int64_t T,
                void* y, void* ws, void* stream, const Epi& epi) {
  const int grid = g.ntiles * p.sl.NG * g.CL * g.NC;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const cudaError_t e =
      p.dtype == TR_F16 ? launch_slab_e<__half>(p, g, packed, x, T, y, ws, grid, epi, st)
                        : launch_slab_e<__nv_bfloat16>(p, g, packed, x, T, y, ws, grid, epi, st);
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_error("slab kernel launch (grid=%d CL=%d NC=%d smem=%zu): %s", grid, g.CL, g.NC, g.smem,
              cudaGetErrorString(e));
    return TR_ERR_CUDA;
  }
  return TR_OK;
}

}  // namespace trr
