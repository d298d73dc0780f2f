// Preparation: pack the caller's three cores [R, o, i, R] into kernel-native layouts.
//
// Replaces pack_cores (factorized_inference/tr_kernel.py:86-99).  The layouts (plan.h describes
// the tcgen05 and slab operand layouts):
//   * generic  -- the canonical cores G1, G2, G3 in natural [l][o][i][r] order, plan dtype;
//   * mma      -- m16n8k16 B-operand fragments (one uint2 per lane per (k-step, n-tile)):
//                   G1 frags  [s][ks1][nt1][lane]       K = i1,     N = (o1,u)   plan dtype
//                   G2 frags  [ks2][nt2][lane]           K = (i2,u), N = (o2,v)   fp16
//                   G3 frags  [piece][ks3][nt3][lane]    K = v,      N = o3       fp16
//                 with piece = i3*R + s.  Ranks pad to RP (8/16/32) and modes to the tile
//                 edges with zeros, which leaves every sum unchanged.
// bf16 plans keep G1 in bf16 (S1 multiplies it with the bf16 x) and convert G2, G3 to fp16:
// the S2/S3 intermediates are fp16 so that bf16 rounding of the ring intermediates does not
// push the result past the 2e-3 relative Frobenius budget.
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>
#include <type_traits>

#include "device_util.cuh"
#include "plan.h"

namespace trr {

// One canonical core read through the reference storage order.  `rev` swaps the two rank
// axes (ring walked backwards).
template <typename E>
struct CoreView {
  const E* p;
  int O, I, R, rev;
  __device__ __forceinline__ float at(int l, int o, int i, int r) const {
    const int lo = rev ? r : l, ro = rev ? l : r;
    return to_f32<E>(p[(((size_t)lo * O + o) * I + i) * R + ro]);
  }
};

struct PackDims {
  int I1, I2, I3, O1, O2, O3, R;
  int RP, KS1, NT1, KS2, NT2, NT3, KS3, npieces;
};

template <typename E>
__global__ void pack_generic_kernel(CoreView<E> c0, CoreView<E> c1, CoreView<E> c2, E* g1, E* g2,
                                    E* g3, size_t n1, size_t n2, size_t n3) {
  const size_t total = n1 + n2 + n3;
  for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < total;
       idx += (size_t)gridDim.x * blockDim.x) {
    const CoreView<E>* c;
    E* out;
    size_t e;
    if (idx < n1) {
      c = &c0; out = g1; e = idx;
    } else if (idx < n1 + n2) {
      c = &c1; out = g2; e = idx - n1;
    } else {
      c = &c2; out = g3; e = idx - n1 - n2;
    }
    const int r = (int)(e % c->R);
    size_t q = e / c->R;
    const int i = (int)(q % c->I);
    q /= c->I;
    const int o = (int)(q % c->O);
    const int l = (int)(q / c->O);
    out[e] = from_f32<E>(c->at(l, o, i, r));
  }
}

// B fragment of m16n8k16 for lane (g, t4) = (lane/4, lane%4):
//   x = {B[2t4][g], B[2t4+1][g]},  y = {B[2t4+8][g], B[2t4+9][g]}   (low half first)
template <typename T, typename F>
__device__ __forceinline__ uint2 make_frag(int kbase, int nbase, int lane, F&& b) {
  const int g = lane >> 2, t4 = lane & 3;
  const int n = nbase + g, k = kbase + 2 * t4;
  uint2 out;
  out.x = pack2<T>(b(k, n), b(k + 1, n));
  out.y = pack2<T>(b(k + 8, n), b(k + 9, n));
  return out;
}

template <typename E>
__global__ void pack_mma_kernel(CoreView<E> c0, CoreView<E> c1, CoreView<E> c2, PackDims d,
                                uint2* f1, uint2* f2, uint2* f3, size_t n1, size_t n2, size_t n3) {
  const size_t total = n1 + n2 + n3;
  for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < total;
       idx += (size_t)gridDim.x * blockDim.x) {
    const int lane = (int)(idx & 31);
    if (idx < n1) {
      // G1 frags [s][ks1][nt1][lane]: B[k = i1][n = o1*RP + u] = G1[s, o1, i1, u]
      size_t q = idx >> 5;
      const int nt = (int)(q % d.NT1);
      q /= d.NT1;
      const int ks = (int)(q % d.KS1);
      const int s = (int)(q / d.KS1);
      f1[idx] = make_frag<E>(ks * 16, nt * 8, lane, [&](int k, int n) -> float {
        const int o1 = n / d.RP, u = n % d.RP;
        return (k < d.I1 && u < d.R) ? c0.at(s, o1, k, u) : 0.f;
      });
    } else if (idx < n1 + n2) {
      // G2 frags [ks2][nt2][lane]: B[k = i2*RP + u][n = o2*RP + v] = G2[u, o2, i2, v]
      const size_t e = idx - n1;
      size_t q = e >> 5;
      const int nt = (int)(q % d.NT2);
      const int ks = (int)(q / d.NT2);
      f2[e] = make_frag<__half>(ks * 16, nt * 8, lane, [&](int k, int n) -> float {
        const int i2 = k / d.RP, u = k % d.RP;
        const int o2 = n / d.RP, v = n % d.RP;
        return (i2 < d.I2 && u < d.R && v < d.R) ? c1.at(u, o2, i2, v) : 0.f;
      });
    } else {
      // G3 frags [piece][ks3][nt3][lane]: B[k = v][n = o3] = G3[v, o3, i3, s], piece = i3*R+s
      const size_t e = idx - n1 - n2;
      size_t q = e >> 5;
      const int nt = (int)(q % d.NT3);
      q /= d.NT3;
      const int ks = (int)(q % d.KS3);
      const int piece = (int)(q / d.KS3);
      const int i3 = piece / d.R, s = piece % d.R;
      f3[e] = make_frag<__half>(ks * 16, nt * 8, lane, [&](int k, int n) -> float {
        return (k < d.R && n < d.O3) ? c2.at(k, n, i3, s) : 0.f;
      });
    }
  }
}

// Byte offset of element (row r, column k) in a K-major UMMA tile with K columns: 8x8 core
// matrices of 128 contiguous bytes, K chunks 128 B apart (LBO), row groups K/8*128 B apart (SBO).
__host__ __device__ inline size_t umma_kmajor_offset(int r, int k, int K) {
  return (size_t)(r >> 3) * (K >> 3) * 128 + (size_t)(k >> 3) * 128 + (r & 7) * 16 + (k & 7) * 2;
}

struct TcPackDims {
  int I1, I2, I3, O1, O2, O3, R, RP, K1P, N1P, K2P, O2G, NG, N2, N3P, K3P, npieces;
};

// tcgen05 B operands: B1 per s [N1P rows (o1, u)] x [K1P i1] in the input dtype E, B2 per o2
// group [N2 rows (o2, v)] x [K2P (i2, u)] and B3 per piece [N3P rows o3] x [K3P v] in fp16; zero
// where a padded index has no core entry.
template <typename E>
__global__ void pack_tc_kernel(CoreView<E> c0, CoreView<E> c1, CoreView<E> c2, TcPackDims d,
                               unsigned char* b1, unsigned char* b2, unsigned char* b3, size_t n1,
                               size_t n2, size_t n3) {
  const size_t total = n1 + n2 + n3;
  for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < total;
       idx += (size_t)gridDim.x * blockDim.x) {
    if (idx < n1) {
      const int k = (int)(idx % d.K1P);
      size_t q = idx / d.K1P;
      const int n = (int)(q % d.N1P);
      const int s = (int)(q / d.N1P);
      const int o1 = n / d.RP, u = n % d.RP;
      const float v = (o1 < d.O1 && u < d.R && k < d.I1) ? c0.at(s, o1, k, u) : 0.f;
      *reinterpret_cast<E*>(b1 + (size_t)s * d.N1P * d.K1P * sizeof(E) +
                            umma_kmajor_offset(n, k, d.K1P)) = from_f32<E>(v);
      continue;
    }
    float v;
    unsigned char* dst;
    if (idx < n1 + n2) {
      const size_t e = idx - n1;
      const int k = (int)(e % d.K2P);
      size_t q = e / d.K2P;
      const int n = (int)(q % d.N2);
      const int grp = (int)(q / d.N2);
      const int o2 = grp * d.O2G + n / d.RP, vv = n % d.RP;
      const int i2 = k / d.RP, u = k % d.RP;
      v = (o2 < d.O2 && vv < d.R && i2 < d.I2 && u < d.R) ? c1.at(u, o2, i2, vv) : 0.f;
      dst = b2 + (size_t)grp * d.N2 * d.K2P * 2 + umma_kmajor_offset(n, k, d.K2P);
    } else {
      const size_t e = idx - n1 - n2;
      const int k = (int)(e % d.K3P);
      size_t q = e / d.K3P;
      const int n = (int)(q % d.N3P);
      const int piece = (int)(q / d.N3P);
      const int i3 = piece / d.R, s = piece % d.R;
      v = (n < d.O3 && k < d.R) ? c2.at(k, n, i3, s) : 0.f;
      dst = b3 + (size_t)piece * d.N3P * d.K3P * 2 + umma_kmajor_offset(n, k, d.K3P);
    }
    *reinterpret_cast<__half*>(dst) = __float2half_rn(v);
  }
}

struct SlabPackDims {
  int I1, I2, I3, O1, O2, O3, R, K1P, SW, NSL, RV, N1S, KSL, K2S, O2G, N2, N3P, K3P, npieces;
};

// Slab-kernel operands (ring_slab.cu): B1 per (s, sl) [N1S rows (o1, ul)] x [K1P i1] in the input
// dtype E, with u = SW sl + ul; B2 per o2 group [N2 rows (o2, v)] x [K2S (sl, i2, ul)] and B3 per
// piece [N3P rows o3] x [K3P v] in fp16; zero where a padded index has no core entry.
template <typename E>
__global__ void pack_slab_kernel(CoreView<E> c0, CoreView<E> c1, CoreView<E> c2, SlabPackDims d,
                                 unsigned char* b1, unsigned char* b2, unsigned char* b3,
                                 size_t n1, size_t n2, size_t n3) {
  const size_t total = n1 + n2 + n3;
  for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < total;
       idx += (size_t)gridDim.x * blockDim.x) {
    if (idx < n1) {
      const int k = (int)(idx % d.K1P);
      size_t q = idx / d.K1P;
      const int n = (int)(q % d.N1S);
      q /= d.N1S;
      const int sl = (int)(q % d.NSL);
      const int s = (int)(q / d.NSL);
      const int o1 = n / d.SW, ul = n % d.SW, u = d.SW * sl + ul;
      const float v = (o1 < d.O1 && u < d.R && k < d.I1) ? c0.at(s, o1, k, u) : 0.f;
      *reinterpret_cast<E*>(b1 + ((size_t)s * d.NSL + sl) * d.N1S * d.K1P * sizeof(E) +
                            umma_kmajor_offset(n, k, d.K1P)) = from_f32<E>(v);
      continue;
    }
    float v;
    unsigned char* dst;
    if (idx < n1 + n2) {
      const size_t e = idx - n1;
      const int k = (int)(e % d.K2S);
      size_t q = e / d.K2S;
      const int n = (int)(q % d.N2);
      const int grp = (int)(q / d.N2);
      const int o2 = grp * d.O2G + n / d.RV, vv = n % d.RV;
      const int sl = k / d.KSL, kk = k % d.KSL;
      const int i2 = kk / d.SW, u = d.SW * sl + kk % d.SW;
      v = (o2 < d.O2 && vv < d.R && i2 < d.I2 && u < d.R) ? c1.at(u, o2, i2, vv) : 0.f;
      dst = b2 + (size_t)grp * d.N2 * d.K2S * 2 + umma_kmajor_offset(n, k, d.K2S);
    } else {
      const size_t e = idx - n1 - n2;
      const int k = (int)(e % d.K3P);
      size_t q = e / d.K3P;
      const int n = (int)(q % d.N3P);
      const int piece = (int)(q / d.N3P);
      const int i3 = piece / d.R, s = piece % d.R;
      v = (n < d.O3 && k < d.R) ? c2.at(k, n, i3, s) : 0.f;
      dst = b3 + (size_t)piece * d.N3P * d.K3P * 2 + umma_kmajor_offset(n, k, d.K3P);
    }
    *reinterpret_cast<__half*>(dst) = __float2half_rn(v);
  }
}

template <typename E>
static int pack_typed(const Plan& p, const void* const cores[3], void* packed, cudaStream_t st) {
  const Canon& c = p.c;
  CoreView<E> v[3];
  for (int k = 0; k < 3; ++k) {
    const int m = c.role[k];
    v[k].p = static_cast<const E*>(cores[m]);
    v[k].O = p.spec.output_modes[m];
    v[k].I = p.spec.input_modes[m];
    v[k].R = c.R;
    v[k].rev = c.reversed;
  }
  char* base = static_cast<char*>(packed);
  bool done = false;
  if constexpr (!std::is_same<E, float>::value) {
    if (p.mma_ok) {
      done = true;
      const MmaLayout& m = p.m;
      PackDims d{c.I1, c.I2, c.I3, c.O1, c.O2, c.O3, c.R, m.RP, m.KS1, m.NT1, m.KS2, m.NT2, m.NT3,
                 m.KS3, m.npieces};
      const size_t n1 = m.bytes_g1 / 8, n2 = m.bytes_g2 / 8, n3 = m.bytes_g3 / 8;
      const size_t total = n1 + n2 + n3;
      const int blocks = (int)std::min<size_t>((total + 255) / 256, 4096);
      pack_mma_kernel<E><<<blocks, 256, 0, st>>>(
          v[0], v[1], v[2], d, reinterpret_cast<uint2*>(base + m.off_g1),
          reinterpret_cast<uint2*>(base + m.off_g2), reinterpret_cast<uint2*>(base + m.off_g3),
          n1, n2, n3);
      if (p.tc_ok) {
        const TcLayout& t = p.t;
        TcPackDims td{c.I1, c.I2, c.I3, c.O1, c.O2, c.O3, c.R, m.RP, m.K1P, t.N1P, m.K2P, t.O2G,
                      t.NG, t.N2, t.N3P, t.K3P, m.npieces};
        const size_t tn1 = (size_t)c.R * t.N1P * m.K1P;
        const size_t tn2 = (size_t)t.NG * t.N2 * m.K2P;
        const size_t tn3 = (size_t)m.npieces * t.N3P * t.K3P;
        const int tb = (int)std::min<size_t>((tn1 + tn2 + tn3 + 255) / 256, 4096);
        pack_tc_kernel<E><<<tb, 256, 0, st>>>(
            v[0], v[1], v[2], td, reinterpret_cast<unsigned char*>(base + t.off_b1),
            reinterpret_cast<unsigned char*>(base + t.off_b2),
            reinterpret_cast<unsigned char*>(base + t.off_b3), tn1, tn2, tn3);
      }
      if (p.slab_ok) {
        const SlabLayout& l = p.sl;
        SlabPackDims sd{c.I1, c.I2, c.I3, c.O1, c.O2, c.O3, c.R, m.K1P, l.SW, l.NSL, l.RV, l.N1S,
                        l.KSL, l.K2S, l.O2G, l.N2, l.N3P, l.K3P, m.npieces};
        const size_t sn1 = (size_t)c.R * l.NSL * l.N1S * m.K1P;
        const size_t sn2 = (size_t)l.NG * l.N2 * l.K2S;
        const size_t sn3 = (size_t)m.npieces * l.N3P * l.K3P;
        const int sb = (int)std::min<size_t>((sn1 + sn2 + sn3 + 255) / 256, 4096);
        pack_slab_kernel<E><<<sb, 256, 0, st>>>(
            v[0], v[1], v[2], sd, reinterpret_cast<unsigned char*>(base + l.off_b1),
            reinterpret_cast<unsigned char*>(base + l.off_b2),
            reinterpret_cast<unsigned char*>(base + l.off_b3), sn1, sn2, sn3);
      }
    }
  }
  if (!done) {
    const GenericLayout& g = p.g;
    const size_t total = g.elems_g1 + g.elems_g2 + g.elems_g3;
    const int blocks = (int)std::min<size_t>((total + 255) / 256, 4096);
    pack_generic_kernel<E><<<blocks, 256, 0, st>>>(
        v[0], v[1], v[2], reinterpret_cast<E*>(base + g.off_g1),
        reinterpret_cast<E*>(base + g.off_g2), reinterpret_cast<E*>(base + g.off_g3), g.elems_g1,
        g.elems_g2, g.elems_g3);
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("pack launch: %s", cudaGetErrorString(e));
    return TR_ERR_CUDA;
  }
  return TR_OK;
}

// Launched (normally, without programmatic serialization) after the pack kernels: the forward
// kernels read packed cores before their griddepcontrol.wait, which is safe because the packed
// buffer is written only here and this launch cannot start before the pack kernels completed.
__global__ void pack_fence_kernel() {}

int launch_pack(const Plan& p, const void* const cores[3], void* packed, void* stream) {
  int cur = -1;
  if (cudaGetDevice(&cur) != cudaSuccess || cur != p.device) {
    cudaGetLastError();
    set_error("current device %d is not the plan's device %d", cur, p.device);
    return TR_ERR_INVALID;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int r = TR_ERR_INVALID;
  switch (p.dtype) {
    case TR_F32: r = pack_typed<float>(p, cores, packed, st); break;
    case TR_F16: r = pack_typed<__half>(p, cores, packed, st); break;
    case TR_BF16: r = pack_typed<__nv_bfloat16>(p, cores, packed, st); break;
    default: set_error("unknown dtype"); return TR_ERR_INVALID;
  }
  if (r != TR_OK) return r;
  pack_fence_kernel<<<1, 32, 0, st>>>();
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("pack launch: %s", cudaGetErrorString(e));
    return TR_ERR_CUDA;
  }
  return TR_OK;
}

// ------------------------------------------------------------------------------------------
// Co-resident cluster counts.  Every kernel of this library holds one CTA per SM (shared memory
// or registers), so the count depends only on the cluster size; it is measured once per device
// with an empty kernel that asks for the opt-in shared memory.
__global__ void cluster_probe_kernel() {}

void query_max_clusters(int device, int num_sms, int out[17]) {
  static std::mutex mu;
  static int cache[64][17];
  static bool have[64] = {};
  // a 148-SM B200 (measured): 148, 74, -, 33, -, -, -, 15, -, -, -, 7, -, -, -, 7
  auto fallback = [&](int c) {
    if (c <= 2) return num_sms / c;
    if (c <= 4) return (num_sms * 33 / 148) * 4 / c;
    if (c <= 8) return (num_sms * 15 / 148) * 8 / c;
    if (c <= 12) return (num_sms * 7 / 148) * 12 / c;
    return num_sms * 7 / 148;
  };
  std::lock_guard<std::mutex> lock(mu);
  if (device >= 0 && device < 64 && have[device]) {
    for (int c = 0; c <= 16; ++c) out[c] = cache[device][c];
    return;
  }
  out[0] = 0;
  for (int c = 1; c <= 16; ++c) out[c] = std::max(1, fallback(c));
  int cur = -1, smem = 0;
  if (device < 0 || device >= 64 || cudaGetDevice(&cur) != cudaSuccess ||
      cudaDeviceGetAttribute(&smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, device) !=
          cudaSuccess) {
    cudaGetLastError();
    return;  // no device here: the B200 figures
  }
  if (cur != device) cudaSetDevice(device);
  bool ok = cudaFuncSetAttribute(cluster_probe_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 smem) == cudaSuccess &&
            cudaFuncSetAttribute(cluster_probe_kernel,
                                 cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess;
  for (int c = 1; ok && c <= 16; ++c) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(c * 8));
    cfg.blockDim = dim3(128);
    cfg.dynamicSmemBytes = (size_t)smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)c;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, cluster_probe_kernel, &cfg) == cudaSuccess && n > 0)
      out[c] = n;
    else
      ok = false;
  }
  cudaGetLastError();
  if (cur != device) cudaSetDevice(cur);
  for (int c = 0; c <= 16; ++c) cache[device][c] = out[c];
  have[device] = true;
}

}  // namespace trr
