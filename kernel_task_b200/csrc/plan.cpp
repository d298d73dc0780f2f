// Host planner of the tensor-ring operator: spec validation, contraction-order choice,
// packed-core layout, per-call kernel geometry, and the C-ABI entry points that do not launch.
//
// Spec rules follow TRSpec.__post_init__ / _validate (reference.py:27-31, 85-96).  The order
// choice replaces the reference's fixed x.A -> .B -> .C sequence (reference.py:122-124) by the
// cheapest of the six ring orders; the arithmetic it evaluates is the same sum.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <new>
#include <string>

#include "plan.h"

namespace trr {

static thread_local std::string g_last_error;

void set_error(const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
}

static int ceil_div(int a, int b) { return (a + b - 1) / b; }
static size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Multiply-adds per token of order (X first, then Y, then Z) on the canonical chain
//   S1: d_in*o_X*R^2   S2: i_Y*i_Z*o_X*o_Y*R^3   S3: d_out*i_Z*R^2
static double order_macs(const tr_spec& s, int X, int Y, int Z) {
  const double R = s.rank;
  const double din = (double)s.input_modes[0] * s.input_modes[1] * s.input_modes[2];
  const double dout = (double)s.output_modes[0] * s.output_modes[1] * s.output_modes[2];
  return din * s.output_modes[X] * R * R +
         (double)s.input_modes[Y] * s.input_modes[Z] * s.output_modes[X] * s.output_modes[Y] * R *
             R * R +
         dout * s.input_modes[Z] * R * R;
}

static void build_canon(const tr_spec& s, int X, int Y, Canon* c) {
  const int Z = 3 - X - Y;
  c->role[0] = X;
  c->role[1] = Y;
  c->role[2] = Z;
  c->reversed = (Y == (X + 2) % 3) ? 1 : 0;  // Y precedes X on the ring A->B->C->A
  c->I1 = s.input_modes[X];
  c->I2 = s.input_modes[Y];
  c->I3 = s.input_modes[Z];
  c->O1 = s.output_modes[X];
  c->O2 = s.output_modes[Y];
  c->O3 = s.output_modes[Z];
  c->R = s.rank;
  c->d_in = s.input_modes[0] * s.input_modes[1] * s.input_modes[2];
  c->d_out = s.output_modes[0] * s.output_modes[1] * s.output_modes[2];
  const int64_t xs[3] = {(int64_t)s.input_modes[1] * s.input_modes[2], s.input_modes[2], 1};
  const int64_t ys[3] = {(int64_t)s.output_modes[1] * s.output_modes[2], s.output_modes[2], 1};
  c->sx1 = xs[X];
  c->sx2 = xs[Y];
  c->sx3 = xs[Z];
  c->sy1 = ys[X];
  c->sy2 = ys[Y];
  c->sy3 = ys[Z];
}

static size_t elem_size(int dtype) { return dtype == TR_F32 ? 4 : 2; }

static void build_mma_layout(Plan* p) {
  const Canon& c = p->c;
  MmaLayout& m = p->m;
  m.RP = c.R <= 8 ? 8 : (c.R <= 16 ? 16 : 32);
  m.K1P = ceil_div(c.I1, 16) * 16;
  m.KS1 = m.K1P / 16;
  m.NT1 = c.O1 * m.RP / 8;
  m.K2P = ceil_div(c.I2 * m.RP, 16) * 16;
  m.KS2 = m.K2P / 16;
  m.NT2 = c.O2 * m.RP / 8;
  m.O3P = ceil_div(c.O3, 8) * 8;
  m.NT3 = m.O3P / 8;
  m.KS3 = m.RP >= 16 ? m.RP / 16 : 1;
  m.npieces = c.I3 * c.R;
  const size_t frag = 32 * 8;  // one B fragment of a warp: 32 lanes x uint2
  m.bytes_g1 = (size_t)c.R * m.KS1 * m.NT1 * frag;
  m.bytes_g2 = (size_t)m.KS2 * m.NT2 * frag;
  m.bytes_g3 = (size_t)m.npieces * m.KS3 * m.NT3 * frag;
  m.off_g1 = 0;
  m.off_g2 = align_up(m.off_g1 + m.bytes_g1, 256);
  m.off_g3 = align_up(m.off_g2 + m.bytes_g2, 256);
}

// Shared memory of one tcgen05 CTA (ring_tc05.cu), relative to a 1024-byte aligned base:
//   A2 x NA2 (S2 A operand, 128-byte swizzle, 64-wide K slabs of 128 rows), B2 of the group,
//   A3 x NA3 (S3 A operands of the group's o2), A1 x 2 (x slices), B1 x NB1, B3 x NB3,
// reused after the piece loop as the CTA's fp32 partial y [128 rows x ystr] and the receive
// buffers of the cluster reduction, then the mbarriers.  `total` includes 1 KB of slack for aligning the dynamic shared-memory window.
struct TcSmem {
  size_t a2_bytes, a3_bytes, a1_bytes;
  size_t off_a2, off_b2, off_a3, off_a1, off_g1, off_b3, off_bar, total;
};

// Row stride of the partial y: at least O2G*O3 floats, 4 times an odd number (16-byte rows for
// vector access, consecutive rows in different bank groups).
static int tc_ystr(const Plan& p, int O2G) {
  int w = (O2G * p.c.O3 + 3) / 4;
  if ((w & 1) == 0) ++w;
  return 4 * w;
}

static TcSmem tc_smem(const Plan& p, int O2G, int NA2, int NA3, int NB1, int NB3) {
  const MmaLayout& m = p.m;
  const TcLayout& t = p.t;
  TcSmem s;
  s.a2_bytes = (size_t)ceil_div(m.K2P, 64) * 128 * 128;
  s.a3_bytes = (size_t)O2G * 128 * t.K3P * 2;
  s.a1_bytes = (size_t)128 * m.K1P * 2;
  const size_t b1 = (size_t)t.N1P * m.K1P * elem_size(p.dtype);
  const size_t b2 = (size_t)O2G * m.RP * m.K2P * 2;
  const size_t b3 = (size_t)t.N3P * t.K3P * 2;
  s.off_a2 = 0;
  s.off_b2 = s.off_a2 + NA2 * s.a2_bytes;
  s.off_a3 = align_up(s.off_b2 + b2, 128);
  s.off_a1 = align_up(s.off_a3 + NA3 * s.a3_bytes, 128);
  s.off_g1 = align_up(s.off_a1 + 2 * s.a1_bytes, 128);
  s.off_b3 = align_up(s.off_g1 + NB1 * b1, 128);
  const size_t main = s.off_b3 + NB3 * b3;
  // the partial y overlays the operands after the piece loop
  const size_t ys = (size_t)128 * tc_ystr(p, O2G) * 4;
  s.off_bar = align_up(std::max(main, ys), 128);
  s.total = s.off_bar + 512 + 1024;
  return s;
}

// tcgen05 operand layout (appended to the mma layout in the packed buffer).  O2 is split into
// NG groups so that a CTA's TMEM holds its S1/S2 accumulators and the S3 accumulators of its
// group (O2G x N3P columns) within 512 columns, and its operands fit in shared memory with
// single buffers.  Of the TMEM arrangements the one giving the widest groups wins (fewer
// groups: less repeated S1 work and fewer MMA instructions per call).  Needs RP <= 16 (one D1
// row per TMEM lane and at most 256 S1 columns) and I2 <= 128.
static void build_tc_layout(Plan* p) {
  const Canon& c = p->c;
  const MmaLayout& m = p->m;
  TcLayout& t = p->t;
  p->tc_ok = 0;
  if (m.RP > 16 || c.O1 > 128 || c.I2 > 128) return;
  t.N1P = ceil_div(c.O1 * m.RP, 16) * 16;
  t.N3P = ceil_div(c.O3, 16) * 16;
  t.K3P = std::max(16, m.RP);
  if (t.N1P > 256 || t.N3P > 256) return;
  const int step = (m.RP == 8) ? 2 : 1;  // S2's N = O2G * RP must be a multiple of 16
  // arrangement: 0 separate ND1 = 2, 1 shared, 2 separate ND1 = 1 (order of preference on ties)
  auto tmem_need = [&](int arr, int o2g) {
    const int n2 = o2g * m.RP, d3 = o2g * t.N3P;
    if (arr == 1) return 2 * std::max(t.N1P, n2) + d3;
    return (arr == 0 ? 2 : 1) * t.N1P + 2 * n2 + d3;
  };
  auto largest_group = [&](int arr) {
    int o2g = std::min(ceil_div(c.O2, step) * step, 256 / m.RP);
    o2g -= o2g % step;
    while (o2g >= step && tmem_need(arr, o2g) > 512) o2g -= step;
    while (o2g >= step && tc_smem(*p, o2g, 1, 1, 2, 4).total > p->smem_optin) o2g -= step;
    return o2g;
  };
  // balanced width of groups at most `o2g` wide: same group count, smallest width
  auto balanced = [&](int o2g) {
    int w = ceil_div(c.O2, ceil_div(c.O2, o2g));
    if (w % step) w += step - w % step;
    return std::min(w, o2g);
  };
  int best = -1, best_w = 0;
  for (int arr = 0; arr < 3; ++arr) {
    const int g = largest_group(arr);
    if (g < step) continue;
    if (balanced(g) > best_w) {
      best_w = balanced(g);
      best = arr;
    }
  }
  if (best < 0) return;
  t.O2G = best_w;
  t.NG = ceil_div(c.O2, t.O2G);
  t.N2 = t.O2G * m.RP;
  t.shared_d12 = best == 1;
  t.ND1 = best == 0 ? 2 : 1;
  t.DBW = std::max(t.N1P, t.N2);
  if (t.shared_d12) {
    t.d2_col = 0;
    t.d3_col = 2 * t.DBW;
  } else {
    t.d2_col = t.ND1 * t.N1P;
    t.d3_col = t.d2_col + 2 * t.N2;
  }
  t.tmem_cols = 32;
  while (t.tmem_cols < tmem_need(best, t.O2G)) t.tmem_cols *= 2;
  t.bytes_b1_slice = (size_t)t.N1P * m.K1P * elem_size(p->dtype);
  t.bytes_b2_group = (size_t)t.N2 * m.K2P * 2;
  t.bytes_b3_piece = (size_t)t.N3P * t.K3P * 2;
  t.off_b1 = align_up(m.off_g3 + m.bytes_g3, 256);
  t.off_b2 = align_up(t.off_b1 + (size_t)c.R * t.bytes_b1_slice, 256);
  t.off_b3 = align_up(t.off_b2 + (size_t)t.NG * t.bytes_b2_group, 256);
  p->tc_ok = p->mma_ok && t.tmem_cols <= 512;
}

// Shared memory of one slab-kernel CTA (ring_slab.cu), relative to a 1024-byte aligned base:
//   A2 slab slots x NA2 (128-byte swizzle, 64-wide K slabs of 128 rows), B2 of the group,
//   A3 x NA3 (S3 A operands of the group's o2), A1 x 2 (x slices), B1 slab slices x NB1,
//   B3 x NB3; reused after the piece loop as the CTA's fp32 partial y [128 rows x ystr];
//   then the mbarriers.  `total` includes 1 KB of slack for aligning the window.
struct SlabSmem {
  size_t a2_bytes, a3_bytes, a1_bytes;
  size_t off_a2, off_b2, off_a3, off_a1, off_g1, off_b3, off_bar, total;
};

static SlabSmem slab_smem(const Plan& p, const SlabLayout& l, int NA2, int NA3, int NB1,
                          int NB3) {
  const MmaLayout& m = p.m;
  SlabSmem s;
  s.a2_bytes = (size_t)ceil_div(l.KSL, 64) * 128 * 128;
  s.a3_bytes = (size_t)l.O2G * 128 * l.K3P * 2;
  s.a1_bytes = (size_t)128 * m.K1P * 2;
  const size_t b1 = (size_t)l.N1S * m.K1P * elem_size(p.dtype);
  const size_t b2 = (size_t)l.N2 * l.K2S * 2;
  const size_t b3 = (size_t)l.N3P * l.K3P * 2;
  s.off_a2 = 0;
  s.off_b2 = (size_t)NA2 * s.a2_bytes;
  s.off_a3 = align_up(s.off_b2 + b2, 128);
  s.off_a1 = align_up(s.off_a3 + NA3 * s.a3_bytes, 128);
  s.off_g1 = align_up(s.off_a1 + 2 * s.a1_bytes, 128);
  s.off_b3 = align_up(s.off_g1 + NB1 * b1, 128);
  const size_t main = s.off_b3 + NB3 * b3;
  const size_t ys = (size_t)128 * tc_ystr(p, l.O2G) * 4;  // partial y overlays the operands
  s.off_bar = align_up(std::max(main, ys), 128);
  s.total = s.off_bar + 1024 + 1024;
  return s;
}

// Which D2 depth the slab layout prefers: 0 the one giving fewer o2 groups (two buffers on a
// tie), 1 one buffer, 2 two buffers whenever a group fits with them.
#ifndef TRR_SLAB_D2_RULE
#define TRR_SLAB_D2_RULE 0
#endif

// Slab-kernel operand layout (appended after the other packed layouts).  The ring rank u of the
// first link is cut into NSL slabs of SW = 8 or 4 ranks.  O2 is split into NG groups so that a
// CTA's TMEM holds two D1 slab buffers (2 * O1 * SW columns), ND2 D2 buffers and the S3
// accumulators of its group within 512 columns, and its operands fit in shared memory.  Of the
// (SW, D2 depth) choices the one with the fewest groups wins (each group repeats S1 and C1):
// slabs of 4 halve D1 and so widen the groups where D1 binds TMEM (config 5: groups of 7 instead
// of 5); SW = 8 and two D2 buffers on ties (fewer slab steps; S2 of the next piece overlaps C2).
// The D2 depth follows TRR_SLAB_D2_RULE.  Needs ranks <= 32, O1 * SW <= 256 and fp16/bf16.
static void build_slab_layout(Plan* p) {
  const Canon& c = p->c;
  SlabLayout& l = p->sl;
  p->slab_ok = 0;
  if (p->dtype == TR_F32 || c.R > 32 || c.O1 > 32 || c.I2 > 128) return;
  SlabLayout best{};
  int best_need = 0;
  // slabs of 4 would halve D1 and widen the groups (config 5: 4 groups of 7 instead of 6 of 5),
  // but a slab step costs about the same whatever its size and they double the steps: measured
  // slower (config 5 28.8 against 26.3 ms at 8192 tokens, config 3 T = 256 8.1 against 6.1 ms),
  // so the layout keeps SW = 8 (the kernel handles both)
  for (int sw = 8; sw >= 8; sw /= 2) {
    SlabLayout t{};
    t.SW = sw;
    t.NSL = ceil_div(c.R, sw);
    t.RV = 8 * ceil_div(c.R, 8);
    t.N1S = ceil_div(c.O1 * sw, 16) * 16;
    t.KSL = ceil_div(c.I2 * sw, 16) * 16;
    t.K2S = t.NSL * t.KSL;
    t.N3P = ceil_div(c.O3, 16) * 16;
    t.K3P = std::max(16, ceil_div(t.RV, 16) * 16);
    if (t.N3P > 256 || t.N1S > 256) continue;
    // the last TMEM column a C1 warp reads (16-column loads from the start of its o1 half)
    const int h = (c.O1 + 1) / 2;
    const int c1_reach = t.N1S + std::max(ceil_div(h * sw, 16) * 16,
                                          h * sw + ceil_div((c.O1 - h) * sw, 16) * 16);
    const int step = (t.RV % 16 == 0) ? 1 : 2;  // S2's N = O2G * RV must be a multiple of 16
    auto tmem_need = [&](int nd2, int o2g) {
      return std::max(2 * t.N1S + nd2 * o2g * t.RV + o2g * t.N3P, c1_reach);
    };
    auto fits = [&](int nd2, int o2g) {
      SlabLayout u = t;
      u.O2G = o2g;
      u.N2 = o2g * t.RV;
      u.ND2 = nd2;
      return tmem_need(nd2, o2g) <= 512 && slab_smem(*p, u, 2, 1, 2, 4).total <= p->smem_optin;
    };
    for (int nd2 = 2; nd2 >= 1; --nd2) {
      if (TRR_SLAB_D2_RULE == 1 && nd2 == 2) continue;
      int o2g = std::min(ceil_div(c.O2, step) * step, 256 / t.RV);
      o2g -= o2g % step;
      while (o2g >= step && !fits(nd2, o2g)) o2g -= step;
      if (o2g < step) continue;
      int w = ceil_div(c.O2, ceil_div(c.O2, o2g));  // balanced width, same group count
      if (w % step) w += step - w % step;
      w = std::min(w, o2g);
      const int ng = ceil_div(c.O2, w);
      if (TRR_SLAB_D2_RULE == 2 && best.ND2 == 2 && best.SW == sw) continue;
      if (best.NG == 0 || ng < best.NG) {
        best = t;
        best.ND2 = nd2;
        best.O2G = w;
        best.NG = ng;
        best.N2 = w * t.RV;
        best_need = tmem_need(nd2, w);
      }
    }
  }
  if (best.NG == 0) return;
  l = best;
  l.d2_col = 2 * l.N1S;
  l.d3_col = l.d2_col + l.ND2 * l.N2;
  l.tmem_cols = 32;
  while (l.tmem_cols < best_need) l.tmem_cols *= 2;
  l.bytes_b1 = (size_t)l.N1S * p->m.K1P * elem_size(p->dtype);
  l.bytes_b2 = (size_t)l.N2 * l.K2S * 2;
  l.bytes_b3 = (size_t)l.N3P * l.K3P * 2;
  p->slab_ok = l.tmem_cols <= 512;
}

static void build_generic_layout(Plan* p) {
  const Canon& c = p->c;
  GenericLayout& g = p->g;
  const size_t es = elem_size(p->dtype);
  g.elems_g1 = (size_t)c.R * c.O1 * c.I1 * c.R;
  g.elems_g2 = (size_t)c.R * c.O2 * c.I2 * c.R;
  g.elems_g3 = (size_t)c.R * c.O3 * c.I3 * c.R;
  g.off_g1 = 0;
  g.off_g2 = align_up(g.elems_g1 * es, 256);
  g.off_g3 = align_up(g.off_g2 + g.elems_g2 * es, 256);
}

// Shared memory of one mma CTA:
//   [x tile NI3L x M1P x (K1P+8)] [2 x T1 M2P x (K2P+8)] [G2 fragments]
//   [G1+G3 fragments of each of the CTA's pieces] [raw x rows TT x d_in]
// reused after the piece loop as [partial y TT x d_out fp32], + 128 B flag word.
void mma_smem_layout(const Plan& p, MmaGeom* g) {
  const MmaLayout& m = p.m;
  const size_t es = 2;
  const size_t xs = align_up((size_t)g->NI3L * g->MT1 * 16 * (m.K1P + 8) * es, 128);
  const size_t t1 = align_up((size_t)g->MT2 * 16 * (m.K2P + 8) * 2, 128);
  const size_t g2 = g->g2_smem ? align_up(m.bytes_g2, 128) : 0;
  const size_t pf = g->pf_smem
      ? align_up((size_t)g->PPC * (m.KS1 * m.NT1 + m.KS3 * m.NT3) * 256, 128) : 0;
  const size_t xr = g->x_async ? align_up((size_t)g->TT * p.c.d_in * es, 128) : 0;
  g->off_t1 = xs;
  g->t1_stride = t1;
  g->off_g2 = xs + 2 * t1;
  g->off_pf = g->off_g2 + g2;
  g->off_xr = g->off_pf + pf;
  const size_t main = g->off_xr + xr;
  const size_t ys = (size_t)g->TT * p.c.d_out * 4;
  g->smem = align_up(std::max(main, ys), 128) + 128;  // + flag word area
}

// Largest count of distinct i3 values among the contiguous piece ranges of NJ CTAs.
static int max_i3_span(int npieces, int R, int NJ) {
  int best = 1;
  for (int j = 0; j < NJ; ++j) {
    const int pa = (int)((long long)j * npieces / NJ);
    const int pb = (int)((long long)(j + 1) * npieces / NJ);
    if (pb <= pa) continue;
    const int span = (pb - 1) / R - pa / R + 1;
    best = std::max(best, span);
  }
  return best;
}

// Split NJ-way piece parallelism into clusters of CL CTAs, NC <= 4 clusters per column of
// output tiles (`cols` columns; the last of a column's clusters adds their slots serially),
// keeping all cols * NC clusters co-resident (one wave): the most CTAs; on a tie one cluster
// per column, else the smaller cluster (when the cross-cluster slot reduction runs anyway,
// smaller clusters halve the partial sums each CTA gathers: c1 T = 8 measured 22.9 us with 4
// clusters of 8 against 25.5 us with 2 of 16).  Cluster sizes are powers of two up to cl_max.
static void one_wave_split(const Plan& p, long long cols, int NJ, int cl_max, int* CL, int* NC) {
  int best_cl = 1, best_nc = 1;
  long long best = 0;
  for (int cl = 16; cl >= 1; cl /= 2) {
    if (cl > cl_max || cl > NJ || cols > p.max_clusters[cl]) continue;
    const long long nc = std::max<long long>(
        1, std::min<long long>(std::min(NJ / cl, 4),
                               p.max_clusters[cl] / std::max(1LL, cols)));
    const long long ctas = cl * nc;
    const bool better = ctas > best || (ctas == best && best_nc > 1 && nc > 1);
    if (better) {
      best = ctas;
      best_cl = cl;
      best_nc = (int)nc;
    }
  }
  *CL = best_cl;
  *NC = best_nc;
}

// Split of the tcgen05 kernel's pieces: for each tile column (`cols` of them, `rows` rows
// (t, o1) each), CL CTAs per cluster and NC clusters, chosen among the splits whose cols * NC
// clusters are all co-resident (one wave) by an estimate of the device time that depends on
// the split, in microseconds:
//   * the longest piece range of a CTA times the cost of one piece's S1 -> C1 -> S2 -> C2 -> S3
//     chain, which the C1 conversion of N1P columns per row sets (0.9 us at 80 columns, 1.4 at
//     160 with D1 and D2 in shared TMEM buffers);
//   * 1 us when a CTA's range crosses an i3 boundary (a second x slice to stage);
//   * with NC > 1, 2 us for the cross-cluster slot pass plus the slot traffic of a CTA,
//     NC / CL of a tile's partial sums (1.4 us per 69 KB).
// At most 5 clusters per column.  Fitted to forced splits of the 1920 -> 2880 ring (R 8 and 16)
// at T = 4-32; against the earlier rule (most CTAs, at most 4 clusters per column, at least 5
// pieces per CTA) every split it changes on the benchmark and config-4 shapes measured equal or
// faster: c1 T = 8 -1.4 us, c2 T = 32 -2 us, config-4 k T = 8 -3.7 us, down T = 8 -9.7 us, gate
// T = 32 -14 us.
static void tc_split(const Plan& p, long long cols, int64_t rows, int* CL, int* NC) {
  const Canon& c = p.c;
  const MmaLayout& m = p.m;
  const TcLayout& t = p.t;
  const double piece_us =
      t.shared_d12 ? 1.4 : 0.5 + 0.005 * t.N1P;
  const double part_kb = (double)rows * t.O2G * c.O3 * 4 / 1024.0;
  double best = 1e30;
  *CL = 1;
  *NC = 1;
  for (int cl = 16; cl >= 1; cl /= 2) {
    if (cl > m.npieces || cols > p.max_clusters[cl]) continue;
    const long long nc_max =
        std::min<long long>(std::min<long long>(p.max_clusters[cl] / cols, m.npieces / cl), 5);
    for (int nc = 1; nc <= nc_max; ++nc) {
      const int NJ = cl * nc;
      double est = piece_us * ceil_div(m.npieces, NJ) +
                   1.0 * (max_i3_span(m.npieces, c.R, NJ) - 1);
      if (nc > 1) est += 2.0 + 1.4 * ((double)nc / cl) * part_kb / 67.5;
      if (est < best - 1e-9) {
        best = est;
        *CL = cl;
        *NC = nc;
      }
    }
  }
}

int resolve_mma_geom(const Plan& p, int64_t T, const tr_tiling* f, MmaGeom* g) {
  const Canon& c = p.c;
  const MmaLayout& m = p.m;
  if (!p.mma_ok) {
    set_error("mma.sync kernel does not support this spec/dtype");
    return TR_ERR_UNSUPPORTED;
  }
  // Compiled variants: (m16 row tiles per warp, max threads) = (1, 1024), (2, 512), (5, 384);
  // one warp per o2, so O2 bounds the row tiles a CTA can hold.
  const int mtw_max = c.O2 <= 12 ? 5 : (c.O2 <= 16 ? 2 : 1);
  const int maxrows = mtw_max * 16;
  int TT;
  if (f && f->tokens_per_tile > 0) {
    TT = f->tokens_per_tile;
  } else if (T * c.O1 <= 16) {
    TT = (int)T;
  } else {
    TT = std::max(1, maxrows / c.O1);
  }
  if (TT > T) TT = (int)T;
  if (TT < 1) TT = 1;
  const int MT2 = ceil_div(TT * c.O1, 16);
  if (MT2 > mtw_max) {
    set_error("tokens_per_tile=%d gives %d m16 tiles of S2 rows (max %d for O2=%d)", TT, MT2,
              mtw_max, c.O2);
    return TR_ERR_INVALID;
  }
  g->TT = TT;
  g->MT2 = MT2;
  g->MT1 = ceil_div(TT * c.I2, 16);
  g->MTW = MT2 <= 1 ? 1 : (MT2 <= 2 ? 2 : 5);
  g->ntiles = (int)((T + TT - 1) / TT);
  g->NW = c.O2;
  int CL, NC;
  if (f && f->cluster > 0) {
    CL = f->cluster;
    NC = f->clusters > 0 ? f->clusters : 1;
  } else {
    int NJ = g->ntiles >= p.num_sms ? 1 : std::max(1, p.num_sms / std::max(1, g->ntiles));
    NJ = std::min(NJ, m.npieces);
    one_wave_split(p, g->ntiles, NJ, 8, &CL, &NC);
  }
  if (CL < 1 || CL > 16 || NC < 1 || (long long)CL * NC > m.npieces) {
    set_error("cluster=%d clusters=%d invalid for %d pieces", CL, NC, m.npieces);
    return TR_ERR_INVALID;
  }
  g->CL = CL;
  g->NC = NC;
  g->NI3L = std::min(c.I3, max_i3_span(m.npieces, c.R, CL * NC));
  g->PPC = ceil_div(m.npieces, CL * NC);
  g->x_async = ((size_t)c.d_in * 2) % 16 == 0;
  g->g2_smem = 1;
  g->pf_smem = 1;
  mma_smem_layout(p, g);
  if (g->smem > p.smem_optin) {  // piece fragments too large to stage: read them from L2
    g->pf_smem = 0;
    mma_smem_layout(p, g);
  }
  if (g->smem > p.smem_optin) {  // G2 too large to stage: S2 reads it from L2
    g->g2_smem = 0;
    mma_smem_layout(p, g);
  }
  if (g->smem > p.smem_optin) {
    g->x_async = 0;
    mma_smem_layout(p, g);
  }
  if (g->smem > p.smem_optin) {
    set_error("mma kernel needs %zu bytes of shared memory (device allows %zu)", g->smem,
              p.smem_optin);
    return TR_ERR_UNSUPPORTED;
  }
  g->ws_bytes = 0;
  if (NC > 1) {
    const size_t counters = align_up((size_t)g->ntiles * CL * sizeof(int), 256);
    g->ws_bytes = counters + (size_t)g->ntiles * NC * TT * c.d_out * sizeof(float);
  }
  return TR_OK;
}

// Decode geometry: S2 rows (t, o1) fit one or two m16 tiles.  Clusters of CL CTAs split the
// pieces; NOC clusters split the output modes o2 into chunks of O2C (at most the compiled
// kernel's capacity: 4 with one row tile, 2 or 1 with two).
int resolve_decode_geom(const Plan& p, int64_t T, const tr_tiling* f, DecodeGeom* g) {
  const Canon& c = p.c;
  const MmaLayout& m = p.m;
  const int variant = decode_variant(p);
  if (!p.mma_ok || variant < 0 || T < 1 || T * c.O1 > 32) {
    set_error("decode kernel needs T*O1 <= 32, rank <= 16 and an fp16/bf16 plan");
    return TR_ERR_UNSUPPORTED;
  }
  g->MT2 = ceil_div((int)T * c.O1, 16);
  g->MT1 = ceil_div((int)T * c.I2, 16);
  if (g->MT1 > 2) {
    set_error("decode kernel: %lld tokens x %d S1 rows exceed two m16 tiles", (long long)T, c.I2);
    return TR_ERR_UNSUPPORTED;
  }
  int CL = (f && f->cluster > 0) ? f->cluster : std::min(16, m.npieces);
  if (!(f && f->cluster > 0)) {
    // one wave: smaller clusters when the fewest o2 chunks the compiled kernel allows do not
    // all fit on the device at once (2880 -> 1920 at R8: 8 chunks, but only 7 clusters of 16)
    const int noc_min = ceil_div(c.O2, decode_max_o2c(variant, g->MT2));
    while (CL > 1 && noc_min > p.max_clusters[CL]) CL = (CL + 1) / 2;
  }
  if (CL < 1 || CL > 16 || CL > m.npieces) {
    set_error("cluster=%d invalid for %d pieces", CL, m.npieces);
    return TR_ERR_INVALID;
  }
  // default: as many o2 chunks as clusters of CL CTAs fit on the device at once
  int NOC = (f && f->clusters > 0) ? f->clusters
                                   : std::max(1, std::min(c.O2, p.max_clusters[CL]));
  const int o2c_max = decode_max_o2c(variant, g->MT2);
  int O2C = ceil_div(c.O2, NOC);
  if (O2C > o2c_max) O2C = o2c_max;
  NOC = ceil_div(c.O2, O2C);
  const int maxw = decode_max_threads(variant, g->MT2) / 32;
  const int ppc = ceil_div(m.npieces, CL);
  g->CL = CL;
  g->NW = std::min(ppc, maxw);
  const size_t t1 = (size_t)16 * g->MT2 * (m.K2P + 8) * 2;
  const size_t yw = (size_t)16 * g->MT2 * o2c_max * m.O3P * 4;
  g->warp_bytes = align_up(std::max(t1, yw), 16);
  for (;;) {
    g->O2C = O2C;
    g->NOC = NOC;
    g->off_warps = align_up((size_t)m.KS2 * O2C * (m.RP / 8) * 256, 128);
    g->off_recv = align_up(g->off_warps + (size_t)g->NW * g->warp_bytes, 128);
    const size_t nout = (size_t)T * c.O1 * O2C * c.O3;
    const size_t slice = (nout + CL - 1) / CL;
    g->smem = align_up(g->off_recv + (size_t)CL * slice * 4, 128);
    if (g->smem <= p.smem_optin) break;
    if (g->NW > 4) {
      g->NW = std::max(4, g->NW / 2);
    } else if (O2C > 1) {
      O2C -= 1;
      NOC = ceil_div(c.O2, O2C);
    } else {
      set_error("decode kernel needs %zu bytes of shared memory", g->smem);
      return TR_ERR_UNSUPPORTED;
    }
  }
  return TR_OK;
}

// tcgen05 geometry: row tiles of TT tokens (TT*O1 <= 128), NG o2 groups, NJ = CL*NC CTAs over
// the pieces of each (tile, group).
int resolve_tc_geom(const Plan& p, int64_t T, const tr_tiling* f, TcGeom* g) {
  const Canon& c = p.c;
  const MmaLayout& m = p.m;
  const TcLayout& t = p.t;
  if (!p.tc_ok) {
    set_error("tcgen05 kernel does not support this spec/dtype");
    return TR_ERR_UNSUPPORTED;
  }
  // a row tile: TT tokens, TT*O1 rows (t, o1) of S2/S3 and TT*I2 rows (t, i2) of S1, each <= 128
  const int tt_max = std::max(1, std::min(128 / c.O1, 128 / c.I2));
  int TT = (f && f->tokens_per_tile > 0) ? f->tokens_per_tile : tt_max;
  if (TT > T) TT = (int)T;
  if (TT < 1) TT = 1;
  if (TT > tt_max) {
    set_error("tokens_per_tile=%d exceeds the 128-row tile (at most %d tokens: O1=%d, I2=%d)",
              TT, tt_max, c.O1, c.I2);
    return TR_ERR_INVALID;
  }
  g->TT = TT;
  g->ntiles = (int)((T + TT - 1) / TT);
  int CL, NC;
  if (f && f->cluster > 0) {
    CL = f->cluster;
    NC = f->clusters > 0 ? f->clusters : 1;
  } else {
    const long long cols = std::max<long long>(1, (long long)g->ntiles * t.NG);
    tc_split(p, cols, std::min<int64_t>(T, TT) * c.O1, &CL, &NC);
  }
  if (CL < 1 || CL > 16 || NC < 1 || (long long)CL * NC > m.npieces) {
    set_error("cluster=%d clusters=%d invalid for %d pieces", CL, NC, m.npieces);
    return TR_ERR_INVALID;
  }
  g->CL = CL;
  g->NC = NC;
  // buffer depths, deepest first: A2, A3 double; B1 all R slices, else a ring; B3 the CTA's
  // whole piece range (at most 64 pieces), else a ring of 16, 8 or 4
  const int NJ = CL * NC;
  const int max_np = (m.npieces + NJ - 1) / NJ;
  TcSmem sm{};
  bool fits = false;
  for (int na2 = 2; na2 >= 1 && !fits; --na2) {
    for (int na3 = 2; na3 >= 1 && !fits; --na3) {
      const int b1_opts[4] = {c.R, 4, 3, 2};
      for (int i1 = 0; i1 < 4 && !fits; ++i1) {
        const int nb1 = b1_opts[i1];
        if (i1 > 0 && nb1 >= c.R) continue;
        const int b3_opts[4] = {max_np, 16, 8, 4};
        for (int i3 = 0; i3 < 4 && !fits; ++i3) {
          const int nb3 = b3_opts[i3];
          if (i3 == 0 && max_np > 64) continue;
          if (i3 > 0 && nb3 >= max_np) continue;
          sm = tc_smem(p, t.O2G, na2, na3, nb1, nb3);
          if (sm.total <= p.smem_optin) {
            fits = true;
            g->NA2 = na2;
            g->NA3 = na3;
            g->NB1 = nb1;
            g->b1_all = nb1 >= c.R;
            g->NB3 = nb3;
            g->b3_all = i3 == 0;
          }
        }
      }
    }
  }
  if (!fits) {
    set_error("tcgen05 kernel needs %zu bytes of shared memory (device allows %zu)", sm.total,
              p.smem_optin);
    return TR_ERR_UNSUPPORTED;
  }
  g->ystr = tc_ystr(p, t.O2G);
  g->a2_bytes = sm.a2_bytes;
  g->a3_bytes = sm.a3_bytes;
  g->a1_bytes = sm.a1_bytes;
  g->off_a2 = sm.off_a2;
  g->off_b2 = sm.off_b2;
  g->off_a3 = sm.off_a3;
  g->off_a1 = sm.off_a1;
  g->off_g1 = sm.off_g1;
  g->off_b3 = sm.off_b3;
  g->off_bar = sm.off_bar;
  const size_t slot_elems = (size_t)128 * t.O2G * c.O3;
  // At least 120 KB, so no two CTAs share an SM: a CTA that holds TMEM and waits at the cluster
  // barrier must never block a cluster peer inside tcgen05.alloc on the same SM.
  g->smem = std::max<size_t>(sm.total, 120 * 1024);
  const size_t counters = align_up((size_t)g->ntiles * t.NG * CL * sizeof(int), 256);
  const size_t slots =
      NC > 1 ? align_up((size_t)g->ntiles * t.NG * NC * slot_elems * sizeof(float), 256) : 0;
  // CL > 1: every CTA's partial sums (rows (t, o1) of the tile x ystr floats) go through L2
  g->part_elems = (size_t)g->TT * c.O1 * g->ystr;
  g->parts_off = 256 + counters + slots;
  const size_t parts =
      CL > 1 ? (size_t)g->ntiles * t.NG * CL * NC * g->part_elems * sizeof(float) : 0;
  g->ws_bytes = g->parts_off + parts;
  return TR_OK;
}

// Split of the slab kernel's pieces for `cols` tile columns: CL CTAs per cluster and NC clusters
// per column (at most 5, or as many as fit one wave), by an estimate of the device time in
// microseconds:
//   waves x pieces per CTA x (NSL slab steps of about 1 us + 0.3 us), where a wave holds
//   max_clusters[CL] clusters (clusters of 8 fill 120 SMs of 148, of 4 132, of 2 all), plus with
//   NC > 1 the slot pass (2 us plus NC / CL of a tile's partial sums at 1.4 us per 69 KB) and
//   1 us per extra x slice of a CTA.
// Fitted to forced splits of config 3 (R32) at T = 1, 2 and 128 (160 columns: one CTA per column
// runs two waves, 4.25 ms; clusters of 4 or 2 x 2 slots, 2.7 ms).
static void slab_split(const Plan& p, long long cols, int64_t rows, int* CL, int* NC) {
  const Canon& c = p.c;
  const MmaLayout& m = p.m;
  const SlabLayout& l = p.sl;
  const double piece_us = 1.0 * l.NSL + 0.3;
  const double part_kb = (double)rows * l.O2G * c.O3 * 4 / 1024.0;
  // the slot pass is real traffic once the columns alone fill the device: at most 2 slots then
  const int nc_cap = cols >= p.num_sms ? 2 : 5;
  double best = 1e30, whole = 0.0;
  *CL = 1;
  *NC = 1;
  for (int cl = 16; cl >= 1; cl /= 2) {
    if (cl > m.npieces || p.max_clusters[cl] < 1) continue;
    // beyond nc_cap only as many clusters as still fit one wave (few columns, small T: config 3
    // at T = 1 and 8 measured 181 -> 161 us and 192 -> 174 us with 7 clusters of 2 against 3
    // of 4)
    const long long nc_wave = std::min<long long>(p.max_clusters[cl] / std::max(1LL, cols),
                                                  p.num_sms / std::max(1LL, cols * cl));
    const int nc_max = (int)std::min<long long>(std::max<long long>(nc_cap, nc_wave),
                                                m.npieces / cl);
    for (int nc = 1; nc <= nc_max; ++nc) {
      const int NJ = cl * nc;
      const long long waves = (cols * nc + p.max_clusters[cl] - 1) / p.max_clusters[cl];
      double est = (double)waves * ceil_div(m.npieces, NJ) * piece_us +
                   1.0 * (max_i3_span(m.npieces, c.R, NJ) - 1);
      if (nc > 1) est += 2.0 + 1.4 * ((double)nc / cl) * part_kb / 67.5;
      if (NJ == 1) whole = est;
      if (est < best - 1e-9) {
        best = est;
        *CL = cl;
        *NC = nc;
      }
    }
  }
  if (whole > 0.0 && whole <= 1.1 * best) {  // a split must gain at least 10%
    *CL = 1;
    *NC = 1;
  }
}

// Slab geometry: row tiles of TT tokens (TT*O1 and TT*I2 <= 128), NG o2 groups, NJ = CL*NC CTAs
// over the pieces of each (tile, group); the deepest operand rings that fit.
int resolve_slab_geom(const Plan& p, int64_t T, const tr_tiling* f, SlabGeom* g) {
  const Canon& c = p.c;
  const MmaLayout& m = p.m;
  const SlabLayout& l = p.sl;
  if (!p.slab_ok) {
    set_error("slab kernel does not support this spec/dtype");
    return TR_ERR_UNSUPPORTED;
  }
  const int tt_max = std::max(1, std::min(128 / c.O1, 128 / c.I2));
  int TT = (f && f->tokens_per_tile > 0) ? f->tokens_per_tile : tt_max;
  if (TT > T) TT = (int)T;
  if (TT < 1) TT = 1;
  if (TT > tt_max) {
    set_error("tokens_per_tile=%d exceeds the 128-row tile (at most %d tokens: O1=%d, I2=%d)",
              TT, tt_max, c.O1, c.I2);
    return TR_ERR_INVALID;
  }
  g->TT = TT;
  g->ntiles = (int)((T + TT - 1) / TT);
  int CL, NC;
  if (f && f->cluster > 0) {
    CL = f->cluster;
    NC = f->clusters > 0 ? f->clusters : 1;
  } else {
    const long long cols = std::max<long long>(1, (long long)g->ntiles * l.NG);
    slab_split(p, cols, std::min<int64_t>(T, TT) * c.O1, &CL, &NC);
  }
  if (CL < 1 || CL > 16 || NC < 1 || (long long)CL * NC > m.npieces) {
    set_error("cluster=%d clusters=%d invalid for %d pieces", CL, NC, m.npieces);
    return TR_ERR_INVALID;
  }
  g->CL = CL;
  g->NC = NC;
  const int NJ = CL * NC;
  const int max_np = ceil_div(m.npieces, NJ);
  SlabSmem sm{};
  bool ok = false;
  const int nb1_opts[4] = {c.R * l.NSL, 4, 3, 2};
  const int nb3_opts[4] = {max_np, 16, 8, 4};
  for (int na2 = 4; na2 >= 2 && !ok; --na2) {
    for (int na3 = 2; na3 >= 1 && !ok; --na3) {
      for (int i1 = 0; i1 < 4 && !ok; ++i1) {
        const int nb1 = nb1_opts[i1];
        if (i1 > 0 && nb1 >= c.R * l.NSL) continue;
        for (int i3 = 0; i3 < 4 && !ok; ++i3) {
          const int nb3 = nb3_opts[i3];
          if (i3 == 0 && max_np > 64) continue;
          if (i3 > 0 && nb3 >= max_np) continue;
          sm = slab_smem(p, l, na2, na3, nb1, nb3);
          if (sm.total <= p.smem_optin) {
            ok = true;
            g->NA2 = na2;
            g->NA3 = na3;
            g->NB1 = nb1;
            g->b1_all = i1 == 0;
            g->NB3 = nb3;
            g->b3_all = i3 == 0;
          }
        }
      }
    }
  }
  if (!ok) {
    set_error("slab kernel needs %zu bytes of shared memory (device allows %zu)", sm.total,
              p.smem_optin);
    return TR_ERR_UNSUPPORTED;
  }
  g->ystr = tc_ystr(p, l.O2G);
  g->a2_bytes = sm.a2_bytes;
  g->a3_bytes = sm.a3_bytes;
  g->a1_bytes = sm.a1_bytes;
  g->off_a2 = sm.off_a2;
  g->off_b2 = sm.off_b2;
  g->off_a3 = sm.off_a3;
  g->off_a1 = sm.off_a1;
  g->off_g1 = sm.off_g1;
  g->off_b3 = sm.off_b3;
  g->off_bar = sm.off_bar;
  // At least 120 KB, so no two CTAs share an SM: a CTA that holds TMEM and waits at the cluster
  // barrier must never block a cluster peer inside tcgen05.alloc on the same SM.
  g->smem = std::max<size_t>(sm.total, 120 * 1024);
  const size_t slot_elems = (size_t)128 * l.O2G * c.O3;
  const size_t counters = align_up((size_t)g->ntiles * l.NG * CL * sizeof(int), 256);
  const size_t slots =
      NC > 1 ? align_up((size_t)g->ntiles * l.NG * NC * slot_elems * sizeof(float), 256) : 0;
  g->part_elems = (size_t)g->TT * c.O1 * g->ystr;
  g->parts_off = 256 + counters + slots;
  const size_t parts =
      CL > 1 ? (size_t)g->ntiles * l.NG * CL * NC * g->part_elems * sizeof(float) : 0;
  g->ws_bytes = g->parts_off + parts;
  return TR_OK;
}

// Which kernel serves `T` tokens on this plan.
static int pick_kind(const Plan& p, int64_t T, const tr_tiling* f) {
  if (f && f->kernel != KIND_AUTO) return f->kernel;
  if (p.mma_ok) {
    DecodeGeom d;
    // the decode kernel while S2's rows (t, o1) fit two m16 tiles (and S1's rows two): at T = 2-3
    // on c1/c2 it takes half the tcgen05 kernel's time (c2 T = 2: 14.5 against 26.8 us cold)
    if (T >= 1 && T * p.c.O1 <= 32 && resolve_decode_geom(p, T, nullptr, &d) == TR_OK)
      return KIND_DECODE;
    // the slab kernel where the tcgen05 kernel does not take the spec (ranks above 16), or where
    // its layout needs at least a quarter fewer o2 groups (each group repeats S1 and C1): config
    // 4 q/o at T = 256 measured 363 us against 532 us; on equal groups the tcgen05 kernel's
    // whole-piece stages win (c2 T = 256: 187 us against 250 us)
    const bool slab_first =
        p.slab_ok && (!p.tc_ok || (long long)p.sl.NG * 4 <= (long long)p.t.NG * 3);
    TcGeom tg;
    SlabGeom sg;
    if (T >= 1 && slab_first && resolve_slab_geom(p, T, nullptr, &sg) == TR_OK) return KIND_SLAB;
    if (T >= 1 && p.tc_ok && resolve_tc_geom(p, T, nullptr, &tg) == TR_OK) return KIND_TC05;
    if (T >= 1 && p.slab_ok && resolve_slab_geom(p, T, nullptr, &sg) == TR_OK) return KIND_SLAB;
    return KIND_MMA;
  }
  return KIND_GENERIC;
}

}  // namespace trr

using namespace trr;

// The geometry the planner picks for a token count, cached per plan (the reference caches its
// tiling per T as well, tr_kernel.py:250-253): a forward call resolves it twice (workspace size,
// launch), and the tcgen05 planner walks buffer-depth options.  Only default tilings that
// resolved are cached; a small direct-mapped table keyed by T.
struct GeomCacheEntry {
  int64_t tokens = -1;
  int kind = 0;
  trr::MmaGeom g;
  trr::DecodeGeom dg;
  trr::TcGeom tg;
  trr::SlabGeom lg;
};

struct tr_plan : public trr::Plan {
  mutable std::mutex cache_mu;
  mutable GeomCacheEntry cache[32];
};

extern "C" {

const char* tr_status_string(int status) {
  switch (status) {
    case TR_OK: return "ok";
    case TR_ERR_INVALID: return "invalid argument";
    case TR_ERR_UNSUPPORTED: return "unsupported shape or dtype";
    case TR_ERR_WORKSPACE: return "workspace missing or too small";
    case TR_ERR_CUDA: return "CUDA error";
    case TR_ERR_ALIGN: return "misaligned pointer";
    case TR_ERR_TIMEOUT: return "device wait timed out";
    default: return "unknown status";
  }
}

const char* tr_last_error(void) { return g_last_error.c_str(); }

int tr_plan_create(const tr_spec* spec, int32_t dtype, int32_t device, tr_plan** out) {
  if (!spec || !out) {
    set_error("null spec or output pointer");
    return TR_ERR_INVALID;
  }
  *out = nullptr;
  for (int k = 0; k < 3; ++k) {
    if (spec->input_modes[k] <= 0 || spec->output_modes[k] <= 0) {
      set_error("All modes and the rank must be positive");
      return TR_ERR_INVALID;
    }
  }
  if (spec->rank <= 0) {
    set_error("All modes and the rank must be positive");
    return TR_ERR_INVALID;
  }
  if (dtype != TR_F32 && dtype != TR_F16 && dtype != TR_BF16) {
    set_error("unknown dtype %d", dtype);
    return TR_ERR_INVALID;
  }
  const long long din = (long long)spec->input_modes[0] * spec->input_modes[1] * spec->input_modes[2];
  const long long dout =
      (long long)spec->output_modes[0] * spec->output_modes[1] * spec->output_modes[2];
  if (din > (1LL << 30) || dout > (1LL << 30) || spec->rank > 4096) {
    set_error("spec too large (d_in=%lld d_out=%lld rank=%d)", din, dout, spec->rank);
    return TR_ERR_UNSUPPORTED;
  }
  tr_plan* p = new (std::nothrow) tr_plan();
  if (!p) {
    set_error("host allocation failed");
    return TR_ERR_INVALID;
  }
  p->spec = *spec;
  p->dtype = dtype;
  p->device = device;
  // cheapest order; ties keep the first in (X, Y) enumeration order
  double best = -1.0;
  int bx = 0, by = 1;
  for (int X = 0; X < 3; ++X) {
    for (int d = 1; d <= 2; ++d) {
      const int Y = (X + d) % 3;
      const int Z = 3 - X - Y;
      const double macs = order_macs(*spec, X, Y, Z);
      if (best < 0 || macs < best * (1.0 - 1e-12)) {
        best = macs;
        bx = X;
        by = Y;
      }
    }
  }
  build_canon(*spec, bx, by, &p->c);
  p->macs_per_token = best;
  build_mma_layout(p);
  build_generic_layout(p);
  p->mma_ok = (dtype != TR_F32) && spec->rank <= 32 && p->c.O2 <= 32 && p->m.O3P <= 32 &&
              p->c.O1 <= 80;
  int nsm = 148;
  int optin = 232448;
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) == cudaSuccess) {
    nsm = prop.multiProcessorCount;
    optin = (int)prop.sharedMemPerBlockOptin;
  } else {
    cudaGetLastError();  // no device here: plan with B200 defaults
  }
  p->num_sms = nsm;
  p->smem_optin = (size_t)optin;
  query_max_clusters(device, nsm, p->max_clusters);
  p->tc_ok = 0;
  p->slab_ok = 0;
  if (p->mma_ok) build_tc_layout(p);
  if (p->tc_ok) {
    p->packed_bytes =
        align_up(p->t.off_b3 + (size_t)p->m.npieces * p->t.bytes_b3_piece, 256);
  } else if (p->mma_ok) {
    p->packed_bytes = align_up(p->m.off_g3 + p->m.bytes_g3, 256);
  } else {
    p->packed_bytes = align_up(p->g.off_g3 + p->g.elems_g3 * elem_size(dtype), 256);
  }
  if (p->mma_ok) build_slab_layout(p);
  if (p->slab_ok) {  // the slab operands follow the others
    SlabLayout& l = p->sl;
    l.off_b1 = p->packed_bytes;
    l.off_b2 = align_up(l.off_b1 + (size_t)p->c.R * l.NSL * l.bytes_b1, 256);
    l.off_b3 = align_up(l.off_b2 + (size_t)l.NG * l.bytes_b2, 256);
    p->packed_bytes = align_up(l.off_b3 + (size_t)p->m.npieces * l.bytes_b3, 256);
  }
  *out = p;
  return TR_OK;
}

void tr_plan_destroy(tr_plan* plan) { delete plan; }

int tr_packed_bytes(const tr_plan* plan, size_t* bytes) {
  if (!plan || !bytes) {
    set_error("null argument");
    return TR_ERR_INVALID;
  }
  *bytes = plan->packed_bytes;
  return TR_OK;
}

int tr_plan_flops_per_token(const tr_plan* plan, double* flops) {
  if (!plan || !flops) {
    set_error("null argument");
    return TR_ERR_INVALID;
  }
  *flops = 2.0 * plan->macs_per_token;
  return TR_OK;
}

static int resolve_geom(const tr_plan* plan, int64_t tokens, const tr_tiling* tiling, int* kind,
                        MmaGeom* g, DecodeGeom* dg, TcGeom* tg, SlabGeom* lg);

static int geom_for(const tr_plan* plan, int64_t tokens, const tr_tiling* tiling, int* kind,
                    MmaGeom* g, DecodeGeom* dg, TcGeom* tg, SlabGeom* lg) {
  if (!plan) {
    set_error("null plan");
    return TR_ERR_INVALID;
  }
  if (tokens < 0) {
    set_error("negative token count");
    return TR_ERR_INVALID;
  }
  if (!tiling && tokens > 0) {
    std::lock_guard<std::mutex> lock(plan->cache_mu);
    const GeomCacheEntry& e = plan->cache[(uint64_t)tokens % 32];
    if (e.tokens == tokens) {
      *kind = e.kind;
      *g = e.g;
      *dg = e.dg;
      *tg = e.tg;
      *lg = e.lg;
      return TR_OK;
    }
  }
  const int st = resolve_geom(plan, tokens, tiling, kind, g, dg, tg, lg);
  if (st == TR_OK && !tiling && tokens > 0) {
    std::lock_guard<std::mutex> lock(plan->cache_mu);
    GeomCacheEntry& e = plan->cache[(uint64_t)tokens % 32];
    e.tokens = tokens;
    e.kind = *kind;
    e.g = *g;
    e.dg = *dg;
    e.tg = *tg;
    e.lg = *lg;
  }
  return st;
}

static int resolve_geom(const tr_plan* plan, int64_t tokens, const tr_tiling* tiling, int* kind,
                        MmaGeom* g, DecodeGeom* dg, TcGeom* tg, SlabGeom* lg) {
  *kind = pick_kind(*plan, tokens, tiling);
  if (*kind == KIND_MMA) {
    if (tokens == 0) {
      memset(g, 0, sizeof(*g));
      return TR_OK;
    }
    return resolve_mma_geom(*plan, tokens, tiling, g);
  }
  if (*kind == KIND_GENERIC) {
    memset(g, 0, sizeof(*g));
    return TR_OK;
  }
  if (*kind == KIND_DECODE) {
    memset(g, 0, sizeof(*g));
    if (tokens == 0) return TR_OK;
    return resolve_decode_geom(*plan, tokens, tiling, dg);
  }
  if (*kind == KIND_TC05) {
    memset(g, 0, sizeof(*g));
    memset(tg, 0, sizeof(*tg));
    if (tokens == 0) return TR_OK;
    return resolve_tc_geom(*plan, tokens, tiling, tg);
  }
  if (*kind == KIND_SLAB) {
    memset(g, 0, sizeof(*g));
    memset(lg, 0, sizeof(*lg));
    if (tokens == 0) return TR_OK;
    return resolve_slab_geom(*plan, tokens, tiling, lg);
  }
  set_error("kernel kind %d not available in this build", *kind);
  return TR_ERR_UNSUPPORTED;
}

int tr_workspace_bytes_tiled(const tr_plan* plan, int64_t tokens, const tr_tiling* tiling,
                             size_t* bytes) {
  if (!bytes) {
    set_error("null argument");
    return TR_ERR_INVALID;
  }
  int kind;
  MmaGeom g;
  DecodeGeom dg;
  TcGeom tg;
  SlabGeom lg;
  const int st = geom_for(plan, tokens, tiling, &kind, &g, &dg, &tg, &lg);
  if (st != TR_OK) return st;
  *bytes = kind == KIND_MMA    ? g.ws_bytes
           : kind == KIND_TC05 ? tg.ws_bytes
           : kind == KIND_SLAB ? lg.ws_bytes
                               : 0;
  return TR_OK;
}

int tr_workspace_bytes(const tr_plan* plan, int64_t tokens, size_t* bytes) {
  return tr_workspace_bytes_tiled(plan, tokens, nullptr, bytes);
}

int tr_workspace_clear(void* workspace, size_t bytes, void* stream) {
  if (bytes == 0) return TR_OK;
  if (!workspace) {
    set_error("null workspace");
    return TR_ERR_INVALID;
  }
  const cudaError_t e = cudaMemsetAsync(workspace, 0, bytes, (cudaStream_t)stream);
  if (e != cudaSuccess) {
    set_error("cudaMemsetAsync: %s", cudaGetErrorString(e));
    return TR_ERR_CUDA;
  }
  return TR_OK;
}

int tr_workspace_status(void* workspace, size_t workspace_bytes, int32_t* status, int32_t reset,
                        void* stream) {
  if (!status) {
    set_error("null status pointer");
    return TR_ERR_INVALID;
  }
  *status = TR_OK;
  if (workspace_bytes == 0) return TR_OK;  // the kernels of this token count keep no status
  if (!workspace || workspace_bytes < sizeof(int32_t)) {
    set_error("null workspace");
    return TR_ERR_INVALID;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int32_t word = 0;
  cudaError_t e = cudaMemcpyAsync(&word, workspace, sizeof(word), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e == cudaSuccess && reset && word != 0) e = cudaMemsetAsync(workspace, 0, sizeof(word), st);
  if (e != cudaSuccess) {
    set_error("reading the workspace status word: %s", cudaGetErrorString(e));
    return TR_ERR_CUDA;
  }
  *status = word;
  return TR_OK;
}

int tr_plan_set_wait_limit(tr_plan* plan, uint32_t polls) {
  if (!plan) {
    set_error("null plan");
    return TR_ERR_INVALID;
  }
  plan->wait_limit = polls;
  return TR_OK;
}

int tr_plan_tiling(const tr_plan* plan, int64_t tokens, tr_tiling* out) {
  if (!out) {
    set_error("null argument");
    return TR_ERR_INVALID;
  }
  int kind;
  MmaGeom g;
  DecodeGeom dg;
  TcGeom tg;
  SlabGeom lg;
  const int st = geom_for(plan, tokens, nullptr, &kind, &g, &dg, &tg, &lg);
  if (st != TR_OK) return st;
  out->kernel = kind;
  if (kind == KIND_TC05) {
    out->tokens_per_tile = tg.TT;
    out->cluster = tg.CL;
    out->clusters = tg.NC;
    return TR_OK;
  }
  if (kind == KIND_SLAB) {
    out->tokens_per_tile = lg.TT;
    out->cluster = lg.CL;
    out->clusters = lg.NC;
    return TR_OK;
  }
  if (kind == KIND_DECODE) {
    out->tokens_per_tile = (int32_t)tokens;
    out->cluster = dg.CL;
    out->clusters = dg.NOC;
    return TR_OK;
  }
  out->tokens_per_tile = g.TT;
  out->cluster = g.CL;
  out->clusters = g.NC;
  return TR_OK;
}

static int forward_impl(const tr_plan* plan, const void* packed, const void* x, int64_t tokens,
                        void* y, void* workspace, size_t workspace_bytes,
                        const tr_tiling* tiling, const Epi& epi, void* stream) {
  int kind;
  MmaGeom g;
  DecodeGeom dg;
  TcGeom tg;
  SlabGeom lg;
  int st = geom_for(plan, tokens, tiling, &kind, &g, &dg, &tg, &lg);
  if (st != TR_OK) return st;
  if (tokens == 0) return TR_OK;
  if (!packed || !x || !y) {
    set_error("null packed, x or y pointer");
    return TR_ERR_INVALID;
  }
  if (((uintptr_t)packed & 15) || ((uintptr_t)x & 15) || ((uintptr_t)y & 15)) {
    set_error("packed, x and y must be 16-byte aligned");
    return TR_ERR_ALIGN;
  }
  if (kind == KIND_GENERIC) return launch_generic(*plan, packed, x, tokens, y, stream, epi);
  if (kind == KIND_DECODE) return launch_decode(*plan, dg, packed, x, tokens, y, stream, epi);
  if (kind == KIND_SLAB) {
    if (!workspace || workspace_bytes < lg.ws_bytes) {
      set_error("workspace of %zu bytes needed, %zu given", lg.ws_bytes,
                workspace ? workspace_bytes : (size_t)0);
      return TR_ERR_WORKSPACE;
    }
    if ((uintptr_t)workspace & 15) {
      set_error("workspace must be 16-byte aligned");
      return TR_ERR_ALIGN;
    }
    return launch_slab(*plan, lg, packed, x, tokens, y, workspace, stream, epi);
  }
  if (kind == KIND_TC05) {
    if (!workspace || workspace_bytes < tg.ws_bytes) {
      set_error("workspace of %zu bytes needed, %zu given", tg.ws_bytes,
                workspace ? workspace_bytes : (size_t)0);
      return TR_ERR_WORKSPACE;
    }
    if ((uintptr_t)workspace & 15) {
      set_error("workspace must be 16-byte aligned");
      return TR_ERR_ALIGN;
    }
    return launch_tc05(*plan, tg, packed, x, tokens, y, workspace, stream, epi);
  }
  if (g.ws_bytes > 0) {
    if (!workspace || workspace_bytes < g.ws_bytes) {
      set_error("workspace of %zu bytes needed, %zu given", g.ws_bytes,
                workspace ? workspace_bytes : (size_t)0);
      return TR_ERR_WORKSPACE;
    }
    if ((uintptr_t)workspace & 15) {
      set_error("workspace must be 16-byte aligned");
      return TR_ERR_ALIGN;
    }
  }
  return launch_mma(*plan, g, packed, x, tokens, y, workspace, stream, epi);
}

int tr_forward_tiled(const tr_plan* plan, const void* packed, const void* x, int64_t tokens,
                     void* y, void* workspace, size_t workspace_bytes, const tr_tiling* tiling,
                     void* stream) {
  return forward_impl(plan, packed, x, tokens, y, workspace, workspace_bytes, tiling,
                      Epi{TR_EPI_NONE, 0, 0, nullptr}, stream);
}

int tr_forward_epilogue(const tr_plan* plan, const void* packed, const void* x, int64_t tokens,
                        void* y, const tr_epilogue* epilogue, void* workspace,
                        size_t workspace_bytes, const tr_tiling* tiling, void* stream) {
  if (!plan) {
    set_error("null plan");
    return TR_ERR_INVALID;
  }
  Epi epi{TR_EPI_NONE, 0, 0, nullptr};
  if (epilogue) {
    const tr_epilogue& e = *epilogue;
    if (e.kind != TR_EPI_NONE && e.kind != TR_EPI_ADD && e.kind != TR_EPI_SILU_MUL) {
      set_error("unknown epilogue kind %d", (int)e.kind);
      return TR_ERR_INVALID;
    }
    if (e.out_dtype != TR_F32 && e.out_dtype != plan->dtype) {
      set_error("epilogue output dtype %d: fp32 or the plan's dtype %d", (int)e.out_dtype,
                (int)plan->dtype);
      return TR_ERR_INVALID;
    }
    epi.kind = e.kind;
    epi.out_f32 = e.out_dtype == TR_F32;
    if (e.kind != TR_EPI_NONE) {
      if (e.aux_dtype != TR_F32 && e.aux_dtype != plan->dtype) {
        set_error("epilogue operand dtype %d: fp32 or the plan's dtype %d", (int)e.aux_dtype,
                  (int)plan->dtype);
        return TR_ERR_INVALID;
      }
      if (tokens > 0 && !e.aux) {
        set_error("null epilogue operand");
        return TR_ERR_INVALID;
      }
      if ((uintptr_t)e.aux & 15) {
        set_error("the epilogue operand must be 16-byte aligned");
        return TR_ERR_ALIGN;
      }
      epi.aux_f32 = e.aux_dtype == TR_F32;
      epi.aux = e.aux;
    }
  }
  return forward_impl(plan, packed, x, tokens, y, workspace, workspace_bytes, tiling, epi,
                      stream);
}

int tr_forward(const tr_plan* plan, const void* packed, const void* x, int64_t tokens, void* y,
               void* workspace, size_t workspace_bytes, void* stream) {
  return tr_forward_tiled(plan, packed, x, tokens, y, workspace, workspace_bytes, nullptr, stream);
}

int tr_forward_host(const tr_plan* plan, const void* packed, const void* x_host, int64_t tokens,
                    void* y_host, void* x_dev, void* y_dev, void* workspace,
                    size_t workspace_bytes, void* stream) {
  if (!plan) {
    set_error("null plan");
    return TR_ERR_INVALID;
  }
  if (tokens < 0) {
    set_error("negative token count");
    return TR_ERR_INVALID;
  }
  if (tokens == 0) return TR_OK;
  if (!x_host || !y_host || !x_dev || !y_dev) {
    set_error("null host buffer or device staging buffer");
    return TR_ERR_INVALID;
  }
  const size_t es = elem_size(plan->dtype);
  const size_t xb = (size_t)tokens * plan->c.d_in * es;
  const size_t yb = (size_t)tokens * plan->c.d_out * es;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(x_dev, x_host, xb, cudaMemcpyHostToDevice, st);
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_error("copy of x to the device: %s", cudaGetErrorString(e));
    return TR_ERR_CUDA;
  }
  const int s = tr_forward_tiled(plan, packed, x_dev, tokens, y_dev, workspace, workspace_bytes,
                                 nullptr, stream);
  if (s != TR_OK) return s;
  e = cudaMemcpyAsync(y_host, y_dev, yb, cudaMemcpyDeviceToHost, st);
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_error("copy of y to the host: %s", cudaGetErrorString(e));
    return TR_ERR_CUDA;
  }
  return TR_OK;
}

int tr_forward_noalloc(const tr_plan* plan, const void* packed, const void* x, int64_t tokens,
                       void* y, void* stream) {
  if (!plan) {
    set_error("null plan");
    return TR_ERR_INVALID;
  }
  if (tokens < 0) {
    set_error("negative token count");
    return TR_ERR_INVALID;
  }
  if (tokens == 0) return TR_OK;
  if (!plan->mma_ok) {
    set_error("the no-alloc entry point serves fp16/bf16 plans of the mma kernel");
    return TR_ERR_UNSUPPORTED;
  }
  if (!packed || !x || !y) {
    set_error("null packed, x or y pointer");
    return TR_ERR_INVALID;
  }
  if (((uintptr_t)packed & 15) || ((uintptr_t)x & 15) || ((uintptr_t)y & 15)) {
    set_error("packed, x and y must be 16-byte aligned");
    return TR_ERR_ALIGN;
  }
  return forward_noalloc(*plan, packed, x, tokens, y, stream);
}

int tr_pack_cores(const tr_plan* plan, const void* const cores[3], void* packed, void* stream) {
  if (!plan || !cores || !cores[0] || !cores[1] || !cores[2] || !packed) {
    set_error("null plan, core or packed pointer");
    return TR_ERR_INVALID;
  }
  if ((uintptr_t)packed & 15) {
    set_error("packed buffer must be 16-byte aligned");
    return TR_ERR_ALIGN;
  }
  return launch_pack(*plan, cores, packed, stream);
}

int tr_plan_describe(const tr_plan* plan, char* buf, size_t len) {
  if (!plan || !buf || len == 0) {
    set_error("null argument");
    return TR_ERR_INVALID;
  }
  const Canon& c = plan->c;
  const MmaLayout& m = plan->m;
  static const char* names = "ABC";
  const int n = snprintf(
      buf, len,
      "{\"order\": \"%c%c%c\", \"reversed\": %d, \"canonical_in\": [%d, %d, %d], "
      "\"canonical_out\": [%d, %d, %d], \"rank\": %d, \"macs_per_token\": %.0f, "
      "\"mma\": %d, \"rank_padded\": %d, \"pieces\": %d, \"packed_bytes\": %zu, "
      "\"dtype\": %d, \"tcgen05\": %d, \"o2_group\": %d, \"groups\": %d, "
      "\"tmem_cols\": %d, \"d1_buffers\": %d, \"shared_d12\": %d, \"slab\": %d, "
      "\"slab_o2_group\": %d, \"slab_groups\": %d, \"slab_d2_buffers\": %d, "
      "\"rank_slabs\": %d}",
      names[c.role[0]], names[c.role[1]], names[c.role[2]], c.reversed, c.I1, c.I2, c.I3, c.O1,
      c.O2, c.O3, c.R, plan->macs_per_token, plan->mma_ok, m.RP, m.npieces, plan->packed_bytes,
      plan->dtype, plan->tc_ok, plan->tc_ok ? plan->t.O2G : 0, plan->tc_ok ? plan->t.NG : 0,
      plan->tc_ok ? plan->t.tmem_cols : 0, plan->tc_ok ? plan->t.ND1 : 0,
      plan->tc_ok ? plan->t.shared_d12 : 0, plan->slab_ok, plan->slab_ok ? plan->sl.O2G : 0,
      plan->slab_ok ? plan->sl.NG : 0, plan->slab_ok ? plan->sl.ND2 : 0,
      plan->slab_ok ? plan->sl.NSL : 0);
  if (n < 0 || (size_t)n >= len) {
    set_error("buffer too small");
    return TR_ERR_INVALID;
  }
  return TR_OK;
}

}  // extern "C"
