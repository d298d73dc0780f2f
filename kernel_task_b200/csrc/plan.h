// Internal plan structures shared by the host planner (plan.cpp) and the kernels (*.cu).
//
// Canonical ring.  Any of the six contraction orders of the three-core ring is rewritten as
//     y[t,o1,o2,o3] = sum_{i1,i2,i3,s,u,v} x[t,i1,i2,i3] G1[s,o1,i1,u] G2[u,o2,i2,v] G3[v,o3,i3,s]
// and contracted as  S1: x.G1 over i1  ->  S2: .G2 over (i2,u)  ->  S3: .G3 over (i3,s,v).
// G1 is the reference core contracted first (role X), G2 the one sharing rank u with it (Y),
// G3 the last (Z).  When Y precedes X on the reference ring (A->B->C->A) every core's two rank
// axes are swapped while packing, so the kernels only ever see this one form.  The input and
// output modes of the canonical form are strided views of x and y.
#pragma once

#include <cstddef>
#include <cstdint>

#include "../../include/trring.h"

namespace trr {

struct Canon {
  int I1, I2, I3;          // canonical input modes  (x modes of cores X, Y, Z)
  int O1, O2, O3;          // canonical output modes (y modes of cores X, Y, Z)
  int R;                   // ring rank (all three links)
  int d_in, d_out;
  int64_t sx1, sx2, sx3;   // strides of i1,i2,i3 inside one x row
  int64_t sy1, sy2, sy3;   // strides of o1,o2,o3 inside one y row
  int role[3];             // reference core index playing X, Y, Z
  int reversed;            // 1: ring walked C->B->A (rank axes swapped while packing)
};

// Fragment-ordered operand layout of the mma.sync fused kernel (ring_mma.cu).  Every packed
// array stores, for each (k-step, n-tile) of an m16n8k16 B operand, the two 32-bit registers
// of all 32 lanes back to back (256 bytes), so a warp loads a B fragment with one coalesced
// 8-byte load per lane straight from L2 or shared memory.
struct MmaLayout {
  int RP;        // rank padded to the mma tile edge: 8, 16 or 32
  int K1P, KS1;  // S1 contraction (i1) padded to 16, and its k16 steps
  int NT1;       // S1 columns (o1,u): O1*RP/8 n8 tiles
  int K2P, KS2;  // S2 contraction (i2,u): I2*RP padded to 16, k16 steps
  int NT2;       // S2 columns (o2,v): O2*RP/8 n8 tiles
  int O3P, NT3;  // S3 columns o3 padded to 8, n8 tiles
  int KS3;       // S3 contraction v: RP/16 k16 steps (RP == 8 uses one m16n8k8 step)
  int npieces;   // I3 * R pieces (i3, s) summed into y
  size_t off_g1, off_g2, off_g3;  // byte offsets in the packed buffer
  size_t bytes_g1, bytes_g2, bytes_g3;
};

// Operand layout of the tcgen05 kernel (ring_tc05.cu): the UMMA B operands, K-major, no
// swizzle, 8x8 core matrices (8 rows x 16 bytes) with LBO = 128 B between the K chunks of a row
// group and SBO = K/8 * 128 B between row groups.
//   B1 per s:          rows (o1, u padded to RP) = N1P, K = K1P (i1)  (S1: G1[s,o1,i1,u], dtype E)
//   B2 per o2 group g: rows (o2 of g, v padded to RP) = N2, K = K2P  (S2: G2[u,o2,i2,v], fp16)
//   B3 per piece:      rows o3 padded to 16 = N3P, K = K3P (v padded to 16)  (S3: G3 slice, fp16)
// TMEM columns of a CTA, in one of two arrangements:
//   separate: D1 x ND1 [0, ND1 N1P), D2 x 2 [d2_col, d2_col + 2 N2), D3 [d3_col, + O2G N3P)
//   shared:   two buffers of DBW = max(N1P, N2) columns, each holding a piece's D1 and then, once
//             the converters have read it, the same piece's D2; D3 [d3_col, + O2G N3P)
struct TcLayout {
  int O2G;       // o2 modes per group (one CTA column of the grid)
  int NG;        // groups
  int shared_d12;  // 1: D1 and D2 share the two buffers
  int ND1;       // separate arrangement: S1 accumulators (1 or 2)
  int DBW;       // shared arrangement: buffer width
  int N1P;       // O1 * RP padded to 16 (S1 N, D1 TMEM columns)
  int N2;        // O2G * RP  (S2 N, D2 TMEM columns)
  int N3P;       // O3 padded to 16 (S3 N per o2)
  int K3P;       // RP padded to 16 (S3 K)
  int d2_col, d3_col;
  int tmem_cols; // power of two >= N1P + 2 N2 + O2G N3P
  size_t off_b1, bytes_b1_slice;
  size_t off_b2, bytes_b2_group;
  size_t off_b3, bytes_b3_piece;
};

// Operand layout of the slab kernel (ring_slab.cu): the ring rank u of the first link in NSL
// slabs of SW = 8 or 4 ranks (u = SW sl + ul), K-major, no swizzle, 8x8 core matrices as above.
//   B1 per (s, sl):   rows (o1, ul) padded to 16 = N1S, K = K1P (i1)    (S1, dtype E)
//   B2 per o2 group:  rows (o2 of group, v padded to RV) = N2, K = K2S = NSL * KSL ordered
//                     (sl, i2, ul), each slab's run padded to KSL = I2*SW rounded up to 16 (fp16)
//   B3 per piece:     rows o3 padded to 16 = N3P, K = K3P (v padded to 16)   (S3, fp16)
// TMEM columns of a CTA: D1 x 2 slabs [0, 2 N1S), D2 x ND2 [d2_col, + ND2 N2),
// D3 [d3_col, + O2G N3P).
struct SlabLayout {
  int SW;        // ranks per slab: 8 or 4
  int NSL;       // rank slabs
  int RV;        // the rank padded to a multiple of 8 (v, the S2 columns per o2)
  int N1S;       // O1 * SW padded to 16: S1 N per slab, D1 columns per slab buffer
  int KSL;       // I2 * SW padded to 16: S2 K per slab
  int K2S;       // NSL * KSL
  int O2G, NG;   // o2 modes per group, groups
  int N2;        // O2G * RV (S2 N, D2 columns)
  int ND2;       // D2 buffers (2: S2 of the next piece overlaps C2; 1: wider groups)
  int N3P;       // O3 padded to 16 (S3 N per o2)
  int K3P;       // RV padded to 16 (S3 K)
  int d2_col, d3_col;
  int tmem_cols;
  size_t off_b1, bytes_b1;  // per (s, slab)
  size_t off_b2, bytes_b2;  // per o2 group
  size_t off_b3, bytes_b3;  // per piece
};

// Canonical cores in natural [l][o][i][r] order (generic CUDA-core kernel, ring_generic.cu).
struct GenericLayout {
  size_t off_g1, off_g2, off_g3;
  size_t elems_g1, elems_g2, elems_g3;
};

enum KernelKind {
  KIND_AUTO = 0,
  KIND_GENERIC = 1,
  KIND_MMA = 2,
  KIND_TC05 = 3,
  KIND_DECODE = 4,
  KIND_SLAB = 5
};

struct Plan {
  tr_spec spec;
  int dtype;
  int device;
  Canon c;
  double macs_per_token;  // chosen order, multiply-adds per token
  int mma_ok;             // the mma.sync kernel handles this shape and dtype
  int tc_ok;              // the tcgen05 kernel handles it (its operands are packed too)
  int slab_ok;            // the slab kernel handles it (its operands are packed too)
  MmaLayout m;
  TcLayout t;
  SlabLayout sl;
  GenericLayout g;
  size_t packed_bytes;
  int num_sms;
  size_t smem_optin;
  // max_clusters[c]: thread-block clusters of c CTAs that are co-resident on this device when
  // every CTA needs a whole SM (the case of every kernel here).  Cluster placement is limited
  // per GPC, so this is below num_sms / c: 7 clusters of 16 CTAs on a 148-SM B200.
  int max_clusters[17];
  // Polls of one bounded device-side wait before it gives up (0: the built-in limit, about a
  // second of spinning).  Set by tr_plan_set_wait_limit; tests shorten it to make waits expire.
  unsigned wait_limit;
};

// Fills out[c] (c = 1..16) for `device` by the CUDA occupancy query (cached per process);
// without a device, the figures of a 148-SM B200.
void query_max_clusters(int device, int num_sms, int out[17]);

// Geometry of one mma.sync launch (resolved from tr_tiling + the planner).
struct MmaGeom {
  int TT;        // tokens per row tile
  int ntiles;    // ceil(T / TT)
  int MT2;       // m16 tiles of S2/S3 rows (t,o1) per row tile
  int MT1;       // m16 tiles of S1 rows (t,i2) per row tile
  int MTW;       // compiled per-warp m16 tile capacity (>= MT2)
  int CL;        // CTAs per cluster
  int NC;        // clusters per row tile
  int NW;        // warps per CTA (= O2)
  int NI3L;      // largest number of distinct i3 values one CTA's pieces touch
  int PPC;       // most pieces one CTA handles
  int g2_smem;   // 1: G2 fragments staged in shared memory once per CTA
  int pf_smem;   // 1: every piece's G1/G3 fragments staged in shared memory up front
  int x_async;   // 1: x rows copied to shared memory asynchronously (rows 16-byte aligned)
  size_t off_t1, t1_stride, off_g2, off_pf, off_xr;  // shared-memory carve-up (bytes)
  size_t smem;   // dynamic shared memory bytes
  size_t ws_bytes;
};

// Geometry of one decode launch (ring_decode.cu): NOC clusters of CL CTAs of NW warps.
struct DecodeGeom {
  int CL;        // CTAs per cluster; they split the I3*R pieces
  int NOC;       // clusters = chunks of O2C output modes o2
  int O2C;       // o2 modes per cluster
  int NW;        // warps per CTA (one piece per warp at a time)
  int MT1;       // m16 tiles of S1 rows (t, i2): 1 or 2
  int MT2;       // m16 tiles of S2/S3 rows (t, o1): 1 or 2
  size_t warp_bytes;  // per-warp shared area (T1 tile, then the warp's partial Y)
  size_t off_warps;   // after the staged G2 chunk
  size_t off_recv;    // cluster-reduction receive slots, after the warp areas
  size_t smem;
};

// Geometry of one tcgen05 launch: row tiles of TT tokens (M = 128 rows (t, o1)) x NG o2
// groups x NJ = CL * NC CTAs splitting the pieces.
struct TcGeom {
  int TT, ntiles;
  int CL, NC;
  int NA2, NA3;        // depths of the A2 and A3 operand buffers
  int NB1, b1_all;     // B1 slots; b1_all: all R slices loaded once, else a ring of NB1
  int NB3, b3_all;     // B3 slots; b3_all: the CTA's whole piece range loaded once, else a ring
  int ystr;            // row stride (floats) of the partial y in shared memory
  size_t a2_bytes, a3_bytes, a1_bytes;
  size_t off_a2, off_b2, off_a3, off_a1, off_g1, off_b3, off_bar;
  size_t smem;
  size_t part_elems;   // floats of one CTA's partial sums in the workspace (CL > 1)
  size_t parts_off;    // workspace offset of the per-CTA partial sums
  size_t ws_bytes;
};

// Geometry of one slab-kernel launch: row tiles of TT tokens x NG o2 groups x NJ = CL * NC
// CTAs splitting the pieces.
struct SlabGeom {
  int TT, ntiles;
  int CL, NC;
  int NA2, NA3;        // A2 slab slots, A3 buffers
  int NB1, b1_all;     // B1 slab-slice slots; b1_all: all R * NSL slices loaded once
  int NB3, b3_all;     // B3 slots; b3_all: the CTA's whole piece range loaded once
  int ystr;            // row stride (floats) of the partial y in shared memory
  size_t a2_bytes, a3_bytes, a1_bytes;
  size_t off_a2, off_b2, off_a3, off_a1, off_g1, off_b3, off_bar;
  size_t smem;
  size_t part_elems;   // floats of one CTA's partial sums in the workspace (CL > 1)
  size_t parts_off;    // workspace offset of the per-CTA partial sums
  size_t ws_bytes;
};

// What a kernel writes for output element y[i] = v (v: the fp32 sum of the ring pieces):
//   kind 0: v;  kind 1: aux[i] + v (residual add);  kind 2: silu(aux[i]) * v (gated MLP);
// stored as fp32 when out_f32, else in the plan's element type.  aux is [T, d_out] row-major,
// fp32 when aux_f32, else the plan's element type.
struct Epi {
  int kind;
  int out_f32;
  int aux_f32;
  const void* aux;
};

// Implemented in plan.cpp
void set_error(const char* fmt, ...);
int resolve_mma_geom(const Plan& p, int64_t T, const tr_tiling* force, MmaGeom* g);
void mma_smem_layout(const Plan& p, MmaGeom* g);

// Implemented in ring_mma.cu / ring_generic.cu / pack.cu
int launch_pack(const Plan& p, const void* const cores[3], void* packed, void* stream);
int launch_generic(const Plan& p, const void* packed, const void* x, int64_t T, void* y,
                   void* stream, const Epi& epi);
int launch_mma(const Plan& p, const MmaGeom& g, const void* packed, const void* x, int64_t T,
               void* y, void* ws, void* stream, const Epi& epi);
int query_max_active_clusters(const Plan& p, const MmaGeom& g, int* n);
int forward_noalloc(const Plan& p, const void* packed, const void* x, int64_t T, void* y,
                    void* stream);
int resolve_decode_geom(const Plan& p, int64_t T, const tr_tiling* force, DecodeGeom* g);
int resolve_tc_geom(const Plan& p, int64_t T, const tr_tiling* force, TcGeom* g);
int launch_tc05(const Plan& p, const TcGeom& g, const void* packed, const void* x, int64_t T,
                void* y, void* ws, void* stream, const Epi& epi);
int resolve_slab_geom(const Plan& p, int64_t T, const tr_tiling* force, SlabGeom* g);
int launch_slab(const Plan& p, const SlabGeom& g, const void* packed, const void* x, int64_t T,
                void* y, void* ws, void* stream, const Epi& epi);
int decode_variant(const Plan& p);
int decode_max_threads(int variant, int mt2);
int decode_max_o2c(int variant, int mt2);
int launch_decode(const Plan& p, const DecodeGeom& g, const void* packed, const void* x,
                  int64_t T, void* y, void* stream, const Epi& epi);

}  // namespace trr
