// Operator shapes seen by the fused kernels.  Kernels are templated on a shape type and read
// every dimension through it (`sh.I1`, `sh.sx2`, ...):
//   * FixedShape<...>  -- a compiled benchmark shape: every dimension is a compile-time
//                         constant, loops unroll exactly and index arithmetic folds away;
//   * DynShape         -- any other spec: the same members as runtime values.
// The member set is the canonical ring of plan.h: G1 = core X (contracted first), G2 = core Y,
// G3 = core Z, plus the strides of their modes inside x and y rows.
#pragma once

#include <cstdint>

namespace trr {

constexpr int pick3(int k, int a, int b, int c) { return k == 0 ? a : (k == 1 ? b : c); }
constexpr int rank_pad(int r) { return r <= 8 ? 8 : (r <= 16 ? 16 : 32); }

struct DynShape {
  int I1, I2, I3, O1, O2, O3, R;
  int d_in, d_out;
  long long sx1, sx2, sx3, sy1, sy2, sy3;
  int KS1, NT1, K2P, KS2, NT2, O3P, NT3, npieces;
  int xm1, xm2, ym1, ym2;        // reference modes 1, 2 (mode 0 is implied)
  int role0, role1, role2;       // reference mode index of canonical mode 1, 2, 3
};

// (IN0, IN1, IN2) -> (ON0, ON1, ON2) at rank RR, contracted X first then Y.
template <int IN0, int IN1, int IN2, int ON0, int ON1, int ON2, int RR, int X, int Y>
struct FixedShape {
  static constexpr int Zc = 3 - X - Y;
  static constexpr int I1 = pick3(X, IN0, IN1, IN2);
  static constexpr int I2 = pick3(Y, IN0, IN1, IN2);
  static constexpr int I3 = pick3(Zc, IN0, IN1, IN2);
  static constexpr int O1 = pick3(X, ON0, ON1, ON2);
  static constexpr int O2 = pick3(Y, ON0, ON1, ON2);
  static constexpr int O3 = pick3(Zc, ON0, ON1, ON2);
  static constexpr int R = RR;
  static constexpr int RPc = rank_pad(RR);
  static constexpr int d_in = IN0 * IN1 * IN2;
  static constexpr int d_out = ON0 * ON1 * ON2;
  static constexpr long long sx1 = pick3(X, IN1 * IN2, IN2, 1);
  static constexpr long long sx2 = pick3(Y, IN1 * IN2, IN2, 1);
  static constexpr long long sx3 = pick3(Zc, IN1 * IN2, IN2, 1);
  static constexpr long long sy1 = pick3(X, ON1 * ON2, ON2, 1);
  static constexpr long long sy2 = pick3(Y, ON1 * ON2, ON2, 1);
  static constexpr long long sy3 = pick3(Zc, ON1 * ON2, ON2, 1);
  static constexpr int KS1 = (I1 + 15) / 16;
  static constexpr int NT1 = O1 * RPc / 8;
  static constexpr int K2P = (I2 * RPc + 15) / 16 * 16;
  static constexpr int KS2 = K2P / 16;
  static constexpr int NT2 = O2 * RPc / 8;
  static constexpr int O3P = (O3 + 7) / 8 * 8;
  static constexpr int NT3 = O3P / 8;
  static constexpr int npieces = I3 * RR;
  static constexpr int xm1 = IN1, xm2 = IN2, ym1 = ON1, ym2 = ON2;
  static constexpr int role0 = X, role1 = Y, role2 = Zc;
  static constexpr int in0 = IN0, in1 = IN1, in2 = IN2, on0 = ON0, on1 = ON1, on2 = ON2;
};

// The compiled benchmark shapes (order = the planner's cheapest ring order):
//   c1/c2  1920->2880 (8,12,20)->(12,10,24), R 8 / 16, order B,A,C
//   c4     4096-hidden decode-chain layers at R 16: q/o, k/v, gate/up (order A,B,C), down (C,B,A)
//   c1 down  2880->1920 (12,10,24)->(8,12,20), R 8, order C,A,B: the down layer of the
//            1920 -> 2880 -> 1920 chain (the reference's multi-layer comparison point)
#define TRR_FIXED_SHAPES(X)                  \
  X(8, 12, 20, 12, 10, 24, 8, 1, 0)          \
  X(8, 12, 20, 12, 10, 24, 16, 1, 0)         \
  X(16, 16, 16, 16, 16, 16, 16, 0, 1)        \
  X(16, 16, 16, 8, 8, 16, 16, 0, 1)          \
  X(16, 16, 16, 16, 28, 32, 16, 0, 1)        \
  X(16, 28, 32, 16, 16, 16, 16, 2, 1)        \
  X(12, 10, 24, 8, 12, 20, 8, 2, 0)

// The slab kernel also compiles the config-3 shape (rank 32, which the other tcgen05 kernel does
// not take).
#define TRR_SLAB_SHAPES(X) \
  TRR_FIXED_SHAPES(X)      \
  X(16, 16, 16, 16, 28, 32, 32, 0, 1)

}  // namespace trr
