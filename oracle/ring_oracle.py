"""TEST INFRASTRUCTURE ONLY -- numpy oracle of the tensor-ring operator (see oracle/__init__.py).

Index convention (reference.py:108-115): x t i j k; A a p i b; B b q j c; C c r k a; y t p q r.
Cores are [rank, output_mode, input_mode, rank]; x rows flatten (i, j, k) and y rows flatten
(p, q, r) row-major with the first mode slowest (reference.py:119,125).
"""
from __future__ import annotations

from typing import Sequence

import numpy as np


def _modes(cores):
    A, B, C = cores
    R = A.shape[0]
    return (A.shape[2], B.shape[2], C.shape[2]), (A.shape[1], B.shape[1], C.shape[1]), R


def tr_forward_reference(x: np.ndarray, cores: Sequence[np.ndarray],
                         dtype=np.float32) -> np.ndarray:
    """The reference's three pairwise contractions in its fixed order (reference.py:117-125):
        tijk,apib->tjkapb ; tjkapb,bqjc->tkapqc ; tkapqc,crka->tpqr
    evaluated with tensordot (BLAS) in `dtype` (float32 = the reference's CPU path)."""
    A, B, C = (np.asarray(c, dtype=dtype) for c in cores)
    (ni, nj, nk), (P, Q, Rr), _ = _modes((A, B, C))
    T = x.shape[0]
    X = np.asarray(x, dtype=dtype).reshape(T, ni, nj, nk)
    s1 = np.tensordot(X, A, axes=([1], [2]))                 # t j k | a p b
    s2 = np.tensordot(s1, B, axes=([1, 5], [2, 0]))          # t k a p | q c
    y = np.tensordot(s2, C, axes=([1, 5, 2], [2, 0, 3]))     # t p q | r
    return np.ascontiguousarray(y.reshape(T, P * Q * Rr))


def materialize_dense_weight(cores: Sequence[np.ndarray], dtype=np.float64) -> np.ndarray:
    """W[(p,q,r),(i,j,k)] = sum_{a,b,c} A[a,p,i,b] B[b,q,j,c] C[c,r,k,a] (reference.py:128-143).
    Validation only, small shapes."""
    A, B, C = (np.asarray(c, dtype=dtype) for c in cores)
    partial = np.einsum("apib,bqjc->apiqjc", A, B)
    W = np.einsum("apiqjc,crka->pqrijk", partial, C)
    P, Q, Rr, ni, nj, nk = W.shape
    return W.reshape(P * Q * Rr, ni * nj * nk)


def dense_forward(x: np.ndarray, W: np.ndarray) -> np.ndarray:
    """y = x W^T (reference.py:146-149)."""
    return np.asarray(x, dtype=W.dtype) @ W.T


def order_macs(input_modes, output_modes, rank, X: int, Y: int) -> float:
    """Multiply-adds per token when core X is contracted first, Y second, the third last:
    d_in*o_X*R^2 + i_Y*i_Z*o_X*o_Y*R^3 + d_out*i_Z*R^2."""
    Z = 3 - X - Y
    R = float(rank)
    din = float(np.prod(input_modes))
    dout = float(np.prod(output_modes))
    return (din * output_modes[X] * R * R
            + input_modes[Y] * input_modes[Z] * output_modes[X] * output_modes[Y] * R ** 3
            + dout * input_modes[Z] * R * R)


def reference_macs(input_modes, output_modes, rank) -> float:
    """Multiply-adds per token of the reference's own order (x.A -> .B -> .C)."""
    return order_macs(input_modes, output_modes, rank, 0, 1)


def order_forward(x: np.ndarray, cores: Sequence[np.ndarray], X: int, Y: int,
                  dtype=np.float64) -> np.ndarray:
    """The same operator contracted in ring order (X, Y, Z), written directly on the reference
    cores with einsum: an independent check that any of the six orders gives the reference's
    result (the product kernel picks the cheapest one)."""
    cores = [np.asarray(c, dtype=dtype) for c in cores]
    (ni, nj, nk), (P, Q, Rr), _ = _modes(cores)
    T = x.shape[0]
    X4 = np.asarray(x, dtype=dtype).reshape(T, ni, nj, nk)
    # subscripts per core: [left rank, out, in, right rank]
    sub = {0: "apib", 1: "bqjc", 2: "crka"}
    seq = (X, Y, 3 - X - Y)
    cur, val = "tijk", X4
    for n, k in enumerate(seq):
        s = sub[k]
        pending = "".join(sub[m] for m in seq[n + 1:])
        # keep output indices and indices a later core still needs; sum the rest
        out = "".join(ch for ch in dict.fromkeys(cur + s) if ch in "tpqr" or ch in pending)
        val = np.einsum(f"{cur},{s}->{out}", val, cores[k])
        cur = out
    y = np.einsum(f"{cur}->tpqr", val)
    return y.reshape(T, P * Q * Rr)
