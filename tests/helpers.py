"""Shared tolerance checks of the parity tests.

Two acceptance rules are applied together for fp16/bf16 results:
  * the reference's: |y - ref| <= atol + rtol*|ref| with atol = rtol = 0.02 (fp16/bf16) or
    1e-4 (fp32)  (IMPLEMENTATION.md:30-36, benchmarks/benchmark.py:182-183);
  * the benchmark spec's: relative Frobenius error <= 2e-3 and
    max|y - ref| <= 1e-2 * max|ref|.
"""
from __future__ import annotations

import numpy as np
import torch

REL_FROB = 2e-3
MAX_ABS_FRAC = 1e-2


def errors(y, ref) -> dict:
    y = y.detach().double().cpu().numpy() if isinstance(y, torch.Tensor) else np.asarray(y, float)
    ref = np.asarray(ref.detach().double().cpu().numpy() if isinstance(ref, torch.Tensor) else ref,
                     dtype=np.float64)
    d = np.abs(y - ref)
    nref = np.linalg.norm(ref)
    return {"max_abs": float(d.max()) if d.size else 0.0,
            "rel_frob": float(np.linalg.norm(y - ref) / nref) if nref > 0 else float(
                np.linalg.norm(y - ref)),
            "ref_inf": float(np.abs(ref).max()) if ref.size else 0.0}


def check_close(y, ref, dtype: torch.dtype) -> dict:
    e = errors(y, ref)
    yv = y.detach().double().cpu() if isinstance(y, torch.Tensor) else torch.from_numpy(y)
    rv = torch.as_tensor(np.asarray(ref, dtype=np.float64))
    assert torch.isfinite(yv).all()
    tol = 1e-4 if dtype == torch.float32 else 2e-2
    torch.testing.assert_close(yv, rv, rtol=tol, atol=tol)
    if dtype != torch.float32 and e["ref_inf"] > 0:
        assert e["rel_frob"] <= REL_FROB, e
        assert e["max_abs"] <= MAX_ABS_FRAC * e["ref_inf"], e
    return e
