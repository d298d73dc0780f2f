"""GPU parity of the slab kernel (ring_slab.cu): the tcgen05 kernel that cuts the ring rank into
slabs of eight and serves ranks up to 32 (config 3) and large token counts.

Forced with kernel=5 through the torch binding, against the reference's own outputs
(tests/golden: the required CUDA workloads, config 3 at T = 1, 2, 8) and the numpy oracle
(odd shapes, ranks that are not a multiple of 8, odd I2 and O2, every ring order); at the
config-3 token counts the oracle cannot finish quickly, sampled rows.  Every call is repeated
and must be bit-identical (ordered reductions), and the workspace status word must stay clear.
"""
from __future__ import annotations

import json

import numpy as np
import pytest
import torch

import oracle
from helpers import check_close
from kernel_task_b200 import abi, prepare_optimized
from kernel_task_b200 import spec as kspec

pytestmark = pytest.mark.gpu
DEV = "cuda"
SLAB = 5


def t(a, dtype):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV, dtype)


def ref_rows(x, cores, rows=None):
    xs = x if rows is None else x[rows]
    return oracle.tr_forward_reference(xs.float().cpu().numpy(),
                                       [c.float().cpu().numpy() for c in cores])


def run_slab(fn, x, TT=0, CL=0, NC=0):
    y1 = fn.call_tiled(x, SLAB, TT, CL, NC)
    y2 = fn.call_tiled(x, SLAB, TT, CL, NC)
    torch.testing.assert_close(y1, y2, rtol=0, atol=0)
    assert fn.workspace_status() == abi.TR_OK
    return y1


@pytest.mark.parametrize("R", [8, 16])
@pytest.mark.parametrize("geom", [(0, 0, 0), (0, 1, 1), (0, 8, 1), (0, 2, 3), (5, 3, 2),
                                  (1, 16, 1)])
def test_slab_required_workloads(golden, R, geom):
    """The reference's required CUDA cases (seed 23, x seed 41 + T) under forced splits."""
    key = f"req_r{R}"
    cores = tuple(t(golden[f"{key}_core{k}"], torch.float16) for k in range(3))
    fn = prepare_optimized(cores, kspec.TRSpec(rank=R))
    for T in (1, 8, 32):
        if f"{key}_x_t{T}" not in golden:
            continue
        x = t(golden[f"{key}_x_t{T}"], torch.float16)
        check_close(run_slab(fn, x, *geom), golden[f"{key}_yref_t{T}"], torch.float16)


def test_slab_config3_against_reference_vectors(golden_baseline):
    """Config 3 (R32, bf16) at the token counts the reference itself evaluated."""
    meta, vec = golden_baseline
    m = meta["c3"]
    s = kspec.SPEC_C3
    cores = kspec.baseline_cores(s, seed=m["core_seed"], dtype=torch.bfloat16, device=DEV)
    fn = prepare_optimized(cores, s)
    for T in m["tokens"]:
        x = torch.from_numpy(vec[f"c3_x_t{T}"]).view(torch.bfloat16).to(DEV)
        y = run_slab(fn, x)
        check_close(y, vec[f"c3_yref_t{T}"], torch.bfloat16)
        torch.testing.assert_close(fn(x), y, rtol=0, atol=0)  # the default path is this kernel


@pytest.mark.parametrize("T", [32, 128, 256])
def test_slab_config3_large_tokens_sampled(T):
    """Config 3 at the larger benchmark token counts: sampled rows against the oracle, and the
    rows independent of the batch they are computed in: the same rows alone, under the same
    split of the pieces (the split fixes the order of the fp32 sums), are bit-identical."""
    s = kspec.SPEC_C3
    cores = kspec.baseline_cores(s, seed=4, dtype=torch.bfloat16, device=DEV)
    fn = prepare_optimized(cores, s)
    x = kspec.baseline_x(s, T, seed=4, dtype=torch.bfloat16, device=DEV)
    geom = fn.tiling(T)
    assert geom["kernel"] == SLAB
    y = fn(x)
    assert fn.workspace_status() == abi.TR_OK
    rows = [0, 7, T // 2 + 1, T - 1]
    check_close(y[rows], ref_rows(x, cores, rows), torch.bfloat16)
    alone = fn.call_tiled(x[rows].contiguous(), SLAB, 0, geom["cluster"], geom["clusters"])
    torch.testing.assert_close(alone, y[rows], rtol=0, atol=0)


@pytest.mark.parametrize("name,T,dtype", [
    ("odd", 9, torch.float16), ("odd_cba", 31, torch.float16), ("odd_bac", 20, torch.float16),
    ("odd_cab", 17, torch.bfloat16), ("r12", 13, torch.float16), ("r20", 11, torch.bfloat16),
    ("r24", 7, torch.float16), ("r32_odd", 5, torch.bfloat16), ("i2_odd", 21, torch.float16),
    ("c5", 40, torch.bfloat16), ("c4_q", 24, torch.bfloat16), ("c4_k", 16, torch.bfloat16),
    ("c4_gate", 8, torch.bfloat16), ("c4_down", 9, torch.bfloat16), ("c1", 64, torch.float16),
    ("c2", 200, torch.float16)])
def test_slab_shapes_against_oracle(name, T, dtype):
    s = {"odd": kspec.TRSpec((2, 3, 4), (5, 6, 7), 3),
         "odd_cba": kspec.TRSpec((6, 5, 12), (7, 6, 9), 11),
         "odd_bac": kspec.TRSpec((5, 7, 6), (9, 3, 10), 13),
         "odd_cab": kspec.TRSpec((4, 6, 10), (6, 11, 7), 9),
         "r12": kspec.TRSpec((8, 12, 20), (12, 10, 24), 12),
         "r20": kspec.TRSpec((8, 10, 6), (6, 9, 14), 20),
         "r24": kspec.TRSpec((6, 8, 10), (10, 7, 12), 24),
         "r32_odd": kspec.TRSpec((6, 10, 8), (9, 5, 12), 32),
         "i2_odd": kspec.TRSpec((7, 9, 5), (6, 11, 13), 6),
         "c5": kspec.SPEC_C5, "c4_q": kspec.SPEC_C4["q"], "c4_k": kspec.SPEC_C4["k"],
         "c4_gate": kspec.SPEC_C4["gate"], "c4_down": kspec.SPEC_C4["down"],
         "c1": kspec.SPEC_C1, "c2": kspec.SPEC_C2}[name]
    cores = kspec.baseline_cores(s, seed=3, dtype=dtype, device=DEV)
    fn = prepare_optimized(cores, s)
    assert json.loads(fn.describe())["slab"] == 1
    x = kspec.baseline_x(s, T, seed=3, dtype=dtype, device=DEV)
    check_close(run_slab(fn, x), ref_rows(x, cores), dtype)


@pytest.mark.parametrize("name", ["c1", "c3"])
def test_slab_changing_tokens_one_workspace(name):
    """Token counts changing between calls on one prepared operator (the workspace grows and
    is left ready by every call), ragged last tiles included."""
    s, dtype = {"c1": (kspec.SPEC_C1, torch.float16),
                "c3": (kspec.SPEC_C3, torch.bfloat16)}[name]
    cores = kspec.baseline_cores(s, seed=6, dtype=dtype, device=DEV)
    fn = prepare_optimized(cores, s)
    for T in (3, 17, 1, 9, 33, 2):
        x = kspec.baseline_x(s, T, seed=6, dtype=dtype, device=DEV)
        rows = list(range(min(T, 3)))
        y = run_slab(fn, x)
        check_close(y[rows], ref_rows(x, cores, rows), dtype)


def test_slab_epilogues():
    """The fused epilogues on the slab kernel equal the fp32 output and torch's fp32 add /
    silu-mul rounded once, bit for bit."""
    s = kspec.SPEC_C3
    cores = kspec.baseline_cores(s, seed=8, dtype=torch.bfloat16, device=DEV)
    fn = prepare_optimized(cores, s)
    T = 16
    x = kspec.baseline_x(s, T, seed=8, dtype=torch.bfloat16, device=DEV)
    acc = fn.call_epilogue(x, abi.TR_EPI_NONE, None, True, SLAB)
    assert acc.dtype == torch.float32
    torch.testing.assert_close(fn.call_tiled(x, SLAB), acc.to(torch.bfloat16), rtol=0, atol=0)
    h = torch.randn(T, s.out_features, device=DEV).to(torch.bfloat16)
    add = fn.call_epilogue(x, abi.TR_EPI_ADD, h, False, SLAB)
    torch.testing.assert_close(add, (h.float() + acc).to(torch.bfloat16), rtol=0, atol=0)
    g = torch.randn(T, s.out_features, device=DEV)
    sm = fn.call_epilogue(x, abi.TR_EPI_SILU_MUL, g, False, SLAB)
    want = (g / (1 + torch.exp(-g)) * acc).to(torch.bfloat16)
    torch.testing.assert_close(sm.float(), want.float(), rtol=1e-2, atol=1e-3)


def test_slab_timeout_is_reported():
    """A one-poll wait limit makes the slab kernel's waits expire: the status word reports the
    timeout, and with the normal limit the next call on the same workspace is correct."""
    s = kspec.SPEC_C3
    cores = kspec.baseline_cores(s, seed=9, dtype=torch.bfloat16, device=DEV)
    fn = prepare_optimized(cores, s)
    x = kspec.baseline_x(s, 8, seed=9, dtype=torch.bfloat16, device=DEV)
    fn.set_wait_limit(1)
    fn.call_tiled(x, SLAB)
    assert fn.workspace_status(reset=True) == abi.TR_ERR_TIMEOUT
    fn.set_wait_limit(0)
    check_close(run_slab(fn, x), ref_rows(x, cores), torch.bfloat16)
