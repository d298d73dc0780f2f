"""GPU: the small-T tcgen05 kernel (kernel 5: cores on the MMA's M side, tokens on N) against
the oracle, over the benchmark shapes at decode sizes, odd shapes of every ring order, forced
cluster splits (one CTA, DSMEM only, workspace slots) and the fused epilogues."""
from __future__ import annotations

import pytest
import torch

import oracle
from helpers import check_close
from kernel_task_b200 import abi, prepare_optimized
from kernel_task_b200 import spec as kspec

pytestmark = pytest.mark.gpu
DEV = "cuda"

SHAPES = {
    "c1": (kspec.SPEC_C1, torch.float16), "c2": (kspec.SPEC_C2, torch.float16),
    "c4_q": (kspec.SPEC_C4["q"], torch.bfloat16), "c4_k": (kspec.SPEC_C4["k"], torch.bfloat16),
    "c4_gate": (kspec.SPEC_C4["gate"], torch.bfloat16),
    "c4_down": (kspec.SPEC_C4["down"], torch.bfloat16),
    "odd": (kspec.TRSpec((2, 3, 4), (5, 6, 7), 3), torch.float16),
    "odd_cba": (kspec.TRSpec((6, 5, 12), (7, 6, 9), 11), torch.float16),
    "odd_bac": (kspec.TRSpec((5, 7, 6), (9, 3, 10), 13), torch.bfloat16),
    "odd_cab": (kspec.TRSpec((4, 6, 10), (6, 11, 7), 9), torch.float16),
}


def _setup(name, T, seed=4):
    s, dtype = SHAPES[name]
    cores = kspec.baseline_cores(s, seed=seed, dtype=dtype, device=DEV)
    fn = prepare_optimized(cores, s)
    x = kspec.baseline_x(s, T, seed=seed + T, dtype=dtype, device=DEV)
    ref = oracle.tr_forward_reference(x.float().cpu().numpy(),
                                      [c.float().cpu().numpy() for c in cores])
    return fn, x, ref, dtype


@pytest.mark.parametrize("name,T", [
    ("c1", 1), ("c1", 2), ("c1", 5), ("c2", 1), ("c2", 3), ("c4_q", 1), ("c4_q", 4),
    ("c4_k", 1), ("c4_k", 7), ("c4_gate", 1), ("c4_down", 1), ("c4_down", 2), ("odd", 1),
    ("odd", 6), ("odd_cba", 1), ("odd_bac", 2), ("odd_cab", 1), ("odd_cab", 9)])
def test_small_t_kernel_against_oracle(name, T):
    fn, x, ref, dtype = _setup(name, T)
    y = fn.call_tiled(x, abi.KERNEL_TCS)
    assert fn.workspace[:4].view(torch.int32).item() == 0  # no bounded wait expired
    check_close(y, ref, dtype)
    torch.testing.assert_close(fn.call_tiled(x, abi.KERNEL_TCS), y, rtol=0, atol=0)


# (cluster, clusters): one CTA for all pieces, DSMEM reductions of 2..16 CTAs, workspace
# slots across 2..7 clusters
GEOMS = [(1, 1), (2, 1), (16, 1), (4, 3), (16, 2), (3, 5), (8, 7)]


@pytest.mark.parametrize("name,T", [("c1", 1), ("c4_q", 1), ("c2", 2)])
@pytest.mark.parametrize("geom", GEOMS)
def test_small_t_kernel_cluster_splits(name, T, geom):
    fn, x, ref, dtype = _setup(name, T)
    CL, NC = geom
    y = fn.call_tiled(x, abi.KERNEL_TCS, 0, CL, NC)
    assert fn.workspace[:4].view(torch.int32).item() == 0
    check_close(y, ref, dtype)
    torch.testing.assert_close(fn.call_tiled(x, abi.KERNEL_TCS, 0, CL, NC), y, rtol=0, atol=0)


@pytest.mark.parametrize("name", ["c1", "c4_down"])
def test_small_t_kernel_epilogues(name):
    fn, x, ref, dtype = _setup(name, 1)
    y32 = fn.call_epilogue(x, abi.TR_EPI_NONE, None, True, abi.KERNEL_TCS)
    check_close(y32, ref, dtype)
    h = torch.randn(y32.shape, device=DEV).to(dtype)
    add = fn.call_epilogue(x, abi.TR_EPI_ADD, h, False, abi.KERNEL_TCS)
    torch.testing.assert_close(add, (h.float() + y32).to(dtype), rtol=0, atol=0)
