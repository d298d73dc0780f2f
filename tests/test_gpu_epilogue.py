"""GPU: the fused forward epilogues (fp32 output, residual add, SiLU-gated product) and the
reference's stand-alone consumers, on the config-4 decode chain shapes (bf16, rank 16).

Reference behaviour mirrored: PreparedTRKernel.accumulate (tr_kernel.py:230-243) returns y in
fp32; consume_silu_mul / consume_add (csrc/v3g/bind.cu:93-148) turn fp32 outputs into bf16 and
clear them; the model chain in tools/qwen_model_chain.py:123-130 runs gate/up -> silu*mul ->
down -> residual add.  Here the consumers also run inside the forward kernel's store.

Exactness: every kernel computes one fp32 value v per y element whatever is stored, so
  * the fp32 output equals the value the plain forward rounds (same bits after rounding);
  * the add epilogue equals torch's fp32 add of the same operands, rounded once (bit-exact);
  * the silu epilogue uses the fast exponential, so it is compared within 2 bf16 ulps.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch
import torch.nn.functional as F

import oracle
from helpers import check_close
from kernel_task_b200 import abi, consume_add, consume_silu_mul, prepare_optimized
from kernel_task_b200 import spec as kspec

pytestmark = pytest.mark.gpu
DEV = "cuda"
BF16_ULP2 = 2.0 ** -7  # two bf16 ulps, relative

# (layer, tokens, kernel, tokens_per_tile, cluster, clusters): the decode kernel (T*O1 <= 16),
# the tcgen05 and slab kernels with one and several clusters per tile (workspace-slot
# reduction), and the mma.sync kernel with a cross-cluster reduction
CASES = [
    ("q", 1, abi.KERNEL_DECODE, 1, 0, 0), ("gate", 1, abi.KERNEL_DECODE, 1, 0, 0),
    ("down", 1, abi.KERNEL_DECODE, 1, 0, 0), ("k", 2, abi.KERNEL_DECODE, 1, 16, 3),
    ("q", 8, abi.KERNEL_TC05, 0, 0, 0), ("gate", 24, abi.KERNEL_TC05, 0, 0, 0),
    ("down", 9, abi.KERNEL_TC05, 0, 2, 3), ("k", 33, abi.KERNEL_TC05, 0, 0, 0),
    ("q", 5, abi.KERNEL_MMA, 0, 0, 0), ("up", 3, abi.KERNEL_MMA, 1, 4, 5),
    ("q", 8, abi.KERNEL_SLAB, 0, 0, 0), ("down", 9, abi.KERNEL_SLAB, 0, 2, 3),
    ("gate", 40, abi.KERNEL_SLAB, 0, 0, 0),
]


def _layer(name, seed=11):
    s = kspec.SPEC_C4[name]
    cores = kspec.baseline_cores(s, seed=seed, dtype=torch.bfloat16, device=DEV)
    return s, cores, prepare_optimized(cores, s)


def _ref(x, cores):
    return oracle.tr_forward_reference(x.double().cpu().numpy(),
                                       [c.double().cpu().numpy() for c in cores])


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"{c[0]}-T{c[1]}-k{c[2]}-{c[4]}x{c[5]}")
def test_epilogues_match_unfused(case):
    name, T, kernel, TT, CL, NC = case
    s, cores, op = _layer(name)
    x = kspec.baseline_x(s, T, seed=T, dtype=torch.bfloat16, device=DEV)
    assert op.tiling(T)["kernel"] in (abi.KERNEL_DECODE, abi.KERNEL_TC05, abi.KERNEL_MMA,
                                      abi.KERNEL_SLAB)
    run = lambda kind, aux=None, f32=False: op.call_epilogue(x, kind, aux, f32, kernel, TT, CL,
                                                             NC)
    y16 = run(abi.TR_EPI_NONE)
    y32 = run(abi.TR_EPI_NONE, f32=True)
    assert y32.dtype == torch.float32 and y32.shape == (T, s.out_features)
    check_close(y32, _ref(x, cores), torch.bfloat16)
    torch.testing.assert_close(y32.to(torch.bfloat16), y16, rtol=0, atol=0)
    g = torch.randn(T, s.out_features, generator=torch.Generator().manual_seed(T)).to(DEV) * 2
    for aux in (g, g.to(torch.bfloat16)):
        a32 = aux.float()
        add = run(abi.TR_EPI_ADD, aux)
        assert add.dtype == torch.bfloat16
        torch.testing.assert_close(add, (a32 + y32).to(torch.bfloat16), rtol=0, atol=0)
        torch.testing.assert_close(run(abi.TR_EPI_ADD, aux, True), a32 + y32, rtol=0, atol=0)
        sm = run(abi.TR_EPI_SILU_MUL, aux)
        torch.testing.assert_close(sm.float(), (F.silu(a32) * y32).to(torch.bfloat16).float(),
                                   rtol=BF16_ULP2, atol=1e-30)
        torch.testing.assert_close(run(abi.TR_EPI_SILU_MUL, aux, True), F.silu(a32) * y32,
                                   rtol=1e-5, atol=1e-6)
    if kernel == abi.KERNEL_TC05:
        assert op.workspace[:4].view(torch.int32).item() == 0  # no bounded wait expired


@pytest.mark.parametrize("T", [1, 4, 40])
def test_gated_mlp_chain_fused_vs_reference_order(T):
    """Config-4 MLP block: gate/up -> silu*mul -> down -> residual add, fused (3 launches) and in
    the reference's order (accumulate x3 + two consumer launches), against the oracle."""
    torch.manual_seed(T)
    _, cg, gate = _layer("gate", 1)
    _, cu, up = _layer("up", 2)
    sd, cd, down = _layer("down", 3)
    x = kspec.baseline_x(kspec.SPEC_C4["gate"], T, seed=T, dtype=torch.bfloat16, device=DEV)
    h = torch.randn(T, sd.out_features, device=DEV).to(torch.bfloat16)
    # fused
    act = up.forward_silu_mul(x, gate.accumulate(x))
    h1 = down.forward_add(act, h)
    # the reference's order
    g32, u32 = gate.accumulate(x), up.accumulate(x)
    act2 = consume_silu_mul(g32, u32)
    assert not g32.any() and not u32.any()  # the consumer clears its fp32 inputs
    d32 = down.accumulate(act2)
    h2 = consume_add(h, d32)
    assert not d32.any()
    torch.testing.assert_close(act.float(), act2.float(), rtol=BF16_ULP2, atol=1e-30)
    # against the oracle: the activation from fp64 gate/up, the block output from the
    # activation the GPU produced (so bf16 rounding of the activation is not counted twice)
    gr, ur = _ref(x, cg), _ref(x, cu)
    act_ref = gr / (1 + np.exp(-gr)) * ur
    check_close(act, act_ref, torch.bfloat16)
    out_ref = h.double().cpu().numpy() + _ref(act, cd)
    check_close(h1, out_ref, torch.bfloat16)
    check_close(h2, out_ref, torch.bfloat16)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("n", [4, 1024, 3 * 14336, 4096 * 37])
def test_consumers_against_torch(dtype, n):
    gen = torch.Generator().manual_seed(n)
    g = (torch.randn(n, generator=gen) * 3).to(DEV)
    u = torch.randn(n, generator=gen).to(DEV)
    want = (F.silu(g) * u).to(dtype)
    gc, uc = g.clone(), u.clone()
    out = consume_silu_mul(gc, uc, dtype)
    assert out.dtype == dtype and not gc.any() and not uc.any()
    torch.testing.assert_close(out.float(), want.float(), rtol=BF16_ULP2, atol=1e-30)
    h = torch.randn(n, generator=gen).to(DEV, dtype)
    yc = u.clone()
    out = consume_add(h, yc)
    assert out.dtype == dtype and not yc.any()
    torch.testing.assert_close(out, (h.float() + u).to(dtype), rtol=0, atol=0)


def test_consumers_reject_bad_arguments():
    g = torch.zeros(6, device=DEV)
    with pytest.raises(ValueError):
        consume_silu_mul(g, g.clone())          # 6 % 4 != 0
    with pytest.raises(ValueError):
        consume_silu_mul(g[:4], torch.zeros(8, device=DEV))
    with pytest.raises(ValueError):
        consume_add(torch.zeros(4, device=DEV), torch.zeros(4, device=DEV))  # h fp32


def test_epilogue_argument_errors():
    s, _, op = _layer("q")
    x = kspec.baseline_x(s, 2, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(ValueError):
        op.forward_add(x, torch.zeros(3, s.out_features, device=DEV))     # wrong rows
    with pytest.raises(ValueError):
        op.forward_add(x, torch.zeros(2, s.out_features, device=DEV, dtype=torch.float16))
    with pytest.raises(ValueError):
        op.forward_silu_mul(x, torch.zeros(2, s.out_features))            # CPU operand
    with pytest.raises(ValueError):
        op.call_epilogue(x, 7, torch.zeros(2, s.out_features, device=DEV))
    assert op.forward_add(x[:0], torch.zeros(0, s.out_features, device=DEV)).shape == (0, 4096)


def test_c_abi_epilogue_in_place_residual():
    """tr_forward_epilogue through ctypes with y == aux (h += TR(x), in place)."""
    s, cores, op = _layer("down")
    plan = abi.Plan(s.input_modes, s.output_modes, s.rank, abi.TR_BF16)
    packed = torch.empty(plan.packed_bytes(), dtype=torch.uint8, device=DEV)
    plan.pack([c.data_ptr() for c in cores], packed.data_ptr(),
              torch.cuda.current_stream().cuda_stream)
    for T in (1, 16):
        x = kspec.baseline_x(s, T, seed=4, dtype=torch.bfloat16, device=DEV)
        h = torch.randn(T, s.out_features, device=DEV).to(torch.bfloat16)
        want = (h.float() + op.accumulate(x)).to(torch.bfloat16)
        ws = torch.zeros(max(plan.workspace_bytes(T), 16), dtype=torch.uint8, device=DEV)
        epi = abi.TrEpilogue(abi.TR_EPI_ADD, abi.TR_BF16, h.data_ptr(), abi.TR_BF16)
        st = plan.forward_epilogue(packed.data_ptr(), x.data_ptr(), T, h.data_ptr(), epi,
                                   ws.data_ptr(), ws.numel(),
                                   torch.cuda.current_stream().cuda_stream)
        assert st == abi.TR_OK
        torch.testing.assert_close(h, want, rtol=0, atol=0)
