"""GPU parity: the CUDA kernels (through prepare_optimized -> torch binding -> C ABI, and through
the C ABI directly) against the reference's own outputs (tests/golden) and the numpy oracle.

Mirrors the reference's tests/test_correctness.py (CPU numerics with changing inputs and token
counts, independent prepared weights, the five required CUDA workloads) and its GPU sweeps
(tools/check_kernel.py: odd shapes, forced/ragged tilings, repeated calls on one workspace).
"""
from __future__ import annotations

import json

import numpy as np
import pytest
import torch

import oracle
from helpers import check_close, errors
from kernel_task_b200 import abi, prepare_optimized
from kernel_task_b200 import spec as kspec

pytestmark = pytest.mark.gpu
DEV = "cuda"


def t(a, dtype):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV, dtype)


def golden_cores(g, key, dtype):
    return tuple(t(g[f"{key}_core{k}"], dtype) for k in range(3))


@pytest.mark.parametrize("R,T", [(8, 1), (8, 8), (8, 32), (16, 1), (16, 32)])
def test_required_cuda_workloads(golden, R, T):
    """test_correctness.py:68-77 on the reference's vectors (fp16)."""
    key = f"req_r{R}"
    cores = golden_cores(golden, key, torch.float16)
    fn = prepare_optimized(cores, kspec.TRSpec(rank=R))
    x = t(golden[f"{key}_x_t{T}"], torch.float16)
    y = fn(x)
    torch.cuda.synchronize()
    assert y.shape == (T, 2880) and y.dtype == torch.float16 and y.device == x.device
    check_close(y, golden[f"{key}_yref_t{T}"], torch.float16)
    # repeated call: same bits (deterministic, workspace left clean)
    torch.testing.assert_close(fn(x), y, rtol=0, atol=0)


@pytest.mark.parametrize("si", range(3))
@pytest.mark.parametrize("seed", [0, 19])
def test_fp32_numerics_and_changing_inputs(golden, si, seed):
    """test_correctness.py:26-46 in fp32 on the GPU (generic fp32 kernel), one prepared object
    across changing values and token counts; inputs and cores stay unmodified."""
    key = f"cpu{si}_s{seed}"
    im, om, R = [((2, 3, 2), (2, 4, 3), 2), ((4, 4, 4), (4, 4, 4), 8),
                 ((4, 4, 4), (4, 4, 4), 16)][si]
    spec = kspec.TRSpec(im, om, R)
    cores = golden_cores(golden, key, torch.float32)
    orig = tuple(c.clone() for c in cores)
    fn = prepare_optimized(cores, spec)
    for n in range(4):
        x = t(golden[f"{key}_x{n}"], torch.float32)
        x0 = x.clone()
        y = fn(x)
        check_close(y, golden[f"{key}_y64_{n}"], torch.float32)
        check_close(y, golden[f"{key}_yref{n}"], torch.float32)
        torch.testing.assert_close(x, x0, rtol=0, atol=0)
        for c, o in zip(cores, orig):
            torch.testing.assert_close(c, o, rtol=0, atol=0)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_prepared_weights_are_independent(dtype):
    """test_correctness.py:49-65: calls a, b, a on two prepared weight sets."""
    spec = kspec.TRSpec((2, 3, 2), (2, 4, 3), 3)
    a = tuple(c.to(DEV, dtype) for c in kspec.make_cores(spec, seed=1))
    b = tuple(c.to(DEV, dtype) for c in kspec.make_cores(spec, seed=2))
    run_a, run_b = prepare_optimized(a, spec), prepare_optimized(b, spec)
    x = torch.randn(3, spec.in_features, generator=torch.Generator().manual_seed(7)).to(DEV, dtype)
    for run, w in [(run_a, a), (run_b, b), (run_a, a)]:
        ref = oracle.dense_forward(x.double().cpu().numpy(),
                                   oracle.materialize_dense_weight([c.double().cpu().numpy()
                                                                    for c in w]))
        check_close(run(x), ref, dtype)


@pytest.mark.parametrize("oi,ntok", [(0, 3), (1, 2), (2, 3), (3, 2)])
def test_odd_shapes_changing_tokens(golden, oi, ntok):
    """tools/check_kernel.py odd shapes (modes not multiples of the tile edges, R=3, R=16)."""
    key = f"odd{oi}"
    im, om, R = [((2, 3, 4), (5, 6, 7), 3), ((2, 3, 2), (2, 4, 3), 3),
                 ((4, 4, 4), (4, 4, 4), 16), ((8, 6, 20), (12, 5, 24), 16)][oi]
    fn = prepare_optimized(golden_cores(golden, key, torch.float16), kspec.TRSpec(im, om, R))
    for n in range(ntok):
        x = t(golden[f"{key}_x{n}"], torch.float16)
        for _ in range(2):
            check_close(fn(x), golden[f"{key}_yref{n}"], torch.float16)


# geometries: (tokens_per_tile, cluster, clusters); exercise the DSMEM reduction, the
# workspace-slot reduction, ragged last tiles and uneven piece ranges
TILINGS = [(1, 1, 1), (1, 16, 1), (1, 8, 3), (1, 3, 7), (2, 5, 2), (3, 4, 5), (8, 8, 2),
           (8, 1, 1), (5, 2, 1), (7, 8, 4)]


@pytest.mark.parametrize("R", [8, 16])
@pytest.mark.parametrize("tiling", TILINGS)
def test_forced_tilings(golden, R, tiling):
    key = f"req_r{R}"
    fn = prepare_optimized(golden_cores(golden, key, torch.float16), kspec.TRSpec(rank=R))
    TT, CL, NC = tiling
    for T in (1, 8, 32):
        if f"{key}_x_t{T}" not in golden:
            continue
        x = t(golden[f"{key}_x_t{T}"], torch.float16)
        y1 = fn.call_tiled(x, 2, TT, CL, NC)
        y2 = fn.call_tiled(x, 2, TT, CL, NC)
        check_close(y1, golden[f"{key}_yref_t{T}"], torch.float16)
        torch.testing.assert_close(y1, y2, rtol=0, atol=0)


# decode kernel geometries: (cluster = CTAs splitting the pieces, clusters = o2 chunks)
DECODE = [(16, 1), (16, 3), (8, 6), (4, 12), (1, 1), (16, 12), (5, 2), (3, 4)]


@pytest.mark.parametrize("R", [8, 16])
@pytest.mark.parametrize("geom", DECODE)
def test_decode_geometries(golden, R, geom):
    key = f"req_r{R}"
    fn = prepare_optimized(golden_cores(golden, key, torch.float16), kspec.TRSpec(rank=R))
    assert fn.tiling(1)["kernel"] == abi.KERNEL_DECODE
    x = t(golden[f"{key}_x_t1"], torch.float16)
    CL, NOC = geom
    y1 = fn.call_tiled(x, abi.KERNEL_DECODE, 1, CL, NOC)
    y2 = fn.call_tiled(x, abi.KERNEL_DECODE, 1, CL, NOC)
    check_close(y1, golden[f"{key}_yref_t1"], torch.float16)
    torch.testing.assert_close(y1, y2, rtol=0, atol=0)
    check_close(y1, fn.call_tiled(x, abi.KERNEL_MMA).double().cpu().numpy(), torch.float16)


@pytest.mark.parametrize("name,T", [("k", 1), ("k", 2), ("down", 1), ("gate", 1), ("q", 1)])
def test_decode_chain_layers(name, T):
    """Config-4 layer shapes in bf16 at decode sizes (k/v at T = 2 fills the m16 tile with two
    tokens and two S1 row tiles), against the oracle."""
    s = kspec.SPEC_C4[name]
    cores = kspec.baseline_cores(s, seed=5, dtype=torch.bfloat16, device=DEV)
    fn = prepare_optimized(cores, s)
    x = kspec.baseline_x(s, T, seed=5, dtype=torch.bfloat16, device=DEV)
    assert fn.tiling(T)["kernel"] == abi.KERNEL_DECODE
    ref = oracle.tr_forward_reference(x.float().cpu().numpy(),
                                      [c.float().cpu().numpy() for c in cores])
    check_close(fn(x), ref, torch.bfloat16)


# the decode kernel with two m16 tiles of S2 rows (16 < T*O1 <= 32): small decode batches on the
# benchmark shapes (fp16) and the config-4 q/gate layers (bf16), and odd shapes of several ring
# orders (run-time shapes)
DECODE2 = {
    "c1": (kspec.SPEC_C1, torch.float16), "c2": (kspec.SPEC_C2, torch.float16),
    "q": (kspec.SPEC_C4["q"], torch.bfloat16), "gate": (kspec.SPEC_C4["gate"], torch.bfloat16),
    "odd": (kspec.TRSpec((2, 3, 4), (5, 6, 7), 3), torch.float16),
    "odd_cba": (kspec.TRSpec((6, 5, 12), (7, 6, 9), 11), torch.float16),
    "odd_bac": (kspec.TRSpec((5, 7, 6), (9, 3, 10), 13), torch.bfloat16),
}


@pytest.mark.parametrize("name,T", [("c1", 2), ("c1", 3), ("c2", 2), ("c2", 3), ("q", 2),
                                    ("gate", 2), ("odd", 3), ("odd", 4), ("odd_cba", 2),
                                    ("odd_cba", 3), ("odd_bac", 6)])
@pytest.mark.parametrize("geom", [(0, 0), (16, 3), (4, 12), (5, 2)])
def test_decode_two_row_tiles(name, T, geom):
    s, dtype = DECODE2[name]
    cores = kspec.baseline_cores(s, seed=7, dtype=dtype, device=DEV)
    fn = prepare_optimized(cores, s)
    if geom[0] > json.loads(fn.describe())["pieces"]:
        pytest.skip("more CTAs per cluster than ring pieces")
    assert fn.tiling(T)["kernel"] == abi.KERNEL_DECODE
    x = kspec.baseline_x(s, T, seed=7 + T, dtype=dtype, device=DEV)
    CL, NOC = geom
    y1 = fn.call_tiled(x, abi.KERNEL_DECODE, T, CL, NOC)
    y2 = fn.call_tiled(x, abi.KERNEL_DECODE, T, CL, NOC)
    ref = oracle.tr_forward_reference(x.float().cpu().numpy(),
                                      [c.float().cpu().numpy() for c in cores])
    check_close(y1, ref, dtype)
    torch.testing.assert_close(y1, y2, rtol=0, atol=0)
    if geom == (0, 0):  # the fused residual add on the same path
        h = torch.randn(y1.shape, generator=torch.Generator().manual_seed(T)).to(DEV, dtype)
        add = fn.call_epilogue(x, abi.TR_EPI_ADD, h, False, abi.KERNEL_DECODE)
        y32 = fn.call_epilogue(x, abi.TR_EPI_NONE, None, True, abi.KERNEL_DECODE)
        torch.testing.assert_close(y32.to(dtype), y1, rtol=0, atol=0)
        torch.testing.assert_close(add, (h.float() + y32).to(dtype), rtol=0, atol=0)


def test_decode_rejects_three_row_tiles():
    s = kspec.SPEC_C1
    fn = prepare_optimized(kspec.baseline_cores(s, device=DEV), s)
    x = kspec.baseline_x(s, 4, device=DEV)  # 4 tokens x 10 rows (t, o1) > 32
    with pytest.raises(RuntimeError):
        fn.call_tiled(x, abi.KERNEL_DECODE, 4, 0, 0)


@pytest.mark.parametrize("name", ["c3", "c5", "c4_q", "c4_k", "c4_gate", "c4_down"])
def test_baseline_configs_bf16(golden_baseline, name):
    meta, vec = golden_baseline
    m = meta[name]
    s = kspec.TRSpec(tuple(m["input_modes"]), tuple(m["output_modes"]), m["rank"])
    cores = kspec.baseline_cores(s, seed=m["core_seed"], dtype=torch.bfloat16, device=DEV)
    fn = prepare_optimized(cores, s)
    for T in m["tokens"]:
        x = torch.from_numpy(vec[f"{name}_x_t{T}"]).view(torch.bfloat16).to(DEV)
        y = fn(x)
        assert y.dtype == torch.bfloat16
        check_close(y, vec[f"{name}_yref_t{T}"], torch.bfloat16)


def test_zero_tokens():
    s = kspec.SPEC_C1
    fn = prepare_optimized(kspec.baseline_cores(s, device=DEV), s)
    y = fn(torch.empty(0, s.in_features, device=DEV, dtype=torch.float16))
    assert y.shape == (0, s.out_features)


def test_wrong_inputs_raise():
    s = kspec.SPEC_C1
    fn = prepare_optimized(kspec.baseline_cores(s, device=DEV), s)
    with pytest.raises(ValueError):
        fn(torch.zeros(1, s.in_features + 1, device=DEV, dtype=torch.float16))
    with pytest.raises(ValueError):
        fn(torch.zeros(1, s.in_features, device=DEV, dtype=torch.float32))
    with pytest.raises(ValueError):
        fn(torch.zeros(1, s.in_features, dtype=torch.float16))


def test_non_contiguous_input():
    s = kspec.SPEC_C1
    fn = prepare_optimized(kspec.baseline_cores(s, device=DEV), s)
    big = kspec.baseline_x(s, 6, device=DEV)
    x = big[::2]
    torch.testing.assert_close(fn(x), fn(x.contiguous()), rtol=0, atol=0)


@pytest.mark.parametrize("s,T", [(kspec.SPEC_C1, 1000), (kspec.SPEC_C2, 257)])
def test_token_permutation_equivariance(s, T):
    """Tokens are independent: permuting the rows of x permutes y (size-independent check at
    sizes the oracle would be slow on)."""
    fn = prepare_optimized(kspec.baseline_cores(s, device=DEV), s)
    x = kspec.baseline_x(s, T, device=DEV)
    perm = torch.randperm(T, generator=torch.Generator().manual_seed(0)).to(DEV)
    y = fn(x)
    torch.testing.assert_close(fn(x[perm]), y[perm], rtol=0, atol=0)


def test_large_batch_against_oracle_sample():
    """c2 at T = 2048: every 97th row against the oracle, plus linearity of the whole batch."""
    s = kspec.SPEC_C2
    cores = kspec.baseline_cores(s, device=DEV)
    fn = prepare_optimized(cores, s)
    x = kspec.baseline_x(s, 2048, device=DEV)
    y = fn(x)
    rows = torch.arange(0, 2048, 97)
    ref = oracle.tr_forward_reference(x[rows].float().cpu().numpy(),
                                      [c.float().cpu().numpy() for c in cores])
    check_close(y[rows], ref, torch.float16)
    x2 = kspec.baseline_x(s, 2048, seed=5, device=DEV)
    e = errors(fn((x + x2) * 0.5), (y.double() + fn(x2).double()).cpu().numpy() * 0.5)
    assert e["rel_frob"] < 2e-3


def test_c_abi_direct_on_current_stream(golden):
    """The C ABI on torch-allocated buffers: pack, workspace sizing/clearing, forward on a
    side stream, and the workspace-too-small status."""
    key = "req_r8"
    cores = golden_cores(golden, key, torch.float16)
    plan = abi.Plan((8, 12, 20), (12, 10, 24), 8, abi.TR_F16, torch.cuda.current_device())
    packed = torch.empty(plan.packed_bytes(), dtype=torch.uint8, device=DEV)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        plan.pack([c.data_ptr() for c in cores], packed.data_ptr(), stream.cuda_stream)
        x = t(golden[f"{key}_x_t8"], torch.float16)
        y = torch.empty(8, 2880, dtype=torch.float16, device=DEV)
        tiling = abi.TrTiling(tokens_per_tile=4, cluster=4, clusters=3, kernel=abi.KERNEL_MMA)
        need = plan.workspace_bytes(8, tiling)
        assert need > 0
        ws = torch.empty(need, dtype=torch.uint8, device=DEV)
        abi.check(abi.lib().tr_workspace_clear(abi.ctypes.c_void_p(ws.data_ptr()), need,
                                               abi.ctypes.c_void_p(stream.cuda_stream)), "clear")
        st = plan.forward(packed.data_ptr(), x.data_ptr(), 8, y.data_ptr(), ws.data_ptr(),
                          need - 16, stream.cuda_stream, tiling)
        assert st == abi.TR_ERR_WORKSPACE
        for _ in range(3):
            st = plan.forward(packed.data_ptr(), x.data_ptr(), 8, y.data_ptr(), ws.data_ptr(),
                              need, stream.cuda_stream, tiling)
            assert st == abi.TR_OK
    stream.synchronize()
    check_close(y, golden[f"{key}_yref_t8"], torch.float16)


@pytest.mark.parametrize("R", [8, 16])
def test_forward_host_equals_device_call(golden, R):
    """forward_host (tr_forward_host: host x and y, device staging owned by the operator) gives
    the device call's y bit for bit, at every suite token count and with the staging reused
    across token counts; into a caller's page-locked `out` or a new one; the empty batch; and
    the reference's vectors."""
    key = f"req_r{R}"
    cores = golden_cores(golden, key, torch.float16)
    fn = prepare_optimized(cores, kspec.TRSpec(rank=R))
    for T in (32, 1, 8, 0):
        x = kspec.baseline_x(kspec.TRSpec(rank=R), T, seed=T, dtype=torch.float16, device=DEV)
        xh = x.cpu().pin_memory()
        out = torch.empty(T, 2880, dtype=torch.float16).pin_memory()
        y = fn.forward_host(xh, out)
        assert y.data_ptr() == out.data_ptr()
        y2 = fn.forward_host(xh)
        torch.cuda.synchronize()
        assert not y2.is_cuda and (T == 0 or y2.is_pinned())  # an empty tensor has no storage
        want = fn(x).cpu()
        torch.testing.assert_close(y, want, rtol=0, atol=0)
        torch.testing.assert_close(y2, want, rtol=0, atol=0)
    for T in (1, 8, 32):
        if f"{key}_x_t{T}" in golden:
            xh = torch.from_numpy(np.ascontiguousarray(golden[f"{key}_x_t{T}"])).half()
            y = fn.forward_host(xh.pin_memory())
            torch.cuda.synchronize()
            check_close(y, golden[f"{key}_yref_t{T}"], torch.float16)
    with pytest.raises(ValueError):
        fn.forward_host(torch.zeros(2, 1920, dtype=torch.float16, device=DEV))
    with pytest.raises(ValueError):
        fn.forward_host(torch.zeros(2, 1920, dtype=torch.float16),
                        torch.empty(3, 2880, dtype=torch.float16))


def test_forward_host_c_abi(golden):
    """tr_forward_host through ctypes with caller-owned staging on a side stream."""
    key = "req_r8"
    cores = golden_cores(golden, key, torch.float16)
    plan = abi.Plan((8, 12, 20), (12, 10, 24), 8, abi.TR_F16, torch.cuda.current_device())
    packed = torch.empty(plan.packed_bytes(), dtype=torch.uint8, device=DEV)
    stream = torch.cuda.Stream()
    xh = torch.from_numpy(np.ascontiguousarray(golden[f"{key}_x_t8"])).half().pin_memory()
    yh = torch.empty(8, 2880, dtype=torch.float16).pin_memory()
    xd = torch.empty(8, 1920, dtype=torch.float16, device=DEV)
    yd = torch.empty(8, 2880, dtype=torch.float16, device=DEV)
    with torch.cuda.stream(stream):
        plan.pack([c.data_ptr() for c in cores], packed.data_ptr(), stream.cuda_stream)
        need = plan.workspace_bytes(8)
        ws = torch.zeros(max(need, 16), dtype=torch.uint8, device=DEV)
        assert plan.forward_host(packed.data_ptr(), xh.data_ptr(), 8, yh.data_ptr(), 0,
                                 yd.data_ptr(), ws.data_ptr(), need,
                                 stream.cuda_stream) == abi.TR_ERR_INVALID
        for _ in range(2):
            st = plan.forward_host(packed.data_ptr(), xh.data_ptr(), 8, yh.data_ptr(),
                                   xd.data_ptr(), yd.data_ptr(), ws.data_ptr(), need,
                                   stream.cuda_stream)
            assert st == abi.TR_OK
    stream.synchronize()
    check_close(yh, golden[f"{key}_yref_t8"], torch.float16)


def test_generic_fp32_kernel_cross_checks_mma():
    """Independent GPU path: fp32 plan (generic CUDA-core kernel) on the fp16 values."""
    s = kspec.SPEC_C1
    cores = kspec.baseline_cores(s, device=DEV)
    x = kspec.baseline_x(s, 8, device=DEV)
    y16 = prepare_optimized(cores, s)(x)
    y32 = prepare_optimized(tuple(c.float() for c in cores), s)(x.float())
    ref = oracle.tr_forward_reference(x.float().cpu().numpy(), [c.float().cpu().numpy()
                                                                 for c in cores])
    check_close(y32, ref, torch.float32)
    check_close(y16, y32.double().cpu().numpy(), torch.float16)


# tcgen05 kernel (forced; planner geometry or (tokens_per_tile, cluster, clusters)): ragged
# row tiles, several o2 groups, DSMEM and workspace-slot reductions, one-piece CTAs
TC_GEOMS = [(0, 0, 0), (0, 1, 1), (0, 4, 0), (0, 16, 1), (0, 2, 3), (5, 3, 2), (1, 8, 2)]


@pytest.mark.parametrize("R", [8, 16])
@pytest.mark.parametrize("geom", TC_GEOMS)
def test_tcgen05_geometries(golden, R, geom):
    key = f"req_r{R}"
    fn = prepare_optimized(golden_cores(golden, key, torch.float16), kspec.TRSpec(rank=R))
    TT, CL, NC = geom
    for T in (8, 32):
        if f"{key}_x_t{T}" not in golden:
            continue
        x = t(golden[f"{key}_x_t{T}"], torch.float16)
        y1 = fn.call_tiled(x, abi.KERNEL_TC05, TT, CL, NC)
        y2 = fn.call_tiled(x, abi.KERNEL_TC05, TT, CL, NC)
        check_close(y1, golden[f"{key}_yref_t{T}"], torch.float16)
        torch.testing.assert_close(y1, y2, rtol=0, atol=0)
        assert fn.workspace[:4].view(torch.int32).item() == 0  # no bounded wait expired


@pytest.mark.parametrize("name,T,dtype", [
    ("odd", 9, torch.float16), ("odd_cba", 31, torch.float16), ("odd_bac", 20, torch.float16),
    ("odd_cab", 17, torch.bfloat16), ("c5", 16, torch.bfloat16), ("c4_q", 24, torch.bfloat16),
    ("c4_gate", 8, torch.bfloat16), ("c4_down", 9, torch.bfloat16), ("c2", 200, torch.float16)])
def test_tcgen05_shapes_against_oracle(name, T, dtype):
    s = {"odd": kspec.TRSpec((2, 3, 4), (5, 6, 7), 3),
         "odd_cba": kspec.TRSpec((6, 5, 12), (7, 6, 9), 11),
         "odd_bac": kspec.TRSpec((5, 7, 6), (9, 3, 10), 13),
         "odd_cab": kspec.TRSpec((4, 6, 10), (6, 11, 7), 9), "c5": kspec.SPEC_C5,
         "c4_q": kspec.SPEC_C4["q"], "c4_gate": kspec.SPEC_C4["gate"],
         "c4_down": kspec.SPEC_C4["down"], "c2": kspec.SPEC_C2}[name]
    cores = kspec.baseline_cores(s, seed=3, dtype=dtype, device=DEV)
    fn = prepare_optimized(cores, s)
    x = kspec.baseline_x(s, T, seed=3, dtype=dtype, device=DEV)
    y = fn.call_tiled(x, abi.KERNEL_TC05)
    assert fn.workspace[:4].view(torch.int32).item() == 0
    ref = oracle.tr_forward_reference(x.float().cpu().numpy(),
                                      [c.float().cpu().numpy() for c in cores])
    check_close(y, ref, dtype)
    torch.testing.assert_close(fn.call_tiled(x, abi.KERNEL_TC05), y, rtol=0, atol=0)


def test_tcgen05_unsupported_shape_raises():
    """O1 * RP above 256 S1 columns: the forced tcgen05 kernel reports UNSUPPORTED, the default
    path serves the spec with another kernel."""
    s = kspec.TRSpec((8, 6, 20), (12, 5, 24), 16)
    fn = prepare_optimized(kspec.baseline_cores(s, device=DEV), s)
    x = kspec.baseline_x(s, 40, device=DEV)
    with pytest.raises(RuntimeError):
        fn.call_tiled(x, abi.KERNEL_TC05)
    assert fn.tiling(40)["kernel"] != abi.KERNEL_TC05
    fn(x)


def test_sharded_ring_single_process_matches_operator():
    """ShardedRing without a process group is the whole operator (world 1): same bits."""
    from kernel_task_b200.shard import ShardedRing
    s = kspec.SPEC_C5
    cores = kspec.baseline_cores(s, seed=2, dtype=torch.bfloat16, device=DEV)
    op = ShardedRing(cores, s)
    x = kspec.baseline_x(s, 300, seed=2, dtype=torch.bfloat16, device=DEV)
    assert op.bounds(300) == (0, 300)
    y = op(x)
    torch.testing.assert_close(y, op(x, gather=True), rtol=0, atol=0)
    torch.testing.assert_close(y, prepare_optimized(cores, s)(x), rtol=0, atol=0)
    rows = torch.arange(0, 300, 37)
    ref = oracle.tr_forward_reference(x[rows].float().cpu().numpy(),
                                      [c.float().cpu().numpy() for c in cores])
    check_close(y[rows], ref, torch.bfloat16)


@pytest.mark.parametrize("T", [1, 2, 8, 32])
def test_c1_chain_down_layer(T):
    """The down layer of the 1920 -> 2880 -> 1920 chain (2880 -> 1920, (12,10,24)->(8,12,20),
    R8, order C,A,B; compiled as a fixed shape) on the kernel the planner picks, against the
    oracle, and the decode kernel's one-wave cluster split."""
    s = kspec.TRSpec((12, 10, 24), (8, 12, 20), 8)
    cores = kspec.baseline_cores(s, seed=11, dtype=torch.float16, device=DEV)
    fn = prepare_optimized(cores, s)
    x = kspec.baseline_x(s, T, seed=11, dtype=torch.float16, device=DEV)
    y = fn(x)
    check_close(y, oracle.tr_forward_reference(x.float().cpu().numpy(),
                                               [c.float().cpu().numpy() for c in cores]),
                torch.float16)
    torch.testing.assert_close(fn(x), y, rtol=0, atol=0)
    if T == 1:
        g = fn.tiling(1)
        assert g["kernel"] == abi.KERNEL_DECODE and g["cluster"] <= 8
