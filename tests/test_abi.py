"""CPU: the C-ABI library loads, exports every function include/trring.h declares, and its host
planner (validation, order choice, layouts, geometry, error codes) behaves; no kernel runs."""
from __future__ import annotations

import ctypes
import json
import re
import subprocess
from pathlib import Path

import pytest

import oracle
from kernel_task_b200 import abi
from kernel_task_b200 import spec as kspec

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "trring.h"


def declared_functions() -> set[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"^\s*(?:const\s+)?\w+\s*\*?\s*(tr_\w+)\s*\(", text, flags=re.M))


def test_header_declares_the_abi():
    names = declared_functions()
    assert {"tr_plan_create", "tr_plan_destroy", "tr_pack_cores", "tr_forward",
            "tr_workspace_bytes", "tr_packed_bytes"} <= names


def test_library_exports_every_declared_symbol():
    out = subprocess.run(["nm", "-D", "--defined-only", str(abi.LIBRARY)], check=True,
                         capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    missing = declared_functions() - exported
    assert not missing, f"declared in trring.h but not exported: {sorted(missing)}"
    # and ctypes can bind all of them with the prototypes abi.py uses
    lib = abi.lib()
    for name in declared_functions():
        assert hasattr(lib, name)
    assert set(abi.PROTOTYPES) == declared_functions()


def test_status_strings():
    lib = abi.lib()
    assert lib.tr_status_string(abi.TR_OK) == b"ok"
    assert b"workspace" in lib.tr_status_string(abi.TR_ERR_WORKSPACE)


@pytest.mark.parametrize("modes,rank", [(((0, 2, 2), (2, 2, 2)), 2), (((2, 2, 2), (2, -1, 2)), 2),
                                        (((2, 2, 2), (2, 2, 2)), 0)])
def test_invalid_spec_is_rejected(modes, rank):
    with pytest.raises(abi.AbiError) as e:
        abi.Plan(modes[0], modes[1], rank, abi.TR_F16)
    assert e.value.status == abi.TR_ERR_INVALID
    assert b"positive" in abi.lib().tr_last_error()


def test_unknown_dtype_is_rejected():
    with pytest.raises(abi.AbiError) as e:
        abi.Plan((2, 2, 2), (2, 2, 2), 2, 7)
    assert e.value.status == abi.TR_ERR_INVALID


def _best(s):
    best = None
    for X in range(3):
        for Y in range(3):
            if X != Y:
                m = oracle.order_macs(s.input_modes, s.output_modes, s.rank, X, Y)
                best = m if best is None else min(best, m)
    return best


@pytest.mark.parametrize("s", [kspec.SPEC_C1, kspec.SPEC_C2, kspec.SPEC_C3, kspec.SPEC_C5,
                               *kspec.SPEC_C4.values(), kspec.TRSpec((2, 3, 4), (5, 6, 7), 3)])
def test_planner_picks_the_cheapest_ring_order(s):
    plan = abi.Plan(s.input_modes, s.output_modes, s.rank, abi.TR_F16)
    assert plan.flops_per_token() == pytest.approx(2 * _best(s), rel=1e-12)
    d = json.loads(plan.describe())
    X, Y, Z = ("ABC".index(ch) for ch in d["order"])
    assert oracle.order_macs(s.input_modes, s.output_modes, s.rank, X, Y) == \
        pytest.approx(_best(s), rel=1e-12)
    assert d["canonical_in"] == [s.input_modes[X], s.input_modes[Y], s.input_modes[Z]]
    assert d["canonical_out"] == [s.output_modes[X], s.output_modes[Y], s.output_modes[Z]]
    assert d["reversed"] == (1 if Y == (X + 2) % 3 else 0)


def test_best_order_figures():
    """Per-token FLOPs of the chosen orders: c1 29.5 M, c2 196.6 M, c3 8120.2 M, c5 1090.5 M."""
    expect = {kspec.SPEC_C1: 29.49e6, kspec.SPEC_C2: 196.6e6, kspec.SPEC_C3: 8120.2e6,
              kspec.SPEC_C5: 1090.5e6, kspec.SPEC_C4["down"]: 1090.5e6,
              kspec.SPEC_C4["q"]: 604.0e6, kspec.SPEC_C4["k"]: 159.4e6}
    for s, f in expect.items():
        plan = abi.Plan(s.input_modes, s.output_modes, s.rank, abi.TR_BF16)
        assert plan.flops_per_token() == pytest.approx(f, rel=2e-3)


def test_packed_bytes_and_dtype_paths():
    s = kspec.SPEC_C1
    p16 = abi.Plan(s.input_modes, s.output_modes, s.rank, abi.TR_F16)
    p32 = abi.Plan(s.input_modes, s.output_modes, s.rank, abi.TR_F32)
    assert json.loads(p16.describe())["mma"] == 1
    assert json.loads(p32.describe())["mma"] == 0
    # fp32 keeps the canonical cores (one copy, 256-byte aligned arrays)
    assert s.factor_parameters * 4 <= p32.packed_bytes() <= s.factor_parameters * 4 + 3 * 256
    # fp16: the operand layouts of the mma.sync, tcgen05 and slab kernels, each padded to tile
    # edges; bounded, and no dense weight (far below d_in * d_out)
    assert p16.packed_bytes() < 8 * s.factor_parameters * 2
    assert p16.packed_bytes() < s.dense_parameters * 2 / 20


def test_geometry_and_workspace():
    s = kspec.SPEC_C1
    p = abi.Plan(s.input_modes, s.output_modes, s.rank, abi.TR_F16)
    t = p.tiling(1)
    assert t.kernel == abi.KERNEL_DECODE and t.tokens_per_tile == 1
    assert p.workspace_bytes(1) == 0          # the decode kernel reduces inside its clusters
    assert p.workspace_bytes(0) == 0
    for T in (2, 3):                             # two m16 tiles of rows (t, o1)
        assert p.tiling(T).kernel == abi.KERNEL_DECODE and p.workspace_bytes(T) == 0
    for T in (4, 8, 32, 33, 1000):
        t = p.tiling(T)
        assert t.kernel == abi.KERNEL_TC05       # tensor-core kernel once T * o1 > 32
        ws = p.workspace_bytes(T)
        assert ws >= 256                         # status word (+ counters)
        # per-CTA partial sums (cluster > 1) and slots across clusters (clusters > 1)
        assert (ws > 256 + 64 * 1024) == (t.cluster > 1 or t.clusters > 1)
        mma = abi.TrTiling(kernel=abi.KERNEL_MMA)
        assert p.workspace_bytes(T, mma) >= 0
    forced = abi.TrTiling(tokens_per_tile=2, cluster=4, clusters=3, kernel=abi.KERNEL_MMA)
    assert p.workspace_bytes(5, forced) > 0
    bad = abi.TrTiling(tokens_per_tile=2, cluster=17, clusters=1, kernel=abi.KERNEL_MMA)
    with pytest.raises(abi.AbiError) as e:
        p.workspace_bytes(5, bad)
    assert e.value.status == abi.TR_ERR_INVALID
    too_many = abi.TrTiling(tokens_per_tile=1, cluster=16, clusters=11, kernel=abi.KERNEL_MMA)
    with pytest.raises(abi.AbiError):   # 176 CTAs > 160 pieces
        p.workspace_bytes(1, too_many)


def test_decode_kernel_only_within_two_row_tiles():
    """The decode kernel serves T while T*O1 <= 32 and T*I2 <= 32 (two m16 tiles of S2 and S1
    rows); beyond that the tcgen05 kernel (config-4 k at T = 3: 48 S1 rows; down at T = 2: 56)."""
    cases = {(kspec.SPEC_C4["k"], 2): abi.KERNEL_DECODE, (kspec.SPEC_C4["k"], 3): abi.KERNEL_TC05,
             (kspec.SPEC_C4["down"], 1): abi.KERNEL_DECODE,
             (kspec.SPEC_C4["down"], 2): abi.KERNEL_TC05,
             (kspec.SPEC_C4["q"], 2): abi.KERNEL_DECODE, (kspec.SPEC_C2, 3): abi.KERNEL_DECODE,
             (kspec.SPEC_C2, 4): abi.KERNEL_TC05}
    for (s, T), kind in cases.items():
        p = abi.Plan(s.input_modes, s.output_modes, s.rank, abi.TR_BF16)
        assert p.tiling(T).kernel == kind, (s, T)


# clusters of 1/2/4/8/16 CTAs co-resident on a B200 (the planner's table without a device)
B200_CLUSTERS = {1: 148, 2: 74, 4: 33, 8: 15, 16: 7}


@pytest.mark.parametrize("name", ["c1", "c2", "q", "k", "gate", "down"])
def test_tcgen05_split_stays_in_one_wave(name):
    """Every default tcgen05 split keeps all its clusters co-resident (at most 5 per column) and
    gives each CTA at least one piece."""
    s = {"c1": kspec.SPEC_C1, "c2": kspec.SPEC_C2}.get(name) or kspec.SPEC_C4[name]
    p = abi.Plan(s.input_modes, s.output_modes, s.rank, abi.TR_BF16)
    d = json.loads(p.describe())
    for T in (2, 3, 8, 17, 32, 64, 200, 4096):
        t = p.tiling(T)
        if t.kernel != abi.KERNEL_TC05:
            continue
        cols = -(-T // t.tokens_per_tile) * d["groups"]
        assert 1 <= t.clusters <= 5 and t.cluster * t.clusters <= d["pieces"]
        if cols <= B200_CLUSTERS[1]:
            assert cols * t.clusters <= B200_CLUSTERS[t.cluster], (T, t.cluster, t.clusters)


def test_tcgen05_split_on_benchmark_shapes():
    """The splits measured fastest among forced splits on B200 (c1 T8: 5 clusters of 8; c2 T32:
    5 clusters of 4; c1 T32: one cluster of 16)."""
    want = {(kspec.SPEC_C1, 8): (8, 5), (kspec.SPEC_C2, 32): (4, 5), (kspec.SPEC_C1, 32): (16, 1)}
    for (s, T), (cl, nc) in want.items():
        t = abi.Plan(s.input_modes, s.output_modes, s.rank, abi.TR_F16).tiling(T)
        assert (t.kernel, t.cluster, t.clusters) == (abi.KERNEL_TC05, cl, nc)


def test_forward_argument_errors_need_no_device():
    s = kspec.SPEC_C1
    p = abi.Plan(s.input_modes, s.output_modes, s.rank, abi.TR_F16)
    assert p.forward(0, 0, 0, 0) == abi.TR_OK               # T == 0 is a no-op
    assert p.forward(0, 16, 1, 16) == abi.TR_ERR_INVALID     # null packed
    assert p.forward(16, 16, -1, 16) == abi.TR_ERR_INVALID   # negative T
    assert p.forward(16, 18, 1, 16) == abi.TR_ERR_ALIGN      # misaligned x
    # a tiling that reduces across clusters needs its workspace
    forced = abi.TrTiling(tokens_per_tile=1, cluster=2, clusters=4, kernel=abi.KERNEL_MMA)
    assert p.forward(16, 16, 1, 16, 0, 0, tiling=forced) == abi.TR_ERR_WORKSPACE
    # fp16 plans pack the mma layout; the generic kernel is for fp32 plans
    generic = abi.TrTiling(kernel=abi.KERNEL_GENERIC)
    assert p.forward(16, 16, 1, 16, tiling=generic) == abi.TR_ERR_UNSUPPORTED
    assert p.forward(16, 16, 1, 16, tiling=abi.TrTiling(kernel=9)) == abi.TR_ERR_UNSUPPORTED


def test_torch_binding_loads():
    from kernel_task_b200._native import binding

    mod = binding()
    assert hasattr(mod, "RingOp") and hasattr(mod, "empty_launch")


def test_cpu_cores_raise_instead_of_falling_back():
    import torch

    from kernel_task_b200 import prepare_optimized

    s = kspec.TRSpec((2, 3, 2), (2, 4, 3), 2)
    cores = kspec.make_cores(s)
    with pytest.raises(RuntimeError, match="CUDA"):
        prepare_optimized(cores, s)
    with pytest.raises(ValueError, match="Core 1 should have shape"):
        prepare_optimized((cores[0], cores[0], cores[2]), s)
    del torch


def test_ctypes_plan_lifecycle():
    lib = abi.lib()
    spec = abi.TrSpec((ctypes.c_int32 * 3)(8, 12, 20), (ctypes.c_int32 * 3)(12, 10, 24), 8)
    h = ctypes.c_void_p()
    assert lib.tr_plan_create(ctypes.byref(spec), abi.TR_F16, 0, ctypes.byref(h)) == abi.TR_OK
    n = ctypes.c_size_t()
    assert lib.tr_packed_bytes(h, ctypes.byref(n)) == abi.TR_OK and n.value > 0
    lib.tr_plan_destroy(h)
    assert lib.tr_plan_create(None, 0, 0, ctypes.byref(h)) == abi.TR_ERR_INVALID


def test_noalloc_entry_point_arguments_need_no_device():
    """tr_forward_noalloc: argument errors are reported before any CUDA call, fp32 plans are
    not served, and the documented scratch size matches the header."""
    text = HEADER.read_text()
    assert re.search(r"#define TR_NOALLOC_SCRATCH_BYTES \(8u << 20\)", text)
    s = kspec.SPEC_C1
    p16 = abi.Plan(s.input_modes, s.output_modes, s.rank, abi.TR_F16)
    p32 = abi.Plan(s.input_modes, s.output_modes, s.rank, abi.TR_F32)
    assert p16.forward_noalloc(0, 0, 0, 0) == abi.TR_OK           # T == 0 is a no-op
    assert p16.forward_noalloc(16, 16, -1, 16) == abi.TR_ERR_INVALID
    assert p16.forward_noalloc(0, 16, 1, 16) == abi.TR_ERR_INVALID
    assert p16.forward_noalloc(16, 24, 1, 16) == abi.TR_ERR_ALIGN
    assert p32.forward_noalloc(16, 16, 1, 16) == abi.TR_ERR_UNSUPPORTED
    # the mma kernel's default geometry (the one the no-alloc entry point runs) fits the
    # built-in scratch for every benchmark shape and size
    mma = abi.TrTiling(kernel=abi.KERNEL_MMA)
    for sp in (kspec.SPEC_C1, kspec.SPEC_C2, *kspec.SPEC_C4.values()):
        p = abi.Plan(sp.input_modes, sp.output_modes, sp.rank, abi.TR_F16)
        for T in (1, 2, 3, 5, 8, 16, 32, 64, 128, 1000):
            assert p.workspace_bytes(T, mma) <= (8 << 20)


def test_epilogue_and_consumer_arguments_need_no_device():
    """tr_forward_epilogue and tr_consume_*: argument errors are reported before any CUDA
    call (the fused forms are checked against the unfused ones on the GPU)."""
    s = kspec.SPEC_C4["down"]
    p = abi.Plan(s.input_modes, s.output_modes, s.rank, abi.TR_BF16)
    E = abi.TrEpilogue
    fwd = lambda epi, T=1, y=16: p.forward_epilogue(16, 16, T, y, epi)
    assert fwd(None, T=0) == abi.TR_OK
    assert fwd(E(abi.TR_EPI_ADD, abi.TR_BF16, 16, abi.TR_F32), T=0) == abi.TR_OK
    assert fwd(E(7, abi.TR_BF16, 16, abi.TR_BF16)) == abi.TR_ERR_INVALID        # unknown kind
    assert fwd(E(abi.TR_EPI_NONE, abi.TR_F16, 0, 0)) == abi.TR_ERR_INVALID      # other dtype
    assert fwd(E(abi.TR_EPI_ADD, abi.TR_F32, 16, abi.TR_F16)) == abi.TR_ERR_INVALID
    assert fwd(E(abi.TR_EPI_SILU_MUL, abi.TR_BF16, 0, abi.TR_F32)) == abi.TR_ERR_INVALID
    assert fwd(E(abi.TR_EPI_ADD, abi.TR_BF16, 24, abi.TR_F32)) == abi.TR_ERR_ALIGN
    assert fwd(E(abi.TR_EPI_ADD, abi.TR_F32, 16, abi.TR_F32), y=0) == abi.TR_ERR_INVALID
    assert fwd(E(abi.TR_EPI_ADD, abi.TR_F32, 16, abi.TR_F32), T=-1) == abi.TR_ERR_INVALID
    assert lib_call("tr_forward_epilogue", None, 16, 16, 1, 16, None, None, 0, None,
                    None) == abi.TR_ERR_INVALID                                  # null plan
    L = abi.lib()
    assert L.tr_consume_silu_mul(16, 16, 16, abi.TR_BF16, 0, None) == abi.TR_OK
    assert L.tr_consume_silu_mul(16, 16, 16, abi.TR_F32, 4, None) == abi.TR_ERR_INVALID
    assert L.tr_consume_silu_mul(16, 16, 16, abi.TR_BF16, 6, None) == abi.TR_ERR_INVALID
    assert L.tr_consume_silu_mul(None, 16, 16, abi.TR_F16, 4, None) == abi.TR_ERR_INVALID
    assert L.tr_consume_silu_mul(16, 20, 16, abi.TR_F16, 4, None) == abi.TR_ERR_ALIGN
    assert L.tr_consume_add(16, 16, 16, abi.TR_BF16, -4, None) == abi.TR_ERR_INVALID
    assert L.tr_consume_add(16, 16, 8, abi.TR_BF16, 4, None) == abi.TR_ERR_ALIGN
    assert L.tr_consume_add(16, 16, 16, 3, 4, None) == abi.TR_ERR_INVALID


def lib_call(name, *args):
    return getattr(abi.lib(), name)(*args)


def test_workspace_status_and_wait_limit_arguments_need_no_device():
    """tr_workspace_status / tr_plan_set_wait_limit: argument errors before any CUDA call; a
    zero-byte workspace (decode and mma kernels) has no status word and reads TR_OK."""
    L = abi.lib()
    st = ctypes.c_int32(123)
    assert L.tr_workspace_status(None, 0, ctypes.byref(st), 1, None) == abi.TR_OK
    assert st.value == abi.TR_OK
    assert L.tr_workspace_status(None, 0, None, 1, None) == abi.TR_ERR_INVALID
    assert L.tr_workspace_status(None, 256, ctypes.byref(st), 1, None) == abi.TR_ERR_INVALID
    assert L.tr_plan_set_wait_limit(None, 1) == abi.TR_ERR_INVALID
    s = kspec.SPEC_C1
    p = abi.Plan(s.input_modes, s.output_modes, s.rank, abi.TR_F16)
    p.set_wait_limit(1)
    p.set_wait_limit(0)
