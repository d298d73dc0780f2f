"""CPU: pin the numpy oracle to the reference's own outputs (tests/golden) before anything is
checked against it.  Mirrors the reference's tests/test_correctness.py:26-46 and :80-91."""
from __future__ import annotations

import hashlib

import numpy as np
import pytest
import torch

import oracle
from kernel_task_b200 import spec as kspec

SPECS = [((2, 3, 2), (2, 4, 3), 2), ((4, 4, 4), (4, 4, 4), 8), ((4, 4, 4), (4, 4, 4), 16)]


def cores_of(g, key):
    return [g[f"{key}_core{k}"] for k in range(3)]


@pytest.mark.parametrize("si", range(3))
@pytest.mark.parametrize("seed", [0, 19])
def test_oracle_matches_reference_fp32(golden, si, seed):
    key = f"cpu{si}_s{seed}"
    cores = cores_of(golden, key)
    for n in range(4):
        x = golden[f"{key}_x{n}"]
        y = oracle.tr_forward_reference(x, cores)
        ref = golden[f"{key}_yref{n}"]
        np.testing.assert_allclose(y, ref, rtol=1e-5, atol=1e-6)
        # and the reference's own fp64 dense oracle at the reference's fp32 tolerance
        np.testing.assert_allclose(y, golden[f"{key}_y64_{n}"], rtol=1e-4, atol=1e-4)


def test_index_convention_known_answer(golden):
    """W[o, in] == trace(A[:,p,i,:] B[:,q,j,:] C[:,r,k,:]) (test_correctness.py:80-91)."""
    cores = cores_of(golden, "kat")
    W = oracle.materialize_dense_weight(cores)
    np.testing.assert_allclose(W, golden["kat_W"], rtol=1e-12, atol=1e-12)
    A, B, C = cores
    for o in range(8):
        p, q, r = o // 4, o // 2 % 2, o % 2
        for inp in range(8):
            i, j, k = inp // 4, inp // 2 % 2, inp % 2
            expect = np.trace(A[:, p, i, :] @ B[:, q, j, :] @ C[:, r, k, :])
            assert abs(W[o, inp] - expect) < 1e-12


@pytest.mark.parametrize("key,ntok", [("odd0", 3), ("odd1", 2), ("odd2", 3), ("odd3", 2)])
def test_every_ring_order_equals_reference(golden, key, ntok):
    """The product contracts in the cheapest of the six ring orders; each order is the same
    sum (checked in fp64 against the reference's fp32 output of the same fp16 inputs)."""
    cores = [c.astype(np.float64) for c in cores_of(golden, key)]
    for n in range(ntok):
        x = golden[f"{key}_x{n}"].astype(np.float64)
        ref = golden[f"{key}_yref{n}"]
        scale = max(1.0, float(np.abs(ref).max()))
        for X in range(3):
            for Y in range(3):
                if X != Y:
                    y = oracle.order_forward(x, cores, X, Y)
                    assert np.abs(y - ref).max() <= 1e-5 * scale


@pytest.mark.parametrize("R,T", [(8, 1), (8, 8), (8, 32), (16, 1), (16, 32)])
def test_required_workloads_oracle(golden, R, T):
    key = f"req_r{R}"
    cores = cores_of(golden, key)
    y = oracle.tr_forward_reference(golden[f"{key}_x_t{T}"], cores)
    np.testing.assert_allclose(y, golden[f"{key}_yref_t{T}"], rtol=1e-4, atol=1e-5)


def test_make_cores_reproduces_reference(golden):
    for si, (im, om, R) in enumerate(SPECS):
        for seed in (0, 19):
            mine = kspec.make_cores(kspec.TRSpec(im, om, R), seed=seed)
            for k, c in enumerate(mine):
                np.testing.assert_array_equal(c.numpy(), golden[f"cpu{si}_s{seed}_core{k}"])


def test_baseline_generator_is_pinned(golden_baseline):
    meta, vec = golden_baseline
    for name, m in meta.items():
        s = kspec.TRSpec(tuple(m["input_modes"]), tuple(m["output_modes"]), m["rank"])
        cores = kspec.baseline_cores(s, seed=m["core_seed"], dtype=torch.bfloat16)
        got = [hashlib.sha256(c.view(torch.int16).numpy().tobytes()).hexdigest() for c in cores]
        assert got == m["core_sha256"], name
        for T in m["tokens"]:
            x = kspec.baseline_x(s, T, seed=m["core_seed"], dtype=torch.bfloat16)
            np.testing.assert_array_equal(x.view(torch.int16).numpy(), vec[f"{name}_x_t{T}"])


@pytest.mark.parametrize("name", ["c3", "c4_q", "c4_k", "c4_gate", "c4_down"])
def test_oracle_matches_reference_baseline_configs(golden_baseline, name):
    meta, vec = golden_baseline
    m = meta[name]
    s = kspec.TRSpec(tuple(m["input_modes"]), tuple(m["output_modes"]), m["rank"])
    cores = [c.float().numpy() for c in kspec.baseline_cores(s, seed=m["core_seed"],
                                                                dtype=torch.bfloat16)]
    T = m["tokens"][0]
    x = torch.from_numpy(vec[f"{name}_x_t{T}"]).view(torch.bfloat16).float().numpy()
    y = oracle.tr_forward_reference(x, cores)
    ref = vec[f"{name}_yref_t{T}"]
    assert np.abs(y - ref).max() <= 1e-4 * max(1.0, float(np.abs(ref).max()))


def test_flop_model_matches_reference_order():
    """The reference's own FLOP count (tools/measure_kernels.py:36-44) is its order's MACs x2."""
    for s in (kspec.SPEC_C1, kspec.SPEC_C2, kspec.SPEC_C3):
        ni, nj, nk = s.input_modes
        P, Q, Rr = s.output_modes
        R = s.rank
        theirs = 2 * (ni * nj * nk * P * R * R + nj * nk * P * Q * R ** 3 + P * Q * Rr * nk * R * R)
        assert 2 * oracle.reference_macs(s.input_modes, s.output_modes, R) == theirs
