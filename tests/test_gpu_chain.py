"""GPU: the config-4 decode chain and the config-5 prefill at full size, against the oracle.

* One transformer layer of tensor-ring projections (q, k, v, o, gate, up, down; attention not
  simulated, o reads q's output as in the reference's chain, tools/qwen_model_chain.py:111-134),
  run with the fused epilogues (o and down add the residual in their store; up multiplies by
  silu(gate) in its store; gate is accumulated in fp32).  Each launch is checked against the
  oracle's float64 contraction of the GPU's own input to that launch (single-operator
  tolerance), and the final output against a numpy chain that rounds to bf16 at the same points
  (q, the residual stream after o, the silu-gated product, the output) under a chain bound.
* The config-5 operator (4096 -> 14336, R16, bf16) on all 65,536 prefill tokens in one call:
  sampled rows against the oracle, and the same rows computed alone, under the same split of
  the pieces, bit-identical.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from helpers import check_close, errors
from kernel_task_b200 import prepare_optimized
from kernel_task_b200 import spec as kspec

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _bf16(a: np.ndarray) -> np.ndarray:
    return torch.from_numpy(np.asarray(a, dtype=np.float32)).to(torch.bfloat16).float().numpy()


def test_decode_chain_layer_against_oracle_chain():
    names = ["q", "k", "v", "o", "gate", "up", "down"]
    cores = {n: kspec.baseline_cores(kspec.SPEC_C4[n], seed=30 + i, dtype=torch.bfloat16,
                                     device=DEV) for i, n in enumerate(names)}
    ops = {n: prepare_optimized(cores[n], kspec.SPEC_C4[n]) for n in names}
    h = kspec.baseline_x(kspec.SPEC_C4["q"], 1, seed=31, dtype=torch.bfloat16, device=DEV)

    # the fused chain (7 launches)
    q = ops["q"](h)
    k = ops["k"](h)
    v = ops["v"](h)
    h1 = ops["o"].forward_add(q, h)
    act = ops["up"].forward_silu_mul(h1, ops["gate"].accumulate(h1))
    h2 = ops["down"].forward_add(act, h1)
    torch.cuda.synchronize()

    # stage by stage: each fused launch against the oracle (float64) applied to the GPU's own
    # input of that launch, under the single-operator tolerance
    c64 = {n: [c.double().cpu().numpy() for c in cores[n]] for n in names}
    f = lambda n, a: oracle.tr_forward_reference(a, c64[n], dtype=np.float64)  # noqa: E731
    npy = lambda a: a.double().cpu().numpy()  # noqa: E731
    h0, q_g, h1_g, act_g = npy(h), npy(q), npy(h1), npy(act)
    check_close(q, f("q", h0), torch.bfloat16)
    check_close(k, f("k", h0), torch.bfloat16)
    check_close(v, f("v", h0), torch.bfloat16)
    check_close(h1, h0 + f("o", q_g), torch.bfloat16)
    g = f("gate", h1_g)
    check_close(act, g / (1.0 + np.exp(-g)) * f("up", h1_g), torch.bfloat16)
    check_close(h2, h1_g + f("down", act_g), torch.bfloat16)

    # end to end: the oracle chain, float64 contractions rounded to bf16 at the same four points
    # as the fused chain (q, h1, act, h2).  One-ulp differences at a rounding point propagate
    # through the next projections, so the chain's bound is the reference's element rule and a
    # relative Frobenius error of 1e-2 (four rounding points of 2^-9 each, amplified by at most
    # the two products of the gated activation)
    q_r = _bf16(f("q", h0))
    h1_r = _bf16(h0 + f("o", q_r))
    g_r = f("gate", h1_r)
    act_r = _bf16(g_r / (1.0 + np.exp(-g_r)) * f("up", h1_r))
    h2_r = h1_r + f("down", act_r)
    e = errors(h2, h2_r)
    torch.testing.assert_close(h2.double().cpu(), torch.from_numpy(h2_r), rtol=2e-2, atol=2e-2)
    assert e["rel_frob"] <= 1e-2, e


def test_prefill_config5_full_size_sampled_rows():
    s = kspec.SPEC_C5
    T = 65536
    cores = kspec.baseline_cores(s, seed=12, dtype=torch.bfloat16, device=DEV)
    fn = prepare_optimized(cores, s)
    gen = torch.Generator(device=DEV).manual_seed(12)
    x = torch.randn(T, s.in_features, generator=gen, device=DEV).to(torch.bfloat16)
    y = fn(x)
    torch.cuda.synchronize()
    assert torch.isfinite(y).all()
    rows = [0, 1, 4095, 32767, 40000, T - 2, T - 1]
    ref = oracle.tr_forward_reference(x[rows].float().cpu().numpy(),
                                      [c.float().cpu().numpy() for c in cores])
    check_close(y[rows], ref, torch.bfloat16)
    geom = fn.tiling(T)
    alone = fn.call_tiled(x[rows].contiguous(), geom["kernel"], 0, geom["cluster"],
                          geom["clusters"])
    torch.testing.assert_close(alone, y[rows], rtol=0, atol=0)
    del x, y
    torch.cuda.empty_cache()
