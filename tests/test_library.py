"""torch.library registration: the ops' fake implementations (shapes and dtypes without a
kernel) and graph capture by torch.compile, on CPU with a stand-in operator; the GPU half runs
the registered CUDA operator."""
from __future__ import annotations

import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

from kernel_task_b200 import library
from kernel_task_b200 import spec as kspec

SPEC = kspec.TRSpec((2, 3, 4), (3, 2, 5), 3)


class _StandIn:
    """CPU stand-in with the prepared operator's methods (shapes only)."""

    def __call__(self, x):
        return torch.zeros(x.shape[0], SPEC.out_features, dtype=x.dtype)

    def accumulate(self, x):
        return torch.zeros(x.shape[0], SPEC.out_features, dtype=torch.float32)

    def forward_add(self, x, h):
        return h + self(x)

    def forward_silu_mul(self, x, g):
        return torch.nn.functional.silu(g.float()).to(x.dtype) * self(x)


def test_fake_shapes_and_errors():
    h = library.register(_StandIn(), SPEC)
    try:
        with FakeTensorMode():
            x = torch.empty(5, SPEC.in_features, dtype=torch.bfloat16)
            y = torch.ops.trring.forward(x, h)
            assert y.shape == (5, SPEC.out_features) and y.dtype == torch.bfloat16
            a = torch.ops.trring.accumulate(x, h)
            assert a.dtype == torch.float32 and a.shape == y.shape
            assert torch.ops.trring.forward_add(x, y, h).shape == y.shape
            assert torch.ops.trring.forward_silu_mul(x, y, h).shape == y.shape
            with pytest.raises(ValueError):
                torch.ops.trring.forward(torch.empty(5, 7), h)
    finally:
        library.unregister(h)
    with pytest.raises(ValueError):
        torch.ops.trring.forward(torch.empty(1, SPEC.in_features), h)


def test_compiles_without_graph_breaks():
    h = library.register(_StandIn(), SPEC)
    try:
        def block(x, res):
            return torch.ops.trring.forward_add(x, res, h) * 2

        f = torch.compile(block, backend="eager", fullgraph=True)
        x = torch.randn(4, SPEC.in_features)
        res = torch.randn(4, SPEC.out_features)
        torch.testing.assert_close(f(x, res), block(x, res))
    finally:
        library.unregister(h)


@pytest.mark.gpu
def test_registered_cuda_operator():
    from kernel_task_b200 import prepare_optimized

    s = kspec.SPEC_C4["down"]
    cores = kspec.baseline_cores(s, seed=2, dtype=torch.bfloat16, device="cuda")
    fn = prepare_optimized(cores, s)
    h = library.register(fn, s)
    try:
        x = kspec.baseline_x(s, 3, seed=2, dtype=torch.bfloat16, device="cuda")
        res = torch.randn(3, s.out_features, device="cuda").to(torch.bfloat16)
        torch.testing.assert_close(torch.ops.trring.forward(x, h), fn(x), rtol=0, atol=0)
        torch.testing.assert_close(torch.ops.trring.forward_add(x, res, h),
                                   fn.forward_add(x, res), rtol=0, atol=0)
        f = torch.compile(lambda a, b: torch.ops.trring.forward_add(a, b, h), backend="eager",
                          fullgraph=True)
        torch.testing.assert_close(f(x, res), fn.forward_add(x, res), rtol=0, atol=0)
        g32 = torch.ops.trring.accumulate(x, h)
        u32 = g32.clone()
        act = torch.ops.trring.consume_silu_mul(g32, u32)
        assert act.dtype == torch.bfloat16 and not g32.any()
    finally:
        library.unregister(h)
