"""torch.library registration of the operator, so that prepared operators compose with
torch.compile, CUDA graphs and other custom-op machinery:

    handle = kernel_task_b200.library.register(fn, spec)     # fn from prepare_optimized
    y = torch.ops.trring.forward(x, handle)                  # same as fn(x)
    h = torch.ops.trring.forward_add(x, h0, handle)          # fn.forward_add(x, h0)
    a = torch.ops.trring.forward_silu_mul(x, g, handle)      # fn.forward_silu_mul(x, g)
    g = torch.ops.trring.accumulate(x, handle)               # fn.accumulate(x), fp32
    torch.ops.trring.consume_silu_mul(g, u), torch.ops.trring.consume_add(h, y)

A prepared operator is a C++ object, which a custom op cannot take as an argument, so operators
are registered in a process-local table and the op takes the integer handle.  Each op has a
fake (meta) implementation giving the output shape and dtype without running a kernel.
"""
from __future__ import annotations

import itertools
import threading

import torch

from .ring import consume_add as _consume_add
from .ring import consume_silu_mul as _consume_silu_mul
from .spec import TRSpec

_lock = threading.Lock()
_ids = itertools.count(1)
_table: dict[int, tuple[object, int, int]] = {}  # handle -> (operator, in_features, out_features)


def register(op, spec: TRSpec) -> int:
    """Make `op` (a prepared operator for `spec`) callable through torch.ops.trring.*."""
    with _lock:
        handle = next(_ids)
        _table[handle] = (op, spec.in_features, spec.out_features)
    return handle


def unregister(handle: int) -> None:
    with _lock:
        _table.pop(handle, None)


def _entry(handle: int, x: torch.Tensor):
    try:
        op, d_in, d_out = _table[handle]
    except KeyError:
        raise ValueError(f"no operator registered under handle {handle}") from None
    if x.dim() != 2 or x.shape[1] != d_in:
        raise ValueError(f"Expected x with shape [tokens, {d_in}]")
    return op, d_out


@torch.library.custom_op("trring::forward", mutates_args=())
def forward(x: torch.Tensor, handle: int) -> torch.Tensor:
    op, _ = _entry(handle, x)
    return op(x)


@forward.register_fake
def _(x, handle):
    _, d_out = _entry(handle, x)
    return x.new_empty((x.shape[0], d_out))


@torch.library.custom_op("trring::accumulate", mutates_args=())
def accumulate(x: torch.Tensor, handle: int) -> torch.Tensor:
    op, _ = _entry(handle, x)
    return op.accumulate(x)


@accumulate.register_fake
def _(x, handle):
    _, d_out = _entry(handle, x)
    return x.new_empty((x.shape[0], d_out), dtype=torch.float32)


@torch.library.custom_op("trring::forward_add", mutates_args=())
def forward_add(x: torch.Tensor, h: torch.Tensor, handle: int) -> torch.Tensor:
    op, _ = _entry(handle, x)
    return op.forward_add(x, h)


@forward_add.register_fake
def _(x, h, handle):
    _, d_out = _entry(handle, x)
    return x.new_empty((x.shape[0], d_out))


@torch.library.custom_op("trring::forward_silu_mul", mutates_args=())
def forward_silu_mul(x: torch.Tensor, g: torch.Tensor, handle: int) -> torch.Tensor:
    op, _ = _entry(handle, x)
    return op.forward_silu_mul(x, g)


@forward_silu_mul.register_fake
def _(x, g, handle):
    _, d_out = _entry(handle, x)
    return x.new_empty((x.shape[0], d_out))


@torch.library.custom_op("trring::consume_silu_mul", mutates_args=("g", "u"))
def consume_silu_mul(g: torch.Tensor, u: torch.Tensor) -> torch.Tensor:
    return _consume_silu_mul(g, u)


@consume_silu_mul.register_fake
def _(g, u):
    return g.new_empty(g.shape, dtype=torch.bfloat16)


@torch.library.custom_op("trring::consume_add", mutates_args=("y",))
def consume_add(h: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
    return _consume_add(h, y)


@consume_add.register_fake
def _(h, y):
    return torch.empty_like(h)
