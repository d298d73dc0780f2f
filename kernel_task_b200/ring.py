"""The drop-in surface: ``prepare_optimized(cores, spec) -> fn(x)``.

Mirrors factorized_inference/submission.py:26-48 and PreparedTRKernel
(factorized_inference/tr_kernel.py:179-319): preparation packs the cores once into the
kernel-native layouts (never a dense weight), and the returned callable runs one fused CUDA
kernel per call on the caller's current stream, for any token count.

Differences from the reference, by design:
  * every call launches this library's sm_100a kernels; there is no CPU or torch fallback.
    CPU tensors, or x of another dtype/device than the cores, raise instead of silently
    running the unoptimized contraction (tr_kernel.py:265-266, submission.py:48);
  * fp32 CUDA cores run the generic fp32 kernel (the reference sends fp32 to its einsum path);
  * the callable is the C++ object itself, so no Python frame runs per call;
  * state is one packed-core buffer and, for tilings that reduce across clusters, one
    workspace that every call leaves ready for the next (stream-ordered; one prepared object
    must not be called concurrently from two streams, as in the reference, tr_kernel.py:185).

Model-chain calls on the prepared object (the reference's PreparedTRKernel.accumulate,
tr_kernel.py:230-243, and its consumers, csrc/v3g/bind.cu:93-156):
  * ``op.accumulate(x)``         y in fp32 (a new tensor; the reference returns a view of its
                                 workspace that the consumer must clear);
  * ``op.forward_add(x, h)``     h + op(x), the residual add done in the forward kernel's store;
  * ``op.forward_silu_mul(x, g)`` silu(g) * op(x), the gated MLP done in the up projection's
                                 store (g = gate.accumulate(x), fp32, or the cores' dtype);
  * ``consume_silu_mul(g, u)`` / ``consume_add(h, y)``: the reference's separate consumers of
    fp32 outputs (they clear the fp32 inputs, as the reference's do).
"""
from __future__ import annotations

from typing import Sequence

import torch

from ._native import binding
from .spec import TRSpec, validate_cores

_SUPPORTED = (torch.float32, torch.float16, torch.bfloat16)


def _ring_op_class():
    return binding().RingOp


def prepare_optimized(cores: Sequence[torch.Tensor], spec: TRSpec):
    """Pack ``cores`` for ``spec`` and return the per-call operator ``fn(x) -> y``.

    cores: three CUDA tensors [R, o_k, i_k, R] of one dtype (float16, bfloat16 or float32)
    on one device.  They are read during packing and neither modified nor retained.
    fn(x):  x [T, in_features] of the same dtype and device, any T >= 0 (may change between
    calls); returns a new y [T, out_features] on the caller's current stream.
    """
    cores = tuple(cores)
    validate_cores(cores, spec)
    if not all(isinstance(c, torch.Tensor) and c.is_cuda for c in cores):
        raise RuntimeError("kernel_task_b200 runs its kernels on CUDA devices only; "
                           "move the cores to a CUDA device")
    dtype, device = cores[0].dtype, cores[0].device
    if dtype not in _SUPPORTED:
        raise ValueError(f"unsupported core dtype {dtype}")
    if any(c.dtype != dtype or c.device != device for c in cores):
        raise ValueError("all cores must share one dtype and device")
    op = _ring_op_class()(list(spec.input_modes), list(spec.output_modes), spec.rank, dtype,
                          device.index if device.index is not None
                          else torch.cuda.current_device())
    with torch.cuda.device(device):
        op.pack([c.contiguous() for c in cores])
    return op


def tr_forward_optimized(x: torch.Tensor, cores: Sequence[torch.Tensor], spec: TRSpec):
    """One-shot form (submission.py:10-23): prepares, runs once, discards the preparation."""
    return prepare_optimized(cores, spec)(x)


def consume_silu_mul(g: torch.Tensor, u: torch.Tensor, dtype: torch.dtype = torch.bfloat16):
    """silu(g) * u -> ``dtype``; g and u are fp32 [T, N] (N % 4 == 0) and are zero-filled
    afterwards, as the reference's consumer does (csrc/v3g/bind.cu:123-133)."""
    return binding().consume_silu_mul(g, u, dtype)


def consume_add(h: torch.Tensor, y: torch.Tensor):
    """h + y -> h's dtype; y is fp32 of h's shape and is zero-filled afterwards
    (csrc/v3g/bind.cu:135-148)."""
    return binding().consume_add(h, y)
