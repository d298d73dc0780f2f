"""Operator spec and seeded cores, mirroring the reference's spec API.

``TRSpec`` and ``make_cores`` keep the names, fields, validation messages and generator
semantics of factorized_inference/reference.py:15-77 so that code written against the
reference runs unchanged: a dense [out, in] weight is represented by three cores, core k of
shape [rank, output_modes[k], input_modes[k], rank], one rank for all three ring links.

``baseline_cores`` generates the synthetic cores of the benchmark configurations: i.i.d.
N(0, sigma^2) with sigma = (R * d_in^(1/3))^(-1/2), drawn in [R, i, o, R] order (input mode
before output mode) and transposed to the reference's [R, o, i, R] storage order.
"""
from __future__ import annotations

from dataclasses import dataclass
from math import prod
from typing import Sequence

import torch


@dataclass(frozen=True)
class TRSpec:
    """Shape of a three-core tensor-ring linear layer (reference.py:15-50)."""

    input_modes: tuple[int, int, int] = (8, 12, 20)
    output_modes: tuple[int, int, int] = (12, 10, 24)
    rank: int = 8

    def __post_init__(self) -> None:
        if len(self.input_modes) != 3 or len(self.output_modes) != 3:
            raise ValueError("Exactly three input and output modes are required")
        if any(v <= 0 for v in (*self.input_modes, *self.output_modes, self.rank)):
            raise ValueError("All modes and the rank must be positive")

    @property
    def in_features(self) -> int:
        return prod(self.input_modes)

    @property
    def out_features(self) -> int:
        return prod(self.output_modes)

    @property
    def factor_parameters(self) -> int:
        return sum(self.rank * o * i * self.rank
                   for o, i in zip(self.output_modes, self.input_modes))

    @property
    def dense_parameters(self) -> int:
        return self.in_features * self.out_features

    def core_shapes(self) -> tuple[tuple[int, int, int, int], ...]:
        return tuple((self.rank, o, i, self.rank)
                     for o, i in zip(self.output_modes, self.input_modes))


def make_cores(spec: TRSpec, *, device: torch.device | str = "cpu",
               dtype: torch.dtype = torch.float32, seed: int = 0):
    """Seeded cores with the reference's generator semantics (reference.py:53-77): one
    ``torch.Generator(device)`` seeded once, cores drawn in order as randn[R, o, i, R] and
    scaled by (R * i)^(-1/2), so that each implied weight entry has variance 1/in_features."""
    generator = torch.Generator(device=device)
    generator.manual_seed(seed)
    cores = []
    for o, i in zip(spec.output_modes, spec.input_modes):
        core = torch.randn(spec.rank, o, i, spec.rank, generator=generator, device=device,
                           dtype=dtype)
        cores.append(core * (1.0 / (spec.rank * i) ** 0.5))
    return tuple(cores)


def baseline_sigma(spec: TRSpec) -> float:
    return (spec.rank * spec.in_features ** (1.0 / 3.0)) ** -0.5


def baseline_cores(spec: TRSpec, *, seed: int = 0, dtype: torch.dtype = torch.float16,
                   device: torch.device | str = "cpu"):
    """Benchmark cores: N(0, sigma^2) drawn on the CPU generator in [R, i, o, R] order, then
    stored as the reference's [R, o, i, R].  Generated on the CPU so every machine draws the
    same values, then cast and moved."""
    generator = torch.Generator().manual_seed(seed)
    sigma = baseline_sigma(spec)
    cores = []
    for o, i in zip(spec.output_modes, spec.input_modes):
        core = torch.randn(spec.rank, i, o, spec.rank, generator=generator) * sigma
        cores.append(core.transpose(1, 2).contiguous().to(dtype=dtype, device=device))
    return tuple(cores)


def baseline_x(spec: TRSpec, tokens: int, *, seed: int = 0, dtype: torch.dtype = torch.float16,
               device: torch.device | str = "cpu") -> torch.Tensor:
    """x ~ N(0, 1) of shape [tokens, in_features], CPU generator seeded with seed + tokens
    (the reference harness's convention, benchmarks/benchmark.py:108)."""
    generator = torch.Generator().manual_seed(seed + tokens)
    x = torch.randn(tokens, spec.in_features, generator=generator)
    return x.to(dtype=dtype, device=device)


def validate(x: torch.Tensor, cores: Sequence[torch.Tensor], spec: TRSpec) -> None:
    """Shape checks with the reference's messages (reference.py:80-96)."""
    if x.ndim != 2 or x.shape[1] != spec.in_features:
        raise ValueError(
            f"Expected x with shape [tokens, {spec.in_features}], got {tuple(x.shape)}")
    validate_cores(cores, spec)


def validate_cores(cores: Sequence[torch.Tensor], spec: TRSpec) -> None:
    if len(cores) != 3:
        raise ValueError(f"Expected three cores, got {len(cores)}")
    for index, (core, expected) in enumerate(zip(cores, spec.core_shapes())):
        if tuple(core.shape) != expected:
            raise ValueError(
                f"Core {index} should have shape {expected}, got {tuple(core.shape)}")


# The benchmark configurations (shapes only; dtype per config).
SPEC_C1 = TRSpec((8, 12, 20), (12, 10, 24), 8)
SPEC_C2 = TRSpec((8, 12, 20), (12, 10, 24), 16)
SPEC_C3 = TRSpec((16, 16, 16), (16, 28, 32), 32)
SPEC_C4 = {
    "q": TRSpec((16, 16, 16), (16, 16, 16), 16),
    "k": TRSpec((16, 16, 16), (8, 8, 16), 16),
    "v": TRSpec((16, 16, 16), (8, 8, 16), 16),
    "o": TRSpec((16, 16, 16), (16, 16, 16), 16),
    "gate": TRSpec((16, 16, 16), (16, 28, 32), 16),
    "up": TRSpec((16, 16, 16), (16, 28, 32), 16),
    "down": TRSpec((16, 28, 32), (16, 16, 16), 16),
}
SPEC_C5 = TRSpec((16, 16, 16), (16, 28, 32), 16)
