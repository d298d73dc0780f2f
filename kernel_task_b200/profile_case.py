"""Run one benchmark case a few times, for profilers (ncu) and quick checks.

    python -m kernel_task_b200.profile_case --rank 16 --tokens 32 [--calls 5] [--tiling TT,CL,NC]

Builds the seeded benchmark operator (1920->2880, modes (8,12,20)->(12,10,24), fp16; or any
--input-modes/--output-modes/--dtype), makes `--calls` calls and synchronises.  Under
`ncu -k regex:ring -s <calls-1> -c 1` it captures the last call's kernel.
"""
from __future__ import annotations

import argparse

import torch

from . import prepare_optimized
from .spec import TRSpec, baseline_cores, baseline_x


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--rank", type=int, default=8)
    ap.add_argument("--tokens", type=int, default=1)
    ap.add_argument("--input-modes", default="8,12,20")
    ap.add_argument("--output-modes", default="12,10,24")
    ap.add_argument("--dtype", default="float16", choices=("float16", "bfloat16", "float32"))
    ap.add_argument("--calls", type=int, default=5)
    ap.add_argument("--tiling", default=None, help="kernel,TT,CL,NC forced geometry")
    a = ap.parse_args()
    spec = TRSpec(tuple(int(v) for v in a.input_modes.split(",")),
                  tuple(int(v) for v in a.output_modes.split(",")), a.rank)
    dtype = getattr(torch, a.dtype)
    dev = torch.device("cuda")
    fn = prepare_optimized(baseline_cores(spec, dtype=dtype, device=dev), spec)
    x = baseline_x(spec, a.tokens, dtype=dtype, device=dev)
    forced = tuple(int(v) for v in a.tiling.split(",")) if a.tiling else None
    for _ in range(a.calls):
        y = fn.call_tiled(x, *forced) if forced else fn(x)
    torch.cuda.synchronize()
    print(f"ok {tuple(y.shape)} tiling={fn.tiling(a.tokens)} {fn.describe()}")


if __name__ == "__main__":
    main()
