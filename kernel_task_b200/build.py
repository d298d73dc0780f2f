"""Build the native parts in-tree: libtrring.so (C ABI, nvcc, sm_100a) and the thin PyTorch
binding _trring_torch.so that links it.  Run ``python -m kernel_task_b200.build``.

Both shared objects land next to this file so they travel with the source tree; nothing is
installed into site-packages and no JIT cache is used at run time.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
LIB = PKG / "libtrring.so"
EXT = PKG / "_trring_torch.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CUDA_SOURCES = ["plan.cpp", "pack.cu", "ring_generic.cu", "ring_mma.cu", "ring_decode.cu",
                "ring_tc05.cu", "ring_slab.cu", "consume.cu"]


def _nvcc() -> str:
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = Path(home) / "bin" / "nvcc"
    return str(cand) if cand.exists() else "nvcc"


def build_library(verbose: bool = False) -> Path:
    """nvcc -> libtrring.so (all kernels + the C ABI)."""
    cmd = [_nvcc(), *ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-shared",
           f"-I{INCLUDE}", "-o", str(LIB), *[str(CSRC / s) for s in CUDA_SOURCES]]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    return LIB


def build_torch_binding(verbose: bool = False) -> Path:
    """torch.utils.cpp_extension -> _trring_torch.so, linked against libtrring.so."""
    from torch.utils import cpp_extension

    build_dir = PKG / "_build"
    build_dir.mkdir(exist_ok=True)
    cpp_extension.load(
        name="_trring_torch",
        sources=[str(CSRC / "torch_ext.cpp")],
        extra_include_paths=[str(INCLUDE)],
        extra_cflags=["-O3"],
        # ninja turns $$ into $ and the shell turns \$ into $: the rpath reads $ORIGIN:$ORIGIN/..
        extra_ldflags=[f"-L{PKG}", "-ltrring", "-Wl,-rpath,\\$$ORIGIN:\\$$ORIGIN/.."],
        build_directory=str(build_dir),
        with_cuda=True,
        verbose=verbose,
    )
    built = build_dir / "_trring_torch.so"
    shutil.copy2(built, EXT)
    return EXT


def build(verbose: bool = False) -> None:
    build_library(verbose)
    build_torch_binding(verbose)


if __name__ == "__main__":
    build(verbose="-v" in sys.argv)
    print(f"built {LIB.name} and {EXT.name} in {PKG}")
