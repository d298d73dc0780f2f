"""Install the reference (danila-permogorskii/kernel-task) into baseline/_ref and build its GPU
kernels for B200, so that its own code can be timed and tested beside this library.

    python baseline/build_reference.py [--src PATH]      (or REFERENCE_SRC=PATH)

Steps, all writing under baseline/_ref/ only (git-ignored; it travels to the GPU box with the
rest of the tree):
  1. ``pip install --no-index --no-build-isolation --no-deps --find-links /opt/wheelhouse
     --target baseline/_ref/site <src>``: the reference package as its own installer lays it
     out.  ``--no-deps``: the reference pins torch 2.14.0, this image has 2.11.0.
  2. A copy of the reference's ``src/``, ``tests/``, ``benchmarks/`` and ``pyproject.toml``
     under baseline/_ref/tree: the installed wheel carries no ``csrc/`` (the CUDA sources are
     not package data), and the reference's own tests and harness drive the drop-in boundary
     (tests/test_reference_callers.py).
  3. The reference's extension ``tr_ring_ext`` (src/factorized_inference/csrc/tr_ring.cu)
     built by the reference's own loader, ``factorized_inference.tr_kernel.load_extension``
     (tr_kernel.py:34-54: torch JIT, ``-O3 -lineinfo``), with TORCH_CUDA_ARCH_LIST=10.0, the
     arch torch picks on a B200.  The V3G extension (csrc/v3g, ~750 variants for the tuned
     5120-hidden shapes) is not built: no benchmark shape here takes that branch
     (tr_kernel.py:215-228 looks the shape up in V3G_TUNED first).

Nothing here is imported by the library.  bench.py (the reference-kernel leg) and
tests/test_reference_callers.py load the built module from baseline/_ref/tree/build in a child
process, never in the process that runs this library's kernels.
"""
from __future__ import annotations

import argparse
import json
import os
import shutil
import subprocess
import sys
import time
from pathlib import Path

HERE = Path(__file__).resolve().parent
REF = HERE / "_ref"
TREE = REF / "tree"
SITE = REF / "site"
EXT_DIR = TREE / "build" / "tr_ring_ext"


def built_extension() -> Path | None:
    """Path of the built reference extension, or None when it was not built."""
    so = EXT_DIR / "tr_ring_ext.so"
    return so if so.exists() else None


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--src", default=os.environ.get("REFERENCE_SRC"),
                    help="reference source tree (or REFERENCE_SRC)")
    ap.add_argument("--skip-build", action="store_true", help="install and copy only")
    a = ap.parse_args()
    if not a.src or not Path(a.src).is_dir():
        print("build_reference: give the reference source with --src or REFERENCE_SRC",
              file=sys.stderr)
        return 2
    src = Path(a.src).resolve()
    REF.mkdir(parents=True, exist_ok=True)
    record = {"src": str(src), "when": time.strftime("%Y-%m-%dT%H:%M:%SZ", time.gmtime())}

    # 1. pip install (the reference's own packaging)
    if SITE.exists():
        shutil.rmtree(SITE)
    cmd = [sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation",
           "--no-deps", "--find-links", "/opt/wheelhouse", "--target", str(SITE), str(src)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    record["pip_install"] = {"rc": r.returncode, "tail": r.stdout.strip().splitlines()[-1:]}
    if r.returncode != 0:
        record["pip_install"]["stderr"] = r.stderr.strip().splitlines()[-3:]

    # 2. the tree copy (CUDA sources, tests, harness)
    if TREE.exists():
        shutil.rmtree(TREE)
    TREE.mkdir(parents=True)
    for part in ("src", "tests", "benchmarks"):
        shutil.copytree(src / part, TREE / part,
                        ignore=shutil.ignore_patterns("__pycache__", "*.pyc"))
    shutil.copy2(src / "pyproject.toml", TREE / "pyproject.toml")

    # 3. the extension, through the reference's own loader
    if not a.skip_build:
        env = dict(os.environ, TORCH_CUDA_ARCH_LIST="10.0", PYTHONPATH=str(TREE / "src"))
        t0 = time.time()
        r = subprocess.run(
            [sys.executable, "-c",
             "from factorized_inference.tr_kernel import load_extension; "
             "m = load_extension(); print(m.__file__)"],
            env=env, capture_output=True, text=True, cwd=str(TREE))
        record["extension"] = {"rc": r.returncode, "seconds": round(time.time() - t0, 1),
                               "arch": "TORCH_CUDA_ARCH_LIST=10.0 (sm_100)",
                               "so": str(built_extension()) if built_extension() else None}
        if r.returncode != 0:
            record["extension"]["stderr"] = r.stderr.strip().splitlines()[-5:]
    (REF / "build_record.json").write_text(json.dumps(record, indent=1))
    print(json.dumps(record, indent=1))
    return 0 if record["pip_install"]["rc"] == 0 and (
        a.skip_build or record["extension"]["rc"] == 0) else 1


if __name__ == "__main__":
    sys.exit(main())
