"""The drop-in boundary driven by the reference's own callers.

The patch that INTEGRATION.md section 1 documents for the reference's submission.py (its
`prepare_optimized` sends CUDA fp16/bf16 cores to kernel_task_b200 and keeps its own path for the
rest) is applied to a temporary copy of the reference tree, then:
  * the reference's own test suite (tests/test_correctness.py, tests/test_benchmark.py) runs
    against it: on a CPU machine its CPU cases, on a GPU machine also its required CUDA
    workloads (test_correctness.py:68-77), which then execute this library's kernels;
  * (GPU) one case of the reference's harness, benchmarks/benchmark.py, whose
    factorized_optimized method then is this library, checked by the harness's own FP32 dense
    oracle (benchmark.py:176-185).
The reference tree comes from $REFERENCE_SRC (the reference's root) or from the copy that
baseline/build_reference.py leaves in baseline/_ref/tree; without either the tests skip.
"""
from __future__ import annotations

import json
import os
import re
import shutil
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def reference_tree() -> Path | None:
    for cand in (os.environ.get("REFERENCE_SRC"), ROOT / "baseline" / "_ref" / "tree"):
        if cand and (Path(cand) / "src" / "factorized_inference" / "submission.py").exists() \
                and (Path(cand) / "tests" / "test_correctness.py").exists():
            return Path(cand)
    return None


def integration_patch() -> str:
    """The code block of INTEGRATION.md section 1 (the patched prepare_optimized)."""
    text = (ROOT / "INTEGRATION.md").read_text()
    m = re.search(r"```python\n# src/factorized_inference/submission.py\n(.*?)```", text, re.S)
    assert m, "INTEGRATION.md section 1 lost its submission.py block"
    return m.group(1)


@pytest.fixture(scope="module")
def patched_tree(tmp_path_factory):
    src = reference_tree()
    if src is None:
        pytest.skip("reference tree not available (REFERENCE_SRC or baseline/_ref/tree)")
    dst = tmp_path_factory.mktemp("reference")
    for part in ("src", "tests", "benchmarks"):
        shutil.copytree(src / part, dst / part,
                        ignore=shutil.ignore_patterns("__pycache__", "*.pyc", "build"))
    sub = dst / "src" / "factorized_inference" / "submission.py"
    text = sub.read_text()
    assert text.count("def prepare_optimized(") == 1
    text = text.replace("def prepare_optimized(", "def _reference_prepare(")
    sub.write_text(text + "\n\n" + integration_patch())
    return dst


def _env(tree: Path) -> dict:
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join([str(tree / "src"), str(ROOT)])
    env.pop("REFERENCE_SRC", None)
    return env


def test_reference_test_suite_through_the_patch(patched_tree):
    """The reference's own tests pass with its submission.py patched to this library."""
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-p", "no:cacheprovider",
                        "tests/test_correctness.py", "tests/test_benchmark.py"],
                       cwd=patched_tree, env=_env(patched_tree), capture_output=True, text=True,
                       timeout=900)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
    assert "passed" in r.stdout


@pytest.mark.gpu
def test_reference_cuda_workloads_run_this_library(patched_tree):
    """On a GPU the reference's required CUDA workloads run (not skipped), through the patch:
    the prepared callable is this library's operator."""
    probe = ("import torch\n"
             "from factorized_inference.submission import prepare_optimized\n"
             "from factorized_inference.reference import TRSpec, make_cores\n"
             "spec = TRSpec(rank=8)\n"
             "cores = make_cores(spec, device='cuda', dtype=torch.float16, seed=23)\n"
             "fn = prepare_optimized(cores, spec)\n"
             "print(type(fn).__module__, type(fn).__name__)\n")
    r = subprocess.run([sys.executable, "-c", probe], cwd=patched_tree, env=_env(patched_tree),
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    assert "RingOp" in r.stdout, r.stdout
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-p", "no:cacheprovider", "-rs",
                        "tests/test_correctness.py", "-k", "required_cuda_workloads"],
                       cwd=patched_tree, env=_env(patched_tree), capture_output=True, text=True,
                       timeout=900)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
    assert "5 passed" in r.stdout and "skipped" not in r.stdout, r.stdout[-1500:]


@pytest.mark.gpu
def test_reference_harness_case_through_the_patch(patched_tree, tmp_path):
    """One case of the reference's harness (benchmarks/benchmark.py: isolated child process per
    method, FP32 dense oracle after timing) with factorized_optimized = this library."""
    out = tmp_path / "results.json"
    # "cuda:0", not "cuda": the harness passes the device to torch.cuda.set_device, which on the
    # torch of this image (2.11; the reference pins 2.14) needs an index
    r = subprocess.run([sys.executable, "benchmarks/benchmark.py", "--device", "cuda:0",
                        "--dtype", "float16", "--rank", "8", "--tokens", "8", "--warmup", "5",
                        "--iterations", "10", "--event-block", "5", "--output", str(out)],
                       cwd=patched_tree, env=_env(patched_tree), capture_output=True, text=True,
                       timeout=900)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    res = json.loads(out.read_text())
    methods = res["cases"][0]["methods"]
    opt, ref = methods["factorized_optimized"], methods["factorized_reference"]
    assert opt["correctness"]["max_absolute_error"] < 0.02
    assert opt["cuda_event_stream_median_ms"] < ref["cuda_event_stream_median_ms"]
