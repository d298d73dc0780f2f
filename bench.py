"""Benchmark of the tensor-ring operator on B200 -- one JSON line on rank 0.

Headline workload: CUDA-event microseconds per call of the fused operator on the 1920->2880
ring, modes (8,12,20)->(12,10,24), fp16, at R=8 with T=1/8/32 and at R=16 with T=1/32, next to
cuBLAS dense fp16 GEMM of the same (d_in, d_out) and to the reference's own GPU kernels.
Synthetic, seeded: cores N(0, sigma^2) with sigma = (R*d_in^(1/3))^(-1/2), x ~ N(0,1).

Per case:
  value leg     one call per step, L2 flushed (256 MiB write) before every step, CUDA events
                around the call on the launching stream: device time of a cold-cache call.
  warm leg      the reference harness's protocol: 5 blocks x 20 back-to-back calls, median
                (benchmarks/benchmark.py:163-174).
  e2e leg       the public API end to end on host buffers: pinned host x -> device, the
                operator, y -> pinned host, after an L2 flush and with the GPU idle, so host
                dispatch is inside the region.  Our operator takes the host buffers in one call
                (fn.forward_host: tr_forward_host issues both copies and the kernel); the same
                through torch copies around fn(x) is reported beside it (e2e_torch_copies_us).
  dense bar     F.linear(x, W) on the materialised fp16 W, same legs (TF32 off).
  reference     the reference's own PreparedTRKernel (its tr_ring.cu built for sm_100 by
                baseline/build_reference.py) in a child process: default dispatch, and with the
                V3 tiling forced at T=1 (TR_KC/TR_QC/TR_TT; its tuned table applies to sm_90
                only, tr_kernel.py:134-139); and its factorized torch path on the GPU.
Extra objects on the line:
  config3          4096->14336 (16,16,16)->(16,28,32) R32 bf16 at T=1/8/32/128/256: ours, dense
                   bf16 and fp16, the reference's generic kernel;
  sharded_prefill  config 5, token-sharded over the ranks;
  decode_chain     config 4: a T=1 decode step through several layers, fused consumers vs the
                   reference's separate consumer launches vs dense bf16;
  c1_chain         1920->2880->1920 up/down layers at R8, T=1: per-layer time from stream
                   launches and from a CUDA graph, against dense fp16 (the launch share a
                   persistent multi-layer kernel could remove);
  premerge         the optional G1.G2 pre-merge measured as two cuBLAS GEMMs next to the
                   fused operator (c1/c2 at T = 8/32);
  cpu_baseline     the reference's CPU contraction at 1 thread and at all host threads.
value = mean over the five cases of the mean value-leg time (the device timer on this part ticks
in ~2 us steps, so single-call medians are quantised; means over the steps are not).
ms_per_step = one call of each case.  --impl reference times the reference's CPU path on the
host cores instead.  Under torchrun (N>1) every rank serves its own replica of the suite
(tokens are independent, no collective on the data path); times are the max over ranks.
--profile-case runs one seeded operator a few times for a profiler (see profiles/).
"""
from __future__ import annotations

import argparse
import json
import os
import platform
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = ("CUDA-event µs/call at T=1/8/32 (r8), T=1/32 (r16) vs cuBLAS dense fp16 GEMM")
WORKLOAD = ("c1+c2 decode suite: 1920->2880 (8,12,20)->(12,10,24), R8 T=1/8/32 and R16 "
            "T=1/32, fp16 (CPU legs fp32)")
CASES = [(8, 1), (8, 8), (8, 32), (16, 1), (16, 32)]
C3_TOKENS = (1, 8, 32, 128, 256)
H100_PUBLISHED = {(8, 1): 8.2, (8, 8): 12.3, (8, 32): 27.9, (16, 1): 10.7, (16, 32): 82.4}
FLUSH_BYTES = 256 << 20
KERNEL_NAMES = {1: "ring_generic_kernel", 2: "ring_mma_kernel", 3: "ring_tc05_kernel",
                4: "ring_decode_kernel", 5: "ring_slab_kernel"}
# the reference install (baseline/build_reference.py); absent -> those legs report why
REF_SITE = ROOT / "baseline" / "_ref" / "site"
REF_EXT = ROOT / "baseline" / "_ref" / "tree" / "build" / "tr_ring_ext" / "tr_ring_ext.so"
# the V3 tilings of the reference's published T=1 runs (its H100_TUNED values), forced
REF_FORCED = {8: {"TR_KC": "2", "TR_QC": "4", "TR_TT": "1"},
              16: {"TR_KC": "4", "TR_QC": "4", "TR_TT": "1"}}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--no-dense", action="store_true")
    ap.add_argument("--no-reference-kernels", action="store_true",
                    help="skip the reference's GPU kernels (child processes)")
    ap.add_argument("--chain-layers", type=int, default=4,
                    help="layers of the config-4 decode chain leg (0 = skip)")
    ap.add_argument("--prefill-tokens", type=int, default=65536,
                    help="tokens of the sharded prefill leg (config 5), split over the ranks; "
                         "0 skips it")
    ap.add_argument("--c3-tokens", default=",".join(map(str, C3_TOKENS)),
                    help="token counts of the config-3 leg ('' skips it)")
    # internal: one leg of the reference's GPU code in a child process
    ap.add_argument("--ref-child", choices=("default", "forced", "torch"), default=None,
                    help=argparse.SUPPRESS)
    # --profile-case: one seeded operator, a few calls (for ncu)
    ap.add_argument("--profile-case", action="store_true")
    ap.add_argument("--rank", type=int, default=8)
    ap.add_argument("--tokens", type=int, default=1)
    ap.add_argument("--input-modes", default="8,12,20")
    ap.add_argument("--output-modes", default="12,10,24")
    ap.add_argument("--dtype", default="float16", choices=("float16", "bfloat16", "float32"))
    ap.add_argument("--calls", type=int, default=5)
    ap.add_argument("--tiling", default=None, help="kernel,TT,CL,NC forced geometry")
    return ap.parse_args()


def reference_flops(spec):
    """FLOPs per token by the reference's own count, 2(ni nj nk P R^2 + nj nk P Q R^3 +
    P Q Rr nk R^2) (tools/measure_kernels.py:36-44), reported beside the chosen order's."""
    (ni, nj, nk), (P, Q, Rr), R = spec.input_modes, spec.output_modes, spec.rank
    return 2 * (ni * nj * nk * P * R * R + nj * nk * P * Q * R ** 3 + P * Q * Rr * nk * R * R)


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return (d.get("hbm_gbs", 6650.0), d.get("bf16_tflops", 1590.0),
                d.get("bf16_tflops_sustained", 1400.0), "measured")
    return 6650.0, 1590.0, 1400.0, "fallback"


def clock_index(local_rank: int) -> int:
    """nvidia-smi's index of this process's GPU (CUDA_VISIBLE_DEVICES renumbers torch's)."""
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    return int(vis.split(",")[local_rank]) if vis else local_rank


class Clocks:
    """nvidia-smi sampling during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={index}", f"--query-gpu={self.Q}", "--format=csv,noheader",
                 "-lms", "100"], stdout=self.file, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def wait_first_sample(self, timeout_s: float = 5.0) -> None:
        """nvidia-smi needs a moment to start: block until it has written a line."""
        t_end = time.perf_counter() + timeout_s
        while self.proc is not None and time.perf_counter() < t_end:
            self.file.flush()
            if os.path.getsize(self.file.name) > 0:
                return
            time.sleep(0.05)

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.file.flush()
        self.file.seek(0)
        sm, smax, watts, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.file.read().splitlines():
            f = [v.strip() for v in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1].split()[0]))
                smax.append(float(f[2].split()[0]))
            except ValueError:
                continue
            try:
                watts.append(float(f[3].split()[0]))
            except ValueError:
                pass
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        os.unlink(self.file.name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None, "reasons": sorted(reasons),
                "samples": len(sm), "power_w": statistics.median(watts) if watts else None}


def dense_weight(cores):
    """The equivalent dense W [d_out, d_in] (the performance bar only; fp32 accumulate)."""
    A, B, C = (c.float() for c in cores)
    part = torch.einsum("apib,bqjc->apiqjc", A, B)
    W = torch.einsum("apiqjc,crka->pqrijk", part, C)
    P, Q, Rr, ni, nj, nk = W.shape
    return W.reshape(P * Q * Rr, ni * nj * nk).to(cores[0].dtype)


def cold_device_us(fn, x, flush, steps, warmup):
    """Per-call device time with L2 flushed before every call (flush outside the events)."""
    for _ in range(warmup):
        flush.add_(1)
        fn(x)
    torch.cuda.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(steps)]
    for s, e in evs:
        flush.add_(1)
        s.record()
        fn(x)
        e.record()
    torch.cuda.synchronize()
    return [s.elapsed_time(e) * 1e3 for s, e in evs]


def warm_stream_us(fn, x, blocks=5, per_block=20):
    for _ in range(20):
        fn(x)
    out = []
    for _ in range(blocks):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        s.record()
        for _ in range(per_block):
            fn(x)
        e.record()
        e.synchronize()
        out.append(s.elapsed_time(e) * 1e3 / per_block)
    return statistics.median(out)


def e2e_us(fn, x_host, flush, steps, warmup, d_out, host_call=True):
    """Public API end to end with host buffers: pinned x -> device, the operator, y -> pinned
    host, the GPU idle and L2 flushed at the start of every step.  With host_call, our operator
    takes the host buffers in one call, fn.forward_host(x, out=y) (tr_forward_host: both copies
    and the kernel); otherwise torch copies around fn(x) (the dense bar, and our operator for
    comparison)."""
    dev = flush.device
    x_dev = torch.empty(x_host.shape, dtype=x_host.dtype, device=dev)
    y_host = torch.empty((x_host.shape[0], d_out), dtype=x_host.dtype, pin_memory=True)
    direct = host_call and hasattr(fn, "forward_host")
    res = []
    for i in range(warmup + steps):
        flush.add_(1)
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        if direct:
            fn.forward_host(x_host, y_host)
        else:
            x_dev.copy_(x_host, non_blocking=True)
            y = fn(x_dev)
            y_host.copy_(y, non_blocking=True)
        e.record()
        e.synchronize()
        if i >= warmup:
            res.append(s.elapsed_time(e) * 1e3)
    return res, x_host.numel() * x_host.element_size(), y_host.numel() * y_host.element_size()


def host_latency_us(fn, x, n=100):
    lat = []
    for _ in range(n):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        fn(x)
        torch.cuda.synchronize()
        lat.append((time.perf_counter() - t0) * 1e6)
    return statistics.median(lat)


def max_over_ranks(vals, world):
    if world == 1:
        return vals
    t = torch.tensor(vals, dtype=torch.float64, device="cuda")
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return t.tolist()


def rel_frob(y, ref):
    import numpy as np

    y = y.double().cpu().numpy() if isinstance(y, torch.Tensor) else y
    ref = ref.double().cpu().numpy() if isinstance(ref, torch.Tensor) else ref
    return float(np.linalg.norm(y - ref) / np.linalg.norm(ref))


def reference_rows_check(x, y, cores, spec, rows):
    """Relative Frobenius error of rows `rows` of y against the reference's own CPU contraction
    (fp32, from the install in baseline/_ref); None when the reference is not installed."""
    if not (REF_SITE / "factorized_inference" / "reference.py").exists():
        return None
    run, _, _ = reference_cpu_forward()
    with torch.inference_mode():
        ref = run(x[rows].float().cpu(), [c.float().cpu() for c in cores], spec)
    return float(f"{rel_frob(y[rows], ref):.3g}")


# ------------------------------------------------------------------------- the CPU baseline
def cpu_info() -> dict:
    model = platform.processor() or platform.machine()
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                model = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    return {"cpu_model": model, "cpu_count": os.cpu_count()}


def reference_cpu_forward():
    """The reference's own factorized contraction on the CPU (tr_forward_reference,
    reference.py:99-125, torch fp32) from the install in baseline/_ref; without the install,
    the numpy restatement in oracle/ (same three contractions, same order)."""
    if (REF_SITE / "factorized_inference" / "reference.py").exists():
        if str(REF_SITE) not in sys.path:
            sys.path.insert(0, str(REF_SITE))
        from factorized_inference.reference import TRSpec as RefSpec
        from factorized_inference.reference import tr_forward_reference

        def run(x, cores, spec):
            return tr_forward_reference(x, cores, RefSpec(spec.input_modes, spec.output_modes,
                                                          spec.rank))
        return run, "reference", "tr_forward_reference (reference.py:99-125), torch fp32"
    import oracle

    def run(x, cores, spec):
        return oracle.tr_forward_reference(x.numpy(), [c.numpy() for c in cores])
    return run, "port", "numpy restatement of tr_forward_reference (oracle/), fp32"


def cpu_leg(threads: int, warm: int = 3, samples: int = 20):
    """The reference's CPU contraction per case with `threads` host threads: 3 warm-up calls,
    then the median of `samples` perf_counter samples (the harness protocol)."""
    from threadpoolctl import threadpool_limits

    from kernel_task_b200.spec import TRSpec, baseline_cores, baseline_x

    run, kind, what = reference_cpu_forward()
    prev = torch.get_num_threads()
    torch.set_num_threads(threads)
    per_case = {}
    try:
        with threadpool_limits(limits=threads):
            for R, T in CASES:
                spec = TRSpec((8, 12, 20), (12, 10, 24), R)
                cores = [c.float() for c in baseline_cores(spec, seed=0, dtype=torch.float32)]
                x = baseline_x(spec, T, seed=0, dtype=torch.float32)
                with torch.inference_mode():
                    for _ in range(warm):
                        run(x, cores, spec)
                    lat = []
                    for _ in range(samples):
                        t0 = time.perf_counter()
                        run(x, cores, spec)
                        lat.append((time.perf_counter() - t0) * 1e6)
                per_case[f"r{R}_t{T}"] = round(statistics.median(lat), 2)
    finally:
        torch.set_num_threads(prev)
    return statistics.mean(per_case.values()), per_case, kind, what


def cpu_baseline_object():
    threads = os.cpu_count() or 1
    v_all, cases_all, kind, what = cpu_leg(threads)
    v_one, cases_one, _, _ = cpu_leg(1)
    return {"value": round(v_all, 2), "unit": "us/call", "cores": threads, "kind": kind,
            "sample": f"{what}; each of the 5 suite cases, 3 warm-up calls then the median of "
                      "20 calls; value = mean over the cases at all host threads",
            "cases": cases_all,
            "one_thread": {"value": round(v_one, 2), "cores": 1, "cases": cases_one},
            **cpu_info()}


def run_reference(args, rank):
    """--impl reference: the reference's CPU path on the host cores (rank 0 only)."""
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    run, kind, what = reference_cpu_forward()
    from threadpoolctl import threadpool_limits

    from kernel_task_b200.spec import TRSpec, baseline_cores, baseline_x

    torch.set_num_threads(threads)
    per_case = {}
    with threadpool_limits(limits=threads), torch.inference_mode():
        for R, T in CASES:
            spec = TRSpec((8, 12, 20), (12, 10, 24), R)
            cores = [c.float() for c in baseline_cores(spec, seed=0, dtype=torch.float32)]
            x = baseline_x(spec, T, seed=0, dtype=torch.float32)
            for _ in range(max(1, args.warmup)):
                run(x, cores, spec)
            lat, t_end = [], time.perf_counter() + 2.0
            while len(lat) < max(3, min(args.steps, 20)) or (time.perf_counter() < t_end
                                                              and len(lat) < args.steps):
                t0 = time.perf_counter()
                run(x, cores, spec)
                lat.append((time.perf_counter() - t0) * 1e6)
            per_case[f"r{R}_t{T}"] = {"us": round(statistics.median(lat), 2), "calls": len(lat)}
    value = statistics.mean(v["us"] for v in per_case.values())
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 2), "unit": "us/call",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(sum(v["us"] for v in per_case.values()) / 1e3, 4),
        "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,sigma^2) cores, N(0,1) x)",
        "config": {"workload": WORKLOAD, "cases": per_case},
        "cpu_baseline": {"value": round(value, 2), "unit": "us/call", "cores": threads,
                         "kind": kind, "sample": f"{what}; each of the 5 suite cases, median "
                         "of repeated calls (at least 3, up to the step count within ~2 s)"},
        "e2e": {"value": round(value, 2), "unit": "us/call", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        **cpu_info(),
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------- the reference's GPU code (children)
def _load_reference_gpu():
    """The reference package from baseline/_ref with its prebuilt extension preloaded into
    tr_kernel._ext (the module load_extension would JIT-build; tr_kernel.py:34-54)."""
    import importlib.machinery
    import importlib.util

    if not REF_EXT.exists() or not (REF_SITE / "factorized_inference").exists():
        raise RuntimeError("reference not installed: run baseline/build_reference.py")
    sys.path.insert(0, str(REF_SITE))
    loader = importlib.machinery.ExtensionFileLoader("tr_ring_ext", str(REF_EXT))
    spec = importlib.util.spec_from_file_location("tr_ring_ext", str(REF_EXT), loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    import factorized_inference.tr_kernel as trk

    trk._ext = mod
    from factorized_inference import reference, submission

    return submission, reference


def ref_child(args):
    """One child-process leg of the reference's GPU code; prints one JSON line.
      default  PreparedTRKernel through submission.prepare_optimized, c1/c2 fp16 and c3 bf16
      forced   the same at T=1 with the V3 tiling forced (TR_KC/TR_QC/TR_TT)
      torch    tr_forward_reference on the GPU (its torch einsum path), same cases"""
    import warnings

    from kernel_task_b200.spec import SPEC_C3, TRSpec, baseline_cores, baseline_x

    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction = False
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    flush = torch.empty(FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    try:
        submission, reference = _load_reference_gpu()
    except Exception as e:  # noqa: BLE001 -- reported on the line
        print(json.dumps({"unavailable": str(e)[:300]}), flush=True)
        return
    cases = [(f"r{R}_t{T}", TRSpec((8, 12, 20), (12, 10, 24), R), T, torch.float16)
             for R, T in CASES]
    cases += [(f"c3_t{T}", SPEC_C3, T, torch.bfloat16) for T in C3_TOKENS]
    if args.ref_child == "forced":
        cases = [c for c in cases if c[2] == 1 and c[0].startswith("r")]
    out = {}
    for name, spec, T, dtype in cases:
        rspec = reference.TRSpec(spec.input_modes, spec.output_modes, spec.rank)
        cores = baseline_cores(spec, seed=0, dtype=dtype, device=dev)
        x = baseline_x(spec, T, seed=0, dtype=dtype, device=dev)
        env_prev = {}
        if args.ref_child == "forced":
            for k, v in REF_FORCED[spec.rank].items():
                env_prev[k] = os.environ.get(k)
                os.environ[k] = v
        rec = {}
        try:
            with warnings.catch_warnings(record=True) as w:
                warnings.simplefilter("always")
                if args.ref_child == "torch":
                    fn = lambda v, c=cores, s=rspec: reference.tr_forward_reference(v, c, s)  # noqa
                else:
                    fn = submission.prepare_optimized(cores, rspec)
                with torch.inference_mode():
                    y = fn(x)
                    torch.cuda.synchronize()
                    big = T > 32
                    steps = 3 if big else min(args.steps, 20)
                    rec["us"] = round(statistics.mean(cold_device_us(fn, x, flush, steps, 2)), 3)
                    if not big:
                        rec["warm_stream_us"] = round(warm_stream_us(fn, x), 3)
                rec["fallback_warnings"] = [str(m.message)[:120] for m in w][:2]
            rec["rel_frob"] = reference_rows_check(x, y, cores, spec, list(range(min(T, 4))))
            if args.ref_child != "torch":
                rec["tiling"] = list(fn._tiling.get(T) or ()) if hasattr(fn, "_tiling") else None
        except Exception as e:  # noqa: BLE001 -- one failing case does not hide the others
            rec = {"error": f"{type(e).__name__}: {str(e)[:200]}"}
        finally:
            for k, v in env_prev.items():
                if v is None:
                    os.environ.pop(k, None)
                else:
                    os.environ[k] = v
        out[name] = rec
        del cores, x
        torch.cuda.empty_cache()
    print(json.dumps({"mode": args.ref_child, "cases": out}), flush=True)


def reference_gpu_legs(args) -> dict:
    """Runs each leg of the reference's GPU code in its own child process, so that the
    reference's extension never maps into the process that runs this library's kernels (as its
    harness isolates each method, benchmarks/benchmark.py:263-283)."""
    if not REF_EXT.exists():
        return {"unavailable": "reference extension not built (baseline/build_reference.py)"}
    res = {}
    for mode in ("default", "forced", "torch"):
        cmd = [sys.executable, str(ROOT / "bench.py"), "--ref-child", mode,
               "--steps", str(args.steps)]
        try:
            p = subprocess.run(cmd, capture_output=True, text=True, timeout=900, cwd=str(ROOT))
            lines = [ln for ln in p.stdout.splitlines() if ln.startswith("{")]
            res[mode] = json.loads(lines[-1]) if lines else {
                "error": f"rc={p.returncode}: {p.stderr.strip()[-300:]}"}
        except subprocess.TimeoutExpired:
            res[mode] = {"error": "timed out after 900 s"}
    return res


# ---------------------------------------------------------------------- the extra legs
def prefill_leg(args, rank, world, dev, tc_peak, tc_sustained):
    """Config 5: 4096 -> 14336, modes (16,16,16)->(16,28,32), R16, bf16, `--prefill-tokens`
    tokens split over the ranks (ShardedRing row split, cores replicated, no collective on the
    data path).  Device time per call (CUDA events), max over ranks; one all_gather of y timed
    separately when world > 1."""
    from kernel_task_b200 import prepare_optimized
    from kernel_task_b200.shard import ShardedRing, shard_bounds
    from kernel_task_b200.spec import SPEC_C5, baseline_cores

    T = args.prefill_tokens
    a, b = shard_bounds(T, world, rank)
    cores = baseline_cores(SPEC_C5, seed=0, dtype=torch.bfloat16, device=dev)
    op = ShardedRing(cores, SPEC_C5, op_factory=prepare_optimized)
    gen = torch.Generator(device=dev)
    gen.manual_seed(5000 + rank)
    x = torch.randn(b - a, SPEC_C5.in_features, generator=gen, device=dev).to(torch.bfloat16)
    for _ in range(2):
        op.local(x)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    steps = max(1, min(args.steps, 3))
    times = []
    # clocks and power of this leg alone: a seconds-long tensor-core load, where a slower box
    # (power cap, temperature) shows in the SM clock
    clocks = Clocks(clock_index(dev.index if dev.index is not None else 0))
    clocks.wait_first_sample()
    for _ in range(steps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        y = op.local(x)
        e1.record()
        e1.synchronize()
        times.append(e0.elapsed_time(e1))
    clk = clocks.stop()
    ms = max_over_ranks([statistics.mean(times)], world)[0]
    out = {"workload": "c5: 4096->14336 (16,16,16)->(16,28,32) R16 bf16, tokens split by rows, "
                       "cores replicated per GPU",
           "tokens": T, "tokens_per_rank_max": shard_bounds(T, world, 0)[1],
           "ms": round(ms, 3), "tokens_per_s": round(T / (ms * 1e-3), 1),
           "steps": steps, "scaling": "strong", "timing": "CUDA events, max over ranks",
           "kernel": KERNEL_NAMES.get(op.fn.tiling(b - a)["kernel"], "?"),
           "tiling": op.fn.tiling(b - a), "clocks": clk}
    flops = op.fn.flops_per_token() * shard_bounds(T, world, 0)[1]
    tf = flops / (ms * 1e-3) / 1e12
    out["tflops_per_gpu"] = round(tf, 2)
    out["frac_of_peak"] = round(tf / tc_peak, 4)
    out["frac_of_sustained_peak"] = round(tf / tc_sustained, 4)
    # parity at full size: sampled rows of rank 0's shard against the reference's CPU path
    if rank == 0:
        out["sampled_rows_rel_frob"] = reference_rows_check(
            x, y, cores, SPEC_C5, [0, (b - a) // 3, (b - a) - 1])
    if world > 1:
        rows_max = shard_bounds(T, world, 0)[1]
        padded = y.new_zeros((rows_max, SPEC_C5.out_features))
        padded[: b - a] = y
        parts = [torch.empty_like(padded) for _ in range(world)]
        torch.distributed.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        torch.distributed.all_gather(parts, padded)
        e1.record()
        e1.synchronize()
        out["gather_ms"] = round(max_over_ranks([e0.elapsed_time(e1)], world)[0], 3)
        del parts, padded
    del x, y, op
    torch.cuda.empty_cache()
    return out


def c3_leg(dev, flush, tokens, tc_peak, dense=True):
    """Config 3: 4096 -> 14336, modes (16,16,16)->(16,28,32), R32, bf16 (seeded benchmark
    inputs): cold device time per call (L2 flushed), our kernel and the dense bars."""
    from kernel_task_b200 import prepare_optimized
    from kernel_task_b200.spec import SPEC_C3, baseline_cores, baseline_x

    cores = baseline_cores(SPEC_C3, seed=0, dtype=torch.bfloat16, device=dev)
    fn = prepare_optimized(cores, SPEC_C3)
    W16 = Wb = None
    if dense:
        Wb = dense_weight(cores)
        W16 = Wb.to(torch.float16)
    out = {"workload": "c3: 4096->14336 (16,16,16)->(16,28,32) R32 bf16", "cases": {}}
    for T in tokens:
        x = baseline_x(SPEC_C3, T, seed=0, dtype=torch.bfloat16, device=dev)
        steps = 3 if T >= 128 else 10
        us = statistics.mean(cold_device_us(fn, x, flush, steps, 2))
        flops = fn.flops_per_token() * T
        rec = {"us": round(us, 3), "kernel": KERNEL_NAMES.get(fn.tiling(T)["kernel"], "?"),
               "tiling": fn.tiling(T), "tflops": round(flops / (us * 1e-6) / 1e12, 2),
               "frac_of_peak": round(flops / (us * 1e-6) / 1e12 / tc_peak, 4)}
        if dense:
            x16 = x.to(torch.float16)
            rec["dense_bf16_us"] = round(statistics.mean(cold_device_us(
                lambda v: torch.nn.functional.linear(v, Wb), x, flush, steps, 2)), 3)
            rec["dense_fp16_us"] = round(statistics.mean(cold_device_us(
                lambda v: torch.nn.functional.linear(v, W16), x16, flush, steps, 2)), 3)
        out["cases"][f"t{T}"] = rec
    del fn, W16, Wb
    torch.cuda.empty_cache()
    return out


def decode_chain_leg(dev, layers, T=1):
    """Config 4: one decode step (T=1, bf16, R16) through `layers` transformer layers of TR
    projections q, k, v, o, gate, up, down (distinct seeded cores per layer; 2.5 MB of packed
    cores a layer, L2-resident when warm).  Attention is not simulated (o reads q's output, as
    in the reference's chain, tools/qwen_model_chain.py:111-134).  Three orders, warm stream
    (5 blocks x 10 steps, median), microseconds per layer:
      fused      o/down with the residual add and up with silu(gate)*up in their own store,
                 gate in fp32: 7 launches a layer;
      unfused    the reference's order: accumulate (fp32) then consume_add / consume_silu_mul
                 launches: 10 launches a layer;
      dense      cuBLAS bf16 F.linear on dense weights of the same shapes (random values; the
                 time does not depend on them) with torch's add / silu / mul.
    The fused step is also captured in a CUDA graph and replayed."""
    import torch.nn.functional as F

    from kernel_task_b200 import consume_add, consume_silu_mul, prepare_optimized
    from kernel_task_b200.spec import SPEC_C4, baseline_cores, baseline_x

    names = ["q", "k", "v", "o", "gate", "up", "down"]
    L = [{n: prepare_optimized(baseline_cores(SPEC_C4[n], seed=100 * l + i,
                                              dtype=torch.bfloat16, device=dev), SPEC_C4[n])
          for i, n in enumerate(names)} for l in range(layers)]
    h0 = baseline_x(SPEC_C4["q"], T, seed=9, dtype=torch.bfloat16, device=dev)

    def fused(h):
        for ops in L:
            q = ops["q"](h)
            ops["k"](h)
            ops["v"](h)
            h = ops["o"].forward_add(q, h)
            act = ops["up"].forward_silu_mul(h, ops["gate"].accumulate(h))
            h = ops["down"].forward_add(act, h)
        return h

    def unfused(h):
        for ops in L:
            q = ops["q"](h)
            ops["k"](h)
            ops["v"](h)
            h = consume_add(h, ops["o"].accumulate(q))
            act = consume_silu_mul(ops["gate"].accumulate(h), ops["up"].accumulate(h))
            h = consume_add(h, ops["down"].accumulate(act))
        return h

    g = torch.Generator(device=dev).manual_seed(1)
    Ws = [{n: (torch.randn(SPEC_C4[n].out_features, SPEC_C4[n].in_features, generator=g,
                           device=dev) * 0.01).to(torch.bfloat16) for n in names}
          for _ in range(layers)]

    def dense(h):
        for W in Ws:
            q = F.linear(h, W["q"])
            F.linear(h, W["k"])
            F.linear(h, W["v"])
            h = h + F.linear(q, W["o"])
            h = h + F.linear(F.silu(F.linear(h, W["gate"])) * F.linear(h, W["up"]), W["down"])
        return h

    out = {"workload": f"config 4 decode step, T={T}, bf16, R16, {layers} layers "
                       "(q,k,v,o,gate,up,down; attention not simulated)",
           "launches_per_layer": {"fused": 7, "unfused": 10}}
    a, b = fused(h0), unfused(h0)
    rel = ((a.float() - b.float()).norm() / b.float().norm()).item()
    out["fused_vs_unfused_rel_frob"] = float(f"{rel:.3g}")
    for name, fn in (("fused", fused), ("unfused", unfused), ("dense_bf16", dense)):
        out[f"{name}_us_per_layer"] = round(warm_stream_us(fn, h0, 5, 10) / layers, 3)
    graph = _graph_of(fused, h0)
    if isinstance(graph, str):
        out["fused_graph_error"] = graph
    else:
        out["fused_graph_us_per_layer"] = round(
            warm_stream_us(lambda _: graph.replay(), None, 5, 10) / layers, 3)
        del graph
    del L, Ws
    torch.cuda.empty_cache()
    return out


def _graph_of(fn, arg):
    """CUDA graph of fn(arg) (warmed on a side stream), or an error string."""
    try:
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(3):
                fn(arg)
        torch.cuda.current_stream().wait_stream(s)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            fn(arg)
        return graph
    except RuntimeError as e:
        return str(e).splitlines()[0][:200]


def premerge_leg(dev, flush):
    """The optional G1.G2 pre-merge (north_star (a); bounded by IMPLEMENTATION.md:25 in the
    reference), measured instead of built: the merged core M[a,(i,j),(p,q),c] = sum_b
    A[a,p,i,b] B[b,q,j,c], then y by two cuBLAS GEMMs, X[(k,t),(i,j)] M[(i,j),(a,p,q,c)] and, after
    a permute, T12[(t,p,q),(k,a,c)] C[(k,a,c),r].  Cold device time per call next to the fused
    operator on the c1/c2 shapes at T = 8 and 32, with both forms' relative Frobenius error
    against the fp32 contraction."""
    from kernel_task_b200 import prepare_optimized
    from kernel_task_b200.spec import SPEC_C1, SPEC_C2, baseline_cores, baseline_x

    out = {}
    for spec in (SPEC_C1, SPEC_C2):
        cores = baseline_cores(spec, seed=0, dtype=torch.float16, device=dev)
        A, B, C = cores
        (ni, nj, nk), (P, Q, Rr), R = spec.input_modes, spec.output_modes, spec.rank
        M = torch.einsum("apib,bqjc->aijpqc", A.float(), B.float()).to(torch.float16)
        Mmat = M.permute(1, 2, 0, 3, 4, 5).reshape(ni * nj, R * P * Q * R).contiguous()
        Cmat = C.permute(2, 3, 0, 1).reshape(nk * R * R, Rr).contiguous()
        fn = prepare_optimized(cores, spec)
        for T in (8, 32):
            x = baseline_x(spec, T, seed=0, dtype=torch.float16, device=dev)

            def merged(x=x, T=T):
                xk = x.view(T, ni, nj, nk).permute(3, 0, 1, 2).reshape(nk * T, ni * nj)
                t12 = (xk @ Mmat).view(nk, T, R, P, Q, R)
                lhs = t12.permute(1, 3, 4, 0, 2, 5).reshape(T * P * Q, nk * R * R)
                return (lhs @ Cmat).view(T, P * Q * Rr)

            ym, yf = merged().float(), fn(x).float()
            ref = torch.einsum("tijk,apib,bqjc,crka->tpqr",
                               x.float().view(T, ni, nj, nk), A.float(), B.float(),
                               C.float()).reshape(T, -1)
            out[f"r{R}_t{T}"] = {
                "merged_us": round(statistics.mean(cold_device_us(lambda _v: merged(), None,
                                                                  flush, 30, 3)), 2),
                "fused_us": round(statistics.mean(cold_device_us(fn, x, flush, 30, 3)), 2),
                "merged_rel_frob": round(float((ym - ref).norm() / ref.norm()), 6),
                "fused_rel_frob": round(float((yf - ref).norm() / ref.norm()), 6),
                "merged_core_bytes": M.numel() * 2,
                "intermediate_bytes": nk * T * R * P * Q * R * 2}
    return out


def c1_chain_leg(dev, layers=16):
    """The reference's comparison point for a persistent multi-layer kernel: a chain of
    1920->2880 (up) and 2880->1920 (down) R8 fp16 layers at T=1 (kernel_work/stack,
    REPORT_TEMPLATE.md:307-310).  Microseconds per layer, warm: stream launches, CUDA-graph
    replay, and dense fp16 cuBLAS both ways; the empty-kernel floor for scale."""
    import torch.nn.functional as F

    from kernel_task_b200 import prepare_optimized
    from kernel_task_b200._native import binding
    from kernel_task_b200.spec import TRSpec, baseline_cores, baseline_x

    up, down = TRSpec((8, 12, 20), (12, 10, 24), 8), TRSpec((12, 10, 24), (8, 12, 20), 8)
    specs = [(up, down)[l % 2] for l in range(layers)]
    cores = [baseline_cores(s, seed=200 + l, dtype=torch.float16, device=dev)
             for l, s in enumerate(specs)]
    ops = [prepare_optimized(c, s) for c, s in zip(cores, specs)]
    Ws = [dense_weight(c) for c in cores]
    h0 = baseline_x(up, 1, seed=3, dtype=torch.float16, device=dev)

    def ring(h):
        for op in ops:
            h = op(h)
        return h

    def dense(h):
        for W in Ws:
            h = F.linear(h, W)
        return h

    empty = binding().empty_launch
    out = {"workload": f"{layers} alternating 1920->2880 / 2880->1920 R8 fp16 layers, T=1",
           "ring_stream_us_per_layer": round(warm_stream_us(ring, h0, 5, 10) / layers, 3),
           "dense_stream_us_per_layer": round(warm_stream_us(dense, h0, 5, 10) / layers, 3),
           "empty_kernel_stream_us": round(warm_stream_us(lambda _: empty(), None), 3)}
    for name, fn in (("ring", ring), ("dense", dense)):
        graph = _graph_of(fn, h0)
        if isinstance(graph, str):
            out[f"{name}_graph_error"] = graph
        else:
            out[f"{name}_graph_us_per_layer"] = round(
                warm_stream_us(lambda _: graph.replay(), None, 5, 10) / layers, 3)
            del graph
    del ops, Ws
    torch.cuda.empty_cache()
    return out


# ---------------------------------------------------------------------------- our arm
def run_ours(args, rank, world, local_rank):
    from kernel_task_b200 import prepare_optimized
    from kernel_task_b200.spec import TRSpec, baseline_cores, baseline_x

    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction = False
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    flush = torch.empty(FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    hbm_peak, tc_peak, tc_sustained, peak_kind = peaks()
    steps, warmup = args.steps, max(3, args.warmup)

    cases = {}
    for R, T in CASES:
        spec = TRSpec((8, 12, 20), (12, 10, 24), R)
        cores = baseline_cores(spec, seed=0, dtype=torch.float16, device=dev)
        x = baseline_x(spec, T, seed=0, dtype=torch.float16, device=dev)
        torch.cuda.synchronize()
        base_mem = torch.cuda.memory_allocated(dev)
        torch.cuda.reset_peak_memory_stats(dev)
        t0 = time.perf_counter()
        fn = prepare_optimized(cores, spec)
        torch.cuda.synchronize()
        prep_ms = (time.perf_counter() - t0) * 1e3
        t0 = time.perf_counter()
        fn(x)
        torch.cuda.synchronize()
        first_ms = (time.perf_counter() - t0) * 1e3
        peak = torch.cuda.max_memory_allocated(dev) - base_mem  # packed cores, workspace, y
        cases[(R, T)] = {"spec": spec, "cores": cores, "x": x, "fn": fn, "prep_ms": prep_ms,
                         "first_ms": first_ms, "peak_mem": int(peak)}

    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    clocks = Clocks(clock_index(local_rank))
    clocks.wait_first_sample()
    launches = 0
    for key, c in cases.items():
        c["cold"] = cold_device_us(c["fn"], c["x"], flush, steps, warmup)
        launches += steps
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()

    for key, c in cases.items():
        c["warm"] = warm_stream_us(c["fn"], c["x"])
        c["host"] = host_latency_us(c["fn"], c["x"])
        xh = c["x"].cpu().pin_memory()
        e2e, c["h2d"], c["d2h"] = e2e_us(c["fn"], xh, flush, steps, warmup,
                                          c["spec"].out_features)
        c["e2e"] = e2e
        # the same through torch copies around fn(x) (three host dispatches)
        c["e2e_torch_copies"] = statistics.mean(e2e_us(c["fn"], xh, flush, steps, warmup,
                                                       c["spec"].out_features,
                                                       host_call=False)[0])
        if not args.no_dense:
            W = dense_weight(c["cores"])
            dfn = lambda v, W=W: torch.nn.functional.linear(v, W)  # noqa: E731
            c["dense_cold"] = statistics.mean(cold_device_us(dfn, c["x"], flush, steps,
                                                             warmup))
            c["dense_warm"] = warm_stream_us(dfn, c["x"])
            c["dense_e2e"] = statistics.mean(e2e_us(dfn, xh, flush, steps, warmup,
                                                    c["spec"].out_features)[0])
            del W
        c["flops"] = c["fn"].flops_per_token() * c["x"].shape[0]
        c["tiling"] = c["fn"].tiling(c["x"].shape[0])

    # the launch floor: an empty kernel of this library, same legs (cold: after the L2 flush)
    from kernel_task_b200._native import binding

    empty = binding().empty_launch
    launch_cold = statistics.mean(cold_device_us(lambda _v: empty(), None, flush, steps, warmup))
    launch_warm = warm_stream_us(lambda _v: empty(), None)
    c3_tokens = [int(v) for v in args.c3_tokens.split(",") if v.strip()]
    c3 = (c3_leg(dev, flush, c3_tokens, tc_peak, dense=not args.no_dense)
          if c3_tokens and world == 1 else None)
    prefill = (prefill_leg(args, rank, world, dev, tc_peak, tc_sustained)
               if args.prefill_tokens > 0 else None)
    chain = (decode_chain_leg(dev, args.chain_layers)
             if args.chain_layers > 0 and world == 1 else None)
    c1_chain = c1_chain_leg(dev) if world == 1 and args.chain_layers > 0 else None
    premerge = premerge_leg(dev, flush) if world == 1 and not args.no_dense else None
    clk = clocks.stop()  # sampled from before the cold legs to the end of the chain legs
    keys = list(cases)
    med = max_over_ranks([statistics.median(cases[k]["cold"]) for k in keys], world)
    mean = max_over_ranks([statistics.mean(cases[k]["cold"]) for k in keys], world)
    e2e = max_over_ranks([statistics.mean(cases[k]["e2e"]) for k in keys], world)
    if rank != 0:
        return
    # the reference's GPU code, in child processes (after our legs, GPU otherwise idle)
    ref_gpu = (reference_gpu_legs(args) if world == 1 and not args.no_reference_kernels
               else None)
    # binding floor per case: max(launch floor, compulsory bytes / HBM, FLOPs / tensor peak)
    floors, warm_floors = [], []
    for k in keys:
        c = cases[k]
        spec_k, T_k = c["spec"], k[1]
        bytes_k = 2 * (spec_k.factor_parameters + T_k * (spec_k.in_features + spec_k.out_features))
        work = max(bytes_k / (hbm_peak * 1e9) * 1e6, c["flops"] / (tc_peak * 1e12) * 1e6)
        floors.append(max(launch_cold, work))
        warm_floors.append(max(launch_warm, work))
    per_case = {}
    for i, k in enumerate(keys):
        c = cases[k]
        R, T = k
        spec = c["spec"]
        name = f"r{R}_t{T}"
        bytes_min = 2 * (spec.factor_parameters + T * (spec.in_features + spec.out_features))
        rec = {
            "us": round(mean[i], 3), "us_median": round(med[i], 3),
            "warm_stream_us": round(c["warm"], 3), "host_latency_us": round(c["host"], 2),
            "e2e_us": round(e2e[i], 3),
            "e2e_torch_copies_us": round(c["e2e_torch_copies"], 3),
            "prep_ms": round(c["prep_ms"], 2),
            "kernel": KERNEL_NAMES.get(c["tiling"]["kernel"], "?"),
            "dense_us": round(c.get("dense_cold", float("nan")), 3),
            "dense_warm_stream_us": round(c.get("dense_warm", float("nan")), 3),
            "dense_e2e_us": round(c.get("dense_e2e", float("nan")), 3),
            "h100_published_warm_stream_us": H100_PUBLISHED[k],
            "flops": c["flops"], "min_bytes": bytes_min,
            "tflops": round(c["flops"] / (mean[i] * 1e-6) / 1e12, 2),
            "tiling": c["tiling"], "packed_bytes": int(c["fn"].packed.numel()),
            "workspace_bytes": int(c["fn"].workspace_bytes(T)),
            "first_call_ms": round(c["first_ms"], 3), "peak_mem_bytes": c["peak_mem"],
            "flops_reference_formula": reference_flops(spec) * T,
            "floor_us": round(floors[i], 3), "frac_of_floor": round(floors[i] / mean[i], 4),
            "warm_floor_us": round(warm_floors[i], 3),
            "warm_frac_of_floor": round(warm_floors[i] / c["warm"], 4),
        }
        if ref_gpu and "default" in ref_gpu:
            d = ref_gpu["default"].get("cases", {}).get(name, {})
            f = ref_gpu.get("forced", {}).get("cases", {}).get(name, {})
            t = ref_gpu.get("torch", {}).get("cases", {}).get(name, {})
            legs = [v for v in (d.get("us"), f.get("us")) if v is not None]
            if legs:
                rec["ref_kernel_us"] = min(legs)
                rec["ref_kernel_default_us"] = d.get("us")
                rec["ref_kernel_forced_us"] = f.get("us")
                warm = [v for v in (d.get("warm_stream_us"), f.get("warm_stream_us"))
                        if v is not None]
                rec["ref_kernel_warm_us"] = min(warm) if warm else None
                rec["ref_kernel_rel_frob"] = d.get("rel_frob")
            rec["ref_torch_us"] = t.get("us")
            rec["ref_torch_warm_us"] = t.get("warm_stream_us")
        per_case[name] = rec
    if c3 is not None and ref_gpu and "default" in ref_gpu:
        for name, rec in c3["cases"].items():
            d = ref_gpu["default"].get("cases", {}).get(f"c3_{name}", {})
            t = ref_gpu.get("torch", {}).get("cases", {}).get(f"c3_{name}", {})
            rec["ref_kernel_us"] = d.get("us", d.get("error"))
            rec["ref_kernel_rel_frob"] = d.get("rel_frob")
            rec["ref_torch_us"] = t.get("us", t.get("error"))
    # roofline of the dominant kernel: the case with the largest device time
    dom = max(range(len(keys)), key=lambda i: mean[i])
    dk = keys[dom]
    achieved = cases[dk]["flops"] / (mean[dom] * 1e-6) / 1e12
    traffic = None
    tf = ROOT / "profiles" / "traffic.json"
    if tf.exists():
        traffic = json.loads(tf.read_text()).get(f"r{dk[0]}_t{dk[1]}")
    value = statistics.mean(mean)
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "us/call", "n_gpus": world,
        "steps": steps, "warmup": warmup, "ms_per_step": round(sum(mean) / 1e3, 5),
        "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic (seeded N(0,sigma^2) cores, N(0,1) x)",
        "config": {"workload": WORKLOAD,
                   "l2": "flushed (256 MiB write) before every timed call",
                   "parallelism": f"replica x{world}" if world > 1 else "single GPU",
                   "cases": per_case},
        "e2e": {"value": round(statistics.mean(e2e), 3), "unit": "us/call",
                "h2d_bytes_per_step": sum(cases[k]["h2d"] for k in keys),
                "d2h_bytes_per_step": sum(cases[k]["d2h"] for k in keys)},
        "gpu_launches": launches,
        "launch_floor_us": {"cold": round(launch_cold, 3), "warm_stream": round(launch_warm, 3),
                            "kernel": "trr empty kernel (tr_empty_launch)"},
        "roofline": {"bound": "tensor",
                     "kernel": f"{KERNEL_NAMES.get(cases[dk]['tiling']['kernel'], '?')} "
                               f"r{dk[0]} t{dk[1]}",
                     "achieved": round(achieved, 2), "peak": tc_peak, "unit": "TFLOP/s",
                     "frac": round(achieved / tc_peak, 4), "traffic": traffic,
                     "peak_kind": f"{peak_kind} bf16 dense (burst)"},
        "clocks": clk,
    }
    if c3 is not None:
        line["config3"] = c3
    if prefill is not None:
        line["sharded_prefill"] = prefill
    if chain is not None:
        line["decode_chain"] = chain
    if c1_chain is not None:
        line["c1_chain"] = c1_chain
    if premerge is not None:
        line["premerge"] = premerge
    if ref_gpu is not None:
        line["reference_gpu"] = {m: {k: v for k, v in r.items() if k != "cases"}
                                 for m, r in ref_gpu.items() if isinstance(r, dict)}
    if world == 1:
        line["cpu_baseline"] = cpu_baseline_object()
    print(json.dumps(line), flush=True)


def profile_case(args):
    """One seeded operator, `--calls` calls, then synchronise: under
    `ncu -k regex:ring -s <calls-1> -c 1` it captures the last call's kernel."""
    from kernel_task_b200 import prepare_optimized
    from kernel_task_b200.spec import TRSpec, baseline_cores, baseline_x

    spec = TRSpec(tuple(int(v) for v in args.input_modes.split(",")),
                  tuple(int(v) for v in args.output_modes.split(",")), args.rank)
    dtype = getattr(torch, args.dtype)
    dev = torch.device("cuda")
    fn = prepare_optimized(baseline_cores(spec, dtype=dtype, device=dev), spec)
    x = baseline_x(spec, args.tokens, dtype=dtype, device=dev)
    forced = tuple(int(v) for v in args.tiling.split(",")) if args.tiling else None
    for _ in range(args.calls):
        y = fn.call_tiled(x, *forced) if forced else fn(x)
    torch.cuda.synchronize()
    print(f"ok {tuple(y.shape)} tiling={fn.tiling(args.tokens)} {fn.describe()}")


def main():
    args = parse()
    if args.ref_child:
        ref_child(args)
        return
    if args.profile_case:
        profile_case(args)
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if world > 1:
        import datetime

        torch.cuda.set_device(local_rank)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local_rank))
    try:
        run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
