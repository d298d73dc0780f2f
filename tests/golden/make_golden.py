"""Generate the golden vectors in tests/golden/ by running the REFERENCE implementation.

    python tests/golden/make_golden.py [--reference-src PATH]

PATH is the reference's src/ directory (package factorized_inference); without the flag the
script reads $REFERENCE_SRC.  Every expected output here comes from the reference's
own functions: make_cores (reference.py:53-77), tr_forward_reference (reference.py:99-125) and
the dense fp64 oracle of its tests (tests/test_correctness.py:12-14).  Inputs are drawn on the
CPU generator so any machine reproduces them.  The files are small and committed; this script
is the record of how they were made and is not run by the tests.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().cpu().numpy().tobytes()).hexdigest()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-src", default=os.environ.get("REFERENCE_SRC"))
    args = ap.parse_args()
    if not args.reference_src:
        ap.error("give --reference-src or set REFERENCE_SRC to the reference's src/ directory")
    sys.path.insert(0, args.reference_src)
    sys.path.insert(0, str(ROOT))
    import factorized_inference as ref  # the reference package
    from kernel_task_b200 import spec as kspec

    torch.set_num_threads(1)

    def oracle64(x, cores, spec):
        return ref.dense_forward(x.double(),
                                 ref.materialize_dense_weight(tuple(c.double() for c in cores),
                                                              spec))

    out: dict[str, np.ndarray] = {}
    meta: dict = {"generator": "tests/golden/make_golden.py", "torch": torch.__version__,
                  "cases": {}}

    # 1. the reference's CPU numerics cases (tests/test_correctness.py:26-46): three specs,
    #    seeds 0 and 19, token/scale sequence (1,1.0) (5,0.0) (3,0.1) (1,2.0); fp32
    specs = [((2, 3, 2), (2, 4, 3), 2), ((4, 4, 4), (4, 4, 4), 8), ((4, 4, 4), (4, 4, 4), 16)]
    for si, (im, om, R) in enumerate(specs):
        spec = ref.TRSpec(im, om, R)
        for seed in (0, 19):
            cores = ref.make_cores(spec, seed=seed)
            key = f"cpu{si}_s{seed}"
            mine = kspec.make_cores(kspec.TRSpec(im, om, R), seed=seed)
            assert all(torch.equal(a, b) for a, b in zip(cores, mine)), "make_cores mismatch"
            for k, c in enumerate(cores):
                out[f"{key}_core{k}"] = c.numpy()
            gen = torch.Generator().manual_seed(seed + 37)
            for n, (tokens, scale) in enumerate([(1, 1.0), (5, 0.0), (3, 0.1), (1, 2.0)]):
                x = torch.randn(tokens, spec.in_features, generator=gen) * scale
                out[f"{key}_x{n}"] = x.numpy()
                out[f"{key}_yref{n}"] = ref.tr_forward_reference(x, cores, spec).numpy()
                out[f"{key}_y64_{n}"] = oracle64(x, cores, spec).numpy()
            meta["cases"][key] = {"input_modes": im, "output_modes": om, "rank": R,
                                  "seed": seed, "dtype": "float32"}

    # 2. known-answer test of the index convention (tests/test_correctness.py:80-91)
    spec = ref.TRSpec((2, 2, 2), (2, 2, 2), 2)
    cores = ref.make_cores(spec, dtype=torch.float64, seed=11)
    for k, c in enumerate(cores):
        out[f"kat_core{k}"] = c.numpy()
    out["kat_W"] = ref.materialize_dense_weight(cores, spec).numpy()

    # 3. the five required GPU workloads (tests/test_correctness.py:68-77): R in {8,16},
    #    cores seed 23 and x seed 41+T.  The reference draws these on the CUDA generator; here
    #    they are drawn on the CPU generator and rounded to fp16, and y is the reference's
    #    contraction of the fp16 values in fp32 (its harness oracle precision).
    for R, toks in ((8, (1, 8, 32)), (16, (1, 32))):
        spec = ref.TRSpec(rank=R)
        cores16 = tuple(c.half() for c in ref.make_cores(spec, seed=23))
        key = f"req_r{R}"
        for k, c in enumerate(cores16):
            out[f"{key}_core{k}"] = c.numpy()
        for T in toks:
            gen = torch.Generator().manual_seed(41 + T)
            x16 = torch.randn(T, spec.in_features, generator=gen).half()
            out[f"{key}_x_t{T}"] = x16.numpy()
            out[f"{key}_yref_t{T}"] = ref.tr_forward_reference(
                x16.float(), tuple(c.float() for c in cores16), spec).numpy()
        meta["cases"][key] = {"rank": R, "tokens": toks, "core_seed": 23, "x_seed": "41+T",
                              "dtype": "float16 (CPU generator)"}

    # 4. odd shapes of the reference's GPU sweep (tools/check_kernel.py:63-84), fp16
    odd = [((2, 3, 4), (5, 6, 7), 3, (1, 5, 2)), ((2, 3, 2), (2, 4, 3), 3, (3, 1)),
           ((4, 4, 4), (4, 4, 4), 16, (1, 4, 9)), ((8, 6, 20), (12, 5, 24), 16, (1, 7))]
    for oi, (im, om, R, toks) in enumerate(odd):
        spec = ref.TRSpec(im, om, R)
        cores16 = tuple(c.half() for c in ref.make_cores(spec, seed=oi))
        key = f"odd{oi}"
        for k, c in enumerate(cores16):
            out[f"{key}_core{k}"] = c.numpy()
        gen = torch.Generator().manual_seed(oi + 5)
        for n, T in enumerate(toks):
            x16 = torch.randn(T, spec.in_features, generator=gen).half()
            out[f"{key}_x{n}"] = x16.numpy()
            out[f"{key}_yref{n}"] = ref.tr_forward_reference(
                x16.float(), tuple(c.float() for c in cores16), spec).numpy()
        meta["cases"][key] = {"input_modes": im, "output_modes": om, "rank": R, "tokens": toks,
                              "seed": oi}

    np.savez_compressed(HERE / "reference_vectors.npz", **out)

    # 5. The benchmark configs 3-5 (bf16): cores from kernel_task_b200.spec.baseline_cores (seeded,
    #    CPU generator), fingerprinted by sha256; y = the reference's contraction in fp32 of the
    #    bf16 values, for a few tokens.  Stored: hashes + x + y (cores are regenerated).
    big = {}
    cfgs = {"c3": (kspec.SPEC_C3, (1, 2, 8)), "c5": (kspec.SPEC_C5, (1, 2))}
    cfgs.update({f"c4_{n}": (s, (1,)) for n, s in kspec.SPEC_C4.items() if n in
                 ("q", "k", "gate", "down")})
    bmeta = {}
    for name, (s, toks) in cfgs.items():
        cores = kspec.baseline_cores(s, seed=3, dtype=torch.bfloat16)
        rspec = ref.TRSpec(s.input_modes, s.output_modes, s.rank)
        bmeta[name] = {"input_modes": s.input_modes, "output_modes": s.output_modes,
                       "rank": s.rank, "core_seed": 3, "dtype": "bfloat16",
                       "core_sha256": [sha(c.view(torch.int16)) for c in cores],
                       "tokens": toks}
        for T in toks:
            x = kspec.baseline_x(s, T, seed=3, dtype=torch.bfloat16)
            big[f"{name}_x_t{T}"] = x.view(torch.int16).numpy()
            big[f"{name}_yref_t{T}"] = ref.tr_forward_reference(
                x.float(), tuple(c.float() for c in cores), rspec).numpy()
    np.savez_compressed(HERE / "baseline_vectors.npz", **big)
    meta["baseline"] = bmeta
    (HERE / "golden_meta.json").write_text(json.dumps(meta, indent=1) + "\n")
    print("wrote", sorted(p.name for p in HERE.glob("*.npz")))


if __name__ == "__main__":
    main()
