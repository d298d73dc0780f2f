"""B200-native (sm_100a) three-core tensor-ring linear operator.

Drop-in for the reference package factorized_inference's hot path:

    from kernel_task_b200 import TRSpec, make_cores, prepare_optimized
    fn = prepare_optimized(cores, spec)     # pack once
    y = fn(x)                               # one fused CUDA kernel per call

The operator is y[t,(p,q,r)] = sum x[t,(i,j,k)] A[a,p,i,b] B[b,q,j,c] C[c,r,k,a] with cores
stored [rank, output_mode, input_mode, rank] (factorized_inference/reference.py:99-125).
The kernels live in libtrring.so behind a C ABI (include/trring.h); _trring_torch.so is the
thin PyTorch binding used here.
"""
from .spec import (SPEC_C1, SPEC_C2, SPEC_C3, SPEC_C4, SPEC_C5, TRSpec, baseline_cores,
                   baseline_sigma, baseline_x, make_cores, validate, validate_cores)
from .ring import consume_add, consume_silu_mul, prepare_optimized, tr_forward_optimized

__all__ = [
    "TRSpec", "make_cores", "baseline_cores", "baseline_sigma", "baseline_x", "validate",
    "validate_cores", "prepare_optimized", "tr_forward_optimized", "consume_silu_mul", "consume_add",
    "SPEC_C1", "SPEC_C2", "SPEC_C3", "SPEC_C4", "SPEC_C5",
]
