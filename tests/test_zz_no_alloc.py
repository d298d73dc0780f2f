"""GPU: tr_forward_noalloc, the entry point for callers that cannot allocate device memory (a
plugin or foreign-language host without a CUDA allocator, or a serving loop that must not call
cudaMalloc once running).  It runs the same slot-reducing kernel as tr_forward, but its scratch
is a fixed array inside libtrring.so instead of a caller workspace.

Called through the C ABI (ctypes) and checked against the CPU oracle and against tr_forward's
output, twice in a row (the array keeps the previous call's contents); a token count whose
scratch exceeds the array is refused with TR_ERR_WORKSPACE.  This file is collected last on
purpose.
"""
from __future__ import annotations

import pytest
import torch

import oracle
from helpers import check_close
from kernel_task_b200 import abi
from kernel_task_b200 import spec as kspec

pytestmark = pytest.mark.gpu


def _cores(spec, dtype, device):
    return kspec.baseline_cores(spec, seed=0, dtype=dtype, device=device)


def _setup(spec, dtype, code, device):
    cores = _cores(spec, dtype, device)
    plan = abi.Plan(spec.input_modes, spec.output_modes, spec.rank, code, device.index)
    packed = torch.empty(plan.packed_bytes(), dtype=torch.uint8, device=device)
    plan.pack([c.data_ptr() for c in cores], packed.data_ptr(),
              torch.cuda.current_stream().cuda_stream)
    return plan, packed


@pytest.mark.parametrize("spec,dtype,code", [(kspec.SPEC_C1, torch.float16, abi.TR_F16),
                                             (kspec.SPEC_C2, torch.float16, abi.TR_F16),
                                             (kspec.SPEC_C4["q"], torch.bfloat16, abi.TR_BF16)])
def test_noalloc_matches_tr_forward(spec, dtype, code):
    device = torch.device("cuda", torch.cuda.current_device())
    plan, packed = _setup(spec, dtype, code, device)
    stream = torch.cuda.current_stream().cuda_stream
    for T in (1, 8, 3):
        x = kspec.baseline_x(spec, T, seed=1, dtype=dtype, device=device)
        mma = abi.TrTiling(kernel=abi.KERNEL_MMA)
        assert plan.workspace_bytes(T, mma) > 0, "the case must exercise the scratch reduction"
        ws_bytes = plan.workspace_bytes(T)
        ws = torch.zeros(max(ws_bytes, 16), dtype=torch.uint8, device=device)
        y_ref = torch.empty(T, spec.out_features, dtype=dtype, device=device)
        abi.check(plan.forward(packed.data_ptr(), x.data_ptr(), T, y_ref.data_ptr(),
                               ws.data_ptr(), ws_bytes, stream), "tr_forward")
        ref = oracle.tr_forward_reference(x.float().cpu().numpy(),
                                          [c.float().cpu().numpy() for c in _cores(spec, dtype,
                                                                                   device)])
        for _ in range(2):
            y = torch.full((T, spec.out_features), float("nan"), dtype=dtype, device=device)
            abi.check(plan.forward_noalloc(packed.data_ptr(), x.data_ptr(), T, y.data_ptr(),
                                           stream), "tr_forward_noalloc")
            torch.cuda.synchronize()
            check_close(y, ref, dtype)
            check_close(y, y_ref.double().cpu().numpy(), dtype)


def test_noalloc_refuses_token_counts_beyond_its_scratch():
    """A call whose mma-kernel scratch exceeds TR_NOALLOC_SCRATCH_BYTES returns
    TR_ERR_WORKSPACE without launching; the next call within the limit is correct."""
    spec = kspec.SPEC_C2
    device = torch.device("cuda", torch.cuda.current_device())
    plan, packed = _setup(spec, torch.float16, abi.TR_F16, device)
    stream = torch.cuda.current_stream().cuda_stream
    mma = abi.TrTiling(kernel=abi.KERNEL_MMA)
    big = next(T for T in range(1, 1024) if plan.workspace_bytes(T, mma) > (8 << 20))
    x = kspec.baseline_x(spec, big, seed=2, dtype=torch.float16, device=device)
    y = torch.zeros(big, spec.out_features, dtype=torch.float16, device=device)
    assert plan.forward_noalloc(packed.data_ptr(), x.data_ptr(), big, y.data_ptr(),
                                stream) == abi.TR_ERR_WORKSPACE
    assert b"scratch" in abi.lib().tr_last_error()
    torch.cuda.synchronize()
    assert torch.count_nonzero(y) == 0  # nothing was launched
    T = 8
    xs = x[:T].contiguous()
    ys = torch.empty(T, spec.out_features, dtype=torch.float16, device=device)
    abi.check(plan.forward_noalloc(packed.data_ptr(), xs.data_ptr(), T, ys.data_ptr(), stream),
              "tr_forward_noalloc")
    torch.cuda.synchronize()
    ref = oracle.tr_forward_reference(xs.float().cpu().numpy(),
                                      [c.float().cpu().numpy()
                                       for c in _cores(spec, torch.float16, device)])
    check_close(ys, ref, torch.float16)
