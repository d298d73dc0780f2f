"""GPU: tr_forward_noalloc, the entry point for callers that cannot allocate device memory (a
plugin or foreign-language host without a CUDA allocator, or a serving loop that must not call
cudaMalloc once running).  It runs the same slot-reducing kernel as tr_forward, but its scratch
is a fixed array inside libtrring.so instead of a caller workspace.

Called through the C ABI (ctypes) and checked against tr_forward's output, twice in a row (the
array keeps the previous call's contents).  This file is collected last on purpose.
"""
from __future__ import annotations

import pytest
import torch

from helpers import check_close
from kernel_task_b200 import abi
from kernel_task_b200 import spec as kspec

pytestmark = pytest.mark.gpu


def _setup(spec, dtype, code, device):
    cores = kspec.baseline_cores(spec, seed=0, dtype=dtype, device=device)
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
        for _ in range(2):
            y = torch.full((T, spec.out_features), float("nan"), dtype=dtype, device=device)
            abi.check(plan.forward_noalloc(packed.data_ptr(), x.data_ptr(), T, y.data_ptr(),
                                           stream), "tr_forward_noalloc")
            torch.cuda.synchronize()
            check_close(y, y_ref.double().cpu().numpy(), dtype)
