"""GPU: the device status word of the tcgen05 kernel's bounded waits.

Every wait of the tcgen05 kernel gives up after a bounded number of polls; the CTA then skips
its remaining work, waits for its own copies and tensor-core operations in flight, releases its
TMEM and records TR_ERR_TIMEOUT in the first workspace word, which tr_workspace_status reads.
These tests make the waits run out on a healthy GPU by shortening the poll limit to one poll
(tr_plan_set_wait_limit), check that the timeout is reported, that the word can be cleared, and
that the next call with the normal limit is correct: the context stays usable.  No fault, trap
or endless loop is involved.
"""
from __future__ import annotations

import pytest
import torch

import oracle
from helpers import check_close
from kernel_task_b200 import abi, prepare_optimized
from kernel_task_b200 import spec as kspec

pytestmark = pytest.mark.gpu


def _ref(x, cores):
    return oracle.tr_forward_reference(x.float().cpu().numpy(),
                                       [c.float().cpu().numpy() for c in cores])


@pytest.mark.parametrize("T", [8, 32])
def test_timeout_is_reported_through_the_c_abi(T):
    spec = kspec.SPEC_C1
    dev = torch.device("cuda", torch.cuda.current_device())
    cores = kspec.baseline_cores(spec, seed=3, dtype=torch.float16, device=dev)
    plan = abi.Plan(spec.input_modes, spec.output_modes, spec.rank, abi.TR_F16, dev.index)
    packed = torch.empty(plan.packed_bytes(), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream().cuda_stream
    plan.pack([c.data_ptr() for c in cores], packed.data_ptr(), stream)
    tc = abi.TrTiling(kernel=abi.KERNEL_TC05)
    ws_bytes = plan.workspace_bytes(T, tc)
    assert ws_bytes >= 256
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=dev)
    x = kspec.baseline_x(spec, T, seed=4, dtype=torch.float16, device=dev)
    y = torch.empty(T, spec.out_features, dtype=torch.float16, device=dev)
    ref = _ref(x, cores)

    plan.set_wait_limit(1)  # every wait that is not already complete gives up at once
    abi.check(plan.forward(packed.data_ptr(), x.data_ptr(), T, y.data_ptr(), ws.data_ptr(),
                           ws_bytes, stream, tc), "tr_forward")
    assert abi.workspace_status(ws.data_ptr(), ws_bytes, reset=False, stream=stream) == \
        abi.TR_ERR_TIMEOUT
    assert abi.workspace_status(ws.data_ptr(), ws_bytes, reset=True, stream=stream) == \
        abi.TR_ERR_TIMEOUT
    assert abi.workspace_status(ws.data_ptr(), ws_bytes, stream=stream) == abi.TR_OK

    plan.set_wait_limit(0)  # the built-in limit: the same workspace serves a correct call
    for _ in range(2):
        y.fill_(float("nan"))
        abi.check(plan.forward(packed.data_ptr(), x.data_ptr(), T, y.data_ptr(), ws.data_ptr(),
                               ws_bytes, stream, tc), "tr_forward")
        assert abi.workspace_status(ws.data_ptr(), ws_bytes, stream=stream) == abi.TR_OK
        check_close(y, ref, torch.float16)


def test_timeout_through_the_torch_binding(monkeypatch):
    """RingOp.workspace_status reads the word; with TRR_CHECK_STATUS=1 every call checks it
    and raises on a timeout (the output is not valid), and the next call is correct."""
    monkeypatch.setenv("TRR_CHECK_STATUS", "1")
    spec = kspec.SPEC_C2
    dev = torch.device("cuda", torch.cuda.current_device())
    cores = kspec.baseline_cores(spec, seed=5, dtype=torch.float16, device=dev)
    op = prepare_optimized(cores, spec)
    T = 32
    x = kspec.baseline_x(spec, T, seed=6, dtype=torch.float16, device=dev)
    assert op.tiling(T)["kernel"] == abi.KERNEL_TC05
    op.set_wait_limit(1)
    with pytest.raises(RuntimeError, match="timed out"):
        op(x)
    assert op.workspace_status() == abi.TR_OK  # the checking call cleared it
    op.set_wait_limit(0)
    check_close(op(x), _ref(x, cores), torch.float16)
    assert op.workspace_status() == abi.TR_OK
