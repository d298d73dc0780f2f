"""TEST INFRASTRUCTURE ONLY -- the CPU oracle of the tensor-ring operator.

A numpy restatement of the reference's factorized contraction
(factorized_inference/reference.py:99-149).  Only tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline / reference legs may import it, and only as the checker or as the
timed CPU baseline; the product package (kernel_task_b200) never imports it.

Parity of this restatement is pinned against vectors produced by the reference itself
(tests/golden/make_golden.py imports factorized_inference and writes tests/golden/*.npz;
tests/test_oracle.py checks the restatement against them).
"""
from .ring_oracle import (dense_forward, materialize_dense_weight, order_forward, order_macs,
                          reference_macs, tr_forward_reference)

__all__ = ["tr_forward_reference", "materialize_dense_weight", "dense_forward", "order_forward",
           "order_macs", "reference_macs"]
