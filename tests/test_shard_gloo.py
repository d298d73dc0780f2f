"""Token sharding over two CPU ranks (gloo), with the numpy oracle standing in for the per-rank
CUDA operator: row partition, the optional gather, uneven and tiny token counts, and a rank that
dies before the gather (the survivor's collective ends with an error after a short
process-group timeout instead of waiting forever).  The GPU path runs the same ShardedRing with
prepare_optimized (bench.py's sharded prefill leg)."""
from __future__ import annotations

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from kernel_task_b200.shard import ShardedRing, shard_bounds
from kernel_task_b200.spec import TRSpec, make_cores


def test_shard_bounds_partition():
    for T in (0, 1, 2, 3, 7, 8, 65536, 65537):
        for G in (1, 2, 3, 4, 8):
            spans = [shard_bounds(T, G, g) for g in range(G)]
            assert spans[0][0] == 0 and spans[-1][1] == T
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1 and sizes == sorted(sizes, reverse=True)
    assert shard_bounds(65536, 8, 3) == (3 * 8192, 4 * 8192)
    with pytest.raises(ValueError):
        shard_bounds(4, 2, 2)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


SPEC = TRSpec((2, 3, 4), (3, 2, 5), 3)


def _oracle_op(cores, spec):
    ref = [c.double().numpy() for c in cores]
    return lambda x: torch.from_numpy(oracle.tr_forward_reference(x.double().numpy(), ref))


def _worker(rank, world, port, mode, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    timeout = datetime.timedelta(seconds=5 if mode == "rank_dies" else 60)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timeout)
    try:
        cores = make_cores(SPEC, seed=3)
        op = ShardedRing(cores, SPEC, op_factory=_oracle_op)
        if mode == "rank_dies":
            if rank == 1:
                os._exit(0)  # leaves between steps, before the collective
            x = torch.randn(6, SPEC.in_features, generator=torch.Generator().manual_seed(1))
            try:
                op(x, gather=True)
                out[rank] = "no error"
            except Exception as e:  # the gather must fail, not hang
                out[rank] = "error: " + type(e).__name__
            return
        results = {}
        for T in (0, 1, 5, 8):
            x = torch.randn(T, SPEC.in_features, generator=torch.Generator().manual_seed(T),
                            dtype=torch.float64)
            a, b = op.bounds(T)
            rows = op(x)
            full = op(x, gather=True)
            results[T] = (a, b, rows.numpy(), full.numpy())
        out[rank] = results
    finally:
        if mode != "rank_dies" or rank == 0:
            dist.destroy_process_group()


def _run(mode, world=2):
    port = _free_port()
    with mp.Manager() as m:
        out = m.dict()
        ctx = mp.get_context("spawn")
        procs = [ctx.Process(target=_worker, args=(r, world, port, mode, out))
                 for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
        for p in procs:
            if p.is_alive():
                p.kill()
                pytest.fail("a rank did not finish")
        return dict(out)


def test_two_ranks_partition_and_gather():
    out = _run("normal")
    cores = [c.double().numpy() for c in make_cores(SPEC, seed=3)]
    for T in (0, 1, 5, 8):
        x = torch.randn(T, SPEC.in_features, generator=torch.Generator().manual_seed(T),
                        dtype=torch.float64).numpy()
        y = oracle.tr_forward_reference(x, cores)
        for rank in (0, 1):
            a, b, rows, full = out[rank][T]
            assert (a, b) == shard_bounds(T, 2, rank)
            # the stand-in's BLAS blocking depends on the batch size: equal to fp32 rounding
            np.testing.assert_allclose(rows, y[a:b], rtol=1e-6, atol=1e-6)
            np.testing.assert_allclose(full, y, rtol=1e-6, atol=1e-6)
            assert rows.shape == (b - a, SPEC.out_features) and full.shape == y.shape


def test_rank_leaving_before_gather_ends_with_error():
    out = _run("rank_dies")
    assert out[0].startswith("error")
