"""Multi-process host logic on CPU with gloo ranks (world size 2): row
sharding, the gradient all-reduce of data-parallel layer training (checked
against the single-process gradient, with the oracle standing in for the
kernels), max-over-ranks timing, and failure detection -- a rank that dies
before the collective makes the survivor's collective fail within the
process-group timeout instead of hanging."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from cliffordcuda_b200 import distributed as D


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, ws, port, timeout_s=60):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=ws,
                            timeout=datetime.timedelta(seconds=timeout_s))


def test_shard_rows_partition():
    for batch in (0, 1, 7, 1000, 524288):
        for ws in (1, 2, 3, 8):
            ranges = [D.shard_rows(batch, ws, r) for r in range(ws)]
            assert ranges[0][0] == 0 and ranges[-1][1] == batch
            for (a, b), (c, d) in zip(ranges, ranges[1:]):
                assert b == c
            sizes = [b - a for a, b in ranges]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        D.shard_rows(10, 2, 2)


def _dp_worker(rank, ws, port, q):
    try:
        _init(rank, ws, port)
        from oracle import ga_oracle as O
        n, metric = 6, (1, 1, 1, 1, 1, -1)
        rng = np.random.default_rng(0)
        B = 37
        x = rng.standard_normal((B, 64))
        g = rng.standard_normal((B, 64))
        w = rng.standard_normal(64)
        s, e = D.shard_rows(B, ws, rank)
        # the layer weight gradient of this rank's rows (oracle as the kernel)
        dw_local = O.product("gp", "grad_b", n, metric, x[s:e], g[s:e]).sum(axis=0)
        layer = torch.nn.Linear(1, 64, bias=False)
        layer.weight.grad = torch.tensor(dw_local, dtype=torch.float32).view(64, 1)
        D.allreduce_grads(layer)
        t = D.max_over_ranks(float(rank + 1))
        q.put((rank, layer.weight.grad.view(-1).numpy().copy(), t))
        dist.destroy_process_group()
    except Exception as exc:  # reported to the parent
        q.put((rank, repr(exc), None))


def test_dp_gradient_allreduce_matches_single_process():
    from oracle import ga_oracle as O
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_dp_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = [q.get(timeout=120) for _ in ps]
    for p in ps:
        p.join(timeout=60)
    rng = np.random.default_rng(0)
    x = rng.standard_normal((37, 64))
    g = rng.standard_normal((37, 64))
    full = O.product("gp", "grad_b", 6, (1, 1, 1, 1, 1, -1), x, g).sum(axis=0)
    for rank, grad, t in res:
        assert not isinstance(grad, str), grad
        np.testing.assert_allclose(grad, full, rtol=1e-5, atol=1e-4)
        assert t == 2.0


def _dying_worker(rank, ws, port, q):
    _init(rank, ws, port, timeout_s=3)
    if rank == 1:
        os._exit(0)  # leaves between steps, before the collective
    t = torch.ones(4)
    try:
        dist.all_reduce(t)
        q.put((rank, "completed"))
    except Exception as exc:
        q.put((rank, "error: " + type(exc).__name__))


def test_dead_rank_is_detected_by_timeout():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_dying_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    rank, status = q.get(timeout=120)
    for p in ps:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert rank == 0 and status.startswith("error"), status
