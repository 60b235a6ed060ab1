"""Multi-process (gloo, CPU) tests of the data-parallel host logic.

Token-sharded DP must give the full-batch gradients: each rank computes the
oracle FFN backward on its token shard, GradAllReduce sums the weight
gradients, and the result equals the single-process gradient.  A rank that
fails before the collective makes its peer's collective end with an error
(short process-group timeout) instead of hanging."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import ROOT


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=60):
    import datetime
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _dp_worker(rank, world, port, q):
    import sys
    sys.path.insert(0, ROOT)
    import oracle
    from autoresearch2_b200.parallel import GradAllReduce
    _init(rank, world, port)
    rng = np.random.default_rng(0)
    T, D, F = 64, 16, 48
    x = rng.standard_normal((T, D)).astype(np.float32)
    W1 = (rng.standard_normal((F, D)) / 4).astype(np.float32)
    W2 = (rng.standard_normal((D, F)) / 7).astype(np.float32)
    dout = rng.standard_normal((T, D)).astype(np.float32)
    sl = slice(rank * T // world, (rank + 1) * T // world)
    r = oracle.ffn_fwd_bwd(x[sl], W1, W2, dout[sl], act="relu2")
    comm = GradAllReduce()
    g1 = torch.from_numpy(r["dW1"].copy())
    g2 = torch.from_numpy(r["dW2"].copy())
    with comm.attached():
        from autoresearch2_b200.parallel import submit_grad
        submit_grad(g2)
        submit_grad(g1)
    comm.wait()
    if rank == 0:
        full = oracle.ffn_fwd_bwd(x, W1, W2, dout, act="relu2")
        q.put((np.abs(g1.numpy() - full["dW1"]).max(), np.abs(g2.numpy() - full["dW2"]).max()))
    dist.destroy_process_group()


def test_token_sharded_grads_equal_full_batch():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dp_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs)
    e1, e2 = q.get(timeout=5)
    assert e1 < 1e-9 and e2 < 1e-9


def _fail_worker(rank, world, port, q):
    _init(rank, world, port, timeout_s=5)
    if rank == 1:
        os._exit(3)  # dies before its collective
    t = torch.ones(4)
    try:
        dist.all_reduce(t)
        q.put("no error")
    except Exception as e:  # noqa: BLE001
        q.put(type(e).__name__)


def test_dead_rank_surfaces_as_error_not_hang():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_fail_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(90)
    assert procs[1].exitcode == 3
    res = q.get(timeout=5)
    assert res != "no error"
