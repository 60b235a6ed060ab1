"""Token-sharded data parallelism on two GPUs over NCCL.

Two ranks (one process per GPU) each run FFNSpRelu2 forward and backward on
half of the tokens with GradAllReduce attached, so the weight-gradient
all-reduces overlap the rest of the backward.  The summed dW1, dW2 and db1
must equal the gradients of the whole batch on one GPU, and each rank's
output rows must equal the matching rows of the whole batch's output, within
the bf16 bar (2e-2, elementwise, absolute floor scaled to the largest
magnitude; the all-reduce adds in bf16).  NVLS is off (NCCL_NVLS_ENABLE=0)
and the process group has a short timeout.  Skipped with fewer than two GPUs."""
import os
import socket
import sys

import pytest
import torch

from conftest import ROOT

pytestmark = pytest.mark.gpu
T, D, F = 2048, 1024, 4096


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    g = torch.Generator().manual_seed(0)
    x = torch.randn(T, D, generator=g).to(torch.bfloat16)
    W1 = (torch.randn(F, D, generator=g) / D ** 0.5).to(torch.bfloat16)
    W2 = (torch.randn(D, F, generator=g) / F ** 0.5).to(torch.bfloat16)
    b1 = torch.full((F,), -1.0).to(torch.bfloat16)
    dout = torch.randn(T, D, generator=g).to(torch.bfloat16)
    return x, W1, W2, b1, dout


def _run(sf, x, W1, W2, b1, dout, comm=None):
    ps = [t.clone().requires_grad_() for t in (W1, W2, b1)]
    out = sf.FFNSpRelu2.apply(x, ps[0], ps[1], None, ps[2])
    if comm is None:
        out.backward(dout)
    else:
        with comm.attached():
            out.backward(dout)
        comm.wait()
    torch.cuda.synchronize()
    return out.detach(), [p.grad for p in ps]


def _worker(rank, world, port, q):
    import datetime
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        import autoresearch2_b200 as sf
        x, W1, W2, b1, dout = (t.to(dev) for t in _inputs())
        rows = slice(rank * T // world, (rank + 1) * T // world)
        comm = sf.parallel.GradAllReduce(dist.group.WORLD)
        out, grads = _run(sf, x[rows].contiguous(), W1, W2, b1, dout[rows].contiguous(), comm)
        sf.check_status(dev)
        res = {}
        if rank == 0:
            full_out, full_grads = _run(sf, x, W1, W2, b1, dout)
            res["out"] = _err(out, full_out[rows])
            for name, g, w in zip(("dW1", "dW2", "db1"), grads, full_grads):
                res[name] = _err(g, w)
        dist.barrier()
        q.put((rank, res))
    finally:
        dist.destroy_process_group()


def _err(got, want):
    """Largest elementwise excess over the bf16 bar (<= 0 passes)."""
    got, want = got.double(), want.double()
    bar = 2e-2 * want.abs() + 2e-2 * want.abs().max()
    return float(((got - want).abs() - bar).max())


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_token_sharded_gradients_equal_the_full_batch():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        results = dict(q.get(timeout=300) for _ in procs)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    for name, excess in results[0].items():
        assert excess <= 0.0, (name, excess)
