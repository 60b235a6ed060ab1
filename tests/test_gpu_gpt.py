"""GPU checks of the GPT harness with the sparse ReLU^2 MLPs: the sparse
model against the same model with dense torch MLPs (loss and every
gradient within the bf16 tolerance 2e-2, elementwise, absolute floor scaled
to the tensor's largest magnitude), and training steps through the fused
AdamW that lower the loss on a fixed batch with the shared arena intact."""
import math

import pytest
import torch

import autoresearch2_b200 as sf
from autoresearch2_b200 import gpt

pytestmark = pytest.mark.gpu
DEV = "cuda"
CFG = gpt.GPTConfig(n_layer=3, n_head=4, n_embd=256, ffn_hidden=1024, vocab=1024, seq_len=128)


def loss_and_grads(sparse, idx, tgt):
    m = gpt.GPT(CFG, sparse=sparse, device=DEV, fill=1.0)
    loss = m(idx, tgt)
    loss.backward()
    return loss.detach(), {n: p.grad for n, p in m.named_parameters()}


def test_sparse_mlps_match_dense():
    idx, tgt = gpt.synthetic_batch(CFG, 4, DEV)
    ls, gs = loss_and_grads(True, idx, tgt)
    ld, gd = loss_and_grads(False, idx, tgt)
    sf.check_status()
    assert abs(float(ls) - float(ld)) <= 2e-2 * abs(float(ld))
    for name, g in gs.items():
        w = gd[name]
        err = (g.float() - w.float()).abs().max().item()
        assert err <= 2e-2 * w.float().abs().max().item(), (name, err)


def test_training_steps_lower_the_loss():
    idx, tgt = gpt.synthetic_batch(CFG, 8, DEV, seed=1)
    m = gpt.GPT(CFG, sparse=True, device=DEV)
    step = gpt.TrainStep(m, idx, tgt, lr=3e-3)
    losses = [float(step()) for _ in range(12)]
    sf.check_status()
    assert all(math.isfinite(v) for v in losses) and losses[-1] < losses[0] - 0.1, losses
    used, cap = m.arena.used(), m.arena.n
    assert 0 < used <= cap


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_data_parallel_ranks_stay_identical():
    """Two ranks (torchrun, NCCL, DistributedDataParallel), different batches:
    after the steps every parameter is bit-identical across the ranks."""
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29531", "-m",
           "autoresearch2_b200.train_gpt", "--check", "--layers=2", "--width=256", "--heads=4", "--hidden=1024",
           "--vocab=1024", "--seq=128", "--batch=4", "--steps=3", "--warmup=1"]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=root)
    r = subprocess.run(cmd, cwd=root, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert '"params_identical": true' in r.stdout, r.stdout
