"""CPU checks of the GPT harness's host side: its FLOP count, the dense
model's wiring (shapes, a loss that falls on a fixed batch), and that the
sparse model refuses CPU tensors (its MLPs run only on the CUDA library)."""
import pytest
import torch

from autoresearch2_b200 import gpt

SMALL = gpt.GPTConfig(n_layer=2, n_head=4, n_embd=64, ffn_hidden=256, vocab=128, seq_len=16)


def test_flops_per_token():
    c = gpt.GPTConfig()
    per_layer = 4 * 768 * 768 + 2 * 768 * 3072
    assert gpt.flops_per_token(c) == 6 * (12 * per_layer + 768 * 50304) + 12 * 12 * 768 * 1024


def test_dense_model_trains_on_cpu():
    torch.manual_seed(0)
    m = gpt.GPT(SMALL, sparse=False, device="cpu", dtype=torch.float32)
    idx, tgt = gpt.synthetic_batch(SMALL, 4, "cpu")
    assert m(idx).shape == (4, SMALL.seq_len, SMALL.vocab)
    step = gpt.TrainStep(m, idx, tgt, lr=1e-2)
    step.opt = torch.optim.AdamW(m.parameters(), lr=1e-2)  # the fused optimizer is CUDA-only
    losses = [float(step()) for _ in range(8)]
    assert losses[-1] < losses[0]


def test_sparse_model_needs_cuda():
    m = gpt.GPT(SMALL, sparse=True, device="cpu", dtype=torch.float32)
    idx, tgt = gpt.synthetic_batch(SMALL, 2, "cpu")
    with pytest.raises(ValueError, match="CUDA tensors only"):
        m(idx, tgt)
