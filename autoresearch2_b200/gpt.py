"""A GPT-style decoder whose MLPs are the sparse ReLU^2 FFN: the end-to-end
consumer of the hot path.  The reference has no GPT model; its nearest
harness is DeepFFN (old/lib_sparse/prepare.py:50-78).

    GPTConfig(n_layer=12, n_head=12, n_embd=768, ffn_hidden=3072, vocab=50304, seq_len=1024)
    GPT(cfg, sparse=True, device="cuda", dtype=torch.bfloat16)
    TrainStep(model, idx, targets, lr=3e-4)  one AdamW step per call, returns the loss tensor
    synthetic_batch(cfg, batch, device)      seeded uniform token ids and next-token targets

Blocks: x += attn(rms_norm(x)); x += mlp(rms_norm(x)); causal attention by
torch's scaled_dot_product_attention; learned positions; the token embedding
is tied to the output projection; weights ~ N(0, 0.02).  With sparse=True
every MLP runs FFNSpRelu2 over one vals arena shared by all layers and
rewound at each step (an arena of `fill` x the dense activation size of all
layers; 0.6 by default, for the ~50% zeros of ReLU at initialisation), so
the stack keeps only the compacted ReLU outputs between forward and
backward; sparse=False runs the same MLP as dense torch matmuls.  An arena
too small for a step's activations sets the library's status word (values
past the end are dropped): check_status() after a step reports it.
"""
from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import bitsparse as bs
from .ffn import FFNSpRelu2

__all__ = ["GPTConfig", "GPT", "TrainStep", "flops_per_token", "synthetic_batch", "mfu"]


@dataclass
class GPTConfig:
    n_layer: int = 12
    n_head: int = 12
    n_embd: int = 768
    ffn_hidden: int = 3072
    vocab: int = 50304
    seq_len: int = 1024


def flops_per_token(cfg: GPTConfig) -> float:
    """Training FLOPs per token: 6 x the matmul parameters (embedding tied to
    the output projection counted once, positions excluded) plus the
    attention scores and values, 12 x layers x width x sequence length."""
    d, L = cfg.n_embd, cfg.n_layer
    per_layer = 4 * d * d + 2 * d * cfg.ffn_hidden
    return 6 * (L * per_layer + d * cfg.vocab) + 12 * L * d * cfg.seq_len


class Block(nn.Module):
    def __init__(self, cfg, sparse, device, dtype):
        super().__init__()
        d, h = cfg.n_embd, cfg.ffn_hidden
        self.n_head = cfg.n_head
        self.qkv = nn.Parameter(torch.empty(3 * d, d, device=device, dtype=dtype))
        self.proj = nn.Parameter(torch.empty(d, d, device=device, dtype=dtype))
        self.W1 = nn.Parameter(torch.empty(h, d, device=device, dtype=dtype))
        self.W2 = nn.Parameter(torch.empty(d, h, device=device, dtype=dtype))
        self.sparse = sparse

    def forward(self, x, arena):
        B, T, d = x.shape
        q, k, v = (F.rms_norm(x, (d,)) @ self.qkv.T).split(d, dim=-1)
        q, k, v = (t.view(B, T, self.n_head, d // self.n_head).transpose(1, 2) for t in (q, k, v))
        y = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        x = x + y.transpose(1, 2).reshape(B, T, d) @ self.proj.T
        h = F.rms_norm(x, (d,)).view(B * T, d)
        if self.sparse:
            m = FFNSpRelu2.apply(h, self.W1, self.W2, arena)
        else:
            m = torch.relu(h @ self.W1.T).square() @ self.W2.T
        return x + m.view(B, T, d)


class GPT(nn.Module):
    def __init__(self, cfg: GPTConfig, sparse=True, device="cuda", dtype=torch.bfloat16, fill=0.6, seed=0):
        super().__init__()
        self.cfg, self.sparse, self.fill = cfg, sparse, fill
        self.wte = nn.Parameter(torch.empty(cfg.vocab, cfg.n_embd, device=device, dtype=dtype))
        self.wpe = nn.Parameter(torch.empty(cfg.seq_len, cfg.n_embd, device=device, dtype=dtype))
        self.blocks = nn.ModuleList(Block(cfg, sparse, device, dtype) for _ in range(cfg.n_layer))
        g = torch.Generator(device=device).manual_seed(seed)
        with torch.no_grad():
            for p in self.parameters():
                p.normal_(0.0, 0.02, generator=g)
        self.arena = None

    def arena_for(self, tokens):
        """The shared vals arena, (re)allocated for `tokens` and rewound."""
        cap = int(tokens * self.cfg.ffn_hidden * self.cfg.n_layer * self.fill)
        if self.arena is None or self.arena.n != cap:
            self.arena = bs.TensorBuffer(cap, self.wte.device, self.wte.dtype).init_buffer()
        return self.arena.reset_buffer()

    def forward(self, idx, targets=None):
        B, T = idx.shape
        x = self.wte[idx] + self.wpe[:T]
        arena = self.arena_for(B * T).as_sparse_data() if self.sparse else None
        for blk in self.blocks:
            x = blk(x, arena)
        logits = F.rms_norm(x, (x.shape[-1],)) @ self.wte.T
        if targets is None:
            return logits
        return F.cross_entropy(logits.float().view(B * T, -1), targets.view(-1))


class TrainStep:
    """forward, backward and one fused AdamW step on a fixed (inputs, targets) batch."""

    def __init__(self, model, idx, targets, lr=3e-4):
        self.model, self.idx, self.targets = model, idx, targets
        self.opt = torch.optim.AdamW(model.parameters(), lr=lr, betas=(0.9, 0.95), weight_decay=0.0,
                                     fused=True)

    def __call__(self):
        loss = self.model(self.idx, self.targets)
        loss.backward()
        self.opt.step()
        self.opt.zero_grad(set_to_none=True)
        return loss.detach()


def synthetic_batch(cfg: GPTConfig, batch, device, seed=0):
    """Uniform random token ids (seeded), inputs and next-token targets."""
    g = torch.Generator(device=device).manual_seed(seed)
    toks = torch.randint(0, cfg.vocab, (batch, cfg.seq_len + 1), generator=g, device=device)
    return toks[:, :-1].contiguous(), toks[:, 1:].contiguous()


def mfu(tokens_per_s, cfg, peak_tflops):
    """Model FLOPs utilisation against a peak in TFLOP/s."""
    return tokens_per_s * flops_per_token(cfg) / (peak_tflops * 1e12)
