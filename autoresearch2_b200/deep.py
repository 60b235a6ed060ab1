"""A stack of sparse FFN layers over one shared vals arena, with the
reference's harness (old/lib_sparse/prepare.py:35-148).

    generate_parameters(dim, G, dtype, expansion=5.25, device="cuda") -> (W1, W2)
    DeepFFN(dtype, layers=12, hidm=4096)        .forward_base / .forward_sparse
    run_step(x, model, sparse, steps=1) -> (loss, grad_stds, peak_MB, ms_per_step)
    memory_report(x, model, fill=0.55, steps=2) -> dict

Each layer is x = x + FFN(rms_norm(x)).  forward_sparse runs FFNSparse (or
FFNSpRelu2) with the package's global arena: every layer appends its
compacted activation to the same vals buffer and advances the same int32
device cursor, which run_step rewinds before each step (prepare.py:84-91), so
the activation memory of the whole stack is one buffer of about fill x the
dense size.  forward_base is the dense baseline: FFNDense keeps the dense
ReLU output for backward, as the reference's FFNv3 does
(old/lib_sparse/prepare_layer.py:117-162).  Both forwards are plain Python
over torch.library ops and compile with torch.compile (compile=True wraps
them, as the reference's @torch.compile does, prepare.py:63,72).
"""
import gc
import math
import time

import torch
import torch.nn as nn
import torch.nn.functional as F
from torch.autograd import Function

from . import bitsparse as bs
from .ffn import FFNSparse, FFNSpRelu2

__all__ = ["generate_parameters", "FFNDense", "DeepFFN", "arena_elements", "run_step", "memory_report"]


def generate_parameters(dim, G, dtype, expansion=5.25, device="cuda"):
    """W1 [floor(dim * expansion), dim] and W2 [dim, floor(dim * expansion)]:
    Xavier-uniform, then shifted by 0.01 * s * std with one shared s ~ N(0, 1)
    (+ for W1, - for W2), as old/lib_sparse/prepare.py:35-47."""
    hdim = math.floor(dim * expansion)
    W1 = torch.empty(hdim, dim, device=device, dtype=dtype)
    nn.init.xavier_uniform_(W1, generator=G)
    W2 = torch.empty(dim, hdim, device=device, dtype=dtype)
    nn.init.xavier_uniform_(W2, generator=G)
    s = torch.randn(1, generator=G, device=device, dtype=dtype)
    return W1 + 0.01 * s * W1.std(), W2 - 0.01 * s * W2.std()


class FFNDense(Function):
    """Dense baseline: out = relu(x @ W1.T) @ W2.T, the dense z kept for
    backward (the memory profile of the reference's FFNv3)."""

    @staticmethod
    def forward(ctx, x, W1, W2, sparse_data=None):
        z = (x @ W1.T).relu_()
        ctx.save_for_backward(x, W1, W2, z)
        return z @ W2.T

    @staticmethod
    def backward(ctx, grad_output):
        x, W1, W2, z = ctx.saved_tensors
        grad_z = grad_output @ W2
        grad_W2 = grad_output.T @ z
        grad_pre = grad_z.masked_fill_(z <= 0, 0)
        del z
        return grad_pre @ W1, grad_pre.T @ x, grad_W2, None


class DeepFFN(nn.Module):
    """`layers` residual FFN blocks of width hidm and hidden floor(5.25 hidm),
    parameters from generate_parameters with one generator seeded 0
    (old/lib_sparse/prepare.py:50-78).  act: "relu" (FFNSparse, the
    reference's forward_sparse) or "relu2" (FFNSpRelu2)."""

    def __init__(self, dtype, layers=12, hidm=4096, act="relu", device="cuda", compile=False):
        super().__init__()
        if act not in ("relu", "relu2"):
            raise ValueError("act is 'relu' or 'relu2'")
        G = torch.Generator(device=device).manual_seed(0)
        self.W1s, self.W2s = nn.ParameterList(), nn.ParameterList()
        for _ in range(layers):
            W1, W2 = generate_parameters(hidm, G, dtype=dtype, device=device)
            self.W1s.append(nn.Parameter(W1))
            self.W2s.append(nn.Parameter(W2))
        self.sparse_fn = FFNSparse if act == "relu" else FFNSpRelu2
        if compile:
            self.forward_base = torch.compile(self.forward_base)
            self.forward_sparse = torch.compile(self.forward_sparse)

    def forward_base(self, x, sparse_data=None):
        for W1, W2 in zip(self.W1s, self.W2s):
            x = x + FFNDense.apply(F.rms_norm(x, x.shape[-1:]), W1, W2, sparse_data)
        return x

    def forward_sparse(self, x, sparse_data):
        for W1, W2 in zip(self.W1s, self.W2s):
            x = x + self.sparse_fn.apply(F.rms_norm(x, x.shape[-1:]), W1, W2, sparse_data)
        return x


def arena_elements(tokens, hidm, layers, fill=0.55, expansion=5.25):
    """Arena size of the reference's harness: tokens * hidden * layers * fill
    (old/lib_sparse/prepare.py:133-135)."""
    return int(tokens * math.floor(hidm * expansion) * layers * fill)


def run_step(x, model, sparse, steps=1, exact=False):
    """`steps` training steps (zero_grad, arena rewind, forward, loss =
    mean((y - x)^2), backward) after resetting the peak-memory counter;
    returns (loss, grad_stds * 1e3 with a leading 0, peak MB allocated,
    ms per step), as old/lib_sparse/prepare.py:80-112.  exact=True gives the
    sparse layers no arena: each keeps a values tensor of exactly its nnz,
    freed after its own backward."""
    dev = x.device
    gc.collect()
    torch.cuda.empty_cache()
    torch.cuda.reset_peak_memory_stats(dev)
    torch.cuda.synchronize(dev)
    sparse_data = None if exact else bs.get_globals()
    start = time.perf_counter()
    for _ in range(steps):
        model.zero_grad()
        bs.reset_sparse_globals()
        y = model.forward_sparse(x, sparse_data) if sparse else model.forward_base(x, sparse_data)
        loss = (y - x).pow(2).mean()
        loss.backward()
    peak = torch.cuda.max_memory_allocated(dev) / 1024 ** 2
    torch.cuda.synchronize(dev)
    ms = (time.perf_counter() - start) * 1000 / steps
    grad_stds = [torch.tensor(0.0)] + [p.grad.float().std().cpu() for p in model.parameters()]
    return loss.detach().cpu(), torch.stack(grad_stds) * 1e3, peak, ms


def steady_ms(x, model, sparse, exact=False, steps=4, warmup=2):
    """ms per training step as run_step takes it, but with the allocator's
    cache kept between steps (run_step empties it first, so its first step
    also pays for fresh device allocations): `warmup` untimed steps, then
    `steps` timed by host clock around synchronised steps."""
    dev = x.device
    sparse_data = None if exact else bs.get_globals()

    def step():
        model.zero_grad()
        bs.reset_sparse_globals()
        y = model.forward_sparse(x, sparse_data) if sparse else model.forward_base(x, sparse_data)
        (y - x).pow(2).mean().backward()

    for _ in range(warmup):
        step()
    torch.cuda.synchronize(dev)
    start = time.perf_counter()
    for _ in range(steps):
        step()
    torch.cuda.synchronize(dev)
    return (time.perf_counter() - start) * 1000 / steps


def memory_report(x, model, fill=0.55, steps=2):
    """Dense and sparse steps of the same model on the same input, each after
    one warm-up step (the reference's evaluate(), prepare.py:115-148, with its
    asserts restated as measurements): peak MB and ms per step of each, also
    as MB above what was resident before the steps (weights, input, other
    live tensors; the arena counts in the sparse step's), the arena's
    capacity and the fraction of it the last sparse step used, and the
    largest relative difference of loss and of gradient std between the two;
    then the sparse step again with no arena ("sparse_exact": each layer's
    values in a tensor of exactly its nnz, freed after its own backward).
    steady_ms_per_step: the same steps with the allocator's cache kept."""
    layers = len(model.W1s)
    hidm = x.shape[-1]
    bs.init_sparse_buffer(0, x.device, x.dtype)  # no arena while the dense step is measured
    model.zero_grad()
    gc.collect()
    resident = torch.cuda.memory_allocated(x.device) / 1024 ** 2  # weights, input, anything else live
    run_step(x, model, sparse=False, steps=1)  # warm-up
    loss_d, gs_d, peak_d, ms_d = run_step(x, model, sparse=False, steps=steps)
    st_d = steady_ms(x, model, sparse=False)
    cap = arena_elements(x.shape[0], hidm, layers, fill, model.W1s[0].shape[0] / hidm)
    buf = bs.init_sparse_buffer(cap, x.device, x.dtype)
    run_step(x, model, sparse=True, steps=steps)  # warm-up
    loss_s, gs_s, peak_s, ms_s = run_step(x, model, sparse=True, steps=steps)
    st_s = steady_ms(x, model, sparse=True)
    bs.check_status(x.device)
    used = buf.used()
    del buf
    bs.init_sparse_buffer(0, x.device, x.dtype)  # the per-layer form holds no arena
    run_step(x, model, sparse=True, steps=steps, exact=True)  # warm-up
    loss_e, gs_e, peak_e, ms_e = run_step(x, model, sparse=True, steps=steps, exact=True)
    st_e = steady_ms(x, model, sparse=True, exact=True)
    bs.check_status(x.device)
    rel = lambda a, b: float(((a.float() - b.float()).abs() / b.float().abs().clamp_min(1e-30)).max())  # noqa: E731
    return {"tokens": x.shape[0], "hidm": hidm, "hidden": model.W1s[0].shape[0], "layers": layers,
            "dtype": str(x.dtype).replace("torch.", ""),
            "resident_mb": round(resident, 1),
            "dense": {"peak_mb": round(peak_d, 1), "above_resident_mb": round(peak_d - resident, 1),
                      "ms_per_step": round(ms_d, 3), "steady_ms_per_step": round(st_d, 3)},
            "sparse": {"peak_mb": round(peak_s, 1), "above_resident_mb": round(peak_s - resident, 1),
                       "ms_per_step": round(ms_s, 3), "steady_ms_per_step": round(st_s, 3)},
            "sparse_exact": {"peak_mb": round(peak_e, 1), "above_resident_mb": round(peak_e - resident, 1),
                             "ms_per_step": round(ms_e, 3), "steady_ms_per_step": round(st_e, 3),
                             "loss_rel_diff": rel(loss_e, loss_d),
                             "grad_std_rel_diff": rel(gs_e[1:], gs_d[1:])},
            "arena": {"capacity_mb": round(cap * x.element_size() / 1024 ** 2, 1),
                      "used_fraction": round(used / cap, 4),
                      "activation_zeros": round(1 - used / (x.shape[0] * model.W1s[0].shape[0] * layers), 4)},
            "loss_rel_diff": rel(loss_s, loss_d), "grad_std_rel_diff": rel(gs_s[1:], gs_d[1:])}
