"""Sparse FFN autograd functions with the reference's forward/backward contract.

FFNSparse   -- out = relu(x @ W1.T) @ W2.T      (old/lib_sparse/sparse.py:56-109)
FFNSpRelu2  -- out = relu(x @ W1.T)^2 @ W2.T    (old/lib_sparse/sparse.py:112-151)

Contract kept from the reference: forward(ctx, x, W1, W2, sparse_data) saves
(x, W1, W2) with save_for_backward and keeps z = relu(x @ W1.T) only as a
tiled BitsparseTensor on ctx.z_sparse (the activation-memory saving);
backward clears it and returns one gradient per input (None for the arena).
Weights use nn.Linear layout: W1 [F, D], W2 [D, F]; x [T, D].

Differences (documented, not inherited defects): FFNSpRelu2 accepts the vals
arena (the reference's forward omits it and raises TypeError,
sparse.py:120), and both accept an optional up-projection bias b1 [F] as a
trailing argument (the reference has none).
"""
import torch
import torch.nn.functional as F
from torch.autograd import Function

from . import bitsparse as bs

__all__ = ["FFNSparse", "FFNSpRelu2"]


def _arena(sparse_data, numel, like):
    if sparse_data is not None:
        return sparse_data
    vals = torch.empty(numel, dtype=like.dtype, device=like.device)
    off = torch.zeros(1, dtype=torch.int32, device=like.device)
    return vals, off


class FFNSparse(Function):
    """ReLU FFN whose backward rebuilds the ReLU mask from the bitmask."""

    @staticmethod
    def forward(ctx, x, W1, W2, sparse_data, b1=None):
        vals, offset = _arena(sparse_data, x.shape[0] * W1.shape[0], x)
        preact = x @ W1.T
        if b1 is not None:
            preact += b1
        z = F.relu(preact)
        output = z @ W2.T
        z_sparse = bs.dense_to_tilesparse(z, vals, offset)
        del z, preact
        ctx.save_for_backward(x, W1, W2)
        ctx.z_sparse = z_sparse
        ctx.has_bias = b1 is not None
        return output

    @staticmethod
    def backward(ctx, grad_output):
        x, W1, W2 = ctx.saved_tensors
        z_sparse = ctx.z_sparse
        ctx.z_sparse = None
        grad_output = grad_output.contiguous()
        grad_z = grad_output @ W2
        grad_W2 = bs.spAx(z_sparse, grad_output.T)
        bs.mask_with_bitmask_(grad_z, z_sparse)
        grad_x = grad_z @ W1
        grad_W1 = grad_z.T @ x
        grad_b1 = grad_z.sum(0) if ctx.has_bias else None
        return grad_x, grad_W1, grad_W2, None, grad_b1


class FFNSpRelu2(Function):
    """ReLU^2 FFN: saves z = relu(pre) sparsely, rebuilds z^2 and 2z in backward."""

    @staticmethod
    def forward(ctx, x, W1, W2, sparse_data=None, b1=None):
        vals, offset = _arena(sparse_data, x.shape[0] * W1.shape[0], x)
        preact = x @ W1.T
        if b1 is not None:
            preact += b1
        z = F.relu(preact)
        output = (z * z) @ W2.T
        z_sparse = bs.dense_to_tilesparse(z, vals, offset)
        del z, preact
        ctx.save_for_backward(x, W1, W2)
        ctx.z_sparse = z_sparse
        ctx.has_bias = b1 is not None
        return output

    @staticmethod
    def backward(ctx, grad_output):
        x, W1, W2 = ctx.saved_tensors
        z_sparse = ctx.z_sparse
        ctx.z_sparse = None
        grad_output = grad_output.contiguous()
        grad_z = grad_output @ W2
        # grad_pre = grad_z * 2z; the stored z become z^2 for dW2 (sparse.py:136-147)
        bs.grad_relu2_(grad_z, z_sparse, square=True)
        grad_W2 = bs.spAx(z_sparse, grad_output.T, square=False)
        grad_x = grad_z @ W1
        grad_W1 = grad_z.T @ x
        grad_b1 = grad_z.sum(0) if ctx.has_bias else None
        return grad_x, grad_W1, grad_W2, None, grad_b1
