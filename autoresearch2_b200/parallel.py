"""Token-sharded data parallelism for the sparse FFN.

Every rank (one process per GPU) holds the full W1/W2 and a disjoint shard of
the tokens; masks, values and the arena cursor are per-token-row, so nothing
about the sparse format crosses GPUs.  The only exchange is the sum of the
weight gradients, an NCCL all_reduce over NVLink/NVSwitch.  (The reference has
no multi-GPU code; its harness runs one GPU, program.md:27.)

GradAllReduce overlaps that sum with the rest of the backward: inside
``with comm.attached():`` the fused FFN backward hands each weight gradient to
the communicator as soon as it is computed -- dW2 comes out of the first
backward GEMM and dW1 out of the next, so their all_reduces run on a side
stream while dW1 and then dX are still being computed; dX, computed last,
needs no reduction.  ``comm.wait()`` makes the current stream wait for all
reductions.  On CPU tensors (the gloo backend) the reduction is synchronous.
"""
import contextlib

import torch
import torch.distributed as dist

__all__ = ["GradAllReduce", "current"]

_current = None


def current():
    """The communicator attached to backward passes, or None."""
    return _current


class GradAllReduce:
    """Sums gradients over a process group as they become ready."""

    def __init__(self, group=None, average=False):
        self.group = group
        self.average = average
        self.stream = None
        self.pending = []

    def submit(self, t: torch.Tensor):
        """Start the all_reduce of `t` (a gradient that is final on the
        current stream).  The result is written into `t` in place."""
        if not dist.is_initialized() or dist.get_world_size(self.group) == 1:
            return t
        if t.is_cuda:
            if self.stream is None:
                self.stream = torch.cuda.Stream(device=t.device)
            ready = torch.cuda.Event()
            ready.record(torch.cuda.current_stream(t.device))
            with torch.cuda.stream(self.stream):
                self.stream.wait_event(ready)
                t.record_stream(self.stream)
                work = dist.all_reduce(t, group=self.group, async_op=True)
            self.pending.append((work, t))
        else:
            dist.all_reduce(t, group=self.group)
            if self.average:
                t.div_(dist.get_world_size(self.group))
        return t

    def wait(self):
        """Make the current stream wait for every submitted reduction."""
        for work, t in self.pending:
            work.wait()
            if self.average:
                t.div_(dist.get_world_size(self.group))
        self.pending.clear()

    @contextlib.contextmanager
    def attached(self):
        """Route the FFN backward's weight gradients to this communicator."""
        global _current
        prev, _current = _current, self
        try:
            yield self
        finally:
            _current = prev


def submit_grad(t):
    """Called by the FFN backward for each weight gradient it produces."""
    comm = _current
    if comm is not None and t is not None:
        comm.submit(t)
    return t
