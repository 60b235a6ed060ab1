"""Bounded device waits that run out.

Every spin-wait in the library's kernels gives up after a wall-time limit,
records SFFN_STATUS_WAIT_TIMEOUT in the caller's status word and returns, so
that a wait that never ends cannot hang the GPU.  sffn_wait_probe runs the two
kinds of wait the kernels use -- an mbarrier wait (GEMM and pack pipelines)
and a decoupled look-back (tiled and flat packs) -- on a condition nothing
makes true, with a short limit.  The checks: the wait lasted at least the
limit, the status bit is set, and the context still gives correct results
afterwards.  Nothing here faults: no memory is out of bounds and no copy is in
flight when a wait gives up."""
import ctypes

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu
DEV = "cuda"
TIMEOUT_BIT = 2


@pytest.mark.parametrize("kind", [0, 1])
@pytest.mark.parametrize("limit_ms", [1, 5])
def test_wait_that_runs_out_sets_the_status_and_returns(kind, limit_ms):
    from autoresearch2_b200 import _lib
    L = _lib.load()
    states = torch.empty(64, dtype=torch.int64, device=DEV)
    elapsed = torch.zeros(1, dtype=torch.int64, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    rc = L.sffn_wait_probe(kind, limit_ms * 1_000_000, _lib.ptr(states), _lib.ptr(elapsed), _lib.ptr(status),
                           _lib.stream_ptr(DEV))
    assert rc == 0, L.sffn_error_string(rc)
    torch.cuda.synchronize()
    assert int(status.item()) & TIMEOUT_BIT
    waited_ns = int(elapsed.item())
    assert limit_ms * 1_000_000 <= waited_ns < 1_000_000_000
    # the context is still usable: a pack afterwards is exact
    import autoresearch2_b200 as sf
    g = torch.Generator(device=DEV).manual_seed(kind + limit_ms)
    d = torch.where(torch.rand(300, 1000, device=DEV, generator=g) < 0.2,
                    torch.randn(300, 1000, device=DEV, generator=g), torch.zeros((), device=DEV))
    vals, mask = sf.bitsparse_pack(d)
    want_vals, want_mask = oracle.flat_pack(d.cpu().numpy())
    assert np.array_equal(mask.cpu().numpy(), want_mask)
    assert np.array_equal(vals.cpu().numpy(), want_vals)
    sf.check_status()


def test_wait_probe_argument_checks():
    from autoresearch2_b200 import _lib
    L = _lib.load()
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    st = _lib.stream_ptr(DEV)
    assert L.sffn_wait_probe(2, 1_000_000, None, None, _lib.ptr(status), st) == 1
    assert L.sffn_wait_probe(0, 0, None, None, _lib.ptr(status), st) == 1
    assert L.sffn_wait_probe(0, 200_000_000, None, None, _lib.ptr(status), st) == 1  # above 100 ms
    assert L.sffn_wait_probe(1, 1_000_000, None, None, _lib.ptr(status), st) == 1  # no states
    torch.cuda.synchronize()
    assert int(status.item()) == 0
