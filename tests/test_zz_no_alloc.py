"""The no-allocation flat pack entry point, called through the C ABI.

sffn_flat_pack_noalloc serves callers that cannot allocate device memory --
plug-ins that are handed only their input and output buffers, programs whose
memory manager owns the device or runs to a fixed budget, and paths that must
not risk the synchronisation a cudaMalloc can cause.  It keeps its scratch in
a fixed array inside the library instead of taking a workspace.  These checks
compare it with the oracle (the C restatement of the reference's bit order,
old/bitpack/prepare.py:6-23) and with the regular sffn_flat_pack (which takes
a workspace) on two calls in a row -- the second call finds the first call's
state in the shared array and must clear it -- over bf16, fp16 and fp32,
values off a 16-byte boundary, a capacity below the count, an empty input and
a last tile shorter than 16 bytes; they check that oversized inputs are
refused and that the caller's current device is the same after the call.
Masks, values and counts are integer/byte results, so they must match exactly.

This file is collected last on purpose: it must pass in a fresh process (the
first call does the per-device set-up) and after every other test.
"""
import ctypes

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu
DEV = "cuda"
SENTINEL = 7


def _oracle_bits(d):
    """The tensor as the oracle's numpy form (bf16 as its uint16 bits)."""
    c = d.detach().cpu().contiguous()
    if c.dtype == torch.bfloat16:
        return c.view(torch.int16).numpy().view(np.uint16).ravel()
    return c.numpy().ravel()


def _pack(d, noalloc, cap=None, vals_offset=0):
    """One pack through the C ABI into fresh sentinel-filled buffers; returns
    (mask, vals buffer, nnz, status).  `vals_offset` elements shift the
    values' start (2 bytes for 16-bit types: off the 16-byte boundary)."""
    from autoresearch2_b200 import _lib
    L = _lib.load()
    n = d.numel()
    cap = n if cap is None else cap
    code = _lib.dtype_code(d)
    st = _lib.stream_ptr(d.device)
    mask = torch.full((max((n + 7) // 8, 1),), 0xAB, dtype=torch.uint8, device=DEV)
    vbuf = torch.full((cap + vals_offset + 8,), SENTINEL, dtype=d.dtype, device=DEV)
    vals = vbuf[vals_offset:]
    out = torch.zeros(2, dtype=torch.int64, device=DEV)  # nnz, status
    nnz_p = ctypes.c_void_p(out.data_ptr())
    status_p = ctypes.c_void_p(out.data_ptr() + 8)
    if noalloc:
        rc = L.sffn_flat_pack_noalloc(_lib.ptr(d), code, n, _lib.ptr(mask), _lib.ptr(vals), cap,
                                      nnz_p, status_p, st)
    else:
        ws = _lib.workspace(L.sffn_flat_pack_workspace_bytes(n, code), d.device)
        rc = L.sffn_flat_pack(_lib.ptr(d), code, n, _lib.ptr(mask), _lib.ptr(vals), cap, nnz_p,
                              _lib.ptr(ws), ws.numel(), status_p, st)
    assert rc == 0, L.sffn_error_string(rc)
    torch.cuda.synchronize()
    nnz, status = out.tolist()
    return mask[:(n + 7) // 8], vals, nnz, status


def _data(rows, cols, p, dtype, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    keep = torch.rand(rows, cols, device=DEV, generator=g) < p
    return torch.where(keep, torch.randn(rows, cols, device=DEV, generator=g),
                       torch.zeros((), device=DEV)).to(dtype).flatten()


def _bits(t):
    return t.view(torch.int16) if t.element_size() == 2 else t.view(torch.int32)


def _check_against_oracle_and_workspace_pack(d):
    want_vals, want_mask = oracle.flat_pack(_oracle_bits(d))
    m1, v1, n1, s1 = _pack(d, noalloc=True)
    m0, v0, n0, s0 = _pack(d, noalloc=False)
    assert s1 == 0 and s0 == 0
    assert n1 == n0 == want_vals.size
    assert np.array_equal(m1.cpu().numpy(), want_mask)
    assert torch.equal(m1, m0)
    assert np.array_equal(_bits(v1[:n1]).cpu().numpy().view(want_vals.dtype), want_vals)
    assert torch.equal(_bits(v1[:n1]), _bits(v0[:n0]))
    assert bool((_bits(v1[n1:]) == _bits(torch.full((1,), SENTINEL, dtype=d.dtype, device=DEV))).all())


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_noalloc_matches_oracle_and_workspace_pack_on_two_calls(dtype):
    # two calls in a row with different sizes and densities
    for k, (rows, cols, p) in enumerate(((1024, 4099, 0.3), (3000, 2048, 0.05))):
        _check_against_oracle_and_workspace_pack(_data(rows, cols, p, dtype, 11 + k))


@pytest.mark.parametrize("dtype,n", [(torch.bfloat16, 16384 * 3 + 5), (torch.float32, 8192 * 2 + 3),
                                     (torch.float16, 7)])
def test_noalloc_last_tile_under_16_bytes(dtype, n):
    _check_against_oracle_and_workspace_pack(_data(1, n, 0.4, dtype, 5))


def test_noalloc_values_off_a_16_byte_boundary():
    d = _data(700, 3001, 0.2, torch.bfloat16, 3)
    want_vals, want_mask = oracle.flat_pack(_oracle_bits(d))
    m, v, nnz, status = _pack(d, noalloc=True, vals_offset=1)
    assert status == 0 and nnz == want_vals.size
    assert np.array_equal(m.cpu().numpy(), want_mask)
    assert np.array_equal(_bits(v[:nnz]).cpu().numpy().view(np.uint16), want_vals)


def test_noalloc_capacity_below_the_count():
    d = _data(512, 4096, 0.3, torch.bfloat16, 9)
    want_vals, want_mask = oracle.flat_pack(_oracle_bits(d))
    cap = want_vals.size // 3
    m, v, nnz, status = _pack(d, noalloc=True, cap=cap)
    assert status & 1  # SFFN_STATUS_VALS_OVERFLOW
    assert nnz == want_vals.size
    assert np.array_equal(m.cpu().numpy(), want_mask)
    assert np.array_equal(_bits(v[:cap]).cpu().numpy().view(np.uint16), want_vals[:cap])
    assert bool((_bits(v[cap:]) == _bits(torch.full((1,), SENTINEL, dtype=d.dtype, device=DEV))).all())


def test_noalloc_empty_input():
    from autoresearch2_b200 import _lib
    L = _lib.load()
    out = torch.full((2,), 5, dtype=torch.int64, device=DEV)
    out[1] = 0
    rc = L.sffn_flat_pack_noalloc(None, _lib.BF16, 0, None, None, 0, ctypes.c_void_p(out.data_ptr()),
                                  ctypes.c_void_p(out.data_ptr() + 8), _lib.stream_ptr(DEV))
    assert rc == 0
    torch.cuda.synchronize()
    assert out.tolist() == [0, 0]


def test_noalloc_refuses_sizes_beyond_its_capacity():
    from autoresearch2_b200 import _lib
    L = _lib.load()
    too_many = 67_108_864 + 1
    dummy = torch.zeros(16, dtype=torch.uint8, device=DEV)
    out = torch.zeros(2, dtype=torch.int64, device=DEV)
    rc = L.sffn_flat_pack_noalloc(_lib.ptr(dummy), _lib.BF16, too_many, _lib.ptr(dummy),
                                  _lib.ptr(dummy), 0, ctypes.c_void_p(out.data_ptr()),
                                  ctypes.c_void_p(out.data_ptr() + 8), _lib.stream_ptr(DEV))
    assert rc == 8  # SFFN_ERR_TOO_LARGE
    assert b"capacity" in L.sffn_last_cuda_error()


def test_noalloc_keeps_the_callers_current_device():
    """A call on a tensor of device 0 made while another device is current
    leaves that device current (skipped with one GPU, where the call must
    still leave device 0 current)."""
    d0 = _data(64, 1024, 0.3, torch.bfloat16, 1)
    if torch.cuda.device_count() < 2:
        _pack(d0, noalloc=True)
        assert torch.cuda.current_device() == 0
        pytest.skip("needs two GPUs to make another device current")
    from autoresearch2_b200 import _lib
    L = _lib.load()
    mask = torch.empty(d0.numel() // 8, dtype=torch.uint8, device="cuda:0")
    vals = torch.empty_like(d0)
    out = torch.zeros(2, dtype=torch.int64, device="cuda:0")
    prev = torch.cuda.current_device()
    try:
        torch.cuda.set_device(1)
        rc = L.sffn_flat_pack_noalloc(_lib.ptr(d0), _lib.BF16, d0.numel(), _lib.ptr(mask), _lib.ptr(vals),
                                      vals.numel(), ctypes.c_void_p(out.data_ptr()),
                                      ctypes.c_void_p(out.data_ptr() + 8),
                                      ctypes.c_void_p(torch.cuda.current_stream(0).cuda_stream))
        assert rc == 0
        assert torch.cuda.current_device() == 1
        # a buffer on another device than the input is refused
        other = torch.zeros(2, dtype=torch.int64, device="cuda:1")
        rc = L.sffn_flat_pack_noalloc(_lib.ptr(d0), _lib.BF16, d0.numel(), _lib.ptr(mask), _lib.ptr(vals),
                                      vals.numel(), ctypes.c_void_p(other.data_ptr()),
                                      ctypes.c_void_p(other.data_ptr() + 8),
                                      ctypes.c_void_p(torch.cuda.current_stream(0).cuda_stream))
        assert rc == 1  # SFFN_ERR_ARG
        assert torch.cuda.current_device() == 1
    finally:
        torch.cuda.set_device(prev)
    torch.cuda.synchronize(0)
    want_vals, _ = oracle.flat_pack(_oracle_bits(d0))
    assert int(out[0].item()) == want_vals.size and int(out[1].item()) == 0
