"""ctypes binding of libsparseffn.so (the C ABI declared in include/sparseffn.h).

The library is the only compute path: if it is missing, every operation
raises instead of falling back to another implementation.
"""
import ctypes
import os

import torch

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libsparseffn.so")

F32, BF16, F16 = 0, 1, 2
_DTYPES = {torch.float32: F32, torch.bfloat16: BF16, torch.float16: F16}

STATUS_BITS = {
    1: "vals capacity exceeded (output clipped)",
    2: "bounded device wait timed out",
    4: "int32 arena cursor overflow",
    8: "mask has more set bits than vals holds",
}


class SparseFFNError(RuntimeError):
    """Raised when the CUDA library reports an error."""


_vp, _i64, _i32, _int, _sz = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_int, ctypes.c_size_t

# name -> (restype, argtypes)
SIGNATURES = {
    "sffn_sp24_compress": (_int, [_vp, _i64, _int, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _vp]),
    "sffn_gemm_sp24": (_int, [_vp, _vp, _i64, _i64, _vp, _i64, _int, _vp, _i64, _i64, _vp, _vp]),
    "sffn_sp24_overflow_add": (_int, [_vp, _vp, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _vp]),
    "sffn_transpose16": (_int, [_vp, _i64, _i64, _i64, _vp, _i64, _vp]),
    "sffn_codec15_bytes": (_i64, [_i64]),
    "sffn_codec15_compress": (_int, [_vp, _i64, _vp, _i64, _vp]),
    "sffn_codec15_uncompress": (_int, [_vp, _i64, _i64, _vp, _vp]),
    "sffn_sp24_mm": (_int, [_vp, _i64, _i64, _vp, _i64, _int, _vp, _i64, _vp, _i64, _int, _i64, _vp, _vp]),
    "sffn_ffn_up_sp24": (_int, [_vp, _i64, _vp, _i64, _vp, _i64, _i64, _i64, _int, _vp, _vp, _vp, _vp,
                                _vp, _vp, _vp]),
    "sffn_ffn_dgrad_sp24": (_int, [_vp, _i64, _vp, _i64, _i64, _i64, _i64, _int, _vp, _i64, _vp, _vp, _vp,
                                   _vp, _vp, _vp, _vp, _vp, _vp]),
    "sffn_version": (_int, []),
    "sffn_error_string": (ctypes.c_char_p, [_int]),
    "sffn_last_cuda_error": (ctypes.c_char_p, []),
    "sffn_flat_workspace_bytes": (_sz, [_i64]),
    "sffn_flat_pack_workspace_bytes": (_sz, [_i64, _int]),
    "sffn_flat_pack_count": (_int, [_vp, _int, _i64, _vp, _vp, _vp, _sz, _vp]),
    "sffn_flat_pack_values": (_int, [_int, _i64, _vp, _i64, _vp, _vp, _sz, _vp, _vp]),
    "sffn_flat_pack": (_int, [_vp, _int, _i64, _vp, _vp, _i64, _vp, _vp, _sz, _vp, _vp]),
    "sffn_flat_unpack": (_int, [_vp, _i64, _vp, _int, _i64, _vp, _vp, _sz, _vp, _vp]),
    "sffn_flat_pack_noalloc": (_int, [_vp, _int, _i64, _vp, _vp, _i64, _vp, _vp, _vp]),
    "sffn_tile_workspace_bytes": (_sz, [_i64, _i64, _int, _int]),
    "sffn_tile_pack": (_int, [_vp, _int, _i64, _i64, _i64, _int, _int, _vp, _vp, _vp, _i64, _vp,
                              _vp, _vp, _sz, _vp, _vp]),
    "sffn_tile_pack_values": (_int, [_vp, _int, _i64, _i64, _i64, _int, _int, _vp, _vp, _vp, _i64, _vp, _vp,
                                     _vp]),
    "sffn_tile_unpack": (_int, [_vp, _i64, _vp, _vp, _vp, _int, _i64, _i64, _int, _int, _i64,
                                _i64, _int, _vp, _int, _i64, _vp]),
    "sffn_tile_mask_grad": (_int, [_vp, _int, _i64, _i64, _i64, _vp, _int, _int, _vp]),
    "sffn_tile_grad_relu2": (_int, [_vp, _int, _i64, _i64, _i64, _vp, _i64, _vp, _vp, _vp, _int,
                                    _int, _int, _vp]),
    "sffn_gemm_bf16": (_int, [_vp, _i64, _int, _vp, _i64, _int, _vp, _i64, _i64, _i64, _i64, _vp,
                              _vp, _int, _vp, _vp]),
    "sffn_ffn_up": (_int, [_vp, _i64, _vp, _i64, _vp, _i64, _i64, _i64, _int, _vp, _i64, _vp, _vp,
                           _vp, _vp, _vp, _vp]),
    "sffn_tile_copy_slots": (_int, [_vp, _vp, _vp, _vp, _i64, _vp, _i64, _vp, _vp, _vp, _vp, _vp]),
    "sffn_tile_scan_counts": (_int, [_vp, _int, _i64, _vp, _vp, _vp, _vp, _vp]),
    "sffn_tile_gather_slots": (_int, [_vp, _vp, _vp, _vp, _i64, _vp, _i64, _int, _vp, _vp, _vp, _vp]),
    "sffn_tile_row_offsets": (_int, [_vp, _vp, _i64, _vp, _vp, _vp]),
    "sffn_ck_lists": (_int, [_vp, _i64, _i64, _vp, _i64, _vp, _vp, _vp]),
    "sffn_ck_gather_packed": (_int, [_vp, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _int, _vp,
                                     _i64, _vp, _vp]),
    "sffn_ck_compact_rows": (_int, [_vp, _i64, _i64, _i64, _vp, _i64, _vp, _vp]),
    "sffn_gemm_ck": (_int, [_vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _vp, _vp, _i64, _i64, _i64, _vp,
                            _vp]),
    "sffn_live_kblocks": (_int, [_vp, _i64, _i64, _vp, _vp, _vp]),
    "sffn_live_kblocks_t": (_int, [_vp, _i64, _i64, _vp, _vp, _vp]),
    "sffn_split_bf16x3": (_int, [_vp, _int, _i64, _i64, _i64, _i64, _vp, _i64, _int, _vp]),
    "sffn_gemm_bf16_f32out": (_int, [_vp, _i64, _int, _vp, _i64, _int, _vp, _i64, _i64, _i64, _i64, _int, _vp,
                                     _vp]),
    "sffn_gemm_relu": (_int, [_vp, _i64, _int, _vp, _i64, _int, _vp, _int, _i64, _i64, _i64, _i64, _vp, _vp, _int,
                              _vp, _vp]),
    "sffn_gemm_bf16_f32acc": (_int, [_vp, _i64, _int, _vp, _i64, _int, _vp, _i64, _i64, _i64, _i64, _int,
                                     _vp, _vp]),
    "sffn_gemm_tf32": (_int, [_vp, _i64, _vp, _i64, _vp, _i64, _i64, _i64, _i64, _int, _vp, _vp]),
    "sffn_round_tf32": (_int, [_vp, _vp, _i64, _vp]),
    "sffn_gemm_bf16_ct": (_int, [_vp, _i64, _int, _vp, _i64, _int, _vp, _i64, _i64, _i64, _i64, _vp,
                                 _vp, _int, _vp, _vp]),
    "sffn_ffn_dgrad": (_int, [_vp, _i64, _vp, _i64, _i64, _i64, _i64, _int, _vp, _i64, _vp, _vp,
                              _vp, _vp, _vp, _i64, _vp, _vp, _vp]),
    "sffn_wait_probe": (_int, [_int, _i64, _vp, _vp, _vp, _vp]),
}

_lib = None


def load():
    """Load libsparseffn.so once; raise if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python -m autoresearch2_b200.build` "
                "(this package has no CPU or fallback path)")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


# Kernels of this library each entry point launches per call.
LAUNCHING = {"sffn_sp24_compress": 1, "sffn_gemm_sp24": 1, "sffn_sp24_overflow_add": 1,
             "sffn_ffn_up_sp24": 1, "sffn_ffn_dgrad_sp24": 1, "sffn_sp24_mm": 1, "sffn_transpose16": 1,
             "sffn_flat_pack": 2, "sffn_flat_pack_count": 2, "sffn_flat_pack_values": 1,
             "sffn_flat_pack_noalloc": 1, "sffn_flat_unpack": 2, "sffn_tile_pack": 3, "sffn_tile_pack_values": 1,
             "sffn_tile_unpack": 1, "sffn_tile_mask_grad": 1, "sffn_tile_grad_relu2": 1,
             "sffn_gemm_bf16": 1, "sffn_ffn_up": 1, "sffn_tile_scan_counts": 1,
             "sffn_tile_gather_slots": 1, "sffn_tile_row_offsets": 1, "sffn_live_kblocks": 1,
             "sffn_ffn_dgrad": 1, "sffn_codec15_compress": 1, "sffn_codec15_uncompress": 1,
             "sffn_wait_probe": 1, "sffn_ck_lists": 1, "sffn_ck_gather_packed": 1,
             "sffn_ck_compact_rows": 1, "sffn_gemm_ck": 1, "sffn_live_kblocks_t": 1, "sffn_gemm_bf16_ct": 1,
             "sffn_split_bf16x3": 1, "sffn_gemm_bf16_f32out": 1, "sffn_tile_copy_slots": 1,
             "sffn_gemm_bf16_f32acc": 1, "sffn_gemm_tf32": 1, "sffn_gemm_relu": 1,
             "sffn_round_tf32": 1}
launch_count = 0

# Per-entry-point CUDA event pairs, recorded while a KernelTimer is active.
_timer = None


class KernelTimer:
    """Brackets every launching entry point called inside ``with`` with CUDA
    events on the current stream (the stream the library launches on), so the
    device time of each kernel can be read inside a timed region without
    synchronising.  ``summary()`` (after a synchronize) gives per entry point
    the call count and mean/total milliseconds."""

    def __init__(self):
        self.events = {}

    def __enter__(self):
        global _timer
        self._prev, _timer = _timer, self
        return self

    def __exit__(self, *exc):
        global _timer
        _timer = self._prev

    def summary(self):
        out = {}
        for name, pairs in self.events.items():
            ms = [a.elapsed_time(b) for a, b in pairs]
            out[name] = {"calls": len(ms), "total_ms": sum(ms), "mean_ms": sum(ms) / len(ms)}
        return out


def _launches(name, args):
    """Kernels one successful call launched: LAUNCHING's count, except where
    it depends on the arguments (the float32-output GEMM runs one launch per
    K chunk of 1024; the tile pack without vals stops after count and scan)."""
    if name == "sffn_gemm_bf16_f32out":
        return -(-int(args[10]) // 1024)
    if name == "sffn_tile_pack":
        v = args[9]
        return 2 if v is None or getattr(v, "value", v) in (None, 0) else 3
    return LAUNCHING.get(name, 0)


def call(name, *args):
    """Call a C-ABI entry point and raise SparseFFNError on a non-zero code."""
    global launch_count
    lib = load()
    timer = _timer if name in LAUNCHING else None
    if timer is not None:
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
    rc = getattr(lib, name)(*args)
    if timer is not None:
        b.record()
        timer.events.setdefault(name, []).append((a, b))
    if rc == 0:
        launch_count += _launches(name, args)
    if rc != 0:
        msg = lib.sffn_error_string(rc).decode()
        if rc == 5:
            msg += f" ({lib.sffn_last_cuda_error().decode()})"
        raise SparseFFNError(f"{name} failed: {msg}")
    return rc


def dtype_code(t):
    try:
        return _DTYPES[t.dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {t.dtype}; expected float32, bfloat16 or float16") from None


def ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def stream_ptr(device=None):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def require_cuda(*tensors):
    for t in tensors:
        if not (isinstance(t, torch.Tensor) and t.is_cuda):
            raise ValueError("autoresearch2_b200 runs on CUDA tensors only (no CPU path)")


# Sticky per-device status word: kernels OR SFFN_STATUS_* bits into it.
_status = {}


def status_word(device):
    idx = torch.device(device).index
    if idx is None:
        idx = torch.cuda.current_device()
    t = _status.get(idx)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=f"cuda:{idx}")
        _status[idx] = t
    return t


def check_status(device=None, raise_on_error=True):
    """Synchronise-read and clear the device status word; raise if bits are set."""
    st = status_word(device if device is not None else torch.cuda.current_device())
    v = int(st.item())
    if v:
        st.zero_()
        if raise_on_error:
            what = ", ".join(m for b, m in STATUS_BITS.items() if v & b)
            raise SparseFFNError(f"device status 0x{v:x}: {what}")
    return v


def workspace(nbytes, device):
    return torch.empty(max(int(nbytes), 16), dtype=torch.uint8, device=device)
