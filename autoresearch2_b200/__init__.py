"""B200-native (sm_100a) activation-sparse FFN hot path with the reference's API.

Reference: Maccy-Z/autoresearch2 (old/lib_sparse/sparse.py, old/sparse_pack.py,
old/sparse_unpack.py, old/full_matmul/sparse_pack.py).  All compute runs in
libsparseffn.so (hand-written CUDA for sm_100a behind a C ABI,
include/sparseffn.h); there is no CPU or fallback path.  The operations are also
registered as torch.library ops (sparseffn::*, library.py) for torch.compile.
"""
from .bitsparse import (BitsparseTensor, TensorBuffer, bitsparse_pack, bitsparse_pack_async, bitsparse_unpack,
                        check_status, compress_dense, dense_to_tilesparse, get_globals, grad_relu2_,
                        init_sparse_buffer, mask_with_bitmask_, reconstruct_bitmask, reset_sparse_globals,
                        spAx, tile_unpack)
from .ffn import (FFNSparse, FFNSpRelu2, backward_mode, compact_k, set_backward, set_compact_k,
                  set_sparse_mma, sparse_mma)
from . import bitshift, deep, ffn, gpt, library, parallel, sp24, tiled  # library registers the sparseffn:: ops

__all__ = [
    "BitsparseTensor", "TensorBuffer", "bitsparse_pack", "bitsparse_pack_async", "bitsparse_unpack", "check_status",
    "compress_dense", "reconstruct_bitmask",
    "dense_to_tilesparse", "get_globals", "grad_relu2_", "init_sparse_buffer",
    "mask_with_bitmask_", "reset_sparse_globals", "spAx", "tile_unpack", "FFNSparse",
    "FFNSpRelu2", "set_sparse_mma", "sparse_mma", "set_compact_k", "compact_k", "set_backward", "backward_mode",
    "bitshift", "deep", "gpt", "library", "parallel", "sp24", "tiled",
]
