"""directcompute_torch_b200 -- B200-native (sm_100a) backend for the tensor hot path
of raviadi12/directcompute_torch.

The product is `libdct_cuda.so` (built in-tree from `csrc/` by `build.py`), a
C-ABI drop-in for the reference's ctypes-loaded `engine.dll`.  This package
holds the loader and the Python host side:

* `tensor`  -- `DeviceTensor`, a device tensor over one library buffer with
  reverse-mode autograd (the reference Tensor's attribute protocol);
* `ops`     -- the NumPy-semantics ops the reference has no GPU kernel for
  (broadcast binary ops with broadcast gradients, exp/log/tanh, axis and full
  reductions, fused softmax-CE, bias + ReLU with the fused backward,
  BatchNorm2d); `ops.bind(nn_engine)` builds them on the reference's own
  Tensor instead;
* `dist`    -- leading-dimension sharding across the GPUs of one node (one
  process per GPU, NCCL for the reduced-axis exchanges).

The reference's own Python tier (`nn_engine.py`) is not part of this package:
it loads `libdct_cuda.so` unmodified in place of `engine.dll`.  There is no CPU
fallback: every entry point runs on the CUDA library.
"""
from __future__ import annotations

import ctypes
import os

__all__ = ["lib_path", "load_library", "LibraryMissing"]

_HERE = os.path.dirname(os.path.abspath(__file__))


class LibraryMissing(RuntimeError):
    """libdct_cuda.so is not built (run `python -m directcompute_torch_b200.build`)."""


def lib_path() -> str:
    return os.environ.get("DCT_LIB", os.path.join(_HERE, "libdct_cuda.so"))


_LIB = None


def load_library() -> ctypes.CDLL:
    """Load libdct_cuda.so (once per process).  Raises LibraryMissing if absent."""
    global _LIB
    if _LIB is None:
        p = lib_path()
        if not os.path.exists(p):
            raise LibraryMissing(f"{p} not found; build it with `python -m directcompute_torch_b200.build`")
        _LIB = ctypes.CDLL(p)
        from . import _abi
        _abi.bind(_LIB)
    return _LIB
