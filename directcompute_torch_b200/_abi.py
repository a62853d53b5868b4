"""ctypes signatures of libdct_cuda.so (mirrors include/dct_cuda.h).

The reference entry points get exactly the argtypes/restypes `nn_engine.py`
sets (nn_engine.py:43-119, :133-134), so code written against the reference's
`lib` object behaves the same; the `dct_*` extensions get full prototypes.
"""
from __future__ import annotations

import ctypes as C

VP = C.c_void_p
U32 = C.c_uint
U64 = C.c_uint64
F32 = C.c_float
PVP = C.POINTER(C.c_void_p)
PU32 = C.POINTER(C.c_uint)
PF32 = C.POINTER(C.c_float)

# op codes (include/dct_cuda.h)
UNARY = {"relu": 0, "relu6": 1, "leaky_relu": 2, "sigmoid": 3, "exp": 4, "log_abs1p": 5, "tanh": 6,
         "neg": 7, "abs": 8}
BINARY = {"add": 20, "sub": 21, "mul": 22, "div": 23, "maximum": 24, "minimum": 25,
          # gradient helpers (same shapes except the pick masks, which broadcast)
          "sigmoid_grad": 19, "pick_max": 27, "pick_min": 28, "exp_grad": 29, "tanh_grad": 30,
          "log_abs1p_grad": 31, "copy": 32}
REDUCE = {"sum": 0, "mean": 1, "max": 2, "argmax": 3, "min": 4, "argmin": 5, "sumsq": 6}

ERRORS = {0: "OK", 1: "NO_DEVICE", 2: "HANDLE", 3: "SIZE", 4: "ARG", 5: "CUDA", 6: "UNKNOWN_SHADER",
          7: "UNSUPPORTED", 8: "DIST"}


class GPUInfo(C.Structure):
    """engine.cpp:14-21; nn_engine.py:124-132."""
    _fields_ = [("vendorId", C.c_uint), ("deviceId", C.c_uint), ("dedicatedVRAM", C.c_uint64),
                ("sharedMemory", C.c_uint64), ("isIntegrated", C.c_uint), ("description", C.c_char * 128)]


class SeqCmd(C.Structure):
    """engine.cpp:940-950; nn_engine.py:2490-2502 (200 bytes on x86-64)."""
    _fields_ = [("shader", C.c_void_p), ("srvs", C.c_void_p * 8), ("srvCount", C.c_uint),
                ("uavs", C.c_void_p * 4), ("uavCount", C.c_uint), ("threads", C.c_uint * 3),
                ("cbData", C.c_ubyte * 64), ("cbSize", C.c_uint), ("pad", C.c_uint * 1)]


#: every exported symbol: name -> (argtypes, restype); None = leave ctypes' default
SIGNATURES = {
    # -- reference entry points (nn_engine.py:43-119, :133-134) --
    "InitEngine": ([], C.c_bool),
    "GetGPUInfo": ([C.POINTER(GPUInfo)], None),
    "CompileShader": ([C.c_char_p, C.c_wchar_p], None),
    "CompileShaderEx": ([C.c_char_p, C.c_wchar_p, C.c_char_p], C.c_bool),
    "CreateBuffer": ([PF32, U32], VP),
    "AddRefBuffer": ([VP], None),
    "ReadBuffer": ([VP, PF32], None),
    "ReleaseBuffer": ([VP], None),
    "ClearBuffer": ([VP], None),
    "UpdateBuffer": ([VP, PF32], None),
    "RunShader": ([C.c_char_p, PVP, U32, PVP, U32, PU32, VP, U32], None),
    "RunShaderRaw": ([C.c_char_p, PVP, U32, PVP, U32, PU32, VP, U32], None),
    "RunShaderAlloc": ([C.c_char_p, PVP, U32, U32, PU32, VP, U32], VP),
    "RunShaderAlloc2": ([C.c_char_p, PVP, U32, U32, VP, PU32, VP, U32], VP),
    "SGDBatch": ([PVP, PVP, PU32, U32, F32, F32], None),
    "SGDBatchClipped": ([PVP, PVP, PU32, U32, F32, F32], F32),
    "ReleaseBufferBatch": ([PVP, U32], None),
    "FlushGPU": ([], None),
    "SyncGPU": ([], None),
    "MatMulAlloc": ([VP, VP, U32, U32, U32, U32], VP),
    "ConvForwardFused": ([VP, VP, VP] + [U32] * 10 + [PVP], VP),
    "ConvBackwardFused": ([VP] * 5 + [U32] * 13 + [PVP, PVP, PVP], None),
    "MaxPoolForwardFused": ([VP] + [U32] * 6 + [PVP], VP),
    "MaxPoolBackwardFused": ([VP, VP] + [U32] * 5, VP),
    "WarmPool": ([PU32, U32, U32], None),
    "GetPoolStats": ([C.POINTER(C.c_uint64), C.POINTER(C.c_uint64)], None),
    "ResetPoolStats": ([], None),
    "GetPoolMemory": ([], C.c_uint64),
    "DrainPool": ([], None),
    "ResolveShader": ([C.c_char_p], VP),
    "RunSequence": ([VP, U32], None),
    "RunSequenceWithSGD": ([VP, U32, PVP, PVP, PU32, U32, F32, F32], None),
    # -- extensions (include/dct_cuda.h) --
    "dct_last_error": ([], C.c_char_p),
    "dct_error_code": ([], C.c_int),
    "dct_clear_error": ([], None),
    "dct_version": ([], C.c_int),
    "dct_device": ([], C.c_int),
    "dct_sm_count": ([], C.c_int),
    "dct_stream": ([], VP),
    "dct_pci_bus_id": ([C.c_char_p, C.c_int], C.c_int),
    "dct_synchronize": ([], C.c_int),
    "dct_timer_start": ([], C.c_int),
    "dct_timer_stop_ms": ([], C.c_float),
    "dct_create_buffer": ([U64], VP),
    "dct_buffer_device_ptr": ([VP], VP),
    "dct_buffer_count": ([VP], U64),
    "dct_buffer_refcount": ([VP], C.c_int),
    "dct_wrap_device_ptr": ([VP, U64], VP),
    "dct_copy_h2d": ([VP, VP, U64, U64], C.c_int),
    "dct_copy_d2h": ([VP, VP, U64, U64], C.c_int),
    "dct_host_alloc": ([U64], VP),
    "dct_host_free": ([VP], None),
    "dct_fill_random": ([VP, U64, U64, C.c_int, F32, F32], C.c_int),
    "dct_scatter": ([VP, C.POINTER(C.c_int64), C.POINTER(C.c_float), U64], C.c_int),
    "dct_unary": ([C.c_int, VP, VP, U64, F32], C.c_int),
    "dct_binary": ([C.c_int, VP, C.POINTER(C.c_int64), C.c_int, VP, C.POINTER(C.c_int64), C.c_int, VP], C.c_int),
    "dct_reduce": ([C.c_int, VP, U64, U64, U64, VP, VP], C.c_int),
    "dct_reduce_all": ([C.c_int, VP, U64, VP, C.POINTER(C.c_double)], C.c_int),
    "dct_softmax_ce": ([VP, VP, C.c_int, U32, U32, VP, VP, VP, VP, F32, F32], C.c_int),
    "dct_adam": ([VP, VP, VP, VP, U64, F32, F32, F32, F32, F32, F32], C.c_int),
    "dct_adam_batch": ([PVP, PVP, PVP, PVP, PU32, U32, F32, F32, F32, F32, F32, F32], C.c_int),
    "dct_batchnorm_forward_train": ([VP] * 8 + [U32, U32, U32, F32, F32], C.c_int),
    "dct_batchnorm_backward": ([VP] * 8 + [U32, U32, U32, F32], C.c_int),
    "dct_batchnorm_forward_train_noalloc": ([VP] * 8 + [U32, U32, U32, F32, F32, VP], C.c_int),
    "dct_sum_to_shape": ([VP, C.POINTER(C.c_int64), C.c_int, C.POINTER(C.c_int64), C.c_int, VP], C.c_int),
    "dct_broadcast_to": ([VP, C.POINTER(C.c_int64), C.c_int, C.POINTER(C.c_int64), C.c_int, VP], C.c_int),
    "dct_bias_relu_backward": ([VP, VP, VP, VP, U32, U32], C.c_int),
    # sharding over NCCL
    "dct_dist_available": ([], C.c_int),
    "dct_dist_nccl_version": ([], C.c_int),
    "dct_dist_shard": ([U64, C.c_int, C.c_int, C.POINTER(U64), C.POINTER(U64)], C.c_int),
    "dct_dist_unique_id": ([VP, C.c_int], C.c_int),
    "dct_dist_init": ([VP, C.c_int, C.c_int, C.c_int, C.c_double], C.c_int),
    "dct_dist_finalize": ([], C.c_int),
    "dct_dist_rank": ([], C.c_int),
    "dct_dist_world": ([], C.c_int),
    "dct_dist_peer_active": ([], C.c_int),
    "dct_dist_allreduce": ([VP, U64, C.c_int], C.c_int),
    "dct_dist_broadcast": ([VP, U64, C.c_int], C.c_int),
    "dct_dist_barrier": ([], C.c_int),
    "dct_dist_reduce": ([C.c_int, VP, U64, U64, U64, U64, U64, VP, VP], C.c_int),
    "dct_dist_reduce_all": ([C.c_int, VP, U64, VP, C.POINTER(C.c_double)], C.c_int),
    "dct_dist_softmax_ce": ([VP, VP, C.c_int, U32, U32, VP, VP, VP, VP, F32, F32], C.c_int),
    "dct_dist_batchnorm_forward_train": ([VP] * 8 + [U32, U32, U32, F32, F32], C.c_int),
    "dct_dist_batchnorm_backward": ([VP] * 8 + [U32, U32, U32, F32], C.c_int),
    "dct_selftest_bounded_wait": ([U32], C.c_int),
}

#: the 32 symbols of the reference engine (31 bound by nn_engine.py + SyncGPU)
REFERENCE_SYMBOLS = tuple(k for k in SIGNATURES if not k.startswith("dct_"))


def bind(lib) -> None:
    for name, (args, res) in SIGNATURES.items():
        f = getattr(lib, name)
        f.argtypes = args
        if res is not None or name in ("GetGPUInfo",):
            f.restype = res


def check(lib, rc: int, what: str = "") -> None:
    """Raise RuntimeError for a non-zero dct_* status, with the library's message."""
    if rc != 0:
        msg = lib.dct_last_error()
        raise RuntimeError(f"libdct_cuda {what}: {ERRORS.get(rc, rc)}: {msg.decode() if msg else ''}")
