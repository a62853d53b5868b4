"""`FakeLib`: the reference's native C-ABI implemented over NumPy (test oracle only).

`nn_engine.py` loads its native engine with `ctypes.CDLL(_find_resource("engine.dll"))`
(nn_engine.py:42) and binds 31 symbols (nn_engine.py:43-119).  This class provides
every one of them as a Python callable with the same argument meaning, backed by
flat float32 NumPy buffers and `oracle.shaders.run_shader`.  `load_reference_engine`
swaps it in for the DLL so the UNMODIFIED reference Python (its Tensor/autograd,
optimizers and its own verification scripts) runs on the CPU.

Semantics restated from engine.cpp:
  CreateBuffer / size-keyed pool / MaxPoolForSize   engine.cpp:181-253
  AddRefBuffer / ReleaseBuffer / ReleaseBufferBatch  engine.cpp:255-290, 676-685
  ReadBuffer / UpdateBuffer / ClearBuffer            engine.cpp:261-265, 292-321, 349-354
  RunShader / RunShaderAlloc(2)                      engine.cpp:396-426
  SGDBatch / SGDBatchClipped                         engine.cpp:436-614
  WarmPool / pool stats / DrainPool                  engine.cpp:617-673
  ResolveShader / RunSequence(WithSGD)               engine.cpp:934-977
"""
from __future__ import annotations

import contextlib
import ctypes
import importlib
import os
import struct
import sys
import tempfile

import numpy as np

from . import shaders

F32 = np.float32


class SeqCmd(ctypes.Structure):
    """The reference's packed dispatch command (engine.cpp:940-950; 200 bytes on x86-64)."""
    _fields_ = [
        ("shader", ctypes.c_void_p),
        ("srvs", ctypes.c_void_p * 8),
        ("srvCount", ctypes.c_uint),
        ("uavs", ctypes.c_void_p * 4),
        ("uavCount", ctypes.c_uint),
        ("threads", ctypes.c_uint * 3),
        ("cbData", ctypes.c_ubyte * 64),
        ("cbSize", ctypes.c_uint),
        ("pad", ctypes.c_uint * 1),
    ]


class GPUInfo(ctypes.Structure):
    """engine.cpp:14-21 / nn_engine.py:124-132."""
    _fields_ = [
        ("vendorId", ctypes.c_uint),
        ("deviceId", ctypes.c_uint),
        ("dedicatedVRAM", ctypes.c_uint64),
        ("sharedMemory", ctypes.c_uint64),
        ("isIntegrated", ctypes.c_uint),
        ("description", ctypes.c_char * 128),
    ]


def _addr(p):
    """Address behind a ctypes pointer / byref / c_void_p / int (None -> 0)."""
    if p is None:
        return 0
    if isinstance(p, int):
        return p
    if hasattr(p, "_obj"):                       # ctypes.byref(...)
        return ctypes.addressof(p._obj)
    if isinstance(p, ctypes.c_void_p):
        return p.value or 0
    if isinstance(p, ctypes.Array):
        return ctypes.addressof(p)
    return ctypes.cast(p, ctypes.c_void_p).value or 0


def _set_out_ptr(p, value) -> None:
    """Store a handle through a `void**` out-parameter (ctypes.byref / pointer / address)."""
    ctypes.c_void_p.from_address(_addr(p)).value = int(value) if value else None


class _Buf:
    __slots__ = ("data", "count", "ref")

    def __init__(self, count):
        self.data = np.zeros(count, dtype=F32)
        self.count = count
        self.ref = 1


class FakeLib:
    """NumPy implementation of the reference engine's exported symbols."""

    def __init__(self, vram_bytes: int = 180 * 1024 ** 3):
        self._bufs: dict[int, _Buf] = {}
        self._next = 0x1000
        self._pool: dict[int, list[int]] = {}
        self.hits = 0
        self.misses = 0
        self.pool_bytes = 0
        self.vram = vram_bytes
        self._compiled: dict[str, int] = {}
        self._by_id: dict[int, str] = {}
        self.log: list[tuple] = []       # (name, srv handles, uav handles, groups, cb bytes)
        self.record = False
        self.initialized = False
        # every symbol is a bound method; ctypes-style attribute assignment
        # (`lib.X.argtypes = ...`) must work, so wrap each in a plain function.
        for name in self.SYMBOLS:
            meth = getattr(self, "_" + name)

            def fn(*a, _m=meth):
                return _m(*a)
            fn.__name__ = name
            setattr(self, name, fn)

    SYMBOLS = (
        "InitEngine", "GetGPUInfo", "CompileShader", "CompileShaderEx", "CreateBuffer",
        "AddRefBuffer", "UpdateBuffer", "ReleaseBuffer", "ReleaseBufferBatch", "ReadBuffer",
        "ClearBuffer", "FlushGPU", "SyncGPU", "RunShader", "RunShaderRaw", "RunShaderAlloc",
        "RunShaderAlloc2", "SGDBatch", "SGDBatchClipped", "MatMulAlloc", "ConvForwardFused",
        "ConvBackwardFused", "MaxPoolForwardFused", "MaxPoolBackwardFused", "WarmPool",
        "GetPoolStats", "ResetPoolStats", "GetPoolMemory", "DrainPool", "ResolveShader",
        "RunSequence", "RunSequenceWithSGD",
    )

    # -- device / info -----------------------------------------------------
    def _InitEngine(self):
        self.initialized = True
        return True

    def _GetGPUInfo(self, out):
        a = _addr(out)
        if not a:
            return
        info = GPUInfo.from_address(a)
        info.vendorId = 0x10DE
        info.deviceId = 0
        info.dedicatedVRAM = self.vram
        info.sharedMemory = 0
        info.isIntegrated = 0
        info.description = b"FakeLib (NumPy oracle)"

    def _CompileShader(self, name, path):
        nm = name.decode() if isinstance(name, bytes) else str(name)
        if nm not in self._compiled:
            sid = 0x5000 + len(self._compiled)
            self._compiled[nm] = sid
            self._by_id[sid] = nm
        return True

    def _CompileShaderEx(self, name, path, entry):
        return False          # arbitrary HLSL cannot be executed by this oracle

    # -- buffers -------------------------------------------------------------
    def _max_pool_for_size(self, count):
        """engine.cpp:186-197."""
        b = count * 4
        if self.vram > 0 and b >= self.vram // 4:
            return 4
        if b >= 4 * 1024 * 1024:
            return 6
        if b >= 256 * 1024:
            return 8
        return 16

    def _CreateBuffer(self, data, count):
        count = int(count)
        lst = self._pool.get(count)
        if lst:
            h = lst.pop()
            self.pool_bytes -= count * 4
            self._bufs[h].ref = 1
            self.hits += 1
        else:
            self.misses += 1
            h = self._next
            self._next += 0x10
            self._bufs[h] = _Buf(count)
        a = _addr(data)
        if a:
            self._bufs[h].data[:] = np.ctypeslib.as_array(
                ctypes.cast(a, ctypes.POINTER(ctypes.c_float)), shape=(count,))
        return h

    def buf(self, h) -> np.ndarray:
        return self._bufs[int(h)].data

    def _AddRefBuffer(self, h):
        if h:
            self._bufs[int(h)].ref += 1

    def _UpdateBuffer(self, h, data):
        a = _addr(data)
        if not h or not a:
            return
        b = self._bufs[int(h)]
        b.data[:] = np.ctypeslib.as_array(ctypes.cast(a, ctypes.POINTER(ctypes.c_float)), shape=(b.count,))

    def _release(self, h):
        b = self._bufs[h]
        b.ref -= 1
        if b.ref == 0:
            lst = self._pool.setdefault(b.count, [])
            if len(lst) < self._max_pool_for_size(b.count):
                lst.append(h)
                self.pool_bytes += b.count * 4
            else:
                del self._bufs[h]

    def _ReleaseBuffer(self, h):
        if h:
            self._release(int(h))

    def _ReleaseBufferBatch(self, handles, n):
        for i in range(int(n)):
            if handles[i]:
                self._release(int(handles[i]))

    def _ReadBuffer(self, h, dst):
        a = _addr(dst)
        if not h or not a:
            return
        b = self._bufs[int(h)]
        ctypes.memmove(a, b.data.ctypes.data, b.count * 4)

    def _ClearBuffer(self, h):
        if h:
            self._bufs[int(h)].data[:] = 0

    def _FlushGPU(self):
        return None

    def _SyncGPU(self):
        return None

    # -- dispatch --------------------------------------------------------------
    def _run(self, name, srv_h, uav_h, groups, cb):
        if self.record:
            self.log.append((name, list(srv_h), list(uav_h), tuple(groups), bytes(cb)))
        srvs = [self._bufs[int(h)].data if h else np.zeros(0, F32) for h in srv_h]
        uavs = [self._bufs[int(h)].data if h else np.zeros(0, F32) for h in uav_h]
        shaders.run_shader(name, srvs, uavs, groups, cb)

    def _RunShader(self, name, srvs, nsrv, uavs, nuav, threads, cb, cbsize):
        nm = name.decode() if isinstance(name, bytes) else str(name)
        if nm not in self._compiled:
            return
        cbb = ctypes.string_at(_addr(cb), int(cbsize)) if cb is not None and cbsize else b""
        srv_h = [srvs[i] for i in range(int(nsrv))]
        uav_h = [uavs[i] for i in range(int(nuav))]
        self._run(nm, srv_h, uav_h, [threads[0], threads[1], threads[2]], cbb)

    _RunShaderRaw = _RunShader

    def _RunShaderAlloc(self, name, srvs, nsrv, out_count, threads, cb, cbsize):
        out = self._CreateBuffer(None, out_count)
        arr = (ctypes.c_void_p * 1)(out)
        self._RunShader(name, srvs, nsrv, arr, 1, threads, cb, cbsize)
        return out

    def _RunShaderAlloc2(self, name, srvs, nsrv, out_count, extra, threads, cb, cbsize):
        out = self._CreateBuffer(None, out_count)
        arr = (ctypes.c_void_p * 2)(out, extra)
        self._RunShader(name, srvs, nsrv, arr, 2, threads, cb, cbsize)
        return out

    def _SGDBatch(self, params, grads, sizes, n, lr, clip):
        cb_lr = struct.pack("<Iff", 0, float(lr), float(clip))
        for i in range(int(n)):
            if not params[i] or not grads[i]:
                continue
            cnt = int(sizes[i])
            cb = struct.pack("<I", cnt) + cb_lr[4:] + b"\0\0\0\0"
            self._run("sgd", [grads[i]], [params[i]], ((cnt + 255) // 256, 1, 1), cb)

    def _SGDBatchClipped(self, params, grads, sizes, n, lr, max_norm):
        n = int(n)
        if n == 0:
            return 0.0
        total = sum((int(sizes[i]) + 255) // 256 for i in range(n))
        partials = self._CreateBuffer(None, total)
        ns = self._CreateBuffer(None, 2)
        off = 0
        for i in range(n):
            if not grads[i]:
                continue
            cnt = int(sizes[i])
            k = (cnt + 255) // 256
            self._run("grad_sq_reduce", [grads[i]], [partials], (k, 1, 1), struct.pack("<II", cnt, off))
            off += k
        self._run("grad_norm_final", [partials], [ns], (1, 1, 1),
                  struct.pack("<If", total, float(max_norm)))
        for i in range(n):
            if not params[i] or not grads[i]:
                continue
            cnt = int(sizes[i])
            self._run("sgd_clipped", [grads[i], ns], [params[i]], ((cnt + 255) // 256, 1, 1),
                      struct.pack("<If", cnt, float(lr)))
        norm = float(self._bufs[ns].data[0])
        self._ReleaseBuffer(partials)
        self._ReleaseBuffer(ns)
        return norm

    def _MatMulAlloc(self, a, b, M, K, N, flags):
        """Dense matmul is outside the hot path; restated with NumPy so reference
        scripts that build Linear layers (nn_verify.verify_linear) can run."""
        A = self._bufs[int(a)].data
        Bm = self._bufs[int(b)].data
        M, K, N = int(M), int(K), int(N)
        Am = A[: M * K].reshape(K, M).T if flags & 1 else A[: M * K].reshape(M, K)
        Bx = Bm[: K * N].reshape(N, K).T if flags & 2 else Bm[: K * N].reshape(K, N)
        out = self._CreateBuffer(None, M * N)
        self._bufs[out].data[:] = (Am.astype(np.float64) @ Bx.astype(np.float64)).astype(F32).ravel()
        return out

    def _ConvForwardFused(self, *a):
        return None

    def _ConvBackwardFused(self, *a):
        return None

    def _MaxPoolForwardFused(self, x, batch, inC, inH, inW, pool, stride, p_indices):
        """engine.cpp:880-902: two buffers of batch*inC*outH*outW, then `maxpool_forward`
        with the cbuffer {batch, inC, inH, inW, pool, stride, outH, outW} and
        ((outW+15)/16, (outH+15)/16, batch*inC) groups; *pIndices = the index buffer."""
        m = 0xFFFFFFFF
        batch, inC, inH, inW, pool, stride = (int(v) & m for v in (batch, inC, inH, inW, pool, stride))
        if stride == 0 or pool == 0 or inH < pool or inW < pool:
            return None                      # the reference divides by zero or wraps to a huge size here
        outH = (inH - pool) // stride + 1
        outW = (inW - pool) // stride + 1
        n = batch * inC * outH * outW
        out = self._CreateBuffer(None, n)
        idx = self._CreateBuffer(None, n)
        if not out or not idx:
            return None
        cb = struct.pack("<8I", batch, inC, inH, inW, pool, stride, outH, outW)
        self._run("maxpool_forward", [x], [out, idx], ((outW + 15) // 16, (outH + 15) // 16, batch * inC), cb)
        if p_indices:
            _set_out_ptr(p_indices, idx)
        return out

    def _MaxPoolBackwardFused(self, grad_out, indices, batch, inC, outH, outW, x_size):
        """engine.cpp:905-929: a zeroed buffer of x_size, `maxpool_backward` with
        {batch, inC, outH, outW} and ((outW+15)/16, (outH+15)/16, batch*inC) groups,
        then the index buffer is released."""
        batch, inC, outH, outW, x_size = (int(v) for v in (batch, inC, outH, outW, x_size))
        d = self._CreateBuffer(None, x_size)
        if not d:
            return None
        self._bufs[d].data[:] = 0
        cb = struct.pack("<4I", batch, inC, outH, outW)
        self._run("maxpool_backward", [grad_out, indices], [d], ((outW + 15) // 16, (outH + 15) // 16, batch * inC), cb)
        self._ReleaseBuffer(indices)
        return d

    # -- pool --------------------------------------------------------------------
    def _WarmPool(self, sizes, n, copies):
        for i in range(int(n)):
            cnt = int(sizes[i])
            lst = self._pool.setdefault(cnt, [])
            target = min(int(copies), self._max_pool_for_size(cnt))
            for _ in range(max(0, target - len(lst))):
                h = self._CreateBuffer(None, cnt)
                self._release(h)
                if self.misses > 0:
                    self.misses -= 1

    def _GetPoolStats(self, hits, misses):
        if hits is not None:
            ctypes.c_uint64.from_address(_addr(hits)).value = self.hits
        if misses is not None:
            ctypes.c_uint64.from_address(_addr(misses)).value = self.misses

    def _ResetPoolStats(self):
        self.hits = 0
        self.misses = 0

    def _GetPoolMemory(self):
        return self.pool_bytes

    def _DrainPool(self):
        for lst in self._pool.values():
            for h in lst:
                del self._bufs[h]
        self._pool.clear()
        self.pool_bytes = 0

    # -- graph replay ------------------------------------------------------------
    def _ResolveShader(self, name):
        nm = name.decode() if isinstance(name, bytes) else str(name)
        return self._compiled.get(nm)

    def _RunSequence(self, cmds, count):
        base = _addr(cmds)
        if not base:
            return
        for i in range(int(count)):
            c = SeqCmd.from_address(base + i * ctypes.sizeof(SeqCmd))
            if not c.shader:
                continue
            nm = self._by_id.get(int(c.shader))
            if nm is None:
                continue
            cb = bytes(c.cbData[: c.cbSize]) if c.cbSize else b""
            self._run(nm, [c.srvs[j] for j in range(c.srvCount)],
                      [c.uavs[j] for j in range(c.uavCount)],
                      [c.threads[0], c.threads[1], c.threads[2]], cb)

    def _RunSequenceWithSGD(self, cmds, count, params, grads, sizes, n, lr, clip):
        self._RunSequence(cmds, count)
        self._SGDBatch(params, grads, sizes, n, lr, clip)


#: the 15 shader names nn_engine.py compiles whose .hlsl is absent from the
#: reference snapshot (nn_engine.py:156-164); `_find_resource` needs a file.
MISSING_HLSL = (
    "gelu", "gelu_grad", "layernorm_forward", "causal_masked_softmax", "attention_forward",
    "layernorm_backward_param", "layernorm_backward_dx", "attention_forward_train",
    "attention_backward_dq", "attention_backward_dk", "attention_backward_dv",
    "attention_forward_full_train", "attention_backward_full_dq",
    "attention_backward_full_dk", "attention_backward_full_dv",
)


@contextlib.contextmanager
def _placeholder_cwd():
    old = os.getcwd()
    with tempfile.TemporaryDirectory(prefix="dct_ref_") as d:
        open(os.path.join(d, "engine.dll"), "wb").close()
        for n in MISSING_HLSL:
            open(os.path.join(d, f"nn_{n}.hlsl"), "w").close()
        os.chdir(d)
        try:
            yield d
        finally:
            os.chdir(old)


def load_reference_engine(ref_dir: str, lib):
    """Import the unmodified reference `nn_engine.py` bound to `lib`.

    `lib` is a FakeLib, or a real `ctypes.CDLL` of `libdct_cuda.so`.  The
    reference module is imported fresh (any previous copy is dropped).
    """
    for m in ("nn_engine", "nn_verify"):
        sys.modules.pop(m, None)
    orig = ctypes.CDLL

    def cdll(path, *a, **k):
        if str(path).endswith("engine.dll"):
            return lib
        return orig(path, *a, **k)

    if ref_dir not in sys.path:
        sys.path.insert(0, ref_dir)
    ctypes.CDLL = cdll
    try:
        with _placeholder_cwd(), contextlib.redirect_stdout(open(os.devnull, "w")):
            mod = importlib.import_module("nn_engine")
    finally:
        ctypes.CDLL = orig
    return mod
