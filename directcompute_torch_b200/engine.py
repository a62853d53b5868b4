"""The reference's Python API for the hot path, bound to libdct_cuda.so.

Mirrors the parts of raviadi12/directcompute_torch `nn_engine.py` that dispatch
the elementwise / reduction / softmax-CE / optimizer / normalization kernels:
same names, same argument meaning, same C-ABI calls with the same cbuffer
words and group counts -- so code written against the reference runs here
unchanged, and the parity tests read like the reference's own.

  ctypes binding + dispatch          nn_engine.py:41-181, 452-484
  Tensor + tape autograd             nn_engine.py:486-614
  elementwise Functions              nn_engine.py:1062-1199, 1369-1399
  softmax + CE, dice loss            nn_engine.py:1268-1317
  global average pool                nn_engine.py:1466-1490
  MaxPool2D, UpSample2D, Concat      nn_engine.py:1018-1047, 1196-1266, 1328-1332
  rms, clip_grad_norm, sgd clipped   nn_engine.py:1335-1367, 1685-1692
  BatchNorm2d                        nn_engine.py:1794-1871, 1904-1916
  SGD, AdamW, Adam                   nn_engine.py:2172-2242
  Metrics, end_batch, pool helpers   nn_engine.py:2322-2475
  ComputeGraph record / replay       nn_engine.py:2490-2771

Dense matmul, convolution and custom-HLSL entry points are outside this
library (the C symbols exist and report DCT_ERR_UNSUPPORTED).
"""
from __future__ import annotations

import ctypes
import struct

import numpy as np

from . import load_library
from ._abi import GPUInfo, SeqCmd

# ---------------------------------------------------------------------------
# library + device (nn_engine.py:41-173)
# ---------------------------------------------------------------------------
lib = load_library()
if not lib.InitEngine():
    raise RuntimeError("libdct_cuda: InitEngine failed: " + (lib.dct_last_error() or b"").decode())

_gpu_info = GPUInfo()
lib.GetGPUInfo(ctypes.byref(_gpu_info))
GPU_NAME = _gpu_info.description.decode("ascii", errors="replace").strip("\x00")
VRAM_BYTES = int(_gpu_info.dedicatedVRAM)

#: kernel names this library implements (the reference compiles these from nn_<name>.hlsl)
SHADERS = (
    "add_bias", "bias_relu", "relu", "relu_grad", "relu6", "relu6_grad", "leaky_relu",
    "leaky_relu_grad", "sigmoid", "sigmoid_grad", "add", "scale_add", "grad_accum", "bias_grad",
    "global_avg_pool", "global_avg_pool_backward", "softmax", "loss", "softmax_ce_grad",
    "argmax_correct", "accumulate_scalar", "rms", "grad_sq_reduce", "grad_norm_final", "sgd",
    "sgd_clipped", "adam", "batchnorm_mean_var", "batchnorm_forward", "batchnorm_backward_reduce",
    "batchnorm_backward_dx", "dice_loss", "dice_loss_sums", "dice_loss_grad",
    "upsample", "upsample_backward", "concat_insert", "slice", "maxpool_forward", "maxpool_backward",
    "conv_reshape", "conv_grad_reshape", "conv_grad_reshape_relu",
)
for _s in SHADERS:
    lib.CompileShader(_s.encode(), "")


def float_to_uint(f):
    """nn_engine.py:10-11: the f32 bit pattern of a Python float."""
    return struct.unpack("I", struct.pack("f", f))[0]


class ParamsCB(ctypes.Structure):
    """nn_engine.py:175-178: nine u32 cbuffer words."""
    _fields_ = [(f"u{i}", ctypes.c_uint) for i in range(1, 10)]


class SGDParamsCB(ctypes.Structure):
    """nn_engine.py:180-181."""
    _fields_ = [("count", ctypes.c_uint), ("lr", ctypes.c_float), ("clip", ctypes.c_float), ("pad", ctypes.c_uint)]


# pre-allocated dispatch arrays, as nn_engine.py:452-456
_srv_arr = (ctypes.c_void_p * 8)()
_uav_arr = (ctypes.c_void_p * 8)()
_threads = (ctypes.c_uint * 3)()
_cb = ParamsCB()


def _fill(srvs, uavs, tx, ty, tz, words, cbSize):
    for i, h in enumerate(srvs):
        _srv_arr[i] = h
    for i, h in enumerate(uavs):
        _uav_arr[i] = h
    _threads[0], _threads[1], _threads[2] = tx, ty, tz
    for i, w in enumerate(words):
        setattr(_cb, f"u{i + 1}", w)
    return (ctypes.byref(_cb), cbSize) if cbSize > 0 else (None, 0)


def _dispatch(name, srvs, uavs, tx, ty, tz, u1=0, u2=0, u3=0, u4=0, u5=0, u6=0, u7=0, u8=0, u9=0, cbSize=16):
    """nn_engine.py:458-470: RunShader with up to nine cbuffer words."""
    cb, n = _fill(srvs, uavs, tx, ty, tz, (u1, u2, u3, u4, u5, u6, u7, u8, u9), cbSize)
    lib.RunShader(name, _srv_arr, len(srvs), _uav_arr, len(uavs), _threads, cb, n)


def _dispatch_raw(name, srvs, uavs, tx, ty, tz, u1=0, u2=0, u3=0, u4=0, u5=0, u6=0, u7=0, u8=0, u9=0, cbSize=16):
    """nn_engine.py:472-484 (RunShaderRaw is the same entry point)."""
    cb, n = _fill(srvs, uavs, tx, ty, tz, (u1, u2, u3, u4, u5, u6, u7, u8, u9), cbSize)
    lib.RunShaderRaw(name, _srv_arr, len(srvs), _uav_arr, len(uavs), _threads, cb, n)


def _groups(n, per=256):
    return (n + per - 1) // per


# ---------------------------------------------------------------------------
# Tensor + autograd (nn_engine.py:486-614)
# ---------------------------------------------------------------------------
_all_tensors = []


def release_all_buffers():
    """nn_engine.py:488-508: drop the batch's graph and return tracked buffers in one call."""
    global _all_tensors
    handles = []
    for t in _all_tensors:
        if t._ctx:
            t._ctx.inputs = ()
            t._ctx = None
        t.grad = None
        if t.gpu_buf:
            handles.append(t.gpu_buf)
            t.gpu_buf = None
    _all_tensors = []
    if handles:
        lib.ReleaseBufferBatch((ctypes.c_void_p * len(handles))(*handles), len(handles))


def _shape_size(shape):
    n = 1
    for d in shape:
        n *= d
    return n


def _fptr(a):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


class Tensor:
    """fp32 device tensor backed by a libdct_cuda buffer handle (nn_engine.py:517-610)."""
    __slots__ = ["data", "shape", "size", "requires_grad", "grad", "gpu_buf", "_ctx", "_cached_topo"]

    def __init__(self, data, requires_grad=False, track=True):
        arr = data if isinstance(data, np.ndarray) else np.array(data, dtype=np.float32)
        if arr.dtype != np.float32:
            arr = arr.astype(np.float32)
        arr = np.ascontiguousarray(arr)
        self.data = arr
        self.shape = arr.shape
        self.size = arr.size
        self.requires_grad = requires_grad
        self.grad = None
        self.gpu_buf = lib.CreateBuffer(_fptr(arr), self.size)
        self._ctx = None
        if track:
            _all_tensors.append(self)

    def __del__(self):
        if getattr(self, "gpu_buf", None):
            lib.ReleaseBuffer(self.gpu_buf)
            self.gpu_buf = None

    @classmethod
    def from_gpu(cls, handle, shape, requires_grad=False, track=True):
        t = object.__new__(cls)
        t.data = None
        t.shape = tuple(shape)
        t.size = _shape_size(shape)
        t.requires_grad = requires_grad
        t.grad = None
        t.gpu_buf = handle
        t._ctx = None
        if track:
            _all_tensors.append(t)
        return t

    @classmethod
    def empty(cls, shape, requires_grad=False, track=True):
        return cls(np.empty(shape, dtype=np.float32), requires_grad=requires_grad, track=track)

    @classmethod
    def empty_like(cls, other, requires_grad=None, track=True):
        req = other.requires_grad if requires_grad is None else bool(requires_grad)
        return cls.empty(other.shape, requires_grad=req, track=track)

    def sync(self):
        """Blocking read of the device buffer into `.data`."""
        if self.gpu_buf:
            if self.data is None or self.data.shape != tuple(self.shape):
                self.data = np.empty(self.shape, dtype=np.float32)
            lib.ReadBuffer(self.gpu_buf, _fptr(self.data))
        return self.data

    def upload(self, data):
        """Upload new contents into the existing buffer."""
        if data.dtype != np.float32:
            data = data.astype(np.float32)
        data = np.ascontiguousarray(data)
        self.data = data
        self.shape = data.shape
        self.size = data.size
        lib.UpdateBuffer(self.gpu_buf, _fptr(data))

    def backward(self, grad=None):
        """Reverse replay of the tape from this tensor (topological order cached)."""
        if grad is None:
            grad = Tensor(np.ones(self.shape, dtype=np.float32), track=False)
        self.grad = grad
        if not hasattr(self, "_cached_topo"):
            order, seen, stack = [], set(), [self]
            while stack:
                v = stack[-1]
                if v in seen:
                    stack.pop()
                    continue
                pending = False
                if v._ctx:
                    for i in v._ctx.inputs:
                        if isinstance(i, Tensor) and i.requires_grad and i not in seen:
                            stack.append(i)
                            pending = True
                if not pending:
                    seen.add(v)
                    stack.pop()
                    order.append(v)
            self._cached_topo = order
        for v in reversed(self._cached_topo):
            if v._ctx and v.grad is not None:
                v._ctx.backward(v.grad)

    def _accumulate_grad(self, grad):
        """First gradient is aliased; later ones are added in place by `grad_accum`."""
        if self.grad is None or self.grad.gpu_buf is None:
            self.grad = grad
        else:
            _dispatch(b"grad_accum", (grad.gpu_buf,), (self.grad.gpu_buf,), _groups(self.size), 1, 1, u1=self.size)


class Function:
    def __init__(self, *inputs):
        self.inputs = inputs

    def backward(self, grad_output):
        raise NotImplementedError


def _new(size):
    return lib.CreateBuffer(None, size)


def _out(handle, shape, ctx, requires_grad):
    res = Tensor.from_gpu(handle, shape, requires_grad=requires_grad)
    res._ctx = ctx
    return res


# ---------------------------------------------------------------------------
# elementwise Functions (nn_engine.py:1062-1199, 1369-1399)
# ---------------------------------------------------------------------------
def _bias_grad(g, B):
    """dB = sum over rows of g (nn_engine.py:1076-1077)."""
    h = _new(B.size)
    _dispatch(b"bias_grad", (g.gpu_buf,), (h,), B.size, 1, 1, u1=g.shape[0], u2=B.size, u3=B.size, u4=1)
    return Tensor.from_gpu(h, B.shape, track=True)


class AddBias(Function):
    def forward(self, A, B):
        self.inputs = (A, B)
        h = _new(A.size)
        _dispatch(b"add_bias", (A.gpu_buf, B.gpu_buf), (h,), _groups(A.size), 1, 1, u1=A.shape[0], u2=A.shape[1])
        return _out(h, A.shape, self, A.requires_grad or B.requires_grad)

    def backward(self, grad_output):
        A, B = self.inputs
        if A.requires_grad:
            A._accumulate_grad(grad_output)
        if B.requires_grad:
            B._accumulate_grad(_bias_grad(grad_output, B))


class BiasReLUFunc(Function):
    def forward(self, A, B):
        self.inputs = (A, B)
        h = _new(A.size)
        _dispatch(b"bias_relu", (A.gpu_buf, B.gpu_buf), (h,), _groups(A.size), 1, 1, u1=A.shape[0], u2=A.shape[1])
        res = _out(h, A.shape, self, A.requires_grad or B.requires_grad)
        self.output = res
        return res

    def backward(self, grad_output):
        A, B = self.inputs
        h = _new(grad_output.size)
        _dispatch(b"relu_grad", (grad_output.gpu_buf, self.output.gpu_buf), (h,), _groups(grad_output.size), 1, 1,
                  u1=grad_output.size)
        eff = Tensor.from_gpu(h, grad_output.shape, track=True)
        self.output = None
        if A.requires_grad:
            A._accumulate_grad(eff)
        if B.requires_grad:
            B._accumulate_grad(_bias_grad(eff, B))


class _Unary(Function):
    """Pointwise op with a saved-tensor backward kernel."""
    fwd = bwd = None
    save_output = False

    def words(self, n):
        return dict(u1=n)

    def forward(self, x):
        self.inputs = (x,)
        h = _new(x.size)
        kw = self.words(x.size)
        if kw is None:
            _dispatch(self.fwd, (x.gpu_buf,), (h,), _groups(x.size), 1, 1, cbSize=0)
        else:
            _dispatch(self.fwd, (x.gpu_buf,), (h,), _groups(x.size), 1, 1, **kw)
        res = _out(h, x.shape, self, x.requires_grad)
        if self.save_output:
            self.out_tensor = res
        return res

    def backward(self, grad_output):
        x = self.inputs[0]
        if x.requires_grad:
            saved = self.out_tensor if self.save_output else x
            h = _new(x.size)
            kw = self.words(x.size) or {}
            kw["u1"] = x.size
            _dispatch(self.bwd, (grad_output.gpu_buf, saved.gpu_buf), (h,), _groups(x.size), 1, 1, **kw)
            x._accumulate_grad(Tensor.from_gpu(h, x.shape, track=True))


class ReLUFunc(_Unary):
    fwd, bwd = b"relu", b"relu_grad"

    def words(self, n):
        return None                     # nn_relu.hlsl has no cbuffer (nn_engine.py:1112-1113)


class ReLU6Func(_Unary):
    fwd, bwd = b"relu6", b"relu6_grad"


class SigmoidFunc(_Unary):
    fwd, bwd, save_output = b"sigmoid", b"sigmoid_grad", True


class LeakyReLUFunc(_Unary):
    fwd, bwd = b"leaky_relu", b"leaky_relu_grad"

    def forward(self, x, alpha=0.1):
        self.alpha = alpha
        return super().forward(x)

    def words(self, n):
        return dict(u1=n, u2=float_to_uint(self.alpha))


class AddFunc(Function):
    """Same-shape add; backward aliases the upstream gradient (nn_engine.py:1379-1397)."""
    def forward(self, A, B):
        self.inputs = (A, B)
        h = _new(A.size)
        _dispatch(b"add", (A.gpu_buf, B.gpu_buf), (h,), _groups(A.size), 1, 1, u1=A.size, u2=1)
        return _out(h, A.shape, self, A.requires_grad or B.requires_grad)

    def backward(self, grad_output):
        for t in self.inputs:
            if t.requires_grad:
                lib.AddRefBuffer(grad_output.gpu_buf)
                t._accumulate_grad(Tensor.from_gpu(grad_output.gpu_buf, t.shape, track=False))


def scale_add(A, B, alpha=1.0, beta=1.0):
    """alpha*A + beta*B (nn_engine.py:1369-1375)."""
    h = _new(A.size)
    _dispatch(b"scale_add", (A.gpu_buf, B.gpu_buf), (h,), _groups(A.size), 1, 1,
              u1=A.size, u2=float_to_uint(alpha), u3=float_to_uint(beta), cbSize=16)
    return Tensor.from_gpu(h, A.shape, track=True)


# ---------------------------------------------------------------------------
# softmax + cross-entropy, dice (nn_engine.py:1268-1317)
# ---------------------------------------------------------------------------
class SoftmaxCEFunc(Function):
    def forward(self, x, labels):
        self.inputs = (x, labels)
        B, K = x.shape
        ph = _new(x.size)
        _dispatch(b"softmax", (x.gpu_buf,), (ph,), _groups(B, 16), 1, 1, u1=B, u2=K)
        self.softmax_out = Tensor.from_gpu(ph, x.shape)
        lh = _new(1)
        _dispatch(b"loss", (x.gpu_buf, labels.gpu_buf), (lh,), 1, 1, 1, u1=B, u2=K)
        return _out(lh, (1,), self, True)

    def backward(self, grad_output):
        x, labels = self.inputs
        B, K = x.shape
        h = _new(x.size)
        _dispatch(b"softmax_ce_grad", (self.softmax_out.gpu_buf, labels.gpu_buf), (h,),
                  _groups(K, 16), _groups(B, 16), 1, u1=B, u2=K)
        x._accumulate_grad(Tensor.from_gpu(h, x.shape, track=True))


class DiceLossFunc(Function):
    def forward(self, pred, target):
        self.inputs = (pred, target)
        b = pred.shape[0]
        size = pred.size // b
        h = _new(b)
        _dispatch(b"dice_loss", (pred.gpu_buf, target.gpu_buf), (h,), b, 1, 1, u1=b, u2=size)
        return _out(h, (b,), self, True)

    def backward(self, grad_output):
        pred, target = self.inputs
        b = pred.shape[0]
        size = pred.size // b
        sums = _new(b * 3)
        _dispatch(b"dice_loss_sums", (pred.gpu_buf, target.gpu_buf), (sums,), b, 1, 1, u1=b, u2=size)
        h = _new(pred.size)
        _dispatch(b"dice_loss_grad", (pred.gpu_buf, target.gpu_buf, sums), (h,), _groups(pred.size), 1, 1,
                  u1=b, u2=size)
        lib.ReleaseBuffer(sums)
        pred._accumulate_grad(Tensor.from_gpu(h, pred.shape, track=True))


class GlobalAvgPool2DFunc(Function):
    """Mean over H*W (nn_engine.py:1466-1488)."""
    def forward(self, x):
        self.inputs = (x,)
        n, c, hh, ww = x.shape
        self.S = hh * ww
        h = _new(n * c)
        _dispatch(b"global_avg_pool", (x.gpu_buf,), (h,), n * c, 1, 1, u1=n, u2=c, u3=self.S)
        return _out(h, (n, c), self, x.requires_grad)

    def backward(self, grad_output):
        x = self.inputs[0]
        if x.requires_grad:
            n, c = grad_output.shape
            h = _new(x.size)
            _dispatch(b"global_avg_pool_backward", (grad_output.gpu_buf,), (h,), _groups(x.size), 1, 1,
                      u1=n, u2=c, u3=self.S)
            x._accumulate_grad(Tensor.from_gpu(h, x.shape, track=True))


# ---------------------------------------------------------------------------
# layout Functions: max pooling, nearest upsample, channel concat
# (nn_engine.py:1018-1047, 1196-1266)
# ---------------------------------------------------------------------------
class MaxPool2D(Function):
    """Window max with its flat index kept on the device (MaxPoolForwardFused);
    the backward call consumes and releases the index buffer."""
    def __del__(self):
        h = getattr(self, "indices_handle", None)
        if h:
            lib.ReleaseBuffer(h)
            self.indices_handle = None

    def forward(self, x, pool_size=2, stride=2):
        self.inputs = (x,)
        batch, inC, inH, inW = x.shape
        outH = (inH - pool_size) // stride + 1
        outW = (inW - pool_size) // stride + 1
        p_idx = ctypes.c_void_p()
        h = lib.MaxPoolForwardFused(x.gpu_buf, batch, inC, inH, inW, pool_size, stride, ctypes.byref(p_idx))
        self.indices_handle = p_idx.value
        return _out(h, (batch, inC, outH, outW), self, x.requires_grad)

    def backward(self, grad_output):
        x = self.inputs[0]
        batch, inC, outH, outW = grad_output.shape
        d = lib.MaxPoolBackwardFused(grad_output.gpu_buf, self.indices_handle, batch, inC, outH, outW, x.size)
        self.indices_handle = None                      # released by MaxPoolBackwardFused
        x._accumulate_grad(Tensor.from_gpu(d, x.shape, track=True))


class UpSample2D(Function):
    """Nearest-neighbour upsample by integer factors."""
    def forward(self, x, scaleH=2, scaleW=2):
        self.inputs = (x,)
        self.scaleH, self.scaleW = scaleH, scaleW
        batch, C, inH, inW = x.shape
        outH, outW = inH * scaleH, inW * scaleW
        n = batch * C * outH * outW
        h = _new(n)
        _dispatch(b"upsample", (x.gpu_buf,), (h,), _groups(n), 1, 1,
                  u1=batch, u2=C, u3=inH, u4=inW, u5=outH, u6=outW, u7=scaleH, u8=scaleW, cbSize=32)
        return _out(h, (batch, C, outH, outW), self, x.requires_grad)

    def backward(self, grad_output):
        x = self.inputs[0]
        if x.requires_grad:
            batch, C, inH, inW = x.shape
            h = _new(x.size)
            _dispatch(b"upsample_backward", (grad_output.gpu_buf,), (h,), _groups(x.size), 1, 1,
                      u1=batch, u2=C, u3=inH, u4=inW, u5=inH * self.scaleH, u6=inW * self.scaleW,
                      u7=self.scaleH, u8=self.scaleW, cbSize=32)
            x._accumulate_grad(Tensor.from_gpu(h, x.shape, track=True))


class Concat(Function):
    """Concatenation along channels (axis 1) of NCHW tensors."""
    def forward(self, tensors, axis=1):
        if axis != 1:
            raise NotImplementedError("Concat currently only supported along channel dimension (axis 1)")
        self.inputs = tuple(tensors)
        batch, _, H, W = tensors[0].shape
        spatial = H * W
        total_C = sum(t.shape[1] for t in tensors)
        h = _new(batch * total_C * spatial)
        self.c_offsets = []
        c_off = 0
        for t in tensors:
            self.c_offsets.append(c_off)
            c_in = t.shape[1]
            _dispatch(b"concat_insert", (t.gpu_buf,), (h,), _groups(batch * c_in * spatial), 1, 1,
                      u1=batch, u2=c_in, u3=spatial, u4=total_C, u5=c_off, cbSize=20)
            c_off += c_in
        return _out(h, (batch, total_C, H, W), self, any(t.requires_grad for t in tensors))

    def backward(self, grad_output):
        batch, total_C, H, W = grad_output.shape
        spatial = H * W
        for t, c_off in zip(self.inputs, self.c_offsets):
            if t.requires_grad:
                c_in = t.shape[1]
                n = batch * c_in * spatial
                h = _new(n)
                _dispatch(b"slice", (grad_output.gpu_buf,), (h,), _groups(n), 1, 1,
                          u1=batch, u2=c_in, u3=spatial, u4=total_C, u5=c_off, cbSize=20)
                t._accumulate_grad(Tensor.from_gpu(h, t.shape, track=True))


def maxpool2d(x, pool_size=2, stride=2): return MaxPool2D().forward(x, pool_size, stride)
def upsample2d(x, scaleH=2, scaleW=2): return UpSample2D().forward(x, scaleH, scaleW)
def concat(tensors, axis=1): return Concat().forward(tensors, axis)


def add_bias(A, B): return AddBias().forward(A, B)
def bias_relu(A, B): return BiasReLUFunc().forward(A, B)
def relu(x): return ReLUFunc().forward(x)
def relu6(x): return ReLU6Func().forward(x)
def sigmoid(x): return SigmoidFunc().forward(x)
def leaky_relu(x, alpha=0.1): return LeakyReLUFunc().forward(x, alpha)
def softmax_ce(x, labels): return SoftmaxCEFunc().forward(x, labels)
def dice_loss(pred, target): return DiceLossFunc().forward(pred, target)
def add(A, B): return AddFunc().forward(A, B)
def global_avg_pool2d(x): return GlobalAvgPool2DFunc().forward(x)


def rms(A):
    """sqrt(mean(A^2)) read back to the host, floored at 1e-8 (nn_engine.py:1685-1692)."""
    h = _new(1)
    _dispatch(b"rms", (A.gpu_buf,), (h,), 1, 1, 1, u1=A.size, cbSize=16)
    v = np.empty(1, dtype=np.float32)
    lib.ReadBuffer(h, _fptr(v))
    lib.ReleaseBuffer(h)
    return max(float(v[0]), 1e-8)


def clip_grad_norm(params, max_norm=1.0):
    """Host-side clip of nn_engine.py:1335-1355 (reads the grads, rescales, uploads)."""
    total = 0.0
    grads = []
    for p in params:
        if p.grad is not None and p.grad.gpu_buf is not None:
            g = p.grad.sync()
            grads.append(g)
            total += float(np.sum(g * g))
        else:
            grads.append(None)
    norm = float(np.sqrt(total))
    if norm > max_norm:
        scale = max_norm / (norm + 1e-6)
        for p, g in zip(params, grads):
            if g is not None:
                p.grad.upload(g * scale)
    return norm


def sgd_step_clipped(params, lr, max_norm=1.0):
    """Device-side clip + SGD; returns the global grad norm (nn_engine.py:1357-1367)."""
    n = len(params)
    pa = (ctypes.c_void_p * n)(*[p.gpu_buf for p in params])
    ga = (ctypes.c_void_p * n)(*[p.grad.gpu_buf for p in params])
    sa = (ctypes.c_uint * n)(*[p.size for p in params])
    return float(lib.SGDBatchClipped(pa, ga, sa, n, lr, max_norm))


# ---------------------------------------------------------------------------
# BatchNorm2d (nn_engine.py:1794-1871, 1904-1916)
# ---------------------------------------------------------------------------
class BatchNorm2dFunc(Function):
    def forward(self, x, gamma, beta, running_mean, running_var, eps=1e-5, momentum=0.1, training=True):
        self.inputs = (x, gamma, beta)
        self.batch, self.channels, hh, ww = x.shape
        self.S = hh * ww
        self.eps = eps
        if training:
            self.batch_mean_handle = _new(self.channels)
            self.batch_var_handle = _new(self.channels)
            _dispatch(b"batchnorm_mean_var", (x.gpu_buf,),
                      (self.batch_mean_handle, self.batch_var_handle, running_mean.gpu_buf, running_var.gpu_buf),
                      self.channels, 1, 1, u1=self.batch, u2=self.channels, u3=self.S, u4=int(training),
                      u5=float_to_uint(momentum), cbSize=20)
            mean_buf, var_buf = self.batch_mean_handle, self.batch_var_handle
        else:
            mean_buf, var_buf = running_mean.gpu_buf, running_var.gpu_buf
            self.batch_mean_handle = self.batch_var_handle = None
        h = _new(x.size)
        _dispatch(b"batchnorm_forward", (x.gpu_buf, mean_buf, var_buf, gamma.gpu_buf, beta.gpu_buf), (h,),
                  _groups(x.size), 1, 1, u1=self.batch, u2=self.channels, u3=self.S, u4=float_to_uint(eps), cbSize=16)
        return _out(h, x.shape, self, x.requires_grad or gamma.requires_grad or beta.requires_grad)

    def backward(self, grad_output):
        x, gamma, beta = self.inputs
        if self.batch_mean_handle is None:
            raise RuntimeError("BatchNorm backward requires training=True during forward")
        dg = _new(self.channels)
        db = _new(self.channels)
        words = dict(u1=self.batch, u2=self.channels, u3=self.S, u4=float_to_uint(self.eps))
        _dispatch(b"batchnorm_backward_reduce",
                  (x.gpu_buf, grad_output.gpu_buf, self.batch_mean_handle, self.batch_var_handle), (dg, db),
                  self.channels, 1, 1, **words)
        dx = _new(x.size)
        _dispatch(b"batchnorm_backward_dx",
                  (x.gpu_buf, grad_output.gpu_buf, self.batch_mean_handle, self.batch_var_handle, gamma.gpu_buf,
                   dg, db), (dx,), _groups(x.size), 1, 1, **words)
        for t, h in ((gamma, dg), (beta, db), (x, dx)):
            if t.requires_grad:
                t._accumulate_grad(Tensor.from_gpu(h, t.shape, track=True))
            else:
                lib.ReleaseBuffer(h)
        lib.ReleaseBuffer(self.batch_mean_handle)
        lib.ReleaseBuffer(self.batch_var_handle)


def batchnorm2d(x, gamma, beta, rm, rv, eps=1e-5, momentum=0.1, training=True):
    return BatchNorm2dFunc().forward(x, gamma, beta, rm, rv, eps, momentum, training)


class BatchNorm2d:
    def __init__(self, num_features, eps=1e-5, momentum=0.1):
        self.num_features = num_features
        self.eps = eps
        self.momentum = momentum
        self.gamma = Tensor(np.ones(num_features, dtype=np.float32), requires_grad=True, track=False)
        self.beta = Tensor(np.zeros(num_features, dtype=np.float32), requires_grad=True, track=False)
        self.running_mean = Tensor(np.zeros(num_features, dtype=np.float32), track=False)
        self.running_var = Tensor(np.ones(num_features, dtype=np.float32), track=False)
        self.training = True

    def __call__(self, x):
        return batchnorm2d(x, self.gamma, self.beta, self.running_mean, self.running_var, self.eps, self.momentum,
                           self.training)


# ---------------------------------------------------------------------------
# optimizers (nn_engine.py:2172-2242)
# ---------------------------------------------------------------------------
class SGD:
    def __init__(self, params, lr):
        self.params = params
        self.lr = lr
        n = len(params)
        self._p = (ctypes.c_void_p * n)()
        self._g = (ctypes.c_void_p * n)()
        self._s = (ctypes.c_uint * n)()

    def zero_grad(self):
        for p in self.params:
            if p.grad:
                p.grad = None

    def step(self, clip=1.0):
        n = 0
        for p in self.params:
            if p.grad:
                self._p[n], self._g[n], self._s[n] = p.gpu_buf, p.grad.gpu_buf, p.size
                n += 1
        if n:
            lib.SGDBatch(self._p, self._g, self._s, n, self.lr, clip)


class AdamW:
    def __init__(self, params, lr=0.001, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01):
        self.params = params
        self.lr = lr
        self.beta1, self.beta2 = betas
        self.eps = eps
        self.weight_decay = weight_decay
        self.t = 0
        self.m = [Tensor(np.zeros(p.shape), track=False) for p in params]
        self.v = [Tensor(np.zeros(p.shape), track=False) for p in params]
        self._m_bufs = [x.gpu_buf for x in self.m]
        self._v_bufs = [x.gpu_buf for x in self.v]

    def zero_grad(self):
        for p in self.params:
            if p.grad:
                p.grad = None

    def step(self, clip=1.0):
        """One `adam` dispatch per parameter, bias correction folded into the step size."""
        self.t += 1
        step = self.lr * (1 - self.beta2 ** self.t) ** 0.5 / (1 - self.beta1 ** self.t)
        for i, p in enumerate(self.params):
            if not p.grad:
                continue
            _dispatch_raw(b"adam", (p.grad.gpu_buf,), (p.gpu_buf, self._m_bufs[i], self._v_bufs[i]),
                          _groups(p.size), 1, 1, u1=p.size, u2=float_to_uint(step), u3=float_to_uint(self.beta1),
                          u4=float_to_uint(self.beta2), u5=float_to_uint(self.eps),
                          u6=float_to_uint(self.lr * self.weight_decay), u7=float_to_uint(clip), cbSize=32)


class Adam(AdamW):
    def __init__(self, params, lr=0.001, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.0):
        super().__init__(params, lr, betas, eps, weight_decay=weight_decay)


# ---------------------------------------------------------------------------
# metrics, batch end, pool (nn_engine.py:2322-2475)
# ---------------------------------------------------------------------------
def gpu_argmax_correct(logits, labels, correct_buf):
    B, K = logits.shape
    _dispatch_raw(b"argmax_correct", (logits.gpu_buf, labels.gpu_buf), (correct_buf,), _groups(B), 1, 1, u1=B, u2=K)


def gpu_accumulate_loss(loss_tensor, accum_buf):
    _dispatch(b"accumulate_scalar", (loss_tensor.gpu_buf,), (accum_buf,), 1, 1, 1, cbSize=0)


class Metrics:
    """Device-side loss sum and correct count, read once per collect()."""
    def __init__(self):
        self._correct_buf = _new(1)
        self._loss_buf = _new(1)
        self._f1 = np.empty(1, dtype=np.float32)
        self._n_batches = 0
        self.reset()

    def reset(self):
        lib.ClearBuffer(self._correct_buf)
        lib.ClearBuffer(self._loss_buf)
        self._n_batches = 0

    def update(self, loss, logits, labels):
        gpu_accumulate_loss(loss, self._loss_buf)
        gpu_argmax_correct(logits, labels, self._correct_buf)
        self._n_batches += 1

    def collect(self, num_samples):
        lib.ReadBuffer(self._loss_buf, _fptr(self._f1))
        avg = float(self._f1[0]) / self._n_batches if self._n_batches else 0.0
        lib.ReadBuffer(self._correct_buf, _fptr(self._f1))
        correct = int(self._f1.view(np.uint32)[0])
        return avg, (correct / num_samples if num_samples else 0.0)

    def __del__(self):
        if getattr(self, "_correct_buf", None):
            lib.ReleaseBuffer(self._correct_buf)
        if getattr(self, "_loss_buf", None):
            lib.ReleaseBuffer(self._loss_buf)


def end_batch():
    release_all_buffers()
    end_batch._count += 1
    if end_batch._count % end_batch.flush_interval == 0:
        lib.FlushGPU()


end_batch._count = 0
end_batch.flush_interval = 10


def warm_pool(sizes, copies=2):
    sizes = list(sizes)
    lib.WarmPool((ctypes.c_uint * len(sizes))(*sizes), len(sizes), copies)


def get_pool_stats():
    h, m = ctypes.c_uint64(0), ctypes.c_uint64(0)
    lib.GetPoolStats(ctypes.byref(h), ctypes.byref(m))
    return h.value, m.value


def get_pool_memory():
    return lib.GetPoolMemory()


def drain_pool():
    lib.DrainPool()


def last_error():
    return (lib.dct_last_error() or b"").decode()


# ---------------------------------------------------------------------------
# ComputeGraph: record one step's dispatches, replay them in one call
# (nn_engine.py:2505-2771)
# ---------------------------------------------------------------------------
class ComputeGraph:
    """Record the RunShader calls of one forward+backward(+SGD) and replay them from C."""

    def __init__(self):
        self._cmds = []
        self._arr = None
        self._keep = []
        self._shader_cache = {}

    def _resolve(self, name):
        if name not in self._shader_cache:
            self._shader_cache[name] = lib.ResolveShader(name)
        return self._shader_cache[name]

    def record(self, fn):
        """Run fn() while recording every RunShader/RunShaderRaw dispatch; returns fn's result."""
        global lib
        real = lib
        rec = self

        class _Recorder:
            def __getattr__(self, k):
                return getattr(real, k)

            def RunShader(self, name, srvs, ns, uavs, nu, threads, cb, cbsize):
                c = SeqCmd()
                c.shader = rec._resolve(name)
                for i in range(ns):
                    c.srvs[i] = srvs[i]
                for i in range(nu):
                    c.uavs[i] = uavs[i]
                c.srvCount, c.uavCount = ns, nu
                c.threads[0], c.threads[1], c.threads[2] = threads[0], threads[1], threads[2]
                if cb is not None and cbsize:
                    ctypes.memmove(c.cbData, ctypes.addressof(cb._obj), min(cbsize, 64))
                c.cbSize = cbsize
                rec._cmds.append(c)
                real.RunShader(name, srvs, ns, uavs, nu, threads, cb, cbsize)

            RunShaderRaw = RunShader

            def CreateBuffer(self, data, count):
                h = real.CreateBuffer(data, count)
                if h:
                    real.AddRefBuffer(h)
                    rec._keep.append(h)
                return h

        lib = _Recorder()
        try:
            out = fn()
        finally:
            lib = real
        self._arr = (SeqCmd * len(self._cmds))(*self._cmds)
        return out

    def replay(self):
        if self._arr is None:
            raise RuntimeError("ComputeGraph: nothing recorded")
        lib.RunSequence(ctypes.cast(self._arr, ctypes.c_void_p), len(self._cmds))

    def release(self):
        for h in self._keep:
            lib.ReleaseBuffer(h)
        self._keep = []
        self._cmds = []
        self._arr = None

    def __len__(self):
        return len(self._cmds)
