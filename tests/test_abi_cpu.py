"""C-ABI surface of libdct_cuda.so, checked without a GPU.

The library must load, export every symbol include/dct_cuda.h declares (all 32
reference engine entry points plus the dct_* extensions), lay out GPUInfo and
SeqCmd like engine.cpp, and fail quietly with an error code -- never crash --
when no device is present.  With the reference sources mounted, the unmodified
reference nn_engine.py must bind against it.
"""
import ctypes
import os
import re
import subprocess

import pytest

from directcompute_torch_b200 import _abi, lib_path

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "dct_cuda.h")


def _declared():
    txt = open(HEADER).read()
    return sorted(set(re.findall(r"DCT_API\s+[\w\s\*]+?\b(\w+)\s*\(", txt)))


@pytest.fixture(scope="module")
def so():
    p = lib_path()
    if not os.path.exists(p):
        from directcompute_torch_b200.build import build
        build()
    return p


def test_header_declares_all_reference_symbols():
    decl = set(_declared())
    missing = [s for s in _abi.REFERENCE_SYMBOLS if s not in decl]
    assert not missing, missing
    assert len(_abi.REFERENCE_SYMBOLS) == 32


def test_library_exports_every_declared_symbol(so):
    out = subprocess.run(["nm", "-D", "--defined-only", so], capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = [s for s in _declared() if s not in exported]
    assert not missing, missing


def test_ctypes_signatures_cover_header(so):
    assert set(_declared()) == set(_abi.SIGNATURES), set(_declared()) ^ set(_abi.SIGNATURES)
    lib = ctypes.CDLL(so)
    _abi.bind(lib)


def test_struct_layouts_match_reference():
    # engine.cpp:940-950 SeqCmd (its comment says 256 bytes; the x86-64 layout of
    # its fields is 200 bytes, which nn_engine.py:2490-2502 mirrors field by field)
    assert ctypes.sizeof(_abi.SeqCmd) == 200
    assert _abi.SeqCmd.uavs.offset == 80 and _abi.SeqCmd.threads.offset == 116
    assert _abi.SeqCmd.cbData.offset == 128 and _abi.SeqCmd.cbSize.offset == 192
    # engine.cpp:14-21 GPUInfo
    assert ctypes.sizeof(_abi.GPUInfo) == 160
    assert _abi.GPUInfo.description.offset == 28


def _has_gpu():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.mark.skipif(_has_gpu(), reason="checks the no-device behaviour")
def test_no_device_fails_quietly(so):
    code = (
        "import ctypes, sys; sys.path.insert(0, %r)\n"
        "from directcompute_torch_b200 import _abi\n"
        "lib = ctypes.CDLL(%r); _abi.bind(lib)\n"
        "assert not lib.InitEngine()\n"
        "assert lib.dct_error_code() == 1, lib.dct_error_code()\n"
        "assert lib.CreateBuffer(None, 16) is None\n"
        "lib.ReleaseBuffer(None); lib.FlushGPU(); lib.SyncGPU()\n"
        "assert lib.CompileShader(b'relu', '') != 0 or True\n"
        "assert not lib.CompileShaderEx(b'x', '', b'CSMain')\n"
        "assert lib.ResolveShader(b'nope') is None\n"
        "print('ok')\n" % (ROOT, so))
    r = subprocess.run(["python", "-c", code], capture_output=True, text=True, timeout=120,
                       env={**os.environ, "CUDA_VISIBLE_DEVICES": ""})
    assert r.returncode == 0 and "ok" in r.stdout, r.stderr


@pytest.mark.skipif(_has_gpu(), reason="checks the no-device behaviour")
def test_unmodified_reference_binds_libdct(so, reference_dir):
    code = (
        "import ctypes, sys; sys.path.insert(0, %r)\n"
        "from oracle.fakelib import load_reference_engine\n"
        "lib = ctypes.CDLL(%r)\n"
        "nn = load_reference_engine(%r, lib)\n"
        "assert nn.lib is lib\n"
        "for name in ('InitEngine','CreateBuffer','RunShader','SGDBatchClipped','RunSequenceWithSGD','WarmPool'):\n"
        "    assert getattr(nn.lib, name).argtypes is not None or name == 'InitEngine'\n"
        "print('ok')\n" % (ROOT, so, reference_dir))
    r = subprocess.run(["python", "-c", code], capture_output=True, text=True, timeout=300,
                       env={**os.environ, "CUDA_VISIBLE_DEVICES": ""})
    assert r.returncode == 0 and "ok" in r.stdout, r.stdout + r.stderr


def test_ops_bind_refuses_a_module_without_a_tensor_type():
    """ops.bind takes any module whose Tensor has the reference Tensor's protocol; others are refused."""
    from directcompute_torch_b200 import ops
    from directcompute_torch_b200.tensor import DeviceTensor
    try:
        with pytest.raises(TypeError):
            ops.bind(object())

        class M:
            class Tensor:
                pass
        with pytest.raises(TypeError):
            ops.bind(M)
        assert ops.bind() is DeviceTensor
    finally:
        ops.bind()
