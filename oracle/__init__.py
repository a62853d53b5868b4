"""CPU oracle for the directcompute_torch hot path -- TEST INFRASTRUCTURE ONLY.

Nothing in the product (`directcompute_torch_b200/`, `libdct_cuda.so`) imports,
links or executes this package.  Only `tests/`, `__graft_entry__.smoke()` and the
`cpu_baseline` / `--impl reference` legs of `bench.py` use it, and only as the
checker or as the timed CPU baseline.

Contents
--------
shaders.py  NumPy restatement of each reference HLSL shader on the hot path
            (one function per shader, each citing the `nn_*.hlsl` file:line it
            follows), plus `run_shader()` which decodes the reference's cbuffer
            layouts exactly as `nn_engine.py` packs them.
newops.py   NumPy-semantics definitions of the ops the reference has no GPU
            kernel for (N-d broadcast binary ops, exp/log/tanh, axis and full
            reductions, fused softmax+CE) with float64-accumulated references.
fakelib.py  `FakeLib`: every C-ABI symbol `nn_engine.py` binds, implemented over
            NumPy buffers.  Swapped in for `ctypes.CDLL("engine.dll")` it lets
            the unmodified reference `nn_engine.py` and its own verification
            scripts run on the CPU -- that is how the oracle is pinned.
rng.py      Host restatement of the device Philox4x32-10 generator (Salmon et
            al., SC'11) used to fill the large synthetic benchmark inputs.
threaded.py Multi-core driver that runs the oracle over row chunks (NumPy
            releases the GIL inside ufuncs) -- the timed CPU baseline.

Parity pinning
--------------
The reference publishes no golden vectors.  Its own checks (nn_verify.py
verify_relu / verify_softmax / verify_linear / grad_check, verify_batchnorm.py,
verify_dice_loss.py) are executed in this container against `FakeLib` by
`tests/test_oracle_pinned.py`; fixtures under `tests/golden/` are produced by
`tests/golden/make_golden.py`, which drives the reference's own `nn_engine.py`
Function classes over `FakeLib` and records every dispatch.
"""
