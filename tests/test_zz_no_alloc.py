"""The allocation-free BatchNorm entry point, omCudaBatchNorm2dNoAlloc.

Some callers of this library cannot allocate device memory once they are running: an
inspection loop that reserved its whole VRAM budget at start-up and must not stall or fail
on an allocation mid-run, or an engine embedded in a host application whose own allocator
owns the device. For them, omCudaBatchNorm2dNoAlloc computes exactly what omCudaBatchNorm2d
computes, but keeps its training-mode partial sums in a fixed per-device array inside the
library instead of pool memory.

This file is named so that pytest collects it last. It checks, through the C ABI, that two
calls in a row match the pool-backed entry point within the fp32 tolerance (1e-4, max-
normalised), and that a channel count beyond the fixed maximum is refused without a launch.
It runs the same alone in a fresh process and after the other tests.
"""
import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu
TOL = 1e-4


def _bn(lib_fn, x, g, b, rm, rv, n, c, h, w, training):
    from omnimatchdeeplearningtool_b200.backend import DeviceBuffer
    keep = [DeviceBuffer.from_numpy(a) for a in (x, g, b, rm, rv)]
    y, sm, si = (DeviceBuffer.zeros(a) for a in (x.nbytes, c * 4, c * 4))
    st = lib_fn(keep[0].ptr, y.ptr, keep[1].ptr, keep[2].ptr, keep[3].ptr, keep[4].ptr, sm.ptr,
                si.ptr, n, c, h, w, 1e-5, 0.1, training)
    assert st == 0, st
    return (y.to_numpy(x.shape), sm.to_numpy((c,)), si.to_numpy((c,)), keep[3].to_numpy((c,)),
            keep[4].to_numpy((c,)))


def test_no_alloc_batchnorm_matches_pool_backed_entry_point(gpu):
    from omnimatchdeeplearningtool_b200._lib import lib
    rng = np.random.Generator(np.random.PCG64(21))
    n, c, h, w = 8, 64, 64, 64   # 32768 values per channel: several partial-sum splits
    g = rng.uniform(0.5, 1.5, c).astype(np.float32)
    b = rng.standard_normal(c).astype(np.float32)
    rm_a = (rng.standard_normal(c) * 0.1).astype(np.float32)
    rv_a = rng.uniform(0.5, 1.5, c).astype(np.float32)
    rm_b, rv_b = rm_a.copy(), rv_a.copy()
    for call_no in range(2):   # two calls in a row; the shared array keeps the first's contents
        x = (rng.standard_normal((n, c, h, w)) * (1 + call_no) + 0.3).astype(np.float32)
        ref = _bn(lib.omCudaBatchNorm2d, x, g, b, rm_a, rv_a, n, c, h, w, 1)
        got = _bn(lib.omCudaBatchNorm2dNoAlloc, x, g, b, rm_b, rv_b, n, c, h, w, 1)
        for a, e in zip(got, ref):
            assert rel_err(a, e) <= TOL, (call_no, rel_err(a, e))
        rm_a, rv_a = ref[3], ref[4]
        rm_b, rv_b = got[3], got[4]
    # eval mode reads the running statistics only
    x = rng.standard_normal((2, c, 5, 5)).astype(np.float32)
    ref = _bn(lib.omCudaBatchNorm2d, x, g, b, rm_a, rv_a, 2, c, 5, 5, 0)
    got = _bn(lib.omCudaBatchNorm2dNoAlloc, x, g, b, rm_b, rv_b, 2, c, 5, 5, 0)
    assert rel_err(got[0], ref[0]) <= TOL


def test_no_alloc_batchnorm_refuses_too_many_channels(gpu):
    from omnimatchdeeplearningtool_b200._lib import lib
    # 4097 channels exceed the fixed array; the call is refused before anything launches
    st = lib.omCudaBatchNorm2dNoAlloc(16, 16, 16, 16, 16, 16, 16, 16, 1, 4097, 1, 1, 1e-5, 0.1, 1)
    assert st == -8
