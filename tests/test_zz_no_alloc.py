"""The allocation-free BatchNorm entry point, omCudaBatchNorm2dNoAlloc.

Some callers of this library cannot allocate device memory once they are running: an
inspection loop that reserved its whole VRAM budget at start-up and must not stall or fail
on an allocation mid-run, or an engine embedded in a host application whose own allocator
owns the device. For them, omCudaBatchNorm2dNoAlloc computes exactly what omCudaBatchNorm2d
computes, but keeps its training-mode partial sums in a fixed per-device array inside the
library instead of pool memory.

This file is named so that pytest collects it last. It checks, through the C ABI, that calls
in a row give bit for bit what the pool-backed entry point gives (both run the same kernels
with the same number of partial-sum splits), including a call whose channel and split counts
differ from the one before, so that slots left over in the shared array would show, and that
a channel count beyond the fixed maximum is refused without a launch. It runs the same alone
in a fresh process and after the other tests.
"""
import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu


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
    # 64 channels of 32768 values (several partial-sum splits), then 24 channels of 6400 values
    # (another split count), then the first shape again
    shapes = [(8, 64, 64, 64), (4, 24, 40, 40), (8, 64, 64, 64)]
    state = {}
    for call_no, (n, c, h, w) in enumerate(shapes):
        if c not in state:
            g = rng.uniform(0.5, 1.5, c).astype(np.float32)
            b = rng.standard_normal(c).astype(np.float32)
            rm = (rng.standard_normal(c) * 0.1).astype(np.float32)
            rv = rng.uniform(0.5, 1.5, c).astype(np.float32)
            state[c] = [g, b, rm, rv, rm.copy(), rv.copy()]
        g, b, rm_a, rv_a, rm_b, rv_b = state[c]
        x = (rng.standard_normal((n, c, h, w)) * (1 + call_no) + 0.3).astype(np.float32)
        ref = _bn(lib.omCudaBatchNorm2d, x, g, b, rm_a, rv_a, n, c, h, w, 1)
        got = _bn(lib.omCudaBatchNorm2dNoAlloc, x, g, b, rm_b, rv_b, n, c, h, w, 1)
        # output, saved mean, saved inverse std, running mean, running variance
        for a, e in zip(got, ref):
            assert np.array_equal(a, e), (call_no, rel_err(a, e))
        state[c] = [g, b, ref[3], ref[4], got[3], got[4]]
    # eval mode reads the running statistics only
    g, b, rm_a, rv_a, rm_b, rv_b = state[64]
    x = rng.standard_normal((2, 64, 5, 5)).astype(np.float32)
    ref = _bn(lib.omCudaBatchNorm2d, x, g, b, rm_a, rv_a, 2, 64, 5, 5, 0)
    got = _bn(lib.omCudaBatchNorm2dNoAlloc, x, g, b, rm_b, rv_b, 2, 64, 5, 5, 0)
    assert np.array_equal(got[0], ref[0])


def test_no_alloc_batchnorm_refuses_too_many_channels(gpu):
    from omnimatchdeeplearningtool_b200._lib import lib
    # 4097 channels exceed the fixed array; the call is refused before anything launches
    st = lib.omCudaBatchNorm2dNoAlloc(16, 16, 16, 16, 16, 16, 16, 16, 1, 4097, 1, 1, 1e-5, 0.1, 1)
    assert st == -8
