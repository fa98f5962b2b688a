"""The bounded in-kernel waits of the tensor-core conv kernel, driven to run out.

omCudaTestStallNextConv arms one launch whose producer stops issuing loads after a few k-blocks
(every load it issued lands), with the role waits limited to 20 ms: the MMA issuer then waits
for a load that nothing will bring, gives up, raises the CTA's abort flag, drains its issued
MMAs, and the epilogue warps leave too. No fault, trap or unbounded wait is involved. Checked:

  * the launch ends within the limits (well under a second), and omCudaSynchronizeChecked
    reports OM_ERR_KERNEL_TIMEOUT with the producer/MMA/epilogue bits in the error word and no
    drain failure (every issued load and MMA completed before the CTA left);
  * the next, normal launch on the same device is correct (against the oracle) and reports no
    error: the context stays usable.
"""
import time

import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu

ERRBIT_TC_PRODUCER, ERRBIT_TC_MMA, ERRBIT_TC_EPILOGUE, ERRBIT_TC_DRAIN = 1, 2, 4, 8


def test_stalled_producer_times_out_and_the_device_stays_usable(gpu):
    import ctypes
    import oracle as orc
    from omnimatchdeeplearningtool_b200 import _lib
    from omnimatchdeeplearningtool_b200._lib import call, lib
    from omnimatchdeeplearningtool_b200.backend import DeviceBuffer
    n, c, h, k = 2, 256, 14, 256      # 36 k-blocks per tile
    rng = np.random.Generator(np.random.PCG64(3))
    x = rng.standard_normal((n, c, h, h), dtype=np.float32)
    w = (rng.standard_normal((k, c, 3, 3)) * np.sqrt(2.0 / (c * 9))).astype(np.float32)
    dt = _lib.DTYPE_BF16
    x32 = DeviceBuffer.from_numpy(x)
    xs = DeviceBuffer(n * h * h * c * 2)
    call("omCudaNchwToNhwc", x32.ptr, xs.ptr, n, c, h, h, c, dt)
    w32 = DeviceBuffer.from_numpy(w)
    packed = DeviceBuffer(int(lib.omCudaPackedConvWeightElems(k, 3, 3, c)) * 2)
    bias = DeviceBuffer.zeros(k * 4)
    call("omCudaPackConvWeight", w32.ptr, None, None, None, None, None, 1e-5, packed.ptr,
         bias.ptr, k, c, 3, 3, c, dt)
    out = DeviceBuffer(n * h * h * k * 2)
    call("omCudaSynchronize")

    # the stalled launch
    call("omCudaTestStallNextConv", 3, 20_000_000)
    t0 = time.perf_counter()
    call("omCudaConv2dBnAct", xs.ptr, packed.ptr, bias.ptr, None, out.ptr, n, h, h, c, k, 3, 3, 1,
         1, 0, dt, dt)
    code = ctypes.c_uint()
    call("omCudaGetKernelError", ctypes.byref(code))
    dt_s = time.perf_counter() - t0
    assert code.value & (ERRBIT_TC_MMA | ERRBIT_TC_EPILOGUE), code.value
    assert not code.value & ERRBIT_TC_DRAIN, code.value
    assert dt_s < 1.0, dt_s
    # the same through the checked synchronisation: a second stalled launch
    call("omCudaTestStallNextConv", 0, 5_000_000)
    call("omCudaConv2dBnAct", xs.ptr, packed.ptr, bias.ptr, None, out.ptr, n, h, h, c, k, 3, 3, 1,
         1, 0, dt, dt)
    assert lib.omCudaSynchronizeChecked() == -6   # OM_ERR_KERNEL_TIMEOUT
    assert lib.omCudaSynchronizeChecked() == 0    # read and cleared

    # a normal launch afterwards is correct
    call("omCudaConv2dBnAct", xs.ptr, packed.ptr, bias.ptr, None, out.ptr, n, h, h, c, k, 3, 3, 1,
         1, 0, dt, dt)
    assert lib.omCudaSynchronizeChecked() == 0
    o32 = DeviceBuffer(n * k * h * h * 4)
    call("omCudaNhwcToNchw", out.ptr, o32.ptr, n, k, h, h, k, dt)
    got = o32.to_numpy((n, k, h, h))
    want = orc.conv2d(x, w, None, 1, 1)
    assert rel_err(got, want) <= 2e-2
    # the tf32 (fp32-layout) path shares the kernel and its waits
    call("omCudaTestStallNextConv", 2, 5_000_000)
    y = DeviceBuffer(n * k * h * h * 4)
    call("omCudaConv2d", x32.ptr, w32.ptr, None, y.ptr, n, c, h, h, k, 3, 3, 1, 1)
    assert lib.omCudaSynchronizeChecked() == -6
    call("omCudaConv2d", x32.ptr, w32.ptr, None, y.ptr, n, c, h, h, k, 3, 3, 1, 1)
    assert lib.omCudaSynchronizeChecked() == 0
    assert rel_err(y.to_numpy((n, k, h, h)), want) <= 1e-4
