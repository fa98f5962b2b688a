"""One conv2d -> BatchNorm2d (eval) -> ReLU layer, the unit of the per-layer sweep.

The reference composes it from three modules (om.engine.conv.ixx Conv2d, BatchNorm2d, ReLU) that
call CPUBackend::conv2d, batchNorm2d and relu (cpu_backend.ixx:619, :781, :317). Here:

* fp32: the reference-layout entry points omCudaConv2d -> omCudaBatchNorm2d (eval) ->
  omCudaReLU on NCHW fp32, three launches;
* bf16 / fp16: the input converted once to NHWC 16-bit, BatchNorm folded into the packed
  weights, and one tcgen05 launch of omCudaConv2dBnAct per forward.

`run()` enqueues one forward on the library's compute stream; `result()` returns the output
as host NCHW fp32.
"""
from __future__ import annotations

from typing import List

import numpy as np

from ._lib import ACT_RELU, DTYPE_BF16, DTYPE_F16, DTYPE_F32, call, lib
from .backend import DeviceBuffer

DTYPES = {"fp32": DTYPE_F32, "bf16": DTYPE_BF16, "fp16": DTYPE_F16}


class ConvBnReluLayer:
    def __init__(self, x: np.ndarray, w: np.ndarray, gamma: np.ndarray, beta: np.ndarray,
                 mean: np.ndarray, var: np.ndarray, stride: int, pad: int, dtype: str,
                 eps: float = 1e-5):
        if dtype not in DTYPES:
            raise ValueError(f"dtype must be one of {sorted(DTYPES)}")
        self.n, self.c, self.h, self.w = x.shape
        self.k, _, self.r, self.s = w.shape
        self.stride, self.pad, self.dtype, self.eps = stride, pad, dtype, eps
        self.p = (self.h + 2 * pad - self.r) // stride + 1
        self.q = (self.w + 2 * pad - self.s) // stride + 1
        self.flops = 2 * self.n * self.p * self.q * self.k * self.c * self.r * self.s
        self._keep: List[DeviceBuffer] = []
        dev = self._dev
        if dtype == "fp32":
            self.x, self.wt = dev(x), dev(w)
            self.bn = [dev(a) for a in (gamma, beta, mean, var)]
            cnt = self.n * self.k * self.p * self.q
            self.z, self.y, self.out = (self._buf(cnt * 4) for _ in range(3))
            self.stats = [self._buf(self.k * 4) for _ in range(2)]
        else:
            dt = DTYPES[dtype]
            self.cs = int(lib.omCudaStoredChannels(self.c))
            x32 = dev(x)
            self.x = self._buf(self.n * self.h * self.w * self.cs * 2)
            call("omCudaNchwToNhwc", x32.ptr, self.x.ptr, self.n, self.c, self.h, self.w, self.cs, dt)
            w32 = dev(w)
            bn = [dev(a) for a in (gamma, beta, mean, var)]
            self.packed = self._buf(int(lib.omCudaPackedConvWeightElems(self.k, self.r, self.s,
                                                                         self.cs)) * 2)
            self.bias = self._buf(self.k * 4)
            call("omCudaPackConvWeight", w32.ptr, None, *[b.ptr for b in bn], eps, self.packed.ptr,
                 self.bias.ptr, self.k, self.c, self.r, self.s, self.cs, dt)
            self.out = self._buf(self.n * self.p * self.q * self.k * 2)

    def _dev(self, a: np.ndarray) -> DeviceBuffer:
        b = DeviceBuffer.from_numpy(np.ascontiguousarray(a, np.float32))
        self._keep.append(b)
        return b

    def _buf(self, nbytes: int) -> DeviceBuffer:
        b = DeviceBuffer(nbytes)
        self._keep.append(b)
        return b

    def run(self) -> None:
        n, c, h, w, k = self.n, self.c, self.h, self.w, self.k
        if self.dtype == "fp32":
            call("omCudaConv2d", self.x.ptr, self.wt.ptr, None, self.z.ptr, n, c, h, w, k, self.r,
                 self.s, self.stride, self.pad)
            call("omCudaBatchNorm2d", self.z.ptr, self.y.ptr, self.bn[0].ptr, self.bn[1].ptr,
                 self.bn[2].ptr, self.bn[3].ptr, self.stats[0].ptr, self.stats[1].ptr, n, k,
                 self.p, self.q, self.eps, 0.1, 0)
            call("omCudaReLU", self.y.ptr, self.out.ptr, n * k * self.p * self.q)
        else:
            call("omCudaConv2dBnAct", self.x.ptr, self.packed.ptr, self.bias.ptr, None,
                 self.out.ptr, n, h, w, self.cs, k, self.r, self.s, self.stride, self.pad,
                 ACT_RELU, DTYPES[self.dtype], DTYPES[self.dtype])

    def result(self) -> np.ndarray:
        shape = (self.n, self.k, self.p, self.q)
        if self.dtype == "fp32":
            return self.out.to_numpy(shape)
        o32 = DeviceBuffer(int(np.prod(shape)) * 4)
        try:
            call("omCudaNhwcToNchw", self.out.ptr, o32.ptr, self.n, self.k, self.p, self.q, self.k,
                 DTYPES[self.dtype])
            return o32.to_numpy(shape)
        finally:
            o32.free()

    def close(self) -> None:
        for b in self._keep:
            b.free()
        self._keep.clear()
