"""Execution plans over the C ABI.

:class:`InferencePlan` is the fused NHWC 16-bit inference path: it walks a network's named
parameters (the names ``Module::namedParameters()`` reports, e.g. ``layer1.0.conv1.weight``,
``layer1.0.bn1.running_mean``), folds each eval-mode BatchNorm into the preceding conv's
weights and bias on the device, and records one launch per fused op:

* conv + BN (+ residual add) (+ ReLU/ReLU6) -> ``omCudaConv2dBnAct`` (tcgen05 implicit GEMM)
* depthwise conv + BN + ReLU6            -> ``omCudaDepthwiseConv2dNhwc``
* max pool / global average pool         -> NHWC bandwidth kernels
* Linear (x @ W + b, W ``[in, out]``)    -> ``omCudaConv2dBnAct`` as a 1x1 conv with fp32 out

The sequence is captured once into a CUDA graph and replayed. Block wiring follows the
reference forward passes: BasicBlock (om.engine.resnet.ixx:55-80) and Bottleneck
(om.engine.resnet50.ixx:62-85) add the shortcut after the last BN and apply ReLU after the
add, so the add and the ReLU fuse into the last conv's epilogue; InvertedResidual
(om.engine.mobilenet.ixx:203-225) adds without an activation.

:class:`Fp32Net` runs the same networks in the reference's own layout (NCHW fp32) through
the reference-named entry points (omCudaConv2d, omCudaBatchNorm2d, ...), including the
training step (forward, CE loss, backward, SGD momentum) of the reference engine.
"""
from __future__ import annotations

import ctypes
from typing import Dict, List, Optional

import numpy as np

from . import _lib
from ._lib import ACT_NONE, ACT_RELU, ACT_RELU6, DTYPE_BF16, DTYPE_F16, DTYPE_F32, call, lib
from .backend import CUDABackend as B
from .backend import DeviceBuffer
from .synth import ConvSpec, NetSpec

_ACT = {"relu": ACT_RELU, "relu6": ACT_RELU6, "none": ACT_NONE}


def stored_channels(c: int) -> int:
    return int(lib.omCudaStoredChannels(c))


class InferencePlan:
    """Fused NHWC inference of a :class:`NetSpec` at a fixed batch size."""

    def __init__(self, net: NetSpec, weights: Dict[str, np.ndarray], batch: int,
                 dtype: int = DTYPE_BF16, h: int = 224, w: int = 224):
        assert dtype in (DTYPE_BF16, DTYPE_F16)
        self.net, self.batch, self.dtype, self.h, self.w = net, batch, dtype, h, w
        self.ops: List = []           # callables, each issuing one C-ABI launch
        self.keep: List[DeviceBuffer] = []
        self.graph = None
        self.conv_flops = 0           # algorithmic FLOPs of the tensor-core convs + FC
        self.n_tc_launches = 0
        self.n_launches = 0
        self.tc_op_index: List[int] = []   # positions in self.ops of tensor-core launches
        self.meta: List[dict] = []         # one descriptor per op (kind, buffers, shape)
        # input staging: NCHW fp32 as the engine hands it over
        self.in_f32 = self._buf(batch * 3 * h * w * 4)
        # the image stem reads the NCHW fp32 input directly (tcgen05 kernel, gathered A tile)
        cur, hh, ww, c = self.in_f32, h, w, 3
        act0 = _ACT[net.stem_act]
        for i, cv in enumerate(net.stem):
            if i == 0 and cv.k <= 8 and cv.groups == 1:
                cur, hh, ww, c = self._stem(cv, weights, hh, ww, act0)
            else:
                cur, hh, ww, c = self._conv(cv, weights, cur, hh, ww, c, act0)
        if net.maxpool:
            p, q = (hh + 2 - 3) // 2 + 1, (ww + 2 - 3) // 2 + 1
            cs = stored_channels(c)
            y = self._buf(batch * p * q * cs * 2)
            src = cur
            self._need(src, batch * hh * ww * cs * 2)
            self._op(lambda src=src, y=y, hh=hh, ww=ww, cs=cs: call(
                "omCudaMaxPool2dNhwc", src.ptr, y.ptr, batch, hh, ww, cs, 3, 2, 1, dtype),
                dict(kind="maxpool", inp=src, out=y, c=c, cs=cs, h=hh, w=ww, p=p, q=q))
            cur, hh, ww = y, p, q
        for blk in net.blocks:
            cur, hh, ww, c = self._block(blk, weights, cur, hh, ww, c)
        # global average pool -> [N, C] 16-bit, then the FC as a 1x1 conv with fp32 logits
        cs = stored_channels(c)
        pooled = self._buf(batch * cs * 2)
        src = cur
        self._need(src, batch * hh * ww * cs * 2)
        self._op(lambda src=src, pooled=pooled, hh=hh, ww=ww, cs=cs: call(
            "omCudaGlobalAvgPoolNhwc", src.ptr, pooled.ptr, batch, hh * ww, cs, dtype, dtype),
            dict(kind="gap", inp=src, out=pooled, c=c, cs=cs, h=hh, w=ww))
        fc_w = np.ascontiguousarray(weights["fc.weight"].T).reshape(net.classes, net.fc_in, 1, 1)
        fc_b = weights["fc.bias"].reshape(-1)
        self.logits = self._buf(batch * net.classes * 4)
        self._conv_raw(fc_w, fc_b, None, pooled, 1, 1, net.fc_in, net.classes, 1, 1, 0,
                       ACT_NONE, None, out=self.logits, out_dtype=DTYPE_F32)

    # -------------------------------------------------------------- building blocks
    @staticmethod
    def _need(buf: DeviceBuffer, nbytes: int) -> None:
        """Every recorded launch is checked against its buffers' sizes when it is recorded."""
        if buf.nbytes < nbytes:
            raise ValueError(f"device buffer of {buf.nbytes} B is smaller than the {nbytes} B "
                             "this launch touches")

    def _buf(self, nbytes: int) -> DeviceBuffer:
        b = DeviceBuffer(nbytes)
        self.keep.append(b)
        return b

    def _op(self, fn, meta=None):
        self.ops.append(fn)
        self.meta.append(meta or {})
        self.n_launches += 1

    def _upload(self, arr: Optional[np.ndarray]) -> Optional[DeviceBuffer]:
        if arr is None:
            return None
        b = DeviceBuffer.from_numpy(np.ascontiguousarray(arr, dtype=np.float32))
        self.keep.append(b)
        return b

    def _conv_raw(self, wt, conv_bias, bn, x, hh, ww, cin, cout, k, stride, pad, act,
                  residual, out=None, out_dtype=None):
        """Pack weights (BN folded) and record one fused tensor-core conv launch."""
        n = self.batch
        cs_in = stored_channels(cin)
        cs_out = stored_channels(cout)
        if cs_out != cout:
            raise ValueError(f"output channels {cout} must be a multiple of 8")
        dt = self.dtype
        od = dt if out_dtype is None else out_dtype
        wbuf = self._upload(wt)
        cb = self._upload(conv_bias)
        g = b_ = m = v = None
        if bn is not None:
            g, b_, m, v = (self._upload(a) for a in bn)
        elems = int(lib.omCudaPackedConvWeightElems(cout, k, k, cs_in))
        packed = self._buf(elems * 2)
        bias = self._buf(cout * 4)
        ptr = lambda d: d.ptr if d is not None else None
        call("omCudaPackConvWeight", wbuf.ptr, ptr(cb), ptr(g), ptr(b_), ptr(m), ptr(v), 1e-5,
             packed.ptr, bias.ptr, cout, cin, k, k, cs_in, dt)
        p = (hh + 2 * pad - k) // stride + 1
        q = (ww + 2 * pad - k) // stride + 1
        obytes = n * p * q * cout * (4 if od == DTYPE_F32 else 2)
        if out is None:
            out = self._buf(obytes)
        self._need(x, n * hh * ww * cs_in * 2)
        self._need(out, obytes)
        if residual is not None:
            self._need(residual, obytes)
        res = residual
        self._op(lambda x=x, out=out, res=res: call(
            "omCudaConv2dBnAct", x.ptr, packed.ptr, bias.ptr, res.ptr if res is not None else None,
            out.ptr, n, hh, ww, cs_in, cout, k, k, stride, pad, act, dt, od),
            dict(kind="conv", inp=x, out=out, res=residual, w=wt, conv_bias=conv_bias, bn=bn,
                 c=cin, cs=cs_in, k=cout, ks=k, stride=stride, pad=pad, act=act, h=hh, wd=ww,
                 p=p, q=q, out_dtype=od))
        self.n_tc_launches += 1
        self.tc_op_index.append(len(self.ops) - 1)
        self.conv_flops += 2 * n * p * q * cout * cin * k * k
        return out, p, q, cout

    def _stem(self, cv: ConvSpec, weights, hh, ww, act):
        """First conv on the NCHW fp32 image with its BN folded (omCudaStemConvBnAct)."""
        n, dt = self.batch, self.dtype
        wbuf = self._upload(weights[cv.name + ".weight"])
        g, b_, m, v = (self._upload(a) for a in self._bn_params(weights, cv.bn))
        packed = self._buf(int(lib.omCudaPackedStemWeightElems(cv.cout, cv.cin, cv.k)) * 2)
        bias = self._buf(cv.cout * 4)
        call("omCudaPackStemWeight", wbuf.ptr, None, g.ptr, b_.ptr, m.ptr, v.ptr, 1e-5, packed.ptr,
             bias.ptr, cv.cout, cv.cin, cv.k, cv.k, dt)
        p = (hh + 2 * cv.pad - cv.k) // cv.stride + 1
        q = (ww + 2 * cv.pad - cv.k) // cv.stride + 1
        out = self._buf(n * p * q * cv.cout * 2)
        x = self.in_f32
        self._need(x, n * cv.cin * hh * ww * 4)
        self._op(lambda x=x, out=out: call(
            "omCudaStemConvBnAct", x.ptr, packed.ptr, bias.ptr, out.ptr, n, cv.cin, hh, ww,
            cv.cout, cv.k, cv.k, cv.stride, cv.pad, act, dt),
            dict(kind="stem", inp=x, out=out, w=weights[cv.name + ".weight"],
                 bn=self._bn_params(weights, cv.bn), c=cv.cin, k=cv.cout, ks=cv.k,
                 stride=cv.stride, pad=cv.pad, act=act, h=hh, wd=ww, p=p, q=q))
        self.n_tc_launches += 1
        self.tc_op_index.append(len(self.ops) - 1)
        self.conv_flops += 2 * n * p * q * cv.cout * cv.cin * cv.k * cv.k
        return out, p, q, cv.cout

    def _bn_params(self, weights, bn: str):
        return (weights[bn + ".gamma"], weights[bn + ".beta"], weights[bn + ".running_mean"],
                weights[bn + ".running_var"])

    def _conv(self, cv: ConvSpec, weights, x, hh, ww, c, act, residual=None):
        assert c == cv.cin
        if cv.groups == 1:
            return self._conv_raw(weights[cv.name + ".weight"], None, self._bn_params(weights, cv.bn),
                                  x, hh, ww, cv.cin, cv.cout, cv.k, cv.stride, cv.pad, act, residual)
        assert cv.groups == cv.cin == cv.cout and residual is None
        return self._depthwise(cv, weights, x, hh, ww, act)

    def _depthwise(self, cv: ConvSpec, weights, x, hh, ww, act):
        n, c = self.batch, cv.cin
        cs = stored_channels(c)
        wbuf = self._upload(weights[cv.name + ".weight"])
        g, b_, m, v = (self._upload(a) for a in self._bn_params(weights, cv.bn))
        packed = self._buf(cv.k * cv.k * cs * 4)
        bias = self._buf(cs * 4)
        call("omCudaPackDepthwiseWeight", wbuf.ptr, g.ptr, b_.ptr, m.ptr, v.ptr, 1e-5, packed.ptr,
             bias.ptr, c, cv.k, cv.k, cs)
        p = (hh + 2 * cv.pad - cv.k) // cv.stride + 1
        q = (ww + 2 * cv.pad - cv.k) // cv.stride + 1
        out = self._buf(n * p * q * cs * 2)
        self._need(x, n * hh * ww * cs * 2)
        dt = self.dtype
        self._op(lambda x=x, out=out: call(
            "omCudaDepthwiseConv2dNhwc", x.ptr, packed.ptr, bias.ptr, out.ptr, n, hh, ww, cs,
            cv.k, cv.k, cv.stride, cv.pad, act, dt),
            dict(kind="depthwise", inp=x, out=out, w=weights[cv.name + ".weight"],
                 bn=self._bn_params(weights, cv.bn), c=c, cs=cs, ks=cv.k, stride=cv.stride,
                 pad=cv.pad, act=act, h=hh, wd=ww, p=p, q=q))
        return out, p, q, c

    def _block(self, blk, weights, x, hh, ww, c):
        if blk.kind in ("basic", "bottleneck"):
            shortcut = x
            if blk.downsample is not None:
                shortcut, _, _, _ = self._conv(blk.downsample, weights, x, hh, ww, c, ACT_NONE)
            cur, h2, w2, c2 = x, hh, ww, c
            for i, cv in enumerate(blk.convs):
                last = i == len(blk.convs) - 1
                cur, h2, w2, c2 = self._conv(cv, weights, cur, h2, w2, c2, ACT_RELU,
                                             residual=shortcut if last else None)
            return cur, h2, w2, c2
        # inverted residual: expand (ReLU6) -> depthwise (ReLU6) -> project (linear) [+ x]
        e, d, pj = blk.convs
        cur, h2, w2, c2 = self._conv(e, weights, x, hh, ww, c, ACT_RELU6)
        cur, h2, w2, c2 = self._conv(d, weights, cur, h2, w2, c2, ACT_RELU6)
        cur, h2, w2, c2 = self._conv(pj, weights, cur, h2, w2, c2, ACT_NONE,
                                     residual=x if blk.residual else None)
        return cur, h2, w2, c2

    # -------------------------------------------------------------- execution
    def launch(self) -> None:
        """Issue the whole forward (graph replay when captured) on the compute stream."""
        if self.graph is not None:
            call("omCudaGraphLaunch", self.graph)
        else:
            for fn in self.ops:
                fn()

    def capture(self) -> None:
        call("omCudaSynchronize")
        call("omCudaGraphBeginCapture")
        try:
            for fn in self.ops:
                fn()
        finally:
            g = ctypes.c_void_p()
            st = lib.omCudaGraphEndCapture(ctypes.byref(g))
        _lib.check(st, "omCudaGraphEndCapture")
        self.graph = g.value

    def set_input(self, x: np.ndarray) -> None:
        assert x.shape == (self.batch, 3, self.h, self.w)
        self.in_f32.upload(np.ascontiguousarray(x, dtype=np.float32))

    def run(self, x: np.ndarray) -> np.ndarray:
        """Host NCHW fp32 input -> host fp32 logits [N, classes]."""
        self.set_input(x)
        self.launch()
        return self.logits.to_numpy((self.batch, self.net.classes))

    def close(self) -> None:
        if self.graph is not None:
            lib.omCudaGraphDestroy(self.graph)
            self.graph = None
        for b in self.keep:
            b.free()
        self.keep.clear()
