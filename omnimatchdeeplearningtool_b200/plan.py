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
from typing import Callable, Dict, List, Optional, Sequence, Tuple

import numpy as np

from . import _lib
from ._lib import (ACT_NONE, ACT_RELU, ACT_RELU6, DTYPE_BF16, DTYPE_F16, DTYPE_F32, DTYPE_U8,
                   call, lib)
from .backend import CUDABackend as B
from .backend import DeviceBuffer
from .synth import ConvSpec, NetSpec

_ACT = {"relu": ACT_RELU, "relu6": ACT_RELU6, "none": ACT_NONE}

# bytes per image sample of each input dtype
_INPUT_SIZE = {DTYPE_F32: 4, DTYPE_BF16: 2, DTYPE_F16: 2, DTYPE_U8: 1}

# the reference's ImageNet preset (om.engine.data_pipeline.ixx:767-771): (mean, std), RGB
IMAGENET_NORM = ((0.485, 0.456, 0.406), (0.229, 0.224, 0.225))


def _norm_arrays(mean: Sequence[float], std: Sequence[float], channels: int):
    """Per-channel mean and 1/std as ctypes float arrays, as the reference's normalizeImage
    derives them: channel c uses entry min(c, 2) when the image has 3 or more channels, entry 0
    otherwise; std below 1e-7 becomes 1e-7; 1/std is computed in fp32."""
    m = np.asarray(mean, np.float32)
    s = np.maximum(np.asarray(std, np.float32), np.float32(1e-7))
    idx = [min(ch, 2) if channels >= 3 else 0 for ch in range(channels)]
    inv = (np.float32(1.0) / s).astype(np.float32)
    arr = ctypes.c_float * channels
    return arr(*[float(m[i]) for i in idx]), arr(*[float(inv[i]) for i in idx])


def stored_channels(c: int) -> int:
    return int(lib.omCudaStoredChannels(c))


def to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 (round to nearest even, as __float2bfloat16_rn), as uint16 bit patterns;
    NaN is not expected in images."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


class InferencePlan:
    """Fused NHWC inference of a :class:`NetSpec` at a fixed batch size."""

    def __init__(self, net: NetSpec, weights: Dict[str, np.ndarray], batch: int,
                 dtype: int = DTYPE_BF16, h: int = 224, w: int = 224, input_slots: int = 2,
                 input_dtype: int = DTYPE_F32, fuse_pairs: bool = True,
                 fuse_stem_pool: bool = True,
                 input_norm: Optional[Tuple[Sequence[float], Sequence[float]]] = None):
        """input_dtype: element type of the NCHW image the plan takes, fp32 (the engine's
        tensors), the plan's own 16-bit dtype (half the bytes per image to copy to the
        device; the stem rounds its input to that type anyway, so the logits are the same), or
        DTYPE_U8: 8-bit samples, read as sample / 255 in fp32 on the device (a quarter of the
        bytes; the logits of the fp32 image sample / 255), usually with input_norm.

        input_norm: (mean, std) per channel, e.g. IMAGENET_NORM: the plan takes images that are
        not normalised yet and normalises them inside the stem's pre-pass as the reference's
        inferBatch does on the host (normalizeImage: (x - mean) * (1 / std) in fp32; images
        with more than 3 channels reuse the third channel's values, 1- and 2-channel images the
        first's). None: the images come normalised."""
        assert dtype in (DTYPE_BF16, DTYPE_F16)
        if input_slots not in (1, 2):
            raise ValueError("input_slots must be 1 or 2")
        if input_dtype not in (DTYPE_F32, dtype, DTYPE_U8):
            raise ValueError("input_dtype must be fp32, the plan's dtype or DTYPE_U8")
        self.net, self.batch, self.dtype, self.h, self.w = net, batch, dtype, h, w
        self.input_dtype = input_dtype
        self.input_norm = None
        if input_norm is not None:
            mean, std = input_norm
            self.input_norm = _norm_arrays(mean, std, 3)
        # a bottleneck's 3x3 conv and the 1x1 expansion after it run as one kernel where it
        # takes the shapes (omCudaConvPairBnAct: the 3x3 output never reaches device memory)
        self.fuse_pairs = fuse_pairs
        # the image stem and the 3x3/2 max pool after it run as one kernel where it takes the
        # shapes (omCudaStemConvBnActPoolIn: the stem output never reaches device memory)
        self.fuse_stem_pool = fuse_stem_pool
        self.ops: List = []           # callables, each issuing one C-ABI launch
        self.keep: List[DeviceBuffer] = []
        self.graphs: List[int] = []   # one captured graph per input slot
        self.conv_flops = 0           # algorithmic FLOPs of the tensor-core convs + FC
        self.n_tc_launches = 0
        self.n_launches = 0
        self.tc_op_index: List[int] = []   # positions in self.ops of tensor-core launches
        self.meta: List[dict] = []         # one descriptor per op (kind, buffers, shape)
        # input staging: NCHW fp32 as the engine hands it over. With two slots the next batch's
        # host->device copy lands in one slot while the forward reads the other (serve()).
        self.in_bytes = batch * 3 * h * w * _INPUT_SIZE[input_dtype]
        self.inputs = [self._buf(self.in_bytes) for _ in range(input_slots)]
        self.in_f32 = self.inputs[0]
        self._slot = 0                # the slot the stem reads when ops are issued
        # the image stem reads the NCHW fp32 input directly (tcgen05 kernel, gathered A tile)
        cur, hh, ww, c = self.in_f32, h, w, 3
        act0 = _ACT[net.stem_act]
        pooled = False
        for i, cv in enumerate(net.stem):
            if i == 0 and cv.k <= 8 and cv.groups == 1:
                pool = net.maxpool and len(net.stem) == 1 and self.fuse_stem_pool
                cur, hh, ww, c, pooled = self._stem(cv, weights, hh, ww, act0, pool)
            elif i == 0 and (input_dtype != DTYPE_F32 or input_norm is not None):
                raise ValueError("a 16-bit or unnormalised input needs the image-stem kernel")
            else:
                cur, hh, ww, c = self._conv(cv, weights, cur, hh, ww, c, act0)
        if net.maxpool and not pooled:
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

    def _stem(self, cv: ConvSpec, weights, hh, ww, act, pool: bool = False):
        """First conv on the NCHW image with its BN folded (omCudaStemConvBnActIn), or, with
        `pool` and shapes the fused kernel takes, that conv and the 3x3/2/1 max pool after it in
        one launch (omCudaStemConvBnActPoolIn). Returns (out, h, w, c, pooled)."""
        n, dt = self.batch, self.dtype
        wbuf = self._upload(weights[cv.name + ".weight"])
        g, b_, m, v = (self._upload(a) for a in self._bn_params(weights, cv.bn))
        packed = self._buf(int(lib.omCudaPackedStemWeightElems(cv.cout, cv.cin, cv.k, cv.k,
                                                               cv.stride)) * 2)
        bias = self._buf(cv.cout * 4)
        call("omCudaPackStemWeight", wbuf.ptr, None, g.ptr, b_.ptr, m.ptr, v.ptr, 1e-5, packed.ptr,
             bias.ptr, cv.cout, cv.cin, cv.k, cv.k, cv.stride, dt)
        p = (hh + 2 * cv.pad - cv.k) // cv.stride + 1
        q = (ww + 2 * cv.pad - cv.k) // cv.stride + 1
        pool = pool and bool(lib.omCudaStemPoolSupported(n, cv.cin, hh, ww, cv.cout, cv.k, cv.k,
                                                         cv.stride, cv.pad, dt))
        p2, q2 = ((p - 1) // 2 + 1, (q - 1) // 2 + 1) if pool else (p, q)
        out = self._buf(n * p2 * q2 * cv.cout * 2)
        ws = self._buf(int(lib.omCudaStemWorkspaceBytes(n, cv.cin, hh, ww, cv.k, cv.k, cv.stride,
                                                        cv.pad)))
        esize = _INPUT_SIZE[self.input_dtype]
        for x in self.inputs:
            self._need(x, n * cv.cin * hh * ww * esize)
        # The input pointer is the one op argument looked up when the op is issued: the slot
        # being captured or launched (every other argument is bound here).
        idt = self.input_dtype
        if self.input_norm is not None:
            # normalisation inside the stem's pre-pass (host arrays, copied at each launch)
            nm, ni = self.input_norm
            issue = lambda out=out, ws=ws: call(
                "omCudaStemConvBnActNormIn", self.inputs[self._slot].ptr, idt, nm, ni, ws.ptr,
                packed.ptr, bias.ptr, out.ptr, n, cv.cin, hh, ww, cv.cout, cv.k, cv.k, cv.stride,
                cv.pad, act, dt, int(pool))
        else:
            fn = "omCudaStemConvBnActPoolIn" if pool else "omCudaStemConvBnActIn"
            issue = lambda out=out, ws=ws: call(
                fn, self.inputs[self._slot].ptr, idt, ws.ptr, packed.ptr, bias.ptr, out.ptr, n,
                cv.cin, hh, ww, cv.cout, cv.k, cv.k, cv.stride, cv.pad, act, dt)
        self._op(issue,
            dict(kind="stem", pool=pool, inp=self.in_f32, out=out, w=weights[cv.name + ".weight"],
                 bn=self._bn_params(weights, cv.bn), c=cv.cin, k=cv.cout, ks=cv.k,
                 stride=cv.stride, pad=cv.pad, act=act, h=hh, wd=ww, p=p, q=q, p2=p2, q2=q2))
        self.n_tc_launches += 1
        self.tc_op_index.append(len(self.ops) - 1)
        self.conv_flops += 2 * n * p * q * cv.cout * cv.cin * cv.k * cv.k
        return out, p2, q2, cv.cout, pool

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

    def _pair_ok(self, a: ConvSpec, b: ConvSpec) -> bool:
        return (self.fuse_pairs and a.groups == 1 and b.groups == 1 and b.k == 1 and
                b.stride == 1 and b.pad == 0 and b.cin == a.cout and
                bool(lib.omCudaConvPairSupported(stored_channels(a.cin), a.cout, b.cout,
                                                 self.dtype)))

    def _conv_pair(self, a: ConvSpec, b: ConvSpec, weights, x, hh, ww, act1, act2, residual):
        """Record conv `a` (BN, act1) and the 1x1 conv `b` after it (BN, + residual, act2) as one
        fused launch (omCudaConvPairBnAct)."""
        n, dt = self.batch, self.dtype
        cs_in = stored_channels(a.cin)
        packs = []
        for cv, cin_s in ((a, cs_in), (b, a.cout)):
            wbuf = self._upload(weights[cv.name + ".weight"])
            g, b_, m, v = (self._upload(t) for t in self._bn_params(weights, cv.bn))
            packed = self._buf(int(lib.omCudaPackedConvWeightElems(cv.cout, cv.k, cv.k, cin_s)) * 2)
            bias = self._buf(cv.cout * 4)
            call("omCudaPackConvWeight", wbuf.ptr, None, g.ptr, b_.ptr, m.ptr, v.ptr, 1e-5,
                 packed.ptr, bias.ptr, cv.cout, cv.cin, cv.k, cv.k, cin_s, dt)
            packs.append((packed, bias))
        p = (hh + 2 * a.pad - a.k) // a.stride + 1
        q = (ww + 2 * a.pad - a.k) // a.stride + 1
        obytes = n * p * q * b.cout * 2
        out = self._buf(obytes)
        self._need(x, n * hh * ww * cs_in * 2)
        if residual is not None:
            self._need(residual, obytes)
        (p1, b1), (p2, b2) = packs
        res = residual
        self._op(lambda x=x, out=out, res=res: call(
            "omCudaConvPairBnAct", x.ptr, p1.ptr, b1.ptr, p2.ptr, b2.ptr,
            res.ptr if res is not None else None, out.ptr, n, hh, ww, cs_in, a.cout, b.cout, a.k,
            a.k, a.stride, a.pad, act1, act2, dt),
            dict(kind="pair", inp=x, out=out, res=residual, c=a.cin, cs=cs_in, mid=a.cout,
                 k=b.cout, ks=a.k, stride=a.stride, pad=a.pad, h=hh, wd=ww, p=p, q=q,
                 flops=2 * n * p * q * (a.cout * a.cin * a.k * a.k + b.cout * b.cin)))
        self.n_tc_launches += 1
        self.tc_op_index.append(len(self.ops) - 1)
        self.conv_flops += 2 * n * p * q * (a.cout * a.cin * a.k * a.k + b.cout * b.cin)
        return out, p, q, b.cout

    def _block(self, blk, weights, x, hh, ww, c):
        if blk.kind in ("basic", "bottleneck"):
            shortcut = x
            if blk.downsample is not None:
                shortcut, _, _, _ = self._conv(blk.downsample, weights, x, hh, ww, c, ACT_NONE)
            cur, h2, w2, c2 = x, hh, ww, c
            convs = list(blk.convs)
            i = 0
            while i < len(convs):
                cv = convs[i]
                if (blk.kind == "bottleneck" and i == len(convs) - 2 and
                        self._pair_ok(cv, convs[i + 1])):
                    return self._conv_pair(cv, convs[i + 1], weights, cur, h2, w2, ACT_RELU,
                                           ACT_RELU, shortcut)
                last = i == len(convs) - 1
                cur, h2, w2, c2 = self._conv(cv, weights, cur, h2, w2, c2, ACT_RELU,
                                             residual=shortcut if last else None)
                i += 1
            return cur, h2, w2, c2
        # inverted residual: expand (ReLU6) -> depthwise (ReLU6) -> project (linear) [+ x]
        e, d, pj = blk.convs
        cur, h2, w2, c2 = self._conv(e, weights, x, hh, ww, c, ACT_RELU6)
        cur, h2, w2, c2 = self._conv(d, weights, cur, h2, w2, c2, ACT_RELU6)
        cur, h2, w2, c2 = self._conv(pj, weights, cur, h2, w2, c2, ACT_NONE,
                                     residual=x if blk.residual else None)
        return cur, h2, w2, c2

    # -------------------------------------------------------------- execution
    @property
    def graph(self):
        """The graph of input slot 0 (None before :meth:`capture`)."""
        return self.graphs[0] if self.graphs else None

    def launch(self, slot: int = 0) -> None:
        """Issue the whole forward on input slot `slot` (graph replay when captured) on the
        compute stream."""
        if self.graphs:
            call("omCudaGraphLaunch", self.graphs[slot])
        else:
            self._slot = slot
            for fn in self.ops:
                fn()

    def capture(self) -> None:
        """Capture one CUDA graph per input slot; they differ only in the stem's input."""
        call("omCudaSynchronize")
        for slot in range(len(self.inputs)):
            self._slot = slot
            call("omCudaGraphBeginCapture")
            try:
                for fn in self.ops:
                    fn()
            finally:
                g = ctypes.c_void_p()
                st = lib.omCudaGraphEndCapture(ctypes.byref(g))
            _lib.check(st, "omCudaGraphEndCapture")
            self.graphs.append(g.value)
        self._slot = 0

    def host_input(self, x: np.ndarray) -> np.ndarray:
        """The NCHW image in the plan's input_dtype, as bytes to copy to the device (DTYPE_U8:
        the caller's uint8 samples as they are)."""
        assert x.shape == (self.batch, 3, self.h, self.w)
        if self.input_dtype == DTYPE_U8:
            if x.dtype != np.uint8:
                raise TypeError("an 8-bit plan takes uint8 images")
            return np.ascontiguousarray(x)
        x = np.ascontiguousarray(x, dtype=np.float32)
        if self.input_dtype == DTYPE_F32:
            return x
        if self.input_dtype == DTYPE_F16:
            return x.astype(np.float16)
        return to_bf16_bits(x)

    def set_input(self, x: np.ndarray, slot: int = 0) -> None:
        self.inputs[slot].upload(self.host_input(x))

    def run(self, x: np.ndarray) -> np.ndarray:
        """Host NCHW fp32 input -> host fp32 logits [N, classes]."""
        self.set_input(x)
        self.launch()
        return self.logits.to_numpy((self.batch, self.net.classes))

    def serve(self, host_inputs: Sequence[int], host_outputs: Sequence[int]) -> None:
        """Enqueue len(host_inputs) forwards without waiting: batch i is copied from the pinned
        host buffer host_inputs[i] (NCHW fp32, ``in_bytes``) and its fp32 logits are copied to
        the pinned host buffer host_outputs[i]. Returns once everything is enqueued;
        ``omCudaSynchronize`` waits for it.

        The copy of batch i+1 runs on the transfer stream while batch i's forward runs on the
        compute stream: with two slots, the copy into slot (i+1) % 2 waits only for forward
        i-1, the last one that read that slot. With one slot, copy and forward alternate."""
        n, slots = len(host_inputs), len(self.inputs)
        if len(host_outputs) != n:
            raise ValueError("serve: host_inputs and host_outputs differ in length")
        if n == 0:
            return
        out_bytes = self.batch * self.net.classes * 4
        call("omCudaTransferWaitCompute")     # slot 0 may still be read by earlier work
        call("omCudaTransferH2D", self.inputs[0].ptr, host_inputs[0], self.in_bytes)
        for i in range(n):
            s = i % slots
            call("omCudaComputeWaitTransfer")     # batch i has landed in slot s
            if slots == 2:
                call("omCudaTransferWaitCompute")  # forward i-1 (the other slot's reader) done
            self.launch(s)
            call("omCudaAsyncCopyD2H", host_outputs[i], self.logits.ptr, out_bytes)
            if slots == 1:
                call("omCudaTransferWaitCompute")  # forward i done with the only slot
            if i + 1 < n:
                call("omCudaTransferH2D", self.inputs[(i + 1) % slots].ptr, host_inputs[i + 1],
                     self.in_bytes)

    def close(self) -> None:
        for g in self.graphs:
            lib.omCudaGraphDestroy(g)
        self.graphs = []
        for b in self.keep:
            b.free()
        self.keep.clear()


class Fp32Net:
    """A ResNet (BasicBlock or Bottleneck) in the reference's own layout, NCHW fp32, run through
    the reference-named C-ABI entry points exactly as the engine's tensor_ops / autograd call
    them: train-mode forward (BatchNorm batch statistics, running-stat update), softmax
    cross-entropy on one-hot targets, the backward pass of every node in the reference
    autograd's formulas (autograd.ixx: Conv2dBackward :492-662, BatchNorm2dBackward :722-782,
    MaxPool2dBackward :900-952, ReLUBackward :368, AdaptiveAvgPool2dBackwardFn :1397,
    MatMulBackward :226, AddBiasBackward :399) and SGD with momentum (optimizer.ixx:71-130).

    Gradients live in one flat fp32 buffer in parameter order, so a data-parallel step needs a
    single all-reduce (``grad_flat`` / ``grad_bytes``) between :meth:`backward` and :meth:`step`.
    """

    def __init__(self, net: NetSpec, weights: Dict[str, np.ndarray], batch: int, h: int = 224,
                 w: int = 224, grad_ptr: Optional[int] = None, fused_bn_stats: bool = False,
                 stem_s2d: bool = False):
        self.net, self.batch, self.h, self.w = net, batch, h, w
        # train-mode BatchNorm statistics from the conv epilogue (omCudaConv2dBatchNorm2dAct),
        # and each conv's two backward passes as one call (omCudaConv2dBackwardSplit); False:
        # the reference's order of calls, conv then omCudaBatchNorm2dAct
        self.fused_bn_stats = fused_bn_stats
        # the train-mode image stem in its space-to-depth form (omCudaStemConv2dBatchNorm2dAct,
        # statistics from its epilogue; its input copy kept for the weight gradient). Same
        # results to fp32 rounding in another summation order, so off by default: the order of
        # the plain form is the one the small parity case was pinned with
        self.stem_s2d = stem_s2d
        self.keep: List[DeviceBuffer] = []
        self._guard: Optional[DeviceBuffer] = None  # the gradient guard's status (device)
        self.param = {}
        self.vel = {}
        self.offsets = {}
        off = 0
        for name, shape in net.params:
            n = int(np.prod(shape))
            self.offsets[name] = (off, n, shape)
            off += n
        self.n_params = off
        self.grad_bytes = off * 4
        if grad_ptr is None:
            self._grad_buf = DeviceBuffer.zeros(self.grad_bytes)
            self.keep.append(self._grad_buf)
            grad_ptr = self._grad_buf.ptr
        self.grad_flat = grad_ptr
        # parameters and momentum are flat too (views per tensor), so SGD is one launch
        flat = np.empty(self.n_params, np.float32)
        for name, (off, n, shape) in self.offsets.items():
            flat[off:off + n] = np.asarray(weights[name], np.float32).reshape(-1)
        self.param_flat = self._dev(flat)
        self.vel_flat = self._zeros(self.grad_bytes)
        for name, (off, n, shape) in self.offsets.items():
            self.param[name] = _Ptr(self.param_flat.ptr + off * 4)
            self.vel[name] = _Ptr(self.vel_flat.ptr + off * 4)
        self.buffers = {name: self._dev(weights[name]) for name, _ in net.buffers}
        self.acts = {}
        # called with a parameter's name once the backward pass has issued the last kernel
        # that writes its gradient (a data-parallel wrapper starts bucket all-reduces from it)
        self.grad_hook: Optional[Callable[[str], None]] = None
        self._step_graph: Optional[int] = None   # capture_step's graph

    def _grad_done(self, *names: str) -> None:
        if self.grad_hook is not None:
            for n in names:
                self.grad_hook(n)

    # ------------------------------------------------------------------ memory helpers
    def _dev(self, a: np.ndarray) -> DeviceBuffer:
        b = DeviceBuffer.from_numpy(np.ascontiguousarray(a, dtype=np.float32))
        self.keep.append(b)
        return b

    def _zeros(self, nbytes: int) -> DeviceBuffer:
        b = DeviceBuffer.zeros(nbytes)
        self.keep.append(b)
        return b

    def _buf(self, key, nbytes: int) -> DeviceBuffer:
        """Activation buffers are allocated once per shape role and reused every step."""
        b = self.acts.get(key)
        if b is None or b.nbytes < nbytes:
            b = DeviceBuffer(nbytes)
            self.keep.append(b)
            self.acts[key] = b
        return b

    def grad(self, name: str) -> int:
        off, _, _ = self.offsets[name]
        return self.grad_flat + off * 4

    # ------------------------------------------------------------------ forward pieces
    def _conv_bn(self, key, cv: ConvSpec, x: DeviceBuffer, n, c, hh, ww, relu: bool,
                 train: bool = True, residual: Optional[DeviceBuffer] = None):
        """conv -> BatchNorm (-> ReLU). With residual (train mode, epilogue statistics only): the
        block's last conv, its shortcut add and the block ReLU, y = relu(BN(conv) + residual)
        (omCudaConv2dBatchNorm2dAddAct); the record's relu stays False (the BN backward takes
        no mask of its own: y > 0 is the block ReLU's mask)."""
        p = (hh + 2 * cv.pad - cv.k) // cv.stride + 1
        q = (ww + 2 * cv.pad - cv.k) // cv.stride + 1
        cnt = n * cv.cout * p * q
        z = self._buf(key + ".z", cnt * 4)
        # BN and the ReLU after it in one pass: y is the activated output, and its sign is the
        # ReLU mask the backward needs
        y = self._buf(key + ".y", cnt * 4)
        mean = self._buf(key + ".mean", cv.cout * 4)
        invstd = self._buf(key + ".invstd", cv.cout * 4)
        act = _lib.ACT_RELU if relu else _lib.ACT_NONE
        gamma, beta = self.param[cv.bn + ".gamma"].ptr, self.param[cv.bn + ".beta"].ptr
        rmean = self.buffers[cv.bn + ".running_mean"].ptr
        rvar = self.buffers[cv.bn + ".running_var"].ptr
        xs = None
        nss = (int(lib.omCudaStemInputSplitBytes(n, c, hh, ww, cv.k, cv.k, cv.stride, cv.pad))
               if train and self.stem_s2d else 0)
        if nss > 0:
            xs = self._buf(key + ".xs", nss)
            call("omCudaStemConv2dBatchNorm2dAct", x.ptr, self.param[cv.name + ".weight"].ptr,
                 None, z.ptr, y.ptr, gamma, beta, rmean, rvar, mean.ptr, invstd.ptr, n, c, hh,
                 ww, cv.cout, cv.k, cv.k, cv.stride, cv.pad, 1e-5, 0.1, act, xs.ptr)
        elif train and self.fused_bn_stats:
            # batch statistics from the conv's epilogue (omCudaConv2dBatchNorm2dAct): z is
            # written once and read once; the conv's tensor-core copy of x is kept for the
            # weight gradient (xs), which then does not make it again
            nxs = int(lib.omCudaConvInputSplitBytes(n, c, hh, ww, cv.stride))
            xs = self._buf(key + ".xs", nxs) if nxs > 0 else None
            if residual is not None:
                call("omCudaConv2dBatchNorm2dAddAct", x.ptr, self.param[cv.name + ".weight"].ptr,
                     None, z.ptr, y.ptr, gamma, beta, rmean, rvar, mean.ptr, invstd.ptr, n, c,
                     hh, ww, cv.cout, cv.k, cv.k, cv.stride, cv.pad, 1e-5, 0.1, _lib.ACT_RELU,
                     xs.ptr if xs is not None else None, residual.ptr)
            else:
                call("omCudaConv2dBatchNorm2dAct", x.ptr, self.param[cv.name + ".weight"].ptr,
                     None, z.ptr, y.ptr, gamma, beta, rmean, rvar, mean.ptr, invstd.ptr, n, c,
                     hh, ww, cv.cout, cv.k, cv.k, cv.stride, cv.pad, 1e-5, 0.1, act,
                     xs.ptr if xs is not None else None)
        else:
            B.conv2d(x.ptr, self.param[cv.name + ".weight"].ptr, None, z.ptr, n, c, hh, ww,
                     cv.cout, cv.k, cv.k, cv.pad, cv.pad, cv.stride, cv.stride)
            call("omCudaBatchNorm2dAct", z.ptr, y.ptr, gamma, beta, rmean, rvar, mean.ptr,
                 invstd.ptr, n, cv.cout, p, q, 1e-5, 0.1, int(train), act)
        out = y
        rec = dict(cv=cv, x=x, z=z, y=y, mean=mean, invstd=invstd, relu=relu, n=n, c=c, h=hh,
                   w=ww, p=p, q=q, xs=xs)
        return out, p, q, rec

    def forward_eval(self, x_ptr: int) -> np.ndarray:
        """Eval-mode forward (BatchNorm on the running statistics, which are left unchanged)
        from device NCHW fp32 input; returns the host fp32 logits [N, classes]."""
        self._forward(x_ptr, train=False)
        out = np.empty((self.batch, self.net.classes), np.float32)
        call("omCudaCopyD2H", out.ctypes.data, self.logits.ptr, out.nbytes)
        return out

    def forward_backward(self, x_ptr: int, onehot_ptr: int, loss_ptr: int) -> None:
        """Train-mode forward from device NCHW fp32 input and one-hot targets, loss into
        loss_ptr (device float), gradients into the flat gradient buffer (overwritten)."""
        st = self._forward(x_ptr, train=True)
        self._loss_backward(st, onehot_ptr, loss_ptr)

    def _forward(self, x_ptr: int, train: bool) -> dict:
        """Forward to the logits (self.logits); returns what the backward pass needs."""
        net, n = self.net, self.batch
        recs = []
        x = _Ptr(x_ptr)
        cur, c, hh, ww = x, 3, self.h, self.w
        for i, cv in enumerate(net.stem):
            cur, hh, ww, rec = self._conv_bn(f"stem{i}", cv, cur, n, c, hh, ww, True, train)
            c = cv.cout
            recs.append(rec)
        pool_in, pc, ph, pw = cur, c, hh, ww
        P = (hh + 2 - 3) // 2 + 1
        pooled = self._buf("pool.y", n * c * P * P * 4)
        idx = self._buf("pool.idx", n * c * P * P * 4)
        B.maxPool2d(cur.ptr, pooled.ptr, idx.ptr, n, c, hh, ww, 3, 3, 2, 1)
        cur, hh, ww = pooled, P, P
        blocks = []
        for bi, blk in enumerate(net.blocks):
            inp, ic, ih, iw = cur, c, hh, ww
            sc, ds_rec = inp, None
            if blk.downsample is not None:
                sc, _, _, ds_rec = self._conv_bn(f"b{bi}.ds", blk.downsample, inp, n, ic, ih, iw,
                                                 False, train)
            main = []
            out, oc, oh, ow = inp, ic, ih, iw
            # train mode with epilogue statistics: the shortcut add and the block ReLU ride on
            # the last BatchNorm's normalisation pass
            fuse_add = train and self.fused_bn_stats
            for j, cv in enumerate(blk.convs):
                last = j == len(blk.convs) - 1
                out, oh, ow, rec = self._conv_bn(f"b{bi}.c{j}", cv, out, n, oc, oh, ow, not last,
                                                 train, sc if (last and fuse_add) else None)
                oc = cv.cout
                main.append(rec)
            cnt = n * oc * oh * ow
            if fuse_add:
                s = a = out   # relu(BN + shortcut); a > 0 where the sum was > 0
            else:
                s = self._buf(f"b{bi}.sum", cnt * 4)
                B.add(out.ptr, sc.ptr, s.ptr, cnt)
                a = self._buf(f"b{bi}.out", cnt * 4)
                B.relu(s.ptr, a.ptr, cnt)
            blocks.append(dict(inp=inp, c=ic, h=ih, w=iw, main=main, ds=ds_rec, s=s, oc=oc, oh=oh,
                               ow=ow))
            cur, c, hh, ww = a, oc, oh, ow
        feat = self._buf("feat", n * c * 4)
        B.adaptiveAvgPool2d(cur.ptr, feat.ptr, n, c, hh, ww, 1, 1)
        K = net.classes
        logits = self._buf("logits", n * K * 4)
        B.matmul(feat.ptr, self.param["fc.weight"].ptr, logits.ptr, n, c, K)
        logits_b = self._buf("logits_b", n * K * 4)
        B.addBias(logits.ptr, self.param["fc.bias"].ptr, logits_b.ptr, n, K, 1)
        self.logits = logits_b
        return dict(recs=recs, pool=(pc, ph, pw, P, idx), blocks=blocks, feat=feat, c=c, hh=hh,
                    ww=ww)

    def _loss_backward(self, st: dict, onehot_ptr: int, loss_ptr: int) -> None:
        """Softmax cross-entropy on self.logits, then the backward pass of every node."""
        n, K = self.batch, self.net.classes
        recs, blocks, feat, c, hh, ww = (st[k] for k in ("recs", "blocks", "feat", "c", "hh", "ww"))
        pc, ph, pw, P, idx = st["pool"]
        logits_b = self.logits
        # softmax, loss and the logits' gradient in one pass (omCudaSoftmaxCrossEntropyFused:
        # the reference's softmax, crossEntropy and crossEntropySoftmaxBackward)
        dlog = self._buf("dlogits", n * K * 4)
        call("omCudaSoftmaxCrossEntropyFused", logits_b.ptr, onehot_ptr, None, dlog.ptr,
             loss_ptr, n, K)

        # ---------------------------------------------------------------- backward
        featT = self._buf("featT", n * c * 4)
        B.transpose(feat.ptr, featT.ptr, n, c)
        B.matmul(featT.ptr, dlog.ptr, self.grad("fc.weight"), c, n, K)
        B.addBiasBackward(dlog.ptr, self.grad("fc.bias"), n, K, 1)
        self._grad_done("fc.weight", "fc.bias")
        WT = self._buf("fcWT", c * K * 4)
        B.transpose(self.param["fc.weight"].ptr, WT.ptr, c, K)
        dfeat = self._buf("dfeat", n * c * 4)
        B.matmul(dlog.ptr, WT.ptr, dfeat.ptr, n, K, c)
        dcur = self._buf("dtop", n * c * hh * ww * 4)
        B.adaptiveAvgPool2dBackward(dfeat.ptr, dcur.ptr, n, c, hh, ww, 1, 1)
        for bi in reversed(range(len(blocks))):
            blk = blocks[bi]
            cnt = n * blk["oc"] * blk["oh"] * blk["ow"]
            ds_ = self._buf(f"g{bi}.ds", cnt * 4)
            B.reluBackward(blk["s"].ptr, dcur.ptr, ds_.ptr, cnt)
            d = ds_
            for j in reversed(range(len(blk["main"]))):
                d = self._conv_bn_backward(f"g{bi}.m{j}", blk["main"][j], d)
            if blk["ds"] is not None:
                dsc = self._conv_bn_backward(f"g{bi}.d", blk["ds"], ds_)
            else:
                dsc = ds_
            incnt = n * blk["c"] * blk["h"] * blk["w"]
            dsum = self._buf(f"g{bi}.in", incnt * 4)
            B.add(d.ptr, dsc.ptr, dsum.ptr, incnt)
            dcur = dsum
        dpool = self._buf("g.pool", n * pc * ph * pw * 4)
        # gather form: deterministic, the CPU backend's sums in its order (the reference's GPU
        # path scatters with atomics)
        call("omCudaMaxPool2dBackwardGather", dcur.ptr, idx.ptr, dpool.ptr, n, pc, ph, pw, 3, 3,
             2, 2, 1, 1)
        d = dpool
        for i in reversed(range(len(recs))):
            d = self._conv_bn_backward(f"g.stem{i}", recs[i], d, need_dx=i > 0)

    def _conv_bn_backward(self, key, rec, dout, need_dx: bool = True) -> Optional[DeviceBuffer]:
        cv, n = rec["cv"], rec["n"]
        cnt = n * cv.cout * rec["p"] * rec["q"]
        dz = self._buf(key + ".dz", cnt * 4)
        call("omCudaBatchNorm2dBackwardAct", dout.ptr, rec["z"].ptr, rec["mean"].ptr,
             rec["invstd"].ptr, self.param[cv.bn + ".gamma"].ptr, rec["y"].ptr, dz.ptr,
             self.grad(cv.bn + ".gamma"), self.grad(cv.bn + ".beta"), n, cv.cout, rec["p"],
             rec["q"], 1e-5, _lib.ACT_RELU if rec["relu"] else _lib.ACT_NONE)
        self._grad_done(cv.bn + ".gamma", cv.bn + ".beta")
        dx = None
        if need_dx:  # the image itself needs no gradient
            dx = self._buf(key + ".dx", n * rec["c"] * rec["h"] * rec["w"] * 4)
        if self.fused_bn_stats:
            # both passes in one call, reading one tensor-core copy of dz (bit-identical)
            xs = rec.get("xs")
            call("omCudaConv2dBackwardSplit", dz.ptr, rec["x"].ptr,
                 xs.ptr if xs is not None else None, self.param[cv.name + ".weight"].ptr,
                 dx.ptr if dx is not None else None, self.grad(cv.name + ".weight"), None, n,
                 rec["c"], rec["h"], rec["w"], cv.cout, cv.k, cv.k, cv.stride, cv.pad)
            self._grad_done(cv.name + ".weight")
            return dx
        if need_dx:
            B.conv2dBackwardInput(dz.ptr, self.param[cv.name + ".weight"].ptr, dx.ptr, n, rec["c"],
                                  rec["h"], rec["w"], cv.cout, cv.k, cv.k, cv.pad, cv.pad, cv.stride,
                                  cv.stride)
        if rec.get("xs") is not None:
            # the forward kept the tensor-core copy of x
            call("omCudaConv2dBackwardWeightSplit", rec["x"].ptr, rec["xs"].ptr, dz.ptr,
                 self.grad(cv.name + ".weight"), None, n, rec["c"], rec["h"], rec["w"], cv.cout,
                 cv.k, cv.k, cv.stride, cv.pad)
        else:
            B.conv2dBackwardWeight(rec["x"].ptr, dz.ptr, self.grad(cv.name + ".weight"), None,
                                   n, rec["c"], rec["h"], rec["w"], cv.cout, cv.k, cv.k, cv.pad,
                                   cv.pad, cv.stride, cv.stride)
        self._grad_done(cv.name + ".weight")
        return dx

    def step(self, lr: float = 0.01, momentum: float = 0.9, grad_scale: float = 1.0,
             max_grad_norm: Optional[float] = None, accum_scale: float = 1.0) -> None:
        """SGD with momentum on every parameter; grad_scale (1/world after a summing
        all-reduce) is applied to the flat gradient first.

        With max_grad_norm set, the training loop's gradient guard (EngineBridge.cpp:1885-1925,
        which uses 5.0) runs first, on the device: a NaN/Inf gradient skips the step, a norm
        above max_grad_norm scales the gradient down to it, then accum_scale (1/accumulation
        steps) applies. :meth:`guard_status` reads the verdict back."""
        if max_grad_norm is None:
            # one launch over the flat parameters (elementwise, so the same as one per tensor),
            # with the data-parallel 1/world scale applied inside the update
            if grad_scale != 1.0:
                call("omCudaSgdStepScaled", self.param_flat.ptr, self.grad_flat,
                     self.vel_flat.ptr, self.n_params, lr, momentum, grad_scale)
            else:
                B.sgdStep(self.param_flat.ptr, self.grad_flat, self.vel_flat.ptr, self.n_params,
                          lr, momentum)
            return
        if grad_scale != 1.0:
            B.mulScalar(self.grad_flat, grad_scale, self.grad_flat, self.n_params)
        if self._guard is None:
            self._guard = DeviceBuffer.zeros(16)
            self.keep.append(self._guard)
        call("omCudaGradNormClip", self.grad_flat, self.n_params, max_grad_norm, accum_scale,
             self._guard.ptr)
        call("omCudaSgdStepGuarded", self.param_flat.ptr, self.grad_flat, self.vel_flat.ptr,
             self.n_params, lr, momentum, self._guard.ptr)

    def guard_status(self) -> Tuple[float, bool, float]:
        """(gradient norm, whether the last guarded step ran, clip coefficient)."""
        v = self._guard.to_numpy((4,))
        return float(v[0]), bool(v[1] != 0), float(v[2])

    def read_grads(self) -> Dict[str, np.ndarray]:
        flat = np.empty(self.n_params, np.float32)
        call("omCudaCopyD2H", flat.ctypes.data, self.grad_flat, self.grad_bytes)
        return {name: flat[off:off + n].reshape(shape) for name, (off, n, shape) in self.offsets.items()}

    def read_param(self, name: str) -> np.ndarray:
        off, n, shape = self.offsets[name]
        out = np.empty(n, np.float32)
        call("omCudaCopyD2H", out.ctypes.data, self.param_flat.ptr + off * 4, n * 4)
        return out.reshape(shape)

    def capture_step(self, x_ptr: int, onehot_ptr: int, loss_ptr: int, lr: float = 0.01,
                     momentum: float = 0.9) -> None:
        """Capture one whole training step (forward_backward on these device buffers, then the
        SGD step) as a CUDA graph; :meth:`replay_step` launches it. One rank only: a gradient
        hook (a data-parallel wrapper's bucket all-reduces) must not be set. Run one eager step
        first, so that every activation buffer exists; the graph reads and writes the same
        buffers, and the results are bit-identical to eager steps."""
        if self.grad_hook is not None:
            raise ValueError("capture_step: a gradient hook (collectives) is set")
        if self._step_graph is not None:
            call("omCudaGraphDestroy", self._step_graph)
            self._step_graph = None
        call("omCudaSynchronize")
        call("omCudaGraphBeginCapture")
        try:
            self.forward_backward(x_ptr, onehot_ptr, loss_ptr)
            self.step(lr, momentum)
        finally:
            g = ctypes.c_void_p()
            st = lib.omCudaGraphEndCapture(ctypes.byref(g))
        _lib.check(st, "omCudaGraphEndCapture")
        self._step_graph = g.value

    def replay_step(self) -> None:
        """Launch the captured training step (asynchronous, on the library's stream)."""
        if self._step_graph is None:
            raise RuntimeError("replay_step: no captured step")
        call("omCudaGraphLaunch", self._step_graph)

    def close(self) -> None:
        if self._step_graph is not None:
            call("omCudaGraphDestroy", self._step_graph)
            self._step_graph = None
        for b in self.keep:
            b.free()
        self.keep.clear()


class _Ptr:
    """A borrowed device pointer with the DeviceBuffer interface the plan code uses."""

    def __init__(self, ptr: int):
        self.ptr = int(ptr)
