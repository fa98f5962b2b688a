"""TEST INFRASTRUCTURE ONLY — Python access to the CPU oracle.

* ``O``: the C restatement (oracle/liboracle.so, om_oracle.c) of the reference CPUBackend ops.
* ``ref()``: the reference engine itself (oracle/_ref/libomref.so, built from the reference
  sources by ``make -C oracle ref``), or None when it was not built.
* ``forward()``: eval-mode network forward in NCHW fp32 composed from oracle ops with the
  reference modules' wiring (BasicBlock resnet.ixx:55-80, Bottleneck resnet50.ixx:62-85,
  InvertedResidual mobilenet.ixx:203-225, ReLU6 = relu + clip mobilenet.ixx:27-39).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this module; the
product never imports it.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import c_float, c_int, c_long, c_size_t, c_void_p

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libomref.so")


def _load_oracle():
    if not os.path.exists(ORACLE_SO):
        raise ImportError(f"{ORACLE_SO} missing: run `make -C {HERE}`")
    L = ctypes.CDLL(ORACLE_SO)
    P, I, F, S = c_void_p, c_int, c_float, c_size_t
    sigs = {
        "oracle_conv2d": [P, P, P, P] + [I] * 9,
        "oracle_grouped_conv2d": [P, P, P, P] + [I] * 11,
        "oracle_conv2d_backward_input": [P, P, P] + [I] * 9,
        "oracle_conv2d_backward_weight": [P, P, P, P] + [I] * 9,
        "oracle_batchnorm2d": [P] * 8 + [I] * 4 + [F, F, I],
        "oracle_batchnorm2d_backward": [P] * 8 + [I] * 4,
        "oracle_maxpool2d": [P, P, P] + [I] * 7,
        "oracle_maxpool2d_backward": [P, P, P] + [I] * 6,
        "oracle_avgpool2d": [P, P] + [I] * 7,
        "oracle_avgpool2d_backward": [P, P] + [I] * 7,
        "oracle_adaptive_avgpool2d": [P, P] + [I] * 6,
        "oracle_adaptive_avgpool2d_backward": [P, P] + [I] * 6,
        "oracle_relu": [P, P, S], "oracle_relu_backward": [P, P, P, S],
        "oracle_add": [P, P, P, S], "oracle_clip": [P, P, S, F, F],
        "oracle_matmul": [P, P, P, I, I, I], "oracle_add_bias": [P, P, P, I, I],
        "oracle_add_bias_backward": [P, P, I, I], "oracle_softmax": [P, P, I, I],
        "oracle_cross_entropy": [P, P, I, I],
        "oracle_ce_softmax_backward": [P, P, P, I, I],
        "oracle_sgd_step": [P, P, P, S, F, F],
    }
    for n, a in sigs.items():
        f = getattr(L, n)
        f.argtypes = a
        f.restype = c_float if n == "oracle_cross_entropy" else None
    return L


O = _load_oracle()
_REF = None


def ref():
    """The reference engine's own CPU code, or None when oracle/_ref was not built."""
    global _REF
    if _REF is None and os.path.exists(REF_SO):
        L = ctypes.CDLL(REF_SO)
        P, I, F, Lg = c_void_p, c_int, c_float, c_long
        sigs = {
            "omref_conv2d": [P, P, P, P] + [I] * 8,
            "omref_conv2d_backward_input": [P, P, P] + [I] * 8,
            "omref_conv2d_backward_weight": [P, P, P, P] + [I] * 8,
            "omref_dilated_conv2d": [P, P, P, P] + [I] * 10,
            "omref_batchnorm2d": [P] * 8 + [I] * 4 + [F, F, I],
            "omref_batchnorm2d_backward": [P] * 8 + [I] * 4,
            "omref_maxpool2d": [P, P, P] + [I] * 7,
            "omref_maxpool2d_backward": [P, P, P] + [I] * 6,
            "omref_avgpool2d": [P, P] + [I] * 7,
            "omref_adaptive_avgpool2d": [P, P] + [I] * 6,
            "omref_adaptive_avgpool2d_backward": [P, P] + [I] * 6,
            "omref_relu": [P, P, Lg], "omref_relu_backward": [P, P, P, Lg],
            "omref_add": [P, P, P, Lg], "omref_clip": [P, P, Lg, F, F],
            "omref_matmul": [P, P, P, I, I, I], "omref_add_bias": [P, P, P, I, I],
            "omref_softmax": [P, P, I, I], "omref_cross_entropy": [P, P, I, I],
            "omref_ce_softmax_backward": [P, P, P, I, I],
            "omref_model_create": [I, I], "omref_model_destroy": [P],
            "omref_model_num_params": [P], "omref_model_num_buffers": [P],
            "omref_model_param_info": [P, I, ctypes.c_char_p, I, P],
            "omref_model_buffer_info": [P, I, ctypes.c_char_p, I, P],
            "omref_model_set_param": [P, I, P], "omref_model_get_param": [P, I, P],
            "omref_model_set_buffer": [P, I, P], "omref_model_get_buffer": [P, I, P],
            "omref_model_forward": [P, P, I, I, I, P],
            "omref_model_train_step": [P, P, P, I, I, I, I, F, F, I, P],
        }
        for n, a in sigs.items():
            f = getattr(L, n)
            f.argtypes = a
        L.omref_model_create.restype = c_void_p
        L.omref_cross_entropy.restype = c_float
        L.omref_model_train_step.restype = c_float
        for n in ("omref_model_num_params", "omref_model_num_buffers", "omref_model_param_info",
                  "omref_model_buffer_info"):
            getattr(L, n).restype = c_int
        _REF = L
    return _REF


def _p(a):
    return None if a is None else a.ctypes.data


def f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


# ------------------------------------------------------------------ op helpers (NCHW fp32)
def conv2d(x, w, b=None, stride=1, pad=0, groups=1):
    x, w = f32(x), f32(w)
    n, c, h, wd = x.shape
    k, _, r, s = w.shape
    p, q = (h + 2 * pad - r) // stride + 1, (wd + 2 * pad - s) // stride + 1
    out = np.empty((n, k, p, q), np.float32)
    bb = None if b is None else f32(b)
    if groups == 1:
        O.oracle_conv2d(_p(x), _p(w), _p(bb), _p(out), n, c, h, wd, k, r, s, stride, pad)
    else:
        O.oracle_grouped_conv2d(_p(x), _p(w), _p(bb), _p(out), n, c, h, wd, k, r, s, stride,
                                pad, 1, groups)
    return out


def batchnorm_eval(x, gamma, beta, mean, var, eps=1e-5):
    x = f32(x)
    n, c, h, w = x.shape
    out = np.empty_like(x)
    rm, rv = f32(mean).copy(), f32(var).copy()
    sm, si = np.empty(c, np.float32), np.empty(c, np.float32)
    O.oracle_batchnorm2d(_p(x), _p(out), _p(f32(gamma)), _p(f32(beta)), _p(rm), _p(rv), _p(sm),
                         _p(si), n, c, h, w, eps, 0.1, 0)
    return out


def relu(x):
    x = f32(x)
    out = np.empty_like(x)
    O.oracle_relu(_p(x), _p(out), x.size)
    return out


def relu6(x):
    y = relu(x)
    out = np.empty_like(y)
    O.oracle_clip(_p(y), _p(out), y.size, 0.0, 6.0)
    return out


def maxpool(x, k=3, stride=2, pad=1):
    x = f32(x)
    n, c, h, w = x.shape
    p, q = (h + 2 * pad - k) // stride + 1, (w + 2 * pad - k) // stride + 1
    out = np.empty((n, c, p, q), np.float32)
    idx = np.empty((n, c, p, q), np.int32)
    O.oracle_maxpool2d(_p(x), _p(out), _p(idx), n, c, h, w, k, stride, pad)
    return out


def global_avgpool(x):
    x = f32(x)
    n, c, h, w = x.shape
    out = np.empty((n, c, 1, 1), np.float32)
    O.oracle_adaptive_avgpool2d(_p(x), _p(out), n, c, h, w, 1, 1)
    return out


def linear(x, w, b):
    x, w = f32(x), f32(w)
    out = np.empty((x.shape[0], w.shape[1]), np.float32)
    O.oracle_matmul(_p(x), _p(w), _p(out), x.shape[0], x.shape[1], w.shape[1])
    res = np.empty_like(out)
    O.oracle_add_bias(_p(out), _p(f32(b).reshape(-1)), _p(res), out.shape[0], out.shape[1])
    return res


def _conv_bn(net_w, cv, x, act):
    y = conv2d(x, net_w[cv.name + ".weight"], None, cv.stride, cv.pad, cv.groups)
    y = batchnorm_eval(y, net_w[cv.bn + ".gamma"], net_w[cv.bn + ".beta"],
                       net_w[cv.bn + ".running_mean"], net_w[cv.bn + ".running_var"])
    if act == "relu":
        y = relu(y)
    elif act == "relu6":
        y = relu6(y)
    return y


def forward(net, weights, x):
    """Eval-mode forward of a synth.NetSpec in NCHW fp32; returns logits [N, classes]."""
    y = f32(x)
    for cv in net.stem:
        y = _conv_bn(weights, cv, y, net.stem_act)
    if net.maxpool:
        y = maxpool(y)
    for blk in net.blocks:
        if blk.kind in ("basic", "bottleneck"):
            sc = y
            if blk.downsample is not None:
                sc = _conv_bn(weights, blk.downsample, y, "none")
            out = y
            for i, cv in enumerate(blk.convs):
                out = _conv_bn(weights, cv, out, "none" if i == len(blk.convs) - 1 else "relu")
            s = np.empty_like(out)
            O.oracle_add(_p(out), _p(f32(sc)), _p(s), out.size)
            y = relu(s)
        else:
            e, d, pj = blk.convs
            out = _conv_bn(weights, e, y, "relu6")
            out = _conv_bn(weights, d, out, "relu6")
            out = _conv_bn(weights, pj, out, "none")
            if blk.residual:
                s = np.empty_like(out)
                O.oracle_add(_p(out), _p(y), _p(s), out.size)
                out = s
            y = out
    y = global_avgpool(y).reshape(y.shape[0], -1)
    return linear(y, weights["fc.weight"], weights["fc.bias"])


def ref_model(kind, classes, weights, net):
    """Instantiate the reference model (0 R18, 1 R50, 2 MobileNet stack) and load weights by
    name; returns the handle, or None when the reference library is absent."""
    L = ref()
    if L is None:
        return None
    h = L.omref_model_create(kind, classes)
    buf = ctypes.create_string_buffer(256)
    shp = (c_int * 4)()
    for i in range(L.omref_model_num_params(h)):
        L.omref_model_param_info(h, i, buf, 256, shp)
        L.omref_model_set_param(h, i, _p(f32(weights[buf.value.decode()])))
    for i in range(L.omref_model_num_buffers(h)):
        L.omref_model_buffer_info(h, i, buf, 256, shp)
        L.omref_model_set_buffer(h, i, _p(f32(weights[buf.value.decode()])))
    return h


def ref_names(h):
    L = ref()
    buf = ctypes.create_string_buffer(256)
    shp = (c_int * 4)()
    ps, bs = [], []
    for i in range(L.omref_model_num_params(h)):
        r = L.omref_model_param_info(h, i, buf, 256, shp)
        ps.append((buf.value.decode(), tuple(shp[j] for j in range(r))))
    for i in range(L.omref_model_num_buffers(h)):
        r = L.omref_model_buffer_info(h, i, buf, 256, shp)
        bs.append((buf.value.decode(), tuple(shp[j] for j in range(r))))
    return ps, bs
