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
    L.oracle_set_num_threads.argtypes = [I]
    L.oracle_set_num_threads.restype = None
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
            "omref_model_save": [P, ctypes.c_char_p, ctypes.c_char_p],
        }
        for n, a in sigs.items():
            f = getattr(L, n)
            f.argtypes = a
        L.omref_set_num_threads.argtypes = [I]
        L.omref_set_num_threads.restype = None
        L.omref_get_max_threads.argtypes = []
        L.omref_get_max_threads.restype = c_int
        L.omref_model_create.restype = c_void_p
        L.omref_cross_entropy.restype = c_float
        L.omref_model_train_step.restype = c_float
        for n in ("omref_model_num_params", "omref_model_num_buffers", "omref_model_param_info",
                  "omref_model_buffer_info", "omref_model_save"):
            getattr(L, n).restype = c_int
        _REF = L
    return _REF


def set_threads(n: int) -> None:
    """OpenMP threads for the oracle and, when built, the reference engine (a process launcher
    such as torchrun may have set OMP_NUM_THREADS=1)."""
    O.oracle_set_num_threads(int(n))
    L = ref()
    if L is not None:
        L.omref_set_num_threads(int(n))


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
    gamma, beta = f32(gamma), f32(beta)
    O.oracle_batchnorm2d(_p(x), _p(out), _p(gamma), _p(beta), _p(rm), _p(rv), _p(sm),
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
    bb = f32(b).reshape(-1)
    O.oracle_add_bias(_p(out), _p(bb), _p(res), out.shape[0], out.shape[1])
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
            sc = f32(sc)
            O.oracle_add(_p(out), _p(sc), _p(s), out.size)
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
        arr = f32(weights[buf.value.decode()])
        L.omref_model_set_param(h, i, _p(arr))
    for i in range(L.omref_model_num_buffers(h)):
        L.omref_model_buffer_info(h, i, buf, 256, shp)
        arr = f32(weights[buf.value.decode()])
        L.omref_model_set_buffer(h, i, _p(arr))
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


# ------------------------------------------------------------------ training step (config 3)
def _bn_train(x, gamma, beta, rm, rv, eps=1e-5, mom=0.1):
    """Train-mode BN (cpu_backend.ixx:781-842); updates rm/rv in place, returns y, mean, invstd."""
    x = f32(x)
    n, c, h, w = x.shape
    y = np.empty_like(x)
    sm, si = np.empty(c, np.float32), np.empty(c, np.float32)
    gamma, beta = f32(gamma), f32(beta)
    O.oracle_batchnorm2d(_p(x), _p(y), _p(gamma), _p(beta), _p(rm), _p(rv), _p(sm),
                         _p(si), n, c, h, w, eps, mom, 1)
    return y, sm, si


def _conv_bwd(x, w, dy, stride, pad):
    x, w, dy = f32(x), f32(w), f32(dy)
    n, c, h, wd = x.shape
    k, _, r, s = w.shape
    dx = np.empty_like(x)
    dw = np.empty_like(w)
    O.oracle_conv2d_backward_input(_p(dy), _p(w), _p(dx), n, c, h, wd, k, r, s, stride, pad)
    O.oracle_conv2d_backward_weight(_p(x), _p(dy), _p(dw), None, n, c, h, wd, k, r, s, stride, pad)
    return dx, dw


def _bn_bwd(dy, x, mean, invstd, gamma):
    dy, x = f32(dy), f32(x)
    n, c, h, w = x.shape
    dx = np.empty_like(x)
    dg, db = np.empty(c, np.float32), np.empty(c, np.float32)
    gamma = f32(gamma)
    O.oracle_batchnorm2d_backward(_p(dy), _p(x), _p(mean), _p(invstd), _p(gamma), _p(dx),
                                  _p(dg), _p(db), n, c, h, w)
    return dx, dg, db


def _relu_bwd(x, dy):
    x, dy = f32(x), f32(dy)
    dx = np.empty_like(x)
    O.oracle_relu_backward(_p(x), _p(dy), _p(dx), x.size)
    return dx


def train_step(net, weights, x, onehot, lr=0.01, momentum=0.9, velocities=None):
    """One reference training step on a BasicBlock/Bottleneck ResNet in NCHW fp32: train-mode
    forward, softmax cross-entropy on one-hot targets (loss.ixx:33-55, tensor_ops.ixx:583-643),
    backward in the reference autograd's formulas (autograd.ixx: Conv2dBackward :492-662,
    BatchNorm2dBackward :722-782, MaxPool2dBackward :900-952, ReLUBackward :368,
    AdaptiveAvgPool2dBackwardFn :1397, MatMulBackward :226, AddBiasBackward :399) and, when
    `velocities` is given, SGD with momentum (optimizer.ixx:103-120).
    Updates BN running statistics in `weights`. Returns (loss, grads)."""
    grads = {}
    rs = {k: f32(v).copy() for k, v in weights.items() if k.endswith("running_mean") or k.endswith("running_var")}
    tape = []

    def conv_bn(cv, inp, act):
        z = conv2d(inp, weights[cv.name + ".weight"], None, cv.stride, cv.pad)
        y, mu, si = _bn_train(z, weights[cv.bn + ".gamma"], weights[cv.bn + ".beta"],
                              rs[cv.bn + ".running_mean"], rs[cv.bn + ".running_var"])
        out = relu(y) if act else y
        tape.append(("conv_bn", cv, inp, z, mu, si, y, act))
        return out

    h = f32(x)
    for cv in net.stem:
        h = conv_bn(cv, h, True)
    pool_in = h
    n, c, hh, ww = h.shape
    P = (hh + 2 - 3) // 2 + 1
    pooled = np.empty((n, c, P, P), np.float32)
    idx = np.empty((n, c, P, P), np.int32)
    O.oracle_maxpool2d(_p(pool_in), _p(pooled), _p(idx), n, c, hh, ww, 3, 2, 1)
    h = pooled
    block_caches = []
    for blk in net.blocks:
        start = len(tape)
        inp = h
        sc = inp
        if blk.downsample is not None:
            sc = conv_bn(blk.downsample, inp, False)
        out = inp
        for i, cv in enumerate(blk.convs):
            out = conv_bn(cv, out, i < len(blk.convs) - 1)
        s = out + sc
        h = relu(s)
        block_caches.append((blk, start, len(tape), inp, s))
    feat_in = h
    n, c, hh, ww = h.shape
    feat = global_avgpool(h).reshape(n, c)
    logits = linear(feat, weights["fc.weight"], weights["fc.bias"])
    p = np.empty_like(logits)
    O.oracle_softmax(_p(logits), _p(p), n, logits.shape[1])
    onehot = f32(onehot)
    loss = O.oracle_cross_entropy(_p(p), _p(onehot), n, logits.shape[1])
    dlogits = np.empty_like(logits)
    O.oracle_ce_softmax_backward(_p(p), _p(onehot), _p(dlogits), n, logits.shape[1])

    # FC: logits = feat @ W + b
    W = f32(weights["fc.weight"])
    dW = np.empty_like(W)
    featT = np.ascontiguousarray(feat.T)   # bound to a name: the C call must see live memory
    O.oracle_matmul(_p(featT), _p(dlogits), _p(dW), W.shape[0], n, W.shape[1])
    db = np.empty(W.shape[1], np.float32)
    O.oracle_add_bias_backward(_p(dlogits), _p(db), n, W.shape[1])
    grads["fc.weight"], grads["fc.bias"] = dW, db.reshape(1, -1)
    dfeat = np.empty((n, W.shape[0]), np.float32)
    WT = np.ascontiguousarray(W.T)
    O.oracle_matmul(_p(dlogits), _p(WT), _p(dfeat), n, W.shape[1], W.shape[0])
    dh = np.empty_like(feat_in)
    dfeat4 = dfeat.reshape(n, c, 1, 1)
    O.oracle_adaptive_avgpool2d_backward(_p(dfeat4), _p(dh), n, c, hh, ww, 1, 1)

    def conv_bn_bwd(entry, dout):
        _, cv, inp, z, mu, si, y, act = entry
        if act:
            dout = _relu_bwd(y, dout)
        dz, dg, dbeta = _bn_bwd(dout, z, mu, si, weights[cv.bn + ".gamma"])
        grads[cv.bn + ".gamma"], grads[cv.bn + ".beta"] = dg, dbeta
        dx, dw = _conv_bwd(inp, weights[cv.name + ".weight"], dz, cv.stride, cv.pad)
        grads[cv.name + ".weight"] = dw
        return dx

    for blk, start, end, inp, s in reversed(block_caches):
        ds = _relu_bwd(s, dh)
        entries = tape[start:end]
        main = [e for e in entries if blk.downsample is None or e[1] is not blk.downsample]
        d = ds
        for e in reversed(main):
            d = conv_bn_bwd(e, d)
        if blk.downsample is not None:
            dsc = conv_bn_bwd([e for e in entries if e[1] is blk.downsample][0], ds)
        else:
            dsc = ds
        dh = d + dsc
    dpool_in = np.empty_like(pool_in)
    n, c, hh, ww = pool_in.shape
    O.oracle_maxpool2d_backward(_p(dh), _p(idx), _p(dpool_in), n, c, P, P, hh, ww)
    d = dpool_in
    for e in reversed(tape[:len(net.stem)]):
        d = conv_bn_bwd(e, d)
    for k, v in rs.items():
        weights[k] = v
    if velocities is not None:
        for name, _ in net.params:
            g = f32(grads[name]).reshape(-1)
            prm = f32(weights[name]).reshape(-1).copy()
            vel = velocities.setdefault(name, np.zeros_like(prm))
            O.oracle_sgd_step(_p(prm), _p(g), _p(vel), prm.size, lr, momentum)
            weights[name] = prm.reshape(weights[name].shape)
    return float(loss), grads
