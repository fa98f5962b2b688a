"""The reference engine, unchanged, running on the B200 backend.

oracle/_ref/libomengine.so is the reference's own Tensor / tensor_ops / autograd / Module /
SGD / CrossEntropyLoss code compiled with OM_HAS_CUDA against this repository's TensorStorage
(include/om_tensor_storage.hpp), om::CUDABackend (include/om_cuda_backend.hpp) and
libomcuda.so (`make -C oracle engine REF=<reference checkout>`, oracle/engine_shim.cpp). Its
ResNet-18 (ImageNet stem, composed from the reference's modules as in the CPU reference) is
moved to the GPU the way EngineBridge.cpp:915-931 moves a model, then:

  * eval forward: logits within max|a-b|/max|b| <= 1e-4 (fp32 path) of the same engine code on
    its CPU backend (oracle/_ref/libomref.so), identical top-1;
  * one training step (train_main.cpp order: train forward, CrossEntropyLoss, tensorBackward,
    SGD momentum 0.9, lr 0.01): loss within 1e-4; every parameter gradient, measured as
    max|a-b|/max|b| against the oracle's double-precision step, with median <= 1e-4 and
    maximum <= 1e-2 (the fp32 bounds of the backend's own training test); the parameters
    after SGD within 1e-5 of the double-precision update.

The backend's launch counter shows the work ran in libomcuda.so, and the parameters stay on
the device.
"""
import ctypes
import os
from ctypes import POINTER, c_char_p, c_float, c_int, c_void_p

import numpy as np
import pytest

from conftest import ROOT, rel_err

pytestmark = pytest.mark.gpu

ENGINE_SO = os.path.join(ROOT, "oracle", "_ref", "libomengine.so")


def _engine():
    if not os.path.exists(ENGINE_SO):
        pytest.fail(f"{ENGINE_SO} is missing: build it with `make -C oracle engine REF=<dir>`")
    L = ctypes.CDLL(ENGINE_SO)
    P, I, F = c_void_p, c_int, c_float
    sigs = {
        "omeng_init": [I], "omeng_model_create": [I, I], "omeng_model_destroy": [P],
        "omeng_model_num_params": [P], "omeng_model_num_buffers": [P],
        "omeng_model_param_info": [P, I, c_char_p, I, POINTER(c_int)],
        "omeng_model_buffer_info": [P, I, c_char_p, I, POINTER(c_int)],
        "omeng_model_set_param": [P, I, P], "omeng_model_set_buffer": [P, I, P],
        "omeng_model_get_param": [P, I, P], "omeng_model_get_buffer": [P, I, P],
        "omeng_model_param_is_cuda": [P, I], "omeng_model_to_cuda": [P],
        "omeng_model_forward": [P, P, I, I, I, P],
        "omeng_model_train_step": [P, P, P, I, I, I, I, F, F, I, P, P],
    }
    for name, args in sigs.items():
        getattr(L, name).argtypes = args
        getattr(L, name).restype = c_int
    L.omeng_model_create.restype = c_void_p
    L.omeng_last_error.restype = c_char_p
    return L


def _ptr(a):
    return a.ctypes.data_as(c_void_p)


def _model(L, kind, classes, weights):
    """The engine's model with every parameter and buffer loaded by name, then on the GPU."""
    h = L.omeng_model_create(kind, classes)
    buf = ctypes.create_string_buffer(256)
    shp = (c_int * 4)()
    names = []
    keep = []
    for i in range(L.omeng_model_num_params(h)):
        L.omeng_model_param_info(h, i, buf, 256, shp)
        names.append(buf.value.decode())
        keep.append(np.ascontiguousarray(weights[names[-1]], np.float32))
        L.omeng_model_set_param(h, i, _ptr(keep[-1]))
    for i in range(L.omeng_model_num_buffers(h)):
        L.omeng_model_buffer_info(h, i, buf, 256, shp)
        keep.append(np.ascontiguousarray(weights[buf.value.decode()], np.float32))
        L.omeng_model_set_buffer(h, i, _ptr(keep[-1]))
    assert L.omeng_model_to_cuda(h) == 0, L.omeng_last_error()
    assert all(L.omeng_model_param_is_cuda(h, i) == 1 for i in range(len(names)))
    return h, names


def _launches():
    from omnimatchdeeplearningtool_b200._lib import call
    n = ctypes.c_ulonglong()
    call("omCudaGetLaunchCount", ctypes.byref(n))
    return n.value


def test_reference_engine_forward_on_backend(gpu):
    import oracle as orc
    from omnimatchdeeplearningtool_b200 import synth
    L = _engine()
    assert L.omeng_init(0) == 0
    net = synth.resnet_spec(18, 1000)
    w = synth.make_weights(net)
    x = synth.imagenet_input(2, 96, 96)
    h, _ = _model(L, 0, 1000, w)
    logits = np.empty((2, 1000), np.float32)
    before = _launches()
    try:
        assert L.omeng_model_forward(h, _ptr(x), 2, 96, 96, _ptr(logits)) == 0, L.omeng_last_error()
    finally:
        L.omeng_model_destroy(h)
    assert _launches() - before >= 20  # convolutions, BN, pooling, FC: the backend's kernels
    assert gpu.kernel_error() == 0
    # the same engine code on its CPU backend
    rh = orc.ref_model(0, 1000, w, net)
    assert rh is not None, "oracle/_ref/libomref.so is missing"
    want = np.empty((2, 1000), np.float32)
    orc.ref().omref_model_forward(rh, _ptr(x), 2, 96, 96, _ptr(want))
    orc.ref().omref_model_destroy(rh)
    e = rel_err(logits, want)
    print(f"engine on backend, ResNet-18 eval logits: max rel err {e:.2e}")
    assert e <= 1e-4, e
    assert np.array_equal(logits.argmax(1), want.argmax(1))


def test_reference_engine_training_step_on_backend(gpu):
    import oracle as orc
    from omnimatchdeeplearningtool_b200 import synth
    L = _engine()
    assert L.omeng_init(0) == 0
    batch, hw, classes = 4, 64, 10
    net = synth.resnet_spec(18, classes)
    w = synth.make_weights(net)
    x = synth.normal_input(batch, 3, hw, hw, seed=11)
    y = synth.onehot_labels(batch, classes, seed=12)
    h, names = _model(L, 0, classes, w)
    total = sum(int(np.prod(w[n].shape)) for n in names)
    flat = np.empty(total, np.float32)
    loss = np.zeros(1, np.float32)
    try:
        st = L.omeng_model_train_step(h, _ptr(x), _ptr(y), batch, hw, hw, classes, 0.01, 0.9, 1,
                                      _ptr(flat), _ptr(loss))
        assert st == 0, L.omeng_last_error()
        after = {}
        for i, n in enumerate(names):
            a = np.empty(w[n].shape, np.float32)
            assert L.omeng_model_get_param(h, i, _ptr(a)) == 0, L.omeng_last_error()
            after[n] = a
    finally:
        L.omeng_model_destroy(h)
    assert gpu.kernel_error() == 0
    grads, off = {}, 0
    for n in names:
        k = int(np.prod(w[n].shape))
        grads[n] = flat[off:off + k].reshape(w[n].shape)
        off += k
    ow = {k: v.copy() for k, v in w.items()}
    oloss, ograds = orc.train_step(net, ow, x, y, 0.01, 0.9, velocities={})
    assert abs(float(loss[0]) - oloss) <= 1e-4 * abs(oloss), (float(loss[0]), oloss)
    errs = {n: rel_err(grads[n], ograds[n]) for n in names}
    med, mx = float(np.median(list(errs.values()))), max(errs.values())
    print(f"engine on backend, ResNet-18 step: loss err {abs(loss[0] - oloss) / abs(oloss):.2e}, "
          f"gradient error median {med:.2e} max {mx:.2e}")
    assert med <= 1e-4, sorted(errs.items(), key=lambda t: -t[1])[:5]
    assert mx <= 1e-2, sorted(errs.items(), key=lambda t: -t[1])[:5]
    for n in ("fc.weight", "conv1.weight", "layer4.1.conv2.weight"):
        assert rel_err(after[n], ow[n]) <= 1e-5, (n, rel_err(after[n], ow[n]))
