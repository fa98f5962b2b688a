"""CPU-only: the oracle (oracle/om_oracle.c, the C restatement of the reference CPUBackend) is
pinned against numbers the reference engine itself produced (tests/golden/golden.npz, written
by tests/golden/make_golden.py from oracle/_ref/libomref.so) and against the known-answer values
in the reference's own unit tests.

Tolerances: the oracle sums in double where the reference sums in fp32, so outputs agree to
fp32 rounding: max|a-b|/max|b| <= 1e-5 for single ops and network logits; integer max-pool
indices exactly; the training step's loss to 1e-5; gradient L2 norms with a median relative error
<= 1e-5 over all parameters and every one within 5e-3. The loose bound covers BatchNorm gamma/beta
gradients, which are cancelling sums over N*H*W where the reference's fp32 sums move by up to
~0.4% against the oracle's double sums; conv and FC weight gradients agree to ~1e-5.
"""
import os

import numpy as np
import pytest

from conftest import rel_err

GOLD = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "golden.npz"))
TOL = 1e-5


def _orc():
    import oracle as orc
    return orc


def P(a):
    return a.ctypes.data


@pytest.mark.parametrize("tag", ["a", "b"])
def test_conv_forward_backward(tag):
    O = _orc().O
    n, c, h, k, r, st, pad = (int(v) for v in GOLD[f"conv_{tag}_geom"])
    x, w, b = GOLD[f"conv_{tag}_x"], GOLD[f"conv_{tag}_w"], GOLD[f"conv_{tag}_b"]
    p = (h + 2 * pad - r) // st + 1
    y = np.empty((n, k, p, p), np.float32)
    O.oracle_conv2d(P(x), P(w), P(b), P(y), n, c, h, h, k, r, r, st, pad)
    assert rel_err(y, GOLD[f"conv_{tag}_y"]) <= TOL
    dy = GOLD[f"conv_{tag}_dy"]
    dx = np.empty_like(x)
    O.oracle_conv2d_backward_input(P(dy), P(w), P(dx), n, c, h, h, k, r, r, st, pad)
    assert rel_err(dx, GOLD[f"conv_{tag}_dx"]) <= TOL
    dw, db = np.empty_like(w), np.empty(k, np.float32)
    O.oracle_conv2d_backward_weight(P(x), P(dy), P(dw), P(db), n, c, h, h, k, r, r, st, pad)
    assert rel_err(dw, GOLD[f"conv_{tag}_dw"]) <= TOL
    assert rel_err(db, GOLD[f"conv_{tag}_db"]) <= TOL


def test_depthwise_conv():
    orc = _orc()
    y = orc.conv2d(GOLD["dw_x"], GOLD["dw_w"], None, 2, 1, groups=6)
    assert rel_err(y, GOLD["dw_y"]) <= TOL


@pytest.mark.parametrize("mode", [0, 1])
def test_batchnorm(mode):
    O = _orc().O
    x, gm, bt = GOLD["bn_x"], GOLD["bn_gamma"], GOLD["bn_beta"]
    rm, rv = GOLD[f"bn{mode}_rm_in"].copy(), GOLD[f"bn{mode}_rv_in"].copy()
    y, sm, si = np.empty_like(x), np.empty(5, np.float32), np.empty(5, np.float32)
    O.oracle_batchnorm2d(P(x), P(y), P(gm), P(bt), P(rm), P(rv), P(sm), P(si), 3, 5, 4, 6, 1e-5,
                         0.1, mode)
    for a, key in ((y, "y"), (rm, "rm"), (rv, "rv"), (sm, "sm"), (si, "si")):
        assert rel_err(a, GOLD[f"bn{mode}_{key}"]) <= TOL, key
    if mode == 1:
        dx, dg, db = np.empty_like(x), np.empty(5, np.float32), np.empty(5, np.float32)
        dy = GOLD["bn_dy"]
        O.oracle_batchnorm2d_backward(P(dy), P(x), P(sm), P(si), P(gm), P(dx), P(dg), P(db), 3, 5,
                                      4, 6)
        assert rel_err(dx, GOLD["bn_dx"]) <= TOL
        assert rel_err(dg, GOLD["bn_dg"]) <= TOL
        assert rel_err(db, GOLD["bn_db"]) <= TOL


def test_pooling():
    O = _orc().O
    x = GOLD["pool_x"]
    y, idx = np.empty((2, 3, 5, 5), np.float32), np.empty((2, 3, 5, 5), np.int32)
    O.oracle_maxpool2d(P(x), P(y), P(idx), 2, 3, 9, 9, 3, 2, 1)
    assert np.array_equal(y, GOLD["maxpool_y"])
    assert np.array_equal(idx, GOLD["maxpool_idx"])
    dx = np.empty_like(x)
    dy = GOLD["maxpool_dy"]
    O.oracle_maxpool2d_backward(P(dy), P(idx), P(dx), 2, 3, 5, 5, 9, 9)
    assert rel_err(dx, GOLD["maxpool_dx"]) <= TOL
    ya = np.empty((2, 3, 5, 5), np.float32)
    O.oracle_avgpool2d(P(x), P(ya), 2, 3, 9, 9, 3, 2, 1)
    assert rel_err(ya, GOLD["avgpool_y"]) <= TOL
    yg = np.empty((2, 3, 2, 3), np.float32)
    O.oracle_adaptive_avgpool2d(P(x), P(yg), 2, 3, 9, 9, 2, 3)
    assert rel_err(yg, GOLD["adapool_y"]) <= TOL
    dxg = np.empty_like(x)
    dg = GOLD["adapool_dy"]
    O.oracle_adaptive_avgpool2d_backward(P(dg), P(dxg), 2, 3, 9, 9, 2, 3)
    assert rel_err(dxg, GOLD["adapool_dx"]) <= TOL


def test_elementwise_matmul_softmax_ce():
    O = _orc().O
    a, b = GOLD["ew_a"], GOLD["ew_b"]
    out = np.empty_like(a)
    O.oracle_relu(P(a), P(out), a.size)
    assert np.array_equal(out, GOLD["relu_y"])
    O.oracle_relu_backward(P(a), P(b), P(out), a.size)
    assert np.array_equal(out, GOLD["relu_dx"])
    O.oracle_clip(P(a), P(out), a.size, 0.0, 0.75)
    assert np.array_equal(out, GOLD["clip_y"])
    O.oracle_add(P(a), P(b), P(out), a.size)
    assert np.array_equal(out, GOLD["add_y"])
    A, B = GOLD["mm_a"], GOLD["mm_b"]
    C = np.empty((7, 9), np.float32)
    O.oracle_matmul(P(A), P(B), P(C), 7, 13, 9)
    assert rel_err(C, GOLD["mm_c"]) <= TOL
    Cb = np.empty_like(C)
    bias = GOLD["mm_bias"]
    O.oracle_add_bias(P(C), P(bias), P(Cb), 7, 9)
    assert rel_err(Cb, GOLD["mm_cb"]) <= TOL
    z, oh = GOLD["sm_z"], GOLD["sm_onehot"]
    sp = np.empty_like(z)
    O.oracle_softmax(P(z), P(sp), 4, 11)
    assert rel_err(sp, GOLD["sm_p"]) <= TOL
    ce = O.oracle_cross_entropy(P(sp), P(oh), 4, 11)
    assert abs(ce - GOLD["ce_loss"][0]) <= TOL * abs(GOLD["ce_loss"][0])
    dz = np.empty_like(z)
    O.oracle_ce_softmax_backward(P(sp), P(oh), P(dz), 4, 11)
    assert rel_err(dz, GOLD["ce_dz"]) <= TOL


@pytest.mark.parametrize("name", ["resnet18", "resnet50", "mobilenet"])
def test_network_forward(name):
    orc = _orc()
    from omnimatchdeeplearningtool_b200 import synth
    net = synth.mobilenet_spec(10) if name == "mobilenet" else synth.resnet_spec(int(name[6:]), 10)
    w = synth.make_weights(net)
    x = synth.normal_input(2, 3, 64, 64, seed=5)
    got = orc.forward(net, w, x)
    want = GOLD[f"net_{name}_logits"]
    assert rel_err(got, want) <= TOL
    assert np.array_equal(got.argmax(1), want.argmax(1))


def test_resnet18_training_step():
    orc = _orc()
    from omnimatchdeeplearningtool_b200 import synth
    net = synth.resnet_spec(18, 10)
    w = synth.make_weights(net)
    x = synth.normal_input(4, 3, 64, 64, seed=6)
    y = synth.onehot_labels(4, 10, seed=7)
    loss, grads = orc.train_step(net, w, x, y)
    want_loss = float(GOLD["train_r18_loss"][0])
    assert abs(loss - want_loss) <= TOL * abs(want_loss)
    summ = GOLD["train_r18_grad_summary"]
    errs = []
    for (name, _), sm in zip(net.params, summ):
        g = grads[name].reshape(-1).astype(np.float64)
        norm = np.sqrt((g * g).sum())
        e = abs(norm - sm[1]) / sm[1]
        assert e <= 5e-3, (name, e)
        errs.append(e)
    assert float(np.median(errs)) <= 1e-5


# ---- known-answer values from the reference's own tests ------------------------------------
def test_reference_kat_matmul():
    # tests/test_tensor_ops.cpp:55-82
    O = _orc().O
    for a, b, want, (m, k, n) in (
            ([[1, 2], [3, 4]], [[5, 6], [7, 8]], [[19, 22], [43, 50]], (2, 2, 2)),
            ([[1, 2, 3], [4, 5, 6]], [[7, 8], [9, 10], [11, 12]], [[58, 64], [139, 154]], (2, 3, 2))):
        A, B = np.array(a, np.float32), np.array(b, np.float32)
        C = np.empty((m, n), np.float32)
        O.oracle_matmul(P(A), P(B), P(C), m, k, n)
        assert np.array_equal(C, np.array(want, np.float32))


def test_reference_kat_pooling():
    # tests/test_conv.cpp:72-116: 2x2/2 max pool of 0..15 is 5,7,13,15; avg pool 2.5,4.5,...
    O = _orc().O
    x = np.arange(16, dtype=np.float32).reshape(1, 1, 4, 4)
    y, idx = np.empty((1, 1, 2, 2), np.float32), np.empty((1, 1, 2, 2), np.int32)
    O.oracle_maxpool2d(P(x), P(y), P(idx), 1, 1, 4, 4, 2, 2, 0)
    assert y.reshape(-1).tolist() == [5.0, 7.0, 13.0, 15.0]
    a = np.empty((1, 1, 2, 2), np.float32)
    O.oracle_avgpool2d(P(x), P(a), 1, 1, 4, 4, 2, 2, 0)
    assert abs(a[0, 0, 0, 0] - 2.5) < 1e-5 and abs(a[0, 0, 0, 1] - 4.5) < 1e-5


def test_reference_kat_sgd():
    # tests/test_nn.cpp:70-104: grad 2, lr 0.1, no momentum: 1 -> 0.8
    O = _orc().O
    p = np.ones(6, np.float32)
    g = np.full(6, 2.0, np.float32)
    v = np.zeros(6, np.float32)
    O.oracle_sgd_step(P(p), P(g), P(v), 6, 0.1, 0.0)
    assert np.allclose(p, 0.8, atol=1e-6)


def test_oracle_matches_reference_library_when_built():
    """When the reference engine is built in this checkout, cross-check one fresh case."""
    orc = _orc()
    L = orc.ref()
    if L is None:
        pytest.skip("oracle/_ref/libomref.so not built here")
    rng = np.random.Generator(np.random.PCG64(99))
    x = rng.standard_normal((2, 8, 12, 12)).astype(np.float32)
    w = rng.standard_normal((16, 8, 3, 3)).astype(np.float32)
    y_ref = np.empty((2, 16, 6, 6), np.float32)
    L.omref_conv2d(P(x), P(w), None, P(y_ref), 2, 8, 12, 12, 16, 3, 2, 1)
    assert rel_err(orc.conv2d(x, w, None, 2, 1), y_ref) <= TOL
