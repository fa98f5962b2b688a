"""Parity of the fp32 NCHW entry points (the reference-named C ABI) with the CPU oracle.

Tolerance: the fp32 path's 1e-4, measured as max |a-b| / max |b| over each output tensor
(the oracle sums in double; fp32 accumulation over hundreds of terms puts isolated
near-zero elements further off in element-wise relative terms). Integer outputs (max-pool
argmax indices) and elementwise ops must match exactly.
"""
import ctypes

import numpy as np
import pytest

from conftest import rel_err as rel_err_floor

pytestmark = pytest.mark.gpu
TOL = 1e-4


_KEEP = []  # device buffers stay alive until the test ends (kernels run asynchronously)


@pytest.fixture(autouse=True)
def _release_buffers():
    yield
    _KEEP.clear()


def _dev(a):
    from omnimatchdeeplearningtool_b200.backend import DeviceBuffer
    b = DeviceBuffer.from_numpy(np.ascontiguousarray(a))
    _KEEP.append(b)
    return b


def _out(shape, dtype=np.float32):
    from omnimatchdeeplearningtool_b200.backend import DeviceBuffer
    b = DeviceBuffer.zeros(int(np.prod(shape)) * np.dtype(dtype).itemsize)
    _KEEP.append(b)
    return b


def _rng(seed):
    return np.random.Generator(np.random.PCG64(seed))


CONV = [  # n, c, h, k, r, stride, pad, bias
    (2, 3, 32, 16, 7, 2, 3, True),
    (2, 16, 15, 32, 3, 1, 1, False),
    (3, 32, 14, 24, 3, 2, 1, True),
    (2, 64, 8, 128, 1, 2, 0, False),
    (1, 8, 9, 8, 5, 1, 2, True),
    # the tensor-core (3xTF32) path: several 32-channel k-blocks and 32..128-wide output tiles,
    # partial tiles in both dimensions, stride-2 backward input by output phase
    (4, 64, 28, 128, 3, 1, 1, False),
    (2, 128, 14, 256, 3, 2, 1, True),
    (8, 96, 16, 40, 1, 1, 0, False),
    (2, 256, 7, 512, 3, 1, 1, False),
    # every conv shape of the batch-4, 64x64 ResNet-18 training test (down to 2x2 maps)
    (4, 3, 64, 64, 7, 2, 3, False),
    (4, 64, 16, 64, 3, 1, 1, False),
    (4, 64, 16, 128, 3, 2, 1, False),
    (4, 64, 16, 128, 1, 2, 0, False),
    (4, 128, 8, 256, 3, 2, 1, False),
    (4, 128, 8, 256, 1, 2, 0, False),
    (4, 256, 4, 256, 3, 1, 1, False),
    (4, 256, 4, 512, 3, 2, 1, False),
    (4, 512, 2, 512, 3, 1, 1, False),
    # stride-2 backward input by output phase: odd maps, 1x1 and 2x2 filters, a 3x3 map; a 5x5
    # filter whose phases need different top and left padding takes zero insertion
    (2, 32, 15, 64, 3, 2, 1, False),
    (3, 48, 9, 32, 1, 2, 0, False),
    (2, 32, 12, 32, 2, 2, 0, False),
    (2, 64, 3, 64, 3, 2, 1, False),
    (2, 16, 13, 32, 5, 2, 2, False),
]


@pytest.mark.parametrize("case", CONV)
def test_conv2d_fwd_bwd(gpu, case):
    import oracle as orc
    from omnimatchdeeplearningtool_b200.backend import CUDABackend as B
    n, c, h, k, r, s, p, use_b = case
    rng = _rng(n * 100 + c)
    x = rng.standard_normal((n, c, h, h), dtype=np.float32)
    w = rng.standard_normal((k, c, r, r), dtype=np.float32) * np.float32(np.sqrt(2 / (c * r * r)))
    b = rng.standard_normal(k, dtype=np.float32) if use_b else None
    P = (h + 2 * p - r) // s + 1
    dy = rng.standard_normal((n, k, P, P), dtype=np.float32)
    dX, dW, dDY = _dev(x), _dev(w), _dev(dy)
    dB = _dev(b) if use_b else None
    y = _out((n, k, P, P))
    B.conv2d(dX.ptr, dW.ptr, dB.ptr if dB else None, y.ptr, n, c, h, h, k, r, r, p, p, s, s)
    want = orc.conv2d(x, w, b, s, p)
    assert rel_err_floor(y.to_numpy(want.shape), want) <= TOL
    # backward input
    dx = _out(x.shape)
    B.conv2dBackwardInput(dDY.ptr, dW.ptr, dx.ptr, n, c, h, h, k, r, r, p, p, s, s)
    want_dx = np.empty_like(x)
    orc.O.oracle_conv2d_backward_input(dy.ctypes.data, w.ctypes.data, want_dx.ctypes.data, n, c, h,
                                       h, k, r, r, s, p)
    assert rel_err_floor(dx.to_numpy(x.shape), want_dx) <= TOL
    # backward weight (+ bias)
    dw = _out(w.shape)
    db = _out((k,))
    B.conv2dBackwardWeight(dX.ptr, dDY.ptr, dw.ptr, db.ptr, n, c, h, h, k, r, r, p, p, s, s)
    want_dw = np.empty_like(w)
    want_db = np.empty(k, np.float32)
    orc.O.oracle_conv2d_backward_weight(x.ctypes.data, dy.ctypes.data, want_dw.ctypes.data,
                                        want_db.ctypes.data, n, c, h, h, k, r, r, s, p)
    assert rel_err_floor(dw.to_numpy(w.shape), want_dw) <= TOL
    assert rel_err_floor(db.to_numpy((k,)), want_db) <= TOL


@pytest.mark.parametrize("n,c,h,k,r,pad", [(4, 64, 28, 128, 3, 1), (4, 64, 16, 128, 1, 0),
                                            (2, 32, 15, 64, 3, 1), (2, 3, 32, 16, 7, 3),
                                            (2, 128, 14, 256, 3, 1)])
def test_stride2_backward_input_phases_match_zero_insertion(gpu, n, c, h, k, r, pad):
    """The stride-2 backward input runs one stride-1 convolution per output phase (no inserted
    zeros). It adds the same nonzero products in the same order as the stride-1 backward input
    of the zero-inserted dY, so the two agree bit for bit."""
    from omnimatchdeeplearningtool_b200.backend import CUDABackend as B
    rng = _rng(900 + c + h)
    w = rng.standard_normal((k, c, r, r), dtype=np.float32) * np.float32(np.sqrt(2 / (c * r * r)))
    P = (h + 2 * pad - r) // 2 + 1
    dy = rng.standard_normal((n, k, P, P), dtype=np.float32)
    P1 = h + 2 * pad - r + 1
    dy1 = np.zeros((n, k, P1, P1), np.float32)
    dy1[:, :, 0:2 * P - 1:2, 0:2 * P - 1:2] = dy
    dW = _dev(w)
    dx2, dx1 = _out((n, c, h, h)), _out((n, c, h, h))
    B.conv2dBackwardInput(_dev(dy).ptr, dW.ptr, dx2.ptr, n, c, h, h, k, r, r, pad, pad, 2, 2)
    B.conv2dBackwardInput(_dev(dy1).ptr, dW.ptr, dx1.ptr, n, c, h, h, k, r, r, pad, pad, 1, 1)
    assert np.array_equal(dx2.to_numpy((n, c, h, h)), dx1.to_numpy((n, c, h, h)))
    assert gpu.kernel_error() == 0


def test_grouped_depthwise_conv(gpu):
    import oracle as orc
    from omnimatchdeeplearningtool_b200.backend import CUDABackend as B
    rng = _rng(7)
    n, c, h = 2, 24, 13
    x = rng.standard_normal((n, c, h, h), dtype=np.float32)
    w = rng.standard_normal((c, 1, 3, 3), dtype=np.float32)
    y = _out((n, c, 7, 7))
    B.dilatedConv2d(_dev(x).ptr, _dev(w).ptr, None, y.ptr, n, c, h, h, c, 3, 3, 2, 1, 1, c)
    want = orc.conv2d(x, w, None, 2, 1, groups=c)
    assert rel_err_floor(y.to_numpy(want.shape), want) <= TOL


@pytest.mark.parametrize("n,c,k,h,stride,pad,dil,groups,kh,kw", [
    (2, 32, 48, 20, 1, 1, 1, 1, 3, 3),    # dense, dilation 1: omCudaConv2d's tensor-core path
    (2, 32, 40, 21, 1, 2, 2, 1, 3, 3),    # dilation 2: dilated taps on the tensor-core path
    (2, 16, 24, 19, 2, 2, 2, 1, 3, 3),    # dilation 2, stride 2
    (2, 8, 16, 23, 1, 3, 3, 1, 3, 3),     # dilation 3
    (2, 4, 8, 24, 1, 9, 9, 1, 3, 3),      # dilation 9 (19x19 extent)
    (2, 4, 8, 24, 1, 13, 13, 1, 3, 3),    # dilation 13 (27x27 extent)
    (2, 20, 24, 30, 1, 4, 4, 1, 3, 1),    # non-square 3x1 filter, dilation 4
    (2, 37, 45, 26, 1, 6, 6, 1, 3, 3),    # channels not a multiple of 32 or 8, dilation 6
    (1, 2, 4, 40, 1, 130, 130, 1, 3, 3),  # 261x261 extent: tensor path refuses, direct kernel
    (2, 12, 18, 17, 1, 2, 2, 3, 3, 3),    # grouped, 4 channels per group: the direct kernel
    (2, 64, 96, 18, 1, 1, 1, 2, 3, 3),    # 2 groups of 32 -> 48: one tensor-core conv per group
    (2, 128, 128, 15, 2, 1, 1, 4, 3, 3),  # 4 groups, stride 2, tensor cores
    (2, 96, 64, 17, 1, 2, 2, 4, 3, 3),    # 4 groups of 24 -> 16, dilation 2, tensor cores
    (3, 64, 64, 9, 1, 0, 1, 2, 1, 1)])    # grouped 1x1, tensor cores
def test_dilated_conv_routes(gpu, n, c, k, h, stride, pad, dil, groups, kh, kw):
    """omCudaDilatedConv2d (cuda_kernels.cu:1201) against the oracle's convolution with the
    filter dilated by zero insertion; bias included."""
    import oracle as orc
    from omnimatchdeeplearningtool_b200.backend import CUDABackend as B
    rng = _rng(70 + dil + groups)
    x = rng.standard_normal((n, c, h, h), dtype=np.float32)
    w = rng.standard_normal((k, c // groups, kh, kw), dtype=np.float32)
    b = rng.standard_normal(k).astype(np.float32)
    er, es = kh + (kh - 1) * (dil - 1), kw + (kw - 1) * (dil - 1)
    wd = np.zeros((k, c // groups, er, es), np.float32)
    wd[:, :, ::dil, ::dil] = w
    want = orc.conv2d(x, wd, b, stride, pad, groups=groups)
    y = _out(want.shape)
    B.dilatedConv2d(_dev(x).ptr, _dev(w).ptr, _dev(b).ptr, y.ptr, n, c, h, h, k, kh, kw, stride,
                    pad, dil, groups)
    assert rel_err_floor(y.to_numpy(want.shape), want) <= TOL
    assert gpu.kernel_error() == 0


# shapes: HW = 63 (scalar planes); HW = 256 (4-float vectors, several blocks per channel);
# HW = 49 over 64 images (several short planes per pass of a block); HW = 4 (one vector per plane)
@pytest.mark.parametrize("shape", [(4, 16, 9, 7), (8, 24, 16, 16), (64, 8, 7, 7), (32, 4, 2, 2)])
@pytest.mark.parametrize("training", [0, 1])
def test_batchnorm_fwd_bwd(gpu, training, shape):
    import oracle as orc
    rng = _rng(11 + training)
    n, c, h, w = shape
    x = (rng.standard_normal((n, c, h, w)) * 2 + 0.5).astype(np.float32)
    g = rng.uniform(0.5, 1.5, c).astype(np.float32)
    b = rng.standard_normal(c).astype(np.float32)
    rm = (rng.standard_normal(c) * 0.1).astype(np.float32)
    rv = rng.uniform(0.5, 1.5, c).astype(np.float32)
    dX, dG, dB, dRM, dRV = _dev(x), _dev(g), _dev(b), _dev(rm), _dev(rv)
    y, sm, si = _out(x.shape), _out((c,)), _out((c,))
    from omnimatchdeeplearningtool_b200._lib import call
    call("omCudaBatchNorm2d", dX.ptr, y.ptr, dG.ptr, dB.ptr, dRM.ptr, dRV.ptr, sm.ptr, si.ptr, n,
         c, h, w, 1e-5, 0.1, training)
    wy, wrm, wrv = np.empty_like(x), rm.copy(), rv.copy()
    wsm, wsi = np.empty(c, np.float32), np.empty(c, np.float32)
    orc.O.oracle_batchnorm2d(x.ctypes.data, wy.ctypes.data, g.ctypes.data, b.ctypes.data,
                             wrm.ctypes.data, wrv.ctypes.data, wsm.ctypes.data, wsi.ctypes.data,
                             n, c, h, w, 1e-5, 0.1, training)
    assert rel_err_floor(y.to_numpy(x.shape), wy) <= TOL
    assert rel_err_floor(dRM.to_numpy((c,)), wrm) <= TOL
    assert rel_err_floor(dRV.to_numpy((c,)), wrv) <= TOL
    assert rel_err_floor(si.to_numpy((c,)), wsi) <= TOL
    # backward with the saved statistics
    dy = rng.standard_normal(x.shape).astype(np.float32)
    dx, dg, db = _out(x.shape), _out((c,)), _out((c,))
    call("omCudaBatchNorm2dBackward", _dev(dy).ptr, dX.ptr, sm.ptr, si.ptr, dG.ptr, dx.ptr, dg.ptr,
         db.ptr, n, c, h, w, 1e-5)
    wdx, wdg, wdb = np.empty_like(x), np.empty(c, np.float32), np.empty(c, np.float32)
    orc.O.oracle_batchnorm2d_backward(dy.ctypes.data, x.ctypes.data, wsm.ctypes.data,
                                      wsi.ctypes.data, g.ctypes.data, wdx.ctypes.data,
                                      wdg.ctypes.data, wdb.ctypes.data, n, c, h, w)
    assert rel_err_floor(dg.to_numpy((c,)), wdg) <= TOL
    assert rel_err_floor(db.to_numpy((c,)), wdb) <= TOL
    assert rel_err_floor(dx.to_numpy(x.shape), wdx) <= TOL


@pytest.mark.parametrize("n,c,h,k,r,stride,pad,act", [
    (4, 16, 15, 24, 3, 1, 1, 1),     # 900 pixels: a partial 32-pixel group at the end
    (2, 32, 28, 160, 3, 2, 1, 1),    # several 128-wide output tiles, stride 2
    (8, 64, 14, 64, 1, 1, 0, 0),     # 1x1, no activation
    (2, 3, 64, 64, 7, 2, 3, 1),      # the ImageNet stem shape (3 input channels)
    (4, 64, 56, 64, 3, 1, 1, 1),     # a ResNet-18 layer-1 conv at batch 4 (392 groups/channel)
    (1, 4, 5, 8, 3, 1, 130, 1)])     # padding the tensor path refuses: the separate kernels
def test_conv_batchnorm_stats_in_epilogue(gpu, n, c, h, k, r, stride, pad, act):
    """omCudaConv2dBatchNorm2dAct (BatchNorm statistics from the conv epilogue, combined in a
    fixed order) against omCudaConv2d + omCudaBatchNorm2dAct (two-pass statistics): the conv
    output bit-identical, everything else within the fp32 tolerance; and against the oracle's
    train-mode BatchNorm of the oracle's conv. The input copy it keeps (pInputSplit) gives
    omCudaConv2dBackwardWeightSplit the bits of omCudaConv2dBackwardWeight."""
    from omnimatchdeeplearningtool_b200._lib import lib
    import oracle as orc
    from omnimatchdeeplearningtool_b200._lib import call
    rng = _rng(500 + c + k)
    x = rng.standard_normal((n, c, h, h), dtype=np.float32)
    w = (rng.standard_normal((k, c, r, r)) * np.sqrt(2.0 / (c * r * r))).astype(np.float32)
    g = rng.uniform(0.5, 1.5, k).astype(np.float32)
    b = rng.standard_normal(k).astype(np.float32)
    rm = (rng.standard_normal(k) * 0.1).astype(np.float32)
    rv = rng.uniform(0.5, 1.5, k).astype(np.float32)
    p = (h + 2 * pad - r) // stride + 1
    dx, dw, dg, db = _dev(x), _dev(w), _dev(g), _dev(b)
    res = []
    nxs = int(lib.omCudaConvInputSplitBytes(n, c, h, h, stride))
    xs = _out((max(nxs, 4) // 4,)) if nxs > 0 else None
    for fused in (True, False):
        z, y, sm, si = _out((n, k, p, p)), _out((n, k, p, p)), _out((k,)), _out((k,))
        drm, drv = _dev(rm), _dev(rv)
        if fused:
            call("omCudaConv2dBatchNorm2dAct", dx.ptr, dw.ptr, None, z.ptr, y.ptr, dg.ptr, db.ptr,
                 drm.ptr, drv.ptr, sm.ptr, si.ptr, n, c, h, h, k, r, r, stride, pad, 1e-5, 0.1, act,
                 xs.ptr if xs is not None else None)
        else:
            call("omCudaConv2d", dx.ptr, dw.ptr, None, z.ptr, n, c, h, h, k, r, r, stride, pad)
            call("omCudaBatchNorm2dAct", z.ptr, y.ptr, dg.ptr, db.ptr, drm.ptr, drv.ptr, sm.ptr,
                 si.ptr, n, k, p, p, 1e-5, 0.1, 1, act)
        res.append([t.to_numpy(s) for t, s in ((z, (n, k, p, p)), (y, (n, k, p, p)), (sm, (k,)),
                                                (si, (k,)), (drm, (k,)), (drv, (k,)))])
    fz, fy, fsm, fsi, frm, frv = res[0]
    assert np.array_equal(fz, res[1][0])
    for a, e in zip(res[0][1:], res[1][1:]):
        assert rel_err_floor(a, e) <= 1e-5
    # the oracle: its conv, then its train-mode BatchNorm (+ ReLU)
    zo = orc.conv2d(x, w, None, stride, pad)
    wy, wrm, wrv = np.empty_like(zo), rm.copy(), rv.copy()
    wsm, wsi = np.empty(k, np.float32), np.empty(k, np.float32)
    orc.O.oracle_batchnorm2d(zo.ctypes.data, wy.ctypes.data, g.ctypes.data, b.ctypes.data,
                             wrm.ctypes.data, wrv.ctypes.data, wsm.ctypes.data, wsi.ctypes.data,
                             n, k, p, p, 1e-5, 0.1, 1)
    if act:
        wy = np.maximum(wy, 0)
    assert rel_err_floor(fy, wy) <= TOL
    assert rel_err_floor(fsi, wsi) <= TOL
    assert rel_err_floor(frm, wrm) <= TOL
    assert rel_err_floor(frv, wrv) <= TOL
    # the weight gradient from the kept input copy
    assert (nxs > 0) == (not (stride == 2 and c * 4 <= 32))
    if xs is not None:
        ddy = _dev(rng.standard_normal((n, k, p, p), dtype=np.float32))
        g1, g2 = _out(w.shape), _out(w.shape)
        call("omCudaConv2dBackwardWeight", dx.ptr, ddy.ptr, g1.ptr, None, n, c, h, h, k, r, r,
             stride, pad)
        call("omCudaConv2dBackwardWeightSplit", dx.ptr, xs.ptr, ddy.ptr, g2.ptr, None, n, c, h, h,
             k, r, r, stride, pad)
        assert np.array_equal(g1.to_numpy(w.shape), g2.to_numpy(w.shape))
    assert gpu.kernel_error() == 0


@pytest.mark.parametrize("n,c,h,k,r,pad,act", [
    (2, 3, 64, 64, 7, 3, 1),      # the ImageNet stem, small image
    (4, 3, 224, 64, 7, 3, 1),     # the ImageNet stem at 224x224 (P = 112)
    (2, 3, 30, 64, 7, 3, 0),      # 15x15 output, no activation
    (2, 8, 33, 32, 3, 1, 1),      # 8 channels (all 32 space-to-depth channels), odd image
    (3, 1, 17, 16, 5, 2, 1),      # one channel, 5x5 filter
    (1, 8, 776, 8, 3, 1, 1)])     # rows too wide for the row-staged copy: the per-element kernel
def test_stem_conv_batchnorm_space_to_depth(gpu, n, c, h, k, r, pad, act):
    """omCudaStemConv2dBatchNorm2dAct (the stride-2 stem in its space-to-depth form) against
    omCudaConv2dBatchNorm2dAct (the plain form; same results up to fp32 rounding in another
    summation order) and against the oracle's conv + train-mode BatchNorm; the space-to-depth
    copy it keeps gives omCudaConv2dBackwardWeightSplit the bits of omCudaConv2dBackwardWeight.
    Shapes outside its scope get OM_ERR_UNSUPPORTED and no copy size."""
    from omnimatchdeeplearningtool_b200._lib import lib, call
    import oracle as orc
    stride = 2
    rng = _rng(700 + c + k + h)
    x = rng.standard_normal((n, c, h, h), dtype=np.float32)
    w = (rng.standard_normal((k, c, r, r)) * np.sqrt(2.0 / (c * r * r))).astype(np.float32)
    g = rng.uniform(0.5, 1.5, k).astype(np.float32)
    b = rng.standard_normal(k).astype(np.float32)
    rm = (rng.standard_normal(k) * 0.1).astype(np.float32)
    rv = rng.uniform(0.5, 1.5, k).astype(np.float32)
    p = (h + 2 * pad - r) // stride + 1
    dx, dw, dg, db = _dev(x), _dev(w), _dev(g), _dev(b)
    nxs = int(lib.omCudaStemInputSplitBytes(n, c, h, h, r, r, stride, pad))
    hs = p + (r + 1) // 2 - 1
    half = (n * hs * hs * 32 * 4 + 255) // 256 * 256
    assert nxs == 2 * half
    xs = _out((nxs // 4,))
    res = []
    for s2d in (True, False):
        z, y, sm, si = _out((n, k, p, p)), _out((n, k, p, p)), _out((k,)), _out((k,))
        drm, drv = _dev(rm), _dev(rv)
        fn = "omCudaStemConv2dBatchNorm2dAct" if s2d else "omCudaConv2dBatchNorm2dAct"
        call(fn, dx.ptr, dw.ptr, None, z.ptr, y.ptr, dg.ptr, db.ptr, drm.ptr, drv.ptr, sm.ptr,
             si.ptr, n, c, h, h, k, r, r, stride, pad, 1e-5, 0.1, act, xs.ptr if s2d else None)
        res.append([t.to_numpy(s) for t, s in ((z, (n, k, p, p)), (y, (n, k, p, p)), (sm, (k,)),
                                                (si, (k,)), (drm, (k,)), (drv, (k,)))])
    for a, e in zip(res[0], res[1]):
        assert rel_err_floor(a, e) <= 1e-5
    fz, fy, fsm, fsi, frm, frv = res[0]
    zo = orc.conv2d(x, w, None, stride, pad)
    assert rel_err_floor(fz, zo) <= TOL
    wy, wrm, wrv = np.empty_like(zo), rm.copy(), rv.copy()
    wsm, wsi = np.empty(k, np.float32), np.empty(k, np.float32)
    orc.O.oracle_batchnorm2d(zo.ctypes.data, wy.ctypes.data, g.ctypes.data, b.ctypes.data,
                             wrm.ctypes.data, wrv.ctypes.data, wsm.ctypes.data, wsi.ctypes.data,
                             n, k, p, p, 1e-5, 0.1, 1)
    if act:
        wy = np.maximum(wy, 0)
    assert rel_err_floor(fy, wy) <= TOL
    assert rel_err_floor(fsi, wsi) <= TOL
    assert rel_err_floor(frm, wrm) <= TOL
    assert rel_err_floor(frv, wrv) <= TOL
    ddy = _dev(rng.standard_normal((n, k, p, p), dtype=np.float32))
    g1, g2 = _out(w.shape), _out(w.shape)
    call("omCudaConv2dBackwardWeight", dx.ptr, ddy.ptr, g1.ptr, None, n, c, h, h, k, r, r,
         stride, pad)
    call("omCudaConv2dBackwardWeightSplit", dx.ptr, xs.ptr, ddy.ptr, g2.ptr, None, n, c, h, h, k,
         r, r, stride, pad)
    assert np.array_equal(g1.to_numpy(w.shape), g2.to_numpy(w.shape))
    assert gpu.kernel_error() == 0
    # outside the space-to-depth scope: stride 1, or more than 8 input channels
    assert lib.omCudaStemInputSplitBytes(n, c, h, h, r, r, 1, pad) == 0
    assert lib.omCudaStemInputSplitBytes(n, 9, h, h, r, r, 2, pad) == 0
    z = _out((n, k, h, h))
    st = lib.omCudaStemConv2dBatchNorm2dAct(dx.ptr, dw.ptr, None, z.ptr, z.ptr, dg.ptr, db.ptr,
                                            drm.ptr, drv.ptr, sm.ptr, si.ptr, n, c, h, h, k, r,
                                            r, 1, (r - 1) // 2, 1e-5, 0.1, act, None)
    assert st == -3


@pytest.mark.parametrize("n,c,h,k,r,stride,pad,act", [
    (4, 64, 28, 64, 3, 1, 1, 1),      # a ResNet-18 block's last conv (4-float path)
    (2, 32, 15, 48, 3, 1, 1, 1),      # odd map: the scalar path
    (2, 64, 14, 128, 1, 1, 0, 0),     # no activation
    (1, 4, 5, 8, 3, 1, 130, 1)])      # padding the tensor path refuses: the separate kernels
def test_conv_batchnorm_residual_relu_matches_separate(gpu, n, c, h, k, r, stride, pad, act):
    """omCudaConv2dBatchNorm2dAddAct (a block's last conv + BN, the shortcut add and the block
    ReLU in the normalisation pass) gives the bits of omCudaConv2dBatchNorm2dAct (no
    activation), omCudaAdd and omCudaReLU."""
    from omnimatchdeeplearningtool_b200._lib import call
    rng = _rng(1300 + c + h)
    x = rng.standard_normal((n, c, h, h), dtype=np.float32)
    w = (rng.standard_normal((k, c, r, r)) * np.sqrt(2.0 / (c * r * r))).astype(np.float32)
    g = rng.uniform(0.5, 1.5, k).astype(np.float32)
    b = rng.standard_normal(k).astype(np.float32)
    p = (h + 2 * pad - r) // stride + 1
    res = rng.standard_normal((n, k, p, p), dtype=np.float32)
    dx, dw, dg, db, dres = _dev(x), _dev(w), _dev(g), _dev(b), _dev(res)
    outs = []
    for fused in (True, False):
        z, y, sm, si = _out((n, k, p, p)), _out((n, k, p, p)), _out((k,)), _out((k,))
        rm, rv = _dev(np.zeros(k, np.float32)), _dev(np.ones(k, np.float32))
        if fused:
            call("omCudaConv2dBatchNorm2dAddAct", dx.ptr, dw.ptr, None, z.ptr, y.ptr, dg.ptr,
                 db.ptr, rm.ptr, rv.ptr, sm.ptr, si.ptr, n, c, h, h, k, r, r, stride, pad, 1e-5,
                 0.1, act, None, dres.ptr)
        else:
            call("omCudaConv2dBatchNorm2dAct", dx.ptr, dw.ptr, None, z.ptr, y.ptr, dg.ptr, db.ptr,
                 rm.ptr, rv.ptr, sm.ptr, si.ptr, n, c, h, h, k, r, r, stride, pad, 1e-5, 0.1, 0,
                 None)
            call("omCudaAdd", y.ptr, dres.ptr, y.ptr, n * k * p * p)
            if act:
                call("omCudaReLU", y.ptr, y.ptr, n * k * p * p)
        outs.append([t.to_numpy(sh) for t, sh in ((z, (n, k, p, p)), (y, (n, k, p, p)),
                                                   (sm, (k,)), (si, (k,)), (rm, (k,)), (rv, (k,)))])
    for a, e in zip(outs[0], outs[1]):
        assert np.array_equal(a, e)
    assert gpu.kernel_error() == 0


@pytest.mark.parametrize("n,c,h,k,r,stride,pad,with_dx", [
    (4, 64, 28, 64, 3, 1, 1, True),     # stride 1: the rotated filter over the shared copy
    (4, 64, 14, 128, 3, 2, 1, True),    # stride 2 by output phase over the shared copy
    (4, 64, 14, 128, 1, 2, 0, True),    # 1x1 stride 2 (memset + one phase)
    (2, 96, 9, 40, 1, 1, 0, True),      # 1x1 stride 1, channels not a multiple of 32
    (2, 32, 11, 48, 3, 1, 2, True),     # pad > R-1: the backward input makes its own copy
    (2, 3, 64, 64, 7, 2, 3, False)])    # the stem: no dX, space-to-depth weight gradient
def test_conv_backward_one_dy_copy_matches_separate(gpu, n, c, h, k, r, stride, pad, with_dx):
    """omCudaConv2dBackwardSplit (one tensor-core copy of dY for the backward-input and the
    weight-gradient passes, the input's kept copy from the forward) gives the bits of
    omCudaConv2dBackwardInput + omCudaConv2dBackwardWeight (+ bias gradient)."""
    from omnimatchdeeplearningtool_b200._lib import lib, call
    rng = _rng(1100 + c + h)
    x = rng.standard_normal((n, c, h, h), dtype=np.float32)
    w = (rng.standard_normal((k, c, r, r)) * np.sqrt(2.0 / (c * r * r))).astype(np.float32)
    p = (h + 2 * pad - r) // stride + 1
    dy = rng.standard_normal((n, k, p, p), dtype=np.float32)
    dx_, dw_, ddy = _dev(x), _dev(w), _dev(dy)
    # the kept input copy, written by the forward
    stem = stride == 2 and c * 4 <= 32
    nxs = int(lib.omCudaStemInputSplitBytes(n, c, h, h, r, r, stride, pad) if stem
              else lib.omCudaConvInputSplitBytes(n, c, h, h, stride))
    xs = _out((nxs // 4,)) if nxs > 0 else None
    if xs is not None:
        g, b = _dev(np.ones(k, np.float32)), _dev(np.zeros(k, np.float32))
        z, y, sm, si = _out((n, k, p, p)), _out((n, k, p, p)), _out((k,)), _out((k,))
        rm, rv = _dev(np.zeros(k, np.float32)), _dev(np.ones(k, np.float32))
        call("omCudaStemConv2dBatchNorm2dAct" if stem else "omCudaConv2dBatchNorm2dAct",
             dx_.ptr, dw_.ptr, None, z.ptr, y.ptr, g.ptr, b.ptr, rm.ptr, rv.ptr, sm.ptr, si.ptr,
             n, c, h, h, k, r, r, stride, pad, 1e-5, 0.1, 1, xs.ptr)
    dx1, dw1, db1 = _out(x.shape), _out(w.shape), _out((k,))
    dx2, dw2, db2 = _out(x.shape), _out(w.shape), _out((k,))
    if with_dx:
        call("omCudaConv2dBackwardInput", ddy.ptr, dw_.ptr, dx1.ptr, n, c, h, h, k, r, r, stride,
             pad)
    call("omCudaConv2dBackwardWeight", dx_.ptr, ddy.ptr, dw1.ptr, db1.ptr, n, c, h, h, k, r, r,
         stride, pad)
    call("omCudaConv2dBackwardSplit", ddy.ptr, dx_.ptr, xs.ptr if xs is not None else None,
         dw_.ptr, dx2.ptr if with_dx else None, dw2.ptr, db2.ptr, n, c, h, h, k, r, r, stride,
         pad)
    if with_dx:
        assert np.array_equal(dx1.to_numpy(x.shape), dx2.to_numpy(x.shape))
    assert np.array_equal(dw1.to_numpy(w.shape), dw2.to_numpy(w.shape))
    assert np.array_equal(db1.to_numpy((k,)), db2.to_numpy((k,)))
    assert gpu.kernel_error() == 0


@pytest.mark.parametrize("shape", [(8, 24, 16, 16), (4, 16, 9, 7)])
def test_batchnorm_relu_fused_matches_separate(gpu, shape):
    """omCudaBatchNorm2dAct / omCudaBatchNorm2dBackwardAct give the bits of omCudaBatchNorm2d +
    omCudaReLU and omCudaReLUBackward + omCudaBatchNorm2dBackward (4-float and scalar paths)."""
    from omnimatchdeeplearningtool_b200 import _lib
    from omnimatchdeeplearningtool_b200._lib import call
    rng = _rng(21)
    n, c, h, w = shape
    x = rng.standard_normal((n, c, h, w)).astype(np.float32)
    g = rng.uniform(0.5, 1.5, c).astype(np.float32)
    b = rng.standard_normal(c).astype(np.float32)
    dy = rng.standard_normal(x.shape).astype(np.float32)
    outs = []
    for fused in (False, True):
        dX, dG, dB = _dev(x), _dev(g), _dev(b)
        rm, rv = _dev(np.zeros(c, np.float32)), _dev(np.ones(c, np.float32))
        y, sm, si = _out(x.shape), _out((c,)), _out((c,))
        dx, dg, db = _out(x.shape), _out((c,)), _out((c,))
        if fused:
            call("omCudaBatchNorm2dAct", dX.ptr, y.ptr, dG.ptr, dB.ptr, rm.ptr, rv.ptr, sm.ptr,
                 si.ptr, n, c, h, w, 1e-5, 0.1, 1, _lib.ACT_RELU)
            call("omCudaBatchNorm2dBackwardAct", _dev(dy).ptr, dX.ptr, sm.ptr, si.ptr, dG.ptr,
                 y.ptr, dx.ptr, dg.ptr, db.ptr, n, c, h, w, 1e-5, _lib.ACT_RELU)
        else:
            pre = _out(x.shape)
            call("omCudaBatchNorm2d", dX.ptr, pre.ptr, dG.ptr, dB.ptr, rm.ptr, rv.ptr, sm.ptr,
                 si.ptr, n, c, h, w, 1e-5, 0.1, 1)
            call("omCudaReLU", pre.ptr, y.ptr, x.size)
            dr = _out(x.shape)
            call("omCudaReLUBackward", pre.ptr, _dev(dy).ptr, dr.ptr, x.size)
            call("omCudaBatchNorm2dBackward", dr.ptr, dX.ptr, sm.ptr, si.ptr, dG.ptr, dx.ptr,
                 dg.ptr, db.ptr, n, c, h, w, 1e-5)
        outs.append([a.to_numpy(s_) for a, s_ in ((y, x.shape), (dx, x.shape), (dg, (c,)),
                                                   (db, (c,)), (rv, (c,)))])
    for a, b_ in zip(*outs):
        assert np.array_equal(a, b_)


@pytest.mark.parametrize("n,c,h,k,st,pad", [(2, 8, 17, 3, 2, 1), (2, 4, 16, 3, 2, 1),
                                          (1, 6, 9, 3, 1, 1), (2, 3, 10, 2, 2, 0)])
def test_maxpool_backward_gather_bit_exact(gpu, n, c, h, k, st, pad):
    """omCudaMaxPool2dBackwardGather (the 2x2-block kernel for 3x3 / 2 / 1, the generic one
    otherwise) against the oracle's sequential loop, bit for bit."""
    import oracle as orc
    from omnimatchdeeplearningtool_b200._lib import call
    from omnimatchdeeplearningtool_b200.backend import CUDABackend as B
    rng = _rng(40 + h + k)
    # few distinct values, so windows often share their maximum
    x = rng.integers(0, 6, (n, c, h, h)).astype(np.float32)
    P = (h + 2 * pad - k) // st + 1
    y, idx = _out((n, c, P, P)), _out((n, c, P, P), np.int32)
    B.maxPool2d(_dev(x).ptr, y.ptr, idx.ptr, n, c, h, h, k, k, st, pad)
    wy, widx = np.empty((n, c, P, P), np.float32), np.empty((n, c, P, P), np.int32)
    orc.O.oracle_maxpool2d(x.ctypes.data, wy.ctypes.data, widx.ctypes.data, n, c, h, h, k, st, pad)
    assert np.array_equal(idx.to_numpy(widx.shape, np.int32), widx)
    dy = rng.standard_normal(wy.shape, dtype=np.float32)
    gdx = _out(x.shape)
    call("omCudaMaxPool2dBackwardGather", _dev(dy).ptr, idx.ptr, gdx.ptr, n, c, h, h, k, k, st, st,
         pad, pad)
    wdx = np.empty_like(x)
    orc.O.oracle_maxpool2d_backward(dy.ctypes.data, widx.ctypes.data, wdx.ctypes.data, n, c, P, P,
                                    h, h)
    assert np.array_equal(gdx.to_numpy(x.shape), wdx)


def test_pooling(gpu):
    import oracle as orc
    from omnimatchdeeplearningtool_b200.backend import CUDABackend as B
    rng = _rng(5)
    n, c, h = 2, 8, 17
    x = rng.standard_normal((n, c, h, h), dtype=np.float32)
    dX = _dev(x)
    P = (h + 2 - 3) // 2 + 1
    y, idx = _out((n, c, P, P)), _out((n, c, P, P), np.int32)
    B.maxPool2d(dX.ptr, y.ptr, idx.ptr, n, c, h, h, 3, 3, 2, 1)
    wy, widx = np.empty((n, c, P, P), np.float32), np.empty((n, c, P, P), np.int32)
    orc.O.oracle_maxpool2d(x.ctypes.data, wy.ctypes.data, widx.ctypes.data, n, c, h, h, 3, 2, 1)
    assert np.array_equal(y.to_numpy(wy.shape), wy)
    assert np.array_equal(idx.to_numpy(widx.shape, np.int32), widx)
    dy = rng.standard_normal(wy.shape, dtype=np.float32)
    dx = _out(x.shape)
    B.maxPool2dBackward(_dev(dy).ptr, idx.ptr, dx.ptr, n, c, h, h, P, P)
    wdx = np.empty_like(x)
    orc.O.oracle_maxpool2d_backward(dy.ctypes.data, widx.ctypes.data, wdx.ctypes.data, n, c, P, P, h, h)
    assert rel_err_floor(dx.to_numpy(x.shape), wdx) <= TOL
    # the gather form: the oracle's sums in the oracle's order, bit for bit
    from omnimatchdeeplearningtool_b200._lib import call
    gdx = _out(x.shape)
    call("omCudaMaxPool2dBackwardGather", _dev(dy).ptr, idx.ptr, gdx.ptr, n, c, h, h, 3, 3, 2, 2,
         1, 1)
    assert np.array_equal(gdx.to_numpy(x.shape), wdx)
    # average pool 3/2/1 and its backward
    ay = _out((n, c, P, P))
    B.avgPool2d(dX.ptr, ay.ptr, n, c, h, h, 3, 3, 2, 1)
    way = np.empty((n, c, P, P), np.float32)
    orc.O.oracle_avgpool2d(x.ctypes.data, way.ctypes.data, n, c, h, h, 3, 2, 1)
    assert rel_err_floor(ay.to_numpy(way.shape), way) <= TOL
    adx = _out(x.shape)
    B.avgPool2dBackward(_dev(dy).ptr, adx.ptr, n, c, h, h, 3, 3, 2, 1)
    wadx = np.empty_like(x)
    orc.O.oracle_avgpool2d_backward(dy.ctypes.data, wadx.ctypes.data, n, c, h, h, 3, 2, 1)
    assert rel_err_floor(adx.to_numpy(x.shape), wadx) <= TOL
    # adaptive average pool to 1x1 and 3x2
    for oh, ow in ((1, 1), (3, 2)):
        g = _out((n, c, oh, ow))
        B.adaptiveAvgPool2d(dX.ptr, g.ptr, n, c, h, h, oh, ow)
        wg = np.empty((n, c, oh, ow), np.float32)
        orc.O.oracle_adaptive_avgpool2d(x.ctypes.data, wg.ctypes.data, n, c, h, h, oh, ow)
        assert rel_err_floor(g.to_numpy(wg.shape), wg) <= TOL
        gd = rng.standard_normal(wg.shape, dtype=np.float32)
        gx = _out(x.shape)
        B.adaptiveAvgPool2dBackward(_dev(gd).ptr, gx.ptr, n, c, h, h, oh, ow)
        wgx = np.empty_like(x)
        orc.O.oracle_adaptive_avgpool2d_backward(gd.ctypes.data, wgx.ctypes.data, n, c, h, h, oh, ow)
        assert rel_err_floor(gx.to_numpy(x.shape), wgx) <= TOL


def test_softmax_ce_sgd_matmul(gpu):
    import oracle as orc
    from omnimatchdeeplearningtool_b200.backend import CUDABackend as B
    rng = _rng(9)
    n, k = 8, 1000
    logits = (rng.standard_normal((n, k)) * 3).astype(np.float32)
    oh = np.zeros((n, k), np.float32)
    oh[np.arange(n), rng.integers(0, k, n)] = 1
    dL, dT = _dev(logits), _dev(oh)
    p = _out((n, k))
    B.softmax(dL.ptr, p.ptr, n, k)
    wp = np.empty_like(logits)
    orc.O.oracle_softmax(logits.ctypes.data, wp.ctypes.data, n, k)
    assert rel_err_floor(p.to_numpy((n, k)), wp) <= TOL
    loss = _out((1,))
    B.crossEntropyForward(p.ptr, dT.ptr, loss.ptr, n, k)
    wl = orc.O.oracle_cross_entropy(wp.ctypes.data, oh.ctypes.data, n, k)
    assert abs(loss.to_numpy((1,))[0] - wl) <= TOL * abs(wl)
    g = _out((n, k))
    B.crossEntropySoftmaxBackward(p.ptr, dT.ptr, g.ptr, n, k)
    wg = np.empty_like(logits)
    orc.O.oracle_ce_softmax_backward(wp.ctypes.data, oh.ctypes.data, wg.ctypes.data, n, k)
    assert rel_err_floor(g.to_numpy((n, k)), wg) <= TOL
    # SGD with momentum, two steps (test_nn.cpp:70-104 pins 1 - 0.1*2 = 0.8 for one plain step)
    prm = rng.standard_normal(1000).astype(np.float32)
    grd = rng.standard_normal(1000).astype(np.float32)
    vel = np.zeros(1000, np.float32)
    dP, dG, dV = _dev(prm), _dev(grd), _dev(vel)
    wprm, wvel = prm.copy(), vel.copy()
    for _ in range(2):
        B.sgdStep(dP.ptr, dG.ptr, dV.ptr, 1000, 0.01, 0.9)
        orc.O.oracle_sgd_step(wprm.ctypes.data, grd.ctypes.data, wvel.ctypes.data, 1000, 0.01, 0.9)
    assert rel_err_floor(dP.to_numpy((1000,)), wprm) <= TOL
    one = _dev(np.array([1.0], np.float32))
    B.sgdStep(one.ptr, _dev(np.array([2.0], np.float32)).ptr, None, 1, 0.1, 0.0)
    assert abs(one.to_numpy((1,))[0] - 0.8) < 1e-7
    # matmul, including the reference KATs (test_tensor_ops.cpp:55-82)
    a = rng.standard_normal((37, 70)).astype(np.float32)
    bm = rng.standard_normal((70, 45)).astype(np.float32)
    c = _out((37, 45))
    B.matmul(_dev(a).ptr, _dev(bm).ptr, c.ptr, 37, 70, 45)
    wc = np.empty((37, 45), np.float32)
    orc.O.oracle_matmul(a.ctypes.data, bm.ctypes.data, wc.ctypes.data, 37, 70, 45)
    assert rel_err_floor(c.to_numpy((37, 45)), wc) <= TOL
    c2 = _out((2, 2))
    B.matmul(_dev(np.array([[1, 2], [3, 4]], np.float32)).ptr,
             _dev(np.array([[5, 6], [7, 8]], np.float32)).ptr, c2.ptr, 2, 2, 2)
    assert np.array_equal(c2.to_numpy((2, 2)), np.array([[19, 22], [43, 50]], np.float32))
    c3 = _out((2, 2))
    B.matmul(_dev(np.array([[1, 2, 3], [4, 5, 6]], np.float32)).ptr,
             _dev(np.array([[7, 8], [9, 10], [11, 12]], np.float32)).ptr, c3.ptr, 2, 3, 2)
    assert np.array_equal(c3.to_numpy((2, 2)), np.array([[58, 64], [139, 154]], np.float32))


def test_elementwise_and_bias(gpu):
    from omnimatchdeeplearningtool_b200.backend import CUDABackend as B
    rng = _rng(13)
    x = rng.standard_normal(1003).astype(np.float32)
    y = rng.standard_normal(1003).astype(np.float32)
    dX, dY = _dev(x), _dev(y)
    o = _out((1003,))
    B.add(dX.ptr, dY.ptr, o.ptr, 1003)
    assert np.array_equal(o.to_numpy((1003,)), x + y)
    B.relu(dX.ptr, o.ptr, 1003)
    assert np.array_equal(o.to_numpy((1003,)), np.maximum(x, 0))
    B.reluBackward(dX.ptr, dY.ptr, o.ptr, 1003)
    assert np.array_equal(o.to_numpy((1003,)), np.where(x > 0, y, 0))
    B.clip(dX.ptr, o.ptr, 1003, 0.0, 0.5)
    assert np.array_equal(o.to_numpy((1003,)), np.clip(x, 0, 0.5))
    # in place (output = first input), and a start 4 bytes past 16-byte alignment (scalar path)
    z = _dev(x)
    B.add(z.ptr, dY.ptr, z.ptr, 1003)
    assert np.array_equal(z.to_numpy((1003,)), x + y)
    o2 = _out((1003,))
    B.relu(z.ptr + 4, o2.ptr + 4, 1002)
    assert np.array_equal(o2.to_numpy((1003,))[1:], np.maximum(x + y, 0)[1:])
    n, c, hw = 3, 5, 7
    a = rng.standard_normal((n, c, hw)).astype(np.float32)
    bias = rng.standard_normal(c).astype(np.float32)
    ob = _out(a.shape)
    B.addBias(_dev(a).ptr, _dev(bias).ptr, ob.ptr, n, c, hw)
    assert np.allclose(ob.to_numpy(a.shape), a + bias[None, :, None], atol=0, rtol=0)
    gb = _out((c,))
    B.addBiasBackward(_dev(a).ptr, gb.ptr, n, c, hw)
    assert rel_err_floor(gb.to_numpy((c,)), a.sum(axis=(0, 2))) <= TOL
    am = _out((n,), np.int32)
    m = rng.standard_normal((n, 1000)).astype(np.float32)
    B.argmax(_dev(m).ptr, am.ptr, n, 1000)
    assert np.array_equal(am.to_numpy((n,), np.int32), m.argmax(1))
    t = _out((1003,))
    B.transpose(_dev(x[:1000].reshape(20, 50)).ptr, t.ptr, 20, 50)
    assert np.array_equal(t.to_numpy((50, 20)), x[:1000].reshape(20, 50).T)


@pytest.mark.parametrize("n,k", [(8, 1000), (130, 1000), (1, 10), (4, 37)])
def test_softmax_ce_fused(gpu, n, k):
    """omCudaSoftmaxCrossEntropyFused against the three reference-named kernels it replaces
    (the softmax and the gradient bit for bit, the loss to summation order) and against the
    oracle (1e-4); two calls in a row, so the last-block ticket is seen to reset."""
    import oracle as orc
    from omnimatchdeeplearningtool_b200._lib import call
    from omnimatchdeeplearningtool_b200.backend import CUDABackend as B
    rng = _rng(31 + n)
    for rep in range(2):
        logits = (rng.standard_normal((n, k)) * 3).astype(np.float32)
        oh = np.zeros((n, k), np.float32)
        oh[np.arange(n), rng.integers(0, k, n)] = 1
        dL, dT = _dev(logits), _dev(oh)
        p, g, loss = _out((n, k)), _out((n, k)), _out((1,))
        call("omCudaSoftmaxCrossEntropyFused", dL.ptr, dT.ptr, p.ptr, g.ptr, loss.ptr, n, k)
        p2, g2, loss2 = _out((n, k)), _out((n, k)), _out((1,))
        B.softmax(dL.ptr, p2.ptr, n, k)
        B.crossEntropyForward(p2.ptr, dT.ptr, loss2.ptr, n, k)
        B.crossEntropySoftmaxBackward(p2.ptr, dT.ptr, g2.ptr, n, k)
        assert np.array_equal(p.to_numpy((n, k)), p2.to_numpy((n, k)))
        assert np.array_equal(g.to_numpy((n, k)), g2.to_numpy((n, k)))
        lv, lv2 = float(loss.to_numpy((1,))[0]), float(loss2.to_numpy((1,))[0])
        assert abs(lv - lv2) <= 1e-6 * abs(lv2)
        wp = np.empty_like(logits)
        orc.O.oracle_softmax(logits.ctypes.data, wp.ctypes.data, n, k)
        wl = orc.O.oracle_cross_entropy(wp.ctypes.data, oh.ctypes.data, n, k)
        assert abs(lv - wl) <= TOL * abs(wl)
        # without the softmax output
        g3, loss3 = _out((n, k)), _out((1,))
        call("omCudaSoftmaxCrossEntropyFused", dL.ptr, dT.ptr, None, g3.ptr, loss3.ptr, n, k)
        assert np.array_equal(g3.to_numpy((n, k)), g2.to_numpy((n, k)))
        assert float(loss3.to_numpy((1,))[0]) == lv


@pytest.mark.parametrize("m,kk,n", [(128, 512, 1000), (512, 128, 1000), (128, 1000, 512),
                                    (8, 2048, 1000), (1, 3, 1), (33, 7, 65), (70000, 8, 16)])
def test_matmul_shapes(gpu, m, kk, n):
    """omCudaMatmul (cuda_kernels.cu:768) on the training path's FC shapes (forward, weight and
    input gradients of 512 -> 1000 at batch 128) through the 3xTF32 tensor-core path, tiny and
    ragged shapes, and M > 65535 (the SIMT kernel), against the oracle's matmul (1e-4)."""
    import oracle as orc
    from omnimatchdeeplearningtool_b200.backend import CUDABackend as B
    rng = _rng(m + kk + n)
    a = rng.standard_normal((m, kk)).astype(np.float32)
    bm = rng.standard_normal((kk, n)).astype(np.float32)
    c = _out((m, n))
    B.matmul(_dev(a).ptr, _dev(bm).ptr, c.ptr, m, kk, n)
    wc = np.empty((m, n), np.float32)
    orc.O.oracle_matmul(a.ctypes.data, bm.ctypes.data, wc.ctypes.data, m, kk, n)
    assert rel_err_floor(c.to_numpy((m, n)), wc) <= TOL
    assert gpu.kernel_error() == 0
