"""Parity of the NHWC 16-bit bandwidth kernels with the CPU oracle, on the same 16-bit values.

* max pool (omCudaMaxPool2dNhwc): a max returns one of its operands, so the result must equal
  the oracle's max pool of the 16-bit-rounded input bit for bit;
* global average pool (omCudaGlobalAvgPoolNhwc) with an fp32 output: fp32 sums of the 16-bit
  values, max|a-b|/max|b| <= 1e-5 against the oracle on the rounded input;
* depthwise conv + BN + ReLU6 (omCudaDepthwiseConv2dNhwc): fp32 accumulation (fp16 3x3 with the
  weights held per thread: fp16 HFMA2 over the 9 taps), 16-bit output: <= 1e-2 against the
  oracle on rounded input and BN-folded fp32 weights. The fp16 3x3 paths (the TMA row-ring
  kernel and the direct kernel) are also checked bit for bit against an exact emulation of
  their arithmetic: the bias and the taps' products accumulated by fused multiply-adds, each
  rounded once to fp16, in tap order;
* residual add + activation (omCudaAddActNhwc): one 16-bit rounding of act(a + b).
Ragged sizes (odd H and W, channels stored padded to a multiple of 8) are included.
"""
import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu

_KEEP = []


def _round16(a, dt):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(a, np.float32))
    return t.to(torch.bfloat16 if dt == "bf16" else torch.float16).to(torch.float32).numpy()


def _to_nhwc(x, cs, dtype):
    from omnimatchdeeplearningtool_b200._lib import call
    from omnimatchdeeplearningtool_b200.backend import DeviceBuffer
    n, c, h, w = x.shape
    d32 = DeviceBuffer.from_numpy(np.ascontiguousarray(x, np.float32))
    d16 = DeviceBuffer(n * h * w * cs * 2)
    call("omCudaNchwToNhwc", d32.ptr, d16.ptr, n, c, h, w, cs, dtype)
    _KEEP.extend([d32, d16])
    return d16


def _from_nhwc(buf, n, c, h, w, cs, dtype):
    from omnimatchdeeplearningtool_b200._lib import call
    from omnimatchdeeplearningtool_b200.backend import DeviceBuffer
    o32 = DeviceBuffer(n * c * h * w * 4)
    call("omCudaNhwcToNchw", buf.ptr, o32.ptr, n, c, h, w, cs, dtype)
    _KEEP.append(o32)
    return o32.to_numpy((n, c, h, w))


@pytest.fixture(autouse=True)
def _release():
    yield
    _KEEP.clear()


@pytest.mark.parametrize("n,c,h,w,k,stride,pad,dt", [
    (4, 64, 112, 112, 3, 2, 1, "bf16"),   # the ResNet max pool
    (3, 24, 9, 7, 3, 2, 1, "f16"),        # ragged H, W; 24 channels
    (2, 5, 8, 8, 2, 2, 0, "bf16"),        # 5 channels stored as 8; 2x2/2
    (1, 16, 5, 6, 3, 1, 1, "bf16"),       # stride 1
])
def test_maxpool_nhwc_bit_exact(gpu, n, c, h, w, k, stride, pad, dt):
    import oracle as orc
    from omnimatchdeeplearningtool_b200 import _lib
    from omnimatchdeeplearningtool_b200._lib import call, lib
    from omnimatchdeeplearningtool_b200.backend import DeviceBuffer
    dtype = _lib.DTYPE_BF16 if dt == "bf16" else _lib.DTYPE_F16
    rng = np.random.Generator(np.random.PCG64(40 + h + c))
    x = rng.standard_normal((n, c, h, w), dtype=np.float32) * 3
    cs = int(lib.omCudaStoredChannels(c))
    din = _to_nhwc(x, cs, dtype)
    p, q = (h + 2 * pad - k) // stride + 1, (w + 2 * pad - k) // stride + 1
    out = DeviceBuffer(n * p * q * cs * 2)
    _KEEP.append(out)
    call("omCudaMaxPool2dNhwc", din.ptr, out.ptr, n, h, w, cs, k, stride, pad, dtype)
    got = _from_nhwc(out, n, c, p, q, cs, dtype)
    want = orc.maxpool(_round16(x, dt), k, stride, pad)
    assert gpu.kernel_error() == 0
    assert np.array_equal(got, want)


@pytest.mark.parametrize("n,c,h,w,dt", [(4, 2048, 7, 7, "bf16"), (3, 40, 5, 3, "f16")])
def test_global_avgpool_nhwc(gpu, n, c, h, w, dt):
    import oracle as orc
    from omnimatchdeeplearningtool_b200 import _lib
    from omnimatchdeeplearningtool_b200._lib import call, lib
    from omnimatchdeeplearningtool_b200.backend import DeviceBuffer
    dtype = _lib.DTYPE_BF16 if dt == "bf16" else _lib.DTYPE_F16
    rng = np.random.Generator(np.random.PCG64(70 + c))
    x = np.abs(rng.standard_normal((n, c, h, w), dtype=np.float32))
    cs = int(lib.omCudaStoredChannels(c))
    din = _to_nhwc(x, cs, dtype)
    out = DeviceBuffer(n * cs * 4)
    _KEEP.append(out)
    call("omCudaGlobalAvgPoolNhwc", din.ptr, out.ptr, n, h * w, cs, dtype, _lib.DTYPE_F32)
    got = out.to_numpy((n, cs))[:, :c]
    want = orc.global_avgpool(_round16(x, dt)).reshape(n, c)
    assert gpu.kernel_error() == 0
    assert rel_err(got, want) <= 1e-5


@pytest.mark.parametrize("n,c,h,k,stride,dt", [(2, 144, 28, 3, 2, "f16"), (3, 32, 15, 3, 1, "bf16"),
                                                (2, 40, 13, 5, 2, "bf16"),   # generic window
                                                (1, 2048, 9, 3, 1, "f16"),   # C/8 = 256 threads
                                                (3, 128, 15, 3, 1, "f16"),   # row pairs, odd P
                                                (2, 64, 16, 3, 2, "f16"),    # fp16 weights held
                                                (4, 128, 112, 3, 1, "f16"),  # row ring, MobileNet size
                                                (2, 192, 7, 3, 1, "f16"),    # ring: 3 channel tiles
                                                (3, 256, 56, 3, 2, "f16")])  # ring, stride 2
def test_depthwise_nhwc(gpu, n, c, h, k, stride, dt):
    import oracle as orc
    from omnimatchdeeplearningtool_b200 import _lib
    from omnimatchdeeplearningtool_b200._lib import call, lib
    from omnimatchdeeplearningtool_b200.backend import DeviceBuffer
    dtype = _lib.DTYPE_BF16 if dt == "bf16" else _lib.DTYPE_F16
    rng = np.random.Generator(np.random.PCG64(90 + c))
    x = rng.standard_normal((n, c, h, h), dtype=np.float32)
    wt = (rng.standard_normal((c, 1, k, k)) * 0.5).astype(np.float32)
    g = rng.uniform(0.5, 1.5, c).astype(np.float32)
    b = (rng.standard_normal(c) * 0.1).astype(np.float32)
    mu = (rng.standard_normal(c) * 0.1).astype(np.float32)
    var = rng.uniform(0.5, 1.5, c).astype(np.float32)
    pad = k // 2
    cs = int(lib.omCudaStoredChannels(c))
    din = _to_nhwc(x, cs, dtype)
    bufs = [DeviceBuffer.from_numpy(a) for a in (wt, g, b, mu, var)]
    packed, bias = DeviceBuffer(k * k * cs * 4), DeviceBuffer(cs * 4)
    _KEEP.extend(bufs + [packed, bias])
    call("omCudaPackDepthwiseWeight", *[t.ptr for t in bufs], 1e-5, packed.ptr, bias.ptr, c, k, k, cs)
    p = (h + 2 * pad - k) // stride + 1
    out = DeviceBuffer(n * p * p * cs * 2)
    _KEEP.append(out)
    call("omCudaDepthwiseConv2dNhwc", din.ptr, packed.ptr, bias.ptr, out.ptr, n, h, h, cs, k, k,
         stride, pad, 2, dtype)
    got = _from_nhwc(out, n, c, p, p, cs, dtype)
    scale = g / np.sqrt(var + 1e-5)
    want = orc.relu6(orc.conv2d(_round16(x, dt), wt * scale[:, None, None, None], b - mu * scale,
                                stride, pad, groups=c))
    assert gpu.kernel_error() == 0
    assert rel_err(got, want) <= 1e-2


def test_add_act_nhwc(gpu):
    from omnimatchdeeplearningtool_b200 import _lib
    from omnimatchdeeplearningtool_b200._lib import call
    from omnimatchdeeplearningtool_b200.backend import DeviceBuffer
    rng = np.random.Generator(np.random.PCG64(5))
    a = rng.standard_normal((3, 8, 5, 7), dtype=np.float32)
    bb = rng.standard_normal((3, 8, 5, 7), dtype=np.float32)
    da, db = _to_nhwc(a, 8, _lib.DTYPE_BF16), _to_nhwc(bb, 8, _lib.DTYPE_BF16)
    out = DeviceBuffer(a.size * 2)
    _KEEP.append(out)
    call("omCudaAddActNhwc", da.ptr, db.ptr, out.ptr, a.size, 1, _lib.DTYPE_BF16)
    got = _from_nhwc(out, 3, 8, 5, 7, 8, _lib.DTYPE_BF16)
    want = _round16(np.maximum(_round16(a, "bf16") + _round16(bb, "bf16"), 0), "bf16")
    assert gpu.kernel_error() == 0
    assert np.array_equal(got, want)


def _hfma_depthwise(x16, w16, b16, stride, act6=True):
    """Exact model of the fp16 3x3 depthwise kernels' arithmetic on NHWC fp16 input x16
    [N, H, W, C]: acc = bias; for the taps t = 0..8 (row-major) acc = fp16(x * w + acc), one
    rounding per fused multiply-add; then ReLU6. The products of two fp16 values and their sum
    with an fp16 accumulator of these magnitudes are exact in fp64, so rounding that sum to
    fp16 once is the fused operation's rounding."""
    n, h, w, c = x16.shape
    p, q = (h - 1) // stride + 1, (w - 1) // stride + 1
    xp = np.zeros((n, h + 2, w + 2, c), np.float16)
    xp[:, 1:h + 1, 1:w + 1] = x16
    acc = np.broadcast_to(b16, (n, p, q, c)).astype(np.float16)
    for t in range(9):
        r, sx = divmod(t, 3)
        tap = xp[:, r:r + stride * (p - 1) + 1:stride, sx:sx + stride * (q - 1) + 1:stride]
        acc = (tap.astype(np.float64) * w16[t].astype(np.float64)
               + acc.astype(np.float64)).astype(np.float16)
    if act6:
        acc = np.minimum(np.maximum(acc, np.float16(0)), np.float16(6))
    return acc


@pytest.mark.parametrize("n,c,h,w,stride", [
    (4, 128, 112, 112, 1),   # ring kernel: MobileNet stage-1 size, whole 128-channel pixels
    (3, 256, 56, 56, 2),     # ring kernel, stride 2, whole 256-channel pixels
    (2, 1024, 14, 14, 1),    # ring kernel, 1024-channel pixels as four 256-channel boxes
    (3, 512, 27, 27, 1),     # ring kernel, 512-channel tiles, odd P
    (2, 512, 28, 28, 2),     # ring kernel, stride 2, 512-channel tiles
    (2, 256, 112, 112, 1),   # ring kernel, two 128-channel tiles per pixel
    (5, 192, 9, 11, 1),      # ring kernel, 64-channel tiles, runs that cross images
    (3, 64, 15, 13, 2),      # ring kernel, stride 2, odd sizes
    (1, 64, 3, 254, 1),      # ring kernel, the widest row a slot takes (256 columns)
    (2, 64, 1, 1, 1),        # ring kernel, 1x1 images
    (1, 128, 2, 3, 2),       # ring kernel, stride 2 on a 2x3 image
    (2, 32, 20, 18, 1),      # direct kernel (32 channels), row pairs
    (1, 64, 9, 300, 2),      # direct kernel (row wider than a ring slot)
])
def test_depthwise_f16_bit_exact(gpu, n, c, h, w, stride):
    from omnimatchdeeplearningtool_b200 import _lib
    from omnimatchdeeplearningtool_b200._lib import call
    from omnimatchdeeplearningtool_b200.backend import DeviceBuffer
    rng = np.random.Generator(np.random.PCG64(300 + c + h))
    x16 = rng.standard_normal((n, h, w, c)).astype(np.float16)
    wt = (rng.standard_normal((c, 1, 3, 3)) * 0.5).astype(np.float32)
    g = rng.uniform(0.5, 1.5, c).astype(np.float32)
    b = (rng.standard_normal(c) * 0.1).astype(np.float32)
    mu = (rng.standard_normal(c) * 0.1).astype(np.float32)
    var = rng.uniform(0.5, 1.5, c).astype(np.float32)
    din = DeviceBuffer.from_numpy(x16)
    bufs = [DeviceBuffer.from_numpy(a) for a in (wt, g, b, mu, var)]
    packed, bias = DeviceBuffer(9 * c * 4), DeviceBuffer(c * 4)
    _KEEP.extend(bufs + [din, packed, bias])
    call("omCudaPackDepthwiseWeight", *[t.ptr for t in bufs], 1e-5, packed.ptr, bias.ptr, c, 3, 3, c)
    p, q = (h - 1) // stride + 1, (w - 1) // stride + 1
    out = DeviceBuffer(n * p * q * c * 2)
    _KEEP.append(out)
    call("omCudaDepthwiseConv2dNhwc", din.ptr, packed.ptr, bias.ptr, out.ptr, n, h, w, c, 3, 3,
         stride, 1, 2, _lib.DTYPE_F16)
    got = out.to_numpy((n, p, q, c), np.float16)
    w16 = packed.to_numpy((9, c)).astype(np.float16)
    b16 = bias.to_numpy((c,)).astype(np.float16)
    want = _hfma_depthwise(x16, w16, b16, stride)
    assert gpu.kernel_error() == 0
    bad = np.flatnonzero(got.view(np.uint16) != want.view(np.uint16))
    assert bad.size == 0, (bad.size, bad[:5], got.ravel()[bad[:5]], want.ravel()[bad[:5]])
