"""Parity of the tcgen05 implicit-GEMM conv (omCudaConv2dBnAct) with the CPU oracle.

Each case runs conv -> eval BatchNorm -> (+ residual) -> activation on seeded inputs in the
reference layout (NCHW fp32) through the oracle, and the same through the NHWC 16-bit fused
kernel. Two checks per case, both with max|a-b|/max|b|:
  * against the oracle fed the same 16-bit-rounded input, weights (BN folded) and residual:
    <= 1e-2 (only accumulation order and the 16-bit output rounding differ);
  * against the fp32 oracle on the unrounded data: <= 2e-2 (the 16-bit tolerance).
"""
import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu

# n, c, h, k, ksize, stride, pad, dtype, residual, act, out_f32
CASES = [
    (2, 64, 14, 64, 3, 1, 1, "bf16", False, "relu", False),       # SW128, BN=64
    (4, 128, 7, 256, 1, 1, 0, "bf16", False, "relu", False),      # 1x1, M < one wave
    (3, 64, 15, 128, 3, 2, 1, "bf16", False, "relu", False),      # stride 2, ragged M
    (2, 64, 14, 256, 1, 2, 0, "bf16", False, "none", False),      # strided 1x1 downsample
    (2, 3, 32, 64, 7, 2, 3, "bf16", False, "relu", False),        # ImageNet stem, Cs=8
    (2, 32, 16, 128, 1, 1, 0, "f16", False, "relu6", False),      # C=32: 64-byte swizzle
    (2, 32, 15, 64, 3, 1, 1, "bf16", True, "relu", False),        # C=32, 9 taps: 2+2+2+2+1
    (3, 32, 17, 96, 3, 2, 1, "f16", False, "relu6", False),       # C=32, stride 2
    (8, 32, 112, 128, 1, 1, 0, "bf16", False, "relu6", False),    # MobileNet expand, large M
    (2, 40, 12, 64, 1, 1, 0, "bf16", False, "relu", False),       # C=40: interleaved boxes
    (2, 128, 8, 32, 1, 1, 0, "f16", True, "none", False),         # BN=32 + residual
    (2, 64, 14, 64, 3, 1, 1, "f16", True, "relu", False),         # fp16 + residual
    (16, 64, 56, 256, 1, 1, 0, "bf16", True, "relu", False),      # BN=256 tiles
    (16, 256, 14, 256, 3, 1, 1, "bf16", False, "relu", False),    # 36 k-blocks
    (5, 2048, 1, 1000, 1, 1, 0, "bf16", False, "none", True),     # FC: M=5, K=1000, fp32 out
    (2, 3, 31, 32, 3, 2, 1, "f16", False, "relu6", False),        # MobileNet stem, odd H
    # two 128-row sub-tiles per tile (>= 2 waves of 256-row tiles), last sub-tile past M
    (25, 64, 56, 64, 3, 1, 1, "bf16", False, "relu", False),      # BN=64, M = 78400
    (25, 64, 56, 128, 3, 1, 1, "bf16", True, "relu", False),      # BN=128 + residual
    (100, 128, 56, 128, 3, 2, 1, "f16", False, "relu", False),    # stride 2, fp16
    # 16 stored channels: one 32-byte-swizzled im2col box per filter tap
    (2, 16, 20, 96, 1, 1, 0, "f16", False, "relu6", False),       # 1x1: one tap per k-block
    (2, 16, 15, 64, 3, 1, 1, "bf16", True, "relu", False),        # 9 taps: 4 + 4 + 1
    (3, 12, 17, 32, 5, 2, 2, "bf16", False, "none", False),       # 12 -> 16 channels, stride 2
    (40, 16, 56, 128, 3, 1, 1, "bf16", False, "relu", False),     # two sub-tiles, 16 epi warps
    # long reductions over a partial last wave of tiles
    (4, 512, 7, 512, 3, 1, 1, "bf16", False, "relu", False),      # 72 k-blocks, 8 tiles
    (8, 128, 56, 128, 3, 1, 1, "f16", False, "relu6", False),     # 196 tiles on 148 SMs
    # 3x3 stride 1 on 28- to 57-wide maps: ragged last tiles, several N tiles, Cout < BN
    (4, 128, 28, 128, 3, 1, 1, "bf16", False, "relu", False),     # two 64-channel slices
    (3, 64, 28, 192, 3, 1, 1, "f16", True, "relu", False),        # two N tiles + residual
    (2, 64, 57, 64, 3, 1, 1, "bf16", True, "none", False),        # odd width, residual
    (2, 192, 30, 96, 3, 1, 1, "bf16", False, "relu6", False),     # three slices, Cout < BN
]


def _round16(a, dtype):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(a, np.float32))
    t = t.to(torch.bfloat16 if dtype == "bf16" else torch.float16).to(torch.float32)
    return t.numpy()


def _reference(x, w, bn, res, stride, pad, act):
    import oracle as orc
    y = orc.conv2d(x, w, None, stride, pad)
    y = orc.batchnorm_eval(y, *bn)
    if res is not None:
        y = y + res
    if act == "relu":
        y = orc.relu(y)
    elif act == "relu6":
        y = orc.relu6(y)
    return y


def _check_case(gpu, case, images=None):
    """Run one case through omCudaConv2dBnAct and check it against the oracle. With `images`,
    the kernel runs on the whole batch and the oracle only on those images (the CPU cost of a
    full batch-256 oracle would be minutes); the comparison covers every output of them."""
    from omnimatchdeeplearningtool_b200 import _lib
    from omnimatchdeeplearningtool_b200.backend import DeviceBuffer
    from omnimatchdeeplearningtool_b200._lib import call, lib

    n, c, h, k, ks, stride, pad, dt, use_res, act, out_f32 = case
    rng = np.random.Generator(np.random.PCG64(1234 + c * 7 + k))
    x = rng.standard_normal((n, c, h, h), dtype=np.float32)
    w = (rng.standard_normal((k, c, ks, ks)) * np.sqrt(2.0 / (c * ks * ks))).astype(np.float32)
    gamma = rng.uniform(0.5, 1.5, k).astype(np.float32)
    beta = (rng.standard_normal(k) * 0.1).astype(np.float32)
    mean = (rng.standard_normal(k) * 0.1).astype(np.float32)
    var = rng.uniform(0.5, 1.5, k).astype(np.float32)
    p = (h + 2 * pad - ks) // stride + 1
    res = rng.standard_normal((n, k, p, p), dtype=np.float32) if use_res else None
    dtype = _lib.DTYPE_BF16 if dt == "bf16" else _lib.DTYPE_F16
    odt = _lib.DTYPE_F32 if out_f32 else dtype
    act_id = {"none": 0, "relu": 1, "relu6": 2}[act]

    cs = int(lib.omCudaStoredChannels(c))
    dx32 = DeviceBuffer.from_numpy(x)
    dx = DeviceBuffer(n * h * h * cs * 2)
    call("omCudaNchwToNhwc", dx32.ptr, dx.ptr, n, c, h, h, cs, dtype)
    dx32.free()
    dw = DeviceBuffer.from_numpy(w)
    bufs = [DeviceBuffer.from_numpy(a) for a in (gamma, beta, mean, var)]
    packed = DeviceBuffer(int(lib.omCudaPackedConvWeightElems(k, ks, ks, cs)) * 2)
    bias = DeviceBuffer(k * 4)
    call("omCudaPackConvWeight", dw.ptr, None, *[b.ptr for b in bufs], 1e-5, packed.ptr, bias.ptr,
         k, c, ks, ks, cs, dtype)
    dres = None
    if use_res:
        if out_f32:
            dres = DeviceBuffer.from_numpy(np.ascontiguousarray(res.transpose(0, 2, 3, 1)))
        else:
            r32 = DeviceBuffer.from_numpy(res)
            dres = DeviceBuffer(n * p * p * k * 2)
            call("omCudaNchwToNhwc", r32.ptr, dres.ptr, n, k, p, p, k, dtype)
            r32.free()
    out = DeviceBuffer(n * p * p * k * (4 if out_f32 else 2))
    out2 = DeviceBuffer(n * p * p * k * (4 if out_f32 else 2))
    for o in (out, out2):
        call("omCudaConv2dBnAct", dx.ptr, packed.ptr, bias.ptr, dres.ptr if dres else None, o.ptr,
             n, h, h, cs, k, ks, ks, stride, pad, act_id, dtype, odt)
    # a second launch gives the same bits
    raw = np.uint8
    assert np.array_equal(out.to_numpy((out.nbytes,), raw), out2.to_numpy((out2.nbytes,), raw))
    if out_f32:
        got = out.to_numpy((n, p, p, k)).transpose(0, 3, 1, 2)
    else:
        o32 = DeviceBuffer(n * k * p * p * 4)
        call("omCudaNhwcToNchw", out.ptr, o32.ptr, n, k, p, p, k, dtype)
        got = o32.to_numpy((n, k, p, p))
        o32.free()
    assert gpu.kernel_error() == 0
    for b in [dx, dw, packed, bias, out, out2] + bufs + ([dres] if dres else []):
        b.free()
    assert np.isfinite(got).all()
    if images is not None:
        got = got[images]
        x = np.ascontiguousarray(x[images])
        res = None if res is None else np.ascontiguousarray(res[images])

    # fp32 reference on the original data
    want = _reference(x, w, (gamma, beta, mean, var), res, stride, pad, act)
    e32 = rel_err(got, want)
    # reference on 16-bit-rounded operands with the BN scale folded as the kernel does
    scale = gamma / np.sqrt(var + 1e-5)
    wf = _round16(w * scale[:, None, None, None], dt)
    bf = beta - mean * scale
    xr = _round16(x, dt)
    rr = None if res is None else (res if out_f32 else _round16(res, dt))
    import oracle as orc
    y = orc.conv2d(xr, wf, bf, stride, pad)
    if rr is not None:
        y = y + rr
    y = orc.relu(y) if act == "relu" else (orc.relu6(y) if act == "relu6" else y)
    e16 = rel_err(got, y)
    assert e16 <= 1e-2, f"vs rounded-operand oracle: {e16}"
    assert e32 <= 2e-2, f"vs fp32 oracle: {e32}"


@pytest.mark.parametrize("case", CASES, ids=[f"c{i}" for i in range(len(CASES))])
def test_conv_bn_act(gpu, case):
    _check_case(gpu, case)


def tile_plan(n, h, cs, k, ks, stride, pad, residual):
    """(BN, CTAs per SM, sub-tiles per tile, epilogue warps) that omCudaConv2dBnAct picks."""
    import ctypes
    from omnimatchdeeplearningtool_b200._lib import call
    plan = (ctypes.c_int * 4)()
    call("omCudaConvTilePlan", n, h, h, cs, k, ks, ks, stride, pad, int(residual), plan)
    return tuple(plan)


# ResNet-50's batch-256 layers whose tile variant only a full batch reaches: 256-wide tiles for
# long reductions (the layer-3/4 3x3 and 1x1 convs), and the sub-tile pairs of the 64- and
# 128-wide 3x3 layers. Each case names the plan it must get, so a retune that stops covering a
# variant fails here instead of leaving it untested. (n, c, h, k, ks, stride, pad, dtype,
# residual, act, out_f32), expected (BN, OCC, MT, EW)
FULL_BATCH_CASES = [
    ((256, 256, 14, 256, 3, 1, 1, "bf16", False, "relu", False), (256, 1, 1, 8)),   # layer-3 3x3
    ((256, 512, 7, 512, 3, 1, 1, "bf16", False, "relu", False), (256, 1, 1, 8)),    # layer-4 3x3
    ((256, 1024, 14, 256, 1, 1, 0, "bf16", False, "relu", False), (256, 1, 1, 8)),  # layer-3 1x1 in
    ((256, 2048, 7, 512, 1, 1, 0, "bf16", False, "relu", False), (256, 1, 1, 8)),   # layer-4 1x1 in
    ((256, 2048, 7, 512, 1, 1, 0, "bf16", True, "relu", False), (256, 1, 1, 4)),    # + residual
    ((256, 1024, 14, 256, 1, 1, 0, "f16", True, "relu", False), (256, 1, 1, 4)),    # + residual
    ((256, 64, 56, 64, 3, 1, 1, "bf16", False, "relu", False), (64, 1, 2, 8)),      # layer-1 3x3
    ((256, 128, 28, 128, 3, 1, 1, "bf16", False, "relu", False), (128, 1, 2, 8)),   # layer-2 3x3
]
FULL_BATCH_IMAGES = [0, 1, 2, 3, 252, 253, 254, 255]


@pytest.mark.parametrize("case,plan", FULL_BATCH_CASES,
                         ids=[f"b256_{c[1]}x{c[2]}_{c[3]}k{c[4]}{'_res' if c[8] else ''}"
                              for c, _ in FULL_BATCH_CASES])
def test_conv_bn_act_full_batch(gpu, case, plan):
    """The tile variants of the benchmarked batch-256 ResNet-50 forward, launched at batch 256
    and compared on its first four and last four images."""
    from omnimatchdeeplearningtool_b200._lib import lib
    n, c, h, k, ks, stride, pad, _, res = case[:9]
    cs = int(lib.omCudaStoredChannels(c))
    assert tile_plan(n, h, cs, k, ks, stride, pad, res) == plan
    _check_case(gpu, case, images=FULL_BATCH_IMAGES)


def test_conv_rejects_bad_shapes(gpu):
    from omnimatchdeeplearningtool_b200._lib import lib
    # Cs not a multiple of 8 and Cout not a multiple of 8 are reported, not launched
    assert lib.omCudaConv2dBnAct(16, 16, None, None, 16, 1, 8, 8, 12, 64, 3, 3, 1, 1, 0, 1, 1) == -3
    assert lib.omCudaConv2dBnAct(16, 16, None, None, 16, 1, 8, 8, 64, 60, 3, 3, 1, 1, 0, 1, 1) == -3
    # misaligned pointers are rejected
    assert lib.omCudaConv2dBnAct(18, 16, None, None, 16, 1, 8, 8, 64, 64, 3, 3, 1, 1, 0, 1, 1) == -2


@pytest.mark.parametrize("n,c,h,k,ks,stride,pad,dt", [(2, 3, 224, 64, 7, 2, 3, "bf16"),
                                                      (3, 3, 37, 64, 7, 2, 3, "bf16"),
                                                      (2, 3, 31, 32, 3, 2, 1, "f16"),
                                                      (1, 3, 300, 64, 7, 2, 3, "bf16"),
                                                      (2, 3, 20, 32, 7, 1, 3, "bf16"),  # stride 1
                                                      (2, 4, 33, 64, 5, 2, 2, "bf16"),  # 16 of 16
                                                      (1, 16, 24, 32, 3, 1, 1, "f16"),
                                                      (2, 1, 40, 8, 7, 2, 3, "bf16")])
def test_stem_conv_from_nchw_image(gpu, n, c, h, k, ks, stride, pad, dt):
    """omCudaStemConvBnAct: the image stem straight from NCHW fp32 (ImageNet 7x7/2 and the
    MobileNet 3x3/2 stem, and other channel counts that fit one 16-channel space-to-depth
    pixel), checked like the other fused convs."""
    import oracle as orc
    from omnimatchdeeplearningtool_b200 import _lib
    from omnimatchdeeplearningtool_b200._lib import call, lib
    from omnimatchdeeplearningtool_b200.backend import DeviceBuffer
    rng = np.random.Generator(np.random.PCG64(77 + h))
    x = rng.standard_normal((n, c, h, h), dtype=np.float32)
    w = (rng.standard_normal((k, c, ks, ks)) * np.sqrt(2.0 / (c * ks * ks))).astype(np.float32)
    g = rng.uniform(0.5, 1.5, k).astype(np.float32)
    b = (rng.standard_normal(k) * 0.1).astype(np.float32)
    mu = (rng.standard_normal(k) * 0.1).astype(np.float32)
    var = rng.uniform(0.5, 1.5, k).astype(np.float32)
    dtype = _lib.DTYPE_BF16 if dt == "bf16" else _lib.DTYPE_F16
    p = (h + 2 * pad - ks) // stride + 1
    keep = [DeviceBuffer.from_numpy(a) for a in (x, w, g, b, mu, var)]
    packed = DeviceBuffer(int(lib.omCudaPackedStemWeightElems(k, c, ks, ks, stride)) * 2)
    bias = DeviceBuffer(k * 4)
    call("omCudaPackStemWeight", keep[1].ptr, None, keep[2].ptr, keep[3].ptr, keep[4].ptr,
         keep[5].ptr, 1e-5, packed.ptr, bias.ptr, k, c, ks, ks, stride, dtype)
    out = DeviceBuffer(n * p * p * k * 2)
    ws = DeviceBuffer(int(lib.omCudaStemWorkspaceBytes(n, c, h, h, ks, ks, stride, pad)))
    keep.append(ws)
    call("omCudaStemConvBnAct", keep[0].ptr, ws.ptr, packed.ptr, bias.ptr, out.ptr, n, c, h, h, k,
         ks, ks, stride, pad, 1, dtype)
    o32 = DeviceBuffer(n * k * p * p * 4)
    call("omCudaNhwcToNchw", out.ptr, o32.ptr, n, k, p, p, k, dtype)
    got = o32.to_numpy((n, k, p, p))
    assert gpu.kernel_error() == 0
    want = orc.relu(orc.batchnorm_eval(orc.conv2d(x, w, None, stride, pad), g, b, mu, var))
    scale = g / np.sqrt(var + 1e-5)
    y16 = orc.relu(orc.conv2d(_round16(x, dt), _round16(w * scale[:, None, None, None], dt),
                              b - mu * scale, stride, pad))
    assert rel_err(got, y16) <= 1e-2
    assert rel_err(got, want) <= 2e-2
