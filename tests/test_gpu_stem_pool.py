"""The fused stem + 3x3/2/1 max pool (omCudaStemConvBnActPoolIn).

Each case runs the image stem (BN folded, act) and the max pool through the fused kernel and
through omCudaStemConvBnActIn followed by omCudaMaxPool2dNhwc: the pooled outputs must be
bit-identical, since both round the stem output the same way and compare the same 16-bit
values in the same order. Against the fp32 oracle (conv -> BN -> act -> max pool, the reference's
stem sequence om.engine.resnet.ixx:236-241): <= 2e-2. The ResNet-50 plan with and without the
fusion gives the same logits.
"""
import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu

# n, h, w, cout, act, dtype, input dtype. Odd sizes give an odd stem output (the last pooled
# row and column have a two-wide window, the last stem row pair has one row); batch 3 and 37
# make CTA ranges cross image boundaries and start at halo pairs.
CASES = [
    (2, 224, 224, 64, "relu", "bf16", "f32"),     # the ResNet-50 stem
    (2, 224, 224, 64, "relu", "bf16", "bf16"),    # the same from a bf16 image
    (3, 221, 221, 64, "relu", "f16", "f32"),      # 111 x 111 stem output
    (37, 64, 48, 64, "none", "bf16", "f32"),      # negative values, 32 x 24 stem output, 37 images
    (2, 100, 90, 64, "relu6", "bf16", "f32"),     # ReLU6, 50 x 45 stem output
    (2, 90, 100, 64, "relu", "f16", "f16"),       # fp16 image, 45 x 50 stem output
    (256, 224, 224, 64, "relu", "bf16", "bf16"),  # the benchmarked batch
]
ACT = {"none": 0, "relu": 1, "relu6": 2}


@pytest.mark.parametrize("case", CASES, ids=[f"s{i}" for i in range(len(CASES))])
def test_stem_pool_matches_two_launches_and_oracle(gpu, case):
    import oracle as orc
    from omnimatchdeeplearningtool_b200 import _lib
    from omnimatchdeeplearningtool_b200._lib import call, lib
    from omnimatchdeeplearningtool_b200.backend import DeviceBuffer
    n, h, wd, k, act, dt_name, in_name = case
    c, ks, stride, pad = 3, 7, 2, 3
    dt = _lib.DTYPE_BF16 if dt_name == "bf16" else _lib.DTYPE_F16
    rng = np.random.Generator(np.random.PCG64(4100 + h + wd + k + n))
    x = rng.standard_normal((n, c, h, wd), dtype=np.float32)
    w = (rng.standard_normal((k, c, ks, ks)) * np.sqrt(2.0 / (c * ks * ks))).astype(np.float32)
    g = rng.uniform(0.5, 1.5, k).astype(np.float32)
    b = (rng.standard_normal(k) * 0.1).astype(np.float32)
    mu = (rng.standard_normal(k) * 0.1).astype(np.float32)
    var = rng.uniform(0.5, 1.5, k).astype(np.float32)
    p = (h + 2 * pad - ks) // stride + 1
    q = (wd + 2 * pad - ks) // stride + 1
    p2, q2 = (p - 1) // 2 + 1, (q - 1) // 2 + 1
    assert lib.omCudaStemPoolSupported(n, c, h, wd, k, ks, ks, stride, pad, dt) == 1

    if in_name == "f32":
        xin, idt = x, _lib.DTYPE_F32
    elif in_name == "bf16":
        from omnimatchdeeplearningtool_b200.plan import to_bf16_bits
        xin, idt = to_bf16_bits(x), _lib.DTYPE_BF16
    else:
        xin, idt = x.astype(np.float16), _lib.DTYPE_F16
    keep = [DeviceBuffer.from_numpy(a) for a in (xin, w, g, b, mu, var)]
    packed = DeviceBuffer(int(lib.omCudaPackedStemWeightElems(k, c, ks, ks, stride)) * 2)
    bias = DeviceBuffer(k * 4)
    call("omCudaPackStemWeight", keep[1].ptr, None, keep[2].ptr, keep[3].ptr, keep[4].ptr,
         keep[5].ptr, 1e-5, packed.ptr, bias.ptr, k, c, ks, ks, stride, dt)
    ws = DeviceBuffer(int(lib.omCudaStemWorkspaceBytes(n, c, h, wd, ks, ks, stride, pad)))
    full = DeviceBuffer(n * p * q * k * 2)
    two = DeviceBuffer(n * p2 * q2 * k * 2)
    fused = DeviceBuffer(n * p2 * q2 * k * 2)
    call("omCudaMemset", fused.ptr, 0xFF, fused.nbytes)   # every element must be written
    call("omCudaStemConvBnActIn", keep[0].ptr, idt, ws.ptr, packed.ptr, bias.ptr, full.ptr, n, c,
         h, wd, k, ks, ks, stride, pad, ACT[act], dt)
    call("omCudaMaxPool2dNhwc", full.ptr, two.ptr, n, p, q, k, 3, 2, 1, dt)
    call("omCudaStemConvBnActPoolIn", keep[0].ptr, idt, ws.ptr, packed.ptr, bias.ptr, fused.ptr,
         n, c, h, wd, k, ks, ks, stride, pad, ACT[act], dt)
    got_bits = fused.to_numpy((n, p2, q2, k), np.uint16)
    want_bits = two.to_numpy((n, p2, q2, k), np.uint16)
    assert gpu.kernel_error() == 0
    assert np.array_equal(got_bits, want_bits)

    # against the fp32 oracle on a few images (the full batch would take the CPU minutes)
    o32 = DeviceBuffer(n * k * p2 * q2 * 4)
    call("omCudaNhwcToNchw", fused.ptr, o32.ptr, n, k, p2, q2, k, dt)
    got = o32.to_numpy((n, k, p2, q2))
    sel = [0, n - 1] if n > 2 else list(range(n))
    y = orc.batchnorm_eval(orc.conv2d(x[sel], w, None, stride, pad), g, b, mu, var)
    if act == "relu":
        y = orc.relu(y)
    elif act == "relu6":
        y = np.clip(y, 0.0, 6.0)
    want = orc.maxpool(y, 3, 2, 1)
    want = want[0] if isinstance(want, tuple) else want
    assert rel_err(got[sel], want) <= 2e-2


def test_stem_pool_rejects_unsupported_shapes(gpu):
    from omnimatchdeeplearningtool_b200 import _lib
    from omnimatchdeeplearningtool_b200._lib import lib
    bf = _lib.DTYPE_BF16
    # 32, 96 or 128 output channels, a stem output wider than 128, a 3x3 stem (two tap
    # columns after space-to-depth), fp32: not taken, nothing launched
    for k in (32, 96, 128):
        assert lib.omCudaStemPoolSupported(2, 3, 224, 224, k, 7, 7, 2, 3, bf) == 0
    assert lib.omCudaStemPoolSupported(2, 3, 224, 224, 64, 3, 3, 2, 1, bf) == 0
    assert lib.omCudaStemPoolSupported(2, 3, 224, 300, 64, 7, 7, 2, 3, bf) == 0
    assert lib.omCudaStemPoolSupported(2, 3, 224, 224, 64, 7, 7, 2, 3, _lib.DTYPE_F32) == 0
    assert lib.omCudaStemConvBnActPoolIn(16, 0, 16, 16, 16, 16, 2, 3, 224, 224, 96, 7, 7, 2, 3,
                                         1, bf) == -3


def test_resnet50_plan_stem_pool_fused_equals_unfused(gpu):
    from omnimatchdeeplearningtool_b200 import _lib, synth
    from omnimatchdeeplearningtool_b200.plan import InferencePlan
    net = synth.resnet_spec(50)
    w = synth.make_weights(net)
    x = synth.normal_input(4)
    fused = InferencePlan(net, w, batch=4, dtype=_lib.DTYPE_BF16)
    plain = InferencePlan(net, w, batch=4, dtype=_lib.DTYPE_BF16, fuse_stem_pool=False)
    assert sum(1 for m in fused.meta if m.get("kind") == "maxpool") == 0
    assert sum(1 for m in plain.meta if m.get("kind") == "maxpool") == 1
    a = fused.run(x)
    b_ = plain.run(x)
    assert gpu.kernel_error() == 0
    assert np.array_equal(a, b_)
