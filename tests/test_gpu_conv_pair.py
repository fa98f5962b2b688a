"""The fused conv pair (omCudaConvPairBnAct): a conv and the 1x1 conv after it in one kernel, the
intermediate map kept on chip.

Each case runs conv 1 (BN folded, act1) -> conv 2 (1x1, BN folded, + residual, act2) through
the fused kernel and through two omCudaConv2dBnAct launches (the intermediate rounded to 16
bits in device memory): the results must be bit-identical, since both round the intermediate
the same way and sum in the same order. Against the fp32 oracle on the same data: <= 2e-2 (the
16-bit tolerance). The ResNet-50 plan with and without the fusion gives the same logits.
"""
import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu

# n, cin, h, mid, cout, k, stride, pad, dtype, residual, act1, act2
CASES = [
    (4, 64, 56, 64, 256, 3, 1, 1, "bf16", True, "relu", "relu"),      # ResNet-50 layer 1
    (2, 128, 28, 128, 512, 3, 1, 1, "bf16", True, "relu", "relu"),    # layer 2
    (3, 128, 56, 128, 512, 3, 2, 1, "bf16", True, "relu", "relu"),    # layer 2, first block
    (1, 64, 15, 64, 256, 3, 1, 1, "f16", True, "relu", "relu"),       # ragged M: 225 pixels
    (2, 64, 20, 64, 384, 3, 1, 1, "bf16", False, "relu6", "none"),    # 3 chunks, no residual
    (2, 256, 14, 64, 256, 1, 1, 0, "bf16", True, "relu", "relu"),     # a 1x1 first conv
    (256, 64, 56, 64, 256, 3, 1, 1, "bf16", True, "relu", "relu"),    # the benchmarked batch
]
ACT = {"none": 0, "relu": 1, "relu6": 2}


def _data(case):
    n, c, h, mid, cout, k, stride, pad, dt, use_res, a1, a2 = case
    rng = np.random.Generator(np.random.PCG64(900 + c + mid + cout + k))
    x = rng.standard_normal((n, c, h, h), dtype=np.float32)
    w1 = (rng.standard_normal((mid, c, k, k)) * np.sqrt(2.0 / (c * k * k))).astype(np.float32)
    w2 = (rng.standard_normal((cout, mid, 1, 1)) * np.sqrt(2.0 / mid)).astype(np.float32)
    bn = []
    for ch in (mid, cout):
        bn.append((rng.uniform(0.5, 1.5, ch).astype(np.float32),
                   (rng.standard_normal(ch) * 0.1).astype(np.float32),
                   (rng.standard_normal(ch) * 0.1).astype(np.float32),
                   rng.uniform(0.5, 1.5, ch).astype(np.float32)))
    p = (h + 2 * pad - k) // stride + 1
    res = rng.standard_normal((n, cout, p, p), dtype=np.float32) if use_res else None
    return x, w1, w2, bn, res, p


@pytest.mark.parametrize("case", CASES, ids=[f"p{i}" for i in range(len(CASES))])
def test_conv_pair_matches_two_launches_and_oracle(gpu, case):
    import oracle as orc
    from omnimatchdeeplearningtool_b200 import _lib
    from omnimatchdeeplearningtool_b200._lib import call, lib
    from omnimatchdeeplearningtool_b200.backend import DeviceBuffer
    n, c, h, mid, cout, k, stride, pad, dt_name, use_res, a1, a2 = case
    dt = _lib.DTYPE_BF16 if dt_name == "bf16" else _lib.DTYPE_F16
    x, w1, w2, bn, res, p = _data(case)
    keep = []

    def dev(a):
        b = DeviceBuffer.from_numpy(np.ascontiguousarray(a, np.float32))
        keep.append(b)
        return b

    def buf(nbytes):
        b = DeviceBuffer(nbytes)
        keep.append(b)
        return b

    try:
        cs = int(lib.omCudaStoredChannels(c))
        assert lib.omCudaConvPairSupported(cs, mid, cout, dt) == 1
        xs = buf(n * h * h * cs * 2)
        call("omCudaNchwToNhwc", dev(x).ptr, xs.ptr, n, c, h, h, cs, dt)
        packs = []
        for w, (g, b, m, v), cin_s in ((w1, bn[0], cs), (w2, bn[1], mid)):
            co, ci, kk = w.shape[0], w.shape[1], w.shape[2]
            packed = buf(int(lib.omCudaPackedConvWeightElems(co, kk, kk, cin_s)) * 2)
            bias = buf(co * 4)
            call("omCudaPackConvWeight", dev(w).ptr, None, dev(g).ptr, dev(b).ptr, dev(m).ptr,
                 dev(v).ptr, 1e-5, packed.ptr, bias.ptr, co, ci, kk, kk, cin_s, dt)
            packs.append((packed, bias))
        rs = None
        if use_res:
            rs = buf(n * p * p * cout * 2)
            call("omCudaNchwToNhwc", dev(res).ptr, rs.ptr, n, cout, p, p, cout, dt)
        out = buf(n * p * p * cout * 2)
        (p1, b1), (p2, b2) = packs
        for _ in range(2):  # a second launch gives the same bits
            call("omCudaConvPairBnAct", xs.ptr, p1.ptr, b1.ptr, p2.ptr, b2.ptr,
                 rs.ptr if rs else None, out.ptr, n, h, h, cs, mid, cout, k, k, stride, pad,
                 ACT[a1], ACT[a2], dt)
        # the same through two launches, the intermediate in device memory
        midbuf = buf(n * p * p * mid * 2)
        out2 = buf(n * p * p * cout * 2)
        call("omCudaConv2dBnAct", xs.ptr, p1.ptr, b1.ptr, None, midbuf.ptr, n, h, h, cs, mid, k,
             k, stride, pad, ACT[a1], dt, dt)
        call("omCudaConv2dBnAct", midbuf.ptr, p2.ptr, b2.ptr, rs.ptr if rs else None, out2.ptr,
             n, p, p, mid, cout, 1, 1, 1, 0, ACT[a2], dt, dt)
        assert gpu.kernel_error() == 0
        raw = np.uint16
        fused = out.to_numpy((n * p * p * cout,), raw)
        ref2 = out2.to_numpy((n * p * p * cout,), raw)
        assert np.array_equal(fused, ref2), int((fused != ref2).sum())
        # against the fp32 oracle (a subset of images at the full batch)
        o32 = buf(n * cout * p * p * 4)
        call("omCudaNhwcToNchw", out.ptr, o32.ptr, n, cout, p, p, cout, dt)
        got = o32.to_numpy((n, cout, p, p))
    finally:
        for b in keep:
            b.free()
    idx = list(range(n)) if n <= 4 else [0, 1, n - 2, n - 1]
    xi = np.ascontiguousarray(x[idx])

    def act(y, a):
        return orc.relu(y) if a == "relu" else (orc.relu6(y) if a == "relu6" else y)

    y = act(orc.batchnorm_eval(orc.conv2d(xi, w1, None, stride, pad), *bn[0]), a1)
    y = orc.batchnorm_eval(orc.conv2d(y, w2, None, 1, 0), *bn[1])
    if use_res:
        y = y + res[idx]
    y = act(y, a2)
    e = rel_err(got[idx], y)
    assert np.isfinite(got).all()
    assert e <= 2e-2, e


def test_resnet50_plan_fused_equals_unfused(gpu):
    """The ResNet-50 plan with its 3x3 + 1x1 pairs fused gives the unfused plan's logits bit for
    bit, and uses fewer launches."""
    from omnimatchdeeplearningtool_b200 import _lib, synth
    from omnimatchdeeplearningtool_b200.plan import InferencePlan
    net = synth.resnet_spec(50)
    w = synth.make_weights(net)
    x = synth.normal_input(4, seed=4)
    fused = InferencePlan(net, w, batch=4, dtype=_lib.DTYPE_BF16)
    plain = InferencePlan(net, w, batch=4, dtype=_lib.DTYPE_BF16, fuse_pairs=False)
    try:
        a = fused.run(x)
        b = plain.run(x)
        n_pairs = sum(1 for m in fused.meta if m.get("kind") == "pair")
        assert n_pairs >= 7  # layers 1 and 2: 3 + 4 blocks
        assert fused.n_launches == plain.n_launches - n_pairs
    finally:
        fused.close()
        plain.close()
    assert np.array_equal(a, b)
