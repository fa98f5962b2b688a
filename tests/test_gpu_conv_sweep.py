"""Config 2 parity: the single conv2d + BatchNorm2d (eval) + ReLU layer sweep.

3x3 stride 1 pad 1 and 1x1 stride 1 convolutions with C = K in {64, 128, 256, 512} and
H = W in {56, 28, 14, 7}, in fp32, bf16 and fp16, on N(0,1) inputs and He-normal weights from a
seed, against the CPU oracle (the reference CPUBackend's arithmetic) on the same data:
max|a-b|/max|b| <= 1e-4 for fp32 and <= 2e-2 for the 16-bit paths. The layers run at the
benchmarked N = 32, so the tile plans checked are the ones the timed sweep uses; the oracle runs
on the first and the last image of the batch (a full batch-32 oracle would take minutes).
"""
import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu

SHAPES = [(ks, c, h) for ks in (3, 1) for c in (64, 128, 256, 512) for h in (56, 28, 14, 7)]


@pytest.mark.parametrize("ks,c,h", SHAPES, ids=[f"k{k}c{c}h{h}" for k, c, h in SHAPES])
def test_conv_bn_relu_sweep(gpu, ks, c, h):
    import oracle as orc
    from omnimatchdeeplearningtool_b200.layers import ConvBnReluLayer
    from omnimatchdeeplearningtool_b200.synth import conv_layer_data
    x, w, g, b, mu, var = conv_layer_data(c, h, ks, 32, seed=500 + c + h + ks)
    pad = ks // 2
    idx = [0, 31]
    want = orc.relu(orc.batchnorm_eval(orc.conv2d(np.ascontiguousarray(x[idx]), w, None, 1, pad),
                                       g, b, mu, var))
    for dt, tol in (("fp32", 1e-4), ("bf16", 2e-2), ("fp16", 2e-2)):
        layer = ConvBnReluLayer(x, w, g, b, mu, var, 1, pad, dt)
        try:
            layer.run()
            got = layer.result()[idx]
        finally:
            layer.close()
        assert gpu.kernel_error() == 0
        e = rel_err(got, want)
        print(f"config2 k{ks} c{c} h{h} {dt}: max rel err {e:.2e}")
        assert e <= tol, (dt, e)
