"""Network-level parity of the fused NHWC 16-bit inference plan with the fp32 CPU oracle.

Configs 1, 4 and 5 at small batch on the full 224x224 input: ResNet-18 and ResNet-50 in bf16,
the MobileNet-style stack in fp16, all with seeded weights. Tolerance (16-bit path):
max |a-b| / max |b| <= 2e-2 over all logits, and identical top-1 per image.
"""
import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name,dtype", [("resnet18", "bf16"), ("resnet50", "bf16"),
                                        ("mobilenet", "f16")])
def test_inference_plan_matches_oracle(gpu, name, dtype):
    import oracle as orc
    from omnimatchdeeplearningtool_b200 import _lib, synth
    from omnimatchdeeplearningtool_b200.plan import InferencePlan
    net = synth.mobilenet_spec() if name == "mobilenet" else synth.resnet_spec(int(name[6:]))
    w = synth.make_weights(net)
    x = synth.imagenet_input(2) if name == "resnet18" else synth.normal_input(2)
    want = orc.forward(net, w, x)
    dt = _lib.DTYPE_BF16 if dtype == "bf16" else _lib.DTYPE_F16
    plan = InferencePlan(net, w, batch=2, dtype=dt)
    try:
        got = plan.run(x)
        plan.capture()
        got2 = plan.run(x)   # graph replay gives the same bits
    finally:
        plan.close()
    assert np.isfinite(got).all()
    assert np.array_equal(got, got2)
    assert rel_err(got, want) <= 2e-2, rel_err(got, want)
    assert np.array_equal(got.argmax(1), want.argmax(1))


def test_resnet50_bf16_batch256_matches_oracle_on_subset(gpu):
    """The benchmarked configuration itself: the ResNet-50 bf16 plan at batch 256 (whose long
    reductions run on 256-wide tiles and whose 64/128-wide 3x3 layers on sub-tile pairs, tile
    variants that small batches never reach), compared with the fp32 oracle on the first four
    and the last four images of the batch: <= 2e-2 and identical top-1."""
    import oracle as orc
    from omnimatchdeeplearningtool_b200 import _lib, synth
    from omnimatchdeeplearningtool_b200._lib import lib
    from omnimatchdeeplearningtool_b200.plan import InferencePlan
    from test_gpu_conv_tc import tile_plan
    # the layer-3/4 3x3 convs of this batch take 256-wide tiles, layer 1's 3x3 sub-tile pairs
    assert tile_plan(256, 14, 256, 256, 3, 1, 1, False)[0] == 256
    assert tile_plan(256, 7, 512, 512, 3, 1, 1, False)[0] == 256
    assert tile_plan(256, 56, 64, 64, 3, 1, 1, False)[2] == 2
    assert int(lib.omCudaStoredChannels(64)) == 64
    net = synth.resnet_spec(50)
    w = synth.make_weights(net)
    x = synth.normal_input(256)
    plan = InferencePlan(net, w, batch=256, dtype=_lib.DTYPE_BF16)
    try:
        plan.capture()
        got = plan.run(x)
    finally:
        plan.close()
    assert np.isfinite(got).all()
    idx = [0, 1, 2, 3, 252, 253, 254, 255]
    want = orc.forward(net, w, np.ascontiguousarray(x[idx]))
    e = rel_err(got[idx], want)
    print(f"resnet50 bf16 batch 256, images {idx}: max rel err {e:.2e}")
    assert e <= 2e-2, e
    assert np.array_equal(got[idx].argmax(1), want.argmax(1))


def test_mobilenet_f16_batch256_matches_oracle_on_subset(gpu):
    """The benchmarked MobileNet-style configuration: the fp16 plan at batch 256, whose
    depthwise layers run on the TMA row-ring kernel with whole-pixel channel tiles and CTA
    ranges that cross images (shapes batch 2 does not reach), compared with the fp32 oracle on
    the first two and the last two images: <= 2e-2 and identical top-1."""
    import oracle as orc
    from omnimatchdeeplearningtool_b200 import _lib, synth
    from omnimatchdeeplearningtool_b200.plan import InferencePlan
    net = synth.mobilenet_spec()
    w = synth.make_weights(net)
    x = synth.normal_input(256, seed=5)
    plan = InferencePlan(net, w, batch=256, dtype=_lib.DTYPE_F16)
    try:
        plan.capture()
        got = plan.run(x)
    finally:
        plan.close()
    assert np.isfinite(got).all()
    idx = [0, 1, 254, 255]
    want = orc.forward(net, w, np.ascontiguousarray(x[idx]))
    e = rel_err(got[idx], want)
    print(f"mobilenet f16 batch 256, images {idx}: max rel err {e:.2e}")
    assert e <= 2e-2, e
    assert np.array_equal(got[idx].argmax(1), want.argmax(1))


@pytest.mark.parametrize("name,dtype", [("resnet50", "bf16"), ("mobilenet", "f16")])
def test_16bit_input_gives_the_same_logits(gpu, name, dtype):
    """A plan that takes its NCHW image in its own 16-bit type (input_dtype; half the bytes to
    copy to the device) gives bit for bit the logits of the fp32-input plan on the same image
    rounded to that type: the stem rounds its fp32 input to the 16-bit type anyway. Also
    checked through serve() (the copies on the transfer stream)."""
    import ctypes
    from omnimatchdeeplearningtool_b200 import _lib, synth
    from omnimatchdeeplearningtool_b200._lib import call
    from omnimatchdeeplearningtool_b200.plan import InferencePlan
    net = synth.mobilenet_spec() if name == "mobilenet" else synth.resnet_spec(50)
    w = synth.make_weights(net)
    dt = _lib.DTYPE_BF16 if dtype == "bf16" else _lib.DTYPE_F16
    x = synth.normal_input(4, seed=9)
    p32 = InferencePlan(net, w, batch=4, dtype=dt)
    p16 = InferencePlan(net, w, batch=4, dtype=dt, input_dtype=dt)
    hin = hout = None
    try:
        assert p16.in_bytes * 2 == p32.in_bytes
        want = p32.run(x)
        got = p16.run(x)
        assert np.array_equal(got, want)
        p16.capture()
        h = ctypes.c_void_p()
        call("omCudaMallocHost", ctypes.byref(h), p16.in_bytes)
        hin = h.value
        src = p16.host_input(x)   # kept alive while it is copied
        ctypes.memmove(hin, src.ctypes.data, p16.in_bytes)
        o = ctypes.c_void_p()
        call("omCudaMallocHost", ctypes.byref(o), want.nbytes)
        hout = o.value
        p16.serve([hin], [hout])
        call("omCudaSynchronize")
        served = np.frombuffer(ctypes.string_at(hout, want.nbytes), np.float32).reshape(want.shape)
        assert np.array_equal(served, want)
    finally:
        p32.close()
        p16.close()
        for ptr in (hin, hout):
            if ptr:
                call("omCudaFreeHost", ptr)


@pytest.mark.parametrize("slots", [1, 2])
def test_serve_pipeline_matches_run(gpu, slots):
    """InferencePlan.serve (copies on the transfer stream, two input slots, one graph each)
    gives, batch by batch, the same bits as the synchronous run() of the same batch."""
    import ctypes
    from omnimatchdeeplearningtool_b200 import _lib, synth
    from omnimatchdeeplearningtool_b200._lib import call
    from omnimatchdeeplearningtool_b200.plan import InferencePlan
    net = synth.resnet_spec(18)
    w = synth.make_weights(net)
    n_steps, batch = 5, 4
    xs = [synth.normal_input(batch, seed=20 + i) for i in range(n_steps)]
    plan = InferencePlan(net, w, batch=batch, dtype=_lib.DTYPE_BF16, input_slots=slots)
    hin, hout = [], []
    try:
        want = [plan.run(x) for x in xs]
        plan.capture()
        out_bytes = batch * net.classes * 4
        for x in xs:
            a, b = ctypes.c_void_p(), ctypes.c_void_p()
            call("omCudaMallocHost", ctypes.byref(a), plan.in_bytes)
            hin.append(a.value)
            ctypes.memmove(a.value, x.ctypes.data, plan.in_bytes)
            call("omCudaMallocHost", ctypes.byref(b), out_bytes)
            hout.append(b.value)
        plan.serve(hin, hout)
        call("omCudaSynchronize")
        got = [np.frombuffer(ctypes.string_at(p, out_bytes), np.float32).reshape(batch, -1)
               for p in hout]
    finally:
        plan.close()
        for p in hin + hout:
            call("omCudaFreeHost", p)
    for g, wnt in zip(got, want):
        assert np.array_equal(g, wnt)
    assert not np.array_equal(got[0], got[1])
