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
