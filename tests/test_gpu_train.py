"""Configs 1 and 3, the fp32 ResNet-18 through the reference-named C ABI.

Config 1 (inference, eval-mode BN) is checked at the end of this file. Config 3 parity: the fp32
ResNet-18 training step (forward with batch-statistics BN,
softmax cross-entropy, backward, SGD momentum 0.9, lr 0.01) through the reference-named C ABI,
against the CPU oracle's training step on the same seeded weights, inputs and labels.

Tolerances (fp32 path), gradients measured per parameter as max|gpu - oracle|/max|oracle|
against the oracle's double-precision training step:
  * small case (batch 4, 64x64, 10 classes): loss within 1e-4, median gradient error <= 1e-4,
    every gradient <= 1e-2; parameters after the SGD step within 1e-5;
  * config 3 (batch 8, 224x224, 1000 classes): loss within 1e-4; gradients no further from the
    exact computation than the reference engine's own fp32 gradients are on the same case
    (median and maximum of its per-parameter errors, measured from the reference library by
    tests/golden/make_golden.py): backpropagating through BatchNorm's
    gamma*invstd/M*(M*dy - sum dy - xhat*sum dy*xhat) with M = N*H*W up to 100k cancels, and
    fp32 accumulation moves early-layer gradients by ~1% in the reference itself.
"""
import os
import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu


def _run(batch, hw, classes, seed, fused_bn_stats=False, stem_s2d=False):
    import oracle as orc
    from omnimatchdeeplearningtool_b200 import synth
    from omnimatchdeeplearningtool_b200._lib import call
    from omnimatchdeeplearningtool_b200.backend import DeviceBuffer
    from omnimatchdeeplearningtool_b200.plan import Fp32Net
    net = synth.resnet_spec(18, classes)
    w = synth.make_weights(net)
    x = synth.normal_input(batch, 3, hw, hw, seed=seed)
    y = synth.onehot_labels(batch, classes, seed=seed + 1)
    fnet = Fp32Net(net, w, batch, hw, hw, fused_bn_stats=fused_bn_stats, stem_s2d=stem_s2d)
    dx, dy = DeviceBuffer.from_numpy(x), DeviceBuffer.from_numpy(y)
    dloss = DeviceBuffer.zeros(4)
    fnet.forward_backward(dx.ptr, dy.ptr, dloss.ptr)
    loss = float(dloss.to_numpy((1,))[0])
    grads = fnet.read_grads()
    fnet.step(0.01, 0.9)
    new_fc = fnet.read_param("fc.weight")
    new_conv1 = fnet.read_param("conv1.weight")
    call("omCudaSynchronize")
    fnet.close()
    ow = {k: v.copy() for k, v in w.items()}
    vel = {}
    oloss, ograds = orc.train_step(net, ow, x, y, 0.01, 0.9, velocities=vel)
    return net, loss, grads, new_fc, new_conv1, oloss, ograds, ow


def test_resnet18_training_step_small(gpu):
    net, loss, grads, new_fc, new_conv1, oloss, ograds, ow = _run(4, 64, 10, 11)
    assert np.isfinite(loss)
    assert abs(loss - oloss) <= 1e-4 * abs(oloss), (loss, oloss)
    errs = {name: rel_err(grads[name], ograds[name]) for name, _ in net.params}
    print(f"small: loss err {abs(loss - oloss) / abs(oloss):.2e}, gradient error median "
          f"{np.median(list(errs.values())):.2e} max {max(errs.values()):.2e}")
    assert float(np.median(list(errs.values()))) <= 1e-4, sorted(errs.items(), key=lambda t: -t[1])[:5]
    assert max(errs.values()) <= 1e-2, sorted(errs.items(), key=lambda t: -t[1])[:5]
    assert rel_err(new_fc, ow["fc.weight"]) <= 1e-5
    assert rel_err(new_conv1, ow["conv1.weight"]) <= 1e-5


@pytest.mark.parametrize("fused_bn_stats,stem_s2d", [(False, False), (True, False),
                                                     (True, True)])
def test_resnet18_training_step_config3(gpu, fused_bn_stats, stem_s2d):
    gold = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "golden.npz"))
    net, loss, grads, new_fc, new_conv1, oloss, ograds, ow = _run(8, 224, 1000, 11,
                                                                  fused_bn_stats, stem_s2d)
    assert abs(loss - oloss) <= 1e-4 * abs(oloss), (loss, oloss)
    errs = np.array([rel_err(grads[name], ograds[name]) for name, _ in net.params])
    ref = gold["train_r18_224_ref_grad_err"]
    print(f"config3 (fused BN statistics: {fused_bn_stats}, stem space-to-depth: {stem_s2d}): "
          f"loss err "
          f"{abs(loss - oloss) / abs(oloss):.2e}, gradient error median "
          f"{np.median(errs):.4f} max {errs.max():.4f} (reference fp32: {np.median(ref):.4f}, "
          f"{ref.max():.4f})")
    assert np.median(errs) <= np.median(ref), (np.median(errs), np.median(ref))
    assert errs.max() <= ref.max(), (errs.max(), ref.max())
    assert rel_err(new_fc, ow["fc.weight"]) <= 1e-4


def test_config1_resnet18_fp32_inference(gpu):
    """Config 1: ResNet-18 fp32 inference, batch 8, the normalised U[0,1) image input, eval-mode
    BatchNorm on the seeded running statistics, through the reference-layout fp32 entry points
    (omCudaConv2d, omCudaBatchNorm2d, ...): 1000 logits within max|a-b|/max|b| <= 1e-4 of the
    oracle, identical top-1."""
    import oracle as orc
    from omnimatchdeeplearningtool_b200 import synth
    from omnimatchdeeplearningtool_b200.backend import DeviceBuffer
    from omnimatchdeeplearningtool_b200.plan import Fp32Net
    net = synth.resnet_spec(18, 1000)
    w = synth.make_weights(net)
    x = synth.imagenet_input(8)
    want = orc.forward(net, w, x)
    fnet = Fp32Net(net, w, 8, 224, 224)
    dx = DeviceBuffer.from_numpy(x)
    try:
        got = fnet.forward_eval(dx.ptr)
        # eval mode leaves the running statistics untouched: a second pass gives the same bits
        again = fnet.forward_eval(dx.ptr)
    finally:
        fnet.close()
        dx.free()
    assert gpu.kernel_error() == 0
    assert np.array_equal(got, again)
    print(f"config1: logits max rel err {rel_err(got, want):.2e}")
    assert rel_err(got, want) <= 1e-4, rel_err(got, want)
    assert np.array_equal(got.argmax(1), want.argmax(1))


def test_guarded_step_clips_like_the_training_loop(gpu):
    """Fp32Net.step(max_grad_norm=...) after a real backward: the parameters move as if the
    flat gradient had been scaled by max_norm / ||g|| (the training loop's clip,
    EngineBridge.cpp:1885-1925), and a limit above the norm leaves the plain step."""
    from omnimatchdeeplearningtool_b200 import synth
    from omnimatchdeeplearningtool_b200.backend import DeviceBuffer
    from omnimatchdeeplearningtool_b200.plan import Fp32Net
    net = synth.resnet_spec(18, 10)
    w = synth.make_weights(net)
    x = synth.normal_input(2, 3, 32, 32, seed=5)
    y = synth.onehot_labels(2, 10, seed=6)
    fnet = Fp32Net(net, w, 2, 32, 32)
    dx, dy, dloss = DeviceBuffer.from_numpy(x), DeviceBuffer.from_numpy(y), DeviceBuffer.zeros(4)
    fnet.forward_backward(dx.ptr, dy.ptr, dloss.ptr)
    g = np.concatenate([v.ravel() for v in fnet.read_grads().values()]).astype(np.float64)
    norm = float(np.sqrt((g ** 2).sum()))
    w0 = fnet.read_param("fc.weight").astype(np.float64)
    g_fc = fnet.read_grads()["fc.weight"].astype(np.float64)
    fnet.step(0.01, 0.0, max_grad_norm=norm / 2)
    got_norm, ran, clip = fnet.guard_status()
    assert ran and abs(got_norm - norm) / norm < 1e-5 and abs(clip - 0.5) < 1e-5
    assert rel_err(fnet.read_param("fc.weight") - w0, -0.01 * 0.5 * g_fc) < 1e-5
    fnet.close()
    assert gpu.kernel_error() == 0


@pytest.mark.parametrize("fused_bn_stats,stem_s2d", [(False, False), (True, False),
                                                     (True, True)])
def test_captured_training_step_matches_eager(gpu, fused_bn_stats, stem_s2d):
    """Fp32Net.capture_step / replay_step: the whole training step (forward, backward, SGD with
    momentum) as one CUDA graph. After one eager step on both, two replays on one net and two
    eager steps on the other give bit-identical loss, parameters, velocities and BatchNorm
    running statistics."""
    from omnimatchdeeplearningtool_b200 import synth
    from omnimatchdeeplearningtool_b200._lib import call
    from omnimatchdeeplearningtool_b200.backend import DeviceBuffer
    from omnimatchdeeplearningtool_b200.plan import Fp32Net
    net = synth.resnet_spec(18, 10)
    w = synth.make_weights(net)
    x = DeviceBuffer.from_numpy(synth.normal_input(4, 3, 64, 64, seed=31))
    y = DeviceBuffer.from_numpy(synth.onehot_labels(4, 10, seed=32))
    out = []
    for graph in (False, True):
        fnet = Fp32Net(net, w, 4, 64, 64, fused_bn_stats=fused_bn_stats, stem_s2d=stem_s2d)
        loss = DeviceBuffer.zeros(4)
        try:
            fnet.forward_backward(x.ptr, y.ptr, loss.ptr)
            fnet.step(0.01, 0.9)
            if graph:
                fnet.capture_step(x.ptr, y.ptr, loss.ptr, 0.01, 0.9)
                fnet.replay_step()
                fnet.replay_step()
            else:
                for _ in range(2):
                    fnet.forward_backward(x.ptr, y.ptr, loss.ptr)
                    fnet.step(0.01, 0.9)
            call("omCudaSynchronize")
            vel = np.empty(fnet.n_params, np.float32)
            call("omCudaCopyD2H", vel.ctypes.data, fnet.vel_flat.ptr, vel.nbytes)
            bufs = {k: b.to_numpy((b.nbytes // 4,)) for k, b in fnet.buffers.items()}
            out.append((loss.to_numpy((1,)), {n: fnet.read_param(n) for n, _ in net.params},
                        vel, bufs))
        finally:
            fnet.close()
            loss.free()
    (l0, p0, v0, b0), (l1, p1, v1, b1) = out
    assert np.array_equal(l0, l1)
    assert all(np.array_equal(p0[k], p1[k]) for k in p0)
    assert np.array_equal(v0, v1)
    assert all(np.array_equal(b0[k], b1[k]) for k in b0)
    assert gpu.kernel_error() == 0
